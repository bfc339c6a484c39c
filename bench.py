"""Benchmark: ViT-L/14 NVFP4 W4A4 inference images/s on 1..8 B200 (one replica per GPU).

    python bench.py [--gpus N --steps K --warmup W] [--impl reference] [--attn bf16|nvfp4]
    torchrun --nproc-per-node N ... bench.py --gpus N ...

Headline workload: DINOv2-style ViT-L/14 at 224x224 (257 tokens), 24 blocks, dim 1024,
16 heads, GELU MLP 4096, LayerScale 1e-5, random N(0, 0.02) weights, N(0,1) bf16 images, global batch
1024 sharded evenly over the ranks.  Every block's qkv/proj are QuantLinear (Four-Over-Six weights,
dynamic NVFP4 activations) and every MLP is FusedNVFP4MLP (bias + erf-GELU + NVFP4 cast fused into the
fc1 epilogue, the reference's function); attention runs the reference's unflagged bf16 route on the
tcgen05 bf16 kernel (default) or the FP4 attention kernels (--attn nvfp4).

Printed JSON line (rank 0):
  value    images/s of the whole job, inputs resident in HBM, the forward replayed from a CUDA graph,
           CUDA events on the replaying stream, max over ranks, nothing else in the timed region;
  e2e      the same through the public runner (vitfp4.pipeline.OverlappedRunner) with every step's
           images copied from pinned host memory and its logits read back inside the timed region;
  kernels / roofline / gemm_roofline / cast_roofline
           per-kernel CUDA events from a separate eager pass after the timed regions;
  host     eager-mode device time and host enqueue time per step (what graph replay removes);
  secondary (1 GPU, rank 0): BASELINE config 2 (cast + GEMM sweep at M = 50432, with cuBLASLt's
           torch._scaled_mm_v2 on the same packed operands), the config-4 GEMM shapes against
           cuBLASLt, config 3 (ViT-B/16 batch 256 with FP4 attention) and config 5 (ViT-H/14 @448,
           the 64 images one GPU of eight processes).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "vit-nvfp4_b200"))

GLOBAL_BATCH = 1024
MODEL = "vit_l14_dinov2_style"
METRIC = "ViT-L/14 W4A4 images/s"
FP4_NOMINAL_TFLOPS = 9000.0
BF16_NOMINAL_TFLOPS = 2250.0
# used when MEASURED_PEAKS.json is absent: an earlier measurement on the same B200 pool
# (STREAM-style copy and cuBLAS bf16 burst)
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
# DRAM bytes (read + write) per unit measured by ncu for the kernels that can dominate, keyed by
# (kernel kind, N, K): ncu dram__bytes_read.sum + dram__bytes_write.sum of one GEMM launch at
# M = 65792 (ViT-L/14, batch 256) per row of A -- the fc1 launch moved 40.5 + 99.2 MB; A and the
# output grow with M while the 2.4 MB of weights do not, so bytes scale with the rows -- and of one
# bf16 attention launch at batch 128 (2048 heads of 257 x 64) per head
NCU_TRAFFIC_PER_ROW = {
    ("gemm_gelu_nvfp4", 4096, 1024): (40.415488e6 + 98.564096e6) / 65792,
    ("gemm_residual", 1024, 4096): (288.748288e6 + 93.634816e6) / 65792,
    ("gemm_bias", 3072, 1024): (39.713280e6 + 350.148864e6) / 65792,
    ("gemm_bias", 1024, 1024): (38.528512e6 + 80.605952e6) / 65792,
    ("attn_bf16", 257, 64): (202.204160e6 + 42.473728e6) / 2048,
}
CAST_PREFIXES = ("cast", "ln_cast")


def gemm_algorithmic_bytes(kind: str, m: int, n: int, k: int) -> int:
    """HBM bytes a GEMM launch must move: A and B codes + E4M3 scales in, plus its output
    (bf16; NVFP4 codes + scales for the GELU epilogue; residual read + bf16 write for fc2).
    For bf16 attention (m heads, n tokens, k head dim): q, k, v read and the output written once."""
    if kind.startswith("attn"):
        return m * n * k * 2 * 4
    operands = (m + n) * (k // 2 + k // 16)
    if kind == "gemm_gelu_nvfp4":
        return operands + m * (n // 2 + n // 16)
    if kind == "gemm_residual":
        return operands + 2 * m * n * 2
    return operands + m * n * 2


def _peak_source(measured: bool, what: str) -> str:
    return (f"measured {what} (MEASURED_PEAKS.json), of measured" if measured else
            f"fallback {what} (MEASURED_PEAKS.json absent), of fallback")


def roofline_entry(name: str, flops: float, ms: float, bf16_tf: float, measured: bool) -> dict:
    """Roofline object of one timed tensor-core kernel kind ("<kind>_<m>x<n>x<k>"): its FLOPs over its
    summed launch durations, against the bf16 peak for bf16 attention and 4 x the bf16 peak for the FP4
    GEMMs and FP4 attention, with the algorithmic bytes of one launch and the ncu DRAM bytes where
    captured."""
    achieved = flops / (ms * 1e-3) / 1e12
    src = _peak_source(measured, "bf16 burst")
    if name.startswith("attn_bf16"):     # bf16 tensor-core kernel
        peak, peak_source, nominal = bf16_tf, src, BF16_NOMINAL_TFLOPS
    else:                                # FP4 / FP8 tensor cores: FP4 itself is not measured
        peak, peak_source, nominal = 4 * bf16_tf, "4 x " + src + "; FP4 itself not measured", FP4_NOMINAL_TFLOPS
    r = {"kernel": name, "bound": "tensor", "achieved": round(achieved, 1), "peak": round(peak, 1),
         "unit": "TFLOP/s", "frac": round(achieved / peak, 4), "peak_source": peak_source,
         "frac_of_nominal": round(achieved / nominal, 4), "nominal_tflops": nominal, "traffic": None}
    kind, dims = name.rsplit("_", 1)
    m_rows, n_cols, k_dim = (int(x) for x in dims.split("x"))
    r["algorithmic_bytes"] = gemm_algorithmic_bytes(kind, m_rows, n_cols, k_dim)
    per_row = NCU_TRAFFIC_PER_ROW.get((kind, n_cols, k_dim))
    if per_row is not None:
        r["traffic"] = round(per_row * m_rows)   # bytes per launch
        r["traffic_source"] = (
            "ncu dram__bytes_read.sum + dram__bytes_write.sum of one launch at batch 128 (2048 heads), "
            "scaled by heads" if kind.startswith("attn") else
            "ncu dram__bytes_read.sum + dram__bytes_write.sum of one launch at M = 65792, scaled by rows")
    return r


def cast_roofline_entry(name: str, nbytes: float, ms: float, hbm_gbs: float, measured: bool) -> dict:
    """Roofline object of an HBM-bound cast kind ("<kind>_<m>x<k>"): algorithmic bytes over time."""
    achieved = nbytes / (ms * 1e-3) / 1e9
    return {"kernel": name, "bound": "hbm", "achieved": round(achieved, 1), "peak": round(hbm_gbs, 1),
            "unit": "GB/s", "frac": round(achieved / hbm_gbs, 4), "peak_source": _peak_source(measured, "HBM copy"),
            "traffic": None, "algorithmic_bytes_per_call": None}


def _args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="vitfp4", choices=["vitfp4", "reference"])
    ap.add_argument("--attn", default="bf16", choices=["bf16", "nvfp4"])
    ap.add_argument("--gelu", default="erf", choices=["erf", "tanh"],
                    help="fc1 epilogue GELU: erf (the reference's function) or the tanh form")
    ap.add_argument("--batch", type=int, default=GLOBAL_BATCH, help="global batch (images)")
    ap.add_argument("--depth", type=int, default=24)
    ap.add_argument("--eager", action="store_true", help="time eager launches instead of CUDA-graph replay")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-secondary", action="store_true", help="skip configs 2/3/5 and the cuBLASLt comparators")
    ap.add_argument("--unfused", action="store_true", help="keep the per-module path (no fused blocks)")
    return ap.parse_args()


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f)
    except Exception:
        return {}


# ------------------------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index, self.rows, self.proc = index, [], None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([c.strip() for c in line.split(",")])

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm = [float(r[1]) for r in self.rows if len(r) >= 9 and r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if len(r) >= 9 and r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows if len(r) >= 9 for i in range(4) if r[5 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


# ------------------------------------------------------------------------------- reference arm
def _oracle_modules():
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import nvfp4_oracle  # noqa: F401
    import vit_oracle
    return vit_oracle


def cpu_forward_rate(attn: str, sample_images: int, steps: int, warmup: int, depth: int):
    """Time the CPU restatement of the reference's torch-backend ViT-L/14 W4A4 forward."""
    import numpy as np
    vo = _oracle_modules()
    W = vo.make_weights(depth=depth)
    rng = np.random.default_rng(0)
    imgs = rng.standard_normal((sample_images, 3, 224, 224)).astype(np.float32)
    for _ in range(warmup):
        vo.forward(W, imgs, attn=attn)
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        vo.forward(W, imgs, attn=attn)
        times.append(time.perf_counter() - t0)
    return sample_images / statistics.median(times), times


def run_reference(args, rank: int, world: int):
    if rank != 0:
        return 0
    cores = os.cpu_count() or 1
    try:
        import torch
        torch.set_num_threads(cores)
    except Exception:
        pass
    os.environ.setdefault("OMP_NUM_THREADS", str(cores))
    sample = 2
    steps = max(1, min(args.steps, 3))
    rate, times = cpu_forward_rate(args.attn, sample, steps, min(args.warmup, 1), args.depth)
    line = {
        "impl": "reference", "metric": METRIC, "value": round(rate, 4), "unit": "images/s", "n_gpus": world,
        "steps": steps, "warmup": min(args.warmup, 1), "ms_per_step": round(1000 * statistics.median(times), 2),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": {"workload": f"{MODEL} W4A4 forward (attention {args.attn})",
                                        "global_batch": args.batch, "seq_len": 257, "parallelism": "cpu"},
        "cpu_baseline": {"value": round(rate, 4), "unit": "images/s", "cores": cores, "kind": "port",
                         "sample": f"{sample} images per step (of the {args.batch}-image batch), "
                                   f"numpy restatement of the reference torch backend"},
        "e2e": {"value": round(rate, 4), "unit": "images/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------------------- models
def build_model(arch: dict, attn: str, device, fused: bool = True, exact_gelu: bool = True, seed: int = 0):
    """A W4A4 ViT as the benchmark runs it: all blocks converted (skip 0/0), Four-Over-Six weights,
    fused MLPs (erf-GELU epilogue unless exact_gelu=False), fused blocks, attention bf16, fp8 or nvfp4
    (QK^T and PV operands; fp8 is the reference's enable_quant_attention default)."""
    import torch
    from vitfp4 import vit
    from vitfp4.ptq import enable_quant_attention, fuse_mlps, fuse_norms, quantize_vit, vit_attn_policy
    model = vit.build_vit(seed=seed, device=device, **arch).to(dtype=torch.bfloat16).eval()
    depth = arch["depth"]
    n_mlp = fuse_mlps(model, skip_ends=0, exact_gelu=exact_gelu)
    n_lin, _ = quantize_vit(model, skip_first=0, skip_last=0, w_block_select="mse")
    n_att = 0
    if attn in ("nvfp4", "fp8"):
        n_att = enable_quant_attention(model, vit_attn_policy(depth, 0, 0, "blocks"), qk=attn, pv=attn)
    n_blk = fuse_norms(model) if fused else 0
    return model, {"fused_mlps": n_mlp, "quant_linears": n_lin, "quant_attention": n_att, "attention_route": attn,
                   "fused_blocks": n_blk}


def _events():
    import torch
    return torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)


def time_forward(fwd, steps: int, barrier=lambda: None) -> float:
    """Device ms of ``steps`` calls of fwd on the current stream (synchronised on both sides)."""
    import torch
    stream = torch.cuda.current_stream()
    barrier()
    torch.cuda.synchronize()
    t0, t1 = _events()
    t0.record(stream)
    for _ in range(steps):
        fwd()
    t1.record(stream)
    torch.cuda.synchronize()
    barrier()
    return t0.elapsed_time(t1)


def probe_pass(model, images, steps: int = 2) -> tuple[dict, int]:
    """Per-kernel-kind CUDA-event timings of ``steps`` eager forwards: {kind: [calls, work, ms]} and the
    library launches of one forward."""
    import torch
    from vitfp4.nvfp4 import ops
    torch.cuda.synchronize()
    ops.probe.reset()
    ops.probe.timing = True
    try:
        for _ in range(steps):
            model(images)
        torch.cuda.synchronize()
    finally:
        ops.probe.timing = False
    by_kind: dict = {}
    for kind, work, s, e in ops.probe.records:
        d = by_kind.setdefault(kind, [0, 0.0, 0.0])
        d[0] += 1
        d[1] += work
        d[2] += s.elapsed_time(e)
    launches = ops.probe.launches // steps
    ops.probe.reset()
    return by_kind, launches


def eager_split(model, images, steps: int = 2) -> dict:
    """Device ms and host enqueue ms per eager step (launch-by-launch, no probe events)."""
    import torch
    torch.cuda.synchronize()
    t0, t1 = _events()
    t0.record()
    h0 = time.perf_counter()
    for _ in range(steps):
        model(images)
    host = (time.perf_counter() - h0) * 1e3 / steps
    t1.record()
    torch.cuda.synchronize()
    return {"device_ms_per_step": round(t0.elapsed_time(t1) / steps, 3), "host_enqueue_ms_per_step": round(host, 3)}


def kernel_table(by_kind: dict, steps: int) -> dict:
    out = {}
    for k, (n, work, ms) in sorted(by_kind.items()):
        e = {"calls_per_step": n // steps, "ms_per_step": round(ms / steps, 3)}
        if k.startswith(CAST_PREFIXES):
            e["gbs"] = round(work / (ms * 1e-3) / 1e9, 1)
        else:
            e["tflops"] = round(work / (ms * 1e-3) / 1e12, 1)
        out[k] = e
    return out


def rooflines(by_kind: dict, peaks: dict) -> dict:
    measured = bool(peaks.get("bf16_tflops"))
    bf16_tf = peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"])
    hbm = peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"])
    res = {}
    tensor = {k: v for k, v in by_kind.items() if not k.startswith(CAST_PREFIXES)}
    gemms = {k: v for k, v in tensor.items() if k.startswith("gemm")}
    casts = {k: v for k, v in by_kind.items() if k.startswith(CAST_PREFIXES)}
    dom_all = max(by_kind.items(), key=lambda kv: kv[1][2]) if by_kind else None
    if dom_all and dom_all[0].startswith(CAST_PREFIXES):
        res["roofline"] = cast_roofline_entry(dom_all[0], dom_all[1][1], dom_all[1][2], hbm, measured)
    elif dom_all:
        res["roofline"] = roofline_entry(dom_all[0], dom_all[1][1], dom_all[1][2], bf16_tf, measured)
    if gemms:
        k, v = max(gemms.items(), key=lambda kv: kv[1][2])
        res["gemm_roofline"] = roofline_entry(k, v[1], v[2], bf16_tf, measured)
    if casts:
        k, v = max(casts.items(), key=lambda kv: kv[1][2])
        c = cast_roofline_entry(k, v[1], v[2], hbm, measured)
        c["algorithmic_bytes_per_call"] = round(v[1] / v[0])
        res["cast_roofline"] = c
    return res


# ------------------------------------------------------------------------------- secondary measurements
def _graph_time(fn, iters: int, repeats: int = 3) -> float:
    """Device ms per call of fn (which must not allocate), from `iters` calls captured in one CUDA
    graph, replayed `repeats` times after one warm replay; the median replay."""
    import torch
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for i in range(3):
            fn(i)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(iters):
            fn(i)
    g.replay()
    torch.cuda.synchronize()
    times = []
    for _ in range(repeats):
        t0, t1 = _events()
        t0.record()
        g.replay()
        t1.record()
        torch.cuda.synchronize()
        times.append(t0.elapsed_time(t1) / iters)
    del g
    return statistics.median(times)


def gemm_sweep(shapes, M: int, peaks: dict, label: str, with_cast: bool = True) -> list:
    """Cast (static global) and GEMM (plain bf16 output; with the weight's B scale image, which the
    K > 1024 kernel uses as the model's fc2 does) at (M, K, N) per shape, plus cuBLASLt's
    torch._scaled_mm_v2 on the same packed operands.  Activations N(0,1) bf16 with 0.1% of channels
    x20 (seeded), weights N(0, 0.02).  Buffers rotate so each call's working set misses L2."""
    import torch
    from vitfp4 import _lib
    from vitfp4.nvfp4 import ops
    hbm = peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"])
    bf16_tf = peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"])
    dev = torch.device("cuda")
    stream = lambda: torch.cuda.current_stream().cuda_stream   # noqa: E731
    rows = []
    for K, N in shapes:
        g = torch.Generator(device=dev).manual_seed(0)
        x = torch.randn(M, K, device=dev, generator=g)
        ch = torch.randperm(K, device=dev, generator=g)[: max(1, -(-K // 1000))]
        x[:, ch] *= 20.0
        x = x.bfloat16()
        w = (torch.randn(N, K, device=dev, generator=g) * 0.02).bfloat16()
        gx = ops.global_scale(ops.amax(x))
        wp, wsf, _, wg = ops.cast(w, None, "mse")
        wimg = ops.b_scale_image(wsf, N, K)   # the weight's B scale image, as the model's fused MLPs hold it
        ap, asf, _, ag = ops.cast(x, gx, "six")
        ws_bytes = M * K * 2 + M * K // 2 + M * N * 2
        R = max(1, -(-3 * 128 * 2 ** 20 // ws_bytes))          # working set of R rotations > 3 x L2
        xs = [x] + [x.clone() for _ in range(R - 1)]
        aps = [torch.empty_like(ap) for _ in range(R)]
        asfs = [torch.empty_like(asf) for _ in range(R)]
        outs = [torch.empty(M, N, dtype=torch.bfloat16, device=dev) for _ in range(R)]
        for i in range(R):
            aps[i].copy_(ap)
            asfs[i].copy_(asf)
        row = {"M": M, "K": K, "N": N}
        if with_cast:
            def cast_call(i):
                _lib.call("vf4_cast_nvfp4", xs[i % R].data_ptr(), _lib.VF4_BF16, M, K, K, gx.data_ptr(), 0, 0, None,
                          aps[i % R].data_ptr(), asfs[i % R].data_ptr(), None, None, stream())
            ms = _graph_time(cast_call, 30)
            gbs = M * K * 2.5625 / (ms * 1e-3) / 1e9
            row["cast_ms"] = round(ms, 4)
            row["cast_gbs"] = round(gbs, 1)
            row["cast_frac_hbm"] = round(gbs / hbm, 4)

        def gemm_call(i):
            _lib.call("vf4_gemm_nvfp4_ex", aps[i % R].data_ptr(), asfs[i % R].data_ptr(), ag.data_ptr(), wp.data_ptr(),
                      wsf.data_ptr(), wimg.data_ptr(), wg.data_ptr(), M, N, K, None, _lib.VF4_EPI_NONE,
                      outs[i % R].data_ptr(), _lib.VF4_BF16, None, None, None, None, None, stream())
        ms = _graph_time(gemm_call, 20)
        tf = 2.0 * M * N * K / (ms * 1e-3) / 1e12
        row.update(gemm_ms=round(ms, 4), gemm_tflops=round(tf, 1), gemm_frac_fp4_nominal=round(tf / FP4_NOMINAL_TFLOPS, 4),
                   gemm_frac_4x_bf16=round(tf / (4 * bf16_tf), 4))
        try:
            from torch.nn.functional import ScalingType, SwizzleType
            rec = [int(ScalingType.BlockWise1x16.value), int(ScalingType.TensorWise.value)]
            swz = [int(SwizzleType.SWIZZLE_32_4_4.value), int(SwizzleType.NO_SWIZZLE.value)]
            a4 = [t.view(torch.float4_e2m1fn_x2) for t in aps]
            b4 = wp.view(torch.float4_e2m1fn_x2).t()
            as8 = [t.view(torch.float8_e4m3fn) for t in asfs]
            bs8 = wsf.view(torch.float8_e4m3fn)
            ag1, wg1 = ag.reshape(1), wg.reshape(1)
            cub_out = [torch.empty(M, N, dtype=torch.bfloat16, device=dev) for _ in range(R)]

            def cublas_call(i):
                torch.ops.aten._scaled_mm_v2.out(a4[i % R], b4, [as8[i % R], ag1], rec, swz, [bs8, wg1], rec, swz,
                                                 None, torch.bfloat16, out=cub_out[i % R])
            cublas_call(0)
            gemm_call(0)
            torch.cuda.synchronize()
            agree = torch.nn.functional.cosine_similarity(cub_out[0].float().flatten(), outs[0].float().flatten(), dim=0)
            ms_c = _graph_time(cublas_call, 20)
            tf_c = 2.0 * M * N * K / (ms_c * 1e-3) / 1e12
            row.update(cublas_ms=round(ms_c, 4), cublas_tflops=round(tf_c, 1), vs_cublas=round(ms_c / ms, 3),
                       cublas_output_cos=round(float(agree), 6))
        except Exception as ex:  # pragma: no cover - depends on the box's torch / cuBLASLt
            row["cublas"] = f"unavailable: {type(ex).__name__}: {str(ex)[:160]}"
        rows.append(row)
        del xs, aps, asfs, outs, x, w
        torch.cuda.empty_cache()
    return rows


def model_rate(arch: dict, batch: int, attn: str, steps: int, peaks: dict, seq: int, label: str) -> dict:
    """images/s of one W4A4 model configuration on this GPU (graph replay), plus its per-kernel table."""
    import torch
    from vitfp4.pipeline import GraphedForward
    dev = torch.device("cuda")
    model, counts = build_model(arch, attn, dev)
    g = torch.Generator(device=dev).manual_seed(7)
    images = torch.randn(batch, 3, arch["img_size"], arch["img_size"], device=dev, generator=g).bfloat16()
    with torch.inference_mode():
        model(images)
        by_kind, launches = probe_pass(model, images, 1)
        gf = GraphedForward(model, images)
        ms = time_forward(lambda: gf.forward(0), steps)
        gf.release()
    res = {"workload": label, "images_per_s": round(batch * steps / (ms * 1e-3), 2), "ms_per_step": round(ms / steps, 3),
           "batch": batch, "seq_len": seq, "attention": attn, "gpu_launches_per_step": launches, **counts,
           "kernels": kernel_table(by_kind, 1)}
    attn_k = {k: v for k, v in by_kind.items() if k.startswith("attn")}
    if attn_k:
        fl = sum(v[1] for v in attn_k.values())
        t = sum(v[2] for v in attn_k.values())
        tf = fl / (t * 1e-3) / 1e12
        res["attention_tflops"] = round(tf, 1)
        nominal = FP4_NOMINAL_TFLOPS if attn == "nvfp4" else BF16_NOMINAL_TFLOPS
        res["attention_frac_of_nominal"] = round(tf / nominal, 4)
        res["attention_share_of_kernel_time"] = round(t / sum(v[2] for v in by_kind.values()), 4)
    del model, images
    torch.cuda.empty_cache()
    return res


def gptq_rate() -> dict:
    """GPTQ weight conversion on the GPU for the headline model's Linear shapes (ViT-L/14: qkv, proj,
    fc1, fc2): ms per layer of gptq_quantize_weight (block scales, Cholesky factors, the vf4_gptq_block
    column loop and the cross-block GEMMs), Hessian from 4096 calibration rows."""
    import torch
    from vitfp4.ptq import gptq_quantize_weight
    rows = []
    g = torch.Generator(device="cuda").manual_seed(5)
    for name, (n, k) in {"qkv": (3072, 1024), "proj": (1024, 1024), "fc1": (4096, 1024), "fc2": (1024, 4096)}.items():
        w = torch.randn(n, k, device="cuda", generator=g) * 0.02
        x = torch.randn(4096, k, device="cuda", generator=g)
        H = x.t() @ x
        gptq_quantize_weight(w, H)
        torch.cuda.synchronize()
        t0, t1 = _events()
        t0.record()
        for _ in range(3):
            gptq_quantize_weight(w, H)
        t1.record()
        torch.cuda.synchronize()
        rows.append({"layer": name, "N": n, "K": k, "ms": round(t0.elapsed_time(t1) / 3, 2)})
    return {"workload": "gptq_quantize_weight per Linear of ViT-L/14 (blocksize 128, percdamp 0.01)", "layers": rows,
            "ms_per_block_of_4": round(sum(r["ms"] for r in rows), 2)}


def secondary(args, peaks: dict) -> dict:
    from vitfp4 import vit
    out = {}
    t = time.time()
    out["config2_cast_gemm_sweep"] = {
        "workload": "BASELINE config 2: NVFP4 cast (static global) + block-scaled GEMM at ViT-B/16 linear shapes, "
                    "M = 256 x 197 = 50432; CUDA-graph timed, median of 3; cuBLASLt = torch._scaled_mm_v2 "
                    "(BlockWise1x16 + TensorWise) on the same packed operands",
        "shapes": gemm_sweep([(768, 2304), (768, 768), (768, 3072), (3072, 768)], 50432, peaks, "config2")}
    m4 = args.batch * 257
    out["config4_gemms_vs_cublas"] = {
        "workload": f"the headline's GEMM shapes at M = {m4} (qkv, proj, fc1, fc2), plain bf16 output",
        "shapes": gemm_sweep([(1024, 3072), (1024, 1024), (1024, 4096), (4096, 1024)], m4, peaks, "config4",
                             with_cast=False)}
    out["config3_vit_b16"] = model_rate(dict(vit.VIT_B16), 256, "nvfp4", 10, peaks, 197,
                                        "BASELINE config 3: ViT-B/16 W4A4, batch 256, FP4 QK^T/PV attention in all 12 blocks")
    out["config3_vit_b16_bf16_attention"] = model_rate(dict(vit.VIT_B16), 256, "bf16", 10, peaks, 197,
                                                       "config 3 model with the bf16 attention route, for comparison")
    out["config3_vit_b16_fp8_attention"] = model_rate(dict(vit.VIT_B16), 256, "fp8", 10, peaks, 197,
                                                      "config 3 model with the FP8 attention route (the reference's "
                                                      "enable_quant_attention default), for comparison")
    for attn in ("bf16", "fp8", "nvfp4"):
        out[f"config5_vit_h14_448_{attn}_attention"] = model_rate(
            dict(vit.VIT_H14_448), 64, attn, 5, peaks, 1025,
            f"BASELINE config 5: ViT-H/14 @448 (1025 tokens, head dim 80) W4A4, the 64 images of one GPU of 8, "
            f"{attn} attention" + {"bf16": " (cuDNN SDPA: the bf16 kernel covers S <= 288)",
                                   "fp8": " (the reference's default route; long-sequence FP8 kernels)",
                                   "nvfp4": " (long-sequence FP4 kernels)"}[attn])
    out["gptq_column_loop"] = gptq_rate()
    out["seconds"] = round(time.time() - t, 1)
    return out


# ------------------------------------------------------------------------------- vitfp4 arm
def run_vitfp4(args, rank: int, world: int, local_rank: int):
    import torch
    import torch.distributed as dist
    from vitfp4 import replica, vit
    from vitfp4.pipeline import GraphedForward, OverlappedRunner

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    _, per_rank = replica.shard_range(args.batch, rank, world)
    arch = dict(vit.VIT_L14)
    arch["depth"] = args.depth
    model, counts = build_model(arch, args.attn, dev, fused=not args.unfused, exact_gelu=args.gelu == "erf")
    gen = torch.Generator(device=dev).manual_seed(100 + rank)
    images = torch.randn(per_rank, 3, 224, 224, device=dev, generator=gen).to(torch.bfloat16)
    host_images = images.cpu().pin_memory()

    def barrier():
        if world > 1:
            dist.barrier()

    with torch.inference_mode():
        for _ in range(args.warmup):
            logits = model(images)
        torch.cuda.synchronize()
        if args.eager:
            fwd = lambda: model(images)   # noqa: E731
            gf = None
        else:
            gf = GraphedForward(model, images)
            fwd = lambda: gf.forward(0)   # noqa: E731
            for _ in range(args.warmup):
                fwd()

        # ---- device-resident timing (the headline `value`): nothing but the forwards in the region
        sampler = ClockSampler(local_rank) if rank == 0 else None
        if sampler:
            sampler.start()
            time.sleep(0.3)
        ms = time_forward(fwd, args.steps, barrier)
        clocks = sampler.stop() if sampler else None
        logits = gf.outputs[0] if gf is not None else model(images)

        # ---- end-to-end through the public runner with host buffers
        runner = OverlappedRunner(model, dev, graphed=not args.eager)
        runner.run([host_images] * min(2, args.steps))      # capture / buffers and pinned outputs
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        e0, e1 = _events()
        e0.record()
        outs = runner.run([host_images] * args.steps)
        e1.record()
        torch.cuda.synchronize()
        barrier()
        ms_e2e = e0.elapsed_time(e1)
        logits = logits.float().clone()
        runner = None
        if gf is not None:
            gf.release()

        # ---- per-kernel events and the eager host/device split, after the timed regions
        by_kind, launches = probe_pass(model, images, 2)
        host = eager_split(model, images, 2)

    ms, ms_e2e = replica.max_over_ranks([ms, ms_e2e], device=dev)
    replica.gather_logits(logits, args.batch)        # the single final gather of logits
    if rank != 0:
        return 0

    peaks = _peaks()
    steps = args.steps
    line = {
        "metric": METRIC, "value": round(args.batch * steps / (ms * 1e-3), 2), "unit": "images/s",
        "n_gpus": world, "steps": steps, "warmup": args.warmup, "ms_per_step": round(ms / steps, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "nvfp4 W4A4 (fp32 accumulate, bf16 activations)", "data": "synthetic",
        "config": {"workload": f"{MODEL} W4A4 forward, attention {args.attn}", "model": "ViT-L/14",
                   "global_batch": args.batch, "per_gpu_batch": per_rank, "seq_len": 257,
                   "depth": args.depth, "parallelism": f"dp{world} (independent replicas)",
                   "gelu": "erf (the reference's function; fc1 epilogue after the bf16 roundings of gemm and +b1)"
                           if args.gelu == "erf" else "tanh form (hardware tanh, not the reference's function)",
                   "launch": "eager" if args.eager else "CUDA graph replay of the whole forward",
                   "weights": "random N(0, 0.02) on the device, Four-Over-Six (mse) qkv/proj, RTN fc1/fc2",
                   "l2": "inputs larger than L2 (activations >= 0.5 GB per tensor), no flush", **counts},
        "e2e": {"value": round(args.batch * steps / (ms_e2e * 1e-3), 2), "unit": "images/s",
                "h2d_bytes_per_step": int(host_images.numel() * host_images.element_size() * world),
                "d2h_bytes_per_step": int(outs[-1].numel() * outs[-1].element_size() * world),
                "runner": "vitfp4.pipeline.OverlappedRunner" + ("" if args.eager else " (graphed)")},
        "gpu_launches": launches * steps,
        "host": {"eager": host, "note": "eager per-step device time vs host enqueue time of the same "
                                        "launches; the timed region replays a CUDA graph"},
        **rooflines(by_kind, peaks),
        "kernels": kernel_table(by_kind, 2),
        "clocks": clocks,
    }
    if world == 1 and not args.no_secondary:
        try:
            line["secondary"] = secondary(args, peaks)
        except Exception as ex:  # pragma: no cover
            line["secondary"] = {"error": f"{type(ex).__name__}: {str(ex)[:300]}"}
    if world == 1 and not args.no_cpu_baseline:
        try:
            cores = os.cpu_count() or 1
            torch.set_num_threads(cores)
            rate, times = cpu_forward_rate(args.attn, 2, 1, 0, args.depth)
            line["cpu_baseline"] = {"value": round(rate, 4), "unit": "images/s", "cores": cores, "kind": "port",
                                    "sample": "2 images, 1 timed forward (numpy restatement of the "
                                              "reference torch backend, same W4A4 ViT-L/14)"}
        except Exception as ex:  # pragma: no cover
            line["cpu_baseline"] = {"value": None, "error": repr(ex)[:200]}
    print(json.dumps(line), flush=True)
    return 0


def main():
    args = _args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch
        import torch.distributed as dist
        from vitfp4 import replica
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        if args.impl == "reference":
            return run_reference(args, rank, world)
        torch.cuda.set_device(local_rank)
        replica.init_from_env("nccl", timeout_s=120.0, device=torch.device("cuda", local_rank))
        try:
            return run_vitfp4(args, rank, world, local_rank)
        finally:
            dist.destroy_process_group()
    if args.impl == "reference":
        return run_reference(args, 0, 1)
    return run_vitfp4(args, 0, 1, 0)


if __name__ == "__main__":
    sys.exit(main())
