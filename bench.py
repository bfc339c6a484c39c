"""Benchmark: ViT-L/14 NVFP4 W4A4 inference images/s on 1..8 B200 (one replica per GPU).

    python bench.py [--gpus N --steps K --warmup W] [--impl reference] [--attn bf16|nvfp4]
    torchrun --nproc-per-node N ... bench.py --gpus N ...

Workload: DINOv2-style ViT-L/14 at 224x224 (257 tokens), 24 blocks, dim 1024,
16 heads, GELU MLP 4096, LayerScale 1e-5, random N(0, 0.02) weights, N(0,1) bf16 images, global
batch 1024 sharded evenly over the ranks.  Every block's qkv/proj are QuantLinear (Four-Over-Six
weights, dynamic NVFP4 activations) and every MLP is FusedNVFP4MLP (fused bias+GELU+NVFP4 fc1
epilogue); attention runs bf16 SDPA (default, the reference's unflagged route) or the FP4
attention kernels (--attn nvfp4).

Printed JSON line (rank 0): ``value`` = images/s of the whole job with inputs resident in HBM,
timed with CUDA events (max over ranks); ``e2e`` = the same through the public module call with
the images copied from pinned host memory and the logits read back every step.
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
# used when MEASURED_PEAKS.json is absent: an earlier measurement on the same B200 pool
# (STREAM-style copy and cuBLAS bf16 burst)
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}
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


def gemm_algorithmic_bytes(kind: str, m: int, n: int, k: int) -> int:
    """HBM bytes a GEMM launch must move: A and B codes + E4M3 scales in, plus its output
    (bf16; NVFP4 codes + scales for the GELU epilogue; residual read + bf16 write for fc2).
    For bf16 attention (m heads, n tokens, k head dim): q, k, v read and the output written once."""
    if kind == "attn_bf16":
        return m * n * k * 2 * 4
    operands = (m + n) * (k // 2 + k // 16)
    if kind == "gemm_gelu_nvfp4":
        return operands + m * (n // 2 + n // 16)
    if kind == "gemm_residual":
        return operands + 2 * m * n * 2
    return operands + m * n * 2


def roofline_entry(name: str, flops: float, ms: float, bf16_tf: float, measured: bool) -> dict:
    """Roofline object of one timed kernel kind ("<kind>_<m>x<n>x<k>"): its FLOPs over its summed
    launch durations, against the bf16 peak for the bf16 attention kernel and 4 x the bf16 peak for
    the FP4 GEMMs, with the algorithmic bytes of one launch and the ncu DRAM bytes where captured."""
    achieved = flops / (ms * 1e-3) / 1e12
    src = "measured bf16 burst (MEASURED_PEAKS.json), of measured" if measured else \
        "fallback bf16 burst 1590 TFLOP/s (MEASURED_PEAKS.json absent), of fallback"
    if name.startswith("attn_bf16"):     # bf16 tensor-core kernel
        peak, peak_source, nominal = bf16_tf, src, 2250.0
    else:                                # FP4 GEMMs: FP4 itself is not measured
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
            "scaled by heads" if kind == "attn_bf16" else
            "ncu dram__bytes_read.sum + dram__bytes_write.sum of one launch at M = 65792, scaled by rows")
    return r


def _args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="vitfp4", choices=["vitfp4", "reference"])
    ap.add_argument("--attn", default="bf16", choices=["bf16", "nvfp4"])
    ap.add_argument("--batch", type=int, default=GLOBAL_BATCH, help="global batch (images)")
    ap.add_argument("--depth", type=int, default=24)
    ap.add_argument("--no-cpu-baseline", action="store_true")
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
    import numpy as np  # noqa: F401
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


# ------------------------------------------------------------------------------- vitfp4 arm
def build_model(depth: int, attn: str, device, fused: bool = True):
    import torch
    from vitfp4 import vit
    from vitfp4.ptq import enable_quant_attention, fuse_mlps, fuse_norms, quantize_vit, vit_attn_policy
    cfg = dict(vit.VIT_L14)
    cfg["depth"] = depth
    model = vit.build_vit(seed=0, **cfg).to(device=device, dtype=torch.bfloat16).eval()
    n_mlp = fuse_mlps(model, skip_ends=0)
    n_lin, spec = quantize_vit(model, skip_first=0, skip_last=0, w_block_select="mse")
    n_att = 0
    if attn == "nvfp4":
        n_att = enable_quant_attention(model, vit_attn_policy(depth, 0, 0, "blocks"), qk="nvfp4", pv="nvfp4")
    n_blk = fuse_norms(model) if fused else 0
    return model, {"fused_mlps": n_mlp, "quant_linears": n_lin, "fp4_attention": n_att, "fused_blocks": n_blk}


def run_vitfp4(args, rank: int, world: int, local_rank: int):
    import torch
    import torch.distributed as dist
    from vitfp4 import replica
    from vitfp4.nvfp4 import ops
    from vitfp4.pipeline import OverlappedRunner

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    _, per_rank = replica.shard_range(args.batch, rank, world)
    torch.manual_seed(1234 + rank)
    model, counts = build_model(args.depth, args.attn, dev, fused=not args.unfused)
    gen = torch.Generator(device=dev).manual_seed(100 + rank)
    images = torch.randn(per_rank, 3, 224, 224, device=dev, generator=gen).to(torch.bfloat16)
    host_images = images.cpu().pin_memory()
    stream = torch.cuda.current_stream()

    def barrier():
        if world > 1:
            dist.barrier()

    with torch.inference_mode():
        for _ in range(args.warmup):
            logits = model(images)
        torch.cuda.synchronize()

        # ---- device-resident timing (the headline `value`)
        sampler = ClockSampler(local_rank) if rank == 0 else None
        if sampler:
            sampler.start()
            time.sleep(0.3)
        ops.probe.reset()
        ops.probe.timing = True
        barrier()
        torch.cuda.synchronize()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for _ in range(args.steps):
            logits = model(images)
        t1.record(stream)
        torch.cuda.synchronize()
        barrier()
        ops.probe.timing = False
        launches = ops.probe.launches
        records = list(ops.probe.records)
        clocks = sampler.stop() if sampler else None
        ms = t0.elapsed_time(t1)

        # ---- end-to-end through the public call with host buffers
        barrier()
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        # every step copies its images from pinned host memory and reads its logits back; the
        # runner overlaps step i+1's copy and step i-1's read-back with step i's forward
        runner = OverlappedRunner(model, dev)
        runner.run([host_images] * min(2, args.steps))      # buffers and pinned outputs allocated
        torch.cuda.synchronize()
        e0.record(stream)
        outs = runner.run([host_images] * args.steps)
        e1.record(stream)
        torch.cuda.synchronize()
        barrier()
        ms_e2e = e0.elapsed_time(e1)

    # per-kernel GEMM timing from the live events of the timed region
    by_kind: dict = {}
    for kind, flops, s, e in records:
        d = by_kind.setdefault(kind, [0, 0.0, 0.0])
        d[0] += 1
        d[1] += flops
        d[2] += s.elapsed_time(e)
    ms, ms_e2e = replica.max_over_ranks([ms, ms_e2e], device=dev)
    replica.gather_logits(logits.float(), args.batch)        # the single final gather of logits
    if rank != 0:
        return 0

    peaks = _peaks()
    measured = bool(peaks.get("bf16_tflops"))
    bf16_tf = peaks["bf16_tflops"] if measured else FALLBACK_PEAKS["bf16_tflops"]
    kernels = {k: {"launches": v[0], "ms_total": round(v[2], 3),
                   "tflops": round(v[1] / (v[2] * 1e-3) / 1e12, 1)} for k, v in sorted(by_kind.items())}
    # the dominant kernel by device time, and (the metric's second figure) the dominant NVFP4 GEMM
    dom = max(by_kind.items(), key=lambda kv: kv[1][2]) if by_kind else None
    gemms = {k: v for k, v in by_kind.items() if k.startswith("gemm")}
    dom_gemm = max(gemms.items(), key=lambda kv: kv[1][2]) if gemms else None
    roofline = roofline_entry(dom[0], dom[1][1], dom[1][2], bf16_tf, measured) if dom else None
    gemm_roofline = roofline_entry(dom_gemm[0], dom_gemm[1][1], dom_gemm[1][2], bf16_tf, measured) if dom_gemm else None
    steps = args.steps
    img_per_step = args.batch
    line = {
        "metric": METRIC, "value": round(img_per_step * steps / (ms * 1e-3), 2), "unit": "images/s",
        "n_gpus": world, "steps": steps, "warmup": args.warmup, "ms_per_step": round(ms / steps, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "nvfp4 W4A4 (fp32 accumulate, bf16 activations)", "data": "synthetic",
        "config": {"workload": f"{MODEL} W4A4 forward, attention {args.attn}", "model": "ViT-L/14",
                   "global_batch": img_per_step, "per_gpu_batch": per_rank, "seq_len": 257,
                   "depth": args.depth, "parallelism": f"dp{world} (independent replicas)",
                   "l2": "inputs larger than L2 (activations >= 0.5 GB per tensor)", **counts},
        "e2e": {"value": round(img_per_step * steps / (ms_e2e * 1e-3), 2), "unit": "images/s",
                "h2d_bytes_per_step": int(host_images.numel() * host_images.element_size() * world),
                "d2h_bytes_per_step": int(outs[-1].numel() * outs[-1].element_size() * world)},
        "gpu_launches": launches,
        "roofline": roofline,
        "gemm_roofline": gemm_roofline,
        "kernels": kernels,
        "clocks": clocks,
    }
    if world == 1 and not args.no_cpu_baseline:
        try:
            cores = os.cpu_count() or 1
            torch.set_num_threads(cores)
            rate, times = cpu_forward_rate(args.attn, 1, 1, 0, args.depth)
            line["cpu_baseline"] = {"value": round(rate, 4), "unit": "images/s", "cores": cores, "kind": "port",
                                    "sample": "1 image, 1 timed forward (numpy restatement of the "
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
