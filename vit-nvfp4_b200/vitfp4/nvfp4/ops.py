"""Tensor-level wrappers over the C ABI (include/vitfp4.h).

Every function here launches the sm_100a kernels of libvitfp4.so on torch's current CUDA
stream and allocates its outputs with torch.  Inputs must be CUDA tensors; there is no
CPU path.
"""
from __future__ import annotations

import torch

from .. import _lib

SF_TORCH_DTYPE = torch.uint8  # E4M3 bytes are carried as uint8 internally


class Probe:
    """Launch accounting for the benchmark: counts libvitfp4 kernel launches and, when
    ``timing`` is on, brackets every GEMM, attention and cast call with CUDA events on the
    launching stream.  Each record is (kind, work, start, end): ``work`` is the call's FLOPs for
    GEMM and attention kinds and its algorithmic HBM bytes for cast kinds (names starting with
    "cast" or "ln_cast")."""

    def __init__(self):
        self.launches = 0
        self.timing = False
        self.records: list = []   # (kind, work, start_event, end_event)

    def reset(self):
        self.launches = 0
        self.records = []


probe = Probe()


def _launched(n: int = 1) -> None:
    probe.launches += n


class _Timed:
    def __init__(self, kind: str, work: float):
        self.kind, self.work = kind, work

    def __enter__(self):
        if probe.timing:
            self.s = torch.cuda.Event(enable_timing=True)
            self.e = torch.cuda.Event(enable_timing=True)
            self.s.record()
        return self

    def __exit__(self, *a):
        if probe.timing:
            self.e.record()
            probe.records.append((self.kind, self.work, self.s, self.e))


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _need_cuda(*ts: torch.Tensor | None) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise _lib.VitFp4Error("vitfp4 kernels run on CUDA (sm_100a) tensors only; got a "
                                   f"{t.device} tensor (no CPU fallback)")


def _dtype_code(t: torch.Tensor) -> int:
    if t.dtype == torch.bfloat16:
        return _lib.VF4_BF16
    if t.dtype == torch.float32:
        return _lib.VF4_F32
    raise _lib.VitFp4Error(f"unsupported dtype {t.dtype} (bf16 or fp32)")


def sf_swizzled_numel(rows: int, k: int) -> int:
    """Bytes of the 128x4-tiled scale layout for (rows, k/16) scales."""
    nb = k // 16
    return ((rows + 127) // 128 * 128) * ((nb + 3) // 4 * 4)


def _as_2d_input(x: torch.Tensor) -> tuple[torch.Tensor, int, int, int]:
    """(M, K) view with unit column stride and 16-byte-aligned rows (copies only if needed)."""
    K = x.shape[-1]
    x2 = x.reshape(-1, K)
    if x2.dtype not in (torch.bfloat16, torch.float32):
        x2 = x2.float()
    esz = x2.element_size()
    if x2.stride(-1) != 1 or (x2.stride(0) * esz) % 16 or x2.data_ptr() % 16 or x2.stride(0) < K:
        x2 = x2.contiguous()
        if x2.data_ptr() % 16:
            x2 = x2.clone()
    return x2, x2.shape[0], K, x2.stride(0) if x2.shape[0] > 1 else K


def amax(x: torch.Tensor, gelu: bool = False) -> torch.Tensor:
    """max|x| (or max|GELU(x)|) as a 0-dim fp32 device tensor."""
    _need_cuda(x)
    xc = x.contiguous()
    if xc.dtype not in (torch.bfloat16, torch.float32):
        xc = xc.float()
    out = torch.empty((), dtype=torch.float32, device=x.device)
    _lib.call("vf4_amax", _ptr(xc), _dtype_code(xc), xc.numel(), int(gelu), _ptr(out), _stream())
    _launched()
    return out


def global_scale(amax_t: torch.Tensor, block_select: str = "six") -> torch.Tensor:
    _need_cuda(amax_t)
    out = torch.empty((), dtype=torch.float32, device=amax_t.device)
    _lib.call("vf4_global_scale", _ptr(amax_t.float().contiguous()), 1 if block_select == "mse" else 0,
              _ptr(out), _stream())
    _launched()
    return out


def cast(x: torch.Tensor, gs: torch.Tensor | None = None, block_select: str = "six", gelu: bool = False,
         bias: torch.Tensor | None = None, swizzled: bool = True, linear: bool = False):
    """NVFP4 cast of x (..., K) along K.

    Returns (packed uint8 (M, K/2), sf_swizzled uint8 flat or None, sf_linear uint8 (M, K/16) or
    None, gs 0-dim fp32).  ``gs`` None -> dynamic global scale from the tensor amax.
    """
    _need_cuda(x, gs, bias)
    x2, M, K, ld = _as_2d_input(x)
    if K % 16:
        raise _lib.VitFp4Error(f"NVFP4 needs K % 16 == 0 (K={K})")
    dev = x.device
    packed = torch.empty((M, K // 2), dtype=torch.uint8, device=dev)
    sfs = torch.empty(sf_swizzled_numel(M, K), dtype=torch.uint8, device=dev) if swizzled else None
    sfl = torch.empty((M, K // 16), dtype=torch.uint8, device=dev) if linear else None
    gs_in = None if gs is None else gs.reshape(()).to(torch.float32).contiguous()
    gs_out = torch.empty((), dtype=torch.float32, device=dev) if gs_in is None else None
    b = None
    if bias is not None:
        b = bias.to(x2.dtype).contiguous()
    esz = x2.element_size()
    with _Timed(f"cast_{'static' if gs_in is not None else 'dynamic'}_{M}x{K}",
                M * K * (esz + 0.5 + 1 / 16 + (0 if gs_in is not None else esz))):
        _lib.call("vf4_cast_nvfp4", _ptr(x2), _dtype_code(x2), M, K, ld, _ptr(gs_in),
                  1 if block_select == "mse" else 0, int(gelu), _ptr(b), _ptr(packed), _ptr(sfs), _ptr(sfl),
                  _ptr(gs_out), _stream())
    _launched(1 if gs_in is not None else 3)
    return packed, sfs, sfl, (gs_out if gs_in is None else gs_in)


def cast_split(x_main: torch.Tensor, x_tail: torch.Tensor, gs: torch.Tensor | None = None):
    """NVFP4 cast (six) of an operand whose rows come in two parts per image: x_main (n, rows_main, K)
    and x_tail (n, rows_tail, K) bf16; output row i * (rows_main + rows_tail) + t is main row t of
    image i, the tail rows follow.  Same codes, scales and global as ``cast`` of the concatenated
    (n, rows_main + rows_tail, K) tensor, without building it.  Returns (packed, sf_swizzled, gs)."""
    _need_cuda(x_main, x_tail, gs)
    a, b = x_main.contiguous(), x_tail.contiguous()
    n, rm, K = a.shape
    rt = b.shape[1]
    M = n * (rm + rt)
    packed = torch.empty((M, K // 2), dtype=torch.uint8, device=a.device)
    sfs = torch.empty(sf_swizzled_numel(M, K), dtype=torch.uint8, device=a.device)
    gs_in = None if gs is None else gs.reshape(()).to(torch.float32).contiguous()
    gs_out = torch.empty((), dtype=torch.float32, device=a.device) if gs_in is None else None
    with _Timed(f"cast_split_{'static' if gs_in is not None else 'dynamic'}_{M}x{K}",
                M * K * (2.5625 + (0 if gs_in is not None else 2))):
        _lib.call("vf4_cast_nvfp4_split", _ptr(a), rm, _ptr(b), rt, n, K, _ptr(gs_in), _ptr(gs_out), _ptr(packed),
                  _ptr(sfs), _stream())
    _launched(2 if gs_in is not None else 5)
    return packed, sfs, (gs_out if gs_in is None else gs_in)


def pack_e2m1(codes: torch.Tensor) -> torch.Tensor:
    _need_cuda(codes)
    c = codes.contiguous()
    assert c.dtype == torch.uint8 and c.shape[-1] % 2 == 0
    out = torch.empty((*c.shape[:-1], c.shape[-1] // 2), dtype=torch.uint8, device=c.device)
    rows = c.numel() // max(c.shape[-1], 1) if c.numel() else 0
    _lib.call("vf4_pack_e2m1", _ptr(c), rows, c.shape[-1], _ptr(out), _stream())
    _launched()
    return out


def unpack_e2m1(packed: torch.Tensor) -> torch.Tensor:
    _need_cuda(packed)
    p = packed.contiguous()
    if p.dtype != torch.uint8:
        p = p.view(torch.uint8)
    out = torch.empty((*p.shape[:-1], p.shape[-1] * 2), dtype=torch.uint8, device=p.device)
    rows = p.numel() // max(p.shape[-1], 1) if p.numel() else 0
    _lib.call("vf4_unpack_e2m1", _ptr(p), rows, p.shape[-1], _ptr(out), _stream())
    _launched()
    return out


def gptq_block(w: torch.Tensor, hinv: torch.Tensor, block_scale: torch.Tensor, global_scale: torch.Tensor,
               col0: int, count: int, codes: torch.Tensor, err: torch.Tensor) -> None:
    """GPTQ column loop over columns [col0, col0 + count) (vf4_gptq_block).

    ``w``: fp32 (N, >= count) view whose column 0 is weight column col0 (unit column stride);
    ``hinv``: fp32 (count, count) view (unit column stride); ``block_scale``: (N, K/16) E4M3 bytes of
    the whole weight; ``global_scale``: one fp32; writes ``codes`` (N, K) uint8 columns
    [col0, col0 + count) and ``err`` (N, count) fp32."""
    _need_cuda(w, hinv, block_scale, global_scale, codes, err)
    if w.dtype != torch.float32 or hinv.dtype != torch.float32 or err.dtype != torch.float32:
        raise _lib.VitFp4Error("gptq_block takes fp32 w / hinv / err")
    bs = block_scale if block_scale.dtype == torch.uint8 else block_scale.view(torch.uint8)
    w, hinv, bs = (t if t.stride(-1) == 1 else t.contiguous() for t in (w, hinv, bs))   # read-only inputs
    for t in (codes, err):
        if t.stride(-1) != 1:
            raise _lib.VitFp4Error("gptq_block writes codes / err with unit column strides")
    gs = global_scale.reshape(()).to(torch.float32)
    _lib.call("vf4_gptq_block", _ptr(w), w.stride(0), _ptr(hinv), hinv.stride(0), _ptr(bs), bs.stride(0), _ptr(gs),
              w.shape[0], col0, count, _ptr(codes), codes.stride(0), _ptr(err), err.stride(0), _stream())
    _launched()


def to_blocked(sf: torch.Tensor) -> torch.Tensor:
    """(R, C) E4M3 scales (uint8 or float8_e4m3fn) -> flat 128x4-tiled uint8."""
    _need_cuda(sf)
    s = sf.contiguous()
    if s.dtype != torch.uint8:
        s = s.view(torch.uint8)
    R, C = s.shape
    out = torch.empty(((R + 127) // 128 * 128) * ((C + 3) // 4 * 4), dtype=torch.uint8, device=s.device)
    _lib.call("vf4_to_blocked", _ptr(s), R, C, _ptr(out), _stream())
    _launched()
    return out


def _u8(t: torch.Tensor) -> torch.Tensor:
    t = t.contiguous()
    return t if t.dtype == torch.uint8 else t.view(torch.uint8)


def gemm(a_packed: torch.Tensor, a_sf: torch.Tensor, a_gs: torch.Tensor, b_packed: torch.Tensor,
         b_sf: torch.Tensor, b_gs: torch.Tensor, bias: torch.Tensor | None = None,
         out_dtype: torch.dtype = torch.bfloat16, b_image: torch.Tensor | None = None) -> torch.Tensor:
    """(M, K/2) x (N, K/2) packed NVFP4 with swizzled scales -> (M, N) out_dtype (+bias); ``b_image``
    (``b_scale_image`` of b_sf) speeds the K > 1024 kernel up."""
    _need_cuda(a_packed, b_packed)
    a, b = _u8(a_packed), _u8(b_packed)
    M, Kh = a.shape
    N = b.shape[0]
    assert b.shape[1] == Kh, (a.shape, b.shape)
    K = Kh * 2
    od = torch.float32 if out_dtype == torch.float32 else torch.bfloat16
    out = torch.empty((M, N), dtype=od, device=a.device)
    bb = None
    epi = _lib.VF4_EPI_NONE
    post_bias = None
    if bias is not None:
        if od == torch.float32 and bias.dtype == torch.float32:
            post_bias = bias
        else:
            bb = bias.to(torch.bfloat16).contiguous()
            epi = _lib.VF4_EPI_BIAS
    with _Timed(f"gemm_{'bias' if epi else 'none'}_{M}x{N}x{K}", 2.0 * M * N * K):
        if b_image is None:
            _lib.call("vf4_gemm_nvfp4", _ptr(a), _ptr(_u8(a_sf)), _ptr(a_gs.float().contiguous()), _ptr(b),
                      _ptr(_u8(b_sf)), _ptr(b_gs.float().contiguous()), M, N, K, _ptr(bb), epi, _ptr(out),
                      _lib.VF4_F32 if od == torch.float32 else _lib.VF4_BF16, None, None, None, _stream())
        else:
            _lib.call("vf4_gemm_nvfp4_ex", _ptr(a), _ptr(_u8(a_sf)), _ptr(a_gs.float().contiguous()), _ptr(b),
                      _ptr(_u8(b_sf)), _ptr(_u8(b_image)), _ptr(b_gs.float().contiguous()), M, N, K, _ptr(bb), epi,
                      _ptr(out), _lib.VF4_F32 if od == torch.float32 else _lib.VF4_BF16, None, None, None, None,
                      None, _stream())
    _launched()
    if post_bias is not None:
        out += post_bias
    if out_dtype not in (torch.float32, torch.bfloat16):
        out = out.to(out_dtype)
    return out


def b_scale_image(b_sf: torch.Tensor, N: int, K: int) -> torch.Tensor:
    """The B scale image of an (N, K) weight's to_blocked scales (``vf4_b_scale_image``): with it the
    streaming GEMM kernel (K > 1024, N >= 256) copies each K64 block's B scales into tensor memory
    with one instruction instead of two.  Build it once per weight."""
    sf = _u8(b_sf)
    _need_cuda(sf)
    img = torch.empty(int(_lib.lib().vf4_b_scale_image_bytes(N, K)), dtype=torch.uint8, device=sf.device)
    _lib.call("vf4_b_scale_image", _ptr(sf), N, K, _ptr(img), _stream())
    _launched()
    return img


def gemm_residual(a_packed, a_sf, a_gs, b_packed, b_sf, b_gs, bias, residual: torch.Tensor,
                  gamma: torch.Tensor | None = None, out: torch.Tensor | None = None,
                  b_image: torch.Tensor | None = None) -> torch.Tensor:
    """``residual + gamma * (A @ B^T + bias)`` in bf16 with the unfused block's roundings (GEMM
    result, bias add, LayerScale product and residual add each round to bf16); ``out`` may be
    ``residual`` itself; ``b_image`` (``b_scale_image`` of b_sf) speeds the K > 1024 kernel up."""
    _need_cuda(a_packed, b_packed, residual)
    a, b = _u8(a_packed), _u8(b_packed)
    M, Kh = a.shape
    N = b.shape[0]
    assert residual.shape == (M, N) and residual.dtype == torch.bfloat16 and residual.is_contiguous()
    if out is None:
        out = torch.empty((M, N), dtype=torch.bfloat16, device=a.device)
    bb = None if bias is None else bias.to(torch.bfloat16).contiguous()
    gg = None if gamma is None else gamma.to(torch.bfloat16).contiguous()
    with _Timed(f"gemm_residual_{M}x{N}x{Kh * 2}", 2.0 * M * N * Kh * 2):
        if b_image is None:
            _lib.call("vf4_gemm_nvfp4_residual", _ptr(a), _ptr(_u8(a_sf)), _ptr(a_gs.float().contiguous()), _ptr(b),
                      _ptr(_u8(b_sf)), _ptr(b_gs.float().contiguous()), M, N, Kh * 2, _ptr(bb), _ptr(residual),
                      _ptr(gg), _ptr(out), _stream())
        else:
            _lib.call("vf4_gemm_nvfp4_ex", _ptr(a), _ptr(_u8(a_sf)), _ptr(a_gs.float().contiguous()), _ptr(b),
                      _ptr(_u8(b_sf)), _ptr(_u8(b_image)), _ptr(b_gs.float().contiguous()), M, N, Kh * 2, _ptr(bb),
                      _lib.VF4_EPI_BIAS_RESIDUAL, _ptr(out), _lib.VF4_BF16, None, None, None, _ptr(residual),
                      _ptr(gg), _stream())
    _launched()
    return out


def gemm_gelu_nvfp4(a_packed, a_sf, a_gs, b_packed, b_sf, b_gs, bias, epi_gs, exact: bool = False):
    """fc1 GEMM with the fused +bias -> GELU -> NVFP4 cast epilogue.

    GELU is the tanh form (hardware tanh, ~1e-3 from erf-GELU) unless ``exact`` (erf to 1.5e-7).
    Returns (packed uint8 (M, N/2), sf_swizzled uint8 flat) quantized with the static epi_gs."""
    _need_cuda(a_packed, b_packed, epi_gs)
    a, b = _u8(a_packed), _u8(b_packed)
    M, Kh = a.shape
    N = b.shape[0]
    packed = torch.empty((M, N // 2), dtype=torch.uint8, device=a.device)
    sf = torch.empty(sf_swizzled_numel(M, N), dtype=torch.uint8, device=a.device)
    bb = None if bias is None else bias.to(torch.bfloat16).contiguous()
    with _Timed(f"gemm_gelu_nvfp4_{M}x{N}x{Kh * 2}", 2.0 * M * N * Kh * 2):
        _lib.call("vf4_gemm_nvfp4", _ptr(a), _ptr(_u8(a_sf)), _ptr(a_gs.float().contiguous()), _ptr(b),
                  _ptr(_u8(b_sf)), _ptr(b_gs.float().contiguous()), M, N, Kh * 2, _ptr(bb),
                  _lib.VF4_EPI_GELU_ERF_NVFP4 if exact else _lib.VF4_EPI_GELU_NVFP4, None, _lib.VF4_BF16,
                  _ptr(epi_gs.reshape(()).float().contiguous()),
                  _ptr(packed), _ptr(sf), _stream())
    _launched()
    return packed, sf


_ws_cache: dict = {}


def _attn_workspace(B: int, H: int, S: int, D: int, device, flags: int = 0) -> torch.Tensor:
    return _workspace(int(_lib.lib().vf4_attn_workspace_size_ex(B, H, S, D, flags)), device)


def _workspace(n: int, device) -> torch.Tensor:
    """An attention workspace of at least ``n`` bytes, kept per (device, stream) and grown on demand."""
    key = (device, torch.cuda.current_stream(device).cuda_stream)
    ws = _ws_cache.get(key)
    if ws is None or ws.numel() < n:
        ws = torch.empty(n, dtype=torch.uint8, device=device)
        _ws_cache[key] = ws
    return ws


def _smooth_flags(smooth_k: bool, smooth_v: bool) -> int:
    return (0 if smooth_k else _lib.VF4_ATTN_NO_SMOOTH_K) | (0 if smooth_v else _lib.VF4_ATTN_NO_SMOOTH_V)


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, B: int, H: int, S: int, D: int,
              strides: tuple[int, int, int], scale: float, out: torch.Tensor,
              out_strides: tuple[int, int, int], head_globals: bool = False, packed: bool = True,
              smooth_k: bool = True, smooth_v: bool = True) -> torch.Tensor:
    """NVFP4 attention over bf16 q/k/v views sharing (stride_b, stride_h, stride_s) element strides.

    Global scales of Q, K~, V~ over the whole tensors (the reference's) unless ``head_globals``.
    ``packed`` (head dim 64, S <= 320): operands quantized by a separate pass into per-head images
    in the workspace (~38 KB per image and head), the faster route; False keeps the quantization
    inside the fused kernel (512 B of workspace per head).  ``smooth_k`` / ``smooth_v`` False switch off
    the reference's smooth-K / smooth-V (tensor-wide globals only)."""
    _need_cuda(q, k, v, out)
    for t in (q, k, v, out):
        if t.dtype != torch.bfloat16:
            raise _lib.VitFp4Error("FP4 attention takes bf16 q/k/v/out")
    flags = (_lib.VF4_ATTN_HEAD_GLOBALS if head_globals else 0) | (_lib.VF4_ATTN_PACKED if packed else 0) | \
        _smooth_flags(smooth_k, smooth_v)
    ws = _attn_workspace(B, H, S, D, q.device, flags)
    with _Timed(f"attn_nvfp4_{B * H}x{S}x{D}", 4.0 * B * H * S * S * D):
        _lib.call("vf4_attn_nvfp4_ex", _ptr(q), _ptr(k), _ptr(v), B, H, S, D, strides[0], strides[1], strides[2],
                  float(scale), _ptr(out), out_strides[0], out_strides[1], out_strides[2], flags,
                  _ptr(ws) if ws.numel() else None, ws.numel(), _stream())
    fused = D == 64 and S <= 320
    _launched((0 if head_globals else 1) + (1 if fused else 2) + (1 if fused and packed else 0))
    return out


def attention_fp8(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, B: int, H: int, S: int, D: int,
                  strides: tuple[int, int, int], scale: float, out: torch.Tensor,
                  out_strides: tuple[int, int, int], smooth_k: bool = True, smooth_v: bool = True) -> torch.Tensor:
    """FP8 (E4M3, per-row scales) attention over bf16 q/k/v views sharing element strides (through the
    unified vf4_attn entry with qk = pv = fp8)."""
    _need_cuda(q, k, v, out)
    for t in (q, k, v, out):
        if t.dtype != torch.bfloat16:
            raise _lib.VitFp4Error("FP8 attention takes bf16 q/k/v/out")
    fp8 = _lib.VF4_ATTN_MODE["fp8"]
    flags = _smooth_flags(smooth_k, smooth_v)
    n = int(_lib.lib().vf4_attn_workspace_size_modes(B, H, S, D, fp8, fp8, flags))
    ws = _workspace(n, q.device) if n > 0 else None
    with _Timed(f"attn_fp8_{B * H}x{S}x{D}", 4.0 * B * H * S * S * D):
        _lib.call("vf4_attn", _ptr(q), _ptr(k), _ptr(v), B, H, S, D, strides[0], strides[1], strides[2],
                  float(scale), fp8, fp8, flags, _ptr(ws) if ws is not None else None, n, _ptr(out),
                  out_strides[0], out_strides[1], out_strides[2], _stream())
    _launched(1 if ws is None else 3)   # short route: one kernel; long: statistics, pack, forward
    return out


def _fp8_long_smem(S: int, D: int) -> int:
    """Shared memory of the long-sequence FP8 kernel (f8l_smem_layout in vf4_attn.cu): the head's K~8 and
    key scales, one Q8 tile, three V~8^T chunks, two P8 chunks, row reductions, barriers, alignment slack."""
    s_pad = -(-S // 128) * 128
    dk = -(-D // 32) * 32
    return s_pad * dk + s_pad * 4 + 128 * dk + 3 * D * 128 + 2 * 128 * 128 + 2 * 4 * 128 * 4 + 256 + 1024


def fp8_kernel_ok(S: int, D: int) -> bool:
    """Shapes the FP8 kernels take: head dim 64 with S <= 320 (one fused kernel), else head dims that are
    multiples of 16 up to 128 whose keys fit shared memory (prep + long-sequence kernel)."""
    if S < 1 or D < 16 or D > 128 or D % 16:
        return False
    return (D == 64 and S <= 320) or _fp8_long_smem(S, D) <= 227 * 1024


def attention_bf16(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, B: int, H: int, S: int, D: int,
                   strides: tuple[int, int, int], scale: float, out: torch.Tensor,
                   out_strides: tuple[int, int, int], out_amax: torch.Tensor | None = None) -> torch.Tensor:
    """Exact-softmax bf16 attention (tcgen05 kind::f16) over bf16 q/k/v views sharing element strides;
    ``out_amax`` (0-dim fp32) receives max |out| when given."""
    _need_cuda(q, k, v, out, out_amax)
    for t in (q, k, v, out):
        if t.dtype != torch.bfloat16:
            raise _lib.VitFp4Error("bf16 attention takes bf16 q/k/v/out")
    if out_amax is not None and (out_amax.dtype != torch.float32 or out_amax.numel() != 1):
        raise _lib.VitFp4Error("out_amax must be one fp32 value")
    with _Timed(f"attn_bf16_{B * H}x{S}x{D}", 4.0 * B * H * S * S * D):
        _lib.call("vf4_attn_bf16", _ptr(q), _ptr(k), _ptr(v), B, H, S, D, strides[0], strides[1], strides[2],
                  float(scale), _ptr(out), out_strides[0], out_strides[1], out_strides[2], _ptr(out_amax), _stream())
    _launched(1)
    return out


def bf16_kernel_ok(S: int, D: int, scale: float = 1.0) -> bool:
    """Shapes (and softmax scales: >= 0) the bf16 attention kernel takes."""
    return D == 64 and 1 <= S <= 288 and scale >= 0.0


def attention_bf16_packed_qkv(qkv: torch.Tensor, num_heads: int, scale: float,
                              out_amax: torch.Tensor | None = None) -> torch.Tensor:
    """Packed (B, S, 3*H*D) bf16 projection output -> (B, S, H*D) bf16 through the bf16 kernel."""
    B, S, C3 = qkv.shape
    H = num_heads
    D = C3 // (3 * H)
    x = qkv if qkv.is_contiguous() else qkv.contiguous()
    out = torch.empty((B, S, H * D), dtype=torch.bfloat16, device=qkv.device)
    attention_bf16(x, x[..., H * D:], x[..., 2 * H * D:], B, H, S, D, (S * C3, D, C3), scale, out,
                   (S * H * D, D, H * D), out_amax=out_amax)
    return out


def _bhsd_operands(q, k, v):
    B, H, S, D = q.shape
    qb, kb, vb = (t if t.dtype == torch.bfloat16 else t.to(torch.bfloat16) for t in (q, k, v))
    st = qb.stride()
    shared = (kb.stride() == st and vb.stride() == st and st[3] == 1 and all(x % 8 == 0 for x in st[:3])
              and all(t.data_ptr() % 16 == 0 for t in (qb, kb, vb)))
    if shared:
        return qb, kb, vb, (st[0], st[1], st[2])
    qb, kb, vb = (t.contiguous() for t in (qb, kb, vb))
    return qb, kb, vb, (H * S * D, S * D, D)


def attention_fp8_bhsd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float, smooth_k: bool = True,
                       smooth_v: bool = True) -> torch.Tensor:
    """(B, H, S, D) q/k/v -> (B, H, S, D) bf16 through the FP8 kernel."""
    B, H, S, D = q.shape
    qb, kb, vb, strides = _bhsd_operands(q, k, v)
    out = torch.empty((B, S, H, D), dtype=torch.bfloat16, device=q.device)
    attention_fp8(qb, kb, vb, B, H, S, D, strides, scale, out, (S * H * D, D, H * D), smooth_k, smooth_v)
    return out.transpose(1, 2)


def attention_bhsd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float,
                   head_globals: bool = False, packed: bool = True, smooth_k: bool = True,
                   smooth_v: bool = True) -> torch.Tensor:
    """(B, H, S, D) q/k/v (any dtype; cast to bf16) -> (B, H, S, D) bf16."""
    B, H, S, D = q.shape
    qb, kb, vb = (t if t.dtype == torch.bfloat16 else t.to(torch.bfloat16) for t in (q, k, v))
    st = qb.stride()
    shared = (kb.stride() == st and vb.stride() == st and st[3] == 1 and all(x % 8 == 0 for x in st[:3])
              and all(t.data_ptr() % 16 == 0 for t in (qb, kb, vb)))
    if shared:          # e.g. the (B,H,S,D) views of a packed qkv projection: read in place
        strides = (st[0], st[1], st[2])
    else:
        qb, kb, vb = (t.contiguous() for t in (qb, kb, vb))
        strides = (H * S * D, S * D, D)
    out = torch.empty((B, S, H, D), dtype=torch.bfloat16, device=q.device)
    attention(qb, kb, vb, B, H, S, D, strides, scale, out, (S * H * D, D, H * D), head_globals=head_globals,
              packed=packed, smooth_k=smooth_k, smooth_v=smooth_v)
    return out.transpose(1, 2)


def attention_packed_qkv(qkv: torch.Tensor, num_heads: int, scale: float, head_globals: bool = False,
                         packed: bool = True) -> torch.Tensor:
    """Packed (B, S, 3*H*D) projection output -> (B, S, H*D) bf16, read in place (no q/k/v copies)."""
    B, S, C3 = qkv.shape
    H = num_heads
    D = C3 // (3 * H)
    x = qkv if qkv.is_contiguous() else qkv.contiguous()
    out = torch.empty((B, S, H * D), dtype=torch.bfloat16, device=qkv.device)
    st = (S * C3, D, C3)
    attention(x, x[..., H * D:], x[..., 2 * H * D:], B, H, S, D, st, scale, out, (S * H * D, D, H * D),
              head_globals=head_globals, packed=packed)
    return out


def ln_cast(x: torch.Tensor, ln_w: torch.Tensor, ln_b: torch.Tensor, eps: float, gs: torch.Tensor | None = None,
            y: torch.Tensor | None = None, gamma: torch.Tensor | None = None, x_out: torch.Tensor | None = None):
    """LayerNorm fused into the NVFP4 cast, optionally after x' = x + y * gamma (written to x_out).

    x, y: (M, K) bf16 contiguous.  Returns (packed (M, K/2), sf_swizzled, gs, x') where x' is x when
    no residual is given.  ``gs`` None -> dynamic global scale of the normalised rows."""
    _need_cuda(x, y, gamma, ln_w, ln_b)
    M, K = x.shape
    dev = x.device
    if y is not None and x_out is None:
        x_out = torch.empty_like(x)
    packed = torch.empty((M, K // 2), dtype=torch.uint8, device=dev)
    sf = torch.empty(sf_swizzled_numel(M, K), dtype=torch.uint8, device=dev)
    gs_in = None if gs is None else gs.reshape(()).to(torch.float32).contiguous()
    gs_out = torch.empty((), dtype=torch.float32, device=dev) if gs_in is None else None
    w = ln_w.to(torch.bfloat16).contiguous()
    b = ln_b.to(torch.bfloat16).contiguous()
    g = None if gamma is None else gamma.to(torch.bfloat16).contiguous()
    # bytes: x (and y, x') in bf16, codes + scales out; the dynamic form reads x twice
    kind = "ln_cast_residual" if y is not None else ("ln_cast_static" if gs_in is not None else "ln_cast_dynamic")
    per = (6 if y is not None else 2) + 0.5 + 1 / 16 + (2 if gs_in is None else 0)
    with _Timed(f"{kind}_{M}x{K}", M * K * per):
        _lib.call("vf4_ln_cast_nvfp4", _ptr(x), _ptr(y), _ptr(g), _ptr(x_out), _ptr(w), _ptr(b), float(eps), M, K,
                  _ptr(gs_in), _ptr(packed), _ptr(sf), _ptr(gs_out), _stream())
    _launched(1 if gs_in is not None else 3)
    return packed, sf, (gs_out if gs_in is None else gs_in), (x if y is None else x_out)


@torch.library.custom_op("vitfp4::patchify", mutates_args=())
def patchify_op(images: torch.Tensor, patch: int, k_pad: int) -> torch.Tensor:
    return patchify(images, patch, k_pad)


@patchify_op.register_fake
def _(images, patch, k_pad):
    B, C, H, W = images.shape
    return images.new_empty((B * (H // patch) * (W // patch), k_pad), dtype=torch.bfloat16)


@torch.library.custom_op("vitfp4::embed_tokens", mutates_args=())
def embed_tokens_op(y: torch.Tensor, cls: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
    return embed_tokens(y, cls, pos)


@embed_tokens_op.register_fake
def _(y, cls, pos):
    B, P, D = y.shape
    return y.new_empty((B, P + 1, D), dtype=torch.bfloat16)


def patchify(images: torch.Tensor, patch: int, k_pad: int) -> torch.Tensor:
    """(B, C, H, W) bf16 images -> (B * H/p * W/p, k_pad) bf16 patch rows in the Conv2d weight's
    (c, i, j) order, zero-padded from C*p*p to k_pad columns (16-byte rows for the GEMM)."""
    _need_cuda(images)
    x = images.contiguous()
    B, C, H, W = x.shape
    out = torch.empty((B * (H // patch) * (W // patch), k_pad), dtype=torch.bfloat16, device=x.device)
    _lib.call("vf4_patchify", _ptr(x), B, C, H, W, patch, k_pad, _ptr(out), _stream())
    _launched()
    return out


def embed_tokens(y: torch.Tensor, cls: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
    """(B, T-1, D) patch projections, (D,) class token, (T, D) position embedding -> (B, T, D)
    = [cls + pos[0]; y + pos[1:]] in bf16 (torch.cat + add in one pass)."""
    _need_cuda(y, cls, pos)
    yb = y.contiguous()
    B, P, D = yb.shape
    c = cls.reshape(D).to(torch.bfloat16).contiguous()
    p = pos.reshape(P + 1, D).to(torch.bfloat16).contiguous()
    out = torch.empty((B, P + 1, D), dtype=torch.bfloat16, device=y.device)
    _lib.call("vf4_embed_tokens", _ptr(yb), _ptr(c), _ptr(p), B, P + 1, D, _ptr(out), _stream())
    _launched()
    return out
