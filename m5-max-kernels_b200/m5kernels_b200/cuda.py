"""quantize / gemm on B200 tensor cores: the `cuda-b200` twin of m5kernels.metal.

Operator contracts follow src/m5kernels/metal.py (reference): the same
argument names and meanings, ValueError for contract violations and
NotImplementedError for unsupported shapes or semantics.  Inputs are never
mutated and outputs are freshly allocated torch CUDA tensors.  The `tile`
argument is accepted for signature compatibility and validated; the B200
kernels choose their own tiles (128 x 256 tcgen05 tiles, 128 x 128 for
narrow outputs).
"""

from __future__ import annotations

import contextlib

import torch

from . import _lib
from ._lib import check, ptr

FLOAT_DTYPES = (torch.float16, torch.bfloat16, torch.float32)


def _validate_tile(tile):
    if not isinstance(tile, (tuple, list)) or len(tile) != 4:
        raise ValueError("tile must contain TM, TN, SIMD groups and M swizzle")


@contextlib.contextmanager
def gemm_schedule(split_k: int = -1, group_m: int = 0):
    """GEMM schedule for the calls made inside the block from this thread.

    The B200 counterpart of the reference's Metal `tile` (what `m5bench tune`
    sweeps, src/m5kernels/cli.py:66-151): split_k -1 = the library's rule,
    0 = data-parallel, 2 = two CTA pairs per 256 x 256 tile in one 4-CTA
    cluster (partial sums through shared memory), 3..4 = CTA pairs per tile
    over equal K ranges through the workspace (INT8 GEMMs, where every unit
    fits on the GPU at once);
    group_m 0 = the library's raster, else M-blocks per raster group.  Results
    are identical under every schedule; only the time changes.
    """
    lib = _lib.lib()
    check(lib.m5b_gemm_set_schedule(int(split_k), int(group_m)))
    try:
        yield
    finally:
        check(lib.m5b_gemm_set_schedule(-1, 0))


def quantize(x: torch.Tensor, mode: str, tag: str = "packed"):
    """Per-row symmetric quantization -> (codes, fp32 scales).

    int8: scale = amax/127, codes = clip(rint(x/scale), +-127) (int8).
    fp8:  scale = amax/448, codes = E4M3 bits (uint8), RNE, saturating.
    All-zero rows use scale 1.
    mxint8: 32-element blocks along each row; returns int8 codes [rows, K] and
    uint8 E8M0 exponent bytes [rows, K/32]: e = floor(log2(block peak)) - 6
    (clipped to +-127, 0 for a zero block), codes = clip(rint(x / 2^e), +-127),
    byte = e + 127.  Mirrors src/m5kernels/metal.py:27-44.
    """
    del tag
    if mode == "mxint8":
        if x.dim() != 2 or 0 in x.shape:
            raise ValueError("input must have nonempty shape [rows, K]")
        if x.shape[1] % 32:
            raise ValueError("MXINT8 requires K divisible by 32")
        if x.dtype not in FLOAT_DTYPES:
            raise ValueError("input dtype must be float16, bfloat16 or float32")
        dev = _lib.require_cuda(x)
        x = x.contiguous()
        rows, k = x.shape
        q = torch.empty((rows, k), dtype=torch.int8, device=dev)
        e = torch.empty((rows, k // 32), dtype=torch.uint8, device=dev)
        check(_lib.lib().m5b_quantize_mxint8(ptr(x), _lib.DTYPE_CODE[x.dtype], rows, k, ptr(q),
                                             ptr(e), _lib.stream_handle(dev)))
        return q, e
    if mode not in ("int8", "fp8"):
        raise ValueError(f"unknown quantization mode {mode!r}")
    if x.dim() != 2 or 0 in x.shape:
        raise ValueError("input must have nonempty shape [rows, K]")
    if x.dtype not in FLOAT_DTYPES:
        raise ValueError("input dtype must be float16, bfloat16 or float32")
    dev = _lib.require_cuda(x)
    x = x.contiguous()
    rows, k = x.shape
    q = torch.empty((rows, k), dtype=torch.int8 if mode == "int8" else torch.uint8, device=dev)
    s = torch.empty((rows,), dtype=torch.float32, device=dev)
    check(_lib.lib().m5b_quantize(ptr(x), _lib.DTYPE_CODE[x.dtype], rows, k, _lib.MODE[mode],
                                  ptr(q), ptr(s), _lib.stream_handle(dev)))
    return q, s


def gemm(a, b, mode="bf16", tile=(64, 64, 4, 1), a_scales=None, b_scales=None,
         output_dtype=None, bias=None, bias_row_map=None, residual=None, gate=None,
         gate_row_map=None):
    """A[M,K] @ B[N,K].T with INT32 (int8) or FP32 accumulation and a fused epilogue.

    mode "fp32" (fp32 operands) runs three TF32 tensor-core products of the
    operands' TF32 parts (A_hi B_hi + A_hi B_lo + A_lo B_hi): FP32 accuracy
    (relative error ~1e-6, the reference's bar is 1e-4 relative L2).

    Quantized modes: out = (float(acc) * a_scales[m]) * b_scales[n].
    INT8 optionally adds an FP32 bias [N] or a bias table [P,N] selected by
    int32 bias_row_map[M].  INT8/BF16 optionally fuse the gated residual
    out = R + bf16(branch) * gate with BF16 residual [M,N] and gate [N] or
    [P,N] + gate_row_map.  Mirrors src/m5kernels/metal.py:158-269; output
    dtype defaults to float32 like the reference.  output_dtype=torch.int32
    (INT8, no scales) returns the raw INT32 accumulators.
    """
    _validate_tile(tile)
    if a.dim() != 2 or b.dim() != 2:
        raise ValueError("A and B must be matrices")
    m, k = a.shape
    n, kb = b.shape
    if k != kb:
        raise ValueError("K mismatch")
    if mode not in _lib.MODE:
        if mode == "mxint8":
            raise NotImplementedError(f"{mode} GEMM is not part of the cuda-b200 backend")
        raise ValueError(f"unknown GEMM mode {mode!r}")
    if mode == "fp8" and k % 128:
        raise NotImplementedError(
            "FP8 requires K/row stride divisible by 128; padding is not implicit")
    if mode == "int8" and k > 133144:
        raise NotImplementedError("INT32 worst-case overflow bound exceeded")
    elem = {"int8": 1, "fp8": 1, "bf16": 2, "fp16": 2, "fp32": 4}[mode]
    if mode != "fp32" and (k * elem) % 16:  # (fp32 operands are re-laid out by the split pass)
        # TMA reads K-major rows whose stride must be a multiple of 16 bytes;
        # the reference keeps padding explicit (metal.py:186-190), so does this.
        raise NotImplementedError(
            f"K*{elem} bytes per row must be a multiple of 16 for TMA; padding is not implicit")
    expected = {"int8": (torch.int8,), "fp8": (torch.uint8,), "bf16": (torch.bfloat16,),
                "fp16": (torch.float16,), "fp32": (torch.float32,)}[mode]
    if a.dtype not in expected or b.dtype not in expected:
        raise ValueError("operand dtypes must match the declared mode")
    out_dtype = output_dtype or torch.float32
    gated = residual is not None or gate is not None or gate_row_map is not None
    if gated:
        if residual is None or gate is None:
            raise ValueError("gated GEMM requires both residual and gate")
        if mode not in ("int8", "bf16"):
            raise NotImplementedError("gated GEMM supports INT8 and BF16 only")
        if output_dtype is None or output_dtype != torch.bfloat16:
            raise NotImplementedError("gated GEMM requires explicit BF16 output_dtype")
        if bias is not None or bias_row_map is not None:
            raise NotImplementedError("combining GEMM bias and gated residual is unsupported")
        if tuple(residual.shape) != (m, n) or residual.dtype != torch.bfloat16:
            raise ValueError("residual must have BF16 dtype and shape [M,N]")
        if gate.dtype != torch.bfloat16:
            raise ValueError("gate must have BF16 dtype")
        if gate_row_map is None:
            if tuple(gate.shape) != (n,):
                raise ValueError("gate must have shape [N] without gate_row_map")
        else:
            if gate.dim() != 2 or 0 in gate.shape or gate.shape[1] != n:
                raise ValueError("mapped gate must have nonempty shape [P,N]")
            if tuple(gate_row_map.shape) != (m,) or gate_row_map.dtype != torch.int32:
                raise ValueError("gate_row_map must be an int32 vector of length M")
        if mode == "int8" and (
            a_scales is None or b_scales is None or tuple(a_scales.shape) != (m,)
            or tuple(b_scales.shape) != (n,) or a_scales.dtype != torch.float32
            or b_scales.dtype != torch.float32
        ):
            raise ValueError("gated INT8 GEMM requires float32 scales with shapes [M] and [N]")
    if bias is None:
        if bias_row_map is not None:
            raise ValueError("bias_row_map requires a bias table")
    else:
        if mode != "int8":
            raise NotImplementedError("optional GEMM bias currently supports INT8 only")
        if bias.dtype != torch.float32:
            raise ValueError("bias must have float32 dtype")
        if bias_row_map is None:
            if tuple(bias.shape) != (n,):
                raise ValueError("bias must have shape [N] without bias_row_map")
        else:
            if bias.dim() != 2 or 0 in bias.shape or bias.shape[1] != n:
                raise ValueError("mapped bias must have nonempty shape [P,N]")
            if tuple(bias_row_map.shape) != (m,) or bias_row_map.dtype != torch.int32:
                raise ValueError("bias_row_map must be an int32 vector of length M")
    quant = mode in ("int8", "fp8")
    if out_dtype == torch.int32:
        if mode != "int8" or a_scales is not None or b_scales is not None or gated or bias is not None:
            raise ValueError("int32 output returns raw INT8 accumulators without scales")
    elif quant:
        if a_scales is None or b_scales is None:
            raise ValueError("scales required")
        if (tuple(a_scales.shape) != (m,) or tuple(b_scales.shape) != (n,)
                or a_scales.dtype != torch.float32 or b_scales.dtype != torch.float32):
            raise ValueError("scales must be float32 vectors of length M and N")
    if out_dtype not in (torch.bfloat16, torch.float16, torch.float32, torch.int32):
        raise NotImplementedError("output dtype must be bfloat16, float16 or float32")
    dev = _lib.require_cuda(a, b, a_scales, b_scales, bias, bias_row_map, residual, gate,
                            gate_row_map)
    if m == 0 or n == 0 or k == 0:
        raise ValueError("A and B must be nonempty matrices")
    a = a.contiguous()
    b = b.contiguous()
    args = [t.contiguous() if t is not None else None
            for t in (a_scales, b_scales, bias, bias_row_map, residual, gate, gate_row_map)]
    a_scales, b_scales, bias, bias_row_map, residual, gate, gate_row_map = args
    out = torch.empty((m, n), dtype=out_dtype, device=dev)
    lib = _lib.lib()
    # split-K workspace (zero-filled once, left zeroed by every call) for the
    # shapes that take the split schedule; None keeps the data-parallel one
    from .linear import fp32_workspace, gemm_workspace

    nbytes = int(lib.m5b_gemm_workspace_bytes(m, n, k, _lib.MODE[mode]))
    # (fp32: scratch for the operands' TF32 parts, separate from split-K's)
    ws = fp32_workspace(dev, nbytes) if mode == "fp32" else gemm_workspace(dev, nbytes)
    check(lib.m5b_gemm_ex(
        ptr(a), ptr(b), m, n, k, _lib.MODE[mode], ptr(a_scales), ptr(b_scales), ptr(out),
        _lib.DTYPE_CODE[out_dtype], ptr(bias), ptr(bias_row_map),
        bias.shape[0] if (bias is not None and bias.dim() == 2) else 0,
        ptr(residual), ptr(gate), ptr(gate_row_map),
        gate.shape[0] if (gate is not None and gate.dim() == 2) else 0,
        ptr(ws), 0 if ws is None else ws.numel(), _lib.stream_handle(dev)))
    return out


def gemm_allgather(a, b, out, col_offset, peer_outs=(), mode="int8", *, a_scales=None,
                   b_scales=None):
    """Store this shard's bf16 projection a @ b^T into columns [col_offset,
    col_offset + N) of `out` [M, N_total] and of every tensor in `peer_outs`
    (other ranks' outputs mapped into this process, or local buffers).

    The column-parallel all-gather fused into the GEMM epilogue
    (m5b_gemm_allgather); sharding.ColumnParallelGather runs it across ranks.
    """
    import ctypes

    if mode not in ("int8", "fp8", "bf16"):
        raise NotImplementedError("the all-gather GEMM supports int8, fp8 and bf16 operands")
    if out.dim() != 2 or out.dtype != torch.bfloat16 or not out.is_contiguous():
        raise ValueError("out must be a contiguous bf16 [M, N_total] tensor")
    peers = list(peer_outs)
    if len(peers) > 7:
        raise NotImplementedError("at most 7 peer outputs (8 ranks)")
    dev = _lib.require_cuda(a, b, out, a_scales, b_scales, *peers)
    a, b = a.contiguous(), b.contiguous()
    arr = (ctypes.c_void_p * 7)(*[p.data_ptr() for p in peers])
    check(_lib.lib().m5b_gemm_allgather(
        ptr(a), ptr(b), a.shape[0], b.shape[0], a.shape[1], _lib.MODE[mode], ptr(a_scales),
        ptr(b_scales), ptr(out), out.shape[1], int(col_offset), arr, len(peers),
        _lib.stream_handle(dev)))
    return out
