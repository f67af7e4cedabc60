"""One-call online projection: quantize([rotate](x)) -> W8A8 / FP8 GEMM.

The reference composes its online stage from two operators
(src/m5kernels/engine.py:180-182: quantize then gemm; hadamard_gemm.py:65-69
with a rotation first).  `linear` does the same through one C-ABI call
(m5b_linear_ex), with the per-token codes and scales in a device workspace
that is allocated once per device and stream and grown on demand, and the
GEMM's split-K workspace beside it.  `OnlineProjection` is the same step
bound to fixed buffers, for loops and CUDA-graph capture.
"""

from __future__ import annotations

import threading

import torch

from . import _lib
from ._lib import check, ptr

_ws_lock = threading.Lock()
_workspaces: dict = {}


def _key(device: torch.device, tag: str):
    return (tag, device.type, device.index, torch.cuda.current_stream(device).cuda_stream)


def workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    """Cached uint8 device buffer of at least nbytes for the codes and scales
    (256-byte aligned by torch), one per device and stream."""
    key = _key(device, "codes")
    with _ws_lock:
        buf = _workspaces.get(key)
        if buf is None or buf.numel() < nbytes:
            buf = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=device)
            _workspaces[key] = buf
        return buf


def gemm_workspace(device: torch.device, nbytes: int):
    """Cached zero-filled split-K workspace of the GEMM (m5b_gemm_ex), one per
    device and stream, or None when nbytes is 0.  It is zeroed once when
    allocated; every GEMM call leaves it zeroed again."""
    if nbytes <= 0:
        return None
    key = _key(device, "gemm")
    with _ws_lock:
        buf = _workspaces.get(key)
        if buf is None or buf.numel() < nbytes:
            buf = torch.zeros(nbytes, dtype=torch.uint8, device=device)
            _workspaces[key] = buf
        return buf


def fp32_workspace(device: torch.device, nbytes: int):
    """Cached scratch of the FP32 GEMM mode (its split operands), one per device
    and stream.  Kept apart from the split-K workspace, which must stay zeroed
    between calls; this one is overwritten by every FP32 GEMM."""
    key = _key(device, "fp32")
    with _ws_lock:
        buf = _workspaces.get(key)
        if buf is None or buf.numel() < nbytes:
            buf = torch.empty(nbytes, dtype=torch.uint8, device=device)
            _workspaces[key] = buf
        return buf


def linear(x, wq, w_scales, mode="int8", *, block_size=0, signs=None,
           output_dtype=torch.bfloat16):
    """y = (acc(quantize(x [D H]), wq) * s_x) * w_scales, one call.

    x: [M, K] bf16 / fp16 / fp32 CUDA tensor; wq: [N, K] codes prepared
    offline (quantize(w) or hadamard_quantize(w, block_size, signs)) in the
    same mode; w_scales: fp32 [N].  K % 16 == 0 (fp8: K % 128 == 0).
    """
    if mode not in ("int8", "fp8"):
        raise NotImplementedError("the online projection supports int8 and fp8 (E4M3)")
    if x.dim() != 2 or wq.dim() != 2 or 0 in x.shape or 0 in wq.shape:
        raise ValueError("x and wq must be nonempty matrices")
    m, k = x.shape
    n, kb = wq.shape
    if k != kb:
        raise ValueError("K mismatch")
    if x.dtype not in (torch.float16, torch.bfloat16, torch.float32):
        raise ValueError("input dtype must be float16, bfloat16 or float32")
    if wq.dtype != (torch.int8 if mode == "int8" else torch.uint8):
        raise ValueError("weight codes must match the declared mode")
    if tuple(w_scales.shape) != (n,) or w_scales.dtype != torch.float32:
        raise ValueError("w_scales must be a float32 vector of length N")
    if block_size and (signs is None or tuple(signs.shape) != (k,) or signs.dtype != torch.int8):
        raise ValueError("signs must be an int8 vector of length K containing only +/-1")
    if output_dtype not in (torch.bfloat16, torch.float16, torch.float32):
        raise NotImplementedError("output dtype must be bfloat16, float16 or float32")
    dev = _lib.require_cuda(x, wq, w_scales, signs)
    x, wq, w_scales = x.contiguous(), wq.contiguous(), w_scales.contiguous()
    lib = _lib.lib()
    need = int(lib.m5b_linear_workspace_bytes(m, k))
    ws = workspace(dev, need)
    gws = gemm_workspace(dev, int(lib.m5b_gemm_workspace_bytes(m, n, k, _lib.MODE[mode])))
    out = torch.empty((m, n), dtype=output_dtype, device=dev)
    check(lib.m5b_linear_ex(ptr(x), _lib.DTYPE_CODE[x.dtype], m, k, int(block_size or 0),
                            ptr(signs) if block_size else None, ptr(wq), ptr(w_scales), n,
                            _lib.MODE[mode], ptr(out), _lib.DTYPE_CODE[output_dtype], ptr(ws),
                            ws.numel(), ptr(gws), 0 if gws is None else gws.numel(),
                            _lib.stream_handle(dev)))
    return out


class OnlineProjection:
    """The online projection step bound to fixed buffers.

    quantize([rotate](x)) into codes / scales owned by this object, then the
    W8A8 / FP8 GEMM with the (acc * s_x) * w_scales epilogue into `out` --
    the kernels and results of `linear`, launched as two C-ABI calls
    (m5b_quantize or m5b_hadamard_quantize, then m5b_gemm_ex) with every
    pointer bound once and nothing allocated per call, so a step can be
    replayed in a tight loop or captured in a CUDA graph.  The inputs are read
    at call time: refill `x` in place between calls.  Launches go to the
    current stream of x's device.
    """

    def __init__(self, x, wq, w_scales, out, mode="int8", *, block_size=0, signs=None):
        if mode not in ("int8", "fp8"):
            raise NotImplementedError("the online projection supports int8 and fp8 (E4M3)")
        if x.dim() != 2 or wq.dim() != 2 or out.dim() != 2:
            raise ValueError("x, wq and out must be matrices")
        m, k = x.shape
        n = wq.shape[0]
        if wq.shape[1] != k:
            raise ValueError("K mismatch")
        if tuple(out.shape) != (m, n) or out.dtype not in (torch.bfloat16, torch.float16,
                                                           torch.float32):
            raise ValueError("out must be a bf16 / fp16 / fp32 [M, N] tensor")
        if not (x.is_contiguous() and wq.is_contiguous() and out.is_contiguous()
                and w_scales.is_contiguous()):
            raise ValueError("x, wq, w_scales and out must be contiguous")
        if tuple(w_scales.shape) != (n,) or w_scales.dtype != torch.float32:
            raise ValueError("w_scales must be a float32 vector of length N")
        if block_size and (signs is None or tuple(signs.shape) != (k,)
                           or signs.dtype != torch.int8):
            raise ValueError("signs must be an int8 vector of length K containing only +/-1")
        self.device = _lib.require_cuda(x, wq, w_scales, out, signs)
        self.x, self.wq, self.w_scales, self.out = x, wq, w_scales, out
        self.signs = signs if block_size else None
        code_dtype = torch.int8 if mode == "int8" else torch.uint8
        self.q = torch.empty((m, k), dtype=code_dtype, device=self.device)
        self.s = torch.empty((m,), dtype=torch.float32, device=self.device)
        self._lib = _lib.lib()
        need = int(self._lib.m5b_gemm_workspace_bytes(m, n, k, _lib.MODE[mode]))
        self.gemm_ws = torch.zeros(need, dtype=torch.uint8, device=self.device) if need else None
        xd, md = _lib.DTYPE_CODE[x.dtype], _lib.MODE[mode]
        if block_size:
            self._qfn = self._lib.m5b_hadamard_quantize
            self._qargs = (ptr(x), xd, m, k, int(block_size), ptr(signs), md, ptr(self.q),
                           ptr(self.s))
        else:
            self._qfn = self._lib.m5b_quantize
            self._qargs = (ptr(x), xd, m, k, md, ptr(self.q), ptr(self.s))
        self._gargs = (ptr(self.q), ptr(wq), m, n, k, md, ptr(self.s), ptr(w_scales), ptr(out),
                       _lib.DTYPE_CODE[out.dtype], None, None, 0, None, None, None, 0,
                       ptr(self.gemm_ws), 0 if self.gemm_ws is None else self.gemm_ws.numel())
        self.shape = (m, n, k)
        self.mode = mode

    def quantize(self):
        check(self._qfn(*self._qargs, _lib.stream_handle(self.device)))

    def gemm(self):
        check(self._lib.m5b_gemm_ex(*self._gargs, _lib.stream_handle(self.device)))

    def __call__(self):
        self.quantize()
        self.gemm()
        return self.out
