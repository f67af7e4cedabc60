"""One-call online projection: quantize([rotate](x)) -> W8A8 / FP8 GEMM.

The reference composes its online stage from two operators
(src/m5kernels/engine.py:180-182: quantize then gemm; hadamard_gemm.py:65-69
with a rotation first).  `linear` does the same through one C-ABI call
(m5b_linear), with the per-token codes and scales in a device workspace that
is allocated once per device and grown on demand.
"""

from __future__ import annotations

import threading

import torch

from . import _lib
from ._lib import check, ptr

_ws_lock = threading.Lock()
_workspaces: dict = {}


def workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    """Cached uint8 device buffer of at least nbytes (256-byte aligned by torch)."""
    key = (device.type, device.index)
    with _ws_lock:
        buf = _workspaces.get(key)
        if buf is None or buf.numel() < nbytes:
            buf = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=device)
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
    out = torch.empty((m, n), dtype=output_dtype, device=dev)
    check(lib.m5b_linear(ptr(x), _lib.DTYPE_CODE[x.dtype], m, k, int(block_size or 0),
                         ptr(signs) if block_size else None, ptr(wq), ptr(w_scales), n,
                         _lib.MODE[mode], ptr(out), _lib.DTYPE_CODE[output_dtype], ptr(ws),
                         ws.numel(), _lib.stream_handle(dev)))
    return out
