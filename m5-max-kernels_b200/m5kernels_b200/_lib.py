"""Loader for libm5b200.so, the C-ABI CUDA library (include/m5b200.h).

There is no fallback: if the library is missing, or no CUDA device is
visible, every operator raises.  Tensors cross the boundary as raw device
pointers; the stream is torch's current stream on the tensors' device.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libm5b200.so"

# status codes and enums (must match include/m5b200.h)
OK, EINVAL, EUNSUPPORTED, ECUDA = 0, 1, 2, 3
F32, F16, BF16, I8, U8, I32 = 0, 1, 2, 3, 4, 5
MODE = {"int8": 0, "fp8": 1, "bf16": 2, "fp16": 3, "fp32": 4}
NORM = {"rms": 1, "layer": 2}
DTYPE_CODE = {torch.float32: F32, torch.float16: F16, torch.bfloat16: BF16, torch.int8: I8,
              torch.uint8: U8, torch.int32: I32}

_lock = threading.Lock()
_lib = None

P, I64, I, F = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float
_SIGNATURES = {
    "m5b_version": ([], I),
    "m5b_last_error": ([], ctypes.c_char_p),
    "m5b_device_status": ([ctypes.POINTER(ctypes.c_uint), I], I),
    "m5b_quantize": ([P, I, I64, I64, I, P, P, P], I),
    "m5b_quantize_mxint8": ([P, I, I64, I64, P, P, P], I),
    "m5b_rotate": ([P, I, I64, I64, I, P, P, P], I),
    "m5b_hadamard_quantize": ([P, I, I64, I64, I, P, I, P, P, P], I),
    "m5b_fused_norm_hadamard_quantize": (
        [P, I, I64, I64, P, I, P, I, P, I, P, I64, P, I, I, F, I, I, P, P, P], I),
    "m5b_fused_gated_residual_norm_hadamard_quantize": (
        [P, P, I, I64, I64, P, I, P, I64, P, I, P, I, P, I, P, I64, P, I, I, F, I, I, P, P, P,
         P], I),
    "m5b_rms_quantize": ([P, I, I64, I64, P, P, I, I, F, P, P, P], I),
    "m5b_unfused_norm": ([P, I, I64, I64, P, I, P, I, P, I, P, I64, I, F, I, P, P], I),
    "m5b_gated_residual_add": ([P, P, I, I64, I64, P, I, P, I64, P, P], I),
    "m5b_qk_norm_rope": ([P, I64, I64, P, P, P, I, F, P, P], I),
    "m5b_gemm": ([P, P, I64, I64, I64, I, P, P, P, I, P, P, I64, P, P, P, I64, P], I),
    "m5b_gemm_workspace_bytes": ([I64, I64, I64, I], I64),
    "m5b_gemm_ex": ([P, P, I64, I64, I64, I, P, P, P, I, P, P, I64, P, P, P, I64, P, I64, P], I),
    "m5b_projection_qk_rope": ([P, P, I64, I64, I64, I, P, P, P, P, P, I, F, P, P], I),
    "m5b_projection_qk_rope_ex": ([P, P, I64, I64, I64, I, P, P, P, P, P, I, F, P, P, I64, P], I),
    "m5b_projection_qkv_rope": ([P, P, I64, I64, I64, I, P, P, P, P, P, P, I, F, P, P, P, P], I),
    "m5b_gemm_allgather": ([P, P, I64, I64, I64, I, P, P, P, I64, I64, P, I, P], I),
    "m5b_ipc_export": ([P, P, ctypes.POINTER(ctypes.c_int64)], I),
    "m5b_ipc_import": ([P, I64, ctypes.POINTER(ctypes.c_void_p)], I),
    "m5b_ipc_release": ([P, I64], I),
    "m5b_linear_workspace_bytes": ([I64, I64], I64),
    "m5b_linear": ([P, I, I64, I64, I, P, P, P, I64, I, P, I, P, I64, P], I),
    "m5b_linear_ex": ([P, I, I64, I64, I, P, P, P, I64, I, P, I, P, I64, P, I64, P], I),
    "m5b_linear_noalloc": ([P, I, I64, I64, I, P, P, P, I64, I, P, I, P], I),
    "m5b_gemm_set_schedule": ([I, I], I),
}


class ExtensionMissing(RuntimeError):
    """The CUDA extension is not built or cannot run here; nothing falls back."""


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise ExtensionMissing(
                    f"{LIB_PATH} is not built; run `python m5-max-kernels_b200/build.py` "
                    "(or __graft_entry__.build()) first")
            handle = ctypes.CDLL(str(LIB_PATH))
            for name, (args, res) in _SIGNATURES.items():
                fn = getattr(handle, name)
                fn.argtypes = args
                fn.restype = res
            _lib = handle
    return _lib


def exported_symbols() -> list[str]:
    return list(_SIGNATURES)


def check(rc: int) -> None:
    """Map a C-ABI status to the reference's exception types."""
    if rc == OK:
        return
    msg = lib().m5b_last_error().decode(errors="replace")
    if rc == EINVAL:
        raise ValueError(msg)
    if rc == EUNSUPPORTED:
        raise NotImplementedError(msg)
    raise RuntimeError(f"CUDA error in libm5b200: {msg}")


def ptr(t) -> ctypes.c_void_p | None:
    if t is None:
        return None
    return ctypes.c_void_p(t.data_ptr())


def require_cuda(*tensors) -> torch.device:
    """All tensors must live on one CUDA device; returns it."""
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not isinstance(t, torch.Tensor):
            raise ValueError("operands must be torch tensors")
        if t.device.type != "cuda":
            raise ExtensionMissing(
                "m5kernels_b200 runs on CUDA devices only; got a tensor on " + str(t.device))
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError("all operands must be on the same CUDA device")
    if dev is None:
        raise ValueError("no tensor operands")
    return dev


def stream_handle(device: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def device_status(clear: bool = False) -> int:
    """Device status word (bounded-wait failures); synchronizes the device."""
    value = ctypes.c_uint(0)
    check(lib().m5b_device_status(ctypes.byref(value), 1 if clear else 0))
    return int(value.value)
