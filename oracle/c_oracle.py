"""ctypes wrapper of the C restatement (oracle/m5_oracle.c).

TEST INFRASTRUCTURE ONLY: the checker for tests/, ``smoke()`` and the
``cpu_baseline`` leg of bench.py.  Arrays are CPU torch tensors (bf16 / fp16 /
fp32 / int8 / uint8 / int32); results come back as CPU torch tensors.
"""

from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
SRC = HERE / "m5_oracle.c"
BUILD = HERE / "_build"
LIB = BUILD / "libm5oracle.so"

# dtype codes shared with the CUDA library
F32, F16, BF16 = 0, 1, 2
_CODES = {torch.float32: F32, torch.float16: F16, torch.bfloat16: BF16}
NORMS = {None: 0, "none": 0, "rms": 1, "layer": 2}
OUTS = {"int8": 0, "fp8": 1, "f32": 2}
EPI = {"plain": 0, "bias_vec": 1, "bias_table": 2, "gate_vec": 3, "gate_table": 4}

_lib = None


def build(force: bool = False) -> Path:
    """Compile libm5oracle.so with IEEE-exact flags (no contraction, no fast math)."""
    BUILD.mkdir(exist_ok=True)
    if LIB.exists() and not force and LIB.stat().st_mtime >= SRC.stat().st_mtime:
        return LIB
    cmd = ["gcc", "-O2", "-std=c11", "-fPIC", "-shared", "-ffp-contract=off", "-fno-fast-math",
           "-fno-builtin-rintf", str(SRC), "-o", str(LIB), "-lm"]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    return LIB


OMP_SRC = HERE / "m5_cpu_omp.c"
OMP_LIB = BUILD / "libm5cpu_omp.so"
_omp = None


def build_omp(force: bool = False) -> Path:
    """Compile the multi-threaded CPU baseline (OpenMP; SIMD kernels chosen at run time)."""
    BUILD.mkdir(exist_ok=True)
    if OMP_LIB.exists() and not force and OMP_LIB.stat().st_mtime >= OMP_SRC.stat().st_mtime:
        return OMP_LIB
    cmd = ["gcc", "-O3", "-std=c11", "-fPIC", "-shared", "-fopenmp", "-ffp-contract=off",
           "-fno-fast-math", str(OMP_SRC), "-o", str(OMP_LIB), "-lm"]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    return OMP_LIB


def omp_lib() -> ctypes.CDLL:
    global _omp
    if _omp is None:
        _omp = ctypes.CDLL(str(build_omp()))
        P, I64 = ctypes.c_void_p, ctypes.c_int64
        _omp.m5c_quantize_bf16.argtypes = [P, I64, I64, P, P]
        _omp.m5c_quantize_bf16.restype = None
        _omp.m5c_gemm_i8_bf16.argtypes = [P, P, I64, I64, I64, P, P, P]
        _omp.m5c_gemm_i8_bf16.restype = None
        _omp.m5c_threads.restype = ctypes.c_int
        _omp.m5c_simd_level.restype = ctypes.c_int
    return _omp


def omp_projection(x_bf16, wq, w_scales):
    """Multi-threaded CPU online projection: INT8 quantize of bf16 rows, then
    bf16((float(acc) * s_x) * w_scales).  Returns (out bf16, codes, scales)."""
    x = _cpu(x_bf16)
    wq, w_scales = _cpu(wq), _cpu(w_scales)
    m, k = x.shape
    n = wq.shape[0]
    q = torch.empty((m, k), dtype=torch.int8)
    s = torch.empty((m,), dtype=torch.float32)
    out = torch.empty((m, n), dtype=torch.bfloat16)
    o = omp_lib()
    o.m5c_quantize_bf16(_ptr(x), m, k, _ptr(q), _ptr(s))
    o.m5c_gemm_i8_bf16(_ptr(q), _ptr(wq), m, n, k, _ptr(s), _ptr(w_scales), _ptr(out))
    return out, q, s


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        _lib = ctypes.CDLL(str(build()))
        P, I64, I32, F = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float
        _lib.m5o_row_prep.argtypes = [P, I32, P, P, I32, P, P, I32, P, I32, P, I32, P, P, I64, I64,
                                      I32, F, I32, I32, I32, P, P, P, P]
        _lib.m5o_row_prep.restype = None
        _lib.m5o_e4m3_encode.argtypes = [F]
        _lib.m5o_e4m3_encode.restype = ctypes.c_uint8
        _lib.m5o_gemm_i8_acc.argtypes = [P, P, I64, I64, I64, P]
        _lib.m5o_gemm_i8_acc.restype = None
        _lib.m5o_gemm_epilogue_i32.argtypes = [P, I64, I64, P, P, I32, P, P, P, P, P, P, I32]
        _lib.m5o_gemm_epilogue_i32.restype = None
        _lib.m5o_qk_rope_from_acc.argtypes = [P, I64, I64, P, P, P, P, P, I32, F, P]
        _lib.m5o_qk_rope_from_acc.restype = None
        _lib.m5o_rms_quantize.argtypes = [P, I32, P, P, I64, I64, I32, I32, F, P, P]
        _lib.m5o_rms_quantize.restype = None
        _lib.m5o_quantize_mxint8.argtypes = [P, I32, I64, I64, P, P]
        _lib.m5o_quantize_mxint8.restype = None
        _lib.m5o_check_i8_div_free.argtypes = [P, I64, P]
        _lib.m5o_check_i8_div_free.restype = I64
        _lib.m5o_check_i8_div_free_f32.argtypes = [I64, ctypes.c_uint64, P]
        _lib.m5o_check_i8_div_free_f32.restype = I64
        _lib.m5o_check_div_free_quotient.argtypes = [P, I64, F, F, I64, ctypes.c_uint64, P]
        _lib.m5o_check_div_free_quotient.restype = I64
    return _lib


def _ptr(t):
    if t is None:
        return None
    return ctypes.c_void_p(t.data_ptr())


def _cpu(t):
    if t is None:
        return None
    return t.detach().to("cpu").contiguous()


def _code(t, default=F32):
    return default if t is None else _CODES[t.dtype]


def row_prep(x, *, block=0, norm=None, eps=1e-5, round_output=False, out="int8", gamma=None,
             scale=None, shift=None, row_map=None, signs=None, branch=None, gate=None,
             gate_row_map=None):
    """Run the row-preparation restatement; returns dict(q, s) / dict(y) (+ residual)."""
    x = _cpu(x)
    rows, k = x.shape
    args = [_cpu(t) for t in (branch, gate, gamma, scale, shift)]
    branch, gate, gamma, scale, shift = args
    row_map = _cpu(row_map.to(torch.int32)) if row_map is not None else None
    gate_row_map = _cpu(gate_row_map.to(torch.int32)) if gate_row_map is not None else None
    signs = _cpu(signs.to(torch.int8)) if signs is not None else None
    res = {}
    q = s = y = r_out = None
    if out == "f32":
        y = torch.empty((rows, k), dtype=torch.float32)
        res["y"] = y
    else:
        q = torch.empty((rows, k), dtype=torch.int8 if out == "int8" else torch.uint8)
        s = torch.empty((rows,), dtype=torch.float32)
        res["q"], res["s"] = q, s
    if branch is not None:
        r_out = torch.empty_like(x)
        res["residual"] = r_out
    lib().m5o_row_prep(
        _ptr(x), _code(x), _ptr(branch), _ptr(gate), _code(gate), _ptr(gate_row_map),
        _ptr(gamma), _code(gamma), _ptr(scale), _code(scale), _ptr(shift), _code(shift),
        _ptr(row_map), _ptr(signs), rows, k, NORMS[norm], float(eps), int(bool(round_output)),
        int(block), OUTS[out], _ptr(q), _ptr(s), _ptr(y), _ptr(r_out))
    return res


def quantize(x, mode="int8"):
    r = row_prep(x, out=mode)
    return r["q"], r["s"]


def quantize_mxint8(x):
    """MXINT8 restatement: (int8 codes [rows, K], uint8 E8M0 bytes [rows, K/32])."""
    x = _cpu(x)
    rows, k = x.shape
    q = torch.empty((rows, k), dtype=torch.int8)
    e = torch.empty((rows, k // 32), dtype=torch.uint8)
    lib().m5o_quantize_mxint8(_ptr(x), _code(x), rows, k, _ptr(q), _ptr(e))
    return q, e


def rotate(x, block, signs=None):
    return row_prep(x, block=block, signs=signs, out="f32")["y"]


def rms_quantize(x, gamma, signs, block_size=1, *, fold_scale=True, epsilon=1e-5):
    """RMS scale-folding (or direct) INT8 preparation; returns (codes, scales).

    block_size 1 means no rotation, as in the reference's rms_quantize.
    """
    x = _cpu(x)
    rows, k = x.shape
    gamma = _cpu(gamma.to(torch.float32))
    signs = _cpu(signs.to(torch.int8))
    q = torch.empty((rows, k), dtype=torch.int8)
    s = torch.empty((rows,), dtype=torch.float32)
    lib().m5o_rms_quantize(_ptr(x), _code(x), _ptr(gamma), _ptr(signs), rows, k,
                           0 if block_size == 1 else int(block_size), int(bool(fold_scale)),
                           float(epsilon), _ptr(q), _ptr(s))
    return q, s


def e4m3_encode_scalar(v: float) -> int:
    return int(lib().m5o_e4m3_encode(float(v)))


def gemm_i8_acc(a, b):
    """Exact INT32 accumulators of int8 A[M,K] . B[N,K]^T."""
    a, b = _cpu(a), _cpu(b)
    m, k = a.shape
    n = b.shape[0]
    acc = torch.empty((m, n), dtype=torch.int32)
    lib().m5o_gemm_i8_acc(_ptr(a), _ptr(b), m, n, k, _ptr(acc))
    return acc


def gemm_i8_acc_fast(a, b):
    """Exact INT32 accumulators via float64 BLAS (|sum| < 2^53 for K <= 2^37)."""
    a64 = _cpu(a).to(torch.float64)
    b64 = _cpu(b).to(torch.float64)
    return (a64 @ b64.T).to(torch.int32)


def gemm_epilogue(acc, sa=None, sb=None, *, epi="plain", bias=None, bias_row_map=None,
                  residual=None, gate=None, gate_row_map=None, out_dtype=torch.bfloat16):
    """Scale / bias / gate epilogue over exact INT32 accumulators."""
    acc = _cpu(acc).to(torch.int32)
    m, n = acc.shape
    out = torch.empty((m, n), dtype=out_dtype)
    sa, sb, bias = _cpu(sa), _cpu(sb), _cpu(bias)
    residual, gate = _cpu(residual), _cpu(gate)
    bias_row_map = _cpu(bias_row_map.to(torch.int32)) if bias_row_map is not None else None
    gate_row_map = _cpu(gate_row_map.to(torch.int32)) if gate_row_map is not None else None
    lib().m5o_gemm_epilogue_i32(_ptr(acc), m, n, _ptr(sa), _ptr(sb), EPI[epi], _ptr(bias),
                                _ptr(bias_row_map), _ptr(residual), _ptr(gate),
                                _ptr(gate_row_map), _ptr(out), _CODES[out_dtype])
    return out


def qk_rope_from_acc(accf, sa, sb, gamma, cos, sin, rope_half, eps):
    """Q/K RMSNorm + RoPE epilogue; accf is float32 [M, N] (exact INT32 values or BF16 sums)."""
    accf = _cpu(accf).to(torch.float32)
    m, n = accf.shape
    out = torch.empty((n // 128, m, 128), dtype=torch.bfloat16)
    lib().m5o_qk_rope_from_acc(_ptr(accf), m, n, _ptr(_cpu(sa)), _ptr(_cpu(sb)),
                               _ptr(_cpu(gamma)), _ptr(_cpu(cos)), _ptr(_cpu(sin)),
                               int(rope_half), float(eps), _ptr(out))
    return out


__all__ = [
    "build", "build_omp", "omp_projection", "quantize_mxint8", "row_prep", "quantize", "rotate", "gemm_i8_acc", "gemm_i8_acc_fast",
    "gemm_epilogue", "qk_rope_from_acc", "e4m3_encode_scalar", "np",
]
