"""m5b_linear_noalloc — the online projection for callers that cannot allocate.

Hosts that have committed all device memory to their own pool, plugin hosts
that forbid extensions from allocating, and hot paths that cannot take
cudaMalloc's device synchronisation use this entry point: it keeps its codes
and scales in a fixed device array inside the library instead of a
caller-provided workspace.  These tests call it through the C ABI and require
its output to equal m5b_linear's (the workspace entry point) bit for bit, on
two calls in a row with different shapes (the shared array keeps the previous
call's contents), and check that sizes beyond its fixed limit are refused.

This file is named to be collected last, so a run that stops at its first
failure has already run every other test; it also passes on its own.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _call_noalloc(lib, x, wq, ws, mode_code, block, signs, out_dtype):
    from m5kernels_b200 import _lib

    m, k = x.shape
    n = wq.shape[0]
    out = torch.empty((m, n), dtype=out_dtype, device=x.device)
    rc = lib.m5b_linear_noalloc(
        ctypes.c_void_p(x.data_ptr()), _lib.DTYPE_CODE[x.dtype], m, k, block,
        ctypes.c_void_p(signs.data_ptr()) if signs is not None else None,
        ctypes.c_void_p(wq.data_ptr()), ctypes.c_void_p(ws.data_ptr()), n, mode_code,
        ctypes.c_void_p(out.data_ptr()), _lib.DTYPE_CODE[out_dtype],
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    _lib.check(rc)
    return out


def test_noalloc_matches_workspace_entry_point_on_two_calls():
    import m5kernels_b200 as m5
    from m5kernels_b200 import _lib

    lib = _lib.lib()
    g = torch.Generator().manual_seed(2024)
    cases = [
        dict(m=512, k=2048, n=1024, block=0, mode="int8"),
        dict(m=300, k=4096, n=520, block=128, mode="int8"),
    ]
    for c in cases:  # two calls in a row, different shapes and rotation
        x = torch.randn(c["m"], c["k"], generator=g).to(torch.bfloat16).to(DEV)
        w = (0.02 * torch.randn(c["n"], c["k"], generator=g)).to(torch.bfloat16).to(DEV)
        signs = None
        if c["block"]:
            signs = (torch.randint(0, 2, (c["k"],), generator=g, dtype=torch.int8) * 2 - 1).to(DEV)
            wq, ws = m5.hadamard_quantize(w, c["block"], signs, c["mode"])
        else:
            wq, ws = m5.quantize(w, c["mode"])
        expect = m5.linear(x, wq, ws, c["mode"], block_size=c["block"], signs=signs)
        got = _call_noalloc(lib, x, wq, ws, _lib.MODE[c["mode"]], c["block"], signs,
                            torch.bfloat16)
        torch.cuda.synchronize()
        assert torch.equal(got, expect), c


def test_noalloc_refuses_sizes_beyond_its_scratch():
    from m5kernels_b200 import _lib

    lib = _lib.lib()
    x = torch.empty(8, 16, dtype=torch.bfloat16, device=DEV)
    wq = torch.empty(8, 16, dtype=torch.int8, device=DEV)
    ws = torch.ones(8, device=DEV)
    out = torch.empty(8, 8, dtype=torch.bfloat16, device=DEV)
    # m * k beyond the 67,108,864-code array: refused on the host, nothing launched
    rc = lib.m5b_linear_noalloc(ctypes.c_void_p(x.data_ptr()), _lib.BF16, 16384, 8192, 0, None,
                                ctypes.c_void_p(wq.data_ptr()), ctypes.c_void_p(ws.data_ptr()), 8,
                                _lib.MODE["int8"], ctypes.c_void_p(out.data_ptr()), _lib.BF16,
                                None)
    assert rc == _lib.EINVAL
    assert b"67108864" in lib.m5b_last_error()
    rc = lib.m5b_linear_noalloc(ctypes.c_void_p(x.data_ptr()), _lib.BF16, 20000, 16, 0, None,
                                ctypes.c_void_p(wq.data_ptr()), ctypes.c_void_p(ws.data_ptr()), 8,
                                _lib.MODE["int8"], ctypes.c_void_p(out.data_ptr()), _lib.BF16,
                                None)
    assert rc == _lib.EINVAL and b"16384 rows" in lib.m5b_last_error()
    # a k so large that m * k would overflow int64: refused, not wrapped around
    rc = lib.m5b_linear_noalloc(ctypes.c_void_p(x.data_ptr()), _lib.BF16, 8, 1 << 61, 0, None,
                                ctypes.c_void_p(wq.data_ptr()), ctypes.c_void_p(ws.data_ptr()), 8,
                                _lib.MODE["int8"], ctypes.c_void_p(out.data_ptr()), _lib.BF16,
                                None)
    assert rc == _lib.EINVAL and b"67108864" in lib.m5b_last_error()
