"""The C-ABI library loads here (no GPU needed) and exports every declared symbol.

No compute call is made: these tests only check the boundary itself and that
the product path has no CPU fallback.
"""

import ctypes
import re
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "m5b200.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"M5B_API\s+[\w\s\*]+?\b(m5b_\w+)\s*\(", text)))


def test_header_declares_the_operator_contracts():
    names = declared_symbols()
    for required in ("m5b_quantize", "m5b_rotate", "m5b_hadamard_quantize",
                     "m5b_fused_norm_hadamard_quantize",
                     "m5b_fused_gated_residual_norm_hadamard_quantize", "m5b_gemm",
                     "m5b_projection_qk_rope", "m5b_last_error", "m5b_device_status",
                     "m5b_unfused_norm", "m5b_gated_residual_add", "m5b_qk_norm_rope",
                     "m5b_projection_qkv_rope", "m5b_gemm_allgather", "m5b_ipc_export",
                     "m5b_ipc_import", "m5b_ipc_release"):
        assert required in names


def test_library_exports_every_declared_symbol():
    from m5kernels_b200 import _lib

    lib = _lib.lib()
    for name in declared_symbols():
        assert isinstance(getattr(lib, name), ctypes._CFuncPtr), name
    assert set(declared_symbols()) <= set(_lib.exported_symbols()) | {"m5b_version"}
    assert lib.m5b_version() >= 100
    assert lib.m5b_last_error() == b""


def test_status_codes_match_header():
    from m5kernels_b200 import _lib

    text = HEADER.read_text()
    for name, value in (("M5B_OK", _lib.OK), ("M5B_EINVAL", _lib.EINVAL),
                        ("M5B_EUNSUPPORTED", _lib.EUNSUPPORTED), ("M5B_ECUDA", _lib.ECUDA),
                        ("M5B_BF16", _lib.BF16), ("M5B_I32", _lib.I32)):
        assert re.search(rf"#define {name} {value}\b", text), name


def test_contract_errors_come_back_through_the_abi_without_a_gpu():
    """Size checks run on the host: bad arguments fail before any CUDA call."""
    from m5kernels_b200 import _lib

    lib = _lib.lib()
    rc = lib.m5b_quantize(None, _lib.BF16, 0, 16, 0, None, None, None)
    assert rc == _lib.EINVAL and b"nonempty" in lib.m5b_last_error()
    rc = lib.m5b_rotate(ctypes.c_void_p(16), _lib.BF16, 4, 96, 64, None, ctypes.c_void_p(16), None)
    assert rc == _lib.EUNSUPPORTED and b"divisible" in lib.m5b_last_error()
    rc = lib.m5b_gemm(ctypes.c_void_p(16), ctypes.c_void_p(16), 4, 4, 96, 1, None, None, None, 2,
                      None, None, 0, None, None, None, 0, None)
    assert rc == _lib.EUNSUPPORTED and b"FP8" in lib.m5b_last_error()
    with pytest.raises(NotImplementedError, match="FP8"):
        _lib.check(rc)
    # staged comparators
    rc = lib.m5b_qk_norm_rope(ctypes.c_void_p(16), 4, 200, ctypes.c_void_p(16), ctypes.c_void_p(16),
                              ctypes.c_void_p(16), 64, 1e-5, ctypes.c_void_p(16), None)
    assert rc == _lib.EINVAL and b"128-wide heads" in lib.m5b_last_error()
    rc = lib.m5b_gated_residual_add(ctypes.c_void_p(16), ctypes.c_void_p(16), _lib.BF16, 0, 64,
                                    ctypes.c_void_p(16), _lib.BF16, None, 0, ctypes.c_void_p(16),
                                    None)
    assert rc == _lib.EINVAL and b"nonempty" in lib.m5b_last_error()
    rc = lib.m5b_unfused_norm(ctypes.c_void_p(16), _lib.BF16, 4, 64, ctypes.c_void_p(16), _lib.F32,
                              ctypes.c_void_p(16), _lib.F32, ctypes.c_void_p(16), _lib.F32, None, 0,
                              3, 1e-5, 1, ctypes.c_void_p(16), None)
    assert rc == _lib.EINVAL and b"norm must be" in lib.m5b_last_error()
    rc = lib.m5b_projection_qkv_rope(ctypes.c_void_p(16), ctypes.c_void_p(16), 4, 0, 128, 0,
                                     None, None, None, None, None, None, 48, 1e-5, None, None,
                                     None, None)
    assert rc == _lib.EINVAL and b"heads" in lib.m5b_last_error()


def test_gemm_schedule_is_validated_on_the_host():
    from m5kernels_b200 import _lib

    lib = _lib.lib()
    for bad in ((1, 0), (-2, 0), (5, 0), (-1, -1)):
        assert lib.m5b_gemm_set_schedule(*bad) == _lib.EINVAL
    assert lib.m5b_gemm_set_schedule(2, 4) == _lib.OK
    assert lib.m5b_gemm_set_schedule(-1, 0) == _lib.OK


def test_fp32_gemm_workspace_contract_without_a_gpu():
    """The FP32 mode's workspace (the operands' TF32 parts) is sized on the host,
    and a call without it fails before touching the device."""
    from m5kernels_b200 import _lib

    lib = _lib.lib()
    fp32 = _lib.MODE["fp32"]
    # [m, 3 K4] and [n, 3 K4] fp32 parts, each rounded to 256 bytes: K4 = 8 -> 96
    # bytes a row, 384 -> 512 and 288 -> 512
    assert lib.m5b_gemm_workspace_bytes(4, 3, 5, fp32) == 1024
    # K = 3000: two chunks of 1500 columns -> [1000, 2, 3, 1500] parts per operand, and the
    # chunks' fp32 running sum [1000, 1000]
    assert lib.m5b_gemm_workspace_bytes(1000, 1000, 3000, fp32) == 2 * 1000 * 9000 * 4 + 4 * 10**6
    fake = 1 << 20  # aligned, never dereferenced: the call fails first
    rc = lib.m5b_gemm(fake, fake, 4, 3, 8, fp32, None, None, fake, _lib.F32, None, None, 0,
                      None, None, None, 0, None)
    assert rc == _lib.EINVAL and b"workspace" in lib.m5b_last_error()


def test_operators_refuse_cpu_tensors():
    import m5kernels_b200 as m
    from m5kernels_b200._lib import ExtensionMissing

    with pytest.raises(ExtensionMissing):
        m.quantize(torch.ones(4, 64), "int8")
    with pytest.raises(ExtensionMissing):
        m.rotate(torch.ones(4, 64), 32, torch.ones(64, dtype=torch.int8))
    with pytest.raises(ExtensionMissing):
        m.gated_residual_add(torch.ones(4, 64), torch.ones(4, 64), torch.ones(64))
    with pytest.raises(ExtensionMissing):
        m.unfused_norm(torch.ones(4, 64), torch.ones(64), torch.ones(64), torch.ones(64))
    with pytest.raises(ExtensionMissing):
        m.qk_norm_rope(torch.ones(4, 128, dtype=torch.bfloat16),
                       torch.ones(128, dtype=torch.bfloat16),
                       torch.ones(4, 64, dtype=torch.bfloat16), torch.ones(4, 64, dtype=torch.bfloat16))


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    from m5kernels_b200 import _lib

    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.setattr(_lib, "LIB_PATH", tmp_path / "libm5b200.so")
    with pytest.raises(_lib.ExtensionMissing, match="not built"):
        _lib.lib()


def test_python_contract_validation_matches_reference_messages():
    import m5kernels_b200 as m

    with pytest.raises(ValueError, match="divisible by 32"):
        m.quantize(torch.ones(2, 48), "mxint8")
    with pytest.raises(ValueError, match="nonempty"):
        m.quantize(torch.ones(0, 64), "int8")
    with pytest.raises(ValueError, match="power of two"):
        m.rotate(torch.ones(2, 96), 48, torch.ones(96, dtype=torch.int8))
    with pytest.raises(NotImplementedError, match="divisible"):
        m.rotate(torch.ones(2, 96), 64, torch.ones(96, dtype=torch.int8))
    a = torch.ones(2, 96, dtype=torch.uint8)
    with pytest.raises(NotImplementedError, match="stride"):
        m.gemm(a, a, "fp8", a_scales=torch.ones(2), b_scales=torch.ones(2))
    with pytest.raises(ValueError, match="norm"):
        m.fused_norm_hadamard_quantize(torch.ones(2, 64), torch.ones(64), torch.ones(64),
                                       torch.ones(64), torch.ones(64, dtype=torch.int8), 32,
                                       norm="batch")
    with pytest.raises(ValueError, match="128-wide"):
        m.projection_qk_rope(torch.ones(2, 64, dtype=torch.int8), torch.ones(100, 64, dtype=torch.int8),
                             torch.ones(128, dtype=torch.bfloat16), torch.ones(2, 4, dtype=torch.bfloat16),
                             torch.ones(2, 4, dtype=torch.bfloat16), a_scales=torch.ones(2),
                             b_scales=torch.ones(100))
