"""Parity at BASELINE's full sizes.

The other GPU tests check every output element at sizes the CPU oracle
finishes quickly.  Here the BASELINE configurations run at full size on the
GPU and are checked on 32 sampled rows against the C restatement (exact INT32
accumulators of those rows through float64 BLAS; every column of a sampled
row), plus whole-tensor properties that hold at any size (the fused Q/K path
equals the staged one bit for bit).
  C2 / C3  FFN-down M4096 K16384 N4096 (plain INT8, and H128 rotation + INT8),
           FFN-down M9914, FFN-up M4096 and M9914 (K4096 N16384), Q M9914
  C3 E4M3  H128 rotation + E4M3 prep and the f8f6f4 FFN-down GEMM, M4096:
           codes and scales bit-exact, output rel-L2 <= 5e-3 vs the float64
           decoded dot (the stated FP8 bar)
  C4       gated LayerNorm + AdaLN + H128 + INT8, M4096 K4096, 2 samples
  C5       H256 + INT8 prep and the Q/K projection, M9914 K4096, 32 heads, R64
  8 ranks  one rank's share of the strong-scaled FFN-down job at 8 GPUs (M512)
           against the C restatement; a 256-row projection at K16384 on the
           split-K schedule against the data-parallel one
"""

import numpy as np
import pytest
import torch

from oracle import c_oracle as co

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(scope="module")
def ops():
    import m5kernels_b200 as m

    return m


def _rows(m, count=32, seed=0):
    g = np.random.default_rng(seed)
    r = np.sort(g.choice(m, size=count - 2, replace=False))
    return np.unique(np.concatenate([[0, m - 1], r]))


def _acc(aq_rows, bq):
    return co.gemm_i8_acc_fast(aq_rows.cpu(), bq.cpu())


@pytest.mark.parametrize("m,k,n,block", [(4096, 16384, 4096, 0), (4096, 16384, 4096, 128),
                                         (9914, 16384, 4096, 0), (4096, 4096, 16384, 0),
                                         (9914, 4096, 16384, 0), (9914, 4096, 4096, 0)])
def test_projection_full_size_sampled_rows(ops, m, k, n, block):
    g = torch.Generator(device=DEV).manual_seed(m + block)
    x = torch.randn(m, k, device=DEV, generator=g)
    cols = torch.randperm(k, device=DEV, generator=g)[: k // 100]
    x[:, cols] *= 50  # BASELINE's outlier variant: 1 % of K channels x50
    x = x.to(torch.bfloat16)
    w = (0.02 * torch.randn(n, k, device=DEV, generator=g)).to(torch.bfloat16)
    signs = torch.ones(k, dtype=torch.int8, device=DEV)
    if block:
        wq, sw = ops.hadamard_quantize(w, block, signs, "int8")
        aq, sa = ops.hadamard_quantize(x, block, signs, "int8")
    else:
        wq, sw = ops.quantize(w, "int8")
        aq, sa = ops.quantize(x, "int8")
    y = ops.gemm(aq, wq, "int8", a_scales=sa, b_scales=sw, output_dtype=torch.bfloat16)
    rows = torch.as_tensor(_rows(m), device=DEV)
    xs = x[rows].cpu()
    o = co.row_prep(xs, block=block, signs=signs.cpu() if block else None)
    assert torch.equal(aq[rows].cpu(), o["q"]) and torch.equal(sa[rows].cpu(), o["s"])
    ow = co.row_prep(w[:64].cpu(), block=block, signs=signs.cpu() if block else None)
    assert torch.equal(wq[:64].cpu(), ow["q"]) and torch.equal(sw[:64].cpu(), ow["s"])
    expect = co.gemm_epilogue(_acc(aq[rows], wq), sa[rows].cpu(), sw.cpu())
    assert torch.equal(y[rows].cpu(), expect)


def test_c4_gated_prep_full_size_sampled_rows(ops):
    m, k, p = 4096, 4096, 2
    g = torch.Generator(device=DEV).manual_seed(4)
    res = torch.randn(m, k, device=DEV, generator=g).to(torch.bfloat16)
    br = torch.randn(m, k, device=DEV, generator=g).to(torch.bfloat16)
    tab = lambda: (0.1 * torch.randn(p, k, device=DEV, generator=g)).to(torch.bfloat16)  # noqa: E731
    gate, scale, shift = tab(), tab(), tab()
    gamma = torch.ones(k, dtype=torch.bfloat16, device=DEV)
    rmap = (torch.arange(m, device=DEV, dtype=torch.int32) // (m // p)).to(torch.int32)
    signs = torch.ones(k, dtype=torch.int8, device=DEV)
    q, s, r2 = ops.fused_gated_residual_norm_hadamard_quantize(
        res, br, gate, gamma, scale, shift, signs, 128, norm="layer", epsilon=1e-6,
        gate_row_map=rmap, row_map=rmap)
    rows = torch.as_tensor(_rows(m, seed=4), device=DEV)
    o = co.row_prep(res[rows].cpu(), block=128, norm="layer", eps=1e-6, round_output=True,
                    gamma=gamma.cpu(), scale=scale.cpu(), shift=shift.cpu(),
                    row_map=rmap[rows].cpu(), signs=signs.cpu(), branch=br[rows].cpu(),
                    gate=gate.cpu(), gate_row_map=rmap[rows].cpu())
    assert torch.equal(r2[rows].cpu(), o["residual"])
    assert torch.equal(q[rows].cpu(), o["q"]) and torch.equal(s[rows].cpu(), o["s"])


def test_c5_qk_full_size(ops):
    m, k, n, half = 9914, 4096, 4096, 64
    g = torch.Generator(device=DEV).manual_seed(5)
    x = torch.randn(m, k, device=DEV, generator=g).to(torch.bfloat16)
    w = (0.02 * torch.randn(n, k, device=DEV, generator=g)).to(torch.bfloat16)
    gamma = (1 + 0.02 * torch.randn(128, device=DEV, generator=g)).to(torch.bfloat16)
    cos, sin = ops.rope_tables(m, half, 10000.0, device=DEV)
    signs = torch.ones(k, dtype=torch.int8, device=DEV)
    wq, sw = ops.hadamard_quantize(w, 256, signs, "int8")
    aq, sa = ops.hadamard_quantize(x, 256, signs, "int8")
    y = ops.projection_qk_rope(aq, wq, gamma, cos, sin, "int8", a_scales=sa, b_scales=sw)
    # whole tensor: fused == staged (bf16 projection, then the standalone post-process)
    proj = ops.gemm(aq, wq, "int8", a_scales=sa, b_scales=sw, output_dtype=torch.bfloat16)
    assert torch.equal(y, ops.qk_norm_rope(proj, gamma, cos, sin))
    # sampled rows: the C restatement on exact accumulators
    rows = torch.as_tensor(_rows(m, seed=5), device=DEV)
    o = co.row_prep(x[rows].cpu(), block=256, signs=signs.cpu())
    assert torch.equal(aq[rows].cpu(), o["q"]) and torch.equal(sa[rows].cpu(), o["s"])
    acc = _acc(aq[rows], wq).float()
    expect = co.qk_rope_from_acc(acc, sa[rows].cpu(), sw.cpu(), gamma.cpu(), cos[rows].cpu(),
                                 sin[rows].cpu(), half, 1e-5)
    assert torch.equal(y[:, rows].cpu(), expect)


def test_c3_e4m3_step_full_size(ops):
    """C3 with E4M3: H128 rotation + per-token E4M3 codes, W rotated offline and
    quantized per channel to E4M3, FP32-accumulating f8f6f4 GEMM to bf16."""
    from oracle import reference_numpy as ref

    m, k, n = 4096, 16384, 4096
    g = torch.Generator(device=DEV).manual_seed(33)
    x = torch.randn(m, k, device=DEV, generator=g)
    cols = torch.randperm(k, device=DEV, generator=g)[: k // 100]
    x[:, cols] *= 50
    x = x.to(torch.bfloat16)
    w = (0.02 * torch.randn(n, k, device=DEV, generator=g)).to(torch.bfloat16)
    signs = torch.ones(k, dtype=torch.int8, device=DEV)
    wq, sw = ops.hadamard_quantize(w, 128, signs, "fp8")
    aq, sa = ops.hadamard_quantize(x, 128, signs, "fp8")
    y = ops.gemm(aq, wq, "fp8", a_scales=sa, b_scales=sw, output_dtype=torch.bfloat16)
    rows = torch.as_tensor(_rows(m, seed=33), device=DEV)
    o = co.row_prep(x[rows].cpu(), block=128, signs=signs.cpu(), out="fp8")
    assert torch.equal(aq[rows].cpu(), o["q"]) and torch.equal(sa[rows].cpu(), o["s"])
    da = ref.dequantize(aq[rows].cpu().numpy(), sa[rows].cpu().numpy(), "fp8").astype(np.float64)
    db = ref.dequantize(wq.cpu().numpy(), sw.cpu().numpy(), "fp8").astype(np.float64)
    rel = ref.metrics(y[rows].float().cpu().numpy(), da @ db.T)["relative_l2"]
    assert rel <= 5e-3, rel


def test_ffn_down_rank_share_8(ops):
    """Rows [0, 512) of the FFN-down job -- one rank's share at 8 GPUs, 32 pair
    tiles for 74 CTA pairs, run as 64 N-halves: codes, scales and the bf16
    output on sampled rows bit-exact vs the C restatement; the bound step,
    the one-call linear and the two-call path agree over the whole tensor."""
    from m5kernels_b200 import _lib

    lib = _lib.lib()
    m, k, n = 512, 16384, 4096
    assert int(lib.m5b_gemm_workspace_bytes(m, n, k, _lib.MODE["int8"])) == 0  # data-parallel
    g = torch.Generator(device=DEV).manual_seed(512)
    x = torch.randn(m, k, device=DEV, generator=g).to(torch.bfloat16)
    w = (0.02 * torch.randn(n, k, device=DEV, generator=g)).to(torch.bfloat16)
    wq, sw = ops.quantize(w, "int8")
    out = torch.empty((m, n), dtype=torch.bfloat16, device=DEV)
    step = ops.OnlineProjection(x, wq, sw, out, "int8")
    step()
    rows = torch.as_tensor(_rows(m, seed=512), device=DEV)
    o = co.row_prep(x[rows].cpu())
    assert torch.equal(step.q[rows].cpu(), o["q"]) and torch.equal(step.s[rows].cpu(), o["s"])
    expect = co.gemm_epilogue(_acc(step.q[rows], wq), step.s[rows].cpu(), sw.cpu())
    assert torch.equal(out[rows].cpu(), expect)
    assert torch.equal(out, _gemm_data_parallel(step.q, wq, step.s, sw))
    assert ops.linear(x, wq, sw).equal(out)


def test_split_k_small_projection_full_k(ops):
    """A projection with very few rows and columns at BASELINE's K (256 x 4096,
    K = 16384: 16 pair tiles) takes the split-K schedule (4 CTA pairs per
    tile): equal to the data-parallel schedule over the whole tensor and to
    the C restatement on sampled rows; the tile counters are zero again after
    two calls."""
    from m5kernels_b200 import _lib

    lib = _lib.lib()
    m, k, n = 256, 16384, 4096
    need = int(lib.m5b_gemm_workspace_bytes(m, n, k, _lib.MODE["int8"]))
    assert need > 0
    g = torch.Generator(device=DEV).manual_seed(256)
    x = torch.randn(m, k, device=DEV, generator=g).to(torch.bfloat16)
    w = (0.02 * torch.randn(n, k, device=DEV, generator=g)).to(torch.bfloat16)
    wq, sw = ops.quantize(w, "int8")
    out = torch.empty((m, n), dtype=torch.bfloat16, device=DEV)
    step = ops.OnlineProjection(x, wq, sw, out, "int8")
    assert step.gemm_ws is not None and step.gemm_ws.numel() == need
    step()
    first = out.clone()
    step()
    torch.cuda.synchronize()
    assert torch.equal(out, first) and _counters_zero(step.gemm_ws)
    assert torch.equal(out, _gemm_data_parallel(step.q, wq, step.s, sw))
    rows = torch.as_tensor(_rows(m, seed=256), device=DEV)
    expect = co.gemm_epilogue(_acc(step.q[rows], wq), step.s[rows].cpu(), sw.cpu())
    assert torch.equal(out[rows].cpu(), expect)


def _counters_zero(ws):
    """The split-K workspace after a call: partial sums may remain, the tile
    counters behind them (two ints per tile and CTA) must all be zero."""
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    part = (sms // 2) * 2 * 128 * 256 * 4
    return int(ws[part:].count_nonzero().item()) == 0


def _gemm_data_parallel(aq, wq, sa, sw):
    """m5b_gemm without a workspace: the data-parallel schedule."""
    from m5kernels_b200 import _lib

    out = torch.empty((aq.shape[0], wq.shape[0]), dtype=torch.bfloat16, device=DEV)
    _lib.check(_lib.lib().m5b_gemm(
        _lib.ptr(aq), _lib.ptr(wq), aq.shape[0], wq.shape[0], aq.shape[1], _lib.MODE["int8"],
        _lib.ptr(sa), _lib.ptr(sw), _lib.ptr(out), _lib.BF16, None, None, 0, None, None, None, 0,
        _lib.stream_handle(out.device)))
    return out
