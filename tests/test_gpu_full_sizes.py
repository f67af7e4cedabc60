"""Parity at BASELINE's full sizes.

The other GPU tests check every output element at sizes the CPU oracle
finishes quickly.  Here the BASELINE configurations run at full size on the
GPU and are checked on 32 sampled rows against the C restatement (exact INT32
accumulators of those rows through float64 BLAS; every column of a sampled
row), plus whole-tensor properties that hold at any size (the fused Q/K path
equals the staged one bit for bit).
  C2 / C3  FFN-down M4096 K16384 N4096 (plain INT8, and H128 rotation + INT8)
  C2 tail  Q projection M9914 K4096 N4096
  C4       gated LayerNorm + AdaLN + H128 + INT8, M4096 K4096, 2 samples
  C5       H256 + INT8 prep and the Q/K projection, M9914 K4096, 32 heads, R64
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
                                         (9914, 4096, 4096, 0)])
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
