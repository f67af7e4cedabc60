"""The hot path under CUDA graph capture.

Every entry point launches on the caller's stream and makes no synchronising
call, so a step (online quantize -> W8A8 GEMM, the one-call projection, the
fused prep + Q/K projection) can be captured once and replayed.  Replays must
equal eager calls bit for bit, also after the captured inputs are overwritten
in place (the graph reads the new contents).
"""

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _capture(fn):
    for _ in range(2):
        fn()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = fn()
    return graph, out


def test_quantize_gemm_graph_matches_eager():
    import m5kernels_b200 as m5

    g = torch.Generator().manual_seed(5)
    x = torch.randn(1024, 4096, generator=g).to(torch.bfloat16).to(DEV)
    w = (0.02 * torch.randn(2048, 4096, generator=g)).to(torch.bfloat16).to(DEV)
    wq, ws = m5.quantize(w, "int8")

    def step():
        q, s = m5.quantize(x, "int8")
        return m5.gemm(q, wq, "int8", a_scales=s, b_scales=ws, output_dtype=torch.bfloat16)

    graph, out = _capture(step)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, step())
    x.copy_(torch.randn(1024, 4096, generator=g).to(torch.bfloat16))
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, step())
    del graph


def test_linear_graph_matches_eager():
    import m5kernels_b200 as m5

    g = torch.Generator().manual_seed(6)
    x = torch.randn(512, 2048, generator=g).to(torch.bfloat16).to(DEV)
    w = (0.02 * torch.randn(1024, 2048, generator=g)).to(torch.bfloat16).to(DEV)
    signs = (torch.randint(0, 2, (2048,), generator=g, dtype=torch.int8) * 2 - 1).to(DEV)
    wq, ws = m5.hadamard_quantize(w, 128, signs, "int8")
    step = lambda: m5.linear(x, wq, ws, "int8", block_size=128, signs=signs)  # noqa: E731
    graph, out = _capture(step)
    x.mul_(-0.5)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, step())
    del graph


def test_prep_qk_graph_matches_eager():
    import m5kernels_b200 as m5

    g = torch.Generator().manual_seed(8)
    m, k, n = 600, 1024, 512
    x = torch.randn(m, k, generator=g).to(torch.bfloat16).to(DEV)
    w = (0.03 * torch.randn(n, k, generator=g)).to(torch.bfloat16).to(DEV)
    signs = torch.ones(k, dtype=torch.int8, device=DEV)
    wq, ws = m5.hadamard_quantize(w, 256, signs, "int8")
    gamma = torch.ones(128, dtype=torch.bfloat16, device=DEV)
    cos, sin = m5.rope_tables(m, 64, 10000.0, device=DEV)

    def step():
        q, s = m5.hadamard_quantize(x, 256, signs, "int8")
        return m5.projection_qk_rope(q, wq, gamma, cos, sin, "int8", a_scales=s, b_scales=ws)

    graph, out = _capture(step)
    x.add_(1.0)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, step())
    del graph
