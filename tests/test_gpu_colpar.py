"""Column-parallel projection with the all-gather fused into the GEMM epilogue.

BASELINE's Q/K configuration adds a column-parallel FFN-up variant whose bf16
output is all-gathered; m5b_gemm_allgather writes each output tile into this
GPU's output and into every peer rank's output.  On one GPU the "peer"
outputs are other local buffers (the epilogue's peer stores are the same
instructions); with two or more GPUs the ranks run under
torch.distributed.run with NCCL and CUDA-IPC peer mappings.  Bar: bit-exact
against the single-GPU projection, columns outside the shard untouched.
"""

import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"
ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def ops():
    import m5kernels_b200 as m

    return m


@pytest.mark.parametrize("mode", ["int8", "bf16"])
@pytest.mark.parametrize("m,k,n,n_total,col,peers", [(300, 512, 256, 1024, 512, 2),
                                                      (4096, 1024, 2048, 8192, 2048, 3),
                                                      (129, 256, 96, 96, 0, 1),
                                                      (1000, 384, 512, 4096, 3584, 7)])
def test_allgather_epilogue_single_gpu(ops, mode, m, k, n, n_total, col, peers):
    g = torch.Generator().manual_seed(3)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16).to(DEV)
    w = (0.05 * torch.randn(n, k, generator=g)).to(torch.bfloat16).to(DEV)
    if mode == "int8":
        a, sa = ops.quantize(x, "int8")
        b, sb = ops.quantize(w, "int8")
        ref = ops.gemm(a, b, "int8", a_scales=sa, b_scales=sb, output_dtype=torch.bfloat16)
    else:
        a, b, sa, sb = x, w, None, None
        ref = ops.gemm(a, b, "bf16", output_dtype=torch.bfloat16)
    sentinel = -3.0
    outs = [torch.full((m, n_total), sentinel, dtype=torch.bfloat16, device=DEV)
            for _ in range(peers + 1)]
    ops.gemm_allgather(a, b, outs[0], col, outs[1:], mode, a_scales=sa, b_scales=sb)
    for o in outs:
        assert torch.equal(o[:, col:col + n], ref)
        rest = torch.cat([o[:, :col], o[:, col + n:]], dim=1)
        assert bool((rest == sentinel).all())


def test_allgather_contract(ops):
    a = torch.zeros(64, 128, dtype=torch.int8, device=DEV)
    b = torch.zeros(48, 128, dtype=torch.int8, device=DEV)
    s = torch.ones(64, device=DEV)
    out = torch.zeros(64, 96, dtype=torch.bfloat16, device=DEV)
    with pytest.raises(NotImplementedError, match="multiples of 32"):
        ops.gemm_allgather(a, b, out, 0, (), "int8", a_scales=s, b_scales=s[:48])
    with pytest.raises(NotImplementedError, match="at most 7"):
        ops.gemm_allgather(a, b[:32], out, 0, [out] * 8, "int8", a_scales=s, b_scales=s[:32])


def _free_port():
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_allgather_two_ranks_nccl():
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", "--nproc-per-node", "2", "--master-addr", "127.0.0.1",
           "--master-port", str(_free_port()), str(ROOT / "tests" / "colpar_worker.py")]
    proc = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert proc.returncode == 0, proc.stdout[-2000:] + proc.stderr[-4000:]
    assert "mismatches=0" in proc.stdout
