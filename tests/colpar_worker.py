"""Rank body of the column-parallel all-gather test (run by tests/test_gpu_colpar.py
under torch.distributed.run, one process per GPU, NCCL with NVLS off).

Every rank builds the same activations and weights, keeps its N / world output
channels of W, and runs the fused path (m5b_gemm_allgather into every rank's
output through CUDA-IPC peer mappings) and the NCCL baseline (local GEMM +
all_gather_into_tensor).  Both must equal the full single-GPU projection bit
for bit on every rank.  Exit status 0 = all ranks agree.
"""

import os
import sys
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
sys.path[:0] = [str(ROOT), str(ROOT / "m5-max-kernels_b200")]

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402


def main() -> int:
    import m5kernels_b200 as m5
    from m5kernels_b200 import sharding

    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)
    world, rank = dist.get_world_size(), dist.get_rank()
    bad = 0
    for (m, k, n) in ((300, 512, 256 * world), (4096, 1024, 2048 * world)):
        g = torch.Generator(device=dev).manual_seed(11)
        x = torch.randn(m, k, device=dev, generator=g).to(torch.bfloat16)
        w = (0.02 * torch.randn(n, k, device=dev, generator=g)).to(torch.bfloat16)
        aq, sa = m5.quantize(x, "int8")
        wq, sw = m5.quantize(w, "int8")
        full = m5.gemm(aq, wq, "int8", a_scales=sa, b_scales=sw, output_dtype=torch.bfloat16)
        c0, c1 = sharding.shard_columns(n, world, rank)
        out = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device=dev)
        gather = sharding.ColumnParallelGather(out)
        for _ in range(2):  # twice: the second step overwrites a full output
            gather.step(aq, wq[c0:c1].contiguous(), sa, sw[c0:c1].contiguous())
        torch.cuda.synchronize()
        bad += int(not torch.equal(out, full))
        local_y = m5.gemm(aq, wq[c0:c1].contiguous(), "int8", a_scales=sa,
                          b_scales=sw[c0:c1].contiguous(), output_dtype=torch.bfloat16)
        bad += int(not torch.equal(sharding.gather_columns(local_y, world), full))
        gather.barrier()
        gather.close()
    flag = torch.tensor([bad], device=dev)
    dist.all_reduce(flag)
    torch.cuda.synchronize()
    dist.destroy_process_group()
    if rank == 0:
        print(f"colpar ranks={world} mismatches={int(flag.item())}", flush=True)
    return 0 if int(flag.item()) == 0 else 1


if __name__ == "__main__":
    sys.exit(main())
