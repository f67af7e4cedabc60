"""Headline benchmark: FFN-down W8A8 projection with online activation quantization.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

Workload (FFN-down at M=4096): A bf16 [4096, 16384] ~N(0,1),
W bf16 [4096, 16384] ~N(0, 0.02) quantized offline per output channel
(symmetric INT8, amax/127).  One step = online per-token INT8 quantization of
A + the tcgen05 W8A8 GEMM with the fused (acc * sa) * sw -> bf16 epilogue.
Tokens are sharded: with N GPUs each rank owns a contiguous block of the
4096 rows (4096 / N), weights are replicated, no collective -- the same total
work at every N (strong scaling).  Metric: 2*M*N*K / step time in TOPS for
the whole job, the step time being the slowest rank's.

Each rank rotates independent operand sets (their total footprint is well
above the 126 MB L2), so no step finds its operands in L2.  The W warm-up
steps run eagerly; the K timed steps are captured once as a CUDA graph (two
kernel launches and three timing events per step) and replayed, bracketed by
a barrier and a device synchronize on both sides; times are CUDA events on
the launching stream, max over ranks.  `e2e` repeats the step through the
public C ABI (m5b_linear_ex) from pinned host memory: H2D of this rank's
activations, the two kernels, D2H of the bf16 output, every step.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for _p in (ROOT, ROOT / "m5-max-kernels_b200"):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

M, K, N = 4096, 16384, 4096  # global rows of the job, reduction width, output channels
L2_BYTES = 126 * 2**20
METRIC = "W8A8 proj TOPS incl. online quant @M=4096 (% INT8 peak); prep HBM GB/s"
WORKLOAD = "ffn_down_w8a8_online_quant_M4096_K16384_N4096"

# DRAM traffic (dram__bytes_read.sum + dram__bytes_write.sum) of one launch of
# the GEMM kernel, from ncu captures of this workload's per-rank shapes
# (rows per rank -> bytes).  Recorded constants, not measured by this script.
GEMM_TRAFFIC_BYTES = {4096: 252967680 + 24065024, 512: 75607552 + 3584512}
GEMM_TRAFFIC_SOURCE = ("ncu capture (1 launch, dram__bytes_read.sum + dram__bytes_write.sum) of "
                       "gemm_tc_kernel<i8,256,pair> on the per-rank shape; recorded constant")


def _peaks():
    """Roofline denominators: MEASURED_PEAKS.json if present, else the fallback."""
    p = ROOT / "MEASURED_PEAKS.json"
    try:
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16": float(d["bf16_tflops"]),
                "bf16_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])),
                "source": "measured"}
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16": 1590.0, "bf16_sustained": 1400.0, "source": "fallback"}


class ClockSampler:
    """SM clock / throttle-reason sampling while the timed regions run.

    Polls NVML about every millisecond from a thread (the same counters as the
    `nvidia-smi --query-gpu=clocks.sm,clocks.max.sm,clocks_event_reasons.*`
    line, but fast enough for a timed region of a few milliseconds).  Samples
    are kept only while `active` is set, i.e. inside the timed regions.
    """

    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20,
               "sw_power_cap": 0x4}

    def __init__(self, index: int):
        self.index = index
        self.samples = []
        self._stop = threading.Event()
        self.active = threading.Event()
        self.thread = None
        self.nvml = None
        self.max_mhz = None

    def __enter__(self):
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nvml = pynvml
            self.handle = pynvml.nvmlDeviceGetHandleByIndex(self.index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM)
            self.thread = threading.Thread(target=self._run, daemon=True)
            self.thread.start()
        except Exception:
            self.nvml = None
        return self

    def _run(self):
        nv = self.nvml
        while not self._stop.is_set():
            if self.active.is_set():
                try:
                    sm = nv.nvmlDeviceGetClockInfo(self.handle, nv.NVML_CLOCK_SM)
                    reasons = nv.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
                    if self.active.is_set():
                        self.samples.append((sm, reasons))
                except Exception:
                    pass
            time.sleep(0.0005)

    def __exit__(self, *exc):
        self._stop.set()
        if self.thread is not None:
            self.thread.join(timeout=5)
        if self.nvml is not None:
            try:
                self.nvml.nvmlShutdown()
            except Exception:
                pass

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        seen = set()
        for _, bits in self.samples:
            for name, mask in self.REASONS.items():
                if bits & mask:
                    seen.add(name)
        return {"sm_mhz": statistics.median(s for s, _ in self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(seen), "samples": len(self.samples),
                "window": "device-timed and e2e regions"}


def _dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def _rows(share: int, rank: int) -> tuple[int, int]:
    """This rank's contiguous [start, stop) block of the job's M rows."""
    base, extra = divmod(M, share)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def _operand_sets(m_local: int) -> int:
    """Operand sets a rank rotates through: at least 3, and together at least
    three times the L2 size, so a step's operands were evicted by the others'."""
    per_set = m_local * K * 2 + N * K + m_local * K + m_local * N * 2
    return max(3, min(8, math.ceil(3 * L2_BYTES / per_set)))


def _config(world: int) -> dict:
    m_local = _rows(world, 0)[1] - _rows(world, 0)[0]
    sets = _operand_sets(m_local)
    return {"workload": WORKLOAD, "global_M": M, "M_per_gpu": m_local, "K": K, "N": N,
            "parallelism": f"token-sharded x{world} (weights replicated, no collective)",
            "l2": f"inputs larger than L2: {sets} rotating operand sets per rank"}


def _thread_env() -> dict:
    env = {k: os.environ.get(k, "unset") for k in ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS",
                                                   "MKL_NUM_THREADS")}
    try:
        from threadpoolctl import threadpool_info

        env["blas"] = [{"api": d.get("internal_api"), "threads": d.get("num_threads")}
                       for d in threadpool_info() if d.get("user_api") == "blas"]
    except Exception:
        pass
    return env


def _bf16_rows(rng, rows):
    """rows x K activations ~N(0,1) rounded to bf16 values, as float32."""
    import numpy as np

    a = rng.standard_normal((rows, K), dtype=np.float32)
    u = a.view(np.uint32)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


def cpu_reference(steps: int, warmup: int, budget_s: float = 150.0):
    """The reference's CPU path of the headline workload, timed on the host cores.

    Per step: per-token INT8 quantization of the activation rows with the
    restated numerics.quantize_reference (float32 NumPy, numerics.py:29-46),
    the decoded float64 BLAS product against the INT8 weight
    (src/m5kernels/engine.py:173-175 -- the reference's own CPU GEMM), the
    scale epilogue and BF16 rounding.  Every timed step runs all M=4096 rows
    of the job unless `steps` of them would exceed `budget_s`, in which case
    each step runs a stated number of rows; the W warm-up steps run 64 rows.
    """
    import numpy as np

    from oracle import reference_numpy as ref

    rng = np.random.default_rng(0)
    w = (rng.standard_normal((N, K), dtype=np.float32) * 0.02)
    wq, ws = ref.quantize_reference(w, "int8")
    wd = wq.astype(np.float64) * ws.astype(np.float64)[:, None]
    del w

    def one(rows):
        a = _bf16_rows(rng, rows)
        t0 = time.perf_counter()
        q, s = ref.quantize_reference(a, "int8")
        y = (q.astype(np.float64) * s.astype(np.float64)[:, None]) @ wd.T
        ref.bf16_round_reference(y)
        return time.perf_counter() - t0

    # every host thread this process may run on, whatever OMP_NUM_THREADS the
    # launcher set (torchrun sets 1 for multi-rank jobs)
    ncores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    try:
        from threadpoolctl import threadpool_limits

        pool = threadpool_limits(limits=ncores, user_api="blas")
    except Exception:
        pool = None
    try:
        for _ in range(max(warmup, 1)):
            t64 = one(64)
        est_full = t64 * M / 64
        steps = max(steps, 1)
        rows = M if steps * est_full <= budget_s else max(64, int(M * budget_s / (steps * est_full)))
        times = [one(rows) for _ in range(steps)]
        threads = _thread_env()
    finally:
        if pool is not None:
            pool.unregister()
    per = statistics.median(times)
    tops = 2.0 * rows * N * K / per / 1e12
    return {"value": tops, "unit": "TOPS", "cores": ncores, "kind": "port",
            "sample": (f"{rows} of {M} activation rows per timed step, {steps} timed steps "
                       f"(median), {max(warmup, 1)} warm-up steps of 64 rows; FFN-down K={K}, "
                       f"N={N}; NumPy float32 quantize_reference + float64 BLAS decoded GEMM"),
            "rows_per_step": rows, "seconds_per_step": per, "steps_timed": steps,
            "threads": threads}


def cpu_omp_baseline(target_s: float = 8.0):
    """The repository's multi-threaded C restatement (OpenMP, INT32 accumulation;
    oracle/m5_cpu_omp.c) of the same step on the host cores: quantization of
    bf16 rows and the W8A8 GEMM with the bf16 epilogue."""
    import torch

    from oracle import c_oracle as co

    g = torch.Generator().manual_seed(0)
    wq = torch.randint(-127, 128, (N, K), dtype=torch.int8, generator=g)
    ws = torch.rand(N, generator=g) * 1e-3
    lib = co.omp_lib()
    t0 = time.perf_counter()
    co.omp_projection(torch.randn(64, K, generator=g).to(torch.bfloat16), wq, ws)
    t64 = time.perf_counter() - t0
    rows = int(min(M, max(64, 64 * (target_s / 3) / max(t64, 1e-4))) // 64 * 64)
    x = torch.randn(rows, K, generator=g).to(torch.bfloat16)
    times = []
    for _ in range(3):
        t0 = time.perf_counter()
        co.omp_projection(x, wq, ws)
        times.append(time.perf_counter() - t0)
    per = statistics.median(times)
    simd = {2: "AVX-512 VNNI", 1: "AVX2", 0: "plain C"}[int(lib.m5c_simd_level())]
    return {"value": 2.0 * rows * N * K / per / 1e12, "unit": "TOPS",
            "cores": int(lib.m5c_threads()), "kind": "port",
            "sample": (f"{rows} of {M} rows per step, median of 3 steps; C restatement "
                       f"(OpenMP, {simd} INT8 dot products, INT32 accumulation)"),
            "threads": _thread_env()}


def run_secondary(args, world, rank, local):
    """Other BASELINE configurations (not the headline line): time one workload.

    prep_c3: online H128 rotation + per-token INT8 of the FFN-down activations
             (M=4096, K=16384; outlier distribution), HBM bytes 3K+4 per row; also
             the whole C3 step (prep + FFN-down GEMM, W rotated offline) in INT8
             and in E4M3 (per-token / per-channel scales, FP32 accumulation).
    prep_c4: gated residual + LayerNorm (eps 1e-6, no affine) + AdaLN (2 samples
             of 2048 tokens) + H128 + INT8 (M=4096, K=4096), bytes 7K+4 per row;
             also the whole C4 step with the Q projection (N=4096, W rotated
             offline).
    qk_c5:   H256 + INT8 online prep and the Q/K projection with RMSNorm + RoPE
             (M=9914, K=4096, 32 heads x 128, theta 10000, R=64), token-sharded
             over the ranks (strong scaling, no collective).
    rms_q:   RMS scale-folding prep (random gamma, H256, INT8) + W8A8 GEMM on the
             reference's rms-quant Q shape (M=4096, K=5376, N=7168).

    Each step runs on one of SETS independent input sets (their footprint is
    above L2), and the SETS steps are captured once as a CUDA graph that is
    replayed: the times are device times of the kernels, without the Python
    launch path between them.  For qk_c5 the prep and the Q/K projection are
    also timed on their own, and the staged comparators (prep_c4:
    gated_residual_add then the fused prep; qk_c5: bf16 projection then
    qk_norm_rope) give the fusion gain = staged time / fused time.
    """
    import torch

    import m5kernels_b200 as m5

    from m5kernels_b200 import sharding

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta

        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))
    g = torch.Generator(device=dev).manual_seed(7 + rank)
    stream = torch.cuda.current_stream(dev)
    peaks = _peaks()
    # qk_c5 is token-sharded: rank r owns a contiguous block of the 9914 rows
    # (weights replicated, no collective); the other workloads run whole per rank.
    r0, r1 = sharding.shard_rows(9914, world, rank)
    m_c5 = r1 - r0

    def make_set():
        """One input set: (step function, {part name: function})."""
        if args.workload == "prep_c3":
            m, k, n = 4096, 16384, 4096
            x = torch.randn(m, k, device=dev, generator=g)
            cols = torch.randperm(k, device=dev, generator=g)[: k // 100]
            x[:, cols] *= 50
            x = x.to(torch.bfloat16)
            signs = torch.ones(k, dtype=torch.int8, device=dev)
            w = (0.02 * torch.randn(n, k, device=dev, generator=g)).to(torch.bfloat16)
            # W rotated offline and quantized per output channel, INT8 and E4M3
            wq8, ws8 = m5.hadamard_quantize(w, 128, signs, "int8")
            wqf, wsf = m5.hadamard_quantize(w, 128, signs, "fp8")
            del w

            def step(mode, wq, ws):
                def run():
                    q, s = m5.hadamard_quantize(x, 128, signs, mode)
                    return m5.gemm(q, wq, mode, a_scales=s, b_scales=ws,
                                   output_dtype=torch.bfloat16)
                return run

            return (lambda: m5.hadamard_quantize(x, 128, signs, "int8")), {  # noqa: E731
                "step_int8": step("int8", wq8, ws8), "step_fp8": step("fp8", wqf, wsf),
                "prep_fp8": lambda: m5.hadamard_quantize(x, 128, signs, "fp8")}  # noqa: E731
        if args.workload == "prep_c4":
            m, k, p = 4096, 4096, 2
            res = torch.randn(m, k, device=dev, generator=g).to(torch.bfloat16)
            br = torch.randn(m, k, device=dev, generator=g).to(torch.bfloat16)
            tab = lambda: (0.1 * torch.randn(p, k, device=dev, generator=g)).to(torch.bfloat16)  # noqa: E731
            gate, scale, shift = tab(), tab(), tab()
            gamma = torch.ones(k, dtype=torch.bfloat16, device=dev)
            rmap = (torch.arange(m, device=dev, dtype=torch.int32) // (m // p)).to(torch.int32)
            signs = torch.ones(k, dtype=torch.int8, device=dev)

            def staged():  # the two-launch comparator: R' update, then the fused prep
                upd = m5.gated_residual_add(res, br, gate, gate_row_map=rmap)
                return m5.fused_norm_hadamard_quantize(upd, gamma, scale, shift, signs, 128,
                                                       norm="layer", epsilon=1e-6, row_map=rmap)

            w = (0.02 * torch.randn(k, k, device=dev, generator=g)).to(torch.bfloat16)
            wq, ws = m5.hadamard_quantize(w, 128, signs, "int8")  # offline, untimed
            del w
            q0, s0, _ = m5.fused_gated_residual_norm_hadamard_quantize(
                res, br, gate, gamma, scale, shift, signs, 128, norm="layer", epsilon=1e-6,
                gate_row_map=rmap, row_map=rmap)

            def full_step():  # BASELINE C4: the fused prep, then the Q projection
                q, s, _ = m5.fused_gated_residual_norm_hadamard_quantize(
                    res, br, gate, gamma, scale, shift, signs, 128, norm="layer", epsilon=1e-6,
                    gate_row_map=rmap, row_map=rmap)
                return m5.gemm(q, wq, "int8", a_scales=s, b_scales=ws,
                               output_dtype=torch.bfloat16)

            return (lambda: m5.fused_gated_residual_norm_hadamard_quantize(  # noqa: E731
                res, br, gate, gamma, scale, shift, signs, 128, norm="layer", epsilon=1e-6,
                gate_row_map=rmap, row_map=rmap)), {
                    "staged": staged, "prep_plus_q_gemm": full_step,
                    "q_gemm": lambda: m5.gemm(q0, wq, "int8", a_scales=s0, b_scales=ws,  # noqa: E731
                                              output_dtype=torch.bfloat16)}
        if args.workload == "rms_q":
            m, k, n = 4096, 5376, 7168
            x = torch.randn(m, k, device=dev, generator=g).to(torch.bfloat16)
            w = torch.randn(n, k, device=dev, generator=g).to(torch.bfloat16)
            gamma = (1 + 0.2 * torch.randn(k, device=dev, generator=g)).float()
            signs = (2 * torch.randint(0, 2, (k,), device=dev, generator=g) - 1).to(torch.int8)
            wq, ws = m5.hadamard_quantize(w, 256, signs, "int8")
            q0, s0 = m5.rms_quantize(x, gamma, signs, 256, fold_scale=True)

            def rms_step():
                q, s = m5.rms_quantize(x, gamma, signs, 256, fold_scale=True)
                return m5.gemm(q, wq, "int8", a_scales=s, b_scales=ws,
                               output_dtype=torch.bfloat16)

            return rms_step, {
                "prep": lambda: m5.rms_quantize(x, gamma, signs, 256, fold_scale=True),  # noqa: E731
                "gemm": lambda: m5.gemm(q0, wq, "int8", a_scales=s0, b_scales=ws,  # noqa: E731
                                        output_dtype=torch.bfloat16),
            }
        m, k, n = m_c5, 4096, 4096  # qk_c5: this rank's rows of M = 9914
        x = torch.randn(m, k, device=dev, generator=g).to(torch.bfloat16)
        w = (0.02 * torch.randn(n, k, device=dev, generator=g)).to(torch.bfloat16)
        signs = torch.ones(k, dtype=torch.int8, device=dev)
        wq, ws = m5.hadamard_quantize(w, 256, signs, "int8")
        gamma = (1 + 0.02 * torch.randn(128, device=dev, generator=g)).to(torch.bfloat16)
        cos, sin = m5.rope_tables(m, 64, 10000.0, device=dev)
        q0, s0 = m5.hadamard_quantize(x, 256, signs, "int8")

        def step():
            q, s = m5.hadamard_quantize(x, 256, signs, "int8")
            return m5.projection_qk_rope(q, wq, gamma, cos, sin, "int8", a_scales=s, b_scales=ws)

        return step, {
            "prep": lambda: m5.hadamard_quantize(x, 256, signs, "int8"),  # noqa: E731
            "qk_gemm": lambda: m5.projection_qk_rope(  # noqa: E731
                q0, wq, gamma, cos, sin, "int8", a_scales=s0, b_scales=ws),
            # staged comparator: bf16 projection stored, then the standalone post-process
            "qk_staged": lambda: m5.qk_norm_rope(  # noqa: E731
                m5.gemm(q0, wq, "int8", a_scales=s0, b_scales=ws, output_dtype=torch.bfloat16),
                gamma, cos, sin),
        }

    SETS = 2
    sets = [make_set() for _ in range(SETS)]
    if args.workload == "prep_c3":
        nbytes, unit, kernel = 4096 * (3 * 16384 + 4), "GB/s", "lean_kernel<bf16,128,int8,plain>"
    elif args.workload == "prep_c4":
        nbytes, unit, kernel = 4096 * (7 * 4096 + 4), "GB/s", "rows16_kernel<bf16,128,int8,norm_gated>"
    elif args.workload == "rms_q":
        nbytes, unit = 2.0 * 4096 * 7168 * 5376, "TOPS"
        kernel = "rows16_kernel<bf16,256,int8,rms> (fold) + gemm_tc_kernel<i8,256,plain,pair>"
    else:
        nbytes, unit = 2.0 * m_c5 * 4096 * 4096, "TOPS"
        kernel = "rows16_kernel<bf16,256,int8,plain> + gemm_tc_kernel<i8,256,qk,pair>"

    def graph_ms(fns):
        for _ in range(args.warmup):
            for f in fns:
                f()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for f in fns:
                f()
        graph.replay()
        torch.cuda.synchronize()
        replays = max(1, args.steps // len(fns))
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(replays):
            graph.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        del graph
        return e0.elapsed_time(e1) / (replays * len(fns))

    if world > 1:
        dist.barrier()
    ms = sharding.max_over_ranks(graph_ms([st for st, _ in sets]), device=dev)
    part_ms = {name: sharding.max_over_ranks(graph_ms([parts[name] for _, parts in sets]),
                                             device=dev)
               for name in sets[0][1]}
    if args.workload == "qk_c5":  # whole job: every rank's rows over the slowest rank
        nbytes = 2.0 * 9914 * 4096 * 4096
    if unit == "GB/s":
        value = nbytes / (ms * 1e-3) / 1e9
        frac = value / peaks["hbm_gbs"]
    else:
        value = nbytes / (ms * 1e-3) / 1e12
        frac = value / (2.0 * peaks["bf16"])
    line = {"workload": args.workload, "kernel": kernel, "ms": ms, "value": value, "unit": unit,
            "frac_of_measured_peak": frac, "steps": args.steps, "n_gpus": world,
            "timing": f"CUDA graph replay, {SETS} input sets rotating; max over ranks"}
    if args.workload == "qk_c5":
        line.update(scaling="strong", rows_per_rank=[sharding.shard_rows(9914, world, r)[1]
                                                     - sharding.shard_rows(9914, world, r)[0]
                                                     for r in range(world)])
        if world > 1:
            frac = value / (2.0 * peaks["bf16"] * world)
            line["frac_of_measured_peak"] = frac
    if part_ms:
        line["parts_ms"] = part_ms
        if "qk_gemm" in part_ms:
            line["qk_gemm_tops"] = nbytes / (part_ms["qk_gemm"] * 1e-3) / 1e12
            line["qk_fusion_gain"] = part_ms["qk_staged"] / part_ms["qk_gemm"]
        if "staged" in part_ms:
            line["fusion_gain"] = part_ms["staged"] / ms
        if "step_int8" in part_ms:  # C3 whole step: H128 prep + FFN-down GEMM, INT8 and E4M3
            c3_ops = 2.0 * 4096 * 4096 * 16384
            line["step_int8_tops"] = c3_ops / (part_ms["step_int8"] * 1e-3) / 1e12
            line["step_fp8_tops"] = c3_ops / (part_ms["step_fp8"] * 1e-3) / 1e12
            line["prep_fp8_gbs"] = nbytes / (part_ms["prep_fp8"] * 1e-3) / 1e9
        if "prep_plus_q_gemm" in part_ms:  # C4 step: prep + Q projection (M=K=N=4096)
            q_ops = 2.0 * 4096 ** 3
            line["step_ms"] = part_ms["prep_plus_q_gemm"]
            line["step_tops"] = q_ops / (part_ms["prep_plus_q_gemm"] * 1e-3) / 1e12
            line["q_gemm_tops"] = q_ops / (part_ms["q_gemm"] * 1e-3) / 1e12
        if args.workload == "rms_q":
            prep_bytes = 4096 * (3 * 5376 + 4)
            line["prep_gbs"] = prep_bytes / (part_ms["prep"] * 1e-3) / 1e9
            line["prep_frac_of_measured_hbm"] = line["prep_gbs"] / peaks["hbm_gbs"]
            line["gemm_tops"] = nbytes / (part_ms["gemm"] * 1e-3) / 1e12
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def run_colpar(args, world, rank, local):
    """Column-parallel FFN-up (BASELINE's C5 variant): M=4096, K=4096, N=16384.

    Each rank holds N / world output channels of W (INT8, offline) and the
    same bf16 activations; a step quantizes A and produces the full [M, N]
    bf16 output on EVERY rank.  Fused: m5b_gemm_allgather stores each output
    tile into all ranks' outputs over NVLink (CUDA-IPC peer mappings), between
    two one-element all-reduces.  Baseline: local GEMM into [M, N/world], NCCL
    all_gather_into_tensor, permute into [M, N].  Total work is fixed
    (strong scaling); times are CUDA events on the stream, max over ranks.
    """
    import torch
    import torch.distributed as dist

    import m5kernels_b200 as m5
    from m5kernels_b200 import sharding

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))
    m, k, n = 4096, 4096, 16384
    c0, c1 = sharding.shard_columns(n, world, rank)
    g = torch.Generator(device=dev).manual_seed(5)  # same activations on every rank
    x = torch.randn(m, k, device=dev, generator=g).to(torch.bfloat16)
    gw = torch.Generator(device=dev).manual_seed(100 + rank)
    w = (0.02 * torch.randn(c1 - c0, k, device=dev, generator=gw)).to(torch.bfloat16)
    wq, sw = m5.quantize(w, "int8")
    del w
    out = torch.empty((m, n), dtype=torch.bfloat16, device=dev)
    gather = sharding.ColumnParallelGather(out) if world > 1 else None

    def fused():
        q, s = m5.quantize(x, "int8")
        if gather is not None:
            gather.step(q, wq, s, sw)
        else:
            m5.gemm_allgather(q, wq, out, 0, (), "int8", a_scales=s, b_scales=sw)

    def baseline():
        q, s = m5.quantize(x, "int8")
        y = m5.gemm(q, wq, "int8", a_scales=s, b_scales=sw, output_dtype=torch.bfloat16)
        if world > 1:
            return sharding.gather_columns(y, world)
        return y

    stream = torch.cuda.current_stream(dev)

    def timed(fn):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / args.steps
        return sharding.max_over_ranks(ms, device=dev)

    with ClockSampler(local) as clocks:
        fused_ms = timed(fused)
        base_ms = timed(baseline)
    ops = 2.0 * m * n * k
    peer_bytes = (world - 1) * m * (c1 - c0) * 2
    line = {"workload": "colpar_ffn_up", "n_gpus": world, "ms": fused_ms,
            "value": ops / (fused_ms * 1e-3) / 1e12, "unit": "TOPS", "scaling": "strong",
            "config": {"M": m, "K": k, "N": n, "N_per_rank": c1 - c0},
            "kernel": "quant_rows + gemm_tc_kernel<i8,256,pair> (all-gather epilogue)",
            "nccl_baseline_ms": base_ms, "nccl_baseline_value": ops / (base_ms * 1e-3) / 1e12,
            "speedup_vs_nccl": base_ms / fused_ms, "steps": args.steps,
            "nvlink_bytes_out_per_rank": peer_bytes,
            "nvlink_gbs_per_rank": peer_bytes / (fused_ms * 1e-3) / 1e9 if world > 1 else 0.0,
            "clocks": clocks.summary()}
    if gather is not None:
        gather.barrier()
        gather.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)
    return 0


def run_reference(args, world, rank):
    """The reference arm: the reference's CPU path on rank 0 (other ranks exit)."""
    if rank != 0:
        return 0
    cb = cpu_reference(args.steps, args.warmup)
    line = {
        "impl": "reference", "metric": METRIC, "value": cb["value"], "unit": "TOPS",
        "n_gpus": args.gpus, "steps": cb["steps_timed"], "warmup": args.warmup,
        "ms_per_step": cb["seconds_per_step"] * 1e3,
        "rows_per_step": cb["rows_per_step"],
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int8",
        "data": "synthetic", "config": _config(args.gpus),
        "cpu_baseline": {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample",
                                            "threads")},
        "e2e": {"value": cb["value"], "unit": "TOPS", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_b200(args, world, rank, local):
    import ctypes

    import torch
    import torch.distributed as dist

    import m5kernels_b200 as m5
    from m5kernels_b200 import _lib

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v):
        t = torch.tensor([v], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # This rank's rows of the job.  --rank-share S (one GPU) runs rank 0's share
    # of an S-GPU job: the per-rank step of that run, on this GPU alone.
    share = world if world > 1 else max(1, args.rank_share)
    r0, r1 = _rows(share, rank if world > 1 else 0)
    m = r1 - r0
    nsets = _operand_sets(m)
    gen = torch.Generator(device=dev).manual_seed(1234 + rank)
    steps_sets = []
    for _ in range(nsets):
        a = torch.randn(m, K, device=dev, generator=gen, dtype=torch.float32).to(torch.bfloat16)
        w = (torch.randn(N, K, device=dev, generator=gen, dtype=torch.float32) * 0.02).to(torch.bfloat16)
        wq, ws = m5.quantize(w, "int8")  # offline weight preparation (untimed)
        del w
        y = torch.empty((m, N), dtype=torch.bfloat16, device=dev)
        steps_sets.append(m5.OnlineProjection(a, wq, ws, y, "int8"))
    torch.cuda.synchronize()
    splitk = steps_sets[0].gemm_ws is not None

    for i in range(args.warmup):
        steps_sets[i % nsets]()
    torch.cuda.synchronize()
    barrier()

    stream = torch.cuda.current_stream(dev)
    K_steps = args.steps

    def graph_of(fn):
        """The K timed launches as one CUDA graph (no events inside: event nodes
        between kernels add their own latency to every step)."""
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for i in range(K_steps):
                fn(steps_sets[i % nsets])
        g.replay()  # untimed first replay (graph upload)
        torch.cuda.synchronize()
        return g

    def replay_ms(g):
        a0 = torch.cuda.Event(enable_timing=True)
        a1 = torch.cuda.Event(enable_timing=True)
        a0.record(stream)
        g.replay()
        a1.record(stream)
        torch.cuda.synchronize()
        return a0.elapsed_time(a1)

    graph = graph_of(lambda st: st())
    # Kernel durations for the roofline: the same K steps replayed once more
    # right after the timed region, now with CUDA events recorded between the
    # kernels (event nodes inside the graph; they lengthen each kernel's
    # interval by their own latency, which is why the headline replay has
    # none).  Without event nodes in graphs, each kernel's K launches alone.
    kernel_timing = ("CUDA events between the kernels in a second replay of the same K steps "
                     "right after the timed region")
    ev = [[torch.cuda.Event(enable_timing=True, external=True) for _ in range(3)]
          for _ in range(K_steps)]
    graph_ev = torch.cuda.CUDAGraph()
    try:
        with torch.cuda.graph(graph_ev):
            for i in range(K_steps):
                st = steps_sets[i % nsets]
                ev[i][0].record()
                st.quantize()
                ev[i][1].record()
                st.gemm()
                ev[i][2].record()
        graph_ev.replay()
        torch.cuda.synchronize()
    except Exception:
        graph_ev = None
        kernel_timing = ("each kernel's K launches alone as a CUDA graph, CUDA events around the "
                         "replay, right after the timed region")
    barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        barrier()
        torch.cuda.synchronize()
        clocks.active.set()
        e0.record(stream)
        graph.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        clocks.active.clear()
        barrier()
        ms_total = e0.elapsed_time(e1)
        del graph
        if graph_ev is not None:
            graph_ev.replay()
            torch.cuda.synchronize()
            prep_ms = sum(e[0].elapsed_time(e[1]) for e in ev) / K_steps
            gemm_ms = sum(e[1].elapsed_time(e[2]) for e in ev) / K_steps
            del graph_ev
        else:
            g_prep = graph_of(lambda st: st.quantize())
            prep_ms = replay_ms(g_prep) / K_steps
            del g_prep
            g_gemm = graph_of(lambda st: st.gemm())
            gemm_ms = replay_ms(g_gemm) / K_steps
            del g_gemm
        ms_per_step = max_over_ranks(ms_total / K_steps)
        prep_ms_max = max_over_ranks(prep_ms)
        gemm_ms_max = max_over_ranks(gemm_ms)
        ops_job = 2.0 * M * N * K
        ops_rank = 2.0 * m * N * K
        # the whole job over the slowest rank (one GPU: the job, or with
        # --rank-share only this GPU's share of it)
        value = (ops_job if world > 1 else ops_rank) / (ms_per_step * 1e-3) / 1e12

        if args.profile:
            if rank == 0:
                print(json.dumps({"profile": True, "ms_per_step": ms_per_step, "gemm_ms": gemm_ms,
                                  "prep_ms": prep_ms, "rows_per_rank": m, "splitk": splitk}),
                      flush=True)
            if world > 1:
                dist.destroy_process_group()
            return 0

        # End to end through the public C ABI (one m5b_linear_ex call per step:
        # online quantize -> GEMM) from pinned host memory: every step copies
        # this rank's activations host -> device and its output device -> host
        # inside the timed region.  Copies run on their own streams so that step
        # i's host -> device copy, step i-1's compute and step i-2's
        # device -> host copy overlap (the link is full duplex); device buffers
        # are double-buffered and events order every reuse.
        host_a = [steps_sets[i].x.to("cpu").pin_memory() for i in range(nsets)]
        host_out = [torch.empty((m, N), dtype=torch.bfloat16).pin_memory() for _ in range(2)]
        dev_a = [torch.empty((m, K), dtype=torch.bfloat16, device=dev) for _ in range(2)]
        dev_y = [torch.empty((m, N), dtype=torch.bfloat16, device=dev) for _ in range(2)]
        h2d_stream = torch.cuda.Stream(dev)
        d2h_stream = torch.cuda.Stream(dev)
        lib = _lib.lib()
        ws_bytes = int(lib.m5b_linear_workspace_bytes(m, K))
        workspace = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
        gws_bytes = int(lib.m5b_gemm_workspace_bytes(m, N, K, _lib.MODE["int8"]))
        gemm_ws = torch.zeros(max(gws_bytes, 1), dtype=torch.uint8, device=dev)

        def linear_into(x, wq, wsc, y):
            _lib.check(lib.m5b_linear_ex(
                ctypes.c_void_p(x.data_ptr()), _lib.BF16, m, K, 0, None,
                ctypes.c_void_p(wq.data_ptr()), ctypes.c_void_p(wsc.data_ptr()), N,
                _lib.MODE["int8"], ctypes.c_void_p(y.data_ptr()), _lib.BF16,
                ctypes.c_void_p(workspace.data_ptr()), ws_bytes,
                ctypes.c_void_p(gemm_ws.data_ptr()) if gws_bytes else None, gws_bytes,
                ctypes.c_void_p(stream.cuda_stream)))

        def run_e2e(n):
            h2d_done = [torch.cuda.Event() for _ in range(n)]
            comp_done = [torch.cuda.Event() for _ in range(n)]
            d2h_done = [torch.cuda.Event() for _ in range(n)]
            for i in range(n):
                b = i % 2
                with torch.cuda.stream(h2d_stream):
                    if i >= 2:
                        h2d_stream.wait_event(comp_done[i - 2])  # dev_a[b] consumed
                    dev_a[b].copy_(host_a[i % nsets], non_blocking=True)
                    h2d_done[i].record(h2d_stream)
                stream.wait_event(h2d_done[i])
                if i >= 2:
                    stream.wait_event(d2h_done[i - 2])  # dev_y[b] copied out
                st = steps_sets[i % nsets]
                linear_into(dev_a[b], st.wq, st.w_scales, dev_y[b])
                comp_done[i].record(stream)
                with torch.cuda.stream(d2h_stream):
                    d2h_stream.wait_event(comp_done[i])
                    host_out[b].copy_(dev_y[b], non_blocking=True)
                    d2h_done[i].record(d2h_stream)
            stream.wait_event(d2h_done[n - 1])  # the timed region ends after the last copy

        run_e2e(min(args.warmup, 3))
        torch.cuda.synchronize()
        barrier()
        e2e_steps = max(3, min(args.steps, 10))
        torch.cuda.synchronize()
        clocks.active.set()
        e0.record(stream)
        h2d_stream.wait_event(e0)
        run_e2e(e2e_steps)
        e1.record(stream)
        torch.cuda.synchronize()
        clocks.active.clear()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / e2e_steps)
    e2e_value = (ops_job if world > 1 else ops_rank) / (e2e_ms * 1e-3) / 1e12

    # The link's own ceiling for the e2e copies: the same pinned host -> device
    # copies of the activations, back to back with nothing else running.
    c0 = torch.cuda.Event(enable_timing=True)
    c1 = torch.cuda.Event(enable_timing=True)
    dev_a[0].copy_(host_a[0], non_blocking=True)
    torch.cuda.synchronize()
    c0.record(stream)
    for i in range(e2e_steps):
        dev_a[i % 2].copy_(host_a[i % nsets], non_blocking=True)
    c1.record(stream)
    torch.cuda.synchronize()
    h2d_copy_ms = max_over_ranks(c0.elapsed_time(c1) / e2e_steps)
    h2d_bytes = m * K * 2

    peaks = _peaks()
    int8_peak = 2.0 * peaks["bf16"]  # dense INT8 = 2x dense BF16 on B200 (4.5 / 2.25 PF nominal)
    gemm_tops = ops_rank / (gemm_ms_max * 1e-3) / 1e12
    prep_bytes = m * (3 * K + 4)
    prep_gbs = prep_bytes / (prep_ms_max * 1e-3) / 1e9
    out = None
    if rank == 0:
        cb = cpu_reference(1, 1, budget_s=12.0) if world == 1 and share == 1 else None
        omp = cpu_omp_baseline() if world == 1 and share == 1 else None
        clock = clocks.summary()
        kernel = "gemm_tc_kernel<i8,256,pair>" + (" split-K" if splitk else "")
        out = {
            "metric": METRIC, "value": value, "unit": "TOPS", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int8",
            "data": "synthetic",
            "config": _config(share),
            "roofline": {"bound": "tensor", "achieved": gemm_tops, "peak": int8_peak,
                         "unit": "TFLOP/s", "frac": gemm_tops / int8_peak,
                         "traffic": GEMM_TRAFFIC_BYTES.get(m),
                         "traffic_source": GEMM_TRAFFIC_SOURCE if m in GEMM_TRAFFIC_BYTES else None,
                         "kernel": kernel,
                         "peak_source": (f"2 x {peaks['source']} dense bf16 ({peaks['bf16']} TF/s); "
                                         "nominal dense INT8 4500 TOPS"),
                         "frac_of_nominal_int8": gemm_tops / 4500.0},
            "prep": {"kernel": "quant_rows_kernel<bf16,int8,VPT=8,exact>", "ms": prep_ms_max,
                     "achieved_gbs": prep_gbs, "peak_gbs": peaks["hbm_gbs"],
                     "frac": prep_gbs / peaks["hbm_gbs"], "bytes": prep_bytes},
            "gemm_ms": gemm_ms_max, "rows_per_rank": m, "kernel_timing": kernel_timing,
            "pct_int8_peak_incl_quant": (ops_rank / (ms_per_step * 1e-3) / 1e12) / int8_peak,
            "cpu_baseline": ({k: cb[k] for k in ("value", "unit", "cores", "kind", "sample",
                                                 "threads")} if cb else None),
            "cpu_baseline_omp": omp,
            "e2e": {"value": e2e_value, "unit": "TOPS", "h2d_bytes_per_step": m * K * 2,
                    "d2h_bytes_per_step": m * N * 2, "api": "m5b_linear_ex",
                    # host -> device rate inside the e2e steps against the same
                    # copies timed alone (the PCIe ceiling of this path)
                    "link": {"bound": "host->device copies",
                             "h2d_gbs_in_e2e": h2d_bytes / (e2e_ms * 1e-3) / 1e9,
                             "h2d_gbs_copies_alone": h2d_bytes / (h2d_copy_ms * 1e-3) / 1e9,
                             "frac": h2d_copy_ms / e2e_ms}},
            "clocks": clock,
            "gpu_launches": 2 * args.steps,
        }
        if world == 1 and share > 1:
            out["rank_share"] = {"of_gpus": share, "note": "rank 0's rows of a " + str(share) +
                                 "-GPU job timed alone on this GPU; value is this GPU's share",
                                 "projected_job_tops": value * share}
        print(json.dumps(out), flush=True)
    if world > 1:
        barrier()
        dist.destroy_process_group()
    return 0


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--workload", default="ffn_down",
                    choices=["ffn_down", "prep_c3", "prep_c4", "qk_c5", "rms_q", "colpar"],
                    help="ffn_down is the headline; the others time one other BASELINE config")
    ap.add_argument("--profile", action="store_true",
                    help="profiling run: timed steps and per-kernel timing only (no e2e, no CPU leg)")
    ap.add_argument("--rank-share", type=int, default=1,
                    help="(one GPU) time rank 0's rows of an N-GPU job on this GPU alone")
    args = ap.parse_args(argv)
    if args.warmup < 3:
        args.warmup = 3
    world, rank, local = _dist()
    if args.impl == "reference":
        return run_reference(args, world, rank)
    if args.workload == "colpar":
        return run_colpar(args, world, rank, local)
    if args.workload != "ffn_down":
        return run_secondary(args, world, rank, local)
    return run_b200(args, world, rank, local)


if __name__ == "__main__":
    sys.exit(main())
