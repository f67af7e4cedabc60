"""Checked, timed experiment cases for the cuda-b200 backends.

Twin of the reference harness (src/m5kernels/engine.py:20-541): a case is
prepared (seeded inputs, offline weight preparation, sampled float64
references), run once and checked against the references, and only timed
when it passed.  The result dict carries the same fields (status
ok / incorrect / unsupported / error, implementation and quality error,
stages, effective TOPS) plus the device-side timing this backend adds.

Backends (the `backend` string of run_case):
    gemm                      cuda-b200            online per-token quant + W8A8 / FP8 GEMM
                              cuda-b200-hadamard   online rotation + quant + GEMM (weights rotated offline)
    norm_hadamard_gemm        cuda-b200-norm-fused fused norm/modulation/rotation/INT8 prep + GEMM
                              cuda-b200-norm-staged      unfused_norm -> rotate -> quantize + GEMM
    gated_norm_hadamard_gemm  cuda-b200-residual-fused   gated residual + the above, R' written once
                              cuda-b200-residual-separate  gated_residual_add -> fused prep + GEMM
    qk_rope                   cuda-b200-qk-fused   H + INT8 prep + projection with RMSNorm + RoPE epilogue
                              cuda-b200-qk-staged  H + INT8 prep + bf16 projection -> qk_norm_rope
    rms_quant_gemm            cuda-b200-rms-folded RMS prep with the inverse RMS folded into the scale + GEMM
                              cuda-b200-rms-direct RMS prep normalizing first + GEMM
"""

from __future__ import annotations

import contextlib
import hashlib
import json
import platform
import statistics
import time
from datetime import datetime, timezone
from pathlib import Path

import numpy as np
import torch

from . import _lib
from .cuda import gemm, gemm_schedule, quantize
from .hadamard import hadamard_quantize, rotate
from .norm_hadamard import (fused_gated_residual_norm_hadamard_quantize,
                            fused_norm_hadamard_quantize, gated_residual_add, unfused_norm)
from .qk_rope import projection_qk_rope, qk_norm_rope, rope_tables
from .rms_quant import rms_quantize

BACKENDS = {
    "gemm": ("cuda-b200", "cuda-b200-hadamard"),
    "norm_hadamard_gemm": ("cuda-b200-norm-fused", "cuda-b200-norm-staged"),
    "gated_norm_hadamard_gemm": ("cuda-b200-residual-fused", "cuda-b200-residual-separate"),
    "qk_rope": ("cuda-b200-qk-fused", "cuda-b200-qk-staged"),
    "rms_quant_gemm": ("cuda-b200-rms-folded", "cuda-b200-rms-direct"),
}


class NumericalMismatch(ValueError):
    """A checked output failed correctness, with serializable diagnostics."""

    def __init__(self, message, **diagnostics):
        super().__init__(message)
        self.diagnostics = diagnostics


# ------------------------------------------------------------------ helpers
def metrics(actual, reference) -> dict:
    """Relative L2 / max abs / RMSE / cosine of two float arrays (float64)."""
    a = np.asarray(actual, dtype=np.float64)
    r = np.asarray(reference, dtype=np.float64)
    if a.shape != r.shape:
        raise ValueError("reference shape mismatch")
    if not (np.isfinite(a).all() and np.isfinite(r).all()):
        return {"finite": False, "relative_l2": None, "max_abs": None, "rmse": None, "cosine": None}
    d = a - r
    rn, an = np.linalg.norm(r), np.linalg.norm(a)
    return {
        "finite": True,
        "relative_l2": float(np.linalg.norm(d) / max(rn, 1e-30)),
        "max_abs": float(np.abs(d).max()) if d.size else 0.0,
        "rmse": float(np.sqrt(np.mean(d * d))) if d.size else 0.0,
        "cosine": float(np.dot(a.ravel(), r.ravel()) / max(rn * an, 1e-30)) if rn else float(an == 0),
    }


def sample_indices(length: int, count: int = 32) -> np.ndarray:
    return np.unique(np.linspace(0, length - 1, min(length, count), dtype=int))


def all_finite(outputs) -> bool:
    if isinstance(outputs, (tuple, list)):
        return all(all_finite(o) for o in outputs)
    if outputs.dtype in (torch.int8, torch.uint8, torch.int32):
        return True
    return bool(torch.isfinite(outputs).all().item())


def _f64(t) -> np.ndarray:
    return t.detach().to("cpu", torch.float64).numpy()


def timed(fn, warmup: int, repeat: int) -> dict:
    """Per-sample device time (CUDA events on the current stream) and host wall time.

    Before each sample a short device spin is queued ahead of the start event,
    so the host-side launch latency of `fn` overlaps the spin instead of being
    counted as device time.
    """
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    dev_ms, wall_ms = [], []
    for _ in range(repeat):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        start = time.perf_counter_ns()
        torch.cuda._sleep(200_000)  # ~0.1 ms at 2 GHz: covers the launch overhead of fn
        e0.record(stream)
        fn()
        e1.record(stream)
        torch.cuda.synchronize()
        wall_ms.append((time.perf_counter_ns() - start) / 1e6)
        dev_ms.append(e0.elapsed_time(e1))
    return dict(
        kind="cuda_event_device_time",
        samples_ms=dev_ms,
        median_ms=statistics.median(dev_ms),
        p10_ms=float(np.percentile(dev_ms, 10)),
        p90_ms=float(np.percentile(dev_ms, 90)),
        min_ms=min(dev_ms),
        host_wall_median_ms=statistics.median(wall_ms),
        warmup=warmup,
        repeat=repeat,
    )


def environment() -> dict:
    env = dict(timestamp_utc=datetime.now(timezone.utc).isoformat(), os=platform.platform(),
               python=platform.python_version(), numpy=np.__version__, torch=torch.__version__,
               library=str(_lib.LIB_PATH))
    if _lib.LIB_PATH.exists():
        env["library_sha256"] = hashlib.sha256(_lib.LIB_PATH.read_bytes()).hexdigest()
    if torch.cuda.is_available():
        p = torch.cuda.get_device_properties(torch.cuda.current_device())
        env["device"] = dict(name=p.name, sms=p.multi_processor_count,
                             memory_gb=round(p.total_memory / 2**30, 1))
    else:
        env["device"] = None
    return env


def _inputs(c, seed, distribution, dev, weight_std=None):
    m, n, k = c["m"], c["n"], c["k"]
    g = torch.Generator(device="cpu").manual_seed(seed)
    a = torch.randn(m, k, generator=g)
    std = c.get("weight_std", weight_std)
    w = torch.randn(n, k, generator=g) * (std if std is not None else k ** -0.5)
    if distribution == "outliers":
        # 1 % of K channels, chosen by seed, scaled x50 (BASELINE outlier variant)
        cols = torch.randperm(k, generator=g)[: max(1, k // 100)]
        a[:, cols] *= 50
    elif distribution == "zeros":
        a.zero_()
        w.zero_()
    elif distribution != "normal":
        raise ValueError("distribution must be normal, outliers or zeros")
    return a.to(torch.bfloat16).to(dev), w.to(torch.bfloat16).to(dev)


def _sampled_dot(x, w, ri, ci):
    return _f64(x[torch.as_tensor(ri, device=x.device)]) @ _f64(w[torch.as_tensor(ci, device=w.device)]).T


def _decoded(q, s, rows, mode):
    from .cuda import quantize as _unused  # noqa: F401  (keeps import graph explicit)
    idx = torch.as_tensor(rows, device=q.device)
    qs = q[idx].cpu()
    ss = s[idx].cpu().double()
    if mode == "fp8":
        vals = qs.view(torch.float8_e4m3fn).to(torch.float64)
    else:
        vals = qs.to(torch.float64)
    return (vals * ss[:, None]).numpy()


# ------------------------------------------------------------------ prepare
def prepare_gemm(c, backend, precision, seed, distribution, tile):
    if precision not in ("int8", "fp8"):
        raise NotImplementedError("the cuda-b200 GEMM backends are W8A8 (int8) and FP8 (E4M3)")
    dev = torch.device("cuda")
    x, w = _inputs(c, seed, distribution, dev)
    m, n, k = c["m"], c["n"], c["k"]
    ri, ci = sample_indices(m), sample_indices(n)
    original = _sampled_dot(x, w, ri, ci)
    meta = dict(mac_operations=2 * m * n * k, sample_rows=ri.tolist(), sample_cols=ci.tolist(),
                input_dtype="bf16", output_dtype="bf16", weight_layout="N,K (K-major)",
                weight_quantization_timed=False,
                quantization="symmetric_per_token_A_per_output_channel_W")
    if backend == "cuda-b200":
        bq, sb = quantize(w, precision)
        prep = lambda: quantize(x, precision)  # noqa: E731
        meta.update(compute_path=f"row_prep_quant + tcgen05_{precision}_gemm")
    elif backend == "cuda-b200-hadamard":
        cfg = c.get("hadamard", {})
        block = cfg.get("block_size", 256)
        sign_seed = cfg.get("sign_seed")
        if sign_seed is not None:
            from numpy.random import PCG64, Generator

            draws = Generator(PCG64(sign_seed)).integers(0, 2, size=k, dtype=np.int8)
            signs = torch.from_numpy((2 * draws - 1).astype(np.int8)).to(dev)
        else:
            signs = torch.ones(k, dtype=torch.int8, device=dev)
        bq, sb = hadamard_quantize(w, block, signs, precision)  # offline weight rotation + quant
        prep = lambda: hadamard_quantize(x, block, signs, precision)  # noqa: E731
        xr = rotate(x[torch.as_tensor(ri, device=dev)], block, signs)
        wr = rotate(w[torch.as_tensor(ci, device=dev)], block, signs)
        rot_dot = _f64(xr) @ _f64(wr).T
        meta.update(compute_path=f"fused_hadamard_quant + tcgen05_{precision}_gemm",
                    transform=dict(kind="normalized_block_sylvester_hadamard", block_size=block,
                                   sign_seed=sign_seed,
                                   rotated_dot_preservation=metrics(rot_dot, original)),
                    transform_pass=metrics(rot_dot, original)["relative_l2"] <= 1e-5)
    else:
        raise NotImplementedError(f"GEMM backend {backend} is not implemented")
    aq, sa = prep()
    expected = _decoded(aq, sa, ri, precision) @ _decoded(bq, sb, ci, precision).T

    def compute(q, s):
        return gemm(q, bq, precision, tile, a_scales=s, b_scales=sb, output_dtype=torch.bfloat16)

    def fn():
        return compute(aq, sa)

    def online():
        return compute(*prep())

    def check(y):
        return _f64(y[torch.as_tensor(ri, device=dev)][:, torch.as_tensor(ci, device=dev)])

    stages = {"activation_prepare": prep, "online_activation_plus_gemm": online}
    return fn, check, expected, original, stages, meta


def prepare_norm_hadamard_gemm(c, backend, precision, seed, distribution, tile):
    gated = c["op"] == "gated_norm_hadamard_gemm"
    allowed = BACKENDS[c["op"]]
    if backend not in allowed or precision != "int8":
        raise NotImplementedError(
            f"supported backend/precision pairs: {sorted((b, 'int8') for b in allowed)}")
    fused_path = backend in ("cuda-b200-norm-fused", "cuda-b200-residual-fused")
    from .reference_checks import norm_reference_rows

    dev = torch.device("cuda")
    m, n, k = c["m"], c["n"], c["k"]
    cfg = c.get("fusion", {})
    norm = cfg.get("norm", "rms")
    eps = cfg.get("epsilon", 1e-5)
    block = cfg.get("block_size", 256)
    samples = cfg.get("samples")
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    w = (torch.randn(n, k, generator=g) * c.get("weight_std", k ** -0.5)).to(torch.bfloat16)
    if samples:  # AdaLN tables per sample, rows map to samples of m / samples tokens
        p = int(samples)
        gamma = torch.ones(k, dtype=torch.bfloat16) if not cfg.get("affine", False) else \
            (1 + 0.1 * torch.randn(k, generator=g)).to(torch.bfloat16)
        scale = (0.1 * torch.randn(p, k, generator=g)).to(torch.bfloat16)
        shift = (0.1 * torch.randn(p, k, generator=g)).to(torch.bfloat16)
        row_map = (torch.arange(m, dtype=torch.int32) * p // m).to(torch.int32)
    else:
        gamma = (1 + 0.1 * torch.randn(k, generator=g)).to(torch.bfloat16)
        scale = (0.2 * torch.randn(k, generator=g)).to(torch.bfloat16)
        shift = (0.1 * torch.randn(k, generator=g)).to(torch.bfloat16)
        row_map = None
    signs = torch.ones(k, dtype=torch.int8)
    if gated:
        branch = torch.randn(m, k, generator=g).to(torch.bfloat16)
        if samples:
            gate = (0.1 * torch.randn(int(samples), k, generator=g)).to(torch.bfloat16)
            gate_row_map = row_map
        else:
            gate = (0.2 * torch.randn(k, generator=g)).to(torch.bfloat16)
            gate_row_map = None
    if distribution == "zeros":
        x.zero_()
        w.zero_()
    ri, ci = sample_indices(m), sample_indices(n)
    T = lambda t: None if t is None else t.to(dev)  # noqa: E731
    xd, wd, gd, scd, shd, sgd, rmd = map(T, (x, w, gamma, scale, shift, signs, row_map))
    wq, sw = hadamard_quantize(wd, block, sgd, "int8")  # offline weight rotation + quant
    if gated:
        bd, gtd, grmd = T(branch), T(gate), T(gate_row_map)

        def prep_fused():
            return fused_gated_residual_norm_hadamard_quantize(
                xd, bd, gtd, gd, scd, shd, sgd, block, norm=norm, epsilon=eps,
                gate_row_map=grmd, row_map=rmd)

        def prep_staged():  # the fair two-launch baseline (norm_hadamard_gemm.py:261-276)
            updated = gated_residual_add(xd, bd, gtd, gate_row_map=grmd)
            q, s = fused_norm_hadamard_quantize(updated, gd, scd, shd, sgd, block, norm=norm,
                                                epsilon=eps, row_map=rmd)
            return q, s, updated
    else:

        def prep_fused():
            return fused_norm_hadamard_quantize(xd, gd, scd, shd, sgd, block, norm=norm,
                                                epsilon=eps, row_map=rmd)

        def prep_staged():  # norm -> rotate -> quantize as three launches (:225-226)
            y = unfused_norm(xd, gd, scd, shd, norm=norm, epsilon=eps, row_map=rmd)
            return quantize(rotate(y, block, sgd), "int8")

    prep = prep_fused if fused_path else prep_staged

    prepared = prep()
    aq, sa = prepared[:2]
    refs = norm_reference_rows(x, gamma, scale, shift, row_map, ri, norm, eps, block, signs,
                               branch=branch if gated else None, gate=gate if gated else None,
                               gate_row_map=gate_row_map if gated else None)
    # The other path of the pair must give the same codes, scales (and R') bit for bit.
    other = (prep_staged if fused_path else prep_fused)()
    paired_exact = all(bool(torch.equal(u, v)) for u, v in zip(prepared, other))
    meta = dict(mac_operations=2 * m * n * k, sample_rows=ri.tolist(), sample_cols=ci.tolist(),
                norm=norm, epsilon=eps, block_size=block, samples=samples, gated=gated,
                compute_path=("fused_row_prep" if fused_path else
                              ("gated_residual_add + fused_row_prep" if gated else
                               "unfused_norm + rotate + quantize")) + " + tcgen05_int8_gemm",
                paired_path_exact=paired_exact)
    # activation checks against the float64 reference on sampled rows (reference gates)
    codes = aq[torch.as_tensor(ri, device=dev)].cpu().numpy().astype(np.int16)
    scales = sa[torch.as_tensor(ri, device=dev)].cpu().numpy()
    code_diff = float(np.abs(codes - refs["codes"].astype(np.int16)).max())
    scale_err = metrics(scales, refs["scales"])
    transform_pass = code_diff <= 1 and scale_err["relative_l2"] <= 0.008 and paired_exact
    if gated:
        r_rows = prepared[2][torch.as_tensor(ri, device=dev)].cpu()
        residual_exact = bool(torch.equal(r_rows, refs["residual_bf16"]))
        transform_pass = transform_pass and residual_exact
        meta.update(residual_update_exact_match=residual_exact)
    meta.update(activation_max_code_difference=code_diff, activation_scale_error=scale_err,
                transform_pass=transform_pass)
    wrows = torch.as_tensor(ci, device=dev)
    dec_w = _decoded(wq, sw, ci, "int8")
    expected = _decoded(aq, sa, ri, "int8") @ dec_w.T
    original = refs["rounded_modulated"] @ _f64(wd[wrows]).T

    def compute(q, s):
        return gemm(q, wq, "int8", tile, a_scales=s, b_scales=sw, output_dtype=torch.bfloat16)

    def fn():
        y = compute(aq, sa)
        return (y, prepared[2]) if gated else y

    def online():
        pp = prep()
        y = compute(pp[0], pp[1])
        return (y, pp[2]) if gated else y

    def check(y):
        if gated:
            y = y[0]
        return _f64(y[torch.as_tensor(ri, device=dev)][:, wrows])

    return fn, check, expected, original, {"activation_prepare": prep,
                                           "online_activation_plus_gemm": online}, meta


def prepare_qk_rope(c, backend, precision, seed, distribution, tile):
    if backend not in BACKENDS["qk_rope"] or precision != "int8":
        raise NotImplementedError("qk_rope supports cuda-b200-qk-fused/cuda-b200-qk-staged with INT8 only")
    from .reference_checks import qk_reference_rows

    dev = torch.device("cuda")
    m, n, k = c["m"], c["n"], c["k"]
    if n % 128:
        raise NotImplementedError("Q/K projection requires complete 128-wide heads")
    half = c.get("rope_half", 64)
    eps = c.get("epsilon", 1e-5)
    block = c.get("block_size", 256)
    theta = c.get("theta", 10000.0)
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16).to(dev)
    w = (torch.randn(n, k, generator=g) * c.get("weight_std", k ** -0.5)).to(torch.bfloat16).to(dev)
    gamma = (1 + c.get("gamma_std", 0.2) * torch.randn(128, generator=g)).to(torch.bfloat16).to(dev)
    cos, sin = rope_tables(m, half, theta, device=dev)
    signs = torch.ones(k, dtype=torch.int8, device=dev)
    bq, sb = hadamard_quantize(w, block, signs, "int8")
    prep = lambda: hadamard_quantize(x, block, signs, "int8")  # noqa: E731
    aq, sa = prep()
    rows = sample_indices(m)
    heads = sample_indices(n // 128, 2)
    cols = (heads[:, None] * 128 + np.arange(128)[None, :]).reshape(-1)
    ridx, hidx = torch.as_tensor(rows, device=dev), torch.as_tensor(heads, device=dev)
    expected = qk_reference_rows(_decoded(aq, sa, rows, "int8") @ _decoded(bq, sb, cols, "int8").T,
                                 gamma, cos[ridx], sin[ridx], eps, len(heads))
    original = qk_reference_rows(_f64(x[ridx]) @ _f64(w[torch.as_tensor(cols, device=dev)]).T,
                                 gamma, cos[ridx], sin[ridx], eps, len(heads))

    def fused(q, s):
        return projection_qk_rope(q, bq, gamma, cos, sin, "int8", tile, a_scales=s, b_scales=sb,
                                  epsilon=eps)

    def staged(q, s):  # bf16 projection stored, then the standalone post-process
        projected = gemm(q, bq, "int8", tile, a_scales=s, b_scales=sb,
                         output_dtype=torch.bfloat16)
        return qk_norm_rope(projected, gamma, cos, sin, epsilon=eps)

    selected = fused if backend == "cuda-b200-qk-fused" else staged
    # Same exact integer dot, FP32 dequantization order and post-processing:
    # the paired paths must agree on every output, not only the sampled rows.
    paired_exact = bool(torch.equal(fused(aq, sa), staged(aq, sa)))

    def fn():
        return selected(aq, sa)

    def online():
        return selected(*prep())

    def check(y):
        return _f64(y[hidx][:, ridx, :]).reshape(-1)

    meta = dict(mac_operations=2 * m * n * k, sample_rows=rows.tolist(),
                sample_heads=heads.tolist(), rope_half=half, theta=theta, epsilon=eps,
                block_size=block, output_layout="head-major [H,M,128]",
                compute_path=("fused_hadamard_quant + tcgen05_int8_qk_rope"
                              if backend == "cuda-b200-qk-fused" else
                              "fused_hadamard_quant + tcgen05_int8_gemm(bf16) + qk_norm_rope"),
                paired_path_exact=paired_exact, transform_pass=paired_exact)
    return fn, check, expected.reshape(-1), original.reshape(-1), {
        "activation_prepare": prep, "online_activation_plus_gemm": online}, meta


def validate_rms_config(c, backend, precision, distribution) -> dict:
    """Semantics of an rms_quant_gemm case (src/m5kernels/rms_quant_gemm.py:14-65)."""
    if backend not in BACKENDS["rms_quant_gemm"] or precision != "int8":
        raise NotImplementedError(
            "rms_quant_gemm supports cuda-b200-rms-direct/cuda-b200-rms-folded with INT8 only")
    if c.get("op") != "rms_quant_gemm":
        raise ValueError("operation must be rms_quant_gemm")
    forbidden = {"shift", "norm", "round_output"}.intersection(c)
    if forbidden:
        raise NotImplementedError(f"unsupported RMS semantics options: {sorted(forbidden)}")
    for key in ("m", "n", "k"):
        if isinstance(c.get(key), bool) or not isinstance(c.get(key), int) or c[key] <= 0:
            raise ValueError(f"{key} must be a positive integer")
    cfg = c.get("rms_quant", {})
    if not isinstance(cfg, dict):
        raise ValueError("rms_quant must be a configuration object")
    unknown = set(cfg) - {"block_size", "gamma", "threads", "epsilon", "sign_seed"}
    if unknown:
        raise NotImplementedError(
            f"unsupported rms_quant options: {sorted(unknown)}; "
            "this experiment requires RMS, zero shift and no BF16 intermediate")
    config = dict(block_size=1, gamma="identity", threads=256, epsilon=1e-5, sign_seed=None)
    config.update(cfg)
    block = config["block_size"]
    if isinstance(block, bool) or not isinstance(block, int) or block <= 0:
        raise ValueError("block_size must be a positive integer")
    if block not in (1, 256):
        raise NotImplementedError("rms_quant_gemm supports block_size 1 or 256")
    if c["k"] % block:
        raise NotImplementedError("K must be divisible by block_size; padding is not implicit")
    if config["gamma"] not in ("identity", "random"):
        raise NotImplementedError("gamma must be identity or random")
    threads = config["threads"]
    if isinstance(threads, bool) or not isinstance(threads, int):
        raise ValueError("threads must be an integer")
    if threads not in (128, 256, 512):
        raise NotImplementedError("supported threadgroup sizes are 128, 256 and 512")
    eps = config["epsilon"]
    if isinstance(eps, bool) or not isinstance(eps, (int, float)) or not np.isfinite(eps) or eps <= 0:
        raise ValueError("epsilon must be positive and finite")
    with np.errstate(over="ignore", under="ignore"):
        eps32 = np.float32(eps)
    if not np.isfinite(eps32) or eps32 <= 0:
        raise ValueError("epsilon must remain positive and finite in float32")
    sign_seed = config["sign_seed"]
    if sign_seed is not None and (isinstance(sign_seed, bool) or not isinstance(sign_seed, int)
                                  or sign_seed < 0):
        raise ValueError("sign_seed must be a nonnegative integer or null")
    if distribution not in ("normal", "outliers", "zeros"):
        raise ValueError("distribution must be normal, outliers or zeros")
    return config


def prepare_rms_quant_gemm(c, backend, precision, seed, distribution, tile):
    """RMS scale-folding (or direct) INT8 preparation + W8A8 GEMM, BF16 out.

    Twin of src/m5kernels/rms_quant_gemm.py:68-260: identical BF16 inputs and
    weights and FP32 gamma for both backends of one seed; weights are signed
    (and rotated for block 256) and quantized per output channel offline.
    """
    cfg = validate_rms_config(c, backend, precision, distribution)
    from .reference_checks import rms_reference_rows

    dev = torch.device("cuda")
    m, n, k = c["m"], c["n"], c["k"]
    block, eps, sign_seed = cfg["block_size"], cfg["epsilon"], cfg["sign_seed"]
    fold = backend == "cuda-b200-rms-folded"
    x, w = _inputs(c, seed, distribution, dev)
    g = torch.Generator(device="cpu").manual_seed(seed + 1)
    gamma = (1 + 0.2 * torch.randn(k, generator=g) if cfg["gamma"] == "random"
             else torch.ones(k)).float()
    if sign_seed is not None:
        from numpy.random import PCG64, Generator

        draws = Generator(PCG64(sign_seed)).integers(0, 2, size=k, dtype=np.int8)
        signs_np = (2 * draws - 1).astype(np.int8)
    else:
        signs_np = np.ones(k, np.int8)
    gamma_d, signs = gamma.to(dev), torch.from_numpy(signs_np).to(dev)
    ri, ci = sample_indices(m), sample_indices(n)

    def offline_weight_prepare():
        if block == 1:
            return quantize(w.float() * signs.float(), "int8")
        return hadamard_quantize(w, block, signs, "int8")

    def activation():
        return rms_quantize(x, gamma_d, signs, block, threads=cfg["threads"], fold_scale=fold,
                            epsilon=eps)

    bq, sb = offline_weight_prepare()
    aq, sa = activation()
    ref_x = _f64(x[torch.as_tensor(ri, device=dev)])
    ref_w = _f64(w[torch.as_tensor(ci, device=dev)])
    ref_a = rms_reference_rows(ref_x, gamma.numpy(), signs_np, block, eps)
    ref_norm = ref_x * ref_a["inverse_rms"][:, None] * gamma.double().numpy()
    original = ref_norm @ ref_w.T
    actual_a = _decoded(aq, sa, ri, "int8")
    expected = actual_a @ _decoded(bq, sb, ci, "int8").T
    idx = torch.as_tensor(ri, device=dev)
    activation_error = metrics(actual_a, ref_a["dequantized"])
    scale_error = metrics(_f64(sa[idx]), ref_a["scales"])
    max_code_error = float(np.max(np.abs(_f64(aq[idx]) - ref_a["quantized"])))
    finite = bool(torch.isfinite(sa).all() and (sa > 0).all() and (aq >= -127).all()
                  and torch.isfinite(sb).all() and (sb > 0).all())
    transform_pass = bool(finite and activation_error["finite"]
                          and activation_error["relative_l2"] <= 0.008
                          and scale_error["finite"] and scale_error["relative_l2"] <= 1e-5
                          and max_code_error <= 1)

    def compute(q, s):
        return gemm(q, bq, "int8", tile, a_scales=s, b_scales=sb, output_dtype=torch.bfloat16)

    def fn():
        return compute(aq, sa)

    def online():
        return compute(*activation())

    def check(y):
        return _f64(y[torch.as_tensor(ri, device=dev)][:, torch.as_tensor(ci, device=dev)])

    meta = dict(compute_path=f"rms_{'folded' if fold else 'direct'}_prep + tcgen05_int8_gemm",
                input_dtype="bf16", output_dtype="bf16", preparation_dtype="fp32",
                mac_operations=2 * m * n * k, sample_rows=ri.tolist(), sample_cols=ci.tolist(),
                norm="rms", epsilon=eps, gamma=cfg["gamma"],
                gamma_sha256=hashlib.sha256(gamma.numpy().tobytes()).hexdigest(),
                fold_scale=fold, additive_shift=False, normalization_rounding="fp32",
                quantization="symmetric_per_token_rotated_A_per_output_channel_rotated_W",
                weight_preparation_in_online=False, weight_preparation_timed=True,
                all_preparation_values_finite=finite, transform_pass=transform_pass,
                activation_implementation_error=activation_error,
                activation_scale_error=scale_error,
                activation_max_code_difference=max_code_error,
                transform=dict(kind="signed_identity" if block == 1
                               else "normalized_block_sylvester_hadamard",
                               block_size=block, sign_seed=sign_seed, threads=cfg["threads"]))
    stages = {"activation_prepare": activation, "online_activation_plus_gemm": online,
              "offline_weight_prepare": offline_weight_prepare}
    return fn, check, expected, original, stages, meta


PREPARE = {
    "gemm": prepare_gemm,
    "norm_hadamard_gemm": prepare_norm_hadamard_gemm,
    "gated_norm_hadamard_gemm": prepare_norm_hadamard_gemm,
    "qk_rope": prepare_qk_rope,
    "rms_quant_gemm": prepare_rms_quant_gemm,
}

QUALITY_LIMIT = {"int8": 0.05, "fp8": 0.10}


def run_case(c, backend, precision, seed=17, distribution="normal", warmup=3, repeat=10,
             tile=(64, 64, 4, 1), schedule=None):
    """Prepare, check and (only if correct) time one case; never raises.

    `schedule` = (split_k, group_m) runs every GEMM of the case under that
    schedule (cuda.gemm_schedule); None keeps the library's choice.
    """
    result = dict(case=c, backend=backend, precision=precision, seed=seed,
                  distribution=distribution, tile=list(tile))
    if schedule is not None:
        result["schedule"] = {"split_k": int(schedule[0]), "group_m": int(schedule[1])}
    meta = {}
    with contextlib.ExitStack() as scope:
        try:
            if schedule is not None:
                scope.enter_context(gemm_schedule(*schedule))
            _run_checked(c, backend, precision, seed, distribution, warmup, repeat, tile, result,
                         meta)
        except NumericalMismatch as e:
            result.update(meta)
            result.update(status="incorrect", reason=str(e), **e.diagnostics)
        except NotImplementedError as e:
            result.update(status="unsupported", reason=str(e))
        except Exception as e:  # noqa: BLE001  (the harness records every failure)
            result.update(status="error", reason=f"{type(e).__name__}: {e}"[:5000])
    if torch.cuda.is_available():
        torch.cuda.empty_cache()
    return result


def _run_checked(c, backend, precision, seed, distribution, warmup, repeat, tile, result, meta):
    """run_case's body: prepare, check, and time only what passed."""
    if c["op"] not in PREPARE:
        raise NotImplementedError(f"op {c['op']} is not part of the cuda-b200 backend")
    if backend not in BACKENDS[c["op"]]:
        raise NotImplementedError(
            f"backend {backend} does not implement {c['op']}; choose one of {BACKENDS[c['op']]}")
    if not torch.cuda.is_available():
        raise _lib.ExtensionMissing("no CUDA device is visible; the cuda-b200 backend has no CPU path")
    est = (c["m"] * c["k"] + c["n"] * c["k"] + c["m"] * c["n"]) * 8
    free = torch.cuda.mem_get_info()[0]
    if est > free:
        raise NotImplementedError("estimated working set exceeds free device memory; split workload")
    fn, check, expected, original, stages, prepared = PREPARE[c["op"]](
        c, backend, precision, seed, distribution, tile)
    meta.update(prepared)
    y = fn()
    torch.cuda.synchronize()
    output_finite = all_finite(y)
    actual = check(y)
    impl = metrics(actual, expected)
    quality = metrics(actual, original)
    tolerance = 0.008
    passed = bool(output_finite and impl["finite"] and impl["relative_l2"] <= tolerance
                  and meta.get("transform_pass", True))
    quality_passed = bool(quality["finite"] and quality["relative_l2"] <= QUALITY_LIMIT[precision])
    result.update(meta, status="ok" if passed else "incorrect", output_finite=output_finite,
                  implementation_error=impl, quality_error=quality,
                  implementation_relative_l2_limit=tolerance,
                  quality_relative_l2_limit=QUALITY_LIMIT[precision],
                  quality_pass=quality_passed)
    online_y = stages["online_activation_plus_gemm"]()
    torch.cuda.synchronize()
    online_error = metrics(check(online_y), expected)
    online_finite = all_finite(online_y)
    result["online_implementation_error"] = online_error
    result["online_output_finite"] = online_finite
    passed = bool(passed and online_finite and online_error["finite"]
                  and online_error["relative_l2"] <= tolerance)
    status_word = _lib.device_status(clear=True)
    if status_word:
        passed = False
        result["device_status"] = status_word
    result["status"] = "ok" if passed else "incorrect"
    del online_y
    if passed:  # never time an incorrect implementation
        result["timing"] = timed(fn, warmup, repeat)
        result["stages"] = {name: timed(f, warmup, repeat) for name, f in stages.items()}
        result["effective_tops"] = meta["mac_operations"] / (result["timing"]["median_ms"] * 1e9)
        result["online_effective_tops"] = meta["mac_operations"] / (
            result["stages"]["online_activation_plus_gemm"]["median_ms"] * 1e9)
    del y, fn, stages


def write_result(path, document) -> None:
    """Exclusive create: experiment evidence is never overwritten."""
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    with path.open("x") as f:
        json.dump(document, f, indent=2, allow_nan=False)
        f.write("\n")
