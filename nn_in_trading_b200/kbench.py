"""Device timing of single library kernels through the C ABI.

    python -m nn_in_trading_b200.kbench [--case NAME ...] [--steps K] [--warmup W]

Each case fills its buffers with seeded data, runs W untimed executions, then times K executions
with CUDA events recorded on the library's own stream, and prints one JSON line: microseconds per
execution, the algorithmic work of one execution (FLOPs and the bytes it must move at least) and
the fraction of the roofline that bounds it.  Denominators: the measured HBM copy bandwidth and
bf16 GEMM rate of this GPU when MEASURED_PEAKS.json is present beside the package (the 3xTF32
tensor-core products count as six bf16 MMAs per fp32 one), and the nominal fp32 FMA rate of the
SIMT cores (148 SMs x 128 lanes x 2 FLOPs at the maximum SM clock).
"""
from __future__ import annotations

import argparse
import json
import os

import numpy as np

from .api import NONE, Context

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def peaks() -> dict:
    p = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "sm_max_mhz": 1965.0, "source": "fallback"}
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            m = json.load(f)
        p.update({k: m[k] for k in ("hbm_gbs", "bf16_tflops", "sm_max_mhz") if k in m})
        p["source"] = "measured"
    p["fp32_simt_tflops"] = 148 * 128 * 2 * p["sm_max_mhz"] * 1e6 / 1e12
    p["tf32x3_tflops"] = p["bf16_tflops"] / 6
    return p


def _flash(B, Q, KV, H, D, mask, grad):
    rng = np.random.default_rng(5)
    q = rng.standard_normal(B * Q * H * D).astype(np.float32)
    kv = rng.standard_normal(B * KV * 2 * H * D).astype(np.float32)
    lse = np.zeros(B * Q * H, np.float32)
    out = np.zeros(B * Q * H * D, np.float32)
    if not grad:
        args = [q, kv, lse, out, D, KV, mask]
        flops = 4.0 * B * H * Q * KV * D
        nbytes = 4.0 * (q.size + kv.size + lse.size + out.size)
        return "MHFlashAttention", args, (Q, D, H), (1, D, 1), B, flops, nbytes, "fp32_simt_tflops"
    g = (rng.standard_normal(q.size) * 0.1).astype(np.float32)
    lse[:] = np.log(KV)
    args = [q, np.zeros_like(q), kv, np.zeros_like(kv), lse, rng.standard_normal(q.size).astype(np.float32) * 0.1,
            g, D, Q, KV, mask]
    flops = 10.0 * B * H * Q * KV * D  # s, g.v, and the three gradient sums of the reference's formula
    nbytes = 4.0 * (4 * q.size + 2 * kv.size + lse.size)
    return "MHFlashAttentionGrad", args, (max(Q, KV), D, H), (1, D, 1), B, flops, nbytes, "fp32_simt_tflops"


def _matmult(rows, dim, cols, var, grad):
    rng = np.random.default_rng(6)
    a = rng.standard_normal(var * rows * dim).astype(np.float32)
    b = rng.standard_normal(var * dim * cols).astype(np.float32)
    r = np.zeros(var * rows * cols, np.float32)
    if not grad:
        args = [a, b, r, dim, 1, 0, 0, 0, np.zeros(1, np.float32), 0]
        return ("MatMult", args, (rows, cols, var), None, 1, 2.0 * var * rows * dim * cols,
                4.0 * (a.size + b.size + r.size), "tf32x3_tflops")
    args = [a, np.zeros_like(a), b, np.zeros_like(b), r + 0.01, dim, 1, 0, 0, 0, 0, 0]
    return ("MatMultGrad", args, (rows, cols, var), None, 1, 4.0 * var * rows * dim * cols,
            4.0 * (2 * a.size + 2 * b.size + r.size), "tf32x3_tflops")


def _conv(kind, units, window, window_out, batch):
    """One 1x1 convolution of the attention encoder (FeedForwardConv, CalcHiddenGradientConv or
    UpdateWeightsConvAdam with step = window) over `batch` sequences of `units` rows."""
    rng = np.random.default_rng(7)
    rows = batch * units
    w = (rng.standard_normal(window_out * (window + 1)) * 0.1).astype(np.float32)
    x = rng.standard_normal(batch * units * window).astype(np.float32)
    y = rng.standard_normal(batch * units * window_out).astype(np.float32)
    in_total, out_total = units * window, units * window_out
    flops = 2.0 * rows * window_out * (window + 1)
    if kind == "ff":
        args = [w, x, np.zeros_like(y), in_total, window, window, window_out, NONE]
        return ("FeedForwardConv", args, (units, window_out, 1), None, batch, flops,
                4.0 * (x.size + y.size + w.size), "tf32x3_tflops")
    if kind == "dgrad":
        args = [w, y, x, np.zeros_like(x), out_total, window, window, window_out, NONE, 0]
        return ("CalcHiddenGradientConv", args, (in_total, 1), None, batch, flops,
                4.0 * (y.size + 2 * x.size + w.size), "tf32x3_tflops")
    m = np.zeros_like(w)
    v = np.zeros_like(w)
    args = [w, y, x, m, v, in_total, 3e-4, 0.9, 0.999, window, window_out, window]
    return ("UpdateWeightsConvAdam", args, ((window + 1) * window_out,), None, batch, flops,
            4.0 * (y.size + x.size + 6 * w.size), "tf32x3_tflops")


CASES = {
    # CCrossMHFlashAttention-shaped self attention: 4 sequences of 512 positions, 8 heads of 64
    "flash_fwd_b4_512x512_h8_d64": lambda: _flash(4, 512, 512, 8, 64, 0, False),
    "flash_grad_b4_512x512_h8_d64": lambda: _flash(4, 512, 512, 8, 64, 0, True),
    # four 4096 x 1024 by 1024 x 1024 products
    "matmult_v4_4096x1024x1024": lambda: _matmult(4096, 1024, 1024, 4, False),
    "matmult_grad_v4_4096x1024x1024": lambda: _matmult(4096, 1024, 1024, 4, True),
    # the attention encoder's 1x1 convolutions at batch 256 (120 bars x 64 features, 8 heads x 32):
    # Q/K/V 64 -> 768 and FF2 256 -> 64
    "conv_ff_qkv_b256": lambda: _conv("ff", 120, 64, 768, 256),
    "conv_dgrad_qkv_b256": lambda: _conv("dgrad", 120, 64, 768, 256),
    "conv_wgrad_adam_qkv_b256": lambda: _conv("wgrad", 120, 64, 768, 256),
    "conv_ff_ff2_b256": lambda: _conv("ff", 120, 256, 64, 256),
    "conv_dgrad_ff2_b256": lambda: _conv("dgrad", 120, 256, 64, 256),
    "conv_wgrad_adam_ff2_b256": lambda: _conv("wgrad", 120, 256, 64, 256),
}


def run_case(ctx, name, steps, warmup, pk):
    import torch

    kernel, args, gsize, lsize, batch, flops, nbytes, peak_key = CASES[name]()
    k = ctx.kernel(kernel)
    handles = []
    for i, a in enumerate(args):
        if isinstance(a, np.ndarray):
            h = ctx.buffer(a.size)
            ctx.write(h, a)
            handles.append(h)
            k.set(i, h)
        else:
            k.set(i, a)
    if batch != 1:
        k.batch(batch)
    stream = torch.cuda.ExternalStream(ctx.stream())
    for _ in range(warmup):
        k.run(gsize, lsize)
    ctx.finish()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for _ in range(steps):
        k.run(gsize, lsize)
    t1.record(stream)
    t1.synchronize()
    us = t0.elapsed_time(t1) * 1e3 / steps
    for h in handles:
        ctx.free(h)
    ctx.lib.nn_kernel_free(k.id)
    tflops = flops / us / 1e6
    gbs = nbytes / us / 1e3
    frac_c = tflops / pk[peak_key]
    frac_m = gbs / pk["hbm_gbs"]
    bound = "compute" if frac_c >= frac_m else "hbm"
    return {"case": name, "kernel": kernel, "us_per_launch": us, "flops": flops, "min_bytes": nbytes,
            "tflops": tflops, "gbs": gbs, "bound": bound, "peak_compute": {peak_key: pk[peak_key]},
            "peak_hbm_gbs": pk["hbm_gbs"], "frac": max(frac_c, frac_m), "peak_source": pk["source"],
            "steps": steps, "warmup": warmup}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--case", action="append", choices=sorted(CASES))
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    a = ap.parse_args(argv)
    pk = peaks()
    ctx = Context(0)
    try:
        for name in a.case or list(CASES):
            print(json.dumps(run_case(ctx, name, a.steps, a.warmup, pk)), flush=True)
    finally:
        ctx.close()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
