"""Smoke check used by __graft_entry__.smoke(): a tiny dense forward, backward and
Adam step through the C ABI on cuda:0, compared with the numpy oracle."""
from __future__ import annotations

import numpy as np

from oracle import kernels as K
from tests.parity import check_close


def run_smoke() -> None:
    from nn_in_trading_b200 import Context
    rng = np.random.default_rng(7)
    n_in, n_out = 24, 9
    w = rng.uniform(-0.2, 0.2, n_out * (n_in + 1)).astype(np.float32)
    x = rng.standard_normal(n_in).astype(np.float32)
    t = rng.uniform(0, 1, n_out).astype(np.float32)
    with Context(0) as ctx:
        hw, hx, hy, hg, hm, hv, hxg = (ctx.buffer(n) for n in (w.size, n_in, n_out, n_out, w.size, w.size, n_in))
        ctx.write(hw, w)
        ctx.write(hx, x)
        loc = (n_in + 3) // 4
        ctx.kernel("FeedForward").args(hw, hx, hy, n_in, K.SIGMOID, hy, 0).run((n_out, loc), (1, loc))
        ht = ctx.buffer(n_out)
        ctx.write(ht, t)
        ctx.kernel("CalcOutputGradient").args(ht, hy, hg, K.SIGMOID, 1.0).run((n_out,))
        ctx.kernel("CalcHiddenGradient").args(hw, hg, hx, hxg, n_out, K.NONE).run((n_in, 3), (1, 3))
        ctx.kernel("UpdateWeightsAdam").args(hw, hg, hx, hm, hv, n_in, 3e-4, 0.9, 0.999).run((n_out, n_in + 1))
        ctx.kernel("NormalizeWeights").args(hw, n_in + 1).run((n_out,))
        got = {k: ctx.read(h) for k, h in (("y", hy), ("g", hg), ("xg", hxg), ("w", hw), ("m", hm), ("v", hv))}
    y = np.zeros(n_out, np.float32)
    K.FeedForward(w, x, y, n_in, K.SIGMOID, y, 0, gsize=(n_out, 1))
    g = np.zeros(n_out, np.float32)
    K.CalcOutputGradient(t, y, g, K.SIGMOID, 1.0, gsize=(n_out,))
    xg = np.zeros(n_in, np.float32)
    K.CalcHiddenGradient(w, g, x, xg, n_out, K.NONE, gsize=(n_in, 3))
    w0 = w.copy()
    m = np.zeros_like(w)
    v = np.zeros_like(w)
    K.UpdateWeightsAdam(w, g, x, m, v, n_in, 3e-4, 0.9, 0.999, gsize=(n_out, n_in + 1))
    K.NormalizeWeights(w, n_in + 1, gsize=(n_out,))
    check_close("smoke output", got["y"], y)
    check_close("smoke output gradient", got["g"], g)
    check_close("smoke input gradient", got["xg"], xg)
    check_close("smoke weights", got["w"][:w.size], w, w0)
    check_close("smoke m", got["m"][:w.size], m)
    check_close("smoke v", got["v"][:w.size], v)
