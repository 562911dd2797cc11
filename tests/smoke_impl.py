"""Smoke check used by __graft_entry__.smoke(): through the C ABI on cuda:0, compared with the
numpy oracle,
  * a tiny dense forward, backward and Adam step (the SIMT kernels), and
  * the attention encoder's kernels at shapes that take the tensor-core paths: MHAttentionScore,
    MHAttentionOut and MHAttentionInsideGradients for 2 sequences x 2 heads of 120 units x 32
    features, and a 1x1 FeedForwardConv of those 240 rows (tcgen05 GEMM)."""
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
    run_smoke_encoder()


def run_smoke_encoder() -> None:
    from nn_in_trading_b200 import Context
    rng = np.random.default_rng(11)
    B, U, H, D, W = 2, 120, 2, 32, 64
    nq = U * 3 * H * D
    qkv = rng.standard_normal(B * nq).astype(np.float32)
    gout = (rng.standard_normal(B * U * H * D) * 0.01).astype(np.float32)
    x = rng.standard_normal(B * U * W).astype(np.float32)
    wc = rng.uniform(-0.12, 0.12, 3 * H * D * (W + 1)).astype(np.float32)
    with Context(0) as ctx:
        hq, hs, ho, hg, hqg = (ctx.buffer(n) for n in (B * nq, B * U * H * U, B * U * H * D, gout.size, B * nq))
        hx, hw, hc = ctx.buffer(x.size), ctx.buffer(wc.size), ctx.buffer(B * U * 3 * H * D)
        for h, a in ((hq, qkv), (hg, gout), (hx, x), (hw, wc)):
            ctx.write(h, a)
        ctx.kernel("MHAttentionScore").args(hq, hs, D, 0).batch(B).run((U, H))
        ctx.kernel("MHAttentionOut").args(hs, hq, ho, D).batch(B).run((U, H))
        ctx.kernel("MHAttentionInsideGradients").args(hq, hqg, hs, hg).batch(B).run((U, H, D))
        ctx.kernel("FeedForwardConv").args(hw, hx, hc, U * W, W, W, 3 * H * D, K.NONE).batch(B).run((U, 3 * H * D, 1))
        got = {k: ctx.read(h) for k, h in (("s", hs), ("o", ho), ("qg", hqg), ("c", hc))}
    for b in range(B):
        q = qkv[b * nq:(b + 1) * nq]
        s = np.zeros(U * H * U, np.float32)
        K.launch("MHAttentionScore", (U, H), None, [q, s, D, 0])
        o = np.zeros(U * H * D, np.float32)
        K.launch("MHAttentionOut", (U, H), None, [s, q, o, D])
        qg = np.zeros(nq, np.float32)
        K.launch("MHAttentionInsideGradients", (U, H, D), None, [q, qg, s, gout[b * U * H * D:(b + 1) * U * H * D]])
        c = np.zeros(U * 3 * H * D, np.float32)
        K.launch("FeedForwardConv", (U, 3 * H * D, 1), None, [wc, x[b * U * W:(b + 1) * U * W], c, U * W, W, W,
                                                              3 * H * D, K.NONE])
        n = U * H * U
        check_close(f"smoke scores {b}", got["s"][b * n:(b + 1) * n], s)
        n = U * H * D
        check_close(f"smoke attention out {b}", got["o"][b * n:(b + 1) * n], o)
        check_close(f"smoke attention gradients {b}", got["qg"][b * nq:(b + 1) * nq], qg)
        n = U * 3 * H * D
        check_close(f"smoke 1x1 convolution {b}", got["c"][b * n:(b + 1) * n], c)
