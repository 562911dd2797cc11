"""ORACLE TEST INFRASTRUCTURE -- numpy restatement of the NeuroNet.cl kernels.

This module is the checker, never the product: only tests/, the golden-vector
generator, __graft_entry__.smoke() and the CPU-baseline leg of bench.py may
use it.  Each function restates one reference kernel of
Experts/NeuroNet_DNG/NeuroNet.cl (cited per function) with the same
positional arguments and the same NDRange meaning (`gsize`/`lsize` are the
global and local work sizes the MQL5 host enqueues), operating in place on
float32 numpy arrays.  Sums are reassociated (vectorised) where the
reference sums serially; parity with the reference is therefore
tolerance-based, and the restatement is pinned against the reference kernels
themselves (oracle/_ref, compiled from the reference source) through the
golden vectors in tests/golden/.
"""
from __future__ import annotations

import numpy as np

F32 = np.float32
L1 = F32(1.0e-4)            # NeuroNet.cl:15
L2 = F32(1.0e-4)            # NeuroNet.cl:16
MAX_GRAD = F32(1.0e-2)      # NeuroNet.cl:17
LOCAL_ARRAY_SIZE = 64       # NeuroNet.cl:18
MAX_VALUE = F32(3.4e37)     # NeuroNet.cl:20
MIN_VALUE = F32(-3.4e37)    # NeuroNet.cl:21

# ENUM_ACTIVATION, NeuroNet.cl:32-39 / NeuroNet_Definitions.mqh:3650-3669
NONE, TANH, SIGMOID, LRELU, SOFTPLUS, GELU, MINUS_SOFTPLUS, ELU = -1, 0, 1, 2, 3, 4, 5, 6
# ENUM_OPTIMIZATION, NeuroNet_Definitions.mqh:3671-3685
SGD, ADAM, LS, ADAM_MINI = 0, 1, 2, 3


def _err():
    return np.errstate(all="ignore")


def nan0(x, default=0.0):
    """IsNaNOrInf (NeuroNet.cl:53-61): non-finite -> default."""
    x = np.asarray(x, dtype=F32)
    return np.where(np.isfinite(x), x, F32(default)).astype(F32)


def cl_clamp(x, lo, hi):
    """OpenCL clamp as min(max(x, lo), hi) with IEEE fmin/fmax (NaN -> lo)."""
    return np.fmin(np.fmax(np.asarray(x, dtype=F32), F32(lo)), F32(hi)).astype(F32)


def cl_sign(x):
    x = np.asarray(x, dtype=F32)
    return np.where(np.isnan(x), F32(0), np.sign(x)).astype(F32)


def f_activation(value, act):
    """fActivation, NeuroNet.cl:88-125."""
    with _err():
        r = nan0(value)
        if act == TANH:
            r = np.tanh(cl_clamp(r, -20.0, 20.0))
        elif act == SIGMOID:
            r = F32(1) / (F32(1) + np.exp(cl_clamp(-r, -20.0, 20.0)))
        elif act == LRELU:
            r = np.where(r < 0, r * F32(0.01), r)
        elif act == SOFTPLUS:
            r = np.where(r >= F32(20), r, nan0(np.log(F32(1) + np.exp(r))))
        elif act == GELU:
            r = r / (F32(1) + np.exp(cl_clamp(F32(-1.702) * r, -20.0, 20.0)))
        elif act == MINUS_SOFTPLUS:
            r = -f_activation(r, SOFTPLUS)
        elif act == ELU:
            r = np.where(r < 0, nan0(np.exp(r)) - F32(1), r)
        return nan0(r)


def deactivation(grad, inp, act):
    """Deactivation, NeuroNet.cl:129-174 (derivative from the activation *output*)."""
    with _err():
        grad = np.asarray(grad, dtype=F32)
        inp = np.asarray(inp, dtype=F32)
        r = nan0(grad)
        if act == TANH:
            r = (cl_clamp(grad + inp, -1.0, 1.0) - inp) * (F32(1) - inp * inp)
        elif act == SIGMOID:
            r = (cl_clamp(grad + inp, 0.0, 1.0) - inp) * (inp * (F32(1) - inp))
        elif act == LRELU:
            r = np.where(inp < 0, r * F32(0.01), r)
        elif act == SOFTPLUS:
            r = r * (F32(1) - np.exp(-inp))
        elif act == GELU:
            r = np.where(inp < F32(0.9), r * f_activation(F32(5) * inp, SIGMOID), r)
        elif act == MINUS_SOFTPLUS:
            r = deactivation(-r, -inp, SOFTPLUS)
            return r
        elif act == ELU:
            r = np.where(inp < 0, r * (inp + F32(1)), r)
        r = np.where(np.isfinite(inp), r, F32(0))
        return cl_clamp(nan0(r), -MAX_GRAD, MAX_GRAD)


# --------------------------------------------------------------------- dense
def FeedForward(matrix_w, matrix_i, matrix_o, inputs, activation, numeric_flags, flags_enabled,
                gsize, lsize=None):
    """NeuroNet.cl:430-512.  o[i] = act(sum_k w[i,k] x[k] + w[i,inputs]); rows of (inputs+1)."""
    total_out = gsize[0]
    with _err():
        w = matrix_w[:total_out * (inputs + 1)].reshape(total_out, inputs + 1)
        x = matrix_i[:inputs]
        xs = nan0(x)
        prod = nan0(xs[None, :] * w[:, :inputs])
        s = prod.sum(axis=1, dtype=F32) + nan0(w[:, inputs])
        y = f_activation(s, activation)
        if flags_enabled:
            bad = (~np.isfinite(x)[None, :] | ~np.isfinite(w[:, :inputs])
                   | ~np.isfinite(x[None, :] * w[:, :inputs])).any(axis=1)
            bad |= ~np.isfinite(w[:, inputs]) | ~np.isfinite(s) | ~np.isfinite(y)
            numeric_flags[:total_out] = bad.astype(F32)
        matrix_o[:total_out] = y


def CalcOutputGradient(matrix_t, matrix_o, matrix_ig, activation, error, gsize, lsize=None):
    """NeuroNet.cl:523-536.  ig = Deactivation(t - o, o, act) (the `error` argument is unused)."""
    n = gsize[0]
    with _err():
        o = matrix_o[:n]
        g = deactivation(matrix_t[:n] - o, o, activation)
        matrix_ig[:n] = np.where(np.isfinite(o), g, F32(0))


def CalcHiddenGradient(matrix_w, matrix_g, matrix_o, matrix_ig, outputs, activation, gsize, lsize=None):
    """NeuroNet.cl:547-613.  ig[i] = Deactivation(sum_k w[k,i] g[k], o[i], act)."""
    inputs = gsize[0]
    with _err():
        w = nan0(matrix_w[:outputs * (inputs + 1)].reshape(outputs, inputs + 1)[:, :inputs])
        g = nan0(matrix_g[:outputs])
        s = (w * g[:, None]).sum(axis=0, dtype=F32)
        matrix_ig[:inputs] = deactivation(s, matrix_o[:inputs], activation)


def UpdateWeightsMomentum(matrix_w, matrix_g, matrix_i, matrix_dw, inputs, learning_rates, momentum,
                          gsize, lsize=None):
    """NeuroNet.cl:624-645.  SGD with momentum; gradient clamped to +-MAX_GRAD per output."""
    n_out, n_col = gsize[0], gsize[1]
    with _err():
        idx = (np.arange(n_out)[:, None] * (inputs + 1) + np.arange(n_col)[None, :])
        grad = cl_clamp(matrix_g[:n_out], -MAX_GRAD, MAX_GRAD)[:, None]
        xj = np.where(np.arange(n_col) < inputs, matrix_i[np.minimum(np.arange(n_col), inputs - 1)], F32(1))
        delta = nan0(F32(learning_rates) * grad * xj[None, :]) + nan0(F32(momentum) * matrix_dw[idx])
        matrix_dw[idx] = delta
        w = matrix_w[idx]
        matrix_w[idx] = np.where(np.abs(delta) > 0, nan0(w + delta), w)


def adam_dense_apply(matrix_w, grad, matrix_m, matrix_v, inputs, l, b1, b2, n_out, n_col):
    """Adam arithmetic of UpdateWeightsAdam (NeuroNet.cl:678-693) given the pre-clamp gradient
    grad[i, j] (i < n_out, j < n_col) of the weight at row i, column j of a (inputs+1)-wide matrix."""
    with _err():
        idx = (np.arange(n_out)[:, None] * (inputs + 1) + np.arange(n_col)[None, :])
        weight = nan0(matrix_w[idx])
        m = nan0(matrix_m[idx])
        v = nan0(matrix_v[idx])
        g = cl_clamp(nan0(grad), -MAX_GRAD, MAX_GRAD)
        b1, b2, l = F32(b1), F32(b2), F32(l)
        mt = nan0(b1 * m + (F32(1) - b1) * g)
        vt = nan0(b2 * v + (F32(1) - b2) * (g * g))
        delta = nan0(l * (mt / (np.sqrt(vt) + F32(1e-37)) - (L1 * cl_sign(weight) + L2 * weight)))
        w = matrix_w[idx]
        matrix_w[idx] = np.where(np.abs(delta) > 0, nan0(w + delta), w)
        matrix_m[idx] = mt
        matrix_v[idx] = vt


def UpdateWeightsAdam(matrix_w, matrix_g, matrix_i, matrix_m, matrix_v, inputs, l, b1, b2, gsize, lsize=None):
    """NeuroNet.cl:657-694.  g = clamp(g_o * x_j); Adam with eps 1e-37 outside the root, l1/l2 decay."""
    n_out, n_col = gsize[0], gsize[1]
    with _err():
        j = np.arange(n_col)
        inp = nan0(np.where(j == inputs, F32(1), matrix_i[np.minimum(j, max(inputs - 1, 0))]))
        grad = nan0(matrix_g[:n_out][:, None] * inp[None, :])
    adam_dense_apply(matrix_w, grad, matrix_m, matrix_v, inputs, l, b1, b2, n_out, n_col)


def NormalizeWeights(buffer, dimension, gsize, lsize=None):
    """NeuroNet.cl:1498-1525.  Each row of `dimension` values is rescaled to unit L2 norm if its norm > 1;
    a row whose sum of squares overflows is retried with the values pre-divided by 10, 100, ..."""
    rows = gsize[0]
    with _err():
        b = buffer[:rows * dimension].reshape(rows, dimension)
        x = nan0(b)
        k = np.ones(rows, F32)
        s = (x ** 2).sum(axis=1, dtype=F32)
        for r in np.nonzero(~np.isfinite(s))[0]:
            while True:
                k[r] = F32(k[r] * 10)
                s[r] = ((x[r] / k[r]) ** 2).sum(dtype=F32)
                if np.isfinite(s[r]):
                    break
        d = k * np.sqrt(s)
        out = np.where((d > 1)[:, None], x / d[:, None], b)
        buffer[:rows * dimension] = out.reshape(-1)


# ---------------------------------------------------------------------- conv
def FeedForwardConv(matrix_w, matrix_i, matrix_o, inputs, step, window_in, window_out, activation,
                    gsize, lsize=None):
    """NeuroNet.cl:887-932.  Strided 1-D conv per variable; w[v][window_out][window_in+1] with bias last."""
    units = gsize[0]
    wout = gsize[1]
    var = gsize[2] if len(gsize) > 2 else 1
    with _err():
        for v in range(var):
            w = matrix_w[v * window_out * (window_in + 1):(v + 1) * window_out * (window_in + 1)]
            w = w.reshape(window_out, window_in + 1)
            x = nan0(matrix_i[v * inputs:(v + 1) * inputs])
            out = np.empty((units, wout), dtype=F32)
            for i in range(units):
                si = step * i
                stop = min(window_in, inputs - si)
                acc = np.zeros(wout, dtype=F32)
                if stop > 0:
                    acc = nan0(x[si:si + stop][None, :] * w[:wout, :stop]).sum(axis=1, dtype=F32)
                acc = acc + nan0(w[:wout, window_in])
                out[i] = acc
            base = v * window_out * units
            o = matrix_o[base:base + units * window_out].reshape(units, window_out)
            o[:, :wout] = f_activation(out, activation)


def CalcHiddenGradientConv(matrix_w, matrix_g, matrix_o, matrix_ig, outputs, step, window_in, window_out,
                           activation, shift_out, gsize, lsize=None):
    """NeuroNet.cl:941-986.  Input gradient of FeedForwardConv (overlap-add over windows) + Deactivation."""
    inputs = gsize[0]
    var = gsize[1] if len(gsize) > 1 else 1
    n_win = outputs // window_out
    with _err():
        for v in range(var):
            w = matrix_w[v * window_out * (window_in + 1):(v + 1) * window_out * (window_in + 1)]
            w = w.reshape(window_out, window_in + 1)
            g = nan0(matrix_g[shift_out + v * outputs: shift_out + v * outputs + n_win * window_out])
            g = g.reshape(n_win, window_out)
            s = np.zeros(inputs, dtype=F32)
            for k in range(n_win):
                lo = k * step
                if lo >= inputs:
                    break
                hi = min(lo + window_in, inputs)
                # contribution of window k to positions lo..hi-1
                s[lo:hi] += nan0(g[k][:, None] * w[:, :hi - lo]).sum(axis=0, dtype=F32)
            o = matrix_o[v * inputs:(v + 1) * inputs]
            matrix_ig[v * inputs:(v + 1) * inputs] = deactivation(s, o, activation)


def _conv_weight_grad_dense(matrix_g, matrix_i, inputs, window_in, window_out, step, n_weights):
    """The Adam variant of conv_weight_grad as one contraction, when nothing in it needs the loop: whole
    variables of weights, every product index inside the arrays, no window cut short by the stop test,
    finite operands and sums.  grad[v][o][s] = sum_t g[v][t][o] x[v*inputs + t*step + s] (s < window_in)
    and grad[v][o][window_in] = sum_t g[v][t][o]; the sums are taken in float64 and rounded once (the
    reference's serial float32 order agrees to the tolerance the golden cases pin).  None otherwise."""
    W1 = window_in + 1
    per_var = W1 * window_out
    total = (inputs - (window_in - step) + (step - 1)) // step
    if n_weights % per_var or total <= 0 or step <= 0 or total * window_in > inputs:
        return None
    V = n_weights // per_var
    if V * total * window_out > matrix_g.size or (V - 1) * inputs + (total - 1) * step + window_in > matrix_i.size:
        return None
    g = matrix_g[:V * total * window_out].reshape(V, total, window_out).astype(np.float64)
    t_idx = (np.arange(V)[:, None, None] * inputs + np.arange(total)[None, :, None] * step
             + np.arange(window_in)[None, None, :])
    x = matrix_i[t_idx].astype(np.float64)
    if not (np.isfinite(g).all() and np.isfinite(x).all()):
        return None
    out = np.empty((V, window_out, W1), np.float64)
    out[:, :, :window_in] = np.einsum("vto,vts->vos", g, x)
    out[:, :, window_in] = g.sum(axis=1)
    out = out.astype(F32).reshape(-1)
    return out if np.isfinite(out).all() else None


def conv_weight_grad(matrix_g, matrix_i, inputs, window_in, window_out, step, n_weights, momentum_variant=False):
    """Per-weight gradient loops of UpdateWeightsConvAdam (NeuroNet.cl:1073-1081) and
    UpdateWeightsConvMomentum (NeuroNet.cl:1016-1031), including their index quirks:
    Adam uses total = (inputs-(window_in-step)+(step-1))/step and shift_out = i/(window_in+1)-v*window_out;
    Momentum uses total = (inputs-window_in+step-1)/step and shift_out = i/(window_in+1)-v;
    both stop at the first t with shift + t*window_in >= inputs (window_in, not step)."""
    fast = None if momentum_variant else _conv_weight_grad_dense(matrix_g, matrix_i, inputs, window_in, window_out,
                                                                 step, n_weights)
    if fast is not None:
        return fast
    i = np.arange(n_weights)
    v = i // ((window_in + 1) * window_out)
    shift = i % (window_in + 1)
    if momentum_variant:
        shift_out = i // (window_in + 1) - v
        total = (inputs - window_in + step - 1) // step
    else:
        shift_out = i // (window_in + 1) - v * window_out
        total = (inputs - (window_in - step) + (step - 1)) // step
    grad = np.zeros(n_weights, dtype=F32)
    with _err():
        alive = np.ones(n_weights, dtype=bool)
        for t in range(max(total, 0)):
            alive &= ~((shift != window_in) & (shift + t * window_in >= inputs))
            if not alive.any():
                break
            gi = t * window_out + shift_out + v * total * window_out
            xi = np.where(shift == window_in, 0, shift + t * step + v * inputs)
            gv = matrix_g[np.clip(gi, 0, matrix_g.size - 1)]
            xv = np.where(shift == window_in, F32(1), matrix_i[np.clip(xi, 0, matrix_i.size - 1)])
            grad = np.where(alive, grad + nan0(gv * xv), grad).astype(F32)
    return grad


def UpdateWeightsConvMomentum(matrix_w, matrix_g, matrix_i, matrix_dw, inputs, learning_rates, momentum,
                              window_in, window_out, step, gsize, lsize=None):
    """NeuroNet.cl:996-1043."""
    n = gsize[0]
    grad = conv_weight_grad(matrix_g, matrix_i, inputs, window_in, window_out, step, n, momentum_variant=True)
    with _err():
        delta = nan0(F32(learning_rates) * grad) + F32(momentum) * matrix_dw[:n]
        ok = ~np.isnan(delta)
        w = matrix_w[:n]
        matrix_dw[:n] = np.where(ok, delta, matrix_dw[:n])
        matrix_w[:n] = np.where(ok & (np.abs(delta) > 0), nan0(w + delta), w)


def adam_conv_apply(matrix_w, grad, matrix_m, matrix_v, l, b1, b2, n):
    """Adam arithmetic of UpdateWeightsConvAdam (NeuroNet.cl:1082-1097): no eps, no l1/l2, vt NaN -> 1."""
    with _err():
        b1, b2, l = F32(b1), F32(b2), F32(l)
        g = cl_clamp(nan0(grad), -MAX_GRAD, MAX_GRAD)
        mt = nan0(b1 * matrix_m[:n] + (F32(1) - b1) * g)
        vt = nan0(b2 * matrix_v[:n] + (F32(1) - b2) * (g * g), 1.0)
        weight = nan0(matrix_w[:n] + nan0(l * mt / np.sqrt(vt)))
        matrix_w[:n] = weight
        matrix_m[:n] = mt
        matrix_v[:n] = vt


def UpdateWeightsConvAdam(matrix_w, matrix_g, matrix_i, matrix_m, matrix_v, inputs, l, b1, b2,
                          window_in, window_out, step, gsize, lsize=None):
    """NeuroNet.cl:1053-1098."""
    n = gsize[0]
    grad = conv_weight_grad(matrix_g, matrix_i, inputs, window_in, window_out, step, n)
    adam_conv_apply(matrix_w, grad, matrix_m, matrix_v, l, b1, b2, n)


# ---------------------------------------------------------- residual / norm
def SumMatrix(matrix1, matrix2, matrix_out, dimension, multiplyer, shift_in1, shift_in2, shift_out,
              numeric_flags, flags_enabled, gsize, lsize=None):
    """NeuroNet.cl:1314-1347.  out = (a + b) * multiplyer, row i offset by i*shift_*."""
    rows = gsize[0]
    with _err():
        r = np.arange(rows)[:, None]
        index = r * dimension + np.arange(dimension)[None, :]
        a = matrix1[r * shift_in1 + index]
        b = matrix2[r * shift_in2 + index]
        raw = (a + b) * F32(multiplyer)
        if flags_enabled:
            bad = ~np.isfinite(a) | ~np.isfinite(b) | ~np.isfinite(a + b) | ~np.isfinite(raw)
            numeric_flags[index] = bad.astype(F32)
        matrix_out[r * shift_out + index] = nan0(raw)


def Normalize(buffer, dimension, gsize, lsize=None):
    """NeuroNet.cl:1455-1486.  Row centring; divide by the (unbiased) *variance* only when it exceeds 1."""
    rows = gsize[0]
    if dimension < 1:
        return
    with _err():
        b = buffer[:rows * dimension].reshape(rows, dimension)
        x = nan0(b)
        mean = x.mean(axis=1, dtype=np.float64).astype(F32)
        var = (((x - mean[:, None]).astype(np.float64) ** 2).sum(axis=1) / (dimension - 1)).astype(F32) \
            if dimension > 1 else np.full(rows, np.nan, F32)
        c = b - mean[:, None]
        out = np.where((var > 1)[:, None], c / var[:, None], c)
        buffer[:rows * dimension] = nan0(out).reshape(-1)


# ----------------------------------------------------------------- attention
def MHAttentionScore(qkv, score, dimension, mask, gsize, lsize=None):
    """NeuroNet.cl:1662-1719.  S[q,h,k] = exp(clamp(q.k/sqrt(d), +-100)), divided by the row sum only
    when that sum exceeds 1 (no max subtraction); qkv is [unit][3][head][dimension]."""
    units, heads = gsize[0], gsize[1]
    koef = max(np.sqrt(F32(dimension)), F32(1))
    with _err():
        t = qkv[:units * 3 * heads * dimension].reshape(units, 3, heads, dimension)
        q = nan0(t[:, 0])
        k = nan0(t[:, 1])
        r = np.einsum("qhd,khd->qhk", q, k).astype(F32)
        s = np.exp(cl_clamp(r / koef, -100.0, 100.0))
        s = np.where(np.isnan(s), F32(0), s)
        if mask > 0:
            keep = np.arange(units)[None, None, :] <= np.arange(units)[:, None, None]
            s = np.where(keep, s, F32(0))
        tot = s.sum(axis=2, dtype=F32)
        s = np.where((tot > 1)[:, :, None], s / tot[:, :, None], s)
        score[:units * heads * units] = s.reshape(-1)


def MHAttentionOut(scores, qkv, out, dimension, gsize, lsize=None):
    """NeuroNet.cl:1730-1759.  O[u,h,:] = sum_v S[u,h,v] V[v,h,:]."""
    units, heads = gsize[0], gsize[1]
    with _err():
        s = scores[:units * heads * units].reshape(units, heads, units)
        v = qkv[:units * 3 * heads * dimension].reshape(units, 3, heads, dimension)[:, 2]
        out[:units * heads * dimension] = np.einsum("uhv,vhd->uhd", s, v).astype(F32).reshape(-1)


def MHAttentionInsideGradients(qkv, qkv_g, scores, gradient, gsize, lsize=None):
    """NeuroNet.cl:1777-1845.  dV = S^T g;  dQ[u,:,d] = g[u,d]/sqrt(d) sum_k S[u,k](V0[k]-A[u]) K[k,d];
    dK[u,:,d] = sum_q g[q,d]/sqrt(d) S[q,u](V0[u]-A[q]) Q[q,d];  A[q] = sum_v S[q,v] V0[v].
    V0 is feature 0 of V: the reference reads V at qkv[dimension*(heads*(3v+2)+h)] without +d
    (NeuroNet.cl:1822, 1840).  The reference's triple loop sum_v S_v V0_v g (d_kv - S_k) is evaluated in
    the algebraically equal factorised form g S_k (V0_k - A)."""
    units, heads, dim = gsize[0], gsize[1], gsize[2]
    koef = max(np.sqrt(F32(dim)), F32(1))
    with _err():
        t = qkv[:units * 3 * heads * dim].reshape(units, 3, heads, dim)
        Q, K, V = t[:, 0], t[:, 1], t[:, 2]
        S = scores[:units * heads * units].reshape(units, heads, units)
        G = gradient[:units * heads * dim].reshape(units, heads, dim)
        V0 = V[:, :, 0]                                         # [v, h]
        A = np.einsum("uhv,vh->uh", S, V0).astype(F32)          # [u, h]
        C = S * (V0.T[None, :, :] - A[:, :, None])              # [u, h, k]
        dV = np.einsum("ihu,ihd->uhd", S, G).astype(F32)
        dQ = (G * np.einsum("uhk,khd->uhd", C, K)) / koef
        dK = np.einsum("qhu,qhd->uhd", C, G * Q) / koef
        g = np.stack([dQ, dK, dV], axis=1).astype(F32)
        qkv_g[:units * 3 * heads * dim] = g.reshape(-1)


# ------------------------------------------------------------------- softmax
def _softmax_rows(x):
    with _err():
        x = nan0(x, MIN_VALUE)
        mx = x.max(axis=-1, keepdims=True)
        e = np.where(x == MIN_VALUE, F32(0), nan0(np.exp(x - mx)))
        s = e.sum(axis=-1, keepdims=True, dtype=F32)
        y = np.where(s == 0, F32(0), nan0(e / s))
        return np.where(mx == MIN_VALUE, F32(0), y).astype(F32)


def SoftMax_FeedForward(inputs, outputs, gsize, lsize):
    """NeuroNet.cl:2479-2492 (LocalSoftMax, NeuroNet.cl:392-408): max-subtracted softmax per head row of
    length local_size(0)."""
    size, heads = lsize[0], gsize[1] if len(gsize) > 1 else 1
    outputs[:size * heads] = _softmax_rows(inputs[:size * heads].reshape(heads, size)).reshape(-1)


def SoftMax_HiddenGradient(outputs, output_gr, input_gr, gsize, lsize):
    """NeuroNet.cl:2496-2510 (LocalSoftMaxGrad, NeuroNet.cl:412-420): y (g - sum y g)."""
    size, heads = lsize[0], gsize[1] if len(gsize) > 1 else 1
    with _err():
        y = nan0(outputs[:size * heads].reshape(heads, size))
        g = nan0(output_gr[:size * heads].reshape(heads, size))
        s = nan0((y * g).sum(axis=1, keepdims=True, dtype=F32))
        input_gr[:size * heads] = nan0(y * (g - s)).reshape(-1)


def SoftMax_OutputGradient(outputs, targets, output_gr, gsize, lsize=None):
    """NeuroNet.cl:2514-2520.  g = t / y (0 where y == 0)."""
    n = gsize[0]
    with _err():
        y = outputs[:n]
        output_gr[:n] = np.where(y == 0, F32(0), targets[:n] / y)


# -------------------------------------------------------------- elementwise
def Activation(inputs, outputs, activation, gsize, lsize=None):
    """NeuroNet.cl:5796-5808."""
    n = gsize[0]
    outputs[:n] = f_activation(nan0(inputs[:n]), activation)


def DeActivation(inputs, inputs_gr, output_gr, activation, gsize, lsize=None):
    """NeuroNet.cl:5811-5823."""
    n = gsize[0]
    inputs_gr[:n] = deactivation(nan0(output_gr[:n]), inputs[:n], activation)


def SoftUpdate(target, source, tau, gsize, lsize=None):
    """NeuroNet.cl:3864-3871.  Polyak averaging."""
    n = gsize[0]
    with _err():
        tau = F32(tau)
        target[:n] = source[:n] * tau + (F32(1) - tau) * target[:n]


def SoftUpdateAdam(target, source, matrix_m, matrix_v, tau, b1, b2, gsize, lsize=None):
    """NeuroNet.cl:3875-3899.  Adam-style soft update on g = source - target, step (1-tau) m/sqrt(v)."""
    n = gsize[0]
    with _err():
        b1, b2, tau = F32(b1), F32(b2), F32(tau)
        w = target[:n].copy()
        g = source[:n] - w
        m = b1 * matrix_m[:n] + (F32(1) - b1) * g
        v = b2 * matrix_v[:n] + (F32(1) - b2) * (g * g)
        delta = (F32(1) - tau) * m / np.where(v != 0, np.sqrt(v), F32(1))
        target[:n] = np.where(np.abs(delta) > 0, w + delta, w)
        matrix_m[:n] = m
        matrix_v[:n] = v


def Transpose(matrix_in, matrix_out, gsize, lsize=None):
    """NeuroNet.cl:4237-4248."""
    rows, cols = gsize[0], gsize[1]
    matrix_out[:rows * cols] = matrix_in[:rows * cols].reshape(rows, cols).T.reshape(-1)


def ConcatenateBuffers(input1, window1, input2, window2, input3, window3, input4, window4, output,
                       gsize, lsize=None):
    """NeuroNet.cl:1538-1576."""
    n = gsize[0]
    tot = window1 + window2 + window3 + window4
    o = output[:n * tot].reshape(n, tot)
    off = 0
    for src, w in ((input1, window1), (input2, window2), (input3, window3), (input4, window4)):
        if w > 0:
            o[:, off:off + w] = nan0(src[:n * w].reshape(n, w))
        off += w


def DeconcatenateBuffers(output1, window1, output2, window2, output3, window3, output4, window4, inputs,
                         gsize, lsize=None):
    """NeuroNet.cl:1601-1650."""
    n = gsize[0]
    tot = window1 + window2 + window3 + window4
    x = inputs[:n * tot].reshape(n, tot)
    off = 0
    for dst, w in ((output1, window1), (output2, window2), (output3, window3), (output4, window4)):
        if w > 0:
            dst[:n * w] = nan0(x[:, off:off + w]).reshape(-1)
        off += w


def RevInFeedForward(inputs, options, output, options_size, optimization, gsize, lsize=None):
    """NeuroNet.cl:5742-5764.  y = sqrt(var) (x - beta) / max(gamma, 1e-3) + mean with BatchNorm options."""
    n = gsize[0]
    with _err():
        shift = (np.arange(n) * (7 if optimization == 0 else 9)) % options_size
        mean, var, k, beta = options[shift], options[shift + 1], options[shift + 3], options[shift + 4]
        res = np.sqrt(var) * (inputs[:n] - beta) / np.fmax(k, F32(0.001)) + mean
        output[:n] = np.where(np.isnan(res), F32(0), res)


def RevInHiddenGraddient(inputs, inputs_gr, options, output_gr, options_size, optimization, activation,
                         gsize, lsize=None):
    """NeuroNet.cl:5767-5793."""
    n = gsize[0]
    with _err():
        shift = (np.arange(n) * (7 if optimization == 0 else 9)) % options_size
        var, k = options[shift + 1], options[shift + 3]
        res = np.sqrt(var) * output_gr[:n]
        res = np.where(np.abs(k) > 1, res / k, res)
        res = np.where(np.isnan(res), F32(0), res)
        inputs_gr[:n] = deactivation(res, inputs[:n], activation)


# ---------------------------------------------------------------- batch norm
def BatchFeedForward(inputs, options, output, batch, optimization, activation, training, gsize, lsize=None):
    """NeuroNet.cl:1900-1953.  Online running mean/variance over the last `batch` calls, gamma/beta, activation.
    With batch <= 1 in training the kernel returns without writing the output."""
    n = gsize[0]
    w = 7 if optimization == 0 else 9
    with _err():
        o = options[:n * w].reshape(n, w)
        inp = nan0(inputs[:n])
        if training == 0:
            mean = nan0(o[:, 0])
            var = nan0(o[:, 1], 1.0)
            var = np.where(var <= 0, F32(1), var)
            gamma = nan0(o[:, 3], 1.0)
            gamma = np.where(gamma == 0, F32(1), gamma)
            beta = nan0(o[:, 4])
            nx = (inp - mean) / np.sqrt(var)
            output[:n] = f_activation(gamma * nx + beta, activation)
            return
        if batch <= 1:
            return
        fb = F32(batch)
        mean = (nan0(o[:, 0]) * max(fb - F32(1), F32(0)) + inp) / max(fb, F32(1))
        delt = inp - mean
        var = (nan0(o[:, 1] * max(fb - F32(1), F32(0))) + delt * delt) / max(fb, F32(1))
        var = np.where(var <= 0, F32(1), var).astype(F32)
        nx = delt / np.sqrt(var)
        gamma = nan0(o[:, 3], 1.0)
        o[:, 3] = np.where(gamma == 0, F32(1), o[:, 3])
        gamma = np.where(gamma == 0, F32(1), gamma)
        beta = nan0(o[:, 4])
        o[:, 0], o[:, 1], o[:, 2] = mean, var, nx
        output[:n] = f_activation(gamma * nx + beta, activation)


def CalcHiddenGradientBatch(options, matrix_g, matrix_i, matrix_ig, activation, batch, optimization, gsize,
                            lsize=None):
    """NeuroNet.cl:1964-1998 (its gvar term multiplies the stored mean by the input, as written)."""
    if batch <= 1:
        return
    n = gsize[0]
    w = 7 if optimization == 0 else 9
    with _err():
        o = options[:n * w].reshape(n, w)
        var = nan0(o[:, 1], 1.0)
        inp = nan0(matrix_i[:n])
        gnx = nan0(matrix_g[:n]) * nan0(o[:, 3], 1.0)
        temp = np.where(var > 0, F32(1) / np.sqrt(var), F32(0))
        gmu = -temp * gnx
        gvar = np.where(var > 0, (nan0(o[:, 0]) * inp) / (F32(2) * np.power(var, F32(1.5))) * gnx, F32(0))
        ratio = F32(max(batch - 1, 0)) / F32(max(batch, 1))
        bd = F32(max(batch, 1))
        gx = temp * gnx + gmu / bd + gvar * F32(2) * inp / bd * ratio * ratio
        matrix_ig[:n] = deactivation(gx, inp, activation)


def bn_adam_apply(options, G_gamma, G_beta, l, b1, b2, n):
    """UpdateBatchOptionsAdam arithmetic (NeuroNet.cl:2061-2097) given the gamma/beta gradients; the beta
    step copies the gamma step (delta.s1 = IsNaNOrInf(delta.s0))."""
    with _err():
        o = options[:n * 9].reshape(n, 9)
        b1, b2, l = F32(b1), F32(b2), F32(l)
        gamma = nan0(o[:, 3], 1.0)
        gamma = np.where(gamma == 0, F32(1), gamma)
        beta = nan0(o[:, 4])
        mg = b1 * nan0(o[:, 5]) + (F32(1) - b1) * G_gamma
        mb = b1 * nan0(o[:, 6]) + (F32(1) - b1) * G_beta
        vg = nan0(b2 * nan0(o[:, 7]) + (F32(1) - b2) * (G_gamma * G_gamma), 1.0)
        vb = nan0(b2 * nan0(o[:, 8]) + (F32(1) - b2) * (G_beta * G_beta), 1.0)
        dg = nan0(l * mg / np.sqrt(vg))
        db = dg
        wg = dg - (L1 * cl_sign(gamma) + L2 * gamma / F32(n))
        wb = db - (L1 * cl_sign(beta) + L2 * beta / F32(n))
        o[:, 3] = nan0(gamma + wg, 1.0)
        o[:, 4] = nan0(beta + wb)
        o[:, 5] = nan0(mg)
        o[:, 6] = nan0(mb)
        o[:, 7] = vg
        o[:, 8] = vb


def UpdateBatchOptionsAdam(options, matrix_g, l, b1, b2, gsize, lsize=None):
    """NeuroNet.cl:2050-2098."""
    n = gsize[0]
    with _err():
        grad = cl_clamp(nan0(matrix_g[:n]), -MAX_GRAD, MAX_GRAD)
        nx = nan0(options[:n * 9].reshape(n, 9)[:, 2])
    bn_adam_apply(options, grad * nx, grad, l, b1, b2, n)


def bn_momentum_apply(options, G_gamma, G_beta, lr, mom, n):
    """UpdateBatchOptionsMomentum arithmetic (NeuroNet.cl:2019-2037)."""
    with _err():
        o = options[:n * 7].reshape(n, 7)
        lr, mom = F32(lr), F32(mom)
        d0 = nan0(lr * G_gamma + mom * nan0(o[:, 5]))
        d1 = nan0(lr * G_beta + mom * nan0(o[:, 6]))
        o[:, 5] = d0
        value = nan0(o[:, 3], 1.0)
        o[:, 3] = value + d0 - lr * (L1 * cl_sign(value) + L2 * value / F32(n))
        o[:, 6] = d1
        value = nan0(o[:, 4])
        o[:, 4] = value + d1 - lr * (L1 * cl_sign(value) + L2 * value / F32(n))


def UpdateBatchOptionsMomentum(options, matrix_g, learning_rates, momentum, gsize, lsize=None):
    """NeuroNet.cl:2010-2038."""
    n = gsize[0]
    with _err():
        grad = cl_clamp(nan0(matrix_g[:n]), -MAX_GRAD, MAX_GRAD)
        nx = nan0(options[:n * 7].reshape(n, 7)[:, 2])
    bn_momentum_apply(options, grad * nx, grad, learning_rates, momentum, n)


# ------------------------------------------------- legacy single-head attention
def AttentionScore(querys, keys, score, dimension, mask, gsize, lsize=None):
    """NeuroNet.cl:1237-1275.  S = exp(q.k/sqrt(d)) (NaN/Inf -> 0), masked k > q -> 0, row / sum when sum > 0."""
    U, D = gsize[0], dimension
    koef = max(np.sqrt(F32(D)), F32(1))
    with _err():
        q = querys[:U * D].reshape(U, D)
        k = keys[:U * D].reshape(U, D)
        s = nan0(np.exp((q @ k.T).astype(F32) / koef))
        if mask > 0:
            s = np.where(np.arange(U)[None, :] <= np.arange(U)[:, None], s, F32(0))
        tot = s.sum(axis=1, dtype=F32)
        s = np.where((tot > 0)[:, None], s / tot[:, None], s)
        score[:U * U] = s.reshape(-1)


def AttentionOut(scores, values, inputs, out, gsize, lsize=None):
    """NeuroNet.cl:1286-1303.  out = nan0(nan0(S) nan0(V)) + inputs."""
    U, D = gsize[0], gsize[1] if len(gsize) > 1 else 1
    with _err():
        s = nan0(scores[:U * U].reshape(U, U))
        v = nan0(values[:U * D].reshape(U, D))
        out[:U * D] = (nan0(s @ v) + inputs[:U * D].reshape(U, D)).reshape(-1)


def AttentionInsideGradients(querys, querys_g, keys, keys_g, values, values_g, scores, gradient, gsize,
                             lsize=None):
    """NeuroNet.cl:1395-1443.  P = g V^T, f(s) = s(1-s) (1e-4 at 0 or 1); vg = S^T g, qg = (f(S) o P) K / koef,
    kg = (f(S) o P)^T Q / koef, each nan0 then clamped to [-1, 1]."""
    U, D = gsize[0], gsize[1] if len(gsize) > 1 else 1
    koef = max(np.sqrt(F32(D)), F32(1))
    with _err():
        S = scores[:U * U].reshape(U, U)
        G = gradient[:U * D].reshape(U, D)
        V = values[:U * D].reshape(U, D)
        Q = querys[:U * D].reshape(U, D)
        Kk = keys[:U * D].reshape(U, D)
        P = (G @ V.T).astype(F32)
        f = np.where((S == 0) | (S == 1), F32(1e-4), S * (F32(1) - S))
        M = (f * P).astype(F32)
        values_g[:U * D] = cl_clamp(nan0(S.T @ G), -1.0, 1.0).reshape(-1)
        querys_g[:U * D] = cl_clamp(nan0((M @ Kk) / koef), -1.0, 1.0).reshape(-1)
        keys_g[:U * D] = cl_clamp(nan0((M.T @ Q) / koef), -1.0, 1.0).reshape(-1)


# ------------------------------------------------------------- MH2 attention
def MH2AttentionOut(q, kv, score, out, dimension, heads_kv, mask, gsize, lsize):
    """NeuroNet.cl:4252-4304.  Softmax (max-subtracted, LocalSoftMax) of q.k/sqrt(d) over the keys of kv head
    h % heads_kv, masked keys k > q excluded; out = sum_k nan0(V[k] * score)."""
    Qn, H = gsize[0], gsize[2]
    Kn, D, Hkv = lsize[1], dimension, heads_kv
    koef = max(np.sqrt(F32(D)), F32(1))
    with _err():
        Q = q[:Qn * H * D].reshape(Qn, H, D)
        KV = kv[:Kn * 2 * Hkv * D].reshape(Kn, 2, Hkv, D)
        hk = np.arange(H) % Hkv
        Kh = KV[:, 0][:, hk]                               # [K][H][D]
        Vh = KV[:, 1][:, hk]
        logits = nan0(np.einsum("qhd,khd->qhk", Q, Kh).astype(F32) / koef, MIN_VALUE)
        if mask != 0:
            keep = np.arange(Kn)[None, None, :] <= np.arange(Qn)[:, None, None]
            logits = np.where(keep, logits, MIN_VALUE)
        S = _softmax_rows(logits)
        score[:Qn * H * Kn] = S.reshape(-1)
        o = nan0(np.einsum("qhk,khd->qhkd", S, Vh)).sum(axis=2, dtype=F32)
        out[:Qn * H * D] = nan0(o).reshape(-1)


def MH2AttentionInsideGradients(q, q_g, kv, kv_g, scores, gradient, kunits, heads_kv, gsize, lsize=None):
    """NeuroNet.cl:4307-4406 with its indexing as written: the query gradient reads the output gradient at
    (q+h)*D+d, the key gradient reads head 0's score rows and q at D*(q0*H+h+r)+d (q0 = k mod Q), runs its head
    loop H-h times, and multiplies by 1 - (sum of a softmax row), i.e. it is rounding-level."""
    Qn, D, H = gsize[0], gsize[1], gsize[2]
    Kn, Hkv = kunits, heads_kv
    koef = max(np.sqrt(F32(D)), F32(1))
    with _err():
        S = scores[:Qn * H * Kn].reshape(Qn, H, Kn)
        G = gradient[:Qn * H * D].reshape(Qn, H, D)
        KV = kv[:Kn * 2 * Hkv * D].reshape(Kn, 2, Hkv, D)
        out_kv = kv_g[:Kn * 2 * Hkv * D].reshape(Kn, 2, Hkv, D)
        gflat = gradient
        # values
        for h in range(Hkv):
            hq = np.arange(h, H, Hkv)
            out_kv[:, 1, h, :] = np.einsum("ghd,ghv->vd", G[:, hq, :], S[:, hq, :]).astype(F32)
        # queries
        hk = np.arange(H) % Hkv
        Vh = KV[:, 1][:, hk]                                 # [K][H][D]
        Kh = KV[:, 0][:, hk]
        A = np.einsum("qhv,vhd->qhd", S, Vh).astype(F32)
        acc = np.einsum("qhk,khd->qhd", S, Vh * Kh) - A * np.einsum("qhk,khd->qhd", S, Kh)
        outg = np.array([[gflat[(qi + h) * D:(qi + h) * D + D] for h in range(H)] for qi in range(Qn)], F32)
        q_g[:Qn * H * D] = (outg * acc.astype(F32) / koef).astype(F32).reshape(-1)
        # keys
        row0 = S[:, 0, :]                                    # [r][k]
        tot = row0.sum(axis=1, dtype=F32)                    # [r]
        for k in range(Kn):
            q0 = k % Qn
            for h in range(Hkv):
                val = KV[k, 1, h, :]
                accd = np.zeros(D, F32)
                for r in range(Qn):
                    sc = row0[r, k]
                    if sc == 0:
                        continue
                    gi = (h + r) * D
                    qi = D * (q0 * H + h + r)
                    accd += gflat[gi:gi + D] * val * sc * (F32(1) - tot[r]) * q[qi:qi + D]
                out_kv[k, 0, h, :] = accd * F32(H - h) / koef


# --------------------------------------------------------------------- LSTM
def _lstm_input_index(H, inputs_size):
    """Input positions the reference's gate loop reads (NeuroNet.cl:2228-2244): float4 blocks while the
    unsigned H - i > 4, otherwise positions i..H-1 (so for inputs > H the block at i = H is skipped)."""
    idx = []
    for i in range(0, inputs_size, 4):
        if ((H - i) & 0xFFFFFFFF) > 4:
            idx += [i, i + 1, i + 2, i + 3]
        else:
            idx += list(range(i, H))
    return np.array(idx, dtype=np.int64)


def LSTM_FeedForward(inputs, inputs_size, weights, concatenated, memory, output, gsize, lsize=None):
    """NeuroNet.cl:2189-2261.  Gate g of neuron id sums weight row g+id over (h(t-1), x(t), 1); f,i,o are
    sigmoid and the new content tanh; c = f c + i g; h = o tanh(c).  Every gate reads h(t-1) (the reference
    overwrites h from other work-groups while they read it)."""
    H, V = gsize[0], gsize[2] if len(gsize) > 2 else 1
    ins = inputs_size
    ws = ins + H + 1
    with _err():
        h_prev = output[:V * H].reshape(V, H).copy()
        xi = _lstm_input_index(H, ins)
        flat_x = inputs
        cat = concatenated[:V * 4 * H].reshape(V, 4, H)
        for gate in range(4):
            rows = np.arange(H) + gate
            W = weights[:(H + 3) * ws].reshape(H + 3, ws)[rows]       # [H][ws]
            hs = h_prev @ W[:, :H].T                                   # [V][H]
            xv = np.stack([flat_x[v * ins + xi] for v in range(V)]) if xi.size else np.zeros((V, 0), F32)
            xs = xv @ W[:, H + xi].T if xi.size else 0
            s = hs + xs + nan0(W[:, H + ins])[None, :]
            cat[:, gate, :] = f_activation(s.astype(F32), SIGMOID if gate < 3 else TANH)
        mem = memory[:2 * V * H].reshape(2, V, H)
        old = mem[0].copy()
        mem[1] = old
        new = nan0(old * cat[:, 0] + cat[:, 1] * cat[:, 3])
        mem[0] = new
        output[:V * H] = nan0(cat[:, 2] * f_activation(new, TANH)).reshape(-1)


def LSTM_ConcatenatedGradient(gradient, concatenated_gradient, memory, concatenated, gsize, lsize=None):
    """NeuroNet.cl:2265-2297: gate gradients from the hidden-state gradient."""
    H, V = gsize[0], gsize[1] if len(gsize) > 1 else 1
    with _err():
        g = gradient[:V * H].reshape(V, H)
        m = memory[:2 * V * H].reshape(2, V, H)
        a = concatenated[:V * 4 * H].reshape(V, 4, H)
        cg = concatenated_gradient[:V * 4 * H].reshape(V, 4, H)
        t = np.tanh(m[0])
        cg[:, 2] = g * t
        mg = g * a[:, 2] * (F32(1) - t * t)
        cg[:, 3] = mg * a[:, 1]
        cg[:, 1] = mg * a[:, 3]
        cg[:, 0] = mg * m[1]


def LSTM_HiddenGradient(concatenated_gradient, inputs_gradient, weights_gradient, hidden_state, inputs, weights,
                        output, hidden_size, inputs_size, gsize, lsize=None):
    """NeuroNet.cl:2301-2441.  Derivative factors from the gradient value (cg(1-cg), cg(1-cg^2)); input
    gradient; weight gradient summed over the series; the "bias" sum of row i written at (i+1)*(H+in+1)
    after the weight loop (and the last one, one element past a (4H)x(H+in+1) matrix, only when the buffer
    holds it); hidden_state <- output."""
    H, V = gsize[0], gsize[1] if len(gsize) > 1 else 1
    ins = inputs_size
    ws = H + ins + 1
    with _err():
        cg = concatenated_gradient[:V * 4 * H].reshape(V, 4 * H)
        a = np.concatenate([cg[:, :3 * H] * (F32(1) - cg[:, :3 * H]),
                            cg[:, 3 * H:] * (F32(1) - cg[:, 3 * H:] ** 2)], axis=1).astype(F32)
        W = weights[:4 * H * ws].reshape(4 * H, ws)
        h_old = hidden_state[:V * H].reshape(V, H).copy()
        x = inputs[:V * ins].reshape(V, ins)
        if ins:
            inputs_gradient[:V * ins] = (a @ W[:, H:H + ins]).astype(F32).reshape(-1)
        opnd = np.concatenate([h_old, x], axis=1)
        wg = weights_gradient
        G = (a.T @ opnd).astype(F32)                       # [4H][H+in]
        wg2 = wg[:4 * H * ws].reshape(4 * H, ws)
        wg2[:, :H + ins] = G
        bias = np.concatenate([cg[:, :3 * H] * (F32(1) - cg[:, :3 * H]),
                               F32(1) - cg[:, 3 * H:] ** 2], axis=1).sum(axis=0, dtype=F32)
        last = 4 * H if wg.size > 4 * H * ws else 4 * H - 1
        for i in range(last):
            wg[(i + 1) * ws] = bias[i]
        hidden_state[:V * H] = output[:V * H]


def LSTM_UpdateWeightsAdam(weights, weights_gradient, matrix_m, matrix_v, l, b1, b2, gsize, lsize=None):
    """NeuroNet.cl:2450-2475: Adam over a (rows x total) block with l2 decay divided by total, raw rate."""
    total, rows = gsize[0], gsize[1] if len(gsize) > 1 else 1
    n = total * rows
    with _err():
        b1, b2, l = F32(b1), F32(b2), F32(l)
        g = cl_clamp(nan0(weights_gradient[:n]), -MAX_GRAD, MAX_GRAD)
        mt = b1 * nan0(matrix_m[:n]) + (F32(1) - b1) * g
        vt = b2 * nan0(matrix_v[:n], 1.0) + (F32(1) - b2) * (g * g)
        w = nan0(weights[:n])
        delta = l * (mt / (np.sqrt(vt) + F32(1e-37)) - (L1 * cl_sign(w) + L2 * w / F32(total)))
        weights[:n] = nan0(w + delta)
        matrix_m[:n] = mt
        matrix_v[:n] = vt


# ------------------------------------------------------------------ ADAM_MINI
LOCAL_ARRAY_SIZE = 64  # NeuroNet.cl:18


def adam_mini_input_scale(x, inputs):
    """The local reduction of UpdateWeightsAdamMini (NeuroNet.cl:7531-7558), which is the same for
    every output row.  Slot s of ls = min(64, inputs) sums inp_i^2 / inputs over the local ids
    i = s, s + ls, ... that its count loop reaches (the bias input, 1, only when inputs % ls != 0);
    the folding loop stops before its last step, so the result is the first slot after the folds."""
    ls = min(LOCAL_ARRAY_SIZE, inputs)
    temp = np.zeros(max(ls, 1), F32)
    with _err():
        n_counts = -(-inputs // ls)
        for count in range(n_counts):
            for shift in range(ls):
                i = count * ls + shift
                if i > inputs:
                    continue
                inp = F32(x[i]) if i < inputs else F32(1)
                term = F32(0) if not np.isfinite(inp) else F32(inp * inp) / F32(inputs)
                temp[shift] = F32((F32(0) if count == 0 else temp[shift]) + term)
        count = (ls + 1) // 2
        while True:
            for i in range(count):
                if i + count < ls:
                    temp[i] = F32(temp[i] + temp[i + count])
                    temp[i + count] = 0
            count = (count + 1) // 2
            if not count > 1:
                break
    return temp[0]


def UpdateWeightsAdamMini(matrix_w, matrix_g, matrix_i, matrix_m, matrix_v, l, b1, b2, gsize, lsize=None):
    """NeuroNet.cl:7515-7612 over global (inputs+1, outputs), local (inputs+1, 1): one second moment
    per output row, v = b2 v + (1-b2) g^2 s with s the input scale above; m per weight; the weight
    moves only when delta > 0 (as written)."""
    inputs = (lsize[0] if lsize is not None else gsize[0]) - 1
    outputs = gsize[1]
    with _err():
        s = adam_mini_input_scale(matrix_i, inputs)
        t0 = s if np.isfinite(s) else F32(1)
        g = matrix_g[:outputs].astype(F32)
        g = np.where(np.isfinite(g), g, F32(0)).astype(F32)
        v = matrix_v[:outputs].astype(F32)
        v = np.where(np.isfinite(v), v, F32(1)).astype(F32)
        b1, b2, l = F32(b1), F32(b2), F32(l)
        vt = (b2 * v + ((F32(1) - b2) * (g * g)) * t0).astype(F32)
        matrix_v[:outputs] = vt
        idx = np.arange(outputs)[:, None] * (inputs + 1) + np.arange(inputs + 1)[None, :]
        inp = np.concatenate([matrix_i[:inputs].astype(F32), np.ones(1, F32)])[None, :]
        weight = matrix_w[idx]
        weight = np.where(np.isfinite(weight), weight, F32(0)).astype(F32)
        m = matrix_m[idx]
        m = np.where(np.isfinite(m), m, F32(0)).astype(F32)
        m = (b1 * m + ((F32(1) - b1) * g[:, None]) * inp).astype(F32)
        m = np.where(np.isfinite(m), m, F32(0)).astype(F32)
        delta = (l * (m / (np.sqrt(vt)[:, None] + F32(1e-37)) - (L1 * cl_sign(weight) + L2 * weight))).astype(F32)
        delta = np.where(np.isfinite(delta), delta, F32(0)).astype(F32)
        matrix_w[idx] = np.where(delta > 0, (weight + delta).astype(F32), matrix_w[idx])
        matrix_m[idx] = m


def conv_adam_mini_grads(matrix_g, matrix_i, inputs, window_in, window_out, variables, step):
    """Per-weight gradients of UpdateWeightsConvAdamMini (NeuroNet.cl:7632-7647): over
    total = (inputs - window_in + step - 1) / step units, stopping once i + t*window_in >= inputs
    (the reference's test, with window_in where the stride is step), non-finite terms skipped.
    Returns [variables][window_out][window_in + 1]."""
    total = (inputs - window_in + step - 1) // step
    G = np.zeros((variables, window_out, window_in + 1), F32)
    with _err():
        for v in range(variables):
            for i in range(window_in + 1):
                acc = np.zeros(window_out, F32)
                for t in range(total):
                    if i != window_in and i + t * window_in >= inputs:
                        break
                    gr = matrix_g[v * total * window_out + t * window_out:v * total * window_out + (t + 1) * window_out]
                    xi = F32(1) if i == window_in else F32(matrix_i[v * inputs + i + t * step])
                    gt = (gr * xi).astype(F32)
                    acc = np.where(np.isfinite(gt), (acc + gt).astype(F32), acc)
                G[v, :, i] = acc
    return G


def conv_adam_mini_scale(G_head, window_in, window_out_h):
    """The local reduction of UpdateWeightsConvAdamMini (NeuroNet.cl:7649-7680) for one head of one
    variable: slot s of ls = min(64, window_in) sums grad^2 / (window_in * window_out_h) over the
    head's rows h (outer) and the local ids i = s, s + ls, ... its count loop reaches (the bias
    column only when window_in % ls != 0), then the fold that stops one step early."""
    ls = min(LOCAL_ARRAY_SIZE, window_in)
    temp = np.zeros(max(ls, 1), F32)
    n_counts = -(-window_in // ls)
    den = F32(window_in * window_out_h)
    with _err():
        for h in range(window_out_h):
            for count in range(n_counts):
                for shift in range(ls):
                    i = count * ls + shift
                    if i > window_in:
                        continue
                    gv = G_head[h, i]
                    term = F32(0) if not np.isfinite(gv) else F32(gv * gv) / den
                    temp[shift] = F32((F32(0) if (count == 0 and h == 0) else temp[shift]) + term)
        count = (ls + 1) // 2
        while True:
            for i in range(count):
                if i + count < ls:
                    temp[i] = F32(temp[i] + temp[i + count])
                    temp[i + count] = 0
            count = (count + 1) // 2
            if not count > 1:
                break
    return temp[0]


def UpdateWeightsConvAdamMini(matrix_w, matrix_g, matrix_i, matrix_m, matrix_v, inputs, l, b1, b2, step, gsize,
                              lsize=None):
    """NeuroNet.cl:7615-7731 over global (window_in+1, window_out, variables), local
    (window_in+1, window_out_h, 1): one second moment per head (window_out_h rows), clamped to
    [1e-6, 1e6]; m clamped to +-1e5; w += l m / sqrt(v) with no decay.  The second moment is indexed
    by head only, so work-groups of different variables update the same entry (a race in the
    reference); here the variables take their turns in order."""
    window_in, window_out = gsize[0] - 1, gsize[1]
    variables = gsize[2] if len(gsize) > 2 else 1
    window_out_h = lsize[1] if lsize is not None and len(lsize) > 1 else 1
    G = conv_adam_mini_grads(matrix_g, matrix_i, inputs, window_in, window_out, variables, step)
    b1, b2, l = F32(b1), F32(b2), F32(l)
    with _err():
        for v in range(variables):
            for head in range(window_out // window_out_h):
                f0 = head * window_out_h
                t0 = conv_adam_mini_scale(G[v, f0:f0 + window_out_h], window_in, window_out_h)
                if not np.isfinite(t0):
                    t0 = F32(1)
                vv = matrix_v[head]
                if not np.isfinite(vv):
                    vv = F32(1)
                t0 = F32(cl_clamp(F32(b2 * vv + (F32(1) - b2) * t0), 1e-6, 1e6))
                matrix_v[head] = t0
                rows = (np.arange(f0, f0 + window_out_h) + v * window_out)[:, None] * (window_in + 1)
                idx = rows + np.arange(window_in + 1)[None, :]
                mt = cl_clamp((b1 * matrix_m[idx] + (F32(1) - b1) * G[v, f0:f0 + window_out_h]).astype(F32), -1e5,
                              1e5)
                mt = np.where(np.isfinite(mt), mt, F32(0)).astype(F32)
                w = (matrix_w[idx] + (l * mt / np.sqrt(t0)).astype(F32)).astype(F32)
                matrix_w[idx] = np.where(np.isfinite(w), w, matrix_w[idx])
                matrix_m[idx] = mt


# ---------------------------------------------------------------- concatenate
def _concat_rows(matrix_w, n_out, inputs1, inputs2):
    return matrix_w[:n_out * (inputs1 + inputs2 + 1)].reshape(n_out, inputs1 + inputs2 + 1)


def Concat_FeedForward(matrix_w, matrix_i1, matrix_i2, matrix_o, inputs1, inputs2, activation, gsize, lsize=None):
    """NeuroNet.cl:3628-3718.  o[i] = act(W[i] . [x1; x2; 1]) over rows of inputs1+inputs2+1 floats; the two
    inputs are summed in float4 groups, a group whose addition makes the sum NaN is skipped, the bias is
    added without a check and a NaN total becomes 0."""
    n_out = gsize[0]
    with _err():
        w = _concat_rows(matrix_w, n_out, inputs1, inputs2)
        s = np.zeros(n_out, F32)
        for x, off, n in ((matrix_i1, 0, inputs1), (matrix_i2, inputs1, inputs2)):
            for k in range(0, n, 4):
                e = min(k + 4, n)
                d = (w[:, off + k:off + e] * x[k:e][None, :]).sum(axis=1, dtype=F32)
                t = (s + d).astype(F32)
                s = np.where(np.isnan(t), s, t).astype(F32)
        s = (s + w[:, inputs1 + inputs2]).astype(F32)
        s = np.where(np.isnan(s), F32(0), s)
        matrix_o[:n_out] = f_activation(s, activation)


def Concat_HiddenGradient(matrix_w, matrix_g, matrix_o1, matrix_o2, matrix_ig1, matrix_ig2, outputs, inputs1,
                          inputs2, activation1, activation2, gsize, lsize=None):
    """NeuroNet.cl:3724-3785.  For input i of [x1; x2]: sum_k g[k] W[k][i] (NaN -> 0), then Deactivation
    with the first or the second input's activation, written to the matching gradient buffer."""
    n = min(gsize[0], inputs1 + inputs2)
    with _err():
        w = _concat_rows(matrix_w, outputs, inputs1, inputs2)[:, :n]
        s = (w * matrix_g[:outputs][:, None]).sum(axis=0, dtype=F32)
        s = np.where(np.isnan(s), F32(0), s)
        n1 = min(n, inputs1)
        matrix_ig1[:n1] = deactivation(s[:n1], matrix_o1[:n1], activation1)
        if n > inputs1:
            matrix_ig2[:n - inputs1] = deactivation(s[inputs1:n], matrix_o2[:n - inputs1], activation2)


def _concat_inputs(matrix_i1, matrix_i2, inputs1, inputs2, n_col):
    """[x1; x2; 1] for columns j < n_col (NeuroNet.cl:3808, 3845)."""
    j = np.arange(n_col)
    return np.where(j < inputs1, matrix_i1[np.minimum(j, max(inputs1 - 1, 0))] if inputs1 else F32(0),
                    np.where(j - inputs1 < inputs2,
                             matrix_i2[np.clip(j - inputs1, 0, max(inputs2 - 1, 0))] if inputs2 else F32(0),
                             F32(1))).astype(F32)


def concat_adam_apply(matrix_w, grad, matrix_m, matrix_v, inputs1, inputs2, l, b1, b2, n_out, n_col):
    """Adam arithmetic of Concat_UpdateWeightsAdam (NeuroNet.cl:3849-3861) for the gradient grad[i, j]:
    no clamp and no NaN guards; a weight moves only when |delta| > 0."""
    with _err():
        idx = np.arange(n_out)[:, None] * (inputs1 + inputs2 + 1) + np.arange(n_col)[None, :]
        weight = matrix_w[idx]
        g = np.asarray(grad, dtype=F32)
        b1, b2, l = F32(b1), F32(b2), F32(l)
        mt = (b1 * matrix_m[idx] + (F32(1) - b1) * g).astype(F32)
        vt = (b2 * matrix_v[idx] + (F32(1) - b2) * (g * g)).astype(F32)
        delta = (l * (mt / (np.sqrt(vt) + F32(1e-37)) - (L1 * cl_sign(weight) + L2 * weight))).astype(F32)
        matrix_w[idx] = np.where(np.abs(delta) > 0, (weight + delta).astype(F32), weight)
        matrix_m[idx] = mt
        matrix_v[idx] = vt


def Concat_UpdateWeightsAdam(matrix_w, matrix_g, matrix_i1, matrix_i2, matrix_m, matrix_v, inputs1, inputs2, l,
                             b1, b2, gsize, lsize=None):
    """NeuroNet.cl:3823-3862.  g = g_o[i] * [x1; x2; 1][j]; Adam as UpdateWeightsAdam but without the
    gradient clamp."""
    n_out, n_col = gsize[0], min(gsize[1], inputs1 + inputs2 + 1)
    with _err():
        inp = _concat_inputs(matrix_i1, matrix_i2, inputs1, inputs2, n_col)
        grad = (matrix_g[:n_out][:, None] * inp[None, :]).astype(F32)
    concat_adam_apply(matrix_w, grad, matrix_m, matrix_v, inputs1, inputs2, l, b1, b2, n_out, n_col)


def concat_momentum_apply(matrix_w, grad, matrix_dw, inputs1, inputs2, learning_rates, momentum, n_out, n_col):
    """Arithmetic of Concat_UpdateWeightsMomentum (NeuroNet.cl:3806-3817) for the gradient grad[i, j]."""
    with _err():
        idx = np.arange(n_out)[:, None] * (inputs1 + inputs2 + 1) + np.arange(n_col)[None, :]
        delta = (F32(learning_rates) * np.asarray(grad, F32) + F32(momentum) * matrix_dw[idx]).astype(F32)
        ok = ~np.isnan(delta)
        matrix_dw[idx] = np.where(ok, delta, matrix_dw[idx])
        w = matrix_w[idx]
        matrix_w[idx] = np.where(ok & (np.abs(delta) > 0), (w + delta).astype(F32), w)


def Concat_UpdateWeightsMomentum(matrix_w, matrix_g, matrix_i1, matrix_i2, matrix_dw, inputs1, inputs2,
                                 learning_rates, momentum, gsize, lsize=None):
    """NeuroNet.cl:3790-3818.  delta = lr g_o[i] [x1; x2; 1][j] + momentum dw; kept unless NaN."""
    n_out, n_col = gsize[0], min(gsize[1], inputs1 + inputs2 + 1)
    with _err():
        inp = _concat_inputs(matrix_i1, matrix_i2, inputs1, inputs2, n_col)
        grad = (matrix_g[:n_out][:, None] * inp[None, :]).astype(F32)
    concat_momentum_apply(matrix_w, grad, matrix_dw, inputs1, inputs2, learning_rates, momentum, n_out, n_col)


# ------------------------------------------------------------ quantile heads
PI_F = F32(np.pi)


def _taus(sm):
    """Fraction midpoints per row: sum_{t<i} p_t + p_i / 2, summed in order (float32)."""
    cs = np.cumsum(sm, axis=1, dtype=F32)
    return ((cs - sm).astype(F32) + sm / F32(2)).astype(F32)


def FQF_Cosine(softmax, output, gsize, lsize=None):
    """NeuroNet.cl:2524-2538 over global (quants, actions): cos(i pi tau_i)."""
    T, R = gsize[0], (tuple(gsize) + (1,))[1]
    with _err():
        sm = softmax[:R * T].reshape(R, T).astype(F32)
        i = np.arange(T, dtype=F32)[None, :]
        output[:R * T] = np.cos((i * PI_F * _taus(sm)).astype(F32)).astype(F32).reshape(-1)


def FQF_Output(quantiles, delta_taus, output, total, gsize, lsize=None):
    """NeuroNet.cl:2543-2553 over global (actions): y = sum_i quantile_i dtau_i."""
    R, T = gsize[0], total
    with _err():
        p = (quantiles[:R * T] * delta_taus[:R * T]).astype(F32).reshape(R, T)
        output[:R] = _seq_sum(p, 1)[0]


def FQF_OutputGradient(quantiles, delta_taus, output_gr, quantiles_gr, taus_gr, gsize, lsize=None):
    """NeuroNet.cl:2560-2573 over global (quants, actions)."""
    T, R = gsize[0], (tuple(gsize) + (1,))[1]
    with _err():
        g = np.repeat(output_gr[:R].astype(F32), T)
        quantiles_gr[:R * T] = (g * delta_taus[:R * T]).astype(F32)
        taus_gr[:R * T] = (g * quantiles[:R * T]).astype(F32)


def FQF_QuantileGradient(state_embeding, taus_embeding, quantiles_gr, state_gr, taus_gr, gsize, lsize=None):
    """NeuroNet.cl:2579-2592 over global (quants, actions)."""
    n = gsize[0] * (tuple(gsize) + (1,))[1]
    with _err():
        g = quantiles_gr[:n].astype(F32)
        state_gr[:n] = (g * taus_embeding[:n]).astype(F32)
        taus_gr[:n] = (g * state_embeding[:n]).astype(F32)


REF_MAX_VALUE = F32(3.4e37)  # MAX_VALUE, NeuroNet.cl:20


def FQF_MonotoneRearrange(quantiles, probabilities, ordered_quantiles, ordered_probabilities, order, diagnostics,
                          gsize, lsize=None):
    """NeuroNet.cl:20716-20817 over global (quants, rows), one work-group per row of a power of two up
    to 64 quants (other rows: nothing written): ascending (value, index) order, a value that is not
    finite taken as MAX_VALUE and a probability that is not finite or negative as 0; diagnostics per
    row: crossing rate and magnitude over adjacent pairs (/ (quants - 1)), probability sum, min, max,
    and the invalid-probability count."""
    T, R = gsize[0], (tuple(gsize) + (1,))[1]
    if T == 0 or (T & (T - 1)) != 0 or T > 64:
        return
    with _err():
        for v in range(R):
            z = quantiles[v * T:(v + 1) * T].astype(F32)
            p = probabilities[v * T:(v + 1) * T].astype(F32)
            lz = np.where(np.isfinite(z), z, REF_MAX_VALUE).astype(F32)
            pbad = ~np.isfinite(p) | (p < 0)
            lp = np.where(pbad, F32(0), p).astype(F32)
            idx = sorted(range(T), key=lambda i: (float(lz[i]), i))
            ordered_quantiles[v * T:(v + 1) * T] = lz[idx]
            ordered_probabilities[v * T:(v + 1) * T] = lp[idx]
            order[v * T:(v + 1) * T] = np.asarray(idx, F32)
            dinv = F32(1) / F32(T - 1) if T > 1 else F32(0)
            cf = F32((lz[1:] < lz[:-1]).sum())
            cm = np.maximum((lz[:-1] - lz[1:]).astype(F32), F32(0)).sum(dtype=F32)
            diagnostics[v * 6:(v + 1) * 6] = [cf * dinv, cm * dinv, lp.sum(dtype=F32), lp.min(), lp.max(),
                                              F32(pbad.sum())]


def srm_cumulative(u, risk_type, risk_parameter, mean_weight):
    """SRMCumulative, NeuroNet.cl:2805-2850 (float32)."""
    eps = F32(1e-6)
    tau = np.clip(np.asarray(u, F32), F32(0), F32(1)).astype(F32)
    c = lambda x: np.clip(np.asarray(x, F32), F32(0), F32(1)).astype(F32)
    if risk_type == 0:
        return tau
    if risk_type == 1:
        alpha = F32(min(max(F32(risk_parameter), eps), F32(1)))
        return c(np.minimum(tau, alpha) / alpha)
    if risk_type == 2:
        alpha = F32(min(max(F32(risk_parameter), eps), F32(1)))
        omega = F32(min(max(F32(mean_weight), F32(0)), F32(1)))
        return c(omega * tau + (F32(1) - omega) * np.minimum(tau, alpha) / alpha)
    if risk_type == 3:
        lam = F32(max(F32(risk_parameter), F32(0)))
        if lam <= eps:
            return tau
        return c(-np.expm1((-lam * tau).astype(F32)) / -np.expm1(-lam))
    if risk_type == 4:
        nu = F32(max(F32(risk_parameter), F32(1)))
        return c(F32(1) - np.power((F32(1) - tau).astype(F32), nu))
    return np.zeros_like(tau)


def FQF_SRMForward(quantiles, probabilities, result, risk_type, risk_parameter, mean_weight, gsize, lsize=None):
    """NeuroNet.cl:2924-3021 over global (quants, rows), one work-group per row: with P_i the running
    sum of max(IsNaNOrInf(p), 0) and M the row's mass, result = sum_i IsNaNOrInf(z_i)
    max(F(P_i / M) - F(P_{i-1} / M), 0) for the spectral weight F; 0 when M <= 1e-37."""
    T, R = gsize[0], (tuple(gsize) + (1,))[1]
    with _err():
        for v in range(R):
            p = np.maximum(nan0(probabilities[v * T:(v + 1) * T]), F32(0)).astype(F32)
            cs = np.cumsum(p, dtype=F32)
            mass = F32(cs[-1]) if T else F32(0)
            if not (nan0(mass) > F32(1e-37)):
                result[v] = 0
                continue
            inv = F32(1) / mass
            hi = np.clip((cs * inv).astype(F32), F32(0), F32(1))
            lo = np.concatenate([[F32(0)], np.clip((cs[:-1] * inv).astype(F32), F32(0), F32(1))]).astype(F32)
            w = np.maximum(srm_cumulative(hi, risk_type, risk_parameter, mean_weight)
                           - srm_cumulative(lo, risk_type, risk_parameter, mean_weight), F32(0)).astype(F32)
            result[v] = nan0((w * nan0(quantiles[v * T:(v + 1) * T])).astype(F32).sum(dtype=F32))


def srm_density(u, risk_type, risk_parameter, mean_weight):
    """SRMDensity, NeuroNet.cl:2855-2900 (float32)."""
    eps = F32(1e-6)
    tau = np.clip(np.asarray(u, F32), F32(0), F32(1)).astype(F32)
    one = np.ones_like(tau)
    if risk_type == 0:
        return one
    if risk_type == 1:
        alpha = F32(min(max(F32(risk_parameter), eps), F32(1)))
        return np.where(tau < alpha, F32(1) / alpha, F32(0)).astype(F32)
    if risk_type == 2:
        alpha = F32(min(max(F32(risk_parameter), eps), F32(1)))
        omega = F32(min(max(F32(mean_weight), F32(0)), F32(1)))
        return np.where(tau < alpha, omega + (F32(1) - omega) / alpha, omega).astype(F32)
    if risk_type == 3:
        lam = F32(max(F32(risk_parameter), F32(0)))
        if lam <= eps:
            return one
        return np.maximum(lam * np.exp((-lam * tau).astype(F32)) / -np.expm1(-lam), F32(0)).astype(F32)
    if risk_type == 4:
        nu = F32(max(F32(risk_parameter), F32(1)))
        if nu == F32(1):
            return one
        return np.maximum(nu * np.power((F32(1) - tau).astype(F32), nu - F32(1)), F32(0)).astype(F32)
    return np.zeros_like(tau)


def FQF_SRMGradient(quantiles, probabilities, result_gradient, quantiles_gradient, probabilities_gradient,
                    risk_type, risk_parameter, mean_weight, gsize, lsize=None):
    """NeuroNet.cl:3027-3200 over global (quants, rows), one work-group per row, upstream u =
    IsNaNOrInf(result_gradient[row]) (u == 0 or no probability mass: zeros): quantile i gets
    IsNaNOrInf(u w_i) (0 when not finite); with b_i = IsNaNOrInf(u (z_i - z_{i+1}) F'(P_i / M)) and
    S_i = sum_{j >= i} b_j, probability i gets IsNaNOrInf((S_i - sum_j (p_j / M) S_j) / M) (0 when not
    finite or negative)."""
    T, R = gsize[0], (tuple(gsize) + (1,))[1]
    with _err():
        for v in range(R):
            sl = slice(v * T, (v + 1) * T)
            raw_p, raw_z = probabilities[sl].astype(F32), quantiles[sl].astype(F32)
            p = np.maximum(nan0(raw_p), F32(0)).astype(F32)
            z = nan0(raw_z)
            up = nan0(result_gradient[v])
            cs = np.cumsum(p, dtype=F32)
            mass = nan0(cs[-1])
            if up == 0 or mass <= F32(1e-37):
                quantiles_gradient[sl] = 0
                probabilities_gradient[sl] = 0
                continue
            inv = F32(1) / mass
            hi = np.clip((cs * inv).astype(F32), F32(0), F32(1))
            lo = np.concatenate([[F32(0)], np.clip((cs[:-1] * inv).astype(F32), F32(0), F32(1))])
            w = np.maximum(srm_cumulative(hi, risk_type, risk_parameter, mean_weight)
                           - srm_cumulative(lo.astype(F32), risk_type, risk_parameter, mean_weight), F32(0))
            quantiles_gradient[sl] = np.where(np.isfinite(raw_z), nan0(up * w.astype(F32)), F32(0))
            nxt = np.concatenate([z[1:], z[-1:]])
            b = nan0((up * (z - nxt)).astype(F32) * srm_density(hi, risk_type, risk_parameter, mean_weight))
            b[-1] = 0
            suffix = np.cumsum(b[::-1], dtype=F32)[::-1].astype(F32)
            corr = ((p * inv).astype(F32) * suffix).astype(F32).sum(dtype=F32)
            pv = np.isfinite(raw_p) & (raw_p >= 0)
            probabilities_gradient[sl] = np.where(pv, nan0(((suffix - corr) * inv).astype(F32)), F32(0))


def FQF_RearrangeGradient(ordered_quantiles_gradient, ordered_probabilities_gradient, order, quantiles_gradient,
                          probabilities_gradient, gsize, lsize=None):
    """NeuroNet.cl:20823-20842 over global (quants, rows): each ordered gradient goes back to the
    index `order` names (entries that are not a valid index are skipped)."""
    T, R = gsize[0], (tuple(gsize) + (1,))[1]
    for v in range(R):
        for j in range(T):
            o = order[v * T + j]
            d = int(o) if np.isfinite(o) else -1
            if 0 <= d < T:
                quantiles_gradient[v * T + d] = ordered_quantiles_gradient[v * T + j]
                probabilities_gradient[v * T + d] = ordered_probabilities_gradient[v * T + j]


def FQF_CosineGradientSRM(softmax, output_gr, softmax_gr, gsize, lsize=None):
    """NeuroNet.cl:2630-2651 over global (quants, actions): softmax_gr[i] += -pi/2 i sin(pi i tau_i) g_i
    + sum_{t>i} -pi t sin(pi t tau_t) g_t (the later terms summed in order)."""
    T, R = gsize[0], (tuple(gsize) + (1,))[1]
    with _err():
        sm = softmax[:R * T].reshape(R, T).astype(F32)
        g = output_gr[:R * T].reshape(R, T).astype(F32)
        tau = _taus(sm)
        i = np.arange(T, dtype=F32)[None, :]
        sn = np.sin((PI_F * i * tau).astype(F32)).astype(F32)
        first = (F32(-0.5) * PI_F * i * sn * g).astype(F32)
        f = (-PI_F * i * sn * g).astype(F32)
        out = softmax_gr[:R * T].reshape(R, T).copy()
        for k in range(T):
            later, _ = _seq_sum(f[:, k + 1:], 1)
            out[:, k] = (out[:, k] + (first[:, k] + later).astype(F32)).astype(F32)
        softmax_gr[:R * T] = out.reshape(-1)


def FQF_DistributionTargetGradient(quantiles, probabilities, quantiles_gr, probabilities_gr, target,
                                   probability_weight, value_weight, gsize, lsize=None):
    """NeuroNet.cl:2663-2716 over global (quants, rows), one work-group per row: the finite quantile
    nearest the target (ties: the larger value, then the lower index) gets value_weight (target - z)
    and probability_weight / (p + 1e-37); every other entry 0 (all of them when the target is not
    finite)."""
    T, R = gsize[0], (tuple(gsize) + (1,))[1]
    with _err():
        z = quantiles[:R * T].reshape(R, T).astype(F32)
        pr = nan0(probabilities[:R * T].reshape(R, T))
        qg = np.zeros((R, T), F32)
        pg = np.zeros((R, T), F32)
        t = F32(target)
        if np.isfinite(t):
            for v in range(R):
                ok = np.isfinite(z[v])
                if not ok.any():
                    continue
                d = np.where(ok, np.abs((z[v] - t).astype(F32)), np.inf)
                cand = ok & (d == d.min())
                c = z[v][cand].max()
                k = int(np.flatnonzero(ok & (z[v] == c))[0])
                qg[v, k] = F32(value_weight) * F32(t - z[v, k])
                pg[v, k] = F32(probability_weight) / F32(pr[v, k] + F32(1e-37))
        quantiles_gr[:R * T] = qg.reshape(-1)
        probabilities_gr[:R * T] = pg.reshape(-1)


def FQF_CosineGradient(softmax, output_gr, softmax_gr, gsize, lsize=None):
    """NeuroNet.cl:2598-2624 over global (quants, actions): softmax_gr[i] += -pi i sin(pi i tau_i) g_i
    + sum_{t>i} -pi t sin(pi t tau_t) g_t p_t / tau_t (the later terms summed in order)."""
    T, R = gsize[0], (tuple(gsize) + (1,))[1]
    with _err():
        sm = softmax[:R * T].reshape(R, T).astype(F32)
        g = output_gr[:R * T].reshape(R, T).astype(F32)
        tau = _taus(sm)
        i = np.arange(T, dtype=F32)[None, :]
        sn = np.sin((PI_F * i * tau).astype(F32)).astype(F32)
        first = (-PI_F * i * sn * g).astype(F32)
        f = ((-PI_F * i * sn * g * sm).astype(F32) / tau).astype(F32)
        out = softmax_gr[:R * T].reshape(R, T).copy()
        for k in range(T):
            later, _ = _seq_sum(f[:, k + 1:], 1)
            out[:, k] = (out[:, k] + (first[:, k] + later).astype(F32)).astype(F32)
        softmax_gr[:R * T] = out.reshape(-1)


def FQF_FractionGradient(matrix_w, gradient, input_gr, outputs, gsize, lsize=None):
    """NeuroNet.cl:3207-3224 over global (inputs, 1): input_gr[i] = IsNaNOrInf(sum_k W[k][i] g[k], 0),
    the operands summed as they are."""
    inputs = gsize[0]
    with _err():
        w = matrix_w[:outputs * (inputs + 1)].reshape(outputs, inputs + 1)[:, :inputs].astype(F32)
        p = (w * gradient[:outputs, None]).astype(F32)
        input_gr[:inputs] = nan0(_seq_sum(p, 0)[0])


def SAC_AlphaLogProbs(outputs, quantiles, probs, alphas, log_probs, random, count_quants, activation,
                      gsize, lsize=None):
    """NeuroNet.cl:3903-3933: the first quantile whose running probability reaches random[i] (the
    last one otherwise), its activation, and -alpha log p of it."""
    n, cq = gsize[0], count_quants
    with _err():
        for i in range(n):
            prob = value = s = F32(0)
            for r in range(cq):
                prob = F32(probs[i * cq + r])
                s = F32(s + prob)
                if s >= random[i] or r == cq - 1:
                    value = quantiles[i * cq + r]
                    break
            outputs[i] = f_activation(value, activation)
            log_probs[i] = -alphas[i] * np.log(prob)


def SAC_AlphaGradients(outputs, gradient, log_probs, alphas_grad, activation, gsize, lsize=None):
    """NeuroNet.cl:3939-3951."""
    n = gsize[0]
    with _err():
        alphas_grad[:n] = deactivation((-gradient[:n] * log_probs[:n]).astype(F32), outputs[:n], activation)


def SAC_OutputGradient(quantiles, delta_taus, output_gr, quantiles_gr, taus_gr, output, count_quants, activation,
                       gsize, lsize=None):
    """NeuroNet.cl:3957-4000: the gradient goes to the largest activated quantile at or below the
    action and the smallest above it; every other quantile and tau gradient is zero."""
    n, cq = gsize[0], count_quants
    with _err():
        for a in range(n):
            sh = a * cq
            q = f_activation(quantiles[sh:sh + cq], activation)
            v = output[a]
            q1, q2, p1, p2 = F32(-1e37), F32(1e37), -1, -1
            for k in range(cq):
                if v >= q[k] and q1 < q[k]:
                    q1, p1 = q[k], sh + k
                if v < q[k] and q2 > q[k]:
                    q2, p2 = q[k], sh + k
            quantiles_gr[sh:sh + cq] = 0
            taus_gr[sh:sh + cq] = 0
            g = F32(output_gr[a])
            if q1 > F32(-1e37):
                quantiles_gr[p1] = g * delta_taus[p1]
                taus_gr[p1] = g * q1
            if q2 < F32(1e37):
                quantiles_gr[p2] = g * delta_taus[p2]
                taus_gr[p2] = g * q2


def SAC_CalcLogProbs(outputs, quantiles, probs, alphas, log_probs, count_quants, activation, gsize, lsize=None):
    """NeuroNet.cl:4006-4036: p interpolated between the quantiles bracketing the action, clamped
    to [1e-3, 1], and -alpha log p."""
    n, cq = gsize[0], count_quants
    with _err():
        for i in range(n):
            sh = i * cq
            q = f_activation(quantiles[sh:sh + cq], activation)
            v = outputs[i]
            q1, q2, pr1, pr2 = F32(-1e37), F32(1e37), F32(0), F32(0)
            for k in range(cq):
                if v >= q[k] and q1 < q[k]:
                    q1, pr1 = q[k], probs[sh + k]
                if v < q[k] and q2 > q[k]:
                    q2, pr2 = q[k], probs[sh + k]
            prob = F32(np.abs(F32(v - q1)) / np.abs(F32(q2 - q1)))
            prob = cl_clamp(F32((F32(1) - prob) * pr1) + F32(prob * pr2), 1.0e-3, 1.0)
            log_probs[i] = -alphas[i] * np.log(prob)


# ------------------------------------------------------------ flash attention
def _flash_blocks(query, key_value, Q, KV, H, D):
    q = query[:Q * H * D].reshape(Q, H, D)
    kv = key_value[:KV * 2 * H * D].reshape(KV, 2 * H, D)
    return q, kv[:, :H, :], kv[:, H:, :]


def _flash_visible(Q, KV, mask_future):
    """Which keys each query sees: all, or with mask_future the keys k >= q (NeuroNet.cl:16096)."""
    if not mask_future:
        return np.ones((Q, KV), bool)
    return np.arange(Q)[:, None] <= np.arange(KV)[None, :]


def MHFlashAttention(query, key_value, logsumexp, output, dimension, total_kv, mask_future, gsize, lsize=None):
    """NeuroNet.cl:16066-16177 over global (queries, local, heads): softmax over the visible keys of
    q.k / sqrt(d), the score summing IsNaNOrInf(dot) over float4 groups of sanitised features;
    out = sum IsNaNOrInf(p v) / sum p for the first `local` features and logsumexp = max + log(sum p);
    rows that see no key get 0."""
    Q, loc, H = (tuple(gsize) + (1, 1))[:3]
    D, KV = dimension, total_kv
    with _err():
        q, k, v = _flash_blocks(query, key_value, Q, KV, H, D)
        Dp = (D + 3) // 4 * 4
        qp = np.zeros((Q, H, Dp), F32)
        kp = np.zeros((KV, H, Dp), F32)
        qp[:, :, :D], kp[:, :, :D] = nan0(q), nan0(k)
        prod = (qp[:, None, :, :] * kp[None, :, :, :]).astype(F32)          # [q][k][h][d]
        groups = nan0(prod.reshape(Q, KV, H, Dp // 4, 4).sum(axis=-1, dtype=F32))
        s = (groups.sum(axis=-1, dtype=F32) / np.sqrt(F32(D))).astype(F32)  # [q][k][h]
        valid = np.broadcast_to(_flash_visible(Q, KV, mask_future)[:, :, None], s.shape)
        m = np.where(valid, s, -np.inf).max(axis=1, initial=-np.inf)        # [q][h]
        seen = np.isfinite(m)
        m0 = np.where(seen, m, 0).astype(F32)
        p = np.where(valid, np.exp((s - m0[:, None, :]).astype(F32)), F32(0)).astype(F32)
        sumexp = p.sum(axis=1, dtype=F32)
        out = nan0(p[:, :, :, None] * v.astype(F32)[None, :, :, :]).sum(axis=1, dtype=F32)
        ok = seen & (sumexp > 0)
        den = np.where(ok, sumexp, F32(1)).astype(F32)
        res = np.where(ok[:, :, None], nan0(out / den[:, :, None]), F32(0)).astype(F32)
        w = min(D, loc)
        o = output[:Q * H * D].reshape(Q, H, D)
        o[:, :, :w] = res[:, :, :w]
        logsumexp[:Q * H] = np.where(ok, nan0(m0 + np.log(den)), F32(0)).astype(F32).reshape(-1)


def MHFlashAttentionGrad(query, query_gr, key_value, key_value_gr, logsumexp, output, output_gr, dimension,
                         total_q, total_kv, mask_future, gsize, lsize=None):
    """NeuroNet.cl:16182-16277 over global (rows, d, heads): p = IsNaNOrInf(exp(clamp(s - lse, -120,
    0))) with s = sum IsNaNOrInf(q k) / sqrt(d); pairs the query cannot see or with p == 0 are
    skipped; ds = IsNaNOrInf(p (g.v - g.o)); grad_q = sum_k k ds, grad_k = sum_q q ds,
    grad_v = sum_q p g, every product and sum sanitised; written for the first `rows` queries and
    keys."""
    rows, D, H = (tuple(gsize) + (1, 1))[:3]
    Qt, KVt = total_q, total_kv
    with _err():
        q, k, v = _flash_blocks(query, key_value, Qt, KVt, H, D)
        q, k, v = nan0(q), nan0(k), nan0(v)
        g = nan0(output_gr[:Qt * H * D].reshape(Qt, H, D))
        o = nan0(output[:Qt * H * D].reshape(Qt, H, D))
        lse = nan0(logsumexp[:Qt * H].reshape(Qt, H))
        Dq = nan0(g * o).sum(axis=-1, dtype=F32)                                    # [q][h]
        s = (nan0(q[:, None] * k[None, :]).sum(axis=-1, dtype=F32) / np.sqrt(F32(D))).astype(F32)
        p = nan0(np.exp(cl_clamp(s - lse[:, None, :], -120.0, 0.0)))                # [q][k][h]
        use = _flash_visible(Qt, KVt, mask_future)[:, :, None] & (p != 0)
        dp = nan0(g[:, None] * v[None, :]).sum(axis=-1, dtype=F32)
        ds = np.where(use, nan0(p * (dp - Dq[:, None, :])), F32(0)).astype(F32)
        gq = nan0(nan0(k[None, :] * ds[..., None]).sum(axis=1, dtype=F32))          # [q][h][d]
        gk = nan0(nan0(q[:, None] * ds[..., None]).sum(axis=0, dtype=F32))          # [k][h][d]
        pg = np.where(use[..., None], nan0(p[..., None] * g[:, None]), F32(0)).astype(F32)
        gv = nan0(pg.sum(axis=0, dtype=F32))
        nq, nk = min(rows, Qt), min(rows, KVt)
        query_gr[:nq * H * D] = gq[:nq].reshape(-1)
        kvg = key_value_gr[:KVt * 2 * H * D].reshape(KVt, 2 * H, D)
        kvg[:nk, :H] = gk[:nk]
        kvg[:nk, H:] = gv[:nk]


# ------------------------------------------------------- general matrix products
def _seq_sum(p, axis):
    """Sequential float32 sums along `axis` (the reference's loop order) and their running values."""
    if p.shape[axis] == 0:
        shape = list(p.shape)
        del shape[axis]
        return np.zeros(shape, F32), np.ones(shape, bool)
    cs = np.cumsum(p, axis=axis, dtype=F32)
    return np.take(cs, -1, axis=axis), np.isfinite(cs).all(axis=axis)


def MatMult(matr1, matr2, result, dimension, multvarsecond, offset_matr1, offset_matr2, offset_result,
            numeric_flags, flags_enabled, gsize, lsize=None):
    """NeuroNet.cl:5969-6013 over global (rows, cols, variables): result[v] = matr1[v] . matr2[v or 0],
    every product through IsNaNOrInf(., 0) and summed in order; with flags_enabled,
    numeric_flags[v][row][col] = 1 where an operand, a product or the running sum was not finite."""
    rows, cols, var = (tuple(gsize) + (1, 1))[:3]
    dim, mvs = dimension, 1 if multvarsecond else 0
    with _err():
        for v in range(var):
            a = matr1[offset_matr1 + v * rows * dim:][:rows * dim].reshape(rows, dim)
            b = matr2[offset_matr2 + mvs * v * dim * cols:][:dim * cols].reshape(dim, cols)
            p = (a[:, :, None] * b[None, :, :]).astype(F32)           # [row][i][col]
            fin = np.isfinite(p)
            res, run_ok = _seq_sum(np.where(fin, p, F32(0)).astype(F32), 1)
            result[offset_result + v * rows * cols:][:rows * cols] = res.reshape(-1)
            if flags_enabled:
                operands_ok = (np.isfinite(a)[:, :, None] & np.isfinite(b)[None, :, :]).all(axis=1)
                invalid = ~(operands_ok & fin.all(axis=1) & run_ok & np.isfinite(res))
                numeric_flags[v * rows * cols:(v + 1) * rows * cols] = invalid.reshape(-1).astype(F32)


def MatMultGrad(matr1, matr1_gr, matr2, matr2_gr, result_gr, dimension, multvarsecond, offset_matr1,
                offset_matr1_gr, offset_matr2, offset_matr2_gr, offset_result_gr, gsize, lsize=None):
    """NeuroNet.cl:6018-6060 over global (rows, cols, variables): matr1_gr[v] = result_gr[v] .
    matr2[v]^T and matr2_gr = matr1[v]^T . result_gr[v] (summed over every variable, into the one
    shared matrix, when multvarsecond is 0); products and sums through IsNaNOrInf(., 0)."""
    rows, cols, var = (tuple(gsize) + (1, 1))[:3]
    dim, mvs = dimension, 1 if multvarsecond else 0
    with _err():
        def blocks(v):
            a = matr1[offset_matr1 + v * rows * dim:][:rows * dim].reshape(rows, dim)
            b = matr2[offset_matr2 + mvs * v * dim * cols:][:dim * cols].reshape(dim, cols)
            g = result_gr[offset_result_gr + v * rows * cols:][:rows * cols].reshape(rows, cols)
            return a, b, g
        for v in range(var):
            a, b, g = blocks(v)
            p = (g[:, None, :] * b[None, :, :]).astype(F32)          # [row][feature][i]
            s, _ = _seq_sum(nan0(p), 2)
            matr1_gr[offset_matr1_gr + v * rows * dim:][:rows * dim] = nan0(s).reshape(-1)
        for v in (range(var) if mvs else [0]):
            parts = [blocks(v)] if mvs else [blocks(u) for u in range(var)]
            a = np.concatenate([q[0] for q in parts], axis=0)             # [(v,) i][feature]
            g = np.concatenate([q[2] for q in parts], axis=0)             # [(v,) i][col]
            p = (a.T[:, :, None] * g[None, :, :]).astype(F32)          # [feature][i][col]
            s, _ = _seq_sum(nan0(p), 1)
            matr2_gr[offset_matr2_gr + v * dim * cols:][:dim * cols] = nan0(s).reshape(-1)


# ------------------------------------------------ masking and patch embedding
def Dropout(inputs, map, out, dimension, gsize, lsize=None):
    """NeuroNet.cl:1855-1884 as written: work-item t = 0 .. gsize[0]-1 loops k over
    [4t, min(dimension, 4t + 4)) and uses element 4t + k, i.e. 8t + j for j < 4 with 4t + j <
    dimension; out = 0 where IsNaNOrInf(map) or IsNaNOrInf(input) is 0, else IsNaNOrInf(inp * m).
    Elements the reference would touch past the end of the arrays are left out."""
    G = gsize[0]
    lim = min(len(inputs), len(map), len(out))
    t = np.arange(G)[:, None]
    j = np.arange(4)[None, :]
    e = (8 * t + j)[(4 * t + j) < dimension]
    e = e[e < lim]
    with _err():
        m = nan0(map[e])
        x = nan0(inputs[e])
        out[e] = np.where((m == 0) | (x == 0), F32(0), nan0(x * m)).astype(F32)


def PatchCreate(inputs, weights, outputs, inputs_total, window_in, step, activation, gsize, lsize=None):
    """NeuroNet.cl:5826-5860 over global (patches, window_out, variables): output (i*variables + v)
    * window_out + w = fActivation(bias + sum_p x[(i*step + p)*variables + v] W[p]) over the p whose
    input index is below inputs_total, W the row (window_in + 1)(v*window_out + w) (bias last); a NaN
    sum becomes 0."""
    P, WO, V = (tuple(gsize) + (1, 1))[:3]
    with _err():
        Wt = weights[:V * WO * (window_in + 1)].reshape(V, WO, window_in + 1)
        for i in range(P):
            for v in range(V):
                idx = i * step * V + v + np.arange(window_in) * V
                ok = idx < inputs_total
                x = np.where(ok, inputs[np.minimum(idx, max(inputs_total - 1, 0))], F32(0)).astype(F32)
                res = (Wt[v, :, window_in] + (Wt[v, :, :window_in] * x[None, :]).sum(axis=1, dtype=F32)).astype(F32)
                res = np.where(np.isnan(res), F32(0), res).astype(F32)
                outputs[(i * V + v) * WO:(i * V + v + 1) * WO] = f_activation(res, activation)


def PatchHiddenGradient(inputs, inputs_gr, weights, outputs_gr, window_in, step, window_out, outputs_total,
                        activation, gsize, lsize=None):
    """NeuroNet.cl:5864-5911 over global (time, variables): input (i, v) collects
    outputs_gr[(row*variables + v)*window_out + wo] * W[v][wo][w_start + (total-p-1)*step] over the
    patches row = r_start + p below outputs_total, with the reference's w_start = i % step, r_start =
    max((i - window_in + step) / step, 0) and total = min((i + step) / step, (window_in - w_start +
    step - 1) / step) (C division, truncating toward zero), then Deactivation by the input."""
    T, V = (tuple(gsize) + (1,))[:2]

    def cdiv(a, b):
        q = abs(a) // abs(b)
        return q if (a >= 0) == (b > 0) else -q
    with _err():
        Wt = weights[:V * window_out * (window_in + 1)].reshape(V, window_out, window_in + 1)
        for i in range(T):
            w_start = i % step
            r_start = max(cdiv(i - window_in + step, step), 0)
            total = min(cdiv(i + step, step), cdiv(window_in - w_start + step - 1, step))
            for v in range(V):
                grad = F32(0)
                for p in range(max(total, 0)):
                    row = r_start + p
                    if row >= outputs_total:
                        break
                    g = outputs_gr[(row * V + v) * window_out:(row * V + v + 1) * window_out]
                    wcol = Wt[v, :, w_start + (total - p - 1) * step]
                    grad = F32(grad + (g * wcol).sum(dtype=F32))
                inputs_gr[i * V + v] = deactivation(grad, inputs[i * V + v], activation)


def FQF_Sample(quantiles, probabilities, random, result, gsize, lsize=None):
    """NeuroNet.cl:2722-2799, one work-group per task (local size = quants): C = the Hillis-Steele
    inclusive scan of max(IsNaNOrInf(p), 0) (Temp[i] += Temp[i - d] for d = 1, 2, 4, ... below the
    row length, each step reading the previous step's values); 0 when IsNaNOrInf(C_last) <= 1e-6,
    else the quantile of the smallest i with C_i >= u*C_last and (i == 0 or C_{i-1} < u*C_last), the
    last one when its C is below u*C_last, u = clamp(IsNaNOrInf(random, 0.5), 0, 1)."""
    T = lsize[0] if lsize is not None else gsize[0]
    R = (tuple(gsize) + (1,))[1]
    with _err():
        for r in range(R):
            c = np.maximum(nan0(probabilities[r * T:(r + 1) * T]), F32(0)).astype(F32)
            d = 1
            while d < T:
                c = np.concatenate([c[:d], (c[d:] + c[:-d]).astype(F32)]).astype(F32)
                d <<= 1
            mass = nan0(c[T - 1])
            if mass <= F32(1e-6):
                result[r] = 0
                continue
            u = F32(min(max(float(nan0(random[r], 0.5)), 0.0), 1.0))
            thr = F32(u * mass)
            prev = np.concatenate([[F32(0)], c[:-1]]).astype(F32)
            sel = (c >= thr) & ((np.arange(T) == 0) | (prev < thr))
            if c[T - 1] < thr:
                sel[T - 1] = True
            hit = np.nonzero(sel)[0]
            if len(hit):
                result[r] = nan0(quantiles[r * T + hit[0]])


# --------------------------------------------------------- soft actor-critic
# The library's squashed-Gaussian SAC kernels (no reference counterpart; the reference's SAC agents
# use quantile heads).  A launch covers gsize[0] * batch samples; here gsize[0] is the sample count.
# kernels the library defines beyond the reference (no reference output pins them; their tests are
# known answers and a finite-difference check of the policy gradient)
LIBRARY_KERNELS = {"SACGaussianPolicy", "SACTargetValue", "SACPolicyGradient"}
LOG_STD_MIN, LOG_STD_MAX = F32(-20.0), F32(2.0)
HALF_LOG_2PI = F32(0.5 * np.log(2.0 * np.pi))
SQUASH_EPS = F32(1e-6)


def SACGaussianPolicy(outputs, noise, actions, log_probs, action_dim, gsize, lsize=None):
    """a = tanh(mu + exp(clamp(log_std, -20, 2)) eps); log pi = sum_j (-eps^2/2 - log_std - log(2 pi)/2
    - log(1 - a^2 + 1e-6)) with outputs [n][2A] = (mu, log_std)."""
    n, A = gsize[0], action_dim
    with _err():
        o = outputs[:n * 2 * A].reshape(n, 2 * A)
        ls = cl_clamp(o[:, A:], LOG_STD_MIN, LOG_STD_MAX)
        e = noise[:n * A].reshape(n, A)
        a = np.tanh((o[:, :A] + np.exp(ls) * e).astype(F32)).astype(F32)
        actions[:n * A] = a.reshape(-1)
        lp = (F32(-0.5) * e * e - ls - HALF_LOG_2PI - np.log(F32(1) - a * a + SQUASH_EPS)).astype(F32)
        log_probs[:n] = lp.sum(axis=1, dtype=F32)


def SACTargetValue(q1, q2, reward, done, log_probs, target, gamma, alpha, gsize, lsize=None):
    """y = r + gamma (1 - done) (min(q1, q2) - alpha log pi)."""
    n = gsize[0]
    with _err():
        target[:n] = (reward[:n] + F32(gamma) * (F32(1) - done[:n])
                      * (np.minimum(q1[:n], q2[:n]) - F32(alpha) * log_probs[:n])).astype(F32)


def SACPolicyGradient(outputs, noise, actions, q1, q2, dq1, dq2, gradient, action_dim, alpha, gsize, lsize=None):
    """Ascent direction of J = min(q1, q2) - alpha log pi for (mu, log_std), dq of the smaller critic,
    each entry clamped to +-MAX_GRAD: s = dq (1 - a^2) - alpha 2a(1 - a^2)/(1 - a^2 + 1e-6);
    dJ/dmu = s; dJ/dlog_std = s exp(log_std) eps + alpha strictly inside (-20, 2), else 0."""
    n, A = gsize[0], action_dim
    with _err():
        o = outputs[:n * 2 * A].reshape(n, 2 * A)
        a = actions[:n * A].reshape(n, A)
        e = noise[:n * A].reshape(n, A)
        dq = np.where((q1[:n] <= q2[:n])[:, None], dq1[:n * A].reshape(n, A), dq2[:n * A].reshape(n, A))
        one = (F32(1) - a * a).astype(F32)
        sgr = (dq * one - F32(alpha) * F32(2) * a * one / (one + SQUASH_EPS)).astype(F32)
        ls_raw = o[:, A:]
        ls = cl_clamp(ls_raw, LOG_STD_MIN, LOG_STD_MAX)
        g = gradient[:n * 2 * A].reshape(n, 2 * A)
        g[:, :A] = cl_clamp(nan0(sgr), -MAX_GRAD, MAX_GRAD)
        inside = (ls_raw > LOG_STD_MIN) & (ls_raw < LOG_STD_MAX)
        g[:, A:] = np.where(inside, cl_clamp(nan0(sgr * np.exp(ls) * e + F32(alpha)), -MAX_GRAD, MAX_GRAD), F32(0))


KERNELS = {name: fn for name, fn in globals().items()
           if callable(fn) and name[:1].isupper() and fn.__module__ == __name__}


def launch(name, gsize, lsize, args):
    """Run restated kernel `name` with the reference argument list and NDRange."""
    KERNELS[name](*args, gsize=tuple(gsize), lsize=None if lsize is None else tuple(lsize))
