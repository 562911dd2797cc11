"""Kernel-level parity of the CUDA library, called through the C ABI.

Every golden case (the reference's own NeuroNet.cl kernels, compiled for the
CPU, on seeded inputs) is replayed through libnn_b200.so with the same
positional arguments and NDRange; every array argument is compared after the
launch.  Batched executions (nn_set_batch) are checked sample by sample
against the numpy oracle.
"""
import os

import numpy as np
import pytest

from oracle import kernels as K
from tests.golden.cases import A, all_cases, prepare_inputs
from tests.golden.make_golden import case_seed
from tests.parity import check_close

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "kernels.npz")
CASES = all_cases()


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


def run_on_gpu(ctx, kernel, args, gsize, lsize, batch=1):
    """Upload array args, bind, execute, read back. Returns list of arrays (None for scalars)."""
    k = ctx.kernel(kernel)
    handles = []
    for i, a in enumerate(args):
        if isinstance(a, np.ndarray):
            h = ctx.buffer(a.size)
            ctx.write(h, a)
            handles.append(h)
            k.set(i, h)
        else:
            handles.append(None)
            k.set(i, a)
    if batch != 1:
        k.batch(batch)
    k.run(gsize, lsize)
    out = []
    for i, a in enumerate(args):
        if isinstance(a, np.ndarray):
            out.append(ctx.read(handles[i], a.size))
            ctx.free(handles[i])
        else:
            out.append(None)
    ctx.lib.nn_kernel_free(k.id)
    return out


@pytest.mark.parametrize("case", CASES, ids=[c.name for c in CASES])
def test_kernel_matches_reference(ctx, case, golden):
    args = prepare_inputs(case, case_seed(case.name))
    before = [a.copy() if isinstance(a, np.ndarray) else None for a in args]
    got = run_on_gpu(ctx, case.kernel, args, case.gsize, case.lsize)
    for i, a in enumerate(args):
        if isinstance(a, np.ndarray):
            check_close(f"{case.name} arg{i}", got[i], golden[f"{case.name}|out{i}"], before[i])


# ---------------------------------------------------------------- batched
PER_SAMPLE_KERNELS = {
    # kernel: indices of per-sample array arguments (the rest are shared parameters)
    "FeedForward": [1, 2], "CalcHiddenGradient": [1, 2, 3], "CalcOutputGradient": [0, 1, 2],
    "Activation": [0, 1], "DeActivation": [0, 1, 2], "FeedForwardConv": [1, 2],
    "CalcHiddenGradientConv": [1, 2, 3], "MHAttentionScore": [0, 1], "MHAttentionOut": [0, 1, 2],
    "MHAttentionInsideGradients": [0, 1, 2, 3], "SumMatrix": [0, 1, 2, 8], "Normalize": [0],
    "SoftMax_FeedForward": [0, 1], "SoftMax_HiddenGradient": [0, 1, 2], "SoftMax_OutputGradient": [0, 1, 2],
    "Transpose": [0, 1], "RevInFeedForward": [0, 2], "RevInHiddenGraddient": [0, 1, 3],
    "FQF_Cosine": [0, 1], "FQF_Output": [0, 1, 2], "FQF_OutputGradient": [0, 1, 2, 3, 4],
    "FQF_QuantileGradient": [0, 1, 2, 3, 4], "FQF_CosineGradient": [0, 1, 2], "FQF_FractionGradient": [1, 2],
    "FQF_CosineGradientSRM": [0, 1, 2], "FQF_DistributionTargetGradient": [0, 1, 2, 3],
    "FQF_MonotoneRearrange": [0, 1, 2, 3, 4, 5], "FQF_RearrangeGradient": [0, 1, 2, 3, 4],
    "FQF_SRMForward": [0, 1, 2], "FQF_SRMGradient": [0, 1, 2, 3, 4],
    "SAC_AlphaLogProbs": [0, 1, 2, 3, 4, 5], "SAC_AlphaGradients": [0, 1, 2, 3],
    "SAC_OutputGradient": [0, 1, 2, 3, 4, 5], "SAC_CalcLogProbs": [0, 1, 2, 3, 4],
    "MHFlashAttention": [0, 1, 2, 3], "MHFlashAttentionGrad": [0, 1, 2, 3, 4, 5, 6],
    "PatchCreate": [0, 2], "PatchHiddenGradient": [0, 1, 3], "FQF_Sample": [0, 1, 2, 3],
}
BATCH_CASES = [c for c in CASES if c.kernel in PER_SAMPLE_KERNELS]


@pytest.mark.parametrize("case", BATCH_CASES, ids=[c.name for c in BATCH_CASES])
def test_batched_kernel_matches_per_sample_oracle(ctx, case):
    B = 3
    per = PER_SAMPLE_KERNELS[case.kernel]
    samples = [prepare_inputs(case, case_seed(case.name) + 17 * s) for s in range(B)]
    # shared parameters come from sample 0
    batched = []
    for i, a in enumerate(samples[0]):
        if isinstance(a, np.ndarray) and i in per:
            batched.append(np.concatenate([s[i] for s in samples]))
        else:
            batched.append(a.copy() if isinstance(a, np.ndarray) else a)
    got = run_on_gpu(ctx, case.kernel, batched, case.gsize, case.lsize, batch=B)
    for s in range(B):
        args = [samples[s][i] if i in per else (batched[i].copy() if isinstance(batched[i], np.ndarray)
                                                  else batched[i]) for i in range(len(batched))]
        K.launch(case.kernel, case.gsize, case.lsize, args)
        for i in per:
            n = samples[s][i].size
            check_close(f"{case.name} sample{s} arg{i}", got[i][s * n:(s + 1) * n], args[i])


UPDATE_CASES = [c for c in CASES if c.kernel in ("UpdateWeightsAdam", "UpdateWeightsConvAdam",
                                                   "UpdateWeightsMomentum", "UpdateWeightsConvMomentum")]


def batched_update_oracle(case, samples, shared):
    """Reference update arithmetic applied once to the batch-mean weight gradient."""
    B = len(samples)
    k = case.kernel
    w, m = shared[0].copy(), shared[3].copy()
    if k == "UpdateWeightsAdam":
        n_out, n_col = case.gsize
        inputs = shared[5]
        grads = []
        for s in samples:
            x = s[2]
            inp = K.nan0(np.where(np.arange(n_col) == inputs, 1.0, x[np.minimum(np.arange(n_col), inputs - 1)]))
            grads.append(K.nan0(s[1][:n_out, None] * inp[None, :]))
        G = np.mean(grads, axis=0, dtype=np.float64).astype(np.float32)
        v = shared[4].copy()
        K.adam_dense_apply(w, G, m, v, inputs, shared[6], shared[7], shared[8], n_out, n_col)
        return {0: w, 3: m, 4: v}
    if k == "UpdateWeightsConvAdam":
        n = case.gsize[0]
        inputs, win, wout, step = shared[5], shared[9], shared[10], shared[11]
        G = np.mean([K.conv_weight_grad(s[1], s[2], inputs, win, wout, step, n) for s in samples], axis=0,
                    dtype=np.float64).astype(np.float32)
        v = shared[4].copy()
        K.adam_conv_apply(w, G, m, v, shared[6], shared[7], shared[8], n)
        return {0: w, 3: m, 4: v}
    if k == "UpdateWeightsMomentum":
        n_out, n_col = case.gsize
        inputs, lr, mom = shared[4], np.float32(shared[5]), np.float32(shared[6])
        grads = []
        for s in samples:
            x = s[2]
            xj = np.where(np.arange(n_col) < inputs, x[np.minimum(np.arange(n_col), inputs - 1)], 1.0)
            grads.append(K.cl_clamp(s[1][:n_out], -K.MAX_GRAD, K.MAX_GRAD)[:, None] * xj[None, :])
        G = np.mean(grads, axis=0, dtype=np.float64).astype(np.float32)
        idx = np.arange(n_out)[:, None] * (inputs + 1) + np.arange(n_col)[None, :]
        delta = K.nan0(lr * G) + K.nan0(mom * m[idx])
        m[idx] = delta
        w[idx] = np.where(np.abs(delta) > 0, K.nan0(w[idx] + delta), w[idx])
        return {0: w, 3: m}
    # UpdateWeightsConvMomentum
    n = case.gsize[0]
    inputs, win, wout, step = shared[4], shared[7], shared[8], shared[9]
    G = np.mean([K.conv_weight_grad(s[1], s[2], inputs, win, wout, step, n, momentum_variant=True)
                 for s in samples], axis=0, dtype=np.float64).astype(np.float32)
    delta = K.nan0(np.float32(shared[5]) * G) + np.float32(shared[6]) * m[:n]
    ok = ~np.isnan(delta)
    m[:n] = np.where(ok, delta, m[:n])
    w[:n] = np.where(ok & (np.abs(delta) > 0), K.nan0(w[:n] + delta), w[:n])
    return {0: w, 3: m}


@pytest.mark.parametrize("case", UPDATE_CASES, ids=[c.name for c in UPDATE_CASES])
def test_batched_update_is_mean_gradient_then_reference_update(ctx, case):
    B = 4
    samples = [prepare_inputs(case, case_seed(case.name) + 31 * s) for s in range(B)]
    shared = samples[0]
    batched = [np.concatenate([s[i] for s in samples]) if i in (1, 2) else
               (shared[i].copy() if isinstance(shared[i], np.ndarray) else shared[i]) for i in range(len(shared))]
    before = [a.copy() if isinstance(a, np.ndarray) else None for a in batched]
    got = run_on_gpu(ctx, case.kernel, batched, case.gsize, case.lsize, batch=B)
    ref = batched_update_oracle(case, samples, shared)
    for i, r in ref.items():
        check_close(f"{case.name} arg{i}", got[i], r, before[i])


@pytest.mark.parametrize("opt", [0, 1])
def test_batched_batchnorm_scans_samples_in_order(ctx, opt):
    """Batched BatchFeedForward == consecutive reference calls; the batched backward and option update
    use every sample's own statistics and the batch-mean gamma/beta gradient."""
    rng = np.random.default_rng(11 + opt)
    N, B, batch = 37, 4, 20
    width = 7 if opt == 0 else 9
    x = rng.standard_normal((B, N)).astype(np.float32)
    opts = rng.uniform(0.05, 1.0, N * width).astype(np.float32)
    g = (rng.standard_normal((B, N)) * 0.01).astype(np.float32)
    # oracle: consecutive per-sample calls
    o = opts.copy()
    ys, hist = [], []
    for b in range(B):
        y = np.zeros(N, np.float32)
        K.BatchFeedForward(x[b], o, y, batch, opt, K.TANH, 1, gsize=(N,))
        ys.append(y)
        hist.append(o.reshape(N, width)[:, :3].copy())
    igs = []
    for b in range(B):
        ob = o.copy().reshape(N, width)
        ob[:, :3] = hist[b]
        ig = np.zeros(N, np.float32)
        K.CalcHiddenGradientBatch(ob.reshape(-1), g[b], x[b], ig, K.NONE, batch, opt, gsize=(N,))
        igs.append(ig)
    clamp = K.cl_clamp(K.nan0(g), -K.MAX_GRAD, K.MAX_GRAD)
    Gg = np.mean([clamp[b] * hist[b][:, 2] for b in range(B)], axis=0).astype(np.float32)
    Gb = np.mean(clamp, axis=0).astype(np.float32)
    o_upd = o.copy()
    if opt == 1:
        K.bn_adam_apply(o_upd, Gg, Gb, 3e-4, 0.9, 0.999, N)
    else:
        K.bn_momentum_apply(o_upd, Gg, Gb, 3e-4, 0.9, N)
    # library, batched
    hx, hy, ho, hg, hig = ctx.buffer(B * N), ctx.buffer(B * N), ctx.buffer(N * width), ctx.buffer(B * N), ctx.buffer(B * N)
    ctx.write(hx, x)
    ctx.write(ho, opts)
    ctx.write(hg, g)
    ctx.kernel("BatchFeedForward").args(hx, ho, hy, batch, opt, K.TANH, 1).batch(B).run((N,))
    check_close("bn forward", ctx.read(hy, B * N), np.concatenate(ys))
    check_close("bn options after forward", ctx.read(ho, N * width), o)
    ctx.kernel("CalcHiddenGradientBatch").args(ho, hg, hx, hig, K.NONE, batch, opt).batch(B).run((N,))
    check_close("bn input gradient", ctx.read(hig, B * N), np.concatenate(igs))
    if opt == 1:
        ctx.kernel("UpdateBatchOptionsAdam").args(ho, hg, 3e-4, 0.9, 0.999).batch(B).run((N,))
    else:
        ctx.kernel("UpdateBatchOptionsMomentum").args(ho, hg, 3e-4, 0.9).batch(B).run((N,))
    check_close("bn options after update", ctx.read(ho, N * width), o_upd, o)
    for h in (hx, hy, ho, hg, hig):
        ctx.free(h)


@pytest.mark.parametrize("variables", [1, 3])
def test_conv_adam_mini_variables_take_turns(ctx, variables):
    """UpdateWeightsConvAdamMini with several variables: the per-head second moment is updated by
    each variable in turn (the reference's work-groups race on it), as the oracle defines."""
    inputs, win, step, wout, heads = 200, 20, 10, 16, 4
    total = (inputs - win + step - 1) // step
    rng = np.random.default_rng(40 + variables)
    nw = variables * wout * (win + 1)
    args = [rng.uniform(-0.2, 0.2, nw).astype(np.float32), (rng.standard_normal(variables * total * wout) * 0.01)
            .astype(np.float32), rng.standard_normal(variables * inputs).astype(np.float32),
            (rng.standard_normal(nw) * 1e-3).astype(np.float32), rng.uniform(0, 1e-5, heads).astype(np.float32),
            inputs, 3e-4, 0.9, 0.999, step]
    gsize, lsize = (win + 1, wout, variables), (win + 1, wout // heads, 1)
    before = [a.copy() if isinstance(a, np.ndarray) else None for a in args]
    got = run_on_gpu(ctx, "UpdateWeightsConvAdamMini", [a.copy() if isinstance(a, np.ndarray) else a for a in args],
                     gsize, lsize)
    K.launch("UpdateWeightsConvAdamMini", gsize, lsize, args)
    for i in (0, 3, 4):
        check_close(f"variables{variables} arg{i}", got[i], args[i], before[i])
