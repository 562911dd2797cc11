"""Dropout, the patch kernels and FQF_Sample through the C ABI, beyond the golden cases: the
buffer sizes the reference's host really allocates, batches, and the calls the library refuses."""
import numpy as np
import pytest

from oracle import kernels as K
from tests.parity import check_close

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("D", [1, 5, 64, 1000, 4099])
def test_dropout_with_buffers_of_exactly_the_dimension(ctx, D):
    """CNeuronDropoutOCL sizes input, map and output to the layer (NeuroNet_Core.mqh:19150-19176);
    the reference's work-items then reach past the end.  Inside the buffers the result is the
    reference's (elements 8t .. 8t+3 written, 8t+4 .. 8t+7 kept), nothing is written outside."""
    rng = np.random.default_rng(D)
    x = rng.standard_normal(D).astype(np.float32)
    m = np.where(rng.uniform(size=D) < 0.3, 0.0, 1 / 0.7).astype(np.float32)
    y0 = rng.standard_normal(D).astype(np.float32)  # what the output held before
    hx, hm, hy = ctx.buffer(D), ctx.buffer(D), ctx.buffer(D)
    ctx.write(hx, x)
    ctx.write(hm, m)
    ctx.write(hy, y0)
    ctx.kernel("Dropout").args(hx, hm, hy, D).run(((D + 3) // 4,))
    want = y0.copy()
    K.Dropout(x, m, want, D, gsize=((D + 3) // 4,))
    np.testing.assert_array_equal(ctx.read(hy, D), want)
    for h in (hx, hm, hy):
        ctx.free(h)


def test_dropout_batched_keeps_each_sample_to_its_own_elements(ctx):
    D, B = 37, 4
    rng = np.random.default_rng(3)
    x = rng.standard_normal(B * D).astype(np.float32)
    m = np.where(rng.uniform(size=B * D) < 0.3, 0.0, 1 / 0.7).astype(np.float32)
    y0 = rng.standard_normal(B * D).astype(np.float32)
    hx, hm, hy = ctx.buffer(B * D), ctx.buffer(B * D), ctx.buffer(B * D)
    ctx.write(hx, x)
    ctx.write(hm, m)
    ctx.write(hy, y0)
    ctx.kernel("Dropout").args(hx, hm, hy, D).batch(B).run(((D + 3) // 4,))
    got = ctx.read(hy, B * D)
    for b in range(B):
        want = y0[b * D:(b + 1) * D].copy()
        K.Dropout(x[b * D:(b + 1) * D], m[b * D:(b + 1) * D], want, D, gsize=((D + 3) // 4,))
        np.testing.assert_array_equal(got[b * D:(b + 1) * D], want)
    for h in (hx, hm, hy):
        ctx.free(h)


def test_dropout_refuses_buffers_below_the_dimension(ctx):
    hx, hm, hy = ctx.buffer(10), ctx.buffer(10), ctx.buffer(5)
    k = ctx.kernel("Dropout").args(hx, hm, hy, 10)
    with pytest.raises(Exception) as e:
        k.run((3,))
    assert "-5" in str(e.value)
    for h in (hx, hm, hy):
        ctx.free(h)


def test_patch_update_weights_adam_is_refused_with_a_reason(ctx):
    hs = [ctx.buffer(64) for _ in range(5)]
    k = ctx.kernel("PatchUpdateWeightsAdam").args(*hs, 32, 3e-4, 0.9, 0.999, 4)
    with pytest.raises(Exception) as e:
        k.run((5, 4, 2))
    assert "-9" in str(e.value) and "undefined" in str(e.value)
    for h in hs:
        ctx.free(h)


@pytest.mark.parametrize("T,R", [(64, 4096), (17, 1000), (1, 7)])
def test_fqf_sample_full_size(ctx, T, R):
    """Many rows at once; probabilities are a softmax (the cSoftMax output the host binds)."""
    rng = np.random.default_rng(T * 31 + R)
    z = rng.standard_normal(R * T).astype(np.float32)
    e = np.exp(rng.standard_normal((R, T)))
    p = (e / e.sum(axis=1, keepdims=True)).astype(np.float32).reshape(-1)
    u = rng.uniform(size=R).astype(np.float32)
    hq, hp, hu, hr = ctx.buffer(R * T), ctx.buffer(R * T), ctx.buffer(R), ctx.buffer(R)
    ctx.write(hq, z)
    ctx.write(hp, p)
    ctx.write(hu, u)
    ctx.kernel("FQF_Sample").args(hq, hp, hu, hr).run((T, R), (T, 1))
    want = np.zeros(R, np.float32)
    K.FQF_Sample(z, p, u, want, gsize=(T, R), lsize=(T, 1))
    np.testing.assert_array_equal(ctx.read(hr, R), want)
    for h in (hq, hp, hu, hr):
        ctx.free(h)


def test_fqf_sample_refuses_more_than_64_quants(ctx):
    hq, hp, hu, hr = ctx.buffer(65 * 2), ctx.buffer(65 * 2), ctx.buffer(2), ctx.buffer(2)
    k = ctx.kernel("FQF_Sample").args(hq, hp, hu, hr)
    with pytest.raises(Exception) as e:
        k.run((65, 2), (65, 1))
    assert "-9" in str(e.value)
    for h in (hq, hp, hu, hr):
        ctx.free(h)


@pytest.mark.parametrize("T,V,win,step,WO", [(512, 32, 16, 8, 128), (100, 7, 12, 5, 9)])
def test_patch_create_and_hidden_gradient_full_size(ctx, T, V, win, step, WO):
    """The PatchTST-style patching shape (32 channels x 512 bars, window 16, stride 8, embed 128)."""
    rng = np.random.default_rng(T + V)
    P = (T - win) // step + 1
    nw = V * WO * (win + 1)
    x = rng.standard_normal(T * V).astype(np.float32)
    w = rng.uniform(-0.25, 0.25, nw).astype(np.float32)
    g = (rng.standard_normal(P * V * WO) * 0.01).astype(np.float32)
    hx, hw, hy, hg, hig = ctx.buffer(T * V), ctx.buffer(nw), ctx.buffer(P * V * WO), ctx.buffer(P * V * WO), \
        ctx.buffer(T * V)
    ctx.write(hx, x)
    ctx.write(hw, w)
    ctx.write(hg, g)
    ctx.kernel("PatchCreate").args(hx, hw, hy, T * V, win, step, K.TANH).run((P, WO, V))
    y = np.zeros(P * V * WO, np.float32)
    K.PatchCreate(x, w, y, T * V, win, step, K.TANH, gsize=(P, WO, V))
    check_close("PatchCreate", ctx.read(hy, P * V * WO), y)
    xa = np.tanh(x).astype(np.float32)
    ctx.write(hx, xa)
    ctx.kernel("PatchHiddenGradient").args(hx, hig, hw, hg, win, step, WO, P, K.TANH).run((T, V))
    ig = np.zeros(T * V, np.float32)
    K.PatchHiddenGradient(xa, ig, w, g, win, step, WO, P, K.TANH, gsize=(T, V))
    check_close("PatchHiddenGradient", ctx.read(hig, T * V), ig)
    for h in (hx, hw, hy, hg, hig):
        ctx.free(h)
