"""Training-step parity of whole networks through the C ABI against the oracle's restatement of
the reference host sequencing (oracle/nets.py).

After every step: every layer's output and gradient, and every post-update weight, first and
second moment are compared.  Each step starts from the oracle's state (weights and moments are
copied to the device after the comparison), so that a step is checked on identical inputs and
rounding differences do not compound.  Weights whose update direction is rounding noise are
excluded from the weight comparison (tests/parity.py: `determinate`).
"""
import numpy as np
import pytest

from nn_in_trading_b200 import configs as C
from oracle import kernels as K
from oracle import nets as O
from tests.parity import check_close, check_weights, deactivation_atol

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def numpy_oracle():
    O.use_backend("numpy")


def oracle_dense(spec, batch, weights):
    layers = []
    for i, (n, a) in enumerate(zip(spec.sizes, spec.acts)):
        outputs = spec.sizes[i + 1] if i + 1 < len(spec.sizes) else 0
        layers.append(O.ODense(n, a, batch, outputs))
    for layer, w in zip(layers, weights):
        layer.weights[:] = w
    return O.ONet(layers)


def dense_gradient_floors(onet):
    """Absolute floor of every layer's gradient: its own TANH/SIGMOID quantisation plus the floor of the
    next layer's gradient carried back through |W| (CalcHiddenGradient is sum_k w[k,i] g[k])."""
    L = len(onet.layers)
    floors = [0.0] * L
    for l in range(L - 1, -1, -1):
        ol = onet.layers[l]
        carried = 0.0
        if l + 1 < L and floors[l + 1] > 0:
            n_out = onet.layers[l + 1].neurons
            w = np.abs(ol.weights.reshape(n_out, ol.neurons + 1)[:, :ol.neurons])
            carried = float(w.sum(axis=0).max()) * floors[l + 1]
        floors[l] = deactivation_atol(ol.activation, ol.output) + carried
    return floors


def check_dense_step(ctx, net, onet, step):
    floors = dense_gradient_floors(onet)
    for li, (gl, ol) in enumerate(zip(net.layers, onet.layers)):
        B = gl.batch
        check_close(f"step{step} layer{li} output", ctx.read(gl.output, gl.neurons * B), ol.output.reshape(-1))
        check_close(f"step{step} layer{li} gradient", ctx.read(gl.gradient, gl.neurons * B), ol.gradient.reshape(-1),
                    atol=floors[li])
    for li in range(len(onet.layers) - 1):
        gl, ol, upd = net.layers[li], onet.layers[li], onet.layers[li + 1]
        n = ol.weights.size
        check_weights(f"step{step} layer{li} weights", ctx.read(gl.weights, n), ol.weights, upd.last_grad,
                      upd.last_grad_abs)
        check_close(f"step{step} layer{li} m", ctx.read(gl.m, n), ol.m)
        check_close(f"step{step} layer{li} v", ctx.read(gl.v, n), ol.v)
        ctx.write(gl.weights, ol.weights)
        ctx.write(gl.m, ol.m)
        ctx.write(gl.v, ol.v)


@pytest.mark.parametrize("batch,replay", [(1, False), (1, True), (5, False)])
def test_dense_mlp_training_steps(ctx, batch, replay):
    spec = C.DenseSpec()
    w = C.dense_weights(spec)
    net = C.build_dense(ctx, spec, batch, w)
    onet = oracle_dense(spec, batch, w)
    steps = 6
    xs, ts = C.dense_data(spec, steps, batch)
    if replay:
        net.capture()
    for s in range(steps):
        net.set_input(xs[s])
        net.set_target(ts[s])
        net.step()
        onet.step(xs[s], ts[s])
        check_dense_step(ctx, net, onet, s)


def oracle_mlmh(spec, batch, weights):
    inp = O.ODense(spec.window * spec.units, K.NONE, batch, 0)
    enc = O.OMLMH(spec.window, spec.dk, spec.heads, spec.units, spec.layers, spec.activation, batch)
    for i, ws in enumerate(weights):
        for name, w in ws.items():
            enc.w[i][name][0][:] = w
    return O.ONet([inp, enc])


def check_mlmh_step(ctx, net, onet, step):
    g_in, o_in = net.layers[0], onet.layers[0]
    g_enc, o_enc = net.layers[1], onet.layers[1]
    B = g_in.batch
    check_close(f"step{step} encoder output", ctx.read(g_enc.output, g_enc.neurons * B), o_enc.output.reshape(-1))
    check_close(f"step{step} input gradient", ctx.read(g_in.gradient, g_in.neurons * B), o_in.gradient.reshape(-1))
    for i in range(o_enc.L):
        check_close(f"step{step} L{i} scores", ctx.read(g_enc.scores[i]), o_enc.scores[i].reshape(-1))
        check_close(f"step{step} L{i} qkv grad", ctx.read(g_enc.qkv_g[i]), o_enc.qkv_g[i].reshape(-1))
        for j in range(6):
            check_close(f"step{step} L{i} ff{j}", ctx.read(g_enc.ff[i][j]), o_enc.ff[i][j].reshape(-1))
        for name in ("qkv", "w0", "ff1", "ff2"):
            n = o_enc.counts[name]
            gw, gm, gv = g_enc.w[i][name]
            ow, om, ov = o_enc.w[i][name]
            check_weights(f"step{step} L{i} {name} weights", ctx.read(gw, n), ow, o_enc.last_grads[(i, name)],
                          o_enc.last_grads_abs[(i, name)])
            check_close(f"step{step} L{i} {name} m", ctx.read(gm, n), om)
            check_close(f"step{step} L{i} {name} v", ctx.read(gv, n), ov)
            for h, a in ((gw, ow), (gm, om), (gv, ov)):
                ctx.write(h, a)


@pytest.mark.parametrize("batch,replay", [(2, False), (2, True)])
def test_attention_encoder_training_steps(ctx, batch, replay):
    spec = C.MLMHSpec()
    w = C.mlmh_weights(spec)
    net = C.build_mlmh(ctx, spec, batch, w)
    onet = oracle_mlmh(spec, batch, w)
    steps = 2
    xs, ts = C.mlmh_data(spec, batch, steps)
    if replay:
        net.capture()
    for s in range(steps):
        net.set_input(xs[s])
        net.set_target(ts[s])
        net.step()
        onet.step(xs[s], ts[s])
        check_mlmh_step(ctx, net, onet, s)
