"""Training steps of the LSTM stack and of the PatchTST-style network through the C ABI against the
oracle's restatement of the reference sequencing, at reduced shapes (same layer types and call
sequence as the full configurations)."""
import numpy as np
import pytest

from nn_in_trading_b200 import configs as C
from oracle import kernels as K
from oracle import nets as O
from tests.parity import check_close

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def numpy_oracle():
    O.use_backend("numpy")


def test_lstm_stack_steps(ctx):
    spec = C.LSTMSpec(inputs=8, hidden=16, layers=2, series=6, seq=4)
    w = C.lstm_weights(spec)
    net = C.build_lstm(ctx, spec, w)
    layers = [O.ODense(spec.inputs * spec.series, K.NONE, 1, 0)]
    ins = spec.inputs
    for l in range(spec.layers):
        L = O.OLSTM(spec.hidden, ins, spec.series, 1)
        L.lstm_w[:] = w[f"lstm{l}"]
        layers.append(L)
        ins = spec.hidden
    head = O.OConv(spec.hidden, spec.hidden, spec.inputs, spec.series, 1, K.NONE, 1)
    head.conv_w[:] = w["head"]
    layers.append(head)
    onet = O.ONet(layers)
    xs = C.lstm_data(spec)
    for t in range(spec.seq):
        net.set_input(xs[t].reshape(-1))
        net.set_target(xs[t + 1].reshape(-1))
        net.step()
        onet.step(xs[t].reshape(1, -1), xs[t + 1].reshape(1, -1))
        for li in (1, 2):
            g, o = net.layers[li], onet.layers[li]
            check_close(f"t{t} lstm{li} output", ctx.read(g.output), o.output.reshape(-1))
            check_close(f"t{t} lstm{li} memory", ctx.read(g.memory), o.memory)
            check_close(f"t{t} lstm{li} weight gradient", ctx.read(g.lstm_wg), o.lstm_wg)
            check_close(f"t{t} lstm{li} weights", ctx.read(g.lstm_w), o.lstm_w)
            ctx.write(g.lstm_w, o.lstm_w)
            ctx.write(g.lstm_m, o.lstm_m)
            ctx.write(g.lstm_v, o.lstm_v)
        check_close(f"t{t} head output", ctx.read(net.layers[3].output), onet.layers[3].output.reshape(-1))
        check_close(f"t{t} input gradient", ctx.read(net.layers[0].gradient), onet.layers[0].gradient.reshape(-1))
        ctx.write(net.layers[3].conv_w, onet.layers[3].conv_w)
        ctx.write(net.layers[3].conv_m, onet.layers[3].conv_m)
        ctx.write(net.layers[3].conv_v, onet.layers[3].conv_v)


def test_patchtst_style_steps(ctx):
    spec = C.PatchSpec(channels=3, bars=64, patch=16, stride=8, embed=16, heads=2, dk=8, layers=1, horizon=12,
                       norm_batch=5)
    B = 2
    w = C.patch_weights(spec)
    net = C.build_patch(ctx, spec, B, w)
    P, E, Cc = spec.patches, spec.embed, spec.channels
    inp = O.ODense(Cc * spec.bars, K.NONE, B, 0)
    norm = O.OBatchNorm(Cc * spec.bars, spec.norm_batch, B)
    conv = O.OConv(spec.patch, spec.stride, E, P, Cc, K.NONE, B)
    conv.conv_w[:] = w["conv"]
    enc = O.OMLMH(E, spec.dk, spec.heads, P, spec.layers, K.NONE, B * Cc)
    for i, ws in enumerate(w["encoder"]):
        for name, arr in ws.items():
            enc.w[i][name][0][:] = arr
    head = O.OConv(P * E, P * E, spec.horizon, Cc, 1, K.NONE, B)
    head.conv_w[:] = w["head"]
    denorm = O.ORevIN(Cc * spec.horizon, norm, B)
    onet = O.ONet([inp, norm, conv, enc, head, denorm])
    xs, ts = C.patch_data(spec, B, 3)
    for s in range(3):
        net.set_input(xs[s])
        net.set_target(ts[s])
        net.step()
        onet.step(xs[s], ts[s])
        names = ["input", "batchnorm", "conv", "encoder", "head", "revin"]
        for li, name in enumerate(names):
            check_close(f"s{s} {name} output", ctx.read(net.layers[li].output), onet.layers[li].output.reshape(-1))
            check_close(f"s{s} {name} gradient", ctx.read(net.layers[li].gradient),
                        onet.layers[li].gradient.reshape(-1))
        check_close(f"s{s} bn options", ctx.read(net.layers[1].options), onet.layers[1].options)
        for gl, ol in ((net.layers[2], conv), (net.layers[4], head)):
            check_close(f"s{s} conv weights", ctx.read(gl.conv_w), ol.conv_w)
            for h, a in ((gl.conv_w, ol.conv_w), (gl.conv_m, ol.conv_m), (gl.conv_v, ol.conv_v)):
                ctx.write(h, a)
        for i in range(spec.layers):
            for name in ("qkv", "w0", "ff1", "ff2"):
                for j in range(3):
                    ctx.write(net.layers[3].w[i][name][j], enc.w[i][name][j])
