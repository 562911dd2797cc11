"""The oracle's restatement of the host sequencing, run over its numpy kernels, against the same
sequencing run over the reference's own kernels (oracle/_ref, NeuroNet.cl compiled for the CPU):
pins the numpy kernels at the real layer shapes of the dense MLP and the attention encoder, and the
sequencing of the LSTM stack and of the PatchTST-style network at reduced shapes."""
import numpy as np
import pytest

from nn_in_trading_b200 import configs as C
from oracle import kernels as K
from oracle import nets as O
from oracle.ref import RefKernels
from tests.parity import check_close, check_weights, deactivation_atol

pytestmark = pytest.mark.skipif(not RefKernels.available(), reason="oracle/_ref not built")


def dense(spec, w):
    layers = [O.ODense(n, a, 1, spec.sizes[i + 1] if i + 1 < len(spec.sizes) else 0)
              for i, (n, a) in enumerate(zip(spec.sizes, spec.acts))]
    for layer, ww in zip(layers, w):
        layer.weights[:] = ww
    return O.ONet(layers)


def test_dense_mlp_numpy_oracle_matches_reference_kernels():
    spec = C.DenseSpec()
    w = C.dense_weights(spec)
    xs, ts = C.dense_data(spec, 5, 1)
    nets = {}
    for kind in ("numpy", "reference"):
        O.use_backend(kind)
        nets[kind] = dense(spec, w)
    try:
        for s in range(5):
            for kind in ("numpy", "reference"):
                O.use_backend(kind)
                nets[kind].step(xs[s], ts[s])
            a, b = nets["numpy"], nets["reference"]
            from tests.test_nets_gpu import dense_gradient_floors
            floors = dense_gradient_floors(b)
            for li in range(len(a.layers)):
                check_close(f"step{s} layer{li} output", a.layers[li].output, b.layers[li].output)
                check_close(f"step{s} layer{li} gradient", a.layers[li].gradient, b.layers[li].gradient,
                            atol=floors[li])
            for li in range(len(a.layers) - 1):
                check_weights(f"step{s} layer{li} weights", a.layers[li].weights, b.layers[li].weights,
                              b.layers[li + 1].last_grad, b.layers[li + 1].last_grad_abs)
                a.layers[li].weights[:] = b.layers[li].weights
                a.layers[li].m[:] = b.layers[li].m
                a.layers[li].v[:] = b.layers[li].v
    finally:
        O.use_backend("numpy")


def test_attention_encoder_numpy_oracle_matches_reference_kernels():
    spec = C.MLMHSpec()
    w = C.mlmh_weights(spec)
    xs, ts = C.mlmh_data(spec, 1, 1)
    nets = {}
    try:
        for kind in ("numpy", "reference"):
            O.use_backend(kind)
            inp = O.ODense(spec.window * spec.units, K.NONE, 1, 0)
            enc = O.OMLMH(spec.window, spec.dk, spec.heads, spec.units, spec.layers, spec.activation, 1)
            for i, ws in enumerate(w):
                for name, ww in ws.items():
                    enc.w[i][name][0][:] = ww
            net = O.ONet([inp, enc])
            net.step(xs[0], ts[0])
            nets[kind] = net
    finally:
        O.use_backend("numpy")
    a, b = nets["numpy"].layers, nets["reference"].layers
    check_close("encoder output", a[1].output, b[1].output)
    check_close("input gradient", a[0].gradient, b[0].gradient)
    for i in range(spec.layers):
        check_close(f"L{i} qkv grad", a[1].qkv_g[i], b[1].qkv_g[i])
        for name in ("qkv", "w0", "ff1", "ff2"):
            check_weights(f"L{i} {name}", a[1].w[i][name][0], b[1].w[i][name][0], b[1].last_grads[(i, name)],
                          b[1].last_grads_abs[(i, name)])
            check_close(f"L{i} {name} v", a[1].w[i][name][2], b[1].w[i][name][2])


def _sac_params(agent):
    """(label, array, updating layer or None) of every parameter array of an oracle SAC agent."""
    out = []
    for name, net, upd in ([("actor", agent.actor, True)] + [(f"critic{k}", c, True) for k, c in enumerate(agent.critics)]
                           + [(f"target{k}", t, False) for k, t in enumerate(agent.targets)]):
        for li, layer in enumerate(net.layers):
            for attr in ("weights", "m", "v", "conc_w", "conc_m", "conc_v"):
                if hasattr(layer, attr):
                    nxt = (layer if attr.startswith("conc") else net.layers[li + 1]) if upd else None
                    out.append((f"{name} layer{li} {attr}", layer, attr, nxt))
    return out


def test_sac_step_numpy_oracle_matches_reference_kernels():
    """The SAC step at batch 1, where every dense and Concat kernel call goes through the reference's
    own kernels (UpdateWeightsAdam, Concat_UpdateWeightsAdam, SoftUpdate included)."""
    from nn_in_trading_b200.sac import SACSpec, sac_data, sac_weights
    spec = SACSpec(state=24, action=3, hidden=32)
    w = sac_weights(spec)
    d = sac_data(spec, 1, 4)
    agents = {kind: O.OSACAgent(spec, 1, w) for kind in ("numpy", "reference")}
    try:
        for s in range(4):
            bt = {k: v[s] for k, v in d.items()}
            for kind in ("numpy", "reference"):
                O.use_backend(kind)
                agents[kind].step(bt)
            a, b = agents["numpy"], agents["reference"]
            check_close(f"step{s} target values", a.y, b.y)
            check_close(f"step{s} log-probs", a.logp, b.logp)
            check_close(f"step{s} actor output gradient", a.actor.layers[-1].gradient, b.actor.layers[-1].gradient)
            for (label, la, attr, upd), (_, lb, _, _) in zip(_sac_params(a), _sac_params(b)):
                got, ref = getattr(la, attr), getattr(lb, attr)
                if upd is not None and attr in ("weights", "conc_w"):
                    check_weights(f"step{s} {label}", got, ref, upd.last_grad, upd.last_grad_abs)
                else:
                    check_close(f"step{s} {label}", got, ref)
                got[:] = ref
    finally:
        O.use_backend("numpy")


def _head_arrays(net):
    """(label, array) of every output, gradient and parameter of a quantile-head oracle net."""
    state, head = net.layers
    out = [("state gradient", state.gradient), ("state weights", state.weights), ("head output", head.output),
           ("head gradient", head.gradient)]
    subs = [("fraction", head.fraction), ("softmax", head.softmax), ("cosine", head.cosine),
            ("cos_emb", head.cos_emb), ("q0", head.q0), ("q1", head.q1), ("q2", head.q2)]
    if hasattr(head, "alphas"):
        subs.append(("alphas", head.alphas))
        out += [("alphas conc_w", head.alphas.conc_w), ("log_probs", head.log_probs)]
    for name, layer in subs:
        out += [(f"{name} output", layer.output), (f"{name} gradient", layer.gradient)]
        if getattr(layer, "outputs", 0):
            out += [(f"{name} weights", layer.weights), (f"{name} m", layer.m), (f"{name} v", layer.v)]
    return out


@pytest.mark.parametrize("sac", [False, True])
def test_quantile_head_numpy_oracle_matches_reference_kernels(sac):
    """CNeuronFQF / CNeuronSoftActorCritic sequencing (NeuroNet_AgentsRL.mqh:32-248, 1655-1990) over
    the numpy kernels against the same sequencing over the reference's own kernels, 3 steps."""
    spec = C.QuantileHeadSpec(inputs=24, actions=3, quantiles=8, sac=sac)
    w = C.quantile_head_weights(spec)
    xs, ts, us = C.quantile_head_data(spec, 3, 1)
    nets = {}
    try:
        for kind in ("numpy", "reference"):
            O.use_backend(kind)
            nets[kind] = O.quantile_head_net(spec, w, 1)
        for s in range(3):
            for kind in ("numpy", "reference"):
                O.use_backend(kind)
                net = nets[kind]
                if sac:
                    net.layers[1].random[...] = us[s]
                net.step(xs[s], ts[s])
                if sac:
                    net.layers[1].alpha_gradient(net.layers[1])
            for (label, a), (_, b) in zip(_head_arrays(nets["numpy"]), _head_arrays(nets["reference"])):
                check_close(f"step{s} {label}", a, b)
                a[...] = b
    finally:
        O.use_backend("numpy")


def _lstm_stack(spec, w):
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
    return O.ONet(layers)


def test_lstm_stack_numpy_oracle_matches_reference_kernels():
    """Two LSTM layers and the 1x1-conv head over six series, bar by bar: every LSTM kernel
    (LSTM_FeedForward, LSTM_ConcatenatedGradient, LSTM_HiddenGradient, LSTM_UpdateWeightsAdam) and
    the head's conv kernels are the reference's own in one run and the numpy restatement in the
    other.  The cell memory carries over from bar to bar in both runs.

    The reference's LSTM_FeedForward reads h(t-1) from the output buffer that its other work-groups
    overwrite with h(t) (NeuroNet.cl:2189-2261); the CPU executor runs work-groups in order, so with
    several neurons per series the reference run would read a mix of h(t-1) and h(t) where the
    restatement (and the CUDA library) read h(t-1).  Both runs therefore zero the recurrent weight
    columns before every bar, which hides that race and nothing else; the golden cases with one
    neuron per series pin the recurrent product itself."""
    spec = C.LSTMSpec(inputs=8, hidden=32, layers=2, series=6, seq=6)
    w = C.lstm_weights(spec)
    xs = C.lstm_data(spec)
    nets = {}
    try:
        for kind in ("numpy", "reference"):
            O.use_backend(kind)
            nets[kind] = _lstm_stack(spec, w)
        for t in range(spec.seq):
            for kind in ("numpy", "reference"):
                for L in nets[kind].layers[1:3]:
                    L.lstm_w.reshape(4 * L.H, L.inputs + L.H + 1)[:, :L.H] = 0.0
                O.use_backend(kind)
                nets[kind].step(xs[t].reshape(1, -1), xs[t + 1].reshape(1, -1))
            a, b = nets["numpy"].layers, nets["reference"].layers
            for li in (1, 2):
                check_close(f"t{t} lstm{li} output", a[li].output, b[li].output)
                check_close(f"t{t} lstm{li} memory", a[li].memory, b[li].memory)
                check_close(f"t{t} lstm{li} weight gradient", a[li].lstm_wg, b[li].lstm_wg)
                check_close(f"t{t} lstm{li} weights", a[li].lstm_w, b[li].lstm_w)
                for name in ("lstm_w", "lstm_m", "lstm_v"):
                    getattr(a[li], name)[:] = getattr(b[li], name)
            check_close(f"t{t} head output", a[3].output, b[3].output)
            check_close(f"t{t} input gradient", a[0].gradient, b[0].gradient)
            for name in ("conv_w", "conv_m", "conv_v"):
                getattr(a[3], name)[:] = getattr(b[3], name)
    finally:
        O.use_backend("numpy")


def _patch_net(spec, B, w):
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
    return O.ONet([inp, norm, conv, enc, head, denorm])


def test_patchtst_style_numpy_oracle_matches_reference_kernels():
    """Batch norm, the overlapping-window patch convolution, one attention encoder layer over the
    channels' patch sequences (7 patches, 2 heads of 8: the shared-memory attention shapes), the
    flattening conv head and RevIN: every forward and backward kernel call is the reference's own in
    one run and the numpy restatement in the other (batch 2: the weight updates are the mean
    gradient's, formed in numpy in both runs)."""
    spec = C.PatchSpec(channels=3, bars=64, patch=16, stride=8, embed=16, heads=2, dk=8, layers=1, horizon=12,
                       norm_batch=5)
    B = 2
    w = C.patch_weights(spec)
    xs, ts = C.patch_data(spec, B, 3)
    nets = {}
    try:
        for kind in ("numpy", "reference"):
            O.use_backend(kind)
            nets[kind] = _patch_net(spec, B, w)
        names = ["input", "batchnorm", "conv", "encoder", "head", "revin"]
        for s in range(3):
            for kind in ("numpy", "reference"):
                O.use_backend(kind)
                nets[kind].step(xs[s], ts[s])
            a, b = nets["numpy"].layers, nets["reference"].layers
            for li, name in enumerate(names):
                check_close(f"s{s} {name} output", a[li].output, b[li].output)
                check_close(f"s{s} {name} gradient", a[li].gradient, b[li].gradient)
            check_close(f"s{s} bn options", a[1].options, b[1].options)
            a[1].options[:] = b[1].options
            for li in (2, 4):
                check_close(f"s{s} layer{li} conv weights", a[li].conv_w, b[li].conv_w)
                for name in ("conv_w", "conv_m", "conv_v"):
                    getattr(a[li], name)[:] = getattr(b[li], name)
            for i in range(spec.layers):
                for name in ("qkv", "w0", "ff1", "ff2"):
                    for j in range(3):
                        a[3].w[i][name][j][:] = b[3].w[i][name][j]
    finally:
        O.use_backend("numpy")
