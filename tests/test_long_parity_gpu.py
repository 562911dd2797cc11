"""The five benchmark configurations trained for many steps through the C ABI beside the oracle, with
no state copied between them: outputs, gradients, weights and Adam moments are compared at
checkpoints along the run, so rounding differences compound as they would between two real
training runs.  Each comparison is bounded by a stated drift bound (the worst |got - ref| over
max|ref| of the tensor) and its element-wise distribution is reported at the end of the session
(tests/parity.py: drift).

  dense MLP      240-500-500-3, batch 1, the full 1000 online steps, against the reference's own
                 kernels (oracle/_ref) sequenced as CNet::feedForward / backPropOCL
  encoder        4 x (120 tokens, 64 features, 8 heads x 32, FF 256), batch 8, 20 steps
  LSTM stack     input 64, 2 layers of 256, 64 series over the full 240-bar window
  PatchTST-style 32 channels x 512 bars, patch 16 / stride 8, embed 128, 3 layers, batch 2, 3 steps
  SAC            state 240, action 6, hidden 512, replay 512, 4 updates

Why drift grows: the reference's Adam has no effective epsilon (m / (sqrt(v) + 1e-37)), so a weight
moves by about lr * 3.16 in the direction of its gradient's sign whatever the gradient's size; where a
gradient is at rounding level (the attention layers' Q/K gradients cancel almost completely), two
correct float32 runs move the weight in opposite directions, and the training dynamics amplify such
differences exponentially.  The reference shows the same growth against itself: the dense MLP test
runs the reference's kernels as the trajectory compared against and as three more valid executions
that differ from it only in rounding (maximum local size 64, a legal change of their summation
order; multiply-adds contracted into FMAs, which OpenCL C allows by default; both), and the library
must stay within 10x of the farthest of them; the LSTM test runs the oracle a second time from
weights one float32 step apart and reports that growth beside the library's.  The other bounds are per checkpoint, about three times the drift measured on a B200
(the library and the oracle are deterministic, so the measurement repeats exactly); the session
summary prints every measured value."""
import numpy as np
import pytest

from nn_in_trading_b200 import configs as C
from nn_in_trading_b200.sac import SACAgent, SACSpec, sac_data, sac_weights
from oracle import kernels as K
from oracle import nets as O
from oracle.ref import LIB_FMA_PATH, RefKernels, host_has_fma
from tests.parity import drift

pytestmark = pytest.mark.gpu

# drift bounds (tensor-relative) per configuration, checkpoint and tensor kind
ENCODER_BOUNDS = {
    1: {"output": 1e-4, "input_gradient": 1e-4, "weights": 2e-2, "m": 1e-4, "v": 1e-4},
    5: {"output": 1e-4, "input_gradient": 1e-4, "weights": 6e-2, "m": 1e-4, "v": 1e-4},
    10: {"output": 1e-3, "input_gradient": 1.0, "weights": 2e-1, "m": 1e-2, "v": 2e-2},
    20: {"output": 1e-1, "input_gradient": 1.0, "weights": 3e-1, "m": 2e-1, "v": 1e-1},
}
BOUNDS = {
    "patchtst": {"output": 1e-4, "encoder": 1e-4, "weights": 1e-1, "options": 1e-5},
    "sac": {"values": 1e-3, "weights": 5e-2, "m": 1.5e-1, "v": 1e-1},
}
# LSTM stack: bound per bar of the window (every compared tensor)
LSTM_BOUNDS = {1: 1e-4, 16: 1e-3, 60: 1e-2, 120: 2e-1, 240: 1.0}


@pytest.fixture(autouse=True)
def numpy_oracle():
    O.use_backend("numpy")
    yield
    O.use_backend("numpy")


def _dense_oracle(spec, w):
    layers = [O.ODense(n, a, 1, spec.sizes[i + 1] if i + 1 < len(spec.sizes) else 0)
              for i, (n, a) in enumerate(zip(spec.sizes, spec.acts))]
    for layer, ww in zip(layers, w):
        layer.weights[:] = ww
    return O.ONet(layers)


def test_dense_mlp_1000_online_steps_against_the_reference_kernels(ctx):
    """The library against the reference's kernels as the MQL5 host runs them on a device whose
    maximum local size is 256, each product and sum rounded on its own (the trajectory compared
    against), beside valid executions of the same kernels that differ from it only in rounding:
    maximum local size 64 (another summation order), multiply-adds contracted into FMAs (OpenCL C's
    default FP_CONTRACT ON, what GPU OpenCL compilers do), and both.  At every checkpoint the
    library may drift from the reference at most 10x as far as the farthest of those executions
    does (their envelope).  Over the first 100 steps the envelope is set by single Adam steps taken
    in opposite directions on cancelled moments, which comes and goes with the execution (on an x86
    host the reference at local size 64 is already 1.2e-4 from itself in layer 0's moments at step
    10, on another 3e-6): there the bound is at least 1e-3."""
    if not RefKernels.available():
        pytest.skip("oracle/_ref not built")
    spec = C.DenseSpec()
    w = C.dense_weights(spec)
    steps = 1000
    xs, ts = C.dense_data(spec, steps, 1)
    net = C.build_dense(ctx, spec, 1, w)
    net.capture()
    plain = O.RefBackend()
    # (backend, maximum local size) of each execution; the first is the one compared against
    runs = {"reference": (plain, 256), "local size 64": (plain, 64)}
    if RefKernels.available(LIB_FMA_PATH) and host_has_fma():
        fma = O.RefBackend(LIB_FMA_PATH)
        runs["FMA"] = (fma, 256)
        runs["FMA, local size 64"] = (fma, 64)
    nets = {name: _dense_oracle(spec, w) for name in runs}
    checkpoints = {1, 10, 100, 250, 500, 1000}
    try:
        for s in range(steps):
            net.set_input(xs[s])
            net.set_target(ts[s])
            net.step()
            for name, (backend, max_local) in runs.items():
                O.BACKEND, O.MAX_LOCAL = backend, max_local
                nets[name].step(xs[s], ts[s])
            if s + 1 not in checkpoints:
                continue
            tag = f"dense step{s + 1}"
            ref = nets["reference"]
            pairs = [("output", ctx.read(net.layers[-1].output, 3), lambda o: o.layers[-1].output)]
            for li in range(3):
                n = ref.layers[li].weights.size
                for kind in ("weights", "m", "v"):
                    pairs.append((f"layer{li} {kind}", ctx.read(getattr(net.layers[li], kind), n),
                                  lambda o, li=li, kind=kind: getattr(o.layers[li], kind)))
            for label, got, pick in pairs:
                envelope = max(drift(f"{tag} {label} (reference, {name})", pick(nets[name]), pick(ref),
                                     float("inf"))["tensor_rel"] for name in runs if name != "reference")
                bound = max(10.0 * envelope, 1e-3 if s + 1 <= 100 else 1e-6)
                drift(f"{tag} {label}", got, pick(ref), bound)
    finally:
        O.BACKEND, O.MAX_LOCAL = K, 256


def test_attention_encoder_20_steps_batch_8(ctx):
    spec = C.MLMHSpec()
    B, steps = 8, 20
    w = C.mlmh_weights(spec)
    net = C.build_mlmh(ctx, spec, B, w)
    net.capture()
    inp = O.ODense(spec.window * spec.units, K.NONE, B, 0)
    enc = O.OMLMH(spec.window, spec.dk, spec.heads, spec.units, spec.layers, spec.activation, B)
    for i, ws in enumerate(w):
        for name, arr in ws.items():
            enc.w[i][name][0][:] = arr
    onet = O.ONet([inp, enc])
    xs, ts = C.mlmh_data(spec, B, steps)
    for s in range(steps):
        net.set_input(xs[s])
        net.set_target(ts[s])
        net.step()
        onet.step(xs[s], ts[s])
        if s + 1 in ENCODER_BOUNDS:
            b = ENCODER_BOUNDS[s + 1]
            tag = f"encoder step{s + 1}"
            g_enc = net.layers[1]
            drift(f"{tag} output", ctx.read(g_enc.output, g_enc.neurons * B), enc.output, b["output"])
            drift(f"{tag} input gradient", ctx.read(net.layers[0].gradient, g_enc.neurons * B), inp.gradient,
                  b["input_gradient"])
            for i in range(spec.layers):
                for name in ("qkv", "w0", "ff1", "ff2"):
                    n = enc.counts[name]
                    for j, kind in enumerate(("weights", "m", "v")):
                        drift(f"{tag} L{i} {name} {kind}", ctx.read(g_enc.w[i][name][j], n), enc.w[i][name][j][:n],
                              b[kind])


def _lstm_oracle(spec, w, nudge=False):
    """The oracle LSTM stack; `nudge`: every weight moved one float32 step up (a rounding-size change)."""
    def put(dst, src):
        dst[:] = np.nextafter(src, np.float32(np.inf)) if nudge else src
    layers = [O.ODense(spec.inputs * spec.series, K.NONE, 1, 0)]
    ins = spec.inputs
    for l in range(spec.layers):
        L = O.OLSTM(spec.hidden, ins, spec.series, 1)
        put(L.lstm_w, w[f"lstm{l}"])
        layers.append(L)
        ins = spec.hidden
    head = O.OConv(spec.hidden, spec.hidden, spec.inputs, spec.series, 1, K.NONE, 1)
    put(head.conv_w, w["head"])
    layers.append(head)
    return O.ONet(layers)


def test_lstm_stack_full_window(ctx):
    """Beside the oracle, a second oracle run whose initial weights differ from the first by one float32
    step: how far rounding-size differences carry over the window in the reference's arithmetic."""
    spec = C.LSTMSpec(inputs=64, hidden=256, layers=2, series=64, seq=240)
    w = C.lstm_weights(spec)
    net = C.build_lstm(ctx, spec, w)
    net.capture()
    onet, nudged = _lstm_oracle(spec, w), _lstm_oracle(spec, w, nudge=True)
    xs = C.lstm_data(spec)
    for t in range(spec.seq):
        net.set_input(xs[t].reshape(-1))
        net.set_target(xs[t + 1].reshape(-1))
        net.step()
        onet.step(xs[t].reshape(1, -1), xs[t + 1].reshape(1, -1))
        nudged.step(xs[t].reshape(1, -1), xs[t + 1].reshape(1, -1))
        if t + 1 not in LSTM_BOUNDS:
            continue
        tag = f"lstm bar{t + 1}"
        bound = LSTM_BOUNDS[t + 1]
        pairs = []
        for li in (1, 2):
            g, o, n = net.layers[li], onet.layers[li], nudged.layers[li]
            pairs += [(f"lstm{li} output", ctx.read(g.output), o.output, n.output),
                      (f"lstm{li} memory", ctx.read(g.memory), o.memory, n.memory),
                      (f"lstm{li} weights", ctx.read(g.lstm_w), o.lstm_w, n.lstm_w)]
        pairs += [("head output", ctx.read(net.layers[3].output), onet.layers[3].output, nudged.layers[3].output),
                  ("head weights", ctx.read(net.layers[3].conv_w), onet.layers[3].conv_w, nudged.layers[3].conv_w)]
        for label, got, ref, own in pairs:
            drift(f"{tag} {label} (oracle from weights 1 ulp apart)", own, ref, float("inf"))
            drift(f"{tag} {label}", got, ref, bound)


def test_patchtst_full_size_3_steps(ctx):
    spec = C.PatchSpec()
    B, steps = 2, 3
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
    onet = O.ONet([inp, norm, conv, enc, head, O.ORevIN(Cc * spec.horizon, norm, B)])
    xs, ts = C.patch_data(spec, B, steps)
    b = BOUNDS["patchtst"]
    for s in range(steps):
        net.set_input(xs[s])
        net.set_target(ts[s])
        net.step()
        onet.step(xs[s], ts[s])
        tag = f"patchtst step{s + 1}"
        drift(f"{tag} output", ctx.read(net.layers[5].output), onet.layers[5].output, b["output"])
        drift(f"{tag} encoder output", ctx.read(net.layers[3].output), enc.output, b["encoder"])
        drift(f"{tag} bn options", ctx.read(net.layers[1].options), norm.options, b["options"])
        drift(f"{tag} patch conv weights", ctx.read(net.layers[2].conv_w), conv.conv_w, b["weights"])
        drift(f"{tag} head weights", ctx.read(net.layers[4].conv_w), head.conv_w, b["weights"])
        for i in range(spec.layers):
            for name in ("qkv", "w0", "ff1", "ff2"):
                n = enc.counts[name]
                drift(f"{tag} L{i} {name} weights", ctx.read(net.layers[3].w[i][name][0], n), enc.w[i][name][0][:n],
                      b["weights"])


def test_sac_full_size_replay_512(ctx):
    spec = SACSpec()
    B, steps = 512, 4
    w = sac_weights(spec)
    agent = SACAgent(ctx, spec, B, w)
    agent.capture()
    oracle = O.OSACAgent(spec, B, w)
    data = sac_data(spec, B, steps=steps)
    b = BOUNDS["sac"]
    for s in range(steps):
        bt = {k: v[s] for k, v in data.items()}
        agent.set_batch(bt)
        agent.step()
        oracle.step(bt)
        tag = f"sac step{s + 1}"
        drift(f"{tag} target values", ctx.read(agent.y, B), oracle.y, b["values"])
        drift(f"{tag} log-probs", ctx.read(agent.logp, B), oracle.logp, b["values"])
        for k in range(2):
            drift(f"{tag} critic{k} q", ctx.read(agent.critics[k][-1].output, B),
                  oracle.critics[k].layers[-1].output.reshape(-1), b["values"])
        for li in range(3):
            gl, ol = agent.actor[li], oracle.actor.layers[li]
            for kind in ("weights", "m", "v"):
                arr = getattr(ol, kind)
                drift(f"{tag} actor{li} {kind}", ctx.read(getattr(gl, kind), arr.size), arr, b[kind])
        for k in range(2):
            for kind, gnet, onet in (("critic", agent.critics[k], oracle.critics[k]),
                                     ("target", agent.targets[k], oracle.targets[k])):
                arr = onet.layers[1].conc_w
                drift(f"{tag} {kind}{k} concat weights", ctx.read(gnet[1].conc_w, arr.size), arr, b["weights"])
                for li in (1, 2):
                    arr = onet.layers[li].weights
                    drift(f"{tag} {kind}{k} layer{li} weights", ctx.read(gnet[li].weights, arr.size), arr,
                          b["weights"])
