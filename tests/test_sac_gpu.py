"""The concatenate input layer (Concat_* kernels, batched) and the soft actor-critic step through the
C ABI, against the oracle (the reference's Concat arithmetic and the library's SAC kernels restated
in numpy, sequenced as nn_in_trading_b200/sac.py).

The SAC step is checked phase by phase after every step (target values, critic outputs, policy
samples and log-probabilities, the actor's output gradient, every weight and moment of the actor,
critics and target critics); each step starts from the oracle's parameters, so rounding does not
compound.  Adam weights whose batch-mean gradient cancelled are compared as in tests/parity.py.
"""
import numpy as np
import pytest

from nn_in_trading_b200.sac import SACAgent, SACSpec, sac_data, sac_weights
from oracle import kernels as K
from oracle import nets as O
from tests.parity import check_close, check_weights
from tests.test_kernels_gpu import run_on_gpu

pytestmark = pytest.mark.gpu

LRELU, NONE, TANH = 2, -1, 0
F32 = np.float32


@pytest.fixture(autouse=True)
def numpy_oracle():
    O.use_backend("numpy")


# (inputs1, inputs2, outputs, batch): the tensor-core product, the SIMT product, the small-batch kernels
CONCAT_SHAPES = [(240, 6, 512, 300), (12, 3, 16, 7), (30, 5, 9, 3)]


def _concat_data(in1, in2, n_out, B, seed):
    rng = np.random.default_rng(seed)
    k = 1 / np.sqrt(in1 + in2 + 1)
    w = rng.uniform(-k, k, n_out * (in1 + in2 + 1)).astype(F32)
    x1 = rng.standard_normal((B, in1)).astype(F32)
    x2 = rng.uniform(-1, 1, (B, in2)).astype(F32)
    g = (rng.standard_normal((B, n_out)) * 0.01).astype(F32)
    return w, x1, x2, g


@pytest.mark.parametrize("in1,in2,n_out,B", CONCAT_SHAPES)
def test_concat_batched_forward_and_gradient(ctx, in1, in2, n_out, B):
    w, x1, x2, g = _concat_data(in1, in2, n_out, B, 10 + in1)
    got = run_on_gpu(ctx, "Concat_FeedForward", [w, x1.ravel(), x2.ravel(), np.zeros(B * n_out, F32), in1, in2,
                                                 LRELU], (n_out,), None, batch=B)
    for b in range(B):
        y = np.zeros(n_out, F32)
        K.Concat_FeedForward(w, x1[b], x2[b], y, in1, in2, LRELU, gsize=(n_out,))
        check_close(f"sample{b} output", got[3][b * n_out:(b + 1) * n_out], y)
    o1 = K.f_activation(x1, LRELU)
    o2 = np.tanh(x2).astype(F32)
    got = run_on_gpu(ctx, "Concat_HiddenGradient",
                     [w, g.ravel(), o1.ravel(), o2.ravel(), np.zeros(B * in1, F32), np.zeros(B * in2, F32), n_out, in1,
                      in2, LRELU, TANH], (in1 + in2,), None, batch=B)
    for b in range(B):
        ig1, ig2 = np.zeros(in1, F32), np.zeros(in2, F32)
        K.Concat_HiddenGradient(w, g[b], o1[b], o2[b], ig1, ig2, n_out, in1, in2, LRELU, TANH, gsize=(in1 + in2,))
        check_close(f"sample{b} input1 gradient", got[4][b * in1:(b + 1) * in1], ig1)
        check_close(f"sample{b} input2 gradient", got[5][b * in2:(b + 1) * in2], ig2, atol=2e-9)


@pytest.mark.parametrize("in1,in2,n_out,B", CONCAT_SHAPES)
def test_concat_batched_updates(ctx, in1, in2, n_out, B):
    """Batch-mean gradient of g_b [x1; x2; 1]_b, then the reference's Adam / momentum arithmetic once."""
    w, x1, x2, g = _concat_data(in1, in2, n_out, B, 20 + in1)
    n_col = in1 + in2 + 1
    rng = np.random.default_rng(30 + in1)
    m = (rng.standard_normal(w.size) * 1e-3).astype(F32)
    v = rng.uniform(0, 1e-5, w.size).astype(F32)
    inp = np.concatenate([x1, x2, np.ones((B, 1), F32)], axis=1)
    terms = g[:, :, None] * inp[:, None, :]
    G = terms.mean(axis=0, dtype=np.float64).astype(F32)
    G_abs = np.abs(terms).mean(axis=0).reshape(-1)
    got = run_on_gpu(ctx, "Concat_UpdateWeightsAdam",
                     [w.copy(), g.ravel(), x1.ravel(), x2.ravel(), m.copy(), v.copy(), in1, in2, 3e-4, 0.9, 0.999],
                     (n_out, n_col), None, batch=B)
    rw, rm, rv = w.copy(), m.copy(), v.copy()
    K.concat_adam_apply(rw, G, rm, rv, in1, in2, 3e-4, 0.9, 0.999, n_out, n_col)
    check_weights("adam weights", got[0], rw, G.reshape(-1), G_abs, w)
    check_close("adam m", got[4], rm)
    check_close("adam v", got[5], rv)
    dw = (rng.standard_normal(w.size) * 1e-4).astype(F32)
    got = run_on_gpu(ctx, "Concat_UpdateWeightsMomentum",
                     [w.copy(), g.ravel(), x1.ravel(), x2.ravel(), dw.copy(), in1, in2, 3e-4, 0.9], (n_out, n_col),
                     None, batch=B)
    rw, rdw = w.copy(), dw.copy()
    K.concat_momentum_apply(rw, G, rdw, in1, in2, 3e-4, 0.9, n_out, n_col)
    check_close("momentum weights", got[0], rw, w)
    check_close("momentum delta", got[4], rdw)


def _param_pairs(agent, oracle):
    """(label, device handle, oracle array, updating oracle layer or None, attribute) of every parameter."""
    pairs = []
    for li in range(3):
        gl, ol = agent.actor[li], oracle.actor.layers[li]
        for a in ("weights", "m", "v"):
            pairs.append((f"actor{li} {a}", getattr(gl, a), getattr(ol, a), oracle.actor.layers[li + 1], a))
    for k in range(2):
        for kind, gnet, onet, upd in (("critic", agent.critics[k], oracle.critics[k], True),
                                      ("target", agent.targets[k], oracle.targets[k], False)):
            for a in ("conc_w", "conc_m", "conc_v"):
                pairs.append((f"{kind}{k} {a}", getattr(gnet[1], a), getattr(onet.layers[1], a),
                              onet.layers[1] if upd else None, a))
            for li in (1, 2):
                for a in ("weights", "m", "v"):
                    pairs.append((f"{kind}{k} layer{li} {a}", getattr(gnet[li], a), getattr(onet.layers[li], a),
                                  onet.layers[li + 1] if upd else None, a))
    return pairs


def _check_step(ctx, agent, oracle, step):
    B, A = agent.B, agent.spec.action
    check_close(f"step{step} target values", ctx.read(agent.y, B), oracle.y)
    check_close(f"step{step} next log-probs", ctx.read(agent.logp_next, B), oracle.logp_next)
    for k in range(2):
        check_close(f"step{step} critic{k} q", ctx.read(agent.critics[k][-1].output, B),
                    oracle.critics[k].layers[-1].output.reshape(-1))
        check_close(f"step{step} critic{k} dq/da", ctx.read(agent.critics_pi[k][1].second_grad, B * A),
                    oracle.critics_pi[k].layers[1].second_grad.reshape(-1))
    check_close(f"step{step} actions", ctx.read(agent.a_pi, B * A), oracle.a_pi)
    check_close(f"step{step} log-probs", ctx.read(agent.logp, B), oracle.logp)
    check_close(f"step{step} actor output gradient", ctx.read(agent.actor[-1].gradient, B * 2 * A),
                oracle.actor.layers[-1].gradient.reshape(-1))
    for label, h, arr, upd, attr in _param_pairs(agent, oracle):
        got = ctx.read(h, arr.size)
        if upd is not None and attr in ("weights", "conc_w"):
            check_weights(f"step{step} {label}", got, arr, upd.last_grad, upd.last_grad_abs)
        else:
            check_close(f"step{step} {label}", got, arr)
        ctx.write(h, arr)


@pytest.mark.parametrize("batch,replay", [(5, False), (256, True)])
def test_sac_steps_match_oracle(ctx, batch, replay):
    spec = SACSpec(state=64, action=6, hidden=128) if batch > 64 else SACSpec(state=12, action=3, hidden=16)
    w = sac_weights(spec)
    agent = SACAgent(ctx, spec, batch, w)
    oracle = O.OSACAgent(spec, batch, w)
    data = sac_data(spec, batch, steps=3)
    if replay:
        agent.capture()
    for s in range(3):
        bt = {k: v[s] for k, v in data.items()}
        agent.set_batch(bt)
        agent.step()
        oracle.step(bt)
        _check_step(ctx, agent, oracle, s)
