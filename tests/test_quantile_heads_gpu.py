"""Training steps of the quantile heads through the C ABI against the oracle's restatement of their
sequencing: CNeuronFQF (NeuroNet_AgentsRL.mqh:32-248) and CNeuronSoftActorCritic
(NeuroNet_AgentsRL.mqh:1655-1990), behind a state layer whose weights feed the fraction proposal.

Every step compares the head's output and gradient, every inner layer's output and gradient, and
every post-update weight, first and second moment; the library's state is then set to the oracle's
so that each step is checked on identical inputs."""
import numpy as np
import pytest

from nn_in_trading_b200 import configs as C
from oracle import nets as O
from tests.parity import check_close, check_weights

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def numpy_oracle():
    O.use_backend("numpy")


# (name of the inner layer holding the weights, name of the layer whose update moves them)
WEIGHT_OWNERS = [("state", "fraction"), ("cosine", "cos_emb"), ("q0", "q1"), ("q1", "q2")]
INNER = ("fraction", "softmax", "cosine", "cos_emb", "q0", "q1", "q2")


def _layer(net, name, head):
    return net.layers[0] if name == "state" else getattr(head, name)


def check_head_step(ctx, net, onet, step, sac):
    g_head, o_head = net.layers[1], onet.layers[1]
    B = g_head.batch
    rd = lambda h, n: ctx.read(h, n)  # noqa: E731
    check_close(f"step{step} head output", rd(g_head.output, g_head.neurons * B), o_head.output.reshape(-1))
    check_close(f"step{step} state gradient", rd(net.layers[0].gradient, net.layers[0].neurons * B),
                onet.layers[0].gradient.reshape(-1))
    for name in INNER:
        gl, ol = getattr(g_head, name), getattr(o_head, name)
        check_close(f"step{step} {name} output", rd(gl.output, gl.neurons * B), ol.output.reshape(-1))
        check_close(f"step{step} {name} gradient", rd(gl.gradient, gl.neurons * B), ol.gradient.reshape(-1))
    if sac:
        check_close(f"step{step} log_probs", rd(g_head.log_probs, g_head.A * B), o_head.log_probs.reshape(-1))
        check_close(f"step{step} alphas output", rd(g_head.alphas.output, g_head.A * B),
                    o_head.alphas.output.reshape(-1))
        check_close(f"step{step} alphas gradient", rd(g_head.alphas.gradient, g_head.A * B),
                    o_head.alphas.gradient.reshape(-1))
    owners = list(WEIGHT_OWNERS)
    for wname, uname in owners:
        gl, ol = _layer(net, wname, g_head), _layer(onet, wname, o_head)
        upd = getattr(o_head, uname)
        n = ol.weights.size
        check_weights(f"step{step} {wname} weights", rd(gl.weights, n), ol.weights, upd.last_grad, upd.last_grad_abs)
        check_close(f"step{step} {wname} m", rd(gl.m, n), ol.m)
        check_close(f"step{step} {wname} v", rd(gl.v, n), ol.v)
        for h, a in ((gl.weights, ol.weights), (gl.m, ol.m), (gl.v, ol.v)):
            ctx.write(h, a)
    if sac:
        ga, oa = g_head.alphas, o_head.alphas
        n = oa.conc_w.size
        check_weights(f"step{step} alphas weights", rd(ga.conc_w, n), oa.conc_w, oa.last_grad, oa.last_grad_abs)
        check_close(f"step{step} alphas m", rd(ga.conc_m, n), oa.conc_m)
        check_close(f"step{step} alphas v", rd(ga.conc_v, n), oa.conc_v)
        for h, a in ((ga.conc_w, oa.conc_w), (ga.conc_m, oa.conc_m), (ga.conc_v, oa.conc_v)):
            ctx.write(h, a)


@pytest.mark.parametrize("sac", [False, True])
@pytest.mark.parametrize("batch,replay", [(1, False), (4, False), (4, True)])
def test_quantile_head_training_steps(ctx, sac, batch, replay):
    spec = C.QuantileHeadSpec(inputs=96, actions=6, quantiles=32, sac=sac)
    w = C.quantile_head_weights(spec)
    net = C.build_quantile_head(ctx, spec, batch, w)
    onet = O.quantile_head_net(spec, w, batch)
    steps = 4
    xs, ts, us = C.quantile_head_data(spec, steps, batch)
    head = net.layers[1]
    if replay:
        net.capture()
    alpha_ops = head.alpha_gradient_ops(head) if sac else []
    for s in range(steps):
        if sac:
            head.set_random(us[s])
            onet.layers[1].random[...] = us[s]
        net.set_input(xs[s])
        net.set_target(ts[s])
        net.step()
        onet.step(xs[s], ts[s])
        for op in alpha_ops:  # calcAlphaGradients, fed with the head's own gradient
            op()
        if sac:
            onet.layers[1].alpha_gradient(onet.layers[1])
        check_head_step(ctx, net, onet, s, sac)


def test_soft_actor_critic_head_samples_a_quantile_per_action(ctx):
    """The SAC head's output is one of each action's quantile values (after the activation, None here)
    and its log-probability is -alpha log p of the sampled quantile's probability."""
    spec = C.QuantileHeadSpec(inputs=64, actions=4, quantiles=16, sac=True)
    net = C.build_quantile_head(ctx, spec, 8)
    xs, ts, us = C.quantile_head_data(spec, 1, 8)
    head = net.layers[1]
    head.set_random(us[0])
    net.set_input(xs[0])
    net.forward()
    y = ctx.read(head.output, 4 * 8).reshape(8, 4)
    q = ctx.read(head.q2.output, 64 * 8).reshape(8, 4, 16)
    p = ctx.read(head.softmax.output, 64 * 8).reshape(8, 4, 16)
    a = ctx.read(head.alphas.output, 4 * 8).reshape(8, 4)
    lp = ctx.read(head.log_probs, 4 * 8).reshape(8, 4)
    for b in range(8):
        for i in range(4):
            r = int(np.nonzero(q[b, i] == y[b, i])[0][0])
            assert abs(lp[b, i] - (-a[b, i] * np.log(p[b, i, r]))) <= 1e-5 * max(1.0, abs(lp[b, i]))
