"""Soft actor-critic update over the C ABI (the squashed-Gaussian SAC workload).

Networks, all Adam, `batch` replay transitions per GPU:
  actor     state 240 -> 512 LReLU -> 512 LReLU -> 12 = (mu[6], log_std[6])   dense (CNeuronBaseOCL)
  critic k  [state 240; action 6] -> 512 LReLU -> 512 LReLU -> 1, k = 1, 2      CNeuronConcatenate input
  target k  the same shape, Polyak-averaged from critic k                       CNet::WeightsUpdate

One step, from one replay batch (s, a, r, s', done) and two standard-normal noise draws:
  1. target value  actor(s') -> SACGaussianPolicy -> a', log pi'; target k(s', a') -> q'_k;
                   SACTargetValue: y = r + gamma (1 - done) (min q' - alpha log pi')
  2. critics       critic k(s, a); CalcOutputGradient against y; backward; Adam updates
                   (data parallel: one allreduce of both critics' gradients, then the updates)
  3. actor         actor(s) -> SACGaussianPolicy -> a~, log pi; critic k(s, a~) from an output
                   gradient of 1 back to the action input (Concat_HiddenGradient) -> dq_k/da;
                   SACPolicyGradient -> the actor's output gradient; backward; Adam updates
                   (data parallel: one allreduce of the actor's gradients)
  4. Polyak        target k <- critic k on every weight buffer: SoftUpdate, t = tau s + (1 - tau) t.
                   (With soft_update_adam=True, SoftUpdateAdam instead, which is what the reference's
                   WeightsUpdate runs for Adam layers with tau != 1, NeuroNet_Core.mqh:20283-20370:
                   an Adam step toward the source that moves each weight by up to about 3 per call.)

Step 3 runs against the critics updated in step 2.  The actor pass through a critic uses a second
set of activation and gradient buffers over the same weights, so the critic's own buffers are not
disturbed.  Every phase is recorded once into a command list and replayed with the per-step Adam
rates patched in.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from .api import ADAM, LRELU, NONE, Context
from .layers import AdamOp, ConcatLayer, DenseLayer, Op
from .net import Net

F32 = np.float32


@dataclass
class SACSpec:
    state: int = 240
    action: int = 6
    hidden: int = 512
    tau: float = 0.005
    gamma: float = 0.99
    alpha: float = 0.2
    seed: int = 5
    soft_update_adam: bool = False


def sac_weights(spec: SACSpec) -> dict:
    """Uniform +-1/sqrt(fan_in) for every weight and bias; the targets start as copies of the critics."""
    rng = np.random.default_rng(spec.seed)
    S, A, H = spec.state, spec.action, spec.hidden

    def u(n_in, n_out):
        k = 1.0 / np.sqrt(n_in)
        return rng.uniform(-k, k, n_out * (n_in + 1)).astype(F32)

    actor = [u(S, H), u(H, H), u(H, 2 * A)]
    critics = [{"conc": u(S + A, H), "w1": u(H, H), "w2": u(H, 1)} for _ in range(2)]
    return {"actor": actor, "critics": critics}


def sac_data(spec: SACSpec, batch: int, steps: int = 1, seed: int | None = None) -> dict:
    """Synthetic replay batches: s, s' ~ N(0,1); a ~ U[-1,1]; r ~ N(0,1); done ~ Bernoulli(0.01);
    eps1, eps2 ~ N(0,1) (the policy noise for s' and s).  Arrays are [steps][batch * width]."""
    rng = np.random.default_rng(spec.seed + 1 if seed is None else seed)
    S, A = spec.state, spec.action
    return {
        "s": rng.standard_normal((steps, batch * S)).astype(F32),
        "a": rng.uniform(-1.0, 1.0, (steps, batch * A)).astype(F32),
        "r": rng.standard_normal((steps, batch)).astype(F32),
        "s2": rng.standard_normal((steps, batch * S)).astype(F32),
        "done": (rng.uniform(0.0, 1.0, (steps, batch)) < 0.01).astype(F32),
        "eps1": rng.standard_normal((steps, batch * A)).astype(F32),
        "eps2": rng.standard_normal((steps, batch * A)).astype(F32),
    }


def _use_buffer(layer, attr: str, handle: int) -> None:
    layer.ctx.free(getattr(layer, attr))
    setattr(layer, attr, handle)


class SACAgent:
    INPUTS = ("s", "a", "r", "s2", "done", "eps1", "eps2")

    def __init__(self, ctx: Context, spec: SACSpec, batch: int, weights: dict | None = None, dp: bool = False):
        self.ctx, self.spec, self.B, self.dp = ctx, spec, int(batch), dp
        S, A, H, B = spec.state, spec.action, spec.hidden, self.B
        w = weights if weights is not None else sac_weights(spec)

        def actor_layers():
            return [DenseLayer(ctx, S, NONE, ADAM, B, H), DenseLayer(ctx, H, LRELU, ADAM, B, H),
                    DenseLayer(ctx, H, LRELU, ADAM, B, 2 * A), DenseLayer(ctx, 2 * A, NONE, ADAM, B, 0)]

        def critic_layers():
            return [DenseLayer(ctx, S, NONE, ADAM, B, 0), ConcatLayer(ctx, H, S, A, LRELU, ADAM, B, H),
                    DenseLayer(ctx, H, LRELU, ADAM, B, 1), DenseLayer(ctx, 1, NONE, ADAM, B, 0)]

        self.actor = actor_layers()
        self.actor_next = actor_layers()
        self.critics = [critic_layers() for _ in range(2)]
        self.critics_pi = [critic_layers() for _ in range(2)]
        self.targets = [critic_layers() for _ in range(2)]
        for view, src in zip(self.actor_next, self.actor):
            view.share_params(src)
        for k in range(2):
            for view, src in zip(self.critics_pi[k], self.critics[k]):
                view.share_params(src)

        # replay inputs and policy buffers
        self.s, self.s2 = self.actor[0].output, self.actor_next[0].output
        self.a = self.critics[0][1].second
        self.r, self.done, self.y = ctx.buffer(B), ctx.buffer(B), ctx.buffer(B)
        self.eps1, self.eps2 = ctx.buffer(B * A), ctx.buffer(B * A)
        self.a_next, self.logp_next = self.targets[0][1].second, ctx.buffer(B)
        self.a_pi, self.logp = self.critics_pi[0][1].second, ctx.buffer(B)
        _use_buffer(self.critics[1][1], "second", self.a)
        _use_buffer(self.targets[1][1], "second", self.a_next)
        _use_buffer(self.critics_pi[1][1], "second", self.a_pi)
        for net in self.critics + self.critics_pi:
            _use_buffer(net[0], "output", self.s)
        for net in self.targets:
            _use_buffer(net[0], "output", self.s2)
        for net in self.critics_pi:  # dQ/dQ = 1 at the critic output of the actor pass
            ctx.fill(net[-1].gradient, 1.0, B)

        self._set_weights(w)
        self.actor_next_net = Net(ctx, self.actor_next, loss=False)
        self.target_nets = [Net(ctx, t, loss=False) for t in self.targets]
        self.critic_nets = [Net(ctx, c, target=self.y) for c in self.critics]
        self.pi_nets = [Net(ctx, c, loss=False) for c in self.critics_pi]
        self.actor_net = Net(ctx, self.actor, loss=False)

        def kern(name, *args):
            return ctx.kernel(name).args(*args).batch(B)

        out_next, out = self.actor_next[-1].output, self.actor[-1].output
        policy_next = Op(kern("SACGaussianPolicy", out_next, self.eps1, self.a_next, self.logp_next, A), (1,))
        target_value = Op(kern("SACTargetValue", self.targets[0][-1].output, self.targets[1][-1].output, self.r,
                               self.done, self.logp_next, self.y, spec.gamma, spec.alpha), (1,))
        policy = Op(kern("SACGaussianPolicy", out, self.eps2, self.a_pi, self.logp, A), (1,))
        policy_grad = Op(kern("SACPolicyGradient", out, self.eps2, self.a_pi, self.critics_pi[0][-1].output,
                              self.critics_pi[1][-1].output, self.critics_pi[0][1].second_grad,
                              self.critics_pi[1][1].second_grad, self.actor[-1].gradient, A, spec.alpha), (1,))
        polyak = []
        for k in range(2):
            for tl, cl in zip(self.targets[k], self.critics[k]):
                polyak += tl.soft_update_ops(cl, spec.tau, spec.soft_update_adam)
        c1, c2 = self.critic_nets
        p1, p2 = self.pi_nets
        # (ops, inside a data-parallel update region)
        self.phases = [
            (self.actor_next_net.fwd_ops + [policy_next] + self.target_nets[0].fwd_ops + self.target_nets[1].fwd_ops
             + [target_value] + c1.fwd_ops + c2.fwd_ops + c1.bwd_ops + c2.bwd_ops, False),
            (c1.upd_ops + c2.upd_ops, True),
            (self.actor_net.fwd_ops + [policy] + p1.fwd_ops + p2.fwd_ops + p1.bwd_ops + p2.bwd_ops + [policy_grad]
             + self.actor_net.bwd_ops, False),
            (self.actor_net.upd_ops, True),
            (polyak, False),
        ]
        self.lists = None

    def _set_weights(self, w: dict) -> None:
        for layer, arr in zip(self.actor[:3], w["actor"]):
            layer.set_weights(arr)
        for k in range(2):
            cw = w["critics"][k]
            for net in (self.critics[k], self.targets[k]):
                net[1].set_conc_weights(cw["conc"])
                net[1].set_weights(cw["w1"])
                net[2].set_weights(cw["w2"])

    # ----------------------------------------------------------------- run
    def set_batch(self, batch: dict) -> None:
        """Write one replay batch (arrays of sac_data for one step) into the agent's input buffers."""
        for name in self.INPUTS:
            self.ctx.write(getattr(self, name), batch[name])

    def launch_count(self) -> int:
        return sum(len(ops) for ops, _ in self.phases)

    def capture(self) -> None:
        """Record every phase into a command list (nothing runs while recording)."""
        ctx = self.ctx
        self.lists = []
        for ops, _ in self.phases:
            ctx.record_begin()
            try:
                for op in ops:
                    op.kernel.run(op.gsize, op.lsize)
            finally:
                self.lists.append(ctx.record_end())

    def step(self) -> None:
        """One SAC update (eager enqueue, or replay of the recorded lists with the Adam rates patched)."""
        ctx = self.ctx
        for p, (ops, region) in enumerate(self.phases):
            if region and self.dp:
                ctx.dp_update_begin()
            if self.lists is None:
                for op in ops:
                    op()
            else:
                lid = self.lists[p]
                for pos, op in enumerate(ops):
                    if isinstance(op, AdamOp):
                        for idx, value in op.patches():
                            ctx.list_set_float(lid, pos, idx, value)
                ctx.run_list(lid)
            if region and self.dp:
                ctx.dp_update_end()

    def q_values(self) -> np.ndarray:
        """[2][batch] critic outputs on (s, a) of the last step (read back)."""
        return np.stack([self.ctx.read(c[-1].output, self.B) for c in self.critics])
