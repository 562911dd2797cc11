"""Network sequencing over the C ABI, mirroring the reference's CNet.

`Net` holds a list of layers (layer 0 is the input layer) and builds, once,
the exact kernel sequence of one training step of CNet::feedForward /
CNet::backPropOCL (NeuroNet_Core.mqh:13246-13417, 13555-13763):

  forward      l = 1..L-1   layer[l] feed forward from layer[l-1]
  output grad  layer[L-1]   CalcOutputGradient against the target
  hidden grads l = L-2..0   layer[l] from layer[l+1] (dense) or
                            layer[l+1].calcInputGradients(layer[l])
  updates      l = L-1..1   layer[l].updateInputWeights(layer[l-1])

`step()` enqueues that sequence; `capture()` records it once into a command
list so that later steps replay it with one C-ABI call after patching the
per-step Adam rates.  Data parallelism (`dp=True`) wraps the updates in an
nn_dp_update_begin/end region: every update kernel contributes its batch-mean
weight gradient to one NCCL allreduce, then the updates run.
"""
from __future__ import annotations

import numpy as np

from .api import Context
from .layers import AdamOp, DenseLayer, Layer, Op


class Net:
    def __init__(self, ctx: Context, layers: list[Layer], dp: bool = False, target: int | None = None,
                 loss: bool = True):
        """`target`: an existing target buffer to train against (default: a new one).  `loss=False`:
        the backward pass starts from whatever the last layer's gradient buffer holds (no
        CalcOutputGradient), for networks whose output gradient comes from another kernel."""
        self.ctx, self.layers, self.dp, self.loss = ctx, layers, dp, loss
        self.batch = layers[0].batch
        self.target = target if target is not None else ctx.buffer(layers[-1].neurons * self.batch)
        self.fwd_ops = self._forward_ops()
        self.bwd_ops = self._backward_ops()
        self.upd_ops = self._update_ops()
        self.adam_ops = [op for op in self.upd_ops if isinstance(op, AdamOp)]
        self.list_id = None
        self.list_positions = None
        self.loss_buf = None

    # ---------------------------------------------------------------- build
    def _forward_ops(self) -> list[Op]:
        ops = []
        for l in range(1, len(self.layers)):
            ops += self.layers[l].forward_ops(self.layers[l - 1])
        return ops

    def _backward_ops(self) -> list[Op]:
        ops = list(self.layers[-1].output_gradient_ops(self.target)) if self.loss else []
        for l in range(len(self.layers) - 2, -1, -1):
            cur, nxt = self.layers[l], self.layers[l + 1]
            if type(nxt) is DenseLayer:  # CNeuronBaseOCL::CalcHiddenGradients dispatch, NeuroNet_Core.mqh:15988-16014
                ops += cur.hidden_gradient_ops(nxt)
            else:
                ops += nxt.input_gradient_ops(cur)
        return ops

    def _update_ops(self) -> list[Op]:
        ops = []
        for l in range(len(self.layers) - 1, 0, -1):
            ops += self.layers[l].update_ops(self.layers[l - 1])
        return ops

    # ----------------------------------------------------------------- run
    def set_input(self, x: np.ndarray) -> None:
        self.ctx.write(self.layers[0].output, x)

    def set_target(self, t: np.ndarray) -> None:
        self.ctx.write(self.target, t)

    def forward(self) -> None:
        for op in self.fwd_ops:
            op()

    def backward(self) -> None:
        for op in self.bwd_ops:
            op()

    def update(self) -> None:
        if self.dp:
            self.ctx.dp_update_begin()
        for op in self.upd_ops:
            op()
        if self.dp:
            self.ctx.dp_update_end()

    def step(self) -> None:
        """One forward + backward + update (eager enqueue)."""
        if self.list_id is not None:
            self.replay()
            return
        self.forward()
        self.backward()
        self.update()

    def capture(self) -> tuple[int, int]:
        """Record the step into two command lists -- forward + backward, and the updates (nothing
        runs while recording).  Two lists so that a data-parallel update region can enclose the
        second one.  Per-step scalars (Adam rates, sample counts) are patched at every replay."""
        ctx = self.ctx
        ops = self.fwd_ops + self.bwd_ops + self.upd_ops
        if not all(op.recordable for op in ops):
            raise RuntimeError("this network has steps that cannot be recorded (gated updates); run it eagerly")
        self.recorded = []
        lists = []
        for group in (self.fwd_ops + self.bwd_ops, self.upd_ops):
            ctx.record_begin()
            try:
                for pos, op in enumerate(group):
                    self.recorded.append((len(lists), pos, op))
                    op.kernel.run(op.gsize, op.lsize)
            finally:
                lists.append(ctx.record_end())
        self.list_fb, self.list_upd = lists
        self.list_id = (self.list_fb, self.list_upd)
        return self.list_id

    def replay(self) -> None:
        ctx = self.ctx
        for li, pos, op in self.recorded:
            for idx, value in op.patches():
                lid = self.list_id[li]
                if op.kernel.sig[idx] == "f":
                    ctx.list_set_float(lid, pos, idx, value)
                else:
                    ctx._check(ctx.lib.nn_cmdlist_set_int(lid, pos, idx, int(value)))
        ctx.run_list(self.list_fb)
        if self.dp:
            ctx.dp_update_begin()
        ctx.run_list(self.list_upd)
        if self.dp:
            ctx.dp_update_end()

    def output(self) -> np.ndarray:
        return self.ctx.read(self.layers[-1].output, self.layers[-1].neurons * self.batch)

    def mse(self) -> float:
        """Host-side MSE of the output against the target (CNet::backPropOCL reads the output,
        NeuroNet_Core.mqh:13584-13599)."""
        y = self.output()
        t = self.ctx.read(self.target, y.size)
        return float(np.mean((y.astype(np.float64) - t) ** 2))

    def launch_count(self) -> int:
        return len(self.fwd_ops) + len(self.bwd_ops) + len(self.upd_ops)
