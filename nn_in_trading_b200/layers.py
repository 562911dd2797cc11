"""Layer classes over the C ABI, mirroring the reference's CNeuron*OCL classes.

Each class owns its device buffers and issues exactly the kernel sequence of
its reference counterpart (cited per method), with the reference's NDRanges
and arguments.  Kernel instances are created per call site and their
arguments bound once (the C ABI keeps arguments between executions), so a
training step only enqueues executions -- and can be recorded once into a
command list and replayed (net.Net).

Batching: every per-sample buffer holds `batch` consecutive samples and every
kernel instance is given nn_set_batch(batch); parameter buffers are shared.
"""
from __future__ import annotations

import math

import numpy as np

from .api import ADAM, GELU, NONE, SGD, Context, Kernel

LR = 3.0e-4       # NeuroNet_Definitions.mqh:38
MOMENTUM = 0.9    # NeuroNet_Definitions.mqh:40
B1 = 0.9          # NeuroNet_Definitions.mqh:44
B2 = 0.999        # NeuroNet_Definitions.mqh:46
MAX_LOCAL = 256   # GetMaxLocalSize(1) reported to the layers


def adam_lt(t: int, lr: float = LR, b1: float = B1, b2: float = B2) -> float:
    """Bias-corrected Adam rate as the MQL5 host computes it, in double, then cast to float
    (NeuroNet_Core.mqh:15903)."""
    return float(np.float32(lr * math.sqrt(1.0 - math.pow(b2, t)) / (1.0 - math.pow(b1, t))))


class Op:
    """One kernel execution of a training step (a bound kernel instance plus its NDRange)."""

    def __init__(self, kernel: Kernel, gsize, lsize=None):
        self.kernel, self.gsize, self.lsize = kernel, tuple(gsize), None if lsize is None else tuple(lsize)

    def prepare(self) -> None:
        """Host-side work before the launch (e.g. the per-step Adam rate)."""

    def __call__(self) -> None:
        self.prepare()
        self.kernel.run(self.gsize, self.lsize)


class AdamOp(Op):
    """An Adam update whose learning-rate argument is bias-corrected from the owner's step counter,
    which is incremented after every update (NeuroNet_Core.mqh:15903-15914; Attention.mqh:2355-2366)."""

    def __init__(self, kernel: Kernel, gsize, lsize, owner, l_index: int):
        super().__init__(kernel, gsize, lsize)
        self.owner, self.l_index = owner, l_index
        self.last_lt = None

    def next_lt(self) -> float:
        lt = adam_lt(self.owner.t)
        self.owner.t += 1
        self.last_lt = lt
        return lt

    def prepare(self) -> None:
        self.kernel.set(self.l_index, self.next_lt())


class Layer:
    """Common state of every layer: output and gradient buffers of `neurons` floats per sample."""

    def __init__(self, ctx: Context, neurons: int, activation: int = NONE, optimization: int = ADAM,
                 batch: int = 1):
        self.ctx, self.neurons, self.activation = ctx, int(neurons), int(activation)
        self.optimization, self.batch = optimization, int(batch)
        self.output = ctx.buffer(self.neurons * self.batch)
        self.gradient = ctx.buffer(self.neurons * self.batch)
        self.t = 1
        self.weights = None

    def kernel(self, name: str) -> Kernel:
        k = self.ctx.kernel(name)
        if self.batch != 1:
            k.batch(self.batch)
        return k

    # sequencing hooks (overridden)
    def forward_ops(self, prev: "Layer") -> list[Op]:
        raise NotImplementedError

    def input_gradient_ops(self, prev: "Layer") -> list[Op]:
        raise NotImplementedError

    def update_ops(self, prev: "Layer") -> list[Op]:
        return []

    def output_gradient_ops(self, target: int) -> list[Op]:
        """CNeuronBaseOCL::calcOutputGradients (NeuroNet_Core.mqh:15800-15837)."""
        k = self.kernel("CalcOutputGradient").args(target, self.output, self.gradient, self.activation, 1.0)
        return [Op(k, (self.neurons,))]


class DenseLayer(Layer):
    """CNeuronBaseOCL (NeuroNet_Core.mqh:15464-16060): a dense layer.  Its `weights` are the
    weights *towards the next dense layer*, [next][neurons+1] with the bias last."""

    def __init__(self, ctx, neurons, activation=NONE, optimization=ADAM, batch=1, outputs=0):
        super().__init__(ctx, neurons, activation, optimization, batch)
        self.outputs = int(outputs)
        if self.outputs:
            n = self.outputs * (self.neurons + 1)
            self.weights = ctx.buffer(n)
            if optimization == SGD:
                self.delta = ctx.buffer(n)
            else:
                self.m = ctx.buffer(n)
                self.v = ctx.buffer(n)

    def set_weights(self, w: np.ndarray) -> None:
        self.ctx.write(self.weights, w)

    def forward_ops(self, prev: "DenseLayer") -> list[Op]:
        """feedForwardChecked, NeuroNet_Core.mqh:15686-15740."""
        loc = min((prev.neurons + 3) // 4, MAX_LOCAL)
        k = self.kernel("FeedForward").args(prev.weights, prev.output, self.output, prev.neurons, self.activation,
                                            self.output, 0)
        return [Op(k, (self.neurons, loc), (1, loc))]

    def hidden_gradient_ops(self, nxt: "DenseLayer") -> list[Op]:
        """calcHiddenGradients, NeuroNet_Core.mqh:15744-15769."""
        loc = min((nxt.neurons + 3) // 4, MAX_LOCAL)
        k = self.kernel("CalcHiddenGradient").args(self.weights, nxt.gradient, self.output, self.gradient,
                                                   nxt.neurons, self.activation)
        return [Op(k, (self.neurons, loc), (1, loc))]

    def update_ops(self, prev: "DenseLayer") -> list[Op]:
        """updateInputWeights, NeuroNet_Core.mqh:15869-15984: the update of prev's weights and NormalizeWeights."""
        if prev.optimization == SGD:
            k = self.kernel("UpdateWeightsMomentum").args(prev.weights, self.gradient, prev.output, prev.delta,
                                                          prev.neurons, LR, MOMENTUM)
            ops = [Op(k, (self.neurons, prev.neurons + 1))]
        else:
            k = self.kernel("UpdateWeightsAdam").args(prev.weights, self.gradient, prev.output, prev.m, prev.v,
                                                      prev.neurons, LR, B1, B2)
            ops = [AdamOp(k, (self.neurons, prev.neurons + 1), None, self, 6)]
        kn = self.ctx.kernel("NormalizeWeights").args(prev.weights, prev.neurons + 1)
        ops.append(Op(kn, (self.neurons,)))
        return ops


class MLMHAttentionLayer(Layer):
    """CNeuronMLMHAttentionOCL (NeuroNet_Attention.mqh:1576-2405): `layers` encoder blocks of
    QKV 1x1-conv, multi-head score/out, W0, Sum&Normalize, FF(4x window, GELU), FF(activation),
    Sum&Normalize over `units` tokens of `window` features."""

    def __init__(self, ctx, window, window_key, heads, units, layers, activation=NONE, optimization=ADAM,
                 batch=1):
        super().__init__(ctx, window * units, activation, optimization, batch)
        if optimization != ADAM:
            raise ValueError("MLMH attention layer: only the Adam path is built")
        self.window, self.dk, self.heads, self.units, self.layers = window, window_key, heads, units, layers
        B = batch
        num = 3 * window_key * heads * units
        out = window * units
        self.qkv_w_count = 3 * (window + 1) * window_key * heads
        self.w0_count = (window_key + 1) * heads * window
        self.ff1_count = 4 * (window + 1) * window
        self.ff2_count = (4 * window + 1) * window
        self.qkv, self.qkv_g, self.scores, self.ao, self.ao_g = [], [], [], [], []
        self.ff = []   # per layer: [attn_out, ff1_out, ff2_out, attn_out_g, ff1_out_g, ff2_out_g]
        self.w = []    # per layer: dict name -> (weights, m, v)
        for i in range(layers):
            self.qkv.append(ctx.buffer(num * B))
            self.qkv_g.append(ctx.buffer(num * B))
            self.scores.append(ctx.buffer(units * units * heads * B))
            self.ao.append(ctx.buffer(window_key * heads * units * B))
            self.ao_g.append(ctx.buffer(window_key * heads * units * B))
            last = i == layers - 1
            t = [ctx.buffer(out * B), ctx.buffer(4 * out * B), self.output if last else ctx.buffer(out * B),
                 ctx.buffer(out * B), ctx.buffer(4 * out * B), self.gradient if last else ctx.buffer(out * B)]
            self.ff.append(t)
            ws = {}
            for name, n in (("qkv", self.qkv_w_count), ("w0", self.w0_count), ("ff1", self.ff1_count),
                            ("ff2", self.ff2_count)):
                ws[name] = (ctx.buffer(n), ctx.buffer(n), ctx.buffer(n))
            self.w.append(ws)

    def weight_shapes(self) -> dict:
        return {"qkv": self.qkv_w_count, "w0": self.w0_count, "ff1": self.ff1_count, "ff2": self.ff2_count}

    def set_weights(self, layer: int, name: str, w: np.ndarray) -> None:
        self.ctx.write(self.w[layer][name][0], w)

    # ConvolutionForward, NeuroNet_Attention.mqh:1944-1992
    def _conv_fwd(self, w, inputs, outputs, in_total, window, window_out, act, n_out):
        k = self.kernel("FeedForwardConv").args(w, inputs, outputs, in_total, window, window, window_out, act)
        return Op(k, (n_out // window_out, window_out, 1))

    # SumAndNormalize, NeuroNet_Core.mqh:17959-18075
    def _sum_norm(self, a, b, out, normalize=True):
        rows = self.window * self.units // self.window
        k = self.kernel("SumMatrix").args(a, b, out, self.window, 0.5, 0, 0, 0, out, 0)
        ops = [Op(k, (rows,))]
        if normalize:
            kn = self.kernel("Normalize").args(out, self.window)
            ops.append(Op(kn, (rows,)))
        return ops

    def forward_ops(self, prev: Layer) -> list[Op]:
        """feedForward, NeuroNet_Attention.mqh:1884-1940."""
        W, U, H, D = self.window, self.units, self.heads, self.dk
        out = W * U
        ops = []
        for i in range(self.layers):
            inputs = prev.output if i == 0 else self.ff[i - 1][2]
            ws = self.w[i]
            ops.append(self._conv_fwd(ws["qkv"][0], inputs, self.qkv[i], out, W, 3 * D * H, NONE, 3 * D * H * U))
            ks = self.kernel("MHAttentionScore").args(self.qkv[i], self.scores[i], D, 0)
            ops.append(Op(ks, (U, H)))
            ko = self.kernel("MHAttentionOut").args(self.scores[i], self.qkv[i], self.ao[i], D)
            ops.append(Op(ko, (U, H)))
            t = self.ff[i]
            ops.append(self._conv_fwd(ws["w0"][0], self.ao[i], t[0], D * H * U, D * H, W, NONE, out))
            ops += self._sum_norm(t[0], inputs, t[0])
            ops.append(self._conv_fwd(ws["ff1"][0], t[0], t[1], out, W, 4 * W, GELU, 4 * out))
            ops.append(self._conv_fwd(ws["ff2"][0], t[1], t[2], 4 * out, 4 * W, W, self.activation, out))
            ops += self._sum_norm(t[2], t[0], t[2])
        return ops

    # ConvolutionInputGradients, NeuroNet_Attention.mqh:2128-2183
    def _conv_dgrad(self, w, grad, inputs, in_grad, grad_total, in_total, window, window_out, act):
        k = self.kernel("CalcHiddenGradientConv").args(w, grad, inputs, in_grad, grad_total, window, window,
                                                       window_out, act, 0)
        return Op(k, (in_total, 1))

    def input_gradient_ops(self, prev: Layer) -> list[Op]:
        """calcInputGradients, NeuroNet_Attention.mqh:2063-2124."""
        W, U, H, D = self.window, self.units, self.heads, self.dk
        out = W * U
        ops = []
        out_grad = self.gradient
        for i in range(self.layers - 1, -1, -1):
            t, ws = self.ff[i], self.w[i]
            ops.append(self._conv_dgrad(ws["ff2"][0], out_grad, t[1], t[4], out, 4 * out, 4 * W, W, NONE))
            ops.append(self._conv_dgrad(ws["ff1"][0], t[4], t[0], t[3], 4 * out, out, W, 4 * W, GELU))
            ops += self._sum_norm(out_grad, t[3], t[3], normalize=False)
            out_grad = t[3]
            ops.append(self._conv_dgrad(ws["w0"][0], out_grad, self.ao[i], self.ao_g[i], out, D * H * U, D * H, W,
                                        NONE))
            kg = self.kernel("MHAttentionInsideGradients").args(self.qkv[i], self.qkv_g[i], self.scores[i],
                                                                self.ao_g[i])
            ops.append(Op(kg, (U, H, D)))
            if i == 0:
                inp, tmp = prev.output, prev.gradient
            else:
                inp, tmp = self.ff[i - 1][2], self.ff[i - 1][5]
            ops.append(self._conv_dgrad(ws["qkv"][0], self.qkv_g[i], inp, tmp, 3 * D * H * U, out, W, 3 * D * H,
                                        NONE))
            ops += self._sum_norm(out_grad, tmp, tmp, normalize=False)
            if i > 0:
                out_grad = tmp
        return ops

    # ConvolutuionUpdateWeights (ADAM), NeuroNet_Attention.mqh:2264-2405
    def _conv_update(self, wmv, grad, inputs, in_total, window, window_out):
        w, m, v = wmv
        k = self.kernel("UpdateWeightsConvAdam").args(w, grad, inputs, m, v, in_total, LR, B1, B2, window,
                                                      window_out, window)
        n = {3 * self.dk * self.heads: self.qkv_w_count}.get(window_out, None)
        total = (window + 1) * window_out
        kn = self.ctx.kernel("NormalizeWeights").args(w, window + 1)
        return [AdamOp(k, (total,), None, self, 6), Op(kn, (window_out,))]

    def update_ops(self, prev: Layer) -> list[Op]:
        """updateInputWeights, NeuroNet_Attention.mqh:2231-2260."""
        W, U, H, D = self.window, self.units, self.heads, self.dk
        out = W * U
        ops = []
        inputs = prev.output
        for l in range(self.layers):
            t, ws = self.ff[l], self.w[l]
            ops += self._conv_update(ws["qkv"], self.qkv_g[l], inputs, out, W, 3 * D * H)
            ops += self._conv_update(ws["w0"], t[3], self.ao[l], D * H * U, D * H, W)
            ops += self._conv_update(ws["ff1"], t[4], t[0], out, W, 4 * W)
            ops += self._conv_update(ws["ff2"], t[5], t[1], 4 * out, 4 * W, W)
            inputs = t[2]
        return ops
