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

from .api import ADAM, ADAM_MINI, GELU, LRELU, NONE, SGD, SIGMOID, Context, Kernel

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

    recordable = True  # may be recorded into a command list

    def __init__(self, kernel: Kernel, gsize, lsize=None):
        self.kernel, self.gsize, self.lsize = kernel, tuple(gsize), None if lsize is None else tuple(lsize)

    def patches(self) -> list:
        """Per-step scalar arguments [(index, value)] computed on the host before the launch (the
        bias-corrected Adam rate, the BatchNorm sample count); advances host state."""
        return []

    def prepare(self) -> None:
        for idx, value in self.patches():
            self.kernel.set(idx, value)

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

    def patches(self) -> list:
        return [(self.l_index, self.next_lt())]


class Layer:
    """CNeuronBaseOCL state shared by every layer: output and gradient buffers of `neurons` floats per
    sample and, when the next layer is dense, the weights toward it, [next][neurons+1] with the bias
    last (NeuroNet_Core.mqh:15496-15649: every layer class derives from CNeuronBaseOCL)."""

    def __init__(self, ctx: Context, neurons: int, activation: int = NONE, optimization: int = ADAM,
                 batch: int = 1, outputs: int = 0):
        self.ctx, self.neurons, self.activation = ctx, int(neurons), int(activation)
        self.optimization, self.batch = optimization, int(batch)
        self.output = ctx.buffer(self.neurons * self.batch)
        self.gradient = ctx.buffer(self.neurons * self.batch)
        self.t = 1
        self.weights = None
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

    def hidden_gradient_ops(self, nxt: "Layer") -> list["Op"]:
        """calcHiddenGradients, NeuroNet_Core.mqh:15744-15769 (next layer dense)."""
        loc = min((nxt.neurons + 3) // 4, MAX_LOCAL)
        k = self.kernel("CalcHiddenGradient").args(self.weights, nxt.gradient, self.output, self.gradient,
                                                   nxt.neurons, self.activation)
        return [Op(k, (self.neurons, loc), (1, loc))]

    def per_sample(self, other: "Layer") -> int:
        """Floats per sample of `other`'s buffers counted in this layer's batch units (a layer may view its
        neighbour's buffer as more, shorter samples, e.g. per-channel sequences)."""
        return other.neurons * other.batch // self.batch

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

    def soft_update_ops(self, source: "Layer", tau: float, adam: bool | None = None) -> list["Op"]:
        """CNeuronBaseOCL::WeightsUpdate (NeuroNet_Core.mqh:20283-20370): SoftUpdateAdam on the weights
        toward the next layer (with this layer's moments) when Adam and tau != 1, else SoftUpdate.
        `adam` overrides that choice (False: plain Polyak averaging whatever the optimizer)."""
        if self.weights is None:
            return []
        n = self.outputs * (self.neurons + 1)
        if adam is None:
            adam = tau != 1.0 and self.optimization == ADAM
        if adam:
            k = self.ctx.kernel("SoftUpdateAdam").args(self.weights, source.weights, self.m, self.v, tau, B1, B2)
        else:
            k = self.ctx.kernel("SoftUpdate").args(self.weights, source.weights, tau)
        return [Op(k, (n,))]

    def param_handles(self) -> list[str]:
        """Attribute names of the parameter buffers (weights and optimizer state)."""
        if self.weights is None:
            return []
        return ["weights", "delta"] if self.optimization == SGD else ["weights", "m", "v"]

    def share_params(self, source: "Layer") -> None:
        """Use `source`'s parameter buffers (a second activation/gradient set over the same weights)."""
        for name in self.param_handles():
            self.ctx.free(getattr(self, name))
            setattr(self, name, getattr(source, name))

    def output_gradient_ops(self, target: int) -> list[Op]:
        """CNeuronBaseOCL::calcOutputGradients (NeuroNet_Core.mqh:15800-15837)."""
        k = self.kernel("CalcOutputGradient").args(target, self.output, self.gradient, self.activation, 1.0)
        return [Op(k, (self.neurons,))]


class DenseLayer(Layer):
    """CNeuronBaseOCL (NeuroNet_Core.mqh:15464-16060): a dense layer fed by the previous layer's weights."""

    def forward_ops(self, prev: "DenseLayer") -> list[Op]:
        """feedForwardChecked, NeuroNet_Core.mqh:15686-15740."""
        loc = min((prev.neurons + 3) // 4, MAX_LOCAL)
        k = self.kernel("FeedForward").args(prev.weights, prev.output, self.output, prev.neurons, self.activation,
                                            self.output, 0)
        return [Op(k, (self.neurons, loc), (1, loc))]

    def update_ops(self, prev: "Layer") -> list[Op]:
        """updateInputWeights, NeuroNet_Core.mqh:15869-15984: the update of prev's weights and NormalizeWeights."""
        if prev.optimization == SGD:
            k = self.kernel("UpdateWeightsMomentum").args(prev.weights, self.gradient, prev.output, prev.delta,
                                                          prev.neurons, LR, MOMENTUM)
            ops = [Op(k, (self.neurons, prev.neurons + 1))]
        elif prev.optimization == ADAM_MINI:  # NeuroNet_Core.mqh:15939-15957: one second moment per output
            k = self.kernel("UpdateWeightsAdamMini").args(prev.weights, self.gradient, prev.output, prev.m, prev.v,
                                                          LR, B1, B2)
            ops = [AdamOp(k, (prev.neurons + 1, self.neurons), (prev.neurons + 1, 1), self, 5)]
        else:
            k = self.kernel("UpdateWeightsAdam").args(prev.weights, self.gradient, prev.output, prev.m, prev.v,
                                                      prev.neurons, LR, B1, B2)
            ops = [AdamOp(k, (self.neurons, prev.neurons + 1), None, self, 6)]
        kn = self.ctx.kernel("NormalizeWeights").args(prev.weights, prev.neurons + 1)
        ops.append(Op(kn, (self.neurons,)))
        return ops


class ConcatLayer(Layer):
    """CNeuronConcatenate (NeuroNet_Misc.mqh:286-680): output = act(W [x1; x2; 1]) with the previous
    layer's output as x1 and a second input buffer x2 (`second`, `inputs2` floats per sample), its own
    weights [neurons][inputs1 + inputs2 + 1] (bias last), no NormalizeWeights after its update.  As a
    CNeuronBaseOCL it also holds the weights toward the next dense layer."""

    def __init__(self, ctx, neurons, inputs1, inputs2, activation=NONE, optimization=ADAM, batch=1, outputs=0):
        super().__init__(ctx, neurons, activation, optimization, batch, outputs)
        self.inputs1, self.inputs2 = int(inputs1), int(inputs2)
        n = self.neurons * (self.inputs1 + self.inputs2 + 1)
        self.conc_w = ctx.buffer(n)
        if optimization == SGD:
            self.conc_dw = ctx.buffer(n)
        else:
            self.conc_m = ctx.buffer(n)
            self.conc_v = ctx.buffer(n)
        self.second = ctx.buffer(self.inputs2 * self.batch)        # x2 of every sample
        self.second_grad = ctx.buffer(self.inputs2 * self.batch)   # d/dx2 written by calcInputGradients
        self.second_activation = NONE

    def set_conc_weights(self, w: np.ndarray) -> None:
        self.ctx.write(self.conc_w, w)

    def forward_ops(self, prev: Layer) -> list[Op]:
        """feedForward, NeuroNet_Misc.mqh:386-418 -> Concat_FeedForward over the layer's outputs."""
        k = self.kernel("Concat_FeedForward").args(self.conc_w, prev.output, self.second, self.output,
                                                   self.per_sample(prev), self.inputs2, self.activation)
        return [Op(k, (self.neurons,))]

    def input_gradient_ops(self, prev: Layer) -> list[Op]:
        """calcInputGradients, NeuroNet_Misc.mqh:421-462 -> Concat_HiddenGradient over inputs1 + inputs2."""
        n1 = self.per_sample(prev)
        k = self.kernel("Concat_HiddenGradient").args(self.conc_w, self.gradient, prev.output, self.second,
                                                      prev.gradient, self.second_grad, self.neurons, n1,
                                                      self.inputs2, prev.activation, self.second_activation)
        return [Op(k, (n1 + self.inputs2,))]

    def update_ops(self, prev: Layer) -> list[Op]:
        """updateInputWeights, NeuroNet_Misc.mqh:465-560: Concat_UpdateWeightsMomentum or _Adam over
        (neurons, inputs1 + inputs2 + 1), the Adam rate bias-corrected from this layer's step counter.
        (The reference's SGD branch binds inputs2 into the inputs1 slot, NeuroNet_Misc.mqh:501-502; this
        host binds both counts.)"""
        n1 = self.per_sample(prev)
        gsize = (self.neurons, n1 + self.inputs2 + 1)
        if prev.optimization == SGD:
            k = self.kernel("Concat_UpdateWeightsMomentum").args(self.conc_w, self.gradient, prev.output, self.second,
                                                                 self.conc_dw, n1, self.inputs2, LR, MOMENTUM)
            return [Op(k, gsize)]
        k = self.kernel("Concat_UpdateWeightsAdam").args(self.conc_w, self.gradient, prev.output, self.second,
                                                         self.conc_m, self.conc_v, n1, self.inputs2, LR, B1, B2)
        return [AdamOp(k, gsize, None, self, 8)]

    def soft_update_ops(self, source: "ConcatLayer", tau: float, adam: bool | None = None) -> list[Op]:
        """WeightsUpdate, NeuroNet_Misc.mqh:628-676: the base weights, then the concat weights."""
        ops = super().soft_update_ops(source, tau, adam)
        if adam is None:
            adam = tau != 1.0 and self.optimization == ADAM
        if adam:
            k = self.ctx.kernel("SoftUpdateAdam").args(self.conc_w, source.conc_w, self.conc_m, self.conc_v, tau,
                                                       B1, B2)
        else:
            k = self.ctx.kernel("SoftUpdate").args(self.conc_w, source.conc_w, tau)
        n = self.neurons * (self.inputs1 + self.inputs2 + 1)
        return ops + [Op(k, (n,))]

    def param_handles(self) -> list[str]:
        return super().param_handles() + (["conc_w", "conc_dw"] if self.optimization == SGD
                                          else ["conc_w", "conc_m", "conc_v"])


class MLMHAttentionLayer(Layer):
    """CNeuronMLMHAttentionOCL (NeuroNet_Attention.mqh:1576-2405): `layers` encoder blocks of
    QKV 1x1-conv, multi-head score/out, W0, Sum&Normalize, FF(4x window, GELU), FF(activation),
    Sum&Normalize over `units` tokens of `window` features."""

    def __init__(self, ctx, window, window_key, heads, units, layers, activation=NONE, optimization=ADAM,
                 batch=1, outputs=0):
        super().__init__(ctx, window * units, activation, optimization, batch, outputs)
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


class ConvLayer(Layer):
    """CNeuronConvOCL (NeuroNet_Core.mqh:17132-17448): strided 1-D convolution over `variables`
    independent channels, weights [var][window_out][window+1]; no NormalizeWeights after its update."""

    def __init__(self, ctx, window, step, window_out, units, variables=1, activation=NONE, optimization=ADAM,
                 batch=1, outputs=0):
        super().__init__(ctx, units * window_out * variables, activation, optimization, batch, outputs)
        self.window, self.step, self.window_out, self.units, self.variables = window, step, window_out, units, variables
        n = (window + 1) * window_out * variables
        self.conv_w = ctx.buffer(n)
        self.conv_m = ctx.buffer(n)
        self.conv_v = ctx.buffer(n)

    def set_conv_weights(self, w: np.ndarray) -> None:
        self.ctx.write(self.conv_w, w)

    def forward_ops(self, prev: Layer) -> list[Op]:
        k = self.kernel("FeedForwardConv").args(self.conv_w, prev.output, self.output,
                                                self.per_sample(prev) // self.variables,
                                                self.step, self.window, self.window_out, self.activation)
        return [Op(k, (self.units, self.window_out, self.variables))]

    def input_gradient_ops(self, prev: Layer) -> list[Op]:
        k = self.kernel("CalcHiddenGradientConv").args(self.conv_w, self.gradient, prev.output, prev.gradient,
                                                       self.neurons // self.variables, self.step, self.window,
                                                       self.window_out, prev.activation, 0)
        return [Op(k, (self.per_sample(prev) // self.variables, self.variables))]

    def update_ops(self, prev: Layer) -> list[Op]:
        n = (self.window + 1) * self.window_out * self.variables
        if self.optimization == ADAM_MINI:
            # NeuroNet_Core.mqh:17355-17435: local (window+1, 1, 1), one second moment per output row
            k = self.kernel("UpdateWeightsConvAdamMini").args(self.conv_w, self.gradient, prev.output, self.conv_m,
                                                              self.conv_v, self.per_sample(prev) // self.variables,
                                                              LR, B1, B2, self.step)
            return [AdamOp(k, (self.window + 1, self.window_out, self.variables), (self.window + 1, 1, 1), self, 6)]
        k = self.kernel("UpdateWeightsConvAdam").args(self.conv_w, self.gradient, prev.output, self.conv_m,
                                                      self.conv_v, self.per_sample(prev) // self.variables, LR, B1, B2,
                                                      self.window, self.window_out, self.step)
        return [AdamOp(k, (n,), None, self, 6)]


class SoftMaxLayer(Layer):
    """CNeuronSoftMaxOCL (NeuroNet_Core.mqh:20037-20150): softmax over `heads` rows of neurons/heads;
    no weights of its own."""

    def __init__(self, ctx, neurons, heads=1, batch=1, outputs=0):
        super().__init__(ctx, neurons, NONE, ADAM, batch, outputs)
        self.heads = heads

    def forward_ops(self, prev: Layer) -> list[Op]:
        size = self.neurons // self.heads
        k = self.kernel("SoftMax_FeedForward").args(prev.output, self.output)
        return [Op(k, (size, self.heads), (size, 1))]

    def input_gradient_ops(self, prev: Layer) -> list[Op]:
        size = self.neurons // self.heads
        k = self.kernel("SoftMax_HiddenGradient").args(self.output, self.gradient, prev.gradient)
        return [Op(k, (size, self.heads), (size, 1))]

    def output_gradient_ops(self, target: int) -> list[Op]:
        """calcOutputGradients: the host copies the target into Gradient, then t / y in place."""
        kc = self.ctx.kernel("Activation").args(target, self.gradient, NONE)
        if self.batch != 1:
            kc.batch(self.batch)
        ko = self.kernel("SoftMax_OutputGradient").args(self.output, self.gradient, self.gradient)
        return [Op(kc, (self.neurons,)), Op(ko, (self.neurons,))]


class BatchNormLayer(Layer):
    """CNeuronBatchNormOCL (NeuroNet_Core.mqh:19404-19590): online normalisation of every neuron over
    the last `batch_size` samples, gamma/beta updated once 100*batch_size samples have been seen."""

    def __init__(self, ctx, neurons, batch_size, optimization=ADAM, batch=1, outputs=0):
        super().__init__(ctx, neurons, NONE, optimization, batch, outputs)
        self.batch_size = int(batch_size)
        self.width = 7 if optimization == SGD else 9
        self.options = ctx.buffer(self.neurons * self.width)
        self.count = 1  # iBatchCount

    class _BNForward(Op):
        def __init__(self, kernel, gsize, layer):
            super().__init__(kernel, gsize)
            self.layer = layer

        def patches(self):
            L = self.layer
            L.count = min(L.count, L.batch_size)
            n = L.count
            L.count += L.batch  # one count per sample trained
            return [(3, n)]

    def forward_ops(self, prev: Layer) -> list[Op]:
        self.activation = prev.activation if self.batch_size <= 1 else self.activation
        k = self.kernel("BatchFeedForward").args(prev.output, self.options, self.output, self.count,
                                                 self.optimization, self.activation, 1)
        return [BatchNormLayer._BNForward(k, (self.neurons,), self)]

    def input_gradient_ops(self, prev: Layer) -> list[Op]:
        k = self.kernel("CalcHiddenGradientBatch").args(self.options, self.gradient, prev.output, prev.gradient,
                                                        prev.activation, self.batch_size, self.optimization)
        return [_BatchArgOp(k, (self.neurons,), self, 5)]

    def update_ops(self, prev: Layer) -> list[Op]:
        if self.optimization == SGD:
            k = self.kernel("UpdateBatchOptionsMomentum").args(self.options, self.gradient, LR, MOMENTUM)
        else:
            k = self.kernel("UpdateBatchOptionsAdam").args(self.options, self.gradient, LR, B1, B2)
        # updateInputWeights runs only once iBatchCount >= 100*iBatchSize; the count is re-capped at
        # iBatchSize by every forward pass, so with iBatchSize > 1 the gate stays closed, as in the reference.
        return [_GatedOp(k, (self.neurons,), lambda: self.count >= 100 * self.batch_size)]


class _BatchArgOp(Op):
    """Binds the layer's current sample count (iBatchCount, already advanced by the forward pass, as
    CNeuronBatchNormOCL::calcInputGradients passes it) before the launch."""

    def __init__(self, kernel, gsize, layer, idx):
        super().__init__(kernel, gsize)
        self.layer, self.idx = layer, idx

    def patches(self):
        return [(self.idx, self.layer.count)]


class _GatedOp(Op):
    """Runs only while `gate()` holds (the BatchNorm update waits for 100 batches)."""

    recordable = False

    def __init__(self, kernel, gsize, gate):
        super().__init__(kernel, gsize)
        self.gate = gate

    def __call__(self):
        if self.gate():
            super().__call__()


class RevINDenormLayer(Layer):
    """CNeuronRevINDenormOCL (NeuroNet_Core.mqh:23006-23130): de-normalises with the running statistics
    (options) of a BatchNorm layer elsewhere in the network; no parameters of its own."""

    def __init__(self, ctx, neurons, norm_layer: BatchNormLayer, batch=1, outputs=0):
        super().__init__(ctx, neurons, NONE, norm_layer.optimization, batch, outputs)
        self.norm = norm_layer

    def forward_ops(self, prev: Layer) -> list[Op]:
        k = self.kernel("RevInFeedForward").args(prev.output, self.norm.options, self.output,
                                                 self.norm.neurons * self.norm.width, self.optimization)
        return [Op(k, (self.neurons,))]

    def input_gradient_ops(self, prev: Layer) -> list[Op]:
        k = self.kernel("RevInHiddenGraddient").args(prev.output, prev.gradient, self.norm.options, self.gradient,
                                                     self.norm.neurons * self.norm.width, self.optimization,
                                                     prev.activation)
        return [Op(k, (self.neurons,))]


class LSTMLayer(Layer):
    """CNeuronLSTMOCL (NeuroNet_RecurrentState.mqh:678-897): one time step per forward for `variables`
    independent series of `hidden` cells; weights [4H][in+H+1]; a batch folds into the series."""

    def __init__(self, ctx, hidden, inputs, variables=1, optimization=ADAM, batch=1, outputs=0):
        super().__init__(ctx, hidden * variables, NONE, optimization, batch, outputs)
        self.H, self.inputs, self.variables = hidden, inputs, variables
        V = variables * batch
        ws = inputs + hidden + 1
        n = 4 * hidden * ws
        self.lstm_w = ctx.buffer(n)
        self.lstm_m = ctx.buffer(n)
        self.lstm_v = ctx.buffer(n)
        self.lstm_wg = ctx.buffer(n)
        self.memory = ctx.buffer(2 * V * hidden)
        self.hidden_state = ctx.buffer(V * hidden)
        self.concatenated = ctx.buffer(V * 4 * hidden)
        self.concatenated_g = ctx.buffer(V * 4 * hidden)

    def set_lstm_weights(self, w: np.ndarray) -> None:
        self.ctx.write(self.lstm_w, w)

    def forward_ops(self, prev: Layer) -> list[Op]:
        k = self.kernel("LSTM_FeedForward").args(prev.output, self.inputs, self.lstm_w, self.concatenated,
                                                 self.memory, self.output)
        return [Op(k, (self.H, 4, self.variables), (1, 4, 1))]

    def input_gradient_ops(self, prev: Layer) -> list[Op]:
        kc = self.kernel("LSTM_ConcatenatedGradient").args(self.gradient, self.concatenated_g, self.memory,
                                                           self.concatenated)
        kh = self.kernel("LSTM_HiddenGradient").args(self.concatenated_g, prev.gradient, self.lstm_wg,
                                                     self.hidden_state, prev.output, self.lstm_w, self.output,
                                                     self.H, self.inputs)
        ops = [Op(kc, (self.H, self.variables)), Op(kh, (self.H, self.variables), (1, self.variables))]
        if prev.activation != NONE:
            kd = self.ctx.kernel("DeActivation").args(prev.output, prev.gradient, prev.gradient, prev.activation)
            if prev.batch != 1:
                kd.batch(prev.batch)
            ops.append(Op(kd, (prev.neurons,)))
        return ops

    def update_ops(self, prev: Layer) -> list[Op]:
        """LSTM_UpdateWeightsAdam over the reference's own NDRange ((in + H*var)/var + 1, H), raw rate."""
        total = (self.inputs + self.H * self.variables) // self.variables + 1
        k = self.kernel("LSTM_UpdateWeightsAdam").args(self.lstm_w, self.lstm_wg, self.lstm_m, self.lstm_v, LR, B1, B2)
        return [Op(k, (total, self.H))]


class FQFLayer(Layer):
    """CNeuronFQF (NeuroNet_Declarations.mqh:3490-3560, NeuroNet_AgentsRL.mqh:32-248): a fully
    parameterised quantile head over `actions` x `quantiles`.  The previous layer's weights
    ([actions*quantiles][inputs+1]) feed the fraction proposal; its softmax gives the quantile
    fractions, their cosine embedding (FQF_Cosine, then a dense LReLU layer of `inputs`) multiplies the
    state element-wise (the reference's ElementMult, i.e. the Dropout kernel), two dense layers
    (4*actions*quantiles LReLU, actions*quantiles) give the quantile values and FQF_Output their
    fraction-weighted sum per action.  `inputs` must equal the previous layer's neurons."""

    def __init__(self, ctx, actions, quantiles, inputs, optimization=ADAM, batch=1, outputs=0, activation=NONE):
        super().__init__(ctx, actions, activation, optimization, batch, outputs)
        A, Q, N = int(actions), int(quantiles), int(inputs)
        self.A, self.Q, self.N = A, Q, N
        AQ = A * Q
        self.fraction = DenseLayer(ctx, AQ, NONE, optimization, batch)
        self.softmax = SoftMaxLayer(ctx, AQ, heads=A, batch=batch)
        self.cosine = Layer(ctx, AQ, NONE, optimization, batch, outputs=N)
        self.cos_emb = DenseLayer(ctx, N, LRELU, optimization, batch)
        self.q0 = Layer(ctx, N, NONE, optimization, batch, outputs=4 * AQ)
        self.q1 = DenseLayer(ctx, 4 * AQ, LRELU, optimization, batch, outputs=AQ)
        self.q2 = DenseLayer(ctx, AQ, NONE, optimization, batch)

    def sublayers(self) -> dict:
        """The inner layers by the reference's member names (weights live on cosine, q0 and q1)."""
        return {"cFraction": self.fraction, "cSoftMax": self.softmax, "cCosine": self.cosine,
                "cCosineEmbeding": self.cos_emb, "cQuantile0": self.q0, "cQuantile1": self.q1, "cQuantile2": self.q2}

    def forward_ops(self, prev: Layer) -> list[Op]:
        """CNeuronFQF::feedForward, NeuroNet_AgentsRL.mqh:96-151."""
        if prev.neurons != self.N:
            raise ValueError(f"FQF layer built for {self.N} inputs, previous layer has {prev.neurons}")
        A, Q, N = self.A, self.Q, self.N
        ops = self.fraction.forward_ops(prev)
        ops += self.softmax.forward_ops(self.fraction)
        kc = self.kernel("FQF_Cosine").args(self.softmax.output, self.cosine.output)
        ops.append(Op(kc, (Q, A)))
        ops += self.cos_emb.forward_ops(self.cosine)
        # ElementMult (NeuroNet_Core.mqh:19163-19176): the Dropout kernel over the embedding's size
        kd = self.kernel("Dropout").args(prev.output, self.cos_emb.output, self.q0.output, N)
        ops.append(Op(kd, ((N + 3) // 4,)))
        ops += self.q1.forward_ops(self.q0)
        ops += self.q2.forward_ops(self.q1)
        ko = self.kernel("FQF_Output").args(self.q2.output, self.softmax.output, self.output, Q)
        ops.append(Op(ko, (A,)))
        return ops

    def _output_gradient_op(self) -> Op:
        k = self.kernel("FQF_OutputGradient").args(self.q2.output, self.softmax.output, self.gradient,
                                                   self.q2.gradient, self.softmax.gradient)
        return Op(k, (self.Q, self.A))

    def input_gradient_ops(self, prev: Layer) -> list[Op]:
        """CNeuronFQF::calcInputGradients, NeuroNet_AgentsRL.mqh:156-224: the state receives only the
        quantile branch's gradient (FQF_QuantileGradient); the fraction branch stops at cFraction."""
        ops = [self._output_gradient_op()]
        ops += self.q1.hidden_gradient_ops(self.q2)
        ops += self.q0.hidden_gradient_ops(self.q1)
        kq = self.kernel("FQF_QuantileGradient").args(prev.output, self.cos_emb.output, self.q0.gradient,
                                                      prev.gradient, self.cos_emb.gradient)
        ops.append(Op(kq, (self.N, 1)))
        ops += self.cosine.hidden_gradient_ops(self.cos_emb)
        kc = self.kernel("FQF_CosineGradient").args(self.softmax.output, self.cosine.gradient, self.softmax.gradient)
        ops.append(Op(kc, (self.Q, self.A)))
        ops += self.softmax.input_gradient_ops(self.fraction)
        return ops

    def update_ops(self, prev: Layer) -> list[Op]:
        """CNeuronFQF::updateInputWeights, NeuroNet_AgentsRL.mqh:230-245: the fraction proposal (the
        previous layer's weights), the cosine embedding and the two quantile layers, in that order, each
        with its own Adam step counter."""
        ops = self.fraction.update_ops(prev)
        ops += self.cos_emb.update_ops(self.cosine)
        ops += self.q1.update_ops(self.q0)
        ops += self.q2.update_ops(self.q1)
        return ops

    def soft_update_ops(self, source: "FQFLayer", tau: float, adam: bool | None = None) -> list[Op]:
        """CNeuronFQF::WeightsUpdate, NeuroNet_AgentsRL.mqh:1985-2010: its own weights, then every inner
        layer's (only cosine, q0 and q1 hold weights)."""
        ops = super().soft_update_ops(source, tau, adam)
        for name in ("cosine", "q0", "q1"):
            ops += getattr(self, name).soft_update_ops(getattr(source, name), tau, adam)
        return ops


class SoftActorCriticLayer(FQFLayer):
    """CNeuronSoftActorCritic (NeuroNet_AgentsRL.mqh:1655-1990): the FQF head whose output is an
    action sampled from each action's quantile distribution (SAC_AlphaLogProbs, with one host-drawn
    uniform per action in `random`, set_random), an entropy temperature per action from a concatenate
    layer over [cQuantile0, cQuantile2] (sigmoid), and their log-probabilities.

    One deviation: the reference's calcInputGradients ends with cSoftMax.CalcHiddenGradients(cFraction)
    (NeuroNet_AgentsRL.mqh:1981), which binds cSoftMax's weights; cSoftMax has none (created with no
    outputs), so that call fails and the fraction layer gets no gradient.  This layer ends as
    CNeuronFQF does, with the softmax gradient into cFraction."""

    def __init__(self, ctx, actions, quantiles, inputs, optimization=ADAM, batch=1, outputs=0, activation=NONE):
        super().__init__(ctx, actions, quantiles, inputs, optimization, batch, outputs, activation)
        AQ = self.A * self.Q
        self.alphas = ConcatLayer(ctx, self.A, self.N, AQ, SIGMOID, optimization, batch)
        # cAlphas reads cQuantile2's output as its second input and writes its gradient there
        ctx.free(self.alphas.second)
        ctx.free(self.alphas.second_grad)
        self.alphas.second, self.alphas.second_grad = self.q2.output, self.q2.gradient
        self.log_probs = ctx.buffer(self.A * batch)
        self.random = ctx.buffer(self.A * batch)

    def sublayers(self) -> dict:
        d = super().sublayers()
        d["cAlphas"] = self.alphas
        return d

    def set_random(self, u: np.ndarray) -> None:
        """The uniforms the host draws per action before each forward pass (MathRand()/32767)."""
        self.ctx.write(self.random, np.asarray(u, np.float32))

    def forward_ops(self, prev: Layer) -> list[Op]:
        """CNeuronSoftActorCritic::feedForward, NeuroNet_AgentsRL.mqh:1688-1725."""
        ops = super().forward_ops(prev)
        ops += self.alphas.forward_ops(self.q0)
        k = self.kernel("SAC_AlphaLogProbs").args(self.output, self.q2.output, self.softmax.output,
                                                  self.alphas.output, self.log_probs, self.random, self.Q,
                                                  self.activation)
        # FQF_Output has already written the output; SAC_AlphaLogProbs overwrites it with the sample
        ops.append(Op(k, (self.A,)))
        return ops

    def _output_gradient_op(self) -> Op:
        k = self.kernel("SAC_OutputGradient").args(self.q2.output, self.softmax.output, self.gradient,
                                                   self.q2.gradient, self.softmax.gradient, self.output, self.Q,
                                                   self.activation)
        return Op(k, (self.A,))

    def alpha_gradient_ops(self, grad_layer: Layer) -> list[Op]:
        """CNeuronSoftActorCritic::calcAlphaGradients (NeuroNet_AgentsRL.mqh:1730-1750), as CNet::
        AlphasGradient calls it with another network's last layer: SAC_AlphaGradients from that layer's
        gradient, then the concatenate layer's input gradients into cQuantile0 and cQuantile2."""
        k = self.kernel("SAC_AlphaGradients").args(self.alphas.output, grad_layer.gradient, self.log_probs,
                                                   self.alphas.gradient, SIGMOID)
        return [Op(k, (self.A,))] + self.alphas.input_gradient_ops(self.q0)

    def update_ops(self, prev: Layer) -> list[Op]:
        """CNeuronSoftActorCritic::updateInputWeights, NeuroNet_AgentsRL.mqh:1755-1762."""
        return super().update_ops(prev) + self.alphas.update_ops(self.q0)

    def soft_update_ops(self, source: "SoftActorCriticLayer", tau: float, adam: bool | None = None) -> list[Op]:
        return super().soft_update_ops(source, tau, adam) + self.alphas.soft_update_ops(source.alphas, tau, adam)
