"""ORACLE TEST INFRASTRUCTURE -- numpy restatement of the reference's layer and network sequencing.

Restates, over the kernels of oracle/kernels.py, the kernel sequence the MQL5
host code issues for one training step: CNet::feedForward / backPropOCL
(NeuroNet_Core.mqh:13246-13417, 13555-13763), CNeuronBaseOCL
(NeuroNet_Core.mqh:15686-15984) and CNeuronMLMHAttentionOCL
(NeuroNet_Attention.mqh:1884-2405), including the per-layer Adam step counter
that advances after every update call.

Batches follow the library's batch contract: forward and input-gradient
kernels run per sample exactly as the reference kernel; every weight update
averages the per-sample weight gradient over the batch, then applies the
reference update arithmetic once.  Only tests/, __graft_entry__.smoke() and
bench.py's CPU baseline may use this module.
"""
from __future__ import annotations

import math

import numpy as np

from . import kernels as K

F32 = np.float32
LR, B1, B2 = 3.0e-4, 0.9, 0.999
MAX_LOCAL = 256


class RefBackend:
    """Kernel backend that runs the reference's own NeuroNet.cl kernels compiled for the CPU
    (oracle/_ref/libnnref.so) with the same call signature as oracle.kernels."""

    def __init__(self, path: str | None = None):
        from .ref import LIB_PATH, RefKernels
        self.ref = RefKernels(path or LIB_PATH)

    def __getattr__(self, name):
        if name not in self.ref.sig:
            raise AttributeError(name)
        if name == "Dropout":
            return self._dropout

        def call(*args, gsize, lsize=None):
            self.ref.launch(name, gsize, lsize, list(args))
        return call

    def _dropout(self, inputs, map, out, dimension, gsize, lsize=None):
        """Dropout's work-items reach about twice the dimension past its arrays
        (NeuroNet.cl:1855-1884): run the reference kernel on zero-padded copies that hold the reach
        and keep what lands inside the real arrays."""
        reach = 8 * int(gsize[0]) + 8
        pads = []
        for a in (inputs, map, out):
            p = np.zeros(max(reach, a.size), F32)
            p[:a.size] = a.reshape(-1)
            pads.append(p)
        self.ref.launch("Dropout", gsize, lsize, pads + [dimension])
        out.reshape(-1)[...] = pads[2][:out.size]


BACKEND = K  # numpy restatement by default
GRAD_HOOK = None  # optional callable G -> G applied to every batch-mean weight gradient (data-parallel mean)


def set_grad_hook(fn) -> None:
    global GRAD_HOOK
    GRAD_HOOK = fn


def use_backend(kind: str) -> None:
    """'numpy' (oracle/kernels.py) or 'reference' (oracle/_ref)."""
    global BACKEND
    BACKEND = K if kind == "numpy" else RefBackend()


def adam_lt(t: int) -> float:
    """NeuroNet_Core.mqh:15903: lr*sqrt(1-b2^t)/(1-b1^t) in double, cast to float."""
    return float(F32(LR * math.sqrt(1.0 - math.pow(B2, t)) / (1.0 - math.pow(B1, t))))


class OLayer:
    def __init__(self, neurons, activation=K.NONE, batch=1):
        self.neurons, self.activation, self.batch = neurons, activation, batch
        self.output = np.zeros((batch, neurons), F32)
        self.gradient = np.zeros((batch, neurons), F32)
        self.t = 1

    def next_lt(self) -> float:
        lt = adam_lt(self.t)
        self.t += 1
        return lt

    def calc_output_gradient(self, target):
        """CNeuronBaseOCL::calcOutputGradients, NeuroNet_Core.mqh:15800-15837."""
        for b in range(self.batch):
            BACKEND.CalcOutputGradient(target[b], self.output[b], self.gradient[b], self.activation, 1.0,
                                 gsize=(self.neurons,))


class ODense(OLayer):
    """CNeuronBaseOCL: weights toward the next dense layer, [outputs][neurons+1]."""

    def __init__(self, neurons, activation=K.NONE, batch=1, outputs=0):
        super().__init__(neurons, activation, batch)
        self.outputs = outputs
        if outputs:
            n = outputs * (neurons + 1)
            self.weights = np.zeros(n, F32)
            self.m = np.zeros(n, F32)
            self.v = np.zeros(n, F32)

    def forward(self, prev: "ODense"):
        """NeuroNet_Core.mqh:15686-15740 -> FeedForward."""
        loc = min((prev.neurons + 3) // 4, MAX_LOCAL)
        for b in range(self.batch):
            BACKEND.FeedForward(prev.weights, prev.output[b], self.output[b], prev.neurons, self.activation,
                          self.output[b], 0, gsize=(self.neurons, loc), lsize=(1, loc))

    def hidden_gradient(self, nxt: "ODense"):
        """NeuroNet_Core.mqh:15744-15769 -> CalcHiddenGradient."""
        loc = min((nxt.neurons + 3) // 4, MAX_LOCAL)
        for b in range(self.batch):
            BACKEND.CalcHiddenGradient(self.weights, nxt.gradient[b], self.output[b], self.gradient[b], nxt.neurons,
                                 self.activation, gsize=(self.neurons, loc), lsize=(1, loc))

    def update(self, prev: "ODense"):
        """NeuroNet_Core.mqh:15869-15984: UpdateWeightsAdam (batch-mean gradient) + NormalizeWeights."""
        n_out, n_col, inputs = self.neurons, prev.neurons + 1, prev.neurons
        inps = [K.nan0(np.concatenate([prev.output[b], np.ones(1, F32)])) for b in range(self.batch)]
        self.last_grad = np.mean([K.nan0(self.gradient[b][:, None] * inps[b][None, :]) for b in range(self.batch)],
                                 axis=0, dtype=np.float64).astype(F32).reshape(-1)
        # sum of |terms| of each weight's gradient: the scale of its rounding error
        self.last_grad_abs = np.mean([np.abs(K.nan0(self.gradient[b]))[:, None] * np.abs(inps[b])[None, :]
                                      for b in range(self.batch)], axis=0).reshape(-1)
        if GRAD_HOOK is not None:
            self.last_grad = GRAD_HOOK(self.last_grad)
        elif self.batch == 1:
            BACKEND.UpdateWeightsAdam(prev.weights, self.gradient[0], prev.output[0], prev.m, prev.v, inputs,
                                      self.next_lt(), B1, B2, gsize=(n_out, n_col))
            BACKEND.NormalizeWeights(prev.weights, prev.neurons + 1, gsize=(self.neurons,))
            return
        G = self.last_grad.reshape(n_out, n_col)
        K.adam_dense_apply(prev.weights, G, prev.m, prev.v, inputs, self.next_lt(), B1, B2, n_out, n_col)
        BACKEND.NormalizeWeights(prev.weights, prev.neurons + 1, gsize=(self.neurons,))


class OMLMH(OLayer):
    """CNeuronMLMHAttentionOCL (NeuroNet_Attention.mqh:1576-2405)."""

    def __init__(self, window, dk, heads, units, layers, activation=K.NONE, batch=1):
        super().__init__(window * units, activation, batch)
        self.W, self.D, self.H, self.U, self.L = window, dk, heads, units, layers
        B, out = batch, window * units
        num = 3 * dk * heads * units
        self.counts = {"qkv": 3 * (window + 1) * dk * heads, "w0": (dk + 1) * heads * window,
                       "ff1": 4 * (window + 1) * window, "ff2": (4 * window + 1) * window}
        z = lambda n: np.zeros((B, n), F32)  # noqa: E731
        self.qkv = [z(num) for _ in range(layers)]
        self.qkv_g = [z(num) for _ in range(layers)]
        self.scores = [z(units * units * heads) for _ in range(layers)]
        self.ao = [z(dk * heads * units) for _ in range(layers)]
        self.ao_g = [z(dk * heads * units) for _ in range(layers)]
        self.ff = []
        for i in range(layers):
            last = i == layers - 1
            self.ff.append([z(out), z(4 * out), self.output if last else z(out), z(out), z(4 * out),
                            self.gradient if last else z(out)])
        self.w = [{k: [np.zeros(n, F32), np.zeros(n, F32), np.zeros(n, F32)] for k, n in self.counts.items()}
                  for _ in range(layers)]
        self.last_grads = {}      # (layer, name) -> batch-mean weight gradient of the last update
        self.last_grads_abs = {}  # (layer, name) -> the same sum over |terms|

    def _conv(self, w, x, o, in_total, window, window_out, act):
        for b in range(self.batch):
            BACKEND.FeedForwardConv(w, x[b], o[b], in_total, window, window, window_out, act,
                              gsize=(o.shape[1] // window_out, window_out, 1))

    def _sum_norm(self, a, bm, out, normalize=True):
        rows = self.U
        for b in range(self.batch):
            BACKEND.SumMatrix(a[b], bm[b], out[b], self.W, 0.5, 0, 0, 0, out[b], 0, gsize=(rows,))
            if normalize:
                BACKEND.Normalize(out[b], self.W, gsize=(rows,))

    def forward(self, prev: OLayer):
        W, U, H, D = self.W, self.U, self.H, self.D
        out = W * U
        for i in range(self.L):
            inputs = prev.output if i == 0 else self.ff[i - 1][2]
            ws, t = self.w[i], self.ff[i]
            self._conv(ws["qkv"][0], inputs, self.qkv[i], out, W, 3 * D * H, K.NONE)
            for b in range(self.batch):
                BACKEND.MHAttentionScore(self.qkv[i][b], self.scores[i][b], D, 0, gsize=(U, H))
                BACKEND.MHAttentionOut(self.scores[i][b], self.qkv[i][b], self.ao[i][b], D, gsize=(U, H))
            self._conv(ws["w0"][0], self.ao[i], t[0], D * H * U, D * H, W, K.NONE)
            self._sum_norm(t[0], inputs, t[0])
            self._conv(ws["ff1"][0], t[0], t[1], out, W, 4 * W, K.GELU)
            self._conv(ws["ff2"][0], t[1], t[2], 4 * out, 4 * W, W, self.activation)
            self._sum_norm(t[2], t[0], t[2])

    def _dgrad(self, w, g, x, ig, g_total, in_total, window, window_out, act):
        for b in range(self.batch):
            BACKEND.CalcHiddenGradientConv(w, g[b], x[b], ig[b], g_total, window, window, window_out, act, 0,
                                     gsize=(in_total, 1))

    def input_gradient(self, prev: OLayer):
        W, U, H, D = self.W, self.U, self.H, self.D
        out = W * U
        out_grad = self.gradient
        for i in range(self.L - 1, -1, -1):
            t, ws = self.ff[i], self.w[i]
            self._dgrad(ws["ff2"][0], out_grad, t[1], t[4], out, 4 * out, 4 * W, W, K.NONE)
            self._dgrad(ws["ff1"][0], t[4], t[0], t[3], 4 * out, out, W, 4 * W, K.GELU)
            self._sum_norm(out_grad, t[3], t[3], normalize=False)
            out_grad = t[3]
            self._dgrad(ws["w0"][0], out_grad, self.ao[i], self.ao_g[i], out, D * H * U, D * H, W, K.NONE)
            for b in range(self.batch):
                BACKEND.MHAttentionInsideGradients(self.qkv[i][b], self.qkv_g[i][b], self.scores[i][b], self.ao_g[i][b],
                                             gsize=(U, H, D))
            if i == 0:
                inp, tmp = prev.output, prev.gradient
            else:
                inp, tmp = self.ff[i - 1][2], self.ff[i - 1][5]
            self._dgrad(ws["qkv"][0], self.qkv_g[i], inp, tmp, 3 * D * H * U, out, W, 3 * D * H, K.NONE)
            self._sum_norm(out_grad, tmp, tmp, normalize=False)
            if i > 0:
                out_grad = tmp

    def _conv_update(self, wmv, grad, inputs, in_total, window, window_out, key=None):
        w, m, v = wmv
        n = (window + 1) * window_out
        G = np.mean([K.conv_weight_grad(grad[b], inputs[b], in_total, window, window_out, window, n)
                     for b in range(self.batch)], axis=0, dtype=np.float64).astype(F32)
        if GRAD_HOOK is not None:
            G = GRAD_HOOK(G)
        self.last_grads[key] = G
        self.last_grads_abs[key] = np.mean(
            [K.conv_weight_grad(np.abs(grad[b]), np.abs(inputs[b]), in_total, window, window_out, window, n)
             for b in range(self.batch)], axis=0, dtype=np.float64)
        if self.batch == 1 and GRAD_HOOK is None:
            BACKEND.UpdateWeightsConvAdam(w, grad[0], inputs[0], m, v, in_total, self.next_lt(), B1, B2, window,
                                          window_out, window, gsize=(n,))
            BACKEND.NormalizeWeights(w, window + 1, gsize=(window_out,))
            return
        K.adam_conv_apply(w, G, m, v, self.next_lt(), B1, B2, n)
        BACKEND.NormalizeWeights(w, window + 1, gsize=(window_out,))

    def update(self, prev: OLayer):
        W, U, H, D = self.W, self.U, self.H, self.D
        out = W * U
        inputs = prev.output
        for l in range(self.L):
            t, ws = self.ff[l], self.w[l]
            self._conv_update(ws["qkv"], self.qkv_g[l], inputs, out, W, 3 * D * H, (l, "qkv"))
            self._conv_update(ws["w0"], t[3], self.ao[l], D * H * U, D * H, W, (l, "w0"))
            self._conv_update(ws["ff1"], t[4], t[0], out, W, 4 * W, (l, "ff1"))
            self._conv_update(ws["ff2"], t[5], t[1], 4 * out, 4 * W, W, (l, "ff2"))
            inputs = t[2]


class _View:
    """A layer's output/gradient seen at another batch granularity (same memory)."""

    def __init__(self, layer, batch):
        self.layer, self.batch = layer, batch
        self.output = layer.output.reshape(batch, -1)
        self.gradient = layer.gradient.reshape(batch, -1)
        self.neurons = self.output.shape[1]
        self.activation = layer.activation


def _as(layer, batch):
    return layer if layer.batch == batch else _View(layer, batch)


class ONet:
    """CNet training step over oracle layers."""

    def __init__(self, layers: list[OLayer]):
        self.layers = layers

    def forward(self, x):
        self.layers[0].output[...] = x.reshape(self.layers[0].output.shape)
        for l in range(1, len(self.layers)):
            cur = self.layers[l]
            cur.forward(_as(self.layers[l - 1], cur.batch))

    def backward(self, target):
        self.layers[-1].calc_output_gradient(target.reshape(self.layers[-1].output.shape))
        for l in range(len(self.layers) - 2, -1, -1):
            cur, nxt = self.layers[l], self.layers[l + 1]
            if type(nxt) is ODense:
                cur.hidden_gradient(nxt)
            else:
                nxt.input_gradient(_as(cur, nxt.batch))

    def update(self):
        for l in range(len(self.layers) - 1, 0, -1):
            cur = self.layers[l]
            cur.update(_as(self.layers[l - 1], cur.batch))

    def step(self, x, target):
        self.forward(x)
        self.backward(target)
        self.update()


def _fold(a, V):
    """[B][var*H] sample-major buffer viewed as the LSTM's [B*var] series."""
    return a.reshape(V, -1)


class OConv(OLayer):
    """CNeuronConvOCL (NeuroNet_Core.mqh:17132-17448): no NormalizeWeights after the update."""

    def __init__(self, window, step, window_out, units, variables=1, activation=K.NONE, batch=1, outputs=0):
        super().__init__(units * window_out * variables, activation, batch)
        self.window, self.step, self.window_out, self.units, self.variables = window, step, window_out, units, variables
        n = (window + 1) * window_out * variables
        self.conv_w, self.conv_m, self.conv_v = np.zeros(n, F32), np.zeros(n, F32), np.zeros(n, F32)
        self.outputs = outputs
        if outputs:
            self.weights = np.zeros(outputs * (self.neurons + 1), F32)
            self.m = np.zeros_like(self.weights)
            self.v = np.zeros_like(self.weights)

    def forward(self, prev):
        for b in range(self.batch):
            BACKEND.FeedForwardConv(self.conv_w, prev.output[b], self.output[b], prev.neurons // self.variables,
                                    self.step, self.window, self.window_out, self.activation,
                                    gsize=(self.units, self.window_out, self.variables))

    def input_gradient(self, prev):
        for b in range(self.batch):
            BACKEND.CalcHiddenGradientConv(self.conv_w, self.gradient[b], prev.output[b], prev.gradient[b],
                                           self.neurons // self.variables, self.step, self.window, self.window_out,
                                           prev.activation, 0, gsize=(prev.neurons // self.variables, self.variables))

    def update(self, prev):
        n = self.conv_w.size
        inputs = prev.neurons // self.variables
        G = np.mean([K.conv_weight_grad(self.gradient[b], prev.output[b], inputs, self.window, self.window_out,
                                        self.step, n) for b in range(self.batch)], axis=0, dtype=np.float64).astype(F32)
        Gabs = np.mean([K.conv_weight_grad(np.abs(self.gradient[b]), np.abs(prev.output[b]), inputs, self.window,
                                           self.window_out, self.step, n) for b in range(self.batch)], axis=0)
        if GRAD_HOOK is not None:
            G = GRAD_HOOK(G)
        self.last_grad, self.last_grad_abs = G, Gabs
        K.adam_conv_apply(self.conv_w, G, self.conv_m, self.conv_v, self.next_lt(), B1, B2, n)

    def hidden_gradient(self, nxt):
        ODense.hidden_gradient(self, nxt)


class OBatchNorm(OLayer):
    """CNeuronBatchNormOCL (NeuroNet_Core.mqh:19404-19590): samples of a batch scanned in order."""

    def __init__(self, neurons, batch_size, batch=1, optimization=K.ADAM, outputs=0):
        super().__init__(neurons, K.NONE, batch)
        self.batch_size, self.opt = batch_size, optimization
        self.width = 7 if optimization == K.SGD else 9
        self.options = np.zeros(neurons * self.width, F32)
        self.count = 1
        self.hist = None
        self.outputs = outputs
        if outputs:
            self.weights = np.zeros(outputs * (neurons + 1), F32)
            self.m = np.zeros_like(self.weights)
            self.v = np.zeros_like(self.weights)

    def forward(self, prev):
        self.count = min(self.count, self.batch_size)
        n = self.count
        self.hist = []
        for b in range(self.batch):
            BACKEND.BatchFeedForward(prev.output[b], self.options, self.output[b], n, self.opt, self.activation, 1,
                                     gsize=(self.neurons,))
            self.hist.append(self.options.reshape(self.neurons, self.width)[:, :3].copy())
        self.count += self.batch

    def input_gradient(self, prev):
        for b in range(self.batch):
            o = self.options.copy().reshape(self.neurons, self.width)
            if self.batch > 1:
                o[:, :3] = self.hist[b]
            BACKEND.CalcHiddenGradientBatch(o.reshape(-1), self.gradient[b], prev.output[b], prev.gradient[b],
                                            prev.activation, self.count, self.opt, gsize=(self.neurons,))

    def update(self, prev):
        if self.count < 100 * self.batch_size:  # NeuroNet_Core.mqh:19558
            return
        raise NotImplementedError("BatchNorm update gate never opens for batch_size > 1")

    def hidden_gradient(self, nxt):
        ODense.hidden_gradient(self, nxt)


class ORevIN(OLayer):
    """CNeuronRevINDenormOCL (NeuroNet_Core.mqh:23006-23130)."""

    def __init__(self, neurons, norm: OBatchNorm, batch=1):
        super().__init__(neurons, K.NONE, batch)
        self.norm = norm

    def forward(self, prev):
        for b in range(self.batch):
            BACKEND.RevInFeedForward(prev.output[b], self.norm.options, self.output[b], self.norm.options.size,
                                     self.norm.opt, gsize=(self.neurons,))

    def input_gradient(self, prev):
        for b in range(self.batch):
            BACKEND.RevInHiddenGraddient(prev.output[b], prev.gradient[b], self.norm.options, self.gradient[b],
                                         self.norm.options.size, self.norm.opt, prev.activation, gsize=(self.neurons,))

    def update(self, prev):
        pass


class OLSTM(OLayer):
    """CNeuronLSTMOCL (NeuroNet_RecurrentState.mqh:678-897); a batch folds into the series."""

    def __init__(self, hidden, inputs, variables=1, batch=1):
        super().__init__(hidden * variables, K.NONE, batch)
        self.H, self.inputs, self.variables = hidden, inputs, variables
        V = variables * batch
        ws = inputs + hidden + 1
        n = 4 * hidden * ws
        self.lstm_w, self.lstm_m, self.lstm_v = np.zeros(n, F32), np.zeros(n, F32), np.zeros(n, F32)
        self.lstm_wg = np.zeros(n, F32)
        self.memory = np.zeros(2 * V * hidden, F32)
        self.hidden_state = np.zeros(V * hidden, F32)
        self.cat = np.zeros(V * 4 * hidden, F32)
        self.cat_g = np.zeros(V * 4 * hidden, F32)

    def forward(self, prev):
        V = self.variables * self.batch
        out = self.output.reshape(-1)
        BACKEND.LSTM_FeedForward(prev.output.reshape(-1), self.inputs, self.lstm_w, self.cat, self.memory, out,
                                 gsize=(self.H, 4, V), lsize=(1, 4, 1))

    def input_gradient(self, prev):
        V = self.variables * self.batch
        BACKEND.LSTM_ConcatenatedGradient(self.gradient.reshape(-1), self.cat_g, self.memory, self.cat,
                                          gsize=(self.H, V))
        pg = prev.gradient.reshape(-1)
        BACKEND.LSTM_HiddenGradient(self.cat_g, pg, self.lstm_wg, self.hidden_state, prev.output.reshape(-1),
                                    self.lstm_w, self.output.reshape(-1), self.H, self.inputs, gsize=(self.H, V),
                                    lsize=(1, V))
        if prev.activation != K.NONE:
            K.DeActivation(prev.output.reshape(-1), pg, pg.copy(), prev.activation, gsize=(pg.size,))

    def update(self, prev):
        total = (self.inputs + self.H * self.variables) // self.variables + 1
        BACKEND.LSTM_UpdateWeightsAdam(self.lstm_w, self.lstm_wg, self.lstm_m, self.lstm_v, LR, B1, B2,
                                       gsize=(total, self.H))


class OConcat(ODense):
    """CNeuronConcatenate (NeuroNet_Misc.mqh:286-680): act(W [x1; x2; 1]) over its own weights
    [neurons][inputs1 + inputs2 + 1]; `second` holds x2 of every sample; no NormalizeWeights."""

    def __init__(self, neurons, inputs1, inputs2, activation=K.NONE, batch=1, outputs=0):
        super().__init__(neurons, activation, batch, outputs)
        self.in1, self.in2 = inputs1, inputs2
        n = neurons * (inputs1 + inputs2 + 1)
        self.conc_w, self.conc_m, self.conc_v = np.zeros(n, F32), np.zeros(n, F32), np.zeros(n, F32)
        self.second = np.zeros((batch, inputs2), F32)
        self.second_grad = np.zeros((batch, inputs2), F32)
        self.second_activation = K.NONE

    def forward(self, prev):
        """NeuroNet_Misc.mqh:386-418 -> Concat_FeedForward."""
        for b in range(self.batch):
            BACKEND.Concat_FeedForward(self.conc_w, prev.output[b], self.second[b], self.output[b], self.in1,
                                       self.in2, self.activation, gsize=(self.neurons,))

    def input_gradient(self, prev):
        """NeuroNet_Misc.mqh:421-462 -> Concat_HiddenGradient."""
        for b in range(self.batch):
            BACKEND.Concat_HiddenGradient(self.conc_w, self.gradient[b], prev.output[b], self.second[b],
                                          prev.gradient[b], self.second_grad[b], self.neurons, self.in1, self.in2,
                                          prev.activation, self.second_activation, gsize=(self.in1 + self.in2,))

    def update(self, prev):
        """NeuroNet_Misc.mqh:465-560 -> Concat_UpdateWeightsAdam on the batch-mean gradient."""
        n_out, n_col = self.neurons, self.in1 + self.in2 + 1
        inps = [np.concatenate([prev.output[b], self.second[b], np.ones(1, F32)]) for b in range(self.batch)]
        self.last_grad = np.mean([self.gradient[b][:, None] * inps[b][None, :] for b in range(self.batch)],
                                 axis=0, dtype=np.float64).astype(F32).reshape(-1)
        self.last_grad_abs = np.mean([np.abs(self.gradient[b])[:, None] * np.abs(inps[b])[None, :]
                                      for b in range(self.batch)], axis=0).reshape(-1)
        if GRAD_HOOK is not None:
            self.last_grad = GRAD_HOOK(self.last_grad)
        elif self.batch == 1:
            BACKEND.Concat_UpdateWeightsAdam(self.conc_w, self.gradient[0], prev.output[0], self.second[0],
                                             self.conc_m, self.conc_v, self.in1, self.in2, self.next_lt(), B1, B2,
                                             gsize=(n_out, n_col))
            return
        K.concat_adam_apply(self.conc_w, self.last_grad.reshape(n_out, n_col), self.conc_m, self.conc_v, self.in1,
                            self.in2, self.next_lt(), B1, B2, n_out, n_col)


class OFQF(OLayer):
    """CNeuronFQF (NeuroNet_AgentsRL.mqh:32-248) over the oracle kernels: fraction proposal from the
    previous layer's weights, softmax per action, cosine embedding (FQF_Cosine + dense LReLU),
    ElementMult with the state (the Dropout kernel), quantile layers 4AQ (LReLU) and AQ, FQF_Output.
    Inner layers are ODense; the weights live on cosine, q0 and q1."""

    def __init__(self, actions, quantiles, inputs, batch=1, outputs=0, activation=K.NONE):
        super().__init__(actions, activation, batch)
        A, Q, N = actions, quantiles, inputs
        self.A, self.Q, self.N, self.outputs = A, Q, N, outputs
        AQ = A * Q
        if outputs:
            n = outputs * (actions + 1)
            self.weights, self.m, self.v = np.zeros(n, F32), np.zeros(n, F32), np.zeros(n, F32)
        self.fraction = ODense(AQ, K.NONE, batch)
        self.softmax = ODense(AQ, K.NONE, batch)
        self.cosine = ODense(AQ, K.NONE, batch, outputs=N)
        self.cos_emb = ODense(N, K.LRELU, batch)
        self.q0 = ODense(N, K.NONE, batch, outputs=4 * AQ)
        self.q1 = ODense(4 * AQ, K.LRELU, batch, outputs=AQ)
        self.q2 = ODense(AQ, K.NONE, batch)

    def forward(self, prev):
        A, Q, N = self.A, self.Q, self.N
        self.fraction.forward(prev)
        for b in range(self.batch):
            BACKEND.SoftMax_FeedForward(self.fraction.output[b], self.softmax.output[b], gsize=(Q, A), lsize=(Q, 1))
            BACKEND.FQF_Cosine(self.softmax.output[b], self.cosine.output[b], gsize=(Q, A))
        self.cos_emb.forward(self.cosine)
        for b in range(self.batch):
            BACKEND.Dropout(prev.output[b], self.cos_emb.output[b], self.q0.output[b], N, gsize=((N + 3) // 4,))
        self.q1.forward(self.q0)
        self.q2.forward(self.q1)
        for b in range(self.batch):
            BACKEND.FQF_Output(self.q2.output[b], self.softmax.output[b], self.output[b], Q, gsize=(A,))

    def _output_gradient(self):
        for b in range(self.batch):
            BACKEND.FQF_OutputGradient(self.q2.output[b], self.softmax.output[b], self.gradient[b],
                                       self.q2.gradient[b], self.softmax.gradient[b], gsize=(self.Q, self.A))

    def input_gradient(self, prev):
        """CNeuronFQF::calcInputGradients, NeuroNet_AgentsRL.mqh:156-224."""
        A, Q, N = self.A, self.Q, self.N
        self._output_gradient()
        self.q1.hidden_gradient(self.q2)
        self.q0.hidden_gradient(self.q1)
        for b in range(self.batch):
            BACKEND.FQF_QuantileGradient(prev.output[b], self.cos_emb.output[b], self.q0.gradient[b],
                                         prev.gradient[b], self.cos_emb.gradient[b], gsize=(N, 1))
        self.cosine.hidden_gradient(self.cos_emb)
        for b in range(self.batch):
            BACKEND.FQF_CosineGradient(self.softmax.output[b], self.cosine.gradient[b], self.softmax.gradient[b],
                                       gsize=(Q, A))
            BACKEND.SoftMax_HiddenGradient(self.softmax.output[b], self.softmax.gradient[b],
                                           self.fraction.gradient[b], gsize=(Q, A), lsize=(Q, 1))

    def update(self, prev):
        """CNeuronFQF::updateInputWeights, NeuroNet_AgentsRL.mqh:230-245."""
        self.fraction.update(prev)
        self.cos_emb.update(self.cosine)
        self.q1.update(self.q0)
        self.q2.update(self.q1)


class OSoftActorCritic(OFQF):
    """CNeuronSoftActorCritic (NeuroNet_AgentsRL.mqh:1655-1990): the FQF head, SAC_AlphaLogProbs
    sampling with `random`, alphas from an OConcat over [q0, q2] (sigmoid).  Its input gradient ends
    as CNeuronFQF's does (the reference's last call fails for lack of weights on cSoftMax)."""

    def __init__(self, actions, quantiles, inputs, batch=1, outputs=0, activation=K.NONE):
        super().__init__(actions, quantiles, inputs, batch, outputs, activation)
        self.alphas = OConcat(actions, inputs, actions * quantiles, K.SIGMOID, batch)
        self.alphas.second = self.q2.output
        self.alphas.second_grad = self.q2.gradient
        self.log_probs = np.zeros((batch, actions), F32)
        self.random = np.zeros((batch, actions), F32)

    def forward(self, prev):
        super().forward(prev)
        self.alphas.forward(self.q0)
        for b in range(self.batch):
            BACKEND.SAC_AlphaLogProbs(self.output[b], self.q2.output[b], self.softmax.output[b],
                                      self.alphas.output[b], self.log_probs[b], self.random[b], self.Q,
                                      self.activation, gsize=(self.A,))

    def _output_gradient(self):
        for b in range(self.batch):
            BACKEND.SAC_OutputGradient(self.q2.output[b], self.softmax.output[b], self.gradient[b],
                                       self.q2.gradient[b], self.softmax.gradient[b], self.output[b], self.Q,
                                       self.activation, gsize=(self.A,))

    def alpha_gradient(self, grad_layer):
        """calcAlphaGradients, NeuroNet_AgentsRL.mqh:1730-1750."""
        for b in range(self.batch):
            BACKEND.SAC_AlphaGradients(self.alphas.output[b], grad_layer.gradient[b], self.log_probs[b],
                                       self.alphas.gradient[b], K.SIGMOID, gsize=(self.A,))
        self.alphas.input_gradient(self.q0)

    def update(self, prev):
        super().update(prev)
        self.alphas.update(self.q0)


def soft_update(target: OLayer, source: OLayer, tau: float, adam: bool) -> None:
    """CNeuronBaseOCL::WeightsUpdate (NeuroNet_Core.mqh:20283-20370) and the CNeuronConcatenate
    override (NeuroNet_Misc.mqh:628-676): SoftUpdateAdam with the target's moments, or SoftUpdate."""
    pairs = []
    if getattr(target, "outputs", 0):
        pairs.append((target.weights, source.weights, target.m, target.v))
    if isinstance(target, OConcat):
        pairs.append((target.conc_w, source.conc_w, target.conc_m, target.conc_v))
    for t, s, m, v in pairs:
        if adam:
            BACKEND.SoftUpdateAdam(t, s, m, v, tau, B1, B2, gsize=(t.size,))
        else:
            BACKEND.SoftUpdate(t, s, tau, gsize=(t.size,))


def _backward_from_output_grad(net: ONet) -> None:
    """ONet.backward without the output gradient (already in the last layer's gradient)."""
    for l in range(len(net.layers) - 2, -1, -1):
        cur, nxt = net.layers[l], net.layers[l + 1]
        if type(nxt) is ODense:
            cur.hidden_gradient(nxt)
        else:
            nxt.input_gradient(_as(cur, nxt.batch))


class OSACAgent:
    """The SAC step of nn_in_trading_b200/sac.py over oracle layers, in the same order: target value,
    critic updates, actor update against the updated critics, Polyak averaging of the targets."""

    def __init__(self, spec, batch, weights):
        S, A, H, B = spec.state, spec.action, spec.hidden, batch
        self.spec, self.B = spec, B

        def actor():
            return [ODense(S, K.NONE, B, H), ODense(H, K.LRELU, B, H), ODense(H, K.LRELU, B, 2 * A),
                    ODense(2 * A, K.NONE, B, 0)]

        def critic():
            return [ODense(S, K.NONE, B, 0), OConcat(H, S, A, K.LRELU, B, H), ODense(H, K.LRELU, B, 1),
                    ODense(1, K.NONE, B, 0)]

        self.actor = ONet(actor())
        self.actor_next = ONet(actor())
        self.critics = [ONet(critic()) for _ in range(2)]
        self.critics_pi = [ONet(critic()) for _ in range(2)]
        self.targets = [ONet(critic()) for _ in range(2)]
        for layer, w in zip(self.actor.layers[:3], weights["actor"]):
            layer.weights[:] = w
        for k in range(2):
            cw = weights["critics"][k]
            for net in (self.critics[k], self.targets[k]):
                net.layers[1].conc_w[:] = cw["conc"]
                net.layers[1].weights[:] = cw["w1"]
                net.layers[2].weights[:] = cw["w2"]
        for view, src in zip(self.actor_next.layers, self.actor.layers):
            _share(view, src)
        for k in range(2):
            for view, src in zip(self.critics_pi[k].layers, self.critics[k].layers):
                _share(view, src)
        self.y = np.zeros(B, F32)

    def step(self, batch: dict) -> None:
        sp, B, A = self.spec, self.B, self.spec.action
        s = batch["s"].reshape(B, -1)
        s2 = batch["s2"].reshape(B, -1)
        # 1. target value
        self.actor_next.forward(s2)
        self.a_next = np.zeros(B * A, F32)
        self.logp_next = np.zeros(B, F32)
        K.SACGaussianPolicy(self.actor_next.layers[-1].output.reshape(-1), batch["eps1"], self.a_next,
                            self.logp_next, A, gsize=(B,))
        for t in self.targets:
            t.layers[1].second[...] = self.a_next.reshape(B, A)
            t.forward(s2)
        K.SACTargetValue(self.targets[0].layers[-1].output.reshape(-1), self.targets[1].layers[-1].output.reshape(-1),
                         batch["r"], batch["done"], self.logp_next, self.y, sp.gamma, sp.alpha, gsize=(B,))
        # 2. critics
        for c in self.critics:
            c.layers[1].second[...] = batch["a"].reshape(B, A)
            c.forward(s)
        for c in self.critics:
            c.backward(self.y.reshape(B, 1))
        for c in self.critics:
            c.update()
        # 3. actor against the updated critics
        self.actor.forward(s)
        self.a_pi = np.zeros(B * A, F32)
        self.logp = np.zeros(B, F32)
        K.SACGaussianPolicy(self.actor.layers[-1].output.reshape(-1), batch["eps2"], self.a_pi, self.logp, A,
                            gsize=(B,))
        for c in self.critics_pi:
            c.layers[1].second[...] = self.a_pi.reshape(B, A)
            c.forward(s)
            c.layers[-1].gradient[...] = 1.0
        for c in self.critics_pi:
            _backward_from_output_grad(c)
        out = self.actor.layers[-1]
        K.SACPolicyGradient(out.output.reshape(-1), batch["eps2"], self.a_pi,
                            self.critics_pi[0].layers[-1].output.reshape(-1),
                            self.critics_pi[1].layers[-1].output.reshape(-1),
                            self.critics_pi[0].layers[1].second_grad.reshape(-1),
                            self.critics_pi[1].layers[1].second_grad.reshape(-1), out.gradient.reshape(-1), A,
                            sp.alpha, gsize=(B,))
        _backward_from_output_grad(self.actor)
        self.actor.update()
        # 4. Polyak averaging
        for k in range(2):
            for tl, cl in zip(self.targets[k].layers, self.critics[k].layers):
                soft_update(tl, cl, sp.tau, sp.soft_update_adam)


def _share(view: OLayer, src: OLayer) -> None:
    """`view` uses `src`'s parameter arrays (the same weights under a second set of activations)."""
    for name in ("weights", "m", "v", "conc_w", "conc_m", "conc_v"):
        if hasattr(src, name):
            setattr(view, name, getattr(src, name))


def quantile_head_net(spec, weights, batch=1) -> ONet:
    """The oracle twin of configs.build_quantile_head: a state layer and an FQF or SAC head."""
    AQ = spec.actions * spec.quantiles
    state = ODense(spec.inputs, K.NONE, batch, AQ)
    cls = OSoftActorCritic if spec.sac else OFQF
    head = cls(spec.actions, spec.quantiles, spec.inputs, batch)
    state.weights[:] = weights["state"]
    head.cosine.weights[:] = weights["cosine"]
    head.q0.weights[:] = weights["q0"]
    head.q1.weights[:] = weights["q1"]
    if spec.sac:
        head.alphas.conc_w[:] = weights["alphas"]
    return ONet([state, head])
