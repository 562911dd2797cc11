"""Checkpoints in the reference's .nnw file layout (CNet::Save / CNet::Load).

A network trained through this library can be written to a file that the reference's MQL5 host
loads with CNet::Load, and a file written by CNet::Save can be loaded into this library's layers.
The layout is the reference's, field for field (little-endian, as MetaTrader writes on x86):

  file      double error, double undefine, double forecast, int64 time        NeuroNet_Core.mqh:13833-13860
            array of layers                                                   NeuroNet_Core.mqh:14382-14470
  array     int64 -1 (start marker), int32 type, int32 count, count elements  (MQL5 standard library
                                                                              CArray/CArrayObj::Save; the
                                                                              marker, type and count are the
                                                                              16 bytes CBufferFloat::Load and
                                                                              CNet::Load check,
                                                                              NeuroNet_Core.mqh:15291-15310,
                                                                              14411-14433)
  buffer    an array of type defBufferDouble (0x7882) whose elements are count raw float32
            (CArrayFloat::Save under CBufferFloat::Save, NeuroNet_Core.mqh:15279-15287)
  layer     an array of type defLayer (0x7787) holding one neuron object; the object starts with its
            int32 type id, which CLayer::CreateElement reads to pick the class (NeuroNet_Core.mqh:347-420)

  CNeuronBaseOCL (NeuroNet_Core.mqh:16425-16490): int32 type, activation, optimization, batch, t,
            train; buffers Output, PrevOutput, Gradient; int32 has_weights; if 1: Weights, then
            DeltaWeights (SGD) or FirstMomentum, SecondMomentum.
  Every other class appends to that record:
  CNeuronConvOCL      int32 window, step (CNeuronProofOCL), WeightsConv, DeltaWeightsConv or the two
                      moments, int32 window_out, variables              NeuroNet_Core.mqh:17772-17798, 17928-17941
  CNeuronMLMHAttentionOCL  int32 layers, heads, window, units, window_key; collections QKV_Tensors,
                      QKV_Weights, S_Tensors, AO_Tensors, FF_Tensors, FF_Weights   NeuroNet_Attention.mqh:2411-2430
  CNeuronSoftMaxOCL   int32 heads                                        NeuroNet_Core.mqh:20148-20157
  CNeuronBatchNormOCL int32 batch size, BatchOptions                     NeuroNet_Core.mqh:19594-19603
  CNeuronRevINDenormOCL  the batch-norm record, int32 index of its normalisation layer  NeuroNet_Core.mqh:23131-23143
  CNeuronLSTMOCL      int32 inputs, variables, Weights, FirstMomentum, SecondMomentum  NeuroNet_RecurrentState.mqh:947-967
  CNeuronConcatenate  int32 second inputs, ConcWeights, ConcDeltaWeights or the two moments  NeuroNet_Misc.mqh:531-556
  CNeuronFQF          the records (type id first) of cFraction, cSoftMax, cCosine, cCosineEmbeding,
                      cQuantile0, cQuantile1, cQuantile2                 NeuroNet_AgentsRL.mqh:401-466
  CNeuronSoftActorCritic  the FQF records, then cAlphas (a CNeuronConcatenate)  NeuroNet_AgentsRL.mqh:1795-1815

The collections of the attention layer are standard-library CArrayObj arrays; their type id, 0x7778,
is the MQL5 standard library's CArrayObj::Type (CCollection does not override it), which no file of
the reference states.  Activation buffers are written for the first sample of a batch.

`capture(net)` reads a Net's state into records, `write(path, records)` writes them, `read(path)`
parses a file, `apply(net, records)` loads parameters and step counters into a Net of the same
structure, and `build(ctx, records, batch)` creates the layers a file describes.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass, field

import numpy as np

from .api import SGD

T_COLLECTION = 0x7778    # CArrayObj (MQL5 standard library)
T_LAYER = 0x7787         # defLayer, NeuroNet_Definitions.mqh:151
T_ARRAY_LAYER = 0x7788   # defArrayLayer, :153
T_BUFFER = 0x7882        # defBufferDouble, :177
T_BASE = 0x7883          # defNeuronBaseOCL, :179
T_CONV = 0x7885          # defNeuronConvOCL, :181
T_MLMH = 0x7889          # defNeuronMLMHAttentionOCL, :189
T_BATCHNORM = 0x7891     # defNeuronBatchNormOCL, :193
T_LSTM = 0x7893          # defNeuronLSTMOCL, :201
T_SOFTMAX = 0x7894       # defNeuronSoftMaxOCL, :203
T_FQF = 0x7895           # defNeuronFQF, :205
T_CONCAT = 0x7898        # defNeuronConcatenate, :210
T_SAC = 0x7899           # defNeuronSoftActorCritic, :211
T_REVIN = 0x7917         # defNeuronRevInDenormOCL, :229

F32 = np.float32
FQF_PARTS = ("fraction", "softmax", "cosine", "cos_emb", "q0", "q1", "q2")


class NNWError(ValueError):
    pass


@dataclass
class Record:
    """One neuron object of the file: its type id, the CNeuronBaseOCL fields, and the fields its
    class appends (`extra`: ints, buffers, collections or nested records, by name)."""
    type: int
    activation: int = -1
    optimization: int = 1
    batch: int = 1
    t: int = 1
    train: int = 1
    output: np.ndarray = field(default_factory=lambda: np.zeros(0, F32))
    prev_output: np.ndarray = field(default_factory=lambda: np.zeros(0, F32))
    gradient: np.ndarray = field(default_factory=lambda: np.zeros(0, F32))
    weights: np.ndarray | None = None
    delta: np.ndarray | None = None      # SGD
    m: np.ndarray | None = None          # Adam
    v: np.ndarray | None = None
    extra: dict = field(default_factory=dict)

    @property
    def neurons(self) -> int:
        return int(self.output.size)


@dataclass
class NNWFile:
    records: list
    error: float = 0.0
    undefine: float = 0.0
    forecast: float = 0.0
    time: int = 0


# ------------------------------------------------------------------------- byte level
class _Writer:
    def __init__(self):
        self.b = bytearray()

    def i32(self, v):
        self.b += struct.pack("<i", int(v))

    def i64(self, v):
        self.b += struct.pack("<q", int(v))

    def f64(self, v):
        self.b += struct.pack("<d", float(v))

    def head(self, type_id, count):
        self.i64(-1)
        self.i32(type_id)
        self.i32(count)

    def buf(self, a):
        a = np.ascontiguousarray(np.asarray(a, F32).reshape(-1))
        self.head(T_BUFFER, a.size)
        self.b += a.astype("<f4").tobytes()

    def coll(self, arrays):
        self.head(T_COLLECTION, len(arrays))
        for a in arrays:
            self.buf(a)


class _Reader:
    def __init__(self, data: bytes):
        self.d, self.p = memoryview(data), 0

    def _take(self, n):
        if self.p + n > len(self.d):
            raise NNWError(f"file ends at byte {len(self.d)}, {n} more bytes needed at {self.p}")
        out = self.d[self.p:self.p + n]
        self.p += n
        return out

    def i32(self):
        return struct.unpack("<i", self._take(4))[0]

    def i64(self):
        return struct.unpack("<q", self._take(8))[0]

    def f64(self):
        return struct.unpack("<d", self._take(8))[0]

    def head(self, type_id):
        at = self.p
        if self.i64() != -1:
            raise NNWError(f"no array start marker at byte {at}")
        t = self.i32()
        if t != type_id:
            raise NNWError(f"array type {t:#x} at byte {at}, expected {type_id:#x}")
        n = self.i32()
        if n < 0:
            raise NNWError(f"negative array length at byte {at}")
        return n

    def buf(self):
        n = self.head(T_BUFFER)
        return np.frombuffer(self._take(4 * n), dtype="<f4").astype(F32)

    def coll(self):
        return [self.buf() for _ in range(self.head(T_COLLECTION))]


# ---------------------------------------------------------------------- records
def _write_record(w: _Writer, r: Record) -> None:
    w.i32(r.type)
    _write_base(w, r)
    x = r.extra
    if r.type == T_CONV:
        w.i32(x["window"])
        w.i32(x["step"])
        w.buf(x["conv_w"])
        if r.optimization == SGD:
            w.buf(x["conv_dw"])
        else:
            w.buf(x["conv_m"])
            w.buf(x["conv_v"])
        w.i32(x["window_out"])
        w.i32(x["variables"])
    elif r.type == T_MLMH:
        for k in ("layers", "heads", "window", "units", "window_key"):
            w.i32(x[k])
        for k in ("qkv_tensors", "qkv_weights", "s_tensors", "ao_tensors", "ff_tensors", "ff_weights"):
            w.coll(x[k])
    elif r.type == T_SOFTMAX:
        w.i32(x["heads"])
    elif r.type in (T_BATCHNORM, T_REVIN):
        w.i32(x["batch_size"])
        w.buf(x["options"])
        if r.type == T_REVIN:
            w.i32(x["norm_layer"])
    elif r.type == T_LSTM:
        w.i32(x["inputs"])
        w.i32(x["variables"])
        for k in ("lstm_w", "lstm_m", "lstm_v"):
            w.buf(x[k])
    elif r.type == T_CONCAT:
        w.i32(x["inputs2"])
        w.buf(x["conc_w"])
        if r.optimization == SGD:
            w.buf(x["conc_dw"])
        else:
            w.buf(x["conc_m"])
            w.buf(x["conc_v"])
    elif r.type in (T_FQF, T_SAC):
        for k in FQF_PARTS:
            _write_record(w, x[k])
        if r.type == T_SAC:
            _write_record(w, x["alphas"])
    elif r.type != T_BASE:
        raise NNWError(f"no writer for layer type {r.type:#x}")


def _write_base(w: _Writer, r: Record) -> None:
    for v in (r.activation, r.optimization, r.batch, r.t, r.train):
        w.i32(v)
    w.buf(r.output)
    w.buf(r.prev_output)
    w.buf(r.gradient)
    if r.weights is None:
        w.i32(0)
        return
    w.i32(1)
    w.buf(r.weights)
    if r.optimization == SGD:
        w.buf(r.delta)
    else:
        w.buf(r.m)
        w.buf(r.v)


def _read_record(rd: _Reader, type_id: int) -> Record:
    r = Record(type_id, rd.i32(), rd.i32(), rd.i32(), rd.i32(), rd.i32(), rd.buf(), rd.buf(), rd.buf())
    if rd.i32() != 0:
        r.weights = rd.buf()
        if r.optimization == SGD:
            r.delta = rd.buf()
        else:
            r.m, r.v = rd.buf(), rd.buf()
    x = r.extra
    if type_id == T_CONV:
        x["window"], x["step"] = rd.i32(), rd.i32()
        x["conv_w"] = rd.buf()
        if r.optimization == SGD:
            x["conv_dw"] = rd.buf()
        else:
            x["conv_m"], x["conv_v"] = rd.buf(), rd.buf()
        x["window_out"], x["variables"] = rd.i32(), rd.i32()
    elif type_id == T_MLMH:
        for k in ("layers", "heads", "window", "units", "window_key"):
            x[k] = rd.i32()
        for k in ("qkv_tensors", "qkv_weights", "s_tensors", "ao_tensors", "ff_tensors", "ff_weights"):
            x[k] = rd.coll()
    elif type_id == T_SOFTMAX:
        x["heads"] = rd.i32()
    elif type_id in (T_BATCHNORM, T_REVIN):
        x["batch_size"] = rd.i32()
        x["options"] = rd.buf()
        if type_id == T_REVIN:
            x["norm_layer"] = rd.i32()
    elif type_id == T_LSTM:
        x["inputs"], x["variables"] = rd.i32(), rd.i32()
        for k in ("lstm_w", "lstm_m", "lstm_v"):
            x[k] = rd.buf()
    elif type_id == T_CONCAT:
        x["inputs2"] = rd.i32()
        x["conc_w"] = rd.buf()
        if r.optimization == SGD:
            x["conc_dw"] = rd.buf()
        else:
            x["conc_m"], x["conc_v"] = rd.buf(), rd.buf()
    elif type_id in (T_FQF, T_SAC):
        for k in FQF_PARTS + (("alphas",) if type_id == T_SAC else ()):
            x[k] = _read_record(rd, rd.i32())
    elif type_id != T_BASE:
        raise NNWError(f"layer type {type_id:#x} is not one this library builds")
    return r


def to_bytes(f: NNWFile) -> bytes:
    w = _Writer()
    w.f64(f.error)
    w.f64(f.undefine)
    w.f64(f.forecast)
    w.i64(f.time)
    w.head(T_ARRAY_LAYER, len(f.records))
    for r in f.records:
        w.head(T_LAYER, 1)
        _write_record(w, r)
    return bytes(w.b)


def from_bytes(data: bytes) -> NNWFile:
    rd = _Reader(data)
    f = NNWFile([], rd.f64(), rd.f64(), rd.f64(), rd.i64())
    n = rd.head(T_ARRAY_LAYER)
    for _ in range(n):
        if rd.head(T_LAYER) != 1:
            raise NNWError("a layer array holds one neuron object")
        f.records.append(_read_record(rd, rd.i32()))
    if rd.p != len(rd.d):
        raise NNWError(f"{len(rd.d) - rd.p} bytes after the last layer")
    return f


def write(path: str, f: NNWFile) -> None:
    with open(path, "wb") as fh:
        fh.write(to_bytes(f))


def read(path: str) -> NNWFile:
    with open(path, "rb") as fh:
        return from_bytes(fh.read())


# ------------------------------------------------------------ library layers <-> records
def _rd(ctx, h, n):
    return ctx.read(h, n) if n else np.zeros(0, F32)


def _base_record(ctx, layer, type_id) -> Record:
    n = layer.neurons
    r = Record(type_id, int(layer.activation), int(layer.optimization), 1, int(layer.t), 1,
               _rd(ctx, layer.output, n), np.zeros(n, F32), _rd(ctx, layer.gradient, n))
    if layer.weights is not None:
        nw = layer.outputs * (n + 1)
        r.weights = ctx.read(layer.weights, nw)
        if layer.optimization == SGD:
            r.delta = ctx.read(layer.delta, nw)
        else:
            r.m, r.v = ctx.read(layer.m, nw), ctx.read(layer.v, nw)
    return r


def layer_record(ctx, layer, layers=None) -> Record:
    """The record CNeuron*::Save would write for a library layer (`layers`: the whole net, for the
    RevIN layer's index of its normalisation layer)."""
    from . import layers as Ly
    if isinstance(layer, Ly.SoftActorCriticLayer) or isinstance(layer, Ly.FQFLayer):
        sac = isinstance(layer, Ly.SoftActorCriticLayer)
        r = _base_record(ctx, layer, T_SAC if sac else T_FQF)
        for k in FQF_PARTS:
            r.extra[k] = layer_record(ctx, getattr(layer, k))
        if sac:
            r.extra["alphas"] = layer_record(ctx, layer.alphas)
        return r
    if isinstance(layer, Ly.ConvLayer):
        r = _base_record(ctx, layer, T_CONV)
        n = (layer.window + 1) * layer.window_out * layer.variables
        r.extra.update(window=layer.window, step=layer.step, conv_w=ctx.read(layer.conv_w, n),
                       conv_m=ctx.read(layer.conv_m, n), conv_v=ctx.read(layer.conv_v, n),
                       window_out=layer.window_out, variables=layer.variables)
        return r
    if isinstance(layer, Ly.MLMHAttentionLayer):
        r = _base_record(ctx, layer, T_MLMH)
        W, D, H, U, L = layer.window, layer.dk, layer.heads, layer.units, layer.layers
        num, sc, ao = 3 * D * H * U, U * U * H, D * H * U
        qkv_t, s_t, ao_t, ff_t, qkv_w, ff_w = [], [], [], [], [], []
        counts = layer.weight_shapes()
        for i in range(L):
            qkv_t += [ctx.read(layer.qkv[i], num), ctx.read(layer.qkv_g[i], num)]
            s_t += [ctx.read(layer.scores[i], sc), np.zeros(sc, F32)]
            ao_t += [ctx.read(layer.ao[i], ao), ctx.read(layer.ao_g[i], ao)]
            sizes = [W * U, 4 * W * U, W * U] * 2
            ff_t += [ctx.read(h, s) for h, s in zip(layer.ff[i], sizes)]
            ws = layer.w[i]
            qkv_w += [ctx.read(ws["qkv"][j], counts["qkv"]) for j in range(3)]
            for j in range(3):  # weights, then first moments, then second moments of W0, FF1, FF2
                ff_w += [ctx.read(ws[k][j], counts[k]) for k in ("w0", "ff1", "ff2")]
        r.extra.update(layers=L, heads=H, window=W, units=U, window_key=D, qkv_tensors=qkv_t, qkv_weights=qkv_w,
                       s_tensors=s_t, ao_tensors=ao_t, ff_tensors=ff_t, ff_weights=ff_w)
        return r
    if isinstance(layer, Ly.SoftMaxLayer):
        r = _base_record(ctx, layer, T_SOFTMAX)
        r.extra["heads"] = layer.heads
        return r
    if isinstance(layer, Ly.RevINDenormLayer):
        r = _base_record(ctx, layer, T_REVIN)
        norm = layer.norm
        idx = next((i for i, l in enumerate(layers or []) if l is norm), -1)
        r.extra.update(batch_size=norm.batch_size, options=ctx.read(norm.options, norm.neurons * norm.width),
                       norm_layer=idx)
        return r
    if isinstance(layer, Ly.BatchNormLayer):
        r = _base_record(ctx, layer, T_BATCHNORM)
        r.extra.update(batch_size=layer.batch_size, options=ctx.read(layer.options, layer.neurons * layer.width))
        return r
    if isinstance(layer, Ly.LSTMLayer):
        r = _base_record(ctx, layer, T_LSTM)
        n = 4 * layer.H * (layer.inputs + layer.H + 1)
        r.extra.update(inputs=layer.inputs, variables=layer.variables, lstm_w=ctx.read(layer.lstm_w, n),
                       lstm_m=ctx.read(layer.lstm_m, n), lstm_v=ctx.read(layer.lstm_v, n))
        return r
    if isinstance(layer, Ly.ConcatLayer):
        r = _base_record(ctx, layer, T_CONCAT)
        n = layer.neurons * (layer.inputs1 + layer.inputs2 + 1)
        r.extra.update(inputs2=layer.inputs2, conc_w=ctx.read(layer.conc_w, n))
        if layer.optimization == SGD:
            r.extra["conc_dw"] = ctx.read(layer.conc_dw, n)
        else:
            r.extra.update(conc_m=ctx.read(layer.conc_m, n), conc_v=ctx.read(layer.conc_v, n))
        return r
    if type(layer) in (Ly.Layer, Ly.DenseLayer):
        return _base_record(ctx, layer, T_BASE)
    raise NNWError(f"{type(layer).__name__} has no .nnw record")


def capture(net, error: float = 0.0, undefine: float = 0.0, forecast: float = 0.0, time: int = 0) -> NNWFile:
    """Read every layer of `net` (device -> host) into the records CNet::Save writes."""
    ctx = net.ctx
    ctx.finish()
    return NNWFile([layer_record(ctx, l, net.layers) for l in net.layers], error, undefine, forecast, time)


def save(net, path: str, **header) -> None:
    write(path, capture(net, **header))


def _need(a, n, what):
    a = np.asarray(a, F32).reshape(-1)
    if a.size != n:
        raise NNWError(f"{what}: file holds {a.size} floats, the layer {n}")
    return a


def _apply_base(ctx, layer, r: Record, what: str):
    if r.neurons != layer.neurons:
        raise NNWError(f"{what}: {r.neurons} neurons in the file, {layer.neurons} in the layer")
    if (r.weights is None) != (layer.weights is None):
        raise NNWError(f"{what}: weights toward the next layer present in only one of file and layer")
    if int(r.activation) != int(layer.activation):
        raise NNWError(f"{what}: activation {r.activation} in the file, {layer.activation} in the layer")
    layer.t = int(r.t)
    if layer.weights is not None:
        nw = layer.outputs * (layer.neurons + 1)
        ctx.write(layer.weights, _need(r.weights, nw, what + " weights"))
        if layer.optimization == SGD:
            ctx.write(layer.delta, _need(r.delta, nw, what + " delta"))
        else:
            ctx.write(layer.m, _need(r.m, nw, what + " m"))
            ctx.write(layer.v, _need(r.v, nw, what + " v"))


def apply_record(ctx, layer, r: Record, what: str = "layer") -> None:
    """Load the parameters, optimizer state and step counter of record `r` into `layer`."""
    want = layer_record_type(layer)
    if r.type != want:
        raise NNWError(f"{what}: file has type {r.type:#x}, the layer is {want:#x}")
    _apply_base(ctx, layer, r, what)
    x = r.extra
    if r.type in (T_FQF, T_SAC):
        for k in FQF_PARTS + (("alphas",) if r.type == T_SAC else ()):
            apply_record(ctx, getattr(layer, k), x[k], f"{what}.{k}")
    elif r.type == T_CONV:
        n = (layer.window + 1) * layer.window_out * layer.variables
        for k in ("conv_w", "conv_m", "conv_v"):
            ctx.write(getattr(layer, k), _need(x[k], n, f"{what} {k}"))
    elif r.type == T_MLMH:
        counts = layer.weight_shapes()
        for i in range(layer.layers):
            ws = layer.w[i]
            for j in range(3):
                ctx.write(ws["qkv"][j], _need(x["qkv_weights"][3 * i + j], counts["qkv"], f"{what} qkv"))
                for c, k in enumerate(("w0", "ff1", "ff2")):
                    ctx.write(ws[k][j], _need(x["ff_weights"][9 * i + 3 * j + c], counts[k], f"{what} {k}"))
    elif r.type in (T_BATCHNORM, T_REVIN):
        norm = layer.norm if r.type == T_REVIN else layer
        ctx.write(norm.options, _need(x["options"], norm.neurons * norm.width, f"{what} options"))
    elif r.type == T_LSTM:
        n = 4 * layer.H * (layer.inputs + layer.H + 1)
        for k in ("lstm_w", "lstm_m", "lstm_v"):
            ctx.write(getattr(layer, k), _need(x[k], n, f"{what} {k}"))
    elif r.type == T_CONCAT:
        n = layer.neurons * (layer.inputs1 + layer.inputs2 + 1)
        keys = ("conc_w", "conc_dw") if layer.optimization == SGD else ("conc_w", "conc_m", "conc_v")
        for k in keys:
            ctx.write(getattr(layer, k), _need(x[k], n, f"{what} {k}"))


def layer_record_type(layer) -> int:
    from . import layers as Ly
    for cls, t in ((Ly.SoftActorCriticLayer, T_SAC), (Ly.FQFLayer, T_FQF), (Ly.ConvLayer, T_CONV),
                   (Ly.MLMHAttentionLayer, T_MLMH), (Ly.SoftMaxLayer, T_SOFTMAX), (Ly.RevINDenormLayer, T_REVIN),
                   (Ly.BatchNormLayer, T_BATCHNORM), (Ly.LSTMLayer, T_LSTM), (Ly.ConcatLayer, T_CONCAT)):
        if isinstance(layer, cls):
            return t
    return T_BASE


def apply(net, f: NNWFile) -> None:
    """Load a file's parameters into a Net of the same structure (CNet::Load into existing layers)."""
    if len(f.records) != len(net.layers):
        raise NNWError(f"file has {len(f.records)} layers, the net {len(net.layers)}")
    for i, (layer, r) in enumerate(zip(net.layers, f.records)):
        apply_record(net.ctx, layer, r, f"layer {i}")


def load(net, path: str) -> NNWFile:
    f = read(path)
    apply(net, f)
    return f


def _outputs(r: Record) -> int:
    return 0 if r.weights is None else r.weights.size // (r.neurons + 1)


def build_layer(ctx, r: Record, batch: int, built: list):
    """The library layer a record describes (`built`: the layers before it, for RevIN)."""
    from . import layers as Ly
    x, n, outs, opt, act = r.extra, r.neurons, _outputs(r), r.optimization, r.activation
    if r.type == T_BASE:
        layer = Ly.DenseLayer(ctx, n, act, opt, batch, outs)
    elif r.type == T_CONV:
        units = n // (x["window_out"] * x["variables"])
        layer = Ly.ConvLayer(ctx, x["window"], x["step"], x["window_out"], units, x["variables"], act, opt, batch, outs)
    elif r.type == T_MLMH:
        layer = Ly.MLMHAttentionLayer(ctx, x["window"], x["window_key"], x["heads"], x["units"], x["layers"], act, opt,
                                      batch, outs)
    elif r.type == T_SOFTMAX:
        layer = Ly.SoftMaxLayer(ctx, n, x["heads"], batch, outs)
    elif r.type == T_BATCHNORM:
        layer = Ly.BatchNormLayer(ctx, n, x["batch_size"], opt, batch, outs)
    elif r.type == T_REVIN:
        k = x["norm_layer"]
        if not (0 <= k < len(built)) or not isinstance(built[k], Ly.BatchNormLayer):
            raise NNWError(f"RevIN layer refers to layer {k}, which is not a batch-norm layer")
        layer = Ly.RevINDenormLayer(ctx, n, built[k], batch, outs)
    elif r.type == T_LSTM:
        layer = Ly.LSTMLayer(ctx, n // x["variables"], x["inputs"], x["variables"], opt, batch, outs)
    elif r.type == T_CONCAT:
        in2 = x["inputs2"]
        in1 = x["conc_w"].size // n - in2 - 1
        layer = Ly.ConcatLayer(ctx, n, in1, in2, act, opt, batch, outs)
    elif r.type in (T_FQF, T_SAC):
        aq = x["fraction"].neurons
        cls = Ly.SoftActorCriticLayer if r.type == T_SAC else Ly.FQFLayer
        layer = cls(ctx, n, aq // n, x["cos_emb"].neurons, opt, batch, outs, act)
    else:
        raise NNWError(f"layer type {r.type:#x} is not one this library builds")
    apply_record(ctx, layer, r)
    return layer


def build(ctx, f: NNWFile, batch: int = 1, **net_kwargs):
    """Create the network a file describes, with its parameters loaded."""
    from .net import Net
    layers = []
    for r in f.records:
        layers.append(build_layer(ctx, r, batch, layers))
    return Net(ctx, layers, **net_kwargs)
