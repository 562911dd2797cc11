"""The training workloads: layer specs, seeded weight initialisation and synthetic inputs.

  dense_mlp     Dense MLP 240 -> 500 tanh -> 500 sigmoid -> 3 linear, batch 1, MSE, Adam
                lr 3e-4 b1 0.9 b2 0.999, seed 42; weights uniform +-1/sqrt(fan_in);
                inputs 20 bars x 12 features N(0,1), targets U[0,1).
  mlmh_encoder  Multi-layer multi-head attention encoder (CNeuronMLMHAttentionOCL): 4 layers,
                120 bars, embed 64, 8 heads x key 32, FF 64 -> 256 (GELU) -> 64 (LReLU), the
                reference's Sum&Normalize; batch 256 independent sequences, inputs N(0,1),
                MSE against N(0,1) targets.  Weight ranges are the layer's own
                (+-1/sqrt(window+1), FF2 +-1/sqrt(4*window+1), NeuroNet_Attention.mqh:1700-1790).

  lstm_stack    2 stacked CNeuronLSTMOCL layers (input 64, hidden 256) over 1024 independent
                series (the layer's `variables`), one time step per training step (the reference
                trains recurrent layers bar by bar, h(t-1) enters as an input); a per-series 1x1
                conv head 256 -> 64 predicts the next step's 64 log-returns (MSE).  Inputs are
                N(0, 0.01) log-returns cumulated along the window.
  quantile_head A state layer feeding a CNeuronFQF or CNeuronSoftActorCritic quantile head
                (actions x quantiles), MSE of the head's output against N(0,1) targets.
  patchtst      RevIN-style: BatchNorm over 32 channels x 512 bars, Conv1D patching (window 16,
                step 8, 63 patches, embed 128, per-channel weights), 3 attention layers over the
                63 patches of every channel (8 heads x key 16, FF 512), a shared conv head
                63*128 -> 96 per channel, RevIN de-normalisation, MSE vs N(0,1) targets.

Data is synthetic and seeded; no market data is involved.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from .api import ADAM, LRELU, NONE, SIGMOID, TANH, Context
from .layers import BatchNormLayer, ConvLayer, DenseLayer, LSTMLayer, MLMHAttentionLayer, RevINDenormLayer
from .net import Net

F32 = np.float32


@dataclass
class DenseSpec:
    sizes: tuple = (240, 500, 500, 3)
    acts: tuple = (NONE, TANH, SIGMOID, NONE)
    seed: int = 42


@dataclass
class MLMHSpec:
    window: int = 64
    dk: int = 32
    heads: int = 8
    units: int = 120
    layers: int = 4
    activation: int = LRELU
    seed: int = 2


def dense_weights(spec: DenseSpec) -> list[np.ndarray]:
    """Uniform +-1/sqrt(fan_in) for weights and bias of every dense connection."""
    rng = np.random.default_rng(spec.seed)
    out = []
    for n_in, n_out in zip(spec.sizes[:-1], spec.sizes[1:]):
        k = 1.0 / np.sqrt(n_in)
        out.append(rng.uniform(-k, k, n_out * (n_in + 1)).astype(F32))
    return out


def dense_data(spec: DenseSpec, steps: int, batch: int = 1, seed: int | None = None):
    rng = np.random.default_rng(spec.seed + 1 if seed is None else seed)
    x = rng.standard_normal((steps, batch, spec.sizes[0])).astype(F32)
    t = rng.uniform(0.0, 1.0, (steps, batch, spec.sizes[-1])).astype(F32)
    return x, t


def build_dense(ctx: Context, spec: DenseSpec, batch: int = 1, weights=None, dp: bool = False) -> Net:
    layers = []
    for i, (n, a) in enumerate(zip(spec.sizes, spec.acts)):
        outputs = spec.sizes[i + 1] if i + 1 < len(spec.sizes) else 0
        layers.append(DenseLayer(ctx, n, a, ADAM, batch, outputs))
    for layer, w in zip(layers, weights if weights is not None else dense_weights(spec)):
        layer.set_weights(w)
    return Net(ctx, layers, dp=dp)


def mlmh_weights(spec: MLMHSpec) -> list[dict]:
    rng = np.random.default_rng(spec.seed)
    W, D, H = spec.window, spec.dk, spec.heads
    k = 1.0 / np.sqrt(W + 1)
    k2 = 1.0 / np.sqrt(4 * W + 1)
    counts = {"qkv": 3 * (W + 1) * D * H, "w0": (D + 1) * H * W, "ff1": 4 * (W + 1) * W, "ff2": (4 * W + 1) * W}
    out = []
    for _ in range(spec.layers):
        out.append({name: rng.uniform(-(k2 if name == "ff2" else k), (k2 if name == "ff2" else k), n).astype(F32)
                    for name, n in counts.items()})
    return out


def mlmh_data(spec: MLMHSpec, batch: int, steps: int = 1, seed: int | None = None):
    rng = np.random.default_rng(spec.seed + 1 if seed is None else seed)
    n = spec.window * spec.units
    x = rng.standard_normal((steps, batch, n)).astype(F32)
    t = rng.standard_normal((steps, batch, n)).astype(F32)
    return x, t


def build_mlmh(ctx: Context, spec: MLMHSpec, batch: int, weights=None, dp: bool = False) -> Net:
    inp = DenseLayer(ctx, spec.window * spec.units, NONE, ADAM, batch, 0)
    enc = MLMHAttentionLayer(ctx, spec.window, spec.dk, spec.heads, spec.units, spec.layers, spec.activation, ADAM,
                             batch)
    for i, ws in enumerate(weights if weights is not None else mlmh_weights(spec)):
        for name, w in ws.items():
            enc.set_weights(i, name, w)
    return Net(ctx, [inp, enc], dp=dp)


# ------------------------------------------------------------------ LSTM stack
@dataclass
class LSTMSpec:
    inputs: int = 64
    hidden: int = 256
    layers: int = 2
    series: int = 1024
    seq: int = 240
    seed: int = 3


def lstm_weights(spec: LSTMSpec) -> dict:
    """Uniform +-1/sqrt(fan_in) for the gate matrices and the head."""
    rng = np.random.default_rng(spec.seed)
    out = {}
    ins = spec.inputs
    for l in range(spec.layers):
        ws = ins + spec.hidden + 1
        k = 1.0 / np.sqrt(ins + spec.hidden)
        out[f"lstm{l}"] = rng.uniform(-k, k, 4 * spec.hidden * ws).astype(F32)
        ins = spec.hidden
    k = 1.0 / np.sqrt(spec.hidden)
    out["head"] = rng.uniform(-k, k, spec.inputs * (spec.hidden + 1)).astype(F32)
    return out


def lstm_data(spec: LSTMSpec, steps: int | None = None, seed: int | None = None):
    """[steps+1][series][inputs] cumulated N(0, 0.01) log-returns; step t trains x_t -> x_{t+1}."""
    rng = np.random.default_rng(spec.seed + 1 if seed is None else seed)
    T = (spec.seq if steps is None else steps) + 1
    r = rng.normal(0.0, 0.01, (T, spec.series, spec.inputs))
    return np.cumsum(r, axis=0).astype(F32)


def build_lstm(ctx: Context, spec: LSTMSpec, weights=None, dp: bool = False) -> Net:
    w = weights if weights is not None else lstm_weights(spec)
    V = spec.series
    layers = [DenseLayer(ctx, spec.inputs * V, NONE, ADAM, 1, 0)]
    ins = spec.inputs
    for l in range(spec.layers):
        L = LSTMLayer(ctx, spec.hidden, ins, V, ADAM, 1)
        L.set_lstm_weights(w[f"lstm{l}"])
        layers.append(L)
        ins = spec.hidden
    head = ConvLayer(ctx, spec.hidden, spec.hidden, spec.inputs, V, 1, NONE, ADAM, 1)
    head.set_conv_weights(w["head"])
    layers.append(head)
    return Net(ctx, layers, dp=dp)


# ------------------------------------------------------------ PatchTST-style
@dataclass
class PatchSpec:
    channels: int = 32
    bars: int = 512
    patch: int = 16
    stride: int = 8
    embed: int = 128
    heads: int = 8
    dk: int = 16
    layers: int = 3
    horizon: int = 96
    norm_batch: int = 1000
    seed: int = 4

    @property
    def patches(self) -> int:
        return (self.bars - self.patch) // self.stride + 1


def patch_weights(spec: PatchSpec) -> dict:
    rng = np.random.default_rng(spec.seed)
    out = {}
    k = 1.0 / np.sqrt(spec.patch + 1)
    out["conv"] = rng.uniform(-k, k, (spec.patch + 1) * spec.embed * spec.channels).astype(F32)
    enc = mlmh_weights(MLMHSpec(window=spec.embed, dk=spec.dk, heads=spec.heads, units=spec.patches,
                                layers=spec.layers, seed=spec.seed + 7))
    out["encoder"] = enc
    fan = spec.patches * spec.embed
    k = 1.0 / np.sqrt(fan + 1)
    out["head"] = rng.uniform(-k, k, spec.horizon * (fan + 1)).astype(F32)
    return out


def patch_data(spec: PatchSpec, batch: int, steps: int = 1, seed: int | None = None):
    rng = np.random.default_rng(spec.seed + 1 if seed is None else seed)
    x = rng.standard_normal((steps, batch, spec.channels * spec.bars)).astype(F32)
    t = rng.standard_normal((steps, batch, spec.channels * spec.horizon)).astype(F32)
    return x, t


def build_patch(ctx: Context, spec: PatchSpec, batch: int, weights=None, dp: bool = False) -> Net:
    w = weights if weights is not None else patch_weights(spec)
    C, P, E = spec.channels, spec.patches, spec.embed
    inp = DenseLayer(ctx, C * spec.bars, NONE, ADAM, batch, 0)
    norm = BatchNormLayer(ctx, C * spec.bars, spec.norm_batch, ADAM, batch)
    conv = ConvLayer(ctx, spec.patch, spec.stride, E, P, C, NONE, ADAM, batch)
    conv.set_conv_weights(w["conv"])
    # the conv output [C][P][E] of every sample is C independent sequences of P patches
    enc = MLMHAttentionLayer(ctx, E, spec.dk, spec.heads, P, spec.layers, NONE, ADAM, batch * C)
    for i, ws in enumerate(w["encoder"]):
        for name, arr in ws.items():
            enc.set_weights(i, name, arr)
    head = ConvLayer(ctx, P * E, P * E, spec.horizon, C, 1, NONE, ADAM, batch)
    head.set_conv_weights(w["head"])
    denorm = RevINDenormLayer(ctx, C * spec.horizon, norm, batch)
    return Net(ctx, [inp, norm, conv, enc, head, denorm], dp=dp)


# ------------------------------------------------------------------ quantile heads
@dataclass
class QuantileHeadSpec:
    """A state layer of `inputs` neurons feeding a CNeuronFQF (sac=False) or CNeuronSoftActorCritic
    (sac=True) head of `actions` x `quantiles`, the shape the reference's distributional agents use."""
    inputs: int = 256
    actions: int = 6
    quantiles: int = 32
    sac: bool = False
    seed: int = 6


def quantile_head_weights(spec: QuantileHeadSpec) -> dict:
    """Uniform +-1/sqrt(fan_in + 1) for every weight matrix of the head (state layer toward the
    fraction proposal, cosine embedding, both quantile layers, and the SAC head's alphas)."""
    rng = np.random.default_rng(spec.seed)
    A, Q, N = spec.actions, spec.quantiles, spec.inputs
    AQ = A * Q

    def u(n_out, n_in):
        k = 1.0 / np.sqrt(n_in + 1)
        return rng.uniform(-k, k, n_out * (n_in + 1)).astype(F32)
    w = {"state": u(AQ, N), "cosine": u(N, AQ), "q0": u(4 * AQ, N), "q1": u(AQ, 4 * AQ)}
    if spec.sac:
        w["alphas"] = u(A, N + AQ)
    return w


def quantile_head_data(spec: QuantileHeadSpec, steps: int, batch: int = 1, seed: int | None = None):
    """States N(0,1), targets N(0,1) per action, and the per-action uniforms of the SAC head."""
    rng = np.random.default_rng(spec.seed + 1 if seed is None else seed)
    x = rng.standard_normal((steps, batch, spec.inputs)).astype(F32)
    t = rng.standard_normal((steps, batch, spec.actions)).astype(F32)
    u = rng.uniform(0.0, 1.0, (steps, batch, spec.actions)).astype(F32)
    return x, t, u


def build_quantile_head(ctx: Context, spec: QuantileHeadSpec, batch: int = 1, weights=None) -> Net:
    from .layers import FQFLayer, SoftActorCriticLayer
    w = weights if weights is not None else quantile_head_weights(spec)
    AQ = spec.actions * spec.quantiles
    state = DenseLayer(ctx, spec.inputs, NONE, ADAM, batch, AQ)
    cls = SoftActorCriticLayer if spec.sac else FQFLayer
    head = cls(ctx, spec.actions, spec.quantiles, spec.inputs, ADAM, batch)
    state.set_weights(w["state"])
    head.cosine.set_weights(w["cosine"])
    head.q0.set_weights(w["q0"])
    head.q1.set_weights(w["q1"])
    if spec.sac:
        head.alphas.set_conc_weights(w["alphas"])
    return Net(ctx, [state, head])
