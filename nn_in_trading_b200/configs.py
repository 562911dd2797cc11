"""The training workloads: layer specs, seeded weight initialisation and synthetic inputs.

  dense_mlp     Dense MLP 240 -> 500 tanh -> 500 sigmoid -> 3 linear, batch 1, MSE, Adam
                lr 3e-4 b1 0.9 b2 0.999, seed 42; weights uniform +-1/sqrt(fan_in);
                inputs 20 bars x 12 features N(0,1), targets U[0,1).
  mlmh_encoder  Multi-layer multi-head attention encoder (CNeuronMLMHAttentionOCL): 4 layers,
                120 bars, embed 64, 8 heads x key 32, FF 64 -> 256 (GELU) -> 64 (LReLU), the
                reference's Sum&Normalize; batch 256 independent sequences, inputs N(0,1),
                MSE against N(0,1) targets.  Weight ranges are the layer's own
                (+-1/sqrt(window+1), FF2 +-1/sqrt(4*window+1), NeuroNet_Attention.mqh:1700-1790).

Data is synthetic and seeded; no market data is involved.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from .api import ADAM, LRELU, NONE, SIGMOID, TANH, Context
from .layers import DenseLayer, MLMHAttentionLayer
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
