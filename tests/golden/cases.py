"""Kernel-level parity cases: one entry per (reference kernel, shape, activation).

Each case lists the reference kernel's positional arguments -- float32 arrays
(`A`) or scalars -- and the NDRange (`gsize`, `lsize`) the MQL5 host would
enqueue.  `make_golden.py` executes every case with the reference kernels
compiled from NeuroNet.cl (oracle/_ref) and stores inputs and outputs in
`kernels.npz`; the tests replay the same cases through the numpy oracle (CPU)
and through the CUDA library (GPU) and compare every array argument.

Shapes follow the edge rows the reference's callers produce: 1, 3, 4, 63, 64,
65 and non-multiples of 4, plus every activation.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

NONE, TANH, SIGMOID, LRELU, SOFTPLUS, GELU, MINUS_SOFTPLUS, ELU = -1, 0, 1, 2, 3, 4, 5, 6
ACTS = [NONE, TANH, SIGMOID, LRELU, SOFTPLUS, GELU, MINUS_SOFTPLUS, ELU]
MAX_LOCAL = 256  # GetMaxLocalSize(1) the golden vectors are generated with


@dataclass
class A:
    """Array argument: size and initial distribution."""
    size: int
    init: str = "normal"      # normal | uniform | zeros | small | pos | unit | act:<id> | grad
    scale: float = 1.0


@dataclass
class Case:
    name: str
    kernel: str
    args: list
    gsize: tuple
    lsize: tuple | None = None
    tol: float = 1e-4
    meta: dict = field(default_factory=dict)


def materialise(case: Case, seed: int) -> list:
    """Deterministic inputs of a case (numpy float32 arrays / python scalars)."""
    rng = np.random.default_rng(seed)
    out = []
    for a in case.args:
        if not isinstance(a, A):
            out.append(a)
            continue
        n = a.size
        if a.init == "normal":
            v = rng.standard_normal(n) * a.scale
        elif a.init == "uniform":
            v = rng.uniform(-a.scale, a.scale, n)
        elif a.init == "zeros":
            v = np.zeros(n)
        elif a.init == "small":
            v = rng.standard_normal(n) * 1e-3 * a.scale
        elif a.init == "pos":
            v = rng.uniform(0.05, 1.0, n) * a.scale
        elif a.init == "unit":
            v = rng.uniform(0.0, 1.0, n)
        elif a.init == "grad":
            v = rng.standard_normal(n) * 0.01 * a.scale
        elif a.init == "nanmix":
            # normal values with a few NaN and +-inf entries (the IsNaNOrInf paths)
            v = rng.standard_normal(n) * a.scale
            pick = rng.uniform(0.0, 1.0, n)
            v[pick < 0.02] = np.nan
            v[(pick >= 0.02) & (pick < 0.03)] = np.inf
            v[(pick >= 0.03) & (pick < 0.04)] = -np.inf
        elif a.init == "huge":
            # normal values, one in ten scaled to 1e20 (products of two of them overflow float)
            v = rng.standard_normal(n) * a.scale
            v[rng.uniform(0.0, 1.0, n) < 0.1] *= 1e20
        elif a.init == "coarse":
            # normal values on a grid of 0.5 (repeated values: the tie rules of searches and sorts)
            v = np.round(rng.standard_normal(n) * a.scale * 2.0) / 2.0
        elif a.init == "perm":
            # rows of int(scale) entries, each a permutation of its indices (as floats), a few NaN
            T = int(a.scale)
            v = np.concatenate([rng.permutation(T) for _ in range(n // T)]).astype(np.float64)
            v[rng.uniform(0.0, 1.0, n) < 0.05] = np.nan
        elif a.init == "dropmask":
            # a dropout map as CNeuronDropoutOCL draws it: 0 with probability 0.3, else 1 / 0.7
            v = np.where(rng.uniform(0.0, 1.0, n) < 0.3, 0.0, 1.0 / 0.7)
        elif a.init.startswith("act:"):
            # a plausible activation output for the given activation (used by Deactivation inputs)
            act = int(a.init[4:])
            x = rng.standard_normal(n)
            v = {TANH: np.tanh(x), SIGMOID: 1 / (1 + np.exp(-x)), LRELU: np.where(x < 0, 0.01 * x, x),
                 SOFTPLUS: np.log1p(np.exp(x)), GELU: x / (1 + np.exp(-1.702 * x)),
                 MINUS_SOFTPLUS: -np.log1p(np.exp(x)), ELU: np.where(x < 0, np.exp(x) - 1, x)}.get(act, x)
        else:
            raise ValueError(a.init)
        out.append(np.ascontiguousarray(v, dtype=np.float32))
    return out


def _dense_cases():
    cases = []
    for n_in, n_out in [(1, 1), (3, 4), (37, 11), (63, 65), (64, 64), (65, 3), (240, 17)]:
        for act in ([TANH, SIGMOID, NONE] if n_in != 37 else ACTS):
            loc = min((n_in + 3) // 4, MAX_LOCAL)
            k = 1 / np.sqrt(n_in)
            cases.append(Case(f"FeedForward/{n_in}x{n_out}/act{act}", "FeedForward",
                              [A(n_out * (n_in + 1), "uniform", k), A(n_in), A(n_out, "zeros"), n_in, act,
                               A(n_out, "zeros"), 0],
                              (n_out, loc), (1, loc)))
        loc = min((n_out + 3) // 4, MAX_LOCAL)
        for act in ([TANH, SIGMOID, NONE] if n_in != 37 else ACTS):
            cases.append(Case(f"CalcHiddenGradient/{n_in}x{n_out}/act{act}", "CalcHiddenGradient",
                              [A(n_out * (n_in + 1), "uniform", 1 / np.sqrt(n_in)), A(n_out, "grad"),
                               A(n_in, f"act:{act}"), A(n_in, "zeros"), n_out, act],
                              (n_in, loc), (1, loc)))
        cases.append(Case(f"UpdateWeightsAdam/{n_in}x{n_out}", "UpdateWeightsAdam",
                          [A(n_out * (n_in + 1), "uniform", 1 / np.sqrt(n_in)), A(n_out, "grad"), A(n_in),
                           A(n_out * (n_in + 1), "small"), A(n_out * (n_in + 1), "pos", 1e-5), n_in,
                           3e-4, 0.9, 0.999],
                          (n_out, n_in + 1)))
        cases.append(Case(f"UpdateWeightsMomentum/{n_in}x{n_out}", "UpdateWeightsMomentum",
                          [A(n_out * (n_in + 1), "uniform", 1 / np.sqrt(n_in)), A(n_out, "grad"), A(n_in),
                           A(n_out * (n_in + 1), "small"), n_in, 3e-4, 0.9],
                          (n_out, n_in + 1)))
        cases.append(Case(f"NormalizeWeights/{n_in}x{n_out}", "NormalizeWeights",
                          [A(n_out * (n_in + 1), "uniform", 0.5), n_in + 1], (n_out,)))
    for act in ACTS:
        cases.append(Case(f"CalcOutputGradient/act{act}", "CalcOutputGradient",
                          [A(67, "unit"), A(67, f"act:{act}"), A(67, "zeros"), act, 0.5], (67,)))
        cases.append(Case(f"Activation/act{act}", "Activation", [A(131, "normal", 3.0), A(131, "zeros"), act],
                          (131,)))
        cases.append(Case(f"DeActivation/act{act}", "DeActivation",
                          [A(131, f"act:{act}"), A(131, "zeros"), A(131, "grad", 50.0), act], (131,)))
    return cases


def _conv_cases():
    cases = []
    # (inputs per variable, step, window_in, window_out, variables, activation)
    shapes = [(64 * 5, 64, 64, 24, 1, NONE),      # MLMH 1x1 "conv": per-unit dense
              (24 * 5, 24, 24, 64, 1, GELU),      # MLMH W0 / FF shape
              (512, 8, 16, 12, 3, NONE),          # PatchTST patching conv, stride < window
              (47, 5, 7, 6, 2, TANH),             # overlapping windows, two variables.  Shapes keep
                                                  # (inputs-window) % step == 0: otherwise the reference's
                                                  # Adam gradient loop reads one window past the buffer
              (33, 3, 3, 5, 1, LRELU)]
    for inputs, step, win, wout, var, act in shapes:
        units = (inputs - win) // step + 1
        nw = var * wout * (win + 1)
        cases.append(Case(f"FeedForwardConv/{inputs}-{step}-{win}-{wout}-{var}", "FeedForwardConv",
                          [A(nw, "uniform", 1 / np.sqrt(win + 1)), A(inputs * var), A(units * wout * var, "zeros"),
                           inputs, step, win, wout, act],
                          (units, wout, var)))
        outputs = units * wout
        cases.append(Case(f"CalcHiddenGradientConv/{inputs}-{step}-{win}-{wout}-{var}", "CalcHiddenGradientConv",
                          [A(nw, "uniform", 1 / np.sqrt(win + 1)), A(outputs * var, "grad"),
                           A(inputs * var, f"act:{act}"), A(inputs * var, "zeros"), outputs, step, win, wout, act, 0],
                          (inputs, var)))
        cases.append(Case(f"UpdateWeightsConvAdam/{inputs}-{step}-{win}-{wout}-{var}", "UpdateWeightsConvAdam",
                          [A(nw, "uniform", 1 / np.sqrt(win + 1)), A(outputs * var, "grad"), A(inputs * var),
                           A(nw, "small"), A(nw, "pos", 1e-5), inputs, 3e-4, 0.9, 0.999, win, wout, step],
                          (nw,)))
        cases.append(Case(f"UpdateWeightsConvMomentum/{inputs}-{step}-{win}-{wout}-{var}",
                          "UpdateWeightsConvMomentum",
                          [A(nw, "uniform", 1 / np.sqrt(win + 1)), A(outputs * var, "grad"), A(inputs * var),
                           A(nw, "small"), inputs, 3e-4, 0.9, win, wout, step],
                          (nw,)))
    return cases


def _attention_cases():
    cases = []
    for units, heads, dim in [(5, 2, 4), (12, 3, 8), (17, 2, 5), (33, 4, 16), (1, 1, 3), (120, 2, 32), (200, 1, 6),
                              (63, 8, 16)]:
        n = units * 3 * heads * dim
        for mask in (0, 1):
            cases.append(Case(f"MHAttentionScore/{units}-{heads}-{dim}/m{mask}", "MHAttentionScore",
                              [A(n), A(units * heads * units, "zeros"), dim, mask], (units, heads)))
        cases.append(Case(f"MHAttentionOut/{units}-{heads}-{dim}", "MHAttentionOut",
                          [A(units * heads * units, "unit"), A(n), A(units * heads * dim, "zeros"), dim],
                          (units, heads)))
        cases.append(Case(f"MHAttentionInsideGradients/{units}-{heads}-{dim}", "MHAttentionInsideGradients",
                          [A(n), A(n, "zeros"), A(units * heads * units, "unit"), A(units * heads * dim, "grad")],
                          (units, heads, dim), meta={"softmax_scores": 1}))
    return cases


def _norm_cases():
    cases = []
    for rows, dim in [(1, 5), (3, 64), (7, 65), (4, 1), (10, 2), (5, 128)]:
        for scale in (0.5, 3.0):
            cases.append(Case(f"Normalize/{rows}x{dim}/s{scale}", "Normalize", [A(rows * dim, "normal", scale), dim],
                              (rows,)))
        cases.append(Case(f"SumMatrix/{rows}x{dim}", "SumMatrix",
                          [A(rows * dim), A(rows * dim), A(rows * dim, "zeros"), dim, 0.5, 0, 0, 0,
                           A(rows * dim, "zeros"), 1],
                          (rows,)))
    for heads, size in [(1, 3), (2, 64), (3, 65), (4, 100), (1, 1)]:
        cases.append(Case(f"SoftMax_FeedForward/{heads}x{size}", "SoftMax_FeedForward",
                          [A(heads * size, "normal", 2.0), A(heads * size, "zeros")], (size, heads), (size, 1)))
        cases.append(Case(f"SoftMax_HiddenGradient/{heads}x{size}", "SoftMax_HiddenGradient",
                          [A(heads * size, "unit"), A(heads * size, "grad"), A(heads * size, "zeros")],
                          (size, heads), (size, 1)))
        cases.append(Case(f"SoftMax_OutputGradient/{heads}x{size}", "SoftMax_OutputGradient",
                          [A(heads * size, "unit"), A(heads * size, "unit"), A(heads * size, "zeros")],
                          (heads * size,)))
    cases.append(Case("SoftUpdate/1000", "SoftUpdate", [A(1000), A(1000), 0.005], (1000,)))
    cases.append(Case("SoftUpdateAdam/1000", "SoftUpdateAdam",
                      [A(1000), A(1000), A(1000, "small"), A(1000, "pos", 1e-4), 0.005, 0.9, 0.999], (1000,)))
    for n in (1, 3, 4, 63, 64, 65):
        cases.append(Case(f"SoftUpdate/{n}", "SoftUpdate", [A(n), A(n), 0.005], (n,)))
        cases.append(Case(f"SoftUpdateAdam/{n}", "SoftUpdateAdam",
                          [A(n), A(n), A(n, "small"), A(n, "pos", 1e-4), 0.005, 0.9, 0.999], (n,)))
    # tau = 1: the target becomes the source (a hard copy)
    cases.append(Case("SoftUpdate/65-tau1", "SoftUpdate", [A(65), A(65), 1.0], (65,)))
    cases.append(Case("Transpose/7x13", "Transpose", [A(91), A(91, "zeros")], (7, 13)))
    for rows, cols in ((1, 1), (1, 65), (65, 1), (3, 4), (63, 64), (64, 65), (33, 97)):
        cases.append(Case(f"Transpose/{rows}x{cols}", "Transpose", [A(rows * cols), A(rows * cols, "zeros")],
                          (rows, cols)))
    cases.append(Case("ConcatenateBuffers/5", "ConcatenateBuffers",
                      [A(15), 3, A(20), 4, A(5), 1, A(10), 2, A(50, "zeros")], (5, 2)))
    cases.append(Case("DeconcatenateBuffers/5", "DeconcatenateBuffers",
                      [A(15, "zeros"), 3, A(20, "zeros"), 4, A(5, "zeros"), 1, A(10, "zeros"), 2, A(50)], (5, 2)))
    # (rows, windows, work-items per row); a zero window leaves its buffer untouched; NaN and inf
    # entries become 0 on the way through
    for n, ws, tw, init in ((1, (1, 0, 0, 0), 1, "normal"), (3, (3, 4, 63, 64), 4, "normal"),
                            (4, (65, 1, 0, 2), 3, "nanmix"), (2, (0, 64, 0, 1), 64, "normal"),
                            (7, (4, 4, 4, 4), 5, "nanmix")):
        tot = sum(ws)
        parts = []
        for w in ws:
            parts += [A(max(n * w, 1), init), w]
        cases.append(Case(f"ConcatenateBuffers/{n}-{'-'.join(map(str, ws))}", "ConcatenateBuffers",
                          parts + [A(n * tot, "zeros")], (n, tw)))
        parts = []
        for w in ws:
            parts += [A(max(n * w, 1), "zeros"), w]
        cases.append(Case(f"DeconcatenateBuffers/{n}-{'-'.join(map(str, ws))}", "DeconcatenateBuffers",
                          parts + [A(n * tot, init)], (n, tw)))
    for opt, width in ((0, 7), (1, 9)):
        cases.append(Case(f"RevInFeedForward/opt{opt}", "RevInFeedForward",
                          [A(96), A(12 * width, "pos"), A(96, "zeros"), 12 * width, opt], (96,)))
        cases.append(Case(f"RevInHiddenGraddient/opt{opt}", "RevInHiddenGraddient",
                          [A(96, "act:-1"), A(96, "zeros"), A(12 * width, "pos", 3.0), A(96, "grad"), 12 * width, opt,
                           NONE], (96,)))
        # options_size a whole number of option records (reads stay inside it), or 3 floats past one
        # (the kernels then read options[shift + 4] up to options_size + 3: the array holds 4 more)
        for n, size in ((1, width), (63, 5 * width), (64, 5 * width + 3), (65, 12 * width)):
            arr = size + (0 if size % width == 0 else 4)
            cases.append(Case(f"RevInFeedForward/opt{opt}/{n}-{size}", "RevInFeedForward",
                              [A(n), A(arr, "pos"), A(n, "zeros"), size, opt], (n,)))
            for act in (NONE, TANH):
                cases.append(Case(f"RevInHiddenGraddient/opt{opt}/{n}-{size}/act{act}", "RevInHiddenGraddient",
                                  [A(n, f"act:{act}"), A(n, "zeros"), A(arr, "pos", 3.0), A(n, "grad"), size, opt,
                                   act], (n,)))
    return cases


def _batchnorm_cases():
    cases = []
    for n in (1, 37, 256):
        for opt, width in ((0, 7), (1, 9)):
            for batch, training in ((1, 1), (2, 1), (50, 1), (50, 0)):
                for act in (NONE, TANH):
                    cases.append(Case(f"BatchFeedForward/{n}/opt{opt}/b{batch}/t{training}/act{act}", "BatchFeedForward",
                                      [A(n), A(n * width, "pos"), A(n, "zeros"), batch, opt, act, training], (n,)))
            for batch in (1, 50):
                cases.append(Case(f"CalcHiddenGradientBatch/{n}/opt{opt}/b{batch}", "CalcHiddenGradientBatch",
                                  [A(n * width, "pos"), A(n, "grad"), A(n), A(n, "zeros"), NONE, batch, opt], (n,)))
        cases.append(Case(f"UpdateBatchOptionsAdam/{n}", "UpdateBatchOptionsAdam",
                          [A(n * 9, "pos"), A(n, "grad"), 3e-4, 0.9, 0.999], (n,)))
        cases.append(Case(f"UpdateBatchOptionsMomentum/{n}", "UpdateBatchOptionsMomentum",
                          [A(n * 7, "pos"), A(n, "grad"), 3e-4, 0.9], (n,)))
    return cases


def _attention2_cases():
    cases = []
    for U, D in ((5, 4), (12, 8), (33, 6)):
        for mask in (0, 1):
            cases.append(Case(f"AttentionScore/{U}-{D}/m{mask}", "AttentionScore",
                              [A(U * D), A(U * D), A(U * U, "zeros"), D, mask], (U,)))
        cases.append(Case(f"AttentionOut/{U}-{D}", "AttentionOut",
                          [A(U * U, "unit"), A(U * D), A(U * D), A(U * D, "zeros")], (U, D)))
        cases.append(Case(f"AttentionInsideGradients/{U}-{D}", "AttentionInsideGradients",
                          [A(U * D), A(U * D, "zeros"), A(U * D), A(U * D, "zeros"), A(U * D), A(U * D, "zeros"),
                           A(U * U, "unit"), A(U * D, "grad", 10.0)], (U, D), meta={"softmax_rows": (U, U)}))
    # (Q, K, H, Hkv, D)
    for Qn, Kn, H, Hkv, D in ((4, 6, 2, 1, 4), (7, 7, 4, 2, 8), (5, 3, 3, 3, 5)):
        for mask in (0, 1):
            cases.append(Case(f"MH2AttentionOut/{Qn}-{Kn}-{H}-{Hkv}-{D}/m{mask}", "MH2AttentionOut",
                              [A(Qn * H * D), A(Kn * 2 * Hkv * D), A(Qn * H * Kn, "zeros"), A(Qn * H * D, "zeros"),
                               D, Hkv, mask], (Qn, Kn, H), (1, Kn, 1)))
        qpad = D * ((Qn - 1) * (H + 1) + Hkv)
        cases.append(Case(f"MH2AttentionInsideGradients/{Qn}-{Kn}-{H}-{Hkv}-{D}", "MH2AttentionInsideGradients",
                          [A(max(Qn * H * D, qpad)), A(Qn * H * D, "zeros"), A(Kn * 2 * Hkv * D),
                           A(Kn * 2 * Hkv * D, "zeros"), A(Qn * H * Kn, "unit"), A(Qn * H * D, "grad", 10.0), Kn, Hkv],
                          (Qn, D, H), meta={"softmax_rows": (Qn * H, Kn), "noise_args": {3: "mh2_key_grad"}}))
    return cases


def _lstm_cases():
    cases = []
    # (H, inputs, V, hidden weights zeroed).  The reference's forward reads h(t-1) from other work-groups
    # while they overwrite it; cases with H > 1 zero the recurrent weights so the race cannot show.
    for H, ins, V, hz in ((1, 4, 3, False), (1, 8, 2, False), (16, 8, 3, True), (6, 12, 2, True), (8, 8, 2, True)):
        ws = ins + H + 1
        cases.append(Case(f"LSTM_FeedForward/{H}-{ins}-{V}", "LSTM_FeedForward",
                          [A(V * ins), ins, A((H + 3) * ws, "uniform", 0.5), A(V * 4 * H, "zeros"),
                           A(2 * V * H, "normal", 0.5), A(V * H, "uniform", 0.9)],
                          (H, 4, V), (1, 4, 1), meta={"lstm_hidden_zero": (H, ins) if hz else None}))
    for H, V in ((16, 3), (5, 2), (1, 1), (3, 2), (4, 1), (63, 2), (64, 3), (65, 1)):
        cases.append(Case(f"LSTM_ConcatenatedGradient/{H}-{V}", "LSTM_ConcatenatedGradient",
                          [A(V * H, "grad", 10.0), A(V * 4 * H, "zeros"), A(2 * V * H), A(V * 4 * H, "unit")],
                          (H, V)))
    for H, ins, V in ((8, 8, 3), (4, 12, 2), (6, 4, 70)):
        ws = H + ins + 1
        cases.append(Case(f"LSTM_HiddenGradient/{H}-{ins}-{V}", "LSTM_HiddenGradient",
                          [A(V * 4 * H, "unit"), A(V * ins, "zeros"), A(4 * H * ws + 1, "zeros"), A(V * H),
                           A(V * ins), A(4 * H * ws, "uniform", 0.5), A(V * H), H, ins],
                          (H, V), (1, V)))
    for total, rows in ((9, 4), (17, 8), (257, 3)):
        n = total * rows
        cases.append(Case(f"LSTM_UpdateWeightsAdam/{total}x{rows}", "LSTM_UpdateWeightsAdam",
                          [A(n, "uniform", 0.3), A(n, "grad"), A(n, "small"), A(n, "pos", 1e-5), 3e-4, 0.9, 0.999],
                          (total, rows)))
    return cases


def _concat_cases():
    """Concat_* (NeuroNet.cl:3628-3862): the critic input layer of state + action."""
    cases = []
    for in1, in2, n_out in [(240, 6, 17), (3, 5, 4), (1, 1, 2), (63, 2, 9)]:
        nw = n_out * (in1 + in2 + 1)
        k = 1 / np.sqrt(in1 + in2 + 1)
        for act in (LRELU, TANH, NONE):
            cases.append(Case(f"Concat_FeedForward/{in1}+{in2}x{n_out}/act{act}", "Concat_FeedForward",
                              [A(nw, "uniform", k), A(in1), A(in2), A(n_out, "zeros"), in1, in2, act], (n_out,)))
        for a1, a2 in ((LRELU, NONE), (SIGMOID, TANH)):
            cases.append(Case(f"Concat_HiddenGradient/{in1}+{in2}x{n_out}/act{a1}-{a2}", "Concat_HiddenGradient",
                              [A(nw, "uniform", k), A(n_out, "grad"), A(in1, f"act:{a1}"), A(in2, f"act:{a2}"),
                               A(in1, "zeros"), A(in2, "zeros"), n_out, in1, in2, a1, a2], (in1 + in2,)))
        cases.append(Case(f"Concat_UpdateWeightsAdam/{in1}+{in2}x{n_out}", "Concat_UpdateWeightsAdam",
                          [A(nw, "uniform", k), A(n_out, "grad"), A(in1), A(in2), A(nw, "small"),
                           A(nw, "pos", 1e-5), in1, in2, 3e-4, 0.9, 0.999], (n_out, in1 + in2 + 1)))
        cases.append(Case(f"Concat_UpdateWeightsMomentum/{in1}+{in2}x{n_out}", "Concat_UpdateWeightsMomentum",
                          [A(nw, "uniform", k), A(n_out, "grad"), A(in1), A(in2), A(nw, "small"), in1, in2,
                           3e-4, 0.9], (n_out, in1 + in2 + 1)))
    return cases


def _adam_mini_cases():
    """UpdateWeightsAdamMini (NeuroNet.cl:7515-7612): inputs below, at and above the 64-slot local
    array, multiples of it (the bias input then drops out of the scale) and not."""
    cases = []
    for n_in, n_out in [(240, 17), (64, 9), (65, 4), (3, 5), (1, 2), (130, 7), (128, 3), (200, 6)]:
        cases.append(Case(f"UpdateWeightsAdamMini/{n_in}x{n_out}", "UpdateWeightsAdamMini",
                          [A(n_out * (n_in + 1), "uniform", 1 / np.sqrt(n_in)), A(n_out, "grad"), A(n_in),
                           A(n_out * (n_in + 1), "small"), A(n_out, "pos", 1e-5), 3e-4, 0.9, 0.999],
                          (n_in + 1, n_out), (n_in + 1, 1)))
    # UpdateWeightsConvAdamMini (NeuroNet.cl:7615-7731), one variable (several race in the reference):
    # (inputs, window, step, window_out, heads)
    for inputs, win, step, wout, heads in [(512, 16, 8, 32, 4), (120, 64, 64, 24, 3), (60, 6, 3, 8, 2),
                                           (130, 65, 65, 4, 1), (96, 128, 128, 5, 5)]:
        if win > inputs:
            continue
        total = (inputs - win + step - 1) // step
        nw = wout * (win + 1)
        cases.append(Case(f"UpdateWeightsConvAdamMini/{inputs}-{win}-{step}-{wout}-h{heads}",
                          "UpdateWeightsConvAdamMini",
                          [A(nw, "uniform", 1 / np.sqrt(win + 1)), A(total * wout, "grad"), A(inputs), A(nw, "small"),
                           A(heads, "pos", 1e-5), inputs, 3e-4, 0.9, 0.999, step],
                          (win + 1, wout, 1), (win + 1, wout // heads, 1)))
    return cases


def _matmul_cases():
    """MatMult / MatMultGrad (NeuroNet.cl:5969-6060): per-variable and shared second matrices, raw
    offsets, the ReduceNumericFlags dot product (NeuroNet_Core.mqh:18606-18636), numeric flags over
    NaN/inf operands and over products that overflow, tensor-core and split-k sizes."""
    cases = []
    # (rows, dim, cols, variables, multvarsecond, (off1, off2, offr), flags, init)
    for rows, dim, cols, var, mvs, offs, flags, init in [
            (5, 7, 3, 1, 1, (0, 0, 0), 0, "normal"), (64, 64, 64, 2, 1, (0, 0, 0), 0, "normal"),
            (130, 96, 72, 3, 0, (3, 5, 2), 0, "normal"), (1, 300, 1, 1, 0, (0, 0, 0), 0, "normal"),
            (256, 128, 96, 2, 1, (0, 0, 0), 0, "normal"), (2, 5000, 3, 1, 1, (1, 0, 4), 0, "normal"),
            (33, 20, 17, 2, 1, (0, 0, 0), 1, "nanmix"), (9, 40, 11, 2, 0, (2, 1, 0), 1, "huge"),
            (70, 33, 65, 1, 1, (0, 0, 0), 1, "normal"), (1, 0, 4, 2, 1, (1, 1, 0), 1, "normal")]:
        o1, o2, orr = offs
        n_out = var * rows * cols
        cases.append(Case(f"MatMult/{rows}x{dim}x{cols}-v{var}-m{mvs}-f{flags}-{init}", "MatMult",
                          [A(o1 + var * rows * dim, init), A(o2 + (var if mvs else 1) * dim * cols, init),
                           A(orr + n_out), dim, mvs, o1, o2, orr, A(n_out, "zeros"), flags],
                          (rows, cols, var)))
    # (rows, dim, cols, variables, multvarsecond, (off1, off1g, off2, off2g, offr), init)
    for rows, dim, cols, var, mvs, offs, init in [
            (5, 7, 3, 1, 1, (0, 0, 0, 0, 0), "normal"), (64, 48, 40, 3, 0, (1, 2, 3, 4, 5), "normal"),
            (256, 128, 96, 2, 1, (0, 0, 0, 0, 0), "normal"), (1000, 16, 8, 4, 0, (0, 0, 0, 0, 0), "normal"),
            (3, 70, 2, 2, 1, (0, 0, 0, 0, 0), "normal"), (17, 9, 33, 2, 1, (0, 0, 0, 0, 0), "nanmix")]:
        o1, o1g, o2, o2g, orr = offs
        n1, n2 = var * rows * dim, (var if mvs else 1) * dim * cols
        cases.append(Case(f"MatMultGrad/{rows}x{dim}x{cols}-v{var}-m{mvs}-{init}", "MatMultGrad",
                          [A(o1 + n1, init), A(o1g + n1, "zeros"), A(o2 + n2, init), A(o2g + n2, "zeros"),
                           A(orr + var * rows * cols, "grad" if init == "normal" else init), dim, mvs,
                           o1, o1g, o2, o2g, orr],
                          (rows, cols, var)))
    return cases


def _quantile_head_cases():
    """CNeuronFQF and the quantile SAC head (NeuroNet.cl:2524-2624, 3903-4036): fractions from a
    softmax (rows of 1, 8, 32 and 100 quants), sampled and interpolated quantiles, activations."""
    cases = []
    for T, R in [(32, 4), (8, 3), (100, 2), (1, 5), (33, 6)]:
        sm = dict(softmax_rows=(R, T))
        cases.append(Case(f"FQF_Cosine/{T}x{R}", "FQF_Cosine", [A(R * T, "unit"), A(R * T, "zeros")], (T, R),
                          meta=sm))
        cases.append(Case(f"FQF_Output/{T}x{R}", "FQF_Output", [A(R * T), A(R * T, "pos"), A(R, "zeros"), T], (R,)))
        cases.append(Case(f"FQF_OutputGradient/{T}x{R}", "FQF_OutputGradient",
                          [A(R * T), A(R * T, "pos"), A(R, "grad"), A(R * T, "zeros"), A(R * T, "zeros")], (T, R)))
        cases.append(Case(f"FQF_QuantileGradient/{T}x{R}", "FQF_QuantileGradient",
                          [A(R * T), A(R * T), A(R * T, "grad"), A(R * T, "zeros"), A(R * T, "zeros")], (T, R)))
        cases.append(Case(f"FQF_CosineGradient/{T}x{R}", "FQF_CosineGradient",
                          [A(R * T, "unit"), A(R * T, "grad"), A(R * T, "small")], (T, R), meta=sm))
        cases.append(Case(f"FQF_CosineGradientSRM/{T}x{R}", "FQF_CosineGradientSRM",
                          [A(R * T, "unit"), A(R * T, "grad"), A(R * T, "small")], (T, R), meta=sm))
        for target, init in [(0.3, "normal"), (-1.2, "nanmix"), (float("nan"), "normal"), (0.25, "coarse")]:
            cases.append(Case(f"FQF_DistributionTargetGradient/{T}x{R}-t{target}-{init}",
                              "FQF_DistributionTargetGradient",
                              [A(R * T, init), A(R * T, "unit"), A(R * T, "small"), A(R * T, "small"), target,
                               0.7, 1.3], (T, R), (T, 1), meta=sm))
    # FQF_FractionGradient (NeuroNet.cl:3207-3224): (inputs, outputs, local size along the outputs)
    for n_in, n_out, loc, init in [(32, 64, 1, "normal"), (100, 33, 16, "normal"), (7, 300, 64, "normal"),
                                   (65, 32, 1, "nanmix")]:
        cases.append(Case(f"FQF_FractionGradient/{n_in}x{n_out}-l{loc}-{init}", "FQF_FractionGradient",
                          [A(n_out * (n_in + 1), init, 0.1), A(n_out, "grad"), A(n_in, "zeros"), n_out],
                          (n_in, loc), (1, loc)))
    # FQF_MonotoneRearrange / FQF_RearrangeGradient (NeuroNet.cl:20716-20842): rows of a power of two up
    # to 64 quants (others are left untouched by the reference), NaN/inf quantiles and probabilities
    for T, R, init in [(32, 5, "normal"), (8, 3, "nanmix"), (64, 2, "normal"), (1, 4, "normal"), (2, 3, "nanmix"),
                       (12, 2, "normal"), (128, 1, "normal"), (32, 4, "coarse")]:
        cases.append(Case(f"FQF_MonotoneRearrange/{T}x{R}-{init}", "FQF_MonotoneRearrange",
                          [A(R * T, init), A(R * T, init), A(R * T, "small"), A(R * T, "small"), A(R * T, "small"),
                           A(R * 6, "small")], (T, R), (T, 1)))
        cases.append(Case(f"FQF_RearrangeGradient/{T}x{R}", "FQF_RearrangeGradient",
                          [A(R * T, "grad"), A(R * T, "grad"), A(R * T, "perm", T), A(R * T, "small"),
                           A(R * T, "small")], (T, R)))
    # FQF_SRMForward (NeuroNet.cl:2924-3021): every risk type (mean, CVaR, mean-CVaR, exponential with
    # a large and a vanishing lambda, dual power, an unknown type), rows of 1-64 quants, zero-mass rows
    for T, R, rt, par, mw, init in [(32, 4, 0, 0.0, 0.0, "unit"), (32, 4, 1, 0.25, 0.0, "unit"),
                                    (16, 3, 2, 0.1, 0.4, "unit"), (64, 2, 3, 2.5, 0.0, "unit"),
                                    (8, 5, 3, 0.0, 0.0, "unit"), (32, 3, 4, 3.0, 0.0, "unit"),
                                    (8, 2, 7, 1.0, 0.0, "unit"), (1, 3, 1, 0.5, 0.0, "unit"),
                                    (16, 2, 1, 0.3, 0.0, "zeros"), (32, 3, 2, 0.2, 0.5, "nanmix")]:
        cases.append(Case(f"FQF_SRMForward/{T}x{R}-r{rt}-p{par}-{init}", "FQF_SRMForward",
                          [A(R * T), A(R * T, init), A(R, "small"), rt, par, mw], (T, R), (T, 1)))
        cases.append(Case(f"FQF_SRMGradient/{T}x{R}-r{rt}-p{par}-{init}", "FQF_SRMGradient",
                          [A(R * T, "nanmix" if init == "nanmix" else "normal"), A(R * T, init), A(R, "grad"),
                           A(R * T, "small"), A(R * T, "small"), rt, par, mw], (T, R), (T, 1)))
    for n, cq, act in [(16, 32, NONE), (7, 8, TANH), (40, 5, SIGMOID), (3, 1, NONE), (9, 64, LRELU)]:
        cases.append(Case(f"SAC_AlphaLogProbs/{n}x{cq}-a{act}", "SAC_AlphaLogProbs",
                          [A(n, "zeros"), A(n * cq), A(n * cq, "unit"), A(n, "pos"), A(n, "zeros"), A(n, "unit"),
                           cq, act], (n,), meta=dict(softmax_rows=(n, cq))))
        cases.append(Case(f"SAC_AlphaGradients/{n}-a{act}", "SAC_AlphaGradients",
                          [A(n, f"act:{act}"), A(n, "grad"), A(n, "pos"), A(n, "zeros"), act], (n,)))
        cases.append(Case(f"SAC_OutputGradient/{n}x{cq}-a{act}", "SAC_OutputGradient",
                          [A(n * cq), A(n * cq, "pos"), A(n, "grad"), A(n * cq, "small"), A(n * cq, "small"),
                           A(n, "normal", 0.7), cq, act], (n,)))
        cases.append(Case(f"SAC_CalcLogProbs/{n}x{cq}-a{act}", "SAC_CalcLogProbs",
                          [A(n, "normal", 0.7), A(n * cq), A(n * cq, "unit"), A(n, "pos"), A(n, "zeros"), cq, act],
                          (n,), meta=dict(softmax_rows=(n, cq))))
    return cases


def _flash_cases():
    """MHFlashAttention / MHFlashAttentionGrad (NeuroNet.cl:16066-16277): self and cross attention,
    the reference's mask (keys before the query dropped), queries that see no key, head dimensions
    that are not multiples of 4, local sizes below the dimension, NaN/inf operands."""
    cases = []
    # (queries, keys, dim, heads, mask, local, init)
    for Q, KV, D, H, mask, loc, init in [(8, 8, 16, 2, 0, 16, "normal"), (10, 7, 32, 3, 1, 32, "normal"),
                                         (33, 40, 8, 1, 0, 40, "normal"), (64, 64, 64, 2, 1, 64, "normal"),
                                         (5, 70, 12, 2, 0, 70, "normal"), (6, 3, 20, 1, 0, 20, "normal"),
                                         (9, 12, 24, 2, 0, 8, "normal"), (12, 12, 16, 2, 1, 16, "nanmix")]:
        cases.append(Case(f"MHFlashAttention/{Q}x{KV}-d{D}-h{H}-m{mask}-l{loc}-{init}", "MHFlashAttention",
                          [A(Q * H * D, init), A(KV * 2 * H * D, init), A(Q * H, "zeros"), A(Q * H * D, "zeros"),
                           D, KV, mask], (Q, loc, H), (1, loc, 1)))
    for Q, KV, D, H, mask, init in [(8, 8, 16, 2, 0, "normal"), (10, 7, 32, 3, 1, "normal"),
                                    (7, 10, 32, 3, 1, "normal"), (33, 40, 8, 1, 0, "normal"),
                                    (64, 64, 64, 2, 1, "normal"), (5, 21, 12, 2, 0, "normal"),
                                    (12, 12, 16, 2, 1, "nanmix")]:
        cases.append(Case(f"MHFlashAttentionGrad/{Q}x{KV}-d{D}-h{H}-m{mask}-{init}", "MHFlashAttentionGrad",
                          [A(Q * H * D, init), A(Q * H * D, "zeros"), A(KV * 2 * H * D, init),
                           A(KV * 2 * H * D, "zeros"), A(Q * H, "pos", 4.0), A(Q * H * D, "normal", 0.5),
                           A(Q * H * D, "grad" if init == "normal" else init), D, Q, KV, mask],
                          (max(Q, KV), D, H), (1, D, 1)))
    return cases


def _patch_cases():
    """Dropout (NeuroNet.cl:1855-1884), PatchCreate / PatchHiddenGradient (NeuroNet.cl:5826-5911) and
    FQF_Sample (NeuroNet.cl:2722-2799)."""
    cases = []
    # Dropout with the host's global size (dimension + 3) / 4 (NeuroNet_Core.mqh:19168): its
    # work-items reach about twice the dimension, so the arrays are sized to hold that reach
    for D, init in [(1, "normal"), (3, "normal"), (4, "normal"), (7, "normal"), (63, "normal"), (64, "normal"),
                    (65, "normal"), (100, "nanmix"), (257, "normal")]:
        n = 2 * D + 8
        cases.append(Case(f"Dropout/{D}-{init}", "Dropout", [A(n, init), A(n, "dropmask"), A(n, "zeros"), D],
                          ((D + 3) // 4,)))
    # (time, variables, window_in, step, window_out, activation): CNeuronPatching shapes, patches
    # past the end of the series, windows wider than the step and narrower
    for T, V, win, step, WO, act in [(32, 3, 8, 4, 5, NONE), (30, 3, 8, 4, 5, TANH), (64, 1, 16, 8, 12, GELU),
                                     (17, 2, 4, 4, 3, SIGMOID), (20, 4, 3, 5, 7, LRELU), (9, 2, 9, 1, 4, NONE)]:
        P = (T - win) // step + 1 if T >= win else 1
        if act != NONE or T == 30:
            P += 1  # one patch that runs past the end of the series
        nw = V * WO * (win + 1)
        cases.append(Case(f"PatchCreate/{T}x{V}-w{win}-s{step}-o{WO}-a{act}", "PatchCreate",
                          [A(T * V), A(nw, "uniform", 1 / np.sqrt(win + 1)), A(P * V * WO, "zeros"), T * V, win,
                           step, act], (P, WO, V)))
        cases.append(Case(f"PatchHiddenGradient/{T}x{V}-w{win}-s{step}-o{WO}-a{act}", "PatchHiddenGradient",
                          [A(T * V, f"act:{act}"), A(T * V, "zeros"), A(nw, "uniform", 1 / np.sqrt(win + 1)),
                           A(P * V * WO, "grad"), win, step, WO, P, act], (T, V)))
    # FQF_Sample: rows of 1-64 quants, zero-mass rows, NaN probabilities and random values
    for T, R, pinit, rinit in [(1, 3, "unit", "unit"), (3, 5, "unit", "unit"), (8, 4, "unit", "unit"),
                               (32, 6, "unit", "unit"), (33, 3, "unit", "unit"), (48, 2, "pos", "unit"),
                               (64, 5, "unit", "unit"), (16, 3, "zeros", "unit"), (32, 6, "nanmix", "nanmix"),
                               (64, 4, "coarse", "unit")]:
        cases.append(Case(f"FQF_Sample/{T}x{R}-{pinit}-{rinit}", "FQF_Sample",
                          [A(R * T), A(R * T, pinit), A(R, rinit), A(R, "zeros")], (T, R), (T, 1)))
    return cases


def all_cases() -> list[Case]:
    return (_dense_cases() + _conv_cases() + _attention_cases() + _norm_cases() + _batchnorm_cases() + _lstm_cases()
            + _attention2_cases() + _concat_cases() + _adam_mini_cases() + _matmul_cases()
            + _quantile_head_cases() + _flash_cases() + _patch_cases())


def prepare_inputs(case: Case, seed: int) -> list:
    """Inputs of a case, with attention scores made row-stochastic where the case asks for it."""
    args = materialise(case, seed)
    rows = case.meta.get("softmax_rows")
    if rows:
        R, C = rows
        for i, a in enumerate(case.args):
            if isinstance(a, A) and a.size == R * C and a.init == "unit":
                s = args[i].reshape(R, C)
                args[i] = np.ascontiguousarray((s / s.sum(axis=1, keepdims=True)).reshape(-1), dtype=np.float32)
    hz = case.meta.get("lstm_hidden_zero")
    if hz:
        H, ins = hz
        w = args[2].reshape(H + 3, ins + H + 1)
        w[:, :H] = 0.0
    if case.meta.get("softmax_scores"):
        units, heads = case.gsize[0], case.gsize[1]
        for i, a in enumerate(case.args):
            if isinstance(a, A) and a.size == units * heads * units and a.init == "unit":
                s = args[i].reshape(units * heads, units)
                args[i] = np.ascontiguousarray((s / s.sum(axis=1, keepdims=True)).reshape(-1), dtype=np.float32)
    return args
