"""Parity of the 3xTF32 tensor-core GEMM path (tcgen05) behind the dense, convolution and LSTM kernels.

The shapes are large enough to take that path (at least 64 rows and M*N*K >= 2^20) and ragged in
every GEMM dimension (partial 128-row tiles, partial 64/128-column tiles, k not a multiple of the
32-wide stage or of the 8-wide MMA step, split-K, weight gradients computed transposed); they cover
the three operand layouts the call sites use (K-major x K-major, K-major x N-major, M-major x
N-major).  Every result is compared with
the numpy oracle at the 1e-4 parity bound.
"""
import numpy as np
import pytest

from oracle import kernels as K
from tests.golden.cases import A, Case, prepare_inputs
from tests.parity import check_close
from tests.test_kernels_gpu import PER_SAMPLE_KERNELS, batched_update_oracle, run_on_gpu

pytestmark = pytest.mark.gpu

NONE, TANH, SIGMOID, LRELU = -1, 0, 1, 2

# (units, window, window_out, batch, activation); step == window, one variable
CONV_SHAPES = [(301, 37, 131, 3, TANH), (120, 64, 200, 5, NONE), (97, 65, 768, 2, LRELU), (2000, 16, 96, 4, NONE),
               # fewer than 128 outputs, at least 128 inputs: the weight gradient runs transposed
               (240, 256, 64, 2, NONE), (150, 130, 100, 3, TANH)]


def conv_cases(units, win, wout, act):
    inputs = units * win
    nw = wout * (win + 1)
    outputs = units * wout
    tag = f"{units}-{win}-{wout}"
    return {
        "FeedForwardConv": Case(f"FeedForwardConv/{tag}", "FeedForwardConv",
                                [A(nw, "uniform", 1 / np.sqrt(win + 1)), A(inputs), A(outputs, "zeros"), inputs, win,
                                 win, wout, act], (units, wout, 1)),
        "CalcHiddenGradientConv": Case(f"CalcHiddenGradientConv/{tag}", "CalcHiddenGradientConv",
                                       [A(nw, "uniform", 1 / np.sqrt(win + 1)), A(outputs, "grad"),
                                        A(inputs, f"act:{act}"), A(inputs, "zeros"), outputs, win, win, wout, act, 0],
                                       (inputs, 1)),
        "UpdateWeightsConvAdam": Case(f"UpdateWeightsConvAdam/{tag}", "UpdateWeightsConvAdam",
                                      [A(nw, "uniform", 1 / np.sqrt(win + 1)), A(outputs, "grad"), A(inputs),
                                       A(nw, "small"), A(nw, "pos", 1e-5), inputs, 3e-4, 0.9, 0.999, win, wout, win],
                                      (nw,)),
    }


def dense_cases(n_in, n_out, act):
    loc_f = min((n_in + 3) // 4, 256)
    loc_b = min((n_out + 3) // 4, 256)
    k = 1 / np.sqrt(n_in)
    nw = n_out * (n_in + 1)
    return {
        "FeedForward": Case(f"FeedForward/{n_in}x{n_out}", "FeedForward",
                            [A(nw, "uniform", k), A(n_in), A(n_out, "zeros"), n_in, act, A(n_out, "zeros"), 0],
                            (n_out, loc_f), (1, loc_f)),
        "CalcHiddenGradient": Case(f"CalcHiddenGradient/{n_in}x{n_out}", "CalcHiddenGradient",
                                   [A(nw, "uniform", k), A(n_out, "grad"), A(n_in, f"act:{act}"), A(n_in, "zeros"),
                                    n_out, act], (n_in, loc_b), (1, loc_b)),
        "UpdateWeightsAdam": Case(f"UpdateWeightsAdam/{n_in}x{n_out}", "UpdateWeightsAdam",
                                  [A(nw, "uniform", k), A(n_out, "grad"), A(n_in), A(nw, "small"), A(nw, "pos", 1e-5),
                                   n_in, 3e-4, 0.9, 0.999], (n_out, n_in + 1)),
    }


def check_batched_per_sample(ctx, case, B, seed):
    per = PER_SAMPLE_KERNELS[case.kernel]
    samples = [prepare_inputs(case, seed + 17 * s) for s in range(B)]
    batched = []
    for i, a in enumerate(samples[0]):
        if isinstance(a, np.ndarray) and i in per:
            batched.append(np.concatenate([s[i] for s in samples]))
        else:
            batched.append(a.copy() if isinstance(a, np.ndarray) else a)
    got = run_on_gpu(ctx, case.kernel, batched, case.gsize, case.lsize, batch=B)
    ctx.finish()  # raises if a tensor-core pipeline wait expired
    for s in range(B):
        args = [samples[s][i] if i in per else (batched[i].copy() if isinstance(batched[i], np.ndarray)
                                                  else batched[i]) for i in range(len(batched))]
        K.launch(case.kernel, case.gsize, case.lsize, args)
        for i in per:
            n = samples[s][i].size
            check_close(f"{case.name} sample{s} arg{i}", got[i][s * n:(s + 1) * n], args[i])


def check_batched_update(ctx, case, B, seed):
    samples = [prepare_inputs(case, seed + 31 * s) for s in range(B)]
    shared = samples[0]
    batched = [np.concatenate([s[i] for s in samples]) if i in (1, 2) else
               (shared[i].copy() if isinstance(shared[i], np.ndarray) else shared[i]) for i in range(len(shared))]
    before = [a.copy() if isinstance(a, np.ndarray) else None for a in batched]
    got = run_on_gpu(ctx, case.kernel, batched, case.gsize, case.lsize, batch=B)
    ctx.finish()
    ref = batched_update_oracle(case, samples, shared)
    for i, r in ref.items():
        check_close(f"{case.name} arg{i}", got[i], r, before[i])


@pytest.mark.parametrize("shape", CONV_SHAPES, ids=[f"{u}-{w}-{o}-b{b}" for u, w, o, b, _ in CONV_SHAPES])
def test_conv_forward_and_input_gradient(ctx, shape):
    units, win, wout, B, act = shape
    cases = conv_cases(units, win, wout, act)
    check_batched_per_sample(ctx, cases["FeedForwardConv"], B, 1000 + units)
    check_batched_per_sample(ctx, cases["CalcHiddenGradientConv"], B, 2000 + units)


@pytest.mark.parametrize("shape", CONV_SHAPES, ids=[f"{u}-{w}-{o}-b{b}" for u, w, o, b, _ in CONV_SHAPES])
def test_conv_weight_update(ctx, shape):
    units, win, wout, B, act = shape
    check_batched_update(ctx, conv_cases(units, win, wout, act)["UpdateWeightsConvAdam"], B, 3000 + units)


@pytest.mark.parametrize("n_in,n_out,B,act", [(300, 257, 70, TANH), (64, 500, 130, SIGMOID), (500, 3, 256, NONE),
                                            (512, 1, 1024, NONE), (512, 12, 600, LRELU)])
def test_dense_batched(ctx, n_in, n_out, B, act):
    cases = dense_cases(n_in, n_out, act)
    check_batched_per_sample(ctx, cases["FeedForward"], B, 4000 + n_in)
    check_batched_per_sample(ctx, cases["CalcHiddenGradient"], B, 5000 + n_in)
    check_batched_update(ctx, cases["UpdateWeightsAdam"], B, 6000 + n_in)


@pytest.mark.parametrize("H,ins,V", [(64, 32, 300), (40, 13, 129), (128, 128, 512)])
def test_lstm_hidden_gradient(ctx, H, ins, V):
    ws = H + ins + 1
    case = Case(f"LSTM_HiddenGradient/{H}-{ins}-{V}", "LSTM_HiddenGradient",
                [A(V * 4 * H, "unit"), A(V * ins, "zeros"), A(4 * H * ws + 1, "zeros"), A(V * H), A(V * ins),
                 A(4 * H * ws, "uniform", 0.5), A(V * H), H, ins], (H, V), (1, V))
    args = prepare_inputs(case, 7000 + H)
    before = [a.copy() if isinstance(a, np.ndarray) else None for a in args]
    got = run_on_gpu(ctx, case.kernel, [a.copy() if isinstance(a, np.ndarray) else a for a in args], case.gsize,
                     case.lsize)
    ctx.finish()
    K.launch(case.kernel, case.gsize, case.lsize, args)
    for i in (1, 2):
        check_close(f"{case.name} arg{i}", got[i], args[i], before[i])


# (H, inputs, V): tensor-core GEMM (>= 64 series), more inputs than cells (the reference's input loop
# skips inputs H..H+3), the SIMT GEMM of a small product, and H not a multiple of 4 (per-gate kernel).
@pytest.mark.parametrize("H,ins,V", [(64, 64, 300), (32, 64, 600), (256, 64, 96), (256, 256, 512), (16, 32, 8),
                                    (6, 8, 5)])
def test_lstm_feed_forward(ctx, H, ins, V):
    ws = H + ins + 1
    case = Case(f"LSTM_FeedForward/{H}-{ins}-{V}", "LSTM_FeedForward",
                [A(V * ins), ins, A(4 * H * ws, "uniform", 1 / np.sqrt(H + ins)), A(V * 4 * H, "zeros"),
                 A(2 * V * H), A(V * H, "uniform", 1.0)], (H, 4, V), (1, 4, 1))
    args = prepare_inputs(case, 7100 + H + V)
    before = [a.copy() if isinstance(a, np.ndarray) else None for a in args]
    got = run_on_gpu(ctx, case.kernel, [a.copy() if isinstance(a, np.ndarray) else a for a in args], case.gsize,
                     case.lsize)
    ctx.finish()
    K.launch(case.kernel, case.gsize, case.lsize, args)
    for i in (3, 4, 5):
        check_close(f"{case.name} arg{i}", got[i], args[i], before[i])
