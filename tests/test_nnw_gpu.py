"""Checkpoints of trained networks through the .nnw layout: a network trained a few steps through the
C ABI is saved, rebuilt from the file (or loaded into a freshly initialised twin), and the copy holds
the same parameters, optimizer moments and step counters and takes the same next step."""
import numpy as np
import pytest

from nn_in_trading_b200 import configs as C
from nn_in_trading_b200 import nnw

pytestmark = pytest.mark.gpu


PARAM_KEYS = ("conv_w", "conv_dw", "conv_m", "conv_v", "lstm_w", "lstm_m", "lstm_v", "conc_w", "conc_dw", "conc_m",
              "conc_v", "options", "qkv_weights", "ff_weights")


def _params(ctx, net):
    """(label, array) of every parameter, optimizer buffer and step counter of a net."""
    out = []

    def walk(r, label):
        out.append((f"{label} t", np.array([r.t])))
        for k in ("weights", "delta", "m", "v"):
            if getattr(r, k) is not None:
                out.append((f"{label} {k}", getattr(r, k)))
        for k, x in sorted(r.extra.items()):
            if isinstance(x, nnw.Record):
                walk(x, f"{label}.{k}")
            elif k in PARAM_KEYS:
                out.extend([(f"{label} {k}[{i}]", a) for i, a in enumerate(x)] if isinstance(x, list)
                           else [(f"{label} {k}", x)])
    for i, r in enumerate(nnw.capture(net).records):
        walk(r, f"layer{i}")
    return out


def _same_params(ctx, a, b):
    pa, pb = _params(ctx, a), _params(ctx, b)
    assert [k for k, _ in pa] == [k for k, _ in pb]
    for (k, x), (_, y) in zip(pa, pb):
        np.testing.assert_array_equal(x, y, err_msg=k)


def _step(net, x, t):
    net.set_input(x)
    net.set_target(t)
    net.step()


def test_dense_mlp_checkpoint_rebuilds_and_continues(ctx, tmp_path):
    spec = C.DenseSpec()
    net = C.build_dense(ctx, spec, 1)
    xs, ts = C.dense_data(spec, 4, 1)
    for s in range(3):
        _step(net, xs[s], ts[s])
    p = str(tmp_path / "mlp.nnw")
    nnw.save(net, p, error=0.125)
    f = nnw.read(p)
    assert f.error == 0.125 and [r.type for r in f.records] == [nnw.T_BASE] * 4
    copy = nnw.build(ctx, f, 1)
    _same_params(ctx, net, copy)
    _step(net, xs[3], ts[3])
    _step(copy, xs[3], ts[3])
    np.testing.assert_array_equal(copy.output(), net.output())
    _same_params(ctx, net, copy)


@pytest.mark.parametrize("sac", [False, True])
def test_quantile_head_checkpoint_rebuilds_and_continues(ctx, tmp_path, sac):
    spec = C.QuantileHeadSpec(inputs=64, actions=4, quantiles=16, sac=sac)
    net = C.build_quantile_head(ctx, spec, 2)
    xs, ts, us = C.quantile_head_data(spec, 3, 2)
    for s in range(2):
        if sac:
            net.layers[1].set_random(us[s])
        _step(net, xs[s], ts[s])
    p = str(tmp_path / "head.nnw")
    nnw.save(net, p)
    copy = nnw.build(ctx, nnw.read(p), 2)
    assert type(copy.layers[1]) is type(net.layers[1])
    _same_params(ctx, net, copy)
    for n in (net, copy):
        if sac:
            n.layers[1].set_random(us[2])
        _step(n, xs[2], ts[2])
    np.testing.assert_array_equal(copy.output(), net.output())


def test_lstm_stack_checkpoint_rebuilds(ctx, tmp_path):
    spec = C.LSTMSpec(inputs=8, hidden=16, layers=2, series=6, seq=3)
    net = C.build_lstm(ctx, spec)
    xs = C.lstm_data(spec)
    for t in range(2):
        _step(net, xs[t].reshape(-1), xs[t + 1].reshape(-1))
    p = str(tmp_path / "lstm.nnw")
    nnw.save(net, p)
    f = nnw.read(p)
    assert [r.type for r in f.records] == [nnw.T_BASE, nnw.T_LSTM, nnw.T_LSTM, nnw.T_CONV]
    copy = nnw.build(ctx, f, 1)
    _same_params(ctx, net, copy)


def test_patchtst_checkpoint_loads_into_a_fresh_network(ctx, tmp_path):
    """BatchNorm options, Conv1D, the attention encoder's weight collections, the head and RevIN's
    reference to its normalisation layer, loaded into a differently initialised twin."""
    spec = C.PatchSpec(channels=3, bars=64, patch=16, stride=8, embed=16, heads=2, dk=8, layers=2, horizon=12,
                       norm_batch=5)
    net = C.build_patch(ctx, spec, 2)
    xs, ts = C.patch_data(spec, 2, 3)
    for s in range(2):
        _step(net, xs[s], ts[s])
    p = str(tmp_path / "patch.nnw")
    nnw.save(net, p)
    f = nnw.read(p)
    assert [r.type for r in f.records] == [nnw.T_BASE, nnw.T_BATCHNORM, nnw.T_CONV, nnw.T_MLMH, nnw.T_CONV,
                                           nnw.T_REVIN]
    assert f.records[5].extra["norm_layer"] == 1
    twin = C.build_patch(ctx, C.PatchSpec(**{**spec.__dict__, "seed": spec.seed + 1}), 2)
    nnw.apply(twin, f)
    # the host-side sample count of the batch-norm layer is not part of the file; carry it over
    twin.layers[1].count = net.layers[1].count
    _same_params(ctx, net, twin)
    _step(net, xs[2], ts[2])
    _step(twin, xs[2], ts[2])
    np.testing.assert_array_equal(twin.output(), net.output())


def test_a_checkpoint_of_another_structure_is_refused(ctx, tmp_path):
    spec = C.DenseSpec()
    net = C.build_dense(ctx, spec, 1)
    p = str(tmp_path / "mlp.nnw")
    nnw.save(net, p)
    other = C.build_dense(ctx, C.DenseSpec(sizes=(240, 400, 500, 3)), 1)
    with pytest.raises(nnw.NNWError):
        nnw.load(other, p)
