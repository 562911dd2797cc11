"""The .nnw checkpoint layout (CNet::Save / CNet::Load) without a GPU: a file built here byte by
byte in the reference's field order parses into the expected records and is written back
identically, every layer class this library builds round-trips, and damaged files are refused."""
import struct

import numpy as np
import pytest

from nn_in_trading_b200 import nnw as N

F32 = np.float32


def _arr_head(type_id, count):
    return struct.pack("<qii", -1, type_id, count)


def _buf(a):
    a = np.asarray(a, F32)
    return _arr_head(0x7882, a.size) + a.astype("<f4").tobytes()


def _base(type_id, act, opt, t, out, grad, w=None, m=None, v=None):
    """CNeuronBaseOCL::Save, NeuroNet_Core.mqh:16425-16490, written out field by field."""
    b = struct.pack("<iiiiii", type_id, act, opt, 1, t, 1) + _buf(out) + _buf(np.zeros(len(out))) + _buf(grad)
    if w is None:
        return b + struct.pack("<i", 0)
    return b + struct.pack("<i", 1) + _buf(w) + _buf(m) + _buf(v)


def test_dense_net_file_matches_the_reference_field_order():
    rng = np.random.default_rng(0)
    x, g0 = rng.standard_normal(3).astype(F32), rng.standard_normal(3).astype(F32)
    w, m, v = (rng.standard_normal(2 * 4).astype(F32) for _ in range(3))
    y, g1 = rng.standard_normal(2).astype(F32), rng.standard_normal(2).astype(F32)
    # CNet::Save (NeuroNet_Core.mqh:13833-13860): error, undefine, forecast, time, then the layers
    expected = struct.pack("<dddq", 0.25, 0.5, 0.75, 1700000000)
    expected += _arr_head(0x7788, 2)
    expected += _arr_head(0x7787, 1) + _base(0x7883, -1, 1, 5, x, g0, w, m, v)
    expected += _arr_head(0x7787, 1) + _base(0x7883, 0, 1, 7, y, g1)
    f = N.from_bytes(expected)
    assert (f.error, f.undefine, f.forecast, f.time) == (0.25, 0.5, 0.75, 1700000000)
    a, b = f.records
    assert a.type == N.T_BASE and a.activation == -1 and a.t == 5 and a.neurons == 3
    np.testing.assert_array_equal(a.weights, w)
    np.testing.assert_array_equal(a.m, m)
    np.testing.assert_array_equal(a.v, v)
    assert b.weights is None and b.activation == 0 and b.t == 7
    np.testing.assert_array_equal(b.output, y)
    assert N.to_bytes(f) == expected


def _rand(rng, n):
    return rng.standard_normal(n).astype(F32)


def _record(rng, t, neurons, outputs=0, opt=1):
    r = N.Record(t, int(rng.integers(-1, 7)), opt, 1, int(rng.integers(1, 100)), 1, _rand(rng, neurons),
                 np.zeros(neurons, F32), _rand(rng, neurons))
    if outputs:
        n = outputs * (neurons + 1)
        r.weights = _rand(rng, n)
        if opt == 0:
            r.delta = _rand(rng, n)
        else:
            r.m, r.v = _rand(rng, n), _rand(rng, n)
    return r


def _all_records(rng):
    recs = [_record(rng, N.T_BASE, 7, 5), _record(rng, N.T_BASE, 4, 3, opt=0)]
    c = _record(rng, N.T_CONV, 24, 2)
    c.extra.update(window=4, step=2, conv_w=_rand(rng, 5 * 3 * 2), conv_m=_rand(rng, 30), conv_v=_rand(rng, 30),
                   window_out=3, variables=2)
    recs.append(c)
    a = _record(rng, N.T_MLMH, 8 * 5)
    a.extra.update(layers=2, heads=2, window=8, units=5, window_key=4,
                   **{k: [_rand(rng, int(rng.integers(1, 30))) for _ in range(n)]
                      for k, n in (("qkv_tensors", 4), ("qkv_weights", 6), ("s_tensors", 4), ("ao_tensors", 4),
                                   ("ff_tensors", 12), ("ff_weights", 18))})
    recs.append(a)
    s = _record(rng, N.T_SOFTMAX, 12)
    s.extra["heads"] = 3
    recs.append(s)
    bn = _record(rng, N.T_BATCHNORM, 6)
    bn.extra.update(batch_size=10, options=_rand(rng, 6 * 9))
    recs.append(bn)
    rv = _record(rng, N.T_REVIN, 6)
    rv.extra.update(batch_size=10, options=_rand(rng, 6 * 9), norm_layer=5)
    recs.append(rv)
    ls = _record(rng, N.T_LSTM, 8, 4)
    ls.extra.update(inputs=3, variables=2, lstm_w=_rand(rng, 16 * 8), lstm_m=_rand(rng, 128), lstm_v=_rand(rng, 128))
    recs.append(ls)
    cc = _record(rng, N.T_CONCAT, 3, 2)
    cc.extra.update(inputs2=4, conc_w=_rand(rng, 3 * 9), conc_m=_rand(rng, 27), conc_v=_rand(rng, 27))
    recs.append(cc)
    for t in (N.T_FQF, N.T_SAC):
        h = _record(rng, t, 2, 3)
        h.extra.update(fraction=_record(rng, N.T_BASE, 8), softmax=_record(rng, N.T_SOFTMAX, 8),
                       cosine=_record(rng, N.T_BASE, 8, 6), cos_emb=_record(rng, N.T_BASE, 6),
                       q0=_record(rng, N.T_BASE, 6, 32), q1=_record(rng, N.T_BASE, 32, 8), q2=_record(rng, N.T_BASE, 8))
        h.extra["softmax"].extra["heads"] = 2
        if t == N.T_SAC:
            al = _record(rng, N.T_CONCAT, 2)
            al.extra.update(inputs2=8, conc_w=_rand(rng, 2 * 15), conc_m=_rand(rng, 30), conc_v=_rand(rng, 30))
            h.extra["alphas"] = al
        recs.append(h)
    return recs


def _same(a, b):
    if isinstance(a, N.Record):
        assert isinstance(b, N.Record) and a.type == b.type
        for k in ("activation", "optimization", "batch", "t", "train"):
            assert getattr(a, k) == getattr(b, k), k
        for k in ("output", "prev_output", "gradient", "weights", "delta", "m", "v"):
            _same(getattr(a, k), getattr(b, k))
        assert a.extra.keys() == b.extra.keys()
        for k in a.extra:
            _same(a.extra[k], b.extra[k])
    elif isinstance(a, list):
        assert len(a) == len(b)
        for x, y in zip(a, b):
            _same(x, y)
    elif a is None:
        assert b is None
    elif isinstance(a, np.ndarray):
        np.testing.assert_array_equal(a, b)
    else:
        assert a == b


def test_every_layer_class_round_trips(tmp_path):
    rng = np.random.default_rng(1)
    f = N.NNWFile(_all_records(rng), 0.1, 0.2, 0.3, 42)
    p = str(tmp_path / "net.nnw")
    N.write(p, f)
    g = N.read(p)
    assert (g.error, g.undefine, g.forecast, g.time) == (0.1, 0.2, 0.3, 42)
    _same(f.records, g.records)
    assert N.to_bytes(g) == open(p, "rb").read()


def test_damaged_files_are_refused():
    rng = np.random.default_rng(2)
    data = N.to_bytes(N.NNWFile(_all_records(rng)))
    with pytest.raises(N.NNWError):
        N.from_bytes(data[:-3])          # truncated
    with pytest.raises(N.NNWError):
        N.from_bytes(data + b"\0")       # trailing bytes
    bad = bytearray(data)
    bad[32:40] = struct.pack("<q", 5)    # the layer array's start marker
    with pytest.raises(N.NNWError):
        N.from_bytes(bytes(bad))
    bad = bytearray(data)
    bad[40:44] = struct.pack("<i", 0x7787)  # wrong array type
    with pytest.raises(N.NNWError):
        N.from_bytes(bytes(bad))
