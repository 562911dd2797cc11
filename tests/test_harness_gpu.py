"""The C++ host (nn_in_trading_b200/harness/dense_online.cpp) trains the 240-500-500-3 dense MLP
online through the C ABI alone and gets bit for bit what the library's Python mirror of CNet gets
with the same kernels, arguments and order (the eager Net path, itself checked against the oracle
step by step in tests/test_nets_gpu.py); its first forward output also matches the oracle."""
import os
import shutil
import subprocess

import numpy as np
import pytest

from nn_in_trading_b200 import configs as C
from nn_in_trading_b200 import harness
from oracle import nets as O
from tests.parity import check_close
from tests.test_nets_gpu import oracle_dense

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(shutil.which("g++") is None, reason="no g++ on this machine")]

STEPS = 8


def _write_case(d, spec, weights, xs, ts):
    with open(os.path.join(d, "net.txt"), "w") as f:
        f.write(",".join(str(n) for n in spec.sizes) + "\n")
        f.write(",".join(str(int(a)) for a in spec.acts) + "\n")
    for l, w in enumerate(weights):
        np.asarray(w, dtype=np.float32).tofile(os.path.join(d, f"w{l}.f32"))
    xs.astype(np.float32).tofile(os.path.join(d, "x.f32"))
    ts.astype(np.float32).tofile(os.path.join(d, "t.f32"))


def test_cpp_host_matches_the_python_mirror_bit_for_bit(ctx, tmp_path):
    O.use_backend("numpy")
    spec = C.DenseSpec()
    w = C.dense_weights(spec)
    xs, ts = C.dense_data(spec, STEPS, 1)
    _write_case(str(tmp_path), spec, w, xs, ts)
    exe = harness.build(out=str(tmp_path / "dense_online"))
    r = subprocess.run([exe, "--dir", str(tmp_path), "--steps", str(STEPS)], capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stderr
    n_out = spec.sizes[-1]
    y_cpp = np.fromfile(tmp_path / "y.f32", dtype=np.float32).reshape(STEPS, n_out)

    net = C.build_dense(ctx, spec, 1, w)
    out = net.layers[-1]
    y_py = np.empty_like(y_cpp)
    for s in range(STEPS):
        net.set_input(xs[s])
        net.set_target(ts[s])
        net.step()  # eager: the same executions the C++ host issues
        y_py[s] = ctx.read(out.output, n_out)
    np.testing.assert_array_equal(y_cpp, y_py)
    for l, layer in enumerate(net.layers[:-1]):
        n = layer.outputs * (layer.neurons + 1)
        for name, h in (("w", layer.weights), ("m", layer.m), ("v", layer.v)):
            got = np.fromfile(tmp_path / f"{name}{l}.out.f32", dtype=np.float32)
            np.testing.assert_array_equal(got, ctx.read(h, n), err_msg=f"layer {l} {name} after {STEPS} steps")

    # the first step's forward output against the oracle's restatement of the reference kernels
    onet = oracle_dense(spec, 1, w)
    onet.step(xs[0], ts[0])
    check_close("C++ host step0 output", y_cpp[0], onet.layers[-1].output.reshape(-1))
