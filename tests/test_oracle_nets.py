"""The oracle's restatement of the host sequencing, run over its numpy kernels, against the same
sequencing run over the reference's own kernels (oracle/_ref, NeuroNet.cl compiled for the CPU):
pins the numpy kernels at the real layer shapes of the dense MLP and the attention encoder."""
import numpy as np
import pytest

from nn_in_trading_b200 import configs as C
from oracle import kernels as K
from oracle import nets as O
from oracle.ref import RefKernels
from tests.parity import check_close, check_weights, deactivation_atol

pytestmark = pytest.mark.skipif(not RefKernels.available(), reason="oracle/_ref not built")


def dense(spec, w):
    layers = [O.ODense(n, a, 1, spec.sizes[i + 1] if i + 1 < len(spec.sizes) else 0)
              for i, (n, a) in enumerate(zip(spec.sizes, spec.acts))]
    for layer, ww in zip(layers, w):
        layer.weights[:] = ww
    return O.ONet(layers)


def test_dense_mlp_numpy_oracle_matches_reference_kernels():
    spec = C.DenseSpec()
    w = C.dense_weights(spec)
    xs, ts = C.dense_data(spec, 5, 1)
    nets = {}
    for kind in ("numpy", "reference"):
        O.use_backend(kind)
        nets[kind] = dense(spec, w)
    try:
        for s in range(5):
            for kind in ("numpy", "reference"):
                O.use_backend(kind)
                nets[kind].step(xs[s], ts[s])
            a, b = nets["numpy"], nets["reference"]
            from tests.test_nets_gpu import dense_gradient_floors
            floors = dense_gradient_floors(b)
            for li in range(len(a.layers)):
                check_close(f"step{s} layer{li} output", a.layers[li].output, b.layers[li].output)
                check_close(f"step{s} layer{li} gradient", a.layers[li].gradient, b.layers[li].gradient,
                            atol=floors[li])
            for li in range(len(a.layers) - 1):
                check_weights(f"step{s} layer{li} weights", a.layers[li].weights, b.layers[li].weights,
                              b.layers[li + 1].last_grad, b.layers[li + 1].last_grad_abs)
                a.layers[li].weights[:] = b.layers[li].weights
                a.layers[li].m[:] = b.layers[li].m
                a.layers[li].v[:] = b.layers[li].v
    finally:
        O.use_backend("numpy")


def test_attention_encoder_numpy_oracle_matches_reference_kernels():
    spec = C.MLMHSpec()
    w = C.mlmh_weights(spec)
    xs, ts = C.mlmh_data(spec, 1, 1)
    nets = {}
    try:
        for kind in ("numpy", "reference"):
            O.use_backend(kind)
            inp = O.ODense(spec.window * spec.units, K.NONE, 1, 0)
            enc = O.OMLMH(spec.window, spec.dk, spec.heads, spec.units, spec.layers, spec.activation, 1)
            for i, ws in enumerate(w):
                for name, ww in ws.items():
                    enc.w[i][name][0][:] = ww
            net = O.ONet([inp, enc])
            net.step(xs[0], ts[0])
            nets[kind] = net
    finally:
        O.use_backend("numpy")
    a, b = nets["numpy"].layers, nets["reference"].layers
    check_close("encoder output", a[1].output, b[1].output)
    check_close("input gradient", a[0].gradient, b[0].gradient)
    for i in range(spec.layers):
        check_close(f"L{i} qkv grad", a[1].qkv_g[i], b[1].qkv_g[i])
        for name in ("qkv", "w0", "ff1", "ff2"):
            check_weights(f"L{i} {name}", a[1].w[i][name][0], b[1].w[i][name][0], b[1].last_grads[(i, name)],
                          b[1].last_grads_abs[(i, name)])
            check_close(f"L{i} {name} v", a[1].w[i][name][2], b[1].w[i][name][2])
