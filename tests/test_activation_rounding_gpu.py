"""Rounding of the sigmoid and GELU activations (NeuroNet.cl:88-125) on the GPU.

Both divide by 1 + e^t with a branch-free Newton-Raphson division instead of the compiler's IEEE
division.  The reference's sigmoid derivative (clamp(g + y) - y) * y * (1 - y) cancels, so the
last bits of y matter for parity: the division must round like IEEE division, not merely stay
within a few ulp.  The expected values are the same float32 operations done by PyTorch on the same
device (its exp is the CUDA expf, its division the IEEE one), so apart from the rare divisor whose
reciprocal lies within about 2^-46 of a rounding midpoint, the results must agree bit for bit.
"""
import numpy as np
import pytest
import torch

from tests.test_kernels_gpu import run_on_gpu

pytestmark = pytest.mark.gpu

SIGMOID, GELU = 1, 4


def torch_reference(x, act):
    xt = torch.from_numpy(x).cuda()
    if act == SIGMOID:
        t = torch.clamp(-xt, -20.0, 20.0)
        num = torch.ones_like(xt)
    else:
        t = torch.clamp(xt * -1.702, -20.0, 20.0)
        num = xt
    return (num / (1.0 + torch.exp(t))).cpu().numpy()


@pytest.mark.parametrize("act", [SIGMOID, GELU], ids=["sigmoid", "gelu"])
def test_activation_rounds_like_ieee_division(ctx, act):
    rng = np.random.default_rng(11 + act)
    # the whole clamped range, dense near zero where sigmoid is far from 0 and 1
    x = np.concatenate([rng.uniform(-25, 25, 60000), rng.normal(0, 2, 60000),
                        rng.uniform(-1e-3, 1e-3, 8000)]).astype(np.float32)
    x = x[np.abs(x) > 1e-30]
    got = run_on_gpu(ctx, "Activation", [x, np.zeros_like(x), act], (x.size,), None)[1]
    ref = torch_reference(x, act)
    d = np.abs(got.view(np.int32).astype(np.int64) - ref.view(np.int32).astype(np.int64))
    assert d.max() <= 1, f"max {d.max()} ulp from the IEEE quotient"
    assert int(np.count_nonzero(d)) <= 2, f"{int(np.count_nonzero(d))} of {d.size} quotients are not rounded to nearest"
