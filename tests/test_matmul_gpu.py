"""MatMult / MatMultGrad (NeuroNet.cl:5969-6060) at sizes past the golden cases.

The golden cases pin both kernels against the reference at small and medium shapes; these run the
tensor-core and split-k paths at full size against a float64 product of the same operands (the
reference's sum in float64: every product of finite operands, non-finite operands adding nothing),
check the numeric flags row by row, and the refusal of nn_set_batch.
"""
import numpy as np
import pytest

from nn_in_trading_b200.api import NNError
from tests.parity import check_close
from tests.test_kernels_gpu import run_on_gpu

pytestmark = pytest.mark.gpu


def _f64(x):
    x = np.asarray(x, np.float64)
    return np.where(np.isfinite(x), x, 0.0)


@pytest.mark.parametrize("rows,dim,cols,var,mvs", [(2048, 1024, 1536, 2, 1), (1000, 777, 515, 3, 0),
                                                    (4, 100000, 6, 1, 1)])
def test_mat_mult_large(ctx, rows, dim, cols, var, mvs):
    rng = np.random.default_rng(rows + dim)
    a = rng.standard_normal(var * rows * dim).astype(np.float32)
    b = rng.standard_normal((var if mvs else 1) * dim * cols).astype(np.float32)
    args = [a, b, np.zeros(var * rows * cols, np.float32), dim, mvs, 0, 0, 0, np.zeros(1, np.float32), 0]
    got = run_on_gpu(ctx, "MatMult", args, (rows, cols, var), None)
    A3 = _f64(a).reshape(var, rows, dim)
    B3 = _f64(b).reshape(var if mvs else 1, dim, cols)
    ref = np.einsum("vrd,vdc->vrc", A3, B3 if mvs else np.broadcast_to(B3, (var, dim, cols)))
    check_close("MatMult result", got[2], ref.reshape(-1).astype(np.float32))


@pytest.mark.parametrize("rows,dim,cols,var,mvs", [(1024, 512, 768, 2, 1), (4096, 256, 128, 8, 0),
                                                    (3, 40000, 5, 2, 1)])
def test_mat_mult_grad_large(ctx, rows, dim, cols, var, mvs):
    rng = np.random.default_rng(rows * 3 + cols)
    nb = (var if mvs else 1) * dim * cols
    m1 = rng.standard_normal(var * rows * dim).astype(np.float32)
    m2 = rng.standard_normal(nb).astype(np.float32)
    g = (rng.standard_normal(var * rows * cols) * 0.01).astype(np.float32)
    args = [m1, np.zeros_like(m1), m2, np.zeros_like(m2), g, dim, mvs, 0, 0, 0, 0, 0]
    got = run_on_gpu(ctx, "MatMultGrad", args, (rows, cols, var), None)
    A3, G3 = _f64(m1).reshape(var, rows, dim), _f64(g).reshape(var, rows, cols)
    B3 = _f64(m2).reshape(var if mvs else 1, dim, cols)
    d1 = np.einsum("vrc,vdc->vrd", G3, B3 if mvs else np.broadcast_to(B3, (var, dim, cols)))
    d2 = np.einsum("vrd,vrc->vdc", A3, G3)
    if not mvs:
        d2 = d2.sum(axis=0, keepdims=True)
    check_close("MatMultGrad matr1_gr", got[1], d1.reshape(-1).astype(np.float32))
    check_close("MatMultGrad matr2_gr", got[3], d2.reshape(-1).astype(np.float32))


def test_mat_mult_flags_mark_rows_and_columns(ctx):
    """A NaN in row r of matr1 flags row r; an inf in column c of matr2 flags column c; the other
    outputs are unflagged and equal the product without the poisoned operands."""
    rows, dim, cols = 512, 384, 640
    rng = np.random.default_rng(11)
    a = rng.standard_normal(rows * dim).astype(np.float32)
    b = rng.standard_normal(dim * cols).astype(np.float32)
    a[7 * dim + 5] = np.nan
    b[100 * cols + 300] = np.inf
    args = [a, b, np.zeros(rows * cols, np.float32), dim, 1, 0, 0, 0, np.full(rows * cols, 7, np.float32), 1]
    got = run_on_gpu(ctx, "MatMult", args, (rows, cols, 1), None)
    flags = got[8].reshape(rows, cols)
    want = np.zeros((rows, cols), np.float32)
    want[7, :] = 1
    want[:, 300] = 1
    np.testing.assert_array_equal(flags, want)
    ref = _f64(a).reshape(rows, dim) @ _f64(b).reshape(dim, cols)
    check_close("MatMult flagged result", got[2], ref.reshape(-1).astype(np.float32))


def test_mat_mult_refuses_a_batch(ctx):
    k = ctx.kernel("MatMult")
    hs = [ctx.buffer(64) for _ in range(4)]
    for i, h in zip((0, 1, 2, 8), hs):
        k.set(i, h)
    for i, v in zip((3, 4, 5, 6, 7, 9), (4, 1, 0, 0, 0, 0)):
        k.set(i, v)
    k.batch(2)
    with pytest.raises(NNError):
        k.run((2, 2, 1))
    for h in hs:
        ctx.free(h)
    ctx.lib.nn_kernel_free(k.id)
