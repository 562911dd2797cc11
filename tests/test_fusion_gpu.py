"""Command lists run some back-to-back executions of the reference's host code as one kernel; the
result must be the executions' own, bit for bit.

SumMatrix followed by Normalize of its output (CNeuronBaseOCL::SumAndNormalize, NeuroNet_Core.mqh:
17976-18075, the attention encoder's residual) runs as one pass over the rows."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _sum_norm(ctx, a, b, rows, dim, batch, mult, record):
    ha, hb, ho = ctx.buffer(a.size), ctx.buffer(b.size), ctx.buffer(a.size)
    ctx.write(ha, a)
    ctx.write(hb, b)
    ks = ctx.kernel("SumMatrix").args(ha, hb, ho, dim, mult, 0, 0, 0, ho, 0).batch(batch)
    kn = ctx.kernel("Normalize").args(ho, dim).batch(batch)
    if record:
        ctx.record_begin()
    ks.run((rows,))
    kn.run((rows,))
    if record:
        lid = ctx.record_end()
        ctx.run_list(lid)
        ctx.free_list(lid)
    out = ctx.read(ho, a.size)
    for h in (ha, hb, ho):
        ctx.free(h)
    return out


@pytest.mark.parametrize("rows,dim,batch", [(120, 64, 256), (63, 128, 64), (7, 5, 3), (1, 33, 1)])
def test_recorded_sum_and_normalize_equals_the_two_executions(ctx, rows, dim, batch):
    rng = np.random.default_rng(rows + dim)
    n = rows * dim * batch
    a = (rng.standard_normal(n) * 3).astype(np.float32)
    b = rng.standard_normal(n).astype(np.float32)
    a[::97] = np.nan
    eager = _sum_norm(ctx, a, b, rows, dim, batch, 0.5, record=False)
    fused = _sum_norm(ctx, a, b, rows, dim, batch, 0.5, record=True)
    np.testing.assert_array_equal(fused, eager)
