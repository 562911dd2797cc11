"""Every reference-kernel call of a training step launches at least one of the library's kernels, and
the library counts it (nn_launch_count): a call whose launches are not counted looks, from outside,
like work done somewhere else.  A replayed step may fuse two calls into one launch (SumMatrix +
Normalize, an update + NormalizeWeights), so a step launches at least half as many kernels as it
makes calls."""
import pytest

from nn_in_trading_b200 import configs as C

pytestmark = pytest.mark.gpu


def _counted_launches(ctx, net) -> int:
    net.capture()
    net.step()
    ctx.finish()
    before = ctx.launch_count()
    net.step()
    ctx.finish()
    return ctx.launch_count() - before


def test_dense_mlp_online_step_counts_its_launches(ctx):
    spec = C.DenseSpec()
    net = C.build_dense(ctx, spec, 1)
    xs, ts = C.dense_data(spec, 1, 1)
    net.set_input(xs[0])
    net.set_target(ts[0])
    calls = net.launch_count()
    assert _counted_launches(ctx, net) >= (calls + 1) // 2


def test_attention_encoder_step_counts_its_launches(ctx):
    spec = C.MLMHSpec()
    net = C.build_mlmh(ctx, spec, 2)
    xs, ts = C.mlmh_data(spec, 2, 1)
    net.set_input(xs[0])
    net.set_target(ts[0])
    calls = net.launch_count()
    assert _counted_launches(ctx, net) >= (calls + 1) // 2
