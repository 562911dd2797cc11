"""nn_update_weights_adam_fixed (batched dense Adam update with its gradient partials in the
library's fixed device array) against the regular entry point: nn_execute of UpdateWeightsAdam
with nn_set_batch, on identical copies of the weights and moments, two calls in a row.

The entry point exists for hosts that cannot allocate device memory once training runs (a host
that hands all free memory to its own pool, or a loop that cannot take an allocation's stall), so
the test also checks that repeated calls leave the device's free memory unchanged."""
import ctypes

import numpy as np
import pytest

from tests.parity import check_close

pytestmark = pytest.mark.gpu

L, B1, B2 = 3e-4, 0.9, 0.999
FIXED_SCRATCH_FLOATS = 1 << 21


def _state(ctx, rng, outputs, inputs, batch):
    nw = outputs * (inputs + 1)
    w = rng.uniform(-0.1, 0.1, nw).astype(np.float32)
    m = rng.normal(0, 1e-3, nw).astype(np.float32)
    v = rng.uniform(0, 1e-5, nw).astype(np.float32)
    g = rng.normal(0, 1e-2, batch * outputs).astype(np.float32)
    x = rng.normal(0, 1, batch * inputs).astype(np.float32)
    bufs = {}
    for name, arr in (("w", w), ("m", m), ("v", v), ("g", g), ("x", x)):
        h = ctx.buffer(arr.size)
        ctx.write(h, arr)
        bufs[name] = h
    return bufs


def _copy_state(ctx, src):
    out = {}
    for name, h in src.items():
        n = ctx.nbytes(h) // 4
        out[name] = ctx.buffer(n)
        ctx.copy(out[name], h, n)
    return out


def _free_bytes(device):
    import torch
    return torch.cuda.mem_get_info(device)[0]


# (256, 256, 1100): the batch split into several parts; (3, 500, 1024): few outputs, many inputs
@pytest.mark.parametrize("outputs,inputs,batch", [(37, 53, 5), (500, 240, 64), (3, 500, 1024),
                                                  (256, 256, 1100)])
def test_fixed_scratch_update_matches_update_weights_adam(ctx, outputs, inputs, batch):
    rng = np.random.default_rng(outputs * 7 + inputs + batch)
    a = _state(ctx, rng, outputs, inputs, batch)
    b = _copy_state(ctx, a)
    k = ctx.kernel("UpdateWeightsAdam")
    k.args(a["w"], a["g"], a["x"], a["m"], a["v"], inputs, L, B1, B2).batch(batch)
    ptr = {n: ctypes.c_void_p(ctx.device_ptr(h)) for n, h in b.items()}
    nw = outputs * (inputs + 1)
    for call in range(2):
        k.run([outputs, inputs + 1])
        ctx.finish()
        free_before = _free_bytes(ctx.device)
        launches = ctx.launch_count()
        rc = ctx.lib.nn_update_weights_adam_fixed(ptr["w"], ptr["g"], ptr["x"], ptr["m"], ptr["v"], outputs,
                                                  inputs, batch, L, B1, B2)
        assert rc == 0, ctx.last_error()
        ctx.finish()
        assert ctx.launch_count() > launches  # its kernels are counted
        assert _free_bytes(ctx.device) == free_before, "the fixed-scratch update allocated device memory"
        for name in ("w", "m", "v"):
            check_close(f"call {call} {name}", ctx.read(b[name], nw), ctx.read(a[name], nw), rtol=1e-5)
    for h in list(a.values()) + list(b.values()):
        ctx.free(h)
    ctx._check(ctx.lib.nn_kernel_free(k.id))


def test_fixed_scratch_rejects_updates_larger_than_the_array(ctx):
    outputs, inputs = 2048, 1024  # 2048 * 1025 floats > 2 Mi
    assert outputs * (inputs + 1) > FIXED_SCRATCH_FLOATS
    h = ctx.buffer(1)
    p = ctypes.c_void_p(ctx.device_ptr(h))
    rc = ctx.lib.nn_update_weights_adam_fixed(p, p, p, p, p, outputs, inputs, 4, L, B1, B2)
    assert rc == -5  # NN_ERR_BOUNDS, before any launch
    assert "exceeds the fixed scratch" in ctx.last_error()
    ctx.free(h)


def test_fixed_scratch_refuses_inside_a_data_parallel_update_region(ctx):
    """Inside nn_dp_update_begin .. end the regular update waits for the ranks' averaged gradient;
    this local update would not, so it is refused (NN_ERR_STATE) and launches nothing."""
    h = ctx.buffer(64)
    p = ctypes.c_void_p(ctx.device_ptr(h))
    ctx.dp_update_begin()
    try:
        launches = ctx.launch_count()
        rc = ctx.lib.nn_update_weights_adam_fixed(p, p, p, p, p, 3, 4, 2, L, B1, B2)
        assert rc == -1
        assert "data-parallel update region" in ctx.last_error()
        assert ctx.launch_count() == launches
    finally:
        ctx.dp_update_end()
    ctx.free(h)
