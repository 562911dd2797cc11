"""Overlapped transfers through the C ABI (nn_buffer_write_async, nn_buffer_read_async,
nn_transfer_wait): round trips, ordering against executions, and the two-deep double-buffered
pipeline `bench.py` drives end to end, each step checked against the synchronous path."""
import numpy as np
import pytest
import torch

from oracle import kernels as K
from tests.parity import check_close

pytestmark = pytest.mark.gpu

TANH = 0


def _pinned(a):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).pin_memory()


def test_round_trip_and_tickets(ctx):
    lib = ctx.lib
    x = _pinned(np.random.default_rng(1).standard_normal(1000))
    y = _pinned(np.zeros(1000))
    h = ctx.buffer(1000)
    ctx._check(lib.nn_buffer_write_async(h, x.data_ptr(), 0, 1000))
    t = lib.nn_buffer_read_async(h, y.data_ptr(), 0, 1000)
    assert t >= 0
    ctx._check(lib.nn_transfer_wait(t))
    np.testing.assert_array_equal(y.numpy(), x.numpy())
    assert lib.nn_transfer_wait(-1) < 0
    assert lib.nn_transfer_wait(t + 1) < 0  # not issued yet
    assert lib.nn_buffer_read_async(h, y.data_ptr(), 990, 20) < 0  # past the buffer
    ctx.free(h)


def test_executions_are_ordered_after_writes_and_before_reads(ctx):
    """write_async -> Activation -> read_async: the kernel sees the written input and the read sees
    the kernel's output."""
    lib = ctx.lib
    n = 1 << 16
    x = np.random.default_rng(2).standard_normal(n).astype(np.float32) * 3
    hx, hy = _pinned(x), _pinned(np.zeros(n))
    bi, bo = ctx.buffer(n), ctx.buffer(n)
    k = ctx.kernel("Activation").args(bi, bo, TANH)
    ctx._check(lib.nn_buffer_write_async(bi, hx.data_ptr(), 0, n))
    k.run((n,))
    t = lib.nn_buffer_read_async(bo, hy.data_ptr(), 0, n)
    ctx._check(lib.nn_transfer_wait(t))
    ref = np.zeros(n, np.float32)
    K.Activation(x, ref, TANH, gsize=(n,))
    check_close("activation through overlapped transfers", hy.numpy(), ref)
    ctx.free(bi)
    ctx.free(bo)


def test_double_buffered_pipeline(ctx):
    """Two steps in flight: step i's input written into staging half i % 2 while step i-1 runs,
    copied into the kernel's input, its result staged and read while step i+1 runs."""
    lib = ctx.lib
    n, steps = 1 << 18, 6
    rng = np.random.default_rng(3)
    xs = [rng.standard_normal(n).astype(np.float32) * 2 for _ in range(steps)]
    hx = [_pinned(x) for x in xs]
    hy = [_pinned(np.zeros(n)) for _ in range(2)]
    stage_in = [ctx.buffer(n) for _ in range(2)]
    stage_out = [ctx.buffer(n) for _ in range(2)]
    bi, bo = ctx.buffer(n), ctx.buffer(n)
    k = ctx.kernel("Activation").args(bi, bo, TANH)

    def enqueue(i):
        half = i % 2
        ctx._check(lib.nn_buffer_write_async(stage_in[half], hx[i].data_ptr(), 0, n))
        ctx.copy(bi, stage_in[half], n)
        k.run((n,))
        ctx.copy(stage_out[half], bo, n)
        t = lib.nn_buffer_read_async(stage_out[half], hy[half].data_ptr(), 0, n)
        assert t >= 0
        return t

    tickets = {0: enqueue(0), 1: enqueue(1)}
    for i in range(steps):
        ctx._check(lib.nn_transfer_wait(tickets.pop(i)))
        ref = np.zeros(n, np.float32)
        K.Activation(xs[i], ref, TANH, gsize=(n,))
        check_close(f"step{i}", hy[i % 2].numpy(), ref)
        if i + 2 < steps:
            tickets[i + 2] = enqueue(i + 2)
    for h in stage_in + stage_out + [bi, bo]:
        ctx.free(h)


def test_buffer_write_ex_and_read_ex_take_a_device_byte_offset_and_a_host_start(ctx):
    """COpenCLMy::BufferWrite(buffer, data, offset, start, count) semantics: `offset` is a byte
    position in the device buffer, `start` an element index into the host array."""
    import ctypes
    lib = ctx.lib
    n = 64
    h = ctx.buffer(n)
    ctx.fill(h, -1.0, n)
    host = np.arange(100, dtype=np.float32) + 0.5
    p = host.ctypes.data_as(ctypes.c_void_p)
    # host elements 10..19 -> device floats 5..14 (byte offset 20)
    ctx._check(lib.nn_buffer_write_ex(h, p, 20, 10, 10))
    dev = ctx.read(h, n)
    want = np.full(n, -1.0, np.float32)
    want[5:15] = host[10:20]
    np.testing.assert_array_equal(dev, want)
    # device floats 7..12 (byte offset 28) -> host elements 40..45, the rest of the array untouched
    out = np.full(50, 7.0, np.float32)
    ctx._check(lib.nn_buffer_read_ex(h, out.ctypes.data_as(ctypes.c_void_p), 28, 40, 6))
    expect = np.full(50, 7.0, np.float32)
    expect[40:46] = want[7:13]
    np.testing.assert_array_equal(out, expect)
    # the whole-buffer call CBufferFloat::BufferRead issues: (0, 0, total)
    ctx._check(lib.nn_buffer_read_ex(h, out.ctypes.data_as(ctypes.c_void_p), 0, 0, 50))
    np.testing.assert_array_equal(out, want[:50])
    # refused: byte offset not a multiple of 4, negative start, range past the buffer
    assert lib.nn_buffer_write_ex(h, p, 2, 0, 1) == -2
    assert lib.nn_buffer_write_ex(h, p, 0, -1, 1) == -2
    assert lib.nn_buffer_read_ex(h, out.ctypes.data_as(ctypes.c_void_p), 4 * 60, 0, 5) == -5
    ctx.free(h)
