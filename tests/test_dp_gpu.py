"""Data parallelism of the library on two GPUs: NCCL allreduce of the weight-gradient arena.

Two child processes (one per GPU) each train on half of a batch through the C ABI with
nn_dp_update_begin/end around the updates; their weights must stay identical and equal the
oracle's full-batch training.  Skipped when fewer than two GPUs are visible.
"""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _gpus() -> int:
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_dir, replay):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    from nn_in_trading_b200 import Context, dp
    from nn_in_trading_b200 import configs as C
    dist = dp.init_host_group("gloo", timeout_s=120)
    try:
        ctx = Context(rank)
        dp.join_dp(ctx, rank, world)
        spec = C.MLMHSpec(layers=2)
        B = 4
        lo, hi = dp.shard(B, rank, world)
        xs, ts = C.mlmh_data(spec, B, 2)
        net = C.build_mlmh(ctx, spec, hi - lo, C.mlmh_weights(spec), dp=True)
        if replay:
            net.capture()
        for s in range(2):
            net.set_input(xs[s][lo:hi])
            net.set_target(ts[s][lo:hi])
            net.step()
        enc = net.layers[1]
        out = {f"{i}_{n}": ctx.read(enc.w[i][n][0]) for i in range(spec.layers) for n in ("qkv", "w0", "ff1", "ff2")}
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), **out)
        ctx.dp_shutdown()
        ctx.close()
    finally:
        dist.barrier()
        dist.destroy_process_group()


@pytest.mark.skipif(_gpus() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("replay", [False, True])
def test_two_gpu_data_parallel_equals_full_batch(tmp_path, replay):
    import torch.multiprocessing as mp

    from nn_in_trading_b200 import configs as C
    from oracle import kernels as K
    from oracle import nets as O
    from tests.parity import check_weights
    world = 2
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path), replay), nprocs=world,
                       start_method="spawn", join=True)
    spec = C.MLMHSpec(layers=2)
    O.use_backend("numpy")
    inp = O.ODense(spec.window * spec.units, K.NONE, 4, 0)
    enc = O.OMLMH(spec.window, spec.dk, spec.heads, spec.units, spec.layers, spec.activation, 4)
    for i, ws in enumerate(C.mlmh_weights(spec)):
        for name, w in ws.items():
            enc.w[i][name][0][:] = w
    net = O.ONet([inp, enc])
    xs, ts = C.mlmh_data(spec, 4, 2)
    r0, r1 = np.load(tmp_path / "rank0.npz"), np.load(tmp_path / "rank1.npz")
    for s in range(2):
        net.step(xs[s], ts[s])
    for i in range(spec.layers):
        for n in ("qkv", "w0", "ff1", "ff2"):
            a, b = r0[f"{i}_{n}"], r1[f"{i}_{n}"]
            np.testing.assert_array_equal(a, b)
            # two steps from the same start: compare the second update against the oracle's
            check_weights(f"L{i} {n}", a, enc.w[i][n][0], enc.last_grads[(i, n)], enc.last_grads_abs[(i, n)])


SAC_B = 8


def _sac_spec():
    from nn_in_trading_b200.sac import SACSpec
    return SACSpec(state=12, action=3, hidden=16)


def _sac_worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    from nn_in_trading_b200 import Context, dp
    from nn_in_trading_b200.sac import SACAgent, sac_data, sac_weights
    dist = dp.init_host_group("gloo", timeout_s=120)
    try:
        ctx = Context(rank)
        dp.join_dp(ctx, rank, world)
        spec = _sac_spec()
        lo, hi = dp.shard(SAC_B, rank, world)
        data = sac_data(spec, SAC_B, 1)
        width = {"s": spec.state, "a": spec.action, "r": 1, "s2": spec.state, "done": 1, "eps1": spec.action,
                 "eps2": spec.action}
        agent = SACAgent(ctx, spec, hi - lo, sac_weights(spec), dp=True)
        agent.capture()
        agent.set_batch({k: v[0][lo * width[k]:hi * width[k]] for k, v in data.items()})
        agent.step()
        out = {f"actor{i}": ctx.read(agent.actor[i].weights) for i in range(3)}
        for k in range(2):
            out[f"critic{k}_conc"] = ctx.read(agent.critics[k][1].conc_w)
            out[f"critic{k}_w1"] = ctx.read(agent.critics[k][1].weights)
            out[f"target{k}_conc"] = ctx.read(agent.targets[k][1].conc_w)
        np.savez(os.path.join(out_dir, f"sac_rank{rank}.npz"), **out)
        ctx.dp_shutdown()
        ctx.close()
    finally:
        dist.barrier()
        dist.destroy_process_group()


@pytest.mark.skipif(_gpus() < 2, reason="needs two GPUs")
def test_two_gpu_sac_equals_full_batch(tmp_path):
    """Two ranks of 4 transitions: the critic and actor gradients are averaged in two update regions;
    weights stay identical on both ranks and equal the oracle's 8-transition step.  One step: a
    weight whose first-step gradient cancelled may legitimately take the other Adam direction
    (tests/parity.py), which a second step's comparison could no longer attribute."""
    import torch.multiprocessing as mp

    from nn_in_trading_b200.sac import sac_data, sac_weights
    from oracle import nets as O
    from tests.parity import check_close, check_weights
    world = 2
    mp.start_processes(_sac_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, start_method="spawn",
                       join=True)
    spec = _sac_spec()
    O.use_backend("numpy")
    oracle = O.OSACAgent(spec, SAC_B, sac_weights(spec))
    data = sac_data(spec, SAC_B, 1)
    oracle.step({k: v[0] for k, v in data.items()})
    r0, r1 = np.load(tmp_path / "sac_rank0.npz"), np.load(tmp_path / "sac_rank1.npz")
    for name in r0.files:
        np.testing.assert_array_equal(r0[name], r1[name])
    for i in range(3):
        upd = oracle.actor.layers[i + 1]
        check_weights(f"actor{i}", r0[f"actor{i}"], oracle.actor.layers[i].weights, upd.last_grad, upd.last_grad_abs)
    for k in range(2):
        c = oracle.critics[k].layers
        check_weights(f"critic{k} conc", r0[f"critic{k}_conc"], c[1].conc_w, c[1].last_grad, c[1].last_grad_abs)
        check_weights(f"critic{k} w1", r0[f"critic{k}_w1"], c[1].weights, c[2].last_grad, c[2].last_grad_abs)
        check_close(f"target{k} conc", r0[f"target{k}_conc"], oracle.targets[k].layers[1].conc_w)
