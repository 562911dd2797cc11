"""Data-parallel contract on CPU with two gloo ranks.

Two spawned processes each train the oracle network on their half of a batch
and average every batch-mean weight gradient over the ranks (gloo allreduce,
the role NCCL plays on the GPUs) before the reference update; the result must
equal one process training on the whole batch.  Also exercises the host-side
plumbing of nn_in_trading_b200.dp (unique-id broadcast, max over ranks,
sharding) that bench.py uses under torchrun.
"""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _dense_oracle(batch, weights, spec):
    from oracle import nets as O
    layers = []
    for i, (n, a) in enumerate(zip(spec.sizes, spec.acts)):
        layers.append(O.ODense(n, a, batch, spec.sizes[i + 1] if i + 1 < len(spec.sizes) else 0))
    for layer, w in zip(layers, weights):
        layer.weights[:] = w
    return O.ONet(layers)


def _worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    import torch
    from nn_in_trading_b200 import dp
    from nn_in_trading_b200 import configs as C
    from oracle import nets as O
    dist = dp.init_host_group("gloo", timeout_s=60)
    try:
        uid = dp.share_unique_id(bytes(range(128)) if rank == 0 else None, rank)
        assert uid == bytes(range(128))
        assert dp.max_over_ranks(float(rank + 1)) == float(world)
        spec = C.DenseSpec(sizes=(24, 16, 8, 3))
        w = C.dense_weights(spec)
        B = 8
        xs, ts = C.dense_data(spec, 3, B)
        lo, hi = dp.shard(B, rank, world)

        def mean_over_ranks(G):
            t = torch.from_numpy(np.ascontiguousarray(G, dtype=np.float64))
            dist.all_reduce(t)
            return (t / world).numpy().astype(np.float32)

        O.set_grad_hook(mean_over_ranks)
        net = _dense_oracle(hi - lo, w, spec)
        for s in range(3):
            net.step(xs[s][lo:hi], ts[s][lo:hi])
        O.set_grad_hook(None)
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), *[l.weights for l in net.layers[:-1]])
    finally:
        dist.barrier()
        dist.destroy_process_group()


def test_two_rank_data_parallel_equals_full_batch(tmp_path):
    world = 2
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, start_method="spawn",
                       join=True)
    from nn_in_trading_b200 import configs as C
    spec = C.DenseSpec(sizes=(24, 16, 8, 3))
    w = C.dense_weights(spec)
    xs, ts = C.dense_data(spec, 3, 8)
    full = _dense_oracle(8, w, spec)
    for s in range(3):
        full.step(xs[s], ts[s])
    r0 = np.load(tmp_path / "rank0.npz")
    r1 = np.load(tmp_path / "rank1.npz")
    for i, layer in enumerate(full.layers[:-1]):
        a, b = r0[f"arr_{i}"], r1[f"arr_{i}"]
        np.testing.assert_array_equal(a, b)  # replicas stay identical
        np.testing.assert_allclose(a, layer.weights, rtol=0, atol=1e-6 * max(1.0, np.abs(layer.weights).max()))


def test_shard_rejects_uneven_split():
    from nn_in_trading_b200 import dp
    assert dp.shard(256, 3, 4) == (192, 256)
    with pytest.raises(ValueError):
        dp.shard(10, 0, 3)


def _sac_worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    import torch
    from nn_in_trading_b200 import dp
    from nn_in_trading_b200.sac import SACSpec, sac_data, sac_weights
    from oracle import nets as O
    dist = dp.init_host_group("gloo", timeout_s=60)
    try:
        spec = SACSpec(state=10, action=2, hidden=12)
        B = 6
        lo, hi = dp.shard(B, rank, world)
        data = sac_data(spec, B, 2)
        width = {"s": spec.state, "a": spec.action, "r": 1, "s2": spec.state, "done": 1, "eps1": spec.action,
                 "eps2": spec.action}

        def mean_over_ranks(G):
            t = torch.from_numpy(np.ascontiguousarray(G, dtype=np.float64))
            dist.all_reduce(t)
            return (t / world).numpy().astype(np.float32)

        O.use_backend("numpy")
        O.set_grad_hook(mean_over_ranks)
        agent = O.OSACAgent(spec, hi - lo, sac_weights(spec))
        for s in range(2):
            agent.step({k: v[s][lo * width[k]:hi * width[k]] for k, v in data.items()})
        O.set_grad_hook(None)
        np.savez(os.path.join(out_dir, f"sac{rank}.npz"), *[l.weights for l in agent.actor.layers[:3]],
                 agent.critics[0].layers[1].conc_w, agent.targets[1].layers[1].conc_w)
    finally:
        dist.barrier()
        dist.destroy_process_group()


def test_two_rank_sac_equals_full_batch(tmp_path):
    """The SAC step's two gradient averages (critics, then the actor) on CPU ranks equal one process
    stepping the whole replay batch."""
    world = 2
    mp.start_processes(_sac_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, start_method="spawn",
                       join=True)
    from nn_in_trading_b200.sac import SACSpec, sac_data, sac_weights
    from oracle import nets as O
    O.use_backend("numpy")
    spec = SACSpec(state=10, action=2, hidden=12)
    full = O.OSACAgent(spec, 6, sac_weights(spec))
    data = sac_data(spec, 6, 2)
    for s in range(2):
        full.step({k: v[s] for k, v in data.items()})
    ref = [l.weights for l in full.actor.layers[:3]] + [full.critics[0].layers[1].conc_w,
                                                        full.targets[1].layers[1].conc_w]
    r0, r1 = np.load(tmp_path / "sac0.npz"), np.load(tmp_path / "sac1.npz")
    for i, w in enumerate(ref):
        a, b = r0[f"arr_{i}"], r1[f"arr_{i}"]
        np.testing.assert_array_equal(a, b)
        np.testing.assert_allclose(a, w, rtol=0, atol=1e-5 * max(1.0, np.abs(w).max()))
