"""Benchmark: fwd+bwd+Adam training throughput (samples/s) through libnn_b200.so.

Default workload (mlmh_encoder): CNeuronMLMHAttentionOCL encoder, 4 layers, 120 bars x 64
features, 8 heads x key 32, FF 64->256(GELU)->64(LReLU), batch 256 independent sequences per GPU,
fp32, MSE vs N(0,1) targets, Adam; synthetic seeded N(0,1) data.  A step = forward + backward +
Adam of one batch, replayed from command lists.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload mlmh_encoder|dense_mlp|lstm_stack|patchtst] [--batch B]

Other workloads: dense_mlp (240-500-500-3 MLP, batch 1, 1000 sequential online steps), lstm_stack
(2 LSTM layers, hidden 256, 1024 series, one bar per step, a sample = one series over 240 bars),
patchtst (BatchNorm + Conv1D patching + 3 attention layers + head + RevIN, batch 512).

N > 1 (torchrun, one process per GPU): weak scaling, every rank trains its own batch and the
weight gradients are averaged with one NCCL allreduce per step before the updates.
`--impl reference` times the reference's own NeuroNet.cl kernels compiled for the host CPU
(oracle/_ref) on a bounded sample of the same workload, on rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "fwd+bwd+Adam samples/sec"
UNIT = "samples/s"


def env_int(name, default):
    try:
        return int(os.environ.get(name, default))
    except ValueError:
        return default


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi sampled during the timed region (clock, throttle reasons)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "100", "-i", str(self.device)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            p = [x.strip() for x in ln.split(",")]
            if len(p) < 9:
                continue
            try:
                sm.append(float(p[1]))
                mx = float(p[2])
            except ValueError:
                continue
            for n, v in zip(names, p[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# --------------------------------------------------- algorithmic work model
# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one call of each reference kernel
# (every CUDA launch the call makes, weight-image packing included), from one single-pass ncu
# capture of a whole training step of the batch-256 encoder:
#   ncu --metrics dram__bytes_read.sum,dram__bytes_write.sum,gpu__time_duration.sum
#       --clock-control none -s 471 -c 157 --csv python bench.py --steps 3 --warmup 3 --no-cpu-baseline
# Keyed by workload and reference kernel; scaled to other batches by the samples a call processes.
NCU_TRAFFIC = {"mlmh_encoder": {k: (v * 1e6, 256) for k, v in {
    "MHAttentionInsideGradients": 309.32, "UpdateWeightsConvAdam": 64.96, "CalcHiddenGradientConv": 55.54,
    "FeedForwardConv": 27.99, "MHAttentionScore": 122.99, "MHAttentionOut": 163.37, "SumMatrix": 15.73,
    "Normalize": 7.87, "NormalizeWeights": 0.11, "CalcOutputGradient": 15.73}.items()}}


def op_work(op):
    """(flops, bytes) a launch must do at minimum: every operand read once, every result written once.
    B is the launch's own batch (nn_set_batch), so a layer that views its input as per-channel
    sequences counts those sequences."""
    k = op.kernel
    name = k.name
    a = k.values
    g = op.gsize
    B = getattr(k, "b", 1)
    f4 = 4
    if name == "FeedForwardConv":
        units, wout, var = g[0], g[1], g[2] if len(g) > 2 else 1
        inputs, win = a[3], a[5]
        flops = 2.0 * B * units * wout * win * var
        byt = f4 * (B * var * inputs + var * wout * (win + 1) + B * var * units * wout)
        return flops, byt
    if name == "CalcHiddenGradientConv":
        inputs, var = g[0], g[1] if len(g) > 1 else 1
        outputs, win, wout = a[4], a[6], a[7]
        flops = 2.0 * B * var * (outputs // wout) * win * wout
        byt = f4 * (B * var * outputs + var * wout * (win + 1) + 2 * B * var * inputs)
        return flops, byt
    if name == "UpdateWeightsConvAdam":
        nw = g[0]
        inputs, win, wout, step = a[5], a[9], a[10], a[11]
        var = nw // (wout * (win + 1))
        total = (inputs - (win - step) + (step - 1)) // step
        flops = 2.0 * B * total * nw
        byt = f4 * (B * var * total * wout + B * var * inputs + 6 * nw)
        return flops, byt
    if name == "MHAttentionScore":
        U, H, D = g[0], g[1], a[2]
        return 2.0 * B * H * U * U * D, f4 * B * (2 * U * H * D + H * U * U)
    if name == "MHAttentionOut":
        U, H, D = g[0], g[1], a[3]
        return 2.0 * B * H * U * U * D, f4 * B * (H * U * U + 2 * U * H * D)
    if name == "MHAttentionInsideGradients":
        U, H, D = g
        return 6.0 * B * H * U * U * D, f4 * B * (H * U * U + 3 * U * H * D + U * H * D + 3 * U * H * D)
    if name == "SumMatrix":
        return 0.0, f4 * 3 * B * g[0] * a[3]
    if name == "Normalize":
        return 0.0, f4 * 2 * B * g[0] * a[1]
    if name == "NormalizeWeights":
        return 0.0, f4 * 2 * g[0] * a[1]
    if name == "CalcOutputGradient":
        return 0.0, f4 * 3 * B * g[0]
    if name == "FeedForward":  # y[out] = act(W [out][in+1] . [x, 1])
        out, n_in = g[0], a[3]
        return 2.0 * B * out * (n_in + 1), f4 * (out * (n_in + 1) + B * n_in + B * out)
    if name == "CalcHiddenGradient":  # g_in[in] = Deact(W^T g_out) at x_in
        n_in, out = g[0], a[4]
        return 2.0 * B * out * n_in, f4 * (out * (n_in + 1) + B * out + 2 * B * n_in)
    if name == "UpdateWeightsAdam":  # w, m, v read and written; g_out and x read
        out, cols = g[0], g[1]
        return 2.0 * B * out * cols, f4 * (6 * out * cols + B * out + B * (cols - 1))
    if name == "LSTM_FeedForward":  # gate pre-activations of rows g+id (H+3 distinct rows), cell update
        H, V, n_in = g[0], (g[2] if len(g) > 2 else 1) * B, a[1]
        ws = n_in + H + 1
        return (2.0 * V * (H + 3) * ws,
                f4 * ((H + 3) * ws + V * n_in + 2 * V * H + V * 4 * H + 2 * V * H + V * H))
    if name == "LSTM_ConcatenatedGradient":
        H, V = g[0], (g[1] if len(g) > 1 else 1) * B
        return 0.0, f4 * (V * H + 2 * V * H + 4 * V * H + 4 * V * H)
    if name == "LSTM_HiddenGradient":  # dx = a W[:, H:], dW = a^T [h; x] summed over the series
        H, V, n_in = g[0], (g[1] if len(g) > 1 else 1) * B, a[8]
        ws = H + n_in + 1
        return (2.0 * V * 4 * H * n_in + 2.0 * V * 4 * H * (H + n_in),
                f4 * (V * 4 * H + 4 * H * ws + V * (H + n_in) + V * H + V * n_in + 4 * H * ws))
    if name == "BatchFeedForward":
        n = g[0]
        return 0.0, f4 * (2 * B * n + 2 * 9 * n)
    if name == "CalcHiddenGradientBatch":
        n = g[0]
        return 0.0, f4 * (3 * B * n + 9 * n)
    if name in ("RevInFeedForward", "RevInHiddenGraddient"):
        n = g[0]
        return 0.0, f4 * ((2 if name == "RevInFeedForward" else 3) * B * n)
    if name == "DeActivation":
        return 0.0, f4 * 3 * B * g[0]
    return 0.0, 0.0


# ------------------------------------------------------------- workloads
class Workload:
    """One training configuration: how to build it through the library, its synthetic data, what a
    sample is, and a bounded CPU sample of the same network through the reference's own kernels."""

    key = ""
    name = ""
    default_batch = 1
    default_steps = 30
    recordable = True

    def __init__(self, batch):
        self.B = batch

    def samples_per_step(self) -> float:
        return float(self.B)

    def build(self, ctx, dp):
        raise NotImplementedError

    def data(self, pool, seed):
        """([pool][n_in], [pool][n_out]) float32 arrays: inputs and targets of `pool` steps."""
        raise NotImplementedError

    # -- the step's inputs and the result read back, for a network trained against targets (Net) --
    def slots(self, pool, seed):
        """Per input buffer: [pool][floats] float32 arrays of `pool` steps."""
        return list(self.data(pool, seed))

    def io(self, obj):
        """(input buffer handles in the order of slots(), output buffer handle, output floats)."""
        out = obj.layers[-1]
        return [obj.layers[0].output, obj.target], out.output, out.neurons * out.batch

    def host_metric(self, y, slots, i):
        """(name, value) the host computes from step i's read-back result: the MSE against the targets."""
        d = y - slots[1][i]
        return "mse_last", float(np.dot(d, d)) / d.size

    def ops(self, obj):
        return obj.fwd_ops + obj.bwd_ops + obj.upd_ops

    def config(self, world) -> dict:
        raise NotImplementedError

    def oracle_net(self, O, K, batch):
        raise NotImplementedError

    def ref_data(self, pool):
        return self.data(pool, 7)

    def ref_sample_desc(self, n, el, backend) -> str:
        raise NotImplementedError

    def ref_samples_per_step(self, batch) -> float:
        return float(batch)


class MLMHWorkload(Workload):
    key = "mlmh_encoder"
    name = "mlmh_encoder_4x120x64_h8k32_ff256"
    default_batch = 256
    default_steps = 400  # about 1.05 s timed

    def __init__(self, batch):
        super().__init__(batch)
        from nn_in_trading_b200 import configs as C
        self.C, self.spec = C, C.MLMHSpec()

    def build(self, ctx, dp):
        return self.C.build_mlmh(ctx, self.spec, self.B, self.C.mlmh_weights(self.spec), dp=dp)

    def data(self, pool, seed):
        xs, ts = self.C.mlmh_data(self.spec, self.B, pool, seed=seed)
        return xs.reshape(pool, -1), ts.reshape(pool, -1)

    def config(self, world):
        s = self.spec
        return {"workload": self.name, "global_batch": self.B * world, "per_gpu_batch": self.B, "seq_len": s.units,
                "embed": s.window, "heads": s.heads, "key": s.dk, "layers": s.layers, "sample": "one sequence",
                "parallelism": f"dp{world}",
                "l2": "no flush: every step streams >1 GB of activations and scores, well above the 126 MB L2"}

    def oracle_net(self, O, K, batch):
        s = self.spec
        inp = O.ODense(s.window * s.units, K.NONE, batch, 0)
        enc = O.OMLMH(s.window, s.dk, s.heads, s.units, s.layers, s.activation, batch)
        for i, ws in enumerate(self.C.mlmh_weights(s)):
            for name, w in ws.items():
                enc.w[i][name][0][:] = w
        return O.ONet([inp, enc])

    def ref_data(self, pool):
        xs, ts = self.C.mlmh_data(self.spec, 1, pool, seed=7)
        return xs.reshape(pool, -1), ts.reshape(pool, -1)

    def ref_sample_desc(self, n, el, backend):
        return (f"{n} training steps of one 120x64 sequence (fwd+bwd+Adam of all 4 layers) through the "
                f"{backend}, {el:.1f} s")


class DenseWorkload(Workload):
    key = "dense_mlp"
    name = "dense_mlp_240_500tanh_500sigmoid_3"
    default_batch = 1
    default_steps = 25000  # 25 runs of the 1000-step online configuration, about 1.05 s timed

    def __init__(self, batch):
        super().__init__(batch)
        from nn_in_trading_b200 import configs as C
        self.C, self.spec = C, C.DenseSpec()

    def build(self, ctx, dp):
        return self.C.build_dense(ctx, self.spec, self.B, self.C.dense_weights(self.spec), dp=dp)

    def data(self, pool, seed):
        xs, ts = self.C.dense_data(self.spec, pool, self.B, seed=seed)
        return xs.reshape(pool, -1), ts.reshape(pool, -1)

    def config(self, world):
        return {"workload": self.name, "global_batch": self.B * world, "per_gpu_batch": self.B,
                "sample": "one online training step (batch 1, sequential)", "parallelism":
                f"dp{world}" if world > 1 else "replicas only: the online steps are sequential",
                "l2": "no flush: the whole state (4.5 MB) is L2-resident, as in the reference's online loop"}

    def oracle_net(self, O, K, batch):
        s = self.spec
        layers = []
        for i, (n, a) in enumerate(zip(s.sizes, s.acts)):
            outputs = s.sizes[i + 1] if i + 1 < len(s.sizes) else 0
            layers.append(O.ODense(n, a, batch, outputs))
        for layer, w in zip(layers, self.C.dense_weights(s)):
            layer.weights[:] = w
        return O.ONet(layers)

    def ref_data(self, pool):
        xs, ts = self.C.dense_data(self.spec, pool, 1, seed=7)
        return xs.reshape(pool, -1), ts.reshape(pool, -1)

    def ref_sample_desc(self, n, el, backend):
        return f"{n} online steps of the 240-500-500-3 MLP (fwd+bwd+Adam) through the {backend}, {el:.1f} s"


class LSTMWorkload(Workload):
    """A step is one bar for every series (the reference trains recurrent layers bar by bar); a sample
    is one series over the full 240-bar window, so samples/step = series / 240."""

    key = "lstm_stack"
    name = "lstm_stack_in64_h256_x2_seq240"
    default_batch = 1024
    default_steps = 5760  # 24 windows of 240 bars, about 1.15 s timed

    def __init__(self, batch):
        super().__init__(batch)
        from nn_in_trading_b200 import configs as C
        self.C, self.spec = C, C.LSTMSpec(series=batch)

    def samples_per_step(self):
        return self.B / self.spec.seq

    def build(self, ctx, dp):
        return self.C.build_lstm(ctx, self.spec, self.C.lstm_weights(self.spec), dp=dp)

    def data(self, pool, seed):
        d = self.C.lstm_data(self.spec, steps=pool, seed=seed)
        return d[:-1].reshape(pool, -1), d[1:].reshape(pool, -1)

    def config(self, world):
        s = self.spec
        return {"workload": self.name, "global_batch": self.B * world, "per_gpu_batch": self.B,
                "seq_len": s.seq, "inputs": s.inputs, "hidden": s.hidden, "layers": s.layers,
                "sample": "one series over the 240-bar window (240 bar steps)", "parallelism": f"dp{world}",
                "l2": "no flush: the 5 MB of weights stay in L2 between bars as in any recurrent loop; "
                      "the per-bar gate and gradient tensors (4-5 MB each) are written and read once"}

    def oracle_net(self, O, K, batch):
        s = self.spec
        w = self.C.lstm_weights(s)
        layers = [O.ODense(s.inputs * batch, K.NONE, 1, 0)]
        ins = s.inputs
        for l in range(s.layers):
            L = O.OLSTM(s.hidden, ins, batch, 1)
            L.lstm_w[:] = w[f"lstm{l}"]
            layers.append(L)
            ins = s.hidden
        head = O.OConv(s.hidden, s.hidden, s.inputs, batch, 1, K.NONE, 1)
        head.conv_w[:] = w["head"]
        layers.append(head)
        return O.ONet(layers)

    def ref_data(self, pool):
        import dataclasses
        d = self.C.lstm_data(dataclasses.replace(self.spec, series=REF_LSTM_SERIES), steps=pool, seed=7)
        return d[:-1].reshape(pool, -1), d[1:].reshape(pool, -1)

    def ref_samples_per_step(self, batch):
        return batch / self.spec.seq

    def ref_sample_desc(self, n, el, backend):
        return (f"{n} bar steps of {REF_LSTM_SERIES} series (fwd+bwd+Adam of both LSTM layers and the head) "
                f"through the {backend}, {el:.1f} s; samples = series x bars / 240")


class PatchWorkload(Workload):
    """The BatchNorm layer's update is gated on its sample count, so the step runs eagerly."""

    key = "patchtst"
    name = "patchtst_32ch_512bars_p16s8_e128_h8k16_x3_ff512_h96"
    default_batch = 512
    default_steps = 15
    recordable = False

    def __init__(self, batch):
        super().__init__(batch)
        from nn_in_trading_b200 import configs as C
        self.C, self.spec = C, C.PatchSpec()

    def build(self, ctx, dp):
        return self.C.build_patch(ctx, self.spec, self.B, self.C.patch_weights(self.spec), dp=dp)

    def data(self, pool, seed):
        xs, ts = self.C.patch_data(self.spec, self.B, pool, seed=seed)
        return xs.reshape(pool, -1), ts.reshape(pool, -1)

    def config(self, world):
        s = self.spec
        return {"workload": self.name, "global_batch": self.B * world, "per_gpu_batch": self.B,
                "channels": s.channels, "bars": s.bars, "patches": s.patches, "embed": s.embed, "heads": s.heads,
                "key": s.dk, "layers": s.layers, "horizon": s.horizon,
                "sample": "one 32-channel x 512-bar window", "parallelism": f"dp{world}",
                "l2": "no flush: every step streams tens of GB of activations, far above the 126 MB L2"}

    def oracle_net(self, O, K, batch):
        s = self.spec
        w = self.C.patch_weights(s)
        P, E, Cc = s.patches, s.embed, s.channels
        inp = O.ODense(Cc * s.bars, K.NONE, batch, 0)
        norm = O.OBatchNorm(Cc * s.bars, s.norm_batch, batch)
        conv = O.OConv(s.patch, s.stride, E, P, Cc, K.NONE, batch)
        conv.conv_w[:] = w["conv"]
        enc = O.OMLMH(E, s.dk, s.heads, P, s.layers, K.NONE, batch * Cc)
        for i, ws in enumerate(w["encoder"]):
            for name, arr in ws.items():
                enc.w[i][name][0][:] = arr
        head = O.OConv(P * E, P * E, s.horizon, Cc, 1, K.NONE, batch)
        head.conv_w[:] = w["head"]
        denorm = O.ORevIN(Cc * s.horizon, norm, batch)
        return O.ONet([inp, norm, conv, enc, head, denorm])

    def ref_data(self, pool):
        xs, ts = self.C.patch_data(self.spec, 1, pool, seed=7)
        return xs.reshape(pool, -1), ts.reshape(pool, -1)

    def ref_sample_desc(self, n, el, backend):
        return f"{n} training steps of one 32x512 window (fwd+bwd+Adam) through the {backend}, {el:.1f} s"


class SACWorkload(Workload):
    """A step is one soft actor-critic update on one replay batch; a sample is one transition."""

    key = "sac"
    name = "sac_actor240x512x512x12_2critics246x512x512x1_tau0.005"
    default_batch = 4096
    default_steps = 800  # about 1.07 s timed

    def __init__(self, batch):
        super().__init__(batch)
        from nn_in_trading_b200 import sac as S
        self.S, self.spec = S, S.SACSpec()

    def build(self, ctx, dp):
        return self.S.SACAgent(ctx, self.spec, self.B, self.S.sac_weights(self.spec), dp=dp)

    def slots(self, pool, seed):
        d = self.S.sac_data(self.spec, self.B, pool, seed=seed)
        return [d[k] for k in self.S.SACAgent.INPUTS]

    def io(self, obj):
        return [getattr(obj, k) for k in obj.INPUTS], obj.critics[0][-1].output, self.B

    def host_metric(self, y, slots, i):
        return "mean_q_last", float(np.mean(y))

    def ops(self, obj):
        return [op for ops, _ in obj.phases for op in ops]

    def config(self, world):
        s = self.spec
        return {"workload": self.name, "global_batch": self.B * world, "per_gpu_batch": self.B,
                "state": s.state, "action": s.action, "hidden": s.hidden, "tau": s.tau, "gamma": s.gamma,
                "alpha": s.alpha, "sample": "one replay transition (critic, actor and target updates)",
                "parallelism": f"dp{world}",
                "l2": "no flush: the weights (6.3 MB with moments) stay in L2 across phases as in any "
                      "training loop; the 4096-row activations (8 MB per 512-wide layer) are streamed"}

    def oracle_net(self, O, K, batch):
        return _OracleSAC(O, self.spec, batch, self.S.sac_weights(self.spec))

    def ref_data(self, pool):
        d = self.S.sac_data(self.spec, 1, pool, seed=7)
        return [{k: v[i] for k, v in d.items()} for i in range(pool)], None

    def ref_sample_desc(self, n, el, backend):
        return (f"{n} SAC updates of one transition (actor, 2 critics, 2 targets) through the {backend}, "
                f"{el:.1f} s")


class _OracleSAC:
    """The oracle SAC agent behind the ONet step(x, target) call shape of reference_sample."""

    def __init__(self, O, spec, batch, weights):
        self.agent = O.OSACAgent(spec, batch, weights)

    def step(self, batch, _target):
        self.agent.step(batch)


REF_LSTM_SERIES = 4
REF_CAP_SECONDS = 90.0  # the reference arm stops after K steps or this long, whichever comes first
WORKLOADS = {w.key: w for w in (MLMHWorkload, DenseWorkload, LSTMWorkload, PatchWorkload, SACWorkload)}


# ------------------------------------------------------------- our arm
def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    from nn_in_trading_b200 import Context

    ctx = Context(local_rank)
    torch.cuda.set_device(local_rank)
    wl = WORKLOADS[args.workload](args.batch)
    net = wl.build(ctx, world > 1)
    if world > 1:
        from nn_in_trading_b200 import dp
        dp.join_dp(ctx, rank, world)

    pool = 4
    slots = wl.slots(pool, 100 + rank)
    inputs, out_h, n_y = wl.io(net)
    sizes = [int(sl.shape[1]) for sl in slots]
    resident = [[ctx.buffer(n) for _ in range(pool)] for n in sizes]
    for sl, res in zip(slots, resident):
        for i in range(pool):
            ctx.write(res[i], sl[i])

    def load(i):
        for h, res, n in zip(inputs, resident, sizes):
            ctx.copy(h, res[i % pool], n)

    if wl.recordable:
        net.capture()
    stream = torch.cuda.ExternalStream(ctx.stream(), device=local_rank)

    def barrier():
        if world > 1:
            dist.barrier()

    for i in range(args.warmup):
        load(i)
        net.step()
    ctx.finish()
    barrier()
    l0 = ctx.launch_count()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clocks:
        time.sleep(0.25)
        torch.cuda.synchronize()
        barrier()
        ev0.record(stream)
        for i in range(args.steps):
            load(i)
            net.step()
        ev1.record(stream)
        ev1.synchronize()
        barrier()
        time.sleep(0.1)
    launches = ctx.launch_count() - l0
    ms = ev0.elapsed_time(ev1)
    ms_max = ms
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_max = float(t.item())
    per_step = wl.samples_per_step()
    value = world * per_step * args.steps / (ms_max / 1000.0)

    # ---- e2e through the public API with host buffers (pinned) ----------
    # Every step: its inputs go host -> device (nn_buffer_write_async into one half of a device
    # staging double buffer, concurrent with the step in flight), a device copy into the network's
    # input buffers, the step, a device copy of the result into a staging buffer, the result
    # device -> host (nn_buffer_read_async, concurrent with the next step) and the host metric of
    # that result (CNet::backPropOCL reads the output back).  Two steps are in flight; a staging
    # half is rewritten only after the read that follows its last use has landed.
    hosts = [torch.from_numpy(np.ascontiguousarray(sl)).pin_memory() for sl in slots]
    hy = [torch.empty(n_y, dtype=torch.float32).pin_memory() for _ in range(2)]
    stage_in = [[ctx.buffer(n) for n in sizes] for _ in range(2)]
    stage_out = [ctx.buffer(n_y) for _ in range(2)]
    lib = ctx.lib
    e2e_steps = max(3, args.steps)

    def enqueue(i):
        half = i % 2
        for st, host, n in zip(stage_in[half], hosts, sizes):
            ctx._check(lib.nn_buffer_write_async(st, host[i % pool].data_ptr(), 0, n))
        for h, st, n in zip(inputs, stage_in[half], sizes):
            ctx.copy(h, st, n)
        net.step()
        ctx.copy(stage_out[half], out_h, n_y)
        ticket = lib.nn_buffer_read_async(stage_out[half], hy[half].data_ptr(), 0, n_y)
        if ticket < 0:
            ctx._check(ticket)
        return ticket

    def run_e2e(n):
        tickets = {0: enqueue(0)}
        if n > 1:
            tickets[1] = enqueue(1)
        metric = (None, None)
        for i in range(n):
            ctx._check(lib.nn_transfer_wait(tickets.pop(i)))
            metric = wl.host_metric(hy[i % 2].numpy(), slots, i % pool)
            if i + 2 < n:
                tickets[i + 2] = enqueue(i + 2)
        return metric

    run_e2e(2)
    ctx.finish()
    barrier()
    t0 = time.perf_counter()
    metric = run_e2e(e2e_steps)
    e2e_s = time.perf_counter() - t0
    if world > 1:
        t = torch.tensor([e2e_s], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e = world * per_step * e2e_steps / e2e_s

    # ---- per-kernel profile pass (CUDA events between launches) --------
    prof = profile_ops(ctx, wl.ops(net), stream, load, torch)
    result = None
    if rank == 0:
        peaks = read_peaks()
        result = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": wl.config(world),
            "e2e": {"value": e2e, "unit": UNIT, "h2d_bytes_per_step": sum(sizes) * 4,
                    "d2h_bytes_per_step": n_y * 4, metric[0]: metric[1]},
            "gpu_launches": launches,
            "roofline": roofline(prof["top"], peaks, wl),
            "kernel_shares": prof["shares"],
            "clocks": clocks.summary(),
        }
    if world > 1:
        ctx.dp_shutdown()
    ctx.close()
    return result


def roofline(top, peaks, wl):
    """The dominant kernel against HBM when its algorithmic intensity is below the ridge of a 3xTF32
    tensor rate, else against that tensor rate (measured bf16 / 2 for TF32, / 3 for three MMAs)."""
    tensor_peak = peaks["bf16_tflops"] / 6.0
    ridge = tensor_peak * 1e12 / (peaks["hbm_gbs"] * 1e9)
    intensity = top["flops_per_launch"] / max(top["bytes_per_launch"], 1.0)
    traffic = None
    measured = NCU_TRAFFIC.get(wl.key, {})
    if top["name"] in measured:
        t_bytes, t_batch = measured[top["name"]]
        traffic = t_bytes * wl.B / t_batch
    if top["bytes_per_launch"] > 0 and intensity < ridge:
        return {"bound": "hbm", "kernel": top["name"], "achieved": top["gbs"], "peak": peaks["hbm_gbs"],
                "unit": "GB/s", "frac": top["gbs"] / peaks["hbm_gbs"], "traffic": traffic,
                "algorithmic_bytes_per_launch": top["bytes_per_launch"], "avg_launch_us": top["avg_us"],
                "peak_source": peaks["source"]}
    return {"bound": "tensor", "kernel": top["name"], "achieved": top["tflops"], "peak": tensor_peak,
            "unit": "TFLOP/s", "frac": top["tflops"] / tensor_peak, "traffic": traffic,
            "algorithmic_flops_per_launch": top["flops_per_launch"], "avg_launch_us": top["avg_us"],
            "peak_source": peaks["source"] + " bf16 / 6 (TF32 runs at half the bf16 rate; 3xTF32 issues three "
                                             "MMAs per fp32 product)"}


def profile_ops(ctx, ops, stream, load, torch):
    """One eager step with a CUDA event after every launch; per kernel-name time and work."""
    load(0)
    ctx.finish()
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(len(ops) + 1)]
    for _ in range(2):  # second pass is measured
        evs[0].record(stream)
        for i, op in enumerate(ops):
            op()
            evs[i + 1].record(stream)
        evs[-1].synchronize()
    per = {}
    total = 0.0
    for i, op in enumerate(ops):
        t = evs[i].elapsed_time(evs[i + 1])
        fl, by = op_work(op)
        d = per.setdefault(op.kernel.name, {"ms": 0.0, "n": 0, "bytes": 0.0, "flops": 0.0})
        d["ms"] += t
        d["n"] += 1
        d["bytes"] += by
        d["flops"] += fl
        total += t
    shares = {k: round(v["ms"] / total, 4) for k, v in sorted(per.items(), key=lambda kv: -kv[1]["ms"])}
    name, d = max(per.items(), key=lambda kv: kv[1]["ms"])
    avg_s = d["ms"] / d["n"] / 1000.0
    bpl = d["bytes"] / d["n"]
    top = {"name": name, "avg_us": avg_s * 1e6, "bytes_per_launch": bpl, "gbs": bpl / avg_s / 1e9,
           "flops_per_launch": d["flops"] / d["n"], "tflops": d["flops"] / d["n"] / avg_s / 1e12}
    return {"shares": shares, "top": top, "step_ms_eager": total}


def read_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]), "source": "measured"}
    except (OSError, KeyError, ValueError):
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


# ------------------------------------------------------ CPU baseline arm
def reference_sample(wl, seconds: float, steps: int | None = None, warmup: int = 1):
    """The reference's NeuroNet.cl kernels compiled for the host (oracle/_ref), OpenMP over all host
    cores, sequenced as the MQL5 host does, on a bounded sample of the workload (one sample per step;
    REF_LSTM_SERIES series per bar step for the LSTM stack).  Returns (samples/s, kind, cores, desc)."""
    from oracle import kernels as K
    from oracle import nets as O
    from oracle.ref import RefKernels
    kind = "reference" if RefKernels.available() else "port"
    O.use_backend("reference" if kind == "reference" else "numpy")
    batch = REF_LSTM_SERIES if isinstance(wl, LSTMWorkload) else 1
    net = wl.oracle_net(O, K, batch)
    xs, ts = wl.ref_data(4)
    if ts is None:
        ts = [None] * 4
    for i in range(warmup):
        net.step(xs[i % 4], ts[i % 4])
    n = 0
    t0 = time.perf_counter()
    while True:
        net.step(xs[n % 4], ts[n % 4])
        n += 1
        el = time.perf_counter() - t0
        if (steps is not None and (n >= steps or el >= REF_CAP_SECONDS)) or (steps is None and el >= seconds):
            break
    cores = RefKernels().max_threads() if kind == "reference" else 1
    backend = ("reference NeuroNet.cl kernels compiled for the CPU (OpenMP)" if kind == "reference"
               else "numpy port")
    return n * wl.ref_samples_per_step(batch) / el, kind, cores, wl.ref_sample_desc(n, el, backend)


def run_reference(args, rank, world):
    if rank != 0:
        return None
    wl = WORKLOADS[args.workload](args.batch)
    value, kind, cores, desc = reference_sample(wl, 0.0, steps=max(1, args.steps),
                                                warmup=max(0, min(args.warmup, 1)))
    cfg = dict(wl.config(1))
    cfg.update({"global_batch": 1, "per_gpu_batch": 1, "parallelism": "host cores"})
    return {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic", "config": cfg, "impl": "reference",
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": kind, "sample": desc},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="mlmh_encoder")
    ap.add_argument("--batch", type=int, default=None)
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    wl_cls = WORKLOADS[args.workload]
    if args.steps is None:
        args.steps = wl_cls.default_steps
    if args.batch is None:
        args.batch = wl_cls.default_batch
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3
    rank = env_int("RANK", 0)
    world = env_int("WORLD_SIZE", 1)
    local_rank = env_int("LOCAL_RANK", 0)
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=300))
    try:
        if args.impl == "reference":
            res = run_reference(args, rank, world)
        else:
            res = run_ours(args, rank, world, local_rank)
            if rank == 0 and res is not None:
                if world == 1 and not args.no_cpu_baseline:
                    v, kind, cores, desc = reference_sample(wl_cls(args.batch), args.cpu_seconds)
                    res["cpu_baseline"] = {"value": v, "unit": UNIT, "cores": cores, "kind": kind, "sample": desc}
                else:
                    res["cpu_baseline"] = None
        if rank == 0 and res is not None:
            print(json.dumps(res), flush=True)
    finally:
        if world > 1:
            import torch.distributed as dist
            if dist.is_initialized():
                dist.barrier()
                dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
