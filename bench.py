"""Benchmark: fwd+bwd+Adam training throughput of the attention encoder (samples/s).

Workload: CNeuronMLMHAttentionOCL encoder, 4 layers, 120 bars x 64 features, 8 heads x key 32,
FF 64->256(GELU)->64(LReLU), batch 256 independent sequences per GPU, fp32, MSE vs N(0,1)
targets, Adam; synthetic seeded N(0,1) data.  A step = forward + backward + Adam of one batch,
replayed from command lists through libnn_b200.so.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--batch B]

N > 1 (torchrun, one process per GPU): weak scaling, every rank trains its own 256 sequences and
the weight gradients are averaged with one NCCL allreduce per step before the updates.
`--impl reference` times the reference's own NeuroNet.cl kernels compiled for the host CPU
(oracle/_ref) on the same workload, one sequence per step, on rank 0 only.
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

WORKLOAD = "mlmh_encoder_4x120x64_h8k32_ff256"
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
# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one launch, from one ncu capture
# of the batch-256 workload:  ncu --set full --clock-control none -k regex:attn_grad -s 4 -c 1
#   python bench.py --steps 3 --warmup 3 --no-cpu-baseline
# Keyed by the reference kernel; scaled to other batches by the sequences a launch processes.
NCU_TRAFFIC = {"MHAttentionInsideGradients": (311.70e6, 256)}


def op_work(op, B):
    """(flops, bytes) a launch must do at minimum: every operand read once, every result written once."""
    k = op.kernel
    name = k.name
    a = k.values
    g = op.gsize
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
    return 0.0, 0.0


# ------------------------------------------------------------- our arm
def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    from nn_in_trading_b200 import Context
    from nn_in_trading_b200 import configs as C

    ctx = Context(local_rank)
    torch.cuda.set_device(local_rank)
    spec = C.MLMHSpec()
    B = args.batch
    net = C.build_mlmh(ctx, spec, B, C.mlmh_weights(spec), dp=world > 1)
    if world > 1:
        from nn_in_trading_b200 import dp
        dp.join_dp(ctx, rank, world)

    n_in = spec.window * spec.units
    pool = 4
    xs, ts = C.mlmh_data(spec, B, pool, seed=100 + rank)
    resident_x = [ctx.buffer(B * n_in) for _ in range(pool)]
    resident_t = [ctx.buffer(B * n_in) for _ in range(pool)]
    for i in range(pool):
        ctx.write(resident_x[i], xs[i])
        ctx.write(resident_t[i], ts[i])
    inp = net.layers[0].output

    def load(i):
        ctx.copy(inp, resident_x[i % pool], B * n_in)
        ctx.copy(net.target, resident_t[i % pool], B * n_in)

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
    value = world * B * args.steps / (ms_max / 1000.0)

    # ---- e2e through the public API with host buffers (pinned) ----------
    hx = torch.from_numpy(xs.reshape(pool, -1)).pin_memory()
    ht = torch.from_numpy(ts.reshape(pool, -1)).pin_memory()
    hy = torch.empty(B * n_in, dtype=torch.float32).pin_memory()
    lib = ctx.lib
    out_h = net.layers[-1].output
    e2e_steps = max(3, args.steps // 2)
    for i in range(2):
        lib.nn_buffer_write(inp, hx[i % pool].data_ptr(), 0, B * n_in)
        lib.nn_buffer_write(net.target, ht[i % pool].data_ptr(), 0, B * n_in)
        net.step()
        lib.nn_buffer_read(out_h, hy.data_ptr(), 0, B * n_in)
    barrier()
    # Every step: H2D of its inputs and targets, the step, a blocking D2H of its output and the host
    # MSE of that output (CNet::backPropOCL reads the output back).  The host work of step i runs
    # while the device already executes step i+1 (enqueued right after step i's read returns).
    t0 = time.perf_counter()
    losses = []

    def enqueue(i):
        ctx._check(lib.nn_buffer_write(inp, hx[i % pool].data_ptr(), 0, B * n_in))
        ctx._check(lib.nn_buffer_write(net.target, ht[i % pool].data_ptr(), 0, B * n_in))
        net.step()

    enqueue(0)
    for i in range(e2e_steps):
        ctx._check(lib.nn_buffer_read(out_h, hy.data_ptr(), 0, B * n_in))
        if i + 1 < e2e_steps:
            enqueue(i + 1)  # hy is written again only by the next iteration's read
        d = hy.numpy() - ts[i % pool].reshape(-1)
        losses.append(float(np.dot(d, d)) / d.size)  # host MSE of step i's output
    e2e_s = time.perf_counter() - t0
    if world > 1:
        t = torch.tensor([e2e_s], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e = world * B * e2e_steps / e2e_s

    # ---- per-kernel profile pass (CUDA events between launches) --------
    prof = profile_ops(ctx, net, stream, B, load, torch)
    result = None
    if rank == 0:
        peaks = read_peaks()
        top = prof["top"]
        roof = {"bound": "hbm", "kernel": top["name"], "achieved": top["gbs"], "peak": peaks["hbm_gbs"],
                "unit": "GB/s", "frac": top["gbs"] / peaks["hbm_gbs"],
                "traffic": (NCU_TRAFFIC[top["name"]][0] * B / NCU_TRAFFIC[top["name"]][1]
                            if top["name"] in NCU_TRAFFIC else None),
                "algorithmic_bytes_per_launch": top["bytes_per_launch"],
                "avg_launch_us": top["avg_us"], "peak_source": peaks["source"]}
        result = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": WORKLOAD, "global_batch": B * world, "per_gpu_batch": B, "seq_len": spec.units,
                       "embed": spec.window, "heads": spec.heads, "key": spec.dk, "layers": spec.layers,
                       "parallelism": f"dp{world}",
                       "l2": "no flush: every step streams >1 GB of activations and scores, well above the 126 MB L2"},
            "e2e": {"value": e2e, "unit": UNIT, "h2d_bytes_per_step": 2 * B * n_in * 4,
                    "d2h_bytes_per_step": B * n_in * 4, "mse_last": losses[-1]},
            "gpu_launches": launches,
            "roofline": roof,
            "kernel_shares": prof["shares"],
            "clocks": clocks.summary(),
        }
    if world > 1:
        ctx.dp_shutdown()
    ctx.close()
    return result


def profile_ops(ctx, net, stream, B, load, torch):
    """One eager step with a CUDA event after every launch; per kernel-name time and work."""
    ops = net.fwd_ops + net.bwd_ops + net.upd_ops
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
        fl, by = op_work(op, B)
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
           "tflops": d["flops"] / d["n"] / avg_s / 1e12}
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
def reference_sample(seconds: float, steps: int | None = None, warmup: int = 1):
    """The reference's NeuroNet.cl kernels compiled for the host (oracle/_ref), OpenMP over all host
    cores, sequenced as the MQL5 host does for the encoder, one sequence per training step.
    Returns (samples/s, kind, cores, description)."""
    from nn_in_trading_b200 import configs as C
    from oracle import kernels as K
    from oracle import nets as O
    from oracle.ref import RefKernels
    kind = "reference" if RefKernels.available() else "port"
    O.use_backend("reference" if kind == "reference" else "numpy")
    spec = C.MLMHSpec()
    inp = O.ODense(spec.window * spec.units, K.NONE, 1, 0)
    enc = O.OMLMH(spec.window, spec.dk, spec.heads, spec.units, spec.layers, spec.activation, 1)
    for i, ws in enumerate(C.mlmh_weights(spec)):
        for name, w in ws.items():
            enc.w[i][name][0][:] = w
    net = O.ONet([inp, enc])
    xs, ts = C.mlmh_data(spec, 1, 4, seed=7)
    for i in range(warmup):
        net.step(xs[i % 4], ts[i % 4])
    n = 0
    t0 = time.perf_counter()
    while True:
        net.step(xs[n % 4], ts[n % 4])
        n += 1
        el = time.perf_counter() - t0
        if (steps is not None and n >= steps) or (steps is None and el >= seconds):
            break
    cores = RefKernels().max_threads() if kind == "reference" else 1
    desc = (f"{n} training steps of one 120x64 sequence (fwd+bwd+Adam of all 4 layers) through the "
            f"{'reference NeuroNet.cl kernels compiled for the CPU (OpenMP)' if kind == 'reference' else 'numpy port'}"
            f", {el:.1f} s")
    return n / el, kind, cores, desc


def run_reference(args, rank, world):
    if rank != 0:
        return None
    value, kind, cores, desc = reference_sample(0.0, steps=max(1, args.steps), warmup=max(0, min(args.warmup, 1)))
    spec_cfg = {"workload": WORKLOAD, "global_batch": 1, "per_gpu_batch": 1, "seq_len": 120, "embed": 64,
                "heads": 8, "key": 32, "layers": 4, "parallelism": "host cores"}
    return {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic", "config": spec_cfg, "impl": "reference",
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": kind, "sample": desc},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--batch", type=int, default=256)
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
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
                    v, kind, cores, desc = reference_sample(args.cpu_seconds)
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
