#!/usr/bin/env python
"""MoE-block tokens/s of the B200 (sm_100a) Qwen3-30B-A3B MoE FFN block.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload config2]
                    [--impl ours|reference]

A step is one MoE block call (router, top-8, dispatch, Q8_0 SwiGLU experts,
weighted combine) over one batch of synthetic tokens with seeded
random-init Q8_0 weights (motoria_b200.synth).  Default workload: config2,
batched decode of 64 tokens per GPU.  Prints ONE JSON line on rank 0.

  value      tokens/s of the whole job, inputs resident in HBM, device-timed
             (CUDA events around each step on the launching stream, L2
             flushed between steps outside the events -- a 256 MiB buffer
             written, then read back -- max over ranks)
  e2e        the same metric through the public host API (miag_moe with
             pinned host buffers: H2D of x and D2H of the result every step)
  roofline   the dominant kernel's algorithmic bytes / its mean duration,
             from CUDA events around each kernel on its stream in a second
             pass of the same steps (the timed pass carries no such events)
  cpu_baseline  the reference engine built from its sources (oracle/_ref)
             or the oracle port, on this host's cores, rank 0 at N=1
  --impl reference  times the reference CPU implementation (all host threads)
             on the same workload and prints its own line.

Multi-GPU (torchrun, N>1), scaling weak (tokens per GPU fixed):
  config5, the expert-parallel configuration: motoria_b200.ep.  Each rank
    holds E/N experts (--ep-placement contiguous, as specified, or strided)
    and routes its own tokens; (row, expert) pairs go to the experts' ranks
    and the results come back stored by the down launch straight into the
    origin rank's memory over NVLink (--ep-exchange peer, the default) or by
    NCCL all-to-all (collective); outputs equal the one-GPU block bit for bit.
  config1-3: replicas.  Every rank holds all experts and serves its own
    batch; the block is independent per token, so there is no data-path
    collective.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

from motoria_b200 import synth  # noqa: E402

SEED, XSEED = 1234, 99
METRIC = "MoE-block tokens/s"
UNIT = "tokens/s"
DTYPE = "int8 dot / f32 accumulate (Q8_0)"

WORKLOADS = {
    "config1": ("MoE block, decode of 1 token (Qwen3-30B-A3B shapes)", 1, True, False),
    "config2": ("MoE block, batched decode of 64 tokens (Qwen3-30B-A3B shapes)", 64, True, False),
    "config3": ("MoE block, prefill of 2048 tokens, Zipf-biased router", 2048, False, True),
    "config5": ("MoE block, 4096 tokens per GPU, Zipf-biased router", 4096, False, True),
}
EP_WORKLOADS = ("config5",)  # the expert-parallel configuration; the others run replicas


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


def host_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


# ---------------------------------------------------------------------------
# CPU side: the reference engine (or the oracle port) on the host cores.

def cpu_arm(shape, lay, x, seconds: float, min_steps: int = 1):
    """Runs the reference CPU block on x repeatedly for ~seconds; returns
    (tokens/s, cores, kind, steps, elapsed)."""
    from oracle import oracle as O

    O.build()
    impl = O.ref() or O.oracle()
    cores = host_cores()
    steps, t0 = 0, time.perf_counter()
    while True:
        impl.moe(shape, lay.ffn_norm, lay.router, lay.bias, lay.blobs, x, threads=cores)
        steps += 1
        el = time.perf_counter() - t0
        if steps >= min_steps and el >= seconds:
            break
    return steps * x.shape[0] / el, cores, impl.kind, steps, el


def run_reference(args, T_desc, T, rms, zipf):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    shape = synth.QWEN3_30B_A3B
    lay = synth.layer(shape, SEED, zipf=zipf)
    x = synth.tokens(shape, XSEED, T, rms_normalise=rms)
    from oracle import oracle as O

    O.build()
    impl = O.ref() or O.oracle()
    cores = host_cores()
    for _ in range(args.warmup):
        impl.moe(shape, lay.ffn_norm, lay.router, lay.bias, lay.blobs, x, threads=cores)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        impl.moe(shape, lay.ffn_norm, lay.router, lay.bias, lay.blobs, x, threads=cores)
    el = time.perf_counter() - t0
    value = args.steps * T / el
    arch = os.uname().machine
    sample = (f"{args.steps} steps x {T} tokens of {args.workload}; "
              f"{'reference built from source' if impl.kind == 'reference' else 'oracle port'}"
              f"{' (x86 scalar path: the NEON path needs an aarch64 host)' if arch == 'x86_64' else ''}")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": el / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": DTYPE, "data": "synthetic",
        "config": {"workload": f"{args.workload}: {T_desc}", "tokens_per_step": T,
                   "threads": cores},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": impl.kind,
                         "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# GPU side.

class ClockSampler:
    """nvidia-smi clock/throttle samples during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "25"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc:
            time.sleep(0.15)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.out = out
        else:
            self.out = ""

    def summary(self):
        rows = [r.split(", ") for r in self.out.strip().splitlines() if r.count(",") >= 8]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm = [float(r[1]) for r in rows]
        mx = max(float(r[2]) for r in rows)
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].strip() == "Active"})
        loaded = [v for v in sm if v >= 0.5 * mx] or sm
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": mx, "reasons": reasons,
                "samples": len(rows)}


def stage_bytes(shape, T, counts, rows=None, pairs=None):
    """Algorithmic HBM bytes per launch of each stage (weights streamed once
    per active expert; activations read/written once).  T tokens are routed
    and combined here; the expert kernels see `pairs` pairs over `rows`
    activation rows (T*K and T on one GPU; what arrived, under expert
    parallelism)."""
    d, eh, E, K = shape.dim, shape.expert_hidden, shape.n_experts, shape.n_active
    P = T * K if pairs is None else pairs
    R = T if rows is None else rows
    n_act = int((counts > 0).sum())
    gu_w = 2 * eh * (d + d // 32 * 4)    # gate + up: int8 rows + f32 block scales
    dn_w = d * (eh + eh // 32 * 4)
    return {
        "route": E * d * 4 + T * d * 4 + T * (d + d // 8) + T * K * 8,
        "permute": P * 4 * 6 + E * 16,
        "gateup": n_act * gu_w + R * (d + d // 8) + P * eh * 4,
        "down": n_act * dn_w + P * eh * 4 + P * d * 4,
        "combine": T * K * d * 4 + 2 * T * d * 4 + T * K * 8,
    }, n_act


def ncu_traffic(workload: str, kernel: str):
    """DRAM bytes (read + write) per launch of `kernel` from the committed ncu
    summary of this workload (profiles/*.md, a `traffic:` marker), or None."""
    import re

    pat = re.compile(r"<!-- traffic: workload=(\S+) kernel=(\S+) bytes=(\d+) -->")
    for f in sorted((ROOT / "profiles").glob("*.md")):
        for w, k, n in pat.findall(f.read_text()):
            if w == workload and k == kernel:
                return int(n)
    return None


def run_ours(args, T_desc, T, rms, zipf):
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(local)

    from motoria_b200 import MoEEngine, build

    build.build()
    shape = synth.QWEN3_30B_A3B
    lay = synth.layer(shape, SEED, zipf=zipf)
    x_host = synth.tokens(shape, XSEED + 1000 * rank, T, rms_normalise=rms)
    eng = MoEEngine(shape, n_layers=1, device=local)
    ep = None
    if world > 1 and args.workload in EP_WORKLOADS:
        # expert parallelism: this rank holds E/N experts (placement below)
        from motoria_b200.ep import EngineOps, ExpertParallelMoE

        ep = ExpertParallelMoE(EngineOps(eng), placement=args.ep_placement,
                               exchange=args.ep_exchange)
        eng.set_layer(0, lay.ffn_norm, lay.router, lay.bias)
        for e in ep.experts_of(rank):
            eng.upload_experts(0, lay.blobs[e:e + 1], first=e)
    else:  # one GPU, or replicas: every rank holds all experts and serves its own batch
        eng.load_layer(0, lay)

    dev = torch.device("cuda", local)
    x0 = torch.from_numpy(x_host).to(dev)
    x = x0.clone()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)  # > 126 MB L2
    # A dedicated stream: the kernels, the restore/flush copies and the timing
    # events all go to it (a NULL handle would mean the library's own stream).
    stream = torch.cuda.Stream(dev)
    torch.cuda.set_stream(stream)
    sp = stream.cuda_stream

    def barrier():
        torch.cuda.synchronize(dev)
        if dist:
            dist.barrier()
            torch.cuda.synchronize(dev)

    flush_sink = torch.zeros((), dtype=torch.int64, device=dev)

    def one_step(ev=None):
        x.copy_(x0)
        # write a buffer larger than L2, then read it: the L2 holds none of the
        # step's data and no dirty lines whose write-back the step would pay
        flush.zero_()
        flush_sink.add_(flush.sum())
        if ev:
            ev[0].record(stream)
        if ep:
            ep.forward(x)
        else:
            eng.moe_device(x.data_ptr(), T, stream=sp)
        if ev:
            ev[1].record(stream)

    for _ in range(args.warmup):
        one_step()
    eng.sync(sp)
    if ep:
        R_in, P_in, pe = ep.last_received
        counts = torch.bincount(pe.long(), minlength=shape.n_experts).cpu().numpy()
        per_stage_bytes, n_act = stage_bytes(shape, T, counts, rows=R_in, pairs=P_in)
    else:
        routing = eng.routing(T)
        per_stage_bytes, n_act = stage_bytes(shape, T, routing["counts"])

    events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(args.steps)]
    barrier()
    with ClockSampler(local) as clk:
        for i in range(args.steps):
            one_step(events[i])
        barrier()
    eng.sync(sp)
    total_ms = sum(a.elapsed_time(b) for a, b in events)
    # Per-kernel durations: the same steps again, each kernel bracketed by
    # CUDA events on the stream it is launched on (kept out of the timed pass
    # above so the brackets do not stretch the step).
    eng.profile(True)
    eng.profile_read()
    for i in range(args.steps):
        one_step()
    eng.sync(sp)
    prof = eng.profile_read()
    eng.profile(False)
    prof = {k: v for k, v in prof.items() if v[1] > 0}  # stages that launched something
    launches_per_step = sum(v[1] for v in prof.values()) // args.steps
    t = torch.tensor([total_ms], dtype=torch.float64, device=dev)
    if dist:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms = float(t.item())
    value = world * T * args.steps / (total_ms / 1e3)

    # e2e: the public host API, pinned host buffers, H2D + D2H every step.
    # Each step's input sits in its own pinned buffer, written before the
    # timed region (the block updates its input in place); up to 1 GiB of
    # them, past which a buffer is rewritten inside the step.
    n_e2e = args.warmup + args.steps
    nbuf = max(1, min(n_e2e, (1 << 30) // max(1, x_host.nbytes)))
    bufs = [torch.empty((T, shape.dim), dtype=torch.float32, pin_memory=True) for _ in range(nbuf)]
    for b in bufs:
        b.numpy()[:] = x_host
    e2e_i = [0]

    def e2e_step():
        xp = bufs[e2e_i[0] % nbuf]
        xp_np = xp.numpy()
        if e2e_i[0] >= nbuf:
            xp_np[:] = x_host
        e2e_i[0] += 1
        if ep:  # H2D, the sharded block, D2H, on this rank's stream
            x.copy_(xp, non_blocking=True)
            ep.forward(x)
            xp.copy_(x, non_blocking=True)
            stream.synchronize()
        else:
            eng.moe_inplace(xp_np)

    for _ in range(args.warmup):
        e2e_step()
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        e2e_step()
    e2e_s = time.perf_counter() - t0
    te = torch.tensor([e2e_s], dtype=torch.float64, device=dev)
    if dist:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_s = float(te.item())
    e2e_value = world * T * args.steps / e2e_s

    hbm_gbs, tflops, peak_kind = load_peaks()
    stage_ms = {k: v[0] / args.steps for k, v in prof.items()}  # mean ms per step
    top = max((k for k in stage_ms if k in per_stage_bytes), key=stage_ms.get)
    achieved = per_stage_bytes[top] / (stage_ms[top] / 1e3) / 1e9
    block_bytes = sum(per_stage_bytes.values())

    line = None
    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            v, cores, kind, steps, el = cpu_arm(shape, lay, x_host, args.cpu_seconds)
            cpu = {"value": v, "unit": UNIT, "cores": cores, "kind": kind,
                   "sample": f"{steps} x {T} tokens of {args.workload} ({el:.1f} s on "
                             f"{cores} threads, {os.uname().machine})"}
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": total_ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": DTYPE,
            "data": "synthetic (seeded random-init Q8_0 weights and N(0,1) tokens)",
            "config": {"workload": f"{args.workload}: {T_desc}", "tokens_per_gpu": T,
                       "experts": shape.n_experts, "top_k": shape.n_active, "dim": shape.dim,
                       "expert_hidden": shape.expert_hidden, "active_experts": n_act,
                       "weights": "Q8_0 HBM-resident",
                       "l2": "flushed between steps outside the timed events (256 MiB written, then read back)",
                       "parallelism": (f"ep{world} ({args.ep_placement}, y back by "
                                       f"{'peer stores' if args.ep_exchange == 'peer' else 'all-to-all'})"
                                       if ep else
                                       "replicas" if world > 1 else "single"),
                       "experts_per_gpu": shape.n_experts // world if ep else shape.n_experts},
            "e2e": {"value": e2e_value, "unit": UNIT,
                    "h2d_bytes_per_step": T * shape.dim * 4,
                    "d2h_bytes_per_step": T * shape.dim * 4,
                    "inputs": ("each step's own pinned buffer, written before the timed region"
                               if nbuf >= n_e2e else
                               f"{nbuf} pinned buffers written before the timed region, "
                               "rewritten in the step past them")},
            "roofline": {"bound": "hbm", "kernel": top, "achieved": achieved, "peak": hbm_gbs,
                         "unit": "GB/s", "frac": achieved / hbm_gbs,
                         "traffic": ncu_traffic(args.workload, top),
                         "peak_source": f"{peak_kind} hbm_gbs",
                         "block_achieved_gbs": block_bytes / (total_ms / args.steps / 1e3) / 1e9},
            "stages_ms": {k: round(v, 5) for k, v in stage_ms.items()},
            "gpu_launches": launches_per_step * args.steps,
            "cpu_baseline": cpu,
            "clocks": clk.summary(),
        }
        print(json.dumps(line), flush=True)
    eng.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return line


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="config2")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--ep-placement", choices=["contiguous", "strided"], default="contiguous",
                    help="expert placement of the expert-parallel run (config5, N>1)")
    ap.add_argument("--ep-exchange", choices=["peer", "collective"], default="peer",
                    help="how the expert results return (config5, N>1): stored by the down "
                         "launch into the origin rank's memory over NVLink, or NCCL all-to-all")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    desc, T, rms, zipf = WORKLOADS[args.workload]
    if args.impl == "reference":
        run_reference(args, desc, T, rms, zipf)
    else:
        run_ours(args, desc, T, rms, zipf)


if __name__ == "__main__":
    main()
