#!/usr/bin/env python
"""MoE-block tokens/s of the B200 (sm_100a) Qwen3-30B-A3B MoE FFN block.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload config5]
                    [--impl ours|reference]

A step is one MoE block call (router, top-8, dispatch, Q8_0 SwiGLU experts,
weighted combine) over one batch of synthetic tokens with seeded
random-init Q8_0 weights (motoria_b200.synth).  Prints ONE JSON line on
rank 0.

Default workload: config5, 4096 tokens per GPU with the Zipf-biased router
(the largest single-GPU configuration, and the expert-parallel one):
  N = 1   one GPU holds all 128 experts;
  N > 1   expert parallelism (motoria_b200.ep): rank g holds experts
          [g*128/N, (g+1)*128/N) (contiguous, as specified); each rank routes
          its own tokens, (row, expert) pairs go to the experts' ranks over
          NCCL, and the down launch stores each result straight into the
          origin rank's memory over NVLink -- all inside libmiag
          (miag_moe_ep_async).  Outputs equal the one-GPU block bit for bit.  The strided placement (expert e on rank e mod N) is
          reported beside it under "ep_strided".
Scaling is weak: tokens per GPU are fixed as N grows.

  value      tokens/s of the whole job, inputs resident in HBM, device-timed
             (CUDA events around each step on the launching stream, L2
             flushed between steps outside the events -- a 256 MiB buffer
             written, then read back -- max over ranks)
  e2e        the same metric through the public host API with pinned host
             buffers, H2D of x and D2H of the result every step (N = 1:
             miag_moe; N > 1: H2D, the sharded block, D2H on each rank);
             "e2e_pageable" repeats it from ordinary (malloc'd) host memory,
             as the reference engine's own buffers are
  roofline   the dominant kernel, from CUDA events around each kernel on its
             stream in a second pass of the same steps (the timed pass has
             none).  Prefill-size batches (config3, config5): tensor FLOP/s of
             the expert products against the measured bf16 peak, and the
             FP32 operations of the reference's exact Q8_0 steps against the
             chip's FP32 lane rate ("epilogue"); decode: HBM bytes/s against
             the measured copy bandwidth
  decode     (N = 1) config2 (64 tokens) and config1 (1 token) measured the
             same way: value, e2e and the HBM roofline
  cpu_baseline  the reference engine built from its sources (oracle/_ref)
             or the oracle port, on this host's cores, rank 0 at N = 1, on a
             bounded sample of the workload's tokens
  --impl reference  times the reference CPU implementation (all host threads)
             on a bounded sample of the same workload and prints its own line.
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

# name: (description, tokens per GPU, RMS-normalised inputs, Zipf-biased router)
WORKLOADS = {
    "config1": ("MoE block, decode of 1 token (Qwen3-30B-A3B shapes)", 1, True, False),
    "config2": ("MoE block, batched decode of 64 tokens (Qwen3-30B-A3B shapes)", 64, True, False),
    "config3": ("MoE block, prefill of 2048 tokens, Zipf-biased router", 2048, False, True),
    "config5": ("MoE block, 4096 tokens per GPU, Zipf-biased router; expert-parallel over "
                "the GPUs when N > 1", 4096, False, True),
}
DEFAULT_WORKLOAD = "config5"
EP_WORKLOADS = ("config5",)       # expert-parallel at N > 1; the others run replicas
PREFILL_WORKLOADS = ("config3", "config5")
DECODE_EXTRAS = ("config2", "config1")
CPU_SAMPLE_TOKENS = 512           # reference-arm tokens per step for the big batches


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16": float(d["bf16_tflops"]),
                "bf16_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])),
                "sm_max_mhz": float(d.get("sm_max_mhz", 1965.0)), "kind": "measured"}
    return {"hbm_gbs": 6650.0, "bf16": 1590.0, "bf16_sustained": 1400.0, "sm_max_mhz": 1965.0,
            "kind": "fallback"}


def host_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_sample(T: int) -> int:
    return min(T, CPU_SAMPLE_TOKENS)


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
    Ts = cpu_sample(T)
    x = synth.tokens(shape, XSEED, T, rms_normalise=rms)[:Ts]
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
    value = args.steps * Ts / el
    arch = os.uname().machine
    sample = (f"{args.steps} steps x {Ts} tokens"
              f"{f' (the first {Ts} of the {T} tokens a GPU holds)' if Ts < T else ''}"
              f" of {args.workload} on {cores} threads; "
              f"{'reference built from source' if impl.kind == 'reference' else 'oracle port'}"
              f"{' (x86 scalar path: the NEON path needs an aarch64 host)' if arch == 'x86_64' else ''}")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": el / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": DTYPE, "data": "synthetic",
        "config": {"workload": f"{args.workload}: {T_desc}", "tokens_per_step": Ts,
                   "tokens_per_gpu": T, "threads": cores},
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
        self.out = ""

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


def stage_work(shape, T, counts, rows=None, pairs=None):
    """Algorithmic work per launch of each stage: HBM bytes (weights streamed
    once per active expert; activations read/written once), tensor FLOPs of
    the expert products, and the FP32 operations of the reference's exact
    Q8_0 steps (four per row, pair and 32-block: the exact int-to-float, two
    rounded products, a rounded add).  T tokens are routed and combined
    here; the expert kernels see `pairs` pairs over `rows` activation rows
    (T*K and T on one GPU; what arrived, under expert parallelism)."""
    d, eh, E, K = shape.dim, shape.expert_hidden, shape.n_experts, shape.n_active
    P = T * K if pairs is None else pairs
    R = T if rows is None else rows
    n_act = int((counts > 0).sum())
    gu_w = 2 * eh * (d + d // 32 * 4)    # gate + up: int8 rows + f32 block scales
    dn_w = d * (eh + eh // 32 * 4)
    nbytes = {
        "route": E * d * 4 + T * d * 4 + T * (d + d // 8) + T * K * 8,
        "permute": P * 4 * 6 + E * 16,
        "gateup": n_act * gu_w + R * (d + d // 8) + P * 2 * eh * 4,
        "down": n_act * dn_w + P * 2 * eh * 4 + P * d * 4,
        "combine": T * K * d * 4 + 2 * T * d * 4 + T * K * 8,
        # tcgen05 prefill only: the activations laid out as pair tiles
        "gather": P * (d + d // 8) * 2,
        "swiglu": P * 2 * eh * 4 + P * (eh + eh // 8),
    }
    flops = {"gateup": 2.0 * P * 2 * eh * d, "down": 2.0 * P * d * eh}
    fp32_ops = {"gateup": 4.0 * P * 2 * eh * (d // 32), "down": 4.0 * P * d * (eh // 32)}
    return nbytes, flops, fp32_ops, n_act


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


class Ctx:
    """Process-wide GPU plumbing of one bench run (torch as plumbing only)."""

    def __init__(self):
        import torch

        self.torch = torch
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(self.local)
        self.dist = None
        if self.world > 1:
            import datetime

            import torch.distributed as dist

            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                    device_id=torch.device("cuda", self.local))
            self.dist = dist
        self.dev = torch.device("cuda", self.local)
        self.flush = torch.empty(256 << 20, dtype=torch.uint8, device=self.dev)  # > 126 MB L2
        self.flush_sink = torch.zeros((), dtype=torch.int64, device=self.dev)
        # A dedicated stream: the kernels, the restore/flush copies and the
        # timing events all go to it (a NULL handle would mean the library's
        # own stream).
        self.stream = torch.cuda.Stream(self.dev)
        torch.cuda.set_stream(self.stream)
        self.num_sms = torch.cuda.get_device_properties(self.dev).multi_processor_count
        self.closers = []  # expert-parallel blocks and communicators, closed before the engines

    def barrier(self):
        self.torch.cuda.synchronize(self.dev)
        if self.dist:
            self.dist.barrier()
            self.torch.cuda.synchronize(self.dev)

    def max_over_ranks(self, v: float) -> float:
        t = self.torch.tensor([v], dtype=self.torch.float64, device=self.dev)
        if self.dist:
            self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def flush_l2(self):
        # write a buffer larger than L2, then read it: the L2 holds none of
        # the step's data and no dirty lines whose write-back the step would pay
        self.flush.zero_()
        self.flush_sink.add_(self.flush.sum())


class SingleRunner:
    """One GPU holding every expert (or a replica): miag_moe_async on the
    device, miag_moe through host buffers."""

    def __init__(self, eng, layer: int):
        self.eng, self.layer = eng, layer

    def device(self, x, sp):
        self.eng.moe_device(x.data_ptr(), x.shape[0], layer=self.layer, stream=sp)

    def host(self, xp_np, x, stream):
        self.eng.moe_inplace(xp_np, layer=self.layer)

    def received(self):
        return None


class EPRunner:
    """libmiag's expert-parallel block (miag_moe_ep_async / miag_moe_ep):
    NCCL, dispatch, the expert products and the peer-memory return all run
    inside the library."""

    def __init__(self, block, eng):
        self.block, self.eng = block, eng

    def device(self, x, sp):
        self.block.forward_device(x.data_ptr(), x.shape[0], stream=sp)

    def host(self, xp_np, x, stream):
        self.block.forward_host(xp_np)

    def received(self):
        return self.block.last_received()


def measure(ctx: Ctx, runner, x_host, steps: int, warmup: int, e2e: bool = True,
            pageable: bool = False, clocks: bool = False):
    """Times `steps` block steps after `warmup` untimed ones.  Returns a dict:
    total_ms (max over ranks), per-stage mean ms and launches of this rank,
    e2e seconds (max over ranks) and the clock summary."""
    torch, dev, stream = ctx.torch, ctx.dev, ctx.stream
    sp = stream.cuda_stream
    T = x_host.shape[0]
    x0 = torch.from_numpy(x_host).to(dev)
    x = x0.clone()

    def one_step(ev=None):
        x.copy_(x0)
        ctx.flush_l2()
        if ev:
            ev[0].record(stream)
        runner.device(x, sp)
        if ev:
            ev[1].record(stream)

    for _ in range(warmup):
        one_step()
    runner.eng.sync(sp)
    events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(steps)]
    ctx.barrier()
    clk = ClockSampler(ctx.local) if clocks else None
    if clk:
        clk.__enter__()
    for i in range(steps):
        one_step(events[i])
    ctx.barrier()
    if clk:
        clk.__exit__(None, None, None)
    runner.eng.sync(sp)
    total_ms = sum(a.elapsed_time(b) for a, b in events)
    # Per-kernel durations: the same steps again, each kernel bracketed by
    # CUDA events on the stream it is launched on.
    runner.eng.profile(True)
    runner.eng.profile_read()
    for _ in range(steps):
        one_step()
    runner.eng.sync(sp)
    prof = runner.eng.profile_read()
    runner.eng.profile(False)
    prof = {k: v for k, v in prof.items() if v[1] > 0}
    out = {"total_ms": ctx.max_over_ranks(total_ms),
           "stage_ms": {k: v[0] / steps for k, v in prof.items()},
           "launches_per_step": sum(v[1] for v in prof.values()) // steps,
           "received": runner.received(),
           "clocks": clk.summary() if clk else None}
    if not e2e:
        return out

    # e2e: the public host API, pinned host buffers, H2D + D2H every step.
    # Each step's input sits in its own host buffer, written before the timed
    # region (the block updates its input in place); up to 1 GiB of them,
    # past which a buffer is rewritten inside the step.
    def e2e_pass(pinned: bool):
        n_e2e = warmup + steps
        nbuf = max(1, min(n_e2e, (1 << 30) // max(1, x_host.nbytes)))
        if pinned:
            bufs = [torch.empty(x_host.shape, dtype=torch.float32, pin_memory=True)
                    for _ in range(nbuf)]
            arrs = [b.numpy() for b in bufs]
            runner._pinned = {id(a): b for a, b in zip(arrs, bufs)}
        else:
            arrs = [np.empty(x_host.shape, np.float32) for _ in range(nbuf)]
            runner._pinned = {id(a): torch.from_numpy(a) for a in arrs}
        for a in arrs:
            a[:] = x_host
        i = [0]

        def step():
            a = arrs[i[0] % nbuf]
            if i[0] >= nbuf:
                a[:] = x_host
            i[0] += 1
            runner.host(a, x, stream)

        for _ in range(warmup):
            step()
        ctx.barrier()
        t0 = time.perf_counter()
        for _ in range(steps):
            step()
        el = time.perf_counter() - t0
        return ctx.max_over_ranks(el), nbuf >= n_e2e

    out["e2e_s"], out["e2e_own_buffers"] = e2e_pass(True)
    if pageable:
        out["e2e_pageable_s"], _ = e2e_pass(False)
    # one more (untimed) call over the whole batch on the device: the host
    # API moves large batches through in chunks, and the routing readback
    # (work_of) describes the last call
    one_step()
    runner.eng.sync(sp)
    return out


def roofline(kind, m, work, peaks, num_sms, workload, kernel_tag=""):
    """The dominant kernel's roofline.  kind "tensor" (prefill-size batches)
    or "hbm" (decode)."""
    nbytes, flops, fp32_ops, _ = work
    st = m["stage_ms"]
    top = max((k for k in st if k in nbytes), key=st.get)
    t = st[top] / 1e3
    hbm = nbytes[top] / t / 1e9
    if kind == "hbm" or top not in flops:
        return {"bound": "hbm", "kernel": top, "achieved": hbm, "peak": peaks["hbm_gbs"],
                "unit": "GB/s", "frac": hbm / peaks["hbm_gbs"],
                "traffic": ncu_traffic(workload, top),
                "peak_source": f"{peaks['kind']} hbm_gbs"}
    tf = flops[top] / t / 1e12
    lane_rate = num_sms * 128 * peaks["sm_max_mhz"] * 1e6 / 1e12  # FP32 lanes x clock, T op/s
    ep = fp32_ops[top] / t / 1e12
    return {"bound": "tensor", "kernel": top, "achieved": tf, "peak": peaks["bf16_sustained"],
            "unit": "TFLOP/s", "frac": tf / peaks["bf16_sustained"],
            "traffic": ncu_traffic(workload, top + kernel_tag),
            "peak_source": f"{peaks['kind']} bf16_tflops_sustained (int8 MMA FLOPs of the "
                           "expert products)",
            "epilogue": {"achieved": ep, "peak": lane_rate, "unit": "T FP32 op/s",
                         "frac": ep / lane_rate,
                         "what": "4 rounded FP32 operations per (row, pair, 32-block): the "
                                 "reference's exact Q8_0 step; peak = SMs x 128 FP32 lanes x "
                                 "max SM clock"},
            "hbm": {"achieved": hbm, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                    "frac": hbm / peaks["hbm_gbs"]}}


def summarise(ctx, args, name, T, m, work, peaks, n_act, dim=2048, steps=None):
    steps = steps or args.steps
    kind = "tensor" if name in PREFILL_WORKLOADS else "hbm"
    block_bytes = sum(work[0].values())
    r = {"value": ctx.world * T * steps / (m["total_ms"] / 1e3),
         "ms_per_step": m["total_ms"] / steps,
         "roofline": roofline(kind, m, work, peaks, ctx.num_sms, name,
                              "_tcgen05" if args.prefill_kernel == "tcgen05" else ""),
         "block_achieved_gbs": block_bytes / (m["total_ms"] / steps / 1e3) / 1e9,
         "active_experts": n_act,
         "stages_ms": {k: round(v, 5) for k, v in m["stage_ms"].items()},
         "gpu_launches": m["launches_per_step"] * steps}
    if "e2e_s" in m:
        r["e2e"] = {"value": ctx.world * T * steps / m["e2e_s"], "unit": UNIT,
                    "h2d_bytes_per_step": T * dim * 4, "d2h_bytes_per_step": T * dim * 4,
                    "inputs": ("each step's own pinned buffer, written before the timed region"
                               if m["e2e_own_buffers"] else
                               "pinned buffers written before the timed region, rewritten in "
                               "the step past 1 GiB of them")}
    if "e2e_pageable_s" in m:
        r["e2e_pageable"] = {"value": ctx.world * T * steps / m["e2e_pageable_s"], "unit": UNIT,
                             "inputs": "ordinary (pageable) host memory, like the reference "
                                       "engine's malloc'd buffers"}
    return r


def work_of(shape, T, m, eng, layer, experts_here=None):
    rec = m["received"]
    if rec is not None:
        R_in, P_in = rec
        counts = np.zeros(shape.n_experts, np.int64)
        counts[:experts_here] = 1  # the rank's experts (each has pairs at these batch sizes)
        return stage_work(shape, T, counts, rows=R_in, pairs=P_in)
    routing = eng.routing(T)
    return stage_work(shape, T, routing["counts"])


def make_ep(ctx, shape, lay, placement):
    """This rank's share of the experts and libmiag's expert-parallel block
    over an NCCL communicator of its own (rank 0's id shared through the
    process group: plumbing, no data)."""
    from motoria_b200 import MoEEngine
    from motoria_b200.ep_native import ExpertParallelBlock, NcclComm, nccl_unique_id

    uid = [nccl_unique_id() if ctx.rank == 0 else None]
    ctx.dist.broadcast_object_list(uid, src=0)
    comm = NcclComm(uid[0], ctx.world, ctx.rank, ctx.local)
    eng = MoEEngine(shape, n_layers=1, device=ctx.local)
    block = ExpertParallelBlock(eng, comm, placement)
    eng.set_layer(0, lay.ffn_norm, lay.router, lay.bias)
    for e in block.experts():
        eng.upload_experts(0, lay.blobs[e:e + 1], first=e)
    ctx.closers.append(block.close)
    ctx.closers.append(comm.close)
    return EPRunner(block, eng), eng


# config4: the whole Qwen3-30B-A3B decode step (miag_model_*), batch 1.
MODEL_DESC = ("Qwen3-30B-A3B, 48 layers, all weights random-init Q8_0 in HBM; batch-1 decode of "
              "256 tokens (positions 512..767, greedy) after a 512-token prompt of uniform-random "
              "ids; f32 KV cache of 4096 positions")
MODEL_PROMPT, MODEL_NEW, MODEL_CTX = 512, 256, 4096


def model_config():
    from motoria_b200.mia import MiaConfig
    return MiaConfig(dim=2048, n_layers=48, n_heads=32, n_kv_heads=4, head_dim=128, vocab=151936,
                     n_experts=128, n_active=8, expert_hidden=768, norm_topk=1, rope_theta=1e6,
                     norm_eps=1e-6)


def model_bytes_per_token(cfg, first_pos: int, n: int) -> float:
    """HBM bytes one decode step reads, averaged over positions
    first_pos .. first_pos + n - 1: per layer the attention matrices, the
    router and 8 experts, the K and V rows up to the position; the LM head."""
    d, qd, kvd = cfg.dim, cfg.n_heads * cfg.head_dim, cfg.n_kv_heads * cfg.head_dim
    row = lambda cols: cols // 32 * 36  # noqa: E731
    attn = (qd + 2 * kvd) * row(d) + d * row(qd)
    router = cfg.n_experts * d * 4
    experts = cfg.n_active * (2 * cfg.expert_hidden * row(d) + d * row(cfg.expert_hidden))
    mean_len = first_pos + (n + 1) / 2  # positions 0..pos are read at pos
    kv = 2 * mean_len * kvd * 4
    return cfg.n_layers * (attn + router + experts + kv) + cfg.vocab * row(d) + row(d)


def run_model_decode(ctx, args, peaks):
    """config4 on one GPU: device-timed prompt (one batched prefill) and
    decode, and the host API end to end (miag_model_generate: prompt in,
    tokens out)."""
    import torch

    from motoria_b200.model import Model

    cfg = model_config()
    P, NEW = MODEL_PROMPT, getattr(args, "model_new", MODEL_NEW)
    prompt = np.random.default_rng(XSEED).integers(0, cfg.vocab, P).astype(np.int32)
    with Model.synthetic(cfg, SEED, MODEL_CTX, device=ctx.local) as m:
        s = torch.cuda.ExternalStream(m.stream)
        for _ in range(max(1, args.warmup // 3)):  # captures the graph for this prompt length
            m.generate(prompt, 1)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        with ClockSampler(ctx.local) as clk:
            ev[0].record(s)
            m.generate_async(prompt, 1)  # positions 0..511; the last yields the first new token
            ev[1].record(s)
            m.continue_async(NEW)        # positions 512..767
            ev[2].record(s)
            m.sync()
        prompt_ms, decode_ms = ev[0].elapsed_time(ev[1]), ev[1].elapsed_time(ev[2])
        t0 = time.perf_counter()
        toks = m.generate(prompt, NEW + 1)
        e2e_s = time.perf_counter() - t0
        launches = m.launches_per_step
    tok_s = NEW / (decode_ms / 1e3)
    bpt = model_bytes_per_token(cfg, P, NEW)
    achieved = bpt * tok_s / 1e9
    return {
        "workload": f"config4: {MODEL_DESC}",
        "metric": "Qwen3-30B-A3B decode tok/s", "value": tok_s, "unit": "tokens/s",
        "ms_per_token": decode_ms / NEW,
        "prompt_positions_per_s": P / (prompt_ms / 1e3),
        "prompt": f"{P} positions in one batched prefill (miag_model_prefill)",
        "e2e": {"value": (P + NEW) / e2e_s, "unit": "positions/s",
                "what": f"miag_model_generate from a host prompt to host tokens: {P} prompt "
                        f"positions (one batched prefill) then {NEW} greedy ones, wall clock",
                "h2d_bytes_per_step": P * 4 / (P + NEW), "d2h_bytes_per_step": (NEW + 1) * 4 / (P + NEW)},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": achieved / peaks["hbm_gbs"], "traffic": None,
                     "basis": f"{bpt / 1e9:.3f} GB read per decode token (attention matrices, "
                              "router and 8 experts per layer, K/V rows, LM head) x tokens/s; "
                              f"peak: {peaks['kind']} copy bandwidth"},
        "gpu_launches_per_step": launches,
        "first_new_tokens": [int(t) for t in toks[:8]],
        "clocks": clk.summary(),
    }


def run_ours(args, T_desc, T, rms, zipf):
    ctx = Ctx()
    from motoria_b200 import PREFILL_MMA, PREFILL_TCGEN05, MoEEngine, build

    build.build()
    shape = synth.QWEN3_30B_A3B
    peaks = load_peaks()
    name = args.workload
    lay = synth.layer(shape, SEED, zipf=zipf)
    x_host = synth.tokens(shape, XSEED + 1000 * ctx.rank, T, rms_normalise=rms)
    use_ep = ctx.world > 1 and name in EP_WORKLOADS
    engines = []
    if use_ep:
        runner, eng = make_ep(ctx, shape, lay, args.ep_placement)
    else:  # one GPU, or replicas: every rank holds all experts and serves its own batch
        eng = MoEEngine(shape, n_layers=1, device=ctx.local)
        eng.load_layer(0, lay)
        runner = SingleRunner(eng, 0)
    engines.append(eng)
    eng.set_prefill_kernel(PREFILL_TCGEN05 if args.prefill_kernel == "tcgen05" else PREFILL_MMA)
    m = measure(ctx, runner, x_host, args.steps, args.warmup, pageable=ctx.world == 1,
                clocks=True)
    work = work_of(shape, T, m, eng, 0, experts_here=shape.n_experts // ctx.world)
    main = summarise(ctx, args, name, T, m, work, peaks, work[3], shape.dim)

    extras = {}
    if use_ep:  # the other placement, device-timed
        other = "strided" if args.ep_placement == "contiguous" else "contiguous"
        r2, e2 = make_ep(ctx, shape, lay, other)
        engines.append(e2)
        e2.set_prefill_kernel(eng.prefill_kernel())
        m2 = measure(ctx, r2, x_host, args.steps, args.warmup, e2e=False)
        extras[f"ep_{other}"] = {"value": ctx.world * T * args.steps / (m2["total_ms"] / 1e3),
                                 "ms_per_step": m2["total_ms"] / args.steps,
                                 "stages_ms_rank0": {k: round(v, 5) for k, v in
                                                     m2["stage_ms"].items()}}
    if ctx.world == 1 and name == DEFAULT_WORKLOAD and not args.no_extras:
        decode = {}
        for dn in DECODE_EXTRAS:
            ddesc, dT, drms, dzipf = WORKLOADS[dn]
            dlay = synth.layer(shape, SEED, zipf=dzipf)
            deng = MoEEngine(shape, n_layers=1, device=ctx.local)
            deng.load_layer(0, dlay)
            engines.append(deng)
            dx = synth.tokens(shape, XSEED, dT, rms_normalise=drms)
            dsteps = max(args.steps, 50)
            dm = measure(ctx, SingleRunner(deng, 0), dx, dsteps, args.warmup)
            dwork = work_of(shape, dT, dm, deng, 0)
            s = summarise(ctx, args, dn, dT, dm, dwork, peaks, dwork[3], shape.dim, steps=dsteps)
            s["steps"] = dsteps
            s["workload"] = f"{dn}: {ddesc}"
            decode[dn] = s
        extras["decode"] = decode
        extras["decode_model"] = run_model_decode(ctx, args, peaks)

    if ctx.rank == 0:
        cpu = None
        if ctx.world == 1 and not args.no_cpu_baseline:
            Ts = cpu_sample(T)
            v, cores, kind, steps, el = cpu_arm(shape, lay, x_host[:Ts], args.cpu_seconds)
            cpu = {"value": v, "unit": UNIT, "cores": cores, "kind": kind,
                   "sample": f"{steps} x {Ts} tokens of {name}"
                             f"{f' (the first {Ts} of {T})' if Ts < T else ''} ({el:.1f} s on "
                             f"{cores} threads, {os.uname().machine})"}
        line = {
            "metric": METRIC, "value": main["value"], "unit": UNIT, "n_gpus": ctx.world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": main["ms_per_step"],
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": DTYPE,
            "data": "synthetic (seeded random-init Q8_0 weights and N(0,1) tokens)",
            "config": {"workload": f"{name}: {T_desc}", "tokens_per_gpu": T,
                       "prefill_kernel": args.prefill_kernel,
                       "experts": shape.n_experts, "top_k": shape.n_active, "dim": shape.dim,
                       "expert_hidden": shape.expert_hidden,
                       "active_experts": main["active_experts"],
                       "weights": "Q8_0 HBM-resident",
                       "l2": "flushed between steps outside the timed events (256 MiB "
                             "written, then read back)",
                       "parallelism": (f"ep{ctx.world} ({args.ep_placement}, y back by peer "
                                       "stores over NVLink)" if use_ep else
                                       "replicas" if ctx.world > 1 else "single"),
                       "experts_per_gpu": shape.n_experts // ctx.world if use_ep
                       else shape.n_experts},
            "e2e": main.get("e2e"),
            "roofline": main["roofline"],
            "stages_ms": main["stages_ms"],
            "gpu_launches": main["gpu_launches"],
            "cpu_baseline": cpu,
            "clocks": m["clocks"],
        }
        if "e2e_pageable" in main:
            line["e2e_pageable"] = main["e2e_pageable"]
        line.update(extras)
        print(json.dumps(line), flush=True)
    for f in ctx.closers:
        f()
    for e in engines:
        e.close()
    if ctx.dist:
        ctx.dist.barrier()
        ctx.dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default=DEFAULT_WORKLOAD)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--ep-placement", choices=["contiguous", "strided"], default="contiguous",
                    help="expert placement of the expert-parallel run (config5, N>1); the "
                         "other placement is reported beside it")
    ap.add_argument("--prefill-kernel", choices=["mma", "tcgen05"], default="mma",
                    help="expert kernels for prefill-size batches (miag_set_prefill_kernel); "
                         "both give the same bits")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the decode figures (config2, config1) of the default run")
    ap.add_argument("--model-only", action="store_true",
                    help="only the whole-model decode (config4); prints its own JSON line")
    ap.add_argument("--model-new", type=int, default=MODEL_NEW,
                    help="decode steps of the whole-model run (after its 512-position prompt)")
    args = ap.parse_args()
    if args.model_only:
        from motoria_b200 import build
        build.build()
        ctx = Ctx()
        line = run_model_decode(ctx, args, load_peaks())
        if ctx.rank == 0:
            print(json.dumps(line), flush=True)
        return
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    desc, T, rms, zipf = WORKLOADS[args.workload]
    if args.impl == "reference":
        run_reference(args, desc, T, rms, zipf)
    else:
        run_ours(args, desc, T, rms, zipf)


if __name__ == "__main__":
    main()
