"""One rank of the NCCL expert-parallel check (launched by torchrun from
test_gpu_ep.py): this rank's engine holds only its own experts; the sharded
block must equal a full single-GPU block on the same tokens, bit for bit.

Two layers run one after the other over the same engine (one
ExpertParallelMoE each, as a layer loop would build them), so they share the
engine's one peer exchange: its step counter and mappings."""

from __future__ import annotations

import datetime
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), ".."))
from motoria_b200 import MoEEngine, synth  # noqa: E402
from motoria_b200.ep import EngineOps, ExpertParallelMoE  # noqa: E402

LAYER_SEEDS = (1234, 4321)


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    shape = synth.QWEN3_30B_A3B
    T = int(os.environ.get("EP_TOKENS", "300"))
    n_layers = len(LAYER_SEEDS)
    lays = [synth.layer(shape, s, zipf=True) for s in LAYER_SEEDS]
    ep_eng = MoEEngine(shape, n_layers=n_layers, device=local)
    eps = [ExpertParallelMoE(EngineOps(ep_eng, layer=l),
                             placement=os.environ.get("EP_PLACEMENT", "contiguous"),
                             exchange=os.environ.get("EP_EXCHANGE", "peer"))
           for l in range(n_layers)]
    full = MoEEngine(shape, n_layers=n_layers, device=local)
    for l, lay in enumerate(lays):
        ep_eng.set_layer(l, lay.ffn_norm, lay.router, lay.bias)
        for e in eps[l].experts_of(rank):  # only this rank's experts
            ep_eng.upload_experts(l, lay.blobs[e:e + 1], first=e)
        full.load_layer(l, lay)
    x_host = synth.tokens(shape, 500 + rank, T)
    want = x_host.copy()
    for l in range(n_layers):
        want = full.moe(want, layer=l)
    ok = True
    for _ in range(2):  # twice: the second call reuses the exchange buffers and flags
        x = torch.from_numpy(x_host).cuda()
        for ep in eps:
            ep.forward(x)
        torch.cuda.synchronize()
        ep_eng.sync()  # reports any device-side error of the sharded steps
        got = x.cpu().numpy()
        ok = ok and np.array_equal(got.view(np.uint32), want.view(np.uint32))
    flags = torch.tensor([int(ok)], device="cuda")
    dist.all_reduce(flags, op=dist.ReduceOp.MIN)
    if rank == 0:
        print(f"EP world {world}, {n_layers} layers: {'bit-exact' if flags.item() else 'MISMATCH'}",
              flush=True)
    ep_eng.close()
    full.close()
    dist.barrier()
    dist.destroy_process_group()
    sys.exit(0 if flags.item() else 1)


if __name__ == "__main__":
    main()
