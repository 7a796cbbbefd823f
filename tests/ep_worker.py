"""One rank of the NCCL expert-parallel check (launched by torchrun from
test_gpu_ep.py): this rank's engine holds only its own experts; the sharded
block must equal a full single-GPU block on the same tokens, bit for bit."""

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


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    shape = synth.QWEN3_30B_A3B
    T = int(os.environ.get("EP_TOKENS", "300"))
    lay = synth.layer(shape, 1234, zipf=True)
    ep_eng = MoEEngine(shape, n_layers=1, device=local)
    ep = ExpertParallelMoE(EngineOps(ep_eng), placement=os.environ.get("EP_PLACEMENT", "contiguous"),
                           exchange=os.environ.get("EP_EXCHANGE", "peer"))
    ep_eng.set_layer(0, lay.ffn_norm, lay.router, lay.bias)
    for e in ep.experts_of(rank):  # only this rank's experts
        ep_eng.upload_experts(0, lay.blobs[e:e + 1], first=e)
    full = MoEEngine(shape, n_layers=1, device=local)
    full.load_layer(0, lay)
    x_host = synth.tokens(shape, 500 + rank, T)
    want = full.moe(x_host.copy())
    ok = True
    for _ in range(2):  # twice: the second call reuses the exchange buffers and flags
        x = torch.from_numpy(x_host).cuda()
        ep.forward(x)
        torch.cuda.synchronize()
        ep_eng.sync()  # reports any device-side error of the sharded steps
        got = x.cpu().numpy()
        ok = ok and np.array_equal(got.view(np.uint32), want.view(np.uint32))
    flags = torch.tensor([int(ok)], device="cuda")
    dist.all_reduce(flags, op=dist.ReduceOp.MIN)
    if rank == 0:
        print(f"EP world {world}: {'bit-exact' if flags.item() else 'MISMATCH'}", flush=True)
    ep_eng.close()
    full.close()
    dist.barrier()
    dist.destroy_process_group()
    sys.exit(0 if flags.item() else 1)


if __name__ == "__main__":
    main()
