"""One rank of the C-ABI expert-parallel check (launched by torchrun from
test_gpu_ep.py): libmiag's own expert-parallel block (miag_ep_*: NCCL,
dispatch, peer stores and combine inside the library) over this rank's
engine, which holds only its own experts.  Two layers run one after the
other, twice, from host arrays (miag_moe_ep), and once more from a device
buffer (miag_moe_ep_async); every output must equal a full one-GPU block on
the same tokens, bit for bit.  torch.distributed (gloo) only shares the NCCL
id and gathers the verdict: it carries none of the data."""

from __future__ import annotations

import datetime
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), ".."))
from motoria_b200 import MoEEngine, synth  # noqa: E402
from motoria_b200.ep_native import ExpertParallelBlock, NcclComm, nccl_unique_id  # noqa: E402

LAYER_SEEDS = (1234, 4321)


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    shape = synth.QWEN3_30B_A3B
    T = int(os.environ.get("EP_TOKENS", "300")) + 37 * rank  # ragged across ranks
    placement = os.environ.get("EP_PLACEMENT", "contiguous")
    uid = [nccl_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(uid, src=0)
    comm = NcclComm(uid[0], world, rank, local)
    lays = [synth.layer(shape, s, zipf=True) for s in LAYER_SEEDS]
    eng = MoEEngine(shape, n_layers=len(lays), device=local)
    block = ExpertParallelBlock(eng, comm, placement)
    full = MoEEngine(shape, n_layers=len(lays), device=local)
    for l, lay in enumerate(lays):
        eng.set_layer(l, lay.ffn_norm, lay.router, lay.bias)
        for e in block.experts():  # only this rank's experts
            eng.upload_experts(l, lay.blobs[e:e + 1], first=e)
        full.load_layer(l, lay)
    x_host = synth.tokens(shape, 500 + rank, T)
    want = x_host.copy()
    for l in range(len(lays)):
        want = full.moe(want, layer=l)
    ok = True
    for _ in range(2):  # twice: the second call reuses the exchange buffers and flags
        x = x_host.copy()
        for l in range(len(lays)):
            block.forward_host(x, layer=l)
        ok = ok and np.array_equal(x.view(np.uint32), want.view(np.uint32))
    xd = torch.from_numpy(x_host).cuda(local)  # a device buffer, the library's own stream
    for l in range(len(lays)):
        block.forward_device(xd.data_ptr(), T, layer=l)
    eng.sync()
    ok = ok and np.array_equal(xd.cpu().numpy().view(np.uint32), want.view(np.uint32))
    flag = torch.tensor([int(ok)])
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    if rank == 0:
        print(f"C-ABI EP world {world} ({placement}), {len(lays)} layers: "
              f"{'bit-exact' if flag.item() else 'MISMATCH'}", flush=True)
    block.close()
    comm.close()
    eng.close()
    full.close()
    dist.barrier()
    dist.destroy_process_group()
    sys.exit(0 if flag.item() else 1)


if __name__ == "__main__":
    main()
