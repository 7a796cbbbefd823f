"""The block in three device steps (route -> expert products -> combine) and
expert parallelism, on the GPU.  Every check is bit for bit against
miag_moe on the same tokens: sharding must not change a single bit.

* the split steps on one GPU (pair p of token t is row t of the router's
  Q8_0 output, against expert idx[t][j]);
* G = 2, 4, 8 ranks played by one process on one GPU (ep.simulate), with the
  Zipf-biased router of config 3 so the ranks see skewed loads;
* with two or more GPUs visible, two NCCL ranks under torchrun, each engine
  holding only its own 64 experts (tests/ep_worker.py).
"""

from __future__ import annotations

import os
import subprocess
import sys

import numpy as np
import pytest

from conftest import get_layer
from motoria_b200 import MoEEngine, synth
from motoria_b200.ep import EngineOps, simulate

pytestmark = pytest.mark.gpu
QWEN = synth.QWEN3_30B_A3B


def _bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


@pytest.mark.parametrize("T", [1, 64, 300])
def test_split_steps_equal_the_block(torch_cuda, T):
    torch = torch_cuda
    lay = get_layer(QWEN, False)
    with MoEEngine(QWEN, n_layers=1) as eng:
        eng.load_layer(0, lay)
        x_host = synth.tokens(QWEN, 40 + T, T)
        want = eng.moe(x_host.copy())
        ops = EngineOps(eng)
        x = torch.from_numpy(x_host).cuda()
        idx, w, xq, dx = ops.route(x)
        rows = torch.arange(T * QWEN.n_active, dtype=torch.int32, device="cuda") // QWEN.n_active
        y = ops.experts(xq, dx, rows, idx.reshape(-1).contiguous())
        ops.combine(x, w, y)
        torch.cuda.synchronize()
        eng.sync()
        assert np.array_equal(_bits(x.cpu().numpy()), _bits(want))


@pytest.mark.parametrize("G,placement", [(2, "contiguous"), (4, "contiguous"), (8, "contiguous"),
                                         (4, "strided")])
def test_simulated_ranks_equal_the_block(torch_cuda, G, placement):
    torch = torch_cuda
    lay = get_layer(QWEN, True)  # Zipf-biased: rank 0 holds the hot experts
    T = 96
    with MoEEngine(QWEN, n_layers=1) as eng:
        eng.load_layer(0, lay)
        xs = np.stack([synth.tokens(QWEN, 900 + r, T) for r in range(G)])
        want = np.stack([eng.moe(xs[r].copy()) for r in range(G)])
        x = torch.from_numpy(xs).cuda()
        simulate(EngineOps(eng), x, G, placement)
        torch.cuda.synchronize()
        eng.sync()
        assert np.array_equal(_bits(x.cpu().numpy()), _bits(want))


def test_nccl_ranks_equal_the_block(torch_cuda):
    torch = torch_cuda
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    here = os.path.dirname(os.path.abspath(__file__))
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", "--nproc-per-node=2", "--master-addr", "127.0.0.1",
           "--master-port", "29517", os.path.join(here, "ep_worker.py")]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=360)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    assert "bit-exact" in r.stdout
