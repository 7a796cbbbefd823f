"""miag_moe_noalloc: the MoE block for callers that cannot let a call
allocate device memory -- an engine that reserves its whole HBM budget up
front, or a serving loop that cannot take cudaMalloc's implicit device-wide
synchronisation mid-step.  Its scratch is a fixed array inside libmiag, so
these checks compare it, through the C ABI, with the allocating entry point
(miag_moe) on consecutive calls that reuse that array, and check that an
oversized batch is refused instead of being allocated for.

Kept in a file of its own that pytest collects last.
"""

from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from conftest import get_layer, rel_l2
from motoria_b200 import MoEEngine, build, synth
from motoria_b200 import _native as N

pytestmark = pytest.mark.gpu

RTOL_L2 = 1e-3  # the block tolerance of the parity tests (per-token update)


def noalloc(eng, x_dev_ptr, n_tokens, layer=0):
    err = N.errbuf()
    rc = N.lib().miag_moe_noalloc(eng._ctx, layer, C.c_void_p(x_dev_ptr), n_tokens, None, err,
                                  len(err))
    return rc, err.value.decode(errors="replace")


def test_noalloc_matches_the_allocating_entry_point_on_consecutive_calls(torch_cuda):
    torch = torch_cuda
    build.build()
    shape = synth.QWEN3_30B_A3B
    with MoEEngine(shape, n_layers=1) as eng:
        eng.load_layer(0, get_layer(shape, False))
        # two calls in a row; the second reuses whatever the first left in the array
        for seed, T in ((11, 64), (12, 17)):
            x = synth.tokens(shape, seed, T)
            want = eng.moe(x)  # miag_moe: host buffers, workspace it may grow
            xd = torch.from_numpy(x).cuda()
            rc, msg = noalloc(eng, xd.data_ptr(), T)
            assert rc == 0, msg
            eng.sync()  # NULL stream = the context's stream; also reports device errors
            got = xd.cpu().numpy()
            # the same kernels on the same bytes: identical bits, like the
            # expert-parallel checks; the block tolerance is only reported
            errs = [rel_l2(g - a, w - a) for g, w, a in zip(got, want, x)]
            print(f"T={T}: max rel-L2 {max(errs):.1e} (block tolerance {RTOL_L2})")
            assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), max(errs)


def test_noalloc_refuses_batches_beyond_its_array(torch_cuda):
    torch = torch_cuda
    build.build()
    shape = synth.QWEN3_30B_A3B
    with MoEEngine(shape, n_layers=1) as eng:
        eng.load_layer(0, get_layer(shape, False))
        T = 200
        xd = torch.zeros((T, shape.dim), dtype=torch.float32, device="cuda")
        rc, msg = noalloc(eng, xd.data_ptr(), T)
        assert rc == -1 and "scratch" in msg
        rc, msg = noalloc(eng, xd.data_ptr(), 93)
        assert rc == -1 and "scratch" in msg
        rc, msg = noalloc(eng, xd.data_ptr(), 92)  # the largest batch that fits
        assert rc == 0, msg
        eng.sync()
