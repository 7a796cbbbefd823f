"""GPU parity of the sm_100a MoE block against the CPU oracle and the golden
vectors of the reference build.  Everything is called through libmiag's C ABI.

Bars:
  * router top-k indices and the dispatch permutation: bit-exact;
  * block output: the MoE update (out - x) within RTOL_L2 = 1e-3 relative L2
    per token.  In practice the GPU repeats the reference's scalar arithmetic
    operation for operation, so most tokens are bit-exact; the only source of
    difference is expf (glibc's vs. the correctly rounded float of CUDA's
    double exp), which can move one routing weight or one SwiGLU value by an
    ulp.
"""

from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from conftest import SEED, XSEED, get_layer, n_threads, rel_l2
from motoria_b200 import (MIA_F32, MIA_Q8_0, PREFILL_MMA, PREFILL_TCGEN05, MoEEngine, build, matvec,
                          quantize_row_q8, synth)
from motoria_b200._native import MiagError

pytestmark = pytest.mark.gpu

QWEN, TINY = synth.QWEN3_30B_A3B, synth.TINY
RTOL_L2 = 1e-3   # per-token relative L2 of the MoE update
W_ULPS = 4       # routing weights: expf may differ by an ulp, renormalisation spreads it


def ulp_diff(a, b):
    a = np.asarray(a, np.float32).view(np.int32).astype(np.int64)
    b = np.asarray(b, np.float32).view(np.int32).astype(np.int64)
    return np.abs(a - b)


def check_block(x_in, gpu, want, label=""):
    """Per-token relative L2 of the update; returns the bit-exact token fraction."""
    errs = [rel_l2(g - x, w - x) for g, w, x in zip(gpu, want, x_in)]
    exact = np.mean([np.array_equal(g.view(np.uint32), w.view(np.uint32))
                     for g, w in zip(gpu, want)])
    print(f"{label}: max rel-L2 {max(errs):.3e}, bit-exact tokens {exact:.3f}")
    assert max(errs) <= RTOL_L2, (label, max(errs))
    return exact


@pytest.fixture(scope="module")
def qwen(torch_cuda):
    """Layer 0: reference router; layer 1: same experts, Zipf logit bias."""
    build.build()
    eng = MoEEngine(QWEN, n_layers=2)
    plain = get_layer(QWEN, False)
    eng.load_layer(0, plain)
    zipf = get_layer(QWEN, True)
    eng.set_layer(1, zipf.ffn_norm, zipf.router, zipf.bias)
    eng.upload_experts(1, zipf.blobs)
    # host calls in one pass, so that the routing readbacks cover every token
    # (test_host_call_in_pieces_equals_one_pass covers the piecewise calls)
    eng.set_transfer_chunks(1)
    yield eng, plain, zipf
    eng.close()


@pytest.fixture(scope="module")
def tiny(torch_cuda):
    build.build()
    eng = MoEEngine(TINY, n_layers=2)
    plain, zipf = get_layer(TINY, False), get_layer(TINY, True)
    eng.load_layer(0, plain)
    eng.load_layer(1, zipf)
    yield eng, plain, zipf
    eng.close()


# ---- reference public math ABI --------------------------------------------

def test_quantize_row_q8_bit_exact(orc, torch_cuda):
    torch = torch_cuda
    rng = np.random.default_rng(11)
    rows = [rng.standard_normal(4096) * s for s in (1e-6, 0.02, 1.0, 300.0)]
    known = np.zeros(32)
    known[3], known[7] = -2.0, 1.0
    rows += [known, np.zeros(64), np.repeat([0.5, -0.5], 32)]
    for r in rows:
        x = np.ascontiguousarray(r, np.float32)
        xd = torch.from_numpy(x).cuda()
        yd = torch.zeros(x.size // 32 * 36, dtype=torch.uint8, device="cuda")
        quantize_row_q8(xd.data_ptr(), yd.data_ptr(), x.size)
        torch.cuda.synchronize()
        assert yd.cpu().numpy().tobytes() == orc.quantize_row_q8(x).tobytes()


@pytest.mark.parametrize("rows,cols", [(5, 64), (768, 2048), (2048, 768)])
def test_matvec_q8_bit_exact(orc, torch_cuda, rows, cols):
    torch = torch_cuda
    rng = np.random.default_rng(rows + cols)
    w = rng.uniform(-1, 1, (rows, cols)).astype(np.float32)
    x = rng.uniform(-1, 1, cols).astype(np.float32)
    wq = np.concatenate([orc.quantize_row_q8(r) for r in w])
    out = torch.zeros(rows, dtype=torch.float32, device="cuda")
    xq = torch.zeros(cols // 32 * 36, dtype=torch.uint8, device="cuda")
    wd = torch.from_numpy(wq).cuda()
    xd = torch.from_numpy(x).cuda()
    matvec(out.data_ptr(), wd.data_ptr(), MIA_Q8_0, xd.data_ptr(), xq.data_ptr(), rows, cols)
    torch.cuda.synchronize()
    want = orc.matvec_q8(wq, x, rows, cols)
    assert np.array_equal(out.cpu().numpy().view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("rows,cols", [(7, 32), (128, 2048)])
def test_matvec_f32_bit_exact(orc, torch_cuda, rows, cols):
    torch = torch_cuda
    rng = np.random.default_rng(rows)
    w = rng.uniform(-1, 1, (rows, cols)).astype(np.float32)
    x = rng.uniform(-1, 1, cols).astype(np.float32)
    out = torch.zeros(rows, dtype=torch.float32, device="cuda")
    wd, xd = torch.from_numpy(w).cuda(), torch.from_numpy(x).cuda()  # keep both alive
    matvec(out.data_ptr(), wd.data_ptr(), MIA_F32, xd.data_ptr(), 0, rows, cols)
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy().view(np.uint32), orc.matvec_f32(w, x).view(np.uint32))


# ---- router logits: the reference's fp32 matvec order, bit for bit ----------

@pytest.mark.parametrize("T,rms,layer", [(1, True, 0), (64, True, 0), (2048, False, 1)])
def test_router_logits_bit_exact(qwen, orc, T, rms, layer):
    eng, plain, zipf = qwen
    lay = plain if layer == 0 else zipf
    x = synth.tokens(QWEN, XSEED + 7, T, rms_normalise=rms)
    eng.moe(x, layer=layer)
    got = eng.router_logits(T)
    want = np.stack([orc.matvec_f32(lay.router, orc.rmsnorm(x[t], lay.ffn_norm, QWEN.norm_eps))
                     for t in range(T)])
    if lay.bias is not None:
        want = want + lay.bias[None, :]
    assert np.array_equal(got.view(np.uint32), want.astype(np.float32).view(np.uint32))


# ---- the MoE block against the reference's golden vectors ------------------

GOLDEN_CASES = {
    "tiny": ("tiny", 0, 64, True),
    "tiny_zipf": ("tiny", 1, 64, False),
    "config1": ("qwen", 0, 1, True),
    "config2": ("qwen", 0, 64, True),
    "config3": ("qwen", 1, 2048, False),
}


@pytest.mark.parametrize("name", list(GOLDEN_CASES))
def test_block_matches_reference_golden(request, golden, name):
    which, layer, T, rms = GOLDEN_CASES[name]
    eng, plain, zipf = request.getfixturevalue(which)
    shape = eng.shape
    x = synth.tokens(shape, XSEED, T, rms_normalise=rms)
    out = eng.moe(x, layer=layer)
    r = eng.routing(T)
    assert np.array_equal(r["idx"], golden[f"{name}/idx"].astype(np.int32))
    assert ulp_diff(r["w"], golden[f"{name}/w_bits"].view(np.float32)).max() <= W_ULPS
    want = golden[f"{name}/out_bits"].view(np.float32)
    check_block(x[:len(want)], out[:len(want)], want, name)


def test_config2_full_batch_matches_oracle(qwen, orc):
    eng, plain, _ = qwen
    x = synth.tokens(QWEN, XSEED + 1, 64)
    out = eng.moe(x, layer=0)
    r = eng.routing(64)
    want, idx, w = orc.moe(QWEN, plain.ffn_norm, plain.router, None, plain.blobs, x,
                           threads=n_threads())
    assert np.array_equal(r["idx"], idx)
    assert ulp_diff(r["w"], w).max() <= W_ULPS
    exact = check_block(x, out, want, "config2-oracle")
    assert exact >= 0.5


def test_config3_routing_permutation_and_every_output(qwen, orc):
    eng, _, zipf = qwen
    T = 2048
    x = synth.tokens(QWEN, XSEED + 2, T, rms_normalise=False)
    out = eng.moe(x, layer=1)
    r = eng.routing(T)
    idx, w = orc.route(QWEN, zipf.ffn_norm, zipf.router, zipf.bias, x, threads=n_threads())
    assert np.array_equal(r["idx"], idx)
    assert ulp_diff(r["w"], w).max() <= W_ULPS
    p = orc.permute(idx, QWEN.n_experts)
    assert np.array_equal(r["perm"], p["perm"])
    assert np.array_equal(r["offsets"], p["offsets"])
    assert np.array_equal(r["counts"], p["counts"])
    assert r["counts"][0] > 4 * r["counts"][-1]  # the Zipf bias skews the load
    # every one of the 2048 tokens against the oracle (threaded on the host)
    want, _, _ = orc.moe(QWEN, zipf.ffn_norm, zipf.router, zipf.bias, zipf.blobs, x,
                         threads=n_threads())
    exact = check_block(x, out, want, "config3-all-2048")
    assert exact >= 0.8  # the rest differ through glibc's expf (rare misroundings)


def test_config5_size_permutation_invariants_and_every_output(qwen, orc):
    eng, _, zipf = qwen
    T = 4096
    x = synth.tokens(QWEN, XSEED + 3, T, rms_normalise=False)
    out = eng.moe(x, layer=1)
    r = eng.routing(T)
    P = T * QWEN.n_active
    perm = r["perm"]
    assert np.array_equal(np.sort(perm), np.arange(P))           # a permutation
    e_sorted = r["idx"].reshape(-1)[perm]
    assert np.all(np.diff(e_sorted) >= 0)                        # grouped by expert
    for e in range(QWEN.n_experts):                              # stable within expert
        seg = perm[r["offsets"][e]:r["offsets"][e + 1]]
        assert np.all(np.diff(seg) > 0)
    assert np.array_equal(np.cumsum(r["counts"]), r["offsets"][1:])
    assert np.allclose(r["w"].sum(1), 1.0, atol=2e-6)
    # every one of the 4096 tokens against the oracle (threaded on the host)
    want, idx, _ = orc.moe(QWEN, zipf.ffn_norm, zipf.router, zipf.bias, zipf.blobs, x,
                           threads=n_threads())
    assert np.array_equal(r["idx"], idx)
    exact = check_block(x, out, want, "config5-size-all-4096")
    assert exact >= 0.8


@pytest.mark.parametrize("T,layer", [(129, 1), (700, 0), (1500, 1), (4096, 1)])
def test_prefill_kernels_agree_bit_for_bit(qwen, T, layer):
    """The tcgen05 prefill kernels (tensor-memory block dots, separate
    epilogue warps) against the mma.sync kernels on the same batch: every
    output bit equal.  129 tokens is just past the prefill threshold (1032
    pairs over 128 experts: many chunks of 1-16 pairs); 4096 with the Zipf
    bias gives full 128-pair chunks and one expert with thousands of pairs."""
    eng, _, _ = qwen
    x = synth.tokens(QWEN, 300 + T, T, rms_normalise=layer == 0)
    default = eng.prefill_kernel()
    try:
        eng.set_prefill_kernel(PREFILL_TCGEN05)
        got = eng.moe(x, layer=layer)
        eng.set_prefill_kernel(PREFILL_MMA)
        want = eng.moe(x, layer=layer)
    finally:
        eng.set_prefill_kernel(default)
    same = np.all(got.view(np.uint32) == want.view(np.uint32), axis=1)
    assert same.all(), f"{int((~same).sum())} of {T} tokens differ"


@pytest.mark.parametrize("T,chunks", [(2048, 4), (4096, 4), (3001, 3), (4096, 16)])
def test_host_call_in_pieces_equals_one_pass(qwen, T, chunks):
    """miag_moe of >= 2048 host tokens moves them through in pieces while the
    block runs (copy stream): every output bit equals one pass, from pinned
    and from pageable host memory."""
    import torch
    eng, _, _ = qwen
    x = synth.tokens(QWEN, 900 + T, T, rms_normalise=False)
    eng.set_transfer_chunks(1)
    want = eng.moe(x, layer=1)
    eng.set_transfer_chunks(chunks)
    try:
        got = eng.moe(x, layer=1)
        pinned = torch.from_numpy(x.copy()).pin_memory()
        arr = pinned.numpy()
        eng.moe_inplace(arr, layer=1)
    finally:
        eng.set_transfer_chunks(1)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    assert np.array_equal(arr.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("T,chunks", [(300, 4), (2048, 4), (4097, 8)])
def test_pageable_staging_equals_direct_copies(qwen, T, chunks):
    """A pageable host buffer of >= 1 MiB goes through the context's pinned
    staging buffer, copied by host threads piece by piece: every output bit
    equals the driver's own pageable copies (0 threads), one copying thread,
    and a pinned buffer."""
    import torch
    eng, _, _ = qwen
    x = synth.tokens(QWEN, 1300 + T, T, rms_normalise=False)
    eng.set_transfer_chunks(chunks)
    try:
        eng.set_host_copy_threads(0)
        want = eng.moe(x, layer=0)
        outs = {}
        for threads in (1, 3, 8):
            eng.set_host_copy_threads(threads)
            outs[threads] = eng.moe(x, layer=0)
        pinned = torch.from_numpy(x.copy()).pin_memory()
        arr = pinned.numpy()
        eng.moe_inplace(arr, layer=0)
        outs["pinned"] = arr
    finally:
        eng.set_host_copy_threads(8)
        eng.set_transfer_chunks(1)
    for k, got in outs.items():
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), k


# ---- size-independent properties -------------------------------------------

def test_batch_invariance_and_determinism(qwen):
    eng, _, _ = qwen
    x = synth.tokens(QWEN, 5, 300)
    full = eng.moe(x, layer=0)
    again = eng.moe(x, layer=0)
    assert np.array_equal(full.view(np.uint32), again.view(np.uint32))
    for lo, hi in ((0, 1), (17, 18), (100, 164), (299, 300)):
        part = eng.moe(x[lo:hi], layer=0)
        assert np.array_equal(part.view(np.uint32), full[lo:hi].view(np.uint32))


def test_sm_shares_leave_results_unchanged(torch_cuda):
    """The expert launches split their items over the SMs by rates measured
    in earlier launches, so shares differ from call to call.  Whatever the
    split, every output bit must equal the first call on a fresh context
    (equal shares); both regimes, and Zipf routing with its hot experts."""
    build.build()
    cases = [(layer, T, 50 + i) for i, (layer, T) in
             enumerate([(0, 64), (1, 64), (0, 200), (0, 1500), (1, 1500)])]
    with MoEEngine(QWEN, n_layers=2) as eng:
        eng.load_layer(0, get_layer(QWEN, False))
        eng.load_layer(1, get_layer(QWEN, True))
        first = {c: eng.moe(synth.tokens(QWEN, c[2], c[1]), layer=c[0]) for c in cases[:1]}
    with MoEEngine(QWEN, n_layers=2) as eng:
        eng.load_layer(0, get_layer(QWEN, False))
        eng.load_layer(1, get_layer(QWEN, True))
        for c in cases[1:]:  # each on a fresh context first: equal shares
            with MoEEngine(QWEN, n_layers=2) as fresh:
                fresh.load_layer(c[0], get_layer(QWEN, c[0] == 1))
                first[c] = fresh.moe(synth.tokens(QWEN, c[2], c[1]), layer=c[0])
        for rep in range(6):  # the same context again and again: weighted shares
            for c in cases:
                got = eng.moe(synth.tokens(QWEN, c[2], c[1]), layer=c[0])
                assert np.array_equal(got.view(np.uint32), first[c].view(np.uint32)), (rep, c)


def test_hot_experts_take_every_token(torch_cuda, orc):
    """A bias that pushes experts 3 and 77 into every token's top-k gives them
    T pairs each, exercising many pair rounds per staged weight tile."""
    eng = MoEEngine(QWEN, n_layers=1)
    try:
        lay = get_layer(QWEN, False)
        bias = np.zeros(QWEN.n_experts, np.float32)
        bias[[3, 77]] = 50.0
        eng.set_layer(0, lay.ffn_norm, lay.router, bias)
        eng.upload_experts(0, lay.blobs)
        T = 300
        x = synth.tokens(QWEN, 8, T)
        out = eng.moe(x)
        r = eng.routing(T)
        assert r["counts"][3] == T and r["counts"][77] == T
        sample = np.arange(0, T, 10)
        want, idx, _ = orc.moe(QWEN, lay.ffn_norm, lay.router, bias, lay.blobs, x[sample],
                               threads=n_threads())
        assert np.array_equal(r["idx"][sample], idx)
        check_block(x[sample], out[sample], want, "hot-experts")
    finally:
        eng.close()


def test_identical_experts_make_output_router_invariant(torch_cuda):
    """tools/internal/ref/ref_test.go:75: with every expert equal, weights that
    sum to one make the block independent of the router."""
    eng = MoEEngine(QWEN, n_layers=2)
    try:
        lay = get_layer(QWEN, False)
        same = np.repeat(lay.blobs[:1], QWEN.n_experts, axis=0)
        eng.set_layer(0, lay.ffn_norm, lay.router)
        eng.set_layer(1, lay.ffn_norm, lay.router * -3.0)
        eng.upload_experts(0, same)
        eng.upload_experts(1, same)
        x = synth.tokens(QWEN, 9, 16)
        a, b = eng.moe(x, layer=0), eng.moe(x, layer=1)
        assert rel_l2(a - x, b - x) < 1e-4
    finally:
        eng.close()


def test_empty_and_tiny_batches(tiny, orc):
    eng, plain, _ = tiny
    x0 = np.zeros((0, TINY.dim), np.float32)
    assert eng.moe(x0).shape == (0, TINY.dim)
    for T in (1, 2, 3, 5, 33):
        x = synth.tokens(TINY, 40 + T, T)
        out = eng.moe(x)
        want, idx, _ = orc.moe(TINY, plain.ffn_norm, plain.router, None, plain.blobs, x)
        assert np.array_equal(eng.routing(T)["idx"], idx)
        check_block(x, out, want, f"tiny-T{T}")


def test_async_device_path_equals_host_path(qwen, torch_cuda):
    torch = torch_cuda
    eng, _, _ = qwen
    x = synth.tokens(QWEN, 21, 64)
    host = eng.moe(x)
    xd = torch.from_numpy(x).cuda()
    s = torch.cuda.current_stream()
    eng.moe_device(xd.data_ptr(), 64, layer=0, stream=s.cuda_stream)
    eng.sync(s.cuda_stream)
    assert np.array_equal(xd.cpu().numpy().view(np.uint32), host.view(np.uint32))
    assert eng.last_launch_count() > 0


# ---- the loader port and its failure path ----------------------------------

def test_loader_port_uploads_like_bulk_upload(torch_cuda):
    lay = get_layer(TINY, False)
    eng = MoEEngine(TINY, n_layers=1)
    try:
        eng.set_layer(0, lay.ffn_norm, lay.router)

        def loader(layer, expert, dst):
            dst[:] = lay.blobs[expert].tobytes()
            return 0

        eng.load_experts(loader)
        x = synth.tokens(TINY, 3, 16)
        a = eng.moe(x)
        eng2 = MoEEngine(TINY, n_layers=1)
        eng2.load_layer(0, lay)
        assert np.array_equal(a.view(np.uint32), eng2.moe(x).view(np.uint32))
        eng2.close()
    finally:
        eng.close()


def test_loader_failure_reports_the_expert(torch_cuda):
    """Like the reference's fake_disk failure (tests/test_cache.c:61-71): a
    failing load returns -1 with a message naming the expert."""
    lay = get_layer(TINY, False)
    eng = MoEEngine(TINY, n_layers=1)
    try:
        def loader(layer, expert, dst):
            if expert == 5:
                return -1
            dst[:] = lay.blobs[expert].tobytes()
            return 0

        with pytest.raises(MiagError, match="expert 5"):
            eng.load_experts(loader)
        with pytest.raises(MiagError, match="layer 3 out of range"):
            eng.moe(np.zeros((1, TINY.dim), np.float32), layer=3)
    finally:
        eng.close()


def test_wait_timeout_is_reported_and_context_survives(torch_cuda):
    """Failure detection without a fault: a bounded wait on a barrier nothing
    completes gives up after its limit, the error comes back through the
    context's error word, and the context then runs the block as before."""
    build.build()
    with MoEEngine(TINY, n_layers=1) as eng:
        eng.load_layer(0, get_layer(TINY, False))
        x = synth.tokens(TINY, 5, 9)
        before = eng.moe(x.copy())
        msg = eng.selftest_wait_timeout(2000)
        assert "timed out" in msg, msg
        after = eng.moe(x.copy())
        assert np.array_equal(before.view(np.uint32), after.view(np.uint32))
        eng.sync()  # the error word was cleared when it was reported


def test_peer_wait_timeout_is_reported_and_context_survives(torch_cuda):
    """Failure detection for the expert-parallel exchange, on one GPU and
    without a fault: the wait for the ranks' flags (miag_ep_wait_async) on a
    flag that no rank will raise gives up after its limit (two seconds), the
    next miag_sync reports it, and the context then runs the block as
    before."""
    build.build()
    with MoEEngine(TINY, n_layers=1) as eng:
        eng.load_layer(0, get_layer(TINY, False))
        x = synth.tokens(TINY, 5, 9)
        before = eng.moe(x.copy())
        _, flags, _ = eng.ep_buffer(4)  # this rank's flags, zero: nothing has stored here
        eng.ep_wait_device(flags, 1, 1)
        with pytest.raises(MiagError, match="another rank"):
            eng.sync()
        after = eng.moe(x.copy())
        assert np.array_equal(before.view(np.uint32), after.view(np.uint32))
        eng.sync()  # the error word was cleared when it was reported
