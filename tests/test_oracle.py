"""The CPU oracle, pinned: known answers from the reference's own tests, the
golden vectors produced by the reference build, and (where the reference
tree is present) a direct bit-for-bit comparison with it."""

from __future__ import annotations

import hashlib

import numpy as np
import pytest

from conftest import SEED, XSEED, get_layer, n_threads
from motoria_b200 import synth

CASES = {
    "tiny": (synth.TINY, 64, True, False),
    "tiny_zipf": (synth.TINY, 64, False, True),
    "config1": (synth.QWEN3_30B_A3B, 1, True, False),
    "config2": (synth.QWEN3_30B_A3B, 64, True, False),
    "config3": (synth.QWEN3_30B_A3B, 2048, False, True),
}


def blocks(buf):
    """36-byte Q8_0 records -> (d [nb], q [nb][32])."""
    b = np.frombuffer(buf, dtype=np.dtype([("d", "<f4"), ("q", "i1", (32,))]))
    return b["d"], b["q"]


# ---- tests/test_quant.c and tools/internal/mia/format_test.go:29 ----------

def test_q8_max_maps_to_127_and_halves_round_away(orc):
    x = np.zeros(32, np.float32)
    x[3], x[7] = -2.0, 1.0
    d, q = blocks(orc.quantize_row_q8(x))
    assert q[0, 3] == -127
    assert q[0, 7] == 64  # round(63.5) = 64 (test_quant.c:40)


def test_q8_zero_block_is_exact(orc):
    d, q = blocks(orc.quantize_row_q8(np.zeros(32, np.float32)))
    assert d[0] == 0.0 and not q.any()


def test_q8_roundtrip_error_is_bounded(orc):
    rng = np.random.default_rng(0)
    x = (rng.uniform(-1, 1, 256) * 3).astype(np.float32)
    d, q = blocks(orc.quantize_row_q8(x))
    y = (d[:, None] * q.astype(np.float32)).reshape(-1)
    half = np.repeat(d * 0.5 + 1e-7, 32)
    assert np.all(np.abs(x - y) <= half)


# ---- tests/test_matmul.c ---------------------------------------------------

@pytest.mark.parametrize("rows,cols", [(7, 32), (1024, 512)])
def test_f32_matvec_matches_double(orc, rows, cols):
    rng = np.random.default_rng(rows)
    w = rng.uniform(-1, 1, (rows, cols)).astype(np.float32)
    x = rng.uniform(-1, 1, cols).astype(np.float32)
    ref = w.astype(np.float64) @ x.astype(np.float64)
    assert np.max(np.abs(orc.matvec_f32(w, x) - ref)) <= 1e-3


@pytest.mark.parametrize("rows,cols", [(5, 64), (2048, 768)])
def test_q8_matvec_stays_near_exact_product(orc, rows, cols):
    rng = np.random.default_rng(cols)
    w = rng.uniform(-1, 1, (rows, cols)).astype(np.float32)
    x = rng.uniform(-1, 1, cols).astype(np.float32)
    wq = np.concatenate([orc.quantize_row_q8(r) for r in w])
    out = orc.matvec_q8(wq, x, rows, cols)
    ref = w.astype(np.float64) @ x.astype(np.float64)
    assert np.max(np.abs(out - ref)) <= 0.02 * np.sqrt(cols)


# ---- tools/internal/ref/ref_test.go:30 (routing known answer) -------------

def test_topk_routing_known_answer(orc):
    p = orc.softmax(np.array([0, 3, 1, 2], np.float32))
    idx = orc.top_k(p, 2)
    assert idx.tolist() == [1, 3]
    w = p[idx] / p[idx].sum()
    assert abs(float(w.sum()) - 1.0) < 1e-6


def test_topk_ties_go_to_lower_index(orc):
    idx = orc.top_k(np.array([0.1, 0.4, 0.4, 0.1, 0.4], np.float32), 4)
    assert idx.tolist() == [1, 2, 4, 0]


# ---- golden vectors written by the reference build -------------------------

def _case_inputs(name):
    shape, T, rms, zipf = CASES[name]
    lay = get_layer(shape, zipf)
    x = synth.tokens(shape, XSEED, T, rms_normalise=rms)
    return shape, lay, x


def _digest(lay, x):
    h = hashlib.sha256()
    for a in (lay.ffn_norm, lay.router, lay.bias, lay.blobs, x):
        if a is not None:
            h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


@pytest.mark.parametrize("name", list(CASES))
def test_generator_reproduces_golden_inputs(golden, name):
    shape, lay, x = _case_inputs(name)
    assert _digest(lay, x) == str(golden[f"{name}/input_sha256"])


@pytest.mark.parametrize("name", list(CASES))
def test_oracle_routing_matches_golden(orc, golden, name):
    shape, lay, x = _case_inputs(name)
    idx, w = orc.route(shape, lay.ffn_norm, lay.router, lay.bias, x, threads=n_threads())
    assert np.array_equal(idx, golden[f"{name}/idx"].astype(np.int32))
    assert np.array_equal(w.view(np.uint32), golden[f"{name}/w_bits"])


@pytest.mark.parametrize("name", list(CASES))
def test_oracle_block_output_matches_golden(orc, golden, name):
    shape, lay, x = _case_inputs(name)
    want = golden[f"{name}/out_bits"]
    n = want.shape[0]
    xo, _, _ = orc.moe(shape, lay.ffn_norm, lay.router, lay.bias, lay.blobs, x[:n],
                       threads=n_threads())
    assert np.array_equal(xo.view(np.uint32), want)


# ---- direct comparison with the reference build (this container only) -----

def test_oracle_equals_reference_on_random_rows(orc, ref):
    if ref is None:
        pytest.skip("reference build absent (expected on the GPU box)")
    rng = np.random.default_rng(7)
    for n in (32, 64, 2048):
        x = (rng.standard_normal(n) * rng.uniform(0.01, 10)).astype(np.float32)
        assert orc.quantize_row_q8(x).tobytes() == ref.quantize_row_q8(x).tobytes()
    x = rng.standard_normal(2048).astype(np.float32)
    w = rng.standard_normal(2048).astype(np.float32)
    assert np.array_equal(orc.rmsnorm(x, w, 1e-6).view(np.uint32),
                          ref.rmsnorm(x, w, 1e-6).view(np.uint32))
    s = rng.standard_normal(128).astype(np.float32)
    assert np.array_equal(orc.softmax(s).view(np.uint32), ref.softmax(s).view(np.uint32))


def test_oracle_equals_reference_moe_tiny(orc, ref):
    if ref is None:
        pytest.skip("reference build absent (expected on the GPU box)")
    for zipf in (False, True):
        lay = get_layer(synth.TINY, zipf)
        x = synth.tokens(synth.TINY, 5, 200, rms_normalise=not zipf)
        a = orc.moe(synth.TINY, lay.ffn_norm, lay.router, lay.bias, lay.blobs, x)
        b = ref.moe(synth.TINY, lay.ffn_norm, lay.router, lay.bias, lay.blobs, x)
        for u, v in zip(a, b):
            assert np.array_equal(u.view(np.uint32), v.view(np.uint32))


# ---- canonical permutation (no reference counterpart) ----------------------

def test_permutation_is_stable_counting_sort(orc):
    rng = np.random.default_rng(3)
    T, K, E = 300, 8, 128
    idx = np.stack([rng.choice(E, K, replace=False) for _ in range(T)]).astype(np.int32)
    r = orc.permute(idx, E)
    pairs = np.arange(T * K)
    want = sorted(pairs, key=lambda p: (idx.reshape(-1)[p], p))
    assert r["perm"].tolist() == want
    assert np.array_equal(r["counts"], np.bincount(idx.reshape(-1), minlength=E))
    assert r["offsets"][0] == 0 and r["offsets"][-1] == T * K
    assert np.array_equal(r["inv"][r["perm"]], pairs)
