"""The seeded generator: deterministic, slice-consistent, right distributions
and the reference's .mia expert blob layout."""

from __future__ import annotations

import numpy as np

from motoria_b200 import synth


def test_streams_are_deterministic_and_slice_consistent():
    k = synth.key(1, 2, 3)
    a = synth.stream_u64(k, 100)
    assert np.array_equal(a, synth.stream_u64(k, 100))
    assert np.array_equal(a[40:60], synth.stream_u64(k, 20, start=40))
    assert not np.array_equal(a, synth.stream_u64(synth.key(1, 2, 4), 100))
    x = synth.tokens(synth.QWEN3_30B_A3B, 5, 10)
    assert np.array_equal(x[3:7], synth.tokens(synth.QWEN3_30B_A3B, 5, 4, start=3))


def test_distributions():
    n = synth.normal(synth.key(9), 200_000)
    assert abs(n.mean()) < 0.01 and abs(n.std() - 1) < 0.01
    q = synth.int8_uniform(synth.key(10), 500_000)
    assert q.min() == -127 and q.max() == 127
    counts = np.bincount(q.astype(np.int16) + 127, minlength=255)
    assert counts.min() > 0.9 * counts.mean()
    w = synth.router(synth.QWEN3_30B_A3B, 1)
    assert abs(w.std() - 0.02) < 0.001
    x = synth.tokens(synth.QWEN3_30B_A3B, 1, 4)
    assert np.allclose(np.sqrt((x.astype(np.float64) ** 2).mean(1)), 1, atol=1e-6)
    b = synth.zipf_bias(synth.QWEN3_30B_A3B)
    assert b[0] == 0 and np.all(np.diff(b) < 0)


def test_blob_layout_follows_mia_format():
    s = synth.QWEN3_30B_A3B
    assert (s.off_up, s.off_down, s.blob_bytes) == (1_769_472, 3_538_944, 5_308_416)
    blob = synth.expert_blob(s, 3, 0, 5)
    rec = np.dtype([("d", "<f4"), ("q", "i1", (32,))])
    gate = np.frombuffer(blob[:s.off_up], rec)
    down = np.frombuffer(blob[s.off_down:s.off_down + 2048 * 24 * 36], rec)
    assert gate.size == 768 * 64 and np.all(gate["d"] > 0)
    assert np.all(np.abs(gate["q"]) <= 127)
    assert abs(np.median(down["d"]) * 127 / 0.02 - 0.674) < 0.05  # median of |N(0,1)|
