"""The .mia writer (miag_mia_write) against the reference's own reader
(mia_file_open, src/storage/mia_file.c:41-111, built from source into
oracle/_ref): the reader's layout walk must accept the file (its dense
section must end exactly where the header says), the header must carry the
model, f32 tensors and expert blobs must read back byte for byte, and the
quantized matrices must equal the reference quantizer's output
(src/tensor/quant.c:11-27) on the same rows.  No GPU needed."""

from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from motoria_b200 import build, synth
from motoria_b200.mia import MiaConfig, expert_blob_bytes, write_mia
from oracle import oracle as O

TINY = synth.TINY


def dense_values(name: str, n: int) -> np.ndarray:
    seed = sum(ord(ch) * (i + 1) for i, ch in enumerate(name))
    rng = np.random.default_rng(seed)
    if "norm" in name:
        return (1.0 + 0.1 * rng.standard_normal(n)).astype(np.float32)
    return (0.02 * rng.standard_normal(n)).astype(np.float32)


def config(n_layers=2, vocab=40):
    return MiaConfig(dim=TINY.dim, n_layers=n_layers, n_heads=2, n_kv_heads=1, head_dim=32,
                     vocab=vocab, n_experts=TINY.n_experts, n_active=TINY.n_active,
                     expert_hidden=TINY.expert_hidden, norm_topk=1, rope_theta=1e6,
                     norm_eps=TINY.norm_eps)


@pytest.fixture(scope="module")
def ref():
    build.build()
    O.build()
    r = O.ref()
    if r is None:
        pytest.skip("the reference build (oracle/_ref) is absent")
    lib = r.dll
    lib.ref_mia_open.restype = C.c_void_p
    lib.ref_mia_open.argtypes = [C.c_char_p, C.c_char_p, C.c_size_t]
    lib.ref_mia_close.argtypes = [C.c_void_p]
    lib.ref_mia_read_expert.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p]
    lib.ref_mia_dims.argtypes = [C.c_void_p, C.c_void_p]
    lib.ref_mia_norm_eps.restype = C.c_float
    lib.ref_mia_norm_eps.argtypes = [C.c_void_p]
    lib.ref_mia_blob_bytes.restype = C.c_uint64
    lib.ref_mia_blob_bytes.argtypes = [C.c_void_p]
    for f in ("ref_mia_ffn_norm", "ref_mia_router"):
        getattr(lib, f).restype = C.c_void_p
        getattr(lib, f).argtypes = [C.c_void_p, C.c_int]
    lib.ref_mia_tensor.restype = C.c_void_p
    lib.ref_mia_tensor.argtypes = [C.c_void_p, C.c_int, C.c_int]
    return r


def test_reference_reader_accepts_the_written_file(ref, tmp_path):
    cfg = config()
    layers = [synth.layer(TINY, 100 + l, layer_id=l) for l in range(cfg.n_layers)]
    nblob = expert_blob_bytes(cfg)
    assert nblob == TINY.blob_bytes
    path = str(tmp_path / "tiny.mia")
    write_mia(path, cfg, dense_values, lambda l, e: layers[l].blobs[e], tokenizer=b"tok\x00en")
    err = C.create_string_buffer(256)
    f = ref.dll.ref_mia_open(path.encode(), err, 256)
    assert f, err.value
    try:
        dims = np.zeros(10, np.int32)
        ref.dll.ref_mia_dims(f, dims.ctypes.data)
        assert dims.tolist() == [cfg.dim, cfg.n_layers, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim,
                                 cfg.vocab, cfg.n_experts, cfg.n_active, cfg.expert_hidden, 1]
        assert ref.dll.ref_mia_norm_eps(f) == np.float32(cfg.norm_eps)
        assert ref.dll.ref_mia_blob_bytes(f) == nblob
        got = np.zeros(nblob, np.uint8)
        for l in range(cfg.n_layers):
            for e in range(cfg.n_experts):
                assert ref.dll.ref_mia_read_expert(f, l, e, got.ctypes.data) == 0
                want = np.zeros(nblob, np.uint8)
                want[:layers[l].blobs.shape[1]] = layers[l].blobs[e]
                assert np.array_equal(got, want), (l, e)
            d = cfg.dim
            ffn = np.ctypeslib.as_array(C.cast(ref.dll.ref_mia_ffn_norm(f, l), C.POINTER(C.c_float)), (d,))
            assert np.array_equal(ffn, dense_values(f"blk.{l}.ffn_norm", d))
            rt = np.ctypeslib.as_array(C.cast(ref.dll.ref_mia_router(f, l), C.POINTER(C.c_float)),
                                       (cfg.n_experts * d,))
            assert np.array_equal(rt, dense_values(f"blk.{l}.router", cfg.n_experts * d))
        # a quantized matrix: each row as the reference quantizer encodes it
        V, d = cfg.vocab, cfg.dim
        emb = np.frombuffer(C.string_at(ref.dll.ref_mia_tensor(f, 0, 0), V * d // 32 * 36), np.uint8)
        src = dense_values("token_embd", V * d).reshape(V, d)
        want = np.concatenate([ref.quantize_row_q8(src[r]) for r in range(V)])
        assert np.array_equal(emb, want)
        qd = cfg.n_heads * cfg.head_dim
        wq = np.frombuffer(C.string_at(ref.dll.ref_mia_tensor(f, 1, 3), qd * d // 32 * 36), np.uint8)
        src = dense_values("blk.1.wq", qd * d).reshape(qd, d)
        assert np.array_equal(wq, np.concatenate([ref.quantize_row_q8(src[r]) for r in range(qd)]))
    finally:
        ref.dll.ref_mia_close(f)


def test_writer_reports_a_failing_source(tmp_path):
    build.build()
    cfg = config(n_layers=1)

    def bad_expert(l, e):
        if e == 3:
            raise IOError("disk gone")
        return np.zeros(16, np.uint8)

    with pytest.raises(Exception, match="expert 3"):
        write_mia(str(tmp_path / "bad.mia"), cfg, dense_values, bad_expert)
