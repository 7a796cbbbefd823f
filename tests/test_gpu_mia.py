"""A .mia file to HBM and through the block: a one-layer Qwen3-30B-A3B-shaped
file written by miag_mia_write, opened by the reference's own reader
(mia_file_open), its experts loaded with miag_load_experts through the
reference's mia_file_read_expert (the loader port, include/mia/
expert_cache.h:8), its ffn_norm and router taken from the reader; the block
must then match the reference engine's moe() on the same file's weights."""

from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from conftest import n_threads, rel_l2
from motoria_b200 import MoEEngine, build, synth
from motoria_b200 import _native as N
from motoria_b200.mia import MiaConfig, write_mia
from oracle import oracle as O

pytestmark = pytest.mark.gpu
QWEN = synth.QWEN3_30B_A3B


def test_mia_file_through_the_loader_port_matches_the_reference(torch_cuda, tmp_path):
    build.build()
    r = O.ref()
    if r is None:
        pytest.skip("the reference build (oracle/_ref) is absent")
    lib = r.dll
    lib.ref_mia_open.restype = C.c_void_p
    lib.ref_mia_open.argtypes = [C.c_char_p, C.c_char_p, C.c_size_t]
    lib.ref_mia_close.argtypes = [C.c_void_p]
    for f in ("ref_mia_ffn_norm", "ref_mia_router"):
        getattr(lib, f).restype = C.c_void_p
        getattr(lib, f).argtypes = [C.c_void_p, C.c_int]
    lay = synth.layer(QWEN, 777)
    cfg = MiaConfig(dim=QWEN.dim, n_layers=1, n_heads=4, n_kv_heads=1, head_dim=128, vocab=32,
                    n_experts=QWEN.n_experts, n_active=QWEN.n_active,
                    expert_hidden=QWEN.expert_hidden, norm_topk=1, rope_theta=1e6,
                    norm_eps=QWEN.norm_eps)

    def dense(name, n):
        if name.endswith("ffn_norm"):
            return lay.ffn_norm
        if name.endswith("router"):
            return lay.router
        return np.full(n, 0.01, np.float32)

    path = str(tmp_path / "qwen_layer.mia")
    write_mia(path, cfg, dense, lambda l, e: lay.blobs[e])
    err = C.create_string_buffer(256)
    f = lib.ref_mia_open(path.encode(), err, 256)
    assert f, err.value
    try:
        d, E = QWEN.dim, QWEN.n_experts
        ffn = np.ctypeslib.as_array(C.cast(lib.ref_mia_ffn_norm(f, 0), C.POINTER(C.c_float)), (d,)).copy()
        router = np.ctypeslib.as_array(C.cast(lib.ref_mia_router(f, 0), C.POINTER(C.c_float)),
                                       (E, d)).copy()
        with MoEEngine(QWEN, n_layers=1) as eng:
            loader = C.cast(lib.ref_mia_read_expert, N.LOADER)  # mia_file_read_expert itself
            e2 = N.errbuf()
            N.check(N.lib().miag_load_experts(eng._ctx, loader, C.c_void_p(f), e2, len(e2)), e2,
                    "miag_load_experts")
            eng.set_layer(0, ffn, router)
            x = synth.tokens(QWEN, 31, 40)
            out = eng.moe(x)
        want, _, _ = r.moe(QWEN, ffn, router, None, lay.blobs, x, threads=n_threads())
        errs = [rel_l2(g - a, w - a) for g, w, a in zip(out, want, x)]
        exact = np.mean([np.array_equal(g.view(np.uint32), w.view(np.uint32)) for g, w in zip(out, want)])
        print(f".mia block: max rel-L2 {max(errs):.2e}, bit-exact tokens {exact:.2f}")
        assert max(errs) <= 1e-3
        assert exact >= 0.5
    finally:
        lib.ref_mia_close(f)
