"""The C-ABI boundary without a GPU: libmiag loads, exports every symbol the
public header declares, sizes blobs like the reference format, and rejects
bad shapes / a missing GPU with -1 and a message instead of crashing."""

from __future__ import annotations

import ctypes as C
import re
from pathlib import Path

import pytest

from conftest import ROOT
from motoria_b200 import _native as N
from motoria_b200 import build, synth
from motoria_b200.engine import blob_bytes

HEADER = ROOT / "include" / "miag" / "miag.h"


def declared_symbols():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(miag_[a-z0-9_]+)\s*\(", text)) - {"miag_expert_loader"})


@pytest.fixture(scope="module")
def lib():
    build.build()
    return N.lib()


def test_library_exports_every_declared_symbol(lib):
    syms = declared_symbols()
    assert len(syms) >= 12
    for s in syms:
        assert hasattr(lib, s), s
    assert sorted(N.SIGNATURES) == syms


def test_blob_bytes_matches_mia_layout(lib):
    # 768 x 2048 Q8_0 = 1,769,472 B per matrix; three matrices; 16 KiB aligned
    assert blob_bytes(synth.QWEN3_30B_A3B) == 5_308_416 == synth.QWEN3_30B_A3B.blob_bytes
    assert blob_bytes(synth.TINY) == synth.TINY.blob_bytes


@pytest.mark.parametrize("kw", [dict(dim=100), dict(n_active=65, n_experts=128),
                                dict(expert_hidden=0), dict(n_experts=2000)])
def test_bad_shapes_are_rejected(lib, kw):
    base = dict(dim=2048, n_layers=1, n_experts=128, n_active=8, expert_hidden=768,
                norm_topk=1, norm_eps=1e-6)
    base.update(kw)
    s = N.Shape(**base)
    ctx = C.c_void_p()
    err = N.errbuf()
    assert lib.miag_open(C.byref(ctx), C.byref(s), 0, err, len(err)) == -1
    assert b"unsupported" in err.value and not ctx.value


def test_open_without_gpu_fails_cleanly(lib):
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    s = N.Shape(2048, 1, 128, 8, 768, 1, 1e-6)
    ctx = C.c_void_p()
    err = N.errbuf()
    assert lib.miag_open(C.byref(ctx), C.byref(s), 0, err, len(err)) == -1
    assert err.value  # message, no crash, no CPU fallback


def test_null_arguments_are_errors(lib):
    err = N.errbuf()
    assert lib.miag_moe(None, 0, None, 1, err, len(err)) == -1
    assert lib.miag_quantize_row_q8(None, None, 32, None) == -1
    assert lib.miag_matvec(None, None, 1, None, None, 4, 32, None) == -1


def test_nccl_loads_and_the_expert_parallel_block_rejects_bad_arguments(lib):
    """libmiag finds NCCL at run time (an id needs no GPU) and its
    expert-parallel entry points refuse null arguments with a message."""
    buf = C.create_string_buffer(128)
    err = N.errbuf()
    assert lib.miag_nccl_unique_id(buf, err, len(err)) == 0, err.value
    assert any(buf.raw)
    ep = C.c_void_p()
    assert lib.miag_ep_open(C.byref(ep), None, None, 0, err, len(err)) == -1
    assert b"null" in err.value
    assert lib.miag_moe_ep_async(None, 0, None, 0, None, err, len(err)) == -1
    assert lib.miag_moe_ep(None, 0, None, 0, err, len(err)) == -1
    lib.miag_ep_close(None)  # a no-op
