"""Writing .mia model files through libmiag (miag_mia_write): the
reference's converter output (tools/internal/mia/format.go:200-263), which
its engine reads with mia_file_open (src/storage/mia_file.c:41-111).

    write_mia(path, config, dense, expert, tokenizer=b"")

config   MiaConfig (the header's model fields)
dense    dense(name, n) -> float32 array of n values: token_embd,
         blk.<l>.attn_norm, wq, wk, wv, wo, q_norm, k_norm, ffn_norm,
         router, output_norm, output (matrices are quantized to Q8_0 by
         the writer, as the reference quantizes)
expert   expert(layer, e) -> uint8 array, the expert's blob in .mia layout
"""

from __future__ import annotations

import ctypes as C

import numpy as np

from . import _native as N


class MiaConfig(C.Structure):
    _fields_ = [("dim", C.c_uint32), ("n_layers", C.c_uint32), ("n_heads", C.c_uint32),
                ("n_kv_heads", C.c_uint32), ("head_dim", C.c_uint32), ("vocab", C.c_uint32),
                ("n_experts", C.c_uint32), ("n_active", C.c_uint32),
                ("expert_hidden", C.c_uint32), ("norm_topk", C.c_uint32),
                ("rope_theta", C.c_float), ("norm_eps", C.c_float)]


DENSE = C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_char_p, C.c_void_p, C.c_size_t)


def expert_blob_bytes(config: MiaConfig) -> int:
    return int(N.lib().miag_mia_expert_blob_bytes(C.byref(config)))


def write_mia(path: str, config: MiaConfig, dense, expert, tokenizer: bytes = b"") -> None:
    nblob = expert_blob_bytes(config)

    def dense_cb(_ctx, name, dst, n):
        try:
            v = np.ascontiguousarray(dense(name.decode(), int(n)), dtype=np.float32).reshape(-1)
            if v.size != n:
                return -1
            C.memmove(dst, v.ctypes.data, v.nbytes)
            return 0
        except Exception:
            return -1

    def expert_cb(_ctx, layer, e, dst):
        try:
            b = np.ascontiguousarray(expert(int(layer), int(e)), dtype=np.uint8).reshape(-1)
            if b.size > nblob:
                return -1
            C.memmove(dst, b.ctypes.data, b.size)
            return 0
        except Exception:
            return -1

    dcb, ecb = DENSE(dense_cb), N.LOADER(expert_cb)
    tok = C.create_string_buffer(tokenizer, len(tokenizer)) if tokenizer else None
    err = N.errbuf()
    rc = N.lib().miag_mia_write(path.encode(), C.byref(config), dcb, ecb, None, tok,
                                len(tokenizer), err, len(err))
    N.check(rc, err, "miag_mia_write")
