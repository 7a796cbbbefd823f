"""Generates tests/golden/moe_golden.npz from the reference engine itself.

    make -C oracle && python tests/golden/make_golden.py

The reference (nextocodeoficial/motorIa) is compiled from its own sources by
oracle/Makefile into oracle/_ref/libmia_ref.so; this script feeds it the
seeded synthetic inputs of motoria_b200.synth and stores what it returns, so
the oracle restatement and the GPU kernels can be checked on machines where
the reference tree is absent.  Stored per case: a SHA-256 of the inputs (to
prove the generator reproduces them), the routing of every token (indices and
weight bits) and the block output of the first tokens (float32 bits).
"""

from __future__ import annotations

import hashlib
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from motoria_b200 import synth  # noqa: E402
from oracle import oracle as O  # noqa: E402

SEED, XSEED = 1234, 99
OUT_TOKENS = 8  # block outputs stored per case

# name -> (shape, T tokens, RMS-normalised x, Zipf bias)
CASES = {
    "tiny": (synth.TINY, 64, True, False),
    "tiny_zipf": (synth.TINY, 64, False, True),
    "config1": (synth.QWEN3_30B_A3B, 1, True, False),
    "config2": (synth.QWEN3_30B_A3B, 64, True, False),
    "config3": (synth.QWEN3_30B_A3B, 2048, False, True),
}


def digest(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        if a is not None:
            h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def main() -> None:
    O.build()
    ref = O.ref()
    if ref is None:
        raise SystemExit("oracle/_ref/libmia_ref.so missing: the reference tree is needed")
    out = {}
    for name, (shape, T, rms, zipf) in CASES.items():
        lay = synth.layer(shape, SEED, zipf=zipf)
        x = synth.tokens(shape, XSEED, T, rms_normalise=rms)
        out[f"{name}/input_sha256"] = np.array(
            digest(lay.ffn_norm, lay.router, lay.bias, lay.blobs, x))
        idx, w = ref.route(shape, lay.ffn_norm, lay.router, lay.bias, x, threads=8)
        n = min(T, OUT_TOKENS)
        xo, idx2, w2 = ref.moe(shape, lay.ffn_norm, lay.router, lay.bias, lay.blobs, x[:n],
                               threads=8)
        assert np.array_equal(idx[:n], idx2) and np.array_equal(w[:n].view(np.uint32),
                                                                w2.view(np.uint32))
        out[f"{name}/idx"] = idx.astype(np.int16)
        out[f"{name}/w_bits"] = w.view(np.uint32)
        out[f"{name}/out_bits"] = xo.view(np.uint32)
        print(f"{name}: T={T} first idx {idx[0].tolist()}")
    np.savez_compressed(Path(__file__).with_name("moe_golden.npz"), **out)


if __name__ == "__main__":
    main()
