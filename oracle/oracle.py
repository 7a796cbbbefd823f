"""Python binding of the CPU oracle -- TEST INFRASTRUCTURE ONLY.

Loads ``oracle/lib/libmoe_oracle.so`` (the C restatement, moe_oracle.c) and,
when it was built, ``oracle/_ref/libmia_ref.so`` (the reference engine's own
sources driven by ref_harness.c) and its diagnostic twin
``oracle/_ref/libmia_ref_crexp.so`` (the same, with a correctly rounded expf).  Only tests/, the smoke check and the
cpu_baseline leg of bench.py use this module, always as the checker.

``build()`` runs ``make -C oracle``; on a machine without the reference tree
only the restatement is built and ``ref()`` returns None.
"""

from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "lib" / "libmoe_oracle.so"
REF_SO = HERE / "_ref" / "libmia_ref.so"
# the same reference build with expf correctly rounded (crexp.h): a diagnostic
REF_CREXP_SO = HERE / "_ref" / "libmia_ref_crexp.so"


class OShape(C.Structure):
    """orc_shape / ref_shape."""

    _fields_ = [("dim", C.c_int32), ("n_experts", C.c_int32), ("n_active", C.c_int32),
                ("expert_hidden", C.c_int32), ("norm_topk", C.c_int32), ("norm_eps", C.c_float)]


def reference_tree() -> str | None:
    """Where the reference sources lie: $MIA_REFERENCE, else BASELINE.json's
    reference_path; None when neither names an existing tree (the GPU box)."""
    import json
    import os

    cand = os.environ.get("MIA_REFERENCE")
    if not cand:
        try:
            cand = json.loads((HERE.parent / "BASELINE.json").read_text()).get("reference_path")
        except (OSError, ValueError):
            cand = None
    if cand and (Path(cand) / "src" / "model" / "forward.c").exists():
        return cand
    return None


def build() -> None:
    cmd = ["make", "-s", "-C", str(HERE)]
    tree = reference_tree()
    if tree:
        cmd.append(f"REF={tree}")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"oracle build failed:\n{r.stdout}\n{r.stderr}")


def _p(a):
    return None if a is None else C.c_void_p(a.ctypes.data)


class _Lib:
    """Common calls of the restatement (prefix orc_) and the reference (ref_)."""

    def __init__(self, path: Path, prefix: str):
        self.dll = C.CDLL(str(path))
        self.prefix = prefix
        self.kind = "port" if prefix == "orc_" else "reference"

    def fn(self, name):
        return getattr(self.dll, self.prefix + name)

    def moe(self, shape, ffn_norm, router, bias, blobs, x, threads=1):
        """x + MoE(x) for x [T][d]; returns (x_out, idx [T][K], w [T][K])."""
        s = OShape(shape.dim, shape.n_experts, shape.n_active, shape.expert_hidden,
                   shape.norm_topk, shape.norm_eps)
        xo = np.array(x, dtype=np.float32, order="C", copy=True)
        T = xo.shape[0]
        idx = np.zeros((T, shape.n_active), np.int32)
        w = np.zeros((T, shape.n_active), np.float32)
        fn = self.fn("moe")
        fn.restype = C.c_int
        rc = fn(C.byref(s), _p(np.ascontiguousarray(ffn_norm, np.float32)),
                _p(np.ascontiguousarray(router, np.float32)),
                None if bias is None else _p(np.ascontiguousarray(bias, np.float32)),
                _p(blobs), C.c_size_t(blobs.shape[1]), _p(xo), T, _p(idx), _p(w), threads)
        if rc != 0:
            raise RuntimeError(f"{self.prefix}moe failed")
        return xo, idx, w

    def route(self, shape, ffn_norm, router, bias, x, threads=1):
        s = OShape(shape.dim, shape.n_experts, shape.n_active, shape.expert_hidden,
                   shape.norm_topk, shape.norm_eps)
        xi = np.ascontiguousarray(x, dtype=np.float32)
        T = xi.shape[0]
        idx = np.zeros((T, shape.n_active), np.int32)
        w = np.zeros((T, shape.n_active), np.float32)
        fn = self.fn("route" if self.prefix == "ref_" else "route_batch")
        fn.restype = C.c_int
        rc = fn(C.byref(s), _p(np.ascontiguousarray(ffn_norm, np.float32)),
                _p(np.ascontiguousarray(router, np.float32)),
                None if bias is None else _p(np.ascontiguousarray(bias, np.float32)),
                _p(xi), T, _p(idx), _p(w), threads)
        if rc != 0:
            raise RuntimeError(f"{self.prefix}route failed")
        return idx, w

    def quantize_row_q8(self, x):
        x = np.ascontiguousarray(x, np.float32)
        y = np.zeros(x.size // 32 * 36, np.uint8)
        self.fn("quantize_row_q8")(_p(x), _p(y), x.size)
        return y

    def rmsnorm(self, x, w, eps):
        x = np.ascontiguousarray(x, np.float32)
        out = np.zeros_like(x)
        self.fn("rmsnorm")(_p(out), _p(x), _p(np.ascontiguousarray(w, np.float32)), x.size,
                           C.c_float(eps))
        return out

    def softmax(self, x):
        y = np.array(x, np.float32, copy=True)
        self.fn("softmax")(_p(y), y.size)
        return y

    def top_k(self, p, k):
        p = np.ascontiguousarray(p, np.float32)
        idx = np.zeros(k, np.int32)
        self.fn("top_k")(_p(p), p.size, k, _p(idx))
        return idx


class Oracle(_Lib):
    def __init__(self):
        super().__init__(ORACLE_SO, "orc_")

    def matvec_q8(self, w_blocks, x, rows, cols):
        out = np.zeros(rows, np.float32)
        xq = np.zeros(cols // 32 * 36, np.uint8)
        self.dll.orc_matvec_q8(_p(out), _p(w_blocks), _p(np.ascontiguousarray(x, np.float32)),
                               _p(xq), rows, cols)
        return out

    def matvec_f32(self, w, x):
        w = np.ascontiguousarray(w, np.float32)
        out = np.zeros(w.shape[0], np.float32)
        self.dll.orc_matvec_f32(_p(out), _p(w), _p(np.ascontiguousarray(x, np.float32)),
                                w.shape[0], w.shape[1])
        return out

    def permute(self, idx, E):
        idx = np.ascontiguousarray(idx, np.int32)
        T, K = idx.shape
        counts = np.zeros(E, np.int32)
        offsets = np.zeros(E + 1, np.int32)
        perm = np.zeros(T * K, np.int32)
        inv = np.zeros(T * K, np.int32)
        self.dll.orc_permute(_p(idx), T, K, E, _p(counts), _p(offsets), _p(perm), _p(inv))
        return dict(counts=counts, offsets=offsets, perm=perm, inv=inv)


class Ref(_Lib):
    def __init__(self, path: Path = REF_SO):
        super().__init__(path, "ref_")

    def matvec(self, w, wtype, x, rows, cols, scalar=False):
        out = np.zeros(rows, np.float32)
        xq = np.zeros(max(cols // 32, 1) * 36, np.uint8)
        fn = self.dll.ref_matvec_scalar if scalar else self.dll.ref_matvec
        fn(_p(out), _p(np.ascontiguousarray(w)), wtype, _p(np.ascontiguousarray(x, np.float32)),
           _p(xq), rows, cols)
        return out


_oracle = None
_ref = None


def oracle() -> Oracle:
    global _oracle
    if _oracle is None:
        if not ORACLE_SO.exists():
            build()
        _oracle = Oracle()
    return _oracle


def ref() -> Ref | None:
    """The reference build, or None where it was never compiled."""
    global _ref
    if _ref is None and REF_SO.exists():
        _ref = Ref()
    return _ref


_ref_crexp = None


def ref_crexp() -> Ref | None:
    """The reference build with expf correctly rounded, or None."""
    global _ref_crexp
    if _ref_crexp is None and REF_CREXP_SO.exists():
        _ref_crexp = Ref(REF_CREXP_SO)
    return _ref_crexp
