"""Seeded synthetic inputs for the Qwen3-30B-A3B MoE block configurations.

No public dataset or checkpoint is involved: every benchmark and parity case
runs on weights and activations generated here from a seed.

Generator: counter-based splitmix64.  Every tensor has its own 64-bit key
derived from (seed, tag, layer, expert, ...); element i of a stream is
``splitmix64(key + i * golden_gamma)``, so any slice can be produced on its
own and the numbers do not depend on generation order.  Normals come from
Box-Muller on two 53-bit uniforms in float64, rounded once to float32.

Distributions (the benchmark configurations):
  * router W  f32 [E][d]          ~ N(0, 0.02)
  * ffn_norm  f32 [d]             = 1
  * experts   Q8_0 (.mia layout)  q uniform integer in [-127, 127],
                                  block scale d = |N(0, 0.02)| / 127
  * x         f32 [T][d]          ~ N(0, 1), optionally RMS-normalised
  * bias      f32 [E]             b_e = 0.5 * ln(1 / (e + 1))   (Zipf-skewed load)
"""

from __future__ import annotations

import concurrent.futures as cf
import os
from dataclasses import dataclass

import numpy as np

GAMMA = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)

TAG_ROUTER, TAG_QW, TAG_DW, TAG_X = 1, 2, 3, 4
MAT_GATE, MAT_UP, MAT_DOWN = 0, 1, 2
QK = 32
BLOCK_BYTES = 36


@dataclass(frozen=True)
class Shape:
    """The MoE fields of a .mia header (include/mia/mia_file.h:10-19)."""

    dim: int = 2048
    n_experts: int = 128
    n_active: int = 8
    expert_hidden: int = 768
    norm_topk: int = 1
    norm_eps: float = 1e-6

    @property
    def off_up(self) -> int:
        mat = self.expert_hidden * (self.dim // QK) * BLOCK_BYTES
        return (mat + 63) // 64 * 64

    @property
    def off_down(self) -> int:
        return 2 * self.off_up

    @property
    def blob_bytes(self) -> int:
        end = self.off_down + self.dim * (self.expert_hidden // QK) * BLOCK_BYTES
        return (end + 16383) // 16384 * 16384


QWEN3_30B_A3B = Shape()
TINY = Shape(dim=64, n_experts=8, n_active=2, expert_hidden=32)  # the reference e2e tiny config


def _mix(z: np.ndarray) -> np.ndarray:
    z = (z ^ (z >> np.uint64(30))) * _M1
    z = (z ^ (z >> np.uint64(27))) * _M2
    return z ^ (z >> np.uint64(31))


def splitmix64(z):
    """One splitmix64 output for state z (state advanced by the gamma first)."""
    with np.errstate(over="ignore"):
        return _mix(np.asarray(z, dtype=np.uint64) + GAMMA)


def key(seed: int, *ids: int) -> np.uint64:
    with np.errstate(over="ignore"):
        k = splitmix64(np.uint64(seed & 0xFFFFFFFFFFFFFFFF))
        for i in ids:
            k = splitmix64(k ^ np.uint64(i & 0xFFFFFFFFFFFFFFFF))
    return np.uint64(k)


def stream_u64(k: np.uint64, n: int, start: int = 0) -> np.ndarray:
    with np.errstate(over="ignore"):
        i = np.arange(start, start + n, dtype=np.uint64)
        return _mix(k + (i + np.uint64(1)) * GAMMA)


def uniform(k: np.uint64, n: int, start: int = 0) -> np.ndarray:
    """float64 uniforms in (0, 1]."""
    u = stream_u64(k, n, start)
    return ((u >> np.uint64(11)).astype(np.float64) + 1.0) * (2.0 ** -53)


def normal(k: np.uint64, n: int) -> np.ndarray:
    """float64 N(0, 1) by Box-Muller; element i uses uniforms 2i and 2i+1."""
    u = uniform(k, 2 * n)
    r = np.sqrt(-2.0 * np.log(u[0::2]))
    return r * np.cos(2.0 * np.pi * u[1::2])


def int8_uniform(k: np.uint64, n: int) -> np.ndarray:
    """Integers uniform on [-127, 127] from 16-bit chunks of the stream."""
    words = stream_u64(k, (n + 3) // 4)
    h = words.view(np.uint16)[:n].astype(np.uint32)
    return (((h * 255) >> 16).astype(np.int16) - 127).astype(np.int8)


def router(shape: Shape, seed: int, layer: int = 0) -> np.ndarray:
    w = normal(key(seed, TAG_ROUTER, layer), shape.n_experts * shape.dim) * 0.02
    return w.astype(np.float32).reshape(shape.n_experts, shape.dim)


def ffn_norm(shape: Shape) -> np.ndarray:
    return np.ones(shape.dim, dtype=np.float32)


def zipf_bias(shape: Shape) -> np.ndarray:
    """b_e = 0.5 * ln(1 / rank_e) with rank_e = e + 1."""
    r = np.arange(1, shape.n_experts + 1, dtype=np.float64)
    return (0.5 * np.log(1.0 / r)).astype(np.float32)


_Q8 = np.dtype([("d", "<f4"), ("q", "i1", (QK,))])


def _q8_matrix(seed: int, layer: int, expert: int, mat: int, rows: int, cols: int) -> np.ndarray:
    nb = rows * (cols // QK)
    blk = np.empty(nb, dtype=_Q8)
    blk["q"] = int8_uniform(key(seed, TAG_QW, layer, expert, mat), nb * QK).reshape(nb, QK)
    d = np.abs(normal(key(seed, TAG_DW, layer, expert, mat), nb)) * 0.02 / 127.0
    blk["d"] = d.astype(np.float32)
    return blk


def expert_blob(shape: Shape, seed: int, layer: int, expert: int, out: np.ndarray | None = None):
    """One expert in .mia layout (gate | up | down; src/storage/mia_file.c:275-278)."""
    if out is None:
        out = np.zeros(shape.blob_bytes, dtype=np.uint8)
    d, eh = shape.dim, shape.expert_hidden
    parts = ((MAT_GATE, 0, eh, d), (MAT_UP, shape.off_up, eh, d), (MAT_DOWN, shape.off_down, d, eh))
    for mat, off, rows, cols in parts:
        b = _q8_matrix(seed, layer, expert, mat, rows, cols).view(np.uint8)
        out[off:off + b.size] = b
    return out


def expert_blobs(shape: Shape, seed: int, layer: int = 0, experts=None) -> np.ndarray:
    """All (or the listed) experts of a layer, [n][blob_bytes] uint8."""
    ids = list(range(shape.n_experts) if experts is None else experts)
    out = np.zeros((len(ids), shape.blob_bytes), dtype=np.uint8)
    workers = max(1, min(len(ids), os.cpu_count() or 1, 16))
    with cf.ThreadPoolExecutor(workers) as ex:  # numpy releases the GIL in the heavy parts
        list(ex.map(lambda ie: expert_blob(shape, seed, layer, ie[1], out[ie[0]]), enumerate(ids)))
    return out


def tokens(shape: Shape, seed: int, T: int, start: int = 0, rms_normalise: bool = True,
           stream: int = 0) -> np.ndarray:
    """x [T][d]: token t's row is its own stream, so slices are consistent."""
    x = np.empty((T, shape.dim), dtype=np.float64)
    for i in range(T):
        x[i] = normal(key(seed, TAG_X, stream, start + i), shape.dim)
    if rms_normalise:
        x /= np.sqrt(np.mean(x * x, axis=1, keepdims=True))
    return x.astype(np.float32)


@dataclass
class Layer:
    shape: Shape
    ffn_norm: np.ndarray
    router: np.ndarray
    bias: np.ndarray | None
    blobs: np.ndarray  # [E][blob_bytes] uint8


def layer(shape: Shape, seed: int, layer_id: int = 0, zipf: bool = False) -> Layer:
    return Layer(shape, ffn_norm(shape), router(shape, seed, layer_id),
                 zipf_bias(shape) if zipf else None, expert_blobs(shape, seed, layer_id))


# The benchmark configurations: (T tokens, RMS-normalised x, Zipf router bias).
CONFIGS = {
    "config1": dict(T=1, rms=True, zipf=False),      # decode of 1 token
    "config2": dict(T=64, rms=True, zipf=False),     # batched decode of 64 tokens
    "config3": dict(T=2048, rms=False, zipf=True),   # prefill, Zipf-skewed expert load
    "config5": dict(T=4096, rms=False, zipf=True),   # expert-parallel, per GPU
}
