"""The whole decode step on the GPU (miag_model_*): the reference engine's
model state and layer loop (mia_model_init / mia_model_step,
src/model/forward.c:36-62, 199-217) with the dense weights, the KV cache and
the experts in HBM.

    m = Model.open_file("model.mia", max_seq=4096)     # a converted Q8_0 model
    logits = m.step(token, pos)                        # mia_model_step
    new = m.generate(prompt, n_new)                    # prompt, then greedy tokens

    m = Model.synthetic(config, seed, max_seq)         # seeded random weights
"""

from __future__ import annotations

import ctypes as C

import numpy as np

from . import _native as N
from .mia import MiaConfig


def moe_shape(config: MiaConfig) -> N.Shape:
    return N.Shape(config.dim, config.n_layers, config.n_experts, config.n_active,
                   config.expert_hidden, config.norm_topk, config.norm_eps)


class Model:
    def __init__(self, handle: int, vocab: int, ctx: int | None = None):
        self._m = handle
        self._ctx = ctx  # a context this object opened, closed with the model
        self.vocab = vocab

    @classmethod
    def open_file(cls, path: str, device: int = 0, max_seq: int = 4096) -> "Model":
        out = C.c_void_p()
        err = N.errbuf()
        N.check(N.lib().miag_model_open_file(C.byref(out), path.encode(), device, max_seq, err,
                                             len(err)), err, "miag_model_open_file")
        vocab = _read_vocab(path)
        return cls(out.value, vocab)

    @classmethod
    def synthetic(cls, config: MiaConfig, seed: int, max_seq: int, device: int = 0) -> "Model":
        lib = N.lib()
        err = N.errbuf()
        ctx = C.c_void_p()
        shape = moe_shape(config)
        N.check(lib.miag_open(C.byref(ctx), C.byref(shape), device, err, len(err)), err, "miag_open")
        out = C.c_void_p()
        rc = lib.miag_model_open(C.byref(out), ctx, C.byref(config), None, 0, max_seq, err, len(err))
        if rc != 0:
            lib.miag_close(ctx)
            N.check(rc, err, "miag_model_open")
        m = cls(out.value, int(config.vocab), ctx.value)
        try:
            N.check(lib.miag_model_synth(m._m, seed, err, len(err)), err, "miag_model_synth")
        except Exception:
            m.close()
            raise
        return m

    @property
    def handle(self) -> int:
        return self._m

    def close(self) -> None:
        if self._m:
            N.lib().miag_model_close(self._m)
            self._m = None
        if self._ctx:
            N.lib().miag_close(self._ctx)
            self._ctx = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def step(self, token: int, pos: int) -> np.ndarray:
        """Logits [vocab] f32 after token at pos (a copy)."""
        err = N.errbuf()
        p = N.lib().miag_model_step(self._m, int(token), int(pos), err, len(err))
        if not p:
            raise N.MiagError(f"miag_model_step: {err.value.decode(errors='replace')}")
        return np.ctypeslib.as_array(C.cast(p, C.POINTER(C.c_float)), (self.vocab,)).copy()

    def generate(self, prompt, n_new: int) -> np.ndarray:
        """The prompt one position at a time, then n_new greedy tokens."""
        pr = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.zeros(max(n_new, 1), np.int32)
        err = N.errbuf()
        N.check(N.lib().miag_model_generate(self._m, pr.ctypes.data, pr.size, n_new,
                                            out.ctypes.data, err, len(err)), err,
                "miag_model_generate")
        return out[:n_new]

    def generate_async(self, prompt, n_new: int) -> None:
        pr = np.ascontiguousarray(prompt, dtype=np.int32)
        err = N.errbuf()
        N.check(N.lib().miag_model_generate_async(self._m, pr.ctypes.data, pr.size, n_new, err,
                                                  len(err)), err, "miag_model_generate_async")

    def continue_async(self, n_steps: int) -> None:
        err = N.errbuf()
        N.check(N.lib().miag_model_continue_async(self._m, n_steps, err, len(err)), err,
                "miag_model_continue_async")

    def sync(self) -> None:
        err = N.errbuf()
        N.check(N.lib().miag_model_sync(self._m, err, len(err)), err, "miag_model_sync")

    def prefill_async(self, tokens, pos: int = 0) -> None:
        """Positions pos .. pos + len(tokens) - 1 in one batched pass; the
        last position's logits and the next (greedy) token stay on the
        device (miag_model_prefill_async)."""
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        err = N.errbuf()
        N.check(N.lib().miag_model_prefill_async(self._m, t.ctypes.data, t.size, int(pos), err,
                                                 len(err)), err, "miag_model_prefill_async")

    def prefill(self, tokens, pos: int = 0) -> np.ndarray:
        """The positions in one batched pass; the last position's logits
        [vocab] (a copy), as miag_model_step returns one position's."""
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        err = N.errbuf()
        p = N.lib().miag_model_prefill(self._m, t.ctypes.data, t.size, int(pos), err, len(err))
        if not p:
            raise N.MiagError(f"miag_model_prefill: {err.value.decode(errors='replace')}")
        return np.ctypeslib.as_array(C.cast(p, C.POINTER(C.c_float)), (self.vocab,)).copy()

    def set_sampler(self, temperature: float, top_p: float = 1.0, seed: int = 0) -> None:
        """Draw each next token as mia_sample does (temperature > 0), or take
        the greedy argmax (temperature <= 0, the default)."""
        err = N.errbuf()
        N.check(N.lib().miag_model_set_sampler(self._m, float(temperature), float(top_p), int(seed),
                                               err, len(err)), err, "miag_model_set_sampler")

    def set_batched_prefill(self, on: bool) -> None:
        N.lib().miag_model_set_batched_prefill(self._m, int(bool(on)))

    @property
    def prefill_launches(self) -> int:
        return N.lib().miag_model_prefill_launches(self._m)

    @property
    def stream(self) -> int:
        return N.lib().miag_model_stream(self._m) or 0

    @property
    def tokens_device(self) -> int:
        return N.lib().miag_model_tokens_device(self._m)

    @property
    def uses_graph(self) -> bool:
        return bool(N.lib().miag_model_uses_graph(self._m))

    @property
    def launches_per_step(self) -> int:
        return N.lib().miag_model_launches_per_step(self._m)


def _read_vocab(path: str) -> int:
    with open(path, "rb") as f:
        h = f.read(112)
    return int(np.frombuffer(h, dtype="<u4", count=1, offset=32)[0])  # mia_header.vocab
