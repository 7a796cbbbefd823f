"""The whole decode step against the reference engine's own mia_model_step
(src/model/forward.c:199-217), on .mia files written by miag_mia_write and
opened by the reference's reader (mia_file_open) on one side and by
miag_model_open_file on the other.  The GPU repeats the reference's
arithmetic operation for operation, so:
  * against the reference built with a correctly rounded expf (oracle/
    crexp.h; the value the GPU computes), logits are equal bit for bit at
    every position;
  * against the stock build, glibc's expf misrounds a few inputs in a
    million; each such call moves a value by an ulp, and the KV cache carries
    it to later positions.  Logits stay within 1e-4 relative to the largest
    (the reference's own e2e precedent allows 3e-2, tools/e2e_test.go:83-85).

Cases: "tiny" (dim 64, 4/2 heads of 16, vocab 100, 8 experts top-2) runs
past 512 positions, so the attention kernel's position slices (256) and V
tiles (64) all wrap; "qwen_heads" has Qwen3-30B-A3B's attention and expert
shapes (dim 2048, 32/4 heads of 128, experts 768 wide, top-8 of 16) over
two layers and a 1000-token vocabulary."""

from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from motoria_b200 import build, synth
from motoria_b200 import _native as N
from motoria_b200.mia import MiaConfig, write_mia
from motoria_b200.model import Model
from oracle import oracle as O

pytestmark = pytest.mark.gpu

CASES = {
    "tiny": dict(cfg=dict(dim=64, n_layers=2, n_heads=4, n_kv_heads=2, head_dim=16, vocab=100,
                          n_experts=8, n_active=2, expert_hidden=32, norm_topk=1,
                          rope_theta=10000.0, norm_eps=1e-6),
                 steps=530, max_seq=600),
    "qwen_heads": dict(cfg=dict(dim=2048, n_layers=2, n_heads=32, n_kv_heads=4, head_dim=128,
                                vocab=1000, n_experts=16, n_active=8, expert_hidden=768,
                                norm_topk=1, rope_theta=1e6, norm_eps=1e-6),
                       steps=40, max_seq=128),
}


def write_model(path: str, cfg: MiaConfig, seed: int) -> None:
    """Random f32 dense tensors (the writer quantizes the matrices) and
    synth.py experts."""
    rng = np.random.default_rng(seed)
    shape = synth.Shape(dim=cfg.dim, n_experts=cfg.n_experts, n_active=cfg.n_active,
                        expert_hidden=cfg.expert_hidden)

    def dense(name, n):
        base = name.split(".")[-1]
        if base.endswith("norm"):
            return (1.0 + 0.1 * rng.standard_normal(n)).astype(np.float32)
        if base == "router":
            return (0.02 * rng.standard_normal(n)).astype(np.float32)
        cols = cfg.n_heads * cfg.head_dim if base == "wo" else cfg.dim
        scale = 1.0 if base == "token_embd" else 1.0 / np.sqrt(cols)
        return (scale * rng.standard_normal(n)).astype(np.float32)

    write_mia(path, cfg, dense, lambda l, e: synth.expert_blob(shape, seed, l, e))


STOCK_RTOL = 1e-4  # max |gpu - ref| / max |ref| per position, stock glibc expf


class RefModel:
    """The reference's model step (oracle/_ref harness: ref_model_*)."""

    def __init__(self, r, path: str, max_seq: int, vocab: int):
        self.lib = lib = r.dll
        lib.ref_model_open.restype = C.c_void_p
        lib.ref_model_open.argtypes = [C.c_char_p, C.c_int, C.c_char_p, C.c_size_t]
        lib.ref_model_step.restype = C.c_void_p
        lib.ref_model_step.argtypes = [C.c_void_p, C.c_int, C.c_int]
        lib.ref_model_close.argtypes = [C.c_void_p]
        err = C.create_string_buffer(256)
        self.h = lib.ref_model_open(path.encode(), max_seq, err, 256)
        assert self.h, err.value
        self.vocab = vocab

    def step(self, token: int, pos: int) -> np.ndarray:
        p = self.lib.ref_model_step(self.h, token, pos)
        assert p, "mia_model_step returned NULL"
        return np.ctypeslib.as_array(C.cast(p, C.POINTER(C.c_float)), (self.vocab,)).copy()

    def close(self):
        self.lib.ref_model_close(self.h)


@pytest.fixture(scope="module", params=list(CASES))
def models(request, tmp_path_factory, torch_cuda):
    build.build()
    if O.ref() is None or O.ref_crexp() is None:
        pytest.skip("the reference builds (oracle/_ref) are absent")
    case = CASES[request.param]
    cfg = MiaConfig(**case["cfg"])
    path = str(tmp_path_factory.mktemp("model") / f"{request.param}.mia")
    write_model(path, cfg, seed=4242)
    stock = RefModel(O.ref(), path, case["max_seq"], cfg.vocab)
    crexp = RefModel(O.ref_crexp(), path, case["max_seq"], cfg.vocab)
    gpu = Model.open_file(path, device=0, max_seq=case["max_seq"])
    yield request.param, case, cfg, stock, crexp, gpu
    gpu.close()
    crexp.close()
    stock.close()


def rel_max(got, want):
    return float(np.max(np.abs(got - want)) / max(np.max(np.abs(want)), 1e-30))


def test_step_logits_equal_the_reference(models):
    name, case, cfg, stock, crexp, gpu = models
    rng = np.random.default_rng(7)
    tokens = rng.integers(0, cfg.vocab, size=case["steps"])
    first_cr, n_stock_exact, worst_stock = None, 0, 0.0
    for pos, tok in enumerate(tokens):
        want_cr = crexp.step(int(tok), pos)
        want = stock.step(int(tok), pos)
        got = gpu.step(int(tok), pos)
        assert np.all(np.isfinite(got))
        if first_cr is None and not np.array_equal(got.view(np.uint32), want_cr.view(np.uint32)):
            first_cr = (pos, rel_max(got, want_cr))
        if np.array_equal(got.view(np.uint32), want.view(np.uint32)):
            n_stock_exact += 1
        worst_stock = max(worst_stock, rel_max(got, want))
    print(f"{name}: {case['steps']} positions; vs the correctly rounded expf build: first "
          f"difference {first_cr}; vs the stock build: {n_stock_exact} positions bit-exact, "
          f"worst rel-max {worst_stock:.2e}")
    assert first_cr is None
    assert worst_stock <= STOCK_RTOL


def test_greedy_generation_equals_the_reference_loop(models):
    name, case, cfg, _, ref, gpu = models
    rng = np.random.default_rng(11)
    n_prompt, n_new = 9, 12
    prompt = rng.integers(0, cfg.vocab, size=n_prompt).astype(np.int32)
    logits = None
    for p, t in enumerate(prompt):
        logits = ref.step(int(t), p)
    want = []
    for i in range(n_new):
        t = int(np.argmax(logits))  # the lowest index among equal maxima
        want.append(t)
        if i + 1 < n_new:
            logits = ref.step(t, n_prompt + i)
    got = gpu.generate(prompt, n_new)
    assert got.tolist() == want


PREFILL = {"tiny": (70, 37), "qwen_heads": (33, 5)}  # prompt length, second chunk


def test_prefill_equals_single_steps(models):
    """A prompt in one batched pass (miag_model_prefill) leaves the logits of
    its last position, and the KV cache the next steps read, equal bit for
    bit to the reference's one step per position; a second chunk prefilled
    from a later position likewise."""
    name, case, cfg, _, ref, gpu = models
    n1, n2 = PREFILL[name]
    rng = np.random.default_rng(23)
    toks = rng.integers(0, cfg.vocab, size=n1 + 1 + n2).astype(np.int32)
    want = None
    for pos in range(n1):
        want = ref.step(int(toks[pos]), pos)
    got = gpu.prefill(toks[:n1], 0)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), \
        f"{name}: prefill logits differ, rel-max {rel_max(got, want):.2e}"
    # one ordinary step after the prefill reads the prefilled cache
    want = ref.step(int(toks[n1]), n1)
    got = gpu.step(int(toks[n1]), n1)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    # a second chunk from position n1 + 1
    for pos in range(n1 + 1, n1 + 1 + n2):
        want = ref.step(int(toks[pos]), pos)
    got = gpu.prefill(toks[n1 + 1:], n1 + 1)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_generation_with_and_without_batched_prefill(models):
    """generate() runs its prompt batched by default; one step per position
    gives the same tokens."""
    name, case, cfg, _, ref, gpu = models
    rng = np.random.default_rng(31)
    prompt = rng.integers(0, cfg.vocab, size=PREFILL[name][0]).astype(np.int32)
    a = gpu.generate(prompt, 6)
    gpu.set_batched_prefill(False)
    try:
        b = gpu.generate(prompt, 6)
    finally:
        gpu.set_batched_prefill(True)
    assert a.tolist() == b.tolist()
    assert gpu.prefill_launches >= 2 + cfg.n_layers * 8


class MiaSampler(C.Structure):
    """mia_sampler (include/mia/sampler.h)."""

    _fields_ = [("temperature", C.c_float), ("top_p", C.c_float), ("n", C.c_int),
                ("rng", C.c_uint64), ("buf", C.c_void_p)]


def reference_sampled_loop(ref: RefModel, prompt, n_new, temp, top_p, seed, vocab):
    """The generation loop of src/app/main.c:118-141: the prompt one step a
    position, then mia_sample on a copy of the logits and a step with the
    drawn token."""
    lib = ref.lib
    lib.mia_sampler_init.argtypes = [C.POINTER(MiaSampler), C.c_float, C.c_float, C.c_int, C.c_uint64]
    lib.mia_sample.argtypes = [C.POINTER(MiaSampler), C.POINTER(C.c_float)]
    lib.mia_sample.restype = C.c_int
    lib.mia_sampler_free.argtypes = [C.POINTER(MiaSampler)]
    smp = MiaSampler()
    assert lib.mia_sampler_init(C.byref(smp), temp, top_p, vocab, seed) == 0
    logits = None
    for p, t in enumerate(prompt):
        logits = ref.step(int(t), p)
    out = []
    for i in range(n_new):
        work = np.ascontiguousarray(logits, dtype=np.float32).copy()
        t = lib.mia_sample(C.byref(smp), work.ctypes.data_as(C.POINTER(C.c_float)))
        out.append(int(t))
        if i + 1 < n_new:
            logits = ref.step(t, len(prompt) + i)
    lib.mia_sampler_free(C.byref(smp))
    return out


@pytest.mark.parametrize("temp,top_p,seed,batched", [(0.7, 0.8, 42, True), (1.3, 1.0, 0, True),
                                                     (0.9, 0.5, 7, False)])
def test_sampled_generation_equals_the_reference_sampler(models, temp, top_p, seed, batched):
    """Temperature / top-p sampling on the device draws the same tokens as
    the reference's mia_sample (sampler.c:33-66) in its generation loop,
    with the same seed; the prompt batched or one step a position."""
    name, case, cfg, _, ref, gpu = models
    rng = np.random.default_rng(41)
    prompt = rng.integers(0, cfg.vocab, size=7).astype(np.int32)
    n_new = 12
    want = reference_sampled_loop(ref, prompt, n_new, temp, top_p, seed, cfg.vocab)
    gpu.set_sampler(temp, top_p, seed)
    gpu.set_batched_prefill(batched)
    try:
        got = gpu.generate(prompt, n_new)
    finally:
        gpu.set_sampler(0.0)
        gpu.set_batched_prefill(True)
    assert got.tolist() == want, f"{name}: {got.tolist()} vs {want}"


def test_long_prefill_equals_single_steps(tmp_path, torch_cuda):
    """A prompt past the tiled prefill attention's 1280 positions (the
    kernel with one CTA per head and position takes it) and one below it,
    on the tiny shapes: the last logits equal the reference's step loop."""
    build.build()
    if O.ref_crexp() is None:
        pytest.skip("the reference builds (oracle/_ref) are absent")
    cfg = MiaConfig(**CASES["tiny"]["cfg"])
    path = str(tmp_path / "tiny_long.mia")
    write_model(path, cfg, seed=515)
    max_seq = 1400
    ref = RefModel(O.ref_crexp(), path, max_seq, cfg.vocab)
    toks = np.random.default_rng(3).integers(0, cfg.vocab, size=1330).astype(np.int32)
    want = {}
    for pos, t in enumerate(toks):
        logits = ref.step(int(t), pos)
        if pos + 1 in (1000, 1330):
            want[pos + 1] = logits
    ref.close()
    with Model.open_file(path, device=0, max_seq=max_seq) as gpu:
        for n in (1000, 1330):
            got = gpu.prefill(toks[:n], 0)
            assert np.array_equal(got.view(np.uint32), want[n].view(np.uint32)), n


def test_prefill_rejects_bad_arguments(models):
    name, case, cfg, _, ref, gpu = models
    with pytest.raises(N.MiagError):
        gpu.prefill(np.array([0, cfg.vocab], np.int32), 0)  # token out of range
    with pytest.raises(N.MiagError):
        gpu.prefill(np.zeros(4, np.int32), case["max_seq"] - 3)  # past the context
    with pytest.raises(N.MiagError):
        gpu.prefill(np.zeros(0, np.int32), 0)
    want = ref.step(3, 0)
    got = gpu.step(3, 0)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_out_of_range_steps_fail_and_leave_the_model_usable(models):
    name, case, cfg, _, ref, gpu = models
    for tok, pos in ((-1, 0), (cfg.vocab, 0), (0, -1), (0, case["max_seq"])):
        with pytest.raises(N.MiagError):
            gpu.step(tok, pos)
    want = ref.step(3, 0)
    got = gpu.step(3, 0)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_synthetic_model_runs_and_replays_identically(torch_cuda):
    build.build()
    cfg = MiaConfig(**CASES["tiny"]["cfg"])
    with Model.synthetic(cfg, seed=5, max_seq=64) as m:
        a = [m.step(t, p) for p, t in enumerate((1, 2, 3, 4))]
        b = [m.step(t, p) for p, t in enumerate((1, 2, 3, 4))]
        for x, y in zip(a, b):
            assert np.all(np.isfinite(x))
            assert np.array_equal(x.view(np.uint32), y.view(np.uint32))
        assert m.launches_per_step >= 2 + cfg.n_layers * 4
