"""Sampling with the reference's own random stream (no GPU): the host sampler
``yuf_sample_host`` / ``yuf_mt19937_*`` and its oracle (oracle/sampler.py)
against draws the reference itself made -- ``sample_token`` of
yufmusicgen/cli/generate.py:45-56 after ``torch.manual_seed``, on rows masked
as its loop masks them (tests/golden/sampler_torch_cpu.npz, written by
tests/golden/make_golden.py on an x86-64 host with AVX-512; the tokens depend
on torch's CPU sort order for equal logits, which the sampler reproduces, and
on float probabilities that may differ in the last bit from torch's vectorised
exp, which can only matter at an exact tie of two keys).

Known answers of MT19937 itself: with seed 5489 the first word is 3499211612
and the 10000th is 4123659995 (the values the C++ standard requires of
std::mt19937).
"""

import numpy as np
import pytest

from oracle.sampler import MT19937, sample_torch_cpu
from yufmusicgen_b200 import _lib
from yufmusicgen_b200.sampler import TorchCpuGenerator, mask_like_reference

FIX = "sampler_torch_cpu.npz"


def test_mt19937_known_answers():
    for words in (TorchCpuGenerator(5489).next_u32(10000), MT19937(5489).u32(10000)):
        assert words[0] == 3499211612 and words[9999] == 4123659995


def test_exponential_draws_equal_torch(golden):
    g = golden(FIX)
    want = g["exp_draws_seed1337"]
    np.testing.assert_array_equal(TorchCpuGenerator(1337).exponential(want.size), want)
    np.testing.assert_array_equal(MT19937(1337).exponential(want.size), want)
    # the stream continues across calls exactly as one long draw
    gen = TorchCpuGenerator(1337)
    np.testing.assert_array_equal(np.concatenate([gen.exponential(1000), gen.exponential(2000)]), want)


@pytest.mark.parametrize("case", ["v20000_t1_p095", "v20000_t08_p05", "v673_t13_p1", "v673_t1_p09_peaked",
                                  "v673_greedy"])
def test_tokens_equal_the_references_draws(golden, case):
    g = golden(FIX)
    temp, top_p = g[f"{case}.knobs"]
    rows = g[f"{case}.logits"].astype(np.float32)
    seed = int(g[f"{case}.seed"])
    want = g[f"{case}.tokens"]
    lib_gen = TorchCpuGenerator(seed)
    got = [lib_gen.sample(rows[i], temp, top_p) for i in range(rows.shape[0])]
    np.testing.assert_array_equal(got, want)
    # a batch draws row after row: the same tokens in one call
    np.testing.assert_array_equal(TorchCpuGenerator(seed).sample(rows, temp, top_p), want)
    ora = MT19937(seed)
    np.testing.assert_array_equal([sample_torch_cpu(rows[i], temp, top_p, ora) for i in range(rows.shape[0])],
                                  want)


def test_library_equals_oracle_on_random_rows_with_ties():
    rng = np.random.default_rng(3)
    for trial in range(6):
        V = int(rng.integers(300, 3000))
        rows = (rng.standard_normal((5, V)) * rng.uniform(0.5, 6)).astype(np.float16).astype(np.float32)
        rows = np.stack([mask_like_reference(r, step) for step, r in enumerate(rows)])
        temp, top_p = float(rng.uniform(0.5, 1.5)), float(rng.uniform(0.3, 1.0))
        seed = int(rng.integers(0, 2**40))
        a = TorchCpuGenerator(seed).sample(rows, temp, top_p)
        ora = MT19937(seed)
        b = [sample_torch_cpu(r, temp, top_p, ora) for r in rows]
        np.testing.assert_array_equal(a, b)
        assert np.all(a >= 260) or np.any(a == 2)  # the reference mask holds


def test_masking_matches_the_reference_loop():
    x = np.arange(700, dtype=np.float32)[None]
    early, late = mask_like_reference(x, 3), mask_like_reference(x, 16)
    assert np.isneginf(early[0, :260]).all() and (early[0, 260:] == x[0, 260:]).all()
    assert late[0, 2] == 2.0 and np.isneginf(late[0, [0, 1, 3, 259]]).all()


def test_host_sampler_rejects_rows_with_nothing_to_draw():
    lib = _lib.load()
    gen = TorchCpuGenerator(1)
    row = np.full(10, -np.inf, np.float32)
    out = np.empty(1, np.int32)
    st = lib.yuf_sample_host(row.ctypes.data, 1, 10, 1.0, 0.9, gen._h, out.ctypes.data)
    assert st == 1 and "no selectable token" in lib.yuf_last_error().decode()
    assert gen.sample(row, 0.0, 0.9) == 0  # greedy takes the first maximum


def test_oracle_loop_reproduces_the_references_sampled_decode(golden):
    """The reference's sampled loop on the 0.1B model (48 steps, temperature 1,
    top-p 0.95, seed 1337; the smallest winning-key margin is 1.4e-3): the
    oracle model with the oracle sampler draws the same tokens."""
    from oracle.model import OracleModel
    from yufmusicgen_b200 import config as C
    from yufmusicgen_b200.weights import init_weights

    g = golden(FIX)
    cfg = C.ModelConfig(**C.BASE_0P1B)
    om = OracleModel(cfg, init_weights(cfg, 1, "baseline"))
    logits, st = om.forward(g["decode.prompt"])
    last = logits[:, -1]
    gen = MT19937(1337)
    toks = []
    for step in range(len(g["decode.tokens"])):
        t = sample_torch_cpu(mask_like_reference(last, step)[0], 1.0, 0.95, gen)
        toks.append(t)
        last, st = om.step(np.asarray([t]), st)
    np.testing.assert_array_equal(toks, g["decode.tokens"])
