"""The sampler (layers/sampler.rs:7-21) on the CPU: the oracle's
Philox4x32-10 against the Random123 known answers, the Gumbel-max form
nvkv_sample computes against the reference's own form (softmax(logits / T) /
max(-log u, 1e-10), arg-max) on the same uniforms, vocab-parallel shards
against the whole row, and the C ABI's argument checks (no GPU needed)."""
import ctypes

import numpy as np

import nvkv_oracle as O

# Random123's known-answer vectors for philox4x32_10 (counter, key, output)
PHILOX_KAT = [
    ((0, 0, 0, 0), (0, 0), (0x6627e8d5, 0xe169c58d, 0xbc57ac4c, 0x9b00dbd8)),
    ((0xffffffff,) * 4, (0xffffffff,) * 2, (0x408f276d, 0x41c83b0e, 0xa20bc7c6, 0x6d5451fd)),
    ((0x243f6a88, 0x85a308d3, 0x13198a2e, 0x03707344), (0xa4093822, 0x299f31d0),
     (0xd16cfe09, 0x94fdcceb, 0x5001e420, 0x24126ea1)),
]


def test_philox_known_answers():
    for ctr, key, want in PHILOX_KAT:
        got = O.philox4x32_10(np.array(ctr, np.uint64)[None], key)[0]
        assert tuple(int(x) for x in got) == want


def test_uniforms_in_open_interval_and_shard_consistent():
    u = O.sample_uniforms(8, 1001, seed=2**40 + 3, step=2**33 + 5)
    assert u.dtype == np.float32 and u.min() > 0 and u.max() < 1
    # a shard starting at any global index draws the same uniforms
    assert np.array_equal(O.sample_uniforms(8, 400, 2**40 + 3, 2**33 + 5, vocab_offset=301),
                          u[:, 301:701])
    # other seeds and steps give other noise
    assert not np.array_equal(O.sample_uniforms(8, 1001, 2**40 + 4, 2**33 + 5), u)
    assert not np.array_equal(O.sample_uniforms(8, 1001, 2**40 + 3, 2**33 + 6), u)


def test_gumbel_form_equals_reference_form():
    """argmax(softmax(l / T) / E) == argmax(l / T - log E) on the same draws."""
    rng = np.random.default_rng(1)
    B, V = 128, 3000
    logits = (rng.normal(size=(B, V)) * 4).astype(np.float32)
    temps = rng.uniform(0.2, 2.0, B).astype(np.float32)
    _, idx = O.gumbel_sample(logits, temps, seed=11, step=3)
    ref = O.reference_sample(logits, temps, O.sample_uniforms(B, V, 11, 3))
    assert (idx == ref).mean() >= 0.99


def test_shards_pick_the_whole_rows_sample():
    rng = np.random.default_rng(2)
    B, V = 32, 1000
    logits = rng.normal(size=(B, V)).astype(np.float32)
    temps = np.full(B, 0.8, np.float32)
    v, i = O.gumbel_sample(logits, temps, 5, 9)
    cands = [O.gumbel_sample(logits[:, a:a + 250], temps, 5, 9, vocab_offset=a)
             for a in range(0, V, 250)]
    vals = np.stack([c[0] for c in cands]), np.stack([c[1] for c in cands])
    pick = vals[1][np.argmax(vals[0], axis=0), np.arange(B)]
    assert np.array_equal(pick, i)


def test_zero_temperature_is_greedy():
    rng = np.random.default_rng(3)
    logits = rng.normal(size=(16, 100)).astype(np.float32)
    _, i = O.gumbel_sample(logits, np.zeros(16, np.float32), 1, 1)
    assert np.array_equal(i, logits.argmax(-1))


def test_sample_abi_validation_host_only():
    from nvkv._lib import lib, ERR_INVALID_ARG, ERR_UNSUPPORTED, OK, DTYPE_BF16
    p = ctypes.c_void_p(16)
    n = None
    assert lib.nvkv_sample(None, 0, 10, 10, 0, None, 1, 1, n, None, None, DTYPE_BF16, None) == OK
    assert lib.nvkv_sample(None, 4, 10, 10, 0, p, 1, 1, n, p, p, DTYPE_BF16,
                           None) == ERR_INVALID_ARG
    assert lib.nvkv_sample(p, 4, 10, 8, 0, p, 1, 1, n, p, p, DTYPE_BF16, None) == ERR_INVALID_ARG
    assert lib.nvkv_sample(p, 4, 0, 8, 0, p, 1, 1, n, p, p, DTYPE_BF16, None) == ERR_INVALID_ARG
    assert lib.nvkv_sample(p, 4, 10, 10, 0, p, 1, 1, n, p, p, 7, None) == ERR_UNSUPPORTED
    assert lib.nvkv_sample(p, 4, 10, 10, 2**34, p, 1, 1, n, p, p, DTYPE_BF16,
                           None) == ERR_UNSUPPORTED


def test_oracle_draws_follow_softmax():
    """The generator's distribution on the CPU: 49152 draws over eight logits
    (rows and steps vary the counter) land within 5 standard deviations of
    softmax(l / T) in every bin."""
    base = np.array([0.0, 1.0, -1.0, 0.5, 2.0, -3.0, 0.2, 1.5], np.float32)
    T, B = 0.7, 4096
    counts = np.zeros(8, np.int64)
    for step in range(12):
        _, idx = O.gumbel_sample(np.tile(base, (B, 1)), np.full(B, T, np.float32), 2024, step)
        counts += np.bincount(idx, minlength=8)
    n = counts.sum()
    p = np.exp(base / T) / np.exp(base / T).sum()
    assert (np.abs(counts - n * p) <= 5 * np.sqrt(n * p * (1 - p)) + 1).all(), (counts, n * p)
