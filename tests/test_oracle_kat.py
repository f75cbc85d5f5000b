"""Pins the CPU oracle against the reference's own known-answer material.

KAT-1: nanovllm_rs/src/bin/repro.rs (generator, two-step store, paged decode
vs manual_attention), via tests/golden/repro_kat.npz.
KAT-2: hand-computed prepare_model_input cases (engine/model_runner.rs:82-131),
via tests/golden/slot_mapping_kat.json.
Plus size-independent properties of the restatement itself.
"""
import json
import os

import numpy as np
import pytest

import nvkv_oracle as O


@pytest.fixture(scope="module")
def kat(golden_dir):
    return np.load(os.path.join(golden_dir, "repro_kat.npz"))


@pytest.mark.parametrize("layer", range(28))
def test_repro_generator_bit_exact(kat, layer):
    kp, vp, kn, vn, qn = O.repro_inputs(layer)
    for name, arr in (("k_prior", kp), ("v_prior", vp), ("k_new", kn), ("v_new", vn),
                      ("q_new", qn)):
        assert np.array_equal(O.bf16_bits(arr), kat[f"l{layer}_{name}"]), name


@pytest.mark.parametrize("layer", range(28))
def test_repro_store_and_paged_decode(kat, layer):
    """repro.rs:75-121: two stores (prefill 6 rows, decode 1 row), cache must
    equal k_full bit for bit, paged attention must equal manual_attention."""
    kp, vp, kn, vn, qn = O.repro_inputs(layer)
    P, hkv, d = O.REPRO_BLOCK_SIZE, O.REPRO_N_KV_HEADS, O.REPRO_HEAD_DIM
    kc = np.zeros((1, P, hkv, d), np.uint16)
    vc = np.zeros((1, P, hkv, d), np.uint16)
    O.store_kvcache(O.bf16_bits(kp), O.bf16_bits(vp), kc, vc, np.arange(6))
    O.store_kvcache(O.bf16_bits(kn), O.bf16_bits(vn), kc, vc, np.array([6]))
    k_full = np.concatenate([kp, kn], 0)
    assert np.array_equal(kc.reshape(P, hkv, d)[:7], O.bf16_bits(k_full))  # cache_write_diff == 0
    assert not kc.reshape(P, hkv, d)[7:].any()
    out = O.paged_attention(qn, O.from_bf16_bits(kc), O.from_bf16_bits(vc),
                            np.array([0, 1], np.uint32), np.array([0, 7], np.uint32),
                            np.zeros((1, 1), np.uint32), 1.0 / np.sqrt(128.0))
    np.testing.assert_allclose(out, kat[f"l{layer}_manual_out"], atol=2e-6, rtol=0)


def _seq_from_case(c, bs):
    toks = list(range(1000, 1000 + c["len"]))
    return O.Seq(toks, list(c["block_table"]), c["num_cached_tokens"], c["num_new_tokens"], bs)


def test_slot_mapping_cases(golden_dir):
    spec = json.load(open(os.path.join(golden_dir, "slot_mapping_kat.json")))
    bs = spec["block_size"]
    for name, c in spec["cases"].items():
        s = _seq_from_case(c, bs)
        ids, pos, ctx = O.prepare_model_input([s], bs)
        assert ctx.slot_mapping.tolist() == c["slots"], name
        assert pos.tolist() == c["positions"], name
        assert ids.tolist() == s.token_ids[c["num_cached_tokens"]:c["num_cached_tokens"] +
                                           c["num_new_tokens"]], name
        assert (ctx.seq_need_compute_logits.tolist() == [0]) == c["need_logits"], name
        if c["num_cached_tokens"] > 0:
            assert ctx.block_tables is not None and ctx.block_tables[0].tolist() == c["block_table"]
        else:
            assert ctx.block_tables is None, name  # model_runner.rs:127-131


def test_slot_mapping_mixed_batch(golden_dir):
    spec = json.load(open(os.path.join(golden_dir, "slot_mapping_kat.json")))
    bs = spec["block_size"]
    b = spec["batch"]
    seqs = [_seq_from_case(spec["cases"][n], bs) for n in b["order"]]
    _, _, ctx = O.prepare_model_input(seqs, bs)
    assert ctx.cu_seqlens_q.tolist() == b["cu_seqlens_q"]
    assert ctx.cu_seqlens_k.tolist() == b["cu_seqlens_k"]
    assert (ctx.max_seqlen_q, ctx.max_seqlen_k) == (b["max_seqlen_q"], b["max_seqlen_k"])
    assert ctx.slot_mapping.tolist() == b["slots"]
    assert ctx.block_tables.tolist() == b["block_tables"]
    assert ctx.context_lens.tolist() == b["context_lens"]
    assert ctx.seq_need_compute_logits.tolist() == b["seq_need_compute_logits"]
    assert ctx.cu_seqlens_q.dtype == np.uint32 and ctx.slot_mapping.dtype == np.int64


def test_block_table_padding():
    seqs = [O.Seq([1] * 5, [3, 4], 4, 1, 4), O.Seq([1] * 2, [9], 1, 1, 4)]
    _, _, ctx = O.prepare_model_input(seqs, 4)
    assert ctx.block_tables.tolist() == [[3, 4], [9, 0]]  # model_runner.rs:53-67


def test_bf16_rounding_ties_to_even():
    # 1 + 2^-8 is a tie between 1 and 1 + 2^-7 -> even (1.0); 1 + 3*2^-8 -> 1 + 2^-6
    x = np.array([1 + 2 ** -8, 1 + 3 * 2 ** -8, -(1 + 2 ** -8), np.inf, 0.0], np.float32)
    assert O.round_bf16(x).tolist() == [1.0, 1 + 2 ** -6, -1.0, np.inf, 0.0]
    assert np.isnan(O.round_bf16(np.array([np.nan], np.float32)))[0]


def test_paged_equals_contiguous_varlen():
    """Gathering through a shuffled block table gives the same attention as
    the contiguous K/V route (attention.rs:38-74 are the same function)."""
    rng = np.random.default_rng(0)
    P, hq, hkv, d = 16, 4, 2, 8
    lens_q = [1, 5, 3]
    lens_k = [9, 5, 20]
    nb = 12
    perm = rng.permutation(nb)
    kc = np.zeros((nb, P, hkv, d), np.float32)
    vc = np.zeros_like(kc)
    bt = np.zeros((3, 2), np.uint32)
    ks, vs = [], []
    used = 0
    for b, L in enumerate(lens_k):
        nblk = (L + P - 1) // P
        bt[b, :nblk] = perm[used:used + nblk]
        used += nblk
        kb = rng.standard_normal((L, hkv, d)).astype(np.float32)
        vb = rng.standard_normal((L, hkv, d)).astype(np.float32)
        slots = [int(bt[b, j // P]) * P + j % P for j in range(L)]
        O.store_kvcache(kb, vb, kc, vc, np.array(slots))
        ks.append(kb)
        vs.append(vb)
    q = rng.standard_normal((sum(lens_q), hq, d)).astype(np.float32)
    cu_q = np.cumsum([0] + lens_q).astype(np.uint32)
    cu_k = np.cumsum([0] + lens_k).astype(np.uint32)
    a = O.paged_attention(q, kc, vc, cu_q, cu_k, bt, 0.3)
    # contiguous route needs one K row per key: compare sequence by sequence
    for b in range(3):
        ob = O.causal_attention_one(q[cu_q[b]:cu_q[b + 1]], ks[b], vs[b], 0.3)
        np.testing.assert_allclose(a[cu_q[b]:cu_q[b + 1]], ob, atol=1e-6)


def test_causal_bottom_right_alignment():
    """Last query of a chunk sees every key; first sees k_len - q_len + 1."""
    rng = np.random.default_rng(1)
    q = rng.standard_normal((3, 1, 4)).astype(np.float32)
    k = rng.standard_normal((7, 1, 4)).astype(np.float32)
    v = rng.standard_normal((7, 1, 4)).astype(np.float32)
    o = O.causal_attention_one(q, k, v, 1.0)
    for i in range(3):
        vis = 7 - 3 + i + 1
        ref = O.causal_attention_one(q[i:i + 1], k[:vis], v[:vis], 1.0, causal=False)
        np.testing.assert_allclose(o[i], ref[0], atol=1e-6)


def test_rope_and_norm_rounding_points():
    """f32 mode is exact math; bf16 mode differs from it only by rounding."""
    rng = np.random.default_rng(2)
    T, hq, hkv, d = 5, 4, 2, 128
    qkv = O.round_bf16(rng.standard_normal((T, (hq + 2 * hkv) * d)).astype(np.float32))
    pos = np.array([0, 1, 17, 4000, 40959])
    w = O.round_bf16(1.0 + 0.1 * rng.standard_normal(d).astype(np.float32))
    q32, k32, v32 = O.qknorm_rope(qkv, pos, hq, hkv, d, w, w, 1e-6, 1e6, "f32")
    q16, k16, v16 = O.qknorm_rope(qkv, pos, hq, hkv, d, w, w, 1e-6, 1e6, "bf16")
    assert np.array_equal(O.round_bf16(q16), q16)
    np.testing.assert_allclose(q16, q32, atol=3e-2)
    np.testing.assert_allclose(k16, k32, atol=3e-2)
    assert np.array_equal(v16, v32)
    # position 0: RoPE is the identity, so q == rms_norm(q)
    qn = O.rms_norm(qkv[0, :hq * d].reshape(hq, d), w, 1e-6, "bf16")
    assert np.array_equal(q16[0], qn)


def _gather_loop(k_cache, v_cache, row, seqlen_k, page):
    """attention.rs:148-163 as the reference writes it: push block*page + s
    page by page, stop at seqlen_k slots."""
    slots = []
    for b in row:
        for s in range(page):
            if len(slots) == seqlen_k:
                break
            slots.append(int(b) * page + s)
        if len(slots) == seqlen_k:
            break
    hkv, d = k_cache.shape[2], k_cache.shape[3]
    idx = np.asarray(slots, dtype=np.int64)
    return k_cache.reshape(-1, hkv, d)[idx], v_cache.reshape(-1, hkv, d)[idx]


def test_gather_paged_kv_equals_the_slot_loop():
    """The oracle's array form of gather_paged_kv gives exactly the rows of
    the reference's slot loop: partial last pages, whole pages, a row with
    more pages than needed, and a row with fewer (the loop then stops short)."""
    rng = np.random.default_rng(5)
    P, nb = 16, 12
    kc = rng.standard_normal((nb, P, 2, 4)).astype(np.float32)
    vc = rng.standard_normal((nb, P, 2, 4)).astype(np.float32)
    for row, L in (([3, 7, 1], 40), ([3, 7, 1], 48), ([5, 2, 9, 0], 17), ([4], 16), ([4, 6], 50),
                   ([8], 0)):
        got = O.gather_paged_kv(kc, vc, np.asarray(row), L, P)
        want = _gather_loop(kc, vc, row, L, P)
        assert got[0].shape == want[0].shape and np.array_equal(got[0], want[0])
        assert np.array_equal(got[1], want[1])


def test_reference_arm_imports_no_native_library():
    """bench.py's CPU arm (the oracle restatement and the shapes it runs)
    must not load libnvkv.so: importing bench, the config module and the
    oracle leaves the nvkv package unimported."""
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    code = ("import sys; sys.path[:0] = [%r, %r, %r]; import bench, qwen3_config, nvkv_oracle, "
            "qwen3_cpu; bad = [m for m in sys.modules if m == 'nvkv' or m.startswith('nvkv.')]; "
            "assert not bad, bad" % (root, os.path.join(root, "nanovllm-rs_b200"),
                                     os.path.join(root, "oracle")))
    subprocess.run([sys.executable, "-c", code], check=True, cwd=root)


def test_e4m3_encoder_every_code_and_midpoint():
    """The oracle's e4m3 encoder (checker of the fp8 pool's store): every
    finite code round-trips, every midpoint between neighbours goes to the
    code with the even mantissa, magnitudes above 448 saturate, signs are
    kept, and values below half the smallest subnormal go to zero."""
    vals = O.E4M3_VALUES
    pos = vals[:0x7F]
    codes = np.arange(0x7F, dtype=np.uint8)
    assert np.array_equal(O.e4m3_encode(pos.astype(np.float32)), codes)
    assert np.array_equal(O.e4m3_encode(-pos[1:].astype(np.float32)), codes[1:] | 0x80)
    mids = ((pos[:-1] + pos[1:]) / 2).astype(np.float32)
    got = O.e4m3_encode(mids)
    even = np.where(codes[:-1] % 2 == 0, codes[:-1], codes[1:])
    assert np.array_equal(got, even)
    assert list(O.e4m3_decode(O.e4m3_encode(np.array([449, 1e30, -500], np.float32)))) == [
        448, 448, -448]
    assert O.e4m3_encode(np.array([2.0 ** -11], np.float32))[0] == 0


def test_fp8_row_quantisation_round_trip():
    """quantize_rows_fp8: scale = amax / 448, codes within half an e4m3 step of
    x / scale, a zero row gives scale 0 and zero codes; the pool store puts
    codes and scales at the slot's page / row and skips negative slots."""
    rng = np.random.default_rng(3)
    x = (rng.standard_normal((6, 2, 128)) * np.exp(rng.uniform(-8, 8, (6, 2, 1)))).astype(np.float32)
    x[2, 1] = 0
    codes, sc = O.quantize_rows_fp8(x)
    amax = np.abs(x).max(-1)
    assert np.array_equal(sc, (amax / np.float32(448)).astype(np.float32))
    back = O.e4m3_decode(codes) * sc[..., None]
    rel = np.abs(back - x) / np.maximum(amax[..., None], 1e-30)
    assert rel.max() <= 16 / 448 * 1.001  # half the widest e4m3 step (32 in [256, 448]) of amax
    assert sc[2, 1] == 0 and not codes[2, 1].any()
    P, nb = 16, 2
    kc = np.zeros((nb, P, 2, 128), np.uint8)
    vc = kc.copy()
    ks = np.full((nb, 2, P), -1, np.float32)
    vs = ks.copy()
    slots = np.array([17, -1, 3, 30, 0, 5])
    O.store_kvcache_fp8(x, x, kc, vc, ks, vs, slots)
    assert np.array_equal(kc[1, 1], codes[0]) and np.array_equal(ks[1, :, 1], sc[0])
    assert np.array_equal(kc[0, 3], codes[2]) and (ks[0, :, 2] == -1).all()
