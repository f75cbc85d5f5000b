"""Kernel 3 (tcgen05 varlen paged prefill, q_len > 1) vs the oracle, and
mixed decode + prefill batches (both kernels in one call).

Tolerance (parity gate): max-abs 2e-2, mean-abs 2e-3 vs the fp64 oracle.
"""
import numpy as np
import pytest
import torch

import nvkv
import nvkv_oracle as O
from helpers import assert_attention_close, cu, f32, gather_seq, make_paged

pytestmark = pytest.mark.gpu


def _contiguous_case(lens, hq, hkv, dtype=torch.bfloat16, causal=True, seed=0, k_gain=None):
    g = torch.Generator().manual_seed(seed)
    d, T = 128, sum(lens)
    q = torch.randn(T, hq, d, generator=g).to(dtype).cuda()
    k = torch.randn(T, hkv, d, generator=g)
    if k_gain is not None:  # per-position key scale: k[t] *= k_gain(position in its sequence)
        pos = np.concatenate([np.arange(L) for L in lens])
        k = k * torch.from_numpy(k_gain(pos).astype(np.float32))[:, None, None]
    k = k.to(dtype).cuda()
    v = torch.randn(T, hkv, d, generator=g).to(dtype).cuda()
    scale = d ** -0.5
    out = nvkv.paged_attention(q, k, v, cu(lens), cu(lens), None, max(lens), max(lens), scale,
                               causal=causal)
    torch.cuda.synchronize()
    assert nvkv.device_error() == 0
    c = np.cumsum([0] + lens)
    for b in range(len(lens)):
        want = O.causal_attention_one(f32(q)[c[b]:c[b + 1]], f32(k)[c[b]:c[b + 1]],
                                      f32(v)[c[b]:c[b + 1]], scale, causal)
        assert_attention_close(out[c[b]:c[b + 1]], want, f"seq {b} len {lens[b]}")


@pytest.mark.parametrize("lens", [[2], [128], [129, 3], [127, 300, 1024], [2048]])
def test_prefill_pure_causal(lens):
    """No block table: flash_attn_varlen(causal=true) on the fresh K/V."""
    _contiguous_case(lens, 8, 2, seed=len(lens))


@pytest.mark.parametrize("group", [1, 4, 8])
def test_prefill_gqa_groups(group):
    _contiguous_case([200, 77], 2 * group, 2, seed=group)


def test_prefill_row_max_growth_rescales():
    """Scores that keep growing along the keys: the row max rises by far more
    than 2^8 (the lazy-rescale threshold) from one 128-key tile to the next,
    so the kernel must rescale O and the row sum on most tiles."""
    _contiguous_case([700, 300], 4, 2, seed=11, k_gain=lambda pos: 1.0 + pos / 64.0)
    _contiguous_case([520], 4, 1, dtype=torch.float16, seed=12,
                     k_gain=lambda pos: np.where(pos >= 256, 6.0, 1.0))


def test_prefill_f16_and_noncausal():
    _contiguous_case([150, 64], 4, 4, dtype=torch.float16, seed=3)
    _contiguous_case([150, 64], 4, 2, causal=False, seed=5)


def _paged_case(q_lens, k_lens, hq, hkv, page=256, seed=0, dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    d = 128
    kc, vc, bt, tables = make_paged(k_lens, page, hkv, d,
                                    sum((L + page - 1) // page for L in k_lens) + 2, g, dtype)
    T = sum(q_lens)
    q = torch.randn(T, hq, d, generator=g).to(dtype).cuda()
    scale = d ** -0.5
    out = nvkv.paged_attention(q, kc, vc, cu(q_lens), cu(k_lens),
                               torch.from_numpy(bt.view(np.int32)).cuda(), max(q_lens),
                               max(k_lens), scale)
    torch.cuda.synchronize()
    assert nvkv.device_error() == 0
    c = np.cumsum([0] + q_lens)
    for b in range(len(q_lens)):
        kb, vb = gather_seq(kc, vc, tables[b], k_lens[b])
        want = O.causal_attention_one(f32(q)[c[b]:c[b + 1]], kb, vb, scale)
        assert_attention_close(out[c[b]:c[b + 1]], want, f"seq {b} q={q_lens[b]} k={k_lens[b]}")


def test_prefill_paged_prefix_cache_hit():
    """Prefix-cache hit / chunked prefill: k_len > q_len, bottom-right causal."""
    _paged_case([100, 256, 300], [356, 512, 377], 8, 2, seed=1)


def test_mixed_decode_and_prefill_batch():
    """One step with decode rows (q_len 1) and prefill chunks: the decode
    kernel and the tcgen05 kernel each take their own sequences."""
    _paged_case([1, 130, 1, 1, 64, 2], [900, 130, 2, 4000, 600, 258], 16, 8, seed=2)


def test_prefill_page_128():
    _paged_case([200, 5], [600, 133], 4, 1, page=128, seed=6)


@pytest.mark.parametrize("tp", [1, 2])
def test_config3_mixed_step_qwen3_4b(tp):
    """benchmark config 3 (Qwen3-4B, 32 q / 8 kv heads, TP1/2): a continuous-
    batching step with decoding sequences (contexts U[129, 2304]) next to
    fresh prompts and a prefix-cache-hit chunk, at the per-rank head counts."""
    rng = np.random.default_rng(30 + tp)
    dec = rng.integers(129, 2305, 24).tolist()
    q_lens = [1] * len(dec) + [700, 1300, 150]
    k_lens = dec + [700, 1300, 150 + 512]
    order = rng.permutation(len(q_lens))  # decode and prefill rows interleaved
    _paged_case([q_lens[i] for i in order], [k_lens[i] for i in order], 32 // tp, 8 // tp,
                seed=40 + tp)


def test_prefill_bad_lengths_reported():
    """The prefill work plan checks each q_len > 1 sequence: k_len < q_len, or
    q_len above max_seqlen_q (whose tail rows the kernel cannot cover), is
    reported as DEVERR_SEQLEN; the other sequences are still computed."""
    g = torch.Generator().manual_seed(21)
    d, hq, hkv = 128, 4, 2
    for q_lens, k_lens, max_q in (([300, 40], [300, 30], 300),   # k_len < q_len
                                  ([300, 40], [300, 40], 200)):  # q_len > max_seqlen_q
        T, Tk = sum(q_lens), sum(k_lens)
        q = torch.randn(T, hq, d, generator=g).bfloat16().cuda()
        k = torch.randn(Tk, hkv, d, generator=g).bfloat16().cuda()
        v = torch.randn(Tk, hkv, d, generator=g).bfloat16().cuda()
        nvkv.device_error()
        out = nvkv.paged_attention(q, k, v, cu(q_lens), cu(k_lens), None, max_q, max(k_lens),
                                   d ** -0.5)
        torch.cuda.synchronize()
        assert nvkv.device_error() == nvkv._lib.DEVERR_SEQLEN
        good = 0 if k_lens[0] == q_lens[0] and q_lens[0] <= max_q else 1
        c, ck = np.cumsum([0] + q_lens), np.cumsum([0] + k_lens)
        want = O.causal_attention_one(f32(q)[c[good]:c[good + 1]], f32(k)[ck[good]:ck[good + 1]],
                                      f32(v)[ck[good]:ck[good + 1]], d ** -0.5, True)
        assert_attention_close(out[c[good]:c[good + 1]], want, "the well-formed sequence")


def test_mixed_many_decode_rows_work_plan():
    """Hundreds of decode rows next to two prompts: the candidate work items
    (q tiles x head slots x sequences) exceed the direct-enumeration limit,
    so the prefill kernel runs from its work plan (prompts sorted by q-tile
    count); every row, decode and prefill, matches the oracle."""
    rng = np.random.default_rng(50)
    dec = rng.integers(2, 700, 300).tolist()
    q_lens = [1] * 300 + [200, 517]
    k_lens = dec + [200, 517 + 300]
    order = rng.permutation(len(q_lens))
    _paged_case([q_lens[i] for i in order], [k_lens[i] for i in order], 8, 2, seed=51)


def test_work_plan_bad_lengths_reported():
    """The work plan's own checks (k_len < q_len; q_len above max_seqlen_q)
    with enough decode rows that the plan is used."""
    g = torch.Generator().manual_seed(52)
    d, hq, hkv = 128, 8, 2
    for q_pre, k_pre, max_q in (([300, 40], [300, 30], 300), ([300, 40], [300, 40], 200)):
        q_lens, k_lens = [1] * 400 + q_pre, [5] * 400 + k_pre
        T, Tk = sum(q_lens), sum(k_lens)
        q = torch.randn(T, hq, d, generator=g).bfloat16().cuda()
        k = torch.randn(Tk, hkv, d, generator=g).bfloat16().cuda()
        v = torch.randn(Tk, hkv, d, generator=g).bfloat16().cuda()
        nvkv.device_error()
        out = nvkv.paged_attention(q, k, v, cu(q_lens), cu(k_lens), None, max_q, max(k_lens),
                                   d ** -0.5)
        torch.cuda.synchronize()
        assert nvkv.device_error() == nvkv._lib.DEVERR_SEQLEN
        good = 400 + (0 if k_pre[0] == q_pre[0] and q_pre[0] <= max_q else 1)
        c, ck = np.cumsum([0] + q_lens), np.cumsum([0] + k_lens)
        want = O.causal_attention_one(f32(q)[c[good]:c[good + 1]], f32(k)[ck[good]:ck[good + 1]],
                                      f32(v)[ck[good]:ck[good + 1]], d ** -0.5, True)
        assert_attention_close(out[c[good]:c[good + 1]], want, "the well-formed prompt")


def _bounds_case(q_lens, k_lens, given_rows, max_q, max_k, hq, hkv, bad, seed):
    """Paged prompts whose metadata is wrong for sequence `bad`, on buffers
    large enough that a kernel ignoring the checks would stay in bounds: q and
    out hold sum(q_lens) rows, but only `given_rows` are passed; the block
    tables are wide enough for every k_len.  Sequence `bad` must leave its
    out rows untouched (canary) and DEVERR_SEQLEN must be reported; every
    other sequence must match the oracle."""
    g = torch.Generator().manual_seed(seed)
    d, P = 128, 256
    nb = sum((k + P - 1) // P for k in k_lens) + 1
    kc, vc, bt, tables = make_paged(k_lens, P, hkv, d, nb, g)
    T = sum(q_lens)
    q_all = torch.randn(T, hq, d, generator=g).to(torch.bfloat16).cuda()
    out_all = torch.full((T, hq, d), 7.0, dtype=torch.bfloat16, device="cuda")
    nvkv.device_error()
    nvkv.paged_attention(q_all[:given_rows], kc, vc, cu(q_lens), cu(k_lens),
                         torch.from_numpy(bt.view(np.int32)).cuda(), max_q, max_k, d ** -0.5,
                         out=out_all[:given_rows])
    torch.cuda.synchronize()
    assert nvkv.device_error() == nvkv._lib.DEVERR_SEQLEN
    c = np.cumsum([0] + list(q_lens))
    assert bool((out_all[c[bad]:c[bad + 1]] == 7.0).all()), "a skipped sequence was written"
    qn = f32(q_all)
    for b in range(len(q_lens)):
        if b == bad:
            continue
        kb, vb = gather_seq(kc, vc, tables[b], k_lens[b])
        want = O.causal_attention_one(qn[c[b]:c[b + 1]], kb, vb, d ** -0.5, True)
        assert_attention_close(out_all[c[b]:c[b + 1]], want, f"sequence {b}")


@pytest.mark.parametrize("decodes", [0, 400])
def test_prefill_k_len_above_max_seqlen_k_is_skipped(decodes):
    """k_len > max_seqlen_k on a prompt: its block-table row only has to
    cover max_seqlen_k keys, so the kernel must not walk it (direct
    enumeration without decode rows; the work plan with 400 of them)."""
    q_lens = [1] * decodes + [300, 200]
    k_lens = [5] * decodes + [300, 700]
    _bounds_case(q_lens, k_lens, sum(q_lens), 300, 600, 8, 2, decodes + 1, seed=60 + decodes)


@pytest.mark.parametrize("decodes", [0, 400])
def test_prefill_rows_past_num_q_tokens_are_skipped(decodes):
    """A prompt whose query rows reach past num_q_tokens: nothing of it is
    computed or written (direct enumeration, and the work plan)."""
    q_lens = [1] * decodes + [300, 200]
    k_lens = [5] * decodes + [300, 450]
    _bounds_case(q_lens, k_lens, sum(q_lens) - 50, 300, 450, 8, 2, decodes + 1,
                 seed=70 + decodes)
