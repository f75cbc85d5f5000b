"""The optional FP8 (e4m3) KV pool against the oracle.

* nvkv_store_kvcache_fp8 is bit-exact with the oracle's quantisation
  (codes and per-row scales, oracle/nvkv_oracle.py quantize_rows_fp8),
  including padded slots, a row of zeros and rows that span the e4m3 range.
* nvkv_paged_attention_fp8 over such a pool matches the oracle's attention
  over the dequantised keys and values (code * scale) within the attention
  tolerance (max-abs 2e-2, mean-abs 2e-3): decode batches (the split-KV plan
  and the one-wave plan, GQA groups up to 16) and mixed batches whose prompts
  are dequantised into the workspace and run through the tcgen05 prefill.
* f16 queries (Q as three e4m3 pieces) and V rows scaled by 1e-4 and 3e3
  (the decode keeps O in a running power-of-two unit) meet the same bar,
  relative to the V scale.
* A prompt whose keys do not fit prompt_kv_tokens is skipped and reported,
  its out rows untouched, the rest of the batch still correct.
"""
import numpy as np
import pytest
import torch

import nvkv
import nvkv_oracle as O
from nvkv import ops
from helpers import assert_attention_close, cu, f32

pytestmark = pytest.mark.gpu

P, D = 256, 128


def _pool(nb, hkv, seed, gain=None, dtype=torch.bfloat16, v_gain=1.0):
    """An fp8 pool filled through nvkv_store_kvcache_fp8 from random rows of
    `dtype`; returns (k, v, k_scale, v_scale) on the GPU and the dequantised
    pool."""
    g = torch.Generator().manual_seed(seed)
    n = nb * P
    k = torch.randn(n, hkv, D, generator=g)
    v = torch.randn(n, hkv, D, generator=g) * v_gain
    if gain is not None:
        k = k * gain(n)[:, None, None]
    k, v = k.to(dtype).cuda(), v.to(dtype).cuda()
    kc = torch.zeros(nb, P, hkv, D, dtype=torch.uint8, device="cuda")
    vc = torch.zeros_like(kc)
    ks = torch.zeros(nb, hkv, P, dtype=torch.float32, device="cuda")
    vs = torch.zeros_like(ks)
    ops.store_kvcache_fp8(k, v, kc, vc, ks, vs, torch.arange(n, device="cuda"))
    torch.cuda.synchronize()
    kd = O.dequantize_pages_fp8(kc.cpu().numpy(), ks.cpu().numpy())
    vd = O.dequantize_pages_fp8(vc.cpu().numpy(), vs.cpu().numpy())
    return (kc, vc, ks, vs), kd, vd


def _tables(lens, nb, seed):
    rng = np.random.default_rng(seed)
    perm = rng.permutation(nb)
    tables, u = [], 0
    for L in lens:
        n = (L + P - 1) // P
        tables.append(perm[u:u + n].tolist())
        u += n
    assert u <= nb
    bt = np.zeros((len(lens), max(len(t) for t in tables)), np.int32)
    for i, t in enumerate(tables):
        bt[i, :len(t)] = t
    return tables, torch.from_numpy(bt).cuda()


def _want(qn, kd, vd, table, q_len, k_len, scale):
    rows = np.concatenate([np.arange(pg * P, (pg + 1) * P) for pg in table])[:k_len]
    kk = kd.reshape(-1, kd.shape[2], D)[rows]
    vv = vd.reshape(-1, vd.shape[2], D)[rows]
    return O.causal_attention_one(qn, kk, vv, scale, True)


def test_store_fp8_bit_exact():
    g = torch.Generator().manual_seed(1)
    hkv, nb = 4, 3
    T = 40
    x = torch.randn(T, hkv, D, generator=g) * torch.exp(4 * torch.randn(T, hkv, 1, generator=g))
    x[3, 1] = 0.0  # a row of zeros: scale 0
    x[5, 2, 7] = 3.0e4  # one large value sets the row's scale
    y = torch.randn(T, hkv, D, generator=g) * 1e-3
    key, value = x.bfloat16().cuda(), y.bfloat16().cuda()
    slots = torch.randperm(nb * P, generator=g)[:T]
    slots[::7] = -1  # padded rows are skipped
    kc = torch.full((nb, P, hkv, D), 0xAB, dtype=torch.uint8, device="cuda")
    vc = kc.clone()
    ks = torch.full((nb, hkv, P), -1.0, device="cuda")
    vs = ks.clone()
    ops.store_kvcache_fp8(key, value, kc, vc, ks, vs, slots.cuda())
    torch.cuda.synchronize()
    assert nvkv.device_error() == 0
    wk = np.full((nb, P, hkv, D), 0xAB, np.uint8)
    wv = wk.copy()
    wks = np.full((nb, hkv, P), -1.0, np.float32)
    wvs = wks.copy()
    O.store_kvcache_fp8(f32(key), f32(value), wk, wv, wks, wvs, slots.numpy())
    assert np.array_equal(kc.cpu().numpy(), wk) and np.array_equal(vc.cpu().numpy(), wv)
    assert np.array_equal(ks.cpu().numpy().view(np.uint32), wks.view(np.uint32))
    assert np.array_equal(vs.cpu().numpy().view(np.uint32), wvs.view(np.uint32))


@pytest.mark.parametrize("lens,hq,hkv", [
    (np.random.default_rng(2).integers(512, 4097, 64).tolist(), 16, 8),  # config 2: split-KV
    (np.random.default_rng(3).integers(1025, 1537, 256).tolist(), 4, 1),  # 8B TP8: one wave
    ([20000, 300, 1, 4096], 16, 1),                                       # long, group 16
])
def test_decode_fp8_matches_oracle(lens, hq, hkv):
    nb = sum((L + P - 1) // P for L in lens) + 2
    pool, kd, vd = _pool(nb, hkv, seed=len(lens))
    tables, bt = _tables(lens, nb, seed=5)
    g = torch.Generator().manual_seed(7)
    B = len(lens)
    q = torch.randn(B, hq, D, generator=g).bfloat16().cuda()
    scale = D ** -0.5
    out = ops.paged_attention_fp8(q, *pool, cu([1] * B), cu(lens), bt, 1, max(lens), scale)
    torch.cuda.synchronize()
    assert nvkv.device_error() == 0
    qn = f32(q)
    for b in sorted(set(range(0, B, max(1, B // 16))) | {B - 1}):
        want = _want(qn[b:b + 1], kd, vd, tables[b], 1, lens[b], scale)
        assert_attention_close(out[b:b + 1], want, f"seq {b} len {lens[b]}")


@pytest.mark.parametrize("dtype,v_gain", [(torch.float16, 1.0), (torch.bfloat16, 1e-4),
                                          (torch.bfloat16, 3e3)])
def test_decode_fp8_dtypes_and_value_ranges(dtype, v_gain):
    """f16 queries (Q split into three e4m3 pieces) and V rows far below and
    far above 1 (the running power-of-two unit of O must keep P' in range)."""
    lens = np.random.default_rng(21).integers(100, 3000, 48).tolist()
    hq, hkv = 8, 2
    nb = sum((L + P - 1) // P for L in lens) + 2
    pool, kd, vd = _pool(nb, hkv, seed=22, dtype=dtype, v_gain=v_gain)
    tables, bt = _tables(lens, nb, seed=23)
    g = torch.Generator().manual_seed(24)
    B = len(lens)
    q = (torch.randn(B, hq, D, generator=g) * 2).to(dtype).cuda()
    scale = D ** -0.5
    out = ops.paged_attention_fp8(q, *pool, cu([1] * B), cu(lens), bt, 1, max(lens), scale)
    torch.cuda.synchronize()
    assert nvkv.device_error() == 0
    qn = f32(q)
    for b in range(0, B, 3):
        want = _want(qn[b:b + 1], kd, vd, tables[b], 1, lens[b], scale)
        got = out[b:b + 1].float().cpu().numpy() / v_gain
        assert_attention_close(torch.from_numpy(got), want / v_gain, f"seq {b} len {lens[b]}")


def test_mixed_fp8_prompts_dequantised_into_workspace():
    """Decode rows next to a fresh prompt, a prefix-cache-hit chunk and a
    second prompt (config-3 shape at TP2 heads), interleaved."""
    rng = np.random.default_rng(8)
    dec = rng.integers(129, 2305, 40).tolist()
    q_lens = [1] * len(dec) + [700, 150, 300]
    k_lens = dec + [700, 150 + 512, 300]
    order = rng.permutation(len(q_lens))
    q_lens = [q_lens[i] for i in order]
    k_lens = [k_lens[i] for i in order]
    hq, hkv = 16, 4
    nb = sum((L + P - 1) // P for L in k_lens) + 2
    pool, kd, vd = _pool(nb, hkv, seed=9)
    tables, bt = _tables(k_lens, nb, seed=10)
    g = torch.Generator().manual_seed(11)
    q = torch.randn(sum(q_lens), hq, D, generator=g).bfloat16().cuda()
    scale = D ** -0.5
    prompt_rows = sum(k for qq, k in zip(q_lens, k_lens) if qq > 1)
    out = ops.paged_attention_fp8(q, *pool, cu(q_lens), cu(k_lens), bt, max(q_lens), max(k_lens),
                                  scale, prompt_kv_tokens=prompt_rows)
    torch.cuda.synchronize()
    assert nvkv.device_error() == 0
    c = np.cumsum([0] + q_lens)
    qn = f32(q)
    for b in range(len(q_lens)):
        if q_lens[b] > 1 or b % 5 == 0:
            want = _want(qn[c[b]:c[b + 1]], kd, vd, tables[b], q_lens[b], k_lens[b], scale)
            assert_attention_close(out[c[b]:c[b + 1]], want, f"seq {b} q={q_lens[b]}")


def test_fp8_prompt_rows_too_few_are_reported():
    """prompt_kv_tokens below the prompts' keys: the prompt that does not fit
    is skipped (its out rows keep a canary) and reported; the one before it
    and the decode row are still right."""
    q_lens, k_lens = [300, 1, 200], [300, 900, 450]
    hq, hkv = 4, 2
    nb = sum((L + P - 1) // P for L in k_lens) + 1
    pool, kd, vd = _pool(nb, hkv, seed=12)
    tables, bt = _tables(k_lens, nb, seed=13)
    g = torch.Generator().manual_seed(14)
    q = torch.randn(sum(q_lens), hq, D, generator=g).bfloat16().cuda()
    out = torch.full_like(q, 7.0)
    nvkv.device_error()
    ops.paged_attention_fp8(q, *pool, cu(q_lens), cu(k_lens), bt, 300, 900, D ** -0.5,
                            prompt_kv_tokens=500, out=out)  # 300 + 450 needed
    torch.cuda.synchronize()
    assert nvkv.device_error() == nvkv._lib.DEVERR_SEQLEN
    assert bool((out[301:] == 7.0).all())
    qn = f32(q)
    assert_attention_close(out[:300], _want(qn[:300], kd, vd, tables[0], 300, 300, D ** -0.5),
                           "first prompt")
    assert_attention_close(out[300:301], _want(qn[300:301], kd, vd, tables[1], 1, 900,
                                               D ** -0.5), "decode row")


def test_decoder_on_fp8_pool():
    """The Qwen3 driver over the fp8 pool (prologue, fp8 store, fp8 attention
    for the prefill step and the decode steps) next to the same model over the
    bf16 pool, teacher forced with the bf16 pool's tokens: finite logits
    throughout and the same logit direction (cosine similarity >= 0.98 at
    every step).  The fp8 pool is not the reference's format, so this bounds
    the quantisation's effect rather than asserting parity."""
    import test_gpu_greedy as G
    from nvkv.decoder import Qwen3TP, Step

    model = Qwen3TP(G.CFG, seed=3, device="cuda", **G.INIT)
    streams = {}
    for fp8 in (False, True):
        model.allocate_kv_cache(G.NB, G.P, kv_fp8=fp8)
        seqs, free = G.make_seqs(11)
        logits, toks = [], []
        for step in range(8):
            ids, pos, ctx = O.prepare_model_input(seqs, G.P)
            bt = O.prepare_block_tables(seqs)
            cu_q = torch.from_numpy(ctx.cu_seqlens_q.view(np.int32)).cuda()
            q_lens = np.diff(ctx.cu_seqlens_q.astype(np.int64))
            k_lens = np.diff(ctx.cu_seqlens_k.astype(np.int64))
            st = Step(torch.from_numpy(ids).cuda(), torch.from_numpy(pos).cuda(),
                      torch.from_numpy(ctx.slot_mapping).cuda(), cu_q,
                      torch.from_numpy(ctx.cu_seqlens_k.view(np.int32)).cuda(),
                      torch.from_numpy(bt.view(np.int32)).cuda(), (cu_q[1:] - 1).long(),
                      ctx.max_seqlen_q, ctx.max_seqlen_k,
                      prompt_kv_tokens=int(k_lens[q_lens > 1].sum()))
            lg = model.forward(st).float()
            logits.append(lg)
            nxt = (streams[False][1][step] if fp8 else lg.argmax(-1).cpu().numpy())
            toks.append(nxt)
            G.Q.advance(seqs, nxt, free, G.P)
        streams[fp8] = (logits, toks)
    torch.cuda.synchronize()
    assert nvkv.device_error() == 0
    cos = [float(torch.nn.functional.cosine_similarity(a, b, dim=-1).min())
           for a, b in zip(streams[False][0], streams[True][0])]
    agree = float(np.mean([(a.argmax(-1) == b.argmax(-1)).float().mean().item()
                           for a, b in zip(streams[False][0], streams[True][0])]))
    print("fp8 pool vs bf16 pool: min cosine per step", [round(c, 4) for c in cos],
          "greedy agreement", agree)
    assert all(torch.isfinite(x).all() for x in streams[True][0])
    assert min(cos) >= 0.98, cos
