"""Kernel 2 (split-KV paged decode, q_len == 1) vs the oracle.

Tolerance (parity gate): max-abs 2e-2 and mean-abs 2e-3 of the bf16 output
against the fp64 oracle on the same bf16 inputs.
"""
import os

import numpy as np
import pytest
import torch

import nvkv
import nvkv_oracle as O
from helpers import assert_attention_close, bits, cu, f32, gather_seq, make_paged

pytestmark = pytest.mark.gpu


def test_repro_kat_through_gpu(golden_dir):
    """KAT-1 (nanovllm_rs/src/bin/repro.rs) end to end on the GPU path: two
    stores then one paged decode per layer; cache_write_diff must be 0 and the
    output must match repro.rs's manual_attention."""
    kat = np.load(os.path.join(golden_dir, "repro_kat.npz"))
    scale = 1.0 / np.sqrt(128.0)
    for layer in range(28):
        def t(name):
            b = kat[f"l{layer}_{name}"]
            return torch.from_numpy(b.view(np.int16)).cuda().view(torch.bfloat16)
        kc = torch.zeros(1, 256, 8, 128, dtype=torch.bfloat16, device="cuda")
        vc = torch.zeros_like(kc)
        nvkv.store_kvcache(t("k_prior"), t("v_prior"), kc, vc, torch.arange(6, device="cuda"))
        nvkv.store_kvcache(t("k_new"), t("v_new"), kc, vc, torch.tensor([6], device="cuda"))
        out = nvkv.paged_attention(t("q_new"), kc, vc, cu([1]), cu([7]),
                                   torch.zeros(1, 1, dtype=torch.int32, device="cuda"), 1, 7,
                                   scale)
        torch.cuda.synchronize()
        k_full = np.concatenate([kat[f"l{layer}_k_prior"], kat[f"l{layer}_k_new"]], 0)
        assert np.array_equal(bits(kc)[0, :7], k_full)
        assert_attention_close(out, kat[f"l{layer}_manual_out"], f"layer {layer}")


def _decode_case(lens_k, hq, hkv, page=256, num_blocks=None, dtype=torch.bfloat16, seed=0,
                 check=None):
    g = torch.Generator().manual_seed(seed)
    d = 128
    B = len(lens_k)
    num_blocks = num_blocks or sum((L + page - 1) // page for L in lens_k) + 3
    kc, vc, bt, tables = make_paged(lens_k, page, hkv, d, num_blocks, g, dtype)
    q = torch.randn(B, hq, d, generator=g).to(dtype).cuda()
    scale = d ** -0.5
    out = nvkv.paged_attention(q, kc, vc, cu([1] * B), cu(lens_k), torch.from_numpy(
        bt.view(np.int32)).cuda(), 1, max(lens_k), scale)
    torch.cuda.synchronize()
    assert nvkv.device_error() == 0
    qn = f32(q)
    for b in (check if check is not None else range(B)):
        kb, vb = gather_seq(kc, vc, tables[b], lens_k[b])
        want = O.causal_attention_one(qn[b:b + 1], kb, vb, scale)
        assert_attention_close(out[b:b + 1], want, f"seq {b} L={lens_k[b]}")
    return out


def test_decode_config2_shapes():
    """Config 2: 16 q / 8 kv heads, L ~ U[512, 4096], P = 256, block tables a
    permutation of a 2048-block pool (checked on 16 sequences of the 64)."""
    rng = np.random.default_rng(2)
    lens = rng.integers(512, 4097, 64).tolist()
    _decode_case(lens, 16, 8, num_blocks=2048, seed=2, check=range(0, 64, 4))


@pytest.mark.parametrize("group", [1, 2, 4, 8, 16])
def test_decode_gqa_groups(group):
    lens = [1, 63, 64, 65, 300, 1000]
    _decode_case(lens, group * 2, 2, seed=group)


def test_decode_long_context_many_splits():
    """Few (sequence, kv-head) items -> many splits + the in-kernel LSE merge
    (the 32B-at-TP8 shape: 1 kv head per GPU, 8 q heads)."""
    _decode_case([32768, 5000, 257], 8, 1, seed=9)


def test_decode_page_128_and_f16():
    _decode_case([129, 700, 1], 8, 4, page=128, dtype=torch.float16, seed=4)


def test_decode_contiguous_route():
    """block_tables == NULL: K/V rows addressed by cu_seqlens_k (flash_attn_varlen)."""
    g = torch.Generator().manual_seed(8)
    lens = [5, 130, 64]
    hq, hkv, d = 8, 2, 128
    K = torch.randn(sum(lens), hkv, d, generator=g).to(torch.bfloat16).cuda()
    V = torch.randn(sum(lens), hkv, d, generator=g).to(torch.bfloat16).cuda()
    q = torch.randn(3, hq, d, generator=g).to(torch.bfloat16).cuda()
    out = nvkv.paged_attention(q, K, V, cu([1, 1, 1]), cu(lens), None, 1, max(lens), 0.1)
    torch.cuda.synchronize()
    ck = np.cumsum([0] + lens)
    for b in range(3):
        want = O.causal_attention_one(f32(q)[b:b + 1], f32(K)[ck[b]:ck[b + 1]],
                                      f32(V)[ck[b]:ck[b + 1]], 0.1)
        assert_attention_close(out[b:b + 1], want, f"seq {b}")


def test_decode_block_id_out_of_range_is_reported():
    kc = torch.zeros(2, 256, 1, 128, dtype=torch.bfloat16, device="cuda")
    q = torch.ones(1, 2, 128, dtype=torch.bfloat16, device="cuda")
    bt = torch.tensor([[7]], dtype=torch.int32, device="cuda")
    nvkv.device_error()
    out = nvkv.paged_attention(q, kc, kc.clone(), cu([1]), cu([10]), bt, 1, 10, 0.1)
    torch.cuda.synchronize()
    assert nvkv.device_error() == nvkv._lib.DEVERR_BLOCK_RANGE
    assert torch.isfinite(out.float()).all()


def _split_case(lens, hq, hkv, seed):
    g = torch.Generator().manual_seed(seed)
    nb = sum((L + 255) // 256 for L in lens) + 2
    kc, vc, bt, tables = make_paged(lens, 256, hkv, 128, nb, g)
    q = torch.randn(len(lens), hq, 128, generator=g).to(torch.bfloat16).cuda()
    return q, kc, vc, torch.from_numpy(bt.view(np.int32)).cuda(), tables


def _oracle(q, kc, vc, tables, lens):
    qn = f32(q)
    return np.concatenate([O.causal_attention_one(qn[b:b + 1], *gather_seq(kc, vc, tables[b], L),
                                                  128 ** -0.5) for b, L in enumerate(lens)])


def test_decode_workspace_reused_across_shapes_with_garbage():
    """The split-KV merge counters live in the caller's workspace: stale bytes
    from other calls (or garbage) must not matter."""
    ws = torch.randint(0, 256, (64 << 20,), dtype=torch.uint8, device="cuda")
    cases = [([5000, 3000, 8000], 8, 1, 1), ([4000] * 40, 16, 8, 2), ([5000, 3000, 8000], 8, 1, 1),
             ([700, 32768], 16, 2, 3)]
    for lens, hq, hkv, seed in cases:
        q, kc, vc, bt, tables = _split_case(lens, hq, hkv, seed)
        assert nvkv.workspace_size(len(lens), hq, hkv, 1, max(lens)) > 0
        out = nvkv.paged_attention(q, kc, vc, cu([1] * len(lens)), cu(lens), bt, 1, max(lens),
                                   128 ** -0.5, workspace=ws)
        torch.cuda.synchronize()
        assert_attention_close(out, _oracle(q, kc, vc, tables, lens), f"{lens}")
    assert nvkv.device_error() == 0


def test_decode_graph_replays_reuse_the_merge_counters():
    lens, hq, hkv = [9000, 2500, 4100, 600], 8, 2
    q, kc, vc, bt, tables = _split_case(lens, hq, hkv, 4)
    ws = torch.zeros(nvkv.workspace_size(len(lens), hq, hkv, 1, max(lens)), dtype=torch.uint8,
                     device="cuda")
    out = torch.empty_like(q)
    cq, ck = cu([1] * len(lens)), cu(lens)
    run = lambda: nvkv.paged_attention(q, kc, vc, cq, ck, bt, 1, max(lens), 128 ** -0.5,  # noqa
                                       out=out, workspace=ws)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        run()
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        run()
    g = torch.Generator().manual_seed(9)
    for _ in range(3):
        q.copy_(torch.randn(q.shape, generator=g).to(torch.bfloat16))
        graph.replay()
        torch.cuda.synchronize()
        assert_attention_close(out, _oracle(q, kc, vc, tables, lens), "replay")
    graph.reset()


def test_decode_large_batch():
    """1100 sequences of up to 3000 keys (a grid of 2200 work items); checked
    on every 37th sequence."""
    rng = np.random.default_rng(11)
    lens = rng.integers(1, 3000, 1100).tolist()
    _decode_case(lens, 8, 2, seed=11, check=range(0, 1100, 37))


def test_decode_ragged_tiny_batch():
    """Ragged tiny batches: most keys in partial tiles, single-tile and
    one-key sequences next to multi-tile ones."""
    _decode_case([1, 65, 3, 200, 64, 1], 16, 2, seed=12)
    _decode_case([130], 4, 1, seed=13)


def test_decode_two_long_sequences_one_kv_head():
    """Two long sequences at one kv head: the plan splits each ~150 ways."""
    _decode_case([20000, 17001], 8, 1, seed=14)


def test_decode_empty_context_writes_zeros_and_reports():
    """A decode row with k_len == 0 (no keys): zeros plus DEVERR_SEQLEN, the
    other rows unaffected (a small batch that splits and a large one that
    does not)."""
    for B in (3, 1030):
        g = torch.Generator().manual_seed(15)
        lens = [0] + [100] * (B - 1)
        nb = B + 2
        kc, vc, bt, tables = make_paged([max(L, 1) for L in lens], 256, 2, 128, nb, g)
        q = torch.randn(B, 4, 128, generator=g).to(torch.bfloat16).cuda()
        nvkv.device_error()
        out = nvkv.paged_attention(q, kc, vc, cu([1] * B), cu(lens), torch.from_numpy(
            bt.view(np.int32)).cuda(), 1, 100, 0.1)
        torch.cuda.synchronize()
        assert nvkv.device_error() == nvkv._lib.DEVERR_SEQLEN
        assert torch.count_nonzero(out[0]) == 0
        kb, vb = gather_seq(kc, vc, tables[1], 100)
        assert_attention_close(out[1:2], O.causal_attention_one(f32(q)[1:2], kb, vb, 0.1), "row 1")


def test_decode_repeated_calls_are_bitwise_identical():
    """Three calls on the 8B TP8 decode shape with one workspace: the
    split-KV plan and every reduction order are fixed, so the outputs are
    bit-identical (and match the oracle)."""
    rng = np.random.default_rng(21)
    lens = rng.integers(1025, 1537, 256).tolist()
    q, kc, vc, bt, tables = _split_case(lens, 4, 1, 21)
    ws = torch.zeros(nvkv.workspace_size(len(lens), 4, 1, 1, max(lens)), dtype=torch.uint8,
                     device="cuda")
    run = lambda: nvkv.paged_attention(q, kc, vc, cu([1] * len(lens)), cu(lens), bt, 1,  # noqa
                                       max(lens), 128 ** -0.5, workspace=ws)
    outs = [run() for _ in range(3)]
    torch.cuda.synchronize()
    assert nvkv.device_error() == 0
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[1], outs[2])
    sub = list(range(0, 256, 16))
    want = _oracle(q[sub], kc, vc, [tables[b] for b in sub], [lens[b] for b in sub])
    assert_attention_close(outs[2][sub], want, "repeat")


def test_decode_context_above_max_seqlen_is_reported():
    """k_len > max_seqlen_k (a caller bug): the block tables only cover
    max_seqlen_k keys, so the kernel must report DEVERR_SEQLEN rather than
    read past them; the other sequences are still correct."""
    g = torch.Generator().manual_seed(31)
    lens = [500, 200]
    kc, vc, bt, tables = make_paged(lens, 256, 1, 128, 6, g)
    q = torch.randn(2, 4, 128, generator=g).to(torch.bfloat16).cuda()
    bt2 = torch.from_numpy(bt[:, :2].copy().view(np.int32)).cuda()  # 2 pages: 512 keys max
    nvkv.device_error()
    out = nvkv.paged_attention(q, kc, vc, cu([1, 1]), cu(lens), bt2, 1, 300, 0.1)
    torch.cuda.synchronize()
    assert nvkv.device_error() == nvkv._lib.DEVERR_SEQLEN
    kb, vb = gather_seq(kc, vc, tables[1], 200)
    assert_attention_close(out[1:2], O.causal_attention_one(f32(q)[1:2], kb, vb, 0.1), "row 1")


def test_decode_rows_past_num_q_tokens_are_skipped():
    """cu_seqlens_q pointing past num_q_tokens (a caller bug): the q and out
    buffers are over-allocated, the call is given only the first rows, and
    the row the metadata places beyond them must be neither computed nor
    written (its out row keeps a canary) while DEVERR_SEQLEN is reported.
    Once with a split-KV plan (long contexts) and once without."""
    for lens, seed in (([300, 2000, 5000], 32), ([100, 90, 80], 33)):
        g = torch.Generator().manual_seed(seed)
        B = len(lens)
        nb = sum((L + 255) // 256 for L in lens) + 1
        kc, vc, bt, tables = make_paged(lens, 256, 2, 128, nb, g)
        q_all = torch.randn(B, 8, 128, generator=g).to(torch.bfloat16).cuda()
        out_all = torch.full((B, 8, 128), 7.0, dtype=torch.bfloat16, device="cuda")
        nvkv.device_error()
        nvkv.paged_attention(q_all[:B - 1], kc, vc, cu([1] * B), cu(lens),
                             torch.from_numpy(bt.view(np.int32)).cuda(), 1, max(lens), 0.1,
                             out=out_all[:B - 1])
        torch.cuda.synchronize()
        assert nvkv.device_error() == nvkv._lib.DEVERR_SEQLEN
        assert bool((out_all[B - 1] == 7.0).all()), "row past num_q_tokens was written"
        for b in range(B - 1):
            kb, vb = gather_seq(kc, vc, tables[b], lens[b])
            assert_attention_close(out_all[b:b + 1],
                                   O.causal_attention_one(f32(q_all)[b:b + 1], kb, vb, 0.1),
                                   f"row {b}")
