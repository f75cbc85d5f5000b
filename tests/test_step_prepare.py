"""nvkv_prepare_step (host C++ ModelRunner::prepare_model_input +
prepare_block_tables, engine/model_runner.rs:53-160) against the KAT-2
fixtures and the oracle's restatement.  Parity bar: bit-exact (integers)."""
import json
import os
import random

import numpy as np

import block_manager_oracle as OB
import nvkv_oracle as O
from nvkv.blocks import BlockManager, Sequence, prepare_step


def _seq(c, bs):
    s = Sequence(list(range(1000, 1000 + c["len"])), bs)
    s.block_table = list(c["block_table"])
    s.num_cached_tokens, s.num_new_tokens = c["num_cached_tokens"], c["num_new_tokens"]
    return s


def _oracle_seq(s):
    return O.Seq(list(s.token_ids), list(s.block_table), s.num_cached_tokens, s.num_new_tokens,
                 s.block_size)


def _same(out, seqs, bs):
    ids, pos, ctx = O.prepare_model_input([_oracle_seq(s) for s in seqs], bs)
    assert out["input_ids"].tolist() == ids.tolist()
    assert out["positions"].tolist() == pos.tolist()
    assert out["cu_seqlens_q"].tolist() == ctx.cu_seqlens_q.tolist()
    assert out["cu_seqlens_k"].tolist() == ctx.cu_seqlens_k.tolist()
    assert (out["max_seqlen_q"], out["max_seqlen_k"]) == (ctx.max_seqlen_q, ctx.max_seqlen_k)
    assert out["slot_mapping"].tolist() == ctx.slot_mapping.tolist()
    assert out["context_lens"].tolist() == ctx.context_lens.tolist()
    assert out["seq_need_compute_logits"].tolist() == ctx.seq_need_compute_logits.tolist()
    if ctx.block_tables is None:
        assert out["block_tables"] is None
    else:
        assert out["block_tables"].tolist() == ctx.block_tables.tolist()
    assert out["cu_seqlens_q"].dtype == np.uint32 and out["slot_mapping"].dtype == np.int64


def test_kat2_cases(golden_dir):
    spec = json.load(open(os.path.join(golden_dir, "slot_mapping_kat.json")))
    bs = spec["block_size"]
    for name, c in spec["cases"].items():
        s = _seq(c, bs)
        out = prepare_step([s], bs)
        assert out["slot_mapping"].tolist() == c["slots"], name
        assert out["positions"].tolist() == c["positions"], name
        assert (out["seq_need_compute_logits"].tolist() == [0]) == c["need_logits"], name
        _same(out, [s], bs)


def test_kat2_mixed_batch(golden_dir):
    spec = json.load(open(os.path.join(golden_dir, "slot_mapping_kat.json")))
    bs = spec["block_size"]
    b = spec["batch"]
    seqs = [_seq(spec["cases"][n], bs) for n in b["order"]]
    out = prepare_step(seqs, bs)
    assert out["cu_seqlens_q"].tolist() == b["cu_seqlens_q"]
    assert out["cu_seqlens_k"].tolist() == b["cu_seqlens_k"]
    assert (out["max_seqlen_q"], out["max_seqlen_k"]) == (b["max_seqlen_q"], b["max_seqlen_k"])
    assert out["slot_mapping"].tolist() == b["slots"]
    assert out["block_tables"].tolist() == b["block_tables"]
    assert out["context_lens"].tolist() == b["context_lens"]
    assert out["seq_need_compute_logits"].tolist() == b["seq_need_compute_logits"]


def test_warmup_and_padding():
    """No blocks (warm-up): no slots, no logits index; block tables padded
    with 0 (model_runner.rs:53-67, :103-106)."""
    a = Sequence([1] * 5, 4)
    a.block_table, a.num_cached_tokens, a.num_new_tokens = [3, 4], 4, 1
    b = Sequence([1] * 2, 4)
    b.block_table, b.num_cached_tokens, b.num_new_tokens = [9], 1, 1
    w = Sequence([5, 6, 7], 4)
    w.num_new_tokens = 3  # warm-up sequence without blocks
    out = prepare_step([a, b, w], 4)
    assert out["block_tables"].tolist() == [[3, 4], [9, 0], [0, 0]]
    _same(out, [a, b, w], 4)


def test_random_steps_match_oracle():
    rng = random.Random(8)
    for _ in range(200):
        bs = rng.choice([4, 16, 256])
        seqs = []
        for _ in range(rng.randrange(1, 12)):
            n = rng.randrange(1, 4 * bs)
            cached = rng.randrange(0, n)
            new = rng.randrange(1 if cached < n else 0, n - cached + 1)
            s = Sequence([rng.randrange(151936) for _ in range(n)], bs)
            s.num_cached_tokens, s.num_new_tokens = cached, new
            if rng.random() < 0.9:
                s.block_table = rng.sample(range(4096), (cached + new + bs - 1) // bs)
            seqs.append(s)
        _same(prepare_step(seqs, bs), seqs, bs)


def test_block_manager_feeds_step_metadata():
    """The host path of a step: the block manager's tables (prefix hits,
    chunked prefill, decode growth) through nvkv_prepare_step equal the
    oracle manager's tables through the oracle's prepare_model_input."""
    rng = random.Random(10)
    bs = 16
    o, c = OB.BlockManager(64, bs), BlockManager(64, bs)
    shared = [rng.randrange(151936) for _ in range(40)]
    pairs = []
    for k in range(6):
        toks = (shared if k % 2 else []) + [rng.randrange(151936) for _ in range(rng.randrange(5, 50))]
        so, sc = OB.Seq(toks, bs), Sequence(toks, bs)
        _, f, n = o.get_token_layout(so)
        n = min(n, 24)  # chunked prefill
        so.num_new_tokens = sc.num_new_tokens = n
        o.allocate(so)
        c.allocate(sc)
        pairs.append((so, sc))
    for step in range(12):
        out = prepare_step([sc for _, sc in pairs], bs)
        _same(out, [sc for _, sc in pairs], bs)
        ids, pos, ctx = O.prepare_model_input(
            [O.Seq(so.token_ids, so.block_table, so.num_cached_tokens, so.num_new_tokens, bs)
             for so, _ in pairs], bs)
        assert out["slot_mapping"].tolist() == ctx.slot_mapping.tolist()
        for so, sc in pairs:  # the step ran: advance, sample where the prompt is done
            done = so.num_cached_tokens + so.num_new_tokens == len(so)
            so.num_cached_tokens += so.num_new_tokens
            sc.num_cached_tokens += sc.num_new_tokens
            so.num_new_tokens = sc.num_new_tokens = 0
            if done:
                t = rng.randrange(151936)
                so.append_token(t)
                sc.append_token(t)
            n = min(len(so) - so.num_cached_tokens, 24)
            so.num_new_tokens = sc.num_new_tokens = n
            o.may_append(so)
            c.may_append(sc)
            assert so.block_table == sc.block_table
