"""Greedy-stream parity gate (benchmark config 1 shape): Qwen3-0.6B
architecture, seeded random-init weights, sequences with prompt lengths
U[64, 256] and uniform token ids, 32 greedy tokens each, KV block size 256.

The GPU side is the nvkv path inside the Qwen3 driver (bf16, one prefill step
through the tcgen05 kernel, then 31 decode steps through the split-KV decode
kernel).  The reference side is the CPU restatement of the reference's model
(oracle/qwen3_cpu.py) with exactly the same weights, rounding to bf16 at
every op boundary of the reference's bf16 GPU route, so both sides compute
the same arithmetic up to summation order.  Both run the same scheduler
bookkeeping (prepare_model_input, model_runner.rs:69-160) and greedy argmax
(the reference's sampler in the temperature -> 0 limit).  Logits are taken in
the model dtype on both sides, as the reference's lm_head gives them
(embed_head.rs:113), and the greedy pick is their first arg-max.

Bars (the north star's: greedy streams agree at >= 95 % of positions), over
two config-1 request sets (8 sequences, 256 positions), both asserted:
  * teacher forced -- the GPU path fed the reference's own greedy stream;
    its greedy choice must equal the reference's at >= 95 % of positions;
  * the GPU's free-running stream checked by the reference -- the GPU
    generates its own tokens, and at every position the reference's greedy
    choice given that same prefix must equal the GPU's token at >= 95 % of
    positions, i.e. the GPU's stream is the reference's greedy stream except
    where the two take different sides of a near-tie.
A position counts as agreeing when the GPU's token equals the reference's
pick or is a bf16 near-tie of it: its reference logit lies within one bf16
ulp (taken at the row maximum) of the reference's maximum logit.  The
reference hands its logits over in bf16 (embed_head.rs:113), so such tokens
are indistinguishable in its own output up to one rounding step; random-init
logits of magnitude ~150 have ulp 1.0, where top-1/top-2 gaps fall often
enough (a few % of positions) that the summation-order noise of any second
implementation flips some of them.  The exact-match figures are reported
beside the tie-aware ones, and the exact teacher-forced figure must still
reach 90 %.

Reported, not asserted: the raw free-running agreement (each side feeds back
its own tokens, compared position by position) and, for scale, the same
figure between the reference's own fp32 and bf16 CPU routes.  On a 28-layer
random network the first position whose top-2 logits sit within the
implementations' summation-order noise (about one bf16 ulp) sends the two
streams apart for the rest of that sequence, so the raw figure measures how
often such near-ties occur, not the kernels: the reference's two routes
themselves stay near 0.85-0.9 on these models (measured), below the bar.

Random weights are drawn so the stream depends on attention: the embedding
is small (std 0.05) so the layers dominate the residual stream, and lm_head
is untied with std 1 so top-1/top-2 logit gaps dwarf bf16 noise at most
positions.  With tied unit-scale random embeddings the token's own embedding
dominates and the stream merely repeats its input
(tests/test_greedy_sensitivity.py shows this configuration's stream changes
when the oracle's attention is broken).
"""
import numpy as np
import pytest
import torch

import nvkv_oracle as O
import qwen3_cpu as Q
from dataclasses import replace

from nvkv.decoder import QWEN3_0_6B, Qwen3TP, Step

pytestmark = pytest.mark.gpu

P = 256
CFG = replace(QWEN3_0_6B, tie_word_embeddings=False)
NB = 12  # pages: 4 sequences x <= 2 pages each (<= 288 tokens) + spare
INIT = dict(embed_std=0.05, head_std=1.0)


def to_numpy_weights(m: Qwen3TP):
    f = lambda t: t.float().cpu().numpy()  # noqa: E731
    w = {"embed": f(m.embed), "norm": f(m.norm), "lm_head": f(m.lm_head)}
    for i, L in enumerate(m.layers):
        for k in ("qkv", "o", "gate_up", "down", "ln1", "ln2", "qn", "kn"):
            w[f"{i}.{k}"] = f(L[k])
    return w


def make_seqs(seed):
    rng = np.random.default_rng(seed)
    lens = rng.integers(64, 257, 4)
    seqs, free = [], list(range(NB))[::-1]
    for L in lens:
        toks = rng.integers(0, QWEN3_0_6B.vocab_size, int(L)).tolist()
        n = (int(L) + P - 1) // P
        seqs.append(O.Seq(toks, [free.pop() for _ in range(n)], 0, int(L), P))
    return seqs, free


def gpu_generate(model, seqs, steps, free, forced=None):
    """Per-step argmax of the GPU path; appends `forced` tokens when given
    (teacher forcing), else its own choices."""
    out = [[] for _ in seqs]
    dev = model.device
    for step in range(steps):
        ids, pos, ctx = O.prepare_model_input(seqs, P)
        bt = O.prepare_block_tables(seqs)  # the driver always attends through the cache
        cu_q = torch.from_numpy(ctx.cu_seqlens_q.view(np.int32)).to(dev)
        st = Step(torch.from_numpy(ids).to(dev), torch.from_numpy(pos).to(dev),
                  torch.from_numpy(ctx.slot_mapping).to(dev), cu_q,
                  torch.from_numpy(ctx.cu_seqlens_k.view(np.int32)).to(dev),
                  torch.from_numpy(bt.view(np.int32)).to(dev),
                  (cu_q[1:] - 1).long(), ctx.max_seqlen_q, ctx.max_seqlen_k)
        nxt = model.forward(st).argmax(-1).cpu().numpy()
        for o, t in zip(out, nxt):
            o.append(int(t))
        Q.advance(seqs, nxt if forced is None else [f[step] for f in forced], free, P)
    return out


def reference_stream(w, seed, steps=32, dtype="bf16", forced=None, near=None):
    seqs, free = make_seqs(seed)
    return Q.greedy_generate(Q.Qwen3CPU(CFG, w, NB, P, dtype), seqs, steps, free, forced=forced,
                             near=near)


def agree(a, b):
    return float(np.mean([x == y for u, v in zip(a, b) for x, y in zip(u, v)]))


def agree_near(a, b, near):
    """Positions where a's token equals b's or lies in b's bf16 near-tie set."""
    return float(np.mean([x == y or x in n for u, v, m in zip(a, b, near)
                          for x, y, n in zip(u, v, m)]))


def _same(x):
    return x


def streams(model, w, seed, root=True, share=_same):
    """(reference stream and its near-tie sets, GPU teacher forced on it, GPU
    free running, the reference's choices on the GPU's free-running prefix
    and their near-tie sets, the reference's fp32 route free running).
    Under tensor parallelism every rank runs the GPU parts; only the `root`
    rank runs the CPU reference, and `share` hands its stream to the others
    (the others' CPU entries are None)."""
    ref_near, chk_near = [], []
    ref = share(reference_stream(w, seed, near=ref_near) if root else None)
    model.allocate_kv_cache(NB, P)
    seqs, free = make_seqs(seed)
    tf = gpu_generate(model, seqs, 32, free, forced=ref)
    model.allocate_kv_cache(NB, P)
    seqs, free = make_seqs(seed)
    fr = gpu_generate(model, seqs, 32, free)
    if not root:
        return ref, None, tf, fr, None, None, None
    chk = reference_stream(w, seed, forced=fr, near=chk_near)
    ref32 = reference_stream(w, seed, dtype="f32")
    return ref, ref_near, tf, fr, chk, chk_near, ref32


def gate(model, w, seeds=(11, 12), root=True, share=_same):
    """The agreement report (None on a non-root rank)."""
    parts = [streams(model, w, sd, root, share) for sd in seeds]
    if not root:
        return None
    ref, ref_near, tf, fr, chk, chk_near, ref32 = ([x for p in parts for x in p[k]]
                                                   for k in range(7))
    return dict(teacher_forced=agree_near(tf, ref, ref_near),
                gpu_stream_checked_by_reference=agree_near(fr, chk, chk_near),
                teacher_forced_exact=agree(tf, ref),
                gpu_stream_checked_exact=agree(fr, chk),
                free_running_raw=agree(fr, ref), reference_fp32_vs_bf16_raw=agree(ref32, ref),
                distinct_tokens=[len(set(x)) for x in ref])


def passes(report):
    return (report["teacher_forced"] >= 0.95 and report["gpu_stream_checked_by_reference"] >= 0.95
            and report["teacher_forced_exact"] >= 0.90)


def test_greedy_streams_match_cpu_reference():
    model = Qwen3TP(CFG, seed=3, device="cuda", **INIT)
    report = gate(model, to_numpy_weights(model))
    print("greedy agreement", report)
    assert passes(report), report
