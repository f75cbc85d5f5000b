"""Per-kernel microbenchmarks of the nvkv path (CUDA-event timed).

    python kbench.py [--case NAME ...] [--iters N]

Cases (one JSON line each; bytes/flops are the algorithmic figures):
  store_cfg2      nvkv_store_kvcache, benchmark config 2: 64 tokens + 8 padded
                  slots, 8 kv heads, 2048-block pool                     (HBM)
  store_prefill   the same at T = 16384 (a full 16384-token prefill step)  (HBM)
  prologue_8b     nvkv_qknorm_rope + fused store, Qwen3-8B TP1 decode T=256 (HBM)
  decode_cfg2     nvkv_paged_attention decode, config 2: B=64, 16q/8kv,
                  L ~ U[512,4096], P=256, 2048-block pool                 (HBM)
  decode_8b_tp1   one layer of the Qwen3-8B TP1 decode step (B=256, 32q/8kv) (HBM)
  decode_8b_tp8   the same layer at TP8 per GPU (4q/1kv)                   (HBM)
  decode_32b_tp8  Qwen3-32B TP8 per GPU: B=64, 8q/1kv, L=32768            (HBM)
  prefill_8b      tcgen05 prefill, Qwen3-8B TP1: 16 prompts x 1024, causal (tensor)
  step_metadata   device-side decode-step metadata, 256 sequences (latency)
  mixed_4b_tp1/2  config 3 (Qwen3-4B): 120 decodes + 8 fresh prompts in one
                  call, with the decode-only and prefill-only parts     (mixed)
  block_manager   host KV block manager: 256 x 1024-token prompts (half
                  sharing a 512-token prefix) admitted, then decode steps (host)
  step_prepare    host step metadata (prepare_model_input): config 4's decode
                  step and a 16 x 1024 prefill step                     (host)
Inputs of every HBM case exceed L2 or are rotated through enough copies
that each timed launch reads cold data.
"""
from __future__ import annotations

import argparse
import json
import os

import sys

import numpy as np
import torch

_ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(_ROOT, "nanovllm-rs_b200"))

from nvkv import ops  # noqa: E402


def _peaks():
    try:
        p = json.load(open(os.path.join(_ROOT, "MEASURED_PEAKS.json")))
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


def _time(fn, iters, warmup=3):
    """Mean device time per launch: `iters` launches are captured into one
    CUDA graph and the replay is timed with two CUDA events, so no host
    overhead sits between launches (what a graph-captured decode step sees)."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(warmup):
            fn(0)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(iters):
            fn(i)
    g.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    g.replay()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) * 1e-3 / iters, None


# --copies N: every paged-decode case keeps only N copies of its pool (a small
# case for an ncu capture; timings then run on L2-warm inputs when N is small)
COPIES = None


def _paged(lens, page, hkv, nblocks, seed, copies=1):
    g = torch.Generator(device="cuda").manual_seed(seed)
    rng = np.random.default_rng(seed)
    need = [(int(L) + page - 1) // page for L in lens]
    assert sum(need) <= nblocks
    perm = rng.permutation(nblocks)
    bt = np.zeros((len(lens), max(need)), np.int32)
    u = 0
    for i, n in enumerate(need):
        bt[i, :n] = perm[u:u + n]
        u += n
    caches = [(torch.randn(nblocks, page, hkv, 128, generator=g, device="cuda",
                           dtype=torch.bfloat16),
               torch.randn(nblocks, page, hkv, 128, generator=g, device="cuda",
                           dtype=torch.bfloat16)) for _ in range(copies)]
    return caches, torch.from_numpy(bt).cuda()


def case_store(T, pad, iters):
    hkv, page, nb = 8, 256, 2048
    rng = np.random.default_rng(0)
    slots = rng.choice(nb * page, T, replace=False).astype(np.int64)
    slots[rng.choice(T, pad, replace=False)] = -1 if pad else slots[:0]
    sm = torch.from_numpy(slots).cuda()
    copies = 8 if T < 4096 else 2
    srcs = [(torch.randn(T, hkv, 128, device="cuda").bfloat16(),
             torch.randn(T, hkv, 128, device="cuda").bfloat16()) for _ in range(copies)]
    kc = torch.zeros(nb, page, hkv, 128, device="cuda", dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    fn = lambda i: ops.store_kvcache(srcs[i % copies][0], srcs[i % copies][1], kc, vc, sm)  # noqa
    med, mn = _time(fn, iters)
    valid = int((slots >= 0).sum())
    nbytes = 2 * 2 * valid * hkv * 128 * 2 + 8 * T
    return dict(kernel="store_kvcache", T=T, valid=valid, bytes=nbytes, s=med, bound="hbm")


def case_prologue(T, iters):
    hq, hkv, page = 32, 8, 256
    nb = (T + page - 1) // page + 4
    qkv = [torch.randn(T, (hq + 2 * hkv) * 128, device="cuda").bfloat16() for _ in range(4)]
    pos = torch.randint(0, 40960, (T,), device="cuda")
    slots = torch.from_numpy(np.random.default_rng(1).choice(nb * page, T, replace=False)).cuda()
    w = torch.ones(128, device="cuda", dtype=torch.bfloat16)
    kc = torch.zeros(nb, page, hkv, 128, device="cuda", dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    qo = torch.empty(T, hq, 128, device="cuda", dtype=torch.bfloat16)
    fn = lambda i: ops.qknorm_rope(qkv[i % 4], pos, hq, hkv, w, w, 1e-6, 1e6, 40960,  # noqa
                                   k_cache=kc, v_cache=vc, slot_mapping=slots, q_out=qo)
    med, _ = _time(fn, iters)
    nbytes = T * (hq + 2 * hkv) * 128 * 2 + T * (hq + 2 * hkv) * 128 * 2 + 2 * 8 * T
    return dict(kernel="qknorm_rope+store", T=T, bytes=nbytes, s=med, bound="hbm")


def case_decode(name, lens, hq, hkv, nblocks, iters, copies=1):
    copies = COPIES or copies
    page = 256
    caches, bt = _paged(lens, page, hkv, nblocks, 3, copies)
    B = len(lens)
    q = torch.randn(B, hq, 128, device="cuda").bfloat16()
    cu_q = torch.arange(B + 1, dtype=torch.int32, device="cuda")
    cu_k = torch.from_numpy(np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)).cuda()
    out = torch.empty_like(q)
    ws = torch.empty(max(16, ops.workspace_size(B, hq, hkv, 1, int(max(lens)))),
                     dtype=torch.uint8, device="cuda")
    fn = lambda i: ops.paged_attention(q, caches[i % copies][0], caches[i % copies][1],  # noqa
                                       cu_q, cu_k, bt, 1, int(max(lens)), 128 ** -0.5, out=out,
                                       workspace=ws)
    med, _ = _time(fn, iters)
    nblk = sum((int(L) + page - 1) // page for L in lens)
    nbytes = int(np.sum(lens)) * hkv * 128 * 2 * 2 + 2 * B * hq * 128 * 2 + 4 * nblk + 8 * (B + 1)
    return dict(kernel=name, B=B, hq=hq, hkv=hkv, L_mean=float(np.mean(lens)), bytes=nbytes, s=med,
                splits=bool(ops.workspace_size(B, hq, hkv, 1, int(max(lens)))), bound="hbm")


def case_decode_fp8(name, lens, hq, hkv, nblocks, iters, copies=1):
    """case_decode over the fp8 (e4m3) pool: codes and per-row scales written
    by nvkv_store_kvcache_fp8 from random rows.  Algorithmic bytes: one byte
    per K/V value plus the 4-byte row scales, q and out, block tables."""
    copies = COPIES or copies
    page = 256
    caches, bt = _paged(lens, page, hkv, nblocks, 3, copies)
    pools = []
    slots = torch.arange(nblocks * page, device="cuda")
    for kc, vc in caches:
        k8 = torch.empty(nblocks, page, hkv, 128, dtype=torch.uint8, device="cuda")
        v8 = torch.empty_like(k8)
        ks = torch.empty(nblocks, hkv, page, dtype=torch.float32, device="cuda")
        vs = torch.empty_like(ks)
        ops.store_kvcache_fp8(kc.view(-1, hkv, 128), vc.view(-1, hkv, 128), k8, v8, ks, vs, slots)
        pools.append((k8, v8, ks, vs))
    del caches
    torch.cuda.empty_cache()
    B = len(lens)
    q = torch.randn(B, hq, 128, device="cuda").bfloat16()
    cu_q = torch.arange(B + 1, dtype=torch.int32, device="cuda")
    cu_k = torch.from_numpy(np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)).cuda()
    out = torch.empty_like(q)
    ws = torch.empty(max(16, ops.workspace_size_fp8(B, hq, hkv, 1, int(max(lens)), 0)),
                     dtype=torch.uint8, device="cuda")
    fn = lambda i: ops.paged_attention_fp8(q, *pools[i % copies], cu_q, cu_k, bt, 1,  # noqa
                                           int(max(lens)), 128 ** -0.5, out=out, workspace=ws)
    med, _ = _time(fn, iters)
    nblk = sum((int(L) + page - 1) // page for L in lens)
    nbytes = (int(np.sum(lens)) * hkv * (128 + 4) * 2 + 2 * B * hq * 128 * 2 + 4 * nblk +
              8 * (B + 1))
    return dict(kernel=name, B=B, hq=hq, hkv=hkv, L_mean=float(np.mean(lens)), bytes=nbytes, s=med,
                bound="hbm", kv="e4m3 + f32 row scales")


def case_sample(name, B, V, iters):
    """nvkv_sample over [B, V] bf16 logits (a TP shard when V < 151936): one
    read of the logits plus 2.5 Philox4x32-10 calls per 8 entries."""
    lg = (torch.randn(B, V, device="cuda") * 3).bfloat16()
    temps = torch.full((B,), 0.8, device="cuda")
    v = torch.empty(B, dtype=torch.float32, device="cuda")
    ix = torch.empty(B, dtype=torch.int64, device="cuda")
    fn = lambda i: ops.sample(lg, temps, 7, i, out_value=v, out_index=ix)  # noqa: E731
    med, _ = _time(fn, iters)
    return dict(kernel=name, B=B, V=V, bytes=B * V * 2, s=med, bound="latency")


def case_step_metadata(B, iters, P=256):
    """nvkv_decode_advance on a B-sequence decode step (lengths U[1025,1536],
    pages appended ahead): the device replacement of the host-side metadata
    build + H2D of positions / slot_mapping / cu_seqlens."""
    rng = np.random.default_rng(7)
    lens = rng.integers(1025, 1537, B)
    width = int((lens.max() + 64 * iters + P - 1) // P)
    bt = torch.from_numpy(rng.permutation(B * width).astype(np.int32).reshape(B, width)).cuda()
    seq_lens = torch.from_numpy(lens - 1).cuda()
    pos = torch.empty(B, dtype=torch.int64, device="cuda")
    slots = torch.empty_like(pos)
    cuq = torch.empty(B + 1, dtype=torch.int32, device="cuda")
    cuk = torch.empty_like(cuq)
    fn = lambda i: ops.decode_advance(seq_lens, bt, B * width, P, pos, slots, cuq, cuk)  # noqa
    med, _ = _time(fn, iters)
    return dict(kernel="decode_advance", B=B, bytes=B * (8 * 3 + 4 * 2 + 4), s=med, bound="latency")


def case_prefill(iters, nseq=16, L=1024, hq=32, hkv=8):
    page = 256
    lens = [L] * nseq
    caches, bt = _paged(lens, page, hkv, nseq * L // page + 2, 5)
    T = nseq * L
    q = torch.randn(T, hq, 128, device="cuda").bfloat16()
    cu = torch.from_numpy(np.arange(0, T + 1, L).astype(np.int32)).cuda()
    out = torch.empty_like(q)
    ws = torch.empty(max(16, ops.workspace_size(nseq, hq, hkv, L, L)), dtype=torch.uint8,
                     device="cuda")
    fn = lambda i: ops.paged_attention(q, caches[0][0], caches[0][1], cu, cu, bt, L, L,  # noqa
                                       128 ** -0.5, out=out, workspace=ws)
    med, _ = _time(fn, iters)
    pairs = nseq * L * (L + 1) // 2
    return dict(kernel="prefill_tcgen05", nseq=nseq, L=L, hq=hq, hkv=hkv,
                flops=4 * 128 * hq * pairs, s=med, bound="tensor")


def case_mixed(iters, tp=1):
    """benchmark config 3 (Qwen3-4B, 32q/8kv, TP1/2): one continuous-batching
    step of 120 decoding sequences (contexts U[129, 2304]) and 8 fresh
    prompts U[128, 2048] in one nvkv_paged_attention call (decode kernel +
    tcgen05 kernel), and each part alone for the split."""
    page, hq, hkv = 256, 32 // tp, 8 // tp
    rng = np.random.default_rng(9)
    dec = rng.integers(129, 2305, 120)
    pre = rng.integers(128, 2049, 8)
    order = rng.permutation(128)
    q_all = np.concatenate([np.ones(120, np.int64), pre])[order]
    k_all = np.concatenate([dec, pre])[order]
    nblk = int(sum((int(L) + page - 1) // page for L in k_all)) + 2
    caches, bt_all = _paged(k_all, page, hkv, nblk, 11)
    kc, vc = caches[0]

    def setup(qs, ks, sel):
        T = int(qs.sum())
        q = torch.randn(T, hq, 128, device="cuda").bfloat16()
        cuq = torch.from_numpy(np.concatenate([[0], np.cumsum(qs)]).astype(np.int32)).cuda()
        cuk = torch.from_numpy(np.concatenate([[0], np.cumsum(ks)]).astype(np.int32)).cuda()
        bt = bt_all[torch.from_numpy(sel).cuda()].contiguous()
        mq, mk = int(qs.max()), int(ks.max())
        ws = torch.empty(max(16, ops.workspace_size(len(qs), hq, hkv, mq, mk)), dtype=torch.uint8,
                         device="cuda")
        out = torch.empty_like(q)
        return lambda i: ops.paged_attention(q, kc, vc, cuq, cuk, bt, mq, mk, 128 ** -0.5,  # noqa
                                             out=out, workspace=ws)

    idx = np.arange(128)
    t_mix, _ = _time(setup(q_all, k_all, idx), iters)
    d = q_all == 1
    t_dec, _ = _time(setup(q_all[d], k_all[d], idx[d]), iters)
    t_pre, _ = _time(setup(q_all[~d], k_all[~d], idx[~d]), iters)
    dbytes = int(k_all[d].sum()) * hkv * 128 * 2 * 2 + 2 * int(d.sum()) * hq * 128 * 2
    pairs = int(sum(int(L) * (int(L) + 1) // 2 for L in k_all[~d]))
    return dict(kernel="mixed_step", tp=tp, hq=hq, hkv=hkv, decode_seqs=int(d.sum()),
                prefill_tokens=int(q_all[~d].sum()), bytes=dbytes, flops=4 * 128 * hq * pairs,
                s=t_mix, decode_only_us=round(t_dec * 1e6, 2), prefill_only_us=round(t_pre * 1e6, 2),
                bound="mixed")


def case_block_manager(iters, B=256, prompt=1024, shared=512, page=256, steps=64):
    """KV block manager (nvkv_block_manager_*, host): admission of B prompts
    (half share a `shared`-token prefix: prefix-cache hits), then `steps`
    decode steps of can_append + may_append for every sequence, through the
    C ABI with each sequence's buffers passed in place, as a compiled caller
    would (ctypes adds ~1 us per call).  Timed on the host clock; the
    reference's Rust manager does the same work (a Python restatement is
    timed beside it as the CPU baseline)."""
    import ctypes
    import time
    from nvkv._lib import BlockSeq, lib
    rng = np.random.default_rng(12)
    pre = rng.integers(0, 151936, shared).astype(np.uint32)
    cap_tok = prompt + steps * iters + 8
    nb = B * ((cap_tok + page - 1) // page) + 8

    def build():
        h = ctypes.c_void_p()
        assert lib.nvkv_block_manager_create(nb, page, ctypes.byref(h)) == 0
        seqs = []
        for b in range(B):
            toks = np.zeros(cap_tok, np.uint32)
            toks[:prompt] = rng.integers(0, 151936, prompt)
            if b % 2 == 0:
                toks[:shared] = pre
            table = np.zeros((cap_tok + page - 1) // page + 1, np.uint32)
            c = BlockSeq(toks.ctypes.data, prompt, 0, prompt, table.ctypes.data, 0, table.size)
            seqs.append((toks, table, c))
        return h, seqs

    def run(h, seqs, n_steps):
        u, f, n, ok = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int()
        t0 = time.perf_counter()
        for toks, table, c in seqs:
            c.num_new_tokens = 0
            assert lib.nvkv_block_manager_get_token_layout(h, ctypes.byref(c), ctypes.byref(u),
                                                           ctypes.byref(f), ctypes.byref(n)) == 0
            assert lib.nvkv_block_manager_can_allocate(h, f.value + n.value, ctypes.byref(ok)) == 0
            c.num_new_tokens = n.value
            assert lib.nvkv_block_manager_allocate(h, ctypes.byref(c)) == 0
            c.num_cached_tokens += c.num_new_tokens
            c.num_new_tokens = 0
        t1 = time.perf_counter()
        for _ in range(n_steps):
            for toks, table, c in seqs:
                toks[c.num_tokens] = 7
                c.num_tokens += 1
                assert lib.nvkv_block_manager_can_append(h, ctypes.byref(c), 1, ctypes.byref(ok)) == 0
                c.num_new_tokens = 1
                assert lib.nvkv_block_manager_may_append(h, ctypes.byref(c)) == 0
                c.num_cached_tokens += 1
                c.num_new_tokens = 0
        t2 = time.perf_counter()
        return t1 - t0, t2 - t1

    def run_batched(h, seqs, n_steps):
        arr = (BlockSeq * len(seqs))(*[c for _, _, c in seqs])
        ones = np.ones(len(seqs), np.int64)
        done = ctypes.c_int64(0)
        t_call = 0.0  # only the library call: the Python field updates around it are the
        for _ in range(n_steps):  # benchmark's own bookkeeping, not the manager's work
            for k, (toks, table, _) in enumerate(seqs):
                toks[arr[k].num_tokens] = 7
                arr[k].num_tokens += 1
            t0 = time.perf_counter()
            rc = lib.nvkv_block_manager_append_batch(h, arr, len(seqs), ones.ctypes.data,
                                                     ctypes.byref(done))
            t_call += time.perf_counter() - t0
            assert rc == 0 and done.value == len(seqs)
            for k in range(len(seqs)):
                arr[k].num_cached_tokens += 1
                arr[k].num_new_tokens = 0
        return t_call

    h, seqs = build()
    adm, dec = run(h, seqs, steps)
    lib.nvkv_block_manager_destroy(h)
    h, seqs = build()
    run(h, seqs, 0)
    dec_b = run_batched(h, seqs, steps)
    lib.nvkv_block_manager_destroy(h)
    return dict(kernel="block_manager (host C++)", B=B, prompt=prompt, shared_prefix=shared,
                page=page, decode_steps=steps, admission_us_per_seq=round(adm / B * 1e6, 2),
                decode_step_us=round(dec / steps * 1e6, 1),
                decode_step_batched_us=round(dec_b / steps * 1e6, 1), s=adm + dec, bound="host")


def step_prepare_inputs(kind, B=256, page=256, seed=13):
    """Sequence views of one step: "decode" = config 4's decode step (B
    sequences, contexts U[1025, 1536], one new token each); "prefill" = 16
    fresh 1024-token prompts."""
    import ctypes
    from nvkv._lib import BlockSeq
    rng = np.random.default_rng(seed)
    if kind == "decode":
        ctx = rng.integers(1025, 1537, B)
        new = np.ones(B, np.int64)
    else:
        ctx = np.full(16, 1024)
        new = ctx.copy()
    keep, seqs = [], []
    perm = rng.permutation(int(((ctx + page - 1) // page).sum()) + 8).astype(np.uint32)
    used = 0
    for L, n in zip(ctx, new):
        toks = rng.integers(0, 151936, int(L)).astype(np.uint32)
        nb = (int(L) + page - 1) // page
        table = np.ascontiguousarray(perm[used:used + nb])
        used += nb
        keep += [toks, table]
        seqs.append(BlockSeq(toks.ctypes.data, int(L), int(L - n), int(n), table.ctypes.data, nb,
                             nb))
    arr = (BlockSeq * len(seqs))(*seqs)
    return arr, keep, [(t, tb) for t, tb in zip(keep[0::2], keep[1::2])], ctx, new


def case_step_prepare(iters, reps=200):
    """nvkv_prepare_step (host): config 4's 256-sequence decode step and a
    16 x 1024 prefill step, outputs in preallocated host buffers; host clock,
    mean over `reps` calls (ctypes adds ~1 us per call)."""
    import ctypes
    import time
    from nvkv._lib import StepSizes, lib
    res = {}
    for kind in ("decode", "prefill"):
        arr, keep, _, ctx, new = step_prepare_inputs(kind)
        B = len(arr)
        sz = StepSizes()
        assert lib.nvkv_prepare_step(arr, B, 256, None, None, None, None, None, None, None, None,
                                     0, 0, 0, ctypes.byref(sz)) == 0
        bufs = [np.zeros(max(int(n), 1), dt) for n, dt in
                ((sz.num_tokens, np.int64), (sz.num_tokens, np.int64), (B + 1, np.uint32),
                 (B + 1, np.uint32), (sz.num_slots, np.int64), (B, np.int64),
                 (sz.num_need_logits, np.int64), (B * sz.block_table_width, np.uint32))]
        args = [b.ctypes.data for b in bufs]
        t0 = time.perf_counter()
        for _ in range(reps):
            rc = lib.nvkv_prepare_step(arr, B, 256, *args, bufs[0].size, bufs[4].size,
                                       bufs[7].size, ctypes.byref(sz))
        dt = (time.perf_counter() - t0) / reps
        assert rc == 0
        res[kind + "_us"] = round(dt * 1e6, 2)
        res[kind + "_tokens"] = int(sz.num_tokens)
    return dict(kernel="prepare_step (host C++)", **res, s=res["decode_us"] * 1e-6, bound="host")


CASES = {
    "store_cfg2": lambda it: case_store(72, 8, it),
    "store_prefill": lambda it: case_store(16384, 0, it),
    "prologue_8b": lambda it: case_prologue(256, it),
    "decode_cfg2": lambda it: case_decode(
        "decode_cfg2", np.random.default_rng(2).integers(512, 4097, 64), 16, 8, 2048, it, 4),
    "decode_8b_tp1": lambda it: case_decode(
        "decode_8b_tp1", np.random.default_rng(4).integers(1025, 1537, 256), 32, 8, 1560, it, 2),
    "decode_8b_tp2": lambda it: case_decode(
        "decode_8b_tp2", np.random.default_rng(4).integers(1025, 1537, 256), 16, 4, 1560, it, 2),
    "decode_8b_tp8": lambda it: case_decode(
        "decode_8b_tp8", np.random.default_rng(4).integers(1025, 1537, 256), 4, 1, 1560, it, 8),
    "decode_8b_tp8_2k": lambda it: case_decode(
        "decode_8b_tp8_2k", np.random.default_rng(5).integers(1537, 2561, 256), 4, 1, 2900, it, 8),
    "decode_8b_tp8_skew": lambda it: case_decode(
        "decode_8b_tp8_skew", np.concatenate([np.random.default_rng(6).integers(64, 513, 255),
                                              [1536]]), 4, 1, 600, it, 8),
    "decode_32b_tp8": lambda it: case_decode(
        "decode_32b_tp8", np.full(64, 32768), 8, 1, 64 * 128 + 2, it, 2),
    "decode_8b_tp1_fp8": lambda it: case_decode_fp8(
        "decode_8b_tp1_fp8", np.random.default_rng(4).integers(1025, 1537, 256), 32, 8, 1560, it,
        2),
    "decode_8b_tp2_fp8": lambda it: case_decode_fp8(
        "decode_8b_tp2_fp8", np.random.default_rng(4).integers(1025, 1537, 256), 16, 4, 1560, it,
        4),
    "decode_8b_tp8_fp8": lambda it: case_decode_fp8(
        "decode_8b_tp8_fp8", np.random.default_rng(4).integers(1025, 1537, 256), 4, 1, 1560, it,
        8),
    "decode_32b_tp8_fp8": lambda it: case_decode_fp8(
        "decode_32b_tp8_fp8", np.full(64, 32768), 8, 1, 64 * 128 + 2, it, 2),
    "sample_8b_tp1": lambda it: case_sample("sample_8b_tp1", 256, 151936, it),
    "sample_8b_tp8": lambda it: case_sample("sample_8b_tp8", 256, 151936 // 8, it),
    "decode_g16": lambda it: case_decode(
        "decode_g16", np.random.default_rng(8).integers(2048, 4097, 64), 16, 1, 1100, it, 8),
    "decode_g16_fp8": lambda it: case_decode_fp8(
        "decode_g16_fp8", np.random.default_rng(8).integers(2048, 4097, 64), 16, 1, 1100, it, 8),
    "prefill_8b": lambda it: case_prefill(it),
    "step_metadata": lambda it: case_step_metadata(256, it),
    "mixed_4b_tp1": lambda it: case_mixed(it, 1),
    "mixed_4b_tp2": lambda it: case_mixed(it, 2),
    "block_manager": lambda it: case_block_manager(it),
    "step_prepare": lambda it: case_step_prepare(it),
}


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--case", nargs="*", default=list(CASES))
    ap.add_argument("--iters", type=int, default=50)
    ap.add_argument("--copies", type=int, default=None,
                    help="pool copies per paged-decode case (default: the case's own)")
    a = ap.parse_args(argv)
    global COPIES
    COPIES = a.copies
    hbm, tf, src = _peaks()
    for name in a.case:
        r = CASES[name](a.iters)
        if r["bound"] in ("latency", "host"):  # only the time means anything
            r.update(case=name, us=round(r["s"] * 1e6, 2))
        elif r["bound"] == "mixed":  # each part against its own roofline, timed alone
            gbs = r["bytes"] / (r["decode_only_us"] * 1e-6) / 1e9
            tfs = r["flops"] / (r["prefill_only_us"] * 1e-6) / 1e12
            r.update(case=name, us=round(r["s"] * 1e6, 2),
                     decode_gbs=round(gbs, 1), decode_frac=round(gbs / hbm, 4),
                     prefill_tflops=round(tfs, 1), prefill_frac=round(tfs / tf, 4),
                     parts_sum_over_mixed=round((r["decode_only_us"] + r["prefill_only_us"])
                                                / (r["s"] * 1e6), 3), peak_source=src)
        elif r["bound"] == "hbm":
            ach = r["bytes"] / r["s"] / 1e9
            r.update(case=name, us=round(r["s"] * 1e6, 2), achieved_gbs=round(ach, 1),
                     peak_gbs=hbm, frac=round(ach / hbm, 4), peak_source=src)
        else:
            ach = r["flops"] / r["s"] / 1e12
            r.update(case=name, us=round(r["s"] * 1e6, 2), achieved_tflops=round(ach, 1),
                     peak_tflops=tf, frac=round(ach / tf, 4), peak_source=src)
        r.pop("s")
        print(json.dumps(r), flush=True)
    if torch.cuda.is_available():
        from nvkv._lib import device_error
        assert device_error() == 0


if __name__ == "__main__":
    main()
