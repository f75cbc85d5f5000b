"""nvkv_paged_attention_noalloc: the paged attention entry point for callers
that cannot allocate device memory on the call path (an engine whose KV pool
took nearly all free GPU memory, code inside a stream capture that may not
allocate).  Its split-KV scratch is a fixed static device array instead of a
caller workspace.

The test calls it through the C ABI: first an empty call (num_seqs = 0),
which only looks the static array up, as a caller does at start-up; then
three batches in a row, so each call runs on the scratch the previous one
left behind: two decode batches that split their keys (split-KV partials in
the scratch) and a mixed continuous-batching step whose prompts use the
prefill work plan kept in the same scratch.  Each output is checked against
the existing nvkv_paged_attention (caller workspace), and the mixed step also
against the oracle, within the attention tolerance (max-abs 2e-2, mean-abs
2e-3).  It also checks that a batch needing more scratch than the fixed
maximum is refused with a clear error.  This file is collected last on
purpose.
"""
import ctypes

import numpy as np
import pytest
import torch

import nvkv
import nvkv_oracle as O
from nvkv import ops
from nvkv._lib import ERR_WORKSPACE, lib
from helpers import (ATT_MAX_ABS, ATT_MEAN_ABS, assert_attention_close, cu, f32, gather_seq,
                     make_paged)

pytestmark = pytest.mark.gpu

LIMIT = 4 << 20  # NVKV_NOALLOC_SCRATCH_BYTES in include/nvkv.h


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _noalloc(q, kc, vc, cu_q, cu_k, bt, max_q, max_k, scale, out):
    T, hq, d = q.shape
    return lib.nvkv_paged_attention_noalloc(
        _p(q), q.stride(0), T, _p(kc), _p(vc), kc.size(0), 0, _p(out), _p(cu_q), _p(cu_k), _p(bt),
        bt.size(1), cu_q.numel() - 1, max_q, max_k, hq, kc.size(2), d, kc.size(1),
        ctypes.c_float(scale), 1, 1, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


def _mixed_step(hq, hkv, seed):
    """A config-3-shaped continuous-batching step (Qwen3-4B heads): 120
    decoding sequences with contexts U[129, 2304], two fresh prompts and one
    prefix-cache-hit chunk, rows interleaved; enough rows that the prefill
    kernel runs from its work plan."""
    rng = np.random.default_rng(seed)
    dec = rng.integers(129, 2305, 120).tolist()
    q_lens = [1] * len(dec) + [700, 1300, 150]
    k_lens = dec + [700, 1300, 150 + 512]
    order = rng.permutation(len(q_lens))
    q_lens = [q_lens[i] for i in order]
    k_lens = [k_lens[i] for i in order]
    g = torch.Generator().manual_seed(seed)
    nb = sum((L + 255) // 256 for L in k_lens) + 2
    kc, vc, bt, tables = make_paged(k_lens, 256, hkv, 128, nb, g)
    q = torch.randn(sum(q_lens), hq, 128, generator=g).to(torch.bfloat16).cuda()
    return (q, kc, vc, cu(q_lens), cu(k_lens), torch.from_numpy(bt.view(np.int32)).cuda(),
            q_lens, k_lens, tables)


def _batch(lens, hq, hkv, seed):
    g = torch.Generator().manual_seed(seed)
    nb = sum((L + 255) // 256 for L in lens) + 2
    kc, vc, bt, _ = make_paged(lens, 256, hkv, 128, nb, g)
    q = torch.randn(len(lens), hq, 128, generator=g).to(torch.bfloat16).cuda()
    return q, kc, vc, cu([1] * len(lens)), cu(lens), torch.from_numpy(bt.view(np.int32)).cuda()


def _close(a, b):
    d = np.abs(f32(a) - f32(b))
    assert d.max() <= ATT_MAX_ABS and d.mean() <= ATT_MEAN_ABS, (d.max(), d.mean())


def test_noalloc_matches_workspace_entry_calls_in_a_row():
    # start-up: an empty call does the one-time lookup of the static array
    rc = lib.nvkv_paged_attention_noalloc(None, 0, 0, None, None, 0, 0, None, None, None, None,
                                          0, 0, 0, 0, 32, 8, 128, 256, ctypes.c_float(0.1), 1, 1,
                                          None)
    assert rc == 0, lib.nvkv_last_error()
    cases = [
        # config 2 shape (16 q / 8 kv heads, L ~ U[512, 4096]): split-KV + combine
        (np.random.default_rng(2).integers(512, 4097, 64).tolist(), 16, 8, 1),
        # long contexts at 1 kv head (the 32B TP8 shape): many splits
        ([32768, 9000, 300, 4096], 8, 1, 2),
    ]
    for lens, hq, hkv, seed in cases:
        q, kc, vc, cq, ck, bt = _batch(lens, hq, hkv, seed)
        assert 0 < ops.workspace_size(len(lens), hq, hkv, 1, max(lens)) <= LIMIT
        ref = ops.paged_attention(q, kc, vc, cq, ck, bt, 1, max(lens), 128 ** -0.5)
        out = torch.full_like(q, float("nan"))
        rc = _noalloc(q, kc, vc, cq, ck, bt, 1, max(lens), 128 ** -0.5, out)
        assert rc == 0, lib.nvkv_last_error()
        torch.cuda.synchronize()
        _close(out, ref)
    # third call: a mixed step, prefill work plan in the static scratch
    q, kc, vc, cq, ck, bt, q_lens, k_lens, tables = _mixed_step(32, 8, 3)
    max_q, max_k = max(q_lens), max(k_lens)
    assert ops.workspace_size(len(q_lens), 32, 8, max_q, max_k) <= LIMIT
    ref = ops.paged_attention(q, kc, vc, cq, ck, bt, max_q, max_k, 128 ** -0.5)
    out = torch.full_like(q, float("nan"))
    rc = _noalloc(q, kc, vc, cq, ck, bt, max_q, max_k, 128 ** -0.5, out)
    assert rc == 0, lib.nvkv_last_error()
    torch.cuda.synchronize()
    _close(out, ref)
    c = np.cumsum([0] + q_lens)
    qn = f32(q)
    for b in range(len(q_lens)):
        if q_lens[b] > 1 or b % 10 == 0:  # every prompt and a sample of decode rows
            kb, vb = gather_seq(kc, vc, tables[b], k_lens[b])
            want = O.causal_attention_one(qn[c[b]:c[b + 1]], kb, vb, 128 ** -0.5, True)
            assert_attention_close(out[c[b]:c[b + 1]], want, f"mixed step, sequence {b}")
    assert nvkv.device_error() == 0


def test_noalloc_refuses_batches_above_the_static_scratch():
    lens = [32768] * 64  # 16 q heads on 1 kv head: plan needs > 4 MiB of partials
    hq, hkv = 16, 1
    need = ops.workspace_size(len(lens), hq, hkv, 1, max(lens))
    assert need > LIMIT
    x = torch.zeros(64, hq, 128, dtype=torch.bfloat16, device="cuda")
    kc = torch.zeros(2, 256, hkv, 128, dtype=torch.bfloat16, device="cuda")
    bt = torch.zeros(64, 128, dtype=torch.int32, device="cuda")
    rc = _noalloc(x, kc, kc, cu([1] * 64), cu(lens), bt, 1, max(lens), 0.1, x)
    assert rc == ERR_WORKSPACE
    assert b"static scratch" in lib.nvkv_last_error()
