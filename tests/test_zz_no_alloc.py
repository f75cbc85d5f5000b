"""nvkv_paged_attention_noalloc: the paged attention entry point for callers
that cannot allocate device memory on the call path (an engine whose KV pool
took nearly all free GPU memory, code inside a stream capture that may not
allocate).  Its split-KV scratch is a fixed static device array instead of a
caller workspace.

The test calls it through the C ABI, twice in a row with different batches
(so the second call runs on the scratch the first one left behind), and
checks each output against the existing nvkv_paged_attention (caller
workspace) within the attention tolerance (max-abs 2e-2, mean-abs 2e-3).  It
also checks that a batch needing more scratch than the fixed maximum is
refused with a clear error.  This file is collected last on purpose.
"""
import ctypes

import numpy as np
import pytest
import torch

import nvkv
from nvkv import ops
from nvkv._lib import ERR_WORKSPACE, lib
from helpers import ATT_MAX_ABS, ATT_MEAN_ABS, cu, f32, make_paged

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


def _batch(lens, hq, hkv, seed):
    g = torch.Generator().manual_seed(seed)
    nb = sum((L + 255) // 256 for L in lens) + 2
    kc, vc, bt, _ = make_paged(lens, 256, hkv, 128, nb, g)
    q = torch.randn(len(lens), hq, 128, generator=g).to(torch.bfloat16).cuda()
    return q, kc, vc, cu([1] * len(lens)), cu(lens), torch.from_numpy(bt.view(np.int32)).cuda()


def _close(a, b):
    d = np.abs(f32(a) - f32(b))
    assert d.max() <= ATT_MAX_ABS and d.mean() <= ATT_MEAN_ABS, (d.max(), d.mean())


def test_noalloc_matches_workspace_entry_two_calls_in_a_row():
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
