"""The reference-shaped surface end to end: set_context + Attention.forward
(store through slot_mapping, then attention through block_tables or on the
fresh K/V), driven by the oracle's prepare_model_input over a prefill step
followed by decode steps -- the way ModelRunner::run drives
layers/attention.rs:24-76.  Compared with the oracle's attention_forward."""
import numpy as np
import pytest
import torch

import nvkv
import nvkv_oracle as O
from helpers import assert_attention_close, bits, f32

pytestmark = pytest.mark.gpu


def _tensor_ctx(ctx):
    dev = "cuda"
    bt = None if ctx.block_tables is None else torch.from_numpy(
        ctx.block_tables.view(np.int32)).to(dev)
    return dict(cu_seqlens_q=torch.from_numpy(ctx.cu_seqlens_q.view(np.int32)).to(dev),
                cu_seqlens_k=torch.from_numpy(ctx.cu_seqlens_k.view(np.int32)).to(dev),
                max_seqlen_q=ctx.max_seqlen_q, max_seqlen_k=ctx.max_seqlen_k,
                slot_mapping=torch.from_numpy(ctx.slot_mapping).to(dev),
                context_lens=torch.from_numpy(ctx.context_lens).to(dev), block_tables=bt)


def test_prefill_then_decode_steps_through_attention_object():
    P, hq, hkv, d, nb = 256, 16, 8, 128, 16
    g = torch.Generator().manual_seed(0)
    rng = np.random.default_rng(0)
    prompts = [300, 17, 512]
    free = list(rng.permutation(nb))
    seqs = []
    for L in prompts:
        nblk = (L + P - 1) // P
        seqs.append(O.Seq(list(rng.integers(0, 1000, L)), [int(free.pop()) for _ in range(nblk)],
                          0, L, P))
    attn = nvkv.Attention(d ** -0.5)
    kc = torch.zeros(nb, P, hkv, d, dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    attn.set_kv_cache(kc, vc)
    kc_ref = np.zeros((nb, P, hkv, d), np.float32)
    vc_ref = np.zeros_like(kc_ref)
    for step in range(4):
        _, _, ctx = O.prepare_model_input(seqs, P)
        T = int(ctx.cu_seqlens_q[-1])
        qkv = torch.randn(T, (hq + 2 * hkv) * d, generator=g).to(torch.bfloat16).cuda()
        q = qkv[:, :hq * d].view(T, hq, d)
        k = qkv[:, hq * d:(hq + hkv) * d].view(T, hkv, d)
        v = qkv[:, (hq + hkv) * d:].view(T, hkv, d)
        nvkv.set_context(**_tensor_ctx(ctx))
        out = attn(q, k, v)
        torch.cuda.synchronize()
        nvkv.reset_context()
        want = O.attention_forward(f32(q), f32(k), f32(v), ctx, kc_ref, vc_ref, d ** -0.5)
        assert np.array_equal(f32(kc), kc_ref) and np.array_equal(f32(vc), vc_ref), step
        assert_attention_close(out, want, f"step {step}")
        # advance every sequence by one decode token (scheduler/postprocess shape)
        for s in seqs:
            s.num_cached_tokens = s.num_context_tokens()
            s.token_ids.append(int(rng.integers(0, 1000)))
            s.num_new_tokens = 1
            if (len(s.token_ids) + P - 1) // P > len(s.block_table):
                s.block_table.append(int(free.pop()))
    assert nvkv.device_error() == 0


def test_warmup_without_cache_uses_fresh_kv():
    """ModelRunner::warmup_model: no cache attached, no block tables, no slots."""
    hq, hkv, d = 8, 2, 128
    g = torch.Generator().manual_seed(1)
    lens = [40, 200]
    T = sum(lens)
    qkv = torch.randn(T, (hq + 2 * hkv) * d, generator=g).to(torch.bfloat16).cuda()
    q = qkv[:, :hq * d].view(T, hq, d)
    k = qkv[:, hq * d:(hq + hkv) * d].view(T, hkv, d)
    v = qkv[:, (hq + hkv) * d:].view(T, hkv, d)
    cu = torch.tensor([0, 40, 240], dtype=torch.int32, device="cuda")
    nvkv.set_context(cu, cu, 200, 200)
    out = nvkv.Attention(0.1)(q, k, v)
    torch.cuda.synchronize()
    nvkv.reset_context()
    want = O.varlen_attention(f32(q), f32(k), f32(v), [0, 40, 240], [0, 40, 240], 0.1)
    assert_attention_close(out, want, "warmup")


def test_missing_context_errors_like_reference():
    nvkv.reset_context()
    x = torch.zeros(1, 8, 128, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(nvkv.NvkvError, match="cu_seqlens_q"):
        nvkv.Attention(0.1)(x, x[:, :2], x[:, :2])
