"""Kernel 4 (nvkv_qknorm_rope, optionally fused with the KV store) vs the
oracle with the reference's rounding points (layernorm.rs:18-25,
rotary_embedding.rs:11-70).

The kernel and the oracle round at the same points, so outputs agree bit for
bit except where an f32 intermediate (cos/sin, the mean of squares) differs in
its last place between CUDA and numpy and lands on the other side of a
bf16/f16 rounding boundary: such elements must stay within one output ulp and
be rare.  V rows and the fused cache writes are pure copies: bit-exact.
"""
import numpy as np
import pytest
import torch

import nvkv
import nvkv_oracle as O
from helpers import bits, f32

pytestmark = pytest.mark.gpu


def _ulp_close(got: np.ndarray, want: np.ndarray, dtype: str, max_frac=1e-3):
    """Bit-identical except rare last-place flips: <= 0.1 % of elements may
    differ, each by at most ~2 output ulps of max(1, |value|) (a one-ulp cos/sin
    flip can cost that much after the rotation's subtraction), and the mean
    absolute difference stays inside the attention parity bound."""
    ulp = 2.0 ** -7 if dtype == "bf16" else 2.0 ** -10
    d = np.abs(got - want)
    tol = 2.0 * ulp * np.maximum(1.0, np.maximum(np.abs(got), np.abs(want)))
    assert (d <= tol).all(), f"max diff {d.max()} beyond two ulps"
    frac = np.mean(d > 0)
    assert frac <= max_frac, f"{frac:.2e} of elements differ"
    assert d.mean() <= 2e-3


@pytest.mark.parametrize("dtype,hq,hkv", [(torch.bfloat16, 32, 8), (torch.bfloat16, 16, 8),
                                          (torch.float16, 4, 1), (torch.bfloat16, 64, 8)])
def test_qknorm_rope_matches_oracle(dtype, hq, hkv):
    name = "bf16" if dtype == torch.bfloat16 else "f16"
    g = torch.Generator().manual_seed(hq)
    T, d = 300, 128
    qkv = (2.0 * torch.randn(T, (hq + 2 * hkv) * d, generator=g)).to(dtype)
    pos = torch.randint(0, 40960, (T,), generator=g)
    pos[:4] = torch.tensor([0, 1, 40959, 1024])
    qw = (1.0 + 0.2 * torch.randn(d, generator=g)).to(dtype)
    kw = (1.0 + 0.2 * torch.randn(d, generator=g)).to(dtype)
    q, k, v = nvkv.qknorm_rope(qkv.cuda(), pos.cuda(), hq, hkv, qw.cuda(), kw.cuda(), 1e-6, 1e6,
                               40960, want_kv=True)
    torch.cuda.synchronize()
    rq, rk, rv = O.qknorm_rope(f32(qkv), pos.numpy(), hq, hkv, d, f32(qw), f32(kw), 1e-6, 1e6, name)
    _ulp_close(f32(q), rq, name)
    _ulp_close(f32(k), rk, name)
    assert np.array_equal(f32(v), rv)
    assert nvkv.device_error() == 0


def test_rope_only_without_norm_weights():
    g = torch.Generator().manual_seed(7)
    T, hq, hkv, d = 33, 8, 2, 128
    qkv = torch.randn(T, (hq + 2 * hkv) * d, generator=g).to(torch.bfloat16)
    pos = torch.arange(T) * 97
    q, k, _ = nvkv.qknorm_rope(qkv.cuda(), pos.cuda(), hq, hkv, None, None, 1e-6, 1e6, 40960,
                               want_kv=True)
    torch.cuda.synchronize()
    rq, rk, _ = O.qknorm_rope(f32(qkv), pos.numpy(), hq, hkv, d, None, None, 1e-6, 1e6, "bf16")
    _ulp_close(f32(q), rq, "bf16")
    _ulp_close(f32(k), rk, "bf16")


def test_fused_store_equals_separate_store():
    """Prologue writing the cache == prologue then nvkv_store_kvcache (bit-exact)."""
    g = torch.Generator().manual_seed(11)
    T, hq, hkv, d, nb, page = 72, 16, 8, 128, 8, 256
    qkv = torch.randn(T, (hq + 2 * hkv) * d, generator=g).to(torch.bfloat16).cuda()
    pos = torch.randint(0, 4096, (T,), generator=g).cuda()
    w = torch.ones(d, dtype=torch.bfloat16, device="cuda")
    slots = torch.tensor(np.random.default_rng(1).choice(nb * page, T, replace=False)).cuda()
    slots[::9] = -1
    kc1 = torch.zeros(nb, page, hkv, d, dtype=torch.bfloat16, device="cuda")
    vc1, kc2, vc2 = kc1.clone(), kc1.clone(), kc1.clone()
    q1, k1, v1 = nvkv.qknorm_rope(qkv, pos, hq, hkv, w, w, 1e-6, 1e6, 40960, want_kv=True,
                                  k_cache=kc1, v_cache=vc1, slot_mapping=slots)
    q2, k2, v2 = nvkv.qknorm_rope(qkv, pos, hq, hkv, w, w, 1e-6, 1e6, 40960, want_kv=True)
    nvkv.store_kvcache(k2, v2, kc2, vc2, slots)
    torch.cuda.synchronize()
    assert np.array_equal(bits(q1), bits(q2))
    assert np.array_equal(bits(kc1), bits(kc2))
    assert np.array_equal(bits(vc1), bits(vc2))
    assert np.array_equal(bits(v1), bits(qkv[:, (hq + hkv) * d:].reshape(T, hkv, d)))


def test_position_out_of_range_reported():
    qkv = torch.zeros(2, (4 + 2) * 128, dtype=torch.bfloat16, device="cuda")
    nvkv.device_error()
    nvkv.qknorm_rope(qkv, torch.tensor([0, 50000], device="cuda"), 4, 1, None, None, 1e-6, 1e6,
                     40960)
    torch.cuda.synchronize()
    assert nvkv.device_error() == nvkv._lib.DEVERR_POSITION_RANGE
