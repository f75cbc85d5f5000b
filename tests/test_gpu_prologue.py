"""Kernel 4 (nvkv_qknorm_rope, optionally fused with the KV store) vs the
oracle with the reference's rounding points (layernorm.rs:18-25,
rotary_embedding.rs:11-70).

The kernel and the oracle round at the same points.  They can differ only
where an f32 intermediate differs in its last place between CUDA's and
numpy's math library (exp/cos/sin for the rotary table; the order of the
mean-of-squares sum) -- the reference builds its table with CUDA's functions
on the GPU, as the kernel does.  The tests bound exactly that: the norm is
checked bit-exact at position 0 (RoPE = identity), the rotation against the
analytic effect of one f32 ulp (see _rope_close).  V rows and the fused cache
writes are pure copies: bit-exact.
"""
import numpy as np
import pytest
import torch

import nvkv
import nvkv_oracle as O
from helpers import bits, f32

pytestmark = pytest.mark.gpu


def _ulp(dtype: str) -> float:
    return 2.0 ** -7 if dtype == "bf16" else 2.0 ** -10


def _rope_close(got, want, x_normed, pos, dtype, head_dim=128, theta=1e6):
    """Per-element bound for the rotation.  Kernel and oracle round at the
    same points; they differ only where the f32 transcendental (exp, cos, sin)
    results of CUDA and numpy differ by an ulp.  A one-ulp change of inv_freq
    moves freq = pos * inv_freq by up to freq * 2^-23, and a cos/sin value can
    then round to the neighbouring dtype value, so element i of the rotated
    pair (x1, x2) may differ by (|x1| + |x2|) * (ulp + 4 * freq_i * 2^-23) plus
    one output ulp.  At most 5 % (bf16) / 20 % (f16) of elements may differ at
    all (numpy's f32 exp/cos already differ from correctly rounded ones on
    ~1.4 % of bf16 outputs; f16 keeps 3 more bits, so ~8x as many flip) and the mean
    absolute difference stays inside the parity bound (2e-3)."""
    half = head_dim // 2
    freq = pos.astype(np.float64)[:, None] * O.rope_inv_freq(head_dim, theta)[None, :]
    freq = np.concatenate([freq, freq], -1)[:, None, :]
    x1, x2 = np.abs(x_normed[..., :half]), np.abs(x_normed[..., half:])
    mag = np.concatenate([x1 + x2, x1 + x2], -1)
    u = _ulp(dtype)
    tol = mag * (u + 4 * freq * 2.0 ** -23) + u * np.maximum(1.0, np.abs(want)) + 1e-12
    d = np.abs(got - want)
    assert (d <= tol).all(), f"{(d > tol).sum()} elements beyond the bound, worst {d.max()}"
    cap = 5e-2 if dtype == "bf16" else 2e-1  # f16 keeps 3 more bits: ~8x the flips
    assert np.mean(d > 0) <= cap, f"{np.mean(d > 0):.2e} of elements differ"
    assert d.mean() <= 2e-3


def test_norm_exact_at_position_zero():
    """pos = 0 makes RoPE the identity (cos 1, sin 0 in any library), so the
    output is the reference's rms_norm: bit-exact except f32 sum-order flips
    (<= 1e-4 of elements, one ulp each)."""
    g = torch.Generator().manual_seed(5)
    T, hq, hkv, d = 256, 32, 8, 128
    qkv = (2.0 * torch.randn(T, (hq + 2 * hkv) * d, generator=g)).to(torch.bfloat16)
    w = (1.0 + 0.2 * torch.randn(d, generator=g)).to(torch.bfloat16)
    pos = torch.zeros(T, dtype=torch.int64)
    q, k, _ = nvkv.qknorm_rope(qkv.cuda(), pos.cuda(), hq, hkv, w.cuda(), w.cuda(), 1e-6, 1e6,
                               40960, want_kv=True)
    torch.cuda.synchronize()
    x = f32(qkv)
    rq = O.rms_norm(x[:, :hq * d].reshape(T, hq, d), f32(w), 1e-6, "bf16")
    rk = O.rms_norm(x[:, hq * d:(hq + hkv) * d].reshape(T, hkv, d), f32(w), 1e-6, "bf16")
    for got, want in ((f32(q), rq), (f32(k), rk)):
        dd = np.abs(got - want)
        assert np.mean(dd > 0) <= 1e-4
        assert (dd <= _ulp("bf16") * np.maximum(1.0, np.abs(want))).all()


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
    x = f32(qkv)
    nq = O.rms_norm(x[:, :hq * d].reshape(T, hq, d), f32(qw), 1e-6, name)
    nk = O.rms_norm(x[:, hq * d:(hq + hkv) * d].reshape(T, hkv, d), f32(kw), 1e-6, name)
    _rope_close(f32(q), rq, nq, pos.numpy(), name)
    _rope_close(f32(k), rk, nk, pos.numpy(), name)
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
    x = f32(qkv)
    _rope_close(f32(q), rq, x[:, :hq * d].reshape(T, hq, d), pos.numpy(), "bf16")
    _rope_close(f32(k), rk, x[:, hq * d:(hq + hkv) * d].reshape(T, hkv, d), pos.numpy(), "bf16")


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
