"""Kernel 1 (nvkv_store_kvcache) vs the oracle scatter: bit-exact."""
import numpy as np
import pytest
import torch

import nvkv
import nvkv_oracle as O
from helpers import bits

pytestmark = pytest.mark.gpu


def _run_case(T, hkv, nb, page, slots, dtype=torch.bfloat16, strided=False, seed=0):
    g = torch.Generator().manual_seed(seed)
    d = 128
    if strided:  # K and V as slices of a fused qkv buffer (models/qwen3.rs:33-38)
        hq = 2 * hkv
        qkv = torch.randn(T, (hq + 2 * hkv) * d, generator=g).to(dtype).cuda()
        key = qkv[:, hq * d:(hq + hkv) * d].view(T, hkv, d)
        value = qkv[:, (hq + hkv) * d:].view(T, hkv, d)
    else:
        key = torch.randn(T, hkv, d, generator=g).to(dtype).cuda()
        value = torch.randn(T, hkv, d, generator=g).to(dtype).cuda()
    poison = torch.randint(-30000, 30000, (nb, page, hkv, d), generator=g, dtype=torch.int16)
    kc = poison.clone().cuda().view(dtype)
    vc = (poison.clone() ^ 0x1234).cuda().view(dtype)
    kc_ref = bits(kc).copy()
    vc_ref = bits(vc).copy()
    sm = torch.tensor(slots, dtype=torch.int64)
    nvkv.store_kvcache(key, value, kc, vc, sm.cuda())
    torch.cuda.synchronize()
    O.store_kvcache(bits(key), bits(value), kc_ref, vc_ref, sm.numpy())
    assert np.array_equal(bits(kc), kc_ref)
    assert np.array_equal(bits(vc), vc_ref)
    assert nvkv.device_error() == 0


def test_store_config2_slots_with_padding():
    """64 new tokens + 8 padded (-1) slots into a 2048-block pool (config 2)."""
    rng = np.random.default_rng(3)
    nb, page, hkv = 64, 256, 8
    slots = rng.choice(nb * page, 64, replace=False).tolist() + [-1] * 8
    rng.shuffle(slots)
    _run_case(72, hkv, nb, page, slots)


@pytest.mark.parametrize("hkv", [1, 2, 8])
def test_store_strided_qkv_slices(hkv):
    rng = np.random.default_rng(hkv)
    nb, page = 8, 256
    slots = rng.choice(nb * page, 37, replace=False).tolist()
    _run_case(37, hkv, nb, page, slots, strided=True, seed=hkv)


def test_store_f16_and_single_token():
    _run_case(1, 8, 4, 256, [700], dtype=torch.float16)


def test_store_all_padded_and_empty():
    _run_case(5, 8, 2, 256, [-1] * 5)
    k = torch.empty(0, 8, 128, dtype=torch.bfloat16, device="cuda")
    c = torch.zeros(1, 256, 8, 128, dtype=torch.bfloat16, device="cuda")
    nvkv.store_kvcache(k, k, c, c.clone(), torch.empty(0, dtype=torch.int64, device="cuda"))


def test_store_prefill_sized():
    """T = 16384 (a full max_num_batched_tokens step) into contiguous pages."""
    T, page, hkv = 16384, 256, 8
    nb = T // page + 4
    perm = np.random.default_rng(5).permutation(nb)[: T // page]
    slots = (perm[:, None] * page + np.arange(page)[None, :]).reshape(-1).tolist()
    _run_case(T, hkv, nb, page, slots, seed=5)


def test_store_out_of_range_slot_is_reported_not_written():
    nb, page, hkv, d = 2, 256, 8, 128
    key = torch.ones(3, hkv, d, dtype=torch.bfloat16, device="cuda")
    big = torch.zeros(nb + 1, page, hkv, d, dtype=torch.bfloat16, device="cuda")
    kc = big[:nb]  # the last page is a canary region just past the cache
    vc = torch.zeros(nb, page, hkv, d, dtype=torch.bfloat16, device="cuda")
    nvkv.device_error()  # clear
    nvkv.store_kvcache(key, key, kc, vc, torch.tensor([0, nb * page, 5], device="cuda"))
    torch.cuda.synchronize()
    assert nvkv.device_error() == nvkv._lib.DEVERR_SLOT_RANGE
    assert big[nb].abs().sum().item() == 0
    assert kc.view(-1, hkv * d)[0].float().sum().item() == hkv * d
    assert kc.view(-1, hkv * d)[5].float().sum().item() == hkv * d


def test_store_shape_errors():
    k = torch.zeros(2, 8, 128, dtype=torch.bfloat16, device="cuda")
    c = torch.zeros(1, 256, 4, 128, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(nvkv.NvkvError, match="width"):
        nvkv.store_kvcache(k, k, c, c, torch.zeros(2, dtype=torch.int64, device="cuda"))
    with pytest.raises(nvkv.NvkvError):
        nvkv.store_kvcache(k.float(), k.float(), c.float(), c.float(),
                           torch.zeros(2, dtype=torch.int64, device="cuda"))
