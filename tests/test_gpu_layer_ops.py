"""Fused epilogues around the path vs the oracle: nvkv_rms_norm (plain and
residual forms, layernorm.rs:18-42) and nvkv_silu_and_mul (activation.rs:5-17).

Both round at the reference's points.  The f32 intermediates can differ in the
last place (sum order of the mean of squares; CUDA's vs numpy's exp in SiLU),
which flips a rounded output by one ulp on rare elements: <= 1e-3 of elements
may differ, each by at most one output ulp of max(1, |value|); the residual
output (a rounded f32 sum) is bit-exact."""
import numpy as np
import pytest
import torch

import nvkv
import nvkv_oracle as O
from helpers import bits, f32

pytestmark = pytest.mark.gpu


def _one_ulp_close(got, want, dtype="bf16", frac=1e-3):
    ulp = 2.0 ** -7 if dtype == "bf16" else 2.0 ** -10
    d = np.abs(got - want)
    assert (d <= ulp * np.maximum(1.0, np.abs(want))).all(), d.max()
    assert np.mean(d > 0) <= frac, np.mean(d > 0)


@pytest.mark.parametrize("H", [1024, 4096, 5120])
def test_rms_norm_plain_and_residual(H):
    g = torch.Generator().manual_seed(H)
    T = 257
    x = (3 * torch.randn(T, H, generator=g)).bfloat16()
    r = torch.randn(T, H, generator=g).bfloat16()
    w = (1 + 0.1 * torch.randn(H, generator=g)).bfloat16()
    xc, rc, wc = x.cuda(), r.clone().cuda(), w.cuda()
    y_plain = nvkv.ops.rms_norm(xc, wc, 1e-6)
    y_res = nvkv.ops.rms_norm(xc, wc, 1e-6, residual=rc)
    torch.cuda.synchronize()
    _one_ulp_close(f32(y_plain), O.rms_norm(f32(x), f32(w), 1e-6, "bf16"))
    want, want_res = O.residual_rms_norm(f32(x), f32(r), f32(w), 1e-6, "bf16")
    _one_ulp_close(f32(y_res), want)
    assert np.array_equal(f32(rc), want_res)


def test_rms_norm_f16_strided_rows():
    g = torch.Generator().manual_seed(1)
    T, H = 64, 2048
    big = torch.randn(T, H + 64, generator=g).half().cuda()
    x = big[:, :H]
    w = torch.ones(H, dtype=torch.float16, device="cuda")
    out = torch.empty(T, H, dtype=torch.float16, device="cuda")
    nvkv.ops.rms_norm(x, w, 1e-6, out=out)
    torch.cuda.synchronize()
    _one_ulp_close(f32(out), O.rms_norm(f32(x), f32(w), 1e-6, "f16"), "f16")


@pytest.mark.parametrize("F", [3072, 12288])
def test_silu_and_mul(F):
    g = torch.Generator().manual_seed(F)
    gu = (2 * torch.randn(300, 2 * F, generator=g)).bfloat16()
    y = nvkv.ops.silu_and_mul(gu.cuda())
    torch.cuda.synchronize()
    _one_ulp_close(f32(y), O.silu_and_mul(f32(gu), "bf16"))


def test_layer_ops_validation():
    x = torch.zeros(4, 100, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(nvkv.NvkvError, match="multiple of 8"):
        nvkv.ops.rms_norm(x, torch.ones(100, dtype=torch.bfloat16, device="cuda"), 1e-6)
