"""Shared helpers for the GPU parity tests (torch <-> oracle numpy)."""
import numpy as np
import torch

import nvkv_oracle as O

# attention tolerances from the parity gate (bf16 kernel vs fp32/fp64 oracle)
ATT_MAX_ABS = 2e-2
ATT_MEAN_ABS = 2e-3


def f32(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def assert_attention_close(got: torch.Tensor, want: np.ndarray, what: str = "") -> None:
    g = f32(got)
    assert np.isfinite(g).all(), f"{what}: non-finite output"
    d = np.abs(g - want)
    assert d.max() <= ATT_MAX_ABS, f"{what}: max-abs {d.max():.3e} > {ATT_MAX_ABS}"
    assert d.mean() <= ATT_MEAN_ABS, f"{what}: mean-abs {d.mean():.3e} > {ATT_MEAN_ABS}"


def make_paged(lens_k, page, hkv, d, num_blocks, gen, dtype=torch.bfloat16, dev="cuda"):
    """Random caches + a block table drawn from a seeded permutation of the pool.
    Returns (k_cache, v_cache, block_tables[u32 B x max_blocks], per-seq block lists)."""
    need = [(L + page - 1) // page for L in lens_k]
    assert sum(need) <= num_blocks
    perm = torch.randperm(num_blocks, generator=gen).tolist()
    tables, used = [], 0
    for n in need:
        tables.append(perm[used:used + n])
        used += n
    width = max(1, max(need))
    bt = np.zeros((len(lens_k), width), np.uint32)
    for i, t in enumerate(tables):
        bt[i, :len(t)] = t
    kc = torch.randn(num_blocks, page, hkv, d, generator=gen).to(dtype).to(dev)
    vc = torch.randn(num_blocks, page, hkv, d, generator=gen).to(dtype).to(dev)
    return kc, vc, bt, tables


def gather_seq(kc: torch.Tensor, vc: torch.Tensor, table, L: int):
    """One sequence's K/V rows, copied to the host and gathered by the oracle
    (layers/attention.rs:143-164) from a compact copy of its own pages."""
    page = kc.size(1)
    idx = torch.tensor(table, dtype=torch.long, device=kc.device)
    kcomp = f32(kc.index_select(0, idx))
    vcomp = f32(vc.index_select(0, idx))
    return O.gather_paged_kv(kcomp, vcomp, np.arange(len(table)), L, page)


def cu(lens, dev="cuda") -> torch.Tensor:
    return torch.tensor(np.cumsum([0] + list(lens)), dtype=torch.int32, device=dev)
