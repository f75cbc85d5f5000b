"""Python mirror of the reference's operator surface for this path.

Same names and argument meaning as nanovllm_rs:
  * ``set_context`` / ``get_context`` / ``reset_context``  (utils/context.rs)
  * ``store_kv_cache(key, value, k_cache, v_cache, slot_mapping)``
    (layers/kv_cache.rs:168-190)
  * ``Attention(scale)`` with ``set_kv_cache`` and ``forward(q, k, v)``
    (layers/attention.rs:7-76)
The context and the attention object live in the C++ host layer of
libnvkv.so (thread-local there, as in the reference); this module only keeps
the Python tensors alive while the library holds their device pointers.
Errors surface as ``NvkvError`` (the reference's ``candle_core::Result``).
"""
from __future__ import annotations

import ctypes
import threading
from dataclasses import dataclass
from typing import Optional

import torch

from ._lib import NvkvError, ERR_INVALID_ARG, check, lib
from . import ops

_tls = threading.local()


@dataclass
class Context:
    """utils/context.rs:4-13."""

    cu_seqlens_q: Optional[torch.Tensor] = None
    cu_seqlens_k: Optional[torch.Tensor] = None
    max_seqlen_q: int = 0
    max_seqlen_k: int = 0
    slot_mapping: Optional[torch.Tensor] = None
    context_lens: Optional[torch.Tensor] = None
    block_tables: Optional[torch.Tensor] = None
    seq_need_compute_logits: Optional[torch.Tensor] = None


def _p(t: Optional[torch.Tensor]):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def set_context(cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k, slot_mapping=None,
                context_lens=None, block_tables=None, seq_need_compute_logits=None) -> None:
    """utils/context.rs:28-50 (thread-local)."""
    ctx = Context(cu_seqlens_q, cu_seqlens_k, int(max_seqlen_q), int(max_seqlen_k), slot_mapping,
                  context_lens, block_tables, seq_need_compute_logits)
    if block_tables is not None and not block_tables.is_contiguous():
        raise NvkvError(ERR_INVALID_ARG, "block_tables must be contiguous")
    check(lib.nvkv_context_set(
        _p(cu_seqlens_q), _p(cu_seqlens_k), cu_seqlens_q.numel() - 1, ctx.max_seqlen_q,
        ctx.max_seqlen_k, _p(slot_mapping), 0 if slot_mapping is None else slot_mapping.numel(),
        _p(context_lens), _p(block_tables), 0 if block_tables is None else block_tables.size(1)))
    _tls.ctx = ctx


def get_context() -> Context:
    """utils/context.rs:23-25."""
    return getattr(_tls, "ctx", Context())


def reset_context() -> None:
    """utils/context.rs:52-54."""
    check(lib.nvkv_context_reset())
    _tls.ctx = Context()


def store_kv_cache(key, value, k_cache, v_cache, slot_mapping) -> None:
    """layers/kv_cache.rs:168-190 (no contiguous copy needed: rows are read
    through their token stride)."""
    ops.store_kvcache(key, value, k_cache, v_cache, slot_mapping)


class Attention:
    """layers/attention.rs:7-76 backed by nvkv_attention_* in libnvkv.so."""

    def __init__(self, scale: float):
        h = ctypes.c_void_p()
        check(lib.nvkv_attention_create(ctypes.c_float(scale), ctypes.byref(h)))
        self._h = h
        self.scale = scale
        self.k_cache: Optional[torch.Tensor] = None
        self.v_cache: Optional[torch.Tensor] = None

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            lib.nvkv_attention_destroy(h)
            self._h = None

    def set_kv_cache(self, k_cache: torch.Tensor, v_cache: torch.Tensor) -> None:
        if not (k_cache.is_contiguous() and v_cache.is_contiguous() and k_cache.dim() == 4):
            raise NvkvError(ERR_INVALID_ARG, "kv caches must be contiguous [Nb, P, Hkv, D]")
        nb, page, hkv, d = k_cache.shape
        check(lib.nvkv_attention_set_kv_cache(self._h, _p(k_cache), _p(v_cache), nb, page, hkv, d,
                                              ops._dtype(k_cache)))
        self.k_cache, self.v_cache = k_cache, v_cache

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """q: [T, Hq, D], k/v: [T, Hkv, D] (token dim may be strided)."""
        ctx = get_context()
        if ctx.cu_seqlens_q is None:
            raise NvkvError(ERR_INVALID_ARG, "cu_seqlens_q must be set")  # attention.rs:26
        T, hq, d = q.shape
        hkv = k.size(1)
        if out is None:
            out = torch.empty(T, hq, d, device=q.device, dtype=q.dtype)
        for t in (q, k, v):
            if not ops._row_view_ok(t):
                raise NvkvError(ERR_INVALID_ARG, "q/k/v rows must be dense")
        check(lib.nvkv_attention_forward(
            self._h, _p(q), q.stride(0) if T > 1 else hq * d, _p(k),
            k.stride(0) if T > 1 else hkv * d, _p(v), v.stride(0) if T > 1 else hkv * d, T, hq, hkv,
            _p(out), ops._dtype(q), ops._stream()))
        return out

    __call__ = forward
