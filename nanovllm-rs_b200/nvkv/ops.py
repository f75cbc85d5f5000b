"""Kernel-level calls on torch tensors, one per C-ABI entry point.

Each function checks shapes, dtypes and devices the way the reference's
candle ops do (layers/kv_cache.rs:111-124) and then calls straight into
libnvkv.so on the current CUDA stream.  Nothing here computes on the host.
"""
from __future__ import annotations

import ctypes
from typing import Optional, Tuple

import torch

from ._lib import DTYPE_BF16, DTYPE_F16, DTYPE_F32, NvkvError, ERR_INVALID_ARG, check, lib

_DT = {torch.bfloat16: DTYPE_BF16, torch.float16: DTYPE_F16}


def _dtype(t: torch.Tensor) -> int:
    try:
        return _DT[t.dtype]
    except KeyError:
        raise NvkvError(-2, f"unsupported dtype {t.dtype} (bf16/f16 only)") from None


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream() -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _need(cond: bool, msg: str) -> None:
    if not cond:
        raise NvkvError(ERR_INVALID_ARG, msg)


def _row_view_ok(t: torch.Tensor) -> bool:
    """dims after the first are dense (the token dim may be strided)."""
    exp = 1
    for d in range(t.dim() - 1, 0, -1):
        if t.size(d) != 1 and t.stride(d) != exp:
            return False
        exp *= t.size(d)
    return True


def store_kvcache(key: torch.Tensor, value: torch.Tensor, k_cache: torch.Tensor,
                  v_cache: torch.Tensor, slot_mapping: torch.Tensor) -> None:
    """store_kv_cache (layers/kv_cache.rs:168-190) through nvkv_store_kvcache."""
    _need(key.is_cuda and k_cache.is_cuda, "store_kvcache is cuda-only")  # kv_cache.rs:90-100
    _need(key.dtype == value.dtype == k_cache.dtype == v_cache.dtype, "dtype mismatch")
    _need(k_cache.is_contiguous() and v_cache.is_contiguous(),
          "store_kvcache requires contiguous caches")
    _need(slot_mapping.dtype == torch.int64 and slot_mapping.is_contiguous(),
          "slot_mapping must be contiguous int64")
    T = key.size(0)
    d = 1
    for s in key.shape[1:]:
        d *= s
    width = 1
    for s in k_cache.shape[2:]:
        width *= s
    _need(width == d, f"store_kvcache: cache per-slot width {tuple(k_cache.shape[2:])} "
                      f"does not match src width {d}")
    _need(value.shape == key.shape and slot_mapping.numel() == T, "shape mismatch")
    _need(_row_view_ok(key) and _row_view_ok(value), "key/value rows must be dense")
    num_slots = k_cache.size(0) * k_cache.size(1)
    check(lib.nvkv_store_kvcache(_ptr(key), _ptr(value), _ptr(k_cache), _ptr(v_cache),
                                 _ptr(slot_mapping), T, d, key.stride(0) if T > 1 else d,
                                 value.stride(0) if T > 1 else d, num_slots, _dtype(key),
                                 _stream()))


def qknorm_rope(qkv: torch.Tensor, positions: torch.Tensor, num_q_heads: int,
                num_kv_heads: int, q_norm_w: Optional[torch.Tensor],
                k_norm_w: Optional[torch.Tensor], eps: float, rope_theta: float,
                max_position: int, head_dim: int = 128,
                k_cache: Optional[torch.Tensor] = None, v_cache: Optional[torch.Tensor] = None,
                slot_mapping: Optional[torch.Tensor] = None, want_kv: bool = False,
                q_out: Optional[torch.Tensor] = None
                ) -> Tuple[torch.Tensor, Optional[torch.Tensor], Optional[torch.Tensor]]:
    """Fused split_qkv + q/k RMSNorm + RoPE (+ KV store) of models/qwen3.rs:128-141."""
    _need(qkv.is_cuda and qkv.dim() == 2 and qkv.stride(1) == 1, "qkv must be [T, W] on cuda")
    _need(positions.dtype == torch.int64 and positions.is_contiguous(), "positions: int64")
    T = qkv.size(0)
    _need(qkv.size(1) >= (num_q_heads + 2 * num_kv_heads) * head_dim, "qkv too narrow")
    dev, dt = qkv.device, qkv.dtype
    if q_out is None:
        q_out = torch.empty(T, num_q_heads, head_dim, device=dev, dtype=dt)
    k_out = torch.empty(T, num_kv_heads, head_dim, device=dev, dtype=dt) if want_kv else None
    v_out = torch.empty(T, num_kv_heads, head_dim, device=dev, dtype=dt) if want_kv else None
    num_slots = 0
    if k_cache is not None:
        _need(k_cache.is_contiguous() and v_cache is not None and v_cache.is_contiguous(),
              "caches must be contiguous")
        _need(slot_mapping is not None and slot_mapping.dtype == torch.int64, "slot_mapping")
        num_slots = k_cache.size(0) * k_cache.size(1)
    for w in (q_norm_w, k_norm_w):
        _need(w is None or (w.dtype == dt and w.is_contiguous()), "norm weights: same dtype")
    check(lib.nvkv_qknorm_rope(_ptr(qkv), qkv.stride(0), T, num_q_heads, num_kv_heads, head_dim,
                               _ptr(positions), _ptr(q_norm_w), _ptr(k_norm_w), float(eps),
                               float(rope_theta), int(max_position), _ptr(q_out), _ptr(k_out),
                               _ptr(v_out), _ptr(k_cache), _ptr(v_cache), _ptr(slot_mapping),
                               num_slots, _dtype(qkv), _stream()))
    return q_out, k_out, v_out


def workspace_size(num_seqs: int, num_q_heads: int, num_kv_heads: int, max_seqlen_q: int,
                   max_seqlen_k: int, head_dim: int = 128) -> int:
    n = ctypes.c_size_t(0)
    check(lib.nvkv_paged_attention_workspace_size(num_seqs, num_q_heads, num_kv_heads, head_dim,
                                                  max_seqlen_q, max_seqlen_k, ctypes.byref(n)))
    return n.value


def paged_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                    cu_seqlens_q: torch.Tensor, cu_seqlens_k: torch.Tensor,
                    block_tables: Optional[torch.Tensor], max_seqlen_q: int, max_seqlen_k: int,
                    softmax_scale: float, causal: bool = True,
                    out: Optional[torch.Tensor] = None,
                    workspace: Optional[torch.Tensor] = None) -> torch.Tensor:
    """flash_attn_varlen[_paged_windowed] replacement (layers/attention.rs:37-75).

    q: [T, Hq, D]; paged caches [Nb, P, Hkv, D] when block_tables is given,
    else contiguous-row K/V [Tk, Hkv, D] (token dim may be strided)."""
    _need(q.is_cuda and q.dim() == 3 and _row_view_ok(q), "q must be [T, Hq, D] on cuda")
    T, hq, d = q.shape
    if block_tables is not None:
        _need(k_cache.dim() == 4 and k_cache.is_contiguous() and v_cache.is_contiguous(),
              "paged caches must be contiguous [Nb, P, Hkv, D]")
        nb, page, hkv = k_cache.size(0), k_cache.size(1), k_cache.size(2)
        kv_stride = 0
        _need(block_tables.dtype in (torch.int32, torch.uint32) and block_tables.is_contiguous(),
              "block_tables must be contiguous 32-bit")
        bt_stride = block_tables.size(1)
    else:
        _need(k_cache.dim() == 3 and _row_view_ok(k_cache) and _row_view_ok(v_cache),
              "contiguous K/V must be [Tk, Hkv, D]")
        _need(k_cache.stride(0) == v_cache.stride(0), "k/v token strides differ")
        nb, page, hkv = k_cache.size(0), 0, k_cache.size(1)
        kv_stride = k_cache.stride(0)
        bt_stride = 0
    for t in (cu_seqlens_q, cu_seqlens_k):
        _need(t.dtype in (torch.int32, torch.uint32) and t.is_contiguous(), "cu_seqlens: u32")
    B = cu_seqlens_q.numel() - 1
    if out is None:
        out = torch.empty(T, hq, d, device=q.device, dtype=q.dtype)
    need = workspace_size(B, hq, hkv, max_seqlen_q, max_seqlen_k, d)
    if need and (workspace is None or workspace.numel() * workspace.element_size() < need):
        workspace = torch.empty(need, device=q.device, dtype=torch.uint8)
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    check(lib.nvkv_paged_attention(
        _ptr(q), q.stride(0) if T > 1 else hq * d, T, _ptr(k_cache), _ptr(v_cache), nb, kv_stride,
        _ptr(out), _ptr(cu_seqlens_q), _ptr(cu_seqlens_k), _ptr(block_tables), bt_stride, B,
        int(max_seqlen_q), int(max_seqlen_k), hq, hkv, d, page, float(softmax_scale),
        1 if causal else 0, _ptr(workspace), ws_bytes, _dtype(q), _stream()))
    return out


def store_kvcache_fp8(key: torch.Tensor, value: torch.Tensor, k_cache: torch.Tensor,
                      v_cache: torch.Tensor, k_scale: torch.Tensor, v_scale: torch.Tensor,
                      slot_mapping: torch.Tensor) -> None:
    """The fp8 (e4m3) pool's store (nvkv_store_kvcache_fp8): key/value
    [T, Hkv, 128] bf16/f16 rows quantised into k_cache/v_cache
    [Nb, P, Hkv, 128] uint8 with one f32 scale per row in k_scale/v_scale
    [Nb, Hkv, P]."""
    _need(key.is_cuda and k_cache.is_cuda, "store_kvcache_fp8 is cuda-only")
    _need(k_cache.dtype == torch.uint8 and v_cache.dtype == torch.uint8, "fp8 caches are uint8")
    _need(k_scale.dtype == torch.float32 and v_scale.dtype == torch.float32, "scales are f32")
    _need(k_cache.dim() == 4 and k_cache.is_contiguous() and v_cache.is_contiguous() and
          k_scale.is_contiguous() and v_scale.is_contiguous(), "contiguous pool")
    Nb, P, hkv, d = k_cache.shape
    _need(tuple(k_scale.shape) == (Nb, hkv, P) == tuple(v_scale.shape), "scales [Nb, Hkv, P]")
    _need(key.dim() == 3 and key.shape[1:] == (hkv, d) and value.shape == key.shape, "key shape")
    _need(slot_mapping.dtype == torch.int64 and slot_mapping.is_contiguous(), "slot_mapping")
    T = key.size(0)
    _need(_row_view_ok(key) and _row_view_ok(value), "key/value rows must be dense")
    check(lib.nvkv_store_kvcache_fp8(_ptr(key), _ptr(value), _ptr(k_cache), _ptr(v_cache),
                                     _ptr(k_scale), _ptr(v_scale), _ptr(slot_mapping), T, hkv, d,
                                     key.stride(0) if T > 1 else hkv * d,
                                     value.stride(0) if T > 1 else hkv * d, Nb, P, _dtype(key),
                                     _stream()))


def workspace_size_fp8(num_seqs: int, num_q_heads: int, num_kv_heads: int, max_seqlen_q: int,
                       max_seqlen_k: int, prompt_kv_tokens: int, head_dim: int = 128) -> int:
    n = ctypes.c_size_t(0)
    check(lib.nvkv_paged_attention_fp8_workspace_size(num_seqs, num_q_heads, num_kv_heads,
                                                      head_dim, max_seqlen_q, max_seqlen_k,
                                                      int(prompt_kv_tokens), ctypes.byref(n)))
    return n.value


def paged_attention_fp8(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                        k_scale: torch.Tensor, v_scale: torch.Tensor,
                        cu_seqlens_q: torch.Tensor, cu_seqlens_k: torch.Tensor,
                        block_tables: torch.Tensor, max_seqlen_q: int, max_seqlen_k: int,
                        softmax_scale: float, prompt_kv_tokens: int = 0, causal: bool = True,
                        out: Optional[torch.Tensor] = None,
                        workspace: Optional[torch.Tensor] = None) -> torch.Tensor:
    """paged_attention over the fp8 (e4m3) pool (nvkv_paged_attention_fp8).
    prompt_kv_tokens: at least the sum of k_len over the q_len > 1 sequences."""
    _need(q.is_cuda and q.dim() == 3 and _row_view_ok(q), "q must be [T, Hq, D] on cuda")
    _need(k_cache.dtype == torch.uint8 and k_cache.dim() == 4 and k_cache.is_contiguous() and
          v_cache.is_contiguous(), "fp8 caches: contiguous uint8 [Nb, P, Hkv, D]")
    _need(block_tables.dtype in (torch.int32, torch.uint32) and block_tables.is_contiguous(),
          "block_tables must be contiguous 32-bit")
    T, hq, d = q.shape
    nb, page, hkv = k_cache.size(0), k_cache.size(1), k_cache.size(2)
    B = cu_seqlens_q.numel() - 1
    if out is None:
        out = torch.empty(T, hq, d, device=q.device, dtype=q.dtype)
    need = workspace_size_fp8(B, hq, hkv, max_seqlen_q, max_seqlen_k, prompt_kv_tokens, d)
    if need and (workspace is None or workspace.numel() * workspace.element_size() < need):
        workspace = torch.empty(need, device=q.device, dtype=torch.uint8)
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    check(lib.nvkv_paged_attention_fp8(
        _ptr(q), q.stride(0) if T > 1 else hq * d, T, _ptr(k_cache), _ptr(v_cache),
        _ptr(k_scale), _ptr(v_scale), nb, _ptr(out), _ptr(cu_seqlens_q), _ptr(cu_seqlens_k),
        _ptr(block_tables), block_tables.size(1), B, int(max_seqlen_q), int(max_seqlen_k), hq, hkv,
        d, page, float(softmax_scale), 1 if causal else 0, int(prompt_kv_tokens),
        _ptr(workspace), ws_bytes, _dtype(q), _stream()))
    return out


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float,
             residual: Optional[torch.Tensor] = None,
             out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """RMSNorm::forward / residual_forward (layernorm.rs:18-42) in one launch.
    With `residual`, it is updated in place to dtype(x + residual) and the
    norm is taken of that sum (the reference returns it as the new residual)."""
    _need(x.is_cuda and x.dim() == 2 and x.stride(1) == 1, "x must be [T, H] on cuda")
    T, H = x.shape
    _need(weight.dtype == x.dtype and weight.is_contiguous() and weight.numel() == H, "weight")
    if residual is not None:
        _need(residual.shape == x.shape and residual.stride(1) == 1 and
              residual.dtype == x.dtype, "residual must match x")
    if out is None:
        out = torch.empty_like(x)
    check(lib.nvkv_rms_norm(_ptr(x), x.stride(0), _ptr(residual),
                            0 if residual is None else residual.stride(0), _ptr(weight),
                            float(eps), _ptr(out), out.stride(0), T, H, _dtype(x), _stream()))
    return out


def silu_and_mul(gate_up: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """SiluAndMul::forward (activation.rs:5-17): silu(gate) * up in one launch."""
    _need(gate_up.is_cuda and gate_up.dim() == 2 and gate_up.stride(1) == 1, "gate_up: [T, 2F]")
    T, W = gate_up.shape
    F = W // 2
    if out is None:
        out = torch.empty(T, F, device=gate_up.device, dtype=gate_up.dtype)
    check(lib.nvkv_silu_and_mul(_ptr(gate_up), gate_up.stride(0), _ptr(out), out.stride(0), T, F,
                                _dtype(gate_up), _stream()))
    return out


def sample(logits: torch.Tensor, temperatures: torch.Tensor, seed: int, step: int,
           vocab_offset: int = 0, out_value: Optional[torch.Tensor] = None,
           out_index: Optional[torch.Tensor] = None, step_device: Optional[torch.Tensor] = None):
    """The reference's Sampler::forward (layers/sampler.rs:7-21) in its
    Gumbel-max form, one launch: per row of `logits` [B, V] (bf16, f16 or
    f32; a vocab-parallel shard whose column 0 is global index
    `vocab_offset`), the score max_v logit / T - log(max(-log u, 1e-10)) and
    its global index, u from Philox4x32-10 keyed by `seed` at counter (global
    index / 4, row, step [+ step_device, an int64 [1] cuda tensor read by the
    kernel, so a graph replay can advance it]).  temperatures [B] f32 (<= 0:
    greedy).  Returns
    (value [B] f32, index [B] int64); over shards, the largest value (ties to
    the lowest index) is the row's token."""
    _need(logits.dim() == 2 and logits.is_cuda and logits.stride(1) == 1, "logits: [B, V] rows")
    B, V = logits.shape
    dt = DTYPE_F32 if logits.dtype == torch.float32 else _dtype(logits)
    _need(temperatures.dtype == torch.float32 and temperatures.numel() == B and
          temperatures.is_contiguous(), "temperatures: f32 [B]")
    if out_value is None:
        out_value = torch.empty(B, dtype=torch.float32, device=logits.device)
    if out_index is None:
        out_index = torch.empty(B, dtype=torch.int64, device=logits.device)
    if step_device is not None:
        _need(step_device.dtype == torch.int64 and step_device.is_cuda, "step_device: int64")
    check(lib.nvkv_sample(_ptr(logits), B, V, logits.stride(0), int(vocab_offset),
                          _ptr(temperatures), int(seed) & (2**64 - 1), int(step) & (2**64 - 1),
                          _ptr(step_device), _ptr(out_value), _ptr(out_index), dt, _stream()))
    return out_value, out_index


def decode_advance(seq_lens: torch.Tensor, block_tables: torch.Tensor, num_blocks: int,
                   page_size: int, positions: torch.Tensor, slot_mapping: torch.Tensor,
                   cu_seqlens_q: torch.Tensor, cu_seqlens_k: torch.Tensor) -> None:
    """Device-side metadata of a pure decode step (model_runner.rs:69-160,
    decode case): seq_lens [B] int64 is advanced by one in place and the
    step's positions / slot_mapping [B] int64 and cu_seqlens_q/k [B+1]
    int32 are written, without a host round trip."""
    B = seq_lens.numel()
    _need(seq_lens.dtype == torch.int64 and seq_lens.is_cuda and seq_lens.is_contiguous(),
          "seq_lens: int64 [B] on cuda")
    _need(block_tables.dim() == 2 and block_tables.size(0) == B and
          block_tables.dtype == torch.int32 and block_tables.stride(1) == 1, "block_tables")
    for t, n, dt in ((positions, B, torch.int64), (slot_mapping, B, torch.int64),
                     (cu_seqlens_q, B + 1, torch.int32), (cu_seqlens_k, B + 1, torch.int32)):
        _need(t.numel() == n and t.dtype == dt and t.is_contiguous(), "output buffer shape")
    check(lib.nvkv_decode_advance(B, page_size, _ptr(seq_lens), _ptr(block_tables),
                                  block_tables.stride(0), int(num_blocks), _ptr(positions),
                                  _ptr(slot_mapping), _ptr(cu_seqlens_q), _ptr(cu_seqlens_k),
                                  _stream()))
