"""CPU restatement of nanovllm_rs's per-layer attention hot path.

TEST INFRASTRUCTURE ONLY.  This module is the checker that the CUDA path is
compared against.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import it; the
product path (``nanovllm-rs_b200/``) never does, and fails loudly when its CUDA
library is missing instead of falling back to anything here.

Parity status: UNPINNED with respect to reference-produced numbers.  The
reference (Athe-kunal/nanovllm-rs) is Rust on candle 0.11 and cannot be built or
run in this container (no cargo/rustc, no vendored crates), and its only
known-answer probe (``nanovllm_rs/src/bin/repro.rs``) prints diffs without
asserting or recording values.  What pins this restatement instead:

* KAT-1: the ``repro.rs`` input generator restated bit-for-bit
  (``repro_inputs``); the store must reproduce ``k_full`` exactly
  (``cache_write_diff == 0``, repro.rs:116-121) and the paged attention must
  equal repro.rs's own ``manual_attention`` (repro.rs:6-32, restated separately
  in ``tests/golden/make_golden.py``).
* KAT-2: hand-computed slot mappings for ``prepare_model_input``
  (model_runner.rs:108-124) committed as literal arrays.

Third-party arithmetic the reference delegates to (not under the reference
tree; pinned in ``nanovllm_rs/Cargo.lock``): candle-flash-attn 0.11.0 (FA2
``flash_attn_varlen`` / ``flash_attn_varlen_paged_windowed``), candle-nn 0.11.0
(``flash_attn_varlen_unfused``), candle-core 0.11.0 (elementwise kernels),
half 2.7.1 (bf16 round-to-nearest-even).  Their published semantics are
restated here: exact softmax attention, causal mask aligned bottom-right
(key j visible to query i iff ``j <= i + k_len - q_len``), GQA head h reads kv
head ``h // (Hq // Hkv)``.

Every array is numpy.  bf16 values are carried as float32 arrays whose values
are bf16-representable; ``bf16_bits``/``from_bf16_bits`` convert to and from
the 16-bit storage pattern.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import List, Optional, Sequence as Seq_, Tuple

import numpy as np

# --------------------------------------------------------------------------
# dtype helpers
# --------------------------------------------------------------------------


def round_bf16(x) -> np.ndarray:
    """float32 -> nearest-even bf16 value, returned as float32.

    Follows half 2.7.1 ``bf16::from_f32`` (round to nearest, ties to even; NaN
    stays NaN), which candle uses for every ``to_dtype(BF16)``.
    """
    x = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
    u = x.view(np.uint32).astype(np.uint64)
    bias = ((u >> 16) & 1) + 0x7FFF
    r = (((u + bias) >> 16) << 16).astype(np.uint32).view(np.float32)
    return np.where(np.isnan(x), np.float32(np.nan), r).astype(np.float32)


def bf16_bits(x) -> np.ndarray:
    """bf16 storage bits (uint16) of float32 values (rounded RNE first)."""
    r = round_bf16(x)
    return (r.view(np.uint32) >> 16).astype(np.uint16)


def from_bf16_bits(b) -> np.ndarray:
    b = np.asarray(b, dtype=np.uint16)
    return (b.astype(np.uint32) << 16).view(np.float32)


def round_to(x, dtype: str) -> np.ndarray:
    """Round float32 values to the activation dtype ('bf16', 'f16' or 'f32')."""
    x = np.asarray(x, dtype=np.float32)
    if dtype == "bf16":
        return round_bf16(x)
    if dtype == "f16":
        return x.astype(np.float16).astype(np.float32)
    if dtype == "f32":
        return x
    raise ValueError(f"unsupported dtype {dtype}")


# --------------------------------------------------------------------------
# a1: KV-cache scatter
# --------------------------------------------------------------------------


def store_kvcache(key, value, k_cache, v_cache, slot_mapping) -> None:
    """In-place row scatter; nanovllm_rs/src/layers/kv_cache.rs:13-24, 168-190.

    ``key``/``value``: [T, Hkv, D] (or [T, d]).  Caches: [Nb, P, Hkv, D],
    viewed as [Nb*P, Hkv*D].  Row t goes to cache row ``slot_mapping[t]``;
    rows whose slot is negative are skipped (kv_cache.rs:19-20).  Works on any
    numpy dtype (uint16 bit patterns included), so it is bit-exact by
    construction.
    """
    T = key.shape[0]
    kc = k_cache.reshape(-1, int(np.prod(k_cache.shape[2:])))
    vc = v_cache.reshape(-1, int(np.prod(v_cache.shape[2:])))
    k2 = key.reshape(T, -1)
    v2 = value.reshape(T, -1)
    if k2.shape[1] != kc.shape[1] or v2.shape[1] != vc.shape[1]:
        raise ValueError("store_kvcache: cache per-slot width does not match src width")
    slots = np.asarray(slot_mapping, dtype=np.int64)
    valid = slots >= 0
    if np.any(slots[valid] >= kc.shape[0]):
        raise IndexError("store_kvcache: slot out of range")
    kc[slots[valid]] = k2[valid]
    vc[slots[valid]] = v2[valid]


# --------------------------------------------------------------------------
# a8: metadata (Sequence -> Context)
# --------------------------------------------------------------------------


@dataclass
class Seq:
    """The fields of ``Sequence`` (engine/sequence.rs:22-36) the runner reads."""

    token_ids: List[int]
    block_table: List[int] = field(default_factory=list)
    num_cached_tokens: int = 0
    num_new_tokens: int = 0
    block_size: int = 256

    def __len__(self) -> int:  # sequence.rs:66-68
        return len(self.token_ids)

    def num_context_tokens(self) -> int:  # sequence.rs:82-84
        return self.num_cached_tokens + self.num_new_tokens

    def num_cached_blocks(self) -> int:  # sequence.rs:99-101
        return self.num_cached_tokens // self.block_size


@dataclass
class Context:
    """utils/context.rs:4-13 (host copy of every field)."""

    cu_seqlens_q: np.ndarray
    cu_seqlens_k: np.ndarray
    max_seqlen_q: int
    max_seqlen_k: int
    slot_mapping: np.ndarray
    context_lens: np.ndarray
    block_tables: Optional[np.ndarray]
    seq_need_compute_logits: np.ndarray


def prepare_block_tables(seqs: Seq_[Seq]) -> np.ndarray:
    """engine/model_runner.rs:53-67: [B, max_blocks] uint32, padded with 0."""
    max_len = max(len(s.block_table) for s in seqs)
    bt = np.zeros((len(seqs), max_len), dtype=np.uint32)
    for i, s in enumerate(seqs):
        bt[i, : len(s.block_table)] = s.block_table
    return bt


def prepare_model_input(seqs: Seq_[Seq], block_size: int) -> Tuple[np.ndarray, np.ndarray, Context]:
    """engine/model_runner.rs:69-160.  Returns (input_ids, positions, context)."""
    input_ids: List[int] = []
    positions: List[int] = []
    cu_q = [0]
    cu_k = [0]
    max_q = 0
    max_k = 0
    slots: List[int] = []
    context_lens: List[int] = []
    need_logits: List[int] = []
    for idx, s in enumerate(seqs):
        n_ctx = s.num_context_tokens()
        if len(s) == n_ctx and s.block_table:  # :85-87
            need_logits.append(idx)
        context_lens.append(n_ctx)
        input_ids.extend(s.token_ids[s.num_cached_tokens:n_ctx])  # :89-93
        positions.extend(range(s.num_cached_tokens, n_ctx))  # :94
        cu_q.append(cu_q[-1] + s.num_new_tokens)  # :96-99
        cu_k.append(cu_k[-1] + n_ctx)
        max_q = max(max_q, s.num_new_tokens)
        max_k = max(max_k, n_ctx)
        if not s.block_table:  # warmup: no slots (:103-106)
            continue
        first = s.num_cached_blocks()
        last = len(s.block_table) - 1
        for i in range(first, len(s.block_table)):  # :108-124
            b = s.block_table[i]
            start = b * block_size + (s.num_cached_tokens % block_size if i == first else 0)
            if i == last and n_ctx % block_size != 0:
                end = b * block_size + n_ctx % block_size
            else:
                end = (b + 1) * block_size
            slots.extend(range(start, end))
    block_tables = prepare_block_tables(seqs) if cu_k[-1] > cu_q[-1] else None  # :127-131
    ctx = Context(
        cu_seqlens_q=np.asarray(cu_q, dtype=np.uint32),
        cu_seqlens_k=np.asarray(cu_k, dtype=np.uint32),
        max_seqlen_q=max_q,
        max_seqlen_k=max_k,
        slot_mapping=np.asarray(slots, dtype=np.int64),
        context_lens=np.asarray(context_lens, dtype=np.int64),
        block_tables=block_tables,
        seq_need_compute_logits=np.asarray(need_logits, dtype=np.int64),
    )
    return np.asarray(input_ids, dtype=np.int64), np.asarray(positions, dtype=np.int64), ctx


# --------------------------------------------------------------------------
# a4: paged gather + causal varlen attention (the fallback route's semantics)
# --------------------------------------------------------------------------


def gather_paged_kv(k_cache, v_cache, block_table_row, seqlen_k: int, page_size: int):
    """layers/attention.rs:143-164: token-ordered rows of one sequence.

    The reference walks the block-table row page by page, pushing
    ``block * page_size + s`` for s = 0..page_size until it holds seqlen_k
    slots (fewer if the row runs out); the same list is formed here as one
    array, ``(row[:, None] * page_size + arange(page_size)).ravel()[:seqlen_k]``.
    """
    row = np.asarray(block_table_row, dtype=np.int64).reshape(-1)
    slots = (row[:, None] * page_size + np.arange(page_size, dtype=np.int64)).reshape(-1)
    idx = slots[:seqlen_k]
    hkv, d = k_cache.shape[2], k_cache.shape[3]
    return k_cache.reshape(-1, hkv, d)[idx], v_cache.reshape(-1, hkv, d)[idx]


def causal_attention_one(q, k, v, scale: float, causal: bool = True, acc=np.float64):
    """Exact softmax attention for one sequence, GQA by head grouping.

    q: [q_len, Hq, D]; k, v: [k_len, Hkv, D].  Causal mask aligned bottom-right:
    key j is visible to query i iff j <= i + (k_len - q_len) (the cache-offset
    case candle_nn's unfused varlen path and FA2's causal mode both implement,
    layers/attention.rs:78-84).  Returns float32 [q_len, Hq, D].
    """
    q_len, hq, d = q.shape
    k_len, hkv, _ = k.shape
    if q_len == 0:
        return np.zeros((0, hq, d), np.float32)
    g = hq // hkv
    qh = q.astype(acc, copy=False).reshape(q_len, hkv, g, d).transpose(1, 2, 0, 3)  # [hkv,g,q,d]
    kh = k.astype(acc, copy=False).transpose(1, 2, 0)  # [hkv,d,k]
    vh = v.astype(acc, copy=False).transpose(1, 0, 2)  # [hkv,k,d]
    s = np.matmul(qh, kh[:, None]) * scale  # [hkv,g,q,k]
    if causal:
        i = np.arange(q_len)[:, None]
        j = np.arange(k_len)[None, :]
        s = np.where(j <= i + (k_len - q_len), s, -np.inf)
    m = np.max(s, axis=-1, keepdims=True)
    m = np.where(np.isfinite(m), m, 0.0)
    p = np.exp(s - m)
    l = np.sum(p, axis=-1, keepdims=True)
    o = np.matmul(p, vh[:, None]) / np.where(l > 0, l, 1.0)  # [hkv,g,q,d]
    return o.transpose(2, 0, 1, 3).reshape(q_len, hq, d).astype(np.float32)


def varlen_attention(q, k, v, cu_seqlens_q, cu_seqlens_k, scale, causal=True, acc=np.float64):
    """flash_attn_varlen semantics on contiguous K/V (layers/attention.rs:60-74)."""
    out = np.zeros(q.shape, np.float32)
    for b in range(len(cu_seqlens_q) - 1):
        q0, q1 = int(cu_seqlens_q[b]), int(cu_seqlens_q[b + 1])
        k0, k1 = int(cu_seqlens_k[b]), int(cu_seqlens_k[b + 1])
        out[q0:q1] = causal_attention_one(q[q0:q1], k[k0:k1], v[k0:k1], scale, causal, acc)
    return out


def paged_attention(q, k_cache, v_cache, cu_seqlens_q, cu_seqlens_k, block_tables, scale,
                    causal=True, acc=np.float64, pool=None):
    """Paged route (layers/attention.rs:38-59) computed the fallback way
    (attention.rs:105-136): gather each sequence's rows, then attend.

    ``pool`` (a concurrent.futures executor) runs the independent
    per-sequence gathers and attentions on several host threads; the result
    is the same as the serial loop."""
    out = np.zeros(q.shape, np.float32)
    page = k_cache.shape[1]

    def one(b):
        q0, q1 = int(cu_seqlens_q[b]), int(cu_seqlens_q[b + 1])
        k_len = int(cu_seqlens_k[b + 1]) - int(cu_seqlens_k[b])
        kb, vb = gather_paged_kv(k_cache, v_cache, block_tables[b], k_len, page)
        out[q0:q1] = causal_attention_one(q[q0:q1], kb, vb, scale, causal, acc)

    seqs = range(len(cu_seqlens_q) - 1)
    if pool is None:
        for b in seqs:
            one(b)
    else:
        list(pool.map(one, seqs))
    return out


def attention_forward(q, k, v, ctx: Context, k_cache, v_cache, scale, acc=np.float64,
                      pool=None):
    """Attention::forward (layers/attention.rs:85-137): store, then attend
    through the block table when present, else on the fresh K/V."""
    if k_cache is not None and v_cache is not None:
        store_kvcache(k, v, k_cache, v_cache, ctx.slot_mapping)
    if ctx.block_tables is not None:
        return paged_attention(q, k_cache, v_cache, ctx.cu_seqlens_q, ctx.cu_seqlens_k,
                               ctx.block_tables, scale, True, acc, pool)
    return varlen_attention(q, k, v, ctx.cu_seqlens_q, ctx.cu_seqlens_k, scale, True, acc)


# --------------------------------------------------------------------------
# a5 / a6: qk-RMSNorm and RoPE with the reference's rounding points
# --------------------------------------------------------------------------


def rms_norm(x, weight, eps: float, dtype: str) -> np.ndarray:
    """layers/layernorm.rs:18-25.

    f32 math; ``x * rsqrt(mean(x^2) + eps)`` is rounded to the activation
    dtype *before* the weight multiply, whose product is rounded again.
    """
    xf = np.asarray(x, np.float32)
    var = np.mean(xf * xf, axis=-1, keepdims=True, dtype=np.float32)
    inv = np.float32(1.0) / np.sqrt(var + np.float32(eps))
    normed = round_to(xf * inv, dtype)
    return round_to(normed * np.asarray(weight, np.float32), dtype)


def residual_rms_norm(x, residual, weight, eps: float, dtype: str):
    """layers/layernorm.rs:27-42: s = x + residual in f32; returns
    (dtype(dtype(s * rsqrt(mean(s^2) + eps)) * w), dtype(s))."""
    s = np.asarray(x, np.float32) + np.asarray(residual, np.float32)
    var = np.mean(s * s, axis=-1, keepdims=True, dtype=np.float32)
    inv = np.float32(1.0) / np.sqrt(var + np.float32(eps))
    out = round_to(round_to(s * inv, dtype) * np.asarray(weight, np.float32), dtype)
    return out, round_to(s, dtype)


def silu_and_mul(gate_up, dtype: str):
    """layers/activation.rs:5-17: dtype(dtype(silu(g)) * u), silu in f32."""
    gu = np.asarray(gate_up, np.float32)
    F = gu.shape[-1] // 2
    g, u = gu[..., :F], gu[..., F:]
    silu = round_to(g / (np.float32(1.0) + np.exp(-g)), dtype)
    return round_to(silu * u, dtype)


def rope_inv_freq(head_dim: int, base: float) -> np.ndarray:
    """layers/rotary_embedding.rs:31-37: 1/exp((2i/D)*ln(base)) in f32."""
    exponent = np.arange(0, head_dim, 2, dtype=np.float32) / np.float32(head_dim)
    ln_base = np.float32(math.log(base))
    return (np.float32(1.0) / np.exp(exponent * ln_base)).astype(np.float32)


def rope_cos_sin(positions, head_dim: int, base: float) -> Tuple[np.ndarray, np.ndarray]:
    """rotary_embedding.rs:38-49 + index_select (:60): f32 cos/sin rows."""
    inv = rope_inv_freq(head_dim, base)
    t = np.asarray(positions, dtype=np.int64).astype(np.float32)
    freqs = (t[:, None] * inv[None, :]).astype(np.float32)
    return np.cos(freqs).astype(np.float32), np.sin(freqs).astype(np.float32)


def apply_rotary_emb(x, cos, sin, dtype: str) -> np.ndarray:
    """rotary_embedding.rs:11-26 (NeoX half split), rounding after each op."""
    half = x.shape[-1] // 2
    x1 = x[..., :half]
    x2 = x[..., half:]
    y1 = round_to(round_to(x1 * cos, dtype) - round_to(x2 * sin, dtype), dtype)
    y2 = round_to(round_to(x2 * cos, dtype) + round_to(x1 * sin, dtype), dtype)
    return np.concatenate([y1, y2], axis=-1)


def rope_forward(positions, q, k, head_dim: int, base: float, dtype: str):
    """rotary_embedding.rs:59-70: cos/sin cast to the activation dtype first."""
    cos, sin = rope_cos_sin(positions, head_dim, base)
    cos = round_to(cos, dtype)[:, None, :]
    sin = round_to(sin, dtype)[:, None, :]
    return apply_rotary_emb(q, cos, sin, dtype), apply_rotary_emb(k, cos, sin, dtype)


def qknorm_rope(qkv, positions, num_q_heads, num_kv_heads, head_dim, q_w, k_w, eps, theta,
                dtype: str):
    """Qwen3Attention::forward prologue (models/qwen3.rs:126-141):
    split_qkv (:33-38) -> per-head q/k RMSNorm -> RoPE.  Returns (q, k, v)."""
    T = qkv.shape[0]
    qs = num_q_heads * head_dim
    ks = num_kv_heads * head_dim
    q = np.asarray(qkv[:, :qs], np.float32).reshape(T, num_q_heads, head_dim)
    k = np.asarray(qkv[:, qs:qs + ks], np.float32).reshape(T, num_kv_heads, head_dim)
    v = np.asarray(qkv[:, qs + ks:qs + 2 * ks], np.float32).reshape(T, num_kv_heads, head_dim)
    if q_w is not None:
        q = rms_norm(q, q_w, eps, dtype)
        k = rms_norm(k, k_w, eps, dtype)
    q, k = rope_forward(positions, q, k, head_dim, theta, dtype)
    return q, k, v


# --------------------------------------------------------------------------
# KAT-1 inputs: nanovllm_rs/src/bin/repro.rs
# --------------------------------------------------------------------------

REPRO_N_HEADS = 16
REPRO_N_KV_HEADS = 8
REPRO_HEAD_DIM = 128
REPRO_BLOCK_SIZE = 256
REPRO_PRIOR_LEN = 6


def repro_mk(seed: np.float32, n: int, h: int, head_dim: int = REPRO_HEAD_DIM) -> np.ndarray:
    """repro.rs:50-53: data[i] = ((i*seed) % 17 - 8) / 8 in f32, then bf16."""
    i = np.arange(n * h * head_dim, dtype=np.float32)
    data = (np.fmod(i * np.float32(seed), np.float32(17.0)) - np.float32(8.0)) / np.float32(8.0)
    return round_bf16(data.astype(np.float32)).reshape(n, h, head_dim)


def repro_inputs(layer: int):
    """repro.rs:55-63 for one layer: (k_prior, v_prior, k_new, v_new, q_new)."""
    base = np.float32(1.0) + np.float32(layer) * np.float32(0.13)
    sd = lambda c: np.float32(np.float32(c) * base)  # noqa: E731
    k_prior = repro_mk(sd(0.7), REPRO_PRIOR_LEN, REPRO_N_KV_HEADS)
    v_prior = repro_mk(sd(1.3), REPRO_PRIOR_LEN, REPRO_N_KV_HEADS)
    k_new = repro_mk(sd(0.9), 1, REPRO_N_KV_HEADS)
    v_new = repro_mk(sd(1.7), 1, REPRO_N_KV_HEADS)
    q_new = repro_mk(sd(2.1), 1, REPRO_N_HEADS)
    return k_prior, v_prior, k_new, v_new, q_new


# --------------------------------------------------------------------------
# f4: FP8 (e4m3) KV-cache format -- no counterpart in the reference, whose
# pool is in the model dtype (engine/model_runner.rs:286-303).  Restated here
# as the checker of nvkv's optional fp8 pool: each (token, kv head) row of D
# values is stored as e4m3 codes with its own f32 scale,
#   scale = amax / 448,  code = e4m3_rn_satfinite(x * (448 / amax))
# (amax = max |x| over the row; an all-zero row gets scale 0 and zero codes),
# and read back as code_value * scale.  Scales are laid out [Nb, Hkv, P].
# --------------------------------------------------------------------------

E4M3_MAX = 448.0


def _e4m3_table():
    """Value of every e4m3 code (OCP E4M3FN: bias 7, no infinities, codes
    0x7F / 0xFF are NaN)."""
    vals = np.zeros(256, np.float64)
    for c in range(256):
        s = -1.0 if c & 0x80 else 1.0
        e = (c >> 3) & 0xF
        m = c & 0x7
        if e == 0xF and m == 0x7:
            vals[c] = np.nan
        elif e == 0:
            vals[c] = s * m * 2.0 ** -9
        else:
            vals[c] = s * (1 + m / 8.0) * 2.0 ** (e - 7)
    return vals


E4M3_VALUES = _e4m3_table()


def e4m3_encode(x) -> np.ndarray:
    """float32 -> e4m3 codes (uint8): round to nearest, ties to the even code,
    magnitudes above 448 saturate to 448 (the satfinite conversion)."""
    x = np.asarray(x, np.float32).astype(np.float64)
    a = np.minimum(np.abs(x), E4M3_MAX)
    e = np.floor(np.log2(np.maximum(a, 2.0 ** -9)))
    e = np.clip(e, -6, 8)  # exponent of the binade; below 2^-6 the subnormal step 2^-9
    q = 2.0 ** (e - 3)
    mag = np.rint(a / q) * q  # exact in f64; rint rounds half to even
    mag = np.minimum(mag, E4M3_MAX)
    pos = E4M3_VALUES[:0x7F]  # the finite non-negative codes, increasing
    code = np.searchsorted(pos, mag).astype(np.uint8)
    return np.where(x < 0, code | 0x80, code).astype(np.uint8)


def e4m3_decode(code) -> np.ndarray:
    return E4M3_VALUES[np.asarray(code, np.uint8)].astype(np.float32)


def quantize_rows_fp8(x):
    """[..., D] float32 rows -> (codes uint8 [..., D], scales float32 [...]),
    with the f32 arithmetic of nvkv's store (division and product rounded to
    nearest)."""
    x = np.asarray(x, np.float32)
    amax = np.max(np.abs(x), axis=-1)
    with np.errstate(divide="ignore"):
        scale = (amax / np.float32(E4M3_MAX)).astype(np.float32)
        inv = np.where(amax > 0, np.float32(E4M3_MAX) / amax, np.float32(0)).astype(np.float32)
    codes = e4m3_encode((x * inv[..., None]).astype(np.float32))
    return codes, scale


def store_kvcache_fp8(key, value, k_cache, v_cache, k_scale, v_scale, slot_mapping) -> None:
    """The fp8 pool's store: caches [Nb, P, Hkv, D] uint8, scales [Nb, Hkv, P]
    float32; row t of key/value ([T, Hkv, D], float32 values) goes to slot
    slot_mapping[t] (negative slots skipped)."""
    P = k_cache.shape[1]
    slots = np.asarray(slot_mapping, np.int64)
    for cache, scales, src in ((k_cache, k_scale, key), (v_cache, v_scale, value)):
        codes, sc = quantize_rows_fp8(np.asarray(src, np.float32))
        for t, s in enumerate(slots):
            if s < 0:
                continue
            cache[s // P, s % P] = codes[t]
            scales[s // P, :, s % P] = sc[t]


def dequantize_pages_fp8(cache, scales) -> np.ndarray:
    """[Nb, P, Hkv, D] codes + [Nb, Hkv, P] scales -> float32 values."""
    vals = e4m3_decode(cache)
    return (vals * np.transpose(scales, (0, 2, 1))[..., None]).astype(np.float32)


# --------------------------------------------------------------------------
# Sampler (layers/sampler.rs:7-21) and the counter-based noise of its
# device form
# --------------------------------------------------------------------------
_PHILOX_M0, _PHILOX_M1 = 0xD2511F53, 0xCD9E8D57
_PHILOX_W0, _PHILOX_W1 = 0x9E3779B9, 0xBB67AE85


def philox4x32_10(ctr, key):
    """Philox4x32-10 (Salmon, Moraes, Dror and Shaw, SC 2011; the Random123
    definition): ctr [..., 4] uint32 words, key [2] uint32 words; ten rounds
    of two 32x32->64 multiplies, key bumped by the Weyl constants between
    rounds.  Returns [..., 4] uint32."""
    c = [np.asarray(ctr[..., i], np.uint64) for i in range(4)]
    k0, k1 = np.uint64(key[0]), np.uint64(key[1])
    m32 = np.uint64(0xFFFFFFFF)
    for _ in range(10):
        p0 = np.uint64(_PHILOX_M0) * c[0]
        p1 = np.uint64(_PHILOX_M1) * c[2]
        c = [((p1 >> np.uint64(32)) ^ c[1] ^ k0) & m32, p1 & m32,
             ((p0 >> np.uint64(32)) ^ c[3] ^ k1) & m32, p0 & m32]
        k0 = (k0 + np.uint64(_PHILOX_W0)) & m32
        k1 = (k1 + np.uint64(_PHILOX_W1)) & m32
    return np.stack(c, -1).astype(np.uint32)


def sample_uniforms(num_rows: int, vocab: int, seed: int, step: int, vocab_offset: int = 0):
    """u [num_rows, vocab] f32 of the device sampler: Philox4x32-10 keyed by
    the 64-bit seed at counter (global index // 4, row, step low, step high),
    word global index % 4, u = ((bits >> 9) + 1/2) 2^-23."""
    g = vocab_offset + np.arange(vocab, dtype=np.int64)
    q0 = int(g[0] // 4) if vocab else 0
    groups = np.arange(q0, int(g[-1] // 4) + 1 if vocab else q0, dtype=np.int64)
    ctr = np.zeros((num_rows, len(groups), 4), np.uint64)
    ctr[..., 0] = groups[None, :]
    ctr[..., 1] = np.arange(num_rows, dtype=np.int64)[:, None]
    ctr[..., 2] = step & 0xFFFFFFFF
    ctr[..., 3] = (step >> 32) & 0xFFFFFFFF
    bits = philox4x32_10(ctr, (seed & 0xFFFFFFFF, (seed >> 32) & 0xFFFFFFFF))
    word = bits[:, g // 4 - q0, g % 4]
    return (((word >> np.uint32(9)).astype(np.float32) + np.float32(0.5)) *
            np.float32(2.0 ** -23))


def reference_sample(logits, temperatures, u):
    """Sampler::forward (sampler.rs:7-21) given its uniforms u: softmax of the
    f32 logits divided by the temperature, divided by max(-log u, 1e-10),
    first arg-max."""
    x = np.asarray(logits, np.float32) / np.asarray(temperatures, np.float32)[:, None]
    x = x - x.max(-1, keepdims=True)
    p = np.exp(x)
    p = p / p.sum(-1, keepdims=True)
    noise = np.maximum(-np.log(u.astype(np.float64)), 1e-10)
    return np.argmax(p / noise, axis=-1)


def gumbel_sample(logits, temperatures, seed: int, step: int, vocab_offset: int = 0):
    """The device sampler's arithmetic (nvkv_sample): per row the largest
    score logit / T - log(max(-log u, 1e-10)) in f32 and its global index
    (first maximum); T <= 0 scores the logit itself.  Returns (value f32,
    index int64)."""
    x = np.asarray(logits, np.float32)
    B, V = x.shape
    t = np.asarray(temperatures, np.float32)
    u = sample_uniforms(B, V, seed, step, vocab_offset)
    e = np.maximum(-np.log(u), np.float32(1e-10)).astype(np.float32)
    z = (x / np.where(t > 0, t, np.float32(1))[:, None]).astype(np.float32) - np.log(e)
    z = np.where((t > 0)[:, None], z, x)
    i = np.argmax(z, axis=-1)
    return z[np.arange(B), i], i.astype(np.int64) + vocab_offset
