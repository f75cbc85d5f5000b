"""KV-pool block manager with prefix caching, through the C ABI.

Mirrors the reference's ``BlockManager`` (nanovllm_rs/src/engine/
block_manager.rs): the same methods, arguments and decisions, so a
scheduler written against the reference's interface gets the same block
tables (page ids for ``block_tables`` / ``slot_mapping``) and the same
prefix-cache hits.  The work runs in the library (``nvkv_block_manager_*``);
calls that the reference would abort on raise ``NvkvError`` and leave the
manager unchanged.
"""
from __future__ import annotations

import ctypes
from typing import List, Sequence as Seq_, Tuple

import numpy as np

from ._lib import BlockSeq, StepSizes, check, lib


class Sequence:
    """The Sequence fields the block manager reads and writes
    (engine/sequence.rs:20-60): token ids, ``num_cached_tokens``,
    ``num_new_tokens`` (set by the scheduler) and ``block_table``."""

    def __init__(self, token_ids: Seq_[int], block_size: int):
        self.token_ids: List[int] = [int(t) for t in token_ids]
        self.block_size = block_size
        self.num_cached_tokens = 0
        self.num_new_tokens = 0
        self.block_table: List[int] = []

    def __len__(self) -> int:
        return len(self.token_ids)

    def num_blocks(self) -> int:
        return (len(self.token_ids) + self.block_size - 1) // self.block_size

    def num_cached_blocks(self) -> int:
        return self.num_cached_tokens // self.block_size

    def append_token(self, token_id: int) -> None:
        self.token_ids.append(int(token_id))


class _Marshal:
    """One C view (nvkv_block_seq) of a Sequence for the duration of a call."""

    def __init__(self, seq: Sequence, extra_blocks: int = 0):
        self.seq = seq
        self.tokens = np.ascontiguousarray(np.asarray(seq.token_ids, dtype=np.uint32))
        cap = max(seq.num_blocks(), len(seq.block_table)) + 1 + extra_blocks
        self.table = np.zeros(cap, dtype=np.uint32)
        self.table[:len(seq.block_table)] = seq.block_table
        self.c = BlockSeq(self.tokens.ctypes.data if self.tokens.size else None, len(self.tokens),
                          seq.num_cached_tokens, seq.num_new_tokens, self.table.ctypes.data,
                          len(seq.block_table), cap)

    def ref(self):
        return ctypes.byref(self.c)

    def write_back(self) -> None:
        self.seq.num_cached_tokens = int(self.c.num_cached_tokens)
        self.seq.num_new_tokens = int(self.c.num_new_tokens)
        self.seq.block_table = [int(b) for b in self.table[:self.c.block_table_len]]


def compute_hash(token_ids: Seq_[int], prefix: int = -1) -> int:
    """BlockManager::compute_hash (block_manager.rs:53-64)."""
    t = np.ascontiguousarray(np.asarray(token_ids, dtype=np.int64))
    out = ctypes.c_int64(0)
    check(lib.nvkv_block_hash(t.ctypes.data if t.size else None, t.size, int(prefix),
                              ctypes.byref(out)))
    return int(out.value)


class BlockManager:
    """BlockManager::new(num_blocks, block_size) (block_manager.rs:44-52)."""

    compute_hash = staticmethod(compute_hash)

    def __init__(self, num_blocks: int, block_size: int):
        self.num_blocks = num_blocks
        self.block_size = block_size
        h = ctypes.c_void_p()
        check(lib.nvkv_block_manager_create(num_blocks, block_size, ctypes.byref(h)))
        self._h = h

    def close(self) -> None:
        if self._h:
            lib.nvkv_block_manager_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # -- the reference's methods ---------------------------------------------
    def can_allocate(self, num_tokens: int) -> bool:
        out = ctypes.c_int(0)
        check(lib.nvkv_block_manager_can_allocate(self._h, num_tokens, ctypes.byref(out)))
        return bool(out.value)

    def get_token_layout(self, seq: Sequence) -> Tuple[int, int, int]:
        m = _Marshal(seq)
        u, f, n = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int64()
        check(lib.nvkv_block_manager_get_token_layout(self._h, m.ref(), ctypes.byref(u),
                                                      ctypes.byref(f), ctypes.byref(n)))
        return int(u.value), int(f.value), int(n.value)

    def allocate(self, seq: Sequence) -> None:
        m = _Marshal(seq)
        check(lib.nvkv_block_manager_allocate(self._h, m.ref()))
        m.write_back()

    def deallocate(self, seq: Sequence) -> None:
        m = _Marshal(seq)
        check(lib.nvkv_block_manager_deallocate(self._h, m.ref()))
        m.write_back()

    def can_append(self, seq: Sequence, num_new_tokens: int) -> bool:
        m = _Marshal(seq)
        out = ctypes.c_int(0)
        check(lib.nvkv_block_manager_can_append(self._h, m.ref(), num_new_tokens,
                                                ctypes.byref(out)))
        return bool(out.value)

    def may_append(self, seq: Sequence) -> None:
        m = _Marshal(seq)
        check(lib.nvkv_block_manager_may_append(self._h, m.ref()))
        m.write_back()

    def append_batch(self, seqs, num_new_tokens) -> int:
        """can_append + may_append over `seqs` in order, stopping at the first
        that does not fit; returns how many were appended (the scheduler's
        running-queue pass, scheduler.rs:103-140, minus the preemption the
        caller does at the returned index)."""
        ms = [_Marshal(s) for s in seqs]
        arr = (BlockSeq * len(ms))(*[m.c for m in ms])
        nn = np.ascontiguousarray(np.asarray(num_new_tokens, dtype=np.int64))
        done = ctypes.c_int64(0)
        try:
            check(lib.nvkv_block_manager_append_batch(self._h, arr, len(ms),
                                                      nn.ctypes.data if nn.size else None,
                                                      ctypes.byref(done)))
        finally:
            for k, m in enumerate(ms):
                m.c = arr[k]
                m.write_back()
        return int(done.value)

    # -- state (no reference counterpart) -------------------------------------
    @property
    def num_free(self) -> int:
        out = ctypes.c_int64(0)
        check(lib.nvkv_block_manager_num_free(self._h, ctypes.byref(out)))
        return int(out.value)

    def free_block_ids(self) -> List[int]:
        """The free list front to back (the reference's free_block_ids)."""
        buf = np.zeros(self.num_blocks, dtype=np.uint32)
        n = ctypes.c_int64(0)
        check(lib.nvkv_block_manager_free_ids(self._h, buf.ctypes.data, buf.size,
                                              ctypes.byref(n)))
        return [int(b) for b in buf[:n.value]]

    def block_info(self, block_id: int) -> Tuple[int, int, int, bool]:
        """(ref_count, hash, number of stored token ids, in the used set)."""
        r, h, n, u = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int()
        check(lib.nvkv_block_manager_block_info(self._h, block_id, ctypes.byref(r),
                                                ctypes.byref(h), ctypes.byref(n),
                                                ctypes.byref(u)))
        return int(r.value), int(h.value), int(n.value), bool(u.value)

    def lookup(self, h: int) -> int:
        """hash_to_block_id.get(h), or -1."""
        out = ctypes.c_int64(0)
        check(lib.nvkv_block_manager_lookup(self._h, int(h), ctypes.byref(out)))
        return int(out.value)


def prepare_step(seqs, block_size: int) -> dict:
    """ModelRunner::prepare_model_input + prepare_block_tables
    (engine/model_runner.rs:53-160) for a list of Sequences: input_ids,
    positions and the Context fields (cu_seqlens_q/k, max_seqlen_q/k,
    slot_mapping, context_lens, block_tables or None, seq_need_compute_logits),
    as numpy arrays of the reference's dtypes."""
    ms = [_Marshal(s) for s in seqs]
    arr = (BlockSeq * max(len(ms), 1))(*[m.c for m in ms])
    sizes = StepSizes()
    check(lib.nvkv_prepare_step(arr, len(ms), block_size, None, None, None, None, None, None,
                                None, None, 0, 0, 0, ctypes.byref(sizes)))  # size query
    B = len(ms)
    w = int(sizes.block_table_width) if sizes.has_block_tables else 0
    out = dict(input_ids=np.zeros(sizes.num_tokens, np.int64),
               positions=np.zeros(sizes.num_tokens, np.int64),
               cu_seqlens_q=np.zeros(B + 1, np.uint32), cu_seqlens_k=np.zeros(B + 1, np.uint32),
               slot_mapping=np.zeros(sizes.num_slots, np.int64),
               context_lens=np.zeros(B, np.int64),
               seq_need_compute_logits=np.zeros(sizes.num_need_logits, np.int64),
               block_tables=np.zeros((B, w), np.uint32) if sizes.has_block_tables else None)

    def ptr(a):
        return a.ctypes.data if a is not None and a.size else None

    check(lib.nvkv_prepare_step(arr, B, block_size, ptr(out["input_ids"]), ptr(out["positions"]),
                                ptr(out["cu_seqlens_q"]), ptr(out["cu_seqlens_k"]),
                                ptr(out["slot_mapping"]), ptr(out["context_lens"]),
                                ptr(out["seq_need_compute_logits"]),
                                ptr(out["block_tables"]), sizes.num_tokens, sizes.num_slots,
                                B * w, ctypes.byref(sizes)))
    out["max_seqlen_q"] = int(sizes.max_seqlen_q)
    out["max_seqlen_k"] = int(sizes.max_seqlen_k)
    return out


def kv_pool_blocks(free_bytes: int, total_bytes: int, gpu_memory_utilization: float,
                   num_layers: int, block_size: int, num_kv_heads: int, head_dim: int,
                   dtype_bytes: int) -> int:
    """ModelRunner::probe_num_kvcache_blocks (engine/model_runner.rs:264-284)
    for given free / total device bytes; raises when no block fits."""
    out = ctypes.c_int64(0)
    check(lib.nvkv_kv_pool_blocks(free_bytes, total_bytes, gpu_memory_utilization, num_layers,
                                  block_size, num_kv_heads, head_dim, dtype_bytes,
                                  ctypes.byref(out)))
    return int(out.value)


def kv_pool_probe(gpu_memory_utilization: float, num_layers: int, block_size: int,
                  num_kv_heads: int, head_dim: int, dtype_bytes: int, group=None) -> int:
    """The same on the current device (cudaMemGetInfo); with a process group,
    the minimum over its ranks (the reconciliation the reference requires
    before allocating)."""
    out = ctypes.c_int64(0)
    check(lib.nvkv_kv_pool_probe(gpu_memory_utilization, num_layers, block_size, num_kv_heads,
                                 head_dim, dtype_bytes, ctypes.byref(out)))
    return kv_pool_reconcile(int(out.value), group)


def kv_pool_reconcile(num_blocks: int, group=None) -> int:
    """The minimum of every rank's block budget (every rank must allocate the
    same pool, model_runner.rs:265-266)."""
    if group is None:
        return num_blocks
    import torch
    import torch.distributed as dist
    t = torch.tensor([num_blocks], dtype=torch.int64,
                     device="cuda" if dist.get_backend(group) == "nccl" else "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MIN, group=group)
    return int(t.item())
