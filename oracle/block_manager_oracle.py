"""CPU restatement of nanovllm_rs's KV block manager (prefix caching).

TEST INFRASTRUCTURE ONLY.  This module is the checker that the C++ block
manager (``nanovllm-rs_b200/csrc/block_manager.cu``, C ABI
``nvkv_block_manager_*``) is compared against.  Only ``tests/`` and the
benchmark's CPU-baseline leg may import it; the product never does.

It follows ``nanovllm_rs/src/engine/block_manager.rs`` method by method
(line numbers below), with Python lists, dicts and a deque standing in for
the reference's Vec, HashMap, HashSet and VecDeque, so the order in which
free blocks are handed out is the reference's.  ``Seq`` carries the fields of
``engine/sequence.rs`` the block manager reads and writes.

The block hash is xxh64 with seed 0 (xxhash-rust 0.8.16, pinned in
``nanovllm_rs/Cargo.lock:2714-2717``; not part of the reference tree).  Its
published algorithm is restated in ``xxh64`` below and pinned against
vectors made by an independent implementation (the ``xxhash`` Python
package) in ``tests/golden/xxh64_kat.json``.

Parity status: pinned for the hash (golden vectors); the block-manager
logic is a line-by-line restatement with no reference-produced fixtures (the
reference has no tests for it and cannot be run here).
"""
from __future__ import annotations

import struct
from collections import deque

_M64 = (1 << 64) - 1
_P1 = 0x9E3779B185EBCA87
_P2 = 0xC2B2AE3D27D4EB4F
_P3 = 0x165667B19E3779F9
_P4 = 0x85EBCA77C2B2AE63
_P5 = 0x27D4EB2F165667C5


def _rotl(x: int, r: int) -> int:
    return ((x << r) | (x >> (64 - r))) & _M64


def _round(acc: int, lane: int) -> int:
    acc = (acc + lane * _P2) & _M64
    return (_rotl(acc, 31) * _P1) & _M64


def xxh64(data: bytes, seed: int = 0) -> int:
    """XXH64 of `data` (the published xxHash 64-bit algorithm), as an
    unsigned 64-bit integer."""
    n = len(data)
    i = 0
    if n >= 32:
        v = [(seed + _P1 + _P2) & _M64, (seed + _P2) & _M64, seed & _M64, (seed - _P1) & _M64]
        while i + 32 <= n:
            for lane in range(4):
                v[lane] = _round(v[lane], int.from_bytes(data[i + 8 * lane:i + 8 * lane + 8],
                                                          "little"))
            i += 32
        h = (_rotl(v[0], 1) + _rotl(v[1], 7) + _rotl(v[2], 12) + _rotl(v[3], 18)) & _M64
        for lane in range(4):
            h ^= _round(0, v[lane])
            h = (h * _P1 + _P4) & _M64
    else:
        h = (seed + _P5) & _M64
    h = (h + n) & _M64
    while i + 8 <= n:
        h ^= _round(0, int.from_bytes(data[i:i + 8], "little"))
        h = (_rotl(h, 27) * _P1 + _P4) & _M64
        i += 8
    if i + 4 <= n:
        h ^= (int.from_bytes(data[i:i + 4], "little") * _P1) & _M64
        h = (_rotl(h, 23) * _P2 + _P3) & _M64
        i += 4
    while i < n:
        h ^= (data[i] * _P5) & _M64
        h = (_rotl(h, 11) * _P1) & _M64
        i += 1
    h ^= h >> 33
    h = (h * _P2) & _M64
    h ^= h >> 29
    h = (h * _P3) & _M64
    h ^= h >> 32
    return h


def compute_hash(token_ids, prefix: int) -> int:
    """BlockManager::compute_hash (block_manager.rs:53-64): xxh64 over
    `prefix` (unless -1) and the token ids, each as a little-endian i64;
    the digest reinterpreted as i64."""
    buf = b""
    if prefix != -1:
        buf += struct.pack("<q", prefix)
    buf += struct.pack(f"<{len(token_ids)}q", *[int(t) for t in token_ids])
    d = xxh64(buf, 0)
    return d - (1 << 64) if d >= (1 << 63) else d


class Seq:
    """The Sequence fields the block manager touches (sequence.rs:20-60)."""

    def __init__(self, token_ids, block_size: int):
        self.token_ids = [int(t) for t in token_ids]
        self.block_size = block_size
        self.num_cached_tokens = 0
        self.num_new_tokens = 0
        self.block_table: list[int] = []

    def __len__(self) -> int:
        return len(self.token_ids)

    def num_blocks(self) -> int:  # sequence.rs:124-126
        return (len(self.token_ids) + self.block_size - 1) // self.block_size

    def block(self, i: int):  # sequence.rs:132-137
        assert i < self.num_blocks()
        return self.token_ids[i * self.block_size:min((i + 1) * self.block_size,
                                                      len(self.token_ids))]

    def slice_tokens(self, a: int, b: int):  # sequence.rs:95-97
        assert 0 <= a <= b <= len(self.token_ids)
        return self.token_ids[a:b]

    def num_cached_blocks(self) -> int:  # sequence.rs:99-101
        return self.num_cached_tokens // self.block_size

    def append_token(self, t: int) -> None:  # sequence.rs:139-144
        self.token_ids.append(int(t))


class Block:  # block_manager.rs:5-33
    def __init__(self, block_id: int):
        self.block_id = block_id
        self.ref_count = 0
        self.hash = -1
        self.token_ids: list[int] = []

    def update(self, h: int, token_ids) -> None:
        self.hash = h
        self.token_ids = list(token_ids)

    def reset(self) -> None:
        self.ref_count = 1
        self.hash = -1
        self.token_ids = []


class BlockManager:  # block_manager.rs:35-52
    def __init__(self, num_blocks: int, block_size: int):
        self.block_size = block_size
        self.blocks = [Block(i) for i in range(num_blocks)]
        self.hash_to_block_id: dict[int, int] = {}
        self.free_block_ids = deque(range(num_blocks))
        self.used_block_ids: set[int] = set()

    compute_hash = staticmethod(compute_hash)

    def _allocate_block(self, block_id: int) -> Block:  # :66-82
        assert self.blocks[block_id].ref_count == 0
        h = self.blocks[block_id].hash
        if self.hash_to_block_id.get(h) == block_id:
            del self.hash_to_block_id[h]
        self.blocks[block_id].reset()
        if block_id in self.free_block_ids:
            self.free_block_ids.remove(block_id)
        self.used_block_ids.add(block_id)
        return self.blocks[block_id]

    def _deallocate_block(self, block_id: int) -> None:  # :84-89
        assert self.blocks[block_id].ref_count == 0
        self.used_block_ids.discard(block_id)
        self.free_block_ids.append(block_id)

    def can_allocate(self, num_tokens: int) -> bool:  # :93-96
        return len(self.free_block_ids) >= (num_tokens + self.block_size - 1) // self.block_size

    def get_token_layout(self, seq: Seq):  # :99-134
        assert not seq.block_table
        in_used = in_free = new = 0
        h = -1
        cache_miss = False
        nb = seq.num_blocks()
        for i in range(nb):
            token_ids = seq.block(i)
            h = compute_hash(token_ids, h) if len(token_ids) == self.block_size else -1
            block_id = self.hash_to_block_id.get(h, -1)
            if block_id == -1 or self.blocks[block_id].token_ids != token_ids or i == nb - 1:
                cache_miss = True
            if cache_miss:
                new += len(token_ids)
            elif block_id in self.used_block_ids:
                in_used += len(token_ids)
            else:
                in_free += len(token_ids)
        return in_used, in_free, new

    def allocate(self, seq: Seq) -> None:  # :136-190
        assert not seq.block_table
        h = -1
        nb = seq.num_blocks()
        for i in range(nb):
            token_ids = seq.block(i)
            h = compute_hash(token_ids, h) if len(token_ids) == self.block_size else -1
            block_id = self.hash_to_block_id.get(h, -1)
            if block_id == -1 or self.blocks[block_id].token_ids != token_ids or i == nb - 1:
                break  # cache miss
            seq.num_cached_tokens += self.block_size
            if block_id in self.used_block_ids:
                self.blocks[block_id].ref_count += 1
            else:
                self._allocate_block(block_id)
            self.blocks[block_id].update(h, token_ids)
            self.hash_to_block_id[h] = block_id
            seq.block_table.append(block_id)
        start = seq.num_cached_tokens
        end = seq.num_cached_tokens + seq.num_new_tokens
        i = start
        while i < end:
            chunk_end = min(i + self.block_size, end)
            token_ids = seq.slice_tokens(i, chunk_end)
            if i != start:
                h = compute_hash(token_ids, h) if len(token_ids) == self.block_size else -1
            block_id = self.free_block_ids[0]
            self._allocate_block(block_id)
            if h != -1:
                self.blocks[block_id].update(h, token_ids)
                self.hash_to_block_id[h] = block_id
            seq.block_table.append(block_id)
            i += self.block_size

    def deallocate(self, seq: Seq) -> None:  # :193-204
        for block_id in reversed(seq.block_table):
            self.blocks[block_id].ref_count -= 1
            assert self.blocks[block_id].ref_count >= 0
            if self.blocks[block_id].ref_count == 0:
                self._deallocate_block(block_id)
        seq.num_cached_tokens = 0
        seq.num_new_tokens = 0
        seq.block_table.clear()

    def can_append(self, seq: Seq, num_new_tokens: int) -> bool:  # :207-220
        bs = self.block_size
        cap = bs - (seq.num_cached_tokens % bs)
        if cap == bs:
            cap = 0
        needed = (num_new_tokens - cap + bs - 1) // bs  # floor division = div_euclid (bs > 0)
        return needed <= len(self.free_block_ids)

    def may_append(self, seq: Seq) -> None:  # :222-284
        bs = self.block_size
        i = seq.num_cached_blocks() * bs
        range_end = seq.num_cached_tokens + seq.num_new_tokens
        while i < range_end:
            chunk_end = min(i + bs, range_end)
            token_ids = seq.slice_tokens(i, chunk_end)
            block_idx = i // bs
            current = seq.block_table[block_idx] if block_idx < len(seq.block_table) else -1
            if current != -1:
                assert self.blocks[current].hash == -1
            if len(token_ids) % bs == 0:
                previous = seq.block_table[block_idx - 1] if i >= bs else -1
                prefix = self.blocks[previous].hash if previous != -1 else -1
                h = compute_hash(token_ids, prefix)
                if current == -1:
                    current = self.free_block_ids[0]
                    self._allocate_block(current)
                    seq.block_table.append(current)
                self.blocks[current].update(h, token_ids)
                self.hash_to_block_id[h] = self.blocks[current].block_id
            elif current == -1:
                block_id = self.free_block_ids[0]
                self._allocate_block(block_id)
                seq.block_table.append(block_id)
            i += bs
