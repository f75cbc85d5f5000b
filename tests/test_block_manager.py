"""The C++ KV block manager (nvkv_block_manager_*, via nvkv.blocks) against
the CPU restatement of engine/block_manager.rs (oracle/block_manager_oracle.py).

Parity bar: exact.  Every answer (hashes, layouts, can_* decisions), every
block table and num_cached_tokens, the free list in order and each block's
(ref count, hash, stored tokens, used) must be identical after every call.
The hash is pinned first against an independent XXH64 implementation
(tests/golden/xxh64_kat.json, made by tests/golden/make_xxh64_golden.py).
The workloads drive both managers the way the reference's scheduler does
(scheduler.rs:96-180: running sequences first with can_append / may_append,
preempting from the back; then waiting ones with get_token_layout /
can_allocate / allocate; chunked prefill; deallocate on finish).
"""
import json
import os
import random

import pytest

import block_manager_oracle as OB
from nvkv import NvkvError
from nvkv.blocks import BlockManager, Sequence, compute_hash

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "xxh64_kat.json")


def test_xxh64_known_answers():
    kat = json.load(open(GOLDEN))
    assert len(kat["bytes"]) > 80 and len(kat["block_hash"]) > 5
    for c in kat["bytes"]:
        assert OB.xxh64(bytes.fromhex(c["hex"])) == c["xxh64"], len(c["hex"]) // 2
    assert OB.xxh64(b"") == 0xEF46DB3751D8E999  # the published empty-input value
    for c in kat["block_hash"]:
        assert OB.compute_hash(c["tokens"], c["prefix"]) == c["hash"]
        assert compute_hash(c["tokens"], c["prefix"]) == c["hash"]  # the C ABI


def test_block_hash_matches_oracle_random():
    rng = random.Random(3)
    for _ in range(200):
        n = rng.randrange(0, 300)
        toks = [rng.randrange(1 << 32) for _ in range(n)]
        prefix = rng.choice([-1, rng.randrange(-(1 << 63), 1 << 63)])
        assert compute_hash(toks, prefix) == OB.compute_hash(toks, prefix)


def _state(bm, n):
    """Comparable state of either manager."""
    if isinstance(bm, OB.BlockManager):
        blocks = [(b.ref_count, b.hash, len(b.token_ids), b.block_id in bm.used_block_ids)
                  for b in bm.blocks]
        return list(bm.free_block_ids), blocks
    return bm.free_block_ids(), [bm.block_info(i) for i in range(n)]


class Pair:
    """The same workload on both managers, compared after every call."""

    def __init__(self, num_blocks, block_size):
        self.n, self.bs = num_blocks, block_size
        self.o = OB.BlockManager(num_blocks, block_size)
        self.c = BlockManager(num_blocks, block_size)

    def check(self, so, sc):
        assert so.block_table == sc.block_table
        assert (so.num_cached_tokens, so.num_new_tokens) == (sc.num_cached_tokens,
                                                              sc.num_new_tokens)
        assert _state(self.o, self.n) == _state(self.c, self.n)
        for b in self.o.blocks:  # the hash map: every registered hash resolves alike
            if b.hash != -1:
                assert self.o.hash_to_block_id.get(b.hash, -1) == self.c.lookup(b.hash)

    def call(self, name, so, sc, *args):
        try:
            a = getattr(self.o, name)(so, *args)
        except AssertionError:  # the reference would panic here
            with pytest.raises(NvkvError):
                getattr(self.c, name)(sc, *args)
            self.check(so, sc)
            raise ReferencePanic(name)
        b = getattr(self.c, name)(sc, *args)
        assert a == b, (name, a, b)
        self.check(so, sc)
        return a


class ReferencePanic(Exception):
    """The restated reference hit one of its asserts; the C ABI refused the
    same call and both states still match."""


def _workload(seed, block_size, num_blocks, steps, budget, max_seqs, prefixes):
    rng = random.Random(seed)
    p = Pair(num_blocks, block_size)
    shared = [[rng.randrange(151936) for _ in range(rng.randrange(1, 4 * block_size))]
              for _ in range(prefixes)]
    waiting, running = [], []
    made = 0
    stats = {"hits": 0, "preempted": 0, "finished": 0, "reference_panics": 0}

    def new_seq():
        base = list(rng.choice(shared)) if shared and rng.random() < 0.7 else []
        toks = base + [rng.randrange(151936) for _ in range(rng.randrange(1, 3 * block_size))]
        return (OB.Seq(toks, block_size), Sequence(toks, block_size),
                rng.randrange(1, 2 * block_size))  # tokens to generate

    for step in range(steps):
        while made < steps // 2 and rng.random() < 0.5:
            waiting.append(new_seq())
            made += 1
        tb = budget
        # running first (scheduler.rs:103-140)
        i, preempted = 0, False
        while i < len(running) and tb > 0:
            so, sc, _ = running[i]
            n = len(so) - so.num_cached_tokens
            n = min(n, tb)
            assert n > 0
            aborted = False
            while True:
                if p.call("can_append", so, sc, n):
                    so.num_new_tokens = sc.num_new_tokens = n
                    try:
                        p.call("may_append", so, sc)
                    except ReferencePanic:
                        # the reference's engine stops here; drop the sequence on
                        # both sides and carry on with the rest of the workload
                        stats["reference_panics"] += 1
                        so.num_new_tokens = sc.num_new_tokens = 0
                        p.call("deallocate", so, sc)
                        running.pop(i)
                        aborted = True
                    break
                vo, vc, g = running.pop()
                p.call("deallocate", vo, vc)
                waiting.insert(0, (vo, vc, g))
                preempted = True
                stats["preempted"] += 1
                if len(running) == i:
                    break
            if aborted:
                continue
            if len(running) == i:
                break
            tb -= so.num_new_tokens
            i += 1
        # then waiting (scheduler.rs:143-180)
        if not preempted:
            while waiting and tb > 0 and len(running) < max_seqs:
                so, sc, g = waiting[0]
                lay = p.call("get_token_layout", so, sc)
                used, free, n = lay
                n = min(n, tb)
                assert n > 0
                if n > tb or not (p.o.can_allocate(free + n) == p.c.can_allocate(free + n)
                                  and p.o.can_allocate(free + n)):
                    break
                so.num_new_tokens = sc.num_new_tokens = n
                p.call("allocate", so, sc)
                assert so.num_cached_tokens == used + free
                stats["hits"] += so.num_cached_tokens > 0
                tb -= n
                waiting.pop(0)
                running.append((so, sc, g))
        # the step ran: advance, sample, finish (scheduler.rs:55-94)
        for k in range(len(running) - 1, -1, -1):
            so, sc, g = running[k]
            done_prefill = so.num_cached_tokens + so.num_new_tokens == len(so)
            so.num_cached_tokens += so.num_new_tokens
            sc.num_cached_tokens += sc.num_new_tokens
            so.num_new_tokens = sc.num_new_tokens = 0
            if done_prefill:
                t = rng.randrange(151936)
                so.append_token(t)
                sc.append_token(t)
                g -= 1
                running[k] = (so, sc, g)
                if g <= 0:
                    p.call("deallocate", so, sc)
                    running.pop(k)
                    stats["finished"] += 1
    return p, stats


@pytest.mark.parametrize("seed,bs,nb", [(0, 4, 64), (1, 4, 24), (4, 4, 16), (5, 4, 14),
                                         (6, 16, 20), (2, 16, 96), (3, 256, 40)])
def test_scheduler_workload_matches_oracle(seed, bs, nb):
    _, stats = _workload(seed, bs, nb, steps=120, budget=6 * bs, max_seqs=8, prefixes=3)
    assert stats["finished"] > 0 and stats["hits"] > 0
    if nb <= 20:
        assert stats["preempted"] > 0  # a tight pool exercises preemption too


def test_workloads_reach_the_reference_assert():
    """The chunked-prefill defect (see test_reference_assert_on_short_first_chunk)
    is common under load: these seeded workloads reach it, and the C ABI
    refuses each of those calls exactly where the reference would panic."""
    panics = sum(_workload(seed, bs, nb, steps=120, budget=6 * bs, max_seqs=8,
                           prefixes=3)[1]["reference_panics"]
                 for seed, bs, nb in [(1, 4, 24), (4, 4, 16), (2, 16, 96)])
    assert panics >= 3


def test_reference_assert_on_short_first_chunk():
    """A reference defect, reproduced for parity.  A chunked prefill whose
    first chunk ends inside a full block that misses the cache: allocate
    registers that full block's hash on a page holding only the chunk
    (block_manager.rs:176-185), and the next may_append trips its
    `hash == -1` assert (block_manager.rs:239-241), which panics the
    reference's engine.  The C ABI refuses the same call and changes nothing."""
    bs = 4
    p = Pair(8, bs)
    toks = list(range(1, 11))
    so, sc = OB.Seq(toks, bs), Sequence(toks, bs)
    so.num_new_tokens = sc.num_new_tokens = 3
    p.call("allocate", so, sc)
    assert p.c.block_info(sc.block_table[0])[1] == compute_hash(toks[:4], -1)
    so.num_cached_tokens = sc.num_cached_tokens = 3
    so.num_new_tokens = sc.num_new_tokens = 7
    with pytest.raises(ReferencePanic):
        p.call("may_append", so, sc)


def test_prefix_hits_in_used_and_free_blocks():
    """Two sequences sharing a 2-block prefix: the second's prefix is cached
    in used blocks; after both finish, a third finds it in free blocks."""
    bs = 4
    p = Pair(16, bs)
    pre = [11, 12, 13, 14, 21, 22, 23, 24]
    seqs = []
    for tail in ([31, 32], [41, 42, 43]):
        so, sc = OB.Seq(pre + tail, bs), Sequence(pre + tail, bs)
        lay = p.call("get_token_layout", so, sc)
        so.num_new_tokens = sc.num_new_tokens = lay[2]
        p.call("allocate", so, sc)
        seqs.append((so, sc, lay))
    assert seqs[0][2] == (0, 0, 10) and seqs[1][2] == (8, 0, 3)
    assert seqs[1][0].block_table[:2] == seqs[0][0].block_table[:2]  # shared pages
    for so, sc, _ in seqs:
        so.num_cached_tokens += so.num_new_tokens
        sc.num_cached_tokens += sc.num_new_tokens
        so.num_new_tokens = sc.num_new_tokens = 0
        p.call("deallocate", so, sc)
    so, sc = OB.Seq(pre + [51], bs), Sequence(pre + [51], bs)
    lay = p.call("get_token_layout", so, sc)
    assert lay == (0, 8, 1)
    so.num_new_tokens = sc.num_new_tokens = 1
    p.call("allocate", so, sc)
    assert so.num_cached_tokens == 8


def test_decode_growth_hashes_full_blocks():
    """may_append over decode steps: a block gets its chain hash when it
    fills, and a new page is taken when the next token starts a block."""
    bs = 4
    p = Pair(8, bs)
    toks = [1, 2, 3, 4, 5, 6]
    so, sc = OB.Seq(toks, bs), Sequence(toks, bs)
    so.num_new_tokens = sc.num_new_tokens = 6
    p.call("allocate", so, sc)
    for step in range(7):
        so.num_cached_tokens += so.num_new_tokens
        sc.num_cached_tokens += sc.num_new_tokens
        so.append_token(100 + step)
        sc.append_token(100 + step)
        so.num_new_tokens = sc.num_new_tokens = 1
        assert p.call("can_append", so, sc, 1)
        p.call("may_append", so, sc)
    hashes = [p.c.block_info(b)[1] for b in sc.block_table]
    assert hashes[0] != -1 and hashes[1] != -1 and hashes[2] != -1 and hashes[3] == -1
    assert hashes[1] == compute_hash(sc.token_ids[4:8], hashes[0])


def test_errors_leave_state_unchanged():
    bs = 4
    bm = BlockManager(3, bs)
    s = Sequence(list(range(10)), bs)
    s.num_new_tokens = 10
    bm.allocate(s)  # 3 blocks, pool empty
    before = (bm.free_block_ids(), [bm.block_info(i) for i in range(3)])
    s2 = Sequence(list(range(100, 105)), bs)
    s2.num_new_tokens = 5
    with pytest.raises(NvkvError):
        bm.allocate(s2)  # no free block
    with pytest.raises(NvkvError):
        bm.allocate(s)  # block table not empty
    with pytest.raises(NvkvError):
        bm.get_token_layout(s)
    s.num_cached_tokens, s.num_new_tokens = 10, 0
    s.append_token(7)
    s.append_token(8)
    s.append_token(9)
    s.num_new_tokens = 3  # needs a fourth page
    assert not bm.can_append(s, 3)
    with pytest.raises(NvkvError):
        bm.may_append(s)
    assert (bm.free_block_ids(), [bm.block_info(i) for i in range(3)]) == before
    s.num_new_tokens = 0
    bm.deallocate(s)
    assert bm.num_free == 3
    stale = Sequence(list(range(10)), bs)
    stale.block_table = [0]
    with pytest.raises(NvkvError):
        bm.deallocate(stale)  # ref count would go below zero
    assert bm.num_free == 3


def test_append_batch_matches_per_sequence_calls():
    """append_batch = can_append then may_append per sequence, in order,
    stopping at the first that does not fit."""
    bs = 4
    rng = random.Random(9)
    o, c = OB.BlockManager(20, bs), BlockManager(20, bs)
    so_l, sc_l = [], []
    for k in range(5):
        toks = [rng.randrange(1000) for _ in range(rng.randrange(3, 9))]
        so, sc = OB.Seq(toks, bs), Sequence(toks, bs)
        so.num_new_tokens = sc.num_new_tokens = len(toks)
        o.allocate(so)
        c.allocate(sc)
        so.num_cached_tokens = sc.num_cached_tokens = len(toks)
        so.num_new_tokens = sc.num_new_tokens = 0
        so_l.append(so)
        sc_l.append(sc)
    for step in range(30):
        want = [rng.choice([1, 1, 1, 5]) for _ in so_l]
        for so, sc, n in zip(so_l, sc_l, want):
            for _ in range(n):
                t = rng.randrange(1000)
                so.append_token(t)
                sc.append_token(t)
        done_o = 0
        for so, n in zip(so_l, want):
            if not o.can_append(so, n):
                break
            so.num_new_tokens = n
            o.may_append(so)
            done_o += 1
        done_c = c.append_batch(sc_l, want)
        assert done_o == done_c
        for so, sc in zip(so_l, sc_l):
            assert so.block_table == sc.block_table and so.num_new_tokens == sc.num_new_tokens
        assert _state(o, 20) == _state(c, 20)
        if done_c < len(sc_l):  # the pool is full: finish the tail sequences
            for so, sc in zip(so_l[done_c:], sc_l[done_c:]):
                so.num_new_tokens = sc.num_new_tokens = 0
                o.deallocate(so)
                c.deallocate(sc)
            del so_l[done_c:], sc_l[done_c:]
            if not so_l:
                break
        for so, sc in zip(so_l, sc_l):
            so.num_cached_tokens += so.num_new_tokens
            sc.num_cached_tokens += sc.num_new_tokens
            so.num_new_tokens = sc.num_new_tokens = 0


def test_create_validation():
    with pytest.raises(NvkvError):
        BlockManager(0, 4)
    with pytest.raises(NvkvError):
        BlockManager(4, 0)
