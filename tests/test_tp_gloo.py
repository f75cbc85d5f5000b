"""Tensor-parallel layout of the decoder around the path, world_size 2 on CPU
(gloo): sharded projections + all-reduce / all-gather reproduce the unsharded
computation (layers/linear.rs, layers/embed_head.rs, dist_util.rs)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from nvkv.decoder import (gather_logits, shard_merged, shard_qkv, shard_row, shard_vocab,
                                  vocab_parallel_argmax, vocab_parallel_embed)
        g = torch.Generator().manual_seed(0)
        H, hq, hkv, D, F, V, T = 64, 4, 2, 8, 48, 40, 5
        x = torch.randn(T, H, generator=g, dtype=torch.float64)
        wq = torch.randn(hq * D, H, generator=g, dtype=torch.float64)
        wk = torch.randn(hkv * D, H, generator=g, dtype=torch.float64)
        wv = torch.randn(hkv * D, H, generator=g, dtype=torch.float64)
        wo = torch.randn(H, hq * D, generator=g, dtype=torch.float64)
        wg = torch.randn(F, H, generator=g, dtype=torch.float64)
        wu = torch.randn(F, H, generator=g, dtype=torch.float64)
        wd = torch.randn(H, F, generator=g, dtype=torch.float64)
        emb = torch.randn(V, H, generator=g, dtype=torch.float64)
        ids = torch.tensor([0, 19, 20, 39, 7])

        # column-parallel qkv: local [q_r; k_r; v_r] rows (linear.rs:253-280)
        qkv_l = x @ shard_qkv(wq, wk, wv, rank, world).T
        q_full, k_full, v_full = x @ wq.T, x @ wk.T, x @ wv.T
        ql, kl = hq * D // world, hkv * D // world
        assert torch.allclose(qkv_l[:, :ql], q_full[:, rank * ql:(rank + 1) * ql])
        assert torch.allclose(qkv_l[:, ql:ql + kl], k_full[:, rank * kl:(rank + 1) * kl])
        assert torch.allclose(qkv_l[:, ql + kl:], v_full[:, rank * kl:(rank + 1) * kl])
        # row-parallel o_proj + all-reduce (linear.rs:187-211)
        o_part = q_full[:, rank * ql:(rank + 1) * ql] @ shard_row(wo, rank, world).T
        dist.all_reduce(o_part)
        assert torch.allclose(o_part, q_full @ wo.T)
        # merged gate_up [gate_r; up_r] + row-parallel down (linear.rs:109-151)
        gu = x @ shard_merged([wg, wu], rank, world).T
        Fl = F // world
        act = torch.nn.functional.silu(gu[:, :Fl]) * gu[:, Fl:]
        d = act @ shard_row(wd, rank, world).T
        dist.all_reduce(d)
        ref = (torch.nn.functional.silu(x @ wg.T) * (x @ wu.T)) @ wd.T
        assert torch.allclose(d, ref)
        # vocab-parallel embedding: masked lookup + all-reduce (embed_head.rs:47-60)
        e = vocab_parallel_embed(ids, shard_vocab(emb, rank, world), rank)
        assert torch.allclose(e, emb[ids])
        # vocab-parallel lm_head: local logits + all-gather concat (embed_head.rs:113-117)
        lg = gather_logits(x @ shard_vocab(emb, rank, world).T)
        assert torch.allclose(lg, x @ emb.T)
        # vocab-parallel greedy pick == argmax of the gathered logits, also on
        # ties inside a shard and across the shard boundary (first index wins)
        full = (x @ emb.T).float()
        full[1, 3] = full[1, 30] = full[1].max() + 1.0   # tie across shards
        full[2, 25] = full[2, 27] = full[2].max() + 1.0  # tie inside shard 1
        full[3, :] = 0.5                                  # all equal
        local = full[:, rank * (V // world):(rank + 1) * (V // world)]
        assert torch.equal(vocab_parallel_argmax(local, rank), full.argmax(-1))
        q.put((rank, "ok"))
    except Exception as ex:  # pragma: no cover - reported to the parent
        q.put((rank, repr(ex)))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def test_tp2_layout_matches_unsharded():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=240) for _ in procs)
    for p in procs:
        p.join(60)
    assert res == {0: "ok", 1: "ok"}, res


def test_divide_rejects_uneven_heads():
    from nvkv.decoder import divide
    assert divide(32, 8) == 4
    with pytest.raises(ValueError):
        divide(8, 3)


def _pool_worker(rank, world, port, q):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from nvkv.blocks import kv_pool_reconcile
        got = kv_pool_reconcile([900, 750][rank], dist.group.WORLD)
        q.put((rank, got))
    except Exception as ex:  # pragma: no cover - reported through the queue
        q.put((rank, repr(ex)))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def test_kv_pool_budget_is_the_minimum_over_ranks():
    """Every rank allocates the same pool: the smallest rank budget
    (model_runner.rs:265-266), reconciled over the process group."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_pool_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=240) for _ in procs)
    for p in procs:
        p.join(60)
    assert res == {0: 750, 1: 750}, res
