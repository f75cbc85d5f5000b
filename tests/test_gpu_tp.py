"""Tensor-parallel model steps (TP=2 and TP=4, one process per GPU) against
TP=1 on the same seeded weights: the check bench.py runs before its numbers
at every N > 1 (bench.tp_parity), here as a test.

Each rank builds a 2-layer slice of the Qwen3-8B shape sharded over the
ranks (column-parallel qkv / gate_up, row-parallel o_proj / down_proj with
their all-reduces, vocab-parallel embedding and lm_head) and the same slice
unsharded, runs four prompts through one prefill step and greedy decode
steps fed with the TP=1 tokens, and requires:
  * the TP=N greedy token equal to TP=1's at >= 95 % of positions;
  * the fused all-reduce + residual + RMSNorm bit-identical to the exact
    reference (partials summed in fp32 in rank order, rounded once, then
    nvkv_rms_norm) at every TP, and to NCCL's all-reduce + nvkv_rms_norm at
    TP2 (within world bf16 ulps of sum |partials| + |residual| at TP4, where
    NCCL's ring rounds at every hop).
Both all-reduce routes of the model are run: the nvkv peer-memory kernel and
NCCL.

The greedy-stream gate of tests/test_gpu_greedy.py also runs at TP2: the
config-1 model sharded over two GPUs against the CPU restatement of the
reference (bf16 rounding points) built from the same weights, with the same
bars (test_gpu_greedy.passes: teacher forced, and the GPU's free-running
stream checked by the reference, each >= 95 % of positions counting bf16
near-ties; exact teacher-forced agreement >= 90 %).

Skipped with fewer GPUs than ranks.  NVLS is off (NCCL_NVLS_ENABLE=0).
"""
import os
import socket
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, route, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        sys.path[:0] = [ROOT, os.path.join(ROOT, "nanovllm-rs_b200")]
        import datetime

        import torch.distributed as dist
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                timeout=datetime.timedelta(seconds=60))
        import bench
        import nvkv
        from nvkv.comm import PeerComm
        from qwen3_config import QWEN3_8B
        if route == "greedy":
            msg = _greedy_tp(rank, world, dev)
        else:
            T = 256
            comm = PeerComm(rank, world, T * QWEN3_8B.hidden_size * 2) if route == "peer" else None
            res = bench.tp_parity(QWEN3_8B, comm, world, rank, dev, T=T, layers=2)
            torch.cuda.synchronize()
            assert nvkv.device_error() == 0
            dist.barrier()
            if comm is not None:
                comm.close()
            msg = "ok" if res["ok"] else repr(res)
        q.put((rank, msg))
    except Exception as ex:  # pragma: no cover - reported to the parent
        q.put((rank, repr(ex)))
    finally:
        import torch.distributed as dist
        if dist.is_initialized():
            dist.destroy_process_group()


def _greedy_tp(rank, world, dev):
    """The config-1 greedy gate with the model at TP=world.  Rank 0 alone
    runs the CPU reference and hands its stream to the other ranks over a
    gloo group with a long timeout (the NCCL group's short one would expire
    while rank 0 computes)."""
    import datetime

    import torch.distributed as dist

    import nvkv
    import test_gpu_greedy as G
    from nvkv.decoder import Qwen3TP
    cpu = dist.new_group(backend="gloo", timeout=datetime.timedelta(seconds=900))

    def share(obj):
        box = [obj]
        dist.broadcast_object_list(box, src=0, group=cpu)
        return box[0]

    w = None
    if rank == 0:
        full = Qwen3TP(G.CFG, 0, 1, seed=3, device=dev, **G.INIT)  # the TP1 weights
        w = G.to_numpy_weights(full)
        del full
    model = Qwen3TP(G.CFG, rank, world, seed=3, device=dev, **G.INIT)
    report = G.gate(model, w, root=rank == 0, share=share)
    torch.cuda.synchronize()
    assert nvkv.device_error() == 0
    ok = share(None if rank else G.passes(report))
    dist.barrier(group=cpu)
    model.close()
    if rank == 0:
        print("TP%d greedy agreement" % world, report)
    return "ok" if ok else repr(report)


def _run(world, route):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, route, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=600) for _ in procs)
    for p in procs:
        p.join(60)
    assert res == {r: "ok" for r in range(world)}, res


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("route", ["peer", "nccl"])
def test_tp2_matches_tp1(route):
    _run(2, route)


@pytest.mark.skipif(torch.cuda.device_count() < 4, reason="needs 4 GPUs")
def test_tp4_matches_tp1():
    _run(4, "peer")


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp2_greedy_streams_match_cpu_reference():
    _run(2, "greedy")
