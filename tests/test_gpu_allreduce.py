"""nvkv_allreduce_rms_norm (all-reduce + residual + RMSNorm over NVLink peer
memory) against torch.distributed's NCCL all-reduce followed by
nvkv_rms_norm on the same inputs.

One GPU: a world-1 communicator (the sum is the input itself), which must
give nvkv_rms_norm's bits exactly, eagerly and under CUDA-graph replay.
Two or more GPUs (skipped otherwise): one spawned process per GPU.  At
every world size the result must equal, bit for bit, the exact reference:
all partials gathered, summed in fp32 in rank order, rounded once, then
nvkv_rms_norm (bench.allreduce_reference).  Against NCCL: at world 2 the sum
of two bf16 values rounded once is what NCCL computes too, so results must be
bit-identical; at larger worlds NCCL's ring rounds at every hop, so the
residual sum may differ by up to world bf16 ulps of sum |partials| +
|residual|.  A timeout case lets one rank skip the call: the other
rank's bounded waits must expire into NVKV_DEVERR_PEER_TIMEOUT with its
context still usable.
"""
import os
import socket

import pytest
import torch

import nvkv
from nvkv import ops
from nvkv._lib import DEVERR_PEER_TIMEOUT

pytestmark = pytest.mark.gpu


def _inputs(T, H, seed, dev="cuda"):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16).to(dev)
    r = torch.randn(T, H, generator=g).to(torch.bfloat16).to(dev)
    w = (1 + 0.1 * torch.randn(H, generator=g)).to(torch.bfloat16).to(dev)
    return x, r, w


def test_world1_matches_rms_norm_bitwise():
    from nvkv.comm import PeerComm
    comm = PeerComm(0, 1, 1024 * 4096 * 2)
    try:
        for T, H in ((1, 4096), (37, 4096), (300, 5120), (1024, 4096), (5, 1024)):
            x, r, w = _inputs(T, H, T + H)
            comm.input(T, H).copy_(x)
            res, out = r.clone(), torch.empty_like(x)
            comm.allreduce_rms_norm(T, H, res, w, 1e-6, out)
            res_ref = r.clone()
            out_ref = ops.rms_norm(x, w, 1e-6, residual=res_ref)
            torch.cuda.synchronize()
            assert torch.equal(res, res_ref) and torch.equal(out, out_ref), (T, H)
            res2, out2 = torch.empty_like(x), torch.empty_like(x)
            comm.allreduce_rms_norm(T, H, res2, w, 1e-6, out2, init=True)
            torch.cuda.synchronize()
            assert torch.equal(res2, x) and torch.equal(out2, ops.rms_norm(x, w, 1e-6)), (T, H)
        assert nvkv.device_error() == 0
    finally:
        torch.cuda.synchronize()
        comm.close()


def test_world1_graph_replays():
    from nvkv.comm import PeerComm
    T, H = 256, 4096
    comm = PeerComm(0, 1, T * H * 2)
    try:
        x, r, w = _inputs(T, H, 3)
        res, out = r.clone(), torch.empty_like(x)
        inp = comm.input(T, H)

        def step():
            inp.copy_(x)
            comm.allreduce_rms_norm(T, H, res, w, 1e-6, out)

        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            step()
        torch.cuda.current_stream().wait_stream(s)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step()
        ref_res = r.clone()
        ops.rms_norm(x, w, 1e-6, residual=ref_res)  # the warm-up call
        for _ in range(4):
            graph.replay()
            ref_out = ops.rms_norm(x, w, 1e-6, residual=ref_res)
            torch.cuda.synchronize()
            assert torch.equal(res, ref_res) and torch.equal(out, ref_out)
        graph.reset()
        assert nvkv.device_error() == 0
    finally:
        torch.cuda.synchronize()
        comm.close()


# ---------------------------------------------------------------------------
# multi-GPU: one process per GPU
# ---------------------------------------------------------------------------

def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, mode, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        import datetime

        import torch.distributed as dist
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                timeout=datetime.timedelta(seconds=60))
        import sys
        sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
        import bench
        from nvkv.comm import PeerComm
        comm = PeerComm(rank, world, 1024 * 5120 * 2, timeout_s=0.2 if mode == "timeout" else None)
        if mode == "timeout":
            T, H = 64, 4096
            x, r, w = _inputs(T, H, 1, dev)
            dist.barrier()
            if rank == 0:  # rank 1 never calls: rank 0's waits must run out
                comm.input(T, H).copy_(x)
                comm.allreduce_rms_norm(T, H, r.clone(), w, 1e-6, torch.empty_like(x))
                torch.cuda.synchronize()
                code = nvkv.device_error()
                assert code == DEVERR_PEER_TIMEOUT, code
                y = ops.rms_norm(x, w, 1e-6)  # the context is still usable
                torch.cuda.synchronize()
                assert torch.isfinite(y.float()).all()
            dist.barrier()
        else:
            for T, H in ((256, 4096), (37, 4096), (1, 4096), (0, 4096), (700, 5120), (64, 1024)):
                x, r, w = _inputs(T, H, 100 + T)  # identical residual / weight on all ranks
                part = (torch.randn(T, H, generator=torch.Generator().manual_seed(rank * 7 + T))
                        .to(torch.bfloat16).to(dev))
                r, w = r.to(dev), w.to(dev)
                comm.input(T, H).copy_(part)
                res, out = r.clone(), torch.empty(T, H, dtype=torch.bfloat16, device=dev)
                comm.allreduce_rms_norm(T, H, res, w, 1e-6, out)
                parts = [torch.empty_like(part) for _ in range(world)]
                dist.all_gather(parts, part)
                ref = part.clone()
                dist.all_reduce(ref)
                res_ref = r.clone()
                out_ref = ops.rms_norm(ref, w, 1e-6, residual=res_ref) if T else ref
                torch.cuda.synchronize()
                if T:
                    res_e, out_e, bound = bench.allreduce_reference(parts, r, w, 1e-6, world)
                    assert torch.equal(res, res_e) and torch.equal(out, out_e), (T, H)
                if world == 2:
                    assert torch.equal(res, res_ref) and torch.equal(out, out_ref), (T, H)
                elif T:
                    assert ((res.float() - res_ref.float()).abs() <= bound).all(), (T, H)
            # graph replays keep the device epochs of all ranks in lockstep
            T, H = 256, 4096
            part = torch.randn(T, H, generator=torch.Generator().manual_seed(rank)).to(
                torch.bfloat16).to(dev)
            x, r, w = _inputs(T, H, 5, dev)
            res, out = r.clone(), torch.empty_like(x)
            inp = comm.input(T, H)

            def step():
                inp.copy_(part)
                comm.allreduce_rms_norm(T, H, res, w, 1e-6, out)

            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):
                step()
            torch.cuda.current_stream().wait_stream(s)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                step()
            ref = part.clone()
            dist.all_reduce(ref)
            res_ref = r.clone()
            ops.rms_norm(ref, w, 1e-6, residual=res_ref)
            for _ in range(3):
                graph.replay()
                out_ref = ops.rms_norm(ref, w, 1e-6, residual=res_ref)
                torch.cuda.synchronize()
                if world == 2:
                    assert torch.equal(res, res_ref) and torch.equal(out, out_ref)
            graph.reset()
            assert nvkv.device_error() == 0
        torch.cuda.synchronize()
        dist.barrier()
        comm.close()
        q.put((rank, "ok"))
    except Exception as ex:  # pragma: no cover - reported to the parent
        q.put((rank, repr(ex)))
    finally:
        import torch.distributed as dist
        if dist.is_initialized():
            dist.destroy_process_group()


def _run(world, mode):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(60)
    assert res == {r: "ok" for r in range(world)}, res


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_ranks_match_nccl_bitwise():
    _run(2, "parity")


@pytest.mark.skipif(torch.cuda.device_count() < 4, reason="needs 4 GPUs")
def test_four_ranks_match_nccl():
    _run(4, "parity")


@pytest.mark.skipif(torch.cuda.device_count() < 8, reason="needs 8 GPUs")
def test_eight_ranks_match_nccl():
    _run(8, "parity")


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_missing_rank_times_out_into_an_error():
    _run(2, "timeout")
