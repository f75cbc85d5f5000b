"""Benchmark: Qwen3-8B bf16 continuous-batching decode step through the nvkv
hot path, tensor-parallel over N GPUs (one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl nvkv|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...

Workload (benchmark config 4, Qwen3-8B shapes, random-init weights): 256
running sequences whose 1024-token prompts are already prefilled and which are
mid-generation, so their contexts are drawn (seeded) uniform in [1025, 1536];
one step decodes one token for every sequence through all 36 layers:
embedding -> 36 x [RMSNorm, qkv GEMM, nvkv_qknorm_rope (+KV store),
nvkv_paged_attention (split-KV decode), o_proj GEMM (+all-reduce), RMSNorm,
gate_up GEMM, SiLU*mul, down GEMM (+all-reduce)] -> norm -> lm_head
(+all-gather) -> argmax.  The per-step KV read (~48 GB at TP1) is far larger
than L2, so no flush is needed between steps.

One JSON line is printed by rank 0 (see the keys in main()).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "nanovllm-rs_b200"))

METRIC = "decode tok/s Qwen3-8B bf16 at TP1/2/4/8; paged-attn HBM GB/s vs 8 TB/s"
NUM_SEQS = 256
PROMPT = 1024
MAX_OUT = 512
PAGE = 256
SEED = 1234


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="nvkv", choices=["nvkv", "reference"])
    ap.add_argument("--no-graph", action="store_true", help="eager launches (no CUDA graph)")
    ap.add_argument("--nccl-allreduce", action="store_true",
                    help="tp > 1: NCCL all-reduce + nvkv_rms_norm instead of the fused "
                         "peer-memory nvkv_allreduce_rms_norm")
    ap.add_argument("--no-workloads", action="store_true",
                    help="skip the whole-workload runs (configs 4, 3, 1, 5) after the timed step")
    ap.add_argument("--layers", type=int, default=None, help=argparse.SUPPRESS)
    return ap.parse_args()


def bench_config(world, cuda_graph=True, nccl_allreduce=False):
    """The `config` object of both arms' JSON lines (the same workload)."""
    return {
        "workload": "Qwen3-8B decode step, 256 seqs, ctx U[1025,1536], P=256, all 36 layers + "
                    "lm_head + vocab-parallel argmax; attention path = nvkv kernels, GEMMs = "
                    "cuBLAS, TP all-reduce + RMSNorm = nvkv peer-memory kernel (NCCL with "
                    "--nccl-allreduce), greedy-pick all-gather = NCCL",
        "model": "Qwen3-8B", "global_batch": NUM_SEQS, "seq_len": PROMPT + MAX_OUT,
        "parallelism": f"tp{world}", "cuda_graph": bool(cuda_graph),
        "allreduce_route": ("none" if world == 1 else
                            "nccl + nvkv_rms_norm" if nccl_allreduce else "nvkv_allreduce_rms_norm"),
        "l2": "inputs larger than L2 (per-step KV read >> 126 MB), no flush",
    }


def workload(seed=SEED):
    """Seeded decode-step metadata, built like ModelRunner::prepare_model_input
    (model_runner.rs:82-131) for 256 sequences each decoding one token."""
    rng = np.random.default_rng(seed)
    ctx = rng.integers(PROMPT + 1, PROMPT + MAX_OUT + 1, NUM_SEQS)  # context incl. new token
    nblk = (ctx + PAGE - 1) // PAGE
    num_blocks = int(nblk.sum()) + 8
    perm = rng.permutation(num_blocks)
    width = int(nblk.max())
    bt = np.zeros((NUM_SEQS, width), np.int32)
    used = 0
    for i, n in enumerate(nblk):
        bt[i, :n] = perm[used:used + n]
        used += n
    pos = ctx - 1
    slots = bt[np.arange(NUM_SEQS), pos // PAGE].astype(np.int64) * PAGE + pos % PAGE
    return dict(ctx=ctx, block_tables=bt, num_blocks=num_blocks, positions=pos.astype(np.int64),
                slot_mapping=slots, input_ids=rng.integers(0, 151936, NUM_SEQS).astype(np.int64),
                cu_q=np.arange(NUM_SEQS + 1, dtype=np.int32),
                cu_k=np.concatenate([[0], np.cumsum(ctx)]).astype(np.int32),
                max_k=int(ctx.max()))


def decode_bytes(w, hq, hkv, D=128):
    """Algorithmic HBM bytes of one decode-attention launch (one layer):
    K+V rows of every context, q and out rows, block-table entries, cu_seqlens."""
    kv = int(w["ctx"].sum()) * hkv * D * 2 * 2
    qo = 2 * NUM_SEQS * hq * D * 2
    meta = 4 * int(((w["ctx"] + PAGE - 1) // PAGE).sum()) + 2 * 4 * (NUM_SEQS + 1)
    return kv + qo + meta


# DRAM bytes per algorithmic byte of the decode attention kernel, from one
# ncu capture of the identical per-layer shape (B=256, 32q/8kv, ctx
# U[1025,1536]; profiles/paged_decode_qwen3-8b-tp1-layer.md):
# (1,386,555,000 read + 7,612,672 written) / 1,355,329,068 algorithmic.
DECODE_DRAM_PER_ALG_BYTE = (1386555000 + 7612672) / 1355329068


def load_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        return float(json.load(open(p))["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled during the timed region."""

    Q = ("pci.bus_id,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, bus_id):
        self.bus = bus_id.lower()
        self.proc = None
        self.path = os.path.join("/tmp", f"nvkv_clocks_{os.getpid()}.csv")

    def start(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(5)
        except Exception:
            self.proc.kill()
        self.f.close()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            f = [x.strip() for x in line.split(",")]
            if len(f) < 8 or f[0].lower() != self.bus:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[4:8]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "samples": len(sm),
                "reasons": sorted(reasons)}


def _dist_setup():
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))
    return rank, world, dev


def _max_over_ranks(x, world, dev):
    import torch
    import torch.distributed as dist
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _barrier(world):
    import torch
    import torch.distributed as dist
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()


def _allreduce_bw(world, dev, nbytes, reps=50):
    """NCCL all-reduce of the step's own message (T x hidden bf16), `reps`
    calls captured in one CUDA graph as in the step, timed with CUDA events,
    max over ranks.  Bus bandwidth as nccl-tests defines it:
    algbw * 2 (n - 1) / n."""
    import torch
    import torch.distributed as dist
    x = torch.zeros(nbytes // 2, dtype=torch.bfloat16, device=dev)
    for _ in range(3):
        dist.all_reduce(x)
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        dist.all_reduce(x)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(reps):
            dist.all_reduce(x)
    g.replay()
    torch.cuda.synchronize()
    _barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    g.replay()
    e1.record()
    torch.cuda.synchronize()
    ms = _max_over_ranks(e0.elapsed_time(e1), world, dev) / reps
    g.reset()  # a graph holding NCCL calls must go before the process group
    torch.cuda.synchronize()
    algbw = nbytes / (ms * 1e-3) / 1e9
    return ms, algbw, algbw * 2 * (world - 1) / world


def _peer_allreduce_bw(model, world, dev, T, reps=50):
    """The fused nvkv_allreduce_rms_norm on the step's shape (T x hidden bf16),
    `reps` calls in one CUDA graph, CUDA events, max over ranks; bus bandwidth
    on the all-reduce's bytes as for NCCL."""
    import torch
    H = model.cfg.hidden_size
    res = torch.zeros(T, H, dtype=model.dtype, device=dev)
    out = torch.empty_like(res)
    w = model.norm
    model.comm.input(T, H, model.dtype).zero_()
    for _ in range(3):
        model.comm.allreduce_rms_norm(T, H, res, w, 1e-6, out)
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        model.comm.allreduce_rms_norm(T, H, res, w, 1e-6, out)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(reps):
            model.comm.allreduce_rms_norm(T, H, res, w, 1e-6, out)
    g.replay()
    torch.cuda.synchronize()
    _barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    g.replay()
    e1.record()
    torch.cuda.synchronize()
    ms = _max_over_ranks(e0.elapsed_time(e1), world, dev) / reps
    g.reset()
    torch.cuda.synchronize()
    nbytes = T * H * 2
    algbw = nbytes / (ms * 1e-3) / 1e9
    return ms, algbw, algbw * 2 * (world - 1) / world


def _bf16_ulps(a, b):
    """Largest distance between two bf16 tensors in units in the last place
    (sign-magnitude bit patterns mapped onto one ordered integer line)."""
    import torch

    def line(t):
        i = t.contiguous().view(torch.int16).to(torch.int32)
        return torch.where(i < 0, -(i & 0x7FFF), i)

    return int((line(a) - line(b)).abs().max()) if a.numel() else 0


def allreduce_reference(parts, residual, w, eps, world):
    """The fused all-reduce + residual + RMSNorm computed the kernel's way:
    the gathered partials summed in fp32 in rank order and rounded once to
    their dtype, then nvkv_rms_norm with the residual.  Returns (residual
    out, out, NCCL bound), the bound being world bf16 ulps of sum_q
    |partial_q| + |residual| (the error NCCL's per-hop rounding can reach)."""
    import torch

    from nvkv import ops
    acc = parts[0].float()
    mag = parts[0].float().abs()
    for q in range(1, len(parts)):
        acc = acc + parts[q].float()
        mag = mag + parts[q].float().abs()
    res = residual.clone()
    out = ops.rms_norm(acc.to(parts[0].dtype), w, eps, residual=res)
    mag = mag + residual.float().abs()
    ulp = torch.exp2(torch.floor(torch.log2(mag.clamp_min(2.0 ** -100))) - 7)
    return res, out, world * ulp


def tp_parity(cfg, comm, world, rank, dev, T=NUM_SEQS, layers=4, num_seqs=4, steps=12, seed=17,
              dtype=None):
    """Correctness of the tensor-parallel step on this run's own ranks, before
    its numbers are trusted.  Every rank takes the same collective calls.

    * allreduce_vs_nccl: the step's fused all-reduce + residual + RMSNorm
      (nvkv_allreduce_rms_norm through `comm`, when the step uses it; comm
      None is the NCCL route) on the same [T, hidden] inputs against
      (a) the exact reference -- every rank's partial gathered, summed in
      fp32 in rank order and rounded once, then nvkv_rms_norm -- bit for bit
      at every world size (the kernel's own arithmetic), and (b) NCCL's
      all-reduce followed by nvkv_rms_norm: bit-identical at TP2 (one
      rounding of a two-term sum on both routes); at TP4/8 NCCL's ring
      rounds at every hop, so the difference is bounded by world_size bf16
      ulps of sum_q |partial_q| + |residual| (cancellation makes ulps of
      the result itself meaningless near zero).
    * greedy_vs_tp1: a `layers`-layer slice of the same Qwen3 shape built at
      TP=N (sharded over the ranks, the step's all-reduce route) and at TP=1
      (every rank builds the whole slice from the same seeds), `num_seqs`
      prompts of U[32, 64] random tokens, one prefill step then greedy decode
      steps, teacher forced with the TP=1 tokens; the TP=N greedy token must
      equal TP=1's at >= 95 % of positions (the north star's bar), and the
      prefill logits' max-abs difference is reported.
    Step metadata comes from nvkv's own prepare_step (the C ABI)."""
    import torch
    import torch.distributed as dist
    from dataclasses import replace

    from nvkv import ops
    from nvkv.blocks import Sequence, prepare_step
    from nvkv.decoder import Qwen3TP, Step

    dtype = dtype or torch.bfloat16
    res = {}
    eps = cfg.rms_norm_eps
    H = cfg.hidden_size
    if comm is not None:
        g = torch.Generator(device=dev).manual_seed(1000 + rank)
        x = torch.randn(T, H, generator=g, device=dev).to(dtype)
        g0 = torch.Generator(device=dev).manual_seed(999)  # replicated: residual, weight
        r0 = torch.randn(T, H, generator=g0, device=dev).to(dtype)
        wn = (1 + 0.1 * torch.randn(H, generator=g0, device=dev)).to(dtype)
        comm.input(T, H, dtype).copy_(x)
        res_a, out_a = r0.clone(), torch.empty_like(r0)
        comm.allreduce_rms_norm(T, H, res_a, wn, eps, out_a)
        parts = [torch.empty_like(x) for _ in range(world)]
        dist.all_gather(parts, x)
        res_e, out_e, bound = allreduce_reference(parts, r0, wn, eps, world)
        xs = x.clone()
        dist.all_reduce(xs)
        res_b = r0.clone()
        out_b = ops.rms_norm(xs, wn, eps, residual=res_b)
        torch.cuda.synchronize()
        exact = int(not (torch.equal(res_a, res_e) and torch.equal(out_a, out_e)))
        nccl = float(((res_a.float() - res_b.float()).abs() / bound).max())
        stats = torch.tensor([exact, _bf16_ulps(res_a, res_b), _bf16_ulps(out_a, out_b),
                              float((out_a.float() - out_b.float()).abs().max()), nccl],
                             dtype=torch.float64, device=dev)
        dist.all_reduce(stats, op=dist.ReduceOp.MAX)
        ex, su, ou, od, nr = [float(v) for v in stats.tolist()]
        ok = ex == 0 and ((su == 0 and ou == 0) if world == 2 else nr <= 1.0)
        res["allreduce_vs_nccl"] = {
            "shape": [T, H], "exact_reference_bitwise": ex == 0, "sum_max_ulps": int(su),
            "out_max_ulps": int(ou), "out_max_abs": od,
            "nccl_sum_diff_over_bound": round(nr, 4),
            "bar": ("bitwise vs the exact reference and vs NCCL" if world == 2 else
                    "bitwise vs the exact reference; NCCL within world bf16 ulps of "
                    "sum |partials| + |residual|"),
            "ok": bool(ok)}
    cfg = replace(cfg, num_hidden_layers=layers)
    kw = dict(seed=seed, device=dev, embed_std=0.05, head_std=1.0, dtype=dtype)
    m_n = Qwen3TP(cfg, rank, world, comm=comm, peer_allreduce=comm is not None, max_tokens=T,
                  **kw)
    m_1 = Qwen3TP(cfg, 0, 1, **kw)
    P = PAGE
    rng = np.random.default_rng(seed)
    seqs = [Sequence(rng.integers(0, cfg.vocab_size, int(L)).tolist(), P)
            for L in rng.integers(32, 65, num_seqs)]
    for i, sq in enumerate(seqs):
        sq.block_table = [i]  # one page holds prompt + steps (<= 64 + 12 tokens)
    for m in (m_n, m_1):
        m.allocate_kv_cache(num_seqs, P)
    agree, total, logit_diff = 0, 0, 0.0
    for step in range(steps):
        for sq in seqs:
            sq.num_new_tokens = len(sq) - sq.num_cached_tokens
        meta = prepare_step(seqs, P)
        bt = np.asarray([sq.block_table for sq in seqs], np.int32)
        t = lambda a, dt=None: torch.from_numpy(np.ascontiguousarray(a)).to(dev)  # noqa: E731
        cu_q = t(meta["cu_seqlens_q"].view(np.int32))
        st = Step(t(meta["input_ids"]), t(meta["positions"]), t(meta["slot_mapping"]), cu_q,
                  t(meta["cu_seqlens_k"].view(np.int32)), t(bt), (cu_q[1:] - 1).long(),
                  meta["max_seqlen_q"], meta["max_seqlen_k"])
        if step == 0:
            ln, l1 = m_n.forward(st), m_1.forward(st)
            logit_diff = float((ln.float() - l1.float()).abs().max())
            tok_n, tok_1 = ln.argmax(-1), l1.argmax(-1)
        else:
            tok_n, tok_1 = m_n.greedy(st), m_1.greedy(st)
        agree += int((tok_n == tok_1).sum())
        total += num_seqs
        for sq, tk in zip(seqs, tok_1.tolist()):  # teacher forced: the TP=1 token
            sq.num_cached_tokens += sq.num_new_tokens
            sq.num_new_tokens = 0
            sq.append_token(tk)
    torch.cuda.synchronize()
    stats = torch.tensor([-agree / total, logit_diff], dtype=torch.float64, device=dev)
    dist.all_reduce(stats, op=dist.ReduceOp.MAX)  # worst rank
    frac = -float(stats[0])
    res["greedy_vs_tp1"] = {"layers": layers, "seqs": num_seqs, "positions": total,
                            "agree": round(frac, 4), "prefill_logits_max_abs": float(stats[1]),
                            "bar": ">= 0.95 of positions", "ok": frac >= 0.95}
    res["ok"] = all(v["ok"] for v in res.values() if isinstance(v, dict))
    m_n.close()
    del m_n, m_1
    torch.cuda.empty_cache()
    return res


MAX_BATCHED = 16384  # EngineConfig default max_num_batched_tokens (config.rs:110-120)


def _timing_max(summary, world, dev):
    """Worst rank's host times, and the rates recomputed from them."""
    for k in ("prefill_s", "decode_s", "total_s"):
        summary[k] = round(_max_over_ranks(summary[k], world, dev), 4)
    summary["prompt_tok_s"] = round(summary["prompt_tokens"] / max(summary["prefill_s"], 1e-9), 1)
    summary["decode_tok_s"] = round(summary["decode_tokens"] / max(summary["decode_s"], 1e-9), 1)
    summary["output_tok_s"] = round(summary["generated_tokens"] / max(summary["total_s"], 1e-9), 1)
    return summary


def run_workload(model, world, dev, prompts, max_tokens, num_blocks, warm_prompts=None,
                 kv_fp8=False):
    """Every prompt to completion through nvkv.engine (the reference's engine
    loop and scheduler defaults, greedy), on a fresh KV pool of `num_blocks`
    pages (the fp8 pool with kv_fp8); host-clock step times (schedule +
    metadata + H2D + model + D2H of the tokens), worst rank.  `warm_prompts`
    run first, untimed, so library warm-up (cuBLAS heuristics for the step
    shapes) stays out of the timing."""
    import torch

    from nvkv.engine import Engine

    model.k_caches, model.v_caches = [], []
    torch.cuda.empty_cache()
    model.allocate_kv_cache(num_blocks, PAGE, kv_fp8=kv_fp8)
    if warm_prompts:
        eng = Engine(model, num_blocks, PAGE, max_num_batched_tokens=MAX_BATCHED)
        eng.generate(warm_prompts, 2)
        eng.close()
    eng = Engine(model, num_blocks, PAGE, max_num_batched_tokens=MAX_BATCHED)
    _barrier(world)
    outs = eng.generate(prompts, max_tokens)
    torch.cuda.synchronize()
    summary = _timing_max(eng.summary(), world, dev)
    eng.close()
    summary["kv_pool_blocks"] = num_blocks
    model.k_caches, model.v_caches = [], []
    torch.cuda.empty_cache()
    return summary, outs


def workload_config4(model, world, dev, kv_fp8=False):
    """benchmark config 4 end to end: 256 requests x 1024-token prompts of
    uniform random ids, 512 greedy tokens each, P=256, every step through the
    engine loop (prefill and mixed steps at the 16384-token budget, then
    decode); kv_fp8 runs it over the optional fp8 (e4m3) pool."""
    rng = np.random.default_rng(41)
    V = model.cfg.vocab_size
    prompts = [rng.integers(0, V, PROMPT).tolist() for _ in range(NUM_SEQS)]
    warm = [rng.integers(0, V, PROMPT).tolist() for _ in range(MAX_BATCHED // PROMPT)]
    need = NUM_SEQS * ((PROMPT + MAX_OUT + PAGE - 1) // PAGE) + 16
    s, _ = run_workload(model, world, dev, prompts, MAX_OUT, need, warm, kv_fp8=kv_fp8)
    s["workload"] = ("config 4: Qwen3-8B, 256 requests x 1024-token prompts, 512 greedy tokens "
                     "each, P=256, max_num_batched_tokens 16384, chunked prefill off" +
                     ("; fp8 (e4m3) KV pool, not the reference's format" if kv_fp8 else ""))
    return s


def workload_config3(world, rank, dev, comm):
    """benchmark config 3: Qwen3-4B (random-init bf16), 128 requests with
    prompts U[128, 2048] of uniform random ids, 256 greedy tokens each,
    continuous batching with mixed prefill/decode steps."""
    import torch

    from nvkv.decoder import QWEN3_4B, Qwen3TP
    m = Qwen3TP(QWEN3_4B, rank, world, seed=4, device=dev, comm=comm,
                peer_allreduce=comm is not None, max_tokens=MAX_BATCHED)
    rng = np.random.default_rng(43)
    lens = rng.integers(128, 2049, 128)
    prompts = [rng.integers(0, QWEN3_4B.vocab_size, int(L)).tolist() for L in lens]
    warm = [rng.integers(0, QWEN3_4B.vocab_size, 2048).tolist() for _ in range(8)]
    need = int(sum((L + 256 + PAGE - 1) // PAGE for L in lens)) + 16
    s, _ = run_workload(m, world, dev, prompts, 256, need, warm)
    s["workload"] = ("config 3: Qwen3-4B, 128 requests, prompts U[128,2048], 256 greedy tokens "
                     f"each, P=256, tp{world}, continuous batching (mixed steps)")
    m.close()
    del m
    torch.cuda.empty_cache()
    return s


def workload_config1(dev, cpu=True):
    """benchmark config 1's workload: Qwen3-0.6B architecture (random-init),
    4 sequences with prompts U[64, 256] of uniform random ids, 32 greedy
    tokens each, P=256.  GPU: the nvkv path in bf16 through the engine loop
    (host clock, end to end).  CPU (`cpu_baseline`): the reference's fp32
    CPU route restated (oracle/qwen3_cpu.py) with the same weights, the same
    loop (one prefill step, then decode steps), all host threads."""
    import torch

    from nvkv.decoder import QWEN3_0_6B, Qwen3TP
    rng = np.random.default_rng(45)
    lens = rng.integers(64, 257, 4)
    prompts = [rng.integers(0, QWEN3_0_6B.vocab_size, int(L)).tolist() for L in lens]
    m = Qwen3TP(QWEN3_0_6B, 0, 1, seed=1, device=dev)
    s, outs = run_workload(m, 1, dev, prompts, 32, 16, prompts)
    s["workload"] = ("config 1: Qwen3-0.6B, 4 sequences, prompts U[64,256], 32 greedy tokens "
                     "each, P=256; GPU bf16")
    if cpu:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import nvkv_oracle as O
        import qwen3_cpu as Q
        cores = _all_host_threads()
        f = lambda t: t.float().cpu().numpy()  # noqa: E731
        wts = {"embed": f(m.embed), "norm": f(m.norm), "lm_head": f(m.lm_head)}
        for i, L in enumerate(m.layers):
            for k in ("qkv", "o", "gate_up", "down", "ln1", "ln2", "qn", "kn"):
                wts[f"{i}.{k}"] = f(L[k])
        nb = 16
        free = list(range(nb))[::-1]
        seqs = [O.Seq(list(p), [free.pop() for _ in range((len(p) + PAGE - 1) // PAGE)], 0,
                      len(p), PAGE) for p in prompts]
        cpu_model = Q.Qwen3CPU(QWEN3_0_6B, wts, nb, PAGE, "f32")
        t0 = time.perf_counter()
        ref = Q.greedy_generate(cpu_model, seqs, 32, free)
        t = time.perf_counter() - t0
        gen = 4 * 32
        s["cpu_baseline"] = {
            "value": round(gen / t, 3), "unit": "generated tok/s", "total_s": round(t, 3),
            "cores": cores, "kind": "port",
            "sample": "the whole config-1 workload (one prefill step + 31 decode steps, 4 "
                      "sequences), numpy fp32 restatement of the reference's CPU route"}
        s["gpu_vs_cpu_speedup"] = round(t / s["total_s"], 1)
        s["greedy_agreement_gpu_bf16_vs_cpu_fp32"] = round(float(np.mean(
            [a == b for u, v in zip(outs, ref) for a, b in zip(u, v)])), 4)
    del m
    torch.cuda.empty_cache()
    return s


def workload_config5(world, rank, dev, comm, steps=128):
    """benchmark config 5 at TP8: Qwen3-32B (random-init bf16), 64 sequences
    whose 32768-token contexts are already in the KV cache (filled with
    random values instead of a 2M-token prefill), then `steps` greedy decode
    tokens each.  One decode step (device-side metadata via
    nvkv_decode_advance, all 64 layers, lm_head, vocab-parallel argmax) is
    captured in a CUDA graph and replayed `steps` times between CUDA events,
    worst rank.  The per-layer decode attention (split-KV at 1 kv head per
    GPU) is timed alone the same way for its roofline."""
    import torch

    from nvkv import ops
    from nvkv.decoder import QWEN3_32B, Qwen3TP, Step
    B, ctx0 = 64, 32768
    m = Qwen3TP(QWEN3_32B, rank, world, seed=6, device=dev, comm=comm,
                peer_allreduce=comm is not None, max_tokens=MAX_BATCHED)
    per = (ctx0 + steps + PAGE - 1) // PAGE
    nb = B * per
    m.allocate_kv_cache(nb, PAGE, fill_random=True)
    bt = torch.arange(nb, dtype=torch.int32, device=dev).view(B, per)
    lens = torch.full((B,), ctx0, dtype=torch.int64, device=dev)
    ids = torch.randint(0, QWEN3_32B.vocab_size, (B,), device=dev)
    pos = torch.empty(B, dtype=torch.int64, device=dev)
    slots = torch.empty_like(pos)
    cu_q = torch.empty(B + 1, dtype=torch.int32, device=dev)
    cu_k = torch.empty_like(cu_q)
    st = Step(ids, pos, slots, cu_q, cu_k, bt, torch.arange(B, device=dev), 1, ctx0 + steps)

    def one():
        ops.decode_advance(lens, bt, nb, PAGE, pos, slots, cu_q, cu_k)
        ids.copy_(m.greedy(st))

    lens0 = lens.clone()
    one()  # warm-up (eager)
    torch.cuda.synchronize()
    s_ = torch.cuda.Stream()
    s_.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s_):
        one()
    torch.cuda.current_stream().wait_stream(s_)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        one()
    lens.copy_(lens0)
    torch.cuda.synchronize()
    _barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    ms = _max_over_ranks(e0.elapsed_time(e1), world, dev)
    g.reset()
    # decode attention alone, one layer's call on the last step's metadata
    q = m._bufs["q"]
    o = m._bufs["o"]
    ws = m._bufs["ws"]
    reps = 20

    def att():
        ops.paged_attention(q, m.k_caches[0], m.v_caches[0], cu_q, cu_k, bt, 1, ctx0 + steps,
                            m.scale, out=o, workspace=ws)

    att()
    torch.cuda.synchronize()
    with torch.cuda.stream(s_):
        att()
    torch.cuda.current_stream().wait_stream(s_)
    ga = torch.cuda.CUDAGraph()
    with torch.cuda.graph(ga):
        for li in range(reps):
            ops.paged_attention(q, m.k_caches[li % len(m.k_caches)],
                                m.v_caches[li % len(m.v_caches)], cu_q, cu_k, bt, 1,
                                ctx0 + steps, m.scale, out=o, workspace=ws)
    ga.replay()
    torch.cuda.synchronize()
    e0.record()
    ga.replay()
    e1.record()
    torch.cuda.synchronize()
    att_ms = _max_over_ranks(e0.elapsed_time(e1) / reps, world, dev)
    ga.reset()
    ctx_now = int(lens.sum().item())  # contexts of the last step (keys read per layer)
    nbytes = ctx_now * m.hkv * 128 * 2 * 2 + 2 * B * m.hq * 128 * 2 + 4 * B * per
    peak, peak_kind = load_peak()
    gbs = nbytes / (att_ms * 1e-3) / 1e9
    res = {"workload": "config 5: Qwen3-32B tp8, 64 sequences x 32768-token cached contexts "
                       "(random KV), 128 greedy decode tokens each, CUDA graph per step",
           "decode_tok_s": round(B * steps / (ms * 1e-3), 1),
           "ms_per_step": round(ms / steps, 4),
           "decode_attention": {"us_per_layer": round(att_ms * 1e3, 2), "bytes": int(nbytes),
                                "achieved_gbs": round(gbs, 1), "peak": peak,
                                "frac": round(gbs / peak, 4), "peak_source": peak_kind}}
    m.close()
    m.k_caches, m.v_caches = [], []
    del m
    torch.cuda.empty_cache()
    return res


def kv_fp8_step(model, w, world, dev, steps, warmup):
    """The same decode step over the optional fp8 (e4m3) pool: K/V codes with
    a f32 scale per (slot, kv head) row, written by the fp8 store, read by the
    fp8 decode kernel at half the bytes.  Not the reference's format (its pool
    is in the model dtype), so it is reported beside the headline, never as
    it.  CUDA graph of one step replayed `steps` times, CUDA events, worst
    rank; plus the decode attention of all layers, graph-replayed, against the
    measured HBM peak (algorithmic bytes: one byte per K/V value plus the
    4-byte row scales, q, out, block tables)."""
    import torch

    from nvkv import ops
    from nvkv.decoder import Step
    model.k_caches, model.v_caches = [], []
    torch.cuda.empty_cache()
    model.allocate_kv_cache(w["num_blocks"], PAGE, fill_random=True, kv_fp8=True)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)  # noqa: E731
    st = Step(t(w["input_ids"]), t(w["positions"]), t(w["slot_mapping"]), t(w["cu_q"]),
              t(w["cu_k"]), t(w["block_tables"]), torch.arange(NUM_SEQS, device=dev), 1, w["max_k"])
    for _ in range(max(1, warmup)):
        model.greedy(st)
    torch.cuda.synchronize()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        model.greedy(st)
    torch.cuda.current_stream().wait_stream(side)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        model.greedy(st)
    g.replay()
    torch.cuda.synchronize()
    _barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    ms = _max_over_ranks(e0.elapsed_time(e1), world, dev)
    g.reset()
    q, o, ws = model._bufs["q"], model._bufs["o"], model._bufs["ws"]
    L = model.cfg.num_hidden_layers

    def att():
        for li in range(L):
            ops.paged_attention_fp8(q, model.k_caches[li], model.v_caches[li], model.k_scales[li],
                                    model.v_scales[li], st.cu_seqlens_q, st.cu_seqlens_k,
                                    st.block_tables, 1, w["max_k"], model.scale, out=o,
                                    workspace=ws)

    att()
    torch.cuda.synchronize()
    with torch.cuda.stream(side):
        att()
    torch.cuda.current_stream().wait_stream(side)
    ga = torch.cuda.CUDAGraph()
    with torch.cuda.graph(ga):
        att()
    ga.replay()
    torch.cuda.synchronize()
    reps = max(3, min(steps, 20))
    e0.record()
    for _ in range(reps):
        ga.replay()
    e1.record()
    torch.cuda.synchronize()
    kern_ms = _max_over_ranks(e0.elapsed_time(e1) / (reps * L), world, dev)
    ga.reset()
    ctx = int(w["ctx"].sum())
    nbytes = (ctx * model.hkv * (128 + 4) * 2 + 2 * NUM_SEQS * model.hq * 128 * 2 +
              4 * int(((w["ctx"] + PAGE - 1) // PAGE).sum()) + 8 * (NUM_SEQS + 1))
    peak, kind = load_peak()
    gbs = nbytes / (kern_ms * 1e-3) / 1e9
    res = {"value": round(NUM_SEQS * steps / (ms * 1e-3), 1), "unit": "tok/s",
           "ms_per_step": round(ms / steps, 4),
           "kv": "e4m3 codes + f32 scale per (slot, kv head) row; not the reference's format",
           "decode_attention": {"us_per_launch": round(kern_ms * 1e3, 2), "bytes": int(nbytes),
                                "achieved_gbs": round(gbs, 1), "peak": peak,
                                "frac": round(gbs / peak, 4), "peak_source": kind}}
    model.k_caches, model.v_caches, model.k_scales, model.v_scales = [], [], [], []
    model.kv_fp8 = False
    model._bufs.pop("ws", None)
    torch.cuda.empty_cache()
    return res


def run_nvkv(a):
    import torch

    import nvkv
    from nvkv import ops
    from nvkv.decoder import QWEN3_8B, Qwen3TP, Step

    rank, world, dev = _dist_setup()
    cfg = QWEN3_8B
    if a.layers:
        from dataclasses import replace
        cfg = replace(cfg, num_hidden_layers=a.layers)
    w = workload()
    model = Qwen3TP(cfg, rank, world, seed=0, device=dev,
                    peer_allreduce=not a.nccl_allreduce, max_tokens=MAX_BATCHED)
    model.allocate_kv_cache(w["num_blocks"], PAGE, fill_random=True)
    host = {k: torch.from_numpy(np.ascontiguousarray(w[k])).pin_memory()
            for k in ("input_ids", "positions", "slot_mapping", "cu_q", "cu_k", "block_tables")}
    dv = {k: v.to(dev) for k, v in host.items()}
    st = Step(dv["input_ids"], dv["positions"], dv["slot_mapping"], dv["cu_q"], dv["cu_k"],
              dv["block_tables"], torch.arange(NUM_SEQS, device=dev), 1, w["max_k"])
    tok_host = torch.empty(NUM_SEQS, dtype=torch.int64).pin_memory()

    def step_fn():
        return model.greedy(st)

    for _ in range(max(1, a.warmup)):
        tok = step_fn()
    torch.cuda.synchronize()
    graph = None
    if not a.no_graph:
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            step_fn()
        torch.cuda.current_stream().wait_stream(s)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            tok = step_fn()
        for _ in range(max(3, a.warmup)):
            graph.replay()
        torch.cuda.synchronize()
    run = graph.replay if graph is not None else step_fn

    props = torch.cuda.get_device_properties(dev)
    bus = f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
    sampler = ClockSampler(bus) if rank == 0 else None

    # ---- timed region: K decode steps, inputs resident in HBM ----
    if sampler:
        sampler.start()
        time.sleep(0.3)  # before the barrier: every rank enters the timed region together
    _barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("bench_timed")  # ncu --nvtx-include "bench_timed/"
    e0.record()
    for _ in range(a.steps):
        run()
    e1.record()
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_pop()
    clocks = sampler.stop() if sampler else None
    ms = _max_over_ranks(e0.elapsed_time(e1), world, dev)
    _barrier(world)

    # ---- e2e: host inputs -> H2D, step, D2H of the sampled tokens, every step ----
    h2d = sum(v.numel() * v.element_size() for v in host.values())
    e0.record()
    for _ in range(a.steps):
        for k, v in host.items():
            dv[k].copy_(v, non_blocking=True)
        r = run()
        tok_host.copy_(tok if r is None else r, non_blocking=True)
        torch.cuda.current_stream().synchronize()
    e1.record()
    torch.cuda.synchronize()
    ms_e2e = _max_over_ranks(e0.elapsed_time(e1), world, dev)
    _barrier(world)

    # ---- roofline: the decode attention of every layer, graph-replayed ----
    # The 36 layers' paged-attention calls (decode kernel + split-KV combine,
    # same inputs as the step) are captured in one CUDA graph, as in the step,
    # so no host launch gap sits between them; `reps` replays between two CUDA
    # events on this stream give the mean device time per call.
    q = model._bufs["q"]
    o = model._bufs["o"]
    ws = model._bufs["ws"]
    reps = max(3, min(a.steps, 20))

    def attn_all_layers():
        for li in range(cfg.num_hidden_layers):
            ops.paged_attention(q, model.k_caches[li], model.v_caches[li], st.cu_seqlens_q,
                                st.cu_seqlens_k, st.block_tables, 1, w["max_k"], model.scale,
                                out=o, workspace=ws)

    attn_all_layers()
    torch.cuda.synchronize()
    s_side = torch.cuda.Stream()
    s_side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s_side):
        attn_all_layers()
    torch.cuda.current_stream().wait_stream(s_side)
    agraph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(agraph):
        attn_all_layers()
    agraph.replay()
    torch.cuda.synchronize()
    e0.record()
    for _ in range(reps):
        agraph.replay()
    e1.record()
    torch.cuda.synchronize()
    kern_ms = e0.elapsed_time(e1) / (reps * cfg.num_hidden_layers)
    agraph.reset()
    kern_ms = _max_over_ranks(kern_ms, world, dev)
    assert nvkv.device_error() == 0
    launches = model.launches_per_step(st) * a.steps
    ar = None
    if world > 1:  # every rank takes this step, in the same order
        ar_bytes = NUM_SEQS * cfg.hidden_size * 2
        ar_ms, ar_alg, ar_bus = _allreduce_bw(world, dev, ar_bytes)
        per_step = 2 * cfg.num_hidden_layers + 1
        ar = {"op": "all_reduce (o_proj, down_proj, embedding)", "bytes": ar_bytes,
              "us_per_call": round(ar_ms * 1e3, 2), "calls_per_step": per_step,
              "algbw_gbs": round(ar_alg, 1), "busbw_gbs": round(ar_bus, 1),
              "peak_gbs": 900.0, "peak_source": "NVLink 5 nominal per direction",
              "frac": round(ar_bus / 900.0, 4),
              "share_of_step": round(per_step * ar_ms / (ms / a.steps), 4),
              "step_route": "nccl all_reduce + nvkv_rms_norm" if model.comm is None else
                            "nvkv_allreduce_rms_norm (peer memory)"}
        if model.comm is not None:
            pm, pa, pb = _peer_allreduce_bw(model, world, dev, NUM_SEQS)
            ar["fused"] = {"op": "nvkv_allreduce_rms_norm (all-reduce + residual + RMSNorm, "
                                 "NVLink peer loads/stores)",
                           "us_per_call": round(pm * 1e3, 2), "algbw_gbs": round(pa, 1),
                           "busbw_gbs": round(pb, 1), "frac": round(pb / 900.0, 4),
                           "share_of_step": round(per_step * pm / (ms / a.steps), 4)}

    parity = tp_parity(model.cfg, model.comm, world, rank, dev) if world > 1 else None
    kv8 = None if a.no_workloads else kv_fp8_step(model, w, world, dev, a.steps, a.warmup)
    wl = None
    if not a.no_workloads:  # whole workloads through the engine loop (every rank)
        wl = {"config4": workload_config4(model, world, dev)}
        if world == 1:
            wl["config4_kv_fp8"] = workload_config4(model, world, dev, kv_fp8=True)
            wl["config3_tp1"] = workload_config3(world, rank, dev, None)
            wl["config1"] = workload_config1(dev)
        elif world == 2:
            wl["config3_tp2"] = workload_config3(world, rank, dev, model.comm)
        elif world == 8:
            wl["config5_tp8"] = workload_config5(world, rank, dev, model.comm)

    if rank == 0:
        peak, peak_kind = load_peak()
        nbytes = decode_bytes(w, model.hq, model.hkv)
        achieved = nbytes / (kern_ms * 1e-3) / 1e9
        val = NUM_SEQS * a.steps / (ms * 1e-3)
        line = {
            "metric": METRIC, "value": round(val, 1), "unit": "tok/s", "n_gpus": world,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(ms / a.steps, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded random-init weights, random prefilled KV, random token ids)",
            "config": bench_config(world, cuda_graph=graph is not None,
                                   nccl_allreduce=model.comm is None),
            "e2e": {"value": round(NUM_SEQS * a.steps / (ms_e2e * 1e-3), 1), "unit": "tok/s",
                    "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": NUM_SEQS * 8},
            "gpu_launches": int(launches),
            "roofline": {"bound": "hbm", "kernel": "nvkv paged decode attention (per layer)",
                         "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_source": peak_kind,
                         "bytes_per_launch": int(nbytes), "us_per_launch": round(kern_ms * 1e3, 2),
                         "traffic": int(nbytes * DECODE_DRAM_PER_ALG_BYTE),
                         "traffic_source": "ncu dram__bytes_read+write of the same per-layer "
                                           "shape, scaled to this launch's algorithmic bytes"},
            "clocks": clocks,
        }
        if ar is not None:
            line["collectives"] = ar
        if parity is not None:
            line["tp_parity"] = parity
        if kv8 is not None:
            line["kv_fp8"] = kv8
        if wl is not None:
            line["workloads"] = wl
        if world == 1:
            line["cpu_baseline"] = cpu_reference()
            line["op_level"] = op_level_config2()
        print(json.dumps(line), flush=True)
    # a graph holding NCCL calls must be released before the process group
    run = None
    if graph is not None:
        graph.reset()
        graph = None
    torch.cuda.synchronize()
    if world > 1:
        import threading
        import torch.distributed as dist

        # every GPU result is final here; never let communicator teardown hold the job
        def _exit_if_stuck():
            time.sleep(30)
            os._exit(0)

        threading.Thread(target=_exit_if_stuck, daemon=True).start()
        dist.barrier()  # every rank's last peer-memory call has completed
        model.close()
        dist.destroy_process_group()


# ---------------------------------------------------------------------------
# CPU restatement of the reference path (the reference's candle-CPU route is
# not buildable here: Rust toolchain absent), timed on the host cores.  This
# part imports neither torch's CUDA side nor nvkv: the oracle is numpy.
# ---------------------------------------------------------------------------

CPU_SAMPLE_SEQS = 16


def _all_host_threads():
    """torchrun sets OMP_NUM_THREADS=1; the CPU arm uses every host core."""
    import threadpoolctl
    n = os.cpu_count() or 1
    threadpoolctl.threadpool_limits(limits=n)
    try:
        import torch
        torch.set_num_threads(n)
    except Exception:
        pass
    return n


class CpuDecodeSample:
    """The reference's CPU route (candle CPU fp32: GEMMs, paged gather, unfused
    causal attention; oracle/qwen3_cpu.py) on a bounded sample of the bench
    workload: the first `num_seqs` of its 256 sequences (same seeded contexts,
    U[1025,1536]), each decoding one token through all 36 Qwen3-8B layers,
    the final norm and the full-vocab lm_head.  Every sequence has its own
    paged KV per layer, filled with random values.

    The 36 layers share one random-init fp32 weight set (0.77 GB per layer,
    far larger than the host caches, so each layer streams its weights from
    DRAM exactly as distinct weights would) so the sample fits in host
    memory; the embedding and lm_head are full size (2.5 GB each)."""

    def __init__(self, num_seqs=CPU_SAMPLE_SEQS, seed=7):
        from concurrent.futures import ThreadPoolExecutor

        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        sys.path.insert(0, os.path.join(ROOT, "nanovllm-rs_b200"))
        import nvkv_oracle as O
        from qwen3_cpu import Qwen3CPU
        from qwen3_config import QWEN3_8B

        self.cores = _all_host_threads()
        cfg = self.cfg = QWEN3_8B
        self.num_seqs = num_seqs
        rng = np.random.default_rng(seed)
        H, D, F = cfg.hidden_size, cfg.head_dim, cfg.intermediate_size
        hq, hkv = cfg.num_attention_heads, cfg.num_key_value_heads
        base = rng.standard_normal(1 << 22, dtype=np.float32)
        pool = ThreadPoolExecutor(self.cores)

        def fill(out, s):  # timing only: one seeded random buffer, tiled, on all cores
            src = np.roll(base, int(rng.integers(0, base.size))) * np.float32(s)
            flat = out.reshape(-1)

            def part(i):
                n = min(base.size, flat.size - i)
                flat[i:i + n] = src[:n]

            list(pool.map(part, range(0, flat.size, base.size)))
            return out

        def r(*shape, s=0.02):
            return fill(np.empty(shape, np.float32), s)

        layer = {"qkv": r((hq + 2 * hkv) * D, H), "o": r(H, hq * D), "gate_up": r(2 * F, H),
                 "down": r(H, F), "ln1": np.ones(H, np.float32), "ln2": np.ones(H, np.float32),
                 "qn": np.ones(D, np.float32), "kn": np.ones(D, np.float32)}
        wts = {"embed": r(cfg.vocab_size, H, s=1.0), "norm": np.ones(H, np.float32),
               "lm_head": r(cfg.vocab_size, H)}
        for i in range(cfg.num_hidden_layers):
            for k, v in layer.items():
                wts[f"{i}.{k}"] = v
        w = workload()
        ctx_lens = w["ctx"][:num_seqs]
        nblk = (ctx_lens + PAGE - 1) // PAGE
        self.model = Qwen3CPU(cfg, wts, int(nblk.sum()), PAGE)
        for kc, vc in zip(self.model.k, self.model.v):
            fill(kc, 1.0)
            fill(vc, 1.0)
        self.model.pool = pool
        seqs, used = [], 0
        for L, n in zip(ctx_lens, nblk):
            seqs.append(O.Seq(list(rng.integers(0, cfg.vocab_size, int(L))),
                              list(range(used, used + n)), int(L) - 1, 1, PAGE))
            used += n
        self.ids, self.pos, self.ctx = O.prepare_model_input(seqs, PAGE)
        self.kv_bytes = int(ctx_lens.sum()) * hkv * D * 2 * 4 * cfg.num_hidden_layers

    def step(self) -> float:
        """One sampled decode step (all layers, lm_head, argmax); host seconds."""
        t0 = time.perf_counter()
        logits = self.model.forward(self.ids, self.pos, self.ctx)
        np.argmax(logits, axis=-1)
        return time.perf_counter() - t0

    def describe(self, steps):
        return (f"{self.num_seqs} of the 256 sequences (contexts {int(self.ctx.max_seqlen_k)} max), "
                f"one decode token each through all {self.cfg.num_hidden_layers} layers + full "
                f"lm_head + argmax per step, {steps} timed steps; numpy fp32 restatement of the "
                f"reference's CPU route (oracle/qwen3_cpu.py), one weight set shared by the "
                f"layers, own paged KV per layer and sequence")


def cpu_reference(steps=3, warmup=1, num_seqs=CPU_SAMPLE_SEQS):
    """The `cpu_baseline` of the GPU arm's line: `steps` sampled decode steps
    (CpuDecodeSample) after `warmup`, tok/s = sampled tokens / host time."""
    smp = CpuDecodeSample(num_seqs)
    for _ in range(warmup):
        smp.step()
    t = sum(smp.step() for _ in range(steps))
    return {"value": round(num_seqs * steps / t, 3), "unit": "tok/s", "cores": smp.cores,
            "kind": "port", "sample": smp.describe(steps),
            "ms_per_step": round(t / steps * 1e3, 1)}


def op_level_config2(seed=2, reps=20):
    """benchmark config 2 at operator level: paged decode attention, B=64 decode
    queries, 16 q / 8 kv heads, L ~ U[512, 4096], P=256, block tables a seeded
    permutation of a 2048-block pool, q/k/v ~ N(0,1).  Reports the nvkv kernel
    (CUDA graph of `reps` calls, CUDA events), the installed flash_attn 2.8.3
    paged varlen kernel on the same tensors as a labelled reference-class
    proxy (the FA2 lineage of the reference's candle-flash-attn, run as a
    black box), and the CPU restatement of the reference path (oracle, numpy
    fp32, all host threads) on the same batch."""
    import torch

    from nvkv import ops
    B, hq, hkv, D, P, pool = 64, 16, 8, 128, 256, 2048
    rng = np.random.default_rng(seed)
    lens = rng.integers(512, 4097, B)
    need = (lens + P - 1) // P
    perm = rng.permutation(pool).astype(np.int32)
    bt = np.zeros((B, int(need.max())), np.int32)
    u = 0
    for i, n in enumerate(need):
        bt[i, :n] = perm[u:u + n]
        u += n
    g = torch.Generator(device="cuda").manual_seed(seed)
    kc = torch.randn(pool, P, hkv, D, generator=g, device="cuda").bfloat16()
    vc = torch.randn(pool, P, hkv, D, generator=g, device="cuda").bfloat16()
    q = torch.randn(B, hq, D, generator=g, device="cuda").bfloat16()
    cu_q = torch.arange(B + 1, dtype=torch.int32, device="cuda")
    cu_k = torch.from_numpy(np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)).cuda()
    btd = torch.from_numpy(bt).cuda()
    max_k, scale = int(lens.max()), D ** -0.5
    out = torch.empty_like(q)
    ws = torch.empty(max(16, ops.workspace_size(B, hq, hkv, 1, max_k)), dtype=torch.uint8,
                     device="cuda")

    def nv():
        ops.paged_attention(q, kc, vc, cu_q, cu_k, btd, 1, max_k, scale, out=out, workspace=ws)

    def graph_us(fn):
        fn()
        torch.cuda.synchronize()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            fn()
        torch.cuda.current_stream().wait_stream(s)
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            for _ in range(reps):
                fn()
        gr.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        gr.replay()
        e1.record()
        torch.cuda.synchronize()
        gr.reset()
        return e0.elapsed_time(e1) * 1e3 / reps

    nbytes = int(lens.sum()) * hkv * D * 2 * 2 + 2 * B * hq * D * 2 + 4 * int(need.sum())
    nv_us = graph_us(nv)
    peak, _ = load_peak()
    res = {"workload": "benchmark config 2: paged decode attention, B=64, 16q/8kv, D=128, "
                       "L~U[512,4096], P=256, 2048-block pool, bf16",
           "nvkv_us": round(nv_us, 2),
           "nvkv_gbs": round(nbytes / (nv_us * 1e-6) / 1e9, 1),
           "nvkv_frac_of_measured_hbm": round(nbytes / (nv_us * 1e-6) / 1e9 / peak, 4),
           "bytes": nbytes}
    try:
        from flash_attn import flash_attn_varlen_func
        fa_out = {}

        def fa():
            fa_out["o"] = flash_attn_varlen_func(q, kc, vc, cu_q, cu_k, 1, max_k,
                                                 softmax_scale=scale, causal=True,
                                                 block_table=btd)

        fa_us = graph_us(fa)
        fa()
        torch.cuda.synchronize()
        res["flash_attn_proxy"] = {
            "us": round(fa_us, 2), "gbs": round(nbytes / (fa_us * 1e-6) / 1e9, 1),
            "nvkv_speedup": round(fa_us / nv_us, 3),
            "max_abs_diff_vs_nvkv": round(float((fa_out["o"].float() - out.float()).abs().max()),
                                          5),
            "label": "flash_attn 2.8.3 flash_attn_varlen_func(block_table=...), black box"}
    except Exception as ex:  # not part of the product path: a proxy only
        res["flash_attn_proxy"] = {"unavailable": repr(ex)[:200]}
    # CPU restatement of the reference path on the same batch (rank 0, host cores)
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import nvkv_oracle as O
    cores = _all_host_threads()
    qn = q.float().cpu().numpy()
    seqs = []
    for b in range(B):  # the paged gather (layers/attention.rs:143-164), done once
        pages = torch.from_numpy(bt[b, :need[b]].astype(np.int64)).cuda()
        kb = kc.index_select(0, pages).reshape(-1, hkv, D)[:lens[b]].float().cpu().numpy()
        vb = vc.index_select(0, pages).reshape(-1, hkv, D)[:lens[b]].float().cpu().numpy()
        seqs.append((kb, vb))
    t0 = time.perf_counter()
    n_done = 0
    while True:
        for b in range(B):
            O.causal_attention_one(qn[b:b + 1], seqs[b][0], seqs[b][1], scale, acc=np.float32)
        n_done += 1
        if time.perf_counter() - t0 > 5.0 or n_done >= 3:
            break
    cpu_us = (time.perf_counter() - t0) / n_done * 1e6
    res["cpu_baseline"] = {"us": round(cpu_us, 1), "cores": cores, "kind": "port",
                           "nvkv_speedup": round(cpu_us / nv_us, 1),
                           "sample": "the whole config-2 batch: oracle causal_attention_one per "
                                     "sequence (numpy fp32, unfused softmax attention), the "
                                     "paged gather done beforehand"}
    return res


def run_reference(a):
    """The reference arm: the CPU restatement of the reference's route on the
    host cores, on this bench's `config`, metric and unit.  Each step is one
    CpuDecodeSample step (a bounded sample of the workload, really run); the
    line's value is sampled tokens / host time over exactly `--steps` steps.
    Under torchrun only rank 0 runs; the other ranks exit at once."""
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    if rank != 0:
        return
    smp = CpuDecodeSample()
    for _ in range(a.warmup):
        smp.step()
    t = sum(smp.step() for _ in range(a.steps))
    val = smp.num_seqs * a.steps / t
    line = {"metric": METRIC, "value": round(val, 3), "unit": "tok/s", "n_gpus": world,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(t / a.steps * 1e3, 3),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded random-init weights, random prefilled KV, random token ids)",
            "impl": "reference", "config": bench_config(world),
            "cpu_baseline": {"value": round(val, 3), "unit": "tok/s", "cores": smp.cores,
                             "kind": "port", "sample": smp.describe(a.steps)},
            "e2e": {"value": round(val, 3), "unit": "tok/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    a = parse()
    if a.impl == "reference":
        run_reference(a)
    else:
        run_nvkv(a)


if __name__ == "__main__":
    main()
