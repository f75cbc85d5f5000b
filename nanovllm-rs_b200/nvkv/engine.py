"""Greedy serving loop over the nvkv path, for whole-workload runs.

The caller side of the hot path, restated so a whole request set (prefill,
continuous batching, decode to the last token) can run through nvkv's own
pieces: the KV block manager (nvkv_block_manager_*), the step metadata
builder (nvkv_prepare_step) and the Qwen3 driver whose attention path is the
nvkv kernels.  It follows the reference's engine loop:

  * LLMEngine::step / generate (engine/llm_engine.rs:63-156): schedule, run
    the model, postprocess, until no request is left;
  * Scheduler::schedule (engine/scheduler.rs:98-188, chunked prefill off as
    the reference's default, EngineConfig config.rs:110-120): the running
    queue first, one token each, preempting from the back when the pool is
    full; then waiting prompts while the token budget, max_num_seqs and the
    pool allow (so prompts and decodes share a step);
  * Scheduler::postprocess (scheduler.rs:53-96): append the sampled token,
    finish on max_tokens / EOS / max_model_len and free the blocks;
  * sampling: each request's temperature (SamplingParams, sampling_params.rs)
    goes to the device sampler (nvkv_sample, the Gumbel-max form of
    sampler.rs:7-21) with the engine's seed and a step counter; temperature
    0 (the default here, as the benchmarks decode greedily) is the greedy
    pick, the temperature -> 0 limit.

Each sequence keeps one C view (nvkv_block_seq) over buffers it owns for its
whole life (token ids up to prompt + max_tokens, its block table), so a step
marshals nothing per token: one append_batch call for the running queue, one
prepare_step call for the step's metadata, written into pinned host buffers
and copied to the device in one batch of copies.  All ranks of a TP group run
the same loop on the same inputs; the tokens are identical on every rank
(the vocab-parallel pick over the ranks' candidates, the same seed and step
on every rank), so the ranks stay in lockstep without a broadcast.
"""
from __future__ import annotations

import ctypes
import time
from collections import deque
from typing import Dict, List, Optional

import numpy as np
import torch

from ._lib import BlockSeq, StepSizes, check, lib
from .blocks import BlockManager
from .decoder import Step


class _Seq:
    """One request: Sequence (engine/sequence.rs) fields the loop needs."""

    __slots__ = ("sid", "tokens", "table", "c", "num_prompt", "max_tokens", "ignore_eos",
                 "temperature")

    def __init__(self, sid: int, prompt, max_tokens: int, block_size: int, ignore_eos: bool,
                 temperature: float = 0.0):
        self.sid = sid
        self.temperature = float(temperature)
        self.num_prompt = len(prompt)
        self.max_tokens = max_tokens
        self.ignore_eos = ignore_eos
        cap = len(prompt) + max_tokens + 1
        self.tokens = np.zeros(cap, np.uint32)
        self.tokens[:len(prompt)] = np.asarray(prompt, np.uint32)
        nb = (cap + block_size - 1) // block_size + 1
        self.table = np.zeros(nb, np.uint32)
        self.c = BlockSeq(self.tokens.ctypes.data, len(prompt), 0, 0, self.table.ctypes.data, 0,
                          nb)

    def __len__(self) -> int:
        return int(self.c.num_tokens)

    def completion(self) -> List[int]:
        return self.tokens[self.num_prompt:len(self)].tolist()


class Engine:
    """LLMEngine over a Qwen3TP model (nvkv attention path) and a KV pool of
    `num_blocks` pages that the model's caches already hold."""

    def __init__(self, model, num_blocks: int, block_size: int = 256, max_num_seqs: int = 512,
                 max_num_batched_tokens: int = 16384, max_model_len: int = 40960,
                 eos: int = -1, cuda_graphs: bool = True, seed: int = 0):
        self.model = model
        self.seed = int(seed)
        self._step_no = 0  # the sampler's counter: one per engine step
        self.block_size = block_size
        self.max_num_seqs = max_num_seqs
        self.budget = max_num_batched_tokens
        self.max_model_len = max_model_len
        self.eos = eos
        self.bm = BlockManager(num_blocks, block_size)
        self.waiting: deque = deque()
        self.running: deque = deque()
        self.finished: Dict[int, List[int]] = {}
        self._next = 0
        dev = model.device
        T, B = max_num_batched_tokens, max_num_seqs
        self._w = (max_model_len + block_size - 1) // block_size
        self._cuda = torch.device(dev).type == "cuda"
        pin = dict(pin_memory=self._cuda)
        self.h = dict(ids=torch.zeros(T, dtype=torch.int64, **pin),
                      pos=torch.zeros(T, dtype=torch.int64, **pin),
                      slots=torch.zeros(T, dtype=torch.int64, **pin),
                      cu_q=torch.zeros(B + 1, dtype=torch.int32, **pin),
                      cu_k=torch.zeros(B + 1, dtype=torch.int32, **pin),
                      ctx=torch.zeros(B, dtype=torch.int64, **pin),
                      need=torch.zeros(B, dtype=torch.int64, **pin),
                      bt=torch.zeros(B * self._w, dtype=torch.int32, **pin))
        self.d = {k: torch.zeros(v.numel(), dtype=v.dtype, device=dev) for k, v in self.h.items()}
        self.tok_h = torch.zeros(B, dtype=torch.int64, **pin)
        self.temp_h = torch.zeros(B, dtype=torch.float32, **pin)
        self.temp_d = torch.zeros(B, dtype=torch.float32, device=dev)
        self.step_d = torch.zeros(1, dtype=torch.int64, device=dev)  # sampler counter (graphs)
        self.stats = []  # per step: (prompt tokens, decode tokens, seconds)
        # pure decode steps replay a CUDA graph per (batch size, context bucket);
        # a key is captured when it repeats on consecutive steps (config-4-like
        # runs decode hundreds of steps at one batch size)
        self.cuda_graphs = cuda_graphs and self._cuda
        self._graphs: Dict[tuple, tuple] = {}
        self._last_key = None
        self.bt_g = torch.zeros(B * self._w, dtype=torch.int32, **pin)
        self.d_bt_g = torch.zeros(B * self._w, dtype=torch.int32, device=dev)
        self.graph_steps = 0

    def close(self) -> None:
        for g, _ in self._graphs.values():  # graphs may hold collectives: drop them first
            g.reset()
        self._graphs.clear()
        self.bm.close()

    # ---- requests ----------------------------------------------------------
    def add_request(self, prompt, max_tokens: int, ignore_eos: bool = True,
                    temperature: float = 0.0) -> int:
        """LLMEngine::add_request + Scheduler::add (scheduler.rs:40-46);
        temperature 0 decodes greedily."""
        if len(prompt) > self.max_model_len - 1:
            raise ValueError("Sequence length exceeds max_model_len")
        if temperature < 0:
            raise ValueError("temperature must be >= 0")
        s = _Seq(self._next, prompt, max_tokens, self.block_size, ignore_eos, temperature)
        self._next += 1
        self.waiting.append(s)
        return s.sid

    def is_finished(self) -> bool:
        return not self.waiting and not self.running

    # ---- scheduler (scheduler.rs:98-188, chunked prefill off) ----------------
    def _preempt(self, s: _Seq) -> None:
        check(lib.nvkv_block_manager_deallocate(self.bm._h, ctypes.byref(s.c)))
        self.waiting.appendleft(s)

    def _schedule(self) -> List[_Seq]:
        budget = self.budget
        preempted = False
        sched: List[_Seq] = []
        i = 0
        while i < len(self.running) and budget > 0:
            run = list(self.running)[i:]
            take = run[:budget]  # one token each: num_new = len - num_cached
            nn = np.asarray([min(len(s) - s.c.num_cached_tokens,
                                 self.max_model_len - 1 - s.c.num_cached_tokens) for s in take],
                            np.int64)
            arr = (BlockSeq * len(take))(*[s.c for s in take])
            done = ctypes.c_int64(0)
            check(lib.nvkv_block_manager_append_batch(self.bm._h, arr, len(take),
                                                      nn.ctypes.data, ctypes.byref(done)))
            for k in range(int(done.value)):
                take[k].c = arr[k]
                budget -= int(nn[k])
            sched.extend(take[:done.value])
            i += int(done.value)
            if done.value == len(take):
                break
            # the sequence at i does not fit: preempt from the back, retry it
            while len(self.running) > i:
                victim = self.running.pop()
                self._preempt(victim)
                preempted = True
                if len(self.running) == i:
                    break
                s = self.running[i]
                ok = ctypes.c_int(0)
                check(lib.nvkv_block_manager_can_append(self.bm._h, ctypes.byref(s.c),
                                                        int(len(s) - s.c.num_cached_tokens),
                                                        ctypes.byref(ok)))
                if ok.value:
                    break
            if len(self.running) == i:
                break
        if not preempted:
            while self.waiting and budget > 0 and len(self.running) < self.max_num_seqs:
                s = self.waiting[0]
                u, f, n = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int64()
                check(lib.nvkv_block_manager_get_token_layout(self.bm._h, ctypes.byref(s.c),
                                                              ctypes.byref(u), ctypes.byref(f),
                                                              ctypes.byref(n)))
                ok = ctypes.c_int(0)
                check(lib.nvkv_block_manager_can_allocate(self.bm._h, f.value + n.value,
                                                          ctypes.byref(ok)))
                if n.value > budget or not ok.value:
                    break
                s.c.num_new_tokens = n.value
                check(lib.nvkv_block_manager_allocate(self.bm._h, ctypes.byref(s.c)))
                budget -= int(n.value)
                self.waiting.popleft()
                self.running.append(s)
                sched.append(s)
        if not sched:
            raise RuntimeError("scheduler: nothing fits the KV pool")
        return sched

    # ---- one step -----------------------------------------------------------
    def _prepare(self, sched: List[_Seq]) -> Step:
        """nvkv_prepare_step into the pinned buffers, then one batch of H2D copies."""
        B = len(sched)
        arr = (BlockSeq * B)(*[s.c for s in sched])
        sizes = StepSizes()
        h = self.h
        p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
        check(lib.nvkv_prepare_step(arr, B, self.block_size, p(h["ids"]), p(h["pos"]),
                                    p(h["cu_q"]), p(h["cu_k"]), p(h["slots"]), p(h["ctx"]),
                                    p(h["need"]), p(h["bt"]), h["ids"].numel(),
                                    h["slots"].numel(), h["bt"].numel(), ctypes.byref(sizes)))
        T, W = int(sizes.num_tokens), int(sizes.block_table_width)
        if not sizes.has_block_tables:  # a fresh-prefill step: the driver still attends
            W = max(int(s.c.block_table_len) for s in sched)  # through the cache, so
            bt = h["bt"][:B * W].view(B, W).numpy()  # build them here (0-padded)
            bt.fill(0)
            for k, s in enumerate(sched):
                n = int(s.c.block_table_len)
                bt[k, :n] = s.table[:n].view(np.int32)
        n_need = int(sizes.num_need_logits)
        d = self.d
        for k, n in (("ids", T), ("pos", T), ("slots", T), ("cu_q", B + 1), ("cu_k", B + 1),
                     ("need", n_need), ("bt", B * W)):
            d[k][:n].copy_(h[k][:n], non_blocking=self._cuda)
        cu_q = d["cu_q"][:B + 1]
        last = cu_q.index_select(0, d["need"][:n_need] + 1).long() - 1
        self._n_need = n_need
        prompt_rows = 0
        self._decode_only = (sizes.max_seqlen_q == 1 and n_need == B and
                             bool(sizes.has_block_tables))
        self._B, self._W, self._max_k = B, W, int(sizes.max_seqlen_k)
        if sizes.max_seqlen_q > 1:  # the fp8 pool dequantises the prompts' keys
            ql = np.diff(h["cu_q"][:B + 1].numpy())
            prompt_rows = int(h["ctx"][:B].numpy()[ql > 1].sum())
        return Step(d["ids"][:T], d["pos"][:T], d["slots"][:T], cu_q, d["cu_k"][:B + 1],
                    d["bt"][:B * W].view(B, W), last, int(sizes.max_seqlen_q),
                    int(sizes.max_seqlen_k), prompt_rows)

    def step(self) -> int:
        """One engine step; returns the number of tokens sampled."""
        t0 = time.perf_counter()
        sched = self._schedule()
        prompt_tok = sum(int(s.c.num_new_tokens) for s in sched if s.c.num_new_tokens > 1)
        decode_tok = sum(1 for s in sched if s.c.num_new_tokens == 1)
        st = self._prepare(sched)
        n = self._n_need
        need = self.h["need"][:n].tolist()
        temps = [sched[i].temperature for i in need]
        step_no = self._step_no
        self._step_no += 1
        sampling = any(t > 0 for t in temps)  # the logits rows' temperatures (0: greedy)
        if sampling:
            self.temp_h[:n] = torch.tensor(temps, dtype=torch.float32)
            self.temp_d[:n].copy_(self.temp_h[:n], non_blocking=self._cuda)
        tok = None
        if self.cuda_graphs and self._decode_only:
            tok = self._decode_graph(st, step_no if sampling else None)
        if tok is None:
            tok = (self.model.sample(st, self.temp_d[:n], self.seed, step_no) if sampling
                   else self.model.greedy(st))
        self.tok_h[:n].copy_(tok[:n], non_blocking=self._cuda)
        if self._cuda:
            torch.cuda.current_stream().synchronize()
        toks = self.tok_h[:n].tolist()
        for idx, t in zip(need, toks):  # postprocess (scheduler.rs:53-96)
            s = sched[idx]
            L = len(s)
            s.tokens[L] = t
            s.c.num_tokens = L + 1
            done = ((not s.ignore_eos and t == self.eos) or L + 1 - s.num_prompt >= s.max_tokens
                    or L + 1 >= self.max_model_len)
            if done:
                check(lib.nvkv_block_manager_deallocate(self.bm._h, ctypes.byref(s.c)))
                self.running.remove(s)
                self.finished[s.sid] = s.completion()
            else:
                s.c.num_cached_tokens += s.c.num_new_tokens
                s.c.num_new_tokens = 0
        for s in sched:  # scheduled but without logits (none without chunked prefill)
            if s.c.num_new_tokens and s.sid not in self.finished:
                s.c.num_cached_tokens += s.c.num_new_tokens
                s.c.num_new_tokens = 0
        self.stats.append((prompt_tok, decode_tok, time.perf_counter() - t0))
        return n

    def _decode_graph(self, st: Step, step_no: Optional[int] = None) -> Optional[torch.Tensor]:
        """A pure decode step through a captured CUDA graph, or None (then the
        step runs eagerly).  The graph's step has fixed shapes: the batch size,
        max_seqlen_k rounded up to a multiple of 1024 (the kernels take it as a
        bound) and block tables padded to that many pages in a fixed buffer;
        the step's own metadata is copied into the same device buffers first.
        With step_no (a sampling step) the graph samples with the rows'
        temperatures from temp_d and the counter from step_d, both set before
        each replay, so replays draw exactly the eager step's noise."""
        B, P = self._B, self.block_size
        bucket = -(-self._max_k // 1024) * 1024
        sampling = step_no is not None
        key = (B, bucket, sampling)
        g = self._graphs.get(key)
        if g is None and (self._last_key != key or len(self._graphs) >= 8):
            self._last_key = key
            return None
        self._last_key = key
        Wg = -(-bucket // P)
        bt = self.bt_g[:B * Wg].view(B, Wg).numpy()
        bt.fill(0)
        bt[:, :self._W] = self.h["bt"][:B * self._W].view(B, self._W).numpy()
        self.d_bt_g[:B * Wg].copy_(self.bt_g[:B * Wg], non_blocking=True)
        d = self.d
        stg = Step(d["ids"][:B], d["pos"][:B], d["slots"][:B], d["cu_q"][:B + 1],
                   d["cu_k"][:B + 1], self.d_bt_g[:B * Wg].view(B, Wg), st.last_idx, 1, bucket, 0)
        if sampling:
            self.step_d.fill_(step_no)
            temps = self.temp_d[:B]

            def pick(s):
                return self.model.sample(s, temps, self.seed, 0, step_device=self.step_d)
        else:
            pick = self.model.greedy
        if g is None:  # capture: one eager warm-up of these shapes, then the graph
            pick(stg)
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                pick(stg)
            torch.cuda.current_stream().wait_stream(side)
            graph = torch.cuda.CUDAGraph()
            last = d["need"][:B]
            # the model's scratch buffers of this graph come from the graph's
            # own memory pool, so later eager steps that reallocate them (other
            # shapes) never hand the graph's memory to anything else
            saved, self.model._bufs = self.model._bufs, {}
            try:
                with torch.cuda.graph(graph):
                    stg.last_idx = d["cu_q"].index_select(0, last + 1).long() - 1
                    out = pick(stg)
            finally:
                self.model._bufs = saved
            g = self._graphs[key] = (graph, out)
        g[0].replay()
        self.graph_steps += 1
        return g[1]

    def generate(self, prompts, max_tokens: int, ignore_eos: bool = True,
                 temperature=0.0) -> List[List[int]]:
        """LLMEngine::generate: every prompt to completion; the completions in
        request order.  temperature: one value for every request or one per
        prompt."""
        temps = (list(temperature) if isinstance(temperature, (list, tuple))
                 else [temperature] * len(prompts))
        ids = [self.add_request(p, max_tokens, ignore_eos, t) for p, t in zip(prompts, temps)]
        while not self.is_finished():
            self.step()
        return [self.finished[i] for i in ids]

    def summary(self) -> dict:
        """Throughput of the run: prompt tokens per second over the steps that
        carried prompts, decode tokens per second over the pure decode steps,
        and the reference's own figure (tokens of finished sequences over the
        whole run, llm_engine.rs:114-126)."""
        pre = [(p, d, t) for p, d, t in self.stats if p > 0]
        dec = [(p, d, t) for p, d, t in self.stats if p == 0]
        tot = sum(t for _, _, t in self.stats)
        fin = sum(len(v) for v in self.finished.values())
        return {"steps": len(self.stats), "prefill_steps": len(pre),
                "prompt_tokens": sum(p for p, _, _ in pre),
                "prefill_s": round(sum(t for _, _, t in pre), 4),
                "prompt_tok_s": round(sum(p for p, _, _ in pre) / max(sum(t for *_, t in pre), 1e-9),
                                      1),
                "decode_steps": len(dec), "decode_tokens": sum(d for _, d, _ in dec),
                "decode_s": round(sum(t for _, _, t in dec), 4),
                "decode_tok_s": round(sum(d for _, d, _ in dec) / max(sum(t for *_, t in dec), 1e-9),
                                      1),
                "generated_tokens": fin, "total_s": round(tot, 4),
                "output_tok_s": round(fin / max(tot, 1e-9), 1)}
