"""nvkv.engine (the greedy serving loop over the C-ABI block manager and
nvkv_prepare_step) against a plain restatement of the reference's engine
loop, on the CPU with a stand-in model.

The stand-in's "greedy token" of a sequence is a fixed function of the step
inputs it is given (the last row's input id and position), so any mistake in
scheduling, preemption, block tables, slot mapping, cu_seqlens or the
postprocess changes some completion.  The restatement runs
Scheduler::schedule / postprocess (scheduler.rs:53-188, chunked prefill off)
over the oracle's BlockManager and prepare_model_input, and its sampled
token is computed from the oracle's own step inputs.  Both must give the
same completions, the same number of steps and the same per-step prompt /
decode token counts, including on pools small enough to preempt.
Per-request temperatures reach the model's sample() with the engine's seed
and step counter, row by row, and greedy rows stay greedy.
"""
from collections import deque

import numpy as np
import pytest
import torch

import block_manager_oracle as OB
import nvkv_oracle as O
from nvkv.engine import Engine

V = 1000


def _token(ids_last, pos_last):
    return (int(ids_last) * 31 + int(pos_last) * 7 + 3) % V


def _sampled(ids_last, pos_last, temp, seed, step):
    """The stand-in's sampled token: the greedy one for temperature 0, else a
    fixed function of the temperature, the seed and the step counter too."""
    if temp <= 0:
        return _token(ids_last, pos_last)
    return (_token(ids_last, pos_last) + int(round(temp * 10)) + 13 * seed + 101 * step) % V


class _FakeModel:
    device = torch.device("cpu")

    def __init__(self, page):
        self.page = page
        self.steps = []

    def greedy(self, st):
        ids, pos = st.input_ids.numpy(), st.positions.numpy()
        last = st.last_idx.numpy()
        # the metadata must be self-consistent: slots follow the block tables
        bt = st.block_tables.numpy()
        cu_q, cu_k = st.cu_seqlens_q.numpy(), st.cu_seqlens_k.numpy()
        # the fp8 pool's dequantisation workspace: the prompts' keys exactly
        ql, kl = np.diff(cu_q.astype(np.int64)), np.diff(cu_k.astype(np.int64))
        assert st.prompt_kv_tokens == (int(kl[ql > 1].sum()) if st.max_seqlen_q > 1 else 0)
        for b in range(len(cu_q) - 1):
            q0, q1 = int(cu_q[b]), int(cu_q[b + 1])
            k_len = int(cu_k[b + 1] - cu_k[b])
            for t in range(q0, q1):
                p = int(pos[t])
                assert p == k_len - (q1 - t)
                want = int(bt[b, p // self.page]) * self.page + p % self.page
                assert int(st.slot_mapping[t]) == want
        return torch.tensor([_token(ids[r], pos[r]) for r in last], dtype=torch.int64)

    def sample(self, st, temps, seed, step):
        greedy = self.greedy(st).numpy()  # the same metadata checks
        ids, pos = st.input_ids.numpy(), st.positions.numpy()
        last = st.last_idx.numpy()
        t = temps.numpy()
        assert len(t) == len(last)
        out = [_sampled(ids[r], pos[r], float(t[k]), seed, step) for k, r in enumerate(last)]
        assert all(o == g for o, g, tk in zip(out, greedy, t) if tk <= 0)
        return torch.tensor(out, dtype=torch.int64)


def _reference(prompts, max_tokens, num_blocks, page, budget, max_seqs, temps=None, seed=0):
    """LLMEngine::generate with Scheduler (non-chunked) on the oracle pieces;
    temps: per-request temperatures (None: greedy)."""
    temps = temps or [0.0] * len(prompts)
    step_no = 0
    bm = OB.BlockManager(num_blocks, page)
    waiting = deque((i, OB.Seq(list(p), page)) for i, p in enumerate(prompts))
    running = deque()
    done, stats = {}, []
    while waiting or running:
        tb, preempted, sched = budget, False, []
        i = 0
        while i < len(running) and tb > 0:  # scheduler.rs:103-140
            sid, s = running[i]
            n = len(s) - s.num_cached_tokens
            while True:
                if bm.can_append(s, n):
                    s.num_new_tokens = n
                    bm.may_append(s)
                    break
                vid, v = running.pop()
                bm.deallocate(v)
                waiting.appendleft((vid, v))
                preempted = True
                if len(running) == i:
                    break
            if len(running) == i:
                break
            tb -= s.num_new_tokens
            sched.append((sid, s))
            i += 1
        if not preempted:  # scheduler.rs:143-180
            while waiting and tb > 0 and len(running) < max_seqs:
                sid, s = waiting[0]
                used, free, n = bm.get_token_layout(s)
                if n > tb or not bm.can_allocate(free + n):
                    break
                s.num_new_tokens = n
                bm.allocate(s)
                tb -= n
                waiting.popleft()
                running.append((sid, s))
                sched.append((sid, s))
        assert sched
        stats.append((sum(s.num_new_tokens for _, s in sched if s.num_new_tokens > 1),
                      sum(1 for _, s in sched if s.num_new_tokens == 1)))
        seqs = [O.Seq(list(s.token_ids), list(s.block_table), s.num_cached_tokens,
                      s.num_new_tokens, page) for _, s in sched]
        ids, pos, ctx = O.prepare_model_input(seqs, page)
        last = ctx.cu_seqlens_q[1:].astype(np.int64) - 1
        for k in ctx.seq_need_compute_logits:  # scheduler.rs:53-96
            sid, s = sched[k]
            t = _sampled(ids[last[k]], pos[last[k]], temps[sid], seed, step_no)
            s.append_token(t)
            if len(s) - len(prompts[sid]) >= max_tokens:
                bm.deallocate(s)
                running.remove((sid, s))
                done[sid] = s.token_ids[len(prompts[sid]):]
            else:
                s.num_cached_tokens += s.num_new_tokens
                s.num_new_tokens = 0
        step_no += 1
    return [done[i] for i in range(len(prompts))], stats


@pytest.mark.parametrize("seed,page,num_blocks,budget,max_seqs", [
    (0, 16, 400, 256, 512),   # roomy: no preemption
    (1, 16, 40, 256, 512),    # tight pool: preemption from the back
    (2, 256, 12, 2048, 4),    # max_num_seqs bounds admission
    (3, 16, 26, 64, 512),     # small budget: prompts wait for it
])
def test_engine_matches_reference_loop(seed, page, num_blocks, budget, max_seqs):
    rng = np.random.default_rng(seed)
    prompts = [rng.integers(0, V, int(L)).tolist() for L in rng.integers(1, 60, 12)]
    max_tokens = 20
    want, want_stats = _reference(prompts, max_tokens, num_blocks, page, budget, max_seqs)
    eng = Engine(_FakeModel(page), num_blocks, page, max_num_seqs=max_seqs,
                 max_num_batched_tokens=budget, max_model_len=4096)
    got = eng.generate(prompts, max_tokens)
    assert got == want
    assert [(p, d) for p, d, _ in eng.stats] == want_stats
    assert eng.bm.num_free == num_blocks  # every block returned
    s = eng.summary()
    assert s["generated_tokens"] == 12 * max_tokens
    eng.close()


def test_engine_temperatures_go_to_the_sampler():
    """Per-request temperatures: rows with T > 0 are sampled (the model's
    sample() with the engine's seed and step counter), T = 0 rows stay
    greedy, and a step with only greedy rows takes the greedy path."""
    rng = np.random.default_rng(7)
    prompts = [rng.integers(0, V, int(L)).tolist() for L in rng.integers(1, 60, 10)]
    temps = [0.0, 0.7, 1.0, 0.0, 1.3, 0.2, 0.0, 0.9, 0.0, 2.0]
    want, _ = _reference(prompts, 15, 400, 16, 256, 512, temps=temps, seed=5)
    eng = Engine(_FakeModel(16), 400, 16, max_num_batched_tokens=256, max_model_len=4096,
                 seed=5)
    assert eng.generate(prompts, 15, temperature=temps) == want
    eng.close()
    greedy, _ = _reference(prompts, 15, 400, 16, 256, 512)
    assert want != greedy  # the sampled rows changed something
    eng = Engine(_FakeModel(16), 400, 16, max_num_batched_tokens=256, max_model_len=4096)
    assert eng.generate(prompts, 15) == greedy
    eng.close()
