"""CPU (numpy) restatement of the reference's Qwen3 forward around the
attention hot path -- the reference's CPU route (candle CPU + the unfused
varlen attention of layers/attention.rs:85-137), in fp32 or with the bf16
rounding points of its GPU route.

TEST INFRASTRUCTURE ONLY (the checker and the timed CPU baseline; see
nvkv_oracle.py).  Layer order follows models/qwen3.rs:126-146 (attention),
:179-183 (MLP), :226-243 (decoder layer), :285-297 (model), and
embed_head.rs:89-119 (last-token logits).
Weights come in as a dict of numpy arrays (unsharded), so a test can hand it
exactly the weights a GPU model uses.
"""
from __future__ import annotations

from typing import Dict, List

import numpy as np

import nvkv_oracle as O


class Qwen3CPU:
    """weights: 'embed' [V,H], 'norm' [H], 'lm_head' [V,H] and per layer i:
    f'{i}.qkv' [(Hq+2Hkv)D, H], f'{i}.o' [H, HqD], f'{i}.gate_up' [2F, H],
    f'{i}.down' [H, F], f'{i}.ln1', f'{i}.ln2' [H], f'{i}.qn', f'{i}.kn' [D]."""

    def __init__(self, cfg, weights: Dict[str, np.ndarray], num_blocks: int, block_size: int,
                 dtype: str = "f32"):
        """dtype 'f32' is config 1's fp32 CPU route; 'bf16' rounds to bf16 at
        every op boundary of the reference's candle bf16 route (GEMM outputs,
        norms, RoPE, attention output, SiLU*mul, residual adds, and the
        lm_head logits, embed_head.rs:113) with f32 arithmetic inside each
        op."""
        self.cfg, self.w, self.dt = cfg, weights, dtype
        D = cfg.head_dim
        self.P = block_size
        shape = (num_blocks, block_size, cfg.num_key_value_heads, D)
        self.k = [np.zeros(shape, np.float32) for _ in range(cfg.num_hidden_layers)]
        self.v = [np.zeros(shape, np.float32) for _ in range(cfg.num_hidden_layers)]
        self.pool = None  # optional executor: per-sequence attention on host threads

    def _mm(self, x, w):
        return O.round_to(x @ w.T, self.dt)

    def layer(self, i: int, h, residual, positions, ctx):
        c, w, dt = self.cfg, self.w, self.dt
        Hq, Hkv, D = c.num_attention_heads, c.num_key_value_heads, c.head_dim
        if residual is None:  # qwen3.rs:232-238
            x, residual = O.rms_norm(h, w[f"{i}.ln1"], c.rms_norm_eps, dt), h
        else:
            x, residual = O.residual_rms_norm(h, residual, w[f"{i}.ln1"], c.rms_norm_eps, dt)
        qkv = self._mm(x, w[f"{i}.qkv"])
        q, k, v = O.qknorm_rope(qkv, positions, Hq, Hkv, D, w[f"{i}.qn"], w[f"{i}.kn"],
                                c.rms_norm_eps, c.rope_theta, dt)
        o = O.round_to(O.attention_forward(q, k, v, ctx, self.k[i], self.v[i], D ** -0.5,
                                           acc=np.float32 if dt == "f32" else np.float64,
                                           pool=self.pool), dt)
        a = self._mm(o.reshape(len(q), -1), w[f"{i}.o"])
        x, residual = O.residual_rms_norm(a, residual, w[f"{i}.ln2"], c.rms_norm_eps, dt)
        act = O.silu_and_mul(self._mm(x, w[f"{i}.gate_up"]), dt)
        return self._mm(act, w[f"{i}.down"]), residual

    def forward(self, input_ids, positions, ctx, layers: int = None) -> np.ndarray:
        """Returns last-token logits [B, V] (embed_head.rs:96-113)."""
        c, w = self.cfg, self.w
        h = w["embed"][input_ids]
        residual = None
        for i in range(layers if layers is not None else c.num_hidden_layers):
            h, residual = self.layer(i, h, residual, positions, ctx)
        h, _ = O.residual_rms_norm(h, residual, w["norm"], c.rms_norm_eps, self.dt)
        last = ctx.cu_seqlens_q[1:].astype(np.int64) - 1
        if len(ctx.seq_need_compute_logits):
            last = last[ctx.seq_need_compute_logits]
        return O.round_to(h[last] @ w["lm_head"].T, self.dt)


def advance(seqs: List[O.Seq], tokens, free_blocks: List[int], P: int) -> None:
    """Scheduler::postprocess + BlockManager::may_append (scheduler.rs:53-96,
    block_manager.rs): append the sampled token and a page when one fills."""
    for s, t in zip(seqs, tokens):
        s.num_cached_tokens = s.num_context_tokens()
        s.token_ids.append(int(t))
        s.num_new_tokens = 1
        if (len(s.token_ids) + P - 1) // P > len(s.block_table):
            s.block_table.append(free_blocks.pop())


def bf16_near_ties(logits: np.ndarray) -> List[frozenset]:
    """Per row, the token ids whose logit lies within one bf16 ulp of the
    row's maximum (the ulp taken at the maximum): the choices that the
    reference's bf16 logits (embed_head.rs:113) cannot tell apart from its
    greedy pick by more than their own rounding step."""
    m = logits.max(axis=-1)
    _, ex = np.frexp(np.abs(m))
    ulp = np.ldexp(1.0, ex - 8)  # |m| in [2^(ex-1), 2^ex): bf16 spacing 2^(ex-1-7)
    return [frozenset(np.nonzero(row >= mm - u)[0].tolist())
            for row, mm, u in zip(logits, m, ulp)]


def greedy_generate(model: Qwen3CPU, seqs: List[O.Seq], steps: int, free_blocks: List[int],
                    forced=None, near=None) -> List[List[int]]:
    """ModelRunner::run with greedy (argmax) sampling, no preemption: one
    prefill step for every prompt, then `steps - 1` decode steps.  With
    `forced` (per-sequence token lists) the forced tokens are appended instead
    of the model's own choices (teacher forcing); the return value is always
    the model's argmax at every step.  With `near` (a list, per sequence) the
    bf16 near-tie set of every step's logits is appended to it."""
    P = model.P
    out: List[List[int]] = [[] for _ in seqs]
    if near is not None:
        near.extend([] for _ in seqs)
    for step in range(steps):
        ids, pos, ctx = O.prepare_model_input(seqs, P)
        logits = model.forward(ids, pos, ctx)
        nxt = np.argmax(logits, axis=-1)
        for o, t in zip(out, nxt):
            o.append(int(t))
        if near is not None:
            for n, t in zip(near, bf16_near_ties(logits)):
                n.append(t)
        feed = nxt if forced is None else [f[step] for f in forced]
        advance(seqs, feed, free_blocks, P)
    return out
