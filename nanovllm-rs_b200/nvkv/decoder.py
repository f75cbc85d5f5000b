"""Qwen3-shaped tensor-parallel decoder driving the nvkv hot path.

This is the caller side of the path (models/qwen3.rs:126-146,179-183,226-297,
layers/linear.rs, layers/embed_head.rs) restated with torch for everything
that is NOT one of the path's kernels: the projections are cuBLAS GEMMs.  Per
layer the attention hot path is two nvkv launches, nvkv_qknorm_rope
(split_qkv + q/k RMSNorm + RoPE + KV-cache store, fused) and
nvkv_paged_attention (split-KV decode or tcgen05 prefill), and the epilogues
around it are nvkv's fused residual RMSNorm (x2) and SiLU*mul.  At tp > 1
each all-reduce and the RMSNorm after it are one nvkv kernel over NVLink
peer memory (nvkv_allreduce_rms_norm); with peer_allreduce=False they are an
NCCL all-reduce (torch.distributed) followed by nvkv_rms_norm.  The greedy
pick and the logit all-gather stay on torch.distributed.

Tensor-parallel layout (one process per GPU), as the reference shards it:
  * qkv_proj   column-parallel, local rows [q_r ; k_r ; v_r]  (linear.rs:214-281)
  * o_proj     row-parallel + all-reduce                      (linear.rs:153-212)
  * gate_up    merged column-parallel [gate_r ; up_r]          (linear.rs:78-151)
  * down_proj  row-parallel + all-reduce
  * embedding  vocab-parallel, masked lookup + all-reduce      (embed_head.rs:47-60)
  * lm_head    vocab-parallel, all-gather of the logit shards  (embed_head.rs:89-119)
Weights are random-initialised from a seed per tensor (no checkpoints exist
here); every rank draws the same full tensor and keeps its shard, so any TP
degree computes the same model.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import List, Optional

import torch
import torch.distributed as dist

from qwen3_config import QWEN3_0_6B, QWEN3_4B, QWEN3_8B, QWEN3_32B, Qwen3Config  # noqa: F401

from . import ops


# ---------------------------------------------------------------------------
# TP sharding helpers (pure host logic; unit-tested with gloo on CPU)
# ---------------------------------------------------------------------------

def divide(n: int, tp: int) -> int:
    if n % tp:
        raise ValueError(f"{n} is not divisible by tp={tp}")  # qwen3.rs:61,65
    return n // tp


def shard_qkv(wq: torch.Tensor, wk: torch.Tensor, wv: torch.Tensor, rank: int, tp: int):
    """QKVParallelLinear::weight_loader (linear.rs:253-280): rank r keeps the
    r-th slice of each of q, k, v along the output dim, fused [q;k;v]."""
    q = wq.narrow(0, rank * divide(wq.size(0), tp), divide(wq.size(0), tp))
    k = wk.narrow(0, rank * divide(wk.size(0), tp), divide(wk.size(0), tp))
    v = wv.narrow(0, rank * divide(wv.size(0), tp), divide(wv.size(0), tp))
    return torch.cat([q, k, v], 0).contiguous()


def shard_merged(ws: List[torch.Tensor], rank: int, tp: int) -> torch.Tensor:
    """MergedColumnParallelLinear (linear.rs:109-151): [gate_r ; up_r]."""
    return torch.cat([w.narrow(0, rank * divide(w.size(0), tp), divide(w.size(0), tp))
                      for w in ws], 0).contiguous()


def shard_row(w: torch.Tensor, rank: int, tp: int) -> torch.Tensor:
    """RowParallelLinear::weight_loader (linear.rs:173-185): input-dim slice."""
    n = divide(w.size(1), tp)
    return w.narrow(1, rank * n, n).contiguous()


def shard_vocab(w: torch.Tensor, rank: int, tp: int) -> torch.Tensor:
    """VocabParallelEmbedding::weight_loader (embed_head.rs:42-45)."""
    n = divide(w.size(0), tp)
    return w.narrow(0, rank * n, n).contiguous()


def vocab_parallel_embed(ids: torch.Tensor, w_local: torch.Tensor, rank: int, group=None):
    """embed_head.rs:47-60: masked local lookup, then sum over ranks."""
    n = w_local.size(0)
    start = rank * n
    mask = (ids >= start) & (ids < start + n)
    y = torch.nn.functional.embedding((ids - start) * mask, w_local) * mask.unsqueeze(-1)
    if dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(y, group=group)
    return y


def gather_logits(local: torch.Tensor, group=None) -> torch.Tensor:
    """gather_concat (dist_util.rs:145-159): all-gather the vocab shards and
    concatenate along the vocab dim."""
    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return local
    ws = dist.get_world_size(group)
    parts = [torch.empty_like(local) for _ in range(ws)]
    dist.all_gather(parts, local.contiguous(), group=group)
    return torch.cat(parts, dim=-1)


def vocab_parallel_argmax(local: torch.Tensor, rank: int, group=None) -> torch.Tensor:
    """Greedy token of vocab-sharded logits without gathering them: each rank
    takes its shard's max and first arg-max, one (value, global index) pair per
    row is all-gathered, and the largest value wins, ties going to the lowest
    index -- exactly argmax over the concatenated logits (gather_logits) at
    T x 16 bytes per rank instead of T x V/tp x 4."""
    v, i = local.max(dim=-1)
    return vocab_parallel_pick(v, i + rank * local.size(-1), group)


def vocab_parallel_pick(v: torch.Tensor, gi: torch.Tensor, group=None) -> torch.Tensor:
    """The row-wise winner over the ranks' (value, global index) candidates:
    the largest value, ties to the lowest index."""
    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return gi
    ws = dist.get_world_size(group)
    pair = torch.stack([v.double(), gi.double()], dim=-1)
    parts = [torch.empty_like(pair) for _ in range(ws)]
    dist.all_gather(parts, pair, group=group)
    allp = torch.stack(parts, 0)  # [ws, T, 2]
    vals, idx = allp[..., 0], allp[..., 1]
    best = vals.max(0).values
    pick = torch.where(vals == best, idx, torch.full_like(idx, float("inf"))).min(0).values
    return pick.long()


# ---------------------------------------------------------------------------
# Step metadata on the device (what ModelRunner::prepare_model_input uploads)
# ---------------------------------------------------------------------------

@dataclass
class Step:
    input_ids: torch.Tensor     # [T] int64
    positions: torch.Tensor     # [T] int64
    slot_mapping: torch.Tensor  # [T] int64
    cu_seqlens_q: torch.Tensor  # [B+1] int32
    cu_seqlens_k: torch.Tensor  # [B+1] int32
    block_tables: torch.Tensor  # [B, W] int32
    last_idx: torch.Tensor      # [B] int64: row of each sequence's last token
    max_seqlen_q: int
    max_seqlen_k: int
    prompt_kv_tokens: int = 0   # fp8 pool: >= sum of k_len over the q_len > 1 sequences


class Qwen3TP:
    """One rank of a TP-sharded Qwen3 decoder whose attention is the nvkv path."""

    def __init__(self, cfg: Qwen3Config, rank: int = 0, tp: int = 1, seed: int = 0,
                 dtype=torch.bfloat16, device="cuda", init_scale: float = 1.0, group=None,
                 embed_std: float = 1.0, head_std: Optional[float] = None,
                 peer_allreduce: bool = True, max_tokens: int = 4096, comm=None):
        """peer_allreduce (tp > 1): every all-reduce + the RMSNorm after it is one
        nvkv kernel over NVLink peer memory (nvkv.comm.PeerComm) instead of an
        NCCL call followed by nvkv_rms_norm; max_tokens bounds the tokens of a
        step on that route.  `comm` hands in an existing PeerComm of the same
        ranks (kept open by its owner) instead of creating one.  With tp == 1
        the model makes no collective call, even inside a multi-rank job."""
        self.cfg, self.rank, self.tp, self.group = cfg, rank, tp, group
        self.dtype, self.device = dtype, torch.device(device)
        self.hq = divide(cfg.num_attention_heads, tp)
        self.hkv = divide(cfg.num_key_value_heads, tp)
        self.ffn = divide(cfg.intermediate_size, tp)
        self.scale = cfg.head_dim ** -0.5  # qwen3.rs:71
        self._seed = seed
        self._n = 0
        H, D = cfg.hidden_size, cfg.head_dim

        def full(rows, cols, std):
            self._n += 1
            g = torch.Generator(device=self.device).manual_seed(seed * 1000003 + self._n)
            return (torch.randn(rows, cols, generator=g, device=self.device) * std).to(dtype)

        def norm_w(n):
            self._n += 1
            g = torch.Generator(device=self.device).manual_seed(seed * 1000003 + self._n)
            return (1.0 + 0.1 * torch.randn(n, generator=g, device=self.device)).to(dtype)

        s_in = init_scale / math.sqrt(H)
        emb = full(cfg.vocab_size, H, embed_std)
        self.embed = shard_vocab(emb, rank, tp)
        self.layers = []
        for _ in range(cfg.num_hidden_layers):
            L = {}
            wq = full(cfg.num_attention_heads * D, H, s_in)
            wk = full(cfg.num_key_value_heads * D, H, s_in)
            wv = full(cfg.num_key_value_heads * D, H, s_in)
            L["qkv"] = shard_qkv(wq, wk, wv, rank, tp)
            del wq, wk, wv
            L["o"] = shard_row(full(H, cfg.num_attention_heads * D,
                                    init_scale / math.sqrt(cfg.num_attention_heads * D)), rank, tp)
            L["gate_up"] = shard_merged([full(cfg.intermediate_size, H, s_in),
                                         full(cfg.intermediate_size, H, s_in)], rank, tp)
            L["down"] = shard_row(full(H, cfg.intermediate_size,
                                       init_scale / math.sqrt(cfg.intermediate_size)), rank, tp)
            L["ln1"], L["ln2"] = norm_w(H), norm_w(H)
            L["qn"], L["kn"] = norm_w(D), norm_w(D)
            self.layers.append(L)
        self.norm = norm_w(H)
        lm = emb if cfg.tie_word_embeddings else full(cfg.vocab_size, H,
                                                       s_in if head_std is None else head_std)
        self.lm_head = shard_vocab(lm, rank, tp)  # tie_weights (qwen3.rs:334-338)
        del emb, lm
        self.k_caches: List[torch.Tensor] = []
        self.v_caches: List[torch.Tensor] = []
        self.k_scales: List[torch.Tensor] = []  # fp8 pool only: [Nb, Hkv, P] f32
        self.v_scales: List[torch.Tensor] = []
        self.kv_fp8 = False
        self._bufs = {}
        self.comm = None
        self._own_comm = False
        if tp > 1 and comm is not None:
            self.comm = comm
        elif tp > 1 and peer_allreduce:
            self._own_comm = True
            from .comm import PeerComm
            self.comm = PeerComm(rank, tp, max_tokens * H * torch.tensor([], dtype=dtype)
                                 .element_size(), group=group)

    def close(self) -> None:
        """Releases the peer communicator (after every rank's last step)."""
        if self.comm is not None and self._own_comm:
            self.comm.close()
        self.comm = None

    # ---- KV pool (model_runner.rs:286-303): per layer [Nb, P, Hkv/tp, D] ----
    def allocate_kv_cache(self, num_blocks: int, block_size: int = 256, fill_random: bool = False,
                          seed: int = 1, kv_fp8: bool = False) -> None:
        """kv_fp8: the optional e4m3 pool (codes [Nb, P, Hkv, D] uint8 + f32 row
        scales [Nb, Hkv, P], nvkv_store_kvcache_fp8 / nvkv_paged_attention_fp8)
        instead of the model dtype.  fill_random fills the pool with random
        rows (through the fp8 store for an fp8 pool)."""
        shape = (num_blocks, block_size, self.hkv, self.cfg.head_dim)
        self.k_caches, self.v_caches, self.k_scales, self.v_scales = [], [], [], []
        self.kv_fp8 = kv_fp8
        g = torch.Generator(device=self.device).manual_seed(seed * 7919 + self.rank)
        slots = torch.arange(num_blocks * block_size, device=self.device) if kv_fp8 else None
        for _ in range(self.cfg.num_hidden_layers):
            if kv_fp8:
                k = torch.zeros(shape, device=self.device, dtype=torch.uint8)
                v = torch.zeros_like(k)
                ks = torch.zeros(num_blocks, self.hkv, block_size, device=self.device)
                vs = torch.zeros_like(ks)
                if fill_random:
                    for lo in range(0, num_blocks, 64):  # bounded temporaries
                        n = min(64, num_blocks - lo)
                        rk = torch.randn((n * block_size,) + shape[2:], generator=g,
                                         device=self.device, dtype=self.dtype)
                        rv = torch.randn_like(rk)
                        ops.store_kvcache_fp8(rk, rv, k, v, ks, vs,
                                              slots[lo * block_size:(lo + n) * block_size])
                self.k_scales.append(ks)
                self.v_scales.append(vs)
            elif fill_random:
                k = torch.randn(shape, generator=g, device=self.device, dtype=self.dtype)
                v = torch.randn(shape, generator=g, device=self.device, dtype=self.dtype)
            else:
                k = torch.zeros(shape, device=self.device, dtype=self.dtype)
                v = torch.zeros(shape, device=self.device, dtype=self.dtype)
            self.k_caches.append(k)
            self.v_caches.append(v)

    def _attend(self, li: int, qkv: torch.Tensor, st: "Step", q_buf, o_buf, ws) -> None:
        """One layer's attention hot path: the q/k-norm + RoPE prologue with the
        KV-cache store, then paged attention (qwen3.rs:128-145), over the
        model-dtype pool (the store fused into the prologue) or the fp8 pool
        (prologue, fp8 store, fp8 attention)."""
        cfg, D, eps = self.cfg, self.cfg.head_dim, self.cfg.rms_norm_eps
        L = self.layers[li]
        if not self.kv_fp8:
            ops.qknorm_rope(qkv, st.positions, self.hq, self.hkv, L["qn"], L["kn"], eps,
                            cfg.rope_theta, cfg.max_position_embeddings, D,
                            k_cache=self.k_caches[li], v_cache=self.v_caches[li],
                            slot_mapping=st.slot_mapping, q_out=q_buf)
            ops.paged_attention(q_buf, self.k_caches[li], self.v_caches[li], st.cu_seqlens_q,
                                st.cu_seqlens_k, st.block_tables, st.max_seqlen_q,
                                st.max_seqlen_k, self.scale, out=o_buf, workspace=ws)
            return
        _, k_out, v_out = ops.qknorm_rope(qkv, st.positions, self.hq, self.hkv, L["qn"],
                                          L["kn"], eps, cfg.rope_theta,
                                          cfg.max_position_embeddings, D, want_kv=True,
                                          q_out=q_buf)
        ops.store_kvcache_fp8(k_out, v_out, self.k_caches[li], self.v_caches[li],
                              self.k_scales[li], self.v_scales[li], st.slot_mapping)
        ops.paged_attention_fp8(q_buf, self.k_caches[li], self.v_caches[li], self.k_scales[li],
                                self.v_scales[li], st.cu_seqlens_q, st.cu_seqlens_k,
                                st.block_tables, st.max_seqlen_q, st.max_seqlen_k, self.scale,
                                prompt_kv_tokens=st.prompt_kv_tokens, out=o_buf, workspace=ws)

    def _ws(self, st: "Step") -> torch.Tensor:
        B = st.cu_seqlens_q.numel() - 1
        if self.kv_fp8:
            n = ops.workspace_size_fp8(B, self.hq, self.hkv, st.max_seqlen_q, st.max_seqlen_k,
                                       st.prompt_kv_tokens, self.cfg.head_dim)
        else:
            n = ops.workspace_size(B, self.hq, self.hkv, st.max_seqlen_q, st.max_seqlen_k,
                                   self.cfg.head_dim)
        return self._buf("ws", (max(n, 16),), torch.uint8)

    def _buf(self, name, shape, dtype=None):
        b = self._bufs.get(name)
        if b is None or b.shape != torch.Size(shape):
            b = torch.empty(shape, device=self.device, dtype=dtype or self.dtype)
            self._bufs[name] = b
        return b

    def _all_reduce(self, x):
        if self.tp > 1:
            dist.all_reduce(x, group=self.group)
        return x

    @torch.no_grad()
    def forward(self, st: Step) -> torch.Tensor:
        """Qwen3ForCausalLM::forward + compute_logits (qwen3.rs:285-297,
        embed_head.rs:89-119): returns the full-vocab logits of each
        sequence's last token, [B, V], in the model dtype."""
        local = self._local_logits(st)
        return gather_logits(local, self.group) if self.tp > 1 else local

    @torch.no_grad()
    def greedy(self, st: Step) -> torch.Tensor:
        """The greedy next token of every sequence, [B] int64: argmax of
        forward()'s logits, taken vocab-parallel (vocab_parallel_argmax)."""
        local = self._local_logits(st)
        if self.tp == 1:
            return local.argmax(dim=-1)
        return vocab_parallel_argmax(local, self.rank, self.group)

    def sample(self, st: Step, temperatures: torch.Tensor, seed: int, step: int,
               step_device: Optional[torch.Tensor] = None) -> torch.Tensor:
        """The sampled next token of every sequence, [B] int64: the
        reference's Sampler::forward (layers/sampler.rs:7-21) over forward()'s
        logits, as nvkv_sample's Gumbel-max scores on this rank's vocab shard
        and the vocab-parallel pick of the winner (no logits gathered).
        temperatures [B] f32 on the device (<= 0: greedy); step_device: an
        int64 [1] device counter added to `step` (for graph replays)."""
        local = self._local_logits(st)
        v, gi = ops.sample(local, temperatures, seed, step, vocab_offset=self.rank * local.size(-1),
                           step_device=step_device)
        return gi if self.tp == 1 else vocab_parallel_pick(v, gi, self.group)

    def _local_logits(self, st: Step) -> torch.Tensor:
        """This rank's vocab shard of the last-token logits, [B, V/tp], model dtype."""
        if self.comm is not None:
            return self._local_logits_peer(st)
        cfg = self.cfg
        T = st.input_ids.numel()
        D = cfg.head_dim
        if self.tp > 1:
            h = vocab_parallel_embed(st.input_ids, self.embed, self.rank, self.group)
        else:
            h = torch.nn.functional.embedding(st.input_ids, self.embed)
        q_buf = self._buf("q", (T, self.hq, D))
        o_buf = self._buf("o", (T, self.hq, D))
        ws = self._ws(st)
        xb = self._buf("x", (T, cfg.hidden_size))
        actb = self._buf("act", (T, self.ffn))
        eps = cfg.rms_norm_eps
        residual = None
        for li, L in enumerate(self.layers):
            # input_layernorm: forward on the first layer, residual_forward after
            # (qwen3.rs:232-238); the residual is updated in place to h + residual
            if residual is None:
                x, residual = ops.rms_norm(h, L["ln1"], eps, out=xb), h
            else:
                x = ops.rms_norm(h, L["ln1"], eps, residual=residual, out=xb)
            qkv = torch.matmul(x, L["qkv"].t())
            self._attend(li, qkv, st, q_buf, o_buf, ws)
            a = self._all_reduce(torch.matmul(o_buf.view(T, -1), L["o"].t()))
            x = ops.rms_norm(a, L["ln2"], eps, residual=residual, out=xb)
            gu = torch.matmul(x, L["gate_up"].t())
            act = ops.silu_and_mul(gu, out=actb)
            h = self._all_reduce(torch.matmul(act, L["down"].t()))
        h = ops.rms_norm(h, self.norm, eps, residual=residual, out=xb)  # qwen3.rs:295
        last = h.index_select(0, st.last_idx)
        # logits in the model dtype, as the reference's lm_head matmul gives
        # them (embed_head.rs:113); its sampler widens them to f32 afterwards
        return torch.mm(last, self.lm_head.t())

    def _local_logits_peer(self, st: Step) -> torch.Tensor:
        """_local_logits with every all-reduce fused into the RMSNorm after it:
        the producers (masked embedding lookup, o_proj, down_proj) write their
        partial sums into the communicator's input buffer, and one kernel
        all-reduces them, updates the residual and normalises
        (qwen3.rs:232-238, 295)."""
        cfg = self.cfg
        T = st.input_ids.numel()
        D = cfg.head_dim
        H = cfg.hidden_size
        eps = cfg.rms_norm_eps
        part = self.comm.input(T, H, self.dtype)
        q_buf = self._buf("q", (T, self.hq, D))
        o_buf = self._buf("o", (T, self.hq, D))
        ws = self._ws(st)
        xb = self._buf("x", (T, H))
        res = self._buf("res", (T, H))
        actb = self._buf("act", (T, self.ffn))
        # embed_head.rs:47-60 without its all-reduce: the masked local lookup
        n = self.embed.size(0)
        start = self.rank * n
        mask = (st.input_ids >= start) & (st.input_ids < start + n)
        torch.mul(torch.nn.functional.embedding((st.input_ids - start) * mask, self.embed),
                  mask.unsqueeze(-1), out=part)
        self.comm.allreduce_rms_norm(T, H, res, self.layers[0]["ln1"], eps, xb, init=True)
        for li, L in enumerate(self.layers):
            qkv = torch.matmul(xb, L["qkv"].t())
            self._attend(li, qkv, st, q_buf, o_buf, ws)
            torch.matmul(o_buf.view(T, -1), L["o"].t(), out=part)
            self.comm.allreduce_rms_norm(T, H, res, L["ln2"], eps, xb)
            gu = torch.matmul(xb, L["gate_up"].t())
            act = ops.silu_and_mul(gu, out=actb)
            torch.matmul(act, L["down"].t(), out=part)
            nxt = self.layers[li + 1]["ln1"] if li + 1 < len(self.layers) else self.norm
            self.comm.allreduce_rms_norm(T, H, res, nxt, eps, xb)
        last = xb.index_select(0, st.last_idx)
        return torch.mm(last, self.lm_head.t())

    def launches_per_step(self, st: Step) -> int:
        """nvkv kernel launches one forward issues: per layer two RMSNorms
        (each fused with the all-reduce before it on the peer route), SiLU*mul,
        the prologue, the decode kernel, the combine kernel when the split-KV
        plan splits, and the prefill work plan + prefill kernel when
        max_seqlen_q > 1 (with an fp8 pool also its store and, for prompts,
        the dequantisation); plus the final norm (on the peer route: the
        embedding's fused call, the final norm being fused into the last
        layer's)."""
        B = st.cu_seqlens_q.numel() - 1
        split = ops.workspace_size(B, self.hq, self.hkv, 1, st.max_seqlen_k) > 0
        per = 5 + (1 if split else 0) + (2 if st.max_seqlen_q > 1 else 0)
        if self.kv_fp8:  # + the fp8 store; prompts: + row offsets and dequantisation
            per += 1 + (2 if st.max_seqlen_q > 1 else 0)
        return per * self.cfg.num_hidden_layers + 1
