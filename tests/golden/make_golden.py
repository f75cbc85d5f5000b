"""Generates the committed known-answer fixtures under tests/golden/.

Run from the repository root:  python tests/golden/make_golden.py

repro_kat.npz -- KAT-1, the reference's own paged-attention probe
  (nanovllm_rs/src/bin/repro.rs) restated independently of ``oracle/``:
  * the deterministic generator of repro.rs:50-63 (28 "layers", f32 math then
    bf16), recorded as bf16 storage bits;
  * the expected cache rows after the two store calls of repro.rs:81-86
    (``k_full``/``v_full``, which repro.rs:116-121 checks with
    ``cache_write_diff``);
  * the expected attention output of repro.rs's ``manual_attention``
    (repro.rs:6-32: f32 q.k^T * scale, softmax, p.v, GQA by broadcasting each
    kv head over its query-head group), in float32.

slot_mapping_kat.json -- KAT-2, hand-computed ``prepare_model_input`` cases
  (engine/model_runner.rs:82-131) with block size 4.  The expected arrays are
  literals worked out by hand from the loop at model_runner.rs:108-124; this
  script only copies them into the JSON file.
"""
import json
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))

N_HEADS, N_KV_HEADS, HEAD_DIM, BLOCK, PRIOR = 16, 8, 128, 256, 6


def _bf16_bits_rne(x: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return (((u + ((u >> 16) & 1) + 0x7FFF) >> 16) & 0xFFFF).astype(np.uint16)


def _bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << 16).view(np.float32)


def _mk(seed, n, h):
    i = np.arange(n * h * HEAD_DIM, dtype=np.float32)
    data = (np.fmod(i * np.float32(seed), np.float32(17.0)) - np.float32(8.0)) / np.float32(8.0)
    return _bf16_bits_rne(data).reshape(n, h, HEAD_DIM)


def _manual_attention(q, k, v, scale):
    """repro.rs:6-32 in float32 (q: [1,Hq,D], k/v: [L,Hkv,D])."""
    g = q.shape[1] // k.shape[1]
    qt = q.transpose(1, 0, 2)  # [Hq,1,D]
    kt = np.repeat(k.transpose(1, 0, 2), g, axis=0)  # [Hq,L,D]
    vt = np.repeat(v.transpose(1, 0, 2), g, axis=0)
    s = np.matmul(qt, kt.transpose(0, 2, 1)).astype(np.float32) * np.float32(scale)
    s = s - s.max(axis=-1, keepdims=True)
    p = np.exp(s)
    p = p / p.sum(axis=-1, keepdims=True)
    return np.matmul(p, vt).transpose(1, 0, 2).astype(np.float32)  # [1,Hq,D]


def make_repro():
    out = {}
    scale = np.float32(1.0) / np.sqrt(np.float32(HEAD_DIM))
    for layer in range(28):
        base = np.float32(1.0) + np.float32(layer) * np.float32(0.13)
        kp = _mk(np.float32(0.7) * base, PRIOR, N_KV_HEADS)
        vp = _mk(np.float32(1.3) * base, PRIOR, N_KV_HEADS)
        kn = _mk(np.float32(0.9) * base, 1, N_KV_HEADS)
        vn = _mk(np.float32(1.7) * base, 1, N_KV_HEADS)
        qn = _mk(np.float32(2.1) * base, 1, N_HEADS)
        k_full = np.concatenate([kp, kn], 0)
        v_full = np.concatenate([vp, vn], 0)
        o = _manual_attention(_bits_to_f32(qn), _bits_to_f32(k_full), _bits_to_f32(v_full), scale)
        out[f"l{layer}_k_prior"] = kp
        out[f"l{layer}_v_prior"] = vp
        out[f"l{layer}_k_new"] = kn
        out[f"l{layer}_v_new"] = vn
        out[f"l{layer}_q_new"] = qn
        out[f"l{layer}_manual_out"] = o
    np.savez_compressed(os.path.join(HERE, "repro_kat.npz"), **out)


# Block size 4.  Each case: the Sequence fields and the hand-derived outputs.
SLOT_CASES = {
    "block_size": 4,
    "cases": {
        "A_fresh_prefill_partial_last_block": {
            "len": 10, "num_cached_tokens": 0, "num_new_tokens": 10, "block_table": [7, 2, 5],
            "slots": [28, 29, 30, 31, 8, 9, 10, 11, 20, 21],
            "positions": [0, 1, 2, 3, 4, 5, 6, 7, 8, 9], "need_logits": True},
        "B_decode_inside_block": {
            "len": 11, "num_cached_tokens": 10, "num_new_tokens": 1, "block_table": [11, 3, 14],
            "slots": [58], "positions": [10], "need_logits": True},
        "C_decode_first_slot_of_new_block": {
            "len": 13, "num_cached_tokens": 12, "num_new_tokens": 1, "block_table": [0, 1, 4, 9],
            "slots": [36], "positions": [12], "need_logits": True},
        "D_prefix_cache_hit_two_full_blocks": {
            "len": 10, "num_cached_tokens": 8, "num_new_tokens": 2, "block_table": [12, 13, 6],
            "slots": [24, 25], "positions": [8, 9], "need_logits": True},
        "E_prefill_exact_block_boundary": {
            "len": 8, "num_cached_tokens": 0, "num_new_tokens": 8, "block_table": [3, 15],
            "slots": [12, 13, 14, 15, 60, 61, 62, 63],
            "positions": [0, 1, 2, 3, 4, 5, 6, 7], "need_logits": True},
        "F_cached_mid_block_then_new_block": {
            "len": 9, "num_cached_tokens": 5, "num_new_tokens": 4, "block_table": [8, 10, 16],
            "slots": [41, 42, 43, 64], "positions": [5, 6, 7, 8], "need_logits": True},
        "G_chunked_prefill_first_chunk": {
            "len": 12, "num_cached_tokens": 0, "num_new_tokens": 6, "block_table": [17, 18],
            "slots": [68, 69, 70, 71, 72, 73], "positions": [0, 1, 2, 3, 4, 5], "need_logits": False},
    },
    # One mixed step made of cases B, F, A (decode + partially cached + fresh).
    "batch": {
        "order": ["B_decode_inside_block", "F_cached_mid_block_then_new_block",
                  "A_fresh_prefill_partial_last_block"],
        "cu_seqlens_q": [0, 1, 5, 15],
        "cu_seqlens_k": [0, 11, 20, 30],
        "max_seqlen_q": 10, "max_seqlen_k": 11,
        "slots": [58, 41, 42, 43, 64, 28, 29, 30, 31, 8, 9, 10, 11, 20, 21],
        "block_tables": [[11, 3, 14], [8, 10, 16], [7, 2, 5]],
        "context_lens": [11, 9, 10],
        "seq_need_compute_logits": [0, 1, 2],
    },
}


def make_slots():
    with open(os.path.join(HERE, "slot_mapping_kat.json"), "w") as f:
        json.dump(SLOT_CASES, f, indent=1, sort_keys=True)


if __name__ == "__main__":
    make_repro()
    make_slots()
    print("wrote", sorted(os.listdir(HERE)))
