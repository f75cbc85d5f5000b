"""The greedy-stream gate can only catch attention bugs if the stream depends
on attention.  On the CPU, with a small Qwen3-shaped model initialised the
way tests/test_gpu_greedy.py initialises its model (small embedding, untied
lm_head with std 1), planting a mistake in the oracle's attention must
change most of the stream."""
import numpy as np

import nvkv_oracle as O
import qwen3_cpu as Q
from qwen3_config import Qwen3Config

CFG = Qwen3Config(256, 2, 4, 2, 512, vocab_size=2000)
P = 256


def _weights(seed=0, embed_std=0.05, head_std=1.0):
    rng = np.random.default_rng(seed)
    H, D, F = CFG.hidden_size, CFG.head_dim, CFG.intermediate_size
    hq, hkv = CFG.num_attention_heads, CFG.num_key_value_heads
    r = lambda *s, std: (rng.standard_normal(s) * std).astype(np.float32)  # noqa: E731
    w = {"embed": r(CFG.vocab_size, H, std=embed_std), "norm": np.ones(H, np.float32),
         "lm_head": r(CFG.vocab_size, H, std=head_std)}
    for i in range(CFG.num_hidden_layers):
        w.update({f"{i}.qkv": r((hq + 2 * hkv) * D, H, std=H ** -0.5),
                  f"{i}.o": r(H, hq * D, std=(hq * D) ** -0.5),
                  f"{i}.gate_up": r(2 * F, H, std=H ** -0.5), f"{i}.down": r(H, F, std=F ** -0.5),
                  f"{i}.ln1": np.ones(H, np.float32), f"{i}.ln2": np.ones(H, np.float32),
                  f"{i}.qn": np.ones(D, np.float32), f"{i}.kn": np.ones(D, np.float32)})
    return w


def _streams(w):
    rng = np.random.default_rng(5)
    free = list(range(12))[::-1]
    seqs = [O.Seq(rng.integers(0, CFG.vocab_size, L).tolist(),
                  [free.pop() for _ in range((L + P - 1) // P)], 0, L, P) for L in (70, 200)]
    return Q.greedy_generate(Q.Qwen3CPU(CFG, w, 12, P), seqs, 12, free)


def test_stream_depends_on_attention(monkeypatch):
    w = _weights()
    good = _streams(w)
    real = O.causal_attention_one

    def first_key_only(q, k, v, scale, causal=True, acc=np.float64):  # planted mistake
        return real(q, k[:1], v[:1], scale, False, acc)

    monkeypatch.setattr(O, "causal_attention_one", first_key_only)
    bad = _streams(w)
    diff = np.mean([a != b for g, h in zip(good, bad) for a, b in zip(g, h)])
    assert diff >= 0.5, (diff, good, bad)
    # the stream is not a trivial repetition of one token
    assert max(len(set(s)) for s in good) > 1
