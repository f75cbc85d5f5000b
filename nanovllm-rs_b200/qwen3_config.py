"""Qwen3 architecture shapes the benchmark and tests run (config.rs:5-27).

Plain data, no torch and no native library: the CPU measurements (the
oracle-driven reference arm of bench.py) import these shapes without loading
libnvkv.so.  nvkv.decoder re-exports them.
"""
from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class Qwen3Config:
    """The config.json fields the reference reads (config.rs:5-27)."""

    hidden_size: int
    num_hidden_layers: int
    num_attention_heads: int
    num_key_value_heads: int
    intermediate_size: int
    vocab_size: int = 151936
    head_dim: int = 128
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1e6
    max_position_embeddings: int = 40960
    tie_word_embeddings: bool = False


QWEN3_0_6B = Qwen3Config(1024, 28, 16, 8, 3072, tie_word_embeddings=True)
QWEN3_4B = Qwen3Config(2560, 36, 32, 8, 9728, tie_word_embeddings=True)
QWEN3_8B = Qwen3Config(4096, 36, 32, 8, 12288)
QWEN3_32B = Qwen3Config(5120, 64, 64, 8, 25600)
