"""KV-pool sizing (nvkv_kv_pool_blocks) against the reference's formula
(engine/model_runner.rs:264-284), restated here in Python integers."""
import random

import pytest

from nvkv import NvkvError
from nvkv._lib import ERR_CUDA, ERR_INVALID_ARG, lib
from nvkv.blocks import kv_pool_blocks


def _reference(free, total, util, layers, bs, hkv, d, nbytes):
    block = 2 * layers * bs * hkv * d * nbytes
    budget = int(total * util) - (total - free)  # f64 product truncated toward zero
    return max(budget // block, 0) if budget > 0 else 0


def test_b200_qwen3_8b_tp1():
    total = 183359 * 2 ** 20  # nvidia-smi's B200 memory
    free = total - 20 * 2 ** 30  # 20 GiB taken by weights and activations
    n = kv_pool_blocks(free, total, 0.9, 36, 256, 8, 128, 2)
    assert n == _reference(free, total, 0.9, 36, 256, 8, 128, 2)
    assert n * 256 >= 256 * 1536  # the 8B bench pool (256 x 1536 tokens) fits


def test_random_inputs_match_formula():
    rng = random.Random(5)
    for _ in range(2000):
        total = rng.randrange(1, 1 << 40)
        free = rng.randrange(0, total + 1)
        util = rng.choice([0.5, 0.8, 0.9, 0.95, 1.0, rng.random() or 0.1])
        args = (rng.randrange(1, 100), rng.choice([16, 128, 256]), rng.randrange(1, 9),
                rng.choice([64, 128]), rng.choice([1, 2, 4]))
        want = _reference(free, total, util, *args)
        if want > 0:
            assert kv_pool_blocks(free, total, util, *args) == want
        else:
            with pytest.raises(NvkvError):  # the reference asserts
                kv_pool_blocks(free, total, util, *args)


def test_bad_arguments():
    with pytest.raises(NvkvError):
        kv_pool_blocks(10, 5, 0.9, 1, 1, 1, 1, 1)  # free > total
    with pytest.raises(NvkvError):
        kv_pool_blocks(5, 10, 1.5, 1, 1, 1, 1, 1)


def test_probe_without_a_device_fails_cleanly():
    import ctypes
    import torch
    if torch.cuda.is_available():
        pytest.skip("a device is present")
    out = ctypes.c_int64(0)
    assert lib.nvkv_kv_pool_probe(0.9, 36, 256, 8, 128, 2, ctypes.byref(out)) in (ERR_CUDA,
                                                                               ERR_INVALID_ARG)
