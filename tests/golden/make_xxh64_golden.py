"""Writes tests/golden/xxh64_kat.json: XXH64 (seed 0) known answers from an
independent implementation (the ``xxhash`` Python package, a binding of the
xxHash C library), to pin the block-hash restatements: the pure-Python one in
oracle/block_manager_oracle.py and the C++ one behind nvkv_block_hash.

* "bytes": raw inputs of every length 0..80 and a few long ones (the 1..3-
  byte, 4-byte, 8-byte and 32-byte-stripe paths of the algorithm).
* "block_hash": BlockManager::compute_hash cases (block_manager.rs:53-64):
  token ids and a prefix hash (-1 = none), each as a little-endian i64, the
  digest reinterpreted as i64.

    python tests/golden/make_xxh64_golden.py
"""
import json
import os
import random
import struct

import xxhash


def block_hash(tokens, prefix):
    buf = (struct.pack("<q", prefix) if prefix != -1 else b"") + struct.pack(
        f"<{len(tokens)}q", *tokens)
    d = xxhash.xxh64(buf, seed=0).intdigest()
    return d - (1 << 64) if d >= (1 << 63) else d


def main():
    rng = random.Random(2024)
    raw = []
    for n in list(range(81)) + [100, 255, 256, 257, 1000, 2056]:
        data = bytes(rng.randrange(256) for _ in range(n))
        raw.append({"hex": data.hex(), "xxh64": xxhash.xxh64(data, seed=0).intdigest()})
    blocks = []
    prefix = -1
    for n in (0, 1, 2, 3, 4, 5, 16, 256, 256, 256, 128):
        tokens = [rng.randrange(151936) for _ in range(n)]
        h = block_hash(tokens, prefix)
        blocks.append({"tokens": tokens, "prefix": prefix, "hash": h})
        prefix = h if n == 256 else rng.choice([-1, rng.randrange(-(1 << 63), 1 << 63)])
    out = {"algorithm": "XXH64 seed 0", "generator": "python xxhash " + xxhash.VERSION,
           "bytes": raw, "block_hash": blocks}
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "xxh64_kat.json")
    with open(path, "w") as f:
        json.dump(out, f, separators=(",", ":"))
    print(path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    main()
