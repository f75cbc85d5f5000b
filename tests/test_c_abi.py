"""include/nvkv.h compiles as C99 and a plain C program linked against
libnvkv.so drives the host entry points (block manager, step metadata).
Expected values follow block_manager.rs / model_runner.rs by hand: two
10-token prompts sharing their first 8 tokens at block size 4 share two
pages (8 cached tokens for the second); one decode token each then gives
contexts 11 and 11, positions 10 and 10, and 2 slots in total."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIBDIR = os.path.join(ROOT, "nanovllm-rs_b200", "nvkv")


@pytest.mark.skipif(shutil.which("gcc") is None, reason="no C compiler")
def test_plain_c_caller(tmp_path):
    exe = str(tmp_path / "abi_host")
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Wextra", "-Werror", "-pedantic",
                    "-I" + os.path.join(ROOT, "include"),
                    os.path.join(ROOT, "tests", "c", "abi_host.c"), "-o", exe, "-L" + LIBDIR,
                    "-lnvkv", "-Wl,-rpath," + LIBDIR], check=True, capture_output=True, text=True)
    r = subprocess.run([exe], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, r.stderr
    out = dict(kv.split("=") for kv in r.stdout.split())
    assert out["cached"] == "8" and out["shared"] == "1"
    assert out["done"] == "2" and out["tokens"] == "2" and out["slots"] == "2"
    assert out["cuk"] == "0,11,22" and out["pos"] == "10,10"
