"""The C ABI library loads and exports every symbol include/nvkv.h declares;
host-side validation rejects bad arguments before anything reaches a GPU."""
import ctypes
import os
import re

import pytest

from conftest import ROOT


def _declared():
    src = open(os.path.join(ROOT, "include", "nvkv.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(nvkv_[a-z0-9_]+)\s*\(", src)))


def test_header_declares_expected_surface():
    names = _declared()
    for n in ("nvkv_store_kvcache", "nvkv_qknorm_rope", "nvkv_paged_attention",
              "nvkv_paged_attention_workspace_size", "nvkv_context_set", "nvkv_attention_forward"):
        assert n in names


def test_library_exports_every_declared_symbol():
    import nvkv
    lib = ctypes.CDLL(nvkv.LIB_PATH)
    missing = [n for n in _declared() if not hasattr(lib, n)]
    assert not missing, missing
    from nvkv._lib import SIGNATURES
    assert sorted(SIGNATURES) == _declared()


def test_version_and_empty_error():
    import nvkv
    assert nvkv.lib.nvkv_version() >= 100
    assert nvkv.lib.nvkv_last_error() == b""


def test_store_rejects_bad_dtype_and_sizes():
    from nvkv._lib import lib, ERR_UNSUPPORTED, ERR_INVALID_ARG, OK
    p = ctypes.c_void_p(16)
    assert lib.nvkv_store_kvcache(p, p, p, p, p, 4, 128, 128, 128, 10, 7, None) == ERR_UNSUPPORTED
    assert b"dtype" in lib.nvkv_last_error()
    assert lib.nvkv_store_kvcache(p, p, p, p, p, -1, 128, 128, 128, 10, 1, None) == ERR_INVALID_ARG
    assert lib.nvkv_store_kvcache(p, p, p, p, p, 4, 128, 64, 128, 10, 1, None) == ERR_INVALID_ARG
    assert b"stride" in lib.nvkv_last_error()
    # zero tokens is a no-op, exactly like kv_cache.rs:128-130
    assert lib.nvkv_store_kvcache(None, None, None, None, None, 0, 128, 128, 128, 10, 1, None) == OK


def test_attention_validation():
    from nvkv._lib import lib, ERR_UNSUPPORTED, ERR_INVALID_ARG, ERR_ALIGNMENT, ERR_WORKSPACE
    p = ctypes.c_void_p(1 << 20)
    args = lambda **kw: dict(dict(q=p, qs=32 * 128, T=64, k=p, v=p, nb=16, kvs=0, out=p, cq=p,
                                  ck=p, bt=p, bts=16, B=64, mq=1, mk=4096, hq=32, hkv=8, d=128,
                                  page=256, scale=0.088, causal=1, ws=None, wsb=0, dt=1), **kw)

    def call(a):
        return lib.nvkv_paged_attention(a["q"], a["qs"], a["T"], a["k"], a["v"], a["nb"], a["kvs"],
                                        a["out"], a["cq"], a["ck"], a["bt"], a["bts"], a["B"],
                                        a["mq"], a["mk"], a["hq"], a["hkv"], a["d"], a["page"],
                                        ctypes.c_float(a["scale"]), a["causal"], a["ws"],
                                        a["wsb"], a["dt"], None)

    assert call(args(d=64)) == ERR_UNSUPPORTED
    assert call(args(hq=30)) == ERR_INVALID_ARG
    assert call(args(hq=8 * 17)) == ERR_UNSUPPORTED  # group > 16
    assert call(args(page=96)) == ERR_UNSUPPORTED
    assert call(args(bts=4)) == ERR_INVALID_ARG  # 4096 keys need 16 pages
    assert call(args(q=ctypes.c_void_p((1 << 20) + 8))) == ERR_ALIGNMENT
    assert call(args(kvs=100)) == ERR_INVALID_ARG
    assert call(args(B=0)) == 0  # empty batch: nothing to do
    # 64 sequences x 8 kv heads with 4096 keys: the split-KV plan needs scratch
    need = ctypes.c_size_t(0)
    assert lib.nvkv_paged_attention_workspace_size(64, 16, 8, 128, 1, 4096, ctypes.byref(need)) == 0
    assert need.value > 0
    assert call(args(hq=16, ws=None, wsb=0)) == ERR_WORKSPACE
    assert b"workspace" in lib.nvkv_last_error()


def test_workspace_zero_when_no_split():
    from nvkv._lib import lib
    need = ctypes.c_size_t(123)
    # 256 x 8 work items fill the GPU without splitting
    assert lib.nvkv_paged_attention_workspace_size(256, 32, 8, 128, 1, 1536, ctypes.byref(need)) == 0
    assert need.value == 0


def test_workspace_holds_prefill_plan():
    """A call that may prefill (max_seqlen_q > 1) needs room for the prefill
    work plan even when the decode plan does not split; the plan grows with
    the batch (a record per sequence) and with max_seqlen_q (a count per
    128-row q tile), and the decode scratch sits in front of it."""
    from nvkv._lib import lib
    def size(B, max_q, max_k, hq=32, hkv=8):
        need = ctypes.c_size_t(0)
        assert lib.nvkv_paged_attention_workspace_size(B, hq, hkv, 128, max_q, max_k,
                                                       ctypes.byref(need)) == 0
        return need.value
    assert size(256, 1, 1536) == 0
    assert size(256, 2, 1536) > 0
    assert size(4096, 1024, 1536) > size(256, 1024, 1536) >= 256 * 20
    assert size(256, 1 << 20, 1536) - size(256, 1024, 1536) >= 4 * ((1 << 20) - 1024) // 128
    for B, max_k in ((64, 4096), (8, 32768)):  # decode splits: scratch + plan
        dec = size(B, 1, max_k)
        assert dec > 0 and size(B, 512, max_k) >= dec + B * 20


def test_context_and_attention_objects_host_only():
    from nvkv._lib import lib, ERR_INVALID_ARG, OK
    assert lib.nvkv_context_set(None, None, 1, 1, 1, None, 0, None, None, 0) == ERR_INVALID_ARG
    assert lib.nvkv_context_reset() == OK
    h = ctypes.c_void_p()
    assert lib.nvkv_attention_create(ctypes.c_float(0.1), ctypes.byref(h)) == OK and h.value
    # forward without a context: "cu_seqlens_q must be set" (attention.rs:26)
    assert lib.nvkv_attention_forward(h, None, 0, None, 0, None, 0, 1, 8, 8, None, 1, None) \
        == ERR_INVALID_ARG
    assert b"cu_seqlens_q" in lib.nvkv_last_error()
    assert lib.nvkv_attention_set_kv_cache(h, None, None, 1, 256, 8, 128, 1) == ERR_INVALID_ARG
    assert lib.nvkv_attention_destroy(h) == OK


def test_qknorm_validation():
    from nvkv._lib import lib, ERR_UNSUPPORTED, ERR_INVALID_ARG, ERR_ALIGNMENT
    p = ctypes.c_void_p(1 << 20)

    def call(d=128, qw=p, kw=p, kc=None, qkv=p, stride=6144):
        return lib.nvkv_qknorm_rope(qkv, stride, 4, 32, 8, d, p, qw, kw, ctypes.c_float(1e-6),
                                    ctypes.c_float(1e6), 40960, p, None, None, kc, None, None, 0,
                                    1, None)

    assert call(d=64) == ERR_UNSUPPORTED
    assert call(kw=None) == ERR_INVALID_ARG
    assert call(kc=p) == ERR_INVALID_ARG  # cache without v_cache / slot_mapping
    assert call(stride=100) == ERR_INVALID_ARG
    assert call(qkv=ctypes.c_void_p((1 << 20) + 2)) == ERR_ALIGNMENT


def test_comm_validation_host_only():
    """nvkv_comm_* / nvkv_allreduce_rms_norm reject bad arguments before any
    device call."""
    from nvkv._lib import lib, ERR_INVALID_ARG, OK
    h = ctypes.c_void_p()
    buf = ctypes.create_string_buffer(64)
    assert lib.nvkv_comm_create(2, 2, 1 << 20, ctypes.byref(h), buf) == ERR_INVALID_ARG
    assert lib.nvkv_comm_create(0, 9, 1 << 20, ctypes.byref(h), buf) == ERR_INVALID_ARG
    assert lib.nvkv_comm_create(0, 2, 0, ctypes.byref(h), buf) == ERR_INVALID_ARG
    assert lib.nvkv_comm_create(0, 2, 1 << 20, None, buf) == ERR_INVALID_ARG
    assert b"rank" in lib.nvkv_last_error() or b"null" in lib.nvkv_last_error()
    assert lib.nvkv_allreduce_rms_norm(None, 4, 4096, None, 0, None, 1e-6, None, 1,
                                       None) == ERR_INVALID_ARG
    assert lib.nvkv_comm_set_timeout(None, 1) == ERR_INVALID_ARG
    assert lib.nvkv_comm_destroy(None) == OK


def test_decode_advance_validation_host_only():
    from nvkv._lib import lib, ERR_INVALID_ARG, OK
    assert lib.nvkv_decode_advance(-1, 256, None, None, 1, 1, None, None, None, None,
                                   None) == ERR_INVALID_ARG
    assert lib.nvkv_decode_advance(4, 0, None, None, 1, 1, None, None, None, None,
                                   None) == ERR_INVALID_ARG
    assert lib.nvkv_decode_advance(4, 256, None, None, 1, 1, None, None, None, None,
                                   None) == ERR_INVALID_ARG
    assert lib.nvkv_decode_advance(0, 256, None, None, 1, 1, None, None, None, None, None) == OK


def test_decode_plan_one_wave_rule():
    """The split-KV plan, seen through the workspace query: a batch whose
    (sequence, kv head) items fill >= 80 % of a 296-CTA wave with contexts of
    at most 48 tiles (3072 keys) is not split (no workspace); longer contexts
    or fewer items keep splitting."""
    from nvkv._lib import lib
    need = ctypes.c_size_t(0)

    def ws(B, hq, hkv, max_k):
        assert lib.nvkv_paged_attention_workspace_size(B, hq, hkv, 128, 1, max_k,
                                                       ctypes.byref(need)) == 0
        return need.value
    assert ws(256, 4, 1, 1536) == 0      # 8B TP8 decode: 256 items, 24 tiles
    assert ws(256, 4, 1, 3072) == 0      # 48 tiles: still one wave
    assert ws(256, 4, 1, 3073) > 0       # 49 tiles: split
    assert ws(237, 4, 1, 1536) == 0      # 237 items >= 0.8 * 296
    assert ws(236, 4, 1, 1536) > 0       # below: split to fill the machine
    assert ws(64, 16, 8, 4096) > 0       # config 2: 64-tile contexts split
    assert ws(64, 8, 1, 32768) > 0       # 32B TP8 long context


def test_fp8_workspace_follows_its_plan():
    """The fp8 pool's decode plan (128-key tiles) seen through its workspace
    query: one wave of unsplit CTAs needs no scratch, a batch that splits
    does, and prompts add their dequantised rows (K and V, 2 bytes a value)
    after the decode scratch and the prefill work plan."""
    from nvkv import ops
    assert ops.workspace_size_fp8(256, 4, 1, 1, 1536, 0) == 0   # 8B TP8 decode: one wave
    split = ops.workspace_size_fp8(64, 16, 8, 1, 4096, 0)       # config 2: splits
    assert split > 0
    with_prompts = ops.workspace_size_fp8(64, 16, 8, 512, 4096, 4096)
    assert with_prompts >= split + 4096 * 8 * 128 * 2 * 2
