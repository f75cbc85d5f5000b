"""ctypes binding of libnvkv.so (the C ABI declared in include/nvkv.h).

The library is loaded from this directory only.  There is no fallback: if
the shared object is missing or does not export a declared symbol, importing
the package raises, so a test or benchmark can never pass on a CPU or
PyTorch stand-in.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libnvkv.so")

OK = 0
ERR_INVALID_ARG = -1
ERR_UNSUPPORTED = -2
ERR_ALIGNMENT = -3
ERR_CUDA = -4
ERR_WORKSPACE = -5
ERR_DEVICE = -6

DTYPE_F16 = 0
DTYPE_BF16 = 1
DTYPE_F32 = 2  # nvkv_sample's logits only

DEVERR_NONE = 0
DEVERR_SLOT_RANGE = 1
DEVERR_BLOCK_RANGE = 2
DEVERR_POSITION_RANGE = 3
DEVERR_SEQLEN = 4
DEVERR_PEER_TIMEOUT = 5

COMM_HANDLE_BYTES = 64
COMM_MAX_RANKS = 8
RESIDUAL_ADD = 0
RESIDUAL_INIT = 1

_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int
_f32 = ctypes.c_float
_sz = ctypes.c_size_t



class BlockSeq(ctypes.Structure):
    """nvkv_block_seq: the block manager's view of a Sequence."""
    _fields_ = [("token_ids", ctypes.c_void_p), ("num_tokens", ctypes.c_int64),
                ("num_cached_tokens", ctypes.c_int64), ("num_new_tokens", ctypes.c_int64),
                ("block_table", ctypes.c_void_p), ("block_table_len", ctypes.c_int64),
                ("block_table_capacity", ctypes.c_int64)]


class StepSizes(ctypes.Structure):
    """nvkv_step_sizes: the output sizes of nvkv_prepare_step."""
    _fields_ = [("num_tokens", ctypes.c_int64), ("num_slots", ctypes.c_int64),
                ("num_need_logits", ctypes.c_int64), ("block_table_width", ctypes.c_int64),
                ("max_seqlen_q", ctypes.c_int64), ("max_seqlen_k", ctypes.c_int64),
                ("has_block_tables", ctypes.c_int)]


_seq = ctypes.POINTER(BlockSeq)
_pi64 = ctypes.POINTER(ctypes.c_int64)
_pi32 = ctypes.POINTER(ctypes.c_int)

# name -> argtypes, in the order of include/nvkv.h
SIGNATURES = {
    "nvkv_version": [],
    "nvkv_last_error": [],
    "nvkv_device_error": [ctypes.POINTER(_i32), _i32],
    "nvkv_store_kvcache": [_p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i32, _p],
    "nvkv_qknorm_rope": [_p, _i64, _i64, _i32, _i32, _i32, _p, _p, _p, _f32, _f32, _i64, _p, _p,
                         _p, _p, _p, _p, _i64, _i32, _p],
    "nvkv_paged_attention_workspace_size": [_i32, _i32, _i32, _i32, _i32, _i32,
                                            ctypes.POINTER(_sz)],
    "nvkv_paged_attention": [_p, _i64, _i64, _p, _p, _i64, _i64, _p, _p, _p, _p, _i64, _i32, _i32,
                             _i32, _i32, _i32, _i32, _i32, _f32, _i32, _p, _sz, _i32, _p],
    "nvkv_paged_attention_noalloc": [_p, _i64, _i64, _p, _p, _i64, _i64, _p, _p, _p, _p, _i64,
                                     _i32, _i32, _i32, _i32, _i32, _i32, _i32, _f32, _i32, _i32,
                                     _p],
    "nvkv_store_kvcache_fp8": [_p, _p, _p, _p, _p, _p, _p, _i64, _i32, _i32, _i64, _i64, _i64,
                               _i32, _i32, _p],
    "nvkv_paged_attention_fp8_workspace_size": [_i32, _i32, _i32, _i32, _i32, _i32, _i64,
                                                ctypes.POINTER(_sz)],
    "nvkv_paged_attention_fp8": [_p, _i64, _i64, _p, _p, _p, _p, _i64, _p, _p, _p, _p, _i64,
                                 _i32, _i32, _i32, _i32, _i32, _i32, _i32, _f32, _i32, _i64, _p,
                                 _sz, _i32, _p],
    "nvkv_rms_norm": [_p, _i64, _p, _i64, _p, _f32, _p, _i64, _i64, _i32, _i32, _p],
    "nvkv_silu_and_mul": [_p, _i64, _p, _i64, _i64, _i32, _i32, _p],
    "nvkv_decode_advance": [_i32, _i32, _p, _p, _i64, _i64, _p, _p, _p, _p, _p],
    "nvkv_sample": [_p, _i64, _i64, _i64, _i64, _p, ctypes.c_uint64, ctypes.c_uint64, _p, _p,
                    _p, _i32, _p],
    "nvkv_comm_create": [_i32, _i32, _sz, ctypes.POINTER(_p), _p],
    "nvkv_comm_open_peers": [_p, _p],
    "nvkv_comm_input": [_p, ctypes.POINTER(_p)],
    "nvkv_comm_set_timeout": [_p, _i64],
    "nvkv_comm_destroy": [_p],
    "nvkv_allreduce_rms_norm": [_p, _i64, _i32, _p, _i32, _p, _f32, _p, _i32, _p],
    "nvkv_context_set": [_p, _p, _i32, _i32, _i32, _p, _i64, _p, _p, _i64],
    "nvkv_context_reset": [],
    "nvkv_attention_create": [_f32, ctypes.POINTER(_p)],
    "nvkv_attention_destroy": [_p],
    "nvkv_attention_set_kv_cache": [_p, _p, _p, _i64, _i32, _i32, _i32, _i32],
    "nvkv_attention_forward": [_p, _p, _i64, _p, _i64, _p, _i64, _i64, _i32, _i32, _p, _i32, _p],
    "nvkv_block_hash": [_p, _i64, _i64, _pi64],
    "nvkv_block_manager_create": [_i64, _i64, ctypes.POINTER(_p)],
    "nvkv_block_manager_destroy": [_p],
    "nvkv_block_manager_num_free": [_p, _pi64],
    "nvkv_block_manager_can_allocate": [_p, _i64, _pi32],
    "nvkv_block_manager_get_token_layout": [_p, _seq, _pi64, _pi64, _pi64],
    "nvkv_block_manager_allocate": [_p, _seq],
    "nvkv_block_manager_deallocate": [_p, _seq],
    "nvkv_block_manager_can_append": [_p, _seq, _i64, _pi32],
    "nvkv_block_manager_may_append": [_p, _seq],
    "nvkv_block_manager_append_batch": [_p, _seq, _i64, _p, _pi64],
    "nvkv_block_manager_block_info": [_p, _i64, _pi64, _pi64, _pi64, _pi32],
    "nvkv_block_manager_free_ids": [_p, _p, _i64, _pi64],
    "nvkv_block_manager_lookup": [_p, _i64, _pi64],
    "nvkv_kv_pool_blocks": [_i64, _i64, ctypes.c_double, _i32, _i32, _i32, _i32, _i32, _pi64],
    "nvkv_kv_pool_probe": [ctypes.c_double, _i32, _i32, _i32, _i32, _i32, _pi64],
    "nvkv_prepare_step": [_p, _i64, _i64, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64,
                          ctypes.POINTER(StepSizes)],
}


class NvkvError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"nvkv error {code}: {msg}")
        self.code = code


def _load() -> ctypes.CDLL:
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python nanovllm-rs_b200/build.py` "
            "(there is no CPU fallback for this path)")
    lib = ctypes.CDLL(LIB_PATH)
    for name, argtypes in SIGNATURES.items():
        fn = getattr(lib, name)  # AttributeError if the symbol is not exported
        fn.argtypes = argtypes
        fn.restype = ctypes.c_char_p if name == "nvkv_last_error" else _i32
    return lib


lib = _load()


def check(rc: int) -> None:
    if rc != OK:
        raise NvkvError(rc, lib.nvkv_last_error().decode(errors="replace"))


def device_error(clear: bool = True) -> int:
    """Reads (and by default clears) the current device's bounds-check word."""
    code = _i32(0)
    check(lib.nvkv_device_error(ctypes.byref(code), 1 if clear else 0))
    return code.value
