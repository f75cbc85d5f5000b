"""nvkv: B200 (sm_100a) attention hot path of nanovllm_rs behind its own
operator surface.  Importing this package loads libnvkv.so and fails if it is
missing; there is no CPU or PyTorch fallback."""
from ._lib import NvkvError, device_error, lib, LIB_PATH  # noqa: F401
from .ops import paged_attention, qknorm_rope, store_kvcache, workspace_size  # noqa: F401
from .layers import (Attention, Context, get_context, reset_context,  # noqa: F401
                     set_context, store_kv_cache)

__all__ = ["Attention", "Context", "NvkvError", "device_error", "get_context", "paged_attention",
           "qknorm_rope", "reset_context", "set_context", "store_kv_cache", "store_kvcache",
           "workspace_size"]
