"""Peer-memory communicator for the fused all-reduce + residual + RMSNorm
epilogue (nvkv_comm_* / nvkv_allreduce_rms_norm in include/nvkv.h).

Replaces, for the decoder's tensor-parallel all-reduces, the NCCL `Comm` of
nanovllm_rs/src/layers/nccl.rs:11-102 used through AllReduce
(layers/dist_util.rs:29-84).  One process per GPU: every rank builds a
`PeerComm` collectively (the IPC handles travel through an all-gather on the
torch process group); afterwards all ranks call `allreduce_rms_norm` with the
same shapes in the same order, after writing their partial sums into
`input(T, H)` (e.g. `torch.matmul(..., out=comm.input(T, H))`).
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch
import torch.distributed as dist

from ._lib import COMM_HANDLE_BYTES, RESIDUAL_ADD, RESIDUAL_INIT, check, lib
from .ops import _dtype, _need, _ptr, _stream


class _DeviceBytes:
    """A borrowed device allocation exposed to torch through the CUDA array
    interface (the communicator keeps ownership)."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1",
                                         "data": (ptr, False), "version": 3, "strides": None}


class PeerComm:
    def __init__(self, rank: int, world: int, max_bytes: int, group=None,
                 timeout_s: Optional[float] = None):
        self.rank, self.world, self.max_bytes = rank, world, int(max_bytes)
        self._h = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(COMM_HANDLE_BYTES)
        check(lib.nvkv_comm_create(rank, world, self.max_bytes, ctypes.byref(self._h), handle))
        if timeout_s is not None:
            check(lib.nvkv_comm_set_timeout(self._h, int(timeout_s * 1e9)))
        mine = torch.frombuffer(bytearray(handle.raw), dtype=torch.uint8).cuda()
        if world > 1:
            parts = [torch.empty_like(mine) for _ in range(world)]
            dist.all_gather(parts, mine, group=group)
        else:
            parts = [mine]
        allh = b"".join(bytes(p.cpu().numpy().tobytes()) for p in parts)
        check(lib.nvkv_comm_open_peers(self._h, ctypes.c_char_p(allh)))
        ptr = ctypes.c_void_p()
        check(lib.nvkv_comm_input(self._h, ctypes.byref(ptr)))
        self._input = torch.as_tensor(_DeviceBytes(ptr.value, self.max_bytes), device="cuda")

    def input(self, T: int, H: int, dtype=torch.bfloat16) -> torch.Tensor:
        """This rank's input buffer as a contiguous [T, H] tensor."""
        n = T * H * torch.tensor([], dtype=dtype).element_size()
        _need(n <= self.max_bytes, f"comm buffer holds {self.max_bytes} bytes, need {n}")
        return self._input[:n].view(dtype).view(T, H)

    def allreduce_rms_norm(self, T: int, H: int, residual: torch.Tensor, weight: torch.Tensor,
                           eps: float, out: torch.Tensor, init: bool = False) -> torch.Tensor:
        """out = rms_norm(sum over ranks of input(T, H) (+ residual)); the
        residual becomes that sum (init) or is updated in place to it."""
        for t in (residual, out):
            _need(t.is_cuda and t.is_contiguous() and t.shape == (T, H), "residual/out: [T, H]")
        _need(weight.is_contiguous() and weight.numel() == H and weight.dtype == out.dtype,
              "weight")
        check(lib.nvkv_allreduce_rms_norm(self._h, T, H, _ptr(residual),
                                          RESIDUAL_INIT if init else RESIDUAL_ADD, _ptr(weight),
                                          float(eps), _ptr(out), _dtype(out), _stream()))
        return out

    def close(self) -> None:
        """Every rank's last call must have completed (synchronize + barrier)."""
        if self._h:
            self._input = None
            check(lib.nvkv_comm_destroy(self._h))
            self._h = ctypes.c_void_p()
