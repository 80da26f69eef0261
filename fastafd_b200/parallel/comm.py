"""Tensor-parallel collectives of the attention side.

:class:`TpComm` is what the model code sees: ``all_reduce``, ``all_gather`` (along dim 0),
``all_gather_last_dim`` and ``reduce_scatter`` (along dim 0). Two implementations:

* :class:`TorchDistComm` - ``torch.distributed`` on a process group (gloo on CPU in tests,
  NCCL on GPUs).
* :class:`NcclComm` - the repository's own communicator (csrc/nccl/nccl_comm.cpp) with a
  registered staging buffer for small all-reduces, async error polling and abort.

Reference: python/minisgl/distributed/impl.py:28-85 (TorchDistributedImpl /
PyNCCLDistributedImpl), python/minisgl/kernel/pynccl.py:92-99 (unique id broadcast).
"""
from __future__ import annotations

import ctypes as C
from typing import List, Optional

import torch
import torch.distributed as dist


class TpComm:
    rank: int = 0
    size: int = 1

    def all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        return x

    def all_gather(self, x: torch.Tensor, lane: int = -1) -> torch.Tensor:
        """Concatenate the ranks' rows. `lane` names the micro-batch for communicators that keep
        per-lane buffers; the others ignore it."""
        return x

    def all_gather_last_dim(self, x: torch.Tensor) -> torch.Tensor:
        return x

    def reduce_scatter(self, x: torch.Tensor) -> torch.Tensor:
        return x


class TorchDistComm(TpComm):
    def __init__(self, group, ranks: List[int]):
        self.group, self.ranks = group, list(ranks)
        self.size = len(ranks)
        self.rank = self.ranks.index(dist.get_rank())

    def all_reduce(self, x):
        dist.all_reduce(x, group=self.group)
        return x

    def all_gather(self, x, lane: int = -1):
        x = x.contiguous()
        out = torch.empty(self.size * x.shape[0], *x.shape[1:], dtype=x.dtype, device=x.device)
        dist.all_gather_into_tensor(out, x, group=self.group) if x.is_cuda else \
            dist.all_gather(list(out.chunk(self.size, 0)), x, group=self.group)
        return out

    def all_gather_last_dim(self, x):
        g = self.all_gather(x)                                   # [size*T, n]
        T = x.shape[0]
        return torch.cat([g[r * T:(r + 1) * T] for r in range(self.size)], dim=-1)

    def reduce_scatter(self, x):
        x = x.contiguous()
        n = x.shape[0] // self.size
        out = torch.empty(n, *x.shape[1:], dtype=x.dtype, device=x.device)
        if x.is_cuda:
            dist.reduce_scatter_tensor(out, x, group=self.group)
        else:                                                    # gloo has no reduce-scatter
            dist.all_reduce(x, group=self.group)
            out.copy_(x[self.rank * n:(self.rank + 1) * n])
        return out


_DTYPES = {torch.bfloat16: 0, torch.float32: 1, torch.float16: 2, torch.int32: 3, torch.uint8: 4}


class NcclError(RuntimeError):
    pass


class NcclComm(TpComm):
    """Own NCCL communicator over `ranks` of the default (host-side) process group."""

    @staticmethod
    def _load():
        from ..build import build_nccl_wrapper, nccl_lib_path

        path = nccl_lib_path()
        if not path.exists():
            path = build_nccl_wrapper()
        lib = C.CDLL(str(path))
        lib.afd_nccl_error_string.restype = C.c_char_p
        return lib

    @classmethod
    def new_unique_id(cls) -> bytes:
        """A fresh NCCL unique id (128 bytes), made by the rank that will be rank 0 of the communicator."""
        lib, uid = cls._load(), C.create_string_buffer(128)
        code = lib.afd_nccl_unique_id(uid)
        if code != 0:
            raise NcclError(f"nccl unique_id: {lib.afd_nccl_error_string(code).decode()} ({code})")
        return uid.raw

    def __init__(self, ranks: List[int], device: torch.device, host_group=None, max_buffer_bytes: int = 64 << 20,
                 uid: Optional[bytes] = None):
        """`uid`: the unique id from the communicator's rank 0 (`new_unique_id`), already delivered to
        every member; without it the id is broadcast over `host_group`, which must contain exactly `ranks`."""
        self.lib = self._load()
        self.ranks, self.size, self.device = list(ranks), len(ranks), device
        me = dist.get_rank()
        self.rank = self.ranks.index(me)
        if uid is None:
            box = [self.new_unique_id() if self.rank == 0 else None]
            dist.broadcast_object_list(box, src=self.ranks[0], group=host_group)
            uid = box[0]
        self.handle = C.c_void_p()
        with torch.cuda.device(device):
            self._check(self.lib.afd_nccl_init(self.rank, self.size, C.create_string_buffer(uid, 128),
                                               C.c_size_t(max_buffer_bytes), C.byref(self.handle)), "init")

    def _check(self, code: int, what: str) -> None:
        if code != 0:
            msg = self.lib.afd_nccl_error_string(code % 1000).decode() if code < 1000 else f"cuda error {code - 1000}"
            raise NcclError(f"nccl {what}: {msg} ({code})")

    @staticmethod
    def _stream() -> C.c_void_p:
        return C.c_void_p(torch.cuda.current_stream().cuda_stream)

    def all_reduce(self, x):
        assert x.is_contiguous()
        self._check(self.lib.afd_nccl_all_reduce(self.handle, C.c_void_p(x.data_ptr()), C.c_size_t(x.numel()),
                                                 _DTYPES[x.dtype], self._stream()), "all_reduce")
        return x

    def all_gather(self, x, lane: int = -1):
        x = x.contiguous()
        out = torch.empty(self.size * x.shape[0], *x.shape[1:], dtype=x.dtype, device=x.device)
        self._check(self.lib.afd_nccl_all_gather(self.handle, C.c_void_p(x.data_ptr()), C.c_void_p(out.data_ptr()),
                                                 C.c_size_t(x.numel()), _DTYPES[x.dtype], self._stream()), "all_gather")
        return out

    def all_gather_last_dim(self, x):
        g = self.all_gather(x)
        T = x.shape[0]
        return torch.cat([g[r * T:(r + 1) * T] for r in range(self.size)], dim=-1)

    def reduce_scatter(self, x):
        x = x.contiguous()
        n = x.shape[0] // self.size
        out = torch.empty(n, *x.shape[1:], dtype=x.dtype, device=x.device)
        self._check(self.lib.afd_nccl_reduce_scatter(self.handle, C.c_void_p(x.data_ptr()), C.c_void_p(out.data_ptr()),
                                                     C.c_size_t(out.numel()), _DTYPES[x.dtype], self._stream()),
                    "reduce_scatter")
        return out

    def async_error(self) -> Optional[str]:
        state = C.c_int(0)
        self._check(self.lib.afd_nccl_async_error(self.handle, C.byref(state)), "async_error")
        return None if state.value == 0 else self.lib.afd_nccl_error_string(state.value).decode()

    def abort(self) -> None:
        if self.handle:
            self.lib.afd_nccl_abort(self.handle)

    def destroy(self) -> None:
        if self.handle:
            self.lib.afd_nccl_destroy(self.handle)
            self.handle = C.c_void_p()
