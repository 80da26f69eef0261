"""Peer-visible device heaps: the memory substrate of N2M / M2N.

Every rank owns one *heap* (a single ``cudaMalloc`` made by the kernel library) and
knows the base address of every other rank's heap as mapped into its own process
(CUDA IPC over NVLink). Sub-buffers are named by byte offsets computed from a
:class:`Layout`, which is a pure function of the model/runtime sizing, so two ranks
agree on where a peer keeps its receive slots without exchanging anything else.

Two constructors:

* :meth:`Fabric.local` - all "ranks" live in this process on one GPU (single-GPU runs
  and tests; peer pointers are plain local pointers).
* :meth:`Fabric.ipc` - one process per GPU; handles are exchanged through a host-side
  ``torch.distributed`` group (gloo).

The reference obtains the same thing from torch symmetric memory
(python/minisgl/kernel/megamoe_m2n_mega.py:163-262) and a 72-entry peer offset table
(python/minisgl/kernel/csrc/deepgemm/deep_gemm/include/deep_gemm/layout/sym_buffer.cuh).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence, Tuple

import torch

_DTYPE_STR = {
    torch.uint8: "|u1", torch.int8: "|i1", torch.int32: "<i4", torch.int64: "<i8",
    torch.float32: "<f4", torch.float16: "<f2", torch.uint32: "<u4",
}


def align_up(x: int, a: int = 256) -> int:
    return (x + a - 1) // a * a


@dataclass
class Layout:
    """Ordered name -> (offset, nbytes) map with 256-byte aligned entries."""
    entries: Dict[str, Tuple[int, int]] = field(default_factory=dict)
    size: int = 0

    def add(self, name: str, nbytes: int) -> int:
        if name in self.entries:
            raise KeyError(f"duplicate layout entry {name}")
        off = self.size
        self.entries[name] = (off, nbytes)
        self.size = align_up(off + nbytes)
        return off

    def offset(self, name: str) -> int:
        return self.entries[name][0]

    def nbytes(self, name: str) -> int:
        return self.entries[name][1]


class _RawArray:
    """Adapter exposing a raw device range through ``__cuda_array_interface__``."""

    def __init__(self, addr: int, nbytes: int, owner):
        self.__cuda_array_interface__ = {
            "shape": (nbytes,), "typestr": "|u1", "data": (addr, False), "version": 3, "strides": None,
        }
        self._owner = owner


class DeviceHeap:
    """One device allocation with typed tensor views at byte offsets."""

    def __init__(self, addr: int, nbytes: int, device: torch.device, owned: bool, ipc_handle: bytes = b""):
        self.addr, self.nbytes, self.device, self.owned, self.ipc_handle = addr, nbytes, device, owned, ipc_handle
        self._bytes: Optional[torch.Tensor] = None

    @staticmethod
    def allocate(nbytes: int, device: torch.device, exportable: bool = False) -> "DeviceHeap":
        from ..ops._lib import check, lib

        nbytes = align_up(max(nbytes, 256))
        p = C.c_void_p()
        with torch.cuda.device(device):
            if exportable:
                handle = C.create_string_buffer(64)
                check(lib().afd_fabric_alloc(nbytes, C.byref(p), handle), "fabric_alloc")
                return DeviceHeap(p.value, nbytes, device, True, handle.raw)
            check(lib().afd_device_alloc(nbytes, C.byref(p)), "device_alloc")
            torch.cuda.synchronize(device)
        return DeviceHeap(p.value, nbytes, device, True)

    def as_bytes(self) -> torch.Tensor:
        if self._bytes is None:
            self._bytes = torch.as_tensor(_RawArray(self.addr, self.nbytes, self), device=self.device)
        return self._bytes

    def view(self, offset: int, shape: Sequence[int], dtype: torch.dtype) -> torch.Tensor:
        n = 1
        for s in shape:
            n *= s
        nbytes = n * torch.empty(0, dtype=dtype).element_size()
        if offset < 0 or offset + nbytes > self.nbytes:
            raise ValueError(f"view [{offset}, {offset + nbytes}) outside heap of {self.nbytes} bytes")
        return self.as_bytes()[offset:offset + nbytes].view(dtype).view(*shape)

    def free(self) -> None:
        from ..ops._lib import lib

        if self.owned and self.addr:
            self._bytes = None
            lib().afd_fabric_free(self.addr)
            self.addr = 0


class Fabric:
    """This rank's heap plus every rank's heap base as seen from this process."""

    def __init__(self, rank: int, heap: DeviceHeap, bases: List[int], sizes: List[int], opened: List[int]):
        self.rank, self.heap, self.bases, self.sizes = rank, heap, bases, sizes
        self._opened = opened

    @property
    def world(self) -> int:
        return len(self.bases)

    def peer_ptr(self, rank: int, offset: int, nbytes: int = 0) -> int:
        if offset < 0 or offset + nbytes > self.sizes[rank]:
            raise ValueError(f"peer range [{offset}, {offset + nbytes}) outside rank {rank}'s heap")
        return self.bases[rank] + offset

    @staticmethod
    def local(sizes: Sequence[int], device: torch.device) -> List["Fabric"]:
        heaps = [DeviceHeap.allocate(s, device) for s in sizes]
        bases = [h.addr for h in heaps]
        nb = [h.nbytes for h in heaps]
        return [Fabric(r, heaps[r], list(bases), list(nb), []) for r in range(len(heaps))]

    @staticmethod
    def ipc(nbytes: int, device: torch.device, group=None) -> "Fabric":
        import torch.distributed as dist

        from ..ops._lib import check, lib

        rank, world = dist.get_rank(group), dist.get_world_size(group)
        heap = DeviceHeap.allocate(nbytes, device, exportable=True)
        infos: List[Optional[tuple]] = [None] * world
        dist.all_gather_object(infos, (heap.ipc_handle, heap.nbytes, device.index), group=group)
        bases, sizes, opened = [], [], []
        with torch.cuda.device(device):
            for r, (handle, size, _dev) in enumerate(infos):
                if r == rank:
                    bases.append(heap.addr)
                else:
                    p = C.c_void_p()
                    buf = C.create_string_buffer(handle, 64)
                    check(lib().afd_fabric_open(buf, C.byref(p)), f"fabric_open(rank {r})")
                    bases.append(p.value)
                    opened.append(p.value)
                sizes.append(size)
        dist.barrier(group)
        return Fabric(rank, heap, bases, sizes, opened)

    def close(self) -> None:
        from ..ops._lib import lib

        for p in self._opened:
            lib().afd_fabric_close(p)
        self._opened = []
        self.heap.free()
