"""Peer-memory all-reduce of the data-parallel gradient buffer (one process per GPU).

The library's exchange kernel (``lsso_peer_allreduce``) sums every rank's
flat FP32 gradient buffer straight over NVLink / NVSwitch: each rank's
buffer lives in a library-allocated region that the other ranks map with
CUDA IPC, and one launch per rank and exchange signals the peers, waits for
them (bounded), reads all ranks' values in rank order and writes the scaled
sum locally.  This module owns the regions and the handle exchange;
``GradientExchange(transport="peer")`` uses it in place of an NCCL
``all_reduce``.  Requires one host, at most eight ranks, and peer access
between the ranks' GPUs; ``PeerGroup`` raises ``PeerUnavailable`` (on every
rank alike) otherwise.
"""

from __future__ import annotations

import ctypes
import socket

import torch
import torch.distributed as dist

from . import _native

HANDLE_BYTES = 64
DATA_OFFSET = 512
HEADER_WORDS = DATA_OFFSET // 4
MAX_RANKS = 8
# Header word indices (u32): arrive flags, depart flags, CTA counter, exchange count.
ARRIVE, DEPART, COUNTER, EPOCH = 0, 32, 64, 96


class PeerUnavailable(RuntimeError):
    """The ranks cannot share memory (several hosts, too many ranks, no peer access)."""


class _Allocation:
    """Owner of one region allocated by the library; frees it when the last view goes."""

    def __init__(self, ptr: int, device: torch.device) -> None:
        self.ptr = ptr
        self.device = device

    def __del__(self) -> None:
        lib = _native._LIBRARY
        if lib is None or not self.ptr:
            return
        try:
            with torch.cuda.device(self.device):
                lib.lib.lsso_peer_region_destroy(ctypes.c_void_p(self.ptr))
        except Exception:  # interpreter shutdown: the CUDA context may be gone already
            pass
        self.ptr = 0


class _DeviceArray:
    """``__cuda_array_interface__`` view of library-owned memory (keeps the allocation alive)."""

    def __init__(self, owner: _Allocation, ptr: int, shape: tuple[int, ...], typestr: str) -> None:
        self._owner = owner
        self.__cuda_array_interface__ = {"shape": shape, "typestr": typestr, "data": (ptr, False), "version": 2}


def _view(owner: _Allocation, ptr: int, count: int, typestr: str, dtype: torch.dtype) -> torch.Tensor:
    if count == 0:
        return torch.empty(0, dtype=dtype, device=owner.device)
    return torch.as_tensor(_DeviceArray(owner, ptr, (count,), typestr), device=owner.device)


class PeerRegion:
    """This rank's exchange region: a flag header and ``count`` FP32 values.

    ``values`` is the flat buffer the backward writes (a tensor over the
    region), ``header`` the 128 flag words (int32 view, for tests), ``handle``
    the 64 bytes the peers open it with.
    """

    def __init__(self, count: int, device: torch.device) -> None:
        lib = _native.library()
        self.count = int(count)
        self.device = torch.device(device)
        ptr = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(HANDLE_BYTES)
        with torch.cuda.device(self.device):
            lib.check(lib.lib.lsso_peer_region_create(self.count, ctypes.byref(ptr), handle))
        self.ptr = int(ptr.value)
        self.handle = handle.raw
        self._allocation = _Allocation(self.ptr, self.device)
        self.header = _view(self._allocation, self.ptr, HEADER_WORDS, "<i4", torch.int32)
        self.values = _view(self._allocation, self.ptr + DATA_OFFSET, self.count, "<f4", torch.float32)


def allreduce(regions: list[int], rank: int, count: int, out: torch.Tensor, *, scale: float = 1.0,
              first: int = 0, wait_limit_ns: int = 0, stream: torch.cuda.Stream | None = None) -> None:
    """Launch one exchange: ``out = scale * sum over r of regions[r]``'s values
    ``[first, first + count)`` (``first`` a multiple of 4).

    ``regions``: every rank's region address as mapped in this process (this
    rank's own at ``rank``).  Asynchronous on ``stream`` (default: current).
    """
    if out.dtype != torch.float32 or not out.is_cuda or not out.is_contiguous() or out.numel() < count:
        raise RuntimeError("out must be a contiguous CUDA float32 tensor of at least count values")
    lib = _native.library()
    world = len(regions)
    array = (ctypes.c_void_p * world)(*regions)
    if stream is None:
        stream = torch.cuda.current_stream(out.device)
    lib.check(lib.lib.lsso_peer_allreduce(array, world, int(rank), int(first), int(count), float(scale),
                                          ctypes.c_void_p(out.data_ptr()), int(wait_limit_ns),
                                          ctypes.c_void_p(stream.cuda_stream)))


class PeerGroup:
    """Every rank's exchange region mapped into this process (collective constructor).

    All ranks of ``group`` construct it together with the same ``count``; the
    handles travel with ``all_gather_object``.  ``reduce(out, scale)`` then
    launches one exchange on the current stream (every rank, same order).
    """

    def __init__(self, count: int, device: torch.device, *, group=None, wait_limit_ns: int = 0) -> None:
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.count = int(count)
        self.wait_limit_ns = int(wait_limit_ns)
        self._opened: list[int] = []
        self.region = None
        if self.world > MAX_RANKS:
            raise PeerUnavailable(f"the peer exchange supports at most {MAX_RANKS} ranks, got {self.world}")
        # Every rank takes part in both gathers whatever fails locally, so that
        # all ranks reach the same verdict.
        error = None
        try:
            self.region = PeerRegion(self.count, device)
        except RuntimeError as exc:
            error = f"the exchange region could not be created: {exc}"
        mine = (socket.gethostname(), self.count, None if self.region is None else self.region.handle, error)
        gathered: list = [None] * self.world
        dist.all_gather_object(gathered, mine, group=group)
        addresses: list[int] = []
        try:
            errors = [e for _, _, _, e in gathered if e]
            if errors:
                raise PeerUnavailable(errors[0])
            if len({host for host, _, _, _ in gathered}) != 1:
                raise PeerUnavailable("the ranks run on more than one host")
            if len({n for _, n, _, _ in gathered}) != 1:
                raise PeerUnavailable("the ranks' gradient buffers differ in size")
            lib = _native.library()
            with torch.cuda.device(self.region.device):
                for r, (_, _, handle, _) in enumerate(gathered):
                    if r == self.rank:
                        addresses.append(self.region.ptr)
                        continue
                    ptr = ctypes.c_void_p()
                    code = lib.lib.lsso_peer_region_open(handle, ctypes.byref(ptr))
                    if code != 0:
                        raise PeerUnavailable(f"rank {r}'s exchange region cannot be mapped: {lib.last_error()}")
                    self._opened.append(int(ptr.value))
                    addresses.append(int(ptr.value))
        except PeerUnavailable as exc:
            error = str(exc)
        outcomes: list = [None] * self.world
        dist.all_gather_object(outcomes, error, group=group)
        failed = [e for e in outcomes if e]
        if failed:
            self.close()
            raise PeerUnavailable(failed[0])
        self.addresses = addresses

    @property
    def values(self) -> torch.Tensor:
        """This rank's flat buffer (the values the exchange sums)."""
        return self.region.values

    def reduce(self, out: torch.Tensor, scale: float = 1.0, first: int = 0, count: int | None = None) -> None:
        """Exchange values ``[first, first + count)`` (default: all) into ``out`` on the current stream."""
        count = self.count - first if count is None else count
        allreduce(self.addresses, self.rank, count, out, scale=scale, first=first, wait_limit_ns=self.wait_limit_ns)

    def close(self) -> None:
        """Unmap the peers' regions (this rank's own is freed with the last view of it)."""
        lib = _native._LIBRARY
        if lib is not None and self._opened:
            with torch.cuda.device(self.region.device):
                for ptr in self._opened:
                    lib.lib.lsso_peer_region_close(ctypes.c_void_p(ptr))
        self._opened = []
        self.addresses = []


__all__ = ["PeerGroup", "PeerRegion", "PeerUnavailable", "allreduce"]
