"""Peer-memory windows of the T-sharded stack: the GroupNorm statistics
gather and the halo exchange as stores into the peers' memory over NVLink.

Each rank allocates one window (b200_peer_window_alloc) holding the exchange
flags, the statistics slots and its haloed conv operand xp
[N, T_local + 2, H, W, C]; the ranks swap CUDA IPC handles once (a host
all-gather) and map each other's windows.  Per block the stack then runs, on
its own stream and with no NCCL call:

    partial statistics -> b200_peer_stats_publish -> b200_peer_stats_merge
    -> GroupNorm + SiLU into xp's interior -> b200_peer_halo_push
    -> b200_peer_halo_wait -> conv3d over xp

The protocol (epochs, slot parities, why one xp buffer suffices) is described
with the C declarations in include/b200conv.h.  Everything here is host
bookkeeping: window geometry, handle exchange, the pointers each call gets.
`PeerWindows.emulate` builds all ranks' windows in one process on one GPU;
running the ranks' calls one after another in stream order then exercises
the same kernels without any kernel waiting on one that has not finished.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import List, Optional, Sequence, Tuple

import torch

from . import _lib

HANDLE_BYTES = 64      # B200_PEER_HANDLE_BYTES
MAX_RANKS = 64         # B200_PEER_MAX_RANKS
PUSH_CTAS = 64         # B200_PEER_PUSH_CTAS


@dataclass(frozen=True)
class HaloSide:
    """One direction of the halo exchange, offsets relative to the xp start
    of the sending (src) and receiving (dst) windows."""
    peer: int
    src_off: int
    src_stride: int
    dst_off: int
    dst_stride: int


def halo_plan(rank: int, t_sizes: Sequence[int],
              frame_bytes: int) -> Tuple[Optional[HaloSide], Optional[HaloSide]]:
    """(lo, hi) sides for `rank`.  xp of rank q is [N, t_sizes[q] + 2, frame],
    frame 0 the bottom halo, frames 1..T the interior, frame T + 1 the top
    halo.  lo: this rank's frame 1 -> the previous rank's top halo; hi: frame
    T -> the next rank's bottom halo; one block of frame_bytes per batch item
    (item strides differ when the ranks' T differ)."""
    world = len(t_sizes)
    T = t_sizes[rank]
    src_stride = (T + 2) * frame_bytes
    lo = hi = None
    if rank > 0:
        Tp = t_sizes[rank - 1]
        lo = HaloSide(rank - 1, 1 * frame_bytes, src_stride, (Tp + 1) * frame_bytes,
                      (Tp + 2) * frame_bytes)
    if rank < world - 1:
        Tn = t_sizes[rank + 1]
        hi = HaloSide(rank + 1, T * frame_bytes, src_stride, 0, (Tn + 2) * frame_bytes)
    return lo, hi


class _DeviceBytes:
    """A raw device range exposed through __cuda_array_interface__ so that
    torch can view it without copying."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1",
                                         "data": (ptr, False), "version": 3, "strides": None}


def _esize(dtype: torch.dtype) -> int:
    return torch.empty((), dtype=dtype).element_size()


class PeerWindows:
    """This rank's window plus the mapped windows of the other ranks."""

    def __init__(self, rank: int, t_sizes: Sequence[int], entries: int,
                 N: int, H: int, W: int, C: int, dtype: torch.dtype, device: torch.device,
                 ptrs: List[int], owned: bool, opened: Sequence[int]):
        self.rank, self.world = rank, len(t_sizes)
        self.t_sizes = list(t_sizes)
        self.entries = entries
        self.N, self.H, self.W, self.C, self.dtype = N, H, W, C, dtype
        self.device = device
        self.ptrs = list(ptrs)
        self._owned = owned
        self._opened = list(opened)
        L = _lib.lib()
        self.xp_off = int(L.b200_peer_window_xp_offset(self.world, entries))
        self.frame_bytes = H * W * C * _esize(dtype)
        self.lo, self.hi = halo_plan(rank, self.t_sizes, self.frame_bytes)
        self.ptrs_dev = torch.tensor(self.ptrs, dtype=torch.int64, device=device)
        T = self.t_sizes[rank]
        xp_bytes = N * (T + 2) * self.frame_bytes
        raw = torch.as_tensor(_DeviceBytes(self.local + self.xp_off, xp_bytes), device=device)
        self.xp = raw.view(dtype).view(N, T + 2, H, W, C)
        self._closed = False

    # -------------------------------------------------------------- set-up
    @staticmethod
    def window_bytes(world: int, entries: int, xp_bytes: int) -> int:
        return int(_lib.lib().b200_peer_window_bytes(world, entries, xp_bytes))

    @staticmethod
    def _alloc(nbytes: int) -> Tuple[int, bytes]:
        L = _lib.lib()
        ptr = ctypes.c_void_p()
        handle = (ctypes.c_char * HANDLE_BYTES)()
        _lib.check(L.b200_peer_window_alloc(nbytes, ctypes.byref(ptr), handle),
                   "b200_peer_window_alloc")
        return int(ptr.value), bytes(handle)

    @classmethod
    def create(cls, group, entries: int, N: int, t_sizes: Sequence[int], H: int, W: int,
               C: int, dtype: torch.dtype, device: torch.device) -> "PeerWindows":
        """Collective over `group`: allocate, swap IPC handles, map peers."""
        import torch.distributed as dist
        rank, world = dist.get_rank(group), dist.get_world_size(group)
        if world > MAX_RANKS:
            raise ValueError(f"peer exchange supports at most {MAX_RANKS} ranks")
        fb = H * W * C * _esize(dtype)
        nbytes = cls.window_bytes(world, entries, max(N * (t + 2) * fb for t in t_sizes))
        ptr, handle = cls._alloc(nbytes)
        handles: List[Optional[bytes]] = [None] * world
        dist.all_gather_object(handles, handle, group=group)
        L = _lib.lib()
        ptrs, opened = [], []
        for q, h in enumerate(handles):
            if q == rank:
                ptrs.append(ptr)
                continue
            p = ctypes.c_void_p()
            buf = ctypes.create_string_buffer(h, HANDLE_BYTES)
            _lib.check(L.b200_peer_window_open(buf, ctypes.byref(p)), "b200_peer_window_open")
            ptrs.append(int(p.value))
            opened.append(int(p.value))
        return cls(rank, t_sizes, entries, N, H, W, C, dtype, device, ptrs, True, opened)

    @classmethod
    def emulate(cls, t_sizes: Sequence[int], entries: int, N: int, H: int, W: int, C: int,
                dtype: torch.dtype, device: torch.device) -> List["PeerWindows"]:
        """All ranks' windows in this process (one GPU): rank q's object sees
        every window at its local address."""
        world = len(t_sizes)
        fb = H * W * C * _esize(dtype)
        nbytes = cls.window_bytes(world, entries, max(N * (t + 2) * fb for t in t_sizes))
        ptrs = [cls._alloc(nbytes)[0] for _ in range(world)]
        out = []
        for q in range(world):
            out.append(cls(q, t_sizes, entries, N, H, W, C, dtype, device, ptrs,
                           owned=False, opened=()))
        out[0]._emulated_all = ptrs
        return out

    @property
    def local(self) -> int:
        return self.ptrs[self.rank]

    # ---------------------------------------------------------- per block
    def _stream(self) -> int:
        return torch.cuda.current_stream(self.device).cuda_stream

    def publish(self, stats: torch.Tensor) -> None:
        stats = stats.contiguous()
        if stats.dtype != torch.float32 or stats.numel() != self.entries * 3:
            raise ValueError("stats must be fp32 [entries, 3]")
        rc = _lib.lib().b200_peer_stats_publish(stats.data_ptr(), self.ptrs_dev.data_ptr(),
                                                self.world, self.rank, self.entries,
                                                self.local, self._stream())
        _lib.check(rc, "b200_peer_stats_publish")

    def merge(self, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        if out is None:
            out = torch.empty(self.entries, 3, dtype=torch.float32, device=self.device)
        rc = _lib.lib().b200_peer_stats_merge(self.local, out.data_ptr(), self.world,
                                              self.entries, self._stream())
        _lib.check(rc, "b200_peer_stats_merge")
        return out

    def push(self) -> None:
        base = self.local + self.xp_off
        def side(s: Optional[HaloSide]):
            if s is None:
                return None, None, None, 0, 0
            peer = self.ptrs[s.peer]
            return (base + s.src_off, peer + self.xp_off + s.dst_off, peer,
                    s.src_stride, s.dst_stride)
        ls, ld, lw, lss, lds = side(self.lo)
        hs, hd, hw, hss, hds = side(self.hi)
        rc = _lib.lib().b200_peer_halo_push(self.local, ls, ld, lw, lss, lds, hs, hd, hw, hss,
                                            hds, self.N, self.frame_bytes, self._stream())
        _lib.check(rc, "b200_peer_halo_push")

    def gate(self) -> Tuple[int, int, int, int]:
        """(epoch, bottom counter, top counter, scale) addresses for
        b200_conv3d_fwd_gated: the conv waits for this block's halo arrivals
        itself, so the push can overlap the interior tiles."""
        lo = self.local + 1024 if self.lo is not None else 0
        hi = self.local + 1024 + 128 if self.hi is not None else 0
        return self.local, lo, hi, PUSH_CTAS

    def wait(self) -> None:
        rc = _lib.lib().b200_peer_halo_wait(self.local, int(self.lo is not None),
                                            int(self.hi is not None), self._stream())
        _lib.check(rc, "b200_peer_halo_wait")

    # ------------------------------------------------------------ tear-down
    def close(self, group=None) -> None:
        """Collective when created with create(): unmap peers after every rank
        stopped using them, free the own window after every peer unmapped."""
        if self._closed:
            return
        self._closed = True
        L = _lib.lib()
        self.xp = None
        torch.cuda.synchronize(self.device)
        if self._owned:
            import torch.distributed as dist
            dist.barrier(group=group)
            for p in self._opened:
                _lib.check(L.b200_peer_window_close(p), "b200_peer_window_close")
            dist.barrier(group=group)
            _lib.check(L.b200_peer_window_free(self.local), "b200_peer_window_free")
        elif getattr(self, "_emulated_all", None):
            for p in self._emulated_all:
                _lib.check(L.b200_peer_window_free(p), "b200_peer_window_free")
