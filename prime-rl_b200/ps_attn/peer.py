"""Peer-memory slabs: one device buffer per rank of a group, mapped into the
other ranks' address spaces with CUDA IPC, for the library's NVLink
exchanges (decode context parallelism, the head all-gather of the
KV-head-sharded decode).

A slab is allocated and zeroed by the library (``ps_dcp_slab_alloc``); its
first 256 bytes are the barrier header the kernels use.  Handles are
exchanged once, through the process group; every call afterwards is device
work only.  :meth:`PeerSlabs.emulated` builds every rank's view of a group on
one GPU for a single process that plays all ranks (the library's ``*_phase``
entry points then run the ranks phase by phase).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _lib


def exchange_handles(handle: bytes, group=None) -> list:
    """All ranks' 64-byte slab handles, in rank order (one all_gather_object)."""
    import torch.distributed as dist

    out = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, bytes(handle), group=group)
    return out


def _alloc(nbytes: int) -> int:
    lib = _lib.load()
    p = ctypes.c_void_p()
    _lib.check(lib.ps_dcp_slab_alloc(nbytes, ctypes.byref(p)))
    return int(p.value)


@dataclass
class PeerSlabs:
    """One rank's view of a group's slabs."""

    world: int
    rank: int
    nbytes: int
    slabs: list            # device addresses, rank order, valid on this GPU
    device: torch.device
    _own: int = 0          # this rank's allocation (freed by close)
    _opened: tuple = ()    # peer mappings (closed by close)

    @property
    def own(self) -> int:
        return self.slabs[self.rank]

    @classmethod
    def from_process_group(cls, nbytes: int, group=None, device=None) -> "PeerSlabs":
        """Collective over ``group`` (one rank per GPU): allocate this rank's
        slab on ``device`` and map every peer's."""
        import torch.distributed as dist

        lib = _lib.load()
        dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        world, rank = dist.get_world_size(group), dist.get_rank(group)
        if world > _lib.PS_DCP_MAX_WORLD:
            raise ValueError(f"peer groups have at most {_lib.PS_DCP_MAX_WORLD} ranks")
        with torch.cuda.device(dev):
            own = _alloc(nbytes)
            h = ctypes.create_string_buffer(_lib.PS_DCP_IPC_HANDLE_BYTES)
            _lib.check(lib.ps_dcp_ipc_handle(own, h))
            handles = exchange_handles(h.raw, group)
            slabs, opened = [], []
            for r, hr in enumerate(handles):
                if r == rank:
                    slabs.append(own)
                    continue
                p = ctypes.c_void_p()
                buf = ctypes.create_string_buffer(hr, _lib.PS_DCP_IPC_HANDLE_BYTES)
                _lib.check(lib.ps_dcp_ipc_open(buf, ctypes.byref(p)))
                slabs.append(int(p.value))
                opened.append(int(p.value))
        dist.barrier(group)  # every mapping exists before any rank signals
        return cls(world, rank, nbytes, slabs, dev, own, tuple(opened))

    @classmethod
    def emulated(cls, world: int, nbytes: int, device=None) -> list:
        """Every rank's view of a ``world``-rank group whose slabs all live on
        one GPU."""
        dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        with torch.cuda.device(dev):
            slabs = [_alloc(nbytes) for _ in range(world)]
        return [cls(world, r, nbytes, list(slabs), dev, slabs[r]) for r in range(world)]

    def close(self) -> None:
        """Unmap the peers' slabs and free this rank's (after a group barrier,
        so that no peer still reads it)."""
        lib = _lib.load()
        with torch.cuda.device(self.device):
            torch.cuda.synchronize(self.device)
            for p in self._opened:
                _lib.check(lib.ps_dcp_ipc_close(p))
            if self._own:
                _lib.check(lib.ps_dcp_slab_free(self._own))
        self._opened, self._own = (), 0
