"""Symmetric device heaps for in-kernel peer-to-peer exchange.

Each rank of a process group allocates one device buffer of the same size (``cudaMalloc``) and the
ranks exchange CUDA IPC handles, so every rank can address every peer's copy. Sub-buffers are carved
out by a deterministic bump allocator keyed by name: all ranks allocate the same keys in the same
order, so a key has the same offset everywhere and a kernel can write ``peer_base[p] + offset``.

Layout: bytes [0, 512) hold the flags ``[purpose][16 sources]`` (int32) that peers write remotely;
bytes [512, 1024) hold this rank's producer completion counters (one per purpose). Both start at 0.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops._ext import ext

FLAGS_OFF = 0
COUNTERS_OFF = 512
DATA_OFF = 1024
ALIGN = 256
_DT = {torch.bfloat16: 0, torch.float32: 1, torch.int32: 2}
_ES = {torch.bfloat16: 2, torch.float32: 4, torch.int32: 4}


class SymmetricHeap:
    def __init__(self, group, nbytes: int, device: torch.device):
        self.group = group
        self.world = dist.get_world_size(group)
        self.my = dist.get_rank(group)
        self.device = torch.device(device)
        self.nbytes = int(nbytes)
        ptr, handle = ext().ipc_alloc(self.nbytes)
        self.local = ptr
        hs = [torch.empty(64, dtype=torch.uint8, device=self.device) for _ in range(self.world)]
        dist.all_gather(hs, handle.to(self.device), group=group)
        self.peers = [ptr if r == self.my else ext().ipc_open(hs[r].cpu()) for r in range(self.world)]
        self.top = DATA_OFF
        self.offsets: dict = {}
        self.epochs = [0] * 32
        self._maps: dict = {}
        self.counters = ext().heap_tensor(self.local, COUNTERS_OFF, [128], _DT[torch.int32], self.device.index)

    def alloc(self, key, nbytes: int) -> int:
        off = self.offsets.get(key)
        if off is None:
            off = self.top
            self.top = (off + int(nbytes) + ALIGN - 1) // ALIGN * ALIGN
            if self.top > self.nbytes:
                raise MemoryError(f"symmetric heap exhausted ({self.top} > {self.nbytes} bytes)")
            self.offsets[key] = (off, int(nbytes))
            return off
        if off[1] < nbytes:
            raise ValueError(f"heap buffer {key!r} was allocated with {off[1]} bytes, {nbytes} requested")
        return off[0]

    def tensor(self, off: int, shape, dtype) -> torch.Tensor:
        return ext().heap_tensor(self.local, off, list(shape), _DT[dtype], self.device.index)

    def peer_store(self, off: int, rows: int, cols: int, epl: int, cap: int):
        """Destination of a grouped GEMM whose epilogue stores group ``s * epl + e``'s rows into rank
        s's bf16 ``[rows, cols]`` buffer at ``off`` (``ops.gemm.PeerStore``). The per-rank tensor maps
        are encoded once per buffer and kept on the device."""
        from ..ops.gemm import PeerStore

        key = ("maps", off, rows, cols)
        maps = self._maps.get(key)
        if maps is None:
            maps = ext().peer_store_maps(self.peers, off, cols, rows).to(self.device)
            self._maps[key] = maps
        return PeerStore(maps, epl, self.my, cap)

    def next_epoch(self, purpose: int) -> int:
        self.epochs[purpose] += 1
        return self.epochs[purpose]

    def counter(self, purpose: int) -> torch.Tensor:
        return self.counters[purpose:purpose + 1]


_HEAPS: dict = {}


def heap_for(group, device, min_bytes: int, name: str = "ep") -> SymmetricHeap:
    """The group's heap called ``name``, created (collectively) on first use with at least
    ``min_bytes``."""
    key = (id(group), torch.device(device).index, name)
    h = _HEAPS.get(key)
    if h is None:
        h = SymmetricHeap(group, min_bytes, device)
        _HEAPS[key] = h
    return h


def nbytes(shape, dtype) -> int:
    n = _ES[dtype]
    for s in shape:
        n *= int(s)
    return n
