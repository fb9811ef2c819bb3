"""B replicated on every rank of a one-process-per-GPU group, over NVLink by peer copies.

The multi-GPU plan keeps one full K x rhs replica of B per rank (each rank multiplies its own
block-row shard by all of B). In a one-process-per-GPU job the replica is filled without NCCL:
every rank allocates its buffer with vbsr_shared_buffer_create, the CUDA IPC handles are exchanged
once over the process group (host objects), and the data moves as copy-engine peer copies
(cudaMemcpyAsync) between the mapped buffers, over NVLink / NVSwitch. B is cut into `world`
chunks, chunk j being rank j's:
  * replicate_from(root): the root's buffer holds all of B; every other rank pulls its own chunk
    from the root, then every rank pulls each other chunk from that chunk's owner (a scatter then
    an allgather: about 2 x |B| / link bandwidth at any rank count);
  * upload_own_chunk + pull_peers: each rank brings only its own chunk from host memory (PCIe) and
    takes the rest from its peers, so the host-to-device traffic per rank is |B| / world.
Ordering between processes is a host barrier on the group (gloo is fine) after each copy phase.
No reference counterpart: the reference is single-GPU.
"""
from __future__ import annotations

import ctypes as C

from . import _check, _lib, _stream_ptr, InvalidArgument


class _IpcHandle(C.Structure):
    _fields_ = [("bytes", C.c_ubyte * 64)]


_vp = C.c_void_p
for _name, _args in {
    "vbsr_shared_buffer_create": [C.c_int, C.c_int64, C.POINTER(_vp)],
    "vbsr_shared_buffer_destroy": [_vp],
    "vbsr_shared_buffer_ptr": [_vp, C.POINTER(_vp)],
    "vbsr_shared_buffer_export": [_vp, C.POINTER(_IpcHandle)],
    "vbsr_shared_buffer_open": [C.POINTER(_IpcHandle), C.c_int, C.POINTER(_vp)],
    "vbsr_shared_buffer_close": [_vp, C.c_int],
    "vbsr_copy_async": [_vp, _vp, C.c_int64, _vp],
}.items():
    getattr(_lib, _name).argtypes = _args
    getattr(_lib, _name).restype = C.c_int


def copy_async(dst: int, src: int, nbytes: int, stream=None) -> None:
    """cudaMemcpyAsync(dst, src, nbytes, cudaMemcpyDefault, stream) on raw pointers."""
    _check(_lib.vbsr_copy_async(dst, src, nbytes, _stream_ptr(stream)))


def chunk_bounds(count: int, world: int, align: int = 64) -> list[tuple[int, int]]:
    """[first, end) of each rank's chunk of `count` floats: contiguous, in rank order, starts on
    multiples of `align` floats, sizes as equal as that allows (the last one takes the rest)."""
    if world < 1 or count < 0:
        raise InvalidArgument("bad chunking arguments")
    cuts = [min(count, (count * j // world) // align * align) for j in range(world)] + [count]
    return [(cuts[j], cuts[j + 1]) for j in range(world)]


class PeerReplica:
    """`buffers` device buffers of `nfloats` floats on `device`, shared with every rank of
    `group` (a torch.distributed process group; host-side use only: handle exchange and
    barriers). Collective: every rank constructs it with the same arguments."""

    def __init__(self, nfloats: int, rank: int, world: int, device: int, group,
                 buffers: int = 1):
        import torch.distributed as dist
        self.n, self.rank, self.world, self.device = int(nfloats), rank, world, device
        self._dist, self._group = dist, group
        self._own = []
        self._peer = [[None] * world for _ in range(buffers)]
        for _ in range(buffers):
            h = _vp()
            _check(_lib.vbsr_shared_buffer_create(device, 4 * max(1, self.n), C.byref(h)))
            self._own.append(h)
        handles = []
        for h in self._own:
            ih = _IpcHandle()
            _check(_lib.vbsr_shared_buffer_export(h, C.byref(ih)))
            handles.append(bytes(ih.bytes))
        every = [None] * world
        dist.all_gather_object(every, handles, group=group)
        for j in range(world):
            for b in range(buffers):
                if j == rank:
                    self._peer[b][j] = self.ptr(b)
                    continue
                ih = _IpcHandle()
                C.memmove(C.addressof(ih), every[j][b], 64)
                p = _vp()
                _check(_lib.vbsr_shared_buffer_open(C.byref(ih), device, C.byref(p)))
                self._peer[b][j] = p.value
        self.chunks = chunk_bounds(self.n, world)

    def ptr(self, b: int = 0) -> int:
        p = _vp()
        _check(_lib.vbsr_shared_buffer_ptr(self._own[b], C.byref(p)))
        return p.value

    def barrier(self) -> None:
        self._dist.barrier(group=self._group)

    def _pull(self, j: int, b: int, stream, src_rank: int | None = None) -> int:
        a, e = self.chunks[j]
        if e > a:
            src = self._peer[b][j if src_rank is None else src_rank]
            copy_async(self.ptr(b) + 4 * a, src + 4 * a, 4 * (e - a), stream)
        return 4 * (e - a)

    def upload_own_chunk(self, host_ptr: int, b: int = 0, stream=None) -> int:
        """Copies this rank's chunk of B from host memory (`host_ptr`: all of B, pinned for an
        asynchronous copy) into buffer b; returns the bytes copied."""
        a, e = self.chunks[self.rank]
        if e > a:
            copy_async(self.ptr(b) + 4 * a, host_ptr + 4 * a, 4 * (e - a), stream)
        return 4 * (e - a)

    def pull_peers(self, b: int = 0, stream=None) -> int:
        """Copies every other rank's chunk from that rank's buffer b (each owner must hold its
        chunk before this is enqueued: a barrier after the owners' uploads); returns the bytes."""
        return sum(self._pull(j, b, stream) for j in range(self.world) if j != self.rank)

    def replicate_from(self, root: int, b: int = 0, stream=None) -> int:
        """Collective: the root's buffer b holds all of B once the root's device work enqueued
        before the call has run; afterwards every rank's does. Returns the bytes this rank
        received."""
        import torch
        got = 0
        torch.cuda.synchronize(self.device)
        self.barrier()  # the root's buffer is complete before anyone reads it
        if self.rank != root:
            got += self._pull(self.rank, b, stream, src_rank=root)
        torch.cuda.synchronize(self.device)
        self.barrier()
        if self.rank != root:  # chunk j from its owner j (the root's own chunk from the root)
            got += self.pull_peers(b, stream)
        torch.cuda.synchronize(self.device)
        self.barrier()
        return got

    def close(self) -> None:
        """Collective: unmaps the peers' buffers, waits for every rank to do the same, frees
        this rank's buffers."""
        if not self._own:
            return
        for b in range(len(self._peer)):
            for j in range(self.world):
                if j != self.rank and self._peer[b][j]:
                    _check(_lib.vbsr_shared_buffer_close(self._peer[b][j], self.device))
                    self._peer[b][j] = None
        self.barrier()
        for h in self._own:
            _lib.vbsr_shared_buffer_destroy(h)
        self._own = []
