"""One track separated by several processes, one GPU each, over a ``torch.distributed`` group.

The reference separates a track chunk by chunk on one device (``src/runtime.rs:103-225``);
the chunks are independent until the weighted overlap-add (``chunk.rs:37-88``), so the plan
shards cleanly: rank r runs a contiguous range of chunk starts on its GPU and keeps the
overlap-add of those chunks over the samples they cover (its span) in device memory. Each rank
uploads only the track samples its chunks read (``ancha_chunk_pcm_range``).

Rank r owns the output samples from the start of its span to the start of the next rank's span.
The only exchange is the chunk-overlap halo: the columns of a rank's span that fall in a later
rank's owned range (at most chunk − step samples, times stems·2 + 1 rows) are sent to that rank
(point-to-point, NCCL on GPUs, gloo on CPU) and added into its span there. Each rank then divides
and crops its owned range on its own device, and one gather brings the stems to the destination
rank, which is the single-process result (``runtime.cpp::separate_pcm``).

The per-rank steps are an object (``ShardOps``) so the sharding and the exchange can run on CPU
ranks (``gloo``) in tests, with a stand-in for the GPU steps.
"""
from __future__ import annotations

import abc
import ctypes as C
from dataclasses import dataclass
from typing import List, Optional, Tuple

import numpy as np

from . import _native as N


@dataclass(frozen=True)
class ChunkPlan:
    """Chunk plan of a track: ``chunks`` starts, reflect ``border``, padded ``length``."""
    samples: int
    chunk_samples: int
    overlap: int
    chunks: int
    border: int
    length: int

    @staticmethod
    def of(samples: int, chunk_samples: int, overlap: int) -> "ChunkPlan":
        n, b, l = C.c_int64(), C.c_int64(), C.c_int64()
        N.check(N.lib().ancha_chunk_plan(samples, chunk_samples, overlap, C.byref(n), C.byref(b), C.byref(l)))
        return ChunkPlan(samples, chunk_samples, overlap, n.value, b.value, l.value)

    def pcm_range(self, first: int, last: int) -> Tuple[int, int]:
        """Track samples ``[lo, hi)`` read by chunks ``[first, last)`` (reflect padding)."""
        lo, hi = C.c_int64(), C.c_int64()
        N.check(N.lib().ancha_chunk_pcm_range(self.samples, self.chunk_samples, self.overlap, first, last,
                                              C.byref(lo), C.byref(hi)))
        return lo.value, hi.value

    def span(self, first: int, last: int) -> Tuple[int, int]:
        """Padded-track samples ``[lo, hi)`` covered by chunks ``[first, last)``."""
        lo, hi = C.c_int64(), C.c_int64()
        N.check(N.lib().ancha_chunk_span(self.samples, self.chunk_samples, self.overlap, first, last,
                                         C.byref(lo), C.byref(hi)))
        return lo.value, hi.value


def shard(chunks: int, rank: int, world: int) -> Tuple[int, int]:
    """Contiguous chunk range ``[first, last)`` of ``rank``: ceil(chunks / world) per rank, the
    split ``ancha_separate_pcm`` uses across GPUs (trailing ranks may be empty)."""
    if world <= 0 or not 0 <= rank < world:
        raise N.AnchaError(N.E_INVALID, "invalid rank / world size")
    per = -(-chunks // world)
    first = min(chunks, rank * per)
    return first, min(chunks, first + per)


def ownership(plan: ChunkPlan, world: int) -> List[Optional[Tuple[int, int]]]:
    """Padded-track samples ``[lo, hi)`` whose output each rank produces (None: empty shard):
    from the start of the rank's span to the start of the next non-empty rank's span."""
    ranks = [r for r in range(world) if shard(plan.chunks, r, world)[1] > shard(plan.chunks, r, world)[0]]
    own: List[Optional[Tuple[int, int]]] = [None] * world
    for k, r in enumerate(ranks):
        lo = 0 if k == 0 else plan.span(*shard(plan.chunks, r, world))[0]
        hi = plan.span(*shard(plan.chunks, ranks[k + 1], world))[0] if k + 1 < len(ranks) else plan.length
        own[r] = (lo, hi)
    return own


class ShardOps(abc.ABC):
    """The per-rank steps of :func:`separate_distributed` (tensors on ``device``)."""

    device = None

    @abc.abstractmethod
    def span(self, planes: np.ndarray, plan: ChunkPlan, first: int, last: int):
        """Overlap-add of chunks ``[first, last)``: sums ``[planes_out, hi − lo]`` and weights
        ``[hi − lo]`` over ``plan.span(first, last)``."""

    @abc.abstractmethod
    def add(self, sums, weights, offset: int, piece) -> None:
        """Add a received ``[planes_out + 1, w]`` piece at span column ``offset``."""

    @abc.abstractmethod
    def finish(self, sums, weights, offset: int, count: int):
        """``sums[:, offset:offset + count] / weights[offset:offset + count]``."""

    def check(self) -> None:
        """Raise if a device status word reports an error (synchronises)."""


class GpuShard(ShardOps):
    """The GPU steps for a :class:`ancha_b200.model.Roformer` on the current CUDA device:
    ``ancha_separate_span_device``, ``ancha_span_add`` and ``ancha_span_finish`` on torch's
    current stream (which the process group's collectives follow)."""

    def __init__(self, model, batch_chunks: int = 0):
        import torch
        self.model, self.batch = model, batch_chunks
        self.device = torch.device("cuda", torch.cuda.current_device())
        self.flag = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.planes_out = model.stems * 2

    def _stream(self):
        import torch
        return C.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)

    def span(self, planes, plan, first, last):
        import torch
        lo, hi = plan.span(first, last)
        plo, phi = plan.pcm_range(first, last)
        # One copy per channel row: each row of the slice is contiguous in the caller's array
        # (asynchronous when that array is in pinned memory).
        pcm = torch.empty((2, phi - plo), dtype=torch.float32, device=self.device)
        for ch in range(2):
            pcm[ch].copy_(torch.from_numpy(planes[ch, plo:phi]), non_blocking=True)
        sums = torch.empty((self.planes_out, hi - lo), dtype=torch.float32, device=self.device)
        weights = torch.empty(hi - lo, dtype=torch.float32, device=self.device)
        N.check(N.lib().ancha_separate_span_device(
            self.model.handle, pcm.data_ptr(), plo, phi - plo, plan.samples, plan.chunk_samples, plan.overlap,
            self.batch, first, last, sums.data_ptr(), weights.data_ptr(), self._stream()))
        self._pcm = pcm  # kept alive until the enqueued work has read it
        return sums, weights

    def add(self, sums, weights, offset, piece):
        N.check(N.lib().ancha_span_add(sums.data_ptr(), weights.data_ptr(), self.planes_out, sums.shape[1],
                                       offset, piece.data_ptr(), piece.shape[1], self._stream()))

    def finish(self, sums, weights, offset, count):
        import torch
        out = torch.empty((self.planes_out, count), dtype=torch.float32, device=self.device)
        N.check(N.lib().ancha_span_finish(sums.data_ptr(), weights.data_ptr(), self.planes_out, sums.shape[1],
                                          offset, count, out.data_ptr(), count, self.flag.data_ptr(),
                                          self._stream()))
        return out

    def check(self):
        N.check(N.lib().ancha_separate_status(self.model.handle, self._stream()))
        bits = int(self.flag.item())
        self.flag.zero_()
        if bits & 1:
            raise N.AnchaError(N.E_NONFINITE, "non-finite chunk output")
        if bits & 4:
            raise N.AnchaError(N.E_INVALID, "uncovered overlap-add sample")


def separate_distributed(planes: np.ndarray, plan: ChunkPlan, ops: ShardOps, planes_out: int,
                         group=None, dst: int = 0, to_host: bool = True, out: Optional[np.ndarray] = None):
    """Stems ``[planes_out // 2, 2, samples]`` of host PCM ``planes [2, samples]`` on rank
    ``dst`` (None on the other ranks; a device tensor when ``to_host`` is False). Every rank of
    ``group`` must call it with the same ``planes`` and ``plan``; each runs ``ops`` on its own
    chunk range. ``out`` (rank ``dst``, optional) is a C-contiguous float32 host array of the
    stems' shape to copy into, e.g. a view of pinned memory for a faster download. Non-finite
    stems are reported by ``ops.check`` from the device status words."""
    import torch
    import torch.distributed as dist
    planes = np.asarray(planes, dtype=np.float32)
    if planes.ndim != 2 or planes.shape[0] != 2 or planes.shape[1] != plan.samples:
        raise N.AnchaError(N.E_INVALID, "planes must be [2, samples] of the plan's track")
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    shards = [shard(plan.chunks, r, world) for r in range(world)]
    spans = [plan.span(f, l) for f, l in shards]
    own = ownership(plan, world)
    first, last = shards[rank]
    lo, hi = spans[rank]
    dev = ops.device
    # Every rank enters the exchange through one collective (the first point-to-point batch of
    # an NCCL group must not be its first collective), which also reports a rank that failed
    # before it as an error on its peers.
    dist.barrier(group=group)
    sums = weights = None
    if own[rank] is not None:
        sums, weights = ops.span(planes, plan, first, last)
        if tuple(sums.shape) != (planes_out, hi - lo) or tuple(weights.shape) != (hi - lo,):
            raise N.AnchaError(N.E_INVALID, "span step returned the wrong shape")
    # Halo exchange: the columns of rank p's span inside rank q's owned range go from p to q.
    ops_list, received = [], []
    for q in range(world):
        if q == rank or own[q] is None or own[rank] is None:
            continue
        if q > rank:  # send to later owners
            a, b = max(lo, own[q][0]), min(hi, own[q][1])
            if b > a:
                piece = torch.cat([sums[:, a - lo:b - lo], weights[None, a - lo:b - lo]]).contiguous()
                ops_list.append(dist.P2POp(dist.isend, piece, q, group))
        else:  # receive from earlier ranks
            plo, phi = spans[q]
            a, b = max(plo, own[rank][0]), min(phi, own[rank][1])
            if b > a:
                piece = torch.empty((planes_out + 1, b - a), dtype=torch.float32, device=dev)
                ops_list.append(dist.P2POp(dist.irecv, piece, q, group))
                received.append((a, piece))
    for req in (dist.batch_isend_irecv(ops_list) if ops_list else []):
        req.wait()
    for a, piece in received:
        ops.add(sums, weights, a - lo, piece)
    # Division and crop of the owned range, then one gather of the stems at dst.
    pieces = []
    for r in range(world):
        if own[r] is None:
            pieces.append(None)
            continue
        o0, o1 = max(own[r][0], plan.border), min(own[r][1], plan.border + plan.samples)
        pieces.append((o0, o1) if o1 > o0 else None)
    mine = None
    if pieces[rank] is not None:
        o0, o1 = pieces[rank]
        mine = ops.finish(sums, weights, o0 - lo, o1 - o0)
    ops.check()
    out = None
    gather_ops = []
    host_out = out
    if host_out is not None and (host_out.dtype != np.float32 or not host_out.flags.c_contiguous or
                                 host_out.shape != (planes_out // 2, 2, plan.samples)):
        raise N.AnchaError(N.E_INVALID, "out must be a C-contiguous float32 [stems, 2, samples] array")
    if rank == dst:
        out = torch.empty((planes_out, plan.samples), dtype=torch.float32, device=dev)
        parts = []
        for r in range(world):
            if pieces[r] is None:
                continue
            o0, o1 = pieces[r]
            if r == rank:
                out[:, o0 - plan.border:o1 - plan.border] = mine
            else:
                buf = torch.empty((planes_out, o1 - o0), dtype=torch.float32, device=dev)
                gather_ops.append(dist.P2POp(dist.irecv, buf, r, group))
                parts.append((o0, buf))
    elif mine is not None:
        gather_ops.append(dist.P2POp(dist.isend, mine.contiguous(), dst, group))
    for req in (dist.batch_isend_irecv(gather_ops) if gather_ops else []):
        req.wait()
    if rank != dst:
        return None
    for o0, buf in parts:
        out[:, o0 - plan.border:o0 - plan.border + buf.shape[1]] = buf
    out = out.reshape(planes_out // 2, 2, plan.samples)
    if not to_host:
        return out
    if host_out is None:
        return out.cpu().numpy()
    torch.from_numpy(host_out).copy_(out)
    return host_out
