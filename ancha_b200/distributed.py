"""One track separated by several processes, one GPU each, over a ``torch.distributed`` group.

The reference separates a track chunk by chunk on one device (``src/runtime.rs:103-225``);
the chunks are independent until the weighted overlap-add (``chunk.rs:37-88``), so the plan
shards cleanly: rank r runs a contiguous range of chunk starts on its GPU
(``ancha_separate_span``) and returns the overlap-add of those chunks over the samples they
cover. The only exchange is the sum of those partial spans, which overlap where two ranks'
chunks overlap: each rank places its span in a zero track-length buffer, one ``reduce``
(SUM) brings them to the destination rank, which divides by the summed weights and crops the
reflect border exactly as the single-process path does (``runtime.cpp::separate_pcm``).

The span step is a parameter (``span_fn``) so the sharding and the exchange can run on CPU
ranks (``gloo``) in tests, with a stand-in for the GPU step.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import Callable, Optional, Tuple

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


SpanFn = Callable[[np.ndarray, ChunkPlan, int, int], Tuple[np.ndarray, np.ndarray]]


def gpu_span(model, batch_chunks: int = 0, cancel: Optional[C.c_int] = None) -> SpanFn:
    """The GPU step: ``ancha_separate_span`` of ``model`` (an :class:`ancha_b200.model.Roformer`)."""

    def run(planes: np.ndarray, plan: ChunkPlan, first: int, last: int):
        lo, hi = plan.span(first, last)
        sums = np.zeros((model.stems * 2, hi - lo), dtype=np.float32)
        weights = np.zeros(hi - lo, dtype=np.float32)
        if last > first:
            fp = C.POINTER(C.c_float)
            N.check(N.lib().ancha_separate_span(
                model.handle, planes.ctypes.data_as(fp), plan.samples, plan.chunk_samples, plan.overlap,
                batch_chunks, first, last, None if cancel is None else C.byref(cancel),
                sums.ctypes.data_as(fp), weights.ctypes.data_as(fp)))
        return sums, weights

    return run


def separate_distributed(planes: np.ndarray, plan: ChunkPlan, span_fn: SpanFn, planes_out: int,
                         group=None, dst: int = 0) -> Optional[np.ndarray]:
    """Stems ``[planes_out // 2, 2, samples]`` of host PCM ``planes [2, samples]`` on rank
    ``dst`` (None on the other ranks). Every rank of ``group`` must call it with the same
    ``planes`` and ``plan``; each runs ``span_fn`` on its own chunk range."""
    import torch
    import torch.distributed as dist
    planes = np.ascontiguousarray(planes, dtype=np.float32)
    if planes.ndim != 2 or planes.shape[0] != 2 or planes.shape[1] != plan.samples:
        raise N.AnchaError(N.E_INVALID, "planes must be [2, samples] of the plan's track")
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    first, last = shard(plan.chunks, rank, world)
    lo, hi = plan.span(first, last)
    sums, weights = span_fn(planes, plan, first, last)
    if sums.shape != (planes_out, hi - lo) or weights.shape != (hi - lo,):
        raise N.AnchaError(N.E_INVALID, "span step returned the wrong shape")
    # One buffer [planes_out + 1, length]: the partial sums, then the weights.
    dev = torch.device("cuda", torch.cuda.current_device()) \
        if dist.get_backend(group) == "nccl" else torch.device("cpu")
    acc = torch.zeros((planes_out + 1, plan.length), dtype=torch.float32, device=dev)
    if hi > lo:
        acc[:planes_out, lo:hi] = torch.from_numpy(sums).to(dev)
        acc[planes_out, lo:hi] = torch.from_numpy(weights).to(dev)
    dist.reduce(acc, dst=dst, op=dist.ReduceOp.SUM, group=group)
    if rank != dst:
        return None
    acc = acc.cpu().numpy()
    if not np.all(acc[planes_out] > 0.0):
        raise N.AnchaError(N.E_INVALID, "uncovered overlap-add sample")
    w = acc[planes_out, plan.border:plan.border + plan.samples]
    out = acc[:planes_out, plan.border:plan.border + plan.samples] / w
    if not np.all(np.isfinite(out)):
        raise N.AnchaError(N.E_NONFINITE, "non-finite chunk output")
    return out.reshape(planes_out // 2, 2, plan.samples)
