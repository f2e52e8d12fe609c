"""Multi-process separation of one track (ancha_b200.distributed) on CPU ranks (gloo).

Rank r runs a contiguous chunk range over the PCM slice it needs; the chunk-overlap halos of
the spans go point to point to the ranks that own those samples, each rank divides its own
range and one gather brings the stems to rank 0. The GPU steps are replaced by an identity
separation (each chunk's output is its own input), so the combined result must reproduce the
input track (the fades sum to the overlap-add weights), and must equal the single-process
overlap-add of the oracle. A rank that fails before the exchange must make the others fail with
an error, not hang.
"""
import os
import socket
import tempfile

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from ancha_b200 import _native as N  # noqa: E402
from ancha_b200.distributed import ChunkPlan, shard  # noqa: E402
from oracle.dsp import Accumulator  # noqa: E402
from oracle.dsp import ChunkPlan as OraclePlan  # noqa: E402
from oracle.runtime import chunk_layout, gather_chunk  # noqa: E402


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("samples,chunk,overlap", [(44100, 8192, 4), (5000, 4096, 2), (100000, 352800, 4),
                                                   (30000, 6000, 3)])
def test_chunk_plan_matches_oracle(samples, chunk, overlap):
    plan = ChunkPlan.of(samples, chunk, overlap)
    _, border, length, starts = chunk_layout(samples, chunk, overlap)
    assert (plan.chunks, plan.border, plan.length) == (len(starts), border, length)
    for first in range(len(starts)):
        for last in range(first + 1, len(starts) + 1):
            assert plan.span(first, last) == (starts[first], min(starts[last - 1] + chunk, length))
    assert plan.span(2, 2) == (0, 0) if len(starts) >= 2 else True


def test_chunk_plan_rejects_invalid():
    # the last three: a chunk past 60 s, an overlap divisor above 16 (config.rs:64), a track past 2^36 samples
    for args in [(0, 4096, 4), (1000, 0, 4), (1000, 4096, 0), (1000, 4, 8), (1000, 44100 * 60 + 1, 1),
                 (100000, 8192, 17), ((1 << 36) + 1, 8192, 4)]:
        with pytest.raises(N.AnchaError):
            ChunkPlan.of(*args)
    plan = ChunkPlan.of(44100, 8192, 4)
    with pytest.raises(N.AnchaError):
        plan.span(0, plan.chunks + 1)
    with pytest.raises(N.AnchaError):
        plan.span(3, 2)


def test_pcm_range_covers_every_sample_the_gather_reads():
    from ancha_b200.distributed import ownership
    from oracle.runtime import chunk_layout
    for samples, chunk, overlap in [(44100, 8192, 4), (5000, 4096, 2), (3000, 2048, 4), (30000, 6000, 3),
                                    (1, 4096, 4), (2, 1024, 1)]:
        plan = ChunkPlan.of(samples, chunk, overlap)
        _, border, length, starts = chunk_layout(samples, chunk, overlap)
        period = max(1, 2 * (samples - 1))
        for first in range(len(starts)):
            for last in range(first + 1, min(len(starts), first + 4) + 1):
                lo, hi = plan.span(first, last)
                q = np.arange(lo, hi) - border
                r = np.mod(q, period)
                r = np.where(r < samples, r, period - r) if samples > 1 else np.zeros_like(r)
                assert plan.pcm_range(first, last) == (int(r.min()), int(r.max()) + 1)
        for world in (1, 2, 3, 5):
            own = [o for o in ownership(plan, world) if o is not None]
            assert own[0][0] == 0 and own[-1][1] == plan.length
            assert all(a[1] == b[0] for a, b in zip(own, own[1:]))


def test_shards_partition_the_plan():
    for chunks in range(0, 40):
        for world in range(1, 9):
            ranges = [shard(chunks, r, world) for r in range(world)]
            covered = [i for f, l in ranges for i in range(f, l)]
            assert covered == list(range(chunks))
            assert all(f <= l for f, l in ranges)
    with pytest.raises(N.AnchaError):
        shard(10, 2, 2)


def _spawn(world, samples, chunk, overlap, fail_rank=-1, timeout_s=20):
    import torch.multiprocessing as mp
    out = tempfile.mkdtemp(prefix="ancha_dist_")
    from tests import _dist_worker
    mp.start_processes(_dist_worker.run, args=(world, _free_port(), out, samples, chunk, overlap, fail_rank,
                                               timeout_s),
                       nprocs=world, join=True, start_method="spawn")
    return out


def _oracle_identity(planes, samples, chunk, overlap):
    op, border, length, starts = chunk_layout(samples, chunk, overlap)
    acc = Accumulator(2, length)
    for start in starts:
        acc.add(op, start, gather_chunk(planes.astype(np.float64), start, border, length, chunk))
    return acc.finish()[:, border:border + samples]


@pytest.mark.parametrize("world,samples,chunk,overlap", [(2, 44100, 8192, 4), (2, 30000, 6000, 3),
                                                         (3, 20000, 4096, 4),
                                                         # two chunks per rank, a 1536-sample halo: rank
                                                         # 0's span reaches into rank 2's owned range
                                                         (4, 3000, 2048, 4)])
def test_ranks_reproduce_single_process_overlap_add(world, samples, chunk, overlap):
    out = _spawn(world, samples, chunk, overlap)
    for r in range(world):
        assert open(os.path.join(out, f"status{r}.txt")).read() == "ok"
    stems = np.load(os.path.join(out, "stems.npy"))
    planes = np.load(os.path.join(out, "planes.npy"))
    assert stems.shape == (1, 2, samples)
    ref = _oracle_identity(planes, samples, chunk, overlap)
    assert np.max(np.abs(stems[0] - ref)) < 1e-6
    assert np.max(np.abs(stems[0] - planes)) < 1e-5  # the fades sum to the weights


def test_failed_rank_surfaces_as_error_on_peers():
    out = _spawn(2, 30000, 6000, 3, fail_rank=1, timeout_s=5)
    s0 = open(os.path.join(out, "status0.txt")).read()
    s1 = open(os.path.join(out, "status1.txt")).read()
    assert "injected rank failure" in s1
    assert s0 != "ok"
    assert not os.path.exists(os.path.join(out, "stems.npy"))
