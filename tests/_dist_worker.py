"""Rank body of the multi-process tests (run under torch.multiprocessing spawn, gloo on CPU).

The GPU steps are replaced by an identity "separation" on the CPU: every chunk's output is its
own gathered input (oracle.runtime.gather_chunk), overlap-added with the reference fades
(oracle.dsp.Accumulator), reading only the PCM slice ancha_chunk_pcm_range names (the rest of the
track is NaN, so a wrong slice shows up as a non-finite result). The sharding, the ownership, the
halo exchange and the gather are the product code of ancha_b200.distributed.
"""
import datetime
import os

import numpy as np


def identity_span(planes, plan, first, last):
    from oracle.dsp import Accumulator
    from oracle.dsp import ChunkPlan as OraclePlan
    from oracle.runtime import gather_chunk
    op = OraclePlan(plan.chunk_samples, plan.overlap)
    starts = op.starts(plan.length)
    acc = Accumulator(2, plan.length)
    for start in starts[first:last]:
        acc.add(op, start, gather_chunk(planes.astype(np.float64), start, plan.border, plan.length,
                                        plan.chunk_samples))
    lo, hi = plan.span(first, last)
    return acc.sums[:, lo:hi].astype(np.float32), acc.weights[lo:hi].astype(np.float32)


class CpuIdentityShard:
    """CPU stand-in for the GPU steps: the identity separation, torch adds and division."""

    def __init__(self, fail=False):
        import torch
        self.device = torch.device("cpu")
        self.fail = fail
        self.pcm_ranges = []

    def span(self, planes, plan, first, last):
        import torch
        if self.fail:
            raise RuntimeError("injected rank failure")
        # The GPU step reads only this slice of the track: the identity span must too.
        plo, phi = plan.pcm_range(first, last)
        self.pcm_ranges.append((plo, phi))
        sliced = np.full_like(planes, np.nan)
        sliced[:, plo:phi] = planes[:, plo:phi]
        s, w = identity_span(sliced, plan, first, last)
        return torch.from_numpy(s), torch.from_numpy(w)

    def add(self, sums, weights, offset, piece):
        sums[:, offset:offset + piece.shape[1]] += piece[:-1]
        weights[offset:offset + piece.shape[1]] += piece[-1]

    def finish(self, sums, weights, offset, count):
        return sums[:, offset:offset + count] / weights[offset:offset + count]

    def check(self):
        pass


def run(rank, world, port, out_dir, samples, chunk, overlap, fail_rank, timeout_s=20):
    import torch.distributed as dist
    from ancha_b200.distributed import ChunkPlan, separate_distributed
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))
    try:
        rng = np.random.default_rng(7)
        planes = (rng.standard_normal((2, samples)) * 0.1).astype(np.float32)
        plan = ChunkPlan.of(samples, chunk, overlap)

        ops = CpuIdentityShard(fail=rank == fail_rank)
        try:
            out = separate_distributed(planes, plan, ops, 2)
            status = "ok"
        except Exception as e:  # the failing rank, or a peer whose exchange lost it
            out, status = None, f"{type(e).__name__}: {e}"
        with open(os.path.join(out_dir, f"status{rank}.txt"), "w") as f:
            f.write(status)
        if out is not None:
            np.save(os.path.join(out_dir, "stems.npy"), out)
            np.save(os.path.join(out_dir, "planes.npy"), planes)
    finally:
        if fail_rank < 0:
            dist.destroy_process_group()
