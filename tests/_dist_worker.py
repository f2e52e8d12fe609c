"""Rank body of the multi-process tests (run under torch.multiprocessing spawn, gloo on CPU).

The GPU span step is replaced by an identity "separation" on the CPU: every chunk's output is
its own gathered input (oracle.runtime.gather_chunk), overlap-added with the reference fades
(oracle.dsp.Accumulator). The sharding, the span placement and the reduction are the product
code of ancha_b200.distributed.
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


def run(rank, world, port, out_dir, samples, chunk, overlap, fail_rank, timeout_s=20):
    import torch.distributed as dist
    from ancha_b200.distributed import ChunkPlan, separate_distributed
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))
    try:
        rng = np.random.default_rng(7)
        planes = (rng.standard_normal((2, samples)) * 0.1).astype(np.float32)
        plan = ChunkPlan.of(samples, chunk, overlap)

        def span(p, pl, first, last):
            if rank == fail_rank:
                raise RuntimeError("injected rank failure")
            return identity_span(p, pl, first, last)

        try:
            out = separate_distributed(planes, plan, span, 2)
            status = "ok"
        except Exception as e:  # the failing rank, or a peer whose reduce lost it
            out, status = None, f"{type(e).__name__}: {e}"
        with open(os.path.join(out_dir, f"status{rank}.txt"), "w") as f:
            f.write(status)
        if out is not None:
            np.save(os.path.join(out_dir, "stems.npy"), out)
            np.save(os.path.join(out_dir, "planes.npy"), planes)
    finally:
        if fail_rank < 0:
            dist.destroy_process_group()
