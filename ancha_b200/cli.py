"""``python -m ancha_b200 separate``: the reference CLI's separate command (src/main.rs:67-134)
for RoFormer packages on this CUDA engine, over ``ancha_separate``.

Same positional input and flags as the reference for what this engine runs: ``--model``,
``-o/--output``, ``--backend`` (only ``cuda``: there is no other backend and no CPU fallback),
``--device``, ``--start``, ``--duration``, ``--chunk-samples``, ``--overlap``; plus ``--devices``
(a comma-separated list, one model per GPU), ``--precision`` and ``--batch-chunks``. Writes the
stem WAVs and ``run.json`` into the output directory (atomic publish) and prints the report.
Exit status: 0 on success, 1 when the engine reports an error, 2 for a usage error.
"""
from __future__ import annotations

import argparse
import json
import sys
from typing import List, Optional

from . import _native as N


def parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(prog="python -m ancha_b200")
    sub = p.add_subparsers(dest="command", required=True)
    s = sub.add_parser("separate", help="separate a WAV file with a RoFormer model package")
    s.add_argument("input")
    s.add_argument("--model", required=True)
    s.add_argument("-o", "--output", required=True)
    s.add_argument("--backend", default="cuda")
    s.add_argument("--device", type=int, default=None)
    s.add_argument("--devices", default=None, help="comma-separated GPU ordinals (one model per GPU)")
    s.add_argument("--start", type=float, default=0.0)
    s.add_argument("--duration", type=float, default=None)
    s.add_argument("--chunk-samples", type=int, default=None)
    s.add_argument("--overlap", type=int, default=None)
    # f16 operands meet the 16-bit parity bar (the model's GEMM inputs are unit-normed or bounded
    # activations, so f16's range suffices); bf16's 8-bit mantissa does not on this model.
    s.add_argument("--precision", default="f16", choices=sorted(N.PRECISIONS))
    s.add_argument("--batch-chunks", type=int, default=0, help="chunks per model call (0: balanced default)")
    return p


def options(args: argparse.Namespace):
    """The SeparateOptions of parsed arguments; ValueError for a usage error."""
    from .model import SeparateOptions
    if args.backend != "cuda":
        raise ValueError(f"backend {args.backend!r} is not built here: only the CUDA engine (--backend cuda)")
    if args.device is not None and args.devices is not None:
        raise ValueError("give --device or --devices, not both")
    if args.devices is not None:
        try:
            devices = [int(d) for d in args.devices.split(",") if d.strip()]
        except ValueError:
            raise ValueError(f"--devices must list GPU ordinals, got {args.devices!r}") from None
        if not devices:
            raise ValueError("--devices is empty")
    else:
        devices = [args.device or 0]
    if args.start < 0 or (args.duration is not None and args.duration <= 0):
        raise ValueError("--start must be >= 0 and --duration > 0")
    return SeparateOptions(input=args.input, model=args.model, output=args.output,
                           chunk_samples=args.chunk_samples, overlap=args.overlap, precision=args.precision,
                           batch_chunks=args.batch_chunks, start_seconds=args.start,
                           duration_seconds=args.duration, devices=devices)


def main(argv: Optional[List[str]] = None) -> int:
    args = parser().parse_args(argv)
    try:
        opts = options(args)
    except ValueError as e:
        print(f"error: {e}", file=sys.stderr)
        return 2
    from .model import separate
    try:
        report = separate(opts)
    except N.AnchaError as e:
        print(f"error: {e}", file=sys.stderr)
        return 1
    print(json.dumps(report, indent=2))
    return 0
