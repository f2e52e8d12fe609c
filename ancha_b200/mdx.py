"""Classic MDX ONNX graphs over the C ABI (``crates/ancha-models/src/mdx.rs``).

:func:`inspect` reads an ONNX model and builds the classic MDX executable graph exactly as
``Graph::from_bytes`` does (validation, BatchNormalization folding, schedule), on the host.
"""
from __future__ import annotations

import ctypes as C

from . import _native as N


def inspect(onnx: bytes, optimized: bool = True) -> dict:
    """Node, instruction, folded-BatchNormalization and constant counts of a valid graph;
    raises ``AnchaError`` (``E_INVALID``) with the reference's message otherwise."""
    vals = [C.c_int() for _ in range(4)]
    buf = C.create_string_buffer(onnx, len(onnx))
    N.check(N.lib().ancha_mdx_graph_inspect(buf, len(onnx), int(optimized), *[C.byref(v) for v in vals]))
    return dict(zip(("nodes", "instructions", "folded_bn", "constants"), (v.value for v in vals)))
