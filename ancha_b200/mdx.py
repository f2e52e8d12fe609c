"""Classic MDX ONNX graphs over the C ABI (``crates/ancha-models/src/mdx.rs``).

:func:`inspect` reads an ONNX model and builds the classic MDX executable graph exactly as
``Graph::from_bytes`` does (validation, BatchNormalization folding, schedule), on the host.
:class:`Graph` is that graph resident on one GPU; ``forward`` is ``Graph::forward`` on CUDA
f32 NCHW tensors.
"""
from __future__ import annotations

import ctypes as C
from typing import Optional

from . import _native as N


def inspect(onnx: bytes, optimized: bool = True) -> dict:
    """Node, instruction, folded-BatchNormalization and constant counts of a valid graph;
    raises ``AnchaError`` (``E_INVALID``) with the reference's message otherwise."""
    vals = [C.c_int() for _ in range(4)]
    buf = C.create_string_buffer(onnx, len(onnx))
    N.check(N.lib().ancha_mdx_graph_inspect(buf, len(onnx), int(optimized), *[C.byref(v) for v in vals]))
    return dict(zip(("nodes", "instructions", "folded_bn", "constants"), (v.value for v in vals)))


class Graph:
    """A classic MDX ONNX graph on one GPU (not re-entrant)."""

    def __init__(self, onnx: bytes, device: int = 0, optimized: bool = True, gemm: Optional[str] = "f32"):
        """``gemm``: "f32" (the default, as the reference's CUDA path runs ``Graph::forward`` with
        conv_gemm, mdx.rs:472-530), "bf16" or "f16" runs eligible convolutions and constant-weight
        MatMuls as GEMMs in that precision (``ancha_mdx_set_gemm``); None runs every operation on
        its direct kernel."""
        self._h = None
        if gemm is not None and gemm not in N.PRECISIONS:
            raise N.AnchaError(N.E_INVALID, f"unknown conv_gemm precision {gemm!r}")
        handle = C.c_void_p()
        buf = C.create_string_buffer(onnx, len(onnx))
        N.check(N.lib().ancha_mdx_load(buf, len(onnx), int(optimized), device, C.byref(handle)))
        self._h = handle
        self.device = device
        if gemm is not None:
            N.check(N.lib().ancha_mdx_set_gemm(self._h, N.PRECISIONS[gemm]))

    def output_shape(self, shape) -> tuple:
        i = (C.c_int64 * 4)(*shape)
        o = (C.c_int64 * 4)()
        N.check(N.lib().ancha_mdx_output_shape(self._h, i, o))
        return tuple(o)

    def forward(self, x, cancel: Optional[C.c_int] = None):
        """Output of the graph for a CUDA f32 NCHW tensor."""
        import torch
        x = x.contiguous().float()
        if x.dim() != 4:
            raise N.AnchaError(N.E_INVALID, "input must be NCHW")
        shape = tuple(x.shape)
        out = torch.empty(self.output_shape(shape), dtype=torch.float32, device=x.device)
        stream = C.c_void_p(torch.cuda.current_stream(x.device).cuda_stream)
        N.check(N.lib().ancha_mdx_forward(self._h, x.data_ptr(), (C.c_int64 * 4)(*shape), out.data_ptr(),
                                          None if cancel is None else C.byref(cancel), stream))
        return out

    def separate_pcm(self, planes, n_fft: int = 6144, hop: int = 1024, bins: int = 3072, frames: int = 256,
                     compensate: float = 1.0, overlap: Optional[float] = None, denoise: bool = False,
                     batch: int = 1, cancel: Optional[C.c_int] = None):
        """``separate_mdx`` on host PCM ``[2, samples]`` → ``(predicted, residual, seconds)``."""
        import numpy as np
        x = np.ascontiguousarray(planes, dtype=np.float32)
        if x.ndim != 2 or x.shape[0] != 2:
            raise N.AnchaError(N.E_INVALID, "planes must be [2, samples]")
        task = N.MdxTask(n_fft, hop, bins, frames, compensate, -1.0 if overlap is None else overlap, int(denoise), batch)
        pred = np.empty_like(x)
        res = np.empty_like(x)
        secs = C.c_double()
        fp = C.POINTER(C.c_float)
        N.check(N.lib().ancha_mdx_separate_pcm(self._h, C.byref(task), x.ctypes.data_as(fp), x.shape[1],
                                               None if cancel is None else C.byref(cancel),
                                               pred.ctypes.data_as(fp), res.ctypes.data_as(fp), C.byref(secs)))
        return pred, res, secs.value

    def close(self) -> None:
        if self._h:
            N.lib().ancha_mdx_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
