"""Model and task API over the C ABI, mirroring the reference's SDK.

* :class:`Roformer` is ``Roformer::load`` / ``forward`` (``crates/ancha-models/src/network.rs:
  80-88, 301-400``): a package loaded onto one GPU; ``forward`` maps a packed spectrum
  ``[chunks, frames, bins·4]`` to complex masks ``[chunks, stems, bins·2, 2, frames]`` on the
  device.
* :func:`separate` is ``backend::separate`` (``src/backend.rs:145-199``) with
  :class:`SeparateOptions` (``src/runtime.rs:21-31``): WAV in, ``vocals.wav`` /
  ``instrument.wav`` / ``run.json`` out, published atomically; it returns the run report.
* :func:`separate_pcm` separates host PCM already in memory on one or more GPUs.
"""
from __future__ import annotations

import ctypes as C
import json
from dataclasses import dataclass, field
from typing import Callable, Optional, Sequence

import numpy as np

from . import _native as N


class Roformer:
    """A model package resident on one GPU (not re-entrant; one per device and thread)."""

    def __init__(self, package: str, device: int = 0, precision: str = "f16"):
        """``precision``: "f16" (the default: 16-bit tensor-core operands within the 16-bit mode's
        50 dB bar), "bf16" (below it on these models) or "f32" (the reference's arithmetic)."""
        self.precision = N.PRECISIONS[precision]
        handle = C.c_void_p()
        N.check(N.lib().ancha_model_load(package.encode(), device, self.precision, C.byref(handle)))
        self._h = handle
        self.device = device
        vals = [C.c_int() for _ in range(7)]
        N.check(N.lib().ancha_model_info(self._h, *[C.byref(v) for v in vals]))
        (self.stems, self.bands, self.dim, self.bins, self.chunk_samples, self.hop,
         self.overlap) = (v.value for v in vals)

    @property
    def handle(self):
        return self._h

    def frames(self, samples: Optional[int] = None) -> int:
        return (samples or self.chunk_samples) // self.hop + 1

    def forward(self, spectrum, cancel: Optional[C.c_int] = None):
        """Masks for a CUDA f32 tensor ``[chunks, frames, bins·4]`` (or ``[frames, bins·4]``)."""
        import torch
        squeeze = spectrum.dim() == 2
        s = spectrum.unsqueeze(0) if squeeze else spectrum
        s = s.contiguous().float()
        chunks, frames, cols = s.shape
        if cols != self.bins * 4:
            raise N.AnchaError(N.E_INVALID, "invalid model spectrum shape")
        masks = torch.empty((chunks, self.stems, self.bins * 2, 2, frames), dtype=torch.float32,
                            device=s.device)
        stream = C.c_void_p(torch.cuda.current_stream(s.device).cuda_stream)
        N.check(N.lib().ancha_model_forward(self._h, s.data_ptr(), chunks, frames, masks.data_ptr(),
                                            None if cancel is None else C.byref(cancel), stream))
        return masks[0] if squeeze else masks

    def close(self):
        if getattr(self, "_h", None):
            N.lib().ancha_model_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def separate_pcm(models: Sequence[Roformer], planes: np.ndarray, chunk_samples: int = 0,
                 overlap: int = 0, batch_chunks: int = 0, cancel: Optional[C.c_int] = None,
                 out: Optional[np.ndarray] = None):
    """Stems ``[stems, 2, samples]`` (host f32) for host PCM ``[2, samples]`` on ``models``
    (one per GPU; chunks are sharded in contiguous ranges). Returns ``(stems, seconds)``.
    ``out`` (optional) is a C-contiguous float32 array of that shape to write into, e.g. a view
    of pinned host memory."""
    planes = np.ascontiguousarray(planes, dtype=np.float32)
    if planes.ndim != 2 or planes.shape[0] != 2:
        raise N.AnchaError(N.E_INVALID, "planes must be [2, samples]")
    samples = planes.shape[1]
    if out is None:
        out = np.empty((models[0].stems, 2, samples), dtype=np.float32)
    elif out.dtype != np.float32 or not out.flags.c_contiguous or out.shape != (models[0].stems, 2, samples):
        raise N.AnchaError(N.E_INVALID, "out must be a C-contiguous float32 [stems, 2, samples] array")
    handles = (C.c_void_p * len(models))(*[m.handle for m in models])
    secs = C.c_double()
    fp = C.POINTER(C.c_float)
    N.check(N.lib().ancha_separate_pcm(handles, len(models), planes.ctypes.data_as(fp), samples,
                                       chunk_samples, overlap, batch_chunks,
                                       None if cancel is None else C.byref(cancel),
                                       out.ctypes.data_as(fp), C.byref(secs)))
    return out, secs.value


@dataclass
class SeparateOptions:
    """``runtime::SeparateOptions`` (runtime.rs:21-31) for the CUDA engine."""
    input: str
    model: str
    output: str
    chunk_samples: Optional[int] = None
    overlap: Optional[int] = None
    precision: str = "f16"
    batch_chunks: int = 0
    start_seconds: float = 0.0
    duration_seconds: Optional[float] = None
    devices: Sequence[int] = field(default_factory=lambda: [0])


def separate(options: SeparateOptions, cancelled: Optional[C.c_int] = None,
             progress: Optional[Callable[[int, int], None]] = None) -> dict:
    """Blocking separation task; returns the ``run.json`` report as a dict."""
    o = N.SeparateOpts(options.input.encode(), options.model.encode(), options.output.encode(),
                       options.chunk_samples or 0, options.overlap or 0,
                       N.PRECISIONS[options.precision],
                       options.batch_chunks, options.start_seconds,
                       options.duration_seconds or 0.0)
    devs = (C.c_int * len(options.devices))(*options.devices)
    cb = N.PROGRESS(lambda d, t, _u: progress(d, t)) if progress else N.PROGRESS()
    out = C.c_void_p()
    N.check(N.lib().ancha_separate(C.byref(o), len(options.devices), devs, cb, None,
                                   None if cancelled is None else C.byref(cancelled), C.byref(out)))
    try:
        return json.loads(C.string_at(out.value).decode())
    finally:
        N.lib().ancha_free_string(out)
