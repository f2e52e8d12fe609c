"""Chunked separation pipeline in numpy (test oracle only).

Restates ``src/runtime.rs:103-238`` of the reference: border and chunk plan (103-116),
per-chunk gather with reflect / zero tail (117-142), per-channel STFT and packing as
``(frame, bin·2 + channel, re/im)`` (143-162), the model call (165-176), the complex mask
multiply with masks ``[stem, row, re/im, frame]`` and iSTFT (181-201), the weighted
overlap-add (204-206), the border crop (210-225) and the one-stem residual (226-238).
"""
from __future__ import annotations

import numpy as np

from .dsp import Accumulator, ChunkPlan, Stft, reflect_index, reflect_indices


def chunk_layout(samples: int, chunk: int, overlap: int):
    """``(plan, border, length, starts)`` for an input of ``samples`` (runtime.rs:103-111)."""
    plan = ChunkPlan(chunk, overlap)
    border = chunk - plan.step
    border = border if samples > 2 * border else 0
    length = samples + 2 * border
    return plan, border, length, plan.starts(length)


def gather_chunk(planes: np.ndarray, start: int, border: int, length: int, chunk: int):
    """``[channels, chunk]`` model input for one chunk start (runtime.rs:117-142)."""
    samples = planes.shape[1]
    remaining = min(length - start, chunk)
    i = np.arange(chunk)
    local = np.where(i < remaining, i, reflect_indices(i, remaining))
    source = reflect_indices(start + local - border, samples)
    out = planes[:, source]
    if remaining <= chunk // 2:
        out = out.copy()
        out[:, i >= remaining] = 0.0
    return out


def pack_spectrum(spectra: list[np.ndarray]) -> np.ndarray:
    """Two ``[frames, bins]`` spectra → ``[frames, bins·4]`` (runtime.rs:148-162)."""
    frames, bins = spectra[0].shape
    packed = np.zeros((frames, bins, 2, 2), dtype=np.float64)
    for ch, s in enumerate(spectra):
        packed[:, :, ch, 0] = s.real
        packed[:, :, ch, 1] = s.imag
    return packed.reshape(frames, bins * 4)


def apply_masks(spectra, masks: np.ndarray, stft: Stft, chunk: int, zero_dc: bool):
    """Complex masks ``[stems, rows, 2, frames]`` → ``[stems, channels, chunk]`` (runtime.rs:181-201)."""
    stems, rows, _, frames = masks.shape
    bins = rows // 2
    out = np.zeros((stems, len(spectra), chunk))
    for s in range(stems):
        for ch, src in enumerate(spectra):
            m = masks[s, ch::2]                     # rows f·2 + ch → [bins, 2, frames]
            mc = (m[:, 0, :] + 1j * m[:, 1, :]).T   # [frames, bins]
            out[s, ch] = stft.inverse(src * mc, chunk, zero_dc)
    return out


def separate(model, planes: np.ndarray, chunk: int | None = None, overlap: int | None = None):
    """Stems ``[stems, 2, samples]`` (and the residual for one-stem models) for stereo input."""
    c = model.config
    chunk = chunk or c["chunk_samples"]
    overlap = overlap or c["overlap"]
    planes = np.asarray(planes, dtype=np.float64)
    samples = planes.shape[1]
    plan, border, length, starts = chunk_layout(samples, chunk, overlap)
    stft = Stft(c["n_fft"], c["hop"])
    accs = [Accumulator(2, length) for _ in c["stems"]]
    for start in starts:
        x = gather_chunk(planes, start, border, length, chunk)
        spectra = [stft.forward(p) for p in x]
        masks = model.forward(pack_spectrum(spectra))
        outputs = apply_masks(spectra, masks, stft, chunk, c["zero_dc"])
        for acc, y in zip(accs, outputs):
            acc.add(plan, start, y)
    stems = np.stack([acc.finish()[:, border:border + samples] for acc in accs])
    residual = planes - stems[0] if stems.shape[0] == 1 else None
    return stems, residual


__all__ = ["chunk_layout", "gather_chunk", "pack_spectrum", "apply_masks", "separate",
           "reflect_index"]
