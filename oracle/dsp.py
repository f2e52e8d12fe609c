"""STFT / iSTFT, reflect padding, chunk plan and overlap-add (test oracle only).

Restates ``crates/ancha-audio/src/dsp.rs`` and ``crates/ancha-audio/src/chunk.rs`` of the
reference. The FFT core of the reference is realfft 3.5.0 / rustfft 6.4.1 (third-party, not
in the reference tree): an unnormalised real-to-complex forward transform and an
unnormalised complex-to-real inverse that ignores the imaginary parts of the DC and Nyquist
bins. ``numpy.fft.rfft`` / ``irfft`` compute the same transforms (``irfft`` divides by n,
which the reference applies explicitly as ``scale = 1/n``, dsp.rs:102).
"""
from __future__ import annotations

import numpy as np


def reflect_index(index: int, length: int) -> int:
    """Reflect padding excluding the edge, repeated as needed (dsp.rs:136-147)."""
    if length <= 1:
        return 0
    period = 2 * (length - 1)
    i = index % period  # Python % is Euclidean for a positive period
    return i if i < length else period - i


def reflect_indices(index: np.ndarray, length: int) -> np.ndarray:
    """Vectorised :func:`reflect_index`."""
    index = np.asarray(index, dtype=np.int64)
    if length <= 1:
        return np.zeros_like(index)
    period = 2 * (length - 1)
    i = np.mod(index, period)
    return np.where(i < length, i, period - i)


def hann(n_fft: int) -> np.ndarray:
    """Periodic Hann window, evaluated in f32 as dsp.rs:40-42 does."""
    i = np.arange(n_fft, dtype=np.float32)
    tau = np.float32(2.0 * np.pi)
    arg = (tau * i) / np.float32(n_fft)
    return (np.float32(0.5) - np.float32(0.5) * np.cos(arg)).astype(np.float32)


class Stft:
    """PyTorch ``center=True`` STFT: periodic Hann, reflect pad, unnormalised FFT (dsp.rs:14-133)."""

    def __init__(self, n_fft: int, hop: int, dtype=np.float64):
        if not (n_fft >= 2 and n_fft % 2 == 0 and 0 < hop <= n_fft // 2):
            raise ValueError("require even FFT >= 2 and hop in 1..=FFT/2")
        self.n_fft, self.hop, self.dtype = n_fft, hop, dtype
        self.window = hann(n_fft).astype(dtype)

    def frames(self, length: int) -> int:
        return length // self.hop + 1

    def forward(self, signal: np.ndarray) -> np.ndarray:
        """``[frames, bins]`` complex spectrum of one channel (dsp.rs:52-79)."""
        signal = np.asarray(signal)
        if signal.shape[0] <= self.n_fft // 2:
            raise ValueError("reflect STFT requires input longer than FFT/2")
        if not np.all(np.isfinite(signal)):
            raise ValueError("non-finite STFT input")
        frames = self.frames(signal.shape[0])
        t = np.arange(frames)[:, None] * self.hop + np.arange(self.n_fft)[None, :]
        idx = reflect_indices(t - self.n_fft // 2, signal.shape[0])
        x = signal.astype(self.dtype)[idx] * self.window[None, :]
        return np.fft.rfft(x, axis=1)

    def inverse(self, spectrum: np.ndarray, length: int, zero_dc: bool) -> np.ndarray:
        """Window-square normalised overlap-add inverse (dsp.rs:82-133)."""
        frames, bins = spectrum.shape
        if bins != self.n_fft // 2 + 1 or frames == 0:
            raise ValueError("invalid spectrum shape")
        total = (frames - 1) * self.hop + self.n_fft
        pad = self.n_fft // 2
        if length + pad > total:
            raise ValueError("requested iSTFT length exceeds frame support")
        spec = np.array(spectrum, dtype=np.complex128 if self.dtype == np.float64 else np.complex64)
        spec[:, 0] = spec[:, 0].real
        spec[:, -1] = spec[:, -1].real
        if zero_dc:
            spec[:, 0] = 0.0
        time = np.fft.irfft(spec, n=self.n_fft, axis=1).astype(self.dtype)  # includes 1/n
        w = self.window
        output = np.zeros(total, dtype=self.dtype)
        denominator = np.zeros(total, dtype=self.dtype)
        for t in range(frames):
            s = t * self.hop
            output[s:s + self.n_fft] += time[t] * w
            denominator[s:s + self.n_fft] += w * w
        seg = denominator[pad:pad + length]
        if np.any(seg <= 1e-11):
            raise ValueError("iSTFT has an uncovered sample")
        result = output[pad:pad + length] / seg
        if not np.all(np.isfinite(result)):
            raise ValueError("non-finite iSTFT output")
        return result


class ChunkPlan:
    """Chunk length and step = chunk / overlap (chunk.rs:1-35)."""

    def __init__(self, samples: int, overlap: int):
        if not (samples > 0 and 0 < overlap <= samples):
            raise ValueError("invalid chunk or overlap divisor")
        self.samples = samples
        self.step = samples // overlap

    def starts(self, length: int) -> list[int]:
        return list(range(0, length, self.step))

    def weight(self, i: int, first: bool, last: bool) -> float:
        fade = max(self.samples // 10, 1)
        if not first and i < fade:
            return (i + 1) / fade
        if not last and i >= self.samples - fade:
            return (self.samples - i) / fade
        return 1.0

    def weights(self, n: int, first: bool, last: bool, dtype=np.float64) -> np.ndarray:
        """``weight(i, first, last)`` for ``i in range(n)``, in f32 as the reference stores it."""
        fade = max(self.samples // 10, 1)
        i = np.arange(n)
        w = np.ones(n, dtype=np.float64)
        if not first:
            head = i < fade
            w[head] = (np.float32(i[head] + 1) / np.float32(fade))
        if not last:
            tail = (i >= self.samples - fade) & ~((not first) & (i < fade))
            w[tail] = (np.float32(self.samples - i[tail]) / np.float32(fade))
        return w.astype(dtype)


class Accumulator:
    """Weighted overlap-add of chunk outputs (chunk.rs:37-88)."""

    def __init__(self, channels: int, length: int, dtype=np.float64):
        if channels <= 0 or length <= 0:
            raise ValueError("empty overlap accumulator")
        self.sums = np.zeros((channels, length), dtype=dtype)
        self.weights = np.zeros(length, dtype=dtype)

    def add(self, plan: ChunkPlan, start: int, planes: np.ndarray) -> None:
        planes = np.asarray(planes)
        if planes.shape != (self.sums.shape[0], plan.samples):
            raise ValueError("chunk output shape mismatch")
        if not np.all(np.isfinite(planes)):
            raise ValueError("non-finite chunk output")
        length = self.weights.shape[0]
        if start >= length:
            raise ValueError("chunk starts past output")
        end = min(start + plan.samples, length)
        n = end - start
        w = plan.weights(n, start == 0, start + plan.samples >= length, self.sums.dtype)
        self.weights[start:end] += w
        self.sums[:, start:end] += w[None, :] * planes[:, :n]

    def finish(self) -> np.ndarray:
        if not np.all(self.weights > 0):
            raise ValueError("uncovered overlap-add sample")
        return self.sums / self.weights[None, :]
