"""Helpers shared by the test modules."""
import numpy as np


def wave(shape, shift):
    """The reference's deterministic test signal (cuda_contracts.rs:183-189)."""
    n = int(np.prod(shape))
    i = np.arange(n, dtype=np.float32)
    return np.tanh(np.sin(i * np.float32(0.731) + np.float32(shift)) * np.float32(1.7)).reshape(shape)


def snr_db(reference, estimate):
    reference = np.asarray(reference, dtype=np.float64)
    err = np.asarray(estimate, dtype=np.float64) - reference
    num = float(np.sum(reference ** 2))
    den = float(np.sum(err ** 2))
    return float("inf") if den == 0 else 10.0 * np.log10(num / den)


def max_abs(a, b):
    return float(np.max(np.abs(np.asarray(a, np.float64) - np.asarray(b, np.float64))))


def bf16_round(x):
    """Round f32 values to bf16 (nearest even), returned as f32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)
