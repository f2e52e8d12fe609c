"""ctypes binding of ``include/ancha_b200.h`` (the library is ``lib/libancha_b200.so``).

The library is required: :func:`lib` raises ``AnchaError`` when it is missing instead of
falling back to any CPU implementation.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "lib", "libancha_b200.so")

OK, E_UNSUPPORTED, E_INVALID, E_CUDA, E_CANCELLED, E_IO, E_TIMEOUT, E_NONFINITE = \
    0, -1, -2, -3, -4, -5, -6, -7
F32, BF16, F16 = 0, 1, 2
PRECISION_F32, PRECISION_BF16, PRECISION_F16 = 0, 1, 2
PRECISIONS = {"f32": PRECISION_F32, "bf16": PRECISION_BF16, "f16": PRECISION_F16}
W_KN, W_NK = 0, 1
ACT_NONE, ACT_GELU, ACT_TANH, ACT_GLU = 0, 1, 2, 3

STATUS_NAMES = {OK: "ok", E_UNSUPPORTED: "unsupported", E_INVALID: "invalid", E_CUDA: "cuda",
                E_CANCELLED: "cancelled", E_IO: "io", E_TIMEOUT: "timeout",
                E_NONFINITE: "non-finite"}

# Every symbol the header declares (checked by the CPU test suite).
EXPORTS = ("ancha_last_error", "ancha_version", "ancha_available", "ancha_wait_selftest", "ancha_attention_fwd",
           "ancha_attention_workspace", "ancha_attention_fwd_ws", "ancha_linear_fwd", "ancha_linear_workspace",
           "ancha_linear_fwd_ws", "ancha_stft_fwd", "ancha_istft_masked", "ancha_istft_masked_static", "ancha_ola_add",
           "ancha_model_load", "ancha_model_info", "ancha_model_forward", "ancha_model_free",
           "ancha_mdx23c_load", "ancha_mdx23c_info", "ancha_mdx23c_forward", "ancha_mdx23c_separate_pcm",
           "ancha_mdx23c_plan", "ancha_mdx23c_free", "ancha_mdx_graph_inspect", "ancha_mdx_load",
           "ancha_mdx_output_shape", "ancha_mdx_forward", "ancha_mdx_separate_pcm", "ancha_mdx_set_gemm", "ancha_mdx_free",
           "ancha_separate", "ancha_separate_pcm", "ancha_separate_device",
           "ancha_separate_status", "ancha_chunk_plan", "ancha_chunk_span", "ancha_chunk_pcm_range",
           "ancha_separate_span", "ancha_separate_span_device", "ancha_span_add", "ancha_span_finish",
           "ancha_free_string")


class AnchaError(RuntimeError):
    """A non-zero status from the library; ``status`` holds the code."""

    def __init__(self, status: int, message: str):
        super().__init__(f"{message} [{STATUS_NAMES.get(status, status)}]")
        self.status = status


class AttnDesc(C.Structure):
    _fields_ = [("groups", C.c_int), ("tokens", C.c_int), ("heads", C.c_int),
                ("head_dim", C.c_int), ("dtype", C.c_int), ("ld", C.c_int64),
                ("out_ld", C.c_int64), ("group_inner", C.c_int64),
                ("group_inner_stride", C.c_int64), ("group_outer_stride", C.c_int64),
                ("token_stride", C.c_int64), ("q_col", C.c_int), ("k_col", C.c_int),
                ("v_col", C.c_int), ("gate_col", C.c_int), ("out_col", C.c_int)]


class LinearDesc(C.Structure):
    _fields_ = [("m", C.c_int), ("n", C.c_int), ("k", C.c_int), ("dtype", C.c_int),
                ("out_dtype", C.c_int), ("weight_layout", C.c_int), ("ldx", C.c_int64),
                ("ldw", C.c_int64), ("ldout", C.c_int64), ("ldres", C.c_int64),
                ("act", C.c_int), ("rope_width", C.c_int), ("rope_tokens", C.c_int),
                ("rope_div", C.c_int), ("row_scale", C.c_void_p)]


class SeparateOpts(C.Structure):
    _fields_ = [("input", C.c_char_p), ("model", C.c_char_p), ("output", C.c_char_p),
                ("chunk_samples", C.c_int64), ("overlap", C.c_int), ("precision", C.c_int),
                ("batch_chunks", C.c_int), ("start_seconds", C.c_double),
                ("duration_seconds", C.c_double)]


class MdxTask(C.Structure):
    _fields_ = [("n_fft", C.c_int), ("hop", C.c_int), ("bins", C.c_int), ("frames", C.c_int),
                ("compensate", C.c_double), ("overlap", C.c_double), ("denoise", C.c_int), ("batch", C.c_int)]


PROGRESS = C.CFUNCTYPE(None, C.c_size_t, C.c_size_t, C.c_void_p)

_lock = threading.Lock()
_lib = None


def lib() -> C.CDLL:
    """The loaded library (raises AnchaError if it was not built)."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise AnchaError(E_UNSUPPORTED, f"CUDA library not built: {LIB_PATH} "
                                            "(run `python -m ancha_b200.build`)")
        L = C.CDLL(LIB_PATH)
        vp, i32, i64 = C.c_void_p, C.c_int, C.c_int64
        fp = C.POINTER(C.c_float)
        sig = {
            "ancha_last_error": (C.c_char_p, []),
            "ancha_version": (C.c_char_p, []),
            "ancha_available": (i32, [i32]),
            "ancha_wait_selftest": (i32, [i64, vp]),
            "ancha_attention_fwd": (i32, [C.POINTER(AttnDesc), vp, vp, vp, vp, vp, vp]),
            "ancha_attention_workspace": (i32, [C.POINTER(AttnDesc), C.POINTER(C.c_size_t)]),
            "ancha_attention_fwd_ws": (i32, [C.POINTER(AttnDesc), vp, vp, vp, vp, vp, vp, C.c_size_t, vp]),
            "ancha_linear_fwd": (i32, [C.POINTER(LinearDesc), vp, vp, vp, vp, vp, vp, vp]),
            "ancha_linear_workspace": (i32, [C.POINTER(LinearDesc), C.POINTER(C.c_size_t)]),
            "ancha_linear_fwd_ws": (i32, [C.POINTER(LinearDesc), vp, vp, vp, vp, vp, vp, vp, C.c_size_t, vp]),
            "ancha_stft_fwd": (i32, [vp, i32, i32, i32, vp, vp]),
            "ancha_istft_masked": (i32, [vp, vp, i32, i32, i32, i32, i32, vp, vp, vp]),
            "ancha_istft_masked_static": (i32, [vp, vp, i32, i32, i32, i32, i32, vp, vp, vp]),
            "ancha_ola_add": (i32, [vp, i32, i32, i32, i32, C.POINTER(i64), i64, vp, vp, vp]),
            "ancha_model_load": (i32, [C.c_char_p, i32, i32, C.POINTER(vp)]),
            "ancha_model_info": (i32, [vp] + [C.POINTER(i32)] * 7),
            "ancha_model_forward": (i32, [vp, vp, i32, i32, vp, C.POINTER(i32), vp]),
            "ancha_model_free": (None, [vp]),
            "ancha_mdx23c_load": (i32, [C.c_char_p, i32, i32, C.POINTER(vp)]),
            "ancha_mdx23c_info": (i32, [vp] + [C.POINTER(i32)] * 7),
            "ancha_mdx23c_forward": (i32, [vp, vp, i32, i32, vp, C.POINTER(i32), vp]),
            "ancha_mdx23c_separate_pcm": (i32, [vp, fp, i64, i32, i32, C.POINTER(i32), fp,
                                                C.POINTER(C.c_double)]),
            "ancha_mdx23c_plan": (i32, [i64, i64, i32] + [C.POINTER(i64)] * 5),
            "ancha_mdx23c_free": (None, [vp]),
            "ancha_mdx_graph_inspect": (i32, [vp, C.c_size_t, i32] + [C.POINTER(i32)] * 4),
            "ancha_mdx_load": (i32, [vp, C.c_size_t, i32, i32, C.POINTER(vp)]),
            "ancha_mdx_output_shape": (i32, [vp, C.POINTER(i64), C.POINTER(i64)]),
            "ancha_mdx_forward": (i32, [vp, vp, C.POINTER(i64), vp, C.POINTER(i32), vp]),
            "ancha_mdx_separate_pcm": (i32, [vp, C.POINTER(MdxTask), fp, i64, C.POINTER(i32), fp, fp,
                                             C.POINTER(C.c_double)]),
            "ancha_mdx_set_gemm": (i32, [vp, i32]),
            "ancha_mdx_free": (None, [vp]),
            "ancha_separate": (i32, [C.POINTER(SeparateOpts), i32, C.POINTER(i32), PROGRESS,
                                     vp, C.POINTER(i32), C.POINTER(C.c_void_p)]),
            "ancha_separate_pcm": (i32, [C.POINTER(vp), i32, fp, i64, i64, i32, i32,
                                         C.POINTER(i32), fp, C.POINTER(C.c_double)]),
            "ancha_separate_device": (i32, [vp, vp, i64, i64, i32, i32, vp, vp]),
            "ancha_separate_status": (i32, [vp, vp]),
            "ancha_chunk_plan": (i32, [i64, i64, i32, C.POINTER(i64), C.POINTER(i64), C.POINTER(i64)]),
            "ancha_chunk_span": (i32, [i64, i64, i32, i64, i64, C.POINTER(i64), C.POINTER(i64)]),
            "ancha_chunk_pcm_range": (i32, [i64, i64, i32, i64, i64, C.POINTER(i64), C.POINTER(i64)]),
            "ancha_separate_span": (i32, [vp, fp, i64, i64, i32, i32, i64, i64, vp, fp, fp]),
            "ancha_separate_span_device": (i32, [vp, vp, i64, i64, i64, i64, i32, i32, i64, i64, vp, vp, vp]),
            "ancha_span_add": (i32, [vp, vp, i32, i64, i64, vp, i64, vp]),
            "ancha_span_finish": (i32, [vp, vp, i32, i64, i64, i64, vp, i64, vp, vp]),
            "ancha_free_string": (None, [vp]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
        return L


def last_error() -> str:
    return lib().ancha_last_error().decode(errors="replace")


def check(status: int) -> int:
    """Raise AnchaError for a non-zero status."""
    if status != OK:
        raise AnchaError(status, last_error())
    return status
