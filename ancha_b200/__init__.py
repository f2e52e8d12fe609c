"""B200-native engine for the RoFormer source-separation hot path of 3tic-project/Ancha.

The arithmetic lives in ``lib/libancha_b200.so`` (hand-written sm_100a CUDA kernels behind
the C ABI of ``include/ancha_b200.h``); this package is the Python mirror of the reference's
SDK and kernel plug-in API over that library. There is no CPU fallback: the functions here
raise ``AnchaError`` when the library or a GPU is missing.
"""
from ._native import AnchaError, LIB_PATH  # noqa: F401
from .config import Manifest, ModelConfig, mel_band_table  # noqa: F401

__version__ = "0.1.0"


def load_library():
    """Load (and return) the native library; raises AnchaError if it was not built."""
    from . import _native
    return _native.lib()
