"""B200-native (sm_100a) grouped-query attention step for OomLlama.

The compute path is liboomattn.so (C ABI in include/oomattn.h); this package is
its host-side mirror of the reference's TurboEngine interface.
"""
from .turbo import Q8DecoderLayer, Q8Matrix, TurboConfig, TurboEngine, compute_rope_freqs, q8_unpack  # noqa: F401

__all__ = ["TurboConfig", "TurboEngine", "compute_rope_freqs", "Q8Matrix", "Q8DecoderLayer", "q8_unpack"]
