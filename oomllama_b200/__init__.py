"""B200-native (sm_100a) grouped-query attention step for OomLlama.

The compute path is liboomattn.so (C ABI in include/oomattn.h); this package is
its host-side mirror of the reference's TurboEngine interface.
"""
from .turbo import (OomFile, Q8DecoderLayer, Q8Matrix, Q8Model, TurboConfig, TurboEngine,  # noqa: F401
                    compute_rope_freqs, oom_scan, q8_unpack)

__all__ = ["TurboConfig", "TurboEngine", "compute_rope_freqs", "Q8Matrix", "Q8DecoderLayer", "Q8Model", "q8_unpack", "OomFile", "oom_scan"]
