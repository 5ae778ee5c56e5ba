"""per_b200 - a B200-native prioritized experience replay engine.

Drop-in for triton-per's `PERBuffer` (triton backend): PyTorch host code over
hand-written sm_100a CUDA kernels behind a C ABI (include/per_b200.h).
"""

from .buffer import BLOCK_P, PERBuffer, SampleOut

__all__ = ["BLOCK_P", "PERBuffer", "SampleOut"]
