"""malaga_b200: B200-native decode engine for NLLB-200 / M2M100 translation.

The compute path is libmalaga_b200.so (hand-written sm_100a CUDA kernels behind
the C ABI of include/malaga_b200.h); this package is its host-side mirror of
rzafiamy/malaga's malaga-core decode API plus the GGUF converter.
"""
from .translator import Batch, Engine, GenOptions, Translator  # noqa: F401
from ._lib import MgbError  # noqa: F401

__all__ = ["Engine", "Batch", "GenOptions", "Translator", "MgbError"]
