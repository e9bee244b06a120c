"""pixelina_b200 -- B200-native backend for Pixelina's quantized-matmul path.

The compute lives in ``libpxq.so`` (hand-written sm_100a CUDA behind the C ABI
in include/pxq.h); :mod:`pixelina_b200.pxq` is its Python host mirror,
:mod:`pixelina_b200.sharded` splits a matmul's weight rows over the ranks of
a node, and :mod:`pixelina_b200.synth` builds seeded synthetic GGUF weights.
"""
from . import synth  # noqa: F401

__all__ = ["pxq", "synth", "sharded"]
