"""aethermind_b200 -- B200-native (sm_100a) Llama prefill/decode hot path.

The compute path is the CUDA library in lib/libaethermind_b200.so (C ABI in
include/aethermind_b200.h). Importing this package loads it and fails loudly
if it has not been built; there is no CPU fallback.
"""
from ._lib import AmError, lib  # noqa: F401

__all__ = ["AmError", "lib"]
