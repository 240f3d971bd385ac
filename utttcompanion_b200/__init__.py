"""B200-native (sm_100a) uTTT serving hot path.

Drop-in replacements for the reference's fast-weight operator functions
(``model/uttt_layer.py`` of Phova/uTTTCompanion) backed by hand-written
tcgen05/TMA CUDA kernels behind a C ABI (``include/uttt_b200.h``).
"""

from ._lib import load as load_library  # noqa: F401

__all__ = ["load_library"]
