"""TinyGiant MoE expert-FFN hot path, B200-native (sm_100a CUDA behind a C ABI)."""
from ._lib import find_library, load_tinygiant_lib  # noqa: F401

__version__ = "0.1.0"
