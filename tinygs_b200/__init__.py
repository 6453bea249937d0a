"""tinygs_b200: B200-native training hot path of tinygs (Gaussian splatting).

The computation lives in libtgs_b200.so (CUDA, sm_100a) behind the C ABI in
include/tgs_abi.h; this package holds the ctypes binding, the Python mirror
of the reference plugin interfaces and the seeded synthetic scenes.
"""
from ._abi import load_library, header_symbols  # noqa: F401
