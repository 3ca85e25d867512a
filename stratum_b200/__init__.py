"""stratum_b200: B200-native (sm_100a) kernels behind Stratum's NF4 frozen-weight path.

The package keeps the reference's hot-path names (stratum/__init__.py:51-54,
stratum/upload.py, stratum/nf4_linear.py) so it drops in for that path; the
compute runs in libstratum_nf4.so (C ABI: include/stratum_nf4.h).
"""

from .functional import QuantState, dequantize_4bit, quantize_4bit

__all__ = [
    "QuantState",
    "quantize_4bit",
    "dequantize_4bit",
]
