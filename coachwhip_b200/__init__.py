"""coachwhip-b200: the mixture-of-experts layer of coachwhip, B200-native.

The product is libcwx.so (CUDA for sm_100a behind the C ABI in include/cwx.h); this package is
the Python host side that mirrors the reference's MoE layer interface (coachwhip_b200.moe) and
builds the library (coachwhip_b200.build). Importing the package loads nothing; the first call
into the library loads libcwx.so and raises if it is missing.
"""

from ._lib import (ACT_CLAMPED_SWIGLU, ACT_MODE_CANDLE, ACT_MODE_F32, ACT_SILU, TYPE_IQ2_S, TYPE_IQ3_S,
                   TYPE_MXFP4, TYPE_Q4_K, TYPE_Q6_K, TYPE_Q8_0, CwxError)

__all__ = ["CwxError", "ACT_MODE_CANDLE", "ACT_MODE_F32", "ACT_SILU", "ACT_CLAMPED_SWIGLU", "TYPE_Q8_0", "TYPE_Q4_K",
           "TYPE_Q6_K", "TYPE_IQ3_S", "TYPE_IQ2_S", "TYPE_MXFP4"]
