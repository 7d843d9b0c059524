"""msb: B200-native expert-indexed matmul over a GPU slot pool.

Drop-in for MoEStream's hot path (expert id -> slot remap, per-slot grouping,
mul_mat_id over quantized IQ4_NL / MXFP4 experts, slot fills). The compute
runs in libmsb.so (hand-written sm_100a CUDA); this package binds its C ABI.
"""
from ._lib import (LIB_PATH, NO_SLOT, TYPE_BF16, TYPE_F32, TYPE_IQ4_NL, TYPE_MXFP4, MsbError,
                   lib)
from .cache import DeviceSlotStreamer, ExpertCache, SlotStreamer

__all__ = ["LIB_PATH", "NO_SLOT", "TYPE_BF16", "TYPE_F32", "TYPE_IQ4_NL", "TYPE_MXFP4",
           "MsbError", "lib", "ExpertCache", "SlotStreamer", "DeviceSlotStreamer"]
