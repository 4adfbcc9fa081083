"""q3b200 -- host side of a B200 (sm_100a) Qwen3-0.6B Q8_0 decode path.

Python over the C ABI of libq3b200.so (include/q3b200.h) through ctypes; no
PyTorch.  Mirrors the public functions of the reference's IREE module
(model/qwen3_full.mlir: @run, @decode, @prefill_all, @init_chat, @chat_turn).
"""
from ._lib import LIB_PATH, Q3Error, lib
from .device import DeviceArray, Events, device_count, device_info, set_device, synchronize
from .model import BatchDecoder, DeviceWeights, Qwen3Decoder
from .weights import synthetic_weights

__all__ = ["LIB_PATH", "Q3Error", "lib", "DeviceArray", "Events", "device_count", "device_info",
           "set_device", "synchronize", "BatchDecoder", "DeviceWeights", "Qwen3Decoder", "synthetic_weights"]
