"""dial_b200 -- B200-native (sm_100a) implementation of DIAL's decoder-layer
forward path with weight-only quantized linears.

Python host mirror of the reference interface over the C ABI in
include/dial_b200.h (libdial_b200.so, built by dial-27b_b200/build.py).
"""

from ._abi import (ACT_BF16, ACT_F16, FMT_DENSE, FMT_FP8_BLOCK128, FMT_FP8_ROW, FMT_NVFP4_G16,
                   FMT_W8A16_ROW, LIB_PATH, DialError)
from .engine import Config, Engine, device_status
from .checkpoint import Checkpoint, config_from_checkpoint, load_checkpoint
from .linear import CudaQuantLinear, CudaW8A16Linear, DenseLinear, w8a16_quantize
from .synth import normal_table_bits
from .topology import Topology

__all__ = [
    "ACT_BF16", "ACT_F16", "FMT_DENSE", "FMT_FP8_BLOCK128", "FMT_FP8_ROW", "FMT_NVFP4_G16",
    "FMT_W8A16_ROW", "LIB_PATH", "DialError", "Config", "Engine", "device_status",
    "CudaQuantLinear", "CudaW8A16Linear", "DenseLinear", "w8a16_quantize", "normal_table_bits",
    "Topology", "Checkpoint", "config_from_checkpoint", "load_checkpoint",
]
