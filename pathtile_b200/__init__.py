"""pathtile_b200 -- B200-native (sm_100a) short depthwise Conv1D training path.

FWD, input gradient (dX) and weight gradient (dK) in FP32 for L <= 48 and
K <= 48, behind the operator API of the reference's kernels/warp_tiled.py
(:mod:`pathtile_b200.warp_tiled`) and kernels/warp_tiled_ampere.py
(:mod:`pathtile_b200.runtime`).  The math runs in hand-written CUDA kernels in
``libpathtile_b200.so`` (C ABI: include/pathtile_b200.h); there is no host
fallback.
"""
from ._lib import PathTileError
from .ops import dk, dx, fwd
from .runtime import (
    AmpereWarpRuntime,
    B200WarpRuntime,
    DepthConvAmpere,
    DepthConvB200,
    depthwise_conv_ampere,
    depthwise_conv_b200,
    get_runtime,
    install_runtime,
)
from .warp_tiled import DepthwiseConvShared, depthwise_conv_shared

__version__ = "0.1.0"

__all__ = [
    "PathTileError",
    "fwd",
    "dx",
    "dk",
    "B200WarpRuntime",
    "AmpereWarpRuntime",
    "DepthConvB200",
    "DepthConvAmpere",
    "depthwise_conv_b200",
    "depthwise_conv_ampere",
    "install_runtime",
    "get_runtime",
    "DepthwiseConvShared",
    "depthwise_conv_shared",
]
