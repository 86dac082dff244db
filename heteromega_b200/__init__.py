"""heteromega_b200: a B200-native drop-in for HeteroMega's W4A16 SwiGLU FFN hot path.

Packed-int4 tile layout and kernel interfaces of glassescrab/HeteroMega, hand-written
sm_100a CUDA behind a C ABI (include/hmb.h, libhmb.so), exposed to Python as
torch.ops.heteromega.* custom operators and as the reference's gpu_ffn / hipkernels APIs.
"""
from . import _lib
from ._lib import HmbError, lib
from .gpu_ffn import (FfnLayerQuant, FfnSliceWeights, GateUpLayout, GemmKernel, GemvKernel, GpuFfnBuffers, GpuFfnModel,
                      LinearOptions, gemm_w4a16, gemm_w4a16_ffn, gemm_w4a16_ffn_supports, gemm_w4a16_supports, gemv_w4a16,
                      gpu_ffn_slice_forward, kTileBytes, kTileK, kTileN, pack_ffn_slice, pack_w4a16, packed_linear,
                      packed_tile_index, padded_rows, residual_add2, silu_mul, slice_packed_ffn)

__all__ = [
    "FfnLayerQuant", "FfnSliceWeights", "GateUpLayout", "GemmKernel", "GemvKernel", "GpuFfnBuffers", "GpuFfnModel",
    "HmbError", "LinearOptions", "gemm_w4a16", "gemm_w4a16_ffn", "gemm_w4a16_ffn_supports", "gemm_w4a16_supports",
    "gemv_w4a16", "gpu_ffn_slice_forward", "kTileBytes", "kTileK", "kTileN", "lib", "pack_ffn_slice", "pack_w4a16",
    "packed_linear", "packed_tile_index", "padded_rows", "residual_add2", "silu_mul", "slice_packed_ffn",
]
