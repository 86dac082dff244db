"""ctypes binding of libhmb.so (the C ABI in include/hmb.h).

The library is built in-tree by ``python -m heteromega_b200.build``. There is no fallback:
if it is missing or fails to load, every operation raises.
"""
import ctypes
import os

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "libhmb.so")

HMB_OK = 0
# hmb_status (include/hmb.h)
HMB_ERR_ARG, HMB_ERR_ALIGN, HMB_ERR_VALUE, HMB_ERR_WORKSPACE, HMB_ERR_UNSUPPORTED, HMB_ERR_CUDA, HMB_ERR_TIMEOUT = -1, -2, -3, -4, -5, -6, -7
HMB_BF16, HMB_FP16, HMB_FP32 = 0, 1, 2
HMB_GATE_UP_BLOCKED, HMB_GATE_UP_INTERLEAVED = 0, 1
HMB_EPI_STORE, HMB_EPI_SWIGLU = 0, 1
HMB_TP_CHAIN_IN, HMB_TP_CHAIN_OUT = 1, 2
TILE_K, TILE_N, TILE_BYTES = 128, 64, 4352

_i64 = ctypes.c_int64
_int = ctypes.c_int
_vp = ctypes.c_void_p
_sz = ctypes.c_size_t

# name -> (restype, argtypes); every symbol that include/hmb.h declares.
SIGNATURES = {
    "hmb_status_string": (ctypes.c_char_p, [_int]),
    "hmb_version": (_int, []),
    "hmb_last_cuda_error": (_int, []),
    "hmb_packed_bytes": (_i64, [_i64, _i64]),
    "hmb_packed_tile_index": (_i64, [_i64, _i64, _i64, _i64]),
    "hmb_pack_w4a16": (_int, [_vp, _vp, _vp, _i64, _i64, _vp]),
    "hmb_slice_tile_counts": (_int, [_i64, _i64, _i64, _i64, _vp, _vp]),
    "hmb_slice_tile_map": (_int, [_i64, _i64, _i64, _i64, _int, _vp, _vp]),
    "hmb_gather_tiles": (_int, [_vp, _i64, _vp, _vp, _i64, _vp, _vp]),
    "hmb_pack_w4a16_device": (_int, [_vp, _vp, _vp, _i64, _i64, _vp, _vp, _vp]),
    "hmb_w4a16_dequant": (_int, [_vp, _i64, _i64, _i64, _i64, _vp, _i64, _vp]),
    "hmb_w4a16_gemv": (_int, [_vp, _i64, _i64, _vp, _i64, _int, _vp, _i64, _int, _i64, _i64, _i64, _i64, _int, _int, _int,
                              _vp, _sz, _vp]),
    "hmb_w4a16_gemv_workspace": (_sz, [_i64, _i64, _i64, _int, _int]),
    "hmb_w4a16_gemv_noalloc": (_int, [_vp, _i64, _i64, _vp, _i64, _int, _vp, _i64, _int, _i64, _i64, _i64, _i64, _int, _int,
                                      _int, _vp]),
    "hmb_w4a16_gemm": (_int, [_vp, _i64, _i64, _vp, _i64, _int, _vp, _i64, _int, _i64, _i64, _i64, _i64, _int, _int, _vp]),
    "hmb_w4a16_gemm_supports": (_int, [_i64, _i64, _i64, _int]),
    "hmb_w4a16_gemm_plan": (_int, [_i64, _i64, _i64, _int, _int, _vp]),
    "hmb_w4a16_ffn": (_int, [_vp, _vp, _i64, _i64, _i64, _int, _vp, _i64, _int, _vp, _i64, _int, _i64, _vp, _sz, _vp]),
    "hmb_w4a16_ffn_workspace": (_sz, [_i64, _i64, _i64]),
    "hmb_selftest_bounded_wait": (_int, [_i64, _vp]),
    "hmb_comm_handle_bytes": (_sz, []),
    "hmb_comm_create": (_int, [_int, _int, _sz, _vp, _vp]),
    "hmb_comm_connect": (_int, [_vp, _vp]),
    "hmb_allreduce_partials": (_int, [_vp, _i64, _int, _vp, _vp, ctypes.c_uint64]),
    "hmb_comm_destroy": (_int, [_vp]),
    "hmb_allreduce_residual_norm": (_int, [_vp, _int, _vp, _vp, _i64, _i64, ctypes.c_float, _vp, _vp, ctypes.c_uint64]),
    "hmb_comm_out": (_int, [_vp, _vp, _vp]),
    "hmb_tp_ffn_layer": (_int, [_vp, _vp, _vp, _i64, _i64, _i64, _int, _vp, _vp, _vp, ctypes.c_float, _i64, _vp, _sz, _vp,
                                ctypes.c_uint64]),
    "hmb_tp_ffn_layer_workspace": (_sz, [_i64, _i64, _i64]),
    "hmb_tp_ffn_layer_chained": (_int, [_vp, _vp, _vp, _i64, _i64, _i64, _int, _vp, _vp, _vp, ctypes.c_float, _i64, _vp, _sz,
                                        _vp, ctypes.c_uint64, _int]),
    "hmb_comm_rows": (_int, [_vp, _i64, _i64, _vp, _vp]),
    "hmb_device_status": (_int, [_vp, _vp]),
    "hmb_silu_mul": (_int, [_vp, _i64, _vp, _i64, _i64, _i64, _int, _vp]),
    "hmb_residual_add2": (_int, [_vp, _i64, _vp, _i64, _int, _vp, _i64, _int, _i64, _i64, _vp]),
    "hmb_residual_norm": (_int, [_vp, _i64, _vp, _i64, _vp, _i64, _vp, _vp, _i64, _i64, _i64, ctypes.c_float, _vp]),
}

_LIB = None


class HmbError(RuntimeError):
    """A libhmb entry point returned a negative hmb_status."""

    def __init__(self, what, status, cuda_error=0):
        self.status = status
        self.cuda_error = cuda_error
        msg = f"{what}: {lib().hmb_status_string(status).decode()} (status {status}"
        msg += f", cudaError {cuda_error})" if status == -6 else ")"
        super().__init__(msg)


def lib():
    """The loaded library. Raises if it was not built."""
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `python -m heteromega_b200.build` "
                              "(heteromega_b200 has no CPU fallback)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = L
    return _LIB


def check(rc, what):
    if rc != HMB_OK:
        raise HmbError(what, rc, lib().hmb_last_cuda_error())
    return rc
