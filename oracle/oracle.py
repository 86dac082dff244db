"""CPU oracle -- TEST INFRASTRUCTURE ONLY.

ctypes access to the two CPU checkers of this repository:

* ``_build/liboracle.so``: the plain-C restatement in ``w4a16_oracle.c`` of HeteroMega's
  packed W4A16 definition (see that file's header for the reference file:line of each
  routine);
* ``_ref/libhm_ref_{avx512,scalar}.so``: the reference's own CPU AVX GEMV
  (``src/cpu_avx_kernels/w4a16_gemv_avx_packed.cpp:28-292``) compiled unchanged by
  ``oracle/Makefile``.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg import this
module, and only to check or time the CPU side. The product never does.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
TILE_K, TILE_N, TILE_BYTES = 128, 64, 4352

_c_i64 = ctypes.c_int64
_ptr = ctypes.c_void_p


def _p(a):
    return ctypes.c_void_p(a.ctypes.data) if a is not None else None


def build():
    """Compile the C restatement (needs gcc only)."""
    subprocess.run(["make", "-s", "-C", HERE, "_build/liboracle.so"], check=True)


def build_reference():
    """Compile the reference's AVX GEMV from its sources (needs the reference tree)."""
    subprocess.run(["make", "-s", "-C", HERE, "ref"], check=True)


_LIB = None


def lib():
    global _LIB
    if _LIB is None:
        path = os.path.join(HERE, "_build", "liboracle.so")
        if not os.path.exists(path):
            build()
        L = ctypes.CDLL(path)
        L.orc_tile_index.restype = _c_i64
        L.orc_tile_index.argtypes = [_c_i64] * 4
        L.orc_pack.restype = ctypes.c_int
        L.orc_pack.argtypes = [_ptr, _ptr, _ptr, _c_i64, _c_i64, _ptr]
        L.orc_unpack.argtypes = [_ptr, _c_i64, _c_i64, _c_i64, _c_i64, _ptr, _ptr, _ptr]
        L.orc_dequant.argtypes = [_ptr, _c_i64, _c_i64, _c_i64, _c_i64, _ptr]
        L.orc_gemv.argtypes = [_ptr, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _ptr, _c_i64, _c_i64, _ptr, _ptr, _c_i64]
        L.orc_silu_mul.argtypes = [_ptr, _c_i64, _ptr, _c_i64, _c_i64, _c_i64, ctypes.c_int]
        L.orc_residual_add2.argtypes = [_ptr, _ptr, ctypes.c_int, _ptr, ctypes.c_int, _c_i64]
        L.orc_ffn.argtypes = [_ptr, _ptr, _c_i64, _c_i64, _c_i64, ctypes.c_int, _ptr, _c_i64, _ptr, _ptr, _ptr]
        L.orc_residual_norm.argtypes = [_ptr, _ptr, ctypes.c_int, _ptr, _ptr, _c_i64, _c_i64, ctypes.c_float]
        _LIB = L
    return _LIB


# ---- bf16 helpers (round to nearest even, as npu/ffn/reference.py:26-35) ---------------------

def bf16_bits(values):
    """fp32 values -> uint16 bf16 bits, ties to even."""
    u = np.ascontiguousarray(np.asarray(values, np.float32)).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def bf16_to_f32(bits):
    return (np.asarray(bits, np.uint16).astype(np.uint32) << 16).view(np.float32)


def bf16_round(values):
    return bf16_to_f32(bf16_bits(values))


# ---- layout ------------------------------------------------------------------------------------

def tile_index(c, r, tiles_k, tiles_n):
    return int(lib().orc_tile_index(c, r, tiles_k, tiles_n))


def pack(q, s_bits, z):
    q = np.ascontiguousarray(q, np.uint8)
    s_bits = np.ascontiguousarray(s_bits, np.uint16)
    z = np.ascontiguousarray(z, np.uint8)
    k, n = q.shape
    out = np.empty((k // TILE_K) * (n // TILE_N) * TILE_BYTES, np.uint8)
    if lib().orc_pack(_p(q), _p(s_bits), _p(z), k, n, _p(out)) != 0:
        raise ValueError("orc_pack: bad shape or value")
    return out


def unpack(packed, packed_k, packed_n, k=None, n=None):
    k = packed_k if k is None else k
    n = packed_n if n is None else n
    packed = np.ascontiguousarray(packed, np.uint8)
    q = np.empty((k, n), np.uint8)
    s = np.empty((k // TILE_K, n), np.uint16)
    z = np.empty((k // TILE_K, n), np.uint8)
    lib().orc_unpack(_p(packed), packed_k, packed_n, k, n, _p(q), _p(s), _p(z))
    return q, s, z


def dequant(packed, packed_k, packed_n, k=None, n=None):
    k = packed_k if k is None else k
    n = packed_n if n is None else n
    packed = np.ascontiguousarray(packed, np.uint8)
    w = np.empty((k, n), np.float32)
    lib().orc_dequant(_p(packed), packed_k, packed_n, k, n, _p(w))
    return w


# ---- arithmetic ---------------------------------------------------------------------------------

def gemv(packed, packed_k, packed_n, x_bits, n=None, k=None, n0=0):
    """Rows of x (bf16 bits [m, >=k]) times columns [n0, n0+n) of the first k rows of a packed
    [packed_k, packed_n] matrix. Returns (fp32 sums [m, n], bf16 bits [m, n])."""
    x_bits = np.ascontiguousarray(np.atleast_2d(x_bits), np.uint16)
    m = x_bits.shape[0]
    k = packed_k if k is None else k
    n = packed_n - n0 if n is None else n
    packed = np.ascontiguousarray(packed, np.uint8)
    y32 = np.empty((m, n), np.float32)
    y16 = np.empty((m, n), np.uint16)
    lib().orc_gemv(_p(packed), packed_k, packed_n, k, n0, n, _p(x_bits), x_bits.shape[1], m, _p(y32), _p(y16), n)
    return y32, y16


def silu_mul(gate_up_bits, n, layout):
    gu = np.ascontiguousarray(np.atleast_2d(gate_up_bits), np.uint16)
    m = gu.shape[0]
    act = np.empty((m, n), np.uint16)
    lib().orc_silu_mul(_p(gu), gu.shape[1], _p(act), n, m, n, int(layout))
    return act


def residual_add2(x_bits, y_g, y_n):
    x = np.ascontiguousarray(x_bits, np.uint16).copy()
    yg = np.ascontiguousarray(y_g)
    yn = np.ascontiguousarray(y_n)
    lib().orc_residual_add2(_p(x), _p(yg), int(yg.dtype == np.float32), _p(yn), int(yn.dtype == np.float32), x.size)
    return x


def residual_norm(x_bits, addends, weight_bits, eps, with_normed=True):
    """The layer boundary (orc_residual_norm): addends is a list of bf16 bit arrays shaped like x (summed
    into x in list order), weight_bits bf16 [h] or None. Returns (new x bits, normed bits or None)."""
    x = np.ascontiguousarray(np.atleast_2d(x_bits), np.uint16).copy()
    m, h = x.shape
    add = np.ascontiguousarray(np.stack([np.atleast_2d(a) for a in addends]) if addends else np.zeros((0, m, h)), np.uint16)
    w = None if weight_bits is None else np.ascontiguousarray(weight_bits, np.uint16)
    normed = np.empty((m, h), np.uint16) if with_normed else None
    lib().orc_residual_norm(_p(x), _p(add) if len(addends) else None, len(addends), _p(w), _p(normed), m, h, float(eps))
    return x, normed


def ffn(gate_up, down, h, n, stored, layout, x_bits):
    """FFN slice of the first n of `stored` packed channels. Returns (y bf16 bits, y fp32) [m, h]."""
    x = np.ascontiguousarray(np.atleast_2d(x_bits), np.uint16)
    m = x.shape[0]
    scratch = np.empty(m * 3 * n, np.uint16)
    y16 = np.empty((m, h), np.uint16)
    y32 = np.empty((m, h), np.float32)
    lib().orc_ffn(_p(np.ascontiguousarray(gate_up, np.uint8)), _p(np.ascontiguousarray(down, np.uint8)), h, n, stored,
                  int(layout), _p(x), m, _p(scratch), _p(y16), _p(y32))
    return y16, y32


# ---- the reference's own AVX kernel, built from its sources --------------------------------------

def _host_has_avx512_bf16():
    try:
        with open("/proc/cpuinfo") as f:
            flags = f.read()
        return "avx512_bf16" in flags and "avx512f" in flags
    except OSError:
        return False


class ReferenceAVX:
    """w4a16_gemv_cpu_fused_packed from oracle/_ref (AVX512-BF16 build when the host has it,
    else the reference's own scalar branch)."""

    def __init__(self):
        self.avx512 = _host_has_avx512_bf16()
        name = "libhm_ref_avx512.so" if self.avx512 else "libhm_ref_scalar.so"
        path = os.path.join(HERE, "_ref", name)
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} is not built (make -C oracle ref, with the reference tree present)")
        self.path = path
        L = ctypes.CDLL(path)
        L.hmref_gemv.restype = ctypes.c_int
        L.hmref_gemv.argtypes = [_ptr, _ptr, _ptr, _c_i64, _c_i64, ctypes.c_int, _c_i64, _c_i64]
        L.hmref_threads.restype = ctypes.c_int
        self._L = L

    @staticmethod
    def available():
        name = "libhm_ref_avx512.so" if _host_has_avx512_bf16() else "libhm_ref_scalar.so"
        return os.path.exists(os.path.join(HERE, "_ref", name))

    def gemv(self, x_bits, packed, k, n, threads=0, out=None, start_col=0, end_col=-1):
        x = np.ascontiguousarray(np.asarray(x_bits, np.uint16).reshape(-1)[:k])
        if out is None:
            out = np.zeros(n, np.uint16)
        rc = self._L.hmref_gemv(_p(out), _p(x), _p(packed), k, n, int(threads), start_col, end_col)
        if rc != 0:
            raise RuntimeError("reference AVX GEMV raised")
        return out

    def threads(self):
        return int(self._L.hmref_threads())

    def ffn_row(self, x_bits, gate, up, down, h, inter, threads=0, scratch=None):
        """The reference model's CPU FFN for one token (unified_llm_w4a16.cpp:2873-2886 with
        the AVX GEMV): gate, up, fp32 SiLU*up rounded once, down. Returns bf16 bits [h]."""
        g = self.gemv(x_bits, gate, h, inter, threads)
        u = self.gemv(x_bits, up, h, inter, threads)
        act = silu_mul(np.concatenate([g, u])[None, :], inter, 0)[0]
        return self.gemv(act, down, inter, h, threads)
