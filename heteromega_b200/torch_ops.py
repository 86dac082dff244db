"""PyTorch custom operators ``torch.ops.heteromega.*`` over the C ABI of libhmb.so.

Each operator checks its tensors the way the reference's TORCH_CHECKs do, then calls the
C entry point on the current CUDA stream of the tensors' device. The operators only
enqueue work; they never synchronize. Split-K workspaces are cached per (device, stream),
like the per-stream scratch of the reference (kernels/gpu/src/gemm_w4a16.cu:364-376).
"""
import threading

import torch

from . import _lib
from ._lib import check, lib

_ws_lock = threading.Lock()
_workspaces = {}


def _stream(t):
    return torch.cuda.current_stream(t.device).cuda_stream


def _ptr(t):
    return t.data_ptr() if t is not None else None


def workspace(device, nbytes, kind="gemv"):
    """A zero-filled uint8 buffer of at least nbytes for the current stream of `device`, one per kind
    of call (their layouts differ). Calls on one stream reuse it; the kernels leave its counter words
    zero."""
    stream = torch.cuda.current_stream(device)
    key = (device.index, stream.cuda_stream, kind)
    with _ws_lock:
        buf = _workspaces.get(key)
        if buf is None or buf.numel() < nbytes:
            size = max(nbytes, 1 << 20)
            if buf is not None:
                size = max(size, 2 * buf.numel())
            buf = torch.zeros(size, dtype=torch.uint8, device=device)
            _workspaces[key] = buf
        return buf


def _dtype_code(t):
    if t.dtype == torch.bfloat16:
        return _lib.HMB_BF16
    if t.dtype == torch.float16:
        return _lib.HMB_FP16
    if t.dtype == torch.float32:
        return _lib.HMB_FP32
    raise TypeError(f"unsupported dtype {t.dtype}")


def _rows(t):
    return t.shape[0] if t.dim() == 2 else 1


def _ld(t):
    return t.stride(0) if t.dim() == 2 else t.shape[-1]


def _check_cuda(*ts):
    dev = ts[0].device
    for t in ts:
        if not t.is_cuda or t.device != dev:
            raise ValueError("heteromega: all tensors must be CUDA tensors on one device")


_defs = torch.library.Library("heteromega", "DEF")
_defs.define("w4a16_gemv(Tensor(a!) out, Tensor x, Tensor packed, int k, int n, int packed_k, int packed_n, "
             "int start_col, int epilogue, int layout, int split_k) -> ()")
_defs.define("w4a16_gemm(Tensor(a!) out, Tensor x, Tensor packed, int k, int n, int packed_k, int packed_n, "
             "int start_col, int epilogue, int layout) -> ()")
_defs.define("w4a16_ffn(Tensor(a!) y, Tensor x, Tensor gate_up, Tensor down, int h, int n, int stored, int layout) -> ()")
_defs.define("w4a16_dequant(Tensor(a!) out, Tensor packed, int k, int n, int packed_k, int packed_n) -> ()")
_defs.define("silu_mul(Tensor gate_up, Tensor(a!) act, int layout) -> ()")
_defs.define("residual_add2(Tensor(a!) x, Tensor y_g, Tensor y_n) -> ()")
_defs.define("residual_norm(Tensor(a!) x, Tensor? a, Tensor? b, Tensor? weight, Tensor(b!)? normed, float eps) -> ()")
_defs.define("gather_tiles(Tensor(a!) dst, Tensor src0, Tensor src1, Tensor idx) -> ()")
_defs.define("pack_w4a16_device(Tensor(a!) out, Tensor q, Tensor scales, Tensor zeros, Tensor(b!) bad) -> ()")


def _w4a16_gemv(out, x, packed, k, n, packed_k, packed_n, start_col, epilogue, layout, split_k):
    _check_cuda(out, x, packed)
    if x.dim() not in (1, 2) or out.dim() not in (1, 2) or x.stride(-1) != 1 or out.stride(-1) != 1:
        raise ValueError("w4a16_gemv: x and out must be [M, K] / [M, N] with contiguous rows")
    m = _rows(x)
    if _rows(out) != m:
        raise ValueError("w4a16_gemv: x and out must have the same number of rows")
    if packed.dtype != torch.uint8 or not packed.is_contiguous():
        raise ValueError("w4a16_gemv: packed must be contiguous uint8")
    if packed.numel() != lib().hmb_packed_bytes(packed_k, packed_n):
        raise ValueError(f"w4a16_gemv: packed has {packed.numel()} bytes, not those of [{packed_k}, {packed_n}]")
    ws_bytes = lib().hmb_w4a16_gemv_workspace(m, k, n, epilogue, split_k)
    ws = workspace(x.device, ws_bytes)
    check(lib().hmb_w4a16_gemv(packed.data_ptr(), packed_k, packed_n, x.data_ptr(), _ld(x), _dtype_code(x), out.data_ptr(),
                               _ld(out), _dtype_code(out), m, k, n, start_col, epilogue, layout, split_k, ws.data_ptr(),
                               ws.numel(), _stream(x)), "w4a16_gemv")


def _w4a16_gemm(out, x, packed, k, n, packed_k, packed_n, start_col, epilogue, layout):
    _check_cuda(out, x, packed)
    if x.dim() != 2 or out.dim() != 2 or x.stride(1) != 1 or out.stride(1) != 1:
        raise ValueError("w4a16_gemm: x and out must be [M, K] / [M, N] with contiguous rows")
    m = x.shape[0]
    if out.shape[0] != m:
        raise ValueError("w4a16_gemm: x and out must have the same number of rows")
    if out.dtype != x.dtype and not (out.dtype == torch.float32 and epilogue == _lib.HMB_EPI_STORE):
        raise ValueError("w4a16_gemm: out must have the activation dtype (or fp32 without an epilogue)")
    if packed.dtype != torch.uint8 or not packed.is_contiguous():
        raise ValueError("w4a16_gemm: packed must be contiguous uint8")
    if packed.numel() != lib().hmb_packed_bytes(packed_k, packed_n):
        raise ValueError(f"w4a16_gemm: packed has {packed.numel()} bytes, not those of [{packed_k}, {packed_n}]")
    check(lib().hmb_w4a16_gemm(packed.data_ptr(), packed_k, packed_n, x.data_ptr(), x.stride(0), _dtype_code(x),
                               out.data_ptr(), out.stride(0), _dtype_code(out), m, k, n, start_col, epilogue, layout,
                               _stream(x)), "w4a16_gemm")


def _w4a16_ffn(y, x, gate_up, down, h, n, stored, layout):
    _check_cuda(y, x, gate_up, down)
    if x.dim() != 2 or y.dim() != 2 or x.stride(1) != 1 or y.stride(1) != 1 or x.shape[1] != h or y.shape[1] != h:
        raise ValueError(f"w4a16_ffn: x and y must be [M, {h}] with contiguous rows")
    m = x.shape[0]
    if y.shape[0] != m:
        raise ValueError("w4a16_ffn: x and y must have the same number of rows")
    if y.dtype != x.dtype and y.dtype != torch.float32:
        raise ValueError("w4a16_ffn: y must have the activation dtype, or fp32 for partial sums")
    for name, p, pk, pn in (("gate_up", gate_up, h, 2 * stored), ("down", down, stored, h)):
        if p.dtype != torch.uint8 or not p.is_contiguous():
            raise ValueError(f"w4a16_ffn: {name} must be contiguous uint8")
        if p.numel() != lib().hmb_packed_bytes(pk, pn):
            raise ValueError(f"w4a16_ffn: {name} has {p.numel()} bytes, not those of [{pk}, {pn}]")
    ws_bytes = lib().hmb_w4a16_ffn_workspace(m, h, n)
    ws = workspace(x.device, ws_bytes, "ffn")
    check(lib().hmb_w4a16_ffn(gate_up.data_ptr(), down.data_ptr(), h, n, stored, layout, x.data_ptr(), x.stride(0),
                              _dtype_code(x), y.data_ptr(), y.stride(0), _dtype_code(y), m, ws.data_ptr(), ws.numel(),
                              _stream(x)), "w4a16_ffn")


def gemm_supported(m, k, n, epilogue):
    return bool(lib().hmb_w4a16_gemm_supports(m, k, n, epilogue))


def gemm_plan(m, k, n, epilogue=0, with_workspace=False):
    """How the GEMM schedules an m x k x n problem on the current device (hmb_w4a16_gemm_plan):
    {"kernel": "cta" | "pair", "band_rows": bool, "band": width in blocks, "k_splits", "grid"}, or
    {"kernel": "skinny", "streamk": bool, "k_splits", "grid"} for the swap-AB kernel of 17 to 128 rows."""
    import ctypes
    plan = (ctypes.c_int * 5)()
    check(lib().hmb_w4a16_gemm_plan(m, k, n, epilogue, int(bool(with_workspace)), plan), "w4a16_gemm_plan")
    if plan[0] == 3:
        return {"kernel": "skinny", "streamk": bool(plan[1]), "k_splits": plan[3], "grid": plan[4]}
    return {"kernel": "pair" if plan[0] == 2 else "cta", "band_rows": bool(plan[1]), "band": plan[2],
            "k_splits": plan[3], "grid": plan[4]}


# Rows above which the tensor-core GEMM takes over from the decode GEMV.
GEMV_MAX_ROWS = 16


def w4a16_linear(out, x, packed, k, n, packed_k, packed_n, start_col=0, epilogue=0, layout=1, split_k=0):
    """The product's packed matmul: the decode GEMV for m <= GEMV_MAX_ROWS, the tcgen05 GEMM above it
    when the shape allows, else the GEMV over row chunks."""
    m = x.shape[0] if x.dim() == 2 else 1
    if m > GEMV_MAX_ROWS and gemm_supported(m, k, n, epilogue):
        ops.w4a16_gemm(out, x, packed, k, n, packed_k, packed_n, start_col, epilogue, layout)
    else:
        ops.w4a16_gemv(out, x, packed, k, n, packed_k, packed_n, start_col, epilogue, layout, split_k)


def device_status(device=None):
    """HMB_OK, or HMB_ERR_TIMEOUT if a kernel gave up a bounded wait since the last call (clears it).
    A kernel that gave up may have left split-K counters raised in its workspace, so on a timeout the
    workspaces cached for this device are zero-filled again before any later call uses them."""
    import ctypes
    v = ctypes.c_int(0)
    stream = torch.cuda.current_stream(device)
    check(lib().hmb_device_status(ctypes.addressof(v), stream.cuda_stream), "device_status")
    if v.value == _lib.HMB_ERR_TIMEOUT:
        index = stream.device.index
        with _ws_lock:
            for (dev_index, _, _), buf in _workspaces.items():
                if dev_index == index:
                    buf.zero_()
        torch.cuda.synchronize(stream.device)
    return v.value


def _w4a16_dequant(out, packed, k, n, packed_k, packed_n):
    _check_cuda(out, packed)
    if out.dtype != torch.float32 or out.dim() != 2 or out.stride(1) != 1 or out.shape[0] != k or out.shape[1] != n:
        raise ValueError("w4a16_dequant: out must be fp32 [k, n] with contiguous rows")
    if packed.numel() != lib().hmb_packed_bytes(packed_k, packed_n):
        raise ValueError("w4a16_dequant: packed size does not match")
    check(lib().hmb_w4a16_dequant(packed.data_ptr(), packed_k, packed_n, k, n, out.data_ptr(), out.stride(0), _stream(out)),
          "w4a16_dequant")


def _silu_mul(gate_up, act, layout):
    _check_cuda(gate_up, act)
    if gate_up.dim() != 2 or act.dim() != 2:
        raise ValueError("silu_mul: expected 2-D tensors")
    if gate_up.dtype != torch.bfloat16 or act.dtype != torch.bfloat16:
        raise ValueError("silu_mul: expected bf16")
    rows, n = act.shape
    if gate_up.shape[0] != rows or gate_up.shape[1] != 2 * n:
        raise ValueError("silu_mul: gate_up must be [M, 2n] and act [M, n]")
    if gate_up.stride(1) != 1 or act.stride(1) != 1:
        raise ValueError("silu_mul: last dimension must be contiguous")
    check(lib().hmb_silu_mul(gate_up.data_ptr(), gate_up.stride(0), act.data_ptr(), act.stride(0), rows, n, layout,
                             _stream(act)), "silu_mul")


def _residual_add2(x, y_g, y_n):
    _check_cuda(x, y_g, y_n)
    if x.dim() != 2 or x.dtype != torch.bfloat16:
        raise ValueError("residual_add2: x must be bf16 [M, H]")
    for name, t in (("y_g", y_g), ("y_n", y_n)):
        if t.dim() != 2 or tuple(t.shape) != tuple(x.shape):
            raise ValueError(f"residual_add2: {name} must match x")
        if t.dtype not in (torch.bfloat16, torch.float32):
            raise ValueError(f"residual_add2: {name} must be bf16 or fp32")
        if t.stride(1) != 1:
            raise ValueError(f"residual_add2: {name} needs a contiguous last dim")
    check(lib().hmb_residual_add2(x.data_ptr(), x.stride(0), y_g.data_ptr(), y_g.stride(0), _dtype_code(y_g), y_n.data_ptr(),
                                  y_n.stride(0), _dtype_code(y_n), x.shape[0], x.shape[1], _stream(x)), "residual_add2")


def _residual_norm(x, a, b, weight, normed, eps):
    """x += a + b ((x + a) + b in fp32, one bf16 rounding), then normed = RMSNorm(x) * weight; the
    arguments of heteromega::residual_norm_bf16 (kernels/gpu/include/heteromega/gpu_ffn.hpp:131-138)."""
    _check_cuda(*[t for t in (x, a, b, weight, normed) if t is not None])
    if x.dim() != 2 or x.dtype != torch.bfloat16 or x.stride(1) != 1:
        raise ValueError("residual_norm: x must be bf16 [M, H] with a contiguous last dim")
    if b is not None and a is None:
        raise ValueError("residual_norm: b needs a")
    for name, t in (("a", a), ("b", b), ("normed", normed)):
        if t is not None and (t.dtype != torch.bfloat16 or t.dim() != 2 or tuple(t.shape) != tuple(x.shape) or t.stride(1) != 1):
            raise ValueError(f"residual_norm: {name} must be bf16 shaped like x")
    if weight is not None and (weight.dtype != torch.bfloat16 or weight.numel() != x.shape[1] or not weight.is_contiguous()):
        raise ValueError("residual_norm: weight must be contiguous bf16 [H]")
    check(lib().hmb_residual_norm(x.data_ptr(), x.stride(0), _ptr(a), a.stride(0) if a is not None else 0, _ptr(b),
                                  b.stride(0) if b is not None else 0, _ptr(weight), _ptr(normed),
                                  normed.stride(0) if normed is not None else 0, x.shape[0], x.shape[1], float(eps), _stream(x)),
          "residual_norm")


def _gather_tiles(dst, src0, src1, idx):
    _check_cuda(dst, src0, src1, idx)
    if idx.dtype != torch.int64 or not idx.is_contiguous():
        raise ValueError("gather_tiles: idx must be contiguous int64")
    if dst.numel() != idx.numel() * _lib.TILE_BYTES:
        raise ValueError("gather_tiles: dst must hold one tile per index")
    check(lib().hmb_gather_tiles(src0.data_ptr(), src0.numel() // _lib.TILE_BYTES, src1.data_ptr(), idx.data_ptr(),
                                 idx.numel(), dst.data_ptr(), _stream(dst)), "gather_tiles")


def _pack_w4a16_device(out, q, scales, zeros, bad):
    _check_cuda(out, q, scales, zeros, bad)
    k, n = q.shape
    check(lib().hmb_pack_w4a16_device(q.data_ptr(), scales.data_ptr(), zeros.data_ptr(), k, n, out.data_ptr(),
                                      bad.data_ptr(), _stream(out)), "pack_w4a16_device")


_impls = torch.library.Library("heteromega", "IMPL", "CUDA")
_impls.impl("w4a16_gemv", _w4a16_gemv)
_impls.impl("w4a16_gemm", _w4a16_gemm)
_impls.impl("w4a16_ffn", _w4a16_ffn)
_impls.impl("w4a16_dequant", _w4a16_dequant)
_impls.impl("silu_mul", _silu_mul)
_impls.impl("residual_add2", _residual_add2)
_impls.impl("residual_norm", _residual_norm)
_impls.impl("gather_tiles", _gather_tiles)
_impls.impl("pack_w4a16_device", _pack_w4a16_device)

ops = torch.ops.heteromega
