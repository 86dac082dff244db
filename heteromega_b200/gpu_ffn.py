"""The GPU FFN slice API of HeteroMega, on B200.

Mirrors ``namespace heteromega`` of kernels/gpu/include/heteromega/gpu_ffn.hpp (same names,
argument meanings and errors: a ValueError where the reference's TORCH_CHECK fails, an
HmbError when a kernel entry point fails). One device owns intermediate channels
[begin, end) of an FFN layer and computes

    Y = (SiLU(X W_gate[:, begin:end]) * (X W_up[:, begin:end])) W_down[begin:end, :]

Differences from the reference, all deliberate:

* The SiLU*up of gate/up is fused into the gate/up kernel's epilogue (the gate and up sums
  are rounded to bf16 first, then SiLU(g)*u in fp32 is rounded once, which is what the
  reference's unfused gate/up -> silu_mul sequence computes). GpuFfnBuffers.gate_up is kept
  for API compatibility and stays unused.
* Inputs need no 128-row padding: the kernels guard M (padded_rows is kept as an API).
* Everything is enqueued on the given (or current) torch CUDA stream; nothing synchronizes.
"""
import dataclasses
import enum
import os
import threading

import numpy as np
import torch

from . import _lib
from ._lib import check, lib
from .torch_ops import ops, w4a16_linear

kTileK = _lib.TILE_K
kTileN = _lib.TILE_N
kTileBytes = _lib.TILE_BYTES


def padded_rows(m):
    """Rows rounded up to a multiple of 128 (gpu_ffn.hpp:24). B200 kernels do not need it."""
    return (m + kTileK - 1) // kTileK * kTileK


class GateUpLayout(enum.IntEnum):
    """Column order of a packed gate_up matrix of n channels (gpu_ffn.hpp:50-54)."""
    kBlocked = _lib.HMB_GATE_UP_BLOCKED  # [gate 0..n) | up 0..n)]
    kInterleaved = _lib.HMB_GATE_UP_INTERLEAVED  # per 64 channels: 64 gate columns, then 64 up columns


class GemvKernel(enum.IntEnum):
    """Kept for API compatibility (gpu_ffn.hpp:185-188): both names select the B200 GEMV."""
    kHeteroMega = 0
    kHeteroMosaic = 1


class GemmKernel(enum.IntEnum):
    """Kept for API compatibility (gpu_ffn.hpp:190-193): both names select the B200 GEMM."""
    kHeteroMosaic = 0
    kHeteroMega = 1


@dataclasses.dataclass
class LinearOptions:
    """Options of packed_linear (gpu_ffn.hpp:198-205)."""
    packed_k: int = 0  # rows of the whole packed matrix; 0 means k
    packed_n: int = 0  # columns of the whole packed matrix; 0 means n
    gemv: GemvKernel = GemvKernel.kHeteroMega
    gemv_split_k: int = 0  # see gemv_w4a16
    fuse_activation: bool = False  # gate/up only: write SiLU(gate)*up [M, n/2]
    gemm: GemmKernel = GemmKernel.kHeteroMosaic
    layout: GateUpLayout = GateUpLayout.kInterleaved  # gate/up column order when fuse_activation


def _stream_ctx(stream):
    return torch.cuda.stream(stream) if stream is not None else _Null()


class _Null:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False


# ---- weight packing ------------------------------------------------------------------------------

def packed_bytes(k, n):
    return (k // kTileK) * (n // kTileN) * kTileBytes


def pack_w4a16(qweight, scales, zeros):
    """Packs a [K, N] W4A16 matrix into the tile layout (gpu_ffn.hpp:28-34).

    qweight [K, N] uint8 (0..15), scales [K/128, N] bfloat16, zeros [K/128, N] int8/uint8 (0..15).
    Returns a flat uint8 tensor on the inputs' device (CPU tensors are packed on the host,
    CUDA tensors by a kernel).
    """
    if qweight.dim() != 2:
        raise ValueError("pack_w4a16: qweight must be [K, N]")
    K, N = qweight.shape
    if K % kTileK or N % kTileN:
        raise ValueError(f"pack_w4a16: K must be a multiple of 128 and N of 64, got {K}x{N}")
    if tuple(scales.shape) != (K // kTileK, N):
        raise ValueError("pack_w4a16: scales must be [K/128, N]")
    if tuple(zeros.shape) != (K // kTileK, N):
        raise ValueError("pack_w4a16: zeros must be [K/128, N]")
    q = qweight.to(torch.uint8).contiguous()
    s = scales.to(torch.bfloat16).contiguous().view(torch.int16)
    z = zeros.to(torch.uint8).contiguous()
    if q.is_cuda:
        out = torch.empty(packed_bytes(K, N), dtype=torch.uint8, device=q.device)
        bad = torch.zeros(1, dtype=torch.int32, device=q.device)
        ops.pack_w4a16_device(out, q, s.to(q.device), z.to(q.device), bad)
        if int(bad.item()) != 0:
            raise ValueError("pack_w4a16: weights and zeros must lie in 0..15")
        return out
    out = torch.empty(packed_bytes(K, N), dtype=torch.uint8)
    rc = lib().hmb_pack_w4a16(q.data_ptr(), s.data_ptr(), z.data_ptr(), K, N, out.data_ptr())
    if rc == -3:
        raise ValueError("pack_w4a16: weights and zeros must lie in 0..15")
    check(rc, "pack_w4a16")
    return out


@dataclasses.dataclass
class FfnLayerQuant:
    """AWQ tensors of one FFN layer in [in_features, out_features] order (gpu_ffn.hpp:37-42)."""
    gate_q: torch.Tensor
    gate_s: torch.Tensor
    gate_z: torch.Tensor
    up_q: torch.Tensor
    up_s: torch.Tensor
    up_z: torch.Tensor
    down_q: torch.Tensor
    down_s: torch.Tensor
    down_z: torch.Tensor


@dataclasses.dataclass
class FfnSliceWeights:
    """One device's packed share of an FFN layer: intermediate channels [begin, end) (gpu_ffn.hpp:56-75)."""
    gate_up: torch.Tensor = None  # packed [H, 2 * stored_channels()], column order `layout`
    down: torch.Tensor = None  # packed [stored_channels(), H]
    begin: int = 0
    end: int = 0
    hidden: int = 0
    layout: GateUpLayout = GateUpLayout.kBlocked
    packed_channels: int = 0  # channels in the packed tensors; 0 means channels()

    def channels(self):
        return self.end - self.begin

    def stored_channels(self):
        return self.packed_channels if self.packed_channels > 0 else self.channels()

    def to(self, device):
        return dataclasses.replace(self, gate_up=self.gate_up.to(device), down=self.down.to(device))

    def prefix(self, n):
        """The same tensors, used for channels [begin, begin + n) only. No copy (gpu_ffn.hpp:70-74)."""
        stored = self.stored_channels()
        if not (0 < n <= stored and n % kTileK == 0):
            raise ValueError(f"FfnSliceWeights::prefix: n must be a multiple of 128 in (0, {stored}], got {n}")
        if n != stored and self.layout != GateUpLayout.kInterleaved:
            raise ValueError("FfnSliceWeights::prefix: a shorter prefix needs GateUpLayout::kInterleaved")
        return dataclasses.replace(self, packed_channels=stored, end=self.begin + n)


def _join_gate_up(g, u, layout):
    if layout == GateUpLayout.kBlocked:
        return torch.cat([g, u], 1)
    r, n = g.shape
    return torch.stack([g.reshape(r, n // kTileN, kTileN), u.reshape(r, n // kTileN, kTileN)], 2).reshape(r, 2 * n)


def pack_ffn_slice(layer, begin, end, layout=GateUpLayout.kBlocked):
    """Packs channels [begin, end), multiples of 128 (gpu_ffn.hpp:77-80; pack_w4a16.cpp:68-98)."""
    if layer.gate_q.dim() != 2:
        raise ValueError("pack_ffn_slice: gate_q must be [H, I]")
    hidden, inter = layer.gate_q.shape
    if not (0 <= begin < end <= inter):
        raise ValueError(f"pack_ffn_slice: bad channel range [{begin}, {end})")
    if begin % kTileK or end % kTileK:
        raise ValueError("pack_ffn_slice: begin and end must be multiples of 128")
    if tuple(layer.down_q.shape) != (inter, hidden):
        raise ValueError("pack_ffn_slice: down_q must be [I, H]")
    cols = lambda t: t[:, begin:end]  # noqa: E731
    rows = lambda t, per: t[begin // per:end // per]  # noqa: E731
    gate_up = pack_w4a16(_join_gate_up(cols(layer.gate_q), cols(layer.up_q), layout),
                         _join_gate_up(cols(layer.gate_s), cols(layer.up_s), layout),
                         _join_gate_up(cols(layer.gate_z), cols(layer.up_z), layout))
    down = pack_w4a16(rows(layer.down_q, 1), rows(layer.down_s, kTileK), rows(layer.down_z, kTileK))
    return FfnSliceWeights(gate_up, down, begin, end, hidden, GateUpLayout(layout))


def packed_tile_index(c, r, tiles_k, tiles_n):
    """Position of tile (column c, row r) in a packed tiles_k x tiles_n matrix (gpu_ffn.hpp:82-83)."""
    v = lib().hmb_packed_tile_index(c, r, tiles_k, tiles_n)
    if v < 0:
        raise ValueError("packed_tile_index: tile outside the matrix")
    return v


def slice_tile_maps(hidden, inter, begin, end, layout):
    """Source tile of each tile of the slice: (gate_up map into [gate | up], down map), int64 numpy."""
    gu_n = np.zeros(1, np.int64)
    dn_n = np.zeros(1, np.int64)
    check(lib().hmb_slice_tile_counts(hidden, inter, begin, end, gu_n.ctypes.data, dn_n.ctypes.data), "slice_tile_counts")
    gu = np.empty(int(gu_n[0]), np.int64)
    dn = np.empty(int(dn_n[0]), np.int64)
    check(lib().hmb_slice_tile_map(hidden, inter, begin, end, int(layout), gu.ctypes.data, dn.ctypes.data), "slice_tile_map")
    return gu, dn


def slice_packed_ffn(gate, up, down, hidden, inter, begin, end, layout=GateUpLayout.kBlocked):
    """pack_ffn_slice from already packed gate [H, I], up [H, I], down [I, H], by whole-tile
    copies on the tensors' device (gpu_ffn.hpp:85-90; pack_w4a16.cpp:109-165). For [0, inter)
    the result's down is `down` itself."""
    if hidden % kTileK or inter % kTileK:
        raise ValueError("slice_packed_ffn: hidden and inter must be multiples of 128")
    if not (0 <= begin < end <= inter):
        raise ValueError(f"slice_packed_ffn: bad channel range [{begin}, {end})")
    if begin % kTileK or end % kTileK:
        raise ValueError("slice_packed_ffn: begin and end must be multiples of 128")
    matrix_tiles = (hidden // kTileK) * (inter // kTileN)
    for t in (gate, up, down):
        if t is None:
            raise ValueError("slice_packed_ffn: a packed matrix is undefined")
        if t.dtype != torch.uint8 or not t.is_contiguous() or t.numel() != matrix_tiles * kTileBytes:
            raise ValueError(f"slice_packed_ffn: expected contiguous uint8 packed matrices of {matrix_tiles * kTileBytes} "
                             f"bytes, got {t.numel()}")
        if t.device != gate.device:
            raise ValueError("slice_packed_ffn: all matrices must be on one device")
    gu_map, dn_map = slice_tile_maps(hidden, inter, begin, end, layout)
    dev = gate.device
    if dev.type == "cuda":
        gate_up = torch.empty(gu_map.size * kTileBytes, dtype=torch.uint8, device=dev)
        ops.gather_tiles(gate_up, gate, up, torch.from_numpy(gu_map).to(dev))
        if begin == 0 and end == inter:
            down_s = down
        else:
            down_s = torch.empty(dn_map.size * kTileBytes, dtype=torch.uint8, device=dev)
            ops.gather_tiles(down_s, down, down, torch.from_numpy(dn_map).to(dev))
    else:
        both = torch.cat([gate.view(-1, kTileBytes), up.view(-1, kTileBytes)])
        gate_up = both.index_select(0, torch.from_numpy(gu_map)).view(-1)
        down_s = down if (begin == 0 and end == inter) else \
            down.view(-1, kTileBytes).index_select(0, torch.from_numpy(dn_map)).view(-1)
    return FfnSliceWeights(gate_up, down_s, begin, end, hidden, GateUpLayout(layout))


# ---- kernels ---------------------------------------------------------------------------------------

def silu_mul(gate_up, act, stream=None, layout=GateUpLayout.kBlocked):
    """act[m, j] = SiLU(gate[m, j]) * up[m, j], bf16 in/out, fp32 math, one rounding (gpu_ffn.hpp:92-93)."""
    with _stream_ctx(stream):
        ops.silu_mul(gate_up, act, int(layout))


def gemv_w4a16(out, x, packed, k, n, packed_k, packed_n, split_k=0, stream=None):
    """out[1, n] = x[1, k] @ W[:k, :n] of a packed [packed_k, packed_n] matrix (gpu_ffn.hpp:95-99).
    split_k = 0 picks a split from the shape."""
    if not (k > 0 and n > 0 and k % kTileK == 0 and n % kTileN == 0):
        raise ValueError("gemv_w4a16: k must be a multiple of 128 and n of 64")
    if not (k <= packed_k and n <= packed_n and packed_k % kTileK == 0 and packed_n % kTileN == 0):
        raise ValueError(f"gemv_w4a16: packed matrix [{packed_k}, {packed_n}] does not contain [{k}, {n}]")
    if x.numel() != k or not x.is_contiguous() or x.dtype != torch.bfloat16:
        raise ValueError(f"gemv_w4a16: x must be contiguous bf16 with {k} elements")
    if out.numel() != n or not out.is_contiguous() or out.dtype != torch.bfloat16:
        raise ValueError(f"gemv_w4a16: out must be contiguous bf16 with {n} elements")
    with _stream_ctx(stream):
        ops.w4a16_gemv(out.view(1, n), x.view(1, k), packed, k, n, packed_k, packed_n, 0, _lib.HMB_EPI_STORE, 0, int(split_k))


def _linear(out, x, packed, k, n, pk, pn, fuse_activation=False, layout=GateUpLayout.kInterleaved, split_k=0):
    epi = _lib.HMB_EPI_SWIGLU if fuse_activation else _lib.HMB_EPI_STORE
    w4a16_linear(out, x, packed, k, n, pk, pn, 0, epi, int(layout), int(split_k))


def gemm_w4a16_supports(m, k, n):
    """Shapes the B200 GEMM path takes: any M > 0, k % 128 == 0, n % 64 == 0 (gpu_ffn.hpp:107)."""
    return m > 0 and k > 0 and n > 0 and k % kTileK == 0 and n % kTileN == 0


def gemm_w4a16(out, x, packed, k, n, packed_k, packed_n, stream=None):
    """out[M, n] = x[M, k] @ W[:k, :n] of a packed [packed_k, packed_n] matrix (gpu_ffn.hpp:101-106)."""
    if not gemm_w4a16_supports(x.shape[0] if x.dim() == 2 else 1, k, n):
        raise ValueError("gemm_w4a16: unsupported shape")
    with _stream_ctx(stream):
        _linear(out, x, packed, k, n, packed_k, packed_n)


def gemm_w4a16_ffn_supports(m, h, n):
    return m > 0 and h % kTileK == 0 and n % kTileK == 0 and n > 0


def gemm_w4a16_ffn(y, x, gate_up, down, h, n, stored, stream=None):
    """The FFN of n channels as one pass: gate_up packed [h, 2*stored] kInterleaved, down packed
    [stored, h] (gpu_ffn.hpp:110-114)."""
    if not gemm_w4a16_ffn_supports(x.shape[0], h, n):
        raise ValueError("gemm_w4a16_ffn: unsupported shape")
    w = FfnSliceWeights(gate_up, down, 0, n, h, GateUpLayout.kInterleaved, stored)
    gpu_ffn_slice_forward(w, x, None, y, stream)


def residual_add2(x, y_g, y_n, stream=None):
    """x += y_g + y_n; partials first, fp32 math, one bf16 rounding (gpu_ffn.hpp:158-159)."""
    with _stream_ctx(stream):
        ops.residual_add2(x, y_g, y_n)


@dataclasses.dataclass
class GpuFfnBuffers:
    """Scratch of gpu_ffn_slice_forward (gpu_ffn.hpp:163-171). Only `act` is used on B200."""
    gate_up: torch.Tensor = None
    act: torch.Tensor = None
    x_pad: torch.Tensor = None

    @staticmethod
    def allocate(max_m, channels, hidden, device):
        opt = dict(dtype=torch.bfloat16, device=device)
        return GpuFfnBuffers(torch.empty(0, **opt), torch.empty(max_m * channels, **opt), torch.empty(0, **opt))


def gpu_ffn_slice_forward(w, x_norm, buf, y, stream=None):
    """GPU share of one FFN sublayer (gpu_ffn.hpp:173-183): enqueues the gate/up + SiLU*up and down
    work on `stream` (hmb_w4a16_ffn); does not synchronize. x_norm and y: bf16 [M, H], contiguous rows
    (y may be fp32 for unrounded partial sums)."""
    n, stored, h = w.channels(), w.stored_channels(), w.hidden
    if n != stored and w.layout != GateUpLayout.kInterleaved:
        raise ValueError("gpu_ffn_slice_forward: a prefix of the packed channels needs GateUpLayout::kInterleaved")
    if x_norm.dim() != 2 or x_norm.shape[1] != h or x_norm.stride(1) != 1:
        raise ValueError("gpu_ffn_slice_forward: x_norm must be contiguous [M, H]")
    m = x_norm.shape[0]
    if tuple(y.shape) != (m, h):
        raise ValueError("gpu_ffn_slice_forward: y must be [M, H]")
    with _stream_ctx(stream):
        # One call: a single fused launch for decode (m <= 16), the two tcgen05 GEMMs for prefill; the
        # intermediate act lives in the library's workspace, so `buf` is not needed.
        ops.w4a16_ffn(y, x_norm, w.gate_up, w.down, h, n, stored, int(w.layout))


def packed_linear(out, inp, packed, k, n, stream=None, opt=None):
    """Packed matmul out[M, n] = in[M, k] @ W[:k, :n] (gpu_ffn.hpp:207-211). With
    opt.fuse_activation, W is gate/up in opt.layout order and out is SiLU(gate)*up [M, n/2]."""
    opt = opt or LinearOptions()
    pk = opt.packed_k if opt.packed_k > 0 else k
    pn = opt.packed_n if opt.packed_n > 0 else n
    if inp.dim() != 2 or inp.shape[1] != k or inp.stride(1) != 1:
        raise ValueError(f"packed_linear: input must be contiguous [M, {k}]")
    m = inp.shape[0]
    if m <= 0:
        raise ValueError("packed_linear: M must be > 0")
    if k % kTileK or n % kTileN:
        raise ValueError("packed_linear: k must be a multiple of 128 and n of 64")
    out_n = n // 2 if opt.fuse_activation else n
    if opt.fuse_activation and n % (2 * kTileN):
        raise ValueError("packed_linear: fused activation needs a gate/up width that is a multiple of 128")
    if out.dim() != 2 or out.shape[0] != m or out.shape[1] != out_n or out.stride(1) != 1:
        raise ValueError(f"packed_linear: output must be contiguous [M, {out_n}]")
    if inp.dtype != torch.bfloat16 or out.dtype != torch.bfloat16:
        raise ValueError("packed_linear: expected bf16")
    if not (k <= pk and n <= pn and pk % kTileK == 0 and pn % kTileN == 0):
        raise ValueError(f"packed_linear: packed matrix [{pk}, {pn}] does not contain [{k}, {n}]")
    if packed.numel() != packed_bytes(pk, pn):
        raise ValueError(f"packed_linear: packed size does not match {pk}x{pn}")
    if packed.device != inp.device or out.device != inp.device:
        raise ValueError("packed_linear: all tensors must be on one device")
    with _stream_ctx(stream):
        _linear(out, inp, packed, k, n, pk, pn, opt.fuse_activation, opt.layout, opt.gemv_split_k)


class GpuFfnModel:
    """The GPU FFN of every layer of a model (gpu_ffn.hpp:213-242). Each layer keeps one packed
    copy of all its channels (gate/up interleaved); a forward pass uses the first s_prefill
    channels when M > 1 and the first s_decode when M == 1, without copies."""

    def __init__(self):
        self._layers = []
        self._s_prefill = 0
        self._s_decode = 0
        self._lock = threading.Lock()
        self._buffers = {}

    def add_layer(self, gate, up, down, hidden, inter):
        if self._layers and (self._layers[0].hidden != hidden or self._layers[0].stored_channels() != inter):
            raise ValueError("GpuFfnModel::add_layer: all layers must have the same shape")
        self._layers.append(slice_packed_ffn(gate, up, down, hidden, inter, 0, inter, GateUpLayout.kInterleaved))
        if self._s_prefill == 0:
            self._s_prefill = self._s_decode = inter

    def set_split(self, s_prefill, s_decode):
        if not self._layers:
            raise ValueError("GpuFfnModel::set_split: add the layers first")
        inter = self._layers[0].stored_channels()
        for s in (s_prefill, s_decode):
            if not (0 < s <= inter and s % kTileK == 0):
                raise ValueError(f"GpuFfnModel::set_split: channels must be a multiple of 128 in (0, {inter}], got {s}")
        self._s_prefill, self._s_decode = s_prefill, s_decode

    def split_from_env(self, environ=None):
        """Applies HETEROMEGA_GPU_FFN_SPLIT="<s_prefill>,<s_decode>" when it is set (the model setup of
        src/unified_llm_w4a16_hetero/unified_llm_w4a16.cpp:2377-2382); returns whether it was."""
        env = os.environ if environ is None else environ
        value = env.get("HETEROMEGA_GPU_FFN_SPLIT")
        if value is None:
            return False
        parts = value.split(",")
        try:
            s_prefill, s_decode = (int(p) for p in parts)
        except ValueError:
            raise ValueError(f"HETEROMEGA_GPU_FFN_SPLIT must be <s_prefill>,<s_decode>, got {value}") from None
        self.set_split(s_prefill, s_decode)
        return True

    def layers(self):
        return len(self._layers)

    def channels(self, m):
        return self._s_prefill if m > 1 else self._s_decode

    def forward(self, layer, x_norm, y, stream=None):
        if not (0 <= layer < self.layers()):
            raise ValueError(f"GpuFfnModel::forward: no layer {layer}")
        full = self._layers[layer]
        m = x_norm.shape[0]
        s = stream if stream is not None else torch.cuda.current_stream(x_norm.device)
        with self._lock:
            key = s.cuda_stream
            b = self._buffers.get(key)
            if b is None or b.act.numel() < m * full.stored_channels():
                b = GpuFfnBuffers.allocate(m, full.stored_channels(), full.hidden, x_norm.device)
                self._buffers[key] = b
        gpu_ffn_slice_forward(full.prefix(self.channels(m)), x_norm, b, y, stream)
