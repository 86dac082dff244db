"""Persistent tensor partition of FFN layers across the ranks of a process group.

HeteroMega keeps a persistent intermediate-channel split of every FFN layer between an NPU
and a GPU and sums the two partial outputs at the layer boundary
(src/unified_llm_w4a16_hetero/merged_ffn.cpp:235-236, 417; kernels/gpu/src/residual_add.cu).
On B200 the devices are P GPUs, one process each: rank r owns channels [b_r, e_r) of every
layer (partition.plan_shards), gate/up column-parallel (an interleaved gate_up slice) and down
row-parallel. Each rank computes its partial output (bf16, as the reference's GPU partial is) and
one all-reduce (sum) per layer replaces the reference's boundary sum: on GPUs the library's own
NVLink peer-memory kernel (hmb_allreduce_partials: fp32 sums in rank order, one rounding, the same
bits on every rank), NCCL on request, and the process group's all-reduce for CPU tensors (gloo).
"""
import ctypes

import torch
import torch.distributed as dist

from . import _lib
from ._lib import check, lib
from .gpu_ffn import FfnSliceWeights, GateUpLayout, slice_packed_ffn
from .partition import plan_shards
from .torch_ops import ops, workspace


class PeerComm:
    """Symmetric NVLink buffers of one process group: every rank allocates its receive slots and flag
    words, and the CUDA IPC handles are exchanged over the group so that each rank can store into its
    peers' slots. Messages up to max_bytes."""

    def __init__(self, max_bytes, group=None, device=None):
        self.group = group
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.max_bytes = int(max_bytes)
        hb = lib().hmb_comm_handle_bytes()
        handle = (ctypes.c_uint8 * hb)()
        ptr = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            check(lib().hmb_comm_create(self.rank, self.world, self.max_bytes, ctypes.byref(ptr), handle), "hmb_comm_create")
        self._ptr = ptr
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        joined = (ctypes.c_uint8 * (hb * self.world)).from_buffer_copy(b"".join(handles))
        with torch.cuda.device(self.device):
            check(lib().hmb_comm_connect(self._ptr, joined), "hmb_comm_connect")
        dist.barrier(group=group, device_ids=[self.device.index])

    def all_reduce(self, t, spin_limit_ns=0):
        """t (bf16/fp16/fp32, contiguous, on this rank's GPU) = the sum over the ranks, in place."""
        if not t.is_contiguous() or t.device != self.device:
            raise ValueError("PeerComm.all_reduce: t must be contiguous on the communicator's device")
        code = {torch.bfloat16: _lib.HMB_BF16, torch.float16: _lib.HMB_FP16, torch.float32: _lib.HMB_FP32}[t.dtype]
        check(lib().hmb_allreduce_partials(t.data_ptr(), t.numel(), code, self._ptr,
                                           torch.cuda.current_stream(t.device).cuda_stream, spin_limit_ns),
              "hmb_allreduce_partials")
        return t

    def out(self, m, h):
        """bf16 [m, h] view of the output region of boundary() (valid while the communicator lives)."""
        if m * h * 2 > self.max_bytes:
            raise ValueError("PeerComm.out: larger than the communicator's max_bytes")
        ptr, nbytes = ctypes.c_void_p(), ctypes.c_size_t()
        check(lib().hmb_comm_out(self._ptr, ctypes.byref(ptr), ctypes.byref(nbytes)), "hmb_comm_out")
        return torch.as_tensor(_DeviceArray(ptr.value, (m, h), self), device=self.device).view(torch.bfloat16)

    def rows(self, m, h):
        """[begin, end): the rows of an m x h boundary whose residual this rank keeps."""
        b, e = ctypes.c_int64(), ctypes.c_int64()
        check(lib().hmb_comm_rows(self._ptr, m, h, ctypes.byref(b), ctypes.byref(e)), "hmb_comm_rows")
        return b.value, e.value

    def boundary(self, y, x, weight=None, eps=1e-5, spin_limit_ns=0):
        """The layer boundary (hmb_allreduce_residual_norm): x[rows] += the rank sum of y, then
        RMSNorm(x) * weight (x itself without weight) into the output region, whose [m, h] view it
        returns. y: contiguous bf16 or fp32 [m, h] partials, x: contiguous bf16 [m, h], both on this
        rank's GPU; weight bf16 [h] or None."""
        m, h = x.shape
        for name, t, dtypes in (("y", y, (torch.bfloat16, torch.float32)), ("x", x, (torch.bfloat16,))):
            if t.dtype not in dtypes or not t.is_contiguous() or tuple(t.shape) != (m, h) or t.device != self.device:
                raise ValueError(f"PeerComm.boundary: {name} must be contiguous {'/'.join(str(d) for d in dtypes)} [m, h] "
                                 "on the communicator's device")
        if weight is not None and (weight.dtype != torch.bfloat16 or weight.numel() != h or not weight.is_contiguous()):
            raise ValueError("PeerComm.boundary: weight must be contiguous bf16 [h]")
        out = self.out(m, h)
        code = _lib.HMB_FP32 if y.dtype == torch.float32 else _lib.HMB_BF16
        check(lib().hmb_allreduce_residual_norm(y.data_ptr(), code, x.data_ptr(), weight.data_ptr() if weight is not None else None,
                                                m, h, float(eps), self._ptr, torch.cuda.current_stream(self.device).cuda_stream,
                                                spin_limit_ns), "hmb_allreduce_residual_norm")
        return out

    def close(self):
        if self._ptr is not None:
            check(lib().hmb_comm_destroy(self._ptr), "hmb_comm_destroy")
            self._ptr = None


class _DeviceArray:
    """A device buffer of int16 elements described by __cuda_array_interface__, so that torch can
    view memory the library owns. Holds `owner` alive."""

    def __init__(self, ptr, shape, owner):
        self._owner = owner
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": "<i2", "data": (ptr, False), "version": 3,
                                         "strides": None}


class TensorParallelFfn:
    def __init__(self, hidden, inter, group=None, ratios=None, rank=None, world=None, collective="hmb"):
        """collective: "hmb" (NVLink peer-memory kernel for CUDA tensors) or "nccl" (the process
        group's all-reduce); CPU tensors always use the process group."""
        self.group = group
        self.rank = dist.get_rank(group) if rank is None else rank
        self.world = dist.get_world_size(group) if world is None else world
        self.hidden, self.inter = hidden, inter
        self.shares = plan_shards(inter, self.world, ratios)
        self.begin, self.end = self.shares[self.rank]
        self.layers = []
        self._partial = None
        if collective not in ("hmb", "nccl"):
            raise ValueError("collective must be 'hmb' or 'nccl'")
        self.collective = collective
        self.comm = None

    @property
    def channels(self):
        return self.end - self.begin

    def add_layer(self, gate, up, down):
        """Keep this rank's shard of a layer given as whole packed gate [H, I], up [H, I], down [I, H]."""
        self.layers.append(slice_packed_ffn(gate, up, down, self.hidden, self.inter, self.begin, self.end,
                                            GateUpLayout.kInterleaved))

    def add_shard(self, w: FfnSliceWeights):
        """Keep an already sliced shard (its channel range must be this rank's)."""
        if (w.begin, w.end) != (self.begin, self.end) or w.layout != GateUpLayout.kInterleaved:
            raise ValueError("add_shard: shard does not match this rank's interleaved channel range")
        self.layers.append(w)

    def partial_buffer(self, m, device, dtype=torch.float32):
        if (self._partial is None or self._partial.numel() < m * self.hidden or self._partial.device != device
                or self._partial.dtype != dtype):
            self._partial = torch.empty(m * self.hidden, dtype=dtype, device=device)
        return self._partial[:m * self.hidden].view(m, self.hidden)

    def connect(self, max_rows, device):
        """Sets up the NVLink communicator for partials of up to max_rows rows (collective "hmb");
        every rank of the group must call it."""
        if self.world > 1 and self.collective == "hmb" and self.comm is None:
            self.comm = PeerComm(max_rows * self.hidden * 4, self.group, device)
        return self.comm

    def close(self):
        if self.comm is not None:
            self.comm.close()
            self.comm = None

    def local_partial(self, layer, x, partial, act=None):
        """partial[m, H] (bf16/fp16, or fp32 for unrounded sums) = this rank's share of FFN layer
        `layer` for x [m, H]."""
        w = self.layers[layer]
        n, stored, h = w.channels(), w.stored_channels(), w.hidden
        ops.w4a16_ffn(partial, x, w.gate_up, w.down, h, n, stored, int(w.layout))
        return partial

    def reduce_partials(self, partial):
        """Sum of every rank's partial, in place (one all-reduce)."""
        if self.world == 1:
            return partial
        if partial.is_cuda and self.collective == "hmb":
            if self.comm is None or partial.numel() * partial.element_size() > self.comm.max_bytes:
                raise RuntimeError("TensorParallelFfn: call connect(max_rows, device) on every rank first")
            return self.comm.all_reduce(partial)
        dist.all_reduce(partial, op=dist.ReduceOp.SUM, group=self.group)
        return partial

    def boundary(self, partial, h, weight, eps, normed=None):
        """The layer boundary after this rank's partial of a layer: h += the sum of every rank's
        partial, then the next input RMSNorm(h) * weight (h itself for weight None). Returns the
        tensor that holds it: the communicator's output region (collective "hmb"; then only this
        rank's rows of h are kept, see PeerComm.rows), else `normed` (NCCL all-reduce, then
        hmb_residual_norm on every row). partial, h: bf16 [m, H] on this rank's GPU."""
        if partial.is_cuda and self.world > 1 and self.collective == "hmb":
            if self.comm is None:
                raise RuntimeError("TensorParallelFfn: call connect(max_rows, device) on every rank first")
            return self.comm.boundary(partial, h, weight, eps)
        if self.world > 1:
            dist.all_reduce(partial, op=dist.ReduceOp.SUM, group=self.group)
        if weight is None:
            ops.residual_norm(h, partial, None, None, None, eps)
            return h
        ops.residual_norm(h, partial, None, weight, normed, eps)
        return normed

    def layer(self, layer, x, h, weight, eps, spin_limit_ns=0, chain_in=False, chain_out=False):
        """One whole layer with its boundary on the NVLink communicator (hmb_tp_ffn_layer_chained): this
        rank's partial of FFN `layer` for x [m, H], summed over the ranks into h's kept rows, and the
        next input RMSNorm(h) * weight (h itself without weight) in the output region, whose view it
        returns. For m > 16 the down GEMM writes its partial rows straight into the peers' slots.
        chain_out: the boundary leaves the gather to complete under the next call, which must be made
        with chain_in (x = this call's output region) before anything else reads the region; its
        gate/up GEMM then waits per row block for the rows to land (same bits as unchained calls)."""
        if self.comm is None:
            raise RuntimeError("TensorParallelFfn: call connect(max_rows, device) on every rank first")
        w = self.layers[layer]
        m = x.shape[0]
        for name, t in (("x", x), ("h", h)):
            if t.dtype != torch.bfloat16 or not t.is_contiguous() or tuple(t.shape) != (m, self.hidden):
                raise ValueError(f"TensorParallelFfn.layer: {name} must be contiguous bf16 [m, hidden]")
        nbytes = lib().hmb_tp_ffn_layer_workspace(m, w.hidden, w.channels())
        ws = workspace(h.device, nbytes, kind="tp_layer")
        chain = (_lib.HMB_TP_CHAIN_IN if chain_in else 0) | (_lib.HMB_TP_CHAIN_OUT if chain_out else 0)
        check(lib().hmb_tp_ffn_layer_chained(self.comm._ptr, w.gate_up.data_ptr(), w.down.data_ptr(), w.hidden, w.channels(),
                                             w.stored_channels(), int(w.layout), x.data_ptr(), h.data_ptr(),
                                             weight.data_ptr() if weight is not None else None, float(eps), m, ws.data_ptr(),
                                             ws.numel(), torch.cuda.current_stream(h.device).cuda_stream, spin_limit_ns, chain),
              "hmb_tp_ffn_layer_chained")
        return self.comm.out(m, self.hidden)

    def forward(self, layer, x, y):
        """y[m, H] (x's dtype) = the whole FFN layer for x, on every rank: this rank's partial written
        into y and summed in place."""
        self.local_partial(layer, x, y)
        self.reduce_partials(y)
        return y
