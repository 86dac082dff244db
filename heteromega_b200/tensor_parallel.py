"""Persistent tensor partition of FFN layers across the ranks of a process group.

HeteroMega keeps a persistent intermediate-channel split of every FFN layer between an NPU
and a GPU and sums the two partial outputs at the layer boundary
(src/unified_llm_w4a16_hetero/merged_ffn.cpp:235-236, 417; kernels/gpu/src/residual_add.cu).
On B200 the devices are P GPUs, one process each: rank r owns channels [b_r, e_r) of every
layer (partition.plan_shards), gate/up column-parallel (an interleaved gate_up slice) and down
row-parallel. Each rank computes its partial output in fp32 and one all-reduce (sum) per layer
over NCCL on the compute stream replaces the reference's boundary sum; the fp32 sum is rounded
to bf16 once, as residual_add2 does.
"""
import torch
import torch.distributed as dist

from .gpu_ffn import FfnSliceWeights, GateUpLayout, slice_packed_ffn
from .partition import plan_shards
from .torch_ops import ops


class TensorParallelFfn:
    def __init__(self, hidden, inter, group=None, ratios=None, rank=None, world=None):
        self.group = group
        self.rank = dist.get_rank(group) if rank is None else rank
        self.world = dist.get_world_size(group) if world is None else world
        self.hidden, self.inter = hidden, inter
        self.shares = plan_shards(inter, self.world, ratios)
        self.begin, self.end = self.shares[self.rank]
        self.layers = []
        self._partial = None

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

    def partial_buffer(self, m, device):
        if self._partial is None or self._partial.numel() < m * self.hidden or self._partial.device != device:
            self._partial = torch.empty(m * self.hidden, dtype=torch.float32, device=device)
        return self._partial[:m * self.hidden].view(m, self.hidden)

    def local_partial(self, layer, x, partial, act=None):
        """partial[m, H] (fp32) = this rank's share of FFN layer `layer` for x [m, H] (bf16)."""
        w = self.layers[layer]
        n, stored, h = w.channels(), w.stored_channels(), w.hidden
        ops.w4a16_ffn(partial, x, w.gate_up, w.down, h, n, stored, int(w.layout))
        return partial

    def reduce_partials(self, partial):
        """Sum of every rank's partial, in place (one all-reduce)."""
        if self.world > 1:
            dist.all_reduce(partial, op=dist.ReduceOp.SUM, group=self.group)
        return partial

    def forward(self, layer, x, y):
        """y[m, H] (bf16) = the whole FFN layer for x, on every rank."""
        partial = self.partial_buffer(x.shape[0], x.device)
        self.local_partial(layer, x, partial)
        self.reduce_partials(partial)
        y.copy_(partial)
        return y
