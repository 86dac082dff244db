"""An FFN stack on one rank, replayed as CUDA graphs.

The reference's model loop calls the GPU FFN once per layer (unified_llm_w4a16.cpp:2852-2865,
GpuFfnModel::forward). On B200 a decode layer takes a few microseconds, so the per-layer host
launches would dominate; FfnStack captures the whole layer sequence for a given M once and
replays it. Layer l reads x[l] and writes y[l] ([L, M, H] bf16 buffers that the graph owns).
With a TensorParallelFfn the layers are this rank's shards and each layer ends with the
boundary all-reduce (the NVLink peer-memory kernel, captured in the same graph).
"""
import torch

from . import _lib
from .gpu_ffn import FfnSliceWeights, gpu_ffn_slice_forward
from .torch_ops import ops


class FfnStack:
    def __init__(self, layers, hidden, device, tp=None):
        """layers: FfnSliceWeights per layer (all channels), or None with `tp` holding the shards."""
        self.device = torch.device(device)
        self.hidden = hidden
        self.tp = tp
        self.layers = list(tp.layers) if tp is not None else list(layers)
        self._graphs = {}

    def __len__(self):
        return len(self.layers)

    def _forward_layer(self, l, x, y, act, partial):
        if self.tp is None:
            w: FfnSliceWeights = self.layers[l]
            gpu_ffn_slice_forward(w, x, _Act(act), y)
        else:
            # this rank's partial straight into y, then summed over the ranks in place
            self.tp.local_partial(l, x, y)
            self.tp.reduce_partials(y)

    def forward(self, x_all, y_all, scratch=None):
        """Eager: y_all[l] = FFN_l(x_all[l]) for every layer, on the current stream."""
        m = x_all.shape[1]
        act, partial = scratch if scratch is not None else self._scratch(m)
        for l in range(len(self.layers)):
            self._forward_layer(l, x_all[l], y_all[l], act, partial)
        return y_all

    def _scratch(self, m):
        n = max(w.channels() for w in self.layers)
        act = torch.empty(m, n, dtype=torch.bfloat16, device=self.device)
        return act, None

    def graph(self, m):
        """(graph, x_all, y_all) for M rows, captured on first use. Fill x_all, replay, read y_all."""
        g = self._graphs.get(m)
        if g is None:
            L = len(self.layers)
            x_all = torch.zeros(L, m, self.hidden, dtype=torch.bfloat16, device=self.device)
            y_all = torch.empty_like(x_all)
            scratch = self._scratch(m)
            s = torch.cuda.Stream(self.device)
            s.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(s):
                self.forward(x_all, y_all, scratch)  # warm-up outside the capture (workspaces, NCCL)
            torch.cuda.current_stream(self.device).wait_stream(s)
            torch.cuda.synchronize(self.device)
            graph = torch.cuda.CUDAGraph()
            # thread_local: NCCL's watchdog thread keeps querying its events while this thread captures.
            with torch.cuda.graph(graph, capture_error_mode="thread_local"):
                self.forward(x_all, y_all, scratch)
            g = (graph, x_all, y_all, scratch)
            self._graphs[m] = g
        return g[0], g[1], g[2]

    def forward_host(self, x_host, y_host):
        """The user-facing call with host buffers: copies x_host [L, M, H] (pinned bf16) in, replays
        the stack, copies y_host out, all on the current stream (no synchronization)."""
        graph, x_all, y_all = self.graph(x_host.shape[1])
        x_all.copy_(x_host, non_blocking=True)
        graph.replay()
        y_host.copy_(y_all, non_blocking=True)
        return y_host

    def kernels_per_step(self):
        """Kernels of this library that one stack pass launches (gate/up + down per layer)."""
        return 2 * len(self.layers)

    def release(self):
        """Free the captured graphs. With a process group this must precede destroy_process_group: a
        live graph that holds an NCCL call keeps the communicator from shutting down. reset() frees
        the executable graph even where a caller still holds a reference to the CUDAGraph object."""
        for g in self._graphs.values():
            g[0].reset()
        self._graphs.clear()


class _Act:
    """GpuFfnBuffers-like holder for a preallocated act buffer."""

    def __init__(self, act):
        self.act = act
