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
        self._copy_streams = None

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

    def graph(self, m, slot=0):
        """(graph, x_all, y_all) for M rows, captured on first use (`slot` > 0: another graph with its
        own buffers). Fill x_all, replay, read y_all."""
        g = self._graphs.get((m, slot))
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
            self._graphs[(m, slot)] = g
        return g[0], g[1], g[2]

    def forward_host(self, x_host, y_host, chunks=None):
        """The user-facing call with host buffers: x_host [L, M, H] (pinned bf16) in, y_host out; no
        synchronization, the current stream sees the whole step. From M = 512 the rows go in two
        chunks, each with its own graph and buffers, so the host-to-device copy of the second chunk
        and the device-to-host copy of the first overlap the compute (copies on two side streams,
        ordered by events)."""
        L, M, _ = x_host.shape
        if chunks is None:
            chunks = 2 if M >= 512 else 1
        cur = torch.cuda.current_stream(self.device)
        if chunks == 1:
            graph, x_all, y_all = self.graph(M)
            x_all.copy_(x_host, non_blocking=True)
            graph.replay()
            y_host.copy_(y_all, non_blocking=True)
            return y_host
        if self._copy_streams is None:
            self._copy_streams = (torch.cuda.Stream(self.device), torch.cuda.Stream(self.device))
        h2d, d2h = self._copy_streams
        h2d.wait_stream(cur)
        d2h.wait_stream(cur)
        computed, copied_out = [None, None], [None, None]
        for c in range(chunks):
            r0, r1 = c * M // chunks, (c + 1) * M // chunks
            slot = c % 2
            graph, xb, yb = self.graph(r1 - r0, slot)
            if computed[slot] is not None:
                h2d.wait_event(computed[slot])  # the slot's x buffer is free again
            with torch.cuda.stream(h2d):
                for l in range(L):
                    xb[l].copy_(x_host[l, r0:r1], non_blocking=True)
            arrived = torch.cuda.Event()
            arrived.record(h2d)
            cur.wait_event(arrived)
            if copied_out[slot] is not None:
                cur.wait_event(copied_out[slot])  # the slot's y buffer has been read out
            graph.replay()
            computed[slot] = torch.cuda.Event()
            computed[slot].record(cur)
            d2h.wait_event(computed[slot])
            with torch.cuda.stream(d2h):
                for l in range(L):
                    y_host[l, r0:r1].copy_(yb[l], non_blocking=True)
            copied_out[slot] = torch.cuda.Event()
            copied_out[slot].record(d2h)
        cur.wait_stream(h2d)
        cur.wait_stream(d2h)
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
