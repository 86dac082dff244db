"""An FFN stack on one rank: the layers chained through the layer boundary, replayed as CUDA graphs.

The reference's model runs, per layer, the FFN on the normalised residual stream and adds its
output back (src/unified_llm_w4a16_hetero/unified_llm_w4a16.cpp:2852-2865 for the FFN call,
:2533-2540 for the boundary residual_norm_bf16 that adds the partials and normalises the next
layer's input). FfnStack keeps exactly that chain for the FFN layers alone:

    x_0 = RMSNorm(h_0) * g_0
    h_{l+1} = h_l + FFN_l(x_l),   x_{l+1} = RMSNorm(h_{l+1}) * g_{l+1}      (one boundary launch)
    result = h_L

With a TensorParallelFfn the layers are this rank's shards: FFN_l gives this rank's partial and
the boundary sums the partials of all ranks too. On the NVLink communicator one call runs the layer
(hmb_tp_ffn_layer: for prefill the down GEMM stores its partial rows straight into the peers'
receive slots and the boundary kernel sums, normalises and gathers); with NCCL the partial is
all-reduced and hmb_residual_norm follows. On B200 a decode layer takes a few microseconds, so the
stack captures the whole chain for a given M once and replays it.
"""
import torch

from .gpu_ffn import FfnSliceWeights
from .torch_ops import ops


class FfnStack:
    def __init__(self, layers, hidden, device, tp=None, norms=None, eps=1e-5):
        """layers: FfnSliceWeights per layer (all channels), or None with `tp` holding the shards.
        norms: the RMSNorm weight of each layer's input (bf16 [hidden]); ones by default."""
        self.device = torch.device(device)
        self.hidden = hidden
        self.tp = tp
        self.layers = list(tp.layers) if tp is not None else list(layers)
        if norms is None:
            norms = [torch.ones(hidden, dtype=torch.bfloat16, device=self.device)] * len(self.layers)
        if len(norms) != len(self.layers):
            raise ValueError("FfnStack: one norm weight per layer")
        self.norms = [n.to(self.device, torch.bfloat16).contiguous() for n in norms]
        self.eps = float(eps)
        self.chain = False  # tensor parallel: overlap each boundary's gather with the next gate/up GEMM
        self._graphs = {}
        self._copy_streams = None

    def __len__(self):
        return len(self.layers)

    def buffers(self, m):
        """Working buffers of one M: the residual h, the layer output y and the next input x."""
        z = lambda: torch.empty(m, self.hidden, dtype=torch.bfloat16, device=self.device)  # noqa: E731
        return {"h": z(), "y": z(), "x": z()}

    def forward(self, h_in, result, bufs=None):
        """result[M, H] = the stack applied to h_in[M, H] (bf16, on this rank's GPU), enqueued on the
        current stream. h_in is not modified."""
        m = h_in.shape[0]
        b = bufs if bufs is not None else self.buffers(m)
        h, y, x = b["h"], b["y"], b["x"]
        h.copy_(h_in)
        L = len(self.layers)
        fused = self.tp is not None and self.tp.comm is not None and self.tp.world > 1 and self.tp.collective == "hmb"
        if fused:
            x = self.tp.comm.out(m, self.hidden)  # the boundary's output region, the next layer's input
        ops.residual_norm(h, None, None, self.norms[0], x, self.eps)
        for l in range(L):
            last = l == L - 1
            g = None if last else self.norms[l + 1]
            if fused:
                # Chained boundaries: each layer's gather completes under the next layer's gate/up GEMM.
                out = self.tp.layer(l, x, h, g, self.eps, chain_in=self.chain and l > 0, chain_out=self.chain and not last)
            elif self.tp is None:
                w: FfnSliceWeights = self.layers[l]
                ops.w4a16_ffn(y, x, w.gate_up, w.down, w.hidden, w.channels(), w.stored_channels(), int(w.layout))
                ops.residual_norm(h, y, None, g, None if last else x, self.eps)
                out = h if last else x
            else:
                self.tp.local_partial(l, x, y)
                out = self.tp.boundary(y, h, g, self.eps, None if last else x)
            if not last:
                x = out
        if out.data_ptr() != result.data_ptr():
            result.copy_(out)
        return result

    def graph(self, m, slot=0):
        """(graph, h_in, result) for M rows, captured on first use (`slot` > 0: another graph with its
        own buffers). Fill h_in, replay, read result."""
        g = self._graphs.get((m, slot))
        if g is None:
            h_in = torch.zeros(m, self.hidden, dtype=torch.bfloat16, device=self.device)
            result = torch.empty_like(h_in)
            bufs = self.buffers(m)
            s = torch.cuda.Stream(self.device)
            s.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(s):
                self.forward(h_in, result, bufs)  # warm-up outside the capture (workspaces, NCCL)
            torch.cuda.current_stream(self.device).wait_stream(s)
            torch.cuda.synchronize(self.device)
            graph = torch.cuda.CUDAGraph()
            # thread_local: NCCL's watchdog thread keeps querying its events while this thread captures.
            with torch.cuda.graph(graph, capture_error_mode="thread_local"):
                self.forward(h_in, result, bufs)
            g = (graph, h_in, result, bufs)
            self._graphs[(m, slot)] = g
        return g[0], g[1], g[2]

    def forward_host(self, h_host, out_host, chunks=None):
        """The user-facing call with host buffers: h_host [M, H] (pinned bf16) in, out_host out; no
        synchronization, the current stream sees the whole step. The rows are independent through
        the whole stack, so from M = 512 they go in two chunks, each with its own graph and
        buffers: the host-to-device copy of the second chunk and the device-to-host copy of the
        first overlap the compute (copies on two side streams, ordered by events)."""
        M = h_host.shape[0]
        if chunks is None:
            chunks = 2 if M >= 512 else 1
        cur = torch.cuda.current_stream(self.device)
        if chunks == 1:
            graph, h_in, result = self.graph(M)
            h_in.copy_(h_host, non_blocking=True)
            graph.replay()
            out_host.copy_(result, non_blocking=True)
            return out_host
        if self._copy_streams is None:
            self._copy_streams = (torch.cuda.Stream(self.device), torch.cuda.Stream(self.device))
        h2d, d2h = self._copy_streams
        h2d.wait_stream(cur)
        d2h.wait_stream(cur)
        computed, copied_out = [None, None], [None, None]
        for c in range(chunks):
            r0, r1 = c * M // chunks, (c + 1) * M // chunks
            slot = c % 2
            graph, h_in, result = self.graph(r1 - r0, slot)
            if computed[slot] is not None:
                h2d.wait_event(computed[slot])  # the slot's input buffer is free again
            with torch.cuda.stream(h2d):
                h_in.copy_(h_host[r0:r1], non_blocking=True)
            arrived = torch.cuda.Event()
            arrived.record(h2d)
            cur.wait_event(arrived)
            if copied_out[slot] is not None:
                cur.wait_event(copied_out[slot])  # the slot's result has been read out
            graph.replay()
            computed[slot] = torch.cuda.Event()
            computed[slot].record(cur)
            d2h.wait_event(computed[slot])
            with torch.cuda.stream(d2h):
                out_host[r0:r1].copy_(result, non_blocking=True)
            copied_out[slot] = torch.cuda.Event()
            copied_out[slot].record(d2h)
        cur.wait_stream(h2d)
        cur.wait_stream(d2h)
        return out_host

    def kernels_per_step(self):
        """Kernels of this library that one stack pass launches: the first norm, then per layer
        gate/up, down and the boundary."""
        return 1 + 3 * len(self.layers)

    def release(self):
        """Free the captured graphs. With a process group this must precede destroy_process_group: a
        live graph that holds an NCCL call keeps the communicator from shutting down. reset() frees
        the executable graph even where a caller still holds a reference to the CUDAGraph object."""
        for g in self._graphs.values():
            g[0].reset()
        self._graphs.clear()
