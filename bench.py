"""Benchmark of the W4A16 SwiGLU FFN path (BASELINE.json metric: FFN tokens/s, with decode HBM GB/s
and prefill TFLOP/s as the roofline terms), one process per GPU.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload cfgX] [--m M] [--impl hmb|reference]

Workloads (seeded synthetic weights and activations; no dataset exists):
  cfg0  Llama-3.2-1B FFN layer (H 2048, I 8192), decode, M = 1
  cfg1  the same layer, prefill, M in {128, 512, 2048}; default M = 2048
  cfg2  Llama-3.1-8B FFN stack, 32 layers (H 4096, I 14336), M in {1, 8, 32, 4096}
  cfg3  Qwen2.5-14B FFN stack, 48 layers (H 5120, I 13824), M in {1, 4096}
  cfg4  Llama-3-70B FFN stack, 80 layers (H 8192, I 28672), M in {1, 4, 16, 64, 8192};
        default M = 8192                                                      <- default
cfg4 is the default because BASELINE.json reports it at 1/2/4/8 GPUs and its scaling target names
it; the single-layer cfg1 is the per-kernel case (--workload cfg1).
A step is one pass of M tokens through the workload's layers, chained as a model chains them:
h += FFN_l(RMSNorm(h)) per layer, the residual add and the next norm fused into one boundary
launch. With N > 1 the layers are tensor-partitioned across the ranks (gate/up column-, down
row-parallel) and the boundary also sums the rank partials over NVLink: total work is fixed,
"scaling": "strong".

Timing: W untimed warm-up steps, then K steps, each bracketed by CUDA events on the stream that
runs it; a >L2 buffer is written between steps when the workload's weights fit in L2. Barrier +
synchronize on both sides; rank 0 prints the max over ranks.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

CONFIGS = {
    "cfg0": dict(model="llama3.2-1b-ffn", hidden=2048, inter=8192, layers=1, ms=[1], m=1),
    "cfg1": dict(model="llama3.2-1b-ffn", hidden=2048, inter=8192, layers=1, ms=[128, 512, 2048], m=2048),
    "cfg2": dict(model="llama3.1-8b-ffn-stack", hidden=4096, inter=14336, layers=32, ms=[1, 8, 32, 4096], m=1),
    "cfg3": dict(model="qwen2.5-14b-ffn-stack", hidden=5120, inter=13824, layers=48, ms=[1, 4096], m=1),
    "cfg4": dict(model="llama3-70b-ffn-stack", hidden=8192, inter=28672, layers=80, ms=[1, 4, 16, 64, 8192], m=8192),
}
L2_BYTES = 126 * 2**20


class L2Flush:
    """Evicts the previous step's data from L2: writes a buffer of twice the L2 size, then reads it
    back, so the lines left in L2 are clean and the timed kernel pays no write-back traffic.
    A spin kernel of about 100 us goes first, so the host has enqueued the start event and the step
    long before the GPU reaches them: the host's launch time stays out of the timed window."""

    LEAD_CYCLES = 200_000

    def __init__(self, device):
        import torch

        self.buf = torch.empty(2 * L2_BYTES // 4, dtype=torch.float32, device=device)
        self.out = torch.empty((), dtype=torch.float32, device=device)

    def __call__(self):
        import torch

        torch.cuda._sleep(self.LEAD_CYCLES)
        self.buf.fill_(1.0)
        torch.sum(self.buf, dim=0, out=self.out)
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
BYTES_PER_WEIGHT = 4352 / 8192


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="cfg4", choices=sorted(CONFIGS))
    ap.add_argument("--m", "--tokens", dest="m", type=int, default=0,
                    help="tokens per step (default: the workload's); --tokens under torchrun")
    ap.add_argument("--layers", type=int, default=0, help="override the layer count (testing only)")
    ap.add_argument("--impl", default="hmb", choices=["hmb", "reference"])
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--cpu-sample-s", type=float, default=10.0)
    ap.add_argument("--timeline", action="store_true",
                    help="add the kernels of one profiled replay per rank to the line (diagnosis only)")
    ap.add_argument("--micro", default="", choices=["", "small", "small-once"],
                    help="instead of the stack: time the small kernels at 70B sizes (small-once: one launch each)")
    return ap.parse_args()


def workload(args):
    c = dict(CONFIGS[args.workload])
    c["m"] = args.m or c["m"]
    if args.layers:
        c["layers"] = args.layers
    c["name"] = args.workload
    return c


def peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return {k: float(p[k]) for k in ("hbm_gbs", "bf16_tflops", "bf16_tflops_sustained")}, "measured"
    except (OSError, KeyError, ValueError):
        return dict(FALLBACK_PEAKS), "fallback"


def l2_flushed(wl, world):
    """Whether a step's weights (this rank's share) fit in L2, so that L2 is flushed between steps."""
    per_rank = wl["layers"] * 3 * wl["hidden"] * -(-wl["inter"] // world) * BYTES_PER_WEIGHT
    return per_rank < 2 * L2_BYTES


def config_of(wl, world, use_graph):
    """The `config` object of the JSON line, the same for both arms of one workload."""
    return {"workload": f"{wl['name']}: {wl['model']} x{wl['layers']} layers, M={wl['m']}", "hidden": wl["hidden"],
            "intermediate": wl["inter"], "layers": wl["layers"], "m": wl["m"],
            "parallelism": f"tp{world}" if world > 1 else "single",
            "l2": "flushed between steps (2x L2 buffer written, then read)" if l2_flushed(wl, world) else "weights larger than L2",
            "graph": use_graph}


def layer_bytes(h, n, m):
    """Algorithmic HBM bytes of one FFN layer (all of its n channels): packed weights once, x in, y out."""
    return 3 * h * n * BYTES_PER_WEIGHT + 2 * m * h * 2


def layer_flops(h, n, m):
    return 6.0 * m * h * n


# ---- clocks during the timed region (NVML, polled from a thread) ------------------------------------

class ClockSampler:
    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20, "sw_power_cap": 0x4,
               "hw_power_brake_slowdown": 0x80}

    def __init__(self, device, period_s=0.005):
        self.period = period_s
        self.samples, self.reasons = [], set()
        self._stop = threading.Event()
        self.max_mhz = None
        try:
            import pynvml
            import torch

            pynvml.nvmlInit()
            self.nv = pynvml
            # The NVML handle of this CUDA device, matched by UUID (CUDA_VISIBLE_DEVICES remaps indices).
            uuid = str(torch.cuda.get_device_properties(device).uuid)
            self.h = None
            for i in range(pynvml.nvmlDeviceGetCount()):
                h = pynvml.nvmlDeviceGetHandleByIndex(i)
                u = pynvml.nvmlDeviceGetUUID(h)
                u = u.decode() if isinstance(u, bytes) else u
                if u.replace("GPU-", "") == uuid.replace("GPU-", ""):
                    self.h = h
            if self.h is None:
                raise RuntimeError("device not found in NVML")
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:  # no NVML: the line says so
            self.nv = None

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                r = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for name, bit in self.REASONS.items():
                    if r & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self.nv is not None:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self.nv is not None:
            self._t.join()

    def summary(self):
        if self.nv is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml unavailable"], "samples": 0}
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ---- the product arm -----------------------------------------------------------------------------------

def trace(*args):
    """Progress lines on stderr when HMB_BENCH_TRACE=1 (debugging multi-rank runs)."""
    if os.environ.get("HMB_BENCH_TRACE") == "1":
        print(f"[bench rank {os.environ.get('RANK', '0')} {time.time():.3f}]", *args, file=sys.stderr, flush=True)


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def run_hmb(args):
    import datetime

    import torch
    import torch.distributed as dist

    import heteromega_b200 as H
    from heteromega_b200.stack import FfnStack
    from heteromega_b200.tensor_parallel import TensorParallelFfn
    from heteromega_b200.weights import synthetic_packed_device

    world, rank, local = dist_env()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE {world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    wl = workload(args)
    h, inter, L, m = wl["hidden"], wl["inter"], wl["layers"], wl["m"]

    # Weights: layer l drawn on the device from seed 1000 + l; with N > 1 each rank keeps its shard.
    # RMSNorm weights 1 + 0.2 N(0, 1) (seed 2000 + l), as the reference's boundary test draws them.
    tp = TensorParallelFfn(h, inter, rank=rank, world=world) if world > 1 else None
    layers, norms = [], []
    gen = torch.Generator(device=dev)
    raw0 = None  # layer 0 unsliced (rank 0), for the parity check after the timed region
    for l in range(L):
        gen.manual_seed(1000 + l)
        g = synthetic_packed_device(h, inter, dev, gen)
        u = synthetic_packed_device(h, inter, dev, gen)
        d = synthetic_packed_device(inter, h, dev, gen)
        if tp is not None:
            tp.add_layer(g, u, d)
        else:
            layers.append(H.slice_packed_ffn(g, u, d, h, inter, 0, inter, H.GateUpLayout.kInterleaved))
        if l == 0 and rank == 0:
            raw0 = (g, u, d)
        del g, u, d
        gen.manual_seed(2000 + l)
        norms.append((torch.randn(h, device=dev, generator=gen) * 0.2 + 1.0).to(torch.bfloat16))
    torch.cuda.synchronize()
    if tp is not None:
        tp.connect(m, dev)  # the NVLink boundary-sum buffers, before any capture
    trace("weights ready")
    stack = FfnStack(layers, h, dev, tp=tp, norms=norms)

    # The stack's input: the residual stream h_0 ~ N(0, 1) (seed 7), resident in HBM; each layer
    # reads RMSNorm of the running residual.
    gen.manual_seed(7)
    h0 = torch.randn(m, h, device=dev, generator=gen).to(torch.bfloat16)
    flush = L2Flush(dev) if l2_flushed(wl, world) else None

    use_graph = not args.no_graph
    if use_graph:
        graph, g_in, g_out = stack.graph(m)
        trace("graph captured")
        g_in.copy_(h0)
        step = graph.replay
    else:
        result, bufs = torch.empty_like(h0), stack.buffers(m)
        step = lambda: stack.forward(h0, result, bufs)  # noqa: E731
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    for _ in range(args.warmup):
        if flush is not None:
            flush()
        step()
    torch.cuda.synchronize()
    trace("warm-up done")

    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(dev) as clocks:
        for i in range(args.steps):
            if flush is not None:
                flush()
            starts[i].record(stream)
            step()
            ends[i].record(stream)
        torch.cuda.synchronize()
    barrier()
    step_ms_local = sum(s.elapsed_time(e) for s, e in zip(starts, ends)) / args.steps
    step_ms = step_ms_local
    if world > 1:
        t = torch.tensor([step_ms_local], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        step_ms = float(t.item())

    trace("timed steps done", step_ms)
    # Dominant kernel, timed alone: the fused gate/up + SiLU*up kernel of layer 0.
    w0 = stack.layers[0]
    dom = dominant_kernel(stack, w0, h0, flush, stream, m)

    trace("dominant kernel done")
    # End to end through the public API with host buffers (H2D of the step's inputs, D2H of its outputs).
    e2e = end_to_end(stack, h0, m, args, flush, barrier, world, dev)
    trace("e2e done")
    # Parity of the timed code path: layer 0 and its boundary at the full M, sampled rows checked.
    parity = parity_layer0(stack, raw0, h0, wl, tp, dev, rank)
    trace("parity done")

    pk, pk_kind = peaks()
    from heteromega_b200.torch_ops import GEMV_MAX_ROWS

    decode = m <= GEMV_MAX_ROWS
    # The metric's decode term on the same stack and weights: one token per step (prefill lines only).
    decode_rec = None if decode else decode_record(stack, wl, args, barrier, world, dev, stream, pk["hbm_gbs"], pk_kind)
    trace("decode record done")
    if decode:
        achieved = dom["bytes"] / (dom["ms"] * 1e-3) / 1e9
        roof = {"bound": "hbm", "achieved": round(achieved, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                "frac": round(achieved / pk["hbm_gbs"], 4), "traffic": traffic_from_profiles(wl, "gate_up")}
    else:
        achieved = dom["flops"] / (dom["ms"] * 1e-3) / 1e12
        roof = {"bound": "tensor", "achieved": round(achieved, 1), "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                "frac": round(achieved / pk["bf16_tflops"], 4), "traffic": traffic_from_profiles(wl, "gate_up"),
                "frac_of_sustained": round(achieved / pk["bf16_tflops_sustained"], 4)}
    roof["peak_source"] = f"of {pk_kind}"
    roof["kernel"] = dom["name"]
    roof["kernel_ms"] = round(dom["ms"], 5)
    roof["algorithmic_per_launch"] = dom["bytes"] if decode else dom["flops"]

    tokens_per_s = m / (step_ms * 1e-3)
    stack_bytes = L * layer_bytes(h, inter, m)
    stack_flops = L * layer_flops(h, inter, m)
    line = {
        "metric": "ffn_tokens_per_s", "value": round(tokens_per_s, 2), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(step_ms, 5), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded W4A16 group-128 weights, RMSNorm weights 1+0.2N(0,1), N(0,1) bf16 input)",
        "config": config_of(wl, world, use_graph),
        "decode_hbm_gbs" if decode else "prefill_tflops":
            round(stack_bytes / (step_ms * 1e-3) / 1e9, 1) if decode else round(stack_flops / (step_ms * 1e-3) / 1e12, 1),
        "roofline": roof,
        "clocks": clocks.summary(),
        "e2e": e2e,
        "gpu_launches": stack.kernels_per_step() * args.steps,
        "parity": parity,
    }
    if decode_rec is not None:
        line["decode"] = decode_rec
    if args.timeline and use_graph:
        line["timeline"] = kernel_timeline(graph, barrier, world, dev)
    if rank == 0 and world == 1:
        line["cpu_baseline"] = cpu_baseline(wl, m, args.cpu_sample_s)
    torch.cuda.synchronize()
    if use_graph:
        del graph, step
    stack.release()
    if world > 1:
        dist.barrier(device_ids=[local])
        tp.close()  # no rank touches a peer's buffers after the barrier
        dist.barrier(device_ids=[local])
        trace("destroying process group")
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


def parity_layer0(stack, raw0, h0, wl, tp, dev, rank, n_rows=64, eps=1e-5):
    """Layer 0 and its boundary at the benchmark's full M through the same calls the timed step makes
    (the first boundary, then hmb_w4a16_ffn and the boundary on one GPU, or hmb_tp_ffn_layer across the
    ranks), checked on sampled rows (one per 256-row block up to n_rows, both CTA halves) against a torch
    fp32 restatement of the reference's definition: weights dequantised exactly by hmb_w4a16_dequant (bit
    for bit the oracle's (q - z) * s, pinned in tests/), gate and up as fp32 matmuls rounded to bf16,
    SiLU(g) * u rounded once, down as an fp32 matmul; then h + y rounded once and RMSNorm * g. Every rank
    runs the product path; rank 0 compares. Returns the `parity` object of the JSON line."""
    import torch

    from heteromega_b200.torch_ops import ops

    m, h, inter, L = h0.shape[0], wl["hidden"], wl["inter"], wl["layers"]
    g0, g1 = stack.norms[0], (stack.norms[1] if L > 1 else None)
    hh = h0.clone()
    if tp is not None and tp.comm is not None:
        x = tp.comm.out(m, h)
        ops.residual_norm(hh, None, None, g0, x, eps)
        x0 = x.clone()
        x1 = tp.layer(0, x, hh, g1, eps)
        kept = tp.comm.rows(m, h)
        y = None
    else:
        x0 = torch.empty_like(hh)
        ops.residual_norm(hh, None, None, g0, x0, eps)
        w = stack.layers[0]
        y = torch.empty_like(hh)
        ops.w4a16_ffn(y, x0, w.gate_up, w.down, w.hidden, w.channels(), w.stored_channels(), int(w.layout))
        x1 = torch.empty_like(hh)
        ops.residual_norm(hh, y, None, g1, x1 if g1 is not None else None, eps)
        if g1 is None:
            x1 = hh
        kept = (0, m)
    torch.cuda.synchronize(dev)
    if rank != 0:
        return None
    blocks = (m + 255) // 256
    step = max(1, blocks // n_rows)
    rows = sorted({min(m - 1, 256 * b + (128 if (b // step) % 2 else 0) + (37 * b) % 128) for b in range(0, blocks, step)}
                  | {0, m - 1})
    rows = torch.tensor(rows, device=dev)
    prev_tf32 = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        def deq(p, k, n):
            out = torch.empty(k, n, dtype=torch.float32, device=dev)
            ops.w4a16_dequant(out, p, k, n, k, n)
            return out

        gate_w, up_w, down_w = raw0
        xr = x0[rows].float()
        gate = (xr @ deq(gate_w, h, inter)).to(torch.bfloat16).float()
        up = (xr @ deq(up_w, h, inter)).to(torch.bfloat16).float()
        act = (gate / (1.0 + torch.exp(-gate)) * up).to(torch.bfloat16).float()
        y_ref = act @ deq(down_w, inter, h)
        h1_ref = (h0[rows].float() + y_ref.to(torch.bfloat16).float()).to(torch.bfloat16).float()
        if g1 is not None:
            x1_ref = (h1_ref * torch.rsqrt((h1_ref * h1_ref).mean(-1, keepdim=True) + eps) * g1.float()).to(torch.bfloat16)
        else:
            x1_ref = h1_ref.to(torch.bfloat16)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev_tf32

    def metrics(got, ref):
        got, ref = got.double(), ref.double()
        d = got - ref
        return {"max_rel": float(d.abs().max() / ref.abs().max()), "rel_l2": float(d.norm() / ref.norm()),
                "cos": float((got * ref).sum() / (got.norm() * ref.norm()))}

    out = {"what": "layer 0 + boundary at full M vs torch fp32 dequant-then-matmul on sampled rows",
           "rows": int(rows.numel()), "tolerance": {"max_rel": 1e-2, "rel_l2": 1e-2, "cos": 0.9999}}
    out["next_input"] = metrics(x1[rows].float(), x1_ref.float())
    own = rows[(rows >= kept[0]) & (rows < kept[1])]
    if own.numel():
        sel = torch.isin(rows, own)
        out["residual"] = metrics(hh[own].float(), h1_ref[sel])
    if y is not None:
        out["ffn"] = metrics(y[rows].float(), y_ref)
    checks = [v for k, v in out.items() if k in ("next_input", "residual", "ffn")]
    out["max_rel"] = max(c["max_rel"] for c in checks)
    out["pass"] = all(c["max_rel"] <= 1e-2 and c["rel_l2"] <= 1e-2 and c["cos"] >= 0.9999 for c in checks)
    return out


def dominant_kernel(stack, w, x, flush, stream, m, reps=20):
    import torch

    from heteromega_b200 import _lib
    from heteromega_b200.torch_ops import w4a16_linear

    n, stored, h = w.channels(), w.stored_channels(), w.hidden
    act = torch.empty(m, n, dtype=torch.bfloat16, device=x.device)

    def launch():
        w4a16_linear(act, x, w.gate_up, h, 2 * n, h, 2 * stored, 0, _lib.HMB_EPI_SWIGLU, int(w.layout))

    launch()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, capture_error_mode="thread_local"):
        launch()
    big = flush if flush is not None else L2Flush(x.device)
    times = []
    for _ in range(reps):
        big()  # evicts the weights from L2 and keeps the GPU busy while the graph is enqueued
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        g.replay()
        e.record(stream)
        torch.cuda.synchronize()
        times.append(s.elapsed_time(e))
    ms = statistics.median(times)
    from heteromega_b200.torch_ops import GEMV_MAX_ROWS

    name = ("gemv_kernel<swiglu> (gate/up + SiLU*up)" if m <= GEMV_MAX_ROWS else
            "gemm_pair_kernel<swiglu> (CTA-pair tcgen05 gate/up + SiLU*up)" if m > 128 else
            "tcgen05 gate/up + SiLU*up (gemm_kernel or gemm_pair_kernel by shape)")
    return {"name": name,
            "ms": ms,
            "bytes": h * 2 * n * BYTES_PER_WEIGHT + m * h * 2 + m * n * 2, "flops": 2.0 * m * h * 2 * n}


def end_to_end(stack, h0, m, args, flush, barrier, world, dev):
    import torch
    import torch.distributed as dist

    x_host = h0.cpu().pin_memory()
    y_host = torch.empty_like(x_host).pin_memory()
    stream = torch.cuda.current_stream(dev)
    for _ in range(args.warmup):
        stack.forward_host(x_host, y_host)
    torch.cuda.synchronize()
    barrier()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    for i in range(args.steps):
        if flush is not None:
            flush()
        starts[i].record(stream)
        stack.forward_host(x_host, y_host)
        ends[i].record(stream)
    torch.cuda.synchronize()
    barrier()
    ms = sum(s.elapsed_time(e) for s, e in zip(starts, ends)) / args.steps
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    nbytes = x_host.numel() * x_host.element_size()
    return {"value": round(m / (ms * 1e-3), 2), "unit": "tokens/s", "h2d_bytes_per_step": nbytes,
            "d2h_bytes_per_step": nbytes, "ms_per_step": round(ms, 5), "api": "FfnStack.forward_host"}


def kernel_timeline(graph, barrier, world, dev):
    """Diagnosis, not a measurement of the line: the kernels of one replay of the step's graph as
    CUPTI records them under torch.profiler (name, start and duration in microseconds from the
    replay's first kernel), on every rank; rank 0 gets all ranks' lists."""
    import torch
    import torch.distributed as dist
    from torch.profiler import ProfilerActivity, profile

    barrier()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        graph.replay()
        torch.cuda.synchronize()
    evs = sorted((ev.time_range.start, ev.time_range.end - ev.time_range.start,
                  ev.name.replace("(anonymous namespace)::", "").split("(")[0][:80])
                 for ev in prof.events() if ev.device_type == torch.autograd.DeviceType.CUDA)
    t0 = evs[0][0] if evs else 0
    mine = [(n, round(st - t0, 1), round(d, 1)) for st, d, n in evs]
    barrier()
    if world == 1:
        return {"note": "profiled replay, diagnosis only", "ranks": [mine]}
    every = [None] * world
    dist.all_gather_object(every, mine)
    return {"note": "profiled replay, diagnosis only", "ranks": every}


def decode_record(stack, wl, args, barrier, world, dev, stream, hbm_gbs, peak_kind):
    """Decode on the benchmark's stack: M = 1 through every layer (the same weights, norms and, with
    N > 1, the same communicator), replayed as its own CUDA graph; max(3, W) warm-up steps, then K
    timed steps with CUDA events, max over ranks. The weights exceed L2, so no flush is needed. GB/s
    counts each layer's packed bytes (scales and zeros included) once per step, against the measured
    copy bandwidth."""
    import torch
    import torch.distributed as dist

    L, h, inter = wl["layers"], wl["hidden"], wl["inter"]
    graph, g_in, _ = stack.graph(1, slot=1)
    gen = torch.Generator(device=dev)
    gen.manual_seed(8)
    g_in.copy_(torch.randn(1, h, device=dev, generator=gen).to(torch.bfloat16))
    for _ in range(max(3, args.warmup)):
        graph.replay()
    torch.cuda.synchronize()
    barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(args.steps):
        graph.replay()
    end.record(stream)
    torch.cuda.synchronize()
    barrier()
    ms = start.elapsed_time(end) / args.steps
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    gbs = L * layer_bytes(h, inter, 1) / world / (ms * 1e-3) / 1e9
    return {"m": 1, "steps": args.steps, "ms_per_step": round(ms, 5), "us_per_layer": round(ms * 1e3 / L, 2),
            "tokens_per_s": round(1.0 / (ms * 1e-3), 2), "hbm_gbs_per_gpu": round(gbs, 1),
            "frac": round(gbs / hbm_gbs, 4), "peak": hbm_gbs, "peak_source": f"of {peak_kind}"}


def traffic_from_profiles(wl, kernel):
    """DRAM bytes per launch of the dominant kernel from a committed ncu summary, if one exists."""
    path = os.path.join(REPO, "profiles", "traffic.json")
    try:
        with open(path) as f:
            t = json.load(f)
        return t[f"{wl['name']}_m{wl['m']}"][kernel]
    except (OSError, KeyError, ValueError):
        return None


# ---- CPU: the reference's own AVX kernel (oracle/_ref), or the oracle port ------------------------------

def physical_cores():
    """Physical cores this process may run on (the reference's AVX kernel gains nothing from SMT)."""
    avail = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    try:
        import psutil

        phys = psutil.cpu_count(logical=False) or avail
    except Exception:
        phys = avail
    return max(1, min(phys, avail))


class CpuFfn:
    """The reference model's FFN on the host for `rows` tokens through one layer
    (src/unified_llm_w4a16_hetero/unified_llm_w4a16.cpp:2872-2887): the gate and up projections as two
    packed [H, I] matrices, each through the reference's own CPU AVX GEMV
    (w4a16_gemv_cpu_fused_packed, src/cpu_avx_kernels/w4a16_gemv_avx_packed.cpp, built unchanged into
    oracle/_ref), then torch's CPU bf16 silu_ and mul_ as the model runs them, then down [I, H] through
    the AVX GEMV, one token at a time (the reference has no CPU GEMM). Without oracle/_ref the C port
    of the same GEMV (oracle/w4a16_oracle.c) stands in and `kind` says "port". Seeded synthetic weights
    with the benchmark's distribution."""

    def __init__(self, wl, rows):
        import numpy as np

        from oracle import oracle as O

        self.O, self.h, self.n, self.rows = O, wl["hidden"], wl["inter"], rows
        rng = np.random.default_rng(1000)

        def packed(k, n):
            p = rng.integers(0, 256, (k // 128) * (n // 64) * 4352, dtype=np.uint8)
            t = p.reshape(-1, 4352)
            t[:, 4096:4224] = O.bf16_bits(rng.uniform(0.002, 0.02, (t.shape[0], 64))).view(np.uint8).reshape(-1, 128)
            z = rng.integers(0, 16, (t.shape[0], 8, 8), dtype=np.uint8)
            t[:, 4224:] = np.concatenate([z, z], 2).reshape(-1, 128)
            return p

        self.gate, self.up, self.down = packed(self.h, self.n), packed(self.h, self.n), packed(self.n, self.h)
        self.x = O.bf16_bits(np.random.default_rng(7).standard_normal((rows, self.h)))
        self.avx = O.ReferenceAVX() if O.ReferenceAVX.available() else None
        if self.avx is not None:
            self.kind = "reference"
            self.what = ("w4a16_gemv_cpu_fused_packed (src/cpu_avx_kernels/w4a16_gemv_avx_packed.cpp, built unchanged, "
                         + ("AVX512-BF16" if self.avx.avx512 else "scalar branch: host lacks AVX512-BF16")
                         + ") for gate, up and down; torch CPU bf16 silu_/mul_")
        else:
            self.kind = "port"
            self.what = "C port of the reference GEMV (oracle/w4a16_oracle.c) for gate, up and down; torch CPU bf16 silu_/mul_"

    def _gemv(self, x, packed, k, n, threads):
        if self.avx is not None:
            return self.avx.gemv(x, packed, k, n, threads)
        return self.O.gemv(packed, k, n, x[None, :])[1][0]

    def run(self, threads, rows=None):
        import numpy as np
        import torch

        torch.set_num_threads(threads)
        for r in range(self.rows if rows is None else rows):
            g = self._gemv(self.x[r], self.gate, self.h, self.n, threads)
            u = self._gemv(self.x[r], self.up, self.h, self.n, threads)
            gt = torch.from_numpy(g.view(np.int16)).view(torch.bfloat16)
            torch.nn.functional.silu(gt, inplace=True)  # torch::silu_(gate_buf)
            gt.mul_(torch.from_numpy(u.view(np.int16)).view(torch.bfloat16))  # gate_buf.mul_(up_buf)
            self._gemv(gt.view(torch.int16).numpy().view(np.uint16), self.down, self.n, self.h, threads)


def time_cpu(run, reps, warmup=1):
    for _ in range(warmup):
        run()
    times = []
    for _ in range(reps):
        t0 = time.perf_counter()
        run()
        times.append(time.perf_counter() - t0)
    return statistics.median(times)


def cpu_single_thread(ffn, wl, budget_s=3.0):
    """One token through one layer on one core, repeated within a small budget."""
    one = time_cpu(lambda: ffn.run(1, rows=1), reps=1, warmup=0)
    reps = max(1, min(5, int(budget_s / max(one, 1e-6))))
    t = time_cpu(lambda: ffn.run(1, rows=1), reps=reps, warmup=0)
    return {"value": round(1.0 / (t * wl["layers"]), 4), "unit": "tokens/s", "cores": 1,
            "sample": f"{reps} x 1 token through one layer (median {t * 1e3:.1f} ms), scaled to {wl['layers']} layer(s)"}


def cpu_baseline(wl, m, budget_s):
    """Rank-0 CPU baseline inside the product arm, on a bounded sample: up to 16 tokens through one
    layer on all physical cores (and one token on one core), scaled to the workload's tokens/s."""
    rows = min(m, 16)
    ffn = CpuFfn(wl, rows)
    threads = physical_cores()
    one = time_cpu(lambda: ffn.run(threads), reps=1)
    reps = max(3, min(50, int(budget_s / max(one, 1e-6))))
    t = time_cpu(lambda: ffn.run(threads), reps=reps, warmup=0)
    return {"value": round(rows / (t * wl["layers"]), 4), "unit": "tokens/s", "cores": threads, "kind": ffn.kind,
            "extrapolated": True,
            "sample": f"{reps} x {rows} token(s) through one {wl['hidden']}x{wl['inter']} layer (median {t * 1e3:.1f} ms), "
                      f"scaled to {wl['layers']} layer(s) and M={m}; {ffn.what}; {threads} physical cores of {cpu_model()}",
            "threads_1": cpu_single_thread(ffn, wl)}


def cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown CPU"


def run_reference(args):
    """The reference arm: the reference's CPU implementation of the path (CpuFfn), timed on the host's
    physical cores on this arm's workload, metric and config. Rank 0 only; other ranks exit without
    work. Each step runs a measured sample, min(M, 128) tokens through one layer (the reference has no
    CPU GEMM: prefill is M GEMVs per projection), and the tokens/s of the whole workload is
    extrapolated from it (per token, a stack of L layers takes L times one layer); the line says so
    and reports the sample's own time as ms_per_step."""
    world, rank, _ = dist_env()
    if rank != 0:
        return
    wl = workload(args)
    m = wl["m"]
    rows = min(m, 128)
    ffn = CpuFfn(wl, rows)
    threads = physical_cores()
    for _ in range(args.warmup):
        ffn.run(threads)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        ffn.run(threads)
        times.append(time.perf_counter() - t0)
    sample_s = statistics.median(times)
    value = rows / (sample_s * wl["layers"])
    single = cpu_single_thread(ffn, wl)
    line = {
        "metric": "ffn_tokens_per_s", "value": round(value, 4), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(sample_s * 1e3, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded W4A16 group-128 weights, N(0,1) bf16 input)", "impl": "reference",
        "config": config_of(wl, world, not args.no_graph),
        "extrapolated": True,
        "sample": {"tokens": rows, "layers": 1, "ms_per_step_measured": round(sample_s * 1e3, 3),
                   "ms_per_full_step_extrapolated": round(m / value * 1e3, 1),
                   "note": f"each step times {rows} token(s) through one layer; value scales that to M={m} x "
                           f"{wl['layers']} layer(s) per step"},
        "cpu_baseline": {"value": round(value, 4), "unit": "tokens/s", "cores": threads, "kind": ffn.kind,
                         "extrapolated": True,
                         "sample": f"each step: {rows} token(s) through one layer, scaled to M={m} x {wl['layers']} "
                                   f"layer(s); {ffn.what}; {threads} physical cores of {cpu_model()}",
                         "threads_1": single},
        "e2e": {"value": round(value, 4), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_small(once):
    """The small kernels at Llama-3-70B sizes on cuda:0, inputs above L2: SiLU*up of [4096, 2 x 28672],
    the boundary sums of [4096, 8192] (residual_add2, residual_norm), and the packed-matrix kernels on
    K = 4096 x N = 28672 (dequant to fp32, a full reversed tile gather, the device packer). Each is timed
    with CUDA events over 5 launches after one warm-up; prints one JSON line of microseconds and
    algorithmic GB/s per kernel. `once`: one launch each and no timing (for a profiler's launch list)."""
    import torch

    from heteromega_b200 import _lib
    from heteromega_b200.torch_ops import ops

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev)
    g.manual_seed(5)
    m, h, inter, k, n = 4096, 8192, 28672, 4096, 28672
    res = {}

    def timed(name, fn, nbytes, reps=5):
        fn()
        torch.cuda.synchronize()
        if once:
            return
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(reps):
            fn()
        e.record()
        torch.cuda.synchronize()
        t = s.elapsed_time(e) / reps
        res[name] = {"us": round(t * 1000, 1), "gbs": round(nbytes / t / 1e6, 1), "bytes": nbytes}

    gu = torch.randn(m, 2 * inter, device=dev, generator=g).to(torch.bfloat16)
    act = torch.empty(m, inter, dtype=torch.bfloat16, device=dev)
    timed("silu_mul", lambda: ops.silu_mul(gu, act, _lib.HMB_GATE_UP_INTERLEAVED), (gu.numel() + act.numel()) * 2)
    del gu, act
    x, a, b = (torch.randn(m, h, device=dev, generator=g).to(torch.bfloat16) for _ in range(3))
    w = torch.ones(h, dtype=torch.bfloat16, device=dev)
    normed = torch.empty_like(x)
    timed("residual_add2", lambda: ops.residual_add2(x, a, b), 4 * x.numel() * 2)
    timed("residual_norm", lambda: ops.residual_norm(x, a, b, w, normed, 1e-5), 5 * x.numel() * 2)
    del x, a, b, normed
    tiles = (k // 128) * (n // 64)
    packed = torch.randint(0, 256, (tiles * 4352,), dtype=torch.uint8, device=dev, generator=g)
    out = torch.empty(k, n, dtype=torch.float32, device=dev)
    timed("w4a16_dequant", lambda: ops.w4a16_dequant(out, packed, k, n, k, n), packed.numel() + out.numel() * 4)
    del out
    idx = torch.arange(tiles - 1, -1, -1, dtype=torch.int64, device=dev)
    dst = torch.empty_like(packed)
    timed("gather_tiles", lambda: ops.gather_tiles(dst, packed, packed, idx), 2 * packed.numel())
    del dst
    q = torch.randint(0, 16, (k, n), dtype=torch.uint8, device=dev, generator=g)
    sc = torch.rand(k // 128, n, device=dev, generator=g).to(torch.bfloat16).view(torch.int16)
    zr = torch.randint(0, 16, (k // 128, n), dtype=torch.uint8, device=dev, generator=g)
    bad = torch.zeros(1, dtype=torch.int32, device=dev)
    timed("pack_w4a16_device", lambda: ops.pack_w4a16_device(packed, q, sc, zr, bad),
          q.numel() + sc.numel() * 2 + zr.numel() + packed.numel())
    print(json.dumps({"micro": "small", "once": once, "kernels": res}), flush=True)


def main():
    args = parse()
    if args.micro:
        run_small(args.micro == "small-once")
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_hmb(args)


if __name__ == "__main__":
    main()
