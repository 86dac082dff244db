"""Channel partition of an FFN layer across devices.

HeteroMega splits the intermediate channels of each FFN layer between an NPU and a GPU
(npu/ffn/reference.py:121-151): device d owns a contiguous, 128-aligned channel range, gate and
up are cut by output columns, down by input rows, and the per-device partial outputs are summed
once at the layer boundary. Here the same algebra runs over P B200 ranks.

* FFNPartition restates the reference's two-device split and its ``from_ratio`` rounding
  (nearest multiple of the alignment, ties upward; reference.py:139-147).
* plan_shards generalises it to P ranks: the cumulative share of rank r is rounded the same
  way, so equal shares come out when I/P is aligned and 128-aligned unequal shares otherwise
  (Qwen2.5-14B, I = 13824 over 8 ranks: 4 x 1792 + 4 x 1664).
* predict_layer_time is the per-layer cost form of tools/split_model/split_cost_model.py:8,
  T = max_r(t_r) + tail, with t_r from a roofline of each rank's shard and tail the boundary
  all-reduce; best_ratios scans candidate splits with it.
"""
import dataclasses
import math
from numbers import Integral

ALIGNMENT = 128
BYTES_PER_WEIGHT = 4352 / (128 * 64)  # packed tile bytes per weight: 0.53125


def _positive_int(value, name):
    if isinstance(value, bool) or not isinstance(value, Integral) or value <= 0:
        raise ValueError(f"{name} must be a positive integer")


def round_aligned(value, alignment=ALIGNMENT):
    """Nearest multiple of `alignment`, ties upward."""
    return math.floor(value / alignment + 0.5) * alignment


@dataclasses.dataclass(frozen=True)
class FFNPartition:
    """The reference's two-way split: device "npu" owns [0, npu_channels), "gpu" the rest."""
    intermediate_channels: int
    npu_channels: int
    alignment: int = ALIGNMENT

    def __post_init__(self):
        _positive_int(self.intermediate_channels, "intermediate_channels")
        _positive_int(self.alignment, "alignment")
        if isinstance(self.npu_channels, bool) or not isinstance(self.npu_channels, Integral):
            raise ValueError("npu_channels must be an integer")
        if not 0 <= self.npu_channels <= self.intermediate_channels:
            raise ValueError("npu_channels must lie within the FFN width")
        if self.intermediate_channels % self.alignment or self.npu_channels % self.alignment:
            raise ValueError("FFN width and NPU channel count must satisfy alignment")

    @classmethod
    def from_ratio(cls, intermediate_channels, npu_ratio, alignment=ALIGNMENT):
        _positive_int(intermediate_channels, "intermediate_channels")
        _positive_int(alignment, "alignment")
        if not math.isfinite(npu_ratio) or not 0 <= npu_ratio <= 1:
            raise ValueError("npu_ratio must be finite and in [0, 1]")
        return cls(intermediate_channels, round_aligned(intermediate_channels * npu_ratio, alignment), alignment)

    @property
    def slices(self):
        return {"npu": (0, self.npu_channels), "gpu": (self.npu_channels, self.intermediate_channels)}


def plan_shards(inter, world, ratios=None, alignment=ALIGNMENT):
    """[(begin, end)] channel range of each of `world` ranks. `ratios` (default: equal) are
    relative speeds; boundaries are cumulative shares rounded to the alignment, ties upward.
    Every rank gets at least one aligned block."""
    _positive_int(inter, "inter")
    _positive_int(world, "world")
    if inter % alignment:
        raise ValueError(f"inter must be a multiple of {alignment}")
    if inter // alignment < world:
        raise ValueError("fewer aligned channel blocks than ranks")
    ratios = [1.0] * world if ratios is None else [float(r) for r in ratios]
    if len(ratios) != world or any(not math.isfinite(r) or r <= 0 for r in ratios):
        raise ValueError("ratios must be `world` positive finite numbers")
    total = sum(ratios)
    bounds = [0]
    acc = 0.0
    for r in range(world - 1):
        acc += ratios[r]
        b = round_aligned(inter * acc / total, alignment)
        lo = bounds[-1] + alignment
        hi = inter - (world - 1 - r) * alignment
        bounds.append(min(max(b, lo), hi))
    bounds.append(inter)
    return [(bounds[i], bounds[i + 1]) for i in range(world)]


@dataclasses.dataclass(frozen=True)
class DeviceModel:
    """Roofline of one rank: HBM GB/s, dense tensor TFLOP/s, fixed per-layer overhead (us)."""
    hbm_gbs: float
    tflops: float
    overhead_us: float = 0.0


def shard_bytes(hidden, channels, m, act_bytes=2):
    """Algorithmic HBM bytes of one FFN shard: packed weights (0.53125 B/weight over 3*H*n
    weights) plus x in and the partial out."""
    return 3 * hidden * channels * BYTES_PER_WEIGHT + 2 * m * hidden * act_bytes


def shard_flops(hidden, channels, m):
    return 6.0 * m * hidden * channels


def predict_layer_time(hidden, shares, m, devices, allreduce_us=0.0):
    """T = max over ranks of max(bytes / BW, flops / peak) + overhead, plus the boundary
    all-reduce (split_cost_model.py:8 with host/tail terms replaced by the collective). Seconds."""
    times = []
    for (b, e), dev in zip(shares, devices):
        n = e - b
        t = max(shard_bytes(hidden, n, m) / (dev.hbm_gbs * 1e9), shard_flops(hidden, n, m) / (dev.tflops * 1e12))
        times.append(t + dev.overhead_us * 1e-6)
    return max(times) + allreduce_us * 1e-6


def best_ratios(hidden, inter, m, devices, allreduce_us=0.0, steps=16):
    """Ratios (of a coarse grid around the devices' relative throughput) that minimise
    predict_layer_time; equal devices give equal shares."""
    world = len(devices)
    base = [1.0 / max(shard_bytes(hidden, 1, m) / (d.hbm_gbs * 1e9), shard_flops(hidden, 1, m) / (d.tflops * 1e12))
            for d in devices]
    best = None
    for i in range(-steps // 2, steps // 2 + 1):
        scale = 1.0 + 0.02 * i
        ratios = [base[0] * scale] + base[1:] if world > 1 else base
        shares = plan_shards(inter, world, ratios)
        t = predict_layer_time(hidden, shares, m, devices, allreduce_us)
        if best is None or t < best[0]:
            best = (t, ratios, shares)
    return best[1], best[2]
