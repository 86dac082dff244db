"""Channel partition of an FFN layer across devices.

HeteroMega splits the intermediate channels of each FFN layer between an NPU and a GPU
(npu/ffn/reference.py:121-151): device d owns a contiguous, 128-aligned channel range, gate and
up are cut by output columns, down by input rows, and the per-device partial outputs are summed
once at the layer boundary. Here the same algebra runs over P B200 ranks.

* ChannelSplit holds the ranges of any number of devices as one list of boundaries. Its
  two-device form, ChannelSplit.two_way, puts the cut where the reference's from_ratio puts it:
  the first device's share rounded to the nearest multiple of the alignment, ties upward
  (reference.py:139-147); that rounding rule is the one thing kept alike, so that both place the
  same partition points.
* plan_shards generalises the cut to P ranks: the cumulative share of rank r is rounded the same
  way, so equal shares come out when I/P is aligned and 128-aligned unequal shares otherwise
  (Qwen2.5-14B, I = 13824 over 8 ranks: 4 x 1792 + 4 x 1664).
* predict_layer_time is the per-layer cost form of tools/split_model/split_cost_model.py:8,
  T = max_r(t_r) + tail, with t_r from a roofline of each rank's shard and tail the boundary
  all-reduce; best_ratios scans candidate splits with it.
"""
import dataclasses
import math

ALIGNMENT = 128
BYTES_PER_WEIGHT = 4352 / (128 * 64)  # packed tile bytes per weight: 0.53125


def _count(value, what, minimum=1):
    """value as an int >= minimum; bools and non-integral numbers are refused."""
    if isinstance(value, bool) or int(value) != value or value < minimum:
        raise ValueError(f"{what}: expected an integer >= {minimum}, got {value!r}")
    return int(value)


def round_aligned(value, alignment=ALIGNMENT):
    """Nearest multiple of `alignment`, ties upward."""
    return math.floor(value / alignment + 0.5) * alignment


@dataclasses.dataclass(frozen=True)
class ChannelSplit:
    """Contiguous channel ranges of one FFN layer, one per device in device order, given by their
    boundaries (0, b_1, ..., inter); every boundary is a multiple of `alignment`. A device may own
    no channels (two equal neighbouring boundaries)."""
    inter: int
    bounds: tuple
    alignment: int = ALIGNMENT

    def __post_init__(self):
        inter, align = _count(self.inter, "ChannelSplit.inter"), _count(self.alignment, "ChannelSplit.alignment")
        b = tuple(_count(v, "ChannelSplit boundary", 0) for v in self.bounds)
        if len(b) < 2 or b[0] != 0 or b[-1] != inter:
            raise ValueError(f"ChannelSplit: boundaries must run from 0 to {inter}, got {b}")
        if any(hi < lo for lo, hi in zip(b, b[1:])):
            raise ValueError(f"ChannelSplit: boundaries must not decrease, got {b}")
        if any(v % align for v in b):
            raise ValueError(f"ChannelSplit: boundaries must be multiples of {align}, got {b}")
        object.__setattr__(self, "bounds", b)

    @classmethod
    def two_way(cls, inter, first_ratio, alignment=ALIGNMENT):
        """Two devices, the first taking `first_ratio` of the channels (the reference's NPU share),
        its width rounded to the nearest aligned count, ties upward."""
        r = float(first_ratio)
        if not (0.0 <= r <= 1.0):
            raise ValueError(f"ChannelSplit.two_way: the ratio must lie in [0, 1], got {first_ratio!r}")
        return cls(inter, (0, round_aligned(inter * r, alignment), inter), alignment)

    @classmethod
    def balanced(cls, inter, world, ratios=None, alignment=ALIGNMENT):
        """`world` devices with shares proportional to `ratios` (default equal), see plan_shards."""
        shares = plan_shards(inter, world, ratios, alignment)
        return cls(inter, tuple(b for b, _ in shares) + (inter,), alignment)

    @property
    def devices(self):
        return len(self.bounds) - 1

    def ranges(self):
        """[(begin, end)] per device."""
        return list(zip(self.bounds, self.bounds[1:]))

    def __getitem__(self, device):
        return self.bounds[device], self.bounds[device + 1]


def plan_shards(inter, world, ratios=None, alignment=ALIGNMENT):
    """[(begin, end)] channel range of each of `world` ranks. `ratios` (default: equal) are
    relative speeds; boundaries are cumulative shares rounded to the alignment, ties upward.
    Every rank gets at least one aligned block."""
    inter, world = _count(inter, "plan_shards inter"), _count(world, "plan_shards world")
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
