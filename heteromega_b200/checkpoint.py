"""The reference's pre-saved weight directory, read on the host and handed to the GPU FFN.

The reference converts a quantized checkpoint once into a directory of raw files
(py/unified_llm_w4a16/llama3_8b_w4a16_model.py:962-1169) and its C++ model loads them from there
(src/unified_llm_w4a16_hetero/helper.cpp:1047-1120):

* ``manifest.json``: format_version 1, use_packed_weights, pad_packed_weights, split_k_by_layer,
  num_hidden_layers, hidden_size, intermediate_size, groupsize, ...
* packed: ``layer_{i}_{name}.packed.bin``, the packed tile layout of the [K, N] matrix, with K and N
  padded (to multiples of 2048 when pad_packed_weights is true); a projection split along K at
  split_k_by_layer[name] comes as ``layer_{i}_{name}.k{split}.packed0.bin`` / ``.packed1.bin``
  (older directories: ``layer_{i}_{name}.packed0.bin`` / ``.packed1.bin``), the tiles of rows below
  and from the split.
* unpacked: ``.qweight.bin`` [N, K/2] bytes (low nibble = even K row), ``.scales.bin`` [N, K/128]
  bf16 and ``.zeros.bin`` [N, K/128] int8.

The FFN projections (gate, up, down) and the attention projections (q, k, v, o, and the fused
``layer_{i}_qkv.packed.bin`` of src/unified_llm_w4a16_hetero/helper.cpp:1163-1181) share the same
packed GEMV/GEMM (``packed_linear``). Every matrix comes back as the unpadded packed [K, N] tensor
on the CPU. ``ffn_slice`` cuts one rank's channel range out of a layer at load time by tile gather,
so a tensor-parallel rank moves only its shard to the GPU. The Qwen writer's variant is read too:
format_version 2 with fused qkv bins, and padding given as an alignment, a (K, N) pair, or per
projection (pad_packed_weights_by_layer).
"""
import json
from pathlib import Path

import numpy as np
import torch

from .gpu_ffn import FfnSliceWeights, GateUpLayout, kTileBytes, kTileK, kTileN, pack_w4a16, slice_packed_ffn

FORMAT_VERSIONS = (1, 2)  # 2: the same files plus fused qkv bins (qwen25_14b_w4a16_model.py:1234-1253)
PAD_ALIGN = 2048  # pad_packed_weights = true (LEGACY_PAD_PACKED_ALIGNMENT, qwen25_14b_w4a16_model.py:93)
FFN_PROJECTIONS = ("gate", "up", "down")
ATTENTION_PROJECTIONS = ("q", "k", "v", "o", "qkv")


def _round_up(v, a):
    return (v + a - 1) // a * a if a > 0 else v


def _pad_pair(value):
    """(K alignment, N alignment) of a [k, n] pair setting; non-positive entries mean none."""
    if isinstance(value, (list, tuple)) and len(value) >= 2:
        k, n = (int(v) if str(v).lstrip("-").isdigit() else 0 for v in value[:2])
        return max(k, 0), max(n, 0)
    return 0, 0


def _pad_scalar(value):
    """The alignment of a scalar pad_packed_weights setting: true = 2048, a positive int, else none."""
    if isinstance(value, bool):
        return PAD_ALIGN if value else 0
    if isinstance(value, str):
        v = value.strip().lower()
        if v in ("true", "on", "yes"):
            return PAD_ALIGN
        value = v
    try:
        return max(int(value), 0)
    except (TypeError, ValueError):
        return 0


def tile_positions(k, n):
    """pos[c, r]: where tile (column c, row r) of a packed [k, n] matrix sits: tiles ordered by column
    modulo 8, then column, then row (the packed layout's order)."""
    tk, tn = k // kTileK, n // kTileN
    cols = np.arange(tn)
    rank = np.empty(tn, np.int64)
    rank[np.lexsort((cols, cols % 8))] = np.arange(tn)
    return rank[:, None] * tk + np.arange(tk)[None, :]


def _grid(packed, k, n):
    """[tiles_n, tiles_k, 4352] view of a packed [k, n] matrix, indexed by (column, row)."""
    tiles = np.asarray(packed, np.uint8).reshape(-1, kTileBytes)
    return tiles[tile_positions(k, n)]


def _from_grid(grid):
    """The packed bytes of a [tiles_n, tiles_k, 4352] grid, in the packed layout's order."""
    tn, tk, _ = grid.shape
    out = np.empty((tn * tk, kTileBytes), np.uint8)
    out[tile_positions(tk * kTileK, tn * kTileN)] = grid
    return out.reshape(-1)


class CheckpointError(ValueError):
    pass


class Checkpoint:
    """A pre-saved weight directory of the reference (manifest.json and the per-layer files)."""

    def __init__(self, path):
        self.path = Path(path)
        mf = self.path / "manifest.json"
        if not mf.is_file():
            raise CheckpointError(f"{self.path}: no manifest.json")
        self.manifest = json.loads(mf.read_text())
        m = self.manifest
        if m.get("format_version") not in FORMAT_VERSIONS:
            raise CheckpointError(f"{mf}: format_version {m.get('format_version')!r}, expected one of {FORMAT_VERSIONS}")
        for key in ("use_packed_weights", "num_hidden_layers", "hidden_size", "intermediate_size"):
            if key not in m:
                raise CheckpointError(f"{mf}: missing {key}")
        if m.get("groupsize", 128) not in (0, 128):
            raise CheckpointError(f"{mf}: groupsize {m['groupsize']}; the packed tiles hold groups of 128")
        self.layers = int(m["num_hidden_layers"])
        self.hidden = int(m["hidden_size"])
        self.inter = int(m["intermediate_size"])
        self.packed = bool(m["use_packed_weights"])
        self.pad_setting = m.get("pad_packed_weights", False) if self.packed else False
        self.pad_by_layer = m.get("pad_packed_weights_by_layer") or {}
        self.split_k = {k: int(v) for k, v in (m.get("split_k_by_layer") or {}).items()} if self.packed else {}
        if self.hidden % kTileK or self.inter % kTileK:
            raise CheckpointError(f"{mf}: hidden and intermediate sizes must be multiples of 128")

    def shape(self, name):
        """(K, N) of a projection: the FFN's gate, up, down, or the attention's q, k, v, o and the
        fused qkv (q, k and v output columns side by side), from the manifest's head counts."""
        if name in ("gate", "up"):
            return self.hidden, self.inter
        if name == "down":
            return self.inter, self.hidden
        if name in ATTENTION_PROJECTIONS:
            m = self.manifest
            try:
                heads, kv, hd = int(m["num_attention_heads"]), int(m["num_key_value_heads"]), int(m["head_dim"])
            except KeyError as e:
                raise CheckpointError(f"{self.path}/manifest.json: missing {e.args[0]} for the attention projections") from None
            return {"q": (self.hidden, heads * hd), "k": (self.hidden, kv * hd), "v": (self.hidden, kv * hd),
                    "o": (heads * hd, self.hidden), "qkv": (self.hidden, (heads + 2 * kv) * hd)}[name]
        raise CheckpointError(f"not a projection: {name}")

    def pad_alignment(self, name):
        """(K, N) padding alignment of a projection's packed file, resolved as the reference's writer
        does (_resolve_layer_pad_packed_alignment, qwen25_14b_w4a16_model.py:197-217): off unless
        pad_packed_weights enables it; then the projection's pad_packed_weights_by_layer entry, else
        the default."""
        d = self.pad_setting
        if isinstance(d, (list, tuple)):
            enabled = _pad_pair(d)
            if enabled == (0, 0):
                return 0, 0
        else:
            a = _pad_scalar(d)
            if a <= 0:
                return 0, 0
            enabled = (a, a)
        spec = self.pad_by_layer.get(name)
        return _pad_pair(spec) if spec is not None else enabled

    def _read(self, path, expect_bytes):
        if not path.is_file():
            raise CheckpointError(f"missing {path}")
        data = np.fromfile(path, np.uint8)
        if data.size != expect_bytes:
            raise CheckpointError(f"{path}: {data.size} bytes, expected {expect_bytes}")
        return data

    def matrix(self, layer, name):
        """The packed [K, N] matrix of projection `name` of layer `layer` (flat uint8, CPU), unpadded."""
        if not 0 <= layer < self.layers:
            raise CheckpointError(f"no layer {layer} (the manifest lists {self.layers})")
        k, n = self.shape(name)
        prefix = f"layer_{layer}_{name}"
        if not self.packed:
            return torch.from_numpy(self._unpacked(prefix, k, n))
        ak, an = self.pad_alignment(name)
        kp, np_ = _round_up(k, ak), _round_up(n, an)
        split = self.split_k.get(name, 0)
        if 0 < split < k:
            grid = self._split_grid(prefix, k, n, kp, np_, split, ak)
        else:
            data = self._read(self.path / f"{prefix}.packed.bin", (kp // kTileK) * (np_ // kTileN) * kTileBytes)
            if (kp, np_) == (k, n):
                return torch.from_numpy(data)
            grid = _grid(data, kp, np_)
        return torch.from_numpy(_from_grid(np.ascontiguousarray(grid[: n // kTileN, : k // kTileK])))

    def _split_grid(self, prefix, k, n, kp, np_, split, ak):
        # The two halves are packed [split, N] and [K - split, N] matrices (the reference filters the
        # whole matrix's tiles by row, keeping their order); with padding the first half must end on a
        # padding boundary, where both of the reference's writers agree on the halves.
        if split % kTileK or (ak and split % ak):
            raise CheckpointError(f"{prefix}: K split {split} is not a multiple of {ak or kTileK}")
        k0, k1 = split, kp - split
        p0 = self.path / f"{prefix}.k{split}.packed0.bin"
        p1 = self.path / f"{prefix}.k{split}.packed1.bin"
        if not (p0.is_file() and p1.is_file()):  # directories written before the files were tagged
            p0, p1 = self.path / f"{prefix}.packed0.bin", self.path / f"{prefix}.packed1.bin"
        tn = np_ // kTileN
        g0 = _grid(self._read(p0, tn * (k0 // kTileK) * kTileBytes), k0, np_)
        g1 = _grid(self._read(p1, tn * (k1 // kTileK) * kTileBytes), k1, np_)
        return np.concatenate([g0[:, : k0 // kTileK], g1[:, : (k - k0) // kTileK]], axis=1)

    def _unpacked(self, prefix, k, n):
        groups = k // kTileK
        qb = self._read(self.path / f"{prefix}.qweight.bin", n * k // 2).reshape(n, k // 2)
        s = self._read(self.path / f"{prefix}.scales.bin", n * groups * 2).view(np.uint16).reshape(n, groups)
        z = self._read(self.path / f"{prefix}.zeros.bin", n * groups).view(np.int8).reshape(n, groups)
        q = np.empty((n, k), np.uint8)
        q[:, 0::2] = qb & 15
        q[:, 1::2] = qb >> 4
        if z.min() < 0 or z.max() > 15:
            raise CheckpointError(f"{prefix}.zeros.bin: zero points outside 0..15")
        packed = pack_w4a16(torch.from_numpy(np.ascontiguousarray(q.T)),
                            torch.from_numpy(np.ascontiguousarray(s.T)).view(torch.bfloat16),
                            torch.from_numpy(np.ascontiguousarray(z.T).astype(np.uint8)))
        return packed.numpy()

    def attention_layer(self, layer, fused_qkv=False):
        """{'q', 'k', 'v', 'o'} (or {'qkv', 'o'}) packed matrices of layer `layer`, on the CPU."""
        names = ("qkv", "o") if fused_qkv else ("q", "k", "v", "o")
        return {name: self.matrix(layer, name) for name in names}

    def ffn_layer(self, layer):
        """(gate [H, I], up [H, I], down [I, H]) packed, on the CPU."""
        return tuple(self.matrix(layer, name) for name in FFN_PROJECTIONS)

    def ffn_slice(self, layer, begin=0, end=None, layout=GateUpLayout.kInterleaved) -> FfnSliceWeights:
        """Channels [begin, end) of layer `layer` as an FfnSliceWeights on the CPU (tile gather)."""
        end = self.inter if end is None else end
        g, u, d = self.ffn_layer(layer)
        return slice_packed_ffn(g, u, d, self.hidden, self.inter, begin, end, layout)


def load_ffn_stack(path, device, tp=None, layers=None):
    """The FFN layers of a pre-saved directory on `device`: a list of FfnSliceWeights with all
    channels, or, given a TensorParallelFfn, its rank's shards (added to it, and returned)."""
    ck = Checkpoint(path)
    if tp is not None and (tp.hidden, tp.inter) != (ck.hidden, ck.inter):
        raise CheckpointError(f"{path}: [{ck.hidden}, {ck.inter}] does not match the tensor-parallel FFN")
    out = []
    for layer in range(ck.layers if layers is None else layers):
        if tp is None:
            out.append(ck.ffn_slice(layer).to(device))
        else:
            w = ck.ffn_slice(layer, tp.begin, tp.end).to(device)
            tp.add_shard(w)
            out.append(w)
    return out
