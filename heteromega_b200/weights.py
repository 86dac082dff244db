"""Weight preparation: AWQ checkpoint unpacking and seeded synthetic W4A16 layers.

* unpack_awq_qweight / unpack_awq_qzeros restate HeteroMosaic's loader
  (py/unified_llm_w4a16/llama3_8b_w4a16_model.py:325-358): an AWQ int32 word holds 8
  consecutive output columns, nibble k of the word at bit 4 * [0, 4, 1, 5, 2, 6, 3, 7][k].
  The kernels never see this order; it is undone before packing tiles.
* synthetic_* draw the benchmark's inputs: q ~ U{0..15}, zeros ~ U{0..15} per (group, column),
  scales ~ U(0.002, 0.02) rounded once to bf16, group 128 along K, activations ~ N(0, 1).
  Weights of layer l use seed 1000 + l, activations seed 7.
"""
import numpy as np
import torch

from .gpu_ffn import FfnLayerQuant, kTileBytes, kTileK, kTileN

AWQ_ORDER = (0, 4, 1, 5, 2, 6, 3, 7)
WEIGHT_SEED_BASE = 1000
ACTIVATION_SEED = 7


def _awq_nibbles(words):
    w = words.to(torch.int64) & 0xFFFFFFFF
    parts = [((w >> (4 * AWQ_ORDER[k])) & 0xF) for k in range(8)]
    return torch.stack(parts, dim=-1)  # [..., cols/8, 8]


def unpack_awq_qweight(qweight):
    """[in, out/8] int32 -> [in, out] uint8 (llama3_8b_w4a16_model.py:340-349)."""
    n = _awq_nibbles(qweight)
    return n.reshape(qweight.shape[0], qweight.shape[1] * 8).to(torch.uint8)


def unpack_awq_qzeros(qzeros):
    """[groups, out/8] int32 -> [groups, out] zero points (llama3_8b_w4a16_model.py:352-358)."""
    n = _awq_nibbles(qzeros)
    return n.reshape(qzeros.shape[0], qzeros.shape[1] * 8).to(torch.uint8)


def bf16_round(values):
    """fp32 -> bf16 (ties to even) as a torch bfloat16 tensor."""
    return torch.from_numpy(np.ascontiguousarray(values, np.float32)).to(torch.bfloat16)


def synthetic_quant(k, n, rng, zero_range=(0, 16), scale_range=(0.002, 0.02)):
    """(q [k, n] uint8, scales [k/128, n] bf16, zeros [k/128, n] uint8) as CPU tensors."""
    q = rng.integers(0, 16, (k, n), dtype=np.uint8)
    s = rng.uniform(scale_range[0], scale_range[1], (k // kTileK, n)).astype(np.float32)
    z = rng.integers(zero_range[0], zero_range[1], (k // kTileK, n), dtype=np.uint8)
    return torch.from_numpy(q), bf16_round(s), torch.from_numpy(z)


def synthetic_layer(hidden, inter, layer=0, zero_range=(0, 16)):
    """A seeded FfnLayerQuant with gate/up [hidden, inter] and down [inter, hidden]."""
    rng = np.random.default_rng(WEIGHT_SEED_BASE + layer)
    g = synthetic_quant(hidden, inter, rng, zero_range)
    u = synthetic_quant(hidden, inter, rng, zero_range)
    d = synthetic_quant(inter, hidden, rng, zero_range)
    return FfnLayerQuant(*g, *u, *d)


def synthetic_activations(m, hidden, seed=ACTIVATION_SEED, dtype=torch.bfloat16):
    rng = np.random.default_rng(seed)
    return torch.from_numpy(rng.standard_normal((m, hidden)).astype(np.float32)).to(dtype)


def synthetic_packed_device(k, n, device, generator, scale_range=(0.002, 0.02), zero_range=(0, 16)):
    """Packed [k, n] tiles drawn directly on the device: uniform nibble bytes (q ~ U{0..15}),
    bf16 scales ~ U(scale_range) and zeros ~ U{zero_range} (stored twice) in their tile slots.
    The same distribution as packing synthetic_quant's output, without a host round trip."""
    tiles = (k // kTileK) * (n // kTileN)
    p = torch.randint(0, 256, (tiles, kTileBytes), dtype=torch.uint8, device=device, generator=generator)
    s = torch.empty(tiles, 64, dtype=torch.float32, device=device).uniform_(scale_range[0], scale_range[1],
                                                                              generator=generator)
    p[:, 4096:4224] = s.to(torch.bfloat16).view(torch.uint8)
    z = torch.randint(zero_range[0], zero_range[1], (tiles, 8, 8), dtype=torch.uint8, device=device, generator=generator)
    p[:, 4224:] = torch.cat([z, z], dim=2).view(tiles, 128)
    return p.view(-1)
