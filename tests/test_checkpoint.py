"""The reference's pre-saved weight directory (its on-disk FFN format) read by heteromega_b200.checkpoint.

tests/golden/checkpoint.npz holds four directories written by the reference's own functions
(tests/golden/make_golden.py: _pack_weights_packed of both model writers, _write_tensor_raw,
_split_packed_bin_from_file, _pack_qweight_out_in2, _resolve_layer_pad_packed_alignment): packed
bins with the down projection split along K and layer 0's attention projections (separate and fused
qkv), the 2048-padded variant, the unpacked qweight/scales/zeros bins, and the Qwen writer's
format_version 2 with a fused qkv bin and per-projection (K, N) padding. Every matrix read back must be
byte-identical to the host packer's output for the same q/s/z (the packer itself is pinned to the
reference's packers by test_oracle_golden), and shards cut at load time to slice_packed_ffn's.
"""
import json

import numpy as np
import pytest
import torch

import heteromega_b200 as H
from heteromega_b200.checkpoint import Checkpoint, CheckpointError, load_ffn_stack, tile_positions
from heteromega_b200.partition import plan_shards
from heteromega_b200.tensor_parallel import TensorParallelFfn


@pytest.fixture(scope="module")
def ck_npz(golden):
    return golden("checkpoint")


def materialize(npz, tag, root):
    d = root / tag
    d.mkdir()
    for f in npz[f"{tag}_files"]:
        (d / str(f)).write_bytes(npz[f"{tag}/{f}"].tobytes())
    return d


def expected(npz, layer, name):
    q = torch.from_numpy(npz[f"src_{layer}_{name}_q"])
    s = torch.from_numpy(npz[f"src_{layer}_{name}_s"].view(np.int16)).view(torch.bfloat16)
    z = torch.from_numpy(npz[f"src_{layer}_{name}_z"])
    return H.pack_w4a16(q, s, z)


@pytest.mark.parametrize("tag", ["packed", "padded", "unpacked"])
def test_matrices_match_the_packer(ck_npz, tmp_path, tag):
    ck = Checkpoint(materialize(ck_npz, tag, tmp_path))
    assert (ck.hidden, ck.inter) == (int(ck_npz["hidden"]), int(ck_npz["inter"]))
    for layer in range(ck.layers):
        for name in ("gate", "up", "down"):
            got = ck.matrix(layer, name)
            assert torch.equal(got, expected(ck_npz, layer, name)), f"{tag} layer {layer} {name}"
    if tag == "packed":
        assert ck.split_k == {"down": 256}
        assert not (ck.path / "layer_1_down.packed.bin").exists()  # read from the .k256 split pair
        assert (ck.path / "layer_0_down.packed0.bin").exists()  # and from the untagged pair


def test_shards_match_slices(ck_npz, tmp_path):
    d = materialize(ck_npz, "packed", tmp_path)
    ck = Checkpoint(d)
    for world in (1, 3):
        for begin, end in plan_shards(ck.inter, world):
            for layer in range(ck.layers):
                got = ck.ffn_slice(layer, begin, end)
                g, u, dn = (expected(ck_npz, layer, n) for n in ("gate", "up", "down"))
                ref = H.slice_packed_ffn(g, u, dn, ck.hidden, ck.inter, begin, end, H.GateUpLayout.kInterleaved)
                assert torch.equal(got.gate_up, ref.gate_up) and torch.equal(got.down, ref.down)
    # a tensor-parallel rank keeps only its shard
    tp = TensorParallelFfn(ck.hidden, ck.inter, rank=1, world=3)
    ws = load_ffn_stack(d, "cpu", tp=tp)
    assert len(tp.layers) == ck.layers and ws[0].channels() == tp.end - tp.begin


def test_tile_positions_follow_the_layout():
    for k, n in ((128, 64), (256, 640), (384, 1152), (1024, 192)):
        pos = tile_positions(k, n)
        tk, tn = k // 128, n // 64
        for c in range(tn):
            for r in range(tk):
                assert pos[c, r] == H.packed_tile_index(c, r, tk, tn)


def test_rejects_bad_directories(ck_npz, tmp_path):
    d = materialize(ck_npz, "packed", tmp_path)
    with pytest.raises(CheckpointError):
        Checkpoint(tmp_path / "nowhere")
    m = json.loads((d / "manifest.json").read_text())
    (d / "manifest.json").write_text(json.dumps(dict(m, format_version=3)))
    with pytest.raises(CheckpointError, match="format_version"):
        Checkpoint(d)
    (d / "manifest.json").write_text(json.dumps(dict(m, split_k_by_layer={"down": 200})))
    with pytest.raises(CheckpointError, match="split"):
        Checkpoint(d).matrix(1, "down")
    (d / "manifest.json").write_text(json.dumps(m))
    (d / "layer_0_up.packed.bin").write_bytes(b"\\0" * 100)
    with pytest.raises(CheckpointError, match="bytes"):
        Checkpoint(d).matrix(0, "up")
    (d / "layer_0_gate.packed.bin").unlink()
    with pytest.raises(CheckpointError, match="missing"):
        Checkpoint(d).matrix(0, "gate")
    with pytest.raises(CheckpointError, match="no layer"):
        Checkpoint(d).matrix(5, "gate")


def _cat_expected(npz, names):
    parts = [(npz[f"src_0_{n}_q"], npz[f"src_0_{n}_s"], npz[f"src_0_{n}_z"]) for n in names]
    q, sb, z = (np.concatenate([p[i] for p in parts], axis=1) for i in range(3))
    return H.pack_w4a16(torch.from_numpy(q), torch.from_numpy(sb.view(np.int16)).view(torch.bfloat16), torch.from_numpy(z))


@pytest.mark.parametrize("tag", ["packed", "qwen"])
def test_attention_projections(ck_npz, tmp_path, tag):
    """q, k, v, o and the fused qkv (q, k, v output columns side by side) run on the same packed
    GEMV/GEMM; they are read like the FFN's projections."""
    ck = Checkpoint(materialize(ck_npz, tag, tmp_path))
    assert ck.shape("qkv") == (128, 384) and ck.shape("o") == (128, 128)
    names = ("q", "k", "v", "o") if tag == "packed" else ("o",)
    for name in names:
        assert torch.equal(ck.matrix(0, name), expected(ck_npz, 0, name)), f"{tag} {name}"
    assert torch.equal(ck.attention_layer(0, fused_qkv=True)["qkv"], _cat_expected(ck_npz, ("q", "k", "v")))


def test_qwen_writer_directory(ck_npz, tmp_path):
    """format_version 2, padding (256, 512) with down overridden to (512, 0) and qkv unpadded."""
    ck = Checkpoint(materialize(ck_npz, "qwen", tmp_path))
    assert ck.pad_alignment("gate") == (256, 512) and ck.pad_alignment("down") == (512, 0)
    assert ck.pad_alignment("qkv") == (0, 0)
    for name in ("gate", "up", "down"):
        assert torch.equal(ck.matrix(0, name), expected(ck_npz, 0, name)), name


def test_pad_alignment_settings(tmp_path):
    """The padding rules of _resolve_layer_pad_packed_alignment: off unless pad_packed_weights enables
    it; true is 2048; an int or a (K, N) pair as given; a per-projection entry replaces the default."""
    base = {"format_version": 1, "use_packed_weights": True, "num_hidden_layers": 1, "hidden_size": 128,
            "intermediate_size": 128}
    cases = [(True, None, "gate", (2048, 2048)), (False, {"gate": [64, 64]}, "gate", (0, 0)),
             (512, None, "down", (512, 512)), ("true", None, "up", (2048, 2048)), ([0, 1024], None, "gate", (0, 1024)),
             ([0, 0], {"gate": [256, 256]}, "gate", (0, 0)), (2048, {"down": [0, 128]}, "down", (0, 128)),
             (2048, {"down": [0, 128]}, "gate", (2048, 2048))]
    for i, (pad, by, name, want) in enumerate(cases):
        d = tmp_path / str(i)
        d.mkdir()
        m = dict(base, pad_packed_weights=pad)
        if by is not None:
            m["pad_packed_weights_by_layer"] = by
        (d / "manifest.json").write_text(json.dumps(m))
        assert Checkpoint(d).pad_alignment(name) == want, (pad, by, name)
