"""Generate the golden fixtures in this folder from the reference's own code.

Run where the reference tree is available, with its location in $HETEROMEGA_REF, after
``make -C oracle ref REF=$HETEROMEGA_REF``:

    HETEROMEGA_REF=<reference checkout> python tests/golden/make_golden.py

It imports the reference's Python packers and oracles and runs its CPU AVX GEMV
(compiled unchanged into oracle/_ref/), and writes small .npz fixtures that the
CPU tests compare the C oracle and the host packer with. Nothing here runs at
test time; the GPU box never sees the reference tree.

Reference code used (paths inside glassescrab/HeteroMega):
  py/unified_llm_w4a16/llama3_8b_w4a16_model.py   _pack_weights_packed (546-656),
                                                  _unpack_awq_qweight/_qzeros (340-358),
                                                  the pre-saved weight directory: _write_tensor_raw (318-322),
                                                  _pack_qweight_out_in2 (410-419), _split_packed_paths
                                                  (460-465), _split_packed_bin_from_file (468-529),
                                                  the manifest keys (962-978) and file names (1069-1168)
  kernels/gpu/tools/check_packing.py              pack (53-69), gemv_packed (91-112)
  experiments/ffn_partition/gpu_backend.py        pack_heteromosaic_weights (33-77)
  experiments/ffn_partition/test_gpu_packing.py   decode_gpu_addresses (18-43)
  experiments/ffn_partition/contract.py           random_weights (76-95), error_metrics (172-208)
  npu/ffn/reference.py                            bf16 (26-35), FFNPartition.from_ratio (139-147),
                                                  ffn_reference / ffn_partitioned (192-221)
  src/cpu_avx_kernels/w4a16_gemv_avx_packed.cpp   w4a16_gemv_cpu_fused_packed (via oracle/_ref)
"""
import hashlib
import os
import sys

import numpy as np

REF = os.environ.get("HETEROMEGA_REF")
if not REF or not os.path.isdir(REF):
    raise SystemExit("make_golden.py: set HETEROMEGA_REF to the reference checkout")
HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
for sub in ("kernels/gpu/tools", "experiments/ffn_partition", "npu/ffn", "py/unified_llm_w4a16"):
    sys.path.insert(0, os.path.join(REF, sub))
sys.path.insert(0, REPO)

import torch  # noqa: E402

import check_packing  # noqa: E402
import contract  # noqa: E402
import gpu_backend  # noqa: E402
import reference  # noqa: E402
import test_gpu_packing  # noqa: E402
import llama3_8b_w4a16_model as hm_model  # noqa: E402
import qwen25_14b_w4a16_model as qwen_model  # noqa: E402

from oracle import oracle as O  # noqa: E402

SEED = 20261201


def rng(tag):
    return np.random.default_rng(SEED + tag)


def quant(r, k, n, zlo=0, zhi=16):
    q = r.integers(0, 16, (k, n), dtype=np.uint8)
    s = reference.bf16(r.uniform(0.002, 0.02, (k // 128, n)).astype(np.float32))
    z = r.integers(zlo, zhi, (k // 128, n), dtype=np.uint8)
    return q, s, z


def bits(f32):
    return np.ascontiguousarray(f32, np.float32).view(np.uint32) >> 16


def torch_pack(q, s_f32, z):
    """The reference model's own packer (torch), [K, N] q, [K/128, N] bf16 scales, int8 zeros."""
    k, n = q.shape
    return hm_model._pack_weights_packed(torch.from_numpy(q.astype(np.int8)), torch.from_numpy(s_f32).to(torch.bfloat16),
                                         torch.from_numpy(z.astype(np.int8)), k, n, False).numpy()


def canonical(q, s_f32, z):
    """[K, N] matrices -> the reference's canonical W4A16 [N, K/2] (npu/ffn/reference.py)."""
    return reference.W4A16(reference.pack_int4(q.T), s_f32.T.copy(), z.T.copy(), 128)


def make_packing():
    out = {}
    # Shapes with uneven modulo-8 column groups (10 and 18 tile columns) and 1..4 tile rows.
    for tag, (k, n) in enumerate(((256, 384), (128, 640), (128, 1152), (512, 192))):
        q, s, z = quant(rng(tag), k, n)
        a = torch_pack(q, s, z)
        b = check_packing.pack(q, bits(s).astype(np.uint16), z.astype(np.int8))
        # The canonical-format adapter only takes N % 128 == 0.
        c = gpu_backend.pack_heteromosaic_weights(canonical(q, s, z)) if n % 128 == 0 else a
        assert np.array_equal(a, b) and np.array_equal(a, c), "the reference's packers disagree"
        dq, ds, dz, dup, sbits = test_gpu_packing.decode_gpu_addresses(a, k, n)
        assert np.array_equal(dq.T, q) and np.array_equal(dz.T, z) and np.array_equal(dup.T, z)
        key = f"k{k}_n{n}"
        out[f"{key}_q"] = q
        out[f"{key}_s"] = bits(s).astype(np.uint16)
        out[f"{key}_z"] = z
        out[f"{key}_packed"] = a
    np.savez_compressed(os.path.join(HERE, "packing.npz"), **out)


def make_awq():
    r = rng(100)
    qweight = r.integers(-2**31, 2**31, (256, 48), dtype=np.int64).astype(np.int32)
    qzeros = r.integers(-2**31, 2**31, (2, 48), dtype=np.int64).astype(np.int32)
    uq = hm_model._unpack_awq_qweight(torch.from_numpy(qweight)).numpy()
    uz = hm_model._unpack_awq_qzeros(torch.from_numpy(qzeros)).numpy()
    np.savez_compressed(os.path.join(HERE, "awq.npz"), qweight=qweight, qzeros=qzeros, q=uq, z=uz.astype(np.uint8))


def make_gemv():
    """The reference AVX kernel and the reference float64 packed GEMV on a few matrices."""
    avx = O.ReferenceAVX()
    out = {"avx512": np.array(avx.avx512)}
    for tag, (k, n) in enumerate(((256, 384), (1024, 256), (2048, 128))):
        r = rng(200 + tag)
        q, s, z = quant(r, k, n)
        p = torch_pack(q, s, z)
        x = reference.bf16(r.standard_normal(k).astype(np.float32))
        key = f"k{k}_n{n}"
        out[f"{key}_packed"] = p
        out[f"{key}_x"] = bits(x).astype(np.uint16)
        out[f"{key}_avx"] = avx.gemv(bits(x).astype(np.uint16), p, k, n, threads=4)
        out[f"{key}_f64"] = check_packing.gemv_packed(p, x.astype(np.float64), k, n)
        # the last 128 columns through start_col/end_col (tile-aligned)
        part = np.zeros(n, np.uint16)
        avx.gemv(bits(x).astype(np.uint16), p, k, n, threads=4, out=part, start_col=n - 128, end_col=n)
        out[f"{key}_avx_lastcols"] = part[n - 128:]
    np.savez_compressed(os.path.join(HERE, "gemv.npz"), **out)


def make_ffn():
    """A small FFN (H=256, I=640) on the contract's seeded weights: the reference float oracle,
    its BF16-boundary contract, and the AVX chain the model's CPU path runs."""
    h, inter = 256, 640
    w = contract.random_weights(h, inter, seed=12832)
    x = np.random.default_rng(SEED + 300).standard_normal((3, h)).astype(np.float32)
    xb = reference.bf16(x)
    packed = {name: gpu_backend.pack_heteromosaic_weights(getattr(w, name)) for name in ("gate", "up", "down")}
    avx = O.ReferenceAVX()
    chain = np.stack([avx.ffn_row(bits(xb[i]).astype(np.uint16), packed["gate"], packed["up"], packed["down"], h, inter,
                                  threads=4) for i in range(3)])
    f32 = reference.ffn_reference(xb, w.gate, w.up, w.down)
    bf16_io = reference.ffn_reference(xb, w.gate, w.up, w.down, bf16_io=True)
    part = reference.FFNPartition(inter, 256)
    reduced, partials = reference.ffn_partitioned(xb, w.gate, w.up, w.down, part)
    np.savez_compressed(os.path.join(HERE, "ffn.npz"), h=h, inter=inter, x=bits(xb).astype(np.uint16),
                        gate=packed["gate"], up=packed["up"], down=packed["down"], avx_chain=chain, f32=f32,
                        bf16_io=bf16_io, part_npu=partials["npu"], part_gpu=partials["gpu"], part_sum=reduced)


def make_contract():
    """error_metrics on fixed vectors, and from_ratio on a table."""
    r = rng(400)
    exp = r.standard_normal(64).astype(np.float32)
    cases = [exp + 0.001 * r.standard_normal(64).astype(np.float32), exp * 1.05, exp + 0.2]
    metrics = [contract.error_metrics(a, exp) for a in cases]
    table = []
    for inter in (8192, 13824, 14336, 28672):
        for ratio in (0.0, 0.125, 0.25, 0.3, 0.5, 0.4464, 1.0):
            table.append((inter, ratio, reference.FFNPartition.from_ratio(inter, ratio).npu_channels))
    np.savez_compressed(os.path.join(HERE, "contract.npz"), expected=exp, actual=np.stack(cases),
                        passed=np.array([m["passed"] for m in metrics]),
                        rel_l2=np.array([m["relative_l2_error"] for m in metrics]),
                        max_abs=np.array([m["max_abs_error"] for m in metrics]),
                        from_ratio=np.array(table, dtype=np.float64))


def make_bf16():
    vals = np.array([0.0, -0.0, 1.0, 1.00390625, 1.005859375, 3.0e38, 1e-40, np.inf, -np.inf, np.nan], np.float32)
    vals = np.concatenate([vals, np.array([0x3F808000, 0x3F818000, 0x3F807FFF, 0x3F808001], np.uint32).view(np.float32),
                           rng(500).standard_normal(4096).astype(np.float32) * 100])
    np.savez_compressed(os.path.join(HERE, "bf16.npz"), values=vals, rounded=reference.bf16(vals))


def make_slices():
    """pack_ffn_slice semantics: slices packed from the sliced matrices with the reference packer;
    stored as sha256 of the bytes next to the seeded inputs."""
    hidden, inter = 128, 1152
    r = rng(600)
    mats = {name: quant(r, *(hidden, inter) if name != "down" else (inter, hidden)) for name in ("gate", "up", "down")}
    out = {}
    for name, (q, s, z) in mats.items():
        out[f"{name}_q"], out[f"{name}_s"], out[f"{name}_z"] = q, bits(s).astype(np.uint16), z
    hashes = []
    for b, e in ((0, 1152), (0, 512), (512, 896), (128, 256), (640, 1152)):
        for layout in (0, 1):
            gq, gs, gz = (a[:, b:e] for a in mats["gate"])
            uq, us, uz = (a[:, b:e] for a in mats["up"])
            n = e - b

            def join(g, u):
                if layout == 0:
                    return np.concatenate([g, u], 1)
                rows = g.shape[0]
                return np.stack([g.reshape(rows, n // 64, 64), u.reshape(rows, n // 64, 64)], 2).reshape(rows, 2 * n)

            gu = torch_pack(join(gq, uq), join(gs, us), join(gz, uz))
            dq, ds, dz = mats["down"]
            dn = torch_pack(dq[b:e], ds[b // 128:e // 128], dz[b // 128:e // 128])
            hashes.append((b, e, layout, hashlib.sha256(gu.tobytes()).hexdigest(), hashlib.sha256(dn.tobytes()).hexdigest()))
    out["ranges"] = np.array([(h[0], h[1], h[2]) for h in hashes], np.int64)
    out["gate_up_sha"] = np.array([h[3] for h in hashes])
    out["down_sha"] = np.array([h[4] for h in hashes])
    out["hidden"], out["inter"] = hidden, inter
    np.savez_compressed(os.path.join(HERE, "slices.npz"), **out)


def make_checkpoint():
    """Three pre-saved weight directories of a 2-layer FFN (hidden 128, intermediate 384), written by
    the reference's own functions: packed bins (down split along K at 256 into its .k256.packed0/1
    pair; layer 0 with the older untagged .packed0/1 names), layer 0 padded to multiples of 2048 (pad_packed_weights), and the
    unpacked qweight/scales/zeros bins. The fixture keeps every file's bytes and the q/s/z drawn."""
    import json
    import tempfile
    from pathlib import Path

    hidden, inter, layers = 128, 384, 2
    specs = [("gate", hidden, inter), ("up", hidden, inter), ("down", inter, hidden)]
    # one attention head and one KV head of 128: q, k, v [128, 128], o [128, 128], fused qkv [128, 384]
    attn = [("q", hidden, 128), ("k", hidden, 128), ("v", hidden, 128), ("o", 128, hidden)]
    out = {"hidden": hidden, "inter": inter, "layers": layers}
    weights = {}
    for l in range(layers):
        for name, k, n in specs:
            q, s, z = quant(rng(500 + 10 * l + len(name)), k, n)
            weights[(l, name)] = (q, s, z)
            out[f"src_{l}_{name}_q"], out[f"src_{l}_{name}_s"], out[f"src_{l}_{name}_z"] = q, bits(s).astype(np.uint16), z
    for name, k, n in attn:
        q, s, z = quant(rng(600 + len(name) + ord(name[0])), k, n)
        weights[(0, name)] = (q, s, z)
        out[f"src_0_{name}_q"], out[f"src_0_{name}_s"], out[f"src_0_{name}_z"] = q, bits(s).astype(np.uint16), z
    for tag, use_packed, pad in (("packed", True, False), ("padded", True, True), ("unpacked", False, False)):
        with tempfile.TemporaryDirectory() as d:
            d = Path(d)
            split = {"down": 256} if tag == "packed" else {}
            n_layers = 1 if pad else layers  # the padded files are 2048 x 2048: one layer is enough
            for l in range(n_layers):
                for name, k, n in specs:
                    q, s, z = weights[(l, name)]
                    if use_packed:
                        packed = hm_model._pack_weights_packed(torch.from_numpy(q.astype(np.int8)),
                                                               torch.from_numpy(s).to(torch.bfloat16),
                                                               torch.from_numpy(z.astype(np.int8)), k, n, pad)
                        path = d / f"layer_{l}_{name}.packed.bin"
                        hm_model._write_tensor_raw(path, packed)
                        if name in split:  # split_k_by_layer applies to this projection of every layer
                            p0, p1 = hm_model._split_packed_paths(d, l, name, split[name])
                            assert hm_model._split_packed_bin_from_file(path, p0, p1, split[name], k, n, pad)
                            path.unlink()  # only the split pair stays, as the split writer leaves it
                            if l == 0:  # the untagged names of older directories, which the C++ loader accepts
                                p0.rename(d / f"layer_{l}_{name}.packed0.bin")
                                p1.rename(d / f"layer_{l}_{name}.packed1.bin")
                    else:
                        hm_model._write_tensor_raw(d / f"layer_{l}_{name}.qweight.bin",
                                                   hm_model._pack_qweight_out_in2(torch.from_numpy(q.astype(np.int8))))
                        # [out, groups], the layout the unpacked writer normalises to
                        # [out, groups] row-major (passed flat: the bytes are the same)
                        hm_model._write_tensor_raw(d / f"layer_{l}_{name}.scales.bin",
                                                   torch.from_numpy(s.T.copy().ravel()).to(torch.bfloat16))
                        hm_model._write_tensor_raw(d / f"layer_{l}_{name}.zeros.bin",
                                                   torch.from_numpy(z.T.copy().ravel().astype(np.int8)))
            if tag == "packed":  # layer 0's attention projections, separate and fused (q|k|v columns)
                for name, k, n in attn:
                    q, s, z = weights[(0, name)]
                    hm_model._write_tensor_raw(d / f"layer_0_{name}.packed.bin", torch.from_numpy(torch_pack(q, s, z)))
                qs = [weights[(0, nm)] for nm in ("q", "k", "v")]
                cat = [np.concatenate([w[i] for w in qs], axis=1) for i in range(3)]
                hm_model._write_tensor_raw(d / "layer_0_qkv.packed.bin", torch.from_numpy(torch_pack(*cat)))
            manifest = {"format_version": 1, "model_name": "tiny-ffn", "use_packed_weights": use_packed,
                        "pad_packed_weights": pad, "heterogeneity": "gpu",
                        "split_k_by_layer": split if use_packed else {}, "num_hidden_layers": n_layers,
                        "hidden_size": hidden, "intermediate_size": inter, "num_attention_heads": 1,
                        "num_key_value_heads": 1, "head_dim": 128, "groupsize": 128}
            if not use_packed:
                manifest["unpacked_layout"] = "out_groups_v2"
            (d / "manifest.json").write_text(json.dumps(manifest, indent=2))
            names = sorted(f.name for f in d.iterdir())
            out[f"{tag}_files"] = np.array(names)
            for f in names:
                out[f"{tag}/{f}"] = np.frombuffer((d / f).read_bytes(), np.uint8)
    # The Qwen writer's variant (qwen25_14b_w4a16_model.py:1230-1253, 1467-1512): format_version 2 with a
    # fused qkv bin, padding given as a (K, N) alignment pair and overridden per projection.
    pad_default, pad_by = (256, 512), {"down": [512, 0], "qkv": [0, 0]}
    with tempfile.TemporaryDirectory() as d:
        d = Path(d)
        for name, k, n in specs + attn[3:]:
            q, s, z = weights[(0, name)]
            spec = qwen_model._resolve_layer_pad_packed_alignment(pad_default, {a: tuple(b) for a, b in pad_by.items()}, name)
            packed = qwen_model._pack_weights_packed(torch.from_numpy(q.astype(np.int8)), torch.from_numpy(s).to(torch.bfloat16),
                                                     torch.from_numpy(z.astype(np.int8)), k, n, spec)
            hm_model._write_tensor_raw(d / f"layer_0_{name}.packed.bin", packed)
        qs = [weights[(0, nm)] for nm in ("q", "k", "v")]
        cat = [np.concatenate([w[i] for w in qs], axis=1) for i in range(3)]
        spec = qwen_model._resolve_layer_pad_packed_alignment(pad_default, {a: tuple(b) for a, b in pad_by.items()}, "qkv")
        packed = qwen_model._pack_weights_packed(torch.from_numpy(cat[0].astype(np.int8)), torch.from_numpy(cat[1]).to(torch.bfloat16),
                                                 torch.from_numpy(cat[2].astype(np.int8)), hidden, 384, spec)
        hm_model._write_tensor_raw(d / "layer_0_qkv.packed.bin", packed)
        manifest = {"format_version": 2, "model_name": "tiny-ffn", "use_packed_weights": True,
                    "pad_packed_weights": list(pad_default), "pad_packed_weights_by_layer": pad_by, "heterogeneity": "gpu",
                    "split_k_by_layer": {}, "num_hidden_layers": 1, "hidden_size": hidden, "intermediate_size": inter,
                    "num_attention_heads": 1, "num_key_value_heads": 1, "head_dim": 128, "groupsize": 128,
                    "qwen_fused_qkv_bins": True}
        (d / "manifest.json").write_text(json.dumps(manifest, indent=2))
        names = sorted(f.name for f in d.iterdir())
        out["qwen_files"] = np.array(names)
        for f in names:
            out[f"qwen/{f}"] = np.frombuffer((d / f).read_bytes(), np.uint8)
    np.savez_compressed(os.path.join(HERE, "checkpoint.npz"), **out)


if __name__ == "__main__":
    only = sys.argv[1:]
    for fn in (make_packing, make_awq, make_gemv, make_ffn, make_contract, make_bf16, make_slices, make_checkpoint):
        if not only or fn.__name__ in only:
            fn()
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".npz"):
            print(f, os.path.getsize(os.path.join(HERE, f)))
