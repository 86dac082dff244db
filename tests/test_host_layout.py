"""Host side of the product, no GPU: the C ABI library loads and exports every declared symbol,
the host packer and slice maps give the reference's bytes, AWQ unpacking, argument errors."""
import hashlib
import os
import re

import numpy as np
import pytest
import torch

import heteromega_b200 as H
from heteromega_b200 import _lib
from heteromega_b200.weights import unpack_awq_qweight, unpack_awq_qzeros

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    src = open(os.path.join(REPO, "include", "hmb.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(hmb_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    L = _lib.lib()
    names = declared_symbols()
    assert len(names) >= 15
    for name in names:
        assert hasattr(L, name), name
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"


def test_status_strings():
    L = _lib.lib()
    for s in range(0, -8, -1):
        assert L.hmb_status_string(s)
    assert L.hmb_version() >= 100


def test_argument_errors_need_no_gpu():
    L = _lib.lib()
    assert L.hmb_w4a16_gemv(None, 128, 64, None, 128, 0, None, 64, 0, 1, 128, 64, 0, 0, 0, 0, None, 0, None) == -1
    buf = np.zeros(64, np.uint8)
    p = buf.ctypes.data
    # k not a multiple of 128, unsupported dtype, bad epilogue, misaligned pointer
    assert L.hmb_w4a16_gemv(p, 128, 64, p, 128, 0, p, 64, 0, 1, 100, 64, 0, 0, 0, 0, None, 0, None) == -1
    assert L.hmb_w4a16_gemv(p, 128, 64, p, 128, 2, p, 64, 0, 1, 128, 64, 0, 0, 0, 0, None, 0, None) == -1
    assert L.hmb_w4a16_gemv(p, 128, 64, p, 128, 0, p, 64, 0, 1, 128, 64, 0, 7, 0, 0, None, 0, None) == -1
    assert L.hmb_w4a16_gemv(p + 1, 128, 64, p, 128, 0, p, 64, 0, 1, 128, 64, 0, 0, 0, 0, None, 0, None) == -2
    assert L.hmb_silu_mul(p, 16, p, 8, 1, 8, 3, None) == -1
    assert L.hmb_packed_bytes(100, 64) == -1 and L.hmb_packed_bytes(256, 128) == 2 * 2 * 4352


def test_host_packer_matches_golden(golden):
    g = golden("packing")
    for key in sorted({k.rsplit("_", 1)[0] for k in g.files}):
        q = torch.from_numpy(g[key + "_q"])
        s = torch.from_numpy(g[key + "_s"].view(np.int16)).view(torch.bfloat16)
        z = torch.from_numpy(g[key + "_z"])
        assert np.array_equal(H.pack_w4a16(q, s, z).numpy(), g[key + "_packed"]), key


def test_packer_rejects_values_above_15():
    q = torch.zeros(128, 64, dtype=torch.uint8)
    s = torch.ones(1, 64, dtype=torch.bfloat16)
    z = torch.zeros(1, 64, dtype=torch.uint8)
    H.pack_w4a16(q, s, z)
    q[5, 7] = 16
    with pytest.raises(ValueError):
        H.pack_w4a16(q, s, z)
    q[5, 7] = 0
    z[0, 3] = 16
    with pytest.raises(ValueError):
        H.pack_w4a16(q, s, z)
    with pytest.raises(ValueError):
        H.pack_w4a16(torch.zeros(100, 64, dtype=torch.uint8), s, z)


def test_tile_index_matches_oracle(oracle):
    for tk, tn in ((1, 1), (3, 10), (2, 18), (7, 64)):
        for c in range(tn):
            for r in range(tk):
                assert H.packed_tile_index(c, r, tk, tn) == oracle.tile_index(c, r, tk, tn)
    with pytest.raises(ValueError):
        H.packed_tile_index(10, 0, 3, 10)


def _slice_inputs(g):
    def mat(name):
        q = torch.from_numpy(g[name + "_q"])
        s = torch.from_numpy(g[name + "_s"].view(np.int16)).view(torch.bfloat16)
        z = torch.from_numpy(g[name + "_z"])
        return q, s, z

    return mat("gate"), mat("up"), mat("down")


def test_pack_ffn_slice_and_slice_packed_ffn_match_reference_bytes(golden):
    g = golden("slices")
    hidden, inter = int(g["hidden"]), int(g["inter"])
    (gq, gs, gz), (uq, us, uz), (dq, ds, dz) = _slice_inputs(g)
    layer = H.FfnLayerQuant(gq, gs, gz, uq, us, uz, dq, ds, dz)
    pg, pu, pd = H.pack_w4a16(gq, gs, gz), H.pack_w4a16(uq, us, uz), H.pack_w4a16(dq, ds, dz)
    for (b, e, layout), gu_sha, dn_sha in zip(g["ranges"], g["gate_up_sha"], g["down_sha"]):
        b, e, layout = int(b), int(e), H.GateUpLayout(int(layout))
        w = H.pack_ffn_slice(layer, b, e, layout)
        assert hashlib.sha256(w.gate_up.numpy().tobytes()).hexdigest() == gu_sha, (b, e, layout)
        assert hashlib.sha256(w.down.numpy().tobytes()).hexdigest() == dn_sha, (b, e, layout)
        v = H.slice_packed_ffn(pg, pu, pd, hidden, inter, b, e, layout)
        assert torch.equal(v.gate_up, w.gate_up) and torch.equal(v.down, w.down), (b, e, layout)


def test_slice_errors():
    p = torch.zeros(H.gpu_ffn.packed_bytes(128, 256), dtype=torch.uint8)
    with pytest.raises(ValueError):
        H.slice_packed_ffn(p, p, p, 128, 256, 64, 256)
    with pytest.raises(ValueError):
        H.slice_packed_ffn(p, p, p, 128, 256, 128, 384)
    w = H.FfnSliceWeights(p, p, 0, 256, 128, H.GateUpLayout.kBlocked)
    with pytest.raises(ValueError):
        w.prefix(128)
    wi = H.FfnSliceWeights(p, p, 0, 256, 128, H.GateUpLayout.kInterleaved)
    assert wi.prefix(128).channels() == 128 and wi.prefix(128).stored_channels() == 256


def test_awq_unpack_matches_reference(golden):
    g = golden("awq")
    assert np.array_equal(unpack_awq_qweight(torch.from_numpy(g["qweight"])).numpy(), g["q"])
    assert np.array_equal(unpack_awq_qzeros(torch.from_numpy(g["qzeros"])).numpy(), g["z"])


def test_gpu_ops_refuse_cpu_tensors():
    """The product has no CPU fallback: kernels only take CUDA tensors."""
    x = torch.zeros(1, 128, dtype=torch.bfloat16)
    y = torch.zeros(1, 64, dtype=torch.bfloat16)
    p = torch.zeros(4352, dtype=torch.uint8)
    with pytest.raises((ValueError, NotImplementedError, RuntimeError)):
        H.gemv_w4a16(y, x, p, 128, 64, 128, 64)


def test_gpu_ffn_split_from_env():
    """HETEROMEGA_GPU_FFN_SPLIT=<s_prefill>,<s_decode> as the reference's model setup reads it
    (unified_llm_w4a16.cpp:2377-2382): both channel counts multiples of 128 within the layer."""
    from heteromega_b200.weights import synthetic_layer

    layer = synthetic_layer(256, 512, layer=0)
    g, u, d = (H.pack_w4a16(q, s, z) for q, s, z in ((layer.gate_q, layer.gate_s, layer.gate_z),
                                                     (layer.up_q, layer.up_s, layer.up_z),
                                                     (layer.down_q, layer.down_s, layer.down_z)))
    model = H.GpuFfnModel()
    model.add_layer(g, u, d, 256, 512)
    assert not model.split_from_env({})
    assert model.split_from_env({"HETEROMEGA_GPU_FFN_SPLIT": "384,128"})
    assert model.channels(7) == 384 and model.channels(1) == 128
    for bad in ("384", "384,100", "a,b", "1024,128"):
        with pytest.raises(ValueError):
            model.split_from_env({"HETEROMEGA_GPU_FFN_SPLIT": bad})
