"""Pins the CPU oracle (oracle/w4a16_oracle.c) to the reference: fixtures made by the reference's
own packers, NumPy oracles and CPU AVX kernel (tests/golden/make_golden.py), and the reference
AVX kernel itself where oracle/_ref is built."""
import numpy as np
import pytest

from metrics import LEVEL, assert_bf16_close, assert_close, error_metrics


def test_pack_matches_reference_packers(oracle, golden):
    g = golden("packing")
    for key in sorted({k.rsplit("_", 1)[0] for k in g.files}):
        packed = oracle.pack(g[key + "_q"], g[key + "_s"], g[key + "_z"])
        assert np.array_equal(packed, g[key + "_packed"]), key


def test_unpack_round_trip(oracle, golden):
    g = golden("packing")
    for key in sorted({k.rsplit("_", 1)[0] for k in g.files}):
        k, n = (int(v[1:]) for v in key.split("_"))
        q, s, z = oracle.unpack(g[key + "_packed"], k, n)
        assert np.array_equal(q, g[key + "_q"]) and np.array_equal(s, g[key + "_s"]) and np.array_equal(z, g[key + "_z"])


def test_dequant_is_exact(oracle, golden):
    g = golden("packing")
    key = "k256_n384"
    w = oracle.dequant(g[key + "_packed"], 256, 384)
    s = oracle.bf16_to_f32(g[key + "_s"]).astype(np.float64)
    ref = (g[key + "_q"].astype(np.float64) - np.repeat(g[key + "_z"], 128, 0)) * np.repeat(s, 128, 0)
    assert np.array_equal(w.astype(np.float64), ref)


def test_tile_index_orders_columns_mod_8(oracle):
    # 10 tile columns: groups 0 and 1 hold two columns, groups 2..7 one (kernels/gpu/src/pack_w4a16.cpp:100-107).
    order = sorted(((c, r) for c in range(10) for r in range(3)), key=lambda t: oracle.tile_index(t[0], t[1], 3, 10))
    expect = [(c, r) for g in range(8) for c in range(g, 10, 8) for r in range(3)]
    assert order == expect


def test_gemv_matches_reference_avx_fixture(oracle, golden):
    g = golden("gemv")
    for key in ("k256_n384", "k1024_n256", "k2048_n128"):
        k, n = (int(v[1:]) for v in key.split("_"))
        y32, y16 = oracle.gemv(g[key + "_packed"], k, n, g[key + "_x"][None])
        assert_bf16_close(y16[0], g[key + "_avx"], min_equal=0.98, what=key)
        rel = np.abs(y32[0] - g[key + "_f64"]).max() / np.abs(g[key + "_f64"]).max()
        assert rel < 1e-5, key
        _, part = oracle.gemv(g[key + "_packed"], k, n, g[key + "_x"][None], n=128, n0=n - 128)
        assert_bf16_close(part[0], g[key + "_avx_lastcols"], min_equal=0.98, what=key + " cols")


def test_ffn_matches_reference_cpu_chain(oracle, golden):
    g = golden("ffn")
    h, inter = int(g["h"]), int(g["inter"])
    # The reference packs gate and up separately; the oracle takes the blocked gate_up concatenation.
    gate_up = oracle.pack(*_concat_unpacked(oracle, g["gate"], g["up"], h, inter))
    y16, y32 = oracle.ffn(gate_up, g["down"], h, inter, inter, 0, g["x"])
    assert_bf16_close(y16, g["avx_chain"], min_equal=0.95, what="ffn vs AVX chain")
    # The float oracle of npu/ffn/reference.py keeps everything fp32: same values within LEVEL.
    assert_close(y32, g["f32"], LEVEL, "ffn vs fp32 reference oracle")
    # Partition algebra: the two partials of the reference's split add up to its full result.
    assert_close(g["part_npu"] + g["part_gpu"], g["f32"], (1e-6, 1e-6, 0.999999), "partials")


def _concat_unpacked(oracle, gate, up, h, inter):
    gq, gs, gz = oracle.unpack(gate, h, inter)
    uq, us, uz = oracle.unpack(up, h, inter)
    return np.concatenate([gq, uq], 1), np.concatenate([gs, us], 1), np.concatenate([gz, uz], 1)


def test_bf16_rounding_matches_reference(oracle, golden):
    g = golden("bf16")
    vals, ref = g["values"], g["rounded"]
    got = oracle.bf16_to_f32(oracle.bf16_bits(vals))
    finite = np.isfinite(ref)
    assert np.array_equal(got[finite], ref[finite])
    assert np.array_equal(np.isnan(got), np.isnan(ref))


def test_error_metrics_restatement(golden):
    g = golden("contract")
    for i in range(len(g["actual"])):
        m = error_metrics(g["actual"][i], g["expected"])
        assert m["passed"] == bool(g["passed"][i])
        assert m["max_abs_error"] == pytest.approx(float(g["max_abs"][i]), rel=1e-12)
        assert m["relative_l2_error"] == pytest.approx(float(g["rel_l2"][i]), rel=1e-9)


def test_oracle_against_reference_build(oracle):
    """When the reference's AVX kernel is built (oracle/_ref), the C oracle agrees with it."""
    if not oracle.ReferenceAVX.available():
        pytest.skip("oracle/_ref not built")
    ref = oracle.ReferenceAVX()
    rng = np.random.default_rng(5)
    k, n = 1536, 640
    q = rng.integers(0, 16, (k, n), dtype=np.uint8)
    s = oracle.bf16_bits(rng.uniform(0.002, 0.02, (k // 128, n)))
    z = rng.integers(0, 16, (k // 128, n), dtype=np.uint8)
    p = oracle.pack(q, s, z)
    x = oracle.bf16_bits(rng.standard_normal(k))
    _, y16 = oracle.gemv(p, k, n, x[None])
    assert_bf16_close(y16[0], ref.gemv(x, p, k, n, threads=2), min_equal=0.98, what="oracle vs reference AVX")


@pytest.mark.parametrize("addends", [2, 1, 0])
def test_residual_norm_matches_reference_test_formula(oracle, addends):
    """The oracle's layer boundary against the expected values of the reference's own boundary test,
    evaluated in torch fp32 exactly as that test writes them (kernels/gpu/tests/test_gpu_ffn.cpp:262-268):
    x = bf16(x + a + b), normed = x * rsqrt(mean(x^2) + eps) * weight. The same RMSNorm is the
    reference model's CPU path (src/unified_llm_w4a16_hetero/unified_llm_w4a16.cpp:543-563)."""
    import torch

    g = torch.Generator().manual_seed(40 + addends)
    m, h, eps = 96, 4096, 1e-5
    rnd = lambda: torch.randn(m, h, generator=g).to(torch.bfloat16)  # noqa: E731
    x, a, b = rnd(), rnd(), rnd()
    weight = (torch.randn(h, generator=g) * 0.2 + 1.0).to(torch.bfloat16)
    expected_x = x.float() + (a.float() if addends > 0 else 0) + (b.float() if addends > 1 else 0)
    rounded_x = expected_x.to(torch.bfloat16).float()
    expected = rounded_x * (rounded_x.square().mean(-1, keepdim=True) + eps).rsqrt() * weight.float()

    bits = lambda t: t.view(torch.int16).numpy().view(np.uint16)  # noqa: E731
    got_x, got_n = oracle.residual_norm(bits(x), [bits(a), bits(b)][:addends], bits(weight), eps)
    assert np.array_equal(got_x, bits(rounded_x.to(torch.bfloat16)))
    assert_bf16_close(got_n, bits(expected.to(torch.bfloat16)), min_equal=0.999, what="oracle normed vs reference formula")
    assert_close(oracle.bf16_to_f32(got_n), expected.numpy(), (1e-2, 5e-3, 0.99999), "EXACT tolerance of the reference test")
    # without a weight the boundary only adds: normed carries x
    x2, n2 = oracle.residual_norm(bits(x), [bits(a)], None, eps)
    assert np.array_equal(x2, n2)
