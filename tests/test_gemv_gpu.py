"""GPU parity of the decode GEMV (hmb_w4a16_gemv) and the exact dequantization against the CPU
oracle. Shapes and splits follow kernels/gpu/tests/test_gpu_ffn.cpp:117-168."""
import numpy as np
import pytest
import torch

import heteromega_b200 as H
from heteromega_b200 import _lib
from heteromega_b200.torch_ops import ops
from metrics import LEVEL, assert_bf16_close, assert_close

pytestmark = pytest.mark.gpu


def rand_matrix(oracle, k, n, seed, zlo=0, zhi=16):
    rng = np.random.default_rng(seed)
    q = rng.integers(0, 16, (k, n), dtype=np.uint8)
    s = oracle.bf16_bits(rng.uniform(0.002, 0.02, (k // 128, n)))
    z = rng.integers(zlo, zhi, (k // 128, n), dtype=np.uint8)
    return oracle.pack(q, s, z)


def rand_x(oracle, m, k, seed, scale=1.0):
    rng = np.random.default_rng(seed)
    return oracle.bf16_bits(rng.standard_normal((m, k)) * scale)


def to_dev_bf16(bits, dev):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).to(dev)


def bits_of(t):
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


@pytest.mark.parametrize("k,n", [(256, 384), (2048, 640), (4096, 1024), (1024, 4096)])
@pytest.mark.parametrize("m", [1, 3, 8, 9, 16, 37])
def test_gemv_matches_oracle(cuda, oracle, k, n, m):
    p = rand_matrix(oracle, k, n, seed=k + n)
    x = rand_x(oracle, m, k, seed=m)
    _, y16 = oracle.gemv(p, k, n, x)
    y = torch.empty(m, n, dtype=torch.bfloat16, device=cuda)
    ops.w4a16_gemv(y, to_dev_bf16(x, cuda), torch.from_numpy(p).to(cuda), k, n, k, n, 0, 0, 0, 0)
    torch.cuda.synchronize()
    assert_bf16_close(bits_of(y), y16, min_equal=0.97, what=f"gemv k={k} n={n} m={m}")


@pytest.mark.parametrize("split", [0, 1, 2, 3, 8, 64])
def test_gemv_split_k(cuda, oracle, split):
    k, n = 14336 // 2, 512
    p = rand_matrix(oracle, k, n, seed=3)
    x = rand_x(oracle, 1, k, seed=4)
    y32, y16 = oracle.gemv(p, k, n, x)
    y = torch.empty(1, n, dtype=torch.bfloat16, device=cuda)
    H.gemv_w4a16(y, to_dev_bf16(x, cuda)[0], torch.from_numpy(p).to(cuda), k, n, k, n, split)
    torch.cuda.synchronize()
    assert_bf16_close(bits_of(y), y16, min_equal=0.97, what=f"split {split}")
    # fp32 output: unrounded sums
    y_f = torch.empty(1, n, dtype=torch.float32, device=cuda)
    ops.w4a16_gemv(y_f, to_dev_bf16(x, cuda), torch.from_numpy(p).to(cuda), k, n, k, n, 0, 0, 0, split)
    torch.cuda.synchronize()
    assert np.abs(y_f.cpu().numpy() - y32).max() <= 1e-5 * np.abs(y32).max()


def test_gemv_leading_block_and_start_col(cuda, oracle):
    """The leading [k, n] block of a larger packed matrix (FfnSliceWeights::prefix), and a column
    window (w4a16_gemv_fused_packed's start_col)."""
    pk, pn = 4096, 1216  # 19 tile columns: uneven modulo-8 groups
    p = rand_matrix(oracle, pk, pn, seed=11)
    pd = torch.from_numpy(p).to(cuda)
    for k, n, start in ((2048, 512, 0), (4096, 256, 0), (1024, 768, 0), (4096, 1152, 64), (3072, 320, 896)):
        for m in (1, 5):
            x = rand_x(oracle, m, k, seed=k + m)
            _, y16 = oracle.gemv(p, pk, pn, x, n=n, k=k, n0=start)
            y = torch.empty(m, n, dtype=torch.bfloat16, device=cuda)
            ops.w4a16_gemv(y, to_dev_bf16(x, cuda), pd, k, n, pk, pn, start, 0, 0, 0)
            torch.cuda.synchronize()
            assert_bf16_close(bits_of(y), y16, min_equal=0.97, what=f"block {k}x{n}@{start} m={m}")


@pytest.mark.parametrize("layout", [0, 1])
@pytest.mark.parametrize("m", [1, 4, 13])
def test_gemv_swiglu_epilogue(cuda, oracle, layout, m):
    h, c = 2048, 1536  # c channels: gate_up [h, 2c]
    p = rand_matrix(oracle, h, 2 * c, seed=21 + layout)
    x = rand_x(oracle, m, h, seed=22)
    _, gu = oracle.gemv(p, h, 2 * c, x)
    act_ref = oracle.silu_mul(gu, c, layout)
    act = torch.empty(m, c, dtype=torch.bfloat16, device=cuda)
    ops.w4a16_gemv(act, to_dev_bf16(x, cuda), torch.from_numpy(p).to(cuda), h, 2 * c, h, 2 * c, 0, 1, layout, 0)
    torch.cuda.synchronize()
    assert_bf16_close(bits_of(act), act_ref, min_equal=0.97, what=f"swiglu layout={layout} m={m}")


def test_gemv_fp16_activations(cuda, oracle):
    """fp16 x (the BASELINE's activation type): checked against fp64 math on the oracle's exact
    dequantized weights, fed the same fp16 values."""
    k, n, m = 4096, 1024, 3
    p = rand_matrix(oracle, k, n, seed=31)
    w = oracle.dequant(p, k, n).astype(np.float64)
    x = np.random.default_rng(32).standard_normal((m, k)).astype(np.float16)
    ref = x.astype(np.float64) @ w
    y = torch.empty(m, n, dtype=torch.float16, device=cuda)
    ops.w4a16_gemv(y, torch.from_numpy(x).to(cuda), torch.from_numpy(p).to(cuda), k, n, k, n, 0, 0, 0, 0)
    torch.cuda.synchronize()
    assert_close(y.float().cpu().numpy(), ref, LEVEL, "fp16 gemv")


def test_dequant_bit_exact(cuda, oracle):
    for pk, pn, k, n in ((512, 640, 512, 640), (1024, 1216, 768, 1152)):
        p = rand_matrix(oracle, pk, pn, seed=pk)
        ref = oracle.dequant(p, pk, pn, k, n)
        out = torch.empty(k, n, dtype=torch.float32, device=cuda)
        ops.w4a16_dequant(out, torch.from_numpy(p).to(cuda), k, n, pk, pn)
        torch.cuda.synchronize()
        assert np.array_equal(out.cpu().numpy(), ref)


def test_device_packer_and_tile_gather(cuda, oracle):
    rng = np.random.default_rng(41)
    k, n = 384, 1152
    q = torch.from_numpy(rng.integers(0, 16, (k, n), dtype=np.uint8))
    s = torch.from_numpy(rng.uniform(0.002, 0.02, (k // 128, n)).astype(np.float32)).to(torch.bfloat16)
    z = torch.from_numpy(rng.integers(0, 16, (k // 128, n), dtype=np.uint8))
    host = H.pack_w4a16(q, s, z)
    dev = H.pack_w4a16(q.to(cuda), s.to(cuda), z.to(cuda))
    assert torch.equal(dev.cpu(), host)
    q[3, 3] = 17
    with pytest.raises(ValueError):
        H.pack_w4a16(q.to(cuda), s.to(cuda), z.to(cuda))
    # slice_packed_ffn by device tile gather gives the host bytes
    hidden, inter = 384, 1152
    mats = [_packed(rng, hidden, inter), _packed(rng, hidden, inter), _packed(rng, inter, hidden)]
    for b, e in ((0, inter), (128, 640), (512, 1152)):
        for layout in (H.GateUpLayout.kBlocked, H.GateUpLayout.kInterleaved):
            h_w = H.slice_packed_ffn(*mats, hidden, inter, b, e, layout)
            d_w = H.slice_packed_ffn(*(t.to(cuda) for t in mats), hidden, inter, b, e, layout)
            assert torch.equal(d_w.gate_up.cpu(), h_w.gate_up) and torch.equal(d_w.down.cpu(), h_w.down)


def _packed(rng, k, n):
    q = torch.from_numpy(rng.integers(0, 16, (k, n), dtype=np.uint8))
    s = torch.from_numpy(rng.uniform(0.002, 0.02, (k // 128, n)).astype(np.float32)).to(torch.bfloat16)
    z = torch.from_numpy(rng.integers(0, 16, (k // 128, n), dtype=np.uint8))
    return H.pack_w4a16(q, s, z)


def test_silu_mul_and_residual_add2(cuda, oracle):
    rng = np.random.default_rng(51)
    for m in (1, 37, 256):
        n = 7168
        gu = oracle.bf16_bits(rng.standard_normal((m, 2 * n)) * 4.0)
        for layout in (0, 1):
            act = torch.empty(m, n, dtype=torch.bfloat16, device=cuda)
            H.silu_mul(to_dev_bf16(gu, cuda), act, layout=H.GateUpLayout(layout))
            torch.cuda.synchronize()
            assert_bf16_close(bits_of(act), oracle.silu_mul(gu, n, layout), min_equal=0.99,
                              what=f"silu_mul m={m} layout={layout}")
    for m in (1, 300):
        h = 4096
        x0 = oracle.bf16_bits(rng.standard_normal((m, h)))
        yg = oracle.bf16_bits(rng.standard_normal((m, h)) * 0.3)
        for yn in (oracle.bf16_bits(rng.standard_normal((m, h)) * 0.3), (rng.standard_normal((m, h)) * 0.3).astype(np.float32)):
            ref = oracle.residual_add2(x0, yg, yn)
            x = to_dev_bf16(x0, cuda)
            yn_d = to_dev_bf16(yn, cuda) if yn.dtype == np.uint16 else torch.from_numpy(yn).to(cuda)
            H.residual_add2(x, to_dev_bf16(yg, cuda), yn_d)
            torch.cuda.synchronize()
            assert np.array_equal(bits_of(x), ref)


def test_errors_raise(cuda, oracle):
    p = torch.zeros(4352, dtype=torch.uint8, device=cuda)
    x = torch.zeros(1, 128, dtype=torch.bfloat16, device=cuda)
    y = torch.zeros(1, 64, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(H.HmbError):
        ops.w4a16_gemv(y, x, p, 128, 64, 128, 64, 0, 1, 0, 0)  # SwiGLU needs 128-column pairs
    with pytest.raises(ValueError):
        ops.w4a16_gemv(y, x, p, 128, 64, 256, 64, 0, 0, 0, 0)  # packed size mismatch
