"""GPU parity of the tcgen05 prefill GEMM (hmb_w4a16_gemm) against the CPU oracle. The GEMM rounds
each dequantized weight to bf16 before the MMA (as the reference GEMM does, w4a16_gemm_packed.cu:491-497),
so it is compared with the oracle's fp32 result under the reference tests' LEVEL tolerance
(kernels/gpu/tests/test_gpu_ffn.cpp:35-36, 112)."""
import numpy as np
import pytest
import torch

import heteromega_b200 as H
from heteromega_b200 import _lib
from heteromega_b200.torch_ops import device_status, ops
from heteromega_b200.weights import synthetic_layer, synthetic_packed_device
from metrics import LEVEL, assert_close

pytestmark = pytest.mark.gpu


def rand_matrix(oracle, k, n, seed):
    rng = np.random.default_rng(seed)
    q = rng.integers(0, 16, (k, n), dtype=np.uint8)
    s = oracle.bf16_bits(rng.uniform(0.002, 0.02, (k // 128, n)))
    z = rng.integers(0, 16, (k // 128, n), dtype=np.uint8)
    return oracle.pack(q, s, z)


def dev16(bits, dev):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).to(dev)


def f32_of(t):
    return t.float().cpu().numpy()


@pytest.mark.parametrize("k,n", [(256, 256), (2048, 1024), (4096, 512)])
@pytest.mark.parametrize("m", [17, 128, 129, 300])
def test_gemm_matches_oracle(cuda, oracle, k, n, m):
    p = rand_matrix(oracle, k, n, seed=k * 7 + n)
    x = oracle.bf16_bits(np.random.default_rng(m).standard_normal((m, k)))
    y32, _ = oracle.gemv(p, k, n, x)
    y = torch.empty(m, n, dtype=torch.bfloat16, device=cuda)
    ops.w4a16_gemm(y, dev16(x, cuda), torch.from_numpy(p).to(cuda), k, n, k, n, 0, 0, 0)
    torch.cuda.synchronize()
    assert device_status(cuda) == 0
    assert_close(f32_of(y), y32, LEVEL, f"gemm k={k} n={n} m={m}")


@pytest.mark.parametrize("layout", [0, 1])
@pytest.mark.parametrize("m", [64, 200])
def test_gemm_swiglu_epilogue(cuda, oracle, layout, m):
    h, c = 2048, 1024
    p = rand_matrix(oracle, h, 2 * c, seed=30 + layout)
    x = oracle.bf16_bits(np.random.default_rng(31).standard_normal((m, h)))
    _, gu = oracle.gemv(p, h, 2 * c, x)
    act_ref = oracle.bf16_to_f32(oracle.silu_mul(gu, c, layout))
    act = torch.empty(m, c, dtype=torch.bfloat16, device=cuda)
    ops.w4a16_gemm(act, dev16(x, cuda), torch.from_numpy(p).to(cuda), h, 2 * c, h, 2 * c, 0, 1, layout)
    torch.cuda.synchronize()
    assert device_status(cuda) == 0
    assert_close(f32_of(act), act_ref, LEVEL, f"gemm swiglu layout={layout} m={m}")


def test_gemm_leading_block_and_start_col(cuda, oracle):
    pk, pn = 4096, 1280  # 20 tile columns: uneven modulo-8 groups
    p = rand_matrix(oracle, pk, pn, seed=41)
    pd = torch.from_numpy(p).to(cuda)
    for k, n, start in ((2048, 512, 0), (4096, 256, 1024), (1024, 768, 256), (3072, 1024, 256)):
        m = 150
        x = oracle.bf16_bits(np.random.default_rng(k + n).standard_normal((m, k)))
        y32, _ = oracle.gemv(p, pk, pn, x, n=n, k=k, n0=start)
        y = torch.empty(m, n, dtype=torch.bfloat16, device=cuda)
        ops.w4a16_gemm(y, dev16(x, cuda), pd, k, n, pk, pn, start, 0, 0)
        torch.cuda.synchronize()
        assert_close(f32_of(y), y32, LEVEL, f"block {k}x{n}@{start}")
    assert device_status(cuda) == 0


def test_gemm_fp16_activations(cuda, oracle):
    k, n, m = 2048, 768, 130
    p = rand_matrix(oracle, k, n, seed=51)
    w = oracle.dequant(p, k, n).astype(np.float64)
    x = np.random.default_rng(52).standard_normal((m, k)).astype(np.float16)
    y = torch.empty(m, n, dtype=torch.float16, device=cuda)
    ops.w4a16_gemm(y, torch.from_numpy(x).to(cuda), torch.from_numpy(p).to(cuda), k, n, k, n, 0, 0, 0)
    torch.cuda.synchronize()
    assert device_status(cuda) == 0
    assert_close(y.float().cpu().numpy(), x.astype(np.float64) @ w, LEVEL, "fp16 gemm")


def test_gemm_fp32_output(cuda, oracle):
    """Unrounded fp32 sums (the tensor-parallel partials): within the bf16-weight error of the oracle."""
    k, n, m = 4096, 512, 200
    p = rand_matrix(oracle, k, n, seed=61)
    x = oracle.bf16_bits(np.random.default_rng(62).standard_normal((m, k)))
    y32, _ = oracle.gemv(p, k, n, x)
    y = torch.empty(m, n, dtype=torch.float32, device=cuda)
    ops.w4a16_gemm(y, dev16(x, cuda), torch.from_numpy(p).to(cuda), k, n, k, n, 0, 0, 0)
    yb = torch.empty(m, n, dtype=torch.bfloat16, device=cuda)
    ops.w4a16_gemm(yb, dev16(x, cuda), torch.from_numpy(p).to(cuda), k, n, k, n, 0, 0, 0)
    torch.cuda.synchronize()
    assert_close(y.cpu().numpy(), y32, LEVEL, "gemm fp32 out")
    # the bf16 output is the fp32 one rounded
    assert torch.equal(y.to(torch.bfloat16), yb)


def test_gemm_rejects_unsupported_width(cuda, oracle):
    p = torch.zeros(H.gpu_ffn.packed_bytes(128, 192), dtype=torch.uint8, device=cuda)
    x = torch.zeros(32, 128, dtype=torch.bfloat16, device=cuda)
    y = torch.zeros(32, 192, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(H.HmbError):
        ops.w4a16_gemm(y, x, p, 128, 192, 128, 192, 0, 0, 0)


@pytest.mark.parametrize("m", [64, 128, 256, 512, 2048])
def test_prefill_ffn_layer_sampled_rows(cuda, oracle, m):
    """The Llama-3.2-1B FFN layer at prefill sizes through gpu_ffn_slice_forward (GEMM
    path; K split across CTA pairs where the output tiles alone would leave the GPU idle: the down
    projection below M=2048, gate/up at M=64), checked on sampled rows against the oracle FFN."""
    hidden, inter = 2048, 8192
    gen = torch.Generator(device=cuda)
    gen.manual_seed(1000)
    gu = synthetic_packed_device(hidden, 2 * inter, cuda, gen)
    dn = synthetic_packed_device(inter, hidden, cuda, gen)
    w = H.FfnSliceWeights(gu, dn, 0, inter, hidden, H.GateUpLayout.kInterleaved)
    x = oracle.bf16_bits(np.random.default_rng(7).standard_normal((m, hidden)))
    y = torch.empty(m, hidden, dtype=torch.bfloat16, device=cuda)
    H.gpu_ffn_slice_forward(w, dev16(x, cuda), None, y)
    torch.cuda.synchronize()
    assert device_status(cuda) == 0
    rows = np.unique(np.r_[0, m - 1, np.random.default_rng(3).integers(0, m, 4)])
    _, ref32 = oracle.ffn(gu.cpu().numpy(), dn.cpu().numpy(), hidden, inter, inter, 1, x[rows])
    assert_close(f32_of(y)[rows], ref32, LEVEL, f"prefill FFN m={m}")
