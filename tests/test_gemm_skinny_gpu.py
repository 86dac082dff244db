"""GPU parity of the swap-AB GEMM for 17 to 128 rows (gemm_w4a16_skinny.cu): the dequantized weights are
the tcgen05 MMA's A operand in TMEM and the x tile its B operand. Like the other GEMMs it rounds each
dequantized weight to bf16 (the reference GEMM's bf16((q - z) * s), src/hipkernels/w4a16_gemm_packed.cu:491-497),
so it is compared with the oracle under the LEVEL tolerance of the reference's tests
(kernels/gpu/tests/test_gpu_ffn.cpp:35-36, 112). hmb_w4a16_gemm (no workspace) runs it on whole column
blocks; hmb_w4a16_ffn (with a workspace) cuts the (block, K step) units into equal shares per SM and
adds the parts of split blocks in a fixed order, which these tests check against the oracle and for
bit-identical repeats. The shapes cover even and odd numbers of 128-column blocks, and a blocked
gate/up layout whose gate half is an odd number of 64-channel tiles (which only this kernel takes)."""
import numpy as np
import pytest
import torch

import heteromega_b200 as H
from heteromega_b200 import _lib
from heteromega_b200.torch_ops import device_status, gemm_plan, ops
from heteromega_b200.weights import synthetic_packed_device
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


def bits_of(t):
    return t.cpu().view(torch.int16).numpy().view(np.uint16)


@pytest.mark.parametrize("m", [17, 40, 64, 100, 128])
def test_skinny_plan(cuda, m):
    for ws in (False, True):
        plan = gemm_plan(m, 8192, 57344, _lib.HMB_EPI_SWIGLU, ws)
        assert plan["kernel"] == "skinny" and plan["streamk"] == ws, plan
    assert gemm_plan(129, 8192, 57344)["kernel"] == "pair"
    assert gemm_plan(16, 8192, 57344)["kernel"] != "skinny"


@pytest.mark.parametrize("k,n", [(256, 128), (2048, 1024), (4096, 640)])
@pytest.mark.parametrize("m", [17, 64, 100, 128])
def test_skinny_gemm_matches_oracle(cuda, oracle, k, n, m):
    p = rand_matrix(oracle, k, n, seed=k + 3 * n)
    x = oracle.bf16_bits(np.random.default_rng(m + 5).standard_normal((m, k)))
    y32, _ = oracle.gemv(p, k, n, x)
    y = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device=cuda)
    ops.w4a16_gemm(y, dev16(x, cuda), torch.from_numpy(p).to(cuda), k, n, k, n, 0, 0, 0)
    torch.cuda.synchronize()
    assert device_status(cuda) == 0
    assert_close(y.float().cpu().numpy(), y32, LEVEL, f"skinny gemm k={k} n={n} m={m}")


@pytest.mark.parametrize("c", [1024, 576])  # 16 and 9 column blocks
@pytest.mark.parametrize("layout", [0, 1])
@pytest.mark.parametrize("m", [33, 128])
def test_skinny_swiglu(cuda, oracle, layout, m, c):
    h = 2048
    p = rand_matrix(oracle, h, 2 * c, seed=70 + layout)
    x = oracle.bf16_bits(np.random.default_rng(71).standard_normal((m, h)))
    _, gu = oracle.gemv(p, h, 2 * c, x)
    act_ref = oracle.bf16_to_f32(oracle.silu_mul(gu, c, layout))
    act = torch.empty(m, c, dtype=torch.bfloat16, device=cuda)
    ops.w4a16_gemm(act, dev16(x, cuda), torch.from_numpy(p).to(cuda), h, 2 * c, h, 2 * c, 0, 1, layout)
    torch.cuda.synchronize()
    assert device_status(cuda) == 0
    assert_close(act.float().cpu().numpy(), act_ref, LEVEL, f"skinny swiglu layout={layout} m={m} c={c}")


def test_skinny_leading_block_start_col_fp32_fp16(cuda, oracle):
    pk, pn = 4096, 1280
    p = rand_matrix(oracle, pk, pn, seed=81)
    pd = torch.from_numpy(p).to(cuda)
    for k, n, start, m in ((2048, 512, 0, 50), (4096, 256, 1024, 96), (3072, 1024, 256, 17)):
        x = oracle.bf16_bits(np.random.default_rng(k + n).standard_normal((m, k)))
        y32, _ = oracle.gemv(p, pk, pn, x, n=n, k=k, n0=start)
        y = torch.empty(m, n, dtype=torch.bfloat16, device=cuda)
        ops.w4a16_gemm(y, dev16(x, cuda), pd, k, n, pk, pn, start, 0, 0)
        yf = torch.empty(m, n, dtype=torch.float32, device=cuda)
        ops.w4a16_gemm(yf, dev16(x, cuda), pd, k, n, pk, pn, start, 0, 0)
        torch.cuda.synchronize()
        assert_close(y.float().cpu().numpy(), y32, LEVEL, f"block {k}x{n}@{start} m={m}")
        assert_close(yf.cpu().numpy(), y32, LEVEL, f"fp32 block {k}x{n}@{start} m={m}")
        assert torch.equal(yf.to(torch.bfloat16), y)
    k, n, m = 2048, 768, 64
    w = oracle.dequant(p, pk, pn, k, n).astype(np.float64)
    xh = np.random.default_rng(9).standard_normal((m, k)).astype(np.float16)
    yh = torch.empty(m, n, dtype=torch.float16, device=cuda)
    ops.w4a16_gemm(yh, torch.from_numpy(xh).to(cuda), pd, k, n, pk, pn, 0, 0, 0)
    torch.cuda.synchronize()
    assert device_status(cuda) == 0
    assert_close(yh.float().cpu().numpy(), xh.astype(np.float64) @ w, LEVEL, "fp16 skinny")


@pytest.mark.parametrize("m", [17, 64, 128])
def test_skinny_streamk_llama70b_ffn(cuda, oracle, m):
    """The Llama-3-70B FFN layer at decode batch sizes through hmb_w4a16_ffn: gate/up (448 column blocks
    x 128 K steps) and down (64 blocks x 448 steps, every block split between CTAs) in stream-K shares.
    Sampled rows against the oracle FFN; a second call gives the same bits (counters reset, fixed
    summation order)."""
    h, inter = 8192, 28672
    assert gemm_plan(m, inter, h, 0, True)["streamk"]
    gen = torch.Generator(device=cuda)
    gen.manual_seed(1000)
    gu = synthetic_packed_device(h, 2 * inter, cuda, gen)
    dn = synthetic_packed_device(inter, h, cuda, gen)
    w = H.FfnSliceWeights(gu, dn, 0, inter, h, H.GateUpLayout.kInterleaved)
    x = torch.randn(m, h, device=cuda, generator=gen).to(torch.bfloat16)
    y1 = torch.empty(m, h, dtype=torch.bfloat16, device=cuda)
    y2 = torch.empty_like(y1)
    H.gpu_ffn_slice_forward(w, x, None, y1)
    H.gpu_ffn_slice_forward(w, x, None, y2)
    torch.cuda.synchronize()
    assert device_status(cuda) == 0
    assert torch.equal(y1, y2), "stream-K results depend on the call"
    rows = np.unique(np.r_[0, m - 1, np.random.default_rng(m).integers(0, m, 3)])
    _, ref32 = oracle.ffn(gu.cpu().numpy(), dn.cpu().numpy(), h, inter, inter, 1, bits_of(x[torch.from_numpy(rows).to(cuda)]))
    assert_close(y1.float().cpu().numpy()[rows], ref32, LEVEL, f"70B FFN m={m}")
