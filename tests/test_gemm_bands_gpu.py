"""GPU parity of the CTA-pair GEMM's banded tile order, the schedule behind the prefill benchmark.

The pair kernel walks its 256 x 256 output tiles in bands: a band of row blocks whose x stays in L2
while the weight column blocks stream past it, or the mirror image with a band of weight column blocks
(gemm_w4a16_pair.cu, pair_band_order). A shape only gets more than one band when one operand's band
exceeds the 48 MB L2 budget, which no small test shape does. These tests run shapes that do, in both
forms and with a short last band, and the exact Llama-3-70B FFN GEMMs of the default benchmark
(gate/up K=8192 N=57344 with the SwiGLU epilogue at M=4096 and 8192, down K=28672 N=8192 at M=8192), and
the 70B stack's host call, which runs 4096-row chunks. Every check compares sampled rows, at least one in
each 256-row block and spread over both CTAs of a pair, across the full width against the CPU oracle
under the reference tests' LEVEL tolerance (kernels/gpu/tests/test_gpu_ffn.cpp:35-36, 112), and reads
the device status word after the call."""
import numpy as np
import pytest
import torch

import heteromega_b200 as H
from heteromega_b200 import _lib
from heteromega_b200.stack import FfnStack
from heteromega_b200.torch_ops import device_status, gemm_plan, ops
from heteromega_b200.weights import synthetic_packed_device
from metrics import LEVEL, assert_close

pytestmark = pytest.mark.gpu

L2_BUDGET = 48.0 * 1024 * 1024  # bytes of one operand's band kept in L2 (pair_band_order)


def band_order(m, k, n):
    """The band choice restated: (band_rows, band) minimising DRAM bytes ~ one operand once plus the
    other once per band of the first."""
    mb, nb = (m + 255) // 256, n // 256
    xrow, wcol = 256.0 * k * 2, k * 256 * 4352 / (128 * 64)
    gm = max(1, min(mb, int(L2_BUDGET / xrow)))
    gn = max(1, min(nb, int(L2_BUDGET / wcol)))
    rows = mb * xrow + -(-mb // gm) * nb * wcol
    cols = nb * wcol + -(-nb // gn) * mb * xrow
    return (True, gm) if rows <= cols else (False, gn)


def sample_rows(m, seed):
    """One row in each 256-row block, alternating between the two CTAs' 128-row halves, plus the last."""
    rng = np.random.default_rng(seed)
    rows = [256 * b + 128 * (b % 2) + int(rng.integers(0, 128)) for b in range((m + 255) // 256)]
    return np.unique(np.minimum(np.r_[rows, m - 1], m - 1))


def bits_of(t):
    return t.cpu().view(torch.int16).numpy().view(np.uint16)


def f32_of(t):
    return t.float().cpu().numpy()


def draw(m, k, cuda, seed):
    gen = torch.Generator(device=cuda)
    gen.manual_seed(seed)
    return torch.randn(m, k, device=cuda, generator=gen).to(torch.bfloat16)


@pytest.mark.parametrize("m,k,n,want", [
    (1024, 28672, 3328, (True, 3)),    # row bands of 3 then 1 row block
    (2560, 28672, 3328, (False, 12)),  # column bands of 12 then 1 column block
])
def test_banded_gemm_short_last_band(cuda, oracle, m, k, n, want):
    plan = gemm_plan(m, k, n, _lib.HMB_EPI_STORE)
    assert plan["kernel"] == "pair"
    assert (plan["band_rows"], plan["band"]) == want == band_order(m, k, n)
    blocks = (m + 255) // 256 if want[0] else n // 256
    assert blocks > want[1] and blocks % want[1] != 0  # several bands, the last one short
    gen = torch.Generator(device=cuda)
    gen.manual_seed(k + n)
    packed = synthetic_packed_device(k, n, cuda, gen)
    x = draw(m, k, cuda, seed=m)
    y = torch.empty(m, n, dtype=torch.bfloat16, device=cuda)
    ops.w4a16_gemm(y, x, packed, k, n, k, n, 0, _lib.HMB_EPI_STORE, 1)
    torch.cuda.synchronize()
    assert device_status(cuda) == 0
    rows = sample_rows(m, seed=n)
    ref32, _ = oracle.gemv(packed.cpu().numpy(), k, n, bits_of(x[rows]))
    assert_close(f32_of(y[rows]), ref32, LEVEL, f"banded gemm m={m} k={k} n={n} plan={plan}")


@pytest.mark.parametrize("m", [4096, 8192])
def test_llama70b_gate_up_swiglu_bands(cuda, oracle, m):
    """The default benchmark's dominant kernel: 70B gate/up (interleaved, SwiGLU) over every band."""
    h, inter = 8192, 28672
    plan = gemm_plan(m, h, 2 * inter, _lib.HMB_EPI_SWIGLU)
    assert plan["kernel"] == "pair" and (plan["band_rows"], plan["band"]) == band_order(m, h, 2 * inter)
    assert plan["band_rows"] and plan["band"] == 12 and (m // 256) > plan["band"]
    gen = torch.Generator(device=cuda)
    gen.manual_seed(1000)
    gate_up = synthetic_packed_device(h, 2 * inter, cuda, gen)
    x = draw(m, h, cuda, seed=7)
    act = torch.empty(m, inter, dtype=torch.bfloat16, device=cuda)
    ops.w4a16_gemm(act, x, gate_up, h, 2 * inter, h, 2 * inter, 0, _lib.HMB_EPI_SWIGLU, _lib.HMB_GATE_UP_INTERLEAVED)
    torch.cuda.synchronize()
    assert device_status(cuda) == 0
    rows = sample_rows(m, seed=m + 1)
    _, gu = oracle.gemv(gate_up.cpu().numpy(), h, 2 * inter, bits_of(x[rows]))
    ref = oracle.bf16_to_f32(oracle.silu_mul(gu, inter, _lib.HMB_GATE_UP_INTERLEAVED))
    assert_close(f32_of(act[rows]), ref, LEVEL, f"70B gate/up m={m} plan={plan}")


def test_llama70b_down_bands(cuda, oracle):
    """70B down at M=8192: column bands of 12, 12 and 8 weight column blocks."""
    m, k, n = 8192, 28672, 8192
    plan = gemm_plan(m, k, n, _lib.HMB_EPI_STORE)
    assert plan["kernel"] == "pair" and (plan["band_rows"], plan["band"]) == band_order(m, k, n) == (False, 12)
    gen = torch.Generator(device=cuda)
    gen.manual_seed(1001)
    down = synthetic_packed_device(k, n, cuda, gen)
    act = draw(m, k, cuda, seed=8)
    y = torch.empty(m, n, dtype=torch.bfloat16, device=cuda)
    ops.w4a16_gemm(y, act, down, k, n, k, n, 0, _lib.HMB_EPI_STORE, 1)
    torch.cuda.synchronize()
    assert device_status(cuda) == 0
    rows = sample_rows(m, seed=9)
    ref32, _ = oracle.gemv(down.cpu().numpy(), k, n, bits_of(act[rows]))
    assert_close(f32_of(y[rows]), ref32, LEVEL, f"70B down m={m} plan={plan}")


def test_llama70b_stack_host_call_chunks(cuda, oracle):
    """FfnStack.forward_host on two 70B layers at M=8192: two 4096-row chunks, each through the
    chained layers (boundary, gate/up, down) on its own graph, against the oracle's chain."""
    h, inter, m, L = 8192, 28672, 8192, 2
    gen = torch.Generator(device=cuda)
    layers, norms, host = [], [], []
    for l in range(L):
        gen.manual_seed(1000 + l)
        g = synthetic_packed_device(h, inter, cuda, gen)
        u = synthetic_packed_device(h, inter, cuda, gen)
        d = synthetic_packed_device(inter, h, cuda, gen)
        w = H.slice_packed_ffn(g, u, d, h, inter, 0, inter, H.GateUpLayout.kInterleaved)
        layers.append(w)
        host.append((w.gate_up.cpu().numpy(), w.down.cpu().numpy()))
        del g, u, d
        gen.manual_seed(2000 + l)
        norms.append((torch.randn(h, device=cuda, generator=gen) * 0.2 + 1.0).to(torch.bfloat16))
    stack = FfnStack(layers, h, cuda, norms=norms)
    h0 = draw(m, h, cuda, seed=7).cpu().pin_memory()
    out = torch.empty_like(h0).pin_memory()
    try:
        stack.forward_host(h0, out)
        torch.cuda.synchronize()
        assert device_status(cuda) == 0
    finally:
        stack.release()
    rows = np.unique(np.r_[sample_rows(m, seed=11)[::2], 4095, 4096])  # both chunks, both sides of the cut
    hb = bits_of(h0[rows])
    norm_bits = [bits_of(g) for g in norms]
    _, x = oracle.residual_norm(hb, [], norm_bits[0], 1e-5)
    for l in range(L):
        y16, _ = oracle.ffn(host[l][0], host[l][1], h, inter, inter, 1, x)
        last = l == L - 1
        hb, x = oracle.residual_norm(hb, [y16], None if last else norm_bits[l + 1], 1e-5, with_normed=not last)
    assert_close(f32_of(out[rows]), oracle.bf16_to_f32(hb), LEVEL, "70B stack host call, 2 layers, M=8192")
