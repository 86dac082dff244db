"""The layer boundary on one GPU (hmb_residual_norm) against the CPU oracle: x = bf16((x + a) + b) bit
for bit, normed within one bf16 rounding of the oracle (the kernel's sum of squares runs in another
order), as the reference's own boundary test checks it (kernels/gpu/tests/test_gpu_ffn.cpp:255-297:
2, 1 and 0 addends, kExact)."""
import numpy as np
import pytest
import torch

from metrics import EXACT, assert_bf16_close, assert_close

pytestmark = pytest.mark.gpu


def _bits(t):
    return t.cpu().view(torch.int16).numpy().view(np.uint16)


def _case(dev, m, h, seed, scale=1.0):
    g = torch.Generator(device=dev).manual_seed(seed)
    rnd = lambda: (torch.randn(m, h, device=dev, generator=g) * scale).to(torch.bfloat16)  # noqa: E731
    w = (torch.randn(h, device=dev, generator=g) * 0.2 + 1.0).to(torch.bfloat16)
    return rnd(), rnd(), rnd(), w


@pytest.mark.parametrize("m,h", [(1, 2048), (7, 8192), (512, 4096), (300, 5120), (33, 16384), (5, 8)])
@pytest.mark.parametrize("addends", [2, 1, 0])
def test_residual_norm_matches_oracle(cuda, oracle, m, h, addends):
    from heteromega_b200.torch_ops import ops

    x, a, b, w = _case(cuda, m, h, 100 + m + addends)
    x0 = _bits(x)
    normed = torch.empty_like(x)
    ops.residual_norm(x, a if addends > 0 else None, b if addends > 1 else None, w, normed, 1e-5)
    torch.cuda.synchronize()
    ref_x, ref_n = oracle.residual_norm(x0, [_bits(a), _bits(b)][:addends], _bits(w), 1e-5)
    assert np.array_equal(_bits(x), ref_x), "x must be the one-rounding sum, bit for bit"
    assert_bf16_close(_bits(normed), ref_n, min_equal=0.99, what=f"normed m={m} h={h} addends={addends}")
    assert_close(oracle.bf16_to_f32(_bits(normed)), oracle.bf16_to_f32(ref_n), EXACT, "normed, EXACT tolerance")


def test_residual_norm_strided_and_without_weight(cuda, oracle):
    from heteromega_b200.torch_ops import ops

    m, h = 64, 2048
    big = torch.randn(m, 3 * h, device=cuda).to(torch.bfloat16)
    x, a = big[:, :h], big[:, h:2 * h]  # row stride 3h
    x0, a0 = _bits(x.contiguous()), _bits(a.contiguous())
    out = torch.empty(m, 2 * h, dtype=torch.bfloat16, device=cuda)[:, :h]
    ops.residual_norm(x, a, None, None, out, 1e-5)
    torch.cuda.synchronize()
    ref_x, ref_n = oracle.residual_norm(x0, [a0], None, 1e-5)
    assert np.array_equal(_bits(x.contiguous()), ref_x)
    assert np.array_equal(_bits(out.contiguous()), ref_n)  # no weight: out is the new x


def test_residual_norm_graph_replay_is_deterministic(cuda):
    from heteromega_b200.torch_ops import ops

    x, a, b, w = _case(cuda, 256, 8192, 9)
    x_start = x.clone()
    n1, n2 = torch.empty_like(x), torch.empty_like(x)
    ops.residual_norm(x, a, b, w, n1, 1e-5)
    x1 = x.clone()
    x.copy_(x_start)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        ops.residual_norm(x, a, b, w, n2, 1e-5)
    x.copy_(x_start)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(x, x1) and torch.equal(n1, n2)


def test_residual_norm_rejects(cuda):
    import ctypes

    from heteromega_b200 import _lib
    from heteromega_b200._lib import lib

    x = torch.zeros(4, 64, dtype=torch.bfloat16, device=cuda)
    s = torch.cuda.current_stream().cuda_stream
    p = x.data_ptr()
    f = ctypes.c_float(1e-5)
    assert lib().hmb_residual_norm(p, 64, None, 0, p, 64, None, None, 0, 4, 64, f, s) == _lib.HMB_ERR_ARG  # b without a
    assert lib().hmb_residual_norm(p, 64, None, 0, None, 0, None, p, 64, 4, 60, f, s) == _lib.HMB_ERR_ARG  # h % 8
    assert lib().hmb_residual_norm(p, 64, None, 0, None, 0, None, p, 64, 4, 16392, f, s) == _lib.HMB_ERR_ARG  # h too big
    assert lib().hmb_residual_norm(p + 2, 64, None, 0, None, 0, None, p, 64, 4, 64, f, s) == _lib.HMB_ERR_ALIGN
    assert lib().hmb_residual_norm(p, 60, None, 0, None, 0, None, p, 64, 4, 56, f, s) == _lib.HMB_ERR_ALIGN  # ldx % 8
