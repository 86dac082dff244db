"""The allocation-free GEMV entry point, hmb_w4a16_gemv_noalloc, called through the C ABI.

It is meant for callers that cannot give this library device memory (a host runtime that owns the
memory pool and has no scratch API, or a plugin ABI that passes only inputs and outputs); it keeps
the GEMV's split-K scratch in a fixed device array instead. It runs the same kernel with the same
split as hmb_w4a16_gemv, which takes caller workspace, so over two calls in a row (the second call
reuses the array the first one left behind) its outputs must equal that entry point's bit for bit,
and, like every GEMV, match the CPU oracle: at least 97% of the bf16 outputs identical and none
further than one bf16 unit at the largest magnitude, the SwiGLU outputs within the LEVEL tolerance.
This file sorts last so that a run that stops at the first failure has run every other test before it."""
import numpy as np
import pytest
import torch

from heteromega_b200 import _lib
from heteromega_b200.torch_ops import ops
from metrics import LEVEL, assert_bf16_close, assert_close

pytestmark = pytest.mark.gpu


def _packed(rng, k, n):
    from oracle import oracle as O

    q = rng.integers(0, 16, (k, n), dtype=np.uint8)
    s = O.bf16_bits(rng.uniform(0.002, 0.02, (k // 128, n)))
    z = rng.integers(0, 16, (k // 128, n), dtype=np.uint8)
    return O.pack(q, s, z)


def _noalloc(out, x, packed, k, n, epilogue, layout):
    stream = torch.cuda.current_stream(x.device).cuda_stream
    rc = _lib.lib().hmb_w4a16_gemv_noalloc(packed.data_ptr(), k, n, x.data_ptr(), x.stride(0), _lib.HMB_BF16,
                                           out.data_ptr(), out.stride(0), _lib.HMB_BF16, x.shape[0], k, n, 0, epilogue,
                                           layout, 0, stream)
    _lib.check(rc, "hmb_w4a16_gemv_noalloc")


def _bits(t):
    return t.cpu().view(torch.int16).numpy().view(np.uint16)


@pytest.mark.parametrize("epilogue,k,n,m", [(0, 14336, 4096, 1), (1, 4096, 2 * 7168, 1), (0, 8192, 2048, 12)])
def test_noalloc_matches_workspace_gemv(cuda, oracle, epilogue, k, n, m):
    rng = np.random.default_rng(k + n + m)
    packed_host = _packed(rng, k, n)
    packed = torch.from_numpy(packed_host).to(cuda)
    cols = n // 2 if epilogue == _lib.HMB_EPI_SWIGLU else n
    for call in range(2):
        x = torch.randn(m, k, device=cuda).to(torch.bfloat16)
        ref = torch.empty(m, cols, dtype=torch.bfloat16, device=cuda)
        got = torch.full_like(ref, float("nan"))
        ops.w4a16_gemv(ref, x, packed, k, n, k, n, 0, epilogue, 1, 0)
        _noalloc(got, x, packed, k, n, epilogue, 1)
        torch.cuda.synchronize()
        assert np.array_equal(_bits(got), _bits(ref)), f"call {call}: differs from hmb_w4a16_gemv"
        y32, y16 = oracle.gemv(packed_host, k, n, _bits(x))
        if epilogue == _lib.HMB_EPI_SWIGLU:
            act = oracle.bf16_to_f32(oracle.silu_mul(y16, cols, 1))
            assert_close(got.float().cpu().numpy(), act, LEVEL, f"call {call}: SwiGLU vs oracle")
        else:
            assert_bf16_close(_bits(got), y16, min_equal=0.97, what=f"call {call}: vs oracle")


def test_noalloc_rejects_oversized_scratch(cuda):
    """A shape that needs more than the fixed array fails with HMB_ERR_WORKSPACE, before any launch."""
    k, n, m = 128, 64 * 16384, 16  # 16384 column sets of 16 rows: far beyond the array
    assert _lib.lib().hmb_w4a16_gemv_workspace(m, k, n, 0, 0) > (16 << 20) + (64 << 10)
    dummy = torch.zeros(16, dtype=torch.uint8, device=cuda)
    rc = _lib.lib().hmb_w4a16_gemv_noalloc(dummy.data_ptr(), k, n, dummy.data_ptr(), k, _lib.HMB_BF16, dummy.data_ptr(),
                                           n, _lib.HMB_BF16, m, k, n, 0, 0, 0, 0,
                                           torch.cuda.current_stream(cuda).cuda_stream)
    assert rc == -4
