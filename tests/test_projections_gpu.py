"""The attention projections of the BASELINE models on the same packed GEMV/GEMM (packed_linear, the
reference's QuantizedLinear path: the GEMV for decode, the GEMM for prefill,
src/unified_llm_w4a16_hetero/unified_llm_w4a16.cpp:1053-1066), at their full shapes, against the CPU
oracle on 128-column windows (the oracle's full product at these sizes would take minutes on the
CPU) at the reference tests' LEVEL tolerance. The fused qkv matrix of the Qwen writer puts q, k and
v output columns side by side; a window across the q/k boundary checks that too."""
import numpy as np
import pytest
import torch

import heteromega_b200 as H
from heteromega_b200.torch_ops import device_status
from heteromega_b200.weights import synthetic_packed_device
from metrics import LEVEL, assert_close

pytestmark = pytest.mark.gpu

# (model, K, N, name): q, k/v, o and fused qkv of Llama-3-70B, Llama-3.1-8B and Qwen2.5-14B
SHAPES = [("70b", 8192, 8192, "q"), ("70b", 8192, 1024, "k"), ("70b", 8192, 8192, "o"), ("70b", 8192, 10240, "qkv"),
          ("8b", 4096, 1024, "v"), ("qwen14b", 5120, 5120, "q"), ("qwen14b", 5120, 7168, "qkv")]


@pytest.mark.parametrize("model,k,n,name", SHAPES)
@pytest.mark.parametrize("m", [1, 16, 300])
def test_projection_windows(cuda, oracle, model, k, n, name, m):
    gen = torch.Generator(device=cuda).manual_seed(k + n + m)
    packed = synthetic_packed_device(k, n, cuda, gen)
    x = torch.randn(m, k, device=cuda, generator=gen).to(torch.bfloat16)
    y = torch.empty(m, n, dtype=torch.bfloat16, device=cuda)
    H.packed_linear(y, x, packed, k, n)
    torch.cuda.synchronize()
    assert device_status(cuda) == 0
    p = packed.cpu().numpy()
    xb = x.cpu().view(torch.int16).numpy().view(np.uint16)
    got = y.float().cpu().numpy()
    # first, last and (for qkv) the window across the q | k boundary
    starts = {0, n - 128} | ({k - 64} if name == "qkv" else set())
    for n0 in sorted(starts):
        ref, _ = oracle.gemv(p, k, n, xb, n=128, n0=n0)
        assert_close(got[:, n0:n0 + 128], ref, LEVEL, f"{model} {name} [{k}x{n}] m={m} columns {n0}..{n0 + 127}")
