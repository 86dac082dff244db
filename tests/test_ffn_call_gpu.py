"""GPU parity of the one-call FFN (hmb_w4a16_ffn, the counterpart of heteromega::gemm_w4a16_ffn,
kernels/gpu/src/gemm_w4a16.cu:463-502): the decode path (gate/up GEMV + SwiGLU, then the down GEMV as a
programmatic dependent) for m <= 16 and per 16-row chunk, the two-GEMM path above, prefixes of the packed channels,
both gate/up layouts, fp16 activations, fp32 partial outputs, and repeated calls (the workspace's
counters and barrier reset themselves). Tolerance: the reference tests' LEVEL bound
(kernels/gpu/tests/test_gpu_ffn.cpp:35-36)."""
import numpy as np
import pytest
import torch

import heteromega_b200 as H
from heteromega_b200 import _lib
from heteromega_b200.torch_ops import device_status, ops
from heteromega_b200.weights import synthetic_layer
from metrics import LEVEL, assert_close

pytestmark = pytest.mark.gpu


def bf16_dev(bits, dev):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).to(dev)


@pytest.fixture(scope="module")
def layer_small():
    """H 1024, I 3072: small enough for many cases, large enough that column sets span warps."""
    hidden, inter = 1024, 3072
    layer = synthetic_layer(hidden, inter, layer=5)
    return hidden, inter, layer


def oracle_ffn(oracle, w, hidden, n, x):
    _, y32 = oracle.ffn(w.gate_up.numpy(), w.down.numpy(), hidden, n, w.stored_channels(), int(w.layout), x)
    return y32


@pytest.mark.parametrize("m", [1, 2, 5, 9, 16, 17, 40, 300])
def test_ffn_rows(cuda, oracle, layer_small, m):
    hidden, inter, layer = layer_small
    w = H.pack_ffn_slice(layer, 0, inter, H.GateUpLayout.kInterleaved)
    x = oracle.bf16_bits(np.random.default_rng(m).standard_normal((m, hidden)))
    ref = oracle_ffn(oracle, w, hidden, inter, x)
    wd = w.to(cuda)
    y = torch.empty(m, hidden, dtype=torch.bfloat16, device=cuda)
    ops.w4a16_ffn(y, bf16_dev(x, cuda), wd.gate_up, wd.down, hidden, inter, inter, 1)
    torch.cuda.synchronize()
    assert device_status(cuda) == _lib.HMB_OK
    assert_close(y.float().cpu().numpy(), ref, LEVEL, f"ffn m={m}")


@pytest.mark.parametrize("layout", [0, 1])
@pytest.mark.parametrize("m", [1, 7])
def test_ffn_prefix_and_layouts(cuda, oracle, layer_small, layout, m):
    """n < stored channels: interleaved takes a prefix; blocked finds the up columns at stored / 64."""
    hidden, inter, layer = layer_small
    w = H.pack_ffn_slice(layer, 0, inter, H.GateUpLayout(layout))
    n = 1920
    x = oracle.bf16_bits(np.random.default_rng(40 + m).standard_normal((m, hidden)))
    _, ref = oracle.ffn(w.gate_up.numpy(), w.down.numpy(), hidden, n, inter, layout, x)
    wd = w.to(cuda)
    y = torch.empty(m, hidden, dtype=torch.bfloat16, device=cuda)
    ops.w4a16_ffn(y, bf16_dev(x, cuda), wd.gate_up, wd.down, hidden, n, inter, layout)
    torch.cuda.synchronize()
    assert device_status(cuda) == _lib.HMB_OK
    assert_close(y.float().cpu().numpy(), ref, LEVEL, f"prefix n={n} layout={layout} m={m}")


def test_ffn_fp32_partials_and_repeats(cuda, oracle, layer_small):
    """fp32 output = the unrounded sums; ten calls in a row agree bit for bit."""
    hidden, inter, layer = layer_small
    w = H.pack_ffn_slice(layer, 0, inter, H.GateUpLayout.kInterleaved).to(cuda)
    m = 3
    x = oracle.bf16_bits(np.random.default_rng(9).standard_normal((m, hidden)))
    ref = oracle_ffn(oracle, w.to("cpu"), hidden, inter, x)
    xd = bf16_dev(x, cuda)
    outs = []
    for _ in range(10):
        y = torch.empty(m, hidden, dtype=torch.float32, device=cuda)
        ops.w4a16_ffn(y, xd, w.gate_up, w.down, hidden, inter, inter, 1)
        outs.append(y)
    torch.cuda.synchronize()
    assert device_status(cuda) == _lib.HMB_OK
    assert_close(outs[0].cpu().numpy(), ref, LEVEL, "fp32 partial")
    for o in outs[1:]:
        assert torch.equal(o, outs[0])


def test_ffn_fp16_activations(cuda, oracle, layer_small):
    hidden, inter, layer = layer_small
    w = H.pack_ffn_slice(layer, 0, inter, H.GateUpLayout.kInterleaved)
    m = 4
    x = np.random.default_rng(11).standard_normal((m, hidden)).astype(np.float16)
    # fp32 restatement fed the same fp16 values: dequantize, fp32 matmuls, fp16 rounding of gate/up and act
    wg = oracle.dequant(w.gate_up.numpy(), hidden, 2 * inter).astype(np.float64)
    gu = (x.astype(np.float64) @ wg).astype(np.float16).astype(np.float64)
    g = gu.reshape(m, inter // 64, 2, 64)[:, :, 0].reshape(m, inter)
    u = gu.reshape(m, inter // 64, 2, 64)[:, :, 1].reshape(m, inter)
    act = (g / (1 + np.exp(-g)) * u).astype(np.float16).astype(np.float64)
    ref = act @ oracle.dequant(w.down.numpy(), inter, hidden).astype(np.float64)
    wd = w.to(cuda)
    y = torch.empty(m, hidden, dtype=torch.float16, device=cuda)
    ops.w4a16_ffn(y, torch.from_numpy(x).to(cuda), wd.gate_up, wd.down, hidden, inter, inter, 1)
    torch.cuda.synchronize()
    assert_close(y.float().cpu().numpy(), ref, LEVEL, "fp16 ffn")


def test_ffn_graph_replay(cuda, oracle, layer_small):
    """Captured once, replayed: the two decode launches (the second a programmatic dependent) in a graph."""
    hidden, inter, layer = layer_small
    w = H.pack_ffn_slice(layer, 0, inter, H.GateUpLayout.kInterleaved).to(cuda)
    m = 1
    x = oracle.bf16_bits(np.random.default_rng(21).standard_normal((m, hidden)))
    ref = oracle_ffn(oracle, w.to("cpu"), hidden, inter, x)
    xd = bf16_dev(x, cuda)
    y = torch.empty(m, hidden, dtype=torch.bfloat16, device=cuda)
    s = torch.cuda.Stream(cuda)
    s.wait_stream(torch.cuda.current_stream(cuda))
    with torch.cuda.stream(s):
        ops.w4a16_ffn(y, xd, w.gate_up, w.down, hidden, inter, inter, 1)
    torch.cuda.current_stream(cuda).wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        ops.w4a16_ffn(y, xd, w.gate_up, w.down, hidden, inter, inter, 1)
    for _ in range(3):
        y.zero_()
        g.replay()
    torch.cuda.synchronize()
    assert device_status(cuda) == _lib.HMB_OK
    assert_close(y.float().cpu().numpy(), ref, LEVEL, "graph replay")
    g.reset()


def test_ffn_rejects_bad_arguments(cuda, layer_small):
    hidden, inter, layer = layer_small
    w = H.pack_ffn_slice(layer, 0, inter, H.GateUpLayout.kInterleaved).to(cuda)
    x = torch.zeros(2, hidden, dtype=torch.bfloat16, device=cuda)
    y = torch.zeros(2, hidden, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(H.HmbError):
        ops.w4a16_ffn(y, x, w.gate_up, w.down, hidden, inter + 128, inter, 1)  # n > stored
    with pytest.raises(H.HmbError):
        ops.w4a16_ffn(y, x, w.gate_up, w.down, hidden, 100, inter, 1)  # n not a multiple of 128
    with pytest.raises(H.HmbError):
        ops.w4a16_ffn(y, x, w.gate_up, w.down, hidden, inter, inter, 5)  # layout
