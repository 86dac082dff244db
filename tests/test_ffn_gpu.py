"""GPU parity of the FFN slice path against the CPU oracle, and the split/prefix/model algebra of
kernels/gpu/tests/test_gpu_ffn.cpp:443-509 (Level 2), plus full-size checks on sampled columns."""
import numpy as np
import pytest
import torch

import heteromega_b200 as H
from heteromega_b200 import _lib
from heteromega_b200.torch_ops import ops
from heteromega_b200.weights import synthetic_layer, synthetic_packed_device
from metrics import LEVEL, assert_bf16_close, assert_close

pytestmark = pytest.mark.gpu


def bf16_dev(bits, dev):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).to(dev)


def bits_of(t):
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


@pytest.fixture(scope="module")
def layer_8b():
    """A seeded Llama-3.1-8B-shaped layer (H 4096, I 14336), packed both ways."""
    hidden, inter = 4096, 14336
    layer = synthetic_layer(hidden, inter, layer=0, zero_range=(6, 10))
    all_i = H.pack_ffn_slice(layer, 0, inter, H.GateUpLayout.kInterleaved)
    return hidden, inter, layer, all_i


@pytest.mark.parametrize("m", [1, 4, 16])
def test_ffn_matches_oracle(cuda, oracle, layer_8b, m):
    hidden, inter, layer, all_i = layer_8b
    x = oracle.bf16_bits(np.random.default_rng(m).standard_normal((m, hidden)) * 0.5)
    y16_ref, y32_ref = oracle.ffn(all_i.gate_up.numpy(), all_i.down.numpy(), hidden, inter, inter, 1, x)
    w = all_i.to(cuda)
    y = torch.empty(m, hidden, dtype=torch.bfloat16, device=cuda)
    H.gpu_ffn_slice_forward(w, bf16_dev(x, cuda), None, y)
    torch.cuda.synchronize()
    got = oracle.bf16_to_f32(bits_of(y))
    assert_close(got, y32_ref, LEVEL, f"ffn m={m}")
    eq = np.mean(bits_of(y) == y16_ref)
    assert eq > 0.9, eq


@pytest.mark.parametrize("s", [512, 7168, 13824])
def test_split_partials_sum_to_full_ffn(cuda, oracle, layer_8b, s):
    hidden, inter, layer, all_i = layer_8b
    m = 3
    x = oracle.bf16_bits(np.random.default_rng(s).standard_normal((m, hidden)) * 0.5)
    _, y32_ref = oracle.ffn(all_i.gate_up.numpy(), all_i.down.numpy(), hidden, inter, inter, 1, x)
    xd = bf16_dev(x, cuda)
    gpu_part = H.pack_ffn_slice(layer, 0, s).to(cuda)
    npu_part = H.pack_ffn_slice(layer, s, inter).to(cuda)
    w_all = all_i.to(cuda)
    y_g, y_n, y_prefix = (torch.empty(m, hidden, dtype=torch.bfloat16, device=cuda) for _ in range(3))
    H.gpu_ffn_slice_forward(gpu_part, xd, None, y_g)
    H.gpu_ffn_slice_forward(npu_part, xd, None, y_n)
    H.gpu_ffn_slice_forward(w_all.prefix(s), xd, None, y_prefix)
    x_out = torch.zeros(m, hidden, dtype=torch.bfloat16, device=cuda)
    H.residual_add2(x_out, y_g, y_n)
    model = H.GpuFfnModel()
    g, u, d = (H.pack_w4a16(*t).to(cuda) for t in ((layer.gate_q, layer.gate_s, layer.gate_z),
                                                     (layer.up_q, layer.up_s, layer.up_z),
                                                     (layer.down_q, layer.down_s, layer.down_z)))
    model.add_layer(g, u, d, hidden, inter)
    model.set_split(s, s)
    y_model = torch.empty_like(y_g)
    model.forward(0, xd, y_model)
    torch.cuda.synchronize()
    assert_close(oracle.bf16_to_f32(bits_of(x_out)), y32_ref, LEVEL, f"Y_G + Y_N s={s}")
    # The prefix of the interleaved full packing is the blocked slice up to column order: same values.
    assert_close(y_prefix.float().cpu().numpy(), y_g.float().cpu().numpy(), (1e-2, 5e-3, 0.99999), "prefix vs slice")
    assert torch.equal(y_model, y_prefix), "GpuFfnModel must give the prefix's bytes"


def test_gemm_w4a16_ffn_api(cuda, oracle, layer_8b):
    hidden, inter, layer, all_i = layer_8b
    m, n = 5, 7168
    x = oracle.bf16_bits(np.random.default_rng(9).standard_normal((m, hidden)) * 0.5)
    _, y32_ref = oracle.ffn(all_i.gate_up.numpy(), all_i.down.numpy(), hidden, n, inter, 1, x)
    w = all_i.to(cuda)
    y = torch.empty(m, hidden, dtype=torch.bfloat16, device=cuda)
    H.gemm_w4a16_ffn(y, bf16_dev(x, cuda), w.gate_up, w.down, hidden, n, inter)
    torch.cuda.synchronize()
    assert_close(y.float().cpu().numpy(), y32_ref, LEVEL, "gemm_w4a16_ffn prefix")


@pytest.mark.parametrize("hidden,inter", [(2048, 8192), (8192, 28672)])
def test_full_size_sampled_columns(cuda, oracle, hidden, inter):
    """Full BASELINE shapes (Llama-3.2-1B and Llama-3-70B layers) on the GPU; 128-column windows of
    each projection checked against the oracle."""
    gen = torch.Generator(device=cuda)
    gen.manual_seed(1000)
    gu = synthetic_packed_device(hidden, 2 * inter, cuda, gen)
    dn = synthetic_packed_device(inter, hidden, cuda, gen)
    m = 2
    x = oracle.bf16_bits(np.random.default_rng(7).standard_normal((m, hidden)))
    xd = bf16_dev(x, cuda)
    act = torch.empty(m, inter, dtype=torch.bfloat16, device=cuda)
    ops.w4a16_gemv(act, xd, gu, hidden, 2 * inter, hidden, 2 * inter, 0, _lib.HMB_EPI_SWIGLU, 1, 0)
    y = torch.empty(m, hidden, dtype=torch.float32, device=cuda)
    ops.w4a16_gemv(y, act, dn, inter, hidden, inter, hidden, 0, _lib.HMB_EPI_STORE, 0, 0)
    torch.cuda.synchronize()
    gu_h, dn_h, act_bits, y_h = gu.cpu().numpy(), dn.cpu().numpy(), bits_of(act), y.cpu().numpy()
    for c0 in (0, inter - 64, (inter // 3) // 64 * 64):
        # channels c0 .. c0+63: gate tile column 2*(c0/64), up tile column +1 (interleaved)
        _, gate_up = oracle.gemv(gu_h, hidden, 2 * inter, x, n=128, n0=2 * c0)
        ref_act = oracle.silu_mul(gate_up, 64, 1)
        assert_bf16_close(act_bits[:, c0:c0 + 64], ref_act, min_equal=0.95, what=f"act @{c0}")
    for c0 in (0, hidden - 128, hidden // 2):
        y32, _ = oracle.gemv(dn_h, inter, hidden, act_bits, n=128, n0=c0)
        assert_close(y_h[:, c0:c0 + 128], y32, (1e-5, 1e-5, 0.9999999), f"down @{c0}")
