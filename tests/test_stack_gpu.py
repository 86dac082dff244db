"""FfnStack: layers chained through the layer boundary (h += FFN_l(RMSNorm(h) * g_l)), replayed as a
CUDA graph, and its host-buffer call.

* The chain against the CPU oracle's chain (the reference CPU FFN and the boundary arithmetic of
  residual_norm_bf16) at the reference tolerance.
* The host call against the device-resident replay. A decode-sized batch (one chunk) gives the same
  bits. The pipelined call (two row chunks, copies on side streams) runs each chunk as its own batch,
  whose GEMMs may split K differently from the whole batch's (a different fp32 summation order), so
  it is held to the reference tolerance.
"""
import numpy as np
import pytest
import torch

import heteromega_b200 as H
from heteromega_b200.stack import FfnStack
from heteromega_b200.weights import synthetic_packed_device
from metrics import LEVEL, assert_close

pytestmark = pytest.mark.gpu

HIDDEN, INTER, LAYERS = 1024, 3072, 3


@pytest.fixture(scope="module")
def stack3(cuda):
    gen = torch.Generator(device=cuda)
    ws, norms = [], []
    for l in range(LAYERS):
        gen.manual_seed(100 + l)
        g = synthetic_packed_device(HIDDEN, INTER, cuda, gen)
        u = synthetic_packed_device(HIDDEN, INTER, cuda, gen)
        d = synthetic_packed_device(INTER, HIDDEN, cuda, gen)
        ws.append(H.slice_packed_ffn(g, u, d, HIDDEN, INTER, 0, INTER, H.GateUpLayout.kInterleaved))
        norms.append((torch.randn(HIDDEN, device=cuda, generator=gen) * 0.2 + 1.0).to(torch.bfloat16))
    st = FfnStack(ws, HIDDEN, cuda, norms=norms)
    yield st
    st.release()


def _bits(t):
    return t.cpu().view(torch.int16).numpy().view(np.uint16)


def oracle_chain(O, st, h0_bits):
    """The stack on the CPU: x = RMSNorm(h) * g_0; per layer h += FFN(x) (bf16 FFN output, the
    reference CPU chain), x = RMSNorm(h) * g_{l+1}."""
    norms = [_bits(n) for n in st.norms]
    h, x = O.residual_norm(h0_bits, [], norms[0], st.eps)
    for l, w in enumerate(st.layers):
        y, _ = O.ffn(w.gate_up.cpu().numpy(), w.down.cpu().numpy(), w.hidden, w.channels(), w.stored_channels(),
                     int(w.layout), x)
        last = l == len(st.layers) - 1
        h, x = O.residual_norm(h, [y], None if last else norms[l + 1], st.eps, with_normed=not last)
    return h


@pytest.mark.parametrize("m", [1, 5, 40])
def test_chain_matches_oracle(cuda, oracle, stack3, m):
    gen = torch.Generator(device=cuda).manual_seed(70 + m)
    h0 = torch.randn(m, HIDDEN, device=cuda, generator=gen).to(torch.bfloat16)
    out = torch.empty_like(h0)
    st = stack3
    st.forward(h0, out)
    torch.cuda.synchronize()
    ref = oracle_chain(oracle, st, _bits(h0))
    assert_close(oracle.bf16_to_f32(_bits(out)), oracle.bf16_to_f32(ref), LEVEL, f"{LAYERS}-layer chain m={m}")
    # the graph replay gives the eager result's bits
    graph, h_in, result = st.graph(m)
    h_in.copy_(h0)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(result, out)


@pytest.mark.parametrize("m", [3, 600, 513])
def test_forward_host_matches_device_replay(cuda, stack3, m):
    st = stack3
    gen = torch.Generator(device=cuda).manual_seed(m)
    h0 = torch.randn(m, HIDDEN, device=cuda, generator=gen).to(torch.bfloat16)
    out_dev = torch.empty_like(h0)
    st.forward(h0, out_dev)
    h_host = h0.cpu().pin_memory()
    out_host = torch.zeros_like(h_host).pin_memory()
    for _ in range(2):  # repeated calls reuse the chunk graphs and their buffers
        st.forward_host(h_host, out_host)
    torch.cuda.synchronize()
    assert torch.equal(h_host, h0.cpu()), "the input is not modified"
    if m < 512:
        assert torch.equal(out_host, out_dev.cpu())
    else:
        assert_close(out_host.float().numpy(), out_dev.float().cpu().numpy(), LEVEL, f"pipelined host call m={m}")
