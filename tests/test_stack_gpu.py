"""FfnStack: the graph-replayed stack and its host-buffer call. A decode-sized batch (one chunk) must
give the same bits as the device-resident replay; the pipelined call (two row chunks, copies on side
streams) runs each chunk as its own batch, whose GEMMs may split K differently from the whole batch's
(a different fp32 summation order), so it is held to the reference tolerance."""
import pytest
import torch

import heteromega_b200 as H
from heteromega_b200.stack import FfnStack
from heteromega_b200.weights import synthetic_packed_device
from metrics import LEVEL, assert_close

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def stack2(cuda):
    hidden, inter, layers = 1024, 3072, 2
    gen = torch.Generator(device=cuda)
    ws = []
    for l in range(layers):
        gen.manual_seed(100 + l)
        g = synthetic_packed_device(hidden, inter, cuda, gen)
        u = synthetic_packed_device(hidden, inter, cuda, gen)
        d = synthetic_packed_device(inter, hidden, cuda, gen)
        ws.append(H.slice_packed_ffn(g, u, d, hidden, inter, 0, inter, H.GateUpLayout.kInterleaved))
    st = FfnStack(ws, hidden, cuda)
    yield st, hidden, layers
    st.release()


@pytest.mark.parametrize("m", [3, 600, 513])
def test_forward_host_matches_device_replay(cuda, stack2, m):
    st, hidden, layers = stack2
    gen = torch.Generator(device=cuda)
    gen.manual_seed(m)
    x = torch.randn(layers, m, hidden, device=cuda, generator=gen).to(torch.bfloat16)
    y_dev = torch.empty_like(x)
    st.forward(x, y_dev)
    x_host = x.cpu().pin_memory()
    y_host = torch.zeros_like(x_host).pin_memory()
    for _ in range(2):  # repeated calls reuse the chunk graphs and their buffers
        st.forward_host(x_host, y_host)
    torch.cuda.synchronize()
    if m < 512:
        assert torch.equal(y_host, y_dev.cpu())
    else:
        assert_close(y_host.float().numpy(), y_dev.float().cpu().numpy(), LEVEL, f"pipelined host call m={m}")
