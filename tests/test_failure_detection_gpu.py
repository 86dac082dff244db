"""Failure detection on the GPU without a fault: a bounded wait that runs out (an mbarrier nothing
arrives on) ends its kernel with HMB_ERR_TIMEOUT in the device status word, the status read clears
it, and the context keeps working (a GEMV and an FFN afterwards match the oracle)."""
import numpy as np
import pytest
import torch

import heteromega_b200 as H
from heteromega_b200 import _lib
from heteromega_b200.torch_ops import device_status, ops
from heteromega_b200.weights import synthetic_layer
from metrics import LEVEL, assert_close

pytestmark = pytest.mark.gpu


def test_wait_that_runs_out_reports_timeout(cuda, oracle):
    assert device_status(cuda) == _lib.HMB_OK
    rc = _lib.lib().hmb_selftest_bounded_wait(2_000_000, torch.cuda.current_stream(cuda).cuda_stream)  # 2 ms
    assert rc == _lib.HMB_OK
    torch.cuda.synchronize()
    assert device_status(cuda) == _lib.HMB_ERR_TIMEOUT
    assert device_status(cuda) == _lib.HMB_OK  # read-and-clear

    # the context is intact: an FFN afterwards is correct and leaves the status clear
    hidden, inter = 512, 1536
    layer = synthetic_layer(hidden, inter, layer=2)
    w = H.pack_ffn_slice(layer, 0, inter, H.GateUpLayout.kInterleaved)
    x = oracle.bf16_bits(np.random.default_rng(3).standard_normal((2, hidden)))
    _, ref = oracle.ffn(w.gate_up.numpy(), w.down.numpy(), hidden, inter, inter, 1, x)
    wd = w.to(cuda)
    y = torch.empty(2, hidden, dtype=torch.bfloat16, device=cuda)
    xd = torch.from_numpy(np.ascontiguousarray(x).view(np.int16)).view(torch.bfloat16).to(cuda)
    ops.w4a16_ffn(y, xd, wd.gate_up, wd.down, hidden, inter, inter, 1)
    torch.cuda.synchronize()
    assert device_status(cuda) == _lib.HMB_OK
    assert_close(y.float().cpu().numpy(), ref, LEVEL, "ffn after a timed-out wait")


def test_selftest_rejects_long_limits(cuda):
    s = torch.cuda.current_stream(cuda).cuda_stream
    assert _lib.lib().hmb_selftest_bounded_wait(0, s) == _lib.HMB_ERR_ARG
    assert _lib.lib().hmb_selftest_bounded_wait(10**9, s) == _lib.HMB_ERR_ARG
