"""Tensor-parallel FFN: the channel partition across ranks and the per-layer boundary all-reduce.

CPU part (gloo, world size 2): each rank slices its shard out of the whole packed layer with the host
slice path, computes its partial output with the CPU oracle, and the all-reduce of the partials must
give the unsharded FFN — the algebra of npu/ffn/reference.py:200-221 over P ranks. Also checks the
partition planner against the reference's from_ratio rounding.
GPU part (2 GPUs): the same through the CUDA kernels, with the library's NVLink all-reduce and with
NCCL; skipped with fewer GPUs.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import heteromega_b200 as H
from heteromega_b200.partition import ChannelSplit, DeviceModel, best_ratios, plan_shards, predict_layer_time
from heteromega_b200.tensor_parallel import TensorParallelFfn
from heteromega_b200.weights import synthetic_layer

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_from_ratio_matches_reference(golden):
    """The two-device cut lands where the reference's FFNPartition.from_ratio puts the NPU share."""
    for inter, ratio, npu in golden("contract")["from_ratio"]:
        split = ChannelSplit.two_way(int(inter), float(ratio))
        assert split[0] == (0, int(npu)) and split[1] == (int(npu), int(inter))
    with pytest.raises(ValueError):
        ChannelSplit.two_way(14336, 1.5)
    with pytest.raises(ValueError):
        ChannelSplit(14336, (0, 100, 14336))
    with pytest.raises(ValueError):
        ChannelSplit(14336, (0, 8192, 4096, 14336))


@pytest.mark.parametrize("inter,world", [(14336, 8), (13824, 8), (13824, 3)])
def test_channel_split_balanced_matches_plan(inter, world):
    split = ChannelSplit.balanced(inter, world)
    assert split.devices == world and split.ranges() == plan_shards(inter, world)


@pytest.mark.parametrize("inter,world", [(8192, 2), (14336, 8), (13824, 8), (28672, 8), (13824, 3), (1024, 8)])
def test_plan_shards_cover_and_align(inter, world):
    shares = plan_shards(inter, world)
    assert shares[0][0] == 0 and shares[-1][1] == inter
    for (b, e), (b2, _) in zip(shares, shares[1:]):
        assert e == b2
    for b, e in shares:
        assert e > b and b % 128 == 0 and e % 128 == 0
    sizes = [e - b for b, e in shares]
    assert max(sizes) - min(sizes) <= 128
    if inter == 13824 and world == 8:
        assert sorted(set(sizes)) == [1664, 1792] and sizes.count(1792) == 4


def test_cost_model_prefers_balanced_shares():
    dev = DeviceModel(hbm_gbs=6457.0, tflops=1677.0, overhead_us=2.0)
    ratios, shares = best_ratios(8192, 28672, 1, [dev] * 4, allreduce_us=5.0)
    assert [e - b for b, e in shares] == [7168] * 4
    t1 = predict_layer_time(8192, [(0, 28672)], 1, [dev])
    t4 = predict_layer_time(8192, shares, 1, [dev] * 4, allreduce_us=5.0)
    assert t4 < t1


def _gloo_rank(rank, world, port, hidden, inter, m, out_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import sys

        sys.path.insert(0, REPO)
        from oracle import oracle as O

        layer = synthetic_layer(hidden, inter, layer=3)
        g = H.pack_w4a16(layer.gate_q, layer.gate_s, layer.gate_z)
        u = H.pack_w4a16(layer.up_q, layer.up_s, layer.up_z)
        d = H.pack_w4a16(layer.down_q, layer.down_s, layer.down_z)
        tp = TensorParallelFfn(hidden, inter)
        tp.add_layer(g, u, d)  # host slice path: CPU tensors
        w = tp.layers[0]
        x = O.bf16_bits(np.random.default_rng(5).standard_normal((m, hidden)))
        _, part = O.ffn(w.gate_up.numpy(), w.down.numpy(), hidden, w.channels(), w.stored_channels(), int(w.layout), x)
        partial = torch.from_numpy(np.ascontiguousarray(part))
        tp.reduce_partials(partial)
        if rank == 0:
            full = H.pack_ffn_slice(layer, 0, inter, H.GateUpLayout.kInterleaved)
            _, ref = O.ffn(full.gate_up.numpy(), full.down.numpy(), hidden, inter, inter, 1, x)
            np.savez(out_path, got=partial.numpy(), ref=ref, shares=np.array(tp.shares))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("inter", [1024, 1152])
def test_gloo_partials_sum_to_full_ffn(tmp_path, inter):
    hidden, m, world = 256, 3, 2
    out = str(tmp_path / "tp.npz")
    mp.start_processes(_gloo_rank, args=(world, free_port(), hidden, inter, m, out), nprocs=world, join=True,
                       start_method="spawn")
    r = np.load(out)
    assert len(r["shares"]) == world
    from metrics import assert_close

    assert_close(r["got"], r["ref"], (1e-5, 1e-5, 0.9999999), "sum of rank partials")


def _gpu_rank(rank, world, port, out_path, collective):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    tp = None
    try:
        from heteromega_b200.weights import synthetic_packed_device

        hidden, inter = 2048, 8192
        gen = torch.Generator(device=dev)
        gen.manual_seed(11)
        g = synthetic_packed_device(hidden, inter, dev, gen)
        u = synthetic_packed_device(hidden, inter, dev, gen)
        d = synthetic_packed_device(inter, hidden, dev, gen)
        tp = TensorParallelFfn(hidden, inter, collective=collective)
        tp.add_layer(g, u, d)
        tp.connect(1024, dev)
        full = H.slice_packed_ffn(g, u, d, hidden, inter, 0, inter, H.GateUpLayout.kInterleaved)
        res = {}
        for m in (1, 7, 300, 1024):
            gen.manual_seed(12 + m)
            x = torch.randn(m, hidden, device=dev, generator=gen).to(torch.bfloat16)
            y = torch.empty(m, hidden, dtype=torch.bfloat16, device=dev)
            for _ in range(3):  # repeated calls: the communicator's epochs and double buffers advance
                tp.forward(0, x, y)
            ref = torch.empty_like(y)
            H.gpu_ffn_slice_forward(full, x, None, ref)
            torch.cuda.synchronize()
            res[f"got{m}"], res[f"ref{m}"] = y.float().cpu().numpy(), ref.float().cpu().numpy()
        # every rank holds the same bits
        mine = torch.cat([torch.from_numpy(res[f"got{m}"]).flatten() for m in (1, 7, 300, 1024)]).to(dev)
        other = mine.clone()
        dist.broadcast(other, src=0)
        res["same_bits"] = np.array(bool(torch.equal(mine, other)))

        # The chained stack (h += FFN(RMSNorm(h)) per layer, boundary fused with the rank sum) against
        # the single-GPU stack with the whole layers.
        from heteromega_b200.stack import FfnStack

        norms = [(torch.randn(hidden, device=dev, generator=gen) * 0.2 + 1.0).to(torch.bfloat16) for _ in range(2)]
        if collective == "hmb":
            # The fused layer (down GEMM scattering its rows into the peers' slots) against the same
            # layer unfused (partial in local memory, then the exchanging boundary): the same bits,
            # at a one-shot size (100 rows) and a two-shot size (300 rows).
            fused_same = []
            for m in (100, 300):
                gen.manual_seed(60 + m)
                x = torch.randn(m, hidden, device=dev, generator=gen).to(torch.bfloat16)
                h_res = torch.randn(m, hidden, device=dev, generator=gen).to(torch.bfloat16)
                h1, h2 = h_res.clone(), h_res.clone()
                out1 = tp.layer(0, x, h1, norms[0], 1e-5).clone()
                part = torch.empty(m, hidden, dtype=torch.bfloat16, device=dev)
                tp.local_partial(0, x, part)
                out2 = tp.comm.boundary(part, h2, norms[0], 1e-5).clone()
                torch.cuda.synchronize()
                b, e = tp.comm.rows(m, hidden)
                fused_same.append(bool(torch.equal(out1, out2)) and bool(torch.equal(h1[b:e], h2[b:e])))
            res["fused_same"] = np.array(all(fused_same))
        tp.add_layer(g, u, d)  # a second layer (the same weights)
        st_tp = FfnStack(None, hidden, dev, tp=tp, norms=norms)
        st_one = FfnStack([full, full], hidden, dev, norms=norms)
        same = []
        for m in (1, 100, 300):
            gen.manual_seed(40 + m)
            h0 = torch.randn(m, hidden, device=dev, generator=gen).to(torch.bfloat16)
            got, ref = torch.empty_like(h0), torch.empty_like(h0)
            st_tp.forward(h0, got)
            graph, h_in, result = st_tp.graph(m)
            h_in.copy_(h0)
            graph.replay()
            st_one.forward(h0, ref)
            torch.cuda.synchronize()
            same.append(bool(torch.equal(result, got)))
            res[f"stack{m}"], res[f"stackref{m}"] = got.float().cpu().numpy(), ref.float().cpu().numpy()
        res["stack_graph_same"] = np.array(all(same))
        st_tp.release()
        from heteromega_b200.torch_ops import device_status

        res["status"] = np.array(device_status(dev))
        np.savez(out_path + f".{rank}.npz", **res)
        dist.barrier(device_ids=[rank])
    finally:
        if tp is not None:
            tp.close()
        dist.barrier(device_ids=[rank])
        dist.destroy_process_group()


BOUNDARY_CASES = [(1, 2048), (7, 2048), (300, 2048), (1024, 2048), (32, 8192), (33, 8192)]


def _gpu_boundary_rank(rank, world, port, out_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    comm = None
    try:
        from heteromega_b200.tensor_parallel import PeerComm

        comm = PeerComm(1024 * 8192 * 2, device=dev)
        res = {}
        for rnd in range(2):  # the second round reuses the double-buffered slots with advanced epochs
            for m, h in BOUNDARY_CASES:
                for weighted, dt in ((True, "bf16"), (False, "bf16"), (True, "f32")):
                    tag = f"{m}_{h}_{int(weighted)}_{rnd}_{dt}"
                    gx = torch.Generator(device=dev).manual_seed(m * 31 + h + rnd)  # the same on every rank
                    x = torch.randn(m, h, device=dev, generator=gx).to(torch.bfloat16)
                    w = (torch.randn(h, device=dev, generator=gx) * 0.2 + 1.0).to(torch.bfloat16)
                    gy = torch.Generator(device=dev).manual_seed(m * 31 + h + rnd + 1000 * (rank + 1))
                    y = torch.randn(m, h, device=dev, generator=gy) * 3
                    y = y.to(torch.bfloat16) if dt == "bf16" else y
                    x0 = x.clone()
                    out = comm.boundary(y, x, w if weighted else None, 1e-5)
                    torch.cuda.synchronize()
                    b, e = comm.rows(m, h)
                    bits = lambda t: t.cpu().view(torch.int16).numpy()  # noqa: E731
                    res[f"x0_{tag}"], res[f"w_{tag}"] = bits(x0), bits(w)
                    res[f"y_{tag}"] = bits(y) if dt == "bf16" else y.cpu().numpy()
                    res[f"out_{tag}"], res[f"x_{tag}"] = bits(out), bits(x[b:e])
                    res[f"rows_{tag}"] = np.array([b, e])
        from heteromega_b200.torch_ops import device_status

        res["status"] = np.array(device_status(dev))
        np.savez(out_path + f".{rank}.npz", **res)
        dist.barrier(device_ids=[rank])
    finally:
        if comm is not None:
            comm.close()
        dist.barrier(device_ids=[rank])
        dist.destroy_process_group()


@pytest.mark.gpu
def test_two_gpu_boundary_matches_oracle(tmp_path, oracle):
    """The fused tensor-parallel boundary (hmb_allreduce_residual_norm) on 2 GPUs, one-shot (up to 512 KB)
    and two-shot (rows split between the ranks) sizes, with and without a norm weight, with bf16 and
    fp32 partials, against the oracle's boundary with the two rank partials as its addends in rank
    order: the kept rows of x bit for bit, the output on both ranks the same bits and within one bf16
    rounding of the oracle."""
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    out = str(tmp_path / "bn")
    mp.start_processes(_gpu_boundary_rank, args=(2, free_port(), out), nprocs=2, join=True, start_method="spawn")
    from metrics import assert_bf16_close

    r = [np.load(out + f".{rank}.npz") for rank in range(2)]
    assert int(r[0]["status"]) == 0 and int(r[1]["status"]) == 0
    u16 = lambda a: a.view(np.uint16)  # noqa: E731
    for rnd in range(2):
        for m, h in BOUNDARY_CASES:
            for weighted, dt in ((1, "bf16"), (0, "bf16"), (1, "f32")):
                tag = f"{m}_{h}_{weighted}_{rnd}_{dt}"
                assert np.array_equal(r[0][f"out_{tag}"], r[1][f"out_{tag}"]), f"ranks disagree {tag}"
                if dt == "bf16":
                    ref_x, ref_n = oracle.residual_norm(u16(r[0][f"x0_{tag}"]), [u16(r[0][f"y_{tag}"]), u16(r[1][f"y_{tag}"])],
                                                        u16(r[0][f"w_{tag}"]) if weighted else None, 1e-5)
                else:
                    # fp32 partials: x + y_0 + y_1 in fp32, left to right, one rounding; then the norm
                    acc = oracle.bf16_to_f32(u16(r[0][f"x0_{tag}"])).astype(np.float32)
                    for rank in range(2):
                        acc = (acc + r[rank][f"y_{tag}"]).astype(np.float32)
                    ref_x, ref_n = oracle.residual_norm(oracle.bf16_bits(acc), [], u16(r[0][f"w_{tag}"]), 1e-5)
                covered = np.zeros(m, bool)
                for rank in range(2):
                    b, e = r[rank][f"rows_{tag}"]
                    covered[b:e] = True
                    assert np.array_equal(u16(r[rank][f"x_{tag}"]), ref_x[b:e]), f"x rows {b}:{e} rank {rank} {tag}"
                assert covered.all()
                if weighted:
                    assert_bf16_close(u16(r[0][f"out_{tag}"]), ref_n, min_equal=0.99, what=f"boundary out {tag}")
                else:
                    assert np.array_equal(u16(r[0][f"out_{tag}"]), ref_x), f"out without weight is x {tag}"


@pytest.mark.gpu
@pytest.mark.parametrize("collective", ["hmb", "nccl"])
def test_two_gpus(tmp_path, collective):
    """Tensor parallel over 2 GPUs against the single-GPU FFN: the NVLink peer-memory all-reduce (both
    its one-shot and two-shot sizes) and NCCL; decode and prefill rows."""
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    out = str(tmp_path / "tp")
    mp.start_processes(_gpu_rank, args=(2, free_port(), out, collective), nprocs=2, join=True, start_method="spawn")
    from metrics import LEVEL, assert_close

    for rank in range(2):
        r = np.load(out + f".{rank}.npz")
        assert int(r["status"]) == 0
        assert bool(r["same_bits"])
        for m in (1, 7, 300, 1024):
            assert_close(r[f"got{m}"], r[f"ref{m}"], LEVEL, f"TP2 {collective} vs single GPU m={m} rank {rank}")
        assert bool(r["stack_graph_same"])
        if collective == "hmb":
            assert bool(r["fused_same"]), "the scattering down GEMM must give the unfused layer's bits"
        for m in (1, 100, 300):
            assert_close(r[f"stack{m}"], r[f"stackref{m}"], LEVEL, f"TP2 {collective} chained stack m={m} rank {rank}")
