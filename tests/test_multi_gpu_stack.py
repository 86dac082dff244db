"""Tensor parallelism over every GPU of the box at the Llama-3-70B FFN shape (hidden 8192, intermediate
28672), the configuration the scaling benchmark runs.

Each rank keeps its channel shard of two layers (gate/up column-parallel, down row-parallel) and the
chained stack runs with the layer boundary fused with the rank sum over NVLink (hmb_tp_ffn_layer). The
same two whole layers run on one GPU as the reference. Checked, on every rank:
  * the stack output against the single-GPU stack, on sampled rows, under the LEVEL tolerance of the
    reference's tests (kernels/gpu/tests/test_gpu_ffn.cpp:35-36), at M = 1 and 16 (decode: fp32 partials
    exchanged by the boundary) and M = 8192 (prefill: the down GEMM scatters bf16 partial rows into the
    owners' receive slots);
  * the same output bits on every rank, on a graph replay, and with the boundaries unchained (each
    gather completed inside its boundary instead of under the next layer's gate/up GEMM);
  * the fused layer against the unfused one (local partial, then the exchanging boundary), bit for bit;
  * a clear device status word.
The rank sum replaces the reference's two-device boundary sum (src/unified_llm_w4a16_hetero/merged_ffn.cpp:417,
kernels/gpu/src/residual_add.cu:55-73). Skipped with fewer than 2 GPUs; test_tensor_parallel.py has
the 2-GPU checks at smaller shapes and against the oracle."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
H_, I_ = 8192, 28672
MS = (1, 16, 8192)


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def sample_rows(m):
    return np.unique(np.r_[np.arange(0, m, max(1, m // 24)), m - 1])


def _rank(rank, world, port, out_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    import datetime

    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev, timeout=datetime.timedelta(seconds=120))
    tp = None
    stacks = []
    try:
        import sys

        sys.path.insert(0, REPO)
        import heteromega_b200 as H
        from heteromega_b200.stack import FfnStack
        from heteromega_b200.tensor_parallel import TensorParallelFfn
        from heteromega_b200.torch_ops import device_status
        from heteromega_b200.weights import synthetic_packed_device

        gen = torch.Generator(device=dev)
        tp = TensorParallelFfn(H_, I_)
        full, norms = [], []
        for l in range(2):
            gen.manual_seed(1000 + l)  # the same weights on every rank
            g = synthetic_packed_device(H_, I_, dev, gen)
            u = synthetic_packed_device(H_, I_, dev, gen)
            d = synthetic_packed_device(I_, H_, dev, gen)
            tp.add_layer(g, u, d)
            full.append(H.slice_packed_ffn(g, u, d, H_, I_, 0, I_, H.GateUpLayout.kInterleaved))
            del g, u, d
            gen.manual_seed(2000 + l)
            norms.append((torch.randn(H_, device=dev, generator=gen) * 0.2 + 1.0).to(torch.bfloat16))
        tp.connect(max(MS), dev)
        st_tp = FfnStack(None, H_, dev, tp=tp, norms=norms)
        st_one = FfnStack(full, H_, dev, norms=norms)
        stacks = [st_tp, st_one]
        res = {"shares": np.array(tp.shares)}
        for m in MS:
            gen.manual_seed(7 + m)
            h0 = torch.randn(m, H_, device=dev, generator=gen).to(torch.bfloat16)
            got, ref = torch.empty_like(h0), torch.empty_like(h0)
            st_tp.chain = True  # chained boundaries (taken at the two-shot sizes), checked below against unchained
            st_tp.forward(h0, got)
            graph, h_in, result = st_tp.graph(m)
            h_in.copy_(h0)
            graph.replay()
            st_one.forward(h0, ref)
            torch.cuda.synchronize()
            rows = torch.from_numpy(sample_rows(m)).to(dev)
            res[f"got{m}"] = got[rows].float().cpu().numpy()
            res[f"ref{m}"] = ref[rows].float().cpu().numpy()
            res[f"graph_same{m}"] = np.array(bool(torch.equal(result, got)))
            # Chained boundaries (each gather completing under the next gate/up GEMM) against unchained
            # layers: the same bits.
            st_tp.chain = False
            unchained = torch.empty_like(h0)
            st_tp.forward(h0, unchained)
            torch.cuda.synchronize()
            res[f"chain_same{m}"] = np.array(bool(torch.equal(unchained, got)))
            mine = got.view(torch.int32).flatten()  # NCCL moves no 16-bit integers
            other = mine.clone()
            dist.broadcast(other, src=0)
            res[f"rank_same{m}"] = np.array(bool(torch.equal(mine, other)))
        # The fused layer against the unfused one at a one-shot (100 rows) and a two-shot (4096 rows) size.
        for m in (100, 4096):
            gen.manual_seed(60 + m)
            x = torch.randn(m, H_, device=dev, generator=gen).to(torch.bfloat16)
            h_res = torch.randn(m, H_, device=dev, generator=gen).to(torch.bfloat16)
            h1, h2 = h_res.clone(), h_res.clone()
            out1 = tp.layer(0, x, h1, norms[1], 1e-5).clone()
            part = torch.empty(m, H_, dtype=torch.bfloat16, device=dev)
            tp.local_partial(0, x, part)
            out2 = tp.comm.boundary(part, h2, norms[1], 1e-5).clone()
            torch.cuda.synchronize()
            b, e = tp.comm.rows(m, H_)
            res[f"fused_same{m}"] = np.array(bool(torch.equal(out1, out2)) and bool(torch.equal(h1[b:e], h2[b:e])))
        res["status"] = np.array(device_status(dev))
        np.savez(out_path + f".{rank}.npz", **res)
        dist.barrier(device_ids=[rank])
    finally:
        for st in stacks:
            st.release()
        if tp is not None:
            dist.barrier(device_ids=[rank])
            tp.close()
        dist.barrier(device_ids=[rank])
        dist.destroy_process_group()


def test_all_gpus_llama70b_stack(tmp_path):
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs 2 or more GPUs")
    world = min(torch.cuda.device_count(), 8)
    out = str(tmp_path / "mg")
    mp.start_processes(_rank, args=(world, free_port(), out), nprocs=world, join=True, start_method="spawn")
    import sys

    sys.path.insert(0, os.path.join(REPO, "tests"))
    from metrics import LEVEL, compare

    summary = []
    for rank in range(world):
        r = np.load(out + f".{rank}.npz")
        assert int(r["status"]) == 0, f"rank {rank}: a bounded wait gave up"
        for m in MS:
            assert bool(r[f"rank_same{m}"]), f"rank {rank} M={m}: output bits differ from rank 0"
            assert bool(r[f"graph_same{m}"]), f"rank {rank} M={m}: graph replay differs"
            assert bool(r[f"chain_same{m}"]), f"rank {rank} M={m}: chained boundaries differ from unchained layers"
            max_rel, rel_l2, cos = compare(r[f"got{m}"], r[f"ref{m}"])
            summary.append((rank, m, max_rel, rel_l2, cos))
            assert max_rel <= LEVEL[0] and rel_l2 <= LEVEL[1] and cos >= LEVEL[2], \
                f"rank {rank} M={m}: max_rel {max_rel:.2e} rel_l2 {rel_l2:.2e} cos {cos:.7f}"
        for m in (100, 4096):
            assert bool(r[f"fused_same{m}"]), f"rank {rank} M={m}: fused layer differs from unfused"
    print(f"world {world}: " + "; ".join(f"r{r} M={m} max_rel {a:.2e} rel_l2 {b:.2e}" for r, m, a, b, _ in summary if r == 0))
