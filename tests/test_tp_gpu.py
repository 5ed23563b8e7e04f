"""Tensor-parallel row-parallel W4A4 layer on every visible GPU (2, 4 or 8;
NCCL process group): both peer-memory paths -- the GEMM storing its tiles into
the peers' inboxes (default) and the GEMM followed by the one-shot all-reduce
kernel, interleaved on the same peer buffers -- must give the NCCL
all-reduce's BF16 result -- exactly on 2 ranks (two FP32 partials are added in
the same order), within BF16 rounding of a different summation order on more
-- identical on every rank, over repeated calls and CUDA-graph replays, and
batches above its token limit must fall back to NCCL.  Skipped with fewer than
2 GPUs."""
import os
import socket
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, failures):
    for p in (ROOT, os.path.join(ROOT, "nano-vllm-int4_b200")):
        sys.path.insert(0, p)
    import datetime
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    graph = None
    try:
        from nanovllm import _native
        from nanovllm.layers import linear_w4a4 as lin
        from nanovllm.layers.linear_w4a4 import W4A4RowParallelLinear
        from nanovllm.utils import synthetic
        for layout, k, n in (("block128", 4096, 4096), ("row_DH_paley12_kron_sylvester_v1", 12288, 1024)):
            g = torch.Generator(device=dev).manual_seed(k + n)
            packed = torch.randint(-128, 128, (n, k // 2), dtype=torch.int8, device=dev, generator=g)
            scale = (torch.rand(n, k // 128, device=dev, generator=g) * 0.003 + 1e-4).bfloat16()
            signs = torch.randint(0, 2, (k,), dtype=torch.int8, device=dev, generator=g) * 2 - 1
            peer = W4A4RowParallelLinear(k, n, layout=layout, tp_rank=rank, tp_size=world).to(dev)
            peer2 = W4A4RowParallelLinear(k, n, layout=layout, tp_rank=rank, tp_size=world).to(dev)
            peer2.fuse_peer_gemm = False
            nccl = W4A4RowParallelLinear(k, n, layout=layout, tp_rank=rank, tp_size=world).to(dev)
            nccl.use_peer_allreduce = False
            for mod in (peer, peer2, nccl):
                mod.load_full(packed, scale, signs)
            kl = k // world

            def same(a, b):
                if world == 2:
                    return torch.equal(a, b)
                return (a.float() - b.float()).norm() <= 1e-2 * b.float().norm()
            for m in (1, 32, 33):
                x = synthetic.activations(m, k, seed=m).to(dev)[:, rank * kl:(rank + 1) * kl].contiguous()
                want = nccl(x)
                for _ in range(2):  # repeated, interleaved calls advance the peer epochs
                    got = peer(x)
                    assert same(got, want), (layout, m, "fused")
                    got2 = peer2(x)
                    assert torch.equal(got2, got), (layout, m, "two-kernel")
                every = [torch.empty_like(got) for _ in range(world)]
                dist.all_gather(every, got)
                assert all(torch.equal(e, every[0]) for e in every), (layout, m, "ranks differ")
            assert any(lin._PEER_STATE.values()), "peer buffers were not set up"
            # CUDA graph replays of the peer path with new inputs
            x = synthetic.activations(32, k, seed=5).to(dev)[:, rank * kl:(rank + 1) * kl].contiguous()
            out = peer(x)
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                out = peer(x)
                out2 = peer2(x)
            for seed in (6, 7, 8):
                x.copy_(synthetic.activations(32, k, seed=seed).to(dev)[:, rank * kl:(rank + 1) * kl])
                graph.replay()
                torch.cuda.synchronize()
                assert same(out, nccl(x)), (layout, seed, "graph replay")
                assert torch.equal(out2, out), (layout, seed, "graph replay, two-kernel")
            del graph
            graph = None
            torch.cuda.synchronize()
        lin.release_peer_buffers()
        assert _native.device_error() == 0
    except Exception as e:
        failures.put(f"rank {rank}: {type(e).__name__}: {e}")
        raise
    finally:
        del graph
        torch.cuda.synchronize()
        dist.destroy_process_group()


def test_peer_allreduce_matches_nccl():
    count = torch.cuda.device_count()
    if count < 2:
        pytest.skip("needs 2 GPUs")
    world = 8 if count >= 8 else (4 if count >= 4 else 2)
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    failures = ctx.Queue()
    mp.start_processes(_worker, args=(world, _free_port(), failures), nprocs=world, join=True, start_method="spawn")
    assert failures.empty(), failures.get()
