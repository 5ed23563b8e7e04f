"""Tensor-parallel W4A4 linears on the host: two `gloo` ranks run the real TP
classes (shard slicing in load_full / load_shard, the BF16 all-gather of the
full-width layout, the FP32 partial all-reduce of the row-parallel layer).

Only the two kernel calls are replaced, inside the worker processes, by
stand-ins built on the numpy oracle (activation prep to k-order codes, and the
grouped GEMM); they agree with each other on the code layout the layer passes
between them, and the oracle stays the checker: every expected value below is
the oracle on the unsharded weights.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _bits(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def _stubs(o):
    """Oracle-backed stand-ins for W4A4Linear.quantize_input and the GEMM."""
    def quantize_input(self, flat):
        _, sbits, codes, _, _ = o.prepare(_bits(flat), self.signs.numpy(), self.layout_id, self.clamp_lo)
        return (torch.from_numpy(codes.astype(np.int8)),
                torch.from_numpy(sbits.astype(np.uint16).view(np.int16)).view(torch.bfloat16))

    def gemm(codes, w_packed, a_scale, w_scale, out=None, *, out_fp32=False, **_):
        qw = o.unpack_int4(w_packed.numpy().view(np.uint8))
        r = o.grouped_gemm_f32(codes.numpy(), qw, a_scale.float().numpy(), w_scale.float().numpy())
        t = torch.from_numpy(np.ascontiguousarray(r, dtype=np.float32))
        return t if out_fp32 else t.bfloat16()
    return quantize_input, gemm


def _full_reference(o, x, packed, scale, signs, layout_id, clamp_lo=-8):
    """Oracle FP32 output of the unsharded projection."""
    _, sbits, codes, _, _ = o.prepare(_bits(x), signs.numpy(), layout_id, clamp_lo)
    sa = torch.from_numpy(sbits.astype(np.uint16).view(np.int16)).view(torch.bfloat16).float().numpy()
    return codes, sa, o.grouped_gemm_f32(codes, o.unpack_int4(packed.numpy().view(np.uint8)), sa,
                                         scale.float().numpy())


def _weights(n, k, seed):
    g = torch.Generator().manual_seed(seed)
    packed = torch.randint(-128, 128, (n, k // 2), generator=g, dtype=torch.int8)
    scale = (torch.rand(n, k // 128, generator=g) * 0.01 + 0.001).bfloat16()
    signs = (torch.randint(0, 2, (k,), generator=g, dtype=torch.int8) * 2 - 1)
    return packed, scale, signs


def _worker(rank, world, port, failures):
    import sys
    for p in (ROOT, os.path.join(ROOT, "nano-vllm-int4_b200")):
        sys.path.insert(0, p)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import nv4_oracle as o
        from nanovllm.layers import linear_w4a4 as lin
        from nanovllm.utils import synthetic
        quantize_input, gemm = _stubs(o)
        lin.W4A4Linear.quantize_input = quantize_input
        lin.w4a4_grouped_gemm_i8 = gemm
        B128, RDH = o.LAYOUT_BLOCK128, o.LAYOUT_ROW_DH
        x = synthetic.activations(3, 512, seed=11)

        # column parallel: each rank's output is its slice of the full output, bit for bit
        packed, scale, signs = _weights(96, 512, 1)
        mod = lin.W4A4ColumnParallelLinear(512, 96, layout="block128", tp_rank=rank, tp_size=world)
        mod.load_full(packed, scale, signs)
        got = mod(x)
        _, _, full = _full_reference(o, x, packed, scale, signs, B128)
        want = o.f32_to_bf16_bits(full)[:, rank * 48:(rank + 1) * 48]
        assert np.array_equal(_bits(got), want), "column-parallel slice"

        # merged gate/up: each half sharded separately
        packed, scale, signs = _weights(64, 512, 2)
        mod = lin.W4A4MergedColumnParallelLinear(512, [32, 32], layout="block128", tp_rank=rank, tp_size=world)
        mod.load_full(packed, scale, signs)
        got = mod(x)
        _, _, full = _full_reference(o, x, packed, scale, signs, B128)
        fb = o.f32_to_bf16_bits(full)
        want = np.concatenate([fb[:, rank * 16:(rank + 1) * 16], fb[:, 32 + rank * 16:32 + (rank + 1) * 16]], 1)
        assert np.array_equal(_bits(got), want), "merged column-parallel slices"

        # fused qkv sharded by heads (4 q heads, 2 kv heads of 16)
        packed, scale, signs = _weights(128, 512, 3)
        mod = lin.W4A4QKVParallelLinear(512, 16, 4, 2, layout="block128", tp_rank=rank, tp_size=world)
        mod.load_full(packed, scale, signs)
        got = mod(x)
        _, _, full = _full_reference(o, x, packed, scale, signs, B128)
        fb = o.f32_to_bf16_bits(full)
        q, kv = 64, 32
        want = np.concatenate([fb[:, rank * 32:(rank + 1) * 32], fb[:, q + rank * 16:q + (rank + 1) * 16],
                               fb[:, q + kv + rank * 16:q + kv + (rank + 1) * 16]], 1)
        assert np.array_equal(_bits(got), want), "qkv head shards"

        # row parallel, group-local layout: BF16(sum of the two FP32 partials)
        packed, scale, signs = _weights(40, 512, 4)
        mod = lin.W4A4RowParallelLinear(512, 40, layout="block128", tp_rank=rank, tp_size=world)
        mod.load_full(packed, scale, signs)
        got = mod(x[:, rank * 256:(rank + 1) * 256].contiguous())
        codes, sa, full = _full_reference(o, x, packed, scale, signs, B128)
        qw = o.unpack_int4(packed.numpy().view(np.uint8))
        sw = scale.float().numpy()
        parts = [o.grouped_gemm_f32(codes[:, r * 256:(r + 1) * 256], qw[:, r * 256:(r + 1) * 256], sa[:, r * 2:r * 2 + 2],
                                    sw[:, r * 2:r * 2 + 2]) for r in range(world)]
        want = o.f32_to_bf16_bits((parts[0] + parts[1]).astype(np.float32))
        assert np.array_equal(_bits(got), want), "row-parallel FP32 all-reduce"
        rel = np.linalg.norm(got.float().numpy() - full) / np.linalg.norm(full)
        assert rel < 1e-2, rel   # BF16 output rounding vs the unsharded FP32 chain

        # row parallel, full-width layout: the BF16 input is all-gathered and quantised whole
        xw = synthetic.activations(2, 4096, seed=12)
        packed, scale, signs = _weights(16, 4096, 5)
        mod = lin.W4A4RowParallelLinear(4096, 16, layout="row_DH_paley12_kron_sylvester_v1", tp_rank=rank,
                                        tp_size=world)
        mod.load_full(packed, scale, signs)
        assert mod.gather_input and mod.signs.shape == (4096,)
        got = mod(xw[:, rank * 2048:(rank + 1) * 2048].contiguous())
        codes, sa, full = _full_reference(o, xw, packed, scale, signs, RDH)
        qw = o.unpack_int4(packed.numpy().view(np.uint8))
        sw = scale.float().numpy()
        parts = [o.grouped_gemm_f32(codes[:, r * 2048:(r + 1) * 2048], qw[:, r * 2048:(r + 1) * 2048],
                                    sa[:, r * 16:(r + 1) * 16], sw[:, r * 16:(r + 1) * 16]) for r in range(world)]
        want = o.f32_to_bf16_bits((parts[0] + parts[1]).astype(np.float32))
        assert np.array_equal(_bits(got), want), "row-parallel gathered input"
    except Exception as e:  # report to the parent instead of hanging the group
        failures.put(f"rank {rank}: {type(e).__name__}: {e}")
        raise
    finally:
        dist.destroy_process_group()


def test_tensor_parallel_linears_two_ranks():
    ctx = mp.get_context("spawn")
    failures = ctx.Queue()
    mp.start_processes(_worker, args=(2, _free_port(), failures), nprocs=2, join=True, start_method="spawn")
    assert failures.empty(), failures.get()


def test_row_parallel_requires_whole_groups():
    import sys
    sys.path.insert(0, os.path.join(ROOT, "nano-vllm-int4_b200"))
    from nanovllm.layers.linear_w4a4 import W4A4RowParallelLinear
    with pytest.raises(ValueError, match="128-groups"):
        W4A4RowParallelLinear(384, 64, layout="block128", tp_rank=0, tp_size=2)
