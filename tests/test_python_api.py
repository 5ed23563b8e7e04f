"""Host-side behaviour of the drop-in Python API (no kernel launches): the
reference's validation errors and messages, module construction and buffers."""
import pytest
import torch

from nanovllm.kernels import rht_a4_tilelang as rk
from nanovllm.kernels import w4a4_grouped_kernel as wk
from nanovllm.layers.linear_w4a16 import W4A16Linear
from nanovllm.layers.linear_w4a4 import (W4A4ColumnParallelLinear, W4A4Linear, W4A4MergedColumnParallelLinear,
                                         W4A4QKVParallelLinear, W4A4RowParallelLinear)


def bufs(m, k):
    return torch.empty(m, k // 2, dtype=torch.int8), torch.empty(m, k // 128, dtype=torch.bfloat16)


def test_rht_validation_messages():
    x = torch.zeros(2, 4096, dtype=torch.bfloat16)
    s = torch.ones(4096, dtype=torch.int8)
    p, sc = bufs(2, 4096)
    with pytest.raises(ValueError, match="Expected BF16 X"):
        rk.rht_quant_pack(x.float(), s, out_packed=p, out_scale=sc)
    with pytest.raises(ValueError, match="Expected BF16 X"):
        rk.rht_quant_pack(torch.zeros(2, 1024, dtype=torch.bfloat16), torch.ones(1024, dtype=torch.int8),
                          out_packed=bufs(2, 1024)[0], out_scale=bufs(2, 1024)[1])
    with pytest.raises(ValueError, match="INT8 signs"):
        rk.rht_quant_pack(x, s.float(), out_packed=p, out_scale=sc)
    with pytest.raises(ValueError, match="INT8 output"):
        rk.rht_quant_pack(x, s, out_packed=p[:1], out_scale=sc)
    with pytest.raises(ValueError, match="BF16 scales"):
        rk.rht_quant_pack(x, s, out_packed=p, out_scale=sc.float())
    with pytest.raises(ValueError, match="contiguous on one CUDA device"):
        rk.rht_quant_pack(x, s, out_packed=p, out_scale=sc)
    with pytest.raises(ValueError, match="unknown layout"):
        rk.rht_quant_pack(x, s, out_packed=p, out_scale=sc, layout="nope")
    with pytest.raises(ValueError, match="Unsupported RHT configuration"):
        rk.compile_kernel(1024)
    assert rk.best_config(32, 4096) == rk.Config()


def test_block128_accepts_any_group_multiple():
    x = torch.zeros(2, 1024, dtype=torch.bfloat16)
    p, sc = bufs(2, 1024)
    # passes shape validation; stops only at the device check
    with pytest.raises(ValueError, match="CUDA device"):
        rk.rht_quant_pack(x, torch.ones(1024, dtype=torch.int8), out_packed=p, out_scale=sc, layout="block128")


def test_gemm_validation_messages():
    a = torch.zeros(4, 64, dtype=torch.int8)
    w = torch.zeros(16, 64, dtype=torch.int8)
    sa = torch.zeros(4, 1, dtype=torch.bfloat16)
    sw = torch.zeros(16, 1, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="compatible"):
        wk.w4a4_grouped_gemm(a, w[:, :32], sa, sw)
    with pytest.raises(TypeError, match="int8 storage"):
        wk.w4a4_grouped_gemm(a.to(torch.uint8), w, sa, sw)
    with pytest.raises(ValueError, match="divisible by 128"):
        wk.w4a4_grouped_gemm(a[:, :32], w[:, :32], sa, sw)
    with pytest.raises(ValueError, match=r"Sa\[M,K/128\]"):
        wk.w4a4_grouped_gemm(a, w, sa[:2], sw)
    with pytest.raises(TypeError, match="BF16"):
        wk.w4a4_grouped_gemm(a, w, sa.float(), sw)
    with pytest.raises(ValueError, match="contiguous CUDA"):
        wk.w4a4_grouped_gemm(a, w, sa, sw)
    with pytest.raises(ValueError, match="whole warps"):
        wk.compile_grouped_gemm(4, 16, 128, wk.GroupedConfig(threads=33))
    assert wk.best_grouped_config(32, 4096, 4096) == wk.GroupedConfig()
    assert wk.best_grouped_config(4096, 4096, 4096).bm == 64


def test_w4a4_linear_buffers_and_checks():
    m = W4A4Linear(4096, 6144)
    assert m.packed_weight.shape == (6144, 2048) and m.packed_weight.dtype == torch.int8
    assert m.weight_scale.shape == (6144, 32) and m.weight_scale.dtype == torch.bfloat16
    assert m.signs.shape == (4096,) and m.signs.dtype == torch.int8
    with pytest.raises(ValueError):
        W4A4Linear(4096, 6144, bias=True)
    with pytest.raises(ValueError):
        W4A4Linear(1024, 6144)                     # reference layout needs K in {4096, 12288}
    W4A4Linear(1024, 64, layout="block128", clamp_lo=-8)
    with pytest.raises(ValueError, match="BF16 activations"):
        m(torch.zeros(2, 4096))


def test_tp_module_shapes():
    col = W4A4ColumnParallelLinear(4096, 6144, tp_rank=1, tp_size=4)
    assert col.packed_weight.shape == (1536, 2048)
    mc = W4A4MergedColumnParallelLinear(4096, [12288, 12288], tp_rank=0, tp_size=8)
    assert mc.packed_weight.shape == (3072, 2048)
    qkv = W4A4QKVParallelLinear(4096, 128, 32, 8, tp_rank=3, tp_size=8)
    assert qkv.packed_weight.shape == ((4 + 2) * 128, 2048)
    row = W4A4RowParallelLinear(12288, 4096, tp_rank=7, tp_size=8)
    assert row.packed_weight.shape == (4096, 768) and row.signs.shape == (1536,)
    row_dh = W4A4RowParallelLinear(12288, 4096, tp_rank=0, tp_size=8, layout="row_DH", clamp_lo=-7)
    assert row_dh.signs.shape == (12288,) and row_dh.gather_input
    with pytest.raises(ValueError):
        W4A4RowParallelLinear(4096, 4096, tp_rank=0, tp_size=64)     # 64-wide shards


def test_w4a16_params():
    m = W4A16Linear(4096, 6144)
    assert m.qweight.shape == (512, 6144) and m.qweight.dtype == torch.int32
    assert m.qzeros.shape == (32, 768) and m.scales.dtype == torch.float16
