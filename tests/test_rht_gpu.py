"""GPU parity of the activation-prep kernel (RHT + INT4 quantisation + packing).

The kernel must reproduce the oracle bit for bit (same FP32 operation order),
and the reference fixtures everywhere except where the reference's own FP32
quotient lies within one ulp of a rounding boundary.  Also checked, as the
reference harness does (benchmarks/bench_rht_a4.py:64-115): outputs written in
place and returned, nothing written outside them, inputs unchanged, a
non-default stream, and CUDA-graph replay after the inputs change.
"""
import json
import os

import numpy as np
import pytest
import torch

import cases
from gpu_helpers import Guarded, assert_prep_matches, u16, u8
from nanovllm import _native
from nanovllm.kernels.rht_a4_tilelang import rht_quant_pack
from nanovllm.utils import synthetic
from oracle import nv4_oracle as o

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
LAYOUTS = {"block128": o.LAYOUT_BLOCK128, "row_DH": o.LAYOUT_ROW_DH}


def run_kernel(x, signs, layout, lo):
    m, k = x.shape
    packed = Guarded((m, k // 2), torch.int8, x.device, -69, 85)
    scale = Guarded((m, k // 128), torch.bfloat16, x.device, -17.0, float("nan"))
    x_before, s_before = x.clone(), signs.clone()
    ret = rht_quant_pack(x, signs, out_packed=packed.view, out_scale=scale.view, layout=layout, clamp_lo=lo)
    torch.cuda.synchronize()
    assert ret[0].data_ptr() == packed.view.data_ptr() and ret[1].data_ptr() == scale.view.data_ptr()
    assert packed.intact() and scale.intact(), "kernel wrote outside its outputs"
    assert torch.equal(x, x_before) and torch.equal(signs, s_before), "kernel modified its inputs"
    assert _native.device_error() == 0
    return u8(packed.view), u16(scale.view)


def assert_matches_oracle(x_cpu, signs_cpu, packed, sbits, layout, lo):
    ref_packed, ref_sbits, _, _, _ = o.prepare(u16(x_cpu), signs_cpu.numpy(), LAYOUTS[layout], lo)
    assert_prep_matches(packed, sbits, ref_packed, ref_sbits, o.unpack_int4)


@pytest.mark.parametrize("layout,lo", [("block128", -8), ("block128", -7), ("row_DH", -7), ("row_DH", -8)])
@pytest.mark.parametrize("k", [4096, 12288])
@pytest.mark.parametrize("m", [1, 7, 17, 31, 32, 33])
def test_matches_oracle_small(cuda_device, layout, lo, k, m):
    x = synthetic.make_input(m, k)
    signs = synthetic.make_signs(k, 20261108 + k)
    packed, sbits = run_kernel(x.to(cuda_device), signs.to(cuda_device), layout, lo)
    assert_matches_oracle(x, signs, packed, sbits, layout, lo)


@pytest.mark.parametrize("layout,k,m", [("block128", 4096, 4097), ("row_DH", 4096, 4097),
                                        ("block128", 12288, 1025), ("row_DH", 12288, 1025)])
def test_matches_oracle_large(cuda_device, layout, k, m):
    x = synthetic.activations(m, k, seed=11)
    x[:6] = synthetic.make_input(6, k)
    signs = synthetic.make_signs(k, 7)
    lo = -8 if layout == "block128" else -7
    packed, sbits = run_kernel(x.to(cuda_device), signs.to(cuda_device), layout, lo)
    assert_matches_oracle(x, signs, packed, sbits, layout, lo)


@pytest.mark.parametrize("k", [128, 512, 1152])
def test_block128_other_widths(cuda_device, k):
    x = synthetic.activations(9, k, seed=3)
    signs = synthetic.make_signs(k, 3)
    packed, sbits = run_kernel(x.to(cuda_device), signs.to(cuda_device), "block128", -8)
    assert_matches_oracle(x, signs, packed, sbits, "block128", -8)


def _fixture_cases():
    out = [("rowdh", kind, k, m, "row_DH", -7) for kind, k, m in cases.ROWDH_CASES]
    for kind, k, m in cases.BLOCK128_CASES:
        out += [(f"block128c{-lo}", kind, k, m, "block128", lo) for lo in (-8, -7)]
    return out


@pytest.mark.parametrize("lname,kind,k,m,layout,lo", _fixture_cases())
def test_reference_fixtures(cuda_device, lname, kind, k, m, layout, lo):
    data = np.load(os.path.join(GOLDEN, "prep.npz"))
    with open(os.path.join(GOLDEN, "manifest.json")) as f:
        hashes = json.load(f)["hashes"]
    key = cases.case_key(lname, kind, k, m)
    x, signs = cases.prep_case(kind, k, m)
    assert cases.sha(x, signs) == hashes[key]
    packed, sbits = run_kernel(x.to(cuda_device), signs.to(cuda_device), layout, lo)
    codes = o.unpack_int4(packed)
    ref = o.unpack_int4(data[key + "_packed"])
    near = np.unpackbits(data[key + "_near"])[: m * k].reshape(m, k).astype(bool)
    mismatch = codes != ref
    assert not (mismatch & ~near).any(), f"{int((mismatch & ~near).sum())} codes differ away from a boundary"
    assert mismatch.mean() <= 1e-4
    np.testing.assert_array_equal(sbits, data[key + "_scale"])


@pytest.mark.parametrize("layout,k", [("block128", 4096), ("row_DH", 12288)])
def test_stream_and_graph_replay(cuda_device, layout, k):
    lo = -8 if layout == "block128" else -7
    x = synthetic.make_input(32, k).to(cuda_device)
    signs = synthetic.make_signs(k, 99).to(cuda_device)
    packed = torch.empty(32, k // 2, dtype=torch.int8, device=cuda_device)
    scale = torch.empty(32, k // 128, dtype=torch.bfloat16, device=cuda_device)

    def invoke():
        rht_quant_pack(x, signs, out_packed=packed, out_scale=scale, layout=layout, clamp_lo=lo)

    for _ in range(3):
        invoke()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        packed.fill_(0)
        invoke()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    assert_matches_oracle(x.cpu(), signs.cpu(), u8(packed), u16(scale), layout, lo)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        invoke()
    for offset in (0.125, -0.25):
        x.add_(offset)
        signs.neg_()
        graph.replay()
        torch.cuda.synchronize()
        assert_matches_oracle(x.cpu(), signs.cpu(), u8(packed), u16(scale), layout, lo)


@pytest.mark.parametrize("layout,lo,k,m", [("block128", -8, 4096, 33), ("block128", -7, 12288, 7),
                                           ("row_DH", -7, 4096, 17), ("row_DH", -7, 12288, 5),
                                           ("block128", -8, 4096, 4097)])
def test_i8_layout_matches_oracle(cuda_device, layout, lo, k, m):
    """nv4_rht_quant_i8: same codes and scales as the packed form, in the GEMM-ready K order."""
    from nanovllm.kernels.rht_a4_tilelang import i8_to_codes, rht_quant_i8
    x = synthetic.activations(m, k, seed=m + k)
    x[: min(m, 6)] = synthetic.make_input(min(m, 6), k)
    signs = synthetic.make_signs(k, 5)
    d = cuda_device
    codes = Guarded((m, k), torch.int8, d, -69, 85)
    scale = Guarded((m, k // 128), torch.bfloat16, d, -17.0, float("nan"))
    rht_quant_i8(x.to(d), signs.to(d), out_codes=codes.view, out_scale=scale.view, layout=layout, clamp_lo=lo)
    torch.cuda.synchronize()
    assert codes.intact() and scale.intact()
    _, ref_sbits, ref_codes, _, _ = o.prepare(u16(x), signs.numpy(), LAYOUTS[layout], lo)
    got = i8_to_codes(codes.view.cpu()).numpy()
    assert int((got != ref_codes).sum()) == 0
    np.testing.assert_array_equal(u16(scale.view), ref_sbits)
