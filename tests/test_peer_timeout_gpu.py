"""Failure detection of the row-parallel peer exchange, without a GPU fault.

A two-rank group in which rank 1 never makes its call: both peer buffers live
on one GPU and only rank 0's kernels are launched, so the flags rank 0 waits
for are never set.  Each bounded wait must give up after its limit (2 s),
record the peer-timeout code (5) in the device error word and return -- the
call ends, nothing hangs, and the context stays usable: the next kernels run
and give correct results.  Both forms are covered: the one-shot all-reduce
(nv4_peer_allreduce_bf16) and the fused GEMM + tile reduce
(nv4_w4a4_gemm_peer_allreduce_bf16).
"""
import time

import numpy as np
import pytest
import torch

from gpu_helpers import u16
from nanovllm import _native
from nanovllm.layers.linear_w4a4 import W4A4Linear
from nanovllm.utils import synthetic
from oracle import nv4_oracle as o

pytestmark = pytest.mark.gpu

PEER_TIMEOUT = 5  # kErrTimeoutPeer
CAPACITY = 32 * 4096


def _context_still_usable(dev):
    m, n, k = 8, 256, 1024
    x, signs, _, packed, scale = synthetic.config0(seed=4, m=m, k=k, n=n)
    layer = W4A4Linear(k, n, layout="block128", clamp_lo=-8).to(dev)
    layer.load_full(packed.to(dev), scale.to(dev), signs.to(dev))
    y = layer(x.to(dev))
    torch.cuda.synchronize()
    expected = o.w4a4_linear(u16(x), signs.numpy(), packed.numpy().view(np.uint8), u16(scale), o.LAYOUT_BLOCK128, -8)
    assert np.array_equal(u16(y), expected)
    assert _native.device_error() == 0


@pytest.fixture
def lonely_pair(cuda_device):
    """Rank 0's buffer and a stand-in for rank 1's on the same GPU."""
    assert _native.device_error() == 0
    a, _ = _native.peer_buffer_alloc(CAPACITY, cuda_device)
    b, _ = _native.peer_buffer_alloc(CAPACITY, cuda_device)
    yield [a, b]
    torch.cuda.synchronize()
    _native.peer_buffer_free(a, cuda_device)
    _native.peer_buffer_free(b, cuda_device)


def _expect_timeout(start):
    torch.cuda.synchronize()
    waited = time.perf_counter() - start
    assert _native.device_error() == PEER_TIMEOUT
    assert 1.5 < waited < 30.0, waited  # the 2 s limit, not a hang


def test_allreduce_wait_runs_out(cuda_device, lonely_pair):
    out = torch.zeros(32 * 4096, dtype=torch.bfloat16, device=cuda_device)
    torch.cuda.synchronize()
    start = time.perf_counter()
    _native.peer_allreduce_bf16(lonely_pair, 0, out, out.numel(), CAPACITY)
    _expect_timeout(start)
    _context_still_usable(cuda_device)


def test_fused_gemm_reduce_wait_runs_out(cuda_device, lonely_pair):
    m, n, k = 32, 4096, 2048
    x, signs, _, packed, scale = synthetic.config0(seed=9, m=m, k=k, n=n)
    layer = W4A4Linear(k, n, layout="block128", clamp_lo=-8).to(cuda_device)
    layer.load_full(packed.to(cuda_device), scale.to(cuda_device), signs.to(cuda_device))
    codes, sa = layer.quantize_input(x.to(cuda_device))
    out = torch.zeros(m, n, dtype=torch.bfloat16, device=cuda_device)
    torch.cuda.synchronize()
    start = time.perf_counter()
    _native.w4a4_gemm_peer_allreduce_bf16(codes, layer.packed_weight, sa, layer.weight_scale, out, lonely_pair, 0,
                                          CAPACITY, _native.GEMM_W_SCALE_GROUPED)
    _expect_timeout(start)
    _context_still_usable(cuda_device)
