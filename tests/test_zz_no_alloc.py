"""nv4_w4a16_gemm_static, the allocation-free W4A16 entry point, called through
the C ABI and compared with nv4_w4a16_gemm (caller workspace) on the same
inputs.  This file is collected last so that it also runs after every other
GPU test in one process; it passes alone as well."""
import ctypes

import numpy as np
import pytest
import torch

from nanovllm import _native
from nanovllm.utils import synthetic
from oracle import nv4_oracle as o
from gpu_helpers import u16

V = ctypes.c_void_p


def _ptr(t):
    return V(t.data_ptr())


def _stream(device):
    return V(torch.cuda.current_stream(device).cuda_stream)


def test_static_scratch_limit_rejected_before_launch():
    """m <= 16 with m * n above the scratch returns NV4_ERR_UNSUPPORTED from
    the argument checks (no device work, so no GPU is needed)."""
    lib = _native.load()
    limit = _native.W4A16_STATIC_SCRATCH_FLOATS
    n_over = (limit // 16 // 64 + 1) * 64
    args = (V(256), V(256), V(256), V(256), V(256))
    assert lib.nv4_w4a16_gemm_static(*args, 16, n_over, 4096, 128, None) == _native.ERR_UNSUPPORTED
    assert lib.nv4_w4a16_gemm_static(*args, 1, 64, 4096, 64, None) == _native.ERR_UNSUPPORTED     # group 64
    assert lib.nv4_w4a16_gemm_static(None, *args[1:], 1, 64, 4096, 128, None) == _native.ERR_INVALID_ARGUMENT
    assert lib.nv4_w4a16_gemm_static(*args, 1, 96, 4096, 128, None) == _native.ERR_INVALID_ARGUMENT  # n % 64


def _device_inputs(m, n, k, device):
    qweight, qzeros, scales = synthetic.w4a16_weights(n, k, seed=n + k + m)
    x = synthetic.activations(m, k, seed=7 * m + 1)
    return x, qweight, qzeros, scales, [t.to(device) for t in (x, qweight, qzeros, scales)]


@pytest.mark.gpu
@pytest.mark.parametrize("m,n,k", [(1, 6144, 4096), (4, 4096, 12288), (16, 24576, 4096), (64, 2048, 4096)])
def test_static_matches_workspace_entry(cuda_device, m, n, k):
    lib = _native.load()
    x, qweight, qzeros, scales, (xd, qwd, qzd, sd) = _device_inputs(m, n, k, cuda_device)
    stream = _stream(cuda_device)

    ws_bytes = lib.nv4_w4a16_workspace_bytes(m, n, k)
    workspace = torch.empty(max(ws_bytes // 4, 1), dtype=torch.float32, device=cuda_device)
    ref = torch.empty((m, n), dtype=torch.bfloat16, device=cuda_device)
    assert lib.nv4_w4a16_gemm(_ptr(xd), _ptr(qwd), _ptr(qzd), _ptr(sd), _ptr(ref), m, n, k, 128,
                              _ptr(workspace), ws_bytes, stream) == _native.OK

    expected = o.w4a16_gemm_f64(u16(x), qweight.numpy(), qzeros.numpy(), scales.numpy())
    ref_f = ref.float().cpu().numpy().astype(np.float64)
    outs = []
    for _ in range(2):  # two calls in a row: the scratch is cleared by each call
        out = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device=cuda_device)
        assert lib.nv4_w4a16_gemm_static(_ptr(xd), _ptr(qwd), _ptr(qzd), _ptr(sd), _ptr(out), m, n, k, 128,
                                         stream) == _native.OK
        outs.append(out.float().cpu().numpy().astype(np.float64))
    assert _native.device_error() == 0
    for got in outs:
        assert np.isfinite(got).all()
        # Split-K partials are added with FP32 atomics in any order, so the two
        # entry points may differ by a BF16 rounding of a slightly different sum.
        assert np.linalg.norm(got - ref_f) / np.linalg.norm(ref_f) < 1e-3
        assert np.mean(got == ref_f) > 0.95
        assert np.linalg.norm(got - expected) / np.linalg.norm(expected) < 4e-3   # tolerance of the W4A16 tests


@pytest.mark.gpu
def test_static_python_binding(cuda_device):
    m, n, k = 8, 4096, 4096
    x, qweight, qzeros, scales, (xd, qwd, qzd, sd) = _device_inputs(m, n, k, cuda_device)
    out = torch.empty((m, n), dtype=torch.bfloat16, device=cuda_device)
    _native.w4a16_gemm_static(xd, qwd, qzd, sd, out, 128)
    expected = o.w4a16_gemm_f64(u16(x), qweight.numpy(), qzeros.numpy(), scales.numpy())
    got = out.float().cpu().numpy().astype(np.float64)
    assert np.linalg.norm(got - expected) / np.linalg.norm(expected) < 4e-3
    big = torch.empty((16, _native.W4A16_STATIC_SCRATCH_FLOATS // 16 + 64), dtype=torch.bfloat16,
                      device=cuda_device)
    qw_big = torch.zeros((k // 8, big.shape[1]), dtype=torch.int32, device=cuda_device)
    with pytest.raises(ValueError, match="static scratch"):
        _native.w4a16_gemm_static(torch.zeros((16, k), dtype=torch.bfloat16, device=cuda_device), qw_big,
                                  qzd, sd, big, 128)
