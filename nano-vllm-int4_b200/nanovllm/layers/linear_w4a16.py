"""GPTQ W4A16 linear (drop-in for ``nanovllm/layers/linear_w4a16.py:98-147``).

Parameters keep the GPTQ names, dtypes and layouts the reference loads
(``qweight`` int32 [K/8, N], ``qzeros`` int32 [K/128, N/8], ``scales`` fp16
[K/128, N]).  The forward is one call into libnv4's sm_100a dequant GEMM
(plus, for small M, an FP32 split-K workspace from torch's caching allocator,
so CUDA-graph capture keeps working).  Unlike the reference it does not need a
zero-filled output and sums split-K partials in FP32 instead of BF16 atomics.
"""
import torch
from torch import nn

from nanovllm import _native


class W4A16Linear(nn.Module):

    def __init__(self, in_features, out_features, group_size=128):
        super().__init__()
        assert group_size == 128
        self.in_features = in_features
        self.out_features = out_features
        self.group_size = group_size
        self.qweight = nn.Parameter(torch.empty(in_features // 8, out_features, dtype=torch.int32),
                                    requires_grad=False)
        self.qzeros = nn.Parameter(torch.empty(in_features // group_size, out_features // 8, dtype=torch.int32),
                                   requires_grad=False)
        self.scales = nn.Parameter(torch.empty(in_features // group_size, out_features, dtype=torch.float16),
                                   requires_grad=False)

    def forward(self, x):
        shape = x.shape
        x = x.reshape(-1, self.in_features)
        if x.dtype != torch.bfloat16:
            raise ValueError("W4A16Linear requires BF16 activations")
        x = x.contiguous()
        m = x.shape[0]
        out = torch.empty((m, self.out_features), device=x.device, dtype=torch.bfloat16)
        ws_bytes = _native.w4a16_workspace_bytes(m, self.out_features, self.in_features, x.device)
        workspace = torch.empty(ws_bytes // 4, device=x.device, dtype=torch.float32) if ws_bytes else None
        _native.w4a16_gemm(x, self.qweight, self.qzeros, self.scales, out, self.group_size, workspace)
        return out.reshape(*shape[:-1], self.out_features)
