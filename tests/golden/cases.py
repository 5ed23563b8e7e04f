"""Input construction for the golden fixtures (pure torch on CPU, no reference import).

``make_golden.py`` builds these inputs, runs the reference implementation on
them and stores the reference outputs; the tests rebuild the same inputs from
the same seeds (CPU ``torch.Generator`` is deterministic) and check a SHA-256
of them against the one stored beside the outputs.
"""
from __future__ import annotations

import hashlib
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(os.path.dirname(os.path.dirname(HERE)), "nano-vllm-int4_b200")
if PKG not in sys.path:
    sys.path.insert(0, PKG)

from nanovllm.utils import synthetic  # noqa: E402

# (layout, name, builder) cases for the activation-prep fixtures.
ROWDH_CASES = [("input", 4096, m) for m in (1, 7, 17, 33)] + \
              [("input", 12288, m) for m in (1, 7)] + \
              [("extremes", 4096, 33), ("extremes", 12288, 10)]
BLOCK128_CASES = [("config0", 4096, 16), ("input", 4096, 7), ("input", 4096, 33),
                  ("input", 12288, 7), ("extremes", 4096, 33)]
GEMM_SHAPES = [(17, 96, 512), (33, 136, 4096), (32, 128, 12288)]


def sha(*tensors) -> str:
    h = hashlib.sha256()
    for t in tensors:
        a = t.contiguous().view(torch.uint8) if isinstance(t, torch.Tensor) else np.ascontiguousarray(t)
        h.update(np.asarray(a).tobytes())
    return h.hexdigest()


def prep_case(kind: str, k: int, m: int):
    """(x bf16 [m,k], signs int8 [k]) for one activation-prep fixture."""
    if kind == "config0":
        x, signs, *_ = synthetic.config0(seed=0, m=m, k=k)
        return x, signs
    if kind == "input":
        x = synthetic.make_input(m, k)
    elif kind == "extremes":
        x = synthetic.exponent_extremes(m, k)
    else:
        raise ValueError(kind)
    return x, synthetic.make_signs(k, 20261108 + k)


def case_key(layout: str, kind: str, k: int, m: int) -> str:
    return f"{layout}_{kind}_k{k}_m{m}"


def gemm_case(m: int, n: int, k: int, grouped: bool):
    """Inputs of the reference GEMM checks (verify_w4a4_aw_grouped.py:154-162 for
    grouped weight scales, verify_w4a4_grouped.py:37-45 for per-channel), generated
    on the CPU from the same seeds."""
    seed = 20261110 if grouped else 20261109
    g = torch.Generator(device="cpu").manual_seed(seed + 1000003 * m + 1009 * n + k)
    qa = torch.randint(-8, 8, (m, k), generator=g, dtype=torch.int8)
    qw = torch.randint(-8, 8, (n, k), generator=g, dtype=torch.int8)
    qa[0].zero_()
    qw[0].zero_()
    sa = (torch.rand(m, k // 128, generator=g) * 2).bfloat16()
    if grouped:
        sw = (torch.rand(n, k // 128, generator=g) * .03).bfloat16()
        sa[1, ::2] = 0
        sw[1, 1::2] = 0
    else:
        sw = (torch.rand(n, generator=g) * .03).bfloat16()
        sa[1, ::2] = 0
        sw[1] = 0
    return qa, qw, sa.contiguous(), sw.contiguous()


def gemm_key(m, n, k, grouped):
    return f"{'aw' if grouped else 'a'}_m{m}_n{n}_k{k}"
