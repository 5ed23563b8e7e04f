"""Generate the W4A16 golden fixtures (CPU, PyTorch only).

    python tests/golden/make_w4a16_golden.py

The reference's W4A16 GEMM is a TileLang kernel
(nanovllm/layers/linear_w4a16.py:11-59) that only runs on a GPU with TileLang,
and the reference ships no W4A16 test, so it cannot be run here.  This script
restates the kernel's arithmetic in torch on the CPU, statement by statement,
and records what that restatement produces on seeded inputs:

* ``<case>_deq``  -- for the small identity case: the dequantized BF16 weights
  W [K, N] (bit patterns), i.e. ``B_dequantized`` of linear_w4a16.py:45-55;
* ``<case>_out``  -- X @ W rounded once to BF16 (bit patterns): the GEMM of
  ``T.gemm(A_shared, B_dequantized, C_local)`` (:57) with exact products and an
  exact sum (float64), correctly rounded to BF16;
* ``<case>_splitk8`` -- the reference kernel's own output order emulated: its
  launch (:132-146) splits K in 8 and adds each split's FP32 partial, rounded
  to BF16, into a zeroed BF16 output with BF16 atomics (:58-59); here the
  splits are added in order 0..7.  It differs from ``_out`` by the reference's
  BF16 accumulation error (recorded in the manifest), which is why the tests
  compare against ``_out``.

Inputs are rebuilt from seeds by ``nanovllm.utils.synthetic`` and pinned by
SHA-256 in ``w4a16_manifest.json``.
"""
from __future__ import annotations

import hashlib
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "nano-vllm-int4_b200"))
from nanovllm.utils import synthetic  # noqa: E402

GROUP = 128
# (name, m, n, k): token counts on both sides of the decode / prefill split,
# K with and without whole 256-wide chunks.
CASES = [
    ("m1_n128_k512", 1, 128, 512),
    ("m5_n192_k1024", 5, 192, 1024),
    ("m16_n256_k2048", 16, 256, 2048),
    ("m32_n128_k1536", 32, 128, 1536),
    ("m40_n64_k384", 40, 64, 384),
    ("m128_n128_k256", 128, 128, 256),
]
IDENTITY = ("identity_n128_k256", 128, 256)  # X = I_K: the output rows are W itself


def case_inputs(m: int, n: int, k: int):
    qweight, qzeros, scales = synthetic.w4a16_weights(n, k, seed=1000 + n + k)
    x = synthetic.activations(m, k, seed=2000 + m + k)
    return x, qweight, qzeros, scales


def identity_inputs(n: int, k: int):
    qweight, qzeros, scales = synthetic.w4a16_weights(n, k, seed=3000 + n + k)
    return torch.eye(k, dtype=torch.bfloat16), qweight, qzeros, scales


def sha(*tensors) -> str:
    h = hashlib.sha256()
    for t in tensors:
        h.update(t.contiguous().view(torch.uint8).numpy().tobytes())
    return h.hexdigest()


def u16(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def reference_dequant(qweight: torch.Tensor, qzeros: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """B_dequantized [K, N] BF16, restating nanovllm/layers/linear_w4a16.py:45-55."""
    k8, n = qweight.shape
    k = k8 * 8
    i = torch.arange(k)
    j = torch.arange(n)
    qw = qweight.to(torch.int64) & 0xFFFFFFFF
    qz = qzeros.to(torch.int64) & 0xFFFFFFFF
    # :45-46  packed_w = B_shared[i // 8, j]; weight_i4 = (packed_w >> ((i % 8) * 4)) & 0xF
    weight_i4 = (qw[i // 8, :] >> ((i % 8) * 4)[:, None]) & 0xF
    # :48-49  packed_z = zero_shared[j // 8]; zero_i4 = (packed_z >> ((j % 8) * 4)) & 0xF  (group of row i)
    group_id = i // GROUP
    zero_i4 = (qz[group_id][:, j // 8] >> ((j % 8) * 4)[None, :]) & 0xF
    # :51  tmp_u16 = T.cast(weight_i4 + 15 - zero_i4, "uint16") | T.uint16(0x4300)
    tmp_u16 = ((weight_i4 + 15 - zero_i4) & 0xFFFF) | 0x4300
    # :52  tmp_fp = T.reinterpret(tmp_u16, dtype="bfloat16") - T.bfloat16(128.0 + 16.0)
    tmp_fp = tmp_u16.to(torch.int16).view(torch.bfloat16) - torch.tensor(144.0, dtype=torch.bfloat16)
    # :40 / :54  scale_shared is a BF16 copy of the FP16 scales; B = tmp_fp * scale_shared[j] in BF16
    scale_shared = scales.to(torch.bfloat16)[group_id]
    return tmp_fp * scale_shared


def bf16_bits_of_f64(v: np.ndarray) -> np.ndarray:
    """Correctly rounded (ties to even) BF16 bit patterns of float64 values."""
    mant, exp = np.frexp(v)
    r = np.ldexp(np.rint(mant * 256.0) / 256.0, exp)
    return (r.astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)


def bf16_value(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32).astype(np.float64)


def exact_product(x: torch.Tensor, w: torch.Tensor) -> np.ndarray:
    """X @ W of BF16 operands in float64 (each product exact)."""
    return x.double().numpy() @ w.double().numpy()


def splitk8_reference_order(x: torch.Tensor, w: torch.Tensor) -> np.ndarray:
    """The reference launch's output (:132-146, SPLIT_K = 8): per split an FP32
    partial (float64 here, then rounded to FP32), cast to BF16 (:57), added into
    a zeroed BF16 output one split after another, each addition rounded to BF16."""
    k = x.shape[1]
    split = k // 8
    out = np.zeros((x.shape[0], w.shape[1]), dtype=np.float64)
    for s in range(8):
        part = exact_product(x[:, s * split:(s + 1) * split], w[s * split:(s + 1) * split])
        part_bf16 = bf16_value(bf16_bits_of_f64(part.astype(np.float32).astype(np.float64)))
        out = bf16_value(bf16_bits_of_f64(out + part_bf16))
    return out


def main():
    out, hashes, stats = {}, {}, {}
    for name, m, n, k in CASES:
        x, qweight, qzeros, scales = case_inputs(m, n, k)
        w = reference_dequant(qweight, qzeros, scales)
        exact = exact_product(x, w)
        out[name + "_out"] = bf16_bits_of_f64(exact)
        if k % 256 == 0:  # the reference's 8 splits of BLOCK_K = 32 need K % 256 == 0
            ref8 = splitk8_reference_order(x, w)
            out[name + "_splitk8"] = bf16_bits_of_f64(ref8)
            ours = bf16_value(out[name + "_out"])
            stats[name] = {"rel_l2_splitk8_vs_exact_bf16": float(np.linalg.norm(ref8 - ours) / np.linalg.norm(ours))}
        hashes[name] = sha(x, qweight, qzeros, scales)
    name, n, k = IDENTITY
    x, qweight, qzeros, scales = identity_inputs(n, k)
    w = reference_dequant(qweight, qzeros, scales)
    out[name + "_deq"] = u16(w)
    hashes[name] = sha(qweight, qzeros, scales)
    np.savez_compressed(os.path.join(HERE, "w4a16.npz"), **out)
    with open(os.path.join(HERE, "w4a16_manifest.json"), "w") as f:
        json.dump({"generator": "tests/golden/make_w4a16_golden.py", "hashes": hashes, "stats": stats,
                   "torch": torch.__version__}, f, indent=1, sort_keys=True)
    print(json.dumps(stats, indent=1))


if __name__ == "__main__":
    main()
