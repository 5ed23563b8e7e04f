"""Generate the golden fixtures from the reference implementation (CPU).

Run once where the reference sources are present (``$NANOVLLM_REF``, default
the read-only reference checkout); the outputs are committed so that tests on
machines without the reference still have them:

    NANOVLLM_REF=<reference checkout> python tests/golden/make_golden.py

What it records, all produced by the reference's own PyTorch code on the CPU:

* ``kat.npz`` -- the known-answer vectors of ``bench_rht_a4.oracle_checks``
  (``benchmarks/bench_rht_a4.py:17-52``), after running that function: impulse
  responses of the K=4096 and K=12288 transforms, the tie/clamp row, the
  BF16-scale-before-codes row, zero and tiny groups, and the packed bytes of the
  codes -8..7.
* ``prep.npz`` -- activation codes (packed) and BF16 scales for
  - layout ``row_DH_paley12_kron_sylvester_v1`` via
    ``rht_a4_bench_common.reference_parts`` (``a4.rotate`` + ``quantize_rotated``,
    clamp [-7, 7]);
  - layout ``block128`` via ``rht_reference.fwht`` on [M, K/128, 128] after the
    sign multiply, then ``quantize_rotated``'s formula with clamp_lo -8 and -7
    (the one-line clamp is the only restated step);
  plus, per case, a bit mask of elements whose reference FP32 quotient x/scale
  lies within 1 ulp of a rounding boundary.
* ``gemm.npz`` -- FP32 and BF16 results of ``verify_w4a4_aw_grouped.reference``
  (grouped weight scales) and ``verify_w4a4_grouped.reference`` (per-channel)
  on the reference test shapes.
* ``config0.npz`` -- the whole config-0 chain (block128, clamp -8): packed
  activations, scales and the BF16 output of the grouped GEMM reference.
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import cases  # noqa: E402

REF = os.environ.get("NANOVLLM_REF", "/root/reference")
sys.path.insert(0, os.path.join(REF, "benchmarks"))
sys.path.insert(0, REF)

import a4_group_quant as a4  # noqa: E402
import bench_rht_a4  # noqa: E402
import rht_a4_bench_common as common  # noqa: E402
import rht_reference as ref  # noqa: E402
import verify_w4a4_aw_grouped as vaw  # noqa: E402
import verify_w4a4_grouped as va  # noqa: E402

sys.path.insert(0, os.path.join(os.path.dirname(HERE), ".."))
from oracle import nv4_oracle as oracle  # noqa: E402  (boundary mask helper only)


def u16(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def u8(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.uint8).numpy()


def quantize_clamped(rotated: torch.Tensor, clamp_lo: int):
    """a4_group_quant.quantize_rotated (a4_group_quant.py:206-216) with a clamp_lo argument."""
    x = rotated.float()
    m, k = x.shape
    grouped = x.reshape(m, k // 128, 128)
    maximum = grouped.abs().amax(-1)
    scale = torch.where(maximum == 0, 1.0,
                        (maximum * 0.9 / 7).clamp_min(torch.finfo(torch.bfloat16).tiny)).bfloat16()
    quotient = grouped / scale.float().unsqueeze(-1)
    codes = quotient.round().clamp(clamp_lo, 7)
    return codes.reshape(m, k).to(torch.int8), scale, quotient.reshape(m, k)


def kat():
    report = bench_rht_a4.oracle_checks()
    out = {"report": np.array(json.dumps(report))}
    for k, index in [(4096, 5), (12288, 1024)]:
        x = torch.zeros(1, k, dtype=torch.float64)
        x[0, index] = 1
        out[f"impulse_k{k}_i{index}"] = ref.rht(x, torch.ones(k, dtype=torch.int8))[0].numpy()
    values = torch.zeros(1, 128)
    values[0, :10] = torch.tensor([-7.5, -6.5, -4.5, -2.5, -.5, .5, 2.5, 4.5, 6.5, 7.5])
    values[0, -1] = 7 / .9
    codes, scales = a4.quantize_rotated(values, 128, .9)
    out["ties_values"], out["ties_codes"], out["ties_scale"] = values.numpy(), codes.numpy(), scales.float().numpy()
    raw = torch.tensor(.9 / 7)
    rounded = raw.bfloat16().float()
    values = torch.zeros(1, 128)
    values[0, 0] = 1
    values[0, 1] = 2.5 * (raw + rounded) / 2
    codes, scales = a4.quantize_rotated(values, 128, .9)
    out["bf16first_values"], out["bf16first_codes"], out["bf16first_scale"] = \
        values.numpy(), codes.numpy(), scales.float().numpy()
    for name, magnitude in [("zero", 0.), ("tiny", 1e-40)]:
        values = torch.full((1, 128), magnitude)
        codes, scales = a4.quantize_rotated(values, 128, .9)
        out[f"{name}_values"], out[f"{name}_codes"], out[f"{name}_scale"] = \
            values.numpy(), codes.numpy(), scales.float().numpy()
    codes = torch.arange(-8, 8, dtype=torch.int8).reshape(1, 16)
    out["pack_codes"], out["pack_bytes"] = codes.numpy(), u8(ref.pack_int4(codes))
    return out


def prep():
    out, hashes = {}, {}
    for kind, k, m in cases.ROWDH_CASES:
        x, signs = cases.prep_case(kind, k, m)
        rotated, codes, scales = common.reference_parts(x, signs)
        quotient = rotated.reshape(m, k // 128, 128) / scales.float().unsqueeze(-1)
        key = cases.case_key("rowdh", kind, k, m)
        out[key + "_packed"] = u8(ref.pack_int4(codes))
        out[key + "_scale"] = u16(scales)
        out[key + "_near"] = np.packbits(oracle.boundary_mask(quotient.reshape(m, k).numpy(), 1))
        hashes[key] = cases.sha(x, signs)
    for kind, k, m in cases.BLOCK128_CASES:
        x, signs = cases.prep_case(kind, k, m)
        rotated = ref.fwht((x.float() * signs.float()).reshape(m, k // 128, 128)).reshape(m, k)
        for lo in (-8, -7):
            codes, scales, quotient = quantize_clamped(rotated, lo)
            key = cases.case_key(f"block128c{-lo}", kind, k, m)
            out[key + "_packed"] = u8(ref.pack_int4(codes))
            out[key + "_scale"] = u16(scales)
            out[key + "_near"] = np.packbits(oracle.boundary_mask(quotient.numpy(), 1))
            hashes[key] = cases.sha(x, signs)
    return out, hashes


def gemm():
    out, hashes = {}, {}
    for grouped in (True, False):
        for m, n, k in cases.GEMM_SHAPES:
            qa, qw, sa, sw = cases.gemm_case(m, n, k, grouped)
            key = cases.gemm_key(m, n, k, grouped)
            expected = vaw.reference(qa, qw, sa, sw) if grouped else va.reference(qa, qw, sa, sw)
            out[key + "_f32"] = expected.numpy().astype(np.float32)
            out[key + "_bf16"] = u16(expected.bfloat16())
            if grouped:
                precise = vaw.reference(qa, qw, sa, sw, precise=True)
            else:
                precise = va.reference(qa, qw, sa, sw, torch.float64)
            out[key + "_f64"] = precise.numpy()
            hashes[key] = cases.sha(qa, qw, sa, sw)
    return out, hashes


def config0():
    x, signs, codes_w, packed_w, sw = cases.synthetic.config0(seed=0)
    rotated = ref.fwht((x.float() * signs.float()).reshape(16, 32, 128)).reshape(16, 4096)
    codes, scales, _ = quantize_clamped(rotated, -8)
    y = vaw.reference(codes, codes_w, scales, sw)
    return ({"packed": u8(ref.pack_int4(codes)), "scale": u16(scales),
             "out_bf16": u16(y.bfloat16())},
            {"config0": cases.sha(x, signs, packed_w, sw)})


def main():
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    manifest = {"generator": "tests/golden/make_golden.py", "torch": torch.__version__, "hashes": {}}
    np.savez_compressed(os.path.join(HERE, "kat.npz"), **kat())
    for name, fn in [("prep", prep), ("gemm", gemm), ("config0", config0)]:
        data, hashes = fn()
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **data)
        manifest["hashes"].update(hashes)
    with open(os.path.join(HERE, "manifest.json"), "w") as f:
        json.dump(manifest, f, indent=1, sort_keys=True)
        f.write("\n")
    print(json.dumps({"written": ["kat.npz", "prep.npz", "gemm.npz", "config0.npz", "manifest.json"]}))


if __name__ == "__main__":
    main()
