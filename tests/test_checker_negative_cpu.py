"""Negative control of the parity gates (the reference harness's own control,
benchmarks/bench_rht_a4.py:143-152: the checker must fail on one corrupt
code, not just report that it ran).  The mistake is planted in a copy of the
oracle's output on the CPU; the gate the GPU tests use must reject it, and
accept the untouched copy."""
import numpy as np
import pytest
import torch

from gpu_helpers import assert_prep_matches
from nanovllm.utils import synthetic
from oracle import nv4_oracle as o


@pytest.mark.parametrize("layout,k", [(o.LAYOUT_BLOCK128, 4096), (o.LAYOUT_ROW_DH, 12288)])
def test_prep_gate_rejects_one_corrupt_code(layout, k):
    x = synthetic.activations(1, k, seed=3)
    signs = synthetic.make_signs(k, 0).numpy()
    bits = x.contiguous().view(torch.int16).numpy().view(np.uint16)
    packed, sbits, _, _, _ = o.prepare(bits, signs, layout, -7)
    assert_prep_matches(packed.copy(), sbits.copy(), packed, sbits, o.unpack_int4)  # accepts the truth
    bad = packed.copy()
    bad[0, 0] ^= 1  # the reference control's corruption: one bit of the first packed byte
    with pytest.raises(AssertionError, match="Quantizer parity failed: 1 codes"):
        assert_prep_matches(bad, sbits, packed, sbits, o.unpack_int4)
    bad_scale = sbits.copy()
    bad_scale[0, 0] ^= 1
    with pytest.raises(AssertionError, match="0 codes and 1 scales"):
        assert_prep_matches(packed, bad_scale, packed, sbits, o.unpack_int4)
