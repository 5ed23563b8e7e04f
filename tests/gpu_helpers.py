"""Shared helpers of the GPU parity tests: canary-guarded output buffers and
conversions between torch tensors and the oracle's numpy arrays."""
import numpy as np
import torch


def u16(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def u8(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.uint8).numpy()


class Guarded:
    """An output tensor carved out of a larger buffer whose 64-element margins
    hold a canary value; ``intact()`` checks nothing was written outside."""

    def __init__(self, shape, dtype, device, canary, fill):
        n = int(np.prod(shape))
        self.store = torch.full((n + 128,), canary, dtype=dtype, device=device)
        self.head = self.store[:64].clone()
        self.view = self.store[64:64 + n].view(*shape)
        self.view.fill_(fill)

    def intact(self) -> bool:
        return bool(torch.equal(self.store[:64], self.head) and torch.equal(self.store[-64:], self.head))


def bf16_bits_to_float(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


def assert_prep_matches(packed: np.ndarray, sbits: np.ndarray, ref_packed: np.ndarray, ref_sbits: np.ndarray,
                        unpack) -> None:
    """The activation-prep parity gate (the reference harness's `compare`,
    benchmarks/bench_rht_a4.py:55-61): every INT4 code and every BF16 scale
    equal, else AssertionError naming how many differ."""
    mism_codes = int((unpack(packed) != unpack(ref_packed)).sum())
    mism_scales = int((sbits != ref_sbits).sum())
    assert mism_codes == 0 and mism_scales == 0, \
        f"Quantizer parity failed: {mism_codes} codes and {mism_scales} scales differ from the oracle"


def codes_to_i8_layout(codes: torch.Tensor) -> torch.Tensor:
    """int8 codes [M, K] in k order -> the GEMM-ready layout of nv4_rht_quant_i8:
    within each 32-wide K chunk, the 16 even-k codes then the 16 odd-k codes."""
    m, k = codes.shape
    return codes.reshape(m, k // 32, 16, 2).permute(0, 1, 3, 2).reshape(m, k).contiguous()
