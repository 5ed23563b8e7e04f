"""The W4A16 dispatch and split planner (nv4_w4a16_plan, host code only).

Up to 16 tokens the weight-streaming decode kernel runs with a cluster K split
whose slices are whole 256-K TMA chunks (at most eight per CTA); above that the
tcgen05 kernel runs, splitting K into 2-8 slices only when its tiles leave
SMs idle in their last round; its FP32 partials then need splits x m x n
floats of workspace.  Every Qwen3-8B projection, its tensor-parallel shards and a sweep
of token counts must get a plan that keeps these rules; the config-3 shapes
pin the measured choices (decode kernel at 1 and 16 tokens, K split at 32 and
128 tokens, none at 2048)."""
import pytest

from nanovllm import _native

SHAPES = {"qkv": (6144, 4096), "o": (4096, 4096), "gate_up": (24576, 4096), "down": (4096, 12288)}
ROW_PARALLEL = ("o", "down")
SMS = _native.SM_COUNT_B200
TOKENS = list(range(1, 41)) + [48, 64, 100, 127, 128, 129, 200, 256, 300, 512, 1000, 2048, 4096]


def shard(name, tp):
    n, k = SHAPES[name]
    return (n, k // tp) if name in ROW_PARALLEL else (n // tp, k)


def check_plan(pl, m, n, k):
    if pl["kernel"] == _native.W4A16_KERNEL_DECODE:
        assert m <= 16 and pl["token_tile"] == 16 and pl["workspace_bytes"] == 0
        ks = pl["splits"]
        assert ks in (1, 2, 4, 8)
        assert (k // ks) % 256 == 0 and k // ks <= 8 * 256  # whole TMA chunks, at most eight per CTA
        assert pl["ctas"] == (n // 64) * ks
    elif pl["kernel"] == _native.W4A16_KERNEL_TC:
        assert m > 16
        assert pl["token_tile"] == (256 if m > 128 else 128)
        s = pl["splits"]
        assert 1 <= s <= 8 and s <= k // 64  # every slice has at least one 64-K chunk
        units = -(-n // 128) * -(-m // pl["token_tile"]) * s
        assert pl["ctas"] == min(units, SMS)
        assert pl["workspace_bytes"] == (s * m * n * 4 if s > 1 else 0)
        if s > 1:  # split only when the unsplit tiles leave SMs idle in their last round
            assert (-(-n // 128) * -(-m // pl["token_tile"])) % SMS != 0
    else:
        pytest.fail(f"mma.sync fallback planned for an aligned Qwen3 shape: {m}x{n}x{k} {pl}")


@pytest.mark.parametrize("tp", [1, 2, 4, 8])
@pytest.mark.parametrize("name", sorted(SHAPES))
def test_every_projection_and_shard(name, tp):
    n, k = shard(name, tp)
    for m in TOKENS:
        check_plan(_native.w4a16_plan(m, n, k), m, n, k)


def test_config3_choices():
    qkv, gate_up, down = SHAPES["qkv"], SHAPES["gate_up"], SHAPES["down"]
    for m in (1, 16):
        for n, k in (qkv, gate_up, down):
            assert _native.w4a16_plan(m, n, k)["kernel"] == _native.W4A16_KERNEL_DECODE
    for m in (17, 32, 128):
        for n, k in (qkv, gate_up, down):
            assert _native.w4a16_plan(m, n, k)["kernel"] == _native.W4A16_KERNEL_TC
    # K slices at 128 tokens: qkv 3 (uneven: 21/21/22 chunks), gate/up 2, down 4
    assert [_native.w4a16_plan(128, n, k)["splits"] for n, k in (qkv, gate_up, down)] == [3, 2, 4]
    for n, k in (qkv, gate_up, down):
        pl = _native.w4a16_plan(2048, n, k)
        assert pl["splits"] == 1 and pl["token_tile"] == 256 and pl["workspace_bytes"] == 0


def test_rejects_what_the_gemm_rejects():
    for m, n, k in ((0, 4096, 4096), (1, 4096 + 32, 4096), (1, 4096, 4096 + 64), (1, 32, 4096)):
        with pytest.raises(ValueError):
            _native.w4a16_plan(m, n, k)
    with pytest.raises(ValueError):
        _native.w4a16_plan(1, 4096, 4096, sm_count=0)
