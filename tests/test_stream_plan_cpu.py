"""The decode stream GEMM's launch planner (nv4_w4a4_stream_plan, host code
only): every Qwen3-8B projection, every tensor-parallel shard of it and every
token count the stream kernel serves must get a plan that keeps the kernel's
invariants.  The stage-ring invariant matters most: producer warps reuse a
ring slot after a parity wait on its empty barrier, which is sound only when
the ring holds at least min(K stages, K-split warps + producer warps) slots;
a plan below it lets a TMA copy overwrite a stage still being read."""
import pytest

from nanovllm import _native

SHAPES = {"qkv": (6144, 4096), "o": (4096, 4096), "gate_up": (24576, 4096), "down": (4096, 12288)}
ROW_PARALLEL = ("o", "down")
SMEM_LIMIT = 227 * 1024


def shard(name, tp):
    n, k = SHAPES[name]
    return (n, k // tp) if name in ROW_PARALLEL else (n // tp, k)


def check_plan(pl, m, n, k, peer):
    assert pl is not None, (m, n, k, peer)
    g = k // 128
    assert pl["n_iters"] == (g + 1) // 2
    # the ring rule
    assert pl["stages"] >= min(pl["n_iters"], pl["k_split"] + pl["producer_warps"]), pl
    assert 1 <= pl["stages"] <= 16
    assert pl["smem_bytes"] <= SMEM_LIMIT
    assert pl["threads"] <= 1024 and pl["threads"] % 32 == 0
    assert pl["threads"] == 32 * (pl["producer_warps"] + pl["slabs"] * pl["token_splits"] * pl["k_split"])
    assert pl["rows_per_cta"] == 16 * pl["slabs"]
    assert pl["grid_x"] * pl["rows_per_cta"] >= n > (pl["grid_x"] - 1) * pl["rows_per_cta"]
    mp = 8 * pl["token_tiles"]
    assert pl["grid_y"] == -(-m // mp)
    assert pl["token_tiles"] == pl["token_splits"] * pl["tiles_per_warp"]
    # template instances the launcher has (token tiles, tiles per warp, K split)
    assert (pl["token_tiles"], pl["tiles_per_warp"], pl["k_split"]) in {
        (1, 1, 1), (1, 1, 4), (2, 1, 1), (2, 2, 1), (2, 2, 4), (4, 1, 1), (4, 2, 1), (4, 4, 1), (4, 2, 4), (4, 4, 4)}
    if peer:
        assert pl["grid_y"] == 1 and pl["grid_x"] <= 256


@pytest.mark.parametrize("tp", [1, 2, 4, 8])
@pytest.mark.parametrize("name", list(SHAPES))
def test_plans_of_every_projection_shard(name, tp):
    n, k = shard(name, tp)
    for m in range(1, 65):
        check_plan(_native.w4a4_stream_plan(m, n, k), m, n, k, False)
        if name in ROW_PARALLEL and tp > 1 and m <= _native.PEER_MAX_TOKENS:
            check_plan(_native.w4a4_stream_plan(m, n, k, peer=True), m, n, k, True)


@pytest.mark.parametrize("sms", [1, 8, 132, 148, 160])
def test_plans_hold_for_other_sm_counts(sms):
    for n, k in [(8, 128), (64, 256), (6144, 4096), (24576, 4096), (4096, 12288), (4096, 1536), (3072, 4096)]:
        for m in (1, 8, 9, 16, 17, 32, 33, 64):
            pl = _native.w4a4_stream_plan(m, n, k, sm_count=sms)
            check_plan(pl, m, n, k, False)


def test_wide_peer_outputs_fit_the_flag_slots():
    # A wide row-parallel output: the plan takes more rows per CTA so that the
    # grid stays within the 256 per-CTA flag slots, or reports it cannot.
    for n in (8192, 16384, 24576, 32768):
        pl = _native.w4a4_stream_plan(32, n, 4096, peer=True)
        if pl is not None:
            check_plan(pl, 32, n, 4096, True)
    pl = _native.w4a4_stream_plan(32, 4096, 1536, peer=True)
    check_plan(pl, 32, 4096, 1536, True)


def test_plan_rejects_bad_shapes():
    lib = _native.load()
    import ctypes
    out = (ctypes.c_int32 * len(_native.STREAM_PLAN_FIELDS))()
    assert lib.nv4_w4a4_stream_plan(0, 64, 128, 1, 148, 0, out) == _native.ERR_INVALID_ARGUMENT
    assert lib.nv4_w4a4_stream_plan(1, 64, 100, 1, 148, 0, out) == _native.ERR_INVALID_ARGUMENT
    assert lib.nv4_w4a4_stream_plan(1, 64, 128, 1, 0, 0, out) == _native.ERR_INVALID_ARGUMENT
    assert lib.nv4_w4a4_stream_plan(1, 64, 128, 1, 148, 0, None) == _native.ERR_INVALID_ARGUMENT
