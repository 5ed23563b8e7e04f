"""ctypes binding of libnv4.so, the sm_100a kernel library (C ABI in include/nv4.h).

This is the only route from Python to the kernels.  There is no fallback: if
the library is missing, or the current device is not an sm_100 GPU, every
entry point raises.  Tensors are passed as raw device pointers and the work is
enqueued on torch's current stream of the tensors' device, so calls compose
with torch's stream semantics and CUDA-graph capture.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_lib", "libnv4.so")

OK = 0
ERR_INVALID_ARGUMENT = -1
ERR_UNSUPPORTED = -2
ERR_ALIGNMENT = -3
ERR_CUDA = -4
ERR_DEVICE = -5

LAYOUT_BLOCK128 = 0
LAYOUT_ROW_DH = 1
LAYOUTS = {"block128": LAYOUT_BLOCK128, "row_DH_paley12_kron_sylvester_v1": LAYOUT_ROW_DH,
           "row_dh": LAYOUT_ROW_DH, "row_DH": LAYOUT_ROW_DH}

GEMM_W_SCALE_GROUPED = 1
GEMM_OUT_FP32 = 2
GEMM_FORCE_STREAM = 4

EXPORTS = ("nv4_rht_quant_pack", "nv4_rht_quant_i8", "nv4_w4a4_grouped_gemm", "nv4_w4a4_gemm_i8", "nv4_w4a4_group_dots", "nv4_w4a16_gemm",
           "nv4_w4a16_workspace_bytes", "nv4_version", "nv4_status_string", "nv4_last_cuda_error",
           "nv4_device_error", "nv4_w4a16_gemm_static", "nv4_peer_header_bytes", "nv4_peer_buffer_alloc",
           "nv4_peer_buffer_open", "nv4_peer_buffer_close", "nv4_peer_buffer_free", "nv4_peer_allreduce_bf16",
           "nv4_w4a4_gemm_peer_allreduce_bf16", "nv4_silu_mul_rht_quant_i8",
           "nv4_add_rmsnorm_rht_quant_i8", "nv4_w4a4_stream_plan", "nv4_paged_attention_workspace_bytes",
           "nv4_paged_decode_attention", "nv4_qk_norm_rope_store", "nv4_w4a16_plan")


class NativeLibraryError(RuntimeError):
    """libnv4.so is missing or failed to load."""


class NativeCallError(RuntimeError):
    """A libnv4 entry point returned an error status."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


_lib = None
_lock = threading.Lock()
_vp, _i64, _int = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int


def _check_fresh(path: str) -> None:
    """Refuse a library built from other sources than the ones beside it (when
    the sources are present): a stale binary would silently run old kernels."""
    pkg = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    builder = os.path.join(pkg, "build_native.py")
    stamp = path + ".srchash"
    if not os.path.exists(builder) or not os.path.isdir(os.path.join(pkg, "csrc")):
        return
    import importlib.util
    spec = importlib.util.spec_from_file_location("_nv4_build_native", builder)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    recorded = open(stamp).read().strip() if os.path.exists(stamp) else ""
    if recorded != mod.source_hash():
        raise NativeLibraryError(
            f"{path} was not built from the current sources; rebuild with "
            f"`python nano-vllm-int4_b200/build_native.py`")


def load(path: str | None = None) -> ctypes.CDLL:
    """Load libnv4.so once (raises NativeLibraryError when it is absent)."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        p = path or LIB_PATH
        if not os.path.exists(p):
            raise NativeLibraryError(
                f"libnv4.so not found at {p}; build it with `python nano-vllm-int4_b200/build_native.py`")
        if path is None:
            _check_fresh(p)
        try:
            lib = ctypes.CDLL(p)
        except OSError as e:  # pragma: no cover - depends on the host
            raise NativeLibraryError(f"failed to load {p}: {e}") from e
        lib.nv4_rht_quant_pack.argtypes = [_vp, _vp, _vp, _vp, _i64, _i64, _int, _int, _vp]
        lib.nv4_rht_quant_i8.argtypes = [_vp, _vp, _vp, _vp, _i64, _i64, _int, _int, _vp]
        lib.nv4_silu_mul_rht_quant_i8.argtypes = [_vp, _vp, _vp, _vp, _i64, _i64, _int, _int, _vp]
        lib.nv4_add_rmsnorm_rht_quant_i8.argtypes = [_vp, _vp, _vp, ctypes.c_float, _vp, _vp, _vp, _vp, _vp, _i64,
                                                     _i64, _int, _int, _vp]
        lib.nv4_w4a4_grouped_gemm.argtypes = [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _int, _vp]
        lib.nv4_w4a4_gemm_i8.argtypes = [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _int, _vp]
        lib.nv4_w4a4_group_dots.argtypes = [_vp, _vp, _vp, _i64, _i64, _i64, _vp]
        lib.nv4_w4a16_gemm.argtypes = [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _vp, _i64, _vp]
        lib.nv4_w4a16_gemm_static.argtypes = [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _vp]
        lib.nv4_w4a16_gemm_static.restype = _int
        lib.nv4_w4a16_workspace_bytes.argtypes = [_i64, _i64, _i64]
        lib.nv4_peer_header_bytes.argtypes = []
        lib.nv4_peer_header_bytes.restype = _i64
        lib.nv4_peer_buffer_alloc.argtypes = [_i64, ctypes.POINTER(_vp), _vp]
        lib.nv4_peer_buffer_open.argtypes = [_vp, ctypes.POINTER(_vp)]
        lib.nv4_peer_buffer_close.argtypes = [_vp]
        lib.nv4_peer_buffer_free.argtypes = [_vp]
        lib.nv4_peer_allreduce_bf16.argtypes = [ctypes.POINTER(_vp), _int, _int, _vp, _i64, _i64, _vp]
        lib.nv4_w4a4_gemm_peer_allreduce_bf16.argtypes = [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _int,
                                                          ctypes.POINTER(_vp), _int, _int, _i64, _vp]
        for name in ("nv4_peer_buffer_alloc", "nv4_peer_buffer_open", "nv4_peer_buffer_close", "nv4_peer_buffer_free",
                     "nv4_peer_allreduce_bf16", "nv4_w4a4_gemm_peer_allreduce_bf16"):
            getattr(lib, name).restype = _int
        lib.nv4_w4a16_workspace_bytes.restype = _i64
        lib.nv4_w4a4_stream_plan.argtypes = [_i64, _i64, _i64, _int, _int, _int, ctypes.POINTER(ctypes.c_int32)]
        lib.nv4_w4a4_stream_plan.restype = _int
        lib.nv4_w4a16_plan.argtypes = [_i64, _i64, _i64, _int, ctypes.POINTER(ctypes.c_int64)]
        lib.nv4_w4a16_plan.restype = _int
        lib.nv4_paged_attention_workspace_bytes.argtypes = [_i64, _i64, _i64]
        lib.nv4_paged_attention_workspace_bytes.restype = _i64
        lib.nv4_paged_decode_attention.argtypes = [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64,
                                                   _i64, _i64, ctypes.c_float, _vp]
        lib.nv4_paged_decode_attention.restype = _int
        lib.nv4_qk_norm_rope_store.argtypes = [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64,
                                               _i64, ctypes.c_float, _vp]
        lib.nv4_qk_norm_rope_store.restype = _int
        lib.nv4_status_string.argtypes = [_int]
        lib.nv4_status_string.restype = ctypes.c_char_p
        lib.nv4_device_error.argtypes = [ctypes.POINTER(_int)]
        for name in ("nv4_rht_quant_pack", "nv4_rht_quant_i8", "nv4_silu_mul_rht_quant_i8",
                     "nv4_add_rmsnorm_rht_quant_i8", "nv4_w4a4_grouped_gemm", "nv4_w4a4_gemm_i8", "nv4_w4a4_group_dots", "nv4_w4a16_gemm",
                     "nv4_version", "nv4_last_cuda_error", "nv4_device_error"):
            getattr(lib, name).restype = _int
        if path is None:
            _lib = lib
        return lib


def check(status: int, what: str) -> None:
    if status == OK:
        return
    lib = load()
    text = lib.nv4_status_string(status).decode()
    if status == ERR_CUDA:
        text += f" (cudaError {lib.nv4_last_cuda_error()})"
    if status in (ERR_INVALID_ARGUMENT, ERR_ALIGNMENT, ERR_UNSUPPORTED):
        raise ValueError(f"{what}: {text}")
    raise NativeCallError(status, f"{what}: {text}")


def ptr(t: torch.Tensor) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr())


def stream_of(t: torch.Tensor) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def device_error() -> int:
    """Read and clear the error word of the current device (synchronises)."""
    code = _int(0)
    check(load().nv4_device_error(ctypes.byref(code)), "nv4_device_error")
    return code.value


def rht_quant_pack(x, signs, packed, scale, layout: int, clamp_lo: int) -> None:
    m, k = x.shape
    with torch.cuda.device(x.device):
        check(load().nv4_rht_quant_pack(ptr(x), ptr(signs), ptr(packed), ptr(scale), m, k, layout, clamp_lo,
                                        stream_of(x)), "nv4_rht_quant_pack")


def rht_quant_i8(x, signs, codes, scale, layout: int, clamp_lo: int) -> None:
    m, k = x.shape
    with torch.cuda.device(x.device):
        check(load().nv4_rht_quant_i8(ptr(x), ptr(signs), ptr(codes), ptr(scale), m, k, layout, clamp_lo,
                                      stream_of(x)), "nv4_rht_quant_i8")


def silu_mul_rht_quant_i8(gate_up, signs, codes, scale, layout: int, clamp_lo: int) -> None:
    """nv4_silu_mul_rht_quant_i8: the prep of bf16(silu(gate) * up) for gate_up [m, 2k]."""
    m, k = gate_up.shape[0], gate_up.shape[1] // 2
    with torch.cuda.device(gate_up.device):
        check(load().nv4_silu_mul_rht_quant_i8(ptr(gate_up), ptr(signs), ptr(codes), ptr(scale), m, k, layout,
                                               clamp_lo, stream_of(gate_up)), "nv4_silu_mul_rht_quant_i8")


def add_rmsnorm_rht_quant_i8(x, residual, weight, eps: float, signs, codes, scale, out_residual, out_normed,
                             layout: int, clamp_lo: int) -> None:
    """nv4_add_rmsnorm_rht_quant_i8 (residual, out_residual, out_normed may be None)."""
    m, k = x.shape
    with torch.cuda.device(x.device):
        check(load().nv4_add_rmsnorm_rht_quant_i8(ptr(x), _vp(0) if residual is None else ptr(residual), ptr(weight),
                                                  float(eps), ptr(signs), ptr(codes), ptr(scale),
                                                  _vp(0) if out_residual is None else ptr(out_residual),
                                                  _vp(0) if out_normed is None else ptr(out_normed), m, k, layout,
                                                  clamp_lo, stream_of(x)), "nv4_add_rmsnorm_rht_quant_i8")


def w4a4_gemm_i8(a_codes, w_packed, a_scale, w_scale, out, flags: int) -> None:
    m, k, n = a_codes.shape[0], a_codes.shape[1], w_packed.shape[0]
    with torch.cuda.device(a_codes.device):
        check(load().nv4_w4a4_gemm_i8(ptr(a_codes), ptr(w_packed), ptr(a_scale), ptr(w_scale), ptr(out),
                                      m, n, k, flags, stream_of(a_codes)), "nv4_w4a4_gemm_i8")


def w4a4_grouped_gemm(a_packed, w_packed, a_scale, w_scale, out, flags: int) -> None:
    m, n, k = a_packed.shape[0], w_packed.shape[0], a_packed.shape[1] * 2
    with torch.cuda.device(a_packed.device):
        check(load().nv4_w4a4_grouped_gemm(ptr(a_packed), ptr(w_packed), ptr(a_scale), ptr(w_scale), ptr(out),
                                           m, n, k, flags, stream_of(a_packed)), "nv4_w4a4_grouped_gemm")


def w4a4_group_dots(a_packed, w_packed, dots) -> None:
    m, n, k = a_packed.shape[0], w_packed.shape[0], a_packed.shape[1] * 2
    with torch.cuda.device(a_packed.device):
        check(load().nv4_w4a4_group_dots(ptr(a_packed), ptr(w_packed), ptr(dots), m, n, k, stream_of(a_packed)),
              "nv4_w4a4_group_dots")


def w4a16_workspace_bytes(m: int, n: int, k: int, device) -> int:
    with torch.cuda.device(device):
        return int(load().nv4_w4a16_workspace_bytes(m, n, k))


def w4a16_gemm(x, qweight, qzeros, scales, out, group_size: int, workspace) -> None:
    m, k = x.shape
    n = qweight.shape[1]
    ws_ptr = ptr(workspace) if workspace is not None else ctypes.c_void_p(0)
    ws_bytes = workspace.numel() * workspace.element_size() if workspace is not None else 0
    with torch.cuda.device(x.device):
        check(load().nv4_w4a16_gemm(ptr(x), ptr(qweight), ptr(qzeros), ptr(scales), ptr(out), m, n, k, group_size,
                                    ws_ptr, ws_bytes, stream_of(x)), "nv4_w4a16_gemm")


W4A16_STATIC_SCRATCH_FLOATS = 512 * 1024  # NV4_W4A16_STATIC_SCRATCH_FLOATS


def w4a16_gemm_static(x, qweight, qzeros, scales, out, group_size: int) -> None:
    """nv4_w4a16_gemm without a workspace: split-K partials go to the library's
    static per-device array, so the call allocates nothing.  Overlapping calls
    on one device race on that array; for m <= 16, m * n is limited to
    W4A16_STATIC_SCRATCH_FLOATS (ValueError beyond it)."""
    m, k = x.shape
    n = qweight.shape[1]
    with torch.cuda.device(x.device):
        status = load().nv4_w4a16_gemm_static(ptr(x), ptr(qweight), ptr(qzeros), ptr(scales), ptr(out), m, n, k,
                                              group_size, stream_of(x))
        if status == ERR_UNSUPPORTED and group_size == 128 and m <= 16 and m * n > W4A16_STATIC_SCRATCH_FLOATS:
            raise ValueError(f"nv4_w4a16_gemm_static: m * n = {m * n} exceeds the static scratch of "
                             f"{W4A16_STATIC_SCRATCH_FLOATS} floats (m <= 16); use nv4_w4a16_gemm with a workspace")
        check(status, "nv4_w4a16_gemm_static")


STREAM_PLAN_FIELDS = ("token_tiles", "slabs", "k_split", "token_splits", "tiles_per_warp", "rows_per_cta", "stages",
                      "n_iters", "smem_bytes", "grid_x", "grid_y", "threads", "producer_warps")
SM_COUNT_B200 = 148


def w4a4_stream_plan(m: int, n: int, k: int, flags: int = GEMM_W_SCALE_GROUPED, sm_count: int = SM_COUNT_B200,
                     peer: bool = False):
    """Host-side launch plan of the decode stream GEMM (nv4_w4a4_stream_plan;
    no GPU needed): a dict of STREAM_PLAN_FIELDS, or None when the kernel
    cannot plan the shape (NV4_ERR_UNSUPPORTED)."""
    out = (ctypes.c_int32 * len(STREAM_PLAN_FIELDS))()
    status = load().nv4_w4a4_stream_plan(m, n, k, flags, sm_count, 1 if peer else 0, out)
    if status == ERR_UNSUPPORTED:
        return None
    check(status, "nv4_w4a4_stream_plan")
    return dict(zip(STREAM_PLAN_FIELDS, list(out)))


W4A16_PLAN_FIELDS = ("kernel", "splits", "token_tile", "ctas", "workspace_bytes")
W4A16_KERNEL_MMA, W4A16_KERNEL_DECODE, W4A16_KERNEL_TC = 0, 1, 2


def w4a16_plan(m: int, n: int, k: int, sm_count: int = SM_COUNT_B200):
    """Which W4A16 kernel nv4_w4a16_gemm runs for a shape and its K split
    (nv4_w4a16_plan; host only, no GPU needed): a dict of W4A16_PLAN_FIELDS."""
    out = (ctypes.c_int64 * len(W4A16_PLAN_FIELDS))()
    check(load().nv4_w4a16_plan(m, n, k, sm_count, out), "nv4_w4a16_plan")
    return dict(zip(W4A16_PLAN_FIELDS, list(out)))


# ---------------------------------------------------------------- tensor-parallel peer buffers
IPC_HANDLE_BYTES = 64


def peer_header_bytes() -> int:
    return int(load().nv4_peer_header_bytes())


def peer_buffer_alloc(capacity: int, device) -> tuple[int, bytes]:
    """Allocate this rank's peer buffer for outputs of up to `capacity` elements
    on `device`: (device address, IPC handle)."""
    buf, handle = _vp(), ctypes.create_string_buffer(IPC_HANDLE_BYTES)
    with torch.cuda.device(device):
        check(load().nv4_peer_buffer_alloc(capacity, ctypes.byref(buf), handle), "nv4_peer_buffer_alloc")
    return buf.value, handle.raw


def peer_buffer_open(handle: bytes, device) -> int:
    buf = _vp()
    with torch.cuda.device(device):
        check(load().nv4_peer_buffer_open(handle, ctypes.byref(buf)), "nv4_peer_buffer_open")
    return buf.value


def peer_buffer_close(addr: int, device) -> None:
    with torch.cuda.device(device):
        check(load().nv4_peer_buffer_close(_vp(addr)), "nv4_peer_buffer_close")


def peer_buffer_free(addr: int, device) -> None:
    with torch.cuda.device(device):
        check(load().nv4_peer_buffer_free(_vp(addr)), "nv4_peer_buffer_free")


def w4a4_gemm_i8_to(a_codes, w_packed, a_scale, w_scale, out_addr: int, flags: int) -> None:
    """nv4_w4a4_gemm_i8 writing to a raw device address (a peer buffer's partial)."""
    m, k, n = a_codes.shape[0], a_codes.shape[1], w_packed.shape[0]
    with torch.cuda.device(a_codes.device):
        check(load().nv4_w4a4_gemm_i8(ptr(a_codes), ptr(w_packed), ptr(a_scale), ptr(w_scale), _vp(out_addr),
                                      m, n, k, flags, stream_of(a_codes)), "nv4_w4a4_gemm_i8")


PEER_MAX_TOKENS = 32  # NV4_PEER_MAX_TOKENS


def w4a4_gemm_peer_allreduce_bf16(a_codes, w_packed, a_scale, w_scale, out, bufs: list[int], rank: int,
                                  capacity: int, flags: int) -> None:
    """Row-parallel GEMM whose CTAs store their FP32 tiles into every rank's
    inbox, then the rank-order sum to BF16 `out` (nv4_w4a4_gemm_peer_allreduce_bf16)."""
    m, k, n = a_codes.shape[0], a_codes.shape[1], w_packed.shape[0]
    arr = (_vp * len(bufs))(*[_vp(b) for b in bufs])
    with torch.cuda.device(a_codes.device):
        check(load().nv4_w4a4_gemm_peer_allreduce_bf16(ptr(a_codes), ptr(w_packed), ptr(a_scale), ptr(w_scale),
                                                       ptr(out), m, n, k, flags, arr, rank, len(bufs), capacity,
                                                       stream_of(a_codes)), "nv4_w4a4_gemm_peer_allreduce_bf16")


def peer_allreduce_bf16(bufs: list[int], rank: int, out, count: int, capacity: int) -> None:
    arr = (_vp * len(bufs))(*[_vp(b) for b in bufs])
    with torch.cuda.device(out.device):
        check(load().nv4_peer_allreduce_bf16(arr, rank, len(bufs), ptr(out), count, capacity, stream_of(out)),
              "nv4_peer_allreduce_bf16")


# ---------------------------------------------------------------- attention of the end-to-end model
def paged_attention_workspace_bytes(batch: int, num_heads: int, max_pages: int) -> int:
    return int(load().nv4_paged_attention_workspace_bytes(batch, num_heads, max_pages))


def paged_decode_attention(q, k_cache, v_cache, block_tables, context_lens, out, workspace, scale: float) -> None:
    """nv4_paged_decode_attention: q [B, Hq, D], caches [pages, 256, Hkv, D],
    block_tables int32 [B, max_pages], context_lens int32 [B] -> out [B, Hq, D]."""
    b, hq, d = q.shape
    hkv = k_cache.shape[2]
    with torch.cuda.device(q.device):
        check(load().nv4_paged_decode_attention(ptr(q), ptr(k_cache), ptr(v_cache), ptr(block_tables),
                                                ptr(context_lens), ptr(out), ptr(workspace),
                                                workspace.numel() * workspace.element_size(), b, hq, hkv, d,
                                                k_cache.shape[1], block_tables.shape[1], float(scale), stream_of(q)),
              "nv4_paged_decode_attention")


def qk_norm_rope_store(qkv, q_weight, k_weight, cos_sin, positions, slot_mapping, q_out, k_out, k_cache, v_cache,
                       num_heads: int, num_kv_heads: int, eps: float) -> None:
    """nv4_qk_norm_rope_store (k_out, and slot_mapping with both caches, may be None)."""
    t = qkv.shape[0]
    nul = ctypes.c_void_p(0)
    opt = lambda x: nul if x is None else ptr(x)
    with torch.cuda.device(qkv.device):
        check(load().nv4_qk_norm_rope_store(ptr(qkv), ptr(q_weight), ptr(k_weight), ptr(cos_sin), ptr(positions),
                                            opt(slot_mapping), ptr(q_out), opt(k_out), opt(k_cache), opt(v_cache), t,
                                            num_heads, num_kv_heads, q_out.shape[-1], float(eps), stream_of(qkv)),
              "nv4_qk_norm_rope_store")
