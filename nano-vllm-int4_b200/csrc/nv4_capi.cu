// C ABI of libnv4 (declared in include/nv4.h): argument checks that mirror the
// reference's Python validation, then dispatch to the kernel launchers.
#include <cstdint>
#include <cstring>
#include <mutex>

#include "nv4_device.cuh"
#include "nv4_launch.h"

namespace nv4 {

static thread_local int t_last_cuda_error = 0;
void set_last_cuda_error(cudaError_t e) { t_last_cuda_error = static_cast<int>(e); }

int current_device() {
  int d = -1;
  if (cudaGetDevice(&d) != cudaSuccess) return -1;
  return d;
}

namespace {
constexpr int kMaxDevices = 64;
int g_sm_count[kMaxDevices] = {};
int g_cc_major[kMaxDevices] = {};
std::mutex g_mutex;

int query_device(int dev) {
  if (dev < 0 || dev >= kMaxDevices) return -1;
  if (g_sm_count[dev] > 0) return dev;
  std::lock_guard<std::mutex> lock(g_mutex);
  if (g_sm_count[dev] == 0) {
    int sms = 0, major = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess)
      return -1;
    g_cc_major[dev] = major;
    g_sm_count[dev] = sms;
  }
  return dev;
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn g_encode = nullptr;

EncodeTiledFn encode_fn() {
  if (g_encode) return g_encode;
  std::lock_guard<std::mutex> lock(g_mutex);
  if (!g_encode) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<EncodeTiledFn>(fn);
  }
  return g_encode;
}
}  // namespace

int device_sm_count() {
  const int dev = query_device(current_device());
  return dev < 0 ? -1 : g_sm_count[dev];
}

static bool device_is_sm100() {
  const int dev = query_device(current_device());
  return dev >= 0 && g_cc_major[dev] == 10;
}

int ensure_smem_attr(const void* kernel, int bytes, int* done_flags) {
  const int dev = current_device();
  if (dev < 0 || dev >= kMaxDevices) return NV4_ERR_CUDA;
  if (done_flags[dev] >= bytes) return NV4_OK;
  const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return NV4_ERR_CUDA;
  }
  done_flags[dev] = bytes;
  return NV4_OK;
}

bool make_tensor_map_2d(CUtensorMap* map, CUtensorMapDataType dtype, int elem_bytes, const void* base, uint64_t rows,
                        uint64_t cols, uint32_t box_rows, uint32_t box_cols, CUtensorMapSwizzle swizzle) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols * static_cast<uint64_t>(elem_bytes)};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool make_tensor_map_u8(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols_bytes, uint32_t box_rows,
                        uint32_t box_cols_bytes, CUtensorMapSwizzle swizzle) {
  return make_tensor_map_2d(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, base, rows, cols_bytes, box_rows, box_cols_bytes,
                            swizzle);
}

int launch_w4a4_tc_gemm(const void* a8, const void* w_packed, const void* a_scale, const void* w_scale, void* out,
                        int64_t m, int64_t n, int64_t k, int flags, cudaStream_t stream);

// Dispatch of the INT8-layout activation path: more than kTcMinTokens tokens go
// to the tiled tcgen05 kernel (tensor-bound prefill shapes); fewer, packed
// activations and NV4_GEMM_FORCE_STREAM to the mma.sync weight-streaming
// kernel.  (At 8-32 tokens one tcgen05 MMA covers 128 weight rows but only the
// few tokens, and its issue cost leaves it no faster than mma.sync there.)
constexpr int64_t kTcMinTokens = 64;

int launch_w4a4_gemm(const void* a_packed, const void* a8, const void* w_packed, const void* a_scale,
                     const void* w_scale, void* out, int64_t m, int64_t n, int64_t k, int flags, cudaStream_t stream) {
  if (a8 != nullptr && !(flags & NV4_GEMM_FORCE_STREAM) && m > kTcMinTokens) {
    const int rc = launch_w4a4_tc_gemm(a8, w_packed, a_scale, w_scale, out, m, n, k, flags, stream);
    if (rc != NV4_ERR_UNSUPPORTED) return rc;
  }
  return launch_w4a4_stream_gemm(a_packed, a8, w_packed, a_scale, w_scale, out, m, n, k, flags, stream);
}

}  // namespace nv4

using namespace nv4;

static inline bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

#pragma GCC visibility push(default)
extern "C" {

int nv4_version(void) { return 100; }  // 0.1.0

int nv4_w4a4_stream_plan(int64_t m, int64_t n, int64_t k, int flags, int sm_count, int peer, int32_t* plan) {
  if (plan == nullptr) return NV4_ERR_INVALID_ARGUMENT;
  StreamPlan pl;
  const int rc = plan_w4a4_stream(m, n, k, (flags & NV4_GEMM_W_SCALE_GROUPED) != 0, sm_count, peer != 0, &pl);
  if (rc != NV4_OK) return rc;
  const int32_t v[NV4_STREAM_PLAN_FIELDS] = {pl.token_tiles, pl.slabs, pl.k_split, pl.token_splits, pl.tiles_per_warp,
                                             pl.rows_per_cta, pl.stages, pl.n_iters, pl.smem_bytes, pl.grid_x,
                                             pl.grid_y, pl.threads, pl.producer_warps};
  for (int i = 0; i < NV4_STREAM_PLAN_FIELDS; ++i) plan[i] = v[i];
  return NV4_OK;
}

const char* nv4_status_string(int status) {
  switch (status) {
    case NV4_OK: return "ok";
    case NV4_ERR_INVALID_ARGUMENT: return "invalid argument";
    case NV4_ERR_UNSUPPORTED: return "unsupported configuration";
    case NV4_ERR_ALIGNMENT: return "misaligned pointer";
    case NV4_ERR_CUDA: return "CUDA runtime error";
    case NV4_ERR_DEVICE: return "current device is not an sm_100 GPU";
    default: return "unknown status";
  }
}

int nv4_last_cuda_error(void) { return t_last_cuda_error; }

int nv4_device_error(int* code) {
  if (!code) return NV4_ERR_INVALID_ARGUMENT;
  cudaError_t e = cudaDeviceSynchronize();
  int v = 0;
  if (e == cudaSuccess) e = cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int));
  const int zero = 0;
  if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int));
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return NV4_ERR_CUDA;
  }
  *code = v;
  return NV4_OK;
}

static int check_prep_args(const void* x, const void* signs, const void* codes, const void* scale, int64_t m,
                           int64_t k, int layout, int clamp_lo, uintptr_t codes_align) {
  if (!x || !signs || !codes || !scale || m < 1 || m > (int64_t(1) << 31) - 1) return NV4_ERR_INVALID_ARGUMENT;
  if (clamp_lo != -7 && clamp_lo != -8) return NV4_ERR_INVALID_ARGUMENT;
  if (layout == NV4_LAYOUT_BLOCK128) {
    if (k < 128 || k % 128 || k > (int64_t(1) << 24)) return NV4_ERR_INVALID_ARGUMENT;
  } else if (layout == NV4_LAYOUT_ROW_DH) {
    if (k != 4096 && k != 12288) return NV4_ERR_INVALID_ARGUMENT;
  } else {
    return NV4_ERR_INVALID_ARGUMENT;
  }
  if (!aligned(x, 16) || !aligned(signs, 8) || !aligned(codes, codes_align) || !aligned(scale, 2))
    return NV4_ERR_ALIGNMENT;
  if (!device_is_sm100()) return NV4_ERR_DEVICE;
  return NV4_OK;
}

int nv4_rht_quant_pack(const void* x, const void* signs, void* out_packed, void* out_scale, int64_t m, int64_t k,
                       int layout, int clamp_lo, void* stream) {
  const int rc = check_prep_args(x, signs, out_packed, out_scale, m, k, layout, clamp_lo, 4);
  if (rc != NV4_OK) return rc;
  return launch_rht_quant(x, signs, out_packed, nullptr, out_scale, m, k, layout, clamp_lo,
                          static_cast<cudaStream_t>(stream));
}

int nv4_rht_quant_i8(const void* x, const void* signs, void* out_codes, void* out_scale, int64_t m, int64_t k,
                     int layout, int clamp_lo, void* stream) {
  const int rc = check_prep_args(x, signs, out_codes, out_scale, m, k, layout, clamp_lo, 16);
  if (rc != NV4_OK) return rc;
  return launch_rht_quant(x, signs, nullptr, out_codes, out_scale, m, k, layout, clamp_lo,
                          static_cast<cudaStream_t>(stream));
}

int nv4_silu_mul_rht_quant_i8(const void* gate_up, const void* signs, void* out_codes, void* out_scale, int64_t m,
                              int64_t k, int layout, int clamp_lo, void* stream) {
  const int rc = check_prep_args(gate_up, signs, out_codes, out_scale, m, k, layout, clamp_lo, 16);
  if (rc != NV4_OK) return rc;
  if (2 * k > (int64_t(1) << 24)) return NV4_ERR_INVALID_ARGUMENT;
  return launch_silu_mul_rht_quant(gate_up, signs, nullptr, out_codes, out_scale, m, k, layout, clamp_lo,
                                   static_cast<cudaStream_t>(stream));
}

int nv4_add_rmsnorm_rht_quant_i8(const void* x, const void* residual, const void* weight, float eps,
                                  const void* signs, void* out_codes, void* out_scale, void* out_residual,
                                  void* out_normed, int64_t m, int64_t k, int layout, int clamp_lo, void* stream) {
  const int rc = check_prep_args(x, signs, out_codes, out_scale, m, k, layout, clamp_lo, 16);
  if (rc != NV4_OK) return rc;
  if (!weight || (residual && !out_residual) || !(eps >= 0.0f) || !(eps < 1.0f)) return NV4_ERR_INVALID_ARGUMENT;
  if ((layout == NV4_LAYOUT_BLOCK128 && (k % 512 || k > 16384)) || (layout == NV4_LAYOUT_ROW_DH && k != 4096))
    return NV4_ERR_UNSUPPORTED;
  if (!aligned(weight, 16) || (residual && !aligned(residual, 16)) || (out_residual && !aligned(out_residual, 16)) ||
      (out_normed && !aligned(out_normed, 16)))
    return NV4_ERR_ALIGNMENT;
  return launch_add_rmsnorm_rht_quant(x, residual, weight, eps, signs, nullptr, out_codes, out_scale,
                                      residual ? out_residual : nullptr, out_normed, m, k, layout, clamp_lo,
                                      static_cast<cudaStream_t>(stream));
}

static int check_gemm_args(const void* a, const void* w_packed, const void* a_scale, const void* w_scale,
                           const void* out, int64_t m, int64_t n, int64_t k, int flags) {
  if (!a || !w_packed || !a_scale || !w_scale || !out) return NV4_ERR_INVALID_ARGUMENT;
  if (m < 1 || n < 1 || k < 128 || k % 128 || n % 8 || m > (int64_t(1) << 31) - 1 || n > (int64_t(1) << 31) - 1 ||
      k > (int64_t(1) << 24))
    return NV4_ERR_INVALID_ARGUMENT;
  if (flags & ~(NV4_GEMM_W_SCALE_GROUPED | NV4_GEMM_OUT_FP32 | NV4_GEMM_FORCE_STREAM))
    return NV4_ERR_INVALID_ARGUMENT;
  if (!aligned(a, 16) || !aligned(w_packed, 16) || !aligned(a_scale, 2) || !aligned(w_scale, 2) ||
      !aligned(out, (flags & NV4_GEMM_OUT_FP32) ? 4 : 2))
    return NV4_ERR_ALIGNMENT;
  if (!device_is_sm100()) return NV4_ERR_DEVICE;
  return NV4_OK;
}

int nv4_w4a4_grouped_gemm(const void* a_packed, const void* w_packed, const void* a_scale, const void* w_scale,
                          void* out, int64_t m, int64_t n, int64_t k, int flags, void* stream) {
  const int rc = check_gemm_args(a_packed, w_packed, a_scale, w_scale, out, m, n, k, flags);
  if (rc != NV4_OK) return rc;
  return launch_w4a4_gemm(a_packed, nullptr, w_packed, a_scale, w_scale, out, m, n, k, flags,
                          static_cast<cudaStream_t>(stream));
}

int nv4_w4a4_gemm_i8(const void* a_codes, const void* w_packed, const void* a_scale, const void* w_scale, void* out,
                     int64_t m, int64_t n, int64_t k, int flags, void* stream) {
  const int rc = check_gemm_args(a_codes, w_packed, a_scale, w_scale, out, m, n, k, flags);
  if (rc != NV4_OK) return rc;
  return launch_w4a4_gemm(nullptr, a_codes, w_packed, a_scale, w_scale, out, m, n, k, flags,
                          static_cast<cudaStream_t>(stream));
}

int nv4_w4a4_group_dots(const void* a_packed, const void* w_packed, int32_t* dots, int64_t m, int64_t n, int64_t k,
                        void* stream) {
  if (!a_packed || !w_packed || !dots || m < 1 || n < 1 || k < 128 || k % 128) return NV4_ERR_INVALID_ARGUMENT;
  if ((k / 128) * m * n > (int64_t(1) << 31)) return NV4_ERR_UNSUPPORTED;
  if (!aligned(dots, 4)) return NV4_ERR_ALIGNMENT;
  if (!device_is_sm100()) return NV4_ERR_DEVICE;
  return launch_w4a4_group_dots(a_packed, w_packed, dots, m, n, k, static_cast<cudaStream_t>(stream));
}

int64_t nv4_w4a16_workspace_bytes(int64_t m, int64_t n, int64_t k) {
  if (m < 1 || n < 1 || k < 128) return 0;
  return w4a16_workspace_bytes(m, n, k);
}

int nv4_w4a16_gemm(const void* x, const void* qweight, const void* qzeros, const void* scales, void* out, int64_t m,
                   int64_t n, int64_t k, int64_t group_size, void* workspace, int64_t workspace_bytes, void* stream) {
  if (!x || !qweight || !qzeros || !scales || !out) return NV4_ERR_INVALID_ARGUMENT;
  if (group_size != 128) return NV4_ERR_UNSUPPORTED;
  if (m < 1 || n < 64 || k < 128 || k % 128 || n % 64 || m > (int64_t(1) << 31) - 1 || k > (int64_t(1) << 24) ||
      n > (int64_t(1) << 24))
    return NV4_ERR_INVALID_ARGUMENT;
  if (!aligned(x, 16) || !aligned(qweight, 4) || !aligned(qzeros, 4) || !aligned(scales, 2) || !aligned(out, 4) ||
      (workspace && !aligned(workspace, 4)))
    return NV4_ERR_ALIGNMENT;
  if (!device_is_sm100()) return NV4_ERR_DEVICE;
  return launch_w4a16_gemm(x, qweight, qzeros, scales, out, m, n, k, workspace, workspace_bytes,
                           static_cast<cudaStream_t>(stream));
}

int nv4_w4a16_plan(int64_t m, int64_t n, int64_t k, int sm_count, int64_t* plan) {
  if (plan == nullptr || sm_count < 1) return NV4_ERR_INVALID_ARGUMENT;
  if (m < 1 || n < 64 || k < 128 || k % 128 || n % 64 || m > (int64_t(1) << 31) - 1 || k > (int64_t(1) << 24) ||
      n > (int64_t(1) << 24))
    return NV4_ERR_INVALID_ARGUMENT;
  w4a16_plan(m, n, k, sm_count, plan);
  return NV4_OK;
}

// Allocation-free variant: the split-K partials go to a static device array
// (see launch_w4a16_gemm_static).  Checks as nv4_w4a16_gemm, plus the
// scratch limit.
int nv4_w4a16_gemm_static(const void* x, const void* qweight, const void* qzeros, const void* scales, void* out,
                          int64_t m, int64_t n, int64_t k, int64_t group_size, void* stream) {
  if (!x || !qweight || !qzeros || !scales || !out) return NV4_ERR_INVALID_ARGUMENT;
  if (group_size != 128) return NV4_ERR_UNSUPPORTED;
  if (m < 1 || n < 64 || k < 128 || k % 128 || n % 64 || m > (int64_t(1) << 31) - 1 || k > (int64_t(1) << 24) ||
      n > (int64_t(1) << 24))
    return NV4_ERR_INVALID_ARGUMENT;
  if (!w4a16_static_fits(m, n)) return NV4_ERR_UNSUPPORTED;
  if (!aligned(x, 16) || !aligned(qweight, 4) || !aligned(qzeros, 4) || !aligned(scales, 2) || !aligned(out, 4))
    return NV4_ERR_ALIGNMENT;
  if (!device_is_sm100()) return NV4_ERR_DEVICE;
  return launch_w4a16_gemm_static(x, qweight, qzeros, scales, out, m, n, k, static_cast<cudaStream_t>(stream));
}

// ---- peer buffers and the one-shot all-reduce of the row-parallel layers
int64_t nv4_peer_header_bytes(void) { return NV4_PEER_HEADER_BYTES; }

int nv4_peer_buffer_alloc(int64_t capacity, void** buf, void* ipc_handle) {
  if (!buf || !ipc_handle || capacity < 4 || capacity % 4 || capacity > (int64_t(1) << 28)) return NV4_ERR_INVALID_ARGUMENT;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, static_cast<size_t>(NV4_PEER_HEADER_BYTES + peer_buffer_data_bytes(capacity)));
  if (e == cudaSuccess) e = cudaMemset(p, 0, static_cast<size_t>(NV4_PEER_HEADER_BYTES));
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    if (p) cudaFree(p);
    set_last_cuda_error(e);
    return NV4_ERR_CUDA;
  }
  memcpy(ipc_handle, &h, sizeof(h));
  *buf = p;
  return NV4_OK;
}

int nv4_peer_buffer_open(const void* ipc_handle, void** buf) {
  if (!ipc_handle || !buf) return NV4_ERR_INVALID_ARGUMENT;
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(buf, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return NV4_ERR_CUDA;
  }
  return NV4_OK;
}

int nv4_peer_buffer_close(void* buf) {
  if (!buf) return NV4_ERR_INVALID_ARGUMENT;
  const cudaError_t e = cudaIpcCloseMemHandle(buf);
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return NV4_ERR_CUDA;
  }
  return NV4_OK;
}

int nv4_peer_buffer_free(void* buf) {
  if (!buf) return NV4_ERR_INVALID_ARGUMENT;
  const cudaError_t e = cudaFree(buf);
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return NV4_ERR_CUDA;
  }
  return NV4_OK;
}

int nv4_peer_allreduce_bf16(void* const* bufs, int rank, int world, void* out, int64_t count, int64_t capacity,
                            void* stream) {
  if (!bufs || !out || world < 2 || world > 8 || rank < 0 || rank >= world || count < 4 || count % 4 ||
      capacity % 4 || count > capacity)
    return NV4_ERR_INVALID_ARGUMENT;
  for (int r = 0; r < world; ++r)
    if (!bufs[r] || !aligned(bufs[r], 256)) return NV4_ERR_ALIGNMENT;
  if (!aligned(out, 8)) return NV4_ERR_ALIGNMENT;
  if (!device_is_sm100()) return NV4_ERR_DEVICE;
  return launch_peer_allreduce_bf16(bufs, rank, world, out, count, capacity, static_cast<cudaStream_t>(stream));
}

int nv4_w4a4_gemm_peer_allreduce_bf16(const void* a_codes, const void* w_packed, const void* a_scale,
                                      const void* w_scale, void* out, int64_t m, int64_t n, int64_t k, int flags,
                                      void* const* bufs, int rank, int world, int64_t capacity, void* stream) {
  if (flags & ~NV4_GEMM_W_SCALE_GROUPED) return NV4_ERR_INVALID_ARGUMENT;
  const int rc = check_gemm_args(a_codes, w_packed, a_scale, w_scale, out, m, n, k, flags);
  if (rc != NV4_OK) return rc;
  if (!bufs || world < 2 || world > 8 || rank < 0 || rank >= world || m > NV4_PEER_MAX_TOKENS || capacity % 4 ||
      m * n > capacity)
    return NV4_ERR_INVALID_ARGUMENT;
  for (int r = 0; r < world; ++r)
    if (!bufs[r] || !aligned(bufs[r], 256)) return NV4_ERR_ALIGNMENT;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  PeerTarget peer;
  peer.bufs = bufs;
  peer.rank = rank;
  peer.world = world;
  peer.capacity = capacity;
  const int g = launch_w4a4_stream_gemm(nullptr, a_codes, w_packed, a_scale, w_scale, nullptr, m, n, k, flags, s, &peer);
  if (g != NV4_OK) return g;
  return launch_peer_reduce_tiles_bf16(bufs, rank, world, out, static_cast<int>(m), static_cast<int>(n),
                                       peer.rows_per_cta, peer.ctas, capacity, s);
}

// ---- attention of the end-to-end model
int64_t nv4_paged_attention_workspace_bytes(int64_t batch, int64_t num_heads, int64_t max_pages) {
  if (batch < 1 || num_heads < 1 || max_pages < 1) return 0;
  return paged_attention_workspace_bytes(batch, num_heads, max_pages);
}

int nv4_paged_decode_attention(const void* q, const void* k_cache, const void* v_cache, const int32_t* block_tables,
                               const int32_t* context_lens, void* out, void* workspace, int64_t workspace_bytes,
                               int64_t batch, int64_t num_heads, int64_t num_kv_heads, int64_t head_dim,
                               int64_t page_size, int64_t max_pages, float scale, void* stream) {
  if (!q || !k_cache || !v_cache || !block_tables || !context_lens || !out || !workspace)
    return NV4_ERR_INVALID_ARGUMENT;
  if (batch < 1 || batch > 65535 || num_kv_heads < 1 || num_heads < num_kv_heads || num_heads % num_kv_heads ||
      max_pages < 1 || max_pages > 65535 || !(scale > 0.0f))
    return NV4_ERR_INVALID_ARGUMENT;
  if (head_dim != 128 || page_size != 256 || num_heads / num_kv_heads > 8) return NV4_ERR_UNSUPPORTED;
  if (workspace_bytes < paged_attention_workspace_bytes(batch, num_heads, max_pages)) return NV4_ERR_INVALID_ARGUMENT;
  if (!aligned(q, 16) || !aligned(k_cache, 16) || !aligned(v_cache, 16) || !aligned(out, 4) ||
      !aligned(workspace, 16) || !aligned(block_tables, 4) || !aligned(context_lens, 4))
    return NV4_ERR_ALIGNMENT;
  if (!device_is_sm100()) return NV4_ERR_DEVICE;
  return launch_paged_decode_attention(q, k_cache, v_cache, block_tables, context_lens, out, workspace, batch,
                                       num_heads, num_kv_heads, max_pages, scale, static_cast<cudaStream_t>(stream));
}

int nv4_qk_norm_rope_store(const void* qkv, const void* q_weight, const void* k_weight, const float* cos_sin,
                           const int64_t* positions, const int32_t* slot_mapping, void* q_out, void* k_out,
                           void* k_cache, void* v_cache, int64_t tokens, int64_t num_heads, int64_t num_kv_heads,
                           int64_t head_dim, float eps, void* stream) {
  if (!qkv || !q_weight || !k_weight || !cos_sin || !positions || !q_out) return NV4_ERR_INVALID_ARGUMENT;
  if ((slot_mapping != nullptr) != (k_cache != nullptr) || (k_cache != nullptr) != (v_cache != nullptr))
    return NV4_ERR_INVALID_ARGUMENT;
  if (tokens < 1 || num_heads < 1 || num_kv_heads < 1 || tokens * (num_heads + 2 * num_kv_heads) > (int64_t(1) << 31))
    return NV4_ERR_INVALID_ARGUMENT;
  if (head_dim != 128) return NV4_ERR_UNSUPPORTED;
  if (!aligned(qkv, 8) || !aligned(q_weight, 8) || !aligned(k_weight, 8) || !aligned(cos_sin, 4) ||
      !aligned(q_out, 8) || (k_out && !aligned(k_out, 8)) || (k_cache && !aligned(k_cache, 8)) ||
      (v_cache && !aligned(v_cache, 8)))
    return NV4_ERR_ALIGNMENT;
  if (!device_is_sm100()) return NV4_ERR_DEVICE;
  return launch_qk_norm_rope_store(qkv, q_weight, k_weight, cos_sin, positions, slot_mapping, q_out, k_out, k_cache,
                                   v_cache, tokens, num_heads, num_kv_heads, eps, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
#pragma GCC visibility pop
