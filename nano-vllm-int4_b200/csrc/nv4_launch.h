// Host-side helpers shared by the kernel launchers (internal to libnv4).
#pragma once

#include <algorithm>
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "../../include/nv4.h"

namespace nv4 {

// Last failing cudaError_t of this host thread (reported by nv4_last_cuda_error).
void set_last_cuda_error(cudaError_t e);

int current_device();
int device_sm_count();  // SMs of the current device (cached), <= 0 on failure

// Launch `kernel` on `stream`.  With `pdl` the launch carries the programmatic
// stream serialization attribute: the kernel may start while the previous
// kernel in the stream is still running and must call griddepcontrol.wait
// before reading that kernel's output.
template <typename... KArgs, typename... Args>
int launch_kernel(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream, bool pdl,
                  Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  if (pdl) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return NV4_ERR_CUDA;
  }
  return NV4_OK;
}

// Opt a kernel into `bytes` of dynamic shared memory once per device.
int ensure_smem_attr(const void* kernel, int bytes, int* done_flags /* [64] */);

// 2-D tensor map over a row-major uint8 matrix [rows, cols_bytes] with a box of
// [box_rows, box_cols_bytes] and the given swizzle; false on failure.
bool make_tensor_map_u8(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols_bytes, uint32_t box_rows,
                        uint32_t box_cols_bytes, CUtensorMapSwizzle swizzle);
bool make_tensor_map_2d(CUtensorMap* map, CUtensorMapDataType dtype, int elem_bytes, const void* base, uint64_t rows,
                        uint64_t cols, uint32_t box_rows, uint32_t box_cols, CUtensorMapSwizzle swizzle);

// ---- launchers (one per kernel family) ----
// Activation prep; `packed` and/or `codes8` (GEMM-ready INT8 layout) receive the codes.
int launch_rht_quant(const void* x, const void* signs, void* packed, void* codes8, void* scale, int64_t m, int64_t k,
                     int layout, int clamp_lo, cudaStream_t stream);
// Same, with the input RMSNorm(x + residual) (residual may be null; then out_residual is unused).
int launch_add_rmsnorm_rht_quant(const void* x, const void* residual, const void* weight, float eps,
                                 const void* signs, void* packed, void* codes8, void* scale, void* out_residual,
                                 void* out_normed, int64_t m, int64_t k, int layout, int clamp_lo,
                                 cudaStream_t stream);
// Same, with the input bf16(silu(gate) * up) of a gate/up source [m, 2k].
int launch_silu_mul_rht_quant(const void* gate_up, const void* signs, void* packed, void* codes8, void* scale,
                              int64_t m, int64_t k, int layout, int clamp_lo, cudaStream_t stream);
// Grouped GEMM; activations from `a8` (INT8 layout) when non-null, else `a_packed`.
int launch_w4a4_gemm(const void* a_packed, const void* a8, const void* w_packed, const void* a_scale,
                     const void* w_scale, void* out, int64_t m, int64_t n, int64_t k, int flags, cudaStream_t stream);
int launch_w4a4_group_dots(const void* a_packed, const void* w_packed, int32_t* dots, int64_t m, int64_t n, int64_t k,
                           cudaStream_t stream);
int launch_w4a16_gemm(const void* x, const void* qweight, const void* qzeros, const void* scales, void* out,
                      int64_t m, int64_t n, int64_t k, void* workspace, int64_t workspace_bytes, cudaStream_t stream);
int64_t w4a16_workspace_bytes(int64_t m, int64_t n, int64_t k);
// W4A16 on tcgen05 (prefill shapes); NV4_ERR_UNSUPPORTED for shapes it does not take.
// K is split (FP32 partials in `workspace`) when its plan asks for it and the
// workspace holds w4a16_tc_workspace_bytes; otherwise it is not.
int launch_w4a16_tc_gemm(const void* x, const void* qweight, const void* qzeros, const void* scales, void* out,
                         int64_t m, int64_t n, int64_t k, void* workspace, int64_t workspace_bytes,
                         cudaStream_t stream);
int64_t w4a16_tc_workspace_bytes(int64_t m, int64_t n, int64_t k);
bool w4a16_tc_plan(int64_t m, int64_t n, int64_t k, int sms, int* bn, int* splits);
void w4a16_plan(int64_t m, int64_t n, int64_t k, int sms, int64_t* plan);  // NV4_W4A16_PLAN_FIELDS values
// Same as launch_w4a16_gemm with the library's static scratch as workspace.
int launch_w4a16_gemm_static(const void* x, const void* qweight, const void* qzeros, const void* scales, void* out,
                             int64_t m, int64_t n, int64_t k, cudaStream_t stream);
bool w4a16_static_fits(int64_t m, int64_t n);  // (m, n) within the static scratch
// Paged decode attention and the q/k norm + rotary + KV store (attention.cu).
int64_t paged_attention_workspace_bytes(int64_t batch, int64_t num_heads, int64_t max_pages);
int launch_paged_decode_attention(const void* q, const void* k_cache, const void* v_cache, const int* block_tables,
                                  const int* context_lens, void* out, void* workspace, int64_t batch,
                                  int64_t num_heads, int64_t num_kv_heads, int64_t max_pages, float scale,
                                  cudaStream_t stream);
int launch_qk_norm_rope_store(const void* qkv, const void* q_weight, const void* k_weight, const float* cos_sin,
                              const int64_t* positions, const int* slot_mapping, void* q_out, void* k_out,
                              void* k_cache, void* v_cache, int64_t tokens, int64_t num_heads, int64_t num_kv_heads,
                              float eps, cudaStream_t stream);
// Peer mode of the stream GEMM (row-parallel layers): the launcher fills in the
// tile geometry the matching tile reduce needs.
// Launch plan of the decode stream GEMM (w4a4_gemm.cu); the C ABI exports it
// as nv4_w4a4_stream_plan for tests and tools.
struct StreamPlan {
  int token_tiles;     // 8-token tiles per CTA (1, 2 or 4)
  int slabs;           // 16-row weight slabs per CTA
  int k_split;         // consumer warps splitting K per slab (1 or 4)
  int token_splits;    // consumer warp groups splitting the token tiles
  int tiles_per_warp;  // token tiles per consumer warp
  int rows_per_cta;    // 16 * slabs
  int stages;          // shared-memory ring stages
  int n_iters;         // stages of K (two 128-groups each)
  int ds_bytes;        // K-split partial buffers
  int smem_bytes;      // dynamic shared memory per CTA
  int grid_x, grid_y;  // CTAs along N and along the token blocks
  int threads;         // threads per CTA (producers + consumers)
  int producer_warps;  // TMA-issuing warps, which take the stages round-robin
};
int plan_w4a4_stream(int64_t m, int64_t n, int64_t k, bool w_scale_grouped, int sms, bool peer, StreamPlan* out);

struct PeerTarget {
  void* const* bufs;  // world peer buffers, this rank's at [rank]
  int rank, world;
  int64_t capacity;
  int rows_per_cta = 0, ctas = 0;  // out
};
int launch_w4a4_stream_gemm(const void* a_packed, const void* a8, const void* w_packed, const void* a_scale,
                            const void* w_scale, void* out, int64_t m, int64_t n, int64_t k, int flags,
                            cudaStream_t stream, PeerTarget* peer = nullptr);
// Sum of the peer-mode GEMM's tiles in rank order to BF16 [m, n] (peer_allreduce.cu).
int launch_peer_reduce_tiles_bf16(void* const* bufs, int rank, int world, void* out, int m, int n, int rows_per_cta,
                                  int ctas, int64_t capacity, cudaStream_t stream);
// One-shot peer-memory all-reduce of FP32 partials to BF16 (peer_allreduce.cu).
int launch_peer_allreduce_bf16(void* const* bufs, int rank, int world, void* out, int64_t count, int64_t capacity,
                               cudaStream_t stream);
int64_t peer_buffer_data_bytes(int64_t capacity);  // partial + inboxes of one peer buffer

}  // namespace nv4
