// Decode attention over the paged BF16 KV cache, and the per-head q/k RMSNorm
// + rotary embedding + KV-cache store that precedes it.  These serve the
// end-to-end model (the reference's nanovllm/layers/attention.py:59-75 calls
// flash_attn_with_kvcache for decode; nanovllm/models/qwen3.py:87-92 applies
// q_norm / k_norm and the rotary embedding; attention.py:10-40 stores K/V).
//
// Cache layout (the reference's): k_cache, v_cache [pages, page_size, Hkv, D]
// BF16 with page_size 256 and D 128; a sequence's token t lives in page
// block_table[t / 256] at row t % 256.
//
// Decode: one CTA per (sequence, KV head, page of the context).  The G = Hq /
// Hkv query heads of the KV head are the MMA's M rows (16 with padding), so
// every K/V row is read from HBM once for all of them.  A CTA streams its page
// in 64-token stages (cp.async, double-buffered, zero-filled past the
// sequence), each of its four warps takes 16 tokens of a stage: S = Q K^T and
// O += P V on mma.sync m16n8k16 BF16 with FP32 accumulators, online softmax in
// the exp2 domain.  The warps' states are merged in shared memory and the
// page's unnormalised output, running max and sum are written to a partial
// buffer; a second kernel merges the pages of each (sequence, head).
#include <cstring>

#include "nv4_device.cuh"
#include "nv4_launch.h"

namespace nv4 {

constexpr int kAttnD = 128;
constexpr int kAttnPage = 256;
constexpr int kAttnStage = 64;                 // tokens per shared-memory stage
constexpr int kAttnRowBytes = kAttnD * 2 + 16;  // padded row: conflict-free ldmatrix
constexpr int kAttnMaxGroup = 16;

struct PagedAttnArgs {
  const uint16_t* q;        // [B, Hq, D]
  const uint16_t* k_cache;  // [pages, 256, Hkv, D]
  const uint16_t* v_cache;
  const int* block_tables;  // [B, max_pages]
  const int* context_lens;  // [B]
  float* o_part;            // [B, Hq, max_pages, D]
  float* ml_part;           // [B, Hq, max_pages, 2]: running max (log2 domain), sum
  int Hq, Hkv, max_pages;
  float scale_log2;         // softmax scale * log2(e)
};

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                                  uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void mma_bf16_m16n8k16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

__global__ void __launch_bounds__(128) paged_decode_attention_kernel(const PagedAttnArgs p) {
  extern __shared__ __align__(128) uint8_t smem_attn[];
  const int b = blockIdx.x, kvh = blockIdx.y, pi = blockIdx.z;
  const int ctx = p.context_lens[b];
  const int t0 = pi * kAttnPage;
  if (t0 >= ctx) return;
  const int ntok = min(kAttnPage, ctx - t0);
  const int page = p.block_tables[static_cast<size_t>(b) * p.max_pages + pi];
  const int G = p.Hq / p.Hkv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gid = lane >> 2, tig = lane & 3;

  // shared memory: q rows (G + one zero row), two stages of K and V
  uint8_t* qs = smem_attn;
  uint8_t* kv = smem_attn + (kAttnMaxGroup + 1) * kAttnRowBytes;
  constexpr int kStageBytes = 2 * kAttnStage * kAttnRowBytes;  // K then V
  const size_t row_stride = static_cast<size_t>(p.Hkv) * kAttnD;  // elements between cache rows
  const uint16_t* kbase = p.k_cache + (static_cast<size_t>(page) * kAttnPage) * row_stride + kvh * kAttnD;
  const uint16_t* vbase = p.v_cache + (static_cast<size_t>(page) * kAttnPage) * row_stride + kvh * kAttnD;

  auto load_stage = [&](int st) {
    uint8_t* dst = kv + (st & 1) * kStageBytes;
    for (int i = threadIdx.x; i < 2 * kAttnStage * 16; i += 128) {
      const int which = i / (kAttnStage * 16), r = (i / 16) % kAttnStage, c = i % 16;
      const int tok = st * kAttnStage + r;
      const uint16_t* src = (which ? vbase : kbase) + static_cast<size_t>(min(tok, ntok - 1)) * row_stride + c * 8;
      cp_async16(smem_u32(dst + which * kAttnStage * kAttnRowBytes + r * kAttnRowBytes + c * 16), src,
                 tok < ntok ? 16u : 0u);
    }
  };
  const int nst = (ntok + kAttnStage - 1) / kAttnStage;
  load_stage(0);
  cp_async_commit();

  // q of the group's heads, and a zero row for the MMA's padding rows
  for (int i = threadIdx.x; i < (G + 1) * 16; i += 128) {
    const int r = i / 16, c = i % 16;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (r < G) v = __ldg(reinterpret_cast<const uint4*>(p.q + (static_cast<size_t>(b) * p.Hq + kvh * G + r) * kAttnD) + c);
    *reinterpret_cast<uint4*>(qs + (r < G ? r : kAttnMaxGroup) * kAttnRowBytes + c * 16) = v;
  }
  __syncthreads();
  uint32_t qa[8][4];
  {
    const int r = lane & 15;
    const uint32_t qaddr = smem_u32(qs) + (r < G ? r : kAttnMaxGroup) * kAttnRowBytes + (lane >> 4) * 16;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) ldmatrix_x4(qaddr + ks * 32, qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3]);
  }

  float o[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) o[i][e] = 0.0f;
  float m_run = -1e30f, l_run = 0.0f;  // of row gid (rows gid + 8 are padding)

  for (int st = 0; st < nst; ++st) {
    if (st + 1 < nst) {
      load_stage(st + 1);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const uint32_t kst = smem_u32(kv + (st & 1) * kStageBytes) + warp * 16 * kAttnRowBytes;
    const uint32_t vst = kst + kAttnStage * kAttnRowBytes;
    // S = Q K^T for this warp's 16 tokens (two n8 tiles)
    float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    {
      const int tok = (lane & 7) + ((lane >> 4) << 3), chunk = (lane >> 3) & 1;
      const uint32_t kaddr = kst + tok * kAttnRowBytes + chunk * 16;
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        uint32_t r0, r1, r2, r3;
        ldmatrix_x4(kaddr + ks * 32, r0, r1, r2, r3);
        mma_bf16_m16n8k16(s[0], qa[ks], r0, r1);
        mma_bf16_m16n8k16(s[1], qa[ks], r2, r3);
      }
    }
    // online softmax over the 16 tokens (row gid: s[j][0], s[j][1])
    const int tbase = st * kAttnStage + warp * 16 + 2 * tig;
    float x[4];
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int t = tbase + j * 8 + e;
        x[j * 2 + e] = t < ntok ? s[j][e] * p.scale_log2 : -INFINITY;
      }
    float mx = fmaxf(fmaxf(x[0], x[1]), fmaxf(x[2], x[3]));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float m_new = fmaxf(m_run, mx);
    const float alpha = exp2f(m_run - m_new);
    float pr[4], rs = 0.0f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      pr[i] = exp2f(x[i] - m_new);
      rs += pr[i];
    }
    rs += __shfl_xor_sync(0xffffffffu, rs, 1);
    rs += __shfl_xor_sync(0xffffffffu, rs, 2);
    l_run = l_run * alpha + rs;
    m_run = m_new;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      o[i][0] *= alpha;
      o[i][1] *= alpha;
    }
    // P as the A fragment (rows gid + 8 are padding: zero)
    uint32_t pa[4];
    pa[0] = pack_bf16x2(pr[0], pr[1]);
    pa[1] = 0u;
    pa[2] = pack_bf16x2(pr[2], pr[3]);
    pa[3] = 0u;
    // O += P V
    {
      const int tok = (lane & 7) + (((lane >> 3) & 1) << 3), chunk = lane >> 4;
      const uint32_t vaddr = vst + tok * kAttnRowBytes + chunk * 16;
#pragma unroll
      for (int dt = 0; dt < 16; dt += 2) {
        uint32_t r0, r1, r2, r3;
        ldmatrix_x4_trans(vaddr + dt * 16, r0, r1, r2, r3);
        mma_bf16_m16n8k16(o[dt], pa, r0, r1);
        mma_bf16_m16n8k16(o[dt + 1], pa, r2, r3);
      }
    }
    __syncthreads();  // the stage buffer is refilled two stages on
  }

  // merge the four warps: per row g < G, each warp's (m, l) and O[g][:]
  float* red = reinterpret_cast<float*>(kv);  // reuse the stage buffers
  float* ml = red + 4 * kAttnMaxGroup * kAttnD;
  if (gid < G) {
#pragma unroll
    for (int dt = 0; dt < 16; ++dt) {
      float* dst = red + (warp * kAttnMaxGroup + gid) * kAttnD + dt * 8 + 2 * tig;
      dst[0] = o[dt][0];
      dst[1] = o[dt][1];
    }
    if (tig == 0) {
      ml[(warp * kAttnMaxGroup + gid) * 2] = m_run;
      ml[(warp * kAttnMaxGroup + gid) * 2 + 1] = l_run;
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < G * kAttnD; i += 128) {
    const int g = i / kAttnD, d = i % kAttnD;
    float M = -1e30f;
#pragma unroll
    for (int w = 0; w < 4; ++w) M = fmaxf(M, ml[(w * kAttnMaxGroup + g) * 2]);
    float acc = 0.0f, L = 0.0f;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const float f = exp2f(ml[(w * kAttnMaxGroup + g) * 2] - M);
      acc += f * red[(w * kAttnMaxGroup + g) * kAttnD + d];
      L += f * ml[(w * kAttnMaxGroup + g) * 2 + 1];
    }
    const size_t part = (static_cast<size_t>(b) * p.Hq + kvh * G + g) * p.max_pages + pi;
    p.o_part[part * kAttnD + d] = acc;
    if (d == 0) {
      p.ml_part[part * 2] = M;
      p.ml_part[part * 2 + 1] = L;
    }
  }
}

// out[b, h, :] = merge of the pages of (b, h): sum_p 2^(m_p - M) o_p / sum_p 2^(m_p - M) l_p.
__global__ void __launch_bounds__(128) paged_attention_merge_kernel(const float* __restrict__ o_part,
                                                                     const float* __restrict__ ml_part,
                                                                     const int* __restrict__ context_lens,
                                                                     uint16_t* __restrict__ out, int Hq,
                                                                     int max_pages) {
  const int bh = blockIdx.x, b = bh / Hq, d = threadIdx.x;
  const int ctx = context_lens[b];
  const int np = min(max_pages, (ctx + kAttnPage - 1) / kAttnPage);
  const size_t base = static_cast<size_t>(bh) * max_pages;
  float M = -1e30f;
  for (int i = 0; i < np; ++i) M = fmaxf(M, ml_part[(base + i) * 2]);
  float acc = 0.0f, L = 0.0f;
  for (int i = 0; i < np; ++i) {
    const float f = exp2f(ml_part[(base + i) * 2] - M);
    acc += f * o_part[(base + i) * kAttnD + d];
    L += f * ml_part[(base + i) * 2 + 1];
  }
  out[static_cast<size_t>(bh) * kAttnD + d] = __bfloat16_as_ushort(__float2bfloat16_rn(np > 0 ? acc / L : 0.0f));
}

constexpr int kAttnSmem = (kAttnMaxGroup + 1) * kAttnRowBytes + 2 * 2 * kAttnStage * kAttnRowBytes;
static_assert(4 * kAttnMaxGroup * kAttnD * 4 + 4 * kAttnMaxGroup * 2 * 4 <= 2 * 2 * kAttnStage * kAttnRowBytes,
              "merge scratch fits in the stage buffers");

int64_t paged_attention_workspace_bytes(int64_t batch, int64_t num_heads, int64_t max_pages) {
  return batch * num_heads * max_pages * (kAttnD + 2) * 4;
}

int launch_paged_decode_attention(const void* q, const void* k_cache, const void* v_cache, const int* block_tables,
                                  const int* context_lens, void* out, void* workspace, int64_t batch,
                                  int64_t num_heads, int64_t num_kv_heads, int64_t max_pages, float scale,
                                  cudaStream_t stream) {
  static int done[64] = {};
  const int rc = ensure_smem_attr(reinterpret_cast<const void*>(&paged_decode_attention_kernel), kAttnSmem, done);
  if (rc != NV4_OK) return rc;
  PagedAttnArgs a;
  a.q = static_cast<const uint16_t*>(q);
  a.k_cache = static_cast<const uint16_t*>(k_cache);
  a.v_cache = static_cast<const uint16_t*>(v_cache);
  a.block_tables = block_tables;
  a.context_lens = context_lens;
  a.o_part = static_cast<float*>(workspace);
  a.ml_part = a.o_part + batch * num_heads * max_pages * kAttnD;
  a.Hq = static_cast<int>(num_heads);
  a.Hkv = static_cast<int>(num_kv_heads);
  a.max_pages = static_cast<int>(max_pages);
  a.scale_log2 = scale * 1.4426950408889634f;
  const dim3 grid(static_cast<unsigned>(batch), static_cast<unsigned>(num_kv_heads), static_cast<unsigned>(max_pages));
  int r = launch_kernel(paged_decode_attention_kernel, grid, dim3(128), kAttnSmem, stream, false, a);
  if (r != NV4_OK) return r;
  return launch_kernel(paged_attention_merge_kernel, dim3(static_cast<unsigned>(batch * num_heads)), dim3(kAttnD), 0,
                       stream, false, static_cast<const float*>(a.o_part), static_cast<const float*>(a.ml_part),
                       context_lens, static_cast<uint16_t*>(out), a.Hq, a.max_pages);
}

// ------------------------------------------------------------ q/k norm, rotary, KV store
// One warp per (token, head) of the fused QKV output [T, (Hq + 2 Hkv) * D]:
// q heads: RMSNorm over D with q_weight, rotary embedding, to q_out [T, Hq, D];
// k heads: RMSNorm with k_weight, rotary, to the cache row slot_mapping[t]
// (and to k_out [T, Hkv, D] when given); v heads: copied to the cache row.
// Slots < 0 (padding rows of a captured batch) store nothing.
// Numerics as the reference: RMSNorm = bf16(bf16(x * rsqrt(mean(x^2) + eps)) *
// w) (nanovllm/layers/layernorm.py:17-27), rotary on FP32 copies of the BF16
// halves, y1 = x1 cos - x2 sin, y2 = x2 cos + x1 sin, rounded to BF16
// (nanovllm/layers/rotary_embedding.py:6-14) with the reference's FP32
// cos/sin table (cos_sin [max_pos, D]: cos in the first D/2 columns).
struct QkNormRopeArgs {
  const uint16_t* qkv;
  const uint16_t* q_weight;
  const uint16_t* k_weight;
  const float* cos_sin;
  const int64_t* positions;
  const int* slot_mapping;
  uint16_t* q_out;
  uint16_t* k_out;  // or nullptr
  uint16_t* k_cache;
  uint16_t* v_cache;
  int T, Hq, Hkv;
  float eps;
};

__device__ __forceinline__ float bf16r(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

__global__ void __launch_bounds__(256) qk_norm_rope_store_kernel(const QkNormRopeArgs p) {
  const int heads = p.Hq + 2 * p.Hkv;
  const int gw = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (gw >= p.T * heads) return;
  const int t = gw / heads, h = gw - t * heads;
  const uint16_t* src = p.qkv + (static_cast<size_t>(t) * heads + h) * kAttnD + lane * 4;
  const uint2 raw = *reinterpret_cast<const uint2*>(src);
  float x[4] = {bf16lo_to_f32(raw.x), bf16hi_to_f32(raw.x), bf16lo_to_f32(raw.y), bf16hi_to_f32(raw.y)};
  const int slot = p.slot_mapping != nullptr ? p.slot_mapping[t] : -1;
  const size_t cache_row = static_cast<size_t>(slot) * p.Hkv * kAttnD;
  if (h >= p.Hq + p.Hkv) {  // v: copied to the cache
    if (slot >= 0) *reinterpret_cast<uint2*>(p.v_cache + cache_row + (h - p.Hq - p.Hkv) * kAttnD + lane * 4) = raw;
    return;
  }
  const bool is_q = h < p.Hq;
  const uint16_t* wgt = (is_q ? p.q_weight : p.k_weight) + lane * 4;
  float ss = 0.0f;
#pragma unroll
  for (int i = 0; i < 4; ++i) ss = fmaf(x[i], x[i], ss);
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, m);
  const float r = rsqrtf(ss * (1.0f / kAttnD) + p.eps);
  const uint2 wr = *reinterpret_cast<const uint2*>(wgt);
  const float w[4] = {bf16lo_to_f32(wr.x), bf16hi_to_f32(wr.x), bf16lo_to_f32(wr.y), bf16hi_to_f32(wr.y)};
  float y[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) y[i] = bf16r(bf16r(x[i] * r) * w[i]);
  // rotary: lane l < 16 holds x1[4l..4l+3], lane l + 16 holds x2[4l..4l+3]
  const int64_t pos = p.positions[t];
  const int fi = (lane & 15) * 4;
  const float* cs = p.cos_sin + pos * kAttnD;
  float other[4], out[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) other[i] = __shfl_xor_sync(0xffffffffu, y[i], 16);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float c = cs[fi + i], s = cs[kAttnD / 2 + fi + i];
    out[i] = lane < 16 ? y[i] * c - other[i] * s : y[i] * c + other[i] * s;
  }
  const uint2 packed = make_uint2(pack_bf16x2(out[0], out[1]), pack_bf16x2(out[2], out[3]));
  if (is_q) {
    *reinterpret_cast<uint2*>(p.q_out + (static_cast<size_t>(t) * p.Hq + h) * kAttnD + lane * 4) = packed;
  } else {
    const int kh = h - p.Hq;
    if (slot >= 0) *reinterpret_cast<uint2*>(p.k_cache + cache_row + kh * kAttnD + lane * 4) = packed;
    if (p.k_out != nullptr)
      *reinterpret_cast<uint2*>(p.k_out + (static_cast<size_t>(t) * p.Hkv + kh) * kAttnD + lane * 4) = packed;
  }
}

int launch_qk_norm_rope_store(const void* qkv, const void* q_weight, const void* k_weight, const float* cos_sin,
                              const int64_t* positions, const int* slot_mapping, void* q_out, void* k_out,
                              void* k_cache, void* v_cache, int64_t tokens, int64_t num_heads, int64_t num_kv_heads,
                              float eps, cudaStream_t stream) {
  QkNormRopeArgs a;
  a.qkv = static_cast<const uint16_t*>(qkv);
  a.q_weight = static_cast<const uint16_t*>(q_weight);
  a.k_weight = static_cast<const uint16_t*>(k_weight);
  a.cos_sin = cos_sin;
  a.positions = positions;
  a.slot_mapping = slot_mapping;
  a.q_out = static_cast<uint16_t*>(q_out);
  a.k_out = static_cast<uint16_t*>(k_out);
  a.k_cache = static_cast<uint16_t*>(k_cache);
  a.v_cache = static_cast<uint16_t*>(v_cache);
  a.T = static_cast<int>(tokens);
  a.Hq = static_cast<int>(num_heads);
  a.Hkv = static_cast<int>(num_kv_heads);
  a.eps = eps;
  const int64_t warps = tokens * (num_heads + 2 * num_kv_heads);
  return launch_kernel(qk_norm_rope_store_kernel, dim3(static_cast<unsigned>((warps + 7) / 8)), dim3(256), 0, stream,
                       false, a);
}

}  // namespace nv4
