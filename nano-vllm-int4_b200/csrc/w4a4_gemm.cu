// Kernel B: grouped INT4 x INT4 GEMM for decode shapes (few tokens).
//
// Semantics (nanovllm/kernels/w4a4_grouped_kernel.py:64-90): for each group g
// of 128 along K, in increasing g, total = fma(f32(dot_g), sa[m,g]*sw[n,g],
// total) with one FP32 rounding per group; BF16 (or FP32) output.  With a
// per-channel weight scale, total = fma(f32(dot_g), sa[m,g], total) and the
// result is multiplied by sw[n] at the end.  There is no split-K: each output
// element's FMA chain runs in one thread, in group order.
//
// Design: the weights are the streamed operand.  Each CTA owns R weight rows
// (a multiple of 16, chosen so the grid is about one CTA per SM) and all K.
// A producer warp streams [R x 256-K] packed weight tiles and the matching
// [MT*8 x 256-K] packed activation tiles into a ring of shared-memory stages
// with 2-D TMA copies (128-byte swizzle, no multicast), completion tracked by
// mbarriers.  Four consumer warps read fragments with ldmatrix straight from
// the packed nibbles (the packed layout is exactly the s4 MMA operand layout)
// and issue mma.sync m16n8k64 s4 with weights as the 16-row operand and tokens
// as the 8-column operand.  The INT32 accumulator starts at the bit pattern of
// 1.5*2^23, so after a group it reads as the float 12582912 + dot exactly and
// the conversion costs one FADD.  The weight tiles for the first stages are
// requested before griddepcontrol.wait, so with programmatic dependent launch
// the weight stream overlaps the activation-prep kernel that precedes it.
#include "nv4_device.cuh"
#include "nv4_launch.h"

namespace nv4 {

struct StreamGemmArgs {
  const uint16_t* a_scale;  // bf16 [M, G]
  const uint16_t* w_scale;  // bf16 [N, G] (grouped) or [N]
  void* out;                // bf16 or fp32 [M, N]
  int M, N, G;
  int R;        // weight rows per CTA (multiple of 16, <= 256)
  int n_iters;  // pipeline iterations = ceil(G / 2) (two groups per stage)
  int stages;
};

constexpr int kConsumerWarps = 4;
constexpr int kStreamThreads = 32 * (1 + kConsumerWarps);
constexpr int kMaxSlabsPerWarp = 4;  // R <= 256 -> 16 slabs of 16 rows

struct StreamSmem {
  uint32_t base;  // 1024-aligned shared address of stage 0
  int stage_bytes, w_bytes;
};

__device__ __forceinline__ bool mbar_wait_drain(uint64_t* bar, uint32_t parity) {
  const uint64_t start = global_timer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_timer_ns() - start > kWaitLimitNs) {
      record_error(kErrTimeoutDrain);
      return false;
    }
  }
  return true;
}

template <int MT, bool WGROUPED, bool OUT_F32>
__global__ void __launch_bounds__(kStreamThreads, 1)
    w4a4_stream_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_a,
                       const StreamGemmArgs p) {
  constexpr int MP = MT * 8;  // token rows per tile
  extern __shared__ uint8_t smem_raw[];
  const int S = p.stages, R = p.R, G = p.G;
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t pad = ((raw + 1023u) & ~1023u) - raw;
  uint8_t* smem = smem_raw + pad;
  const int w_bytes = R * 128, stage_bytes = w_bytes + MP * 128;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * stage_bytes);
  uint64_t* empty = full + S;
  int* issued = reinterpret_cast<int*>(empty + S);
  uint16_t* sw_s = reinterpret_cast<uint16_t*>(issued + 4);            // [G][R] (or [R])
  float* sa_s = reinterpret_cast<float*>(sw_s + (WGROUPED ? G * R : R) + 8);  // [G][MP]
  sa_s = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(sa_s) + 15) & ~uintptr_t(15));

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * R, m0 = blockIdx.y * MP;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    *issued = 0;
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == 0) {
    // ---------------- producer
    if (lane == 0) {
      tma_prefetch_desc(&tmap_w);
      tma_prefetch_desc(&tmap_a);
      const uint64_t wpol = policy_evict_first();
      const uint32_t bytes = static_cast<uint32_t>(stage_bytes);
      const int first = min(S, p.n_iters);
      for (int s = 0; s < first; ++s) {
        mbar_arrive_expect_tx(&full[s], bytes);
        tma_load_2d_hint(smem + s * stage_bytes, &tmap_w, &full[s], s * 128, n0, wpol);
      }
      grid_dependency_wait();  // activations come from the preceding kernel
      for (int s = 0; s < first; ++s) tma_load_2d(smem + s * stage_bytes + w_bytes, &tmap_a, &full[s], s * 128, m0);
      *reinterpret_cast<volatile int*>(issued) = first;
      for (int it = S; it < p.n_iters; ++it) {
        const int slot = it % S;
        if (!mbar_wait(&empty[slot], ((it / S) - 1) & 1, kErrTimeoutEmpty)) break;
        mbar_arrive_expect_tx(&full[slot], bytes);
        tma_load_2d_hint(smem + slot * stage_bytes, &tmap_w, &full[slot], it * 128, n0, wpol);
        tma_load_2d(smem + slot * stage_bytes + w_bytes, &tmap_a, &full[slot], it * 128, m0);
        *reinterpret_cast<volatile int*>(issued) = it + 1;
      }
    }
    return;
  }

  // ---------------- consumers
  const int ct = threadIdx.x - 32;
  const int cw = warp - 1;
  const int gid = lane >> 2, tig = lane & 3;
  if (WGROUPED) {
    for (int i = ct; i < R * G; i += 32 * kConsumerWarps) {
      const int r = i / G, g = i - r * G;
      sw_s[g * R + r] = (n0 + r < p.N) ? p.w_scale[static_cast<size_t>(n0 + r) * G + g] : uint16_t(0);
    }
  } else {
    for (int r = ct; r < R; r += 32 * kConsumerWarps) sw_s[r] = (n0 + r < p.N) ? p.w_scale[n0 + r] : uint16_t(0);
  }
  grid_dependency_wait();
  for (int i = ct; i < MP * G; i += 32 * kConsumerWarps) {
    const int t = i / G, g = i - t * G;
    sa_s[g * MP + t] = (m0 + t < p.M) ? bf16_bits_to_f32(p.a_scale[static_cast<size_t>(m0 + t) * G + g]) : 0.0f;
  }
  named_barrier_sync(1, 32 * kConsumerWarps);

  const int nslab = R / 16;
  float tot[kMaxSlabsPerWarp][MT][4];
#pragma unroll
  for (int s = 0; s < kMaxSlabsPerWarp; ++s)
#pragma unroll
    for (int t = 0; t < MT; ++t)
#pragma unroll
      for (int i = 0; i < 4; ++i) tot[s][t][i] = 0.0f;

  const uint32_t sbase = smem_u32(smem);
  int it = 0;
  bool ok = true;
  for (; it < p.n_iters; ++it) {
    const int slot = it % S;
    if (!mbar_wait(&full[slot], (it / S) & 1, kErrTimeoutFull)) {
      ok = false;
      break;
    }
    const uint32_t wbase = sbase + slot * stage_bytes, abase = wbase + w_bytes;
#pragma unroll
    for (int gg = 0; gg < 2; ++gg) {
      const int g = it * 2 + gg;
      if (g >= G) break;
      uint32_t bf[MT][4];
#pragma unroll
      for (int tt = 0; tt < MT; ++tt)
        ldmatrix_x4(abase + sw128_offset(tt * 8 + (lane & 7), gg * 4 + (lane >> 3)), bf[tt][0], bf[tt][1],
                    bf[tt][2], bf[tt][3]);
      float sa0[MT], sa1[MT];
#pragma unroll
      for (int tt = 0; tt < MT; ++tt) {
        const float2 v = *reinterpret_cast<const float2*>(sa_s + g * MP + tt * 8 + tig * 2);
        sa0[tt] = v.x;
        sa1[tt] = v.y;
      }
#pragma unroll
      for (int si = 0; si < kMaxSlabsPerWarp; ++si) {
        const int slab = cw + kConsumerWarps * si;
        if (slab >= nslab) break;
        uint32_t af0[4], af1[4];
        const uint32_t row = slab * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        ldmatrix_x4(wbase + sw128_offset(row, gg * 4 + (lane >> 4)), af0[0], af0[1], af0[2], af0[3]);
        ldmatrix_x4(wbase + sw128_offset(row, gg * 4 + 2 + (lane >> 4)), af1[0], af1[1], af1[2], af1[3]);
        float sw0 = 0.0f, sw1 = 0.0f;
        if (WGROUPED) {
          sw0 = bf16_bits_to_f32(sw_s[g * R + slab * 16 + gid]);
          sw1 = bf16_bits_to_f32(sw_s[g * R + slab * 16 + gid + 8]);
        }
#pragma unroll
        for (int tt = 0; tt < MT; ++tt) {
          int acc[4] = {kMagicBits, kMagicBits, kMagicBits, kMagicBits};
          mma_s4_16864(acc, af0, bf[tt][0], bf[tt][1]);
          mma_s4_16864(acc, af1, bf[tt][2], bf[tt][3]);
          const float d0 = __fsub_rn(__int_as_float(acc[0]), kMagic);
          const float d1 = __fsub_rn(__int_as_float(acc[1]), kMagic);
          const float d2 = __fsub_rn(__int_as_float(acc[2]), kMagic);
          const float d3 = __fsub_rn(__int_as_float(acc[3]), kMagic);
          if (WGROUPED) {
            tot[si][tt][0] = fmaf(d0, __fmul_rn(sa0[tt], sw0), tot[si][tt][0]);
            tot[si][tt][1] = fmaf(d1, __fmul_rn(sa1[tt], sw0), tot[si][tt][1]);
            tot[si][tt][2] = fmaf(d2, __fmul_rn(sa0[tt], sw1), tot[si][tt][2]);
            tot[si][tt][3] = fmaf(d3, __fmul_rn(sa1[tt], sw1), tot[si][tt][3]);
          } else {
            tot[si][tt][0] = fmaf(d0, sa0[tt], tot[si][tt][0]);
            tot[si][tt][1] = fmaf(d1, sa1[tt], tot[si][tt][1]);
            tot[si][tt][2] = fmaf(d2, sa0[tt], tot[si][tt][2]);
            tot[si][tt][3] = fmaf(d3, sa1[tt], tot[si][tt][3]);
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
  }

  if (!ok) {
    // Let every copy this CTA issued land before the CTA's shared memory is released.
    if (cw == 0 && lane == 0) {
      const int iss = *reinterpret_cast<volatile int*>(issued);
      for (int j = it; j < iss; ++j) mbar_wait_drain(&full[j % S], (j / S) & 1);
    }
    return;
  }

#pragma unroll
  for (int si = 0; si < kMaxSlabsPerWarp; ++si) {
    const int slab = cw + kConsumerWarps * si;
    if (slab >= nslab) break;
    const int r0 = n0 + slab * 16 + gid, r1 = r0 + 8;
    float swc0 = 1.0f, swc1 = 1.0f;
    if (!WGROUPED) {
      swc0 = bf16_bits_to_f32(sw_s[slab * 16 + gid]);
      swc1 = bf16_bits_to_f32(sw_s[slab * 16 + gid + 8]);
    }
#pragma unroll
    for (int tt = 0; tt < MT; ++tt) {
      const int t0 = m0 + tt * 8 + tig * 2, t1 = t0 + 1;
      float v[4] = {tot[si][tt][0], tot[si][tt][1], tot[si][tt][2], tot[si][tt][3]};
      if (!WGROUPED) {
        v[0] = __fmul_rn(v[0], swc0);
        v[1] = __fmul_rn(v[1], swc0);
        v[2] = __fmul_rn(v[2], swc1);
        v[3] = __fmul_rn(v[3], swc1);
      }
      const int rr[4] = {r0, r0, r1, r1}, tk[4] = {t0, t1, t0, t1};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        if (tk[i] < p.M && rr[i] < p.N) {
          const size_t o = static_cast<size_t>(tk[i]) * p.N + rr[i];
          if (OUT_F32)
            static_cast<float*>(p.out)[o] = v[i];
          else
            static_cast<__nv_bfloat16*>(p.out)[o] = __float2bfloat16_rn(v[i]);
        }
      }
    }
  }
}

// ------------------------------------------------------------ diagnostics
// dots[g, m, n] = exact INT32 dot of group g (one thread per output element).
__global__ void w4a4_group_dots_kernel(const uint8_t* __restrict__ a, const uint8_t* __restrict__ w,
                                       int32_t* __restrict__ dots, int M, int N, int K) {
  const int G = K / 128;
  const int64_t total = static_cast<int64_t>(G) * M * N;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int n = static_cast<int>(i % N);
    const int m = static_cast<int>((i / N) % M);
    const int g = static_cast<int>(i / (int64_t(N) * M));
    const uint8_t* pa = a + static_cast<size_t>(m) * (K / 2) + g * 64;
    const uint8_t* pw = w + static_cast<size_t>(n) * (K / 2) + g * 64;
    int acc = 0;
    for (int b = 0; b < 64; ++b) {
      const int a0 = (static_cast<int>(pa[b] << 28)) >> 28, a1 = (static_cast<int>(pa[b] << 24)) >> 28;
      const int w0 = (static_cast<int>(pw[b] << 28)) >> 28, w1 = (static_cast<int>(pw[b] << 24)) >> 28;
      acc += a0 * w0 + a1 * w1;
    }
    dots[i] = acc;
  }
}

// ------------------------------------------------------------ host side
template <int MT, bool WG, bool F32>
static int launch_stream_t(const CUtensorMap& tw, const CUtensorMap& ta, const StreamGemmArgs& a, dim3 grid,
                           int smem, cudaStream_t stream) {
  static int done[64] = {};
  const int rc = ensure_smem_attr(reinterpret_cast<const void*>(&w4a4_stream_kernel<MT, WG, F32>), smem, done);
  if (rc != NV4_OK) return rc;
  return launch_kernel(w4a4_stream_kernel<MT, WG, F32>, grid, dim3(kStreamThreads), smem, stream, true, tw, ta, a);
}

template <int MT>
static int launch_stream_mt(const CUtensorMap& tw, const CUtensorMap& ta, const StreamGemmArgs& a, dim3 grid,
                            int smem, bool wg, bool f32, cudaStream_t stream) {
  if (wg) return f32 ? launch_stream_t<MT, true, true>(tw, ta, a, grid, smem, stream)
                     : launch_stream_t<MT, true, false>(tw, ta, a, grid, smem, stream);
  return f32 ? launch_stream_t<MT, false, true>(tw, ta, a, grid, smem, stream)
             : launch_stream_t<MT, false, false>(tw, ta, a, grid, smem, stream);
}

constexpr int kSmemLimit = 227 * 1024;

int launch_w4a4_stream_gemm(const void* a_packed, const void* w_packed, const void* a_scale, const void* w_scale,
                            void* out, int64_t m, int64_t n, int64_t k, int flags, cudaStream_t stream) {
  const int sms = device_sm_count();
  if (sms <= 0) return NV4_ERR_CUDA;
  const bool wg = (flags & NV4_GEMM_W_SCALE_GROUPED) != 0;
  const bool f32 = (flags & NV4_GEMM_OUT_FP32) != 0;
  const int MT = m <= 8 ? 1 : (m <= 16 ? 2 : 4);
  const int MP = MT * 8;
  const int64_t mblocks = (m + MP - 1) / MP;
  const int G = static_cast<int>(k / 128);
  // About one CTA per SM: rows per CTA, rounded up to whole 16-row slabs.
  const int64_t ctas_per_mblock = std::max<int64_t>(1, sms / std::min<int64_t>(mblocks, sms));
  int64_t R = (n + ctas_per_mblock - 1) / ctas_per_mblock;
  R = std::min<int64_t>(256, std::max<int64_t>(16, (R + 15) / 16 * 16));
  const int scale_bytes = (wg ? G * static_cast<int>(R) : static_cast<int>(R)) * 2 + 16 + G * MP * 4 + 16;
  const int stage_bytes = static_cast<int>(R + MP) * 128;
  const int n_iters = (G + 1) / 2;
  int stages = (kSmemLimit - 1024 - scale_bytes - 64) / (stage_bytes + 16);
  stages = std::min(stages, std::min(8, n_iters));
  if (stages < 1) return NV4_ERR_UNSUPPORTED;
  const int smem = 1024 + stages * (stage_bytes + 16) + 16 + scale_bytes + 64;

  CUtensorMap tw, ta;
  if (!make_tensor_map_u8(&tw, w_packed, n, k / 2, static_cast<uint32_t>(R), 128, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_tensor_map_u8(&ta, a_packed, m, k / 2, static_cast<uint32_t>(MP), 128, CU_TENSOR_MAP_SWIZZLE_128B))
    return NV4_ERR_CUDA;
  StreamGemmArgs a;
  a.a_scale = static_cast<const uint16_t*>(a_scale);
  a.w_scale = static_cast<const uint16_t*>(w_scale);
  a.out = out;
  a.M = static_cast<int>(m);
  a.N = static_cast<int>(n);
  a.G = G;
  a.R = static_cast<int>(R);
  a.n_iters = n_iters;
  a.stages = stages;
  const dim3 grid(static_cast<unsigned>((n + R - 1) / R), static_cast<unsigned>(mblocks));
  if (MT == 1) return launch_stream_mt<1>(tw, ta, a, grid, smem, wg, f32, stream);
  if (MT == 2) return launch_stream_mt<2>(tw, ta, a, grid, smem, wg, f32, stream);
  return launch_stream_mt<4>(tw, ta, a, grid, smem, wg, f32, stream);
}

int launch_w4a4_group_dots(const void* a_packed, const void* w_packed, int32_t* dots, int64_t m, int64_t n, int64_t k,
                           cudaStream_t stream) {
  const int64_t total = (k / 128) * m * n;
  const int blocks = static_cast<int>(std::min<int64_t>((total + 255) / 256, 4096));
  return launch_kernel(w4a4_group_dots_kernel, dim3(blocks), dim3(256), 0, stream, false,
                       static_cast<const uint8_t*>(a_packed), static_cast<const uint8_t*>(w_packed), dots,
                       static_cast<int>(m), static_cast<int>(n), static_cast<int>(k));
}

}  // namespace nv4
