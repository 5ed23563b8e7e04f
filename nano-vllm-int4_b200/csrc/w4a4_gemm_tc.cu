// Kernel C: grouped INT4 x INT4 GEMM on 5th-generation tensor cores (tcgen05).
//
// Same semantics as Kernel B (nanovllm/kernels/w4a4_grouped_kernel.py:64-90):
// per 128-wide K group g, in increasing g, total = fma(f32(dot_g),
// sa[m,g]*sw[n,g], total); BF16 (or FP32) output; no split-K.
//
// One CTA computes a tile of 128 weight rows x BN tokens over all of K:
//   warp 0      TMA producer: per group, the packed weight tile [128 x 64 B]
//               (64-byte swizzle) and the token tile [BN x 128 B] of INT8 codes
//               in the GEMM-ready layout (128-byte swizzle, which is exactly
//               the K-major UMMA operand layout) into a ring of stages.
//   warp 1      TMEM allocation and the single MMA-issuing thread:
//               4 x tcgen05.mma kind::i8 (M=128, N=BN, K=32) per group into
//               one of two TMEM accumulators, then tcgen05.commit.
//   warps 2-5   widen the packed weights to INT8 (16*code, each 32-wide K chunk
//               as its 16 even-k codes then its 16 odd-k codes -- the token
//               operand's K order) into 128-byte-swizzled K-major smem.
//   warps 6-    epilogue: tcgen05.ld the INT32 partials of a group (thread =
//               weight row), re-seed the buffer with the bias bits of 1.5*2^23
//               (so the MMAs accumulate onto it and the INT32 reads as the
//               float 12582912 + 16*dot), and apply the group's scales in FP32.
// When the scales of a group are in range (always, for the quantizer's), the
// epilogue uses two FMAs per element: ds = fma(F, sw/16, -786432*sw) = dot*sw
// exactly, total = fma(ds, sa, total) = fma(dot, sa*sw, total) since sa*sw is
// exact in FP32; otherwise the reference's three-step form.
//
// Weights and weight scales are requested before griddepcontrol.wait, so with
// programmatic dependent launch they stream while the activation-prep kernel
// before this one is still running.  Every wait is bounded; on a timeout the
// roles stop, the MMA thread waits for its issued MMAs and the TMEM is freed.
#include <cstring>

#include "nv4_device.cuh"
#include "nv4_launch.h"

namespace nv4 {

struct TcArgs {
  const uint16_t* a_scale;  // bf16 [M, G]
  const uint16_t* w_scale;  // bf16 [N, G] (grouped) or [N]
  void* out;                // bf16 or fp32 [M, N]
  int M, N, G;
  int stages;       // TMA ring depth
  int scale_tma;    // scales by TMA (row bytes multiple of 16)
};

constexpr int kTcWidenWarps = 4;
constexpr int kTcFirstEpiWarp = 2 + kTcWidenWarps;
constexpr int kTcWBufs = 2;  // widened weight buffers

__host__ __device__ constexpr int tc_epi_warps(int bn) { return bn >= 128 ? 8 : 4; }
__host__ __device__ constexpr int tc_threads(int bn) { return 32 * (kTcFirstEpiWarp + tc_epi_warps(bn)); }
__host__ __device__ constexpr int tc_tmem_cols(int bn) { return 2 * bn < 32 ? 32 : 2 * bn; }

struct TcLayout {
  int w_bytes, a_bytes, stage_bytes, wide_off, sw_off, sa_off, saf_off, flag_off, bar_off, total;
  __host__ __device__ TcLayout(int BN, int G, int S, bool wg) {
    w_bytes = 128 * 64;
    a_bytes = BN * 128;
    stage_bytes = ((w_bytes + a_bytes) + 1023) & ~1023;
    wide_off = S * stage_bytes;
    sw_off = wide_off + kTcWBufs * 16384;
    const int sw_bytes = (wg ? 128 * G : 128) * 2;
    sa_off = (sw_off + sw_bytes + 1023) & ~1023;
    saf_off = (sa_off + BN * G * 2 + 15) & ~15;
    flag_off = saf_off + G * BN * 4;
    bar_off = (flag_off + G * 4 + 7) & ~7;
    // full_w[S], full_a[S], sfree[S], wfull[2], wfree[2], tfull[2], tfree[2], scale[2], done[1], tmem slot
    total = bar_off + (3 * S + 11) * 8 + 16;
  }
};

__device__ __forceinline__ bool tc_fast_scale(float s) {
  const float a = fabsf(s);
  return a == 0.0f || (a >= 0x1.0p-60f && a <= 0x1.0p+60f);
}

template <int BN, bool WG, bool F32>
__global__ void __launch_bounds__(tc_threads(BN), 1)
    w4a4_tc_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_a,
                   const __grid_constant__ CUtensorMap tmap_sw, const __grid_constant__ CUtensorMap tmap_sa,
                   const TcArgs p) {
  constexpr int EW = tc_epi_warps(BN);
  constexpr int COLS = BN / (EW / 4);  // token columns per epilogue thread
  constexpr uint32_t IDESC = umma_idesc_s8(128, BN);
  extern __shared__ uint8_t smem_raw[];
  const int S = p.stages, G = p.G;
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  const TcLayout L(BN, G, S, WG);
  uint16_t* sw_s = reinterpret_cast<uint16_t*>(smem + L.sw_off);  // [128][G] (or [128])
  uint16_t* sa_s = reinterpret_cast<uint16_t*>(smem + L.sa_off);  // [BN][G]
  float* saf = reinterpret_cast<float*>(smem + L.saf_off);         // [G][BN]
  int* fast_g = reinterpret_cast<int*>(smem + L.flag_off);         // [G]
  uint64_t* full_w = reinterpret_cast<uint64_t*>(smem + L.bar_off);
  uint64_t* full_a = full_w + S;
  uint64_t* sfree = full_a + S;
  uint64_t* wfull = sfree + S;
  uint64_t* wfree = wfull + kTcWBufs;
  uint64_t* tfull = wfree + kTcWBufs;
  uint64_t* tfree = tfull + 2;
  uint64_t* scale_bar = tfree + 2;
  uint64_t* done_bar = scale_bar + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done_bar + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * 128, m0 = blockIdx.y * BN;
  grid_dependents_launch();

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full_w[s], 1);
      mbar_init(&full_a[s], 1);
      mbar_init(&sfree[s], kTcWidenWarps + 1);
    }
    for (int i = 0; i < kTcWBufs; ++i) {
      mbar_init(&wfull[i], kTcWidenWarps);
      mbar_init(&wfree[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tfree[i], EW);
      mbar_init(&scale_bar[i], 1);
    }
    mbar_init(done_bar, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, tc_tmem_cols(BN));
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool ok = true;

  if (warp == 0) {
    // ---------------- TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tmap_w);
      tma_prefetch_desc(&tmap_a);
      const uint64_t wpol = policy_evict_first();
      if (p.scale_tma) {
        mbar_arrive_expect_tx(&scale_bar[0], static_cast<uint32_t>((WG ? 128 * G : 128) * 2));
        if (WG)
          tma_load_2d(sw_s, &tmap_sw, &scale_bar[0], 0, n0);
        else
          tma_load_2d(sw_s, &tmap_sw, &scale_bar[0], n0, 0);
      }
      const int first = min(S, G);
      for (int g = 0; g < first; ++g) {
        mbar_arrive_expect_tx(&full_w[g], static_cast<uint32_t>(L.w_bytes));
        tma_load_2d_hint(smem + g * L.stage_bytes, &tmap_w, &full_w[g], g * 64, n0, wpol);
      }
      grid_dependency_wait();  // the token codes and scales come from the preceding kernel
      if (p.scale_tma) {
        mbar_arrive_expect_tx(&scale_bar[1], static_cast<uint32_t>(BN * G * 2));
        tma_load_2d(sa_s, &tmap_sa, &scale_bar[1], 0, m0);
      }
      for (int g = 0; g < first; ++g) {
        mbar_arrive_expect_tx(&full_a[g], static_cast<uint32_t>(L.a_bytes));
        tma_load_2d(smem + g * L.stage_bytes + L.w_bytes, &tmap_a, &full_a[g], g * 128, m0);
      }
      int issued = first;
      for (int g = first; g < G && ok; ++g) {
        const int s = g % S;
        if (!mbar_wait(&sfree[s], ((g / S) - 1) & 1, kErrTimeoutEmpty)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&full_w[s], static_cast<uint32_t>(L.w_bytes));
        tma_load_2d_hint(smem + s * L.stage_bytes, &tmap_w, &full_w[s], g * 64, n0, wpol);
        mbar_arrive_expect_tx(&full_a[s], static_cast<uint32_t>(L.a_bytes));
        tma_load_2d(smem + s * L.stage_bytes + L.w_bytes, &tmap_a, &full_a[s], g * 128, m0);
        issued = g + 1;
      }
      // Before the CTA may exit, every copy issued must have landed.
      for (int g = max(0, issued - S); g < issued; ++g) {
        const int s = g % S;
        if (!mbar_wait(&full_a[s], (g / S) & 1, kErrTimeoutDrain)) break;
        if (!mbar_wait(&full_w[s], (g / S) & 1, kErrTimeoutDrain)) break;
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer
    if (lane == 0) {
      const uint32_t wide_base = smem_u32(smem + L.wide_off);
      const uint32_t stage_base = smem_u32(smem);
      for (int g = 0; g < G && ok; ++g) {
        const int s = g % S, w = g % kTcWBufs, b = g & 1;
        ok = mbar_wait(&wfull[w], (g / kTcWBufs) & 1, kErrTimeoutMma) &&
             mbar_wait(&full_a[s], (g / S) & 1, kErrTimeoutMma) && mbar_wait(&tfree[b], (g >> 1) & 1, kErrTimeoutMma);
        if (!ok) break;
        tc_fence_after();
        const uint32_t a_addr = wide_base + w * 16384;
        const uint32_t b_addr = stage_base + s * L.stage_bytes + L.w_bytes;
#pragma unroll
        for (int k = 0; k < 4; ++k)
          umma_s8(tmem + b * BN, umma_desc_sw128(a_addr + k * 32), umma_desc_sw128(b_addr + k * 32), IDESC, 1);
        umma_commit(&tfull[b]);
        umma_commit(&wfree[w]);
        umma_commit(&sfree[s]);
      }
      // all issued MMAs must finish before the TMEM is released
      umma_commit(done_bar);
      mbar_wait(done_bar, 0, kErrTimeoutDrain);
    }
  } else if (warp < kTcFirstEpiWarp) {
    // ---------------- widen: thread t owns weight row t of the tile
    const int t = (warp - 2) * 32 + lane;
    const uint32_t stage_base = smem_u32(smem);
    const uint32_t wide_base = smem_u32(smem + L.wide_off);
    for (int g = 0; g < G && ok; ++g) {
      const int s = g % S, w = g % kTcWBufs;
      ok = mbar_wait(&full_w[s], (g / S) & 1, kErrTimeoutFull);
      if (ok && g >= kTcWBufs) ok = mbar_wait(&wfree[w], ((g / kTcWBufs) - 1) & 1, kErrTimeoutFull);
      if (!ok) break;
      uint4 pk[4];
      const uint8_t* src = smem + s * L.stage_bytes + t * 64;
#pragma unroll
      for (int c = 0; c < 4; ++c)
        pk[c] = *reinterpret_cast<const uint4*>(src + ((c ^ ((t >> 1) & 3)) << 4));
      __syncwarp();
      if (lane == 0) mbar_arrive(&sfree[s]);  // packed weights read
      const uint32_t row_base = wide_base + w * 16384 + (t >> 3) * 1024 + (t & 7) * 128;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const uint4 e = make_uint4(nib_even16(pk[c].x), nib_even16(pk[c].y), nib_even16(pk[c].z),
                                   nib_even16(pk[c].w));
        const uint4 o = make_uint4(nib_odd16(pk[c].x), nib_odd16(pk[c].y), nib_odd16(pk[c].z), nib_odd16(pk[c].w));
        const uint32_t pe = ((2 * c) ^ (t & 7)) << 4, po = ((2 * c + 1) ^ (t & 7)) << 4;
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(row_base + pe), "r"(e.x), "r"(e.y), "r"(e.z),
                     "r"(e.w)
                     : "memory");
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(row_base + po), "r"(o.x), "r"(o.y), "r"(o.z),
                     "r"(o.w)
                     : "memory");
      }
      fence_proxy_async_smem();  // make the generic-proxy stores visible to the tensor core
      __syncwarp();
      if (lane == 0) mbar_arrive(&wfull[w]);
    }
  } else {
    // ---------------- epilogue: thread = weight row (TMEM lane), COLS token columns
    const int ew = warp - kTcFirstEpiWarp;
    const int sub = warp & 3;                  // TMEM lane quarter this warp may access
    const int row = sub * 32 + lane;
    const int c0 = (ew >> 2) * COLS;           // first token column of this thread
    const int et = ew * 32 + lane, ethreads = EW * 32;
    const uint32_t taddr = tmem + (static_cast<uint32_t>(sub * 32) << 16) + c0;
    // seed both accumulators with the bias bits
#pragma unroll
    for (int b = 0; b < 2; ++b)
#pragma unroll
      for (int c = 0; c < COLS; c += 16) tmem_st16(taddr + b * BN + c, static_cast<uint32_t>(kMagicBits));
    tmem_wait_st();
    tc_fence_before();
    __syncwarp();
    if (lane == 0) {
      mbar_arrive(&tfree[0]);
      mbar_arrive(&tfree[1]);
    }
    // scales
    if (!p.scale_tma) {
      const int nsw = WG ? 128 * G : 128;
      for (int i = et; i < nsw; i += ethreads) {
        const int r = WG ? i / G : i;
        sw_s[i] = (n0 + r < p.N) ? p.w_scale[static_cast<size_t>(n0) * (WG ? G : 1) + i] : uint16_t(0);
      }
    } else {
      ok = mbar_wait(&scale_bar[0], 0, kErrTimeoutFull);
    }
    for (int g = et; g < G; g += ethreads) fast_g[g] = 1;
    grid_dependency_wait();
    if (!p.scale_tma) {
      for (int i = et; i < BN * G; i += ethreads)
        sa_s[i] = (m0 + i / G < p.M) ? p.a_scale[static_cast<size_t>(m0) * G + i] : uint16_t(0);
    } else {
      ok = mbar_wait(&scale_bar[1], 0, kErrTimeoutFull) && ok;
    }
    named_barrier_sync(1, ethreads);
    for (int i = et; i < BN * G; i += ethreads) {
      const int j = i / G, g = i - j * G;
      const float sa = bf16_bits_to_f32(sa_s[i]);
      saf[g * BN + j] = sa;
      if (!tc_fast_scale(sa)) fast_g[g] = 0;
    }
    if (WG)
      for (int i = et; i < 128 * G; i += ethreads)
        if (!tc_fast_scale(bf16_bits_to_f32(sw_s[i]))) fast_g[i % G] = 0;
    named_barrier_sync(1, ethreads);

    float tot[COLS];
#pragma unroll
    for (int j = 0; j < COLS; ++j) tot[j] = 0.0f;
    for (int g = 0; g < G && ok; ++g) {
      const int b = g & 1;
      if (!mbar_wait(&tfull[b], (g >> 1) & 1, kErrTimeoutMma)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const float sw = WG ? bf16_bits_to_f32(sw_s[row * G + g]) : 1.0f;
      const float* sag = saf + g * BN + c0;
      const bool fast = WG && fast_g[g] != 0;
      const float cw1 = __fmul_rn(sw, 0.0625f), cw2 = __fmul_rn(sw, -786432.0f);
      constexpr int CH = COLS < 32 ? COLS : 32;  // columns per TMEM read batch
#pragma unroll
      for (int c = 0; c < COLS; c += CH) {
        uint32_t v[CH];
#pragma unroll
        for (int h = 0; h < CH; h += 16) tmem_ld16(taddr + b * BN + c + h, *reinterpret_cast<uint32_t(*)[16]>(&v[h]));
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < CH; j += 4) {
          const float4 sa4 = *reinterpret_cast<const float4*>(sag + c + j);
          const float s4[4] = {sa4.x, sa4.y, sa4.z, sa4.w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float f = __uint_as_float(v[j + q]);
            float& t = tot[c + j + q];
            if (fast) {
              t = fmaf(fmaf(f, cw1, cw2), s4[q], t);                        // dot*sw exact, then one rounding
            } else {
              const float d = fmaf(f, 0.0625f, -786432.0f);                 // exact dot
              t = fmaf(d, WG ? __fmul_rn(s4[q], sw) : s4[q], t);
            }
          }
        }
      }
      // hand the accumulator back, re-seeded with the bias bits
#pragma unroll
      for (int c = 0; c < COLS; c += 16) tmem_st16(taddr + b * BN + c, static_cast<uint32_t>(kMagicBits));
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tfree[b]);
    }
    if (ok) {
      const int n = n0 + row;
      const float swc = WG ? 1.0f : bf16_bits_to_f32(sw_s[row]);
      if (n < p.N) {
#pragma unroll
        for (int j = 0; j < COLS; ++j) {
          const int m = m0 + c0 + j;
          if (m < p.M) {
            const float val = WG ? tot[j] : __fmul_rn(tot[j], swc);
            const size_t o = static_cast<size_t>(m) * p.N + n;
            if (F32)
              static_cast<float*>(p.out)[o] = val;
            else
              static_cast<__nv_bfloat16*>(p.out)[o] = __float2bfloat16_rn(val);
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, tc_tmem_cols(BN));
  }
}

// ------------------------------------------------------------ host side
constexpr int kTcSmemLimit = 227 * 1024;

template <int BN, bool WG, bool F32>
static int launch_tc_t(const CUtensorMap* maps, const TcArgs& a, dim3 grid, int smem, cudaStream_t stream) {
  static int done[64] = {};
  auto* kern = &w4a4_tc_kernel<BN, WG, F32>;
  const int rc = ensure_smem_attr(reinterpret_cast<const void*>(kern), smem, done);
  if (rc != NV4_OK) return rc;
  return launch_kernel(kern, grid, dim3(tc_threads(BN)), smem, stream, true, maps[0], maps[1], maps[2], maps[3], a);
}

template <int BN>
static int launch_tc_bn(const CUtensorMap* maps, const TcArgs& a, dim3 grid, int smem, bool wg, bool f32,
                        cudaStream_t s) {
  if (wg) return f32 ? launch_tc_t<BN, true, true>(maps, a, grid, smem, s) : launch_tc_t<BN, true, false>(maps, a, grid, smem, s);
  return f32 ? launch_tc_t<BN, false, true>(maps, a, grid, smem, s) : launch_tc_t<BN, false, false>(maps, a, grid, smem, s);
}

int tc_token_tile(int64_t m) { return m <= 16 ? 16 : (m <= 32 ? 32 : (m <= 64 ? 64 : 128)); }

int launch_w4a4_tc_gemm(const void* a8, const void* w_packed, const void* a_scale, const void* w_scale, void* out,
                        int64_t m, int64_t n, int64_t k, int flags, cudaStream_t stream) {
  const bool wg = (flags & NV4_GEMM_W_SCALE_GROUPED) != 0;
  const bool f32 = (flags & NV4_GEMM_OUT_FP32) != 0;
  const int BN = tc_token_tile(m);
  const int G = static_cast<int>(k / 128);
  const bool scale_tma = (G % 8) == 0 && G <= 256 && (reinterpret_cast<uintptr_t>(a_scale) & 15) == 0 &&
                         (reinterpret_cast<uintptr_t>(w_scale) & 15) == 0;
  const TcLayout one(BN, G, 1, wg);
  int stages = (kTcSmemLimit - 1024 - (one.total - one.stage_bytes) - 3 * 8 * 8) / (one.stage_bytes + 24);
  stages = std::min(stages, std::min(G, BN >= 128 ? 4 : 8));
  if (stages < 2) return NV4_ERR_UNSUPPORTED;
  const TcLayout lay(BN, G, stages, wg);
  const int smem = lay.total + 1024;

  CUtensorMap maps[4];
  memset(maps, 0, sizeof(maps));
  bool okm = make_tensor_map_u8(&maps[0], w_packed, n, k / 2, 128, 64, CU_TENSOR_MAP_SWIZZLE_64B) &&
             make_tensor_map_u8(&maps[1], a8, m, k, static_cast<uint32_t>(BN), 128, CU_TENSOR_MAP_SWIZZLE_128B);
  if (scale_tma) {
    if (wg)
      okm = okm && make_tensor_map_2d(&maps[2], CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, w_scale, n, G, 128, G,
                                      CU_TENSOR_MAP_SWIZZLE_NONE);
    else
      okm = okm && make_tensor_map_2d(&maps[2], CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, w_scale, 1, n, 1, 128,
                                      CU_TENSOR_MAP_SWIZZLE_NONE);
    okm = okm && make_tensor_map_2d(&maps[3], CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, a_scale, m, G,
                                    static_cast<uint32_t>(BN), G, CU_TENSOR_MAP_SWIZZLE_NONE);
  }
  if (!okm) return NV4_ERR_CUDA;
  TcArgs a;
  a.a_scale = static_cast<const uint16_t*>(a_scale);
  a.w_scale = static_cast<const uint16_t*>(w_scale);
  a.out = out;
  a.M = static_cast<int>(m);
  a.N = static_cast<int>(n);
  a.G = G;
  a.stages = stages;
  a.scale_tma = scale_tma ? 1 : 0;
  const dim3 grid(static_cast<unsigned>((n + 127) / 128), static_cast<unsigned>((m + BN - 1) / BN));
  switch (BN) {
    case 16: return launch_tc_bn<16>(maps, a, grid, smem, wg, f32, stream);
    case 32: return launch_tc_bn<32>(maps, a, grid, smem, wg, f32, stream);
    case 64: return launch_tc_bn<64>(maps, a, grid, smem, wg, f32, stream);
    default: return launch_tc_bn<128>(maps, a, grid, smem, wg, f32, stream);
  }
}

}  // namespace nv4
