// Kernel C2: grouped INT4 x INT4 GEMM for decode batches (M <= 32 tokens) on
// 5th-generation tensor cores, with the widened weights as the TMEM operand.
//
// Same semantics as Kernels B and C (nanovllm/kernels/w4a4_grouped_kernel.py:64-90):
// per 128-wide K group g, in increasing g, total = fma(f32(dot_g),
// sa[m,g]*sw[n,g], total); BF16 (or FP32) output; no split-K.
//
// At decode sizes the GEMM streams the weights once and does 2*M MACs per
// weight byte.  The MMAs run on tcgen05 (M = 128 weight rows, N = 8/16/32
// tokens, K = 32 per instruction).  An instruction this narrow costs the
// tensor core about 40-45 cycles whatever N is, and every mbarrier wait or
// tcgen05.commit on the issuing thread costs about as much again, so the work
// is organised in steps of STEP groups: one set of waits and two commits per
// step, and TMEM double-buffered per step.
//
// One CTA owns R weight rows (a multiple of 16, about N / #SMs so that one wave
// covers the layer), held as T = ceil(R / 128) UMMA tiles.  A tile's rows are
// spread evenly over the four TMEM lane quarters (row q*RQ + l of the tile in
// lane 32q + l), so the widen and epilogue warps of all four quarters work
// even when R is small.
//
//   warp 0      TMA producer: per step, the packed weight rows [R x 128 B] for
//               every two groups (128-byte swizzle) and one token tile
//               [NT x 128 B] of INT8 codes per group in the GEMM-ready layout
//               (128-byte swizzle = the K-major UMMA operand layout).  Weights
//               are requested before griddepcontrol.wait, so with programmatic
//               dependent launch they stream while the activation prep runs.
//   warp 1      TMEM allocation and the MMA-issuing thread: per step, group
//               and tile, 4 x tcgen05.mma kind::i8 with A = widened weights in
//               TMEM and B = token tile in smem; one commit tells the widen and
//               epilogue warps that the step's MMAs are done, one frees the stage.
//   warps 4..   widen (4 per tile): thread = weight row; the 64 packed bytes
//               of a group become 128 INT8 values 16*code, each 32-wide K chunk
//               as its 16 even-k then its 16 odd-k codes (the token operand's K
//               order), written with tcgen05.st -- no shared-memory round trip.
//   then        epilogue (4 per tile and token share): tcgen05.ld of a group's
//               INT32 partials (thread = weight row), re-seed the columns with
//               the bias bits of 1.5*2^23 (the MMAs add onto them, so the INT32
//               reads as the float 12582912 + 16*dot), apply the group's scales.
// Fast epilogue (scales of the group within [2^-60, 2^60], always for the
// quantizer's): ds = fma(F, sw/16, -786432*sw) = dot*sw exactly, then
// total = fma(ds, sa, total) = fma(dot, sa*sw, total) because sa*sw is exact
// in FP32; otherwise the reference's three-step form.
//
// Every wait is bounded; on a timeout the roles stop, the MMA thread waits for
// its issued MMAs and the TMEM is freed before the CTA exits.
#include <cstring>

#include "nv4_device.cuh"
#include "nv4_launch.h"

namespace nv4 {

struct TcdArgs {
  const uint16_t* a_scale;  // bf16 [M, G]
  const uint16_t* w_scale;  // bf16 [N, G] (grouped) or [N]
  void* out;                // bf16 or fp32 [M, N]
  int M, N, G;
  int R;          // weight rows per CTA
  int steps;      // ceil(G / STEP)
  int stages;     // TMA ring depth (in steps)
  int scale_tma;  // scales by TMA (row bytes multiple of 16)
};

constexpr int kTcdFirstWiden = 4;  // warps 0-3: producer, MMA, two that only help with set-up
constexpr int kTcdBufs = 2;        // TMEM buffers (widened weights and accumulators) per step

__host__ __device__ constexpr int tcd_threads(int T, int ES) { return 32 * (kTcdFirstWiden + 4 * T + 4 * T * ES); }
__host__ __device__ constexpr int tcd_tmem_needed(int T, int NT, int STEP) {
  return kTcdBufs * STEP * T * (32 + NT);
}
__host__ __device__ constexpr int tcd_tmem_cols(int T, int NT, int STEP) {
  return tcd_tmem_needed(T, NT, STEP) <= 128 ? 128 : (tcd_tmem_needed(T, NT, STEP) <= 256 ? 256 : 512);
}

struct TcdLayout {
  int a_bytes, w_bytes, stage_bytes, sw_off, sa_off, saf_off, flag_off, bar_off, total;
  __host__ __device__ TcdLayout(int R, int NT, int STEP, int G, int S, bool wg) {
    a_bytes = STEP * NT * 128;   // token tiles first: each 1024-byte aligned for the 128-byte swizzle
    w_bytes = (STEP / 2) * R * 128;
    stage_bytes = (a_bytes + w_bytes + 1023) & ~1023;
    sw_off = S * stage_bytes;
    const int sw_bytes = (wg ? R * G : R) * 2;
    sa_off = (sw_off + sw_bytes + 127) & ~127;
    saf_off = (sa_off + NT * G * 2 + 15) & ~15;
    flag_off = saf_off + G * NT * 4;
    bar_off = (flag_off + G * 4 + 7) & ~7;
    // full[S], sfree[S], afull/mdone/dfree[bufs], scale[2], done[1], tmem slot
    total = bar_off + (2 * S + 3 * kTcdBufs + 3) * 8 + 16;
  }
};

template <int C>
__device__ __forceinline__ void tcd_load_cols(uint32_t taddr, uint32_t (&v)[C]) {
  if constexpr (C == 8) {
    tmem_ld8(taddr, v);
  } else {
#pragma unroll
    for (int c = 0; c < C; c += 16) tmem_ld16(taddr + c, *reinterpret_cast<uint32_t(*)[16]>(&v[c]));
  }
}

template <int C>
__device__ __forceinline__ void tcd_seed_cols(uint32_t taddr) {
  if constexpr (C == 8) {
    tmem_st8(taddr, static_cast<uint32_t>(kMagicBits));
  } else {
#pragma unroll
    for (int c = 0; c < C; c += 16) tmem_st16(taddr + c, static_cast<uint32_t>(kMagicBits));
  }
}

// NT: token tile (8/16/32); T: UMMA tiles per CTA; STEP: groups per step (2 or 4);
// ES: epilogue warps per lane quarter and tile (token shares).
template <int NT, int T, int STEP, int ES, bool WG, bool F32>
__global__ void __launch_bounds__(tcd_threads(T, ES), 1)
    w4a4_tcd_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_a,
                    const __grid_constant__ CUtensorMap tmap_sw, const __grid_constant__ CUtensorMap tmap_sa,
                    const TcdArgs p) {
  constexpr int NB = kTcdBufs;
  constexpr uint32_t IDESC = umma_idesc_s8(128, NT);
  constexpr int DCOLS = NB * STEP * T * NT;  // accumulators first, widened weights after them
  constexpr int WW = 4 * T;                  // widen warps
  constexpr int EW = 4 * T * ES;             // epilogue warps
  constexpr int CT = NT / ES;                // token columns per epilogue thread
  extern __shared__ uint8_t smem_raw[];
  const int S = p.stages, G = p.G, R = p.R, NS = p.steps;
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  const TcdLayout L(R, NT, STEP, G, S, WG);
  uint16_t* sw_s = reinterpret_cast<uint16_t*>(smem + L.sw_off);  // [R][G] (or [R])
  uint16_t* sa_s = reinterpret_cast<uint16_t*>(smem + L.sa_off);  // [NT][G]
  float* saf = reinterpret_cast<float*>(smem + L.saf_off);         // [G][NT]
  int* fast_g = reinterpret_cast<int*>(smem + L.flag_off);         // [G]
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bar_off);
  uint64_t* sfree = full + S;
  uint64_t* afull = sfree + S;   // widened weights of the step written
  uint64_t* mdone = afull + NB;  // MMAs of the step complete (accumulators full, widened buffer free)
  uint64_t* dfree = mdone + NB;  // accumulators read and re-seeded
  uint64_t* scale_bar = dfree + NB;
  uint64_t* done_bar = scale_bar + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done_bar + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * R, m0 = blockIdx.y * NT;
  grid_dependents_launch();

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&sfree[s], WW + 1);
    }
    for (int i = 0; i < NB; ++i) {
      mbar_init(&afull[i], WW);
      mbar_init(&mdone[i], 1);
      mbar_init(&dfree[i], EW);
    }
    mbar_init(&scale_bar[0], 1);
    mbar_init(&scale_bar[1], 1);
    mbar_init(done_bar, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, tcd_tmem_cols(T, NT, STEP));
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
        mbar_arrive_expect_tx(&scale_bar[0], static_cast<uint32_t>((WG ? R * G : R) * 2));
        if (WG)
          tma_load_2d(sw_s, &tmap_sw, &scale_bar[0], 0, n0);
        else
          tma_load_2d(sw_s, &tmap_sw, &scale_bar[0], n0, 0);
      }
      auto groups_in = [&](int st) { return min(STEP, G - st * STEP); };
      auto load_w = [&](int st) {
        const int s = st % S, gs = groups_in(st);
        mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(((gs + 1) / 2) * R * 128 + gs * NT * 128));
        for (int j = 0; j < gs; j += 2)
          tma_load_2d_hint(smem + s * L.stage_bytes + L.a_bytes + (j / 2) * R * 128, &tmap_w, &full[s],
                           (st * STEP + j) * 64, n0, wpol);
      };
      auto load_a = [&](int st) {
        const int s = st % S, gs = groups_in(st);
        for (int j = 0; j < gs; ++j)
          tma_load_2d(smem + s * L.stage_bytes + j * NT * 128, &tmap_a, &full[s], (st * STEP + j) * 128, m0);
      };
      const int first = min(S, NS);
      for (int st = 0; st < first; ++st) load_w(st);
      grid_dependency_wait();  // the token codes and scales come from the preceding kernel
      if (p.scale_tma) {
        mbar_arrive_expect_tx(&scale_bar[1], static_cast<uint32_t>(NT * G * 2));
        tma_load_2d(sa_s, &tmap_sa, &scale_bar[1], 0, m0);
      }
      for (int st = 0; st < first; ++st) load_a(st);
      int issued = first;
      for (int st = first; st < NS; ++st) {
        if (!mbar_wait(&sfree[st % S], ((st / S) - 1) & 1, kErrTimeoutEmpty)) break;
        load_w(st);
        load_a(st);
        issued = st + 1;
      }
      // Before the CTA may exit, every copy issued must have landed.
      for (int st = max(0, issued - S); st < issued; ++st)
        if (!mbar_wait(&full[st % S], (st / S) & 1, kErrTimeoutDrain)) break;
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer
    if (lane == 0) {
      const uint32_t stage_base = smem_u32(smem);
      for (int st = 0; st < NS; ++st) {
        const int s = st % S, b = st % NB, gs = min(STEP, G - st * STEP);
        const uint32_t ph = (st / NB) & 1;
        ok = mbar_wait(&afull[b], ph, kErrTimeoutMma) && mbar_wait(&full[s], (st / S) & 1, kErrTimeoutMma) &&
             mbar_wait(&dfree[b], ph, kErrTimeoutMma);
        if (!ok) break;
        tc_fence_after();
        const uint32_t a_tiles = stage_base + s * L.stage_bytes;
#pragma unroll
        for (int j = 0; j < STEP; ++j) {
          if (j < gs) {
#pragma unroll
            for (int t = 0; t < T; ++t) {
              const uint32_t d_col = tmem + ((b * STEP + j) * T + t) * NT;
              const uint32_t a_col = tmem + DCOLS + ((b * STEP + j) * T + t) * 32;
              const uint32_t b_tile = a_tiles + j * NT * 128;
#pragma unroll
              for (int k = 0; k < 4; ++k)
                umma_s8_ts(d_col, a_col + k * 8, umma_desc_sw128(b_tile + k * 32), IDESC, 1);
            }
          }
        }
        umma_commit(&mdone[b]);
        umma_commit(&sfree[s]);
      }
      // all issued MMAs must finish before the TMEM is released
      umma_commit(done_bar);
      mbar_wait(done_bar, 0, kErrTimeoutDrain);
    }
  } else if (warp < kTcdFirstWiden) {
    // helpers: nothing in the main loop
  } else if (warp < kTcdFirstWiden + WW) {
    // ---------------- widen: thread = weight row of its tile's lane quarter
    const int t = (warp - kTcdFirstWiden) >> 2, q = warp & 3;
    const int rq = (min(128, R - 128 * t)) >> 2;  // rows per lane quarter of this tile
    const bool valid = lane < rq;
    const int r = 128 * t + q * rq + lane;       // CTA row (when valid)
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(q * 32) << 16) + DCOLS + t * 32;
    for (int st = 0; st < NS; ++st) {
      const int s = st % S, b = st % NB, gs = min(STEP, G - st * STEP);
      ok = mbar_wait(&full[s], (st / S) & 1, kErrTimeoutFull);
      if (ok && st >= NB) ok = mbar_wait(&mdone[b], ((st / NB) - 1) & 1, kErrTimeoutFull);
      if (!ok) break;
      const uint8_t* wrow = smem + s * L.stage_bytes + L.a_bytes + r * 128;
#pragma unroll
      for (int j = 0; j < STEP; ++j) {
        if (j < gs) {
          uint4 pk[4];
#pragma unroll
          for (int c = 0; c < 4; ++c) pk[c] = make_uint4(0u, 0u, 0u, 0u);
          if (valid) {
            const uint8_t* src = wrow + (j / 2) * R * 128;
#pragma unroll
            for (int c = 0; c < 4; ++c)
              pk[c] = *reinterpret_cast<const uint4*>(src + (((((j & 1) * 4) + c) ^ (r & 7)) << 4));
          }
          uint32_t w[32];
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            w[8 * c + 0] = nib_even16(pk[c].x);
            w[8 * c + 1] = nib_even16(pk[c].y);
            w[8 * c + 2] = nib_even16(pk[c].z);
            w[8 * c + 3] = nib_even16(pk[c].w);
            w[8 * c + 4] = nib_odd16(pk[c].x);
            w[8 * c + 5] = nib_odd16(pk[c].y);
            w[8 * c + 6] = nib_odd16(pk[c].z);
            w[8 * c + 7] = nib_odd16(pk[c].w);
          }
          tmem_st32(lane_base + (b * STEP + j) * T * 32, w);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sfree[s]);  // packed weights read
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&afull[b]);
    }
  } else {
    // ---------------- epilogue: thread = weight row (TMEM lane), CT token columns
    const int ew = warp - kTcdFirstWiden - WW;
    const int t = (ew >> 2) % T, e = (ew >> 2) / T, q = warp & 3;
    const int rq = (min(128, R - 128 * t)) >> 2;
    const bool valid = lane < rq;
    const int r = valid ? 128 * t + q * rq + lane : 0;
    const int c0 = e * CT;  // first token column
    const int et = ew * 32 + lane, ethreads = EW * 32;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(q * 32) << 16) + t * NT + c0;
    // seed every accumulator this thread owns with the bias bits
#pragma unroll
    for (int b = 0; b < NB; ++b)
#pragma unroll
      for (int j = 0; j < STEP; ++j) tcd_seed_cols<CT>(lane_base + (b * STEP + j) * T * NT);
    tmem_wait_st();
    tc_fence_before();
    __syncwarp();
    if (lane == 0)
      for (int b = 0; b < NB; ++b) mbar_arrive(&dfree[b]);
    // scales
    if (!p.scale_tma) {
      const int nsw = WG ? R * G : R;
      for (int i = et; i < nsw; i += ethreads) {
        const int rr = WG ? i / G : i;
        sw_s[i] = (n0 + rr < p.N) ? p.w_scale[static_cast<size_t>(n0) * (WG ? G : 1) + i] : uint16_t(0);
      }
    } else {
      ok = mbar_wait(&scale_bar[0], 0, kErrTimeoutFull);
    }
    for (int g = et; g < G; g += ethreads) fast_g[g] = 1;
    grid_dependency_wait();
    if (!p.scale_tma) {
      for (int i = et; i < NT * G; i += ethreads)
        sa_s[i] = (m0 + i / G < p.M) ? p.a_scale[static_cast<size_t>(m0) * G + i] : uint16_t(0);
    } else {
      ok = mbar_wait(&scale_bar[1], 0, kErrTimeoutFull) && ok;
    }
    named_barrier_sync(1, ethreads);
    for (int i = et; i < NT * G; i += ethreads) {
      const int j = i / G, g = i - j * G;
      const float sa = bf16_bits_to_f32(sa_s[i]);
      saf[g * NT + j] = sa;
      if (!tc_fast_scale(sa)) fast_g[g] = 0;
    }
    if (WG)
      for (int i = et; i < R * G; i += ethreads)
        if (!tc_fast_scale(bf16_bits_to_f32(sw_s[i]))) fast_g[i % G] = 0;
    named_barrier_sync(1, ethreads);

    float tot[CT];
#pragma unroll
    for (int j = 0; j < CT; ++j) tot[j] = 0.0f;
    for (int st = 0; st < NS && ok; ++st) {
      const int b = st % NB, gs = min(STEP, G - st * STEP);
      if (!mbar_wait(&mdone[b], (st / NB) & 1, kErrTimeoutMma)) {
        ok = false;
        break;
      }
      tc_fence_after();
      // All of the step's columns in one batch of loads behind one wait, then
      // hand them back re-seeded before the FMAs so the next MMAs can start.
      uint32_t v[STEP][CT];
#pragma unroll
      for (int jj = 0; jj < STEP; ++jj)
        if (jj < gs) tcd_load_cols<CT>(lane_base + (b * STEP + jj) * T * NT, v[jj]);
      tmem_wait_ld();
#pragma unroll
      for (int jj = 0; jj < STEP; ++jj)
        if (jj < gs) tcd_seed_cols<CT>(lane_base + (b * STEP + jj) * T * NT);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&dfree[b]);
#pragma unroll
      for (int jj = 0; jj < STEP; ++jj) {
        if (jj < gs) {
          const int g = st * STEP + jj;
          const float sw = WG ? bf16_bits_to_f32(sw_s[r * G + g]) : 1.0f;
          const float* sag = saf + g * NT + c0;
          const bool fast = WG && fast_g[g] != 0;
          const float cw1 = __fmul_rn(sw, 0.0625f), cw2 = __fmul_rn(sw, -786432.0f);
#pragma unroll
          for (int j = 0; j < CT; j += 4) {
            const float4 sa4 = *reinterpret_cast<const float4*>(sag + j);
            const float s4[4] = {sa4.x, sa4.y, sa4.z, sa4.w};
#pragma unroll
            for (int x = 0; x < 4; ++x) {
              const float f = __uint_as_float(v[jj][j + x]);
              if (fast) {
                tot[j + x] = fmaf(fmaf(f, cw1, cw2), s4[x], tot[j + x]);  // dot*sw exact, then one rounding
              } else {
                const float d = fmaf(f, 0.0625f, -786432.0f);               // exact dot
                tot[j + x] = fmaf(d, WG ? __fmul_rn(s4[x], sw) : s4[x], tot[j + x]);
              }
            }
          }
        }
      }
    }
    if (ok && valid) {
      const int n = n0 + r;
      const float swc = WG ? 1.0f : bf16_bits_to_f32(sw_s[r]);
      if (n < p.N) {
#pragma unroll
        for (int j = 0; j < CT; ++j) {
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
    tmem_dealloc(tmem, tcd_tmem_cols(T, NT, STEP));
  }
}

// ------------------------------------------------------------ host side
template <int NT, int T, int STEP, int ES, bool WG, bool F32>
static int launch_tcd_t(const CUtensorMap* maps, const TcdArgs& a, dim3 grid, int smem, cudaStream_t stream) {
  static int done[64] = {};
  auto* kern = &w4a4_tcd_kernel<NT, T, STEP, ES, WG, F32>;
  const int rc = ensure_smem_attr(reinterpret_cast<const void*>(kern), smem, done);
  if (rc != NV4_OK) return rc;
  return launch_kernel(kern, grid, dim3(tcd_threads(T, ES)), smem, stream, true, maps[0], maps[1], maps[2], maps[3],
                       a);
}

template <int NT, int T, int STEP, int ES>
static int launch_tcd_flags(const CUtensorMap* maps, const TcdArgs& a, dim3 grid, int smem, bool wg, bool f32,
                            cudaStream_t s) {
  if (wg) return f32 ? launch_tcd_t<NT, T, STEP, ES, true, true>(maps, a, grid, smem, s)
                     : launch_tcd_t<NT, T, STEP, ES, true, false>(maps, a, grid, smem, s);
  return f32 ? launch_tcd_t<NT, T, STEP, ES, false, true>(maps, a, grid, smem, s)
             : launch_tcd_t<NT, T, STEP, ES, false, false>(maps, a, grid, smem, s);
}

int launch_w4a4_tcd_gemm(const void* a8, const void* w_packed, const void* a_scale, const void* w_scale, void* out,
                         int64_t m, int64_t n, int64_t k, int flags, cudaStream_t stream) {
  if (m < 1 || m > 32) return NV4_ERR_UNSUPPORTED;  // token tiles of 8, 16 or 32
  const int sms = device_sm_count();
  if (sms <= 0) return NV4_ERR_CUDA;
  const bool wg = (flags & NV4_GEMM_W_SCALE_GROUPED) != 0;
  const bool f32 = (flags & NV4_GEMM_OUT_FP32) != 0;
  const int NT = m <= 8 ? 8 : (m <= 16 ? 16 : 32);
  const int G = static_cast<int>(k / 128);
  // About one CTA per SM: rows per CTA a multiple of 16, at most two UMMA tiles.
  const int64_t per = (n + sms - 1) / sms;
  const int R = static_cast<int>(std::min<int64_t>(256, std::max<int64_t>(16, (per + 15) / 16 * 16)));
  const int T = R > 128 ? 2 : 1;
  // Steps of 4 groups for one tile, 2 for two (TMEM holds two steps of
  // widened weights and accumulators); the kernel variants below use two
  // epilogue warps per lane quarter (token halves) from 16 tokens up.
  const int STEP = T == 1 ? 4 : 2;
  const bool scale_tma = (G % 8) == 0 && G <= 256 && (reinterpret_cast<uintptr_t>(a_scale) & 15) == 0 &&
                         (reinterpret_cast<uintptr_t>(w_scale) & 15) == 0;
  const int steps = (G + STEP - 1) / STEP;
  const TcdLayout one(R, NT, STEP, G, 1, wg);
  int stages = (227 * 1024 - 1024 - (one.total - one.stage_bytes) - 64) / (one.stage_bytes + 16);
  stages = std::min(stages, std::min(steps, 8));
  if (stages < 2 && steps > 1) return NV4_ERR_UNSUPPORTED;
  stages = std::max(stages, 1);
  const TcdLayout lay(R, NT, STEP, G, stages, wg);
  const int smem = lay.total + 1024;

  CUtensorMap maps[4];
  memset(maps, 0, sizeof(maps));
  bool okm = make_tensor_map_u8(&maps[0], w_packed, n, k / 2, static_cast<uint32_t>(R), 128, CU_TENSOR_MAP_SWIZZLE_128B) &&
             make_tensor_map_u8(&maps[1], a8, m, k, static_cast<uint32_t>(NT), 128, CU_TENSOR_MAP_SWIZZLE_128B);
  if (scale_tma) {
    if (wg)
      okm = okm && make_tensor_map_2d(&maps[2], CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, w_scale, n, G,
                                      static_cast<uint32_t>(R), G, CU_TENSOR_MAP_SWIZZLE_NONE);
    else
      okm = okm && make_tensor_map_2d(&maps[2], CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, w_scale, 1, n, 1,
                                      static_cast<uint32_t>(R), CU_TENSOR_MAP_SWIZZLE_NONE);
    okm = okm && make_tensor_map_2d(&maps[3], CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, a_scale, m, G,
                                    static_cast<uint32_t>(NT), G, CU_TENSOR_MAP_SWIZZLE_NONE);
  }
  if (!okm) return NV4_ERR_CUDA;
  TcdArgs a;
  a.a_scale = static_cast<const uint16_t*>(a_scale);
  a.w_scale = static_cast<const uint16_t*>(w_scale);
  a.out = out;
  a.M = static_cast<int>(m);
  a.N = static_cast<int>(n);
  a.G = G;
  a.R = R;
  a.steps = steps;
  a.stages = stages;
  a.scale_tma = scale_tma ? 1 : 0;
  const dim3 grid(static_cast<unsigned>((n + R - 1) / R), 1);
  switch (NT * 10 + T) {
    case 81: return launch_tcd_flags<8, 1, 4, 1>(maps, a, grid, smem, wg, f32, stream);
    case 82: return launch_tcd_flags<8, 2, 2, 1>(maps, a, grid, smem, wg, f32, stream);
    case 161: return launch_tcd_flags<16, 1, 4, 2>(maps, a, grid, smem, wg, f32, stream);
    case 162: return launch_tcd_flags<16, 2, 2, 2>(maps, a, grid, smem, wg, f32, stream);
    case 321: return launch_tcd_flags<32, 1, 4, 2>(maps, a, grid, smem, wg, f32, stream);
    default: return launch_tcd_flags<32, 2, 2, 2>(maps, a, grid, smem, wg, f32, stream);
  }
}

}  // namespace nv4
