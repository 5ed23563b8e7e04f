// Kernel D2: GPTQ W4A16 dequant GEMM on 5th-generation tensor cores (tcgen05
// kind::f16), for more than 16 tokens.
//
// out[m, n] = sum_k x[m, k] * Wdq[k, n] with the reference's dequantisation
// (nanovllm/layers/linear_w4a16.py:45-55): Wdq = bf16((w - z - 1) * bf16(scale)),
// computed as bf16(128 + w) - bf16(129 + z) (exact) times the BF16-rounded FP16
// scale (one BF16 rounding).  FP32 accumulation in tensor memory.  When the
// tiles do not fill the SMs (few weight-column blocks, up to a few hundred
// tokens), K is split into up to 8 slices: each slice's FP32 partial tile goes
// to a workspace and a second kernel adds the slices in slice order (fixed
// order, deterministic) and rounds to BF16 once; otherwise one BF16 rounding of
// the full-K accumulator.  (The reference adds BF16-rounded split-K partials
// with BF16 atomics, so results agree within a tolerance.)
//
// The MMA computes D[n, t] = A[n, k] * B[t, k]^T with
//   A = dequantised weights: M = 128 weight columns n, held in tensor memory
//       (column n in TMEM lane n, two BF16 k per 32-bit column, K-major), so
//       the widened weights never touch shared memory;
//   B = activations: N = BN tokens, BF16 K-major with the 128-byte swizzle,
//       exactly as TMA lands them.
// Persistent: one CTA per SM walks work units -- a tile of 128 weight columns x
// BN tokens over one K slice -- 64 K per pipeline chunk:
//   warp 0      TMA producer: per chunk, the x tile [BN x 64 k], the packed
//               weight tile [8 rows of k/8 x 128 columns] and the chunk's group
//               row of scales [128] and zero points [16 words] into an S-slot
//               ring (no global loads on the dequantisation path).
//   warp 1      TMEM allocation (all 512 columns) and the single MMA-issuing
//               thread: 4 x tcgen05.mma kind::f16 (K = 16) per chunk.
//   warps 2-9   dequantisation, two warps per TMEM lane quarter taking
//               alternate chunks: thread = weight column; 8 packed words -> 32
//               BF16 pairs -> tcgen05.st into the chunk's A buffer.  (The
//               dequantisation is the kernel's busiest ALU work; two warps per
//               sub-partition keep it ahead of the tensor core.)
//   warps 10-25 epilogue, four per lane quarter (BN/4 tokens each, 32 at a
//               time): tcgen05.ld, round to BF16, store out[t, n], then hand the
//               accumulator back.
// TMEM columns: accumulators [0, 256) (one of 256 tokens or two of 128), A
// buffers [256, 512) (32 columns per chunk, up to 8).
//
// Every wait is bounded; on a timeout the roles stop, the MMA thread waits for
// its issued MMAs and the TMEM is freed before the CTA exits.
#include <cstring>

#include "nv4_device.cuh"
#include "nv4_launch.h"

namespace nv4 {

constexpr int kD2Chunk = 64;          // K per pipeline chunk

struct W4A16TcArgs {
  uint16_t* out;           // bf16 [M, N] (one K slice)
  float* partial;          // fp32 [splits, M, N] (more than one K slice)
  int M, N, K;
  int tiles_m, splits;     // token blocks; K slices
  int units;               // column blocks x splits x token blocks (token blocks fastest, then slices)
};

// One work unit: column block, token block, K slice and its chunk range
// [cb, ce) (slices differ by at most one chunk).
struct D2Unit {
  int nb, mb, split, cb, ce;
};

__device__ __forceinline__ D2Unit d2_unit(const W4A16TcArgs& p, int t) {
  D2Unit u;
  u.mb = t % p.tiles_m;
  const int r = t / p.tiles_m;
  u.split = r % p.splits;
  u.nb = r / p.splits;
  const int kct = p.K / kD2Chunk;
  u.cb = (u.split * kct) / p.splits;
  u.ce = ((u.split + 1) * kct) / p.splits;
  return u;
}

constexpr int kD2DequantWarps = 8;    // two per TMEM lane quarter (alternate chunks)
constexpr int kD2EpiWarps = 16;       // four per lane quarter
constexpr int kD2FirstEpiWarp = 2 + kD2DequantWarps;
constexpr int kD2Threads = 32 * (kD2FirstEpiWarp + kD2EpiWarps);
constexpr uint32_t kD2ACol = 256;     // first TMEM column of the A buffers

template <int BN>
struct D2Layout {
  static constexpr int kStages = BN == 256 ? 5 : 8;  // at most 8 A buffers of 32 columns
  static constexpr int kX = BN * 128;                 // x tile: BN rows of 64 BF16
  static constexpr int kW = 8 * 128 * 4;              // packed weights: 8 rows of 128 int32
  static constexpr int kS = 128 * 2;                  // the group's scales of the 128 columns (fp16)
  static constexpr int kZ = 16 * 4;                   // the group's zero-point words of the 128 columns
  static constexpr int kBytes = kX + kW + kS + kZ;    // TMA bytes per stage
  static constexpr int kStage = (kBytes + 1023) & ~1023;  // a multiple of 1024 (SW128 atoms)
  static constexpr int kAcc = 256 / BN;               // accumulators
  static constexpr int kBar = kStages * kStage;
  // full[S], afull[S], consumed[S], tfull[A], tfree[A], done, tmem slot
  static constexpr int kTotal = kBar + (3 * kStages + 2 * kAcc + 1) * 8 + 16;
};

// Instruction descriptor of tcgen05.mma kind::f16: BF16 A and B, both K-major,
// FP32 accumulator, M x N.
__host__ __device__ constexpr uint32_t umma_idesc_bf16(int m, int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(m >> 4) << 24);
}

// D[tmem] (+)= A[tmem] * B[smem]^T, BF16 operands, A in tensor memory.
__device__ __forceinline__ void umma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.u32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 32 lanes x 32 columns of 32-bit TMEM -> 32 registers per thread.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// The packed word w holds k0..k7 of one column (k_i in nibble i).  Returns the
// BF16 pairs (k0, k1), (k2, k3), (k4, k5), (k6, k7) of bf16(128 + nibble): the
// nibble fills the low mantissa bits of bf16(128) = 0x4300.
__device__ __forceinline__ void nib_pairs_128(uint32_t w, uint32_t (&p)[4]) {
  p[0] = (w & 0x0000000Fu) | ((w << 12) & 0x000F0000u) | 0x43004300u;
  p[1] = ((w >> 8) & 0x0000000Fu) | ((w << 4) & 0x000F0000u) | 0x43004300u;
  p[2] = ((w >> 16) & 0x0000000Fu) | ((w >> 4) & 0x000F0000u) | 0x43004300u;
  p[3] = ((w >> 24) & 0x0000000Fu) | ((w >> 12) & 0x000F0000u) | 0x43004300u;
}

__device__ __forceinline__ uint32_t bf16x2_sub_u(uint32_t a, uint32_t b) {
  __nv_bfloat162 r = __hsub2(*reinterpret_cast<__nv_bfloat162*>(&a), *reinterpret_cast<__nv_bfloat162*>(&b));
  return *reinterpret_cast<uint32_t*>(&r);
}

__device__ __forceinline__ uint32_t bf16x2_mul_u(uint32_t a, uint32_t b) {
  __nv_bfloat162 r = __hmul2(*reinterpret_cast<__nv_bfloat162*>(&a), *reinterpret_cast<__nv_bfloat162*>(&b));
  return *reinterpret_cast<uint32_t*>(&r);
}

// Bounded wait used on the way out (also after an error was recorded).
__device__ __forceinline__ bool mbar_wait_drain_d2(uint64_t* bar, uint32_t parity) {
  const uint64_t start = global_timer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_timer_ns() - start > kWaitLimitNs) {
      record_error(kErrTimeoutDrain);
      return false;
    }
  }
  return true;
}

// (129 + z) and the BF16-rounded scale of column `col` of the tile, each as a
// BF16 pair, from the stage's scale row and zero-point words.
__device__ __forceinline__ void d2_zero_scale(const uint8_t* stage_zs, int col, uint32_t& cz, uint32_t& s2) {
  const uint16_t* sc = reinterpret_cast<const uint16_t*>(stage_zs);
  const uint32_t* zw = reinterpret_cast<const uint32_t*>(stage_zs + 256);
  const uint32_t z = (zw[col >> 3] >> (4 * (col & 7))) & 15u;
  const uint32_t czb = __bfloat16_as_ushort(__float2bfloat16_rn(static_cast<float>(129u + z)));
  cz = czb | (czb << 16);
  const uint32_t sb = __bfloat16_as_ushort(__float2bfloat16_rn(__half2float(__ushort_as_half(sc[col]))));
  s2 = sb | (sb << 16);
}

template <int BN>
__global__ void __launch_bounds__(kD2Threads, 1)
    w4a16_tc_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_qw,
                    const __grid_constant__ CUtensorMap tmap_sc, const __grid_constant__ CUtensorMap tmap_qz,
                    const W4A16TcArgs p) {
  using L = D2Layout<BN>;
  constexpr int S = L::kStages, NA = L::kAcc;
  constexpr uint32_t IDESC = umma_idesc_bf16(128, BN);
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBar);
  uint64_t* afull = full + S;
  uint64_t* consumed = afull + S;
  uint64_t* tfull = consumed + S;
  uint64_t* tfree = tfull + NA;
  uint64_t* done_bar = tfree + NA;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done_bar + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int my_units = p.units > static_cast<int>(blockIdx.x)
                           ? (p.units - static_cast<int>(blockIdx.x) + gridDim.x - 1) / gridDim.x : 0;
  auto unit_of = [&](int i) { return d2_unit(p, static_cast<int>(blockIdx.x) + i * static_cast<int>(gridDim.x)); };
  int total = 0;  // pipeline chunks of this CTA (every unit has at least one)
  for (int i = 0; i < my_units; ++i) {
    const D2Unit u = unit_of(i);
    total += u.ce - u.cb;
  }
  grid_dependents_launch();

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&afull[s], kD2DequantWarps / 2);  // the four warps of the chunk's parity
      mbar_init(&consumed[s], 1);
    }
    for (int i = 0; i < NA; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tfree[i], kD2EpiWarps);
    }
    mbar_init(done_bar, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
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
      tma_prefetch_desc(&tmap_x);
      tma_prefetch_desc(&tmap_qw);
      tma_prefetch_desc(&tmap_sc);
      tma_prefetch_desc(&tmap_qz);
      const uint64_t wpol = policy_evict_first();
      // (unit, chunk) walk over this CTA's units in order
      struct Walk {
        D2Unit u;
        int i, kc;
      };
      auto walk_start = [&]() { Walk w{unit_of(0), 0, 0}; w.kc = w.u.cb; return w; };
      auto walk_step = [&](Walk& w) {
        if (++w.kc == w.u.ce && ++w.i < my_units) {
          w.u = unit_of(w.i);
          w.kc = w.u.cb;
        }
      };
      auto load_w = [&](int c, const Walk& w) {  // first of a slot's copies: expects all of them
        const int s = c % S, n0 = w.u.nb * 128;
        uint8_t* st = smem + s * L::kStage;
        mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(L::kBytes));
        tma_load_2d_hint(st + L::kX, &tmap_qw, &full[s], n0, w.kc * 8, wpol);
        tma_load_2d(st + L::kX + L::kW, &tmap_sc, &full[s], n0, (w.kc * kD2Chunk) / 128);
        tma_load_2d(st + L::kX + L::kW + L::kS, &tmap_qz, &full[s], n0 / 8, (w.kc * kD2Chunk) / 128);
      };
      auto load_x = [&](int c, const Walk& w) {
        tma_load_2d(smem + (c % S) * L::kStage, &tmap_x, &full[c % S], w.kc * kD2Chunk, w.u.mb * BN);
      };
      // the first chunks' weights stream while the preceding kernel finishes
      const int first = min(S, total);
      Walk wk = walk_start();
      for (int c = 0; c < first; ++c, walk_step(wk)) load_w(c, wk);
      grid_dependency_wait();  // the activations come from the preceding kernel
      Walk wx = walk_start();
      for (int c = 0; c < first; ++c, walk_step(wx)) load_x(c, wx);
      int issued = first;
      for (int c = first; c < total; ++c, walk_step(wk)) {
        const int s = c % S;
        if (!mbar_wait(&consumed[s], ((c / S) - 1) & 1, kErrTimeoutEmpty)) break;
        load_w(c, wk);
        load_x(c, wk);
        issued = c + 1;
      }
      // every copy issued must land before the CTA may exit
      for (int c = max(0, issued - S); c < issued; ++c)
        if (!mbar_wait_drain_d2(&full[c % S], (c / S) & 1)) break;
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer: 4 x (M=128 columns, N=BN tokens, K=16) per chunk
    if (lane == 0) {
      const uint32_t stage_base = smem_u32(smem);
      int c = 0;
      for (int ui = 0; ui < my_units && ok; ++ui) {
        const D2Unit u = unit_of(ui);
        const int b = ui % NA;
        for (int kc = u.cb; kc < u.ce; ++kc, ++c) {
          const int s = c % S;
          if (kc == u.cb) ok = mbar_wait(&tfree[b], (ui / NA) & 1, kErrTimeoutMma);
          // afull[s] implies full[s]: the dequant warps waited for both copies
          ok = ok && mbar_wait(&afull[s], (c / S) & 1, kErrTimeoutMma);
          if (!ok) break;
          tc_fence_after();
          const uint32_t x_addr = stage_base + s * L::kStage;
          const uint32_t a_tmem = tmem + kD2ACol + 32u * s;
#pragma unroll
          for (int j = 0; j < 4; ++j)
            umma_bf16_ts(tmem + b * BN, a_tmem + 8u * j, umma_desc_sw128(x_addr + 32 * j), IDESC,
                         (kc > u.cb || j > 0) ? 1u : 0u);
          umma_commit(&consumed[s]);
          if (kc == u.ce - 1) umma_commit(&tfull[b]);
        }
      }
      // all issued MMAs must finish before the TMEM is released
      umma_commit(done_bar);
      mbar_wait(done_bar, 0, kErrTimeoutDrain);
    }
  } else if (warp < kD2FirstEpiWarp) {
    // ---------------- dequantisation: thread = weight column (its TMEM lane);
    // the two warps of a lane quarter take alternate chunks
    const int quarter = warp & 3;
    const int parity = (warp - 2) >> 2;
    const int col = quarter * 32 + lane;
    const uint32_t a_lane = tmem + (static_cast<uint32_t>(quarter * 32) << 16) + kD2ACol;
    for (int c = parity; c < total && ok; c += 2) {
      const int s = c % S;
      ok = __all_sync(0xffffffffu, mbar_wait(&full[s], (c / S) & 1, kErrTimeoutFull));
      if (!ok) break;
      const uint8_t* st = smem + s * L::kStage;
      const uint32_t* wq = reinterpret_cast<const uint32_t*>(st + L::kX);
      uint32_t cz, s2;
      d2_zero_scale(st + L::kX + L::kW, col, cz, s2);
      uint32_t w[8];
#pragma unroll
      for (int r = 0; r < 8; ++r) w[r] = wq[r * 128 + col];
      uint32_t v[32];
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        uint32_t pr[4];
        nib_pairs_128(w[r], pr);
#pragma unroll
        for (int j = 0; j < 4; ++j) v[r * 4 + j] = bf16x2_mul_u(bf16x2_sub_u(pr[j], cz), s2);
      }
      tmem_st32(a_lane + 32u * s, v);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&afull[s]);
    }
  } else {
    // ---------------- epilogue: thread = weight column, BN/4 token columns;
    // BF16 out (one K slice) or the slice's FP32 partial
    constexpr int kCols = BN / 4;
    const int ew = warp - kD2FirstEpiWarp;
    const int quarter = warp & 3;
    const int c0 = (ew >> 2) * kCols;
    const uint32_t taddr = tmem + (static_cast<uint32_t>(quarter * 32) << 16) + c0;
    __syncwarp();
    if (lane == 0)
      for (int b = 0; b < NA; ++b) mbar_arrive(&tfree[b]);  // every accumulator starts free
    for (int ui = 0; ui < my_units && ok; ++ui) {
      const int b = ui % NA;
      ok = mbar_wait(&tfull[b], (ui / NA) & 1, kErrTimeoutMma);
      if (!ok) break;
      tc_fence_after();
      const D2Unit u = unit_of(ui);
      const int n = u.nb * 128 + quarter * 32 + lane;
      const int m0 = u.mb * BN + c0;
      float* part = p.partial + static_cast<size_t>(u.split) * p.M * p.N;
#pragma unroll
      for (int c = 0; c < kCols; c += 32) {
        uint32_t v[32];
        tmem_ld32(taddr + b * BN + c, v);
        tmem_wait_ld();
        if (n < p.N) {
          if (p.splits == 1) {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const int m = m0 + c + j;
              if (m < p.M)
                p.out[static_cast<size_t>(m) * p.N + n] =
                    __bfloat16_as_ushort(__float2bfloat16_rn(__uint_as_float(v[j])));
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const int m = m0 + c + j;
              if (m < p.M) part[static_cast<size_t>(m) * p.N + n] = __uint_as_float(v[j]);
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tfree[b]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Split-K sum: out = bf16(partial[0] + partial[1] + ...), slices added in
// order, four outputs per thread.
constexpr int kD2MaxSplits = 8;

__global__ void __launch_bounds__(256) w4a16_split_sum_kernel(const float* __restrict__ partial,
                                                              uint16_t* __restrict__ out, int64_t count4,
                                                              int64_t slice4, int splits) {
  grid_dependency_wait();  // the partials come from the preceding GEMM
  grid_dependents_launch();
  const float4* src = reinterpret_cast<const float4*>(partial);
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count4;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float4 v[kD2MaxSplits];
#pragma unroll
    for (int s = 0; s < kD2MaxSplits; ++s)  // every load before the sum
      if (s < splits) v[s] = __ldcs(src + s * slice4 + i);
    float4 a = v[0];
#pragma unroll
    for (int s = 1; s < kD2MaxSplits; ++s)
      if (s < splits) {
        a.x = __fadd_rn(a.x, v[s].x);
        a.y = __fadd_rn(a.y, v[s].y);
        a.z = __fadd_rn(a.z, v[s].z);
        a.w = __fadd_rn(a.w, v[s].w);
      }
    uint2 o;
    o.x = __bfloat16_as_ushort(__float2bfloat16_rn(a.x)) | (static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(a.y))) << 16);
    o.y = __bfloat16_as_ushort(__float2bfloat16_rn(a.z)) | (static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(a.w))) << 16);
    reinterpret_cast<uint2*>(out)[i] = o;
  }
}

// ------------------------------------------------------------ host side
template <int BN>
static int launch_w4a16_tc_t(const CUtensorMap* maps, const W4A16TcArgs& a, int sms, cudaStream_t stream) {
  static int done[64] = {};
  auto* kern = &w4a16_tc_kernel<BN>;
  const int smem = D2Layout<BN>::kTotal + 1024;
  const int rc = ensure_smem_attr(reinterpret_cast<const void*>(kern), smem, done);
  if (rc != NV4_OK) return rc;
  const dim3 grid(static_cast<unsigned>(std::min<int64_t>(a.units, sms)));
  return launch_kernel(kern, grid, dim3(kD2Threads), smem, stream, true, maps[0], maps[1], maps[2], maps[3], a);
}

// Token tile (256 when there are more than 128 tokens, else 128) and K split.
// The split count comes from a cost model: a 64-K chunk takes ~0.55 us per SM
// whatever the token tile (the dequantisation sets the rate), units run in
// rounds of `sms`, and a split adds its FP32 partials' write and read (at
// ~6 TB/s) plus ~2 us for the sum kernel; a split count is taken only when it
// is at least 5% faster than the best fewer splits.
struct D2Plan {
  int bn, splits;
};

static D2Plan plan_w4a16_tc(int64_t m, int64_t n, int64_t k, int sms) {
  constexpr double kChunkUs = 0.55, kSumUs = 2.0, kBytesPerUs = 6.0e6;
  D2Plan pl;
  pl.bn = m > 128 ? 256 : 128;
  pl.splits = 1;
  const int64_t base = ((n + 127) / 128) * ((m + pl.bn - 1) / pl.bn), kct = k / kD2Chunk;
  double best = 0.0;
  for (int s = 1; s <= kD2MaxSplits && s <= kct; ++s) {
    const int64_t rounds = (base * s + sms - 1) / sms, span = (kct + s - 1) / s;
    double t = static_cast<double>(rounds * span) * kChunkUs;
    if (s > 1) t += kSumUs + static_cast<double>(s) * static_cast<double>(m * n) * 8.0 / kBytesPerUs;
    if (s == 1 || t < 0.95 * best) {
      best = t;
      pl.splits = s;
    }
  }
  return pl;
}

// The shape rules of this kernel (pointer alignment aside) and its plan.
bool w4a16_tc_plan(int64_t m, int64_t n, int64_t k, int sms, int* bn, int* splits) {
  if (m < 1 || n < 32 || n % 32 || k < 128 || k % 128 || m > (int64_t(1) << 30) || n > (int64_t(1) << 30) ||
      sms < 1)
    return false;
  const D2Plan pl = plan_w4a16_tc(m, n, k, sms);
  *bn = pl.bn;
  *splits = pl.splits;
  return true;
}

// Workspace the split plan of a shape wants (0: no split).
int64_t w4a16_tc_workspace_bytes(int64_t m, int64_t n, int64_t k) {
  int bn = 0, splits = 1;
  if (!w4a16_tc_plan(m, n, k, device_sm_count(), &bn, &splits)) return 0;
  return splits > 1 ? splits * m * n * static_cast<int64_t>(sizeof(float)) : 0;
}

// Shapes outside the kernel's alignment rules return NV4_ERR_UNSUPPORTED (the
// caller then takes the mma.sync kernel).  Without a workspace of the plan's
// size (or with one not 16-byte aligned, or `out` not 8-byte aligned) K is
// not split.
int launch_w4a16_tc_gemm(const void* x, const void* qweight, const void* qzeros, const void* scales, void* out,
                         int64_t m, int64_t n, int64_t k, void* workspace, int64_t workspace_bytes,
                         cudaStream_t stream) {
  if ((reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(qweight) & 15) ||
      (reinterpret_cast<uintptr_t>(qzeros) & 15) || (reinterpret_cast<uintptr_t>(scales) & 15))
    return NV4_ERR_UNSUPPORTED;
  const int sms = device_sm_count();
  if (sms <= 0) return NV4_ERR_CUDA;
  D2Plan pl;
  if (!w4a16_tc_plan(m, n, k, sms, &pl.bn, &pl.splits)) return NV4_ERR_UNSUPPORTED;
  if (pl.splits > 1 && (workspace == nullptr || workspace_bytes < pl.splits * m * n * static_cast<int64_t>(sizeof(float)) ||
                        (reinterpret_cast<uintptr_t>(workspace) & 15) || (reinterpret_cast<uintptr_t>(out) & 7)))
    pl.splits = 1;
  const int bn = pl.bn;
  CUtensorMap maps[4];
  memset(maps, 0, sizeof(maps));
  const bool okm = make_tensor_map_2d(&maps[0], CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, x, static_cast<uint64_t>(m),
                                      static_cast<uint64_t>(k), static_cast<uint32_t>(bn), kD2Chunk,
                                      CU_TENSOR_MAP_SWIZZLE_128B) &&
                   make_tensor_map_2d(&maps[1], CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, qweight, static_cast<uint64_t>(k / 8),
                                      static_cast<uint64_t>(n), 8, 128, CU_TENSOR_MAP_SWIZZLE_NONE) &&
                   make_tensor_map_2d(&maps[2], CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, scales, static_cast<uint64_t>(k / 128),
                                      static_cast<uint64_t>(n), 1, 128, CU_TENSOR_MAP_SWIZZLE_NONE) &&
                   make_tensor_map_2d(&maps[3], CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, qzeros, static_cast<uint64_t>(k / 128),
                                      static_cast<uint64_t>(n / 8), 1, 16, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (!okm) return NV4_ERR_CUDA;
  W4A16TcArgs a;
  a.out = static_cast<uint16_t*>(out);
  a.partial = pl.splits > 1 ? static_cast<float*>(workspace) : nullptr;
  a.M = static_cast<int>(m);
  a.N = static_cast<int>(n);
  a.K = static_cast<int>(k);
  a.tiles_m = static_cast<int>((m + bn - 1) / bn);
  a.splits = pl.splits;
  const int64_t units = ((n + 127) / 128) * a.tiles_m * pl.splits;
  if (units > (int64_t(1) << 30)) return NV4_ERR_UNSUPPORTED;
  a.units = static_cast<int>(units);
  const int rc = bn == 256 ? launch_w4a16_tc_t<256>(maps, a, sms, stream) : launch_w4a16_tc_t<128>(maps, a, sms, stream);
  if (rc != NV4_OK || pl.splits == 1) return rc;
  const int64_t count4 = m * n / 4;  // n is a multiple of 32
  const int blocks = static_cast<int>(std::min<int64_t>((count4 + 255) / 256, 2 * static_cast<int64_t>(sms)));
  return launch_kernel(w4a16_split_sum_kernel, dim3(blocks), dim3(256), 0, stream, true,
                       static_cast<const float*>(workspace), static_cast<uint16_t*>(out), count4, count4, pl.splits);
}

}  // namespace nv4
