// Kernel C: grouped INT4 x INT4 GEMM on 5th-generation tensor cores (tcgen05).
//
// Same semantics as Kernel B (nanovllm/kernels/w4a4_grouped_kernel.py:64-90):
// per 128-wide K group g, in increasing g, total = fma(f32(dot_g),
// sa[m,g]*sw[n,g], total); BF16 (or FP32) output; no split-K.
//
// Persistent: one CTA per SM walks 128-weight-row x 128-token tiles over all
// of K, in a fixed order shared by its warps:
//   warp 0      TMA producer: per group, the packed weight tile [128 x 64 B]
//               (64-byte swizzle) and the token tile [128 x 128 B] of INT8
//               codes in the GEMM-ready layout (128-byte swizzle, which is
//               exactly the K-major UMMA operand layout) into a 5-slot ring.
//   warp 1      TMEM allocation (all 512 columns: four 128-column
//               accumulators) and the single MMA-issuing thread: 4 x
//               tcgen05.mma kind::i8 (M=128 weights, N=128 tokens, K=32) per
//               group, the first overwriting the accumulator, then
//               tcgen05.commit.
//   warps 2-3   widen the packed weights to INT8 (16*code, each 32-wide K chunk
//               as its 16 even-k codes then its 16 odd-k codes -- the token
//               operand's K order) into 128-byte-swizzled K-major smem.
//   warps 4-19  epilogue, four per TMEM lane quarter (32 token columns each):
//               tcgen05.ld the INT32 partials of a group (thread = weight row),
//               hand the accumulator back at once, add the bits of 1.5*2^23
//               (so the INT32 16*dot reads as the float 12582912 + 16*dot),
//               and apply the group's scales in FP32; the tile's BF16 outputs
//               are stored after its last group.
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
  int tiles_m, tiles;       // token blocks; tiles (token blocks fastest)
};

constexpr int kTcBN = 128;         // tokens per tile (the MMA's N)
constexpr int kTcStages = 5;       // ring of (packed weights, token codes, widened weights) per group
constexpr int kTcWidenWarps = 2;  // thread t widens weight rows t and t + 64
constexpr int kTcAcc = 4;          // TMEM accumulators (4 x 128 columns: all of TMEM)
constexpr int kTcEpiWarps = 16;    // four per TMEM lane quarter, 32 token columns each
constexpr int kTcFirstEpiWarp = 2 + kTcWidenWarps;
constexpr int kTcThreads = 32 * (kTcFirstEpiWarp + kTcEpiWarps);
constexpr int kTcBlock = 8;        // groups per scale block
constexpr int kTcCols = kTcBN / 4; // token columns per epilogue thread

struct TcLayout {
  static constexpr int kW = 128 * 64;             // packed weights of one group
  static constexpr int kA = kTcBN * 128;          // token codes of one group
  static constexpr int kStage = kW + kA;          // 24 KB (1024-aligned)
  static constexpr int kWide = kTcStages * kStage;  // widened weights [stage][128 x 128 B]
  static constexpr int kSaf = kWide + kTcStages * 16384;  // token scales [2][kTcBlock][kTcBN] float
  static constexpr int kSwf = kSaf + 2 * kTcBlock * kTcBN * 4;  // weight scales [2][kTcBlock][128] float
  static constexpr int kMask = kSwf + 2 * kTcBlock * 128 * 4;   // [2][kTcEpiWarps] int
  static constexpr int kBar = kMask + 2 * kTcEpiWarps * 4;
  // full[S], consumed[S], wfull[S], tfull[A], tfree[A], done, tmem slot
  static constexpr int kTotal = kBar + (3 * kTcStages + 2 * kTcAcc + 1) * 8 + 16;
};

// Bounded wait for a copy this CTA issued, used on the way out (also after an
// error has been recorded, unlike mbar_wait which gives up on one).
__device__ __forceinline__ bool mbar_wait_drain_tc(uint64_t* bar, uint32_t parity) {
  const uint64_t start = global_timer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_timer_ns() - start > kWaitLimitNs) {
      record_error(kErrTimeoutDrain);
      return false;
    }
  }
  return true;
}

__device__ __forceinline__ bool tc_fast_scale(float s) {
  const float a = fabsf(s);
  return a == 0.0f || (a >= 0x1.0p-60f && a <= 0x1.0p+60f);
}

// Persistent: CTA c takes tiles c, c + gridDim.x, ...; tile t covers weight
// rows (t / tiles_m) * 128 and tokens (t % tiles_m) * 128, so the CTAs running
// at one time share a few weight blocks and all token blocks (L2 reuse).
// Every role walks the same (tile, group) sequence; ring slots and mbarrier
// phases run on from tile to tile.
template <bool WG, bool F32>
__global__ void __launch_bounds__(kTcThreads, 1)
    w4a4_tc_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_a,
                   const TcArgs p) {
  constexpr uint32_t IDESC = umma_idesc_s8(128, kTcBN);
  extern __shared__ uint8_t smem_raw[];
  const int G = p.G;
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  float* saf = reinterpret_cast<float*>(smem + TcLayout::kSaf);  // [2][kTcBlock][kTcBN]
  float* swf = reinterpret_cast<float*>(smem + TcLayout::kSwf);  // [2][kTcBlock][128]
  int* wmask = reinterpret_cast<int*>(smem + TcLayout::kMask);   // [2][kTcEpiWarps]: groups with a slow scale
  // Ring slot s holds group gc's packed weights and token codes (full[s]: both
  // TMA copies landed) and its widened weights (wfull[s]: the widen warps are
  // done); consumed[s] (the MMAs' commit) frees all three at once.
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + TcLayout::kBar);
  uint64_t* consumed = full + kTcStages;
  uint64_t* wfull = consumed + kTcStages;
  uint64_t* tfull = wfull + kTcStages;
  uint64_t* tfree = tfull + kTcAcc;
  uint64_t* done_bar = tfree + kTcAcc;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done_bar + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int my_tiles = p.tiles > static_cast<int>(blockIdx.x)
                           ? (p.tiles - static_cast<int>(blockIdx.x) + gridDim.x - 1) / gridDim.x : 0;
  const int total_groups = my_tiles * G;
  auto tile_of = [&](int i) { return static_cast<int>(blockIdx.x) + i * static_cast<int>(gridDim.x); };
  grid_dependents_launch();

  if (threadIdx.x == 0) {
    for (int s = 0; s < kTcStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&consumed[s], 1);
      mbar_init(&wfull[s], kTcWidenWarps);
    }
    for (int i = 0; i < kTcAcc; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tfree[i], kTcEpiWarps);
    }
    mbar_init(done_bar, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTcAcc * kTcBN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool ok = true;

  if (warp == 0) {
    // ---------------- TMA producer: packed weights and token codes per group
    if (lane == 0) {
      tma_prefetch_desc(&tmap_w);
      tma_prefetch_desc(&tmap_a);
      const uint64_t wpol = policy_evict_first();
      auto load_w = [&](int gc) {  // first of a slot's two copies: expects both
        const int s = gc % kTcStages, t = tile_of(gc / G), g = gc % G;
        mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(TcLayout::kW + TcLayout::kA));
        tma_load_2d_hint(smem + s * TcLayout::kStage, &tmap_w, &full[s], g * 64, (t / p.tiles_m) * 128, wpol);
      };
      auto load_a = [&](int gc) {
        const int s = gc % kTcStages, t = tile_of(gc / G), g = gc % G;
        tma_load_2d(smem + s * TcLayout::kStage + TcLayout::kW, &tmap_a, &full[s], g * 128, (t % p.tiles_m) * kTcBN);
      };
      // the first stages' weights stream while the preceding kernel finishes
      const int first = min(kTcStages, total_groups);
      for (int gc = 0; gc < first; ++gc) load_w(gc);
      grid_dependency_wait();  // the token codes come from the preceding kernel
      for (int gc = 0; gc < first; ++gc) load_a(gc);
      int issued = first;
      for (int gc = first; gc < total_groups; ++gc) {
        const int s = gc % kTcStages;
        if (!mbar_wait(&consumed[s], ((gc / kTcStages) - 1) & 1, kErrTimeoutEmpty)) break;
        load_w(gc);
        load_a(gc);
        issued = gc + 1;
      }
      // every copy issued must land before the CTA may exit
      for (int gc = max(0, issued - kTcStages); gc < issued; ++gc)
        if (!mbar_wait_drain_tc(&full[gc % kTcStages], (gc / kTcStages) & 1)) break;
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer: 4 x (M=128 weights, N=128 tokens, K=32) per group
    if (lane == 0) {
      const uint32_t wide_base = smem_u32(smem + TcLayout::kWide);
      const uint32_t stage_base = smem_u32(smem);
      for (int gc = 0; gc < total_groups && ok; ++gc) {
        const int s = gc % kTcStages, b = gc % kTcAcc;
        // wfull[s] implies full[s]: the widen warps waited for both copies
        ok = mbar_wait(&wfull[s], (gc / kTcStages) & 1, kErrTimeoutMma) &&
             mbar_wait(&tfree[b], (gc / kTcAcc) & 1, kErrTimeoutMma);
        if (!ok) break;
        tc_fence_after();
        const uint32_t a_addr = wide_base + s * 16384;
        const uint32_t b_addr = stage_base + s * TcLayout::kStage + TcLayout::kW;
#pragma unroll
        for (int k = 0; k < 4; ++k)  // the first K step overwrites the accumulator: no re-seeding
          umma_s8(tmem + b * kTcBN, umma_desc_sw128(a_addr + k * 32), umma_desc_sw128(b_addr + k * 32), IDESC,
                  k > 0 ? 1u : 0u);
        umma_commit(&tfull[b]);
        umma_commit(&consumed[s]);
      }
      // all issued MMAs must finish before the TMEM is released
      umma_commit(done_bar);
      mbar_wait(done_bar, 0, kErrTimeoutDrain);
    }
  } else if (warp < kTcFirstEpiWarp) {
    // ---------------- widen: thread t owns weight rows t and t + 64 of the tile
    const int t0 = (warp - 2) * 32 + lane;
    const uint32_t wide_base = smem_u32(smem + TcLayout::kWide);
    for (int gc = 0; gc < total_groups && ok; ++gc) {
      const int s = gc % kTcStages, w = s;
      // the slot's copies landed (its widened buffer was freed by the same
      // consumed[s] commit the producer waited for before refilling it)
      ok = mbar_wait(&full[s], (gc / kTcStages) & 1, kErrTimeoutFull);
      if (!ok) break;
#pragma unroll 1
      for (int h = 0; h < 2; ++h) {
        const int t = t0 + 64 * h;
        const uint8_t* src = smem + s * TcLayout::kStage + t * 64;
        uint4 pk[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) pk[c] = *reinterpret_cast<const uint4*>(src + ((c ^ ((t >> 1) & 3)) << 4));
        const uint32_t row_base = wide_base + w * 16384 + (t >> 3) * 1024 + (t & 7) * 128;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const uint4 q = pk[c];
          const uint4 e = make_uint4(nib_even16(q.x), nib_even16(q.y), nib_even16(q.z), nib_even16(q.w));
          const uint4 o = make_uint4(nib_odd16(q.x), nib_odd16(q.y), nib_odd16(q.z), nib_odd16(q.w));
          const uint32_t pe = ((2 * c) ^ (t & 7)) << 4, po = ((2 * c + 1) ^ (t & 7)) << 4;
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(row_base + pe), "r"(e.x), "r"(e.y), "r"(e.z),
                       "r"(e.w)
                       : "memory");
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(row_base + po), "r"(o.x), "r"(o.y), "r"(o.z),
                       "r"(o.w)
                       : "memory");
        }
      }
      fence_proxy_async_smem();  // the generic-proxy stores become visible to the tensor core
      __syncwarp();
      if (lane == 0) mbar_arrive(&wfull[w]);
    }
  } else {
    // ---------------- epilogue: thread = weight row (TMEM lane), 32 token columns
    const int ew = warp - kTcFirstEpiWarp;
    const int quarter = warp & 3;          // the TMEM lane quarter this warp may access
    const int row = quarter * 32 + lane;
    const int c0 = (ew >> 2) * kTcCols;  // warps 4q..4q+3 of the role share lane quarter q
    const int et = ew * 32 + lane;
    const uint32_t taddr = tmem + (static_cast<uint32_t>(quarter * 32) << 16) + c0;
    // every accumulator starts free (the first K step of a group overwrites it)
    __syncwarp();
    if (lane == 0)
      for (int b = 0; b < kTcAcc; ++b) mbar_arrive(&tfree[b]);

    // Scales per block of kTcBlock groups: this thread's weight-row scales in
    // registers; the tile's token scales as floats in shared memory (double
    // buffered), loaded one block ahead; a block takes the two-FMA path unless
    // some scale of the tile is out of range (per-warp masks, no reset needed).
    const int nblocks = (G + kTcBlock - 1) / kTcBlock;
    const int total_blocks = my_tiles * nblocks;
    uint32_t sa_next = 0;
    uint4 sw_next = make_uint4(0, 0, 0, 0);
    const int ld_tok = et % kTcBN, ld_g = (et / kTcBN) * 2;  // this thread loads 2 token scales
    auto load_block = [&](int bc) {
      if (bc >= total_blocks) return;
      const int t = tile_of(bc / nblocks), gb = (bc % nblocks) * kTcBlock;
      const int m = (t % p.tiles_m) * kTcBN + ld_tok, n = (t / p.tiles_m) * 128 + row;
      sa_next = (m < p.M) ? __ldg(reinterpret_cast<const uint32_t*>(p.a_scale + static_cast<size_t>(m) * G + gb + ld_g))
                          : 0u;
      if (WG)
        sw_next = (n < p.N) ? __ldg(reinterpret_cast<const uint4*>(p.w_scale + static_cast<size_t>(n) * G + gb))
                            : make_uint4(0, 0, 0, 0);
    };
    // stage block bc's prefetched scales in shared memory
    auto stage_block = [&](int bc) {
      const int buf = bc & 1;
      float* dst = saf + buf * kTcBlock * kTcBN;
      const float sav[2] = {bf16lo_to_f32(sa_next), bf16hi_to_f32(sa_next)};
      int bad = 0;
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        dst[(ld_g + i) * kTcBN + ld_tok] = sav[i];
        if (WG && !tc_fast_scale(sav[i])) bad |= 1 << (ld_g + i);
      }
      const uint32_t sww[4] = {sw_next.x, sw_next.y, sw_next.z, sw_next.w};
#pragma unroll
      for (int i = 0; i < kTcBlock; ++i) {
        const float v = WG ? ((i & 1) ? bf16hi_to_f32(sww[i >> 1]) : bf16lo_to_f32(sww[i >> 1])) : 1.0f;
        if (c0 == 0) swf[(buf * kTcBlock + i) * 128 + row] = v;
        if (WG && !tc_fast_scale(v)) bad |= 1 << i;
      }
      bad = __reduce_or_sync(0xffffffffu, bad);
      if (lane == 0) wmask[buf * kTcEpiWarps + ew] = bad;
    };

    grid_dependency_wait();  // the token scales come from the preceding kernel
    load_block(0);
    stage_block(0);
    named_barrier_sync(1, kTcEpiWarps * 32);
    float tot[kTcCols];
    int gc = 0;
    for (int bc = 0; bc < total_blocks; ++bc) {
      const int buf = bc & 1;
      const int tile_block = bc % nblocks;
      load_block(bc + 1);  // in flight while this block is processed
      int slow = 0;
#pragma unroll
      for (int w = 0; w < kTcEpiWarps; ++w) slow |= wmask[buf * kTcEpiWarps + w];
      if (tile_block == 0) {
#pragma unroll
        for (int j = 0; j < kTcCols; ++j) tot[j] = 0.0f;
      }
      const int gend = min(kTcBlock, G - tile_block * kTcBlock);
      for (int gl = 0; gl < gend; ++gl, ++gc) {
        const int b = gc % kTcAcc;
        if (ok) ok = mbar_wait(&tfull[b], (gc / kTcAcc) & 1, kErrTimeoutMma);
        if (!ok) continue;  // every warp still reaches the block barrier below
        tc_fence_after();
        const float sw = swf[(buf * kTcBlock + gl) * 128 + row];
        const float* sag = saf + (buf * kTcBlock + gl) * kTcBN + c0;
        const bool fast = ((slow >> gl) & 1) == 0;
        const float2 cw1 = make_float2(__fmul_rn(sw, 0.0625f), __fmul_rn(sw, 0.0625f));
        const float2 cw2 = make_float2(__fmul_rn(sw, -786432.0f), __fmul_rn(sw, -786432.0f));
        // all 32 columns in one round trip; the accumulator goes back to the MMA
        // as soon as the values are in registers
        uint32_t v[kTcCols];
#pragma unroll
        for (int c = 0; c < kTcCols; c += 16)
          tmem_ld16(taddr + b * kTcBN + c, *reinterpret_cast<uint32_t(*)[16]>(&v[c]));
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tfree[b]);
        // the INT32 16*dot plus the bits of 1.5*2^23 reads as the float 12582912 + 16*dot (|16*dot| < 2^22)
#pragma unroll
        for (int j = 0; j < kTcCols; ++j) v[j] += static_cast<uint32_t>(kMagicBits);
        if (fast) {
#pragma unroll
          for (int j = 0; j < kTcCols; j += 4) {
            const float4 s4 = *reinterpret_cast<const float4*>(sag + j);
            // ds = dot * sw exactly, then total = fma(ds, sa, total)
            const float2 d01 = ffma2(make_float2(__uint_as_float(v[j]), __uint_as_float(v[j + 1])), cw1, cw2);
            const float2 d23 = ffma2(make_float2(__uint_as_float(v[j + 2]), __uint_as_float(v[j + 3])), cw1, cw2);
            const float2 t01 = ffma2(d01, make_float2(s4.x, s4.y), make_float2(tot[j], tot[j + 1]));
            const float2 t23 = ffma2(d23, make_float2(s4.z, s4.w), make_float2(tot[j + 2], tot[j + 3]));
            tot[j] = t01.x;
            tot[j + 1] = t01.y;
            tot[j + 2] = t23.x;
            tot[j + 3] = t23.y;
          }
        } else {
#pragma unroll
          for (int j = 0; j < kTcCols; ++j) {
            const float d = fmaf(__uint_as_float(v[j]), 0.0625f, -786432.0f);  // the exact dot
            tot[j] = fmaf(d, WG ? __fmul_rn(sag[j], sw) : sag[j], tot[j]);
          }
        }
      }
      if (tile_block == nblocks - 1 && ok) {  // the tile's outputs
        const int t = tile_of(bc / nblocks);
        const int n = (t / p.tiles_m) * 128 + row, mbase = (t % p.tiles_m) * kTcBN + c0;
        const float swc = (!WG && n < p.N) ? bf16_bits_to_f32(p.w_scale[n]) : 1.0f;
        if (n < p.N) {
#pragma unroll
          for (int j = 0; j < kTcCols; ++j) {
            const int m = mbase + j;
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
      // next block's scales into the other buffer (its last readers finished
      // before the previous barrier), then the barrier every epilogue warp reaches
      if (bc + 1 < total_blocks) stage_block(bc + 1);
      named_barrier_sync(1, kTcEpiWarps * 32);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTcAcc * kTcBN);
  }
}

// ------------------------------------------------------------ host side
template <bool WG, bool F32>
static int launch_tc_t(const CUtensorMap* maps, const TcArgs& a, dim3 grid, int smem, cudaStream_t stream) {
  static int done[64] = {};
  auto* kern = &w4a4_tc_kernel<WG, F32>;
  const int rc = ensure_smem_attr(reinterpret_cast<const void*>(kern), smem, done);
  if (rc != NV4_OK) return rc;
  return launch_kernel(kern, grid, dim3(kTcThreads), smem, stream, true, maps[0], maps[1], a);
}

// Shapes the persistent kernel takes: whole 8-group scale blocks with 4- and
// 16-byte aligned scale rows (every Qwen3-8B projection and TP shard up to 4);
// anything else goes to the streaming kernel.
int launch_w4a4_tc_gemm(const void* a8, const void* w_packed, const void* a_scale, const void* w_scale, void* out,
                        int64_t m, int64_t n, int64_t k, int flags, cudaStream_t stream) {
  const bool wg = (flags & NV4_GEMM_W_SCALE_GROUPED) != 0;
  const bool f32 = (flags & NV4_GEMM_OUT_FP32) != 0;
  const int G = static_cast<int>(k / 128);
  if (G % kTcBlock || (reinterpret_cast<uintptr_t>(a_scale) & 3) || (reinterpret_cast<uintptr_t>(w_scale) & 15))
    return NV4_ERR_UNSUPPORTED;
  const int sms = device_sm_count();
  if (sms <= 0) return NV4_ERR_CUDA;
  const int smem = TcLayout::kTotal + 1024;
  CUtensorMap maps[2];
  memset(maps, 0, sizeof(maps));
  const bool okm = make_tensor_map_u8(&maps[0], w_packed, n, k / 2, 128, 64, CU_TENSOR_MAP_SWIZZLE_64B) &&
                   make_tensor_map_u8(&maps[1], a8, m, k, kTcBN, 128, CU_TENSOR_MAP_SWIZZLE_128B);
  if (!okm) return NV4_ERR_CUDA;
  TcArgs a;
  a.a_scale = static_cast<const uint16_t*>(a_scale);
  a.w_scale = static_cast<const uint16_t*>(w_scale);
  a.out = out;
  a.M = static_cast<int>(m);
  a.N = static_cast<int>(n);
  a.G = G;
  a.tiles_m = static_cast<int>((m + kTcBN - 1) / kTcBN);
  const int64_t tiles = ((n + 127) / 128) * a.tiles_m;
  if (tiles > (int64_t(1) << 30)) return NV4_ERR_UNSUPPORTED;
  a.tiles = static_cast<int>(tiles);
  const dim3 grid(static_cast<unsigned>(std::min<int64_t>(tiles, sms)));
  if (wg) return f32 ? launch_tc_t<true, true>(maps, a, grid, smem, stream) : launch_tc_t<true, false>(maps, a, grid, smem, stream);
  return f32 ? launch_tc_t<false, true>(maps, a, grid, smem, stream) : launch_tc_t<false, false>(maps, a, grid, smem, stream);
}

}  // namespace nv4
