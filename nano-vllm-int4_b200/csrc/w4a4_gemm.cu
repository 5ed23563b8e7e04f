// Kernel B: grouped INT4 x INT4 GEMM for decode shapes (few tokens).
//
// Semantics (nanovllm/kernels/w4a4_grouped_kernel.py:64-90): for each group g
// of 128 along K, in increasing g, total = fma(f32(dot_g), sa[m,g]*sw[n,g],
// total) with one FP32 rounding per group; BF16 (or FP32) output.  With a
// per-channel weight scale, total = fma(f32(dot_g), sa[m,g], total) and the
// result is multiplied by sw[n] at the end.  There is no split-K: each output
// element's FMA chain runs in one thread, in group order.
//
// Design: the weights are the streamed operand.  A CTA owns R = 16*S weight
// rows (S "slabs", chosen so the grid is about one CTA per SM) and all of K.
// One producer warp streams [R x 256-K] packed weight tiles, and the matching
// activation tiles, into a ring of shared-memory stages with 2-D TMA copies
// (128-byte swizzle, no multicast); mbarriers track completion.  The weight
// tiles of the first stages and the weight scales are requested before
// griddepcontrol.wait, so under programmatic dependent launch they stream
// while the activation-prep kernel before this one is still running.
//
// Each consumer warp owns one 16-row slab (and, for narrow layers, a share of
// the token tiles).  It reads packed weight fragments with ldmatrix, widens
// the nibbles to INT8 in registers (16*code, even K then odd K of each 8-code
// word) and issues mma.sync m16n8k32 s8 (INT4 mma.sync is not native on
// sm_100).  Activations arrive either already widened (the "A8" layout the
// prep kernel writes: INT8 codes with the same even/odd K order, so ldmatrix
// yields MMA fragments directly) or packed (widened in registers).
//
// K split (narrow layers): a warp walks its stages in order, so a CTA with few
// slabs is bound by one warp's per-stage latency times the number of stages.
// With KS > 1 the KS warps of a slab take every KS-th stage, write the exact
// per-group partials (dot*sa, or the dot itself off the fast path) to a
// shared-memory block of 2*KS groups, meet at a named barrier, and then each
// applies the FMA chain, in group order, to its 1/KS of the slab's outputs:
// the chain and its roundings are unchanged, only the dot products run in
// parallel.  Wide layers (many slabs per CTA) keep KS = 1 with the chain in
// the warp that computed the dots.
//
// Epilogue per group: the INT32 accumulator starts at the bit pattern of
// 1.5*2^23 and reads as the float 12582912 + 16*dot.  When both scales are in
// a range where sa*sw is exact in FP32 (always, for the quantizer's scales),
//   ds = fma(F, sa/16, -786432*sa) = dot*sa  (exact)   and
//   total = fma(ds, sw, total)                 (= fma(dot, sa*sw, total)),
// two FMAs per element, with the per-token pair (sa/16, -786432*sa) computed
// once per CTA.  Otherwise the reference's three-step form is used.
#include <cstring>

#include "nv4_device.cuh"
#include "nv4_launch.h"
#include "peer_common.cuh"

namespace nv4 {

struct StreamGemmArgs {
  const uint16_t* a_scale;  // bf16 [M, G]
  const uint16_t* w_scale;  // bf16 [N, G] (grouped) or [N]
  void* out;                // bf16 or fp32 [M, N]
  int M, N, G;
  int R;          // weight rows per CTA (16 * slabs)
  int slabs;      // R / 16
  int n_iters;    // ceil(G / 2): two groups per stage
  int stages;
  int scale_tma;  // 1: weight scales arrive by TMA (G % 8 == 0, 16-byte aligned rows)
  // Peer mode (peer_world > 0, FP32 tiles, one token block): CTA j stores its
  // FP32 tile into inbox[parity][peer_rank] of every rank's peer buffer and
  // releases flag[peer_rank][j] on the others (peer_common.cuh); `out` is unused.
  uint8_t* peer_bufs[kPeerMaxRanks];
  int64_t peer_capacity;
  int peer_rank, peer_world;
};

constexpr int kMaxConsumerWarps = 16;
constexpr int kMaxWideSlabs = 12;  // one warp per slab (K not split): at most 16 warps, 128 registers each
constexpr int kProducerWarps = 4;

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

__device__ __forceinline__ bool scale_in_fast_range(float s, float lo, float hi) {
  const float a = fabsf(s);
  return a == 0.0f || (a >= lo && a <= hi);
}

// Shared-memory carve-up (byte offsets from the 1024-aligned base).
struct StreamLayout {
  int w_bytes, a_bytes, stage_bytes, sw_off, sa_off, sac_off, flags_off, ds_off, pt_off, bar_off, total;
  // pt_bytes: the FP32 output tile staged for the peer stores (peer mode), else 0
  __host__ __device__ StreamLayout(int R, int MP, int G, int S, bool wg, int ds_bytes, int pt_bytes) {
    w_bytes = R * 128;
    a_bytes = MP * 128;  // per group (A8) or per stage (packed)
    stage_bytes = w_bytes + 2 * a_bytes;
    sw_off = S * stage_bytes;
    const int sw_bytes = (wg ? R * G : R) * 2;
    sa_off = (sw_off + sw_bytes + 1023) & ~1023;
    sac_off = (sa_off + MP * G * 2 + 15) & ~15;
    flags_off = sac_off + MP * G * 8;
    ds_off = (flags_off + (2 * G + 4) * 4 + 15) & ~15;  // K-split partials (KS > 1)
    pt_off = (ds_off + ds_bytes + 15) & ~15;
    bar_off = (pt_off + pt_bytes + 7) & ~7;
    total = bar_off + (2 * S + 2) * 8 + 16;
  }
};

// Bytes of the K-split partial blocks: per (slab, token share), two buffers of
// 2*KS groups x 16 rows x 8*TPW tokens of FP32.
__host__ __device__ constexpr int stream_ds_bytes(int groups_of_warps, int ks, int tpw) {
  return ks > 1 ? groups_of_warps * 2 * (2 * ks) * (tpw * 128) * 4 : 0;
}

// MT: token tiles of 8 per CTA; TPW: token tiles per consumer warp; KS: warps
// splitting K per slab and token share; A8: activations in the widened layout;
// WG: grouped weight scales; F32: FP32 out.
template <int MT, int TPW, int KS, bool A8, bool WG, bool F32>
__global__ void __launch_bounds__(32 * (kProducerWarps + (KS == 1 && TPW == MT ? kMaxWideSlabs : kMaxConsumerWarps)), 1)
    w4a4_stream_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_a,
                       const __grid_constant__ CUtensorMap tmap_sw, const StreamGemmArgs p) {
  constexpr int MP = MT * 8;
  constexpr int TS = MT / TPW;        // token splits per slab
  constexpr int GI = TPW >= 4 ? 1 : 2;  // groups whose MMAs are interleaved
  constexpr int E = TPW * 4 / KS;       // chain elements per lane and warp (K split)
  extern __shared__ uint8_t smem_raw[];
  const int S = p.stages, R = p.R, G = p.G;
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  const StreamLayout L(R, MP, G, S, WG, stream_ds_bytes(p.slabs * TS, KS, TPW), p.peer_world ? MP * R * 4 : 0);
  uint16_t* sw_s = reinterpret_cast<uint16_t*>(smem + L.sw_off);   // [R][G] (or [R])
  uint16_t* sa_s = reinterpret_cast<uint16_t*>(smem + L.sa_off);   // [MP][G]
  // [G][MP/2] float4 per token pair (t, t+1): (sa_t/16, sa_t+1/16, -786432*sa_t, -786432*sa_t+1)
  float* sac = reinterpret_cast<float*>(smem + L.sac_off);
  int* fast_g = reinterpret_cast<int*>(smem + L.flags_off);        // [G]: both scales in range; [G]: some group not;
                                                                    // [G + 1]: peer-mode epoch of this call
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bar_off);
  uint64_t* empty = full + S;
  uint64_t* scale_bar = empty + S;      // weight scales

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int consumer_warps = p.slabs * TS * KS;
  const int n0 = blockIdx.x * R, m0 = blockIdx.y * MP;
  const uint32_t a_tile_bytes = A8 ? 2u * L.a_bytes : static_cast<uint32_t>(L.a_bytes);

  // The next kernel (activation prep, all-reduce) may launch now: its small
  // CTAs fit beside this one and then wait in griddepcontrol.wait, which still
  // returns only after this whole grid has completed and its writes are visible.
  grid_dependents_launch();
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], consumer_warps / KS);  // one warp per (slab, token share) reads a stage
    }
    mbar_init(&scale_bar[0], 1);
    fence_mbar_init();
  }
  __syncthreads();

  if (warp < kProducerWarps) {
    // ---------------- producers: warp w issues stages w, w + P, ... (one
    // thread each).  Issuing a TMA copy costs the issuing thread ~100 cycles,
    // so one thread cannot keep a narrow layer's stages coming; the copies of
    // several issuing warps overlap.
    if (lane == 0) {
      const int pw = warp;
      const uint64_t wpol = policy_evict_first();
      if (pw == 0) {
        tma_prefetch_desc(&tmap_w);
        tma_prefetch_desc(&tmap_a);
        if (p.scale_tma) {
          mbar_arrive_expect_tx(&scale_bar[0], static_cast<uint32_t>((WG ? R * G : R) * 2));
          if (WG)
            tma_load_2d(sw_s, &tmap_sw, &scale_bar[0], 0, n0);
          else
            tma_load_2d(sw_s, &tmap_sw, &scale_bar[0], n0, 0);
        }
      }
      const uint32_t bytes = static_cast<uint32_t>(L.w_bytes) + a_tile_bytes;
      auto load_w = [&](int it) {
        const int slot = it % S;
        mbar_arrive_expect_tx(&full[slot], bytes);
        tma_load_2d_hint(smem + slot * L.stage_bytes, &tmap_w, &full[slot], it * 128, n0, wpol);
      };
      auto load_a = [&](int it) {
        const int slot = it % S;
        uint8_t* dst = smem + slot * L.stage_bytes + L.w_bytes;
        if (A8) {
          tma_load_2d(dst, &tmap_a, &full[slot], it * 256, m0);
          tma_load_2d(dst + L.a_bytes, &tmap_a, &full[slot], it * 256 + 128, m0);
        } else {
          tma_load_2d(dst, &tmap_a, &full[slot], it * 128, m0);
        }
      };
      // Every ring slot's weight tile goes out before griddepcontrol.wait: it
      // streams while the preceding kernel finishes (the activation scales
      // come by plain loads, so nothing the consumers need first queues
      // behind these copies).
      const int early = min(S, p.n_iters);
      for (int it = pw; it < early; it += kProducerWarps) load_w(it);
      grid_dependency_wait();  // the activations come from the preceding kernel
      int last = -1;
      for (int it = pw; it < p.n_iters; it += kProducerWarps) {
        if (it >= early) {
          if (it >= S && !mbar_wait(&empty[it % S], ((it / S) - 1) & 1, kErrTimeoutEmpty)) break;
          load_w(it);
        }
        load_a(it);
        last = it;
      }
      if (error_raised()) {
        // Before the CTA may exit, the copies this thread issued must have
        // landed: its stages, and (warp 0) the weight scales, which consumers
        // that gave up may not have waited for.
        for (int it = last; it >= 0 && it > last - S; it -= kProducerWarps) mbar_wait_drain(&full[it % S], (it / S) & 1);
        if (pw == 0 && p.scale_tma) mbar_wait_drain(&scale_bar[0], 0);
      }
    }
    return;
  }

  // ---------------- consumers
  const int cw = warp - kProducerWarps;
  const int ct = threadIdx.x - 32 * kProducerWarps, cthreads = 32 * consumer_warps;
  const bool active = cw < consumer_warps;
  const int grp = cw / KS, ks = cw % KS;  // (slab, token share) group; K-split index within it
  const int slab = grp / TS, tile0 = (grp % TS) * TPW;
  const int gid = lane >> 2, tig = lane & 3;

  // Weight scales (by TMA when the rows are 16-byte multiples, else cooperative
  // loads) and their range check do not depend on the preceding kernel, so they
  // run before griddepcontrol.wait.  The activation scales (a few KB) are then
  // read with plain loads straight into the per-token epilogue constants.  A
  // group leaves the two-FMA path if any of its scales is out of range (every
  // thread checks a slice; clearing is idempotent).  No early return before the
  // named barriers: every consumer reaches them.
  bool ok = true;
  if (!p.scale_tma) {
    if (active) {
      const int nsw = WG ? R * G : R;
      for (int i = ct; i < nsw; i += cthreads) {
        const int r = WG ? i / G : i;
        sw_s[i] = (n0 + r < p.N) ? p.w_scale[static_cast<size_t>(n0) * (WG ? G : 1) + i] : uint16_t(0);
      }
    }
  } else {
    ok = mbar_wait(&scale_bar[0], 0, kErrTimeoutFull);
  }
  for (int g = ct; g <= G; g += cthreads) fast_g[g] = g < G ? 1 : 0;
  named_barrier_sync(1, cthreads);
  if (WG && active)
    for (int i = ct; i < R * G; i += cthreads)
      if (!scale_in_fast_range(bf16_bits_to_f32(sw_s[i]), 0x1.0p-30f, 0x1.0p+27f)) fast_g[i % G] = 0, fast_g[G] = 1;
  grid_dependency_wait();
  if (p.peer_world) {
    uint8_t* own = p.peer_bufs[p.peer_rank];
    peer_advance_epochs(own, blockIdx.x, gridDim.x, ct, cthreads);
    if (ct == 0) fast_g[G + 1] = static_cast<int>(peer_epochs(own)[blockIdx.x]);
  }
  if (active) {
    // eight independent loads per thread in flight: one L2 round trip for the
    // whole [MP x G] block at decode sizes
    constexpr int kBatch = 8;
    const int nsa = MP * G;
    for (int i0 = ct; i0 < nsa; i0 += kBatch * cthreads) {
      uint16_t bits[kBatch];
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        const int i = i0 + u * cthreads;
        bits[u] = (i < nsa && m0 + i / G < p.M) ? p.a_scale[static_cast<size_t>(m0) * G + i] : uint16_t(0);
      }
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        const int i = i0 + u * cthreads;
        if (i >= nsa) break;
        const int t = i / G, g = i - t * G;
        sa_s[i] = bits[u];
        const float sa = bf16_bits_to_f32(bits[u]);
        float* q = sac + (g * MP + (t & ~1)) * 2 + (t & 1);
        q[0] = __fmul_rn(sa, 0.0625f);
        q[2] = __fmul_rn(sa, -786432.0f);
        if (!scale_in_fast_range(sa, 0x1.0p-100f, 0x1.0p+100f)) fast_g[g] = 0, fast_g[G] = 1;
      }
    }
  }
  named_barrier_sync(1, cthreads);
  if (!active) return;
  // Every group on the two-FMA path (the quantizer's scales always are): the
  // epilogues take their loads out of the per-group branches.
  const bool all_fast = A8 && fast_g[G] == 0;

  const uint32_t sbase = smem_u32(smem);
  const int row_lo = slab * 16 + gid, row_hi = row_lo + 8;
  const uint32_t lrow = slab * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
  constexpr uint32_t kATile = MP * 128;  // bytes of one token tile per group
  // Loop-invariant swizzled ldmatrix offsets of this lane: weights [group][half],
  // widened tokens [tile][half] or packed tokens [group][tile].
  uint32_t off_w[2][2], off_a[TPW][2];
#pragma unroll
  for (int gg = 0; gg < 2; ++gg)
#pragma unroll
    for (int h = 0; h < 2; ++h) off_w[gg][h] = sw128_offset(lrow, gg * 4 + 2 * h + (lane >> 4));
#pragma unroll
  for (int t = 0; t < TPW; ++t) {
    const uint32_t trow = (tile0 + t) * 8 + (lane & 7);
#pragma unroll
    for (int h = 0; h < 2; ++h) off_a[t][h] = A8 ? sw128_offset(trow, 4 * h + (lane >> 3)) : sw128_offset(trow, h * 4 + (lane >> 3));
  }
  // acc reads as F = 12582912 + S*dot, S = 16 (A8: codes x 16-weights) or 256
  constexpr float kInvS = A8 ? 0.0625f : 0.00390625f;
  constexpr float kOff = A8 ? -786432.0f : -49152.0f;
  const int bias[4] = {kMagicBits, kMagicBits, kMagicBits, kMagicBits};  // MMA C of a group's first step

  // Bias-seeded INT32 accumulators of groups gb .. gb+GI-1 of the stage at
  // (wbase, abase), for this warp's slab and token tiles.  GI groups are
  // processed together so that GI * TPW independent MMA chains are in flight;
  // all fragment loads of a batch are issued before its MMAs.
  auto stage_mma = [&](uint32_t wbase, uint32_t abase, int gb, int (&acc)[GI][TPW][4]) {
    uint32_t aw[GI][4][4];    // widened weight fragments [group][k32 step][a0..a3]
    uint32_t bq[GI][TPW][8];  // token fragments [group][tile][k32 step x (b0, b1)]
#pragma unroll
    for (int gi = 0; gi < GI; ++gi) {
      const int gg = gb + gi;
      uint32_t af[2][4];
      ldmatrix_x4(wbase + off_w[gg][0], af[0][0], af[0][1], af[0][2], af[0][3]);
      ldmatrix_x4(wbase + off_w[gg][1], af[1][0], af[1][1], af[1][2], af[1][3]);
#pragma unroll
      for (int t = 0; t < TPW; ++t) {
        if (A8) {
          const uint32_t ab = abase + gg * kATile;
          ldmatrix_x4(ab + off_a[t][0], bq[gi][t][0], bq[gi][t][1], bq[gi][t][2], bq[gi][t][3]);
          ldmatrix_x4(ab + off_a[t][1], bq[gi][t][4], bq[gi][t][5], bq[gi][t][6], bq[gi][t][7]);
        } else {
          uint32_t bf[4];
          ldmatrix_x4(abase + off_a[t][gg], bf[0], bf[1], bf[2], bf[3]);
#pragma unroll
          for (int w = 0; w < 4; ++w) {
            bq[gi][t][2 * w] = nib_even16(bf[w]);
            bq[gi][t][2 * w + 1] = nib_odd16(bf[w]);
          }
        }
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        aw[gi][2 * h][0] = nib_even16(af[h][0]);
        aw[gi][2 * h][1] = nib_even16(af[h][1]);
        aw[gi][2 * h][2] = nib_odd16(af[h][0]);
        aw[gi][2 * h][3] = nib_odd16(af[h][1]);
        aw[gi][2 * h + 1][0] = nib_even16(af[h][2]);
        aw[gi][2 * h + 1][1] = nib_even16(af[h][3]);
        aw[gi][2 * h + 1][2] = nib_odd16(af[h][2]);
        aw[gi][2 * h + 1][3] = nib_odd16(af[h][3]);
      }
    }
#pragma unroll
    for (int q = 0; q < 4; ++q)
#pragma unroll
      for (int gi = 0; gi < GI; ++gi)
#pragma unroll
        for (int t = 0; t < TPW; ++t) {
          if (q == 0)
            mma_s8_16832_c(acc[gi][t], aw[gi][q][0], aw[gi][q][1], aw[gi][q][2], aw[gi][q][3], bq[gi][t][0],
                           bq[gi][t][1], bias);
          else
            mma_s8_16832(acc[gi][t], aw[gi][q][0], aw[gi][q][1], aw[gi][q][2], aw[gi][q][3], bq[gi][t][2 * q],
                         bq[gi][t][2 * q + 1]);
        }
  };

  const int peer_parity = p.peer_world ? (fast_g[G + 1] & 1) : 0;
  float* ptile = reinterpret_cast<float*>(smem + L.pt_off);  // peer mode: [MP tokens][R rows] FP32
  auto store_out = [&](int row, int tok, float v) {
    const int rr = n0 + row, tk = m0 + tok;
    if (tk < p.M && rr < p.N) {
      if (!WG) v = __fmul_rn(v, bf16_bits_to_f32(sw_s[row]));
      const size_t o = static_cast<size_t>(tk) * p.N + rr;
      if (p.peer_world) {
        ptile[tok * R + row] = v;  // copied to the ranks' inboxes in 16-byte stores below
      } else if (F32)
        static_cast<float*>(p.out)[o] = v;
      else
        static_cast<__nv_bfloat16*>(p.out)[o] = __float2bfloat16_rn(v);
    }
  };

  if constexpr (KS == 1) {
    float tot[TPW][4];
#pragma unroll
    for (int t = 0; t < TPW; ++t)
#pragma unroll
      for (int i = 0; i < 4; ++i) tot[t][i] = 0.0f;
    int it = 0;
    for (; ok && it < p.n_iters; ++it) {
      const int slot = it % S;
      if (!mbar_wait(&full[slot], (it / S) & 1, kErrTimeoutFull)) {
        ok = false;
        break;
      }
      const uint32_t wbase = sbase + slot * L.stage_bytes, abase = wbase + L.w_bytes;
#pragma unroll
      for (int gb = 0; gb < 2; gb += GI) {
        int acc[GI][TPW][4];
        stage_mma(wbase, abase, gb, acc);
#pragma unroll
        for (int gi = 0; gi < GI; ++gi) {  // groups in increasing order
          const int g = it * 2 + gb + gi;
          if (g >= G) break;
          float sw0 = 1.0f, sw1 = 1.0f;
          if (WG) {
            sw0 = bf16_bits_to_f32(sw_s[row_lo * G + g]);
            sw1 = bf16_bits_to_f32(sw_s[row_hi * G + g]);
          }
          const bool fast = all_fast || (A8 && fast_g[g] != 0);
#pragma unroll
          for (int t = 0; t < TPW; ++t) {
            const int* a = acc[gi][t];
            const int tok = (tile0 + t) * 8 + tig * 2;
            if (fast) {
              // (sa0/16, sa1/16, c0, c1); ds = dot*sa, then total = fma(ds, sw, total),
              // two elements per packed FMA
              const float4 c = *reinterpret_cast<const float4*>(&sac[(g * MP + tok) * 2]);
              const float2 s01 = make_float2(c.x, c.y), c01 = make_float2(c.z, c.w);
              const float2 ds01 = ffma2(make_float2(__int_as_float(a[0]), __int_as_float(a[1])), s01, c01);
              const float2 ds23 = ffma2(make_float2(__int_as_float(a[2]), __int_as_float(a[3])), s01, c01);
              const float2 w0 = WG ? make_float2(sw0, sw0) : make_float2(1.0f, 1.0f);  // fma(x, 1, y) = x + y
              const float2 w1 = WG ? make_float2(sw1, sw1) : make_float2(1.0f, 1.0f);
              const float2 t01 = ffma2(ds01, w0, make_float2(tot[t][0], tot[t][1]));
              const float2 t23 = ffma2(ds23, w1, make_float2(tot[t][2], tot[t][3]));
              tot[t][0] = t01.x;
              tot[t][1] = t01.y;
              tot[t][2] = t23.x;
              tot[t][3] = t23.y;
            } else {
              const float sa0 = bf16_bits_to_f32(sa_s[tok * G + g]);
              const float sa1 = bf16_bits_to_f32(sa_s[(tok + 1) * G + g]);
              const float d0 = fmaf(__int_as_float(a[0]), kInvS, kOff);
              const float d1 = fmaf(__int_as_float(a[1]), kInvS, kOff);
              const float d2 = fmaf(__int_as_float(a[2]), kInvS, kOff);
              const float d3 = fmaf(__int_as_float(a[3]), kInvS, kOff);
              if (WG) {
                tot[t][0] = fmaf(d0, __fmul_rn(sa0, sw0), tot[t][0]);
                tot[t][1] = fmaf(d1, __fmul_rn(sa1, sw0), tot[t][1]);
                tot[t][2] = fmaf(d2, __fmul_rn(sa0, sw1), tot[t][2]);
                tot[t][3] = fmaf(d3, __fmul_rn(sa1, sw1), tot[t][3]);
              } else {
                tot[t][0] = fmaf(d0, sa0, tot[t][0]);
                tot[t][1] = fmaf(d1, sa1, tot[t][1]);
                tot[t][2] = fmaf(d2, sa0, tot[t][2]);
                tot[t][3] = fmaf(d3, sa1, tot[t][3]);
              }
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
    }

    if (ok) {  // on error the producers let their copies land before the CTA exits
#pragma unroll
      for (int t = 0; t < TPW; ++t) {
        const int t0 = (tile0 + t) * 8 + tig * 2;
        store_out(row_lo, t0, tot[t][0]);
        store_out(row_lo, t0 + 1, tot[t][1]);
        store_out(row_hi, t0, tot[t][2]);
        store_out(row_hi, t0 + 1, tot[t][3]);
      }
    }
  } else {
    // K split.  Partials of a block of 2*KS groups (KS stages, one per warp):
    // [2 buffers][2*KS groups][KS chunks][32 lanes][E] FP32 per (slab, token
    // share); chunk c of a lane holds its accumulator elements e = t*4 + i in
    // [c*E, (c+1)*E), and warp ks applies the chain to chunk ks.
    constexpr int BUF = 2 * KS * KS * 32 * E;
    float* dsb = reinterpret_cast<float*>(smem + L.ds_off) + grp * 2 * BUF;
    float tot[E];
#pragma unroll
    for (int o = 0; o < E; ++o) tot[o] = 0.0f;
    const int nblk = (p.n_iters + KS - 1) / KS;
    for (int blk = 0; blk < nblk; ++blk) {
      float* buf = dsb + (blk & 1) * BUF;
      const int it = blk * KS + ks;
      if (ok && it < p.n_iters) {
        const int slot = it % S;
        ok = mbar_wait(&full[slot], (it / S) & 1, kErrTimeoutFull);
        if (ok) {
          const uint32_t wbase = sbase + slot * L.stage_bytes, abase = wbase + L.w_bytes;
#pragma unroll
          for (int gb = 0; gb < 2; gb += GI) {
            int acc[GI][TPW][4];
            stage_mma(wbase, abase, gb, acc);
#pragma unroll
            for (int gi = 0; gi < GI; ++gi) {
              const int gg = gb + gi, g = it * 2 + gg;
              if (g >= G) break;
              const bool fast = all_fast || (A8 && fast_g[g] != 0);
              float v[TPW * 4];
#pragma unroll
              for (int t = 0; t < TPW; ++t) {
                const int tok = (tile0 + t) * 8 + tig * 2;
                // fast: dot*sa (exact), with (sa0/16, sa1/16, c0, c1); otherwise the exact dot
                const float4 c = *reinterpret_cast<const float4*>(&sac[(g * MP + tok) * 2]);
                const float2 s01 = fast ? make_float2(c.x, c.y) : make_float2(kInvS, kInvS);
                const float2 c01 = fast ? make_float2(c.z, c.w) : make_float2(kOff, kOff);
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                  const float2 d = ffma2(make_float2(__int_as_float(acc[gi][t][2 * h]), __int_as_float(acc[gi][t][2 * h + 1])),
                                         s01, c01);
                  v[t * 4 + 2 * h] = d.x;
                  v[t * 4 + 2 * h + 1] = d.y;
                }
              }
              float* dst = buf + ((2 * ks + gg) * KS * 32 + lane) * E;
#pragma unroll
              for (int c = 0; c < KS; ++c) {
                float* d = dst + c * 32 * E;
                if constexpr (E % 4 == 0) {
#pragma unroll
                  for (int o = 0; o < E; o += 4)
                    *reinterpret_cast<float4*>(d + o) = make_float4(v[c * E + o], v[c * E + o + 1], v[c * E + o + 2],
                                                                     v[c * E + o + 3]);
                } else if constexpr (E == 2) {
                  *reinterpret_cast<float2*>(d) = make_float2(v[c * E], v[c * E + 1]);
                } else {
                  d[0] = v[c];
                }
              }
            }
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&empty[slot]);
        }
      }
      named_barrier_sync(2 + grp, KS * 32);
      // the chain over the block's groups, in increasing g, for chunk ks
      const int gbase = blk * 2 * KS;
      if (all_fast) {
        // every load of the block first (partials, and the weight scales of the
        // at most two rows this lane's elements lie in), then the FMA chain
        float v[2 * KS][E];
        float swv[2][2 * KS];
#pragma unroll
        for (int gl = 0; gl < 2 * KS; ++gl) {
          const int g = gbase + gl;
          const float* src = buf + ((gl * KS + ks) * 32 + lane) * E;
          if (g < G) {
            if constexpr (E % 4 == 0) {
#pragma unroll
              for (int o = 0; o < E; o += 4) {
                const float4 x = *reinterpret_cast<const float4*>(src + o);
                v[gl][o] = x.x;
                v[gl][o + 1] = x.y;
                v[gl][o + 2] = x.z;
                v[gl][o + 3] = x.w;
              }
            } else if constexpr (E == 2) {
              const float2 x = *reinterpret_cast<const float2*>(src);
              v[gl][0] = x.x;
              v[gl][1] = x.y;
            } else {
              v[gl][0] = src[0];
            }
          } else {
#pragma unroll
            for (int o = 0; o < E; ++o) v[gl][o] = 0.0f;
          }
#pragma unroll
          for (int h = 0; h < 2; ++h)
            swv[h][gl] = (WG && g < G) ? bf16_bits_to_f32(sw_s[(h ? row_hi : row_lo) * G + g]) : 1.0f;
        }
#pragma unroll
        for (int gl = 0; gl < 2 * KS; ++gl) {
          if (gbase + gl >= G) break;
          if constexpr (E % 2 == 0) {
#pragma unroll
            for (int o = 0; o < E; o += 2) {
              const float sw = ((ks * E + o) & 3) < 2 ? swv[0][gl] : swv[1][gl];  // 1 without WG: fma(x, 1, y) = x + y
              const float2 r = ffma2(make_float2(v[gl][o], v[gl][o + 1]), make_float2(sw, sw),
                                     make_float2(tot[o], tot[o + 1]));
              tot[o] = r.x;
              tot[o + 1] = r.y;
            }
          } else {
#pragma unroll
            for (int o = 0; o < E; ++o) tot[o] = fmaf(v[gl][o], ((ks * E + o) & 3) < 2 ? swv[0][gl] : swv[1][gl], tot[o]);
          }
        }
        continue;
      }
      for (int gl = 0; gl < 2 * KS; ++gl) {
        const int g = blk * 2 * KS + gl;
        if (g >= G) break;
        const bool fast = A8 && fast_g[g] != 0;
        const float* src = buf + ((gl * KS + ks) * 32 + lane) * E;
        float v[E];
        if constexpr (E % 4 == 0) {
#pragma unroll
          for (int o = 0; o < E; o += 4) {
            const float4 x = *reinterpret_cast<const float4*>(src + o);
            v[o] = x.x;
            v[o + 1] = x.y;
            v[o + 2] = x.z;
            v[o + 3] = x.w;
          }
        } else if constexpr (E == 2) {
          const float2 x = *reinterpret_cast<const float2*>(src);
          v[0] = x.x;
          v[1] = x.y;
        } else {
          v[0] = src[0];
        }
        if (fast && E % 2 == 0) {
          // elements (o, o+1) are tokens (t, t+1) of one row: one packed FMA
#pragma unroll
          for (int o = 0; o < E; o += 2) {
            const int e = ks * E + o, i = e & 3;
            const float sw = WG ? bf16_bits_to_f32(sw_s[(i < 2 ? row_lo : row_hi) * G + g]) : 1.0f;
            const float2 r = ffma2(make_float2(v[o], v[o + 1]), make_float2(sw, sw), make_float2(tot[o], tot[o + 1]));
            tot[o] = r.x;
            tot[o + 1] = r.y;
          }
          continue;
        }
#pragma unroll
        for (int o = 0; o < E; ++o) {
          const int e = ks * E + o, t = e >> 2, i = e & 3;
          const int row = i < 2 ? row_lo : row_hi, tok = (tile0 + t) * 8 + tig * 2 + (i & 1);
          if (WG) {
            const float sw = bf16_bits_to_f32(sw_s[row * G + g]);
            tot[o] = fast ? fmaf(v[o], sw, tot[o])
                          : fmaf(v[o], __fmul_rn(bf16_bits_to_f32(sa_s[tok * G + g]), sw), tot[o]);
          } else {
            tot[o] = fast ? __fadd_rn(tot[o], v[o]) : fmaf(v[o], bf16_bits_to_f32(sa_s[tok * G + g]), tot[o]);
          }
        }
      }
    }
    if (!error_raised()) {  // on error the producers let their copies land before the CTA exits
#pragma unroll
      for (int o = 0; o < E; ++o) {
        const int e = ks * E + o, t = e >> 2, i = e & 3;
        store_out(i < 2 ? row_lo : row_hi, (tile0 + t) * 8 + tig * 2 + (i & 1), tot[o]);
      }
    }
  }
  if (p.peer_world) {
    // The staged tile goes to every rank's inbox in 16-byte stores (whole
    // token rows of the CTA's R columns; each CTA starts with a different
    // rank, spreading the NVLink traffic), then, after every consumer's
    // stores, one thread's system-scope release of this CTA's flag on each
    // peer (released on error too, so that the peers do not wait out their
    // limit; the error word marks the call as failed).
    named_barrier_sync(1, cthreads);
    const int wq = min(R, p.N - n0) >> 2, rows = min(MP, p.M - m0);
    for (int j = 0; j < p.peer_world; ++j) {
      const int r = (static_cast<int>(blockIdx.x) + j) % p.peer_world;
      float* dst = peer_inbox(p.peer_bufs[r], p.peer_capacity, peer_parity, p.peer_rank);
      for (int i = ct; i < rows * wq; i += cthreads) {
        const int t = i / wq, c = i - t * wq;
        *reinterpret_cast<float4*>(dst + static_cast<size_t>(m0 + t) * p.N + n0 + 4 * c) =
            *reinterpret_cast<const float4*>(ptile + t * R + 4 * c);
      }
    }
    named_barrier_sync(1, cthreads);
    if (ct == 0) {
      const uint32_t e = static_cast<uint32_t>(fast_g[G + 1]);
      for (int r = 0; r < p.peer_world; ++r)
        if (r != p.peer_rank) st_release_sys(peer_flags(p.peer_bufs[r]) + p.peer_rank * kPeerSlots + blockIdx.x, e);
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
template <int MT, int TPW, int KS, bool A8, bool WG, bool F32>
static int launch_t(const CUtensorMap* maps, const StreamGemmArgs& a, dim3 grid, int threads, int smem,
                    cudaStream_t stream) {
  static int done[64] = {};
  auto* kern = &w4a4_stream_kernel<MT, TPW, KS, A8, WG, F32>;
  const int rc = ensure_smem_attr(reinterpret_cast<const void*>(kern), smem, done);
  if (rc != NV4_OK) return rc;
  return launch_kernel(kern, grid, dim3(threads), smem, stream, true, maps[0], maps[1], maps[2], a);
}

template <int MT, int TPW, int KS>
static int launch_flags(const CUtensorMap* maps, const StreamGemmArgs& a, dim3 grid, int threads, int smem, bool a8,
                        bool wg, bool f32, cudaStream_t s) {
  if (a8) {
    if (wg) return f32 ? launch_t<MT, TPW, KS, true, true, true>(maps, a, grid, threads, smem, s)
                       : launch_t<MT, TPW, KS, true, true, false>(maps, a, grid, threads, smem, s);
    return f32 ? launch_t<MT, TPW, KS, true, false, true>(maps, a, grid, threads, smem, s)
               : launch_t<MT, TPW, KS, true, false, false>(maps, a, grid, threads, smem, s);
  }
  if (wg) return f32 ? launch_t<MT, TPW, KS, false, true, true>(maps, a, grid, threads, smem, s)
                     : launch_t<MT, TPW, KS, false, true, false>(maps, a, grid, threads, smem, s);
  return f32 ? launch_t<MT, TPW, KS, false, false, true>(maps, a, grid, threads, smem, s)
             : launch_t<MT, TPW, KS, false, false, false>(maps, a, grid, threads, smem, s);
}

constexpr int kSmemLimit = 227 * 1024;

static bool make_map_u16(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows,
                         uint32_t box_cols) {
  return make_tensor_map_2d(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, base, rows, cols, box_rows, box_cols,
                            CU_TENSOR_MAP_SWIZZLE_NONE);
}

// Launch plan of the stream kernel: a pure function of the shape, the flags
// and the SM count (no device calls), so the CPU tests can sweep it.
int plan_w4a4_stream(int64_t m, int64_t n, int64_t k, bool wg, int sms, bool peer, StreamPlan* out) {
  if (m < 1 || n < 1 || k < 128 || k % 128 || sms < 1 || out == nullptr) return NV4_ERR_INVALID_ARGUMENT;
  const int MT = m <= 8 ? 1 : (m <= 16 ? 2 : 4);
  const int MP = MT * 8;
  const int64_t mblocks = (m + MP - 1) / MP;
  const int G = static_cast<int>(k / 128);
  const int64_t total_slabs = (n + 15) / 16;
  // About one CTA per SM: slabs (16-row units) per CTA.
  const int64_t ctas_per_mblock = std::max<int64_t>(1, sms / std::min<int64_t>(mblocks, sms));
  int slabs = static_cast<int>(std::min<int64_t>(kMaxConsumerWarps, (total_slabs + ctas_per_mblock - 1) / ctas_per_mblock));
  slabs = std::max(1, slabs);
  // Narrow layers (up to 4 slabs per CTA): split K over 4 warps per slab, and
  // with 32 tokens and at most 2 slabs also split the token tiles over two
  // warps (16 consumer warps).  Wider ones: one warp per slab (see below for
  // 5-8 slabs).
  //
  // Ring rule.  A producer warp reuses a slot after waiting on its empty
  // barrier by phase parity, which is only sound if the slot's previous phase
  // has completed.  Producers issue stages round-robin (kProducerWarps of
  // them) and, with a K split, the KS warps of a block release their stages in
  // any order, so the ring must hold KS + kProducerWarps stages (or all of K):
  // with fewer, a producer can pass the wait one phase early and a TMA copy
  // can overwrite a slot still being read.  Fewer slabs per CTA until it fits.
  // With more than 8 tokens, 5-8 slab CTAs keep their slabs with one warp per
  // slab and the token tiles split over two warps (measured: 16 us against
  // 22 us for 4-slab CTAs in two waves at N = 12288, K = 4096, M = 32); with
  // up to 8 tokens there are no token tiles to split, and 4-slab CTAs with the
  // 4-way K split are faster.
  if (slabs > 4 && slabs <= 8 && MT < 2) slabs = 4;
  // Peer mode stores one flag per CTA, so the grid must fit kPeerSlots: start
  // from enough slabs per CTA for that (the ring rule may still lower it).
  if (peer) slabs = std::max<int>(slabs, static_cast<int>(std::min<int64_t>(kMaxWideSlabs, (total_slabs + kPeerSlots - 1) / kPeerSlots)));
  const int n_iters = (G + 1) / 2;
  int ks = 0, ts = 1, tpw = MT, ds_bytes = 0, pt_bytes = 0, R = 0, stages = 0;
  for (;;) {
    ks = slabs <= 4 ? 4 : 1;
    if (ks == 1) slabs = std::min(slabs, kMaxWideSlabs);  // wider layers take more CTAs
    ts = (ks == 4 && MT == 4 && slabs <= 2) ? 2 : 1;
    if (ks == 1 && MT >= 2 && slabs * 2 <= kMaxConsumerWarps && slabs < 8) ts = 2;
    tpw = MT / ts;
    ds_bytes = stream_ds_bytes(slabs * ts, ks, tpw);
    R = slabs * 16;
    pt_bytes = peer ? MP * R * 4 : 0;
    const StreamLayout one(R, MP, G, 1, wg, ds_bytes, pt_bytes);
    const int fixed = one.total - one.stage_bytes;
    stages = (kSmemLimit - 1024 - fixed - 64) / (one.stage_bytes + 16);
    stages = std::min(stages, std::min(16, n_iters));
    if (stages >= std::min(n_iters, ks + kProducerWarps) || slabs == 1) break;
    slabs = slabs > 4 ? 4 : slabs - 1;
  }
  if (stages < 1 || stages < std::min(n_iters, ks + kProducerWarps)) return NV4_ERR_UNSUPPORTED;
  const StreamLayout lay(R, MP, G, stages, wg, ds_bytes, pt_bytes);
  StreamPlan pl;
  pl.token_tiles = MT;
  pl.slabs = slabs;
  pl.k_split = ks;
  pl.token_splits = ts;
  pl.tiles_per_warp = tpw;
  pl.rows_per_cta = R;
  pl.stages = stages;
  pl.n_iters = n_iters;
  pl.ds_bytes = ds_bytes;
  pl.smem_bytes = lay.total + 1024;
  pl.grid_x = static_cast<int>((n + R - 1) / R);
  pl.grid_y = static_cast<int>(mblocks);
  pl.threads = 32 * (kProducerWarps + slabs * ts * ks);
  pl.producer_warps = kProducerWarps;
  if (pl.smem_bytes > kSmemLimit) return NV4_ERR_UNSUPPORTED;
  if (peer && (mblocks != 1 || pl.grid_x > kPeerSlots)) return NV4_ERR_UNSUPPORTED;
  *out = pl;
  return NV4_OK;
}

// a8 != nullptr: activations in the widened INT8 layout [m, k]; else a_packed [m, k/2].
int launch_w4a4_stream_gemm(const void* a_packed, const void* a8, const void* w_packed, const void* a_scale,
                            const void* w_scale, void* out, int64_t m, int64_t n, int64_t k, int flags,
                            cudaStream_t stream, PeerTarget* peer) {
  const int sms = device_sm_count();
  if (sms <= 0) return NV4_ERR_CUDA;
  const bool wg = (flags & NV4_GEMM_W_SCALE_GROUPED) != 0;
  const bool f32 = peer != nullptr || (flags & NV4_GEMM_OUT_FP32) != 0;
  const bool use_a8 = a8 != nullptr;
  if (peer && (peer->world < 2 || peer->world > kPeerMaxRanks)) return NV4_ERR_UNSUPPORTED;
  StreamPlan pl;
  const int prc = plan_w4a4_stream(m, n, k, wg, sms, peer != nullptr, &pl);
  if (prc != NV4_OK) return prc;
  const int MT = pl.token_tiles, MP = MT * 8, G = static_cast<int>(k / 128);
  const int R = pl.rows_per_cta, stages = pl.stages, slabs = pl.slabs, ks = pl.k_split, tpw = pl.tiles_per_warp;
  const int smem = pl.smem_bytes;
  const bool scale_tma = (G % 8) == 0 && (reinterpret_cast<uintptr_t>(w_scale) & 15) == 0;

  CUtensorMap maps[3];
  memset(maps, 0, sizeof(maps));
  bool okm = make_tensor_map_u8(&maps[0], w_packed, n, k / 2, static_cast<uint32_t>(R), 128,
                                CU_TENSOR_MAP_SWIZZLE_128B);
  if (use_a8)
    okm = okm && make_tensor_map_u8(&maps[1], a8, m, k, static_cast<uint32_t>(MP), 128, CU_TENSOR_MAP_SWIZZLE_128B);
  else
    okm = okm && make_tensor_map_u8(&maps[1], a_packed, m, k / 2, static_cast<uint32_t>(MP), 128,
                                    CU_TENSOR_MAP_SWIZZLE_128B);
  if (scale_tma) {
    if (wg)
      okm = okm && make_map_u16(&maps[2], w_scale, n, G, static_cast<uint32_t>(R), G);
    else
      okm = okm && make_map_u16(&maps[2], w_scale, 1, n, 1, static_cast<uint32_t>(R));
  }
  if (!okm) return NV4_ERR_CUDA;

  StreamGemmArgs a;
  a.a_scale = static_cast<const uint16_t*>(a_scale);
  a.w_scale = static_cast<const uint16_t*>(w_scale);
  a.out = out;
  a.M = static_cast<int>(m);
  a.N = static_cast<int>(n);
  a.G = G;
  a.R = R;
  a.slabs = slabs;
  a.n_iters = pl.n_iters;
  a.stages = stages;
  a.scale_tma = scale_tma ? 1 : 0;
  const dim3 grid(static_cast<unsigned>(pl.grid_x), static_cast<unsigned>(pl.grid_y));
  for (int r = 0; r < kPeerMaxRanks; ++r) a.peer_bufs[r] = nullptr;
  a.peer_capacity = 0;
  a.peer_rank = 0;
  a.peer_world = 0;
  if (peer) {
    for (int r = 0; r < peer->world; ++r) a.peer_bufs[r] = static_cast<uint8_t*>(peer->bufs[r]);
    a.peer_capacity = peer->capacity;
    a.peer_rank = peer->rank;
    a.peer_world = peer->world;
    peer->rows_per_cta = R;
    peer->ctas = static_cast<int>(grid.x);
  }
  const int threads = pl.threads;
  switch (MT * 100 + tpw * 10 + ks) {
    case 111: return launch_flags<1, 1, 1>(maps, a, grid, threads, smem, use_a8, wg, f32, stream);
    case 114: return launch_flags<1, 1, 4>(maps, a, grid, threads, smem, use_a8, wg, f32, stream);
    case 211: return launch_flags<2, 1, 1>(maps, a, grid, threads, smem, use_a8, wg, f32, stream);
    case 221: return launch_flags<2, 2, 1>(maps, a, grid, threads, smem, use_a8, wg, f32, stream);
    case 224: return launch_flags<2, 2, 4>(maps, a, grid, threads, smem, use_a8, wg, f32, stream);
    case 411: return launch_flags<4, 1, 1>(maps, a, grid, threads, smem, use_a8, wg, f32, stream);
    case 421: return launch_flags<4, 2, 1>(maps, a, grid, threads, smem, use_a8, wg, f32, stream);
    case 441: return launch_flags<4, 4, 1>(maps, a, grid, threads, smem, use_a8, wg, f32, stream);
    case 424: return launch_flags<4, 2, 4>(maps, a, grid, threads, smem, use_a8, wg, f32, stream);
    case 444: return launch_flags<4, 4, 4>(maps, a, grid, threads, smem, use_a8, wg, f32, stream);
    default: return NV4_ERR_UNSUPPORTED;
  }
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
