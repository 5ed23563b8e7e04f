// Kernel D: GPTQ W4A16 dequant GEMM, out[m, n] = x[m, k] @ W[k, n].
//
// Dequantisation is the reference's (nanovllm/layers/linear_w4a16.py:45-55):
// bf16(0x4300 | (w + 15 - z)) - 144 = w - z - 1 exactly, times the scale after
// rounding the FP16 scale to BF16, with one BF16 rounding of the product.  Here
// the nibble lands in a BF16 lane as 128 + w (bit trick), the subtraction of
// 129 + z is exact, and the product is one BF16x2 multiply, so the dequantised
// weight equals the reference's bit for bit.  The GEMM runs on BF16 tensor
// cores (mma.sync m16n8k16, FP32 accumulate).
//
// Operand permutation: within each 16-wide K block a thread reads one packed
// int32 (8 consecutive k of one column) and feeds nibble pairs (0,4),(1,5) or
// (2,6),(3,7) as its two BF16x2 B registers; the activation fragment applies
// the same permutation of k, which leaves every dot product unchanged.
//
// Split-K (grid.z > 1, used when the output tiles alone cannot fill the GPU)
// adds FP32 partials into the caller's workspace with atomics; a second kernel
// rounds it to BF16.  The reference instead adds BF16-rounded partials with
// BF16 atomics into a pre-zeroed output.
#include <cstring>

#include "nv4_device.cuh"
#include "nv4_launch.h"

namespace nv4 {

struct W4A16Args {
  const uint16_t* x;       // bf16 [M, K]
  const uint32_t* qw;      // int32 [K/8, N]
  const uint32_t* qz;      // int32 [K/128, N/8]
  const uint16_t* scales;  // fp16 [K/128, N]
  void* out;               // bf16 [M, N], or float [M, N] workspace when split
  int M, N, K;
  int groups_per_split;
};

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t bf16x2_sub(uint32_t a, uint32_t b) {
  __nv_bfloat162 r = __hsub2(*reinterpret_cast<__nv_bfloat162*>(&a), *reinterpret_cast<__nv_bfloat162*>(&b));
  return *reinterpret_cast<uint32_t*>(&r);
}

__device__ __forceinline__ uint32_t bf16x2_mul(uint32_t a, uint32_t b) {
  __nv_bfloat162 r = __hmul2(*reinterpret_cast<__nv_bfloat162*>(&a), *reinterpret_cast<__nv_bfloat162*>(&b));
  return *reinterpret_cast<uint32_t*>(&r);
}

// WM x WN warps; each warp owns MT m16 tiles x NT n8 tiles.
template <int WM, int WN, int MT, int NT, bool SPLIT>
__global__ void __launch_bounds__(128) w4a16_mma_kernel(const W4A16Args p) {
  static_assert(WM * WN == 4, "four warps");
  constexpr int BM = WM * MT * 16, BN = WN * NT * 8;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int wm = warp / WN, wn = warp % WN;
  const int gid = lane >> 2, tig = lane & 3;
  const int m_base = blockIdx.y * BM + wm * MT * 16;
  const int n_base = blockIdx.x * BN + wn * NT * 8;
  const int G = p.K / 128;
  const int g_begin = blockIdx.z * p.groups_per_split;
  const int g_end = min(G, g_begin + p.groups_per_split);

  float acc[MT][NT][4];
#pragma unroll
  for (int i = 0; i < MT; ++i)
#pragma unroll
    for (int j = 0; j < NT; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[i][j][e] = 0.0f;

  const int sel = (tig & 1) * 8;        // nibble pair shift inside the packed word
  const int half = tig >> 1;            // which of the two words of a 16-K block

  for (int g = g_begin; g < g_end; ++g) {
    // per-column zero point and BF16-rounded scale for this group
    uint32_t cz[NT], s2[NT];
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      const int n = min(n_base + j * 8 + gid, p.N - 1);  // tiles past N compute on a valid column, store nothing
      const uint32_t zw = p.qz[static_cast<size_t>(g) * (p.N / 8) + (n >> 3)];
      const uint32_t z = (zw >> (4 * (n & 7))) & 15u;
      const uint32_t czb = __bfloat16_as_ushort(__float2bfloat16_rn(static_cast<float>(129u + z)));
      cz[j] = czb | (czb << 16);
      const __half h = __ushort_as_half(p.scales[static_cast<size_t>(g) * p.N + n]);
      const uint32_t sb = __bfloat16_as_ushort(__float2bfloat16_rn(__half2float(h)));
      s2[j] = sb | (sb << 16);
    }
#pragma unroll 2
    for (int kb = 0; kb < 8; ++kb) {
      const int k0 = g * 128 + kb * 16;
      uint32_t wq[NT];
#pragma unroll
      for (int j = 0; j < NT; ++j)
        wq[j] = __ldg(p.qw + static_cast<size_t>(k0 / 8 + half) * p.N + min(n_base + j * 8 + gid, p.N - 1));
      uint32_t af[MT][4];
#pragma unroll
      for (int i = 0; i < MT; ++i) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int row = m_base + i * 16 + gid + h * 8;
          uint4 v = make_uint4(0, 0, 0, 0);
          if (row < p.M) v = __ldg(reinterpret_cast<const uint4*>(p.x + static_cast<size_t>(row) * p.K + k0 + half * 8));
          const uint32_t u_lo = (tig & 1) ? v.y : v.x, u_hi = (tig & 1) ? v.w : v.z;
          af[i][h] = __byte_perm(u_lo, u_hi, 0x5410);      // k pair (0,4) or (2,6)
          af[i][h + 2] = __byte_perm(u_lo, u_hi, 0x7632);  // k pair (1,5) or (3,7)
        }
      }
#pragma unroll
      for (int j = 0; j < NT; ++j) {
        const uint32_t w = wq[j] >> sel;
        const uint32_t b0 = bf16x2_mul(bf16x2_sub((w & 0x000F000Fu) | 0x43004300u, cz[j]), s2[j]);
        const uint32_t b1 = bf16x2_mul(bf16x2_sub(((w >> 4) & 0x000F000Fu) | 0x43004300u, cz[j]), s2[j]);
#pragma unroll
        for (int i = 0; i < MT; ++i) mma_bf16_16816(acc[i][j], af[i], b0, b1);
      }
    }
  }

#pragma unroll
  for (int i = 0; i < MT; ++i)
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      const int n = n_base + j * 8 + tig * 2;
      if (n >= p.N) continue;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int row = m_base + i * 16 + gid + h * 8;
        if (row >= p.M) continue;
        const size_t o = static_cast<size_t>(row) * p.N + n;
        if (SPLIT) {
          atomicAdd(static_cast<float*>(p.out) + o, acc[i][j][2 * h]);
          atomicAdd(static_cast<float*>(p.out) + o + 1, acc[i][j][2 * h + 1]);
        } else {
          *reinterpret_cast<__nv_bfloat162*>(static_cast<__nv_bfloat16*>(p.out) + o) =
              __floats2bfloat162_rn(acc[i][j][2 * h], acc[i][j][2 * h + 1]);
        }
      }
    }
}

__global__ void f32_to_bf16_kernel(const float* __restrict__ src, __nv_bfloat16* __restrict__ dst, int64_t count) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < count; i += int64_t(gridDim.x) * blockDim.x)
    dst[i] = __float2bfloat16_rn(src[i]);
}

// Tile and split choice shared by the workspace query and the launcher.
struct W4A16Plan {
  bool small;  // decode tiles (16 x 128) vs prefill tiles (64 x 64)
  int bm, bn, splits, groups_per_split;
};

static W4A16Plan plan_w4a16(int64_t m, int64_t n, int64_t k, int sms) {
  W4A16Plan pl;
  pl.small = m <= 16;
  pl.bm = pl.small ? 16 : 64;
  pl.bn = pl.small ? 128 : 64;
  const int64_t tiles = ((n + pl.bn - 1) / pl.bn) * ((m + pl.bm - 1) / pl.bm);
  const int G = static_cast<int>(k / 128);
  int splits = 1;
  if (pl.small && tiles < 2 * sms) splits = static_cast<int>(std::min<int64_t>(G, (2 * sms + tiles - 1) / tiles));
  pl.groups_per_split = (G + splits - 1) / splits;
  pl.splits = (G + pl.groups_per_split - 1) / pl.groups_per_split;
  return pl;
}

static int64_t w4a16_mma_workspace_bytes(int64_t m, int64_t n, int64_t k, int sms) {
  const W4A16Plan pl = plan_w4a16(m, n, k, sms);
  return pl.splits > 1 ? m * n * 4 : 0;
}

// The mma.sync kernel, split-K partials added into `workspace` with FP32
// atomics and rounded by a second kernel (the path of the allocation-free
// entry point, and of shapes Kernel D1 does not plan).
static int launch_w4a16_mma(const void* x, const void* qweight, const void* qzeros, const void* scales, void* out,
                      int64_t m, int64_t n, int64_t k, void* workspace, int64_t workspace_bytes, cudaStream_t stream) {
  const int sms = device_sm_count();
  if (sms <= 0) return NV4_ERR_CUDA;
  const W4A16Plan pl = plan_w4a16(m, n, k, sms);
  W4A16Args a;
  a.x = static_cast<const uint16_t*>(x);
  a.qw = static_cast<const uint32_t*>(qweight);
  a.qz = static_cast<const uint32_t*>(qzeros);
  a.scales = static_cast<const uint16_t*>(scales);
  a.M = static_cast<int>(m);
  a.N = static_cast<int>(n);
  a.K = static_cast<int>(k);
  a.groups_per_split = pl.groups_per_split;
  const dim3 grid(static_cast<unsigned>((n + pl.bn - 1) / pl.bn), static_cast<unsigned>((m + pl.bm - 1) / pl.bm),
                  static_cast<unsigned>(pl.splits));
  if (pl.splits > 1) {
    if (workspace == nullptr || workspace_bytes < m * n * 4) return NV4_ERR_INVALID_ARGUMENT;
    cudaError_t e = cudaMemsetAsync(workspace, 0, static_cast<size_t>(m * n * 4), stream);
    if (e != cudaSuccess) {
      set_last_cuda_error(e);
      return NV4_ERR_CUDA;
    }
    a.out = workspace;
    int rc = launch_kernel(w4a16_mma_kernel<1, 4, 1, 4, true>, grid, dim3(128), 0, stream, false, a);
    if (rc != NV4_OK) return rc;
    const int64_t count = m * n;
    const int blocks = static_cast<int>(std::min<int64_t>((count + 255) / 256, 8 * sms));
    return launch_kernel(f32_to_bf16_kernel, dim3(blocks), dim3(256), 0, stream, false,
                         static_cast<const float*>(workspace), static_cast<__nv_bfloat16*>(out), count);
  }
  a.out = out;
  if (pl.small) return launch_kernel(w4a16_mma_kernel<1, 4, 1, 4, false>, grid, dim3(128), 0, stream, false, a);
  return launch_kernel(w4a16_mma_kernel<2, 2, 2, 4, false>, grid, dim3(128), 0, stream, false, a);
}

// ------------------------------------------------------------ Kernel D1: decode
// W4A16 for up to 16 tokens: the weights are the streamed operand.  A CTA
// owns 64 output columns and a K slice; the KS CTAs of one column block form
// a thread-block cluster along K (split-K, the reference's SPLIT_K for small
// M), and their FP32 partial tiles are summed through distributed shared
// memory in cluster-rank order -- no workspace, no atomics, no second kernel.
//
//  * The CTA's packed weights [K_slice/8 rows][64 columns] of int32 arrive by
//    2-D TMA in chunks of 32 rows (256 K, two groups), one mbarrier each, so
//    compute starts on the first chunk while the rest stream in.
//  * Activations [M, K_slice] are read once with 16-byte loads, their K order
//    permuted inside every 8-wide block to (0,4,1,5,2,6,3,7), and stored in
//    shared memory; ldmatrix then yields MMA A fragments whose K pairs match
//    the nibble pairs (j, j+4) that one shift and mask pull out of a packed
//    word (a consistent K permutation of both operands leaves every dot
//    product unchanged).
//  * mma.sync m16n8k16 BF16 with tokens as M (one 16-row tile) and weight
//    columns as N: warp w owns columns 16w .. 16w+15.
//  * From 17 tokens on, Kernel D2 (tcgen05, K split over the SMs) is faster
//    at every config-3 shape: a second 16-row tile doubles this kernel's
//    activation footprint and halves its CTAs per SM (at 32 tokens gate/up
//    73.6 us and down 64.5 us here against 58.2 us and 30.6 us there).
//  * Dequantisation as the reference (nanovllm/layers/linear_w4a16.py:45-55):
//    bf16(128 + w) - bf16(129 + z) = w - z - 1 exactly, times the BF16-rounded
//    FP16 scale with one BF16 rounding (BF16x2 subtract and multiply).
struct W4A16StreamArgs {
  const uint16_t* x;       // bf16 [M, K]
  const uint32_t* qz;      // int32 [K/128, N/8]
  const uint16_t* scales;  // fp16 [K/128, N]
  uint16_t* out;           // bf16 [M, N]
  int M, N, K;
  int k_slice;             // K of one CTA (a multiple of 256)
  int chunks;              // k_slice / 256 TMA chunks
  int x_stride;            // shared-memory row stride of the activations, bytes
};

constexpr int kW4A16StreamCols = 64;
constexpr int kW4A16ChunkRows = 32;  // k8 rows per TMA chunk (256 K)
constexpr int kW4A16MaxChunks = 8;

// Shared memory: the CTA's packed weights, its `rows` activation rows plus one
// zero row (the MMA's padding rows past M all read it), per-(group, column)
// zero/scale pairs, the FP32 partial tile, the chunk barriers.
struct W4A16StreamLayout {
  int wq_off, x_off, sz_off, red_off, bar_off, total;
  __host__ __device__ W4A16StreamLayout(int k_slice, int rows, int x_stride) {
    wq_off = 0;
    x_off = wq_off + (k_slice / 8) * kW4A16StreamCols * 4;
    sz_off = x_off + (rows + 1) * x_stride;
    red_off = sz_off + (k_slice / 128) * kW4A16StreamCols * 8;
    bar_off = red_off + rows * kW4A16StreamCols * 4;
    total = bar_off + kW4A16MaxChunks * 8;
  }
};

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ float ld_dsmem_f32(uint32_t local_addr, uint32_t rank) {
  uint32_t remote;
  float v;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local_addr), "r"(rank));
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(remote) : "memory");
  return v;
}

template <int MT>
__global__ void __launch_bounds__(128) w4a16_stream_kernel(const __grid_constant__ CUtensorMap tmap_qw,
                                                           const W4A16StreamArgs p) {
  extern __shared__ __align__(128) uint8_t smem_w16[];
  const int rows = min(p.M, MT * 16);  // activation rows held (the rest of the MMA's M is padding)
  const W4A16StreamLayout L(p.k_slice, rows, p.x_stride);
  uint32_t* wq = reinterpret_cast<uint32_t*>(smem_w16 + L.wq_off);
  uint8_t* xs = smem_w16 + L.x_off;
  uint2* sz = reinterpret_cast<uint2*>(smem_w16 + L.sz_off);  // [group][column]: (129+z, scale) as BF16x2
  float* red = reinterpret_cast<float*>(smem_w16 + L.red_off);  // [MT*16][64]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem_w16 + L.bar_off);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gid = lane >> 2, tig = lane & 3;
  const int n0 = blockIdx.x * kW4A16StreamCols;
  const int ks = blockIdx.y, KS = gridDim.y;
  const int k0 = ks * p.k_slice;
  const int G = p.k_slice / 128;

  grid_dependents_launch();
  if (threadIdx.x == 0) {
    for (int c = 0; c < p.chunks; ++c) mbar_init(&bars[c], 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmap_qw);
    const uint64_t pol = policy_evict_first();
    for (int c = 0; c < p.chunks; ++c) {
      mbar_arrive_expect_tx(&bars[c], kW4A16ChunkRows * kW4A16StreamCols * 4);
      tma_load_2d_hint(wq + c * kW4A16ChunkRows * kW4A16StreamCols, &tmap_qw, &bars[c], n0,
                       k0 / 8 + c * kW4A16ChunkRows, pol);
    }
  }

  // Per-(group, column) zero point 129 + z and BF16-rounded scale as BF16x2
  // pairs.  They do not depend on the preceding kernel, so they load before
  // griddepcontrol.wait; every load of a thread is issued before any is used.
  {
    constexpr int kMaxPerThread = (kW4A16MaxChunks * 2 * kW4A16StreamCols) / 128;
    uint32_t zw[kMaxPerThread];
    uint16_t sh[kMaxPerThread];
    const int total = G * kW4A16StreamCols;
#pragma unroll
    for (int u = 0; u < kMaxPerThread; ++u) {
      const int i = threadIdx.x + u * 128;
      if (i < total) {
        const int g = i / kW4A16StreamCols, n = n0 + (i - g * kW4A16StreamCols), gg = k0 / 128 + g;
        zw[u] = __ldg(p.qz + static_cast<size_t>(gg) * (p.N / 8) + (n >> 3));
        sh[u] = __ldg(p.scales + static_cast<size_t>(gg) * p.N + n);
      }
    }
#pragma unroll
    for (int u = 0; u < kMaxPerThread; ++u) {
      const int i = threadIdx.x + u * 128;
      if (i < total) {
        const int n = n0 + (i % kW4A16StreamCols);
        const uint32_t z = (zw[u] >> (4 * (n & 7))) & 15u;
        const uint32_t zb = __bfloat16_as_ushort(__float2bfloat16_rn(static_cast<float>(129u + z)));
        const uint32_t sb = __bfloat16_as_ushort(__float2bfloat16_rn(__half2float(__ushort_as_half(sh[u]))));
        sz[i] = make_uint2(zb | (zb << 16), sb | (sb << 16));
      }
    }
  }
  grid_dependency_wait();  // the activations come from the preceding kernel
  // Activations, K-permuted within each 8-block, and the zero row.  Loads go
  // out in batches of 8 per thread before their stores.
  {
    const int vec_per_row = p.k_slice / 8;
    for (int v = threadIdx.x; v < vec_per_row; v += blockDim.x)
      *reinterpret_cast<uint4*>(xs + rows * p.x_stride + v * 16) = make_uint4(0, 0, 0, 0);
    const int total = rows * vec_per_row;
    for (int i0 = threadIdx.x; i0 < total; i0 += 8 * 128) {
      uint4 u[8];
#pragma unroll
      for (int b = 0; b < 8; ++b) {
        const int i = i0 + b * 128;
        const int row = i / vec_per_row, v = i - row * vec_per_row;
        u[b] = make_uint4(0, 0, 0, 0);
        if (i < total)
          u[b] = __ldg(reinterpret_cast<const uint4*>(p.x + static_cast<size_t>(row) * p.K + k0) + v);
      }
#pragma unroll
      for (int b = 0; b < 8; ++b) {
        const int i = i0 + b * 128;
        if (i >= total) break;
        const int row = i / vec_per_row, v = i - row * vec_per_row;
        uint4 o;
        o.x = __byte_perm(u[b].x, u[b].z, 0x5410);  // (k0, k4)
        o.y = __byte_perm(u[b].x, u[b].z, 0x7632);  // (k1, k5)
        o.z = __byte_perm(u[b].y, u[b].w, 0x5410);  // (k2, k6)
        o.w = __byte_perm(u[b].y, u[b].w, 0x7632);  // (k3, k7)
        *reinterpret_cast<uint4*>(xs + row * p.x_stride + v * 16) = o;
      }
    }
  }
  __syncthreads();

  float acc[MT][2][4];
#pragma unroll
  for (int i = 0; i < MT; ++i)
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[i][j][e] = 0.0f;

  // ldmatrix row address of this lane for each 16-row M tile (padding rows
  // read the zero row), and the shared-memory words of its two columns.
  uint32_t xaddr[MT];
#pragma unroll
  for (int i = 0; i < MT; ++i) {
    const int r = i * 16 + (lane & 15);
    xaddr[i] = smem_u32(xs) + (r < rows ? r : rows) * p.x_stride + (lane >> 4) * 16;
  }
  const int col0 = warp * 16 + gid;  // columns col0 and col0 + 8
  const uint32_t* wcol = wq + col0;
  const int shift = 4 * tig;
  bool ok = true;
  for (int c = 0; c < p.chunks; ++c) {
    if (ok) ok = mbar_wait(&bars[c], 0, kErrTimeoutFull);
    if (!ok) break;
    const uint32_t* wc = wcol + c * kW4A16ChunkRows * kW4A16StreamCols;
    const uint32_t xc = c * 512;  // byte offset of the chunk's 256 K in an activation row
#pragma unroll
    for (int gl = 0; gl < 2; ++gl) {  // two groups per chunk
      const uint2 zs0 = sz[(c * 2 + gl) * kW4A16StreamCols + col0];
      const uint2 zs1 = sz[(c * 2 + gl) * kW4A16StreamCols + col0 + 8];
#pragma unroll
      for (int kb = 0; kb < 8; ++kb) {
        const int step = gl * 8 + kb;  // 16-K step within the chunk
        uint32_t a[MT][4];
#pragma unroll
        for (int i = 0; i < MT; ++i) ldmatrix_x4(xaddr[i] + xc + step * 32, a[i][0], a[i][1], a[i][2], a[i][3]);
        const uint32_t w00 = wc[(2 * step) * kW4A16StreamCols] >> shift;
        const uint32_t w01 = wc[(2 * step + 1) * kW4A16StreamCols] >> shift;
        const uint32_t w10 = wc[(2 * step) * kW4A16StreamCols + 8] >> shift;
        const uint32_t w11 = wc[(2 * step + 1) * kW4A16StreamCols + 8] >> shift;
        const uint32_t b00 = bf16x2_mul(bf16x2_sub((w00 & 0x000F000Fu) | 0x43004300u, zs0.x), zs0.y);
        const uint32_t b01 = bf16x2_mul(bf16x2_sub((w01 & 0x000F000Fu) | 0x43004300u, zs0.x), zs0.y);
        const uint32_t b10 = bf16x2_mul(bf16x2_sub((w10 & 0x000F000Fu) | 0x43004300u, zs1.x), zs1.y);
        const uint32_t b11 = bf16x2_mul(bf16x2_sub((w11 & 0x000F000Fu) | 0x43004300u, zs1.x), zs1.y);
#pragma unroll
        for (int i = 0; i < MT; ++i) {
          mma_bf16_16816(acc[i][0], a[i], b00, b01);
          mma_bf16_16816(acc[i][1], a[i], b10, b11);
        }
      }
    }
  }

  // C fragment: (row gid, columns 2tig, 2tig+1) and row gid + 8
  if (KS == 1) {
    if (ok) {
#pragma unroll
      for (int i = 0; i < MT; ++i)
#pragma unroll
        for (int j = 0; j < 2; ++j)
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int row = i * 16 + gid + h * 8;
            if (row < p.M)
              *reinterpret_cast<__nv_bfloat162*>(p.out + static_cast<size_t>(row) * p.N + n0 + warp * 16 + j * 8 + 2 * tig) =
                  __floats2bfloat162_rn(acc[i][j][2 * h], acc[i][j][2 * h + 1]);
          }
    }
  } else {
#pragma unroll
    for (int i = 0; i < MT; ++i)
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int row = i * 16 + gid + h * 8;
          if (row < rows)
            *reinterpret_cast<float2*>(red + row * kW4A16StreamCols + warp * 16 + j * 8 + 2 * tig) =
                make_float2(acc[i][j][2 * h], acc[i][j][2 * h + 1]);
        }
    cluster_sync_all();
    // this CTA sums its share of the columns over the cluster's ranks, in rank order
    const int share = kW4A16StreamCols / KS, c_begin = static_cast<int>(cluster_rank()) * share;
    const uint32_t red_base = smem_u32(red);
    for (int i = threadIdx.x; i < p.M * share; i += blockDim.x) {
      const int row = i / share, col = c_begin + (i - row * share);
      const uint32_t addr = red_base + (row * kW4A16StreamCols + col) * 4;
      float v[8];
#pragma unroll
      for (int r = 0; r < 8; ++r) v[r] = r < KS ? ld_dsmem_f32(addr, r) : 0.0f;  // all loads before the sum
      float s = v[0];
#pragma unroll
      for (int r = 1; r < 8; ++r)
        if (r < KS) s = __fadd_rn(s, v[r]);
      p.out[static_cast<size_t>(row) * p.N + n0 + col] = __bfloat16_as_ushort(__float2bfloat16_rn(s));
    }
    cluster_sync_all();  // no CTA leaves while a peer may still read its partials
  }
  if (!ok && threadIdx.x == 0)  // let every copy this CTA issued land before it exits
    for (int c = 0; c < p.chunks; ++c) mbar_wait_drain(&bars[c], 0);
}

// Launch plan of Kernel D1: K split, in powers of two up to the portable
// cluster size of 8, until the grid reaches about three CTAs per SM and a CTA's
// K slice is at most 1024 (its weights and activations then fit several CTAs
// per SM, so one CTA's loads overlap another's math).
struct W4A16StreamPlan {
  int ks, k_slice, x_stride, smem;
};

constexpr int64_t kW4A16StreamMaxM = 16;  // tokens Kernel D1 takes (one MMA tile)

static bool plan_w4a16_stream(int64_t m, int64_t n, int64_t k, int sms, W4A16StreamPlan* out) {
  if (m > kW4A16StreamMaxM || n % kW4A16StreamCols || k % 256) return false;
  const int64_t tiles = n / kW4A16StreamCols;
  int ks = 1;
  while (ks < 8 && (tiles * ks < 3 * static_cast<int64_t>(sms) || k / ks > 1024) && (k / (2 * ks)) % 256 == 0)
    ks *= 2;
  W4A16StreamPlan pl;
  pl.ks = ks;
  pl.k_slice = static_cast<int>(k / ks);
  if (pl.k_slice / 256 > kW4A16MaxChunks) return false;
  pl.x_stride = pl.k_slice * 2 + 16;  // 16 bytes of padding: conflict-free ldmatrix rows
  const W4A16StreamLayout L(pl.k_slice, static_cast<int>(m), pl.x_stride);
  pl.smem = L.total;
  if (pl.smem > 227 * 1024) return false;
  *out = pl;
  return true;
}

template <int MT>
static int launch_w4a16_stream_t(const CUtensorMap& map, const W4A16StreamArgs& a, const W4A16StreamPlan& pl,
                                 int64_t n, cudaStream_t stream) {
  static int done[64] = {};
  auto* kern = &w4a16_stream_kernel<MT>;
  int rc = ensure_smem_attr(reinterpret_cast<const void*>(kern), pl.smem, done);
  if (rc != NV4_OK) return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(n / kW4A16StreamCols), static_cast<unsigned>(pl.ks));
  cfg.blockDim = dim3(128);
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = static_cast<unsigned>(pl.ks);
  attr[0].val.clusterDim.z = 1;
  // programmatic dependent launch: weights, scales and zero points load while
  // the preceding kernel drains; the activations only after griddepcontrol.wait
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, map, a);
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return NV4_ERR_CUDA;
  }
  return NV4_OK;
}

static int launch_w4a16_stream(const void* x, const void* qweight, const void* qzeros, const void* scales, void* out,
                               int64_t m, int64_t n, int64_t k, const W4A16StreamPlan& pl, cudaStream_t stream) {
  CUtensorMap map;
  memset(&map, 0, sizeof(map));
  if (!make_tensor_map_2d(&map, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, qweight, static_cast<uint64_t>(k / 8),
                          static_cast<uint64_t>(n), kW4A16ChunkRows, kW4A16StreamCols, CU_TENSOR_MAP_SWIZZLE_NONE))
    return NV4_ERR_CUDA;
  W4A16StreamArgs a;
  a.x = static_cast<const uint16_t*>(x);
  a.qz = static_cast<const uint32_t*>(qzeros);
  a.scales = static_cast<const uint16_t*>(scales);
  a.out = static_cast<uint16_t*>(out);
  a.M = static_cast<int>(m);
  a.N = static_cast<int>(n);
  a.K = static_cast<int>(k);
  a.k_slice = pl.k_slice;
  a.chunks = pl.k_slice / 256;
  a.x_stride = pl.x_stride;
  return launch_w4a16_stream_t<1>(map, a, pl, n, stream);
}

int64_t w4a16_workspace_bytes(int64_t m, int64_t n, int64_t k) {
  const int sms = device_sm_count();
  if (sms <= 0) return 0;
  W4A16StreamPlan sp;
  if (plan_w4a16_stream(m, n, k, sms, &sp)) return 0;
  if (m > kW4A16StreamMaxM)
    return std::max(w4a16_tc_workspace_bytes(m, n, k), w4a16_mma_workspace_bytes(m, n, k, sms));
  return w4a16_mma_workspace_bytes(m, n, k, sms);
}

// The dispatch of launch_w4a16_gemm below for 16-byte aligned operands and a
// workspace of w4a16_workspace_bytes, on `sms` SMs, as plain numbers: kernel
// (1 decode stream, 2 tcgen05, 0 mma.sync), K splits, token tile, CTAs,
// workspace bytes.
void w4a16_plan(int64_t m, int64_t n, int64_t k, int sms, int64_t* plan) {
  W4A16StreamPlan sp;
  int bn = 0, splits = 1;
  if (plan_w4a16_stream(m, n, k, sms, &sp)) {
    const int64_t v[5] = {1, sp.ks, 16, (n / kW4A16StreamCols) * sp.ks, 0};
    for (int i = 0; i < 5; ++i) plan[i] = v[i];
  } else if (m > kW4A16StreamMaxM && w4a16_tc_plan(m, n, k, sms, &bn, &splits)) {
    const int64_t units = ((n + 127) / 128) * ((m + bn - 1) / bn) * splits;
    const int64_t v[5] = {2, splits, bn, std::min<int64_t>(units, sms),
                          splits > 1 ? splits * m * n * static_cast<int64_t>(sizeof(float)) : 0};
    for (int i = 0; i < 5; ++i) plan[i] = v[i];
  } else {
    const W4A16Plan pl = plan_w4a16(m, n, k, sms);
    const int64_t v[5] = {0, pl.splits, pl.bm, ((n + pl.bn - 1) / pl.bn) * ((m + pl.bm - 1) / pl.bm) * pl.splits,
                          pl.splits > 1 ? m * n * static_cast<int64_t>(sizeof(float)) : 0};
    for (int i = 0; i < 5; ++i) plan[i] = v[i];
  }
}

// Up to 16 tokens: Kernel D1 (no workspace); more: Kernel D2 (tcgen05, split-K
// partials in the workspace when its plan splits); shapes neither takes: the
// mma.sync kernel.
int launch_w4a16_gemm(const void* x, const void* qweight, const void* qzeros, const void* scales, void* out,
                      int64_t m, int64_t n, int64_t k, void* workspace, int64_t workspace_bytes, cudaStream_t stream) {
  const int sms = device_sm_count();
  if (sms <= 0) return NV4_ERR_CUDA;
  W4A16StreamPlan sp;
  if (plan_w4a16_stream(m, n, k, sms, &sp) && (reinterpret_cast<uintptr_t>(qweight) & 15) == 0)
    return launch_w4a16_stream(x, qweight, qzeros, scales, out, m, n, k, sp, stream);
  if (m > kW4A16StreamMaxM) {
    const int rc = launch_w4a16_tc_gemm(x, qweight, qzeros, scales, out, m, n, k, workspace, workspace_bytes, stream);
    if (rc != NV4_ERR_UNSUPPORTED) return rc;
  }
  return launch_w4a16_mma(x, qweight, qzeros, scales, out, m, n, k, workspace, workspace_bytes, stream);
}

}  // namespace nv4

// ---- Allocation-free variant (nv4_w4a16_gemm_static) -----------------------
// The split-K partials go to this fixed array instead of a caller workspace.
// Static device memory is set up when the library's module loads, so a call
// that uses it allocates nothing.  One array per device; calls that overlap in
// time on one device race on it (documented at the C entry point).
#include <atomic>
#include <mutex>

namespace nv4 {

constexpr int64_t kW4A16StaticScratchFloats = NV4_W4A16_STATIC_SCRATCH_FLOATS;
constexpr int64_t kW4A16SplitMaxM = 16;  // plan_w4a16: split-K only for m <= 16

static __device__ __align__(256) float g_w4a16_static_scratch[kW4A16StaticScratchFloats];

// Device address of the scratch array on the current device, looked up once
// per device (with that device current) and cached.
static int w4a16_static_scratch(float** ptr) {
  constexpr int kDevices = 64;
  static std::atomic<float*> cache[kDevices];
  static std::mutex mu;
  const int dev = current_device();
  if (dev < 0 || dev >= kDevices) return NV4_ERR_CUDA;
  float* p = cache[dev].load(std::memory_order_acquire);
  if (p == nullptr) {
    std::lock_guard<std::mutex> lock(mu);
    p = cache[dev].load(std::memory_order_relaxed);
    if (p == nullptr) {
      void* addr = nullptr;
      const cudaError_t e = cudaGetSymbolAddress(&addr, g_w4a16_static_scratch);
      if (e != cudaSuccess) {
        set_last_cuda_error(e);
        return NV4_ERR_CUDA;
      }
      p = static_cast<float*>(addr);
      cache[dev].store(p, std::memory_order_release);
    }
  }
  *ptr = p;
  return NV4_OK;
}

// True when (m, n) fits the scratch: m > 16 never splits K, m <= 16 may.
bool w4a16_static_fits(int64_t m, int64_t n) {
  return m > kW4A16SplitMaxM || m * n <= kW4A16StaticScratchFloats;
}

int launch_w4a16_gemm_static(const void* x, const void* qweight, const void* qzeros, const void* scales, void* out,
                             int64_t m, int64_t n, int64_t k, cudaStream_t stream) {
  float* scratch = nullptr;
  const int rc = w4a16_static_scratch(&scratch);
  if (rc != NV4_OK) return rc;
  // The mma.sync launcher zeroes the first m * n floats before the split-K pass.
  return launch_w4a16_mma(x, qweight, qzeros, scales, out, m, n, k, scratch,
                           kW4A16StaticScratchFloats * static_cast<int64_t>(sizeof(float)), stream);
}

}  // namespace nv4
