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

int64_t w4a16_workspace_bytes(int64_t m, int64_t n, int64_t k) {
  const int sms = device_sm_count();
  if (sms <= 0) return 0;
  const W4A16Plan pl = plan_w4a16(m, n, k, sms);
  return pl.splits > 1 ? m * n * 4 : 0;
}

int launch_w4a16_gemm(const void* x, const void* qweight, const void* qzeros, const void* scales, void* out,
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
  // The shared launcher zeroes the first m * n floats before the split-K pass.
  return launch_w4a16_gemm(x, qweight, qzeros, scales, out, m, n, k, scratch,
                           kW4A16StaticScratchFloats * static_cast<int64_t>(sizeof(float)), stream);
}

}  // namespace nv4
