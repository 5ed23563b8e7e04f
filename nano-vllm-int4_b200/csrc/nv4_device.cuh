// Device-side building blocks shared by the nv4 kernels (sm_100a only).
//
// Everything here is a thin wrapper over one PTX instruction (mbarrier, bulk
// tensor copy, grid-dependency control, ldmatrix, mma.sync, tcgen05) plus the
// exact FP32 constants the quantizer semantics need.  Every spin-wait is
// bounded by %globaltimer: when a wait gives up it records an error word that
// the host can read with nv4_device_error(), and the kernel returns instead of
// hanging the GPU.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace nv4 {

// ----------------------------------------------------------------- constants
// Exact float32 values (hex literals): fl32(sqrt(128)), fl32(1/sqrt(12)),
// fl32(1/7), fl32(0.9) and the BF16 "tiny" (2^-126).
constexpr float kSqrt128 = 0x1.6a09e6p+3f;
constexpr float kInvSqrt12 = 0x1.279a74p-2f;
constexpr float kInv7 = 0x1.24924ap-3f;
constexpr float kClip = 0x1.ccccccp-1f;
constexpr float kBf16Tiny = 0x1.0p-126f;
// 1.5 * 2^23: adding an integer |v| < 2^22 to this float's bit pattern gives the
// float 12582912 + v exactly.
constexpr int kMagicBits = 0x4B400000;
constexpr float kMagic = 12582912.0f;

// Error words written by bounded waits (one per device, read/cleared by host).
enum DeviceError : int {
  kErrNone = 0,
  kErrTimeoutFull = 1,      // consumer waited too long for a loaded stage
  kErrTimeoutEmpty = 2,     // producer waited too long for a free stage
  kErrTimeoutMma = 3,       // tensor-core pipeline wait timed out
  kErrTimeoutDrain = 4,     // wait for in-flight copies at exit timed out
};

// Defined here: the library is one translation unit (nv4_unity.cu).
__device__ int g_device_error = 0;

__device__ __forceinline__ void record_error(int code) {
  atomicCAS(&g_device_error, 0, code);
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// A wait longer than this is a bug, not a slow GPU: record and bail out.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

__device__ __forceinline__ bool error_raised() {
  return *((volatile int*)&g_device_error) != 0;
}

// ----------------------------------------------------------------- bf16 bits
__device__ __forceinline__ float bf16lo_to_f32(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16hi_to_f32(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
__device__ __forceinline__ float bf16_bits_to_f32(uint16_t b) { return __uint_as_float(uint32_t(b) << 16); }

// ----------------------------------------------------------------- smem addr
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ----------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait on an mbarrier phase.  Returns false (and records `err`) when
// the phase did not complete within kWaitLimitNs or another CTA already
// reported an error.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int err) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = global_timer_ns();
  uint32_t spins = 0;
  while (!mbar_try_wait(bar, parity)) {
    if ((++spins & 255u) == 0) {
      if (error_raised()) return false;
      if (global_timer_ns() - start > kWaitLimitNs) {
        record_error(err);
        return false;
      }
    }
  }
  return true;
}

// ----------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 2-D tiled bulk tensor copy global -> shared, completion signalled on `bar`.
// (x, y) are element coordinates; x must be a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void tma_load_2d_hint(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y,
                                                 uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y),
      "l"(policy)
      : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// ----------------------------------------------------------------- PDL
// Programmatic dependent launch: the consumer kernel starts while its
// producer finishes and waits here before touching the producer's output.
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dependents_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ----------------------------------------------------------------- named barrier
__device__ __forceinline__ void named_barrier_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ----------------------------------------------------------------- ldmatrix / mma.sync
__device__ __forceinline__ void ldmatrix_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// D = A(16x64 s4, row) * B(64x8 s4, col) + C, INT32 accumulate.
__device__ __forceinline__ void mma_s4_16864(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k64.row.col.s32.s4.s4.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Byte offset of 16-byte chunk `chunk` (0..7) of row `row` in a 128-byte-row
// tile written by TMA with CU_TENSOR_MAP_SWIZZLE_128B (1024-byte aligned tile).
__device__ __forceinline__ uint32_t sw128_offset(uint32_t row, uint32_t chunk) {
  return row * 128u + ((chunk ^ (row & 7u)) << 4);
}

}  // namespace nv4
