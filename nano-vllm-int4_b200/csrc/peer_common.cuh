// Layout of a tensor-parallel peer buffer and the device primitives of the
// peer-memory exchange (used by the one-shot all-reduce and by the row-parallel
// GEMM that stores its tiles straight into the peers' inboxes).
//
//   header  [NV4_PEER_HEADER_BYTES]
//             flag[sender][slot]  uint32, kPeerMaxRanks x kPeerSlots
//             epoch[slot]         uint32, kPeerSlots (this rank's call count)
//   partial [capacity] FP32       this rank's partial (two-kernel path)
//   inbox   [2][kPeerMaxRanks][capacity] FP32: slot (parity, sender) holds that
//           sender's partial of a call with epoch parity `parity`
//
// Epochs: every call advances all kPeerSlots counters by one (a kernel's CTA s
// advances slot s, its CTA 0 the slots beyond its grid), so all slots hold the
// call count and the inbox parity is the same for every slot of a call.
// Kernels touch the counters only after griddepcontrol.wait, so under
// programmatic dependent launch the updates stay in stream order.  A sender
// publishes data for slot s of a call by storing the call's epoch into
// flag[sender][s] of the receiver with a system-scope release; the receiver
// polls its own flags with acquire loads.  A rank can be at most one call ahead
// of a peer (it waits for the peer's data of every call), so two inbox
// parities keep a sender from overwriting data a receiver has not read.
#pragma once

#include "nv4_device.cuh"

namespace nv4 {

constexpr int kPeerMaxRanks = 8;
constexpr int kPeerSlots = 256;
constexpr int kPeerHeaderBytes = NV4_PEER_HEADER_BYTES;
constexpr int kErrTimeoutPeer = 5;  // a peer rank did not reach the same call in time
static_assert((kPeerMaxRanks + 1) * kPeerSlots * 4 <= kPeerHeaderBytes, "peer header too small");

__device__ __forceinline__ uint32_t* peer_flags(uint8_t* buf) { return reinterpret_cast<uint32_t*>(buf); }
__device__ __forceinline__ uint32_t* peer_epochs(uint8_t* buf) {
  return reinterpret_cast<uint32_t*>(buf) + kPeerMaxRanks * kPeerSlots;
}
__device__ __forceinline__ float* peer_partial(uint8_t* buf) {
  return reinterpret_cast<float*>(buf + kPeerHeaderBytes);
}
__device__ __forceinline__ float* peer_inbox(uint8_t* buf, int64_t capacity, int parity, int sender) {
  return peer_partial(buf) + capacity * (1 + parity * kPeerMaxRanks + sender);
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ float4 ld_volatile_f4(const float* p) {
  float4 v;
  asm volatile("ld.volatile.global.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(p));
  return v;
}
__device__ __forceinline__ float ld_volatile_f(const float* p) {
  float v;
  asm volatile("ld.volatile.global.f32 %0, [%1];" : "=f"(v) : "l"(p));
  return v;
}

// Bounded wait until the flag reaches `epoch` (wrap-safe); false (and an error
// recorded) when it does not within kWaitLimitNs or another CTA reported one.
__device__ __forceinline__ bool peer_wait_flag(const uint32_t* flag, uint32_t epoch) {
  const uint64_t start = global_timer_ns();
  uint32_t spins = 0;
  while (static_cast<int32_t>(ld_acquire_sys(flag) - epoch) < 0) {
    if ((++spins & 1023u) == 0) {
      if (error_raised()) return false;
      if (global_timer_ns() - start > kWaitLimitNs) {
        record_error(kErrTimeoutPeer);
        return false;
      }
    }
  }
  return true;
}

// Advance the epoch counters for one call, after griddepcontrol.wait: CTA
// `cta` of a grid of `ctas` takes slot `cta` (returned by thread `lead`), CTA 0
// also the slots beyond the grid.  `tid`/`nthreads` index the participating
// threads of the CTA.
__device__ __forceinline__ void peer_advance_epochs(uint8_t* own, int cta, int ctas, int tid, int nthreads) {
  uint32_t* ep = peer_epochs(own);
  if (tid == 0) ep[cta] = ep[cta] + 1;
  if (cta == 0)
    for (int s = ctas + tid; s < kPeerSlots; s += nthreads) ep[s] = ep[s] + 1;
}

}  // namespace nv4
