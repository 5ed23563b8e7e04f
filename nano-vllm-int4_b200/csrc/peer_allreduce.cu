// Kernel E: one-shot all-reduce of the row-parallel FP32 partials over
// NVLink peer memory, with the BF16 conversion fused.
//
// Replaces, for decode-sized outputs, the NCCL all-reduce of the row-parallel
// layers (the W4A4 counterpart of nanovllm/layers/linear.py:154-155).  Each
// rank owns one peer buffer (cudaMalloc at set-up, mapped into the other ranks
// with CUDA IPC), shared by all row-parallel layers of its process group:
//
//   header  [NV4_PEER_HEADER_BYTES]: flag[sender][cta] (uint32), epoch[cta]
//   partial [capacity] FP32: this rank's GEMM writes its partial here
//   inbox   [2][8][capacity] FP32: slot (parity, sender) receives that
//           sender's partial
//
// One launch per call; CTA c owns the fixed element chunk c of the capacity:
//   1. takes the next epoch e of its local counter (parity e & 1);
//   2. stores its chunk of the local partial into inbox[e & 1][rank] of every
//      peer (remote stores), fences, and stores flag[rank][c] = e there;
//   3. waits until its own flag[r][c] >= e for every peer r (local polling,
//      bounded);
//   4. sums the chunk in rank order 0 .. world-1 (its own partial for its own
//      rank, the inbox for the others) -- the same order on every rank, so all
//      ranks get identical BF16 -- and writes the BF16 output.
// A rank can be at most one call ahead of a peer (it waits for the peer's data
// of every call), so alternating the inbox parity is enough to keep a sender
// from overwriting data a receiver has not read.  The epochs are device state,
// so CUDA-graph replays keep the protocol; all ranks must make the same
// sequence of calls with the same counts and capacity.  Every wait gives up
// after 2 s, records an error word and returns.
#include "nv4_device.cuh"
#include "nv4_launch.h"

namespace nv4 {

constexpr int kPeerMaxRanks = 8;
constexpr int kPeerCtas = 64;
constexpr int kPeerHeaderBytes = NV4_PEER_HEADER_BYTES;  // flag[8][64], epoch[64] (uint32), padding
constexpr int kErrTimeoutPeer = 5;                        // a peer rank did not reach the same all-reduce in time
static_assert((kPeerMaxRanks + 1) * kPeerCtas * 4 <= kPeerHeaderBytes, "peer header too small");

struct PeerArgs {
  uint8_t* bufs[kPeerMaxRanks];  // every rank's peer buffer (this rank's own at [rank])
  __nv_bfloat16* out;
  int64_t count;                 // elements of this call (multiple of 4, <= capacity)
  int64_t capacity;              // elements of a partial (multiple of 4), the same on every rank
  int rank, world;
};

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

__device__ __forceinline__ float* peer_partial(uint8_t* buf) {
  return reinterpret_cast<float*>(buf + kPeerHeaderBytes);
}
__device__ __forceinline__ float* peer_inbox(uint8_t* buf, int64_t capacity, int parity, int sender) {
  return peer_partial(buf) + capacity * (1 + parity * kPeerMaxRanks + sender);
}

__global__ void __launch_bounds__(256) peer_allreduce_bf16_kernel(const PeerArgs p) {
  __shared__ uint32_t epoch_s;
  __shared__ int go;
  uint8_t* own = p.bufs[p.rank];
  uint32_t* flags = reinterpret_cast<uint32_t*>(own);
  uint32_t* epochs = flags + kPeerMaxRanks * kPeerCtas;
  const int c = blockIdx.x;
  if (threadIdx.x == 0) {
    epoch_s = epochs[c] + 1;
    epochs[c] = epoch_s;
  }
  __syncthreads();
  const uint32_t e = epoch_s;
  // Dependents may launch once every CTA has taken its epoch (a following
  // all-reduce reads the counters only after that).
  grid_dependents_launch();
  grid_dependency_wait();  // the partial comes from the GEMM before this kernel
  const int parity = static_cast<int>(e & 1u);
  const int64_t per = (p.capacity / 4 + kPeerCtas - 1) / kPeerCtas;  // float4 words of a chunk
  const int64_t w0 = c * per, w1 = min(p.count / 4, w0 + per);
  const float* mine = peer_partial(own);

  // 2. push this chunk of the partial to every peer
  for (int r = 0; r < p.world; ++r) {
    if (r == p.rank) continue;
    float* dst = peer_inbox(p.bufs[r], p.capacity, parity, p.rank);
    for (int64_t w = w0 + threadIdx.x; w < w1; w += blockDim.x)
      *reinterpret_cast<float4*>(dst + 4 * w) = *reinterpret_cast<const float4*>(mine + 4 * w);
  }
  // The barrier orders every thread's stores before thread 0's system-scope
  // release of the flags (release is cumulative over what happens before it).
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int r = 0; r < p.world; ++r)
      if (r != p.rank) st_release_sys(reinterpret_cast<uint32_t*>(p.bufs[r]) + p.rank * kPeerCtas + c, e);
    // 3. wait for every peer's chunk (local flags)
    bool ok = true;
    const uint64_t start = global_timer_ns();
    for (int r = 0; r < p.world && ok; ++r) {
      if (r == p.rank) continue;
      uint32_t spins = 0;
      while (static_cast<int32_t>(ld_acquire_sys(flags + r * kPeerCtas + c) - e) < 0) {
        if ((++spins & 1023u) == 0) {
          if (error_raised() || global_timer_ns() - start > kWaitLimitNs) {
            record_error(kErrTimeoutPeer);
            ok = false;
            break;
          }
        }
      }
    }
    go = ok ? 1 : 0;
  }
  __syncthreads();
  if (!go) return;
  // 4. sum in rank order and write BF16
  for (int64_t w = w0 + threadIdx.x; w < w1; w += blockDim.x) {
    float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int r = 0; r < p.world; ++r) {
      const float4 v = r == p.rank ? *reinterpret_cast<const float4*>(mine + 4 * w)
                                   : ld_volatile_f4(peer_inbox(own, p.capacity, parity, r) + 4 * w);
      if (r == 0) {
        s = v;
      } else {
        s.x = __fadd_rn(s.x, v.x);
        s.y = __fadd_rn(s.y, v.y);
        s.z = __fadd_rn(s.z, v.z);
        s.w = __fadd_rn(s.w, v.w);
      }
    }
    __nv_bfloat162* o = reinterpret_cast<__nv_bfloat162*>(p.out + 4 * w);
    o[0] = __floats2bfloat162_rn(s.x, s.y);
    o[1] = __floats2bfloat162_rn(s.z, s.w);
  }
}

int64_t peer_buffer_data_bytes(int64_t capacity) { return capacity * 4 * (1 + 2 * kPeerMaxRanks); }

int launch_peer_allreduce_bf16(void* const* bufs, int rank, int world, void* out, int64_t count, int64_t capacity,
                               cudaStream_t stream) {
  PeerArgs a;
  for (int r = 0; r < kPeerMaxRanks; ++r) a.bufs[r] = r < world ? static_cast<uint8_t*>(bufs[r]) : nullptr;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.count = count;
  a.capacity = capacity;
  a.rank = rank;
  a.world = world;
  // Programmatic dependent launch: nothing before griddepcontrol.wait touches
  // memory another kernel writes (only this kernel's own epoch counters).
  return launch_kernel(peer_allreduce_bf16_kernel, dim3(kPeerCtas), dim3(256), 0, stream, true, a);
}

}  // namespace nv4
