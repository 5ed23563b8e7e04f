// Kernel E: one-shot all-reduce of the row-parallel FP32 partials over
// NVLink peer memory, with the BF16 conversion fused (buffer layout, epochs and
// flags: peer_common.cuh).
//
// Replaces, for decode-sized outputs, the NCCL all-reduce of the row-parallel
// layers (the W4A4 counterpart of nanovllm/layers/linear.py:154-155).  Two
// forms share one peer buffer per process group:
//
// E1, peer_allreduce_bf16_kernel (after any GEMM that wrote its FP32 partial
//   to the buffer's partial area): CTA c owns element chunk c of the output;
//   it pushes the chunk into inbox[parity][rank] of every peer (remote stores),
//   releases flag[rank][c] there, waits for its own flag[r][c] of every peer
//   and sums the chunk in rank order 0 .. world-1.
// E2, peer_reduce_tiles_bf16_kernel (after the row-parallel stream GEMM run in
//   peer mode, whose CTA j stored its [M x R] FP32 tile into inbox[parity][rank]
//   of every rank and released flag[rank][j] on the peers): CTA j waits for
//   flag[r][j] of every peer and sums tile j in rank order.
// Both sum in the same order on every rank, so all ranks get identical BF16
// (equal to NCCL's two-rank sum at TP=2).  Every wait gives up after 2 s,
// records an error word and returns.
#include "nv4_device.cuh"
#include "nv4_launch.h"
#include "peer_common.cuh"

namespace nv4 {

constexpr int kPeerCtas = 64;  // E1 grid

struct PeerArgs {
  uint8_t* bufs[kPeerMaxRanks];  // every rank's peer buffer (this rank's own at [rank])
  __nv_bfloat16* out;
  int64_t count;                 // elements of this call (multiple of 4, <= capacity)
  int64_t capacity;              // elements of a partial (multiple of 4), the same on every rank
  int rank, world;
};

__global__ void __launch_bounds__(256) peer_allreduce_bf16_kernel(const PeerArgs p) {
  __shared__ uint32_t epoch_s;
  __shared__ int go;
  uint8_t* own = p.bufs[p.rank];
  uint32_t* flags = peer_flags(own);
  const int c = blockIdx.x;
  // Dependents may launch now: they touch the epochs only after their own
  // griddepcontrol.wait, which returns after this grid has completed.
  grid_dependents_launch();
  grid_dependency_wait();  // the partial comes from the GEMM before this kernel
  peer_advance_epochs(own, c, kPeerCtas, threadIdx.x, blockDim.x);
  if (threadIdx.x == 0) epoch_s = peer_epochs(own)[c];
  __syncthreads();
  const uint32_t e = epoch_s;
  const int parity = static_cast<int>(e & 1u);
  const int64_t per = (p.capacity / 4 + kPeerCtas - 1) / kPeerCtas;  // float4 words of a chunk
  const int64_t w0 = c * per, w1 = min(p.count / 4, w0 + per);
  const float* mine = peer_partial(own);

  // push this chunk of the partial to every peer
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
      if (r != p.rank) st_release_sys(peer_flags(p.bufs[r]) + p.rank * kPeerSlots + c, e);
    bool ok = true;
    for (int r = 0; r < p.world && ok; ++r)
      if (r != p.rank) ok = peer_wait_flag(flags + r * kPeerSlots + c, e);
    go = ok ? 1 : 0;
  }
  __syncthreads();
  if (!go) return;
  // sum in rank order and write BF16
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

struct PeerTileArgs {
  uint8_t* bufs[kPeerMaxRanks];
  __nv_bfloat16* out;  // [M, N]
  int64_t capacity;
  int M, N, R;         // CTA j owns columns [j*R, min(N, (j+1)*R)) of all M rows
  int rank, world;
};

__global__ void __launch_bounds__(256) peer_reduce_tiles_bf16_kernel(const PeerTileArgs p) {
  __shared__ uint32_t epoch_s;
  uint8_t* own = p.bufs[p.rank];
  const int j = blockIdx.x;
  grid_dependents_launch();
  grid_dependency_wait();  // the peer-mode GEMM of this call took the epoch and wrote this rank's tiles
  if (threadIdx.x == 0) epoch_s = peer_epochs(own)[j];
  __syncthreads();
  const uint32_t e = epoch_s;
  const int parity = static_cast<int>(e & 1u);
  bool ok = true;
  if (threadIdx.x < p.world && threadIdx.x != p.rank)
    ok = peer_wait_flag(peer_flags(own) + threadIdx.x * kPeerSlots + j, e);
  if (!__syncthreads_and(ok)) return;
  const int n0 = j * p.R, w = min(p.R, p.N - n0);
  if (w <= 0) return;
  if ((w & 3) == 0) {
    const int wq = w >> 2;
    for (int i = threadIdx.x; i < p.M * wq; i += blockDim.x) {
      const int m = i / wq;
      const int64_t o = static_cast<int64_t>(m) * p.N + n0 + 4 * (i - m * wq);
      float4 s = ld_volatile_f4(peer_inbox(own, p.capacity, parity, 0) + o);
      for (int r = 1; r < p.world; ++r) {
        const float4 v = ld_volatile_f4(peer_inbox(own, p.capacity, parity, r) + o);
        s.x = __fadd_rn(s.x, v.x);
        s.y = __fadd_rn(s.y, v.y);
        s.z = __fadd_rn(s.z, v.z);
        s.w = __fadd_rn(s.w, v.w);
      }
      __nv_bfloat162* d = reinterpret_cast<__nv_bfloat162*>(p.out + o);
      d[0] = __floats2bfloat162_rn(s.x, s.y);
      d[1] = __floats2bfloat162_rn(s.z, s.w);
    }
  } else {
    for (int i = threadIdx.x; i < p.M * w; i += blockDim.x) {
      const int m = i / w;
      const int64_t o = static_cast<int64_t>(m) * p.N + n0 + (i - m * w);
      float s = ld_volatile_f(peer_inbox(own, p.capacity, parity, 0) + o);
      for (int r = 1; r < p.world; ++r) s = __fadd_rn(s, ld_volatile_f(peer_inbox(own, p.capacity, parity, r) + o));
      p.out[o] = __float2bfloat16_rn(s);
    }
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
  return launch_kernel(peer_allreduce_bf16_kernel, dim3(kPeerCtas), dim3(256), 0, stream, true, a);
}

int launch_peer_reduce_tiles_bf16(void* const* bufs, int rank, int world, void* out, int m, int n, int rows_per_cta,
                                  int ctas, int64_t capacity, cudaStream_t stream) {
  PeerTileArgs a;
  for (int r = 0; r < kPeerMaxRanks; ++r) a.bufs[r] = r < world ? static_cast<uint8_t*>(bufs[r]) : nullptr;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.capacity = capacity;
  a.M = m;
  a.N = n;
  a.R = rows_per_cta;
  a.rank = rank;
  a.world = world;
  return launch_kernel(peer_reduce_tiles_bf16_kernel, dim3(ctas), dim3(256), 0, stream, true, a);
}

}  // namespace nv4
