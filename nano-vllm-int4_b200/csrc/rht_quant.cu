// Kernel A: randomized Hadamard transform + per-128-group INT4 quantisation +
// nibble packing, for the two activation layouts of the quantized-linear path.
//
//  * block128 (layout 0): a normalized 128-point Walsh-Hadamard transform of
//    each K group after the sign multiply, with the arithmetic of the reference
//    PyTorch path on CPU (benchmarks/rht_reference.py:26-39 fwht, then
//    benchmarks/a4_group_quant.py:206-216 quantize_rotated): butterflies lowest
//    index bit first, x / fl32(sqrt(128)) and scale = bf16(fl(fl(absmax*0.9)/7)),
//    both IEEE divisions.
//  * row_DH_paley12_kron_sylvester_v1 (layout 1): the reference checkpoint
//    layout, with the arithmetic of nanovllm/kernels/rht_a4_tilelang.py:38-135:
//    full-width H4096, or H1024 per factor followed by the Paley H12 mix summed
//    source 0..11 and multiplied by fl32(1/sqrt(12)); scale uses
//    __fmul_rn(__fmul_rn(absmax, 0.9f), fl32(1/7)).
//
// Both: scale rounded to BF16 before codes, 1.0 for an all-zero group, floor at
// the BF16 tiny, code = round-half-even(__fdiv_rn(x, scale)) clamped to
// [clamp_lo, 7], two codes per byte with the even K index in the low nibble.
//
// The two divisions are computed without the IEEE division sequence where
// that gives the same result (div_sqrt128 and quant_code below say why), and
// fall back to __fdiv_rn where it might not.
//
// The butterflies map index bits to registers (3 low bits inside a 16-byte
// load), to lanes (warp shuffles) and, for the full-width layout, to warps (one
// shared-memory exchange); the FP32 result of every butterfly equals the
// reference's because each output is the same single-rounded a+b or a-b.
#include "nv4_device.cuh"
#include "nv4_launch.h"

namespace nv4 {

constexpr unsigned kFull = 0xffffffffu;

__device__ __forceinline__ float scale_block128(float mx) {
  float t = __fmul_rn(mx, kClip);
  float u = __fdiv_rn(t, 7.0f);
  u = fmaxf(u, kBf16Tiny);
  return (mx == 0.0f) ? 1.0f : u;
}

__device__ __forceinline__ float scale_rowdh(float mx) {
  float t = __fmul_rn(mx, kClip);
  t = __fmul_rn(t, kInv7);
  t = fmaxf(t, kBf16Tiny);
  return (mx == 0.0f) ? 1.0f : t;
}

// BF16-round the FP32 scale; returns the rounded value, bits in *bits.
__device__ __forceinline__ float round_scale(float s, uint16_t* bits) {
  __nv_bfloat16 b = __float2bfloat16_rn(s);
  *bits = __bfloat16_as_ushort(b);
  return __bfloat162float(b);
}

// x / fl32(sqrt(128)), correctly rounded: q0 = x*r with r = RN(1/d), then one
// residual correction q1 = fma(fma(-q0, d, x), r, q0) -- Markstein's
// correction step (P. Markstein, "Computation of elementary functions on the
// IBM RISC System/6000 processor", IBM J. Res. Dev. 34(1), 1990), used here in
// the setting of a divisor known in advance studied by N. Brisebarre,
// J.-M. Muller and S. K. Raina ("Accelerating correctly rounded floating-point
// division when the divisor is known in advance", IEEE Trans. Computers 53(8),
// 2004).  For this divisor the result equals the IEEE quotient for every
// significand once |x| >= 2^-100 (checked exhaustively on the host,
// tests/test_prep_arith_cpu.py); below that the intermediates may be subnormal
// and the IEEE division is used.
__device__ __forceinline__ float div_sqrt128(float x) {
  const float q0 = x * kInvSqrt128;
  const float q1 = fmaf(fmaf(-q0, kSqrt128, x), kInvSqrt128, q0);
  return fabsf(x) >= 0x1p-100f ? q1 : __fdiv_rn(x, kSqrt128);
}

// round-half-even(fl32(v / sf)) clamped, with rs = RN(1/sf).  The scale makes
// |v / sf| < 7.82, where q = RN(v * rs) is within 2^-19 of the rounded
// quotient, so both round to the same integer unless q is within 2^-17 of a
// half-integer; there the IEEE quotient decides.
__device__ __forceinline__ int quant_code(float v, float sf, float rs, int clamp_lo) {
  const float q = v * rs;
  float k = rintf(q);
  if (fabsf(fabsf(q - k) - 0.5f) < 0x1p-17f) k = rintf(__fdiv_rn(v, sf));
  int c = __float2int_rn(k);
  c = max(c, clamp_lo);
  return min(c, 7);
}

// Quantise the 8 values of k = k8 .. k8+7 (k8 % 8 == 0) of one row and store
// them in the requested forms:
//  * packed (two codes per byte, even k in the low nibble) at packed_row + k8/2;
//  * GEMM-ready INT8 codes (i8_row != nullptr): within each 32-wide K chunk the
//    16 even-k codes come first, then the 16 odd-k codes -- the K order the
//    GEMM's INT4->INT8 weight widening produces, so its MMA operands match.
__device__ __forceinline__ void store_codes(const float (&v)[8], float sf, int clamp_lo, uint8_t* packed_row,
                                            int8_t* i8_row, int k8) {
  const float rs = __frcp_rn(sf);
  int c[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) c[e] = quant_code(v[e], sf, rs, clamp_lo);
  if (packed_row != nullptr) {
    uint32_t word = 0;
#pragma unroll
    for (int e = 0; e < 8; ++e) word |= (static_cast<uint32_t>(c[e]) & 15u) << (4 * e);
    *reinterpret_cast<uint32_t*>(packed_row + k8 / 2) = word;
  }
  if (i8_row != nullptr) {
    uint32_t even = 0, odd = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      even |= (static_cast<uint32_t>(c[2 * i]) & 255u) << (8 * i);
      odd |= (static_cast<uint32_t>(c[2 * i + 1]) & 255u) << (8 * i);
    }
    int8_t* chunk = i8_row + (k8 & ~31);
    const int q = (k8 & 31) >> 3;
    *reinterpret_cast<uint32_t*>(chunk + q * 4) = even;
    *reinterpret_cast<uint32_t*>(chunk + 16 + q * 4) = odd;
  }
}

// Load 8 BF16 values (16 bytes) and apply 8 sign bits (bit e set = negate).
__device__ __forceinline__ void load8_signed(const uint16_t* src, uint32_t sbits, float (&v)[8]) {
  const uint4 w = __ldg(reinterpret_cast<const uint4*>(src));
  const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[2 * i] = __uint_as_float((ws[i] << 16) ^ (((sbits >> (2 * i)) & 1u) << 31));
    v[2 * i + 1] = __uint_as_float((ws[i] & 0xFFFF0000u) ^ (((sbits >> (2 * i + 1)) & 1u) << 31));
  }
}

// bf16(silu(g) * u) in FP32 with one rounding at the end, as the reference's
// compiled SiluAndMul (nanovllm/layers/activation.py:8-11: torch.compile keeps
// the product in FP32): silu(g) = g / (1 + exp(-g)) with CUDA's expf and IEEE
// division, as PyTorch's FP32 silu.
__device__ __forceinline__ uint32_t silu_mul_bf16_bits(float g, float u) {
  const float s = __fdiv_rn(g, 1.0f + expf(-g));
  return static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(__fmul_rn(s, u))));
}

// 8 prep input values at element k of a source row, signs applied: the BF16
// input itself, or (SILU) the fused activation of a gate/up row [gate | up]
// (each kdim wide), rounded to BF16 as the unfused SiluAndMul output would be.
template <bool SILU>
__device__ __forceinline__ void load8_input(const uint16_t* row, int k, int kdim, uint32_t sbits, float (&v)[8]) {
  if constexpr (!SILU) {
    load8_signed(row + k, sbits, v);
  } else {
    const uint4 gw = __ldg(reinterpret_cast<const uint4*>(row + k));
    const uint4 uw = __ldg(reinterpret_cast<const uint4*>(row + kdim + k));
    const uint32_t gs[4] = {gw.x, gw.y, gw.z, gw.w}, us[4] = {uw.x, uw.y, uw.z, uw.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t h0 = silu_mul_bf16_bits(__uint_as_float(gs[i] << 16), __uint_as_float(us[i] << 16));
      const uint32_t h1 =
          silu_mul_bf16_bits(__uint_as_float(gs[i] & 0xFFFF0000u), __uint_as_float(us[i] & 0xFFFF0000u));
      v[2 * i] = __uint_as_float((h0 << 16) ^ (((sbits >> (2 * i)) & 1u) << 31));
      v[2 * i + 1] = __uint_as_float((h1 << 16) ^ (((sbits >> (2 * i + 1)) & 1u) << 31));
    }
  }
}

// 8 sign bytes (int8 +-1) -> 8 bits, bit e set for a negative sign.
__device__ __forceinline__ uint32_t sign_bits8(const int8_t* s) {
  const uint2 w = *reinterpret_cast<const uint2*>(s);
  uint32_t bits = 0;
#pragma unroll
  for (int e = 0; e < 4; ++e) bits |= ((w.x >> (8 * e + 7)) & 1u) << e;
#pragma unroll
  for (int e = 0; e < 4; ++e) bits |= ((w.y >> (8 * e + 7)) & 1u) << (e + 4);
  return bits;
}

// Butterflies over index bits 0..2 held in registers (lowest bit first).
__device__ __forceinline__ void butterfly8(float (&v)[8]) {
#pragma unroll
  for (int s = 1; s < 8; s <<= 1) {
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      if (!(e & s)) {
        const float a = v[e], b = v[e + s];
        v[e] = a + b;
        v[e + s] = a - b;
      }
    }
  }
}

// One butterfly stage across lanes (partner = lane ^ mask).  The lane holding
// the low element computes a+b, the high one a-b; fma with +-1 rounds once.
__device__ __forceinline__ float butterfly_lane(float v, int mask, bool high) {
  const float other = __shfl_xor_sync(kFull, v, mask);
  return fmaf(v, high ? -1.0f : 1.0f, other);
}

// ============================================================ block128
struct Block128Args {
  const uint16_t* x;  // rows of x_stride elements (K, or 2K for a gate/up source)
  const int8_t* signs;
  uint8_t* packed;   // or nullptr
  int8_t* codes8;    // or nullptr
  uint16_t* scale;
  int M, K, G, ncb, warps_used, clamp_lo, x_stride;
};

// The block128 transform and quantisation of one group held by LPG lanes
// (lane l of the group holds elements j*8*LPG + l*8 + e, signs applied):
// butterflies over index bits 0-2 (registers), the lane bits (shuffles) and the
// register-block bits, 1/sqrt(128), group absmax, BF16 scale, codes.
template <int LPG>
__device__ __forceinline__ void block128_quant_group(float (&v)[16 / LPG][8], int l, bool active, int clamp_lo,
                                                     uint8_t* prow, int8_t* irow, uint16_t* scale_row, int g) {
  constexpr int J = 16 / LPG;
#pragma unroll
  for (int j = 0; j < J; ++j) butterfly8(v[j]);  // bits 0-2
#pragma unroll
  for (int m = 1; m < LPG; m <<= 1)               // the lane bits
#pragma unroll
    for (int j = 0; j < J; ++j)
#pragma unroll
      for (int e = 0; e < 8; ++e) v[j][e] = butterfly_lane(v[j][e], m, (l & m) != 0);
#pragma unroll
  for (int s = 1; s < J; s <<= 1) {               // the register-block bits
#pragma unroll
    for (int j = 0; j < J; ++j) {
      if (!(j & s)) {
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float a = v[j][e], b = v[j + s][e];
          v[j][e] = a + b;
          v[j + s][e] = a - b;
        }
      }
    }
  }
  float mx = 0.0f;
#pragma unroll
  for (int j = 0; j < J; ++j)
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      v[j][e] = div_sqrt128(v[j][e]);
      mx = fmaxf(mx, fabsf(v[j][e]));
    }
#pragma unroll
  for (int m = 1; m < LPG; m <<= 1) mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, m));
  uint16_t sbits;
  const float sf = round_scale(scale_block128(mx), &sbits);
  if (active) {
#pragma unroll
    for (int j = 0; j < J; ++j) store_codes(v[j], sf, clamp_lo, prow, irow, g * 128 + j * 8 * LPG + l * 8);
    if (l == 0) scale_row[g] = sbits;
  }
}

// A warp owns GPW = 32 / LPG consecutive groups (one "column block") of a row;
// the LPG lanes of group slot `slot` hold elements idx = j*8*LPG + l*8 + e of
// group cb*GPW + slot (e: index bits 0-2, l: the next log2(LPG) bits, j: the
// rest).  Warps keep their column block, and so their signs, while striding
// over rows.  LPG = 8 halves each lane's work for decode batches; LPG = 4
// needs fewer shuffles for large batches.
template <int LPG, bool SILU>
__global__ void __launch_bounds__(256) rht_block128_kernel(const Block128Args p) {
  constexpr int J = 16 / LPG;    // 8-element register blocks per lane
  constexpr int GPW = 32 / LPG;  // groups per warp
  grid_dependents_launch();
  const int lane = threadIdx.x & 31;
  const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (gw >= p.warps_used) return;
  const int cb = gw % p.ncb;
  const int row_step = p.warps_used / p.ncb;
  const int slot = lane / LPG, l = lane % LPG;
  const int g = cb * GPW + slot;
  const bool active = g < p.G;

  uint32_t sb[J];
#pragma unroll
  for (int j = 0; j < J; ++j) sb[j] = active ? sign_bits8(p.signs + g * 128 + j * 8 * LPG + l * 8) : 0u;
  grid_dependency_wait();

  for (int row = gw / p.ncb; row < p.M; row += row_step) {
    float v[J][8];
    if (active) {
      const uint16_t* src = p.x + static_cast<size_t>(row) * p.x_stride;
#pragma unroll
      for (int j = 0; j < J; ++j) load8_input<SILU>(src, g * 128 + j * 8 * LPG + l * 8, p.K, sb[j], v[j]);
    } else {
#pragma unroll
      for (int j = 0; j < J; ++j)
#pragma unroll
        for (int e = 0; e < 8; ++e) v[j][e] = 0.0f;
    }
    block128_quant_group<LPG>(v, l, active, p.clamp_lo, p.packed ? p.packed + static_cast<size_t>(row) * (p.K / 2) : nullptr,
                              p.codes8 ? p.codes8 + static_cast<size_t>(row) * p.K : nullptr,
                              p.scale + static_cast<size_t>(row) * p.G, g);
  }
}

// ============================================================ row_DH
struct RowDHArgs {
  const uint16_t* x;  // rows of x_stride elements (K, or 2K for a gate/up source)
  const int8_t* signs;
  uint8_t* packed;   // or nullptr
  int8_t* codes8;    // or nullptr
  uint16_t* scale;
  int M, clamp_lo, x_stride;
};

// Shared-memory index with 4 floats of padding per 32 (keeps float4 accesses
// of consecutive lanes on distinct banks).
__host__ __device__ constexpr int padded(int k) { return k + ((k >> 5) << 2); }

// Combine the four values at warp-index bits (b, b+1) into this warp's output
// of two butterfly stages: stage b pairs (0,1),(2,3); stage b+1 pairs (0,2),(1,3).
__device__ __forceinline__ float two_stages(float v0, float v1, float v2, float v3, int w) {
  const float lo = (w & 1) ? v0 - v1 : v0 + v1;
  const float hi = (w & 1) ? v2 - v3 : v2 + v3;
  return (w & 2) ? lo - hi : lo + hi;
}

// The rest of the full-width H4096 transform of one row and its quantisation,
// after each thread's register and lane butterflies: the warp bits through
// shared memory (two __syncthreads, all 128 threads), x 1/64, groups of 16
// lanes x 8 values, BF16 scales, codes.
__device__ __forceinline__ void rowdh4096_quant_row(float (&v)[4][8], float* sh, int w, int l, int clamp_lo,
                                                    uint8_t* prow, int8_t* irow, uint16_t* scale_row) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float4* d = reinterpret_cast<float4*>(sh + padded(w * 1024 + j * 256 + l * 8));
    d[0] = make_float4(v[j][0], v[j][1], v[j][2], v[j][3]);
    d[1] = make_float4(v[j][4], v[j][5], v[j][6], v[j][7]);
  }
  __syncthreads();
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float u[4][8];
#pragma unroll
    for (int ww = 0; ww < 4; ++ww) {
      const float4* s4 = reinterpret_cast<const float4*>(sh + padded(ww * 1024 + j * 256 + l * 8));
      const float4 a = s4[0], b = s4[1];
      u[ww][0] = a.x; u[ww][1] = a.y; u[ww][2] = a.z; u[ww][3] = a.w;
      u[ww][4] = b.x; u[ww][5] = b.y; u[ww][6] = b.z; u[ww][7] = b.w;
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) v[j][e] = two_stages(u[0][e], u[1][e], u[2][e], u[3][e], w) * 0.015625f;
  }
  __syncthreads();
  // groups: k >> 7 = w*8 + j*2 + (l >> 4); 16 lanes x 8 values each
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float mx = 0.0f;
#pragma unroll
    for (int e = 0; e < 8; ++e) mx = fmaxf(mx, fabsf(v[j][e]));
#pragma unroll
    for (int m = 1; m < 16; m <<= 1) mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, m));
    uint16_t sbits;
    const float sf = round_scale(scale_rowdh(mx), &sbits);
    store_codes(v[j], sf, clamp_lo, prow, irow, w * 1024 + j * 256 + l * 8);
    if ((l & 15) == 0) scale_row[w * 8 + j * 2 + (l >> 4)] = sbits;
  }
}

// Butterflies of the H4096 row transform inside a thread (index bits 0-2), the
// lanes (bits 3-7) and the register blocks (bits 8-9).
__device__ __forceinline__ void rowdh4096_local_stages(float (&v)[4][8], int l) {
#pragma unroll
  for (int j = 0; j < 4; ++j) butterfly8(v[j]);
#pragma unroll
  for (int m = 1; m < 32; m <<= 1)
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int e = 0; e < 8; ++e) v[j][e] = butterfly_lane(v[j][e], m, (l & m) != 0);
#pragma unroll
  for (int s = 1; s < 4; s <<= 1)
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (!(j & s)) {
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float a = v[j][e], b = v[j + s][e];
          v[j][e] = a + b;
          v[j + s][e] = a - b;
        }
      }
}

// K = 4096.  Thread (warp w, lane l) holds k = w*1024 + j*256 + l*8 + e:
// e bits 0-2, lane bits 3-7, j bits 8-9, warp bits 10-11.
template <bool SILU>
__global__ void __launch_bounds__(128) rht_rowdh4096_kernel(const RowDHArgs p) {
  grid_dependents_launch();
  constexpr int K = 4096, G = 32;
  __shared__ __align__(16) float sh[padded(K)];
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  uint32_t sb[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) sb[j] = sign_bits8(p.signs + w * 1024 + j * 256 + l * 8);
  grid_dependency_wait();

  for (int row = blockIdx.x; row < p.M; row += gridDim.x) {
    float v[4][8];
    const uint16_t* src = p.x + static_cast<size_t>(row) * p.x_stride;
#pragma unroll
    for (int j = 0; j < 4; ++j) load8_input<SILU>(src, w * 1024 + j * 256 + l * 8, K, sb[j], v[j]);
    rowdh4096_local_stages(v, l);
    rowdh4096_quant_row(v, sh, w, l, p.clamp_lo, p.packed ? p.packed + static_cast<size_t>(row) * (K / 2) : nullptr,
                        p.codes8 ? p.codes8 + static_cast<size_t>(row) * K : nullptr,
                        p.scale + static_cast<size_t>(row) * G);
  }
}

__device__ __forceinline__ bool h12_positive(int source, int destination) {
  if (source == 0 || destination == 0) return true;
  const int d = (destination - source + 11) % 11;
  return d == 1 || d == 3 || d == 4 || d == 5 || d == 9;
}

// K = 12288 = 12 x 1024.  Thread (warp w, lane l) holds, for each factor f,
// k = f*1024 + w*256 + l*8 + e: e bits 0-2, lane bits 3-7, warp bits 8-9 of
// the 1024-point transform; the 12 factors of a position live in one thread,
// so the H12 mix is register-local.
template <bool SILU>
__global__ void __launch_bounds__(128) rht_rowdh12288_kernel(const RowDHArgs p) {
  grid_dependents_launch();
  constexpr int K = 12288, G = 96;
  extern __shared__ __align__(16) float shd[];
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  uint32_t sb[12];
#pragma unroll
  for (int f = 0; f < 12; ++f) sb[f] = sign_bits8(p.signs + f * 1024 + w * 256 + l * 8);
  grid_dependency_wait();

  for (int row = blockIdx.x; row < p.M; row += gridDim.x) {
    float v[12][8];
    const uint16_t* src = p.x + static_cast<size_t>(row) * p.x_stride;
#pragma unroll
    for (int f = 0; f < 12; ++f) load8_input<SILU>(src, f * 1024 + w * 256 + l * 8, K, sb[f], v[f]);
#pragma unroll
    for (int f = 0; f < 12; ++f) butterfly8(v[f]);
#pragma unroll
    for (int m = 1; m < 32; m <<= 1)
#pragma unroll
      for (int f = 0; f < 12; ++f)
#pragma unroll
        for (int e = 0; e < 8; ++e) v[f][e] = butterfly_lane(v[f][e], m, (l & m) != 0);
#pragma unroll
    for (int f = 0; f < 12; ++f) {
      float4* d = reinterpret_cast<float4*>(shd + padded(f * 1024 + w * 256 + l * 8));
      d[0] = make_float4(v[f][0], v[f][1], v[f][2], v[f][3]);
      d[1] = make_float4(v[f][4], v[f][5], v[f][6], v[f][7]);
    }
    __syncthreads();
#pragma unroll
    for (int f = 0; f < 12; ++f) {
      float u[4][8];
#pragma unroll
      for (int ww = 0; ww < 4; ++ww) {
        const float4* s4 = reinterpret_cast<const float4*>(shd + padded(f * 1024 + ww * 256 + l * 8));
        const float4 a = s4[0], b = s4[1];
        u[ww][0] = a.x; u[ww][1] = a.y; u[ww][2] = a.z; u[ww][3] = a.w;
        u[ww][4] = b.x; u[ww][5] = b.y; u[ww][6] = b.z; u[ww][7] = b.w;
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) v[f][e] = two_stages(u[0][e], u[1][e], u[2][e], u[3][e], w) * 0.03125f;
    }
    __syncthreads();
    // Paley H12 across the factors: out[d] = sum_s H12[s,d] z[s], s = 0..11.
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      float b[12];
#pragma unroll
      for (int d = 0; d < 12; ++d) {
        float acc = 0.0f;
#pragma unroll
        for (int s = 0; s < 12; ++s) acc = h12_positive(s, d) ? acc + v[s][e] : acc - v[s][e];
        b[d] = acc * kInvSqrt12;
      }
#pragma unroll
      for (int d = 0; d < 12; ++d) v[d][e] = b[d];
    }
    uint8_t* prow = p.packed ? p.packed + static_cast<size_t>(row) * (K / 2) : nullptr;
    int8_t* irow = p.codes8 ? p.codes8 + static_cast<size_t>(row) * K : nullptr;
#pragma unroll
    for (int f = 0; f < 12; ++f) {
      float mx = 0.0f;
#pragma unroll
      for (int e = 0; e < 8; ++e) mx = fmaxf(mx, fabsf(v[f][e]));
#pragma unroll
      for (int m = 1; m < 16; m <<= 1) mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, m));
      uint16_t sbits;
      const float sf = round_scale(scale_rowdh(mx), &sbits);
      store_codes(v[f], sf, p.clamp_lo, prow, irow, f * 1024 + w * 256 + l * 8);
      if ((l & 15) == 0) p.scale[static_cast<size_t>(row) * G + f * 8 + w * 2 + (l >> 4)] = sbits;
    }
  }
}

// ============================================================ add + RMSNorm fused
// The QKV / gate-up prep fused with its producer, the decoder layer's residual
// add and RMSNorm (nanovllm/layers/layernorm.py:33-45 add_rms_forward, :17-27
// rms_forward without a residual): xf = f32(x) + f32(residual) (new residual
// = bf16(xf)), var = mean(xf^2) in FP32, h = bf16(bf16(xf * rsqrt(var + eps)) *
// weight) -- the two BF16 roundings the reference's compiled code keeps (the
// explicit .to(bf16) and the BF16 product with the weight) -- then the prep of
// h.  The sum of squares runs in a fixed order (per thread in element order,
// warp xor tree, warps in order), so the result is deterministic; torch's
// reduction order differs, so var, and through it h, can differ from torch's
// in the last bit.
struct NormArgs {
  const uint16_t* x;         // [M, K]
  const uint16_t* residual;  // [M, K] or nullptr
  const uint16_t* weight;    // [K]
  uint16_t* out_residual;    // [M, K], written when residual != nullptr
  uint16_t* out_normed;      // [M, K] or nullptr: h
  const int8_t* signs;
  uint8_t* packed;           // or nullptr
  int8_t* codes8;            // or nullptr
  uint16_t* scale;
  float eps, inv_k;          // inv_k = 1/K when K is a power of two (exact), else 0
  int M, K, G, clamp_lo;
};

// xf of 8 elements at k of a row (the BF16 sum stored as the new residual) and
// their sum of squares in element order.
__device__ __forceinline__ float load8_add(const NormArgs& p, size_t off, int k, float (&xf)[8]) {
  const uint4 xw = __ldg(reinterpret_cast<const uint4*>(p.x + off + k));
  const uint32_t xs[4] = {xw.x, xw.y, xw.z, xw.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    xf[2 * i] = __uint_as_float(xs[i] << 16);
    xf[2 * i + 1] = __uint_as_float(xs[i] & 0xFFFF0000u);
  }
  if (p.residual != nullptr) {
    const uint4 rw = __ldg(reinterpret_cast<const uint4*>(p.residual + off + k));
    const uint32_t rs[4] = {rw.x, rw.y, rw.z, rw.w};
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      xf[2 * i] = __fadd_rn(xf[2 * i], __uint_as_float(rs[i] << 16));
      xf[2 * i + 1] = __fadd_rn(xf[2 * i + 1], __uint_as_float(rs[i] & 0xFFFF0000u));
      o[i] = static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(xf[2 * i]))) |
             (static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(xf[2 * i + 1]))) << 16);
    }
    *reinterpret_cast<uint4*>(p.out_residual + off + k) = make_uint4(o[0], o[1], o[2], o[3]);
  }
  float ss = 0.0f;
#pragma unroll
  for (int e = 0; e < 8; ++e) ss = __fadd_rn(ss, __fmul_rn(xf[e], xf[e]));
  return ss;
}

// FP32 sum over the CTA, the same value in every thread: warp xor tree (each
// step adds the same two operands in both lanes), then the warps' sums in warp
// order.  `red` holds at least blockDim.x / 32 floats.
__device__ __forceinline__ float block_sum(float s, float* red) {
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) s = __fadd_rn(s, __shfl_xor_sync(kFull, s, m));
  const int nw = blockDim.x >> 5;
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  float t = red[0];
  for (int i = 1; i < nw; ++i) t = __fadd_rn(t, red[i]);
  __syncthreads();
  return t;
}

__device__ __forceinline__ float rms_scale(const NormArgs& p, float sumsq) {
  const float var = p.inv_k != 0.0f ? __fmul_rn(sumsq, p.inv_k) : __fdiv_rn(sumsq, static_cast<float>(p.K));
  return rsqrtf(__fadd_rn(var, p.eps));
}

// h of 8 elements (signs applied into v), and h stored when requested.
__device__ __forceinline__ void rms_apply8(const NormArgs& p, size_t off, int k, const float (&xf)[8], float r,
                                           const float (&wt)[8], uint32_t sbits, float (&v)[8]) {
  uint32_t hb[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const float y = __bfloat162float(__float2bfloat16_rn(__fmul_rn(xf[e], r)));
    hb[e] = __bfloat16_as_ushort(__float2bfloat16_rn(__fmul_rn(y, wt[e])));
    v[e] = __uint_as_float((hb[e] << 16) ^ (((sbits >> e) & 1u) << 31));
  }
  if (p.out_normed != nullptr)
    *reinterpret_cast<uint4*>(p.out_normed + off + k) =
        make_uint4(hb[0] | (hb[1] << 16), hb[2] | (hb[3] << 16), hb[4] | (hb[5] << 16), hb[6] | (hb[7] << 16));
}

__device__ __forceinline__ void load8_weight(const uint16_t* w, float (&wt)[8]) {
  const uint4 ww = __ldg(reinterpret_cast<const uint4*>(w));
  const uint32_t ws[4] = {ww.x, ww.y, ww.z, ww.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    wt[2 * i] = __uint_as_float(ws[i] << 16);
    wt[2 * i + 1] = __uint_as_float(ws[i] & 0xFFFF0000u);
  }
}

// block128: one CTA per row (rows strided over the grid) of G*LPG threads;
// warp w holds groups GPW*w .. GPW*w+GPW-1 with LPG lanes per group and
// 128/LPG values per lane, the layout of rht_block128_kernel<LPG>.
template <int LPG>
__global__ void __launch_bounds__(1024) rht_block128_addnorm_kernel(const NormArgs p) {
  constexpr int J = 16 / LPG, GPW = 32 / LPG;
  __shared__ float red[32];
  grid_dependents_launch();
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int slot = lane / LPG, l = lane % LPG, g = w * GPW + slot;
  uint32_t sb[J];
  float wt[J][8];
#pragma unroll
  for (int j = 0; j < J; ++j) {
    sb[j] = sign_bits8(p.signs + g * 128 + j * 8 * LPG + l * 8);
    load8_weight(p.weight + g * 128 + j * 8 * LPG + l * 8, wt[j]);
  }
  grid_dependency_wait();
  for (int row = blockIdx.x; row < p.M; row += gridDim.x) {
    const size_t off = static_cast<size_t>(row) * p.K;
    float xf[J][8];
    float ss = 0.0f;
#pragma unroll
    for (int j = 0; j < J; ++j) ss = __fadd_rn(ss, load8_add(p, off, g * 128 + j * 8 * LPG + l * 8, xf[j]));
    const float r = rms_scale(p, block_sum(ss, red));
    float v[J][8];
#pragma unroll
    for (int j = 0; j < J; ++j) rms_apply8(p, off, g * 128 + j * 8 * LPG + l * 8, xf[j], r, wt[j], sb[j], v[j]);
    block128_quant_group<LPG>(v, l, true, p.clamp_lo, p.packed ? p.packed + off / 2 : nullptr,
                              p.codes8 ? p.codes8 + off : nullptr, p.scale + static_cast<size_t>(row) * p.G, g);
  }
}

// row_DH, K = 4096: the layout of rht_rowdh4096_kernel (one CTA of 128 threads per row).
__global__ void __launch_bounds__(128) rht_rowdh4096_addnorm_kernel(const NormArgs p) {
  constexpr int K = 4096, G = 32;
  __shared__ __align__(16) float sh[padded(K)];
  __shared__ float red[4];
  grid_dependents_launch();
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  uint32_t sb[4];
  float wt[4][8];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    sb[j] = sign_bits8(p.signs + w * 1024 + j * 256 + l * 8);
    load8_weight(p.weight + w * 1024 + j * 256 + l * 8, wt[j]);
  }
  grid_dependency_wait();
  for (int row = blockIdx.x; row < p.M; row += gridDim.x) {
    const size_t off = static_cast<size_t>(row) * K;
    float xf[4][8];
    float ss = 0.0f;
#pragma unroll
    for (int j = 0; j < 4; ++j) ss = __fadd_rn(ss, load8_add(p, off, w * 1024 + j * 256 + l * 8, xf[j]));
    const float r = rms_scale(p, block_sum(ss, red));
    float v[4][8];
#pragma unroll
    for (int j = 0; j < 4; ++j) rms_apply8(p, off, w * 1024 + j * 256 + l * 8, xf[j], r, wt[j], sb[j], v[j]);
    rowdh4096_local_stages(v, l);
    rowdh4096_quant_row(v, sh, w, l, p.clamp_lo, p.packed ? p.packed + off / 2 : nullptr,
                        p.codes8 ? p.codes8 + off : nullptr, p.scale + static_cast<size_t>(row) * G);
  }
}

// ============================================================ host launchers
constexpr int kRowDH12288Smem = padded(12288) * 4;

template <bool SILU>
static int launch_rht_quant_t(const void* x, const void* signs, void* packed, void* codes8, void* scale, int64_t m,
                              int64_t k, int layout, int clamp_lo, cudaStream_t stream) {
  const int sms = device_sm_count();
  if (sms <= 0) return NV4_ERR_CUDA;
  if (layout == NV4_LAYOUT_BLOCK128) {
    Block128Args a;
    a.x = static_cast<const uint16_t*>(x);
    a.signs = static_cast<const int8_t*>(signs);
    a.packed = static_cast<uint8_t*>(packed);
    a.codes8 = static_cast<int8_t*>(codes8);
    a.scale = static_cast<uint16_t*>(scale);
    a.M = static_cast<int>(m);
    a.K = static_cast<int>(k);
    a.G = static_cast<int>(k / 128);
    a.clamp_lo = clamp_lo;
    a.x_stride = static_cast<int>(SILU ? 2 * k : k);
    // Decode-sized batches: 16 lanes per group (8 values each) and 4-warp CTAs,
    // so the few rows spread over many SMs with little work per lane; large
    // batches: 4 lanes per group, 8-warp CTAs.
    const bool small = m <= 256;
    const int lpg = small ? 16 : 4;
    const int gpw = 32 / lpg, wpb = small ? 4 : 8;
    a.ncb = (a.G + gpw - 1) / gpw;
    const int64_t tasks = m * a.ncb;
    int64_t warps = std::min<int64_t>(tasks, static_cast<int64_t>(sms) * 32);
    warps = std::max<int64_t>(a.ncb, (warps / a.ncb) * a.ncb);
    a.warps_used = static_cast<int>(warps);
    const int blocks = static_cast<int>((warps + wpb - 1) / wpb);
    // Programmatic dependent launch: the kernels read only the sign vector before
    // griddepcontrol.wait and write nothing before it, so they may start while
    // the kernel before them in the stream drains.
    if (lpg == 16)
      return launch_kernel(rht_block128_kernel<16, SILU>, dim3(blocks), dim3(32 * wpb), 0, stream, true, a);
    return launch_kernel(rht_block128_kernel<4, SILU>, dim3(blocks), dim3(32 * wpb), 0, stream, true, a);
  }
  RowDHArgs a;
  a.x = static_cast<const uint16_t*>(x);
  a.signs = static_cast<const int8_t*>(signs);
  a.packed = static_cast<uint8_t*>(packed);
  a.codes8 = static_cast<int8_t*>(codes8);
  a.scale = static_cast<uint16_t*>(scale);
  a.M = static_cast<int>(m);
  a.clamp_lo = clamp_lo;
  a.x_stride = static_cast<int>(SILU ? 2 * k : k);
  if (k == 4096) {
    const int blocks = static_cast<int>(std::min<int64_t>(m, static_cast<int64_t>(sms) * 8));
    return launch_kernel(rht_rowdh4096_kernel<SILU>, dim3(blocks), dim3(128), 0, stream, true, a);
  }
  static bool attr_set[64] = {};
  const int dev = current_device();
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    if (cudaFuncSetAttribute(rht_rowdh12288_kernel<SILU>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kRowDH12288Smem) != cudaSuccess)
      return NV4_ERR_CUDA;
    attr_set[dev] = true;
  }
  const int blocks = static_cast<int>(std::min<int64_t>(m, static_cast<int64_t>(sms) * 4));
  return launch_kernel(rht_rowdh12288_kernel<SILU>, dim3(blocks), dim3(128), kRowDH12288Smem, stream, true, a);
}

// `packed` and/or `codes8` receive the codes (at least one is non-null).
int launch_rht_quant(const void* x, const void* signs, void* packed, void* codes8, void* scale, int64_t m, int64_t k,
                     int layout, int clamp_lo, cudaStream_t stream) {
  return launch_rht_quant_t<false>(x, signs, packed, codes8, scale, m, k, layout, clamp_lo, stream);
}

// Same, with the prep input RMSNorm(x + residual) (residual may be null).
int launch_add_rmsnorm_rht_quant(const void* x, const void* residual, const void* weight, float eps,
                                 const void* signs, void* packed, void* codes8, void* scale, void* out_residual,
                                 void* out_normed, int64_t m, int64_t k, int layout, int clamp_lo,
                                 cudaStream_t stream) {
  const int sms = device_sm_count();
  if (sms <= 0) return NV4_ERR_CUDA;
  NormArgs a;
  a.x = static_cast<const uint16_t*>(x);
  a.residual = static_cast<const uint16_t*>(residual);
  a.weight = static_cast<const uint16_t*>(weight);
  a.out_residual = static_cast<uint16_t*>(out_residual);
  a.out_normed = static_cast<uint16_t*>(out_normed);
  a.signs = static_cast<const int8_t*>(signs);
  a.packed = static_cast<uint8_t*>(packed);
  a.codes8 = static_cast<int8_t*>(codes8);
  a.scale = static_cast<uint16_t*>(scale);
  a.eps = eps;
  a.inv_k = (k & (k - 1)) == 0 ? 1.0f / static_cast<float>(k) : 0.0f;  // a power of two: exact
  a.M = static_cast<int>(m);
  a.K = static_cast<int>(k);
  a.G = static_cast<int>(k / 128);
  a.clamp_lo = clamp_lo;
  const int blocks = static_cast<int>(std::min<int64_t>(m, static_cast<int64_t>(sms) * 4));
  if (layout == NV4_LAYOUT_BLOCK128) {
    if (k % 512 || k > 16384) return NV4_ERR_UNSUPPORTED;
    // 16 lanes per group (8 values each) while a row fits in 1024 threads
    if (k <= 8192)
      return launch_kernel(rht_block128_addnorm_kernel<16>, dim3(blocks), dim3(static_cast<unsigned>(k / 8)), 0,
                           stream, true, a);
    return launch_kernel(rht_block128_addnorm_kernel<8>, dim3(blocks), dim3(static_cast<unsigned>(k / 16)), 0,
                         stream, true, a);
  }
  if (k != 4096) return NV4_ERR_UNSUPPORTED;
  return launch_kernel(rht_rowdh4096_addnorm_kernel, dim3(blocks), dim3(128), 0, stream, true, a);
}

// Same, with the prep input computed from a gate/up row [m, 2k] as bf16(silu(gate) * up).
int launch_silu_mul_rht_quant(const void* gate_up, const void* signs, void* packed, void* codes8, void* scale,
                              int64_t m, int64_t k, int layout, int clamp_lo, cudaStream_t stream) {
  return launch_rht_quant_t<true>(gate_up, signs, packed, codes8, scale, m, k, layout, clamp_lo, stream);
}

}  // namespace nv4
