// INT4 -> fp16 / fp32 decode of one packed word (eight codes along K).
//
// Word layout: logical k (0..7) lives in nibble slot (k odd ? 4 + k/2 : k/2),
// i.e. slots 0..3 hold k = 0,2,4,6 and slots 4..7 hold k = 1,3,5,7.  Slot s and
// slot s+4 are therefore exactly 16 bits apart and hold the adjacent pair
// (k = 2s, k = 2s+1): one 32-bit AND/OR over the word yields both halves of a
// packed pair already in ascending-k order.  That is why the format
// interleaves the codes, and every decode below relies on it.
#pragma once

#include "ng_common.cuh"

namespace ngb {

__device__ __forceinline__ __half2 h2_from_bits(uint32_t b) {
  __half2_raw r;
  r.x = static_cast<unsigned short>(b & 0xFFFFu);
  r.y = static_cast<unsigned short>(b >> 16);
  return __half2(r);
}

__device__ __forceinline__ uint32_t h2_bits(__half2 h) {
  __half2_raw r = static_cast<__half2_raw>(h);
  return static_cast<uint32_t>(r.x) | (static_cast<uint32_t>(r.y) << 16);
}

// ---------------------------------------------------------------------------
// fp16 decode (magic-number method).
//
// An fp16 with biased exponent 25 and zero mantissa is 1024.0 (0x6400); its
// mantissa ulp is exactly 1, so OR-ing a code u into bits 0..3 of each half
// gives 1024 + u and OR-ing it into bits 4..7 gives 1024 + 16u -- no integer
// to float conversion.  Four AND/ORs (two on the word, two on the word >> 8)
// extract the four (k even, k odd) pairs; the offset and the zero point 8 are
// removed with one packed subtract (low slots) or one packed fma by 1/16 (high
// slots).  Every intermediate is an integer below 2048, so the result u - 8 is
// exact.
// ---------------------------------------------------------------------------
constexpr uint32_t kF16Magic = 0x64006400u;      // {1024, 1024}
constexpr uint32_t kF16Bias = 0x64086408u;       // {1032, 1032} = 1024 + 8
constexpr uint32_t kF16Sixteenth = 0x2C002C00u;  // {1/16, 1/16}
constexpr uint32_t kF16NegBias16 = 0xD480D480u;  // {-72, -72}  = -(1024/16 + 8)

// w[i] = (u(k=2i) - 8, u(k=2i+1) - 8) for i = 0..3, exact.
__device__ __forceinline__ void decode8_f16(uint32_t q, __half2 (&w)[4]) {
  const uint32_t q8 = q >> 8;
  const uint32_t p01 = and_or(q, 0x000F000Fu, kF16Magic);   // slots 0,4 -> k 0,1 : 1024+u
  const uint32_t p23 = and_or(q, 0x00F000F0u, kF16Magic);   // slots 1,5 -> k 2,3 : 1024+16u
  const uint32_t p45 = and_or(q8, 0x000F000Fu, kF16Magic);  // slots 2,6 -> k 4,5
  const uint32_t p67 = and_or(q8, 0x00F000F0u, kF16Magic);  // slots 3,7 -> k 6,7
  const __half2 bias = h2_from_bits(kF16Bias);
  const __half2 sixteenth = h2_from_bits(kF16Sixteenth);
  const __half2 nbias16 = h2_from_bits(kF16NegBias16);
  w[0] = __hsub2(h2_from_bits(p01), bias);
  w[1] = __hfma2(h2_from_bits(p23), sixteenth, nbias16);
  w[2] = __hsub2(h2_from_bits(p45), bias);
  w[3] = __hfma2(h2_from_bits(p67), sixteenth, nbias16);
}

// ---------------------------------------------------------------------------
// fp32 decode (magic-number method, one exponent per slot position).
//
// In an fp32 of value 2^E, mantissa bit b weighs 2^(E-23+b).  For a nibble at
// bits 4j..4j+3 (j = 0..3) choose E = 23 - 4j, so bit 4j weighs exactly 1 and
// OR-ing the nibble into that float's mantissa gives 2^(23-4j) + u exactly.
// The low half of the word holds slots 0..3 (even k), the word >> 16 holds
// slots 4..7 (odd k), so j selects the pair (k = 2j, k = 2j+1) and the same
// magic serves both lanes of a packed fp32x2.  Subtracting 2^(23-4j) + 8
// (exactly representable) leaves u - 8.
// ---------------------------------------------------------------------------
__host__ __device__ constexpr uint32_t f32_magic_bits(int j) {
  return static_cast<uint32_t>(150 - 4 * j) << 23;  // 2^(23 - 4j)
}

// 2^(23-4j) + 8 as fp32 bits: +8 is mantissa bit 3 + 4j at that exponent.
__host__ __device__ constexpr uint32_t f32_bias_bits(int j) {
  return f32_magic_bits(j) | (1u << (3 + 4 * j));
}

// Returns the exact pair (u(k=2j) - 8, u(k=2j+1) - 8) as fp32x2.
template <int J>
__device__ __forceinline__ f2 decode_pair_f32(uint32_t q, uint32_t q16) {
  const uint32_t lo = and_or(q, 0xFu << (4 * J), f32_magic_bits(J));
  const uint32_t hi = and_or(q16, 0xFu << (4 * J), f32_magic_bits(J));
  const f2 bias = f2_from_bits(f32_bias_bits(J), f32_bias_bits(J));
  f2 d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d.v) : "l"(f2_from_bits(lo, hi).v), "l"(bias.v));
  return d;
}

// Plain shift / mask decode of logical offset k (0..7), no tricks; u - 8.
__device__ __forceinline__ int code_minus8(uint32_t q, int k) {
  const int slot = (k & 1) ? 4 + (k >> 1) : (k >> 1);
  return static_cast<int>((q >> (4 * slot)) & 0xFu) - 8;
}

}  // namespace ngb
