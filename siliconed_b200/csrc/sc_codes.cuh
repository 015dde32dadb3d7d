// Exact decoding of the arena's 8-bit codes on the device.
//
// int8 values are stored biased (u = q + 128, an unsigned byte) so that a byte placed under the
// fp32 pattern 0x4B000000 reads 2^23 + u; subtracting 2^23 + 128 leaves q exactly.
// e4m3fn codes are stored as published: the 7 magnitude bits placed at bits 20..26 of an fp32
// read the value times 2^-120 (normal and subnormal alike), and one multiply by 2^120 (exact: a
// power of two, no overflow, no flush to zero in this build) restores it.  0x7F / 0xFF are NaN.
// Every int8 and e4m3 value is exactly representable in bf16, so the high half of each fp32 is the
// bf16 operand with no rounding.
#pragma once

#include <cstdint>

namespace sc {

constexpr float kInt8Magic = 8388736.0f;      // 2^23 + 128
constexpr uint32_t kTwoPow120Bits = 0x7B800000u;

__device__ __forceinline__ float int8_code_to_f32(uint32_t word, int j) {
  // Byte j of `word` under 0x4B0000xx: selector bytes (j, 0x00, 0x00, 0x4B).
  const uint32_t bits = __byte_perm(word, 0x4B000000u, 0x7440u | static_cast<uint32_t>(j));
  return __fsub_rn(__uint_as_float(bits), kInt8Magic);
}

// fp32 pattern of e4m3 code j of `word`, scaled by 2^-120, sign in bit 31.
__device__ __forceinline__ uint32_t e4m3_code_scaled_bits(uint32_t word, int j) {
  const int32_t top = static_cast<int32_t>(__byte_perm(word, 0u, 0x0444u | (static_cast<uint32_t>(j) << 12)));
  return static_cast<uint32_t>(top >> 4) & 0x87F00000u;
}

template <bool kNaNCodes>
__device__ __forceinline__ float e4m3_code_to_f32(uint32_t word, int j) {
  const float v = __fmul_rn(__uint_as_float(e4m3_code_scaled_bits(word, j)), __uint_as_float(kTwoPow120Bits));
  if (kNaNCodes) {
    if (((word >> (8 * j)) & 0x7Fu) == 0x7Fu) return __uint_as_float(0x7FC00000u);
  }
  return v;
}

// Low half = bf16 of `lo`, high half = bf16 of `hi` (truncation: exact for these values).
__device__ __forceinline__ uint32_t pack_bf16_hi(float lo, float hi) {
  return __byte_perm(__float_as_uint(lo), __float_as_uint(hi), 0x7632u);
}

// 16 codes (one uint4, K order) -> 16 bf16 (two uint4, K order).
template <int kKind, bool kNaNCodes>
__device__ __forceinline__ void codes16_to_bf16(const uint4 in, uint4& lo, uint4& hi) {
  const uint32_t w[4] = {in.x, in.y, in.z, in.w};
  uint32_t r[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float f0, f1, f2, f3;
    if (kKind == 1) {
      f0 = int8_code_to_f32(w[i], 0);
      f1 = int8_code_to_f32(w[i], 1);
      f2 = int8_code_to_f32(w[i], 2);
      f3 = int8_code_to_f32(w[i], 3);
    } else {
      f0 = e4m3_code_to_f32<kNaNCodes>(w[i], 0);
      f1 = e4m3_code_to_f32<kNaNCodes>(w[i], 1);
      f2 = e4m3_code_to_f32<kNaNCodes>(w[i], 2);
      f3 = e4m3_code_to_f32<kNaNCodes>(w[i], 3);
    }
    r[2 * i] = pack_bf16_hi(f0, f1);
    r[2 * i + 1] = pack_bf16_hi(f2, f3);
  }
  lo = make_uint4(r[0], r[1], r[2], r[3]);
  hi = make_uint4(r[4], r[5], r[6], r[7]);
}

// One stored code as fp32 (the slow, general path: dequantization export, GEMV).
template <int kKind>
__device__ __forceinline__ float code_to_f32(uint8_t code) {
  if (kKind == 1) return static_cast<float>(static_cast<int>(code) - 128);
  return e4m3_code_to_f32<true>(static_cast<uint32_t>(code), 0);
}

// fp32 -> bf16 bits, nearest-even; a NaN stays a quiet NaN with its sign and high payload
// (the rounding rule of the reference's bf16 kernels).
__device__ __forceinline__ uint16_t f32_to_bf16_rne(float f) {
  const uint32_t u = __float_as_uint(f);
  if ((u & 0x7FFFFFFFu) > 0x7F800000u) return static_cast<uint16_t>((u >> 16) | 0x40u);
  return static_cast<uint16_t>((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
}

}  // namespace sc
