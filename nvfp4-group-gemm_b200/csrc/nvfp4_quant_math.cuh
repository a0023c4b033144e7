// NVFP4 quantisation arithmetic shared by the activation quantiser and the GEMM epilogues
// that write NVFP4 output. Two-level scaling, every fp32 operation rounded to nearest (no
// contraction), for one block of 16 values with per-tensor scale sg:
//   d6 = 6 * sg; sf = E4M3_rn_sat(amax16 / d6); enc = 1 / (value(sf) * sg) (0 if sf is 0);
//   q  = E2M1_rn_sat(x * enc)
// so that x ~= value(q) * value(sf) * sg.
#pragma once

#include <cstdint>

namespace nvfp4 {

// Eight fp32 values -> four bytes of packed e2m1 (element 2i in the low nibble of byte i).
__device__ __forceinline__ uint32_t cvt_e2m1x8(const float* v) {
  uint32_t out;
  asm("{\n"
      ".reg .b8 b0, b1, b2, b3;\n"
      "cvt.rn.satfinite.e2m1x2.f32 b0, %2, %1;\n"
      "cvt.rn.satfinite.e2m1x2.f32 b1, %4, %3;\n"
      "cvt.rn.satfinite.e2m1x2.f32 b2, %6, %5;\n"
      "cvt.rn.satfinite.e2m1x2.f32 b3, %8, %7;\n"
      "mov.b32 %0, {b0, b1, b2, b3};\n"
      "}"
      : "=r"(out)
      : "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]));
  return out;
}

// fp32 -> float8_e4m3fn code (round to nearest even, saturate to +-448).
__device__ __forceinline__ uint32_t cvt_e4m3(float v) {
  uint16_t out;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(out) : "f"(0.0f), "f"(v));
  return out & 0xFFu;
}

// Value of a non-negative, non-NaN E4M3 code (exact in fp32).
__device__ __forceinline__ float e4m3_value(uint32_t code) {
  const uint32_t e = (code >> 3) & 0xFu;
  const uint32_t m = code & 0x7u;
  if (e == 0) return static_cast<float>(m) * 0.001953125f;  // m/8 * 2^-6
  return __uint_as_float(((e + 120u) << 23) | (m << 20));   // (1 + m/8) * 2^(e-7)
}

// Scale code of a block whose largest magnitude is amax, and the factor that encodes its
// values (0 when the scale is 0).
__device__ __forceinline__ uint32_t block_scale(float amax, float sg, float d6, float& enc) {
  const uint32_t code = cvt_e4m3(__fdiv_rn(amax, d6));
  const float sval = e4m3_value(code);
  enc = sval > 0.0f ? __fdiv_rn(1.0f, __fmul_rn(sval, sg)) : 0.0f;
  return code;
}

// One whole block of 16 values held by one thread: eight bytes of codes, and its scale code.
__device__ __forceinline__ uint2 quantize16(const float* v, float sg, float d6, uint32_t& code) {
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(v[i]));
  float enc;
  code = block_scale(amax, sg, d6, enc);
  float q[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) q[i] = __fmul_rn(v[i], enc);
  return make_uint2(cvt_e2m1x8(q), cvt_e2m1x8(q + 8));
}

// Byte offset of scale (row, column block c16) in the 128x4-blocked layout of a matrix with
// rest_k = ceil(cols / 64) column blocks of four scales.
__device__ __forceinline__ size_t blocked_sf_offset(int64_t row, int c16, int rest_k) {
  return ((static_cast<size_t>(row >> 7) * rest_k + (c16 >> 2)) * 32 + (row & 31)) * 16 +
         ((row >> 5) & 3) * 4 + (c16 & 3);
}

}  // namespace nvfp4
