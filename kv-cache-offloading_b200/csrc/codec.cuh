// Bit-exact number-format helpers for the FP8 KV codec (device side).
//
// The reference quantizer (nanovllm/engine/cpu_prefix_cache.py:20-28) runs as
// torch ops: bf16 amax, fp32 divide by 448, clamp_min(1e-30), round to a bf16
// scale, fp32 divide by that rounded scale, clamp to +-448, round to
// float8_e4m3fn; dequantization multiplies in fp32 and rounds to bf16. Every
// rounding is IEEE round-to-nearest-even, so the kernels reproduce them with
// correctly rounded __fdiv_rn / __fmul_rn (no FTZ: the library is built
// without --use_fast_math), documented PTX cvt instructions and integer RNE.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

namespace kvoff {

// bf16 bit pattern of a NaN row scale: the one the reference quantizer writes
// (torch's fp32 -> bf16 conversion on the CPU).
constexpr uint32_t kBf16NaN = 0xFFFFu;
constexpr float kFp8Max = 448.0f;   // largest finite float8_e4m3fn magnitude
constexpr float kMinScale = 1e-30f; // clamp_min of the reference scale
// RN(1/448). bf16_rne(max(amax * kInvFp8Max, 1e-30)) equals the reference's
// bf16_rne(max(amax / 448, 1e-30)) for every finite bf16 amax (all 32,640 are
// checked by oracle kvo_fast_quotient_mismatches).
constexpr float kInvFp8Max = 1.0f / 448.0f;

__device__ __forceinline__ float bf16_to_f32(uint32_t bits16) {
  return __uint_as_float(bits16 << 16);
}

// fp32 -> bf16, round to nearest even; NaN -> kBf16NaN. Overflow rounds to
// +-Inf exactly as IEEE RNE does (the carry propagates into the exponent).
__device__ __forceinline__ uint32_t f32_to_bf16_rne(float f) {
  const uint32_t u = __float_as_uint(f);
  if ((u & 0x7FFFFFFFu) > 0x7F800000u) return kBf16NaN;
  return (u + 0x7FFFu + ((u >> 16) & 1u)) >> 16;
}

// Two fp32 -> packed float8_e4m3fn pair, RNE with saturation to +-448
// (inputs are already clamped); `lo` lands in the low byte.
__device__ __forceinline__ uint32_t f32x2_to_e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

// Packed float8_e4m3fn pair -> two fp32 (exact: e4m3 is a subset of f16).
__device__ __forceinline__ float2 e4m3x2_to_f32x2(uint32_t pair) {
  uint32_t h2;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h2) : "h"((uint16_t)pair));
  __half2 h;
  *reinterpret_cast<uint32_t*>(&h) = h2;
  return __half22float2(h);
}

// Row scale from the row's amax bit pattern (|bf16| bits, NaN-propagating).
// Returns the bf16 scale bits; the three cases are finite, Inf and NaN rows.
__device__ __forceinline__ uint32_t scale_from_amax(uint32_t amax_bits) {
  if (amax_bits > 0x7F80u) return kBf16NaN;  // a NaN in the row
  if (amax_bits == 0x7F80u) return 0x7F80u;  // +Inf amax -> +Inf scale
  const float s = fmaxf(__fmul_rn(bf16_to_f32(amax_bits), kInvFp8Max), kMinScale);
  return f32_to_bf16_rne(s);
}

// x / s for one element of a finite-scale row, ready for the saturating e4m3
// conversion (cvt ... .satfinite maps |q| > 448 to 448 exactly as the
// reference's clamp(-448, 448) followed by RNE does). Division-free: with
// r = RN(1/s) (one correctly rounded reciprocal per row) and q1 = RN(x * r),
// the residual q1 * s - x is exact in one FMA, and q1 - residual * r refines q1
// to within half an ulp plus a hair of x / s. x / s cannot lie that close to an
// e4m3 rounding boundary without being exactly on it (x and s carry 8
// significant bits, e4m3 midpoints 5), and on it the refinement is exact, so the
// e4m3 byte equals that of IEEE division; computing the residual negated keeps
// the sign of zero quotients. Checked exhaustively against IEEE division over all
// 929,598,054 (x, s) pairs a row can produce (oracle kvo_fast_quotient_mismatches,
// tests/test_quotient_proof.py).
__device__ __forceinline__ float quant_input(float x, float s, float r) {
  const float q1 = __fmul_rn(x, r);
  const float neg_rem = __fmaf_rn(q1, s, -x);
  return __fmaf_rn(-neg_rem, r, q1);
}

// Two fp32 -> packed bf16 pair, round to nearest even (hardware cvt; a NaN
// becomes the canonical 0x7FFF, the encoding CUDA's own conversion writes);
// `lo` lands in the low half.
__device__ __forceinline__ uint32_t f32x2_to_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// e4m3 byte of one element of a row whose scale is Inf or NaN. These rows
// follow IEEE division as the reference's CPU path evaluates it: finite/Inf
// is a signed zero, Inf/Inf is the default NaN (sign set), x/NaN keeps x's
// NaN (with its sign) when x is NaN and otherwise the scale's NaN, whose
// encoding kBf16NaN has the sign set. e4m3 NaN is 0x7F with the sign bit.
__device__ __forceinline__ uint32_t special_row_byte(uint32_t xbits16, uint32_t scale_bits) {
  const uint32_t sign = (xbits16 >> 8) & 0x80u;
  const uint32_t mag = xbits16 & 0x7FFFu;
  if (scale_bits == 0x7F80u) return mag == 0x7F80u ? 0xFFu : sign;
  return mag > 0x7F80u ? (0x7Fu | sign) : 0xFFu;
}

}  // namespace kvoff
