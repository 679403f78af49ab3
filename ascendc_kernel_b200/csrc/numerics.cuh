// Rounding helpers shared by the Lightning Indexer kernels.
//
// Contract: every bf16 that the indexer produces from a dot product is the
// round-to-nearest-even value of the exact dot product ("correct rounding").
// The tensor cores deliver an fp32 approximation v with |v - exact| <= E for a
// bound E computed from operand norms (see certified_bf16); when the interval
// [v - E, v + E] cannot contain a bf16 rounding boundary, RNE(v) is the
// correctly rounded result. Otherwise the element is recomputed as an fp64 sum
// of the exact products in ascending index order and rounded with
// round_f64_to_bf16 -- the same arithmetic as the CPU oracle.
//
// Error model of the tensor-core accumulator (measured on B200 for bf16
// inputs, fp32 accumulate, K in {64, 256, 1024}, random, wide-range and
// same-sign data): each K=16 MMA step adds at most ~0.5 fp32 ulp of the sum of
// the magnitudes accumulated so far. The kernels use twice that, per step, and
// bound the sum of magnitudes by ||a|| * ||b|| (Cauchy-Schwarz).
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

namespace dsa {

constexpr float kTwoM23 = 1.1920928955078125e-07f;  // 2^-23
constexpr float kTwoM24 = 5.9604644775390625e-08f;  // 2^-24

// RNE of a finite fp32 to bf16 bits.
__device__ __forceinline__ uint32_t f32_to_bf16_rne(float v) {
  uint32_t u = __float_as_uint(v);
  return (u + 0x7FFFu + ((u >> 16) & 1u)) >> 16;
}

// Correctly rounded fp64 -> bf16 bits: round to odd into fp32 (24 bits), then
// RNE into bf16 (8 bits); 24 >= 8 + 2 makes the double rounding exact.
__device__ __forceinline__ uint32_t round_f64_to_bf16(double d) {
  float f = __double2float_rz(d);
  if (static_cast<double>(f) != d) f = __uint_as_float(__float_as_uint(f) | 1u);
  return f32_to_bf16_rne(f);
}

// The CPU oracle rounds a dot product of bf16 inputs by summing the exact fp64
// products in one sequential chain (ascending k) and rounding that sum
// (round_f64_to_bf16). `sum` is the same products summed by a warp: each lane's
// <= 32 terms in order, the lanes by a 5-step xor tree (every lane holds the
// same bits); `mag` the same sum of |products|. Both chains lie within
// (K - 1 + 36) 2^-53 mag (1 + 2^-40) of the exact value, so for K <= 1024 the
// oracle's sum lies within 2^-42 mag of `sum`. When both ends of that interval
// round to the same bf16 (monotone rounding), that is the oracle's result:
// returns true and the bits; false sends the caller to the sequential chain.
__device__ __forceinline__ bool certify_seq_dot_bf16(double sum, double mag, uint32_t* bits) {
  const double bnd = mag * 0x1p-42;
  if (!isfinite(sum) || !isfinite(bnd)) return false;
  const uint32_t lo = round_f64_to_bf16(__dadd_rd(sum, -bnd));
  const uint32_t hi = round_f64_to_bf16(__dadd_ru(sum, bnd));
  *bits = lo;
  return lo == hi;
}

// Certified rounding. v: fp32 approximation of an exact real x with
// |v - x| <= E. Returns true and the bf16 bits of RNE(x) in *bits when that
// can be decided from v alone, false when x may lie on the other side of a
// rounding boundary (the caller then recomputes x exactly).
// RNE is monotone, so if lo = v - E (rounded down) and hi = v + E (rounded up)
// have the same RNE, every x in [lo, hi] rounds to it. *bits is RNE(lo).
__device__ __forceinline__ bool certified_bf16(float v, float E, uint32_t* bits) {
  const float lo = __fsub_rd(v, E);
  const float hi = __fadd_ru(v, E);
  uint32_t pair;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(pair) : "f"(hi), "f"(lo));
  *bits = pair & 0xFFFFu;
  return (pair >> 16) == (pair & 0xFFFFu);
}

// Upper bound of sqrt(sum of squares) accumulated in fp32 as `ss`, n terms.
__device__ __forceinline__ float norm_upper(float ss, int n) {
  return sqrtf(ss * (1.0f + static_cast<float>(n + 4) * kTwoM24)) * (1.0f + 4.0f * kTwoM24);
}

__device__ __forceinline__ float bf16lo_to_f32(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16hi_to_f32(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

// Lowest set bit position (value 2^pos) over the two bf16 of a word; 1 << 30
// when both are zero.
__device__ __forceinline__ int bf16x2_low_bit(uint32_t w) {
  int low = 1 << 30;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const uint32_t b = (w >> (16 * h)) & 0x7FFFu;
    const uint32_t e = b >> 7, m = b & 0x7Fu;
    const uint32_t M = e ? (m | 0x80u) : m;
    if (M) low = min(low, (e ? static_cast<int>(e) : 1) - 134 + (__ffs(M) - 1));
  }
  return low;
}

}  // namespace dsa
