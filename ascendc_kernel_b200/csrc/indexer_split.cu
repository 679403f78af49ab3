// Exact int8 slicing of bf16 rows for the indexer q projection.
//
// A bf16 x is M * 2^(eb - 134) with an integer significand M < 256 (eb the
// biased exponent, 1 for subnormals). For a row with max|x| < 2^sigma, every
// element is written in units of 2^(sigma - 21) as X (an integer < 2^21, the
// bits below the unit truncated toward zero into a remainder r), and X is cut
// into three signed 7-bit slices
//     x = 2^(sigma-7) S1 + 2^(sigma-14) S2 + 2^(sigma-21) S3 + r,   |S_j| <= 127.
// Slices of two rows multiply and accumulate EXACTLY on the int8 tensor cores
// (int32 accumulators: |sum| < 2^24 per slice pair for K <= 1024). Per row the kernel also
// writes sigma, err = sum|r| / 2^sigma (rounded up), which bounds r.y
// relative to 2^(sigma + sigma_y) for any row y with |y| < 2^sigma_y, and
// n3 = ||S3||_2 (rounded up), which bounds the S3 x S3 product that the
// projection leaves out (Cauchy-Schwarz), and span = sigma - (lowest set bit
// position over the row's nonzero elements): the products of two rows are all
// multiples of 2^(lsb_x + lsb_y) below 2^(sigma_x + sigma_y), so when
// span_x + span_y + log2 K <= 53 every partial sum of their dot product is
// exact in fp64, whatever the order.
// K <= 1024 (one 16-byte chunk per lane per 256 elements).
// Rows holding an Inf or NaN get sigma = kSigmaNonFinite, which the projection
// treats as "recompute exactly".
#include "common.cuh"
#include "host_util.h"
#include "numerics.cuh"

namespace dsa {

constexpr int kSigmaNonFinite = 1 << 20;

namespace {

// Leading-bit position + 1 of a bf16 magnitude (x < 2^result), or INT_MIN for 0.
__device__ __forceinline__ int bf16_top(uint32_t bits) {
  const uint32_t e = (bits >> 7) & 0xFFu, m = bits & 0x7Fu;
  const uint32_t M = e ? (m | 0x80u) : m;
  if (M == 0) return -(1 << 30);
  const int eb = e ? static_cast<int>(e) : 1;
  return (31 - __clz(M)) + eb - 134 + 1;
}

// 2^d as a float upper bound for d < -126 (clamped to 2^-126).
__device__ __forceinline__ float pow2_up(int d) {
  d = d < -126 ? -126 : d;
  return __int_as_float((d + 127) << 23);
}

// NC: 256-element chunks per row (lane l holds elements [256 j + 8 l, +8) of chunk j).
template <int NC>
__global__ void row_split_s8_kernel(const uint16_t* __restrict__ src, int64_t rows, int K,
                                    int8_t* __restrict__ slices, int* __restrict__ sig,
                                    float* __restrict__ err, float* __restrict__ n3,
                                    int* __restrict__ span) {
  const int64_t row = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  // each pass reads the row again (the second read hits L1), so that no chunk
  // has to stay in registers between the passes
  auto load = [&](int j, uint32_t (&w)[4]) {
    const int c = j * 256 + lane * 8;
    w[0] = w[1] = w[2] = w[3] = 0u;
    if (c < K) {
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(src + row * K + c));
      w[0] = v.x, w[1] = v.y, w[2] = v.z, w[3] = v.w;
    }
  };
  // sigma: max over elements of (leading bit + 1); non-finite marks the row
  int top = -(1 << 30);
  int low = 1 << 30;  // lowest set bit position of a nonzero element
  bool finite = true;
#pragma unroll
  for (int j = 0; j < NC; ++j) {
    uint32_t w[4];
    load(j, w);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t b = (w[q] >> (16 * h)) & 0xFFFFu;
        finite &= ((b >> 7) & 0xFFu) != 0xFFu;
        top = max(top, bf16_top(b));
        const uint32_t e = (b >> 7) & 0xFFu, m = b & 0x7Fu;
        const uint32_t M = e ? (m | 0x80u) : m;
        if (M) low = min(low, (e ? static_cast<int>(e) : 1) - 134 + (__ffs(M) - 1));
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    top = max(top, __shfl_xor_sync(0xFFFFFFFFu, top, o));
    low = min(low, __shfl_xor_sync(0xFFFFFFFFu, low, o));
  }
  finite = __all_sync(0xFFFFFFFFu, finite);
  const int sigma = top < -(1 << 29) ? 0 : top;

  float rsum = 0.f;  // sum |r| / 2^sigma, rounded up
  int s3sq = 0;      // sum S3^2 < 2^24 for K <= 1024
  const int64_t plane = rows * K;
#pragma unroll
  for (int j = 0; j < NC; ++j) {
    uint32_t w[4];
    load(j, w);
    uint32_t s[3][2] = {{0, 0}, {0, 0}, {0, 0}};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t b = (w[q] >> (16 * h)) & 0xFFFFu;
        const uint32_t e = (b >> 7) & 0xFFu, m = b & 0x7Fu;
        const uint32_t M = e ? (m | 0x80u) : m;
        const int eb = e ? static_cast<int>(e) : 1;
        const int sh = eb - 113 - sigma;  // X = M * 2^sh
        uint32_t X, rem;
        if (sh >= 0) {
          X = M << sh;
          rem = 0;
        } else if (sh > -8) {
          X = M >> (-sh);
          rem = M & ((1u << (-sh)) - 1u);
        } else {
          X = 0;
          rem = M;
        }
        if (rem) rsum = __fadd_ru(rsum, static_cast<float>(rem) * pow2_up(eb - 134 - sigma));
        const bool neg = (b >> 15) & 1u;
        const uint32_t v1 = X >> 14, v2 = (X >> 7) & 127u, v3 = X & 127u;
        s3sq += static_cast<int>(v3 * v3);
        const int idx = q * 2 + h;
        const int byte = (idx & 3) * 8;
        s[0][idx >> 2] |= ((neg ? 0u - v1 : v1) & 0xFFu) << byte;
        s[1][idx >> 2] |= ((neg ? 0u - v2 : v2) & 0xFFu) << byte;
        s[2][idx >> 2] |= ((neg ? 0u - v3 : v3) & 0xFFu) << byte;
      }
    }
    const int c = j * 256 + lane * 8;
    if (c < K) {
#pragma unroll
      for (int t = 0; t < 3; ++t)
        *reinterpret_cast<uint2*>(slices + t * plane + row * K + c) = make_uint2(s[t][0], s[t][1]);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    rsum = __fadd_ru(rsum, __shfl_xor_sync(0xFFFFFFFFu, rsum, o));
    s3sq += __shfl_xor_sync(0xFFFFFFFFu, s3sq, o);
  }
  if (lane == 0) {
    sig[row] = finite ? sigma : kSigmaNonFinite;
    err[row] = rsum;
    n3[row] = __fsqrt_ru(static_cast<float>(s3sq));  // s3sq < 2^24 converts exactly
    span[row] = (top < -(1 << 29) || !finite) ? (finite ? 0 : 1 << 20) : top - low;
  }
}

}  // namespace

int launch_row_split(const void* src, int64_t rows, int K, void* slices, int* sig, float* err,
                     float* n3, int* span, cudaStream_t stream) {
  if (rows <= 0) return DSA_OK;
  if (K <= 0 || K > 1024 || K % 8 != 0) return DSA_ERR_UNSUPPORTED;
  const int threads = 256;
  const int64_t blocks = (rows * 32 + threads - 1) / threads;
  const uint16_t* s16 = static_cast<const uint16_t*>(src);
  int8_t* s8 = static_cast<int8_t*>(slices);
  if (K <= 256)
    row_split_s8_kernel<1><<<static_cast<unsigned>(blocks), threads, 0, stream>>>(
        s16, rows, K, s8, sig, err, n3, span);
  else if (K <= 512)
    row_split_s8_kernel<2><<<static_cast<unsigned>(blocks), threads, 0, stream>>>(
        s16, rows, K, s8, sig, err, n3, span);
  else
    row_split_s8_kernel<4><<<static_cast<unsigned>(blocks), threads, 0, stream>>>(
        s16, rows, K, s8, sig, err, n3, span);
  return cuda_status(cudaGetLastError());
}

}  // namespace dsa
