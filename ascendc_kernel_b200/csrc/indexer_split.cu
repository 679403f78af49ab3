// Exact int8 slicing of bf16 rows for the indexer projections.
//
// For a row with max|x| < 2^sigma, every element is written in units of
// 2^(sigma - 21) as Xs = sign(x) * floor(|x| / 2^(sigma-21)) (an integer with
// |Xs| < 2^21; the bits below the unit go into a remainder r, |r| < 2^(sigma-21)),
// and Xs is cut into its two's-complement bit fields
//     Xs = 2^14 S1 + 2^7 S2 + S3,  S1 in [-128, 127], S2, S3 in [0, 127],
//     x  = 2^(sigma-7) S1 + 2^(sigma-14) S2 + 2^(sigma-21) S3 + r.
// Slices of two rows multiply and accumulate EXACTLY on the int8 tensor cores
// (int32 accumulators: |sum| <= 2^24 per slice pair for K <= 1024). Per row the
// kernel also writes sigma, err = sum|r| / 2^sigma (rounded up), which bounds r.y
// relative to 2^(sigma + sigma_y) for any row y with |y| < 2^sigma_y, and
// n3 = ||S3||_2 (rounded up), which bounds the S3 x S3 product that the
// projections leave out (Cauchy-Schwarz), and, when asked for, span = sigma -
// (lowest set bit position over the row's nonzero elements): the products of two
// rows are all multiples of 2^(lsb_x + lsb_y) below 2^(sigma_x + sigma_y), so when
// span_x + span_y + log2 K <= 53 every partial sum of their dot product is
// exact in fp64, whatever the order.
// K <= 1024 (one 16-byte chunk per lane per 256 elements).
// Rows holding an Inf or NaN get sigma = kSigmaNonFinite, which the projections
// treat as "recompute exactly".
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

// Four bytes (the low byte of each argument) packed into one word.
__device__ __forceinline__ uint32_t pack4(uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  return __byte_perm(__byte_perm(a, b, 0x0040u), __byte_perm(c, d, 0x0040u), 0x5410u);
}

// NC: 256-element chunks per row (lane l holds elements [256 j + 8 l, +8) of chunk j).
// SPAN: also write the row's bit span.
template <int NC, bool SPAN>
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
  // pass 1: the largest magnitude (two elements per operation) and, for the
  // span, the lowest set bit
  uint32_t mx = 0;
  int low = 1 << 30;
#pragma unroll
  for (int j = 0; j < NC; ++j) {
    uint32_t w[4];
    load(j, w);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      mx = __vmaxu2(mx, w[q] & 0x7FFF7FFFu);
      if (SPAN) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint32_t b = (w[q] >> (16 * h)) & 0x7FFFu;
          const uint32_t e = b >> 7, m = b & 0x7Fu;
          const uint32_t M = e ? (m | 0x80u) : m;
          if (M) low = min(low, (e ? static_cast<int>(e) : 1) - 134 + (__ffs(M) - 1));
        }
      }
    }
  }
  mx = __reduce_max_sync(0xFFFFFFFFu, max(mx & 0xFFFFu, mx >> 16));
  if (SPAN) low = __reduce_min_sync(0xFFFFFFFFu, low);
  const bool finite = mx < 0x7F80u;
  const int top = bf16_top(mx);
  const int sigma = top < -(1 << 29) ? 0 : top;

  // pass 2: y = |x| 2^(21 - sigma) (exact scaling), X = floor(y) by the
  // round-toward-zero add of 2^23, the fraction y - X (exact) into err
  float rsum = 0.f;  // sum |r| / 2^sigma, rounded up
  int s3sq = 0;      // sum S3^2 < 2^24 for K <= 1024
  const int64_t plane = rows * K;
  const int se = 21 - sigma;
  const bool fast = finite && se >= -126 && se <= 127;  // the scale is a normal float
  const float scale = fast ? __int_as_float((se + 127) << 23) : 0.f;
#pragma unroll
  for (int j = 0; j < NC; ++j) {
    uint32_t w[4];
    load(j, w);
    uint32_t v[3][8];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t b = (w[q] >> (16 * h)) & 0xFFFFu;
        uint32_t X;
        if (fast) {
          const float y = __uint_as_float((b & 0x7FFFu) << 16) * scale;
          const float t = __fadd_rz(y, 0x1p23f);
          X = __float_as_uint(t) - 0x4B000000u;
          rsum = __fmaf_ru(y - (t - 0x1p23f), 0x1p-21f, rsum);
        } else {  // extreme exponents or Inf/NaN: integer path
          const uint32_t e = (b >> 7) & 0xFFu, m = b & 0x7Fu;
          const uint32_t M = e ? (m | 0x80u) : m;
          const int eb = e ? static_cast<int>(e) : 1;
          const int sh = eb - 113 - sigma;  // X = M * 2^sh
          uint32_t rem;
          if (sh >= 0) {
            X = sh < 21 ? M << sh : 0u;
            rem = 0;
          } else if (sh > -8) {
            X = M >> (-sh);
            rem = M & ((1u << (-sh)) - 1u);
          } else {
            X = 0;
            rem = M;
          }
          if (rem) rsum = __fadd_ru(rsum, static_cast<float>(rem) * pow2_up(eb - 134 - sigma));
        }
        const uint32_t sm = static_cast<uint32_t>(static_cast<int32_t>(b << 16) >> 31);
        const uint32_t Xs = (X ^ sm) - sm;                      // sign(x) X
        const uint32_t v3 = Xs & 127u;
        s3sq += static_cast<int>(v3 * v3);
        const int idx = q * 2 + h;
        v[0][idx] = static_cast<uint32_t>(static_cast<int32_t>(Xs) >> 14);  // S1, arithmetic
        v[1][idx] = (Xs >> 7) & 127u;
        v[2][idx] = v3;
      }
    }
    const int c = j * 256 + lane * 8;
    if (c < K) {
#pragma unroll
      for (int t = 0; t < 3; ++t)
        *reinterpret_cast<uint2*>(slices + t * plane + row * K + c) =
            make_uint2(pack4(v[t][0], v[t][1], v[t][2], v[t][3]),
                       pack4(v[t][4], v[t][5], v[t][6], v[t][7]));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    rsum = __fadd_ru(rsum, __shfl_xor_sync(0xFFFFFFFFu, rsum, o));
    s3sq += __shfl_xor_sync(0xFFFFFFFFu, s3sq, o);
  }
  // for sigma > 14 a bf16 below 2^(sigma - 147) scales to a float subnormal, where
  // the product may round (by at most 2^-150, so 2^-161 in units of 2^sigma over
  // the row): the smallest float covers it
  if (fast && sigma > 14) rsum = __fadd_ru(rsum, 0x1p-149f);
  if (lane == 0) {
    sig[row] = finite ? sigma : kSigmaNonFinite;
    err[row] = rsum;
    n3[row] = __fsqrt_ru(static_cast<float>(s3sq));  // s3sq < 2^24 converts exactly
    if (SPAN) span[row] = !finite ? (1 << 20) : (top < -(1 << 29) ? 0 : top - low);
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
  const dim3 g(static_cast<unsigned>(blocks));
  if (span != nullptr) {
    if (K <= 256)
      row_split_s8_kernel<1, true><<<g, threads, 0, stream>>>(s16, rows, K, s8, sig, err, n3, span);
    else if (K <= 512)
      row_split_s8_kernel<2, true><<<g, threads, 0, stream>>>(s16, rows, K, s8, sig, err, n3, span);
    else
      row_split_s8_kernel<4, true><<<g, threads, 0, stream>>>(s16, rows, K, s8, sig, err, n3, span);
  } else {
    if (K <= 256)
      row_split_s8_kernel<1, false><<<g, threads, 0, stream>>>(s16, rows, K, s8, sig, err, n3, span);
    else if (K <= 512)
      row_split_s8_kernel<2, false><<<g, threads, 0, stream>>>(s16, rows, K, s8, sig, err, n3, span);
    else
      row_split_s8_kernel<4, false><<<g, threads, 0, stream>>>(s16, rows, K, s8, sig, err, n3, span);
  }
  return cuda_status(cudaGetLastError());
}

}  // namespace dsa
