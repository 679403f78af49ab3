// Exact int8 slicing of bf16 rows for the indexer projections.
//
// For a row with max|x| < 2^sigma, every element is written in units of
// 2^(sigma - 21) as the integer Xs = floor(x / 2^(sigma-21)), |Xs| <= 2^21 (rows
// below 2^-106 use sign(x) floor(|x| / 2^(sigma-21)) instead); the bits below
// the unit go into a remainder r, |r| < 2^(sigma-21). Xs is cut into its
// two's-complement bit fields
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

// The three slice words (4 elements each) of four two's-complement values
// X0..X3 (|X| <= 2^21): S1 = bits 14..21, S2 = bits 7..13, S3 = bits 0..6.
__device__ __forceinline__ void slice_words(uint32_t x0, uint32_t x1, uint32_t x2, uint32_t x3,
                                            uint32_t& s1, uint32_t& s2, uint32_t& s3) {
  const uint32_t a01 = __byte_perm(x0, x1, 0x5410u), a23 = __byte_perm(x2, x3, 0x5410u);
  const uint32_t b01 = __byte_perm(x0, x1, 0x6521u), b23 = __byte_perm(x2, x3, 0x6521u);
  s3 = __byte_perm(a01, a23, 0x6420u) & 0x7F7F7F7Fu;
  s2 = __byte_perm(a01 >> 7, a23 >> 7, 0x6420u) & 0x7F7F7F7Fu;
  s1 = __byte_perm(b01 >> 6, b23 >> 6, 0x6420u);
}

struct SplitSeg {
  const uint16_t* src;  // bf16 [rows, K]
  int64_t rows;
  int8_t* slices;       // 3 planes [rows, K]
  int* sig;
  float* err;
  float* n3;
  int* span;            // nullptr: not wanted
};

// One row per warp. NC: 256-element chunks per row (lane l holds elements
// [256 j + 8 l, +8) of chunk j). SPAN: also write the row's bit span.
template <int NC, bool SPAN>
__device__ __forceinline__ void split_row(const SplitSeg& sg, int64_t row, int K, int lane) {
  const uint16_t* src = sg.src + row * K;
  // each pass reads the row again (the second read hits L1), so that no chunk
  // has to stay in registers between the passes
  auto load = [&](int j, uint32_t (&w)[4]) {
    const int c = j * 256 + lane * 8;
    w[0] = w[1] = w[2] = w[3] = 0u;
    if (c < K) {
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(src + c));
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

  float rsum = 0.f;  // sum |r| / 2^sigma, rounded up
  uint32_t s3sq = 0;  // sum S3^2 < 2^24 for K <= 1024
  const int64_t plane = sg.rows * K;
  int8_t* dst = sg.slices + row * K;
  const int se = 21 - sigma;
  if (finite && se <= 127) {
    // y = x 2^(21 - sigma) (|y| < 2^21, exact), Xs = floor(y) from the rounded-down
    // add of 1.5 2^23 (the sum stays in [2^23, 2^24), whose grid is the integers),
    // r = y - Xs in [0, 1) (exact) into the bound; pairs of elements per instruction
    const uint64_t scale2 = f2_pack(__int_as_float((se + 127) << 23), __int_as_float((se + 127) << 23));
    const uint64_t magic2 = f2_pack(0x1.8p23f, 0x1.8p23f);
    const uint64_t unit2 = f2_pack(0x1p-21f, 0x1p-21f);
    uint64_t rs2 = f2_pack(0.f, 0.f);
#pragma unroll
    for (int j = 0; j < NC; ++j) {
      uint32_t w[4];
      load(j, w);
      uint32_t X[8];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint64_t x2 = f2_pack(__uint_as_float(w[q] << 16), __uint_as_float(w[q] & 0xFFFF0000u));
        const uint64_t y2 = f2_mul(x2, scale2);
        const uint64_t t2 = f2_add_rm(y2, magic2);
        rs2 = f2_fma_rp(f2_sub(y2, f2_sub(t2, magic2)), unit2, rs2);
        float t0, t1;
        f2_unpack(t2, t0, t1);
        X[2 * q] = __float_as_uint(t0) - 0x4B400000u;
        X[2 * q + 1] = __float_as_uint(t1) - 0x4B400000u;
      }
      uint32_t s1[2], s2[2], s3[2];
      slice_words(X[0], X[1], X[2], X[3], s1[0], s2[0], s3[0]);
      slice_words(X[4], X[5], X[6], X[7], s1[1], s2[1], s3[1]);
      s3sq = __dp4a(s3[0], s3[0], s3sq);
      s3sq = __dp4a(s3[1], s3[1], s3sq);
      const int c = j * 256 + lane * 8;
      if (c < K) {
        *reinterpret_cast<uint2*>(dst + c) = make_uint2(s1[0], s1[1]);
        *reinterpret_cast<uint2*>(dst + plane + c) = make_uint2(s2[0], s2[1]);
        *reinterpret_cast<uint2*>(dst + 2 * plane + c) = make_uint2(s3[0], s3[1]);
      }
    }
    float r0, r1;
    f2_unpack(rs2, r0, r1);
    rsum = __fadd_ru(r0, r1);
    // for sigma > 14 a bf16 below 2^(sigma - 147) scales to a float subnormal,
    // where the product may round (by at most 2^-150, so at most 2^-161 in units
    // of 2^sigma over the row): the smallest float covers it
    if (sigma > 14) rsum = __fadd_ru(rsum, 0x1p-149f);
  } else {
    // rows below 2^-106 (and rows holding Inf / NaN, whose slices are never
    // used): integer arithmetic, X = sign(x) floor(|x| / 2^(sigma - 21))
#pragma unroll
    for (int j = 0; j < NC; ++j) {
      uint32_t w[4];
      load(j, w);
      uint32_t X[8];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint32_t b = (w[q] >> (16 * h)) & 0xFFFFu;
          const uint32_t e = (b >> 7) & 0xFFu, m = b & 0x7Fu;
          const uint32_t M = e ? (m | 0x80u) : m;
          const int eb = e ? static_cast<int>(e) : 1;
          const int sh = eb - 113 - sigma;  // |x| / 2^(sigma - 21) = M 2^sh
          uint32_t Xa, rem;
          if (sh >= 0) {
            Xa = sh < 21 ? M << sh : 0u;
            rem = 0;
          } else if (sh > -8) {
            Xa = M >> (-sh);
            rem = M & ((1u << (-sh)) - 1u);
          } else {
            Xa = 0;
            rem = M;
          }
          if (rem) rsum = __fadd_ru(rsum, static_cast<float>(rem) * pow2_up(eb - 134 - sigma));
          const uint32_t sm = static_cast<uint32_t>(static_cast<int32_t>(b << 16) >> 31);
          X[2 * q + h] = (Xa ^ sm) - sm;
        }
      }
      uint32_t s1[2], s2[2], s3[2];
      slice_words(X[0], X[1], X[2], X[3], s1[0], s2[0], s3[0]);
      slice_words(X[4], X[5], X[6], X[7], s1[1], s2[1], s3[1]);
      s3sq = __dp4a(s3[0], s3[0], s3sq);
      s3sq = __dp4a(s3[1], s3[1], s3sq);
      const int c = j * 256 + lane * 8;
      if (c < K) {
        *reinterpret_cast<uint2*>(dst + c) = make_uint2(s1[0], s1[1]);
        *reinterpret_cast<uint2*>(dst + plane + c) = make_uint2(s2[0], s2[1]);
        *reinterpret_cast<uint2*>(dst + 2 * plane + c) = make_uint2(s3[0], s3[1]);
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) rsum = __fadd_ru(rsum, __shfl_xor_sync(0xFFFFFFFFu, rsum, o));
  s3sq = __reduce_add_sync(0xFFFFFFFFu, s3sq);
  if (lane == 0) {
    sg.sig[row] = finite ? sigma : kSigmaNonFinite;
    sg.err[row] = rsum;
    sg.n3[row] = __fsqrt_ru(static_cast<float>(s3sq));  // s3sq < 2^24 converts exactly
    if (SPAN) sg.span[row] = !finite ? (1 << 20) : (top < -(1 << 29) ? 0 : top - low);
  }
}

// Rows of two operands in one launch: warps [0, a.rows) split a's rows, the
// next b.rows warps b's (both with K columns).
template <int NC>
__global__ void row_split_s8_kernel(const SplitSeg a, const SplitSeg b, int K) {
  int64_t row = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row < a.rows) {
    if (a.span != nullptr) split_row<NC, true>(a, row, K, lane);
    else split_row<NC, false>(a, row, K, lane);
    return;
  }
  row -= a.rows;
  if (row >= b.rows) return;
  if (b.span != nullptr) split_row<NC, true>(b, row, K, lane);
  else split_row<NC, false>(b, row, K, lane);
}

}  // namespace

// Slices the rows of two operands (a then b, same K) in one launch; either may
// have no rows, and a null span pointer skips that operand's bit spans.
int launch_row_split2(const void* a_src, int64_t a_rows, void* a_slices, int* a_sig,
                      float* a_err, float* a_n3, int* a_span, const void* b_src, int64_t b_rows,
                      void* b_slices, int* b_sig, float* b_err, float* b_n3, int* b_span, int K,
                      cudaStream_t stream) {
  if (a_rows < 0 || b_rows < 0) return DSA_ERR_INVALID_ARGUMENT;
  const int64_t rows = a_rows + b_rows;
  if (rows == 0) return DSA_OK;
  if (K <= 0 || K > 1024 || K % 8 != 0) return DSA_ERR_UNSUPPORTED;
  const SplitSeg a{static_cast<const uint16_t*>(a_src), a_rows, static_cast<int8_t*>(a_slices),
                   a_sig, a_err, a_n3, a_span};
  const SplitSeg b{static_cast<const uint16_t*>(b_src), b_rows, static_cast<int8_t*>(b_slices),
                   b_sig, b_err, b_n3, b_span};
  const int threads = 256;
  const dim3 g(static_cast<unsigned>((rows * 32 + threads - 1) / threads));
  if (K <= 256) row_split_s8_kernel<1><<<g, threads, 0, stream>>>(a, b, K);
  else if (K <= 512) row_split_s8_kernel<2><<<g, threads, 0, stream>>>(a, b, K);
  else row_split_s8_kernel<4><<<g, threads, 0, stream>>>(a, b, K);
  return cuda_status(cudaGetLastError());
}

}  // namespace dsa
