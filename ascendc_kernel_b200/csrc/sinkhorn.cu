// Sinkhorn (mHC) normalisation of [n_mat, 4, 4] fp32 matrices.
//
// Semantics (reference/task3_v0_ref.py:8-14):
//   y = softmax(x, -1) + eps
//   y = y / (sum(y, -2) + eps)
//   repeat-1 times: y = y / (sum(y, -1) + eps); y = y / (sum(y, -2) + eps)
// i.e. the softmax (a row normalisation) plus 2*repeat-1 further alternating
// column/row normalisations, all in fp32 with IEEE division.
//
// B200 mapping: the op is latency bound (64 KB at the reference shape), so one
// thread owns one 4x4 matrix in 16 registers for the whole sequence; there is
// no shared memory and no synchronisation. Loads and stores are 4 x 16-byte
// vector accesses per thread (a warp covers 2 KB of contiguous memory). Sums
// run in index order (r = 0..3 / c = 0..3) like the reference's sequential
// reductions; the softmax uses expf on (x - rowmax) and divides by the sum.
#include "common.cuh"
#include "host_util.h"

namespace dsa {
namespace {

__global__ void __launch_bounds__(128) sinkhorn4_kernel(const float4* x, float4* y,
                                                        int64_t n_mat,
                                                        int repeat, float eps) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n_mat) return;
  float a[4][4];
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const float4 v = x[i * 4 + r];  // y may alias x: each thread reads before it writes
    a[r][0] = v.x;
    a[r][1] = v.y;
    a[r][2] = v.z;
    a[r][3] = v.w;
  }
  // softmax over the last dim, then + eps
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const float mx = fmaxf(fmaxf(a[r][0], a[r][1]), fmaxf(a[r][2], a[r][3]));
    float e[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) e[c] = expf(__fsub_rn(a[r][c], mx));
    const float s = __fadd_rn(__fadd_rn(__fadd_rn(e[0], e[1]), e[2]), e[3]);
#pragma unroll
    for (int c = 0; c < 4; ++c) a[r][c] = __fadd_rn(__fdiv_rn(e[c], s), eps);
  }
  // column normalisation
  auto col_norm = [&]() {
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const float s =
          __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(a[0][c], a[1][c]), a[2][c]), a[3][c]), eps);
#pragma unroll
      for (int r = 0; r < 4; ++r) a[r][c] = __fdiv_rn(a[r][c], s);
    }
  };
  auto row_norm = [&]() {
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const float s =
          __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(a[r][0], a[r][1]), a[r][2]), a[r][3]), eps);
#pragma unroll
      for (int c = 0; c < 4; ++c) a[r][c] = __fdiv_rn(a[r][c], s);
    }
  };
  col_norm();
  for (int it = 1; it < repeat; ++it) {
    row_norm();
    col_norm();
  }
#pragma unroll
  for (int r = 0; r < 4; ++r) y[i * 4 + r] = make_float4(a[r][0], a[r][1], a[r][2], a[r][3]);
}

}  // namespace
}  // namespace dsa

extern "C" int dsa_sinkhorn_fwd(const float* x, float* y, int64_t n_mat, int n, int repeat,
                                float eps, void* stream) {
  if (x == nullptr || y == nullptr || n_mat < 0 || repeat < 1) return DSA_ERR_INVALID_ARGUMENT;
  if (n != 4) return DSA_ERR_UNSUPPORTED;
  if (!dsa::aligned16(x) || !dsa::aligned16(y)) return DSA_ERR_MISALIGNED;
  if (n_mat == 0) return DSA_OK;
  // 32 threads per block spreads the 1024 matrices of the reference shape over
  // 32 SMs; larger batches use 128-thread blocks.
  const int threads = n_mat <= 4096 ? 32 : 128;
  const int64_t blocks = (n_mat + threads - 1) / threads;
  if (blocks > 0x7FFFFFFF) return DSA_ERR_UNSUPPORTED;
  dsa::sinkhorn4_kernel<<<static_cast<unsigned>(blocks), threads, 0,
                          static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const float4*>(x), reinterpret_cast<float4*>(y), n_mat, repeat, eps);
  return dsa::cuda_status(cudaGetLastError());
}
