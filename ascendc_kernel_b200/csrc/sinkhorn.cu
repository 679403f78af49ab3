// Sinkhorn (mHC) normalisation of [n_mat, 4, 4] fp32 matrices.
//
// Semantics (reference/task3_v0_ref.py:8-14):
//   y = softmax(x, -1) + eps
//   y = y / (sum(y, -2) + eps)
//   repeat-1 times: y = y / (sum(y, -1) + eps); y = y / (sum(y, -2) + eps)
// i.e. the softmax (a row normalisation) plus 2*repeat-1 further alternating
// column/row normalisations, all in fp32 with IEEE division.
//
// B200 mapping: the op is latency bound (64 KB at the reference shape), so the
// work is spread as wide as it goes: one thread per matrix element, 16 lanes
// per matrix (lane 4r + c of its half-warp holds element (r, c)), no shared
// memory and no synchronisation beyond warp shuffles. A row or column sum
// gathers its four values with four shuffles and adds them in index order
// (r = 0..3 / c = 0..3) like the reference's sequential reductions, so every
// lane of the row (column) computes the same sum bit for bit; the softmax uses
// expf on (x - rowmax) and divides by the sum. Loads and stores are one
// coalesced 4-byte access per thread (a warp covers two matrices, 128 B).
#include "common.cuh"
#include "host_util.h"

namespace dsa {
namespace {

constexpr int kSinkThreads = 128;

__global__ void __launch_bounds__(kSinkThreads) sinkhorn4_kernel(const float* x, float* y,
                                                                 int64_t n_mat, int repeat,
                                                                 float eps) {
  const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int lane = threadIdx.x & 31;
  const int g = lane & 16;              // first lane of this matrix in the warp
  const int r = (lane >> 2) & 3, c = lane & 3;
  const bool valid = (t >> 4) < n_mat;  // whole matrices are valid or not
  // y may alias x: each element is read by its own thread before it writes it
  float a = valid ? x[t] : 0.f;
  // the four values of this element's row (k = column) or column (k = row)
  auto row_val = [&](float v, int k) { return __shfl_sync(0xFFFFFFFFu, v, g + 4 * r + k); };
  auto col_val = [&](float v, int k) { return __shfl_sync(0xFFFFFFFFu, v, g + 4 * k + c); };
  // softmax over the last dim, then + eps
  {
    const float v0 = row_val(a, 0), v1 = row_val(a, 1), v2 = row_val(a, 2), v3 = row_val(a, 3);
    const float mx = fmaxf(fmaxf(v0, v1), fmaxf(v2, v3));
    const float e = expf(__fsub_rn(a, mx));
    const float e0 = row_val(e, 0), e1 = row_val(e, 1), e2 = row_val(e, 2), e3 = row_val(e, 3);
    const float s = __fadd_rn(__fadd_rn(__fadd_rn(e0, e1), e2), e3);
    a = __fadd_rn(__fdiv_rn(e, s), eps);
  }
  auto col_norm = [&]() {
    const float v0 = col_val(a, 0), v1 = col_val(a, 1), v2 = col_val(a, 2), v3 = col_val(a, 3);
    const float s = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(v0, v1), v2), v3), eps);
    a = __fdiv_rn(a, s);
  };
  auto row_norm = [&]() {
    const float v0 = row_val(a, 0), v1 = row_val(a, 1), v2 = row_val(a, 2), v3 = row_val(a, 3);
    const float s = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(v0, v1), v2), v3), eps);
    a = __fdiv_rn(a, s);
  };
  col_norm();
  for (int it = 1; it < repeat; ++it) {
    row_norm();
    col_norm();
  }
  if (valid) y[t] = a;
}

}  // namespace
}  // namespace dsa

extern "C" int dsa_sinkhorn_fwd(const float* x, float* y, int64_t n_mat, int n, int repeat,
                                float eps, void* stream) {
  if (x == nullptr || y == nullptr || n_mat < 0 || repeat < 1) return DSA_ERR_INVALID_ARGUMENT;
  if (n != 4) return DSA_ERR_UNSUPPORTED;
  if (!dsa::aligned16(x) || !dsa::aligned16(y)) return DSA_ERR_MISALIGNED;
  if (n_mat == 0) return DSA_OK;
  // 16 threads per matrix: the 1024 matrices of the reference shape make 128
  // blocks of 128 threads, one per SM
  if (n_mat > (int64_t{1} << 40)) return DSA_ERR_UNSUPPORTED;
  const int64_t blocks = (n_mat * 16 + dsa::kSinkThreads - 1) / dsa::kSinkThreads;
  if (blocks > 0x7FFFFFFF) return DSA_ERR_UNSUPPORTED;
  dsa::sinkhorn4_kernel<<<static_cast<unsigned>(blocks), dsa::kSinkThreads, 0,
                          static_cast<cudaStream_t>(stream)>>>(x, y, n_mat, repeat, eps);
  return dsa::cuda_status(cudaGetLastError());
}
