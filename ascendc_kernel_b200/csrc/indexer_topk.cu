// Lightning Indexer top-k for long candidate lists (n_cand > 1024 or
// top-k > 256): the score kernel writes every valid bf16 score of a token to
// a [rows, n_cand] buffer and this kernel sorts them.
//
// Order (reference/task2_v0_ref.py:141-143, canonical tie rule): score
// descending, then candidate index ascending; slots past the token's valid
// count n are -1, valid slots hold k + offset.
//
// One 512-thread block per token. The n scores are loaded in index order and
// sorted by a stable LSD radix sort over the 16-bit orderable score (two 8-bit
// passes). Stability keeps equal scores in index order, which is exactly the
// tie rule. Each warp owns a contiguous range of 32*J elements (lane l of step
// j holds element 32 j + l of it), so a warp's running per-digit counts plus
// the block-wide prefix over warps give every element its stable rank.
#include "common.cuh"
#include "host_util.h"

namespace dsa {
namespace ixt {

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxJ = 16;                  // steps of 32 per warp: n <= 8192
constexpr int kMaxN = kWarps * 32 * kMaxJ;

struct Params {
  const uint16_t* scores;  // [rows, ld] bf16, valid for k < n(t)
  int64_t ld;
  int64_t* out;            // [rows, K]
  int K;
  int64_t S;
  int64_t T;
  int ratio;
  int causal;
  int64_t offset;
  int64_t rows;
};

// Orderable 16-bit image of a bf16 score (-0 counts as +0); larger is better.
__device__ __forceinline__ uint32_t ord16(uint32_t sb) {
  if (sb == 0x8000u) sb = 0;
  return (sb & 0x8000u) ? (~sb & 0xFFFFu) : (sb | 0x8000u);
}

// J: the launch's step bound; jr <= J: steps this row needs (a warp owns
// elements [32 jr warp, 32 jr (warp + 1))).
template <int J>
__device__ __forceinline__ void sort_row(const Params& p, int64_t row, int n, int jr,
                                         uint32_t* buf0, uint32_t* buf1, uint32_t* hist,
                                         uint32_t* scan) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t lt_mask = (1u << lane) - 1u;
  const uint16_t* src = p.scores + row * p.ld;
  const int wbase = warp * 32 * jr;
  uint32_t v[J];
#pragma unroll
  for (int j = 0; j < J; ++j) {
    const int e = wbase + 32 * j + lane;  // element index = candidate k
    // padding elements carry order 0, below every real score, and sort last
    v[j] = (j < jr && e < n)
               ? (ord16(__ldg(src + e)) << 16) | (0xFFFFu - static_cast<uint32_t>(e))
               : 0u;
  }
  uint32_t* cur = buf0;
  uint32_t* nxt = buf1;
#pragma unroll 1
  for (int pass = 0; pass < 2; ++pass) {
    const int shift = 16 + 8 * pass;
    uint32_t* wh = hist + warp * 256;
    // phase A: per-warp running counts per digit and each element's rank in the warp
    reinterpret_cast<uint4*>(wh)[lane * 2] = make_uint4(0, 0, 0, 0);
    reinterpret_cast<uint4*>(wh)[lane * 2 + 1] = make_uint4(0, 0, 0, 0);
    __syncwarp();
    uint32_t rank[J];
#pragma unroll
    for (int j = 0; j < J; ++j) {
      if (j >= jr) break;
      const uint32_t d = 255u - ((v[j] >> shift) & 0xFFu);  // ascending digit = descending score
      const uint32_t peers = __match_any_sync(0xFFFFFFFFu, d);
      rank[j] = wh[d] + static_cast<uint32_t>(__popc(peers & lt_mask));
      __syncwarp();
      if ((peers & lt_mask) == 0) wh[d] += static_cast<uint32_t>(__popc(peers));
      __syncwarp();
    }
    __syncthreads();
    // phase B: offset of (warp, digit) = elements of smaller digits + same digit in earlier warps
    if (tid < 256) {
      const int d = tid;  // one thread per digit
      uint32_t tot = 0;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        const uint32_t c = hist[w * 256 + d];
        hist[w * 256 + d] = tot;  // exclusive prefix over warps
        tot += c;
      }
      // block-wide exclusive scan of tot over digits
      uint32_t incl = tot;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t x = __shfl_up_sync(0xFFFFFFFFu, incl, o);
        if (lane >= o) incl += x;
      }
      if (lane == 31) scan[warp] = incl;
      named_bar_sync(1, 256);
      uint32_t wpre = 0;
#pragma unroll
      for (int w = 0; w < 8; ++w) wpre += w < warp ? scan[w] : 0u;
      const uint32_t base = wpre + incl - tot;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) hist[w * 256 + d] += base;
    }
    __syncthreads();
    // phase C: scatter
#pragma unroll
    for (int j = 0; j < J; ++j) {
      if (j >= jr) break;
      const uint32_t d = 255u - ((v[j] >> shift) & 0xFFu);
      nxt[wh[d] + rank[j]] = v[j];
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < J; ++j) {
      if (j >= jr) break;
      v[j] = nxt[wbase + 32 * j + lane];
    }
    uint32_t* t = cur;
    cur = nxt;
    nxt = t;
    __syncthreads();
  }
  // cur holds the keys in output order (padding last)
  int64_t* o = p.out + row * p.K;
  const int take = n < p.K ? n : p.K;
  for (int i = tid; i < p.K; i += kThreads) {
    o[i] = i < take ? static_cast<int64_t>(0xFFFFu - (cur[i] & 0xFFFFu)) + p.offset
                    : static_cast<int64_t>(-1);
  }
}

// J: step bound of this launch (n_cand <= kThreads * J).
template <int J>
__global__ void __launch_bounds__(kThreads)
    topk_sort_kernel(const Params p) {
  extern __shared__ uint32_t sm[];
  uint32_t* hist = sm;                       // [warps][256]
  uint32_t* scan = hist + kWarps * 256;      // [8] (padded to 32)
  uint32_t* buf0 = scan + 32;                // [kThreads * J] x 2
  uint32_t* buf1 = buf0 + kThreads * J;
  for (int64_t row = blockIdx.x; row < p.rows; row += gridDim.x) {
    const int64_t t = row % p.S;
    int64_t n = p.T;
    if (p.causal) {
      n = (t + 1) / p.ratio;
      if (n > p.T) n = p.T;
    }
    int jr = static_cast<int>((n + kThreads - 1) / kThreads);  // steps per warp
    if (jr < 1) jr = 1;
    sort_row<J>(p, row, static_cast<int>(n), jr, buf0, buf1, hist, scan);
    __syncthreads();
  }
}

template <int J>
int launch_sort(const Params& p, const DeviceInfo& di, cudaStream_t stream) {
  const int smem = (kWarps * 256 + 32 + 2 * kThreads * J) * 4;
  static bool attr_done[64] = {false};
  if (!attr_done[di.device]) {
    const int st = cuda_status(cudaFuncSetAttribute(
        topk_sort_kernel<J>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    if (st != DSA_OK) return st;
    attr_done[di.device] = true;
  }
  int64_t grid = static_cast<int64_t>(di.num_sms) * 4;
  if (grid > p.rows) grid = p.rows;
  topk_sort_kernel<J><<<static_cast<unsigned>(grid), kThreads, smem, stream>>>(p);
  return cuda_status(cudaGetLastError());
}

}  // namespace ixt

// Largest candidate count the sort path takes.
int topk_sort_max_cand() { return ixt::kMaxN; }

int launch_topk_sort(const void* scores, int64_t ld, int64_t* out, int64_t batch, int64_t seqlen,
                     int64_t n_cand, int topk, int64_t start_pos, int ratio, int64_t offset,
                     cudaStream_t stream) {
  using namespace ixt;
  DeviceInfo di;
  int st = current_device_info(&di);
  if (st != DSA_OK) return st;
  if (n_cand > kMaxN) return DSA_ERR_UNSUPPORTED;
  Params p;
  p.scores = static_cast<const uint16_t*>(scores);
  p.ld = ld;
  p.out = out;
  p.K = topk;
  p.S = seqlen;
  p.T = n_cand;
  p.ratio = ratio;
  p.causal = start_pos == 0 ? 1 : 0;
  p.offset = offset;
  p.rows = batch * seqlen;
  if (n_cand <= kThreads * 2) return launch_sort<2>(p, di, stream);
  if (n_cand <= kThreads * 4) return launch_sort<4>(p, di, stream);
  if (n_cand <= kThreads * 8) return launch_sort<8>(p, di, stream);
  return launch_sort<16>(p, di, stream);
}

}  // namespace dsa
