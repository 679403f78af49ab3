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
      const uint32_t base = wh[d];
      rank[j] = base + static_cast<uint32_t>(__popc(peers & lt_mask));
      __syncwarp();
      // every lane of the digit stores the same new count: no divergent branch
      wh[d] = base + static_cast<uint32_t>(__popc(peers));
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

// Resident blocks per SM the launch is compiled for: the sort is bound by the
// latency of its shared-memory chains, so three blocks (40 registers a thread)
// run it faster than two (64); n_cand > 4096 needs more registers.
template <int J>
constexpr int sort_blocks_per_sm() { return J <= 8 ? 3 : 1; }

// J: step bound of this launch (n_cand <= kThreads * J).
template <int J>
__global__ void __launch_bounds__(kThreads, sort_blocks_per_sm<J>())
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
  int st = set_max_dynamic_smem(reinterpret_cast<const void*>(topk_sort_kernel<J>), smem);
  if (st != DSA_OK) return st;
  st = set_func_attribute_once(reinterpret_cast<const void*>(topk_sort_kernel<J>),
                               cudaFuncAttributePreferredSharedMemoryCarveout,
                               cudaSharedmemCarveoutMaxShared);
  if (st != DSA_OK) return st;
  int64_t grid = static_cast<int64_t>(di.num_sms) * sort_blocks_per_sm<J>();
  if (grid > p.rows) grid = p.rows;
  topk_sort_kernel<J><<<static_cast<unsigned>(grid), kThreads, smem, stream>>>(p);
  return cuda_status(cudaGetLastError());
}

// ------------------------------------------------------------------ top-k set
// For a consumer that only needs WHICH candidates are selected (attention in
// the multiplicity form is order-independent): the same selection as the sort
// (score descending, then index ascending), written as a bitmap, one bit per
// candidate, by a radix select instead of a sort. Pass 1 histograms the high
// byte of the 16-bit orderable score and finds the bin holding the k-th key,
// pass 2 does the same with the low byte inside that bin, so T, the k-th key,
// and the number of keys equal to T still to take are known; keys above T are
// in, and keys equal to T are taken in ascending index order (a block scan of
// per-thread tie counts over contiguous index ranges).
constexpr int kMaskThreads = 256;

struct MaskParams {
  const uint16_t* scores;  // [rows, ld] bf16, valid for k < n(t)
  int64_t ld;
  uint32_t* mask;          // [rows, words]
  int words;               // >= ceil(n_cand / 32)
  int K;
  int64_t S;
  int64_t T;
  int ratio;
  int causal;
  int64_t rows;
};

// Inclusive sum of v over the block's 256 threads (thread order); `tmp` holds 8 ints.
__device__ __forceinline__ int block_incl_sum(int v, int* tmp) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int x = __shfl_up_sync(0xFFFFFFFFu, v, o);
    if (lane >= o) v += x;
  }
  if (lane == 31) tmp[warp] = v;
  __syncthreads();
  int pre = 0;
#pragma unroll
  for (int w = 0; w < kMaskThreads / 32; ++w) pre += w < warp ? tmp[w] : 0;
  __syncthreads();
  return v + pre;
}

// J: candidates per thread (contiguous), n_cand <= 256 J.
template <int J>
__global__ void __launch_bounds__(kMaskThreads)
    topk_mask_kernel(const MaskParams p) {
  __shared__ int hist[256];
  __shared__ int tmp[8];
  __shared__ int sel[2];  // the bin holding the k-th key, keys above it
  __shared__ uint32_t bits[256 * J / 32];
  const int tid = threadIdx.x;
  for (int64_t row = blockIdx.x; row < p.rows; row += gridDim.x) {
    const int64_t t = row % p.S;
    int64_t n64 = p.T;
    if (p.causal) {
      n64 = (t + 1) / p.ratio;
      if (n64 > p.T) n64 = p.T;
    }
    const int n = static_cast<int>(n64);
    uint32_t* out = p.mask + row * p.words;
    if (n <= p.K) {  // every valid candidate is selected
      for (int i = tid; i < p.words; i += kMaskThreads) {
        const int lo = i * 32;
        out[i] = n >= lo + 32 ? 0xFFFFFFFFu : (n > lo ? (1u << (n - lo)) - 1u : 0u);
      }
      continue;
    }
    const uint16_t* src = p.scores + row * p.ld;
    const int e0 = tid * J;
    uint32_t key[J];  // orderable 16-bit score, or 0x10000 for "not a candidate"
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const int e = e0 + j;
      key[j] = e < n ? ord16(__ldg(src + e)) : 0x10000u;
    }
    // pass 1: the high byte of the k-th key (bins walked from the top, thread i
    // holds bin 255 - i)
    hist[tid] = 0;
    __syncthreads();
#pragma unroll
    for (int j = 0; j < J; ++j)
      if (key[j] < 0x10000u) atomicAdd(&hist[key[j] >> 8], 1);
    __syncthreads();
    int c = hist[255 - tid];
    int incl = block_incl_sum(c, tmp);
    if (incl >= p.K && incl - c < p.K) {
      sel[0] = 255 - tid;
      sel[1] = incl - c;
    }
    __syncthreads();
    const int hb = sel[0];
    const int need1 = p.K - sel[1];
    // pass 2: the low byte, among keys whose high byte is hb
    hist[tid] = 0;
    __syncthreads();
#pragma unroll
    for (int j = 0; j < J; ++j)
      if (key[j] < 0x10000u && static_cast<int>(key[j] >> 8) == hb) atomicAdd(&hist[key[j] & 0xFFu], 1);
    __syncthreads();
    c = hist[255 - tid];
    incl = block_incl_sum(c, tmp);
    if (incl >= need1 && incl - c < need1) {
      sel[0] = 255 - tid;
      sel[1] = incl - c;
    }
    __syncthreads();
    const uint32_t thr = (static_cast<uint32_t>(hb) << 8) | static_cast<uint32_t>(sel[0]);
    const int need = need1 - sel[1];
    // keys above thr are taken; keys equal to thr (need of them) in index order
    int ties = 0;
#pragma unroll
    for (int j = 0; j < J; ++j) ties += key[j] == thr ? 1 : 0;
    const int tie_base = block_incl_sum(ties, tmp) - ties;
    uint32_t b = 0;
    int ti = tie_base;
#pragma unroll
    for (int j = 0; j < J; ++j) {
      bool take = false;
      if (key[j] < 0x10000u) {
        if (key[j] > thr) {
          take = true;
        } else if (key[j] == thr) {
          take = ti < need;
          ++ti;
        }
      }
      b |= (take ? 1u : 0u) << j;
    }
    if (J == 32) {
      bits[tid] = b;
    } else {  // J == 16: two threads per word
      const uint32_t other = __shfl_xor_sync(0xFFFFFFFFu, b, 1);
      if ((tid & 1) == 0) bits[tid >> 1] = b | (other << 16);
    }
    __syncthreads();
    for (int i = tid; i < p.words; i += kMaskThreads) out[i] = i < 256 * J / 32 ? bits[i] : 0u;
    __syncthreads();
  }
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

namespace dsa {

// Top-k set of each token as a bitmap [rows, words] (bit k of a row: candidate k
// is among the token's top-k by score descending, index ascending).
int launch_topk_mask(const void* scores, int64_t ld, uint32_t* mask, int words, int64_t batch,
                     int64_t seqlen, int64_t n_cand, int topk, int64_t start_pos, int ratio,
                     cudaStream_t stream) {
  using namespace ixt;
  DeviceInfo di;
  int st = current_device_info(&di);
  if (st != DSA_OK) return st;
  if (n_cand > kMaskThreads * 32 || words * 32 < n_cand) return DSA_ERR_UNSUPPORTED;
  MaskParams p;
  p.scores = static_cast<const uint16_t*>(scores);
  p.ld = ld;
  p.mask = mask;
  p.words = words;
  p.K = topk;
  p.S = seqlen;
  p.T = n_cand;
  p.ratio = ratio;
  p.causal = start_pos == 0 ? 1 : 0;
  p.rows = batch * seqlen;
  int64_t grid = static_cast<int64_t>(di.num_sms) * 8;
  if (grid > p.rows) grid = p.rows;
  if (n_cand <= kMaskThreads * 16)
    topk_mask_kernel<16><<<static_cast<unsigned>(grid), kMaskThreads, 0, stream>>>(p);
  else
    topk_mask_kernel<32><<<static_cast<unsigned>(grid), kMaskThreads, 0, stream>>>(p);
  return cuda_status(cudaGetLastError());
}

}  // namespace dsa
