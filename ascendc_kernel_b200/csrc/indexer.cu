// Lightning Indexer C-ABI entry points: argument checks, workspace layout and
// the three launches (q projection + RoPE, weights projection, scores + top-k).
#include "common.cuh"
#include "host_util.h"

namespace dsa {
int launch_qproj_rope(const void* qr, const void* wq, const float* cos_tab, const float* sin_tab,
                      void* q_out, int64_t rows, int K, int n_heads, int rope_dim, int64_t seqlen,
                      const void* a_slices, const int* a_sig, const float* a_err,
                      const float* a_n3, const void* b_slices, const int* b_sig,
                      const float* b_err, const float* b_n3, const int* b_span,
                      uint32_t* open_bits, cudaStream_t stream);
int launch_row_split2(const void* a_src, int64_t a_rows, void* a_slices, int* a_sig,
                      float* a_err, float* a_n3, int* a_span, const void* b_src, int64_t b_rows,
                      void* b_slices, int* b_sig, float* b_err, float* b_n3, int* b_span, int K,
                      cudaStream_t stream);
int launch_wproj_s8(const void* x, const void* wp, void* w_out, int64_t rows, int K, float scale,
                    void* scratch, cudaStream_t stream);
size_t wproj_s8_scratch_bytes(int64_t rows, int K);
int launch_score_topk(const void* q, const void* w, const void* kv, int64_t kv_bstride,
                      int64_t* out, void* scores, int64_t batch, int64_t seqlen, int64_t n_cand,
                      int topk, int64_t start_pos, int ratio, int64_t offset, cudaStream_t stream);
int launch_topk_sort(const void* scores, int64_t ld, int64_t* out, int64_t batch, int64_t seqlen,
                     int64_t n_cand, int topk, int64_t start_pos, int ratio, int64_t offset,
                     cudaStream_t stream);
int topk_sort_max_cand();

namespace {
constexpr int kHeadDim = 64;
constexpr int kScoreHeads = 16;
constexpr int kMaxQprojHeads = 16;
constexpr int64_t kMaxCand = 1024;
constexpr int kMaxTopk = 256;
constexpr int64_t kMaxRowsTma = (int64_t{1} << 31) - 1;

size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

// Front part of the workspace: the int8 slices of wq_b and of qr for the q
// projection (indexer_split.cu), 3 planes each, sized for q_lora_rank <= 256,
// with the per-row exponent, remainder bound and ||S3|| (and the bit span of
// the wq_b rows), and the bitmask of output elements left to the exact fix-up.
struct SliceRegion {
  size_t b_slices, b_sig, b_err, b_n3, b_span, a_slices, a_sig, a_err, a_n3, open, bytes;
};
constexpr size_t kMaxQLora = 256;
SliceRegion slice_region(int n_heads, int head_dim, int64_t rows) {
  const size_t N = static_cast<size_t>(n_heads) * head_dim;
  const size_t R = static_cast<size_t>(rows);
  SliceRegion r;
  r.b_slices = 0;
  r.b_sig = r.b_slices + align256(3 * N * kMaxQLora);
  r.b_err = r.b_sig + align256(N * 4);
  r.b_n3 = r.b_err + align256(N * 4);
  r.b_span = r.b_n3 + align256(N * 4);
  r.a_slices = r.b_span + align256(N * 4);
  r.a_sig = r.a_slices + align256(3 * R * kMaxQLora);
  r.a_err = r.a_sig + align256(R * 4);
  r.a_n3 = r.a_err + align256(R * 4);
  r.open = r.a_n3 + align256(R * 4);
  r.bytes = r.open + align256(R * (N / 8));
  return r;
}

// Front of every indexer workspace: the q projection's slices (above), reused
// afterwards (same stream) by the w projection's slices of x [rows, dim <= 1024].
constexpr int kMaxDim = 1024;
size_t front_bytes(int n_heads, int head_dim, int64_t rows) {
  const size_t a = slice_region(n_heads, head_dim, rows).bytes;
  const size_t b = wproj_s8_scratch_bytes(rows, kMaxDim);
  return a > b ? a : b;
}

// Scratch of the q projection alone (slices, row data, fix-up bitmask).
size_t qproj_scratch_bytes(int n_heads, int head_dim, int64_t rows) {
  return align256(slice_region(n_heads, head_dim, rows).bytes);
}

// Slices wq_b and qr into the workspace, then runs the q projection.
int run_qproj(const void* qr, const void* wq, const float* cos_tab, const float* sin_tab,
              void* q_out, int64_t rows, int K, int n_heads, int head_dim, int rope_dim,
              int64_t seqlen, uint8_t* ws, cudaStream_t s) {
  const SliceRegion r = slice_region(n_heads, head_dim, rows);
  int* b_sig = reinterpret_cast<int*>(ws + r.b_sig);
  float* b_err = reinterpret_cast<float*>(ws + r.b_err);
  float* b_n3 = reinterpret_cast<float*>(ws + r.b_n3);
  int* a_sig = reinterpret_cast<int*>(ws + r.a_sig);
  float* a_err = reinterpret_cast<float*>(ws + r.a_err);
  float* a_n3 = reinterpret_cast<float*>(ws + r.a_n3);
  int* b_span = reinterpret_cast<int*>(ws + r.b_span);
  // wq_b rows (with bit spans, for the exact fix-up) and qr rows in one launch
  const int st = launch_row_split2(wq, static_cast<int64_t>(n_heads) * head_dim, ws + r.b_slices,
                                   b_sig, b_err, b_n3, b_span, qr, rows, ws + r.a_slices, a_sig,
                                   a_err, a_n3, nullptr, K, s);
  if (st != DSA_OK) return st;
  return launch_qproj_rope(qr, wq, cos_tab, sin_tab, q_out, rows, K, n_heads, rope_dim, seqlen,
                           ws + r.a_slices, a_sig, a_err, a_n3, ws + r.b_slices, b_sig, b_err,
                           b_n3, b_span, reinterpret_cast<uint32_t*>(ws + r.open), s);
}

// The q projection (qr, wq_b -> q with RoPE) and the w projection (x, w_proj ->
// w), which are independent until the scores. `front` holds either one's
// scratch (front_bytes). With `extra` (qproj_scratch_bytes more, disjoint from
// everything else) the w chain runs on the calling thread's side stream over
// `front` while the q chain runs on `s` over `extra`, and `s` waits for both;
// otherwise they run one after the other on `s` over `front`. Same results.
int run_projections(const void* x, const void* qr, const void* wq_b, const void* w_proj,
                    const float* cos_tab, const float* sin_tab, void* q, void* w, int64_t rows,
                    int dim, int q_lora_rank, int n_heads, int head_dim, int rope_dim,
                    int64_t seqlen, float w_scale, uint8_t* front, uint8_t* extra,
                    cudaStream_t s) {
  SideStream side;
  bool overlap = extra != nullptr;
  if (overlap) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    const int st = cuda_status(cudaStreamIsCapturing(s, &cs));
    if (st != DSA_OK) return st;
    overlap = thread_side_stream(&side, cs == cudaStreamCaptureStatusNone) == DSA_OK;
  }
  if (!overlap) {
    const int st = run_qproj(qr, wq_b, cos_tab, sin_tab, q, rows, q_lora_rank, n_heads, head_dim,
                             rope_dim, seqlen, front, s);
    if (st != DSA_OK) return st;
    return launch_wproj_s8(x, w_proj, w, rows, dim, w_scale, front, s);
  }
  int st = cuda_status(cudaEventRecord(side.fork, s));
  if (st == DSA_OK) st = cuda_status(cudaStreamWaitEvent(side.stream, side.fork, 0));
  if (st != DSA_OK) return st;
  const int st_w = launch_wproj_s8(x, w_proj, w, rows, dim, w_scale, front, side.stream);
  // the join is recorded and awaited even after a failed launch, so the side
  // stream never leaves work (or a capture) behind
  int st_j = cuda_status(cudaEventRecord(side.join, side.stream));
  const int st_q = st_w != DSA_OK ? DSA_OK
                                   : run_qproj(qr, wq_b, cos_tab, sin_tab, q, rows, q_lora_rank,
                                               n_heads, head_dim, rope_dim, seqlen, extra, s);
  if (st_j == DSA_OK) st_j = cuda_status(cudaStreamWaitEvent(s, side.join, 0));
  if (st_w != DSA_OK) return st_w;
  if (st_q != DSA_OK) return st_q;
  return st_j;
}

int check_qproj(const void* qr, const void* wq, const float* cos_tab, const float* sin_tab,
                const void* q_out, int64_t rows, int K, int n_heads, int head_dim, int rope_dim,
                int64_t seqlen) {
  if (!qr || !wq || !q_out || rows < 0 || K <= 0 || n_heads <= 0 || seqlen <= 0)
    return DSA_ERR_INVALID_ARGUMENT;
  if (rope_dim < 0 || rope_dim > head_dim || (rope_dim & 1)) return DSA_ERR_INVALID_ARGUMENT;
  if (rope_dim > 0 && (!cos_tab || !sin_tab)) return DSA_ERR_INVALID_ARGUMENT;
  if (head_dim != kHeadDim || K % 64 != 0 || K > 256 || n_heads > kMaxQprojHeads)
    return DSA_ERR_UNSUPPORTED;
  if (rows > kMaxRowsTma) return DSA_ERR_UNSUPPORTED;
  if (!aligned16(qr) || !aligned16(wq) || !aligned16(q_out)) return DSA_ERR_MISALIGNED;
  return DSA_OK;
}

int check_wproj(const void* x, const void* wp, const void* w_out, int64_t rows, int dim,
                int n_heads) {
  if (!x || !wp || !w_out || rows < 0 || dim <= 0 || n_heads <= 0) return DSA_ERR_INVALID_ARGUMENT;
  if (n_heads != kScoreHeads || dim % 64 != 0 || dim > 1024) return DSA_ERR_UNSUPPORTED;
  if (rows > kMaxRowsTma) return DSA_ERR_UNSUPPORTED;
  if (!aligned16(x) || !aligned16(wp) || !aligned16(w_out)) return DSA_ERR_MISALIGNED;
  return DSA_OK;
}

// Short candidate lists are scored and selected in one kernel (keys in shared
// memory); longer ones go through a score buffer and a sort kernel.
bool score_fused(int64_t n_cand, int topk) { return n_cand <= kMaxCand && topk <= kMaxTopk; }

size_t score_buffer_bytes(int64_t batch, int64_t seqlen, int64_t n_cand, int topk) {
  if (batch <= 0 || seqlen <= 0 || n_cand <= 0 || score_fused(n_cand, topk)) return 0;
  return align256(static_cast<size_t>(batch) * static_cast<size_t>(seqlen) *
                  static_cast<size_t>(n_cand) * 2);
}

int check_score(const void* q, const void* w, const void* kv, int64_t kv_bstride,
                const int64_t* out, int64_t batch, int64_t seqlen, int n_heads, int head_dim,
                int64_t n_cand, int topk, int64_t start_pos, int ratio) {
  if (!q || !w || !kv || !out || batch < 0 || seqlen < 0 || n_cand < 0 || topk < 0 ||
      start_pos < 0 || ratio <= 0)
    return DSA_ERR_INVALID_ARGUMENT;
  if (n_heads != kScoreHeads || head_dim != kHeadDim) return DSA_ERR_UNSUPPORTED;
  if (topk > n_cand) return DSA_ERR_INVALID_ARGUMENT;
  if (!score_fused(n_cand, topk) && n_cand > topk_sort_max_cand()) return DSA_ERR_UNSUPPORTED;
  if (kv_bstride < n_cand * kHeadDim || kv_bstride % kHeadDim != 0) return DSA_ERR_INVALID_ARGUMENT;
  if (batch * seqlen * kScoreHeads > kMaxRowsTma) return DSA_ERR_UNSUPPORTED;
  if ((batch - 1) * (kv_bstride / kHeadDim) + n_cand > kMaxRowsTma) return DSA_ERR_UNSUPPORTED;
  if (!aligned16(q) || !aligned16(w) || !aligned16(kv) || !aligned16(out))
    return DSA_ERR_MISALIGNED;
  return DSA_OK;
}
}  // namespace
}  // namespace dsa

extern "C" int dsa_indexer_qproj_rope(const void* qr, const void* wq_b, const float* cos_tab,
                                      const float* sin_tab, void* q_out, int64_t rows,
                                      int q_lora_rank, int n_heads, int head_dim, int rope_dim,
                                      int64_t seqlen, void* workspace, size_t workspace_bytes,
                                      void* stream) {
  int st = dsa::check_qproj(qr, wq_b, cos_tab, sin_tab, q_out, rows, q_lora_rank, n_heads,
                            head_dim, rope_dim, seqlen);
  if (st != DSA_OK || rows == 0) return st;
  if (workspace == nullptr || (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0 ||
      workspace_bytes < dsa::slice_region(n_heads, head_dim, rows).bytes)
    return DSA_ERR_WORKSPACE;
  return dsa::run_qproj(qr, wq_b, cos_tab, sin_tab, q_out, rows, q_lora_rank, n_heads, head_dim,
                        rope_dim, seqlen, static_cast<uint8_t*>(workspace),
                        static_cast<cudaStream_t>(stream));
}

extern "C" size_t dsa_indexer_wproj_workspace_bytes(int64_t rows, int dim) {
  if (rows <= 0 || dim <= 0) return 0;
  return dsa::wproj_s8_scratch_bytes(rows, dim);
}

extern "C" int dsa_indexer_wproj(const void* x, const void* w_proj, void* w_out, int64_t rows,
                                 int dim, int n_heads, float scale, void* workspace,
                                 size_t workspace_bytes, void* stream) {
  int st = dsa::check_wproj(x, w_proj, w_out, rows, dim, n_heads);
  if (st != DSA_OK || rows == 0) return st;
  if (workspace == nullptr || (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0 ||
      workspace_bytes < dsa::wproj_s8_scratch_bytes(rows, dim))
    return DSA_ERR_WORKSPACE;
  return dsa::launch_wproj_s8(x, w_proj, w_out, rows, dim, scale, workspace,
                              static_cast<cudaStream_t>(stream));
}

namespace dsa {
namespace {
// Scores, then (long lists) the sort; `scores` is the score buffer or null.
int run_score(const void* q, const void* w, const void* kv, int64_t kv_bstride, int64_t* out,
              void* scores, int64_t batch, int64_t seqlen, int64_t n_cand, int topk,
              int64_t start_pos, int ratio, int64_t offset, cudaStream_t s) {
  if (score_fused(n_cand, topk))
    return launch_score_topk(q, w, kv, kv_bstride, out, nullptr, batch, seqlen, n_cand, topk,
                             start_pos, ratio, offset, s);
  int st = launch_score_topk(q, w, kv, kv_bstride, out, scores, batch, seqlen, n_cand, topk,
                             start_pos, ratio, offset, s);
  if (st != DSA_OK) return st;
  return launch_topk_sort(scores, n_cand, out, batch, seqlen, n_cand, topk, start_pos, ratio,
                          offset, s);
}
}  // namespace
}  // namespace dsa

extern "C" size_t dsa_indexer_score_workspace_bytes(int64_t batch, int64_t seqlen, int64_t n_cand,
                                                    int topk) {
  return dsa::score_buffer_bytes(batch, seqlen, n_cand, topk);
}

extern "C" int dsa_indexer_score_topk(const void* q, const void* w, const void* kv_cache,
                                      int64_t kv_batch_stride, int64_t* out, int64_t batch,
                                      int64_t seqlen, int n_heads, int head_dim, int64_t n_cand,
                                      int topk, int64_t start_pos, int ratio, int64_t offset,
                                      void* workspace, size_t workspace_bytes, void* stream) {
  int st = dsa::check_score(q, w, kv_cache, kv_batch_stride, out, batch, seqlen, n_heads,
                            head_dim, n_cand, topk, start_pos, ratio);
  if (st != DSA_OK || batch == 0 || seqlen == 0 || topk == 0) return st;
  const size_t need = dsa::score_buffer_bytes(batch, seqlen, n_cand, topk);
  if (need > 0 && (workspace == nullptr || workspace_bytes < need ||
                   (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0))
    return DSA_ERR_WORKSPACE;
  return dsa::run_score(q, w, kv_cache, kv_batch_stride, out, workspace, batch, seqlen, n_cand,
                        topk, start_pos, ratio, offset, static_cast<cudaStream_t>(stream));
}

extern "C" size_t dsa_indexer_workspace_bytes(int64_t batch, int64_t seqlen, int n_heads,
                                              int head_dim, int64_t n_cand, int topk) {
  if (batch <= 0 || seqlen <= 0 || n_heads <= 0 || head_dim <= 0) return 0;
  const size_t rows = static_cast<size_t>(batch) * static_cast<size_t>(seqlen);
  return dsa::front_bytes(n_heads, head_dim, static_cast<int64_t>(rows)) +
         dsa::align256(rows * n_heads * head_dim * 2) + dsa::align256(rows * n_heads * 2) +
         dsa::score_buffer_bytes(batch, seqlen, n_cand, topk);
}

extern "C" int dsa_indexer_fwd(const void* x, const void* qr, const void* wq_b,
                               const void* w_proj, const float* cos_tab, const float* sin_tab,
                               const void* kv_cache, int64_t kv_batch_stride, int64_t* out,
                               void* workspace, size_t workspace_bytes, int64_t batch,
                               int64_t seqlen, int dim, int q_lora_rank, int n_heads,
                               int head_dim, int rope_dim, int index_topk, int64_t start_pos,
                               int ratio, int64_t offset, float w_scale, void* stream) {
  if (batch < 0 || seqlen < 0 || index_topk <= 0 || ratio <= 0 || start_pos < 0)
    return DSA_ERR_INVALID_ARGUMENT;
  if (batch == 0 || seqlen == 0) return DSA_OK;
  const int64_t rows = batch * seqlen;
  const int64_t n_cand = (start_pos + seqlen) / ratio;
  const int topk = static_cast<int>(index_topk < n_cand ? index_topk : n_cand);
  if (topk <= 0) return DSA_ERR_INVALID_ARGUMENT;
  const size_t need =
      dsa_indexer_workspace_bytes(batch, seqlen, n_heads, head_dim, n_cand, topk);
  if (workspace == nullptr || workspace_bytes < need ||
      (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
    return DSA_ERR_WORKSPACE;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  const size_t wreg = dsa::front_bytes(n_heads, head_dim, rows);
  void* q = ws + wreg;
  void* w = ws + wreg + dsa::align256(static_cast<size_t>(rows) * n_heads * head_dim * 2);
  void* scores = static_cast<uint8_t*>(w) + dsa::align256(static_cast<size_t>(rows) * n_heads * 2);
  int st = dsa::check_qproj(qr, wq_b, cos_tab, sin_tab, q, rows, q_lora_rank, n_heads, head_dim,
                            rope_dim, seqlen);
  if (st != DSA_OK) return st;
  st = dsa::check_wproj(x, w_proj, w, rows, dim, n_heads);
  if (st != DSA_OK) return st;
  st = dsa::check_score(q, w, kv_cache, kv_batch_stride, out, batch, seqlen, n_heads, head_dim,
                        n_cand, topk, start_pos, ratio);
  if (st != DSA_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // room after the layout for a second projection scratch: the projections overlap
  const size_t extra = dsa::qproj_scratch_bytes(n_heads, head_dim, rows);
  st = dsa::run_projections(x, qr, wq_b, w_proj, cos_tab, sin_tab, q, w, rows, dim, q_lora_rank,
                            n_heads, head_dim, rope_dim, seqlen, w_scale, ws,
                            workspace_bytes >= need + extra ? ws + need : nullptr, s);
  if (st != DSA_OK) return st;
  return dsa::run_score(q, w, kv_cache, kv_batch_stride, out, scores, batch, seqlen, n_cand, topk,
                        start_pos, ratio, offset, s);
}

extern "C" size_t dsa_indexer_overlap_extra_bytes(int64_t rows, int n_heads, int head_dim) {
  if (rows <= 0 || n_heads <= 0 || head_dim <= 0) return 0;
  return dsa::qproj_scratch_bytes(n_heads, head_dim, rows);
}
// ---------------------------------------------------------------- chained path
namespace dsa {
int launch_topk_mask(const void* scores, int64_t ld, uint32_t* mask, int words, int64_t batch,
                     int64_t seqlen, int64_t n_cand, int topk, int64_t start_pos, int ratio,
                     cudaStream_t stream);
bool sa_long_supported(int heads, int head_dim, int nkv);
int launch_sa_long_mask(const void* q, const void* kv, const uint32_t* mask, int mask_words,
                        int64_t mask_offset, const float* sink, void* out, int64_t batch,
                        int64_t m, int heads, int nkv, float scale, cudaStream_t stream);
namespace {
constexpr int64_t kMaxChainCand = 8192;
int mask_words(int64_t n_cand) { return static_cast<int>(((n_cand + 127) / 128) * 4); }
struct ChainLayout {
  size_t slices, q, w, scores, mask, bytes;
};
ChainLayout chain_layout(int64_t batch, int64_t seqlen, int n_heads, int head_dim, int64_t n_cand) {
  const size_t rows = static_cast<size_t>(batch) * static_cast<size_t>(seqlen);
  ChainLayout l;
  l.slices = 0;
  l.q = l.slices + front_bytes(n_heads, head_dim, static_cast<int64_t>(rows));
  l.w = l.q + align256(rows * n_heads * head_dim * 2);
  l.scores = l.w + align256(rows * n_heads * 2);
  l.mask = l.scores + align256(rows * static_cast<size_t>(n_cand) * 2);
  l.bytes = l.mask + align256(rows * static_cast<size_t>(mask_words(n_cand)) * 4);
  return l;
}
}  // namespace
}  // namespace dsa

extern "C" size_t dsa_chain_workspace_bytes(int64_t batch, int64_t seqlen, int n_heads,
                                            int head_dim, int64_t n_cand) {
  if (batch <= 0 || seqlen <= 0 || n_heads <= 0 || head_dim <= 0 || n_cand <= 0) return 0;
  return dsa::chain_layout(batch, seqlen, n_heads, head_dim, n_cand).bytes;
}

extern "C" int dsa_chain_fwd(const void* x, const void* qr, const void* wq_b, const void* w_proj,
                             const float* cos_tab, const float* sin_tab, const void* kv_cache,
                             int64_t kv_batch_stride, int64_t batch, int64_t seqlen, int dim,
                             int q_lora_rank, int ix_heads, int ix_head_dim, int rope_dim,
                             int index_topk, int64_t start_pos, int ratio, int64_t offset,
                             float w_scale, const void* q, const void* kv, int n_kv,
                             int attn_heads, int attn_head_dim, const float* sink,
                             float softmax_scale, void* out, void* workspace,
                             size_t workspace_bytes, void* stream) {
  if (batch < 0 || seqlen < 0 || index_topk <= 0 || ratio <= 0 || start_pos < 0 || n_kv <= 0 ||
      !q || !kv || !sink || !out)
    return DSA_ERR_INVALID_ARGUMENT;
  if (batch == 0 || seqlen == 0) return DSA_OK;
  const int64_t rows = batch * seqlen;
  const int64_t n_cand = (start_pos + seqlen) / ratio;
  const int topk = static_cast<int>(index_topk < n_cand ? index_topk : n_cand);
  if (topk <= 0) return DSA_ERR_INVALID_ARGUMENT;
  if (n_cand > dsa::kMaxChainCand || !dsa::sa_long_supported(attn_heads, attn_head_dim, n_kv))
    return DSA_ERR_UNSUPPORTED;
  if (!dsa::aligned16(q) || !dsa::aligned16(kv) || !dsa::aligned16(out)) return DSA_ERR_MISALIGNED;
  const dsa::ChainLayout l = dsa::chain_layout(batch, seqlen, ix_heads, ix_head_dim, n_cand);
  if (workspace == nullptr || workspace_bytes < l.bytes ||
      (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
    return DSA_ERR_WORKSPACE;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  void* qi = ws + l.q;
  void* wi = ws + l.w;
  void* scores = ws + l.scores;
  uint32_t* mask = reinterpret_cast<uint32_t*>(ws + l.mask);
  int st = dsa::check_qproj(qr, wq_b, cos_tab, sin_tab, qi, rows, q_lora_rank, ix_heads,
                            ix_head_dim, rope_dim, seqlen);
  if (st != DSA_OK) return st;
  st = dsa::check_wproj(x, w_proj, wi, rows, dim, ix_heads);
  if (st != DSA_OK) return st;
  // the score checks (the buffer path writes no index list: the bitmap stands in)
  st = dsa::check_score(qi, wi, kv_cache, kv_batch_stride, reinterpret_cast<const int64_t*>(mask),
                        batch, seqlen, ix_heads, ix_head_dim, n_cand, topk, start_pos, ratio);
  if (st != DSA_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t extra = dsa::qproj_scratch_bytes(ix_heads, ix_head_dim, rows);
  st = dsa::run_projections(x, qr, wq_b, w_proj, cos_tab, sin_tab, qi, wi, rows, dim,
                            q_lora_rank, ix_heads, ix_head_dim, rope_dim, seqlen, w_scale,
                            ws + l.slices,
                            workspace_bytes >= l.bytes + extra ? ws + l.bytes : nullptr, s);
  if (st != DSA_OK) return st;
  st = dsa::launch_score_topk(qi, wi, kv_cache, kv_batch_stride, nullptr, scores, batch, seqlen,
                              n_cand, topk, start_pos, ratio, offset, s);
  if (st != DSA_OK) return st;
  const int words = dsa::mask_words(n_cand);
  st = dsa::launch_topk_mask(scores, n_cand, mask, words, batch, seqlen, n_cand, topk, start_pos,
                             ratio, s);
  if (st != DSA_OK) return st;
  return dsa::launch_sa_long_mask(q, kv, mask, words, offset, sink, out, batch, seqlen,
                                  attn_heads, n_kv, softmax_scale, s);
}

// ---------------------------------------------------------------- fp8 path
namespace dsa {
int launch_fp8_quant_rows(const void* src, int64_t rows, int64_t rows_per_group,
                          int64_t group_stride, void* dst, float* scale, const void* w,
                          float* w_out, cudaStream_t stream);
int launch_score_fp8(const void* q8, const float* wq, const void* k8, const float* ks,
                     int64_t* out, float* scores, int64_t batch, int64_t seqlen, int64_t n_cand,
                     int topk, int64_t start_pos, int ratio, int64_t offset, cudaStream_t stream);
namespace {
struct Fp8Layout {
  size_t q, w, q8, wq, k8, ks, bytes;
};
Fp8Layout fp8_layout(int64_t batch, int64_t seqlen, int n_heads, int head_dim, int64_t n_cand) {
  const size_t rows = static_cast<size_t>(batch) * static_cast<size_t>(seqlen);
  const size_t qe = rows * n_heads * head_dim;
  const size_t kr = static_cast<size_t>(batch) * static_cast<size_t>(n_cand);
  Fp8Layout l;
  l.q = front_bytes(n_heads, head_dim, static_cast<int64_t>(rows));
  l.w = l.q + align256(qe * 2);
  l.q8 = l.w + align256(rows * n_heads * 2);
  l.wq = l.q8 + align256(qe);
  l.k8 = l.wq + align256(rows * n_heads * 4);
  l.ks = l.k8 + align256(kr * head_dim);
  l.bytes = l.ks + align256(kr * 4);
  return l;
}

int check_score_fp8(const void* q8, const float* wq, const void* k8, const float* ks,
                    const int64_t* out, int64_t batch, int64_t seqlen, int n_heads, int head_dim,
                    int64_t n_cand, int topk, int64_t start_pos, int ratio) {
  if (!q8 || !wq || !k8 || !ks || !out || batch < 0 || seqlen < 0 || n_cand < 0 || topk < 0 ||
      start_pos < 0 || ratio <= 0)
    return DSA_ERR_INVALID_ARGUMENT;
  if (n_heads != kScoreHeads || head_dim != kHeadDim) return DSA_ERR_UNSUPPORTED;
  if (topk > n_cand) return DSA_ERR_INVALID_ARGUMENT;
  if (!score_fused(n_cand, topk)) return DSA_ERR_UNSUPPORTED;
  if (batch * seqlen * kScoreHeads > kMaxRowsTma || batch * n_cand > kMaxRowsTma)
    return DSA_ERR_UNSUPPORTED;
  if (!aligned16(q8) || !aligned16(wq) || !aligned16(k8) || !aligned16(ks) || !aligned16(out))
    return DSA_ERR_MISALIGNED;
  return DSA_OK;
}
}  // namespace
}  // namespace dsa

extern "C" int dsa_indexer_fp8_quant_rows(const void* x, int64_t rows, int64_t rows_per_group,
                                          int64_t group_stride, int head_dim, void* y,
                                          float* scale, const void* w, float* w_out,
                                          void* stream) {
  if (!x || !y || rows < 0 || rows_per_group <= 0 || group_stride < 0 ||
      ((w == nullptr) != (w_out == nullptr)))
    return DSA_ERR_INVALID_ARGUMENT;
  if (head_dim != dsa::kHeadDim) return DSA_ERR_UNSUPPORTED;
  if (rows_per_group < rows && group_stride < rows_per_group * dsa::kHeadDim)
    return DSA_ERR_INVALID_ARGUMENT;
  if (!dsa::aligned16(x) || !dsa::aligned16(y) || (group_stride % 8) != 0)
    return DSA_ERR_MISALIGNED;
  if (rows == 0) return DSA_OK;
  return dsa::launch_fp8_quant_rows(x, rows, rows_per_group, group_stride, y, scale, w, w_out,
                                    static_cast<cudaStream_t>(stream));
}

extern "C" int dsa_indexer_score_topk_fp8(const void* q8, const float* wq, const void* k8,
                                          const float* ks, int64_t* out, float* scores,
                                          int64_t batch, int64_t seqlen, int n_heads,
                                          int head_dim, int64_t n_cand, int topk,
                                          int64_t start_pos, int ratio, int64_t offset,
                                          void* stream) {
  const int st = dsa::check_score_fp8(q8, wq, k8, ks, out, batch, seqlen, n_heads, head_dim,
                                      n_cand, topk, start_pos, ratio);
  if (st != DSA_OK || batch == 0 || seqlen == 0 || topk == 0) return st;
  return dsa::launch_score_fp8(q8, wq, k8, ks, out, scores, batch, seqlen, n_cand, topk,
                               start_pos, ratio, offset, static_cast<cudaStream_t>(stream));
}

extern "C" size_t dsa_indexer_fp8_workspace_bytes(int64_t batch, int64_t seqlen, int n_heads,
                                                  int head_dim, int64_t n_cand) {
  if (batch <= 0 || seqlen <= 0 || n_heads <= 0 || head_dim <= 0 || n_cand <= 0) return 0;
  return dsa::fp8_layout(batch, seqlen, n_heads, head_dim, n_cand).bytes;
}

extern "C" int dsa_indexer_fwd_fp8(const void* x, const void* qr, const void* wq_b,
                                   const void* w_proj, const float* cos_tab,
                                   const float* sin_tab, const void* kv_cache,
                                   int64_t kv_batch_stride, int64_t* out, void* workspace,
                                   size_t workspace_bytes, int64_t batch, int64_t seqlen, int dim,
                                   int q_lora_rank, int n_heads, int head_dim, int rope_dim,
                                   int index_topk, int64_t start_pos, int ratio, int64_t offset,
                                   float w_scale, void* stream) {
  if (batch < 0 || seqlen < 0 || index_topk <= 0 || ratio <= 0 || start_pos < 0 || !kv_cache)
    return DSA_ERR_INVALID_ARGUMENT;
  if (batch == 0 || seqlen == 0) return DSA_OK;
  const int64_t rows = batch * seqlen;
  const int64_t n_cand = (start_pos + seqlen) / ratio;
  const int topk = static_cast<int>(index_topk < n_cand ? index_topk : n_cand);
  if (topk <= 0) return DSA_ERR_INVALID_ARGUMENT;
  if (kv_batch_stride < n_cand * head_dim) return DSA_ERR_INVALID_ARGUMENT;
  if (!dsa::aligned16(kv_cache) || kv_batch_stride % 8 != 0) return DSA_ERR_MISALIGNED;
  const dsa::Fp8Layout l = dsa::fp8_layout(batch, seqlen, n_heads, head_dim, n_cand);
  if (workspace == nullptr || workspace_bytes < l.bytes ||
      (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
    return DSA_ERR_WORKSPACE;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  void* q = ws + l.q;
  void* w = ws + l.w;
  void* q8 = ws + l.q8;
  float* wq = reinterpret_cast<float*>(ws + l.wq);
  void* k8 = ws + l.k8;
  float* ks = reinterpret_cast<float*>(ws + l.ks);
  int st = dsa::check_qproj(qr, wq_b, cos_tab, sin_tab, q, rows, q_lora_rank, n_heads, head_dim,
                            rope_dim, seqlen);
  if (st != DSA_OK) return st;
  st = dsa::check_wproj(x, w_proj, w, rows, dim, n_heads);
  if (st != DSA_OK) return st;
  st = dsa::check_score_fp8(q8, wq, k8, ks, out, batch, seqlen, n_heads, head_dim, n_cand, topk,
                            start_pos, ratio);
  if (st != DSA_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t extra = dsa::qproj_scratch_bytes(n_heads, head_dim, rows);
  st = dsa::run_projections(x, qr, wq_b, w_proj, cos_tab, sin_tab, q, w, rows, dim, q_lora_rank,
                            n_heads, head_dim, rope_dim, seqlen, w_scale, ws,
                            workspace_bytes >= l.bytes + extra ? ws + l.bytes : nullptr, s);
  if (st != DSA_OK) return st;
  st = dsa::launch_fp8_quant_rows(q, rows * n_heads, rows * n_heads, 0, q8, nullptr, w, wq, s);
  if (st != DSA_OK) return st;
  st = dsa::launch_fp8_quant_rows(kv_cache, batch * n_cand, n_cand, kv_batch_stride, k8, ks,
                                  nullptr, nullptr, s);
  if (st != DSA_OK) return st;
  return dsa::launch_score_fp8(q8, wq, k8, ks, out, nullptr, batch, seqlen, n_cand, topk,
                               start_pos, ratio, offset, s);
}

// ------------------------------------------------------------ kv_cache writer
namespace dsa {
int launch_kv_writer(const void* x, const void* wk, const float* g, const float* b,
                     const float* cos_t, const float* sin_t, void* kv, int64_t kv_bstride,
                     int64_t batch, int64_t seqlen, int dim, int rope_dim, int64_t start_pos,
                     int ratio, cudaStream_t stream);
}  // namespace dsa

extern "C" int dsa_kv_cache_write(const void* x, const void* wk, const float* ln_weight,
                                  const float* ln_bias, const float* cos_tab,
                                  const float* sin_tab, void* kv_cache, int64_t kv_batch_stride,
                                  int64_t kv_rows, int64_t batch, int64_t seqlen, int dim,
                                  int head_dim, int rope_dim, int64_t start_pos, int ratio,
                                  void* stream) {
  if (!x || !wk || !ln_weight || !ln_bias || !kv_cache || batch < 0 || seqlen < 0 || dim <= 0 ||
      start_pos < 0 || ratio <= 0 || rope_dim < 0 || (rope_dim & 1) || kv_rows < 0)
    return DSA_ERR_INVALID_ARGUMENT;
  if (rope_dim > 0 && (!cos_tab || !sin_tab)) return DSA_ERR_INVALID_ARGUMENT;
  if (head_dim != dsa::kHeadDim || rope_dim > head_dim || dim % 64 != 0 || 128 % ratio != 0)
    return DSA_ERR_UNSUPPORTED;
  if (start_pos % ratio != 0) return DSA_ERR_INVALID_ARGUMENT;
  if (batch == 0 || seqlen < ratio) return DSA_OK;  // no complete block
  if ((start_pos + seqlen) / ratio > kv_rows || kv_batch_stride < kv_rows * head_dim)
    return DSA_ERR_INVALID_ARGUMENT;
  if (batch * seqlen > dsa::kMaxRowsTma) return DSA_ERR_UNSUPPORTED;
  if (!dsa::aligned16(x) || !dsa::aligned16(wk) || !dsa::aligned16(kv_cache) ||
      kv_batch_stride % 8 != 0)
    return DSA_ERR_MISALIGNED;
  return dsa::launch_kv_writer(x, wk, ln_weight, ln_bias, cos_tab, sin_tab, kv_cache,
                               kv_batch_stride, batch, seqlen, dim, rope_dim, start_pos, ratio,
                               static_cast<cudaStream_t>(stream));
}
