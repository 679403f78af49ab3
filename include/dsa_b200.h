/*
 * dsa_b200.h -- C ABI of the B200 (sm_100a) DeepSeek sparse-attention operator
 * path: SparseAttention, Lightning Indexer and Sinkhorn (mHC).
 *
 * Conventions shared by every entry point:
 *  - All tensor arguments are raw DEVICE pointers to contiguous row-major data
 *    (bf16 passed as `const void*`, 2 bytes per element). Sizes are element
 *    counts. Nothing here allocates device memory; scratch is passed in.
 *  - `stream` is a cudaStream_t (NULL = legacy default stream). Every call is
 *    asynchronous with respect to the host, like a kernel launch.
 *  - The return value is a dsa_status_t. Argument problems are caught on the
 *    host before any launch. A bounded device-side wait that times out does not
 *    fail the call; it sets a code in the per-device error word, which
 *    dsa_device_error_read() returns (after synchronizing the device).
 *  - No entry point throws, calls exit(), or falls back to a CPU path.
 *
 * The reference binds each operator through pybind functions that take
 * at::Tensor and call an `extern "C" launch_*(blockDim, stream, uint8_t* ...)`
 * kernel launcher; the functions below take the place of those pairs.
 */
#ifndef DSA_B200_H_
#define DSA_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum dsa_status {
  DSA_OK = 0,
  DSA_ERR_INVALID_ARGUMENT = 1, /* null pointer, negative or inconsistent size */
  DSA_ERR_UNSUPPORTED = 2,      /* shape outside what the kernels are built for */
  DSA_ERR_MISALIGNED = 3,       /* a pointer or stride breaks the 16-byte TMA rule */
  DSA_ERR_CUDA = 4,             /* a CUDA runtime/driver call failed; see dsa_last_cuda_error */
  DSA_ERR_WORKSPACE = 5,        /* workspace pointer missing or too small */
  DSA_ERR_NO_DEVICE = 6         /* no usable sm_100 device */
} dsa_status_t;

/* Bits of the per-device error word written by kernels (bounded waits that
 * ran out of time, or out-of-contract data detected on the device). */
#define DSA_DEVERR_SA_WAIT 0x0001u     /* sparse attention pipeline wait timed out */
#define DSA_DEVERR_IX_WAIT 0x0002u     /* indexer pipeline wait timed out */
#define DSA_DEVERR_GEMM_WAIT 0x0004u   /* projection GEMM pipeline wait timed out */
#define DSA_DEVERR_TOPK_RANGE 0x0010u  /* top-k selection found fewer keys than expected */

/* Human-readable name of a dsa_status_t value (static storage). */
const char* dsa_status_string(int status);

/* The cudaError_t of the most recent failing CUDA call made by this library
 * on the calling thread (0 when none). */
int dsa_last_cuda_error(void);

/* Synchronizes `device`, then stores the device error word in *code_out and,
 * when `clear` is non-zero, resets it to 0. The word belongs to a CUDA context:
 * the calling thread's current one when it is on `device` (the primary context,
 * or one the caller created), else the primary context of `device`.
 * Returns DSA_OK or DSA_ERR_CUDA. */
int dsa_device_error_read(int device, unsigned int* code_out, int clear);

/* Library version as MAJOR*10000 + MINOR*100 + PATCH. */
int dsa_version(void);

/* ------------------------------------------------------------------------
 * Sinkhorn (mHC) normalisation, fp32, in registers, one launch.
 *   y = softmax(x, -1) + eps;  y /= (sum(y, -2) + eps);
 *   repeat (repeat-1) times: y /= (sum(y, -1) + eps); y /= (sum(y, -2) + eps)
 * x, y: [n_mat, n, n] fp32 (y may equal x). Supported: n == 4, repeat >= 1.
 * Replaces launch_sinkhorn (src/sinkhorn_kernel.asc:175-179) and its pybind
 * wrapper run_sinkhorn (src/task3_sinkhorn.py:227-237); semantics follow
 * Model.forward in reference/task3_v0_ref.py:8-14.
 */
int dsa_sinkhorn_fwd(const float* x, float* y, int64_t n_mat, int n, int repeat, float eps,
                     void* stream);

/* ------------------------------------------------------------------------
 * SparseAttention forward (multiplicity softmax, fused mm1 -> softmax -> mm2).
 *   q      [batch, m, n_heads, head_dim] bf16
 *   kv     [batch, n_kv, head_dim] bf16 (shared as K and V)
 *   idx    [batch, m, topk] int32 (idx_elem_bytes 4) or int64 (8); entries < 0
 *          or >= n_kv are masked out
 *   sink   [n_heads] fp32 attention-sink logits
 *   out    [batch, m, n_heads, head_dim] bf16
 * out[b,t,h,:] = sum_j w_j kv[b, idx_j], w = softmax over the valid j of
 * (q.kv*scale) with the sink logit in the max and the denominator.
 * Supported: head_dim == 128; n_heads in {16,32,64,128}, 1 <= n_kv <= 32,
 * topk*idx_elem_bytes a multiple of 16 and topk <= 128 (one fused pass over the
 * whole pool); or, for larger pools or lists (the chained long-context case),
 * n_heads in {64,128}, n_kv <= 4096 and any topk (128-row pool chunks);
 * q, kv, idx, out 16-byte aligned.
 * Replaces launch_sa_fused (src/sparse_attn_kernel_mm.asc:310-313) and its
 * pybind wrapper run_fused (src/task1_sparse_attn.py:420-429); semantics follow
 * sparse_attn_ref in reference/task1_v0_ref.py:5-24.
 */
int dsa_sparse_attn_fwd(const void* q, const void* kv, const void* idx, int idx_elem_bytes,
                        const float* sink, void* out, int64_t batch, int64_t m, int n_heads,
                        int head_dim, int n_kv, int topk, float softmax_scale, void* stream);

/* ------------------------------------------------------------------------
 * Lightning Indexer. Rounding contract (the same in every step): each bf16
 * result is the correctly rounded (round-to-nearest-even) value of the exact
 * fp32/fp64 quantity it names, the same values the reference's torch ops
 * produce up to the GEMM accumulation order.
 *
 * (a) q = RoPE(bf16(qr . wq_b^T)), rotation on the last rope_dim dims of every
 *     head (interleaved pairs, fp32 non-fused a*c - b*s / a*s + b*c, one RNE).
 *     qr [rows, q_lora_rank] bf16, wq_b [n_heads*head_dim, q_lora_rank] bf16,
 *     cos/sin [seqlen, rope_dim/2] fp32 (position of row r is r % seqlen),
 *     q_out [rows, n_heads*head_dim] bf16.
 *     Supported: n_heads <= 16, head_dim == 64, q_lora_rank a multiple of 64 and <= 256,
 *     rope_dim even and <= head_dim. workspace (256-byte aligned) receives the
 *     int8 slices of wq_b and qr that the call builds;
 *     dsa_indexer_workspace_bytes(rows, 1, n_heads, head_dim, 0, 0) bytes are enough.
 *     Replaces the aclnnMatmul executor (src/task2_indexer.py:763-809) plus
 *     launch_ix_rope / run_rope (src/indexer_kernel_aiv.asc:110-111,
 *     src/task2_indexer.py:724-728); semantics reference/task2_v0_ref.py:129-131.
 */
int dsa_indexer_qproj_rope(const void* qr, const void* wq_b, const float* cos_tab,
                           const float* sin_tab, void* q_out, int64_t rows, int q_lora_rank,
                           int n_heads, int head_dim, int rope_dim, int64_t seqlen,
                           void* workspace, size_t workspace_bytes, void* stream);

/* (b) w = bf16(bf16(x . w_proj^T) * scale).  x [rows, dim] bf16,
 *     w_proj [n_heads, dim] bf16, w_out [rows, n_heads] bf16.
 *     Supported: n_heads == 16, dim a multiple of 64 and <= 1024. The dot
 *     products are exact (int8 slices of both operands on the tensor cores);
 *     workspace: dsa_indexer_wproj_workspace_bytes(rows, dim) bytes, 256-byte
 *     aligned (the slices and per-row exponents).
 *     Replaces the weights_proj executor (src/task2_indexer.py:817-839);
 *     semantics reference/task2_v0_ref.py:132. */
size_t dsa_indexer_wproj_workspace_bytes(int64_t rows, int dim);
int dsa_indexer_wproj(const void* x, const void* w_proj, void* w_out, int64_t rows, int dim,
                      int n_heads, float scale, void* workspace, size_t workspace_bytes,
                      void* stream);

/* (c) Scores and top-k:
 *     score[t,k] = bf16( sum_h bf16( relu(bf16(q[t,h].kv[k])) * w[t,h] ) )
 *     over k < n_cand; with start_pos == 0 the causal mask drops k >= (t+1)/ratio.
 *     out[t, 0:topk] = the candidates in descending score order, ties broken by
 *     ascending k; masked slots are -1; valid slots hold k + offset.
 *     q [batch*seqlen, n_heads*head_dim] bf16, w [batch*seqlen, n_heads] bf16,
 *     kv_cache rows [k] of batch b at kv_cache + b*kv_batch_stride + k*head_dim,
 *     out [batch*seqlen, topk] int64.
 *     Supported: n_heads == 16, head_dim == 64, topk <= n_cand <= 8192;
 *     kv_batch_stride a multiple of 64 and >= n_cand*64. Beyond 1024 candidates
 *     or top-256 the call needs dsa_indexer_score_workspace_bytes of workspace.
 *     Replaces launch_ix_fused / run_fused_t2 (src/indexer_kernel_mm.asc:434-436,
 *     src/task2_indexer.py:730-738); semantics reference/task2_v0_ref.py:133-144.
 */
int dsa_indexer_score_topk(const void* q, const void* w, const void* kv_cache,
                           int64_t kv_batch_stride, int64_t* out, int64_t batch, int64_t seqlen,
                           int n_heads, int head_dim, int64_t n_cand, int topk, int64_t start_pos,
                           int ratio, int64_t offset, void* workspace, size_t workspace_bytes,
                           void* stream);

/* Score-buffer bytes dsa_indexer_score_topk needs (256-byte aligned workspace):
 * 0 when n_cand <= 1024 and topk <= 256 (scores and selection in one kernel),
 * else batch * seqlen * n_cand bf16 scores, sorted by a second kernel
 * (n_cand <= 8192). No counterpart in the reference, whose kernels stop at
 * 672 candidates. */
size_t dsa_indexer_score_workspace_bytes(int64_t batch, int64_t seqlen, int64_t n_cand, int topk);

/* Scratch bytes dsa_indexer_fwd needs: operand slices, the q and w
 * intermediates and the score buffer of dsa_indexer_score_workspace_bytes.
 * n_cand and topk as dsa_indexer_fwd derives them (0, 0 for the projections
 * alone). */
size_t dsa_indexer_workspace_bytes(int64_t batch, int64_t seqlen, int n_heads, int head_dim,
                                   int64_t n_cand, int topk);

/* Extra workspace bytes that let dsa_indexer_fwd, dsa_indexer_fwd_fp8 and
 * dsa_chain_fwd run the q projection (a) and the w projection (b), which are
 * independent, concurrently: given at least their own workspace size plus this
 * (rows = batch * seqlen), (b) runs on a side stream of the calling host thread
 * (created on its first such call outside stream capture, kept until exit) and
 * is joined back into the caller's stream before the scores; with no more than
 * their own size they run one after the other. The results are identical either
 * way. No counterpart in the reference (whose v1 overlaps its weights projection
 * on a side stream of its own, src/task2_indexer.py:817-839). */
size_t dsa_indexer_overlap_extra_bytes(int64_t rows, int n_heads, int head_dim);

/* (a)+(b)+(c) in one call, ordered on `stream`. workspace must hold at least
 * dsa_indexer_workspace_bytes(batch, seqlen, n_heads, head_dim, n_cand, topk)
 * bytes, 256-byte aligned (plus dsa_indexer_overlap_extra_bytes to overlap (a)
 * and (b)). cos/sin cover positions start_pos .. start_pos+seqlen-1.
 * n_cand = (start_pos + seqlen) / ratio; topk = min(index_topk, n_cand).
 * Replaces the whole ModelNew.forward path (src/task2_indexer.py:1056-1349),
 * semantics Model.forward in reference/task2_v0_ref.py:123-144. */
int dsa_indexer_fwd(const void* x, const void* qr, const void* wq_b, const void* w_proj,
                    const float* cos_tab, const float* sin_tab, const void* kv_cache,
                    int64_t kv_batch_stride, int64_t* out, void* workspace,
                    size_t workspace_bytes, int64_t batch, int64_t seqlen, int dim,
                    int q_lora_rank, int n_heads, int head_dim, int rope_dim, int index_topk,
                    int64_t start_pos, int ratio, int64_t offset, float w_scale, void* stream);

/* ---- fp8 index path: ModelArgs.dtype = "fp8", scale_fmt = "ue8m0"
 * (reference/task2_v0_ref.py:25-26; declared there, unused by the bf16 v0
 * path). Definition after DeepSeek-V3.2-Exp's published indexer
 * (inference/model.py Indexer.forward, inference/kernel.py act_quant and
 * fp8_index), one quantization block per 64-wide head row:
 *   h = bf16(FWHT64(x) * 2^-3)          Walsh-Hadamard rotation, fp32 butterflies
 *                                       over strides 1, 2, ..., 32
 *   s = 2^ceil(log2(fp32(max(amax(h), 1e-4) / 448)))      (ue8m0 scale)
 *   y = e4m3(h / s)                     RNE, |h / s| <= 448
 *   score[t,k] = ks[k] * sum_h relu(fp32(q8[t,h] . k8[k])) * wq[t,h]
 *                (wq = w * qs, the head sum an fp32 fma chain in ascending h)
 *   top-k, mask, -1 and offset as dsa_indexer_score_topk.
 * The q8 . k8 products run on tcgen05.mma kind::f8f6f4 with fp32 accumulate. */

/* Rotates and quantizes `rows` 64-wide bf16 rows: row r of group g = r /
 * rows_per_group at x + g*group_stride + (r % rows_per_group)*64 (group_stride
 * in elements, a multiple of 8; rows_per_group >= rows for one contiguous
 * block). y [rows, 64] e4m3 contiguous; scale [rows] f32 or NULL; with w (bf16
 * [rows]) w_out[r] = w[r] * s[r] (exact). Supported: head_dim == 64. */
int dsa_indexer_fp8_quant_rows(const void* x, int64_t rows, int64_t rows_per_group,
                               int64_t group_stride, int head_dim, void* y, float* scale,
                               const void* w, float* w_out, void* stream);

/* Scores and top-k on quantized rows: q8 [batch*seqlen*n_heads, 64] e4m3, wq
 * [batch*seqlen, n_heads] f32, k8 [batch*n_cand, 64] e4m3, ks [batch*n_cand] f32,
 * out [batch*seqlen, topk] int64; scores (NULL or [batch*seqlen, n_cand] f32)
 * receives the fp32 score of every valid candidate (others untouched).
 * Supported: n_heads == 16, head_dim == 64, topk <= 256, n_cand <= 1024. */
int dsa_indexer_score_topk_fp8(const void* q8, const float* wq, const void* k8, const float* ks,
                               int64_t* out, float* scores, int64_t batch, int64_t seqlen,
                               int n_heads, int head_dim, int64_t n_cand, int topk,
                               int64_t start_pos, int ratio, int64_t offset, void* stream);

/* Workspace bytes of dsa_indexer_fwd_fp8 (256-byte aligned). */
size_t dsa_indexer_fp8_workspace_bytes(int64_t batch, int64_t seqlen, int n_heads, int head_dim,
                                       int64_t n_cand);

/* The fp8 variant of dsa_indexer_fwd, same arguments: the bf16 projections and
 * RoPE (bit-exact, as dsa_indexer_fwd), then the rotation and quantization of q
 * (with wq = w * qs) and of kv_cache rows 0 .. n_cand-1 of every batch, then
 * dsa_indexer_score_topk_fp8. Same limits as that call. */
int dsa_indexer_fwd_fp8(const void* x, const void* qr, const void* wq_b, const void* w_proj,
                        const float* cos_tab, const float* sin_tab, const void* kv_cache,
                        int64_t kv_batch_stride, int64_t* out, void* workspace,
                        size_t workspace_bytes, int64_t batch, int64_t seqlen, int dim,
                        int q_lora_rank, int n_heads, int head_dim, int rope_dim, int index_topk,
                        int64_t start_pos, int ratio, int64_t offset, float w_scale,
                        void* stream);

/* ---- kv_cache writer: the producer of the compressed index-key cache that
 * dsa_indexer_fwd reads (reference/task2_v0_ref.py:119,133 read
 * kv_cache[:bsz, :end_pos // ratio]; the reference contains no producer).
 * Definition after DeepSeek-V3.2-Exp's indexer key path (inference/model.py
 * Indexer.forward: k = wk(x), LayerNorm, RoPE), the rotary dims last as this
 * reference's q, and each block of `ratio` tokens pooled by its mean:
 *   kl[t] = bf16(x[t] . wk^T)       (tensor cores, fp32 accumulation)
 *   kn[t] = bf16(((kl - mean) * (1 / sqrt(var + 1e-6))) * ln_weight + ln_bias)
 *   k[t]  = RoPE of kn's last rope_dim dims at position start_pos + t
 *   kv_cache[b, start_pos / ratio + j] = bf16(mean_{i < ratio} k[j ratio + i])
 * for the seqlen / ratio complete blocks (j = 0 .. seqlen / ratio - 1); other rows
 * are untouched. x [batch*seqlen, dim] bf16, wk [head_dim, dim] bf16, ln_weight /
 * ln_bias [head_dim] f32, cos/sin [seqlen, rope_dim/2] f32 (positions start_pos..),
 * kv_cache rows of batch b at kv_cache + b*kv_batch_stride (kv_rows rows of
 * head_dim). Supported: head_dim == 64, dim a multiple of 64, ratio dividing 128,
 * start_pos a multiple of ratio. No counterpart in the reference (see above). */
int dsa_kv_cache_write(const void* x, const void* wk, const float* ln_weight,
                       const float* ln_bias, const float* cos_tab, const float* sin_tab,
                       void* kv_cache, int64_t kv_batch_stride, int64_t kv_rows, int64_t batch,
                       int64_t seqlen, int dim, int head_dim, int rope_dim, int64_t start_pos,
                       int ratio, void* stream);

/* dsa_indexer_fwd for callers that cannot allocate device memory at call
 * time -- plug-ins whose host framework owns all device memory and forbids
 * allocating inside an operator, or latency-critical paths where a
 * cudaMalloc/cudaFree (which can synchronize the device) is not acceptable.
 * Same arguments and result as dsa_indexer_fwd, without the workspace: the
 * operand slices and the q and w intermediates live in a fixed 128 MiB array inside the library, one per
 * device that loads it, held until the process exits. The request needs
 * dsa_indexer_workspace_bytes(batch, seqlen, n_heads, head_dim, n_cand, topk)
 * <= 128 MiB, i.e. at most 25,981 tokens (batch*seqlen) at 16 heads x 64 dims
 * with n_cand <= 1024 and topk <= 256 (fewer with a score buffer); larger
 * requests return DSA_ERR_WORKSPACE and launch nothing. Each CUDA context that
 * loads the library (the device's primary context, or a context the caller
 * created and made current) holds its own copy of the array; the first call in
 * a context looks up that copy's address; make it before any stream capture.
 * Every call on a device uses the same array, so calls that overlap on the GPU
 * race. This entry point has no counterpart in the reference. */
int dsa_indexer_fwd_noalloc(const void* x, const void* qr, const void* wq_b, const void* w_proj,
                            const float* cos_tab, const float* sin_tab, const void* kv_cache,
                            int64_t kv_batch_stride, int64_t* out, int64_t batch, int64_t seqlen,
                            int dim, int q_lora_rank, int n_heads, int head_dim, int rope_dim,
                            int index_topk, int64_t start_pos, int ratio, int64_t offset,
                            float w_scale, void* stream);

/* ------------------------------------------------------------------------
 * Chained path: the indexer's top-k selection feeding SparseAttention over a kv
 * pool in one call (x[4,16384,1024], kv_cache[4,4096,64],
 * top-2048, then q[4,16384,64,128] over a kv pool [4,4096,128]). The result is
 * the one of dsa_indexer_fwd followed by dsa_sparse_attn_fwd on its int64
 * output, i.e. sparse_attn_ref(q, kv, sink, Model.forward(x, qr, start_pos,
 * offset), scale) (reference/task2_v0_ref.py:123-144, reference/task1_v0_ref.py
 * :5-24): attention in the multiplicity form depends only on which pool rows a
 * token selected, so the selection travels as one bitmap per token (n_cand bits,
 * bit k = pool row k + offset) instead of an int64 list, and no sort runs.
 * Indexer arguments as dsa_indexer_fwd; attention arguments as
 * dsa_sparse_attn_fwd (q [batch, seqlen, attn_heads, attn_head_dim], kv
 * [batch, n_kv, attn_head_dim], out like q). Supported: n_cand <= 8192,
 * attn_heads in {64,128}, attn_head_dim 128, n_kv <= 4096. workspace:
 * dsa_chain_workspace_bytes(batch, seqlen, ix_heads, ix_head_dim, n_cand)
 * bytes, 256-byte aligned. The reference runs the two modules one after the
 * other; it has no fused counterpart. */
size_t dsa_chain_workspace_bytes(int64_t batch, int64_t seqlen, int n_heads, int head_dim,
                                 int64_t n_cand);
int dsa_chain_fwd(const void* x, const void* qr, const void* wq_b, const void* w_proj,
                  const float* cos_tab, const float* sin_tab, const void* kv_cache,
                  int64_t kv_batch_stride, int64_t batch, int64_t seqlen, int dim,
                  int q_lora_rank, int ix_heads, int ix_head_dim, int rope_dim, int index_topk,
                  int64_t start_pos, int ratio, int64_t offset, float w_scale, const void* q,
                  const void* kv, int n_kv, int attn_heads, int attn_head_dim,
                  const float* sink, float softmax_scale, void* out, void* workspace,
                  size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* DSA_B200_H_ */
