/*
 * dsa_oracle.c -- CPU restatement of the reference's three v0 operators.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the parity checker for the CUDA
 * library (and the timed CPU baseline of the bench). It is never linked into,
 * loaded by, or called from the product path in ascendc_kernel_b200/.
 *
 * Each function cites the reference lines it restates (paths relative to the
 * reference repository). Numeric contract, shared with the CUDA kernels:
 *  - A bf16 "GEMM" result (F.linear / einsum with bf16 inputs and output) is
 *    the correctly rounded (RNE) bf16 value of the dot product, which is formed
 *    in fp64 in ascending index order. Every bf16 x bf16 product is exact in
 *    fp64, so the fp64 sum is the exact dot product whenever the terms span
 *    fewer than 2^(53-16-log2 K) in magnitude, i.e. for all practical data.
 *  - Elementwise bf16 ops (x * w, x * scale) are fp32 products rounded to
 *    bf16 (torch's opmath), RoPE is the non-fused fp32 complex product
 *    (a*c - b*s, a*s + b*c) rounded once to bf16, and the head sum is exact
 *    then rounded once.
 *  - SparseAttention is computed in fp64 (gather form) and rounded to bf16;
 *    Sinkhorn follows the reference's fp32 op order.
 * Compile with -ffp-contract=off (oracle/Makefile does).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------ bf16 */
static inline float bf2f(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

static inline uint16_t f2bf(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((u >> 16) | 0x40u); /* quiet NaN */
  u += 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

/* Correctly rounded double -> bf16: round to odd into fp32 (24 bits), then
 * RNE to bf16 (8 bits); 24 >= 8 + 2 makes the double rounding exact. */
static inline uint16_t d2bf(double d) {
  float f = (float)d;
  if (isfinite(f) && (double)f != d) {
    if (fabs((double)f) > fabs(d)) f = nextafterf(f, 0.0f);
    uint32_t u;
    memcpy(&u, &f, 4);
    u |= 1u;
    memcpy(&f, &u, 4);
  }
  return f2bf(f);
}

int oracle_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

void oracle_set_num_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

/* --------------------------------------------------------------- Sinkhorn
 * reference/task3_v0_ref.py:8-14:
 *   x = x.softmax(-1) + eps
 *   x = x / (x.sum(-2, keepdim=True) + eps)
 *   for _ in range(repeat - 1):
 *       x = x / (x.sum(-1, keepdim=True) + eps)
 *       x = x / (x.sum(-2, keepdim=True) + eps)
 * x, y: [n_mat, n, n] fp32. Sums run in index order in fp32; exp is the
 * correctly rounded fp32 exp (computed in double and rounded).
 */
void oracle_sinkhorn(const float* x, float* y, int64_t n_mat, int n, int repeat, float eps) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n_mat; ++i) {
    float a[16 * 16];
    const float* xi = x + i * n * n;
    for (int r = 0; r < n; ++r) {
      float mx = xi[r * n];
      for (int c = 1; c < n; ++c) mx = fmaxf(mx, xi[r * n + c]);
      float s = 0.f;
      for (int c = 0; c < n; ++c) {
        a[r * n + c] = (float)exp((double)(xi[r * n + c] - mx));
        s += a[r * n + c];
      }
      for (int c = 0; c < n; ++c) a[r * n + c] = a[r * n + c] / s + eps;
    }
    for (int it = 0; it < 2 * repeat - 1; ++it) {
      if (it % 2 == 0) { /* column normalisation: sum over dim -2 */
        for (int c = 0; c < n; ++c) {
          float s = 0.f;
          for (int r = 0; r < n; ++r) s += a[r * n + c];
          s += eps;
          for (int r = 0; r < n; ++r) a[r * n + c] = a[r * n + c] / s;
        }
      } else { /* row normalisation: sum over dim -1 */
        for (int r = 0; r < n; ++r) {
          float s = 0.f;
          for (int c = 0; c < n; ++c) s += a[r * n + c];
          s += eps;
          for (int c = 0; c < n; ++c) a[r * n + c] = a[r * n + c] / s;
        }
      }
    }
    memcpy(y + i * n * n, a, sizeof(float) * n * n);
  }
}

/* --------------------------------------------------------- SparseAttention
 * reference/task1_v0_ref.py:5-24 (gather form), fp64 throughout:
 *   s_j  = (q[b,t,h] . kv[b, idx_j]) * scale   for valid j (idx_j >= 0)
 *   mx   = max(max_j s_j, sink[h])
 *   w_j  = exp(s_j - mx) / (sum_j exp(s_j - mx) + exp(sink[h] - mx))
 *   out  = bf16(sum_j w_j kv[b, idx_j])
 * idx: int32 (idx_bytes 4) or int64 (8); entries < 0 or >= n_kv are masked
 * (the reference indexes out of range for >= n_kv; the CUDA path masks them).
 */
void oracle_sparse_attn(const uint16_t* q, const uint16_t* kv, const void* idx, int idx_bytes,
                        const float* sink, uint16_t* out, int64_t B, int64_t M, int H, int D,
                        int NKV, int TOPK, double scale) {
#pragma omp parallel
  {
    int64_t* ids = (int64_t*)malloc(sizeof(int64_t) * (size_t)TOPK);
    double* sc = (double*)malloc(sizeof(double) * (size_t)TOPK);
    double* acc = (double*)malloc(sizeof(double) * (size_t)D);
#pragma omp for schedule(dynamic, 16)
    for (int64_t bt = 0; bt < B * M; ++bt) {
      const int64_t b = bt / M;
      int nv = 0;
      for (int j = 0; j < TOPK; ++j) {
        int64_t v = idx_bytes == 8 ? ((const int64_t*)idx)[bt * TOPK + j]
                                   : (int64_t)((const int32_t*)idx)[bt * TOPK + j];
        if (v >= 0 && v < NKV) ids[nv++] = v;
      }
      for (int h = 0; h < H; ++h) {
        const uint16_t* qh = q + (bt * H + h) * D;
        double mx = (double)sink[h];
        for (int j = 0; j < nv; ++j) {
          const uint16_t* kr = kv + (b * NKV + ids[j]) * D;
          double s = 0.0;
          for (int d = 0; d < D; ++d) s += (double)bf2f(qh[d]) * (double)bf2f(kr[d]);
          sc[j] = s * scale;
          if (sc[j] > mx) mx = sc[j];
        }
        double den = exp((double)sink[h] - mx);
        for (int j = 0; j < nv; ++j) {
          sc[j] = exp(sc[j] - mx);
          den += sc[j];
        }
        for (int d = 0; d < D; ++d) acc[d] = 0.0;
        for (int j = 0; j < nv; ++j) {
          const uint16_t* kr = kv + (b * NKV + ids[j]) * D;
          const double wj = sc[j] / den;
          for (int d = 0; d < D; ++d) acc[d] += wj * (double)bf2f(kr[d]);
        }
        uint16_t* o = out + (bt * H + h) * D;
        for (int d = 0; d < D; ++d) o[d] = d2bf(acc[d]);
      }
    }
    free(ids);
    free(sc);
    free(acc);
  }
}

/* ------------------------------------------------------------ bf16 linear
 * F.linear(x, W) for bf16 x [rows, K] and W [N, K] (reference/task2_v0_ref.py:
 * 75-77,83-84): out[r, n] = RNE_bf16(sum_k x[r,k] W[n,k]), the sum formed in
 * fp64 in ascending k. W is transposed once so the inner loop runs over n
 * (each output still accumulates in ascending k).
 */
void oracle_linear_bf16(const uint16_t* x, const uint16_t* w, uint16_t* out, int64_t rows, int K,
                        int N) {
  double* wt = (double*)malloc(sizeof(double) * (size_t)K * N);
  for (int n = 0; n < N; ++n)
    for (int k = 0; k < K; ++k) wt[(size_t)k * N + n] = (double)bf2f(w[(size_t)n * K + k]);
#pragma omp parallel
  {
    double* acc = (double*)malloc(sizeof(double) * (size_t)N);
#pragma omp for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
      for (int n = 0; n < N; ++n) acc[n] = 0.0;
      const uint16_t* xr = x + r * K;
      for (int k = 0; k < K; ++k) {
        const double xv = (double)bf2f(xr[k]);
        const double* wk = wt + (size_t)k * N;
        for (int n = 0; n < N; ++n) acc[n] += xv * wk[n];
      }
      for (int n = 0; n < N; ++n) out[r * N + n] = d2bf(acc[n]);
    }
    free(acc);
  }
  free(wt);
}

/* ------------------------------------------------------------------ RoPE
 * apply_rotary_emb on q[..., -rope_dim:] (reference/task2_v0_ref.py:93-104,131):
 * interleaved pairs (re, im) = (x[2i], x[2i+1]) of the rope part, times
 * freqs_cis = cos + i sin in fp32 complex arithmetic, written back as bf16:
 *   re' = RNE(fl(re*c) - fl(im*s)),  im' = RNE(fl(re*s) + fl(im*c)).
 * q: [rows, n_heads, head_dim] bf16 in place; cos/sin: [seqlen, rope_dim/2]
 * fp32; row r is at position r % seqlen of the table.
 */
void oracle_rope(uint16_t* q, const float* cos_t, const float* sin_t, int64_t rows, int n_heads,
                 int head_dim, int rope_dim, int64_t seqlen) {
  const int half = rope_dim / 2;
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r) {
    const int64_t pos = r % seqlen;
    for (int h = 0; h < n_heads; ++h) {
      uint16_t* x = q + (r * n_heads + h) * head_dim + (head_dim - rope_dim);
      for (int i = 0; i < half; ++i) {
        const float re = bf2f(x[2 * i]);
        const float im = bf2f(x[2 * i + 1]);
        const float c = cos_t[pos * half + i];
        const float s = sin_t[pos * half + i];
        const float ac = re * c;
        const float bs = im * s;
        const float as = re * s;
        const float bc = im * c;
        x[2 * i] = f2bf(ac - bs);
        x[2 * i + 1] = f2bf(as + bc);
      }
    }
  }
}

/* w = bf16(fp32(w) * scale)  (reference/task2_v0_ref.py:132, the `* scalar`). */
void oracle_scale_bf16(uint16_t* w, int64_t n, float scale) {
  for (int64_t i = 0; i < n; ++i) w[i] = f2bf(bf2f(w[i]) * scale);
}

/* ------------------------------------------------------- index scores/top-k
 * reference/task2_v0_ref.py:133-143:
 *   s      = bf16(q[t,h] . kv[k])                          (einsum, bf16 out)
 *   e      = bf16(fp32(relu(s)) * fp32(w[t,h]))            (relu_, * weights)
 *   score  = bf16(sum_h e)                                 (.sum(dim=2))
 *   mask   : start_pos == 0 -> k >= (t+1)//ratio is -inf
 *   topk(min(index_topk, T)) then -1 for masked slots, else k + offset
 * Ordering of the selection: descending score, ties by ascending k (-0 == +0).
 * q [B*S, H*Dh] bf16, w [B*S, H] bf16, kv rows at kv + b*kv_bstride + k*Dh.
 * out [B*S, K] int64; scores (optional) [B*S, T] bf16 with masked = 0xFF80
 * (bf16 -inf).
 */
static int cmp_desc_u64(const void* a, const void* b) {
  const uint64_t x = *(const uint64_t*)a, y = *(const uint64_t*)b;
  return x < y ? 1 : (x > y ? -1 : 0);
}

void oracle_index_topk(const uint16_t* q, const uint16_t* w, const uint16_t* kv,
                       int64_t kv_bstride, int64_t* out, uint16_t* scores_out, int64_t B,
                       int64_t S, int H, int Dh, int64_t T, int K, int64_t start_pos, int ratio,
                       int64_t offset) {
#pragma omp parallel
  {
    double* kvt = NULL;
    int64_t kvt_b = -1;
    double* dots = (double*)malloc(sizeof(double) * (size_t)T);
    uint64_t* keys = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)T);
    float* tot = (float*)malloc(sizeof(float) * (size_t)T);
    double* etot = (double*)malloc(sizeof(double) * (size_t)T);
    kvt = (double*)malloc(sizeof(double) * (size_t)T * Dh);
#pragma omp for schedule(dynamic, 8)
    for (int64_t bt = 0; bt < B * S; ++bt) {
      const int64_t b = bt / S, t = bt % S;
      if (kvt_b != b) { /* transposed fp64 copy of kv[b]: kvt[d][k] */
        for (int64_t k = 0; k < T; ++k)
          for (int d = 0; d < Dh; ++d)
            kvt[(size_t)d * T + k] = (double)bf2f(kv[b * kv_bstride + k * Dh + d]);
        kvt_b = b;
      }
      int64_t nv = T;
      if (start_pos == 0) {
        nv = (t + 1) / ratio;
        if (nv > T) nv = T;
      }
      for (int64_t k = 0; k < nv; ++k) etot[k] = 0.0;
      for (int h = 0; h < H; ++h) {
        const uint16_t* qh = q + (bt * H + h) * Dh;
        for (int64_t k = 0; k < nv; ++k) dots[k] = 0.0;
        for (int d = 0; d < Dh; ++d) {
          const double qv = (double)bf2f(qh[d]);
          const double* kd = kvt + (size_t)d * T;
          for (int64_t k = 0; k < nv; ++k) dots[k] += qv * kd[k];
        }
        const float wh = bf2f(w[bt * H + h]);
        for (int64_t k = 0; k < nv; ++k) {
          float s = bf2f(d2bf(dots[k]));
          if (!(s > 0.f)) s = 0.f; /* relu (and -0 -> +0) */
          etot[k] += (double)bf2f(f2bf(s * wh));
        }
      }
      for (int64_t k = 0; k < nv; ++k) {
        uint16_t sb = d2bf(etot[k]);
        if (sb == 0x8000u) sb = 0;
        tot[k] = bf2f(sb);
        const uint16_t ord = (sb & 0x8000u) ? (uint16_t)~sb : (uint16_t)(sb | 0x8000u);
        keys[k] = ((uint64_t)ord << 32) | (uint64_t)(0xFFFFFFFFu - (uint32_t)k);
      }
      if (scores_out) {
        for (int64_t k = 0; k < T; ++k)
          scores_out[bt * T + k] = k < nv ? d2bf(etot[k]) : (uint16_t)0xFF80u;
      }
      qsort(keys, (size_t)nv, sizeof(uint64_t), cmp_desc_u64);
      int64_t* o = out + bt * K;
      for (int j = 0; j < K; ++j) {
        if (j < nv) {
          const int64_t k = (int64_t)(0xFFFFFFFFu - (uint32_t)(keys[j] & 0xFFFFFFFFu));
          o[j] = k + offset;
        } else {
          o[j] = start_pos == 0 ? -1 : 0; /* only reachable when start_pos == 0 */
        }
      }
      (void)tot;
    }
    free(dots);
    free(keys);
    free(tot);
    free(etot);
    free(kvt);
  }
}

/* ------------------------------------------------------------ fp8 index path
 * The fp8 variant that ModelArgs.dtype = "fp8", scale_fmt = "ue8m0" declares
 * (reference/task2_v0_ref.py:25-26) and the reference's bf16 v0 path never
 * uses. Restated from the published indexer of DeepSeek-V3.2-Exp
 * (inference/model.py, Indexer.forward: rotate_activation, act_quant with
 * scale_fmt, weights * q_scale, fp8_index; inference/kernel.py, act_quant and
 * fp8_index), with one quantization block per 64-wide head row:
 *   h = bf16(FWHT64(x) * 2^-3)   Walsh-Hadamard in fp32, butterflies (a+b, a-b)
 *                                over strides 1, 2, 4, ..., 32
 *   s = 2^ceil(log2(fp32(max(max|h|, 1e-4) / 448)))      (ue8m0 scale)
 *   y = e4m3(h / s)              RNE, |h / s| <= 448
 *   score[t,k] = ks[k] * sum_h relu(fp32(q8[t,h] . k8[k])) * wq[t,h]
 *     with the e4m3 dot product exact (fp64) then rounded once to fp32, the
 *     head sum an fp32 fma chain in ascending h, wq = fp32(w) * qs.
 *   Mask, top-k order (score desc, k asc, -0 == +0), -1 and offset as
 *   oracle_index_topk.
 */

/* fp32 -> e4m3 (float8_e4m3fn) bits, RNE, saturating to +-448; NaN -> 0x7F. */
uint8_t oracle_e4m3_from_f32(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  const uint8_t sign = (uint8_t)((u >> 24) & 0x80u);
  const float a = fabsf(f);
  if (a != a) return 0x7Fu;
  if (a >= 448.0f) return (uint8_t)(sign | 0x7Eu);
  if (a < 0.015625f) { /* below 2^-6: multiples of 2^-9 (subnormals) */
    const int m = (int)rintf(a * 512.0f); /* a * 2^9 exact; rintf is RNE */
    return (uint8_t)(sign | (uint8_t)m);  /* m == 8 encodes 2^-6 */
  }
  int e;
  const float fr = frexpf(a, &e); /* a = fr * 2^e, fr in [0.5, 1) */
  int q = (int)rintf((fr * 2.0f - 1.0f) * 8.0f); /* exact: 24-bit significand */
  int ex = e - 1 + 7;
  if (q == 8) {
    q = 0;
    ex += 1;
  }
  return (uint8_t)(sign | (uint8_t)(ex << 3) | (uint8_t)q);
}

static inline double e4m3_to_f64(uint8_t b) {
  const int s = b >> 7, ex = (b >> 3) & 15, m = b & 7;
  double v;
  if (ex == 0)
    v = ldexp((double)m, -9);
  else
    v = ldexp((double)(8 + m), ex - 10);
  return s ? -v : v;
}

static inline float bf16_round_f32(float f) { return bf2f(f2bf(f)); }

/* x [rows, 64] bf16 -> y [rows, 64] e4m3 bits, scale [rows] (may be NULL). */
void oracle_fp8_quant_rows(const uint16_t* x, int64_t rows, uint8_t* y, float* scale) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r) {
    float h[64];
    for (int i = 0; i < 64; ++i) h[i] = bf2f(x[r * 64 + i]);
    for (int len = 1; len < 64; len <<= 1)
      for (int i = 0; i < 64; i += 2 * len)
        for (int j = i; j < i + len; ++j) {
          const float a = h[j], b = h[j + len];
          h[j] = a + b;
          h[j + len] = a - b;
        }
    float amax = 0.0f;
    for (int i = 0; i < 64; ++i) {
      h[i] = bf16_round_f32(h[i] * 0.125f);
      const float ah = fabsf(h[i]);
      if (ah > amax) amax = ah;
    }
    if (amax < 1e-4f) amax = 1e-4f;
    const float q = amax / 448.0f;
    uint32_t qu;
    memcpy(&qu, &q, 4);
    const int e = (int)((qu >> 23) & 0xFFu) - 127 + ((qu & 0x7FFFFFu) != 0u ? 1 : 0);
    const float s = ldexpf(1.0f, e);
    for (int i = 0; i < 64; ++i) y[r * 64 + i] = oracle_e4m3_from_f32(h[i] / s);
    if (scale) scale[r] = s;
  }
}

/* q8 [B*S*H, Dh] e4m3, wq [B*S*H] f32, k8 [B*T, Dh] e4m3, ks [B*T] f32;
 * out [B*S, K] int64; scores_out (NULL or [B*S, T] f32, masked = -inf). */
void oracle_index_topk_fp8(const uint8_t* q8, const float* wq, const uint8_t* k8,
                           const float* ks, int64_t* out, float* scores_out, int64_t B,
                           int64_t S, int H, int Dh, int64_t T, int K, int64_t start_pos,
                           int ratio, int64_t offset) {
#pragma omp parallel
  {
    uint64_t* keys = (uint64_t*)malloc(sizeof(uint64_t) * (size_t)T);
    double* qd = (double*)malloc(sizeof(double) * (size_t)H * Dh);
#pragma omp for schedule(dynamic, 8)
    for (int64_t bt = 0; bt < B * S; ++bt) {
      const int64_t b = bt / S, t = bt % S;
      int64_t nv = T;
      if (start_pos == 0) {
        nv = (t + 1) / ratio;
        if (nv > T) nv = T;
      }
      for (int i = 0; i < H * Dh; ++i) qd[i] = e4m3_to_f64(q8[bt * H * Dh + i]);
      for (int64_t k = 0; k < nv; ++k) {
        const uint8_t* kr = k8 + (b * T + k) * Dh;
        double kd[256];
        for (int d = 0; d < Dh; ++d) kd[d] = e4m3_to_f64(kr[d]);
        float acc = 0.0f;
        for (int h = 0; h < H; ++h) {
          double dot = 0.0; /* exact: e4m3 products and their sum fit in fp64 */
          for (int d = 0; d < Dh; ++d) dot += qd[h * Dh + d] * kd[d];
          float df = (float)dot;
          if (!(df > 0.0f)) df = 0.0f;
          acc = fmaf(df, wq[bt * H + h], acc);
        }
        float sc = acc * ks[b * T + k];
        if (scores_out) scores_out[bt * T + k] = sc;
        uint32_t u;
        memcpy(&u, &sc, 4);
        if (u == 0x80000000u) u = 0;
        const uint32_t ord = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
        keys[k] = ((uint64_t)ord << 32) | (uint64_t)(0xFFFFFFFFu - (uint32_t)k);
      }
      if (scores_out)
        for (int64_t k = nv; k < T; ++k) scores_out[bt * T + k] = -INFINITY;
      qsort(keys, (size_t)nv, sizeof(uint64_t), cmp_desc_u64);
      int64_t* o = out + bt * K;
      for (int j = 0; j < K; ++j)
        o[j] = j < nv ? (int64_t)(0xFFFFFFFFu - (uint32_t)(keys[j] & 0xFFFFFFFFu)) + offset : -1;
    }
    free(keys);
    free(qd);
  }
}

void oracle_e4m3_array(const float* x, int64_t n, uint8_t* y) {
  for (int64_t i = 0; i < n; ++i) y[i] = oracle_e4m3_from_f32(x[i]);
}

/* --------------------------------------------------------- kv_cache writer
 * Producer of the compressed cache the indexer reads (reference/task2_v0_ref.py:
 * 119,133: kv_cache[:bsz, :end_pos // ratio], compress_ratio), which the
 * reference itself does not contain. Restated from the indexer key path of
 * DeepSeek-V3.2-Exp (inference/model.py, Indexer.forward: k = wk(x),
 * k = k_norm(k) (LayerNorm, fp32, eps 1e-6), RoPE on the rotary dims, written to
 * the cache at the token positions), with the rotary dims taken as the last
 * rope_dim dims as this reference's q (reference/task2_v0_ref.py:131), and
 * blocks of `ratio` consecutive tokens pooled by their mean (NSA-style block
 * compression with a uniform map; ratio 1 writes every token as V3.2-Exp does):
 *   kl[t]  = bf16(x[t] . wk^T)                       (correctly rounded)
 *   mu     = fp32(sum_i kl_i) / 64, var = fp32(sum_i (kl_i - mu)^2) / 64
 *                                                     (sequential, separately rounded)
 *   kn_i   = bf16(((kl_i - mu) * (1 / sqrt(var + 1e-6))) * g_i + b_i)
 *   k[t]   = RoPE of kn's last rope_dim dims at position start_pos + t (as
 *            oracle_rope), bf16
 *   cache[b, start_pos / ratio + j] = bf16(fp32(sum_{i<ratio} k[j ratio + i]) / ratio)
 *            for every block j with (j + 1) ratio <= seqlen.
 * x [B*S, dim] bf16, wk [64, dim] bf16, g/b [64] f32, cos/sin [S, rope_dim/2] f32,
 * kv [B, ...] with batch stride kv_bstride elements.
 */
void oracle_kv_writer(const uint16_t* x, const uint16_t* wk, const float* g, const float* bta,
                      const float* cos_t, const float* sin_t, uint16_t* kv, int64_t kv_bstride,
                      int64_t B, int64_t S, int dim, int rope_dim, int64_t start_pos,
                      int ratio) {
  const int64_t rows = B * S;
  uint16_t* keys = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)rows * 64);
  oracle_linear_bf16(x, wk, keys, rows, dim, 64);
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r) {
    uint16_t* k = keys + r * 64;
    float v[64];
    float s = 0.0f;
    for (int i = 0; i < 64; ++i) {
      v[i] = bf2f(k[i]);
      s += v[i];
    }
    const float mu = s / 64.0f;
    float q = 0.0f;
    for (int i = 0; i < 64; ++i) {
      const float d = v[i] - mu;
      q += d * d;
    }
    const float var = q / 64.0f;
    const float rstd = 1.0f / sqrtf(var + 1e-6f);
    for (int i = 0; i < 64; ++i) k[i] = f2bf(((v[i] - mu) * rstd) * g[i] + bta[i]);
  }
  oracle_rope(keys, cos_t, sin_t, rows, 1, 64, rope_dim, S);
  const int64_t nblk = S / ratio;
  for (int64_t b = 0; b < B; ++b)
    for (int64_t j = 0; j < nblk; ++j) {
      uint16_t* dst = kv + b * kv_bstride + (start_pos / ratio + j) * 64;
      for (int d = 0; d < 64; ++d) {
        float s = 0.0f;
        for (int i = 0; i < ratio; ++i) s += bf2f(keys[(b * S + j * ratio + i) * 64 + d]);
        dst[d] = f2bf(s / (float)ratio);
      }
    }
  free(keys);
}
