// Lightning Indexer scores + causal mask + top-k for sm_100a.
//
// Semantics (reference/task2_v0_ref.py:133-143), for token t of batch b:
//   s[h,k]   = bf16(q[t,h] . kv[b,k])                (correctly rounded)
//   e[h,k]   = bf16(relu(s[h,k]) * w[t,h])           (fp32 product, RNE)
//   score[k] = bf16(sum_h e[h,k])                    (fp64 sum in h order, RNE)
//   valid k  < n_r = (start_pos == 0 ? min((t+1)/ratio, T) : T)
//   out[t]   = top-K valid k by (score desc, k asc); slots past n_r are -1,
//              valid slots hold k + offset.
//
// B200 mapping (one CTA per SM, persistent; a work unit is one batch and 16
// consecutive tokens, scheduled heaviest causal block first):
//   warp 0      TMA: the unit's q tile (16 tokens x 16 heads = 256 rows x 64,
//               32 KB, double buffered) and 128-row kv chunks (16 KB, 3 stages)
//   warp 1      tcgen05: D[128 kv rows x 256 (t,h)] = KV_chunk . Q^T (K = 64)
//               into one of two 256-column TMEM buffers
//   warps 4..11 two epilogue warpgroups (tokens 0-7 / 8-15 of the unit). A
//               thread owns one kv row: it loads its 16 head values per token,
//               certifies each bf16 rounding against the accumulation bound
//               (numerics.cuh; elements that cannot be certified are
//               recomputed exactly by the whole warp), runs the relu / *w /
//               head-sum chain and stores the orderable 16-bit score of every
//               valid candidate in one of two key buffers in shared memory.
//   warps 2, 3, 12..15  top-K selection, one unit behind the epilogue: the
//               six warps take the unit's eight token pairs in turn (a binary
//               search over the 16 score bits, ties by ascending k, then a
//               register bitonic sort), write the int64 indices and hand the
//               key buffer back once all eight pairs are done. The selection of
//               one unit thus overlaps the score chain of the next.
// Registers: 512 threads launch with 128 each; the epilogue warpgroups raise
// theirs to 144 and the other two lower theirs to 112 (setmaxnreg), which adds
// up to the launch's 65,536.
#include "common.cuh"
#include "host_util.h"
#include "numerics.cuh"

namespace dsa {
namespace ixs {

constexpr int kHeads = 16;
constexpr int kDim = 64;
constexpr int kTB = 16;                  // tokens per unit
constexpr int kQRows = kTB * kHeads;     // 256
constexpr int kChunk = 128;              // kv rows per MMA
constexpr int kMaxT = 1024;              // candidates held in smem per token
constexpr int kMaxK = 256;               // top-k held in registers
constexpr int kKVStages = 3;
constexpr int kThreads = 512;  // warps 0 TMA, 1 MMA, 2-3 and 12-15 selection, 4-11 epilogue
constexpr int kSelWarps = 6;
constexpr int kEpiWarp0 = 4;
constexpr int kLaunchRegs = 128;   // 65536 / kThreads: the kernel must compile to exactly this
constexpr int kEpiRegs = 144;      // epilogue warpgroups (1, 2)
constexpr int kOtherRegs = 112;    // warpgroups 0 (producers, 2 selection warps) and 3 (selection)
static_assert(2 * kEpiRegs + 2 * kOtherRegs == 4 * kLaunchRegs, "register split must add up");
constexpr uint32_t kTmemCols = 512;

constexpr int kQBytes = kQRows * 128;    // 32 KB
constexpr int kKVBytes = kChunk * 128;   // 16 KB
constexpr int kKeyBufBytes = kTB * kMaxT * 2;                 // 32 KB: [16 tokens][1024] u16
constexpr int kOffQ = 0;
constexpr int kOffKV = kOffQ + 2 * kQBytes;                   // 65536
constexpr int kOffKeys = kOffKV + kKVStages * kKVBytes;       // 114688: two key buffers
constexpr int kOffQN = kOffKeys + 2 * kKeyBufBytes;           // 180224
constexpr int kOffW = kOffQN + kQRows * 4;                    // 181248
constexpr int kOffRq = kOffW + kQRows * 4;                    // 182272: drain queue per epilogue warp
constexpr int kRqBytes = 4096;  // also the warp's selection scratch between units
static_assert(kRqBytes >= 2 * kMaxK * 4, "drain queue region too small for selection scratch");
constexpr int kOffSel = kOffRq + 8 * kRqBytes;                // 223232: two [kMaxK] lists per selection warp
constexpr int kSelBytes = 2 * kMaxK * 4;
constexpr int kOffNV = kOffSel + kSelWarps * kSelBytes;       // 227328: [16] int
constexpr int kOffWP = kOffNV + kTB * 4;                      // [256] w as bf16x2 {w, w}
constexpr int kOffPS = kOffWP + kQRows * 4;                   // [256] prmt selector
constexpr int kOffBar = kOffPS + kQRows * 4;
constexpr int kNumBars = 2 + 2 + 2 * kKVStages + 2 + 2 + 2 + 2;
constexpr int kOffMisc = kOffBar + kNumBars * 8;
constexpr int kSmem = kOffMisc + 16 + 1024;
static_assert(kSmem <= 232448, "shared memory above the 227 KB per-block limit");

// Accumulation bound for one K = 64 accumulator (4 MMA steps at 3 fp32 ulps
// each, in units of ||q|| * ||kv||).
constexpr float kGamma = 24.0f * kTwoM24 * 1.0001f;

struct Params {
  int B;
  int64_t S;
  int64_t T;          // candidates (end_pos / ratio)
  int K;              // top-k (min(index_topk, T))
  int ratio;
  int causal;         // start_pos == 0
  int64_t offset;
  int n_tb;           // token blocks per batch
  int units;
  int64_t kv_rows_per_batch;  // kv_batch_stride / 64
  const uint16_t* w;  // [B*S, 16]
  int64_t* out;       // [B*S, K] (top-k in the kernel), or
  uint16_t* scores;   // [B*S, score_ld] bf16 scores of the valid candidates (sorted later)
  int64_t score_ld;
  unsigned int* err;
};

__device__ __forceinline__ uint32_t sw128_off(int row, int chunk16) {
  return static_cast<uint32_t>(row * 128 + ((chunk16 ^ (row & 7)) << 4));
}

__device__ __forceinline__ int64_t n_valid(const Params& p, int64_t t) {
  if (!p.causal) return p.T;
  const int64_t n = (t + 1) / p.ratio;
  return n < p.T ? n : p.T;
}

// Row norm (upper bound) of a 64-wide bf16 row stored SW128 in smem.
// The squares go straight from the bf16 halves into four partial sums (mixed
// bf16 x bf16 + fp32 fma, one rounding each); norm_upper's bound holds for any
// summation order of the 64 terms.
__device__ __forceinline__ float row_norm64(const uint8_t* base, int row) {
  float ss[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int ch = 0; ch < 8; ++ch) {
    const uint4 v = *reinterpret_cast<const uint4*>(base + sw128_off(row, ch));
    const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      ss[e] = fma_bf16lo(w4[e], w4[e], ss[e]);
      ss[e] = fma_bf16hi(w4[e], w4[e], ss[e]);
    }
  }
  return norm_upper((ss[0] + ss[1]) + (ss[2] + ss[3]), kDim);
}

// score key of candidate k from its 16 correctly rounded bf16 head scores:
// e_h = bf16(relu(s_h) * w_h), score = bf16(sum_h e_h) (pairwise fp64; the 16
// terms have 8 significant bits, so the sum is exact like the oracle's),
// key = orderable score << 16 | (0xFFFF - k), -0 treated as +0.
__device__ __forceinline__ uint32_t score_key(const uint32_t (&sb)[16], const float (&wf)[16],
                                              int k) {
  double e[16];
#pragma unroll
  for (int h = 0; h < 16; ++h) {
    const float sv = fmaxf(__uint_as_float(sb[h] << 16), 0.f);
    e[h] = static_cast<double>(__uint_as_float(f32_to_bf16_rne(__fmul_rn(sv, wf[h])) << 16));
  }
#pragma unroll
  for (int st = 1; st < 16; st <<= 1)
#pragma unroll
    for (int h = 0; h < 16; h += 2 * st) e[h] += e[h + st];
  uint32_t tb = round_f64_to_bf16(e[0]);
  if (tb == 0x8000u) tb = 0;
  const uint32_t ord = (tb & 0x8000u) ? (~tb & 0xFFFFu) : (tb | 0x8000u);
  return (ord << 16) | (0xFFFFu - static_cast<uint32_t>(k));
}

__device__ __forceinline__ void load_token_vectors(const float* qn, const float* wv, int tt,
                                                   float (&qv)[16], float (&wf)[16]) {
#pragma unroll
  for (int h4 = 0; h4 < 4; ++h4) {
    const float4 a = reinterpret_cast<const float4*>(qn + tt * 16)[h4];
    const float4 c = reinterpret_cast<const float4*>(wv + tt * 16)[h4];
    qv[4 * h4 + 0] = a.x; qv[4 * h4 + 1] = a.y; qv[4 * h4 + 2] = a.z; qv[4 * h4 + 3] = a.w;
    wf[4 * h4 + 0] = c.x; wf[4 * h4 + 1] = c.y; wf[4 * h4 + 2] = c.z; wf[4 * h4 + 3] = c.w;
  }
}

// Exact dot product of q row `qrow` and kv row `krow` (both SW128 in smem):
// exact fp64 products summed in ascending dimension order (the oracle's
// order), rounded once to bf16.
__device__ __noinline__ uint32_t exact_dot_seq(const uint8_t* qbase, int qrow,
                                               const uint8_t* kvbase, int krow) {
  double acc = 0.0;
#pragma unroll
  for (int ch = 0; ch < 8; ++ch) {
    const uint4 a = *reinterpret_cast<const uint4*>(qbase + sw128_off(qrow, ch));
    const uint4 b = *reinterpret_cast<const uint4*>(kvbase + sw128_off(krow, ch));
    const uint32_t aw[4] = {a.x, a.y, a.z, a.w};
    const uint32_t bw[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      acc = fma(static_cast<double>(bf16lo_to_f32(aw[e])), static_cast<double>(bf16lo_to_f32(bw[e])),
                acc);
      acc = fma(static_cast<double>(bf16hi_to_f32(aw[e])), static_cast<double>(bf16hi_to_f32(bw[e])),
                acc);
    }
  }
  return round_f64_to_bf16(acc);
}

// The same bf16 value without fp64 conversions: the products of two bf16 are
// exact in fp32 (up to underflow, below 2^-144 in total), and TwoSum chains
// (Knuth; two of them, one per f32x2 lane) carry them as an unevaluated sum
// s + c within 2^-30 sum|p| of the exact dot (compensated summation, Ogita,
// Rump and Oishi 2005, with a wide margin); the oracle's sequential fp64 sum is
// within 64 2^-53 sum|p| of it. sum|p| <= ||q|| ||kv|| <= bound / kGamma, so
// the value is decided when the bf16 rounding agrees at both ends of
// s + c -+ bound 2^-10; otherwise the sequential fp64 sum decides.
// `bound` >= kGamma ||q|| ||kv||.
__device__ __forceinline__ uint32_t exact_dot_bits(const uint8_t* qbase, int qrow,
                                                   const uint8_t* kvbase, int krow, float bound) {
  uint64_t s2 = f2_pack(0.f, 0.f), c2 = f2_pack(0.f, 0.f);
#pragma unroll 2
  for (int ch = 0; ch < 8; ++ch) {
    const uint4 a = *reinterpret_cast<const uint4*>(qbase + sw128_off(qrow, ch));
    const uint4 b = *reinterpret_cast<const uint4*>(kvbase + sw128_off(krow, ch));
    const uint32_t aw[4] = {a.x, a.y, a.z, a.w};
    const uint32_t bw[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const uint64_t p2 = f2_pack(mul_bf16lo(aw[e], bw[e]), mul_bf16hi(aw[e], bw[e]));
      const uint64_t t2 = f2_add(s2, p2);
      const uint64_t bp2 = f2_sub(t2, s2);
      const uint64_t e2 = f2_add(f2_sub(s2, f2_sub(t2, bp2)), f2_sub(p2, bp2));
      s2 = t2;
      c2 = f2_add(c2, e2);
    }
  }
  float s0, s1, c0, c1;
  f2_unpack(s2, s0, s1);
  f2_unpack(c2, c0, c1);
  const float t = __fadd_rn(s0, s1);
  const float bp = __fsub_rn(t, s0);
  const float c = __fadd_rn(__fadd_rn(c0, c1), __fadd_rn(__fsub_rn(s0, __fsub_rn(t, bp)),
                                                        __fsub_rn(s1, bp)));
  const float d = __fmaf_ru(bound, 0x1p-10f, 0x1p-140f);
  if (isfinite(t) && isfinite(c) && isfinite(d)) {
    const float lo = __fadd_rd(t, __fsub_rd(c, d)), hi = __fadd_ru(t, __fadd_ru(c, d));
    const uint32_t blo = f32_to_bf16_rne(lo);
    if (blo == f32_to_bf16_rne(hi)) return blo;
  }
  return exact_dot_seq(qbase, qrow, kvbase, krow);
}

// score_key over a queue entry's head scores (the low halves of words 1..16).
__device__ __noinline__ uint32_t score_key_slow(const uint32_t* e, const float* wv, int k) {
  uint32_t sb[16];
#pragma unroll
  for (int h = 0; h < 16; ++h) sb[h] = e[1 + h] & 0xFFFFu;
  float wf[16];
#pragma unroll
  for (int h = 0; h < 16; ++h) wf[h] = wv[h];
  return score_key(sb, wf, k);
}

// Score key of a drained pair from its 16 exact head scores (the low halves of
// words 1..16 of the entry): e_h = bf16(relu(s_h) * w_h) two heads at a time
// (bf16x2, RNE), their sum in fp32 rounded down and up; when both round to the
// same bf16 that is the exact sum's rounding, otherwise the fp64 chain
// (score_key) decides. wpk: per head {w, w} as bf16x2, wv: per head w.
__device__ __forceinline__ uint32_t drained_key(const uint32_t* e, const uint32_t* wpk,
                                                const float* wv, int k) {
  float lo[2] = {0.f, 0.f}, hi[2] = {0.f, 0.f};
#pragma unroll
  for (int hp = 0; hp < 8; ++hp) {
    uint32_t x = __byte_perm(e[1 + 2 * hp], e[2 + 2 * hp], 0x5410u);
    const uint32_t w2 = __byte_perm(wpk[2 * hp], wpk[2 * hp + 1], 0x5410u);
    asm("max.bf16x2 %0, %1, %2;" : "=r"(x) : "r"(x), "r"(0u));
    asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(x) : "r"(x), "r"(w2));
    lo[hp & 1] = add_rd_bf16hi(x, add_rd_bf16lo(x, lo[hp & 1]));
    hi[hp & 1] = add_ru_bf16hi(x, add_ru_bf16lo(x, hi[hp & 1]));
  }
  const float ls = __fadd_rd(lo[0], lo[1]), hs = __fadd_ru(hi[0], hi[1]);
  if (isfinite(ls) && isfinite(hs)) {
    uint32_t tp;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(tp) : "f"(hs), "f"(ls));
    uint32_t tlo = tp & 0xFFFFu, thi = tp >> 16;
    if (tlo == 0x8000u) tlo = 0;  // -0 == +0
    if (thi == 0x8000u) thi = 0;
    if (tlo == thi) {
      const uint32_t ord = (tlo & 0x8000u) ? (~tlo & 0xFFFFu) : (tlo | 0x8000u);
      return (ord << 16) | (0xFFFFu - static_cast<uint32_t>(k));
    }
  }
  return score_key_slow(e, wv, k);
}

// Per-warp queue of (token, candidate) pairs of the last one or two chunks
// whose score could not be certified. Entry: word 0 = kv stage << 28 | token
// slot << 16 | candidate k, words 1..16 = per head the bf16 pair
// {relu(RNE(v+E)), relu(RNE(v-E))} of the interval that holds the head's exact
// bf16 score after the relu (a negative score is 0 either way), word 17 =
// the kv row's norm bound times kGamma (19 words: an odd stride keeps the
// lanes' reads of one word on distinct banks).
constexpr int kRqWords = 19;

__device__ __forceinline__ bool bf16_positive(uint32_t h16) {
  return h16 != 0u && !(h16 & 0x8000u);
}

// bf16 bits of a score from its orderable image.
__device__ __forceinline__ uint32_t ord_to_bf16(uint32_t ord) {
  return (ord & 0x8000u) ? (ord & 0x7FFFu) : (~ord & 0xFFFFu);
}

// Queued pairs, 32 at a time: exact recomputation of the heads whose interval
// is open and can be positive (spread one per lane), then the exact score
// chain, one lane per pair; writes the orderable score (or, with gs, the bf16
// score to gs[token slot * gld + k]).
__device__ __noinline__ void drain_queue(uint32_t* rq, int n, const uint8_t* qs, const float* qn,
                                         const uint8_t* kv_stages, const float* wv,
                                         const uint32_t* wpk, uint16_t* keys, uint16_t* gs,
                                         int64_t gld, int lane) {
  __syncwarp();
  for (int i0 = 0; i0 < n; i0 += 32) {
    const int i = i0 + lane;
    uint32_t* e = rq + i * kRqWords;
    uint32_t open = 0;  // heads whose interval is open and can be positive
    if (i < n) {
#pragma unroll
      for (int h = 0; h < 16; ++h) {
        const uint32_t pr = e[1 + h];
        const uint32_t lo16 = pr & 0xFFFFu, hi16 = pr >> 16;
        if (lo16 != hi16 && bf16_positive(hi16)) open |= 1u << h;
      }
    }
    // the (entry, head) recomputations of these 32 entries are spread over the
    // lanes, one per lane and round; the exact value replaces the interval
    const int cnt = __popc(open);
    int incl = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xFFFFFFFFu, incl, o);
      if (lane >= o) incl += v;
    }
    const int total = __shfl_sync(0xFFFFFFFFu, incl, 31);
#pragma unroll 1
    for (int j0 = 0; j0 < total; j0 += 32) {
      const int j = j0 + lane;
      // owner: the first lane whose inclusive count exceeds j
      int own = 0;
#pragma unroll
      for (int step = 16; step > 0; step >>= 1) {
        const int v = __shfl_sync(0xFFFFFFFFu, incl, own + step - 1);
        if (v <= j) own += step;
      }
      const int excl = __shfl_sync(0xFFFFFFFFu, incl - cnt, own);
      const uint32_t om = __shfl_sync(0xFFFFFFFFu, open, own);
      if (j < total) {
        const int h = static_cast<int>(__fns(om, 0u, j - excl + 1));
        uint32_t* eo = rq + (i0 + own) * kRqWords;
        const uint32_t w0 = eo[0];
        const int tt = static_cast<int>((w0 >> 16) & 0xFFFu);
        const int row = static_cast<int>(w0 & 0xFFFFu) & (kChunk - 1);
        eo[1 + h] = exact_dot_bits(qs, tt * 16 + h, kv_stages + (w0 >> 28) * kKVBytes, row,
                                   qn[tt * 16 + h] * __uint_as_float(eo[17]));
      }
    }
    __syncwarp();
    if (i < n) {
      // head scores now certified, exact, or relu'd to 0
      const int tt = static_cast<int>((e[0] >> 16) & 0xFFFu);
      const int k = static_cast<int>(e[0] & 0xFFFFu);
      const uint32_t key = drained_key(e, wpk + tt * 16, wv + tt * 16, k);
      if (gs)
        gs[tt * gld + k] = static_cast<uint16_t>(ord_to_bf16(key >> 16));
      else
        keys[tt * kMaxT + k] = static_cast<uint16_t>(key >> 16);
    }
  }
  __syncwarp();
}

// Descending bitonic sorts of two tokens' 32*R keys, held as v[r] (u[r]) =
// element r*32 + lane, interleaved (independent chains hide each other's
// shuffle latency).
template <int R>
__device__ __forceinline__ void warp_bitonic_desc2(uint32_t (&v)[R], uint32_t (&u)[R], int lane) {
#pragma unroll
  for (int size = 2; size <= 32 * R; size <<= 1) {
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      if (stride >= 32) {
        const int rs = stride >> 5;
#pragma unroll
        for (int r = 0; r < R; ++r) {
          if ((r & rs) == 0) {
            const int i = r * 32 + lane;
            const bool desc_block = (i & size) == 0;
            const uint32_t a = v[r], b = v[r | rs], c = u[r], d = u[r | rs];
            if (desc_block ? (a < b) : (a > b)) {
              v[r] = b;
              v[r | rs] = a;
            }
            if (desc_block ? (c < d) : (c > d)) {
              u[r] = d;
              u[r | rs] = c;
            }
          }
        }
      } else {
#pragma unroll
        for (int r = 0; r < R; ++r) {
          const int i = r * 32 + lane;
          const uint32_t o = __shfl_xor_sync(0xFFFFFFFFu, v[r], stride);
          const uint32_t q = __shfl_xor_sync(0xFFFFFFFFu, u[r], stride);
          const bool keep_max = (((i & stride) == 0) == ((i & size) == 0));
          v[r] = keep_max ? max(v[r], o) : min(v[r], o);
          u[r] = keep_max ? max(u[r], q) : min(u[r], q);
        }
      }
    }
  }
}

template <int R>
__device__ __forceinline__ void sort_and_store2(const uint32_t* sel0, int nsel0, int64_t* out0,
                                                const uint32_t* sel1, int nsel1, int64_t* out1,
                                                int K_out, int64_t offset, int lane) {
  uint32_t v[R], u[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int i = r * 32 + lane;
    v[r] = i < nsel0 ? sel0[i] : 0u;
    u[r] = i < nsel1 ? sel1[i] : 0u;
  }
  warp_bitonic_desc2<R>(v, u, lane);
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int i = r * 32 + lane;
    if (i < K_out) {
      out0[i] = i < nsel0 ? static_cast<int64_t>(0xFFFFu - (v[r] & 0xFFFFu)) + offset
                          : static_cast<int64_t>(-1);
      if (out1)
        out1[i] = i < nsel1 ? static_cast<int64_t>(0xFFFFu - (u[r] & 0xFFFFu)) + offset
                            : static_cast<int64_t>(-1);
    }
  }
}

// Top-Ksel of the n orderable scores in `keys` (smem, in candidate order) by one warp, for
// two tokens at once (their steps interleaved; the second may be absent:
// n1 = 0, out1 = nullptr). A key is (orderable score << 16) | (0xFFFF - k), so
// the order is score descending, then k ascending. The keys are held in
// registers (key r*32+lane in v[r]); a binary search over the 16 score bits
// finds the largest score thr with at least Ksel keys scoring >= thr, and keys
// scoring exactly thr are taken in k order (the order they are stored in) up
// to Ksel. The selected keys are then compacted and sorted.
template <int R>
__device__ __forceinline__ void warp_topk2_r(const uint16_t* keys0, int n0, const uint16_t* keys1,
                                             int n1, int K_out, uint32_t* sel0, uint32_t* sel1,
                                             int64_t* out0, int64_t* out1, int64_t offset,
                                             int lane) {
  const int ksel0 = n0 < K_out ? n0 : K_out, ksel1 = n1 < K_out ? n1 : K_out;
  const uint32_t lt_mask = (1u << lane) - 1u;
  uint32_t v[R], u[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int i = r * 32 + lane;
    // key = orderable score << 16 | (0xFFFF - k); a real key scores >= 1, padding 0
    v[r] = i < n0 ? (static_cast<uint32_t>(keys0[i]) << 16) | (0xFFFFu - i) : 0u;
    u[r] = i < n1 ? (static_cast<uint32_t>(keys1[i]) << 16) | (0xFFFFu - i) : 0u;
  }
  const bool all0 = n0 <= ksel0, all1 = n1 <= ksel1;
  uint32_t thr0 = 0, thr1 = 0;
  int need0 = 0, need1 = 0;
  if (!(all0 && all1)) {
    for (int bit = 15; bit >= 0; --bit) {
      const uint32_t cand0 = (thr0 | (1u << bit)) << 16, cand1 = (thr1 | (1u << bit)) << 16;
      int c0 = 0, c1 = 0;
#pragma unroll
      for (int r = 0; r < R; ++r) {
        c0 += v[r] >= cand0 ? 1 : 0;
        c1 += u[r] >= cand1 ? 1 : 0;
      }
      c0 = static_cast<int>(__reduce_add_sync(0xFFFFFFFFu, static_cast<unsigned>(c0)));
      c1 = static_cast<int>(__reduce_add_sync(0xFFFFFFFFu, static_cast<unsigned>(c1)));
      if (c0 >= ksel0) thr0 |= 1u << bit;
      if (c1 >= ksel1) thr1 |= 1u << bit;
    }
    const uint32_t above0 = (thr0 + 1) << 16, above1 = (thr1 + 1) << 16;
    int c0 = 0, c1 = 0;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      c0 += v[r] >= above0 ? 1 : 0;
      c1 += u[r] >= above1 ? 1 : 0;
    }
    need0 = ksel0 - static_cast<int>(__reduce_add_sync(0xFFFFFFFFu, static_cast<unsigned>(c0)));
    need1 = ksel1 - static_cast<int>(__reduce_add_sync(0xFFFFFFFFu, static_cast<unsigned>(c1)));
  }
  int base0 = 0, ties0 = 0, base1 = 0, ties1 = 0;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const bool valid0 = r * 32 + lane < n0, valid1 = r * 32 + lane < n1;
    const uint32_t sc0 = v[r] >> 16, sc1 = u[r] >> 16;
    const bool tie0 = !all0 && valid0 && sc0 == thr0, tie1 = !all1 && valid1 && sc1 == thr1;
    const uint32_t tb0 = __ballot_sync(0xFFFFFFFFu, tie0), tb1 = __ballot_sync(0xFFFFFFFFu, tie1);
    const bool take0 =
        valid0 && (all0 || sc0 > thr0 || (tie0 && ties0 + __popc(tb0 & lt_mask) < need0));
    const bool take1 =
        valid1 && (all1 || sc1 > thr1 || (tie1 && ties1 + __popc(tb1 & lt_mask) < need1));
    ties0 += __popc(tb0);
    ties1 += __popc(tb1);
    const uint32_t b0 = __ballot_sync(0xFFFFFFFFu, take0), b1 = __ballot_sync(0xFFFFFFFFu, take1);
    if (take0) sel0[base0 + __popc(b0 & lt_mask)] = v[r];
    if (take1) sel1[base1 + __popc(b1 & lt_mask)] = u[r];
    base0 += __popc(b0);
    base1 += __popc(b1);
  }
  __syncwarp();
  if (K_out <= 128)
    sort_and_store2<4>(sel0, base0, out0, sel1, base1, out1, K_out, offset, lane);
  else
    sort_and_store2<8>(sel0, base0, out0, sel1, base1, out1, K_out, offset, lane);
  __syncwarp();
}

// One token's top-Ksel, the same steps as warp_topk2_r for a single list (used
// for lists longer than 512, where two lists' keys would not fit the selection
// warps' registers).
template <int R>
__device__ __forceinline__ void warp_bitonic_desc1(uint32_t (&v)[R], int lane) {
#pragma unroll
  for (int size = 2; size <= 32 * R; size <<= 1) {
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      if (stride >= 32) {
        const int rs = stride >> 5;
#pragma unroll
        for (int r = 0; r < R; ++r) {
          if ((r & rs) == 0) {
            const bool desc_block = ((r * 32 + lane) & size) == 0;
            const uint32_t a = v[r], b = v[r | rs];
            if (desc_block ? (a < b) : (a > b)) {
              v[r] = b;
              v[r | rs] = a;
            }
          }
        }
      } else {
#pragma unroll
        for (int r = 0; r < R; ++r) {
          const int i = r * 32 + lane;
          const uint32_t o = __shfl_xor_sync(0xFFFFFFFFu, v[r], stride);
          const bool keep_max = (((i & stride) == 0) == ((i & size) == 0));
          v[r] = keep_max ? max(v[r], o) : min(v[r], o);
        }
      }
    }
  }
}

template <int R>
__device__ __forceinline__ void sort_and_store1(const uint32_t* sel, int nsel, int64_t* out,
                                                int K_out, int64_t offset, int lane) {
  uint32_t v[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int i = r * 32 + lane;
    v[r] = i < nsel ? sel[i] : 0u;
  }
  warp_bitonic_desc1<R>(v, lane);
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int i = r * 32 + lane;
    if (i < K_out)
      out[i] = i < nsel ? static_cast<int64_t>(0xFFFFu - (v[r] & 0xFFFFu)) + offset
                        : static_cast<int64_t>(-1);
  }
}

template <int R>
__device__ __forceinline__ void warp_topk1_r(const uint16_t* keys, int n, int K_out,
                                             uint32_t* sel, int64_t* out, int64_t offset,
                                             int lane) {
  const int ksel = n < K_out ? n : K_out;
  const uint32_t lt_mask = (1u << lane) - 1u;
  uint32_t v[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int i = r * 32 + lane;
    v[r] = i < n ? (static_cast<uint32_t>(keys[i]) << 16) | (0xFFFFu - i) : 0u;
  }
  const bool all = n <= ksel;
  uint32_t thr = 0;
  int need = 0;
  if (!all) {
    for (int bit = 15; bit >= 0; --bit) {
      const uint32_t cand = (thr | (1u << bit)) << 16;
      int c = 0;
#pragma unroll
      for (int r = 0; r < R; ++r) c += v[r] >= cand ? 1 : 0;
      c = static_cast<int>(__reduce_add_sync(0xFFFFFFFFu, static_cast<unsigned>(c)));
      if (c >= ksel) thr |= 1u << bit;
    }
    const uint32_t above = (thr + 1) << 16;
    int c = 0;
#pragma unroll
    for (int r = 0; r < R; ++r) c += v[r] >= above ? 1 : 0;
    need = ksel - static_cast<int>(__reduce_add_sync(0xFFFFFFFFu, static_cast<unsigned>(c)));
  }
  int base = 0, ties = 0;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const bool valid = r * 32 + lane < n;
    const uint32_t sc = v[r] >> 16;
    const bool tie = !all && valid && sc == thr;
    const uint32_t tb = __ballot_sync(0xFFFFFFFFu, tie);
    const bool take = valid && (all || sc > thr || (tie && ties + __popc(tb & lt_mask) < need));
    ties += __popc(tb);
    const uint32_t bm = __ballot_sync(0xFFFFFFFFu, take);
    if (take) sel[base + __popc(bm & lt_mask)] = v[r];
    base += __popc(bm);
  }
  __syncwarp();
  if (K_out <= 128)
    sort_and_store1<4>(sel, base, out, K_out, offset, lane);
  else
    sort_and_store1<8>(sel, base, out, K_out, offset, lane);
  __syncwarp();
}

__device__ void warp_topk2(const uint16_t* keys0, int n0, const uint16_t* keys1, int n1, int K_out,
                           uint32_t* sel0, uint32_t* sel1, int64_t* out0, int64_t* out1,
                           int64_t offset, int lane) {
  const int n = n0 > n1 ? n0 : n1;
  if (n <= 256) {
    warp_topk2_r<8>(keys0, n0, keys1, n1, K_out, sel0, sel1, out0, out1, offset, lane);
  } else if (n <= 512) {
    warp_topk2_r<16>(keys0, n0, keys1, n1, K_out, sel0, sel1, out0, out1, offset, lane);
  } else if (n <= 768) {
    warp_topk1_r<24>(keys0, n0, K_out, sel0, out0, offset, lane);
    if (out1) warp_topk1_r<24>(keys1, n1, K_out, sel0, out1, offset, lane);
  } else {
    warp_topk1_r<32>(keys0, n0, K_out, sel0, out0, offset, lane);
    if (out1) warp_topk1_r<32>(keys1, n1, K_out, sel0, out1, offset, lane);
  }
}

// Selection of token pair g of the CTA's sequence (unit lu = g / 8 of this
// CTA, tokens 2 (g % 8) and 2 (g % 8) + 1): waits until the unit's keys are
// written (every lane acquires them; immediate when they already are), selects
// both tokens, writes their indices and arrives on the key buffer's release
// barrier. Returns false past the CTA's last unit or when the wait gave up.
__device__ __forceinline__ bool select_pair(const Params& p, int g, const uint8_t* smem,
                                         uint64_t* keys_full, uint64_t* keys_empty,
                                         uint32_t* sel0, uint32_t* sel1, volatile int* abort_flag,
                                         int lane) {
  constexpr int kPairs = kTB / 2;
  const int lu = g / kPairs, pr = g % kPairs;
  const int u = blockIdx.x + lu * gridDim.x;
  if (u >= p.units) return false;
  const int b = u % p.B;
  const int64_t t0 = static_cast<int64_t>(p.n_tb - 1 - u / p.B) * kTB;
  const int kb = lu & 1;
  if (!__all_sync(0xFFFFFFFFu, mbar_wait(&keys_full[kb], (lu >> 1) & 1, abort_flag, p.err,
                                         DSA_DEVERR_IX_WAIT)))
    return false;
  const uint16_t* kbuf = reinterpret_cast<const uint16_t*>(smem + kOffKeys + kb * kKeyBufBytes);
  // the pair's two tokens, selected together (the second may lie past the end)
  const int tt = 2 * pr;
  const int64_t tok = t0 + tt;
  if (tok < p.S) {
    const bool two = tok + 1 < p.S;
    int64_t* out0 = p.out + (static_cast<int64_t>(b) * p.S + tok) * p.K;
    warp_topk2(kbuf + tt * kMaxT, static_cast<int>(n_valid(p, tok)), kbuf + (tt + 1) * kMaxT,
               two ? static_cast<int>(n_valid(p, tok + 1)) : 0, p.K, sel0, sel1, out0,
               two ? out0 + p.K : nullptr, p.offset, lane);
  }
  __syncwarp();
  if (lane == 0) mbar_arrive(&keys_empty[kb]);
  return true;
}

// Next pair of the CTA's selection sequence (one atomic per warp).
__device__ __forceinline__ int grab_pair(int* next, int lane) {
  int g = 0;
  if (lane == 0) g = atomicAdd(next, 1);
  return __shfl_sync(0xFFFFFFFFu, g, 0);
}

__global__ void __launch_bounds__(kThreads, 1)
    score_topk_kernel(const __grid_constant__ CUtensorMap tm_q,
                      const __grid_constant__ CUtensorMap tm_kv, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* q_full = bars;                       // [2]
  uint64_t* q_empty = bars + 2;                  // [2], 2 arrivals (one per warpgroup)
  uint64_t* kv_full = bars + 4;                  // [3]
  uint64_t* kv_empty = kv_full + kKVStages;      // [3], 2 arrivals
  uint64_t* acc_full = kv_empty + kKVStages;     // [2]
  uint64_t* acc_empty = acc_full + 2;            // [2], 256 arrivals
  uint64_t* keys_full = acc_empty + 2;           // [2], 256 arrivals (epilogue threads)
  uint64_t* keys_empty = keys_full + 2;          // [2], 8 arrivals (one per token pair)
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kOffMisc + 4);
  int* sel_next = reinterpret_cast<int*>(smem + kOffMisc + 8);  // next token pair to select
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 256);
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 256);
    }
    for (int i = 0; i < kKVStages; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 256);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&keys_full[i], 256);
      mbar_init(&keys_empty[i], kTB / 2);
    }
    *abort_flag = 0;
    *sel_next = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_kv);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  // unit u -> (b, token block), heaviest (latest) token blocks first
  auto unit_of = [&](int u, int& b, int64_t& t0) {
    b = u % p.B;
    t0 = static_cast<int64_t>(p.n_tb - 1 - u / p.B) * kTB;
  };
  auto unit_chunks = [&](int64_t t0) -> int {
    int64_t tl = t0 + kTB - 1;
    if (tl > p.S - 1) tl = p.S - 1;
    const int64_t nv = n_valid(p, tl);
    return static_cast<int>((nv + kChunk - 1) / kChunk);
  };

  // Roles by warpgroup, each region under its own register limit (setmaxnreg
  // is warpgroup-wide; see kLaunchRegs): warpgroups 1 and 2 are the epilogue,
  // warpgroups 0 and 3 the producers and the selection warps.
  if ((warp >> 2) == 1 || (warp >> 2) == 2) {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;\n" ::"n"(kEpiRegs));
    // ------------------------------------------------------------ epilogue
    const int wg = (warp - kEpiWarp0) >> 2;  // tokens [8 wg, 8 wg + 8) of the unit
    const int t_in = threadIdx.x - 32 * kEpiWarp0 - 128 * wg;  // 0..127
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;     // kv row of the chunk = TMEM lane
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const int ew = warp - kEpiWarp0;         // 0..7
    float* qn = reinterpret_cast<float*>(smem + kOffQN);
    float* wv = reinterpret_cast<float*>(smem + kOffW);
    // this warp's queue of pairs that need an exact recomputation; empty
    // between units, when it serves as selection scratch
    uint32_t* rq = reinterpret_cast<uint32_t*>(smem + kOffRq + ew * kRqBytes);
    bool ok = true;
    int lu = 0, gc = 0;
    for (int u = blockIdx.x; u < p.units; u += gridDim.x, ++lu) {
      int b;
      int64_t t0;
      unit_of(u, b, t0);
      const int nch = unit_chunks(t0);
      const int qb = lu & 1;
      const int kb = lu & 1;
      uint16_t* keys = reinterpret_cast<uint16_t*>(smem + kOffKeys + kb * kKeyBufBytes);
      const uint8_t* qs = smem + kOffQ + qb * kQBytes;
      uint16_t* gs = p.scores ? p.scores + (static_cast<int64_t>(b) * p.S + t0) * p.score_ld
                              : nullptr;
      // (t,h) row of this thread for norms / weights: token 8wg + t_in/16, head t_in%16
      const int qrow = wg * 128 + t_in;
      int* nvs = reinterpret_cast<int*>(smem + kOffNV);
      if (t_in < 8) {
        const int64_t tok = t0 + wg * 8 + t_in;
        nvs[wg * 8 + t_in] = tok < p.S ? static_cast<int>(n_valid(p, tok)) : 0;
      }
      {
        const int64_t tok = t0 + (qrow >> 4);
        uint32_t wb = 0;
        if (tok < p.S) wb = p.w[(static_cast<int64_t>(b) * p.S + tok) * kHeads + (qrow & 15)];
        wv[qrow] = bf16lo_to_f32(wb);
        reinterpret_cast<uint32_t*>(smem + kOffWP)[qrow] = wb | (wb << 16);
        // an interval times a negative weight swaps its ends
        reinterpret_cast<uint32_t*>(smem + kOffPS)[qrow] = (wb & 0x8000u) ? 0x1032u : 0x3210u;
      }
      ok = __all_sync(0xFFFFFFFFu, mbar_wait(&q_full[qb], (lu >> 1) & 1, abort_flag, p.err,
                                             DSA_DEVERR_IX_WAIT));
      if (ok) qn[qrow] = row_norm64(qs, qrow);
      // the key buffer of this unit is free once the selection of unit lu - 2 is done
      if (ok && gs == nullptr)
        ok = __all_sync(0xFFFFFFFFu, mbar_wait(&keys_empty[kb], ((lu >> 1) & 1) ^ 1, abort_flag,
                                               p.err, DSA_DEVERR_IX_WAIT));
      ok = named_bar_and(1 + wg, 128, ok);
      constexpr int kRqCap = kRqBytes / 4 / kRqWords;
      const uint8_t* kv_stages = smem + kOffKV;
      // queued pairs are drained every second chunk (or when the queue would
      // overflow, or at the unit's end); a thread releases a kv stage only after
      // the pairs that read it are drained
      int rq_n = 0;
      int held = -1;  // stage of the previous chunk, not yet released
      for (int c = 0; ok && c < nch; ++c, ++gc) {
        const int s = gc % kKVStages;
        const int ab = gc & 1;
        const uint8_t* kvs = smem + kOffKV + s * kKVBytes;
        const int k = c * kChunk + row;
        ok = __all_sync(0xFFFFFFFFu, mbar_wait(&kv_full[s], (gc / kKVStages) & 1, abort_flag,
                                               p.err, DSA_DEVERR_IX_WAIT));
        if (ok)
          ok = __all_sync(0xFFFFFFFFu, mbar_wait(&acc_full[ab], (gc >> 1) & 1, abort_flag, p.err,
                                                 DSA_DEVERR_IX_WAIT));
        if (ok) {
          tc_fence_after();
          const float kvn = row_norm64(kvs, row) * kGamma;
          const uint64_t kv2 = f2_pack(kvn, kvn), nkv2 = f2_pack(-kvn, -kvn);
          const uint32_t* wpk = reinterpret_cast<const uint32_t*>(smem + kOffWP);
          const uint32_t* psel = reinterpret_cast<const uint32_t*>(smem + kOffPS);
#pragma unroll 1
          for (int tl = 0; tl < 8; tl += 2) {
            // two tokens per TMEM load: 32 columns = 2 tokens x 16 heads
            const int tt0 = wg * 8 + tl;
            // nothing to do when all 32 rows of this warp lie past both tokens'
            // valid candidates (the unit's last chunk under the causal mask)
            if (c * kChunk + quarter * 32 >= max(nvs[tt0], nvs[tt0 + 1])) continue;
            uint32_t r[32];
            tmem_ld_32x32b_x32(tmem + lane_off + static_cast<uint32_t>(ab * 256 + tt0 * 16), r);
            // both tokens' interval chains first (one basic block, so their
            // instructions interleave), then their queue entries and keys
            uint32_t prs[2][16];
            uint32_t tlo[2], thi[2];
#pragma unroll
            for (int j = 0; j < 2; ++j) {
              const int tt = tt0 + j;
              // Each head score s_h is known to lie in [v - E, v + E] (E = q_h's
              // norm bound times kvn); carry the interval [RNE(v-E), RNE(v+E)]
              // through relu, *w (bf16 RNE, both monotone) and the head sum
              // (fp32, rounded outward). If both ends of the sum round to the
              // same bf16, that is the exact score. The ends v +- E come from
              // one directed-rounding fma per two heads.
              float slo[4] = {0.f, 0.f, 0.f, 0.f}, shi[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
              for (int h4 = 0; h4 < 4; ++h4) {
                const float4 qv4 = reinterpret_cast<const float4*>(qn + tt * 16)[h4];
                const uint4 wp4 = reinterpret_cast<const uint4*>(wpk + tt * 16)[h4];
                const uint4 ps4 = reinterpret_cast<const uint4*>(psel + tt * 16)[h4];
                const uint64_t qq[2] = {f2_pack(qv4.x, qv4.y), f2_pack(qv4.z, qv4.w)};
                const uint32_t wpa[4] = {wp4.x, wp4.y, wp4.z, wp4.w};
                const uint32_t psa[4] = {ps4.x, ps4.y, ps4.z, ps4.w};
#pragma unroll
                for (int hp = 0; hp < 2; ++hp) {
                  const int h = h4 * 4 + hp * 2;
                  const uint64_t v2 = f2_pack(__uint_as_float(r[j * 16 + h]),
                                              __uint_as_float(r[j * 16 + h + 1]));
                  float hv[2], lv[2];
                  f2_unpack(f2_fma_rp(qq[hp], kv2, v2), hv[0], hv[1]);
                  f2_unpack(f2_fma_rm(qq[hp], nkv2, v2), lv[0], lv[1]);
#pragma unroll
                  for (int m = 0; m < 2; ++m) {
                    const int i = hp * 2 + m;
                    // upper half relu(RNE(v+E)), lower half relu(RNE(v-E)): the
                    // relu rides on the conversion (RNE is monotone and keeps signs)
                    uint32_t pr;
                    asm("cvt.rn.relu.bf16x2.f32 %0, %1, %2;" : "=r"(pr) : "f"(hv[m]), "f"(lv[m]));
                    prs[j][h + m] = pr;
                    uint32_t e2 = __byte_perm(pr, 0, psa[i]);
                    asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(e2) : "r"(e2), "r"(wpa[i]));
                    slo[i] = add_rd_bf16lo(e2, slo[i]);
                    shi[i] = add_ru_bf16hi(e2, shi[i]);
                  }
                }
              }
              const float lo_sum = __fadd_rd(__fadd_rd(slo[0], slo[1]), __fadd_rd(slo[2], slo[3]));
              const float hi_sum = __fadd_ru(__fadd_ru(shi[0], shi[1]), __fadd_ru(shi[2], shi[3]));
              uint32_t tp;
              asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(tp) : "f"(hi_sum), "f"(lo_sum));
              tlo[j] = tp & 0xFFFFu;
              thi[j] = tp >> 16;
              if (tlo[j] == 0x8000u) tlo[j] = 0;  // -0 == +0
              if (thi[j] == 0x8000u) thi[j] = 0;
            }
#pragma unroll
            for (int j = 0; j < 2; ++j) {
              const int tt = tt0 + j;
              const bool active = k < nvs[tt];
              // a NaN head score (relu keeps it NaN here) goes the exact way, where
              // the relu maps it to 0 like the oracle's
              const bool need = active && (tlo[j] != thi[j] || (tlo[j] & 0x7FFFu) > 0x7F80u);
              const uint32_t bal = __ballot_sync(0xFFFFFFFFu, need);
              if (bal) {
                if (rq_n + __popc(bal) > kRqCap) {
                  drain_queue(rq, rq_n, qs, qn, kv_stages, wv, wpk, keys, gs, p.score_ld, lane);
                  rq_n = 0;
                }
                if (need) {
                  uint32_t* e = rq + (rq_n + __popc(bal & ((1u << lane) - 1u))) * kRqWords;
                  e[0] = (static_cast<uint32_t>(s) << 28) | (static_cast<uint32_t>(tt) << 16) |
                         static_cast<uint32_t>(k);
#pragma unroll
                  for (int h = 0; h < 16; ++h) e[1 + h] = prs[j][h];
                  e[17] = __float_as_uint(kvn);
                }
                rq_n += __popc(bal);
              }
              if (active && !need) {
                if (gs) {
                  gs[tt * p.score_ld + k] = static_cast<uint16_t>(tlo[j]);
                } else {
                  const uint32_t ord = (tlo[j] & 0x8000u) ? (~tlo[j] & 0xFFFFu) : (tlo[j] | 0x8000u);
                  keys[tt * kMaxT + k] = static_cast<uint16_t>(ord);
                }
              }
            }
          }
          tc_fence_before();
          mbar_arrive(&acc_empty[ab]);
          if ((c & 1) || c == nch - 1) {
            if (rq_n > 0) drain_queue(rq, rq_n, qs, qn, kv_stages, wv, wpk, keys, gs, p.score_ld, lane);
            rq_n = 0;
          }
        }
        // every epilogue thread releases its stages itself, so a warp busy with
        // exact recomputations holds up no other warp
        if (ok) {
          if (rq_n == 0) {
            if (held >= 0) mbar_arrive(&kv_empty[held]);
            mbar_arrive(&kv_empty[s]);
            held = -1;
          } else {
            held = s;  // pairs of this chunk wait for the next drain
          }
        }
      }
      // the warpgroup leaves the unit together: its per-token arrays are rewritten next
      ok = named_bar_and(1 + wg, 128, ok);
      if (!ok) break;
      mbar_arrive(&q_empty[qb]);
      // this thread's keys of the unit are written (with gs the scores went to
      // global memory and the top-k runs in its own kernel)
      if (gs == nullptr) mbar_arrive(&keys_full[kb]);
    }
    // after the last unit: help select the pairs still pending
    if (ok && p.scores == nullptr) {
      while (select_pair(p, grab_pair(sel_next, lane), smem, keys_full, keys_empty, rq, rq + kMaxK,
                         abort_flag, lane)) {
      }
    }
    } else {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;\n" ::"n"(kOtherRegs));
    if (warp == 0) {
      if (lane == 0) {
        int lu = 0, gc = 0;
        bool ok = true;
        for (int u = blockIdx.x; ok && u < p.units; u += gridDim.x, ++lu) {
          int b;
          int64_t t0;
          unit_of(u, b, t0);
          const int nch = unit_chunks(t0);
          const int qb = lu & 1;
          if (!mbar_wait(&q_empty[qb], ((lu >> 1) & 1) ^ 1, abort_flag, p.err, DSA_DEVERR_IX_WAIT))
            break;
          mbar_arrive_expect_tx(&q_full[qb], kQBytes);
          tma_load_2d(smem + kOffQ + qb * kQBytes, &tm_q, 0,
                      static_cast<int32_t>((static_cast<int64_t>(b) * p.S + t0) * kHeads), &q_full[qb]);
          for (int c = 0; c < nch; ++c, ++gc) {
            const int s = gc % kKVStages;
            if (!mbar_wait(&kv_empty[s], ((gc / kKVStages) & 1) ^ 1, abort_flag, p.err,
                           DSA_DEVERR_IX_WAIT)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&kv_full[s], kKVBytes);
            tma_load_2d(smem + kOffKV + s * kKVBytes, &tm_kv, 0,
                        static_cast<int32_t>(b * p.kv_rows_per_batch + c * kChunk), &kv_full[s]);
          }
        }
        if (lu > 0) mbar_drain(&q_full[(lu - 1) & 1], ((lu - 1) >> 1) & 1);
        if (lu > 1) mbar_drain(&q_full[(lu - 2) & 1], ((lu - 2) >> 1) & 1);
        for (int i = (gc > kKVStages ? gc - kKVStages : 0); i < gc; ++i)
          mbar_drain(&kv_full[i % kKVStages], (i / kKVStages) & 1);
      }
    } else if (warp == 1) {
      if (lane == 0) {
        constexpr uint32_t idesc = make_idesc_bf16_f32(128, kQRows, 0, 0);
        int lu = 0, gc = 0;
        bool ok = true;
        for (int u = blockIdx.x; ok && u < p.units; u += gridDim.x, ++lu) {
          int b;
          int64_t t0;
          unit_of(u, b, t0);
          const int nch = unit_chunks(t0);
          const int qb = lu & 1;
          // Every unit runs the full q-buffer handshake, even one without chunks.
          if (!mbar_wait(&q_full[qb], (lu >> 1) & 1, abort_flag, p.err, DSA_DEVERR_IX_WAIT)) break;
          const uint32_t qaddr = smem_u32(smem + kOffQ + qb * kQBytes);
          for (int c = 0; c < nch; ++c, ++gc) {
            const int s = gc % kKVStages;
            const int ab = gc & 1;
            if (!mbar_wait(&kv_full[s], (gc / kKVStages) & 1, abort_flag, p.err,
                           DSA_DEVERR_IX_WAIT) ||
                !mbar_wait(&acc_empty[ab], ((gc >> 1) & 1) ^ 1, abort_flag, p.err,
                           DSA_DEVERR_IX_WAIT)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t kvaddr = smem_u32(smem + kOffKV + s * kKVBytes);
  #pragma unroll
            for (int k4 = 0; k4 < kDim / 16; ++k4) {
              const uint64_t ad = make_smem_desc(kvaddr + k4 * 32, 16u, 1024u, kLayoutSW128);
              const uint64_t bd = make_smem_desc(qaddr + k4 * 32, 16u, 1024u, kLayoutSW128);
              umma_bf16(tmem + static_cast<uint32_t>(ab) * 256u, ad, bd, idesc, k4 > 0 ? 1u : 0u);
            }
            umma_commit(&acc_full[ab]);
          }
        }
        if (gc > 0) mbar_drain(&acc_full[(gc - 1) & 1], ((gc - 1) >> 1) & 1);
        if (gc > 1) mbar_drain(&acc_full[(gc - 2) & 1], ((gc - 2) >> 1) & 1);
      }
    } else {
      // ----------------------------------------------------------- selection
      // One unit behind the epilogue. The units' token pairs form one sequence
      // (unit lu holds pairs 8 lu .. 8 lu + 7), handed out by a shared counter
      // to these six warps and, once their last unit is done, to the epilogue
      // warps; per pair the taker writes the two tokens' indices and arrives on
      // the key buffer's release barrier (8 arrivals per unit).
      if (p.scores == nullptr) {
        const int sw = warp < kEpiWarp0 ? warp - 2 : warp - kEpiWarp0 - 6;  // 0..5
        uint32_t* sel0 = reinterpret_cast<uint32_t*>(smem + kOffSel + sw * kSelBytes);
        uint32_t* sel1 = sel0 + kMaxK;
        while (select_pair(p, grab_pair(sel_next, lane), smem, keys_full, keys_empty, sel0, sel1,
                           abort_flag, lane)) {
        }
      }
    }
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace ixs

int launch_score_topk(const void* q, const void* w, const void* kv, int64_t kv_bstride,
                      int64_t* out, void* scores, int64_t batch, int64_t seqlen, int64_t n_cand,
                      int topk, int64_t start_pos, int ratio, int64_t offset, cudaStream_t stream) {
  using namespace ixs;
  DeviceInfo di;
  int st = current_device_info(&di);
  if (st != DSA_OK) return st;
  if (di.max_smem_optin < kSmem) return DSA_ERR_UNSUPPORTED;
  unsigned int* err = nullptr;
  st = device_error_word(&err);
  if (st != DSA_OK) return st;
  CUtensorMap tm_q, tm_kv;
  {
    const uint64_t dims[2] = {kDim, static_cast<uint64_t>(batch * seqlen * kHeads)};
    const uint64_t strides[1] = {kDim * 2};
    const uint32_t box[2] = {kDim, kQRows};
    st = encode_tensor_map(&tm_q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, q, dims, strides, box,
                           CU_TENSOR_MAP_SWIZZLE_128B);
    if (st != DSA_OK) return st;
  }
  const int64_t rows_per_batch = kv_bstride / kDim;
  {
    const uint64_t rows = static_cast<uint64_t>((batch - 1) * rows_per_batch + n_cand);
    const uint64_t dims[2] = {kDim, rows};
    const uint64_t strides[1] = {kDim * 2};
    const uint32_t box[2] = {kDim, kChunk};
    st = encode_tensor_map(&tm_kv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, kv, dims, strides, box,
                           CU_TENSOR_MAP_SWIZZLE_128B);
    if (st != DSA_OK) return st;
  }
  Params p;
  p.B = static_cast<int>(batch);
  p.S = seqlen;
  p.T = n_cand;
  p.K = topk;
  p.ratio = ratio;
  p.causal = start_pos == 0 ? 1 : 0;
  p.offset = offset;
  p.n_tb = static_cast<int>((seqlen + kTB - 1) / kTB);
  p.units = p.n_tb * p.B;
  p.kv_rows_per_batch = rows_per_batch;
  p.w = static_cast<const uint16_t*>(w);
  p.out = out;
  p.scores = static_cast<uint16_t*>(scores);
  p.score_ld = n_cand;
  p.err = err;
  st = set_max_dynamic_smem(reinterpret_cast<const void*>(score_topk_kernel), kSmem);
  if (st != DSA_OK) return st;
  {
    // the setmaxnreg split assumes exactly kLaunchRegs per thread at launch; a
    // build with fewer would make the epilogue's increase wait forever
    static int regs = -1;
    if (regs < 0) {
      cudaFuncAttributes fa;
      st = cuda_status(cudaFuncGetAttributes(&fa, score_topk_kernel));
      if (st != DSA_OK) return st;
      regs = fa.numRegs;
    }
    if (regs != kLaunchRegs) return DSA_ERR_UNSUPPORTED;
  }
  const int grid = p.units < di.num_sms ? p.units : di.num_sms;
  score_topk_kernel<<<grid, kThreads, kSmem, stream>>>(tm_q, tm_kv, p);
  return cuda_status(cudaGetLastError());
}

}  // namespace dsa
