// Lightning Indexer, fp8 index path (ModelArgs.dtype = "fp8", scale_fmt =
// "ue8m0", declared at reference/task2_v0_ref.py:25-26 and unused by the
// reference's bf16 v0 path). The definition follows the published indexer of
// DeepSeek-V3.2-Exp (inference/model.py Indexer.forward; inference/kernel.py
// act_quant and fp8_index), restated for this operator's shapes (64-wide head
// rows, so one quantization block per row):
//
//   rotate   h   = bf16(FWHT64(x) * 2^-3)   (Walsh-Hadamard in fp32, butterfly
//                  strides 1, 2, 4, ..., 32 in that order), every 64-wide row of
//                  q [rows, 16, 64] and of kv_cache [b, T, 64]
//   quantize s   = 2^ceil(log2(fp32(max(amax(h), 1e-4) / 448)))   (ue8m0)
//            y   = e4m3(h / s)              (RNE; |h / s| <= 448 by construction)
//   score    score[t,k] = ks[k] * sum_h relu(fp32(q8[t,h] . k8[k])) * wq[t,h],
//            wq[t,h] = fp32(w[t,h]) * qs[t,h]; the head sum is an fp32 fma chain
//            in ascending h
//   select   causal mask and top-k exactly as the bf16 path: score descending,
//            ties by ascending k (-0 == +0), -1 in masked slots, k + offset.
//
// Kernels:
//   fp8_quant_rows_kernel  one thread per 64-wide row: 8 x 16-byte loads, the
//                          FWHT on 64 fp32 registers, the ue8m0 scale, e4m3
//                          conversion (cvt.rn.satfinite.e4m3x2.f32), 4 x 16-byte
//                          stores; optionally folds the row's scale into its
//                          weight (wq = w * s, exact: s is a power of two).
//   score_fp8_kernel       the bf16 score kernel's pipeline on fp8 operands:
//                          tcgen05.mma kind::f8f6f4 (E4M3 x E4M3 -> fp32 TMEM),
//                          D[128 kv rows x 256 (token, head)] per 128-row kv
//                          chunk (two K = 32 instructions), SWIZZLE_64B tiles by
//                          TMA; an fp32 epilogue (relu, fma chain, * ks) that
//                          stores orderable 32-bit keys in shared memory (two
//                          epilogue warpgroups); top-K per token in six
//                          selection warps (warp_select.cuh), joined between
//                          units by the eight epilogue warps.
#include "common.cuh"
#include "host_util.h"
#include "numerics.cuh"
#include "warp_select.cuh"

namespace dsa {
namespace ix8 {

constexpr int kDim = 64;

// -------------------------------------------------------------- quantization
struct QuantParams {
  const uint16_t* src;     // bf16 rows of 64
  int64_t rows;
  int64_t rows_per_group;  // rows of one batch (kv) or all rows (q)
  int64_t group_stride;    // elements between groups
  uint8_t* dst;            // e4m3 [rows, 64], contiguous
  float* scale;            // [rows] or null
  const uint16_t* w;       // bf16 [rows] or null
  float* w_out;            // [rows] = w * scale, or null
};

__device__ __forceinline__ uint32_t cvt_e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

// ue8m0 scale of a row: 2^ceil(log2(fp32(max(amax, 1e-4) / 448))), from the
// exponent and mantissa bits of the quotient.
__device__ __forceinline__ float ue8m0_scale(float amax) {
  const float s = __fdiv_rn(fmaxf(amax, 1e-4f), 448.0f);
  const uint32_t u = __float_as_uint(s);
  const int e = static_cast<int>((u >> 23) & 0xFFu) - 127 + ((u & 0x7FFFFFu) != 0u ? 1 : 0);
  return __uint_as_float(static_cast<uint32_t>(e + 127) << 23);
}

__global__ void __launch_bounds__(256) fp8_quant_rows_kernel(const QuantParams p) {
  const int64_t r = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (r >= p.rows) return;
  const int64_t g = r / p.rows_per_group;
  const uint4* src = reinterpret_cast<const uint4*>(p.src + g * p.group_stride +
                                                    (r - g * p.rows_per_group) * kDim);
  float x[kDim];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint4 v = src[i];
    const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      x[8 * i + 2 * j] = __uint_as_float(w4[j] << 16);
      x[8 * i + 2 * j + 1] = __uint_as_float(w4[j] & 0xFFFF0000u);
    }
  }
  // Walsh-Hadamard transform, butterflies (a + b, a - b) over strides 1..32
#pragma unroll
  for (int lg = 0; lg < 6; ++lg) {
    const int len = 1 << lg;
#pragma unroll
    for (int m = 0; m < kDim / 2; ++m) {  // butterflies in ascending j
      const int j = ((m >> lg) << (lg + 1)) + (m & (len - 1));
      const float a = x[j], b = x[j + len];
      x[j] = __fadd_rn(a, b);
      x[j + len] = __fsub_rn(a, b);
    }
  }
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < kDim; ++i) {
    // * 2^-3 is exact; the rotated value is rounded to bf16
    x[i] = __uint_as_float(f32_to_bf16_rne(x[i] * 0.125f) << 16);
    amax = fmaxf(amax, fabsf(x[i]));
  }
  const float s = ue8m0_scale(amax);
  const float inv = __uint_as_float((254u << 23) - __float_as_uint(s));  // 1 / s, exact
  uint4* dst = reinterpret_cast<uint4*>(p.dst + r * kDim);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int e = 16 * i + 4 * j;
      o[j] = cvt_e4m3x2(x[e] * inv, x[e + 1] * inv) |
             (cvt_e4m3x2(x[e + 2] * inv, x[e + 3] * inv) << 16);
    }
    dst[i] = make_uint4(o[0], o[1], o[2], o[3]);
  }
  if (p.scale) p.scale[r] = s;
  if (p.w_out) p.w_out[r] = __uint_as_float(static_cast<uint32_t>(p.w[r]) << 16) * s;
}

}  // namespace ix8
}  // namespace dsa

namespace dsa {
namespace ix8 {

// ------------------------------------------------------------ score + top-k
constexpr int kHeads = 16;
constexpr int kTB = 16;                  // tokens per unit
constexpr int kQRows = kTB * kHeads;     // 256 (token, head) rows
constexpr int kChunk = 128;              // kv rows per MMA
constexpr int kMaxT = 1024;              // candidates held in smem per token
constexpr int kMaxK = 256;
constexpr int kStages = 4;
constexpr int kThreads = 512;  // warp 0 TMA, 1 MMA, 4-11 epilogue, 2-3 and 12-15 selection
constexpr int kEpiWarp0 = 4;
// Two epilogue warpgroups (tokens 0-7 / 8-15 of a unit); warps 2, 3 and
// 12..15 select, joined by the epilogue warps between units.
constexpr int kEpiWarps = 8;
constexpr int kEpiThreads = 32 * kEpiWarps;
constexpr int kEpiTokens = kTB * 4 / kEpiWarps;  // tokens per epilogue warpgroup
constexpr uint32_t kTmemCols = 512;      // two 256-column accumulators

constexpr int kQBytes = kQRows * kDim;                    // 16 KB
constexpr int kKVBytes = kChunk * kDim;                   // 8 KB
// Key buffers: two units of [16 tokens][1024] u32; a token's slot doubles as
// its selection's scratch (>= 3 KB). (Three 768-key buffers measured slower.)
constexpr int kKeyBufs = 2;
constexpr int kKeyRegion = kKeyBufs * kTB * kMaxT * 4;    // 128 KB
constexpr int kOffQ = 0;
constexpr int kOffKV = kOffQ + 2 * kQBytes;               // 32768
constexpr int kOffKeys = kOffKV + kStages * kKVBytes;     // 65536
constexpr int kOffWq = kOffKeys + kKeyRegion;             // 196608: [256] f32
constexpr int kOffNV = kOffWq + kQRows * 4;               // [16] int
constexpr int kOffBar = kOffNV + kTB * 4;
constexpr int kNumBars = 2 + 2 + 2 * kStages + 2 + 2 + 2 * kKeyBufs;
constexpr int kOffMisc = kOffBar + kNumBars * 8;
constexpr int kSmem = kOffMisc + 16 + 1024;
static_assert(kSmem <= 232448, "shared memory above the 227 KB per-block limit");

// Instruction descriptor for tcgen05.mma kind::f8f6f4 with E4M3 A and B,
// fp32 D, both K-major: [4,6) D fmt 1 (f32), [7,10) / [10,13) A / B fmt 0
// (E4M3), [17,23) N >> 3, [24,29) M >> 4.
constexpr uint32_t make_idesc_e4m3_f32(int M, int N) {
  return (1u << 4) | (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

// D[tmem] (+)= A[smem] * B[smem]^T for E4M3 operands, K = 32 per instruction.
__device__ __forceinline__ void umma_e4m3(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

struct Params {
  int B;
  int64_t S;
  int64_t T;          // candidates per batch (rows of k8 per batch)
  int K;              // top-k
  int ratio;
  int causal;
  int64_t offset;
  int n_tb;
  int units;
  const float* wq;    // [B*S, 16] weights times the q rows' scales
  const float* ks;    // [B*T] kv rows' scales
  int64_t* out;       // [B*S, K]
  float* scores;      // [B*S, T] or null (fp32 scores of the valid candidates)
  unsigned int* err;
};

__device__ __forceinline__ int64_t n_valid(const Params& p, int64_t t) {
  if (!p.causal) return p.T;
  const int64_t n = (t + 1) / p.ratio;
  return n < p.T ? n : p.T;
}

// Orderable image of an fp32 score (larger key = larger score, -0 == +0).
__device__ __forceinline__ uint32_t score_key(float s) {
  uint32_t u = __float_as_uint(s);
  if (u == 0x80000000u) u = 0u;
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Selection of token g of the CTA's sequence (unit lu = g / 16 of this CTA,
// token g % 16): waits until the unit's keys are written, selects the token's
// top-K, writes its indices and arrives on the key buffer's release barrier.
// Returns false past the CTA's last unit or when the wait gave up.
__device__ __forceinline__ bool select_token(const Params& p, int g, uint8_t* smem,
                                             uint64_t* keys_full, uint64_t* keys_empty,
                                             volatile int* abort_flag, int lane) {
  const int lu = g / kTB, tt = g % kTB;
  const int u = blockIdx.x + lu * gridDim.x;
  if (u >= p.units) return false;
  const int b = u % p.B;
  const int64_t t0 = static_cast<int64_t>(p.n_tb - 1 - u / p.B) * kTB;
  const int kb = lu & 1;
  if (!__all_sync(0xFFFFFFFFu, mbar_wait(&keys_full[kb], (lu >> 1) & 1, abort_flag, p.err,
                                         DSA_DEVERR_IX_WAIT)))
    return false;
  const int64_t tok = t0 + tt;
  if (tok < p.S) {
    uint32_t* keys = reinterpret_cast<uint32_t*>(smem + kOffKeys) + (kb * kTB + tt) * kMaxT;
    wsel::select_sorted_any(keys, static_cast<int>(n_valid(p, tok)), p.K,
                            p.out + (static_cast<int64_t>(b) * p.S + tok) * p.K, p.offset, lane);
  }
  __syncwarp();
  if (lane == 0) mbar_arrive(&keys_empty[kb]);
  return true;
}

// Next token of the CTA's selection sequence (one atomic per warp).
__device__ __forceinline__ int grab_token(int* next, int lane) {
  int g = 0;
  if (lane == 0) g = atomicAdd(next, 1);
  return __shfl_sync(0xFFFFFFFFu, g, 0);
}

// The next token if it lies below `limit` (tokens of units whose keys are
// complete), else -1; never takes a token at or past the limit.
__device__ __forceinline__ int try_grab_token(int* next, int limit, int lane) {
  int g = -1;
  if (lane == 0) {
    int cur = *reinterpret_cast<volatile int*>(next);
    while (cur < limit) {
      const int prev = atomicCAS(next, cur, cur + 1);
      if (prev == cur) {
        g = cur;
        break;
      }
      cur = prev;
    }
  }
  return __shfl_sync(0xFFFFFFFFu, g, 0);
}

__global__ void __launch_bounds__(kThreads, 1)
    score_fp8_kernel(const __grid_constant__ CUtensorMap tm_q,
                     const __grid_constant__ CUtensorMap tm_kv, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* q_full = bars;                     // [2] TMA
  uint64_t* q_empty = bars + 2;                // [2] MMA commit after the unit's last chunk
  uint64_t* kv_full = bars + 4;                // [kStages] TMA
  uint64_t* kv_empty = kv_full + kStages;      // [kStages] MMA commit
  uint64_t* acc_full = kv_empty + kStages;     // [2] MMA commit
  uint64_t* acc_empty = acc_full + 2;          // [2] one arrival per epilogue thread
  uint64_t* keys_full = acc_empty + 2;         // [2] one arrival per epilogue thread
  uint64_t* keys_empty = keys_full + kKeyBufs; // [2] 16 arrivals (one per token)
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kOffMisc + 4);
  int* sel_next = reinterpret_cast<int*>(smem + kOffMisc + 8);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], kEpiThreads);
    }
    for (int i = 0; i < kKeyBufs; ++i) {
      mbar_init(&keys_full[i], kEpiThreads);
      mbar_init(&keys_empty[i], kTB);
    }
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
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

  auto unit_of = [&](int u, int& b, int64_t& t0) {
    b = u % p.B;
    t0 = static_cast<int64_t>(p.n_tb - 1 - u / p.B) * kTB;  // heaviest token blocks first
  };
  auto unit_chunks = [&](int64_t t0) -> int {
    int64_t tl = t0 + kTB - 1;
    if (tl > p.S - 1) tl = p.S - 1;
    return static_cast<int>((n_valid(p, tl) + kChunk - 1) / kChunk);
  };

  if (warp >= kEpiWarp0 && warp < kEpiWarp0 + kEpiWarps) {
    // ------------------------------------------------------------- epilogue
    const int et = threadIdx.x - 32 * kEpiWarp0;   // 0 .. kEpiThreads - 1
    const int wg = et >> 7;                        // tokens [kEpiTokens wg, +kEpiTokens)
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;           // kv row of the chunk = TMEM lane
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    float* wq_s = reinterpret_cast<float*>(smem + kOffWq);
    int* nvs = reinterpret_cast<int*>(smem + kOffNV);
    bool ok = true;
    int lu = 0, gc = 0;
    for (int u = blockIdx.x; u < p.units; u += gridDim.x, ++lu) {
      int b;
      int64_t t0;
      unit_of(u, b, t0);
      const int nch = unit_chunks(t0);
      const int kb = lu & 1;
      uint32_t* keys = reinterpret_cast<uint32_t*>(smem + kOffKeys) + kb * kTB * kMaxT;
      for (int i = et; i < kQRows; i += kEpiThreads) {
        const int64_t tok = t0 + (i >> 4);
        wq_s[i] = tok < p.S ? p.wq[(static_cast<int64_t>(b) * p.S + tok) * kHeads + (i & 15)]
                            : 0.f;
      }
      {
        if (et < kTB) {
          const int64_t tk = t0 + et;
          nvs[et] = tk < p.S ? static_cast<int>(n_valid(p, tk)) : 0;
        }
      }
      // the key buffer is free once the selection of unit lu - 2 is done
      ok = __all_sync(0xFFFFFFFFu, mbar_wait(&keys_empty[kb], ((lu >> 1) & 1) ^ 1, abort_flag,
                                             p.err, DSA_DEVERR_IX_WAIT));
      ok = named_bar_and(1, kEpiThreads, ok);
      for (int c = 0; ok && c < nch; ++c, ++gc) {
        const int ab = gc & 1;
        const int k = c * kChunk + row;
        ok = __all_sync(0xFFFFFFFFu, mbar_wait(&acc_full[ab], (gc >> 1) & 1, abort_flag, p.err,
                                               DSA_DEVERR_IX_WAIT));
        if (!ok) break;
        tc_fence_after();
        const float ksv = k < p.T ? p.ks[static_cast<int64_t>(b) * p.T + k] : 0.f;
#pragma unroll 1
        for (int tl = 0; tl < kEpiTokens; tl += 2) {
          const int tt0 = wg * kEpiTokens + tl;
          // nothing to do when all 32 rows of this warp lie past both tokens'
          // valid candidates (the unit's last chunk under the causal mask)
          if (c * kChunk + quarter * 32 >= max(nvs[tt0], nvs[tt0 + 1])) continue;
          uint32_t r[32];
          tmem_ld_32x32b_x32(tmem + lane_off + static_cast<uint32_t>(ab * 256 + tt0 * 16), r);
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const int tt = tt0 + j;
            const float4* wv = reinterpret_cast<const float4*>(wq_s + tt * kHeads);
            float acc = 0.f;
#pragma unroll
            for (int h4 = 0; h4 < 4; ++h4) {
              const float4 w4 = wv[h4];
              const float wa[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
              for (int i = 0; i < 4; ++i)
                acc = __fmaf_rn(fmaxf(__uint_as_float(r[j * 16 + h4 * 4 + i]), 0.f), wa[i], acc);
            }
            const float score = __fmul_rn(acc, ksv);
            if (k < nvs[tt]) {
              keys[tt * kMaxT + k] = score_key(score);
              if (p.scores)
                p.scores[(static_cast<int64_t>(b) * p.S + t0 + tt) * p.T + k] = score;
            }
          }
        }
        tc_fence_before();
        mbar_arrive(&acc_empty[ab]);
      }
      // the epilogue leaves the unit together: its per-unit tables are rewritten next
      ok = named_bar_and(1, kEpiThreads, ok);
      if (!ok) break;
      mbar_arrive(&keys_full[kb]);
      // the selection is the longer stage: between units this warp also takes
      // pending tokens of the units before this one (their keys are complete)
      for (int g = try_grab_token(sel_next, lu * kTB, lane); g >= 0;
           g = try_grab_token(sel_next, lu * kTB, lane)) {
        if (!select_token(p, g, smem, keys_full, keys_empty, abort_flag, lane)) {
          ok = false;
          break;
        }
      }
      if (!__all_sync(0xFFFFFFFFu, ok)) break;
    }
    // after the last unit: help select the pairs still pending
    if (ok) {
      while (select_token(p, grab_token(sel_next, lane), smem, keys_full, keys_empty, abort_flag,
                          lane)) {
      }
    }
  } else if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
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
                    static_cast<int32_t>((static_cast<int64_t>(b) * p.S + t0) * kHeads),
                    &q_full[qb]);
        for (int c = 0; c < nch; ++c, ++gc) {
          const int s = gc % kStages;
          if (!mbar_wait(&kv_empty[s], ((gc / kStages) & 1) ^ 1, abort_flag, p.err,
                         DSA_DEVERR_IX_WAIT)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&kv_full[s], kKVBytes);
          tma_load_2d(smem + kOffKV + s * kKVBytes, &tm_kv, 0,
                      static_cast<int32_t>(static_cast<int64_t>(b) * p.T + c * kChunk),
                      &kv_full[s]);
        }
      }
      // wait for the copies still in flight (only after an abort can there be any)
      if (lu > 0) mbar_drain(&q_full[(lu - 1) & 1], ((lu - 1) >> 1) & 1);
      if (lu > 1) mbar_drain(&q_full[(lu - 2) & 1], ((lu - 2) >> 1) & 1);
      for (int i = (gc > kStages ? gc - kStages : 0); i < gc; ++i)
        mbar_drain(&kv_full[i % kStages], (i / kStages) & 1);
    }
  } else if (warp == 1) {
    // -------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_e4m3_f32(kChunk, kQRows);
      int lu = 0, gc = 0;
      bool ok = true;
      for (int u = blockIdx.x; ok && u < p.units; u += gridDim.x, ++lu) {
        int b;
        int64_t t0;
        unit_of(u, b, t0);
        const int nch = unit_chunks(t0);
        const int qb = lu & 1;
        if (!mbar_wait(&q_full[qb], (lu >> 1) & 1, abort_flag, p.err, DSA_DEVERR_IX_WAIT)) break;
        const uint32_t qaddr = smem_u32(smem + kOffQ + qb * kQBytes);
        for (int c = 0; c < nch; ++c, ++gc) {
          const int s = gc % kStages;
          const int ab = gc & 1;
          if (!mbar_wait(&kv_full[s], (gc / kStages) & 1, abort_flag, p.err, DSA_DEVERR_IX_WAIT) ||
              !mbar_wait(&acc_empty[ab], ((gc >> 1) & 1) ^ 1, abort_flag, p.err,
                         DSA_DEVERR_IX_WAIT)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t kvaddr = smem_u32(smem + kOffKV + s * kKVBytes);
#pragma unroll
          for (int kk = 0; kk < kDim / 32; ++kk) {
            const uint64_t ad = make_smem_desc(kvaddr + kk * 32, 16u, 512u, kLayoutSW64);
            const uint64_t bd = make_smem_desc(qaddr + kk * 32, 16u, 512u, kLayoutSW64);
            umma_e4m3(tmem + static_cast<uint32_t>(ab) * 256u, ad, bd, idesc, kk > 0 ? 1u : 0u);
          }
          umma_commit(&kv_empty[s]);
          umma_commit(&acc_full[ab]);
        }
        if (!ok) break;
        umma_commit(&q_empty[qb]);  // every unit releases its q tile, even one without chunks
      }
      if (gc > 0) mbar_drain(&acc_full[(gc - 1) & 1], ((gc - 1) >> 1) & 1);
      if (gc > 1) mbar_drain(&acc_full[(gc - 2) & 1], ((gc - 2) >> 1) & 1);
    }
  } else {
    // ------------------------------------------------------------- selection
    while (select_token(p, grab_token(sel_next, lane), smem, keys_full, keys_empty, abort_flag,
                        lane)) {
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

}  // namespace ix8

int launch_fp8_quant_rows(const void* src, int64_t rows, int64_t rows_per_group,
                          int64_t group_stride, void* dst, float* scale, const void* w,
                          float* w_out, cudaStream_t stream) {
  using namespace ix8;
  if (rows <= 0) return DSA_OK;
  QuantParams p;
  p.src = static_cast<const uint16_t*>(src);
  p.rows = rows;
  p.rows_per_group = rows_per_group;
  p.group_stride = group_stride;
  p.dst = static_cast<uint8_t*>(dst);
  p.scale = scale;
  p.w = static_cast<const uint16_t*>(w);
  p.w_out = w_out;
  const int64_t blocks = (rows + 255) / 256;
  fp8_quant_rows_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(p);
  return cuda_status(cudaGetLastError());
}

// q8 [batch*seqlen*16, 64] e4m3, wq [batch*seqlen, 16] f32, k8 [batch*n_cand, 64]
// e4m3, ks [batch*n_cand] f32; n_cand <= 1024, topk <= 256.
int launch_score_fp8(const void* q8, const float* wq, const void* k8, const float* ks,
                     int64_t* out, float* scores, int64_t batch, int64_t seqlen, int64_t n_cand,
                     int topk, int64_t start_pos, int ratio, int64_t offset,
                     cudaStream_t stream) {
  using namespace ix8;
  if (n_cand > kMaxT || topk > kMaxK) return DSA_ERR_UNSUPPORTED;
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
    const uint64_t strides[1] = {kDim};
    const uint32_t box[2] = {kDim, kQRows};
    st = encode_tensor_map(&tm_q, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, q8, dims, strides, box,
                           CU_TENSOR_MAP_SWIZZLE_64B);
    if (st != DSA_OK) return st;
  }
  {
    const uint64_t dims[2] = {kDim, static_cast<uint64_t>(batch * n_cand)};
    const uint64_t strides[1] = {kDim};
    const uint32_t box[2] = {kDim, kChunk};
    st = encode_tensor_map(&tm_kv, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, k8, dims, strides, box,
                           CU_TENSOR_MAP_SWIZZLE_64B);
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
  p.wq = wq;
  p.ks = ks;
  p.out = out;
  p.scores = scores;
  p.err = err;
  st = set_max_dynamic_smem(reinterpret_cast<const void*>(score_fp8_kernel), kSmem);
  if (st != DSA_OK) return st;
  const int grid = p.units < di.num_sms ? p.units : di.num_sms;
  score_fp8_kernel<<<grid, kThreads, kSmem, stream>>>(tm_q, tm_kv, p);
  return cuda_status(cudaGetLastError());
}

}  // namespace dsa
