// Lightning Indexer weights projection for sm_100a, exact int8 slicing:
//
//   w = bf16(bf16(x . w_proj^T) * scale)      reference/task2_v0_ref.py:132
//
// with x [M, K] bf16 (K = dim <= 1024) and w_proj [16, K] bf16. As for the q
// projection, both operands are cut into three signed 7-bit slices on their
// rows' own exponent grids (indexer_split.cu):
//   a = 2^(sa-7) A1 + 2^(sa-14) A2 + 2^(sa-21) A3 + ra   (same for b),
// and the slice products with i + j <= 5 accumulate EXACTLY on the int8 tensor
// cores (int32, |level| < 2^26 for K <= 1024), one TMEM accumulator per level
// s = i + j (L2..L5):
//   a.b = 2^(sa+sb) (L2 2^-14 + L3 2^-21 + L4 2^-28 + L5 2^-35) + d,
//   |d| <= 2^(sa+sb) (err_a + err_b + 2^-42 ||A3|| ||B3||).
// The epilogue forms T = H + G 2^-14 (H = 128 L2 + L3, G = 128 L4 + L5, exact
// in 64-bit integers, converted to fp32 with a rigorous bound), certifies the
// bf16 rounding of T, adds the exponent sa + sb - 21 to the bf16 bits (exact for
// normal results, checked per row), and applies the scale (fp32 product, RNE).
// The rare elements it cannot certify are recomputed in the epilogue as the
// sequential fp64 dot product of the bf16 inputs (the CPU oracle's arithmetic),
// split over a warp when the rows' bit spans make any summation order exact.
//
// MMA shape: the three w_proj slices sit one after another in smem ([B1; B2; B3],
// 16 rows each) and the level accumulators 16 TMEM columns apart, so one MMA of
// A_i against the stacked B (N = 48) adds A_i.B1, A_i.B2, A_i.B3 into levels
// i+1, i+2, i+3: three MMAs per 32-wide k step.
//
// One CTA per SM, persistent over 128-row tiles: warp 0 TMA (w_proj slices once,
// then the three x slices of each 128-wide k atom into a 3-stage ring), warp 1
// tcgen05 issuer, warps 2..5 epilogue (one thread per row, two TMEM buffers).
#include "common.cuh"
#include "host_util.h"
#include "numerics.cuh"

namespace dsa {
namespace ixw {

constexpr int kBM = 128;
constexpr int kBN = 16;
constexpr int kMaxK = 1024;
constexpr int kSlices = 3;
constexpr int kStages = 3;
constexpr int kThreads = 192;
constexpr int kABox = kBM * 128;                       // 16 KB: 128 rows x 128 k
constexpr int kAStage = kSlices * kABox;               // 48 KB
constexpr int kBAtom = kSlices * kBN * 128;            // 6 KB: [B1; B2; B3] of one k atom
constexpr int kOffA = 0;
constexpr int kOffB = kOffA + kStages * kAStage;       // 147456
constexpr int kOffCol = kOffB + (kMaxK / 128) * kBAtom;  // 196608: per column sb, eb, nb
constexpr int kQueueCap = 512;                         // per warp
constexpr int kOffQueue = kOffCol + 3 * kBN * 4;
constexpr int kOffBar = kOffQueue + 4 * kQueueCap * 4;
constexpr int kNumBars = 2 * kStages + 1 + 2 * 2;
constexpr int kOffMisc = kOffBar + kNumBars * 8;
constexpr int kSmem = kOffMisc + 16 + 1024;
constexpr uint32_t kTmemCols = 128;                    // 2 buffers x 4 levels x 16 columns
constexpr uint32_t kBufCols = 64;

struct Params {
  int M;
  int K;          // multiple of 64, <= 1024
  int m_tiles;
  float scale;
  const int* a_sig;     // [M]
  const float* a_err;   // [M]
  const float* a_n3;    // [M]
  const int* b_sig;     // [16]
  const float* b_err;   // [16]
  const float* b_n3;    // [16]
  const int* b_span;    // [16] bit spans (indexer_split.cu)
  const uint16_t* x;    // bf16 [M, K], for the exact recomputation
  const uint16_t* wp;   // bf16 [16, K]
  uint16_t* w_out;      // bf16 [M, 16]
  unsigned int* err;
};

__global__ void __launch_bounds__(kThreads, 1)
    wproj_s8_kernel(const __grid_constant__ CUtensorMap tm_a,  // int8 [3][M][K]
                    const __grid_constant__ CUtensorMap tm_b,  // int8 [3][16][K]
                    const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* a_full = bars;                   // [kStages]
  uint64_t* a_empty = bars + kStages;        // [kStages]
  uint64_t* b_full = bars + 2 * kStages;
  uint64_t* acc_full = b_full + 1;           // [2]
  uint64_t* acc_empty = acc_full + 2;        // [2], 128 arrivals
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kOffMisc + 4);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int katoms = p.K / 128 + ((p.K % 128) ? 1 : 0);
  const int ksteps = p.K / 32;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&a_full[s], 1);
      mbar_init(&a_empty[s], 1);
    }
    mbar_init(b_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 128);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_a);
    tma_prefetch_desc(&tm_b);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      mbar_arrive_expect_tx(b_full, katoms * kBAtom);
      for (int kb = 0; kb < katoms; ++kb)
        for (int j = 0; j < kSlices; ++j)
          tma_load_3d(smem + kOffB + kb * kBAtom + j * kBN * 128, &tm_b, kb * 128, 0, j, b_full);
      int it = 0;
      bool ok = true;
      for (int mt = blockIdx.x; ok && mt < p.m_tiles; mt += gridDim.x) {
        for (int kb = 0; kb < katoms; ++kb, ++it) {
          const int s = it % kStages;
          if (!mbar_wait(&a_empty[s], ((it / kStages) & 1) ^ 1, abort_flag, p.err,
                         DSA_DEVERR_GEMM_WAIT)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&a_full[s], kAStage);
          for (int j = 0; j < kSlices; ++j)
            tma_load_3d(smem + kOffA + s * kAStage + j * kABox, &tm_a, kb * 128, mt * kBM, j,
                        &a_full[s]);
        }
      }
      mbar_drain(b_full, 0);
      for (int i = (it > kStages ? it - kStages : 0); i < it; ++i)
        mbar_drain(&a_full[i % kStages], (i / kStages) & 1);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc48 = make_idesc_s8_s32(128, 3 * kBN);
      constexpr uint32_t idesc32 = make_idesc_s8_s32(128, 2 * kBN);
      constexpr uint32_t idesc16 = make_idesc_s8_s32(128, kBN);
      const uint32_t a_base = smem_u32(smem + kOffA);
      const uint32_t b_base = smem_u32(smem + kOffB);
      int it = 0, lt = 0;
      bool ok = mbar_wait(b_full, 0, abort_flag, p.err, DSA_DEVERR_GEMM_WAIT);
      for (int mt = blockIdx.x; ok && mt < p.m_tiles; mt += gridDim.x, ++lt) {
        const int ab = lt & 1;
        if (!mbar_wait(&acc_empty[ab], ((lt >> 1) & 1) ^ 1, abort_flag, p.err,
                       DSA_DEVERR_GEMM_WAIT))
          break;
        tc_fence_after();
        const uint32_t d = tmem + static_cast<uint32_t>(ab) * kBufCols;
        for (int kb = 0; kb < katoms; ++kb, ++it) {
          const int s = it % kStages;
          if (!mbar_wait(&a_full[s], (it / kStages) & 1, abort_flag, p.err,
                         DSA_DEVERR_GEMM_WAIT)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t as = a_base + static_cast<uint32_t>(s) * kAStage;
          const uint32_t bs = b_base + static_cast<uint32_t>(kb) * kBAtom;
          const int nstep = min(4, ksteps - kb * 4);
          for (int step = 0; step < nstep; ++step) {
            const uint32_t ko = static_cast<uint32_t>(step) * 32u;
            const uint64_t da1 = make_smem_desc(as + 0 * kABox + ko, 16u, 1024u, kLayoutSW128);
            const uint64_t da2 = make_smem_desc(as + 1 * kABox + ko, 16u, 1024u, kLayoutSW128);
            const uint64_t da3 = make_smem_desc(as + 2 * kABox + ko, 16u, 1024u, kLayoutSW128);
            const uint64_t db123 = make_smem_desc(bs + ko, 16u, 1024u, kLayoutSW128);
            // the A3 product between the other two, as in the q projection
            // (after the A2 MMA, whose columns it overlaps, it stalls the pipe)
            if (kb == 0 && step == 0) {
              // first k step: every level's first writer overwrites it
              const uint64_t db3 = make_smem_desc(bs + 2 * kBN * 128 + ko, 16u, 1024u,
                                                  kLayoutSW128);
              umma_s8(d + 0 * kBN, da1, db123, idesc48, 0u);  // L2, L3, L4
              umma_s8(d + 3 * kBN, da2, db3, idesc16, 0u);    // L5
              umma_s8(d + 2 * kBN, da3, db123, idesc32, 1u);  // L4, L5
              umma_s8(d + 1 * kBN, da2, db123, idesc32, 1u);  // L3, L4
            } else {
              umma_s8(d + 0 * kBN, da1, db123, idesc48, 1u);  // L2, L3, L4
              umma_s8(d + 2 * kBN, da3, db123, idesc32, 1u);  // L4, L5
              umma_s8(d + 1 * kBN, da2, db123, idesc48, 1u);  // L3, L4, L5
            }
          }
          umma_commit(&a_empty[s]);
        }
        if (!ok) break;
        umma_commit(&acc_full[ab]);
      }
      if (lt > 0) mbar_drain(&acc_full[(lt - 1) & 1], ((lt - 1) >> 1) & 1);
      if (lt > 1) mbar_drain(&acc_full[(lt - 2) & 1], ((lt - 2) >> 1) & 1);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int ew = warp - 2;                 // 0..3
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;     // tile row = TMEM lane
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    uint32_t* queue = reinterpret_cast<uint32_t*>(smem + kOffQueue) + ew * kQueueCap;
    int* csb = reinterpret_cast<int*>(smem + kOffCol);
    float* ceb = reinterpret_cast<float*>(smem + kOffCol) + kBN;
    float* cnb = reinterpret_cast<float*>(smem + kOffCol) + 2 * kBN;
    const int t = threadIdx.x - 64;          // 0..127
    if (t < kBN) {
      csb[t] = __ldg(p.b_sig + t);
      ceb[t] = __ldg(p.b_err + t) * 0x1p21f;              // exact scaling
      cnb[t] = __fmul_ru(__ldg(p.b_n3 + t), 0x1p-21f);
    }
    named_bar_sync(1, 128);
    int sb_min = 1 << 30, sb_max = -(1 << 30);
#pragma unroll
    for (int i = 0; i < kBN; ++i) {
      sb_min = min(sb_min, csb[i]);
      sb_max = max(sb_max, csb[i]);
    }
    bool ok = true;
    int lt = 0;
    for (int mt = blockIdx.x; ok && mt < p.m_tiles; mt += gridDim.x, ++lt) {
      const int ab = lt & 1;
      const int m0 = mt * kBM;
      const bool row_valid = (m0 + row) < p.M;
      const int sa = row_valid ? __ldg(p.a_sig + m0 + row) : 0;
      const float eaT = row_valid ? __ldg(p.a_err + m0 + row) * 0x1p21f : 0.f;
      const float na3 = row_valid ? __ldg(p.a_n3 + m0 + row) : 0.f;
      const int ex_row = sa - 21 + 127;
      const uint32_t rsh = static_cast<uint32_t>(sa - 21) << 7;
      // a certified T (|T| >= 2^-6, below 2^33) scales into a normal bf16 when the
      // biased exponent sa + sb - 21 + 127 stays in [15, 221]
      const bool row_ok = row_valid && ex_row + sb_min >= 15 && ex_row + sb_max <= 221;
      ok = __all_sync(0xFFFFFFFFu, mbar_wait(&acc_full[ab], (lt >> 1) & 1, abort_flag, p.err,
                                             DSA_DEVERR_GEMM_WAIT));
      if (!named_bar_and(1, 128, ok)) break;
      tc_fence_after();
      uint32_t l2[16], l3[16], l4[16], l5[16];
      const uint32_t d = tmem + lane_off + static_cast<uint32_t>(ab) * kBufCols;
      tmem_ld4_32x32b_x16(d + 0 * kBN, d + 1 * kBN, d + 2 * kBN, d + 3 * kBN, l2, l3, l4, l5);
      tc_fence_before();
      mbar_arrive(&acc_empty[ab]);
      uint32_t bits[kBN];
      uint32_t flagged = 0;
#pragma unroll
      for (int i = 0; i < kBN; ++i) {
        const long long H = 128ll * static_cast<int>(l2[i]) + static_cast<int>(l3[i]);
        const long long G = 128ll * static_cast<int>(l4[i]) + static_cast<int>(l5[i]);
        const float Hf = __ll2float_rn(H);
        const float Gs = __ll2float_rn(G) * 0x1p-14f;  // exact power-of-two scaling
        const float T = __fadd_rn(Hf, Gs);
        // |T - (H + G 2^-14)| <= 2^-24 (|H| + |G 2^-14| + |T|) <= 2^-22 (|Hf| + |Gs|),
        // plus the data's remainder and A3.B3 bounds and a floor of 2^-5
        const float e_data = __fadd_ru(__fmaf_ru(na3, cnb[i], __fadd_ru(eaT, ceb[i])), 0x1p-5f);
        const float E = __fmaf_ru(__fadd_ru(fabsf(Hf), fabsf(Gs)), 0x1p-22f, e_data);
        uint32_t pr;
        asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(pr) : "f"(__fadd_ru(T, E)), "f"(__fsub_rd(T, E)));
        bits[i] = (pr >> 16) + rsh + (static_cast<uint32_t>(csb[i]) << 7);
        if (((pr ^ (pr >> 16)) & 0xFFFFu) != 0 || !row_ok) flagged |= 1u << i;
      }
      if (!row_valid) flagged = 0;
      // exact recomputation of the uncertain elements, one lane per element
      // (sequential fp64 dot of the bf16 inputs, ascending k)
      const int cnt = __popc(flagged);
      int incl = cnt;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xFFFFFFFFu, incl, o);
        if (lane >= o) incl += v;
      }
      const int total = __shfl_sync(0xFFFFFFFFu, incl, 31);
      if (total > 0) {
        int wpos = incl - cnt;
        uint32_t f = flagged;
        while (f) {
          const int col = __ffs(static_cast<int>(f)) - 1;
          f &= f - 1;
          queue[wpos++] = static_cast<uint32_t>((row << 8) | col);
        }
        __syncwarp();
        const int n = total;  // <= 32 rows x 16 columns = kQueueCap
        // one element at a time by the whole warp: when the rows' bit spans make
        // every partial sum exact in fp64 (span_x + span_w + log2 K <= 53), any
        // order gives the sequential sum, so each lane sums a 32-wide slice of k
        // and the warp adds the lanes' sums; otherwise lane 0 sums in order
        int log2k = 0;
        while ((1 << log2k) < p.K) ++log2k;
        for (int i = 0; i < n; ++i) {
          const uint32_t e = queue[i];
          const int r = static_cast<int>(e >> 8), c = static_cast<int>(e & 0xFF);
          const uint16_t* xr = p.x + static_cast<int64_t>(m0 + r) * p.K;
          const uint16_t* wr = p.wp + static_cast<int64_t>(c) * p.K;
          // the x row's span (sigma - lowest set bit), from the lanes' slices of k
          const int k0 = lane * 32;
          uint4 av[4], bv[4];
          int low = 1 << 30;
          if (k0 < p.K) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              av[j] = __ldg(reinterpret_cast<const uint4*>(xr + k0 + 8 * j));
              bv[j] = __ldg(reinterpret_cast<const uint4*>(wr + k0 + 8 * j));
              low = min(low, min(min(bf16x2_low_bit(av[j].x), bf16x2_low_bit(av[j].y)),
                                 min(bf16x2_low_bit(av[j].z), bf16x2_low_bit(av[j].w))));
            }
          }
          low = __reduce_min_sync(0xFFFFFFFFu, low);
          const int sg = __ldg(p.a_sig + m0 + r);
          const int a_span = sg >= (1 << 20) ? (1 << 20) : (low == (1 << 30) ? 0 : sg - low);
          const bool any_order = a_span + __ldg(p.b_span + c) + log2k <= 53;
          // the warp's sum of the exact fp64 products (each lane a 32-wide slice
          // of k, then the lanes), and of their magnitudes: equal to the oracle's
          // sequential sum when any order is exact, else certified against it
          double acc64 = 0.0, mag64 = 0.0;
          if (k0 < p.K) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const uint32_t aw[4] = {av[j].x, av[j].y, av[j].z, av[j].w};
              const uint32_t bw[4] = {bv[j].x, bv[j].y, bv[j].z, bv[j].w};
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                const double p0 = static_cast<double>(bf16lo_to_f32(aw[q])) *
                                  static_cast<double>(bf16lo_to_f32(bw[q]));
                const double p1 = static_cast<double>(bf16hi_to_f32(aw[q])) *
                                  static_cast<double>(bf16hi_to_f32(bw[q]));
                acc64 = __dadd_rn(acc64, p0);
                acc64 = __dadd_rn(acc64, p1);
                mag64 += fabs(p0) + fabs(p1);
              }
            }
          }
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) {
            acc64 += __shfl_xor_sync(0xFFFFFFFFu, acc64, o);
            mag64 += __shfl_xor_sync(0xFFFFFFFFu, mag64, o);
          }
          uint32_t cert_bits;
          if (!any_order && !certify_seq_dot_bf16(acc64, mag64, &cert_bits) && lane == 0) {
            // the oracle's own chain: one lane, ascending k
            acc64 = 0.0;
            for (int k8 = 0; k8 < p.K; k8 += 8) {
              const uint4 av8 = __ldg(reinterpret_cast<const uint4*>(xr + k8));
              const uint4 bv8 = __ldg(reinterpret_cast<const uint4*>(wr + k8));
              const uint32_t aw[4] = {av8.x, av8.y, av8.z, av8.w};
              const uint32_t bw[4] = {bv8.x, bv8.y, bv8.z, bv8.w};
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                acc64 = fma(static_cast<double>(bf16lo_to_f32(aw[q])),
                            static_cast<double>(bf16lo_to_f32(bw[q])), acc64);
                acc64 = fma(static_cast<double>(bf16hi_to_f32(aw[q])),
                            static_cast<double>(bf16hi_to_f32(bw[q])), acc64);
              }
            }
          }
          if (lane == 0) queue[i] = (e & 0xFFFFu) | (round_f64_to_bf16(acc64) << 16);
        }
        __syncwarp();
        for (int i = 0; i < n; ++i) {
          const uint32_t e = queue[i];
          if (static_cast<int>((e >> 8) & 0xFF) == row) {
            const uint32_t c = e & 0xFFu;
#pragma unroll
            for (int j = 0; j < kBN; ++j)
              if (static_cast<uint32_t>(j) == c) bits[j] = e >> 16;
          }
        }
        __syncwarp();
      }
      if (row_valid) {
        uint32_t o[kBN / 2];
#pragma unroll
        for (int i = 0; i < kBN; i += 2) {
          const uint32_t lo = f32_to_bf16_rne(__fmul_rn(__uint_as_float(bits[i] << 16), p.scale));
          const uint32_t hi =
              f32_to_bf16_rne(__fmul_rn(__uint_as_float(bits[i + 1] << 16), p.scale));
          o[i >> 1] = lo | (hi << 16);
        }
        uint4* dst = reinterpret_cast<uint4*>(p.w_out + static_cast<int64_t>(m0 + row) * kBN);
        dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
        dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
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

}  // namespace ixw

int launch_row_split2(const void* a_src, int64_t a_rows, void* a_slices, int* a_sig,
                      float* a_err, float* a_n3, int* a_span, const void* b_src, int64_t b_rows,
                      void* b_slices, int* b_sig, float* b_err, float* b_n3, int* b_span, int K,
                      cudaStream_t stream);

// Scratch the sliced w projection needs (256-byte aligned pieces).
size_t wproj_s8_scratch_bytes(int64_t rows, int K) {
  auto a256 = [](size_t v) { return (v + 255) & ~static_cast<size_t>(255); };
  const size_t R = static_cast<size_t>(rows), Kz = static_cast<size_t>(K);
  return a256(3 * R * Kz) + 3 * a256(R * 4) + a256(3 * 16 * Kz) + 4 * a256(16 * 4);
}

int launch_wproj_s8(const void* x, const void* wp, void* w_out, int64_t rows, int K, float scale,
                    void* scratch, cudaStream_t stream) {
  using namespace ixw;
  if (rows <= 0) return DSA_OK;
  if (K <= 0 || K > kMaxK || K % 64 != 0) return DSA_ERR_UNSUPPORTED;
  DeviceInfo di;
  int st = current_device_info(&di);
  if (st != DSA_OK) return st;
  if (di.max_smem_optin < kSmem) return DSA_ERR_UNSUPPORTED;
  unsigned int* err = nullptr;
  st = device_error_word(&err);
  if (st != DSA_OK) return st;
  auto a256 = [](size_t v) { return (v + 255) & ~static_cast<size_t>(255); };
  const size_t R = static_cast<size_t>(rows), Kz = static_cast<size_t>(K);
  uint8_t* ws = static_cast<uint8_t*>(scratch);
  int8_t* a_sl = reinterpret_cast<int8_t*>(ws);
  ws += a256(3 * R * Kz);
  int* a_sig = reinterpret_cast<int*>(ws);
  ws += a256(R * 4);
  float* a_err = reinterpret_cast<float*>(ws);
  ws += a256(R * 4);
  float* a_n3 = reinterpret_cast<float*>(ws);
  ws += a256(R * 4);
  int8_t* b_sl = reinterpret_cast<int8_t*>(ws);
  ws += a256(3 * 16 * Kz);
  int* b_sig = reinterpret_cast<int*>(ws);
  ws += a256(16 * 4);
  float* b_err = reinterpret_cast<float*>(ws);
  ws += a256(16 * 4);
  float* b_n3 = reinterpret_cast<float*>(ws);
  ws += a256(16 * 4);
  int* b_span = reinterpret_cast<int*>(ws);
  // w_proj rows (with bit spans, for the exact fix-up) and x rows in one launch
  st = launch_row_split2(wp, kBN, b_sl, b_sig, b_err, b_n3, b_span, x, rows, a_sl, a_sig, a_err,
                         a_n3, nullptr, K, stream);
  if (st != DSA_OK) return st;
  CUtensorMap tm_a, tm_b;
  {
    const uint64_t dims[3] = {Kz, R, 3};
    const uint64_t strides[2] = {Kz, R * Kz};
    const uint32_t box[3] = {128, kBM, 1};
    st = encode_tensor_map(&tm_a, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, a_sl, dims, strides, box,
                           CU_TENSOR_MAP_SWIZZLE_128B);
    if (st != DSA_OK) return st;
  }
  {
    const uint64_t dims[3] = {Kz, static_cast<uint64_t>(kBN), 3};
    const uint64_t strides[2] = {Kz, static_cast<uint64_t>(kBN) * Kz};
    const uint32_t box[3] = {128, kBN, 1};
    st = encode_tensor_map(&tm_b, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, b_sl, dims, strides, box,
                           CU_TENSOR_MAP_SWIZZLE_128B);
    if (st != DSA_OK) return st;
  }
  Params p;
  p.M = static_cast<int>(rows);
  p.K = K;
  p.m_tiles = static_cast<int>((rows + kBM - 1) / kBM);
  p.scale = scale;
  p.a_sig = a_sig;
  p.a_err = a_err;
  p.a_n3 = a_n3;
  p.b_sig = b_sig;
  p.b_err = b_err;
  p.b_n3 = b_n3;
  p.b_span = b_span;
  p.x = static_cast<const uint16_t*>(x);
  p.wp = static_cast<const uint16_t*>(wp);
  p.w_out = static_cast<uint16_t*>(w_out);
  p.err = err;
  st = set_max_dynamic_smem(reinterpret_cast<const void*>(wproj_s8_kernel), kSmem);
  if (st != DSA_OK) return st;
  const int grid = p.m_tiles < di.num_sms ? p.m_tiles : di.num_sms;
  wproj_s8_kernel<<<grid, kThreads, kSmem, stream>>>(tm_a, tm_b, p);
  return cuda_status(cudaGetLastError());
}

}  // namespace dsa
