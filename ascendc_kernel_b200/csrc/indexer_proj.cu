// Lightning Indexer projections for sm_100a, with correctly rounded bf16 outputs.
//
//   q = RoPE(bf16(qr . wq_b^T))          reference/task2_v0_ref.py:129-131
//   w = bf16(bf16(x . w_proj^T) * scale) reference/task2_v0_ref.py:132
//
// Both are tcgen05 GEMMs (TMA -> SW128 smem -> UMMA -> TMEM). The K sum is
// split over TMEM accumulators of kKC = 32 (two K=16 MMA steps each) so that
// the accumulation error bound stays small; the epilogue merges the chunks in
// fp32, certifies the bf16 rounding against the bound (numerics.cuh) and
// recomputes the few uncertain elements exactly (fp64, ascending k, one lane
// per element) before applying RoPE / the scale.
//
// q projection kernel (one CTA per SM, persistent):
//   work unit = (128-row M tile, group of 4 heads); the A tile (128 x K,
//   K <= 256) stays resident in smem for the unit, the B tile of each head
//   (64 x K) is double buffered; TMEM holds K/32 accumulators of 64 columns.
//   warp 0 TMA, warp 1 MMA, warps 2..5 epilogue (one thread per row).
// w projection kernel: work unit = 128-row M tile; x streams through a
//   4-stage ring of 128 x 64 boxes, w_proj (16 x K, K <= 1024) is resident;
//   TMEM holds K/32 accumulators of 16 columns. The epilogue threads also read
//   every x stage to form their row norm before the stage is released.
#include "common.cuh"
#include "host_util.h"
#include "numerics.cuh"

namespace dsa {
namespace ixp {

constexpr int kBM = 128;
constexpr int kKC = 32;
constexpr int kBox = kBM * 128;  // 128 rows x 64 bf16 = 16 KB
constexpr uint32_t kTmemCols = 512;

// Accumulation error bound factor (units of ||a||*||b||): 3 fp32 ulps per
// K=16 step of the chunk (the measured worst case is ~1) plus the sequential
// fp32 merge of the chunk sums.
__host__ __device__ constexpr float gamma_for(int nchunks) {
  return (3.0f * (kKC / 16) * 2.0f + static_cast<float>(nchunks)) * kTwoM24 * 1.0001f;
}

// ------------------------------------------------------------------ q proj
constexpr int kQBN = 64;
constexpr int kQMaxK = 256;
constexpr int kQGroup = 4;
constexpr int kQThreads = 192;
constexpr int kQBBox = kQBN * 128;  // 8 KB
constexpr int kQOffA = 0;
constexpr int kQOffB = kQOffA + (kQMaxK / 64) * kBox;             // 65536
constexpr int kQOffOut = kQOffB + 2 * (kQMaxK / 64) * kQBBox;     // 131072
constexpr int kQOffNB = kQOffOut + 2 * kBox;                      // 163840
constexpr int kQQueueCap = 2048;                                  // per warp
constexpr int kQOffQueue = kQOffNB + kQBN * 4;                    // 164096
constexpr int kQOffBar = kQOffQueue + 4 * kQQueueCap * 4;         // 196864
constexpr int kQNumBars = 8;
constexpr int kQOffMisc = kQOffBar + kQNumBars * 8;
constexpr int kQSmem = kQOffMisc + 16 + 1024;

struct QParams {
  int M;           // rows (tokens)
  int K;           // q_lora_rank, multiple of 64, <= 256
  int n_tiles;     // heads (N / 64)
  int m_tiles;
  int units;       // m_tiles * n_groups
  int n_groups;
  int rope_dim;    // even, <= 64
  int64_t seqlen;  // row r is at position r % seqlen of cos/sin
  float gamma;
  const float* cos_tab;
  const float* sin_tab;
  unsigned int* err;
};

__device__ __forceinline__ uint32_t sw128_off(int row, int chunk16) {
  return static_cast<uint32_t>(row * 128 + ((chunk16 ^ (row & 7)) << 4));
}

// Exact dot product of two smem rows stored as SW128 boxes of 64 columns,
// fp64 in ascending k, rounded once to bf16.
__device__ __forceinline__ uint32_t exact_dot_sw128(const uint8_t* a_base, int a_row,
                                                    int a_box_bytes, const uint8_t* b_base,
                                                    int b_row, int b_box_bytes, int K) {
  double acc = 0.0;
  for (int kb = 0; kb < K / 64; ++kb) {
#pragma unroll
    for (int ch = 0; ch < 8; ++ch) {
      const uint4 av =
          *reinterpret_cast<const uint4*>(a_base + kb * a_box_bytes + sw128_off(a_row, ch));
      const uint4 bv =
          *reinterpret_cast<const uint4*>(b_base + kb * b_box_bytes + sw128_off(b_row, ch));
      const uint32_t aw[4] = {av.x, av.y, av.z, av.w};
      const uint32_t bw[4] = {bv.x, bv.y, bv.z, bv.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        acc = fma(static_cast<double>(bf16lo_to_f32(aw[e])),
                  static_cast<double>(bf16lo_to_f32(bw[e])), acc);
        acc = fma(static_cast<double>(bf16hi_to_f32(aw[e])),
                  static_cast<double>(bf16hi_to_f32(bw[e])), acc);
      }
    }
  }
  return round_f64_to_bf16(acc);
}

__global__ void __launch_bounds__(kQThreads, 1)
    qproj_rope_kernel(const __grid_constant__ CUtensorMap tm_a,
                      const __grid_constant__ CUtensorMap tm_b,
                      const __grid_constant__ CUtensorMap tm_q, const QParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kQOffBar);
  uint64_t* a_full = bars + 0;
  uint64_t* a_empty = bars + 1;
  uint64_t* b_full = bars + 2;   // [2]
  uint64_t* b_empty = bars + 4;  // [2]
  uint64_t* acc_full = bars + 6;
  uint64_t* acc_empty = bars + 7;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + kQOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kQOffMisc + 4);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int KB = p.K / 64;
  const int nch = p.K / kKC;

  if (threadIdx.x == 0) {
    mbar_init(a_full, 1);
    mbar_init(a_empty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&b_full[i], 1);
      mbar_init(&b_empty[i], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, 128);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_a);
    tma_prefetch_desc(&tm_b);
    tma_prefetch_desc(&tm_q);
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
    if (lane == 0) {
      int lu = 0, g = 0;
      bool ok = true;
      for (int u = blockIdx.x; ok && u < p.units; u += gridDim.x, ++lu) {
        const int mt = u / p.n_groups;
        const int ng = u - mt * p.n_groups;
        if (!mbar_wait(a_empty, (lu & 1) ^ 1, abort_flag, p.err, DSA_DEVERR_GEMM_WAIT)) break;
        mbar_arrive_expect_tx(a_full, KB * kBox);
        for (int kb = 0; kb < KB; ++kb)
          tma_load_2d(smem + kQOffA + kb * kBox, &tm_a, kb * 64, mt * kBM, a_full);
        for (int j = 0; j < kQGroup; ++j, ++g) {
          const int nt = ng * kQGroup + j;
          if (nt >= p.n_tiles) break;
          const int bs = g & 1;
          if (!mbar_wait(&b_empty[bs], ((g >> 1) & 1) ^ 1, abort_flag, p.err,
                         DSA_DEVERR_GEMM_WAIT)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&b_full[bs], KB * kQBBox);
          for (int kb = 0; kb < KB; ++kb)
            tma_load_2d(smem + kQOffB + (bs * (kQMaxK / 64) + kb) * kQBBox, &tm_b, kb * 64,
                        nt * kQBN, &b_full[bs]);
        }
      }
      // Teardown: the last loads land before the CTA exits.
      if (lu > 0) mbar_drain(a_full, (lu - 1) & 1);
      for (int i = (g > 2 ? g - 2 : 0); i < g; ++i) mbar_drain(&b_full[i & 1], (i >> 1) & 1);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_bf16_f32(128, kQBN, 0, 0);
      const uint32_t a_base = smem_u32(smem + kQOffA);
      const uint32_t b_base = smem_u32(smem + kQOffB);
      int lu = 0, g = 0;
      bool ok = true;
      for (int u = blockIdx.x; ok && u < p.units; u += gridDim.x, ++lu) {
        const int ng = u % p.n_groups;
        if (!mbar_wait(a_full, lu & 1, abort_flag, p.err, DSA_DEVERR_GEMM_WAIT)) break;
        for (int j = 0; j < kQGroup; ++j, ++g) {
          const int nt = ng * kQGroup + j;
          if (nt >= p.n_tiles) break;
          const int bs = g & 1;
          if (!mbar_wait(&b_full[bs], (g >> 1) & 1, abort_flag, p.err, DSA_DEVERR_GEMM_WAIT) ||
              !mbar_wait(acc_empty, (g & 1) ^ 1, abort_flag, p.err, DSA_DEVERR_GEMM_WAIT)) {
            ok = false;
            break;
          }
          tc_fence_after();
          for (int ks = 0; ks < p.K / 16; ++ks) {
            const int kb = ks >> 2;
            const uint32_t koff = static_cast<uint32_t>(ks & 3) * 32u;
            const uint64_t ad = make_smem_desc(a_base + kb * kBox + koff, 16u, 1024u, kLayoutSW128);
            const uint64_t bd = make_smem_desc(
                b_base + (bs * (kQMaxK / 64) + kb) * kQBBox + koff, 16u, 1024u, kLayoutSW128);
            const uint32_t chunk = static_cast<uint32_t>(ks / (kKC / 16));
            umma_bf16(tmem + chunk * kQBN, ad, bd, idesc, (ks % (kKC / 16)) != 0 ? 1u : 0u);
          }
          umma_commit(acc_full);
        }
      }
      // Teardown: the last commit covers every MMA this thread issued.
      if (g > 0) mbar_drain(acc_full, (g - 1) & 1);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int ew = warp - 2;               // 0..3
    const int t = threadIdx.x - 64;        // 0..127
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;   // row of the tile = TMEM lane
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    uint32_t* queue = reinterpret_cast<uint32_t*>(smem + kQOffQueue) + ew * kQQueueCap;
    float* nb = reinterpret_cast<float*>(smem + kQOffNB);
    const uint8_t* a_smem = smem + kQOffA;
    const int half_rd = p.rope_dim / 2;
    const int rope_c0 = kQBN - p.rope_dim;
    bool ok = true;
    int lu = 0, g = 0;
    float na = 0.f;
    for (int u = blockIdx.x; u < p.units; u += gridDim.x, ++lu) {
      const int mt = u / p.n_groups;
      const int ng = u - mt * p.n_groups;
      const int m0 = mt * kBM;
      const bool row_valid = (m0 + row) < p.M;
      ok = __all_sync(0xFFFFFFFFu, mbar_wait(a_full, lu & 1, abort_flag, p.err,
                                             DSA_DEVERR_GEMM_WAIT));
      if (ok) {
        float ss = 0.f;
        for (int kb = 0; kb < KB; ++kb) {
#pragma unroll
          for (int ch = 0; ch < 8; ++ch) {
            const uint4 v =
                *reinterpret_cast<const uint4*>(a_smem + kb * kBox + sw128_off(row, ch));
            const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float lo = bf16lo_to_f32(w4[e]), hi = bf16hi_to_f32(w4[e]);
              ss = fmaf(lo, lo, ss);
              ss = fmaf(hi, hi, ss);
            }
          }
        }
        na = norm_upper(ss, p.K);
      }
      int pos = static_cast<int>((static_cast<int64_t>(m0 + row)) % p.seqlen);
      for (int j = 0; j < kQGroup; ++j, ++g) {
        const int nt = ng * kQGroup + j;
        if (nt >= p.n_tiles) break;
        const int bs = g & 1;
        const uint8_t* b_smem = smem + kQOffB + bs * (kQMaxK / 64) * kQBBox;
        uint8_t* stage = smem + kQOffOut + (g & 1) * kBox;
        ok = ok && __all_sync(0xFFFFFFFFu, mbar_wait(&b_full[bs], (g >> 1) & 1, abort_flag,
                                                     p.err, DSA_DEVERR_GEMM_WAIT));
        if (ok && t < kQBN) {
          float ss = 0.f;
          for (int kb = 0; kb < KB; ++kb) {
#pragma unroll
            for (int ch = 0; ch < 8; ++ch) {
              const uint4 v =
                  *reinterpret_cast<const uint4*>(b_smem + kb * kQBBox + sw128_off(t, ch));
              const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float lo = bf16lo_to_f32(w4[e]), hi = bf16hi_to_f32(w4[e]);
                ss = fmaf(lo, lo, ss);
                ss = fmaf(hi, hi, ss);
              }
            }
          }
          nb[t] = norm_upper(ss, p.K);
        }
        // The store that last used this staging buffer (two n-tiles ago) has read it.
        if (t == 0) bulk_wait_group_read<1>();
        if (!named_bar_and(1, 128, ok)) {
          ok = false;
          break;
        }
        ok = __all_sync(0xFFFFFFFFu, mbar_wait(acc_full, g & 1, abort_flag, p.err,
                                               DSA_DEVERR_GEMM_WAIT));
        uint64_t flagged = 0;
        if (ok) {
          tc_fence_after();
#pragma unroll
          for (int grp = 0; grp < 2; ++grp) {
            float acc[32];
            {
              uint32_t r[32];
              tmem_ld_32x32b_x32(tmem + lane_off + static_cast<uint32_t>(grp * 32), r);
#pragma unroll
              for (int i = 0; i < 32; ++i) acc[i] = __uint_as_float(r[i]);
            }
            for (int c = 1; c < nch; ++c) {
              uint32_t r[32];
              tmem_ld_32x32b_x32(
                  tmem + lane_off + static_cast<uint32_t>(c * kQBN + grp * 32), r);
#pragma unroll
              for (int i = 0; i < 32; ++i) acc[i] = __fadd_rn(acc[i], __uint_as_float(r[i]));
            }
            const float ea = p.gamma * na;
#pragma unroll
            for (int q8 = 0; q8 < 4; ++q8) {
              uint32_t packed[4];
#pragma unroll
              for (int e = 0; e < 8; e += 2) {
                const int col0 = grp * 32 + q8 * 8 + e;
                uint32_t b0 = 0, b1 = 0;
                const bool c0 = certified_bf16(acc[q8 * 8 + e], ea * nb[col0], &b0);
                const bool c1 = certified_bf16(acc[q8 * 8 + e + 1], ea * nb[col0 + 1], &b1);
                if (!c0 && row_valid) flagged |= 1ull << col0;
                if (!c1 && row_valid) flagged |= 1ull << (col0 + 1);
                packed[e >> 1] = (b0 & 0xFFFFu) | (b1 << 16);
              }
              const int chunk16 = grp * 4 + q8;
              st_shared_v4(smem_u32(stage) + sw128_off(row, chunk16), packed[0], packed[1],
                           packed[2], packed[3]);
            }
          }
          tc_fence_before();
          mbar_arrive(acc_empty);
        }
        // Exact recomputation of the uncertain elements: gather this warp's
        // (row, col) list, then one lane per element.
        if (ok) {
          const int cnt = __popcll(flagged);
          int incl = cnt;
#pragma unroll
          for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(0xFFFFFFFFu, incl, o);
            if (lane >= o) incl += v;
          }
          const int total = __shfl_sync(0xFFFFFFFFu, incl, 31);
          int w = incl - cnt;
          uint64_t f = flagged;
          while (f) {
            const int col = __ffsll(static_cast<long long>(f)) - 1;
            f &= f - 1;
            queue[w++] = static_cast<uint32_t>((row << 8) | col);
          }
          __syncwarp();
          for (int i = lane; i < total; i += 32) {
            const uint32_t e = queue[i];
            const int r = static_cast<int>(e >> 8), c = static_cast<int>(e & 0xFF);
            const uint32_t bits = exact_dot_sw128(a_smem, r, kBox, b_smem, c, kQBBox, p.K);
            uint16_t* dst = reinterpret_cast<uint16_t*>(stage + sw128_off(r, c >> 3)) + (c & 7);
            *dst = static_cast<uint16_t>(bits);
          }
          __syncwarp();
          // RoPE on the last rope_dim columns of the head, fp32 non-fused,
          // one rounding (reference/task2_v0_ref.py:93-104).
          if (half_rd > 0 && row_valid) {
            const float* ct = p.cos_tab + static_cast<int64_t>(pos) * half_rd;
            const float* st = p.sin_tab + static_cast<int64_t>(pos) * half_rd;
            for (int c8 = rope_c0 >> 3; c8 < (kQBN >> 3); ++c8) {
              uint4* addr = reinterpret_cast<uint4*>(stage + sw128_off(row, c8));
              uint4 v = *addr;
              uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const int col = c8 * 8 + 2 * e;
                if (col < rope_c0) continue;
                const int pi = (col - rope_c0) >> 1;
                const float re = bf16lo_to_f32(w4[e]), im = bf16hi_to_f32(w4[e]);
                const float c = __ldg(ct + pi), s = __ldg(st + pi);
                const float nre = __fsub_rn(__fmul_rn(re, c), __fmul_rn(im, s));
                const float nim = __fadd_rn(__fmul_rn(re, s), __fmul_rn(im, c));
                w4[e] = f32_to_bf16_rne(nre) | (f32_to_bf16_rne(nim) << 16);
              }
              *addr = make_uint4(w4[0], w4[1], w4[2], w4[3]);
            }
          }
          fence_proxy_async_smem();
        }
        if (!named_bar_and(1, 128, ok)) {
          ok = false;
          break;
        }
        if (t == 0) {
          tma_store_2d(&tm_q, stage, nt * kQBN, m0);
          bulk_commit_group();
          mbar_arrive(&b_empty[bs]);
        }
      }
      if (!ok) break;
      if (t == 0) mbar_arrive(a_empty);
    }
    if (t == 0) bulk_wait_group<0>();
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ------------------------------------------------------------------ w proj
constexpr int kWBN = 16;
constexpr int kWMaxK = 1024;
constexpr int kWStages = 4;
constexpr int kWThreads = 192;
constexpr int kWBBox = kWBN * 128;  // 2 KB: 16 rows x 64 bf16
constexpr int kWOffA = 0;
constexpr int kWOffB = kWOffA + kWStages * kBox;               // 65536
constexpr int kWOffNB = kWOffB + (kWMaxK / 64) * kWBBox;       // 98304
constexpr int kWQueueCap = 512;                                // per warp
constexpr int kWOffQueue = kWOffNB + kWBN * 4;
constexpr int kWOffBar = kWOffQueue + 4 * kWQueueCap * 4;
constexpr int kWNumBars = 2 * kWStages + 3;
constexpr int kWOffMisc = kWOffBar + kWNumBars * 8;
constexpr int kWSmem = kWOffMisc + 16 + 1024;

struct WParams {
  int M;
  int K;  // dim, multiple of 64, <= 1024
  int m_tiles;
  float gamma;
  float scale;
  const uint16_t* x;  // for the exact recomputation
  uint16_t* w_out;
  unsigned int* err;
};

__global__ void __launch_bounds__(kWThreads, 1)
    wproj_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                 const WParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kWOffBar);
  uint64_t* full = bars;                  // [stages]
  uint64_t* empty = bars + kWStages;      // [stages]: MMA commit + 128 epilogue threads
  uint64_t* b_full = bars + 2 * kWStages;
  uint64_t* acc_full = b_full + 1;
  uint64_t* acc_empty = b_full + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + kWOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kWOffMisc + 4);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int KB = p.K / 64;
  const int nch = p.K / kKC;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kWStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1 + 128);
    }
    mbar_init(b_full, 1);
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, 128);
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
    if (lane == 0) {
      mbar_arrive_expect_tx(b_full, KB * kWBBox);
      for (int kb = 0; kb < KB; ++kb)
        tma_load_2d(smem + kWOffB + kb * kWBBox, &tm_b, kb * 64, 0, b_full);
      int it = 0;
      bool ok = true;
      for (int mt = blockIdx.x; ok && mt < p.m_tiles; mt += gridDim.x) {
        for (int kb = 0; kb < KB; ++kb, ++it) {
          const int s = it % kWStages;
          if (!mbar_wait(&empty[s], ((it / kWStages) & 1) ^ 1, abort_flag, p.err,
                         DSA_DEVERR_GEMM_WAIT)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[s], kBox);
          tma_load_2d(smem + kWOffA + s * kBox, &tm_a, kb * 64, mt * kBM, &full[s]);
        }
      }
      mbar_drain(b_full, 0);
      for (int i = (it > kWStages ? it - kWStages : 0); i < it; ++i)
        mbar_drain(&full[i % kWStages], (i / kWStages) & 1);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_bf16_f32(128, kWBN, 0, 0);
      const uint32_t a_base = smem_u32(smem + kWOffA);
      const uint32_t b_base = smem_u32(smem + kWOffB);
      int it = 0, lt = 0;
      bool ok = mbar_wait(b_full, 0, abort_flag, p.err, DSA_DEVERR_GEMM_WAIT);
      for (int mt = blockIdx.x; ok && mt < p.m_tiles; mt += gridDim.x, ++lt) {
        if (!mbar_wait(acc_empty, (lt & 1) ^ 1, abort_flag, p.err, DSA_DEVERR_GEMM_WAIT)) break;
        tc_fence_after();
        for (int kb = 0; kb < KB; ++kb, ++it) {
          const int s = it % kWStages;
          if (!mbar_wait(&full[s], (it / kWStages) & 1, abort_flag, p.err,
                         DSA_DEVERR_GEMM_WAIT)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int k4 = 0; k4 < 4; ++k4) {
            const uint64_t ad = make_smem_desc(a_base + s * kBox + k4 * 32, 16u, 1024u, kLayoutSW128);
            const uint64_t bd =
                make_smem_desc(b_base + kb * kWBBox + k4 * 32, 16u, 1024u, kLayoutSW128);
            const int ks = kb * 4 + k4;
            const uint32_t chunk = static_cast<uint32_t>(ks / (kKC / 16));
            umma_bf16(tmem + chunk * kWBN, ad, bd, idesc, (ks % (kKC / 16)) != 0 ? 1u : 0u);
          }
          umma_commit(&empty[s]);
        }
        if (!ok) break;
        umma_commit(acc_full);
      }
      if (lt > 0) mbar_drain(acc_full, (lt - 1) & 1);
    }
  } else {
    const int ew = warp - 2;
    const int t = threadIdx.x - 64;
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    uint32_t* queue = reinterpret_cast<uint32_t*>(smem + kWOffQueue) + ew * kWQueueCap;
    float* nb = reinterpret_cast<float*>(smem + kWOffNB);
    const uint8_t* b_smem = smem + kWOffB;
    bool ok = __all_sync(0xFFFFFFFFu, mbar_wait(b_full, 0, abort_flag, p.err,
                                                DSA_DEVERR_GEMM_WAIT));
    if (ok && t < kWBN) {
      float ss = 0.f;
      for (int kb = 0; kb < KB; ++kb) {
#pragma unroll
        for (int ch = 0; ch < 8; ++ch) {
          const uint4 v =
              *reinterpret_cast<const uint4*>(b_smem + kb * kWBBox + sw128_off(t, ch));
          const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float lo = bf16lo_to_f32(w4[e]), hi = bf16hi_to_f32(w4[e]);
            ss = fmaf(lo, lo, ss);
            ss = fmaf(hi, hi, ss);
          }
        }
      }
      nb[t] = norm_upper(ss, p.K);
    }
    ok = named_bar_and(1, 128, ok);
    int it = 0, lt = 0;
    for (int mt = blockIdx.x; ok && mt < p.m_tiles; mt += gridDim.x, ++lt) {
      const int m0 = mt * kBM;
      const bool row_valid = (m0 + row) < p.M;
      // Row norm of x from every stage before it is released.
      float ss = 0.f;
      for (int kb = 0; kb < KB; ++kb, ++it) {
        const int s = it % kWStages;
        ok = __all_sync(0xFFFFFFFFu, mbar_wait(&full[s], (it / kWStages) & 1, abort_flag, p.err,
                                               DSA_DEVERR_GEMM_WAIT));
        if (!ok) break;
        const uint8_t* a = smem + kWOffA + s * kBox;
#pragma unroll
        for (int ch = 0; ch < 8; ++ch) {
          const uint4 v = *reinterpret_cast<const uint4*>(a + sw128_off(row, ch));
          const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float lo = bf16lo_to_f32(w4[e]), hi = bf16hi_to_f32(w4[e]);
            ss = fmaf(lo, lo, ss);
            ss = fmaf(hi, hi, ss);
          }
        }
        mbar_arrive(&empty[s]);
      }
      if (!named_bar_and(1, 128, ok)) break;
      const float na = norm_upper(ss, p.K);
      ok = __all_sync(0xFFFFFFFFu, mbar_wait(acc_full, lt & 1, abort_flag, p.err,
                                             DSA_DEVERR_GEMM_WAIT));
      uint32_t flagged = 0;
      uint32_t bits[kWBN];
      if (ok) {
        tc_fence_after();
        float acc[kWBN];
        {
          uint32_t r[16];
          tmem_ld_32x32b_x16(tmem + lane_off, r);
#pragma unroll
          for (int i = 0; i < kWBN; ++i) acc[i] = __uint_as_float(r[i]);
        }
        for (int c = 1; c < nch; ++c) {
          uint32_t r[16];
          tmem_ld_32x32b_x16(tmem + lane_off + static_cast<uint32_t>(c * kWBN), r);
#pragma unroll
          for (int i = 0; i < kWBN; ++i) acc[i] = __fadd_rn(acc[i], __uint_as_float(r[i]));
        }
        tc_fence_before();
        mbar_arrive(acc_empty);
        const float ea = p.gamma * na;
#pragma unroll
        for (int i = 0; i < kWBN; ++i) {
          bits[i] = 0;
          if (!certified_bf16(acc[i], ea * nb[i], &bits[i]) && row_valid) flagged |= 1u << i;
        }
        // Exact recomputation of uncertain elements, one lane per element;
        // the x row is re-read from global memory (L2).
        const int cnt = __popc(flagged);
        int incl = cnt;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int v = __shfl_up_sync(0xFFFFFFFFu, incl, o);
          if (lane >= o) incl += v;
        }
        const int total = __shfl_sync(0xFFFFFFFFu, incl, 31);
        int wpos = incl - cnt;
        uint32_t f = flagged;
        while (f) {
          const int col = __ffs(static_cast<int>(f)) - 1;
          f &= f - 1;
          queue[wpos++] = static_cast<uint32_t>((row << 8) | col);
        }
        __syncwarp();
        for (int i = lane; i < total; i += 32) {
          const uint32_t e = queue[i];
          const int r = static_cast<int>(e >> 8), c = static_cast<int>(e & 0xFF);
          const uint16_t* xr = p.x + static_cast<int64_t>(m0 + r) * p.K;
          double acc64 = 0.0;
          for (int kb = 0; kb < KB; ++kb) {
#pragma unroll
            for (int ch = 0; ch < 8; ++ch) {
              const uint4 av = __ldg(reinterpret_cast<const uint4*>(xr + kb * 64 + ch * 8));
              const uint4 bv =
                  *reinterpret_cast<const uint4*>(b_smem + kb * kWBBox + sw128_off(c, ch));
              const uint32_t aw[4] = {av.x, av.y, av.z, av.w};
              const uint32_t bw[4] = {bv.x, bv.y, bv.z, bv.w};
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                acc64 = fma(static_cast<double>(bf16lo_to_f32(aw[q])),
                            static_cast<double>(bf16lo_to_f32(bw[q])), acc64);
                acc64 = fma(static_cast<double>(bf16hi_to_f32(aw[q])),
                            static_cast<double>(bf16hi_to_f32(bw[q])), acc64);
              }
            }
          }
          queue[i] = (e & 0xFFFFu) | (round_f64_to_bf16(acc64) << 16);
        }
        __syncwarp();
        for (int i = 0; i < total; ++i) {
          const uint32_t e = queue[i];
          if (static_cast<int>((e >> 8) & 0xFF) == row) {
            const uint32_t c = e & 0xFFu;
#pragma unroll
            for (int j = 0; j < kWBN; ++j)
              if (static_cast<uint32_t>(j) == c) bits[j] = e >> 16;
          }
        }
        __syncwarp();
        if (row_valid) {
          uint32_t o[kWBN / 2];
#pragma unroll
          for (int i = 0; i < kWBN; i += 2) {
            const uint32_t lo = f32_to_bf16_rne(__fmul_rn(__uint_as_float(bits[i] << 16), p.scale));
            const uint32_t hi =
                f32_to_bf16_rne(__fmul_rn(__uint_as_float(bits[i + 1] << 16), p.scale));
            o[i >> 1] = lo | (hi << 16);
          }
          uint4* dst = reinterpret_cast<uint4*>(p.w_out + static_cast<int64_t>(m0 + row) * kWBN);
          dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
          dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
        }
      }
      if (!named_bar_and(1, 128, ok)) break;
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

int set_smem_attr(const void* fn, int bytes, bool* done, int dev) {
  if (done[dev]) return DSA_OK;
  const int st = cuda_status(
      cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  if (st == DSA_OK) done[dev] = true;
  return st;
}

}  // namespace ixp

int launch_qproj_rope(const void* qr, const void* wq, const float* cos_tab, const float* sin_tab,
                      void* q_out, int64_t rows, int K, int n_heads, int rope_dim, int64_t seqlen,
                      cudaStream_t stream) {
  using namespace ixp;
  DeviceInfo di;
  int st = current_device_info(&di);
  if (st != DSA_OK) return st;
  if (di.max_smem_optin < kQSmem) return DSA_ERR_UNSUPPORTED;
  unsigned int* err = nullptr;
  st = device_error_word(&err);
  if (st != DSA_OK) return st;
  const int N = n_heads * kQBN;
  CUtensorMap tm_a, tm_b, tm_q;
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(rows)};
    const uint64_t strides[1] = {static_cast<uint64_t>(K) * 2};
    const uint32_t box[2] = {64, kBM};
    st = encode_tensor_map(&tm_a, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, qr, dims, strides, box,
                           CU_TENSOR_MAP_SWIZZLE_128B);
    if (st != DSA_OK) return st;
  }
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(N)};
    const uint64_t strides[1] = {static_cast<uint64_t>(K) * 2};
    const uint32_t box[2] = {64, kQBN};
    st = encode_tensor_map(&tm_b, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, wq, dims, strides, box,
                           CU_TENSOR_MAP_SWIZZLE_128B);
    if (st != DSA_OK) return st;
  }
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(N), static_cast<uint64_t>(rows)};
    const uint64_t strides[1] = {static_cast<uint64_t>(N) * 2};
    const uint32_t box[2] = {64, kBM};
    st = encode_tensor_map(&tm_q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, q_out, dims, strides, box,
                           CU_TENSOR_MAP_SWIZZLE_128B);
    if (st != DSA_OK) return st;
  }
  QParams p;
  p.M = static_cast<int>(rows);
  p.K = K;
  p.n_tiles = n_heads;
  p.m_tiles = static_cast<int>((rows + kBM - 1) / kBM);
  p.n_groups = (n_heads + kQGroup - 1) / kQGroup;
  p.units = p.m_tiles * p.n_groups;
  p.rope_dim = rope_dim;
  p.seqlen = seqlen;
  p.gamma = gamma_for(K / kKC);
  p.cos_tab = cos_tab;
  p.sin_tab = sin_tab;
  p.err = err;
  static bool attr_done[64] = {false};
  st = set_smem_attr(reinterpret_cast<const void*>(qproj_rope_kernel), kQSmem, attr_done,
                     di.device);
  if (st != DSA_OK) return st;
  const int grid = p.units < di.num_sms ? p.units : di.num_sms;
  qproj_rope_kernel<<<grid, kQThreads, kQSmem, stream>>>(tm_a, tm_b, tm_q, p);
  return cuda_status(cudaGetLastError());
}

int launch_wproj(const void* x, const void* wp, void* w_out, int64_t rows, int K, float scale,
                 cudaStream_t stream) {
  using namespace ixp;
  DeviceInfo di;
  int st = current_device_info(&di);
  if (st != DSA_OK) return st;
  if (di.max_smem_optin < kWSmem) return DSA_ERR_UNSUPPORTED;
  unsigned int* err = nullptr;
  st = device_error_word(&err);
  if (st != DSA_OK) return st;
  CUtensorMap tm_a, tm_b;
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(rows)};
    const uint64_t strides[1] = {static_cast<uint64_t>(K) * 2};
    const uint32_t box[2] = {64, kBM};
    st = encode_tensor_map(&tm_a, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, x, dims, strides, box,
                           CU_TENSOR_MAP_SWIZZLE_128B);
    if (st != DSA_OK) return st;
  }
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(kWBN)};
    const uint64_t strides[1] = {static_cast<uint64_t>(K) * 2};
    const uint32_t box[2] = {64, kWBN};
    st = encode_tensor_map(&tm_b, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, wp, dims, strides, box,
                           CU_TENSOR_MAP_SWIZZLE_128B);
    if (st != DSA_OK) return st;
  }
  WParams p;
  p.M = static_cast<int>(rows);
  p.K = K;
  p.m_tiles = static_cast<int>((rows + kBM - 1) / kBM);
  p.gamma = gamma_for(K / kKC);
  p.scale = scale;
  p.x = static_cast<const uint16_t*>(x);
  p.w_out = static_cast<uint16_t*>(w_out);
  p.err = err;
  static bool attr_done[64] = {false};
  st = set_smem_attr(reinterpret_cast<const void*>(wproj_kernel), kWSmem, attr_done, di.device);
  if (st != DSA_OK) return st;
  const int grid = p.m_tiles < di.num_sms ? p.m_tiles : di.num_sms;
  wproj_kernel<<<grid, kWThreads, kWSmem, stream>>>(tm_a, tm_b, p);
  return cuda_status(cudaGetLastError());
}

}  // namespace dsa
