// Lightning Indexer q projection for sm_100a, with correctly rounded bf16 outputs.
//
//   q = RoPE(bf16(qr . wq_b^T))          reference/task2_v0_ref.py:129-131
//
// (the w projection, w = bf16(bf16(x . w_proj^T) * scale), is in
// indexer_wproj.cu). A tcgen05 GEMM (TMA -> SW128 smem -> UMMA -> TMEM) whose
// epilogue certifies the bf16 rounding of the exact dot product against an
// error bound and leaves the few uncertain elements to an exact fix-up before
// applying RoPE.
//
// q projection kernel (one CTA per SM, persistent): exact int8 slice products
//   (see below). Work unit = (128-row M tile, 4 heads); the A slices
//   (3 x 128 x K int8, K <= 256) stay resident in smem for the unit, the B
//   slices of each head (3 x 64 rows) stream through a 3-stage ring, one
//   128-wide k atom per stage; TMEM holds two buffers of 4 level accumulators
//   of 64 columns, one per epilogue warpgroup (alternate heads).
//   warp 0 TMA, warp 1 MMA, warps 2..9 epilogue (two warpgroups, one thread
//   per row).
#include "common.cuh"
#include "host_util.h"
#include "numerics.cuh"

namespace dsa {
namespace ixp {

constexpr int kBM = 128;
constexpr int kBox = kBM * 128;  // 128 rows x 64 bf16 = 16 KB
constexpr uint32_t kTmemCols = 512;

// ------------------------------------------------------------------ q proj
// Exact slicing on the int8 tensor cores (Ozaki scheme). qr rows and wq_b rows
// are cut into three signed 7-bit slices each (indexer_split.cu):
//   a = 2^(sa-7) A1 + 2^(sa-14) A2 + 2^(sa-21) A3 + ra   (same for b).
// The slice products A_i.B_j with i + j <= 5 accumulate EXACTLY in int32 TMEM
// accumulators, one per level s = i + j (L2..L5):
//   a.b = 2^(sa+sb) (L2 2^-14 + L3 2^-21 + L4 2^-28 + L5 2^-35) + d,
//   |d| <= 2^(sa+sb) (err_a + err_b + 2^-42 ||A3|| ||B3||)
// (remainders, and the A3.B3 product by Cauchy-Schwarz). The epilogue
// evaluates T = H + G 2^-14 (H = 128 L2 + L3 and G = 128 L4 + L5 are exact
// int32) in fp32 with a rigorous error bound and certifies the bf16 rounding of
// T (numerics.cuh); the exponent sa+sb-21 is then added to the bf16 bits, which
// is exact for normal results (checked per row and tile). Elements it cannot
// certify are marked in a bitmask and recomputed afterwards by
// qproj_fixup_kernel as the sequential fp64 dot product of the bf16 inputs, the
// CPU oracle's arithmetic (both columns of a RoPE pair, so that the rotation
// sees final values).
//
// MMA shape: the three B slices of a tile sit one after another in smem
// ([B1; B2; B3], 64 rows each), and the level accumulators 64 TMEM columns
// apart, so one MMA of A_i against the stacked B (N = 192) adds A_i.B1,
// A_i.B2, A_i.B3 into levels i+1, i+2, i+3 at once: three MMAs per 32-wide k
// step instead of eight.
constexpr int kQBN = 64;                  // one head per tile
constexpr int kQMaxK = 256;
constexpr int kQGroup = 4;                // tiles (heads) per unit
constexpr int kQThreads = 320;
constexpr int kQStages = 3;
constexpr int kQSlices = 3;
constexpr int kQKAtoms = kQMaxK / 128;                         // 128 int8 k per SW128 row
constexpr int kQABox = kBM * 128;                              // 16 KB: 128 rows x 128 k
constexpr int kQBBox = kQBN * 128;                             // 8 KB: 64 rows x 128 k
constexpr int kQOffA = 0;                                      // [slice][k atom]
constexpr int kQOffB = kQOffA + kQSlices * kQKAtoms * kQABox;  // 98304
constexpr int kQStageBytes = kQSlices * kQBBox;                // 24576: [B1; B2; B3], one k atom
constexpr int kQOffOut = kQOffB + kQStages * kQStageBytes;     // 172032: [2] x 16 KB
constexpr int kQMaxHeads = 16;
constexpr int kQOffCol = kQOffOut + 2 * kBox;                  // 204800: sb[N]
constexpr int kQOffColExt = kQOffCol + kQMaxHeads * kQBN * 4;  // 208896: [head][4]
constexpr int kQOffBar = kQOffColExt + kQMaxHeads * 4 * 4;     // 209152
constexpr int kQNumBars = 2 + 2 * kQStages + 4;
constexpr int kQOffMisc = kQOffBar + kQNumBars * 8;
constexpr int kQSmem = kQOffMisc + 16 + 1024;
constexpr uint32_t kQBufCols = 256;                            // 4 levels x 64 per buffer
constexpr int kQRopeRegs = 16;                                 // rope pairs kept in registers

struct QParams {
  int M;           // rows (tokens)
  int K;           // q_lora_rank, multiple of 64, <= 256
  int n_tiles;     // heads
  int m_tiles;
  int units;       // m_tiles * n_groups
  int n_groups;
  int rope_dim;    // even, <= 64
  int64_t seqlen;  // row r is at position r % seqlen of cos/sin
  const float* cos_tab;
  const float* sin_tab;
  const int* a_sig;       // [M]
  const float* a_err;     // [M]
  const float* a_n3;      // [M]
  const int* b_sig;       // [N]
  const float* b_err;     // [N]
  const float* b_n3;      // [N]
  uint32_t* open_bits;    // [M, N / 32]: elements left to qproj_fixup_kernel
  unsigned int* err;
};

__device__ __forceinline__ uint32_t sw128_off(int row, int chunk16) {
  return static_cast<uint32_t>(row * 128 + ((chunk16 ^ (row & 7)) << 4));
}

// RoPE of one (re, im) pair, fp32 non-fused, one rounding per output
// (reference/task2_v0_ref.py:93-104); returns the two bf16 packed.
__device__ __forceinline__ uint32_t rope_pair(uint32_t w, float c, float sn) {
  const float re = bf16lo_to_f32(w), im = bf16hi_to_f32(w);
  const float nre = __fsub_rn(__fmul_rn(re, c), __fmul_rn(im, sn));
  const float nim = __fadd_rn(__fmul_rn(re, sn), __fmul_rn(im, c));
  return f32_to_bf16_rne(nre) | (f32_to_bf16_rne(nim) << 16);
}

__global__ void __launch_bounds__(kQThreads, 1)
    qproj_rope_kernel(const __grid_constant__ CUtensorMap tm_a,  // int8 [3][M][K]
                      const __grid_constant__ CUtensorMap tm_b,  // int8 [3][N][K]
                      const __grid_constant__ CUtensorMap tm_q,  // bf16 [M][N]
                      const QParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kQOffBar);
  uint64_t* a_full = bars + 0;     // TMA landed the unit's A slices
  uint64_t* a_empty = bars + 1;    // the unit's MMAs are done with them
  uint64_t* b_full = bars + 2;     // [kQStages]
  uint64_t* b_empty = b_full + kQStages;
  uint64_t* acc_full = b_empty + kQStages;  // [2], one per epilogue warpgroup
  uint64_t* acc_empty = acc_full + 2;       // [2], 128 arrivals
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + kQOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kQOffMisc + 4);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int ksteps = p.K / 32;
  const int katoms = (p.K + 127) / 128;

  if (threadIdx.x == 0) {
    mbar_init(a_full, 1);
    mbar_init(a_empty, 1);
    for (int i = 0; i < kQStages; ++i) {
      mbar_init(&b_full[i], 1);
      mbar_init(&b_empty[i], 1);
    }
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
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int lu = 0, it = 0;
      bool ok = true;
      for (int u = blockIdx.x; ok && u < p.units; u += gridDim.x, ++lu) {
        const int mt = u / p.n_groups;
        const int ng = u - mt * p.n_groups;
        if (!mbar_wait(a_empty, (lu & 1) ^ 1, abort_flag, p.err, DSA_DEVERR_GEMM_WAIT)) break;
        mbar_arrive_expect_tx(a_full, kQSlices * katoms * kQABox);
        for (int j = 0; j < kQSlices; ++j)
          for (int kb = 0; kb < katoms; ++kb)
            tma_load_3d(smem + kQOffA + (j * kQKAtoms + kb) * kQABox, &tm_a, kb * 128, mt * kBM,
                        j, a_full);
        for (int jn = 0; ok && jn < kQGroup; ++jn) {
          const int nt = ng * kQGroup + jn;
          if (nt >= p.n_tiles) break;
          for (int kb = 0; kb < katoms; ++kb, ++it) {
            const int s = it % kQStages;
            if (!mbar_wait(&b_empty[s], ((it / kQStages) & 1) ^ 1, abort_flag, p.err,
                           DSA_DEVERR_GEMM_WAIT)) {
              ok = false;
              break;
            }
            uint8_t* st = smem + kQOffB + s * kQStageBytes;
            mbar_arrive_expect_tx(&b_full[s], kQStageBytes);
            for (int j = 0; j < kQSlices; ++j)
              tma_load_3d(st + j * kQBBox, &tm_b, kb * 128, nt * kQBN, j, &b_full[s]);
          }
        }
      }
      if (lu > 0) mbar_drain(a_full, (lu - 1) & 1);
      for (int i = (it > kQStages ? it - kQStages : 0); i < it; ++i)
        mbar_drain(&b_full[i % kQStages], (i / kQStages) & 1);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc192 = make_idesc_s8_s32(128, 3 * kQBN);
      constexpr uint32_t idesc128 = make_idesc_s8_s32(128, 2 * kQBN);
      constexpr uint32_t idesc64 = make_idesc_s8_s32(128, kQBN);
      const uint32_t a_base = smem_u32(smem + kQOffA);
      const uint32_t b_base = smem_u32(smem + kQOffB);
      int lu = 0, g = 0, it = 0;
      bool ok = true;
      for (int u = blockIdx.x; ok && u < p.units; u += gridDim.x, ++lu) {
        const int ng = u % p.n_groups;
        if (!mbar_wait(a_full, lu & 1, abort_flag, p.err, DSA_DEVERR_GEMM_WAIT)) break;
        tc_fence_after();
        for (int jn = 0; ok && jn < kQGroup; ++jn, ++g) {
          const int nt = ng * kQGroup + jn;
          if (nt >= p.n_tiles) break;
          const int ab = g & 1;
          if (!mbar_wait(&acc_empty[ab], ((g >> 1) & 1) ^ 1, abort_flag, p.err,
                         DSA_DEVERR_GEMM_WAIT)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d = tmem + static_cast<uint32_t>(ab) * kQBufCols;
          for (int kb = 0; kb < katoms; ++kb, ++it) {
            const int s = it % kQStages;
            if (!mbar_wait(&b_full[s], (it / kQStages) & 1, abort_flag, p.err,
                           DSA_DEVERR_GEMM_WAIT)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t st = b_base + s * kQStageBytes;
            const int nstep = min(4, ksteps - kb * 4);
            for (int step = 0; step < nstep; ++step) {
              const uint32_t ko = static_cast<uint32_t>(step) * 32u;
              const uint32_t a1 = a_base + (0 * kQKAtoms + kb) * kQABox + ko;
              const uint32_t a2 = a_base + (1 * kQKAtoms + kb) * kQABox + ko;
              const uint32_t a3 = a_base + (2 * kQKAtoms + kb) * kQABox + ko;
              const uint64_t da1 = make_smem_desc(a1, 16u, 1024u, kLayoutSW128);
              const uint64_t da2 = make_smem_desc(a2, 16u, 1024u, kLayoutSW128);
              const uint64_t da3 = make_smem_desc(a3, 16u, 1024u, kLayoutSW128);
              const uint64_t db123 = make_smem_desc(st + ko, 16u, 1024u, kLayoutSW128);
              // The A3 product is issued between the other two: after the A2
              // MMA (whose columns it overlaps entirely) the same work ran
              // 1.4x slower, MMA-only. Integer sums: any order is exact.
              if (kb == 0 && step == 0) {
                // first k step: every level's first writer overwrites it
                const uint64_t db3 =
                    make_smem_desc(st + 2 * kQBBox + ko, 16u, 1024u, kLayoutSW128);
                umma_s8(d + 0 * kQBN, da1, db123, idesc192, 0u);  // L2, L3, L4
                umma_s8(d + 3 * kQBN, da2, db3, idesc64, 0u);     // L5
                umma_s8(d + 2 * kQBN, da3, db123, idesc128, 1u);  // L4, L5
                umma_s8(d + 1 * kQBN, da2, db123, idesc128, 1u);  // L3, L4
              } else {
                umma_s8(d + 0 * kQBN, da1, db123, idesc192, 1u);  // L2, L3, L4
                umma_s8(d + 2 * kQBN, da3, db123, idesc128, 1u);  // L4, L5
                umma_s8(d + 1 * kQBN, da2, db123, idesc192, 1u);  // L3, L4, L5
              }
            }
            umma_commit(&b_empty[s]);
          }
          if (!ok) break;
          umma_commit(&acc_full[ab]);
        }
        if (!ok) break;
        umma_commit(a_empty);
      }
      if (g > 0) mbar_drain(&acc_full[(g - 1) & 1], ((g - 1) >> 1) & 1);
      if (g > 1) mbar_drain(&acc_full[(g - 2) & 1], ((g - 2) >> 1) & 1);
      if (lu > 0) mbar_drain(a_empty, (lu - 1) & 1);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int wg = (warp - 2) >> 2;        // warpgroup 0 / 1 = TMEM buffer
    const int ew = warp - 2;               // 0..7
    const int t = threadIdx.x - 64 - wg * 128;  // 0..127 within the warpgroup
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;   // row of the tile = TMEM lane
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t bar_id = 1 + wg;
    const int N = p.n_tiles * kQBN;
    const int words = N / 32;
    int* csig_all = reinterpret_cast<int*>(smem + kQOffCol);
    int* cext = reinterpret_cast<int*>(smem + kQOffColExt);   // [head]: min/max sb, max err, max n3
    {
      // column data of all heads, once per CTA; warp ew takes heads ew, ew + 8
      for (int h = ew; h < p.n_tiles; h += 8) {
        int mn = 1 << 30, mx = -(1 << 30);
        unsigned me = 0, mnb = 0;
        for (int c = lane; c < kQBN; c += 32) {
          const int n = h * kQBN + c;
          const int sb = __ldg(p.b_sig + n);
          const float eb = __ldg(p.b_err + n) * 0x1p21f;
          const float nb = __fmul_ru(__ldg(p.b_n3 + n), 0x1p-21f);
          csig_all[n] = sb;
          mn = min(mn, sb);
          mx = max(mx, sb);
          me = max(me, __float_as_uint(eb));  // non-negative floats order as their bits
          mnb = max(mnb, __float_as_uint(nb));
        }
        mn = __reduce_min_sync(0xFFFFFFFFu, mn);
        mx = __reduce_max_sync(0xFFFFFFFFu, mx);
        me = __reduce_max_sync(0xFFFFFFFFu, me);
        mnb = __reduce_max_sync(0xFFFFFFFFu, mnb);
        if (lane == 0) {
          cext[h * 4 + 0] = mn;
          cext[h * 4 + 1] = mx;
          cext[h * 4 + 2] = static_cast<int>(me);
          cext[h * 4 + 3] = static_cast<int>(mnb);
        }
      }
      named_bar_sync(3, 256);
    }
    uint8_t* stage = smem + kQOffOut + wg * kBox;
    const int half_rd = p.rope_dim / 2;
    const int rope_c0 = kQBN - p.rope_dim;  // first rotated column of the head
    const bool rope_regs = half_rd > 0 && half_rd <= kQRopeRegs && (rope_c0 & 7) == 0;
    // rotated columns of a head as two 32-bit masks
    const uint32_t rope_lo = rope_c0 >= 32 ? 0u : (0xFFFFFFFFu << rope_c0);
    const uint32_t rope_hi = rope_c0 >= 64 ? 0u : rope_c0 >= 32 ? (0xFFFFFFFFu << (rope_c0 - 32))
                                                                 : 0xFFFFFFFFu;
    const uint32_t dbase = tmem + lane_off + static_cast<uint32_t>(wg) * kQBufCols;
    bool ok = true;
    int g = 0;
    for (int u = blockIdx.x; ok && u < p.units; u += gridDim.x) {
      const int mt = u / p.n_groups;
      const int ng = u - mt * p.n_groups;
      const int m0 = mt * kBM;
      const bool row_valid = (m0 + row) < p.M;
      const int sa = row_valid ? __ldg(p.a_sig + m0 + row) : 0;
      const float eaT = row_valid ? __ldg(p.a_err + m0 + row) * 0x1p21f : 0.f;  // exact scaling
      const float na3 = row_valid ? __ldg(p.a_n3 + m0 + row) : 0.f;
      const int ex_row = sa - 21 + 127;
      const uint32_t rsh = static_cast<uint32_t>(sa - 21) << 7;
      const int pos = static_cast<int>(static_cast<int64_t>(m0 + row) % p.seqlen);
      // RoPE tables of this row, once per unit (every head of it rotates the
      // same row), 16-byte loads where the rows allow; loaded per head they
      // cost the kernel 12 of its 64 us
      float rc[kQRopeRegs], rs[kQRopeRegs];
      if (rope_regs && row_valid) {
        const float* ct = p.cos_tab + static_cast<int64_t>(pos) * half_rd;
        const float* stt = p.sin_tab + static_cast<int64_t>(pos) * half_rd;
        if (half_rd == kQRopeRegs &&
            ((reinterpret_cast<uintptr_t>(ct) | reinterpret_cast<uintptr_t>(stt)) & 15) == 0) {
#pragma unroll
          for (int i = 0; i < kQRopeRegs / 4; ++i) {
            const float4 c4 = __ldg(reinterpret_cast<const float4*>(ct) + i);
            const float4 s4 = __ldg(reinterpret_cast<const float4*>(stt) + i);
            rc[4 * i] = c4.x;
            rc[4 * i + 1] = c4.y;
            rc[4 * i + 2] = c4.z;
            rc[4 * i + 3] = c4.w;
            rs[4 * i] = s4.x;
            rs[4 * i + 1] = s4.y;
            rs[4 * i + 2] = s4.z;
            rs[4 * i + 3] = s4.w;
          }
        } else {
#pragma unroll
          for (int i = 0; i < kQRopeRegs; ++i) {
            rc[i] = i < half_rd ? __ldg(ct + i) : 0.f;
            rs[i] = i < half_rd ? __ldg(stt + i) : 0.f;
          }
        }
      }
      for (int jn = 0; ok && jn < kQGroup; ++jn, ++g) {
        const int nt = ng * kQGroup + jn;
        if (nt >= p.n_tiles) break;
        if ((g & 1) != wg) continue;
        const int n0 = nt * kQBN;
        const int* csig = csig_all + n0;
        // per (row, tile): error bound in units of T and the exponent range check
        const int sb_min = cext[nt * 4 + 0], sb_max = cext[nt * 4 + 1];
        const float eb_max = __int_as_float(cext[nt * 4 + 2]);
        const float nb_max = __int_as_float(cext[nt * 4 + 3]);
        // |T - fp32 value| <= 2^-23 |value| + 2^-6 (two conversions, one fma;
        // |G 2^-14| < 2^17), plus the data's remainder and A3.B3 bounds
        const float e_row =
            __fadd_ru(__fmaf_ru(na3, nb_max, __fadd_ru(eaT, eb_max)), 0x1p-5f);
        // a certified T (|T| in [2^-6, 2^31)) scales into a normal bf16 when
        // the biased exponent sa + sb - 21 + 127 stays in [15, 223]
        const bool row_ok = row_valid && ex_row + sb_min >= 15 && ex_row + sb_max <= 223;
        // this warpgroup's previous TMA store has finished reading the staging tile
        if (t == 0) bulk_wait_group_read<0>();
        if (!named_bar_and(bar_id, 128, ok)) {
          ok = false;
          break;
        }
        ok = __all_sync(0xFFFFFFFFu, mbar_wait(&acc_full[wg], (g >> 1) & 1, abort_flag, p.err,
                                               DSA_DEVERR_GEMM_WAIT));
        if (!ok) break;
        tc_fence_after();
        uint32_t open_lo = 0, open_hi = 0;  // columns 0..31 / 32..63 left open
#pragma unroll
        for (int q16 = 0; q16 < 4; ++q16) {
          uint32_t l2[16], l3[16], l4[16], l5[16];
          tmem_ld4_32x32b_x16(dbase + 0 * kQBN + q16 * 16, dbase + 1 * kQBN + q16 * 16,
                              dbase + 2 * kQBN + q16 * 16, dbase + 3 * kQBN + q16 * 16, l2, l3,
                              l4, l5);
          uint32_t packed[8];
          uint32_t open = 0;
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int col = q16 * 16 + i;
            const int H = static_cast<int>(l2[i]) * 128 + static_cast<int>(l3[i]);
            const int G = static_cast<int>(l4[i]) * 128 + static_cast<int>(l5[i]);
            const float T = fmaf(__int2float_rn(G), 0x1p-14f, __int2float_rn(H));
            const float E = __fmaf_ru(fabsf(T), 0x1.000002p-23f, e_row);
            uint32_t pr;
            asm("cvt.rn.bf16x2.f32 %0, %1, %2;"
                : "=r"(pr)
                : "f"(__fadd_ru(T, E)), "f"(__fsub_rd(T, E)));
            open |= static_cast<uint32_t>(((pr ^ (pr >> 16)) & 0xFFFFu) != 0) << i;
            const uint32_t bits = (pr >> 16) + rsh + (static_cast<uint32_t>(csig[col]) << 7);
            if (i & 1) packed[i >> 1] |= bits << 16;
            else packed[i >> 1] = bits & 0xFFFFu;
          }
          if (q16 < 2) open_lo |= open << (16 * (q16 & 1));
          else open_hi |= open << (16 * (q16 & 1));
          const uint32_t sbase = smem_u32(stage);
          st_shared_v4(sbase + sw128_off(row, q16 * 2 + 0), packed[0], packed[1], packed[2],
                       packed[3]);
          st_shared_v4(sbase + sw128_off(row, q16 * 2 + 1), packed[4], packed[5], packed[6],
                       packed[7]);
        }
        tc_fence_before();
        mbar_arrive(&acc_empty[wg]);
        if (!row_ok) open_lo = open_hi = 0xFFFFFFFFu;
        // a rotated pair is finished by the fix-up as a whole
        open_lo |= (((open_lo & 0x55555555u) << 1) | ((open_lo & 0xAAAAAAAAu) >> 1)) & rope_lo;
        open_hi |= (((open_hi & 0x55555555u) << 1) | ((open_hi & 0xAAAAAAAAu) >> 1)) & rope_hi;
        if (row_valid) {
          uint32_t* ob = p.open_bits + static_cast<int64_t>(m0 + row) * words + nt * 2;
          *reinterpret_cast<uint2*>(ob) = make_uint2(open_lo, open_hi);
        }
        // RoPE on the last rope_dim columns of the head, fp32 non-fused, one
        // rounding (reference/task2_v0_ref.py:93-104); open pairs are left to
        // the fix-up.
        if (half_rd > 0 && row_valid) {
          const uint64_t open = (static_cast<uint64_t>(open_hi) << 32) | open_lo;
          if (rope_regs) {
            const int c8_0 = rope_c0 >> 3;
#pragma unroll
            for (int j = 0; j < kQRopeRegs / 4; ++j) {
              if (c8_0 + j < (kQBN >> 3)) {
                uint4* addr = reinterpret_cast<uint4*>(stage + sw128_off(row, c8_0 + j));
                uint4 v = *addr;
                uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  const int col = (c8_0 + j) * 8 + 2 * e;
                  if (!((open >> col) & 1ull))
                    w4[e] = rope_pair(w4[e], rc[4 * j + e], rs[4 * j + e]);
                }
                *addr = make_uint4(w4[0], w4[1], w4[2], w4[3]);
              }
            }
          } else {
            const float* ct = p.cos_tab + static_cast<int64_t>(pos) * half_rd;
            const float* stt = p.sin_tab + static_cast<int64_t>(pos) * half_rd;
            // a chunk's four pairs are four consecutive table entries: one
            // 16-byte load of each table when the chunks and rows line up
            const bool tab_vec =
                (rope_c0 & 7) == 0 && (half_rd & 3) == 0 &&
                ((reinterpret_cast<uintptr_t>(ct) | reinterpret_cast<uintptr_t>(stt)) & 15) == 0;
            for (int c8 = rope_c0 >> 3; c8 < (kQBN >> 3); ++c8) {
              uint4* addr = reinterpret_cast<uint4*>(stage + sw128_off(row, c8));
              uint4 v = *addr;
              uint32_t w4[4] = {v.x, v.y, v.z, v.w};
              if (tab_vec) {
                const int pi0 = (c8 * 8 - rope_c0) >> 1;
                const float4 c4 = __ldg(reinterpret_cast<const float4*>(ct + pi0));
                const float4 s4 = __ldg(reinterpret_cast<const float4*>(stt + pi0));
                const float cv[4] = {c4.x, c4.y, c4.z, c4.w};
                const float sv[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
                for (int e = 0; e < 4; ++e)
                  if (!((open >> (c8 * 8 + 2 * e)) & 1ull)) w4[e] = rope_pair(w4[e], cv[e], sv[e]);
              } else {
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  const int col = c8 * 8 + 2 * e;
                  if (col < rope_c0 || ((open >> col) & 1ull)) continue;
                  const int pi = (col - rope_c0) >> 1;
                  w4[e] = rope_pair(w4[e], __ldg(ct + pi), __ldg(stt + pi));
                }
              }
              *addr = make_uint4(w4[0], w4[1], w4[2], w4[3]);
            }
          }
        }
        fence_proxy_async_smem();
        if (!named_bar_and(bar_id, 128, ok)) {
          ok = false;
          break;
        }
        if (t == 0) {
          tma_store_2d(&tm_q, stage, n0, m0);
          bulk_commit_group();
        }
      }
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

// Fix-up of the elements the projection left open. Warps walk the rows; a row
// with open columns is staged in shared memory and becomes a list of units
// (one open column, or one rotated pair, whose RoPE needs both final values).
// A dot product whose fp64 sum is exact in any order (bit spans of the two
// rows, indexer_split.cu) is split over the warp; the others are summed by one
// lane each in ascending k, the CPU oracle's order -- either way the oracle's
// fp64 value. It is rounded once; a pair then gets its RoPE.
constexpr int kFixWarps = 8;
constexpr int kFixCap = 128;   // units per warp and round
constexpr int kFixRowChunk = 256;  // rows a block scans at a time
constexpr int kFixBlocksPerSm = 4;

struct FixParams {
  int M;
  int K;
  int N;
  int rope_dim;
  int64_t seqlen;
  const uint16_t* qr;     // [M, K]
  const uint16_t* wq;     // [N, K]
  const int* a_sig;       // [M] row exponents (indexer_split.cu)
  const int* b_span;      // [N]
  const float* cos_tab;
  const float* sin_tab;
  const uint32_t* open_bits;  // [M, N / 32]
  uint16_t* q;            // [M, N]
};

// Sequential fp64 dot product, a in shared memory, b from global memory.
__device__ __forceinline__ double dot_f64_seq(const uint4* a, const uint16_t* b, int K) {
  double acc = 0.0;
#pragma unroll 8
  for (int k = 0; k < K; k += 8) {
    const uint4 av = a[k >> 3];
    const uint4 bv = __ldg(reinterpret_cast<const uint4*>(b + k));
    const uint32_t aw[4] = {av.x, av.y, av.z, av.w};
    const uint32_t bw[4] = {bv.x, bv.y, bv.z, bv.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      acc = fma(static_cast<double>(bf16lo_to_f32(aw[q])),
                static_cast<double>(bf16lo_to_f32(bw[q])), acc);
      acc = fma(static_cast<double>(bf16hi_to_f32(aw[q])),
                static_cast<double>(bf16hi_to_f32(bw[q])), acc);
    }
  }
  return acc;
}

// The same sum split over the warp (K <= 256: 8 terms per lane), valid when
// every partial sum is exact; all lanes return it.
__device__ __forceinline__ double dot_f64_warp(const uint4* a, const uint16_t* b, int K,
                                               int lane) {
  double acc = 0.0;
  if (lane * 8 < K) {
    const uint4 av = a[lane];
    const uint4 bv = __ldg(reinterpret_cast<const uint4*>(b) + lane);
    const uint32_t aw[4] = {av.x, av.y, av.z, av.w};
    const uint32_t bw[4] = {bv.x, bv.y, bv.z, bv.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      acc = fma(static_cast<double>(bf16lo_to_f32(aw[q])),
                static_cast<double>(bf16lo_to_f32(bw[q])), acc);
      acc = fma(static_cast<double>(bf16hi_to_f32(aw[q])),
                static_cast<double>(bf16hi_to_f32(bw[q])), acc);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xFFFFFFFFu, acc, o);
  return acc;
}

// rt: the row's RoPE tables (cos at [0, 32), sin at [32, 64)), staged with the row.
__device__ __forceinline__ void fix_store(const FixParams& p, int row, int col, bool pair,
                                          uint32_t v0, uint32_t v1, int rope_c0, const float* rt) {
  uint16_t* dst = p.q + static_cast<int64_t>(row) * p.N + col;
  if (pair) {
    const int pi = ((col % kQBN) - rope_c0) >> 1;
    *reinterpret_cast<uint32_t*>(dst) = rope_pair(v0 | (v1 << 16), rt[pi], rt[32 + pi]);
  } else {
    *dst = static_cast<uint16_t>(v0);
  }
}

__global__ void __launch_bounds__(kFixWarps * 32, kFixBlocksPerSm)
    qproj_fixup_kernel(const FixParams p) {
  __shared__ uint16_t units[kFixWarps][kFixCap];
  __shared__ uint4 arow[kFixWarps][kQMaxK / 8];
  __shared__ float rtab[kFixWarps][64];  // the staged row's cos / sin (rope_dim <= 64)
  __shared__ uint32_t row_seen[kFixRowChunk / 32];
  __shared__ int row_list[kFixRowChunk];
  __shared__ int n_list;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int words = p.N / 32;
  const int rope_c0 = kQBN - p.rope_dim;
  const int log2k = 32 - __clz(p.K - 1);  // ceil(log2 K)
  uint16_t* u = units[warp];
  uint4* a = arow[warp];
  // The block owns a contiguous range of rows. Few rows have open elements, so
  // the whole block first scans the range's bitmask (one round of coalesced
  // loads) and lists those rows; each warp then takes listed rows, so that a
  // row's chain of dependent loads (qr row, weight rows, RoPE tables) is not
  // queued behind other rows' bitmask loads in the same warp.
  const int per_block = static_cast<int>((p.M + gridDim.x - 1) / gridDim.x);
  const int r_begin = blockIdx.x * per_block;
  const int r_end = min(p.M, r_begin + per_block);
  const int hwords = words / 2;  // one uint2 per head
  for (int c0 = r_begin; c0 < r_end; c0 += kFixRowChunk) {
    const int c1 = min(r_end, c0 + kFixRowChunk);
    if (threadIdx.x < kFixRowChunk / 32) row_seen[threadIdx.x] = 0u;
    if (threadIdx.x == 0) n_list = 0;
    __syncthreads();
    const uint2* ob2 =
        reinterpret_cast<const uint2*>(p.open_bits + static_cast<int64_t>(c0) * words);
    const int n2 = (c1 - c0) * hwords;
    for (int i = threadIdx.x; i < n2; i += kFixWarps * 32) {
      const uint2 v = __ldg(ob2 + i);
      if ((v.x | v.y) != 0u) {
        const int r = i / hwords;
        const uint32_t bit = 1u << (r & 31);
        if (!(atomicOr(&row_seen[r >> 5], bit) & bit)) row_list[atomicAdd(&n_list, 1)] = c0 + r;
      }
    }
    __syncthreads();
    const int n_rows = n_list;
    for (int li = warp; li < n_rows; li += kFixWarps) {
      const int row = row_list[li];
      const uint32_t* ob = p.open_bits + static_cast<int64_t>(row) * words;
      bool staged = false;
      int span_a = 0;
      for (int w0 = 0; w0 < words; w0 += 32) {
        const uint32_t bits = (w0 + lane < words) ? __ldg(ob + w0 + lane) : 0u;
        if (!__any_sync(0xFFFFFFFFu, bits != 0)) continue;
        if (!staged) {
          // the row, its exponent and its RoPE tables: independent loads, issued together
          const int sg = __ldg(p.a_sig + row);
          const int half_rd = p.rope_dim / 2;
          const int64_t pos = row % p.seqlen;
          float ct = 0.f, stb = 0.f;
          if (lane < half_rd) {
            ct = __ldg(p.cos_tab + pos * half_rd + lane);
            stb = __ldg(p.sin_tab + pos * half_rd + lane);
          }
          if (lane * 8 < p.K)
            a[lane] = __ldg(reinterpret_cast<const uint4*>(p.qr + static_cast<int64_t>(row) * p.K) +
                            lane);
          rtab[warp][lane] = ct;
          rtab[warp][32 + lane] = stb;
          // the row's bit span (sigma - lowest set bit), from the staged row
          int low = 1 << 30;
          if (lane * 8 < p.K) {
            const uint4 v = a[lane];
            low = min(min(bf16x2_low_bit(v.x), bf16x2_low_bit(v.y)),
                      min(bf16x2_low_bit(v.z), bf16x2_low_bit(v.w)));
          }
          low = __reduce_min_sync(0xFFFFFFFFu, low);
          span_a = sg >= (1 << 20) ? (1 << 20) : (low == (1 << 30) ? 0 : sg - low);
          staged = true;
          __syncwarp();
        }
        // one unit per open non-rotated column and per open rotated pair (even column)
        const int base = (w0 + lane) * 32;
        const bool head_lo = (base % kQBN) == 0;  // the word holds head columns 0..31
        const uint32_t rmask = head_lo ? (rope_c0 >= 32 ? 0u : (0xFFFFFFFFu << rope_c0))
                                       : (rope_c0 >= 64 ? 0u
                                          : rope_c0 >= 32 ? (0xFFFFFFFFu << (rope_c0 - 32))
                                                          : 0xFFFFFFFFu);
        uint32_t emit = (bits & ~rmask) | (bits & rmask & 0x55555555u);
        while (__any_sync(0xFFFFFFFFu, emit != 0)) {
          const int cnt = __popc(emit);
          int incl = cnt;
  #pragma unroll
          for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(0xFFFFFFFFu, incl, o);
            if (lane >= o) incl += v;
          }
          const int total = __shfl_sync(0xFFFFFFFFu, incl, 31);
          int w = incl - cnt;
          while (emit && w < kFixCap) {
            const int b = __ffs(emit) - 1;
            emit &= emit - 1;
            u[w++] = static_cast<uint16_t>(base + b);
          }
          __syncwarp();
          const int n = total < kFixCap ? total : kFixCap;
          // units whose dots are exact in any order: the whole warp, one by one
          for (int i0 = 0; i0 < n; i0 += 32) {
            const int my = i0 + lane;
            bool ordered = false;
            if (my < n) {
              const int col = u[my];
              const bool pair = (col % kQBN) >= rope_c0;
              ordered = span_a + __ldg(p.b_span + col) + log2k > 53 ||
                        (pair && span_a + __ldg(p.b_span + col + 1) + log2k > 53);
            }
            const uint32_t ord = __ballot_sync(0xFFFFFFFFu, ordered);
            const int cnt_g = min(32, n - i0);
            for (int j = 0; j < cnt_g; ++j) {
              if ((ord >> j) & 1u) continue;
              const int col = u[i0 + j];
              const bool pair = (col % kQBN) >= rope_c0;
              const uint16_t* b0 = p.wq + static_cast<int64_t>(col) * p.K;
              const uint32_t v0 = round_f64_to_bf16(dot_f64_warp(a, b0, p.K, lane));
              const uint32_t v1 =
                  pair ? round_f64_to_bf16(dot_f64_warp(a, b0 + p.K, p.K, lane)) : 0u;
              if (lane == 0) fix_store(p, row, col, pair, v0, v1, rope_c0, rtab[warp]);
            }
            // the others: one lane each, ascending k
            if (ordered) {
              const int col = u[my];
              const bool pair = (col % kQBN) >= rope_c0;
              const uint16_t* b0 = p.wq + static_cast<int64_t>(col) * p.K;
              const uint32_t v0 = round_f64_to_bf16(dot_f64_seq(a, b0, p.K));
              const uint32_t v1 = pair ? round_f64_to_bf16(dot_f64_seq(a, b0 + p.K, p.K)) : 0u;
              fix_store(p, row, col, pair, v0, v1, rope_c0, rtab[warp]);
            }
          }
          __syncwarp();
        }
      }
    }
    __syncthreads();
  }
}

}  // namespace ixp

int launch_qproj_rope(const void* qr, const void* wq, const float* cos_tab, const float* sin_tab,
                      void* q_out, int64_t rows, int K, int n_heads, int rope_dim, int64_t seqlen,
                      const void* a_slices, const int* a_sig, const float* a_err,
                      const float* a_n3, const void* b_slices, const int* b_sig,
                      const float* b_err, const float* b_n3, const int* b_span,
                      uint32_t* open_bits, cudaStream_t stream) {
  using namespace ixp;
  DeviceInfo di;
  int st = current_device_info(&di);
  if (st != DSA_OK) return st;
  if (di.max_smem_optin < kQSmem) return DSA_ERR_UNSUPPORTED;
  if (n_heads > kQMaxHeads) return DSA_ERR_UNSUPPORTED;
  unsigned int* err = nullptr;
  st = device_error_word(&err);
  if (st != DSA_OK) return st;
  const int N = n_heads * kQBN;
  CUtensorMap tm_a, tm_b, tm_q;
  {
    const uint64_t dims[3] = {static_cast<uint64_t>(K), static_cast<uint64_t>(rows), 3};
    const uint64_t strides[2] = {static_cast<uint64_t>(K),
                                 static_cast<uint64_t>(rows) * static_cast<uint64_t>(K)};
    const uint32_t box[3] = {128, kBM, 1};
    st = encode_tensor_map(&tm_a, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, a_slices, dims, strides, box,
                           CU_TENSOR_MAP_SWIZZLE_128B);
    if (st != DSA_OK) return st;
  }
  {
    const uint64_t dims[3] = {static_cast<uint64_t>(K), static_cast<uint64_t>(N), 3};
    const uint64_t strides[2] = {static_cast<uint64_t>(K),
                                 static_cast<uint64_t>(N) * static_cast<uint64_t>(K)};
    const uint32_t box[3] = {128, kQBN, 1};
    st = encode_tensor_map(&tm_b, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, b_slices, dims, strides, box,
                           CU_TENSOR_MAP_SWIZZLE_128B);
    if (st != DSA_OK) return st;
  }
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(N), static_cast<uint64_t>(rows)};
    const uint64_t strides[1] = {static_cast<uint64_t>(N) * 2};
    const uint32_t box[2] = {kQBN, kBM};
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
  p.cos_tab = cos_tab;
  p.sin_tab = sin_tab;
  p.a_sig = a_sig;
  p.a_err = a_err;
  p.a_n3 = a_n3;
  p.b_sig = b_sig;
  p.b_err = b_err;
  p.b_n3 = b_n3;
  p.open_bits = open_bits;
  p.err = err;
  st = set_max_dynamic_smem(reinterpret_cast<const void*>(qproj_rope_kernel), kQSmem);
  if (st != DSA_OK) return st;
  const int grid = p.units < di.num_sms ? p.units : di.num_sms;
  qproj_rope_kernel<<<grid, kQThreads, kQSmem, stream>>>(tm_a, tm_b, tm_q, p);
  st = cuda_status(cudaGetLastError());
  if (st != DSA_OK) return st;
  FixParams f;
  f.M = static_cast<int>(rows);
  f.K = K;
  f.N = N;
  f.rope_dim = rope_dim;
  f.seqlen = seqlen;
  f.qr = static_cast<const uint16_t*>(qr);
  f.wq = static_cast<const uint16_t*>(wq);
  f.a_sig = a_sig;
  f.b_span = b_span;
  f.cos_tab = cos_tab;
  f.sin_tab = sin_tab;
  f.open_bits = open_bits;
  f.q = static_cast<uint16_t*>(q_out);
  // one wave: kFixBlocksPerSm resident blocks per SM (registers, shared memory)
  st = set_func_attribute_once(reinterpret_cast<const void*>(qproj_fixup_kernel),
                               cudaFuncAttributePreferredSharedMemoryCarveout,
                               cudaSharedmemCarveoutMaxShared);
  if (st != DSA_OK) return st;
  const int64_t fblocks = (rows + kFixWarps - 1) / kFixWarps;
  const int64_t fmax = static_cast<int64_t>(kFixBlocksPerSm) * di.num_sms;
  const int64_t fgrid = fblocks < fmax ? fblocks : fmax;
  qproj_fixup_kernel<<<static_cast<unsigned>(fgrid), kFixWarps * 32, 0, stream>>>(f);
  return cuda_status(cudaGetLastError());
}

}  // namespace dsa
