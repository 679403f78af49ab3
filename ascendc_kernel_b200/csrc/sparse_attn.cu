// SparseAttention forward for sm_100a: one persistent, warp-specialised kernel.
//
// Semantics (reference/task1_v0_ref.py:5-24): for every (b, t, h)
//   s_j = q[b,t,h] . kv[b, idx_j] * scale  over the valid j (0 <= idx_j < n_kv)
//   mx  = max(max_j s_j, sink[h])
//   out = sum_j exp(s_j - mx) kv[b, idx_j] / (sum_j exp(s_j - mx) + exp(sink[h] - mx))
// computed here in the multiplicity form used by the reference's fused kernel
// (src/sparse_attn_kernel_mm.asc:155-292): with c_k = #{j : idx_j == k},
//   sum_j f(idx_j) = sum_k c_k f(k),
// so both GEMMs run over all n_kv rows of kv[b] and the gather disappears.
//
// B200 mapping. A tile is 128 consecutive (token, head) rows of one batch
// (128 / n_heads tokens). Per CTA (one per SM, persistent over tiles):
//   warp 0       TMA producer: q tile (2 x 16 KB SW128 boxes) and the tile's
//                top-k indices into a 4-deep ring; kv[b] (2 x 4 KB SW128 boxes)
//                into one of two kv slots whenever the batch changes. A ring
//                stage is free once mm1 has read q and the epilogue has
//                counted the indices, long before the tile's output is done.
//   warp 1       TMEM allocator + single-thread tcgen05 issuer:
//                  mm1  S[128 x 32]  = Q[128 x 128] . KV^T        (8 x K16)
//                  mm2  O[128 x 128] = (P_hi + P_mid + P_lo) . KV (6 x K16)
//                P is split into three bf16 pieces so that the weights keep
//                fp32-level precision (~24 bits) through the bf16 MMA.
//   warps 2..9   two epilogue warpgroups that own alternate tiles. Each
//                thread owns one TMEM lane (= one (token, head) row): it reads
//                its 32 scores, forms the multiplicity softmax with the sink
//                logit, writes P to its shared-memory region (K-major, no
//                swizzle), waits for mm2, converts O to bf16 into the same
//                region (SW128 layout, P is dead after mm2) and one thread
//                TMA-stores it.
// TMEM: S[w] at columns [32w, 32w+32), O[w] at [128+128w, 256+128w); 512
// columns allocated. q and out stream through HBM once; the indices are read
// once per tile, kv once per batch change.
#include "common.cuh"
#include "host_util.h"

namespace dsa {
namespace sa {

constexpr int kRows = 128;
constexpr int kD = 128;
constexpr int kNKV = 32;
constexpr int kStages = 4;
constexpr int kQBytes = kRows * kD * 2;     // 32768
constexpr int kQBoxBytes = kRows * 64 * 2;  // 16384
constexpr int kKVBytes = kNKV * kD * 2;     // 8192
constexpr int kKVBoxBytes = kNKV * 64 * 2;  // 4096
constexpr int kIdxBytes = 2048;             // per stage, tpt * topk * sizeof(idx) <= 2048
constexpr int kPBytes = kRows * kNKV * 2;   // 8192 per piece
constexpr int kPPieces = 3;                 // hi, mid, lo
constexpr int kThreads = 320;
constexpr uint32_t kTmemCols = 512;

constexpr int kKVSlots = 2;
constexpr int kPRegion = kQBytes;           // per warpgroup: P pieces, then the output tile
constexpr int kOffQ = 0;
constexpr int kOffKV = kOffQ + kStages * kQBytes;
constexpr int kOffIdx = kOffKV + kKVSlots * kKVBytes;
constexpr int kOffP = kOffIdx + kStages * kIdxBytes;  // [2 wg][hi, mid, lo | out]
constexpr int kOffCnt = kOffP + 2 * kPRegion;          // [2 wg][8 tokens][32] bytes
constexpr int kOffBar = kOffCnt + 2 * 8 * 32;
constexpr int kNumBars = 2 * kStages + 5 * 2 + kKVSlots + 1;
constexpr int kOffMisc = kOffBar + kNumBars * 8;
constexpr int kSmemBytes = kOffMisc + 16 + 1024;  // + alignment slack

struct Params {
  int tiles_per_batch;
  int total_tiles;
  int heads;
  int tpt;  // tokens per tile
  int topk;
  int nkv;
  float scale_log2;  // softmax_scale * log2(e)
  uint32_t tx_bytes;  // q tile + indices of one stage
  const float* sink;
  unsigned int* err;
};

constexpr float kLog2e = 1.4426950408889634f;

template <typename IdxT>
__global__ void __launch_bounds__(kThreads, 1)
    sa_fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_kv,
                  const __grid_constant__ CUtensorMap tm_idx,
                  const __grid_constant__ CUtensorMap tm_out, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* full = bars;                  // [kStages] TMA -> MMA / epilogue
  uint64_t* empty = bars + kStages;       // [kStages] mm1 done + indices counted -> producer
  uint64_t* s_full = bars + 2 * kStages;  // [2] mm1 done -> epilogue w
  uint64_t* s_empty = s_full + 2;         // [2] S read -> MMA
  uint64_t* p_full = s_empty + 2;         // [2] P written -> MMA
  uint64_t* o_full = p_full + 2;          // [2] mm2 done -> epilogue w
  uint64_t* o_empty = o_full + 2;         // [2] O read -> MMA
  uint64_t* kv_empty = o_empty + 2;       // [kKVSlots] last mm2 of a batch done -> producer
  uint64_t* drain_bar = kv_empty + kKVSlots;  // MMA completion on teardown
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kOffMisc + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 2);
    }
    for (int k = 0; k < kKVSlots; ++k) mbar_init(&kv_empty[k], 1);
    for (int w = 0; w < 2; ++w) {
      mbar_init(&s_full[w], 1);
      mbar_init(&s_empty[w], 128);
      mbar_init(&p_full[w], 128);
      mbar_init(&o_full[w], 1);
      mbar_init(&o_empty[w], 128);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_kv);
    tma_prefetch_desc(&tm_idx);
    tma_prefetch_desc(&tm_out);
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
      int it = 0, kvc = -1, prev_b = -1;  // kvc: kv loads so far - 1
      for (int tile = blockIdx.x; tile < p.total_tiles; tile += gridDim.x, ++it) {
        const int s = it % kStages;
        const uint32_t ph = static_cast<uint32_t>(it / kStages) & 1u;
        if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag, p.err, DSA_DEVERR_SA_WAIT)) break;
        const int b = tile / p.tiles_per_batch;
        const int r0 = (tile - b * p.tiles_per_batch) * kRows;
        const bool new_kv = b != prev_b;
        if (new_kv) {
          ++kvc;
          prev_b = b;
          // the slot's previous batch (two kv loads ago) is no longer read
          if (kvc >= kKVSlots &&
              !mbar_wait(&kv_empty[kvc % kKVSlots],
                         static_cast<uint32_t>((kvc - kKVSlots) / kKVSlots) & 1u, abort_flag,
                         p.err, DSA_DEVERR_SA_WAIT))
            break;
        }
        uint8_t* qs = smem + kOffQ + s * kQBytes;
        mbar_arrive_expect_tx(&full[s], p.tx_bytes + (new_kv ? kKVBytes : 0u));
        tma_load_3d(qs, &tm_q, 0, r0, b, &full[s]);
        tma_load_3d(qs + kQBoxBytes, &tm_q, 64, r0, b, &full[s]);
        tma_load_3d(smem + kOffIdx + s * kIdxBytes, &tm_idx, 0, r0 / p.heads, b, &full[s]);
        if (new_kv) {
          uint8_t* kvs = smem + kOffKV + (kvc % kKVSlots) * kKVBytes;
          tma_load_3d(kvs, &tm_kv, 0, 0, b, &full[s]);
          tma_load_3d(kvs + kKVBoxBytes, &tm_kv, 64, 0, b, &full[s]);
        }
      }
      // Teardown: every load this thread issued must land before the CTA exits.
      for (int i = (it > kStages ? it - kStages : 0); i < it; ++i)
        mbar_drain(&full[i % kStages], static_cast<uint32_t>(i / kStages) & 1u);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc1 = make_idesc_bf16_f32(128, kNKV, 0, 0);
      constexpr uint32_t idesc2 = make_idesc_bf16_f32(128, kD, 0, 1);
      const uint32_t q_base = smem_u32(smem + kOffQ);
      const uint32_t kv_base = smem_u32(smem + kOffKV);
      const uint32_t p_base = smem_u32(smem + kOffP);
      bool ok = true;
      // kv slot of a tile: the producer's count of batch changes, mod kKVSlots
      auto issue_mm2 = [&](int i, int slot, bool last_of_batch) -> bool {
        const int w = i & 1;
        const uint32_t jph = static_cast<uint32_t>(i >> 1) & 1u;
        if (!mbar_wait(&p_full[w], jph, abort_flag, p.err, DSA_DEVERR_SA_WAIT)) return false;
        if (!mbar_wait(&o_empty[w], jph ^ 1u, abort_flag, p.err, DSA_DEVERR_SA_WAIT)) return false;
        tc_fence_after();
        const uint32_t d = tmem + 128u + static_cast<uint32_t>(w) * 128u;
        const uint32_t kvb = kv_base + static_cast<uint32_t>(slot) * kKVBytes;
        const uint32_t pw = p_base + static_cast<uint32_t>(w) * kPRegion;
#pragma unroll
        for (int piece = 0; piece < kPPieces; ++piece) {
#pragma unroll
          for (int kk = 0; kk < 2; ++kk) {
            // B = kv as [K = 16 kv rows] x [N = 128 dims], MN-major SW128:
            // MN atoms (64 dims) 4096 B apart, K atoms (8 rows) 1024 B apart.
            const uint64_t bd = make_smem_desc(kvb + kk * 2048u, 4096u, 1024u, kLayoutSW128);
            // A = P as [M = 128] x [K = 16], K-major, no swizzle: 8x16B core
            // matrices, K-adjacent 128 B apart, M-adjacent 512 B apart.
            const uint64_t ad = make_smem_desc(pw + piece * kPBytes + kk * 256u, 128u, 512u,
                                               kLayoutNone);
            umma_bf16(d, ad, bd, idesc2, (piece | kk) ? 1u : 0u);
          }
        }
        umma_commit(&o_full[w]);
        if (last_of_batch) umma_commit(&kv_empty[slot]);
        return true;
      };
      int it = 0, kvc = -1, prev_b = -1, prev_slot = 0;
      for (int tile = blockIdx.x; tile < p.total_tiles; tile += gridDim.x, ++it) {
        const int s = it % kStages;
        const uint32_t ph = static_cast<uint32_t>(it / kStages) & 1u;
        const int w = it & 1;
        const int b = tile / p.tiles_per_batch;
        const bool new_kv = b != prev_b;
        if (new_kv) {
          ++kvc;
          prev_b = b;
        }
        const int slot = kvc % kKVSlots;
        const uint32_t jph = static_cast<uint32_t>(it >> 1) & 1u;
        if (!mbar_wait(&full[s], ph, abort_flag, p.err, DSA_DEVERR_SA_WAIT) ||
            !mbar_wait(&s_empty[w], jph ^ 1u, abort_flag, p.err, DSA_DEVERR_SA_WAIT)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + static_cast<uint32_t>(w) * 32u;
        const uint32_t qb = q_base + static_cast<uint32_t>(s) * kQBytes;
        const uint32_t kvb = kv_base + static_cast<uint32_t>(slot) * kKVBytes;
#pragma unroll
        for (int k = 0; k < kD / 16; ++k) {
          const uint32_t box = static_cast<uint32_t>(k >> 2);
          const uint32_t koff = static_cast<uint32_t>(k & 3) * 32u;
          const uint64_t ad = make_smem_desc(qb + box * kQBoxBytes + koff, 16u, 1024u, kLayoutSW128);
          const uint64_t bd =
              make_smem_desc(kvb + box * kKVBoxBytes + koff, 16u, 1024u, kLayoutSW128);
          umma_bf16(d, ad, bd, idesc1, k > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[w]);
        umma_commit(&empty[s]);  // q read: the stage's second arrival
        if (it >= 1 && !issue_mm2(it - 1, prev_slot, new_kv)) {
          ok = false;
          break;
        }
        prev_slot = slot;
      }
      if (ok && it >= 1) issue_mm2(it - 1, prev_slot, false);
      // Teardown: all tcgen05 ops issued by this thread complete before exit.
      umma_commit(drain_bar);
      mbar_drain(drain_bar, 0);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int w = (warp - 2) >> 2;         // warpgroup 0 or 1
    const int t = threadIdx.x - 64 - 128 * w;  // 0..127 within the warpgroup
    const int quarter = warp & 3;          // TMEM lane quarter this warp may access
    const int row = quarter * 32 + lane;   // (token, head) row of the tile
    const int h = row % p.heads;
    const int tok = row / p.heads;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const float sink2 = p.sink[h] * kLog2e;
    uint8_t* cnt = smem + kOffCnt + w * 256;
    uint8_t* preg = smem + kOffP + w * kPRegion;
    const uint32_t p_hi = smem_u32(preg);
    const uint32_t p_mid = p_hi + kPBytes;
    const uint32_t p_lo = p_mid + kPBytes;
    const uint32_t prow = static_cast<uint32_t>((row >> 3) * 512 + (row & 7) * 16);

    // Every early exit is agreed by the whole warpgroup (named_bar_and) and
    // every TMEM access is warp-uniform (__all_sync), so an aborted wait can
    // never leave part of the group stuck at a barrier.
    bool ok = true;
    int it = w;
    for (int tile = blockIdx.x + w * gridDim.x; tile < p.total_tiles;
         tile += 2 * gridDim.x, it += 2) {
      const int s = it % kStages;
      const uint32_t ph = static_cast<uint32_t>(it / kStages) & 1u;
      const uint32_t jph = static_cast<uint32_t>(it >> 1) & 1u;
      const int b = tile / p.tiles_per_batch;
      const int r0 = (tile - b * p.tiles_per_batch) * kRows;
      ok = __all_sync(0xFFFFFFFFu, mbar_wait(&full[s], ph, abort_flag, p.err, DSA_DEVERR_SA_WAIT));

      // Multiplicity of every kv row in each token's top-k list (rows >= n_kv
      // and negative indices count as masked).
      // (token, bin) pairs: tpt * 32 of them, up to 256 for 8 tokens per tile.
      for (int pr = t; ok && pr < p.tpt * 32; pr += 128) {
        const int ct = pr >> 5;
        const int bin = pr & 31;
        const IdxT* ix = reinterpret_cast<const IdxT*>(smem + kOffIdx + s * kIdxBytes) + ct * p.topk;
        int c = 0;
        if (bin < p.nkv) {
          constexpr int kVec = 16 / static_cast<int>(sizeof(IdxT));  // indices per 16-byte load
          if (p.topk % kVec == 0) {
            // 16-byte loads, several in flight (the row is 16-byte aligned)
#pragma unroll 4
            for (int j = 0; j < p.topk; j += kVec) {
              const uint4 v = *reinterpret_cast<const uint4*>(ix + j);
              if (sizeof(IdxT) == 4) {
                c += (static_cast<int>(v.x) == bin) + (static_cast<int>(v.y) == bin) +
                     (static_cast<int>(v.z) == bin) + (static_cast<int>(v.w) == bin);
              } else {
                c += (v.x == static_cast<uint32_t>(bin) && v.y == 0u) +
                     (v.z == static_cast<uint32_t>(bin) && v.w == 0u);
              }
            }
          } else {
            for (int j = 0; j < p.topk; ++j) c += (static_cast<long long>(ix[j]) == bin) ? 1 : 0;
          }
        }
        cnt[pr] = static_cast<uint8_t>(c);
      }
      // the previous output store of this warpgroup has read its staging (the
      // P region, rewritten below)
      if (t == 0) bulk_wait_group_read<0>();
      if (!named_bar_and(1 + w, 128, ok)) break;
      if (t == 0) mbar_arrive(&empty[s]);  // indices counted: the stage's first arrival

      ok = __all_sync(0xFFFFFFFFu, mbar_wait(&s_full[w], jph, abort_flag, p.err, DSA_DEVERR_SA_WAIT));
      if (ok) {
        tc_fence_after();
        uint32_t sv[32];
        tmem_ld_32x32b_x32(tmem + lane_off + static_cast<uint32_t>(w) * 32u, sv);
        tc_fence_before();
        mbar_arrive(&s_empty[w]);

        uint32_t cw[8];
        {
          const uint4 c0 = *reinterpret_cast<const uint4*>(cnt + tok * 32);
          const uint4 c1 = *reinterpret_cast<const uint4*>(cnt + tok * 32 + 16);
          cw[0] = c0.x; cw[1] = c0.y; cw[2] = c0.z; cw[3] = c0.w;
          cw[4] = c1.x; cw[5] = c1.y; cw[6] = c1.z; cw[7] = c1.w;
        }
        // logits of the selected rows (-inf for rows of count 0), their max as a
        // tree, and the multiplicities as floats from their bits (c < 2^8: the
        // low bits of 2^23 + c), so that no conversion instruction is needed
        float z[32], cf[32];
        const uint64_t sc2 = f2_pack(p.scale_log2, p.scale_log2);
#pragma unroll
        for (int k = 0; k < 32; k += 2) {
          float z0, z1;
          f2_unpack(f2_mul(f2_pack(__uint_as_float(sv[k]), __uint_as_float(sv[k + 1])), sc2), z0,
                    z1);
          const uint32_t c0 = (cw[k >> 2] >> ((k & 3) * 8)) & 0xFFu;
          const uint32_t c1 = (cw[k >> 2] >> (((k + 1) & 3) * 8)) & 0xFFu;
          z[k] = c0 != 0u ? z0 : -INFINITY;
          z[k + 1] = c1 != 0u ? z1 : -INFINITY;
          cf[k] = __uint_as_float(0x4B000000u | c0) - 8388608.0f;
          cf[k + 1] = __uint_as_float(0x4B000000u | c1) - 8388608.0f;
        }
        float m8[11];
#pragma unroll
        for (int i = 0; i < 10; ++i) m8[i] = fmax3(z[3 * i], z[3 * i + 1], z[3 * i + 2]);
        m8[10] = fmax3(z[30], z[31], sink2);
        const float mx = fmaxf(fmax3(fmax3(m8[0], m8[1], m8[2]), fmax3(m8[3], m8[4], m8[5]),
                                     fmax3(m8[6], m8[7], m8[8])),
                               fmaxf(m8[9], m8[10]));
        float e[32];
        float ps[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int k = 0; k < 32; ++k) {
          e[k] = cf[k] * ex2_approx(z[k] - mx);  // 2^-inf = 0 for unselected rows
          ps[k & 3] += e[k];
        }
        float sum = (ps[0] + ps[1]) + (ps[2] + ps[3]);
        sum += ex2_approx(sink2 - mx);
        const float inv = __frcp_rn(sum);  // the same value as 1 / sum, fewer steps
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          // p = hi + mid + lo exactly up to the rounding of lo: hi and mid are
          // truncations to bf16 (byte permutes) and each residual (p - hi,
          // r - mid) is exact in fp32; two weights per f32x2 instruction.
          uint32_t hi[4], mid[4], lo[4];
          const uint64_t inv2 = f2_pack(inv, inv);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            float a0, a1;
            f2_unpack(f2_mul(f2_pack(e[c * 8 + 2 * j], e[c * 8 + 2 * j + 1]), inv2), a0, a1);
            // hi and mid by truncation (byte permutes), lo rounded
            hi[j] = __byte_perm(__float_as_uint(a0), __float_as_uint(a1), 0x7632u);
            float r0, r1;
            f2_unpack(f2_sub(f2_pack(a0, a1),
                             f2_pack(__uint_as_float(__float_as_uint(a0) & 0xFFFF0000u),
                                     __uint_as_float(__float_as_uint(a1) & 0xFFFF0000u))),
                      r0, r1);
            mid[j] = __byte_perm(__float_as_uint(r0), __float_as_uint(r1), 0x7632u);
            float q0, q1;
            f2_unpack(f2_sub(f2_pack(r0, r1),
                             f2_pack(__uint_as_float(__float_as_uint(r0) & 0xFFFF0000u),
                                     __uint_as_float(__float_as_uint(r1) & 0xFFFF0000u))),
                      q0, q1);
            lo[j] = pack_bf16x2(q0, q1);
          }
          st_shared_v4(p_hi + prow + c * 128, hi[0], hi[1], hi[2], hi[3]);
          st_shared_v4(p_mid + prow + c * 128, mid[0], mid[1], mid[2], mid[3]);
          st_shared_v4(p_lo + prow + c * 128, lo[0], lo[1], lo[2], lo[3]);
        }
        fence_proxy_async_smem();
        mbar_arrive(&p_full[w]);
        ok = __all_sync(0xFFFFFFFFu, mbar_wait(&o_full[w], jph, abort_flag, p.err, DSA_DEVERR_SA_WAIT));
      }
      uint8_t* ob = preg;  // P is dead after mm2: stage the output tile here
      if (ok) {
        tc_fence_after();
        const uint32_t ob_row = smem_u32(ob) + static_cast<uint32_t>(row) * 128u;
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
          uint32_t ov[32];
          tmem_ld_32x32b_x32(tmem + lane_off + 128u + static_cast<uint32_t>(w) * 128u +
                                 static_cast<uint32_t>(cc) * 32u,
                             ov);
          const uint32_t box_addr = ob_row + static_cast<uint32_t>(cc >> 1) * kQBoxBytes;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint32_t chunk = static_cast<uint32_t>((cc & 1) * 4 + j);
            const uint32_t a = pack_bf16x2(__uint_as_float(ov[8 * j + 0]), __uint_as_float(ov[8 * j + 1]));
            const uint32_t bb = pack_bf16x2(__uint_as_float(ov[8 * j + 2]), __uint_as_float(ov[8 * j + 3]));
            const uint32_t c = pack_bf16x2(__uint_as_float(ov[8 * j + 4]), __uint_as_float(ov[8 * j + 5]));
            const uint32_t d = pack_bf16x2(__uint_as_float(ov[8 * j + 6]), __uint_as_float(ov[8 * j + 7]));
            st_shared_v4(box_addr + ((chunk ^ static_cast<uint32_t>(row & 7)) << 4), a, bb, c, d);
          }
        }
        tc_fence_before();
        mbar_arrive(&o_empty[w]);
        fence_proxy_async_smem();
      }
      if (!named_bar_and(1 + w, 128, ok)) break;
      if (t == 0) {
        tma_store_3d(&tm_out, ob, 0, r0, b);
        tma_store_3d(&tm_out, ob + kQBoxBytes, 64, r0, b);
        bulk_commit_group();
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

template <typename IdxT>
int launch(const void* q, const void* kv, const void* idx, const float* sink, void* out,
           int64_t batch, int64_t m, int heads, int nkv, int topk, float scale,
           cudaStream_t stream) {
  DeviceInfo di;
  int st = current_device_info(&di);
  if (st != DSA_OK) return st;
  if (di.max_smem_optin < kSmemBytes) return DSA_ERR_UNSUPPORTED;
  unsigned int* err = nullptr;
  st = device_error_word(&err);
  if (st != DSA_OK) return st;

  const int64_t rows = m * heads;
  const int64_t tpb = (rows + kRows - 1) / kRows;
  const int64_t total = tpb * batch;
  if (total > 0x7FFFFFFF || rows > 0x7FFFFFFF || batch > 0x7FFFFFFF) return DSA_ERR_UNSUPPORTED;
  const int eb = static_cast<int>(sizeof(IdxT));
  const int tpt = kRows / heads;

  CUtensorMap tm_q, tm_kv, tm_idx, tm_out;
  {
    const uint64_t dims[3] = {static_cast<uint64_t>(kD), static_cast<uint64_t>(rows),
                              static_cast<uint64_t>(batch)};
    const uint64_t strides[2] = {static_cast<uint64_t>(kD) * 2,
                                 static_cast<uint64_t>(rows) * kD * 2};
    const uint32_t box[3] = {64, kRows, 1};
    st = encode_tensor_map(&tm_q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, q, dims, strides, box,
                           CU_TENSOR_MAP_SWIZZLE_128B);
    if (st != DSA_OK) return st;
    st = encode_tensor_map(&tm_out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, out, dims, strides, box,
                           CU_TENSOR_MAP_SWIZZLE_128B);
    if (st != DSA_OK) return st;
  }
  {
    const uint64_t dims[3] = {static_cast<uint64_t>(kD), static_cast<uint64_t>(nkv),
                              static_cast<uint64_t>(batch)};
    const uint64_t strides[2] = {static_cast<uint64_t>(kD) * 2,
                                 static_cast<uint64_t>(nkv) * kD * 2};
    const uint32_t box[3] = {64, kNKV, 1};
    st = encode_tensor_map(&tm_kv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, kv, dims, strides, box,
                           CU_TENSOR_MAP_SWIZZLE_128B);
    if (st != DSA_OK) return st;
  }
  {
    const uint64_t dims[3] = {static_cast<uint64_t>(topk), static_cast<uint64_t>(m),
                              static_cast<uint64_t>(batch)};
    const uint64_t strides[2] = {static_cast<uint64_t>(topk) * eb,
                                 static_cast<uint64_t>(m) * topk * eb};
    const uint32_t box[3] = {static_cast<uint32_t>(topk), static_cast<uint32_t>(tpt), 1};
    st = encode_tensor_map(&tm_idx,
                           eb == 8 ? CU_TENSOR_MAP_DATA_TYPE_INT64 : CU_TENSOR_MAP_DATA_TYPE_INT32,
                           3, idx, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (st != DSA_OK) return st;
  }

  Params p;
  p.tiles_per_batch = static_cast<int>(tpb);
  p.total_tiles = static_cast<int>(total);
  p.heads = heads;
  p.tpt = tpt;
  p.topk = topk;
  p.nkv = nkv;
  p.scale_log2 = scale * kLog2e;
  p.tx_bytes = static_cast<uint32_t>(kQBytes + tpt * topk * eb);
  p.sink = sink;
  p.err = err;

  st = set_max_dynamic_smem(reinterpret_cast<const void*>(sa_fwd_kernel<IdxT>), kSmemBytes);
  if (st != DSA_OK) return st;
  const int grid = static_cast<int>(total < di.num_sms ? total : di.num_sms);
  sa_fwd_kernel<IdxT><<<grid, kThreads, kSmemBytes, stream>>>(tm_q, tm_kv, tm_idx, tm_out, p);
  return cuda_status(cudaGetLastError());
}

}  // namespace sa
}  // namespace dsa

namespace dsa {
bool sa_long_supported(int heads, int head_dim, int nkv);
int launch_sa_long(const void* q, const void* kv, const void* idx, int idx_elem_bytes,
                   const float* sink, void* out, int64_t batch, int64_t m, int heads, int nkv,
                   int topk, float scale, cudaStream_t stream);
}  // namespace dsa

extern "C" int dsa_sparse_attn_fwd(const void* q, const void* kv, const void* idx,
                                   int idx_elem_bytes, const float* sink, void* out, int64_t batch,
                                   int64_t m, int n_heads, int head_dim, int n_kv, int topk,
                                   float softmax_scale, void* stream) {
  if (q == nullptr || kv == nullptr || idx == nullptr || sink == nullptr || out == nullptr)
    return DSA_ERR_INVALID_ARGUMENT;
  if (batch < 0 || m < 0 || n_heads <= 0 || head_dim <= 0 || n_kv <= 0 || topk <= 0)
    return DSA_ERR_INVALID_ARGUMENT;
  if (idx_elem_bytes != 4 && idx_elem_bytes != 8) return DSA_ERR_INVALID_ARGUMENT;
  if (head_dim != dsa::sa::kD) return DSA_ERR_UNSUPPORTED;
  if (n_kv > dsa::sa::kNKV || topk > 128) {
    // long kv pool (the chained configuration): chunked kernel
    if (!dsa::sa_long_supported(n_heads, head_dim, n_kv)) return DSA_ERR_UNSUPPORTED;
    if (!dsa::aligned16(q) || !dsa::aligned16(kv) || !dsa::aligned16(out) ||
        (reinterpret_cast<uintptr_t>(idx) % idx_elem_bytes) != 0)
      return DSA_ERR_MISALIGNED;
    if (batch == 0 || m == 0) return DSA_OK;
    return dsa::launch_sa_long(q, kv, idx, idx_elem_bytes, sink, out, batch, m, n_heads, n_kv,
                               topk, softmax_scale, static_cast<cudaStream_t>(stream));
  }
  if (n_heads != 16 && n_heads != 32 && n_heads != 64 && n_heads != 128) return DSA_ERR_UNSUPPORTED;
  if ((topk * idx_elem_bytes) % 16 != 0) return DSA_ERR_UNSUPPORTED;
  if ((dsa::sa::kRows / n_heads) * topk * idx_elem_bytes > dsa::sa::kIdxBytes)
    return DSA_ERR_UNSUPPORTED;
  if (!dsa::aligned16(q) || !dsa::aligned16(kv) || !dsa::aligned16(idx) || !dsa::aligned16(out))
    return DSA_ERR_MISALIGNED;
  if (batch == 0 || m == 0) return DSA_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (idx_elem_bytes == 8)
    return dsa::sa::launch<int64_t>(q, kv, idx, sink, out, batch, m, n_heads, n_kv, topk,
                                    softmax_scale, s);
  return dsa::sa::launch<int32_t>(q, kv, idx, sink, out, batch, m, n_heads, n_kv, topk,
                                  softmax_scale, s);
}
