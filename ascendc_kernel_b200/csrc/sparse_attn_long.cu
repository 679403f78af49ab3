// SparseAttention forward over a long kv pool (n_kv up to 4096, any top-k), for
// sm_100a: the chained long-context configuration, where the Lightning
// Indexer's top-2048 of 4096 compressed kv rows feed the attention.
//
// Semantics (reference/task1_v0_ref.py:5-24), for every (b, t, h):
//   s_j = q[b,t,h] . kv[b, idx_j] * scale  over the valid j (0 <= idx_j < n_kv)
//   mx  = max(max_j s_j, sink[h])
//   out = sum_j exp(s_j - mx) kv[b, idx_j] / (sum_j exp(s_j - mx) + exp(sink[h] - mx))
// in the multiplicity form (c_k = #{j : idx_j == k}, sum_j f(idx_j) =
// sum_k c_k f(k)), so the GEMMs stream contiguous 128-row chunks of kv[b]
// instead of gathering rows; chunks past the tile's largest index are skipped
// (with causal indexer output that is about half of the pool on average).
//
// B200 mapping. A tile is 128 (token, head) rows (2 tokens of 64 heads, or 1 of
// 128); a work item is two consecutive tiles of one batch, which share every
// 128-row kv chunk. Per CTA (one per SM, persistent, 384 threads):
//   warp 0      TMA: kv chunks (128 rows x 128 dims, 32 KB) into a 2-stage ring
//               (an item's first two chunks before its q tiles, so they arrive
//               during the previous item's epilogue), the two q tiles.
//   warp 1      tcgen05 issuer, per chunk and tile:
//                 S[128 x 128]  = Q . KV_c^T              (K-major smem operands)
//                 O[128 x 128] += (P_hi + P_lo) . KV_c    (P read from TMEM, kv
//                                                          as an MN-major operand)
//               in the order PV(c) of a tile, then S(c+1) of the same tile into
//               the columns PV(c) read, so one tile's softmax overlaps the other
//               tile's products; a q tile is released once its last S completed.
//   warps 2..9  softmax: both warpgroups serve both tiles; a thread owns one row
//               and one half (64 keys) of every chunk: z = s scale log2(e) +
//               log2(c_k) (-inf for c_k = 0), P = 2^(z - m) written back over S
//               as two bf16 pieces (P_hi + P_lo carries ~16 bits). The two
//               threads of a row agree the reference m through a 64-thread named
//               barrier per TMEM lane quarter; it is set by the item's first
//               chunk and moves (rescaling O and the sum) only when a chunk's max
//               exceeds it by more than 2^32. After the last chunk O is divided
//               by the sum plus the sink term and stored through the (then free)
//               log2-count buffer.
//   warps 10,11 count builders: the counts c_k of the NEXT item's tokens
//               (shared-memory atomics on 16-bit counters) and its chunk
//               count, while the current item computes.
// TMEM per tile w: its S/P columns [256w, 256w+128) and O [256w+128, 256w+256).
#include "common.cuh"
#include "host_util.h"

namespace dsa {
namespace sal {

constexpr int kRows = 128;
constexpr int kD = 128;
constexpr int kChunk = 128;
constexpr int kMaxNkv = 4096;
constexpr int kKVStages = 2;
constexpr int kThreads = 384;
constexpr uint32_t kTmemCols = 512;
constexpr int kQBytes = kRows * kD * 2;           // 32768
constexpr int kQBoxBytes = kRows * 64 * 2;        // 16384
constexpr int kKVBytes = kChunk * kD * 2;         // 32768
constexpr int kKVBoxBytes = kChunk * 64 * 2;      // 16384
constexpr int kOffQ = 0;                                        // [2 wg]
constexpr int kOffKV = kOffQ + 2 * kQBytes;                     // 65536
constexpr int kOffBias = kOffKV + kKVStages * kKVBytes;         // 131072: [2 wg][2 tok][n] f32
constexpr int kOffCnt = kOffBias + 2 * 2 * kMaxNkv * 4;         // 196608: [2 wg][2 tok][n] u16
constexpr int kOffMeta = kOffCnt + 2 * 2 * kMaxNkv * 2;         // 229376
constexpr int kOffX = kOffMeta + 64;                            // [2 half][128 rows] f32
constexpr int kOffBar = kOffX + 2 * kRows * 4;
constexpr int kNumBars = 2 + 2 + 4 + 2 + 2 + 2 * kKVStages + 2 * 3 + 2 + 1;
constexpr int kOffMisc = kOffBar + kNumBars * 8;
constexpr int kSmemBytes = kOffMisc + 16 + 1024;
static_assert(kRows * kD * 2 == 2 * kMaxNkv * 4, "output staging reuses a log2-count buffer");
constexpr float kLog2e = 1.4426950408889634f;
// The softmax reference max moves (and O is rescaled) only when a group's max
// exceeds it by more than 2^32.
constexpr float kRescaleLog2 = 32.0f;

struct Params {
  int64_t m;               // tokens per batch
  int heads;               // 64 or 128
  int tpt;                 // tokens per tile
  int tiles_per_batch;
  int items_per_batch;
  int64_t total_items;
  int topk;
  int nkv;
  float scale_log2;
  const float* sink;
  const void* idx;         // [batch, m, topk] int32 / int64 (when mask is null)
  const uint32_t* mask;    // or: [batch, m, mask_words] selection bitmaps, bit k = row k + mask_offset
  int mask_words;
  int64_t mask_offset;
  unsigned int* err;
};

template <typename IdxT>
__global__ void __launch_bounds__(kThreads, 1)
    sa_long_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_kv,
                   const __grid_constant__ CUtensorMap tm_out, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* q_full = bars;                       // [2] TMA -> MMA
  uint64_t* q_empty = bars + 2;                  // [2] last S product of the tile done -> TMA
  uint64_t* meta_full = bars + 4;                // [2 wg][2 slot] counts and chunk count ready
  uint64_t* cnt_empty = bars + 8;                // [2] counts turned into log2 -> count warps
  uint64_t* meta_empty = bars + 10;              // [2 slot] chunk counts read by TMA and MMA
  uint64_t* kv_full = bars + 12;                 // [kKVStages]
  uint64_t* kv_empty = kv_full + kKVStages;      // [kKVStages]
  uint64_t* s_full = kv_empty + kKVStages;       // [2] S of a chunk in TMEM
  uint64_t* p_full = s_full + 2;                 // [2] P written (256 arrivals)
  uint64_t* o_done = p_full + 2;                 // [2] PV product of a chunk completed
  uint64_t* o_empty = o_done + 2;                // [2] O read by the epilogue (256 arrivals)
  uint64_t* drain_bar = o_empty + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kOffMisc + 4);
  // meta[2 w + slot]: chunks of tile w of the item in slot (li & 1); red: count-warp maxima
  volatile int* meta = reinterpret_cast<volatile int*>(smem + kOffMeta);
  volatile int* red = meta + 4;
  uint32_t* cnt32 = reinterpret_cast<uint32_t*>(smem + kOffCnt);  // two 16-bit counters a word
  float* bias = reinterpret_cast<float*>(smem + kOffBias);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int w = 0; w < 2; ++w) {
      mbar_init(&q_full[w], 1);
      mbar_init(&q_empty[w], 1);
      mbar_init(&meta_full[2 * w], 1);
      mbar_init(&meta_full[2 * w + 1], 1);
      mbar_init(&cnt_empty[w], 1);
      mbar_init(&meta_empty[w], 2);
      mbar_init(&o_empty[w], 256);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 256);
      mbar_init(&o_done[i], 1);
    }
    for (int s = 0; s < kKVStages; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_kv);
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

  auto tile_of = [&](int64_t item, int w, int& b, int& tb, bool& valid) {
    b = static_cast<int>(item / p.items_per_batch);
    tb = static_cast<int>(item - static_cast<int64_t>(b) * p.items_per_batch) * 2 + w;
    valid = tb < p.tiles_per_batch;
  };

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int li = 0, gc = 0;
      bool ok = true;
      auto load_kv = [&](int b, int c) -> bool {
        const int s = gc % kKVStages;
        if (!mbar_wait(&kv_empty[s], ((gc / kKVStages) & 1) ^ 1, abort_flag, p.err,
                       DSA_DEVERR_SA_WAIT))
          return false;
        uint8_t* kvs = smem + kOffKV + s * kKVBytes;
        mbar_arrive_expect_tx(&kv_full[s], kKVBytes);
        tma_load_3d(kvs, &tm_kv, 0, c * kChunk, b, &kv_full[s]);
        tma_load_3d(kvs + kKVBoxBytes, &tm_kv, 64, c * kChunk, b, &kv_full[s]);
        ++gc;
        return true;
      };
      for (int64_t item = blockIdx.x; ok && item < p.total_items; item += gridDim.x, ++li) {
        int nc = 0;
        for (int w = 0; w < 2; ++w) {
          if (!mbar_wait(&meta_full[2 * w + (li & 1)], (li >> 1) & 1, abort_flag, p.err,
                         DSA_DEVERR_SA_WAIT)) {
            ok = false;
            break;
          }
          nc = max(nc, static_cast<int>(meta[2 * w + (li & 1)]));
        }
        if (!ok) break;
        mbar_arrive(&meta_empty[li & 1]);
        const int b = static_cast<int>(item / p.items_per_batch);
        // the first kKVStages chunks reuse stages that earlier items' products free
        const int npre = min(nc, kKVStages);
        for (int c = 0; c < npre && ok; ++c) ok = load_kv(b, c);
        for (int w = 0; w < 2 && ok; ++w) {
          int bb, tb;
          bool valid;
          tile_of(item, w, bb, tb, valid);
          if (!mbar_wait(&q_empty[w], (li & 1) ^ 1, abort_flag, p.err, DSA_DEVERR_SA_WAIT)) {
            ok = false;
            break;
          }
          uint8_t* qs = smem + kOffQ + w * kQBytes;
          if (valid) {
            mbar_arrive_expect_tx(&q_full[w], kQBytes);
            tma_load_3d(qs, &tm_q, 0, tb * kRows, b, &q_full[w]);
            tma_load_3d(qs + kQBoxBytes, &tm_q, 64, tb * kRows, b, &q_full[w]);
          } else {
            mbar_arrive(&q_full[w]);
          }
        }
        for (int c = npre; c < nc && ok; ++c) ok = load_kv(b, c);
      }
      for (int i = (gc > kKVStages ? gc - kKVStages : 0); i < gc; ++i)
        mbar_drain(&kv_full[i % kKVStages], (i / kKVStages) & 1);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    // Per chunk c: S of chunk c for both tiles (into S buffer c % 2, free once
    // the PV product of chunk c - 2 completed), then the PV products of chunk
    // c - 1; so the softmax of one chunk overlaps the QK^T of the next.
    if (lane == 0) {
      constexpr uint32_t idesc1 = make_idesc_bf16_f32(128, kChunk, 0, 0);
      constexpr uint32_t idesc2 = make_idesc_bf16_f32(128, kD, 0, 1);
      // Descriptors are built once; per MMA only the 14-bit start-address field
      // (low word, 16-byte units) moves, by compile-time offsets, so the single
      // issuing thread spends a few instructions per MMA (every smem address
      // here is below 256 KB, so the field never carries into the LBO bits).
      const uint64_t dq = make_smem_desc(smem_u32(smem + kOffQ), 16u, 1024u, kLayoutSW128);
      const uint64_t dkv = make_smem_desc(smem_u32(smem + kOffKV), 16u, 1024u, kLayoutSW128);
      const uint32_t hi = static_cast<uint32_t>(dkv >> 32);  // SBO 1024, SW128: shared by all
      const uint32_t q_lo = static_cast<uint32_t>(dq);
      const uint32_t kvk_lo = static_cast<uint32_t>(dkv);  // K-major kv (S operand B)
      const uint32_t kvmn_lo = static_cast<uint32_t>(      // MN-major kv (PV operand B)
          make_smem_desc(smem_u32(smem + kOffKV), static_cast<uint32_t>(kKVBoxBytes), 1024u,
                         kLayoutSW128));
      int li = 0, gc = 0;
      int gs[2] = {0, 0};     // S products issued per warpgroup (all items)
      int gm[2] = {0, 0};     // PV products issued per warpgroup
      int uses[2] = {0, 0};   // items per warpgroup that wrote O
      int ncw[2] = {0, 0};
      bool ok = true;
      // S of chunk c for warpgroup w from kv stage s (K-major operands); the S/P
      // columns are free once the previous chunk's PV product completed
      auto issue_s = [&](int w, int c, int s) -> bool {
        if (c >= ncw[w]) return true;
        if (gs[w] >= 1 && !mbar_wait(&o_done[w], (gs[w] - 1) & 1, abort_flag, p.err,
                                     DSA_DEVERR_SA_WAIT))
          return false;
        tc_fence_after();
        const uint32_t d = tmem + static_cast<uint32_t>(w * 256);
        const uint32_t qa = q_lo + static_cast<uint32_t>(w * (kQBytes >> 4));
        const uint32_t kb = kvk_lo + static_cast<uint32_t>(s * (kKVBytes >> 4));
#pragma unroll
        for (int k = 0; k < kD / 16; ++k) {
          const uint32_t ao = static_cast<uint32_t>(((k >> 2) * kQBoxBytes + (k & 3) * 32) >> 4);
          const uint32_t bo = static_cast<uint32_t>(((k >> 2) * kKVBoxBytes + (k & 3) * 32) >> 4);
          umma_bf16(d, desc_from_words(qa + ao, hi), desc_from_words(kb + bo, hi), idesc1,
                    k > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[w]);
        if (c == ncw[w] - 1) umma_commit(&q_empty[w]);  // q tile no longer read
        ++gs[w];
        return true;
      };
      // PV of chunk c for warpgroup w from kv stage s (P in TMEM, MN-major kv)
      auto issue_pv = [&](int w, int c, int s) -> bool {
        if (c >= ncw[w]) return true;
        if (!mbar_wait(&p_full[w], gm[w] & 1, abort_flag, p.err, DSA_DEVERR_SA_WAIT))
          return false;
        if (c == 0) {
          if (uses[w] > 0 && !mbar_wait(&o_empty[w], (uses[w] - 1) & 1, abort_flag, p.err,
                                        DSA_DEVERR_SA_WAIT))
            return false;
          ++uses[w];
        }
        tc_fence_after();
        const uint32_t sp = tmem + static_cast<uint32_t>(w * 256);
        const uint32_t d = sp + static_cast<uint32_t>(kChunk);
        const uint32_t kb = kvmn_lo + static_cast<uint32_t>(s * (kKVBytes >> 4));
#pragma unroll
        for (int st = 0; st < kChunk / 16; ++st) {
          // B = kv as [K = 16 kv rows] x [N = 128 dims], MN-major SW128:
          // dim atoms (64) one box apart, row atoms (8) 1024 B apart.
          const uint64_t bd = desc_from_words(kb + static_cast<uint32_t>((st * 2048) >> 4), hi);
          // A = P in TMEM: keys [32h, 32h+32) hold P_hi in columns [32h, 32h+16)
          // and P_lo in [32h+16, 32h+32) (two bf16 per column)
          const uint32_t a_hi = sp + static_cast<uint32_t>((st >> 1) * 32 + (st & 1) * 8);
          umma_bf16_tmem_a(d, a_hi, bd, idesc2, (c > 0 || st > 0) ? 1u : 0u);
          umma_bf16_tmem_a(d, a_hi + 16u, bd, idesc2, 1u);
        }
        umma_commit(&o_done[w]);
        ++gm[w];
        return true;
      };
      auto wait_kv = [&](int i) -> bool {  // i: global chunk number
        return mbar_wait(&kv_full[i % kKVStages], (i / kKVStages) & 1, abort_flag, p.err,
                         DSA_DEVERR_SA_WAIT);
      };
      for (int64_t item = blockIdx.x; ok && item < p.total_items; item += gridDim.x, ++li) {
#pragma unroll
        for (int w = 0; w < 2; ++w) {
          ok = ok &&
               mbar_wait(&meta_full[2 * w + (li & 1)], (li >> 1) & 1, abort_flag, p.err,
                         DSA_DEVERR_SA_WAIT) &&
               mbar_wait(&q_full[w], li & 1, abort_flag, p.err, DSA_DEVERR_SA_WAIT);
          if (ok) {
            ncw[w] = meta[2 * w + (li & 1)];
            if (ncw[w] == 0) umma_commit(&q_empty[w]);
          }
        }
        if (!ok) break;
        mbar_arrive(&meta_empty[li & 1]);
        const int nc = max(ncw[0], ncw[1]);
        // per chunk c: PV(c) of a tile, then S(c+1) of the same tile into the
        // columns PV(c) just read, so one tile's S overlaps the other's softmax
        if (nc > 0) {
          ok = wait_kv(gc) && issue_s(0, 0, gc % kKVStages) && issue_s(1, 0, gc % kKVStages);
        }
        for (int c = 0; c < nc && ok; ++c) {
          const int s = (gc + c) % kKVStages;
          const int sn = (gc + c + 1) % kKVStages;
          const bool more = c + 1 < nc;
          ok = issue_pv(0, c, s) && (!more || (wait_kv(gc + c + 1) && issue_s(0, c + 1, sn))) &&
               issue_pv(1, c, s) && (!more || issue_s(1, c + 1, sn));
          if (!ok) break;
          umma_commit(&kv_empty[s]);
        }
        gc += nc;
      }
      umma_commit(drain_bar);
      mbar_drain(drain_bar, 0);
    }
  } else if (warp < 10) {
    // ------------------------------------------------------------ softmax warps
    // Both warpgroups serve both tiles: a thread owns one row and one half of the
    // keys of every chunk (warps 2..5 keys [0, 64), warps 6..9 keys [64, 128)) and
    // the same half of the O columns in the epilogue. The two threads of a row
    // sit in warps with the same TMEM lane quarter and pair up through a 64-thread
    // named barrier per quarter.
    const int half = (warp - 2) >> 2;
    const int t = threadIdx.x - 64;             // 0..255
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;        // (token, head) row of the tile
    const int tok = row / p.heads;
    const int h = row % p.heads;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const float sink2 = p.sink[h] * kLog2e;
    const uint32_t pair_bar = 4 + static_cast<uint32_t>(quarter);
    float* xbuf = reinterpret_cast<float*>(smem + kOffX);  // [2 half][128 rows]
    const uint64_t scale2 = f2_pack(p.scale_log2, p.scale_log2);
    bool ok = true;
    int li = 0;
    int g0 = 0, g1 = 0;  // chunks processed per tile (all items)

    // One chunk of tile w: S of this thread's 64 keys, z = s scale log2e + log2 c
    // (-inf if c = 0), P = 2^(z - m) as bf16 hi + lo over the S columns of the
    // same keys (keys [32j, 32j+32) -> P_hi in columns [32j, 32j+16), P_lo in
    // [32j+16, 32j+32)). The reference m of a row is agreed by its two threads:
    // it is set from the item's first chunk and moves (rescaling O and the sum)
    // only when a chunk's max exceeds it by more than 2^kRescaleLog2, so P <=
    // 2^kRescaleLog2 c and keys flushed to 0 are below 2^-126 of the max.
    auto chunk = [&](int w, int c, float& m, float& l, int& gw) -> bool {
      // the row's two threads leave together (they meet at the pair barrier below)
      if (!named_bar_and(pair_bar, 64, mbar_wait(&s_full[w], gw & 1, abort_flag, p.err,
                                                 DSA_DEVERR_SA_WAIT)))
        return false;
      tc_fence_after();
      const uint32_t sp = tmem + lane_off + static_cast<uint32_t>(w * 256 + half * 64);
      const uint32_t od = tmem + lane_off + static_cast<uint32_t>(w * 256 + kChunk + half * 64);
      const float* cb = bias + (w * 2 + tok) * kMaxNkv + c * kChunk + half * 64;
      uint64_t z[32];
      float mh;
      {
        uint32_t va[32], vb[32];
        tmem_ld_32x32b_x32_nowait(sp, va);
        tmem_ld_32x32b_x32_nowait(sp + 32u, vb);
        tmem_wait_ld_dep(va);
        tmem_wait_ld_dep(vb);
#pragma unroll
        for (int q4 = 0; q4 < 16; ++q4) {
          const float4 bv = reinterpret_cast<const float4*>(cb)[q4];
          const uint32_t* v = q4 < 8 ? va : vb;
          const int o = (q4 & 7) * 4;
          z[2 * q4] = f2_fma(f2_pack(__uint_as_float(v[o]), __uint_as_float(v[o + 1])), scale2,
                             f2_pack(bv.x, bv.y));
          z[2 * q4 + 1] = f2_fma(f2_pack(__uint_as_float(v[o + 2]), __uint_as_float(v[o + 3])),
                                 scale2, f2_pack(bv.z, bv.w));
        }
        // the max as a tree of three-input maxes (64 values, depth 4)
        float t1[22];
#pragma unroll
        for (int i = 0; i < 21; ++i) {
          float a0, a1, b0, b1, c0, c1;
          const int e0 = 3 * i, e1 = 3 * i + 1, e2 = 3 * i + 2;  // elements of the 64
          f2_unpack(z[e0 >> 1], a0, a1);
          f2_unpack(z[e1 >> 1], b0, b1);
          f2_unpack(z[e2 >> 1], c0, c1);
          t1[i] = fmax3((e0 & 1) ? a1 : a0, (e1 & 1) ? b1 : b0, (e2 & 1) ? c1 : c0);
        }
        {
          float a0, a1;
          f2_unpack(z[31], a0, a1);
          t1[21] = a1;  // element 63
        }
        float t2[8];
#pragma unroll
        for (int i = 0; i < 7; ++i) t2[i] = fmax3(t1[3 * i], t1[3 * i + 1], t1[3 * i + 2]);
        t2[7] = t1[21];
        mh = fmaxf(fmax3(t2[0], t2[1], t2[2]), fmax3(t2[3], t2[4], fmax3(t2[5], t2[6], t2[7])));
      }
      // the item's first chunk always agrees a reference; later chunks only when
      // some row of the quarter went more than 2^kRescaleLog2 above its reference
      if (named_bar_or(pair_bar, 64, c == 0 || mh > m + kRescaleLog2)) {
        xbuf[half * kRows + row] = mh;
        named_bar_sync(pair_bar, 64);
        const float mx = fmaxf(mh, xbuf[(half ^ 1) * kRows + row]);
        float factor = 1.f;
        if (c == 0) {
          m = fmaxf(m, mx);  // nothing accumulated yet for this item
        } else if (mx > m + kRescaleLog2) {
          factor = ex2_approx(m - mx);
          m = mx;
          l *= factor;
        }
        if (__any_sync(0xFFFFFFFFu, factor != 1.f)) {
          // O holds every earlier chunk's product: this chunk's S was issued
          // after the previous PV product completed
#pragma unroll 1
          for (int q = 0; q < 2; ++q) {
            uint32_t ov[32];
            tmem_ld_32x32b_x32(od + static_cast<uint32_t>(q * 32), ov);
#pragma unroll
            for (int k = 0; k < 32; ++k) ov[k] = __float_as_uint(__uint_as_float(ov[k]) * factor);
            tmem_st_32x32b_x32(od + static_cast<uint32_t>(q * 32), ov);
          }
        }
      }
      const uint64_t negm2 = f2_pack(-m, -m);
      uint64_t ls2[2] = {0ull, 0ull};
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        uint32_t pk[32];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          float d0, d1;
          f2_unpack(f2_add(z[16 * j + i], negm2), d0, d1);
          const float e0 = ex2_approx(d0), e1 = ex2_approx(d1);  // 2^-inf = 0
          const uint64_t e2 = f2_pack(e0, e1);
          ls2[i & 1] = f2_add(ls2[i & 1], e2);
          const uint32_t hb = pack_bf16x2(e0, e1);
          pk[i] = hb;
          float r0, r1;
          f2_unpack(f2_sub(e2, f2_pack(__uint_as_float(hb << 16), __uint_as_float(hb & 0xFFFF0000u))),
                    r0, r1);
          pk[16 + i] = pack_bf16x2(r0, r1);
        }
        tmem_st_32x32b_x32_nowait(sp + static_cast<uint32_t>(j * 32), pk);
      }
      float a0, a1, b0, b1;
      f2_unpack(ls2[0], a0, a1);
      f2_unpack(ls2[1], b0, b1);
      l += (a0 + a1) + (b0 + b1);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&p_full[w]);
      ++gw;
      return true;
    };

    // Epilogue of tile w: O / (l + sink term) -> bf16 -> staging box `half` (SW128).
    auto epilogue = [&](int w, int nc, bool valid, float m, float l) {
      // the row's total: this thread's half plus its partner's
      xbuf[half * kRows + row] = l;
      named_bar_sync(pair_bar, 64);
      const float lt = l + xbuf[(half ^ 1) * kRows + row];
      if (ok && valid) {
        const float inv = 1.0f / (lt + ex2_approx(sink2 - m));
        const uint32_t od = tmem + lane_off + static_cast<uint32_t>(w * 256 + kChunk + half * 64);
        uint8_t* stage = smem + kOffBias + w * 2 * kMaxNkv * 4;
        const uint32_t box_row = smem_u32(stage) + static_cast<uint32_t>(half * kQBoxBytes + row * 128);
#pragma unroll 1
        for (int cc = 0; cc < 2; ++cc) {
          uint32_t ov[32];
          if (nc > 0) {
            tmem_ld_32x32b_x32(od + static_cast<uint32_t>(cc) * 32u, ov);
          } else {
#pragma unroll
            for (int k = 0; k < 32; ++k) ov[k] = 0u;  // only the sink: the output is 0
          }
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint32_t c16 = static_cast<uint32_t>(cc * 4 + j);
            uint32_t wv[4];
#pragma unroll
            for (int u = 0; u < 4; ++u)
              wv[u] = pack_bf16x2(__uint_as_float(ov[8 * j + 2 * u]) * inv,
                                  __uint_as_float(ov[8 * j + 2 * u + 1]) * inv);
            st_shared_v4(box_row + ((c16 ^ static_cast<uint32_t>(row & 7)) << 4), wv[0], wv[1],
                         wv[2], wv[3]);
          }
        }
        fence_proxy_async_smem();
      }
      if (nc > 0) {
        tc_fence_before();
        mbar_arrive(&o_empty[w]);
      }
    };

    for (int64_t item = blockIdx.x; item < p.total_items; item += gridDim.x, ++li) {
      int b, tb0, tb1;
      bool valid0, valid1;
      tile_of(item, 0, b, tb0, valid0);
      tile_of(item, 1, b, tb1, valid1);
      // the previous item's outputs have left the staging buffers
      if (t == 0) bulk_wait_group_read<0>();
      const bool okm =
          mbar_wait(&meta_full[li & 1], (li >> 1) & 1, abort_flag, p.err, DSA_DEVERR_SA_WAIT) &&
          mbar_wait(&meta_full[2 + (li & 1)], (li >> 1) & 1, abort_flag, p.err, DSA_DEVERR_SA_WAIT);
      ok = named_bar_and(1, 256, okm);
      if (!ok) break;
      const int nc0 = meta[li & 1], nc1 = meta[2 + (li & 1)];
      // ---- counts -> log2(c) per key (-inf for c = 0), zeroing the counters;
      // the softmax weight c e^s becomes 2^(s log2e + log2 c)
#pragma unroll 1
      for (int w = 0; w < 2; ++w) {
        const int nc = w ? nc1 : nc0;
        const int n8 = nc * (kChunk / 8);  // 8-key groups per token
        uint32_t* wcnt = cnt32 + w * kMaxNkv;
        float* wbias = bias + w * 2 * kMaxNkv;
        for (int i = t; i < p.tpt * n8; i += 256) {
          const int tk = i / n8, q8 = i - tk * n8;
          uint4* cp = reinterpret_cast<uint4*>(wcnt + tk * (kMaxNkv / 2)) + q8;
          const uint4 v = *cp;
          *cp = make_uint4(0u, 0u, 0u, 0u);
          const uint32_t wd[4] = {v.x, v.y, v.z, v.w};
          float f[8];
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const uint32_t cnt = (wd[u >> 1] >> ((u & 1) * 16)) & 0xFFFFu;
            f[u] = cnt ? 0.f : -INFINITY;
            if (cnt > 1) f[u] = log2f(static_cast<float>(cnt));
          }
          float4* bp = reinterpret_cast<float4*>(wbias + tk * kMaxNkv) + q8 * 2;
          bp[0] = make_float4(f[0], f[1], f[2], f[3]);
          bp[1] = make_float4(f[4], f[5], f[6], f[7]);
        }
      }
      named_bar_sync(1, 256);
      if (t == 0) {
        mbar_arrive(&cnt_empty[0]);
        mbar_arrive(&cnt_empty[1]);
      }
      // ---- chunks, alternating tiles (the issuer's order)
      float m0 = sink2, l0 = 0.f, m1 = sink2, l1 = 0.f;
      const int ncm = max(nc0, nc1);
      for (int c = 0; ok && c < ncm; ++c) {
        if (c < nc0) ok = chunk(0, c, m0, l0, g0);
        if (ok && c < nc1) ok = chunk(1, c, m1, l1, g1);
      }
      // ---- epilogues: every chunk product of both tiles complete first, so
      // no thread still reads the exchange buffer or a log2-count buffer
      if (ok && nc0 > 0)
        ok = __all_sync(0xFFFFFFFFu, mbar_wait(&o_done[0], (g0 - 1) & 1, abort_flag, p.err,
                                               DSA_DEVERR_SA_WAIT));
      if (ok && nc1 > 0)
        ok = __all_sync(0xFFFFFFFFu, mbar_wait(&o_done[1], (g1 - 1) & 1, abort_flag, p.err,
                                               DSA_DEVERR_SA_WAIT));
      if (ok) tc_fence_after();
      epilogue(0, nc0, valid0, m0, l0);
      if (!named_bar_and(1, 256, ok)) break;
      if (t == 0 && valid0) {
        uint8_t* stage = smem + kOffBias;
        tma_store_3d(&tm_out, stage, 0, tb0 * kRows, b);
        tma_store_3d(&tm_out, stage + kQBoxBytes, 64, tb0 * kRows, b);
        bulk_commit_group();
      }
      epilogue(1, nc1, valid1, m1, l1);
      if (!named_bar_and(1, 256, ok)) break;
      if (t == 0 && valid1) {
        uint8_t* stage = smem + kOffBias + 2 * kMaxNkv * 4;
        tma_store_3d(&tm_out, stage, 0, tb1 * kRows, b);
        tma_store_3d(&tm_out, stage + kQBoxBytes, 64, tb1 * kRows, b);
        bulk_commit_group();
      }
    }
    if (t == 0) bulk_wait_group<0>();
  } else {
    // ------------------------------------------------------------ count builders
    // counts of item li go to the shared counters once both warpgroups turned
    // item li-1's counts into log2 (and zeroed them); 16-bit counters, two per word
    const int ct = threadIdx.x - 320;  // 0..63
    const IdxT* idx = static_cast<const IdxT*>(p.idx);
    for (int i = ct * 4; i < 2 * 2 * kMaxNkv / 2; i += 64 * 4)
      *reinterpret_cast<uint4*>(&cnt32[i]) = make_uint4(0u, 0u, 0u, 0u);
    named_bar_sync(3, 64);
    int li = 0;
    bool ok = true;
    for (int64_t item = blockIdx.x; item < p.total_items; item += gridDim.x, ++li) {
      bool okw = true;
      for (int w = 0; w < 2; ++w)
        okw = okw && mbar_wait(&cnt_empty[w], (li & 1) ^ 1, abort_flag, p.err, DSA_DEVERR_SA_WAIT);
      ok = named_bar_and(3, 64, okw);
      if (!ok) break;
      for (int w = 0; w < 2; ++w) {
        int b, tb;
        bool valid;
        tile_of(item, w, b, tb, valid);
        int maxidx = -1;
        if (valid) {
          const int64_t tok0 = static_cast<int64_t>(tb) * kRows / p.heads;
          uint32_t* wcnt = cnt32 + w * kMaxNkv;
          if (p.mask != nullptr) {
            // selection bitmaps (one per token): every set bit counts once
            const uint32_t* msrc = p.mask + (static_cast<int64_t>(b) * p.m + tok0) * p.mask_words;
            const int n_w = p.tpt * p.mask_words;
            for (int i = ct; i < n_w; i += 64) {
              const int tk = i / p.mask_words;
              const int64_t kb = static_cast<int64_t>(i - tk * p.mask_words) * 32 + p.mask_offset;
              uint32_t bits = __ldg(msrc + i);
              while (bits) {
                const int jb = __ffs(static_cast<int>(bits)) - 1;
                bits &= bits - 1u;
                const int64_t k = kb + jb;
                if (k >= 0 && k < p.nkv) {
                  const int kk = static_cast<int>(k);
                  atomicAdd(&wcnt[tk * (kMaxNkv / 2) + (kk >> 1)], 1u << ((kk & 1) * 16));
                  maxidx = max(maxidx, kk);
                }
              }
            }
          } else {
          const IdxT* src = idx + (static_cast<int64_t>(b) * p.m + tok0) * p.topk;
          const int n_ent = p.tpt * p.topk;
          // batches of 8 independent loads ahead of their shared-memory atomics
          for (int i0 = 0; i0 < n_ent; i0 += 8 * 64) {
            int64_t kb[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
              const int i = i0 + u * 64 + ct;
              kb[u] = i < n_ent ? static_cast<int64_t>(__ldg(src + i)) : -1;
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) {
              const int64_t k = kb[u];
              if (k >= 0 && k < p.nkv) {
                const int i = i0 + u * 64 + ct;
                const int kk = static_cast<int>(k);
                atomicAdd(&wcnt[(i / p.topk) * (kMaxNkv / 2) + (kk >> 1)], 1u << ((kk & 1) * 16));
                maxidx = max(maxidx, kk);
              }
            }
          }
          }
        }
        maxidx = __reduce_max_sync(0xFFFFFFFFu, maxidx);
        if (lane == 0) red[2 * (warp - 10) + w] = maxidx;
      }
      // the TMA and MMA warps have read this slot's chunk counts of item li-2
      const bool okm = mbar_wait(&meta_empty[li & 1], ((li >> 1) & 1) ^ 1, abort_flag, p.err,
                                 DSA_DEVERR_SA_WAIT);
      ok = named_bar_and(3, 64, okm);
      if (!ok) break;
      if (ct == 0) {
        for (int w = 0; w < 2; ++w) {
          int b, tb;
          bool valid;
          tile_of(item, w, b, tb, valid);
          const int mx = max(red[w], red[2 + w]);
          meta[2 * w + (li & 1)] = valid ? (mx + kChunk) / kChunk : 0;  // chunks with a counted row
          mbar_arrive(&meta_full[2 * w + (li & 1)]);
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

template <typename IdxT>
int launch(const void* q, const void* kv, const void* idx, const uint32_t* mask, int mask_words,
           int64_t mask_offset, const float* sink, void* out, int64_t batch, int64_t m, int heads,
           int nkv, int topk, float scale, cudaStream_t stream) {
  DeviceInfo di;
  int st = current_device_info(&di);
  if (st != DSA_OK) return st;
  if (di.max_smem_optin < kSmemBytes) return DSA_ERR_UNSUPPORTED;
  unsigned int* err = nullptr;
  st = device_error_word(&err);
  if (st != DSA_OK) return st;
  const int64_t rows = m * heads;
  if (rows % kRows != 0) return DSA_ERR_UNSUPPORTED;  // whole tokens per tile
  const int64_t tiles = rows / kRows;
  const int64_t items_pb = (tiles + 1) / 2;
  if (tiles > 0x7FFFFFFF || batch * items_pb > (int64_t{1} << 40)) return DSA_ERR_UNSUPPORTED;
  CUtensorMap tm_q, tm_kv, tm_out;
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
    const uint32_t box[3] = {64, kChunk, 1};
    st = encode_tensor_map(&tm_kv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, kv, dims, strides, box,
                           CU_TENSOR_MAP_SWIZZLE_128B);
    if (st != DSA_OK) return st;
  }
  Params p;
  p.m = m;
  p.heads = heads;
  p.tpt = kRows / heads;
  p.tiles_per_batch = static_cast<int>(tiles);
  p.items_per_batch = static_cast<int>(items_pb);
  p.total_items = items_pb * batch;
  p.topk = topk;
  p.nkv = nkv;
  p.scale_log2 = scale * kLog2e;
  p.sink = sink;
  p.idx = idx;
  p.mask = mask;
  p.mask_words = mask_words;
  p.mask_offset = mask_offset;
  p.err = err;
  st = set_max_dynamic_smem(reinterpret_cast<const void*>(sa_long_kernel<int32_t>), kSmemBytes);
  if (st == DSA_OK)
    st = set_max_dynamic_smem(reinterpret_cast<const void*>(sa_long_kernel<int64_t>), kSmemBytes);
  if (st != DSA_OK) return st;
  const int64_t grid64 = p.total_items < di.num_sms ? p.total_items : di.num_sms;
  sa_long_kernel<IdxT><<<static_cast<unsigned>(grid64), kThreads, kSmemBytes, stream>>>(
      tm_q, tm_kv, tm_out, p);
  return cuda_status(cudaGetLastError());
}

}  // namespace sal

// Long-pool SparseAttention: heads in {64, 128}, head_dim 128, n_kv <= 4096.
bool sa_long_supported(int heads, int head_dim, int nkv) {
  return (heads == 64 || heads == 128) && head_dim == sal::kD && nkv >= 1 && nkv <= sal::kMaxNkv;
}

int launch_sa_long(const void* q, const void* kv, const void* idx, int idx_elem_bytes,
                   const float* sink, void* out, int64_t batch, int64_t m, int heads, int nkv,
                   int topk, float scale, cudaStream_t stream) {
  if (idx_elem_bytes == 8)
    return sal::launch<int64_t>(q, kv, idx, nullptr, 0, 0, sink, out, batch, m, heads, nkv, topk,
                                scale, stream);
  return sal::launch<int32_t>(q, kv, idx, nullptr, 0, 0, sink, out, batch, m, heads, nkv, topk,
                              scale, stream);
}

// Long-pool SparseAttention whose per-token selection comes as bitmaps
// [batch, m, mask_words] (bit k: pool row k + mask_offset is selected once), as
// written by the indexer's top-k set kernel: the chained path's hand-off.
int launch_sa_long_mask(const void* q, const void* kv, const uint32_t* mask, int mask_words,
                        int64_t mask_offset, const float* sink, void* out, int64_t batch,
                        int64_t m, int heads, int nkv, float scale, cudaStream_t stream) {
  return sal::launch<int32_t>(q, kv, nullptr, mask, mask_words, mask_offset, sink, out, batch, m,
                              heads, nkv, 0, scale, stream);
}

}  // namespace dsa
