// kv_cache writer for sm_100a: the producer of the compressed index-key cache
// that the Lightning Indexer reads (reference/task2_v0_ref.py:119,133 read
// kv_cache[:bsz, :end_pos // ratio]; the reference holds no producer). Restated
// from the indexer key path of DeepSeek-V3.2-Exp (inference/model.py,
// Indexer.forward), with the rotary dims last as this reference's q, and
// blocks of `ratio` tokens pooled by their mean:
//
//   kl[t] = bf16(x[t] . wk^T)              tcgen05 bf16 MMA, fp32 accumulate
//   kn[t] = bf16(LayerNorm(kl[t]) * g + b) fp32, eps 1e-6, sums in index order
//   k[t]  = RoPE(kn[t][64-rd:], position start_pos + t), bf16
//   kv[b, start_pos / ratio + j] = bf16(mean_i k[j ratio + i]), i < ratio
//
// Persistent: one CTA per SM (320 threads) walks the 128-token tiles of all
// batches. Warp 0 streams TMA chunks (x tile 128 x 64 and wk 64 x 64 per 64-wide
// k chunk, SW128) through a 5-stage ring without stopping between tiles; warp 1
// owns 128 TMEM columns and issues the tcgen05 MMAs (D[128 tokens x 64], four
// K = 16 MMAs per chunk) into two accumulators, alternating tiles; warps 2-5 and
// 6-9 are two epilogue warpgroups, one per accumulator (one token per thread:
// the tile's RoPE factors staged in shared memory by coalesced loads while the
// accumulator fills, the LayerNorm and RoPE chain, the key staged in the
// group's shared-memory buffer, then the block means written as 16-byte rows),
// so each group has two tiles' load time for one tile's chain. Roofline: HBM, x read once
// (dim * 2 bytes per token), 128 / ratio bytes written per token.
#include "common.cuh"
#include "host_util.h"
#include "numerics.cuh"

namespace dsa {
namespace kvw {

constexpr int kTile = 128;
constexpr int kN = 64;
constexpr int kKC = 64;                   // k per chunk
constexpr int kStages = 5;
constexpr int kThreads = 320;
constexpr int kABytes = kTile * kKC * 2;  // 16 KB
constexpr int kBBytes = kN * kKC * 2;     // 8 KB
constexpr int kStageBytes = kABytes + kBBytes;
constexpr int kOffStage = 0;
constexpr int kOffKeys = kStages * kStageBytes;        // [2 groups][128][64] bf16
constexpr int kOffAffine = kOffKeys + 2 * kTile * kN * 2;  // LayerNorm weight, bias (f32)
constexpr int kRopeStride = kN / 2 + 1;  // floats per token row of a staged table (odd: no bank conflicts)
constexpr int kRopeTable = kTile * kRopeStride * 4;
constexpr int kOffRope = kOffAffine + 2 * kN * 4;          // [2 groups][cos, sin][128][33] f32
constexpr int kOffBar = kOffRope + 4 * kRopeTable;
constexpr int kNumBars = 2 * kStages + 5;  // full, empty, acc_full[2], tmem_empty[2], done
constexpr int kOffMisc = kOffBar + kNumBars * 8;
constexpr int kSmem = kOffMisc + 16 + 1024;
constexpr uint32_t kTmemCols = 128;  // two 64-column accumulators

struct Params {
  int64_t S;
  int64_t ntiles;
  int tiles_per_batch;
  int dim;
  int rope_dim;
  int rope_vec;  // RoPE tables 16-byte aligned with rope_dim / 2 a multiple of 4
  int ratio;
  int64_t entry0;      // start_pos / ratio
  int64_t kv_bstride;  // elements
  const float* g;
  const float* b;
  const float* cos_t;  // [S, rope_dim / 2]
  const float* sin_t;
  uint16_t* kv;
  unsigned int* err;
};

__global__ void __launch_bounds__(kThreads, 1)
    kv_writer_kernel(const __grid_constant__ CUtensorMap tm_x,
                     const __grid_constant__ CUtensorMap tm_w, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* empty = full + kStages;
  uint64_t* acc_full = empty + kStages;  // [2]
  uint64_t* tmem_empty = acc_full + 2;   // [2]
  uint64_t* mma_done = tmem_empty + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kOffMisc + 4);
  float* affine = reinterpret_cast<float*>(smem + kOffAffine);  // g[64], b[64]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nchunks = p.dim / kKC;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&tmem_empty[i], 4);  // one arrival per warp of the accumulator's group
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (threadIdx.x >= 64 && threadIdx.x < 64 + 2 * kN)
    affine[threadIdx.x - 64] = threadIdx.x < 64 + kN ? p.g[threadIdx.x - 64]
                                                     : p.b[threadIdx.x - 64 - kN];
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_x);
    tma_prefetch_desc(&tm_w);
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
      int it = 0;
      bool ok = true;
      for (int64_t tile = blockIdx.x; ok && tile < p.ntiles; tile += gridDim.x) {
        const int64_t bi = tile / p.tiles_per_batch;
        const int64_t t0 = (tile % p.tiles_per_batch) * kTile;
        const int32_t row0 = static_cast<int32_t>(bi * p.S + t0);
        for (int c = 0; c < nchunks; ++c, ++it) {
          const int s = it % kStages;
          if (!mbar_wait(&empty[s], ((it / kStages) & 1) ^ 1, abort_flag, p.err,
                         DSA_DEVERR_GEMM_WAIT)) {
            ok = false;
            break;
          }
          uint8_t* st = smem + kOffStage + s * kStageBytes;
          mbar_arrive_expect_tx(&full[s], kStageBytes);
          tma_load_2d(st, &tm_x, c * kKC, row0, &full[s]);
          tma_load_2d(st + kABytes, &tm_w, c * kKC, 0, &full[s]);
        }
      }
      // copies in flight complete before the CTA exits (a no-op unless aborted)
      for (int i = (it > kStages ? it - kStages : 0); i < it; ++i)
        mbar_drain(&full[i % kStages], (i / kStages) & 1);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_bf16_f32(kTile, kN, 0, 0);
      int it = 0, lt = 0;
      bool ok = true;
      for (int64_t tile = blockIdx.x; ok && tile < p.ntiles; tile += gridDim.x, ++lt) {
        const int buf = lt & 1;
        if (!mbar_wait(&tmem_empty[buf], ((lt >> 1) & 1) ^ 1, abort_flag, p.err,
                       DSA_DEVERR_GEMM_WAIT))
          break;
        tc_fence_after();
        const uint32_t d = tmem + static_cast<uint32_t>(buf * kN);
        for (int c = 0; c < nchunks; ++c, ++it) {
          const int s = it % kStages;
          if (!mbar_wait(&full[s], (it / kStages) & 1, abort_flag, p.err, DSA_DEVERR_GEMM_WAIT)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a = smem_u32(smem + kOffStage + s * kStageBytes);
          const uint32_t bb = a + kABytes;
#pragma unroll
          for (int k = 0; k < kKC / 16; ++k) {
            const uint64_t ad = make_smem_desc(a + k * 32, 16u, 1024u, kLayoutSW128);
            const uint64_t bd = make_smem_desc(bb + k * 32, 16u, 1024u, kLayoutSW128);
            umma_bf16(d, ad, bd, idesc, (c > 0 || k > 0) ? 1u : 0u);
          }
          umma_commit(&empty[s]);
        }
        if (ok) umma_commit(&acc_full[buf]);
      }
      // every MMA issued has finished before TMEM is freed
      umma_commit(mma_done);
      mbar_drain(mma_done, 0);
    }
  } else {
    // ------------------------------------------------------------- epilogue
    // group g (warps 2-5 or 6-9) takes the CTA's tiles lt = g, g + 2, ... from
    // accumulator g
    const int grp = (warp - 2) >> 2;
    const int quarter = warp & 3;         // TMEM lanes this warp may read
    const int row = quarter * 32 + lane;  // token of the tile = TMEM lane
    const int et = row;                   // 0..127 within the group
    const uint32_t bar_id = 1 + grp;
    uint16_t* keys = reinterpret_cast<uint16_t*>(smem + kOffKeys) + grp * kTile * kN;
    const float4* g4 = reinterpret_cast<const float4*>(affine);
    const float4* b4 = reinterpret_cast<const float4*>(affine + kN);
    const int half = p.rope_dim / 2;
    const int base = kN - p.rope_dim;
    const float inv_r = __frcp_rn(static_cast<float>(p.ratio));  // a power of two: exact
    int lt = grp;
    for (int64_t tile = blockIdx.x + static_cast<int64_t>(grp) * gridDim.x; tile < p.ntiles;
         tile += 2 * static_cast<int64_t>(gridDim.x), lt += 2) {
      const int64_t bi = tile / p.tiles_per_batch;
      const int64_t t0 = (tile % p.tiles_per_batch) * kTile;
      // stage the tile's RoPE factors (coalesced rows [t0, t0 + 128) of the tables)
      // while the accumulator fills; read back after the barrier below
      float* rc = reinterpret_cast<float*>(smem + kOffRope + grp * 2 * kRopeTable);
      float* rsn = rc + kTile * kRopeStride;
      if (half > 0) {
        const int64_t nv = p.S - t0 < kTile ? p.S - t0 : kTile;
        const int nel = static_cast<int>(nv) * half;
        const float* gc = p.cos_t + t0 * half;
        const float* gsn = p.sin_t + t0 * half;
        if (p.rope_vec) {  // 16-byte rows: float4 loads
          for (int i = et; i < nel / 4; i += 128) {
            const float4 c4 = __ldg(reinterpret_cast<const float4*>(gc) + i);
            const float4 s4 = __ldg(reinterpret_cast<const float4*>(gsn) + i);
            const int tok = (4 * i) / half, j = (4 * i) % half;
            float* dc = rc + tok * kRopeStride + j;
            float* ds = rsn + tok * kRopeStride + j;
            dc[0] = c4.x; dc[1] = c4.y; dc[2] = c4.z; dc[3] = c4.w;
            ds[0] = s4.x; ds[1] = s4.y; ds[2] = s4.z; ds[3] = s4.w;
          }
        } else {
          for (int i = et; i < nel; i += 128) {
            rc[(i / half) * kRopeStride + i % half] = __ldg(gc + i);
            rsn[(i / half) * kRopeStride + i % half] = __ldg(gsn + i);
          }
        }
      }
      bool ok = __all_sync(0xFFFFFFFFu, mbar_wait(&acc_full[grp], (lt >> 1) & 1, abort_flag,
                                                  p.err, DSA_DEVERR_GEMM_WAIT));
      // also orders this tile's key writes after every thread's reads of the last one,
      // and the staged RoPE factors before their reads
      if (!named_bar_and(bar_id, 128, ok)) break;
      tc_fence_after();
      uint32_t r0[32], r1[32];
      const uint32_t ta = tmem + static_cast<uint32_t>(grp * kN) +
                          (static_cast<uint32_t>(quarter * 32) << 16);
      tmem_ld_32x32b_x32(ta, r0);
      tmem_ld_32x32b_x32(ta + 32, r1);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tmem_empty[grp]);  // the MMA may refill this accumulator
      // kl = bf16(accumulator), two per conversion
      float v[kN];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const uint32_t a = pack_bf16x2(__uint_as_float(r0[2 * i]), __uint_as_float(r0[2 * i + 1]));
        const uint32_t c = pack_bf16x2(__uint_as_float(r1[2 * i]), __uint_as_float(r1[2 * i + 1]));
        v[2 * i] = __uint_as_float(a << 16);
        v[2 * i + 1] = __uint_as_float(a & 0xFFFF0000u);
        v[32 + 2 * i] = __uint_as_float(c << 16);
        v[32 + 2 * i + 1] = __uint_as_float(c & 0xFFFF0000u);
      }
      // LayerNorm over the 64 values, sums in index order, every op rounded once
      // (x / 64 and x / ratio as products with the exact reciprocal)
      float s = 0.f;
#pragma unroll
      for (int i = 0; i < kN; ++i) s = __fadd_rn(s, v[i]);
      const float mu = __fmul_rn(s, 1.0f / 64.0f);
      const int64_t t = t0 + row;
      const bool rope = t < p.S;
      float q = 0.f;
#pragma unroll
      for (int i = 0; i < kN; ++i) {
        v[i] = __fsub_rn(v[i], mu);
        q = __fadd_rn(q, __fmul_rn(v[i], v[i]));
      }
      const float rstd =
          __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fmul_rn(q, 1.0f / 64.0f), 1e-6f)));
      uint32_t kb[kN / 2];  // bf16 pairs
#pragma unroll
      for (int i4 = 0; i4 < kN / 4; ++i4) {
        const float4 gg = g4[i4], bb = b4[i4];
        const float n0 = __fadd_rn(__fmul_rn(__fmul_rn(v[4 * i4], rstd), gg.x), bb.x);
        const float n1 = __fadd_rn(__fmul_rn(__fmul_rn(v[4 * i4 + 1], rstd), gg.y), bb.y);
        const float n2 = __fadd_rn(__fmul_rn(__fmul_rn(v[4 * i4 + 2], rstd), gg.z), bb.z);
        const float n3 = __fadd_rn(__fmul_rn(__fmul_rn(v[4 * i4 + 3], rstd), gg.w), bb.w);
        kb[2 * i4] = pack_bf16x2(n0, n1);
        kb[2 * i4 + 1] = pack_bf16x2(n2, n3);
      }
      // RoPE on the last rope_dim dims (interleaved pairs) at the token's position
#pragma unroll
      for (int j = 0; j < kN / 2; ++j) {
        if (rope && 2 * j >= base) {
          const int jj = j - base / 2;
          const float c = rc[row * kRopeStride + jj], sn = rsn[row * kRopeStride + jj];
          const float re = __uint_as_float(kb[j] << 16);
          const float im = __uint_as_float(kb[j] & 0xFFFF0000u);
          kb[j] = pack_bf16x2(__fsub_rn(__fmul_rn(re, c), __fmul_rn(im, sn)),
                              __fadd_rn(__fmul_rn(re, sn), __fmul_rn(im, c)));
        }
      }
      // the row's 16-byte chunk i sits at slot i ^ (row & 7): conflict-free stores
      uint4* dst = reinterpret_cast<uint4*>(keys + row * kN);
#pragma unroll
      for (int i = 0; i < 8; ++i)
        dst[i ^ (row & 7)] = make_uint4(kb[4 * i], kb[4 * i + 1], kb[4 * i + 2], kb[4 * i + 3]);
      named_bar_sync(bar_id, 128);
      // block means: (block, 8-dim group) items over the group's 128 threads
      const int64_t valid = p.S - t0 < kTile ? p.S - t0 : kTile;
      const int nb = static_cast<int>(valid / p.ratio);
      for (int item = et; item < nb * 8; item += 128) {
        const int j = item >> 3, c8 = item & 7;
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (int i = 0; i < p.ratio; ++i) {
          const int kr = j * p.ratio + i;
          const uint4 w = reinterpret_cast<const uint4*>(keys + kr * kN)[c8 ^ (kr & 7)];
          const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            acc[2 * e] = __fadd_rn(acc[2 * e], __uint_as_float(ww[e] << 16));
            acc[2 * e + 1] = __fadd_rn(acc[2 * e + 1], __uint_as_float(ww[e] & 0xFFFF0000u));
          }
        }
        uint32_t o[4];
#pragma unroll
        for (int e = 0; e < 4; ++e)
          o[e] = pack_bf16x2(__fmul_rn(acc[2 * e], inv_r), __fmul_rn(acc[2 * e + 1], inv_r));
        uint16_t* out = p.kv + bi * p.kv_bstride + (p.entry0 + t0 / p.ratio + j) * kN + c8 * 8;
        *reinterpret_cast<uint4*>(out) = make_uint4(o[0], o[1], o[2], o[3]);
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

}  // namespace kvw

int launch_kv_writer(const void* x, const void* wk, const float* g, const float* b,
                     const float* cos_t, const float* sin_t, void* kv, int64_t kv_bstride,
                     int64_t batch, int64_t seqlen, int dim, int rope_dim, int64_t start_pos,
                     int ratio, cudaStream_t stream) {
  using namespace kvw;
  DeviceInfo di;
  int st = current_device_info(&di);
  if (st != DSA_OK) return st;
  if (di.max_smem_optin < kSmem) return DSA_ERR_UNSUPPORTED;
  unsigned int* err = nullptr;
  st = device_error_word(&err);
  if (st != DSA_OK) return st;
  CUtensorMap tm_x, tm_w;
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(dim), static_cast<uint64_t>(batch * seqlen)};
    const uint64_t strides[1] = {static_cast<uint64_t>(dim) * 2};
    const uint32_t box[2] = {kKC, kTile};
    st = encode_tensor_map(&tm_x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, x, dims, strides, box,
                           CU_TENSOR_MAP_SWIZZLE_128B);
    if (st != DSA_OK) return st;
  }
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(dim), static_cast<uint64_t>(kN)};
    const uint64_t strides[1] = {static_cast<uint64_t>(dim) * 2};
    const uint32_t box[2] = {kKC, kN};
    st = encode_tensor_map(&tm_w, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, wk, dims, strides, box,
                           CU_TENSOR_MAP_SWIZZLE_128B);
    if (st != DSA_OK) return st;
  }
  Params p;
  p.S = seqlen;
  p.tiles_per_batch = static_cast<int>((seqlen + kTile - 1) / kTile);
  p.ntiles = batch * p.tiles_per_batch;
  p.dim = dim;
  p.rope_dim = rope_dim;
  p.rope_vec = (rope_dim % 8 == 0) && aligned16(cos_t) && aligned16(sin_t) ? 1 : 0;
  p.ratio = ratio;
  p.entry0 = start_pos / ratio;
  p.kv_bstride = kv_bstride;
  p.g = g;
  p.b = b;
  p.cos_t = cos_t;
  p.sin_t = sin_t;
  p.kv = static_cast<uint16_t*>(kv);
  p.err = err;
  st = set_max_dynamic_smem(reinterpret_cast<const void*>(kv_writer_kernel), kSmem);
  if (st != DSA_OK) return st;
  const int64_t grid = p.ntiles < di.num_sms ? p.ntiles : di.num_sms;
  kv_writer_kernel<<<static_cast<unsigned>(grid), kThreads, kSmem, stream>>>(tm_x, tm_w, p);
  return cuda_status(cudaGetLastError());
}

}  // namespace dsa
