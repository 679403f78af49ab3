// Warp-level top-K of up to 1024 32-bit keys held in shared memory, output in
// descending key order with ties by ascending position (the index order the
// keys are stored in), as int64 position + offset, -1 past the selected count.
//
// One warp, three phases with short dependency chains:
//  1. threshold: the keys' highest differing bit (two warp reductions), then an
//     8-bit radix histogram per round (shared-memory atomics) over the keys
//     still in the boundary range, a descending scan of the 256 bins across the
//     lanes and the bin where the count reaches K: 1-4 rounds instead of a
//     32-step bit search;
//  2. compaction: keys above the threshold, and keys equal to it in ascending
//     position up to K, placed by two sets of independent ballots;
//  3. sort: a bitonic network on (key << 32 | ~position) laid out lane-major
//     (element i = lane * E + e), so that the strides below E are exchanges
//     inside a lane and only 15 of the 28 stages (K = 128) need shuffles.
// Scratch: the key list itself (read into registers first): its first 2 KB take
// the compacted entries, the next 1 KB the radix bins.
#pragma once

#include <stdint.h>

namespace dsa {
namespace wsel {

constexpr unsigned kFull = 0xFFFFFFFFu;

// Threshold of the n keys v (key i = r * 32 + lane, valid for i < n) for
// ksel < n: the largest thr with at least ksel keys >= thr, and need = ksel -
// #(keys > thr). hist: 256 u32 of warp-private shared memory.
template <int R>
__device__ __forceinline__ void radix_threshold(const uint32_t (&v)[R], int n, int ksel,
                                                uint32_t* hist, int lane, uint32_t& thr,
                                                int& need) {
  uint32_t mx = 0u, mn = 0xFFFFFFFFu;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    if (r * 32 + lane < n) {
      mx = max(mx, v[r]);
      mn = min(mn, v[r]);
    }
  }
  mx = __reduce_max_sync(kFull, mx);
  mn = __reduce_min_sync(kFull, mn);
  if (mx == mn) {  // every key equal: the first ksel positions
    thr = mx;
    need = ksel;
    return;
  }
  // bits [shift, 32) are common to all keys; the candidate range is the keys
  // whose bits [shift, 32) equal `prefix` (all of them at first)
  int shift = 32 - __clz(mx ^ mn);
  uint32_t prefix = shift >= 32 ? 0u : (mx >> shift);
  int above = 0;  // keys above the candidate range
  for (int round = 0; round < 4; ++round) {
    const int lo = shift > 8 ? shift - 8 : 0;
    const int nb = shift - lo;
    const uint32_t mask = (1u << nb) - 1u;
#pragma unroll
    for (int j = 0; j < 8; ++j) hist[lane * 8 + j] = 0u;
    __syncwarp();
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const bool in = r * 32 + lane < n && (shift >= 32 || (v[r] >> shift) == prefix);
      if (in) atomicAdd(&hist[(v[r] >> lo) & mask], 1u);
    }
    __syncwarp();
    // lane L holds bins 255 - 8L - j, j = 0..7 (descending)
    const uint4 h1 = *reinterpret_cast<const uint4*>(hist + 248 - 8 * lane);
    const uint4 h0 = *reinterpret_cast<const uint4*>(hist + 252 - 8 * lane);
    const int c[8] = {static_cast<int>(h0.w), static_cast<int>(h0.z), static_cast<int>(h0.y),
                      static_cast<int>(h0.x), static_cast<int>(h1.w), static_cast<int>(h1.z),
                      static_cast<int>(h1.y), static_cast<int>(h1.x)};
    int ls = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) ls += c[j];
    int incl = ls;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(kFull, incl, o);
      if (lane >= o) incl += t;
    }
    const int rem = ksel - above;  // >= 1
    const int excl = incl - ls;
    const unsigned bal = __ballot_sync(kFull, excl < rem && rem <= incl);
    const int L = __ffs(bal) - 1;
    int bj = 0, bef = excl, cnt = 0;
    {
      int acc = excl;
      bool found = false;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (!found && acc + c[j] >= rem) {
          found = true;
          bj = j;
          bef = acc;
          cnt = c[j];
        }
        acc += c[j];
      }
    }
    bj = __shfl_sync(kFull, bj, L);
    bef = __shfl_sync(kFull, bef, L);
    cnt = __shfl_sync(kFull, cnt, L);
    const uint32_t bin = static_cast<uint32_t>(255 - (L * 8 + bj));
    above += bef;
    prefix = (shift >= 32 ? 0u : (prefix << nb)) | bin;
    shift = lo;
    if (lo == 0) {  // the range is one key value
      thr = prefix;
      need = ksel - above;
      return;
    }
    if (cnt == ksel - above && prefix != 0u) {  // the whole range is taken
      thr = (prefix << lo) - 1u;
      need = 0;
      return;
    }
    __syncwarp();  // bins read before the next round clears them
  }
  thr = prefix << shift;  // not reached: four rounds cover 32 bits
  need = ksel - above;
}

// Lane-major bitonic sort, descending, of 32 * E 64-bit keys (element i = lane
// * E + e in v[e]).
template <int E>
__device__ __forceinline__ void bitonic_desc_lane_major(uint64_t (&v)[E], int lane) {
#pragma unroll
  for (int size = 2; size <= 32 * E; size <<= 1) {
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      if (stride < E) {
#pragma unroll
        for (int e = 0; e < E; ++e) {
          if ((e & stride) == 0) {
            const int i = lane * E + e;
            const bool desc = (i & size) == 0;
            const uint64_t a = v[e], b = v[e | stride];
            const bool sw = desc ? (a < b) : (a > b);
            v[e] = sw ? b : a;
            v[e | stride] = sw ? a : b;
          }
        }
      } else {
        const int lx = stride / E;
#pragma unroll
        for (int e = 0; e < E; ++e) {
          const int i = lane * E + e;
          const uint64_t o = __shfl_xor_sync(kFull, v[e], lx);
          const bool keep_max = (((i & stride) == 0) == ((i & size) == 0));
          v[e] = keep_max ? (v[e] > o ? v[e] : o) : (v[e] < o ? v[e] : o);
        }
      }
    }
  }
}

template <int E>
__device__ __forceinline__ void sort_store(const uint64_t* sel, int nsel, int64_t* out, int K_out,
                                           int64_t offset, int lane) {
  uint64_t v[E];
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const int i = lane * E + e;
    v[e] = i < nsel ? sel[i] : 0ull;
  }
  bitonic_desc_lane_major<E>(v, lane);
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const int i = lane * E + e;
    if (i < K_out)
      out[i] = i < nsel ? static_cast<int64_t>(0xFFFFFFFFu - static_cast<uint32_t>(v[e])) + offset
                        : static_cast<int64_t>(-1);
  }
}

// Top-K_out of the n keys at `keys` (smem, 16-byte aligned, >= 3 KB, overwritten);
// K_out <= 256, n <= 32 * R. A real key must be nonzero... any value is fine:
// validity comes from the position, not the key.
template <int R>
__device__ __forceinline__ void select_sorted(uint32_t* keys, int n, int K_out, int64_t* out,
                                              int64_t offset, int lane) {
  const int ksel = n < K_out ? n : K_out;
  const uint32_t lt = (1u << lane) - 1u;
  uint32_t v[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int i = r * 32 + lane;
    v[r] = i < n ? keys[i] : 0u;
  }
  __syncwarp();  // the list is scratch from here on
  uint64_t* sel = reinterpret_cast<uint64_t*>(keys);
  uint32_t* hist = keys + 512;
  const bool all = n <= ksel;
  uint32_t thr = 0u;
  int need = 0;
  if (!all) radix_threshold<R>(v, n, ksel, hist, lane, thr, need);
  uint32_t tb[R];
#pragma unroll
  for (int r = 0; r < R; ++r)
    tb[r] = __ballot_sync(kFull, !all && need > 0 && r * 32 + lane < n && v[r] == thr);
  uint32_t tk[R];
  int ties = 0;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const bool valid = r * 32 + lane < n;
    const bool tie = (tb[r] >> lane) & 1u;
    const bool take = valid && (all || v[r] > thr || (tie && ties + __popc(tb[r] & lt) < need));
    ties += __popc(tb[r]);
    tk[r] = __ballot_sync(kFull, take);
  }
  int base = 0;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    if ((tk[r] >> lane) & 1u)
      sel[base + __popc(tk[r] & lt)] =
          (static_cast<uint64_t>(v[r]) << 32) | (0xFFFFFFFFu - static_cast<uint32_t>(r * 32 + lane));
    base += __popc(tk[r]);
  }
  __syncwarp();
  if (K_out <= 128)
    sort_store<4>(sel, base, out, K_out, offset, lane);
  else
    sort_store<8>(sel, base, out, K_out, offset, lane);
  __syncwarp();
}

__device__ __forceinline__ void select_sorted_any(uint32_t* keys, int n, int K_out, int64_t* out,
                                                  int64_t offset, int lane) {
  if (n <= 256)
    select_sorted<8>(keys, n, K_out, out, offset, lane);
  else if (n <= 512)
    select_sorted<16>(keys, n, K_out, out, offset, lane);
  else if (n <= 768)
    select_sorted<24>(keys, n, K_out, out, offset, lane);
  else
    select_sorted<32>(keys, n, K_out, out, offset, lane);
}

}  // namespace wsel
}  // namespace dsa
