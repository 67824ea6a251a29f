// Top-K index producer: the step before the decode path. For each row of a
// [rows, ctx] fp32 score matrix it writes the positions of the K highest
// scores, in ascending position order, as the int32 Top-K indices the decode
// reads (-1 padding). The reference consumes such indices but does not make
// them (its fixtures are sequential, sm89_cutedsl.py:72-76).
//
// Rule: a position t of row r is a candidate when t < len[r] (ctx without
// lengths) and its score is neither NaN nor -inf. The K candidates with the
// highest scores are taken; at the K-th score, lower positions win. Fewer
// than K candidates: all of them, then -1.
//
// One CTA of 1024 threads per row, two CTAs per SM. Scores map to
// order-preserving uint32 keys; a radix select over three digits of 11, 11
// and 10 bits gives the threshold key T and how many keys equal to T to take.
// The row is read three times, the last two from L2:
//   1. histogram of the top digit (bits 31..21) in shared memory; a block
//      prefix sum over the bins finds the digit d1 that holds the K-th key;
//   2. the keys whose top digit is d1 (the threshold bucket, a few percent of
//      the row for smooth score distributions) are appended to a buffer in
//      shared memory, and the two lower digits are selected from the buffer
//      alone. A bucket larger than the buffer (heavy ties, very long rows)
//      takes both lower digits over the row instead;
//   3. ordered compaction over tiles of 32768 positions: each thread flags
//      its positions (key > T, key == T) for 8 groups of 4 consecutive
//      positions, warp scans give each lane's offsets, and ONE block scan over
//      the 256 (group, warp) counts gives every group's offset, so a
//      position's output slot is (# greater before it) + min(# equal before
//      it, equal keys to take).
// Scores are read as float4 when the row start and stride allow it.
#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/qsa_b200.h"
#include "qsa_internal.h"

namespace qsa {
namespace {

constexpr int kTopkThreads = 1024;
constexpr int kTopkWarps = kTopkThreads / 32;
constexpr int kGroups = 8;                              // 4-position groups per thread per tile
constexpr int kTilePositions = 4 * kTopkThreads * kGroups;  // 32768
constexpr int kCandidates = 8192;                       // threshold-bucket buffer (keys)

// order-preserving key of a score; 0 for a position that is not a candidate
__device__ __forceinline__ uint32_t score_key(float s) {
  const uint32_t u = __float_as_uint(s);
  if (s != s || s == -INFINITY) return 0u;  // NaN or -inf
  if (s == 0.f) return 0x80000000u;          // -0 and +0 are the same score
  const uint32_t k = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return k == 0u ? 1u : k;  // 0 is reserved for non-candidates
}

// Keys of positions t .. t+3 of the row (0 at and past len). kVec: the row
// start is 16-byte aligned and t + 3 < ctx whenever t < len (ctx % 4 == 0).
template <bool kVec>
__device__ __forceinline__ void load_keys(const float* sc, int t, int len, uint32_t (&key)[4]) {
  if (kVec) {
    if (t < len) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(sc + t));
      key[0] = score_key(v.x);
      key[1] = t + 1 < len ? score_key(v.y) : 0u;
      key[2] = t + 2 < len ? score_key(v.z) : 0u;
      key[3] = t + 3 < len ? score_key(v.w) : 0u;
    } else {
      key[0] = key[1] = key[2] = key[3] = 0u;
    }
  } else {
#pragma unroll
    for (int u = 0; u < 4; ++u) key[u] = t + u < len ? score_key(__ldg(sc + t + u)) : 0u;
  }
}

// exclusive block prefix sum of one value per thread; also returns the total
__device__ __forceinline__ int block_scan(int v, int* warp_sums, int& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_sums[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = warp_sums[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    warp_sums[lane] = w;  // inclusive
  }
  __syncthreads();
  total = warp_sums[kTopkWarps - 1];
  const int before = (warp > 0 ? warp_sums[warp - 1] : 0) + x - v;
  __syncthreads();  // warp_sums is reused by the next scan
  return before;
}

struct TopkShared {
  int hist[2048];
  int warp_sums[kTopkWarps];
  uint32_t cand[kCandidates];       // keys of the threshold bucket
  uint32_t counts[kGroups * kTopkWarps];  // compaction: (greater | equal << 16) per (group, warp)
  uint32_t sel_prefix, sel_mask;
  int sel_remaining, bucket, n_cand;
};

// Digit search of one radix pass: with hist[] holding the counts of the
// digits (nb bins, bits shift .. shift + log2(nb) - 1) among the keys that
// match the selected prefix, finds the digit holding the remaining rank and
// narrows the prefix to it. Thread tid owns digits nb-1-2*tid and nb-2-2*tid;
// a block prefix sum gives the count above each pair. On the first pass a
// total below the rank marks the row as taking every candidate (remaining
// -1). Ends with a barrier.
__device__ __forceinline__ void digit_search(TopkShared& sh, int nb, int shift, bool first) {
  const int tid = threadIdx.x;
  const uint32_t prefix = sh.sel_prefix, mask = sh.sel_mask;
  const int need = sh.sel_remaining;
  const uint32_t dmask = (uint32_t)nb - 1u;
  const int d0 = nb - 1 - 2 * tid, d1 = d0 - 1;
  const int c0 = d0 >= 0 ? sh.hist[d0] : 0, c1 = d1 >= 0 ? sh.hist[d1] : 0;
  int total;
  const int before = block_scan(c0 + c1, sh.warp_sums, total);
  if (before < need && before + c0 + c1 >= need) {
    const bool hi = before + c0 >= need;
    const int digit = hi ? d0 : d1;
    sh.sel_prefix = prefix | ((uint32_t)digit << shift);
    sh.sel_mask = mask | (dmask << shift);
    sh.sel_remaining = need - (hi ? before : before + c0);
    sh.bucket = hi ? c0 : c1;
  }
  if (first && tid == 0 && total < need) sh.sel_remaining = -1;
  __syncthreads();
}

template <bool kVec>
__global__ void __launch_bounds__(kTopkThreads, 2) qsa_topk_kernel(const TopkParams p) {
  __shared__ TopkShared sh;
  const int row = blockIdx.x;
  const int tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5;
  const float* sc = p.scores + (int64_t)row * p.score_stride;
  int32_t* out = p.out + (int64_t)row * p.out_stride;
  int len = p.ctx;
  if (p.lengths) {
    const int l = p.lengths[row];
    len = l < 0 ? 0 : (l > p.ctx ? p.ctx : l);
  }

  // ---- pass 1: top digit (bits 31..21) ----------------------------------------
  for (int b = tid; b < 2048; b += kTopkThreads) sh.hist[b] = 0;
  if (tid == 0) {
    sh.sel_prefix = 0u;
    sh.sel_mask = 0u;
    sh.sel_remaining = p.k;
    sh.bucket = 0;
    sh.n_cand = 0;
  }
  __syncthreads();
  for (int t = 4 * tid; t < len; t += 4 * kTopkThreads) {
    uint32_t key[4];
    load_keys<kVec>(sc, t, len, key);
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (key[u] != 0u) atomicAdd(&sh.hist[key[u] >> 21], 1);
  }
  __syncthreads();
  digit_search(sh, 2048, 21, true);

  if (sh.sel_remaining >= 0) {
    const uint32_t d1 = sh.sel_prefix >> 21;
    if (sh.bucket <= kCandidates) {
      // ---- pass 2: the threshold bucket's keys into shared memory -------------
      // (every warp runs the same iterations, so the ballots see all lanes)
      for (int t0 = 0; t0 < len; t0 += 4 * kTopkThreads) {
        uint32_t key[4];
        load_keys<kVec>(sc, t0 + 4 * tid, len, key);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const bool in = key[u] != 0u && (key[u] >> 21) == d1;
          const uint32_t b = __ballot_sync(0xffffffffu, in);
          if (b) {
            const int leader = __ffs(b) - 1;
            int base = 0;
            if (lane == leader) base = atomicAdd(&sh.n_cand, __popc(b));
            base = __shfl_sync(0xffffffffu, base, leader);
            if (in) sh.cand[base + __popc(b & ((1u << lane) - 1u))] = key[u];
          }
        }
      }
      __syncthreads();
      const int n = sh.n_cand;
      for (int pass = 1; pass < 3; ++pass) {
        const int shift = pass == 1 ? 10 : 0;
        const int nb = pass == 1 ? 2048 : 1024;
        const uint32_t dmask = (uint32_t)nb - 1u;
        for (int b = tid; b < 2048; b += kTopkThreads) sh.hist[b] = 0;
        __syncthreads();
        const uint32_t prefix = sh.sel_prefix, mask = sh.sel_mask;
        for (int i = tid; i < n; i += kTopkThreads) {
          const uint32_t key = sh.cand[i];
          if ((key & mask) == prefix) atomicAdd(&sh.hist[(key >> shift) & dmask], 1);
        }
        __syncthreads();
        digit_search(sh, nb, shift, false);
      }
    } else {
      // a bucket larger than the buffer: both lower digits over the row
      for (int pass = 1; pass < 3; ++pass) {
        const int shift = pass == 1 ? 10 : 0;
        const int nb = pass == 1 ? 2048 : 1024;
        const uint32_t dmask = (uint32_t)nb - 1u;
        for (int b = tid; b < 2048; b += kTopkThreads) sh.hist[b] = 0;
        __syncthreads();
        const uint32_t prefix = sh.sel_prefix, mask = sh.sel_mask;
        for (int t = 4 * tid; t < len; t += 4 * kTopkThreads) {
          uint32_t key[4];
          load_keys<kVec>(sc, t, len, key);
#pragma unroll
          for (int u = 0; u < 4; ++u)
            if (key[u] != 0u && (key[u] & mask) == prefix) atomicAdd(&sh.hist[(key[u] >> shift) & dmask], 1);
        }
        __syncthreads();
        digit_search(sh, nb, shift, false);
      }
    }
  }
  // threshold key T; with fewer than K candidates every candidate is taken
  const bool all = sh.sel_remaining < 0;
  const uint32_t T = all ? 1u : sh.sel_prefix;
  const int take_eq = all ? 0 : sh.sel_remaining;

  // ---- pass 3: ordered compaction, one block scan per 32768 positions -------
  // position order within a tile: group j, then thread, then the 4 positions
  int gt_run = 0, eq_run = 0;  // selected-greater and equal keys before the tile
  for (int base = 0; base < len; base += kTilePositions) {
    uint32_t gtb = 0u, eqb = 0u;  // bit 4j+u: position base + 4096j + 4tid + u
    uint32_t lpre[kGroups];       // this lane's exclusive prefix in its warp (greater | equal << 16)
#pragma unroll
    for (int j = 0; j < kGroups; ++j) {
      lpre[j] = 0u;
      const int t0 = base + j * 4 * kTopkThreads;
      if (t0 >= len) continue;  // uniform over the block
      uint32_t key[4];
      load_keys<kVec>(sc, t0 + 4 * tid, len, key);
      uint32_t g = 0u, e = 0u;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        g |= (all ? key[u] != 0u : key[u] > T) ? (1u << u) : 0u;
        e |= (!all && key[u] == T) ? (1u << u) : 0u;
      }
      gtb |= g << (4 * j);
      eqb |= e << (4 * j);
      const uint32_t c = (uint32_t)__popc(g) | ((uint32_t)__popc(e) << 16);
      uint32_t x = c;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
      }
      lpre[j] = x - c;
      if (lane == 31) sh.counts[j * kTopkWarps + warp] = x;
    }
    const int groups = min(kGroups, (len - base + 4 * kTopkThreads - 1) / (4 * kTopkThreads));
    for (int i = groups * kTopkWarps + tid; i < kGroups * kTopkWarps; i += kTopkThreads) sh.counts[i] = 0u;
    __syncthreads();
    // exclusive scan of the 256 (group, warp) counts by the first 8 warps
    // (per-field totals stay below 2^16: a tile holds 32768 positions)
    uint32_t cnt = 0u, incl = 0u;
    if (tid < kGroups * kTopkWarps) {
      cnt = sh.counts[tid];
      incl = cnt;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      if (lane == 31) sh.warp_sums[warp] = (int)incl;
    }
    __syncthreads();
    uint32_t tile_total = 0u;
#pragma unroll
    for (int w = 0; w < kGroups; ++w) tile_total += (uint32_t)sh.warp_sums[w];
    if (tid < kGroups * kTopkWarps) {
      uint32_t off = incl - cnt;
      for (int w = 0; w < warp; ++w) off += (uint32_t)sh.warp_sums[w];
      sh.counts[tid] = off;
    }
    __syncthreads();
    // write the selected positions of this thread
    uint32_t sel = gtb | eqb;
    while (sel) {
      const int bit = __ffs(sel) - 1;
      sel &= sel - 1u;
      const int j = bit >> 2;
      const uint32_t below = ((1u << bit) - 1u) & (0xfu << (4 * j));
      const uint32_t pre = sh.counts[j * kTopkWarps + warp] + lpre[j];
      const int gt_before = gt_run + (int)(pre & 0xffffu) + __popc(gtb & below);
      const int eq_before = eq_run + (int)(pre >> 16) + __popc(eqb & below);
      const int t = base + j * 4 * kTopkThreads + 4 * tid + (bit & 3);
      if ((gtb >> bit) & 1u) {
        const int pos = gt_before + min(eq_before, take_eq);
        if (pos < p.k) out[pos] = t;
      } else if (eq_before < take_eq) {
        const int pos = gt_before + eq_before;
        if (pos < p.k) out[pos] = t;
      }
    }
    gt_run += (int)(tile_total & 0xffffu);
    eq_run += (int)(tile_total >> 16);
    __syncthreads();  // counts and warp_sums are reused by the next tile
  }
  const int selected = min(p.k, gt_run + min(eq_run, take_eq));
  for (int i = selected + tid; i < p.k; i += kTopkThreads) out[i] = -1;
}

}  // namespace

cudaError_t launch_topk(const TopkParams& p, cudaStream_t stream) {
  if (p.rows <= 0) return cudaSuccess;
  const bool vec = (reinterpret_cast<uintptr_t>(p.scores) & 15u) == 0 && p.score_stride % 4 == 0 && p.ctx % 4 == 0;
  if (vec)
    qsa_topk_kernel<true><<<(unsigned)p.rows, kTopkThreads, 0, stream>>>(p);
  else
    qsa_topk_kernel<false><<<(unsigned)p.rows, kTopkThreads, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace qsa
