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
// order-preserving uint32 keys. Radix selects (digits of 11, 11 and 10 bits:
// a shared-memory histogram, then a block prefix sum over the bins finds the
// digit that holds the wanted rank) give the threshold key T and how many
// keys equal to T to take.
//
// Sampled path (rows of at most kBitmapMax positions): the row is read from
// HBM once.
//   1. a sample of up to 1024 keys (32 pieces of 32 consecutive positions,
//      spread evenly over the row) gives a lower bound L: the top 22
//      bits of the sample key whose rank is the expected rank of the K-th key
//      plus six standard deviations (and 8), so that the row holds at least K
//      keys >= L except with negligible probability;
//   2. one pass over the row appends every key >= L with its position to a
//      buffer in shared memory;
//   3. when the buffer holds at least K and at most kBuffer keys, T is
//      selected from the buffer alone, the selected positions are set in a
//      bitmap of the row, and two block scans (equal keys by position, then
//      the selected bits) write the positions in ascending order.
// Otherwise (too few keys >= L, an overflowing buffer, a longer row) the
// row takes the radix path, reading it three times, the last two from L2:
//   1. histogram of the top digit; a block prefix sum finds its digit d1;
//   2. the keys whose top digit is d1 go to the buffer and the two lower
//      digits are selected from it (a bucket larger than the buffer takes
//      both lower digits over the row instead);
//   3. ordered compaction over tiles of 16384 positions with one block scan
//      over the (group, warp) counts of each tile.
// Scores are read as float4 when the row start and stride allow it.
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>

#include "../../include/qsa_b200.h"
#include "qsa_internal.h"

namespace qsa {
namespace {

constexpr int kTopkThreads = 1024;
constexpr int kTopkWarps = kTopkThreads / 32;
constexpr int kGroups = 4;                              // 4-position groups per thread per tile
constexpr int kTilePositions = 4 * kTopkThreads * kGroups;  // 16384
constexpr int kBuffer = 8192;                           // keys (and positions) kept in shared memory
constexpr int kBitmapMax = 65536;                       // longest row of the sampled path
constexpr int kBitmapWords = kBitmapMax / 32;
constexpr int kSample = 1024;                           // sampled keys (one a thread)
#ifndef QSA_TOPK_PASS_GROUPS
#define QSA_TOPK_PASS_GROUPS 4
#endif
constexpr int kPassGroups = QSA_TOPK_PASS_GROUPS;       // 4-position loads in flight a thread in the pass
#ifndef QSA_TOPK_SAMPLE_DIGITS
#define QSA_TOPK_SAMPLE_DIGITS 2
#endif
constexpr int kSampleDigits = QSA_TOPK_SAMPLE_DIGITS;   // radix digits of the sample's bound (1 or 2)

// order-preserving key of a score; 0 for a position that is not a candidate
__device__ __forceinline__ uint32_t score_key(float s) {
  const uint32_t u = __float_as_uint(s);
  if (s != s || s == -INFINITY) return 0u;  // NaN or -inf
  if (s == 0.f) return 0x80000000u;          // -0 and +0 are the same score
  const uint32_t k = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return k == 0u ? 1u : k;  // 0 is reserved for non-candidates
}

// The score of a key (the inverse of score_key for keys of finite or
// infinite scores; the key of +-0 gives +0).
__device__ __forceinline__ float key_score(uint32_t key) {
  return __uint_as_float((key & 0x80000000u) ? (key & 0x7fffffffu) : ~key);
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

// Scores of positions t .. t+3 of the row (-inf at and past len, which no
// candidate bound admits). kVec as for load_keys.
template <bool kVec>
__device__ __forceinline__ void load_scores(const float* sc, int t, int len, float (&v)[4]) {
  if (kVec) {
    if (t < len) {
      const float4 f = __ldg(reinterpret_cast<const float4*>(sc + t));
      v[0] = f.x;
      v[1] = t + 1 < len ? f.y : -INFINITY;
      v[2] = t + 2 < len ? f.z : -INFINITY;
      v[3] = t + 3 < len ? f.w : -INFINITY;
    } else {
      v[0] = v[1] = v[2] = v[3] = -INFINITY;
    }
  } else {
#pragma unroll
    for (int u = 0; u < 4; ++u) v[u] = t + u < len ? __ldg(sc + t + u) : -INFINITY;
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

// Selection state of the sampled path, identical in every thread: the key
// prefix found so far, its mask, and the rank still wanted inside it (-1:
// fewer keys than the rank).
struct Sel {
  uint32_t prefix, mask;
  int need;
};

struct TopkShared {
  int hist[2][2048];                      // radix path: hist[0]; sampled path: both, alternately
  Sel sel_state;                          // sampled path: the state warp 0 publishes
  int warp_sums[kTopkWarps];
  uint32_t cand[kBuffer];                 // keys: >= L (sampled path), of the threshold bucket (radix path)
  int32_t cand_pos[kBuffer];              // positions of the sampled path's keys
  uint32_t sel_bits[kBitmapWords];        // sampled path: selected positions
  uint32_t eq_bits[kBitmapWords];         // sampled path: positions whose key equals T
  uint32_t counts[kGroups * kTopkWarps];  // radix path compaction: (greater | equal << 16) per (group, warp)
  uint32_t sel_prefix, sel_mask;
  int sel_remaining, bucket, n_cand, n_eq;
};
constexpr size_t kTopkSmem = sizeof(TopkShared);

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
  const int c0 = d0 >= 0 ? sh.hist[0][d0] : 0, c1 = d1 >= 0 ? sh.hist[0][d1] : 0;
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

// The radix path: three reads of the row (see the top of the file). Starts
// after a barrier; every thread of the CTA calls it.
template <bool kVec>
__device__ __forceinline__ void radix_path(TopkShared& sh, const float* sc, int len, int32_t* out, int k) {
  const int tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5;

  // ---- pass 1: top digit (bits 31..21) ----------------------------------------
  for (int b = tid; b < 2048; b += kTopkThreads) sh.hist[0][b] = 0;
  if (tid == 0) {
    sh.sel_prefix = 0u;
    sh.sel_mask = 0u;
    sh.sel_remaining = k;
    sh.bucket = 0;
    sh.n_cand = 0;
  }
  __syncthreads();
  for (int t = 4 * tid; t < len; t += 4 * kTopkThreads) {
    uint32_t key[4];
    load_keys<kVec>(sc, t, len, key);
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (key[u] != 0u) atomicAdd(&sh.hist[0][key[u] >> 21], 1);
  }
  __syncthreads();
  digit_search(sh, 2048, 21, true);

  if (sh.sel_remaining >= 0) {
    const uint32_t d1 = sh.sel_prefix >> 21;
    if (sh.bucket <= kBuffer) {
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
        for (int b = tid; b < 2048; b += kTopkThreads) sh.hist[0][b] = 0;
        __syncthreads();
        const uint32_t prefix = sh.sel_prefix, mask = sh.sel_mask;
        for (int i = tid; i < n; i += kTopkThreads) {
          const uint32_t key = sh.cand[i];
          if ((key & mask) == prefix) atomicAdd(&sh.hist[0][(key >> shift) & dmask], 1);
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
        for (int b = tid; b < 2048; b += kTopkThreads) sh.hist[0][b] = 0;
        __syncthreads();
        const uint32_t prefix = sh.sel_prefix, mask = sh.sel_mask;
        for (int t = 4 * tid; t < len; t += 4 * kTopkThreads) {
          uint32_t key[4];
          load_keys<kVec>(sc, t, len, key);
#pragma unroll
          for (int u = 0; u < 4; ++u)
            if (key[u] != 0u && (key[u] & mask) == prefix) atomicAdd(&sh.hist[0][(key[u] >> shift) & dmask], 1);
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

  // ---- pass 3: ordered compaction, one block scan per kTilePositions -------
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
    // exclusive scan of the (group, warp) counts by the first kGroups warps
    // (per-field totals stay below 2^16: a tile holds 16384 positions)
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
        if (pos < k) out[pos] = t;
      } else if (eq_before < take_eq) {
        const int pos = gt_before + eq_before;
        if (pos < k) out[pos] = t;
      }
    }
    gt_run += (int)(tile_total & 0xffffu);
    eq_run += (int)(tile_total >> 16);
    __syncthreads();  // counts and warp_sums are reused by the next tile
  }
  const int selected = min(k, gt_run + min(eq_run, take_eq));
  for (int i = selected + tid; i < k; i += kTopkThreads) out[i] = -1;
}


// ---- the sampled path's selection: two barriers a digit ---------------------
// Warp 0 finds the digit of the rank-s.need key (bits shift .. of the keys
// matching s.prefix) from histogram H (nb bins): each lane sums one group of
// nb/32 bins (the groups from the top, lane l holding group 31 - l; reads
// rotated by lane, so the 16-byte loads spread over the banks), a warp scan
// finds the group, a second the bin. `first`: a total below the rank sets
// need to -1.
__device__ __forceinline__ Sel warp_find(const int* H, Sel s, int nb, int shift, bool first) {
  const int lane = threadIdx.x & 31;
  if (s.need < 0) return s;
  const int gs = nb / 32;  // 64 or 32 bins a group
  const int4* hp = reinterpret_cast<const int4*>(H + (31 - lane) * gs);
  int wc = 0;
#pragma unroll 2
  for (int i = 0; i < gs / 4; ++i) {
    const int4 q = hp[(i + lane) & (gs / 4 - 1)];
    wc += q.x + q.y + q.z + q.w;
  }
  int cum = wc;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, cum, o);
    if (lane >= o) cum += y;
  }
  const int total = __shfl_sync(0xffffffffu, cum, 31);
  if (total < s.need) {
    if (first) s.need = -1;
    return s;
  }
  const int lg = __ffs(__ballot_sync(0xffffffffu, cum >= s.need)) - 1;
  const int g = 31 - lg;
  const int need = s.need - __shfl_sync(0xffffffffu, cum - wc, lg);  // rank inside group g
  // bins of group g from the top: two a lane (64-bin groups) or one
  const int b0 = g * gs + gs - 1 - (gs == 64 ? 2 * lane : lane);
  const int c0 = H[b0];
  const int c1 = gs == 64 ? H[b0 - 1] : 0;
  int cb = c0 + c1;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, cb, o);
    if (lane >= o) cb += y;
  }
  const int lb = __ffs(__ballot_sync(0xffffffffu, cb >= need)) - 1;
  const int before = __shfl_sync(0xffffffffu, cb - c0 - c1, lb);
  const int d0 = __shfl_sync(0xffffffffu, b0, lb);
  const int k0 = __shfl_sync(0xffffffffu, c0, lb);
  const bool hi = before + k0 >= need;
  s.prefix |= (uint32_t)(hi ? d0 : d0 - 1) << shift;
  s.mask |= ((uint32_t)nb - 1u) << shift;
  s.need = need - (hi ? before : before + k0);
  return s;
}

// After the barrier that completes histogram H: warp 0 finds the digit and
// publishes the new state, the other warps zero histogram Z for the next
// digit. Ends with a barrier; returns the state in every thread.
__device__ __forceinline__ Sel digit_step(TopkShared& sh, const int* H, int* Z, Sel s, int nb, int shift,
                                          bool first) {
  const int tid = threadIdx.x;
  if (tid < 32) {
    const Sel r = warp_find(H, s, nb, shift, first);
    if (tid == 0) sh.sel_state = r;
  } else {
    for (int b = tid - 32; b < 2048; b += kTopkThreads - 32) Z[b] = 0;
  }
  __syncthreads();
  return sh.sel_state;
}

// One digit over n keys of shared memory (histogram into H, which is zero;
// zeroes Z). Starts after the barrier that made the keys and H ready.
__device__ __forceinline__ Sel digit_over(TopkShared& sh, const uint32_t* keys, int n, int* H, int* Z, Sel s,
                                          int nb, int shift, bool first) {
  const uint32_t dmask = (uint32_t)nb - 1u;
  if (s.need >= 0)
    for (int i = threadIdx.x; i < n; i += kTopkThreads) {
      const uint32_t key = keys[i];
      if (key != 0u && (key & s.mask) == s.prefix) atomicAdd(&H[(key >> shift) & dmask], 1);
    }
  __syncthreads();
  return digit_step(sh, H, Z, s, nb, shift, first);
}

// Valid positions of a row (its length, clamped to [0, ctx]).
__device__ __forceinline__ int row_len(const TopkParams& p, int row) {
  if (!p.lengths) return p.ctx;
  const int l = __ldg(p.lengths + row);
  return l < 0 ? 0 : (l > p.ctx ? p.ctx : l);
}

// One row; every thread of the CTA calls it, after a barrier.
template <bool kVec>
__device__ __forceinline__ void topk_row(TopkShared& sh, const TopkParams& p, int row) {
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const float* sc = p.scores + (int64_t)row * p.score_stride;
  int32_t* out = p.out + (int64_t)row * p.out_stride;
  const int len = row_len(p, row);
  const int k = p.k;

  bool sampled = len > 0 && len <= kBitmapMax;
  if (sampled) {
    // H0: the histogram the pass over the row fills (zeroed), H1 the other
    int* H0 = sh.hist[0];
    int* H1 = sh.hist[1];
    // ---- 1. the bound L from a sample ------------------------------------------
    // (32 pieces of 32 consecutive positions, spread evenly over the row:
    // warp w reads one 128-byte piece, 32 DRAM requests a row instead of one
    // per sampled position)
    const int n_s = len < kSample ? len : kSample;
    if (tid < n_s) {
      const int t = len <= kSample ? tid : (tid >> 5) * (len >> 5) + (tid & 31);
      sh.cand[tid] = score_key(__ldg(sc + t));
    }
    const int words = (len + 31) / 32;
    for (int i = tid; i < words; i += kTopkThreads) {
      sh.sel_bits[i] = 0u;
      sh.eq_bits[i] = 0u;
    }
    for (int b = tid; b < 2048; b += kTopkThreads) H0[b] = 0;
    if (tid == 0) {
      sh.n_cand = 0;
      sh.n_eq = 0;
    }
    // rank of L among the sample: the K-th key's expected rank + 6 sd + 8
    const float e = (float)k * (float)n_s / (float)len;
    const float q = fminf(fmaxf(1.0f - (float)k / (float)len, 0.0f), 1.0f);
    Sel s{0u, 0u, (int)fminf(ceilf(e + 6.0f * sqrtf(e * q) + 8.0f), (float)(n_s + 1))};
    __syncthreads();
    s = digit_over(sh, sh.cand, n_s, H0, H1, s, 2048, 21, true);
    if (kSampleDigits == 2) {
      s = digit_over(sh, sh.cand, n_s, H1, H0, s, 2048, 10, false);
    } else {
      int* const h = H0;  // H1 is the zeroed one
      H0 = H1;
      H1 = h;
    }
    // the top 22 bits of that sample key; fewer sampled keys: every candidate
    const uint32_t L = s.need < 0 ? 1u : s.prefix;

    // ---- 2. every key >= L, with its position, into the buffer ------------------
    // Compared as scores: key(x) >= L exactly when x >= key_score(L) (the key
    // is monotone in the score, NaN compares false, -0 >= +0); L == 1 takes
    // every candidate, x >= -FLT_MAX. kPassGroups groups of 4 positions a
    // thread a step (all loads in flight), one warp scan and one claim. The
    // top digit of every kept key goes into H0 (the buffer's first digit).
    const float Lf = L == 1u ? -3.402823466e38f : key_score(L);
    for (int t0 = 0; t0 < len; t0 += 4 * kPassGroups * kTopkThreads) {
      float v[4 * kPassGroups];  // position t0 + (j / 4) * 4 * kTopkThreads + 4 * tid + j % 4
#pragma unroll
      for (int h = 0; h < kPassGroups; ++h)
        load_scores<kVec>(sc, t0 + h * 4 * kTopkThreads + 4 * tid, len,
                          *reinterpret_cast<float(*)[4]>(&v[4 * h]));
      uint32_t in = 0u;
#pragma unroll
      for (int j = 0; j < 4 * kPassGroups; ++j) in |= v[j] >= Lf ? 1u << j : 0u;
      const int c = __popc(in);
      int x = c;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
      }
      const int n_w = __shfl_sync(0xffffffffu, x, 31);
      if (n_w) {  // uniform over the warp
        int base = 0;
        if (lane == 31) base = atomicAdd(&sh.n_cand, n_w);
        int idx = __shfl_sync(0xffffffffu, base, 31) + x - c;
        // only the set bits (one or two a thread a step); the value is picked
        // by a tree of selects, so v stays in registers
        while (in) {
          const int b = __ffs(in) - 1;
          in &= in - 1u;
          float t[4 * kPassGroups];
#pragma unroll
          for (int j = 0; j < 4 * kPassGroups; ++j) t[j] = v[j];
#pragma unroll
          for (int w = 1; w < 4 * kPassGroups; w <<= 1)
#pragma unroll
            for (int j = 0; j < 4 * kPassGroups; j += 2 * w) t[j] = (b & w) ? t[j + w] : t[j];
          if (idx < kBuffer) {
            const uint32_t key = score_key(t[0]);
            sh.cand[idx] = key;
            sh.cand_pos[idx] = t0 + (b >> 2) * 4 * kTopkThreads + 4 * tid + (b & 3);
            atomicAdd(&H0[key >> 21], 1);
          }
          ++idx;
        }
      }
    }
    __syncthreads();
    const int n = sh.n_cand;
    sampled = n >= k && n <= kBuffer;  // uniform
    if (sampled) {
      // ---- 3. T from the buffer; selected positions into the bitmap -------------
      s = digit_step(sh, H0, H1, Sel{0u, 0u, k}, 2048, 21, true);
      s = digit_over(sh, sh.cand, n, H1, H0, s, 2048, 10, false);
      s = digit_over(sh, sh.cand, n, H0, H1, s, 1024, 0, false);
      const uint32_t T = s.prefix;
      const int take_eq = s.need;
      for (int i0 = 0; i0 < n; i0 += kTopkThreads) {
        const int i = i0 + tid;
        const uint32_t key = i < n ? sh.cand[i] : 0u;
        const int t = i < n ? sh.cand_pos[i] : 0;
        if (key > T) atomicOr(&sh.sel_bits[t >> 5], 1u << (t & 31));
        const uint32_t eq = __ballot_sync(0xffffffffu, key == T);
        if (key == T) atomicOr(&sh.eq_bits[t >> 5], 1u << (t & 31));
        if (eq && lane == 0) atomicAdd(&sh.n_eq, __popc(eq));
      }
      __syncthreads();
      // thread tid owns words 2tid, 2tid+1 (64 consecutive positions)
      uint32_t sw[2] = {0u, 0u}, ew[2] = {0u, 0u};
      const int w0 = 2 * tid;
#pragma unroll
      for (int i = 0; i < 2; ++i)
        if (w0 + i < words) {
          sw[i] = sh.sel_bits[w0 + i];
          ew[i] = sh.eq_bits[w0 + i];
        }
      if (sh.n_eq == take_eq) {  // uniform: every equal key is taken
        sw[0] |= ew[0];
        sw[1] |= ew[1];
      } else {
        // equal keys: the first take_eq by position
        int eq_total;
        int eq_rank = block_scan(__popc(ew[0]) + __popc(ew[1]), sh.warp_sums, eq_total);
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          uint32_t m = ew[i];
          while (m) {
            const uint32_t bit = m & (0u - m);
            m ^= bit;
            if (eq_rank < take_eq) sw[i] |= bit;
            ++eq_rank;
          }
        }
      }
      int sel_total;
      int pos = block_scan(__popc(sw[0]) + __popc(sw[1]), sh.warp_sums, sel_total);
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        uint32_t m = sw[i];
        while (m) {
          const int bit = __ffs(m) - 1;
          m &= m - 1u;
          out[pos++] = 32 * (w0 + i) + bit;  // sel_total == k: no padding
        }
      }
      return;
    }
  }
  __syncthreads();
  radix_path<kVec>(sh, sc, len, out, k);
}

// One CTA per row, two CTAs per SM.
template <bool kVec>
__global__ void __launch_bounds__(kTopkThreads, 2) qsa_topk_kernel(const TopkParams p) {
  extern __shared__ __align__(16) uint8_t topk_smem[];
  topk_row<kVec>(*reinterpret_cast<TopkShared*>(topk_smem), p, blockIdx.x);
}

}  // namespace

cudaError_t launch_topk(const TopkParams& p, cudaStream_t stream) {
  if (p.rows <= 0) return cudaSuccess;
  const bool vec = (reinterpret_cast<uintptr_t>(p.scores) & 15u) == 0 && p.score_stride % 4 == 0 && p.ctx % 4 == 0;
  static std::atomic<uint64_t> configured{0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t bit = 1ull << (dev & 63);
  if (!(configured.load(std::memory_order_acquire) & bit)) {
    e = cudaFuncSetAttribute(qsa_topk_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kTopkSmem);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(qsa_topk_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kTopkSmem);
    if (e != cudaSuccess) return e;
    configured.fetch_or(bit, std::memory_order_acq_rel);
  }
  const unsigned grid = (unsigned)p.rows;
  if (vec)
    qsa_topk_kernel<true><<<grid, kTopkThreads, kTopkSmem, stream>>>(p);
  else
    qsa_topk_kernel<false><<<grid, kTopkThreads, kTopkSmem, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace qsa
