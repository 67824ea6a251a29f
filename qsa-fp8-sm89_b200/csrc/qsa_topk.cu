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
// One CTA of 1024 threads per row. Scores map to order-preserving uint32
// keys. A radix select over three digits of 11, 11 and 10 bits (histogram in
// shared memory; a block prefix sum over the bins finds the digit that holds
// the K-th key) gives the threshold key
// T and how many keys equal to T to take. An ordered compaction (block
// prefix sums over 1024-position pieces) then writes the selected positions
// in ascending order; each thread takes 4 consecutive positions a step, so
// two block scans cover 4096 positions. The kernel reads the row's scores
// four times, from L2 after the first pass.
#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/qsa_b200.h"
#include "qsa_internal.h"

namespace qsa {
namespace {

constexpr int kTopkThreads = 1024;
constexpr int kTopkWarps = kTopkThreads / 32;

// order-preserving key of a score; 0 for a position that is not a candidate
__device__ __forceinline__ uint32_t score_key(float s) {
  const uint32_t u = __float_as_uint(s);
  if (s != s || s == -INFINITY) return 0u;  // NaN or -inf
  if (s == 0.f) return 0x80000000u;          // -0 and +0 are the same score
  const uint32_t k = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return k == 0u ? 1u : k;  // 0 is reserved for non-candidates
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

__global__ void __launch_bounds__(kTopkThreads) qsa_topk_kernel(const TopkParams p) {
  __shared__ int hist[2048];
  __shared__ int warp_sums[kTopkWarps];
  __shared__ uint32_t sel_prefix, sel_mask;
  __shared__ int sel_remaining;
  const int row = blockIdx.x;
  const int tid = threadIdx.x;
  const float* sc = p.scores + (int64_t)row * p.score_stride;
  int32_t* out = p.out + (int64_t)row * p.out_stride;
  int len = p.ctx;
  if (p.lengths) {
    const int l = p.lengths[row];
    len = l < 0 ? 0 : (l > p.ctx ? p.ctx : l);
  }

  // ---- radix select: the K-th largest candidate key ------------------------
  // three digits of 11, 11 and 10 bits
  if (tid == 0) {
    sel_prefix = 0u;
    sel_mask = 0u;
    sel_remaining = p.k;
  }
  for (int pass = 0; pass < 3; ++pass) {
    const int shift = pass == 0 ? 21 : (pass == 1 ? 10 : 0);
    const int nb = pass == 2 ? 1024 : 2048;
    const uint32_t dmask = (uint32_t)nb - 1u;
    for (int b = tid; b < 2048; b += kTopkThreads) hist[b] = 0;
    __syncthreads();
    const uint32_t prefix = sel_prefix, mask = sel_mask;
    const int need = sel_remaining;
    for (int t = tid; t < len; t += kTopkThreads) {
      const uint32_t key = score_key(sc[t]);
      if (key != 0u && (key & mask) == prefix) atomicAdd(&hist[(key >> shift) & dmask], 1);
    }
    __syncthreads();
    // digits from the top: thread tid owns digits nb-1-2*tid and nb-2-2*tid; a
    // block prefix sum gives the count above each pair, and the thread whose
    // pair reaches the remaining rank records the digit
    const int d0 = nb - 1 - 2 * tid, d1 = d0 - 1;
    const int c0 = d0 >= 0 ? hist[d0] : 0, c1 = d1 >= 0 ? hist[d1] : 0;
    int total;
    const int before = block_scan(c0 + c1, warp_sums, total);
    if (before < need && before + c0 + c1 >= need) {
      const int digit = before + c0 >= need ? d0 : d1;
      const int above = before + c0 >= need ? before : before + c0;
      sel_prefix = prefix | ((uint32_t)digit << shift);
      sel_mask = mask | (dmask << shift);
      sel_remaining = need - above;
    }
    if (tid == 0 && total < need) sel_remaining = -1;  // fewer than K candidates (first pass only)
    __syncthreads();
    if (sel_remaining < 0) break;
  }
  // threshold key T; with fewer than K candidates every candidate is taken
  const bool all = sel_remaining < 0;
  const uint32_t T = all ? 1u : sel_prefix;
  const int take_eq = all ? 0x7fffffff : sel_remaining;

  // ---- ordered compaction: 4 consecutive positions a thread, 4096 a step ----
  int eq_before = 0, sel_before = 0;
  for (int t0 = 0; t0 < len; t0 += 4 * kTopkThreads) {
    const int tb = t0 + 4 * tid;
    bool gt[4], eq[4];
    int n_eq = 0;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const uint32_t key = tb + u < len ? score_key(sc[tb + u]) : 0u;
      gt[u] = key != 0u && (all || key > T);
      eq[u] = !all && key == T && key != 0u;
      n_eq += eq[u] ? 1 : 0;
    }
    int eq_total;
    int eq_rank = eq_before + block_scan(n_eq, warp_sums, eq_total);
    bool sel[4];
    int n_sel = 0;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      sel[u] = gt[u] || (eq[u] && eq_rank < take_eq);
      eq_rank += eq[u] ? 1 : 0;
      n_sel += sel[u] ? 1 : 0;
    }
    int sel_total;
    int pos = sel_before + block_scan(n_sel, warp_sums, sel_total);
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (sel[u]) {
        if (pos < p.k) out[pos] = tb + u;
        ++pos;
      }
    eq_before += eq_total;
    sel_before += sel_total;
  }
  for (int i = sel_before + tid; i < p.k; i += kTopkThreads) out[i] = -1;
}

}  // namespace

cudaError_t launch_topk(const TopkParams& p, cudaStream_t stream) {
  if (p.rows <= 0) return cudaSuccess;
  qsa_topk_kernel<<<(unsigned)p.rows, kTopkThreads, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace qsa
