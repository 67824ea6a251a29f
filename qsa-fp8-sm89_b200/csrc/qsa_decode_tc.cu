// Tensor-core decode kernel for sm_100a (tcgen05, FP8 operands, TMEM
// accumulators).
//
// One CTA (128 threads) serves one (row, KV head, chunk of up to 512 Top-K
// entries). Every selected 128-byte K/V row is read from HBM once and shared
// by the G query heads of the group.
//
// Layout of the work, per CTA:
//   1. decode the chunk's Top-K entries to K/V row offsets (smem table);
//   2. split each query head into four FP8 E4M3 terms,
//        q * 2^E_h = t0 + t1/16 + t2/256 + t3/4096   (exact for bf16 q),
//      stored as the N x 128 B operand Qs, row h*4+j = term j of head h;
//   3. stream K tiles then V tiles (128 tokens x 128 B, 16 KB each) through a
//      4-slot ring with 16-byte cp.async, written in the 128-byte-swizzled
//      K-major layout the tensor core reads directly -- no dequantisation;
//   4. S = K_tile . Qs^T on the tensor core (M=128 tokens, N = 4G padded to a
//      multiple of 16, K=128 dims) into TMEM, one column block per tile;
//   5. softmax over the whole chunk (two-pass: exact max and sum), the
//      probabilities split into four FP8 terms of p*256 the same way and
//      written as the operand Ps (row h*4+j, one byte per token);
//   6. O^T = V_tile^T . Ps^T on the tensor core (V read MN-major from the same
//      swizzled tile, M=128 dims, N as above, K=128 tokens), accumulated in
//      TMEM across tiles;
//   7. epilogue: recombine the terms, normalise, v_scale, sigmoid gate, bf16
//      store (or a normalised partial + log-sum-exp for the split combine).
//
// Every mbarrier wait is bounded; on a timeout the CTA records an error in the
// device error word, drains its copies, frees its TMEM and returns.
#include <atomic>

#include "qsa_common.cuh"

namespace qsa {
namespace {

constexpr int kTile = 128;           // tokens per tile
constexpr int kTilesPerChunk = 4;    // tiles per CTA (512 tokens)
constexpr int kStages = 4;           // K/V tile slots in shared memory
constexpr int kThreads = 128;
constexpr int kTileBytes = kTile * kHeadDim;  // 16 KiB
constexpr int kTerms = 4;            // FP8 terms per Q / P value
constexpr uint64_t kWaitLimitNs = 1000000000ull;  // 1 s
constexpr int kErrTimeout = 1;

__host__ __device__ constexpr int pow2_at_least(int x) {
  int v = 32;
  while (v < x) v <<= 1;
  return v;
}

template <int G>
struct Cfg {
  static constexpr int N = ((G * kTerms + 15) / 16) * 16;  // MMA N
  static constexpr int kColS = 0;                           // S tile i at column i*N
  static constexpr int kColO = kTilesPerChunk * N;          // O accumulator
  static constexpr int kTmemCols = pow2_at_least(kColO + N);
  // shared memory carve-up (offsets from a 1024-byte aligned base)
  static constexpr int kRing = 0;
  static constexpr int kQs = kRing + kStages * kTileBytes;
  static constexpr int kPs = kQs + N * 128;
  static constexpr int kRowOff = kPs + kTilesPerChunk * N * 128;
  static constexpr int kRed = kRowOff + kTilesPerChunk * kTile * 8;   // float [4][G] (max) + [4][G] (sum)
  static constexpr int kQinv = kRed + 2 * 4 * G * 4;                  // float [G]
  static constexpr int kBars = ((kQinv + G * 4 + 7) / 8) * 8;         // uint64 [kStages + 2]
  static constexpr int kTmemSlot = kBars + (kStages + 2) * 8;         // uint32
  static constexpr int kBytes = kTmemSlot + 16;
  // alignment slack; a CTA that needs all 512 TMEM columns asks for enough
  // shared memory to be alone on its SM, so no second CTA waits in alloc
  static constexpr int kSmemAlloc = (kTmemCols == 512 && kBytes + 1024 < 120 * 1024) ? 120 * 1024 : kBytes + 1024;
  static constexpr uint32_t kIdescS = idesc_e4m3(128, N, false, false);
  static constexpr uint32_t kIdescO = idesc_e4m3(128, N, true, false);
};

// Split x (|x| < 448) into four E4M3 terms: x ~= t0 + t1/16 + t2/256 + t3/4096.
__device__ __forceinline__ void split4(float x, uint8_t (&t)[4]) {
#pragma unroll
  for (int j = 0; j < kTerms; ++j) {
    t[j] = f32_to_e4m3(x);
    x = (x - e4m3_to_f32(t[j])) * 16.0f;
  }
}

template <int G>
__global__ void __launch_bounds__(kThreads, 1)
qsa_decode_tc_kernel(DecodeParams p) {
  using C = Cfg<G>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_s = smem_u32(smem_raw);
  const uint32_t base_s = (raw_s + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base_s - raw_s);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int g = blockIdx.x % p.num_kv_heads;
  const int row = blockIdx.x / p.num_kv_heads;
  const int chunk = blockIdx.y;

  int64_t* rowoff = reinterpret_cast<int64_t*>(smem + C::kRowOff);
  float* red_max = reinterpret_cast<float*>(smem + C::kRed);
  float* red_sum = red_max + 4 * G;
  float* qinv = reinterpret_cast<float*>(smem + C::kQinv);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kBars);
  uint64_t* bar_slot = bars;              // [kStages]: MMA finished reading slot
  uint64_t* bar_s = bars + kStages;       // all S tiles computed
  uint64_t* bar_o = bars + kStages + 1;   // O accumulation finished
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kTmemSlot);

  const uint32_t ring_s = base_s + C::kRing;
  const uint32_t qs_s = base_s + C::kQs;
  const uint32_t ps_s = base_s + C::kPs;

  // ---- set-up: barriers, TMEM ------------------------------------------------
  if (tid == 0) {
    for (int i = 0; i < kStages + 2; ++i) mbar_init(bars + i, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
    tc_fence_before();
  }

  // ---- 1. decode the chunk's Top-K entries -----------------------------------
  const int64_t req = row_request(p, row);
  const int count = row_count(p, row);
  const int c0 = chunk * p.chunk_tokens;
  const int clen = max(0, min(p.chunk_tokens, p.topk - c0));
  const int ntiles = (clen + kTile - 1) / kTile;
  int mine_valid = 0;
  for (int i = tid; i < ntiles * kTile; i += kThreads) {
    const int64_t slot = (i < clen) ? token_slot(p, row, req, count, c0 + i) : -1;
    rowoff[i] = slot >= 0 ? (slot * p.num_kv_heads + g) * kHeadDim : -1;
    mine_valid |= slot >= 0;
  }

  // ---- 2. query split into FP8 terms (warp w: heads w, w+4, ...) --------------
  for (int h = warp; h < G; h += 4) {
    const int64_t qoff = ((int64_t)row * p.num_q_heads + g * G + h) * kHeadDim + lane * 4;
    const uint2 raw = *reinterpret_cast<const uint2*>(p.q + qoff);
    const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.x));
    const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.y));
    const float x[4] = {a.x, a.y, b.x, b.y};
    float amax = fmaxf(fmaxf(fabsf(x[0]), fabsf(x[1])), fmaxf(fabsf(x[2]), fabsf(x[3])));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    // 2^E maps the head's largest |q| into [128, 256).
    int e = 0;
    if (amax > 0.f && amax <= 3.0e38f) {
      const int ex = (int)((__float_as_uint(amax) >> 23) & 0xff) - 127;
      e = min(max(7 - ex, -120), 120);
    }
    const float sc = __uint_as_float((uint32_t)(127 + e) << 23);
    uint32_t packed[kTerms] = {0u, 0u, 0u, 0u};
#pragma unroll
    for (int d = 0; d < 4; ++d) {
      uint8_t t[kTerms];
      split4(x[d] * sc, t);
#pragma unroll
      for (int j = 0; j < kTerms; ++j) packed[j] |= (uint32_t)t[j] << (8 * d);
    }
#pragma unroll
    for (int j = 0; j < kTerms; ++j)
      *reinterpret_cast<uint32_t*>(smem + C::kQs + sw128_offset(h * kTerms + j, lane * 4)) = packed[j];
    if (lane == 0) qinv[h] = __uint_as_float((uint32_t)(127 - e) << 23) * p.score_scale_log2;
  }
  // zero the padding rows of Qs and Ps (rows 4G .. N-1)
  constexpr int kPadRows = C::N - G * kTerms;
  if (kPadRows > 0) {
    for (int i = tid; i < kPadRows * 8; i += kThreads) {
      const int r = G * kTerms + i / 8;
      const int ch = i % 8;
      *reinterpret_cast<uint4*>(smem + C::kQs + r * 128 + ch * 16) = make_uint4(0, 0, 0, 0);
      for (int t = 0; t < kTilesPerChunk; ++t)
        *reinterpret_cast<uint4*>(smem + C::kPs + t * C::N * 128 + r * 128 + ch * 16) = make_uint4(0, 0, 0, 0);
    }
  }
  fence_proxy_async_smem();
  const int any_valid = __syncthreads_or(mine_valid);
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool failed = false;

  if (any_valid) {
    // ---- 3. start streaming: stream tile s < ntiles is K tile s, else V tile s-ntiles
    auto issue_tile = [&](int s) {
      const uint8_t* src_base = s < ntiles ? p.k : p.v;
      const int tile = s < ntiles ? s : s - ntiles;
      const uint32_t dst = ring_s + (uint32_t)(s % kStages) * kTileBytes;
#pragma unroll
      for (int it = 0; it < kTileBytes / 16 / kThreads; ++it) {
        const int idx = it * kThreads + tid;
        const int r = idx >> 3;
        const int ch = idx & 7;
        const int64_t off = rowoff[tile * kTile + r];
        const uint8_t* src = off >= 0 ? src_base + off + ch * 16 : src_base;
        cp_async_16(dst + sw128_offset(r, ch * 16), src, off >= 0 ? 16u : 0u);
      }
    };
    const int nstream = 2 * ntiles;
#pragma unroll
    for (int s = 0; s < kStages; ++s) {
      if (s < nstream) issue_tile(s);
      cp_async_commit();
    }

    // ---- 4. K phase: S_j = K_j . Qs^T ---------------------------------------
    for (int j = 0; j < ntiles; ++j) {
      cp_async_wait<kStages - 1>();
      fence_proxy_async_smem();
      __syncthreads();
      if (tid == 0) {
        tc_fence_after();
        const uint32_t a0 = ring_s + (uint32_t)(j % kStages) * kTileBytes;
#pragma unroll
        for (int kk = 0; kk < kHeadDim / 32; ++kk) {
          const uint64_t ad = smem_desc_sw128(a0 + kk * 32, 16, 1024);
          const uint64_t bd = smem_desc_sw128(qs_s + kk * 32, 16, 1024);
          mma_f8(tmem + C::kColS + j * C::N, ad, bd, C::kIdescS, kk > 0 ? 1u : 0u);
        }
        mma_commit(bar_slot + (j % kStages));
        if (j == ntiles - 1) mma_commit(bar_s);
      }
      if (j + kStages < nstream) {
        // the slot is refilled only once the MMA that read it has finished
        const bool ok = mbar_wait_bounded(bar_slot + (j % kStages), (uint32_t)((j / kStages) & 1), kWaitLimitNs);
        if (__syncthreads_or(!ok)) { failed = true; break; }
        issue_tile(j + kStages);
      }
      cp_async_commit();
    }

    // ---- 5. softmax over the chunk ------------------------------------------
    float sc[kTilesPerChunk][G];
    float m_h[G], l_h[G];
    if (!failed) {
      const bool ok = mbar_wait_bounded(bar_s, 0, kWaitLimitNs);
      failed = __syncthreads_or(!ok);
    }
    if (!failed) {
      tc_fence_after();
      const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
#pragma unroll
      for (int i = 0; i < kTilesPerChunk; ++i) {
        if (i < ntiles) {
          float v[C::N];
#pragma unroll
          for (int cb = 0; cb < C::N; cb += 16) {
            float tmp[16];
            tmem_ld16(tmem + lane_base + C::kColS + i * C::N + cb, tmp);
            tmem_wait_ld();
#pragma unroll
            for (int c = 0; c < 16; ++c) v[cb + c] = tmp[c];
          }
          const bool valid = rowoff[i * kTile + tid] >= 0;
#pragma unroll
          for (int h = 0; h < G; ++h) {
            const float s = v[h * 4] + v[h * 4 + 1] * 0.0625f + v[h * 4 + 2] * 0.00390625f +
                            v[h * 4 + 3] * 0.000244140625f;
            sc[i][h] = valid ? s * qinv[h] : -INFINITY;
          }
        } else {
#pragma unroll
          for (int h = 0; h < G; ++h) sc[i][h] = -INFINITY;
        }
      }
      // exact max per head over the chunk
#pragma unroll
      for (int h = 0; h < G; ++h) {
        float mx = sc[0][h];
#pragma unroll
        for (int i = 1; i < kTilesPerChunk; ++i) mx = fmaxf(mx, sc[i][h]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        if (lane == 0) red_max[warp * G + h] = mx;
      }
      __syncthreads();
#pragma unroll
      for (int h = 0; h < G; ++h) {
        m_h[h] = fmaxf(fmaxf(red_max[h], red_max[G + h]), fmaxf(red_max[2 * G + h], red_max[3 * G + h]));
        float sum = 0.f;
#pragma unroll
        for (int i = 0; i < kTilesPerChunk; ++i) {
          const float pr = (sc[i][h] == -INFINITY) ? 0.f : exp2f(sc[i][h] - m_h[h]);
          sc[i][h] = pr;
          sum += pr;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        if (lane == 0) red_sum[warp * G + h] = sum;
      }
      // probabilities -> FP8 terms of p*256, one byte per token per row
#pragma unroll
      for (int i = 0; i < kTilesPerChunk; ++i) {
        if (i < ntiles) {
          uint8_t* ps = smem + C::kPs + i * C::N * 128;
#pragma unroll
          for (int h = 0; h < G; ++h) {
            uint8_t t[kTerms];
            split4(sc[i][h] * 256.0f, t);
#pragma unroll
            for (int j = 0; j < kTerms; ++j) ps[sw128_offset(h * kTerms + j, tid)] = t[j];
          }
        }
      }
      fence_proxy_async_smem();
      __syncthreads();
#pragma unroll
      for (int h = 0; h < G; ++h)
        l_h[h] = red_sum[h] + red_sum[G + h] + red_sum[2 * G + h] + red_sum[3 * G + h];

      // ---- 6. V phase: O^T += V_j^T . Ps_j^T ----------------------------------
      for (int jv = 0; jv < ntiles; ++jv) {
        cp_async_wait_dyn(kStages - 1 - jv);
        fence_proxy_async_smem();
        __syncthreads();
        if (tid == 0) {
          tc_fence_after();
          const int s = ntiles + jv;
          const uint32_t a0 = ring_s + (uint32_t)(s % kStages) * kTileBytes;
          const uint32_t b0 = ps_s + (uint32_t)(jv * C::N * 128);
#pragma unroll
          for (int kk = 0; kk < kTile / 32; ++kk) {
            const uint64_t ad = smem_desc_sw128(a0 + kk * 32 * 128, kTileBytes, 1024);
            const uint64_t bd = smem_desc_sw128(b0 + kk * 32, 16, 1024);
            mma_f8(tmem + C::kColO, ad, bd, C::kIdescO, (jv > 0 || kk > 0) ? 1u : 0u);
          }
          if (jv == ntiles - 1) mma_commit(bar_o);
        }
      }
      const bool ok = mbar_wait_bounded(bar_o, 0, kWaitLimitNs);
      failed = __syncthreads_or(!ok);
    }

    // ---- 7. epilogue: thread = head dim d ------------------------------------
    if (!failed) {
      tc_fence_after();
      const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
      float v[C::N];
#pragma unroll
      for (int cb = 0; cb < C::N; cb += 16) {
        float tmp[16];
        tmem_ld16(tmem + lane_base + C::kColO + cb, tmp);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < 16; ++c) v[cb + c] = tmp[c];
      }
      const int d = tid;
#pragma unroll
      for (int h = 0; h < G; ++h) {
        const float acc = v[h * 4] + v[h * 4 + 1] * 0.0625f + v[h * 4 + 2] * 0.00390625f +
                          v[h * 4 + 3] * 0.000244140625f;
        const float o = l_h[h] > 0.f ? acc * (1.0f / 256.0f) / l_h[h] : 0.f;
        const int64_t off = ((int64_t)row * p.num_q_heads + g * G + h) * kHeadDim + d;
        if (p.num_chunks == 1) {
          const float gt = __bfloat162float(p.gate[off]);
          p.out[off] = __float2bfloat16_rn(o * p.v_scale * (1.0f / (1.0f + expf(-gt))));
        } else {
          const int64_t pidx = ((int64_t)row * p.num_q_heads + g * G + h) * p.num_chunks + chunk;
          p.part_o[pidx * kHeadDim + d] = o;
          if (d == 0) p.part_lse[pidx] = l_h[h] > 0.f ? m_h[h] + log2f(l_h[h]) : -INFINITY;
        }
      }
    }
  }

  if (!any_valid) {
    // no valid entry in this chunk: zeros (or an empty partial)
    for (int i = tid; i < G * kHeadDim; i += kThreads) {
      const int h = i / kHeadDim;
      const int d = i % kHeadDim;
      const int64_t off = ((int64_t)row * p.num_q_heads + g * G + h) * kHeadDim + d;
      if (p.num_chunks == 1) {
        p.out[off] = __float2bfloat16_rn(0.f);
      } else {
        const int64_t pidx = ((int64_t)row * p.num_q_heads + g * G + h) * p.num_chunks + chunk;
        p.part_o[pidx * kHeadDim + d] = 0.f;
        if (d == 0) p.part_lse[pidx] = -INFINITY;
      }
    }
  }

  if (failed && tid == 0) report_error(p, kErrTimeout);
  // ---- teardown ---------------------------------------------------------------
  cp_async_wait<0>();
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}

template <int G>
cudaError_t launch_g(const DecodeParams& p, cudaStream_t stream) {
  using C = Cfg<G>;
  // The shared-memory opt-in is per device; remember which devices have it.
  static std::atomic<uint64_t> configured{0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t bit = 1ull << (dev & 63);
  if (!(configured.load(std::memory_order_acquire) & bit)) {
    e = cudaFuncSetAttribute(qsa_decode_tc_kernel<G>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemAlloc);
    if (e != cudaSuccess) return e;
    configured.fetch_or(bit, std::memory_order_acq_rel);
  }
  dim3 grid((unsigned)(p.rows * p.num_kv_heads), (unsigned)p.num_chunks, 1);
  qsa_decode_tc_kernel<G><<<grid, kThreads, C::kSmemAlloc, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace

int tc_chunk_tokens() { return kTile * kTilesPerChunk; }

bool tc_supports_group(int group) {
  return group == 1 || group == 2 || group == 4 || group == 8 || group == 16;
}

cudaError_t launch_decode_tc(const DecodeParams& p, cudaStream_t stream) {
  switch (p.group) {
    case 1: return launch_g<1>(p, stream);
    case 2: return launch_g<2>(p, stream);
    case 4: return launch_g<4>(p, stream);
    case 8: return launch_g<8>(p, stream);
    case 16: return launch_g<16>(p, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace qsa
