// Tensor-core decode kernel for sm_100a: persistent, warp-specialised,
// cp.async gathers into swizzled shared memory, FP8 tcgen05 MMAs with TMEM
// accumulators.
//
// Work item = (Top-K row, KV head, chunk of up to kTiles*128 Top-K entries).
// Each CTA (one per SM) walks items blockIdx.x, blockIdx.x + gridDim.x, ...
// with three roles that overlap across items:
//
//   warps 0-3 loaders  warp j owns tile j (128 Top-K entries) of every item:
//                      it decodes its entries (index -> block table -> K/V
//                      row), copies the K tile and the V tile (128 rows x
//                      128 B each) into ring slots with coalesced 16-byte
//                      cp.async in the 128-byte-swizzled layout the tensor
//                      core reads (zero fill for masked rows; completion via
//                      cp.async.mbarrier.arrive), and splits its share of the
//                      G query heads into FP8 terms (operand Qs);
//   warp 4    MMA      one thread issues S = K_tile . Qs^T into TMEM for every
//                      K tile of item i+1 before O^T += V_tile^T . Ps^T for
//                      item i, so the tensor core never waits on a softmax;
//   warps 5-8          softmax over the chunk's scores (exact max and sum),
//                      probabilities as FP8 terms of p*256 (operand Ps), then
//                      the epilogue: recombine, normalise, v_scale, sigmoid
//                      gate, bf16 store (or a partial for the split combine).
//
// Every selected 128-byte K/V row is read from HBM once and shared by the G
// query heads. Q and P keep their precision through the term split:
//   q * 2^E = t0 + t1/16 + t2/256,   p * 256 = t0 + t1/16 + t2/256
// with each term an E4M3 value (two terms already hold a bf16 q exactly; p
// keeps about 13 bits), so the FP8 x FP8 tensor-core products reproduce the
// reference's fp32 products of the FP8 cache values with bf16 q and fp32 p.
//
// Synchronisation is by mbarriers: kv_full/kv_empty per ring slot, and
// per item buffer (double-buffered TMEM and operands) q_full, meta_empty,
// s_full, p_full, o_full, tmem_empty. Every wait is bounded; a CTA that gives
// up records an error in the device error word, raises a CTA-wide abort
// flag so the other roles leave their loops, frees its TMEM and returns.
#include <atomic>

#include "qsa_common.cuh"

namespace qsa {
namespace {

constexpr int kTile = 128;                    // tokens per tile
constexpr int kTileBytes = kTile * kHeadDim;  // 16 KiB of FP8
constexpr int kTerms = 3;                     // FP8 terms per Q / P value
constexpr int kLoaders = 4;                   // loader warps (tile j -> warp j % 4)
constexpr int kMmaWarp = kLoaders;            // warp 4
constexpr int kThreads = 32 * (kLoaders + 1 + 4);
constexpr int kSmemLimit = 232448;            // 227 KiB opt-in per CTA
constexpr uint64_t kWaitLimitNs = 1000000000ull;
constexpr int kErrTimeout = 1;

__host__ __device__ constexpr int align128(int x) { return (x + 127) / 128 * 128; }

__host__ __device__ constexpr int pow2_at_least(int x) {
  int v = 32;
  while (v < x) v <<= 1;
  return v;
}

template <int G>
struct Cfg {
  static constexpr int N = ((G * kTerms + 15) / 16) * 16;  // MMA N (rows of Qs / Ps)
  static constexpr int kTiles = G <= 8 ? 4 : 2;             // tiles per item
  static constexpr int kChunk = kTiles * kTile;             // Top-K entries per item
  static constexpr int kBufCols = (kTiles * N + N + 31) / 32 * 32;  // S tiles + O, per buffer
  static constexpr int kTmemCols = pow2_at_least(2 * kBufCols);
  static constexpr int kQsBytes = N * 128;
  static constexpr int kPsBytes = kTiles * N * 128;
  // shared memory layout (offsets from a 1024-byte aligned base)
  static constexpr int kQs = 0;                                 // [2][N][128]
  static constexpr int kPs = kQs + 2 * kQsBytes;                // [2][kTiles][N][128]
  // every region starts on a 128-byte boundary (the row table takes 16-byte
  // vector stores, the barriers need 8)
  static constexpr int kValid = kPs + 2 * kPsBytes;                  // uint8 [2][kChunk]
  static constexpr int kQinv = align128(kValid + 2 * kChunk);        // float [2][G]
  static constexpr int kRedMax = align128(kQinv + 2 * G * 4);        // float [2][4][G]
  static constexpr int kRedSum = align128(kRedMax + 2 * 4 * G * 4);  // float [2][4][G]
  static constexpr int kRowTab = align128(kRedSum + 2 * 4 * G * 4);  // int32 [kLoaders][128] K/V rows
  static constexpr int kBars = align128(kRowTab + kLoaders * kTile * 4);
  static constexpr int kMaxSlots = 16;
  static constexpr int kNumBars = 2 * kMaxSlots + 12;
  static constexpr int kMisc = kBars + kNumBars * 8;            // tmem address, abort flag
  static constexpr int kSlotBase = ((kMisc + 16 + 1023) / 1024) * 1024;
  static constexpr int kSlots0 = (kSmemLimit - 1024 - kSlotBase) / kTileBytes;
  static constexpr int kSlots = kSlots0 > kMaxSlots ? kMaxSlots : kSlots0;
  static constexpr int kSmemAlloc = kSlotBase + kSlots * kTileBytes + 1024;
  static constexpr uint32_t kIdescS = idesc_e4m3(128, N, false, false);
  static constexpr uint32_t kIdescO = idesc_e4m3(128, N, true, false);
  static_assert(kSlots >= 2 * kTiles, "ring must hold a K and a V chunk");
  static_assert(kSmemAlloc <= kSmemLimit, "shared memory budget");
  static_assert(kTmemCols <= 512, "TMEM budget");
  static_assert(kQs % 1024 == 0 && kPs % 1024 == 0 && kSlotBase % 1024 == 0 && kQsBytes % 1024 == 0 &&
                    (N * 128) % 1024 == 0,
                "MMA operands must start on 1024-byte swizzle atoms");
  static_assert(kRowTab % 16 == 0 && kBars % 8 == 0 && kMisc % 8 == 0, "alignment of the small arrays");
};

struct Item {
  int row, g, chunk;
};

__device__ __forceinline__ Item item_of(const DecodeParams& p, int item) {
  Item it;
  it.g = item % p.num_kv_heads;
  const int rc = item / p.num_kv_heads;
  it.chunk = rc % p.num_chunks;
  it.row = rc / p.num_chunks;
  return it;
}

__device__ __forceinline__ int item_tiles(const DecodeParams& p, int chunk, int chunk_tokens) {
  const int c0 = chunk * chunk_tokens;
  const int clen = max(0, min(chunk_tokens, p.topk - c0));
  return (clen + kTile - 1) / kTile;
}

// ------------------------------------------------------------------ PTX ----
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_u32(bar)) : "memory");
}
// Arrive on `bar` once every cp.async this thread issued so far has landed.
__device__ __forceinline__ void cp_async_mbar_arrive_noinc(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];\n" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void named_bar_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;\n" ::"r"(id), "r"(count) : "memory");
}

// Bounded wait that also gives up once another role raised the abort flag.
__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  uint64_t t0;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    uint64_t t1;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t1));
    if (t1 - t0 > kWaitLimitNs) return false;
  }
}

// Split x (|x| < 448) into E4M3 terms: x ~= t0 + t1/16 + t2/256.
__device__ __forceinline__ void split_terms(float x, uint8_t (&t)[kTerms]) {
#pragma unroll
  for (int j = 0; j < kTerms; ++j) {
    t[j] = f32_to_e4m3(x);
    x = (x - e4m3_to_f32(t[j])) * 16.0f;
  }
}

__device__ __forceinline__ float combine_terms(const float* v) {
  return v[0] + v[1] * 0.0625f + v[2] * 0.00390625f;
}

template <int G>
__global__ void __launch_bounds__(kThreads, 1) qsa_decode_tc_kernel(const __grid_constant__ DecodeParams p,
                                                                   int num_items) {
  using C = Cfg<G>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_s = smem_u32(smem_raw);
  const uint32_t base_s = (raw_s + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base_s - raw_s);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kBars);
  uint64_t* kv_full = bars;                    // [kSlots] 32 cp.async arrivals -> MMA
  uint64_t* kv_empty = bars + C::kMaxSlots;    // [kSlots] MMA commit -> loader
  uint64_t* q_full = bars + 2 * C::kMaxSlots;  // [2] loaders (kLoaders arrivals) -> MMA, softmax
  uint64_t* meta_empty = q_full + 2;           // [2] softmax -> loaders
  uint64_t* s_full = q_full + 4;               // [2] MMA commit -> softmax
  uint64_t* p_full = q_full + 6;               // [2] softmax -> MMA
  uint64_t* o_full = q_full + 8;               // [2] MMA commit -> epilogue
  uint64_t* tmem_empty = q_full + 10;          // [2] epilogue (128 arrivals) -> MMA
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::kMisc + 8);
  float* qinv = reinterpret_cast<float*>(smem + C::kQinv);
  float* red_max = reinterpret_cast<float*>(smem + C::kRedMax);
  float* red_sum = reinterpret_cast<float*>(smem + C::kRedSum);
  uint8_t* valid = smem + C::kValid;

  if (tid == 0) {
    for (int i = 0; i < C::kSlots; ++i) {
      mbar_init(kv_full + i, 32);
      mbar_init(kv_empty + i, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(q_full + b, kLoaders);
      mbar_init(meta_empty + b, 1);
      mbar_init(s_full + b, 1);
      mbar_init(p_full + b, 1);
      mbar_init(o_full + b, 1);
      mbar_init(tmem_empty + b, 128);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool failed = false;

  if (warp < kLoaders) {
    // =============================== loaders ================================
    const int lw = warp;
    int32_t* rowtab = reinterpret_cast<int32_t*>(smem + C::kRowTab) + lw * kTile;
    int pos0 = 0;  // ring position of the first tile of the current item
    for (int it = 0, item = blockIdx.x; item < num_items; ++it, item += gridDim.x) {
      const Item w = item_of(p, item);
      const int b = it & 1;
      const int ub = it >> 1;
      const int c0 = w.chunk * C::kChunk;
      const int ntiles = item_tiles(p, w.chunk, C::kChunk);
      const int64_t req = row_request(p, w.row);
      const int count = row_count(p, w.row);
      const int limit = min(p.topk, count);

      // ---- this warp's query heads -> FP8 terms (lane owns dims 4*lane..+3)
      constexpr int kHeadsPerLoader = (G + kLoaders - 1) / kLoaders;
      uint32_t qpk[kHeadsPerLoader][kTerms];
      float qsc[kHeadsPerLoader];
#pragma unroll
      for (int hh = 0; hh < kHeadsPerLoader; ++hh) {
        const int h = lw + hh * kLoaders;
        qsc[hh] = 0.f;
#pragma unroll
        for (int j = 0; j < kTerms; ++j) qpk[hh][j] = 0u;
        if (h < G) {
          const int64_t qoff = ((int64_t)w.row * p.num_q_heads + w.g * G + h) * kHeadDim + lane * 4;
          const uint2 raw = *reinterpret_cast<const uint2*>(p.q + qoff);
          const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.x));
          const float2 c = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.y));
          const float x[4] = {a.x, a.y, c.x, c.y};
          float amax = fmaxf(fmaxf(fabsf(x[0]), fabsf(x[1])), fmaxf(fabsf(x[2]), fabsf(x[3])));
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
          int e = 0;  // 2^e maps the head's largest |q| into [128, 256)
          if (amax > 0.f && amax <= 3.0e38f) {
            const int ex = (int)((__float_as_uint(amax) >> 23) & 0xff) - 127;
            e = min(max(7 - ex, -120), 120);
          }
          const float sc = __uint_as_float((uint32_t)(127 + e) << 23);
#pragma unroll
          for (int d = 0; d < 4; ++d) {
            uint8_t tt[kTerms];
            split_terms(x[d] * sc, tt);
#pragma unroll
            for (int j = 0; j < kTerms; ++j) qpk[hh][j] |= (uint32_t)tt[j] << (8 * d);
          }
          qsc[hh] = __uint_as_float((uint32_t)(127 - e) << 23) * p.score_scale_log2;
        }
      }

      // ---- decode this warp's tile(s): index loads, then block-table loads
      constexpr int kMyTiles = (C::kTiles + kLoaders - 1) / kLoaders;
      int coord[kMyTiles][4];
#pragma unroll
      for (int mt = 0; mt < kMyTiles; ++mt) {
        const int j = lw + mt * kLoaders;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int col = c0 + j * kTile + lane * 4 + e;
          coord[mt][e] = (req >= 0 && j < ntiles && col < limit)
                             ? __ldg(p.indices + (int64_t)w.row * p.indices_stride + col)
                             : -1;
        }
      }
      const int32_t* bt_row = p.btable + (req >= 0 ? req : 0) * p.btable_stride;
#pragma unroll
      for (int mt = 0; mt < kMyTiles; ++mt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int t = coord[mt][e];
          int lp, po;
          if (p.page_shift >= 0) {
            lp = t >> p.page_shift;
            po = t & ((1 << p.page_shift) - 1);
          } else {
            lp = t / p.page_size;
            po = t - lp * p.page_size;
          }
          const bool ok = t >= 0 && lp < p.pages_per_req;
          const int64_t phys = ok ? (int64_t)__ldg(bt_row + lp) : -1;
          coord[mt][e] = (phys >= 0 && phys < p.num_pages)
                             ? (int)((phys * p.page_size + po) * p.num_kv_heads + w.g)
                             : -1;
        }

      // ---- per-item operands into buffer b once the softmax of item it-2 is done
      if (ub > 0 && !__all_sync(0xffffffffu, wait_or_abort(meta_empty + b, (uint32_t)((ub - 1) & 1), abort_flag))) {
        failed = true;
        break;
      }
      uint8_t* qs = smem + C::kQs + b * C::kQsBytes;
#pragma unroll
      for (int hh = 0; hh < kHeadsPerLoader; ++hh) {
        const int h = lw + hh * kLoaders;
        if (h < G) {
#pragma unroll
          for (int j = 0; j < kTerms; ++j)
            *reinterpret_cast<uint32_t*>(qs + sw128_offset(h * kTerms + j, lane * 4)) = qpk[hh][j];
          if (lane == 0) qinv[b * G + h] = qsc[hh];
        }
      }
      if (lw == 0)
        for (int r = G * kTerms; r < C::N; ++r)  // zero padding rows of Qs
          *reinterpret_cast<uint32_t*>(qs + r * 128 + lane * 4) = 0u;
#pragma unroll
      for (int mt = 0; mt < kMyTiles; ++mt) {
        const int j = lw + mt * kLoaders;
        if (j < C::kTiles) {
          const uint32_t vb = (coord[mt][0] >= 0 ? 1u : 0u) | (coord[mt][1] >= 0 ? 0x100u : 0u) |
                              (coord[mt][2] >= 0 ? 0x10000u : 0u) | (coord[mt][3] >= 0 ? 0x1000000u : 0u);
          *reinterpret_cast<uint32_t*>(valid + b * C::kChunk + j * kTile + lane * 4) = vb;
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(q_full + b);

      // ---- K tile and V tile of each of this warp's tiles into the ring
#pragma unroll
      for (int mt = 0; mt < kMyTiles; ++mt) {
        const int j = lw + mt * kLoaders;
        if (j >= ntiles) break;
        *reinterpret_cast<int4*>(rowtab + lane * 4) = make_int4(coord[mt][0], coord[mt][1], coord[mt][2], coord[mt][3]);
        __syncwarp();
#pragma unroll
        for (int kv = 0; kv < 2; ++kv) {
          const int pos = pos0 + kv * ntiles + j;  // K tiles first, then V tiles
          const int slot = pos % C::kSlots;
          const int use = pos / C::kSlots;
          if (use > 0 &&
              !__all_sync(0xffffffffu, wait_or_abort(kv_empty + slot, (uint32_t)((use - 1) & 1), abort_flag))) {
            failed = true;
            break;
          }
          const uint8_t* src_base = kv == 0 ? p.k : p.v;
          const uint32_t dst = base_s + C::kSlotBase + (uint32_t)slot * kTileBytes;
          // a warp instruction copies 4 whole 128-byte rows (8 lanes per row)
#pragma unroll 8
          for (int i = 0; i < kTile / 4; ++i) {
            const int r = i * 4 + (lane >> 3);
            const int ch = lane & 7;
            const int rc = rowtab[r];
            const uint8_t* src = rc >= 0 ? src_base + (int64_t)rc * kHeadDim + ch * 16 : src_base;
            cp_async_16(dst + sw128_offset(r, ch * 16), src, rc >= 0 ? 16u : 0u);
          }
          cp_async_mbar_arrive_noinc(kv_full + slot);
        }
        if (failed) break;
        __syncwarp();
      }
      if (failed) break;
      pos0 += 2 * ntiles;
    }
    cp_async_wait<0>();
  } else if (warp == kMmaWarp) {
    // ================================= MMA ==================================
    if (lane == 0) {
      int t = 0;           // ring position of the next K tile
      int prev_v = 0;      // ring position of the previous item's first V tile
      int prev_tiles = 0;  // tiles of the previous item
      int prev_it = -1;
      auto issue_o = [&](int jt, int vpos, int ntiles) -> bool {
        const int b = jt & 1;
        if (!wait_or_abort(p_full + b, (uint32_t)((jt >> 1) & 1), abort_flag)) return false;
        tc_fence_after();
        const uint32_t d = tmem + b * C::kBufCols + C::kTiles * C::N;
        for (int j = 0; j < ntiles; ++j) {
          const int pos = vpos + j;
          const int slot = pos % C::kSlots;
          if (!wait_or_abort(kv_full + slot, (uint32_t)((pos / C::kSlots) & 1), abort_flag)) return false;
          tc_fence_after();
          const uint32_t a0 = base_s + C::kSlotBase + (uint32_t)slot * kTileBytes;
          const uint32_t b0 = base_s + C::kPs + b * C::kPsBytes + j * C::N * 128;
#pragma unroll
          for (int kk = 0; kk < kTile / 32; ++kk) {
            const uint64_t ad = smem_desc_sw128(a0 + kk * 32 * 128, kTileBytes, 1024);
            const uint64_t bd = smem_desc_sw128(b0 + kk * 32, 16, 1024);
            mma_f8(d, ad, bd, C::kIdescO, (j > 0 || kk > 0) ? 1u : 0u);
          }
          mma_commit(kv_empty + slot);
        }
        mma_commit(o_full + b);
        return true;
      };
      for (int it = 0, item = blockIdx.x; item < num_items; ++it, item += gridDim.x) {
        const Item w = item_of(p, item);
        const int b = it & 1;
        const int ub = it >> 1;
        const int ntiles = item_tiles(p, w.chunk, C::kChunk);
        if (ub > 0 && !wait_or_abort(tmem_empty + b, (uint32_t)((ub - 1) & 1), abort_flag)) {
          failed = true;
          break;
        }
        tc_fence_after();
        if (!wait_or_abort(q_full + b, (uint32_t)(ub & 1), abort_flag)) {
          failed = true;
          break;
        }
        tc_fence_after();
        const uint32_t qs0 = base_s + C::kQs + b * C::kQsBytes;
        for (int j = 0; j < ntiles; ++j) {
          const int slot = t % C::kSlots;
          if (!wait_or_abort(kv_full + slot, (uint32_t)((t / C::kSlots) & 1), abort_flag)) {
            failed = true;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = base_s + C::kSlotBase + (uint32_t)slot * kTileBytes;
#pragma unroll
          for (int kk = 0; kk < kHeadDim / 32; ++kk) {
            const uint64_t ad = smem_desc_sw128(a0 + kk * 32, 16, 1024);
            const uint64_t bd = smem_desc_sw128(qs0 + kk * 32, 16, 1024);
            mma_f8(tmem + b * C::kBufCols + j * C::N, ad, bd, C::kIdescS, kk > 0 ? 1u : 0u);
          }
          mma_commit(kv_empty + slot);
          ++t;
        }
        if (failed) break;
        mma_commit(s_full + b);
        const int vpos = t;  // this item's V tiles follow its K tiles
        t += ntiles;
        if (prev_it >= 0 && !issue_o(prev_it, prev_v, prev_tiles)) {
          failed = true;
          break;
        }
        prev_it = it;
        prev_v = vpos;
        prev_tiles = ntiles;
      }
      if (!failed && prev_it >= 0 && !issue_o(prev_it, prev_v, prev_tiles)) failed = true;
    }
  } else {
    // ======================== softmax + epilogue (128 thr) ==================
    const int q4 = warp & 3;              // TMEM lane quadrant of this warp
    const int sw = warp - (kMmaWarp + 1);  // 0..3
    const int tk = q4 * 32 + lane;        // token within a tile / head dim in the epilogue
    const uint32_t lane_base = (uint32_t)(q4 * 32) << 16;
    for (int it = 0, item = blockIdx.x; item < num_items; ++it, item += gridDim.x) {
      const Item w = item_of(p, item);
      const int b = it & 1;
      const int ub = it >> 1;
      const int ntiles = item_tiles(p, w.chunk, C::kChunk);

      // gate of this thread's dim for every head, fetched early
      float gate[G];
#pragma unroll
      for (int h = 0; h < G; ++h)
        gate[h] = __bfloat162float(p.gate[((int64_t)w.row * p.num_q_heads + w.g * G + h) * kHeadDim + tk]);

      // q_full publishes the loaders' validity bytes and query scales; s_full
      // the scores. Once anything failed the group keeps walking its items
      // (the named barriers must still match) but skips the tensor memory.
      if (!failed) {
        const bool ok = wait_or_abort(q_full + b, (uint32_t)(ub & 1), abort_flag) &&
                        wait_or_abort(s_full + b, (uint32_t)(ub & 1), abort_flag);
        failed = !__all_sync(0xffffffffu, ok);
      }
      tc_fence_after();
      float sc[C::kTiles][G];
#pragma unroll
      for (int j = 0; j < C::kTiles; ++j) {
        if (j < ntiles && !failed) {
          float v[C::N];
#pragma unroll
          for (int cb = 0; cb < C::N; cb += 16) {
            float tmp[16];
            tmem_ld16(tmem + lane_base + b * C::kBufCols + j * C::N + cb, tmp);
            tmem_wait_ld();
#pragma unroll
            for (int c = 0; c < 16; ++c) v[cb + c] = tmp[c];
          }
          const bool ok = valid[b * C::kChunk + j * kTile + tk] != 0;
#pragma unroll
          for (int h = 0; h < G; ++h)
            sc[j][h] = ok ? combine_terms(v + h * kTerms) * qinv[b * G + h] : -INFINITY;
        } else {
#pragma unroll
          for (int h = 0; h < G; ++h) sc[j][h] = -INFINITY;
        }
      }
      // exact max per head over the chunk
#pragma unroll
      for (int h = 0; h < G; ++h) {
        float mx = sc[0][h];
#pragma unroll
        for (int j = 1; j < C::kTiles; ++j) mx = fmaxf(mx, sc[j][h]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        if (lane == 0) red_max[(b * 4 + sw) * G + h] = mx;
      }
      named_bar_sync(1, 128);
      float m_h[G];
#pragma unroll
      for (int h = 0; h < G; ++h) {
        const float* rm = red_max + b * 4 * G + h;
        m_h[h] = fmaxf(fmaxf(rm[0], rm[G]), fmaxf(rm[2 * G], rm[3 * G]));
        float sum = 0.f;
#pragma unroll
        for (int j = 0; j < C::kTiles; ++j) {
          const float pr = sc[j][h] == -INFINITY ? 0.f : exp2f(sc[j][h] - m_h[h]);
          sc[j][h] = pr;
          sum += pr;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        if (lane == 0) red_sum[(b * 4 + sw) * G + h] = sum;
      }
      // probabilities -> FP8 terms of p*256 (row h*kTerms+j of Ps, one byte per token)
      uint8_t* ps = smem + C::kPs + b * C::kPsBytes;
#pragma unroll
      for (int j = 0; j < C::kTiles; ++j) {
        if (j < ntiles) {
#pragma unroll
          for (int h = 0; h < G; ++h) {
            uint8_t tt[kTerms];
            split_terms(sc[j][h] * 256.0f, tt);
#pragma unroll
            for (int jj = 0; jj < kTerms; ++jj) ps[j * C::N * 128 + sw128_offset(h * kTerms + jj, tk)] = tt[jj];
          }
          for (int r = G * kTerms; r < C::N; ++r) ps[j * C::N * 128 + sw128_offset(r, tk)] = 0;
        }
      }
      fence_proxy_async_smem();
      named_bar_sync(1, 128);
      if (sw == 0 && lane == 0 && !failed) {
        mbar_arrive(p_full + b);
        mbar_arrive(meta_empty + b);
      }
      float l_h[G];
#pragma unroll
      for (int h = 0; h < G; ++h) {
        const float* rs = red_sum + b * 4 * G + h;
        l_h[h] = rs[0] + rs[G] + rs[2 * G] + rs[3 * G];
      }

      // ---- epilogue: thread = head dim tk ----------------------------------
      if (!failed) failed = !__all_sync(0xffffffffu, wait_or_abort(o_full + b, (uint32_t)(ub & 1), abort_flag));
      if (failed) continue;
      tc_fence_after();
      float v[C::N];
#pragma unroll
      for (int cb = 0; cb < C::N; cb += 16) {
        float tmp[16];
        tmem_ld16(tmem + lane_base + b * C::kBufCols + C::kTiles * C::N + cb, tmp);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < 16; ++c) v[cb + c] = tmp[c];
      }
      tc_fence_before();
      mbar_arrive(tmem_empty + b);
#pragma unroll
      for (int h = 0; h < G; ++h) {
        const float o =
            (ntiles > 0 && l_h[h] > 0.f) ? combine_terms(v + h * kTerms) * (1.0f / 256.0f) / l_h[h] : 0.f;
        const int64_t hrow = (int64_t)w.row * p.num_q_heads + w.g * G + h;
        if (p.num_chunks == 1) {
          p.out[hrow * kHeadDim + tk] = __float2bfloat16_rn(o * p.v_scale * (1.0f / (1.0f + expf(-gate[h]))));
        } else {
          const int64_t pidx = hrow * p.num_chunks + w.chunk;
          p.part_o[pidx * kHeadDim + tk] = o;
          if (tk == 0) p.part_lse[pidx] = l_h[h] > 0.f ? m_h[h] + log2f(l_h[h]) : -INFINITY;
        }
      }
    }
  }

  if (failed) {
    *abort_flag = 1;
    report_error(p, kErrTimeout);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}

// ------------------------------------------------------------------ host ----
int sm_count() {
  static std::atomic<int> counts[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  int c = counts[dev & 63].load(std::memory_order_acquire);
  if (!c) {
    if (cudaDeviceGetAttribute(&c, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || c <= 0) c = 148;
    counts[dev & 63].store(c, std::memory_order_release);
  }
  return c;
}

template <int G>
cudaError_t launch_g(const DecodeParams& p, cudaStream_t stream) {
  using C = Cfg<G>;
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
  const int64_t items = (int64_t)p.rows * p.num_kv_heads * p.num_chunks;
  if (items <= 0) return cudaSuccess;
  if (items > 0x7fffffffll) return cudaErrorInvalidValue;
  if (p.num_pages * p.page_size * p.num_kv_heads > 0x7fffffffll) return cudaErrorInvalidValue;
  const int grid = (int)(items < sm_count() ? items : sm_count());
  qsa_decode_tc_kernel<G><<<grid, kThreads, C::kSmemAlloc, stream>>>(p, (int)items);
  return cudaGetLastError();
}

}  // namespace

int tc_chunk_tokens(int group) { return group <= 8 ? 4 * kTile : 2 * kTile; }

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
