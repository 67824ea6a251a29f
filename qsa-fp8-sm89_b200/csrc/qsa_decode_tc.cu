// Tensor-core decode kernel for sm_100a: persistent, warp-specialised,
// register-staged gathers into swizzled shared memory, FP8 tcgen05 MMAs with
// TMEM accumulators.
//
// Work item = (Top-K row, KV head, chunk of up to kTiles*128 Top-K entries).
// Each CTA (one per SM) walks items blockIdx.x, blockIdx.x + gridDim.x, ...
// with four roles that overlap across items:
//
//   decoder (warp 0)   runs up to kMeta-1 items ahead: decodes the item's
//                      Top-K entries (index -> block table -> K/V row) into a
//                      row table, writes the validity bytes and the gate, and
//                      splits the G query heads into FP8 terms (operand Qs)
//                      with their scales -- one slot of a kMeta-deep
//                      metadata ring. It also starts every selected K/V row
//                      of the item on its way from HBM into L2. Its
//                      global loads are pipelined two items deep with no
//                      dependent chain: request id, count and index loads of
//                      item i+2, block-table and query loads of item i+1 are
//                      in flight while item i is finished;
//   loaders            one warp per ring slot; an item occupies consecutive
//                      ring positions (its K tiles, then its V tiles) and
//                      loader L fills the positions that map to slot L, in
//                      order: the tile's 128 rows of 128 B go through
//                      registers with coalesced 16-byte loads into the slot,
//                      stored in the 128-byte-swizzled layout the tensor core
//                      reads (zeros for masked rows);
//   MMA warp           one thread issues S = K_tile . Qs^T into TMEM for every
//                      K tile of item i+1 before O^T += V_tile^T . Ps^T for
//                      item i, so the tensor core never waits on a softmax;
//   4 softmax warps    softmax over the chunk's scores (exact max and sum),
//                      probabilities as FP8 terms of p*256 (operand Ps); then
//                      the epilogue of the previous item (its O is complete
//                      by then): recombine, normalise, v_scale, sigmoid gate,
//                      bf16 store (or a partial for the split combine).
//
// Every selected 128-byte K/V row is read from HBM once and shared by the G
// query heads. Q and P keep their precision through a split into E4M3 terms:
//   q * 2^E = t0 + t1/16                    (exact for bf16 q)
//   p * 256 = t0 + t1/16 + t2/256 + t3/2048 (about 15 bits of p)
// so the FP8 x FP8 tensor-core products reproduce the reference's fp32
// products of the FP8 cache values with bf16 q and fp32 p.
//
// Synchronisation is by mbarriers: kv_full/kv_empty per K/V ring slot,
// meta_full/meta_empty per metadata slot, s_full/o_full/tmem_empty per TMEM
// accumulator buffer (three), p_full per probability buffer (two). Every wait is bounded; a CTA
// that gives up records an error in the device error word, raises a CTA-wide
// abort flag so the other roles leave their loops, frees its TMEM and returns.
#include <atomic>

#include "qsa_common.cuh"

namespace qsa {
namespace {

constexpr int kTile = 128;                    // tokens per tile
constexpr int kTileBytes = kTile * kHeadDim;  // 16 KiB of FP8
constexpr int kTermsQ = 2;                    // FP8 terms per query value (exact for bf16)
constexpr int kTermsP = 4;                    // FP8 terms per probability
constexpr int kMeta = 4;                      // metadata ring depth (items)
constexpr int kTmemBufs = 3;                  // TMEM accumulator buffers (items)
constexpr int kDecoderWarp = 0;
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
  static constexpr int NS = ((G * kTermsQ + 15) / 16) * 16;  // N of the S MMA (rows of Qs)
  static constexpr int NO = ((G * kTermsP + 15) / 16) * 16;  // N of the O MMA (rows of a Ps tile)
  static constexpr int kTiles = G <= 8 ? 4 : 2;             // tiles per item
  static constexpr int kChunk = kTiles * kTile;             // Top-K entries per item
  // 16 warps (10 loaders) for G <= 8, 12 warps (6 loaders) for G = 16: whole
  // multiples of 4 warps, so the four 16K-register sub-partitions of the SM
  // are evenly loaded
  static constexpr int kMaxLoaders = G <= 8 ? 10 : 6;
  static constexpr int kBufCols = (kTiles * NS + NO + 31) / 32 * 32;  // S tiles + O, per TMEM buffer
  static constexpr int kTmemCols = pow2_at_least(kTmemBufs * kBufCols);
  static constexpr int kQsBytes = NS * 128;
  static constexpr int kPsBytes = kTiles * NO * 128;
  // shared memory layout (offsets from a 1024-byte aligned base); every
  // region starts on a 128-byte boundary, the MMA operands on 1024
  static constexpr int kQs = 0;                                       // [kMeta][NS][128]
  static constexpr int kPs = kQs + kMeta * kQsBytes;                  // [2][kTiles][NO][128]
  static constexpr int kRowTab = kPs + 2 * kPsBytes;                  // int32 [kMeta][kChunk] K/V rows
  static constexpr int kValid = kRowTab + kMeta * kChunk * 4;         // uint8 [kMeta][kChunk]
  static constexpr int kQinv = align128(kValid + kMeta * kChunk);     // float [kMeta][G]
  static constexpr int kGate = align128(kQinv + kMeta * G * 4);      // bf16 [kMeta][G][128]
  static constexpr int kRedMax = align128(kGate + kMeta * G * kHeadDim * 2);  // float [2][4][G]
  static constexpr int kRedSum = align128(kRedMax + 2 * 4 * G * 4);   // float [2][4][G]
  static constexpr int kBars = align128(kRedSum + 2 * 4 * G * 4);
  static constexpr int kMaxSlots = 16;
  static constexpr int kNumBars = 2 * kMaxSlots + 2 * kMeta + 3 * kTmemBufs + 2;
  static constexpr int kMisc = kBars + kNumBars * 8;                  // tmem address, abort flag
  static constexpr int kSlotBase = ((kMisc + 16 + 1023) / 1024) * 1024;
  static constexpr int kSlots0 = (kSmemLimit - 1024 - kSlotBase) / kTileBytes;
  static constexpr int kSlots = kSlots0 > kMaxLoaders ? kMaxLoaders : kSlots0;
  // warp roles: decoder, one loader warp per ring slot (loader L refills slot
  // L only, so every slot is refilled in order by one warp and no parity wait
  // can be two phases off), the MMA warp, four softmax / epilogue warps
  static constexpr int kLoaders = kSlots;                   // warps 1 .. kLoaders
  static constexpr int kMmaWarp = 1 + kLoaders;
  static constexpr int kSoftmax0 = kMmaWarp + 1;
  static constexpr int kThreads = 32 * (kSoftmax0 + 4);
  // registers per thread: each SM sub-partition has 16K registers and holds
  // a quarter of the CTA's warps
  static constexpr int kMaxRegs = (16384 / (((kThreads / 32 + 3) / 4) * 32)) / 8 * 8;
  static constexpr int kSmemAlloc = kSlotBase + kSlots * kTileBytes + 1024;
  static constexpr uint32_t kIdescS = idesc_e4m3(128, NS, false, false);
  static constexpr uint32_t kIdescO = idesc_e4m3(128, NO, true, false);
  static_assert(kSlots >= 2 * kTiles, "ring must hold a K and a V chunk");
  static_assert(kSlots <= kMaxSlots, "barrier array size");
  static_assert(kSmemAlloc <= kSmemLimit, "shared memory budget");
  static_assert(kTmemCols <= 512, "TMEM budget");
  static_assert(kQs % 1024 == 0 && kPs % 1024 == 0 && kSlotBase % 1024 == 0 && kQsBytes % 1024 == 0 &&
                    (NO * 128) % 1024 == 0,
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
// Start moving the 128-byte line at `ptr` from HBM into L2 (no data returns
// to the SM, so it occupies no shared memory and no load slot).
__device__ __forceinline__ void prefetch_l2(const void* ptr) {
  asm volatile("prefetch.global.L2 [%0];\n" ::"l"(ptr));
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

// Splits an f16 pair into nt E4M3 terms per value, two values per
// conversion: x ~= t0 + t1/16 + t2/256 (t[j] = hi byte : lo byte). Every step
// is exact (x - t_j fits in f16, the scaling by 16 is a power of two); three
// terms hold any f16 value, two hold any value with at most 8 significant bits.
template <int nt>
__device__ __forceinline__ void split_f16x2(__half2 x, uint16_t (&t)[nt]) {
  const __half2 sixteen = __float2half2_rn(16.0f);
#pragma unroll
  for (int j = 0; j < nt; ++j) {
    t[j] = __nv_cvt_halfraw2_to_fp8x2(static_cast<__half2_raw>(x), __NV_SATFINITE, __NV_E4M3);
    if (j + 1 < nt) {
      const __half2 back(__nv_cvt_fp8x2_to_halfraw2(t[j], __NV_E4M3));
      x = __hmul2(__hsub2(x, back), sixteen);
    }
  }
}

// Query pair (|x| < 448, bf16 values scaled by a power of two): two exact
// E4M3 terms each, x = t0 + t1/16.
__device__ __forceinline__ void split_q2(float lo, float hi, uint16_t (&t)[kTermsQ]) {
  split_f16x2<kTermsQ>(__floats2half2_rn(lo, hi), t);
}

// Probability pair (x = p * 256 <= 256): x ~= t0 + t1/16 + t2/256 + t3/2048,
// the first three terms the exact split of f16(x), the fourth the E4M3
// rounding of the f16 residual (x - f16(x)) * 2^11 -- about 15 bits of p.
__device__ __forceinline__ void split_p2(float lo, float hi, uint16_t (&t)[kTermsP]) {
  const __half2 h = __floats2half2_rn(lo, hi);
  const float2 hf = __half22float2(h);
  uint16_t t3[3];
  split_f16x2<3>(h, t3);
  t[0] = t3[0];
  t[1] = t3[1];
  t[2] = t3[2];
  const __half2 r = __floats2half2_rn((lo - hf.x) * 2048.0f, (hi - hf.y) * 2048.0f);
  t[3] = __nv_cvt_halfraw2_to_fp8x2(static_cast<__half2_raw>(r), __NV_SATFINITE, __NV_E4M3);
}

// Recombine the per-term accumulator columns of one head.
__device__ __forceinline__ float combine_q(const float* v) { return v[0] + v[1] * 0.0625f; }
__device__ __forceinline__ float combine_p(const float* v) {
  return v[0] + v[1] * 0.0625f + v[2] * 0.00390625f + v[3] * 0.00048828125f;
}

// First-stage loads of one item for the decoder, all independent of each
// other: the request id, the row's valid count and the Top-K indices (lane
// owns entries lane*4..+3 of every tile). Columns past the selection read -1;
// the count and the request id are applied when the item is finished.
template <int kTiles>
struct IndexStage {
  int tok[kTiles][4];
  int req;    // t2r[row] (unchecked)
  int limit;  // min(topk, count)
};

template <int kTiles>
__device__ __forceinline__ void load_index_stage(const DecodeParams& p, int item, int chunk_tokens, int lane,
                                                 IndexStage<kTiles>& st) {
  const Item w = item_of(p, item);
  const int c0 = w.chunk * chunk_tokens;
  st.req = p.t2r ? __ldg(p.t2r + w.row) : w.row;
  st.limit = p.counts ? __ldg(p.counts + w.row)
                      : (p.count_column ? __ldg(p.indices + (int64_t)w.row * p.indices_stride + p.topk) : p.topk);
  const int32_t* idx_row = p.indices + (int64_t)w.row * p.indices_stride;
#pragma unroll
  for (int j = 0; j < kTiles; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int col = c0 + j * kTile + lane * 4 + e;
      st.tok[j][e] = col < p.topk ? __ldg(idx_row + col) : -1;
    }
}

// Applies the row rules of token_slot to a loaded stage: the request id must
// index the block table and the column must lie below the row's count.
template <int kTiles>
__device__ __forceinline__ void mask_index_stage(const DecodeParams& p, int item, int chunk_tokens, int lane,
                                                 IndexStage<kTiles>& st) {
  const Item w = item_of(p, item);
  const int c0 = w.chunk * chunk_tokens;
  const bool req_ok = st.req >= 0 && st.req < p.num_reqs;
  const int limit = min(p.topk, max(st.limit, 0));
#pragma unroll
  for (int j = 0; j < kTiles; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int col = c0 + j * kTile + lane * 4 + e;
      if (!req_ok || col >= limit) st.tok[j][e] = -1;
    }
  if (!req_ok) st.req = 0;
}

template <int G>
__global__ void __launch_bounds__(Cfg<G>::kThreads) __maxnreg__(Cfg<G>::kMaxRegs)
    qsa_decode_tc_kernel(const __grid_constant__ DecodeParams p, int num_items) {
  using C = Cfg<G>;
  constexpr int kLoaders = C::kLoaders;
  constexpr int kMmaWarp = C::kMmaWarp;
  constexpr int kSoftmax0 = C::kSoftmax0;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_s = smem_u32(smem_raw);
  const uint32_t base_s = (raw_s + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base_s - raw_s);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kBars);
  uint64_t* kv_full = bars;                        // [kSlots] loader -> MMA
  uint64_t* kv_empty = bars + C::kMaxSlots;        // [kSlots] MMA commit -> loader
  uint64_t* meta_full = bars + 2 * C::kMaxSlots;   // [kMeta] decoder -> loaders, MMA, softmax
  uint64_t* meta_empty = meta_full + kMeta;        // [kMeta] loaders + MMA commit + softmax -> decoder
  uint64_t* s_full = meta_empty + kMeta;           // [kTmemBufs] MMA commit -> softmax
  uint64_t* o_full = s_full + kTmemBufs;           // [kTmemBufs] MMA commit -> epilogue
  uint64_t* tmem_empty = o_full + kTmemBufs;       // [kTmemBufs] epilogue (128 arrivals) -> MMA
  uint64_t* p_full = tmem_empty + kTmemBufs;       // [2] softmax -> MMA (Ps double buffer)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::kMisc + 8);
  float* qinv = reinterpret_cast<float*>(smem + C::kQinv);
  float* red_max = reinterpret_cast<float*>(smem + C::kRedMax);
  float* red_sum = reinterpret_cast<float*>(smem + C::kRedSum);
  uint8_t* valid = smem + C::kValid;
  int32_t* rowtab = reinterpret_cast<int32_t*>(smem + C::kRowTab);

  if (tid == 0) {
    for (int i = 0; i < C::kSlots; ++i) {
      mbar_init(kv_full + i, 1);
      mbar_init(kv_empty + i, 1);
    }
    for (int m = 0; m < kMeta; ++m) {
      mbar_init(meta_full + m, 1);
      mbar_init(meta_empty + m, kLoaders + 2);
    }
    for (int b = 0; b < kTmemBufs; ++b) {
      mbar_init(s_full + b, 1);
      mbar_init(o_full + b, 1);
      mbar_init(tmem_empty + b, 128);
    }
    for (int b = 0; b < 2; ++b) mbar_init(p_full + b, 1);
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

  if (warp == kDecoderWarp) {
    // =============================== decoder ================================
    // Software pipeline, two items deep: while item i is finished, the block
    // table and query loads of item i+1 and the index loads of item i+2 are
    // in flight, so one memory round trip per item overlaps everything else.
    const int stride = gridDim.x;
    IndexStage<C::kTiles> st_a;  // item i+2: indices, request id, count (in flight)
    IndexStage<C::kTiles> st_b;  // item i+1: masked indices
    int phys_b[C::kTiles][4];    // block-table entries of item i+1 (in flight), -1 = masked
    uint2 q_b[G];                // query of item i+1 (in flight)
    uint2 gate_b[G];             // gate of item i+1 (in flight)
    auto issue_rest = [&](int item) {  // block-table + query loads of `item`, from st_b
      const Item w = item_of(p, item);
      const int32_t* bt_row = p.btable + (int64_t)st_b.req * p.btable_stride;
#pragma unroll
      for (int j = 0; j < C::kTiles; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int t = st_b.tok[j][e];
          const int lp = p.page_shift >= 0 ? (t >> p.page_shift) : t / p.page_size;
          const bool ok = t >= 0 && lp < p.pages_per_req;
          phys_b[j][e] = ok ? __ldg(bt_row + lp) : -1;
        }
#pragma unroll
      for (int h = 0; h < G; ++h) {
        const int64_t off = ((int64_t)w.row * p.num_q_heads + w.g * G + h) * kHeadDim + lane * 4;
        q_b[h] = *reinterpret_cast<const uint2*>(p.q + off);
        gate_b[h] = *reinterpret_cast<const uint2*>(p.gate + off);
      }
    };
    const int item0 = blockIdx.x;
    if (item0 < num_items) {
      load_index_stage<C::kTiles>(p, item0, C::kChunk, lane, st_b);
      mask_index_stage<C::kTiles>(p, item0, C::kChunk, lane, st_b);
      issue_rest(item0);
      if (item0 + stride < num_items) load_index_stage<C::kTiles>(p, item0 + stride, C::kChunk, lane, st_a);
    }
    for (int it = 0, item = item0; item < num_items; ++it, item += stride) {
      const Item w = item_of(p, item);
      const int m = it % kMeta;
      const int um = it / kMeta;

      // results of item i (loads issued one iteration ago)
      int coord[C::kTiles][4];
      uint2 q_c[G];
#pragma unroll
      for (int j = 0; j < C::kTiles; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int t = st_b.tok[j][e];
          const int po = p.page_shift >= 0 ? (t & ((1 << p.page_shift) - 1)) : t % p.page_size;
          const int64_t phys = phys_b[j][e];
          coord[j][e] = (t >= 0 && phys >= 0 && phys < p.num_pages)
                            ? (int)((phys * p.page_size + po) * p.num_kv_heads + w.g)
                            : -1;
        }
      uint2 gate_c[G];
#pragma unroll
      for (int h = 0; h < G; ++h) {
        q_c[h] = q_b[h];
        gate_c[h] = gate_b[h];
      }
      // pull every selected K and V row of item i towards L2 now: the loaders
      // copy them into shared memory an item or more later, and by then the
      // copies hit L2, so the ring never has to cover a full HBM round trip
#pragma unroll
      for (int j = 0; j < C::kTiles; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e)
          if (coord[j][e] >= 0) {
            prefetch_l2(p.k + (int64_t)coord[j][e] * kHeadDim);
            prefetch_l2(p.v + (int64_t)coord[j][e] * kHeadDim);
          }
      // launch the loads of items i+1 and i+2
      if (item + stride < num_items) {
        st_b = st_a;
        mask_index_stage<C::kTiles>(p, item + stride, C::kChunk, lane, st_b);
        issue_rest(item + stride);
        if (item + 2 * stride < num_items)
          load_index_stage<C::kTiles>(p, item + 2 * stride, C::kChunk, lane, st_a);
      }

      // query heads -> FP8 terms (lane owns dims 4*lane .. 4*lane+3)
      uint32_t qpk[G][kTermsQ];
      float qsc[G];
#pragma unroll
      for (int h = 0; h < G; ++h) {
        const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&q_c[h].x));
        const float2 c = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&q_c[h].y));
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
        uint16_t t01[kTermsQ], t23[kTermsQ];
        split_q2(x[0] * sc, x[1] * sc, t01);
        split_q2(x[2] * sc, x[3] * sc, t23);
#pragma unroll
        for (int j = 0; j < kTermsQ; ++j) qpk[h][j] = (uint32_t)t01[j] | ((uint32_t)t23[j] << 16);
        qsc[h] = __uint_as_float((uint32_t)(127 - e) << 23) * p.score_scale_log2;
      }

      // metadata slot m is free once item it-kMeta is fully consumed
      if (um > 0 &&
          !__all_sync(0xffffffffu, wait_or_abort(meta_empty + m, (uint32_t)((um - 1) & 1), abort_flag))) {
        failed = true;
        break;
      }
      uint8_t* qs = smem + C::kQs + m * C::kQsBytes;
#pragma unroll
      for (int h = 0; h < G; ++h) {
#pragma unroll
        for (int j = 0; j < kTermsQ; ++j)
          *reinterpret_cast<uint32_t*>(qs + sw128_offset(h * kTermsQ + j, lane * 4)) = qpk[h][j];
        if (lane == h) qinv[m * G + h] = qsc[h];
        *reinterpret_cast<uint2*>(smem + C::kGate + ((m * G + h) * kHeadDim + lane * 4) * 2) = gate_c[h];
      }
      for (int r = G * kTermsQ; r < C::NS; ++r)  // zero padding rows of Qs
        *reinterpret_cast<uint32_t*>(qs + r * 128 + lane * 4) = 0u;
#pragma unroll
      for (int j = 0; j < C::kTiles; ++j) {
        *reinterpret_cast<int4*>(rowtab + m * C::kChunk + j * kTile + lane * 4) =
            make_int4(coord[j][0], coord[j][1], coord[j][2], coord[j][3]);
        const uint32_t vb = (coord[j][0] >= 0 ? 1u : 0u) | (coord[j][1] >= 0 ? 0x100u : 0u) |
                            (coord[j][2] >= 0 ? 0x10000u : 0u) | (coord[j][3] >= 0 ? 0x1000000u : 0u);
        *reinterpret_cast<uint32_t*>(valid + m * C::kChunk + j * kTile + lane * 4) = vb;
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(meta_full + m);
    }
  } else if (warp <= kLoaders) {
    // =============================== loaders ================================
    // Loader warp 1+L owns ring slot L: it copies every ring position p with
    // p % kSlots == L, in order. An item's positions are its K tiles, then its
    // V tiles. The 128 rows of a tile go through registers into the swizzled
    // slot, then one fence + arrive publishes the tile.
    const int L = warp - 1;
    int pos0 = 0;  // ring position of the first tile of the current item
    int use = 0;   // fills of slot L so far
    for (int it = 0, item = blockIdx.x; item < num_items; ++it, item += gridDim.x) {
      const Item w = item_of(p, item);
      const int m = it % kMeta;
      const int ntiles = item_tiles(p, w.chunk, C::kChunk);
      if (!__all_sync(0xffffffffu, wait_or_abort(meta_full + m, (uint32_t)((it / kMeta) & 1), abort_flag))) {
        failed = true;
        break;
      }
      for (int pos = pos0 + (L - pos0 % C::kSlots + C::kSlots) % C::kSlots; pos < pos0 + 2 * ntiles;
           pos += C::kSlots, ++use) {
        const int s = pos - pos0;
        const bool is_v = s >= ntiles;
        const int j = is_v ? s - ntiles : s;
        const uint8_t* src_base = is_v ? p.v : p.k;
        const int32_t* tab = rowtab + m * C::kChunk + j * kTile;
        if (use > 0 &&
            !__all_sync(0xffffffffu, wait_or_abort(kv_empty + L, (uint32_t)((use - 1) & 1), abort_flag))) {
          failed = true;
          break;
        }
        uint8_t* dst = smem + C::kSlotBase + L * kTileBytes;
        // two batches of 16 warp loads; a warp load covers 4 whole 128-byte
        // rows (8 lanes per row)
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          uint4 buf[kTile / 8];
#pragma unroll
          for (int i = 0; i < kTile / 8; ++i) {
            const int r = (half * (kTile / 8) + i) * 4 + (lane >> 3);
            const int rc = tab[r];
            buf[i] = rc >= 0 ? __ldcs(reinterpret_cast<const uint4*>(src_base + (int64_t)rc * kHeadDim +
                                                                    (lane & 7) * 16))
                             : make_uint4(0u, 0u, 0u, 0u);
          }
#pragma unroll
          for (int i = 0; i < kTile / 8; ++i) {
            const int r = (half * (kTile / 8) + i) * 4 + (lane >> 3);
            *reinterpret_cast<uint4*>(dst + sw128_offset(r, (lane & 7) * 16)) = buf[i];
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(kv_full + L);
      }
      if (failed) break;
      __syncwarp();
      if (lane == 0) mbar_arrive(meta_empty + m);  // this warp is done with the row table
      pos0 += 2 * ntiles;
    }
  } else if (warp == kMmaWarp) {
    // ================================= MMA ==================================
    if (lane == 0) {
      int t = 0;           // ring position of the next K tile
      int prev_v = 0;      // ring position of the previous item's first V tile
      int prev_tiles = 0;  // tiles of the previous item
      int prev_it = -1;
      auto issue_o = [&](int jt, int vpos, int ntiles) -> bool {
        const int pb = jt & 1;
        if (!wait_or_abort(p_full + pb, (uint32_t)((jt >> 1) & 1), abort_flag)) return false;
        tc_fence_after();
        const int tb = jt % kTmemBufs;
        const uint32_t d = tmem + tb * C::kBufCols + C::kTiles * C::NS;
        for (int j = 0; j < ntiles; ++j) {
          const int pos = vpos + j;
          const int slot = pos % C::kSlots;
          if (!wait_or_abort(kv_full + slot, (uint32_t)((pos / C::kSlots) & 1), abort_flag)) return false;
          tc_fence_after();
          const uint32_t a0 = base_s + C::kSlotBase + (uint32_t)slot * kTileBytes;
          const uint32_t b0 = base_s + C::kPs + pb * C::kPsBytes + j * C::NO * 128;
#pragma unroll
          for (int kk = 0; kk < kTile / 32; ++kk) {
            const uint64_t ad = smem_desc_sw128(a0 + kk * 32 * 128, kTileBytes, 1024);
            const uint64_t bd = smem_desc_sw128(b0 + kk * 32, 16, 1024);
            mma_f8(d, ad, bd, C::kIdescO, (j > 0 || kk > 0) ? 1u : 0u);
          }
          mma_commit(kv_empty + slot);
        }
        mma_commit(o_full + tb);
        return true;
      };
      for (int it = 0, item = blockIdx.x; item < num_items; ++it, item += gridDim.x) {
        const Item w = item_of(p, item);
        const int tb = it % kTmemBufs;
        const int ut = it / kTmemBufs;
        const int m = it % kMeta;
        const int ntiles = item_tiles(p, w.chunk, C::kChunk);
        if (ut > 0 && !wait_or_abort(tmem_empty + tb, (uint32_t)((ut - 1) & 1), abort_flag)) {
          failed = true;
          break;
        }
        tc_fence_after();
        if (!wait_or_abort(meta_full + m, (uint32_t)((it / kMeta) & 1), abort_flag)) {
          failed = true;
          break;
        }
        tc_fence_after();
        const uint32_t qs0 = base_s + C::kQs + m * C::kQsBytes;
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
            mma_f8(tmem + tb * C::kBufCols + j * C::NS, ad, bd, C::kIdescS, kk > 0 ? 1u : 0u);
          }
          mma_commit(kv_empty + slot);
          ++t;
        }
        if (failed) break;
        mma_commit(s_full + tb);
        mma_commit(meta_empty + m);  // Qs of slot m is read once these MMAs finish
        const int vpos = t;          // this item's V tiles follow its K tiles
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
    // Software pipelined: the softmax of item i runs before the epilogue of
    // item i-1, whose O accumulation has finished meanwhile.
    const int q4 = warp & 3;          // TMEM lane quadrant of this warp
    const int sw = warp - kSoftmax0;  // 0..3
    const int tk = q4 * 32 + lane;    // token within a tile / head dim in the epilogue
    const uint32_t lane_base = (uint32_t)(q4 * 32) << 16;
    // state of the item whose epilogue is pending
    int e_it = -1, e_row = 0, e_g = 0, e_chunk = 0, e_ntiles = 0;
    float e_m[G], e_l[G], e_gate[G];
    auto epilogue = [&]() {
      const int tb = e_it % kTmemBufs;
      if (!failed)
        failed = !__all_sync(0xffffffffu, wait_or_abort(o_full + tb, (uint32_t)((e_it / kTmemBufs) & 1), abort_flag));
      if (failed) return;
      tc_fence_after();
      float v[C::NO];
#pragma unroll
      for (int cb = 0; cb < C::NO; cb += 16) {
        float tmp[16];
        tmem_ld16(tmem + lane_base + tb * C::kBufCols + C::kTiles * C::NS + cb, tmp);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < 16; ++c) v[cb + c] = tmp[c];
      }
      tc_fence_before();
      mbar_arrive(tmem_empty + tb);
#pragma unroll
      for (int h = 0; h < G; ++h) {
        const float o = (e_ntiles > 0 && e_l[h] > 0.f) ? combine_p(v + h * kTermsP) * (1.0f / 256.0f) / e_l[h]
                                                         : 0.f;
        const int64_t hrow = (int64_t)e_row * p.num_q_heads + e_g * G + h;
        if (p.num_chunks == 1) {
          p.out[hrow * kHeadDim + tk] = __float2bfloat16_rn(o * p.v_scale * (1.0f / (1.0f + expf(-e_gate[h]))));
        } else {
          const int64_t pidx = hrow * p.num_chunks + e_chunk;
          p.part_o[pidx * kHeadDim + tk] = o;
          if (tk == 0) p.part_lse[pidx] = e_l[h] > 0.f ? e_m[h] + log2f(e_l[h]) : -INFINITY;
        }
      }
    };
    for (int it = 0, item = blockIdx.x; item < num_items; ++it, item += gridDim.x) {
      const Item w = item_of(p, item);
      const int tb = it % kTmemBufs;
      const int pb = it & 1;
      const int m = it % kMeta;
      const int ntiles = item_tiles(p, w.chunk, C::kChunk);

      // meta_full publishes the decoder's validity bytes, query scales and gate;
      // s_full the scores. Once anything failed the group keeps walking its
      // items (the named barriers must still match) but skips tensor memory.
      if (!failed) {
        const bool ok = wait_or_abort(meta_full + m, (uint32_t)((it / kMeta) & 1), abort_flag) &&
                        wait_or_abort(s_full + tb, (uint32_t)((it / kTmemBufs) & 1), abort_flag);
        failed = !__all_sync(0xffffffffu, ok);
      }
      tc_fence_after();
      float qi[G], gate[G];
      const __nv_bfloat16* gsm = reinterpret_cast<const __nv_bfloat16*>(smem + C::kGate) + m * G * kHeadDim;
#pragma unroll
      for (int h = 0; h < G; ++h) {
        qi[h] = qinv[m * G + h];
        gate[h] = __bfloat162float(gsm[h * kHeadDim + tk]);
      }
      float sc[C::kTiles][G];
#pragma unroll
      for (int j = 0; j < C::kTiles; ++j) {
        if (j < ntiles && !failed) {
          float v[C::NS];
#pragma unroll
          for (int cb = 0; cb < C::NS; cb += 16) {
            float tmp[16];
            tmem_ld16(tmem + lane_base + tb * C::kBufCols + j * C::NS + cb, tmp);
            tmem_wait_ld();
#pragma unroll
            for (int c = 0; c < 16; ++c) v[cb + c] = tmp[c];
          }
          const bool ok = valid[m * C::kChunk + j * kTile + tk] != 0;
#pragma unroll
          for (int h = 0; h < G; ++h) sc[j][h] = ok ? combine_q(v + h * kTermsQ) * qi[h] : -INFINITY;
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
        if (lane == 0) red_max[(pb * 4 + sw) * G + h] = mx;
      }
      named_bar_sync(1, 128);
      if (sw == 0 && lane == 0 && !failed) mbar_arrive(meta_empty + m);  // validity, scales and gate read
      float m_h[G];
#pragma unroll
      for (int h = 0; h < G; ++h) {
        const float* rm = red_max + pb * 4 * G + h;
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
        if (lane == 0) red_sum[(pb * 4 + sw) * G + h] = sum;
      }
      // probabilities -> FP8 terms of p*256 (row h*kTermsP+j of Ps, one byte per
      // token), two heads per conversion
      uint8_t* ps = smem + C::kPs + pb * C::kPsBytes;
#pragma unroll
      for (int j = 0; j < C::kTiles; ++j) {
        if (j < ntiles) {
          uint8_t* pt = ps + j * C::NO * 128;
#pragma unroll
          for (int h = 0; h < G; h += 2) {
            uint16_t tt[kTermsP];
            split_p2(sc[j][h] * 256.0f, h + 1 < G ? sc[j][h + 1] * 256.0f : 0.f, tt);
#pragma unroll
            for (int jj = 0; jj < kTermsP; ++jj) {
              pt[sw128_offset(h * kTermsP + jj, tk)] = (uint8_t)(tt[jj] & 0xffu);
              if (h + 1 < G) pt[sw128_offset((h + 1) * kTermsP + jj, tk)] = (uint8_t)(tt[jj] >> 8);
            }
          }
          for (int r = G * kTermsP; r < C::NO; ++r) pt[sw128_offset(r, tk)] = 0;
        }
      }
      fence_proxy_async_smem();
      named_bar_sync(1, 128);
      if (sw == 0 && lane == 0 && !failed) mbar_arrive(p_full + pb);
      float l_h[G];
#pragma unroll
      for (int h = 0; h < G; ++h) {
        const float* rs = red_sum + pb * 4 * G + h;
        l_h[h] = rs[0] + rs[G] + rs[2 * G] + rs[3 * G];
      }

      // ---- epilogue of the previous item, then this item becomes pending ---
      if (e_it >= 0) epilogue();
      e_it = it;
      e_row = w.row;
      e_g = w.g;
      e_chunk = w.chunk;
      e_ntiles = ntiles;
#pragma unroll
      for (int h = 0; h < G; ++h) {
        e_m[h] = m_h[h];
        e_l[h] = l_h[h];
        e_gate[h] = gate[h];
      }
    }
    if (e_it >= 0) epilogue();
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
  qsa_decode_tc_kernel<G><<<grid, C::kThreads, C::kSmemAlloc, stream>>>(p, (int)items);
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
