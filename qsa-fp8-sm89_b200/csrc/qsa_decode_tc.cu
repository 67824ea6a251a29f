// Tensor-core decode kernel for sm_100a: persistent, warp-specialised, TMA
// gathers into swizzled shared memory, FP8 tcgen05 MMAs with TMEM accumulators.
//
// The index decode runs first, in its own small kernel (qsa_rowmap_kernel):
// every Top-K entry becomes its physical token slot phys * P + t % P (or -1)
// in a row map in the workspace, in parallel over the whole GPU, before the
// K/V gathers saturate HBM (under that load a dependent global read waits
// several microseconds). The decode kernel is a programmatic dependent launch
// of it: its prologue (barriers, TMEM, tensor maps) overlaps the row map, and
// only the decoder warp (and, for split rows, the softmax warps, which read
// the tile flags) waits for the row map (griddepcontrol.wait) before its
// first read of it. The pipeline then needs no dependent global reads of
// its own.
//
// Work item = (Top-K row, KV head, chunk of up to kTiles*128 Top-K entries).
// A group of more than 16 query heads runs as two virtual KV heads per cache
// KV head, each with about half of the query heads (launch_decode_tc).
// With unsplit rows each CTA (one per SM) takes items blockIdx.x,
// blockIdx.x + gridDim.x, ... (its k-th item is blockIdx.x + k * gridDim.x,
// k < n_my). With split rows it walks windows of items claimed from a
// per-call counter and leaves out the chunks that hold no valid entry (see
// ItemWalk). The decoder publishes the item id with the item's metadata
// slot, and an id of -1 after the last item ends the loaders', the MMA
// warp's and (split rows) the softmax warps' loops. Four roles overlap
// across items:
//
//   decoder (warp 0)   for a kMeta-deep metadata ring: TMA bulk copies bring
//                      the item's chunk of the row map into the slot's row
//                      table, with the chunk's tile flags (which 128-entry
//                      tiles hold a valid entry; the others are skipped by
//                      every role), and the G query heads are split into FP8
//                      terms (operand Qs) with their scales;
//   loaders            the ring of 16 KiB tile slots is filled in the order
//                      the MMA warp drains it: K tiles of item k, then V tiles
//                      of item k-1. Slot s belongs to loader s % kLoaders, which
//                      refills it in order. A tile is 128 rows of 128 B: each
//                      lane issues one TMA tile::gather4 of four rows (the
//                      cache viewed as a [rows, 128] byte tensor, row
//                      slot * Hkv + g; a masked entry has row -1 and reads
//                      zeros), which lands in the 128-byte-swizzled layout the
//                      tensor core reads and completes the slot's transaction
//                      count;
//   MMA warp           one thread issues S = K_tile . Qs^T into TMEM for every
//                      K tile of item k, then O^T += V_tile^T . Ps^T for item
//                      k-1 (its probabilities are ready by then);
//   softmax warps      one set of four (one per TMEM lane quadrant), or for
//                      G >= 5 two independent sets, each taking half of the
//                      heads (odd G padded by one head) with its own named
//                      barrier: softmax over the chunk's scores (exact max and
//                      sum), probabilities as FP8 terms of p*256 (operand Ps,
//                      token-major: 16 bytes per store);
//                      then the epilogue of the previous item (its O is
//                      complete by then): recombine, normalise, v_scale,
//                      sigmoid gate, bf16 store (or a partial for the split
//                      combine).
//
// Every selected 128-byte K/V row is read from HBM once and shared by the G
// query heads. Q and P keep their precision through a split into E4M3 terms:
//   q * 2^E = t0 + t1/16, where 2^E maps the head's largest |q| into
//     [128, 256): exact for every bf16 element within 2^13 of that largest
//     |q|; a smaller element keeps an absolute error of at most 2^-14 in the
//     scaled domain (under 2^-21 of the largest |q|), and one below about
//     2^-21 of it becomes 0 (E4M3's subnormals end at 2^-9);
//   p * 256 = t0 + t1/16 + t2/256 + t3/2048: about 15 significant bits of p,
//     and an absolute error under 2^-29 for the smallest p (p <= 1, the
//     chunk's maximum being 1);
// so the FP8 x FP8 tensor-core products reproduce the reference's fp32
// products of the FP8 cache values with bf16 q and fp32 p to within those
// bounds.
//
// Synchronisation is by mbarriers: kv_full/kv_empty per K/V ring slot,
// meta_full/meta_empty per metadata slot, s_full/o_full/tmem_empty per TMEM
// accumulator buffer (three, or two for G > 8), p_full per probability buffer
// (two). Every wait
// is bounded; a CTA that gives up records an error in the device error word,
// raises a CTA-wide abort flag so the other roles leave their loops, waits for
// its own copies in flight, frees its TMEM and returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <atomic>

#include "qsa_common.cuh"

namespace qsa {
namespace {

constexpr int kTile = 128;                    // tokens per tile
constexpr int kTileBytes = kTile * kHeadDim;  // 16 KiB of FP8
constexpr int kTermsQ = 2;                    // FP8 terms per query value (bounds above)
constexpr int kTermsP = 4;                    // FP8 terms per probability
constexpr int kMeta = 4;                      // metadata ring depth (items)
constexpr int kMaxTmemBufs = 3;               // TMEM accumulator buffers (items), at most
constexpr int kDecoderWarp = 0;
constexpr int kLoaders = 6;                   // loader warps 1 .. kLoaders
constexpr int kMmaWarp = 1 + kLoaders;
constexpr int kSoftmax0 = kMmaWarp + 1;       // softmax / epilogue warps
static_assert(kSoftmax0 % 4 == 0, "softmax warps must cover the four TMEM lane quadrants in order");
constexpr int kSmemLimit = 232448;            // 227 KiB opt-in per CTA
// Limit of the drain waits for a CTA's own copies and MMAs in flight (the
// pipeline's waits take DecodeParams::wait_limit_ns, 1 s unless a test sets it).
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
  // softmax / epilogue warps: one set of four (one warp per TMEM lane
  // quadrant), or two sets where G >= 8 makes one set's per-item softmax
  // longer than the item's K/V transfer; each set takes half of the heads
  // (so two sets only for even G) over all score tiles and runs independently
  // of the other. 12 warps leave up to 168 registers a thread, 16 warps 128
  // (one CTA per SM; an SM sub-partition has 16K registers and holds a
  // quarter of the warps).
  // GP: the heads the softmax handles -- an odd G from 5 up gets one padding
  // head (zero query rows, never written out) so that two sets split it
  static constexpr int GP = (G >= 5 && G % 2 == 1) ? G + 1 : G;
  static constexpr int kSoftmaxWarps = (GP >= 6 && GP % 2 == 0) ? 8 : 4;
  static constexpr int kSoftmaxSets = kSoftmaxWarps / 4;
  static constexpr int kThreads = 32 * (kSoftmax0 + kSoftmaxWarps);
  static_assert(kThreads % 128 == 0, "whole warpgroups, so the four sub-partitions hold equal shares");
  static constexpr int NS = ((G * kTermsQ + 15) / 16) * 16;  // N of the S MMA (rows of Qs)
  static constexpr int kHalfHeads = GP / kSoftmaxSets;       // heads of one softmax set
  // Ps is token-major (the MN-major B operand of the O MMA): each token's
  // probability terms are contiguous, so a thread stores its set's terms of
  // a tile in 16-byte pieces, and each set's heads are padded to whole
  // 16-byte columns (4 heads x 4 terms)
  static constexpr int kSetN = ((kHalfHeads * kTermsP + 15) / 16) * 16;  // O columns of one set
  static constexpr int NO = kSoftmaxSets * kSetN;  // N of the O MMA (terms of a Ps tile)
  static constexpr int kTiles = 4;                          // tiles per item
  static constexpr int kChunk = kTiles * kTile;             // Top-K entries per item
  static constexpr int kBufCols = (kTiles * NS + NO + 31) / 32 * 32;  // S tiles + O, per TMEM buffer
  // three accumulator buffers where they fit the 512 TMEM columns, else two
  // (groups above 8: 128 score + up to 64 output columns per item)
  static constexpr int kTmemBufs = 3 * kBufCols <= 512 ? 3 : 2;
  static constexpr int kTmemCols = pow2_at_least(kTmemBufs * kBufCols);
  static constexpr int kQsBytes = NS * 128;
  static_assert(kTiles * NS <= 128 && NO % 16 == 0 && NO <= 64, "TMEM budget and MMA N");
  static_assert(kSoftmaxSets == 2 || kTiles * NS == 64, "a single softmax set loads its scores at once");
  static_assert(GP * kTermsQ <= NS && GP * kTermsP <= NO, "a padding head fits the S and O columns");
  static constexpr int kHeadCols = kHalfHeads * kTermsP;  // O columns of one softmax warp's heads
  // ... loaded as a supported tcgen05.ld width (the extra columns lie inside
  // the TMEM buffer and are not used)
  static constexpr int kHeadColsLd = kHeadCols <= 4 ? 4 : kHeadCols <= 8 ? 8 : kHeadCols <= 16 ? 16
                                                                          : kHeadCols <= 32 ? 32 : 64;
  // score columns of one set's heads in one tile, and the stride between
  // tiles in the warp's score registers
  static constexpr int kSetCols = kHalfHeads * kTermsQ;
  static constexpr int kRawStride = kSoftmaxSets == 1 ? NS : kSetCols <= 8 ? 8 : 16;  // 4 x 8 or 4 x 16 columns
  static_assert(kSoftmaxSets == 1 || kSetCols <= kRawStride, "two-set score loads: 4 x 8 or 4 x 16 columns");
  static constexpr int kPsBytes = kTiles * NO * 128;
  // shared memory layout (offsets from a 1024-byte aligned base); every
  // region starts on a 128-byte boundary, the MMA operands on 1024
  static constexpr int kQs = 0;                                        // [kMeta][NS][128]
  static constexpr int kPs = kQs + kMeta * kQsBytes;                   // [2][kTiles][NO][128]
  static constexpr int kRowTab = kPs + 2 * kPsBytes;                   // int32 [kMeta][kChunk] token slots
  static constexpr int kTileFlags = kRowTab + kMeta * kChunk * 4;      // uint8 [kMeta][16] (kTiles used)
  static constexpr int kQinv = kTileFlags + kMeta * 16;                // float [kMeta][G]
  static constexpr int kRedMax = align128(kQinv + kMeta * G * 4);      // float [2][kSoftmaxWarps][GP]
  static constexpr int kRedSum = align128(kRedMax + 2 * kSoftmaxWarps * GP * 4);  // float [2][kSoftmaxWarps][GP]
  static constexpr int kBars = align128(kRedSum + 2 * kSoftmaxWarps * GP * 4);
  static constexpr int kMaxSlots = 16;
  static constexpr int kNumBars = 2 * kMaxSlots + 2 * kMeta + 3 * kMaxTmemBufs + 2 + 1;
  // tmem address (+0), abort flag (+8), item ids of the metadata slots
  // (+16, kMeta ints)
  static constexpr int kMisc = kBars + kNumBars * 8;
  static constexpr int kSlotBase = ((kMisc + 48 + 1023) / 1024) * 1024;
  static constexpr int kSlots0 = (kSmemLimit - 1024 - kSlotBase) / kTileBytes;
  static constexpr int kSlots = kSlots0 > kMaxSlots ? kMaxSlots : kSlots0;
  static constexpr int kSmemAlloc = kSlotBase + kSlots * kTileBytes + 1024;
  static constexpr uint32_t kIdescS = idesc_e4m3(128, NS, false, false);
  static constexpr uint32_t kIdescO = idesc_e4m3(128, NO, true, true);
  static_assert(kSlots >= 2 * kTiles, "ring must hold a K and a V chunk");
  static_assert(kSmemAlloc <= kSmemLimit, "shared memory budget");
  static_assert(kTmemCols <= 512, "TMEM budget");
  static_assert(kQs % 1024 == 0 && kPs % 1024 == 0 && kSlotBase % 1024 == 0 && kQsBytes % 1024 == 0 &&
                    (NO * 128) % 1024 == 0,
                "MMA operands must start on 1024-byte swizzle atoms");
  static_assert(kRowTab % 128 == 0 && kTileFlags % 16 == 0 && kBars % 8 == 0 && kMisc % 8 == 0 && kMeta <= 8 &&
                    kTiles <= 16,
                "alignment of the small arrays");
};

struct Item {
  int row, g, chunk;
};

// Published item ids of split rows may carry kLastChunk: the last published
// chunk of its (row, KV head) when the CTA merges the chunks itself.
constexpr int kLastChunk = 1 << 30;
constexpr int kItemMask = kLastChunk - 1;

__device__ __forceinline__ Item item_of(const DecodeParams& p, int item) {
  item &= kItemMask;
  Item it;
  it.g = item % p.num_kv_heads;
  const int rc = item / p.num_kv_heads;
  it.chunk = rc % p.num_chunks;
  it.row = rc / p.num_chunks;
  return it;
}

// Query heads of (virtual) KV head g: they start at q_head0 and there are
// q_heads of them. Without kMap, head g's are g * G .. g * G + G - 1 (also for
// an even group above 16 split into two virtual heads of G each). With kMap
// (an odd group above 16, split into virtual heads of G and G - 1 query
// heads), the first half of cache head g >> 1 holds G of its real_group
// heads and the second half the rest plus a padding head: zero query rows,
// never stored. The kernel instances without kMap carry none of this.
template <int G, bool kMap>
__device__ __forceinline__ int q_head0(const DecodeParams& p, int g) {
  if constexpr (kMap) return (g >> 1) * p.real_group + (g & 1) * G;
  return g * G;
}
template <int G, bool kMap>
__device__ __forceinline__ int q_heads(const DecodeParams& p, int g) {
  if constexpr (kMap) return (g & 1) ? p.real_group - G : G;
  return G;
}

// The decoder's walk over the items when rows are split (num_chunks > 1).
// Items are taken in windows of w claim indices. Claim index c stands for
// (row, chunk) rc = c % (rows * num_chunks) and KV head c / (rows *
// num_chunks), so a window holds consecutive chunks of one row for one head.
// A CTA's first window is static (c from blockIdx.x * w); later ones are
// claimed from the per-call counter, from gridDim.x * w on, so a CTA that
// draws long rows (or runs slow) takes fewer: ragged rows make the work per
// window uneven. An item whose chunk holds no valid tile (past a ragged
// row's end) is left out and never published. Each window's claim is issued
// two windows and its tile flags one window before it is walked, so neither
// wait shows.
//   Partials (merge_chunks == 0): w = kWalkWindow; a left-out item's
//     partials get a log-sum of -inf, which tells the split combine that the
//     chunk is empty.
//   Merged (merge_chunks == 1): w = num_chunks, so a window is exactly the
//     chunks of one (row, KV head), published in order; the last one carries
//     kLastChunk. A window with no valid chunk (a fully masked row) gets its
//     zero output here.
constexpr int kWalkWindow = 4;
struct ItemWalk {
  int w;                // claim indices per window
  int base;             // first claim index of the current window
  uint32_t live;        // bit b: claim index base + b is still to be published
  int next_base;        // first claim index of the next window
  uint32_t next_flags;  // lane b < w: tile flags word of claim index next_base + b
  int claim;            // lane 0: first claim index of the window after next (in flight)
};

__device__ __forceinline__ int claim_rc(const DecodeParams& p, int c) { return c % (p.rows * p.num_chunks); }
__device__ __forceinline__ int claim_item(const DecodeParams& p, int c) {
  return claim_rc(p, c) * p.num_kv_heads + c / (p.rows * p.num_chunks);
}
__device__ __forceinline__ uint32_t claim_flags(const DecodeParams& p, int w, int c, int num_items, int lane) {
  return (lane < w && c < num_items)
             ? *reinterpret_cast<const uint32_t*>(p.tile_flags + (int64_t)claim_rc(p, c) * 16)
             : 0u;
}
__device__ __forceinline__ int claim_window(const DecodeParams& p, int w) {
  return (int)gridDim.x * w + atomicAdd(p.item_counter, w);
}

// Must follow griddepcontrol.wait (the flags and the counter come from the
// row-map kernel).
__device__ __forceinline__ void walk_init(ItemWalk& wk, const DecodeParams& p, int num_items, int lane) {
  wk.w = p.merge_chunks ? p.num_chunks : kWalkWindow;
  wk.base = 0;
  wk.live = 0;
  wk.next_base = (int)blockIdx.x * wk.w;
  wk.next_flags = claim_flags(p, wk.w, wk.next_base + lane, num_items, lane);
  wk.claim = lane == 0 ? claim_window(p, wk.w) : 0;
}

// The next item of the walk (with kLastChunk where it applies), -1 at its end.
template <int G, bool kMap>
__device__ __forceinline__ int walk_next(ItemWalk& wk, const DecodeParams& p, int num_items, int lane) {
  while (wk.live == 0u) {
    if (wk.next_base >= num_items) return -1;
    // the next window becomes the current one
    wk.base = wk.next_base;
    const int c = wk.base + lane;
    const bool in = lane < wk.w && c < num_items;
    const bool keep = in && wk.next_flags != 0u;
    wk.live = __ballot_sync(0xffffffffu, keep);
    if (!p.merge_chunks) {
      if (in && !keep) {
        const Item w = item_of(p, claim_item(p, c));
#pragma unroll 1
        for (int h = 0; h < q_heads<G, kMap>(p, w.g); ++h)
          p.part_lse[((int64_t)w.row * p.num_q_heads + q_head0<G, kMap>(p, w.g) + h) * p.num_chunks + w.chunk] =
              -INFINITY;
      }
    } else if (wk.live == 0u) {
      // a (row, KV head) without a valid entry: its G heads are zeros
      const Item w = item_of(p, claim_item(p, wk.base));
#pragma unroll 1
      for (int h = 0; h < q_heads<G, kMap>(p, w.g); ++h)
        *reinterpret_cast<uint2*>(p.out + ((int64_t)w.row * p.num_q_heads + q_head0<G, kMap>(p, w.g) + h) * kHeadDim +
                                  lane * 4) = make_uint2(0u, 0u);
    }
    // the window after it (claimed one window ago) and a claim for the one after that
    wk.next_base = __shfl_sync(0xffffffffu, wk.claim, 0);
    wk.next_flags = claim_flags(p, wk.w, wk.next_base + lane, num_items, lane);
    if (lane == 0 && wk.next_base < num_items) wk.claim = claim_window(p, wk.w);
  }
  const int b = __ffs(wk.live) - 1;
  wk.live &= wk.live - 1u;
  const int item = claim_item(p, wk.base + b);
  return (p.merge_chunks && wk.live == 0u) ? (item | kLastChunk) : item;
}

// Named-barrier vote of count threads: true when pred holds in any of them.
__device__ __forceinline__ bool bar_red_or(int id, int count, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred q, %2, %3, p;\n selp.u32 %0, 1, 0, q;\n}\n"
      : "=r"(r)
      : "r"((uint32_t)pred), "r"(id), "r"(count)
      : "memory");
  return r != 0u;
}

// ------------------------------------------------------------------ PTX ----
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
// `bytes` (a multiple of 16, both addresses 16-byte aligned) from global to
// shared memory through the TMA engine; completes `bytes` on `bar`.
__device__ __forceinline__ void bulk_copy_g2s(uint32_t dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}
// Four 128-byte rows (row coordinates r0..r3 of a 2-D [rows, 128] byte tensor)
// into 512 contiguous bytes of shared memory, 128-byte swizzled by address;
// a row outside the tensor reads zeros. Completes 512 bytes on `bar`.
__device__ __forceinline__ void tma_gather4(uint32_t dst, const CUtensorMap* map, uint64_t* bar, int r0, int r1,
                                            int r2, int r3) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6, %7}], [%2];\n" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(0), "r"(r0), "r"(r1), "r"(r2), "r"(r3)
      : "memory");
}
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
// Maximum over the warp's 32 lanes in one instruction (sm_100a); NaN inputs
// are ignored, as fmaxf ignores them.
__device__ __forceinline__ float warp_max(float x) {
  float r;
  asm volatile("redux.sync.max.f32 %0, %1, 0xffffffff;\n" : "=f"(r) : "f"(x));
  return r;
}
__device__ __forceinline__ void named_bar_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;\n" ::"r"(id), "r"(count) : "memory");
}

// Warp sums of four values at once (butterfly): each step across lane bits
// 4 and 3 hands half of the remaining values to the partner lane, so the
// four sums take 6 shuffles instead of 20. Returns the sum of value
// 2 * (lane bit 4) + (lane bit 3), in every lane that has those bits.
__device__ __forceinline__ float warp_sum4(const float (&v)[4], int lane) {
  const bool b4 = (lane & 16) != 0, b3 = (lane & 8) != 0;
  float s0 = b4 ? v[2] : v[0], s1 = b4 ? v[3] : v[1];
  const float g0 = b4 ? v[0] : v[2], g1 = b4 ? v[1] : v[3];
  s0 += __shfl_xor_sync(0xffffffffu, g0, 16);
  s1 += __shfl_xor_sync(0xffffffffu, g1, 16);
  float t = b3 ? s1 : s0;
  t += __shfl_xor_sync(0xffffffffu, b3 ? s0 : s1, 8);
  t += __shfl_xor_sync(0xffffffffu, t, 4);
  t += __shfl_xor_sync(0xffffffffu, t, 2);
  t += __shfl_xor_sync(0xffffffffu, t, 1);
  return t;
}

// 2^x with the MUFU approximation (a relative error of a few ulp; 2^-inf = 0)
__device__ __forceinline__ float ex2_approx(float x) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(r) : "f"(x));
  return r;
}

// Bounded wait (limit_ns of globaltimer, DecodeParams::wait_limit_ns) that
// also gives up once another role raised the abort flag.
__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                              uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  uint64_t t0;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    uint64_t t1;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t1));
    if (t1 - t0 > limit_ns) {
      *abort_flag = 1;  // the other roles leave their loops at their next wait
      return false;
    }
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

// Query pair (|x| < 256, bf16 values scaled by a power of two): two E4M3
// terms each, x = t0 + t1/16, exact for |x| >= 2^-6 (the residual x - t0 then
// has at most 4 significant bits, all within E4M3's range once scaled by 16),
// else within 2^-14.
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

// kSplit: rows are split into several chunks (num_chunks > 1). A separate
// instance keeps the unsplit loop free of the walk's code.
template <int G, bool kSplit, bool kMap>
__global__ void __launch_bounds__(Cfg<G>::kThreads, 1)
    qsa_decode_tc_kernel(const __grid_constant__ DecodeParams p, const __grid_constant__ CUtensorMap tmap_k,
                         const __grid_constant__ CUtensorMap tmap_v, int num_items) {
  using C = Cfg<G>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_s = smem_u32(smem_raw);
  const uint32_t base_s = (raw_s + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base_s - raw_s);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kBars);
  uint64_t* kv_full = bars;                        // [kSlots] loader TMA -> MMA
  uint64_t* kv_empty = bars + C::kMaxSlots;        // [kSlots] MMA commit -> loader
  uint64_t* meta_full = bars + 2 * C::kMaxSlots;   // [kMeta] decoder -> loaders, MMA, softmax
  uint64_t* meta_empty = meta_full + kMeta;        // [kMeta] loaders + MMA commit + softmax -> decoder
  uint64_t* s_full = meta_empty + kMeta;           // [kTmemBufs] MMA commit -> softmax
  uint64_t* o_full = s_full + kMaxTmemBufs;        // [kTmemBufs] MMA commit -> epilogue
  uint64_t* tmem_empty = o_full + kMaxTmemBufs;    // [kTmemBufs] epilogue (softmax threads) -> MMA
  uint64_t* p_full = tmem_empty + kMaxTmemBufs;    // [2] softmax -> MMA (Ps double buffer)
  uint64_t* mma_drain = p_full + 2;                // MMA warp's final commit (its MMAs have completed)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::kMisc + 8);
  volatile int* item_ids = reinterpret_cast<volatile int*>(smem + C::kMisc + 16);  // [kMeta]

  // unsplit rows: the items of this CTA are blockIdx.x + k * gridDim.x for
  // k < n_my (grid <= items)
  const int n_my = (num_items - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
  auto item_at = [&](int k) { return (int)blockIdx.x + k * (int)gridDim.x; };
  float* qinv = reinterpret_cast<float*>(smem + C::kQinv);
  float* red_max = reinterpret_cast<float*>(smem + C::kRedMax);
  float* red_sum = reinterpret_cast<float*>(smem + C::kRedSum);
  int32_t* rowtab = reinterpret_cast<int32_t*>(smem + C::kRowTab);
  const uint8_t* tflags = smem + C::kTileFlags;
  // bit j: tile j of the item in metadata slot m holds a valid entry
  auto tile_mask = [&](int m) -> uint32_t {
    const uint32_t w = *reinterpret_cast<const uint32_t*>(tflags + m * 16);
    uint32_t mask = 0;
#pragma unroll
    for (int j = 0; j < C::kTiles; ++j) mask |= ((w >> (8 * j)) & 0xffu) ? (1u << j) : 0u;
    return mask;
  };

  if (tid == 0) {
    for (int i = 0; i < C::kSlots; ++i) {
      mbar_init(kv_full + i, 1);  // the loader's expect_tx arrival; the gathers complete the bytes
      mbar_init(kv_empty + i, 1);
    }
    for (int m = 0; m < kMeta; ++m) {
      mbar_init(meta_full + m, 1);
      mbar_init(meta_empty + m, kLoaders + 1 + C::kSoftmaxSets);
    }
    for (int b = 0; b < C::kTmemBufs; ++b) {
      mbar_init(s_full + b, 1);
      mbar_init(o_full + b, 1);
      mbar_init(tmem_empty + b, 32 * C::kSoftmaxWarps);
    }
    for (int b = 0; b < 2; ++b) mbar_init(p_full + b, C::kSoftmaxSets);
    mbar_init(mma_drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
    tc_fence_before();
  }
  // every warp reaches the CTA barriers converged: a warp that arrives in
  // pieces would be counted more than once and release the barrier early
  __syncwarp();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool failed = false;
  constexpr bool split = kSplit;  // the decoder walks the items (ItemWalk), else they are counted

  if (warp == kDecoderWarp) {
    // =============================== decoder ================================
    auto load_q = [&](int item, uint2 (&q)[G]) {
      if ((item & kItemMask) < num_items) {
        const Item w = item_of(p, item);
        const int h0 = q_head0<G, kMap>(p, w.g), nh = q_heads<G, kMap>(p, w.g);
#pragma unroll
        for (int h = 0; h < G; ++h)
          q[h] = h < nh ? *reinterpret_cast<const uint2*>(p.q + ((int64_t)w.row * p.num_q_heads + h0 + h) * kHeadDim +
                                                          lane * 4)
                        : make_uint2(0u, 0u);  // a split odd group's padding head
      }
    };
    uint2 q_n[G];
    load_q(item_at(0), q_n);  // the first item, unless the walk starts elsewhere
    // the row map, the tile flags and the claim counter are written by the
    // preceding kernel of this programmatic dependent launch
    asm volatile("griddepcontrol.wait;\n" ::: "memory");
    ItemWalk wk;
    // the next item to publish: unsplit rows, its local index; split rows,
    // its id (-1: the end)
    int nx = 0;
    if (split) {
      walk_init(wk, p, num_items, lane);
      nx = walk_next<G, kMap>(wk, p, num_items, lane);
      if (nx >= 0 && (nx & kItemMask) != item_at(0)) load_q(nx, q_n);
    }
    int k = 0;  // published items so far
    for (;; ++k) {
      const bool last = nx < 0;
      const int item = last ? 0 : (split ? nx : item_at(nx));
      const int m = k % kMeta;
      uint2 q_c[G];
#pragma unroll
      for (int h = 0; h < G; ++h) q_c[h] = q_n[h];
      if (!last) {
        nx = split ? walk_next<G, kMap>(wk, p, num_items, lane) : (nx + 1 < n_my ? nx + 1 : -1);
        if (nx >= 0) load_q(split ? nx : item_at(nx), q_n);
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
        if constexpr (G >= 8) {  // large groups: the decoder's per-item work shows
          amax = warp_max(amax);
        } else {
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        }
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

      // metadata slot m is free once item k-kMeta is fully consumed
      const int um = k / kMeta;
      if (um > 0 &&
          !__all_sync(0xffffffffu, wait_or_abort(meta_empty + m, (uint32_t)((um - 1) & 1), abort_flag, p.wait_limit_ns))) {
        failed = true;
        break;
      }
      if (last) {
        // end of work: id -1 in slot m tells every role to finish
        if (lane == 0) {
          item_ids[m] = -1;
          mbar_arrive(meta_full + m);
        }
        break;
      }
      const Item w = item_of(p, item);
      // the item's chunk of the row map -> row table of slot m (completes on
      // meta_full together with the arrival below)
      if (lane == 0) {
        mbar_expect_tx(meta_full + m, C::kChunk * 4 + 16);
        bulk_copy_g2s(smem_u32(rowtab + m * C::kChunk),
                      p.rowmap + (int64_t)w.row * p.rowmap_stride + (int64_t)w.chunk * C::kChunk, C::kChunk * 4,
                      meta_full + m);
        bulk_copy_g2s(smem_u32(tflags + m * 16), p.tile_flags + ((int64_t)w.row * p.num_chunks + w.chunk) * 16, 16,
                      meta_full + m);
        item_ids[m] = item;
      }
      uint8_t* qs = smem + C::kQs + m * C::kQsBytes;
#pragma unroll
      for (int h = 0; h < G; ++h) {
#pragma unroll
        for (int j = 0; j < kTermsQ; ++j)
          *reinterpret_cast<uint32_t*>(qs + sw128_offset(h * kTermsQ + j, lane * 4)) = qpk[h][j];
        if (lane == h) qinv[m * G + h] = qsc[h];
      }
      for (int r = G * kTermsQ; r < C::NS; ++r)  // zero padding rows of Qs
        *reinterpret_cast<uint32_t*>(qs + r * 128 + lane * 4) = 0u;
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(meta_full + m);
    }
    // drain: the last row-map copies have landed before the warp leaves (the
    // end-of-work slot k took the slot of item k - kMeta, whose copy the
    // consumers had already waited for -- unless the wait for that slot is
    // what failed, and then item k - kMeta's copy is drained too)
    for (int kk = max(0, k - kMeta + (failed ? 0 : 1)); kk < k; ++kk)
      if (!mbar_wait_bounded(meta_full + kk % kMeta, (uint32_t)((kk / kMeta) & 1), kWaitLimitNs)) failed = true;
  } else if (warp <= kLoaders) {
    // =============================== loaders ================================
    // The ring sequence is K(0), K(1), V(0), K(2), V(1), ..., V(last): the
    // MMA warp's order. Position pos lands in slot pos % kSlots; loader L
    // fills the positions of the slots s with s % kLoaders == L, in order.
    const int L = warp - 1;
    if (lane == 0) {
      prefetch_tmap(&tmap_k);
      prefetch_tmap(&tmap_v);
    }
    int pos = 0;
    auto load_tiles = [&](int m, int g, uint32_t mask, const CUtensorMap* map) -> bool {
      const int32_t* tab = rowtab + m * C::kChunk;
      #pragma unroll 1  // one copy of the loop body: the warp roles share the instruction cache
      for (int j = 0; j < C::kTiles; ++j) {
        if (!((mask >> j) & 1u)) continue;
        const int s = pos++ % C::kSlots;
        if (s % kLoaders != L) continue;
        const int fill = (pos - 1) / C::kSlots;
        if (fill > 0 &&
            !__all_sync(0xffffffffu, wait_or_abort(kv_empty + s, (uint32_t)((fill - 1) & 1), abort_flag, p.wait_limit_ns))) {
          --pos;  // this position was not issued: the drain below counts issued fills only
          return false;
        }
        const int4 t = *reinterpret_cast<const int4*>(tab + j * kTile + lane * 4);
        // the cache's own KV heads (items count the virtual ones of a split group)
        const int hkv = p.num_kv_heads >> p.kv_shift;
        const int gk = g >> p.kv_shift;
        if (lane == 0) mbar_arrive_expect_tx(kv_full + s, kTileBytes);
        __syncwarp();
        tma_gather4(base_s + C::kSlotBase + (uint32_t)s * kTileBytes + (uint32_t)lane * 512u, map, kv_full + s,
                    t.x >= 0 ? t.x * hkv + gk : -1, t.y >= 0 ? t.y * hkv + gk : -1,
                    t.z >= 0 ? t.z * hkv + gk : -1, t.w >= 0 ? t.w * hkv + gk : -1);
      }
      return true;
    };
    uint32_t prev_mask = 0;
    int prev_g = 0;
    bool have_prev = false;
    for (int k = 0; !failed; ++k) {
      const int m = k % kMeta;
      if (!__all_sync(0xffffffffu, wait_or_abort(meta_full + m, (uint32_t)((k / kMeta) & 1), abort_flag, p.wait_limit_ns))) {
        failed = true;
        break;
      }
      const int item = item_ids[m];
      const Item w = item_of(p, item >= 0 ? item : 0);
      const uint32_t mask = item >= 0 ? tile_mask(m) : 0u;
      if (item >= 0 && !load_tiles(m, w.g, mask, &tmap_k)) {
        failed = true;
        break;
      }
      if (have_prev) {
        const int m1 = (k - 1) % kMeta;
        if (!load_tiles(m1, prev_g, prev_mask, &tmap_v)) {
          failed = true;
          break;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(meta_empty + m1);  // this warp is done with item k-1's row table
      }
      if (item < 0) break;
      prev_mask = mask;
      prev_g = w.g;
      have_prev = true;
    }
    // drain: the gathers this warp issued have all landed before it leaves
    // (immediate on the normal path, where the MMA warp consumed every fill)
    for (int s = L; s < C::kSlots; s += kLoaders) {
      const int fills = pos > s ? (pos - s + C::kSlots - 1) / C::kSlots : 0;
      if (fills > 0 && !mbar_wait_bounded(kv_full + s, (uint32_t)((fills - 1) & 1), kWaitLimitNs)) failed = true;
    }
  } else if (warp == kMmaWarp) {
    // ================================= MMA ==================================
    if (lane == 0) {
      int t = 0;  // ring position of the next tile
      uint32_t prev_mask = 0;
      bool have_prev = false;
      for (int k = 0; !failed; ++k) {
        const int m = k % kMeta;
        if (!wait_or_abort(meta_full + m, (uint32_t)((k / kMeta) & 1), abort_flag, p.wait_limit_ns)) {
          failed = true;
          break;
        }
        const int item = item_ids[m];
        const uint32_t mask = item >= 0 ? tile_mask(m) : 0u;
        if (item >= 0) {
          // S(k) = K tiles of item k . Qs^T
          const int tb = k % C::kTmemBufs;
          const int ut = k / C::kTmemBufs;
          if (ut > 0 && !wait_or_abort(tmem_empty + tb, (uint32_t)((ut - 1) & 1), abort_flag, p.wait_limit_ns)) {
            failed = true;
            break;
          }
          tc_fence_after();
          const uint32_t qs0 = base_s + C::kQs + m * C::kQsBytes;
          #pragma unroll 1  // one copy of the loop body: the warp roles share the instruction cache
          for (int j = 0; j < C::kTiles; ++j) {
            if (!((mask >> j) & 1u)) continue;
            const int slot = t % C::kSlots;
            if (!wait_or_abort(kv_full + slot, (uint32_t)((t / C::kSlots) & 1), abort_flag, p.wait_limit_ns)) {
              failed = true;
              break;
            }
            ++t;
            tc_fence_after();
            const uint32_t a0 = base_s + C::kSlotBase + (uint32_t)slot * kTileBytes;
#pragma unroll
            for (int kk = 0; kk < kHeadDim / 32; ++kk) {
              const uint64_t ad = smem_desc_sw128(a0 + kk * 32, 16, 1024);
              const uint64_t bd = smem_desc_sw128(qs0 + kk * 32, 16, 1024);
              mma_f8(tmem + tb * C::kBufCols + j * C::NS, ad, bd, C::kIdescS, kk > 0 ? 1u : 0u);
            }
            mma_commit(kv_empty + slot);
          }
          if (failed) break;
          mma_commit(s_full + tb);
          mma_commit(meta_empty + m);  // Qs of slot m is read once these MMAs finish
        }
        if (have_prev) {
          // O^T(k-1) += V tiles of item k-1 ^T . Ps^T
          const int jt = k - 1;
          const int pb = jt & 1;
          const int tb = jt % C::kTmemBufs;
          if (!wait_or_abort(p_full + pb, (uint32_t)((jt >> 1) & 1), abort_flag, p.wait_limit_ns)) {
            failed = true;
            break;
          }
          tc_fence_after();
          const uint32_t d = tmem + tb * C::kBufCols + C::kTiles * C::NS;
          bool first = true;  // the first multiplied tile overwrites the accumulator
          #pragma unroll 1  // one copy of the loop body: the warp roles share the instruction cache
          for (int j = 0; j < C::kTiles; ++j) {
            if (!((prev_mask >> j) & 1u)) continue;
            const int slot = t % C::kSlots;
            if (!wait_or_abort(kv_full + slot, (uint32_t)((t / C::kSlots) & 1), abort_flag, p.wait_limit_ns)) {
              failed = true;
              break;
            }
            ++t;
            tc_fence_after();
            const uint32_t a0 = base_s + C::kSlotBase + (uint32_t)slot * kTileBytes;
            const uint32_t b0 = base_s + C::kPs + pb * C::kPsBytes + j * C::NO * 128;
#pragma unroll
            for (int kk = 0; kk < kTile / 32; ++kk) {
              const uint64_t ad = smem_desc_sw128(a0 + kk * 32 * 128, kTileBytes, 1024);
              // Ps: 16-byte columns of 128 tokens, 2048 bytes apart (K step:
              // 32 tokens of 16 bytes)
              const uint64_t bd = smem_desc_mn_interleave(b0 + kk * 32 * 16, 128, 2048);
              mma_f8(d, ad, bd, C::kIdescO, (!first || kk > 0) ? 1u : 0u);
            }
            first = false;
            mma_commit(kv_empty + slot);
          }
          if (failed) break;
          mma_commit(o_full + tb);
        }
        if (item < 0) break;
        prev_mask = mask;
        have_prev = true;
      }
    }
    // drain: every MMA this thread issued has completed (and made its commit
    // arrivals) before TMEM is freed and the CTA exits -- immediate on the
    // normal path, where the epilogue waited for the last one
    if (lane == 0) {
      mma_commit(mma_drain);
      if (!mbar_wait_bounded(mma_drain, 0u, kWaitLimitNs)) failed = true;
    }
    // the other 31 lanes wait here for lane 0, so that the whole warp reaches
    // the CTA barrier below together (a barrier met by a diverged warp would
    // let the CTA pass it before lane 0 is done)
    __syncwarp();
  } else {
    // ======================== softmax + epilogue ==========================
    // Software pipelined: the softmax of item k runs before the epilogue of
    // item k-1, whose O accumulation has finished meanwhile. With two sets of
    // softmax warps, warps sw and sw + 4 share a TMEM lane quadrant and `half`
    // picks their heads (it only offsets addresses: every register array is
    // indexed by compile-time constants); each set reduces over its own four
    // warps with its own named barrier.
    const int q4 = warp & 3;                // TMEM lane quadrant of this warp
    const int sw = warp - kSoftmax0;        // 0 .. C::kSoftmaxWarps-1
    const int half = C::kSoftmaxSets > 1 ? (sw >> 2) : 0;  // softmax set
    const int tk = q4 * 32 + lane;          // token within a tile / head dim in the epilogue
    const uint32_t lane_base = (uint32_t)(q4 * 32) << 16;
    const int h0 = half * C::kHalfHeads;    // first head of this warp's set
    const int set_bar = 1 + half;           // named barrier of the set
    const int vote_bar = 3 + half;          // named barrier of the set's votes (split rows)
    // state of the item whose epilogue is pending
    int e_k = -1, e_row = 0, e_g = 0, e_chunk = 0;
    bool e_any = false;  // the pending item has a valid tile
    bool e_last = false;  // merged split rows: the pending item ends its (row, KV head)
    float e_m[C::kHalfHeads], e_l[C::kHalfHeads];
    __nv_bfloat16 e_gate[C::kHalfHeads];
    // merged split rows: the running merge of the current (row, KV head)'s
    // chunks, per head (unnormalised output of dim tk, its log2 maximum and
    // sum), the flash-decoding combine done in registers
    float mg_u[C::kHalfHeads], mg_m[C::kHalfHeads], mg_l[C::kHalfHeads];
#pragma unroll
    for (int hh = 0; hh < C::kHalfHeads; ++hh) {
      mg_u[hh] = 0.f;
      mg_m[hh] = -INFINITY;
      mg_l[hh] = 0.f;
    }
    auto epilogue = [&]() {
      const int tb = e_k % C::kTmemBufs;
      if (!failed)
        failed = !__all_sync(0xffffffffu, wait_or_abort(o_full + tb, (uint32_t)((e_k / C::kTmemBufs) & 1), abort_flag, p.wait_limit_ns));
      if (failed) return;
      tc_fence_after();
      // the O columns of this warp's heads (their kTermsP terms each)
      float v[C::kHeadColsLd];
      tmem_ld_wait<C::kHeadColsLd>(tmem + lane_base + tb * C::kBufCols + C::kTiles * C::NS + half * C::kSetN, v);
      tc_fence_before();
      mbar_arrive(tmem_empty + tb);
#pragma unroll
      for (int hh = 0; hh < C::kHalfHeads; ++hh) {
        const int h = h0 + hh;
        // branch-free division and exponential (the intrinsics), so the
        // heads' chains interleave; their few-ulp fp32 error is far below the
        // bf16 rounding of the result
        const float o = (e_any && e_l[hh] > 0.f)
                            ? __fdividef(combine_p(v + hh * kTermsP) * (1.0f / 256.0f), e_l[hh])
                            : 0.f;
        if (h >= q_heads<G, kMap>(p, e_g)) continue;  // a padding head (odd group, or a split odd group's half)
        const int64_t hrow = (int64_t)e_row * p.num_q_heads + q_head0<G, kMap>(p, e_g) + h;
        if (p.num_chunks == 1) {
          const float gt = __bfloat162float(e_gate[hh]);
          // exp(80) keeps 1 + e below 2^126, where the fast division is exact enough
          const float sig = __fdividef(1.0f, 1.0f + __expf(fminf(-gt, 80.0f)));
          p.out[hrow * kHeadDim + tk] = __float2bfloat16_rn(o * p.v_scale * sig);
        } else {
          if constexpr (split && G <= 8) {  // (tc_merges_chunks holds only for G <= 8)
            if (p.merge_chunks) {
              if (e_any && e_l[hh] > 0.f) {
                const float u = combine_p(v + hh * kTermsP) * (1.0f / 256.0f);
                const float mn = fmaxf(mg_m[hh], e_m[hh]);
                const float a = ex2_approx(mg_m[hh] - mn), b = ex2_approx(e_m[hh] - mn);
                mg_u[hh] = mg_u[hh] * a + u * b;
                mg_l[hh] = mg_l[hh] * a + e_l[hh] * b;
                mg_m[hh] = mn;
              }
              if (e_last) {  // the (row, KV head)'s last chunk: normalise, gate, store
                const float gt = __bfloat162float(e_gate[hh]);
                const float sig = __fdividef(1.0f, 1.0f + __expf(fminf(-gt, 80.0f)));
                const float om = mg_l[hh] > 0.f ? __fdividef(mg_u[hh], mg_l[hh]) : 0.f;
                p.out[hrow * kHeadDim + tk] = __float2bfloat16_rn(om * p.v_scale * sig);
                mg_u[hh] = 0.f;
                mg_m[hh] = -INFINITY;
                mg_l[hh] = 0.f;
              }
              continue;
            }
          }
          const int64_t pidx = hrow * p.num_chunks + e_chunk;
          p.part_o[pidx * kHeadDim + tk] = o;
          if (tk == 0) p.part_lse[pidx] = e_l[hh] > 0.f ? e_m[hh] + log2f(e_l[hh]) : -INFINITY;
        }
      }
    };
    for (int k = 0;; ++k) {
      // unsplit rows: the local index of item k; split rows: the walk's
      // item, which comes with the metadata slot (meta_full publishes its
      // id). There the set's warps leave together, after the last item or
      // once any of them failed (its id could be stale), so that their named
      // barriers match.
      int li;
      if constexpr (split) {
        const int m = k % kMeta;
        if (!failed)
          failed = !__all_sync(0xffffffffu, wait_or_abort(meta_full + m, (uint32_t)((k / kMeta) & 1), abort_flag, p.wait_limit_ns));
        if (bar_red_or(vote_bar, 128, failed)) {
          failed = true;
          break;
        }
        li = item_ids[m];
      } else {
        li = k < n_my ? k : -1;
      }
      if (li < 0) break;
      const int tb = k % C::kTmemBufs;
      const int pb = k & 1;
      const int m = k % kMeta;
      const Item w = item_of(p, split ? li : item_at(li));
      // the gate of this warp's heads, needed by the epilogue one iteration later
      __nv_bfloat16 gate[C::kHalfHeads];
      if (split ? p.merge_chunks != 0 : p.num_chunks == 1) {
#pragma unroll
        for (int hh = 0; hh < C::kHalfHeads; ++hh)
          gate[hh] = h0 + hh < q_heads<G, kMap>(p, w.g)
                         ? p.gate[((int64_t)w.row * p.num_q_heads + q_head0<G, kMap>(p, w.g) + h0 + hh) * kHeadDim + tk]
                         : __float2bfloat16_rn(0.f);
      }
      // meta_full publishes the row table and query scales; s_full the
      // scores. Once anything failed the group keeps walking its items (the
      // named barriers must still match) but skips tensor memory.
      if (!failed) {
        const bool ok = (split || wait_or_abort(meta_full + m, (uint32_t)((k / kMeta) & 1), abort_flag, p.wait_limit_ns)) &&
                        wait_or_abort(s_full + tb, (uint32_t)((k / C::kTmemBufs) & 1), abort_flag, p.wait_limit_ns);
        failed = !__all_sync(0xffffffffu, ok);
      }
      tc_fence_after();
      const uint32_t mask = tile_mask(m);
      constexpr int kSH = C::kHalfHeads;
      float qi[kSH];
#pragma unroll
      for (int hh = 0; hh < kSH; ++hh) qi[hh] = h0 + hh < G ? qinv[m * G + h0 + hh] : 0.f;
      // this set's score columns of every tile: (tile j, head hh, term t) at
      // raw[j * kRawStride + hh * kTermsQ + t] -- all tiles in one load, or
      // (16 columns a tile, groups above 8) one tile at a time for registers
      const uint32_t s0 = tmem + lane_base + tb * C::kBufCols + h0 * kTermsQ;
      float sc[C::kTiles][kSH];
      if constexpr (C::kSoftmaxSets == 2 && C::kRawStride == 16) {
#pragma unroll
        for (int j = 0; j < C::kTiles; ++j) {
          float raw[16];
          if (!failed) tmem_ld_wait<16>(s0 + j * C::NS, raw);
          const bool ok = !failed && ((mask >> j) & 1u) && rowtab[m * C::kChunk + j * kTile + tk] >= 0;
#pragma unroll
          for (int hh = 0; hh < kSH; ++hh)
            sc[j][hh] = ok ? combine_q(&raw[hh * kTermsQ]) * qi[hh] : -INFINITY;
        }
      } else {
        float raw[C::kTiles * C::kRawStride];
        if (!failed) {
          if constexpr (C::kSoftmaxSets == 1)
            tmem_ld_wait<C::kTiles * C::NS>(s0, raw);
          else
            tmem_ld_4x8_wait(s0, C::NS, raw);
        }
#pragma unroll
        for (int j = 0; j < C::kTiles; ++j) {
          const bool ok = !failed && ((mask >> j) & 1u) && rowtab[m * C::kChunk + j * kTile + tk] >= 0;
#pragma unroll
          for (int hh = 0; hh < kSH; ++hh)
            sc[j][hh] = ok ? combine_q(&raw[j * C::kRawStride + hh * kTermsQ]) * qi[hh] : -INFINITY;
        }
      }
      // exact max per head over the chunk (one partial maximum per warp of the set)
      float* rmax = red_max + (pb * C::kSoftmaxWarps + half * 4) * C::GP + h0;
      float* rsum = red_sum + (pb * C::kSoftmaxWarps + half * 4) * C::GP + h0;
#pragma unroll
      for (int hh = 0; hh < kSH; ++hh) {
        float mx = sc[0][hh];
#pragma unroll
        for (int j = 1; j < C::kTiles; ++j) mx = fmaxf(mx, sc[j][hh]);
        // one redux for the large groups, whose softmax bounds the kernel; the
        // shuffle tree has the shorter latency that the small groups' pipeline
        // (softmax -> P -> O MMA -> ring slot) prefers
        if constexpr (G >= 8) {
          mx = warp_max(mx);
        } else {
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        }
        if (lane == 0) rmax[q4 * C::GP + hh] = mx;
      }
      named_bar_sync(set_bar, 128);
      if (q4 == 0 && lane == 0 && !failed) mbar_arrive(meta_empty + m);  // row table and scales read
      // probabilities by the MUFU 2^x; for four heads a set the sums go through
      // one butterfly (lanes 0, 8, 16, 24 end with heads 0..3), other counts
      // reduce head by head
      float psum[4];
#pragma unroll
      for (int hh = 0; hh < kSH; ++hh) {
        float mx = rmax[hh];
#pragma unroll
        for (int i = 1; i < 4; ++i) mx = fmaxf(mx, rmax[i * C::GP + hh]);
        // a head with no valid entry (mx = -inf) keeps p = 2^-inf = 0
        if (mx == -INFINITY) mx = 0.f;
        float sum = 0.f;
#pragma unroll
        for (int j = 0; j < C::kTiles; ++j) {
          const float pr = ex2_approx(sc[j][hh] - mx);
          sc[j][hh] = pr;
          sum += pr;
        }
        if constexpr (kSH == 4) {
          psum[hh] = sum;
        } else {
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
          if (lane == 0) rsum[q4 * C::GP + hh] = sum;
        }
      }
      if constexpr (kSH == 4) {
        const float sum = warp_sum4(psum, lane);
        if ((lane & 7) == 0) rsum[q4 * C::GP + (lane >> 3)] = sum;
      }
      // probabilities -> FP8 terms of p*256 (row h*kTermsP+t of Ps, one byte per
      // token), two heads per conversion
      uint8_t* ps = smem + C::kPs + pb * C::kPsBytes;
      // the set's 16-byte columns of this token: column c holds heads 4c..4c+3
      // of the set, 4 terms each (heads past the set's are zero)
#pragma unroll
      for (int j = 0; j < C::kTiles; ++j) {
        if ((mask >> j) & 1u) {
          uint8_t* pt = ps + j * C::NO * 128 + half * (C::kSetN / 16) * 2048 + tk * 16;
#pragma unroll
          for (int c = 0; c < C::kSetN / 16; ++c) {
            uint32_t w[4];
#pragma unroll
            for (int q = 0; q < 4; q += 2) {
              const int hh = 4 * c + q;
              if (hh < kSH) {
                uint16_t tt[kTermsP];
                split_p2(sc[j][hh] * 256.0f, hh + 1 < kSH ? sc[j][hh + 1] * 256.0f : 0.f, tt);
                const uint32_t a = (uint32_t)tt[0] | ((uint32_t)tt[1] << 16);
                const uint32_t b = (uint32_t)tt[2] | ((uint32_t)tt[3] << 16);
                w[q] = __byte_perm(a, b, 0x6420);      // head hh: terms 0..3
                w[q + 1] = __byte_perm(a, b, 0x7531);  // head hh + 1
              } else {
                w[q] = w[q + 1] = 0u;
              }
            }
            *reinterpret_cast<uint4*>(pt + c * 2048) = make_uint4(w[0], w[1], w[2], w[3]);
          }
        }
      }
      fence_proxy_async_smem();
      named_bar_sync(set_bar, 128);
      if (q4 == 0 && lane == 0 && !failed) mbar_arrive(p_full + pb);

      // ---- epilogue of the previous item, then this item becomes pending ---
      if (e_k >= 0) epilogue();
      e_k = k;
      e_row = w.row;
      e_g = w.g;
      e_chunk = w.chunk;
      if constexpr (split) e_last = (li & kLastChunk) != 0;
      e_any = mask != 0;
#pragma unroll
      for (int hh = 0; hh < C::kHalfHeads; ++hh) {
        // this warp's heads, read back from the group's partials (a head index
        // that is not a compile-time constant must not index a register array)
        const float* rs = red_sum + (pb * C::kSoftmaxWarps + half * 4) * C::GP + h0 + hh;
        const float* rm = red_max + (pb * C::kSoftmaxWarps + half * 4) * C::GP + h0 + hh;
        float l = 0.f, mx = rm[0];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          l += rs[i * C::GP];
          mx = fmaxf(mx, rm[i * C::GP]);
        }
        e_m[hh] = mx;
        e_l[hh] = l;
        e_gate[hh] = (split ? p.merge_chunks != 0 : p.num_chunks == 1) ? gate[hh] : __float2bfloat16_rn(0.f);
      }
    }
    if (e_k >= 0) epilogue();
  }

  if (failed) {
    *abort_flag = 1;
    report_error(p, kErrTimeout);
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}

// Row map: the token slot (phys * P + t % P) of every Top-K entry, -1 when
// masked (the rule of token_slot). Each thread handles kBatch quads of four
// entries, spaced a grid apart, with all their index loads and then all
// their block-table loads in flight together.
constexpr int kRowmapBatch = 1;
constexpr int kRowmapThreads = 256;

__global__ void __launch_bounds__(kRowmapThreads) qsa_rowmap_kernel(const __grid_constant__ DecodeParams p) {
  // let the decode kernel launch now; it waits for this grid before reading
  // the map
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
  if (blockIdx.x == 0 && threadIdx.x == 0) *p.item_counter = 0;  // the decode's claims start here
  const int quads = p.rowmap_stride / 4;
  const int64_t total = (int64_t)p.rows * quads;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t q0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  int t[kRowmapBatch][4], lim[kRowmapBatch], col0[kRowmapBatch], row[kRowmapBatch];
  int64_t req[kRowmapBatch];
#pragma unroll
  for (int b = 0; b < kRowmapBatch; ++b) {
    const int64_t q = q0 + b * stride;
    row[b] = -1;
    if (q < total) {
      row[b] = (int)(q / quads);
      col0[b] = (int)(q - (int64_t)row[b] * quads) * 4;
      req[b] = row_request(p, row[b]);
      lim[b] = row_count(p, row[b]);
      const int32_t* ip = p.indices + (int64_t)row[b] * p.indices_stride;
#pragma unroll
      for (int e = 0; e < 4; ++e) t[b][e] = col0[b] + e < p.topk ? __ldg(ip + col0[b] + e) : -1;
    }
  }
  int64_t ph[kRowmapBatch][4];
  int po[kRowmapBatch][4];
#pragma unroll
  for (int b = 0; b < kRowmapBatch; ++b)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      int lp = 0;
      po[b][e] = 0;
      const bool ok = row[b] >= 0 && req[b] >= 0 && col0[b] + e < lim[b] && token_page(p, t[b][e], lp, po[b][e]);
      ph[b][e] = ok ? (int64_t)__ldg(p.btable + req[b] * p.btable_stride + lp) : -1;
    }
#pragma unroll
  for (int b = 0; b < kRowmapBatch; ++b)
    if (row[b] >= 0)
      *reinterpret_cast<int4*>(p.rowmap + (int64_t)row[b] * p.rowmap_stride + col0[b]) =
          make_int4((int)token_slot_from(p, ph[b][0], po[b][0]), (int)token_slot_from(p, ph[b][1], po[b][1]),
                    (int)token_slot_from(p, ph[b][2], po[b][2]), (int)token_slot_from(p, ph[b][3], po[b][3]));
  // tile flags: the 32 quads of a warp are one 128-entry tile of one row
  // (rows are whole tiles long), so the warp votes whether the tile holds a
  // valid entry
  bool any_valid = false;
#pragma unroll
  for (int b = 0; b < kRowmapBatch; ++b)
#pragma unroll
    for (int e = 0; e < 4; ++e) any_valid |= row[b] >= 0 && token_slot_from(p, ph[b][e], po[b][e]) >= 0;
  any_valid = __any_sync(0xffffffffu, any_valid);
  if ((threadIdx.x & 31) == 0 && row[0] >= 0) {
    const int tile = col0[0] / 128;
    const int tiles_per_chunk = p.chunk_tokens / 128;
    p.tile_flags[((int64_t)row[0] * p.num_chunks + tile / tiles_per_chunk) * 16 + tile % tiles_per_chunk] =
        any_valid ? 1 : 0;
  }
  // the decode kernel reads the map through TMA (the async proxy)
  fence_proxy_async_global();
}

// ------------------------------------------------------------------ host ----
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static std::atomic<void*> fn{nullptr};
  void* f = fn.load(std::memory_order_acquire);
  if (!f) {
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    fn.store(f, std::memory_order_release);
  }
  return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
}

// A cache viewed as a 2-D byte tensor [num_pages * P * Hkv rows, 128]; one box
// is one 128-byte row (gather4 moves four of them), 128-byte swizzled.
bool encode_rows(CUtensorMap* map, const void* base, int64_t rows) {
  auto fn = encode_fn();
  if (!fn || rows <= 0 || rows > 0x7fffffffll) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)kHeadDim, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)kHeadDim};
  const cuuint32_t box[2] = {(cuuint32_t)kHeadDim, 1u};
  const cuuint32_t estr[2] = {1u, 1u};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

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

template <int G, bool kMap = false>
cudaError_t launch_g(const DecodeParams& p, cudaStream_t stream) {
  using C = Cfg<G>;
  static std::atomic<uint64_t> configured{0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t bit = 1ull << (dev & 63);
  if (!(configured.load(std::memory_order_acquire) & bit)) {
    e = cudaFuncSetAttribute(qsa_decode_tc_kernel<G, false, kMap>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             C::kSmemAlloc);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(qsa_decode_tc_kernel<G, true, kMap>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             C::kSmemAlloc);
    if (e != cudaSuccess) return e;
    // the row-map kernel asks for the decode's shared-memory carveout, so
    // that the decode CTAs (its programmatic dependents) start, and run their
    // prologue, on SMs that still hold row-map blocks instead of waiting for
    // those to leave
    e = cudaFuncSetAttribute(qsa_rowmap_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                             cudaSharedmemCarveoutMaxShared);
    if (e != cudaSuccess) return e;
    configured.fetch_or(bit, std::memory_order_acq_rel);
  }
  const int64_t items = (int64_t)p.rows * p.num_kv_heads * p.num_chunks;
  if (items <= 0) return cudaSuccess;
  if (items > 0x7fffffffll) return cudaErrorInvalidValue;
  const int64_t rows = p.num_pages * p.page_size * (p.num_kv_heads >> p.kv_shift);  // of the caches
  if (rows > 0x7fffffffll) return cudaErrorInvalidValue;
  if (!p.rowmap || !p.tile_flags || !p.item_counter || p.rowmap_stride != p.num_chunks * C::kChunk)
    return cudaErrorInvalidValue;
  CUtensorMap mk, mv;
  if (!encode_rows(&mk, p.k, rows) || !encode_rows(&mv, p.v, rows)) return cudaErrorInvalidValue;
  const int grid = (int)(items < sm_count() ? items : sm_count());

  // the row map, then the decode as its programmatic dependent
  const int64_t quads = (int64_t)p.rows * (p.rowmap_stride / 4);
  const int64_t per_block = (int64_t)kRowmapThreads * kRowmapBatch;
  qsa_rowmap_kernel<<<(unsigned)((quads + per_block - 1) / per_block), kRowmapThreads, 0, stream>>>(p);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3((unsigned)C::kThreads);
  cfg.dynamicSmemBytes = (size_t)C::kSmemAlloc;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return p.num_chunks > 1 ? cudaLaunchKernelEx(&cfg, qsa_decode_tc_kernel<G, true, kMap>, p, mk, mv, (int)items)
                          : cudaLaunchKernelEx(&cfg, qsa_decode_tc_kernel<G, false, kMap>, p, mk, mv, (int)items);
}

}  // namespace

int tc_chunk_tokens(int) { return 4 * kTile; }

bool tc_supports_group(int group) {
  return group >= 1 && group <= 2 * kMaxGroupTc;
}

// Split rows merge in the CTA when there are enough (row, KV head) pairs to
// share out (at least two per SM), the chunks fit a warp's ballot, and the
// group leaves the softmax warps room for the merge registers; otherwise the
// chunks go out as partials to the combine kernel, which also spreads a few
// long rows over all SMs.
bool tc_merges_chunks(const DecodeParams& p) {
  return p.num_chunks > 1 && p.num_chunks <= 32 && p.group <= 8 &&
         (int64_t)p.rows * p.num_kv_heads >= 2 * (int64_t)sm_count() &&
         (int64_t)p.rows * p.num_kv_heads * p.num_chunks < kLastChunk;
}

cudaError_t launch_decode_tc(const DecodeParams& params, cudaStream_t stream) {
  DecodeParams p = params;
  p.kv_shift = 0;
  p.real_group = p.group;
  if (p.group > kMaxGroupTc) {
    // a group of 17 .. 32 query heads runs as two virtual KV heads, the
    // first with ceil(G / 2) of the query heads and the second with the
    // rest (for an odd G one less, plus a padding head): virtual head gv
    // reads cache head gv >> 1, and q_head0 / q_heads map it to its query
    // heads; the two items of a KV head run on neighbouring CTAs
    if (p.group > 2 * kMaxGroupTc) return cudaErrorInvalidValue;
    p.group = (p.group + 1) / 2;
    p.num_kv_heads *= 2;
    p.kv_shift = 1;
  }
  p.merge_chunks = tc_merges_chunks(p) ? 1 : 0;
  if (p.kv_shift && p.real_group % 2 != 0) {  // an odd group above 16: the explicit head map
    switch (p.group) {
      case 9: return launch_g<9, true>(p, stream);
      case 10: return launch_g<10, true>(p, stream);
      case 11: return launch_g<11, true>(p, stream);
      case 12: return launch_g<12, true>(p, stream);
      case 13: return launch_g<13, true>(p, stream);
      case 14: return launch_g<14, true>(p, stream);
      case 15: return launch_g<15, true>(p, stream);
      case 16: return launch_g<16, true>(p, stream);
      default: return cudaErrorInvalidValue;
    }
  }
  switch (p.group) {
    case 1: return launch_g<1>(p, stream);
    case 2: return launch_g<2>(p, stream);
    case 3: return launch_g<3>(p, stream);
    case 4: return launch_g<4>(p, stream);
    case 5: return launch_g<5>(p, stream);
    case 6: return launch_g<6>(p, stream);
    case 7: return launch_g<7>(p, stream);
    case 8: return launch_g<8>(p, stream);
    case 9: return launch_g<9>(p, stream);
    case 10: return launch_g<10>(p, stream);
    case 11: return launch_g<11>(p, stream);
    case 12: return launch_g<12>(p, stream);
    case 13: return launch_g<13>(p, stream);
    case 14: return launch_g<14>(p, stream);
    case 15: return launch_g<15>(p, stream);
    case 16: return launch_g<16>(p, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace qsa
