// Internal launch parameters shared by the C-ABI layer and the kernels.
// Not part of the public interface (that is include/qsa_b200.h).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

namespace qsa {

struct DecodeParams {
  // Tensors (device pointers). Q, gate and out are contiguous [rows, Hq, 128]
  // bf16; the caches are contiguous [num_pages, P, Hkv, 128] FP8 E4M3FN.
  const __nv_bfloat16* q;
  const __nv_bfloat16* gate;
  __nv_bfloat16* out;
  const uint8_t* k;
  const uint8_t* v;
  const int32_t* indices;  // [rows, indices_stride]; the first topk columns are the Top-K list
  const int32_t* counts;   // optional [rows]
  const int32_t* btable;   // [num_reqs, btable_stride]; the first pages_per_req columns are used
  const int32_t* t2r;      // optional [rows]

  float score_scale_log2;  // softmax_scale * k_scale * log2(e)
  float v_scale;

  int rows;
  int num_q_heads;
  int num_kv_heads;
  int group;  // num_q_heads / num_kv_heads
  int page_size;
  int page_shift;  // log2(page_size) when it is a power of two, else -1
  int pages_per_req;
  int num_reqs;
  int64_t num_pages;
  int topk;
  int64_t indices_stride;
  int count_column;  // count read from indices[row * stride + topk]
  int64_t btable_stride;

  // Split of each Top-K row into chunks of `chunk_tokens` (flash-decoding).
  // With num_chunks == 1 the kernel writes `out` directly; otherwise it writes
  // per-chunk partial results that qsa_combine merges.
  int chunk_tokens;
  int num_chunks;
  float* part_o;    // [rows, Hq, num_chunks, 128] normalised partial outputs
  float* part_lse;  // [rows, Hq, num_chunks] log2-sum-exp2 of each chunk (-inf if empty)

  // Row map of the tensor-core kernel (workspace, filled by its row-map
  // kernel): for every Top-K entry of every row, the physical token slot
  // phys * P + t % P, or -1 when masked; row r's entries start at
  // rowmap + r * rowmap_stride (num_chunks * chunk_tokens entries, the tail
  // past topk -1).
  int32_t* rowmap;
  int rowmap_stride;
  // Tile flags (workspace, filled with the row map): one byte per 128-entry
  // tile of each (row, chunk), nonzero when the tile holds a valid entry;
  // 16 bytes per (row, chunk).
  uint8_t* tile_flags;
  // Claim counter of the tensor-core kernel (workspace, zeroed by its row-map
  // kernel): with split rows, CTAs claim windows of items from it.
  int* item_counter;
  // Tensor-core kernel, split rows: 1 when each CTA walks all chunks of a
  // (row, KV head) in turn and merges them itself (no partials, no combine
  // kernel); set by the launcher from tc_merges_chunks.
  int merge_chunks;
  // Tensor-core kernel: log2 of the virtual KV heads per cache KV head (1
  // when a group above 16 runs as two halves), and the caches' own group
  // size Hq / Hkv; set by the launcher.
  int kv_shift;
  int real_group;

  int* err;  // device error word of the current device
  // Limit of each pipeline wait of the tensor-core kernel, in ns of
  // globaltimer: 1 s, unless the test hook qsa_b200_testing_set_wait_limit_ns
  // shortened it. A CTA whose wait runs out sets err and returns.
  uint64_t wait_limit_ns;
};

// Wait limit the launches of this process use (the test hook's value, else
// the 1 s default).
uint64_t wait_limit_ns();

// Kernel launchers (return cudaGetLastError() of the launch).
cudaError_t launch_decode_tc(const DecodeParams& p, cudaStream_t stream);
cudaError_t launch_decode_simt(const DecodeParams& p, cudaStream_t stream);
cudaError_t launch_combine(const DecodeParams& p, cudaStream_t stream);
cudaError_t launch_slots(const DecodeParams& p, int64_t* slots, cudaStream_t stream);
// Paged FP8 cache writer (qsa_cache_write.cu).
struct CacheWriteParams {
  const void* k;  // [tokens, Hkv, 128] new keys, rows token_stride elements apart
  const void* v;
  const int64_t* slots;  // [tokens] physical token slots; outside [0, num_pages * P) = skipped
  uint8_t* k_cache;      // [num_pages, P, Hkv, 128] e4m3fn
  uint8_t* v_cache;
  float k_inv_scale, v_inv_scale;  // 1 / scale, rounded to fp32
  int tokens;
  int num_kv_heads;
  int page_size;
  int64_t num_pages;
  int64_t token_stride;
  int dtype;  // QSA_B200_DTYPE_*
};
cudaError_t launch_cache_write(const CacheWriteParams& p, cudaStream_t stream);

// Top-K index producer (qsa_topk.cu).
struct TopkParams {
  const float* scores;
  const int32_t* lengths;  // may be null
  int32_t* out;
  int rows, ctx, k;
  int64_t score_stride, out_stride;
};
cudaError_t launch_topk(const TopkParams& p, cudaStream_t stream);

// Top-K entries per work item for a GQA group size (both kernels split rows
// the same way, so the workspace size depends only on the shape), and the
// group sizes of the tensor-core kernel.
int tc_chunk_tokens(int group);
bool tc_supports_group(int group);
// Whether the tensor-core decode merges the chunks of split rows itself, so
// that the split combine is not launched.
bool tc_merges_chunks(const DecodeParams& p);

// Largest group size (Hq / Hkv) the tensor-core kernel handles.
constexpr int kMaxGroupTc = 16;

}  // namespace qsa
