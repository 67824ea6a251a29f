// C ABI of libqsa_b200.so (declared in include/qsa_b200.h).
//
// Validates arguments, turns them into qsa::DecodeParams and launches the
// decode (the tensor-core kernel for group sizes 1-8, 10, 12, 14, 16, otherwise the
// CUDA-core kernel), plus the split combine when a Top-K row is longer than
// one chunk. Workspace layout (each part 256-byte aligned): the row map and
// the tile flags (tensor-core kernel only), the partial outputs and the
// partial log-sum-exps (split rows only). No entry
// point allocates, synchronises or traps.
#include <cuda_runtime.h>

#include <atomic>
#include <cmath>
#include <cstdint>

#include "../../include/qsa_b200.h"
#include "../../include/qsa_b200_testing.h"
#include "qsa_internal.h"

namespace qsa {

// Device error word (one per device that loads the library).
__device__ int g_device_error = 0;

constexpr uint64_t kDefaultWaitLimitNs = 1000000000ull;
std::atomic<uint64_t> g_wait_limit_ns{kDefaultWaitLimitNs};

uint64_t wait_limit_ns() { return g_wait_limit_ns.load(std::memory_order_relaxed); }

namespace {

thread_local int t_last_status = QSA_B200_OK;

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
bool aligned4(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 3u) == 0; }

// Is the current device an sm_100 part? Cached per device ordinal.
int check_device() {
  static std::atomic<uint64_t> ok_mask{0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return QSA_B200_ERR_DEVICE;
  const uint64_t bit = 1ull << (dev & 63);
  if (ok_mask.load(std::memory_order_acquire) & bit) return QSA_B200_OK;
  int major = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess)
    return QSA_B200_ERR_DEVICE;
  if (major != 10) return QSA_B200_ERR_DEVICE;
  ok_mask.fetch_or(bit, std::memory_order_acq_rel);
  return QSA_B200_OK;
}

// Device address of g_device_error on the current device (cached per device).
int* device_error_word() {
  static std::atomic<int*> addr[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
  int* a = addr[dev & 63].load(std::memory_order_acquire);
  if (!a) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_device_error) != cudaSuccess) return nullptr;
    a = static_cast<int*>(ptr);
    addr[dev & 63].store(a, std::memory_order_release);
  }
  return a;
}

int num_chunks_for(int topk, int group) {
  const int c = tc_chunk_tokens(group);
  return topk <= c ? 1 : (topk + c - 1) / c;
}

// Validation of the index / table part of the arguments (shared by slots).
int check_index_args(const qsa_b200_decode_args* a) {
  if (!a) return QSA_B200_ERR_NULL_POINTER;
  if (a->rows < 0 || a->topk < 0 || a->page_size < 1 || a->pages_per_req < 1 || a->num_reqs < 1 ||
      a->num_pages < 1)
    return QSA_B200_ERR_BAD_SHAPE;
  if (a->rows == 0) return QSA_B200_OK;
  if (!a->indices || !a->btable) return QSA_B200_ERR_NULL_POINTER;
  if (a->indices_stride < (int64_t)a->topk + (a->count_column ? 1 : 0)) return QSA_B200_ERR_BAD_SHAPE;
  if (a->btable_stride < a->pages_per_req) return QSA_B200_ERR_BAD_SHAPE;
  if (!aligned4(a->indices) || !aligned4(a->btable) || (a->t2r && !aligned4(a->t2r)) ||
      (a->counts && !aligned4(a->counts)))
    return QSA_B200_ERR_MISALIGNED;
  return QSA_B200_OK;
}

int check_decode_args(const qsa_b200_decode_args* a) {
  int st = check_index_args(a);
  if (st != QSA_B200_OK) return st;
  if (a->num_q_heads < 1 || a->num_kv_heads < 1 || a->num_q_heads % a->num_kv_heads != 0)
    return QSA_B200_ERR_BAD_SHAPE;
  if (a->head_dim != 128) return QSA_B200_ERR_UNSUPPORTED;
  const int group = a->num_q_heads / a->num_kv_heads;
  if (group > 32) return QSA_B200_ERR_UNSUPPORTED;
  if (a->kernel == QSA_B200_KERNEL_TC && !tc_supports_group(group)) return QSA_B200_ERR_UNSUPPORTED;
  if (a->kernel < QSA_B200_KERNEL_AUTO || a->kernel > QSA_B200_KERNEL_SIMT) return QSA_B200_ERR_UNSUPPORTED;
  if ((int64_t)a->rows * a->num_kv_heads > 0x7fffffffll) return QSA_B200_ERR_BAD_SHAPE;
  if (a->kernel == QSA_B200_KERNEL_TC || (a->kernel == QSA_B200_KERNEL_AUTO && tc_supports_group(group))) {
    // the tensor-core kernel's limits: its row map holds token slots as
    // int32 and its tensor maps address at most 2^31 - 1 (slot, KV head)
    // rows of 128 bytes (256 GiB per cache); its work items are counted in
    // int32
    if (a->num_pages * a->page_size * a->num_kv_heads > 0x7fffffffll) return QSA_B200_ERR_UNSUPPORTED;
    const int64_t chunk = tc_chunk_tokens(group);
    const int64_t chunks = a->topk <= chunk ? 1 : (a->topk + chunk - 1) / chunk;
    const int64_t heads = (int64_t)a->num_kv_heads * (group > kMaxGroupTc ? 2 : 1);  // items count virtual heads
    if ((int64_t)a->rows * heads * chunks > 0x3fffffffll) return QSA_B200_ERR_UNSUPPORTED;
  }
  if (a->rows == 0) return QSA_B200_OK;
  if (!a->q || !a->k_cache || !a->v_cache || !a->gate || !a->out) return QSA_B200_ERR_NULL_POINTER;
  if (!aligned16(a->q) || !aligned16(a->k_cache) || !aligned16(a->v_cache) || !aligned16(a->gate) ||
      !aligned16(a->out))
    return QSA_B200_ERR_MISALIGNED;
  return QSA_B200_OK;
}

void fill_params(const qsa_b200_decode_args* a, DecodeParams* p) {
  p->q = static_cast<const __nv_bfloat16*>(a->q);
  p->gate = static_cast<const __nv_bfloat16*>(a->gate);
  p->out = static_cast<__nv_bfloat16*>(a->out);
  p->k = static_cast<const uint8_t*>(a->k_cache);
  p->v = static_cast<const uint8_t*>(a->v_cache);
  p->indices = a->indices;
  p->counts = a->counts;
  p->btable = a->btable;
  p->t2r = a->t2r;
  p->score_scale_log2 = a->softmax_scale * a->k_scale * 1.4426950408889634f;
  p->v_scale = a->v_scale;
  p->rows = a->rows;
  p->num_q_heads = a->num_q_heads;
  p->num_kv_heads = a->num_kv_heads;
  p->group = a->num_kv_heads > 0 ? a->num_q_heads / a->num_kv_heads : 0;
  p->page_size = a->page_size;
  int shift = -1;
  for (int s = 0; s < 31; ++s)
    if ((1 << s) == a->page_size) shift = s;
  p->page_shift = shift;
  p->pages_per_req = a->pages_per_req;
  p->num_reqs = a->num_reqs;
  p->num_pages = a->num_pages;
  p->topk = a->topk;
  p->indices_stride = a->indices_stride;
  p->count_column = a->count_column;
  p->btable_stride = a->btable_stride;
  p->chunk_tokens = tc_chunk_tokens(p->group);
  p->num_chunks = num_chunks_for(a->topk, p->group);
  p->part_o = nullptr;
  p->part_lse = nullptr;
  p->rowmap = nullptr;
  p->rowmap_stride = p->num_chunks * p->chunk_tokens;
  p->tile_flags = nullptr;
  p->item_counter = nullptr;
  p->merge_chunks = 0;
  p->err = nullptr;
  p->wait_limit_ns = wait_limit_ns();
}

bool uses_tc(const qsa_b200_decode_args* a, int group) {
  return a->kernel == QSA_B200_KERNEL_TC || (a->kernel == QSA_B200_KERNEL_AUTO && tc_supports_group(group));
}

int64_t align256(int64_t x) { return (x + 255) / 256 * 256; }

// Workspace parts: [row map, tile flags, claim counter][partial outputs][partial log-sum-exps].
struct WorkspaceLayout {
  int64_t rowmap_bytes, part_o_bytes, part_lse_bytes;
  int64_t total() const { return rowmap_bytes + part_o_bytes + part_lse_bytes; }
};

// The split partials are left out when the tensor-core kernel merges the
// chunks of each (row, KV head) itself (tc_merges_chunks on the current
// device), since then nothing writes or reads them.
WorkspaceLayout workspace_for(const DecodeParams& p, bool tc) {
  WorkspaceLayout w{0, 0, 0};
  if (tc)
    w.rowmap_bytes = align256((int64_t)p.rows * p.rowmap_stride * 4) + align256((int64_t)p.rows * p.num_chunks * 16) + 256;
  if (p.num_chunks > 1 && !(tc && tc_merges_chunks(p))) {
    const int64_t n = (int64_t)p.rows * p.num_q_heads * p.num_chunks;
    w.part_o_bytes = align256(n * 128 * 4);
    w.part_lse_bytes = align256(n * 4);
  }
  return w;
}

}  // namespace
}  // namespace qsa

using namespace qsa;

extern "C" {

int qsa_b200_abi_version(void) { return QSA_B200_ABI_VERSION; }

const char* qsa_b200_status_string(int status) {
  switch (status) {
    case QSA_B200_OK: return "ok";
    case QSA_B200_ERR_NULL_POINTER: return "a required pointer is NULL";
    case QSA_B200_ERR_BAD_SHAPE: return "invalid or inconsistent sizes";
    case QSA_B200_ERR_UNSUPPORTED: return "unsupported shape (head_dim must be 128, group size <= 32)";
    case QSA_B200_ERR_MISALIGNED: return "a tensor is not aligned (16 bytes for q/k/v/gate/out, 4 for int32)";
    case QSA_B200_ERR_WORKSPACE: return "workspace missing or too small";
    case QSA_B200_ERR_DEVICE: return "current CUDA device is not an sm_100 (B200) part";
    case QSA_B200_ERR_LAUNCH: return "CUDA kernel launch failed";
    case QSA_B200_ERR_KERNEL: return "a kernel reported a device-side failure";
    case QSA_B200_ERR_TOO_LARGE:
      return "workspace needed exceeds QSA_B200_NOALLOC_SCRATCH_BYTES (use qsa_b200_decode with a workspace)";
    case QSA_B200_ERR_BAD_VALUE: return "a scale is not a positive finite number";
    default: return "unknown status";
  }
}

int64_t qsa_b200_workspace_bytes(const qsa_b200_decode_args* args) {
  const int st = check_decode_args(args);
  if (st != QSA_B200_OK) return st;
  DecodeParams p;
  fill_params(args, &p);
  if (args->rows == 0) return 0;
  return workspace_for(p, uses_tc(args, p.group)).total();
}

int qsa_b200_decode(const qsa_b200_decode_args* args, void* workspace, size_t workspace_bytes,
                    qsa_b200_stream_t stream) {
  int st = check_decode_args(args);
  if (st != QSA_B200_OK) return st;
  if (args->rows == 0) return QSA_B200_OK;
  st = check_device();
  if (st != QSA_B200_OK) return st;
  DecodeParams p;
  fill_params(args, &p);
  p.err = device_error_word();
  const bool use_tc = uses_tc(args, p.group);
  const WorkspaceLayout lay = workspace_for(p, use_tc);
  if (lay.total() > 0) {
    if (!workspace || (int64_t)workspace_bytes < lay.total()) return QSA_B200_ERR_WORKSPACE;
    if (reinterpret_cast<uintptr_t>(workspace) & 255u) return QSA_B200_ERR_MISALIGNED;
    char* ws = static_cast<char*>(workspace);
    if (use_tc) {
      p.rowmap = reinterpret_cast<int32_t*>(ws);
      p.tile_flags = reinterpret_cast<uint8_t*>(ws + align256((int64_t)p.rows * p.rowmap_stride * 4));
      p.item_counter = reinterpret_cast<int*>(reinterpret_cast<char*>(p.tile_flags) +
                                              align256((int64_t)p.rows * p.num_chunks * 16));
    }
    if (lay.part_o_bytes > 0) {
      p.part_o = reinterpret_cast<float*>(ws + lay.rowmap_bytes);
      p.part_lse = reinterpret_cast<float*>(ws + lay.rowmap_bytes + lay.part_o_bytes);
    }
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t e = use_tc ? launch_decode_tc(p, s) : launch_decode_simt(p, s);
  if (e != cudaSuccess) return QSA_B200_ERR_LAUNCH;
  if (p.num_chunks > 1 && !(use_tc && tc_merges_chunks(p))) {
    e = launch_combine(p, s);
    if (e != cudaSuccess) return QSA_B200_ERR_LAUNCH;
  }
  return QSA_B200_OK;
}

int qsa_b200_slots(const qsa_b200_decode_args* args, int64_t* slots, qsa_b200_stream_t stream) {
  int st = check_index_args(args);
  if (st != QSA_B200_OK) return st;
  if (args->rows == 0 || args->topk == 0) return QSA_B200_OK;
  if (!slots) return QSA_B200_ERR_NULL_POINTER;
  if (reinterpret_cast<uintptr_t>(slots) & 7u) return QSA_B200_ERR_MISALIGNED;
  st = check_device();
  if (st != QSA_B200_OK) return st;
  DecodeParams p;
  fill_params(args, &p);
  const cudaError_t e = launch_slots(p, slots, reinterpret_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? QSA_B200_OK : QSA_B200_ERR_LAUNCH;
}

void launch_qsa_cuda(const void* q, const void* k, const void* v, const void* indices, const void* btable,
                     const int32_t* t2r, const void* gate, void* out, float softmax_scale, float v_scale,
                     int32_t nblocks, int32_t nreqs, int32_t num_q_heads, int32_t num_kv_heads, int32_t topk,
                     int32_t page_sz, int32_t max_pages, int32_t head_dim, int32_t group_sz,
                     qsa_b200_stream_t stream) {
  if (num_kv_heads < 1 || group_sz * num_kv_heads != num_q_heads || !t2r) {
    t_last_status = QSA_B200_ERR_BAD_SHAPE;
    return;
  }
  qsa_b200_decode_args a = {};
  a.q = q;
  a.k_cache = k;
  a.v_cache = v;
  a.indices = static_cast<const int32_t*>(indices);
  a.counts = nullptr;
  a.btable = static_cast<const int32_t*>(btable);
  a.t2r = t2r;
  a.gate = gate;
  a.out = out;
  // The reference passes k_scale * log2(e) / sqrt(D); the library takes the
  // natural-log score scale and folds log2(e) itself.
  a.softmax_scale = softmax_scale / 1.4426950408889634f;
  a.k_scale = 1.0f;
  a.v_scale = v_scale;
  a.rows = nreqs;
  a.num_q_heads = num_q_heads;
  a.num_kv_heads = num_kv_heads;
  a.head_dim = head_dim;
  a.page_size = page_sz;
  a.pages_per_req = max_pages;
  a.num_reqs = nreqs;
  a.num_pages = nblocks;
  a.topk = topk;
  a.indices_stride = (int64_t)topk + 1;
  a.count_column = 1;
  a.btable_stride = max_pages;
  a.kernel = QSA_B200_KERNEL_AUTO;
  // This signature takes no workspace: the row map (and any split partials)
  // go to the library's fixed per-device scratch.
  t_last_status = qsa_b200_decode_noalloc(&a, stream);
}

int qsa_b200_cache_write(const qsa_b200_cache_write_args* a, qsa_b200_stream_t stream) {
  if (!a) return QSA_B200_ERR_NULL_POINTER;
  if (a->tokens < 0 || a->num_kv_heads < 1 || a->page_size < 1 || a->num_pages < 1) return QSA_B200_ERR_BAD_SHAPE;
  if (a->head_dim != 128) return QSA_B200_ERR_UNSUPPORTED;
  if (a->input_dtype < QSA_B200_DTYPE_BF16 || a->input_dtype > QSA_B200_DTYPE_F32) return QSA_B200_ERR_UNSUPPORTED;
  if (!(a->k_scale > 0.f) || !(a->v_scale > 0.f) || !std::isfinite(a->k_scale) || !std::isfinite(a->v_scale))
    return QSA_B200_ERR_BAD_VALUE;
  const int64_t row_elems = (int64_t)a->num_kv_heads * a->head_dim;
  if (a->token_stride < row_elems) return QSA_B200_ERR_BAD_SHAPE;
  if (a->tokens == 0) return QSA_B200_OK;
  if (!a->k || !a->v || !a->slots || !a->k_cache || !a->v_cache) return QSA_B200_ERR_NULL_POINTER;
  const int64_t elem = a->input_dtype == QSA_B200_DTYPE_F32 ? 4 : 2;
  if (!aligned16(a->k) || !aligned16(a->v) || !aligned16(a->k_cache) || !aligned16(a->v_cache) ||
      (a->token_stride * elem) % 16 != 0 || (reinterpret_cast<uintptr_t>(a->slots) & 7u))
    return QSA_B200_ERR_MISALIGNED;
  const int st = check_device();
  if (st != QSA_B200_OK) return st;
  CacheWriteParams p;
  p.k = a->k;
  p.v = a->v;
  p.slots = a->slots;
  p.k_cache = static_cast<uint8_t*>(a->k_cache);
  p.v_cache = static_cast<uint8_t*>(a->v_cache);
  // one fp32 reciprocal per call; every element is then multiplied by it
  p.k_inv_scale = 1.0f / a->k_scale;
  p.v_inv_scale = 1.0f / a->v_scale;
  p.tokens = a->tokens;
  p.num_kv_heads = a->num_kv_heads;
  p.page_size = a->page_size;
  p.num_pages = a->num_pages;
  p.token_stride = a->token_stride;
  p.dtype = a->input_dtype;
  const cudaError_t e = launch_cache_write(p, reinterpret_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? QSA_B200_OK : QSA_B200_ERR_LAUNCH;
}

int qsa_b200_topk_select(const qsa_b200_topk_args* a, qsa_b200_stream_t stream) {
  if (!a) return QSA_B200_ERR_NULL_POINTER;
  if (a->rows < 0 || a->ctx < 1 || a->ctx > QSA_B200_TOPK_MAX_CTX || a->score_stride < a->ctx ||
      a->out_stride < a->k)
    return QSA_B200_ERR_BAD_SHAPE;
  if (a->k < 1) return QSA_B200_ERR_BAD_VALUE;
  if (a->rows == 0) return QSA_B200_OK;
  if (!a->scores || !a->out) return QSA_B200_ERR_NULL_POINTER;
  if ((reinterpret_cast<uintptr_t>(a->scores) & 3u) || (reinterpret_cast<uintptr_t>(a->out) & 3u) ||
      (reinterpret_cast<uintptr_t>(a->lengths) & 3u))
    return QSA_B200_ERR_MISALIGNED;
  const int st = check_device();
  if (st != QSA_B200_OK) return st;
  TopkParams p;
  p.scores = a->scores;
  p.lengths = a->lengths;
  p.out = a->out;
  p.rows = a->rows;
  p.ctx = a->ctx;
  p.k = a->k;
  p.score_stride = a->score_stride;
  p.out_stride = a->out_stride;
  const cudaError_t e = launch_topk(p, reinterpret_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? QSA_B200_OK : QSA_B200_ERR_LAUNCH;
}

int qsa_b200_last_status(void) { return t_last_status; }

uint64_t qsa_b200_testing_set_wait_limit_ns(uint64_t ns) {
  return g_wait_limit_ns.exchange(ns == 0 ? kDefaultWaitLimitNs : ns, std::memory_order_relaxed);
}

int qsa_b200_device_error(int clear) {
  int val = 0;
  if (cudaMemcpyFromSymbol(&val, qsa::g_device_error, sizeof(int)) != cudaSuccess) return QSA_B200_ERR_LAUNCH;
  if (clear) {
    const int zero = 0;
    if (cudaMemcpyToSymbol(qsa::g_device_error, &zero, sizeof(int)) != cudaSuccess) return QSA_B200_ERR_LAUNCH;
  }
  return val;
}

}  // extern "C"
