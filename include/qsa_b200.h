/*
 * qsa_b200.h -- C ABI of the B200 (sm_100a) sparse paged GQA FP8 decode
 * attention library (libqsa_b200.so).
 *
 * The operation, for each Top-K row r, query head h and KV head g = h / G:
 *
 *   out[r,h,:] = softmax_t( q[r,h] . K[slot_t, g] * k_scale * softmax_scale )
 *                . V[slot_t, g] * v_scale  (*)  sigmoid(gate[r,h,:])
 *
 *   slot_t = btable[t2r[r], t / P] * P + t % P   for each selected token t
 *
 * with bf16 q / gate / out [rows, Hq, 128], FP8 E4M3FN K/V caches
 * [num_pages, P, Hkv, 128], int32 block table, Top-K indices and request map.
 *
 * All pointers are device pointers owned by the caller. Calls are
 * asynchronous on the given stream and never synchronise, trap or allocate.
 * Entry points return 0 or a negative QSA_B200_ERR_* status.
 *
 * Reference interfaces this library replaces (Ammar-Alnagar/QSA-FP8-SM89):
 *   - the C-ABI launcher  launch_qsa_cuda        sm89_cuda.cu:232-253
 *   - the Python entry    run(q, k, v, k_scale, v_scale, btable, t2r,
 *                          indices, gate)        sm89_cutedsl.py:311-351
 *   - the eager oracle    torch_eager(...)       sm89_torch.py:27-54
 *   - the Triton launch   launch(q, k, v, indices, btable, t2r, gate, out,
 *                          k_scale, v_scale)     sm89_triton.py:118-142
 *   - the cache producer  (randn * 0.1).to(float8_e4m3fn) into the paged
 *                          [num_pages, P, Hkv, 128] layout, with the scales
 *                          returned beside it    sm89_cutedsl.py:48-62, :79
 *                          (qsa_b200_cache_write: the same layout, written
 *                          at given token slots, saturating at +-448)
 */
#ifndef QSA_B200_H_
#define QSA_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define QSA_B200_API __attribute__((visibility("default")))
#else
#define QSA_B200_API
#endif

/* A CUDA stream handle (cudaStream_t / CUstream); NULL is the legacy stream. */
typedef struct CUstream_st* qsa_b200_stream_t;

#define QSA_B200_ABI_VERSION 1

enum {
  QSA_B200_OK = 0,
  QSA_B200_ERR_NULL_POINTER = -1, /* a required pointer is NULL */
  QSA_B200_ERR_BAD_SHAPE = -2,    /* a size is negative / inconsistent */
  QSA_B200_ERR_UNSUPPORTED = -3,  /* head_dim != 128, group > 32, or past a tensor-core kernel limit */
  QSA_B200_ERR_MISALIGNED = -4,   /* a tensor is not 16-byte aligned */
  QSA_B200_ERR_WORKSPACE = -5,    /* workspace missing or too small */
  QSA_B200_ERR_DEVICE = -6,       /* current device is not sm_100 */
  QSA_B200_ERR_LAUNCH = -7,       /* the CUDA launch itself failed */
  QSA_B200_ERR_KERNEL = -8,       /* a kernel reported a device-side failure */
  QSA_B200_ERR_TOO_LARGE = -9,    /* workspace above the fixed scratch of qsa_b200_decode_noalloc */
  QSA_B200_ERR_BAD_VALUE = -10    /* a scale is not a positive finite number */
};

/* Kernel selection. AUTO picks the tensor-core kernel for every group size
 * (Hq / Hkv) from 1 to 32; above 16 each KV head's query heads go in two
 * halves, each half reading the KV rows. The CUDA-core kernel (SIMT) takes
 * the same sizes. The tensor-core kernel (explicit or through AUTO)
 * returns QSA_B200_ERR_UNSUPPORTED for a cache of more than 2^31 - 1 rows of
 * 128 bytes (num_pages * page_size * num_kv_heads; 256 GiB per cache) and
 * for more than 2^30 - 1 work items (rows * num_kv_heads * ceil(topk / 512)). */
enum { QSA_B200_KERNEL_AUTO = 0, QSA_B200_KERNEL_TC = 1, QSA_B200_KERNEL_SIMT = 2 };

typedef struct qsa_b200_decode_args {
  const void* q;          /* bf16 [rows, num_q_heads, head_dim], contiguous */
  const void* k_cache;    /* fp8 e4m3fn [num_pages, page_size, num_kv_heads, head_dim] */
  const void* v_cache;    /* same layout as k_cache */
  const int32_t* indices; /* [rows, indices_stride]; first `topk` columns = logical tokens, <0 = masked */
  const int32_t* counts;  /* optional [rows]: only the first counts[r] columns may be valid */
  const int32_t* btable;  /* [num_reqs, btable_stride]; first pages_per_req columns = physical pages */
  const int32_t* t2r;     /* optional [rows]: Top-K row -> block-table row (NULL = identity) */
  const void* gate;       /* bf16 [rows, num_q_heads, head_dim], contiguous */
  void* out;              /* bf16 [rows, num_q_heads, head_dim], contiguous */
  float softmax_scale;    /* natural-log domain score scale, e.g. 1/sqrt(head_dim) */
  float k_scale;          /* K dequantisation scale (folded into the score scale) */
  float v_scale;          /* V dequantisation scale */
  int32_t rows;
  int32_t num_q_heads;
  int32_t num_kv_heads;
  int32_t head_dim;       /* must be 128 */
  int32_t page_size;
  int32_t pages_per_req;
  int32_t num_reqs;
  int64_t num_pages;
  int32_t topk;
  int64_t indices_stride; /* >= topk (+1 with count_column) */
  int32_t count_column;   /* nonzero: counts[r] = indices[r * indices_stride + topk] */
  int64_t btable_stride;  /* >= pages_per_req */
  int32_t kernel;         /* QSA_B200_KERNEL_* */
} qsa_b200_decode_args;

/* Bytes of device workspace qsa_b200_decode needs, each part 256-byte
 * aligned: the tensor-core kernel's row map (one int32 token slot per Top-K
 * entry: rows x chunks x 512 entries), its tile flags (16 bytes per row and
 * chunk) and its item claim counter (256 bytes), then, when a Top-K row spans
 * more than one chunk, the split partial outputs and log-sum-exps.
 * 0 only for the CUDA-core kernel without a split. Negative on invalid
 * arguments. */
QSA_B200_API int64_t qsa_b200_workspace_bytes(const qsa_b200_decode_args* args);

/* The decode. `workspace` (256-byte aligned) must hold
 * qsa_b200_workspace_bytes(args) bytes; it may be NULL when that is 0. The
 * workspace needs no clearing and may be reused by the next call on the same
 * stream.
 * Replaces launch_qsa_cuda (sm89_cuda.cu:232-301) / run (sm89_cutedsl.py:311). */
QSA_B200_API int qsa_b200_decode(const qsa_b200_decode_args* args, void* workspace, size_t workspace_bytes,
                    qsa_b200_stream_t stream);

/* The index decode alone: slots[r * topk + c] = physical token slot
 * (phys_page * page_size + t % page_size) of Top-K entry (r, c), or -1 when it
 * is masked -- the bit-exact part of the path (sm89_torch.py:30-39;
 * sm89_cuda.cu:110-115, :147-164). Only the index/table fields of `args` are
 * read; q, caches, gate and out may be NULL. */
QSA_B200_API int qsa_b200_slots(const qsa_b200_decode_args* args, int64_t* slots, qsa_b200_stream_t stream);

/* Drop-in for the reference's C-ABI launcher, same signature and argument
 * meaning (sm89_cuda.cu:232-253): indices are [nreqs, topk + 1] with the valid
 * count in the last column, softmax_scale is in the log2 domain
 * (k_scale * log2(e) / sqrt(head_dim)), rows == nreqs and t2r is required.
 * Returns void like the reference; the status of the call is available from
 * qsa_b200_last_status(). Rows with an out-of-range t2r entry or no valid
 * token are written as zeros (the reference leaves them unwritten). This
 * signature takes no workspace: the call runs as qsa_b200_decode_noalloc, on
 * the library's fixed per-device scratch (QSA_B200_ERR_TOO_LARGE beyond it),
 * so calls that overlap in time on one device race. */
QSA_B200_API void launch_qsa_cuda(const void* q, const void* k, const void* v, const void* indices, const void* btable,
                     const int32_t* t2r, const void* gate, void* out, float softmax_scale, float v_scale,
                     int32_t nblocks, int32_t nreqs, int32_t num_q_heads, int32_t num_kv_heads, int32_t topk,
                     int32_t page_sz, int32_t max_pages, int32_t head_dim, int32_t group_sz,
                     qsa_b200_stream_t stream);

/* Status of the calling thread's last launch_qsa_cuda. */
QSA_B200_API int qsa_b200_last_status(void);

/* Reads the device-side error word of the current device (nonzero when a
 * kernel gave up on a bounded wait); clears it when `clear` is nonzero.
 * Synchronous; returns a negative status if the read itself fails. */
QSA_B200_API int qsa_b200_device_error(int clear);

/* Human-readable text of a status code. */
QSA_B200_API const char* qsa_b200_status_string(int status);

/* QSA_B200_ABI_VERSION of the loaded library. */
QSA_B200_API int qsa_b200_abi_version(void);

/* Fixed workspace of qsa_b200_decode_noalloc, per device: 32 MiB, room for
 * the row map and split partials of, for example, 128 rows x 64 query heads x
 * 4 chunks of 512 Top-K entries (18 MiB). */
#define QSA_B200_NOALLOC_SCRATCH_BYTES (32u * 1024u * 1024u)

/* Allocation-free qsa_b200_decode. This entry point has NO counterpart in
 * the reference. It serves callers that cannot allocate device memory at
 * call time: a runtime with a fixed device budget, a latency-critical loop,
 * an FFI caller without an allocator.
 *   - The workspace (row map and split partials) is a file-scope device
 *     array of QSA_B200_NOALLOC_SCRATCH_BYTES per device; the call makes no
 *     cudaMalloc, cudaFree or other allocating call.
 *   - Returns QSA_B200_ERR_TOO_LARGE, before touching the device, when
 *     qsa_b200_workspace_bytes(args) exceeds that maximum; otherwise the
 *     statuses and results of qsa_b200_decode.
 *   - The first call on each device looks up the array's address
 *     (cudaGetSymbolAddress) with that device current: make that first call
 *     before any stream capture.
 *   - Calls that overlap in time on one device (other streams or threads)
 *     share the scratch and race; the caller serialises them. */
QSA_B200_API int qsa_b200_decode_noalloc(const qsa_b200_decode_args* args, qsa_b200_stream_t stream);

/* Element types of the new keys and values of qsa_b200_cache_write. */
enum { QSA_B200_DTYPE_BF16 = 0, QSA_B200_DTYPE_F16 = 1, QSA_B200_DTYPE_F32 = 2 };

typedef struct qsa_b200_cache_write_args {
  const void* k;         /* new keys [tokens, num_kv_heads, head_dim] of input_dtype */
  const void* v;         /* new values, same shape, type and strides as k */
  const int64_t* slots;  /* [tokens]: physical token slot phys_page * page_size + offset of each token;
                            a negative slot or one past the cache is skipped */
  void* k_cache;         /* fp8 e4m3fn [num_pages, page_size, num_kv_heads, head_dim] */
  void* v_cache;         /* same layout as k_cache */
  float k_scale;         /* dequantisation scales (cache value * scale = stored value) */
  float v_scale;
  int32_t tokens;
  int32_t num_kv_heads;
  int32_t head_dim;      /* must be 128 */
  int32_t page_size;
  int64_t num_pages;
  int64_t token_stride;  /* elements from one token of k / v to the next, >= num_kv_heads * head_dim */
  int32_t input_dtype;   /* QSA_B200_DTYPE_* */
} qsa_b200_cache_write_args;

/* Quantises new keys and values into the paged FP8 caches:
 *   cache[slot, g, d] = e4m3fn(x[t, g, d] * inv)   for slot = slots[t]
 * with inv = 1 / scale rounded to fp32 once, an fp32 product, and the
 * conversion rounding to the nearest E4M3FN value (ties to even), saturating
 * at +-448: a finite value
 * beyond the range and an infinity become +-448, NaN stays NaN (torch's cast
 * turns |x| >= 464 into NaN instead). Rows of skipped tokens are left as they
 * were. Two tokens with the same slot race (the caller gives each slot once).
 * Needs k, v 16-byte aligned with token_stride * element size a multiple of
 * 16, and 16-byte aligned caches. Asynchronous on `stream`. */
QSA_B200_API int qsa_b200_cache_write(const qsa_b200_cache_write_args* args, qsa_b200_stream_t stream);

typedef struct qsa_b200_topk_args {
  const float* scores;    /* [rows, ctx] fp32 per-position scores, row stride score_stride */
  const int32_t* lengths; /* optional [rows]: valid positions of each row (clamped to [0, ctx]); NULL = ctx */
  int32_t* out;           /* [rows, k] int32 Top-K indices, row stride out_stride */
  int32_t rows;
  int32_t ctx;            /* positions per row, 1 .. QSA_B200_TOPK_MAX_CTX */
  int32_t k;              /* selections per row, >= 1 */
  int64_t score_stride;   /* >= ctx */
  int64_t out_stride;     /* >= k */
} qsa_b200_topk_args;

#define QSA_B200_TOPK_MAX_CTX (1 << 20)

/* The Top-K index producer, the step before the decode: for each row, the
 * positions of the k highest scores, in ascending position order, as the
 * decode's [rows, k] int32 indices. A position t is a candidate when t is
 * below the row's length and its score is neither NaN nor -inf; at the k-th
 * score lower positions win; a row with fewer than k candidates is padded
 * with -1. No reference counterpart: the reference consumes Top-K indices but
 * does not produce them (sm89_cutedsl.py:72-76 builds sequential ones).
 * Needs 4-byte aligned scores, lengths and out. Asynchronous on `stream`. */
QSA_B200_API int qsa_b200_topk_select(const qsa_b200_topk_args* args, qsa_b200_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* QSA_B200_H_ */
