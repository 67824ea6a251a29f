// torch.ops.qsa_b200.* -- a thin PyTorch operator layer over the C ABI of
// libqsa_b200.so. It checks tensor dtypes / devices / layouts, takes the
// current CUDA stream, allocates the split workspace through PyTorch's caching
// allocator when one is needed and calls qsa_b200_decode / qsa_b200_slots.
// Only CUDA tensors are accepted (ops are registered for the CUDA dispatch
// key alone); there is no CPU implementation.
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/library.h>

#include <optional>

#include "../../include/qsa_b200.h"

namespace {

void check_i32(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.scalar_type() == at::kInt, name, " must be int32, got ", t.scalar_type());
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
}

void check_same_device(const at::Tensor& t, const at::Tensor& ref, const char* name) {
  TORCH_CHECK(t.device() == ref.device(), name, " is on ", t.device(), " but q is on ", ref.device());
}

void check_index_tensors(const at::Tensor& ref, const at::Tensor& btable, const std::optional<at::Tensor>& t2r,
                         const at::Tensor& indices, const std::optional<at::Tensor>& counts, int64_t rows,
                         int64_t topk, bool count_column) {
  check_i32(btable, "btable");
  check_i32(indices, "indices");
  check_same_device(btable, ref, "btable");
  check_same_device(indices, ref, "indices");
  TORCH_CHECK(btable.dim() == 2 && btable.stride(1) == 1, "btable must be 2-D [num_reqs, pages_per_req] with unit column stride");
  TORCH_CHECK(indices.dim() == 2 && indices.stride(1) == 1, "indices must be 2-D [rows, K] with unit column stride");
  TORCH_CHECK(indices.size(0) == rows, "indices has ", indices.size(0), " rows, expected ", rows);
  TORCH_CHECK(topk >= 0 && indices.size(1) >= topk + (count_column ? 1 : 0),
              "indices has ", indices.size(1), " columns; topk=", topk, count_column ? " plus the count column" : "");
  if (t2r) {
    check_i32(*t2r, "t2r");
    check_same_device(*t2r, ref, "t2r");
    TORCH_CHECK(t2r->dim() == 1 && t2r->size(0) == rows && t2r->is_contiguous(), "t2r must be contiguous [rows]");
  }
  if (counts) {
    check_i32(*counts, "counts");
    check_same_device(*counts, ref, "counts");
    TORCH_CHECK(counts->dim() == 1 && counts->size(0) == rows && counts->is_contiguous(),
                "counts must be contiguous [rows]");
  }
}

void fill_index_args(qsa_b200_decode_args& a, const at::Tensor& btable, const std::optional<at::Tensor>& t2r,
                     const at::Tensor& indices, const std::optional<at::Tensor>& counts, int64_t topk,
                     bool count_column) {
  a.indices = indices.data_ptr<int32_t>();
  a.counts = counts ? counts->data_ptr<int32_t>() : nullptr;
  a.btable = btable.data_ptr<int32_t>();
  a.t2r = t2r ? t2r->data_ptr<int32_t>() : nullptr;
  a.num_reqs = (int32_t)btable.size(0);
  a.pages_per_req = (int32_t)btable.size(1);
  a.btable_stride = btable.stride(0);
  a.topk = (int32_t)topk;
  a.indices_stride = indices.stride(0);
  a.count_column = count_column ? 1 : 0;
}

void decode(const at::Tensor& q, const at::Tensor& k_cache, const at::Tensor& v_cache, const at::Tensor& btable,
            const std::optional<at::Tensor>& t2r, const at::Tensor& indices, const at::Tensor& gate,
            const std::optional<at::Tensor>& counts, double softmax_scale, double k_scale, double v_scale,
            bool count_column, int64_t topk, int64_t kernel, at::Tensor& out) {
  TORCH_CHECK(q.is_cuda(), "q must be a CUDA tensor");
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && gate.scalar_type() == at::kBFloat16 &&
                  out.scalar_type() == at::kBFloat16,
              "q, gate and out must be bfloat16");
  TORCH_CHECK(k_cache.scalar_type() == at::kFloat8_e4m3fn || k_cache.scalar_type() == at::kByte,
              "k_cache must be float8_e4m3fn (or its uint8 bytes)");
  TORCH_CHECK(v_cache.scalar_type() == k_cache.scalar_type(), "v_cache must have k_cache's dtype");
  TORCH_CHECK(q.dim() == 3 && q.is_contiguous(), "q must be contiguous [rows, Hq, D]");
  TORCH_CHECK(gate.sizes() == q.sizes() && gate.is_contiguous(), "gate must be contiguous and shaped like q");
  TORCH_CHECK(out.sizes() == q.sizes() && out.is_contiguous(), "out must be contiguous and shaped like q");
  TORCH_CHECK(k_cache.dim() == 4 && k_cache.is_contiguous(), "k_cache must be contiguous [pages, P, Hkv, D]");
  TORCH_CHECK(v_cache.sizes() == k_cache.sizes() && v_cache.is_contiguous(), "v_cache must match k_cache");
  TORCH_CHECK(k_cache.size(3) == q.size(2), "head_dim of q (", q.size(2), ") and cache (", k_cache.size(3), ") differ");
  check_same_device(k_cache, q, "k_cache");
  check_same_device(v_cache, q, "v_cache");
  check_same_device(gate, q, "gate");
  check_same_device(out, q, "out");
  const int64_t rows = q.size(0);
  check_index_tensors(q, btable, t2r, indices, counts, rows, topk, count_column);

  c10::cuda::CUDAGuard guard(q.device());
  qsa_b200_decode_args a = {};
  a.q = q.data_ptr();
  a.k_cache = k_cache.data_ptr();
  a.v_cache = v_cache.data_ptr();
  a.gate = gate.data_ptr();
  a.out = out.data_ptr();
  fill_index_args(a, btable, t2r, indices, counts, topk, count_column);
  a.softmax_scale = (float)softmax_scale;
  a.k_scale = (float)k_scale;
  a.v_scale = (float)v_scale;
  a.rows = (int32_t)rows;
  a.num_q_heads = (int32_t)q.size(1);
  a.num_kv_heads = (int32_t)k_cache.size(2);
  a.head_dim = (int32_t)q.size(2);
  a.page_size = (int32_t)k_cache.size(1);
  a.num_pages = k_cache.size(0);
  a.kernel = (int32_t)kernel;

  const int64_t ws = qsa_b200_workspace_bytes(&a);
  TORCH_CHECK(ws >= 0, "qsa_b200: ", qsa_b200_status_string((int)ws));
  at::Tensor workspace;
  if (ws > 0) workspace = at::empty({ws}, q.options().dtype(at::kByte));
  const cudaStream_t stream = c10::cuda::getCurrentCUDAStream(q.device().index()).stream();
  const int st = qsa_b200_decode(&a, ws > 0 ? workspace.data_ptr() : nullptr, (size_t)ws,
                                 reinterpret_cast<qsa_b200_stream_t>(stream));
  TORCH_CHECK(st == QSA_B200_OK, "qsa_b200_decode failed: ", qsa_b200_status_string(st));
}

void slots(const at::Tensor& btable, const std::optional<at::Tensor>& t2r, const at::Tensor& indices,
           const std::optional<at::Tensor>& counts, bool count_column, int64_t topk, int64_t page_size,
           int64_t num_pages, at::Tensor& out) {
  TORCH_CHECK(indices.is_cuda(), "indices must be a CUDA tensor");
  const int64_t rows = indices.size(0);
  check_index_tensors(indices, btable, t2r, indices, counts, rows, topk, count_column);
  TORCH_CHECK(out.scalar_type() == at::kLong && out.is_contiguous() && out.dim() == 2 && out.size(0) == rows &&
                  out.size(1) == topk,
              "out must be contiguous int64 [rows, topk]");
  check_same_device(out, indices, "out");
  c10::cuda::CUDAGuard guard(indices.device());
  qsa_b200_decode_args a = {};
  fill_index_args(a, btable, t2r, indices, counts, topk, count_column);
  a.rows = (int32_t)rows;
  a.page_size = (int32_t)page_size;
  a.num_pages = num_pages;
  const cudaStream_t stream = c10::cuda::getCurrentCUDAStream(indices.device().index()).stream();
  const int st = qsa_b200_slots(&a, out.data_ptr<int64_t>(), reinterpret_cast<qsa_b200_stream_t>(stream));
  TORCH_CHECK(st == QSA_B200_OK, "qsa_b200_slots failed: ", qsa_b200_status_string(st));
}

void cache_write(const at::Tensor& k_new, const at::Tensor& v_new, const at::Tensor& slots_t, double k_scale,
                 double v_scale, at::Tensor& k_cache, at::Tensor& v_cache) {
  TORCH_CHECK(k_new.is_cuda(), "k_new must be a CUDA tensor");
  int32_t dtype = -1;
  if (k_new.scalar_type() == at::kBFloat16) dtype = QSA_B200_DTYPE_BF16;
  if (k_new.scalar_type() == at::kHalf) dtype = QSA_B200_DTYPE_F16;
  if (k_new.scalar_type() == at::kFloat) dtype = QSA_B200_DTYPE_F32;
  TORCH_CHECK(dtype >= 0, "k_new must be bfloat16, float16 or float32, got ", k_new.scalar_type());
  TORCH_CHECK(v_new.scalar_type() == k_new.scalar_type(), "v_new must have k_new's dtype");
  TORCH_CHECK(k_new.dim() == 3 && k_new.stride(2) == 1 && k_new.stride(1) == k_new.size(2),
              "k_new must be [tokens, Hkv, D] with contiguous heads");
  TORCH_CHECK(v_new.sizes() == k_new.sizes() && v_new.strides() == k_new.strides(),
              "v_new must have k_new's shape and strides");
  TORCH_CHECK(slots_t.scalar_type() == at::kLong && slots_t.dim() == 1 && slots_t.size(0) == k_new.size(0) &&
                  slots_t.is_contiguous(),
              "slots must be contiguous int64 [tokens]");
  TORCH_CHECK(k_cache.scalar_type() == at::kFloat8_e4m3fn || k_cache.scalar_type() == at::kByte,
              "k_cache must be float8_e4m3fn (or its uint8 bytes)");
  TORCH_CHECK(v_cache.scalar_type() == k_cache.scalar_type(), "v_cache must have k_cache's dtype");
  TORCH_CHECK(k_cache.dim() == 4 && k_cache.is_contiguous() && v_cache.sizes() == k_cache.sizes() &&
                  v_cache.is_contiguous(),
              "k_cache / v_cache must be contiguous [pages, P, Hkv, D]");
  TORCH_CHECK(k_cache.size(2) == k_new.size(1) && k_cache.size(3) == k_new.size(2),
              "heads / head_dim of the new rows and the cache differ");
  for (const at::Tensor* t : std::initializer_list<const at::Tensor*>{&v_new, &slots_t, &k_cache, &v_cache})
    TORCH_CHECK(t->device() == k_new.device(), "all tensors must be on k_new's device");
  c10::cuda::CUDAGuard guard(k_new.device());
  qsa_b200_cache_write_args a = {};
  a.k = k_new.data_ptr();
  a.v = v_new.data_ptr();
  a.slots = slots_t.data_ptr<int64_t>();
  a.k_cache = k_cache.data_ptr();
  a.v_cache = v_cache.data_ptr();
  a.k_scale = (float)k_scale;
  a.v_scale = (float)v_scale;
  a.tokens = (int32_t)k_new.size(0);
  a.num_kv_heads = (int32_t)k_cache.size(2);
  a.head_dim = (int32_t)k_cache.size(3);
  a.page_size = (int32_t)k_cache.size(1);
  a.num_pages = k_cache.size(0);
  a.token_stride = k_new.size(0) > 1 ? k_new.stride(0) : k_new.size(1) * k_new.size(2);
  a.input_dtype = dtype;
  const cudaStream_t stream = c10::cuda::getCurrentCUDAStream(k_new.device().index()).stream();
  const int st = qsa_b200_cache_write(&a, reinterpret_cast<qsa_b200_stream_t>(stream));
  TORCH_CHECK(st == QSA_B200_OK, "qsa_b200_cache_write failed: ", qsa_b200_status_string(st));
}

}  // namespace

TORCH_LIBRARY(qsa_b200, m) {
  m.def(
      "decode(Tensor q, Tensor k_cache, Tensor v_cache, Tensor btable, Tensor? t2r, Tensor indices, "
      "Tensor gate, Tensor? counts, float softmax_scale, float k_scale, float v_scale, bool count_column, "
      "int topk, int kernel, Tensor(a!) out) -> ()");
  m.def(
      "slots(Tensor btable, Tensor? t2r, Tensor indices, Tensor? counts, bool count_column, int topk, "
      "int page_size, int num_pages, Tensor(a!) out) -> ()");
  m.def(
      "cache_write(Tensor k_new, Tensor v_new, Tensor slots, float k_scale, float v_scale, Tensor(a!) k_cache, "
      "Tensor(b!) v_cache) -> ()");
}

TORCH_LIBRARY_IMPL(qsa_b200, CUDA, m) {
  m.impl("decode", &decode);
  m.impl("slots", &slots);
  m.impl("cache_write", &cache_write);
}
