// Allocation-free decode entry point, qsa_b200_decode_noalloc (no counterpart
// in the reference).
//
// Some callers cannot allocate device memory at call time: a host runtime that
// owns a fixed device budget, a latency-critical loop that must not enter the
// CUDA allocator, or an FFI caller with no allocator (the reference-shaped
// launch_qsa_cuda runs here too). For them the workspace (the tensor-core
// kernel's row map, and the partial outputs and log2-sum-exps of Top-K rows
// longer than one chunk) comes from a fixed file-scope device array instead
// of a caller-supplied buffer. The array sits in this translation unit alone,
// so under CUDA's lazy module loading only callers of this entry point reserve
// it.
//
// Nothing in the scratch must start at zero: the row-map kernel writes every
// entry of the row map, and every chunk of every row writes its partial output
// and its log2-sum-exp, before the kernels launched after them on the same
// stream read them. So no clearing pass is needed.
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>

#include "../../include/qsa_b200.h"

namespace {

static __device__ __align__(256) unsigned char g_noalloc_scratch[QSA_B200_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;

// Device address of g_noalloc_scratch on the current device, looked up once
// per device with that device current.
void* scratch_address(int* status) {
  static std::atomic<void*> addr[kMaxDevices] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    cudaGetLastError();
    *status = QSA_B200_ERR_DEVICE;
    return nullptr;
  }
  void* a = addr[dev].load(std::memory_order_acquire);
  if (!a) {
    const cudaError_t e = cudaGetSymbolAddress(&a, g_noalloc_scratch);
    if (e != cudaSuccess || !a) {
      cudaGetLastError();
      *status = QSA_B200_ERR_DEVICE;
      return nullptr;
    }
    addr[dev].store(a, std::memory_order_release);
  }
  *status = QSA_B200_OK;
  return a;
}

}  // namespace

extern "C" int qsa_b200_decode_noalloc(const qsa_b200_decode_args* args, qsa_b200_stream_t stream) {
  // validates the arguments (no device call) and sizes the workspace
  const int64_t need = qsa_b200_workspace_bytes(args);
  if (need < 0) return (int)need;
  if (need > (int64_t)QSA_B200_NOALLOC_SCRATCH_BYTES) return QSA_B200_ERR_TOO_LARGE;
  if (args->rows == 0) return QSA_B200_OK;
  int status = QSA_B200_OK;
  void* scratch = scratch_address(&status);
  if (!scratch) return status;
  return qsa_b200_decode(args, scratch, (size_t)QSA_B200_NOALLOC_SCRATCH_BYTES, stream);
}
