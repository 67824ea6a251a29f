// Paged FP8 K/V cache writer: new keys and values of some tokens, quantised
// to E4M3FN and stored at the tokens' physical slots of the
// [num_pages, P, Hkv, 128] caches the decode reads.
//
// The reference produces its caches with (randn * 0.1).to(float8_e4m3fn) in
// this layout and hands the scales over beside them (sm89_cutedsl.py:48-62,
// :79). Here the producer is a kernel: cache = e4m3fn(x / scale), the
// division an IEEE fp32 division and the conversion round-to-nearest-even
// with saturation at +-448 (torch's cast turns |x| >= 464 into NaN).
//
// One thread quantises 8 consecutive elements of one (token, KV head) row of
// both K and V: 16 threads per 128-element row, so a half warp reads the
// row's 256 bytes (bf16) and writes its 128 bytes with full-line accesses.
// The kernel is HBM-bound: 2 x (128 x input size + 128) bytes per row. The
// grid strides over the rows; a row whose slot is negative or past the
// cache is skipped.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

#include "../../include/qsa_b200.h"
#include "qsa_common.cuh"
#include "qsa_internal.h"

namespace qsa {
namespace {

constexpr int kCwThreads = 256;
constexpr int kCwPerRow = 16;  // threads per 128-element row, 8 elements each

template <typename T>
struct Load8;
template <>
struct Load8<__nv_bfloat16> {
  __device__ static void run(const void* base, int64_t off, float (&x)[8]) {
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(base) + off));
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
      x[2 * i] = f.x;
      x[2 * i + 1] = f.y;
    }
  }
};
template <>
struct Load8<__half> {
  __device__ static void run(const void* base, int64_t off, float (&x)[8]) {
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(static_cast<const __half*>(base) + off));
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
      x[2 * i] = f.x;
      x[2 * i + 1] = f.y;
    }
  }
};
template <>
struct Load8<float> {
  __device__ static void run(const void* base, int64_t off, float (&x)[8]) {
    const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(base) + off);
    const float4 a = __ldg(p), b = __ldg(p + 1);
    x[0] = a.x, x[1] = a.y, x[2] = a.z, x[3] = a.w;
    x[4] = b.x, x[5] = b.y, x[6] = b.z, x[7] = b.w;
  }
};

// 8 values / scale -> 8 E4M3FN bytes (round to nearest even, saturating)
__device__ __forceinline__ uint2 quantise8(const float (&x)[8], float scale) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = make_float2(__fdiv_rn(x[2 * i], scale), __fdiv_rn(x[2 * i + 1], scale));
    w[i] = (uint32_t)__nv_cvt_float2_to_fp8x2(f, __NV_SATFINITE, __NV_E4M3);
  }
  return make_uint2(w[0] | (w[1] << 16), w[2] | (w[3] << 16));
}

template <typename T>
__global__ void __launch_bounds__(kCwThreads) qsa_cache_write_kernel(const CacheWriteParams p) {
  const int64_t total = (int64_t)p.tokens * p.num_kv_heads * kCwPerRow;
  const int64_t cache_slots = p.num_pages * p.page_size;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int part = (int)(i % kCwPerRow);
    const int64_t row = i / kCwPerRow;
    const int g = (int)(row % p.num_kv_heads);
    const int64_t t = row / p.num_kv_heads;
    const int64_t slot = __ldg(p.slots + t);
    if (slot < 0 || slot >= cache_slots) continue;
    const int64_t src = t * p.token_stride + (int64_t)g * kHeadDim + part * 8;
    const int64_t dst = (slot * p.num_kv_heads + g) * kHeadDim + part * 8;
    float xk[8], xv[8];
    Load8<T>::run(p.k, src, xk);
    Load8<T>::run(p.v, src, xv);
    *reinterpret_cast<uint2*>(p.k_cache + dst) = quantise8(xk, p.k_scale);
    *reinterpret_cast<uint2*>(p.v_cache + dst) = quantise8(xv, p.v_scale);
  }
}

int sm_count_cw() {
  int dev = 0, c = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&c, cudaDevAttrMultiProcessorCount, dev);
  return c > 0 ? c : 148;
}

}  // namespace

cudaError_t launch_cache_write(const CacheWriteParams& p, cudaStream_t stream) {
  const int64_t threads = (int64_t)p.tokens * p.num_kv_heads * kCwPerRow;
  if (threads <= 0) return cudaSuccess;
  // up to 8 resident blocks of 256 threads per SM, striding over the rest
  static int sms = sm_count_cw();
  const int64_t want = (threads + kCwThreads - 1) / kCwThreads;
  const int grid = (int)(want < (int64_t)sms * 8 ? want : (int64_t)sms * 8);
  switch (p.dtype) {
    case QSA_B200_DTYPE_BF16: qsa_cache_write_kernel<__nv_bfloat16><<<grid, kCwThreads, 0, stream>>>(p); break;
    case QSA_B200_DTYPE_F16: qsa_cache_write_kernel<__half><<<grid, kCwThreads, 0, stream>>>(p); break;
    case QSA_B200_DTYPE_F32: qsa_cache_write_kernel<float><<<grid, kCwThreads, 0, stream>>>(p); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace qsa
