// Paged FP8 K/V cache writer: new keys and values of some tokens, quantised
// to E4M3FN and stored at the tokens' physical slots of the
// [num_pages, P, Hkv, 128] caches the decode reads.
//
// The reference produces its caches with (randn * 0.1).to(float8_e4m3fn) in
// this layout and hands the scales over beside them (sm89_cutedsl.py:48-62,
// :79). Here the producer is a kernel: cache = e4m3fn(x * inv_scale), with
// inv_scale = 1 / scale rounded to fp32 once on the host, an fp32 product
// and the conversion round-to-nearest-even with saturation at +-448
// (torch's cast turns |x| >= 464 into NaN). (An IEEE division per element
// instead of the product halves the bandwidth.)
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

#include <type_traits>

#include "../../include/qsa_b200.h"
#include "qsa_common.cuh"
#include "qsa_internal.h"

namespace qsa {
namespace {

constexpr int kCwThreads = 256;
constexpr int kCwPerRow = 16;  // threads per 128-element row, 8 elements each
constexpr int kCwMinBlocks = 4;  // resident blocks per SM (register cap)
// row pieces per thread and pass: all their loads are in flight together
template <typename T>
__host__ __device__ constexpr int cw_unroll() {
  return sizeof(T) == 4 ? 2 : 4;
}

// 8 consecutive input elements: the raw 16 (or 32, fp32) bytes, loaded
// before any conversion so the loads of several pieces overlap
struct Raw8 {
  uint4 a, b;
};
template <typename T>
__device__ __forceinline__ void load8(const void* base, int64_t off, Raw8& r) {
  const uint4* p = reinterpret_cast<const uint4*>(static_cast<const T*>(base) + off);
  r.a = __ldg(p);
  if (sizeof(T) == 4) r.b = __ldg(p + 1);
}
template <typename T>
__device__ __forceinline__ void widen8(const Raw8& r, float (&x)[8]) {
  if constexpr (sizeof(T) == 4) {
    const uint32_t w[8] = {r.a.x, r.a.y, r.a.z, r.a.w, r.b.x, r.b.y, r.b.z, r.b.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) x[i] = __uint_as_float(w[i]);
  } else {
    const uint32_t w[4] = {r.a.x, r.a.y, r.a.z, r.a.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 f;
      if constexpr (std::is_same<T, __nv_bfloat16>::value)
        f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
      else
        f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
      x[2 * i] = f.x;
      x[2 * i + 1] = f.y;
    }
  }
}

// 8 values * inv_scale -> 8 E4M3FN bytes (round to nearest even, saturating)
template <typename T>
__device__ __forceinline__ uint2 quantise8(const Raw8& r, float inv_scale) {
  float x[8];
  widen8<T>(r, x);
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = make_float2(x[2 * i] * inv_scale, x[2 * i + 1] * inv_scale);
    w[i] = (uint32_t)__nv_cvt_float2_to_fp8x2(f, __NV_SATFINITE, __NV_E4M3);
  }
  return make_uint2(w[0] | (w[1] << 16), w[2] | (w[3] << 16));
}

template <typename T>
__global__ void __launch_bounds__(kCwThreads, kCwMinBlocks) qsa_cache_write_kernel(const CacheWriteParams p) {
  constexpr int kCwUnroll = cw_unroll<T>();
  const int64_t total = (int64_t)p.tokens * p.num_kv_heads * kCwPerRow;
  const int64_t cache_slots = p.num_pages * p.page_size;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  // kCwUnroll row pieces per thread and pass, all loads issued before the
  // first conversion, so that each thread keeps 2 * kCwUnroll 16-byte loads
  // in flight
  for (int64_t i0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i0 < total; i0 += stride * kCwUnroll) {
    Raw8 rk[kCwUnroll], rv[kCwUnroll];
    int64_t slot[kCwUnroll], dst[kCwUnroll];
    // the loads do not depend on the slot (which only places the stores), so
    // all of them leave together
#pragma unroll
    for (int u = 0; u < kCwUnroll; ++u) {
      const int64_t i = i0 + u * stride;
      slot[u] = -1;
      dst[u] = 0;
      if (i >= total) continue;
      const int part = (int)(i % kCwPerRow);
      const int64_t row = i / kCwPerRow;
      const int g = (int)(row % p.num_kv_heads);
      const int64_t t = row / p.num_kv_heads;
      slot[u] = __ldg(p.slots + t);
      const int64_t src = t * p.token_stride + (int64_t)g * kHeadDim + part * 8;
      dst[u] = (int64_t)g * kHeadDim + part * 8;
      load8<T>(p.k, src, rk[u]);
      load8<T>(p.v, src, rv[u]);
    }
#pragma unroll
    for (int u = 0; u < kCwUnroll; ++u) {
      if (slot[u] < 0 || slot[u] >= cache_slots) continue;
      const int64_t d = slot[u] * p.num_kv_heads * kHeadDim + dst[u];
      *reinterpret_cast<uint2*>(p.k_cache + d) = quantise8<T>(rk[u], p.k_inv_scale);
      *reinterpret_cast<uint2*>(p.v_cache + d) = quantise8<T>(rv[u], p.v_inv_scale);
    }
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
  // kCwMinBlocks resident blocks of 256 threads per SM, striding over the rest
  static int sms = sm_count_cw();
  const int unroll = p.dtype == QSA_B200_DTYPE_F32 ? cw_unroll<float>() : cw_unroll<__half>();
  const int64_t want = (threads + (int64_t)kCwThreads * unroll - 1) / ((int64_t)kCwThreads * unroll);
  const int grid = (int)(want < (int64_t)sms * kCwMinBlocks ? want : (int64_t)sms * kCwMinBlocks);
  switch (p.dtype) {
    case QSA_B200_DTYPE_BF16: qsa_cache_write_kernel<__nv_bfloat16><<<grid, kCwThreads, 0, stream>>>(p); break;
    case QSA_B200_DTYPE_F16: qsa_cache_write_kernel<__half><<<grid, kCwThreads, 0, stream>>>(p); break;
    case QSA_B200_DTYPE_F32: qsa_cache_write_kernel<float><<<grid, kCwThreads, 0, stream>>>(p); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace qsa
