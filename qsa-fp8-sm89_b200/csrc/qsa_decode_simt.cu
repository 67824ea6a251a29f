// General-shape decode kernel (CUDA cores), plus the slot and combine kernels.
//
// qsa_decode_simt_kernel covers every GQA group size (the tensor-core kernel
// in qsa_decode_tc.cu handles group sizes 1-8, 10, 12, 14 and 16). One CTA serves
// one (row, KV head, chunk) with one warp per query head of the group; lane l
// owns dims 4l..4l+3. Tokens go in 32-token tiles: lane j decodes token j of
// the tile, every lane forms its 4-dim partial dot product for all 32 tokens
// and a 31-shuffle transpose-reduction leaves token j's score on lane j, so the
// online softmax runs once per tile rather than once per token.
#include "qsa_common.cuh"

namespace qsa {
namespace {

// Query heads (warps) per CTA; larger groups spread over gridDim.z.
constexpr int kSimtHeadsPerBlock = 8;

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// part[i] is this lane's contribution to token i. Returns, on lane j, the sum
// over all lanes of part[j] (recursive halving: 16+8+4+2+1 shuffles).
__device__ __forceinline__ float transpose_reduce(float (&part)[32], int lane) {
#pragma unroll
  for (int s = 16; s >= 1; s >>= 1) {
    const bool upper = (lane & s) != 0;
#pragma unroll
    for (int k = 0; k < s; ++k) {
      const float send = upper ? part[k] : part[k + s];
      const float keep = upper ? part[k + s] : part[k];
      part[k] = keep + __shfl_xor_sync(0xffffffffu, send, s);
    }
  }
  return part[0];
}

__device__ __forceinline__ void fp8x4_to_f32(uint32_t w, float (&f)[4]) {
  const float2 lo = e4m3x2_to_f32x2((uint16_t)(w & 0xffffu));
  const float2 hi = e4m3x2_to_f32x2((uint16_t)(w >> 16));
  f[0] = lo.x; f[1] = lo.y; f[2] = hi.x; f[3] = hi.y;
}

__device__ __forceinline__ void bf16x4_to_f32(const __nv_bfloat16* src, float (&f)[4]) {
  const uint2 raw = *reinterpret_cast<const uint2*>(src);
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.x));
  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.y));
  f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y;
}

__device__ __forceinline__ float sigmoidf_(float x) { return 1.0f / (1.0f + expf(-x)); }

__global__ void qsa_decode_simt_kernel(DecodeParams p) {
  const int g = blockIdx.x % p.num_kv_heads;
  const int row = blockIdx.x / p.num_kv_heads;
  const int chunk = blockIdx.y;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int hg = blockIdx.z * kSimtHeadsPerBlock + warp;  // head within the group
  if (hg >= p.group) return;                               // warp-uniform
  const int h = g * p.group + hg;

  const int64_t req = row_request(p, row);
  const int count = row_count(p, row);
  const int c0 = chunk * p.chunk_tokens;
  const int c1 = min(c0 + p.chunk_tokens, p.topk);

  const int64_t qoff = ((int64_t)row * p.num_q_heads + h) * kHeadDim + lane * 4;
  float q[4];
  bf16x4_to_f32(p.q + qoff, q);
#pragma unroll
  for (int i = 0; i < 4; ++i) q[i] *= p.score_scale_log2;

  float m = -INFINITY, l = 0.f;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int base = c0; base < c1; base += 32) {
    const int col = base + lane;
    const int64_t slot = (col < c1) ? token_slot(p, row, req, count, col) : -1;
    const long long off = slot >= 0 ? (long long)(slot * p.num_kv_heads + g) * kHeadDim : -1ll;
    float part[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const long long o = __shfl_sync(0xffffffffu, off, i);
      float dot = 0.f;
      if (o >= 0) {
        float kf[4];
        fp8x4_to_f32(__ldg(reinterpret_cast<const uint32_t*>(p.k + o + lane * 4)), kf);
        dot = q[0] * kf[0] + q[1] * kf[1] + q[2] * kf[2] + q[3] * kf[3];
      }
      part[i] = dot;
    }
    float s = transpose_reduce(part, lane);
    const bool valid = off >= 0;
    s = valid ? s : -INFINITY;
    const float m_new = fmaxf(m, warp_max(s));
    if (m_new == -INFINITY) continue;  // nothing valid yet (warp-uniform)
    const float alpha = exp2f(m - m_new);
    const float pj = valid ? exp2f(s - m_new) : 0.f;
    l = l * alpha + warp_sum(pj);
#pragma unroll
    for (int d = 0; d < 4; ++d) acc[d] *= alpha;
#pragma unroll 8
    for (int i = 0; i < 32; ++i) {
      const long long o = __shfl_sync(0xffffffffu, off, i);
      const float pi = __shfl_sync(0xffffffffu, pj, i);
      if (o >= 0) {
        float vf[4];
        fp8x4_to_f32(__ldg(reinterpret_cast<const uint32_t*>(p.v + o + lane * 4)), vf);
#pragma unroll
        for (int d = 0; d < 4; ++d) acc[d] = fmaf(pi, vf[d], acc[d]);
      }
    }
    m = m_new;
  }

  const float inv_l = l > 0.f ? 1.0f / l : 0.f;
  if (p.num_chunks == 1) {
    float gt[4];
    bf16x4_to_f32(p.gate + qoff, gt);
    const float sc = inv_l * p.v_scale;
    __nv_bfloat162 lo = __floats2bfloat162_rn(acc[0] * sc * sigmoidf_(gt[0]), acc[1] * sc * sigmoidf_(gt[1]));
    __nv_bfloat162 hi = __floats2bfloat162_rn(acc[2] * sc * sigmoidf_(gt[2]), acc[3] * sc * sigmoidf_(gt[3]));
    uint2 o;
    o.x = *reinterpret_cast<uint32_t*>(&lo);
    o.y = *reinterpret_cast<uint32_t*>(&hi);
    *reinterpret_cast<uint2*>(p.out + qoff) = o;
  } else {
    const int64_t pidx = ((int64_t)row * p.num_q_heads + h) * p.num_chunks + chunk;
    float4 o = make_float4(acc[0] * inv_l, acc[1] * inv_l, acc[2] * inv_l, acc[3] * inv_l);
    *reinterpret_cast<float4*>(p.part_o + pidx * kHeadDim + lane * 4) = o;
    if (lane == 0) p.part_lse[pidx] = l > 0.f ? m + log2f(l) : -INFINITY;
  }
}

// Merge the per-chunk partial results of one (row, query head): the
// flash-decoding combine, in the log2 domain of the kernels' softmax.
// One warp per (row, query head), lane l owning dims 4l .. 4l+3: the chunk
// partials merge by their log2-sum-exp2 weights (flash-decoding), then the
// gate and v_scale. Every chunk's partial loads leave before the first
// weighted sum, so the kernel streams at HBM rate.
constexpr int kCombineWarps = 8;
__global__ void __launch_bounds__(32 * kCombineWarps) qsa_combine_kernel(DecodeParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t hr = (int64_t)blockIdx.x * kCombineWarps + (threadIdx.x >> 5);  // row * Hq + head
  if (hr >= (int64_t)p.rows * p.num_q_heads) return;
  const int64_t base = hr * p.num_chunks;
  const float* lse = p.part_lse + base;
  const float4* po = reinterpret_cast<const float4*>(p.part_o + base * kHeadDim) + lane;
  float mx = -INFINITY;
  for (int c = 0; c < p.num_chunks; ++c) mx = fmaxf(mx, __ldg(lse + c));
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  float wsum = 0.f;
  if (mx != -INFINITY) {
#pragma unroll 4
    for (int c = 0; c < p.num_chunks; ++c) {
      const float l = __ldg(lse + c);
      // an empty chunk (log-sum -inf) may have no partial output written
      if (l == -INFINITY) continue;
      const float4 v = __ldg(po + c * (kHeadDim / 4));
      const float w = exp2f(l - mx);
      wsum += w;
      acc.x = fmaf(w, v.x, acc.x);
      acc.y = fmaf(w, v.y, acc.y);
      acc.z = fmaf(w, v.z, acc.z);
      acc.w = fmaf(w, v.w, acc.w);
    }
    const float inv = 1.0f / wsum;
    acc.x *= inv, acc.y *= inv, acc.z *= inv, acc.w *= inv;
  }
  const int64_t off = hr * kHeadDim + lane * 4;
  const uint2 gu = __ldg(reinterpret_cast<const uint2*>(p.gate + off));
  const float2 g01 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&gu.x));
  const float2 g23 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&gu.y));
  const __nv_bfloat162 o01 = __floats2bfloat162_rn(acc.x * p.v_scale * sigmoidf_(g01.x),
                                                   acc.y * p.v_scale * sigmoidf_(g01.y));
  const __nv_bfloat162 o23 = __floats2bfloat162_rn(acc.z * p.v_scale * sigmoidf_(g23.x),
                                                   acc.w * p.v_scale * sigmoidf_(g23.y));
  uint2 ou;
  ou.x = *reinterpret_cast<const uint32_t*>(&o01);
  ou.y = *reinterpret_cast<const uint32_t*>(&o23);
  *reinterpret_cast<uint2*>(p.out + off) = ou;
}

// Physical slot of every Top-K entry (-1 where masked): the bit-exact view of
// the index decode that every kernel runs.
__global__ void qsa_slots_kernel(DecodeParams p, int64_t* slots) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)p.rows * p.topk) return;
  const int row = (int)(i / p.topk);
  const int col = (int)(i - (int64_t)row * p.topk);
  slots[i] = token_slot(p, row, row_request(p, row), row_count(p, row), col);
}

}  // namespace

cudaError_t launch_decode_simt(const DecodeParams& p, cudaStream_t stream) {
  const int heads = p.group < kSimtHeadsPerBlock ? p.group : kSimtHeadsPerBlock;
  dim3 grid((unsigned)(p.rows * p.num_kv_heads), (unsigned)p.num_chunks,
            (unsigned)((p.group + kSimtHeadsPerBlock - 1) / kSimtHeadsPerBlock));
  dim3 block((unsigned)(32 * heads), 1, 1);
  qsa_decode_simt_kernel<<<grid, block, 0, stream>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_combine(const DecodeParams& p, cudaStream_t stream) {
  const int64_t warps = (int64_t)p.rows * p.num_q_heads;
  qsa_combine_kernel<<<(unsigned)((warps + kCombineWarps - 1) / kCombineWarps), 32 * kCombineWarps, 0, stream>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_slots(const DecodeParams& p, int64_t* slots, cudaStream_t stream) {
  const int64_t n = (int64_t)p.rows * p.topk;
  if (n == 0) return cudaSuccess;
  const int threads = 256;
  qsa_slots_kernel<<<(unsigned)((n + threads - 1) / threads), threads, 0, stream>>>(p, slots);
  return cudaGetLastError();
}

}  // namespace qsa
