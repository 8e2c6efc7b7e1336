// Fused per-head Q/K RMSNorm + RoPE prologue (HBM-bound).
//
// Replaces qkNormRopeShader (src/webgpu/ops.ts:104-150): for each token and
// each of 16 q-heads + 8 k-heads, n = x / sqrt(mean(x^2) + eps) * w, then the
// NEOX half rotation out[d] = n[d]*cos + (d<64 ? -n[d+64] : n[d-64])*sin with
// (cos, sin) = table[pos*64 + d%64].
//
// One warp per token: the token's 24 heads (16 q + 8 k) are 24 consecutive
// 256-byte rows of qkv, so lane l issues all 12 of its 16-byte loads before
// any math (half-warp per head per load: lanes 0-15 head 2i, 16-31 head 2i+1,
// eight dims per lane). The per-head sum of squares is a 16-lane butterfly and
// the RoPE partner d +/- 64 is lane l ^ 8. The token's position, its cos/sin
// row and both weight vectors are read once per warp.
#include "internal.h"

namespace qwa {
namespace {

// Occupancy sets the bytes in flight, and so the bandwidth: 64-thread
// blocks with at least 10 resident per SM cap a thread at 96 registers (no
// spills) for 20 warps per SM, each with a token's 6 KB of loads in flight.
// Measured on 80,000 tokens: 6.16 TB/s, against 5.25 TB/s with 256-thread
// blocks (99 registers, 16 warps, a quarter of the register file idle).
#ifndef QWA_PRO_WPB
#define QWA_PRO_WPB 2
#endif
constexpr int kWarpsPerBlock = QWA_PRO_WPB;
#ifndef QWA_PRO_MINB
#define QWA_PRO_MINB 10
#endif
constexpr int kHeads = kQHeads + kKVHeads;  // 24
constexpr int kLoads = kHeads / 2;          // 12

__device__ __forceinline__ int position_in_request(const int32_t* cu, int batch, int t) {
  int lo = 0, hi = batch - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (__ldg(cu + mid) <= t) lo = mid;
    else hi = mid - 1;
  }
  return t - __ldg(cu + lo);
}

__device__ __forceinline__ void unpack8(const uint4& v, float (&x)[8]) {
  const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(h[i]);
    x[2 * i] = f.x;
    x[2 * i + 1] = f.y;
  }
}

__global__ void __launch_bounds__(kWarpsPerBlock * 32, QWA_PRO_MINB)
    qk_norm_rope_kernel(const __half* __restrict__ qkv, int64_t stride,
                        const float* __restrict__ q_weight, const float* __restrict__ k_weight,
                        const float2* __restrict__ table, __half* __restrict__ q_out,
                        __half* __restrict__ k_out, const int32_t* __restrict__ cu, int batch,
                        int tokens, int padded_sequence, float eps) {
  const int t = blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5);
  if (t >= tokens) return;
  const int lane = threadIdx.x & 31;
  const int half = lane >> 4;  // which head of the pair
  const int sub = lane & 15;   // dims 8*sub .. 8*sub+7

  // issue every load of the token first
  const uint4* src = reinterpret_cast<const uint4*>(qkv + static_cast<int64_t>(t) * stride) +
                     half * 16 + sub;
  uint4 raw[kLoads];
#pragma unroll
  for (int i = 0; i < kLoads; ++i) raw[i] = __ldcs(src + i * 32);
  const int pos = padded_sequence > 0 ? t % padded_sequence : position_in_request(cu, batch, t);
  const float4* wq = reinterpret_cast<const float4*>(q_weight + sub * 8);
  const float4* wk = reinterpret_cast<const float4*>(k_weight + sub * 8);
  const float4 wq0 = __ldg(wq), wq1 = __ldg(wq + 1), wk0 = __ldg(wk), wk1 = __ldg(wk + 1);
  const float4* tp =
      reinterpret_cast<const float4*>(table + static_cast<int64_t>(pos) * 64 + (sub & 7) * 8);
  float c[8], sn[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float4 v = __ldg(tp + i);  // (cos, sin) of two consecutive dims
    c[2 * i] = v.x;
    sn[2 * i] = v.y;
    c[2 * i + 1] = v.z;
    sn[2 * i + 1] = v.w;
  }
  const float wqa[8] = {wq0.x, wq0.y, wq0.z, wq0.w, wq1.x, wq1.y, wq1.z, wq1.w};
  const float wka[8] = {wk0.x, wk0.y, wk0.z, wk0.w, wk1.x, wk1.y, wk1.z, wk1.w};
  const float sign = sub < 8 ? -1.f : 1.f;  // d < 64 takes -x[d+64]

#pragma unroll
  for (int i = 0; i < kLoads; ++i) {
    const int head = 2 * i + half;  // 0..15 q heads, 16..23 k heads
    const bool is_q = i < kQHeads / 2;
    float x[8];
    unpack8(raw[i], x);
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) ss = fmaf(x[e], x[e], ss);
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float inv = 1.0f / sqrtf(ss * (1.0f / kHeadDim) + eps);
    float n[8], r[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) n[e] = x[e] * inv * (is_q ? wqa[e] : wka[e]);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float partner = __shfl_xor_sync(0xffffffffu, n[e], 8);
      r[e] = fmaf(n[e], c[e], sign * partner * sn[e]);
    }
    uint4 packed;
    __half2* ph = reinterpret_cast<__half2*>(&packed);
#pragma unroll
    for (int e = 0; e < 4; ++e) ph[e] = __floats2half2_rn(r[2 * e], r[2 * e + 1]);
    __half* dst = is_q ? q_out + (static_cast<int64_t>(t) * kQHeads + head) * kHeadDim
                       : k_out + (static_cast<int64_t>(t) * kKVHeads + head - kQHeads) * kHeadDim;
    reinterpret_cast<uint4*>(dst)[sub] = packed;
  }
}

}  // namespace

cudaError_t launch_qk_norm_rope(const __half* qkv, int64_t qkv_stride, const float* q_weight,
                                const float* k_weight, const float2* rope_table, __half* q_out,
                                __half* k_out, const int32_t* cu_seqlens, int batch, int tokens,
                                int padded_sequence, float eps, cudaStream_t stream) {
  if (tokens <= 0) return cudaSuccess;
  const int blocks = (tokens + kWarpsPerBlock - 1) / kWarpsPerBlock;
  qk_norm_rope_kernel<<<blocks, kWarpsPerBlock * 32, 0, stream>>>(
      qkv, qkv_stride, q_weight, k_weight, rope_table, q_out, k_out, cu_seqlens, batch, tokens,
      padded_sequence, eps);
  return cudaGetLastError();
}

}  // namespace qwa
