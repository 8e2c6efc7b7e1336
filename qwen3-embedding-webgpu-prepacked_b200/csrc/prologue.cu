// Fused per-head Q/K RMSNorm + RoPE prologue (HBM-bound).
//
// Replaces qkNormRopeShader (src/webgpu/ops.ts:104-150): for each token and
// each of 16 q-heads + 8 k-heads, n = x / sqrt(mean(x^2) + eps) * w, then the
// NEOX half rotation out[d] = n[d]*cos + (d<64 ? -n[d+64] : n[d-64])*sin with
// (cos, sin) = table[pos*64 + d%64].
//
// One warp per (token, head): lane l owns dims 4l..4l+3 (one 8-byte load and
// store per lane, 256 contiguous bytes per warp), the sum of squares is a
// warp butterfly, and the RoPE partner d +/- 64 lives in lane l ^ 16.
#include "internal.h"

namespace qwa {
namespace {

constexpr int kWarpsPerBlock = 8;

__device__ __forceinline__ int position_in_request(const int32_t* cu, int batch, int t) {
  int lo = 0, hi = batch - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (__ldg(cu + mid) <= t) lo = mid;
    else hi = mid - 1;
  }
  return t - __ldg(cu + lo);
}

__global__ void __launch_bounds__(kWarpsPerBlock * 32)
    qk_norm_rope_kernel(const __half* __restrict__ qkv, int64_t stride,
                        const float* __restrict__ q_weight, const float* __restrict__ k_weight,
                        const float2* __restrict__ table, __half* __restrict__ q_out,
                        __half* __restrict__ k_out, const int32_t* __restrict__ cu, int batch,
                        int tokens, int padded_sequence, float eps) {
  const int64_t item = static_cast<int64_t>(blockIdx.x) * kWarpsPerBlock + (threadIdx.x >> 5);
  if (item >= static_cast<int64_t>(tokens) * (kQHeads + kKVHeads)) return;
  const int lane = threadIdx.x & 31;
  const int t = static_cast<int>(item / (kQHeads + kKVHeads));
  const int ch = static_cast<int>(item % (kQHeads + kKVHeads));
  const bool is_q = ch < kQHeads;
  const int h = is_q ? ch : ch - kQHeads;
  const int pos = padded_sequence > 0 ? t % padded_sequence : position_in_request(cu, batch, t);

  const __half* src = qkv + static_cast<int64_t>(t) * stride + (is_q ? 0 : kQHeads * kHeadDim) +
                      h * kHeadDim + lane * 4;
  const uint2 raw = __ldg(reinterpret_cast<const uint2*>(src));
  const float2 lo = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
  const float2 hi = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
  float x[4] = {lo.x, lo.y, hi.x, hi.y};

  float ss = x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float inv = 1.0f / sqrtf(ss * (1.0f / kHeadDim) + eps);

  const float4 w = __ldg(reinterpret_cast<const float4*>((is_q ? q_weight : k_weight) + lane * 4));
  const float n[4] = {x[0] * inv * w.x, x[1] * inv * w.y, x[2] * inv * w.z, x[3] * inv * w.w};
  float partner[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) partner[i] = __shfl_xor_sync(0xffffffffu, n[i], 16);
  const float sign = lane < 16 ? -1.f : 1.f;

  const int rd = (lane & 15) * 4;  // d % 64
  const float4* tp = reinterpret_cast<const float4*>(table + static_cast<int64_t>(pos) * 64 + rd);
  const float4 cs01 = __ldg(tp), cs23 = __ldg(tp + 1);
  const float c[4] = {cs01.x, cs01.z, cs23.x, cs23.z};
  const float s[4] = {cs01.y, cs01.w, cs23.y, cs23.w};
  float r[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) r[i] = n[i] * c[i] + sign * partner[i] * s[i];

  __half2 o01 = __floats2half2_rn(r[0], r[1]);
  __half2 o23 = __floats2half2_rn(r[2], r[3]);
  uint2 packed;
  packed.x = *reinterpret_cast<uint32_t*>(&o01);
  packed.y = *reinterpret_cast<uint32_t*>(&o23);
  __half* dst = is_q ? q_out + (static_cast<int64_t>(t) * kQHeads + h) * kHeadDim
                     : k_out + (static_cast<int64_t>(t) * kKVHeads + h) * kHeadDim;
  *reinterpret_cast<uint2*>(dst + lane * 4) = packed;
}

}  // namespace

cudaError_t launch_qk_norm_rope(const __half* qkv, int64_t qkv_stride, const float* q_weight,
                                const float* k_weight, const float2* rope_table, __half* q_out,
                                __half* k_out, const int32_t* cu_seqlens, int batch, int tokens,
                                int padded_sequence, float eps, cudaStream_t stream) {
  if (tokens <= 0) return cudaSuccess;
  const int64_t items = static_cast<int64_t>(tokens) * (kQHeads + kKVHeads);
  const int64_t blocks = (items + kWarpsPerBlock - 1) / kWarpsPerBlock;
  qk_norm_rope_kernel<<<static_cast<unsigned>(blocks), kWarpsPerBlock * 32, 0, stream>>>(
      qkv, qkv_stride, q_weight, k_weight, rope_table, q_out, k_out, cu_seqlens, batch, tokens,
      padded_sequence, eps);
  return cudaGetLastError();
}

}  // namespace qwa
