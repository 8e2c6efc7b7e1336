// Residual add + RMSNorm over rows of the residual stream (HBM-bound).
//
// Replaces rmsNormShader / RmsNormKernel (src/webgpu/ops.ts:21-64). Per row:
//   with residual: v = f32(x) + f32(residual); x = f16(v)   (x updated in place)
//   without:       v = f32(x)
//   inv = 1 / sqrt(sum(v^2) / width + eps)      (sum over the unrounded f32 v)
//   normalized = f16(f32(x) * inv * weight)     (x as stored, i.e. f16-rounded)
//
// Register path (width = 256 * kChunks, kChunks <= 8; Qwen3-0.6B: 1024): one
// warp per row, lane l holds chunks l, l+32, ... of 8 halves (16-byte loads),
// so a row is read once and written once; the sum is a warp butterfly.
// Other widths (multiples of 8): one 256-thread CTA per row, two passes over
// the row (the second pass hits L1/L2).
#include "internal.h"

namespace qwa {
namespace {

constexpr int kRowsPerBlock = 8;  // warps per CTA in the register path

__device__ __forceinline__ void unpack8f(const uint4& v, float (&x)[8]) {
  const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(h[i]);
    x[2 * i] = f.x;
    x[2 * i + 1] = f.y;
  }
}

__device__ __forceinline__ uint4 pack8h(const float (&x)[8]) {
  uint4 r;
  __half2* h = reinterpret_cast<__half2*>(&r);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(x[2 * i], x[2 * i + 1]);
  return r;
}

template <int kChunks, bool kResidual>
__global__ void __launch_bounds__(kRowsPerBlock * 32)
    rms_norm_warp_kernel(__half* __restrict__ x, const __half* __restrict__ residual,
                         const float* __restrict__ weight, __half* __restrict__ normalized,
                         int rows, float eps) {
  constexpr int kWidth = kChunks * 256;
  const int row = blockIdx.x * kRowsPerBlock + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int lane = threadIdx.x & 31;
  uint4* xr = reinterpret_cast<uint4*>(x + static_cast<int64_t>(row) * kWidth);
  const uint4* rr = reinterpret_cast<const uint4*>(residual + static_cast<int64_t>(row) * kWidth);
  uint4 raw[kChunks], res[kChunks];
#pragma unroll
  for (int c = 0; c < kChunks; ++c) raw[c] = xr[lane + 32 * c];
  if constexpr (kResidual) {
#pragma unroll
    for (int c = 0; c < kChunks; ++c) res[c] = __ldcs(rr + lane + 32 * c);
  }
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < kChunks; ++c) {
    float v[8];
    unpack8f(raw[c], v);
    if constexpr (kResidual) {
      float r[8];
      unpack8f(res[c], r);
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] += r[e];
      raw[c] = pack8h(v);  // x = f16(x + residual)
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) ss = fmaf(v[e], v[e], ss);
  }
  if constexpr (kResidual) {
#pragma unroll
    for (int c = 0; c < kChunks; ++c) xr[lane + 32 * c] = raw[c];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float inv = 1.0f / sqrtf(ss * (1.0f / kWidth) + eps);
  uint4* nr = reinterpret_cast<uint4*>(normalized + static_cast<int64_t>(row) * kWidth);
#pragma unroll
  for (int c = 0; c < kChunks; ++c) {
    const int col = (lane + 32 * c) * 8;
    const float4 w0 = __ldg(reinterpret_cast<const float4*>(weight + col));
    const float4 w1 = __ldg(reinterpret_cast<const float4*>(weight + col) + 1);
    const float w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
    float v[8];
    unpack8f(raw[c], v);
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = v[e] * inv * w[e];
    __stcs(nr + lane + 32 * c, pack8h(v));
  }
}

constexpr int kRowThreads = 256;

__global__ void __launch_bounds__(kRowThreads)
    rms_norm_row_kernel(__half* __restrict__ x, const __half* __restrict__ residual,
                        const float* __restrict__ weight, __half* __restrict__ normalized,
                        int width, int has_residual, float eps) {
  const int64_t base = static_cast<int64_t>(blockIdx.x) * width;
  uint4* xr = reinterpret_cast<uint4*>(x + base);
  const uint4* rr = reinterpret_cast<const uint4*>(residual + base);
  const int chunks = width / 8;
  float ss = 0.f;
  for (int c = threadIdx.x; c < chunks; c += kRowThreads) {
    float v[8];
    uint4 raw = xr[c];
    unpack8f(raw, v);
    if (has_residual) {
      float r[8];
      unpack8f(rr[c], r);
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] += r[e];
      xr[c] = pack8h(v);
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) ss = fmaf(v[e], v[e], ss);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  __shared__ float partial[kRowThreads / 32];
  if ((threadIdx.x & 31) == 0) partial[threadIdx.x >> 5] = ss;
  __syncthreads();
  float total = 0.f;
#pragma unroll
  for (int w = 0; w < kRowThreads / 32; ++w) total += partial[w];
  const float inv = 1.0f / sqrtf(total / width + eps);
  uint4* nr = reinterpret_cast<uint4*>(normalized + base);
  for (int c = threadIdx.x; c < chunks; c += kRowThreads) {
    float v[8];
    unpack8f(xr[c], v);
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = v[e] * inv * __ldg(weight + c * 8 + e);
    nr[c] = pack8h(v);
  }
}

template <int kChunks>
cudaError_t launch_warp(__half* x, const __half* residual, const float* weight,
                        __half* normalized, int rows, bool has_residual, float eps,
                        cudaStream_t stream) {
  const int blocks = (rows + kRowsPerBlock - 1) / kRowsPerBlock;
  if (has_residual)
    rms_norm_warp_kernel<kChunks, true>
        <<<blocks, kRowsPerBlock * 32, 0, stream>>>(x, residual, weight, normalized, rows, eps);
  else
    rms_norm_warp_kernel<kChunks, false>
        <<<blocks, kRowsPerBlock * 32, 0, stream>>>(x, residual, weight, normalized, rows, eps);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_rms_norm(__half* x, const __half* residual, const float* weight,
                            __half* normalized, int rows, int width, bool has_residual, float eps,
                            cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  if (width % 256 == 0) {
    switch (width / 256) {
      case 1: return launch_warp<1>(x, residual, weight, normalized, rows, has_residual, eps, stream);
      case 2: return launch_warp<2>(x, residual, weight, normalized, rows, has_residual, eps, stream);
      case 4: return launch_warp<4>(x, residual, weight, normalized, rows, has_residual, eps, stream);
      case 8: return launch_warp<8>(x, residual, weight, normalized, rows, has_residual, eps, stream);
      default: break;
    }
  }
  rms_norm_row_kernel<<<rows, kRowThreads, 0, stream>>>(x, residual, weight, normalized, width,
                                                        has_residual ? 1 : 0, eps);
  return cudaGetLastError();
}

}  // namespace qwa
