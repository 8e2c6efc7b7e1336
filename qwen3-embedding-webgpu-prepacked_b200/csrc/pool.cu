// Last-token L2 pooling: the embedding of a request is its last token's
// hidden row, L2-normalised to f32.
//
// Replaces poolShader / LastTokenPoolKernel (src/webgpu/ops.ts:347-379): the
// reference reads row b*sequence + lengths[b]-1 of a padded batch and scales
// it by inverseSqrt(sum of squares) (no epsilon). Here the row comes either
// from packed cu_seqlens (row cu[b+1]-1) or from the padded layout with the
// reference's device `lengths` buffer.
//
// One CTA per request, 128 threads; each thread owns 16-byte chunks of the
// row (8 halves), the sum of squares is a warp butterfly plus a shared-memory
// combine. A request of length 0 produces a zero vector.
#include "internal.h"

namespace qwa {
namespace {

constexpr int kPoolThreads = 128;

__global__ void __launch_bounds__(kPoolThreads)
    last_token_pool_kernel(const __half* __restrict__ hidden, int width,
                           const int32_t* __restrict__ cu, const uint32_t* __restrict__ lengths,
                           int sequence, float* __restrict__ out) {
  const int b = blockIdx.x;
  int64_t row;
  bool empty;
  if (cu) {
    const int start = cu[b], end = cu[b + 1];
    empty = end <= start;
    row = end - 1;
  } else {
    // lengths > sequence would read the next request's rows (or past the
    // buffer for the last one); clamp to the padded row instead.
    const uint32_t len = min(lengths[b], static_cast<uint32_t>(sequence));
    empty = len == 0;
    row = static_cast<int64_t>(b) * sequence + len - 1;
  }
  float* dst = out + static_cast<int64_t>(b) * width;
  const int chunks = width / 8;
  if (empty) {
    for (int c = threadIdx.x; c < chunks; c += kPoolThreads) {
      reinterpret_cast<float4*>(dst)[2 * c] = make_float4(0.f, 0.f, 0.f, 0.f);
      reinterpret_cast<float4*>(dst)[2 * c + 1] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    return;
  }
  const uint4* src = reinterpret_cast<const uint4*>(hidden + row * width);
  float ss = 0.f;
  for (int c = threadIdx.x; c < chunks; c += kPoolThreads) {
    const uint4 v = __ldg(src + c);
    const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __half22float2(h[e]);
      ss = fmaf(f.x, f.x, fmaf(f.y, f.y, ss));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  __shared__ float partial[kPoolThreads / 32];
  if ((threadIdx.x & 31) == 0) partial[threadIdx.x >> 5] = ss;
  __syncthreads();
  float total = 0.f;
#pragma unroll
  for (int w = 0; w < kPoolThreads / 32; ++w) total += partial[w];
  const float inv = 1.0f / sqrtf(total);
  for (int c = threadIdx.x; c < chunks; c += kPoolThreads) {
    const uint4 v = __ldg(src + c);
    const __half2* h = reinterpret_cast<const __half2*>(&v);
    float r[8];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __half22float2(h[e]);
      r[2 * e] = f.x * inv;
      r[2 * e + 1] = f.y * inv;
    }
    reinterpret_cast<float4*>(dst)[2 * c] = make_float4(r[0], r[1], r[2], r[3]);
    reinterpret_cast<float4*>(dst)[2 * c + 1] = make_float4(r[4], r[5], r[6], r[7]);
  }
}

}  // namespace

cudaError_t launch_last_token_pool(const __half* hidden, int width, const int32_t* cu_seqlens,
                                   const uint32_t* lengths, int sequence, int batch, float* out,
                                   cudaStream_t stream) {
  if (batch <= 0) return cudaSuccess;
  last_token_pool_kernel<<<batch, kPoolThreads, 0, stream>>>(hidden, width, cu_seqlens, lengths,
                                                              sequence, out);
  return cudaGetLastError();
}

}  // namespace qwa
