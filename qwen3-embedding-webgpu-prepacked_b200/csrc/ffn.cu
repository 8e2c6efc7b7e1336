// The two element-wise kernels around the model's projections (HBM-bound):
//
// * SwiGLU of the FFN (swigluShader / SwiGLUKernel, src/webgpu/ops.ts:74-102):
//     g = f32(combined[r, c]), u = f32(combined[r, width + c])
//     out[r, c] = f16(silu(g) * u),  silu(g) = g / (1 + exp(-g)) in f32
//   with the fast exponential and division (silu in internal.h)
//   combined is the ffn_gate_up projection's output, gate columns first.
//   One thread per 8 columns: two 16-byte loads, one 16-byte store.
//
// * Token embedding lookup from a Q6_K matrix (embeddingShader /
//   EmbeddingLookupKernel, ops.ts:381-426; block layout of
//   dequantizeQ6KBlock, src/gguf/quantization.ts:46-72): a row of `width`
//   values is width/256 blocks of 210 bytes -- ql[128] low nibbles, qh[64]
//   high bit pairs, 16 int8 scales, f16 d. Value i of a block (half = i/128,
//   quadrant = (i%128)/32, lane = i%32):
//     low  = ql[64 half + lane + 32 (quadrant & 1)], nibble quadrant >= 2
//     high = (qh[32 half + lane] >> 2 quadrant) & 3
//     q    = (low | high << 4) - 32
//     v    = f16((d * scale[8 half + lane/16 + 2 quadrant]) * q)   (f32 math)
//   One thread per 8 consecutive values, which share one scale and one d.
#include "internal.h"

namespace qwa {
namespace {

__global__ void __launch_bounds__(256)
    swiglu_kernel(const __half* __restrict__ combined, __half* __restrict__ out, int64_t rows,
                  int width) {
  const int vec_per_row = width >> 3;
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= rows * vec_per_row) return;
  const int64_t r = i / vec_per_row;
  const int c = static_cast<int>(i - r * vec_per_row);
  const uint4* src = reinterpret_cast<const uint4*>(combined + r * 2 * width);
  const uint4 gv = __ldcs(src + c);
  const uint4 uv = __ldcs(src + vec_per_row + c);
  const __half2* g2 = reinterpret_cast<const __half2*>(&gv);
  const __half2* u2 = reinterpret_cast<const __half2*>(&uv);
  uint4 o;
  __half2* o2 = reinterpret_cast<__half2*>(&o);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float2 g = __half22float2(g2[k]);
    const float2 u = __half22float2(u2[k]);
    const float s0 = silu(g.x);
    const float s1 = silu(g.y);
    o2[k] = __floats2half2_rn(s0 * u.x, s1 * u.y);
  }
  __stcs(reinterpret_cast<uint4*>(out + r * width) + c, o);
}

__global__ void __launch_bounds__(256)
    q6k_embedding_kernel(const uint32_t* __restrict__ ids, const uint8_t* __restrict__ table,
                         int vocab, __half* __restrict__ out, int64_t tokens, int width) {
  const int vec_per_row = width >> 3;
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= tokens * vec_per_row) return;
  const int64_t t = i / vec_per_row;
  const int col = static_cast<int>(i - t * vec_per_row) * 8;
  const uint32_t id = __ldg(ids + t);
  uint4 o = make_uint4(0, 0, 0, 0);
  if (id < static_cast<uint32_t>(vocab)) {
    const int blocks_per_row = width >> 8;
    const uint8_t* block =
        table + (static_cast<int64_t>(id) * blocks_per_row + (col >> 8)) * 210;
    const int within = col & 255, half = within >> 7, pos = within & 127;
    const int quadrant = pos >> 5, lane = pos & 31;
    // blocks start on even addresses (210-byte stride), so 2-byte loads
    const uint16_t* low2 =
        reinterpret_cast<const uint16_t*>(block + half * 64 + lane + (quadrant & 1) * 32);
    const uint16_t* high2 = reinterpret_cast<const uint16_t*>(block + 128 + half * 32 + lane);
    const int8_t scale = static_cast<int8_t>(__ldg(block + 192 + half * 8 + (lane >> 4) +
                                                   quadrant * 2));
    const float d = __half2float(
        __ushort_as_half(__ldg(reinterpret_cast<const unsigned short*>(block + 208))));
    const float ds = d * static_cast<float>(scale);
    __half2* o2 = reinterpret_cast<__half2*>(&o);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint32_t lo = __ldg(low2 + k), hi = __ldg(high2 + k);
      float v[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const uint32_t lb = (lo >> (8 * e)) & 0xffu, hb = (hi >> (8 * e)) & 0xffu;
        const uint32_t low = quadrant >= 2 ? (lb >> 4) : (lb & 15u);
        const uint32_t high = (hb >> (2 * quadrant)) & 3u;
        v[e] = ds * static_cast<float>(static_cast<int>(low | (high << 4)) - 32);
      }
      o2[k] = __floats2half2_rn(v[0], v[1]);
    }
  }
  reinterpret_cast<uint4*>(out + t * width)[col >> 3] = o;
}

}  // namespace

cudaError_t launch_swiglu(const __half* combined, __half* out, int rows, int width,
                          cudaStream_t stream) {
  const int64_t n = static_cast<int64_t>(rows) * (width / 8);
  if (n == 0) return cudaSuccess;
  swiglu_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, stream>>>(combined, out, rows,
                                                                           width);
  return cudaGetLastError();
}

cudaError_t launch_q6k_embedding(const uint32_t* ids, const uint8_t* table, int vocab,
                                 __half* out, int tokens, int width, cudaStream_t stream) {
  const int64_t n = static_cast<int64_t>(tokens) * (width / 8);
  if (n == 0) return cudaSuccess;
  q6k_embedding_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, stream>>>(
      ids, table, vocab, out, tokens, width);
  return cudaGetLastError();
}

}  // namespace qwa
