// Q4_0 "tile32-compact" weights -> f16 row-major W[n, k] (HBM-bound, once
// per weight).
//
// Layout (src/prepacked/format.ts:65-99, packQ40Tile32): the n output rows are
// cut into tiles of 32; for tile t, k-block b (32 values) and local row r the
// 20-byte record at ((t * k/32 + b) * 32 + r) * 20 holds the GGML Q4_0 block
// of row 32t + r: f16 scale at +0, two zero bytes, then 16 bytes whose low
// nibble j is value j and high nibble j is value j + 16. Rows past n in the
// last tile are zero records.
//
// Value (quant-matmul.ts:98-107, q40PrepackedDequant): f16(scale) *
// (f16(q) - 8), both operations in f16; q - 8 is exact and the product is
// rounded to nearest even, so __hmul reproduces it bit for bit.
//
// One thread per record: five 4-byte loads (records are 4-byte aligned),
// four 16-byte stores of the row's 32 values.
#include "internal.h"

namespace qwa {
namespace {

__global__ void __launch_bounds__(256)
    q40_tile32_dequant_kernel(const uint32_t* __restrict__ packed, int n, int kblocks,
                              int64_t records, __half* __restrict__ out) {
  const int64_t rec = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (rec >= records) return;
  const int r = static_cast<int>(rec & 31);
  const int64_t tb = rec >> 5;  // tile * kblocks + kblock
  const int b = static_cast<int>(tb % kblocks);
  const int row = static_cast<int>(tb / kblocks) * 32 + r;
  if (row >= n) return;
  const uint32_t* p = packed + rec * 5;
  const __half scale = __ushort_as_half(static_cast<unsigned short>(__ldg(p) & 0xffffu));
  uint32_t q[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) q[i] = __ldg(p + 1 + i);
  uint32_t lo[8], hi[8];  // packed half2 of values 0..15 and 16..31
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t word = q[i >> 1];
    const int sh = (i & 1) * 16;  // bytes 2i, 2i+1 of the 16 nibble bytes
    const uint32_t b0 = (word >> sh) & 0xffu, b1 = (word >> (sh + 8)) & 0xffu;
    const __half l0 = __hmul(scale, __int2half_rn(static_cast<int>(b0 & 15u) - 8));
    const __half l1 = __hmul(scale, __int2half_rn(static_cast<int>(b1 & 15u) - 8));
    const __half h0 = __hmul(scale, __int2half_rn(static_cast<int>(b0 >> 4) - 8));
    const __half h1 = __hmul(scale, __int2half_rn(static_cast<int>(b1 >> 4) - 8));
    lo[i] = static_cast<uint32_t>(__half_as_ushort(l0)) |
            (static_cast<uint32_t>(__half_as_ushort(l1)) << 16);
    hi[i] = static_cast<uint32_t>(__half_as_ushort(h0)) |
            (static_cast<uint32_t>(__half_as_ushort(h1)) << 16);
  }
  uint4* dst = reinterpret_cast<uint4*>(out + static_cast<int64_t>(row) * (kblocks * 32) + b * 32);
  dst[0] = make_uint4(lo[0], lo[1], lo[2], lo[3]);
  dst[1] = make_uint4(lo[4], lo[5], lo[6], lo[7]);
  dst[2] = make_uint4(hi[0], hi[1], hi[2], hi[3]);
  dst[3] = make_uint4(hi[4], hi[5], hi[6], hi[7]);
}

}  // namespace

cudaError_t launch_q40_tile32_dequant(const uint8_t* packed, int n, int k, __half* out,
                                      cudaStream_t stream) {
  const int kblocks = k / 32;
  const int64_t records = static_cast<int64_t>((n + 31) / 32) * kblocks * 32;
  if (records == 0) return cudaSuccess;
  const int threads = 256;
  const int64_t blocks = (records + threads - 1) / threads;
  q40_tile32_dequant_kernel<<<static_cast<unsigned>(blocks), threads, 0, stream>>>(
      reinterpret_cast<const uint32_t*>(packed), n, kblocks, records, out);
  return cudaGetLastError();
}

}  // namespace qwa
