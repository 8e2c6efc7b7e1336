// Small-batch projection straight from Q4_0 tile32 weights (tcgen05):
//   C[M, N] (f16) = A[M, K] (f16) x W[N, K]^T, W in q4_0-tile32-compact records,
// for M <= 64 rows. The reference picks a latency pipeline for small m
// (src/webgpu/quant-matmul.ts:495-540) that reads the 4.5-bit weights; at such
// sizes the weight bytes are the cost, so this path reads the 20-byte records
// (0.625 B per weight) instead of a dequantised f16 copy (2 B per weight).
//
// Roles swap: the MMA's M dimension is 128 weight rows and its N dimension
// the M activation rows padded to a multiple of 16, so a tile of
// D[n, m] = sum_k W[n, k] A[m, k] lives in TMEM with one weight row per lane.
// Grid: (N / 128 weight-row tiles) x (K split into `splits` ranges), so a
// matrix of 1024 or 4096 rows still fills the GPU; each CTA writes its f32
// partial tile to ws[split][m][n], and a second kernel sums the splits in a
// fixed order (deterministic) and rounds to f16.
//
// CTA of 160 threads:
//   warps 0..3  dequantise the CTA's weight rows (thread = row) chunk by chunk
//               (64 values of K), f16(scale) * (q - 8) in f16 as
//               q40PrepackedDequant (quant-matmul.ts:98-107), written in the
//               128-byte-swizzled K-major layout the MMA reads; then the
//               epilogue (thread = weight row: tcgen05.ld of its M values);
//   warp 4      lane 0: TMA loads of the activation chunks and the MMAs;
//               the warp owns the TMEM allocation.
// Every K chunk of the CTA has its own buffer (at most kMaxChunks), so the
// loads, the dequantisation and the MMAs of different chunks overlap without
// a ring.
#include "internal.h"
#include "ptx.cuh"

namespace qwa {
namespace {

constexpr int kThreads = 160;
constexpr int kMaxChunks = 8;             // K values per CTA <= 512
constexpr uint32_t kWBytes = 128 * 128;   // 128 weight rows x 64 values (f16)
constexpr uint32_t kXBytes = 64 * 128;    // <= 64 activation rows x 64 values
constexpr uint32_t kChunkBytes = kWBytes + kXBytes;
// barriers: x_full[c], w_full[c], done; they follow the CTA's chunk buffers
constexpr int kXFull = 0, kWFull = kMaxChunks, kDone = 2 * kMaxChunks, kNumBars = kDone + 1;
__host__ __device__ constexpr uint32_t bar_offset(int chunks) { return chunks * kChunkBytes; }
__host__ __device__ constexpr uint32_t smem_bytes(int chunks) {
  return bar_offset(chunks) + 8 * kNumBars + 8 + 1024;  // + holder, abort flag, alignment
}

__global__ void __launch_bounds__(kThreads)
    q40_small_gemm_kernel(const __grid_constant__ CUtensorMap tm_x,
                          const uint32_t* __restrict__ packed, int n, int k, int m, int mpad,
                          int chunks, float* __restrict__ ws, int* status) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = smem_addr(smem);
  const uint32_t bar_off = bar_offset(chunks);
  uint32_t* holder = reinterpret_cast<uint32_t*>(smem + bar_off + 8 * kNumBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + bar_off + 8 * kNumBars + 4);
  auto bar = [&](int i) -> uint32_t { return sbase + bar_off + 8u * i; };
  auto w_buf = [&](int c) -> uint32_t { return sbase + c * kChunkBytes; };
  auto x_buf = [&](int c) -> uint32_t { return sbase + c * kChunkBytes + kWBytes; };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * 128;
  const int split = blockIdx.y;
  const int kblocks = k / 32;
  const int kb0 = split * chunks * 2;  // first 32-value block of this CTA
  const uint32_t tmem_cols = mpad <= 32 ? 32 : 64;

  if (threadIdx.x == 0) {
    for (int c = 0; c < kMaxChunks; ++c) {
      mbar_init(bar(kXFull + c), 1);
      mbar_init(bar(kWFull + c), 128);
    }
    mbar_init(bar(kDone), 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 4) {
    tmem_alloc(smem_addr(holder), tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *holder;

  if (warp == 4) {
    if (lane == 0) {
      tma_prefetch_desc(&tm_x);
      for (int c = 0; c < chunks; ++c) {
        mbar_arrive_expect_tx(bar(kXFull + c), static_cast<uint32_t>(mpad) * 128u);
        tma_load_2d(x_buf(c), &tm_x, bar(kXFull + c), (kb0 + 2 * c) * 32, 0);
      }
      const uint32_t idesc = idesc_f16_f32(128, static_cast<uint32_t>(mpad), false);
      bool ok = true;
      for (int c = 0; ok && c < chunks; ++c) {
        ok = mbar_wait(bar(kXFull + c), 0, abort_flag, status, kDevTimeoutSmallGemm) &&
             mbar_wait(bar(kWFull + c), 0, abort_flag, status, kDevTimeoutSmallGemm);
        if (!ok) break;
        tc_fence_after();
        const uint64_t a_desc = smem_desc_sw128(w_buf(c), 16, 1024);
        const uint64_t b_desc = smem_desc_sw128(x_buf(c), 16, 1024);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)  // K = 16 per step: 32 bytes along the swizzled row
          mma_ss(tmem, a_desc + ((kk * 32) >> 4), b_desc + ((kk * 32) >> 4), idesc,
                 (c > 0 || kk > 0) ? 1u : 0u);
      }
      // arrives once every issued MMA has completed (also after an abort)
      tc_commit(bar(kDone));
      // every activation load has landed before the CTA may exit
      bool drained = true;
      for (int c = 0; c < chunks; ++c) drained &= mbar_drain(bar(kXFull + c), 0, kWaitTimeoutNs);
      if (!drained) atomicCAS(status, 0, kDevTimeoutSmallGemm);
    }
  } else {
    // ---- dequantise: thread = weight row r of the tile
    const int r = threadIdx.x;  // 0..127
    const int row = n0 + r;
    const int t32 = row >> 5, rr = row & 31;
    for (int c = 0; c < chunks; ++c) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {  // the chunk's two 32-value blocks
        const int kb = kb0 + 2 * c + h;
        const uint32_t* p =
            packed + (static_cast<int64_t>(t32) * kblocks + kb) * 32 * 5 + rr * 5;
        const __half scale = __ushort_as_half(static_cast<unsigned short>(__ldg(p) & 0xffffu));
        uint32_t q[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) q[i] = __ldg(p + 1 + i);
        uint32_t lo[8], hi[8];  // half2 pairs of values 0..15 and 16..31 of the block
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const uint32_t word = q[i >> 1];
          const int sh = (i & 1) * 16;
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
        // 16-byte units h*4 .. h*4+3 of the 128-byte row, 128-byte swizzle
        const uint32_t row_base = w_buf(c) + r * 128;
        const uint32_t words[4][4] = {{lo[0], lo[1], lo[2], lo[3]},
                                      {lo[4], lo[5], lo[6], lo[7]},
                                      {hi[0], hi[1], hi[2], hi[3]},
                                      {hi[4], hi[5], hi[6], hi[7]}};
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const uint32_t unit = static_cast<uint32_t>(h * 4 + u) ^ static_cast<uint32_t>(r & 7);
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(row_base + unit * 16),
                       "r"(words[u][0]), "r"(words[u][1]), "r"(words[u][2]), "r"(words[u][3])
                       : "memory");
        }
      }
      // the MMA reads these stores through the async proxy
      fence_proxy_async_smem();
      mbar_arrive(bar(kWFull + c));
    }
    // ---- epilogue: D[r][0..mpad) of this weight row
    const bool ok = mbar_wait(bar(kDone), 0, abort_flag, status, kDevTimeoutSmallGemm);
    tc_fence_after();
    const int sub = warp;  // warps 0..3 own TMEM lanes 32*warp ..
    const uint32_t t_lane = tmem + (static_cast<uint32_t>(sub * 32) << 16);
    float* dst = ws + static_cast<int64_t>(split) * m * n + row;
#pragma unroll
    for (int cc = 0; cc < 2; ++cc) {
      if (cc * 32 >= mpad) break;  // warp-uniform
      uint32_t v[32];
      tmem_ld32(t_lane + cc * 32, v);
      tmem_wait_ld();
      reg_fence32(v);
      if (ok) {
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int mi = cc * 32 + i;
          if (mi < m) dst[static_cast<int64_t>(mi) * n] = __uint_as_float(v[i]);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 4) {
    tc_fence_after();
    tmem_dealloc(tmem, tmem_cols);
  }
}

// out[m][n] = f16(sum over splits of ws[s][m][n]), splits summed in order.
__global__ void __launch_bounds__(256)
    q40_small_finish_kernel(const float4* __restrict__ ws, uint2* __restrict__ out,
                            int64_t elems4, int splits) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= elems4) return;
  float4 acc = __ldcs(ws + i);
  for (int s = 1; s < splits; ++s) {
    const float4 v = __ldcs(ws + s * elems4 + i);
    acc.x += v.x;
    acc.y += v.y;
    acc.z += v.z;
    acc.w += v.w;
  }
  const __half2 a = __floats2half2_rn(acc.x, acc.y), b = __floats2half2_rn(acc.z, acc.w);
  out[i] = make_uint2(*reinterpret_cast<const uint32_t*>(&a), *reinterpret_cast<const uint32_t*>(&b));
}

}  // namespace

int q40_small_splits(int n, int k, int sms) {
  const int chunks = k / 64, tiles = n / 128;
  int best = chunks;
  for (int d = 1; d <= chunks; ++d) {
    if (chunks % d || chunks / d > kMaxChunks) continue;
    best = d;
    if (tiles * d >= 128 || tiles * d >= sms) break;  // enough CTAs to fill the GPU
  }
  return best;
}

cudaError_t launch_q40_small_gemm(const CUtensorMap& tm_x, const uint8_t* packed, __half* out,
                                  int m, int n, int k, int splits, float* ws, int* status,
                                  cudaStream_t stream) {
  static bool configured[kMaxDevices] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  if (!configured[dev]) {
    e = cudaFuncSetAttribute(q40_small_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             smem_bytes(kMaxChunks));
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  const int mpad = (m + 15) / 16 * 16;
  const int chunks = k / 64 / splits;
  dim3 grid(n / 128, splits);
  q40_small_gemm_kernel<<<grid, kThreads, smem_bytes(chunks), stream>>>(
      tm_x, reinterpret_cast<const uint32_t*>(packed), n, k, m, mpad, chunks, ws, status);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const int64_t elems4 = static_cast<int64_t>(m) * n / 4;
  q40_small_finish_kernel<<<static_cast<unsigned>((elems4 + 255) / 256), 256, 0, stream>>>(
      reinterpret_cast<const float4*>(ws), reinterpret_cast<uint2*>(out), elems4, splits);
  return cudaGetLastError();
}

}  // namespace qwa
