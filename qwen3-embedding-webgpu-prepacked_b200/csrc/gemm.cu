// Projection GEMM on the 5th-generation tensor cores:
//   C[M, N] (f16) = A[M, K] (f16, row-major) x W[N, K]^T (f16, row-major)
// with f32 accumulation in TMEM. W is the dequantised weight of a
// QuantMatmulKernel run (src/webgpu/quant-matmul.ts:495-540): the reference
// multiplies `input` [m, k] by the Q4_0 matrix whose row n holds output
// column n, i.e. output[m, n] = sum_k input[m, k] * W[n, k].
//
// Persistent kernel, one CTA per SM, 192 threads:
//   warp 0      TMA producer: A tile 128 x 64 and W tile 256 x 64 per stage
//               (128-byte swizzle), 4-stage ring;
//   warp 1      TMEM owner and single MMA issuer: per stage 4 x
//               tcgen05.mma M=128 N=256 K=16 into one of two accumulators;
//   warps 2..5  epilogue: tcgen05.ld of the accumulator (thread = row),
//               f32 -> f16, 16-byte stores; releases the accumulator so the
//               MMAs of the next tile overlap this tile's stores.
// Output tiles are walked n-fastest so consecutive tiles of a CTA (and the
// CTAs running at the same time) share the A rows in L2; W (<= 12 MB for
// Qwen3-0.6B) stays L2-resident.
#include "internal.h"
#include "ptx.cuh"

namespace qwa {
namespace {

constexpr int kBM = 128, kBN = 256, kBK = 64;
constexpr int kStages = 4;
constexpr int kGemmThreads = 192;
constexpr uint32_t kABytes = kBM * kBK * 2;  // 16 KB
constexpr uint32_t kBBytes = kBN * kBK * 2;  // 32 KB
constexpr uint32_t kStageBytes = kABytes + kBBytes;
constexpr uint32_t kBarOff = kStages * kStageBytes;  // 192 KB
// barriers: full[4], empty[4], acc_full[2], acc_empty[2]
constexpr int kFull = 0, kEmpty = kStages, kAccFull = 2 * kStages, kAccEmpty = 2 * kStages + 2;
constexpr int kNumBars = 2 * kStages + 4;
constexpr uint32_t kHolderOff = kBarOff + 8 * kNumBars;
constexpr uint32_t kAbortOff = kHolderOff + 4;
constexpr uint32_t kGemmSmem = kAbortOff + 4 + 1024;  // + alignment slack
static_assert(kGemmSmem <= 232448, "shared memory budget");
constexpr uint32_t kIdesc = idesc_f16_f32(kBM, kBN, false);

__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_f16_kernel(const __grid_constant__ CUtensorMap tm_a,
                    const __grid_constant__ CUtensorMap tm_w, __half* __restrict__ out, int M,
                    int N, int K, int* status) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = smem_addr(smem);
  uint32_t* holder = reinterpret_cast<uint32_t*>(smem + kHolderOff);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kAbortOff);
  auto bar = [&](int i) -> uint32_t { return sbase + kBarOff + 8u * i; };
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(bar(kFull + s), 1);
      mbar_init(bar(kEmpty + s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(bar(kAccFull + a), 1);
      mbar_init(bar(kAccEmpty + a), 128);
    }
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tm_a);
    tma_prefetch_desc(&tm_w);
  }
  if (warp == 1) {
    tmem_alloc(smem_addr(holder), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *holder;

  const int tiles_n = N / kBN;
  const int num_tiles = ((M + kBM - 1) / kBM) * tiles_n;
  const int kblocks = K / kBK;

  if (warp == 0) {
    if (lane == 0) {
      bool ok = true;
      int c = 0;  // stage uses
      for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x) {
        const int m0 = (tile / tiles_n) * kBM, n0 = (tile % tiles_n) * kBN;
        for (int kb = 0; kb < kblocks; ++kb, ++c) {
          const int s = c % kStages;
          if (!(ok = mbar_wait(bar(kEmpty + s), ((c / kStages) & 1) ^ 1, abort_flag, status,
                               kDevTimeoutGemmEmpty)))
            break;
          const uint32_t dst = sbase + s * kStageBytes;
          mbar_arrive_expect_tx(bar(kFull + s), kStageBytes);
          tma_load_2d(dst, &tm_a, bar(kFull + s), kb * kBK, m0);
          tma_load_2d(dst + kABytes, &tm_w, bar(kFull + s), kb * kBK, n0);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      bool ok = true;
      int c = 0, lt = 0;  // stage uses, local tiles
      const uint64_t a_desc0 = smem_desc_sw128(sbase, 16, 1024);
      const uint64_t b_desc0 = smem_desc_sw128(sbase + kABytes, 16, 1024);
      for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x, ++lt) {
        const int acc = lt & 1;
        if (!(ok = mbar_wait(bar(kAccEmpty + acc), ((lt >> 1) & 1) ^ 1, abort_flag, status,
                             kDevTimeoutAccEmpty)))
          break;
        tc_fence_after();
        const uint32_t d = tmem + acc * kBN;
        for (int kb = 0; kb < kblocks; ++kb, ++c) {
          const int s = c % kStages;
          if (!(ok = mbar_wait(bar(kFull + s), (c / kStages) & 1, abort_flag, status,
                               kDevTimeoutGemmFull)))
            break;
          tc_fence_after();
          const uint64_t so = (s * kStageBytes) >> 4;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            mma_ss(d, a_desc0 + so + ((kk * 32) >> 4), b_desc0 + so + ((kk * 32) >> 4), kIdesc,
                   (kb > 0 || kk > 0) ? 1u : 0u);
          tc_commit(bar(kEmpty + s));
        }
        if (ok) tc_commit(bar(kAccFull + acc));
      }
    }
  } else {
    // epilogue: warp w reads TMEM lanes 32*(w%4) .. +31 (its sub-partition)
    const int sub = warp & 3;
    const int r = sub * 32 + lane;
    bool ok = true;
    int lt = 0;
    for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x, ++lt) {
      const int acc = lt & 1;
      const int m0 = (tile / tiles_n) * kBM, n0 = (tile % tiles_n) * kBN;
      if (!(ok = mbar_wait(bar(kAccFull + acc), (lt >> 1) & 1, abort_flag, status,
                           kDevTimeoutAccFull)))
        break;
      tc_fence_after();
      const uint32_t t_row = tmem + (static_cast<uint32_t>(sub * 32) << 16) + acc * kBN;
      const int row = m0 + r;
      uint4* dst = reinterpret_cast<uint4*>(out + static_cast<int64_t>(row) * N + n0);
#pragma unroll 1
      for (int ch = 0; ch < kBN / 32; ++ch) {
        uint32_t v[32];
        tmem_ld32(t_row + 32 * ch, v);
        tmem_wait_ld();
        reg_fence32(v);
        if (row < M) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 w;
            w.x = pack_half2(__uint_as_float(v[8 * q + 0]), __uint_as_float(v[8 * q + 1]));
            w.y = pack_half2(__uint_as_float(v[8 * q + 2]), __uint_as_float(v[8 * q + 3]));
            w.z = pack_half2(__uint_as_float(v[8 * q + 4]), __uint_as_float(v[8 * q + 5]));
            w.w = pack_half2(__uint_as_float(v[8 * q + 6]), __uint_as_float(v[8 * q + 7]));
            dst[4 * ch + q] = w;
          }
        }
      }
      tc_fence_before();
      mbar_arrive(bar(kAccEmpty + acc));
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace

cudaError_t launch_gemm_f16(const CUtensorMap& tm_a, const CUtensorMap& tm_w, __half* out, int M,
                            int N, int K, int* status, cudaStream_t stream) {
  static bool configured[kMaxDevices] = {};
  static int sm_count[kMaxDevices] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  if (!configured[dev]) {
    e = cudaFuncSetAttribute(gemm_f16_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kGemmSmem);
    if (e == cudaSuccess)
      e = cudaDeviceGetAttribute(&sm_count[dev], cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  const int sms = sm_count[dev];
  const int tiles = ((M + kBM - 1) / kBM) * (N / kBN);
  const int grid = tiles < sms ? tiles : sms;
  if (grid <= 0) return cudaSuccess;
  gemm_f16_kernel<<<grid, kGemmThreads, kGemmSmem, stream>>>(tm_a, tm_w, out, M, N, K, status);
  return cudaGetLastError();
}

}  // namespace qwa
