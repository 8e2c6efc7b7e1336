// Projection GEMM on the 5th-generation tensor cores:
//   C[M, N] (f16) = A[M, K] (f16, row-major) x W[N, K]^T (f16, row-major)
// with f32 accumulation in TMEM. W is the dequantised weight of a
// QuantMatmulKernel run (src/webgpu/quant-matmul.ts:495-540): the reference
// multiplies `input` [m, k] by the Q4_0 matrix whose row n holds output
// column n, i.e. output[m, n] = sum_k input[m, k] * W[n, k].
//
// Persistent kernel, one CTA per SM, 320 threads:
//   warp 0      TMA producer (per stage an A tile of 128 rows x 64 and a W
//               tile, 128-byte swizzle);
//   warp 1      TMEM owner and single MMA issuer (tcgen05.mma K=16 steps
//               into one of two 256-column accumulators);
//   warps 2..9  epilogue: tcgen05.ld of the accumulator (thread = row; the
//               two warps of a TMEM sub-partition take one 128-column half
//               each), f32 -> f16, 16-byte stores; releases the accumulator
//               so the MMAs of the next tile overlap this tile's stores.
// Two shapes of the same kernel:
//   single CTA  (kPair = false): 128 x 256 tiles, W tile 256 x 64, 4 stages
//               of 48 KB, tcgen05.mma.cta_group::1 M=128 N=256;
//   CTA pair    (kPair = true, clusters of 2): 256 x 256 tiles; each CTA
//               loads its own 128 rows of A and its 128-row half of the W
//               tile (32 KB per stage, 6 stages), both CTAs' loads complete
//               on the even CTA's barrier, and the even CTA alone issues
//               tcgen05.mma.cta_group::2 M=256 N=256, which reads the odd
//               CTA's operands at the same shared-memory offsets and
//               accumulates rows 128..255 in the odd CTA's TMEM. Per FLOP
//               this halves the W traffic and cuts the shared-memory operand
//               feed by a third. No load is multicast.
// With the QKV epilogue (N = 4096, the attn_qkv projection of
// src/webgpu/model.ts:93), a 256-column tile holds two whole heads of each
// row, so the epilogue also applies the per-head Q/K RMSNorm + RoPE of
// qkNormRopeShader (src/webgpu/ops.ts:104-150) to the q and k tiles and
// writes q [T,16,128], k [T,8,128] and v [T,1024] directly: the [T, 4096]
// qkvRaw round trip and the separate prologue launch disappear. The
// arithmetic is the unfused pipeline's, step for step (accumulator rounded to
// f16 as qkvRaw would be, the prologue kernel's f32 sum order, normalisation
// and rotation), so both paths give identical bits.
// Output tiles are walked n-fastest so consecutive tiles of a CTA (and the
// CTAs running at the same time) share the A rows in L2; W (<= 12 MB for
// Qwen3-0.6B) stays L2-resident.
#include "internal.h"
#include "ptx.cuh"

namespace qwa {
namespace {

constexpr int kBK = 64, kBN = 256;
constexpr int kCuSmem = 1024;  // requests whose cu_seqlens are staged in shared memory
constexpr int kGemmThreads = 320;
constexpr int kEpiWarps = 8;

// Shared-memory layout of one shape. On CTA pairs the epilogue stages its
// output in shared memory for TMA stores (kTmaOut, 4 KB per epilogue warp).
// The plain GEMM keeps six pipeline stages beside that, having none of the QKV
// epilogue's regions; the fused QKV GEMM drops to five.
template <bool kQkv, bool kPair>
struct Layout {
  static constexpr bool kTmaOut = kPair;
  static constexpr int kStages = kPair ? (kQkv ? 5 : 6) : 4;
  static constexpr uint32_t kABytes = 128 * kBK * 2;                      // 16 KB
  static constexpr uint32_t kBBytes = (kPair ? 128 : 256) * kBK * 2;      // 16 / 32 KB
  static constexpr uint32_t kStageBytes = kABytes + kBBytes;
  static constexpr uint32_t kBarOff = kStages * kStageBytes;              // 192 KB
  // barriers: full[S], empty[S], acc_full[2], acc_empty[2]
  static constexpr int kFull = 0, kEmpty = kStages, kAccFull = 2 * kStages,
                       kAccEmpty = 2 * kStages + 2, kNumBars = 2 * kStages + 4;
  // the QKV epilogue's regions (empty for the plain GEMM)
  static constexpr uint32_t kNormWOff = kBarOff + 8 * kNumBars;           // 2 x 128 f32
  static constexpr uint32_t kCuOff = kNormWOff + (kQkv ? 2 * 128 * 4 : 0);  // kCuSmem + 1 ints
  static constexpr uint32_t kXchOff = kCuOff + (kQkv ? (kCuSmem + 4) * 4 : 0);  // partial sums
  static constexpr uint32_t kPairOkOff = kXchOff + (kQkv ? 4 * 2 * 2 * 128 * 4 : 0);
  static constexpr uint32_t kHolderOff = kPairOkOff + 8 * 4;
  static constexpr uint32_t kAbortOff = kHolderOff + 4;
  // output staging: 4 KB (32 rows x 64 columns, 128-byte swizzle) per epilogue warp
  static constexpr uint32_t kOutOff = (kAbortOff + 4 + 1023) & ~1023u;
  static constexpr uint32_t kOutBytes = kTmaOut ? kEpiWarps * 4096 : 0;
  static constexpr uint32_t kSmem = kOutOff + kOutBytes + 1024;  // + alignment slack
  static_assert(kSmem <= 232448, "shared memory budget");
  static constexpr uint32_t kIdesc = idesc_f16_f32(kPair ? 256 : 128, kBN, false);
  static constexpr int kRowsPerTile = kPair ? 256 : 128;
  // arrivals that free an accumulator: one per epilogue warp of each CTA
  static constexpr uint32_t kAccEmptyCount = kPair ? 2 * kEpiWarps : kEpiWarps;
};

// Start row of the request holding row t: binary search over cu[0..batch].
__device__ __forceinline__ int request_start(const int32_t* cu, int batch, int t) {
  int lo = 0, hi = batch - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (cu[mid] <= t) lo = mid;
    else hi = mid - 1;
  }
  return cu[lo];
}

__device__ __forceinline__ float f16_round(float x) { return __half2float(__float2half_rn(x)); }

__device__ __forceinline__ void pair_sync(int sub) {
  asm volatile("bar.sync %0, 64;" ::"r"(1 + sub) : "memory");
}

// Q/K norm + RoPE of one row of a q or k tile, for the quarter of each head
// this warp owns. The two warps of a TMEM sub-partition split every head's
// 128 dims: warp c (0 or 1) takes dims [32c, 32c+32) and their RoPE partners
// [64+32c, 96+32c), so it needs only table entries [32c, 32c+32) of the row
// (16 float4, loaded once for both heads). Per head the warps exchange the
// four first-level sums of squares through shared memory; the sum is then
// combined in the order of the prologue kernel's butterfly (dims in groups of
// 8, xor 8, 4, 2, 1), so inv equals the prologue's bit for bit.
// 64-byte-row staging (TMA SWIZZLE_64B layout: 16-byte chunk XOR (row / 2) % 4).
__device__ __forceinline__ void stage_row64(uint32_t buf, int row, int chunk, uint32_t w0,
                                            uint32_t w1, uint32_t w2, uint32_t w3) {
  const uint32_t addr =
      buf + row * 64 + ((static_cast<uint32_t>(chunk) ^ ((static_cast<uint32_t>(row) >> 1) & 3u)) << 4);
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(w0), "r"(w1), "r"(w2),
               "r"(w3)
               : "memory");
}

// kTma: instead of 16-byte stores to dst0, each head's two 32-dim segments of
// the warp's 32 rows go through the warp's two 2 KB staging buffers (stage,
// stage + 2048) and two TMA stores of boxes {32 dims, 1 head, 32 rows} at
// (32c / 64 + 32c, head0 + hh, r0); tm is the q or k output map.
template <bool kTma>
__device__ __forceinline__ void norm_rope_quarter(uint32_t t_tile, int c, int sub, int lane,
                                                  const float* w, const float4 (&tab)[16],
                                                  float eps, bool valid, float* xch,
                                                  __half* dst0, uint32_t stage,
                                                  const CUtensorMap* tm, int head0, int r0) {
#pragma unroll 1
  for (int hh = 0; hh < 2; ++hh) {
    uint32_t lo[32], hi[32];
    tmem_ld32(t_tile + 128 * hh + 32 * c, lo);
    tmem_ld32(t_tile + 128 * hh + 64 + 32 * c, hi);
    tmem_wait_ld();
    reg_fence32(lo);
    reg_fence32(hi);
    // first level: groups j (dims 8j..8j+7) = 4c..4c+3 and 8+4c..; l1[i] = p[4c+i] + p[8+4c+i]
    float l1[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float sa = 0.f, sb = 0.f;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float xa = f16_round(__uint_as_float(lo[8 * i + e]));
        const float xb = f16_round(__uint_as_float(hi[8 * i + e]));
        sa = fmaf(xa, xa, sa);
        sb = fmaf(xb, xb, sb);
      }
      l1[i] = sa + sb;
    }
    float* mine = xch + ((sub * 2 + hh) * 2 + c) * 128 + lane * 4;
    float* other = xch + ((sub * 2 + hh) * 2 + (c ^ 1)) * 128 + lane * 4;
    *reinterpret_cast<float4*>(mine) = make_float4(l1[0], l1[1], l1[2], l1[3]);
    pair_sync(sub);
    const float4 o = *reinterpret_cast<const float4*>(other);
    // second level: groups j < 4 (warp 0's) + groups j + 4 (warp 1's)
    const float4 g0 = c == 0 ? make_float4(l1[0], l1[1], l1[2], l1[3]) : o;
    const float4 g1 = c == 0 ? o : make_float4(l1[0], l1[1], l1[2], l1[3]);
    const float m0 = g0.x + g1.x, m1 = g0.y + g1.y, m2 = g0.z + g1.z, m3 = g0.w + g1.w;
    const float ss = (m0 + m2) + (m1 + m3);
    const float inv = 1.0f / sqrtf(ss * (1.0f / 128) + eps);
    if (!kTma && !valid) continue;
    if (kTma) {  // both buffers free: the previous head's / tile's stores have read them
      if (lane == 0) bulk_wait_read();
      __syncwarp();
    }
    uint4* d4 = reinterpret_cast<uint4*>(dst0 + 128 * hh);
#pragma unroll
    for (int q = 0; q < 4; ++q) {  // 8 dims per 16-byte store
      uint32_t lo_out[4], hi_out[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int i = 8 * q + 2 * e;  // index inside the quarter
        const int d = 32 * c + i;     // dim in [0, 64)
        const float4 cs = tab[i / 2];  // (cos, sin) of dims d, d+1
        const float na0 = f16_round(__uint_as_float(lo[i])) * inv * w[d];
        const float na1 = f16_round(__uint_as_float(lo[i + 1])) * inv * w[d + 1];
        const float nb0 = f16_round(__uint_as_float(hi[i])) * inv * w[64 + d];
        const float nb1 = f16_round(__uint_as_float(hi[i + 1])) * inv * w[65 + d];
        lo_out[e] = pack_half2(fmaf(na0, cs.x, -1.f * nb0 * cs.y), fmaf(na1, cs.z, -1.f * nb1 * cs.w));
        hi_out[e] = pack_half2(fmaf(nb0, cs.x, 1.f * na0 * cs.y), fmaf(nb1, cs.z, 1.f * na1 * cs.w));
      }
      if (kTma) {
        stage_row64(stage, lane, q, lo_out[0], lo_out[1], lo_out[2], lo_out[3]);
        stage_row64(stage + 2048, lane, q, hi_out[0], hi_out[1], hi_out[2], hi_out[3]);
      } else {
        d4[4 * c + q] = make_uint4(lo_out[0], lo_out[1], lo_out[2], lo_out[3]);
        d4[8 + 4 * c + q] = make_uint4(hi_out[0], hi_out[1], hi_out[2], hi_out[3]);
      }
    }
    if (kTma) {
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {  // rows >= M are clipped by the map
        tma_store_3d(tm, stage, 32 * c, head0 + hh, r0);
        tma_store_3d(tm, stage + 2048, 64 + 32 * c, head0 + hh, r0);
        bulk_commit();
      }
    }
  }
}

template <bool kQkv, bool kPair, bool kGlu = false>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_f16_kernel(const __grid_constant__ CUtensorMap tm_a,
                    const __grid_constant__ CUtensorMap tm_w,
                    const __grid_constant__ CUtensorMap tm_out,
                    const __grid_constant__ CUtensorMap tm_qo,
                    const __grid_constant__ CUtensorMap tm_ko, __half* __restrict__ out, int M,
                    int N, int K, int* status, const QkvEpilogue qkv) {
  using L = Layout<kQkv, kPair>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = smem_addr(smem);
  uint32_t* holder = reinterpret_cast<uint32_t*>(smem + L::kHolderOff);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kAbortOff);
  auto bar = [&](int i) -> uint32_t { return sbase + L::kBarOff + 8u * i; };
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // CTA pair: rank 0 (even) is the leader that issues the MMAs
  const uint32_t rank = kPair ? cluster_ctarank() : 0u;
  const bool leader = rank == 0;
  const int unit = kPair ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
  const int units = kPair ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);

  if (threadIdx.x == 0) {
    for (int s = 0; s < L::kStages; ++s) {
      mbar_init(bar(L::kFull + s), 1);
      mbar_init(bar(L::kEmpty + s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(bar(L::kAccFull + a), 1);
      mbar_init(bar(L::kAccEmpty + a), L::kAccEmptyCount);
    }
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tm_a);
    tma_prefetch_desc(&tm_w);
  }
  float* norm_w = reinterpret_cast<float*>(smem + L::kNormWOff);
  int32_t* cu_s = reinterpret_cast<int32_t*>(smem + L::kCuOff);
  float* xch = reinterpret_cast<float*>(smem + L::kXchOff);
  volatile int* pair_ok = reinterpret_cast<volatile int*>(smem + L::kPairOkOff);
  if (kQkv) {
    for (int i = threadIdx.x; i < 256; i += kGemmThreads)
      norm_w[i] = i < 128 ? qkv.q_weight[i] : qkv.k_weight[i - 128];
    if (qkv.batch <= kCuSmem)
      for (int i = threadIdx.x; i <= qkv.batch; i += kGemmThreads) cu_s[i] = qkv.cu[i];
  }
  const int32_t* cu_tab = (kQkv && qkv.batch > kCuSmem) ? qkv.cu : cu_s;
  if (warp == 1) {
    if (kPair) {
      tmem_alloc_pair(smem_addr(holder), 512);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(smem_addr(holder), 512);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  if (kPair) cluster_sync();  // barriers and TMEM of both CTAs are ready
  else __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *holder;

  const int tiles_n = N / kBN;
  const int num_tiles = ((M + L::kRowsPerTile - 1) / L::kRowsPerTile) * tiles_n;
  const int kblocks = K / kBK;

  if (warp == 0) {
    // ---------------------------------------------------------- producer
    if (lane == 0) {
      bool ok = true;
      int c = 0;  // stage uses
      const uint32_t full0 = kPair ? mapa_shared(bar(L::kFull), 0) : bar(L::kFull);
      for (int tile = unit; ok && tile < num_tiles; tile += units) {
        const int m0 = (tile / tiles_n) * L::kRowsPerTile + static_cast<int>(rank) * 128;
        const int n0 = (tile % tiles_n) * kBN + (kPair ? static_cast<int>(rank) * 128 : 0);
        for (int kb = 0; kb < kblocks; ++kb, ++c) {
          const int s = c % L::kStages;
          if (!(ok = mbar_wait(bar(L::kEmpty + s), ((c / L::kStages) & 1) ^ 1, abort_flag, status,
                               kDevTimeoutGemmEmpty)))
            break;
          const uint32_t dst = sbase + s * L::kStageBytes;
          if (kPair) {
            // the leader's full barrier counts both CTAs' bytes
            if (leader) mbar_arrive_expect_tx(bar(L::kFull + s), 2 * L::kStageBytes);
            tma_load_2d_pair(dst, &tm_a, full0 + 8u * s, kb * kBK, m0);
            tma_load_2d_pair(dst + L::kABytes, &tm_w, full0 + 8u * s, kb * kBK, n0);
          } else {
            mbar_arrive_expect_tx(bar(L::kFull + s), L::kStageBytes);
            tma_load_2d(dst, &tm_a, bar(L::kFull + s), kb * kBK, m0);
            tma_load_2d(dst + L::kABytes, &tm_w, bar(L::kFull + s), kb * kBK, n0);
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------- MMA issuer
    if (lane == 0 && leader) {
      bool ok = true;
      int c = 0, lt = 0;  // stage uses, local tiles
      const uint64_t a_desc0 = smem_desc_sw128(sbase, 16, 1024);
      const uint64_t b_desc0 = smem_desc_sw128(sbase + L::kABytes, 16, 1024);
      for (int tile = unit; ok && tile < num_tiles; tile += units, ++lt) {
        const int acc = lt & 1;
        if (!(ok = mbar_wait(bar(L::kAccEmpty + acc), ((lt >> 1) & 1) ^ 1, abort_flag, status,
                             kDevTimeoutAccEmpty)))
          break;
        tc_fence_after();
        const uint32_t d = tmem + acc * kBN;
        for (int kb = 0; kb < kblocks; ++kb, ++c) {
          const int s = c % L::kStages;
          if (!(ok = mbar_wait(bar(L::kFull + s), (c / L::kStages) & 1, abort_flag, status,
                               kDevTimeoutGemmFull)))
            break;
          tc_fence_after();
          const uint64_t so = (s * L::kStageBytes) >> 4;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            const uint64_t ko = so + ((kk * 32) >> 4);
            if (kPair)
              mma_ss_pair(d, a_desc0 + ko, b_desc0 + ko, L::kIdesc, (kb > 0 || kk > 0) ? 1u : 0u);
            else
              mma_ss(d, a_desc0 + ko, b_desc0 + ko, L::kIdesc, (kb > 0 || kk > 0) ? 1u : 0u);
          }
          if (kPair) tc_commit_pair(bar(L::kEmpty + s), 0x3);
          else tc_commit(bar(L::kEmpty + s));
        }
        if (ok) {
          if (kPair) tc_commit_pair(bar(L::kAccFull + acc), 0x3);
          else tc_commit(bar(L::kAccFull + acc));
        }
      }
    }
  } else {
    // --------------------------------------------------------- epilogue
    // warp w reads TMEM lanes 32*(w%4) .. +31 (its sub-partition); warps
    // 2..5 take columns 0..127 of the tile, warps 6..9 columns 128..255
    const int sub = warp & 3;
    const int half = (warp - 2) >> 2;
    const int r = sub * 32 + lane;
    const uint32_t acc_empty0 = kPair ? mapa_shared(bar(L::kAccEmpty), 0) : bar(L::kAccEmpty);
    bool ok = true;
    int lt = 0;
    for (int tile = unit; ok && tile < num_tiles; tile += units, ++lt) {
      const int acc = lt & 1;
      const int m0 = (tile / tiles_n) * L::kRowsPerTile + static_cast<int>(rank) * 128;
      const int n0 = (tile % tiles_n) * kBN;
      const int row = m0 + r;
      const int nt = n0 / kBN;
      // RoPE table entries of this row, fetched before the accumulator wait
      float4 tab[16];
      if (kQkv && nt < 12) {
        const int pos = row < M ? row - request_start(cu_tab, qkv.batch, row) : 0;
        const float4* trow =
            reinterpret_cast<const float4*>(qkv.table + static_cast<int64_t>(pos) * 64) + 16 * half;
#pragma unroll
        for (int i = 0; i < 16; ++i) tab[i] = __ldg(trow + i);
      }
      ok = mbar_wait(bar(L::kAccFull + acc), (lt >> 1) & 1, abort_flag, status, kDevTimeoutAccFull);
      if (kQkv) {
        // the pair meets at named barriers below: leave the loop together
        // (each wait above is bounded, so both warps always reach this point)
        if (lane == 0) pair_ok[sub * 2 + half] = ok ? 1 : 0;
        pair_sync(sub);
        ok = pair_ok[sub * 2] && pair_ok[sub * 2 + 1];
        pair_sync(sub);  // both read before the next tile's write
      }
      if (!ok) break;
      tc_fence_after();
      const uint32_t t_tile = tmem + (static_cast<uint32_t>(sub * 32) << 16) + acc * kBN;
      const uint32_t t_cols = t_tile + 128 * half;
      if constexpr (kGlu) {
        // Fused SwiGLU (gate_up weight rows interleaved in 128-row blocks):
        // tile columns 0..127 are gate values g, 128..255 the up values u of
        // the same 128 outputs. Warp half h produces outputs [64h, 64h + 64):
        // f16(silu(g) * u) with g and u first rounded to f16, as the unfused
        // GEMM stores them and swiglu_kernel reads them.
        const int oc = nt * 128 + 64 * half;  // output column in [M, N / 2]
        auto glu_pack = [&](const uint32_t (&g)[32], const uint32_t (&u)[32], int i) {
          const float g0 = f16_round(__uint_as_float(g[2 * i]));
          const float g1 = f16_round(__uint_as_float(g[2 * i + 1]));
          const float u0 = f16_round(__uint_as_float(u[2 * i]));
          const float u1 = f16_round(__uint_as_float(u[2 * i + 1]));
          const float s0 = silu(g0);
          const float s1 = silu(g1);
          return pack_half2(s0 * u0, s1 * u1);
        };
        if constexpr (L::kTmaOut) {
          const uint32_t stage = sbase + L::kOutOff + (warp - 2) * 4096;
          if (lane == 0) bulk_wait_read();  // the previous store has read the buffer
          __syncwarp();
#pragma unroll 1
          for (int b = 0; b < 2; ++b) {
            uint32_t g[32], u[32];
            tmem_ld32(t_tile + 64 * half + 32 * b, g);
            tmem_ld32(t_tile + 128 + 64 * half + 32 * b, u);
            tmem_wait_ld();
            reg_fence32(g);
            reg_fence32(u);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const uint32_t w0 = glu_pack(g, u, 4 * q + 0), w1 = glu_pack(g, u, 4 * q + 1);
              const uint32_t w2 = glu_pack(g, u, 4 * q + 2), w3 = glu_pack(g, u, 4 * q + 3);
              const uint32_t unit = static_cast<uint32_t>(4 * b + q);
              const uint32_t addr = stage + lane * 128 + ((unit ^ (lane & 7)) << 4);
              asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(w0),
                           "r"(w1), "r"(w2), "r"(w3)
                           : "memory");
            }
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tm_out, stage, oc, m0 + sub * 32);  // rows >= M are clipped
            bulk_commit();
          }
        } else {
          uint4* dst = reinterpret_cast<uint4*>(out + static_cast<int64_t>(row) * (N / 2) + oc);
#pragma unroll 1
          for (int b = 0; b < 2; ++b) {
            uint32_t g[32], u[32];
            tmem_ld32(t_tile + 64 * half + 32 * b, g);
            tmem_ld32(t_tile + 128 + 64 * half + 32 * b, u);
            tmem_wait_ld();
            reg_fence32(g);
            reg_fence32(u);
            if (row < M) {
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                uint4 wv;
                wv.x = glu_pack(g, u, 4 * q + 0);
                wv.y = glu_pack(g, u, 4 * q + 1);
                wv.z = glu_pack(g, u, 4 * q + 2);
                wv.w = glu_pack(g, u, 4 * q + 3);
                dst[4 * b + q] = wv;
              }
            }
          }
        }
      } else if (kQkv && nt < 12) {
        // q tiles 0..7 (heads 2nt, 2nt+1), k tiles 8..11 (kv heads 2(nt-8), +1)
        const bool is_q = nt < 8;
        const int head0 = is_q ? 2 * nt : 2 * (nt - 8);
        __half* dst = is_q ? qkv.q_out + (static_cast<int64_t>(row) * 16 + head0) * 128
                           : qkv.k_out + (static_cast<int64_t>(row) * 8 + head0) * 128;
        norm_rope_quarter<L::kTmaOut>(t_tile, half, sub, lane, norm_w + (is_q ? 0 : 128), tab,
                                      qkv.eps, row < M, xch, dst,
                                      sbase + L::kOutOff + (warp - 2) * 4096,
                                      is_q ? &tm_qo : &tm_ko, head0, m0 + sub * 32);
      } else if constexpr (L::kTmaOut && kQkv) {
        // v tiles: 32 rows x 32 columns per box through the two 2 KB buffers
        const uint32_t stage = sbase + L::kOutOff + (warp - 2) * 4096;
        const int r0 = m0 + sub * 32;
#pragma unroll 1
        for (int b = 0; b < 4; ++b) {
          uint32_t v[32];
          tmem_ld32(t_cols + 32 * b, v);
          tmem_wait_ld();
          reg_fence32(v);
          if (lane == 0) {
            if (b < 2) bulk_wait_read();  // earlier tiles' stores
            else bulk_wait_read_but_one();  // the store of box b - 2
          }
          __syncwarp();
          const uint32_t buf = stage + (b & 1) * 2048;
#pragma unroll
          for (int u = 0; u < 4; ++u)
            stage_row64(buf, lane, u,
                        pack_half2(__uint_as_float(v[8 * u + 0]), __uint_as_float(v[8 * u + 1])),
                        pack_half2(__uint_as_float(v[8 * u + 2]), __uint_as_float(v[8 * u + 3])),
                        pack_half2(__uint_as_float(v[8 * u + 4]), __uint_as_float(v[8 * u + 5])),
                        pack_half2(__uint_as_float(v[8 * u + 6]), __uint_as_float(v[8 * u + 7])));
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tm_out, buf, n0 - 3072 + 128 * half + 32 * b, r0);
            bulk_commit();
          }
        }
      } else if constexpr (L::kTmaOut) {
        // 32 rows x 64 columns at a time through this warp's staging buffer
        // (the swizzled layout of a 128-byte TMA box), then one TMA store: the
        // direct stores below touch 32 rows per warp instruction, and their
        // L1 traffic competed with the MMAs' operand reads (measured ~17%).
        const uint32_t stage = sbase + L::kOutOff + (warp - 2) * 4096;
        const int r0 = m0 + sub * 32;
#pragma unroll 1
        for (int b = 0; b < 2; ++b) {
          uint32_t v0[32], v1[32];
          tmem_ld32(t_cols + 64 * b, v0);
          tmem_ld32(t_cols + 64 * b + 32, v1);
          tmem_wait_ld();
          reg_fence32(v0);
          reg_fence32(v1);
          if (lane == 0) bulk_wait_read();  // the previous store has read the buffer
          __syncwarp();
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const uint32_t* src = u < 4 ? v0 + 8 * u : v1 + 8 * (u - 4);
            const uint32_t w0 = pack_half2(__uint_as_float(src[0]), __uint_as_float(src[1]));
            const uint32_t w1 = pack_half2(__uint_as_float(src[2]), __uint_as_float(src[3]));
            const uint32_t w2 = pack_half2(__uint_as_float(src[4]), __uint_as_float(src[5]));
            const uint32_t w3 = pack_half2(__uint_as_float(src[6]), __uint_as_float(src[7]));
            const uint32_t addr = stage + lane * 128 + ((static_cast<uint32_t>(u) ^ (lane & 7)) << 4);
            asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(w0), "r"(w1),
                         "r"(w2), "r"(w3)
                         : "memory");
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tm_out, stage, n0 + 128 * half + 64 * b, r0);  // rows >= M are clipped
            bulk_commit();
          }
        }
      } else {
        __half* orow = kQkv ? qkv.v_out + static_cast<int64_t>(row) * 1024 + (n0 - 3072)
                            : out + static_cast<int64_t>(row) * N + n0;
        uint4* dst = reinterpret_cast<uint4*>(orow + 128 * half);
#pragma unroll 1
        for (int ch = 0; ch < 4; ++ch) {
          uint32_t v[32];
          tmem_ld32(t_cols + 32 * ch, v);
          tmem_wait_ld();
          reg_fence32(v);
          if (row < M) {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              uint4 wv;
              wv.x = pack_half2(__uint_as_float(v[8 * q + 0]), __uint_as_float(v[8 * q + 1]));
              wv.y = pack_half2(__uint_as_float(v[8 * q + 2]), __uint_as_float(v[8 * q + 3]));
              wv.z = pack_half2(__uint_as_float(v[8 * q + 4]), __uint_as_float(v[8 * q + 5]));
              wv.w = pack_half2(__uint_as_float(v[8 * q + 6]), __uint_as_float(v[8 * q + 7]));
              dst[4 * ch + q] = wv;
            }
          }
        }
      }
      // this warp's reads of the accumulator are complete (wait::ld above)
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (kPair) mbar_arrive_cluster(acc_empty0 + 8u * acc);
        else mbar_arrive(bar(L::kAccEmpty + acc));
      }
    }
  }

  if (L::kTmaOut) bulk_wait_all();  // epilogue stores (no-op for threads without any)
  tc_fence_before();
  if (kPair) cluster_sync();  // no CTA leaves while its peer may still signal it
  else __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    if (kPair) tmem_dealloc_pair(tmem, 512);
    else tmem_dealloc(tmem, 512);
  }
}

template <bool kQkv, bool kPair, bool kGlu = false>
cudaError_t launch_gemm(const CUtensorMap& tm_a, const CUtensorMap& tm_w,
                        const CUtensorMap& tm_out, const CUtensorMap& tm_qo,
                        const CUtensorMap& tm_ko, __half* out, int M, int N, int K, int* status,
                        const QkvEpilogue& qkv, cudaStream_t stream) {
  using L = Layout<kQkv, kPair>;
  static bool configured[kMaxDevices] = {};
  static int sm_count[kMaxDevices] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  if (!configured[dev]) {
    e = cudaFuncSetAttribute(gemm_f16_kernel<kQkv, kPair, kGlu>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, L::kSmem);
    if (e == cudaSuccess)
      e = cudaDeviceGetAttribute(&sm_count[dev], cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  const int tiles = ((M + L::kRowsPerTile - 1) / L::kRowsPerTile) * (N / kBN);
  if (tiles <= 0) return cudaSuccess;
  if (kPair) {
    const int pairs = sm_count[dev] / 2;
    const int grid = 2 * (tiles < pairs ? tiles : pairs);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid, 1, 1);
    cfg.blockDim = dim3(kGemmThreads, 1, 1);
    cfg.dynamicSmemBytes = L::kSmem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, gemm_f16_kernel<kQkv, kPair, kGlu>, tm_a, tm_w, tm_out, tm_qo, tm_ko,
                              out, M, N, K, status, qkv);
  }
  const int grid = tiles < sm_count[dev] ? tiles : sm_count[dev];
  gemm_f16_kernel<kQkv, kPair, kGlu><<<grid, kGemmThreads, L::kSmem, stream>>>(
      tm_a, tm_w, tm_out, tm_qo, tm_ko, out, M, N, K, status, qkv);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_gemm_f16(const CUtensorMap& tm_a, const CUtensorMap& tm_w,
                            const CUtensorMap& tm_out, __half* out, int M, int N, int K,
                            int* status, bool pair, cudaStream_t stream) {
  // tm_out stands in for the q / k maps, which the plain epilogue never uses
  return pair ? launch_gemm<false, true>(tm_a, tm_w, tm_out, tm_out, tm_out, out, M, N, K, status,
                                         QkvEpilogue{}, stream)
              : launch_gemm<false, false>(tm_a, tm_w, tm_out, tm_out, tm_out, out, M, N, K, status,
                                          QkvEpilogue{}, stream);
}

cudaError_t launch_gemm_glu(const CUtensorMap& tm_a, const CUtensorMap& tm_w,
                            const CUtensorMap& tm_out, __half* out, int M, int N, int K,
                            int* status, bool pair, cudaStream_t stream) {
  return pair ? launch_gemm<false, true, true>(tm_a, tm_w, tm_out, tm_out, tm_out, out, M, N, K,
                                               status, QkvEpilogue{}, stream)
              : launch_gemm<false, false, true>(tm_a, tm_w, tm_out, tm_out, tm_out, out, M, N, K,
                                                status, QkvEpilogue{}, stream);
}

cudaError_t launch_gemm_qkv(const CUtensorMap& tm_a, const CUtensorMap& tm_w,
                            const CUtensorMap& tm_vo, const CUtensorMap& tm_qo,
                            const CUtensorMap& tm_ko, int M, int K, const QkvEpilogue& qkv,
                            int* status, bool pair, cudaStream_t stream) {
  return pair ? launch_gemm<true, true>(tm_a, tm_w, tm_vo, tm_qo, tm_ko, nullptr, M, 4096, K,
                                        status, qkv, stream)
              : launch_gemm<true, false>(tm_a, tm_w, tm_vo, tm_qo, tm_ko, nullptr, M, 4096, K,
                                         status, qkv, stream);
}

}  // namespace qwa
