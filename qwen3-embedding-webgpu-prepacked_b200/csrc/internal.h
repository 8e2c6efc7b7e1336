// Internal declarations shared by the .cu files of libqwa (not part of the ABI).
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace qwa {

constexpr int kQHeads = 16;
constexpr int kKVHeads = 8;
constexpr int kHeadDim = 128;
constexpr int kBlockM = 128;  // query rows per tile
constexpr int kBlockN = 128;  // keys per tile
constexpr int kSparseMaxSeq = 8192;             // src/webgpu/ops.ts:328
constexpr float kScale = 0.08838834764831845f;  // 1/sqrt(128), ops.ts:224
constexpr float kLog2e = 1.4426950408889634f;

// Attention mode -> 1 (sparse keep rule) or 0 (full causal). AUTO follows
// the reference: the sparse rule whenever the longest request has at most
// 8192 tokens (ops.ts:328). Modes are the qwa_mode values 0/1/2.
inline int resolve_sparse(int mode, int max_len) {
  if (mode == 1) return 0;
  if (mode == 2) return 1;
  return max_len <= kSparseMaxSeq ? 1 : 0;
}

// One unit of attention work: a 128-row query tile of one request for the
// two query heads (2g, 2g+1) that share key/value head g.
//   x = global row of the tile's first query, y = its position in the request,
//   z = request length, w = kv head g.
using AttnItem = int4;

// Work items of a packed batch: one per 128-row query tile per kv head.
inline size_t count_work_items(const int32_t* cu, int batch) {
  size_t n = 0;
  for (int b = 0; b < batch; ++b)
    n += static_cast<size_t>((cu[b + 1] - cu[b] + kBlockM - 1) / kBlockM) * kKVHeads;
  return n;
}

// Key-tile schedule of one query tile. Shared by host (work counts, plan
// ordering) and device (every warp role walks the same sequence).
struct KeySchedule {
  int n;         // key tiles visited
  int n_prefix;  // leading tiles that only cover keys < prefix (split mode)
  int ws;        // first key of the window tiles (split mode)
  int split;     // 1: prefix tiles + window tiles; 0: contiguous from key 0
};

__host__ __device__ inline KeySchedule make_key_schedule(int q0, int len, int sparse, int prefix,
                                                         int window) {
  KeySchedule s;
  const int q_last = (q0 + kBlockM < len ? q0 + kBlockM : len) - 1;
  const int ws = q0 - (window - 1);  // first key any query of the tile keeps in its window
  if (!sparse || ws <= prefix) {
    s.split = 0;
    s.n_prefix = 0;
    s.ws = 0;
    s.n = q_last / kBlockN + 1;
  } else {
    s.split = 1;
    s.n_prefix = (prefix + kBlockN - 1) / kBlockN;
    s.ws = ws;
    s.n = s.n_prefix + (q_last - ws) / kBlockN + 1;
  }
  return s;
}

// Keys of tile j that can hold a kept pair, rounded up to a multiple of 16
// (the MMA's N granularity): in split mode the last prefix tile stops at
// `prefix` and the last window tile at the tile's last query; all other
// tiles are kBlockN wide. Columns past the width are masked anyway (prefix
// cap or causal bound).
__host__ __device__ inline int key_tile_width(const KeySchedule& s, int j, int q_last, int prefix);

__host__ __device__ inline int key_tile_start(const KeySchedule& s, int j) {
  return (!s.split || j < s.n_prefix) ? j * kBlockN : s.ws + (j - s.n_prefix) * kBlockN;
}

__host__ __device__ inline int key_tile_width(const KeySchedule& s, int j, int q_last, int prefix) {
  if (!s.split) return kBlockN;
  int rem = kBlockN;
  if (j < s.n_prefix) rem = prefix - j * kBlockN;
  else if (j == s.n - 1) rem = q_last - key_tile_start(s, j) + 1;
  if (rem >= kBlockN) return kBlockN;
  return ((rem + 15) / 16) * 16;
}

// Attention kernel arguments besides the three tensor maps.
struct AttnArgs {
  const AttnItem* items;
  __half* out;  // [T, 16, 128]
  int sparse;
  int prefix;
  int window;
  float scale_log2;  // softmax scale * log2(e)
  int* status;       // device status word (DeviceError codes)
  unsigned long long* trace;  // QWA_TRACE builds only: per-role clock64 timeline
  unsigned long long wait_ns = 2000000000ull;  // bounded-wait limit of every mbarrier wait
  int skip_load = -1;  // test hook: CTA 0 never issues its K/V load number skip_load
  // Per-CTA item lists: CTA c runs items [cta_offsets[c], cta_offsets[c+1]) of
  // a grid of num_ctas. nullptr: CTA c runs items c, c + grid, c + 2 grid, ...
  const int* cta_offsets = nullptr;
  int num_ctas = 0;
};

// The items one CTA runs: it = beg, beg + stride, ... < end.
struct ItemRange {
  int beg, end, stride;
};
__device__ __forceinline__ ItemRange item_range(const AttnArgs& a, int num_items) {
  if (a.cta_offsets)
    return {a.cta_offsets[blockIdx.x], a.cta_offsets[blockIdx.x + 1], 1};
  return {static_cast<int>(blockIdx.x), num_items, static_cast<int>(gridDim.x)};
}

// Timeline layout of a QWA_TRACE build: trace[(cta * kTraceEvents + event) *
// kTraceIters + key_tile] = clock64() for the first kTraceCtas CTAs (key_tile
// counts the CTA's tiles across its work items).
// Rows of one TMA box of the attention output map tm_o.
constexpr int kOutBoxRows = 32;

#ifdef QWA_TRACE_ALL_CTAS
constexpr int kTraceCtas = 148;
#else
constexpr int kTraceCtas = 4;
#endif
constexpr int kTraceEvents = 69;
constexpr int kTraceIters = 256;

// tm_o: the output [T, 16, 128] with tm_q's geometry (full query tiles are
// written with TMA stores).
cudaError_t launch_attention(const CUtensorMap& tm_q, const CUtensorMap& tm_k,
                             const CUtensorMap& tm_v, const CUtensorMap& tm_o,
                             const AttnArgs& args, int num_items,
                             cudaStream_t stream);

cudaError_t launch_selftest_tile(const CUtensorMap& tm_a, const CUtensorMap& tm_b,
                                 const CUtensorMap& tm_v, float* c, float* d, int* status,
                                 cudaStream_t stream);

// Prologue. padded_sequence > 0: position = row % padded_sequence (the
// reference's padded layout); otherwise positions come from cu_seqlens.
cudaError_t launch_qk_norm_rope(const __half* qkv, int64_t qkv_stride, const float* q_weight,
                                const float* k_weight, const float2* rope_table, __half* q_out,
                                __half* k_out, const int32_t* cu_seqlens, int batch, int tokens,
                                int padded_sequence, float eps, cudaStream_t stream);

// Last-token L2 pool. cu_seqlens != nullptr: request b ends at row
// cu[b+1]-1; otherwise row b*sequence + lengths[b]-1 (padded layout).
cudaError_t launch_last_token_pool(const __half* hidden, int width, const int32_t* cu_seqlens,
                                   const uint32_t* lengths, int sequence, int batch, float* out,
                                   cudaStream_t stream);

constexpr int kMaxDevices = 64;

// silu(g) = g / (1 + exp(-g)) of the FFN's SwiGLU (ops.ts:74-102), with the
// fast exponential and division intrinsics (errors of a few f32 ulp, far
// below the f16 rounding of the product that follows). The unfused SwiGLU
// kernel and the gate_up GEMM's fused epilogue share it, so both give the
// same bits.
__device__ __forceinline__ float silu(float g) { return __fdividef(g, 1.0f + __expf(-g)); }

// C[M,N] = A[M,K] W[N,K]^T, f16 in/out, f32 accumulate (tcgen05). tm_a: 2-D
// map {K, M} box {64, 128}; tm_w: {K, N} box {64, kGemmWBoxRows(pair)};
// 128-byte swizzle. N % 256 == 0, K % 64 == 0. pair: 256-row tiles on CTA
// pairs (cta_group::2), for large M.
constexpr int kGemmWBoxRows(bool pair) { return pair ? 128 : 256; }
constexpr int kGemmPairMinRows = 4096;
// tm_out: the output C as a 2-D map {N, M}, box {64, 32}, 128-byte swizzle
// (CTA-pair launches write through it with TMA).
cudaError_t launch_gemm_f16(const CUtensorMap& tm_a, const CUtensorMap& tm_w,
                            const CUtensorMap& tm_out, __half* out, int M, int N, int K,
                            int* status, bool pair, cudaStream_t stream);
// The same GEMM with the FFN's SwiGLU in the epilogue: W's rows are the
// gate_up matrix interleaved in 128-row blocks (gate block b, then up block
// b), and the output is [M, N / 2] (tm_out: {N / 2, M}, box {64, 32}).
cudaError_t launch_gemm_glu(const CUtensorMap& tm_a, const CUtensorMap& tm_w,
                            const CUtensorMap& tm_out, __half* out, int M, int N, int K,
                            int* status, bool pair, cudaStream_t stream);

// Fused attn_qkv projection epilogue: per-head Q/K RMSNorm + RoPE on the q/k
// tiles, v written as [T, 1024]. Positions are row - cu[request(row)].
struct QkvEpilogue {
  __half* q_out = nullptr;  // [T, 16, 128]
  __half* k_out = nullptr;  // [T, 8, 128]
  __half* v_out = nullptr;  // [T, 1024]
  const float* q_weight = nullptr;
  const float* k_weight = nullptr;
  const float2* table = nullptr;  // (cos, sin) [positions, 64]
  const int32_t* cu = nullptr;    // device cu_seqlens [batch + 1]
  int batch = 0;
  float eps = 0.f;
};

// QKV projection (N = 4096) with the QkvEpilogue; K % 64 == 0. CTA-pair
// launches write through TMA maps with 32 x 32 boxes and 64-byte swizzle:
// tm_vo 2-D {1024, M}; tm_qo / tm_ko 3-D {128 dims, 16 / 8 heads, M}.
cudaError_t launch_gemm_qkv(const CUtensorMap& tm_a, const CUtensorMap& tm_w,
                            const CUtensorMap& tm_vo, const CUtensorMap& tm_qo,
                            const CUtensorMap& tm_ko, int M, int K, const QkvEpilogue& qkv,
                            int* status, bool pair, cudaStream_t stream);

// Q4_0 tile32-compact records (20 bytes: f16 scale, 2 pad bytes, 16 bytes of
// nibbles) -> f16 W[n, k] row-major.
cudaError_t launch_q40_tile32_dequant(const uint8_t* packed, int n, int k, __half* out,
                                      cudaStream_t stream);

// Residual add + RMSNorm (ops.ts:21-64); x updated in place when has_residual.
cudaError_t launch_rms_norm(__half* x, const __half* residual, const float* weight,
                            __half* normalized, int rows, int width, bool has_residual, float eps,
                            cudaStream_t stream);

// Small-M projection from Q4_0 tile32 records (m <= kQ40SmallMaxRows, n % 128
// == 0, k % 64 == 0): tm_x is the 2-D map of A {k, m} with box {64, m padded
// to 16}; ws holds splits * m * n floats of partial sums.
constexpr int kQ40SmallMaxRows = 64;
int q40_small_splits(int n, int k, int sms);
cudaError_t launch_q40_small_gemm(const CUtensorMap& tm_x, const uint8_t* packed, __half* out,
                                  int m, int n, int k, int splits, float* ws, int* status,
                                  cudaStream_t stream);

// SwiGLU: out[r, c] = f16(silu(g) * u), g = combined[r, c], u = combined[r, width + c].
cudaError_t launch_swiglu(const __half* combined, __half* out, int rows, int width,
                          cudaStream_t stream);

// Token rows of a Q6_K matrix [vocab, width] as f16; ids >= vocab give zeros.
cudaError_t launch_q6k_embedding(const uint32_t* ids, const uint8_t* table, int vocab,
                                 __half* out, int tokens, int width, cudaStream_t stream);

}  // namespace qwa
