// Device helpers shared by the attention kernels: MMA issue for S = Q K^T and
// O += P V on 128-key tiles, the kept-pair mask, the row max, and the exp2 of
// a 32-score chunk packed to f16 P.
#pragma once
#include <cuda_fp16.h>

#include "internal.h"
#include "ptx.cuh"

namespace qwa {
namespace attn {

constexpr uint32_t kTileBytes = kBlockN * kHeadDim * 2;  // 32 KB (two 16 KB swizzled halves)
constexpr uint32_t kHalfBytes = kTileBytes / 2;
constexpr uint32_t kIdescS = idesc_f16_f32(128, 128, false);   // Q K^T, both K-major
constexpr uint32_t kIdescPV = idesc_f16_f32(128, 128, true);   // P V, V N-contiguous
constexpr uint32_t kTmemCols = 512;

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// S = Q K^T for a 128x128 tile, K = 128 in eight K=16 steps. Q and K tiles are
// two 16 KB halves (dims 0-63, 64-127), each 128 rows x 128 B, 128B-swizzled.
// q_desc/k_desc are the tiles' base descriptors (built once per CTA): a K step
// only adds its byte offset >> 4 to the start-address field, so nothing but
// the MMAs sits between consecutive issues. (Building a 64-bit descriptor
// between tcgen05.mma issues halves the issue rate of a single thread:
// measured 130 vs 64 cycles per 128x128x16 MMA on B200.)
__device__ __forceinline__ void issue_qk(uint32_t d_tmem, uint64_t q_desc, uint64_t k_desc,
                                         uint32_t idesc = kIdescS) {
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) {
    const uint64_t off = ((kk >> 2) * kHalfBytes + (kk & 3) * 32) >> 4;
    mma_ss(d_tmem, q_desc + off, k_desc + off, idesc, kk > 0 ? 1u : 0u);
  }
}

// O (+)= P V: P (f16) from TMEM columns [p_tmem, p_tmem+64), V tile N-contiguous
// (key rows of 128 B per 64-dim half): K=16 step = 16 key rows = 2048 B;
// LBO = distance between dim halves, SBO = 8 key rows (both in v_desc).
// nk = key steps of 16 actually used (tile width / 16).
__device__ __forceinline__ void issue_pv(uint32_t d_tmem, uint32_t p_tmem, uint64_t v_desc,
                                         bool accumulate, int nk = 8) {
#pragma unroll
  for (int kk = 0; kk < 8; ++kk)
    if (kk < nk)
      mma_ts(d_tmem, p_tmem + kk * 8, v_desc + ((kk * 2048) >> 4), kIdescPV,
             (accumulate || kk > 0) ? 1u : 0u);
}
// One half of PV: K steps 4*half .. 4*half+3 (keys 64*half .. 64*half+63),
// whose P the softmax publishes separately (kPLo / kPHi).
__device__ __forceinline__ void issue_pv_half(uint32_t d_tmem, uint32_t p_tmem, uint64_t v_desc,
                                              bool accumulate, int nk, int half) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int kk = 4 * half + i;
    if (kk < nk)
      mma_ts(d_tmem, p_tmem + kk * 8, v_desc + ((kk * 2048) >> 4), kIdescPV,
             (accumulate || kk > 0) ? 1u : 0u);
  }
}

__device__ __forceinline__ uint32_t low_bits(int n) {
  return n <= 0 ? 0u : (n >= 32 ? 0xffffffffu : ((1u << n) - 1u));
}

// Scores of keys k0..k0+31 for query q: dropped pairs become -inf. The kept
// set {k <= q, k < kcap, (k < prefix || k + window > q)} is built as a 32-bit
// mask so the per-element cost is one bit test.
__device__ __forceinline__ void mask_chunk(uint32_t (&a)[32], int k0, int q, int kcap, int sparse,
                                           int prefix, int window) {
  uint32_t m = low_bits(min(q, kcap - 1) - k0 + 1);
  if (sparse) m &= low_bits(prefix - k0) | ~low_bits(q - window + 1 - k0);
  // The window and causal edges are diagonals: a warp's 32 rows cut at most
  // two of a tile's four chunks, and the others need no per-element work.
  if (__all_sync(0xffffffffu, m == 0xffffffffu)) return;
#pragma unroll
  for (int c = 0; c < 32; ++c)
    if (!((m >> c) & 1u)) a[c] = __float_as_uint(-INFINITY);
}

__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Row max of 32 raw scores: four independent chains of 3-input max (a single
// dependent chain costs ~400 cycles per 128-column row).
__device__ __forceinline__ float chunk_max(const uint32_t (&a)[32]) {
  float m[4];
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const uint32_t* p = a + 8 * c;
    float v = fmax3(__uint_as_float(p[0]), __uint_as_float(p[1]), __uint_as_float(p[2]));
    v = fmax3(v, __uint_as_float(p[3]), __uint_as_float(p[4]));
    v = fmax3(v, __uint_as_float(p[5]), __uint_as_float(p[6]));
    m[c] = fmaxf(v, __uint_as_float(p[7]));
  }
  return fmax3(fmaxf(m[0], m[1]), m[2], m[3]);
}

// p = 2^(s*scale - m) for 32 raw scores; packs them as f16 pairs into a[0..15]
// (in place, ascending, so every pair is read before its slot is reused) and
// returns their fp32 sum.
// exp2(a * scale - m) of 32 scores, packed to f16 pairs in a[0..15]; returns
// their sum (even and odd columns summed separately, then added). The scale
// and the sums run as paired f32 instructions (same rounding per lane).
__device__ __forceinline__ float exp_pack_chunk(uint32_t (&a)[32], float scale, float m) {
  const uint64_t s2 = f2_pack(scale, scale), nm2 = f2_pack(-m, -m);
  uint64_t sum2 = f2_pack(0.f, 0.f);
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    float y0, y1;
    f2_unpack(fma2(f2_pack(__uint_as_float(a[2 * i]), __uint_as_float(a[2 * i + 1])), s2, nm2),
              y0, y1);
    const float e0 = ex2(y0), e1 = ex2(y1);
    sum2 = add2(sum2, f2_pack(e0, e1));
    a[i] = pack_half2(e0, e1);
  }
  float sum0, sum1;
  f2_unpack(sum2, sum0, sum1);
  return sum0 + sum1;
}

__device__ __forceinline__ bool tile_needs_mask(const KeySchedule& s, int j, int ks, int q0,
                                                int q_last, int sparse, int prefix, int window) {
  const int k_end = ks + kBlockN - 1;
  if (k_end > q0) return true;  // causal edge
  if (!sparse) return false;
  if (s.split && j < s.n_prefix) return k_end >= prefix;  // prefix cut only
  // window edge: some key of the tile at or above the prefix falls out of
  // some query's window (keys below the prefix are always kept)
  return k_end >= prefix && ks + window <= q_last;
}


}  // namespace attn
}  // namespace qwa
