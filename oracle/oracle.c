/*
 * CPU ORACLE -- test infrastructure only, never the product path.
 *
 * A plain-C restatement of the math of the reference's attention hot path
 * (shihanqu/qwen3-embedding-webgpu-prepacked, WGSL shaders in
 * src/webgpu/ops.ts), used by tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py as the checker.
 * Nothing in the shipped library links or calls this file.
 *
 * Parity status: UNPINNED against the reference itself. The reference has no
 * CPU implementation of attention, RMSNorm or RoPE (its src/math holds only an
 * f32->f16 converter) and its shaders run only under a browser WebGPU, which is
 * unavailable on this box. What is pinned: the f32->f16 conversion
 * (src/math/f16.ts:4-25) and halfToFloat known answers
 * (tests/quantization.test.ts:5-9), plus analytic known-answer tests of
 * the mask, RoPE and softmax semantics (tests/test_oracle.py).
 *
 * Numerics: inputs are the f16 values the kernels see; all arithmetic is
 * fp64; results are returned unrounded (fp64) so a test can measure the
 * device's error against the exact math.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* IEEE binary16 -> double. Follows halfToFloat semantics
 * (src/gguf/quantization.ts; KATs tests/quantization.test.ts:5-9). */
static double half_to_double(uint16_t h) {
  int sign = (h >> 15) & 1;
  int exponent = (h >> 10) & 0x1f;
  int mantissa = h & 0x3ff;
  double v;
  if (exponent == 0) v = ldexp((double)mantissa, -24);
  else if (exponent == 31) v = mantissa ? NAN : INFINITY;
  else v = ldexp((double)(mantissa | 0x400), exponent - 25);
  return sign ? -v : v;
}

double oracle_half_to_double(uint16_t h) { return half_to_double(h); }

/* All 65536 f16 values as doubles, so the inner loops decode by lookup. */
static double h2d_lut[65536];
static int h2d_ready = 0;
static void init_lut(void) {
  if (h2d_ready) return;
  for (int i = 0; i < 65536; ++i) h2d_lut[i] = half_to_double((uint16_t)i);
  h2d_ready = 1;
}
#define H2D(x) h2d_lut[(x)]

/* f32 -> f16 bits, round to nearest even; restates floatToHalf
 * (src/math/f16.ts:4-25) bit for bit, including its subnormal path. */
uint16_t oracle_float_to_half(float value) {
  uint32_t bits;
  memcpy(&bits, &value, 4);
  uint32_t sign = (bits >> 16) & 0x8000u;
  int exponent = (int)((bits >> 23) & 0xffu) - 127 + 15;
  uint32_t mantissa = bits & 0x7fffffu;
  if (exponent <= 0) {
    if (exponent < -10) return (uint16_t)sign;
    mantissa = (mantissa | 0x800000u) >> (1 - exponent);
    return (uint16_t)(sign | ((mantissa + 0x1000u) >> 13));
  }
  if (exponent >= 31) return (uint16_t)(sign | 0x7c00u);
  if (mantissa & 0x1000u) {
    mantissa += 0x2000u;
    if (mantissa & 0x800000u) {
      mantissa = 0;
      exponent += 1;
      if (exponent >= 31) return (uint16_t)(sign | 0x7c00u);
    }
  }
  return (uint16_t)(sign | ((uint32_t)exponent << 10) | (mantissa >> 13));
}

/* RoPE cos/sin table, src/webgpu/model.ts:76-83: angle = pos * theta^(-d/64)
 * computed in double, stored as f32 pairs (cos, sin) at [(pos*64 + d)*2]. */
void oracle_rope_table(double theta, int positions, float *table) {
  for (int p = 0; p < positions; ++p)
    for (int d = 0; d < 64; ++d) {
      double angle = (double)p * pow(theta, -(double)d / 64.0);
      table[(p * 64 + d) * 2] = (float)cos(angle);
      table[(p * 64 + d) * 2 + 1] = (float)sin(angle);
    }
}

/* Position of every packed token inside its request (cu_seqlens form). */
static int position_of(const int32_t *cu, int batch, int64_t t) {
  int lo = 0, hi = batch - 1;
  while (lo < hi) {
    int mid = (lo + hi + 1) / 2;
    if (cu[mid] <= t) lo = mid; else hi = mid - 1;
  }
  return (int)(t - cu[lo]);
}

/* Fused per-head RMSNorm + RoPE, src/webgpu/ops.ts:104-150.
 * For token t and each of 16 q-heads and 8 k-heads:
 *   x = qkv[t*stride + (q ? 0 : 2048) + h*128 + d]
 *   n = x / sqrt(sum(x^2)/128 + eps) * w[d]         (weights before RoPE)
 *   out[d] = n[d]*cos + (d < 64 ? -n[d+64] : n[d-64]) * sin
 * with (cos, sin) = table[pos*64 + d%64], pos = position inside the request
 * (the reference's t % sequence for a padded batch).
 * q_out: [T,16,128], k_out: [T,8,128], both fp64 unrounded. */
void oracle_qk_norm_rope(const uint16_t *qkv, int64_t stride, const float *q_weight,
                         const float *k_weight, const float *table, const int32_t *cu,
                         int batch, double eps, double *q_out, double *k_out) {
  int64_t tokens = cu[batch];
#pragma omp parallel for schedule(static)
  for (int64_t t = 0; t < tokens; ++t) {
    int pos = position_of(cu, batch, t);
    for (int ch = 0; ch < 24; ++ch) {
      int is_q = ch < 16;
      int h = is_q ? ch : ch - 16;
      const uint16_t *src = qkv + t * stride + (is_q ? 0 : 2048) + h * 128;
      const float *w = is_q ? q_weight : k_weight;
      double x[128], n[128], sum = 0.0;
      for (int d = 0; d < 128; ++d) { x[d] = half_to_double(src[d]); sum += x[d] * x[d]; }
      double inv = 1.0 / sqrt(sum / 128.0 + eps);
      for (int d = 0; d < 128; ++d) n[d] = x[d] * inv * (double)w[d];
      double *dst = is_q ? q_out + (t * 16 + h) * 128 : k_out + (t * 8 + h) * 128;
      for (int d = 0; d < 128; ++d) {
        double c = table[(pos * 64 + d % 64) * 2], s = table[(pos * 64 + d % 64) * 2 + 1];
        double rot = d < 64 ? -n[d + 64] : n[d - 64];
        dst[d] = n[d] * c + rot * s;
      }
    }
  }
}

/* Keep predicate of src/webgpu/ops.ts:220 for one request:
 * keep key k for query q iff k <= q and, in sparse mode,
 * (k < prefix || k + window > q). prefix/window are the reference's
 * min(S,176) / min(S,432); using the unclipped constants gives the same
 * kept set for every valid query (q < S). */
int oracle_keep(int q, int k, int sparse, int prefix, int window) {
  if (k > q) return 0;
  if (!sparse) return 1;
  return (k < prefix) || (k + window > q);
}

/* Mode rule of src/webgpu/ops.ts:328: the tiled kernel (sparse predicate)
 * runs for sequence <= 8192, the chunked full-causal path above that.
 * mode: 0 = AUTO (that rule on max_seqlen), 1 = FULL, 2 = SPARSE. */
int oracle_resolve_sparse(int mode, int max_seqlen) {
  if (mode == 1) return 0;
  if (mode == 2) return 1;
  return max_seqlen <= 8192;
}

/* Causal GQA attention, src/webgpu/ops.ts:168-241 (math only, fp64):
 * out[t,h,:] = sum_k softmax_k(q.k / sqrt(128)) v_k over kept keys of the
 * same request, kv head = h / 2. q: [T,16,128] f16, k: [T,8,128] f16,
 * v: f16 at v[t*v_stride + v_offset + g*128 + d]. out: [T,16,128] fp64. */
void oracle_attention(const uint16_t *q, const uint16_t *k, const uint16_t *v, int64_t v_stride,
                      int64_t v_offset, const int32_t *cu, int batch, int mode, int prefix,
                      int window, double *out) {
  int max_len = 0;
  for (int b = 0; b < batch; ++b) if (cu[b + 1] - cu[b] > max_len) max_len = cu[b + 1] - cu[b];
  int sparse = oracle_resolve_sparse(mode, max_len);
  int64_t tokens = cu[batch];
  init_lut();
  const double scale = 0.08838834764831845; /* 1/sqrt(128), ops.ts:224 */
#pragma omp parallel
  {
    double *scores = (double *)malloc(sizeof(double) * (size_t)(max_len > 0 ? max_len : 1));
    double acc[128], qv[128];
#pragma omp for schedule(dynamic, 16)
    for (int64_t idx = 0; idx < tokens * 16; ++idx) {
      int64_t t = idx / 16;
      int h = (int)(idx % 16), g = h / 2;
      int b = 0;
      while (cu[b + 1] <= t) ++b;
      int64_t base = cu[b];
      int qpos = (int)(t - base);
      for (int d = 0; d < 128; ++d) qv[d] = H2D(q[(t * 16 + h) * 128 + d]);
      double mx = -INFINITY;
      for (int kp = 0; kp <= qpos; ++kp) {
        if (!oracle_keep(qpos, kp, sparse, prefix, window)) { scores[kp] = -INFINITY; continue; }
        const uint16_t *kr = k + ((base + kp) * 8 + g) * 128;
        double s = 0.0;
        for (int d = 0; d < 128; ++d) s += qv[d] * H2D(kr[d]);
        s *= scale;
        scores[kp] = s;
        if (s > mx) mx = s;
      }
      double den = 0.0;
      for (int d = 0; d < 128; ++d) acc[d] = 0.0;
      for (int kp = 0; kp <= qpos; ++kp) {
        if (scores[kp] == -INFINITY) continue;
        double p = exp(scores[kp] - mx);
        den += p;
        const uint16_t *vr = v + (base + kp) * v_stride + v_offset + g * 128;
        for (int d = 0; d < 128; ++d) acc[d] += p * H2D(vr[d]);
      }
      for (int d = 0; d < 128; ++d) out[(t * 16 + h) * 128 + d] = acc[d] / den;
    }
    free(scores);
  }
}

/* Same math as oracle_attention for a sample of output rows only: rows[i]
 * = t*16 + h; out_rows is [nrows,128] fp64. Lets tests check full-size
 * workloads (e.g. 16x5000) against the oracle on a bounded sample. */
void oracle_attention_rows(const uint16_t *q, const uint16_t *k, const uint16_t *v,
                           int64_t v_stride, int64_t v_offset, const int32_t *cu, int batch,
                           int mode, int prefix, int window, const int64_t *rows, int64_t nrows,
                           double *out_rows) {
  int max_len = 0;
  for (int b = 0; b < batch; ++b) if (cu[b + 1] - cu[b] > max_len) max_len = cu[b + 1] - cu[b];
  int sparse = oracle_resolve_sparse(mode, max_len);
  const double scale = 0.08838834764831845;
  init_lut();
#pragma omp parallel
  {
    double *scores = (double *)malloc(sizeof(double) * (size_t)(max_len > 0 ? max_len : 1));
    double acc[128], qv[128];
#pragma omp for schedule(dynamic, 1)
    for (int64_t i = 0; i < nrows; ++i) {
      int64_t t = rows[i] / 16;
      int h = (int)(rows[i] % 16), g = h / 2;
      int b = 0;
      while (cu[b + 1] <= t) ++b;
      int64_t base = cu[b];
      int qpos = (int)(t - base);
      for (int d = 0; d < 128; ++d) qv[d] = H2D(q[(t * 16 + h) * 128 + d]);
      double mx = -INFINITY;
      for (int kp = 0; kp <= qpos; ++kp) {
        if (!oracle_keep(qpos, kp, sparse, prefix, window)) { scores[kp] = -INFINITY; continue; }
        const uint16_t *kr = k + ((base + kp) * 8 + g) * 128;
        double s = 0.0;
        for (int d = 0; d < 128; ++d) s += qv[d] * H2D(kr[d]);
        scores[kp] = s * scale;
        if (scores[kp] > mx) mx = scores[kp];
      }
      double den = 0.0;
      for (int d = 0; d < 128; ++d) acc[d] = 0.0;
      for (int kp = 0; kp <= qpos; ++kp) {
        if (scores[kp] == -INFINITY) continue;
        double p = exp(scores[kp] - mx);
        den += p;
        const uint16_t *vr = v + (base + kp) * v_stride + v_offset + g * 128;
        for (int d = 0; d < 128; ++d) acc[d] += p * H2D(vr[d]);
      }
      for (int d = 0; d < 128; ++d) out_rows[i * 128 + d] = acc[d] / den;
    }
    free(scores);
  }
}

/* Number of kept (q,k) pairs of one request of length len (for FLOP counts). */
int64_t oracle_kept_pairs(int len, int sparse, int prefix, int window) {
  int64_t n = 0;
  for (int q = 0; q < len; ++q) {
    if (!sparse) { n += q + 1; continue; }
    for (int k = 0; k <= q; ++k) n += oracle_keep(q, k, sparse, prefix, window);
  }
  return n;
}

/* Use n OpenMP threads for the calls that follow (n <= 0: leave unchanged). */
void oracle_set_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

int oracle_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* Last-token L2 pooling, src/webgpu/ops.ts:347-359 (poolShader): request b's
 * embedding is row cu[b+1]-1 of hidden [T, width] (f16) scaled by
 * 1/sqrt(sum of squares), computed in fp64 here (the shader sums in f32).
 * An empty request gives a zero row (the reference never pools one: every
 * request carries at least its EOS token). */
void oracle_last_token_pool(const uint16_t *hidden, int width, const int32_t *cu, int batch,
                            double *out) {
  init_lut();
  for (int b = 0; b < batch; ++b) {
    double *dst = out + (int64_t)b * width;
    if (cu[b + 1] <= cu[b]) {
      for (int i = 0; i < width; ++i) dst[i] = 0.0;
      continue;
    }
    const uint16_t *row = hidden + (int64_t)(cu[b + 1] - 1) * width;
    double ss = 0.0;
    for (int i = 0; i < width; ++i) {
      const double x = half_to_double(row[i]);
      ss += x * x;
    }
    const double inv = 1.0 / sqrt(ss);
    for (int i = 0; i < width; ++i) dst[i] = half_to_double(row[i]) * inv;
  }
}

/* f32 -> f16 bits with IEEE round-to-nearest-even (the conversion WGSL's
 * f16() and CUDA's __float2half_rn perform; floatToHalf in src/math/f16.ts
 * rounds ties away from zero instead and is only used for host uploads). */
static uint16_t float_to_half_rne(float value) {
  uint32_t bits;
  memcpy(&bits, &value, 4);
  const uint32_t sign = (bits >> 16) & 0x8000u;
  const uint32_t absb = bits & 0x7fffffffu;
  if (absb >= 0x7f800000u) return (uint16_t)(sign | 0x7c00u | (absb > 0x7f800000u ? 0x200u : 0));
  if (absb >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* rounds to >= 65520: inf */
  int exponent = (int)(absb >> 23) - 127 + 15;
  uint32_t mantissa = (absb & 0x7fffffu) | 0x800000u;
  int shift;
  if (exponent <= 0) {
    if (exponent < -10) return (uint16_t)sign;
    shift = 14 - exponent; /* subnormal: keep 10 bits of m * 2^(e-1) */
    exponent = 0;
  } else {
    shift = 13;
  }
  uint32_t kept = mantissa >> shift;
  const uint32_t rest = mantissa & ((1u << shift) - 1);
  const uint32_t halfway = 1u << (shift - 1);
  if (rest > halfway || (rest == halfway && (kept & 1u))) kept += 1;
  /* kept includes the implicit bit for normals; adding the exponent field
   * lets a mantissa carry roll into the exponent */
  uint32_t out = exponent == 0 ? kept : (((uint32_t)(exponent - 1) << 10) + kept);
  return (uint16_t)(sign | out);
}

uint16_t oracle_float_to_half_rne(float value) { return float_to_half_rne(value); }

/* Residual add + RMSNorm, src/webgpu/ops.ts:21-57 (rmsNormShader), in the
 * shader's f32 arithmetic: with residual, v = f32(x) + f32(r) (exact in f32)
 * and x := f16_rne(v); sum of v^2 (kept in fp64 here, f32 tree in the
 * shader); inv = 1/sqrt(sum/width + eps); normalized = f16_rne(x*inv*w).
 * x is updated in place like the shader's read_write binding. */
void oracle_rms_norm(uint16_t *x, const uint16_t *residual, const float *weight,
                     uint16_t *normalized, int rows, int width, float eps, int has_residual) {
  init_lut();
#pragma omp parallel for schedule(static)
  for (int row = 0; row < rows; ++row) {
    uint16_t *xr = x + (int64_t)row * width;
    const uint16_t *rr = residual ? residual + (int64_t)row * width : NULL;
    double ss = 0.0;
    for (int i = 0; i < width; ++i) {
      float v = (float)half_to_double(xr[i]);
      if (has_residual) {
        v += (float)half_to_double(rr[i]);
        xr[i] = float_to_half_rne(v);
      }
      ss += (double)v * (double)v;
    }
    const float inv = (float)(1.0 / sqrt(ss / width + (double)eps));
    uint16_t *nr = normalized + (int64_t)row * width;
    for (int i = 0; i < width; ++i)
      nr[i] = float_to_half_rne((float)half_to_double(xr[i]) * inv * weight[i]);
  }
}

/* ------------------------------------------------------------------------
 * "WGSL-faithful" mode: the reference's own arithmetic, not the exact math.
 *
 * Emulates tiledFlashAttentionShader (src/webgpu/ops.ts:168-241) with its
 * rounding points, for one padded request of `S` rows (S <= 8192, the tiled
 * path of ops.ts:328): 16-row query tiles x 16-key blocks, the block-skip
 * test (:209), the keep test (:220), f16 dot products summed in f32 (:221),
 * the f32 scale (:222), update_stats (:186-193: f32 block max and exps, f16
 * weights, alphas, betas and running denominator), the f16 P.V and output
 * accumulators (:227-232) and the f16 division (:238).
 *
 * WGSL leaves two things to the implementation, so they are parameters:
 *   fused = 1: a*b + c in f16 is one rounding (an FMA, as GPU compilers
 *              usually contract it); 0: product and sum rounded separately.
 *   exp: C's expf (the shader's f32 exp has implementation-defined ulp
 *        error; both are close to the exact exponential).
 * The f16 dot(vec4, vec4) is an FMA chain over the four lanes (one rounding
 * per lane with fused = 1, two without).
 * ------------------------------------------------------------------------ */

/* double -> nearest f16 value (ties to even), as a double; +-inf past 65504 */
static double rf16(double x) {
  if (x == 0.0 || isnan(x) || isinf(x)) return x;
  int e;
  frexp(x, &e);
  int lead = e - 1;
  if (lead < -14) lead = -14; /* subnormal spacing 2^-24 */
  const double step = ldexp(1.0, lead - 10);
  const double r = nearbyint(x / step) * step;
  if (fabs(r) > 65504.0) return copysign(INFINITY, x);
  return r;
}

static double f16_fma(double a, double b, double c, int fused) {
  return fused ? rf16(a * b + c) : rf16(rf16(a * b) + c);
}

/* q: [T,16,128] f16, k: [T,8,128] f16, v at v[t*v_stride + v_offset + g*128],
 * requests of cu (each its own padded sequence), out: [T,16,128] as the f16
 * values the shader would write (in doubles). */
void oracle_attention_wgsl(const uint16_t *q, const uint16_t *k, const uint16_t *v,
                           int64_t v_stride, int64_t v_offset, const int32_t *cu, int batch,
                           int fused, double *out) {
  init_lut();
  int64_t n_units = 0; /* (request, head, 16-row tile) */
  for (int b = 0; b < batch; ++b) n_units += (int64_t)((cu[b + 1] - cu[b] + 15) / 16) * 16;
  const float scale = 0.08838834764831845f;
  const float lowest = -3.402823e38f;
#pragma omp parallel for schedule(dynamic, 4)
  for (int64_t u = 0; u < n_units; ++u) {
    int b = 0;
    int64_t acc = 0;
    for (;; ++b) {
      const int64_t n = (int64_t)((cu[b + 1] - cu[b] + 15) / 16) * 16;
      if (u < acc + n) break;
      acc += n;
    }
    const int64_t local = u - acc;
    const int head = (int)(local % 16), gx = (int)(local / 16), kv = head / 2;
    const int S = cu[b + 1] - cu[b];
    const int64_t base = cu[b];
    float maxima[16];
    double den[16], total[16][128], weights[16][16], alpha16[16], beta16[16];
    for (int r = 0; r < 16; ++r) {
      maxima[r] = lowest;
      den[r] = 0.0;
      for (int d = 0; d < 128; ++d) total[r][d] = 0.0;
    }
    const int key_limit = S < (gx + 1) * 16 ? S : (gx + 1) * 16;
    const int prefix_size = S < 176 ? S : 176, local_window = S < 432 ? S : 432;
    const int qts = gx * 16;
    const int local_start = qts + 1 > local_window ? qts + 1 - local_window : 0;
    for (int kb = 0; kb < key_limit; kb += 16) {
      if (kb >= prefix_size && kb + 15 < local_start) continue;
      for (int r = 0; r < 16; ++r) {
        const int qp = qts + r;
        float sc[16];
        for (int c = 0; c < 16; ++c) {
          const int kp = kb + c;
          float s = lowest;
          if (qp < S && kp <= qp && kp < S && (kp < prefix_size || kp + local_window > qp)) {
            s = 0.f;
            const uint16_t *qr = q + ((base + qp) * 16 + head) * 128;
            const uint16_t *kr = k + ((base + kp) * 8 + kv) * 128;
            for (int d4 = 0; d4 < 32; ++d4) {
              double dv = rf16(H2D(qr[4 * d4]) * H2D(kr[4 * d4]));
              for (int i = 1; i < 4; ++i)
                dv = f16_fma(H2D(qr[4 * d4 + i]), H2D(kr[4 * d4 + i]), dv, fused);
              s += (float)dv;
            }
            s *= scale;
          }
          sc[c] = s;
        }
        /* update_stats (ops.ts:186-193) */
        float block_max = lowest;
        for (int c = 0; c < 16; ++c) block_max = fmaxf(block_max, sc[c]);
        float block_den = 0.f;
        for (int c = 0; c < 16; ++c) {
          const float w = expf(sc[c] - block_max);
          weights[r][c] = rf16(w);
          block_den += w;
        }
        const float next_max = fmaxf(maxima[r], block_max);
        const float alpha = expf(maxima[r] - next_max), beta = expf(block_max - next_max);
        alpha16[r] = rf16(alpha);
        beta16[r] = rf16(beta);
        den[r] = f16_fma(den[r], alpha16[r], rf16(beta * block_den), fused);
        maxima[r] = next_max;
      }
      /* P.V in f16 and the rescaled running output (ops.ts:227-232) */
      for (int r = 0; r < 16; ++r)
        for (int d = 0; d < 128; ++d) {
          double av = 0.0;
          for (int c = 0; c < 16; ++c) {
            const int kp = kb + c;
            const double vv =
                kp < S ? H2D(v[(base + kp) * v_stride + v_offset + kv * 128 + d]) : 0.0;
            av = f16_fma(weights[r][c], vv, av, fused);
          }
          total[r][d] = f16_fma(total[r][d], alpha16[r], rf16(beta16[r] * av), fused);
        }
    }
    for (int r = 0; r < 16; ++r) {
      const int qp = qts + r;
      if (qp >= S) continue;
      for (int d = 0; d < 128; ++d)
        out[((base + qp) * 16 + head) * 128 + d] = rf16(total[r][d] / den[r]);
    }
  }
}
