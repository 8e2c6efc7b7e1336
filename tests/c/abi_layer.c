/*
 * One prologue + attention layer through the C ABI alone (include/qwa.h), as a
 * host program in C would call it: no Python and no torch. Used by
 * tests/test_gpu_c_abi.py, which writes the inputs and checks the outputs
 * against the oracle.
 *
 *   abi_layer <dir>
 *
 * <dir>/in.bin:  int32 batch, int32 cu[batch+1], f32 q_w[128], f32 k_w[128],
 *                f16 qkv[T*4096]
 * <dir>/out.bin: f16 q[T*2048], f16 k[T*1024], f16 o[T*2048]
 * Exit status 0 on success; a failing call prints qwa_last_error.
 */
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>

#include "qwa.h"

#define CK(x)                                                   \
  do {                                                          \
    cudaError_t e_ = (x);                                       \
    if (e_ != cudaSuccess) {                                    \
      fprintf(stderr, "%s: %s\n", #x, cudaGetErrorString(e_));  \
      return 2;                                                 \
    }                                                           \
  } while (0)
#define QK(ctx, x)                                                          \
  do {                                                                      \
    qwa_status s_ = (x);                                                    \
    if (s_ != QWA_OK) {                                                     \
      fprintf(stderr, "%s: %s (%s)\n", #x, qwa_status_string(s_),           \
              (ctx) ? qwa_last_error(ctx) : "");                            \
      return 3;                                                             \
    }                                                                       \
  } while (0)

static int read_all(FILE* f, void* p, size_t n) { return fread(p, 1, n, f) == n; }

int main(int argc, char** argv) {
  if (argc != 2) return 1;
  char path[4096];
  snprintf(path, sizeof path, "%s/in.bin", argv[1]);
  FILE* f = fopen(path, "rb");
  if (!f) return 1;
  int32_t batch = 0;
  if (!read_all(f, &batch, 4) || batch < 1) return 1;
  int32_t* cu = malloc(sizeof(int32_t) * (batch + 1));
  float qw[128], kw[128];
  if (!read_all(f, cu, sizeof(int32_t) * (batch + 1)) || !read_all(f, qw, sizeof qw) ||
      !read_all(f, kw, sizeof kw))
    return 1;
  const size_t T = (size_t)cu[batch];
  uint16_t* qkv = malloc(T * 4096 * 2);
  if (!read_all(f, qkv, T * 4096 * 2)) return 1;
  fclose(f);

  qwa_ctx* ctx = NULL;
  QK(ctx, qwa_create(0, &ctx));
  void *d_qkv, *d_q, *d_k, *d_o;
  float *d_qw, *d_kw;
  CK(cudaMalloc(&d_qkv, T * 4096 * 2));
  CK(cudaMalloc(&d_q, T * 2048 * 2));
  CK(cudaMalloc(&d_k, T * 1024 * 2));
  CK(cudaMalloc(&d_o, T * 2048 * 2));
  CK(cudaMalloc((void**)&d_qw, sizeof qw));
  CK(cudaMalloc((void**)&d_kw, sizeof kw));
  CK(cudaMemcpy(d_qkv, qkv, T * 4096 * 2, cudaMemcpyHostToDevice));
  CK(cudaMemcpy(d_qw, qw, sizeof qw, cudaMemcpyHostToDevice));
  CK(cudaMemcpy(d_kw, kw, sizeof kw, cudaMemcpyHostToDevice));
  cudaStream_t s;
  CK(cudaStreamCreate(&s));
  /* the reference's per-layer pair (model.ts:94-95), varlen form */
  QK(ctx, qwa_qk_norm_rope(ctx, d_qkv, 4096, d_qw, d_kw, d_q, d_k, cu, batch, 1e-6f, 1e6f, NULL,
                           s));
  QK(ctx, qwa_attention(ctx, d_q, d_k, d_qkv, 4096, 3072, d_o, cu, batch, QWA_MODE_AUTO, 176, 432,
                        s));
  QK(ctx, qwa_check(ctx, s));
  /* a bad argument is reported, not fatal */
  if (qwa_attention(ctx, d_q, d_k, d_qkv, 4096, 3071, d_o, cu, batch, QWA_MODE_AUTO, 176, 432,
                    s) != QWA_ERR_INVALID_ARG)
    return 4;

  uint16_t* out = malloc(T * 5120 * 2);
  CK(cudaMemcpy(out, d_q, T * 2048 * 2, cudaMemcpyDeviceToHost));
  CK(cudaMemcpy(out + T * 2048, d_k, T * 1024 * 2, cudaMemcpyDeviceToHost));
  CK(cudaMemcpy(out + T * 3072, d_o, T * 2048 * 2, cudaMemcpyDeviceToHost));
  snprintf(path, sizeof path, "%s/out.bin", argv[1]);
  f = fopen(path, "wb");
  if (!f || fwrite(out, 2, T * 5120, f) != T * 5120) return 1;
  fclose(f);
  QK(ctx, qwa_destroy(ctx));
  cudaFree(d_qkv);
  cudaFree(d_q);
  cudaFree(d_k);
  cudaFree(d_o);
  cudaFree(d_qw);
  cudaFree(d_kw);
  cudaStreamDestroy(s);
  free(out);
  free(qkv);
  free(cu);
  return 0;
}
