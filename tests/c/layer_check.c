/*
 * The attention layer through the C ABI from C: no Python, no torch.
 *
 * Builds seeded fp16 inputs and weights on the host, runs
 * ttj_attn_layer_fwd (out = x + BaselineSelfAttention(x, mask, causal),
 * torch_transformer_benchmark.py:85-122 with the block residual of :140) on
 * the GPU, and checks every output element against a double-precision
 * restatement of the same layer computed here on the CPU from the same
 * fp16-rounded values, with the intermediates rounded where the reference's
 * fp16 run rounds them (q/k/v after the projections, the probabilities after
 * the fp32 softmax at :111, the merged context).  Pass/fail uses the
 * reference's predicate: |gpu - ref| <= 2e-3 + 2e-2 * |ref| per element
 * (torch_transformer_benchmark.py:306-318, atol 2e-3 / rtol 2e-2 at :618-619).
 *
 * Exit status 0 when every case passes.  Prints one line per case.
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <cuda_runtime_api.h>

#include "ttj_attn.h"

typedef _Float16 half_t;

static uint64_t rng_state;
static double uniform(void) { /* xorshift64*, in [0, 1) */
  rng_state ^= rng_state >> 12;
  rng_state ^= rng_state << 25;
  rng_state ^= rng_state >> 27;
  return (double)((rng_state * 2685821657736338717ull) >> 11) * (1.0 / 9007199254740992.0);
}
static double symmetric(double a) { return (2.0 * uniform() - 1.0) * a; }
static double r16(double v) { return (double)(half_t)v; } /* round to fp16 */

#define CHECK_CUDA(call)                                                        \
  do {                                                                          \
    cudaError_t e_ = (call);                                                    \
    if (e_ != cudaSuccess) {                                                    \
      fprintf(stderr, "%s:%d %s: %s\n", __FILE__, __LINE__, #call,             \
              cudaGetErrorString(e_));                                          \
      exit(2);                                                                  \
    }                                                                           \
  } while (0)

static int run_case(int B, int S, int D, int H, int causal, int masked, uint64_t seed) {
  const int hd = D / H, T = B * S;
  rng_state = seed * 0x9E3779B97F4A7C15ull + 1;
  /* host tensors, already rounded to fp16 */
  size_t nx = (size_t)T * D, nwq = (size_t)3 * D * D, nwo = (size_t)D * D;
  double *x = malloc(nx * sizeof(double)), *wq = malloc(nwq * sizeof(double));
  double *bq = malloc(3 * D * sizeof(double)), *wo = malloc(nwo * sizeof(double));
  double *bo = malloc(D * sizeof(double));
  uint8_t* mask = malloc((size_t)T);
  for (size_t i = 0; i < nx; ++i) x[i] = r16(symmetric(1.7));          /* ~ unit variance */
  for (size_t i = 0; i < nwq; ++i) wq[i] = r16(symmetric(0.035));      /* ~ N(0, 0.02) */
  for (int i = 0; i < 3 * D; ++i) bq[i] = r16(symmetric(0.035));
  for (size_t i = 0; i < nwo; ++i) wo[i] = r16(symmetric(0.035));
  for (int i = 0; i < D; ++i) bo[i] = r16(symmetric(0.035));
  for (int b = 0; b < B; ++b) /* prefix masks, at least one valid key (Ref :261-271) */
    for (int s = 0; s < S; ++s) mask[b * S + s] = !masked || s < S - 1 - (b * 37) % (S / 2);

  /* CPU restatement in double */
  double* qkv = malloc((size_t)T * 3 * D * sizeof(double));
  double* ctx = calloc((size_t)T * D, sizeof(double));
  double* ref = malloc(nx * sizeof(double));
  double* p = malloc((size_t)S * sizeof(double));
  for (int t = 0; t < T; ++t)
    for (int n = 0; n < 3 * D; ++n) {
      double acc = bq[n];
      for (int k = 0; k < D; ++k) acc += x[(size_t)t * D + k] * wq[(size_t)n * D + k];
      qkv[(size_t)t * 3 * D + n] = r16(acc);
    }
  const double scale = 1.0 / sqrt((double)hd);
  for (int b = 0; b < B; ++b)
    for (int h = 0; h < H; ++h)
      for (int i = 0; i < S; ++i) {
        const double* q = qkv + ((size_t)(b * S + i)) * 3 * D + h * hd;
        double mx = -INFINITY;
        for (int j = 0; j < S; ++j) {
          const double* k = qkv + ((size_t)(b * S + j)) * 3 * D + D + h * hd;
          double s = 0.0;
          for (int c = 0; c < hd; ++c) s += q[c] * k[c];
          s *= scale;
          if ((causal && j > i) || !mask[b * S + j]) s = -INFINITY;
          p[j] = s;
          if (s > mx) mx = s;
        }
        double l = 0.0;
        for (int j = 0; j < S; ++j) {
          p[j] = p[j] == -INFINITY ? 0.0 : exp(p[j] - mx);
          l += p[j];
        }
        double* o = ctx + ((size_t)(b * S + i)) * D + h * hd;
        for (int j = 0; j < S; ++j) {
          const double pj = r16(p[j] / l);
          if (pj == 0.0) continue;
          const double* v = qkv + ((size_t)(b * S + j)) * 3 * D + 2 * D + h * hd;
          for (int c = 0; c < hd; ++c) o[c] += pj * v[c];
        }
        for (int c = 0; c < hd; ++c) o[c] = r16(o[c]);
      }
  for (int t = 0; t < T; ++t)
    for (int n = 0; n < D; ++n) {
      double acc = bo[n];
      for (int k = 0; k < D; ++k) acc += ctx[(size_t)t * D + k] * wo[(size_t)n * D + k];
      /* output rows of invalid query tokens are zeroed before the residual (Ref :120-121) */
      ref[(size_t)t * D + n] = x[(size_t)t * D + n] + (mask[t] ? acc : 0.0);
    }

  /* device side */
  half_t *hx = malloc(nx * sizeof(half_t)), *hwq = malloc(nwq * sizeof(half_t));
  half_t *hbq = malloc(3 * D * sizeof(half_t)), *hwo = malloc(nwo * sizeof(half_t));
  half_t *hbo = malloc(D * sizeof(half_t)), *hout = malloc(nx * sizeof(half_t));
  for (size_t i = 0; i < nx; ++i) hx[i] = (half_t)x[i];
  for (size_t i = 0; i < nwq; ++i) hwq[i] = (half_t)wq[i];
  for (int i = 0; i < 3 * D; ++i) hbq[i] = (half_t)bq[i];
  for (size_t i = 0; i < nwo; ++i) hwo[i] = (half_t)wo[i];
  for (int i = 0; i < D; ++i) hbo[i] = (half_t)bo[i];
  void *dx, *dwq, *dbq, *dwo, *dbo, *dout, *dws;
  uint8_t* dmask = NULL;
  int* dstatus;
  const size_t ws = ttj_attn_layer_workspace_size(B, S, D, TTJ_F16);
  CHECK_CUDA(cudaMalloc(&dx, nx * 2));
  CHECK_CUDA(cudaMalloc(&dwq, nwq * 2));
  CHECK_CUDA(cudaMalloc(&dbq, (size_t)3 * D * 2));
  CHECK_CUDA(cudaMalloc(&dwo, nwo * 2));
  CHECK_CUDA(cudaMalloc(&dbo, (size_t)D * 2));
  CHECK_CUDA(cudaMalloc(&dout, nx * 2));
  CHECK_CUDA(cudaMalloc(&dws, ws));
  CHECK_CUDA(cudaMalloc((void**)&dstatus, sizeof(int)));
  CHECK_CUDA(cudaMemset(dstatus, 0, sizeof(int)));
  CHECK_CUDA(cudaMemcpy(dx, hx, nx * 2, cudaMemcpyHostToDevice));
  CHECK_CUDA(cudaMemcpy(dwq, hwq, nwq * 2, cudaMemcpyHostToDevice));
  CHECK_CUDA(cudaMemcpy(dbq, hbq, (size_t)3 * D * 2, cudaMemcpyHostToDevice));
  CHECK_CUDA(cudaMemcpy(dwo, hwo, nwo * 2, cudaMemcpyHostToDevice));
  CHECK_CUDA(cudaMemcpy(dbo, hbo, (size_t)D * 2, cudaMemcpyHostToDevice));
  if (masked) {
    CHECK_CUDA(cudaMalloc((void**)&dmask, (size_t)T));
    CHECK_CUDA(cudaMemcpy(dmask, mask, (size_t)T, cudaMemcpyHostToDevice));
  }
  cudaStream_t stream;
  CHECK_CUDA(cudaStreamCreate(&stream));

  ttj_attn_layer_args a;
  memset(&a, 0, sizeof(a));
  a.x = dx;
  a.w_qkv = dwq;
  a.b_qkv = dbq;
  a.w_o = dwo;
  a.b_o = dbo;
  a.valid_token_mask = dmask;
  a.residual = dx;
  a.out = dout;
  a.workspace = dws;
  a.workspace_bytes = ws;
  a.status = dstatus;
  a.batch = B;
  a.seq_len = S;
  a.d_model = D;
  a.num_heads = H;
  a.causal = causal;
  a.dtype = TTJ_F16;
  int rc = ttj_attn_layer_fwd(&a, (ttj_stream_t)stream);
  if (rc != TTJ_OK) {
    fprintf(stderr, "ttj_attn_layer_fwd: %s (%s)\n", ttj_status_string(rc), ttj_last_error());
    return 1;
  }
  int code = 0;
  rc = ttj_read_status(dstatus, &code, (ttj_stream_t)stream);
  if (rc != TTJ_OK) {
    fprintf(stderr, "device status %d\n", code);
    return 1;
  }
  CHECK_CUDA(cudaMemcpy(hout, dout, nx * 2, cudaMemcpyDeviceToHost));

  double max_err = 0.0, worst_ratio = 0.0;
  size_t bad = 0;
  for (size_t i = 0; i < nx; ++i) {
    const double g = (double)hout[i], r = ref[i];
    const double err = fabs(g - r), allowed = 2e-3 + 2e-2 * fabs(r);
    if (!(err <= allowed)) ++bad; /* NaN counts as bad */
    if (err > max_err) max_err = err;
    if (err / allowed > worst_ratio) worst_ratio = err / allowed;
  }
  printf("B%d S%d D%d H%d hd%d causal=%d masked=%d: max |gpu - ref| %.3g, worst err/allowed %.3f, "
         "%zu of %zu outside the predicate\n",
         B, S, D, H, hd, causal, masked, max_err, worst_ratio, bad, nx);

  cudaStreamDestroy(stream);
  cudaFree(dx); cudaFree(dwq); cudaFree(dbq); cudaFree(dwo); cudaFree(dbo); cudaFree(dout);
  cudaFree(dws); cudaFree(dstatus);
  if (dmask) cudaFree(dmask);
  free(x); free(wq); free(bq); free(wo); free(bo); free(mask); free(qkv); free(ctx); free(ref);
  free(p); free(hx); free(hwq); free(hbq); free(hwo); free(hbo); free(hout);
  return bad == 0 ? 0 : 1;
}

int main(void) {
  printf("libttj_attn_sm100 version %d\n", ttj_version());
  int fails = 0;
  fails += run_case(2, 100, 128, 2, 1, 0, 1234);  /* head_dim 64, causal, ragged S */
  fails += run_case(2, 130, 128, 2, 0, 1, 1235);  /* head_dim 64, key padding mask */
  fails += run_case(1, 200, 256, 2, 1, 1, 1236);  /* head_dim 128, causal + mask */
  fails += run_case(3, 128, 128, 4, 1, 0, 1237);  /* head_dim 32 (the reference's shapes 1-6, 12, 13) */
  fails += run_case(2, 90, 32, 4, 1, 1, 1238);    /* head_dim 8, d_model 32 (shape 7), ragged + mask */
  fails += run_case(2, 140, 512, 2, 1, 0, 1239);  /* head_dim 256 (shape 8), ragged S */
  return fails == 0 ? 0 : 1;
}
