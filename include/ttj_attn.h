/*
 * ttj_attn.h — C ABI of the B200 (sm_100a) attention-layer forward.
 *
 * One shared library, libttj_attn_sm100.so, exports these entry points.  All
 * pointers are DEVICE pointers unless stated; sizes are element counts.  Every
 * function only enqueues work on `stream` (no host synchronisation, no
 * allocation), returns TTJ_OK (0) or a negative ttj_status, and never throws.
 * ttj_last_error() gives a one-line reason for the last failure on the calling
 * thread.
 *
 * Reference interfaces replaced (file:line in yyan115/Tiktok_TechJam_2026_Track3):
 *   torch_transformer_benchmark.py:85-122  BaselineSelfAttention.forward
 *   torch_transformer_benchmark.py:140     block residual  x + attention(...)
 *   torch_transformer_benchmark.py:125-172 BaselineTransformerBlock / final norm
 *   Project/kernels/k008_int8_gemm.py:148-185  W8A8 recipe (_quant_rows,
 *                                           _int8_pack, _int8_linear)
 *
 * Layouts (row-major, innermost last):
 *   x, out      [B, S, D]     D = num_heads * head_dim
 *   w_qkv       [3D, D]       rows 0..D-1 = q_proj.weight, D..2D-1 = k_proj.weight,
 *                             2D..3D-1 = v_proj.weight  (nn.Linear (out, in) layout)
 *   b_qkv       [3D]          q_proj.bias | k_proj.bias | v_proj.bias
 *   w_o, b_o    [D, D], [D]   out_proj.weight, out_proj.bias
 *   qkv         [B, S, 3D]    packed projections; head h of q is columns
 *                             [h*hd, (h+1)*hd), of k [D + h*hd, ...), of v [2D + h*hd, ...)
 *   ctx         [B, S, D]     attention context with heads already merged
 *   valid_token_mask [B, S]   uint8 (torch.bool), 1 = valid; may be NULL (all valid)
 *
 * Supported: dtype fp16 or bf16; head_dim a multiple of 8 up to 256; D a
 * multiple of 32; any B >= 1, 1 <= S <= 8388480.  Anything else returns
 * TTJ_ERR_UNSUPPORTED.
 */
#ifndef TTJ_ATTN_H_
#define TTJ_ATTN_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* ttj_stream_t; /* == cudaStream_t; NULL = legacy default stream */

enum ttj_dtype {
  TTJ_F16 = 0,
  TTJ_BF16 = 1,
  TTJ_F32 = 2  /* fp32 residual stream: only where an entry point says so */
};

enum ttj_status {
  TTJ_OK = 0,
  TTJ_ERR_INVALID_ARG = -1,   /* null pointer, non-positive size, bad enum */
  TTJ_ERR_UNSUPPORTED = -2,   /* shape or dtype outside the supported set */
  TTJ_ERR_ALIGNMENT = -3,     /* pointer not 16-byte aligned */
  TTJ_ERR_CUDA = -4,          /* a CUDA runtime / driver call failed */
  TTJ_ERR_DEVICE_TIMEOUT = -5,/* a kernel's bounded wait expired (see ttj_read_status) */
  TTJ_ERR_WORKSPACE = -6,     /* workspace missing or smaller than required */
};

/* Library version (major*10000 + minor*100 + patch). */
int ttj_version(void);
/* Static string for a ttj_status code. */
const char* ttj_status_string(int code);
/* Detail of the last failure on this thread ("" if none). */
const char* ttj_last_error(void);

/*
 * Device status word.  Kernels given a non-NULL `status` (a device int,
 * zero-initialised by the caller) write a nonzero code there if one of their
 * bounded internal waits expires, then stop and return instead of hanging.
 * ttj_read_status copies it to the host (synchronising `stream`) and returns
 * TTJ_OK if it is zero, TTJ_ERR_DEVICE_TIMEOUT otherwise, with the code in
 * *code_out.
 */
int ttj_read_status(const int* status, int* code_out, ttj_stream_t stream);

/*
 * Failure-path self-test: launches one warp that waits on a barrier nothing
 * arrives on, gives up after limit_us microseconds (<= 1 s), writes a nonzero
 * code into *status and exits.  Exercises the bounded-wait path of every
 * kernel without faulting or hanging the GPU.  No reference counterpart (the
 * reference's failure handling is host-side, dispatcher_region.py:107-128).
 */
int ttj_selftest_wait_timeout(int* status, int64_t limit_us, ttj_stream_t stream);

/*
 * y[M,N] = x[M,K] . w[N,K]^T + bias[N]           (residual == NULL)
 * y[M,N] = residual[M,N] + mask(x . w^T + bias)    (residual != NULL)
 * where mask() zeroes row m when row_mask != NULL and row_mask[m] == 0.
 * tcgen05 GEMM, fp32 accumulate in tensor memory, fused epilogue.
 * Replaces the nn.Linear calls of torch_transformer_benchmark.py:93-95, :118
 * and the residual of :140 / the output masking of :120-121.
 * Requires N % 32 == 0 and K % 8 == 0.
 */
int ttj_linear_fwd(const void* x, const void* w, const void* bias, const void* residual,
                   const uint8_t* row_mask, void* y, int64_t m, int64_t n, int64_t k,
                   int dtype, int* status, ttj_stream_t stream);

/*
 * ttj_linear_fwd with the input stored K-chunk-major:
 *   x(m, k) = x_chunks[k / k_chunk][m][k % k_chunk],  x_chunks [k/k_chunk][m][k_chunk]
 * This is the layout a head-sharded attention context arrives in when each of
 * k/k_chunk ranks contributes the columns of its heads ([m][k_chunk] each): the
 * out-projection reads it in place (a 3-D tensor map), so the gathered slices
 * need no re-packing into [m][k].  Requires k_chunk % 64 == 0, k % k_chunk == 0,
 * n % 32 == 0.  Used by the multi-GPU head partitioner; the reference has no
 * multi-GPU path (its out_proj is torch_transformer_benchmark.py:118).
 */
int ttj_linear_kchunked_fwd(const void* x_chunks, int64_t k_chunk, const void* w, const void* bias,
                            const void* residual, const uint8_t* row_mask, void* y, int64_t m,
                            int64_t n, int64_t k, int dtype, int* status, ttj_stream_t stream);

/*
 * Fused QKV projection: qkv[T,3D] = x[T,D] . w_qkv[3D,D]^T + b_qkv.
 * Replaces q_proj/k_proj/v_proj + _split_heads (torch_transformer_benchmark.py:77-83,
 * :93-95): the head split is free because attention reads head slices of the
 * packed buffer directly.
 */
int ttj_qkv_proj_fwd(const void* x, const void* w_qkv, const void* b_qkv, void* qkv,
                     int64_t tokens, int64_t d_model, int dtype, int* status,
                     ttj_stream_t stream);

/*
 * Flash attention forward from the packed qkv buffer into ctx [B,S,D]:
 * softmax(q k^T * head_dim^-0.5 + masks) v per (batch, head), fp32 softmax,
 * probabilities rounded to `dtype` before the P.V product (as the reference's
 * .to(dtype=x.dtype) at torch_transformer_benchmark.py:111), no S x S
 * materialisation.  causal != 0 masks keys after the query
 * (torch_transformer_benchmark.py:99-103); key_mask (may be NULL) masks keys
 * whose entry is 0 (torch_transformer_benchmark.py:105-108).  Replaces
 * torch_transformer_benchmark.py:97-117.
 */
int ttj_flash_attn_fwd(const void* qkv, const uint8_t* key_mask, void* ctx, int64_t batch,
                       int64_t seq_len, int64_t num_heads, int64_t head_dim, int causal,
                       int dtype, int* status, ttj_stream_t stream);

/*
 * out[T,D] = x + mask(ctx . w_o^T + b_o): out-proj with bias, output-row
 * masking and the block residual in one epilogue
 * (torch_transformer_benchmark.py:118-121 and :140).
 */
int ttj_out_proj_residual_fwd(const void* ctx, const void* w_o, const void* b_o,
                              const void* x, const uint8_t* row_mask, void* out,
                              int64_t tokens, int64_t d_model, int dtype, int* status,
                              ttj_stream_t stream);

/* Arguments of the whole attention layer. */
typedef struct ttj_attn_layer_args {
  const void* x;                   /* [B,S,D] */
  const void* w_qkv;               /* [3D,D] */
  const void* b_qkv;               /* [3D]   */
  const void* w_o;                 /* [D,D]  */
  const void* b_o;                 /* [D]    */
  const uint8_t* valid_token_mask; /* [B,S] or NULL */
  const void* residual;            /* [B,S,D] added in the out-proj epilogue (x for the
                                      attention layer, the pre-norm stream inside a
                                      transformer block); NULL = no residual */
  void* out;                       /* [B,S,D], must not alias x or residual */
  void* workspace;                 /* >= ttj_attn_layer_workspace_size() bytes */
  size_t workspace_bytes;
  int* status;                     /* device status word or NULL */
  int64_t batch, seq_len, d_model, num_heads;
  int causal;
  int dtype;                       /* enum ttj_dtype */
} ttj_attn_layer_args;

/* Bytes of device workspace the layer needs (qkv + ctx intermediates). */
size_t ttj_attn_layer_workspace_size(int64_t batch, int64_t seq_len, int64_t d_model,
                                     int dtype);

/*
 * out = residual + BaselineSelfAttention(x, valid_token_mask, causal)
 * (residual = x gives the attention layer x + attn(x)): three kernels
 * (QKV GEMM, flash attention, out-proj GEMM with bias+mask+residual epilogue),
 * no elementwise kernel in between.  torch_transformer_benchmark.py:85-122, :140.
 */
int ttj_attn_layer_fwd(const ttj_attn_layer_args* args, ttj_stream_t stream);

/*
 * The same layer for callers that cannot allocate device memory (a host
 * runtime that owns all device allocations, or one that must not grow its
 * footprint after start-up): identical kernels and results, but the qkv and
 * context intermediates live in a fixed 32 MiB array in device memory owned
 * by the library, so args->workspace / workspace_bytes are ignored.
 * No counterpart in the reference (its layer always allocates through torch).
 * Limit: layers whose ttj_attn_layer_workspace_size() exceeds 32 MiB
 * (33554432 bytes) are rejected with TTJ_ERR_WORKSPACE.  Calls no allocator.
 * One array per GPU, shared by every call: calls that overlap on the same GPU
 * race; calls ordered on one stream are safe.  The first call on a device
 * looks up the array's address with that device current; make it before any
 * stream capture.  Because the CUDA runtime loads device code lazily, that
 * first call is also when the array is mapped: it grows device memory by
 * 32 MiB once (TTJ_ERR_CUDA if the device has no 32 MiB free), so a caller
 * that reserves the rest of device memory up front makes it during start-up,
 * before the reservation.  From then on the device holds the array until the
 * process exits and calls map nothing more.
 */
int ttj_attn_layer_fwd_noalloc(const ttj_attn_layer_args* args, ttj_stream_t stream);

/* ------------------------------------------------------------------ int8 */

/*
 * Per-row symmetric int8 quantisation (k008_int8_gemm.py:148-151):
 * scale[r] = max(max_c |x[r,c]|, 1e-6) / 127, q = round_half_even(x / scale).
 * x is fp16/bf16 [rows, cols]; q int8 [rows, cols]; scale fp32 [rows].
 */
int ttj_int8_quant_rows(const void* x, int8_t* q, float* scale, int64_t rows, int64_t cols,
                        int dtype, ttj_stream_t stream);

/*
 * Raw int32 accumulators acc[M,N] = a[M,K] . w[N,K]^T on tcgen05 kind::i8
 * (torch._int_mm of k008_int8_gemm.py:183).  For bit-exact checking.
 * Requires N % 32 == 0 and K % 16 == 0.
 */
int ttj_int8_gemm_s32(const int8_t* a, const int8_t* w, int32_t* acc, int64_t m, int64_t n,
                      int64_t k, int* status, ttj_stream_t stream);

/*
 * Dequantising int8 GEMM (k008_int8_gemm.py:181-185):
 *   y = acc * (s_a[m] * s_w[n]) + bias[n]                      (residual == NULL)
 *   y = residual + mask(acc * (s_a[m] * s_w[n]) + bias[n])     (residual != NULL)
 * s_a, s_w, bias fp32; residual and y in `out_dtype` (fp16/bf16).
 */
int ttj_int8_linear_fwd(const int8_t* a, const float* s_a, const int8_t* w, const float* s_w,
                        const float* bias, const void* residual, const uint8_t* row_mask,
                        void* y, int64_t m, int64_t n, int64_t k, int out_dtype, int* status,
                        ttj_stream_t stream);

/* Arguments of the int8-projection attention layer (benchmark configuration 3). */
typedef struct ttj_int8_attn_layer_args {
  const void* x;                   /* [B,S,D] fp16/bf16 */
  const int8_t* w_qkv;             /* [3D,D] int8, per-output-channel quantised */
  const float* s_qkv;              /* [3D] weight scales */
  const float* b_qkv;              /* [3D] fp32 bias */
  const int8_t* w_o;               /* [D,D] int8 */
  const float* s_o;                /* [D] */
  const float* b_o;                /* [D] fp32 bias */
  const uint8_t* valid_token_mask; /* [B,S] or NULL */
  const void* residual;            /* [B,S,D] or NULL, as in ttj_attn_layer_args */
  void* out;                       /* [B,S,D] */
  void* workspace;
  size_t workspace_bytes;
  int* status;
  int64_t batch, seq_len, d_model, num_heads;
  int causal;
  int dtype;
} ttj_int8_attn_layer_args;

size_t ttj_int8_attn_layer_workspace_size(int64_t batch, int64_t seq_len, int64_t d_model,
                                          int dtype);

/*
 * W8A8 attention layer: quantise x per token, int8 QKV GEMM with fused dequant
 * + bias, 16-bit flash attention, quantise ctx per token, int8 out-proj GEMM
 * with fused dequant + bias + mask + residual.
 */
int ttj_int8_attn_layer_fwd(const ttj_int8_attn_layer_args* args, ttj_stream_t stream);

/* ------------------------------------------------------- transformer block */

/*
 * y[r,:] = (x[r,:] - mean) / sqrt(var + eps) * gamma + beta over rows of length
 * d (biased variance, fp32 arithmetic), i.e. nn.LayerNorm(d, eps) of
 * torch_transformer_benchmark.py:128-130 (norm1, norm2) and :159 (final_norm).
 * Rows with row_mask[r] == 0 are written as zeros (the model's final
 * masked_fill, :170-171); row_mask may be NULL.  gamma/beta are [d] in the same
 * dtype as x.  Requires d % 8 == 0 and d <= 8192.  dtype TTJ_F32: x, gamma,
 * beta and y are all fp32 (d <= 4096), e.g. the final norm of an fp32 model.
 */
int ttj_layernorm_fwd(const void* x, const void* gamma, const void* beta, const uint8_t* row_mask,
                      void* y, int64_t rows, int64_t d, float eps, int dtype, ttj_stream_t stream);

/*
 * y[M,N] = gelu(x[M,K] . w[N,K]^T + bias[N]) with the exact (erf) GELU:
 * the block's F.gelu(self.ffn_in(...), approximate="none")
 * (torch_transformer_benchmark.py:141) as one GEMM with a fused epilogue.
 * erf(z) is evaluated as 1 - erfc(z) with an erfc of fractional error below
 * 1.2e-7 (Numerical Recipes' Chebyshev fit), so the 16-bit result is the
 * correctly rounded exact GELU in almost every case and never more than one
 * unit in the last place off.
 * Requires N % 32 == 0 and K % 8 == 0.
 */
int ttj_linear_gelu_fwd(const void* x, const void* w, const void* bias, void* y, int64_t m,
                        int64_t n, int64_t k, int dtype, int* status, ttj_stream_t stream);

/* Arguments of one pre-norm transformer block (BaselineTransformerBlock). */
typedef struct ttj_block_args {
  const void* x;                   /* [B,S,D] block input */
  const void* ln1_w;               /* [D] norm1.weight */
  const void* ln1_b;               /* [D] norm1.bias */
  const void* w_qkv;               /* [3D,D] packed q/k/v_proj weights (as ttj_attn_layer_args) */
  const void* b_qkv;               /* [3D] */
  const void* w_o;                 /* [D,D] attention.out_proj.weight */
  const void* b_o;                 /* [D] */
  const void* ln2_w;               /* [D] norm2.weight */
  const void* ln2_b;               /* [D] norm2.bias */
  const void* w_in;                /* [F,D] ffn_in.weight */
  const void* b_in;                /* [F] */
  const void* w_out;               /* [D,F] ffn_out.weight */
  const void* b_out;               /* [D] */
  const uint8_t* valid_token_mask; /* [B,S] or NULL */
  void* out;                       /* [B,S,D], must not alias x */
  void* workspace;                 /* >= ttj_block_workspace_size() bytes */
  size_t workspace_bytes;
  int* status;                     /* device status word or NULL */
  int64_t batch, seq_len, d_model, num_heads, ffn_dim;
  float eps1, eps2;                /* norm1.eps, norm2.eps */
  int causal;
  int dtype;                       /* enum ttj_dtype */
} ttj_block_args;

/* Bytes of device workspace one block needs. */
size_t ttj_block_workspace_size(int64_t batch, int64_t seq_len, int64_t d_model, int64_t ffn_dim,
                                int dtype);

/*
 * One BaselineTransformerBlock.forward (torch_transformer_benchmark.py:134-145):
 *   x1  = x + mask(attention(norm1(x)))            (LayerNorm kernel + the layer's three)
 *   out = mask_rows(x1 + ffn_out(gelu(ffn_in(norm2(x1)))))
 * as six kernels: LayerNorm, QKV GEMM, flash attention, out-proj GEMM with
 * bias+mask+residual, LayerNorm, ffn_in GEMM with bias+GELU, ffn_out GEMM with
 * bias+residual and the block's final row zeroing (masked_fill, :143-144).
 * Requires ffn_dim % 32 == 0 plus the attention layer's shape rules.
 *
 * dtype TTJ_F32 runs the block of an fp32 model with an fp32 residual stream
 * and fp16 tensor-core operands: x, out, ln1_w/ln1_b, ln2_w/ln2_b, b_o and
 * b_out are fp32; w_qkv, b_qkv, w_o, w_in, b_in and w_out are fp16.  The
 * LayerNorms read the fp32 stream and write fp16 GEMM operands; the out-proj
 * and ffn_out epilogues add their fp32 bias and residual in fp32 and write the
 * fp32 stream.  d_model <= 4096.  The reference's optimised route runs fp32
 * models on fp16 kernels with an fp16 stream
 * (Project/submission/dispatcher_region.py:760-801); kept in fp32, the stream
 * meets the benchmark tolerance on the official shapes where an fp16 stream
 * misses it on a few elements.
 */
int ttj_transformer_block_fwd(const ttj_block_args* args, ttj_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* TTJ_ATTN_H_ */
