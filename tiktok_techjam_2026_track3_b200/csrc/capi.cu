// extern "C" entry points of libttj_attn_sm100.so (declared in include/ttj_attn.h):
// argument validation, workspace carving and kernel sequencing.  No entry point
// allocates, synchronises (except ttj_read_status) or throws.
#include <cstdio>
#include <mutex>
#include <string>

#include "ttj_internal.h"

namespace ttj {

namespace {
thread_local std::string g_last_error;

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

constexpr int kMaxDevices = 64;
int g_sm_count[kMaxDevices] = {0};
}  // namespace

int fail(int code, const std::string& why) {
  g_last_error = why;
  return code;
}

int sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 148;
  if (g_sm_count[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    g_sm_count[dev] = n;
  }
  return g_sm_count[dev];
}

int encode_tmap(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base,
                const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return fail(TTJ_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  cuuint64_t d[5];
  cuuint64_t s[4];
  cuuint32_t bx[5];
  cuuint32_t es[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    bx[i] = box[i];
    es[i] = 1;
    if (i + 1 < rank) s[i] = strides_bytes[i];
  }
  CUresult r = fn(map, dtype, (cuuint32_t)rank, const_cast<void*>(base), d, s, bx, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char buf[160];
    snprintf(buf, sizeof(buf), "cuTensorMapEncodeTiled failed (CUresult %d, rank %d)", (int)r, rank);
    return fail(TTJ_ERR_CUDA, buf);
  }
  return TTJ_OK;
}

}  // namespace ttj

namespace ttj {

int check_dtype(int dtype) {
  return (dtype == TTJ_F16 || dtype == TTJ_BF16) ? TTJ_OK
                                                 : fail(TTJ_ERR_INVALID_ARG, "dtype must be TTJ_F16 or TTJ_BF16");
}

int check_layer_shape(int64_t batch, int64_t seq_len, int64_t d_model, int64_t num_heads) {
  if (batch <= 0 || seq_len <= 0 || d_model <= 0 || num_heads <= 0)
    return fail(TTJ_ERR_INVALID_ARG, "batch, seq_len, d_model and num_heads must be positive");
  // Each factor is bounded before any product is formed, so none can overflow.
  if (batch >= kMaxBatch || seq_len > kMaxSeqLen || d_model > kMaxDModel)
    return fail(TTJ_ERR_UNSUPPORTED, "batch, seq_len or d_model above the supported maximum");
  if (d_model % num_heads != 0)
    return fail(TTJ_ERR_INVALID_ARG, "d_model must be divisible by num_heads");
  const int64_t hd = d_model / num_heads;
  if (hd % 8 != 0 || hd > 256)
    return fail(TTJ_ERR_UNSUPPORTED, "head_dim must be a multiple of 8 and at most 256");
  if (d_model % 32 != 0) return fail(TTJ_ERR_UNSUPPORTED, "d_model must be a multiple of 32");
  const int64_t tokens = batch * seq_len;  // < 2^31 * 2^23: no overflow
  if (tokens > (((int64_t)1 << 46) - 1) / (3 * d_model))
    return fail(TTJ_ERR_UNSUPPORTED, "tensor too large");
  return TTJ_OK;
}

}  // namespace ttj

using ttj::aligned16;
using ttj::check_dtype;
using ttj::check_layer_shape;
using ttj::fail;

namespace {

size_t round_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Workspace sizes are only meaningful for shapes the layer accepts; outside the
// per-factor limits the byte counts could overflow, so they report 0.
bool size_args_ok(int64_t batch, int64_t seq_len, int64_t d_model) {
  return batch > 0 && seq_len > 0 && d_model > 0 && batch < ttj::kMaxBatch &&
         seq_len <= ttj::kMaxSeqLen && d_model <= ttj::kMaxDModel;
}

}  // namespace

extern "C" {

int ttj_version(void) { return 100; }

const char* ttj_status_string(int code) {
  switch (code) {
    case TTJ_OK: return "ok";
    case TTJ_ERR_INVALID_ARG: return "invalid argument";
    case TTJ_ERR_UNSUPPORTED: return "unsupported shape or dtype";
    case TTJ_ERR_ALIGNMENT: return "pointer not 16-byte aligned";
    case TTJ_ERR_CUDA: return "CUDA error";
    case TTJ_ERR_DEVICE_TIMEOUT: return "device wait timed out";
    case TTJ_ERR_WORKSPACE: return "workspace missing or too small";
    default: return "unknown status";
  }
}

const char* ttj_last_error(void) { return ttj::g_last_error.c_str(); }

int ttj_read_status(const int* status, int* code_out, ttj_stream_t stream) {
  TTJ_CHECK_ARG(status != nullptr, TTJ_ERR_INVALID_ARG, "status is NULL");
  int host = 0;
  TTJ_CUDA_TRY(cudaMemcpyAsync(&host, status, sizeof(int), cudaMemcpyDeviceToHost, (cudaStream_t)stream));
  TTJ_CUDA_TRY(cudaStreamSynchronize((cudaStream_t)stream));
  if (code_out) *code_out = host;
  if (host != 0) {
    char buf[96];
    snprintf(buf, sizeof(buf), "device status word = %d (a bounded wait expired)", host);
    return fail(TTJ_ERR_DEVICE_TIMEOUT, buf);
  }
  return TTJ_OK;
}

int ttj_selftest_wait_timeout(int* status, int64_t limit_us, ttj_stream_t stream) {
  TTJ_CHECK_ARG(status != nullptr, TTJ_ERR_INVALID_ARG, "status is NULL");
  TTJ_CHECK_ARG(limit_us > 0 && limit_us <= 1000000, TTJ_ERR_INVALID_ARG, "limit_us must be in (0, 1e6]");
  return ttj::launch_wait_timeout_selftest(status, limit_us, (cudaStream_t)stream);
}

int ttj_linear_fwd(const void* x, const void* w, const void* bias, const void* residual,
                   const uint8_t* row_mask, void* y, int64_t m, int64_t n, int64_t k, int dtype,
                   int* status, ttj_stream_t stream) {
  if (int rc = check_dtype(dtype)) return rc;
  TTJ_CHECK_ARG(x && w && bias && y, TTJ_ERR_INVALID_ARG, "x, w, bias and y must be non-NULL");
  TTJ_CHECK_ARG(m > 0 && n > 0 && k > 0, TTJ_ERR_INVALID_ARG, "m, n, k must be positive");
  TTJ_CHECK_ARG(n % 32 == 0, TTJ_ERR_UNSUPPORTED, "n must be a multiple of 32");
  TTJ_CHECK_ARG(k % 8 == 0, TTJ_ERR_UNSUPPORTED, "k must be a multiple of 8");
  TTJ_CHECK_ARG(m < (1ll << 31) && n < (1ll << 31) && k < (1ll << 31), TTJ_ERR_UNSUPPORTED, "dimension too large");
  TTJ_CHECK_ARG(aligned16(x) && aligned16(w) && aligned16(bias) && aligned16(y) &&
                    (residual == nullptr || aligned16(residual)),
                TTJ_ERR_ALIGNMENT, "x, w, bias, residual and y must be 16-byte aligned");
  ttj::GemmArgs g{};
  g.a = x;
  g.b = w;
  g.bias = bias;
  g.residual = residual;
  g.row_mask = row_mask;
  g.out = y;
  g.m = m;
  g.n = n;
  g.k = k;
  g.in_dtype = dtype;
  g.out_dtype = dtype;
  g.epi = residual ? ttj::Epi::kBiasResidual : ttj::Epi::kBias;
  g.status = status;
  return ttj::launch_gemm(g, (cudaStream_t)stream);
}

int ttj_linear_kchunked_fwd(const void* x_chunks, int64_t k_chunk, const void* w, const void* bias,
                            const void* residual, const uint8_t* row_mask, void* y, int64_t m,
                            int64_t n, int64_t k, int dtype, int* status, ttj_stream_t stream) {
  if (int rc = check_dtype(dtype)) return rc;
  TTJ_CHECK_ARG(x_chunks && w && bias && y, TTJ_ERR_INVALID_ARG, "x_chunks, w, bias and y must be non-NULL");
  TTJ_CHECK_ARG(m > 0 && n > 0 && k > 0 && k_chunk > 0, TTJ_ERR_INVALID_ARG, "m, n, k, k_chunk must be positive");
  TTJ_CHECK_ARG(k_chunk % 64 == 0 && k % k_chunk == 0, TTJ_ERR_UNSUPPORTED,
                "k_chunk must be a multiple of 64 that divides k");
  TTJ_CHECK_ARG(n % 32 == 0, TTJ_ERR_UNSUPPORTED, "n must be a multiple of 32");
  TTJ_CHECK_ARG(m < (1ll << 31) && n < (1ll << 31) && k < (1ll << 31), TTJ_ERR_UNSUPPORTED, "dimension too large");
  TTJ_CHECK_ARG(aligned16(x_chunks) && aligned16(w) && aligned16(bias) && aligned16(y) &&
                    (residual == nullptr || aligned16(residual)),
                TTJ_ERR_ALIGNMENT, "pointers must be 16-byte aligned");
  ttj::GemmArgs g{};
  g.a = x_chunks;
  g.a_kchunk = k_chunk;
  g.b = w;
  g.bias = bias;
  g.residual = residual;
  g.row_mask = row_mask;
  g.out = y;
  g.m = m;
  g.n = n;
  g.k = k;
  g.in_dtype = dtype;
  g.out_dtype = dtype;
  g.epi = residual ? ttj::Epi::kBiasResidual : ttj::Epi::kBias;
  g.status = status;
  return ttj::launch_gemm(g, (cudaStream_t)stream);
}

int ttj_qkv_proj_fwd(const void* x, const void* w_qkv, const void* b_qkv, void* qkv,
                     int64_t tokens, int64_t d_model, int dtype, int* status, ttj_stream_t stream) {
  return ttj_linear_fwd(x, w_qkv, b_qkv, nullptr, nullptr, qkv, tokens, 3 * d_model, d_model, dtype,
                        status, stream);
}

int ttj_flash_attn_fwd(const void* qkv, const uint8_t* key_mask, void* ctx, int64_t batch,
                       int64_t seq_len, int64_t num_heads, int64_t head_dim, int causal, int dtype,
                       int* status, ttj_stream_t stream) {
  if (int rc = check_dtype(dtype)) return rc;
  TTJ_CHECK_ARG(qkv && ctx, TTJ_ERR_INVALID_ARG, "qkv and ctx must be non-NULL");
  if (int rc = check_layer_shape(batch, seq_len, num_heads * head_dim, num_heads)) return rc;
  TTJ_CHECK_ARG(aligned16(qkv) && aligned16(ctx), TTJ_ERR_ALIGNMENT, "qkv and ctx must be 16-byte aligned");
  ttj::AttnArgs a{};
  a.qkv = qkv;
  a.key_mask = key_mask;
  a.ctx = ctx;
  a.batch = batch;
  a.seq_len = seq_len;
  a.num_heads = num_heads;
  a.head_dim = head_dim;
  a.causal = causal ? 1 : 0;
  a.dtype = dtype;
  a.status = status;
  return ttj::launch_flash_attn(a, (cudaStream_t)stream);
}

int ttj_out_proj_residual_fwd(const void* ctx, const void* w_o, const void* b_o, const void* x,
                              const uint8_t* row_mask, void* out, int64_t tokens, int64_t d_model,
                              int dtype, int* status, ttj_stream_t stream) {
  TTJ_CHECK_ARG(x != nullptr, TTJ_ERR_INVALID_ARG, "residual x must be non-NULL");
  return ttj_linear_fwd(ctx, w_o, b_o, x, row_mask, out, tokens, d_model, d_model, dtype, status, stream);
}

size_t ttj_attn_layer_workspace_size(int64_t batch, int64_t seq_len, int64_t d_model, int dtype) {
  (void)dtype;
  if (!size_args_ok(batch, seq_len, d_model)) return 0;
  const size_t t = (size_t)batch * (size_t)seq_len;
  return round_up(t * 3 * d_model * 2, 256) + round_up(t * d_model * 2, 256);
}

int ttj_attn_layer_fwd(const ttj_attn_layer_args* a, ttj_stream_t stream) {
  TTJ_CHECK_ARG(a != nullptr, TTJ_ERR_INVALID_ARG, "args is NULL");
  if (int rc = check_dtype(a->dtype)) return rc;
  if (int rc = check_layer_shape(a->batch, a->seq_len, a->d_model, a->num_heads)) return rc;
  TTJ_CHECK_ARG(a->x && a->w_qkv && a->b_qkv && a->w_o && a->b_o && a->out, TTJ_ERR_INVALID_ARG,
                "x, weights, biases and out must be non-NULL");
  TTJ_CHECK_ARG(a->out != a->x && a->out != a->residual, TTJ_ERR_INVALID_ARG,
                "out must not alias x or residual");
  const size_t need = ttj_attn_layer_workspace_size(a->batch, a->seq_len, a->d_model, a->dtype);
  TTJ_CHECK_ARG(a->workspace != nullptr && a->workspace_bytes >= need, TTJ_ERR_WORKSPACE,
                "workspace missing or smaller than ttj_attn_layer_workspace_size()");
  TTJ_CHECK_ARG(aligned16(a->workspace), TTJ_ERR_ALIGNMENT, "workspace must be 16-byte aligned");
  const int64_t T = a->batch * a->seq_len, D = a->d_model;
  uint8_t* ws = static_cast<uint8_t*>(a->workspace);
  void* qkv = ws;
  void* ctx = ws + round_up((size_t)T * 3 * D * 2, 256);
  int rc = ttj_qkv_proj_fwd(a->x, a->w_qkv, a->b_qkv, qkv, T, D, a->dtype, a->status, stream);
  if (rc) return rc;
  rc = ttj_flash_attn_fwd(qkv, a->valid_token_mask, ctx, a->batch, a->seq_len, a->num_heads,
                          D / a->num_heads, a->causal, a->dtype, a->status, stream);
  if (rc) return rc;
  return ttj_linear_fwd(ctx, a->w_o, a->b_o, a->residual, a->valid_token_mask, a->out, T, D, D,
                        a->dtype, a->status, stream);
}

int ttj_int8_quant_rows(const void* x, int8_t* q, float* scale, int64_t rows, int64_t cols,
                        int dtype, ttj_stream_t stream) {
  if (int rc = check_dtype(dtype)) return rc;
  TTJ_CHECK_ARG(x && q && scale, TTJ_ERR_INVALID_ARG, "x, q and scale must be non-NULL");
  TTJ_CHECK_ARG(rows > 0 && cols > 0, TTJ_ERR_INVALID_ARG, "rows and cols must be positive");
  TTJ_CHECK_ARG(cols % 8 == 0, TTJ_ERR_UNSUPPORTED, "cols must be a multiple of 8");
  TTJ_CHECK_ARG(aligned16(x) && aligned16(q), TTJ_ERR_ALIGNMENT, "x and q must be 16-byte aligned");
  return ttj::launch_quant_rows(x, q, scale, rows, cols, dtype, (cudaStream_t)stream);
}

int ttj_int8_gemm_s32(const int8_t* a, const int8_t* w, int32_t* acc, int64_t m, int64_t n, int64_t k,
                      int* status, ttj_stream_t stream) {
  TTJ_CHECK_ARG(a && w && acc, TTJ_ERR_INVALID_ARG, "a, w and acc must be non-NULL");
  TTJ_CHECK_ARG(m > 0 && n > 0 && k > 0, TTJ_ERR_INVALID_ARG, "m, n, k must be positive");
  TTJ_CHECK_ARG(n % 32 == 0 && k % 16 == 0, TTJ_ERR_UNSUPPORTED, "need n % 32 == 0 and k % 16 == 0");
  TTJ_CHECK_ARG(aligned16(a) && aligned16(w) && aligned16(acc), TTJ_ERR_ALIGNMENT, "pointers must be 16-byte aligned");
  ttj::GemmArgs g{};
  g.a = a;
  g.b = w;
  g.out = acc;
  g.m = m;
  g.n = n;
  g.k = k;
  g.in_dtype = -1;
  g.epi = ttj::Epi::kRawS32;
  g.status = status;
  return ttj::launch_gemm(g, (cudaStream_t)stream);
}

int ttj_int8_linear_fwd(const int8_t* a, const float* s_a, const int8_t* w, const float* s_w,
                        const float* bias, const void* residual, const uint8_t* row_mask, void* y,
                        int64_t m, int64_t n, int64_t k, int out_dtype, int* status, ttj_stream_t stream) {
  if (int rc = check_dtype(out_dtype)) return rc;
  TTJ_CHECK_ARG(a && s_a && w && s_w && bias && y, TTJ_ERR_INVALID_ARG, "operands must be non-NULL");
  TTJ_CHECK_ARG(m > 0 && n > 0 && k > 0, TTJ_ERR_INVALID_ARG, "m, n, k must be positive");
  TTJ_CHECK_ARG(n % 32 == 0 && k % 16 == 0, TTJ_ERR_UNSUPPORTED, "need n % 32 == 0 and k % 16 == 0");
  TTJ_CHECK_ARG(aligned16(a) && aligned16(w) && aligned16(y) && aligned16(s_w) && aligned16(bias) &&
                    (residual == nullptr || aligned16(residual)),
                TTJ_ERR_ALIGNMENT, "pointers must be 16-byte aligned");
  ttj::GemmArgs g{};
  g.a = a;
  g.b = w;
  g.bias = bias;
  g.residual = residual;
  g.row_mask = row_mask;
  g.scale_a = s_a;
  g.scale_b = s_w;
  g.out = y;
  g.m = m;
  g.n = n;
  g.k = k;
  g.in_dtype = -1;
  g.out_dtype = out_dtype;
  g.epi = residual ? ttj::Epi::kDequantResidual : ttj::Epi::kDequant;
  g.status = status;
  return ttj::launch_gemm(g, (cudaStream_t)stream);
}

size_t ttj_int8_attn_layer_workspace_size(int64_t batch, int64_t seq_len, int64_t d_model, int dtype) {
  (void)dtype;
  if (!size_args_ok(batch, seq_len, d_model)) return 0;
  const size_t t = (size_t)batch * (size_t)seq_len, d = (size_t)d_model;
  return round_up(t * d, 256)            /* int8 activations (x, then ctx) */
         + round_up(t * 4, 256)          /* per-token scales */
         + round_up(t * 3 * d * 2, 256)  /* qkv (16-bit) */
         + round_up(t * d * 2, 256);     /* ctx (16-bit) */
}

int ttj_int8_attn_layer_fwd(const ttj_int8_attn_layer_args* a, ttj_stream_t stream) {
  TTJ_CHECK_ARG(a != nullptr, TTJ_ERR_INVALID_ARG, "args is NULL");
  if (int rc = check_dtype(a->dtype)) return rc;
  if (int rc = check_layer_shape(a->batch, a->seq_len, a->d_model, a->num_heads)) return rc;
  TTJ_CHECK_ARG(a->x && a->w_qkv && a->s_qkv && a->b_qkv && a->w_o && a->s_o && a->b_o && a->out,
                TTJ_ERR_INVALID_ARG, "operands must be non-NULL");
  TTJ_CHECK_ARG(a->out != a->x && a->out != a->residual, TTJ_ERR_INVALID_ARG,
                "out must not alias x or residual");
  const size_t need = ttj_int8_attn_layer_workspace_size(a->batch, a->seq_len, a->d_model, a->dtype);
  TTJ_CHECK_ARG(a->workspace != nullptr && a->workspace_bytes >= need, TTJ_ERR_WORKSPACE,
                "workspace missing or smaller than ttj_int8_attn_layer_workspace_size()");
  TTJ_CHECK_ARG(aligned16(a->workspace), TTJ_ERR_ALIGNMENT, "workspace must be 16-byte aligned");
  const int64_t T = a->batch * a->seq_len, D = a->d_model;
  uint8_t* ws = static_cast<uint8_t*>(a->workspace);
  int8_t* act8 = reinterpret_cast<int8_t*>(ws);
  ws += round_up((size_t)T * D, 256);
  float* s_tok = reinterpret_cast<float*>(ws);
  ws += round_up((size_t)T * 4, 256);
  void* qkv = ws;
  ws += round_up((size_t)T * 3 * D * 2, 256);
  void* ctx = ws;
  int rc = ttj_int8_quant_rows(a->x, act8, s_tok, T, D, a->dtype, stream);
  if (rc) return rc;
  rc = ttj_int8_linear_fwd(act8, s_tok, a->w_qkv, a->s_qkv, a->b_qkv, nullptr, nullptr, qkv, T, 3 * D,
                           D, a->dtype, a->status, stream);
  if (rc) return rc;
  rc = ttj_flash_attn_fwd(qkv, a->valid_token_mask, ctx, a->batch, a->seq_len, a->num_heads,
                          D / a->num_heads, a->causal, a->dtype, a->status, stream);
  if (rc) return rc;
  rc = ttj_int8_quant_rows(ctx, act8, s_tok, T, D, a->dtype, stream);
  if (rc) return rc;
  return ttj_int8_linear_fwd(act8, s_tok, a->w_o, a->s_o, a->b_o, a->residual, a->valid_token_mask,
                             a->out, T, D, D, a->dtype, a->status, stream);
}

int ttj_layernorm_fwd(const void* x, const void* gamma, const void* beta, const uint8_t* row_mask,
                      void* y, int64_t rows, int64_t d, float eps, int dtype, ttj_stream_t stream) {
  if (dtype != TTJ_F32)
    if (int rc = check_dtype(dtype)) return rc;
  TTJ_CHECK_ARG(x && gamma && beta && y, TTJ_ERR_INVALID_ARG, "x, gamma, beta and y must be non-NULL");
  TTJ_CHECK_ARG(rows > 0 && d > 0, TTJ_ERR_INVALID_ARG, "rows and d must be positive");
  TTJ_CHECK_ARG(eps >= 0.f, TTJ_ERR_INVALID_ARG, "eps must be non-negative");
  TTJ_CHECK_ARG(d % 8 == 0 && d <= (dtype == TTJ_F32 ? 4096 : 8192), TTJ_ERR_UNSUPPORTED,
                "d must be a multiple of 8 and at most 8192 (4096 for fp32)");
  TTJ_CHECK_ARG(aligned16(x) && aligned16(gamma) && aligned16(beta) && aligned16(y), TTJ_ERR_ALIGNMENT,
                "x, gamma, beta and y must be 16-byte aligned");
  return ttj::launch_layernorm(x, gamma, beta, row_mask, y, rows, d, eps, dtype, (cudaStream_t)stream,
                               dtype);
}

int ttj_linear_gelu_fwd(const void* x, const void* w, const void* bias, void* y, int64_t m, int64_t n,
                        int64_t k, int dtype, int* status, ttj_stream_t stream) {
  if (int rc = check_dtype(dtype)) return rc;
  TTJ_CHECK_ARG(x && w && bias && y, TTJ_ERR_INVALID_ARG, "x, w, bias and y must be non-NULL");
  TTJ_CHECK_ARG(m > 0 && n > 0 && k > 0, TTJ_ERR_INVALID_ARG, "m, n, k must be positive");
  TTJ_CHECK_ARG(n % 32 == 0, TTJ_ERR_UNSUPPORTED, "n must be a multiple of 32");
  TTJ_CHECK_ARG(k % 8 == 0, TTJ_ERR_UNSUPPORTED, "k must be a multiple of 8");
  TTJ_CHECK_ARG(m < (1ll << 31) && n < (1ll << 31) && k < (1ll << 31), TTJ_ERR_UNSUPPORTED, "dimension too large");
  TTJ_CHECK_ARG(aligned16(x) && aligned16(w) && aligned16(bias) && aligned16(y), TTJ_ERR_ALIGNMENT,
                "x, w, bias and y must be 16-byte aligned");
  ttj::GemmArgs g{};
  g.a = x;
  g.b = w;
  g.bias = bias;
  g.out = y;
  g.m = m;
  g.n = n;
  g.k = k;
  g.in_dtype = dtype;
  g.out_dtype = dtype;
  g.epi = ttj::Epi::kBiasGelu;
  g.status = status;
  return ttj::launch_gemm(g, (cudaStream_t)stream);
}

size_t ttj_block_workspace_size(int64_t batch, int64_t seq_len, int64_t d_model, int64_t ffn_dim,
                                int dtype) {
  (void)dtype;
  if (!size_args_ok(batch, seq_len, d_model) || ffn_dim <= 0 || ffn_dim >= (1ll << 31)) return 0;
  const size_t t = (size_t)batch * (size_t)seq_len, d = (size_t)d_model, f = (size_t)ffn_dim;
  const size_t wide = 3 * d > f ? 3 * d : f;
  const size_t stream_bytes = dtype == TTJ_F32 ? 4 : 2;
  return round_up(t * d * 2, 256)        /* normalised input (norm1, then norm2) */
         + round_up(t * wide * 2, 256)   /* qkv, then the GELU activations */
         + round_up(t * d * 2, 256)      /* attention context */
         + round_up(t * d * stream_bytes, 256);  /* x1 = x + attention (residual stream) */
}

int ttj_transformer_block_fwd(const ttj_block_args* a, ttj_stream_t stream) {
  TTJ_CHECK_ARG(a != nullptr, TTJ_ERR_INVALID_ARG, "args is NULL");
  const bool f32 = a->dtype == TTJ_F32;  // fp32 residual stream, fp16 operands inside
  if (!f32)
    if (int rc = check_dtype(a->dtype)) return rc;
  TTJ_CHECK_ARG(!f32 || a->d_model <= 4096, TTJ_ERR_UNSUPPORTED, "fp32 residual stream: d_model at most 4096");
  if (int rc = check_layer_shape(a->batch, a->seq_len, a->d_model, a->num_heads)) return rc;
  TTJ_CHECK_ARG(a->ffn_dim > 0 && a->ffn_dim % 32 == 0 && a->ffn_dim < (1ll << 31), TTJ_ERR_UNSUPPORTED,
                "ffn_dim must be a positive multiple of 32");
  TTJ_CHECK_ARG(a->batch * a->seq_len <= (((int64_t)1 << 46) - 1) / a->ffn_dim, TTJ_ERR_UNSUPPORTED,
                "tensor too large");
  TTJ_CHECK_ARG(a->x && a->ln1_w && a->ln1_b && a->w_qkv && a->b_qkv && a->w_o && a->b_o && a->ln2_w &&
                    a->ln2_b && a->w_in && a->b_in && a->w_out && a->b_out && a->out,
                TTJ_ERR_INVALID_ARG, "x, parameters and out must be non-NULL");
  TTJ_CHECK_ARG(a->out != a->x, TTJ_ERR_INVALID_ARG, "out must not alias x");
  TTJ_CHECK_ARG(aligned16(a->x) && aligned16(a->ln1_w) && aligned16(a->ln1_b) && aligned16(a->w_qkv) &&
                    aligned16(a->b_qkv) && aligned16(a->w_o) && aligned16(a->b_o) && aligned16(a->ln2_w) &&
                    aligned16(a->ln2_b) && aligned16(a->w_in) && aligned16(a->b_in) && aligned16(a->w_out) &&
                    aligned16(a->b_out) && aligned16(a->out),
                TTJ_ERR_ALIGNMENT, "x, parameters and out must be 16-byte aligned");
  const size_t need = ttj_block_workspace_size(a->batch, a->seq_len, a->d_model, a->ffn_dim, a->dtype);
  TTJ_CHECK_ARG(a->workspace != nullptr && a->workspace_bytes >= need, TTJ_ERR_WORKSPACE,
                "workspace missing or smaller than ttj_block_workspace_size()");
  TTJ_CHECK_ARG(aligned16(a->workspace), TTJ_ERR_ALIGNMENT, "workspace must be 16-byte aligned");
  const int64_t T = a->batch * a->seq_len, D = a->d_model, F = a->ffn_dim;
  const size_t wide = (size_t)(3 * D > F ? 3 * D : F);
  const int op = f32 ? TTJ_F16 : a->dtype;        // tensor-core operand / activation type
  uint8_t* ws = static_cast<uint8_t*>(a->workspace);
  void* h = ws;                                   // norm1(x), later norm2(x1)
  ws += round_up((size_t)T * D * 2, 256);
  void* big = ws;                                 // qkv, later gelu(ffn_in(.))
  ws += round_up((size_t)T * wide * 2, 256);
  void* ctx = ws;
  ws += round_up((size_t)T * D * 2, 256);
  void* x1 = ws;                                  // residual stream after attention
  const uint8_t* mask = a->valid_token_mask;
  cudaStream_t st = (cudaStream_t)stream;
  int rc = f32 ? ttj::launch_layernorm(a->x, a->ln1_w, a->ln1_b, nullptr, h, T, D, a->eps1, TTJ_F32, st, op)
               : ttj_layernorm_fwd(a->x, a->ln1_w, a->ln1_b, nullptr, h, T, D, a->eps1, a->dtype, stream);
  if (rc) return rc;
  rc = ttj_qkv_proj_fwd(h, a->w_qkv, a->b_qkv, big, T, D, op, a->status, stream);
  if (rc) return rc;
  rc = ttj_flash_attn_fwd(big, mask, ctx, a->batch, a->seq_len, a->num_heads, D / a->num_heads, a->causal,
                          op, a->status, stream);
  if (rc) return rc;
  // x1 = x + mask(ctx w_o^T + b_o), in the residual stream's type
  ttj::GemmArgs g{};
  g.a = ctx;
  g.b = a->w_o;
  g.bias = a->b_o;
  g.residual = a->x;
  g.row_mask = mask;
  g.out = x1;
  g.m = T;
  g.n = D;
  g.k = D;
  g.in_dtype = op;
  g.out_dtype = a->dtype;
  g.epi = ttj::Epi::kBiasResidual;
  g.status = a->status;
  rc = ttj::launch_gemm(g, st);
  if (rc) return rc;
  rc = f32 ? ttj::launch_layernorm(x1, a->ln2_w, a->ln2_b, nullptr, h, T, D, a->eps2, TTJ_F32, st, op)
           : ttj_layernorm_fwd(x1, a->ln2_w, a->ln2_b, nullptr, h, T, D, a->eps2, a->dtype, stream);
  if (rc) return rc;
  rc = ttj_linear_gelu_fwd(h, a->w_in, a->b_in, big, T, F, D, op, a->status, stream);
  if (rc) return rc;
  // out = mask_rows(x1 + ffn_out(.)): rows of invalid tokens become zero
  g.a = big;
  g.b = a->w_out;
  g.bias = a->b_out;
  g.residual = x1;
  g.out = a->out;
  g.k = F;
  g.epi = ttj::Epi::kBiasResidualZeroRows;
  return ttj::launch_gemm(g, st);
}

}  // extern "C"
