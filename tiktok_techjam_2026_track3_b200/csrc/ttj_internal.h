// Host-side helpers shared by the kernel translation units: error reporting,
// tensor-map encoding (through the driver entry point, so the library does not
// link libcuda directly), per-device SM counts and the kernel launchers.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string>

#include "../../include/ttj_attn.h"

namespace ttj {

// Remember a failure for ttj_last_error() and return `code`.
int fail(int code, const std::string& why);

// Check a CUDA runtime result; on failure remember it and return TTJ_ERR_CUDA.
#define TTJ_CUDA_TRY(expr)                                                          \
  do {                                                                              \
    cudaError_t _e = (expr);                                                        \
    if (_e != cudaSuccess)                                                          \
      return ::ttj::fail(TTJ_ERR_CUDA, std::string(#expr) + ": " + cudaGetErrorString(_e)); \
  } while (0)

#define TTJ_CHECK_ARG(cond, code, msg)               \
  do {                                               \
    if (!(cond)) return ::ttj::fail((code), (msg));  \
  } while (0)

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Per-factor limits of the layer entry points, checked before any product of
// sizes is formed.  kMaxSeqLen keeps every query-tile row coordinate of the
// attention kernel below 2^23.
constexpr int64_t kMaxBatch = (int64_t)1 << 31;
constexpr int64_t kMaxSeqLen = (int64_t)65535 * 128;
constexpr int64_t kMaxDModel = (int64_t)1 << 16;

// Argument checks shared by every layer entry point (TTJ_OK or a ttj_status).
int check_dtype(int dtype);
int check_layer_shape(int64_t batch, int64_t seq_len, int64_t d_model, int64_t num_heads);

// Number of SMs of the current device (cached per device).
int sm_count();

// Launch a kernel of this library with programmatic stream serialisation: it
// may begin while the previous kernel on `stream` finishes, and waits for it
// on the device (grid_dependency_wait() in sm100_ptx.cuh) before touching
// global memory.  Works under CUDA-graph capture.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

// Encode a tiled TMA descriptor with 128-byte swizzle, zero out-of-bounds fill.
// dims/strides are innermost-first; strides in bytes for dims 1..rank-1.
int encode_tmap(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base,
                const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box);

// Launchers (one per kernel family).  They validate nothing beyond what the
// kernels need; the extern "C" layer validates arguments first.
enum class Epi : int {
  kBias = 0,            // y = acc + bias
  kBiasResidual = 1,    // y = residual + mask(acc + bias)
  kRawS32 = 2,          // y = acc (int32)
  kDequant = 3,         // y = acc * (s_a * s_w) + bias
  kDequantResidual = 4, // y = residual + mask(acc * (s_a * s_w) + bias)
  kBiasGelu = 5,        // y = gelu_erf(acc + bias)
  kBiasResidualZeroRows = 6, // y = mask(residual + acc + bias): masked rows become 0
};

struct GemmArgs {
  const void* a;          // [M, K], or [K / a_kchunk][M][a_kchunk] when a_kchunk > 0
  const void* b;          // [N, K]
  const void* bias;       // [N]  (16-bit for kBias*, fp32 for kDequant*)
  const void* residual;   // [M, N]
  const uint8_t* row_mask;// [M]
  const float* scale_a;   // [M]
  const float* scale_b;   // [N]
  void* out;              // [M, N]
  int64_t m, n, k;
  int in_dtype;           // TTJ_F16 / TTJ_BF16, or -1 for int8 operands
  int out_dtype;          // TTJ_F16 / TTJ_BF16 (ignored for kRawS32)
  Epi epi;
  int* status;
  int64_t a_kchunk = 0;   // > 0: A is stored K-chunk-major (see above); multiple of 64
};
int launch_gemm(const GemmArgs& g, cudaStream_t stream);

struct AttnArgs {
  const void* qkv;        // [B, S, 3D]
  const uint8_t* key_mask;// [B, S] or null
  void* ctx;              // [B, S, D]
  int64_t batch, seq_len, num_heads, head_dim;
  int causal;
  int dtype;
  int* status;
};
int launch_flash_attn(const AttnArgs& a, cudaStream_t stream);

int launch_wait_timeout_selftest(int* status, int64_t limit_us, cudaStream_t stream);

// LayerNorm over rows of length d (d % 8 == 0, d <= 8192; fp32 input: d <= 4096);
// rows with a zero row_mask byte are written as zeros.  dtype is the input's
// (and, for 16-bit input, gamma/beta/output's); with dtype TTJ_F32, gamma and
// beta are fp32 and out_dtype picks the output type (TTJ_F16 / TTJ_BF16 / TTJ_F32).
int launch_layernorm(const void* x, const void* gamma, const void* beta, const uint8_t* row_mask,
                     void* y, int64_t rows, int64_t d, float eps, int dtype, cudaStream_t stream,
                     int out_dtype = -1);

int launch_quant_rows(const void* x, int8_t* q, float* scale, int64_t rows, int64_t cols,
                      int dtype, cudaStream_t stream);

}  // namespace ttj
