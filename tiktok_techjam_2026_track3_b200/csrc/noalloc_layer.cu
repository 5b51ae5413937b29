// ttj_attn_layer_fwd_noalloc: the attention layer for callers that cannot
// allocate device memory.
//
// Who needs it: code that runs where cudaMalloc is off limits -- a host
// runtime that owns every device allocation itself and forbids libraries from
// making their own, an embedding that must not grow its memory footprint after
// start-up, or a caller whose allocator cannot be reached from the thread that
// launches work.  Such a caller can pass the layer's inputs and output but has
// no way to hand over the qkv / context workspace that ttj_attn_layer_fwd takes.
//
// What it does instead: the two intermediates (packed q|k|v, then the
// head-merged context) live in one fixed array in device global memory,
// declared below at file scope.  The array's size is the limit: a layer whose
// workspace (ttj_attn_layer_workspace_size) exceeds kNoAllocScratchBytes is
// rejected with TTJ_ERR_WORKSPACE.  Every GPU that loads this code holds the
// array until the process exits.
//
// Sharing rules: there is one array per device and every call uses it, so two
// calls whose work overlaps on the same GPU (different streams, or different
// host threads without ordering) race on it and corrupt each other's results.
// Calls ordered on one stream are safe.  The array keeps whatever the last call
// left in it; nothing here needs it to start at zero, because each stage writes
// every element that the next stage reads.
//
// Set-up: the device address of the array is looked up (cudaGetSymbolAddress)
// the first time the entry point runs on a device, with that device current,
// and cached.  Make that first call before any stream capture begins.  The
// CUDA runtime loads a library's device code onto a device lazily (the default
// module-loading mode), so that same first call is also when the 32 MiB array
// is mapped on the device: it grows device memory by 32 MiB once, and fails
// with TTJ_ERR_CUDA if the device has no 32 MiB left.  A caller that reserves
// the rest of device memory up front should make its first call on each device
// during start-up, before that reservation; later calls map nothing more.
#include <cstdio>
#include <mutex>

#include "ttj_internal.h"

namespace {

// 32 MiB: enough for the layer at T * D <= 4 Mi elements (e.g. B2 S2048 D1024).
constexpr size_t kNoAllocScratchBytes = size_t(32) << 20;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_ptr[kMaxDevices] = {nullptr};

// Device address of the scratch array on the current device (set-up on first use).
int scratch_for_current_device(void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return ttj::fail(TTJ_ERR_CUDA, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return ttj::fail(TTJ_ERR_CUDA, "device index out of range");
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr)
      return ttj::fail(TTJ_ERR_CUDA, std::string("cudaGetSymbolAddress(scratch): ") + cudaGetErrorString(e));
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return TTJ_OK;
}

size_t round_up256(size_t v) { return (v + 255) / 256 * 256; }

}  // namespace

extern "C" int ttj_attn_layer_fwd_noalloc(const ttj_attn_layer_args* a, ttj_stream_t stream) {
  if (a == nullptr) return ttj::fail(TTJ_ERR_INVALID_ARG, "args is NULL");
  // The same checks, in the same order, as ttj_attn_layer_fwd: a rejected call
  // launches nothing.
  if (int rc = ttj::check_dtype(a->dtype)) return rc;
  if (int rc = ttj::check_layer_shape(a->batch, a->seq_len, a->d_model, a->num_heads)) return rc;
  if (a->x == nullptr || a->w_qkv == nullptr || a->b_qkv == nullptr || a->w_o == nullptr ||
      a->b_o == nullptr || a->out == nullptr)
    return ttj::fail(TTJ_ERR_INVALID_ARG, "x, weights, biases and out must be non-NULL");
  if (a->out == a->x || a->out == a->residual)
    return ttj::fail(TTJ_ERR_INVALID_ARG, "out must not alias x or residual");
  const size_t need = ttj_attn_layer_workspace_size(a->batch, a->seq_len, a->d_model, a->dtype);
  if (need > kNoAllocScratchBytes) {
    char buf[200];
    snprintf(buf, sizeof(buf),
             "layer needs %zu bytes of scratch; the no-allocation entry point has a fixed "
             "%zu-byte array (use ttj_attn_layer_fwd with a caller workspace)",
             need, kNoAllocScratchBytes);
    return ttj::fail(TTJ_ERR_WORKSPACE, buf);
  }
  void* scratch = nullptr;
  if (int rc = scratch_for_current_device(&scratch)) return rc;
  const int64_t T = a->batch * a->seq_len, D = a->d_model;
  unsigned char* base = static_cast<unsigned char*>(scratch);
  void* qkv = base;
  void* ctx = base + round_up256((size_t)T * 3 * D * 2);
  int rc = ttj_qkv_proj_fwd(a->x, a->w_qkv, a->b_qkv, qkv, T, D, a->dtype, a->status, stream);
  if (rc) return rc;
  rc = ttj_flash_attn_fwd(qkv, a->valid_token_mask, ctx, a->batch, a->seq_len, a->num_heads,
                          D / a->num_heads, a->causal, a->dtype, a->status, stream);
  if (rc) return rc;
  return ttj_linear_fwd(ctx, a->w_o, a->b_o, a->residual, a->valid_token_mask, a->out, T, D, D,
                        a->dtype, a->status, stream);
}
