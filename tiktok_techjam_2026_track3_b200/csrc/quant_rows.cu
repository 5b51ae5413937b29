// Per-token symmetric int8 quantisation, one warp per row (HBM-bound).
//
// scale = max(max|x|, 1e-6) / 127 and q = round_half_even(x / scale), every
// step an IEEE fp32 operation in the same order as the reference recipe
// (Project/kernels/k008_int8_gemm.py:148-151), so q and scale match it bit for
// bit.  Rows are read twice (max, then quantise); the second read hits L1/L2
// for rows up to a few tens of KB, so DRAM sees each byte once.
#include "sm100_ptx.cuh"
#include "ttj_internal.h"

namespace ttj {
namespace {

template <typename T>
__global__ void __launch_bounds__(256)
quant_rows_kernel(const T* __restrict__ x, int8_t* __restrict__ q, float* __restrict__ scale,
                  int64_t rows, int64_t cols) {
  grid_dependency_wait();  // x may be the previous kernel's output
  grid_launch_dependents();
  const int64_t warps_total = (int64_t)gridDim.x * (blockDim.x / 32);
  const int lane = threadIdx.x & 31;
  for (int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5); row < rows;
       row += warps_total) {
    const T* xr = x + row * cols;
    const uint4* x8 = reinterpret_cast<const uint4*>(xr);   // 8 elements per load
    const int64_t n8 = cols / 8;
    float amax = 0.f;
    for (int64_t i = lane; i < n8; i += 32) {
      const uint4 w = __ldg(x8 + i);
      const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = Pack<T>::unpack(ws[j]);
        amax = fmaxf(amax, fmaxf(fabsf(f.x), fabsf(f.y)));
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float s = __fdiv_rn(fmaxf(amax, 1e-6f), 127.0f);
    if (lane == 0) scale[row] = s;
    uint2* q8 = reinterpret_cast<uint2*>(q + row * cols);
    for (int64_t i = lane; i < n8; i += 32) {
      const uint4 w = __ldg(x8 + i);
      const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
      uint32_t packed[2] = {0u, 0u};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = Pack<T>::unpack(ws[j]);
        const int a = __float2int_rn(__fdiv_rn(f.x, s));
        const int c = __float2int_rn(__fdiv_rn(f.y, s));
        const uint32_t two = (uint32_t)(a & 0xff) | ((uint32_t)(c & 0xff) << 8);
        packed[j >> 1] |= two << ((j & 1) * 16);
      }
      q8[i] = make_uint2(packed[0], packed[1]);
    }
  }
}

}  // namespace

int launch_quant_rows(const void* x, int8_t* q, float* scale, int64_t rows, int64_t cols,
                      int dtype, cudaStream_t stream) {
  const int threads = 256;
  const int64_t want = (rows + 7) / 8;
  const int64_t cap = (int64_t)sm_count() * 8;  // 8 CTAs of 8 warps per SM
  const int grid = (int)(want < cap ? want : cap);
  if (dtype == TTJ_F16)
    TTJ_CUDA_TRY(launch_pdl(quant_rows_kernel<__half>, dim3(grid), dim3(threads), 0, stream,
                            static_cast<const __half*>(x), q, scale, rows, cols));
  else
    TTJ_CUDA_TRY(launch_pdl(quant_rows_kernel<__nv_bfloat16>, dim3(grid), dim3(threads), 0, stream,
                            static_cast<const __nv_bfloat16*>(x), q, scale, rows, cols));
  return TTJ_OK;
}

}  // namespace ttj
