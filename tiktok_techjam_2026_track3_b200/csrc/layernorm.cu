// LayerNorm over the last dimension, one warp per row (HBM-bound).
//
// y = (x - mean) / sqrt(var + eps) * gamma + beta with the biased variance, as
// nn.LayerNorm computes it for the reference block's norm1 / norm2 / final_norm
// (torch_transformer_benchmark.py:128-130, :159).  The row is read once into
// registers (16-byte vectors), reduced in fp32 in two passes (mean, then the
// centred sum of squares, which avoids the cancellation of E[x^2] - mean^2), and
// written once.  Rows whose row_mask byte is 0 are written as zeros (the
// model's final masked_fill, torch_transformer_benchmark.py:170-171).
#include <type_traits>

#include "sm100_ptx.cuh"
#include "ttj_internal.h"

namespace ttj {
namespace {

template <typename T, int VPL>  // VPL = 16-byte vectors (8 elements) per lane
__global__ void __launch_bounds__(256)
layernorm_kernel(const T* __restrict__ x, const T* __restrict__ gamma, const T* __restrict__ beta,
                 const uint8_t* __restrict__ row_mask, T* __restrict__ y, int64_t rows, int d,
                 float eps) {
  grid_dependency_wait();  // x may be the previous kernel's output
  grid_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int nvec = d / 8;
  const int64_t warps_total = (int64_t)gridDim.x * (blockDim.x / 32);
  const float inv_d = 1.f / (float)d;
  for (int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5); row < rows;
       row += warps_total) {
    const uint4* xr = reinterpret_cast<const uint4*>(x + row * d);
    uint4* yr = reinterpret_cast<uint4*>(y + row * d);
    if (row_mask != nullptr && __ldg(row_mask + row) == 0) {
      for (int i = lane; i < nvec; i += 32) yr[i] = make_uint4(0u, 0u, 0u, 0u);
      continue;
    }
    uint4 v[VPL];
    float sum = 0.f;
#pragma unroll
    for (int q = 0; q < VPL; ++q) {
      const int i = lane + 32 * q;
      v[q] = i < nvec ? __ldg(xr + i) : make_uint4(0u, 0u, 0u, 0u);
      const uint32_t ws[4] = {v[q].x, v[q].y, v[q].z, v[q].w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = Pack<T>::unpack(ws[j]);
        sum += f.x + f.y;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    const float mean = sum * inv_d;
    float sq = 0.f;
#pragma unroll
    for (int q = 0; q < VPL; ++q) {
      if (lane + 32 * q >= nvec) continue;
      const uint32_t ws[4] = {v[q].x, v[q].y, v[q].z, v[q].w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = Pack<T>::unpack(ws[j]);
        const float a = f.x - mean, b = f.y - mean;
        sq = fmaf(a, a, sq);
        sq = fmaf(b, b, sq);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
    const float rstd = rsqrtf(sq * inv_d + eps);
#pragma unroll
    for (int q = 0; q < VPL; ++q) {
      const int i = lane + 32 * q;
      if (i >= nvec) continue;
      const uint4 gw = __ldg(reinterpret_cast<const uint4*>(gamma) + i);
      const uint4 bw = __ldg(reinterpret_cast<const uint4*>(beta) + i);
      const uint32_t ws[4] = {v[q].x, v[q].y, v[q].z, v[q].w};
      const uint32_t gs[4] = {gw.x, gw.y, gw.z, gw.w};
      const uint32_t bs[4] = {bw.x, bw.y, bw.z, bw.w};
      uint32_t out[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = Pack<T>::unpack(ws[j]);
        const float2 g = Pack<T>::unpack(gs[j]);
        const float2 b = Pack<T>::unpack(bs[j]);
        out[j] = Pack<T>::two((f.x - mean) * rstd * g.x + b.x, (f.y - mean) * rstd * g.y + b.y);
      }
      yr[i] = make_uint4(out[0], out[1], out[2], out[3]);
    }
  }
}

// Output of 8 consecutive normalised values: one 16-byte store of 16-bit
// values, or two of fp32.
template <typename TOut>
__device__ __forceinline__ void store8(TOut* y, const float (&v)[8]) {
  if constexpr (std::is_same<TOut, float>::value) {
    reinterpret_cast<float4*>(y)[0] = make_float4(v[0], v[1], v[2], v[3]);
    reinterpret_cast<float4*>(y)[1] = make_float4(v[4], v[5], v[6], v[7]);
  } else {
    *reinterpret_cast<uint4*>(y) = make_uint4(Pack<TOut>::two(v[0], v[1]), Pack<TOut>::two(v[2], v[3]),
                                              Pack<TOut>::two(v[4], v[5]), Pack<TOut>::two(v[6], v[7]));
  }
}

// The same LayerNorm over an fp32 row (the residual stream of an fp32 model),
// fp32 gamma / beta, written as TOut: 16-bit for the next GEMM's operand, or
// fp32 for the model's final norm.  Lane l holds 8-element groups l, l+32, ...
// of the row in registers (two 16-byte loads each); d <= 4096.
template <typename TOut, int VPL>
__global__ void __launch_bounds__(256)
layernorm_f32in_kernel(const float* __restrict__ x, const float* __restrict__ gamma,
                       const float* __restrict__ beta, const uint8_t* __restrict__ row_mask,
                       TOut* __restrict__ y, int64_t rows, int d, float eps) {
  grid_dependency_wait();
  grid_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int ngrp = d / 8;
  const int64_t warps_total = (int64_t)gridDim.x * (blockDim.x / 32);
  const float inv_d = 1.f / (float)d;
  for (int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5); row < rows;
       row += warps_total) {
    const float4* xr = reinterpret_cast<const float4*>(x + row * d);
    TOut* yr = y + row * d;
    if (row_mask != nullptr && __ldg(row_mask + row) == 0) {
      const float zero[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (int i = lane; i < ngrp; i += 32) store8<TOut>(yr + 8 * i, zero);
      continue;
    }
    float v[VPL][8];
    float sum = 0.f;
#pragma unroll
    for (int q = 0; q < VPL; ++q) {
      const int i = lane + 32 * q;
      const float4 a = i < ngrp ? __ldg(xr + 2 * i) : make_float4(0.f, 0.f, 0.f, 0.f);
      const float4 b = i < ngrp ? __ldg(xr + 2 * i + 1) : make_float4(0.f, 0.f, 0.f, 0.f);
      v[q][0] = a.x; v[q][1] = a.y; v[q][2] = a.z; v[q][3] = a.w;
      v[q][4] = b.x; v[q][5] = b.y; v[q][6] = b.z; v[q][7] = b.w;
#pragma unroll
      for (int j = 0; j < 8; ++j) sum += v[q][j];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    const float mean = sum * inv_d;
    float sq = 0.f;
#pragma unroll
    for (int q = 0; q < VPL; ++q) {
      if (lane + 32 * q >= ngrp) continue;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float a = v[q][j] - mean;
        sq = fmaf(a, a, sq);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
    const float rstd = rsqrtf(sq * inv_d + eps);
#pragma unroll
    for (int q = 0; q < VPL; ++q) {
      const int i = lane + 32 * q;
      if (i >= ngrp) continue;
      const float4 g0 = __ldg(reinterpret_cast<const float4*>(gamma) + 2 * i);
      const float4 g1 = __ldg(reinterpret_cast<const float4*>(gamma) + 2 * i + 1);
      const float4 b0 = __ldg(reinterpret_cast<const float4*>(beta) + 2 * i);
      const float4 b1 = __ldg(reinterpret_cast<const float4*>(beta) + 2 * i + 1);
      const float g[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
      const float bb[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
      float out[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) out[j] = (v[q][j] - mean) * rstd * g[j] + bb[j];
      store8<TOut>(yr + 8 * i, out);
    }
  }
}

template <typename TOut>
int launch_f32in(const void* x, const void* gamma, const void* beta, const uint8_t* row_mask, void* y,
                 int64_t rows, int d, float eps, cudaStream_t stream) {
  const int64_t want = (rows + 7) / 8;
  const int64_t cap = (int64_t)sm_count() * 8;
  const int grid = (int)(want < cap ? want : cap);
  const float* xf = static_cast<const float*>(x);
  const float* gf = static_cast<const float*>(gamma);
  const float* bf = static_cast<const float*>(beta);
  TOut* yo = static_cast<TOut*>(y);
  if (d <= 1024) TTJ_CUDA_TRY(launch_pdl(layernorm_f32in_kernel<TOut, 4>, dim3(grid), dim3(256), 0, stream, xf, gf, bf, row_mask, yo, rows, d, eps));
  else if (d <= 2048) TTJ_CUDA_TRY(launch_pdl(layernorm_f32in_kernel<TOut, 8>, dim3(grid), dim3(256), 0, stream, xf, gf, bf, row_mask, yo, rows, d, eps));
  else TTJ_CUDA_TRY(launch_pdl(layernorm_f32in_kernel<TOut, 16>, dim3(grid), dim3(256), 0, stream, xf, gf, bf, row_mask, yo, rows, d, eps));
  return TTJ_OK;
}

template <typename T, int VPL>
cudaError_t launch_vpl(const void* x, const void* gamma, const void* beta, const uint8_t* row_mask, void* y,
                       int64_t rows, int d, float eps, int grid, cudaStream_t stream) {
  return launch_pdl(layernorm_kernel<T, VPL>, dim3(grid), dim3(256), 0, stream, static_cast<const T*>(x),
                    static_cast<const T*>(gamma), static_cast<const T*>(beta), row_mask, static_cast<T*>(y),
                    rows, d, eps);
}

template <typename T>
int launch_t(const void* x, const void* gamma, const void* beta, const uint8_t* row_mask, void* y,
             int64_t rows, int d, float eps, cudaStream_t stream) {
  const int64_t want = (rows + 7) / 8;
  const int64_t cap = (int64_t)sm_count() * 8;  // 8 CTAs of 8 warps per SM
  const int grid = (int)(want < cap ? want : cap);
  if (d <= 1024) TTJ_CUDA_TRY((launch_vpl<T, 4>(x, gamma, beta, row_mask, y, rows, d, eps, grid, stream)));
  else if (d <= 2048) TTJ_CUDA_TRY((launch_vpl<T, 8>(x, gamma, beta, row_mask, y, rows, d, eps, grid, stream)));
  else if (d <= 4096) TTJ_CUDA_TRY((launch_vpl<T, 16>(x, gamma, beta, row_mask, y, rows, d, eps, grid, stream)));
  else TTJ_CUDA_TRY((launch_vpl<T, 32>(x, gamma, beta, row_mask, y, rows, d, eps, grid, stream)));
  return TTJ_OK;
}

}  // namespace

int launch_layernorm(const void* x, const void* gamma, const void* beta, const uint8_t* row_mask,
                     void* y, int64_t rows, int64_t d, float eps, int dtype, cudaStream_t stream,
                     int out_dtype) {
  if (dtype == TTJ_F32) {
    if (out_dtype == TTJ_F16) return launch_f32in<__half>(x, gamma, beta, row_mask, y, rows, (int)d, eps, stream);
    if (out_dtype == TTJ_BF16) return launch_f32in<__nv_bfloat16>(x, gamma, beta, row_mask, y, rows, (int)d, eps, stream);
    return launch_f32in<float>(x, gamma, beta, row_mask, y, rows, (int)d, eps, stream);
  }
  if (dtype == TTJ_F16) return launch_t<__half>(x, gamma, beta, row_mask, y, rows, (int)d, eps, stream);
  return launch_t<__nv_bfloat16>(x, gamma, beta, row_mask, y, rows, (int)d, eps, stream);
}

}  // namespace ttj
