// Per-token symmetric int8 quantisation, one warp per row (HBM-bound).
//
// scale = max(max|x|, 1e-6) / 127 and q = round_half_even(x / scale), as the
// reference recipe computes them (Project/kernels/k008_int8_gemm.py:148-151),
// bit for bit.  Rows of up to 4096 elements are held in registers between the
// max and the quantisation (one read); longer rows are read twice, the second
// read hitting L1/L2.
//
// The element step avoids a full IEEE division per element (measured: with
// one, the special-function pipe was 72% busy and the kernel moved 3.0 TB/s).
// Per row, y = 1/s correctly rounded; per element the quotient is x * y with
// one residual correction, r = fma(-q0, s, x), q = fma(r, y, q0) (division by
// a correctly rounded reciprocal, P. Markstein, IBM J. Res. Dev. 34(1), 1990),
// and round-half-even to an integer is the addition of 1.5 * 2^23, whose low
// byte is the int8 value.  tests/c/quant_div_check.c compares this with the
// IEEE quotient and rint() over every finite fp16 and bf16 x and every scale a
// row can produce (|x| <= amax): the int8 values agree everywhere; quotients
// agree bit for bit except for |x| < 2^-100 (the residual underflows) and the
// sign of a zero quotient, all of which become 0.  Inputs are assumed finite.
#include "sm100_ptx.cuh"
#include "ttj_internal.h"

namespace ttj {
namespace {

// x / s rounded half-to-even, as the low byte of the returned bits (see above).
__device__ __forceinline__ uint32_t quant_bits(float x, float s, float y) {
  const float q0 = __fmul_rn(x, y);
  const float r = __fmaf_rn(-q0, s, x);
  const float q = __fmaf_rn(r, y, q0);
  return __float_as_uint(__fadd_rn(q, 12582912.0f));  // 1.5 * 2^23: |q| <= 127.5
}

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
    const float y = __frcp_rn(s);
    if (lane == 0) scale[row] = s;
    uint2* q8 = reinterpret_cast<uint2*>(q + row * cols);
    for (int64_t i = lane; i < n8; i += 32) {
      const uint4 w = __ldg(x8 + i);
      const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
      uint32_t t[8];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = Pack<T>::unpack(ws[j]);
        t[2 * j] = quant_bits(f.x, s, y);
        t[2 * j + 1] = quant_bits(f.y, s, y);
      }
      // low bytes of t[0..3] and t[4..7], in element order
      const uint32_t lo = __byte_perm(__byte_perm(t[0], t[1], 0x0040), __byte_perm(t[2], t[3], 0x0040), 0x5410);
      const uint32_t hi = __byte_perm(__byte_perm(t[4], t[5], 0x0040), __byte_perm(t[6], t[7], 0x0040), 0x5410);
      q8[i] = make_uint2(lo, hi);
    }
  }
}

// Rows of at most 32 lanes x NCH x 8 elements: each lane loads its 16-byte
// chunks once (coalesced across the warp) and keeps them in registers for the
// max and the quantisation.  Chunks past the row's end are zeros (they leave
// the max unchanged) and are not stored.  Launch shape per row length
// (measured, 65536 rows): 4096 elements in 128-thread CTAs, three per SM
// (6.2 TB/s; 256-thread CTAs: 5.4-5.6 TB/s); shorter rows with fewer chunks
// per lane, so that more warps fit.
template <int NCH> struct RegShape;
template <> struct RegShape<4> { static constexpr int kThreads = 256, kMinBlocks = 4; };
template <> struct RegShape<8> { static constexpr int kThreads = 256, kMinBlocks = 2; };
template <> struct RegShape<16> { static constexpr int kThreads = 128, kMinBlocks = 3; };

template <typename T, int NCH>
__global__ void __launch_bounds__(RegShape<NCH>::kThreads, RegShape<NCH>::kMinBlocks)
quant_rows_reg_kernel(const T* __restrict__ x, int8_t* __restrict__ q, float* __restrict__ scale,
                      int64_t rows, int64_t cols) {
  grid_dependency_wait();  // x may be the previous kernel's output
  grid_launch_dependents();
  const int64_t warps_total = (int64_t)gridDim.x * (blockDim.x / 32);
  const int lane = threadIdx.x & 31;
  const int n8 = (int)(cols / 8);
  for (int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5); row < rows;
       row += warps_total) {
    const uint4* x8 = reinterpret_cast<const uint4*>(x + row * cols);
    uint4 w[NCH];
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int i = c * 32 + lane;
      w[c] = i < n8 ? __ldg(x8 + i) : make_uint4(0u, 0u, 0u, 0u);
    }
    float amax = 0.f;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const uint32_t ws[4] = {w[c].x, w[c].y, w[c].z, w[c].w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = Pack<T>::unpack(ws[j]);
        amax = fmaxf(amax, fmaxf(fabsf(f.x), fabsf(f.y)));
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float s = __fdiv_rn(fmaxf(amax, 1e-6f), 127.0f);
    const float y = __frcp_rn(s);
    if (lane == 0) scale[row] = s;
    uint2* q8 = reinterpret_cast<uint2*>(q + row * cols);
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int i = c * 32 + lane;
      if (i < n8) {
        const uint32_t ws[4] = {w[c].x, w[c].y, w[c].z, w[c].w};
        uint32_t t[8];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = Pack<T>::unpack(ws[j]);
          t[2 * j] = quant_bits(f.x, s, y);
          t[2 * j + 1] = quant_bits(f.y, s, y);
        }
        const uint32_t lo = __byte_perm(__byte_perm(t[0], t[1], 0x0040), __byte_perm(t[2], t[3], 0x0040), 0x5410);
        const uint32_t hi = __byte_perm(__byte_perm(t[4], t[5], 0x0040), __byte_perm(t[6], t[7], 0x0040), 0x5410);
        q8[i] = make_uint2(lo, hi);
      }
    }
  }
}

template <typename T, int NCH>
cudaError_t launch_reg(const void* x, int8_t* q, float* scale, int64_t rows, int64_t cols,
                       cudaStream_t stream) {
  constexpr int threads = RegShape<NCH>::kThreads;
  const int64_t want = (rows + threads / 32 - 1) / (threads / 32);
  const int64_t cap = (int64_t)sm_count() * RegShape<NCH>::kMinBlocks;
  const int grid = (int)(want < cap ? want : cap);
  return launch_pdl(quant_rows_reg_kernel<T, NCH>, dim3(grid), dim3(threads), 0, stream,
                    static_cast<const T*>(x), q, scale, rows, cols);
}

template <typename T>
cudaError_t launch_typed(const void* x, int8_t* q, float* scale, int64_t rows, int64_t cols,
                         cudaStream_t stream) {
  if (cols <= 32 * 8 * 4) return launch_reg<T, 4>(x, q, scale, rows, cols, stream);
  if (cols <= 32 * 8 * 8) return launch_reg<T, 8>(x, q, scale, rows, cols, stream);
  if (cols <= 32 * 8 * 16) return launch_reg<T, 16>(x, q, scale, rows, cols, stream);
  const int threads = 256;
  const int64_t want = (rows + 7) / 8;
  const int64_t cap = (int64_t)sm_count() * 8;  // 8 CTAs of 8 warps per SM
  const int grid = (int)(want < cap ? want : cap);
  return launch_pdl(quant_rows_kernel<T>, dim3(grid), dim3(threads), 0, stream,
                    static_cast<const T*>(x), q, scale, rows, cols);
}

}  // namespace

int launch_quant_rows(const void* x, int8_t* q, float* scale, int64_t rows, int64_t cols,
                      int dtype, cudaStream_t stream) {
  if (dtype == TTJ_F16)
    TTJ_CUDA_TRY(launch_typed<__half>(x, q, scale, rows, cols, stream));
  else
    TTJ_CUDA_TRY(launch_typed<__nv_bfloat16>(x, q, scale, rows, cols, stream));
  return TTJ_OK;
}

}  // namespace ttj
