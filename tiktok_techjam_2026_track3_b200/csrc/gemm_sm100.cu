// Persistent tcgen05 GEMM  y[M,N] = a[M,K] . b[N,K]^T  with fused epilogues.
//
// Roles (192 threads, one CTA per SM, persistent over output tiles):
//   warp 0      TMA producer: A and B K-slices into a STAGES-deep shared ring
//   warp 1      MMA issuer: one thread issues tcgen05.mma into a TMEM accumulator
//   warps 2..5  epilogue: tcgen05.ld the accumulator (one TMEM lane = one output
//               row per thread), add bias / dequantise / add residual, store
// The accumulator is double-buffered in TMEM (2 x BN fp32 columns) so the
// epilogue of tile i overlaps the MMAs of tile i+1.
//
// Operand tiles are 128-byte rows (64 fp16/bf16 or 128 int8 elements of K)
// in TMA's 128-byte swizzle; each tcgen05.mma consumes 32 bytes of K.
// Tiles are visited N-fastest so the CTAs resident at one time share a few
// A row-blocks while the (smaller) weight matrix stays L2 resident.
#include <type_traits>

#include "sm100_ptx.cuh"
#include "ttj_internal.h"

namespace ttj {
namespace {

constexpr int kBM = 128;
constexpr int kRowBytes = 128;  // bytes of K per smem row (one swizzle atom)

struct GemmParams {
  int M, N, K;
  int num_m_blocks, num_n_blocks;
  const void* bias;
  const void* residual;
  const uint8_t* row_mask;
  const float* scale_a;
  const float* scale_b;
  void* out;
  int* status;
};

template <typename TIn, int BN, int STAGES>
struct GemmSmem {
  static constexpr int kABytes = kBM * kRowBytes;
  static constexpr int kBBytes = BN * kRowBytes;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kBarrierBytes = 256;
  static constexpr int kTotal = 1024 /*align slack*/ + STAGES * kStageBytes + kBarrierBytes;
};

// Load 32 consecutive 16-bit values as floats (four 16-byte loads).
template <typename T>
__device__ __forceinline__ void load32_f(const T* src, float (&v)[32]) {
  const uint4* s = reinterpret_cast<const uint4*>(src);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint4 w = __ldg(s + q);
    uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float2 f = Pack<T>::unpack(ws[j]);
      v[q * 8 + 2 * j] = f.x;
      v[q * 8 + 2 * j + 1] = f.y;
    }
  }
}

template <typename T>
__device__ __forceinline__ void store32_f(T* dst, const float (&v)[32]) {
  uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint4 w;
    w.x = Pack<T>::two(v[q * 8 + 0], v[q * 8 + 1]);
    w.y = Pack<T>::two(v[q * 8 + 2], v[q * 8 + 3]);
    w.z = Pack<T>::two(v[q * 8 + 4], v[q * 8 + 5]);
    w.w = Pack<T>::two(v[q * 8 + 6], v[q * 8 + 7]);
    d[q] = w;
  }
}

template <typename TIn, typename TOut, int BN, int STAGES, int EPI>
__global__ void __launch_bounds__(192, 1)
gemm_tn_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
               const GemmParams p) {
  using L = GemmSmem<TIn, BN, STAGES>;
  constexpr bool kInt8 = std::is_same<TIn, int8_t>::value;
  constexpr int kBK = kRowBytes / sizeof(TIn);             // K elements per stage
  constexpr uint32_t kTmemCols = 2 * BN;                   // 256 or 512
  constexpr uint32_t kIdesc =
      kInt8 ? idesc_i8(kBM, BN)
            : idesc_f16(kBM, BN, std::is_same<TIn, __nv_bfloat16>::value ? 1 : 0, 0);
  static_assert(kTmemCols == 256 || kTmemCols == 512, "TMEM columns must be a power of 2");

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * L::kABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * L::kStageBytes);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 128);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    __syncwarp();
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int num_tiles = p.num_m_blocks * p.num_n_blocks;
  const int num_kb = (p.K + kBK - 1) / kBK;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x) {
        const int m_blk = tile / p.num_n_blocks;
        const int n_blk = tile - m_blk * p.num_n_blocks;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, p.status, kDevTimeoutSmemEmpty, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], L::kStageBytes);
          tma_load_2d(sA + stage * L::kABytes, &tmA, &full[stage], kb * kBK, m_blk * kBM);
          tma_load_2d(sB + stage * L::kBBytes, &tmB, &full[stage], kb * kBK, n_blk * BN);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1u, p.status, kDevTimeoutAccEmpty, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, p.status, kDevTimeoutTmaFull, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * L::kABytes);
          const uint32_t b_addr = smem_u32(sB + stage * L::kBBytes);
#pragma unroll
          for (int kk = 0; kk < kRowBytes / 32; ++kk) {
            const uint64_t ad = smem_desc_sw128(a_addr + kk * 32, 16, 1024);
            const uint64_t bd = smem_desc_sw128(b_addr + kk * 32, 16, 1024);
            const uint32_t accum = (kb | kk) != 0 ? 1u : 0u;
            if constexpr (kInt8)
              umma_i8_ss(d_tmem, ad, bd, kIdesc, accum);
            else
              umma_f16_ss(d_tmem, ad, bd, kIdesc, accum);
          }
          umma_commit(&empty[stage]);  // stage is free once these MMAs have read it
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&acc_full[acc]);
      }
      // Drain: nothing may still write TMEM when it is released.
      umma_commit(drain);
      mbar_wait(drain, 0, p.status, kDevTimeoutAccFull, nullptr);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int lane_grp = warp & 3;  // TMEM lane quarter this warp may access
    const int row = lane_grp * 32 + lane;
    int local = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait_warp(&acc_full[acc], acc_phase, p.status, kDevTimeoutAccFull, abort_flag)) break;
      tc_fence_after();
      const int m_blk = tile / p.num_n_blocks;
      const int n_blk = tile - m_blk * p.num_n_blocks;
      const int m = m_blk * kBM + row;
      const bool row_ok = m < p.M;
      float row_scale = 0.f;
      bool row_keep = true;
      if constexpr (EPI == (int)Epi::kDequant || EPI == (int)Epi::kDequantResidual) {
        if (row_ok) row_scale = __ldg(p.scale_a + m);
      }
      if constexpr (EPI != (int)Epi::kRawS32) {
        if (row_ok && p.row_mask != nullptr) row_keep = __ldg(p.row_mask + m) != 0;
      }
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(lane_grp * 32) << 16) + acc * BN;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(t_row + c * 32, r);  // warp-collective: every lane executes it
        const int n0 = n_blk * BN + c * 32;
        if (!row_ok || n0 >= p.N) continue;
        if constexpr (EPI == (int)Epi::kRawS32) {
          int4* dst = reinterpret_cast<int4*>(static_cast<int32_t*>(p.out) + (int64_t)m * p.N + n0);
#pragma unroll
          for (int q = 0; q < 8; ++q)
            dst[q] = make_int4((int)r[4 * q], (int)r[4 * q + 1], (int)r[4 * q + 2], (int)r[4 * q + 3]);
        } else {
          float v[32];
          if constexpr (EPI == (int)Epi::kBias || EPI == (int)Epi::kBiasResidual) {
            float b[32];
            load32_f(static_cast<const TOut*>(p.bias) + n0, b);
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]) + b[i];
          } else {
            // k008 recipe order: acc * (s_a * s_w) + bias, each step rounded.
            const float4* sb = reinterpret_cast<const float4*>(p.scale_b + n0);
            const float4* bb = reinterpret_cast<const float4*>(static_cast<const float*>(p.bias) + n0);
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              const float4 s4 = __ldg(sb + q);
              const float4 b4 = __ldg(bb + q);
              const float ss[4] = {s4.x, s4.y, s4.z, s4.w};
              const float bs[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const float acc_f = static_cast<float>(static_cast<int32_t>(r[4 * q + j]));
                v[4 * q + j] = __fadd_rn(__fmul_rn(acc_f, __fmul_rn(row_scale, ss[j])), bs[j]);
              }
            }
          }
          if constexpr (EPI == (int)Epi::kBiasResidual || EPI == (int)Epi::kDequantResidual) {
            float res[32];
            load32_f(static_cast<const TOut*>(p.residual) + (int64_t)m * p.N + n0, res);
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = row_keep ? res[i] + v[i] : res[i];
          } else {
            // Output-row masking without a residual (reference masked_fill of the
            // attention output, torch_transformer_benchmark.py:120-121).
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = row_keep ? v[i] : 0.f;
          }
          store32_f(static_cast<TOut*>(p.out) + (int64_t)m * p.N + n0, v);
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[acc]);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem_base, kTmemCols);
}

template <typename TIn, typename TOut, int BN, int STAGES, int EPI>
int launch_one(const GemmArgs& g, cudaStream_t stream) {
  using L = GemmSmem<TIn, BN, STAGES>;
  constexpr int kBK = kRowBytes / sizeof(TIn);
  const CUtensorMapDataType dt = std::is_same<TIn, int8_t>::value ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                 : std::is_same<TIn, __half>::value
                                     ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                     : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUtensorMap ta, tb;
  {
    const uint64_t dims[2] = {(uint64_t)g.k, (uint64_t)g.m};
    const uint64_t strides[1] = {(uint64_t)g.k * sizeof(TIn)};
    const uint32_t box[2] = {(uint32_t)kBK, (uint32_t)kBM};
    int rc = encode_tmap(&ta, dt, 2, g.a, dims, strides, box);
    if (rc) return rc;
  }
  {
    const uint64_t dims[2] = {(uint64_t)g.k, (uint64_t)g.n};
    const uint64_t strides[1] = {(uint64_t)g.k * sizeof(TIn)};
    const uint32_t box[2] = {(uint32_t)kBK, (uint32_t)BN};
    int rc = encode_tmap(&tb, dt, 2, g.b, dims, strides, box);
    if (rc) return rc;
  }
  GemmParams p;
  p.M = (int)g.m;
  p.N = (int)g.n;
  p.K = (int)g.k;
  p.num_m_blocks = (int)((g.m + kBM - 1) / kBM);
  p.num_n_blocks = (int)((g.n + BN - 1) / BN);
  p.bias = g.bias;
  p.residual = g.residual;
  p.row_mask = g.row_mask;
  p.scale_a = g.scale_a;
  p.scale_b = g.scale_b;
  p.out = g.out;
  p.status = g.status;
  const int tiles = p.num_m_blocks * p.num_n_blocks;
  const int grid = tiles < sm_count() ? tiles : sm_count();
  auto kern = gemm_tn_kernel<TIn, TOut, BN, STAGES, EPI>;
  TTJ_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kTotal));
  kern<<<grid, 192, L::kTotal, stream>>>(ta, tb, p);
  TTJ_CUDA_TRY(cudaGetLastError());
  return TTJ_OK;
}

template <typename TIn, typename TOut, int EPI>
int dispatch_bn(const GemmArgs& g, cudaStream_t stream) {
  // BN = 256 halves the A re-reads; BN = 128 when N is small or would waste a
  // half-empty tile column.
  if (g.n % 256 == 0 && g.n >= 512) return launch_one<TIn, TOut, 256, 4, EPI>(g, stream);
  return launch_one<TIn, TOut, 128, 6, EPI>(g, stream);
}

template <typename TIn, typename TOut>
int dispatch_epi(const GemmArgs& g, cudaStream_t stream) {
  switch (g.epi) {
    case Epi::kBias: return dispatch_bn<TIn, TOut, (int)Epi::kBias>(g, stream);
    case Epi::kBiasResidual: return dispatch_bn<TIn, TOut, (int)Epi::kBiasResidual>(g, stream);
    default: return fail(TTJ_ERR_INVALID_ARG, "epilogue not valid for 16-bit operands");
  }
}

template <typename TOut>
int dispatch_int8(const GemmArgs& g, cudaStream_t stream) {
  switch (g.epi) {
    case Epi::kDequant: return dispatch_bn<int8_t, TOut, (int)Epi::kDequant>(g, stream);
    case Epi::kDequantResidual:
      return dispatch_bn<int8_t, TOut, (int)Epi::kDequantResidual>(g, stream);
    default: return fail(TTJ_ERR_INVALID_ARG, "epilogue not valid for int8 operands");
  }
}

}  // namespace

int launch_gemm(const GemmArgs& g, cudaStream_t stream) {
  if (g.in_dtype == TTJ_F16) return dispatch_epi<__half, __half>(g, stream);
  if (g.in_dtype == TTJ_BF16) return dispatch_epi<__nv_bfloat16, __nv_bfloat16>(g, stream);
  // int8 operands
  if (g.epi == Epi::kRawS32) return dispatch_bn<int8_t, int32_t, (int)Epi::kRawS32>(g, stream);
  if (g.out_dtype == TTJ_F16) return dispatch_int8<__half>(g, stream);
  return dispatch_int8<__nv_bfloat16>(g, stream);
}

}  // namespace ttj
