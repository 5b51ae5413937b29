// Flash-attention forward for sm_100a: one CTA per (128-query tile, batch, head).
//
// Q, K and V are read straight from the packed projection buffer qkv[B,S,3D]
// through one 3-D TMA descriptor (dims 3D x S x B, box 64 x 128 x 1, 128-byte
// swizzle), so the reference's head split (.view/.transpose/.contiguous) is a
// coordinate choice, and rows past S arrive as zeros.
//
// Roles (256 threads):
//   warp 0      TMA: Q once, then K_j / V_j tiles into KV_STAGES-deep rings
//   warp 1      MMA: S_j = Q K_j^T into TMEM (two S buffers, so QK_{j+1}
//               runs while softmax works on S_j), then O += P_j V_j with P
//               read from TMEM (tcgen05 "ts" form) and V from shared memory
//   warps 4..7  softmax: thread r owns query row r; loads its S row from
//               TMEM, masks, updates the running max / sum in fp32, writes P
//               (rounded to the input dtype) back to TMEM, rescales its O row
//               when the max grew, and finally normalises O and stores the
//               context row into ctx[B,S,D] at the head's columns (head merge).
//
// TMEM columns: S0 [0,128) S1 [128,256) P0 [256,320) P1 [320,384) O [384,384+HD).
#include "sm100_ptx.cuh"
#include "ttj_internal.h"

namespace ttj {
namespace {

constexpr int kBM = 128;     // queries per CTA
constexpr int kBN = 128;     // keys per KV tile
constexpr int kChunkBytes = 128 * 128;  // one [128 rows][64 cols] 16-bit swizzled box

constexpr uint32_t kColS = 0;
constexpr uint32_t kColP = 256;
constexpr uint32_t kColO = 384;
constexpr uint32_t kTmemCols = 512;

struct AttnParams {
  void* ctx;
  const uint8_t* key_mask;
  int B, S, H, D;
  int num_q_tiles;
  float scale_log2;  // head_dim^-0.5 * log2(e)
  int* status;
};

template <int HD>
struct AttnSmem {
  static constexpr int kStages = HD == 64 ? 3 : 2;
  static constexpr int kTileBytes = HD * 2 * 128;  // 128 rows x HD x 2 bytes
  static constexpr int kQOff = 0;
  static constexpr int kKOff = kTileBytes;
  static constexpr int kVOff = kKOff + kStages * kTileBytes;
  static constexpr int kBarOff = kVOff + kStages * kTileBytes;
  static constexpr int kTotal = 1024 + kBarOff + 512;
};

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <typename T, int HD, bool CAUSAL>
__global__ void __launch_bounds__(256, 1)
flash_fwd_kernel(const __grid_constant__ CUtensorMap tm, const AttnParams p) {
  using L = AttnSmem<HD>;
  constexpr int ST = L::kStages;
  constexpr int kChunks = HD / 64;
  constexpr int kBf16 = std::is_same<T, __nv_bfloat16>::value ? 1 : 0;
  constexpr uint32_t kIdescQK = idesc_f16(kBM, kBN, kBf16, 0);
  constexpr uint32_t kIdescPV = idesc_f16(kBM, HD, kBf16, 1);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sQ = smem + L::kQOff;
  uint8_t* sK = smem + L::kKOff;
  uint8_t* sV = smem + L::kVOff;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* q_full = bars;
  uint64_t* k_full = q_full + 1;
  uint64_t* k_empty = k_full + ST;
  uint64_t* v_full = k_empty + ST;
  uint64_t* v_empty = v_full + ST;
  uint64_t* s_full = v_empty + ST;   // [2]
  uint64_t* s_free = s_full + 2;     // [2]
  uint64_t* p_full = s_free + 2;     // [2]
  uint64_t* o_done = p_full + 2;     // [1] one phase per completed P.V
  uint64_t* drain = o_done + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int bh = blockIdx.x;
  const int b = bh / p.H;
  const int h = bh - b * p.H;
  const int qt = p.num_q_tiles - 1 - (int)blockIdx.y;  // heaviest causal tiles first
  const int q0 = qt * kBM;
  const int kv_tiles_total = (p.S + kBN - 1) / kBN;
  const int n_kv = CAUSAL ? min(qt + 1, kv_tiles_total) : kv_tiles_total;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < ST; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 128);
      mbar_init(&p_full[i], 128);
    }
    mbar_init(o_done, 1);
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
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tm);
      const int xq = h * HD, xk = p.D + h * HD, xv = 2 * p.D + h * HD;
      mbar_arrive_expect_tx(q_full, L::kTileBytes);
      for (int c = 0; c < kChunks; ++c) tma_load_3d(sQ + c * kChunkBytes, &tm, q_full, xq + 64 * c, q0, b);
      bool ok = true;
      for (int j = 0; ok && j < n_kv; ++j) {
        const int st = j % ST;
        const uint32_t ph = (j / ST) & 1;
        if (!mbar_wait(&k_empty[st], ph ^ 1u, p.status, kDevTimeoutSmemEmpty, abort_flag)) break;
        mbar_arrive_expect_tx(&k_full[st], L::kTileBytes);
        for (int c = 0; c < kChunks; ++c)
          tma_load_3d(sK + st * L::kTileBytes + c * kChunkBytes, &tm, &k_full[st], xk + 64 * c, j * kBN, b);
        if (!mbar_wait(&v_empty[st], ph ^ 1u, p.status, kDevTimeoutSmemEmpty, abort_flag)) break;
        mbar_arrive_expect_tx(&v_full[st], L::kTileBytes);
        for (int c = 0; c < kChunks; ++c)
          tma_load_3d(sV + st * L::kTileBytes + c * kChunkBytes, &tm, &v_full[st], xv + 64 * c, j * kBN, b);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      bool ok = mbar_wait(q_full, 0, p.status, kDevTimeoutTmaFull, abort_flag);
      const uint32_t q_addr = smem_u32(sQ);
      auto issue_qk = [&](int j) -> bool {
        const int st = j % ST;
        const uint32_t ph = (j / ST) & 1;
        const int sb = j & 1;
        if (!mbar_wait(&k_full[st], ph, p.status, kDevTimeoutTmaFull, abort_flag)) return false;
        if (j >= 2 && !mbar_wait(&s_free[sb], ((j >> 1) - 1) & 1, p.status, kDevTimeoutSoftmax, abort_flag))
          return false;
        tc_fence_after();
        const uint32_t k_addr = smem_u32(sK + st * L::kTileBytes);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t off = (kk >> 2) * kChunkBytes + (kk & 3) * 32;
          umma_f16_ss(tmem + kColS + sb * 128, smem_desc_sw128(q_addr + off, 16, 1024),
                      smem_desc_sw128(k_addr + off, 16, 1024), kIdescQK, kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[sb]);
        umma_commit(&k_empty[st]);
        return true;
      };
      auto issue_pv = [&](int j) -> bool {
        const int st = j % ST;
        const uint32_t ph = (j / ST) & 1;
        const int pb = j & 1;
        if (!mbar_wait(&v_full[st], ph, p.status, kDevTimeoutTmaFull, abort_flag)) return false;
        if (!mbar_wait(&p_full[pb], (j >> 1) & 1, p.status, kDevTimeoutSoftmax, abort_flag)) return false;
        tc_fence_after();
        const uint32_t v_addr = smem_u32(sV + st * L::kTileBytes);
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk) {
          // V is MN-major: 16 keys = 16 rows of 128 bytes; next 64-column chunk at +16 KB.
          umma_f16_ts(tmem + kColO, tmem + kColP + pb * 64 + kk * 8,
                      smem_desc_sw128(v_addr + kk * 16 * 128, kChunkBytes, 1024), kIdescPV,
                      (j > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&v_empty[st]);
        umma_commit(o_done);
        return true;
      };
      if (ok) ok = issue_qk(0);
      for (int j = 0; ok && j < n_kv; ++j) {
        if (j + 1 < n_kv && !issue_qk(j + 1)) break;
        if (!issue_pv(j)) break;
      }
      umma_commit(drain);
      mbar_wait(drain, 0, p.status, kDevTimeoutSoftmax, nullptr);
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ softmax
    const int lg = warp & 3;             // TMEM lane quarter
    const int r = lg * 32 + lane;        // query row within the tile
    const int q_row = q0 + r;
    const uint32_t t_lane = tmem + (static_cast<uint32_t>(lg * 32) << 16);
    const uint8_t* kmask = p.key_mask != nullptr ? p.key_mask + (int64_t)b * p.S : nullptr;
    float m_run = -INFINITY;  // running max, log2 domain
    float l_run = 0.f;        // running sum of P (fp32, before rounding)
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      const int sb = j & 1;
      if (!mbar_wait_warp(&s_full[sb], (j >> 1) & 1, p.status, kDevTimeoutSoftmax, abort_flag)) { ok = false; break; }
      tc_fence_after();
      float s[kBN];
#pragma unroll
      for (int c = 0; c < kBN / 32; ++c) {
        uint32_t u[32];
        tmem_ld32(t_lane + kColS + sb * 128 + c * 32, u);
#pragma unroll
        for (int i = 0; i < 32; ++i) s[c * 32 + i] = __uint_as_float(u[i]);
      }
      tc_fence_before();
      mbar_arrive(&s_free[sb]);

      const int k0 = j * kBN;
      const bool need_mask = (k0 + kBN > p.S) || (CAUSAL && k0 + kBN - 1 > q0) || kmask != nullptr;
      if (need_mask) {
        // Validity bits for the tile's 128 keys, built cooperatively: lane l
        // reads keys l, l+32, l+64, l+96 and one ballot per group of 32.
        uint32_t vbits[4];
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          const int key = k0 + g * 32 + lane;
          bool v = key < p.S;
          if (v && kmask != nullptr) v = kmask[key] != 0;
          vbits[g] = __ballot_sync(0xffffffffu, v);
        }
#pragma unroll
        for (int i = 0; i < kBN; ++i) {
          bool v = (vbits[i >> 5] >> (i & 31)) & 1u;
          if (CAUSAL) v = v && (k0 + i <= q_row);
          s[i] = v ? s[i] : -INFINITY;
        }
      }
      float mx = -INFINITY;
#pragma unroll
      for (int i = 0; i < kBN; ++i) mx = fmaxf(mx, s[i]);
      const float m_new = fmaxf(m_run, mx * p.scale_log2);
      const float m_use = m_new == -INFINITY ? 0.f : m_new;
      const float alpha = fast_exp2(m_run - m_use);  // 0 when m_run = -inf
      float sum = 0.f;
      const uint32_t t_p = t_lane + kColP + sb * 64;
#pragma unroll
      for (int c = 0; c < kBN / 32; ++c) {
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float e0 = fast_exp2(fmaf(s[c * 32 + 2 * i], p.scale_log2, -m_use));
          const float e1 = fast_exp2(fmaf(s[c * 32 + 2 * i + 1], p.scale_log2, -m_use));
          sum += e0 + e1;
          pk[i] = Pack<T>::two(e0, e1);
        }
        tmem_st16(t_p + c * 16, pk);
      }
      l_run = l_run * alpha + sum;
      // O may only be rescaled once P_{j-1} V_{j-1} has landed.
      if (j > 0) {
        if (!mbar_wait_warp(o_done, (j - 1) & 1, p.status, kDevTimeoutSoftmax, abort_flag)) { ok = false; break; }
        tc_fence_after();
        if (__any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll
          for (int c = 0; c < HD / 32; ++c) {
            uint32_t o[32];
            tmem_ld32(t_lane + kColO + c * 32, o);
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st32(t_lane + kColO + c * 32, o);
          }
        }
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&p_full[sb]);
      m_run = m_new;
    }
    if (ok && mbar_wait_warp(o_done, (n_kv - 1) & 1, p.status, kDevTimeoutSoftmax, abort_flag)) {
      tc_fence_after();
      const float inv_l = 1.f / l_run;
      T* dst = static_cast<T*>(p.ctx) + ((int64_t)b * p.S + q_row) * p.D + h * HD;
#pragma unroll
      for (int c = 0; c < HD / 32; ++c) {
        uint32_t o[32];
        tmem_ld32(t_lane + kColO + c * 32, o);
        if (q_row < p.S) {
          uint4* d4 = reinterpret_cast<uint4*>(dst + c * 32);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 w;
            w.x = Pack<T>::two(__uint_as_float(o[8 * q + 0]) * inv_l, __uint_as_float(o[8 * q + 1]) * inv_l);
            w.y = Pack<T>::two(__uint_as_float(o[8 * q + 2]) * inv_l, __uint_as_float(o[8 * q + 3]) * inv_l);
            w.z = Pack<T>::two(__uint_as_float(o[8 * q + 4]) * inv_l, __uint_as_float(o[8 * q + 5]) * inv_l);
            w.w = Pack<T>::two(__uint_as_float(o[8 * q + 6]) * inv_l, __uint_as_float(o[8 * q + 7]) * inv_l);
            d4[q] = w;
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, kTmemCols);
}

template <typename T, int HD, bool CAUSAL>
int launch_attn(const AttnArgs& a, cudaStream_t stream) {
  using L = AttnSmem<HD>;
  const int64_t D = a.num_heads * a.head_dim;
  CUtensorMap tm;
  const uint64_t dims[3] = {(uint64_t)(3 * D), (uint64_t)a.seq_len, (uint64_t)a.batch};
  const uint64_t strides[2] = {(uint64_t)(3 * D * 2), (uint64_t)(a.seq_len * 3 * D * 2)};
  const uint32_t box[3] = {64, 128, 1};
  int rc = encode_tmap(&tm, std::is_same<T, __half>::value ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                           : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                       3, a.qkv, dims, strides, box);
  if (rc) return rc;
  AttnParams p;
  p.ctx = a.ctx;
  p.key_mask = a.key_mask;
  p.B = (int)a.batch;
  p.S = (int)a.seq_len;
  p.H = (int)a.num_heads;
  p.D = (int)D;
  p.num_q_tiles = (int)((a.seq_len + kBM - 1) / kBM);
  p.scale_log2 = (float)(1.0 / sqrt((double)HD) * 1.4426950408889634);
  p.status = a.status;
  auto kern = flash_fwd_kernel<T, HD, CAUSAL>;
  TTJ_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kTotal));
  dim3 grid((unsigned)(a.batch * a.num_heads), (unsigned)p.num_q_tiles);
  kern<<<grid, 256, L::kTotal, stream>>>(tm, p);
  TTJ_CUDA_TRY(cudaGetLastError());
  return TTJ_OK;
}

template <typename T>
int dispatch_hd(const AttnArgs& a, cudaStream_t stream) {
  if (a.head_dim == 64) return a.causal ? launch_attn<T, 64, true>(a, stream) : launch_attn<T, 64, false>(a, stream);
  return a.causal ? launch_attn<T, 128, true>(a, stream) : launch_attn<T, 128, false>(a, stream);
}

}  // namespace

int launch_flash_attn(const AttnArgs& a, cudaStream_t stream) {
  return a.dtype == TTJ_F16 ? dispatch_hd<__half>(a, stream) : dispatch_hd<__nv_bfloat16>(a, stream);
}

}  // namespace ttj
