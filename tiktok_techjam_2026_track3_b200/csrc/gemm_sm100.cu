// Persistent tcgen05 GEMM  y[M,N] = a[M,K] . b[N,K]^T  with fused epilogues.
//
// Roles (320 threads per CTA, one CTA per SM, persistent over output tiles):
//   warp 0      TMA producer: A and B K-slices into a STAGES-deep shared ring
//   warp 1      MMA issuer: one thread issues tcgen05.mma into a TMEM accumulator
//   warps 2..9  epilogue: two warps per TMEM lane quarter (32 output rows), each
//               taking half of the tile's columns in 64-column chunks
// The accumulator is double-buffered in TMEM (2 x BN fp32 columns) so the
// epilogue of tile i overlaps the MMAs of tile i+1.
//
// Epilogue data path: for each 32-row x 64-column chunk a warp TMA-loads the
// residual box (if any) into one of its two 4 KB staging buffers (128-byte
// swizzle), tcgen05.ld's the 64 accumulator columns of its rows, adds bias /
// dequantises / adds the residual in fp32, writes the 16-bit result back into
// the same buffer and TMA-stores the box.  Full 128-byte lines move in both
// directions; per-thread row-segment loads and stores (32 rows x 16 bytes per
// warp instruction) were measured to cost more than the MMAs themselves.
//
// Operand tiles are 128-byte rows (64 fp16/bf16 or 128 int8 elements of K)
// in TMA's 128-byte swizzle; each tcgen05.mma consumes 32 bytes of K.
// Tiles are visited N-fastest so the CTAs resident at one time share a few
// A row-blocks while the (smaller) weight matrix stays L2 resident.
//
// Two kernels share this epilogue: a single-CTA 128 x BN tile (for M <= 128)
// and a CTA-pair (tcgen05 cta_group::2) 256 x BN tile for everything larger.
#include <type_traits>

#include "sm100_ptx.cuh"
#include "ttj_internal.h"

namespace ttj {
namespace {

constexpr int kBM = 128;
constexpr int kRowBytes = 128;  // bytes of K per smem row (one swizzle atom)
constexpr int kEpiWarps = 8;
constexpr int kGemmThreads = 64 + 32 * kEpiWarps;
constexpr int kEpiBoxRows = 32;
constexpr int kEpiBoxCols = 64;                       // 16-bit: one 128-byte swizzle row
constexpr int kEpiBoxBytes = kEpiBoxRows * 128;       // 4 KB
// Staging buffers per epilogue warp.  One (32 KB in all) leaves room for a
// deeper operand ring (measured: 6 stages + 1 buffer beat 5 stages + 2 buffers
// by 2% on the layer's projections; the epilogue overlaps the next tile's MMAs
// and has slack for the serialisation).
constexpr int kEpiBufs = 1;
constexpr int kEpiBytes = kEpiWarps * kEpiBufs * kEpiBoxBytes;
constexpr int kBarrierBytes = 512;

struct GemmParams {
  int M, N, K;
  int a_kchunk;  // > 0: A is K-chunk-major [K/a_kchunk][M][a_kchunk] (3-D tensor map)
  int num_m_blocks, num_n_blocks;
  // CTA pairs with 256-column tiles: tiles [0, full_tiles) run whole, the rest
  // (a last partial wave) as two 128-column halves each, so the pairs share
  // that wave's work; num_units = full_tiles + 2 * (tiles - full_tiles).
  int full_tiles, num_units;
  const void* bias;
  const uint8_t* row_mask;
  const float* scale_a;
  const float* scale_b;
  void* out;  // only used by the int32 (raw accumulator) epilogue
  int* status;
};

// Shared-memory layout common to both kernels: [stages][epilogue buffers][barriers].
template <int STAGE_BYTES, int STAGES>
struct GemmLayout {
  static constexpr int kEpiOff = STAGES * STAGE_BYTES;
  static constexpr int kBarOff = kEpiOff + kEpiBytes;
  static constexpr int kTotal = 1024 /*align slack*/ + kBarOff + kBarrierBytes;
  static_assert(kTotal <= 232448, "shared memory budget");
};

// Per-warp epilogue state kept across tiles (scalars, so it stays in registers).
struct EpiState {
  uint8_t* buf0;       // kEpiBufs 1024-aligned 4 KB staging buffers (buf1 == buf0 if one)
  uint8_t* buf1;
  uint64_t* bar0;      // residual-load barriers, one per buffer
  uint64_t* bar1;
  uint32_t phase0, phase1;
  int next;            // buffer to use next
  int pending;         // the residual box of this warp's first chunk is already requested
};

// Hands a tile's TMEM accumulator back to the MMA thread once this warp has
// read its part of it (one arrival per epilogue warp and tile), before the
// warp's stores: on this CTA's barrier, or on the pair leader's (cluster
// address) for a CTA pair.  arrive() is idempotent, so every exit path of an
// epilogue can end with it.
struct AccRelease {
  uint64_t* local;   // this CTA's barrier, or null
  uint32_t remote;   // shared::cluster address of the leader's barrier (local == null)
  bool done;
  __device__ __forceinline__ void arrive() {
    if (done) return;
    tc_fence_before();
    __syncwarp();
    if ((threadIdx.x & 31) == 0) {
      if (local != nullptr) mbar_arrive(local);
      else mbar_arrive_cluster(remote);
    }
    done = true;
  }
};

__device__ __forceinline__ uint32_t swz(int row, int chunk16) {
  return static_cast<uint32_t>(row * 128 + ((chunk16 ^ (row & 7)) << 4));
}

template <typename T>
__device__ __forceinline__ void unpack8(uint4 w, float (&v)[8]) {
  const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 f = Pack<T>::unpack(ws[j]);
    v[2 * j] = f.x;
    v[2 * j + 1] = f.y;
  }
}

template <typename T>
__device__ __forceinline__ uint4 pack8(const float (&v)[8]) {
  uint4 w;
  w.x = Pack<T>::two(v[0], v[1]);
  w.y = Pack<T>::two(v[2], v[3]);
  w.z = Pack<T>::two(v[4], v[5]);
  w.w = Pack<T>::two(v[6], v[7]);
  return w;
}

// Packed fp32 pairs (sm_100 f32x2 arithmetic: two lanes per instruction).
__device__ __forceinline__ uint64_t x2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void x2_split(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t x2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t x2_mul(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// Exact-erf GELU of two values, v/2 * (1 + erf(v / sqrt 2)), as F.gelu with
// approximate="none" (torch_transformer_benchmark.py:141), through the
// complementary error function: with z = v / sqrt 2, a = |z| and s = sign(z),
// 1 + erf(z) = (1 + s) - s * erfc(a), which for z < 0 is erfc(a) itself, so the
// negative tail keeps full relative precision.  erfc is the Chebyshev-fitted
// form of Numerical Recipes (Press et al., 2nd ed., section 6.2, "erfcc"):
//   erfc(a) = t * exp(-a^2 + P(t)),  t = 1 / (1 + a/2),  P of degree 9,
// fractional error below 1.2e-7 for every a >= 0.  Checked against float64
// exact GELU: results round to the same 16-bit value (tests/test_gpu_block.py).
// Measured: the library erff made this epilogue issue-bound (143 us for the
// 16384x1024->4096 FFN GEMM against 102 us without GELU); here two MUFU
// operations per value and paired fp32 arithmetic (two lanes per instruction).
__device__ __forceinline__ void gelu_erf_pair(float& v0, float& v1) {
  const uint64_t v = x2(v0, v1);
  const uint64_t z = x2_mul(v, x2(0.70710678118654752f, 0.70710678118654752f));
  float z0, z1;
  x2_split(z, z0, z1);
  const uint64_t a = x2(fabsf(z0), fabsf(z1));
  float d0, d1;
  x2_split(x2_fma(a, x2(0.5f, 0.5f), x2(1.f, 1.f)), d0, d1);
  float t0, t1;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(t0) : "f"(d0));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(t1) : "f"(d1));
  const uint64_t t = x2(t0, t1);
  uint64_t q = x2_fma(t, x2(0.17087277f, 0.17087277f), x2(-0.82215223f, -0.82215223f));
  q = x2_fma(q, t, x2(1.48851587f, 1.48851587f));
  q = x2_fma(q, t, x2(-1.13520398f, -1.13520398f));
  q = x2_fma(q, t, x2(0.27886807f, 0.27886807f));
  q = x2_fma(q, t, x2(-0.18628806f, -0.18628806f));
  q = x2_fma(q, t, x2(0.09678418f, 0.09678418f));
  q = x2_fma(q, t, x2(0.37409196f, 0.37409196f));
  q = x2_fma(q, t, x2(1.00002368f, 1.00002368f));
  q = x2_fma(q, t, x2(-1.26551223f, -1.26551223f));
  // exp(-a^2 + P) = 2^((P - a^2) * log2 e)
  const uint64_t neg_a = x2(-fabsf(z0), -fabsf(z1));
  const uint64_t expo = x2_mul(x2_fma(neg_a, a, q), x2(1.4426950408889634f, 1.4426950408889634f));
  float x0e, x1e;
  x2_split(expo, x0e, x1e);
  float e0, e1;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e0) : "f"(x0e));
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e1) : "f"(x1e));
  const uint64_t erfc = x2_mul(t, x2(e0, e1));
  // -s as +-1.0: the sign bit of z flipped onto 1.0f
  const uint64_t neg_s = x2(__uint_as_float((__float_as_uint(z0) & 0x80000000u) ^ 0xbf800000u),
                            __uint_as_float((__float_as_uint(z1) & 0x80000000u) ^ 0xbf800000u));
  const uint64_t one_p_s = x2_fma(neg_s, x2(-1.f, -1.f), x2(1.f, 1.f));  // 1 + s
  const uint64_t one_p_erf = x2_fma(neg_s, erfc, one_p_s);
  x2_split(x2_mul(x2_mul(v, x2(0.5f, 0.5f)), one_p_erf), v0, v1);
}

// fp32-output epilogue (16-bit operands, fp32 bias, fp32 residual and output):
// the residual stream of an fp32 model.  Same data path as the 16-bit one, with
// 32-column boxes (128 bytes of fp32 per row) instead of 64.
//   kBias                  y = mask(acc + bias)
//   kBiasResidual          y = residual + mask(acc + bias)
//   kBiasResidualZeroRows  y = mask(residual + acc + bias)
template <int BN, int EPI>
__device__ __forceinline__ void epilogue_tile_f32(const GemmParams& p, const CUtensorMap* tm_out,
                                                  const CUtensorMap* tm_res, uint32_t t_row, int row0,
                                                  int n_blk, int col_half, EpiState& es, AccRelease& rel,
                                                  int* status, volatile int* abort_flag) {
  constexpr bool kZeroRows = EPI == (int)Epi::kBiasResidualZeroRows;
  constexpr bool kResidual = EPI == (int)Epi::kBiasResidual || kZeroRows;
  static_assert(kResidual || EPI == (int)Epi::kBias, "fp32 output: bias / residual epilogues only");
  constexpr int kChunks = BN / 32 / 2;
  const int lane = threadIdx.x & 31;
  const int m = row0 + lane;
  if (row0 >= p.M) return;  // the warp's 32 rows are all past the last row (uniform)
  bool row_keep = true;
  if (m < p.M && p.row_mask != nullptr) row_keep = __ldg(p.row_mask + m) != 0;
#pragma unroll 1
  for (int cc = 0; cc < kChunks; ++cc) {
    const int c = col_half * kChunks + cc;
    const int n0 = n_blk * BN + c * 32;
    const int b = es.next;
    if (kEpiBufs == 2) es.next ^= 1;
    uint8_t* buf = b ? es.buf1 : es.buf0;
    uint64_t* bar = b ? es.bar1 : es.bar0;
    if (lane == 0) bulk_wait_group_read<kEpiBufs - 1>();
    __syncwarp();
    if (n0 >= p.N) continue;  // whole chunk past the last column (uniform)
    if constexpr (kResidual) {
      if (lane == 0) {
        mbar_arrive_expect_tx(bar, kEpiBoxBytes);
        tma_load_2d(buf, tm_res, bar, n0, row0);
      }
    }
    uint32_t r[32];
    tmem_ld32(t_row + c * 32, r);  // warp-collective
    if (cc == kChunks - 1) rel.arrive();  // the accumulator is in registers
    // Every load of the chunk is issued before any arithmetic (16-byte slot q:
    // columns n0 + 4q .. +3; N % 32 == 0, so all valid).
    float4 bias[8];
#pragma unroll
    for (int q = 0; q < 8; ++q)
      bias[q] = __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(p.bias) + n0 + 4 * q));
    float4 res[8];
    if constexpr (kResidual) {
      const uint32_t ph = b ? es.phase1 : es.phase0;
      if (!mbar_wait_warp<true>(bar, ph, status, kDevTimeoutTmaFull, abort_flag)) return;
      if (b) es.phase1 ^= 1u; else es.phase0 ^= 1u;
#pragma unroll
      for (int q = 0; q < 8; ++q) res[q] = *reinterpret_cast<const float4*>(buf + swz(lane, q));
    }
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      float v[4] = {__uint_as_float(r[4 * q]) + bias[q].x, __uint_as_float(r[4 * q + 1]) + bias[q].y,
                    __uint_as_float(r[4 * q + 2]) + bias[q].z, __uint_as_float(r[4 * q + 3]) + bias[q].w};
      if constexpr (kResidual) {
        const float rr[4] = {res[q].x, res[q].y, res[q].z, res[q].w};
#pragma unroll
        for (int i = 0; i < 4; ++i) v[i] = row_keep ? rr[i] + v[i] : (kZeroRows ? 0.f : rr[i]);
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) v[i] = row_keep ? v[i] : 0.f;
      }
      res[q] = make_float4(v[0], v[1], v[2], v[3]);
    }
#pragma unroll
    for (int q = 0; q < 8; ++q) *reinterpret_cast<float4*>(buf + swz(lane, q)) = res[q];
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      tma_store_2d(tm_out, buf, n0, row0);  // rows >= M are clipped
      bulk_commit_group();
    }
  }
}

// Epilogue of one output tile for one warp.  t_row = TMEM address of this
// thread's lane at the accumulator buffer's first column; row0 = first of the
// warp's 32 output rows; the warp handles columns half `col_half` of
// [n_blk*BN, n_blk*BN + BN).  `rel` hands the accumulator back as soon as the
// warp's last TMEM load has completed.  next_row0 / next_n0 locate the warp's
// part of its next tile (first row, first column; next_row0 < 0: none): with a residual and one
// staging buffer, that tile's first residual box is requested at the end of
// this one, so it arrives while the next accumulator is still being computed.
// Measured (cfg2 out-proj, 16384 x 1024 -> 1024 + residual, in the layer):
// 41.0 -> 37-38 us, same output bits; per %globaltimer stamps, the residual
// box used to arrive ~1 us after its request and the accumulator was held
// through the stores.
template <typename TOut, int BN, int EPI>
__device__ __forceinline__ void epilogue_tile(const GemmParams& p, const CUtensorMap* tm_out,
                                              const CUtensorMap* tm_res, uint32_t t_row, int row0,
                                              int n_blk, int col_half, EpiState& es, AccRelease& rel,
                                              int* status, volatile int* abort_flag,
                                              int next_row0, int next_n0) {
  if constexpr (std::is_same<TOut, float>::value) {
    epilogue_tile_f32<BN, EPI>(p, tm_out, tm_res, t_row, row0, n_blk, col_half, es, rel, status, abort_flag);
    return;
  }
  const int lane = threadIdx.x & 31;
  const int m = row0 + lane;
  const bool row_ok = m < p.M;
  if (row0 >= p.M) return;  // the warp's 32 rows are all past the last row (uniform)
  if constexpr (EPI == (int)Epi::kRawS32) {
    // Raw int32 accumulators (bit-exactness checks only): direct row stores.
    constexpr int kChunks = BN / 32 / 2;
#pragma unroll 1
    for (int cc = 0; cc < kChunks; ++cc) {
      const int c = col_half * kChunks + cc;
      const int n0 = n_blk * BN + c * 32;
      uint32_t r[32];
      tmem_ld32(t_row + c * 32, r);
      if (cc == kChunks - 1) rel.arrive();
      if (!row_ok || n0 >= p.N) continue;
      int4* dst = reinterpret_cast<int4*>(static_cast<int32_t*>(p.out) + (int64_t)m * p.N + n0);
#pragma unroll
      for (int q = 0; q < 8; ++q)
        dst[q] = make_int4((int)r[4 * q], (int)r[4 * q + 1], (int)r[4 * q + 2], (int)r[4 * q + 3]);
    }
    return;
  } else if constexpr (!std::is_same<TOut, float>::value) {
    constexpr bool kZeroRows = EPI == (int)Epi::kBiasResidualZeroRows;
    constexpr bool kGelu = EPI == (int)Epi::kBiasGelu;
    constexpr bool kResidual =
        EPI == (int)Epi::kBiasResidual || EPI == (int)Epi::kDequantResidual || kZeroRows;
    constexpr bool kDequant = EPI == (int)Epi::kDequant || EPI == (int)Epi::kDequantResidual;
    constexpr int kChunks = BN / kEpiBoxCols / 2;
    float row_scale = 0.f;
    bool row_keep = true;
    if (kDequant && row_ok) row_scale = __ldg(p.scale_a + m);
    if (row_ok && p.row_mask != nullptr) row_keep = __ldg(p.row_mask + m) != 0;
#pragma unroll 1
    for (int cc = 0; cc < kChunks; ++cc) {
      const int c = col_half * kChunks + cc;
      const int n0 = n_blk * BN + c * kEpiBoxCols;
      const int b = es.next;
      if (kEpiBufs == 2) es.next ^= 1;
      uint8_t* buf = b ? es.buf1 : es.buf0;
      uint64_t* bar = b ? es.bar1 : es.bar0;
      // The store issued from this buffer kEpiBufs chunks ago must have read it.
      if (lane == 0) bulk_wait_group_read<kEpiBufs - 1>();
      __syncwarp();
      if (n0 >= p.N) continue;  // whole chunk past the last column (uniform)
      if constexpr (kResidual) {
        if (lane == 0 && !(cc == 0 && es.pending)) {
          mbar_arrive_expect_tx(bar, kEpiBoxBytes);
          tma_load_2d(buf, tm_res, bar, n0, row0);
        }
        if (cc == 0) es.pending = 0;
      }
      uint32_t r[64];
      tmem_ld64(t_row + c * kEpiBoxCols, r);  // warp-collective
      if (cc == kChunks - 1) rel.arrive();     // the accumulator is in registers
      if constexpr (!kDequant) {
        // Every load of the chunk before any arithmetic: bias (8 columns per
        // 16-byte word), then the residual box from shared memory.
        uint4 bw[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int col = n0 + 8 * j;
          bw[j] = col < p.N ? __ldg(reinterpret_cast<const uint4*>(static_cast<const TOut*>(p.bias) + col))
                            : make_uint4(0u, 0u, 0u, 0u);
        }
        uint4 w[8];
        if constexpr (kResidual) {
          const uint32_t ph = b ? es.phase1 : es.phase0;
          if (!mbar_wait_warp<true>(bar, ph, status, kDevTimeoutTmaFull, abort_flag)) return;
          if (b) es.phase1 ^= 1u; else es.phase0 ^= 1u;
#pragma unroll
          for (int j = 0; j < 8; ++j) w[j] = *reinterpret_cast<const uint4*>(buf + swz(lane, j));
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          float v[8], bias[8];
          unpack8<TOut>(bw[j], bias);
#pragma unroll
          for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[8 * j + i]) + bias[i];
          if constexpr (kResidual) {
            float res[8];
            unpack8<TOut>(w[j], res);
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = row_keep ? res[i] + v[i] : (kZeroRows ? 0.f : res[i]);
          } else if constexpr (kGelu) {
            // Exact (erf) GELU of the biased product (gelu_erf_pair above).
#pragma unroll
            for (int i = 0; i < 8; i += 2) gelu_erf_pair(v[i], v[i + 1]);
          } else {
            // Output-row masking without a residual (the reference's masked_fill
            // of the attention output, torch_transformer_benchmark.py:120-121).
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = row_keep ? v[i] : 0.f;
          }
          w[j] = pack8<TOut>(v);
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) *reinterpret_cast<uint4*>(buf + swz(lane, j)) = w[j];
      } else {
        if constexpr (kResidual) {
          const uint32_t ph = b ? es.phase1 : es.phase0;
          if (!mbar_wait_warp<true>(bar, ph, status, kDevTimeoutTmaFull, abort_flag)) return;
          if (b) es.phase1 ^= 1u; else es.phase0 ^= 1u;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int col = n0 + 8 * j;
          // k008 recipe order: acc * (s_a * s_w) + bias, each step rounded.
          float ss[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
          float bs[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
          if (col < p.N) {
            const float4* sp = reinterpret_cast<const float4*>(p.scale_b + col);
            const float4* bp = reinterpret_cast<const float4*>(static_cast<const float*>(p.bias) + col);
            const float4 s0 = __ldg(sp), s1 = __ldg(sp + 1), b0 = __ldg(bp), b1 = __ldg(bp + 1);
            ss[0] = s0.x; ss[1] = s0.y; ss[2] = s0.z; ss[3] = s0.w;
            ss[4] = s1.x; ss[5] = s1.y; ss[6] = s1.z; ss[7] = s1.w;
            bs[0] = b0.x; bs[1] = b0.y; bs[2] = b0.z; bs[3] = b0.w;
            bs[4] = b1.x; bs[5] = b1.y; bs[6] = b1.z; bs[7] = b1.w;
          }
          float v[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float acc_f = static_cast<float>(static_cast<int32_t>(r[8 * j + i]));
            v[i] = __fadd_rn(__fmul_rn(acc_f, __fmul_rn(row_scale, ss[i])), bs[i]);
          }
          uint4* slot = reinterpret_cast<uint4*>(buf + swz(lane, j));
          if constexpr (kResidual) {
            float res[8];
            unpack8<TOut>(*slot, res);
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = row_keep ? res[i] + v[i] : res[i];
          } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = row_keep ? v[i] : 0.f;
          }
          *slot = pack8<TOut>(v);
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        tma_store_2d(tm_out, buf, n0, row0);  // rows >= M / cols >= N are clipped
        bulk_commit_group();
      }
    }
    if constexpr (kResidual && kEpiBufs == 1) {
      // Request the next tile's first residual box into the (only) buffer once
      // the last store has read it.
      const int nn0 = next_n0;
      if (next_row0 >= 0 && next_row0 < p.M && nn0 < p.N) {
        rel.arrive();
        if (lane == 0) {
          bulk_wait_group_read<0>();
          mbar_arrive_expect_tx(es.bar0, kEpiBoxBytes);
          tma_load_2d(es.buf0, tm_res, es.bar0, nn0, next_row0);
        }
        es.pending = 1;
        __syncwarp();
      }
    }
  }
}

template <typename TIn>
constexpr CUtensorMapDataType tmap_dtype() {
  return std::is_same<TIn, int8_t>::value    ? CU_TENSOR_MAP_DATA_TYPE_UINT8
         : std::is_same<TIn, float>::value  ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
         : std::is_same<TIn, __half>::value ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                            : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
}

template <typename TOut>
__device__ __forceinline__ void init_epi_state(EpiState& es, uint8_t* epi_base, uint64_t* res_bars, int ew) {
  es.buf0 = epi_base + (kEpiBufs * ew) * kEpiBoxBytes;
  es.buf1 = es.buf0 + (kEpiBufs - 1) * kEpiBoxBytes;
  es.bar0 = res_bars + 2 * ew;
  es.bar1 = es.bar0 + (kEpiBufs - 1);
  es.phase0 = es.phase1 = 0u;
  es.next = 0;
  es.pending = 0;
}

// ---------------------------------------------------------------------------
// Single-CTA kernel: one 128 x BN tile per CTA.
template <typename TIn, typename TOut, int BN, int STAGES, int EPI>
__global__ void __launch_bounds__(kGemmThreads, 1)
gemm_tn_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
               const __grid_constant__ CUtensorMap tmOut, const __grid_constant__ CUtensorMap tmRes,
               const GemmParams p) {
  constexpr int kABytes = kBM * kRowBytes;
  constexpr int kBBytes = BN * kRowBytes;
  using L = GemmLayout<kABytes + kBBytes, STAGES>;
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
  uint8_t* sB = smem + STAGES * kABytes;
  uint8_t* epi_base = smem + L::kEpiOff;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint64_t* res_bars = drain + 1;  // [2 * kEpiWarps]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(res_bars + 2 * kEpiWarps);
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
      mbar_init(&acc_empty[a], kEpiWarps);
    }
    mbar_init(drain, 1);
    for (int i = 0; i < 2 * kEpiWarps; ++i) mbar_init(&res_bars[i], 1);
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
  grid_dependency_wait();  // the previous kernel's writes are visible from here
  grid_launch_dependents();

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
          if (!mbar_wait<true>(&empty[stage], phase ^ 1u, p.status, kDevTimeoutSmemEmpty, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], kABytes + kBBytes);
          if (p.a_kchunk > 0)
            tma_load_3d(sA + stage * kABytes, &tmA, &full[stage], (kb * kBK) % p.a_kchunk, m_blk * kBM,
                        (kb * kBK) / p.a_kchunk);
          else
            tma_load_2d(sA + stage * kABytes, &tmA, &full[stage], kb * kBK, m_blk * kBM);
          tma_load_2d(sB + stage * kBBytes, &tmB, &full[stage], kb * kBK, n_blk * BN);
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
        if (!mbar_wait<true>(&acc_empty[acc], acc_phase ^ 1u, p.status, kDevTimeoutAccEmpty, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait<true>(&full[stage], phase, p.status, kDevTimeoutTmaFull, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * kABytes);
          const uint32_t b_addr = smem_u32(sB + stage * kBBytes);
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
    const int lane_grp = warp & 3;            // TMEM lane quarter this warp may access
    const int col_half = (warp - 2) >> 2;     // which half of the tile's columns
    EpiState es;
    init_epi_state<TOut>(es, epi_base, res_bars, warp - 2);
    int local = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait_warp<true>(&acc_full[acc], acc_phase, p.status, kDevTimeoutAccFull, abort_flag)) break;
      tc_fence_after();
      const int m_blk = tile / p.num_n_blocks;
      const int n_blk = tile - m_blk * p.num_n_blocks;
      const int nt = tile + (int)gridDim.x;
      const int nm = nt / p.num_n_blocks;
      AccRelease rel{&acc_empty[acc], 0u, false};
      epilogue_tile<TOut, BN, EPI>(p, &tmOut, &tmRes,
                                   tmem_base + (static_cast<uint32_t>(lane_grp * 32) << 16) + acc * BN,
                                   m_blk * kBM + lane_grp * 32, n_blk, col_half, es, rel, p.status, abort_flag,
                                   nt < num_tiles ? nm * kBM + lane_grp * 32 : -1,
                                   (nt - nm * p.num_n_blocks) * BN + col_half * (BN / 2));
      rel.arrive();
    }
    // A next-tile residual box still in flight (only after an abort) lands before exit.
    if (es.pending) mbar_wait_warp<true>(es.bar0, es.phase0, p.status, kDevTimeoutTmaFull, nullptr);
    if (lane == 0) bulk_wait_group_all();
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem_base, kTmemCols);
}

// ---------------------------------------------------------------------------
// CTA-pair kernel (cluster of 2, tcgen05 cta_group::2): one 256 x BN output
// tile per pair.  Each CTA loads its own 128 rows of A and its half (BN/2 rows)
// of B, so per SM the operand traffic per FLOP is 2/3 of the single-CTA
// 128 x BN tile.  The leader CTA (rank 0) issues every MMA; D rows 0..127 land
// in the leader's TMEM, rows 128..255 in the peer's.  Both CTAs' TMA loads count
// their bytes on the leader's full barrier; the leader commits stage-free and
// accumulator-full events to both CTAs' barriers (two plain commits, no
// multicast); both CTAs' epilogue warps release an accumulator by arriving on
// the leader's barrier.
template <typename TIn, typename TOut, int BN, int STAGES, int EPI>
__global__ void __launch_bounds__(kGemmThreads, 1) __cluster_dims__(2, 1, 1)
gemm_tn_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const __grid_constant__ CUtensorMap tmOut, const __grid_constant__ CUtensorMap tmRes,
                    const __grid_constant__ CUtensorMap tmBh, const GemmParams p) {
  constexpr int kABytes = kBM * kRowBytes;         // this CTA's 128 rows of A
  constexpr int kBBytes = (BN / 2) * kRowBytes;    // this CTA's half of B
  constexpr int kStageBytes = kABytes + kBBytes;
  using L = GemmLayout<kStageBytes, STAGES>;
  constexpr bool kInt8 = std::is_same<TIn, int8_t>::value;
  constexpr int kBK = kRowBytes / sizeof(TIn);
  constexpr uint32_t kTmemCols = 2 * BN;
  constexpr uint32_t kIdesc =
      kInt8 ? idesc_i8(2 * kBM, BN)
            : idesc_f16(2 * kBM, BN, std::is_same<TIn, __nv_bfloat16>::value ? 1 : 0, 0);
  static_assert(kTmemCols == 256 || kTmemCols == 512, "TMEM columns must be a power of 2");
  // Half units (256 x 128, a tail tile's column half): tmBh boxes are BN/4 rows per CTA.
  constexpr bool kHalves = BN == 256;
  constexpr uint32_t kIdescHalf =
      kInt8 ? idesc_i8(2 * kBM, BN / 2)
            : idesc_f16(2 * kBM, BN / 2, std::is_same<TIn, __nv_bfloat16>::value ? 1 : 0, 0);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * kABytes;
  uint8_t* epi_base = smem + L::kEpiOff;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint64_t* res_bars = drain + 1;  // [2 * kEpiWarps]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(res_bars + 2 * kEpiWarps);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);    // the leader's copy counts both CTAs' bytes
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 2 * kEpiWarps);  // leader's copy: every epilogue warp of both CTAs
    }
    mbar_init(drain, 1);
    for (int i = 0; i < 2 * kEpiWarps; ++i) mbar_init(&res_bars[i], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    __syncwarp();
    tmem_alloc_pair(tmem_slot, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialised before any remote arrival
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  grid_dependency_wait();  // the previous kernel's writes are visible from here
  grid_launch_dependents();

  const int num_kb = (p.K + kBK - 1) / kBK;
  const int pair_id = blockIdx.x >> 1;
  const int num_pairs = gridDim.x >> 1;
  // Work unit u -> tile (m blocks of 256 rows, n blocks of BN columns) and
  // column half (-1: the whole tile).
  auto unit = [&](int u, int& m_blk, int& n_blk, int& half) {
    int tile = u;
    half = -1;
    if (kHalves && u >= p.full_tiles) {
      const int h = u - p.full_tiles;
      tile = p.full_tiles + (h >> 1);
      half = h & 1;
    }
    m_blk = tile / p.num_n_blocks;
    n_blk = tile - m_blk * p.num_n_blocks;
  };

  if (warp == 0) {
    // ------------------------------------------------------------ producer (both CTAs)
    if (lane == 0) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int u = pair_id; ok && u < p.num_units; u += num_pairs) {
        int m_blk, n_blk, half;
        unit(u, m_blk, n_blk, half);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait<true>(&empty[stage], phase ^ 1u, p.status, kDevTimeoutSmemEmpty, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t leader_full = mapa_shared(smem_u32(&full[stage]), 0);
          if (leader) mbar_arrive_expect_tx(&full[stage], half < 0 ? 2 * kStageBytes : 2 * (kABytes + kBBytes / 2));
          if (p.a_kchunk > 0)
            tma_load_3d_pair(sA + stage * kABytes, &tmA, leader_full, (kb * kBK) % p.a_kchunk,
                             m_blk * 2 * kBM + (int)rank * kBM, (kb * kBK) / p.a_kchunk);
          else
            tma_load_2d_pair(sA + stage * kABytes, &tmA, leader_full, kb * kBK,
                             m_blk * 2 * kBM + (int)rank * kBM);
          if (half < 0)
            tma_load_2d_pair(sB + stage * kBBytes, &tmB, leader_full, kb * kBK,
                             n_blk * BN + (int)rank * (BN / 2));
          else
            tma_load_2d_pair(sB + stage * kBBytes, &tmBh, leader_full, kb * kBK,
                             n_blk * BN + half * (BN / 2) + (int)rank * (BN / 4));
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader only)
    if (leader && lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int u = pair_id; ok && u < p.num_units; u += num_pairs, ++local) {
        const uint32_t idesc = (kHalves && u >= p.full_tiles) ? kIdescHalf : kIdesc;
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait<true>(&acc_empty[acc], acc_phase ^ 1u, p.status, kDevTimeoutAccEmpty, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait<true>(&full[stage], phase, p.status, kDevTimeoutTmaFull, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * kABytes);
          const uint32_t b_addr = smem_u32(sB + stage * kBBytes);
#pragma unroll
          for (int kk = 0; kk < kRowBytes / 32; ++kk) {
            const uint64_t ad = smem_desc_sw128(a_addr + kk * 32, 16, 1024);
            const uint64_t bd = smem_desc_sw128(b_addr + kk * 32, 16, 1024);
            const uint32_t accum = (kb | kk) != 0 ? 1u : 0u;
            if constexpr (kInt8)
              umma_i8_ss_pair(d_tmem, ad, bd, idesc, accum);
            else
              umma_f16_ss_pair(d_tmem, ad, bd, idesc, accum);
          }
          const uint32_t e = smem_u32(&empty[stage]);
          umma_commit_pair(mapa_shared(e, 0));  // stage free in both CTAs once read
          umma_commit_pair(mapa_shared(e, 1));
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        const uint32_t f = smem_u32(&acc_full[acc]);
        umma_commit_pair(mapa_shared(f, 0));
        umma_commit_pair(mapa_shared(f, 1));
      }
      umma_commit_pair(mapa_shared(smem_u32(drain), 0));
      mbar_wait(drain, 0, p.status, kDevTimeoutAccFull, nullptr);
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int lane_grp = warp & 3;
    const int col_half = (warp - 2) >> 2;
    EpiState es;
    init_epi_state<TOut>(es, epi_base, res_bars, warp - 2);
    int local = 0;
    for (int u = pair_id; u < p.num_units; u += num_pairs, ++local) {
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait_warp<true>(&acc_full[acc], acc_phase, p.status, kDevTimeoutAccFull, abort_flag)) break;
      tc_fence_after();
      int m_blk, n_blk, half;
      unit(u, m_blk, n_blk, half);
      // this warp's first row and column in the next unit (for its early residual request)
      int next_row0 = -1, next_n0 = 0;
      if (u + num_pairs < p.num_units) {
        int nm, nn, nh;
        unit(u + num_pairs, nm, nn, nh);
        next_row0 = nm * 2 * kBM + (int)rank * kBM + lane_grp * 32;
        next_n0 = nh < 0 ? nn * BN + col_half * (BN / 2) : nn * BN + nh * (BN / 2) + col_half * (BN / 4);
      }
      AccRelease rel{nullptr, mapa_shared(smem_u32(&acc_empty[acc]), 0), false};
      const uint32_t t_acc = tmem_base + (static_cast<uint32_t>(lane_grp * 32) << 16) + acc * BN;
      const int row0 = m_blk * 2 * kBM + (int)rank * kBM + lane_grp * 32;
      if (half < 0) {
        epilogue_tile<TOut, BN, EPI>(p, &tmOut, &tmRes, t_acc, row0, n_blk, col_half, es, rel, p.status,
                                     abort_flag, next_row0, next_n0);
      } else if constexpr (kHalves) {
        // columns [n_blk * BN + half * BN/2, + BN/2): 128-column block 2 * n_blk + half
        epilogue_tile<TOut, BN / 2, EPI>(p, &tmOut, &tmRes, t_acc, row0, 2 * n_blk + half, col_half, es, rel,
                                         p.status, abort_flag, next_row0, next_n0);
      }
      rel.arrive();
    }
    // A next-tile residual box still in flight (only after an abort) lands before exit.
    if (es.pending) mbar_wait_warp<true>(es.bar0, es.phase0, p.status, kDevTimeoutTmaFull, nullptr);
    if (lane == 0) bulk_wait_group_all();
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // the leader's MMAs into the peer's TMEM / smem are complete
  tc_fence_after();
  if (warp == 0) tmem_dealloc_pair(tmem_base, kTmemCols);
}

// ---------------------------------------------------------------------------
// Host side.
template <typename TIn, typename TOut, int EPI>
int make_maps(const GemmArgs& g, int box_a_rows, int box_b_rows, CUtensorMap* ta, CUtensorMap* tb,
              CUtensorMap* tout, CUtensorMap* tres) {
  constexpr int kBK = kRowBytes / sizeof(TIn);
  const CUtensorMapDataType dt = tmap_dtype<TIn>();
  if (g.a_kchunk > 0) {
    // A(m, k) = a[k / kc][m][k % kc]: a 3-D map, one K-chunk per z.
    const uint64_t kc = (uint64_t)g.a_kchunk;
    const uint64_t dims[3] = {kc, (uint64_t)g.m, (uint64_t)g.k / kc};
    const uint64_t strides[2] = {kc * sizeof(TIn), kc * (uint64_t)g.m * sizeof(TIn)};
    const uint32_t box[3] = {(uint32_t)kBK, (uint32_t)box_a_rows, 1};
    if (int rc = encode_tmap(ta, dt, 3, g.a, dims, strides, box)) return rc;
  } else {
    const uint64_t dims[2] = {(uint64_t)g.k, (uint64_t)g.m};
    const uint64_t strides[1] = {(uint64_t)g.k * sizeof(TIn)};
    const uint32_t box[2] = {(uint32_t)kBK, (uint32_t)box_a_rows};
    if (int rc = encode_tmap(ta, dt, 2, g.a, dims, strides, box)) return rc;
  }
  {
    const uint64_t dims[2] = {(uint64_t)g.k, (uint64_t)g.n};
    const uint64_t strides[1] = {(uint64_t)g.k * sizeof(TIn)};
    const uint32_t box[2] = {(uint32_t)kBK, (uint32_t)box_b_rows};
    if (int rc = encode_tmap(tb, dt, 2, g.b, dims, strides, box)) return rc;
  }
  if constexpr (EPI == (int)Epi::kRawS32) {
    *tout = *ta;  // unused by the raw epilogue
    *tres = *ta;
  } else {
    const CUtensorMapDataType odt = tmap_dtype<TOut>();
    const uint64_t dims[2] = {(uint64_t)g.n, (uint64_t)g.m};
    const uint64_t strides[1] = {(uint64_t)g.n * sizeof(TOut)};
    // one 128-byte row per box row: 64 16-bit or 32 fp32 columns
    const uint32_t box[2] = {(uint32_t)(128 / sizeof(TOut)), (uint32_t)kEpiBoxRows};
    if (int rc = encode_tmap(tout, odt, 2, g.out, dims, strides, box)) return rc;
    if (g.residual != nullptr) {
      if (int rc = encode_tmap(tres, odt, 2, g.residual, dims, strides, box)) return rc;
    } else {
      *tres = *tout;  // unused
    }
  }
  return TTJ_OK;
}

GemmParams make_params(const GemmArgs& g, int tile_m, int bn) {
  GemmParams p;
  p.M = (int)g.m;
  p.N = (int)g.n;
  p.K = (int)g.k;
  p.a_kchunk = (int)g.a_kchunk;
  p.num_m_blocks = (int)((g.m + tile_m - 1) / tile_m);
  p.num_n_blocks = (int)((g.n + bn - 1) / bn);
  p.full_tiles = p.num_m_blocks * p.num_n_blocks;
  p.num_units = p.full_tiles;
  p.bias = g.bias;
  p.row_mask = g.row_mask;
  p.scale_a = g.scale_a;
  p.scale_b = g.scale_b;
  p.out = g.out;
  p.status = g.status;
  return p;
}

template <typename TIn, typename TOut, int BN, int STAGES, int EPI>
int launch_one(const GemmArgs& g, cudaStream_t stream) {
  using L = GemmLayout<kBM * kRowBytes + BN * kRowBytes, STAGES>;
  CUtensorMap ta, tb, tout, tres;
  if (int rc = make_maps<TIn, TOut, EPI>(g, kBM, BN, &ta, &tb, &tout, &tres)) return rc;
  const GemmParams p = make_params(g, kBM, BN);
  const int tiles = p.num_m_blocks * p.num_n_blocks;
  const int grid = tiles < sm_count() ? tiles : sm_count();
  auto kern = gemm_tn_kernel<TIn, TOut, BN, STAGES, EPI>;
  TTJ_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kTotal));
  TTJ_CUDA_TRY(launch_pdl(kern, dim3(grid), dim3(kGemmThreads), L::kTotal, stream, ta, tb, tout, tres, p));
  return TTJ_OK;
}

template <typename TIn, typename TOut, int BN, int STAGES, int EPI>
int launch_pair(const GemmArgs& g, cudaStream_t stream) {
  using L = GemmLayout<kBM * kRowBytes + (BN / 2) * kRowBytes, STAGES>;
  CUtensorMap ta, tb, tout, tres, tbh;
  if (int rc = make_maps<TIn, TOut, EPI>(g, kBM, BN / 2, &ta, &tb, &tout, &tres)) return rc;
  GemmParams p = make_params(g, 2 * kBM, BN);
  const int tiles = p.num_m_blocks * p.num_n_blocks;
  const int max_pairs = sm_count() / 2;
  const int pairs = tiles < max_pairs ? tiles : max_pairs;
  const int grid = 2 * pairs;
  tbh = tb;
  if constexpr (BN == 256) {
    // A last partial wave of `rem` tiles runs as 2 * rem column halves when they
    // fit in one wave: every pair then ends within half a tile of the others.
    // Measured (cfg2 out-proj, 256 tiles on 74 pairs: 222 tiles + 68 halves):
    // 36.9 -> 34.8 us between the layer's kernels, 40.9 -> 38.9 us alone, same
    // output bits; the layer step is unchanged (230.4 -> 230.9 us).
    const int rem = tiles % pairs;
    if (rem > 0 && 2 * rem <= pairs) {
      p.full_tiles = tiles - rem;
      p.num_units = p.full_tiles + 2 * rem;
      constexpr int kBK = kRowBytes / sizeof(TIn);
      const uint64_t dims[2] = {(uint64_t)g.k, (uint64_t)g.n};
      const uint64_t strides[1] = {(uint64_t)g.k * sizeof(TIn)};
      const uint32_t box[2] = {(uint32_t)kBK, (uint32_t)(BN / 4)};
      if (int rc = encode_tmap(&tbh, tmap_dtype<TIn>(), 2, g.b, dims, strides, box)) return rc;
    }
  }
  auto kern = gemm_tn_pair_kernel<TIn, TOut, BN, STAGES, EPI>;
  TTJ_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kTotal));
  TTJ_CUDA_TRY(launch_pdl(kern, dim3(grid), dim3(kGemmThreads), L::kTotal, stream, ta, tb, tout, tres, tbh, p));
  return TTJ_OK;
}

template <typename TIn, typename TOut, int EPI>
int dispatch_bn(const GemmArgs& g, cudaStream_t stream) {
  // More than one 128-row block: CTA pairs with 256 x 256 (or 256 x 128) tiles.
  // Otherwise one CTA per 128 x BN tile.  BN = 256 halves the A re-reads; 128
  // when N is small or would leave a half-empty tile column.
  // 256 x 256 pairs keep 6 stages (192 KB) in flight: the layer's projections
  // stream their operands from L2 and measured faster with every added stage.
  const bool wide = g.n % 256 == 0 && g.n >= 512;
  if (g.m > kBM) {
    if (wide) return launch_pair<TIn, TOut, 256, 6, EPI>(g, stream);
    return launch_pair<TIn, TOut, 128, 7, EPI>(g, stream);
  }
  if (wide) return launch_one<TIn, TOut, 256, 4, EPI>(g, stream);
  return launch_one<TIn, TOut, 128, 6, EPI>(g, stream);
}

template <typename TIn, typename TOut>
int dispatch_epi(const GemmArgs& g, cudaStream_t stream) {
  switch (g.epi) {
    case Epi::kBias: return dispatch_bn<TIn, TOut, (int)Epi::kBias>(g, stream);
    case Epi::kBiasResidual: return dispatch_bn<TIn, TOut, (int)Epi::kBiasResidual>(g, stream);
    case Epi::kBiasGelu: return dispatch_bn<TIn, TOut, (int)Epi::kBiasGelu>(g, stream);
    case Epi::kBiasResidualZeroRows:
      return dispatch_bn<TIn, TOut, (int)Epi::kBiasResidualZeroRows>(g, stream);
    default: return fail(TTJ_ERR_INVALID_ARG, "epilogue not valid for 16-bit operands");
  }
}

// 16-bit operands, fp32 output (bias and residual fp32): the fp32 residual stream.
template <typename TIn>
int dispatch_epi_f32(const GemmArgs& g, cudaStream_t stream) {
  switch (g.epi) {
    case Epi::kBias: return dispatch_bn<TIn, float, (int)Epi::kBias>(g, stream);
    case Epi::kBiasResidual: return dispatch_bn<TIn, float, (int)Epi::kBiasResidual>(g, stream);
    case Epi::kBiasResidualZeroRows: return dispatch_bn<TIn, float, (int)Epi::kBiasResidualZeroRows>(g, stream);
    default: return fail(TTJ_ERR_INVALID_ARG, "epilogue not valid for fp32 output");
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
  if (g.out_dtype == TTJ_F32 && g.in_dtype == TTJ_F16) return dispatch_epi_f32<__half>(g, stream);
  if (g.out_dtype == TTJ_F32 && g.in_dtype == TTJ_BF16) return dispatch_epi_f32<__nv_bfloat16>(g, stream);
  if (g.in_dtype == TTJ_F16) return dispatch_epi<__half, __half>(g, stream);
  if (g.in_dtype == TTJ_BF16) return dispatch_epi<__nv_bfloat16, __nv_bfloat16>(g, stream);
  // int8 operands
  if (g.epi == Epi::kRawS32) return dispatch_bn<int8_t, int32_t, (int)Epi::kRawS32>(g, stream);
  if (g.out_dtype == TTJ_F16) return dispatch_int8<__half>(g, stream);
  return dispatch_int8<__nv_bfloat16>(g, stream);
}

}  // namespace ttj
