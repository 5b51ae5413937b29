// Flash-attention forward for sm_100a (persistent, two query tiles per work item).
//
// Q, K and V are read straight from the packed projection buffer qkv[B,S,3D]
// through one 4-D TMA descriptor (dims head_dim x 3H x S x B, box 64 x 1 x 128
// x 1, 128-byte swizzle): the reference's head split (.view/.transpose/
// .contiguous) becomes a coordinate choice, rows past S arrive as zeros, and so
// do the columns past head_dim.  The kernel is compiled for padded head sizes
// HD = 64, 128 and 256 and runs any head_dim that is a multiple of 8 up to HD:
// the zero columns add nothing to Q K^T and give zero columns of P V, which the
// context store (a 4-D map of the same shape) clips away.
//
// Work item = (batch, head, 256 consecutive queries) = two 128-row query tiles
// A and B that share every K/V tile (HD 256: one 128-row tile, tensor memory
// holds one S and one 256-column O per tile).  One CTA per SM loops over work
// items, heaviest (longest causal key range) first.
//
// Roles (head_dim 128 / 256: 384 threads = 3 warpgroups; head_dim 64: 640 = 5):
//   warp 0       TMA: K_j / V_j tiles into KV_STAGES-deep rings, item after item
//   warps 1, 3   MMA issue, one thread: S_t = Q_t K_j^T into TMEM, O_t += P_t V_j
//                with P read from TMEM (tcgen05 "ts" form); head_dim 64: warp 1
//                for tile A, warp 3 for tile B; head_dim 128: warp 1 for both
//   warp 2       TMA: the two Q tiles of each work item
//   softmax      head_dim 128 / 256: warps 4..7 for tile A, 8..11 for tile B,
//                thread = query row; head_dim 64: warps 4..11 for tile A,
//                12..19 for tile B, two warps per TMEM lane quarter, each with
//                16 rows (softmax_split below).  Load S from TMEM, mask, online
//                softmax in fp32 with a lazily moved row max, write P (input
//                dtype) to TMEM, rescale O when the max moved, and at the end
//                normalise O and store the context rows at the head's columns
//                of ctx[B,S,D] (head merge).
//
// Two schedules, chosen by what fits in the 512 TMEM columns:
//
// head_dim 64 ("separate P"): S_A [0,128) S_B [128,256) P_A [256,320)
//   P_B [320,384) O_A [384,448) O_B [448,512).  S_t(j+1) = Q_t K_{j+1}^T is
//   issued as soon as the softmax has read S_t(j) out of TMEM, so it is ready
//   when the softmax finishes tile j.  P_t(j) is computed into registers and
//   stored to its own buffer only then, after P_t(j-1) V_{j-1} has completed
//   (o_done): that product was issued a whole softmax step earlier, so in
//   steady state the softmax waits for neither S nor O (measured: with P
//   written over S the softmax idled ~40% of each step on the P.V -> Q.K round
//   trip; waiting for o_done before the exponentials cost ~15%).
// head_dim 128 ("P over S"): S_A [0,128) S_B [128,256) O_A [256,384)
//   O_B [384,512); P_t overwrites the first 64 columns of S_t, so the issue
//   order per tile is PV_t(j-1), QK_t(j), commit s_full_t.  tcgen05.commit
//   arrives only when every earlier MMA of the issuing thread has completed,
//   so "S_t(j) is ready" also means P_t(j-1) was consumed and O_t is stable.
// head_dim 256: the same schedule for tile A alone, S_A [0,128) O_A [256,512),
//   one K and one V stage (64 KB each).
#include "sm100_ptx.cuh"
#include "ttj_internal.h"

namespace ttj {
namespace {

constexpr int kBM = 128;     // queries per tile
constexpr int kBN = 128;     // keys per KV tile
constexpr int kChunkBytes = 128 * 128;  // one [128 rows][64 cols] 16-bit swizzled box
constexpr uint32_t kTmemCols = 512;
constexpr int64_t kHeadMajorKvBytes = int64_t(96) << 20;

struct AttnParams {
  void* ctx;
  const uint8_t* key_mask;
  int B, S, H;
  int hd;            // real head_dim (<= the kernel's padded HD)
  int num_pairs;     // ceil(S / (128 * tiles per item))
  int num_items;     // B * H * num_pairs
  int head_major;    // item order: 1 = a head's pairs consecutive, 0 = pair index outermost
  float scale_log2;  // head_dim^-0.5 * log2(e)
  int* status;
};

template <int HD>
struct AttnSmem {
  static_assert(HD == 64 || HD == 128 || HD == 256, "padded head sizes");
  static constexpr int kNT = HD == 256 ? 1 : 2;     // query tiles per work item
  static constexpr bool kSepP = HD == 64;           // separate P buffers in TMEM
  // head_dim 64: two softmax warps per tile on each SM sub-partition, each
  // owning 16 of the quarter's 32 rows (16-lane TMEM shapes), so two
  // exponential streams of a tile run at once on each sub-partition.  (The
  // same split of the head_dim-128 schedule, P over S, measured 5-22% slower:
  // B2 S4096 H32 causal 289 -> 351 us, non-causal 466 -> 493 us.)
  static constexpr bool kSplit = HD == 64;
  static constexpr int kThreads = kSplit ? 640 : 384;
  // Register split (setmaxnreg): the block launches with kLaunchRegs per
  // thread; the first warpgroup (producers, MMA issuers) gives registers back
  // to the softmax warpgroups.
  static constexpr int kLaunchRegs = kSplit ? 96 : 168;
  // (136 / 184: the smallest control share whose producer and MMA-issuer code
  // compiles without spills at head_dim 128 and 256.)
  static constexpr uint32_t kRegsCtl = kSplit ? 64 : 136;
  static constexpr uint32_t kRegsSoftmax = kSplit ? 104 : 184;
  static_assert(128 * kRegsCtl + (kThreads - 128) * kRegsSoftmax == kThreads * kLaunchRegs,
                "register split must use the launch budget");
  static constexpr int kEpiRows = kSplit ? 16 : 32;  // rows of a softmax warp's context box
  static constexpr int kStages = HD == 64 ? 4 : (HD == 128 ? 2 : 1);
  static constexpr int kTileBytes = HD * 2 * 128;  // 128 rows x HD x 2 bytes
  // Q tiles: head_dim 64 double-buffers them (the next item's Q arrives while
  // this item runs); the larger heads have no room.
  static constexpr int kQBufs = HD == 64 ? 2 : 1;
  static constexpr int kQOff = 0;                   // [kQBufs][Q_A, Q_B]
  static constexpr int kKOff = kNT * kQBufs * kTileBytes;
  static constexpr int kVOff = kKOff + kStages * kTileBytes;
  // The context rows leave through TMA stores from a 4 KB staging box per
  // softmax warp (32 rows x 64 columns, 128-byte swizzle; larger heads reuse
  // it for each further 64 columns); measured: per-thread 16-byte row stores
  // took 1-2.5K cycles per item end at head_dim 64, ~3.5K at head_dim 128.
  static constexpr int kEpiOff = kVOff + kStages * kTileBytes;
  static constexpr int kBarOff = kEpiOff + (kThreads / 32 - 4) * kEpiRows * 128;
  static constexpr int kTotal = 1024 + kBarOff + 512;
  static_assert(kTotal <= 232448, "shared memory budget");
  // TMEM columns
  static constexpr uint32_t kColP = kSepP ? 256 : 0;      // + t*64 (separate) / + t*128 (over S)
  static constexpr uint32_t kColO = kSepP ? 384 : 256;    // + t*HD
};

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// sm_100 packed fp32 pairs (two lanes per instruction) and 3-input max.
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// The k-th work item of this CTA: item indices are dealt out in rounds of
// gridDim.x, alternating direction each round ("snake" order).  With items
// sorted heaviest first this keeps the per-CTA totals within ~3% of the mean
// for causal attention (plain striding: ~11% for benchmark configuration 2).
__device__ __forceinline__ int item_of(int k) {
  return k * (int)gridDim.x + ((k & 1) ? (int)gridDim.x - 1 - (int)blockIdx.x : (int)blockIdx.x);
}

// Decode work item -> (b, h, pair); a "pair" is the item's group of query tiles.  Causal pairs come in decreasing pair
// index (longest key range first).  Pair-major order (the pair index
// outermost) keeps the whole grid on items of equal length, which balances
// short sequences best.  Head-major order (a head's pairs consecutive) is used
// when every head's K and V together exceed what L2 can hold: the CTAs then
// running work on a few heads and read their K/V tiles from L2 instead of
// each streaming its own head's from DRAM.
struct Item {
  int b, h, pair;
};
template <bool CAUSAL>
__device__ __forceinline__ Item decode_item(int item, const AttnParams& p) {
  int bh, r;
  if (p.head_major) {
    bh = item / p.num_pairs;
    r = item - bh * p.num_pairs;
  } else {
    const int bh_count = p.B * p.H;
    r = item / bh_count;
    bh = item - r * bh_count;
  }
  Item it;
  it.pair = CAUSAL ? p.num_pairs - 1 - r : r;
  it.b = bh / p.H;
  it.h = bh - it.b * p.H;
  return it;
}

// Number of key tiles tile `t` (0 = A, 1 = B) of a pair attends to (NT tiles per pair).
template <bool CAUSAL, int NT>
__device__ __forceinline__ int kv_tiles(int pair, int t, int S) {
  const int total = (S + kBN - 1) / kBN;
  return CAUSAL ? min(NT * pair + 1 + t, total) : total;
}

// Softmax warps, two per query tile on each SM sub-partition (the head_dim-64
// kernel: separate P buffers, two query tiles per item; the P-over-S layout of
// head_dim 128 is handled too, but measured slower there): warp w (4..19)
// serves tile t = (w - 4) / 8 and rows 16 * sub .. 16 * sub + 15 (sub =
// ((w - 4) / 4) & 1) of TMEM lane quarter w % 4, through the 16-lane TMEM
// shapes.  Thread lane = 4g + k holds rows g and g + 8 of the warp's 16 and,
// of each 8-key group n of the key tile, keys 8n + 2k and 8n + 2k + 1; the
// four threads of a row combine its max and sum with two shuffles.  Per key
// tile: wait for S, load it, release it (the next S may be computed), mask,
// row max, P = 2^(s*scale - m) into registers, wait for the previous P.V,
// store P (P word 4n + k of a row = keys 8n + 2k, 8n + 2k + 1), rescale O when
// the exponent reference moved, signal.  At an item's end: O / l into a
// 16-row staging box, one TMA store per warp.
// Four softmax warps share each sub-partition and run their exponential loops
// whenever their data is ready.  Measured against one softmax warp per tile
// and sub-partition (with the two tiles' warps taking turns on the exponential
// unit): cfg2 shapes non-causal 206.9 -> 194.6 us, B4 S8192 causal 885 -> 797
// us, B2 S25000 H8 causal 3.43 -> 2.94 ms, cfg2 causal unchanged (127 us);
// turns between the tiles' warp pairs measured 3-12% slower than none.
template <typename T, int HD, bool CAUSAL>
__device__ __forceinline__ void softmax_split(const AttnParams& p, uint8_t* epi_base, uint32_t tmem,
                                              const CUtensorMap* tm_ctx, uint64_t* s_full, uint64_t* s_free,
                                              uint64_t* p_full, uint64_t* o_done, volatile int* abort_flag) {
  using L = AttnSmem<HD>;
  constexpr int NT = L::kNT;
  constexpr bool kSepP = L::kSepP;  // head_dim 64: separate P buffers; 128: P over S
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int t = (warp - 4) >> 3;
  const int sub = ((warp - 4) >> 2) & 1;
  const int lg = warp & 3;
  const int g = lane >> 2, kq = lane & 3;
  const int ra = lg * 32 + sub * 16 + g;  // this thread's rows within the tile: ra, ra + 8
  const uint32_t t_lane = tmem + (static_cast<uint32_t>(lg * 32 + sub * 16) << 16);
  const uint32_t t_s = t_lane + t * 128;
  const uint32_t t_p = t_lane + L::kColP + t * (kSepP ? 64 : 128);
  const uint32_t t_o = t_lane + L::kColO + t * HD;
  // this warp's context staging box, as a shared-memory address
  const uint32_t box = smem_u32(epi_base) + (warp - 4) * (L::kEpiRows * 128);
  uint32_t sf_phase = 0, od_phase = 0;
  auto row_max4 = [](float v) {  // max over the four threads of a row
    v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 1));
    return fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 2));
  };
  auto row_sum4 = [](float v) {
    v += __shfl_xor_sync(0xffffffffu, v, 1);
    return v + __shfl_xor_sync(0xffffffffu, v, 2);
  };
  bool ok = true;
  for (int k = 0; ok; ++k) {
    const int item = item_of(k);
    if (item >= p.num_items) break;
    const Item it = decode_item<CAUSAL>(item, p);
    const int n_kv = kv_tiles<CAUSAL, NT>(it.pair, t, p.S);
    const int q0 = it.pair * NT * kBM + t * kBM;
    const int qa = q0 + ra, qb = qa + 8;
    const bool has_mask = p.key_mask != nullptr;
    const uint8_t* kmask = has_mask ? p.key_mask + (int64_t)it.b * p.S : nullptr;
    // bit gg: key gg * 32 + lane of the current key tile is valid (one register
    // for the lane's four keys; with fewer registers held across the loop the
    // causal kernel compiles without spills: cfg2 causal 129.0 -> 126.0 us,
    // non-causal 205.8 -> 199.7 us together with the 32-bit box address and
    // 1 / l taken before the last P.V wait, same output bits)
    uint32_t mbits = 0u;
    if (has_mask) {
#pragma unroll
      for (int gg = 0; gg < 4; ++gg) {
        const int key = gg * 32 + lane;
        mbits |= (key < p.S && __ldg(kmask + key) != 0) ? 1u << gg : 0u;
      }
    }
    float m_a = -INFINITY, m_b = -INFINITY;  // exponent references (log2 units), moved lazily
    float l_a = 0.f, l_b = 0.f;              // this thread's part of each row's sum of P
    for (int j = 0; j < n_kv; ++j) {
      if (!mbar_wait_warp(&s_full[t], sf_phase, p.status, kDevTimeoutSoftmax, abort_flag)) { ok = false; break; }
      sf_phase ^= 1u;
      tc_fence_after();
      float s[64];  // s[4n + e]: row (e < 2 ? a : b), key 8n + 2k + (e & 1)
      {
        uint32_t u[64];
        tmem_ld_16x256b_x16(t_s, u);
#pragma unroll
        for (int i = 0; i < 64; ++i) s[i] = __uint_as_float(u[i]);
      }
      if constexpr (kSepP) {
        tc_fence_before();
        mbar_arrive(&s_free[t]);  // the tensor core may overwrite S_t now
      }
      const int k0 = j * kBN;
      const bool tail = k0 + kBN > p.S;
      const bool diag = CAUSAL && k0 + kBN - 1 > q0;
      uint32_t vbits[4] = {~0u, ~0u, ~0u, ~0u};
      if (tail || has_mask) {
#pragma unroll
        for (int gg = 0; gg < 4; ++gg) {
          const int key = k0 + gg * 32 + lane;
          bool v = key < p.S;
          if (has_mask) v = v && ((mbits >> gg) & 1u);
          vbits[gg] = __ballot_sync(0xffffffffu, v);
        }
        if (has_mask && j + 1 < n_kv) {  // the next tile's bits
          mbits = 0u;
#pragma unroll
          for (int gg = 0; gg < 4; ++gg) {
            const int key = k0 + kBN + gg * 32 + lane;
            mbits |= (key < p.S && __ldg(kmask + key) != 0) ? 1u << gg : 0u;
          }
        }
      }
      if ((vbits[0] & vbits[1] & vbits[2] & vbits[3]) == ~0u) {
        if (diag) {
          // key k0 + 8n + 2k + (e & 1) is visible to row q iff 8n + (e & 1) <=
          // q - k0 - 2k: one compare with a constant per score (measured: cfg2
          // causal 131.1 -> 129.0 us against computing each key's index)
          const int da = qa - k0 - 2 * kq, db = qb - k0 - 2 * kq;
#pragma unroll
          for (int n = 0; n < 16; ++n) {
            s[4 * n + 0] = 8 * n <= da ? s[4 * n + 0] : -INFINITY;
            s[4 * n + 1] = 8 * n + 1 <= da ? s[4 * n + 1] : -INFINITY;
            s[4 * n + 2] = 8 * n <= db ? s[4 * n + 2] : -INFINITY;
            s[4 * n + 3] = 8 * n + 1 <= db ? s[4 * n + 3] : -INFINITY;
          }
        }
      } else {
#pragma unroll
        for (int n = 0; n < 16; ++n)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            // keys 8n .. 8n + 7 lie in word n / 4 of vbits
            const int key = 8 * n + 2 * kq + (e & 1);
            bool v = (vbits[n >> 2] >> (8 * (n & 3) + 2 * kq + (e & 1))) & 1u;
            if (CAUSAL) v = v && (k0 + key <= (e < 2 ? qa : qb));
            s[4 * n + e] = v ? s[4 * n + e] : -INFINITY;
          }
      }
      // row maxima: four independent chains per row, then the row's four threads
      float ma[4], mb[4];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        ma[c] = fmaxf(s[16 * c + 0], s[16 * c + 1]);
        mb[c] = fmaxf(s[16 * c + 2], s[16 * c + 3]);
#pragma unroll
        for (int n = 4 * c + 1; n < 4 * c + 4; ++n) {
          ma[c] = fmax3(ma[c], s[4 * n], s[4 * n + 1]);
          mb[c] = fmax3(mb[c], s[4 * n + 2], s[4 * n + 3]);
        }
      }
      const float mxa = row_max4(fmaxf(fmaxf(ma[0], ma[1]), fmaxf(ma[2], ma[3])));
      const float mxb = row_max4(fmaxf(fmaxf(mb[0], mb[1]), fmaxf(mb[2], mb[3])));
      // Lazy rescaling as in the other schedules: the reference only moves when
      // the tile max exceeds it by more than 8 (log2 units).
      const float mta = mxa * p.scale_log2, mtb = mxb * p.scale_log2;
      const float mna = (mta > m_a + 8.f) ? mta : m_a;
      const float mnb = (mtb > m_b + 8.f) ? mtb : m_b;
      const float mua = mna == -INFINITY ? 0.f : mna;
      const float mub = mnb == -INFINITY ? 0.f : mnb;
      const float alpha_a = fast_exp2(m_a - mua);
      const float alpha_b = fast_exp2(m_b - mub);
      const uint64_t c2 = f2_pack(p.scale_log2, p.scale_log2);
      const uint64_t nma = f2_pack(-mua, -mua), nmb = f2_pack(-mub, -mub);
      uint32_t pk[32];  // P words: pk[2n] row a, pk[2n + 1] row b, word column 4n + k
      uint64_t sa2[2] = {0ull, 0ull}, sb2[2] = {0ull, 0ull};
#pragma unroll
      for (int n = 0; n < 16; ++n) {
        float x0, x1;
        f2_unpack(ffma2(f2_pack(s[4 * n], s[4 * n + 1]), c2, nma), x0, x1);
        const float e0 = fast_exp2(x0), e1 = fast_exp2(x1);
        pk[2 * n] = Pack<T>::two(e0, e1);
        sa2[n & 1] = fadd2(sa2[n & 1], f2_pack(e0, e1));
        f2_unpack(ffma2(f2_pack(s[4 * n + 2], s[4 * n + 3]), c2, nmb), x0, x1);
        const float e2 = fast_exp2(x0), e3 = fast_exp2(x1);
        pk[2 * n + 1] = Pack<T>::two(e2, e3);
        sb2[n & 1] = fadd2(sb2[n & 1], f2_pack(e2, e3));
      }
      float a0, a1, b0, b1;
      f2_unpack(fadd2(sa2[0], sa2[1]), a0, a1);
      f2_unpack(fadd2(sb2[0], sb2[1]), b0, b1);
      l_a = l_a * alpha_a + (a0 + a1);
      l_b = l_b * alpha_b + (b0 + b1);
      m_a = mna;
      m_b = mnb;
      if (kSepP && j > 0) {
        // P_t(j-1) V must have completed: it reads the P buffer written here and
        // it is the last write to O_t before a rescale.  (With P over S, S_t(j)
        // being ready already means that P.V has completed.)
        if (!mbar_wait_warp(&o_done[t], od_phase, p.status, kDevTimeoutSoftmax, abort_flag)) { ok = false; break; }
        od_phase ^= 1u;
        tc_fence_after();
      }
      tmem_st_16x128b_x16(t_p, pk);  // P over S: only this warp's rows, already loaded
      if (j > 0 && __any_sync(0xffffffffu, alpha_a != 1.f || alpha_b != 1.f)) {
#pragma unroll 1
        for (int hh = 0; hh < HD / 64; ++hh) {
          uint32_t o[32];
          tmem_ld_16x256b_x8(t_o + 64 * hh, o);
#pragma unroll
          for (int n = 0; n < 8; ++n) {
            o[4 * n + 0] = __float_as_uint(__uint_as_float(o[4 * n + 0]) * alpha_a);
            o[4 * n + 1] = __float_as_uint(__uint_as_float(o[4 * n + 1]) * alpha_a);
            o[4 * n + 2] = __float_as_uint(__uint_as_float(o[4 * n + 2]) * alpha_b);
            o[4 * n + 3] = __float_as_uint(__uint_as_float(o[4 * n + 3]) * alpha_b);
          }
          tmem_st_16x256b_x8(t_o + 64 * hh, o);
        }
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&p_full[t]);
    }
    if (!ok) break;
    // epilogue: 1 / l, wait for the last P.V, then O_t / l -> this warp's 16 context rows
    const float inv_a = 1.f / row_sum4(l_a);
    const float inv_b = 1.f / row_sum4(l_b);
    if (!mbar_wait_warp(&o_done[t], od_phase, p.status, kDevTimeoutSoftmax, abort_flag)) break;
    od_phase ^= 1u;
    tc_fence_after();
#pragma unroll 1
    for (int hh = 0; hh < HD / 64; ++hh) {
      if (64 * hh >= p.hd) break;  // only zero padding left (uniform)
      if (lane == 0) bulk_wait_group_read<0>();  // the previous store has read the box
      __syncwarp();
      uint32_t o[32];  // o[4n + e]: row (e < 2 ? a : b), column 64hh + 8n + 2k + (e & 1)
      tmem_ld_16x256b_x8(t_o + 64 * hh, o);
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        // 128-byte rows, 16-byte chunk n holds columns 8n..8n+7, swizzled by row & 7
        const uint32_t wa = Pack<T>::two(__uint_as_float(o[4 * n]) * inv_a, __uint_as_float(o[4 * n + 1]) * inv_a);
        const uint32_t wb = Pack<T>::two(__uint_as_float(o[4 * n + 2]) * inv_b, __uint_as_float(o[4 * n + 3]) * inv_b);
        st_shared_u32(box + g * 128 + ((n ^ (g & 7)) << 4) + 4 * kq, wa);
        st_shared_u32(box + (g + 8) * 128 + ((n ^ ((g + 8) & 7)) << 4) + 4 * kq, wb);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        // rows >= S and columns >= head_dim are clipped by the map
        tma_store_4d(tm_ctx, box, 64 * hh, it.h, q0 + lg * 32 + sub * 16, it.b);
        bulk_commit_group();
      }
    }
    // The next item's first P.V overwrites O_t only after this thread's next
    // p_full arrival, which follows these TMEM loads.
  }
  if (lane == 0) bulk_wait_group_all();  // context stores complete before exit
}

template <typename T, int HD, bool CAUSAL>
__global__ void __launch_bounds__(AttnSmem<HD>::kThreads, 1)
flash_fwd_kernel(const __grid_constant__ CUtensorMap tm, const __grid_constant__ CUtensorMap tm_ctx,
                 const AttnParams p) {
  using L = AttnSmem<HD>;
  constexpr int ST = L::kStages;
  constexpr int NT = L::kNT;
  constexpr bool kSepP = L::kSepP;
  constexpr int kChunks = HD / 64;
  constexpr int kBf16 = std::is_same<T, __nv_bfloat16>::value ? 1 : 0;
  constexpr uint32_t kIdescQK = idesc_f16(kBM, kBN, kBf16, 0);
  constexpr uint32_t kIdescPV = idesc_f16(kBM, HD, kBf16, 1);
  constexpr uint32_t kPStride = kSepP ? 64 : 128;  // P column stride between tiles

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sQ = smem + L::kQOff;
  uint8_t* sK = smem + L::kKOff;
  uint8_t* sV = smem + L::kVOff;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* q_full = bars;              // [kQBufs][2] per tile: Q_t loaded
  uint64_t* q_empty = q_full + 4;       // [kQBufs][2] per tile: last Q_t K^T of the item done
  uint64_t* k_full = q_empty + 4;       // [ST]
  uint64_t* k_empty = k_full + ST;      // [2][ST] per tile: its Q_t K^T done with the stage
  uint64_t* v_full = k_empty + 2 * ST;  // [ST]
  uint64_t* v_empty = v_full + ST;      // [2][ST] per tile: its P_t V done with the stage
  uint64_t* s_full = v_empty + 2 * ST;  // [2] per tile: S_t written
  uint64_t* s_free = s_full + 2;        // [2] per tile: S_t read by the softmax (separate P)
  uint64_t* p_full = s_free + 2;        // [2] per tile: P_t written
  uint64_t* o_done = p_full + 2;        // [2] per tile: one phase per completed P_t V
  uint64_t* drain = o_done + 2;         // [2] per tile: every MMA of its issuer completed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < ST; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&v_full[s], 1);
      for (int t = 0; t < 2; ++t) {
        mbar_init(&k_empty[t * ST + s], 1);
        mbar_init(&v_empty[t * ST + s], 1);
      }
    }
    for (int t = 0; t < 2; ++t) {
      for (int b = 0; b < L::kQBufs; ++b) {
        mbar_init(&q_full[b * 2 + t], 1);
        mbar_init(&q_empty[b * 2 + t], 1);
      }
      mbar_init(&s_full[t], 1);
      mbar_init(&s_free[t], L::kSplit ? 256 : 128);   // every softmax thread of the tile
      mbar_init(&p_full[t], L::kSplit ? 256 : 128);
      mbar_init(&o_done[t], 1);
      mbar_init(&drain[t], 1);
    }
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
  grid_dependency_wait();  // the previous kernel's writes (qkv) are visible from here
  grid_launch_dependents();

  if (warp < 4) {
    setmaxnreg_dec<L::kRegsCtl>();
    if (warp == 0 && lane == 0) {
      // ------------------------------------------------------------ K/V producer
      // A stage is refilled once every tile that used its previous key tile has
      // released it (tile A skips the last key tile of a causal item).  Bit st
      // of pend[t]: tile t still holds stage st; bit st of ph[t]: parity of
      // tile t's next release of it.
      tma_prefetch_desc(&tm);
      uint32_t kpend[2] = {0u, 0u}, kph[2] = {0u, 0u}, vpend[2] = {0u, 0u}, vph[2] = {0u, 0u};
      auto reclaim = [&](uint64_t* empty, uint32_t (&pend)[2], uint32_t (&ph)[2], int st,
                         uint32_t users) -> bool {
        for (int t = 0; t < 2; ++t) {
          if ((pend[t] >> st) & 1u) {
            if (!mbar_wait(&empty[t * ST + st], (ph[t] >> st) & 1u, p.status, kDevTimeoutSmemEmpty, abort_flag))
              return false;
            ph[t] ^= 1u << st;
          }
          pend[t] = (pend[t] & ~(1u << st)) | (((users >> t) & 1u) << st);
        }
        return true;
      };
      int kv = 0;  // running K/V tile counter across items
      bool ok = true;
      for (int k = 0; ok; ++k) {
        const int item = item_of(k);
        if (item >= p.num_items) break;
        const Item it = decode_item<CAUSAL>(item, p);
        const int n_a = kv_tiles<CAUSAL, NT>(it.pair, 0, p.S);
        // key tiles of the item's last tile (with one tile per item, tile A's)
        const int n_kv = kv_tiles<CAUSAL, NT>(it.pair, NT - 1, p.S);
        const int yk = p.H + it.h, yv = 2 * p.H + it.h;  // head index of K / V in the 3H axis
        for (int j = 0; j < n_kv; ++j, ++kv) {
          const int st = kv % ST;
          // bit t: tile t releases this key tile (with P over S one thread issues
          // both tiles' products and releases through tile B's barrier)
          const uint32_t users = (kSepP && j < n_a) ? 3u : 2u;
          if (!reclaim(k_empty, kpend, kph, st, users)) { ok = false; break; }
          mbar_arrive_expect_tx(&k_full[st], L::kTileBytes);
          for (int c = 0; c < kChunks; ++c)
            tma_load_4d(sK + st * L::kTileBytes + c * kChunkBytes, &tm, &k_full[st], 64 * c, yk, j * kBN, it.b);
          if (!reclaim(v_empty, vpend, vph, st, users)) { ok = false; break; }
          mbar_arrive_expect_tx(&v_full[st], L::kTileBytes);
          for (int c = 0; c < kChunks; ++c)
            tma_load_4d(sV + st * L::kTileBytes + c * kChunkBytes, &tm, &v_full[st], 64 * c, yv, j * kBN, it.b);
        }
      }
    } else if (warp == 2 && lane == 0) {
      // ------------------------------------------------------------ Q producer
      for (int k = 0;; ++k) {
        const int item = item_of(k);
        if (item >= p.num_items) break;
        const Item it = decode_item<CAUSAL>(item, p);
        bool ok = true;
        for (int t = 0; t < NT && ok; ++t) {
          const int qb = k % L::kQBufs;
          const uint32_t qph = (k / L::kQBufs) & 1;
          ok = mbar_wait(&q_empty[qb * 2 + t], qph ^ 1u, p.status, kDevTimeoutSmemEmpty, abort_flag);
          if (!ok) break;
          mbar_arrive_expect_tx(&q_full[qb * 2 + t], L::kTileBytes);
          for (int c = 0; c < kChunks; ++c)
            tma_load_4d(sQ + (qb * NT + t) * L::kTileBytes + c * kChunkBytes, &tm, &q_full[qb * 2 + t], 64 * c, it.h,
                        it.pair * NT * kBM + t * kBM, it.b);
        }
        if (!ok) break;
      }
    } else if (lane == 0 && (warp == 1 || (kSepP && warp == 3))) {
      // ------------------------------------------------------------ MMA issue
      auto qk = [&](int t, int st, int qb) {
        const uint32_t q_addr = smem_u32(sQ + (qb * NT + t) * L::kTileBytes);
        const uint32_t k_addr = smem_u32(sK + st * L::kTileBytes);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t off = (kk >> 2) * kChunkBytes + (kk & 3) * 32;
          umma_f16_ss(tmem + t * 128, smem_desc_sw128(q_addr + off, 16, 1024),
                      smem_desc_sw128(k_addr + off, 16, 1024), kIdescQK, kk > 0 ? 1u : 0u);
        }
      };
      auto pv = [&](int t, int st, bool accumulate) {
        const uint32_t v_addr = smem_u32(sV + st * L::kTileBytes);
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk) {
          // V is MN-major: 16 keys = 16 rows of 128 bytes; next 64-column chunk at +16 KB.
          umma_f16_ts(tmem + L::kColO + t * HD, tmem + L::kColP + t * kPStride + kk * 8,
                      smem_desc_sw128(v_addr + kk * 16 * 128, kChunkBytes, 1024), kIdescPV,
                      (accumulate || kk > 0) ? 1u : 0u);
        }
      };
      if constexpr (kSepP) {
        // Separate P: one issuing thread per tile (warp 1: A, warp 3: B).
        // Measured: one thread issuing both tiles' products, waits and commits
        // spent the whole step on that serial work while the tensor pipe idled
        // more than half of it.  Per tile the QK cursor runs one key tile ahead
        // of the P.V cursor, across items: S_t(j+1) is issued once the softmax
        // has read S_t(j) (s_free), then O_t += P_t(j) V_j once P_t(j) is written.
        const int t = warp == 3 ? 1 : 0;
        int qk_k = 0, qk_j = 0, qk_kv0 = 0, qk_n = 0, qk_nb = 0;
        bool qk_first = true;
        auto qk_open = [&]() -> bool {
          const int item = item_of(qk_k);
          if (item >= p.num_items) return false;
          const Item it = decode_item<CAUSAL>(item, p);
          qk_n = kv_tiles<CAUSAL, NT>(it.pair, t, p.S);
          qk_nb = kv_tiles<CAUSAL, NT>(it.pair, NT - 1, p.S);
          return true;
        };
        bool qk_live = qk_open();
        uint32_t sfree_ph = 0u, pf_ph = 0u;
        auto issue_qk = [&]() -> bool {
          if (!qk_live) return true;
          const int qb = qk_k % L::kQBufs;
          if (qk_j == 0 && !mbar_wait(&q_full[qb * 2 + t], (qk_k / L::kQBufs) & 1, p.status, kDevTimeoutTmaFull,
                                      abort_flag))
            return false;
          if (!qk_first) {
            if (!mbar_wait(&s_free[t], sfree_ph, p.status, kDevTimeoutSoftmax, abort_flag)) return false;
            sfree_ph ^= 1u;
          }
          const int kvi = qk_kv0 + qk_j;
          const int st = kvi % ST;
          if (!mbar_wait(&k_full[st], (kvi / ST) & 1, p.status, kDevTimeoutTmaFull, abort_flag)) return false;
          tc_fence_after();
          qk(t, st, qb);
          umma_commit(&s_full[t]);
          umma_commit(&k_empty[t * ST + st]);
          qk_first = false;
          if (++qk_j == qk_n) {  // last S_t of the item: Q_t may be replaced
            umma_commit(&q_empty[qb * 2 + t]);
            qk_kv0 += qk_nb;
            qk_j = 0;
            ++qk_k;
            qk_live = qk_open();
          }
          return true;
        };
        bool ok = issue_qk();
        int kv0 = 0;
        for (int k = 0; ok; ++k) {
          const int item = item_of(k);
          if (item >= p.num_items) break;
          const Item it = decode_item<CAUSAL>(item, p);
          const int n = kv_tiles<CAUSAL, NT>(it.pair, t, p.S);
          const int n_b = kv_tiles<CAUSAL, NT>(it.pair, NT - 1, p.S);
          for (int j = 0; j < n; ++j) {
            // S_t(j+1), or the next item's S_t(0) (its Q is double-buffered, so
            // normally already loaded), then this key tile's P.V.  Issuing the
            // item's last P.V first measured slower for causal items.
            if (!issue_qk()) { ok = false; break; }
            if (!mbar_wait(&p_full[t], pf_ph, p.status, kDevTimeoutSoftmax, abort_flag)) { ok = false; break; }
            pf_ph ^= 1u;
            const int kvi = kv0 + j;
            const int st = kvi % ST;
            if (!mbar_wait(&v_full[st], (kvi / ST) & 1, p.status, kDevTimeoutTmaFull, abort_flag)) { ok = false; break; }
            tc_fence_after();
            pv(t, st, j > 0);
            umma_commit(&o_done[t]);
            umma_commit(&v_empty[t * ST + st]);
          }
          kv0 += n_b;
        }
        // Nothing of this thread's may still run on the tensor core when TMEM
        // is released (matters only after an abort).
        umma_commit(&drain[t]);
        mbar_wait(&drain[t], 0, p.status, kDevTimeoutSoftmax, nullptr);
      } else {
        static_assert(L::kQBufs == 1, "the single-issuer schedule uses one Q buffer per tile");
        // P over S: one thread issues both tiles, PV_A(j) QK_A(j+1) PV_B(j)
        // QK_B(j+1) (measured faster here than one thread per tile: each tile's
        // next S waits for its own P.V, and the fixed interleave keeps the two
        // tiles' softmax steps half a step apart).  With one tile per item
        // (head_dim 256) only the tile-A half of each step is issued; the
        // stage releases still go through tile B's barriers, which is where
        // the producer waits for them.
        int kv = 0;
        uint32_t pf_phase[2] = {0u, 0u};
        bool ok = true;
        // One commit per stage, through tile B's barrier: it arrives once every
        // earlier product of this thread (tile A's included) has completed.
        auto release = [&](uint64_t* empty, int st) { umma_commit(&empty[ST + st]); };
        for (int k = 0; ok; ++k) {
          const int item = item_of(k);
          if (item >= p.num_items) break;
          const Item it = decode_item<CAUSAL>(item, p);
          const int n_a = kv_tiles<CAUSAL, NT>(it.pair, 0, p.S);
          // key tiles of the item's last tile (n_b >= n_a)
          const int n_b = kv_tiles<CAUSAL, NT>(it.pair, NT - 1, p.S);
          if (!mbar_wait(&q_full[0], k & 1, p.status, kDevTimeoutTmaFull, abort_flag)) break;
          if (NT == 2 && !mbar_wait(&q_full[1], k & 1, p.status, kDevTimeoutTmaFull, abort_flag)) break;
          const int kv0 = kv;
          {
            const int st = kv0 % ST;
            if (!mbar_wait(&k_full[st], (kv0 / ST) & 1, p.status, kDevTimeoutTmaFull, abort_flag)) break;
            tc_fence_after();
            qk(0, st, 0);
            umma_commit(&s_full[0]);
            if (n_a == 1) umma_commit(&q_empty[0]);
            if constexpr (NT == 2) {
              qk(1, st, 0);
              umma_commit(&s_full[1]);
              if (n_b == 1) umma_commit(&q_empty[1]);
            }
            release(k_empty, st);
          }
          for (int j = 0; j < n_b; ++j) {
            const int st = (kv0 + j) % ST;
            const uint32_t ph = ((kv0 + j) / ST) & 1;
            const int st_n = (kv0 + j + 1) % ST;
            const uint32_t ph_n = ((kv0 + j + 1) / ST) & 1;
            const bool next_b = j + 1 < n_b;
            if (next_b && !mbar_wait(&k_full[st_n], ph_n, p.status, kDevTimeoutTmaFull, abort_flag)) { ok = false; break; }
            if (!mbar_wait(&v_full[st], ph, p.status, kDevTimeoutTmaFull, abort_flag)) { ok = false; break; }
            if constexpr (NT == 2) {
              if (j < n_a) {
                if (!mbar_wait(&p_full[0], pf_phase[0], p.status, kDevTimeoutSoftmax, abort_flag)) { ok = false; break; }
                pf_phase[0] ^= 1u;
                tc_fence_after();
                pv(0, st, j > 0);
                if (j + 1 < n_a) {
                  qk(0, st_n, 0);
                  umma_commit(&s_full[0]);
                  if (j + 2 == n_a) umma_commit(&q_empty[0]);
                } else {
                  umma_commit(&o_done[0]);
                }
              }
            }
            // The item's last tile (tile B, or tile A alone with one tile per item).
            constexpr int tl = NT - 1;
            if (!mbar_wait(&p_full[tl], pf_phase[tl], p.status, kDevTimeoutSoftmax, abort_flag)) { ok = false; break; }
            pf_phase[tl] ^= 1u;
            tc_fence_after();
            pv(tl, st, j > 0);
            release(v_empty, st);
            if (next_b) {
              qk(tl, st_n, 0);
              umma_commit(&s_full[tl]);
              release(k_empty, st_n);
              if (j + 2 == n_b) umma_commit(&q_empty[tl]);
            } else {
              umma_commit(&o_done[tl]);
            }
          }
          kv = kv0 + n_b;
        }
        umma_commit(&drain[0]);
        mbar_wait(&drain[0], 0, p.status, kDevTimeoutSoftmax, nullptr);
      }
    }
  } else {
    setmaxnreg_inc<L::kRegsSoftmax>();
    if constexpr (L::kSplit) {
      softmax_split<T, HD, CAUSAL>(p, smem + L::kEpiOff, tmem, &tm_ctx, s_full, s_free, p_full, o_done, abort_flag);
    } else {
    // ------------------------------------------------------------ softmax (tile A or B)
    // One warp per tile and TMEM lane quarter, P written over S (head_dim 128 / 256).
    static_assert(!kSepP, "separate-P schedules use softmax_split");
    const int t = warp >= 8 ? 1 : 0;
    if (t < NT) {  // one tile per item: warps 8..11 have no work
    const int lg = warp & 3;             // TMEM lane quarter of this warp
    const int r = lg * 32 + lane;        // query row within the tile
    const uint32_t t_lane = tmem + (static_cast<uint32_t>(lg * 32) << 16);
    const uint32_t t_s = t_lane + t * 128;
    const uint32_t t_p = t_lane + L::kColP + t * kPStride;
    const uint32_t t_o = t_lane + L::kColO + t * HD;
    uint32_t sf_phase = 0;
    uint32_t od_phase = 0;  // o_done parity of the next P.V to wait for
    bool ok = true;
    for (int k = 0; ok; ++k) {
      const int item = item_of(k);
      if (item >= p.num_items) break;
      const Item it = decode_item<CAUSAL>(item, p);
      const int n_kv = kv_tiles<CAUSAL, NT>(it.pair, t, p.S);
      const int q0 = it.pair * NT * kBM + t * kBM;
      const int q_row = q0 + r;
      const uint8_t* kmask = p.key_mask != nullptr ? p.key_mask + (int64_t)it.b * p.S : nullptr;
      // Key-mask bytes of the current key tile (lane l: keys l, l+32, l+64,
      // l+96), loaded one step ahead so the load overlaps the previous step.
      uint32_t mbyte[4] = {0u, 0u, 0u, 0u};
      if (kmask != nullptr) {
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          const int key = g * 32 + lane;
          mbyte[g] = key < p.S ? __ldg(kmask + key) : 0u;
        }
      }
      float m_run = -INFINITY;  // exponent reference (log2 units), moved lazily
      float l_run = 0.f;        // running sum of P in fp32
      for (int j = 0; j < n_kv; ++j) {
        if (!mbar_wait_warp(&s_full[t], sf_phase, p.status, kDevTimeoutSoftmax, abort_flag)) { ok = false; break; }
        sf_phase ^= 1u;
        tc_fence_after();
        float s[kBN];
        {
          uint32_t u[kBN];
          tmem_ld128(t_s, u);
#pragma unroll
          for (int i = 0; i < kBN; ++i) s[i] = __uint_as_float(u[i]);
        }
        const int k0 = j * kBN;
        // Which of the tile's 128 keys this row may see: keys past S, keys the
        // key mask drops, and (causal) keys after the query are masked to -inf.
        const bool tail = k0 + kBN > p.S;
        const bool diag = CAUSAL && k0 + kBN - 1 > q0;  // the tile straddles the diagonal
        // Validity bits of the tile's keys (key < S and, with a key mask, its
        // byte set), built cooperatively: lane l holds keys l, l+32, l+64,
        // l+96, one ballot per group of 32.  Warp-uniform.
        uint32_t vbits[4] = {~0u, ~0u, ~0u, ~0u};
        if (tail || kmask != nullptr) {
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            const int key = k0 + g * 32 + lane;
            bool v = key < p.S;
            if (kmask != nullptr) v = v && mbyte[g] != 0u;
            vbits[g] = __ballot_sync(0xffffffffu, v);
          }
          if (kmask != nullptr && j + 1 < n_kv) {  // the next tile's bytes
#pragma unroll
            for (int g = 0; g < 4; ++g) {
              const int key = k0 + kBN + g * 32 + lane;
              mbyte[g] = key < p.S ? __ldg(kmask + key) : 0u;
            }
          }
        }
        if ((vbits[0] & vbits[1] & vbits[2] & vbits[3]) == ~0u) {
          // Every key valid (no mask, or an all-true mask such as the
          // benchmark's unpadded inputs): only the causal limit can apply.
          // Key k0 + i is visible to this row iff i <= q_row - k0: one compare
          // and one select per score.  (The general path below measured
          // ~2.5K cycles per step.)
          if (diag) {
            const int lim = q_row - k0;
#pragma unroll
            for (int i = 0; i < kBN; ++i) s[i] = i <= lim ? s[i] : -INFINITY;
          }
        } else {
#pragma unroll
          for (int i = 0; i < kBN; ++i) {
            bool v = (vbits[i >> 5] >> (i & 31)) & 1u;
            if (CAUSAL) v = v && (k0 + i <= q_row);
            s[i] = v ? s[i] : -INFINITY;
          }
        }
        // Row max: eight independent chains of 3-input max.
        float mx8[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) mx8[q] = fmax3(s[q], s[8 + q], s[16 + q]);
#pragma unroll
        for (int i = 24; i < kBN - 8; i += 16)
#pragma unroll
          for (int q = 0; q < 8; ++q) mx8[q] = fmax3(mx8[q], s[i + q], s[i + 8 + q]);
#pragma unroll
        for (int q = 0; q < 8; ++q) mx8[q] = fmaxf(mx8[q], s[kBN - 8 + q]);
        const float mx = fmax3(fmax3(mx8[0], mx8[1], mx8[2]), fmax3(mx8[3], mx8[4], mx8[5]),
                               fmaxf(mx8[6], mx8[7]));
        // Lazy rescaling: the exponent reference only moves when the tile max
        // exceeds it by more than 8 (log2 units), so P <= 2^8 and O rescales
        // are rare.  Exact in real arithmetic: the factor cancels in O / l.
        const float m_tile = mx * p.scale_log2;
        const float m_new = (m_tile > m_run + 8.f) ? m_tile : m_run;
        const float m_use = m_new == -INFINITY ? 0.f : m_new;
        const float alpha = fast_exp2(m_run - m_use);  // 1 unchanged, 0 from -inf
        // x = s * scale_log2 - m as packed pairs; P = 2^x, written over the S
        // columns already read 16 columns (32 keys) at a time.
        const uint64_t c2 = f2_pack(p.scale_log2, p.scale_log2);
        const uint64_t nm2 = f2_pack(-m_use, -m_use);
        // One MUFU exponential per element in fp32 (measured faster than the
        // paired fp16 form, which issues half the instructions but at half rate),
        // row sums as fp32 pairs in four chains.
        uint32_t pk[2][32];
        uint64_t sum2[4] = {0ull, 0ull, 0ull, 0ull};
#pragma unroll
        for (int c = 0; c < kBN / 32; ++c) {
          uint32_t (&pc)[16] = *reinterpret_cast<uint32_t(*)[16]>(&pk[c >> 1][(c & 1) * 16]);
#pragma unroll
          for (int ii = 0; ii < 16; ++ii) {
            const int i = c * 16 + ii;
            float x0, x1;
            f2_unpack(ffma2(f2_pack(s[2 * i], s[2 * i + 1]), c2, nm2), x0, x1);
            const float e0 = fast_exp2(x0);
            const float e1 = fast_exp2(x1);
            pc[ii] = Pack<T>::two(e0, e1);
            sum2[i & 3] = fadd2(sum2[i & 3], f2_pack(e0, e1));
          }
          tmem_st16(t_p + c * 16, pc);  // over the S columns already read
        }
        float a0, a1;
        f2_unpack(fadd2(fadd2(sum2[0], sum2[1]), fadd2(sum2[2], sum2[3])), a0, a1);
        const float sum = a0 + a1;
        l_run = l_run * alpha + sum;
        m_run = m_new;
        // Rescale O_t when the exponent reference moved (O_t holds P(0..j-1) V).
        if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll
          for (int c = 0; c < HD / 32; ++c) {
            uint32_t o[32];
            tmem_ld32(t_o + c * 32, o);
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st32(t_o + c * 32, o);
          }
        }
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(&p_full[t]);
      }
      if (!ok) break;
      // epilogue: wait for the last P.V, then O_t / l -> ctx rows (heads merged)
      if (!mbar_wait_warp(&o_done[t], od_phase, p.status, kDevTimeoutSoftmax, abort_flag)) break;
      od_phase ^= 1u;
      tc_fence_after();
      const float inv_l = 1.f / l_run;
      // this warp's 32 rows, 64 columns at a time: swizzled staging box, one
      // TMA store each (the box is reused once the previous store has read it)
      uint8_t* box = smem + L::kEpiOff + (warp - 4) * (32 * 128);
#pragma unroll
      for (int hh = 0; hh < HD / 64; ++hh) {
        if (64 * hh >= p.hd) break;  // only zero padding left (uniform)
        if (lane == 0) bulk_wait_group_read<0>();  // the previous store has read the box
        __syncwarp();
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t o[32];
          tmem_ld32(t_o + hh * 64 + c * 32, o);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 w;
            w.x = Pack<T>::two(__uint_as_float(o[8 * q + 0]) * inv_l, __uint_as_float(o[8 * q + 1]) * inv_l);
            w.y = Pack<T>::two(__uint_as_float(o[8 * q + 2]) * inv_l, __uint_as_float(o[8 * q + 3]) * inv_l);
            w.z = Pack<T>::two(__uint_as_float(o[8 * q + 4]) * inv_l, __uint_as_float(o[8 * q + 5]) * inv_l);
            w.w = Pack<T>::two(__uint_as_float(o[8 * q + 6]) * inv_l, __uint_as_float(o[8 * q + 7]) * inv_l);
            const int chunk = c * 4 + q;  // 16-byte chunk of the 128-byte row
            *reinterpret_cast<uint4*>(box + lane * 128 + ((chunk ^ (lane & 7)) << 4)) = w;
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          // rows >= S and columns >= head_dim are clipped by the map
          tma_store_4d(&tm_ctx, box, 64 * hh, it.h, q0 + lg * 32, it.b);
          bulk_commit_group();
        }
      }
      // The next item's first P.V overwrites O_t only after this thread's next
      // p_full arrival, which follows these TMEM loads.
    }
    if (lane == 0) bulk_wait_group_all();  // context stores complete before exit
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
  constexpr int NT = L::kNT;
  const CUtensorMapDataType dt = std::is_same<T, __half>::value ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                                : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const uint64_t hd = (uint64_t)a.head_dim, H = (uint64_t)a.num_heads, D = H * hd;
  // qkv [B, S, 3D] seen as [B][S][3H][head_dim]: head h of q / k / v is index
  // h / H + h / 2H + h of the 3H axis.  The box is 64 columns wide whatever
  // head_dim is; columns past head_dim read as zeros.
  CUtensorMap tm;
  const uint64_t dims[4] = {hd, 3 * H, (uint64_t)a.seq_len, (uint64_t)a.batch};
  const uint64_t strides[3] = {hd * 2, 3 * D * 2, (uint64_t)a.seq_len * 3 * D * 2};
  const uint32_t box[4] = {64, 1, 128, 1};
  int rc = encode_tmap(&tm, dt, 4, a.qkv, dims, strides, box);
  if (rc) return rc;
  // ctx [B, S, D] seen as [B][S][H][head_dim]: the epilogue's 32-row x 64-column
  // boxes, clipped at head_dim and at S.
  CUtensorMap tm_ctx;
  const uint64_t cdims[4] = {hd, H, (uint64_t)a.seq_len, (uint64_t)a.batch};
  const uint64_t cstrides[3] = {hd * 2, D * 2, (uint64_t)a.seq_len * D * 2};
  const uint32_t cbox[4] = {64, 1, (uint32_t)L::kEpiRows, 1};
  rc = encode_tmap(&tm_ctx, dt, 4, a.ctx, cdims, cstrides, cbox);
  if (rc) return rc;
  AttnParams p;
  p.ctx = a.ctx;
  p.key_mask = a.key_mask;
  p.B = (int)a.batch;
  p.S = (int)a.seq_len;
  p.H = (int)a.num_heads;
  p.hd = (int)a.head_dim;
  p.num_pairs = (int)((a.seq_len + NT * kBM - 1) / (NT * kBM));
  const int64_t items = a.batch * a.num_heads * (int64_t)p.num_pairs;
  // K and V of every head (2 x S x head_dim x 2 bytes each) against ~3/4 of the 126 MB L2.
  p.head_major = a.batch * a.num_heads * a.seq_len * a.head_dim * 4 > kHeadMajorKvBytes ? 1 : 0;
  if (items >= (int64_t)1 << 31) return fail(TTJ_ERR_UNSUPPORTED, "too many attention work items");
  p.num_items = (int)items;
  p.scale_log2 = (float)(1.0 / sqrt((double)a.head_dim) * 1.4426950408889634);
  p.status = a.status;
  auto kern = flash_fwd_kernel<T, HD, CAUSAL>;
  {
    // The register split inside the kernel assumes this launch allocation;
    // with any other the softmax warps' setmaxnreg.inc could never complete.
    cudaFuncAttributes fa;
    TTJ_CUDA_TRY(cudaFuncGetAttributes(&fa, kern));
    if (fa.numRegs != L::kLaunchRegs)
      return fail(TTJ_ERR_UNSUPPORTED, "attention kernel register count differs from its register split");
  }
  TTJ_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kTotal));
  const int grid = p.num_items < sm_count() ? p.num_items : sm_count();
  TTJ_CUDA_TRY(launch_pdl(kern, dim3(grid), dim3(L::kThreads), L::kTotal, stream, tm, tm_ctx, p));
  return TTJ_OK;
}

// head_dim runs on the kernel of the next padded size: up to 64, up to 128, up to 256.
template <typename T, int HD>
int dispatch_causal(const AttnArgs& a, cudaStream_t stream) {
  return a.causal ? launch_attn<T, HD, true>(a, stream) : launch_attn<T, HD, false>(a, stream);
}

template <typename T>
int dispatch_hd(const AttnArgs& a, cudaStream_t stream) {
  if (a.head_dim <= 64) return dispatch_causal<T, 64>(a, stream);
  if (a.head_dim <= 128) return dispatch_causal<T, 128>(a, stream);
  return dispatch_causal<T, 256>(a, stream);
}

}  // namespace

int launch_flash_attn(const AttnArgs& a, cudaStream_t stream) {
  return a.dtype == TTJ_F16 ? dispatch_hd<__half>(a, stream) : dispatch_hd<__nv_bfloat16>(a, stream);
}

}  // namespace ttj
