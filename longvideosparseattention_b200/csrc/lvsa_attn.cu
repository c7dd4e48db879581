// Block-sparse LVSA attention forward for sm_100a (tcgen05 + TMEM + TMA).
//
// Two kernels share the softmax and MMA code: lvsa_attn_kernel (one query
// tile per CTA, described here; D = 64 and FP8) and lvsa_attn_pair_kernel
// (two query tiles per CTA sharing their K/V loads; bf16/f16 D = 128),
// described above its definition.
//
// One CTA per (128-row query tile, head, batch); 320 threads:
//   warps 0-7  softmax, one thread per query row and key-tile class: warps
//              0-3 take the even entries j of the row's tile list, warps 4-7
//              the odd ones (warp w reads TMEM lanes 32 (w % 4) .. +32, so a
//              row's two threads sit on the same SM sub-partition).  Each
//              class keeps its own running max / sum and its own O
//              accumulator, so the two warps of a sub-partition never wait
//              for each other inside the loop: while one exponentiates (MUFU),
//              the other loads, masks and reduces.  The two partial results
//              are merged once, in the epilogue.
//   warp 8     TMA producer: the query tile once, then K and V tiles of the
//              row's CSR list, read in place from the [B, N, H, D] tensors
//              into a ring of shared-memory stages (K and V released
//              separately).
//   warp 9     TMEM allocator + single-thread tcgen05.mma issuer, in the
//              order S(0) S(1) PV(0) S(2) PV(1) S(3) ...:  S(j) = Q K_j^T
//              (both operands in shared memory) into S buffer j % 2; PV(j)
//              = P(j) V_j accumulates into O buffer j % 2 with P read from
//              the same TMEM columns that held S(j).  S(j+2) reuses that
//              buffer and is issued after PV(j); tcgen05.mma operations of one
//              thread execute in issue order.
// TMEM columns: S/P buffer c at [128 c, 128 c + 128), O buffer c at
// [256 + 128 c, 256 + 128 c + D).  Per key tile the softmax thread loads S
// columns [0,64), then [64,128) (row max), writes P of keys 0-63 into
// columns [0,32) (bf16 pairs; E4M3 quads: [0,16)), reloads [64,128) and
// writes P of keys 64-127 after it.
//
// Semantics follow lvsa_sdpa (lvsa/sparse_attention.py:643-706) with the
// processor's text handling (lvsa/lvsa_processor.py:545-549, 584-591):
// every video query attends to all tokens of its frame's attended set and all
// text tokens; text queries attend to everything.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <type_traits>

#include "../../include/lvsa_b200.h"
#include "lvsa_ptx.cuh"

// Instrumentation build only (-DLVSA_PROFILE): clock64 totals per role of
// the tile-pair kernel, read back by lvsa_prof_read.  Compiled out otherwise.
#ifdef LVSA_PROFILE
__device__ unsigned long long g_lvsa_prof[16];
#define LVSA_CLK(x) const long long x = clock64()
#define LVSA_PROF_ADD(i, v) atomicAdd(&g_lvsa_prof[i], static_cast<unsigned long long>(v))
#else
#define LVSA_CLK(x)
#define LVSA_PROF_ADD(i, v)
#endif

namespace lvsa {
namespace {

constexpr int kBM = 128;           // query rows per CTA (= CSR block_q)
constexpr int kBlockQ = kBM;
constexpr int kBN = 128;           // key tokens per tile (= CSR block_k)
constexpr int kChunk = 128 * 128;  // one 128-row x 128-byte swizzle-128B slab
constexpr int kSoftmaxWarps = 8;
constexpr int kProducerWarp = kSoftmaxWarps;
constexpr int kMmaWarp = kSoftmaxWarps + 1;
constexpr int kThreads = 32 * (kSoftmaxWarps + 2);
constexpr uint32_t kTmemCols = 512;
constexpr float kNegInf = -INFINITY;
#ifndef LVSA_S3
#define LVSA_S3 1
#endif
#ifndef LVSA_TEXT_FIRST
#define LVSA_TEXT_FIRST 1
#endif
constexpr float kRescaleThreshold = 8.0f;  // log2 units: rescale O only when the max grows by > 2^8

struct AttnParams {
  const void* q;
  const void* text_q;
  int64_t q_sb, q_st, q_sh, tq_sb, tq_st, tq_sh;
  void* o;
  void* text_o;
  float* lse;
  float* text_lse;
  int64_t o_sb, o_st, o_sh, to_sb, to_st, to_sh;
  int n_video, n_kv, n_text, heads, kv_heads, T, P, words, nqv, nkv;  // n_kv: video keys
  float scale_log2;
  const uint32_t* frame_bits;
  const int32_t* indptr;
  const int32_t* indices;
  const uint8_t* flags;
  int* err;
  // FP8 mode only: per-tile scales [B, H(kv), tiles] and the per-head V reference.
  const float* qs;
  const float* ks;
  const float* vs;
  const float* tqs;
  const float* tks;
  const float* tvs;
  const float* vref;
  int nqt_all, nkt;  // query / key tiles of the text segment
  int tok_off;       // global token of the video segment's first token (sequence shards)
  int row0;          // first tile-CSR row of this launch
  // Tile-pair kernel: video rows [row0, pair_ve) in pair_nv pairs, then text
  // rows [pair_ts, pair_end).
  int pair_ve, pair_ts, pair_end, pair_nv;
  uint64_t wait_ns;  // limit of every bounded wait
  int inject;        // test hook: CTA (0, 0, 0) never loads its query tile
};


template <int D, int SK, int SV, bool kFp8 = false>
struct Smem {
  static constexpr int kElem = kFp8 ? 1 : 2;       // bytes per element
  static constexpr int kCh = D * kElem / 128;      // 128-byte column slabs per row
  static constexpr int kTile = kCh * kChunk;       // bytes of one 128 x D tile
  static constexpr int kQ = 0;                     // query tile; the epilogue's merge buffer afterwards
  static constexpr int kK = kQ + kTile;
  static constexpr int kV = kK + SK * kTile;
  static constexpr int kBar = kV + SV * kTile;
  static constexpr int kNumBars = 2 * SK + 2 * SV + 12;
  static constexpr int kMisc = kBar + kNumBars * 8;
  static constexpr int kBytes = kMisc + 16 + 1024;  // + alignment slack
  static_assert(kBytes <= 232448, "shared memory");
  static_assert(2 * 2 * kBM * 4 <= kTile, "merge buffer fits in the query tile");
};

__device__ __forceinline__ uint32_t pack2(float a, float b, bool bf16) {
  if (bf16) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ void set_cols(uint32_t (&am)[4], int a, int b) {  // [a, b)
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    const int lo = max(a, w * 32), hi = min(b, w * 32 + 32);
    if (lo < hi) {
      const int n = hi - lo;
      const uint32_t m = (n == 32) ? 0xFFFFFFFFu : ((1u << n) - 1u);
      am[w] |= m << (lo - w * 32);
    }
  }
}

// Allowed-column mask of one key tile for one query row.
__device__ __forceinline__ void tile_mask(uint32_t (&am)[4], const AttnParams& prm, int kt, bool text_row,
                                          const uint32_t* fbits) {
  am[0] = am[1] = am[2] = am[3] = 0u;
  if (kt >= prm.nkv) {
    set_cols(am, 0, min(kBN, prm.n_text - (kt - prm.nkv) * kBN));
  } else if (text_row) {
    set_cols(am, 0, min(kBN, prm.n_kv - kt * kBN));
  } else {
    // Key tokens are numbered from the shard start; frames from the grid start.
    const int ks = kt * kBN, kend = min(ks + kBN, prm.n_kv);
    int f = (prm.tok_off + ks) / prm.P, c0 = 0;
    while (ks + c0 < kend) {
      const int ce = min((f + 1) * prm.P - prm.tok_off, kend) - ks;
      if ((fbits[f >> 5] >> (f & 31)) & 1u) set_cols(am, c0, ce);
      c0 = ce;
      ++f;
    }
  }
}

// tcgen05.mma kind::f8f6f4 (E4M3 x E4M3 -> fp32), A from TMEM.
__device__ __forceinline__ void mma_ts_f8(uint32_t d, uint32_t a_tmem, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

template <bool kFp8>
__device__ __forceinline__ void mma_ts_any(uint32_t d, uint32_t a_tmem, uint64_t b, uint32_t idesc, uint32_t acc) {
  if constexpr (kFp8) mma_ts_f8(d, a_tmem, b, idesc, acc);
  else mma_ts(d, a_tmem, b, idesc, acc);
}

__device__ __forceinline__ uint32_t pack4_e4m3(float a, float b, float c, float d) {
  const __nv_fp8x2_storage_t lo = __nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, __NV_E4M3);
  const __nv_fp8x2_storage_t hi = __nv_cvt_float2_to_fp8x2(make_float2(c, d), __NV_SATFINITE, __NV_E4M3);
  return static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
}


// tcgen05.mma kind::f8f6f4, both operands in shared memory.
__device__ __forceinline__ void mma_ss_f8(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

template <bool kFp8>
__device__ __forceinline__ void mma_ss_any(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  if constexpr (kFp8) mma_ss_f8(d, a, b, idesc, acc);
  else mma_ss(d, a, b, idesc, acc);
}

__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Sets masked-out columns of one 64-column half to -inf (bits of w0 | w1 << 32).
__device__ __forceinline__ void mask64(uint32_t (&sv)[64], uint32_t w0, uint32_t w1) {
#pragma unroll
  for (int i = 0; i < 64; ++i)
    if (!((((i < 32) ? w0 : w1) >> (i & 31)) & 1u)) sv[i] = __float_as_uint(kNegInf);
}

__device__ __forceinline__ float max64(const uint32_t (&sv)[64]) {
  float mx[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) mx[i] = fmax3(__uint_as_float(sv[i]), __uint_as_float(sv[8 + i]), __uint_as_float(sv[16 + i]));
#pragma unroll
  for (int i = 0; i < 8; ++i) mx[i] = fmax3(mx[i], __uint_as_float(sv[24 + i]), __uint_as_float(sv[32 + i]));
#pragma unroll
  for (int i = 0; i < 8; ++i) mx[i] = fmax3(mx[i], __uint_as_float(sv[40 + i]), __uint_as_float(sv[48 + i]));
#pragma unroll
  for (int i = 0; i < 8; ++i) mx[i] = fmaxf(mx[i], __uint_as_float(sv[56 + i]));
  return fmaxf(fmax3(mx[0], mx[1], mx[2]), fmax3(fmax3(mx[3], mx[4], mx[5]), mx[6], mx[7]));
}

// P = 2^(s * sl2 - mu) for 64 key columns, packed for the PV MMA: bf16/f16
// pairs (32 words) or, with kFp8, E4M3 quads of P * pscale (words 0-15).
// Returns the row sum of the unscaled P.
template <bool kBf16, bool kFp8>
__device__ __forceinline__ float exp64(const uint32_t (&sv)[64], uint64_t sl2x2, uint64_t nmu2, float pscale,
                                       uint32_t (&pk)[32]) {
  uint64_t acc2[4] = {0ull, 0ull, 0ull, 0ull};
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const uint64_t x2 = f2_fma(f2_pack(__uint_as_float(sv[2 * i]), __uint_as_float(sv[2 * i + 1])), sl2x2, nmu2);
    float xa, xc;
    f2_unpack(x2, xa, xc);
    const float a = ex2_approx(xa), c = ex2_approx(xc);
    acc2[i & 3] = f2_add(acc2[i & 3], f2_pack(a, c));
    if constexpr (kFp8) {
      if (i & 1) {
        const float a0 = __uint_as_float(pk[i - 1]), c0 = __uint_as_float(pk[i]);  // held pair i-1
        pk[i >> 1] = pack4_e4m3(a0, c0, a * pscale, c * pscale);
      } else {
        pk[i] = __float_as_uint(a * pscale);
        pk[i + 1] = __float_as_uint(c * pscale);
      }
    } else {
      pk[i] = pack2(a, c, kBf16);
    }
  }
  float acc[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) f2_unpack(acc2[i], acc[2 * i], acc[2 * i + 1]);
  return ((acc[0] + acc[1]) + (acc[2] + acc[3])) + ((acc[4] + acc[5]) + (acc[6] + acc[7]));
}

template <bool kFp8>
__device__ __forceinline__ void store_p(uint32_t taddr, const uint32_t (&pk)[32]) {
  if constexpr (kFp8) {
    uint32_t pk8[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) pk8[i] = pk[i];
    tmem_st16(taddr, pk8);
  } else {
    tmem_st32(taddr, pk);
  }
}

// kBf16: type of O (and of Q/K/V unless kFp8).  kFp8: Q/K/V are E4M3 copies
// with per-tile scales (QK^T and PV on kind::f8f6f4, P rounded to E4M3).
template <int D, int SK, int SV, bool kBf16, bool kFp8 = false>
__global__ void __launch_bounds__(kThreads, 1)
    lvsa_attn_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                     const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_tq,
                     const __grid_constant__ CUtensorMap tm_tk, const __grid_constant__ CUtensorMap tm_tv,
                     const AttnParams prm) {
  using L = Smem<D, SK, SV, kFp8>;
  // S/P buffers in TMEM: two (the classes alternate buffers, so S(j+2) waits
  // for PV(j)); three when the O buffers are narrow enough to leave room
  // (D = 64: 3 x 128 + 2 x 64 = 512 columns), so S(j+3) follows PV(j) and a
  // class's next S is issued while the other class still runs its softmax.
  constexpr int kNB = (D == 64 && LVSA_S3) ? 3 : 2;
  constexpr int kOStride = kNB == 3 ? D : 128;
  static_assert(kNB * 128 + 2 * kOStride <= static_cast<int>(kTmemCols), "TMEM columns");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem + L::kQ;
  uint8_t* sK = smem + L::kK;
  uint8_t* sV = smem + L::kV;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBar);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* v_full = k_full + SK;       // [SV]
  uint64_t* k_empty = v_full + SV;       // [SK] K stage free: the S of its tile is done
  uint64_t* v_empty = k_empty + SK;      // [SV] V stage free: the PV of its tile is done
  uint64_t* s_full = v_empty + SV;       // [kNB] S buffer b holds S(j), j % kNB == b
  uint64_t* p_full = s_full + 3;         // [kNB] P(j) written into buffer b
  uint64_t* pv_done = p_full + 3;        // [2] (kNB == 3) PV of class c retired
  uint64_t* o_done = pv_done + 2;        // every MMA of the CTA retired
  uint64_t* drain = o_done + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kMisc);
  volatile int* abort = reinterpret_cast<volatile int*>(smem + L::kMisc + 4);
  volatile int* never = reinterpret_cast<volatile int*>(smem + L::kMisc + 8);  // stays 0: drain waits

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Text query rows (dense: every key tile) are the longest CTAs of a head;
  // they take the first block indices so they start early instead of
  // forming the launch's tail.
  const int n_text_rows = prm.pair_end - max(prm.row0, prm.nqv);
  const int xr = (LVSA_TEXT_FIRST && n_text_rows > 0)
                     ? static_cast<int>((blockIdx.x + gridDim.x - n_text_rows) % gridDim.x)
                     : static_cast<int>(blockIdx.x);
  const int row = xr + prm.row0, h = blockIdx.y, b = blockIdx.z;
  const int beg = prm.indptr[row];
  const int n = prm.indptr[row + 1] - beg;
  const bool text_row = row >= prm.nqv;
  const int tok0 = (text_row ? row - prm.nqv : row) * kBM;
  const int hk = h / (prm.heads / prm.kv_heads);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < SK; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
    }
    for (int s = 0; s < SV; ++s) {
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int i = 0; i < kNB; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 128);
    }
    for (int i = 0; i < 2; ++i) mbar_init(&pv_done[i], 1);
    mbar_init(o_done, 1);
    mbar_init(drain, 1);
    *abort = 0;
    *never = 0;
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // TMEM: kNB S/P buffers of 128 columns, then the two classes' O buffers.
  const uint32_t tS = tmem, tO = tmem + kNB * 128;

  if (warp == kProducerWarp) {
    // ---------------------------------------------------------- producer
    if (lane == 0 && n > 0) {
      const CUtensorMap* mq = text_row ? &tm_tq : &tm_q;
      tma_prefetch_desc(mq);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      const bool skip_q = prm.inject && (blockIdx.x | blockIdx.y | blockIdx.z) == 0;
      if (!skip_q) {
        mbar_expect_tx(q_full, L::kTile);
#pragma unroll
        for (int c = 0; c < L::kCh; ++c) tma_load_4d(sQ + c * kChunk, mq, q_full, c * (128 / L::kElem), h, tok0, b);
      }
      int k_issued = 0, v_issued = 0;
      for (int j = 0; j < n; ++j) {
        const int s = j % SK, sv = j % SV;
        const int kt = prm.indices[beg + j];
        const bool tt = kt >= prm.nkv;
        const int ktok = (tt ? kt - prm.nkv : kt) * kBN;
        const CUtensorMap* mk = tt ? &tm_tk : &tm_k;
        const CUtensorMap* mv = tt ? &tm_tv : &tm_v;
        if (j >= SK && !mbar_wait(&k_empty[s], ((j / SK) - 1) & 1, abort, prm.err, LVSA_ERR_DEVICE_TIMEOUT, prm.wait_ns))
          break;
        mbar_expect_tx(&k_full[s], L::kTile);
#pragma unroll
        for (int c = 0; c < L::kCh; ++c)
          tma_load_4d(sK + s * L::kTile + c * kChunk, mk, &k_full[s], c * (128 / L::kElem), hk, ktok, b);
        k_issued = j + 1;
        if (j >= SV && !mbar_wait(&v_empty[sv], ((j / SV) - 1) & 1, abort, prm.err, LVSA_ERR_DEVICE_TIMEOUT, prm.wait_ns))
          break;
        mbar_expect_tx(&v_full[sv], L::kTile);
#pragma unroll
        for (int c = 0; c < L::kCh; ++c)
          tma_load_4d(sV + sv * L::kTile + c * kChunk, mv, &v_full[sv], c * (128 / L::kElem), hk, ktok, b);
        v_issued = j + 1;
      }
      if (*abort) {
        // Drain our own copies still in flight before the CTA retires.
        if (!skip_q) mbar_wait(q_full, 0, never, nullptr, 0);
        for (int j = max(0, k_issued - SK); j < k_issued; ++j)
          mbar_wait(&k_full[j % SK], (j / SK) & 1, never, nullptr, 0);
        for (int j = max(0, v_issued - SV); j < v_issued; ++j)
          mbar_wait(&v_full[j % SV], (j / SV) & 1, never, nullptr, 0);
      }
    }
  } else if (warp == kMmaWarp) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0 && n > 0) {
      // Operand format code 1 means BF16 for kind::f16 but E5M2 for kind::f8f6f4,
      // whose E4M3 code is 0.
      constexpr bool kFmt1 = kBf16 && !kFp8;
      constexpr uint32_t idS = idesc_f16(kBM, kBN, kFmt1, false);
      constexpr uint32_t idO = idesc_f16(kBM, D, kFmt1, true);
      const uint32_t q_base = smem_u32(sQ), k_base = smem_u32(sK), v_base = smem_u32(sV);
      auto issue_s = [&](int jj) {
        const uint32_t kb = k_base + (jj % SK) * L::kTile, dS = tS + (jj % kNB) * 128;
#pragma unroll
        for (int kk = 0; kk < D * L::kElem / 32; ++kk) {  // 32 bytes of Q and K per instruction
          const uint32_t off = (kk >> 2) * kChunk + (kk & 3) * 32;
          mma_ss_any<kFp8>(dS, sdesc_sw128(q_base + off, 16, 1024), sdesc_sw128(kb + off, 16, 1024), idS, kk > 0);
        }
        mma_commit(&s_full[jj % kNB]);
        mma_commit(&k_empty[jj % SK]);
      };
      bool ok = mbar_wait(q_full, 0, abort, prm.err, LVSA_ERR_DEVICE_TIMEOUT, prm.wait_ns) &&
                mbar_wait(&k_full[0], 0, abort, prm.err, LVSA_ERR_DEVICE_TIMEOUT, prm.wait_ns);
      if (ok) {
        tc_fence_after();
        issue_s(0);
      }
      for (int jj = 1; ok && jj < kNB && jj < n; ++jj)
        if ((ok = mbar_wait(&k_full[jj % SK], (jj / SK) & 1, abort, prm.err, LVSA_ERR_DEVICE_TIMEOUT,
                            prm.wait_ns))) {
          tc_fence_after();
          issue_s(jj);
        }
      for (int j = 0; ok && j < n; ++j) {
        const int c = j & 1, it = j >> 1;
        if (!(ok = mbar_wait(&p_full[j % kNB], (j / kNB) & 1, abort, prm.err, LVSA_ERR_DEVICE_TIMEOUT,
                             prm.wait_ns)))
          break;
        if (!(ok = mbar_wait(&v_full[j % SV], (j / SV) & 1, abort, prm.err, LVSA_ERR_DEVICE_TIMEOUT, prm.wait_ns))) break;
        tc_fence_after();
        const uint32_t vb = v_base + (j % SV) * L::kTile, pa = tS + (j % kNB) * 128, dO = tO + c * kOStride;
#pragma unroll
        for (int kk = 0; kk < kBN * L::kElem / 32; ++kk)  // 32 / kElem keys per instruction
          mma_ts_any<kFp8>(dO, pa + kk * 8, sdesc_sw128(vb + kk * (32 / L::kElem) * 128, kChunk, 1024), idO,
                           (it > 0 || kk > 0));
        mma_commit(&v_empty[j % SV]);
        if constexpr (kNB == 3) mma_commit(&pv_done[c]);
        if (j + kNB < n) {
          // S buffer j % kNB: P(j) was read by PV(j), issued just before.
          if (!(ok = mbar_wait(&k_full[(j + kNB) % SK], ((j + kNB) / SK) & 1, abort, prm.err,
                               LVSA_ERR_DEVICE_TIMEOUT, prm.wait_ns)))
            break;
          tc_fence_after();
          issue_s(j + kNB);
        }
      }
      if (ok) mma_commit(o_done);
      // Make sure every MMA this thread issued has retired before TMEM is freed.
      mma_commit(drain);
      mbar_wait(drain, 0, never, nullptr, 0);
    }
  } else {
    // ---------------------------------------------------------- softmax
    const int cls = warp >> 2;                   // tile-list entries j with j % 2 == cls
    const int r = ((warp & 3) << 5) | lane;      // query row = TMEM lane
    const uint32_t pair_bar = 1 + (warp & 3);    // named barrier shared with the other class's warp
    const int seg_len = text_row ? prm.n_text : prm.n_video;
    const int tok = tok0 + r;
    const bool valid = tok < seg_len;
    const int fq = text_row ? 0 : min((prm.tok_off + tok) / prm.P, prm.T - 1);
    const uint32_t* fbits = prm.frame_bits + static_cast<size_t>(fq) * prm.words;
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const float sl2_base = prm.scale_log2;
    float sq = 1.f, vref = 1.f;
    if constexpr (kFp8) {
      sq = text_row ? prm.tqs[(static_cast<int64_t>(b) * prm.heads + h) * prm.nqt_all + (row - prm.nqv)]
                    : prm.qs[(static_cast<int64_t>(b) * prm.heads + h) * prm.nqv + row];
      vref = prm.vref[static_cast<int64_t>(b) * prm.kv_heads + hk];
    }
    constexpr int kPHalf = kFp8 ? 16 : 32;  // TMEM columns of P for 64 keys
    float m = kNegInf, l = 0.f;
    bool ok = true;
    int flag_next = cls < n ? prm.flags[beg + cls] : 0;
    int kt_next = cls < n ? prm.indices[beg + cls] : 0;
    for (int j = cls, it = 0; j < n; j += 2, ++it) {
      const int flag = flag_next, kt = kt_next;
      if (j + 2 < n) {
        flag_next = prm.flags[beg + j + 2];
        kt_next = prm.indices[beg + j + 2];
      }
      float sl2 = sl2_base, pscale = 1.f;  // FP8: dequantise S; fold V's tile scale into P
      if constexpr (kFp8) {
        const int64_t hb = static_cast<int64_t>(b) * prm.kv_heads + hk;
        const bool tt = kt >= prm.nkv;
        const float skj = tt ? prm.tks[hb * prm.nkt + (kt - prm.nkv)] : prm.ks[hb * prm.nkv + kt];
        const float svj = tt ? prm.tvs[hb * prm.nkt + (kt - prm.nkv)] : prm.vs[hb * prm.nkv + kt];
        sl2 = sl2_base * sq * skj;
        pscale = svj / vref;
      }
      uint32_t am[4] = {~0u, ~0u, ~0u, ~0u};
      if (flag) tile_mask(am, prm, kt, text_row, fbits);
      const uint32_t tSc = tS + (j % kNB) * 128 + lane_base;  // this tile's S / P buffer
      if (!__all_sync(0xFFFFFFFFu, mbar_wait(&s_full[j % kNB], (j / kNB) & 1, abort, prm.err,
                                             LVSA_ERR_DEVICE_TIMEOUT, prm.wait_ns))) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t sv[64];
      float mx_hi;
      {
        uint32_t hv[64];
        tmem_ld64x2(tSc, tSc + 64, sv, hv);  // keys 0-63 kept; keys 64-127 only for the max
        if (flag) mask64(hv, am[2], am[3]);
        mx_hi = max64(hv);
      }
      if (flag) mask64(sv, am[0], am[1]);
      const float m_new = fmaxf(m, fmaxf(max64(sv), mx_hi) * sl2);
      if (it == 0) {
        m = m_new;  // my O buffer has not been written yet
      } else {
        // Lazy rescale of my O buffer.  It last received PV(j-2).  With two
        // S buffers that was issued before S(j), so the s_full commit above
        // covers it; with three, S(j) follows PV(j-3): wait for PV(j-2).
        const bool need = m_new > m + kRescaleThreshold;
        if (__any_sync(0xFFFFFFFFu, need)) {
          if constexpr (kNB == 3) {
            if (!__all_sync(0xFFFFFFFFu, mbar_wait(&pv_done[cls], (it - 1) & 1, abort, prm.err,
                                                   LVSA_ERR_DEVICE_TIMEOUT, prm.wait_ns))) {
              ok = false;
              break;
            }
            tc_fence_after();
          }
          const float alpha = need ? ex2_approx(m - m_new) : 1.f;
          if (need) m = m_new;
          const uint32_t tOc = tO + cls * kOStride + lane_base;
#pragma unroll
          for (int c = 0; c < D / 32; ++c) {
            uint32_t t[32];
            tmem_ld32(tOc + c * 32, t);
#pragma unroll
            for (int i = 0; i < 32; ++i) t[i] = __float_as_uint(__uint_as_float(t[i]) * alpha);
            tmem_st32(tOc + c * 32, t);
          }
          l *= alpha;
        }
      }
      const float mu = (m == kNegInf) ? 0.f : m;
      const uint64_t sl2x2 = f2_pack(sl2, sl2), nmu2 = f2_pack(-mu, -mu);
      uint32_t pk[32];
      l += exp64<kBf16, kFp8>(sv, sl2x2, nmu2, pscale, pk);
      store_p<kFp8>(tSc, pk);  // over S columns [0, 32) / [0, 16), already read
      tmem_ld64(tSc + 64, sv);  // keys 64-127
      if (flag) mask64(sv, am[2], am[3]);
      l += exp64<kBf16, kFp8>(sv, sl2x2, nmu2, pscale, pk);
      store_p<kFp8>(tSc + kPHalf, pk);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&p_full[j % kNB]);
    }
    // ---------------------------------------------------------- epilogue
    // Merge the two classes: O = (a0 O0 + a1 O1) / (a0 l0 + a1 l1) with
    // a_c = 2^(m_c - max(m0, m1)).  Each class writes half of the D columns.
    using Elem = typename std::conditional<kBf16, __nv_bfloat16, __half>::type;
    Elem* obase = nullptr;
    float* lse = nullptr;
    if (text_row) {
      if (prm.text_o)
        obase = reinterpret_cast<Elem*>(prm.text_o) + b * prm.to_sb + static_cast<int64_t>(tok) * prm.to_st +
                h * prm.to_sh;
      if (prm.text_lse) lse = prm.text_lse + (static_cast<int64_t>(b) * prm.heads + h) * prm.n_text + tok;
    } else {
      obase = reinterpret_cast<Elem*>(prm.o) + b * prm.o_sb + static_cast<int64_t>(tok) * prm.o_st + h * prm.o_sh;
      if (prm.lse) lse = prm.lse + (static_cast<int64_t>(b) * prm.heads + h) * prm.n_video + tok;
    }
    if (obase) obase += cls * (D / 2);
    if (n > 0) {
      const bool got =
          ok && __all_sync(0xFFFFFFFFu, mbar_wait(o_done, 0, abort, prm.err, LVSA_ERR_DEVICE_TIMEOUT, prm.wait_ns));
      // After o_done no MMA reads the query tile any more: reuse it.
      float* red_m = reinterpret_cast<float*>(sQ);   // [2 classes][128 rows]
      float* red_l = red_m + 2 * kBM;                // NaN marks a class that timed out
      red_m[cls * kBM + r] = m;
      red_l[cls * kBM + r] = got ? l : __int_as_float(0x7FC00000);
      asm volatile("bar.sync %0, 64;" ::"r"(pair_bar) : "memory");
      const float m_o = red_m[(cls ^ 1) * kBM + r], l_o = red_l[(cls ^ 1) * kBM + r];
      if (__all_sync(0xFFFFFFFFu, got && !isnan(l_o))) {
        tc_fence_after();
        const float mm = fmaxf(m, m_o);
        const float a_me = (m == kNegInf) ? 0.f : ex2_approx(m - mm);
        const float a_ot = (m_o == kNegInf) ? 0.f : ex2_approx(m_o - mm);
        const float lt = l * a_me + l_o * a_ot;
        const float inv = (lt > 0.f) ? vref / lt : 0.f;
        const float s0 = (cls == 0 ? a_me : a_ot) * inv, s1 = (cls == 1 ? a_me : a_ot) * inv;
        const bool use1 = n > 1;  // O buffer 1 is written only when the list has two or more tiles
#pragma unroll
        for (int c = 0; c < D / 64; ++c) {
          const uint32_t col = cls * (D / 2) + c * 32;
          uint32_t t0[32], t1[32];
          tmem_ld32(tO + lane_base + col, t0);
          if (use1) tmem_ld32(tO + kOStride + lane_base + col, t1);
          if (valid && obase) {
            uint32_t pk[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              float x0 = __uint_as_float(t0[2 * i]) * s0, x1 = __uint_as_float(t0[2 * i + 1]) * s0;
              if (use1) {
                x0 = fmaf(__uint_as_float(t1[2 * i]), s1, x0);
                x1 = fmaf(__uint_as_float(t1[2 * i + 1]), s1, x1);
              }
              pk[i] = pack2(x0, x1, kBf16);
            }
            uint4* dst = reinterpret_cast<uint4*>(obase + c * 32);
#pragma unroll
            for (int i = 0; i < 4; ++i) dst[i] = make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
          }
        }
        if (valid && lse && cls == 0) *lse = (lt > 0.f) ? (mm + __log2f(lt)) * 0.69314718055994531f : kNegInf;
      }
    } else if (valid) {
      if (obase) {
        uint4* dst = reinterpret_cast<uint4*>(obase);
#pragma unroll
        for (int i = 0; i < D / 16; ++i) dst[i] = make_uint4(0u, 0u, 0u, 0u);
      }
      if (lse && cls == 0) *lse = kNegInf;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ------------------------------------------------------------------ tile pairs
// Two consecutive query tiles of one segment per CTA (same head, batch).
// Class c (warps 4c .. 4c+3) owns query tile c of the pair with its own tile
// list, S/P buffer, O accumulator and running max; nothing is merged.  Step i
// of the CTA is entry i of both lists: when the two entries name the same key
// tile (every step for two tiles of one frame) it is loaded once and read by
// both classes' MMAs, which halves the L2 -> shared-memory traffic per
// computed tile; otherwise each class's tile is loaded on its own.  The load
// sequence (index g) is a function of the two lists, walked identically by
// the producer and the MMA issuer.  MMA order: S_0(0) S_1(0), then per step i
// PV_0(i) S_0(i+1) PV_1(i) S_1(i+1) -- the same two interleaved chains as the
// single-tile kernel.
template <int D, int SK, int SV, bool kFp8 = false>
struct SmemPair {
  static constexpr int kElem = kFp8 ? 1 : 2;
  static constexpr int kCh = D * kElem / 128;
  static constexpr int kTile = kCh * kChunk;
  static constexpr int kQ = 0;  // two query tiles
  static constexpr int kK = kQ + 2 * kTile;
  static constexpr int kV = kK + SK * kTile;
  static constexpr int kBar = kV + SV * kTile;
  static constexpr int kNumBars = 2 * SK + 2 * SV + 8;
  static constexpr int kMisc = kBar + kNumBars * 8;
  static constexpr int kBytes = kMisc + 16 + 1024;
  static_assert(kBytes <= 232448, "shared memory");
};

// Loads of step i: g0 / g1 = load index read by class 0 / 1 (-1: the class has
// no entry i); shared when both read one load.
struct PairStep {
  int g0, g1;
  bool shared;
};
__device__ __forceinline__ PairStep pair_step(int i, const int32_t* l0, int n0, const int32_t* l1, int n1, int& gc) {
  PairStep s;
  s.g0 = i < n0 ? gc++ : -1;
  s.shared = i < n0 && i < n1 && l0[i] == l1[i];
  s.g1 = i < n1 ? (s.shared ? s.g0 : gc++) : -1;
  return s;
}

template <int D, int SK, int SV, bool kBf16, bool kFp8 = false>
__global__ void __launch_bounds__(kThreads, 1)
    lvsa_attn_pair_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                          const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_tq,
                          const __grid_constant__ CUtensorMap tm_tk, const __grid_constant__ CUtensorMap tm_tv,
                          const AttnParams prm) {
  using L = SmemPair<D, SK, SV, kFp8>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem + L::kQ;
  uint8_t* sK = smem + L::kK;
  uint8_t* sV = smem + L::kV;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBar);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* v_full = k_full + SK;
  uint64_t* k_empty = v_full + SV;
  uint64_t* v_empty = k_empty + SK;
  uint64_t* s_full = v_empty + SV;  // [2] per class
  uint64_t* p_full = s_full + 2;    // [2] per class
  uint64_t* o_done = p_full + 2;
  uint64_t* drain = o_done + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kMisc);
  volatile int* abort = reinterpret_cast<volatile int*>(smem + L::kMisc + 4);
  volatile int* never = reinterpret_cast<volatile int*>(smem + L::kMisc + 8);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  LVSA_CLK(t_cta0);
  const int h = blockIdx.y, b = blockIdx.z;
  // Pairs of video rows [row0, pair_ve), then pairs of text rows [pair_ts, pair_end).
  // Text pairs (dense rows, the longest CTAs) take the first block indices.
  const int x = (LVSA_TEXT_FIRST && static_cast<int>(gridDim.x) > prm.pair_nv)
                    ? static_cast<int>((blockIdx.x + prm.pair_nv) % gridDim.x)
                    : static_cast<int>(blockIdx.x);
  const bool text_row = x >= prm.pair_nv;
  const int row_a = text_row ? prm.pair_ts + 2 * (x - prm.pair_nv) : prm.row0 + 2 * x;
  const bool has_b = row_a + 1 < (text_row ? prm.pair_end : prm.pair_ve);
  const int beg0 = prm.indptr[row_a], n0 = prm.indptr[row_a + 1] - beg0;
  const int beg1 = has_b ? prm.indptr[row_a + 1] : 0, n1 = has_b ? prm.indptr[row_a + 2] - beg1 : 0;
  const int32_t* l0 = prm.indices + beg0;
  const int32_t* l1 = prm.indices + beg1;
  const int nmax = max(n0, n1);
  const int tok_a = (text_row ? row_a - prm.nqv : row_a) * kBM;
  const int hk = h / (prm.heads / prm.kv_heads);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < SK; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
    }
    for (int s = 0; s < SV; ++s) {
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 128);
    }
    mbar_init(o_done, 1);
    mbar_init(drain, 1);
    *abort = 0;
    *never = 0;
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem, tO = tmem + 256;

  if (warp == kProducerWarp) {
    // ---------------------------------------------------------- producer
    if (lane == 0 && nmax > 0) {
      const CUtensorMap* mq = text_row ? &tm_tq : &tm_q;
      tma_prefetch_desc(mq);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      const bool skip_q = prm.inject && (blockIdx.x | blockIdx.y | blockIdx.z) == 0;
      if (!skip_q) {
        mbar_expect_tx(q_full, (has_b ? 2 : 1) * L::kTile);
        for (int t = 0; t < (has_b ? 2 : 1); ++t)
#pragma unroll
          for (int c = 0; c < L::kCh; ++c)
            tma_load_4d(sQ + t * L::kTile + c * kChunk, mq, q_full, c * (128 / L::kElem), h, tok_a + t * kBM, b);
      }
      int gc = 0, issued = 0;
      bool ok = true;
      for (int i = 0; ok && i < nmax; ++i) {
        const PairStep st = pair_step(i, l0, n0, l1, n1, gc);
        for (int t = 0; t < 2; ++t) {
          const int g = t == 0 ? st.g0 : (st.shared ? -1 : st.g1);
          if (g < 0) continue;
          const int kt = t == 0 ? l0[i] : l1[i];
          const int s = g % SK, sv = g % SV;
          const bool tt = kt >= prm.nkv;
          const int ktok = (tt ? kt - prm.nkv : kt) * kBN;
          const CUtensorMap* mk = tt ? &tm_tk : &tm_k;
          const CUtensorMap* mv = tt ? &tm_tv : &tm_v;
          if (g >= SK && !(ok = mbar_wait(&k_empty[s], ((g / SK) - 1) & 1, abort, prm.err, LVSA_ERR_DEVICE_TIMEOUT, prm.wait_ns)))
            break;
          mbar_expect_tx(&k_full[s], L::kTile);
#pragma unroll
          for (int c = 0; c < L::kCh; ++c)
            tma_load_4d(sK + s * L::kTile + c * kChunk, mk, &k_full[s], c * (128 / L::kElem), hk, ktok, b);
          if (g >= SV && !(ok = mbar_wait(&v_empty[sv], ((g / SV) - 1) & 1, abort, prm.err, LVSA_ERR_DEVICE_TIMEOUT, prm.wait_ns))) {
            issued = -(g + 1);  // K of load g issued, V not
            break;
          }
          mbar_expect_tx(&v_full[sv], L::kTile);
#pragma unroll
          for (int c = 0; c < L::kCh; ++c)
            tma_load_4d(sV + sv * L::kTile + c * kChunk, mv, &v_full[sv], c * (128 / L::kElem), hk, ktok, b);
          issued = g + 1;
        }
      }
      if (*abort) {
        // Drain our own copies still in flight before the CTA retires.
        const int k_issued = issued < 0 ? -issued : issued, v_issued = issued < 0 ? -issued - 1 : issued;
        if (!skip_q) mbar_wait(q_full, 0, never, nullptr, 0);
        for (int g = max(0, k_issued - SK); g < k_issued; ++g)
          mbar_wait(&k_full[g % SK], (g / SK) & 1, never, nullptr, 0);
        for (int g = max(0, v_issued - SV); g < v_issued; ++g)
          mbar_wait(&v_full[g % SV], (g / SV) & 1, never, nullptr, 0);
      }
    }
  } else if (warp == kMmaWarp) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0 && nmax > 0) {
      constexpr bool kFmt1 = kBf16 && !kFp8;
      constexpr uint32_t idS = idesc_f16(kBM, kBN, kFmt1, false);
      constexpr uint32_t idO = idesc_f16(kBM, D, kFmt1, true);
      const uint32_t q_base = smem_u32(sQ), k_base = smem_u32(sK), v_base = smem_u32(sV);
      const int nc[2] = {n0, n1};
      // S_c(i) from load g; `last`: no later S reads that K stage.
      auto issue_s = [&](int c, int g, bool last) -> bool {
        LVSA_CLK(t_k0);
        if (!mbar_wait(&k_full[g % SK], (g / SK) & 1, abort, prm.err, LVSA_ERR_DEVICE_TIMEOUT, prm.wait_ns)) return false;
        LVSA_CLK(t_k1);
        LVSA_PROF_ADD(4, t_k1 - t_k0);
        tc_fence_after();
        const uint32_t kb = k_base + (g % SK) * L::kTile, qb = q_base + c * L::kTile, dS = tS + c * 128;
#pragma unroll
        for (int kk = 0; kk < D * L::kElem / 32; ++kk) {
          const uint32_t off = (kk >> 2) * kChunk + (kk & 3) * 32;
          mma_ss_any<kFp8>(dS, sdesc_sw128(qb + off, 16, 1024), sdesc_sw128(kb + off, 16, 1024), idS, kk > 0);
        }
        mma_commit(&s_full[c]);
        if (last) mma_commit(&k_empty[g % SK]);
        return true;
      };
      auto issue_pv = [&](int c, int i, int g, bool last) -> bool {
        LVSA_CLK(t_p0);
        if (!mbar_wait(&p_full[c], i & 1, abort, prm.err, LVSA_ERR_DEVICE_TIMEOUT, prm.wait_ns)) return false;
        LVSA_CLK(t_p1);
        if (!mbar_wait(&v_full[g % SV], (g / SV) & 1, abort, prm.err, LVSA_ERR_DEVICE_TIMEOUT, prm.wait_ns)) return false;
        LVSA_CLK(t_p2);
        LVSA_PROF_ADD(2, t_p1 - t_p0);
        LVSA_PROF_ADD(3, t_p2 - t_p1);
        tc_fence_after();
        const uint32_t vb = v_base + (g % SV) * L::kTile, pa = tS + c * 128, dO = tO + c * 128;
#pragma unroll
        for (int kk = 0; kk < kBN * L::kElem / 32; ++kk)
          mma_ts_any<kFp8>(dO, pa + kk * 8, sdesc_sw128(vb + kk * (32 / L::kElem) * 128, kChunk, 1024), idO,
                           (i > 0 || kk > 0));
        if (last) mma_commit(&v_empty[g % SV]);
        return true;
      };
      bool ok = mbar_wait(q_full, 0, abort, prm.err, LVSA_ERR_DEVICE_TIMEOUT, prm.wait_ns);
      int gc = 0;
      PairStep cur = pair_step(0, l0, n0, l1, n1, gc);
      if (ok && cur.g0 >= 0) ok = issue_s(0, cur.g0, !cur.shared);
      if (ok && cur.g1 >= 0) ok = issue_s(1, cur.g1, true);
      for (int i = 0; ok && i < nmax; ++i) {
        PairStep nxt = {-1, -1, false};
        if (i + 1 < nmax) nxt = pair_step(i + 1, l0, n0, l1, n1, gc);
        for (int c = 0; ok && c < 2; ++c) {
          if (i >= nc[c]) continue;
          // PV_c(i); class 0 leaves a shared V stage to class 1.
          ok = issue_pv(c, i, c == 0 ? cur.g0 : cur.g1, c == 1 || !cur.shared);
          // S_c(i+1) reuses buffer c: P_c(i) was read by PV_c(i), issued just before.
          if (ok && i + 1 < nc[c]) ok = issue_s(c, c == 0 ? nxt.g0 : nxt.g1, c == 1 || !nxt.shared);
        }
        cur = nxt;
      }
      if (ok) mma_commit(o_done);
      mma_commit(drain);
      mbar_wait(drain, 0, never, nullptr, 0);
    }
  } else {
    // ---------------------------------------------------------- softmax
    const int cls = warp >> 2;                // query tile of the pair
    const int r = ((warp & 3) << 5) | lane;   // query row = TMEM lane
    const int row = row_a + cls;
    const int beg = cls ? beg1 : beg0, n = cls ? n1 : n0;
    const bool mine = cls == 0 || has_b;
    const int seg_len = text_row ? prm.n_text : prm.n_video;
    const int tok = tok_a + cls * kBM + r;
    const bool valid = mine && tok < seg_len;
    const int fq = text_row ? 0 : min((prm.tok_off + tok) / prm.P, prm.T - 1);
    const uint32_t* fbits = prm.frame_bits + static_cast<size_t>(fq) * prm.words;
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t tSc = tS + cls * 128 + lane_base;
    const uint32_t tOc = tO + cls * 128 + lane_base;
    const float sl2_base = prm.scale_log2;
    float sq = 1.f, vref = 1.f;
    if constexpr (kFp8) {
      if (mine) {
        sq = text_row ? prm.tqs[(static_cast<int64_t>(b) * prm.heads + h) * prm.nqt_all + (row - prm.nqv)]
                      : prm.qs[(static_cast<int64_t>(b) * prm.heads + h) * prm.nqv + row];
        vref = prm.vref[static_cast<int64_t>(b) * prm.kv_heads + hk];
      }
    }
    constexpr int kPHalf = kFp8 ? 16 : 32;
    float m = kNegInf, l = 0.f;
    bool ok = true;
    int flag_next = n > 0 ? prm.flags[beg] : 0;
    int kt_next = n > 0 ? prm.indices[beg] : 0;
    for (int it = 0; it < n; ++it) {
      const int flag = flag_next, kt = kt_next;
      if (it + 1 < n) {
        flag_next = prm.flags[beg + it + 1];
        kt_next = prm.indices[beg + it + 1];
      }
      float sl2 = sl2_base, pscale = 1.f;
      if constexpr (kFp8) {
        const int64_t hb = static_cast<int64_t>(b) * prm.kv_heads + hk;
        const bool tt = kt >= prm.nkv;
        const float skj = tt ? prm.tks[hb * prm.nkt + (kt - prm.nkv)] : prm.ks[hb * prm.nkv + kt];
        const float svj = tt ? prm.tvs[hb * prm.nkt + (kt - prm.nkv)] : prm.vs[hb * prm.nkv + kt];
        sl2 = sl2_base * sq * skj;
        pscale = svj / vref;
      }
      uint32_t am[4] = {~0u, ~0u, ~0u, ~0u};
      if (flag) tile_mask(am, prm, kt, text_row, fbits);
      LVSA_CLK(t_w0);
      if (!__all_sync(0xFFFFFFFFu, mbar_wait(&s_full[cls], it & 1, abort, prm.err, LVSA_ERR_DEVICE_TIMEOUT, prm.wait_ns))) {
        ok = false;
        break;
      }
      LVSA_CLK(t_w1);
      if (lane == 0) LVSA_PROF_ADD(0, t_w1 - t_w0);
      tc_fence_after();
      uint32_t sv[64];
      float mx_hi;
      {
        uint32_t hv[64];
        tmem_ld64x2(tSc, tSc + 64, sv, hv);
        if (flag) mask64(hv, am[2], am[3]);
        mx_hi = max64(hv);
      }
      if (flag) mask64(sv, am[0], am[1]);
      const float m_new = fmaxf(m, fmaxf(max64(sv), mx_hi) * sl2);
      if (it == 0) {
        m = m_new;
      } else {
        // Lazy rescale of my O buffer: PV_c(it-1) was issued before S_c(it).
        const bool need = m_new > m + kRescaleThreshold;
        if (__any_sync(0xFFFFFFFFu, need)) {
          const float alpha = need ? ex2_approx(m - m_new) : 1.f;
          if (need) m = m_new;
#pragma unroll
          for (int c = 0; c < D / 32; ++c) {
            uint32_t t[32];
            tmem_ld32(tOc + c * 32, t);
#pragma unroll
            for (int i = 0; i < 32; ++i) t[i] = __float_as_uint(__uint_as_float(t[i]) * alpha);
            tmem_st32(tOc + c * 32, t);
          }
          l *= alpha;
        }
      }
      const float mu = (m == kNegInf) ? 0.f : m;
      const uint64_t sl2x2 = f2_pack(sl2, sl2), nmu2 = f2_pack(-mu, -mu);
      uint32_t pk[32];
      l += exp64<kBf16, kFp8>(sv, sl2x2, nmu2, pscale, pk);
      store_p<kFp8>(tSc, pk);
      tmem_ld64(tSc + 64, sv);
      if (flag) mask64(sv, am[2], am[3]);
      l += exp64<kBf16, kFp8>(sv, sl2x2, nmu2, pscale, pk);
      store_p<kFp8>(tSc + kPHalf, pk);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&p_full[cls]);
      LVSA_CLK(t_w2);
      if (lane == 0) {
        LVSA_PROF_ADD(1, t_w2 - t_w1);
        LVSA_PROF_ADD(5, 1);
      }
    }
    // ---------------------------------------------------------- epilogue
    using Elem = typename std::conditional<kBf16, __nv_bfloat16, __half>::type;
    Elem* obase = nullptr;
    float* lse = nullptr;
    if (text_row) {
      if (prm.text_o)
        obase = reinterpret_cast<Elem*>(prm.text_o) + b * prm.to_sb + static_cast<int64_t>(tok) * prm.to_st +
                h * prm.to_sh;
      if (prm.text_lse) lse = prm.text_lse + (static_cast<int64_t>(b) * prm.heads + h) * prm.n_text + tok;
    } else {
      obase = reinterpret_cast<Elem*>(prm.o) + b * prm.o_sb + static_cast<int64_t>(tok) * prm.o_st + h * prm.o_sh;
      if (prm.lse) lse = prm.lse + (static_cast<int64_t>(b) * prm.heads + h) * prm.n_video + tok;
    }
    if (n > 0) {
      const bool got =
          ok && __all_sync(0xFFFFFFFFu, mbar_wait(o_done, 0, abort, prm.err, LVSA_ERR_DEVICE_TIMEOUT, prm.wait_ns));
      if (got) {
        tc_fence_after();
        const float inv = (l > 0.f) ? vref / l : 0.f;
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t t[32];
          tmem_ld32(tOc + c * 32, t);
          if (valid && obase) {
            uint32_t pk[16];
#pragma unroll
            for (int i = 0; i < 16; ++i)
              pk[i] = pack2(__uint_as_float(t[2 * i]) * inv, __uint_as_float(t[2 * i + 1]) * inv, kBf16);
            uint4* dst = reinterpret_cast<uint4*>(obase + c * 32);
#pragma unroll
            for (int i = 0; i < 4; ++i) dst[i] = make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
          }
        }
        if (valid && lse) *lse = (l > 0.f) ? (m + __log2f(l)) * 0.69314718055994531f : kNegInf;
      }
    } else if (valid) {
      if (obase) {
        uint4* dst = reinterpret_cast<uint4*>(obase);
#pragma unroll
        for (int i = 0; i < D / 8; ++i) dst[i] = make_uint4(0u, 0u, 0u, 0u);
      }
      if (lse) *lse = kNegInf;
    }
  }

  tc_fence_before();
  __syncthreads();
  LVSA_CLK(t_cta1);
  if (threadIdx.x == 0) {
    LVSA_PROF_ADD(6, t_cta1 - t_cta0);
    LVSA_PROF_ADD(7, 1);
  }
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ------------------------------------------------------------------ host side
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn() {
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

// [B, N, Hx, D] view -> 4-D map (D, Hx, N, B) with a (128 bytes, 1, 128, 1)
// box, 128B swizzle.  dt: LVSA_DTYPE_BF16 / _F16 / _E4M3.
int make_map(CUtensorMap* map, const LvsaTensor& t, int B, int N, int Hx, int D, int dt) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return LVSA_ERR_CUDA;
  if (!t.ptr || N < 1) return LVSA_ERR_INVALID_ARG;
  const int64_t es = dt == LVSA_DTYPE_E4M3 ? 1 : 2;
  if ((reinterpret_cast<uintptr_t>(t.ptr) & 15) || (t.stride_h * es) % 16 || (t.stride_t * es) % 16 ||
      (B > 1 && (t.stride_b * es) % 16))
    return LVSA_ERR_ALIGNMENT;
  if (t.stride_h < D || t.stride_t < 1) return LVSA_ERR_INVALID_ARG;
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(Hx), static_cast<cuuint64_t>(N),
                        static_cast<cuuint64_t>(B)};
  const int64_t sb = (B > 1) ? t.stride_b : t.stride_t * N;
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(t.stride_h * es), static_cast<cuuint64_t>(t.stride_t * es),
                           static_cast<cuuint64_t>(sb * es)};
  cuuint32_t box[4] = {static_cast<cuuint32_t>(128 / es), 1, static_cast<cuuint32_t>(kBM), 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUtensorMapDataType ty = dt == LVSA_DTYPE_E4M3 ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                 : dt == LVSA_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                         : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = enc(map, ty, 4, t.ptr, dims,
                   strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? LVSA_OK : LVSA_ERR_ALIGNMENT;
}

template <int D, int SK, int SV, bool kBf16_, bool kFp8 = false, bool kPair = false>
int launch(const LvsaAttnArgs* a, cudaStream_t stream, const LvsaFp8Scales* sc = nullptr) {
  CUtensorMap mq, mk, mv, mtq, mtk, mtv;
  int st;
  const int dt = kFp8 ? LVSA_DTYPE_E4M3 : (kBf16_ ? LVSA_DTYPE_BF16 : LVSA_DTYPE_F16);
  if ((st = make_map(&mq, a->q, a->batch, a->n_video, a->heads, D, dt))) return st;
  const int n_kv = a->n_kv_video > 0 ? a->n_kv_video : a->n_video;
  if ((st = make_map(&mk, a->k, a->batch, n_kv, a->kv_heads, D, dt))) return st;
  if ((st = make_map(&mv, a->v, a->batch, n_kv, a->kv_heads, D, dt))) return st;
  const bool text_rows = a->n_text > 0 && a->text_q.ptr != nullptr;
  if (a->n_text > 0) {
    if ((st = make_map(&mtk, a->text_k, a->batch, a->n_text, a->kv_heads, D, dt))) return st;
    if ((st = make_map(&mtv, a->text_v, a->batch, a->n_text, a->kv_heads, D, dt))) return st;
  } else {
    mtk = mk;
    mtv = mv;
  }
  if (text_rows) {
    if ((st = make_map(&mtq, a->text_q, a->batch, a->n_text, a->heads, D, dt))) return st;
  } else {
    mtq = mq;
  }
  AttnParams p;
  p.q = a->q.ptr;
  p.text_q = text_rows ? a->text_q.ptr : nullptr;
  p.q_sb = a->q.stride_b; p.q_st = a->q.stride_t; p.q_sh = a->q.stride_h;
  p.tq_sb = a->text_q.stride_b; p.tq_st = a->text_q.stride_t; p.tq_sh = a->text_q.stride_h;
  p.o = a->o.ptr;
  p.text_o = text_rows ? a->text_o.ptr : nullptr;
  p.lse = a->lse;
  p.text_lse = text_rows ? a->text_lse : nullptr;
  p.o_sb = a->o.stride_b; p.o_st = a->o.stride_t; p.o_sh = a->o.stride_h;
  p.to_sb = a->text_o.stride_b; p.to_st = a->text_o.stride_t; p.to_sh = a->text_o.stride_h;
  p.n_video = a->n_video; p.n_kv = n_kv; p.n_text = a->n_text; p.heads = a->heads; p.kv_heads = a->kv_heads;
  p.T = a->total_frames; p.P = a->num_patches; p.words = a->frame_words;
  p.nqv = a->n_q_video_tiles; p.nkv = a->n_k_video_tiles;
  const float scale = a->scale > 0.f ? a->scale : 1.0f / std::sqrt(static_cast<float>(D));
  p.scale_log2 = scale * 1.4426950408889634f;
  p.frame_bits = a->frame_bits; p.indptr = a->tile_indptr; p.indices = a->tile_indices; p.flags = a->tile_flags;
  p.err = a->error_word;
  p.wait_ns = a->wait_timeout_us > 0 ? static_cast<uint64_t>(a->wait_timeout_us) * 1000ull : kWaitTimeoutNs;
  p.inject = a->inject_fault;
  p.qs = p.ks = p.vs = p.tqs = p.tks = p.tvs = p.vref = nullptr;
  p.nqt_all = (a->n_text + kBlockQ - 1) / kBlockQ;
  p.nkt = (a->n_text + kBN - 1) / kBN;
  if (kFp8) {
    if (!sc || !sc->q || !sc->k || !sc->v || !sc->v_ref) return LVSA_ERR_INVALID_ARG;
    if (a->n_text > 0 && (!sc->text_k || !sc->text_v || (text_rows && !sc->text_q))) return LVSA_ERR_INVALID_ARG;
    p.qs = sc->q; p.ks = sc->k; p.vs = sc->v; p.tqs = sc->text_q; p.tks = sc->text_k; p.tvs = sc->text_v;
    p.vref = sc->v_ref;
  }

  p.tok_off = a->token_offset;
  p.row0 = a->first_q_tile;
  const int end = std::min(text_rows ? a->n_q_tiles : a->n_q_video_tiles,
                           a->end_q_tile > 0 ? a->end_q_tile : a->n_q_tiles);
  const int rows = end - a->first_q_tile;
  if (rows <= 0) return LVSA_OK;
  p.pair_end = end;
  p.pair_ve = std::min(end, a->n_q_video_tiles);
  p.pair_ts = std::max(a->first_q_tile, a->n_q_video_tiles);
  p.pair_nv = p.pair_ve > p.row0 ? (p.pair_ve - p.row0 + 1) / 2 : 0;
  if constexpr (kPair) {
    using L = SmemPair<D, SK, SV, kFp8>;
    auto kern = lvsa_attn_pair_kernel<D, SK, SV, kBf16_, kFp8>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes) != cudaSuccess)
      return LVSA_ERR_CUDA;
    const int pair_nt = end > p.pair_ts ? (end - p.pair_ts + 1) / 2 : 0;
    dim3 grid(p.pair_nv + pair_nt, a->heads, a->batch);
    kern<<<grid, kThreads, L::kBytes, stream>>>(mq, mk, mv, mtq, mtk, mtv, p);
  } else {
    using L = Smem<D, SK, SV, kFp8>;
    auto kern = lvsa_attn_kernel<D, SK, SV, kBf16_, kFp8>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes) != cudaSuccess)
      return LVSA_ERR_CUDA;
    dim3 grid(rows, a->heads, a->batch);
    kern<<<grid, kThreads, L::kBytes, stream>>>(mq, mk, mv, mtq, mtk, mtv, p);
  }
  return cudaGetLastError() == cudaSuccess ? LVSA_OK : LVSA_ERR_CUDA;
}

}  // namespace
}  // namespace lvsa

namespace lvsa {
namespace {
int validate(const LvsaAttnArgs* a) {
  if (!a || !a->q.ptr || !a->k.ptr || !a->v.ptr || !a->o.ptr || !a->frame_bits || !a->tile_indptr ||
      !a->tile_indices || !a->tile_flags)
    return LVSA_ERR_INVALID_ARG;
  if (a->batch < 1 || a->n_video < 1 || a->n_text < 0 || a->heads < 1 || a->kv_heads < 1 ||
      a->heads % a->kv_heads)
    return LVSA_ERR_INVALID_ARG;
  if (a->block_q != kBlockQ || a->block_k != kBN) return LVSA_ERR_UNSUPPORTED;
  // The video segment is the T x P grid or, for a sequence shard, the token
  // range [token_offset, token_offset + n_video) inside it.
  const long long grid_tokens = static_cast<long long>(a->total_frames) * a->num_patches;
  if (a->total_frames < 1 || a->num_patches < 1 || a->token_offset < 0 ||
      a->token_offset + static_cast<long long>(a->n_video) > grid_tokens)
    return LVSA_ERR_GEOMETRY;
  if (a->first_q_tile < 0 || a->first_q_tile > a->n_q_tiles) return LVSA_ERR_INVALID_ARG;
  if (a->end_q_tile > 0 && (a->end_q_tile < a->first_q_tile || a->end_q_tile > a->n_q_tiles))
    return LVSA_ERR_INVALID_ARG;
  const long long n_kv = a->n_kv_video > 0 ? a->n_kv_video : a->n_video;
  if (a->n_kv_video < 0 || a->token_offset + n_kv > grid_tokens) return LVSA_ERR_GEOMETRY;
  if (a->n_q_video_tiles != (a->n_video + kBlockQ - 1) / kBlockQ || a->n_k_video_tiles != (n_kv + kBN - 1) / kBN ||
      a->frame_words != (a->total_frames + 31) / 32)
    return LVSA_ERR_GEOMETRY;
  if (a->n_text > 0 && (!a->text_k.ptr || !a->text_v.ptr)) return LVSA_ERR_INVALID_ARG;
  if (a->n_text > 0 && a->text_q.ptr && !a->text_o.ptr) return LVSA_ERR_INVALID_ARG;
  if (a->n_text > 0 && a->n_q_tiles != a->n_q_video_tiles + (a->n_text + kBlockQ - 1) / kBlockQ) return LVSA_ERR_GEOMETRY;
  return LVSA_OK;
}
}  // namespace

// bf16/f16 at D = 128: the tile-pair kernel (two query tiles per CTA share
// their K/V loads) when its grid holds at least LVSA_PAIR_MIN_WAVES waves of
// CTAs, else the single-tile kernel, whose CTAs are half as long and so
// leave half the last-wave tail.  Measured (ms per launch): cfg2, 12 heads,
// 40 waves: pair 32.25 vs single 32.61; cfg4 with 2 heads (one rank's share
// on 8 GPUs), 4.1 waves: pair 2.52 vs single 2.30.  LVSA_ATTN_KERNEL=pair /
// single in the environment forces one (tests).
#ifndef LVSA_PAIR_MIN_WAVES
#define LVSA_PAIR_MIN_WAVES 16
#endif
bool use_pair_kernel(const LvsaAttnArgs* a) {
  if (const char* e = std::getenv("LVSA_ATTN_KERNEL")) {
    if (!std::strcmp(e, "pair")) return true;
    if (!std::strcmp(e, "single")) return false;
  }
  const bool text_rows = a->n_text > 0 && a->text_q.ptr != nullptr;
  const int end = std::min(text_rows ? a->n_q_tiles : a->n_q_video_tiles,
                           a->end_q_tile > 0 ? a->end_q_tile : a->n_q_tiles);
  const int first = a->first_q_tile, nqv = a->n_q_video_tiles;
  const int ve = std::min(end, nqv), ts = std::max(first, nqv);
  const long long pairs = (ve > first ? (ve - first + 1) / 2 : 0) + (end > ts ? (end - ts + 1) / 2 : 0);
  const long long ctas = pairs * a->heads * a->batch;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return ctas >= static_cast<long long>(LVSA_PAIR_MIN_WAVES) * sms;
}

// The argument and geometry checks of lvsa_attn_fwd / lvsa_attn_fwd_fp8, for
// entry points that must reject a call before they launch anything.
int validate_attn_args(const LvsaAttnArgs* a) { return validate(a); }
}  // namespace lvsa

extern "C" int lvsa_attn_fwd(const LvsaAttnArgs* a, void* stream) {
  using namespace lvsa;
  const int v = validate(a);
  if (v != LVSA_OK) return v;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool bf16 = a->dtype == LVSA_DTYPE_BF16;
  if (a->dtype != LVSA_DTYPE_BF16 && a->dtype != LVSA_DTYPE_F16) return LVSA_ERR_UNSUPPORTED;
  switch (a->head_dim) {
// Kernel choice and K / V ring depths (K stages free after their S MMA, V
// stages after their PV MMA), measured in a 10-launch loop:
//  * D = 128, bf16/f16: the tile-pair kernel with 3 K + 2 V stages, 32.25
//    ms/layer on cfg2 against 32.61-32.73 for the single-tile kernel on the
//    same GPU (2 + 2: 32.39, 2 + 3: 32.34).  Single-tile ring: 4 K + 2 V
//    stages 32.07 (another GPU), 3 + 3 32.42, 2 + 4 32.65, 5 + 1 47.8 --
//    K(j+2) is on its critical chain (S(j+2) is issued right after PV(j)).
//  * D = 64 and FP8 (16 KB tiles): the single-tile kernel with 6 + 6 stages
//    (within noise of 8 + 5, 9 + 4 and 10 + 3).  The tile-pair kernel was
//    slower there: cfg5 37.84-38.12 vs 37.28, FP8 cfg2 28.87-29.02 vs 27.86
//    (LVSA_PAIR64 / LVSA_PAIR8 = 1 select it).
#ifndef LVSA_SK
#define LVSA_SK 4
#define LVSA_SV 2
#endif
#ifndef LVSA_SK64
#define LVSA_SK64 6
#define LVSA_SV64 6
#endif
#ifndef LVSA_PAIR
#define LVSA_PAIR 1
#define LVSA_SKP 3
#define LVSA_SVP 2
#endif
#if LVSA_PAIR
    case 128:
      if (use_pair_kernel(a))
        return bf16 ? launch<128, LVSA_SKP, LVSA_SVP, true, false, true>(a, s)
                    : launch<128, LVSA_SKP, LVSA_SVP, false, false, true>(a, s);
      return bf16 ? launch<128, LVSA_SK, LVSA_SV, true>(a, s) : launch<128, LVSA_SK, LVSA_SV, false>(a, s);
#else
    case 128: return bf16 ? launch<128, LVSA_SK, LVSA_SV, true>(a, s) : launch<128, LVSA_SK, LVSA_SV, false>(a, s);
#endif
#ifndef LVSA_PAIR64
#define LVSA_PAIR64 0
#define LVSA_SKP64 6
#define LVSA_SVP64 6
#endif
#if LVSA_PAIR64
    case 64: return bf16 ? launch<64, LVSA_SKP64, LVSA_SVP64, true, false, true>(a, s)
                         : launch<64, LVSA_SKP64, LVSA_SVP64, false, false, true>(a, s);
#else
    case 64: return bf16 ? launch<64, LVSA_SK64, LVSA_SV64, true>(a, s) : launch<64, LVSA_SK64, LVSA_SV64, false>(a, s);
#endif
    default: return LVSA_ERR_UNSUPPORTED;
  }
}

#ifndef LVSA_SK8
#define LVSA_SK8 6
#define LVSA_SV8 6
#endif
extern "C" int lvsa_attn_fwd_fp8(const LvsaAttnArgs* a, const LvsaFp8Scales* sc, void* stream) {
  using namespace lvsa;
  const int v = validate(a);
  if (v != LVSA_OK) return v;
  if (!sc) return LVSA_ERR_INVALID_ARG;
  if (a->head_dim != 128) return LVSA_ERR_UNSUPPORTED;
  if (a->dtype != LVSA_DTYPE_BF16 && a->dtype != LVSA_DTYPE_F16) return LVSA_ERR_UNSUPPORTED;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
#ifndef LVSA_PAIR8
#define LVSA_PAIR8 0
#define LVSA_SKP8 6
#define LVSA_SVP8 6
#endif
#if LVSA_PAIR8
  return a->dtype == LVSA_DTYPE_BF16 ? launch<128, LVSA_SKP8, LVSA_SVP8, true, true, true>(a, s, sc)
                                      : launch<128, LVSA_SKP8, LVSA_SVP8, false, true, true>(a, s, sc);
#else
  return a->dtype == LVSA_DTYPE_BF16 ? launch<128, LVSA_SK8, LVSA_SV8, true, true>(a, s, sc)
                                      : launch<128, LVSA_SK8, LVSA_SV8, false, true>(a, s, sc);
#endif
}

extern "C" const char* lvsa_status_str(int status) {
  switch (status) {
    case LVSA_OK: return "ok";
    case LVSA_ERR_INVALID_ARG: return "invalid argument";
    case LVSA_ERR_GEOMETRY: return "geometry mismatch";
    case LVSA_ERR_UNSUPPORTED: return "unsupported head_dim/dtype/block size";
    case LVSA_ERR_ALIGNMENT: return "pointer or stride not 16-byte aligned for TMA";
    case LVSA_ERR_CAPACITY: return "buffer capacity too small";
    case LVSA_ERR_CUDA: return "CUDA runtime error";
    case LVSA_ERR_DEVICE_TIMEOUT: return "device wait timed out";
    default: return "unknown status";
  }
}

extern "C" int lvsa_abi_version(void) { return 102; }

#ifdef LVSA_PROFILE
// Instrumentation build only: copy out and clear the role totals.
extern "C" int lvsa_prof_read(unsigned long long* out16) {
  if (cudaMemcpyFromSymbol(out16, g_lvsa_prof, sizeof(g_lvsa_prof)) != cudaSuccess) return LVSA_ERR_CUDA;
  unsigned long long z[16] = {};
  return cudaMemcpyToSymbol(g_lvsa_prof, z, sizeof(z)) == cudaSuccess ? LVSA_OK : LVSA_ERR_CUDA;
}
#endif
