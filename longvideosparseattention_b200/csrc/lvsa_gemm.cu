// Output projection of an attention layer on tcgen05: out[M, N] =
// A[M, K] . W[N, K]^T (+ bias[N]), bf16 / f16 in and out, fp32 accumulation
// in tensor memory.  A is the attention output read in place: [B, S, H, D]
// token-major is exactly [M = B*S, K = H*D] with K contiguous, the K-major A
// operand; W is an nn.Linear weight [out_features, in_features], the K-major
// B operand.  Replaces the model's `attn.to_out[0]` Linear after attention
// (lvsa/adapters/wan.py:121-131, lvsa/adapters/hunyuan_video.py:207-217).
//
// Persistent: one CTA per SM walks 128 x 256 output tiles (N tiles fastest,
// so the CTAs on one row block of A read it from L2).  Warp 0 streams A and
// W tiles of 64 K-columns through a 4-stage TMA ring (128B swizzle, no
// multicast) across tile boundaries; warp 1 allocates two 256-column TMEM
// accumulators and issues the MMAs (128 x 256 x 16 per instruction) from
// one thread, alternating accumulators per tile; warps 2-5 read a finished
// accumulator back (one row per thread), add the bias and store while the
// MMAs of the next tile run into the other one.  Every wait is bounded
// (error word, drain, free TMEM, return).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>
#include <type_traits>

#include "../../include/lvsa_b200.h"
#include "lvsa_ptx.cuh"

namespace lvsa {
namespace {

constexpr int kGM = 128, kGN = 256, kGK = 64;       // tile; kGK bf16 = one 128-byte swizzle row
constexpr int kGStages = 4;
constexpr int kATile = kGM * kGK * 2;                // 16 KB
constexpr int kBTile = kGN * kGK * 2;                // 32 KB
constexpr int kGThreads = 6 * 32;
constexpr int kGSmem = kGStages * (kATile + kBTile) + 1024 + 256;

struct GemmParams {
  void* out;
  const void* bias;
  int64_t ldo;  // elements
  int M, N, K;
  int* err;
};

__device__ __forceinline__ void tma_load_2d(void* dst, const void* map, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}

template <bool kBf16>
__global__ void __launch_bounds__(kGThreads, 1)
    lvsa_out_proj_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_w,
                         const GemmParams prm) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + kGStages * kATile;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kGStages * (kATile + kBTile));
  uint64_t* full = bars;                  // [stages] A and W tiles landed
  uint64_t* empty = bars + kGStages;      // [stages] their MMAs retired
  uint64_t* acc_full = bars + 2 * kGStages;  // [2] accumulator b holds a finished tile
  uint64_t* acc_empty = acc_full + 2;        // [2] epilogue has read accumulator b
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* never = reinterpret_cast<volatile int*>(tmem_slot + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kblocks = prm.K / kGK;
  const int n_tiles_n = (prm.N + kGN - 1) / kGN;
  const int n_tiles = n_tiles_n * ((prm.M + kGM - 1) / kGM);
  // Persistent: CTA c takes tiles c, c + grid, ...; N tiles fastest, so the
  // CTAs working on one row block of A at a time read it from L2.

  if (threadIdx.x == 0) {
    for (int s = 0; s < kGStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 128);
    }
    mbar_init(drain, 1);
    *abort = 0;
    *never = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 2 * kGN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tm_a);
      tma_prefetch_desc(&tm_w);
      int g = 0;  // global load counter across tiles
      bool ok = true;
      for (int t = blockIdx.x; ok && t < n_tiles; t += gridDim.x) {
        const int n0 = (t % n_tiles_n) * kGN, m0 = (t / n_tiles_n) * kGM;
        for (int kb = 0; kb < kblocks; ++kb, ++g) {
          const int s = g % kGStages;
          if (g >= kGStages &&
              !(ok = mbar_wait(&empty[s], ((g / kGStages) - 1) & 1, abort, prm.err, LVSA_ERR_DEVICE_TIMEOUT)))
            break;
          mbar_expect_tx(&full[s], kATile + kBTile);
          tma_load_2d(sA + s * kATile, &tm_a, &full[s], kb * kGK, m0);
          tma_load_2d(sB + s * kBTile, &tm_w, &full[s], kb * kGK, n0);
        }
      }
      if (*abort)  // drain our own copies before the CTA retires
        for (int x = g > kGStages ? g - kGStages : 0; x < g; ++x)
          mbar_wait(&full[x % kGStages], (x / kGStages) & 1, never, nullptr, 0);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16(kGM, kGN, kBf16, false);
      const uint32_t a_base = smem_u32(sA), b_base = smem_u32(sB);
      bool ok = true;
      int g = 0, it = 0;
      for (int t = blockIdx.x; ok && t < n_tiles; t += gridDim.x, ++it) {
        const int buf = it & 1;
        const uint32_t tacc = tmem + buf * kGN;
        // Accumulator `buf` was last used by tile it - 2: wait for its epilogue.
        if (it >= 2 && !(ok = mbar_wait(&acc_empty[buf], ((it >> 1) - 1) & 1, abort, prm.err,
                                        LVSA_ERR_DEVICE_TIMEOUT)))
          break;
        tc_fence_after();
        for (int kb = 0; kb < kblocks; ++kb, ++g) {
          const int s = g % kGStages;
          if (!(ok = mbar_wait(&full[s], (g / kGStages) & 1, abort, prm.err, LVSA_ERR_DEVICE_TIMEOUT))) break;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < kGK / 16; ++kk)  // 32 bytes of K per instruction
            mma_ss(tacc, sdesc_sw128(a_base + s * kATile + kk * 32, 16, 1024),
                   sdesc_sw128(b_base + s * kBTile + kk * 32, 16, 1024), idesc, (kb | kk) > 0);
          mma_commit(&empty[s]);
        }
        if (ok) mma_commit(&acc_full[buf]);
      }
      mma_commit(drain);
      mbar_wait(drain, 0, never, nullptr, 0);
    }
  } else {
    // warps 2..5: TMEM lanes 32 * (warp % 4) .. + 31, one output row each
    using Elem = typename std::conditional<kBf16, __nv_bfloat16, __half>::type;
    const int q = warp & 3;
    const Elem* bias = static_cast<const Elem*>(prm.bias);
    int it = 0;
    for (int t = blockIdx.x; t < n_tiles; t += gridDim.x, ++it) {
      const int buf = it & 1;
      const int n0 = (t % n_tiles_n) * kGN, m0 = (t / n_tiles_n) * kGM;
      if (!__all_sync(0xFFFFFFFFu, mbar_wait(&acc_full[buf], (it >> 1) & 1, abort, prm.err,
                                             LVSA_ERR_DEVICE_TIMEOUT)))
        break;
      tc_fence_after();
      const uint32_t tacc = tmem + buf * kGN + (static_cast<uint32_t>(q * 32) << 16);
      const int row = m0 + q * 32 + lane;
      Elem* orow = static_cast<Elem*>(prm.out) + static_cast<int64_t>(row) * prm.ldo + n0;
#pragma unroll 1
      for (int c = 0; c < kGN / 32; ++c) {
        uint32_t t32[32];
        tmem_ld32(tacc + c * 32, t32);
        const int col = n0 + c * 32;
        if (row < prm.M && col < prm.N) {
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            float x0 = __uint_as_float(t32[2 * i]), x1 = __uint_as_float(t32[2 * i + 1]);
            if (bias) {
              x0 += static_cast<float>(bias[col + 2 * i]);
              x1 += static_cast<float>(bias[col + 2 * i + 1]);
            }
            if constexpr (kBf16) {
              __nv_bfloat162 h = __floats2bfloat162_rn(x0, x1);
              pk[i] = *reinterpret_cast<uint32_t*>(&h);
            } else {
              __half2 h = __floats2half2_rn(x0, x1);
              pk[i] = *reinterpret_cast<uint32_t*>(&h);
            }
          }
          uint4* dst = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
          for (int i = 0; i < 4; ++i) dst[i] = make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
        }
      }
      // The accumulator's columns are read: the next tile's MMAs may reuse it.
      tc_fence_before();
      mbar_arrive(&acc_empty[buf]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 2 * kGN);
  }
}

using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeFn encode_fn() {
  static EncodeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeFn>(p);
  });
  return fn;
}

// [rows, cols] row-major 16-bit matrix, row stride ld elements -> 2-D map
// with a (64 columns = 128 bytes) x box_rows box, 128B swizzle.
int map_2d(CUtensorMap* m, const void* ptr, int rows, int cols, int64_t ld, int box_rows, bool bf16) {
  EncodeFn enc = encode_fn();
  if (!enc) return LVSA_ERR_CUDA;
  if ((reinterpret_cast<uintptr_t>(ptr) & 15) || (ld * 2) % 16) return LVSA_ERR_ALIGNMENT;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * 2)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(kGK), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                   const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? LVSA_OK : LVSA_ERR_ALIGNMENT;
}

}  // namespace
}  // namespace lvsa

extern "C" int lvsa_out_proj(const LvsaOutProjArgs* a, void* stream) {
  using namespace lvsa;
  if (!a || !a->a || !a->weight || !a->out) return LVSA_ERR_INVALID_ARG;
  if (a->m < 1 || a->n < 1 || a->k < 1) return LVSA_ERR_INVALID_ARG;
  if (a->dtype != LVSA_DTYPE_BF16 && a->dtype != LVSA_DTYPE_F16) return LVSA_ERR_UNSUPPORTED;
  if (a->k % kGK || a->n % 32) return LVSA_ERR_UNSUPPORTED;
  if (a->lda < a->k || a->ldw < a->k || a->ldo < a->n) return LVSA_ERR_INVALID_ARG;
  if ((reinterpret_cast<uintptr_t>(a->out) & 15) || (a->ldo * 2) % 16) return LVSA_ERR_ALIGNMENT;
  const bool bf16 = a->dtype == LVSA_DTYPE_BF16;
  CUtensorMap ma, mw;
  int st;
  if ((st = map_2d(&ma, a->a, a->m, a->k, a->lda, kGM, bf16))) return st;
  if ((st = map_2d(&mw, a->weight, a->n, a->k, a->ldw, kGN, bf16))) return st;
  GemmParams p;
  p.out = a->out;
  p.bias = a->bias;
  p.ldo = a->ldo;
  p.M = a->m;
  p.N = a->n;
  p.K = a->k;
  p.err = a->error_word;
  auto kern = bf16 ? lvsa_out_proj_kernel<true> : lvsa_out_proj_kernel<false>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kGSmem) != cudaSuccess)
    return LVSA_ERR_CUDA;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const long long tiles = static_cast<long long>((a->n + kGN - 1) / kGN) * ((a->m + kGM - 1) / kGM);
  dim3 grid(static_cast<unsigned>(tiles < sms ? tiles : sms));
  kern<<<grid, kGThreads, kGSmem, static_cast<cudaStream_t>(stream)>>>(ma, mw, p);
  return cudaGetLastError() == cudaSuccess ? LVSA_OK : LVSA_ERR_CUDA;
}
