// QK prologue: per-token norm (RMS over the row, RMS per head, or LayerNorm
// per head) and interleaved-pair rotary embedding, fused into one pass over
// q or k in HBM (in place).  The adapters' unfused path reads and writes the
// tensor once for the norm and once more for the rotary embedding
// (lvsa/adapters/wan.py:48-67 + lvsa/rope.py:10-28;
// lvsa/adapters/hunyuan_video.py:71-103, :156-205;
// lvsa/adapters/cogvideox.py:88-117, :169-217).
//
// One warp per token: each lane holds VPL 16-byte vectors (8 values) of the
// H*D row in registers, so the row is read once; the norm statistics are
// warp (row norm) or lane-group (per-head norm, D/8 lanes per head)
// shuffle reductions; the rotary angles of the token are read as float4s.
// Bound: HBM bandwidth (2 * 2 bytes per element moved, bf16/f16).
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <type_traits>

#include "../../include/lvsa_b200.h"

namespace lvsa {
namespace {

constexpr int kWarpsPerBlock = 8;

template <typename T>
__device__ __forceinline__ void unpack8(const uint4& u, float (&f)[8]) {
  const T* h = reinterpret_cast<const T*>(&u);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    if constexpr (std::is_same<T, __nv_bfloat16>::value) f[i] = __bfloat162float(h[i]);
    else f[i] = __half2float(h[i]);
  }
}

template <typename T>
__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  uint4 u;
  T* h = reinterpret_cast<T*>(&u);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    if constexpr (std::is_same<T, __nv_bfloat16>::value) h[i] = __float2bfloat16_rn(f[i]);
    else h[i] = __float2half_rn(f[i]);
  }
  return u;
}

// 8 consecutive parameters (weight or bias) starting at element i, as fp32.
__device__ __forceinline__ void load_param8(const void* p, int dt, int64_t i, float (&f)[8]) {
  if (dt == LVSA_DTYPE_F32) {
    const float4 a = reinterpret_cast<const float4*>(static_cast<const float*>(p) + i)[0];
    const float4 b = reinterpret_cast<const float4*>(static_cast<const float*>(p) + i)[1];
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
  } else if (dt == LVSA_DTYPE_BF16) {
    unpack8<__nv_bfloat16>(*reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(p) + i), f);
  } else {
    unpack8<__half>(*reinterpret_cast<const uint4*>(static_cast<const __half*>(p) + i), f);
  }
}

// Sum over aligned groups of `group` lanes (a power of two <= 32).
__device__ __forceinline__ float group_sum(float v, int group) {
  for (int o = group >> 1; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}

// Norm + rotary embedding of one 16-byte vector (8 values at dims d0..d0+7).
template <typename T>
__device__ __forceinline__ uint4 finish8(const LvsaQkPrologue& a, const uint4& u, float mean, float rstd,
                                         int64_t w_idx, int d0, const float* cs, const float* sn) {
  float f[8];
  unpack8<T>(u, f);
  if (a.norm != LVSA_NORM_NONE) {
    float w[8] = {1.f, 1.f, 1.f, 1.f, 1.f, 1.f, 1.f, 1.f}, bb[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (a.weight) load_param8(a.weight, a.weight_dtype, w_idx, w);
    if (a.bias && a.norm == LVSA_NORM_LAYER_HEAD) load_param8(a.bias, a.weight_dtype, d0, bb);
#pragma unroll
    for (int k = 0; k < 8; ++k) f[k] = (f[k] - mean) * rstd * w[k] + bb[k];
  }
  if (cs) {
    const float4 c = *reinterpret_cast<const float4*>(cs + d0 / 2);
    const float4 s = *reinterpret_cast<const float4*>(sn + d0 / 2);
    const float cc[4] = {c.x, c.y, c.z, c.w}, ss[4] = {s.x, s.y, s.z, s.w};
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const float x0 = f[2 * p], x1 = f[2 * p + 1];
      f[2 * p] = x0 * cc[p] - x1 * ss[p];
      f[2 * p + 1] = x0 * ss[p] + x1 * cc[p];
    }
  }
  return pack8<T>(f);
}

// VPL: vectors per lane (the row holds at most 32 VPL vectors).  kKeep: the
// row norm keeps the row in registers between its two passes; otherwise the
// second pass reads it again (an L1 hit).
template <typename T, int VPL, bool kKeep>
__global__ void __launch_bounds__(32 * kWarpsPerBlock)
    qk_prologue_kernel(const LvsaQkPrologue a, int64_t rows) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kWarpsPerBlock + (threadIdx.x >> 5);
  if (row >= rows) return;  // whole warp
  const int bi = static_cast<int>(row / a.seq), t = static_cast<int>(row % a.seq);
  const int D = a.head_dim, G = D / 8;  // vectors per head (a power of two <= 32)
  const int nv = a.heads * G;           // vectors per row
  T* base = static_cast<T*>(a.x.ptr) + bi * a.x.stride_b + static_cast<int64_t>(t) * a.x.stride_t;
  auto vaddr = [&](int v) { return base + (v / G) * a.x.stride_h + (v % G) * 8; };
  const float* cs = nullptr;
  const float* sn = nullptr;
  if (a.cos) {
    const int64_t off = bi * a.rope_stride_b + static_cast<int64_t>(a.rope_offset + t) * (D / 2);
    cs = a.cos + off;
    sn = a.sin + off;
  }

  if (a.norm == LVSA_NORM_RMS_ROW) {
    uint4 raw[kKeep ? VPL : 1];
    float sq = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int v = lane + 32 * i;
      uint4 u = make_uint4(0u, 0u, 0u, 0u);
      if (v < nv) u = *reinterpret_cast<const uint4*>(vaddr(v));
      if constexpr (kKeep) raw[i] = u;
      float f[8];
      unpack8<T>(u, f);
#pragma unroll
      for (int k = 0; k < 8; ++k) sq += f[k] * f[k];
    }
    const float rstd = rsqrtf(group_sum(sq, 32) / (a.heads * D) + a.eps);
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int v = lane + 32 * i;
      if (v >= nv) continue;
      uint4 u;
      if constexpr (kKeep) u = raw[i];
      else u = *reinterpret_cast<const uint4*>(vaddr(v));
      *reinterpret_cast<uint4*>(vaddr(v)) = finish8<T>(a, u, 0.f, rstd, int64_t(v) * 8, (v % G) * 8, cs, sn);
    }
    return;
  }
  // Per-head norms (or none): the G vectors of a head are G consecutive lanes
  // of one iteration, so each iteration is self-contained.
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int v = lane + 32 * i;
    uint4 u = make_uint4(0u, 0u, 0u, 0u);
    if (v < nv) u = *reinterpret_cast<const uint4*>(vaddr(v));
    float mean = 0.f, rstd = 1.f;
    if (a.norm != LVSA_NORM_NONE) {
      float f[8];
      unpack8<T>(u, f);
      if (a.norm == LVSA_NORM_LAYER_HEAD) {
        float sum = 0.f;
#pragma unroll
        for (int k = 0; k < 8; ++k) sum += f[k];
        mean = group_sum(sum, G) / D;
      }
      float q = 0.f;
#pragma unroll
      for (int k = 0; k < 8; ++k) q += (f[k] - mean) * (f[k] - mean);
      rstd = rsqrtf(group_sum(q, G) / D + a.eps);
    }
    if (v < nv) *reinterpret_cast<uint4*>(vaddr(v)) = finish8<T>(a, u, mean, rstd, (v % G) * 8, (v % G) * 8, cs, sn);
  }
}

template <typename T>
int launch_prologue(const LvsaQkPrologue* a, cudaStream_t s) {
  const int64_t rows = static_cast<int64_t>(a->batch) * a->seq;
  const int nv = a->heads * (a->head_dim / 8);
  const dim3 grid(static_cast<unsigned>((rows + kWarpsPerBlock - 1) / kWarpsPerBlock)), block(32 * kWarpsPerBlock);
  if (nv <= 32) qk_prologue_kernel<T, 1, true><<<grid, block, 0, s>>>(*a, rows);
  else if (nv <= 64) qk_prologue_kernel<T, 2, true><<<grid, block, 0, s>>>(*a, rows);
  else if (nv <= 128) qk_prologue_kernel<T, 4, true><<<grid, block, 0, s>>>(*a, rows);
  else if (nv <= 256) qk_prologue_kernel<T, 8, true><<<grid, block, 0, s>>>(*a, rows);
  else if (nv <= 512) qk_prologue_kernel<T, 16, true><<<grid, block, 0, s>>>(*a, rows);
  else qk_prologue_kernel<T, 32, false><<<grid, block, 0, s>>>(*a, rows);
  return cudaGetLastError() == cudaSuccess ? LVSA_OK : LVSA_ERR_CUDA;
}

}  // namespace
}  // namespace lvsa

extern "C" int lvsa_qk_prologue(const LvsaQkPrologue* a, void* stream) {
  using namespace lvsa;
  if (!a || !a->x.ptr) return LVSA_ERR_INVALID_ARG;
  if (a->dtype != LVSA_DTYPE_BF16 && a->dtype != LVSA_DTYPE_F16) return LVSA_ERR_UNSUPPORTED;
  if (a->batch < 1 || a->seq < 0 || a->heads < 1 || a->norm < LVSA_NORM_NONE || a->norm > LVSA_NORM_LAYER_HEAD)
    return LVSA_ERR_INVALID_ARG;
  const int D = a->head_dim;
  if (D < 8 || D % 8 || (D / 8) & (D / 8 - 1) || D / 8 > 32 || a->heads * (D / 8) > 1024) return LVSA_ERR_UNSUPPORTED;
  if (a->norm != LVSA_NORM_NONE && a->weight && a->weight_dtype != LVSA_DTYPE_BF16 &&
      a->weight_dtype != LVSA_DTYPE_F16 && a->weight_dtype != LVSA_DTYPE_F32)
    return LVSA_ERR_UNSUPPORTED;
  if ((a->cos == nullptr) != (a->sin == nullptr) || a->rope_offset < 0 || a->rope_stride_b < 0)
    return LVSA_ERR_INVALID_ARG;
  const int64_t es = 2;
  if ((reinterpret_cast<uintptr_t>(a->x.ptr) & 15) || (a->x.stride_h * es) % 16 || (a->x.stride_t * es) % 16 ||
      (a->batch > 1 && (a->x.stride_b * es) % 16))
    return LVSA_ERR_ALIGNMENT;
  if ((a->weight && (reinterpret_cast<uintptr_t>(a->weight) & 15)) ||
      (a->bias && (reinterpret_cast<uintptr_t>(a->bias) % 16)) ||
      (a->cos && ((reinterpret_cast<uintptr_t>(a->cos) | reinterpret_cast<uintptr_t>(a->sin)) & 15)) ||
      (a->cos && (a->rope_stride_b * 4) % 16))
    return LVSA_ERR_ALIGNMENT;
  if (a->seq == 0) return LVSA_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return a->dtype == LVSA_DTYPE_BF16 ? launch_prologue<__nv_bfloat16>(a, s) : launch_prologue<__half>(a, s);
}
