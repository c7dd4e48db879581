// QK prologue: per-token norm (RMS over the row, RMS per head, or LayerNorm
// per head) and interleaved-pair rotary embedding, fused into one pass over
// q or k in HBM (in place).  The adapters' unfused path reads and writes the
// tensor once for the norm and once more for the rotary embedding
// (lvsa/adapters/wan.py:48-67 + lvsa/rope.py:10-28;
// lvsa/adapters/hunyuan_video.py:71-103, :156-205;
// lvsa/adapters/cogvideox.py:88-117, :169-217).
//
// A warp handles one token row at a time: lane l owns the 16-byte vectors
// (8 values) l, l + 32, ... of the H*D row, so the row is read once; the norm
// statistics are warp (row norm) or lane-group (per-head norm, D/8 lanes per
// head) shuffle reductions; the rotary angles of the token are read as
// float4s.  Rows of up to 512 vectors go through the persistent ring kernel
// (rows staged in shared memory ahead of use); longer rows through the
// one-row-per-warp kernels.  Bound: HBM bandwidth (2 * 2 bytes per element
// moved, bf16/f16).
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
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

// Sum over aligned groups of `group` lanes (a power of two <= 32).
__device__ __forceinline__ float group_sum(float v, int group) {
  for (int o = group >> 1; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}

// Eight norm parameters in their storage type: one 16-byte load for bf16 /
// f16, two for fp32.
template <typename WT>
struct WPack {
  uint4 u;
  __device__ __forceinline__ void load(const void* p, int64_t i) {
    u = __ldg(reinterpret_cast<const uint4*>(static_cast<const WT*>(p) + i));
  }
  __device__ __forceinline__ void get(float (&f)[8]) const { unpack8<WT>(u, f); }
};
template <>
struct WPack<float> {
  float4 a, b;
  __device__ __forceinline__ void load(const void* p, int64_t i) {
    a = __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(p) + i));
    b = __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(p) + i) + 1);
  }
  __device__ __forceinline__ void get(float (&f)[8]) const {
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
  }
};

// Rotation of the 4 pairs of a vector by the angles (c, s).
__device__ __forceinline__ void rotate8(float (&f)[8], const float4& c, const float4& s) {
  const float cc[4] = {c.x, c.y, c.z, c.w}, ss[4] = {s.x, s.y, s.z, s.w};
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float x0 = f[2 * q], x1 = f[2 * q + 1];
    f[2 * q] = x0 * cc[q] - x1 * ss[q];
    f[2 * q + 1] = x0 * ss[q] + x1 * cc[q];
  }
}

// With D/8 lanes per head (a power of two <= 32), vector v = lane + 32 i
// always covers dims d0 = (lane % (D/8)) * 8 .. +7 of its head: the rotation
// angles and per-head norm parameters are one load per lane and row.
struct LaneRow {
  int bi, t, d0;
  bool rope;
  float4 c, s;
};

__device__ __forceinline__ LaneRow lane_row(const LvsaQkPrologue& a, int64_t row, int lane) {
  LaneRow r;
  r.bi = static_cast<int>(row / a.seq);
  r.t = static_cast<int>(row % a.seq);
  r.d0 = (lane % (a.head_dim / 8)) * 8;
  r.rope = a.cos != nullptr;
  r.c = r.s = make_float4(0.f, 0.f, 0.f, 0.f);
  if (r.rope) {
    const int64_t off = r.bi * a.rope_stride_b + static_cast<int64_t>(a.rope_offset + r.t) * (a.head_dim / 2) + r.d0 / 2;
    r.c = __ldg(reinterpret_cast<const float4*>(a.cos + off));
    r.s = __ldg(reinterpret_cast<const float4*>(a.sin + off));
  }
  return r;
}

// Row norm: one warp per token row (the statistic spans the row); all of the
// row's vectors are loaded before any arithmetic.  kKeep: the row stays in
// registers; otherwise the output pass reads it again (L1 hit).  The weights
// are read in the output pass (L1 hits after the first rows), which keeps the
// kernel at <= 85 registers, 3 blocks per SM: enough rows in flight to cover
// HBM latency (keeping them as well halved the bandwidth).
template <typename T, typename WT, int VPL, bool kKeep>
__global__ void __launch_bounds__(32 * kWarpsPerBlock, 3)
    qk_prologue_row_kernel(const LvsaQkPrologue a, int64_t rows) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kWarpsPerBlock + (threadIdx.x >> 5);
  if (row >= rows) return;  // whole warp
  const LaneRow lr = lane_row(a, row, lane);
  const int G = a.head_dim / 8, nv = a.heads * G;
  T* base = static_cast<T*>(a.x.ptr) + lr.bi * a.x.stride_b + static_cast<int64_t>(lr.t) * a.x.stride_t;
  auto vaddr = [&](int v) { return base + (v / G) * a.x.stride_h + lr.d0; };
  uint4 raw[kKeep ? VPL : 1];
  float sq = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int v = lane + 32 * i;
    uint4 u = make_uint4(0u, 0u, 0u, 0u);
    if (v < nv) {
      u = *reinterpret_cast<const uint4*>(vaddr(v));

    }
    if constexpr (kKeep) raw[i] = u;
    float f[8];
    unpack8<T>(u, f);
#pragma unroll
    for (int k = 0; k < 8; ++k) sq += f[k] * f[k];
  }
  const float rstd = rsqrtf(group_sum(sq, 32) / (a.heads * a.head_dim) + a.eps);
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int v = lane + 32 * i;
    if (v >= nv) continue;
    float f[8], w[8] = {1.f, 1.f, 1.f, 1.f, 1.f, 1.f, 1.f, 1.f};
    if constexpr (kKeep) {
      unpack8<T>(raw[i], f);
      if (a.weight) {
        WPack<WT> p;
        p.load(a.weight, int64_t(v) * 8);
        p.get(w);
      }
    } else {
      unpack8<T>(*reinterpret_cast<const uint4*>(vaddr(v)), f);
      if (a.weight) {
        WPack<WT> p;
        p.load(a.weight, int64_t(v) * 8);
        p.get(w);
      }
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) f[k] = f[k] * rstd * w[k];
    if (lr.rope) rotate8(f, lr.c, lr.s);
    *reinterpret_cast<uint4*>(vaddr(v)) = pack8<T>(f);
  }
}

// Persistent ring kernel (every norm, rows of up to 512 vectors): a few
// blocks per SM, each warp walking rows row, row + stride, ...  The vectors of
// the next S - 1 rows are copied into the warp's shared-memory ring
// (cp.async, 16 bytes per lane and vector) while the current row is
// normalised, rotated and stored from the ring, so every warp keeps S - 1 rows
// of loads in flight without holding them in registers.  Rows of up to 8
// vectors per lane are normalised from registers (one ring read), longer
// ones in two passes over the ring.  Measured on q + k (two launches, L2
// flushed before), GB/s:
//   cfg2 (row RMSNorm, 12 x 128): S = 2 with 2 blocks per SM 5 378-5 402,
//     3 blocks 4 186, 4 blocks 3 832; S = 3 5 135-5 225; S = 4-6 with 1 block
//     3 695-3 933; the one-row-per-warp kernels below 2 980-2 996.
//   cfg4 (per-head RMSNorm, 16 x 128): 2 blocks 4 161-4 178, 3 blocks
//     4 321-4 429; per-head kernel below 3 450-3 479.
//   cfg5 (per-head LayerNorm, 48 x 64): 2 blocks 3 413, 3 blocks 3 342-3 348;
//     per-head kernel below 3 061-3 064.
#ifndef LVSA_PRO_S
#define LVSA_PRO_S 2
#endif

// Lane-constant part of a row's vector addresses: vector v = lane + 32 i
// lies in head v / G = lane / G + i (32 / G) at dims d0 .. d0 + 7.
struct LaneOff {
  int64_t off0, step;
  int nvl;  // vectors of this lane: lane + 32 i < nv for i < nvl
};

__device__ __forceinline__ LaneOff lane_off(const LvsaQkPrologue& a, int lane) {
  const int G = a.head_dim / 8, nv = a.heads * G;
  LaneOff o;
  o.off0 = static_cast<int64_t>(lane / G) * a.x.stride_h + (lane % G) * 8;
  o.step = static_cast<int64_t>(32 / G) * a.x.stride_h;
  o.nvl = (nv - lane + 31) / 32;
  return o;
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool full) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(full ? 16 : 0) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// One row from the ring (xs[32 i] = vector lane + 32 i; zero past the row).
// Every lane runs every i (the per-head reductions shuffle over all 32
// lanes); only vectors inside the row are stored.
template <typename T, typename WT, int VPL>
__device__ __forceinline__ void ring_row(const uint4* xs, const LvsaQkPrologue& a, const LaneOff& lo, int64_t row,
                                         int lane, const float (&wh)[8], const float (&bh)[8]) {
  const LaneRow lr = lane_row(a, row, lane);
  T* p = static_cast<T*>(a.x.ptr) + lr.bi * a.x.stride_b + static_cast<int64_t>(lr.t) * a.x.stride_t + lo.off0;
  const int D = a.head_dim, G = D / 8;
  if (VPL <= 8 && a.norm == LVSA_NORM_RMS_ROW) {
    // Row statistic: the row is read from the ring once, into registers.
    uint4 x[VPL];
#pragma unroll
    for (int i = 0; i < VPL; ++i) x[i] = xs[32 * i];
    float sq = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      float f[8];
      unpack8<T>(x[i], f);
#pragma unroll
      for (int k = 0; k < 8; ++k) sq += f[k] * f[k];
    }
    const float rstd = rsqrtf(group_sum(sq, 32) / (a.heads * D) + a.eps);
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      if (i >= lo.nvl) break;
      float f[8], w[8] = {1.f, 1.f, 1.f, 1.f, 1.f, 1.f, 1.f, 1.f};
      unpack8<T>(x[i], f);
      if (a.weight) {
        WPack<WT> wp;
        wp.load(a.weight, int64_t(lane + 32 * i) * 8);
        wp.get(w);
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) f[k] = f[k] * rstd * w[k];
      if (lr.rope) rotate8(f, lr.c, lr.s);
      *reinterpret_cast<uint4*>(p + i * lo.step) = pack8<T>(f);
    }
    return;
  }
  float rstd_row = 1.f;
  if (a.norm == LVSA_NORM_RMS_ROW) {  // longer rows: two passes over the ring
    float sq = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      float f[8];
      unpack8<T>(xs[32 * i], f);
#pragma unroll
      for (int k = 0; k < 8; ++k) sq += f[k] * f[k];
    }
    rstd_row = rsqrtf(group_sum(sq, 32) / (a.heads * D) + a.eps);
  }
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    float f[8];
    unpack8<T>(xs[32 * i], f);
    if (a.norm == LVSA_NORM_RMS_ROW) {
      float w[8] = {1.f, 1.f, 1.f, 1.f, 1.f, 1.f, 1.f, 1.f};
      if (a.weight && i < lo.nvl) {
        WPack<WT> wp;
        wp.load(a.weight, int64_t(lane + 32 * i) * 8);
        wp.get(w);
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) f[k] = f[k] * rstd_row * w[k];
    } else if (a.norm != LVSA_NORM_NONE) {
      float mean = 0.f;
      if (a.norm == LVSA_NORM_LAYER_HEAD) {
        float sum = 0.f;
#pragma unroll
        for (int k = 0; k < 8; ++k) sum += f[k];
        mean = group_sum(sum, G) / D;
      }
      float q = 0.f;
#pragma unroll
      for (int k = 0; k < 8; ++k) q += (f[k] - mean) * (f[k] - mean);
      const float rstd = rsqrtf(group_sum(q, G) / D + a.eps);
#pragma unroll
      for (int k = 0; k < 8; ++k) f[k] = (f[k] - mean) * rstd * wh[k] + bh[k];
    }
    if (lr.rope) rotate8(f, lr.c, lr.s);
    if (i < lo.nvl) *reinterpret_cast<uint4*>(p + i * lo.step) = pack8<T>(f);
  }
}

#ifndef LVSA_PRO_B
#define LVSA_PRO_B 2
#endif
template <typename T, typename WT, int VPL, int S>
__global__ void __launch_bounds__(32 * kWarpsPerBlock, LVSA_PRO_B)
    qk_prologue_ring_kernel(const LvsaQkPrologue a, int64_t rows) {
  extern __shared__ uint4 pro_ring[];  // [warp][S][VPL][32 lanes]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint4* ring = pro_ring + warp * (S * VPL * 32);
  const uint32_t ring_s = static_cast<uint32_t>(__cvta_generic_to_shared(ring));
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kWarpsPerBlock;
  const int64_t row0 = static_cast<int64_t>(blockIdx.x) * kWarpsPerBlock + warp;
  const LaneOff lo = lane_off(a, lane);
  // Per-head norm parameters are lane-constant (dims d0 .. d0 + 7 of every head).
  float wh[8] = {1.f, 1.f, 1.f, 1.f, 1.f, 1.f, 1.f, 1.f}, bh[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (a.norm != LVSA_NORM_NONE && a.norm != LVSA_NORM_RMS_ROW) {
    const int d0 = (lane % (a.head_dim / 8)) * 8;
    if (a.weight) {
      WPack<WT> wp;
      wp.load(a.weight, d0);
      wp.get(wh);
    }
    if (a.norm == LVSA_NORM_LAYER_HEAD && a.bias) {
      WPack<WT> wp;
      wp.load(a.bias, d0);
      wp.get(bh);
    }
  }
  auto fetch = [&](int slot, int64_t row) {
    if (row < rows) {
      const int64_t bi = row / a.seq, t = row % a.seq;
      const T* p = static_cast<const T*>(a.x.ptr) + bi * a.x.stride_b + t * a.x.stride_t + lo.off0;
#pragma unroll
      for (int i = 0; i < VPL; ++i)  // vectors past the row: zero-filled, nothing read
        cp_async16(ring_s + ((slot * VPL + i) * 32 + lane) * 16, i < lo.nvl ? p + i * lo.step : p, i < lo.nvl);
    }
    cp_async_commit();  // one group per row, empty past the end
  };
#pragma unroll
  for (int k = 0; k < S - 1; ++k) fetch(k, row0 + k * stride);
  int slot = 0;
  for (int64_t row = row0; row < rows; row += stride) {
    fetch(slot == 0 ? S - 1 : slot - 1, row + (S - 1) * stride);  // the slot read last iteration
    cp_async_wait<S - 1>();                                         // this row's group has landed
    ring_row<T, WT, VPL>(ring + slot * VPL * 32 + lane, a, lo, row, lane, wh, bh);
    slot = slot + 1 == S ? 0 : slot + 1;
  }
  cp_async_wait<0>();
}

template <typename T, typename WT, int VPL>
int launch_ring(const LvsaQkPrologue* a, int64_t rows, cudaStream_t s) {
  constexpr int S = LVSA_PRO_S;
  constexpr int kSmem = kWarpsPerBlock * S * VPL * 32 * 16;
  auto kern = qk_prologue_ring_kernel<T, WT, VPL, S>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem) != cudaSuccess)
    return LVSA_ERR_CUDA;
  int dev = 0, sms = 148, per_sm = 1;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, 32 * kWarpsPerBlock, kSmem) != cudaSuccess ||
      per_sm < 1)
    per_sm = 1;
  per_sm = std::min(per_sm, LVSA_PRO_B);
  const int64_t want = (rows + kWarpsPerBlock - 1) / kWarpsPerBlock;
  const dim3 grid(static_cast<unsigned>(std::min<int64_t>(want, static_cast<int64_t>(per_sm) * sms)));
  kern<<<grid, 32 * kWarpsPerBlock, kSmem, s>>>(*a, rows);
  return LVSA_OK;
}

// Per-head norm (or none): the G = D/8 vectors of a head are G consecutive
// lanes of one 32-vector slice, so a warp takes VPL slices of a row
// (blockIdx.y picks which) and needs no row-wide reduction.
template <typename T, typename WT, int VPL>
__global__ void __launch_bounds__(32 * kWarpsPerBlock)
    qk_prologue_head_kernel(const LvsaQkPrologue a, int64_t rows) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kWarpsPerBlock + (threadIdx.x >> 5);
  if (row >= rows) return;  // whole warp
  const LaneRow lr = lane_row(a, row, lane);
  const int D = a.head_dim, G = D / 8, nv = a.heads * G;
  const int v0 = blockIdx.y * 32 * VPL;
  T* base = static_cast<T*>(a.x.ptr) + lr.bi * a.x.stride_b + static_cast<int64_t>(lr.t) * a.x.stride_t;
  auto vaddr = [&](int v) { return base + (v / G) * a.x.stride_h + lr.d0; };
  uint4 raw[VPL];
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int v = v0 + lane + 32 * i;
    raw[i] = v < nv ? *reinterpret_cast<const uint4*>(vaddr(v)) : make_uint4(0u, 0u, 0u, 0u);
  }
  float w[8] = {1.f, 1.f, 1.f, 1.f, 1.f, 1.f, 1.f, 1.f}, bb[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (a.norm != LVSA_NORM_NONE && a.weight) {
    WPack<WT> p;
    p.load(a.weight, lr.d0);
    p.get(w);
  }
  if (a.norm == LVSA_NORM_LAYER_HEAD && a.bias) {
    WPack<WT> p;
    p.load(a.bias, lr.d0);
    p.get(bb);
  }
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int v = v0 + lane + 32 * i;
    float f[8];
    unpack8<T>(raw[i], f);
    if (a.norm != LVSA_NORM_NONE) {
      float mean = 0.f;
      if (a.norm == LVSA_NORM_LAYER_HEAD) {
        float sum = 0.f;
#pragma unroll
        for (int k = 0; k < 8; ++k) sum += f[k];
        mean = group_sum(sum, G) / D;
      }
      float q = 0.f;
#pragma unroll
      for (int k = 0; k < 8; ++k) q += (f[k] - mean) * (f[k] - mean);
      const float rstd = rsqrtf(group_sum(q, G) / D + a.eps);
#pragma unroll
      for (int k = 0; k < 8; ++k) f[k] = (f[k] - mean) * rstd * w[k] + bb[k];
    }
    if (lr.rope) rotate8(f, lr.c, lr.s);
    if (v < nv) *reinterpret_cast<uint4*>(vaddr(v)) = pack8<T>(f);
  }
}

template <typename T, typename WT>
int launch_prologue_t(const LvsaQkPrologue* a, cudaStream_t s) {
  const int64_t rows = static_cast<int64_t>(a->batch) * a->seq;
  const int nv = a->heads * (a->head_dim / 8);
  const unsigned gx = static_cast<unsigned>((rows + kWarpsPerBlock - 1) / kWarpsPerBlock);
  const dim3 block(32 * kWarpsPerBlock);
#ifndef LVSA_PRO_RING
#define LVSA_PRO_RING 1
#endif
  if (LVSA_PRO_RING && nv <= 512) {
    const int st = nv <= 32    ? launch_ring<T, WT, 1>(a, rows, s)
                   : nv <= 64  ? launch_ring<T, WT, 2>(a, rows, s)
                   : nv <= 128 ? launch_ring<T, WT, 4>(a, rows, s)
                   : nv <= 256 ? launch_ring<T, WT, 8>(a, rows, s)
                   : nv <= 384 ? launch_ring<T, WT, 12>(a, rows, s)
                               : launch_ring<T, WT, 16>(a, rows, s);
    if (st != LVSA_OK) return st;
  } else if (a->norm == LVSA_NORM_RMS_ROW) {
    const dim3 grid(gx);
    if (nv <= 32) qk_prologue_row_kernel<T, WT, 1, true><<<grid, block, 0, s>>>(*a, rows);
    else if (nv <= 64) qk_prologue_row_kernel<T, WT, 2, true><<<grid, block, 0, s>>>(*a, rows);
    else if (nv <= 128) qk_prologue_row_kernel<T, WT, 4, true><<<grid, block, 0, s>>>(*a, rows);
    else if (nv <= 256) qk_prologue_row_kernel<T, WT, 8, true><<<grid, block, 0, s>>>(*a, rows);
    else if (nv <= 512) qk_prologue_row_kernel<T, WT, 16, false><<<grid, block, 0, s>>>(*a, rows);
    else qk_prologue_row_kernel<T, WT, 32, false><<<grid, block, 0, s>>>(*a, rows);
  } else if (nv <= 32) {
    qk_prologue_head_kernel<T, WT, 1><<<dim3(gx, 1), block, 0, s>>>(*a, rows);
  } else {
    qk_prologue_head_kernel<T, WT, 4><<<dim3(gx, (nv + 127) / 128), block, 0, s>>>(*a, rows);
  }
  return cudaGetLastError() == cudaSuccess ? LVSA_OK : LVSA_ERR_CUDA;
}

template <typename T>
int launch_prologue(const LvsaQkPrologue* a, cudaStream_t s) {
  if (a->weight_dtype == LVSA_DTYPE_F32 || a->weight == nullptr) return launch_prologue_t<T, float>(a, s);
  if (a->weight_dtype == LVSA_DTYPE_BF16) return launch_prologue_t<T, __nv_bfloat16>(a, s);
  return launch_prologue_t<T, __half>(a, s);
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
