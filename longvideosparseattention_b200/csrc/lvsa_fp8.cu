// E4M3 quantisation for the FP8 attention mode: per (batch, head, 128-token
// tile) scale = amax / 448 (the largest finite E4M3 value), saturating
// round-to-nearest conversion, optional atomicMax of the tile scales into a
// per-(batch, head) reference.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/lvsa_b200.h"

namespace lvsa {
namespace {

constexpr float kE4M3Max = 448.0f;

template <typename T, int D>
__global__ void __launch_bounds__(128) quantize_kernel(const T* __restrict__ in, int64_t sb, int64_t st,
                                                        int64_t sh, int n, int heads, uint8_t* __restrict__ out8,
                                                        float* __restrict__ scales, float* head_max) {
  __shared__ float red[4];
  const int tile = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int t = tile * 128 + threadIdx.x;
  const bool valid = t < n;
  float v[D];
  float amax = 0.f;
  if (valid) {
    const T* row = in + b * sb + static_cast<int64_t>(t) * st + h * sh;
#pragma unroll
    for (int i = 0; i < D; ++i) {
      v[i] = static_cast<float>(row[i]);
      amax = fmaxf(amax, fabsf(v[i]));
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  amax = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
  const float scale = amax > 0.f ? amax / kE4M3Max : 1.0f;
  const int ntiles = (n + 127) / 128;
  if (threadIdx.x == 0) {
    scales[(static_cast<int64_t>(b) * heads + h) * ntiles + tile] = scale;
    if (head_max) atomicMax(reinterpret_cast<int*>(head_max + static_cast<int64_t>(b) * heads + h), __float_as_int(scale));
  }
  if (!valid) return;
  const float inv = 1.0f / scale;
  uint8_t* dst = out8 + ((static_cast<int64_t>(b) * n + t) * heads + h) * D;
#pragma unroll
  for (int i = 0; i < D; i += 16) {
    uint32_t w[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const __nv_fp8x2_storage_t lo =
          __nv_cvt_float2_to_fp8x2(make_float2(v[i + 4 * k] * inv, v[i + 4 * k + 1] * inv), __NV_SATFINITE, __NV_E4M3);
      const __nv_fp8x2_storage_t hi =
          __nv_cvt_float2_to_fp8x2(make_float2(v[i + 4 * k + 2] * inv, v[i + 4 * k + 3] * inv), __NV_SATFINITE, __NV_E4M3);
      w[k] = static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
    }
    *reinterpret_cast<uint4*>(dst + i) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

template <typename T>
int launch_quant(const LvsaTensor* in, int B, int n, int H, int D, void* out8, float* scales, float* head_max,
                 cudaStream_t s) {
  dim3 grid((n + 127) / 128, H, B);
  const T* p = static_cast<const T*>(in->ptr);
  if (D == 128)
    quantize_kernel<T, 128><<<grid, 128, 0, s>>>(p, in->stride_b, in->stride_t, in->stride_h, n, H,
                                                static_cast<uint8_t*>(out8), scales, head_max);
  else if (D == 64)
    quantize_kernel<T, 64><<<grid, 128, 0, s>>>(p, in->stride_b, in->stride_t, in->stride_h, n, H,
                                               static_cast<uint8_t*>(out8), scales, head_max);
  else
    return LVSA_ERR_UNSUPPORTED;
  return cudaGetLastError() == cudaSuccess ? LVSA_OK : LVSA_ERR_CUDA;
}

}  // namespace
}  // namespace lvsa

extern "C" int lvsa_quantize_e4m3(const LvsaTensor* in, int32_t dtype, int32_t batch, int32_t n, int32_t heads,
                                  int32_t head_dim, void* out8, float* scales, float* head_max, void* stream) {
  if (!in || !in->ptr || !out8 || !scales || batch < 1 || n < 1 || heads < 1) return LVSA_ERR_INVALID_ARG;
  if ((reinterpret_cast<uintptr_t>(out8) & 15)) return LVSA_ERR_ALIGNMENT;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == LVSA_DTYPE_BF16)
    return lvsa::launch_quant<__nv_bfloat16>(in, batch, n, heads, head_dim, out8, scales, head_max, s);
  if (dtype == LVSA_DTYPE_F16) return lvsa::launch_quant<__half>(in, batch, n, heads, head_dim, out8, scales, head_max, s);
  return LVSA_ERR_UNSUPPORTED;
}
