// Batched strided row copies: the gather / scatter steps of the Ulysses
// exchange in one launch.  Each segment moves batch x rows x heads vectors of
// `row_bytes` (one head's head_dim values) between two [B, N, H, *] views
// with arbitrary byte strides.  HBM-bound: one read and one write per byte.
//
// The work is flattened over 16-byte chunks of every segment; a thread finds
// its segment by binary search over the chunk prefix (at most
// LVSA_MAX_COPY_SEGMENTS entries, kept in the kernel's parameter space), so
// consecutive threads move consecutive 16-byte pieces of one row: coalesced
// reads and writes whatever the segments' sizes.
#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/lvsa_b200.h"

namespace lvsa {
namespace {

struct CopyParams {
  LvsaCopySegment seg[LVSA_MAX_COPY_SEGMENTS];
  int64_t prefix[LVSA_MAX_COPY_SEGMENTS + 1];  // chunk offsets
  int32_t n;
  int32_t chunks_per_row;  // row_bytes / 16
};

__global__ void __launch_bounds__(256) copy_segments_kernel(const __grid_constant__ CopyParams p) {
  const int64_t total = p.prefix[p.n];
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t c = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; c < total; c += stride) {
    int lo = 0, hi = p.n - 1;  // last segment with prefix <= c
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (p.prefix[mid] <= c) lo = mid;
      else hi = mid - 1;
    }
    const LvsaCopySegment& s = p.seg[lo];
    const int64_t local = c - p.prefix[lo];
    const int64_t vec = local / p.chunks_per_row;
    const int part = static_cast<int>(local - vec * p.chunks_per_row);
    const int64_t h = vec % s.heads;
    const int64_t rt = vec / s.heads;
    const int64_t t = rt % s.rows;
    const int64_t b = rt / s.rows;
    const char* src = static_cast<const char*>(s.src) + b * s.src_sb + t * s.src_st + h * s.src_sh + part * 16;
    char* dst = static_cast<char*>(s.dst) + b * s.dst_sb + t * s.dst_st + h * s.dst_sh + part * 16;
    *reinterpret_cast<uint4*>(dst) = __ldg(reinterpret_cast<const uint4*>(src));
  }
}

}  // namespace
}  // namespace lvsa

extern "C" int lvsa_copy_segments(const LvsaCopySegment* segs, int32_t n, int32_t row_bytes, void* stream) {
  using namespace lvsa;
  if (n < 0 || n > LVSA_MAX_COPY_SEGMENTS || (n > 0 && !segs)) return LVSA_ERR_INVALID_ARG;
  if (row_bytes < 16 || row_bytes % 16) return LVSA_ERR_ALIGNMENT;
  CopyParams p;
  p.n = 0;
  p.chunks_per_row = row_bytes / 16;
  p.prefix[0] = 0;
  for (int i = 0; i < n; ++i) {
    const LvsaCopySegment& s = segs[i];
    if (s.batch < 0 || s.rows < 0 || s.heads < 0) return LVSA_ERR_INVALID_ARG;
    const int64_t vecs = static_cast<int64_t>(s.batch) * s.rows * s.heads;
    if (vecs == 0) continue;
    if (!s.src || !s.dst) return LVSA_ERR_INVALID_ARG;
    if ((reinterpret_cast<uintptr_t>(s.src) | reinterpret_cast<uintptr_t>(s.dst)) & 15) return LVSA_ERR_ALIGNMENT;
    if ((s.src_sb | s.src_st | s.src_sh | s.dst_sb | s.dst_st | s.dst_sh) & 15) return LVSA_ERR_ALIGNMENT;
    p.seg[p.n] = s;
    p.prefix[p.n + 1] = p.prefix[p.n] + vecs * p.chunks_per_row;
    ++p.n;
  }
  if (p.n == 0) return LVSA_OK;
  const int64_t total = p.prefix[p.n];
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t want = (total + 255) / 256;
  const int blocks = static_cast<int>(want < static_cast<int64_t>(sms) * 8 ? want : static_cast<int64_t>(sms) * 8);
  copy_segments_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(p);
  return cudaGetLastError() == cudaSuccess ? LVSA_OK : LVSA_ERR_CUDA;
}
