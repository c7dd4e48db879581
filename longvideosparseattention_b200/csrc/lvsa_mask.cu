// GPU mask builder: the LVSA anchor / rotating-keyframe / expanded-window
// pattern of one denoising step -> frame-level structures + tile CSR.
//
// Kernel 1 (one CTA): global set, per-frame window bounds, attended bitsets,
//   attended_indices, frame-level compact CSR.  Restates
//   lvsa/sparse_attention.py:40-104 (windows), :198-216 (globals),
//   :335-484 (build), :510-547, :550-635 (frame CSR).
// Kernel 2 (one warp per query tile): count active key tiles.
// Kernel 3 (one CTA): exclusive scan of the counts -> tile_indptr.
// Kernel 4 (one warp per query tile): write tile indices and mask flags.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstring>

#include "../../include/lvsa_b200.h"

namespace lvsa {
namespace {

constexpr int kMaxWords = LVSA_MAX_FRAMES / 32;

struct FrameParams {
  int T, P, W, n_first, kfi, offset, expand, words;
  const int32_t* step;  // device step index (offset = step mod kfi), or null
  uint32_t guard_bits[kMaxWords];
};

struct TileParams {
  int T, P, words, n_video, n_text, BQ, BK, nqv, nq, nkv, nkt;
};

__device__ __forceinline__ bool test_bit(const uint32_t* bits, int f) {
  return (bits[f >> 5] >> (f & 31)) & 1u;
}

// Bits [lo, hi] (inclusive) restricted to word w.
__device__ __forceinline__ uint32_t range_word(int w, int lo, int hi) {
  if (lo > hi) return 0u;
  const int a = max(lo, w * 32), b = min(hi, w * 32 + 31);
  if (a > b) return 0u;
  const int n = b - a + 1;
  const uint32_t m = (n == 32) ? 0xFFFFFFFFu : ((1u << n) - 1u);
  return m << (a - w * 32);
}

__global__ void __launch_bounds__(1024) frame_pattern_kernel(FrameParams prm, LvsaMaskBuffers out) {
  __shared__ uint32_t gbits[kMaxWords];
  __shared__ uint32_t allbits[kMaxWords];
  __shared__ int cprefix[kMaxWords];
  __shared__ int counts[LVSA_MAX_FRAMES];
  __shared__ int s_gcount, s_maxc;
  const int T = prm.T, W = prm.W, words = prm.words, tid = threadIdx.x, nt = blockDim.x;

  for (int w = tid; w < words; w += nt) gbits[w] = prm.guard_bits[w];
  if (tid == 0) { s_gcount = 0; s_maxc = 0; }
  __syncthreads();
  for (int i = tid; i < min(prm.n_first, T); i += nt) atomicOr(&gbits[i >> 5], 1u << (i & 31));
  if (prm.kfi > 0) {
    const int nk = (T + prm.kfi - 1) / prm.kfi;
    const int off = prm.step ? ((*prm.step % prm.kfi) + prm.kfi) % prm.kfi : prm.offset;
    for (int i = tid; i < nk; i += nt) {
      long long x = static_cast<long long>(off) + static_cast<long long>(i) * prm.kfi;
      int g = static_cast<int>(((x % T) + T) % T);  // Python modulo
      atomicOr(&gbits[g >> 5], 1u << (g & 31));
    }
  }
  __syncthreads();
  for (int w = tid; w < words; w += nt) atomicAdd(&s_gcount, __popc(gbits[w]));
  __syncthreads();
  const int gcount = s_gcount;

  for (int f = tid; f < T; f += nt) {
    int lo, hi;
    if (W == 0) {
      lo = f; hi = f - 1;
    } else {
      lo = max(0, min(f - W, T - 1 - 2 * W));
      hi = min(T - 1, max(f + W, 2 * W));
      if (prm.expand) {
        const int need = min(2 * W + 1, T - gcount);
        int have = 0;
        for (int x = lo; x <= hi; ++x) have += test_bit(gbits, x) ? 0 : 1;
        while (have < need) {
          bool grew = false;
          if (lo > 0) { --lo; grew = true; if (!test_bit(gbits, lo)) ++have; }
          if (have >= need) break;
          if (hi < T - 1) { ++hi; grew = true; if (!test_bit(gbits, hi)) ++have; }
          if (!grew) break;
        }
      }
    }
    out.window_bounds[2 * f] = lo;
    out.window_bounds[2 * f + 1] = hi;
    out.global_frame_mask[f] = test_bit(gbits, f) ? 1 : 0;
    int c = 0;
    for (int w = 0; w < words; ++w) {
      const uint32_t b = gbits[w] | range_word(w, lo, hi);
      out.frame_bits[static_cast<size_t>(f) * words + w] = b;
      c += __popc(b);
    }
    counts[f] = c;
    atomicMax(&s_maxc, c);
  }
  __syncthreads();
  for (int w = tid; w < words; w += nt) {
    uint32_t a = 0;
    for (int f = 0; f < T; ++f) a |= out.frame_bits[static_cast<size_t>(f) * words + w];
    allbits[w] = a;
  }
  __syncthreads();
  if (tid == 0) {
    int acc = 0;
    for (int w = 0; w < words; ++w) { cprefix[w] = acc; acc += __popc(allbits[w]); }
    out.counters[3] = acc;  // compact_n
    int p = 0;
    out.frame_indptr[0] = 0;
    for (int f = 0; f < T; ++f) { p += counts[f]; out.frame_indptr[f + 1] = p; }
    out.counters[2] = p;
    out.counters[1] = s_maxc;
  }
  __syncthreads();
  for (int f = tid; f < T; f += nt) {
    const uint32_t* fb = out.frame_bits + static_cast<size_t>(f) * words;
    int32_t* row = out.attended_indices + static_cast<size_t>(f) * T;
    int32_t* fi = out.frame_indices + out.frame_indptr[f];
    int n = 0, last = 0;
    for (int w = 0; w < words; ++w) {
      uint32_t b = fb[w];
      while (b) {
        const int bit = __ffs(b) - 1;
        b &= b - 1;
        const int g = w * 32 + bit;
        row[n] = g;
        fi[n] = cprefix[w] + __popc(allbits[w] & ((1u << bit) - 1u));
        last = g;
        ++n;
      }
    }
    for (int i = n; i < T; ++i) row[i] = last;
  }
}

// One warp per query tile.  fill == false: write the count to tile_indptr[row+1].
// fill == true: write indices/flags starting at tile_indptr[row].
template <bool kFill>
__global__ void __launch_bounds__(256) tile_rows_kernel(TileParams prm, LvsaMaskBuffers out) {
  __shared__ uint32_t s_union[8][kMaxWords];
  __shared__ uint32_t s_inter[8][kMaxWords];
  const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
  const int row = blockIdx.x * 8 + wib;
  if (row >= prm.nq) return;
  const int nkv = prm.nkv, nkt = prm.nkt, BK = prm.BK, P = prm.P, Nv = prm.n_video;
  int pos = kFill ? out.tile_indptr[row] : 0;
  int count = 0;

  if (row < prm.nqv) {
    const int t0 = row * prm.BQ, t1 = min(Nv, t0 + prm.BQ);
    const int f0 = t0 / P, f1 = (t1 - 1) / P;
    uint32_t* U = s_union[wib];
    uint32_t* I = s_inter[wib];
    for (int w = lane; w < prm.words; w += 32) {
      uint32_t u = 0, it = 0xFFFFFFFFu;
      for (int f = f0; f <= f1; ++f) {
        const uint32_t b = out.frame_bits[static_cast<size_t>(f) * prm.words + w];
        u |= b;
        it &= b;
      }
      U[w] = u;
      I[w] = it;
    }
    __syncwarp();
    int carry = -1;  // highest key tile emitted so far
    for (int base = 0; base < prm.T; base += 32) {
      const int g = base + lane;
      const bool att = g < prm.T && test_bit(U, g);
      const long long gs = static_cast<long long>(g) * P;
      const int tlo = static_cast<int>(gs / BK);
      const int thi = static_cast<int>((min(static_cast<long long>(Nv), gs + P) - 1) / BK);
      int incl = att ? thi : -1;
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const int o = __shfl_up_sync(0xFFFFFFFFu, incl, d);
        if (lane >= d) incl = max(incl, o);
      }
      int excl = __shfl_up_sync(0xFFFFFFFFu, incl, 1);
      if (lane == 0) excl = -1;
      excl = max(excl, carry);
      const int start = max(tlo, excl + 1);
      const int cnt = att ? max(0, thi - start + 1) : 0;
      int off = cnt;
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const int o = __shfl_up_sync(0xFFFFFFFFu, off, d);
        if (lane >= d) off += o;
      }
      const int total = __shfl_sync(0xFFFFFFFFu, off, 31);
      off -= cnt;
      if (kFill) {
        for (int i = 0; i < cnt; ++i) {
          const int t = start + i;
          uint8_t flag = 0;
          if ((t + 1) * BK > Nv) {
            flag = 1;
          } else {
            const int fa = (t * BK) / P, fb = ((t + 1) * BK - 1) / P;
            for (int f = fa; f <= fb; ++f)
              if (!test_bit(I, f)) { flag = 1; break; }
          }
          out.tile_indices[pos + off + i] = t;
          out.tile_flags[pos + off + i] = flag;
        }
      }
      pos += total;
      count += total;
      carry = max(carry, __shfl_sync(0xFFFFFFFFu, incl, 31));
    }
    if (kFill) {
      for (int j = lane; j < nkt; j += 32) {
        out.tile_indices[pos + j] = nkv + j;
        out.tile_flags[pos + j] = ((j + 1) * BK > prm.n_text) ? 1 : 0;
      }
    }
    count += nkt;
  } else {
    if (kFill) {
      for (int t = lane; t < nkv + nkt; t += 32) {
        out.tile_indices[pos + t] = t;
        out.tile_flags[pos + t] =
            (t < nkv) ? (((t + 1) * BK > Nv) ? 1 : 0) : (((t - nkv + 1) * BK > prm.n_text) ? 1 : 0);
      }
    }
    count = nkv + nkt;
  }
  if (!kFill && lane == 0) out.tile_indptr[row + 1] = count;
}

// In-place inclusive scan of tile_indptr[1..n]; tile_indptr[0] = 0.
__global__ void __launch_bounds__(1024) scan_kernel(int n, LvsaMaskBuffers out) {
  __shared__ int warp_sums[32];
  __shared__ int s_carry;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  if (tid == 0) { s_carry = 0; out.tile_indptr[0] = 0; }
  __syncthreads();
  for (int base = 0; base < n; base += 1024) {
    const int i = base + tid;
    int v = (i < n) ? out.tile_indptr[i + 1] : 0;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int o = __shfl_up_sync(0xFFFFFFFFu, v, d);
      if (lane >= d) v += o;
    }
    if (lane == 31) warp_sums[wid] = v;
    __syncthreads();
    if (wid == 0) {
      int s = warp_sums[lane];
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const int o = __shfl_up_sync(0xFFFFFFFFu, s, d);
        if (lane >= d) s += o;
      }
      warp_sums[lane] = s;
    }
    __syncthreads();
    const int carry = s_carry;
    const int pre = (wid > 0 ? warp_sums[wid - 1] : 0) + carry;
    if (i < n) out.tile_indptr[i + 1] = v + pre;
    __syncthreads();
    if (tid == 0) s_carry = carry + warp_sums[31];
    __syncthreads();
  }
  if (tid == 0) out.counters[0] = s_carry;
}

int check_pattern(const LvsaPattern* p) {
  if (!p) return LVSA_ERR_INVALID_ARG;
  if (p->total_frames < 1 || p->total_frames > LVSA_MAX_FRAMES) return LVSA_ERR_GEOMETRY;
  if (p->num_patches < 1 || p->window_size < 0 || p->n_first_frames < 0 || p->n_text < 0)
    return LVSA_ERR_GEOMETRY;
  if (static_cast<long long>(p->total_frames) * p->num_patches > (1ll << 30)) return LVSA_ERR_GEOMETRY;
  if (p->block_q < 16 || p->block_q > 256 || p->block_q % 16) return LVSA_ERR_UNSUPPORTED;
  if (p->block_k < 16 || p->block_k > 256 || p->block_k % 16) return LVSA_ERR_UNSUPPORTED;
  if (p->n_guards < 0 || (p->n_guards > 0 && !p->guards)) return LVSA_ERR_INVALID_ARG;
  for (int i = 0; i < p->n_guards; ++i)
    if (p->guards[i] < 0 || p->guards[i] >= p->total_frames) return LVSA_ERR_GEOMETRY;
  return LVSA_OK;
}

}  // namespace
}  // namespace lvsa

using namespace lvsa;

extern "C" int lvsa_mask_layout(const LvsaPattern* p, LvsaMaskLayout* L) {
  const int st = check_pattern(p);
  if (st != LVSA_OK) return st;
  if (!L) return LVSA_ERR_INVALID_ARG;
  const long long T = p->total_frames, P = p->num_patches, nv = T * P;
  L->n_video = static_cast<int32_t>(nv);
  L->n_q_video_tiles = static_cast<int32_t>((nv + p->block_q - 1) / p->block_q);
  L->n_q_tiles = L->n_q_video_tiles + (p->n_text + p->block_q - 1) / p->block_q;
  L->n_k_video_tiles = static_cast<int32_t>((nv + p->block_k - 1) / p->block_k);
  const int nkt = (p->n_text + p->block_k - 1) / p->block_k;
  L->n_k_tiles = L->n_k_video_tiles + nkt;
  L->frame_words = static_cast<int32_t>((T + 31) / 32);
  // Upper bound per video row: frames its rows span x attended frames per
  // frame x key tiles a frame can touch, capped by the dense row.
  long long nglob = p->n_first_frames + p->n_guards;
  if (p->key_frame_interval > 0) nglob += (T + p->key_frame_interval - 1) / p->key_frame_interval;
  const long long per_frame = std::min(T, nglob + 2ll * p->window_size + 1);
  const long long span = (p->block_q + P - 1) / P + 1;
  const long long tiles_per_frame = (P + p->block_k - 1) / p->block_k + 1;
  const long long row_bound = std::min<long long>(L->n_k_video_tiles,
                                                  std::min(T, span * per_frame) * tiles_per_frame);
  const long long nqt = L->n_q_tiles - L->n_q_video_tiles;
  L->max_nnz = L->n_q_video_tiles * (row_bound + nkt) + nqt * L->n_k_tiles;
  return LVSA_OK;
}

extern "C" int lvsa_build_mask(const LvsaPattern* p, const LvsaMaskBuffers* out, void* stream) {
  LvsaMaskLayout L;
  int st = lvsa_mask_layout(p, &L);
  if (st != LVSA_OK) return st;
  if (!out || !out->global_frame_mask || !out->window_bounds || !out->frame_bits ||
      !out->attended_indices || !out->frame_indptr || !out->frame_indices || !out->tile_indptr ||
      !out->tile_indices || !out->tile_flags || !out->counters)
    return LVSA_ERR_INVALID_ARG;
  cudaStream_t s = static_cast<cudaStream_t>(stream);

  FrameParams fp;
  std::memset(&fp, 0, sizeof(fp));
  fp.T = p->total_frames; fp.P = p->num_patches; fp.W = p->window_size;
  fp.n_first = p->n_first_frames; fp.kfi = p->key_frame_interval; fp.offset = p->keyframe_offset;
  fp.expand = p->expand_window ? 1 : 0; fp.words = L.frame_words;
  fp.step = p->device_step;
  for (int i = 0; i < p->n_guards; ++i) fp.guard_bits[p->guards[i] >> 5] |= 1u << (p->guards[i] & 31);
  frame_pattern_kernel<<<1, 1024, 0, s>>>(fp, *out);

  TileParams tp;
  tp.T = p->total_frames; tp.P = p->num_patches; tp.words = L.frame_words; tp.n_video = L.n_video;
  tp.n_text = p->n_text; tp.BQ = p->block_q; tp.BK = p->block_k; tp.nqv = L.n_q_video_tiles;
  tp.nq = L.n_q_tiles; tp.nkv = L.n_k_video_tiles; tp.nkt = L.n_k_tiles - L.n_k_video_tiles;
  const int blocks = (L.n_q_tiles + 7) / 8;
  tile_rows_kernel<false><<<blocks, 256, 0, s>>>(tp, *out);
  scan_kernel<<<1, 1024, 0, s>>>(L.n_q_tiles, *out);
  tile_rows_kernel<true><<<blocks, 256, 0, s>>>(tp, *out);
  return cudaGetLastError() == cudaSuccess ? LVSA_OK : LVSA_ERR_CUDA;
}
