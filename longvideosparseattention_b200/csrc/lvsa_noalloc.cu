// FP8 block-sparse attention with no device allocation, for callers that
// cannot call cudaMalloc (a serving runtime that owns all device memory
// through its own pool, a host binding with no CUDA allocator, a loop that
// must keep its footprint constant).  The E4M3 copies of the inputs, their
// tile scales and the per-head V reference go to one file-scope device array
// instead of memory allocated per call.  Capacity and concurrency rules are
// stated beside the declaration of lvsa_attn_fwd_fp8_noalloc in lvsa_b200.h.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "../../include/lvsa_b200.h"

namespace {

// Held by every GPU that loads the library, until the process exits.
static __device__ __align__(256) uint8_t g_noalloc_scratch[LVSA_NOALLOC_SCRATCH_BYTES];

// The device address of g_noalloc_scratch, per CUDA context (the array is
// instantiated once per context that loads this module, so an address found
// in one context is not valid in another, even on the same device).
struct ScratchSlot {
  CUcontext ctx;
  uint8_t* addr;
};
constexpr int kMaxContexts = 64;
ScratchSlot g_slots[kMaxContexts] = {};
int g_n_slots = 0;
std::mutex g_setup_mutex;

using CtxGetCurrentFn = CUresult (*)(CUcontext*);

CtxGetCurrentFn ctx_get_current() {
  static CtxGetCurrentFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrentFn>(p);
  });
  return fn;
}

// In host code g_noalloc_scratch names a host-side stand-in; the device
// address is looked up once per context, with that context current.
int scratch_address(uint8_t** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) return LVSA_ERR_CUDA;
  CtxGetCurrentFn get = ctx_get_current();
  CUcontext ctx = nullptr;
  if (!get || get(&ctx) != CUDA_SUCCESS) return LVSA_ERR_CUDA;
  if (!ctx) {
    // No context current yet: the runtime call makes the device's primary
    // context current as a side effect.
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || get(&ctx) != CUDA_SUCCESS || !ctx)
      return LVSA_ERR_CUDA;
  }
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  for (int i = 0; i < g_n_slots; ++i)
    if (g_slots[i].ctx == ctx) {
      *out = g_slots[i].addr;
      return LVSA_OK;
    }
  if (g_n_slots == kMaxContexts) return LVSA_ERR_CAPACITY;
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) return LVSA_ERR_CUDA;
  g_slots[g_n_slots++] = ScratchSlot{ctx, static_cast<uint8_t*>(p)};
  *out = static_cast<uint8_t*>(p);
  return LVSA_OK;
}

size_t round256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

}  // namespace

namespace lvsa {
int validate_attn_args(const LvsaAttnArgs* a);
}

extern "C" int lvsa_attn_fwd_fp8_noalloc(const LvsaAttnArgs* a, void* stream) {
  // Every check lvsa_attn_fwd_fp8 makes, before anything is cleared or
  // launched: a rejected call leaves the scratch array and the GPU untouched.
  int st = lvsa::validate_attn_args(a);
  if (st != LVSA_OK) return st;
  if (a->dtype != LVSA_DTYPE_BF16 && a->dtype != LVSA_DTYPE_F16) return LVSA_ERR_UNSUPPORTED;
  if (a->head_dim != 128) return LVSA_ERR_UNSUPPORTED;
  const bool has_text = a->n_text > 0;
  const bool text_rows = has_text && a->text_q.ptr != nullptr;
  if (has_text && (!a->text_k.ptr || !a->text_v.ptr)) return LVSA_ERR_INVALID_ARG;

  const size_t B = a->batch, Nv = a->n_video, Nt = a->n_text, H = a->heads, Hk = a->kv_heads, D = a->head_dim;
  const size_t Nk = a->n_kv_video > 0 ? a->n_kv_video : Nv;  // video keys
  const size_t tv = (Nv + 127) / 128, tk = (Nk + 127) / 128, tt = (Nt + 127) / 128;
  // Scratch layout: each part starts on a 256-byte boundary.
  size_t off = 0;
  auto take = [&off](size_t bytes) {
    const size_t at = off;
    off += round256(bytes);
    return at;
  };
  const size_t o_q = take(B * Nv * H * D), o_k = take(B * Nk * Hk * D), o_v = take(B * Nk * Hk * D);
  const size_t o_tq = text_rows ? take(B * Nt * H * D) : 0;
  const size_t o_tk = has_text ? take(B * Nt * Hk * D) : 0;
  const size_t o_tv = has_text ? take(B * Nt * Hk * D) : 0;
  const size_t o_sq = take(B * H * tv * 4), o_sk = take(B * Hk * tk * 4), o_sv = take(B * Hk * tk * 4);
  const size_t o_stq = text_rows ? take(B * H * tt * 4) : 0;
  const size_t o_stk = has_text ? take(B * Hk * tt * 4) : 0;
  const size_t o_stv = has_text ? take(B * Hk * tt * 4) : 0;
  const size_t o_ref = take(B * Hk * 4);
  if (off > LVSA_NOALLOC_SCRATCH_BYTES) return LVSA_ERR_CAPACITY;

  uint8_t* base = nullptr;
  st = scratch_address(&base);
  if (st != LVSA_OK) return st;
  auto f32 = [base](size_t at) { return reinterpret_cast<float*>(base + at); };
  // The V reference is a running atomic max over this call's tiles: clear it.
  if (cudaMemsetAsync(f32(o_ref), 0, B * Hk * 4, static_cast<cudaStream_t>(stream)) != cudaSuccess)
    return LVSA_ERR_CUDA;

  const int dt = a->dtype, b = a->batch, h = a->heads, hk = a->kv_heads, d = a->head_dim;
  if ((st = lvsa_quantize_e4m3(&a->q, dt, b, a->n_video, h, d, base + o_q, f32(o_sq), nullptr, stream))) return st;
  const int nk = static_cast<int>(Nk);
  if ((st = lvsa_quantize_e4m3(&a->k, dt, b, nk, hk, d, base + o_k, f32(o_sk), nullptr, stream))) return st;
  if ((st = lvsa_quantize_e4m3(&a->v, dt, b, nk, hk, d, base + o_v, f32(o_sv), f32(o_ref), stream)))
    return st;
  if (has_text) {
    if ((st = lvsa_quantize_e4m3(&a->text_k, dt, b, a->n_text, hk, d, base + o_tk, f32(o_stk), nullptr, stream)))
      return st;
    if ((st = lvsa_quantize_e4m3(&a->text_v, dt, b, a->n_text, hk, d, base + o_tv, f32(o_stv), f32(o_ref),
                                 stream)))
      return st;
  }
  if (text_rows &&
      (st = lvsa_quantize_e4m3(&a->text_q, dt, b, a->n_text, h, d, base + o_tq, f32(o_stq), nullptr, stream)))
    return st;

  // The caller's arguments, pointed at the contiguous E4M3 copies
  // ([B, N, heads, D] bytes, strides in elements of one byte).
  LvsaAttnArgs q8 = *a;
  auto view = [base, D](size_t at, size_t n, size_t heads) {
    LvsaTensor t;
    t.ptr = base + at;
    t.stride_h = static_cast<int64_t>(D);
    t.stride_t = static_cast<int64_t>(heads * D);
    t.stride_b = static_cast<int64_t>(n * heads * D);
    return t;
  };
  q8.q = view(o_q, Nv, H);
  q8.k = view(o_k, Nk, Hk);
  q8.v = view(o_v, Nk, Hk);
  if (has_text) {
    q8.text_k = view(o_tk, Nt, Hk);
    q8.text_v = view(o_tv, Nt, Hk);
  }
  if (text_rows) q8.text_q = view(o_tq, Nt, H);
  LvsaFp8Scales sc;
  sc.q = f32(o_sq);
  sc.k = f32(o_sk);
  sc.v = f32(o_sv);
  sc.text_q = text_rows ? f32(o_stq) : nullptr;
  sc.text_k = has_text ? f32(o_stk) : nullptr;
  sc.text_v = has_text ? f32(o_stv) : nullptr;
  sc.v_ref = f32(o_ref);
  return lvsa_attn_fwd_fp8(&q8, &sc, stream);
}
