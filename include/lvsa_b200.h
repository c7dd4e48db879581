/*
 * lvsa_b200.h -- C ABI of the B200 (sm_100a) LVSA block-sparse attention path.
 *
 * Plain C: pointers, sizes and status codes; no torch or CUDA types in the
 * signatures (a stream is passed as `void*`, i.e. a cudaStream_t / CUstream).
 * Every buffer is caller-owned device memory; nothing here allocates device
 * memory and nothing throws across the boundary.  A non-zero return is one of
 * the LVSA_* status codes below; lvsa_status_str() names it.
 *
 * The reference (JiusiServe/LongVideoSparseAttention v1.2.0) has no native
 * code; each entry point names the Python interface it replaces.
 */
#ifndef LVSA_B200_H_
#define LVSA_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  LVSA_OK = 0,
  LVSA_ERR_INVALID_ARG = 1,  /* null pointer, negative size, bad enum            */
  LVSA_ERR_GEOMETRY = 2,     /* pattern/sequence geometry inconsistent           */
  LVSA_ERR_UNSUPPORTED = 3,  /* head_dim / dtype / block size not built          */
  LVSA_ERR_ALIGNMENT = 4,    /* pointer or stride violates the 16-byte TMA rule  */
  LVSA_ERR_CAPACITY = 5,     /* a buffer is too small: the caller's (vs
                                lvsa_mask_layout) or the library's fixed
                                no-allocation scratch                          */
  LVSA_ERR_CUDA = 6,         /* a CUDA runtime call failed                       */
  LVSA_ERR_DEVICE_TIMEOUT = 7 /* a kernel's bounded wait expired (error word)    */
};

enum { LVSA_DTYPE_BF16 = 0, LVSA_DTYPE_F16 = 1 };

/* Largest total_frames the mask builder accepts. */
#define LVSA_MAX_FRAMES 2048

/* Sparsity pattern of one denoising step (world = 1 semantics).
 * Mirrors LVSAMetadata.build(total_latent_frames, num_patches, window_size,
 * n_first_frames, key_frame_interval, rank=0, world=1, expand_window,
 * keyframe_offset, boundary_guards)  -- lvsa/sparse_attention.py:339-353.  */
typedef struct LvsaPattern {
  int32_t total_frames;       /* T                                          */
  int32_t num_patches;        /* P, tokens per latent frame                 */
  int32_t window_size;        /* W (0 = globals only)                       */
  int32_t n_first_frames;     /* anchor frames 0..n_first-1                 */
  int32_t key_frame_interval; /* <= 0 means None                            */
  int32_t keyframe_offset;    /* step % kfi                                 */
  int32_t expand_window;      /* 0/1                                        */
  int32_t n_text;             /* text tokens (own segment, dense)           */
  int32_t block_q;            /* query tile rows (multiple of 16, <= 256)   */
  int32_t block_k;            /* key tile columns (multiple of 16, <= 256)  */
  int32_t n_guards;           /* extra global frames (boundary guards)      */
  const int32_t* guards;      /* HOST array of n_guards frame indices       */
  /* Optional DEVICE int32 (ABI 102): the denoising step index.  When set,
   * the builder reads it on the GPU and uses step % key_frame_interval as
   * the keyframe offset (keyframe_offset is then ignored), so a captured
   * CUDA graph or a shared mask rotates by updating one device word. */
  const int32_t* device_step;
} LvsaPattern;

/* Sizes of every output of lvsa_build_mask for a pattern. */
typedef struct LvsaMaskLayout {
  int32_t n_video;           /* T * P                                        */
  int32_t n_q_video_tiles;   /* ceil(n_video / block_q)                      */
  int32_t n_q_tiles;         /* + ceil(n_text / block_q) text query tiles    */
  int32_t n_k_video_tiles;   /* ceil(n_video / block_k)                      */
  int32_t n_k_tiles;         /* + ceil(n_text / block_k) text key tiles      */
  int32_t frame_words;       /* ceil(T / 32): words per attended-frame bitset */
  int64_t max_nnz;           /* capacity needed for tile_indices/tile_flags  */
} LvsaMaskLayout;

/* Device output buffers of lvsa_build_mask (all caller-owned). */
typedef struct LvsaMaskBuffers {
  int8_t* global_frame_mask;   /* [T]            LVSAMetadata.global_frame_mask */
  int32_t* window_bounds;      /* [T, 2]         LVSAMetadata.window_bounds     */
  uint32_t* frame_bits;        /* [T, frame_words] attended frames per frame  */
  int32_t* attended_indices;   /* [T, T] row-padded; columns [0, C) equal
                                  LVSAMetadata.attended_indices                 */
  int32_t* frame_indptr;       /* [T + 1]        LVSAMetadata.fi_indptr         */
  int32_t* frame_indices;      /* [T * T] first frame_nnz = LVSAMetadata.fi_indices */
  int32_t* tile_indptr;        /* [n_q_tiles + 1] tile CSR row pointers        */
  int32_t* tile_indices;       /* [max_nnz]      active key tiles, ascending    */
  uint8_t* tile_flags;         /* [max_nnz]      bit0: tile needs in-tile mask  */
  int32_t* counters;           /* [4]: tile nnz, attended C, frame nnz, compact_n */
} LvsaMaskBuffers;

/* Host-only: sizes for a pattern.  Replaces nothing in the reference (its
 * builder sizes Python lists as it goes). */
int lvsa_mask_layout(const LvsaPattern* pattern, LvsaMaskLayout* layout);

/* GPU mask builder: frame-level pattern + tile CSR for one denoising step,
 * enqueued on `stream` (no host synchronisation).
 * Replaces LVSAMetadata.build + _build_attended_indices + _build_flashinfer_csr
 * (lvsa/sparse_attention.py:335-484, :510-547, :550-635), which the reference
 * re-runs on the host at every keyframe rotation (lvsa/lvsa_processor.py:362-405). */
int lvsa_build_mask(const LvsaPattern* pattern, const LvsaMaskBuffers* out, void* stream);

/* A [B, N, heads, head_dim] tensor view: element strides, last dim contiguous. */
typedef struct LvsaTensor {
  void* ptr;
  int64_t stride_b;
  int64_t stride_t;
  int64_t stride_h;
} LvsaTensor;

typedef struct LvsaAttnArgs {
  /* video segment: q/o [B, n_video, heads, D]; k/v [B, n_video, kv_heads, D] */
  LvsaTensor q, k, v, o;
  /* text segment (n_text tokens): text_k/text_v required when n_text > 0;
   * text_q/text_o optional (NULL ptr: text query rows are skipped).          */
  LvsaTensor text_q, text_k, text_v, text_o;
  float* lse;       /* optional [B, heads, n_video] natural-log LSE (fp32) */
  float* text_lse;  /* optional [B, heads, n_text]                          */
  int32_t batch, n_video, n_text, heads, kv_heads, head_dim, dtype;
  float scale;      /* <= 0: 1/sqrt(head_dim)                               */
  /* pattern + tile CSR from lvsa_build_mask (block_q = block_k = 128) */
  int32_t total_frames, num_patches, frame_words, block_q, block_k;
  int32_t n_q_video_tiles, n_q_tiles, n_k_video_tiles;
  const uint32_t* frame_bits;
  const int32_t* tile_indptr;
  const int32_t* tile_indices;
  const uint8_t* tile_flags;
  int32_t* error_word; /* optional device int: LVSA_ERR_DEVICE_TIMEOUT on a stalled wait */
  /* Sequence shards (context parallelism, ABI 101): the video segment holds
   * global tokens [token_offset, token_offset + n_video) of the T x P grid;
   * frames of query and key tokens are counted from there.  A whole
   * sequence is token_offset 0 and n_video = T x P. */
  int32_t token_offset;
  /* First tile-CSR row to compute (rows [first_q_tile, n_q_tiles)); 0: all. */
  int32_t first_q_tile;
  /* One past the last tile-CSR row to compute (ABI 102); <= 0: n_q_tiles.
   * With first_q_tile it selects a row range, e.g. one rank's share of a
   * head under head-and-tile partitioned Ulysses parallelism.  Rows outside
   * the range (and their LSE entries) are not written. */
  int32_t end_q_tile;
  /* Limit of every bounded wait inside the kernel, in microseconds (ABI
   * 102); <= 0: 2 s.  On expiry the CTA records LVSA_ERR_DEVICE_TIMEOUT in
   * *error_word, drains its own copies and MMAs, frees its tensor memory and
   * returns; the context stays usable. */
  int32_t wait_timeout_us;
  /* Test hook (0 in normal use): 1 makes CTA (0, 0, 0) skip its query-tile
   * load, so its waits expire and the path above runs. */
  int32_t inject_fault;
  /* Video KEY tokens in k / v when they differ from the query tokens (ABI
   * 102); <= 0: n_video.  A block-sparse layout whose key blocks are frames
   * of another sequence (the reference's compact FlashInfer K/V): key token
   * j belongs to frame (token_offset + j) / num_patches of frame_bits'
   * column space, n_k_video_tiles = ceil(n_kv_video / block_k). */
  int32_t n_kv_video;
} LvsaAttnArgs;

/* Block-sparse attention forward on tcgen05/TMEM, K/V read in place.
 * Replaces lvsa_sdpa (lvsa/sparse_attention.py:643-706), lvsa_flashinfer
 * (:709-742), DistributedLVSAProcessor._compute_lvsa_flashinfer with its text
 * LSE merge (lvsa/lvsa_processor.py:832-913) and the dense encoder-query
 * attention _compute_full_attention (:710-735): video rows attend their
 * frame's attended set plus all text, text rows attend everything. */
int lvsa_attn_fwd(const LvsaAttnArgs* args, void* stream);

/* ---------------------------------------------------------------- FP8 mode
 * E4M3 QK / PV with per-tile scales (no counterpart in the reference, which
 * has no FP8 path; BASELINE cfg3 asks for this variant).
 *   Q, K: one scale per (batch, head, 128-token tile) = amax / 448.
 *   V:    one scale per (batch, head, 128-token tile) plus a per-(batch, head)
 *         reference (the max tile scale); the kernel folds scale_j / reference
 *         into P before rounding it to E4M3, and multiplies O by the reference.
 */
enum { LVSA_DTYPE_E4M3 = 2 };

/* Quantise one [B, N, heads, D] bf16/f16 tensor to a contiguous
 * [B, N, heads, D] E4M3 copy `out8` with scales [B, heads, ceil(N/128)].
 * `head_max` (optional, [B, heads] fp32) receives atomicMax of the tile scales
 * and must hold zeros (or a smaller running max) before the call. */
int lvsa_quantize_e4m3(const LvsaTensor* in, int32_t dtype, int32_t batch, int32_t n, int32_t heads,
                       int32_t head_dim, void* out8, float* scales, float* head_max, void* stream);

typedef struct LvsaFp8Scales {
  const float* q;       /* [B, heads, ceil(n_video/128)]       */
  const float* k;       /* [B, kv_heads, ceil(n_video/128)]    */
  const float* v;       /* [B, kv_heads, ceil(n_video/128)]    */
  const float* text_q;  /* [B, heads, ceil(n_text/128)] or NULL  */
  const float* text_k;
  const float* text_v;
  const float* v_ref;   /* [B, kv_heads]: max V tile scale over video + text */
} LvsaFp8Scales;

/* FP8 attention: `args` as for lvsa_attn_fwd with q/k/v/text_* pointing at the
 * E4M3 copies (contiguous [B, N, H, D] bytes; strides in elements = bytes) and
 * `dtype` naming the OUTPUT type (bf16 or f16).  head_dim 128 only. */
int lvsa_attn_fwd_fp8(const LvsaAttnArgs* args, const LvsaFp8Scales* scales, void* stream);

/* ---- QK prologue: per-token norm + rotary embedding, fused, in place ----
 * Replaces, for one of q or k, the two elementwise passes the adapters run
 * before attention: the QK norm and the interleaved-pair RoPE
 *   Wan:          norm_q/norm_k = RMSNorm over the H*D row
 *                 (lvsa/adapters/wan.py:48-67) + apply_rotary_emb
 *                 (lvsa/rope.py:10-28, lvsa/adapters/wan.py:103-119)
 *   HunyuanVideo: RMSNorm per head (lvsa/adapters/hunyuan_video.py:71-103)
 *                 + RoPE on video tokens (:156-205)
 *   CogVideoX:    LayerNorm per head (lvsa/adapters/cogvideox.py:88-117)
 *                 + RoPE on video tokens (:169-217)
 * x [B, S, H, D] is read once and written once (fp32 arithmetic, one
 * rounding to the storage type).  RoPE: pair (x0, x1) at dims (2p, 2p+1)
 * becomes (x0 c - x1 s, x0 s + x1 c) with c = cos[t][p], s = sin[t][p] for
 * token t = rope_offset + position in x; cos/sin are [*, S_table, D/2] fp32
 * (the even entries of the reference's cos table and the odd entries of its
 * sin table).  cos = NULL: norm only (text tokens). */
enum { LVSA_DTYPE_F32 = 3 };
enum {
  LVSA_NORM_NONE = 0,
  LVSA_NORM_RMS_ROW = 1,   /* RMS over all H*D values of a token; weight [H*D] */
  LVSA_NORM_RMS_HEAD = 2,  /* RMS over each head's D values; weight [D]        */
  LVSA_NORM_LAYER_HEAD = 3 /* LayerNorm over each head's D values; weight, bias [D] */
};
typedef struct LvsaQkPrologue {
  LvsaTensor x;            /* in/out, stride 1 over D, 16-byte aligned rows     */
  int32_t dtype;           /* LVSA_DTYPE_BF16 / _F16                            */
  int32_t batch, seq, heads, head_dim; /* head_dim 64 or 128; H*D <= 8192       */
  int32_t norm;            /* LVSA_NORM_*                                       */
  int32_t weight_dtype;    /* LVSA_DTYPE_BF16 / _F16 / _F32 (weight and bias)   */
  const void* weight;      /* NULL: no scale                                    */
  const void* bias;        /* LayerNorm only; NULL: no shift                    */
  float eps;
  const float* cos;        /* NULL: no rotary embedding                         */
  const float* sin;
  int64_t rope_stride_b;   /* elements between batches of the tables; 0: shared */
  int32_t rope_offset;     /* table row of x's first token (sequence shards)    */
} LvsaQkPrologue;
int lvsa_qk_prologue(const LvsaQkPrologue* args, void* stream);

/* FP8 attention that allocates no device memory.  No counterpart in the
 * reference: an addition of this library.
 *
 * For callers that cannot call cudaMalloc on this path: serving runtimes
 * whose device memory is a fixed pool owned by their own allocator, hosts
 * that bind this library from a language runtime with no CUDA allocator,
 * and loops that must keep a constant memory footprint.  Arguments are those
 * of lvsa_attn_fwd (bf16/f16 q, k, v and optional text inputs, outputs, the
 * tile CSR); the inputs are quantised to E4M3 into a scratch array owned by
 * the library, then the lvsa_attn_fwd_fp8 kernel runs on them.
 *
 *  - Limit: LVSA_NOALLOC_SCRATCH_BYTES (96 MiB) of scratch, which every GPU
 *    that loads the library holds until the process exits.  A call needs the
 *    E4M3 copies of q, k, v (+ text q, k, v), one fp32 scale per 128-token
 *    tile and head of each, and one fp32 per batch and K/V head, each part
 *    rounded up to 256 bytes; a larger call returns LVSA_ERR_CAPACITY and
 *    launches nothing.
 *  - The first call in each CUDA context (normally a device's primary
 *    context) looks up the array's device address with that context
 *    current; make that first call before any stream capture.
 *  - Every argument check runs before anything is cleared or launched: a
 *    rejected call (bad geometry, null pointers, over capacity) leaves the
 *    scratch array and the stream untouched.
 *  - All calls share the one array and it keeps the previous call's
 *    contents; the part that must start at zero (the per-head V reference)
 *    is cleared by each call.  Calls that overlap on the GPU (different
 *    streams, or host threads on one device) race on the array: the caller
 *    must serialise them.
 *  - head_dim 128 only, as lvsa_attn_fwd_fp8. */
#define LVSA_NOALLOC_SCRATCH_BYTES (96u * 1024u * 1024u)
int lvsa_attn_fwd_fp8_noalloc(const LvsaAttnArgs* args, void* stream);

/* ---- output projection (the to_out Linear after attention) ----------
 * out[m, n] = sum_k a[m, k] * weight[n, k] (+ bias[n]) on tcgen05 / TMEM,
 * bf16 or f16 in and out, fp32 accumulation.  `a` is the attention output
 * read in place: an [B, S, H, D] token-major o is [m = B*S, k = H*D] with
 * lda = H*D (or its token stride); `weight` is an nn.Linear weight
 * [out_features, in_features].  Replaces attn.to_out[0] after the LVSA
 * attention (lvsa/adapters/wan.py:121-131, lvsa/adapters/hunyuan_video.py:
 * 207-217).  k must be a multiple of 64, n of 32; rows 16-byte aligned. */
typedef struct LvsaOutProjArgs {
  const void* a;       /* [m, k], row stride lda elements                      */
  const void* weight;  /* [n, k], row stride ldw elements                      */
  const void* bias;    /* [n] or NULL                                          */
  void* out;           /* [m, n], row stride ldo elements                      */
  int64_t lda, ldw, ldo;
  int32_t m, n, k, dtype;
  int32_t* error_word; /* optional device int: LVSA_ERR_DEVICE_TIMEOUT          */
} LvsaOutProjArgs;
int lvsa_out_proj(const LvsaOutProjArgs* args, void* stream);

/* ---- batched strided row copies (gather / scatter of an exchange) ----
 * No counterpart in the reference (its only multi-GPU exchange is one
 * all_reduce).  Packs and unpacks the Ulysses all-to-all buffers in one
 * launch: each segment copies batch x rows x heads vectors of `row_bytes`
 * from src to dst, element (b, t, h) at byte offset b*sb + t*st + h*sh of
 * each side.  Pointers, strides and row_bytes must be multiples of 16 bytes;
 * segments must not overlap in dst. */
#define LVSA_MAX_COPY_SEGMENTS 64
typedef struct LvsaCopySegment {
  const void* src;
  void* dst;
  int64_t src_sb, src_st, src_sh;  /* byte strides */
  int64_t dst_sb, dst_st, dst_sh;
  int32_t batch, rows, heads;
} LvsaCopySegment;
int lvsa_copy_segments(const LvsaCopySegment* segs, int32_t n, int32_t row_bytes, void* stream);

/* Human-readable name of a status code. */
const char* lvsa_status_str(int status);

/* ABI version (major * 100 + minor). */
int lvsa_abi_version(void);

#ifdef __cplusplus
}
#endif
#endif /* LVSA_B200_H_ */
