/*
 * dfm.h -- C ABI of the B200-native (sm_100a) MeanFlow flow-matching DiT head
 * of dots.tts ("FM head").
 *
 * The reference runs this head from Python: DotsBatchEngine._batched_fm
 * (nanovllm_dots/models/dots/engine.py:615-633) dispatches to a padded full
 * O(P^2) DiT forward per solver step (batched_fm.py:82-126) or, for the
 * flow-matching checkpoint only, to one per-request KV-cache head
 * (flash_cached_fm.py:279-360).  This library replaces that call: one
 * dfm_step per engine tick runs every in-flight request's graduating-row
 * extend plus all NFE MeanFlow steps against a paged per-(layer, step) K/V
 * cache, on the caller's CUDA stream, without host synchronisation.
 *
 * Conventions
 *   - Every pointer inside the structs below is a DEVICE pointer unless noted.
 *   - bf16 matrices are row-major [out, in] (the nn.Linear weight layout);
 *     biases and norm parameters are fp32.
 *   - The caller (PyTorch on the host side) owns every buffer: weights, the
 *     K/V pool, inputs, outputs and the workspace.  The library owns only the
 *     handle and its TMA descriptors.  dfm_step allocates nothing.
 *   - Functions return DFM_OK or a DFM_ERR_* code; they never throw.
 */
#ifndef DFM_H_
#define DFM_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DFM_OK 0
#define DFM_ERR_INVALID_ARG 1   /* a shape, pointer or length failed validation */
#define DFM_ERR_UNSUPPORTED 2   /* a configuration this build does not implement */
#define DFM_ERR_CUDA 3          /* a CUDA runtime/driver call failed */
#define DFM_ERR_WORKSPACE 4     /* workspace too small */
#define DFM_ERR_DEVICE 5        /* a kernel reported an error (dfm_read_error bits) */
#define DFM_ERR_SCRATCH_LIMIT 6 /* a call needs more than the fixed scratch of a no-allocation entry point */

/* DfmConfig.precision.  FP8: the QKV and fc1 projections run on e4m3 operands
 * (the cfg 3 path of the FP8 replacement of the reference's Int8DynamicLinear,
 * int8_dit.py:34-65): per-output-row weight scales from the caller and per-row
 * activation scales computed where the LayerNorm writes its rows; every other
 * GEMM stays bf16. */
#define DFM_PRECISION_BF16 0
#define DFM_PRECISION_FP8 1

/* Bits of the device error word returned by dfm_read_error. */
#define DFM_DEVERR_TIMEOUT 1u   /* a bounded in-kernel wait gave up */
#define DFM_DEVERR_PAGE 2u      /* a block-table entry was outside [0, num_pages) */
#define DFM_DEVERR_LEN 4u       /* a position exceeded the block-table width */

/* Model and pool shape.  Mirrors the checkpoint's DiT sub-config
 * (nanovllm_dots/models/dots/native/config.py:6-51, layers.py:141-144) plus
 * the engine-side sizes (DotsCore latent_dim/patch sizes, core.py:58-68). */
typedef struct DfmConfig {
  int32_t layers;            /* DiT blocks (12) */
  int32_t hidden;            /* model width H (1024; the only width this build supports) */
  int32_t heads;             /* attention heads (16) */
  int32_t head_dim;          /* 64 */
  int32_t ffn;               /* MLP width (4096) */
  int32_t latent_dim;        /* 64 */
  int32_t latent_patch;      /* latent rows per patch (16) */
  int32_t hidden_patch;      /* hidden rows per patch (1) */
  int32_t cond_dim;          /* LLM hidden width fed to hidden_proj (1536) */
  int32_t nfe;               /* MeanFlow solver steps (4, at most 8) */
  int32_t page_rows;         /* rows per K/V page (16) */
  int32_t num_pages;         /* pages in the pool */
  int32_t max_pages_per_req; /* block-table width */
  int32_t max_requests;      /* largest n a dfm_step may carry */
  float ln_eps;              /* LayerNorm eps (1e-5) */
  int32_t precision;         /* DFM_PRECISION_BF16 (0) or DFM_PRECISION_FP8 (1) */
} DfmConfig;

/* Weights.  Replaces the module tree read by the reference accelerators:
 * DiT leaves (native/dit.py:113-133, native/layers.py:152-161) and the core
 * projections (native/core.py:66-68). */
typedef struct DfmWeights {
  const void* input_w;   const float* input_b;    /* input_layer [H, H] */
  const void* temb_w1;   const float* temb_b1;    /* time_embedder.mlp.0 [H, 256] */
  const void* temb_w2;   const float* temb_b2;    /* time_embedder.mlp.2 [H, H] */
  const void* demb_w1;   const float* demb_b1;    /* duration_embedder.mlp.0 */
  const void* demb_w2;   const float* demb_b2;    /* duration_embedder.mlp.2 */
  const void* ada_w;     const float* ada_b;      /* [layers*6H + 2H, H]: every block's
                                                     adaLN_modulation.1, then the final
                                                     layer's */
  const void* qkv_w;                              /* [layers, 3H, H]: q_proj; k_proj; v_proj */
  const float* qk_norm;                           /* [layers, 4, head_dim]: q_norm w, b; k_norm w, b */
  const void* o_w;       const float* o_b;        /* [layers, H, H], [layers, H] */
  const void* fc1_w;     const float* fc1_b;      /* [layers, F, H], [layers, F] */
  const void* fc2_w;     const float* fc2_b;      /* [layers, H, F], [layers, H] */
  const void* final_w;   const float* final_b;    /* output_layer.linear [ld, H] */
  const void* coord_w;   const float* coord_b;    /* coordinate_proj [H, ld] */
  const void* hidden_w;  const float* hidden_b;   /* hidden_proj [H, cond_dim] */
  const void* latent_w;  const float* latent_b;   /* latent_proj [H, ld] */
  const float* rope_inv_freq;                     /* [head_dim/2], theta^(-2i/head_dim) */
  /* precision DFM_PRECISION_FP8 only (qkv_w and fc1_w may then be NULL):
   * e4m3 bytes of the same matrices with one fp32 scale per output row
   * (W ~= w8 * scale[row]; scale = row absmax / 448) */
  const void* qkv_w8;    const float* qkv_ws;     /* [layers, 3H, H] e4m3, [layers, 3H] */
  const void* fc1_w8;    const float* fc1_ws;     /* [layers, F, H] e4m3, [layers, F] */
} DfmWeights;

/* One engine tick for n requests.  Replaces the payload list handed to
 * DotsBatchEngine._batched_fm (engine.py:615-688): per request the history
 * rows that graduate into the cache this tick, the active hidden row, the
 * solver noise, g_cond and the request's cache position.
 *
 * Rows: each request graduates n_extend[i] rows (0 for its first patch, else
 * hidden_patch + latent_patch) at positions cache_len[i]..; its active rows
 * (hidden row + latent patch) follow at cache_len[i] + n_extend[i]...  Pass
 * either raw inputs (act_hidden / ext_hidden + ext_latent, projected here by
 * hidden_proj / latent_proj) or pre-projected rows (act_row / ext_rows). */
typedef struct DfmBatch {
  int32_t n;
  const void* noise;        /* bf16 [n, latent_patch, latent_dim] */
  const void* act_hidden;   /* bf16 [n, cond_dim] LLM hidden of this tick, or NULL */
  const void* act_row;      /* bf16 [n, H] hidden_proj output, or NULL */
  const void* ext_hidden;   /* bf16 [n, cond_dim] previous tick's LLM hidden, or NULL */
  const void* ext_latent;   /* bf16 [n, latent_patch, latent_dim] previous patch, or NULL */
  const void* ext_rows;     /* bf16 [n, hidden_patch + latent_patch, H] pre-projected, or NULL */
  const void* g_cond;       /* bf16 [n, H], or NULL for zeros */
  const int32_t* cache_len; /* [n] rows already in the cache */
  const int32_t* n_extend;  /* [n] graduating rows this tick */
  const int32_t* block_table; /* [n, max_pages_per_req] page ids */
  void* kv_pool;            /* bf16 pool, dfm_pool_bytes() bytes, zero-filled at allocation */
  void* out;                /* bf16 [n, latent_patch, latent_dim] next latent patch */
} DfmBatch;

/* Build a handle.  Validates the config, encodes the weight TMA descriptors.
 * Replaces the accelerator construction in DotsBatchEngine.__init__
 * (engine.py:125-185) and FlashCachedFMHead.__init__ (flash_cached_fm.py:84-110). */
int dfm_create(const DfmConfig* cfg, const DfmWeights* w, void** handle);

/* Bytes of workspace dfm_step needs for cfg->max_requests requests. */
size_t dfm_workspace_size(void* handle);

/* Bytes of the K/V pool for cfg: layers*nfe*2*num_pages*heads*page_rows*head_dim*2.
 * Replaces FlashFMCache's preallocation (flash_cached_fm.py:55-78). */
size_t dfm_pool_bytes(const DfmConfig* cfg);

/* Run one tick on `stream` (a cudaStream_t; NULL = legacy default stream).
 * Replaces DotsBatchEngine._batched_fm (engine.py:615-633) for MeanFlow, i.e.
 * the per-tick work of batched_meanflow (batched_fm.py:82-126) and of
 * FlashCachedFMHead.decode_patch (flash_cached_fm.py:350-360). */
int dfm_step(void* handle, const DfmBatch* batch, void* workspace, size_t workspace_bytes,
             void* stream);

/* Synchronise `stream` and read (then clear) the device error word the kernels
 * of the last dfm_step on this workspace set (DFM_DEVERR_* bits).  When the
 * word was non-zero it also zeroes the workspace's attention completion
 * counters, which a launch that stopped on an error may have left set. */
int dfm_read_error(void* handle, void* workspace, void* stream, uint32_t* err_word);

int dfm_destroy(void* handle);
const char* dfm_error_string(int code);

/* One of the per-layer launches of dfm_step, alone, with exactly the
 * arguments the tick gives it (same kernel, tiles, epilogue and workspace
 * buffers), for timing the tick's own kernels one at a time.  The inputs the
 * launch reads must hold what a dfm_step on the same batch and workspace left
 * there; a LayerNorm launch adds the pending sublayer into the residual stream
 * again, so run a full dfm_step before using its results.  No reference
 * counterpart: the reference times its stages with CUDA events around torch
 * calls (scripts/profile_mf_stages.py:25-48). */
#define DFM_TICK_LN_ATTN 0    /* residual + adaLN LayerNorm before the attention */
#define DFM_TICK_QKV 1        /* QKV GEMM + qk-norm + rotary + K/V append */
#define DFM_TICK_ATTENTION 2  /* paged prefix attention */
#define DFM_TICK_OPROJ 3      /* attention output projection (split-K partials) */
#define DFM_TICK_LN_MLP 4     /* residual + adaLN LayerNorm before the MLP */
#define DFM_TICK_FC1 5        /* fc1 + GELU(tanh) */
#define DFM_TICK_FC2 6        /* fc2 (split-K partials) */
int dfm_tick_launch(void* handle, const DfmBatch* batch, void* workspace, size_t workspace_bytes,
                    int32_t kernel, int32_t step, int32_t layer, void* stream);

/* ------------------------------------------------------------------ ops
 * Building blocks of the head, exported for unit tests and for callers that
 * compose their own pipeline. */

/* out[M, N] = act(A[M, K] . W[N, K]^T + bias) on tcgen05 tensor cores.
 * Replaces nn.Linear (autocast bf16) at the DiT call sites (native/layers.py:82-84,
 * 152-161; native/dit.py:26-30,53-58,76-79,122).  A and W bf16 row-major with
 * row strides lda/ldw elements; K % 64 == 0; N % 64 == 0; out_f32 selects
 * fp32 output; gelu applies GELU(tanh) after the bias.  bias may be NULL. */
int dfm_linear(const void* A, int64_t lda, int32_t M, int32_t K, const void* W, int64_t ldw,
               int32_t N, const float* bias, void* out, int32_t out_f32, int32_t gelu,
               void* stream);

/* The engine dispatch's per-tick input rows, gathered from each request's own
 * FM history buffer (gen_state.fm_sequence, engine.py:635-688 reads the same
 * rows) in one launch.  table: device int64 [n][4] = {address of the request's
 * history row 0 (bf16, row stride `hidden` elements, 16-byte aligned), first
 * graduating row, graduating row count (0..stride), address of its bf16
 * g_cond row or 0}.  Writes ext [n, stride, hidden] (rows past the count are
 * zero), act [n, hidden] (the row after the graduating rows: the active hidden
 * row) and g_cond [n, hidden] (zeros where the address is 0).  The caller
 * guarantees every row it names lies inside its buffer. */
int dfm_gather_rows(const int64_t* table, int32_t n, int32_t hidden, int32_t stride, void* act,
                    void* ext, void* g_cond, void* stream);

/* Paged prefix attention of one (layer, step) plane pair.  Replaces
 * flash_attn_with_kvcache in the cached FM head (flash_cached_fm.py:158-161)
 * and the SDPA calls of cached_fm.extend_cache/active_forward
 * (cached_fm.py:162,194).  q, out: bf16 [n*34, heads*64] in the 34-row
 * request layout (17 graduating rows, then 17 active rows); keys and values
 * come from pool planes plane_k / plane_v.  workspace holds split-key
 * partials: at least dfm_attention_workspace_size(n, max_pages, heads) bytes;
 * its first word is the device error word (DFM_DEVERR_* bits, ORed, never
 * cleared by the call); the call zeroes its completion counters itself. */
size_t dfm_attention_workspace_size(int32_t n, int32_t max_pages, int32_t heads);
int dfm_paged_attention(const void* q, void* out, const void* kv_pool, int32_t num_pages,
                        int32_t num_planes, int32_t heads, int32_t plane_k, int32_t plane_v,
                        const int32_t* cache_len, const int32_t* n_extend,
                        const int32_t* block_table, int32_t max_pages, int32_t n,
                        void* workspace, size_t workspace_bytes, void* stream);

/* Paged prefix attention with no workspace argument and no allocation.
 * This entry point has no counterpart in the reference.  It is for callers
 * that cannot allocate device memory at the point of the call, for example a
 * host framework whose allocator is not reachable from the thread that
 * launches work, or code running inside a tight memory budget that may not
 * grow.  It computes exactly what dfm_paged_attention computes; its split-key
 * partials and completion counters live in one fixed array inside the library
 * (DFM_NOALLOC_SCRATCH_BYTES on every GPU that loads the library, held until
 * the process exits) instead of a caller workspace.
 *   - Calls needing more than that scratch (dfm_attention_workspace_size(n,
 *     max_pages, heads) > DFM_NOALLOC_SCRATCH_BYTES) return
 *     DFM_ERR_SCRATCH_LIMIT and launch nothing.
 *   - The first call on a device looks up the scratch's device address (a
 *     synchronous runtime call); make that first call before any stream
 *     capture.
 *   - All calls share the one array, which keeps the last call's contents:
 *     calls that overlap on the GPU (different streams, no ordering between
 *     them) race and corrupt each other's results.
 *   - err_word (a device word, required: NULL returns DFM_ERR_INVALID_ARG)
 *     receives the DFM_DEVERR_* bits of the launch, e.g. a block-table entry
 *     outside the pool; the call ORs bits into it and never clears it, so the
 *     caller zeroes it and reads it back after the stream has reached the call. */
#define DFM_NOALLOC_SCRATCH_BYTES (8u << 20)
int dfm_paged_attention_noalloc(const void* q, void* out, const void* kv_pool, int32_t num_pages,
                                int32_t num_planes, int32_t heads, int32_t plane_k, int32_t plane_v,
                                const int32_t* cache_len, const int32_t* n_extend,
                                const int32_t* block_table, int32_t max_pages, int32_t n,
                                uint32_t* err_word, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* DFM_H_ */
