/*
 * dpe.h -- C ABI of the B200-native (sm_100a) patch encoder of dots.tts.
 *
 * The patch encoder (VAESemanticEncoder, nanovllm_dots/models/dots/native/
 * patch_encoder.py:139-235) turns each latent patch the FM head emits into the
 * LLM's next input embedding.  The reference runs it batched through
 * FlashPatchEncoder.decode_patch (nanovllm_dots/models/dots/flash_patch_encoder.py:104-139,
 * called from engine.py:743-765): a causal stride-2 conv, in_proj, a causal
 * transformer over each request's own history (flash_attn_with_kvcache over a
 * per-request cache row), then out_proj of the patch's 8 rows.  dpe_decode is
 * that call: one launch sequence for every request in the call, on the
 * caller's stream, without host synchronisation or allocation.
 *
 * The same shared library (libdfm.so) exports these symbols next to the FM
 * head's (dfm.h); status codes and device error bits are dfm.h's.
 *
 * Conventions: as in dfm.h.  Every pointer inside the structs is a DEVICE
 * pointer; bf16 matrices are row-major [out, in]; biases and norm parameters
 * are fp32; the caller owns every buffer.
 */
#ifndef DPE_H_
#define DPE_H_

#include <stddef.h>
#include <stdint.h>

#include "dfm.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Model and cache shape.  Mirrors VAESemanticEncoder's constructor arguments
 * (patch_encoder.py:139-150: in_dim = latent_dim, out_dim = the LLM width,
 * config.patch_size, config.PatchEncoder.{hidden_size, num_heads,
 * ffn_hidden_size, num_layers}) and FlashPatchEncoder's pool sizes
 * (flash_patch_encoder.py:40-69: max_batch rows of max_seq_len positions). */
typedef struct DpeConfig {
  int32_t layers;            /* encoder layers (synthetic default 6) */
  int32_t hidden;            /* encoder width (1024; the only width this build supports) */
  int32_t heads;             /* attention heads (16) */
  int32_t head_dim;          /* 64 */
  int32_t ffn;               /* MLP width (4096) */
  int32_t latent_dim;        /* conv channels = latent_dim (64) */
  int32_t patch;             /* latent frames per patch (16); rows per patch = patch / 2 */
  int32_t out_dim;           /* embedding width (1536) */
  int32_t max_rows;          /* cache rows (FlashPatchEncoder max_batch) */
  int32_t max_pages_per_row; /* row capacity in 16-position pages (max_seq_len / 16) */
  int32_t max_batch;         /* largest n one dpe_decode may carry */
  float ln_eps;              /* LayerNorm eps (1e-5) */
} DpeConfig;

/* Weights (the VAESemanticEncoder state dict, repacked). */
typedef struct DpeWeights {
  const void* conv_w;      /* ds_proj as bf16 [latent_dim, 2*latent_dim]: [W[:,:,0] | W[:,:,1]] */
  const float* conv_b;     /* [latent_dim] */
  const void* in_w;        /* in_proj bf16 [hidden, latent_dim] */
  const float* in_b;       /* [hidden] */
  const float* attn_norm;  /* [layers][2][hidden]: weight, bias */
  const float* ffn_norm;   /* [layers][2][hidden]: weight, bias */
  const void* qkv_w;       /* bf16 [layers][3*hidden, hidden]: q_proj; k_proj; v_proj (no bias) */
  const void* o_w;         /* bf16 [layers][hidden, hidden] */
  const float* o_b;        /* [layers][hidden] */
  const void* fc1_w;       /* bf16 [layers][ffn, hidden] */
  const float* fc1_b;      /* [layers][ffn] */
  const void* fc2_w;       /* bf16 [layers][hidden, ffn] */
  const float* fc2_b;      /* [layers][hidden] */
  const void* out_w;       /* out_proj bf16 [out_dim, (patch/2)*hidden] */
  const float* out_b;      /* [out_dim] */
} DpeWeights;

/* One call.  Replaces FlashPatchEncoder.decode_patch(latent_patches, rows)
 * (flash_patch_encoder.py:104-139) and its state (self.seqlens, self.conv_tail,
 * self.kbuf/vbuf). */
typedef struct DpeBatch {
  int32_t n;               /* requests in this call, 1..max_batch */
  const void* patches;     /* bf16 [n, patch, latent_dim] (denormalised latents) */
  const int32_t* rows;     /* [n] distinct cache rows in [0, max_rows) */
  int32_t* seqlens;        /* [max_rows] positions cached per row; each row in `rows` advances by patch/2 */
  void* conv_tail;         /* bf16 [max_rows, latent_dim]; each row in `rows` becomes its patch's last frame */
  void* kv_pool;           /* dpe_pool_bytes(config) bytes, zero-initialised once */
  void* out;               /* bf16 [n, out_dim] embeddings */
} DpeBatch;

/* Validate the config, encode the weight descriptors and return a handle.
 * Replaces FlashPatchEncoder.__init__ (flash_patch_encoder.py:40-69) minus the
 * allocations, which the caller makes. */
int dpe_create(const DpeConfig* config, const DpeWeights* weights, void** handle);

/* Bytes of the per-handle workspace dpe_decode needs. */
size_t dpe_workspace_size(void* handle);

/* Bytes of the K/V pool: [layers * 2][max_rows * max_pages_per_row][heads][16][head_dim] bf16.
 * Cache row r owns pages [r * max_pages_per_row, (r + 1) * max_pages_per_row). */
size_t dpe_pool_bytes(const DpeConfig* config);

/* One decode step for n requests (flash_patch_encoder.py:104-139): stream
 * ordered, no host synchronisation, no allocation; capturable in a CUDA graph
 * once the workspace has been seen by one eager call.  A cache row is reset by
 * zeroing its seqlens entry and conv tail (FlashPatchEncoder.reset_rows,
 * flash_patch_encoder.py:71-76); its stale K/V are never read. */
int dpe_decode(void* handle, const DpeBatch* batch, void* workspace, size_t workspace_bytes,
               void* stream);

/* Read and clear the device error word (DFM_DEVERR_* bits); synchronises `stream`. */
int dpe_read_error(void* handle, void* workspace, void* stream, uint32_t* err_word);

int dpe_destroy(void* handle);

#ifdef __cplusplus
}
#endif

#endif /* DPE_H_ */
