/*
 * dllm.h -- C ABI of the B200-native (sm_100a) paged decode attention of the
 * dots.tts LLM backbone (Qwen2: GQA, 12 query heads over 2 kv heads,
 * head_dim 128, paged K/V cache of 256-position blocks).
 *
 * Replaces the decode branch of the reference's Attention layer
 * (nanovllm_dots/layers/attention.py:60-97): the Triton store_kvcache
 * (attention.py:10-47) followed by flash-attn's flash_attn_with_kvcache(q,
 * k_cache, v_cache, cache_seqlens=context_lens, block_table=block_tables,
 * softmax_scale, causal=True) (flash-attn 2.8.3, attention.py:88-97), as driven
 * one token per sequence by BatchedPagedLLM._decode_batch
 * (nanovllm_dots/models/dots/batched_llm.py:177-236).
 *
 * Same library (libdfm.so), status codes and device error bits as dfm.h.
 * Every pointer is a DEVICE pointer; the caller owns every buffer.
 */
#ifndef DLLM_H_
#define DLLM_H_

#include <stddef.h>
#include <stdint.h>

#include "dfm.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Workspace bytes of dllm_decode_attention for these bounds (zero-fill it
 * once; it holds the device error word and the split-key partials). */
size_t dllm_decode_workspace_size(int32_t n, int32_t num_heads, int32_t head_dim,
                                  int32_t max_blocks, int32_t block_size);

/* One decode step of one attention layer for n sequences.
 *   q            bf16 [n, num_heads, head_dim]      (after rotary)
 *   k, v         bf16 [n, num_kv_heads, head_dim]   this step's token; NULL with
 *                slot_mapping NULL skips the store
 *   k_cache, v_cache  bf16 [num_blocks, block_size, num_kv_heads, head_dim]
 *   slot_mapping int32 [n]: block * block_size + offset of the token, -1 = no store
 *   context_lens int32 [n]: cached positions the query sees, the token included
 *   block_table  int32 [n, max_blocks]
 *   out          bf16 [n, num_heads, head_dim]
 * head_dim 64 or 128; num_heads a multiple of num_kv_heads with at most 8
 * query heads per kv head; block_size a multiple of 64.  Stream ordered, no
 * allocation, no host synchronisation.  An out-of-range block id or slot, or
 * a context_len outside [1, max_blocks * block_size], sets a device error bit
 * (dllm_read_error) and reads zeros / writes nothing for it. */
int dllm_decode_attention(const void* q, const void* k, const void* v, void* k_cache,
                          void* v_cache, const int32_t* slot_mapping, const int32_t* context_lens,
                          const int32_t* block_table, int32_t n, int32_t num_heads,
                          int32_t num_kv_heads, int32_t head_dim, int32_t num_blocks,
                          int32_t block_size, int32_t max_blocks, float softmax_scale, void* out,
                          void* workspace, size_t workspace_bytes, void* stream);

/* Read and clear the device error word of a workspace; synchronises `stream`. */
int dllm_read_error(void* workspace, void* stream, uint32_t* err_word);

/* ---------------------------------------------------------------------------
 * The whole backbone decode step: QwenLLM.forward over one new token per
 * sequence (nanovllm_dots/models/dots/model_llm.py:113-171, as
 * BatchedPagedLLM._decode_batch drives it, batched_llm.py:177-236):
 * per layer RMSNorm -> QKV (+bias) -> rotary -> store + paged attention ->
 * o_proj -> residual -> RMSNorm -> gate|up -> SiLU * up -> down -> residual,
 * then the final RMSNorm.  The residual stream is kept in fp32.
 * ------------------------------------------------------------------------- */

/* Model shape (the Qwen2 config fields) and batch / cache bounds.  hidden a
 * multiple of 512 (1024, 1536 or 2048 in this build); head_dim 128; 2*inter a
 * multiple of 256. */
typedef struct DllmConfig {
  int32_t layers, hidden, heads, kv_heads, head_dim, inter;
  float rms_eps;
  int32_t block_size;   /* cache positions per block (a multiple of 64) */
  int32_t max_blocks;   /* block-table width */
  int32_t max_batch;    /* most sequences per step */
} DllmConfig;

/* Weights, stacked over layers (bf16 [out, in] matrices, fp32 vectors); the
 * layouts of the reference's packed projections (QKVParallelLinear q|k|v,
 * MergedColumnParallelLinear gate|up). */
typedef struct DllmWeights {
  const float* in_norm;     /* [layers][hidden] input_layernorm.weight */
  const void* qkv_w;        /* [layers][(heads + 2 kv_heads) head_dim][hidden] */
  const float* qkv_b;       /* [layers][(heads + 2 kv_heads) head_dim] */
  const void* o_w;          /* [layers][hidden][heads head_dim] (no bias) */
  const float* post_norm;   /* [layers][hidden] post_attention_layernorm.weight */
  const void* gate_up_w;    /* [layers][2 inter][hidden] (no bias) */
  const void* down_w;       /* [layers][hidden][inter] (no bias) */
  const float* final_norm;  /* [hidden] */
  const float* inv_freq;    /* [head_dim / 2] rotary base^(-2i / head_dim) */
} DllmWeights;

/* One step.  k_caches / v_caches are HOST arrays of `layers` device pointers
 * (one cache pair per layer, [num_blocks, block_size, kv_heads, head_dim] bf16);
 * the other pointers are device pointers. */
typedef struct DllmStep {
  int32_t n;
  const void* embeds;             /* bf16 [n, hidden] this step's input embeddings */
  const int32_t* positions;       /* [n] the token's position (its rotary angle) */
  const int32_t* slot_mapping;    /* [n] cache slot of the token */
  const int32_t* context_lens;    /* [n] positions attended, the token included */
  const int32_t* block_table;     /* [n, max_blocks] */
  void* const* k_caches;
  void* const* v_caches;
  int32_t num_blocks;
  void* out;                      /* bf16 [n, hidden] final hidden states */
} DllmStep;

int dllm_create(const DllmConfig* config, const DllmWeights* weights, void** handle);
size_t dllm_step_workspace_size(void* handle);
/* Stream ordered, no allocation, no host synchronisation; the first call with
 * a given workspace or set of caches encodes their TMA descriptors (host work,
 * so make it before stream capture). */
int dllm_decode_step(void* handle, const DllmStep* step, void* workspace, size_t workspace_bytes,
                     void* stream);
int dllm_destroy(void* handle);

#ifdef __cplusplus
}
#endif

#endif /* DLLM_H_ */
