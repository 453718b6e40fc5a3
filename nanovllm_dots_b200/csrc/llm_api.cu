// Host side of the LLM decode-attention C ABI (include/dllm.h).  Compiled
// inside dfm_api.cu's translation unit (included at its end), whose TMA
// encoder and launch helpers it uses.
#include "../../include/dllm.h"
#include "llm_attn.cuh"

namespace {

struct LlmWs {
  size_t part_o, part_ml, total;
};

int llm_max_chunks(int max_blocks, int block_size) {
  return static_cast<int>((static_cast<long long>(max_blocks) * block_size + LA_CHUNK - 1) / LA_CHUNK);
}

LlmWs llm_ws(int n, int H, int D, int max_blocks, int block_size) {
  auto up = [](size_t x) { return (x + 1023) & ~static_cast<size_t>(1023); };
  const size_t mc = llm_max_chunks(max_blocks, block_size);
  LlmWs w;
  w.part_o = 1024;   // after the error word
  w.part_ml = w.part_o + up(static_cast<size_t>(n) * H * mc * D * 4);
  w.total = w.part_ml + up(static_cast<size_t>(n) * H * mc * 2 * 4);
  return w;
}

// One of the paged caches as a 4-D tensor [num_blocks][block_size][kv_heads][D];
// a box is 64 dims x 1 head x 64 positions x 1 block (128-byte swizzle).
bool map_llm_cache(CUtensorMap* m, const void* base, int num_blocks, int block_size, int kvh, int D) {
  auto fn = encode_fn();
  if (!fn || !base) return false;
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(kvh),
                        static_cast<cuuint64_t>(block_size), static_cast<cuuint64_t>(num_blocks)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(D) * 2, static_cast<cuuint64_t>(kvh) * D * 2,
                           static_cast<cuuint64_t>(block_size) * kvh * D * 2};
  cuuint32_t box[4] = {64, 1, static_cast<cuuint32_t>(LA_SUB), 1};
  cuuint32_t es[4] = {1, 1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int D>
cudaError_t launch_llm_decode(const CUtensorMap& mk, const CUtensorMap& mv, const LlmAttnParams& p,
                              __nv_bfloat16* out, cudaStream_t s) {
  static std::atomic<uint64_t> attr_done{0};
  constexpr int smem = LlmAttnSmem<D>::BYTES;
  cudaError_t r = smem_attr_once(attr_done, llm_decode_attn_kernel<D>, smem);
  if (r != cudaSuccess) return r;
  r = launch_pdl(llm_decode_attn_kernel<D>, dim3(p.max_chunks, p.KVH, p.n), dim3(LA_THREADS), smem,
                 s, mk, mv, p);
  if (r != cudaSuccess) return r;
  return launch_pdl(llm_attn_combine_kernel<D>, dim3(p.n * p.H), dim3(D), 0, s,
                    static_cast<const float*>(p.part_o), static_cast<const float*>(p.part_ml),
                    p.context_lens, p.H, p.max_chunks, p.max_blocks * p.block_size, out);
}

}  // namespace

extern "C" {

size_t dllm_decode_workspace_size(int32_t n, int32_t num_heads, int32_t head_dim,
                                  int32_t max_blocks, int32_t block_size) {
  if (n < 1 || num_heads < 1 || (head_dim != 64 && head_dim != 128) || max_blocks < 1 ||
      block_size < LA_SUB)
    return 0;
  return llm_ws(n, num_heads, head_dim, max_blocks, block_size).total;
}

int dllm_decode_attention(const void* q, const void* k, const void* v, void* k_cache,
                          void* v_cache, const int32_t* slot_mapping, const int32_t* context_lens,
                          const int32_t* block_table, int32_t n, int32_t num_heads,
                          int32_t num_kv_heads, int32_t head_dim, int32_t num_blocks,
                          int32_t block_size, int32_t max_blocks, float softmax_scale, void* out,
                          void* workspace, size_t workspace_bytes, void* stream) {
  if (!q || !k_cache || !v_cache || !context_lens || !block_table || !out || !workspace)
    return DFM_ERR_INVALID_ARG;
  if ((k == nullptr) != (v == nullptr) || ((k == nullptr) != (slot_mapping == nullptr)))
    return DFM_ERR_INVALID_ARG;
  if (n < 1 || num_heads < 1 || num_kv_heads < 1 || num_blocks < 1 || max_blocks < 1)
    return DFM_ERR_INVALID_ARG;
  if (head_dim != 64 && head_dim != 128) return DFM_ERR_UNSUPPORTED;
  if (num_heads % num_kv_heads || num_heads / num_kv_heads > LA_MAXG) return DFM_ERR_UNSUPPORTED;
  if (block_size < LA_SUB || block_size % LA_SUB) return DFM_ERR_UNSUPPORTED;
  if (!(softmax_scale > 0.f)) return DFM_ERR_INVALID_ARG;
  const LlmWs w = llm_ws(n, num_heads, head_dim, max_blocks, block_size);
  if (workspace_bytes < w.total) return DFM_ERR_WORKSPACE;
  if (reinterpret_cast<uintptr_t>(workspace) % 256 != 0) return DFM_ERR_INVALID_ARG;
  CUtensorMap mk, mv;
  if (!map_llm_cache(&mk, k_cache, num_blocks, block_size, num_kv_heads, head_dim) ||
      !map_llm_cache(&mv, v_cache, num_blocks, block_size, num_kv_heads, head_dim))
    return DFM_ERR_CUDA;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  uint32_t* err = reinterpret_cast<uint32_t*>(ws);
  const int row_elems = num_kv_heads * head_dim;
  if (k) {
    const int cnt = 2 * n * (row_elems / 8);
    CK(launch_pdl(llm_store_kv_kernel, dim3((cnt + 255) / 256), dim3(256), 0, s,
                  static_cast<const __nv_bfloat16*>(k), static_cast<const __nv_bfloat16*>(v),
                  static_cast<__nv_bfloat16*>(k_cache), static_cast<__nv_bfloat16*>(v_cache),
                  slot_mapping, n, row_elems, static_cast<long long>(num_blocks) * block_size, err));
  }
  LlmAttnParams p{};
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.context_lens = context_lens;
  p.block_table = block_table;
  p.part_o = reinterpret_cast<float*>(ws + w.part_o);
  p.part_ml = reinterpret_cast<float*>(ws + w.part_ml);
  p.n = n;
  p.H = num_heads;
  p.KVH = num_kv_heads;
  p.G = num_heads / num_kv_heads;
  p.max_blocks = max_blocks;
  p.num_blocks = num_blocks;
  p.block_size = block_size;
  p.max_chunks = llm_max_chunks(max_blocks, block_size);
  p.scale_log2 = softmax_scale * 1.4426950408889634f;
  p.err = err;
  __nv_bfloat16* o = static_cast<__nv_bfloat16*>(out);
  const cudaError_t r = head_dim == 128 ? launch_llm_decode<128>(mk, mv, p, o, s)
                                        : launch_llm_decode<64>(mk, mv, p, o, s);
  return r == cudaSuccess ? DFM_OK : DFM_ERR_CUDA;
}

int dllm_read_error(void* workspace, void* stream, uint32_t* err_word) {
  if (!workspace || !err_word) return DFM_ERR_INVALID_ARG;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint32_t v = 0;
  CK(cudaMemcpyAsync(&v, workspace, sizeof(v), cudaMemcpyDeviceToHost, s));
  CK(cudaStreamSynchronize(s));
  CK(cudaMemsetAsync(workspace, 0, sizeof(uint32_t), s));
  *err_word = v;
  return DFM_OK;
}

}  // extern "C"
