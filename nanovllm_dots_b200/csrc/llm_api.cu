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

// ---------------------------------------------------------------- backbone decode step
#include "llm_step.cuh"

namespace {

// Split-K partial planes of the decode projections (llm_swap_gemm_kernel:
// 128 output features per work unit, so N = 1536-2048 alone gives 12-16 units)
constexpr int kLlmOSplit = 8;      // O-projection
constexpr int kLlmQkvSplit = 8;    // QKV
constexpr int kLlmSubPlanes = 12;  // the most partial planes a sublayer writes (O, down)

struct LlmStepWs {
  size_t err, h, xn, qkv, qr, ao, sub, act, part_o, part_ml, total;
};

struct LlmHandle {
  DllmConfig c;
  DllmWeights w;
  int device;
  int qkvw, down_split, mc;
  LlmStepWs ws;
  CUtensorMap* m_qkv;
  CUtensorMap* m_o;
  CUtensorMap* m_gu;
  CUtensorMap* m_down;
  CUtensorMap* m_kc;      // per layer, for the cache pointers in kc_ptr
  CUtensorMap* m_vc;
  const void** kc_ptr;
  const void** vc_ptr;
  int cache_blocks = 0;
  const void* plan_ws = nullptr;
  CUtensorMap a_xn, a_ao, a_act;   // the GEMMs' activation operands (64-token boxes)
};

// K splits of the down-projection: the most (up to kLlmSubPlanes, among the
// plane counts the RMSNorm kernel is built for) that divide its k-blocks and
// keep its units (hidden / 128 per split) within one wave.
int llm_down_split(int inter, int hidden, int sms) {
  const int kb = inter / 64, tiles = hidden / LS_BM;
  for (int s : {12, 10, 8, 7, 5, 4, 2})
    if (kb % s == 0 && tiles * s <= sms) return s;
  return 1;
}

LlmStepWs llm_step_layout(const DllmConfig& c, int qkvw, int mc) {
  LlmStepWs L{};
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off += (bytes + 1023) & ~static_cast<size_t>(1023);
    return o;
  };
  const size_t NR = c.max_batch, Hd = c.hidden, HD = static_cast<size_t>(c.heads) * c.head_dim;
  L.err = take(256);   // offset 0: dllm_read_error reads it
  L.h = take(NR * Hd * 4);
  L.xn = take(NR * Hd * 2);
  L.qkv = take(kLlmQkvSplit * NR * qkvw * 4);   // fp32 split-K planes
  L.qr = take(NR * HD * 2);
  L.ao = take(NR * HD * 2);
  L.sub = take(kLlmSubPlanes * NR * Hd * 4);
  L.act = take(NR * static_cast<size_t>(c.inter) * 2);
  L.part_o = take(NR * c.heads * mc * static_cast<size_t>(c.head_dim) * 4);
  L.part_ml = take(NR * c.heads * mc * 2 * 4);
  L.total = off;
  return L;
}

int llm_validate(const DllmConfig& c) {
  if (c.hidden != 1024 && c.hidden != 1536 && c.hidden != 2048) return DFM_ERR_UNSUPPORTED;
  if (c.head_dim != 128 || c.heads < 1 || c.kv_heads < 1 || c.heads % c.kv_heads ||
      c.heads / c.kv_heads > LA_MAXG)
    return DFM_ERR_UNSUPPORTED;
  if (c.inter < 64 || c.inter % 128 || c.hidden % LS_BM) return DFM_ERR_UNSUPPORTED;
  if (c.block_size < LA_SUB || c.block_size % LA_SUB) return DFM_ERR_UNSUPPORTED;
  if (c.layers < 1 || c.max_blocks < 1 || c.max_batch < 1 || !(c.rms_eps > 0.f))
    return DFM_ERR_INVALID_ARG;
  if ((c.heads * c.head_dim) / 64 % kLlmOSplit || (c.hidden / 64) % kLlmQkvSplit ||
      ((c.heads + 2 * c.kv_heads) * c.head_dim) % LS_BM)
    return DFM_ERR_UNSUPPORTED;
  return DFM_OK;
}

template <int NSUB>
cudaError_t launch_rms(int hidden, cudaStream_t s, int M, float* h, const __nv_bfloat16* in,
                       const float* sub, size_t plane, const float* w, float eps,
                       __nv_bfloat16* out) {
  const dim3 grid(M);
  switch (hidden) {
    case 1024: return launch_pdl(llm_rms_kernel<1024, NSUB>, grid, dim3(256), 0, s, h, in, sub, plane, M, w, eps, out);
    case 1536: return launch_pdl(llm_rms_kernel<1536, NSUB>, grid, dim3(384), 0, s, h, in, sub, plane, M, w, eps, out);
    case 2048: return launch_pdl(llm_rms_kernel<2048, NSUB>, grid, dim3(512), 0, s, h, in, sub, plane, M, w, eps, out);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_rms_n(int nsub, int hidden, cudaStream_t s, int M, float* h,
                         const __nv_bfloat16* in, const float* sub, size_t plane, const float* w,
                         float eps, __nv_bfloat16* out) {
  switch (nsub) {
    case 0: return launch_rms<0>(hidden, s, M, h, in, sub, plane, w, eps, out);
    case 1: return launch_rms<1>(hidden, s, M, h, in, sub, plane, w, eps, out);
    case 2: return launch_rms<2>(hidden, s, M, h, in, sub, plane, w, eps, out);
    case 4: return launch_rms<4>(hidden, s, M, h, in, sub, plane, w, eps, out);
    case 5: return launch_rms<5>(hidden, s, M, h, in, sub, plane, w, eps, out);
    case 7: return launch_rms<7>(hidden, s, M, h, in, sub, plane, w, eps, out);
    case 8: return launch_rms<8>(hidden, s, M, h, in, sub, plane, w, eps, out);
    case 10: return launch_rms<10>(hidden, s, M, h, in, sub, plane, w, eps, out);
    case 12: return launch_rms<12>(hidden, s, M, h, in, sub, plane, w, eps, out);
    default: return cudaErrorInvalidValue;
  }
}

// One decode projection on llm_swap_gemm_kernel: out = X W^T for n tokens,
// as `splits` fp32 partial planes (LS_F32), one bf16 result (LS_BF16), or
// silu(gate) * up of a [gate; up] weight with nout = I (LS_SILU, W's tensor
// map in 32-row boxes).
template <int kMode>
cudaError_t llm_swap(const CUtensorMap& w, const CUtensorMap& x, int nout, int K, int n, int splits,
                     void* out, size_t plane, uint32_t* err, cudaStream_t s) {
  static std::atomic<uint64_t> attr_done{0};
  auto fn = llm_swap_gemm_kernel<kMode>;
  constexpr int smem = kMode == LS_SILU ? LsShape::SMEM_SILU : LsShape::SMEM;
  cudaError_t r = smem_attr_once(attr_done, fn, smem);
  if (r != cudaSuccess) return r;
  LsArgs p;
  p.tiles_m = (kMode == LS_SILU ? 2 * nout : nout) / LS_BM;
  p.tok_blocks = (n + LS_BN - 1) / LS_BN;
  p.splits = splits;
  p.nk = K / LS_BK / splits;
  p.n = n;
  p.nout = nout;
  p.out = out;
  p.plane = plane;
  const int total = p.tiles_m * p.tok_blocks * splits;
  const int grid = total < sm_count() ? total : sm_count();
  return launch_pdl(fn, dim3(grid), dim3(LS_THREADS), smem, s, w, x, p, err);
}

bool llm_plan(LlmHandle* h, void* ws) {
  if (h->plan_ws == ws) return true;
  const DllmConfig& c = h->c;
  uint8_t* b = static_cast<uint8_t*>(ws);
  const uint64_t NR = c.max_batch, Hd = c.hidden, HD = static_cast<uint64_t>(c.heads) * c.head_dim;
  bool ok = map_2d(&h->a_xn, b + h->ws.xn, NR, Hd, Hd, LS_BN) &&
            map_2d(&h->a_ao, b + h->ws.ao, NR, HD, HD, LS_BN) &&
            map_2d(&h->a_act, b + h->ws.act, NR, c.inter, c.inter, LS_BN);
  if (!ok) {
    h->plan_ws = nullptr;
    return false;
  }
  if (cudaMemset(b + h->ws.err, 0, sizeof(uint32_t)) != cudaSuccess) return false;
  h->plan_ws = ws;
  return true;
}

}  // namespace

extern "C" {

int dllm_destroy(void* handle) {
  LlmHandle* h = static_cast<LlmHandle*>(handle);
  if (!h) return DFM_ERR_INVALID_ARG;
  delete[] h->m_qkv;
  delete[] h->m_o;
  delete[] h->m_gu;
  delete[] h->m_down;
  delete[] h->m_kc;
  delete[] h->m_vc;
  delete[] h->kc_ptr;
  delete[] h->vc_ptr;
  delete h;
  return DFM_OK;
}

int dllm_create(const DllmConfig* cfg, const DllmWeights* w, void** out) {
  if (!cfg || !w || !out) return DFM_ERR_INVALID_ARG;
  *out = nullptr;
  int rc = llm_validate(*cfg);
  if (rc != DFM_OK) return rc;
  const void* req[] = {w->in_norm, w->qkv_w, w->qkv_b, w->o_w, w->post_norm, w->gate_up_w,
                       w->down_w, w->final_norm, w->inv_freq};
  for (const void* p : req)
    if (!p) return DFM_ERR_INVALID_ARG;
  if (!encode_fn()) return DFM_ERR_CUDA;
  LlmHandle* h = new (std::nothrow) LlmHandle();
  if (!h) return DFM_ERR_CUDA;
  h->c = *cfg;
  h->w = *w;
  if (cudaGetDevice(&h->device) != cudaSuccess) {
    delete h;
    return DFM_ERR_CUDA;
  }
  const DllmConfig& c = h->c;
  const int L = c.layers, Hd = c.hidden, HD = c.heads * c.head_dim;
  h->qkvw = (c.heads + 2 * c.kv_heads) * c.head_dim;
  h->down_split = llm_down_split(c.inter, c.hidden, sm_count());
  h->mc = llm_max_chunks(c.max_blocks, c.block_size);
  h->ws = llm_step_layout(c, h->qkvw, h->mc);
  h->m_qkv = new CUtensorMap[L];
  h->m_o = new CUtensorMap[L];
  h->m_gu = new CUtensorMap[L];
  h->m_down = new CUtensorMap[L];
  h->m_kc = new CUtensorMap[L];
  h->m_vc = new CUtensorMap[L];
  h->kc_ptr = new const void*[L]();
  h->vc_ptr = new const void*[L]();
  auto bw = [](const void* p) { return static_cast<const __nv_bfloat16*>(p); };
  bool ok = true;
  for (int l = 0; ok && l < L; ++l) {
    ok = map_2d(&h->m_qkv[l], bw(w->qkv_w) + static_cast<size_t>(l) * h->qkvw * Hd, h->qkvw, Hd,
                Hd, LS_BM) &&
         map_2d(&h->m_o[l], bw(w->o_w) + static_cast<size_t>(l) * Hd * HD, Hd, HD, HD, LS_BM) &&
         map_2d(&h->m_gu[l], bw(w->gate_up_w) + static_cast<size_t>(l) * 2 * c.inter * Hd,
                2 * static_cast<uint64_t>(c.inter), Hd, Hd, 32) &&
         map_2d(&h->m_down[l], bw(w->down_w) + static_cast<size_t>(l) * Hd * c.inter, Hd, c.inter,
                c.inter, LS_BM);
  }
  if (!ok) {
    dllm_destroy(h);
    return DFM_ERR_CUDA;
  }
  *out = h;
  return DFM_OK;
}

size_t dllm_step_workspace_size(void* handle) {
  return handle ? static_cast<LlmHandle*>(handle)->ws.total : 0;
}

int dllm_decode_step(void* handle, const DllmStep* st, void* workspace, size_t workspace_bytes,
                     void* stream) {
  LlmHandle* hd = static_cast<LlmHandle*>(handle);
  if (!hd || !st || !workspace) return DFM_ERR_INVALID_ARG;
  const DllmConfig& c = hd->c;
  const DllmWeights& w = hd->w;
  const int n = st->n;
  if (n < 1 || n > c.max_batch) return DFM_ERR_INVALID_ARG;
  if (!st->embeds || !st->positions || !st->slot_mapping || !st->context_lens ||
      !st->block_table || !st->k_caches || !st->v_caches || !st->out || st->num_blocks < 1)
    return DFM_ERR_INVALID_ARG;
  if (workspace_bytes < hd->ws.total) return DFM_ERR_WORKSPACE;
  if (reinterpret_cast<uintptr_t>(workspace) % 256 != 0) return DFM_ERR_INVALID_ARG;
  int dev = -1;
  CK(cudaGetDevice(&dev));
  if (dev != hd->device) return DFM_ERR_INVALID_ARG;
  if (!llm_plan(hd, workspace)) return DFM_ERR_CUDA;
  const int L = c.layers;
  // cache descriptors: encoded when a layer's cache pointer (or the block count) changes
  for (int l = 0; l < L; ++l) {
    if (!st->k_caches[l] || !st->v_caches[l]) return DFM_ERR_INVALID_ARG;
    if (hd->kc_ptr[l] != st->k_caches[l] || hd->vc_ptr[l] != st->v_caches[l] ||
        hd->cache_blocks != st->num_blocks) {
      if (!map_llm_cache(&hd->m_kc[l], st->k_caches[l], st->num_blocks, c.block_size, c.kv_heads,
                         c.head_dim) ||
          !map_llm_cache(&hd->m_vc[l], st->v_caches[l], st->num_blocks, c.block_size, c.kv_heads,
                         c.head_dim))
        return DFM_ERR_CUDA;
      hd->kc_ptr[l] = st->k_caches[l];
      hd->vc_ptr[l] = st->v_caches[l];
    }
  }
  hd->cache_blocks = st->num_blocks;

  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  uint32_t* err = reinterpret_cast<uint32_t*>(ws + hd->ws.err);
  auto bf = [&](size_t off) { return reinterpret_cast<__nv_bfloat16*>(ws + off); };
  auto f32 = [&](size_t off) { return reinterpret_cast<float*>(ws + off); };
  const int Hd = c.hidden, H = c.heads, KVH = c.kv_heads, D = c.head_dim, I = c.inter;
  const size_t plane = static_cast<size_t>(c.max_batch) * Hd;
  float* h = f32(hd->ws.h);
  __nv_bfloat16* xn = bf(hd->ws.xn);

  LlmAttnParams ap{};
  ap.q = bf(hd->ws.qr);
  ap.context_lens = st->context_lens;
  ap.block_table = st->block_table;
  ap.part_o = f32(hd->ws.part_o);
  ap.part_ml = f32(hd->ws.part_ml);
  ap.n = n;
  ap.H = H;
  ap.KVH = KVH;
  ap.G = H / KVH;
  ap.max_blocks = c.max_blocks;
  ap.num_blocks = st->num_blocks;
  ap.block_size = c.block_size;
  ap.max_chunks = hd->mc;
  ap.scale_log2 = (1.0f / sqrtf(static_cast<float>(D))) * 1.4426950408889634f;
  ap.err = err;

  // the input embeddings into the fp32 residual stream, and the first RMSNorm
  CK(launch_rms_n(0, Hd, s, n, h, static_cast<const __nv_bfloat16*>(st->embeds), nullptr, 0,
                  w.in_norm, c.rms_eps, xn));
  for (int l = 0; l < L; ++l) {
    const int qkvw = hd->qkvw;
    CK(llm_swap<LS_F32>(hd->m_qkv[l], hd->a_xn, qkvw, Hd, n, kLlmQkvSplit, f32(hd->ws.qkv),
                      static_cast<size_t>(c.max_batch) * qkvw, err, s));
    const int cnt = n * (H + 2 * KVH) * (D / 2);
    CK(launch_pdl(llm_rope_kernel<kLlmQkvSplit>, dim3((cnt + 255) / 256), dim3(256), 0, s,
                  static_cast<const float*>(f32(hd->ws.qkv)), static_cast<size_t>(c.max_batch) * qkvw,
                  static_cast<const float*>(w.qkv_b + static_cast<size_t>(l) * qkvw), st->positions,
                  w.inv_freq, n, H, KVH, D, bf(hd->ws.qr),
                  static_cast<__nv_bfloat16*>(const_cast<void*>(hd->kc_ptr[l])),
                  static_cast<__nv_bfloat16*>(const_cast<void*>(hd->vc_ptr[l])), st->slot_mapping,
                  static_cast<long long>(st->num_blocks) * c.block_size, err));
    CK(launch_llm_decode<128>(hd->m_kc[l], hd->m_vc[l], ap, bf(hd->ws.ao), s));
    CK(llm_swap<LS_F32>(hd->m_o[l], hd->a_ao, Hd, H * D, n, kLlmOSplit, f32(hd->ws.sub), plane, err, s));
    CK(launch_rms_n(kLlmOSplit, Hd, s, n, h, nullptr, f32(hd->ws.sub), plane,
                    w.post_norm + static_cast<size_t>(l) * Hd, c.rms_eps, xn));
    CK(llm_swap<LS_SILU>(hd->m_gu[l], hd->a_xn, I, Hd, n, 1, bf(hd->ws.act), 0, err, s));
    CK(llm_swap<LS_F32>(hd->m_down[l], hd->a_act, Hd, I, n, hd->down_split, f32(hd->ws.sub), plane,
                      err, s));
    // residual + the next layer's input norm, or the final norm into the output
    const bool last = l == L - 1;
    CK(launch_rms_n(hd->down_split, Hd, s, n, h, nullptr, f32(hd->ws.sub), plane,
                    last ? w.final_norm : w.in_norm + static_cast<size_t>(l + 1) * Hd, c.rms_eps,
                    last ? static_cast<__nv_bfloat16*>(st->out) : xn));
  }
  return DFM_OK;
}

}  // extern "C"
