// Host side of the FM-head C ABI (include/dfm.h): handle, workspace layout,
// TMA descriptor encoding and the per-tick launch sequence.
#include <cudaTypedefs.h>

#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <new>
#include <utility>

#include "../../include/dfm.h"
#include "attn_tc.cuh"
#include "ew.cuh"
#include "gemm.cuh"

using namespace dfm;

namespace {

constexpr int kH = 1024;
constexpr int kStride = 17;      // hidden_patch + latent_patch
constexpr int kSlot = 2 * kStride;  // graduating + active rows per request
// Tile widths of the per-layer CTA-pair GEMMs (output tiles 256 x BN).
constexpr int kQkvBN = 256, kQkvST = 6;
constexpr int kFc1BN = 256, kFc1ST = 5;
constexpr int kOutBN = 256, kOutST = 5;  // O-projection and fc2 (N = hidden) ...
constexpr int kOutSplit = 2;             // ... as two split-K partial sums (72 units at n = 64)
constexpr int kAdaBN = 256, kAdaST = 5;  // the all-layer adaLN GEMM (one 256-row tile of steps x requests)

// ---------------------------------------------------------------- TMA encoding
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// 2-D bf16 K-major operand [rows, cols] with row stride ld elements, box
// {64, box_rows}, 128-byte swizzle, zero fill out of bounds.
bool map_2d(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols, uint64_t ld,
            uint32_t box_rows) {
  auto fn = encode_fn();
  if (!fn || !base) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld * 2};
  cuuint32_t box[2] = {64, box_rows};
  cuuint32_t es[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
            es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 2-D 8-bit K-major operand [rows, cols] (e4m3 bytes) with row stride ld bytes,
// box {128, box_rows}, 128-byte swizzle, zero fill out of bounds.
bool map_2d_u8(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols, uint64_t ld,
               uint32_t box_rows) {
  auto fn = encode_fn();
  if (!fn || !base) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld};
  cuuint32_t box[2] = {128, box_rows};
  cuuint32_t es[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The K/V pool as a 5-D tensor [planes][pages][heads][16][64]; one box is one
// (page, head) block of 16 rows x 64 dims.
bool map_pool(CUtensorMap* m, const void* base, int num_pages, int heads, int planes) {
  auto fn = encode_fn();
  if (!fn || !base) return false;
  cuuint64_t dims[5] = {64, 16, static_cast<cuuint64_t>(heads), static_cast<cuuint64_t>(num_pages),
                        static_cast<cuuint64_t>(planes)};
  cuuint64_t strides[4] = {128, 2048, 2048ull * heads, 2048ull * heads * num_pages};
  cuuint32_t box[5] = {64, 16, 1, 1, 1};
  cuuint32_t es[5] = {1, 1, 1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 5, const_cast<void*>(base), dims, strides, box,
            es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// ---------------------------------------------------------------- launches
// Raise a kernel's dynamic shared-memory limit once per device (the attribute
// call is host-expensive and must not sit on the per-launch path).
template <class K>
cudaError_t smem_attr_once(std::atomic<uint64_t>& done, K fn, int smem) {
  int dev = 0;
  cudaError_t r = cudaGetDevice(&dev);
  if (r != cudaSuccess) return r;
  const uint64_t bit = 1ull << (dev & 63);
  if (done.load(std::memory_order_acquire) & bit) return cudaSuccess;
  r = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (r == cudaSuccess) done.fetch_or(bit, std::memory_order_acq_rel);
  return r;
}

int sm_count() {
  static std::atomic<int> cache[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  int v = cache[dev & 63].load(std::memory_order_relaxed);
  if (v > 0) return v;
  if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0)
    v = 148;
  cache[dev & 63].store(v, std::memory_order_relaxed);
  return v;
}

// Launch with programmatic stream serialization (PDL): the kernel may begin
// while the previous kernel in the stream drains; it waits in pdl_wait()
// before touching activations.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                       Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

template <int BN, int ST, class Epi>
cudaError_t gemm(const CUtensorMap& a, const CUtensorMap& b, int M, int N, int K, const Epi& e,
                 uint32_t* err, cudaStream_t s) {
  if (M <= 0) return cudaSuccess;
  static std::atomic<uint64_t> attr_done{0};
  auto fn = gemm_bf16_tn<BN, ST, Epi>;
  constexpr int smem = GemmShape<BN, ST>::SMEM;
  cudaError_t r = smem_attr_once(attr_done, fn, smem);
  if (r != cudaSuccess) return r;
  const int tiles = ((M + GEMM_BM - 1) / GEMM_BM) * (N / BN);
  const int grid = tiles < sm_count() ? tiles : sm_count();
  return launch_pdl(fn, dim3(grid), dim3(GEMM_THREADS), smem, s, a, b, M, N, K, e, err);
}

// CTA-pair GEMM (256 x BN output tiles on two SMs).  The grid is the number
// of work units or the number of pairs that fit on the device at once,
// whichever is smaller, so the kernel stays persistent.  W's tensor map must
// have box rows BN / 2; `c` is the output map of staged epilogues (ignored by
// the others); ksplit > 1 splits K into that many partial sums.
template <int BN, int ST, class Epi, bool FP8 = false>
cudaError_t gemm2(const CUtensorMap& a, const CUtensorMap& b, const CUtensorMap& c, int M, int N,
                  int K, int ksplit, const Epi& e, uint32_t* err, cudaStream_t s) {
  if (M <= 0) return cudaSuccess;
  if (ksplit < 1 || (K / (FP8 ? 2 * GEMM_BK : GEMM_BK)) % ksplit) return cudaErrorInvalidValue;
  static std::atomic<uint64_t> attr_done{0};
  static std::atomic<int> pairs_cache[64];
  auto fn = gemm2_bf16_tn<BN, ST, Epi, FP8>;
  constexpr int smem = Gemm2Shape<BN, ST, Epi::kStageBytes, Epi::kEpiWarps>::SMEM;
  cudaError_t r = smem_attr_once(attr_done, fn, smem);
  if (r != cudaSuccess) return r;
  int dev = 0;
  if ((r = cudaGetDevice(&dev)) != cudaSuccess) return r;
  int pairs = pairs_cache[dev & 63].load(std::memory_order_relaxed);
  if (pairs <= 0) {
    cudaLaunchConfig_t q = {};
    q.gridDim = dim3(2 * (sm_count() / 2));
    q.blockDim = dim3(gemm2_threads<Epi>());
    q.dynamicSmemBytes = smem;
    int nc = 0;
    r = cudaOccupancyMaxActiveClusters(&nc, fn, &q);
    if (r != cudaSuccess) return r;
    pairs = nc > 0 ? nc : 1;
    pairs_cache[dev & 63].store(pairs, std::memory_order_relaxed);
  }
  const int units = ((M + 2 * GEMM_BM - 1) / (2 * GEMM_BM)) * (N / BN) * ksplit;
  const int grid = 2 * (units < pairs ? units : pairs);
  return launch_pdl(fn, dim3(grid), dim3(gemm2_threads<Epi>()), smem, s, a, b, c, M, N, K, ksplit,
                    e, err);
}

// Output map of the staged (TMA-store) epilogue: {cols, rows, planes} of fp32
// or bf16 with plane stride `plane_bytes`, box {128 bytes of columns, 32, 1}.
bool map_out(CUtensorMap* m, void* base, bool f32, uint64_t rows, uint64_t cols, uint64_t planes,
             uint64_t plane_bytes) {
  auto fn = encode_fn();
  if (!fn || !base) return false;
  const uint64_t es = f32 ? 4 : 2;
  cuuint64_t dims[3] = {cols, rows, planes};
  cuuint64_t strides[2] = {cols * es, plane_bytes};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(128 / es), 32, 1};
  cuuint32_t el[3] = {1, 1, 1};
  return fn(m, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, base,
            dims, strides, box, el, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

constexpr int kActNone = 0, kActGelu = 1, kActSilu = 2;

template <bool F32>
EpiStoreT<F32> store_t(const float* bias, int act) {
  EpiStoreT<F32> e;
  e.bias = bias;
  e.act = act;
  return e;
}

constexpr RowMap kIdentity{1 << 30, 0, 0};

EpiStore store(void* out, int ldo, bool f32, const float* bias, bool gelu, RowMap m = kIdentity) {
  EpiStore e;
  e.out = out;
  e.ldo = ldo;
  e.out_f32 = f32 ? 1 : 0;
  e.bias = bias;
  e.gelu = gelu ? 1 : 0;
  e.omap = m;
  return e;
}

// Residual + LayerNorm launch (ln_mod_kernel: two rows per block; every block
// resident at once, so all rows' loads are in flight together).
template <int NSUB, int MODE>
cudaError_t launch_ln(cudaStream_t s, int M, float* h, const float* sub, size_t sub_plane,
                      const float* gate, RowMap map, const float* shift, const float* scale,
                      int mod_ld, int rows_per_req, __nv_bfloat16* out, float eps, uint8_t* out8,
                      float* out_scale) {
  return launch_pdl(ln_mod_kernel<NSUB, MODE>,
                    dim3((M + LN_ROWS_PER_BLOCK - 1) / LN_ROWS_PER_BLOCK), dim3(LN_THREADS), 0, s,
                    h, sub, sub_plane, gate, M, map, shift, scale, mod_ld, rows_per_req, out, eps,
                    out8, out_scale);
}

int attn_chunks(int max_pages) { return (max_pages * 16 + kSlot + TA_CH - 1) / TA_CH; }

// The attention kernel is persistent: two CTAs per SM (its register bound
// and shared-memory budget are sized for that), or one per work unit if there
// are fewer units.
cudaError_t launch_attention(const CUtensorMap& pool_map, const CUtensorMap& q_map,
                             const AttnParams& p, cudaStream_t s) {
  static std::atomic<uint64_t> attr_done{0};
  cudaError_t r = smem_attr_once(attr_done, attn_tc_kernel, TA_SMEM);
  if (r != cudaSuccess) return r;
  const int ctas = TA_CTAS_PER_SM * sm_count();
  const int units = p.n * p.MC * p.heads;
  return launch_pdl(attn_tc_kernel, dim3(units < ctas ? units : ctas), dim3(TA_THREADS), TA_SMEM, s,
                    pool_map, q_map, p);
}

// Query rows of the 34-row request layout as TMA boxes of 40 rows x 64 dims.
bool map_q(CUtensorMap* m, const void* q, uint64_t rows, int heads) {
  return map_2d(m, q, rows, static_cast<uint64_t>(heads) * 64, static_cast<uint64_t>(heads) * 64,
                TA_QROWS);
}

// ---------------------------------------------------------------- handle
struct WsLayout {
  size_t err, csilu, mod, emb1, xrows, h, sub, xm, xm8, xs, qb, ob, u, z, zb, xmf, st_act, st_exth, st_extl,
      part_o, part_ml, sem, rope, total;
};

struct Handle {
  DfmConfig c;
  DfmWeights w;
  int device;
  int mod_w;  // adaLN output width
  int mc;     // attention chunks per request
  WsLayout ws;
  CUtensorMap m_ada, m_in, m_final, m_coord, m_hid, m_lat;
  CUtensorMap* m_qkv;
  CUtensorMap* m_o;
  CUtensorMap* m_fc1;
  CUtensorMap* m_fc2;
  CUtensorMap* m_qkv8;   // precision 1: e4m3 QKV and fc1 weights
  CUtensorMap* m_fc18;
  CUtensorMap a_xm8;     // precision 1: e4m3 LayerNorm output rows
  // per-workspace/pool descriptors
  const void* plan_ws = nullptr;
  const void* plan_pool = nullptr;
  CUtensorMap a_csilu, a_xrows, a_xm, a_ob, a_u, a_zb, a_xmf, a_act, a_exth, a_extl, pool, q_att;
  CUtensorMap o_sub, o_u;  // staged-epilogue outputs: fp32 sub planes, bf16 MLP hidden
  CUtensorMap o_mod;       // ... and the fp32 modulation rows of every step
};

WsLayout layout_for(const DfmConfig& c, int mc) {
  WsLayout L{};
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off += (bytes + 1023) & ~static_cast<size_t>(1023);
    return o;
  };
  const size_t NR = c.max_requests, R = kSlot * NR, H = c.hidden;
  const size_t modw = static_cast<size_t>(c.layers) * 6 * H + 2 * H;
  L.err = take(256);
  L.csilu = take(c.nfe * NR * H * 2);
  L.mod = take(c.nfe * NR * modw * 4);
  L.emb1 = take(2ull * c.nfe * H * 4);
  L.xrows = take(R * H * 2);
  L.h = take(R * H * 4);
  L.sub = take(2 * R * H * 4);   // two split-K partial planes
  L.xm = take(R * H * 2);
  L.xm8 = take(R * H);        // e4m3 rows (precision 1)
  L.xs = take(R * 4);         // their per-row scales
  L.qb = take(R * H * 2);
  L.ob = take(R * H * 2);
  L.u = take(R * c.ffn * 2);
  L.z = take(NR * c.latent_patch * c.latent_dim * 4);
  L.zb = take(NR * c.latent_patch * c.latent_dim * 2);
  L.xmf = take(NR * c.latent_patch * H * 2);
  L.st_act = take(NR * c.cond_dim * 2);
  L.st_exth = take(NR * c.cond_dim * 2);
  L.st_extl = take(NR * c.latent_patch * c.latent_dim * 2);
  L.part_o = take(NR * mc * c.heads * TA_ROWS * 64 * 4);
  L.part_ml = take(NR * mc * c.heads * TA_ROWS * 2 * 4);
  L.sem = take(NR * c.heads * 4);
  L.rope = take(static_cast<size_t>(c.max_pages_per_req) * 16 * 32 * 8);
  L.total = off;
  return L;
}

int validate_config(const DfmConfig& c) {
  if (c.hidden != kH || c.heads * c.head_dim != c.hidden || c.head_dim != 64) return DFM_ERR_UNSUPPORTED;
  if (c.latent_patch != 16 || c.hidden_patch != 1 || c.latent_dim != 64) return DFM_ERR_UNSUPPORTED;
  if (c.ffn % 256 != 0 || c.cond_dim % 64 != 0 || c.cond_dim <= 0) return DFM_ERR_UNSUPPORTED;
  if (c.page_rows != 16 || (c.precision != DFM_PRECISION_BF16 && c.precision != DFM_PRECISION_FP8))
    return DFM_ERR_UNSUPPORTED;
  if (c.nfe < 1 || c.nfe > EMB_MAX_STEPS) return DFM_ERR_UNSUPPORTED;
  if (c.layers < 1 || c.num_pages < 1 || c.max_pages_per_req < 1 || c.max_requests < 1)
    return DFM_ERR_INVALID_ARG;
  if (static_cast<long long>(c.max_requests) * kSlot * c.ffn >= (1ll << 31)) return DFM_ERR_INVALID_ARG;
  return DFM_OK;
}

bool ensure_plan(Handle* h, void* ws, void* pool, cudaStream_t s) {
  if (h->plan_ws == ws && h->plan_pool == pool) return true;
  const DfmConfig& c = h->c;
  uint8_t* b = static_cast<uint8_t*>(ws);
  const uint64_t NR = c.max_requests, R = kSlot * NR, H = c.hidden;
  const uint64_t LP = NR * c.latent_patch;
  bool ok = map_2d(&h->a_csilu, b + h->ws.csilu, c.nfe * NR, H, H, 128) &&
            map_2d(&h->a_xrows, b + h->ws.xrows, R, H, H, 128) &&
            map_2d(&h->a_xm, b + h->ws.xm, R, H, H, 128) &&
            map_2d(&h->a_ob, b + h->ws.ob, R, H, H, 128) &&
            map_2d(&h->a_u, b + h->ws.u, R, c.ffn, c.ffn, 128) &&
            map_2d(&h->a_zb, b + h->ws.zb, LP, c.latent_dim, c.latent_dim, 128) &&
            map_2d(&h->a_xmf, b + h->ws.xmf, LP, H, H, 128) &&
            map_2d(&h->a_act, b + h->ws.st_act, NR, c.cond_dim, c.cond_dim, 128) &&
            map_2d(&h->a_exth, b + h->ws.st_exth, NR, c.cond_dim, c.cond_dim, 128) &&
            map_2d(&h->a_extl, b + h->ws.st_extl, LP, c.latent_dim, c.latent_dim, 128) &&
            map_q(&h->q_att, b + h->ws.qb, R, c.heads) &&
            map_out(&h->o_sub, b + h->ws.sub, true, R, H, 2, R * H * 4) &&
            map_2d_u8(&h->a_xm8, b + h->ws.xm8, R, H, H, 128) &&
            map_out(&h->o_u, b + h->ws.u, false, R, c.ffn, 1, R * c.ffn * 2) &&
            map_out(&h->o_mod, b + h->ws.mod, true, c.nfe * NR, h->mod_w, 1,
                    c.nfe * NR * static_cast<uint64_t>(h->mod_w) * 4) &&
            map_pool(&h->pool, pool, c.num_pages, c.heads, c.layers * c.nfe * 2);
  if (!ok) {
    h->plan_ws = h->plan_pool = nullptr;
    return false;
  }
  // A workspace seen for the first time starts with a clear error word.
  if (h->plan_ws != ws && (cudaMemset(b + h->ws.err, 0, sizeof(uint32_t)) != cudaSuccess ||
                           cudaMemset(b + h->ws.sem, 0, h->ws.rope - h->ws.sem) != cudaSuccess))
    return false;
  if (h->plan_ws != ws) {
    const int cnt = h->c.max_pages_per_req * 16 * 32;
    rope_table_kernel<<<(cnt + 255) / 256, 256, 0, s>>>(h->w.rope_inv_freq, h->c.max_pages_per_req * 16,
                                                        reinterpret_cast<float2*>(b + h->ws.rope));
    if (cudaGetLastError() != cudaSuccess) return false;
  }
  h->plan_ws = ws;
  h->plan_pool = pool;
  return true;
}

#define CK(...)                                 \
  do {                                          \
    cudaError_t e_ = (__VA_ARGS__);             \
    if (e_ != cudaSuccess) return DFM_ERR_CUDA; \
  } while (0)

}  // namespace

extern "C" {

const char* dfm_error_string(int code) {
  switch (code) {
    case DFM_OK: return "ok";
    case DFM_ERR_INVALID_ARG: return "invalid argument";
    case DFM_ERR_UNSUPPORTED: return "unsupported configuration";
    case DFM_ERR_CUDA: return "CUDA error";
    case DFM_ERR_WORKSPACE: return "workspace too small";
    case DFM_ERR_DEVICE: return "device-side error";
    case DFM_ERR_SCRATCH_LIMIT:
      return "call exceeds the fixed scratch of the no-allocation entry point";
    default: return "unknown error";
  }
}

size_t dfm_pool_bytes(const DfmConfig* c) {
  if (!c) return 0;
  return static_cast<size_t>(c->layers) * c->nfe * 2 * static_cast<size_t>(c->num_pages) *
         c->heads * c->page_rows * c->head_dim * 2;
}

int dfm_create(const DfmConfig* cfg, const DfmWeights* w, void** out) {
  if (!cfg || !w || !out) return DFM_ERR_INVALID_ARG;
  *out = nullptr;
  int rc = validate_config(*cfg);
  if (rc != DFM_OK) return rc;
  const bool fp8 = cfg->precision == DFM_PRECISION_FP8;
  const void* req[] = {w->input_w, w->input_b, w->temb_w1, w->temb_b1, w->temb_w2, w->temb_b2,
                       w->demb_w1, w->demb_b1, w->demb_w2, w->demb_b2, w->ada_w, w->ada_b,
                       fp8 ? w->qkv_w8 : w->qkv_w, w->qk_norm, w->o_w, w->o_b,
                       fp8 ? w->fc1_w8 : w->fc1_w, w->fc1_b, w->fc2_w, w->fc2_b, w->final_w,
                       w->final_b, w->coord_w, w->coord_b, w->hidden_w, w->hidden_b, w->latent_w,
                       w->latent_b, w->rope_inv_freq, fp8 ? w->qkv_ws : w->rope_inv_freq,
                       fp8 ? w->fc1_ws : w->rope_inv_freq};
  for (const void* p : req)
    if (!p) return DFM_ERR_INVALID_ARG;
  if (!encode_fn()) return DFM_ERR_CUDA;
  Handle* h = new (std::nothrow) Handle();
  if (!h) return DFM_ERR_CUDA;
  h->c = *cfg;
  h->w = *w;
  if (cudaGetDevice(&h->device) != cudaSuccess) {
    delete h;
    return DFM_ERR_CUDA;
  }
  const DfmConfig& c = h->c;
  const int H = c.hidden, L = c.layers;
  h->mod_w = L * 6 * H + 2 * H;
  h->mc = attn_chunks(c.max_pages_per_req);
  h->ws = layout_for(c, h->mc);
  h->m_qkv = new CUtensorMap[L];
  h->m_o = new CUtensorMap[L];
  h->m_fc1 = new CUtensorMap[L];
  h->m_fc2 = new CUtensorMap[L];
  h->m_qkv8 = new CUtensorMap[L];
  h->m_fc18 = new CUtensorMap[L];
  auto bw = [](const void* p) { return static_cast<const __nv_bfloat16*>(p); };
  auto b8 = [](const void* p) { return static_cast<const uint8_t*>(p); };
  bool ok = map_2d(&h->m_ada, w->ada_w, h->mod_w, H, H, kAdaBN / 2) &&
            map_2d(&h->m_in, w->input_w, H, H, H, 128) &&
            map_2d(&h->m_final, w->final_w, c.latent_dim, H, H, 64) &&
            map_2d(&h->m_coord, w->coord_w, H, c.latent_dim, c.latent_dim, 128) &&
            map_2d(&h->m_hid, w->hidden_w, H, c.cond_dim, c.cond_dim, 128) &&
            map_2d(&h->m_lat, w->latent_w, H, c.latent_dim, c.latent_dim, 128);
  for (int l = 0; ok && l < L; ++l) {
    // per-layer weights feed the CTA-pair GEMM: box rows = half the tile's N
    ok = map_2d(&h->m_o[l], bw(w->o_w) + static_cast<size_t>(l) * H * H, H, H, H, kOutBN / 2) &&
         map_2d(&h->m_fc2[l], bw(w->fc2_w) + static_cast<size_t>(l) * H * c.ffn, H, c.ffn, c.ffn,
                kOutBN / 2);
    if (ok && fp8)
      ok = map_2d_u8(&h->m_qkv8[l], b8(w->qkv_w8) + static_cast<size_t>(l) * 3 * H * H, 3 * H, H, H,
                     kQkvBN / 2) &&
           map_2d_u8(&h->m_fc18[l], b8(w->fc1_w8) + static_cast<size_t>(l) * c.ffn * H, c.ffn, H, H,
                     kFc1BN / 2);
    else if (ok)
      ok = map_2d(&h->m_qkv[l], bw(w->qkv_w) + static_cast<size_t>(l) * 3 * H * H, 3 * H, H, H,
                  kQkvBN / 2) &&
           map_2d(&h->m_fc1[l], bw(w->fc1_w) + static_cast<size_t>(l) * c.ffn * H, c.ffn, H, H,
                  kFc1BN / 2);
  }
  if (!ok) {
    dfm_destroy(h);
    return DFM_ERR_CUDA;
  }
  *out = h;
  return DFM_OK;
}

size_t dfm_workspace_size(void* handle) {
  return handle ? static_cast<Handle*>(handle)->ws.total : 0;
}

int dfm_destroy(void* handle) {
  Handle* h = static_cast<Handle*>(handle);
  if (!h) return DFM_ERR_INVALID_ARG;
  delete[] h->m_qkv;
  delete[] h->m_o;
  delete[] h->m_fc1;
  delete[] h->m_fc2;
  delete[] h->m_qkv8;
  delete[] h->m_fc18;
  delete h;
  return DFM_OK;
}

int dfm_read_error(void* handle, void* workspace, void* stream, uint32_t* err_word) {
  Handle* h = static_cast<Handle*>(handle);
  if (!h || !workspace || !err_word) return DFM_ERR_INVALID_ARG;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint32_t v = 0;
  uint8_t* e = static_cast<uint8_t*>(workspace) + h->ws.err;
  CK(cudaMemcpyAsync(&v, e, sizeof(v), cudaMemcpyDeviceToHost, s));
  CK(cudaStreamSynchronize(s));
  CK(cudaMemsetAsync(e, 0, sizeof(uint32_t), s));
  // a launch that stopped on an error may leave attention completion counters
  // set; the next tick on this workspace must start them at zero
  if (v) CK(cudaMemsetAsync(static_cast<uint8_t*>(workspace) + h->ws.sem, 0, h->ws.rope - h->ws.sem, s));
  *err_word = v;
  return DFM_OK;
}

}  // extern "C"

namespace {

// The per-layer launches of one tick for a given batch and workspace.  dfm_step
// runs them in order; dfm_tick_launch runs a single one (for timing the tick's
// own kernels in isolation).
struct Tick {
  Handle* hd;
  const DfmBatch* b;
  uint8_t* ws;
  cudaStream_t s;
  uint32_t* err;
  int n, R, RL;
  size_t modw, plane_elems, sub_plane;
  bool fp8;
  AttnParams ap;

  Tick(Handle* h, const DfmBatch* bb, void* workspace, cudaStream_t st) : hd(h), b(bb), s(st) {
    const DfmConfig& c = hd->c;
    ws = static_cast<uint8_t*>(workspace);
    err = reinterpret_cast<uint32_t*>(ws + hd->ws.err);
    n = b->n;
    R = kSlot * n;
    RL = c.latent_patch * n;
    modw = hd->mod_w;
    plane_elems = static_cast<size_t>(c.num_pages) * c.heads * 16 * 64;
    // the second split-K partial of `sub` (O-projection and fc2 outputs)
    sub_plane = kOutSplit > 1 ? static_cast<size_t>(kSlot) * c.max_requests * c.hidden : 0;
    fp8 = c.precision == DFM_PRECISION_FP8;
    ap = AttnParams{};
    ap.q = bf(hd->ws.qb);
    ap.out = bf(hd->ws.ob);
    ap.part_o = f32(hd->ws.part_o);
    ap.part_ml = f32(hd->ws.part_ml);
    ap.sem = reinterpret_cast<int*>(ws + hd->ws.sem);
    ap.cache_len = b->cache_len;
    ap.n_ext = b->n_extend;
    ap.block_table = b->block_table;
    ap.n = n;
    ap.max_pages = c.max_pages_per_req;
    ap.num_pages = c.num_pages;
    ap.heads = c.heads;
    ap.H = c.hidden;
    ap.MC = hd->mc;
    ap.ext_slots = kStride;
    ap.q_rows = kSlot;
    ap.err = err;
  }
  __nv_bfloat16* bf(size_t off) const { return reinterpret_cast<__nv_bfloat16*>(ws + off); }
  float* f32(size_t off) const { return reinterpret_cast<float*>(ws + off); }
  const float* mod(int k, int l) const {   // layer l's six modulation vectors at step k
    return f32(hd->ws.mod) + static_cast<size_t>(k) * n * modw + static_cast<size_t>(l) * 6 * hd->c.hidden;
  }
  float* sub() const { return f32(hd->ws.sub); }

  // Residual add of the pending sublayer (gate * (sub0 + sub1), when `gate`)
  // and adaLN LayerNorm + modulate into the next GEMM's operand rows.
  cudaError_t ln(int M, RowMap map, const float* gate, const float* shift, const float* scale,
                 int rows_per_req, __nv_bfloat16* out, bool to_fp8) const {
    return launch_ln<kOutSplit, LN_ADALN>(s, M, f32(hd->ws.h), gate ? sub() : nullptr, sub_plane,
                                          gate, map, shift, scale, static_cast<int>(modw),
                                          rows_per_req, out, hd->c.ln_eps,
                                          to_fp8 ? ws + hd->ws.xm8 : nullptr, f32(hd->ws.xs));
  }
  // LayerNorm before the attention of layer l (after layer l-1's MLP residual)
  cudaError_t ln_attn(int k, int l) const {
    const float* mb = mod(k, l);
    return ln(R, kIdentity, l > 0 ? mod(k, l - 1) + 5 * hd->c.hidden : nullptr, mb,
              mb + hd->c.hidden, kSlot, bf(hd->ws.xm), fp8);
  }
  // LayerNorm before the MLP of layer l (after its attention residual)
  cudaError_t ln_mlp(int k, int l) const {
    const int H = hd->c.hidden;
    const float* mb = mod(k, l);
    return ln(R, kIdentity, mb + 2 * H, mb + 3 * H, mb + 4 * H, kSlot, bf(hd->ws.xm), fp8);
  }
  cudaError_t qkv(int k, int l) const {
    const DfmConfig& c = hd->c;
    const DfmWeights& w = hd->w;
    const int H = c.hidden;
    EpiQKV eq;
    eq.q_out = bf(hd->ws.qb);
    eq.pool = static_cast<__nv_bfloat16*>(b->kv_pool);
    eq.plane_elems = plane_elems;
    eq.plane_k = (l * c.nfe + k) * 2;
    eq.plane_v = eq.plane_k + 1;
    eq.cache_len = b->cache_len;
    eq.n_ext = b->n_extend;
    eq.block_table = b->block_table;
    eq.max_pages = c.max_pages_per_req;
    eq.num_pages = c.num_pages;
    eq.heads = c.heads;
    eq.H = H;
    eq.slot = kSlot;
    eq.ext_slots = kStride;
    eq.qk_norm = w.qk_norm + static_cast<size_t>(l) * 4 * c.head_dim;
    eq.rope = reinterpret_cast<const float2*>(ws + hd->ws.rope);
    eq.max_pos = c.max_pages_per_req * 16;
    eq.eps = c.ln_eps;
    eq.err = err;
    if (fp8) {
      eq.a_scale = f32(hd->ws.xs);
      eq.w_scale = w.qkv_ws + static_cast<size_t>(l) * 3 * H;
      return gemm2<kQkvBN, kQkvST, EpiQKV, true>(hd->a_xm8, hd->m_qkv8[l], hd->a_xm8, R, 3 * H, H, 1,
                                                 eq, err, s);
    }
    return gemm2<kQkvBN, kQkvST>(hd->a_xm, hd->m_qkv[l], hd->a_xm, R, 3 * H, H, 1, eq, err, s);
  }
  cudaError_t attention(int k, int l) {
    ap.plane_k = (l * hd->c.nfe + k) * 2;
    ap.plane_v = ap.plane_k + 1;
    return launch_attention(hd->pool, hd->q_att, ap, s);
  }
  // attention out projection -> sub (two split-K planes); h += gate_a * sub inside the next LN
  cudaError_t oproj(int l) const {
    const int H = hd->c.hidden;
    return gemm2<kOutBN, kOutST>(hd->a_ob, hd->m_o[l], hd->o_sub, R, H, H, kOutSplit,
                                 store_t<true>(hd->w.o_b + static_cast<size_t>(l) * H, kActNone),
                                 err, s);
  }
  cudaError_t fc1(int l) const {
    const DfmConfig& c = hd->c;
    auto e1 = store_t<false>(hd->w.fc1_b + static_cast<size_t>(l) * c.ffn, kActGelu);
    if (fp8) {
      e1.a_scale = f32(hd->ws.xs);
      e1.w_scale = hd->w.fc1_ws + static_cast<size_t>(l) * c.ffn;
      return gemm2<kFc1BN, kFc1ST, EpiStoreT<false>, true>(hd->a_xm8, hd->m_fc18[l], hd->o_u, R,
                                                          c.ffn, c.hidden, 1, e1, err, s);
    }
    return gemm2<kFc1BN, kFc1ST>(hd->a_xm, hd->m_fc1[l], hd->o_u, R, c.ffn, c.hidden, 1, e1, err, s);
  }
  cudaError_t fc2(int l) const {
    const DfmConfig& c = hd->c;
    return gemm2<kOutBN, kOutST>(hd->a_u, hd->m_fc2[l], hd->o_sub, R, c.hidden, c.ffn, kOutSplit,
                                 store_t<true>(hd->w.fc2_b + static_cast<size_t>(l) * c.hidden,
                                               kActNone),
                                 err, s);
  }
};

// Validation shared by dfm_step and dfm_tick_launch; plans the workspace.
int check_tick(Handle* hd, const DfmBatch* b, void* workspace, size_t workspace_bytes,
               void* stream) {
  if (!hd || !b || !workspace) return DFM_ERR_INVALID_ARG;
  const DfmConfig& c = hd->c;
  const int n = b->n;
  if (n < 1 || n > c.max_requests) return DFM_ERR_INVALID_ARG;
  if (!b->noise || !b->out || !b->cache_len || !b->n_extend || !b->block_table || !b->kv_pool)
    return DFM_ERR_INVALID_ARG;
  if ((b->act_hidden == nullptr) == (b->act_row == nullptr)) return DFM_ERR_INVALID_ARG;
  const bool ext_raw = b->ext_hidden != nullptr || b->ext_latent != nullptr;
  if (ext_raw && (!b->ext_hidden || !b->ext_latent || b->ext_rows)) return DFM_ERR_INVALID_ARG;
  if (workspace_bytes < hd->ws.total) return DFM_ERR_WORKSPACE;
  if (reinterpret_cast<uintptr_t>(workspace) % 256 != 0) return DFM_ERR_INVALID_ARG;
  int dev = -1;
  CK(cudaGetDevice(&dev));
  if (dev != hd->device) return DFM_ERR_INVALID_ARG;
  if (!ensure_plan(hd, workspace, b->kv_pool, static_cast<cudaStream_t>(stream))) return DFM_ERR_CUDA;
  return DFM_OK;
}

}  // namespace

extern "C" {

int dfm_step(void* handle, const DfmBatch* b, void* workspace, size_t workspace_bytes,
             void* stream) {
  Handle* hd = static_cast<Handle*>(handle);
  const int rc = check_tick(hd, b, workspace, workspace_bytes, stream);
  if (rc != DFM_OK) return rc;
  const DfmConfig& c = hd->c;
  const DfmWeights& w = hd->w;
  Tick tk(hd, b, workspace, static_cast<cudaStream_t>(stream));
  cudaStream_t s = tk.s;
  uint8_t* ws = tk.ws;
  uint32_t* err = tk.err;
  const int n = b->n;
  const int H = c.hidden, L = c.layers, NFE = c.nfe, LD = c.latent_dim, LPAT = c.latent_patch;
  const int R = tk.R, RL = tk.RL;
  const size_t modw = hd->mod_w;
  const bool ext_raw = b->ext_hidden != nullptr;
  auto bf = [&](size_t off) { return tk.bf(off); };
  auto f32 = [&](size_t off) { return tk.f32(off); };
  auto W = [](const void* p) { return static_cast<const __nv_bfloat16*>(p); };

  // ---- stage inputs into fixed workspace slots (fixed TMA descriptors)
  if (b->act_hidden)
    CK(cudaMemcpyAsync(ws + hd->ws.st_act, b->act_hidden, static_cast<size_t>(n) * c.cond_dim * 2,
                       cudaMemcpyDeviceToDevice, s));
  if (ext_raw) {
    CK(cudaMemcpyAsync(ws + hd->ws.st_exth, b->ext_hidden, static_cast<size_t>(n) * c.cond_dim * 2,
                       cudaMemcpyDeviceToDevice, s));
    CK(cudaMemcpyAsync(ws + hd->ws.st_extl, b->ext_latent, static_cast<size_t>(RL) * LD * 2,
                       cudaMemcpyDeviceToDevice, s));
  }
  {
    const int cnt = RL * LD;
    CK(launch_pdl(init_z_kernel, dim3((cnt + 255) / 256), dim3(256), 0, s,
                  static_cast<const __nv_bfloat16*>(b->noise), cnt, f32(hd->ws.z), bf(hd->ws.zb)));
  }

  // ---- condition and adaLN modulation for every step (one GEMM)
  TimeGrid grid{};
  for (int k = 0; k < NFE; ++k) {
    // linspace(0, 1, nfe + 1) as the reference builds it (batched_fm.py:113-116)
    const float t0 = static_cast<float>(k) / NFE, t1 = static_cast<float>(k + 1) / NFE;
    grid.t[k] = __bfloat162float(__float2bfloat16(t0));
    grid.dt[k] = __bfloat162float(__float2bfloat16(t1)) - grid.t[k];
  }
  CK(launch_pdl(embed1_kernel, dim3((2 * H * 32 + 255) / 256), dim3(256), 0, s, W(w.temb_w1),
                w.temb_b1, W(w.demb_w1), w.demb_b1, grid, NFE, H, f32(hd->ws.emb1)));
  CK(launch_pdl(embed2_kernel, dim3((H + 7) / 8), dim3(256), 0, s, W(w.temb_w2), w.temb_b2,
                W(w.demb_w2), w.demb_b2, static_cast<const float*>(f32(hd->ws.emb1)),
                static_cast<const __nv_bfloat16*>(b->g_cond), n, NFE, H, bf(hd->ws.csilu)));
  // every step's modulation for every block and the final layer: one CTA-pair
  // GEMM (each pair reads its weight tile once; the GEMM streams ~155 MB of weights)
  CK(gemm2<kAdaBN, kAdaST>(hd->a_csilu, hd->m_ada, hd->o_mod, NFE * n, static_cast<int>(modw), H, 1,
                           store_t<true>(w.ada_b, kActNone), err, s));

  // ---- DiT-input rows: [graduating 17 | active hidden | active latents 16] per request
  __nv_bfloat16* xrows = bf(hd->ws.xrows);
  if (b->act_hidden) {
    CK(gemm<128, 6>(hd->a_act, hd->m_hid, n, H, c.cond_dim,
                    store(xrows, H, false, w.hidden_b, false, RowMap{1, kSlot, kStride}), err, s));
  } else {
    CK(cudaMemcpy2DAsync(xrows + static_cast<size_t>(kStride) * H, kSlot * H * 2, b->act_row, H * 2,
                         H * 2, n, cudaMemcpyDeviceToDevice, s));
  }
  if (ext_raw) {
    CK(gemm<128, 6>(hd->a_exth, hd->m_hid, n, H, c.cond_dim,
                    store(xrows, H, false, w.hidden_b, false, RowMap{1, kSlot, 0}), err, s));
    CK(gemm<128, 6>(hd->a_extl, hd->m_lat, RL, H, LD,
                    store(xrows, H, false, w.latent_b, false, RowMap{LPAT, kSlot, 1}), err, s));
  } else if (b->ext_rows) {
    CK(cudaMemcpy2DAsync(xrows, kSlot * H * 2, b->ext_rows, kStride * H * 2, kStride * H * 2, n,
                         cudaMemcpyDeviceToDevice, s));
  } else {
    CK(cudaMemset2DAsync(xrows, kSlot * H * 2, 0, kStride * H * 2, n, s));
  }

  float* hbuf = f32(hd->ws.h);
  for (int k = 0; k < NFE; ++k) {
    // active latent rows = coordinate_proj(z) (batched_fm.py:117-119)
    CK(gemm<128, 6>(hd->a_zb, hd->m_coord, RL, H, LD,
                    store(xrows, H, false, w.coord_b, false, RowMap{LPAT, kSlot, kStride + 1}), err, s));
    CK(gemm<128, 6>(hd->a_xrows, hd->m_in, R, H, H, store(hbuf, H, true, w.input_b, false), err, s));
    for (int l = 0; l < L; ++l) {
      CK(tk.ln_attn(k, l));
      CK(tk.qkv(k, l));
      CK(tk.attention(k, l));
      CK(tk.oproj(l));
      CK(tk.ln_mlp(k, l));
      CK(tk.fc1(l));
      CK(tk.fc2(l));
    }
    // final layer on the 16 latent rows of each request (after the last MLP
    // residual), then z += dt * v
    const float* mf = tk.mod(k, L);
    CK(tk.ln(RL, RowMap{LPAT, kSlot, kStride + 1}, tk.mod(k, L - 1) + 5 * H, mf, mf + H, LPAT,
             bf(hd->ws.xmf), false));
    EpiSolver es;
    es.z = f32(hd->ws.z);
    es.zb = k == NFE - 1 ? static_cast<__nv_bfloat16*>(b->out) : bf(hd->ws.zb);
    es.bias = w.final_b;
    es.dt = grid.dt[k];
    CK(gemm<64, 8>(hd->a_xmf, hd->m_final, RL, LD, H, es, err, s));
  }
  (void)modw;
  return DFM_OK;
}

int dfm_tick_launch(void* handle, const DfmBatch* b, void* workspace, size_t workspace_bytes,
                    int32_t kernel, int32_t step, int32_t layer, void* stream) {
  Handle* hd = static_cast<Handle*>(handle);
  const int rc = check_tick(hd, b, workspace, workspace_bytes, stream);
  if (rc != DFM_OK) return rc;
  if (step < 0 || step >= hd->c.nfe || layer < 0 || layer >= hd->c.layers) return DFM_ERR_INVALID_ARG;
  Tick tk(hd, b, workspace, static_cast<cudaStream_t>(stream));
  cudaError_t r;
  switch (kernel) {
    case DFM_TICK_LN_ATTN: r = tk.ln_attn(step, layer); break;
    case DFM_TICK_QKV: r = tk.qkv(step, layer); break;
    case DFM_TICK_ATTENTION: r = tk.attention(step, layer); break;
    case DFM_TICK_OPROJ: r = tk.oproj(layer); break;
    case DFM_TICK_LN_MLP: r = tk.ln_mlp(step, layer); break;
    case DFM_TICK_FC1: r = tk.fc1(layer); break;
    case DFM_TICK_FC2: r = tk.fc2(layer); break;
    default: return DFM_ERR_INVALID_ARG;
  }
  return r == cudaSuccess ? DFM_OK : DFM_ERR_CUDA;
}

// ---------------------------------------------------------------- ops
int dfm_linear(const void* A, int64_t lda, int32_t M, int32_t K, const void* Wt, int64_t ldw,
               int32_t N, const float* bias, void* out, int32_t out_f32, int32_t gelu, void* stream) {
  if (!A || !Wt || !out || M < 1 || K < 64 || K % 64 || N < 64 || N % 64) return DFM_ERR_INVALID_ARG;
  if (lda < K || ldw < K || (lda * 2) % 16 || (ldw * 2) % 16) return DFM_ERR_INVALID_ARG;
  if (out_f32 && N % 4) return DFM_ERR_INVALID_ARG;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  CUtensorMap ma, mw, mo;
  int bn = N % 256 == 0 ? 256 : (N % 128 == 0 ? 128 : 64);
  // CTA pairs (256-row tiles) once there is more than one 128-row tile of A;
  // 128-wide tiles when 256-wide ones would leave most SM pairs idle
  const bool pair = M > GEMM_BM && bn >= 128;
  const int tiles_m2 = (M + 2 * GEMM_BM - 1) / (2 * GEMM_BM);
  if (pair && bn == 256 && tiles_m2 * (N / 256) < 64) bn = 128;
  if (!map_2d(&ma, A, M, K, lda, 128) || !map_2d(&mw, Wt, N, K, ldw, pair ? bn / 2 : bn))
    return DFM_ERR_CUDA;
  if (pair && !map_out(&mo, out, out_f32 != 0, M, N, 1, static_cast<uint64_t>(M) * N * 4))
    return DFM_ERR_CUDA;
  EpiStore e = store(out, N, out_f32 != 0, bias, gelu != 0);
  const int act = gelu ? kActGelu : kActNone;
  cudaError_t r;
  if (pair && bn == 256 && out_f32)
    r = gemm2<256, 5>(ma, mw, mo, M, N, K, 1, store_t<true>(bias, act), nullptr, s);
  else if (pair && bn == 256)
    r = gemm2<256, 5>(ma, mw, mo, M, N, K, 1, store_t<false>(bias, act), nullptr, s);
  else if (pair && out_f32)
    r = gemm2<128, 6>(ma, mw, mo, M, N, K, 1, store_t<true>(bias, act), nullptr, s);
  else if (pair)
    r = gemm2<128, 6>(ma, mw, mo, M, N, K, 1, store_t<false>(bias, act), nullptr, s);
  else if (bn == 256)
    r = gemm<256, 4>(ma, mw, M, N, K, e, nullptr, s);
  else if (bn == 128)
    r = gemm<128, 6>(ma, mw, M, N, K, e, nullptr, s);
  else
    r = gemm<64, 8>(ma, mw, M, N, K, e, nullptr, s);
  return r == cudaSuccess ? DFM_OK : DFM_ERR_CUDA;
}

int dfm_gather_rows(const int64_t* table, int32_t n, int32_t hidden, int32_t stride, void* act,
                    void* ext, void* g_cond, void* stream) {
  if (!table || !act || !ext || !g_cond || n < 1 || stride < 1 || hidden < 8 || hidden % 8)
    return DFM_ERR_INVALID_ARG;
  gather_rows_kernel<<<dim3(n, stride + 2), 128, 0, static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const long long*>(table), hidden, stride, static_cast<__nv_bfloat16*>(act),
      static_cast<__nv_bfloat16*>(ext), static_cast<__nv_bfloat16*>(g_cond));
  return cudaGetLastError() == cudaSuccess ? DFM_OK : DFM_ERR_CUDA;
}

// Standalone attention workspace: [error word | partial O | partial (m, l) | counters].
struct AttnWs {
  size_t part_o, part_ml, sem, total;
};
AttnWs attn_ws(int32_t n, int32_t max_pages, int32_t heads) {
  const size_t mc = attn_chunks(max_pages);
  auto up = [](size_t x) { return (x + 1023) & ~static_cast<size_t>(1023); };
  AttnWs a;
  a.part_o = 1024;
  a.part_ml = a.part_o + up(static_cast<size_t>(n) * mc * heads * TA_ROWS * 64 * 4);
  a.sem = a.part_ml + up(static_cast<size_t>(n) * mc * heads * TA_ROWS * 2 * 4);
  a.total = a.sem + up(static_cast<size_t>(n) * heads * 4);
  return a;
}

size_t dfm_attention_workspace_size(int32_t n, int32_t max_pages, int32_t heads) {
  if (n < 1 || max_pages < 1 || heads < 1) return 0;
  return attn_ws(n, max_pages, heads).total;
}

int dfm_paged_attention(const void* q, void* out, const void* kv_pool, int32_t num_pages,
                        int32_t num_planes, int32_t heads, int32_t plane_k, int32_t plane_v,
                        const int32_t* cache_len, const int32_t* n_extend, const int32_t* block_table,
                        int32_t max_pages, int32_t n, void* workspace, size_t workspace_bytes,
                        void* stream) {
  if (!q || !out || !kv_pool || !cache_len || !n_extend || !block_table || !workspace)
    return DFM_ERR_INVALID_ARG;
  if (n < 1 || heads < 1 || num_pages < 1 || max_pages < 1 || plane_k < 0 || plane_v < 0 ||
      plane_k >= num_planes || plane_v >= num_planes)
    return DFM_ERR_INVALID_ARG;
  if (workspace_bytes < dfm_attention_workspace_size(n, max_pages, heads)) return DFM_ERR_WORKSPACE;
  CUtensorMap pm, qm;
  if (!map_pool(&pm, kv_pool, num_pages, heads, num_planes)) return DFM_ERR_CUDA;
  if (!map_q(&qm, q, static_cast<uint64_t>(n) * TA_ROWS, heads)) return DFM_ERR_CUDA;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  const int mc = attn_chunks(max_pages);
  const AttnWs aw = attn_ws(n, max_pages, heads);
  // The kernel resets each completion counter it uses, but a launch that
  // stopped early (a timed-out wait) can leave one set: start from zero.
  if (cudaMemsetAsync(ws + aw.sem, 0, aw.total - aw.sem, s) != cudaSuccess) return DFM_ERR_CUDA;
  AttnParams p{};
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.out = static_cast<__nv_bfloat16*>(out);
  p.err = reinterpret_cast<uint32_t*>(ws);
  p.part_o = reinterpret_cast<float*>(ws + aw.part_o);
  p.part_ml = reinterpret_cast<float*>(ws + aw.part_ml);
  p.sem = reinterpret_cast<int*>(ws + aw.sem);
  p.cache_len = cache_len;
  p.n_ext = n_extend;
  p.block_table = block_table;
  p.n = n;
  p.max_pages = max_pages;
  p.num_pages = num_pages;
  p.heads = heads;
  p.H = heads * 64;
  p.MC = mc;
  p.plane_k = plane_k;
  p.plane_v = plane_v;
  p.ext_slots = kStride;
  p.q_rows = kSlot;
  return launch_attention(pm, qm, p, s) == cudaSuccess ? DFM_OK : DFM_ERR_CUDA;
}

}  // extern "C"

// ---------------------------------------------------------------- no-allocation attention
// Scratch of dfm_paged_attention_noalloc: [error word | partial O | partial
// (m, l) | counters], laid out as for dfm_paged_attention's workspace.  In host
// code `g_noalloc_scratch` names a host-side stand-in, not device memory: the
// kernel gets the address cudaGetSymbolAddress returns for the current device.
static __device__ __align__(256) uint8_t g_noalloc_scratch[DFM_NOALLOC_SCRATCH_BYTES];

namespace {

std::mutex g_noalloc_mu;
void* g_noalloc_ptr[64] = {};

// Device address of the scratch on the current device, looked up once per
// device (a synchronous runtime call: the first call must precede capture).
cudaError_t noalloc_scratch(void** out) {
  int dev = 0;
  cudaError_t r = cudaGetDevice(&dev);
  if (r != cudaSuccess) return r;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* ptr = nullptr;
    r = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (r != cudaSuccess) return r;
    g_noalloc_ptr[dev] = ptr;
  }
  *out = g_noalloc_ptr[dev];
  return cudaSuccess;
}

}  // namespace

extern "C" int dfm_paged_attention_noalloc(const void* q, void* out, const void* kv_pool,
                                           int32_t num_pages, int32_t num_planes, int32_t heads,
                                           int32_t plane_k, int32_t plane_v,
                                           const int32_t* cache_len, const int32_t* n_extend,
                                           const int32_t* block_table, int32_t max_pages,
                                           int32_t n, uint32_t* err_word, void* stream) {
  if (!q || !out || !kv_pool || !cache_len || !n_extend || !block_table || !err_word)
    return DFM_ERR_INVALID_ARG;
  if (n < 1 || heads < 1 || num_pages < 1 || max_pages < 1 || plane_k < 0 || plane_v < 0 ||
      plane_k >= num_planes || plane_v >= num_planes)
    return DFM_ERR_INVALID_ARG;
  const AttnWs aw = attn_ws(n, max_pages, heads);
  if (aw.total > DFM_NOALLOC_SCRATCH_BYTES) return DFM_ERR_SCRATCH_LIMIT;
  void* scratch = nullptr;
  if (noalloc_scratch(&scratch) != cudaSuccess) return DFM_ERR_CUDA;
  CUtensorMap pm, qm;
  if (!map_pool(&pm, kv_pool, num_pages, heads, num_planes)) return DFM_ERR_CUDA;
  if (!map_q(&qm, q, static_cast<uint64_t>(n) * TA_ROWS, heads)) return DFM_ERR_CUDA;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(scratch);
  // the array keeps the previous call's contents: clear the counters this
  // call relies on starting at zero
  if (cudaMemsetAsync(ws + aw.sem, 0, aw.total - aw.sem, s) != cudaSuccess) return DFM_ERR_CUDA;
  AttnParams p{};
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.out = static_cast<__nv_bfloat16*>(out);
  p.err = err_word;
  p.part_o = reinterpret_cast<float*>(ws + aw.part_o);
  p.part_ml = reinterpret_cast<float*>(ws + aw.part_ml);
  p.sem = reinterpret_cast<int*>(ws + aw.sem);
  p.cache_len = cache_len;
  p.n_ext = n_extend;
  p.block_table = block_table;
  p.n = n;
  p.max_pages = max_pages;
  p.num_pages = num_pages;
  p.heads = heads;
  p.H = heads * 64;
  p.MC = attn_chunks(max_pages);
  p.plane_k = plane_k;
  p.plane_v = plane_v;
  p.ext_slots = kStride;
  p.q_rows = kSlot;
  return launch_attention(pm, qm, p, s) == cudaSuccess ? DFM_OK : DFM_ERR_CUDA;
}

// ---------------------------------------------------------------- patch encoder
// The patch encoder's entry points (include/dpe.h) share this translation
// unit's helpers and kernels.
#include "dpe_api.cu"

// ---------------------------------------------------------------- LLM decode attention
// The LLM backbone's paged decode attention (include/dllm.h) shares them too.
#include "llm_api.cu"

// The vocoder (include/dvoc.h).
#include "voc_api.cu"
