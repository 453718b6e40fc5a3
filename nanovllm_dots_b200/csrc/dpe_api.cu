// Host side of the patch-encoder C ABI (include/dpe.h): handle, workspace
// layout and the per-call launch sequence.  Compiled inside dfm_api.cu's
// translation unit (included at its end), whose TMA encoders, GEMM launchers
// and attention launcher it uses; the kernels are the FM head's, with the
// encoder's switches (no qk-norm or rotary, affine LayerNorm, SiLU, causal
// 8-row blocks).
#include "../../include/dpe.h"
#include "pe.cuh"

namespace {

constexpr int kPeRows = PE_ROWS;      // encoder rows per patch (out_ds_rate)
constexpr int kPeOutBN = 128, kPeOutST = 6;
constexpr int kPeOutSplit = 8;        // split-K of out_proj (K = 8 * hidden, M = n is small)
// Calls of at most this many encoder rows (128 requests) run the layer GEMMs
// on 256 x 128 tiles and the O-projection / fc2 as four split-K partials:
// at M = 512 the 256 x 256 tiles would give 24-32 work units for 74 SM pairs.
constexpr int kPeNarrowRows = 1024;
constexpr int kPeNarrowBN = 128, kPeNarrowST = 6, kPeNarrowSplit = 4;
constexpr int kPeSubPlanes = 4;

struct PeLayout {
  size_t err, cl, nn, bt, xc, xd, h, sub, xm, qb, ob, u, part_o, part_ml, sem, outp, total;
};

struct PeHandle {
  DpeConfig c;
  DpeWeights w;
  int device;
  int mc;   // attention chunks per request
  PeLayout ws;
  CUtensorMap m_conv, m_in, m_out;
  CUtensorMap* m_qkv;
  CUtensorMap* m_o;
  CUtensorMap* m_fc1;
  CUtensorMap* m_fc2;
  CUtensorMap* m_n;   // per layer: qkv, o, fc1, fc2 with box rows kPeNarrowBN / 2
  const void* plan_ws = nullptr;
  const void* plan_pool = nullptr;
  CUtensorMap a_xc, a_xd, a_xm, a_ob, a_u, a_xo, pool, q_att, o_sub, o_u, o_outp;
};

PeLayout pe_layout(const DpeConfig& c, int mc) {
  PeLayout L{};
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off += (bytes + 1023) & ~static_cast<size_t>(1023);
    return o;
  };
  const size_t NR = c.max_batch, R = kPeRows * NR, H = c.hidden;
  L.err = take(256);
  L.cl = take(NR * 4);
  L.nn = take(NR * 4);
  L.bt = take(NR * c.max_pages_per_row * 4);
  L.xc = take(R * 2 * c.latent_dim * 2);
  L.xd = take(R * c.latent_dim * 2);
  L.h = take(R * H * 4);
  L.sub = take(kPeSubPlanes * R * H * 4);
  L.xm = take(R * H * 2);
  L.qb = take(R * H * 2);
  L.ob = take(R * H * 2);
  L.u = take(R * c.ffn * 2);
  L.part_o = take(NR * mc * c.heads * TA_ROWS * 64 * 4);
  L.part_ml = take(NR * mc * c.heads * TA_ROWS * 2 * 4);
  L.sem = take(NR * c.heads * 4);
  L.outp = take(static_cast<size_t>(kPeOutSplit) * NR * c.out_dim * 4);
  L.total = off;
  return L;
}

int pe_validate(const DpeConfig& c) {
  if (c.hidden != kH || c.heads * c.head_dim != c.hidden || c.head_dim != 64) return DFM_ERR_UNSUPPORTED;
  if (c.latent_dim != PE_LD || c.patch != PE_FRAMES) return DFM_ERR_UNSUPPORTED;
  if (c.ffn % 256 != 0 || c.ffn <= 0 || c.out_dim % kPeOutBN != 0 || c.out_dim <= 0)
    return DFM_ERR_UNSUPPORTED;
  if (c.layers < 1 || c.max_rows < 1 || c.max_pages_per_row < 1 || c.max_batch < 1)
    return DFM_ERR_INVALID_ARG;
  if (static_cast<long long>(c.max_batch) * kPeRows * c.ffn >= (1ll << 31) ||
      static_cast<long long>(c.max_rows) * c.max_pages_per_row >= (1ll << 31) / 1024)
    return DFM_ERR_INVALID_ARG;
  return DFM_OK;
}

int pe_num_pages(const DpeConfig& c) { return c.max_rows * c.max_pages_per_row; }

bool pe_plan(PeHandle* h, void* ws, void* pool) {
  if (h->plan_ws == ws && h->plan_pool == pool) return true;
  const DpeConfig& c = h->c;
  uint8_t* b = static_cast<uint8_t*>(ws);
  const uint64_t NR = c.max_batch, R = kPeRows * NR, H = c.hidden;
  bool ok = map_2d(&h->a_xc, b + h->ws.xc, R, 2 * c.latent_dim, 2 * c.latent_dim, 128) &&
            map_2d(&h->a_xd, b + h->ws.xd, R, c.latent_dim, c.latent_dim, 128) &&
            map_2d(&h->a_xm, b + h->ws.xm, R, H, H, 128) &&
            map_2d(&h->a_ob, b + h->ws.ob, R, H, H, 128) &&
            map_2d(&h->a_u, b + h->ws.u, R, c.ffn, c.ffn, 128) &&
            // the final rows of request i, concatenated: [NR, 8 * H] over xm
            map_2d(&h->a_xo, b + h->ws.xm, NR, kPeRows * H, kPeRows * H, 128) &&
            map_q(&h->q_att, b + h->ws.qb, R, c.heads) &&
            map_out(&h->o_sub, b + h->ws.sub, true, R, H, kPeSubPlanes, R * H * 4) &&
            map_out(&h->o_u, b + h->ws.u, false, R, c.ffn, 1, R * c.ffn * 2) &&
            map_out(&h->o_outp, b + h->ws.outp, true, NR, c.out_dim, kPeOutSplit,
                    NR * c.out_dim * 4) &&
            map_pool(&h->pool, pool, pe_num_pages(c), c.heads, c.layers * 2);
  if (!ok) {
    h->plan_ws = h->plan_pool = nullptr;
    return false;
  }
  // A workspace seen for the first time starts with a clear error word and
  // clear split-key counters.
  if (h->plan_ws != ws &&
      (cudaMemset(b + h->ws.err, 0, sizeof(uint32_t)) != cudaSuccess ||
       cudaMemset(b + h->ws.sem, 0, NR * c.heads * 4) != cudaSuccess))
    return false;
  h->plan_ws = ws;
  h->plan_pool = pool;
  return true;
}

}  // namespace

extern "C" {

size_t dpe_pool_bytes(const DpeConfig* c) {
  if (!c || pe_validate(*c) != DFM_OK) return 0;
  return static_cast<size_t>(c->layers) * 2 * static_cast<size_t>(pe_num_pages(*c)) * c->heads *
         16 * c->head_dim * 2;
}

int dpe_destroy(void* handle) {
  PeHandle* h = static_cast<PeHandle*>(handle);
  if (!h) return DFM_ERR_INVALID_ARG;
  delete[] h->m_qkv;
  delete[] h->m_o;
  delete[] h->m_fc1;
  delete[] h->m_fc2;
  delete[] h->m_n;
  delete h;
  return DFM_OK;
}

int dpe_create(const DpeConfig* cfg, const DpeWeights* w, void** out) {
  if (!cfg || !w || !out) return DFM_ERR_INVALID_ARG;
  *out = nullptr;
  int rc = pe_validate(*cfg);
  if (rc != DFM_OK) return rc;
  const void* req[] = {w->conv_w, w->conv_b, w->in_w, w->in_b, w->attn_norm, w->ffn_norm,
                       w->qkv_w, w->o_w, w->o_b, w->fc1_w, w->fc1_b, w->fc2_w, w->fc2_b,
                       w->out_w, w->out_b};
  for (const void* p : req)
    if (!p) return DFM_ERR_INVALID_ARG;
  if (!encode_fn()) return DFM_ERR_CUDA;
  PeHandle* h = new (std::nothrow) PeHandle();
  if (!h) return DFM_ERR_CUDA;
  h->c = *cfg;
  h->w = *w;
  if (cudaGetDevice(&h->device) != cudaSuccess) {
    delete h;
    return DFM_ERR_CUDA;
  }
  const DpeConfig& c = h->c;
  const int H = c.hidden, L = c.layers;
  h->mc = (c.max_pages_per_row * 16 + TA_CH - 1) / TA_CH;
  h->ws = pe_layout(c, h->mc);
  h->m_qkv = new CUtensorMap[L];
  h->m_o = new CUtensorMap[L];
  h->m_fc1 = new CUtensorMap[L];
  h->m_fc2 = new CUtensorMap[L];
  h->m_n = new CUtensorMap[4 * L];
  auto bw = [](const void* p) { return static_cast<const __nv_bfloat16*>(p); };
  bool ok = map_2d(&h->m_conv, w->conv_w, c.latent_dim, 2 * c.latent_dim, 2 * c.latent_dim, 64) &&
            map_2d(&h->m_in, w->in_w, H, c.latent_dim, c.latent_dim, 128) &&
            map_2d(&h->m_out, w->out_w, c.out_dim, kPeRows * H, kPeRows * H, kPeOutBN / 2);
  for (int l = 0; ok && l < L; ++l) {
    const size_t HH = static_cast<size_t>(H) * H, HF = static_cast<size_t>(H) * c.ffn;
    ok = map_2d(&h->m_qkv[l], bw(w->qkv_w) + l * 3 * HH, 3 * H, H, H, kQkvBN / 2) &&
         map_2d(&h->m_o[l], bw(w->o_w) + l * HH, H, H, H, kOutBN / 2) &&
         map_2d(&h->m_fc1[l], bw(w->fc1_w) + l * HF, c.ffn, H, H, kFc1BN / 2) &&
         map_2d(&h->m_fc2[l], bw(w->fc2_w) + l * HF, H, c.ffn, c.ffn, kOutBN / 2);
    CUtensorMap* mn = h->m_n + 4 * l;
    ok = ok && map_2d(&mn[0], bw(w->qkv_w) + l * 3 * HH, 3 * H, H, H, kPeNarrowBN / 2) &&
         map_2d(&mn[1], bw(w->o_w) + l * HH, H, H, H, kPeNarrowBN / 2) &&
         map_2d(&mn[2], bw(w->fc1_w) + l * HF, c.ffn, H, H, kPeNarrowBN / 2) &&
         map_2d(&mn[3], bw(w->fc2_w) + l * HF, H, c.ffn, c.ffn, kPeNarrowBN / 2);
  }
  if (!ok) {
    dpe_destroy(h);
    return DFM_ERR_CUDA;
  }
  *out = h;
  return DFM_OK;
}

size_t dpe_workspace_size(void* handle) {
  return handle ? static_cast<PeHandle*>(handle)->ws.total : 0;
}

int dpe_read_error(void* handle, void* workspace, void* stream, uint32_t* err_word) {
  PeHandle* h = static_cast<PeHandle*>(handle);
  if (!h || !workspace || !err_word) return DFM_ERR_INVALID_ARG;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint32_t v = 0;
  uint8_t* e = static_cast<uint8_t*>(workspace) + h->ws.err;
  CK(cudaMemcpyAsync(&v, e, sizeof(v), cudaMemcpyDeviceToHost, s));
  CK(cudaStreamSynchronize(s));
  CK(cudaMemsetAsync(e, 0, sizeof(uint32_t), s));
  *err_word = v;
  return DFM_OK;
}

int dpe_decode(void* handle, const DpeBatch* b, void* workspace, size_t workspace_bytes,
               void* stream) {
  PeHandle* hd = static_cast<PeHandle*>(handle);
  if (!hd || !b || !workspace) return DFM_ERR_INVALID_ARG;
  const DpeConfig& c = hd->c;
  const DpeWeights& w = hd->w;
  const int n = b->n;
  if (n < 1 || n > c.max_batch) return DFM_ERR_INVALID_ARG;
  if (!b->patches || !b->rows || !b->seqlens || !b->conv_tail || !b->kv_pool || !b->out)
    return DFM_ERR_INVALID_ARG;
  if (workspace_bytes < hd->ws.total) return DFM_ERR_WORKSPACE;
  if (reinterpret_cast<uintptr_t>(workspace) % 256 != 0) return DFM_ERR_INVALID_ARG;
  int dev = -1;
  CK(cudaGetDevice(&dev));
  if (dev != hd->device) return DFM_ERR_INVALID_ARG;
  if (!pe_plan(hd, workspace, b->kv_pool)) return DFM_ERR_CUDA;

  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  uint32_t* err = reinterpret_cast<uint32_t*>(ws + hd->ws.err);
  const int H = c.hidden, L = c.layers, R = kPeRows * n;
  auto bf = [&](size_t off) { return reinterpret_cast<__nv_bfloat16*>(ws + off); };
  auto f32 = [&](size_t off) { return reinterpret_cast<float*>(ws + off); };
  int* cl = reinterpret_cast<int*>(ws + hd->ws.cl);
  int* nn = reinterpret_cast<int*>(ws + hd->ws.nn);
  int* bt = reinterpret_cast<int*>(ws + hd->ws.bt);
  const int num_pages = pe_num_pages(c);

  // ---- per-request state from the cache rows; conv input rows
  CK(launch_pdl(pe_prep_kernel, dim3((R * 32 + 255) / 256), dim3(256), 0, s,
                static_cast<const __nv_bfloat16*>(b->patches), b->rows, n, b->seqlens,
                static_cast<__nv_bfloat16*>(b->conv_tail), c.max_rows, c.max_pages_per_row,
                bf(hd->ws.xc), cl, nn, bt, err));
  // ---- ds_proj (the stride-2 conv as a K = 128 GEMM), then in_proj into the fp32 stream
  CK(gemm<64, 8>(hd->a_xc, hd->m_conv, R, c.latent_dim, 2 * c.latent_dim,
                 store(bf(hd->ws.xd), c.latent_dim, false, w.conv_b, false), err, s));
  float* hbuf = f32(hd->ws.h);
  CK(gemm<128, 6>(hd->a_xd, hd->m_in, R, H, c.latent_dim, store(hbuf, H, true, w.in_b, false),
                  err, s));

  AttnParams ap{};
  ap.q = bf(hd->ws.qb);
  ap.out = bf(hd->ws.ob);
  ap.part_o = f32(hd->ws.part_o);
  ap.part_ml = f32(hd->ws.part_ml);
  ap.sem = reinterpret_cast<int*>(ws + hd->ws.sem);
  ap.cache_len = cl;
  ap.n_ext = nn;
  ap.block_table = bt;
  ap.n = n;
  ap.max_pages = c.max_pages_per_row;
  ap.num_pages = num_pages;
  ap.heads = c.heads;
  ap.H = H;
  ap.MC = hd->mc;
  ap.ext_slots = TA_ROWS;   // all 8 rows causal; none sees a fixed block
  ap.q_rows = kPeRows;
  ap.err = err;

  float* sub = f32(hd->ws.sub);
  __nv_bfloat16* xm = bf(hd->ws.xm);
  const size_t sub_plane = static_cast<size_t>(kPeRows) * c.max_batch * H;
  const bool narrow = R <= kPeNarrowRows;
  const int nsub = narrow ? kPeNarrowSplit : kOutSplit;
  // x += the pending sublayer (nsub split-K partials) inside the LayerNorm; norm = the
  // [weight | bias] pair of an affine LayerNorm, or null for the plain residual rows
  auto ln = [&](const float* subp, const float* norm) {
    const float* shift = norm ? norm + H : nullptr;
    if (norm && nsub == kPeNarrowSplit)
      return launch_ln<kPeNarrowSplit, LN_AFFINE>(s, R, hbuf, subp, sub_plane, nullptr, kIdentity,
                                                  shift, norm, 0, kPeRows, xm, c.ln_eps, nullptr,
                                                  nullptr);
    if (norm)
      return launch_ln<kOutSplit, LN_AFFINE>(s, R, hbuf, subp, sub_plane, nullptr, kIdentity,
                                             shift, norm, 0, kPeRows, xm, c.ln_eps, nullptr,
                                             nullptr);
    if (nsub == kPeNarrowSplit)
      return launch_ln<kPeNarrowSplit, LN_NONE>(s, R, hbuf, subp, sub_plane, nullptr, kIdentity,
                                                nullptr, nullptr, 0, kPeRows, xm, c.ln_eps,
                                                nullptr, nullptr);
    return launch_ln<kOutSplit, LN_NONE>(s, R, hbuf, subp, sub_plane, nullptr, kIdentity, nullptr,
                                         nullptr, 0, kPeRows, xm, c.ln_eps, nullptr, nullptr);
  };

  const size_t plane_elems = static_cast<size_t>(num_pages) * c.heads * 16 * 64;
  for (int l = 0; l < L; ++l) {
    // x += previous MLP (inside the LayerNorm), h = attn_norm(x)
    CK(ln(l > 0 ? sub : nullptr, w.attn_norm + static_cast<size_t>(l) * 2 * H));
    EpiQKVT<false> eq{};
    eq.q_out = bf(hd->ws.qb);
    eq.pool = static_cast<__nv_bfloat16*>(b->kv_pool);
    eq.plane_elems = plane_elems;
    eq.plane_k = 2 * l;
    eq.plane_v = 2 * l + 1;
    eq.cache_len = cl;
    eq.n_ext = nn;
    eq.block_table = bt;
    eq.max_pages = c.max_pages_per_row;
    eq.num_pages = num_pages;
    eq.heads = c.heads;
    eq.H = H;
    eq.slot = kPeRows;
    eq.ext_slots = kPeRows;
    eq.qk_norm = nullptr;
    eq.rope = nullptr;
    eq.max_pos = 1;
    eq.eps = c.ln_eps;
    eq.err = err;
    const CUtensorMap* mn = hd->m_n + 4 * l;
    const auto e_o = store_t<true>(w.o_b + static_cast<size_t>(l) * H, kActNone);
    const auto e_fc1 = store_t<false>(w.fc1_b + static_cast<size_t>(l) * c.ffn, kActSilu);
    const auto e_fc2 = store_t<true>(w.fc2_b + static_cast<size_t>(l) * H, kActNone);
    if (narrow)
      CK((gemm2<kPeNarrowBN, kPeNarrowST>(hd->a_xm, mn[0], hd->a_xm, R, 3 * H, H, 1, eq, err, s)));
    else
      CK(gemm2<kQkvBN, kQkvST>(hd->a_xm, hd->m_qkv[l], hd->a_xm, R, 3 * H, H, 1, eq, err, s));
    ap.plane_k = eq.plane_k;
    ap.plane_v = eq.plane_v;
    CK(launch_attention(hd->pool, hd->q_att, ap, s));
    if (narrow)
      CK((gemm2<kPeNarrowBN, kPeNarrowST>(hd->a_ob, mn[1], hd->o_sub, R, H, H, nsub, e_o, err, s)));
    else
      CK(gemm2<kOutBN, kOutST>(hd->a_ob, hd->m_o[l], hd->o_sub, R, H, H, nsub, e_o, err, s));
    // x += attention (inside the LayerNorm), h = ffn_norm(x)
    CK(ln(sub, w.ffn_norm + static_cast<size_t>(l) * 2 * H));
    if (narrow) {
      CK((gemm2<kPeNarrowBN, kPeNarrowST>(hd->a_xm, mn[2], hd->o_u, R, c.ffn, H, 1, e_fc1, err, s)));
      CK((gemm2<kPeNarrowBN, kPeNarrowST>(hd->a_u, mn[3], hd->o_sub, R, H, c.ffn, nsub, e_fc2, err,
                                          s)));
    } else {
      CK(gemm2<kFc1BN, kFc1ST>(hd->a_xm, hd->m_fc1[l], hd->o_u, R, c.ffn, H, 1, e_fc1, err, s));
      CK(gemm2<kOutBN, kOutST>(hd->a_u, hd->m_fc2[l], hd->o_sub, R, H, c.ffn, nsub, e_fc2, err, s));
    }
  }
  // x += last MLP; the bf16 rows, 8 per request, are out_proj's [n, 8H] operand
  CK(ln(sub, nullptr));
  CK(gemm2<kPeOutBN, kPeOutST>(hd->a_xo, hd->m_out, hd->o_outp, n, c.out_dim, kPeRows * H,
                               kPeOutSplit, store_t<true>(w.out_b, kActNone), err, s));
  const int cnt = n * c.out_dim / 4;
  CK(launch_pdl(pe_out_reduce_kernel, dim3((cnt + 255) / 256), dim3(256), 0, s,
                static_cast<const float*>(f32(hd->ws.outp)), kPeOutSplit,
                static_cast<size_t>(c.max_batch) * c.out_dim, n, c.out_dim,
                static_cast<__nv_bfloat16*>(b->out)));
  return DFM_OK;
}

}  // extern "C"
