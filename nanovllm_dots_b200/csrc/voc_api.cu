// Host side of the vocoder C ABI (include/dvoc.h): configuration checks, the
// table of the decoder's convolutions and activations (execution order),
// workspace layout, TMA descriptors and the launch sequence of one call.
// Included into dfm_api.cu (one translation unit, one library).
#include <vector>

#include "../../include/dvoc.h"
#include "voc.cuh"

namespace {

// The LSTM step keeps 32 requests' h (4L floats each, transposed) and its
// block's 32 rows of W_hh (4L floats each) in shared memory.
constexpr int kVocMaxLatent = 192;
constexpr int kVocLstmSmem = 4 * kVocMaxLatent * (33 + 4 * VS_J) * 4;

int vpad(int c) { return (c + 31) / 32 * 32; }
size_t valign(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }
int round128(long long x) { return static_cast<int>((x + 127) / 128 * 128); }
int round256(long long x) { return static_cast<int>((x + 255) / 256 * 256); }

// One convolution of the decoder as the conv kernel sees it.
struct VocConv {
  int cin_p;          // padded input channels (K per tap)
  int N;              // output columns
  int taps, off0, dil;
  int u, cp_out;      // transposed conv: u phases of cp_out columns; else u = 1
  bool rows128 = false;  // input rows only a multiple of 128 (conv_pre's output)
  size_t w_off, b_off;
  CUtensorMap wmap;
};

struct VocHandle {
  DvocConfig c;
  DvocWeights w;
  int device = 0;
  int L = 0, Lp = 0, Hm = 0, per = 0, nk = 0, ns = 0;
  int ch[DVOC_MAX_STAGES] = {};   // unpadded channels per stage
  std::vector<VocConv> convs;
  std::vector<size_t> act_off;
  std::vector<int> act_cp;
  size_t conv_floats = 0, bias_floats = 0, act_floats = 0;
  // workspace (maxima)
  size_t o_err = 0, o_p = 0, o_s = 0, o_gx = 0, o_y0 = 0, o_y1 = 0, o_z = 0, o_h0 = 0, o_h1 = 0,
         o_din = 0, o_din32 = 0, o_x = 0, o_x16 = 0, o_u = 0, o_h = 0, o_a = 0, o_c1 = 0, total = 0;
  // tensor maps of the last call's shape
  const void* plan_ws = nullptr;
  int plan_n = -1, plan_t = -1;
  CUtensorMap m_din;
  CUtensorMap m_xin[DVOC_MAX_STAGES];
  CUtensorMap m_xin_h[DVOC_MAX_STAGES];  // 64-frame boxes (transposed convs on the halo kernel)
  CUtensorMap m_act[DVOC_MAX_STAGES];
  CUtensorMap m_act_h[DVOC_MAX_STAGES];  // 64-frame boxes (halo kernel)
  CUtensorMap m_u[DVOC_MAX_STAGES];      // residual sources of the resblock convs
  CUtensorMap m_h[DVOC_MAX_STAGES];
};

int voc_validate(const DvocConfig& c) {
  if (c.latent_dim < 2 || c.latent_dim > kVocMaxLatent || c.latent_dim % 2) return DFM_ERR_UNSUPPORTED;
  if (c.num_stages < 1 || c.num_stages > DVOC_MAX_STAGES) return DFM_ERR_UNSUPPORTED;
  if (c.num_kernels < 1 || c.num_kernels > DVOC_MAX_KERNELS) return DFM_ERR_UNSUPPORTED;
  if (c.resblock_type != 1 && c.resblock_type != 2) return DFM_ERR_UNSUPPORTED;
  if (c.mi_layers < 1 || c.mi_layers > 16) return DFM_ERR_UNSUPPORTED;
  if (c.lookahead < 0 || c.lookahead > 16) return DFM_ERR_UNSUPPORTED;
  if (c.max_batch < 1 || c.max_frames < 1) return DFM_ERR_INVALID_ARG;
  if (c.initial_channels < 1 || c.initial_channels > 8192) return DFM_ERR_UNSUPPORTED;
  long long hop = 1;
  for (int i = 0; i < c.num_stages; ++i) {
    if (c.upsample_rates[i] < 1 || c.upsample_rates[i] > 64) return DFM_ERR_UNSUPPORTED;
    if ((c.initial_channels >> (i + 1)) < 1) return DFM_ERR_UNSUPPORTED;
    hop *= c.upsample_rates[i];
  }
  if (hop > (1 << 20)) return DFM_ERR_UNSUPPORTED;
  // the activation kernel's grid covers the longest signal in its y dimension
  if (static_cast<long long>(c.max_frames) * hop > 65535ll * VA_R * VA_WARPS) return DFM_ERR_UNSUPPORTED;
  for (int j = 0; j < c.num_kernels; ++j) {
    if (c.resblock_kernel_sizes[j] < 1 || c.resblock_kernel_sizes[j] > 64) return DFM_ERR_UNSUPPORTED;
    for (int l = 0; l < 3; ++l)
      if (c.resblock_dilations[j][l] < 1 || c.resblock_dilations[j][l] > 64)
        return DFM_ERR_UNSUPPORTED;
  }
  // the longest decoded signal must index in 32 bits
  if (static_cast<long long>(c.max_frames) * hop * vpad(c.initial_channels) > (1ll << 31))
    return DFM_ERR_UNSUPPORTED;
  return DFM_OK;
}

// Fill the layer tables (no device work).
void voc_tables(VocHandle& h) {
  const DvocConfig& c = h.c;
  h.L = c.latent_dim;
  h.Lp = vpad(c.latent_dim);
  h.Hm = 4 * c.latent_dim;
  h.ns = c.num_stages;
  h.nk = c.num_kernels;
  h.per = c.resblock_type == 1 ? 6 : 2;
  for (int i = 0; i < h.ns; ++i) h.ch[i] = c.initial_channels >> (i + 1);
  size_t wo = 0, bo = 0;
  auto add = [&](int cin_p, int N, int taps, int off0, int dil, int u, int cp_out) {
    VocConv v;
    v.cin_p = cin_p; v.N = N; v.taps = taps; v.off0 = off0; v.dil = dil; v.u = u; v.cp_out = cp_out;
    v.w_off = wo; v.b_off = bo;
    wo += static_cast<size_t>(N) * taps * cin_p;
    bo += N;
    h.convs.push_back(v);
  };
  const int c0p = vpad(c.initial_channels);
  add(h.Lp, c0p, 2 * c.lookahead + 1, -c.lookahead, 1, 1, c0p);
  size_t ao = 0;
  for (int i = 0; i < h.ns; ++i) {
    const int cin_p = i ? vpad(h.ch[i - 1]) : c0p, cp = vpad(h.ch[i]), u = c.upsample_rates[i];
    add(cin_p, u * cp, 2, -1, 1, u, cp);
    h.convs.back().rows128 = i == 0;
    for (int j = 0; j < h.nk; ++j) {
      const int k = c.resblock_kernel_sizes[j];
      const int nl = c.resblock_type == 1 ? 3 : 2;
      for (int l = 0; l < nl; ++l) {
        const int d = c.resblock_dilations[j][l];
        add(cp, cp, k, -(k - 1) * d, d, 1, cp);
        if (c.resblock_type == 1) add(cp, cp, k, -(k - 1), 1, 1, cp);
      }
      for (int a = 0; a < h.per; ++a) {
        h.act_off.push_back(ao);
        h.act_cp.push_back(cp);
        ao += 26 * static_cast<size_t>(cp);
      }
    }
  }
  const int cpl = vpad(h.ch[h.ns - 1]);
  h.act_off.push_back(ao);
  h.act_cp.push_back(cpl);
  ao += 26 * static_cast<size_t>(cpl);
  h.conv_floats = wo;
  h.bias_floats = bo;
  h.act_floats = ao;
}

// Frames per request at each point of the decoder for a call of T latent frames.
struct VocRows {
  int tpre, cpre;                 // conv_pre: T, rounded to 128
  long long t[DVOC_MAX_STAGES];   // valid frames after stage i
  int cap[DVOC_MAX_STAGES];       // rounded to 256
};

VocRows voc_rows(const VocHandle& h, int T) {
  VocRows r;
  r.tpre = T;
  r.cpre = round128(T);
  long long t = T;
  for (int i = 0; i < h.ns; ++i) {
    t *= h.c.upsample_rates[i];
    r.t[i] = t;
    r.cap[i] = round256(t);   // whole 256-frame tiles of the narrow convolutions
  }
  return r;
}

void voc_layout(VocHandle& h) {
  const DvocConfig& c = h.c;
  const size_t nb = c.max_batch, F = c.max_frames;
  const VocRows r = voc_rows(h, c.max_frames);
  size_t big = static_cast<size_t>(r.cpre) * vpad(c.initial_channels);
  for (int i = 0; i < h.ns; ++i) {
    const size_t s = static_cast<size_t>(r.cap[i]) * vpad(h.ch[i]);
    big = s > big ? s : big;
  }
  big *= nb;
  size_t o = 0;
  auto take = [&](size_t floats) {
    const size_t at = o;
    o = valign(o + floats * 4);
    return at;
  };
  h.o_err = take(64);
  h.o_p = take(nb * F * h.L);
  h.o_s = take(nb * F * h.Hm);
  h.o_gx = take(nb * F * 4 * h.Hm);
  h.o_y0 = take(nb * F * h.Hm);
  h.o_y1 = take(nb * F * h.Hm);
  h.o_z = take(nb * F * h.L);
  h.o_h0 = take(nb * h.Hm);
  h.o_h1 = take(nb * h.Hm);
  h.o_din = take(nb * static_cast<size_t>(r.cpre) * h.Lp / 2);  // fp16
  h.o_din32 = take(nb * static_cast<size_t>(r.cpre) * h.Lp);
  h.o_x = take(big);
  h.o_x16 = take(big / 2);                                        // fp16 copy of X
  h.o_u = take(big);
  h.o_h = take(big);
  h.o_a = take(big);
  h.o_c1 = take(big);
  h.total = o;
}

// 3-D fp16 operand [n][rows][cp], box {32 channels, box_rows frames, 1},
// 64-byte swizzle (one 64-byte row per frame).
bool voc_map_act(CUtensorMap* m, const void* base, int n, int rows, int cp, int box_rows = VC_BM) {
  auto fn = encode_fn();
  if (!fn || !base) return false;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(cp), static_cast<cuuint64_t>(rows),
                        static_cast<cuuint64_t>(n)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(cp) * 2,
                           static_cast<cuuint64_t>(cp) * rows * 2};
  cuuint32_t box[3] = {32, static_cast<cuuint32_t>(box_rows), 1};
  cuuint32_t es[3] = {1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 3-D fp32 tensor [n][rows][cp] (a residual source), box {32 channels, 128
// frames, 1}, 128-byte swizzle.
bool voc_map_f32(CUtensorMap* m, const void* base, int n, int rows, int cp) {
  auto fn = encode_fn();
  if (!fn || !base) return false;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(cp), static_cast<cuuint64_t>(rows),
                        static_cast<cuuint64_t>(n)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(cp) * 4,
                           static_cast<cuuint64_t>(cp) * rows * 4};
  cuuint32_t box[3] = {32, static_cast<cuuint32_t>(VC_BM), 1};
  cuuint32_t es[3] = {1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<void*>(base), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 2-D fp16 weight [N][K], box {32, bn}, 64-byte swizzle.
bool voc_map_w(CUtensorMap* m, const void* base, int N, int K, int bn) {
  auto fn = encode_fn();
  if (!fn || !base) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(N)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(K) * 2};
  cuuint32_t box[2] = {32, static_cast<cuuint32_t>(bn)};
  cuuint32_t es[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int voc_bn(int N) {
  if (N % 256 == 0) return 256;
  if (N % 128 == 0) return 128;
  if (N % 96 == 0) return 96;
  if (N % 64 == 0) return 64;
  return 32;
}

// Conv CTAs that fit on one SM by shared memory and TMEM (the kernels allow 2;
// a CTA that holds more than half of the 512 TMEM columns runs alone).
int voc_ctas_per_sm(int smem, uint32_t tmem_cols) {
  return 2 * (smem + 1024) <= 233472 && tmem_cols <= 256 ? 2 : 1;
}

template <int BN, int ST>
cudaError_t voc_conv_launch(const CUtensorMap& a, const CUtensorMap& w, const VcArgs& p,
                            uint32_t* err, cudaStream_t s) {
  static std::atomic<uint64_t> attr_done{0};
  auto fn = voc_conv_kernel<BN, ST>;
  constexpr int smem = VcShape<BN, ST>::SMEM;
  cudaError_t r = smem_attr_once(attr_done, fn, smem);
  if (r != cudaSuccess) return r;
  const int tiles = p.tiles_m * (p.N / BN);
  const int ctas = voc_ctas_per_sm(smem, VcShape<BN, ST>::TMEM_COLS) * sm_count();
  const int grid = tiles < ctas ? tiles : ctas;
  return launch_pdl(fn, dim3(grid), dim3(VC_THREADS), smem, s, a, w, p, err);
}

template <int BN, int SA, int SB, int SE = 0, int MT = 1, int NB = 2>
cudaError_t voc_halo_launch(const CUtensorMap& a, const CUtensorMap& w, const CUtensorMap& res,
                            VcArgs p, uint32_t* err, cudaStream_t s) {
  static std::atomic<uint64_t> attr_done{0};
  auto fn = voc_conv_halo_kernel<BN, SA, SB, SE, MT, NB>;
  using S = VhShape<BN, SA, SB, SE, MT, NB>;
  constexpr int smem = S::SMEM;
  cudaError_t r = smem_attr_once(attr_done, fn, smem);
  if (r != cudaSuccess) return r;
  p.tiles_t /= MT;                  // tiles of MT x 128 frames (rows are multiples of 256)
  p.tiles_m /= MT;
  const int tiles = p.tiles_m * (p.N / BN);
  const int ctas = voc_ctas_per_sm(smem, S::TMEM_COLS) * sm_count();
  const int grid = tiles < ctas ? tiles : ctas;
  return launch_pdl(fn, dim3(grid), dim3(VC_THREADS), smem, s, a, w, res, p, err);
}

int voc_halo_bn(int N);

// The resblock convolutions and the transposed convs (causal, taps spanning at
// most VH_HALO frames) run on the halo kernel: one A tile per channel block
// for all taps.  conv_pre (centred) stays on voc_conv_kernel, and so does a
// transposed conv whose tile would be 256 frames (N <= 64) over conv_pre's
// output, whose rows are only a multiple of 128.
bool voc_halo(const VocConv& v) {
  return v.taps > 1 && (v.taps - 1) * v.dil <= VH_HALO && v.off0 == -(v.taps - 1) * v.dil &&
         !(v.rows128 && voc_halo_bn(v.N) <= 64);
}

// Tiles of the resblock convolutions: one tile of N = 32 or 64, else 256 or
// 192 columns with one accumulator buffer (256 TMEM columns, so two CTAs per
// SM still fit), else 128/96 double-buffered.  At N = 32 the residual is
// staged by TMA in two buffers; at 64 a single buffer measured slower than
// the direct loads, which the wider tiles keep.
int voc_halo_bn(int N) {
  return N == 32 ? 32 : N == 64 ? 64 : N % 256 == 0 ? 256 : N % 192 == 0 ? 192 : N % 128 == 0 ? 128
         : N % 96 == 0 ? 96 : 32;
}

cudaError_t voc_conv(const VocHandle& h, const VocConv& v, const CUtensorMap& amap, int n,
                     int rows_in, float* out, long long out_b, int out_rows, const float* res,
                     int accum, float div, uint32_t* err, cudaStream_t s,
                     const CUtensorMap* halo_map = nullptr, const CUtensorMap* res_map = nullptr,
                     __half* out16 = nullptr) {
  VcArgs p;
  p.tiles_t = rows_in / VC_BM;
  p.tiles_m = n * p.tiles_t;
  p.N = v.N;
  p.nkb_c = v.cin_p / VC_BK;
  p.taps = v.taps;
  p.off0 = v.off0;
  p.dil = v.dil;
  p.bias = h.w.conv_b + v.b_off;
  p.out = out;
  p.out_b = out_b;
  p.out_ld = v.N;
  p.u = v.u;
  p.cp_out = v.cp_out;
  p.out_rows = out_rows;
  p.res = res;
  p.accum = accum;
  p.div = div;
  p.out16 = out16;
  if (halo_map && voc_halo(v)) {
    switch (voc_halo_bn(v.N)) {
      case 256: return voc_halo_launch<256, 3, 4, 0, 1, 1>(*halo_map, v.wmap, *halo_map, p, err, s);
      case 192: return voc_halo_launch<192, 3, 6, 0, 1, 1>(*halo_map, v.wmap, *halo_map, p, err, s);
      case 128: return voc_halo_launch<128, 3, 6>(*halo_map, v.wmap, *halo_map, p, err, s);
      case 96: return voc_halo_launch<96, 3, 8>(*halo_map, v.wmap, *halo_map, p, err, s);
      case 64: return voc_halo_launch<64, 2, 8, 0, 2>(*halo_map, v.wmap, *halo_map, p, err, s);
      default:
        if (res && res_map)
          return voc_halo_launch<32, 2, 8, 1, 2>(*halo_map, v.wmap, *res_map, p, err, s);
        return voc_halo_launch<32, 2, 8, 0, 2>(*halo_map, v.wmap, *halo_map, p, err, s);
    }
  }
  switch (voc_bn(v.N)) {
    case 256: return voc_conv_launch<256, 8>(amap, v.wmap, p, err, s);
    case 128: return voc_conv_launch<128, 6>(amap, v.wmap, p, err, s);
    case 96: return voc_conv_launch<96, 7>(amap, v.wmap, p, err, s);
    case 64: return voc_conv_launch<64, 8>(amap, v.wmap, p, err, s);
    default: return voc_conv_launch<32, 8>(amap, v.wmap, p, err, s);
  }
}

// half_out: the output is a convolution operand (fp16); else fp32.
cudaError_t voc_act(const float* in, void* out, int n, int rows, int cp, const float* prm,
                    int half_out, cudaStream_t s) {
  const int per_block = VA_R * VA_WARPS;
  const dim3 grid(cp / 32, (rows + per_block - 1) / per_block, n);
  if (half_out)
    return launch_pdl(voc_act_kernel<true>, grid, dim3(32 * VA_WARPS), 0, s, in, out, rows, cp, prm);
  return launch_pdl(voc_act_kernel<false>, grid, dim3(32 * VA_WARPS), 0, s, in, out, rows, cp, prm);
}

// The resblock activations (shared fixed filters): fp32 or fp16 input, fp16 output.
template <typename Tin>
cudaError_t voc_act2(const Tin* in, __half* out, int n, int rows, int cp, const float* prm,
                     cudaStream_t s) {
  const int per_block = 2 * VB_R * VA_WARPS;
  const dim3 grid(cp / 32, (rows + per_block - 1) / per_block, n);
  return launch_pdl(voc_act2_kernel<Tin>, grid, dim3(32 * VA_WARPS), 0, s, in, out, rows, cp, prm);
}

cudaError_t voc_linear(const float* X, int ldx, const float* W, const float* b, float* Y, int ldy,
                       int M, int N, int K, cudaStream_t s) {
  return launch_pdl(voc_linear_kernel, dim3((N + VL_T - 1) / VL_T, (M + VL_T - 1) / VL_T),
                    dim3(256), 0, s, X, ldx, W, b, Y, ldy, M, N, K, M, 0);
}

int grid_for(size_t count) {
  const size_t g = (count + 255) / 256;
  const size_t cap = static_cast<size_t>(sm_count()) * 8;
  return static_cast<int>(g < 1 ? 1 : (g > cap ? cap : g));
}

}  // namespace

extern "C" {

size_t dvoc_conv_floats(const DvocConfig* cfg) {
  if (!cfg || voc_validate(*cfg) != DFM_OK) return 0;
  VocHandle h;
  h.c = *cfg;
  voc_tables(h);
  return h.conv_floats;
}

size_t dvoc_bias_floats(const DvocConfig* cfg) {
  if (!cfg || voc_validate(*cfg) != DFM_OK) return 0;
  VocHandle h;
  h.c = *cfg;
  voc_tables(h);
  return h.bias_floats;
}

size_t dvoc_act_floats(const DvocConfig* cfg) {
  if (!cfg || voc_validate(*cfg) != DFM_OK) return 0;
  VocHandle h;
  h.c = *cfg;
  voc_tables(h);
  return h.act_floats;
}

int32_t dvoc_hop(const DvocConfig* cfg) {
  if (!cfg || voc_validate(*cfg) != DFM_OK) return 0;
  int32_t hop = 1;
  for (int i = 0; i < cfg->num_stages; ++i) hop *= cfg->upsample_rates[i];
  return hop;
}

int32_t dvoc_stream_left_context(const DvocConfig* cfg) {
  if (!cfg || voc_validate(*cfg) != DFM_OK) return -1;
  const DvocConfig& c = *cfg;
  // exact sum of fractions of a frame: accumulate in units of 1/hop
  long long hop = 1;
  for (int i = 0; i < c.num_stages; ++i) hop *= c.upsample_rates[i];
  const long long act = (11 + 11 + 1) / 2;  // one alias-free activation: ceil(22 / 2)
  long long num = static_cast<long long>(c.lookahead) * hop;  // conv_pre's padding
  long long scale = hop;                                     // current scale in 1/hop units
  for (int i = 0; i < c.num_stages; ++i) {
    num += scale;  // the causal transposed conv
    scale /= c.upsample_rates[i];
    long long stage = 0;
    for (int j = 0; j < c.num_kernels; ++j) {
      const long long k = c.resblock_kernel_sizes[j];
      long long ctx = 0;
      if (c.resblock_type == 1) {
        for (int l = 0; l < 3; ++l) ctx += act + c.resblock_dilations[j][l] * (k - 1) + act + (k - 1);
      } else {
        for (int l = 0; l < 2; ++l) ctx += act + c.resblock_dilations[j][l] * (k - 1);
      }
      stage = ctx > stage ? ctx : stage;
    }
    num += scale * stage;
  }
  num += scale * (act + 6);  // activation_post, conv_post (7 causal taps)
  return static_cast<int32_t>((num + hop - 1) / hop);
}

int dvoc_destroy(void* handle) {
  VocHandle* h = static_cast<VocHandle*>(handle);
  if (!h) return DFM_ERR_INVALID_ARG;
  delete h;
  return DFM_OK;
}

int dvoc_create(const DvocConfig* cfg, const DvocWeights* w, void** out) {
  if (!cfg || !w || !out) return DFM_ERR_INVALID_ARG;
  *out = nullptr;
  int rc = voc_validate(*cfg);
  if (rc != DFM_OK) return rc;
  const void* req[] = {w->post_w, w->post_b, w->mi_in_w, w->mi_in_b, w->lstm_w_ih, w->lstm_w_hh,
                       w->lstm_b_ih, w->lstm_b_hh, w->mi_out_w, w->mi_out_b, w->conv_w, w->conv_b,
                       w->act, w->post_conv_w};
  for (const void* p : req)
    if (!p) return DFM_ERR_INVALID_ARG;
  // TMA reads the weights and the kernels read biases and activation
  // parameters as 16-byte vectors
  if ((reinterpret_cast<uintptr_t>(w->conv_w) & 15) != 0 ||
      (reinterpret_cast<uintptr_t>(w->conv_b) & 15) != 0 ||
      (reinterpret_cast<uintptr_t>(w->act) & 15) != 0 ||
      (reinterpret_cast<uintptr_t>(w->lstm_w_hh) & 15) != 0)
    return DFM_ERR_INVALID_ARG;
  if (!encode_fn()) return DFM_ERR_CUDA;
  VocHandle* h = new (std::nothrow) VocHandle();
  if (!h) return DFM_ERR_CUDA;
  h->c = *cfg;
  h->w = *w;
  if (cudaGetDevice(&h->device) != cudaSuccess) {
    delete h;
    return DFM_ERR_CUDA;
  }
  voc_tables(*h);
  voc_layout(*h);
  for (VocConv& v : h->convs) {
    const int bn = voc_halo(v) ? voc_halo_bn(v.N) : voc_bn(v.N);
    if (!voc_map_w(&v.wmap, static_cast<const __half*>(w->conv_w) + v.w_off, v.N, v.taps * v.cin_p, bn)) {
      delete h;
      return DFM_ERR_CUDA;
    }
  }
  *out = h;
  return DFM_OK;
}

size_t dvoc_workspace_size(void* handle) {
  return handle ? static_cast<VocHandle*>(handle)->total : 0;
}

int dvoc_read_error(void* handle, void* workspace, void* stream, uint32_t* err_word) {
  VocHandle* h = static_cast<VocHandle*>(handle);
  if (!h || !workspace || !err_word) return DFM_ERR_INVALID_ARG;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint32_t* dev = reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(workspace) + h->o_err);
  if (cudaMemcpyAsync(err_word, dev, 4, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess)
    return DFM_ERR_CUDA;
  if (*err_word && cudaMemsetAsync(dev, 0, 4, s) != cudaSuccess) return DFM_ERR_CUDA;
  return DFM_OK;
}

// One call (dvoc_decode), or, with only >= 0, only the decoder convolution of
// that index with the call's arguments (dvoc_conv_launch).
static int voc_run(void* handle, const DvocBatch* b, void* workspace, size_t workspace_bytes,
                   void* stream, int only) {
  VocHandle* h = static_cast<VocHandle*>(handle);
  const bool all = only < 0;
  if (!h || !b || !workspace) return DFM_ERR_INVALID_ARG;
  const DvocConfig& c = h->c;
  const int n = b->n, F = b->frames, W = b->window;
  if (n < 1 || n > c.max_batch || F < 0 || W < 0) return DFM_ERR_INVALID_ARG;
  const bool streaming = W > 0;
  const int T = streaming ? W : F;
  if (T < 1 || T > c.max_frames) return DFM_ERR_INVALID_ARG;
  if (streaming && F >= W) return DFM_ERR_INVALID_ARG;
  if (streaming && (!b->windows || !b->valid)) return DFM_ERR_INVALID_ARG;
  if (F > 0 && (!b->latents || !b->lstm_h || !b->lstm_c)) return DFM_ERR_INVALID_ARG;
  if (!b->audio) return DFM_ERR_INVALID_ARG;
  if (workspace_bytes < h->total || (reinterpret_cast<uintptr_t>(workspace) & 255))
    return workspace_bytes < h->total ? DFM_ERR_WORKSPACE : DFM_ERR_INVALID_ARG;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev != h->device) return DFM_ERR_INVALID_ARG;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  auto P = [&](size_t off) { return reinterpret_cast<float*>(ws + off); };
  uint32_t* err = reinterpret_cast<uint32_t*>(ws + h->o_err);
  const VocRows r = voc_rows(*h, T);
  const int c0p = vpad(c.initial_channels);

  // tensor maps of this call's shape (kept while the shape and workspace repeat)
  if (h->plan_ws != workspace || h->plan_n != n || h->plan_t != T) {
    bool ok = voc_map_act(&h->m_din, P(h->o_din), n, r.cpre, h->Lp);
    for (int i = 0; ok && i < h->ns; ++i) {
      const int cin_p = i ? vpad(h->ch[i - 1]) : c0p, rows_in = i ? r.cap[i - 1] : r.cpre;
      ok = voc_map_act(&h->m_xin[i], P(h->o_x16), n, rows_in, cin_p) &&
           voc_map_act(&h->m_xin_h[i], P(h->o_x16), n, rows_in, cin_p, VH_BOX) &&
           voc_map_act(&h->m_act[i], P(h->o_a), n, r.cap[i], vpad(h->ch[i])) &&
           voc_map_act(&h->m_act_h[i], P(h->o_a), n, r.cap[i], vpad(h->ch[i]), VH_BOX) &&
           voc_map_f32(&h->m_u[i], P(h->o_u), n, r.cap[i], vpad(h->ch[i])) &&
           voc_map_f32(&h->m_h[i], P(h->o_h), n, r.cap[i], vpad(h->ch[i]));
    }
    if (!ok) {
      h->plan_ws = nullptr;
      return DFM_ERR_CUDA;
    }
    h->plan_ws = workspace;
    h->plan_n = n;
    h->plan_t = T;
  }

#define VCK(x)                          \
  do {                                  \
    if ((x) != cudaSuccess) return DFM_ERR_CUDA; \
  } while (0)

  const int L = h->L, Hm = h->Hm, M = n * F;
  // ---- front: post_proj, Linear(L, 4L), LSTM, Linear(4L, L)
  if (all && F > 0) {
    VCK(voc_linear(b->latents, L, h->w.post_w, h->w.post_b, P(h->o_p), L, M, L, L, s));
    VCK(voc_linear(P(h->o_p), L, h->w.mi_in_w, h->w.mi_in_b, P(h->o_s), Hm, M, Hm, L, s));
    const float* in = P(h->o_s);
    const size_t gsz = static_cast<size_t>(4) * Hm * Hm, state = static_cast<size_t>(n) * Hm;
    for (int l = 0; l < c.mi_layers; ++l) {
      float* y = P(l & 1 ? h->o_y1 : h->o_y0);
      VCK(voc_linear(in, Hm, h->w.lstm_w_ih + l * gsz, h->w.lstm_b_ih + static_cast<size_t>(l) * 4 * Hm,
                     P(h->o_gx), 4 * Hm, M, 4 * Hm, Hm, s));
      const int smem = Hm * (33 + 4 * VS_J) * 4;
      static std::atomic<uint64_t> attr_done{0};
      VCK(smem_attr_once(attr_done, voc_lstm_step_kernel, kVocLstmSmem));
      for (int f = 0; f < F; ++f) {
        const float* hp = f == 0 ? b->lstm_h + l * state : P(f & 1 ? h->o_h0 : h->o_h1);
        float* hn = P(f & 1 ? h->o_h1 : h->o_h0);
        VCK(launch_pdl(voc_lstm_step_kernel, dim3(Hm / VS_J, (n + 31) / 32), dim3(32 * VS_J), smem,
                       s, static_cast<const float*>(P(h->o_gx)), F, f,
                       static_cast<const float*>(h->w.lstm_w_hh + l * gsz),
                       static_cast<const float*>(h->w.lstm_b_hh + static_cast<size_t>(l) * 4 * Hm),
                       hp, hn, b->lstm_c + l * state, y,
                       l == c.mi_layers - 1 ? static_cast<const float*>(P(h->o_s)) : nullptr, n,
                       Hm));
      }
      VCK(launch_pdl(voc_copy_kernel, dim3(grid_for(state)), dim3(256), 0, s,
                     static_cast<const float*>(P((F - 1) & 1 ? h->o_h1 : h->o_h0)),
                     b->lstm_h + l * state, state));
      in = y;
    }
    VCK(voc_linear(in, Hm, h->w.mi_out_w, h->w.mi_out_b, P(h->o_z), L, M, L, Hm, s));
  }
  // ---- decoder input
  const size_t din = static_cast<size_t>(n) * r.cpre * h->Lp;
  if (all)
    VCK(launch_pdl(voc_pack_kernel, dim3(grid_for(din)), dim3(256), 0, s,
                 static_cast<const float*>(P(h->o_z)), static_cast<const float*>(b->windows),
                 b->valid, b->lengths, reinterpret_cast<__half*>(P(h->o_din)),
                 streaming ? P(h->o_din32) : nullptr, n, F, W, L, h->Lp, r.cpre));
  if (all && streaming && F > 0)
    VCK(launch_pdl(voc_window_store_kernel, dim3(grid_for(static_cast<size_t>(n) * W * L)), dim3(256),
                   0, s, static_cast<const float*>(P(h->o_din32)), b->windows, n, W, L, h->Lp, r.cpre));
  // ---- decoder
  size_t li = 0, ai = 0;
  auto pick = [&](size_t i) { return all || static_cast<int>(i) == only; };
  __half* X16 = reinterpret_cast<__half*>(P(h->o_x16));  // fp16 copy of each stage's output
  const VocConv& pre = h->convs[li];
  if (pick(li++))
    VCK(voc_conv(*h, pre, h->m_din, n, r.cpre, P(h->o_x), static_cast<long long>(r.cpre) * c0p,
               r.cpre, nullptr, 0, 1.0f, err, s, nullptr, nullptr, X16));
  for (int i = 0; i < h->ns; ++i) {
    const int cp = vpad(h->ch[i]), rows = r.cap[i], rows_in = i ? r.cap[i - 1] : r.cpre;
    const long long ob = static_cast<long long>(rows) * cp;
    float* X = P(h->o_x);
    float* U = P(h->o_u);
    float* H = P(h->o_h);
    __half* A = reinterpret_cast<__half*>(P(h->o_a));     // activation outputs (conv operands)
    __half* C1 = reinterpret_cast<__half*>(P(h->o_c1));   // conv1 outputs (read only by act2)
    if (pick(li))
      VCK(voc_conv(*h, h->convs[li], h->m_xin[i], n, rows_in, U, ob, rows, nullptr, 0, 1.0f, err, s,
                   &h->m_xin_h[i]));
    ++li;
    for (int j = 0; j < h->nk; ++j) {
      const int nl = c.resblock_type == 1 ? 3 : 2;
      for (int l = 0; l < nl; ++l) {
        const float* src = l == 0 ? U : H;
        const bool last = l == nl - 1;
        float* dst = last ? X : H;
        const int acc = last && j > 0;
        const float dv = last && j == h->nk - 1 ? static_cast<float>(h->nk) : 1.0f;
        if (all) VCK(voc_act2(src, A, n, rows, cp, h->w.act + h->act_off[ai], s));
        ++ai;
        if (c.resblock_type == 1) {
          if (pick(li))
            VCK(voc_conv(*h, h->convs[li], h->m_act[i], n, rows, nullptr, ob, rows, nullptr, 0, 1.0f,
                         err, s, &h->m_act_h[i], nullptr, C1));
          ++li;
          if (all) VCK(voc_act2(static_cast<const __half*>(C1), A, n, rows, cp, h->w.act + h->act_off[ai], s));
          ++ai;
        }
        // the stage's final sum also feeds the next stage's transposed conv (fp16)
        __half* d16 = last && j == h->nk - 1 && i + 1 < h->ns ? X16 : nullptr;
        if (pick(li))
          VCK(voc_conv(*h, h->convs[li], h->m_act[i], n, rows, dst, ob, rows, src, acc, dv, err, s,
                       &h->m_act_h[i], l == 0 ? &h->m_u[i] : &h->m_h[i], d16));
        ++li;
      }
    }
  }
  // ---- activation_post, conv_post, tanh
  if (!all) return DFM_OK;
  const int last = h->ns - 1, cpl = vpad(h->ch[last]), rows = r.cap[last];
  VCK(voc_act(P(h->o_x), P(h->o_a), n, rows, cpl, h->w.act + h->act_off[ai++], 0, s));
  const long long samples = r.t[last];
  VCK(launch_pdl(voc_post_kernel, dim3(static_cast<int>((samples + VP_T - 1) / VP_T), n), dim3(VP_T), 0,
                 s, static_cast<const float*>(P(h->o_a)), b->audio, rows, cpl,
                 static_cast<int>(samples), samples, h->w.post_conv_w, h->w.post_conv_b,
                 c.use_tanh));
#undef VCK
  return DFM_OK;
}

int dvoc_decode(void* handle, const DvocBatch* b, void* workspace, size_t workspace_bytes,
                void* stream) {
  return voc_run(handle, b, workspace, workspace_bytes, stream, -1);
}

int32_t dvoc_num_convs(void* handle) {
  return handle ? static_cast<int32_t>(static_cast<VocHandle*>(handle)->convs.size()) : 0;
}

int dvoc_conv_launch(void* handle, const DvocBatch* b, void* workspace, size_t workspace_bytes,
                     int32_t index, void* stream) {
  VocHandle* h = static_cast<VocHandle*>(handle);
  if (!h || index < 0 || index >= static_cast<int32_t>(h->convs.size())) return DFM_ERR_INVALID_ARG;
  return voc_run(handle, b, workspace, workspace_bytes, stream, index);
}

}  // extern "C"
