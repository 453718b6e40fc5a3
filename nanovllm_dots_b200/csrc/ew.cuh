// Row-wise kernels of the FM head: adaLN LayerNorm + modulate, the timestep /
// duration embedders, and solver-state initialisation.
#pragma once

#include "common.cuh"

namespace dfm {

enum LnMode : int { LN_ADALN = 0, LN_AFFINE = 1, LN_NONE = 2 };
constexpr int LN_ROWS_PER_BLOCK = 2;
constexpr int LN_THREADS = 128 * LN_ROWS_PER_BLOCK;

// Residual update + adaLN LayerNorm + modulate, one row per 128 threads:
//   x = h[in_map(r)] (+ gate[req] * sub[in_map(r)], written back to h; sub is
//   the sum of NSUB split-K partial planes sub[. + p * sub_plane], p < NSUB)
//   out[r] = LN(x) * (1 + scale[req]) + shift[req],   req = r / rows_per_req
//   (bf16; or, with out8, e4m3 values out8[r] with out[r] = out8[r] * out_scale[r])
// LayerNorm without affine over H = 1024 (``native/dit.py:70-71,19-20``).  The
// residual add of the previous sublayer (``dit.py:102-107``: x + gate * f(x))
// is applied here, on coalesced rows, instead of in that sublayer's GEMM
// epilogue.  h is the fp32 residual stream, out the bf16 GEMM operand.
// MODE selects the row transform after the residual add:
//   LN_ADALN   LN(x) * (1 + scale) + shift  (the DiT's modulate)
//   LN_AFFINE  LN(x) * scale + shift        (nn.LayerNorm with affine, the patch
//              encoder's attn_norm / ffn_norm, ``patch_encoder.py:34-38``; mod_ld = 0)
//   LN_NONE    x                            (the residual stream itself)
// Only LN_ADALN reads a gate; the others add sub with a gate of ones (the
// encoder's plain residual, ``patch_encoder.py:82-86``).
template <int NSUB, int MODE>
__global__ void __launch_bounds__(LN_THREADS, NSUB <= 2 ? 8 : 5)
    ln_mod_kernel(float* __restrict__ h, const float* __restrict__ sub, size_t sub_plane,
                  const float* __restrict__ gate, int M, RowMap in_map,
                  const float* __restrict__ shift, const float* __restrict__ scale, int mod_ld,
                  int rows_per_req, __nv_bfloat16* __restrict__ out, float eps,
                  uint8_t* __restrict__ out8, float* __restrict__ out_scale) {
  // 128 threads (4 warps) per row, two rows per block: thread t of a row owns
  // the 16-byte column groups t and t + 128 (each warp's accesses are 512
  // contiguous bytes).  The shift / scale vectors are read after the row
  // statistics, which keeps the kernel at 32 registers: 8 blocks (16 rows)
  // per SM, so config 2's 1088 blocks run in one wave (loaded with the row,
  // 54 registers allowed 4 blocks per SM: 1.84 waves, measured slower).  One
  // warp per row left the kernel latency-bound (few warps per SM, each
  // waiting on its own chain of loads).
  constexpr int H = 1024;
  __shared__ float red[LN_ROWS_PER_BLOCK][3][4];   // [row][sum | centred squares | absmax][warp]
  const int rb = threadIdx.x >> 7;
  const int t = threadIdx.x & 127;
  const int w = t >> 5, lane = threadIdx.x & 31;
  const int r = blockIdx.x * LN_ROWS_PER_BLOCK + rb;
  pdl_trigger();
  pdl_wait();
  const bool valid = r < M;
  const size_t hrow = valid ? static_cast<size_t>(in_map(r)) * H : 0;
  const size_t req = valid ? static_cast<size_t>(r / rows_per_req) : 0;
  float* hr = h + hrow;
  float4 x[2], a_sh[2], b_sc[2];
  constexpr bool norm = MODE != LN_NONE;
  if (valid) {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int col = j * 512 + t * 4;
      x[j] = *reinterpret_cast<const float4*>(hr + col);
    }
    if (sub) {
      const float* sr = sub + hrow;
      const float* gr = gate + req * mod_ld;
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int col = j * 512 + t * 4;
        float4 a = *reinterpret_cast<const float4*>(sr + col);
#pragma unroll
        for (int p = 1; p < NSUB; ++p) {  // split-K: the other partial sums
          const float4 a2 = *reinterpret_cast<const float4*>(sr + p * sub_plane + col);
          a.x += a2.x; a.y += a2.y; a.z += a2.z; a.w += a2.w;
        }
        float4 g = make_float4(1.f, 1.f, 1.f, 1.f);
        if constexpr (MODE == LN_ADALN) g = *reinterpret_cast<const float4*>(gr + col);
        x[j].x += g.x * a.x;
        x[j].y += g.y * a.y;
        x[j].z += g.z * a.z;
        x[j].w += g.w * a.w;
        *reinterpret_cast<float4*>(hr + col) = x[j];
      }
    }
  } else {
    x[0] = x[1] = a_sh[0] = a_sh[1] = b_sc[0] = b_sc[1] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  if constexpr (!norm) {
    if (valid) {
      __nv_bfloat16* o = out + static_cast<size_t>(r) * H;
#pragma unroll
      for (int j = 0; j < 2; ++j)
        *reinterpret_cast<uint2*>(o + j * 512 + t * 4) =
            make_uint2(pack_bf16(x[j].x, x[j].y), pack_bf16(x[j].z, x[j].w));
    }
  } else {
    float s = (x[0].x + x[0].y) + (x[0].z + x[0].w) + (x[1].x + x[1].y) + (x[1].z + x[1].w);
    s = warp_sum(s);
    if (lane == 0) red[rb][0][w] = s;
    __syncthreads();
    const float mean = ((red[rb][0][0] + red[rb][0][1]) + (red[rb][0][2] + red[rb][0][3])) * (1.0f / H);
    float v = 0.f;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const float a = x[j].x - mean, b = x[j].y - mean, c = x[j].z - mean, d = x[j].w - mean;
      v += a * a + b * b + c * c + d * d;
    }
    v = warp_sum(v);
    if (lane == 0) red[rb][1][w] = v;
    __syncthreads();
    const float var = ((red[rb][1][0] + red[rb][1][1]) + (red[rb][1][2] + red[rb][1][3])) * (1.0f / H);
    const float rstd = rsqrtf(var + eps);
    constexpr float one = MODE == LN_ADALN ? 1.f : 0.f;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int col = j * 512 + t * 4;
      a_sh[j] = b_sc[j] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (valid) {
        a_sh[j] = *reinterpret_cast<const float4*>(shift + req * mod_ld + col);
        b_sc[j] = *reinterpret_cast<const float4*>(scale + req * mod_ld + col);
      }
    }
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      x[j].x = (x[j].x - mean) * rstd * (one + b_sc[j].x) + a_sh[j].x;
      x[j].y = (x[j].y - mean) * rstd * (one + b_sc[j].y) + a_sh[j].y;
      x[j].z = (x[j].z - mean) * rstd * (one + b_sc[j].z) + a_sh[j].z;
      x[j].w = (x[j].w - mean) * rstd * (one + b_sc[j].w) + a_sh[j].w;
    }
    if (out8) {
      // e4m3 row with one fp32 scale per row (row absmax / 448)
      float m = 0.f;
#pragma unroll
      for (int j = 0; j < 2; ++j)
        m = fmaxf(m, fmaxf(fmaxf(fabsf(x[j].x), fabsf(x[j].y)), fmaxf(fabsf(x[j].z), fabsf(x[j].w))));
      m = warp_max(m);
      if (lane == 0) red[rb][2][w] = m;
      __syncthreads();
      m = fmaxf(fmaxf(red[rb][2][0], red[rb][2][1]), fmaxf(red[rb][2][2], red[rb][2][3]));
      if (!valid) return;
      const float sc = m > 0.f ? m * (1.0f / 448.0f) : 1.0f;
      const float inv = 1.0f / sc;
      uint8_t* o8 = out8 + static_cast<size_t>(r) * H;
#pragma unroll
      for (int j = 0; j < 2; ++j)
        *reinterpret_cast<uint32_t*>(o8 + j * 512 + t * 4) =
            pack_e4m3x4(x[j].x * inv, x[j].y * inv, x[j].z * inv, x[j].w * inv);
      if (t == 0) out_scale[r] = sc;
      return;
    }
    if (!valid) return;
    __nv_bfloat16* o = out + static_cast<size_t>(r) * H;
#pragma unroll
    for (int j = 0; j < 2; ++j)
      *reinterpret_cast<uint2*>(o + j * 512 + t * 4) =
          make_uint2(pack_bf16(x[j].x, x[j].y), pack_bf16(x[j].z, x[j].w));
  }
}

constexpr int EMB_MAX_STEPS = 8;
struct TimeGrid {
  float t[EMB_MAX_STEPS];   // timesteps seen by the DiT
  float dt[EMB_MAX_STEPS];  // durations seen by the duration embedder
};

// Sinusoidal embedding component idx of 256: cos(t f_i) for idx < 128, sin for
// idx >= 128, f_i = exp(-ln(10000) * i / 128) (``native/dit.py:33-42``).
DFM_DEV float sinusoid(float t, int idx) {
  const int i = idx & 127;
  const float f = expf(-9.210340371976184f * static_cast<float>(i) / 128.0f);
  const float a = t * f;
  return idx < 128 ? cosf(a) : sinf(a);
}

// First embedder layer for both embedders and every step:
// out1[e][k][j] = silu(W1_e[j, :] . emb(x_{e,k}) + b1_e[j]); e = 0 time, 1 duration.
// The 256-d embeddings of the (at most 2 x 8) scalars are built once per block
// in shared memory; then one warp per (e, j) does the 256-wide dot product,
// 8 bf16 per lane.
__global__ void __launch_bounds__(256)
    embed1_kernel(const __nv_bfloat16* __restrict__ w_t, const float* __restrict__ b_t,
                  const __nv_bfloat16* __restrict__ w_d, const float* __restrict__ b_d,
                  TimeGrid grid, int nfe, int H, float* __restrict__ out1) {
  __shared__ float emb_s[2][EMB_MAX_STEPS][256];
  const int wid = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  pdl_trigger();
  pdl_wait();
  for (int idx = threadIdx.x; idx < 2 * nfe * 256; idx += blockDim.x) {
    const int e = idx / (nfe * 256), k = (idx >> 8) % nfe, d = idx & 255;
    emb_s[e][k][d] = sinusoid(e == 0 ? grid.t[k] : grid.dt[k], d);
  }
  __syncthreads();
  if (wid >= 2 * H) return;
  const int e = wid / H, j = wid - e * H;
  const __nv_bfloat16* w = (e == 0 ? w_t : w_d) + static_cast<size_t>(j) * 256 + lane * 8;
  const uint4 wv = *reinterpret_cast<const uint4*>(w);
  const __nv_bfloat16* wp = reinterpret_cast<const __nv_bfloat16*>(&wv);
  float wf[8];
#pragma unroll
  for (int q = 0; q < 8; ++q) wf[q] = __bfloat162float(wp[q]);
  const float bias = (e == 0 ? b_t : b_d)[j];
#pragma unroll 1
  for (int k = 0; k < nfe; ++k) {
    const float* x = &emb_s[e][k][lane * 8];
    float acc = 0.f;
#pragma unroll
    for (int q = 0; q < 8; ++q) acc += wf[q] * x[q];
    acc = warp_sum(acc);
    if (lane == 0) out1[(static_cast<size_t>(e) * nfe + k) * H + j] = silu(acc + bias);
  }
}

// Second embedder layer, the condition sum and the adaLN input:
// c_k[j] = (W2_t[j].out1[0][k] + b2_t[j]) + (W2_d[j].out1[1][k] + b2_d[j])
// csilu[(k*n + i), j] = bf16(silu(c_k[j] + g_cond[i][j]))    (``native/dit.py:137-143``;
// adaLN_modulation = SiLU -> Linear, ``dit.py:75-79``).  One warp per j; a
// block's 8 warps cover 8 consecutive j, whose c_k go through shared memory so
// the block writes each csilu row's 8 columns as one 16-byte store.
__global__ void __launch_bounds__(256)
    embed2_kernel(const __nv_bfloat16* __restrict__ w_t, const float* __restrict__ b_t,
                  const __nv_bfloat16* __restrict__ w_d, const float* __restrict__ b_d,
                  const float* __restrict__ out1, const __nv_bfloat16* __restrict__ g_cond, int n,
                  int nfe, int H, __nv_bfloat16* __restrict__ csilu) {
  __shared__ float ck_s[EMB_MAX_STEPS][8];
  const int warp = threadIdx.x >> 5;
  const int j = blockIdx.x * 8 + warp;
  const int lane = threadIdx.x & 31;
  pdl_trigger();
  pdl_wait();
  if (j < H) {
    float ck[EMB_MAX_STEPS];
#pragma unroll
    for (int k = 0; k < EMB_MAX_STEPS; ++k) ck[k] = 0.f;
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const __nv_bfloat16* w = (e == 0 ? w_t : w_d) + static_cast<size_t>(j) * H;
      float acc[EMB_MAX_STEPS];
#pragma unroll
      for (int k = 0; k < EMB_MAX_STEPS; ++k) acc[k] = 0.f;
#pragma unroll 1
      for (int c = lane * 8; c < H; c += 256) {
        const uint4 wv = *reinterpret_cast<const uint4*>(w + c);
        const __nv_bfloat16* wp = reinterpret_cast<const __nv_bfloat16*>(&wv);
#pragma unroll
        for (int k = 0; k < EMB_MAX_STEPS; ++k) {
          if (k >= nfe) break;
          const float4* x4 =
              reinterpret_cast<const float4*>(out1 + (static_cast<size_t>(e) * nfe + k) * H + c);
          const float4 xa = x4[0], xb = x4[1];
          acc[k] += __bfloat162float(wp[0]) * xa.x + __bfloat162float(wp[1]) * xa.y +
                    __bfloat162float(wp[2]) * xa.z + __bfloat162float(wp[3]) * xa.w +
                    __bfloat162float(wp[4]) * xb.x + __bfloat162float(wp[5]) * xb.y +
                    __bfloat162float(wp[6]) * xb.z + __bfloat162float(wp[7]) * xb.w;
        }
      }
      const float bias = (e == 0 ? b_t : b_d)[j];
#pragma unroll
      for (int k = 0; k < EMB_MAX_STEPS; ++k) {
        if (k >= nfe) break;
        ck[k] += warp_sum(acc[k]) + bias;
      }
    }
    if (lane == 0)
      for (int k = 0; k < nfe; ++k) ck_s[k][warp] = ck[k];
  }
  __syncthreads();
  // rows (k, i): 8 columns j0 .. j0 + 7 per thread
  const int j0 = blockIdx.x * 8;
  if (j0 + 8 > H) return;
  for (int idx = threadIdx.x; idx < nfe * n; idx += blockDim.x) {
    const int k = idx / n, i = idx - k * n;
    float g[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (g_cond) {
      const uint4 gv = *reinterpret_cast<const uint4*>(g_cond + static_cast<size_t>(i) * H + j0);
      const __nv_bfloat16* gp = reinterpret_cast<const __nv_bfloat16*>(&gv);
#pragma unroll
      for (int q = 0; q < 8; ++q) g[q] = __bfloat162float(gp[q]);
    }
    float v[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) v[q] = silu(ck_s[k][q] + g[q]);
    *reinterpret_cast<uint4*>(csilu + static_cast<size_t>(idx) * H + j0) =
        make_uint4(pack_bf16(v[0], v[1]), pack_bf16(v[2], v[3]), pack_bf16(v[4], v[5]),
                   pack_bf16(v[6], v[7]));
  }
}

// Rotary table: tab[pos * 32 + d] = (cos, sin)(pos * inv_freq[d]), the angles
// of ``layers.py:95-134`` for every cache position, computed once per workspace.
__global__ void rope_table_kernel(const float* __restrict__ inv_freq, int max_pos,
                                  float2* __restrict__ tab) {
  // tab[d][pos]: consecutive positions are adjacent, so the 32 rows of an
  // epilogue warp (consecutive positions of one or two requests) read one
  // frequency's (cos, sin) in one or two 256-byte segments.
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= max_pos * 32) return;
  const int d = idx / max_pos, pos = idx - d * max_pos;
  float sn, co;
  sincosf(static_cast<float>(pos) * inv_freq[d], &sn, &co);
  tab[idx] = make_float2(co, sn);
}

// The engine dispatch's per-tick inputs gathered from every request's own FM
// history buffer in one launch.  table[i] = {row0 pointer of request i's bf16
// history rows (row stride H), first graduating row, graduating count (<=
// stride), g_cond pointer or 0}; then
//   ext[i][j] = rows[first + j]   (j < count; zero rows up to stride)
//   act[i]    = rows[first + count]       (the active hidden row)
//   g[i]      = g_cond (or zeros)
// (``DotsBatchEngine._pack_fm_inputs``, ``engine.py:635-688``, reads the same
// rows of ``gen_state.fm_sequence``).  Block (i, r): one 2 KB row, 16 bytes
// per thread.
__global__ void __launch_bounds__(128)
    gather_rows_kernel(const long long* __restrict__ table, int H, int stride,
                       __nv_bfloat16* __restrict__ act, __nv_bfloat16* __restrict__ ext,
                       __nv_bfloat16* __restrict__ g) {
  const int i = blockIdx.x, r = blockIdx.y;
  const long long* t = table + 4 * static_cast<size_t>(i);
  const int count = static_cast<int>(t[2]);
  const __nv_bfloat16* src = nullptr;
  __nv_bfloat16* dst;
  if (r < stride) {
    dst = ext + (static_cast<size_t>(i) * stride + r) * H;
    if (r < count) src = reinterpret_cast<const __nv_bfloat16*>(t[0]) + (t[1] + r) * H;
  } else if (r == stride) {
    dst = act + static_cast<size_t>(i) * H;
    src = reinterpret_cast<const __nv_bfloat16*>(t[0]) + (t[1] + count) * H;
  } else {
    dst = g + static_cast<size_t>(i) * H;
    src = reinterpret_cast<const __nv_bfloat16*>(t[3]);
  }
  for (int c = threadIdx.x * 8; c < H; c += blockDim.x * 8) {
    const uint4 v = src ? *reinterpret_cast<const uint4*>(src + c) : make_uint4(0, 0, 0, 0);
    *reinterpret_cast<uint4*>(dst + c) = v;
  }
}

// z = float(noise), zb = noise (the solver state and its bf16 GEMM copy).
__global__ void init_z_kernel(const __nv_bfloat16* __restrict__ noise, int count,
                              float* __restrict__ z, __nv_bfloat16* __restrict__ zb) {
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  pdl_trigger();
  pdl_wait();
  if (idx >= count) return;
  const __nv_bfloat16 v = noise[idx];
  z[idx] = __bfloat162float(v);
  zb[idx] = v;
}

}  // namespace dfm
