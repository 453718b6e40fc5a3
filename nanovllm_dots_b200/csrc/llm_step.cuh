// Row kernels of the LLM backbone's decode step (``QwenDecoderLayer``,
// ``nanovllm_dots/models/dots/model_llm.py:113-147``): RMSNorm with the
// residual add of the previous sublayer's split-K partials, NeoX rotary of q
// and k, and SiLU-and-mul.  The GEMMs are the CTA-pair tcgen05 kernels of
// gemm.cuh and the attention the paged decode kernels of llm_attn.cuh.
#pragma once

#include "common.cuh"

namespace dfm {

constexpr int LR_ROWS_PER_BLOCK = 2;
constexpr int LR_THREADS = 128 * LR_ROWS_PER_BLOCK;

// One row per 128 threads (HD / 512 float4 column groups per thread):
//   NSUB == 0: x = float(in[r])                 (the step's input embeddings)
//   NSUB >  0: x = h[r] + sum_p sub[p][r]       (residual + the sublayer's partials)
//   h[r] = x;  out[r] = bf16(x * rsqrt(mean(x^2) + eps) * w)
// (``layers/layernorm.py:17-26``; the residual stream h is kept in fp32.)
template <int HD, int NSUB>
__global__ void __launch_bounds__(LR_THREADS)
    llm_rms_kernel(float* __restrict__ h, const __nv_bfloat16* __restrict__ in,
                   const float* __restrict__ sub, size_t sub_plane, int M,
                   const float* __restrict__ w, float eps, __nv_bfloat16* __restrict__ out) {
  static_assert(HD % 512 == 0, "width: a multiple of 512");
  constexpr int V = HD / 512;   // float4 groups per thread
  __shared__ float red[LR_ROWS_PER_BLOCK][4];
  const int rb = threadIdx.x >> 7, t = threadIdx.x & 127;
  const int wi = t >> 5, lane = threadIdx.x & 31;
  const int r = blockIdx.x * LR_ROWS_PER_BLOCK + rb;
  pdl_trigger();
  pdl_wait();
  const bool valid = r < M;
  float4 x[V], wv[V];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < V; ++j) {
    const int col = j * 512 + t * 4;
    x[j] = make_float4(0.f, 0.f, 0.f, 0.f);
    wv[j] = x[j];
    if (!valid) continue;
    wv[j] = *reinterpret_cast<const float4*>(w + col);
    const size_t off = static_cast<size_t>(r) * HD + col;
    if constexpr (NSUB == 0) {
      const uint2 u = *reinterpret_cast<const uint2*>(in + off);
      const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
      const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
      x[j] = make_float4(a.x, a.y, b.x, b.y);
    } else {
      x[j] = *reinterpret_cast<const float4*>(h + off);
#pragma unroll
      for (int p = 0; p < NSUB; ++p) {
        const float4 s = *reinterpret_cast<const float4*>(sub + p * sub_plane + off);
        x[j].x += s.x; x[j].y += s.y; x[j].z += s.z; x[j].w += s.w;
      }
    }
    *reinterpret_cast<float4*>(h + off) = x[j];
    ss += x[j].x * x[j].x + x[j].y * x[j].y + x[j].z * x[j].z + x[j].w * x[j].w;
  }
  ss = warp_sum(ss);
  if (lane == 0) red[rb][wi] = ss;
  __syncthreads();
  if (!valid) return;
  const float ms = ((red[rb][0] + red[rb][1]) + (red[rb][2] + red[rb][3])) * (1.0f / HD);
  const float rs = rsqrtf(ms + eps);
#pragma unroll
  for (int j = 0; j < V; ++j) {
    const int col = j * 512 + t * 4;
    *reinterpret_cast<uint2*>(out + static_cast<size_t>(r) * HD + col) =
        make_uint2(pack_bf16(x[j].x * rs * wv[j].x, x[j].y * rs * wv[j].y),
                   pack_bf16(x[j].z * rs * wv[j].z, x[j].w * rs * wv[j].w));
  }
}

// qkv = bias + sum of the QKV projection's nsplit fp32 split-K planes
// [p][n][(H + 2 KVH) D] -> q [n][H][D], k [n][KVH][D] rotated at positions[i]
// (NeoX halves: y1 = x1 cos - x2 sin, y2 = x2 cos + x1 sin, angle
// pos * inv_freq[d], ``layers/rotary_embedding.py:6-47``) and v [n][KVH][D].
// One thread per (row, head, rotary pair).
__global__ void __launch_bounds__(256)
    llm_rope_kernel(const float* __restrict__ qkv, int nsplit, size_t plane,
                    const float* __restrict__ bias, const int* __restrict__ positions,
                    const float* __restrict__ inv_freq, int n, int H, int KVH, int D,
                    __nv_bfloat16* __restrict__ q, __nv_bfloat16* __restrict__ k,
                    __nv_bfloat16* __restrict__ v) {
  const int half = D / 2, heads = H + 2 * KVH;
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  pdl_trigger();
  pdl_wait();
  if (idx >= n * heads * half) return;
  const int i = idx / (heads * half);
  const int rem = idx - i * heads * half;
  const int hd = rem / half, d = rem - hd * half;
  const int c1 = hd * D + d, c2 = c1 + half;
  const float* src = qkv + static_cast<size_t>(i) * heads * D;
  float x1 = bias[c1], x2 = bias[c2];
  for (int p = 0; p < nsplit; ++p) {
    x1 += src[p * plane + c1];
    x2 += src[p * plane + c2];
  }
  if (hd >= H + KVH) {   // v: no rotation
    __nv_bfloat16* dst = v + (static_cast<size_t>(i) * KVH + (hd - H - KVH)) * D;
    dst[d] = __float2bfloat16(x1);
    dst[d + half] = __float2bfloat16(x2);
    return;
  }
  float s, c;
  sincosf(static_cast<float>(positions[i]) * inv_freq[d], &s, &c);
  __nv_bfloat16* dst = hd < H ? q + (static_cast<size_t>(i) * H + hd) * D
                              : k + (static_cast<size_t>(i) * KVH + (hd - H)) * D;
  dst[d] = __float2bfloat16(x1 * c - x2 * s);
  dst[d + half] = __float2bfloat16(x2 * c + x1 * s);
}

// gu [n][2 I] = [gate | up] -> act [n][I] = silu(gate) * up (``layers/activation.py:5-14``);
// one thread per 8 outputs.
__global__ void __launch_bounds__(256)
    llm_silu_mul_kernel(const __nv_bfloat16* __restrict__ gu, int n, int I,
                        __nv_bfloat16* __restrict__ act) {
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  pdl_trigger();
  pdl_wait();
  const int per = I / 8;
  if (idx >= n * per) return;
  const int i = idx / per, c = (idx - i * per) * 8;
  const uint4 g4 = *reinterpret_cast<const uint4*>(gu + static_cast<size_t>(i) * 2 * I + c);
  const uint4 u4 = *reinterpret_cast<const uint4*>(gu + static_cast<size_t>(i) * 2 * I + I + c);
  const __nv_bfloat162* g2 = reinterpret_cast<const __nv_bfloat162*>(&g4);
  const __nv_bfloat162* u2 = reinterpret_cast<const __nv_bfloat162*>(&u4);
  uint32_t o[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 g = __bfloat1622float2(g2[e]), u = __bfloat1622float2(u2[e]);
    o[e] = pack_bf16(silu(g.x) * u.x, silu(g.y) * u.y);
  }
  *reinterpret_cast<uint4*>(act + static_cast<size_t>(i) * I + c) = make_uint4(o[0], o[1], o[2], o[3]);
}

}  // namespace dfm
