// Row kernels of the LLM backbone's decode step (``QwenDecoderLayer``,
// ``nanovllm_dots/models/dots/model_llm.py:113-147``): RMSNorm with the
// residual add of the previous sublayer's split-K partials, NeoX rotary of q
// and k, and SiLU-and-mul.  The GEMMs are the CTA-pair tcgen05 kernels of
// gemm.cuh and the attention the paged decode kernels of llm_attn.cuh.
#pragma once

#include "common.cuh"

namespace dfm {

// One row per block, one float4 column group per thread (HD / 4 threads), so
// every load of a row (residual, the NSUB partial planes, the weight) is in
// flight at once:
//   NSUB == 0: x = float(in[r])                 (the step's input embeddings)
//   NSUB >  0: x = h[r] + sum_p sub[p][r]       (residual + the sublayer's partials)
//   h[r] = x;  out[r] = bf16(x * rsqrt(mean(x^2) + eps) * w)
// (``layers/layernorm.py:17-26``; the residual stream h is kept in fp32.)
// The weight does not depend on the previous kernel and is read before the
// dependency wait.
template <int HD, int NSUB>
__global__ void __launch_bounds__(HD / 4)
    llm_rms_kernel(float* __restrict__ h, const __nv_bfloat16* __restrict__ in,
                   const float* __restrict__ sub, size_t sub_plane, int M,
                   const float* __restrict__ w, float eps, __nv_bfloat16* __restrict__ out) {
  static_assert(HD % 128 == 0 && HD / 4 <= 1024, "width");
  constexpr int NW = HD / 128;   // warps per row
  __shared__ float red[NW];
  const int r = blockIdx.x, t = threadIdx.x, lane = t & 31, col = t * 4;
  const float4 wv = *reinterpret_cast<const float4*>(w + col);
  pdl_trigger();
  pdl_wait();
  if (r >= M) return;
  const size_t off = static_cast<size_t>(r) * HD + col;
  float4 x;
  if constexpr (NSUB == 0) {
    const uint2 u = *reinterpret_cast<const uint2*>(in + off);
    const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
    const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
    x = make_float4(a.x, a.y, b.x, b.y);
  } else {
    float4 sp[NSUB];
    x = *reinterpret_cast<const float4*>(h + off);
#pragma unroll
    for (int p = 0; p < NSUB; ++p) sp[p] = *reinterpret_cast<const float4*>(sub + p * sub_plane + off);
#pragma unroll
    for (int p = 0; p < NSUB; ++p) {
      x.x += sp[p].x; x.y += sp[p].y; x.z += sp[p].z; x.w += sp[p].w;
    }
  }
  *reinterpret_cast<float4*>(h + off) = x;
  float ss = x.x * x.x + x.y * x.y + x.z * x.z + x.w * x.w;
  ss = warp_sum(ss);
  if (lane == 0) red[t >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < NW; ++i) tot += red[i];
  const float rs = rsqrtf(tot * (1.0f / HD) + eps);
  *reinterpret_cast<uint2*>(out + off) =
      make_uint2(pack_bf16(x.x * rs * wv.x, x.y * rs * wv.y), pack_bf16(x.z * rs * wv.z, x.w * rs * wv.w));
}

// qkv = bias + sum of the QKV projection's nsplit fp32 split-K planes
// [p][n][(H + 2 KVH) D] -> q [n][H][D] and k rotated at positions[i] (NeoX
// halves: y1 = x1 cos - x2 sin, y2 = x2 cos + x1 sin, angle pos * inv_freq[d],
// ``layers/rotary_embedding.py:6-47``), v unrotated; k and v go straight into
// the paged caches at the token's slot (``store_kvcache``,
// ``layers/attention.py:10-47``: slot < 0 skips the token, a slot past the
// cache is reported and skipped).  One thread per (row, head, rotary pair);
// the plane count is a compile-time constant so every plane load is issued
// before the first add.
template <int NSPLIT>
__global__ void __launch_bounds__(256)
    llm_rope_kernel(const float* __restrict__ qkv, size_t plane,
                    const float* __restrict__ bias, const int* __restrict__ positions,
                    const float* __restrict__ inv_freq, int n, int H, int KVH, int D,
                    __nv_bfloat16* __restrict__ q, __nv_bfloat16* __restrict__ k_cache,
                    __nv_bfloat16* __restrict__ v_cache, const int* __restrict__ slot_mapping,
                    long long num_slots, uint32_t* err) {
  const int half = D / 2, heads = H + 2 * KVH;
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  pdl_trigger();
  pdl_wait();
  if (idx >= n * heads * half) return;
  const int i = idx / (heads * half);
  const int rem = idx - i * heads * half;
  const int hd = rem / half, d = rem - hd * half;
  __nv_bfloat16* dst;
  if (hd < H) {
    dst = q + (static_cast<size_t>(i) * H + hd) * D;
  } else {
    const int slot = slot_mapping[i];
    if (slot < 0) return;
    if (slot >= num_slots) {
      if (d == 0) atomicOr(err, DFM_DEV_ERR_PAGE);
      return;
    }
    const int kvh = hd < H + KVH ? hd - H : hd - H - KVH;
    dst = (hd < H + KVH ? k_cache : v_cache) + (static_cast<size_t>(slot) * KVH + kvh) * D;
  }
  const int c1 = hd * D + d, c2 = c1 + half;
  const float* src = qkv + static_cast<size_t>(i) * heads * D;
  float x1 = bias[c1], x2 = bias[c2];
  float a1[NSPLIT], a2[NSPLIT];
#pragma unroll
  for (int p = 0; p < NSPLIT; ++p) {
    a1[p] = src[p * plane + c1];
    a2[p] = src[p * plane + c2];
  }
#pragma unroll
  for (int p = 0; p < NSPLIT; ++p) {
    x1 += a1[p];
    x2 += a2[p];
  }
  if (hd >= H + KVH) {   // v: no rotation
    dst[d] = __float2bfloat16(x1);
    dst[d + half] = __float2bfloat16(x2);
    return;
  }
  float s, c;
  sincosf(static_cast<float>(positions[i]) * inv_freq[d], &s, &c);
  dst[d] = __float2bfloat16(x1 * c - x2 * s);
  dst[d + half] = __float2bfloat16(x2 * c + x1 * s);
}

}  // namespace dfm

namespace dfm {

// ---------------------------------------------------------------- decode GEMM
// The decode step's projections have M = n tokens (64) and stream their
// weights: as an A operand of M = n they would fill a fraction of each MMA and
// of each CTA pair.  Here the operands are swapped: the weight W [N_out][K]
// (K-major, the nn.Linear layout) is the MMA's A operand, 128 output features
// per tile, and the activations X [n][K] its B operand, 64 tokens per tile, so
//   out_plane[s][t][j] = sum_{k in K-split s} W[j][k] X[t][k]
// with every weight byte read once.  Work units (feature tile, token block,
// K split) run on a persistent grid, feature tiles fastest so the CTAs at work
// at once stream different weight rows; the first stages' weight tiles are
// loaded before the dependency wait.  The epilogue reads one feature per
// thread (TMEM lane) and writes the transpose: for each token the warp's 32
// lanes store 32 consecutive features (coalesced).  Roles as gemm_bf16_tn.
//
// Output modes:
//   LS_BF16  one bf16 result [n][nout]
//   LS_F32   `splits` fp32 partial planes [s][n][nout]
//   LS_SILU  the MLP's gate|up projection with SiLU-and-mul in the epilogue
//            (``layers/activation.py:5-14``): W = [gate; up] [2I][K] and
//            act[t][f] = silu(gate_t[f]) * up_t[f] for f < I = nout.  Each
//            128-row W tile is loaded as four 32-row boxes, gate rows
//            64m..64m+31, up rows I+64m.., gate 64m+32.., up I+64m+32.., so
//            TMEM lane quadrants 0/1 (and 2/3) hold the gate and up values of
//            the same 32 features.  The two warps of a pair swap half of
//            their (bf16-rounded, as the reference's bf16 linear output)
//            values through shared memory and each writes act for half of
//            the tokens.  The separate [n][2I] gate|up tensor never exists.
constexpr int LS_BM = 128, LS_BN = 64, LS_BK = 64, LS_ST = 8, LS_THREADS = 192;
constexpr int LS_BF16 = 0, LS_F32 = 1, LS_SILU = 2;

struct LsShape {
  static constexpr int A_BYTES = LS_BM * LS_BK * 2;   // 16 KB of W
  static constexpr int B_BYTES = LS_BN * LS_BK * 2;   // 8 KB of X
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int SMEM = LS_ST * STAGE_BYTES + 1024 + 256;
  static constexpr int XBUF_FLOATS = 2 * 2 * 32 * 32;  // LS_SILU: [pair][chunk parity][token][lane]
  static constexpr int SMEM_SILU = SMEM + XBUF_FLOATS * 4;
  static constexpr uint32_t TMEM_COLS = 2 * LS_BN;    // double-buffered accumulators
};

// Named barrier over `nthreads` threads (whole warps) that also returns the
// AND of every participant's predicate.
DFM_DEV bool bar_red_and(int id, int nthreads, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(pred)), "r"(id), "r"(nthreads)
      : "memory");
  return r != 0;
}

DFM_DEV void bar_sync_n(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

struct LsArgs {
  int tiles_m, tok_blocks, splits, nk;   // feature tiles, token blocks, K splits, k-blocks per split
  int n, nout;                           // tokens, output features (row stride of out; I for LS_SILU)
  void* out;                             // fp32 planes [splits][rows][nout] or bf16 [rows][nout]
  size_t plane;                          // elements between planes
};

template <int kMode>
__global__ void __launch_bounds__(LS_THREADS, 1)
    llm_swap_gemm_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                         LsArgs p, uint32_t* err) {
  using S = LsShape;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + LS_ST * S::A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + LS_ST * S::STAGE_BYTES);
  uint64_t* empty = full + LS_ST;
  uint64_t* tm_full = empty + LS_ST;  // [2]
  uint64_t* tm_empty = tm_full + 2;   // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tm_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* xbuf = reinterpret_cast<float*>(smem + LS_ST * S::STAGE_BYTES + 256);   // LS_SILU only
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int total = p.tiles_m * p.tok_blocks * p.splits;
  // one W tile: a 128-row box, or (LS_SILU) four 32-row boxes of gate and up rows
  auto load_w = [&](uint8_t* dst, uint64_t* bar, int kx, int m0) {
    if constexpr (kMode == LS_SILU) {
#pragma unroll
      for (int q = 0; q < 4; ++q)
        tma_load_2d(dst + q * (S::A_BYTES / 4), &tmW, bar, kx,
                    (q & 1) * p.nout + (m0 >> 1) + 32 * (q >> 1));
    } else {
      tma_load_2d(dst, &tmW, bar, kx, m0);
    }
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < LS_ST; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tm_full[b], 1);
      mbar_init(&tm_empty[b], 4);
    }
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch(&tmW);
    tma_prefetch(&tmX);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, S::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_trigger();

  auto unit = [&](int t, int& m0, int& t0, int& kb0, int& s) {
    const int mt = t % p.tiles_m, rest = t / p.tiles_m;
    const int tb = rest % p.tok_blocks;
    s = rest / p.tok_blocks;
    m0 = mt * LS_BM;
    t0 = tb * LS_BN;
    kb0 = s * p.nk;
  };

  if (warp == 0) {
    if (lane == 0) {
      // the weights do not depend on the previous kernel: the first stages'
      // W tiles go out before the dependency wait
      int m0, t0, kb0, s;
      unit(blockIdx.x, m0, t0, kb0, s);
      const int pre = static_cast<int>(blockIdx.x) < total ? (p.nk < LS_ST ? p.nk : LS_ST) : 0;
      for (int kb = 0; kb < pre; ++kb) {
        mbar_arrive_expect_tx(&full[kb], S::STAGE_BYTES);
        load_w(sA + kb * S::A_BYTES, &full[kb], (kb0 + kb) * LS_BK, m0);
      }
      pdl_wait();
      int g = 0;
      bool ok = true;
#pragma unroll 1
      for (int t = blockIdx.x; ok && t < total; t += gridDim.x) {
        unit(t, m0, t0, kb0, s);
#pragma unroll 1
        for (int kb = 0; kb < p.nk; ++kb, ++g) {
          const int st = g % LS_ST;
          const uint32_t ph = (g / LS_ST) & 1;
          if (g >= pre) {
            if (g >= LS_ST && !mbar_wait(&empty[st], ph ^ 1, abort_flag, err)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&full[st], S::STAGE_BYTES);
            load_w(sA + st * S::A_BYTES, &full[st], (kb0 + kb) * LS_BK, m0);
          }
          tma_load_2d(sB + st * S::B_BYTES, &tmX, &full[st], (kb0 + kb) * LS_BK, t0);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_bf16(LS_BM, LS_BN);
      int g = 0, u = 0;
      bool ok = true;
#pragma unroll 1
      for (int t = blockIdx.x; ok && t < total; t += gridDim.x, ++u) {
        const int b = u & 1;
        if (u >= 2 && !mbar_wait(&tm_empty[b], ((u >> 1) & 1) ^ 1, abort_flag, err)) break;
        tc_fence_after();
        const uint32_t acc = tmem + b * LS_BN;
#pragma unroll 1
        for (int kb = 0; kb < p.nk; ++kb, ++g) {
          const int st = g % LS_ST;
          if (!mbar_wait(&full[st], (g / LS_ST) & 1, abort_flag, err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a = smem_u32(sA + st * S::A_BYTES);
          const uint32_t bb = smem_u32(sB + st * S::B_BYTES);
#pragma unroll
          for (int kk = 0; kk < LS_BK / 16; ++kk)
            umma_bf16(acc, umma_desc_sw128(a + kk * 32), umma_desc_sw128(bb + kk * 32), idesc,
                      (kb | kk) != 0);
          umma_commit(&empty[st]);
        }
        if (ok) umma_commit(&tm_full[b]);
      }
    }
  } else {
    pdl_wait();
    const int q = warp & 3;
    const int pair = q >> 1;           // LS_SILU: quadrants 0/1 and 2/3 hold gate/up of one feature set
    const bool gate = (q & 1) == 0;
    int u = 0, ch = 0;
#pragma unroll 1
    for (int t = blockIdx.x; t < total; t += gridDim.x, ++u) {
      const int b = u & 1;
      bool ready = __all_sync(0xffffffffu, mbar_wait(&tm_full[b], (u >> 1) & 1, abort_flag, err));
      // the two warps of a pair meet at named barriers below: both leave together
      if constexpr (kMode == LS_SILU) ready = bar_red_and(1 + pair, 64, ready);
      if (!ready) break;
      tc_fence_after();
      int m0, t0, kb0, s;
      unit(t, m0, t0, kb0, s);
      const int j = kMode == LS_SILU ? (m0 >> 1) + 32 * pair + lane   // this thread's output feature
                                     : m0 + q * 32 + lane;
#pragma unroll 1
      for (int c = 0; c < LS_BN; c += 32, ++ch) {
        uint32_t r[32];
        tmem_ld32(tmem + b * LS_BN + c + (static_cast<uint32_t>(q * 32) << 16), r);
        tmem_wait_ld();
        if constexpr (kMode == LS_SILU) {
          // the pair splits the chunk's 32 tokens: the gate warp finishes
          // tokens 0-15 (with the up warp's values), the up warp 16-31
          float* xb = xbuf + (pair * 2 + (ch & 1)) * 1024;   // [16 tokens][lane] from each warp
          float v[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = __bfloat162float(__float2bfloat16(__uint_as_float(r[i])));
          if (gate) {
#pragma unroll
            for (int i = 0; i < 16; ++i) xb[512 + i * 32 + lane] = v[16 + i];
          } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) xb[i * 32 + lane] = v[i];
          }
          bar_sync_n(1 + pair, 64);
          __nv_bfloat16* act = static_cast<__nv_bfloat16*>(p.out) + static_cast<size_t>(t0 + c) * p.nout + j;
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            float g, up;
            int tok;
            if (gate) {
              g = v[i], up = xb[i * 32 + lane], tok = i;
            } else {
              g = xb[512 + i * 32 + lane], up = v[16 + i], tok = 16 + i;
            }
            if (t0 + c + tok < p.n)
              act[static_cast<size_t>(tok) * p.nout] = __float2bfloat16(__fdividef(g, 1.0f + __expf(-g)) * up);
          }
          continue;
        }
        if (j >= p.nout) continue;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int tok = t0 + c + i;
          if (tok < p.n) {
            const size_t o = (kMode == LS_F32 ? static_cast<size_t>(s) * p.plane : 0) +
                             static_cast<size_t>(tok) * p.nout + j;
            if constexpr (kMode == LS_F32)
              static_cast<float*>(p.out)[o] = __uint_as_float(r[i]);
            else
              static_cast<__nv_bfloat16*>(p.out)[o] = __float2bfloat16(__uint_as_float(r[i]));
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tm_empty[b]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, S::TMEM_COLS);
  }
}

}  // namespace dfm
