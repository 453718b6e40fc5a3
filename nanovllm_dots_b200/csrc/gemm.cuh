// tcgen05 GEMM for the FM head: C[M, N] = A[M, K] . W[N, K]^T with the
// epilogue fused (bias, GELU, per-head LayerNorm + rotary + paged K/V write,
// MeanFlow solver update).
//
// Output tiles are 128 x BN.  Warp roles (192 threads):
//   warp 0      TMA producer: A and W tiles (128-byte swizzle) into a
//               STAGES-deep shared-memory ring, one mbarrier per stage
//   warp 1      TMEM allocator + the single thread that issues tcgen05.mma
//               (128 x BN x 16 per instruction, fp32 accumulator in TMEM) and
//               commits each stage back to the producer
//   warps 2..5  epilogue: tcgen05.ld of the accumulator (warp w reads TMEM
//               lanes 32*(w%4)..+31, i.e. one output row per thread), the fused
//               math, and global stores
// Operands are bf16 and K-major (nn.Linear weight layout), K % 64 == 0.
// Rows of A beyond M read as zeros (TMA out-of-bounds fill) or as rows of
// the workspace that the epilogue never stores.
#pragma once

#include "common.cuh"

namespace dfm {

constexpr int GEMM_BM = 128;
constexpr int GEMM_BK = 64;  // one 128-byte swizzle row of bf16
constexpr int GEMM_THREADS = 192;

template <int BN, int STAGES>
struct GemmShape {
  static constexpr int A_BYTES = GEMM_BM * GEMM_BK * 2;
  static constexpr int B_BYTES = BN * GEMM_BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + 256;
  // two accumulator buffers of BN fp32 columns, rounded up to a power of two
  static constexpr uint32_t TMEM_COLS = 2 * BN <= 32 ? 32 : 2 * BN <= 64 ? 64 : 2 * BN <= 128 ? 128
                                        : 2 * BN <= 256 ? 256 : 512;
};

// ---------------------------------------------------------------- epilogues
// Each epilogue reads its thread's accumulator row from TMEM (all lanes of the
// warp must execute the loads; rows >= M only skip the stores).

// out[omap(row), col] = act(acc + bias[col]) in bf16 or fp32.
struct EpiStore {
  void* out;
  int ldo;
  int out_f32;
  const float* bias;
  int gelu;
  RowMap omap;

  template <int BN>
  DFM_DEV void run(uint32_t taddr, int row, int n0, int M) const {
#pragma unroll 1
    for (int c = 0; c < BN; c += 32) {
      uint32_t r[32];
      tmem_ld32(taddr + c, r);
      tmem_wait_ld();
      if (row >= M) continue;
      float v[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
      if (bias) {
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
          const float4 b = *reinterpret_cast<const float4*>(bias + n0 + c + j);
          v[j] += b.x; v[j + 1] += b.y; v[j + 2] += b.z; v[j + 3] += b.w;
        }
      }
      if (gelu) {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = gelu_tanh(v[j]);
      }
      const size_t o = static_cast<size_t>(omap(row)) * ldo + n0 + c;
      if (out_f32) {
        float4* dst = reinterpret_cast<float4*>(static_cast<float*>(out) + o);
#pragma unroll
        for (int j = 0; j < 8; ++j) dst[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
      } else {
        uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(out) + o);
#pragma unroll
        for (int j = 0; j < 4; ++j)
          dst[j] = make_uint4(pack_bf16(v[8 * j], v[8 * j + 1]), pack_bf16(v[8 * j + 2], v[8 * j + 3]),
                              pack_bf16(v[8 * j + 4], v[8 * j + 5]), pack_bf16(v[8 * j + 6], v[8 * j + 7]));
      }
    }
  }
};

// Fused QKV epilogue.  Output columns [0,H) are q, [H,2H) k, [2H,3H) v, 64
// per head.  q and k get LayerNorm(head_dim) with affine, then NeoX rotary at
// the row's position; q goes to q_out, k and v are written into the paged
// K/V pool at (page = block_table[req][pos/16], row pos%16).
//
// Row layout: request i owns rows [slot*i, slot*(i+1)); the first ext_slots
// rows are graduating rows (live when j < n_ext[i], position P_i + j), the
// rest are active rows (position P_i + n_ext[i] + (j - ext_slots)).  Dead
// graduating rows write nothing to the pool.
struct EpiQKV {
  __nv_bfloat16* q_out;
  __nv_bfloat16* pool;
  size_t plane_elems;  // elements of one (layer, step, K|V) plane: pages*heads*16*dh
  int plane_k, plane_v;
  const int* cache_len;
  const int* n_ext;
  const int* block_table;
  int max_pages, num_pages, heads, H;
  int slot, ext_slots;
  const float* qk_norm;   // this layer's [4][64]: q_w, q_b, k_w, k_b
  const float2* rope;     // [max_pages*16][32] (cos, sin) of pos * inv_freq[d]
  int max_pos;
  float eps;
  uint32_t* err;

  template <int BN>
  DFM_DEV void run(uint32_t taddr, int row, int n0, int M) const {
    // Row metadata (position and destination page) once per row, not per head.
    const bool in_range = row < M;
    const int i = in_range ? row / slot : 0;
    const int j = in_range ? row - i * slot : 0;
    const int ne = n_ext[i], P = cache_len[i];
    const bool ext = j < ext_slots;
    const bool live = in_range && (!ext || j < ne);
    const int pos = ext ? P + j : P + ne + (j - ext_slots);
    const int pidx = pos >> 4;
    int page = -1;
    if (live && n0 >= H) {
      if (pos < 0 || pidx >= max_pages || ne < 0 || ne > ext_slots) {
        atomicOr(err, DFM_DEV_ERR_LEN);
      } else {
        page = block_table[static_cast<size_t>(i) * max_pages + pidx];
        if (page < 0 || page >= num_pages) {
          atomicOr(err, DFM_DEV_ERR_PAGE);
          page = -1;
        }
      }
    }
#pragma unroll 1
    for (int c = 0; c < BN; c += 64) {
      uint32_t r0[32], r1[32];
      tmem_ld32(taddr + c, r0);
      tmem_ld32(taddr + c + 32, r1);
      tmem_wait_ld();
      if (!in_range) continue;
      const int col = n0 + c;
      const int sec = col / H;
      const int head = (col - sec * H) >> 6;
      if (sec > 0 && page < 0) continue;
      float x[64];
#pragma unroll
      for (int d = 0; d < 32; ++d) {
        x[d] = __uint_as_float(r0[d]);
        x[d + 32] = __uint_as_float(r1[d]);
      }
      if (sec < 2) {
        float mean = 0.f;
#pragma unroll
        for (int d = 0; d < 64; ++d) mean += x[d];
        mean *= (1.0f / 64.0f);
        float var = 0.f;
#pragma unroll
        for (int d = 0; d < 64; ++d) {
          const float t = x[d] - mean;
          var += t * t;
        }
        const float rstd = rsqrtf(var * (1.0f / 64.0f) + eps);
        const float* w = qk_norm + sec * 128;
#pragma unroll
        for (int d = 0; d < 64; ++d) x[d] = (x[d] - mean) * rstd * __ldg(w + d) + __ldg(w + 64 + d);
        const float2* cs = rope + static_cast<size_t>(pos < 0 ? 0 : (pos < max_pos ? pos : max_pos - 1)) * 32;
#pragma unroll
        for (int d = 0; d < 32; ++d) {
          const float2 t = __ldg(cs + d);
          const float a = x[d], b = x[d + 32];
          x[d] = a * t.x - b * t.y;
          x[d + 32] = b * t.x + a * t.y;
        }
      }
      __nv_bfloat16* dst;
      if (sec == 0) {
        dst = q_out + static_cast<size_t>(row) * H + head * 64;
      } else {
        dst = pool + static_cast<size_t>(sec == 1 ? plane_k : plane_v) * plane_elems +
              (static_cast<size_t>(page) * heads + head) * 1024 + (pos & 15) * 64;
      }
      uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
      for (int q = 0; q < 8; ++q)
        d4[q] = make_uint4(pack_bf16(x[8 * q], x[8 * q + 1]), pack_bf16(x[8 * q + 2], x[8 * q + 3]),
                           pack_bf16(x[8 * q + 4], x[8 * q + 5]), pack_bf16(x[8 * q + 6], x[8 * q + 7]));
    }
  }
};

// MeanFlow update fused into the final projection (N = latent_dim = 64):
// z[row] += dt * (acc + bias); zb[row] = bf16(z[row]).  Loads are batched per
// chunk.
struct EpiSolver {
  float* z;
  __nv_bfloat16* zb;
  const float* bias;
  float dt;

  template <int BN>
  DFM_DEV void run(uint32_t taddr, int row, int n0, int M) const {
    const bool live = row < M;
    float* zp = z + static_cast<size_t>(live ? row : 0) * 64 + n0;
#pragma unroll 1
    for (int c = 0; c < BN; c += 32) {
      uint32_t r[32];
      tmem_ld32(taddr + c, r);
      float4 zv[8], bv[8];
      if (live) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          zv[j] = *reinterpret_cast<const float4*>(zp + c + 4 * j);
          bv[j] = __ldg(reinterpret_cast<const float4*>(bias + n0 + c + 4 * j));
        }
      }
      tmem_wait_ld();
      if (!live) continue;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        zv[j].x += dt * (__uint_as_float(r[4 * j]) + bv[j].x);
        zv[j].y += dt * (__uint_as_float(r[4 * j + 1]) + bv[j].y);
        zv[j].z += dt * (__uint_as_float(r[4 * j + 2]) + bv[j].z);
        zv[j].w += dt * (__uint_as_float(r[4 * j + 3]) + bv[j].w);
        *reinterpret_cast<float4*>(zp + c + 4 * j) = zv[j];
      }
      uint4* d4 = reinterpret_cast<uint4*>(zb + static_cast<size_t>(row) * 64 + n0 + c);
#pragma unroll
      for (int q = 0; q < 4; ++q)
        d4[q] = make_uint4(pack_bf16(zv[2 * q].x, zv[2 * q].y), pack_bf16(zv[2 * q].z, zv[2 * q].w),
                           pack_bf16(zv[2 * q + 1].x, zv[2 * q + 1].y),
                           pack_bf16(zv[2 * q + 1].z, zv[2 * q + 1].w));
    }
  }
};

// ---------------------------------------------------------------- kernel
// Persistent: grid = min(tiles, SMs); CTA b computes tiles b, b + grid, ...
// in (m fastest) order, so CTAs working at the same time share weight tiles in
// L2.  The TMEM accumulator is double-buffered: the epilogue of tile u drains
// buffer u%2 while the MMA thread fills the other buffer for tile u+1.
template <int BN, int STAGES, class Epi>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    gemm_bf16_tn(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                 int M, int N, int K, Epi epi, uint32_t* err) {
  using S = GemmShape<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * S::A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * S::STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tm_full = empty + STAGES;   // [2]
  uint64_t* tm_empty = tm_full + 2;     // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tm_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles_m = (M + GEMM_BM - 1) / GEMM_BM;
  const int total = tiles_m * (N / BN);
  const int nk = K / GEMM_BK;

  if (threadIdx.x == 0) {
#pragma unroll 1
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tm_full[b], 1);
      mbar_init(&tm_empty[b], 4);
    }
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch(&tmA);
    tma_prefetch(&tmB);
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

  if (warp == 0) {
    if (lane == 0) {
      // Weights do not depend on the previous kernel: fetch the first stages of
      // the first tile's W before waiting for it, then its activations.
      const int pre = (blockIdx.x < total) ? (nk < STAGES ? nk : STAGES) : 0;
      const int n00 = (blockIdx.x / tiles_m) * BN;
      for (int kb = 0; kb < pre; ++kb) {
        mbar_arrive_expect_tx(&full[kb], S::STAGE_BYTES);
        tma_load_2d(sB + kb * S::B_BYTES, &tmB, &full[kb], kb * GEMM_BK, n00);
      }
      pdl_wait();
      int g = 0;
      bool ok = true;
#pragma unroll 1
      for (int t = blockIdx.x; ok && t < total; t += gridDim.x) {
        const int m0 = (t % tiles_m) * GEMM_BM, n0 = (t / tiles_m) * BN;
#pragma unroll 1
        for (int kb = 0; kb < nk; ++kb, ++g) {
          const int s = g % STAGES;
          const uint32_t ph = (g / STAGES) & 1;
          if (g >= pre) {
            if (g >= STAGES && !mbar_wait(&empty[s], ph ^ 1, abort_flag, err)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&full[s], S::STAGE_BYTES);
            tma_load_2d(sB + s * S::B_BYTES, &tmB, &full[s], kb * GEMM_BK, n0);
          }
          tma_load_2d(sA + s * S::A_BYTES, &tmA, &full[s], kb * GEMM_BK, m0);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_bf16(GEMM_BM, BN);
      int g = 0, u = 0;
      bool ok = true;
#pragma unroll 1
      for (int t = blockIdx.x; ok && t < total; t += gridDim.x, ++u) {
        const int b = u & 1;
        if (u >= 2 && !mbar_wait(&tm_empty[b], ((u >> 1) & 1) ^ 1, abort_flag, err)) break;
        tc_fence_after();
        const uint32_t acc = tmem + b * BN;
#pragma unroll 1
        for (int kb = 0; kb < nk; ++kb, ++g) {
          const int s = g % STAGES;
          const uint32_t ph = (g / STAGES) & 1;
          if (!mbar_wait(&full[s], ph, abort_flag, err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a = smem_u32(sA + s * S::A_BYTES);
          const uint32_t bb = smem_u32(sB + s * S::B_BYTES);
#pragma unroll
          for (int kk = 0; kk < GEMM_BK / 16; ++kk)
            umma_bf16(acc, umma_desc_sw128(a + kk * 32), umma_desc_sw128(bb + kk * 32), idesc,
                      (kb | kk) != 0);
          umma_commit(&empty[s]);
        }
        if (ok) umma_commit(&tm_full[b]);
      }
    }
  } else {
    pdl_wait();
    const int q = warp & 3;
    int u = 0;
#pragma unroll 1
    for (int t = blockIdx.x; t < total; t += gridDim.x, ++u) {
      const int b = u & 1;
      // The TMEM loads are warp-collective: decide for the whole warp.
      const bool ready =
          __all_sync(0xffffffffu, mbar_wait(&tm_full[b], (u >> 1) & 1, abort_flag, err));
      if (!ready) break;
      tc_fence_after();
      const int m0 = (t % tiles_m) * GEMM_BM, n0 = (t / tiles_m) * BN;
      epi.template run<BN>(tmem + b * BN + (static_cast<uint32_t>(q * 32) << 16), m0 + q * 32 + lane,
                           n0, M);
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
