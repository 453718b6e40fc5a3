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
// CTA-pair kernel: TMA warp, MMA warp, and Epi::kEpiWarps epilogue warps (4:
// one per TMEM lane quadrant; 8: two per quadrant, each taking half of the
// tile's columns).
template <class Epi>
constexpr int gemm2_threads() { return 64 + 32 * Epi::kEpiWarps; }

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
  static constexpr int kStageBytes = 0;
  static constexpr int kEpiWarps = 4;
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

// out[split][row][col] = act(acc + (split == 0 ? bias[col] : 0)) in fp32 or
// bf16, written through a shared-memory staging box and TMA stores, so global
// memory sees whole 128-byte lines.  The output tensor map is 3-D
// {cols, rows, splits} with box {128 bytes of columns, 32 rows, 1} and the
// 128-byte swizzle; rows beyond the map are clipped by the TMA unit.  Used by
// the CTA-pair kernel (which passes each epilogue warp its staging buffers).
template <bool F32>
struct EpiStoreT {
  static constexpr int kStageBytes = 8192;  // per epilogue warp: two 4 KB boxes
  static constexpr int kEpiWarps = 8;
  static constexpr int CW = F32 ? 32 : 64;  // columns per 128-byte line
  const float* bias;
  int act;                         // 0 none, 1 GELU(tanh) (the DiT MLP), 2 SiLU (the patch encoder's)
  const float* a_scale = nullptr;  // FP8 operands: per-row scale of A ...
  const float* w_scale = nullptr;  // ... and per-output-column scale of W

  // Loaded before the accumulator is ready: lane l holds the bias and weight
  // scale of columns n0 + 4l .. 4l + 3 (the warp's BN <= 128 columns), handed
  // to the other lanes by shuffles, and the scale of its own row.
  struct Row {
    float4 b4, w4;
    float sa;
  };
  template <int BN>
  DFM_DEV Row row_state(int row0, int lane, int n0, int M) const {
    static_assert(BN <= 128, "four columns per lane");
    Row st;
    st.b4 = make_float4(0.f, 0.f, 0.f, 0.f);
    st.w4 = make_float4(1.f, 1.f, 1.f, 1.f);
    st.sa = 1.f;
    if (4 * lane < BN) {
      if (bias) st.b4 = __ldg(reinterpret_cast<const float4*>(bias + n0) + lane);
      if (a_scale) st.w4 = __ldg(reinterpret_cast<const float4*>(w_scale + n0) + lane);
    }
    if (a_scale) st.sa = row0 + lane < M ? a_scale[row0 + lane] : 0.f;
    return st;
  }

  template <int BN>
  DFM_DEV void run_staged(const Row& st, uint32_t taddr, int row0, int lane, int n0, int M, int split,
                          uint8_t* stage, const CUtensorMap* map) const {
    static_assert(BN % CW == 0, "tile width");
    if (row0 >= M) return;  // all 32 rows of this warp are padding
    const bool add_bias = bias != nullptr && split == 0;
    const float bsel[4] = {st.b4.x, st.b4.y, st.b4.z, st.b4.w};
    const float wsel[4] = {st.w4.x, st.w4.y, st.w4.z, st.w4.w};
    uint8_t* rowp = stage + lane * 128;
    const int sw = lane & 7;
    int it = 0;
#pragma unroll 1
    for (int c = 0; c < BN; c += CW, ++it) {
      float v[CW];
      {
        uint32_t r[32];
        tmem_ld32(taddr + c, r);
        if constexpr (F32) {
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
        } else {
          uint32_t r1[32];
          tmem_ld32(taddr + c + 32, r1);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            v[j] = __uint_as_float(r[j]);
            v[j + 32] = __uint_as_float(r1[j]);
          }
        }
      }
      if (a_scale) {
#pragma unroll
        for (int j = 0; j < CW; ++j)
          v[j] *= st.sa * __shfl_sync(0xffffffffu, wsel[j & 3], (c + j) >> 2);
      }
      if (add_bias) {
#pragma unroll
        for (int j = 0; j < CW; ++j) v[j] += __shfl_sync(0xffffffffu, bsel[j & 3], (c + j) >> 2);
      }
      if (act == 1) {
#pragma unroll
        for (int j = 0; j < CW; ++j) v[j] = gelu_tanh(v[j]);
      } else if (act == 2) {
#pragma unroll
        for (int j = 0; j < CW; ++j) v[j] = silu(v[j]);
      }
      uint8_t* buf = rowp + (it & 1) * 4096;
      if (lane == 0) bulk_wait_read<1>();  // the store that last used this buffer has read it
      __syncwarp();
      // row `lane` of the box: 16-byte chunk k sits at chunk k ^ (row % 8)
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        uint4 w;
        if constexpr (F32) {
          w = make_uint4(__float_as_uint(v[4 * k]), __float_as_uint(v[4 * k + 1]),
                         __float_as_uint(v[4 * k + 2]), __float_as_uint(v[4 * k + 3]));
        } else {
          w = make_uint4(pack_bf16(v[8 * k], v[8 * k + 1]), pack_bf16(v[8 * k + 2], v[8 * k + 3]),
                         pack_bf16(v[8 * k + 4], v[8 * k + 5]), pack_bf16(v[8 * k + 6], v[8 * k + 7]));
        }
        *reinterpret_cast<uint4*>(buf + ((k ^ sw) << 4)) = w;
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        tma_store_3d(map, stage + (it & 1) * 4096, n0 + c, row0, split);
        bulk_commit();
      }
    }
  }
};

// Fused QKV epilogue.  Output columns [0,H) are q, [H,2H) k, [2H,3H) v, 64
// per head.  With kNormRope (the FM head) q and k get LayerNorm(head_dim)
// with affine, then NeoX rotary at the row's position; without it (the patch
// encoder, whose attention has neither, ``patch_encoder.py:31-32``) they pass
// through.  q goes to q_out, k and v are written into the paged K/V pool at
// (page = block_table[req][pos/16], row pos%16).
//
// Row layout: request i owns rows [slot*i, slot*(i+1)); the first ext_slots
// rows are graduating rows (live when j < n_ext[i], position P_i + j), the
// rest are active rows (position P_i + n_ext[i] + (j - ext_slots)).  Dead
// graduating rows write nothing to the pool.
//
// Each thread computes one row of a head (64 values, 128 bytes); the warp
// then copies its 32 rows out through a shared-memory box so that every store
// instruction writes four whole 128-byte rows instead of 32 scattered
// 16-byte pieces.
template <bool kNormRope>
struct EpiQKVT {
  static constexpr int kStageBytes = 4096;  // per epilogue warp: 32 rows x 128 bytes
  static constexpr int kEpiWarps = 4;       // the row state needs the registers
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
  const float2* rope;     // [32][max_pos] (cos, sin) of pos * inv_freq[d]
  int max_pos;
  float eps;
  uint32_t* err;
  const float* a_scale = nullptr;  // FP8 operands: per-row scale of A ...
  const float* w_scale = nullptr;  // ... and per-output-column scale of W

  // Per-row state gathered before the accumulator is ready (the loads overlap
  // the mainloop): position, destination page (k/v tiles) and the rotary
  // (cos, sin) of the row's position (q/k tiles; shared by all heads).
  struct Row {
    int pos, page;
    bool in_range;
    float2 cs[32];
    float sa;        // FP8: this row's activation scale
    float4 wlo, whi; // FP8: weight scales of columns n0 + 8l .. 8l + 7 (lane l)
  };

  template <int BN>
  DFM_DEV Row row_state(int row0, int lane, int n0, int M) const {
    static_assert(1024 % BN == 0 || BN % 64 == 0, "tile width");
    Row st;
    const int row = row0 + lane;
    st.in_range = row < M;
    const int i = st.in_range ? row / slot : 0;
    const int j = st.in_range ? row - i * slot : 0;
    const int ne = n_ext[i], P = cache_len[i];
    const bool ext = j < ext_slots;
    const bool live = st.in_range && (!ext || j < ne);
    st.pos = ext ? P + j : P + ne + (j - ext_slots);
    st.page = -1;
    if (live && n0 + BN > H) {  // the tile holds k or v columns
      const int pidx = st.pos >> 4;
      if (st.pos < 0 || pidx >= max_pages || ne < 0 || ne > ext_slots) {
        atomicOr(err, DFM_DEV_ERR_LEN);
      } else {
        st.page = block_table[static_cast<size_t>(i) * max_pages + pidx];
        if (st.page < 0 || st.page >= num_pages) {
          atomicOr(err, DFM_DEV_ERR_PAGE);
          st.page = -1;
        }
      }
    }
    st.sa = 1.f;
    st.wlo = st.whi = make_float4(1.f, 1.f, 1.f, 1.f);
    if (a_scale) {
      static_assert(BN <= 256, "eight columns per lane");
      st.sa = st.in_range ? a_scale[row] : 0.f;
      if (8 * lane < BN) {
        st.wlo = __ldg(reinterpret_cast<const float4*>(w_scale + n0) + 2 * lane);
        st.whi = __ldg(reinterpret_cast<const float4*>(w_scale + n0) + 2 * lane + 1);
      }
    }
    if (kNormRope && n0 < 2 * H) {  // q or k columns: rotary at this row's position
      const float2* cs = rope + (st.pos < 0 ? 0 : (st.pos < max_pos ? st.pos : max_pos - 1));
#pragma unroll
      for (int d = 0; d < 32; ++d) st.cs[d] = __ldg(cs + static_cast<size_t>(d) * max_pos);
    }
    return st;
  }

  template <int BN>
  DFM_DEV void run_staged(const Row& st, uint32_t taddr, int row0, int lane, int n0, int M, int,
                          uint8_t* stage, const CUtensorMap*) const {
    const int row = row0 + lane;
    uint8_t* rowp = stage + lane * 128;
    const int sw = lane & 7;
#pragma unroll 1
    for (int c = 0; c < BN; c += 64) {
      float x[64];
      {
        uint32_t r0[32], r1[32];
        tmem_ld32(taddr + c, r0);
        tmem_ld32(taddr + c + 32, r1);
        tmem_wait_ld();
#pragma unroll
        for (int d = 0; d < 32; ++d) {
          x[d] = __uint_as_float(r0[d]);
          x[d + 32] = __uint_as_float(r1[d]);
        }
      }
      const int col = n0 + c;
      if (a_scale) {
        const float wsel[8] = {st.wlo.x, st.wlo.y, st.wlo.z, st.wlo.w,
                               st.whi.x, st.whi.y, st.whi.z, st.whi.w};
#pragma unroll
        for (int d = 0; d < 64; ++d)
          x[d] *= st.sa * __shfl_sync(0xffffffffu, wsel[d & 7], (c + d) >> 3);
      }
      const int sec = col / H;
      const int head = (col - sec * H) >> 6;
      __nv_bfloat16* dst = nullptr;
      if (st.in_range && sec == 0)
        dst = q_out + static_cast<size_t>(row) * H + head * 64;
      else if (sec > 0 && st.page >= 0)
        dst = pool + static_cast<size_t>(sec == 1 ? plane_k : plane_v) * plane_elems +
              (static_cast<size_t>(st.page) * heads + head) * 1024 + (st.pos & 15) * 64;
      if (kNormRope && dst && sec < 2) {
        // LayerNorm(64) with four partial sums (short dependency chains)
        float s4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int d = 0; d < 64; ++d) s4[d & 3] += x[d];
        const float mean = ((s4[0] + s4[1]) + (s4[2] + s4[3])) * (1.0f / 64.0f);
        float v4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int d = 0; d < 64; ++d) {
          const float t = x[d] - mean;
          v4[d & 3] += t * t;
        }
        const float rstd = rsqrtf(((v4[0] + v4[1]) + (v4[2] + v4[3])) * (1.0f / 64.0f) + eps);
        const float4* w4 = reinterpret_cast<const float4*>(qk_norm + sec * 128);
#pragma unroll
        for (int d = 0; d < 64; d += 4) {
          const float4 w = __ldg(w4 + d / 4), bb = __ldg(w4 + 16 + d / 4);
          x[d] = (x[d] - mean) * rstd * w.x + bb.x;
          x[d + 1] = (x[d + 1] - mean) * rstd * w.y + bb.y;
          x[d + 2] = (x[d + 2] - mean) * rstd * w.z + bb.z;
          x[d + 3] = (x[d + 3] - mean) * rstd * w.w + bb.w;
        }
#pragma unroll
        for (int d = 0; d < 32; ++d) {
          const float2 t = st.cs[d];
          const float a = x[d], b = x[d + 32];
          x[d] = a * t.x - b * t.y;
          x[d + 32] = b * t.x + a * t.y;
        }
      }
      // this row into the box (16-byte chunk k at chunk k ^ (row % 8)) ...
#pragma unroll
      for (int k = 0; k < 8; ++k)
        *reinterpret_cast<uint4*>(rowp + ((k ^ sw) << 4)) =
            make_uint4(pack_bf16(x[8 * k], x[8 * k + 1]), pack_bf16(x[8 * k + 2], x[8 * k + 3]),
                       pack_bf16(x[8 * k + 4], x[8 * k + 5]), pack_bf16(x[8 * k + 6], x[8 * k + 7]));
      __syncwarp();
      // ... then out four whole rows per instruction: lane l copies chunk l % 8 of row 4 p + l / 8
      const unsigned long long mine = reinterpret_cast<unsigned long long>(dst);
#pragma unroll
      for (int p = 0; p < 8; ++p) {
        const int r = p * 4 + (lane >> 3), k = lane & 7;
        const unsigned long long d = __shfl_sync(0xffffffffu, mine, r);
        const uint4 v = *reinterpret_cast<const uint4*>(stage + r * 128 + ((k ^ (r & 7)) << 4));
        if (d) reinterpret_cast<uint4*>(d)[k] = v;
      }
      __syncwarp();
    }
  }
};

using EpiQKV = EpiQKVT<true>;

// MeanFlow update fused into the final projection (N = latent_dim = 64):
// z[row] += dt * (acc + bias); zb[row] = bf16(z[row]).  Loads are batched per
// chunk.
struct EpiSolver {
  static constexpr int kStageBytes = 0;
  static constexpr int kEpiWarps = 4;
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

// ---------------------------------------------------------------- CTA-pair kernel
// Output tiles of 256 x BN computed by a cluster of two CTAs (cta_group::2).
// CTA r of the pair loads rows [m0 + 128 r, +128) of A and rows
// [n0 + r BN/2, +BN/2) of W into its own ring; one thread of CTA 0 issues
// 256 x BN x 16 MMAs that read both CTAs' shared memory, and each CTA's TMEM
// receives its own 128 output rows.  Each SM thus streams 128 x 64 of A and
// BN/2 x 64 of W per 128 x BN x 64 of math: half the weight bytes of the
// single-CTA kernel per FLOP.  All completion signals that cross the pair:
//   - TMA bytes of both CTAs count on CTA 0's full[s] (CTA 0 expects both);
//   - CTA 0's MMA commits to empty[s] and tm_full[b] of both CTAs;
//   - the epilogue warps of both CTAs arrive on CTA 0's tm_empty[b].
template <int BN, int STAGES, int EPI_STAGE = 0, int EPI_WARPS = 4>
struct Gemm2Shape {
  static_assert(BN % 32 == 0 && BN >= 64 && BN <= 256, "pair MMA N");
  static constexpr int A_BYTES = GEMM_BM * GEMM_BK * 2;     // this CTA's 128 rows of A
  static constexpr int B_BYTES = (BN / 2) * GEMM_BK * 2;    // this CTA's half of the W tile
  static_assert(B_BYTES % 1024 == 0, "swizzle atoms");
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int EPI_BYTES = EPI_WARPS * EPI_STAGE;  // staging boxes of the epilogue warps
  static constexpr int SMEM = STAGES * STAGE_BYTES + EPI_BYTES + 1024 + 256;
  static_assert(SMEM <= 232448, "shared memory per CTA");
  static constexpr uint32_t TMEM_COLS = 2 * BN <= 256 ? 256 : 512;
};

// Work units are (output tile, K split): unit t covers tile t % tiles and
// k-blocks [s * nk / ksplit, (s + 1) * nk / ksplit) with s = t / tiles; the
// epilogue gets s (split-K partial sums go to separate output planes).
// FP8: both operands e4m3 (one 128-byte swizzle row = 128 elements of K per
// k-block, kind::f8f6f4 MMAs); the epilogue applies the row and column scales.
template <int BN, int STAGES, class Epi, bool FP8 = false>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(gemm2_threads<Epi>(), 1)
    gemm2_bf16_tn(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                  const __grid_constant__ CUtensorMap tmC, int M, int N, int K, int ksplit, Epi epi,
                  uint32_t* err) {
  using S = Gemm2Shape<BN, STAGES, Epi::kStageBytes, Epi::kEpiWarps>;
  static_assert(Epi::kEpiWarps == 4 || Epi::kEpiWarps == 8, "epilogue warps");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * S::A_BYTES;
  uint8_t* sE = smem + STAGES * S::STAGE_BYTES;  // epilogue staging (1024-aligned)
  uint64_t* full = reinterpret_cast<uint64_t*>(sE + S::EPI_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tm_full = empty + STAGES;   // [2]
  uint64_t* tm_empty = tm_full + 2;     // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tm_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int tiles_m = (M + 2 * GEMM_BM - 1) / (2 * GEMM_BM);
  const int tiles = tiles_m * (N / BN);
  const int total = tiles * ksplit;
  constexpr int BKE = FP8 ? 2 * GEMM_BK : GEMM_BK;  // K elements per 128-byte k-block
  const int nkb = K / BKE / ksplit;  // k-blocks per unit

  if (threadIdx.x == 0) {
#pragma unroll 1
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tm_full[b], 1);
      mbar_init(&tm_empty[b], 2 * Epi::kEpiWarps);
    }
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch(&tmA);
    tma_prefetch(&tmB);
    if (Epi::kStageBytes) tma_prefetch(&tmC);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, S::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialised before either signals the other
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_trigger();

  if (warp == 0) {
    if (lane == 0) {
      const int a_row = static_cast<int>(rank) * GEMM_BM;
      const int b_row = static_cast<int>(rank) * (BN / 2);
      // Weights do not depend on the previous kernel: fetch the first stages
      // of the first unit's W before waiting for it, then its activations.
      const int pre = (pair < total) ? (nkb < STAGES ? nkb : STAGES) : 0;
      const int t00 = pair % tiles;
      const int n00 = (t00 / tiles_m) * BN + b_row, k00 = (pair / tiles) * nkb;
      for (int kb = 0; kb < pre; ++kb) {
        if (rank == 0) mbar_arrive_expect_tx(&full[kb], 2 * S::STAGE_BYTES);
        tma_load_2d_pair(sB + kb * S::B_BYTES, &tmB, cluster_map(smem_u32(&full[kb]), 0),
                         (k00 + kb) * BKE, n00);
      }
      pdl_wait();
      int g = 0;
      bool ok = true;
#pragma unroll 1
      for (int t = pair; ok && t < total; t += npairs) {
        const int tile = t % tiles, k0 = (t / tiles) * nkb;
        const int m0 = (tile % tiles_m) * 2 * GEMM_BM + a_row, n0 = (tile / tiles_m) * BN + b_row;
#pragma unroll 1
        for (int kb = 0; kb < nkb; ++kb, ++g) {
          const int s = g % STAGES;
          const uint32_t ph = (g / STAGES) & 1;
          const uint32_t bar = cluster_map(smem_u32(&full[s]), 0);
          if (g >= pre) {
            if (g >= STAGES && !mbar_wait(&empty[s], ph ^ 1, abort_flag, err)) {
              ok = false;
              break;
            }
            if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * S::STAGE_BYTES);
            tma_load_2d_pair(sB + s * S::B_BYTES, &tmB, bar, (k0 + kb) * BKE, n0);
          }
          tma_load_2d_pair(sA + s * S::A_BYTES, &tmA, bar, (k0 + kb) * BKE, m0);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc = FP8 ? umma_idesc_e4m3(2 * GEMM_BM, BN) : umma_idesc_bf16(2 * GEMM_BM, BN);
      int g = 0, u = 0;
      bool ok = true;
#pragma unroll 1
      for (int t = pair; ok && t < total; t += npairs, ++u) {
        const int b = u & 1;
        if (u >= 2 && !mbar_wait(&tm_empty[b], ((u >> 1) & 1) ^ 1, abort_flag, err)) break;
        tc_fence_after();
        const uint32_t acc = tmem + b * BN;
#pragma unroll 1
        for (int kb = 0; kb < nkb; ++kb, ++g) {
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
          for (int kk = 0; kk < 4; ++kk) {  // 32 bytes of K per MMA
            if constexpr (FP8)
              umma_fp8_pair(acc, umma_desc_sw128(a + kk * 32), umma_desc_sw128(bb + kk * 32), idesc,
                            (kb | kk) != 0);
            else
              umma_bf16_pair(acc, umma_desc_sw128(a + kk * 32), umma_desc_sw128(bb + kk * 32), idesc,
                             (kb | kk) != 0);
          }
          const uint32_t e = smem_u32(&empty[s]);
          umma_commit_pair(cluster_map(e, 0));
          umma_commit_pair(cluster_map(e, 1));
        }
        if (ok) {
          const uint32_t f = smem_u32(&tm_full[b]);
          umma_commit_pair(cluster_map(f, 0));
          umma_commit_pair(cluster_map(f, 1));
        }
      }
    }
  } else {
    pdl_wait();
    const int q = warp & 3;               // TMEM lane quadrant (rows 32q .. 32q + 31)
    const int half = (warp - 2) >> 2;     // which part of the tile's columns
    constexpr int HB = BN * 4 / Epi::kEpiWarps;
    int u = 0;
#pragma unroll 1
    for (int t = pair; t < total; t += npairs, ++u) {
      const int b = u & 1;
      const int tile = t % tiles;
      const int row0 = (tile % tiles_m) * 2 * GEMM_BM + static_cast<int>(rank) * GEMM_BM + q * 32;
      const int n0 = (tile / tiles_m) * BN + half * HB;
      const uint32_t taddr = tmem + b * BN + half * HB + (static_cast<uint32_t>(q * 32) << 16);
      if constexpr (Epi::kStageBytes > 0) {
        // row-only state first: its loads overlap the wait for the accumulator
        const auto st = epi.template row_state<HB>(row0, lane, n0, M);
        const bool ready =
            __all_sync(0xffffffffu, mbar_wait(&tm_full[b], (u >> 1) & 1, abort_flag, err));
        if (!ready) break;
        tc_fence_after();
        epi.template run_staged<HB>(st, taddr, row0, lane, n0, M, t / tiles,
                                    sE + (warp - 2) * Epi::kStageBytes, &tmC);
      } else {
        const bool ready =
            __all_sync(0xffffffffu, mbar_wait(&tm_full[b], (u >> 1) & 1, abort_flag, err));
        if (!ready) break;
        tc_fence_after();
        epi.template run<HB>(taddr, row0 + lane, n0, M);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(cluster_map(smem_u32(&tm_empty[b]), 0));
    }
    if (Epi::kStageBytes && lane == 0) bulk_wait_all();  // staged stores complete before exit
  }
  tc_fence_before();
  cluster_sync();  // no CTA leaves while the pair may still read its memory or signal it
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, S::TMEM_COLS);
  }
}

}  // namespace dfm
