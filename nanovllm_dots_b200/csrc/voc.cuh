// Kernels of the vocoder's decode path (BigVGAN AudioVAE decoder,
// ``nanovllm_dots/models/dots/native/vocoder/bigvgan.py``).
//
// Activations are frames-first: [request][frame][Cp] with Cp the channel
// count padded to a multiple of 32.  Convolution operands (the activation
// outputs, the decoder input, each stage's output copy, the weights) are fp16
// (10-bit mantissa, as tf32) in 64-byte swizzle rows of 32 channels; the
// residual stream, conv outputs and accumulators are fp32.
//
//   voc_conv_kernel   every convolution of the decoder as an implicit GEMM on
//                     the tcgen05 tensor cores (kind::f16 with fp16 operands,
//                     fp32 accumulate in TMEM): out[t] = sum over taps j of
//                     x[t + off0 + j*dil] W_j;
//                     tap j's A tile is a TMA box at the shifted frame
//                     coordinate, frames outside the request read as zeros;
//                     the epilogue adds bias, the residual, and the stage's
//                     resblock sum
//   voc_act_kernel    anti-aliased SnakeBeta (x2 upsample, activation, x2
//                     downsample; ``alias_free_act.py:12-48``)
//   voc_post_kernel   conv_post (7 causal taps to one channel) + tanh
//   voc_linear_kernel fp32 linear layers of the front
//   voc_lstm_step_kernel  one frame of one LSTM layer for every request
//   voc_pack_kernel   the decoder input: a stream window after appending a
//                     chunk, or one-shot latents masked to each length
#pragma once

#include <cuda_fp16.h>

#include "common.cuh"

namespace dfm {

// ---------------------------------------------------------------- tcgen05 f16
// Instruction descriptor of kind::f16 with fp16 A/B (format 0), fp32 D, both K-major.
__host__ __device__ constexpr uint32_t umma_idesc_f16(int M, int N) {
  return (1u << 4) | (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

// Shared-memory descriptor of a K-major tile with the 64-byte swizzle: rows
// of 32 fp16 (64 bytes), 8-row atoms of 512 bytes packed densely.  As with
// the 128-byte swizzle, the start may sit at any row of a 512-byte-aligned
// tile (the swizzle applies to the address bits, as TMA wrote them).
DFM_DEV uint64_t umma_desc_sw64(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr & 0x3FFFFu) >> 4);  // start address
  d |= static_cast<uint64_t>(1) << 16;                      // leading byte offset (unused)
  d |= static_cast<uint64_t>(512 >> 4) << 32;               // stride byte offset: 8 rows
  d |= static_cast<uint64_t>(1) << 46;                      // descriptor version (sm100)
  d |= static_cast<uint64_t>(4) << 61;                      // layout: 64-byte swizzle
  return d;
}

DFM_DEV void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// ---------------------------------------------------------------- conv
constexpr int VC_BM = 128;
constexpr int VC_BK = 32;    // channels (fp16) per 64-byte swizzle row
constexpr int VC_ROWB = 64;  // bytes per row of an operand tile
constexpr int VC_THREADS = 192;

template <int BN, int STAGES>
struct VcShape {
  static_assert(BN % 32 == 0 && BN >= 32 && BN <= 256, "MMA N");
  static constexpr int A_BYTES = VC_BM * VC_ROWB;  // 8 KB: 128 frames x 32 channels
  static constexpr int B_BYTES = BN * VC_ROWB;
  static_assert(B_BYTES % 1024 == 0, "swizzle atoms");
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + 256;
  static_assert(SMEM <= 232448, "shared memory per CTA");
  static constexpr uint32_t TMEM_COLS = 2 * BN <= 64 ? 64 : 2 * BN <= 128 ? 128
                                        : 2 * BN <= 256 ? 256 : 512;
};

struct VcArgs {
  int tiles_m;        // M tiles over all requests: n * tiles_t
  int tiles_t;        // 128-frame tiles per request
  int N;              // output columns (a multiple of BN)
  int nkb_c;          // 32-channel blocks of the input per tap
  int taps, off0, dil;  // tap j reads frame t + off0 + j * dil
  const float* bias;  // [N]
  float* out;         // fp32 output, or null (out16 only)
  long long out_b;    // elements between requests of out (and of res, out16)
  int out_ld;         // floats between frames t of out
  int u, cp_out;      // column col of frame t is output frame t*u + col / cp_out ...
  int out_rows;       // ... stored only below out_rows
  const float* res;   // residual with out's layout, or null
  int accum;          // 1: out += value (the stage's resblock sum)
  float div;          // then out /= div (1: none)
  __half* out16;      // optional fp16 copy of out (same layout), the next conv's operand
};

DFM_DEV uint32_t pack_half(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// Inputs of the conv epilogue that do not depend on the accumulator: the
// first 32 columns of the thread's residual row and running sum, loaded
// before the accumulator wait so their latency overlaps the mainloop.
struct VcPre {
  float4 r[8], o[8];
};

DFM_DEV void voc_conv_prefetch(const VcArgs& p, int b, int f, int n0, VcPre& pre,
                               bool res = true) {
  const size_t at = static_cast<size_t>(b) * p.out_b + static_cast<size_t>(f) * p.out_ld + n0;
  if (f * p.u + n0 / p.cp_out >= p.out_rows) return;
  if (res && p.res) {
#pragma unroll
    for (int j = 0; j < 8; ++j) pre.r[j] = reinterpret_cast<const float4*>(p.res + at)[j];
  }
  if (p.accum) {
#pragma unroll
    for (int j = 0; j < 8; ++j) pre.o[j] = reinterpret_cast<const float4*>(p.out + at)[j];
  }
}

// The conv epilogue of one thread: frame f of request b, columns [n0, n0+BN)
// of the accumulator at taddr (this warp's TMEM lanes):
//   v = acc + bias (+ residual);  out = v, or (out + v) [/ div]
// ebuf (optional): this tile's residual in shared memory, BN/32 boxes of 128
// rows x 128 bytes with the 128-byte swizzle (row `row` of the tile).
template <int BN>
DFM_DEV void voc_conv_epilogue(const VcArgs& p, uint32_t taddr, int b, int f, int n0,
                               const VcPre& pre, const uint8_t* ebuf = nullptr, int row = 0) {
  const size_t rowoff = static_cast<size_t>(b) * p.out_b + static_cast<size_t>(f) * p.out_ld;
#pragma unroll 1
  for (int c = 0; c < BN; c += 32) {
    uint32_t r[32];
    tmem_ld32(taddr + c, r);
    tmem_wait_ld();
    const int col = n0 + c;
    if (f * p.u + col / p.cp_out >= p.out_rows) continue;
    float v[32];
    const float4* b4 = reinterpret_cast<const float4*>(p.bias + col);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float4 bb = __ldg(b4 + j);
      v[4 * j] = __uint_as_float(r[4 * j]) + bb.x;
      v[4 * j + 1] = __uint_as_float(r[4 * j + 1]) + bb.y;
      v[4 * j + 2] = __uint_as_float(r[4 * j + 2]) + bb.z;
      v[4 * j + 3] = __uint_as_float(r[4 * j + 3]) + bb.w;
    }
    float4* o4 = reinterpret_cast<float4*>(p.out + rowoff + col);
    if (ebuf) {
      const uint8_t* er = ebuf + (c / 32) * (VC_BM * 128) + row * 128;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float4 x = *reinterpret_cast<const float4*>(er + ((j ^ (row & 7)) << 4));
        v[4 * j] += x.x; v[4 * j + 1] += x.y; v[4 * j + 2] += x.z; v[4 * j + 3] += x.w;
      }
    } else if (p.res) {
      const float4* r4 = reinterpret_cast<const float4*>(p.res + rowoff + col);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float4 x = c == 0 ? pre.r[j] : r4[j];
        v[4 * j] += x.x; v[4 * j + 1] += x.y; v[4 * j + 2] += x.z; v[4 * j + 3] += x.w;
      }
    }
    if (p.accum) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float4 x = c == 0 ? pre.o[j] : o4[j];
        v[4 * j] = x.x + v[4 * j]; v[4 * j + 1] = x.y + v[4 * j + 1];
        v[4 * j + 2] = x.z + v[4 * j + 2]; v[4 * j + 3] = x.w + v[4 * j + 3];
      }
    }
    if (p.div != 1.0f) {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = v[j] / p.div;
    }
    if (p.out) {
#pragma unroll
      for (int j = 0; j < 8; ++j) o4[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
    }
    if (p.out16) {
      uint4* h4 = reinterpret_cast<uint4*>(p.out16 + rowoff + col);
#pragma unroll
      for (int j = 0; j < 4; ++j)
        h4[j] = make_uint4(pack_half(v[8 * j], v[8 * j + 1]), pack_half(v[8 * j + 2], v[8 * j + 3]),
                           pack_half(v[8 * j + 4], v[8 * j + 5]), pack_half(v[8 * j + 6], v[8 * j + 7]));
    }
  }
}

// Persistent: CTA b takes tiles b, b + grid, ... with the M tiles fastest, so
// CTAs working at once share W tiles in L2.  Warp 0 lane 0 loads (TMA), warp 1
// owns TMEM and issues the MMAs, warps 2..5 run the epilogue from a
// double-buffered TMEM accumulator.  Every wait is bounded.
template <int BN, int STAGES>
__global__ void __launch_bounds__(VC_THREADS, 2)
    voc_conv_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
                    VcArgs p, uint32_t* err) {
  using S = VcShape<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * S::A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * S::STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tm_full = empty + STAGES;  // [2]
  uint64_t* tm_empty = tm_full + 2;    // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tm_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int total = p.tiles_m * (p.N / BN);
  const int nk = p.taps * p.nkb_c;

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
    tma_prefetch(&tmW);
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
      // The first stages' weights do not depend on the previous kernel.
      const int pre = (static_cast<int>(blockIdx.x) < total) ? (nk < STAGES ? nk : STAGES) : 0;
      const int n00 = (blockIdx.x / p.tiles_m) * BN;
      for (int kb = 0; kb < pre; ++kb) {
        mbar_arrive_expect_tx(&full[kb], S::STAGE_BYTES);
        tma_load_2d(sB + kb * S::B_BYTES, &tmW, &full[kb], kb * VC_BK, n00);
      }
      pdl_wait();
      int g = 0;
      bool ok = true;
#pragma unroll 1
      for (int t = blockIdx.x; ok && t < total; t += gridDim.x) {
        const int m = t % p.tiles_m, n0 = (t / p.tiles_m) * BN;
        const int b = m / p.tiles_t, f0 = (m - b * p.tiles_t) * VC_BM;
        int tap = 0, cb = 0;
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
            tma_load_2d(sB + s * S::B_BYTES, &tmW, &full[s], kb * VC_BK, n0);
          }
          tma_load_3d(sA + s * S::A_BYTES, &tmA, &full[s], cb * VC_BK, f0 + p.off0 + tap * p.dil, b);
          if (++cb == p.nkb_c) {
            cb = 0;
            ++tap;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_f16(VC_BM, BN);
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
          for (int kk = 0; kk < VC_BK / 16; ++kk)  // K = 16 fp16 (32 bytes) per MMA
            umma_bf16(acc, umma_desc_sw64(a + kk * 32), umma_desc_sw64(bb + kk * 32), idesc,
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
      const int buf = u & 1;
      const int m = t % p.tiles_m, n0 = (t / p.tiles_m) * BN;
      const int b = m / p.tiles_t;
      const int f = (m - b * p.tiles_t) * VC_BM + q * 32 + lane;
      VcPre pre;
      voc_conv_prefetch(p, b, f, n0, pre);
      const bool ready =
          __all_sync(0xffffffffu, mbar_wait(&tm_full[buf], (u >> 1) & 1, abort_flag, err));
      if (!ready) break;
      tc_fence_after();
      voc_conv_epilogue<BN>(p, tmem + buf * BN + (static_cast<uint32_t>(q * 32) << 16), b, f, n0, pre);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tm_empty[buf]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, S::TMEM_COLS);
  }
}

// ---------------------------------------------------------------- conv, halo tiles
// For narrow convolutions (N <= 192) whose taps span at most 64 frames
// ((taps-1)*dil <= VH_HALO): per 32-channel block ONE A tile of 128 + halo
// frames (three 64-frame TMA boxes) serves every tap; tap j's MMA reads it
// from frame j*dil on, through a descriptor whose start address moves by
// j*dil rows of 128 bytes (the base-offset field carries the 128-byte swizzle
// phase of that start).  The weights of each (tap, block) pair stream through
// their own ring.  Same epilogue and roles as voc_conv_kernel.
constexpr int VH_HALO = 64;
constexpr int VH_ROWS = VC_BM + VH_HALO;   // frames staged per A tile
constexpr int VH_BOX = 64;                 // frames per TMA box

// MT: 128-frame accumulators per tile (a tile is MT x 128 frames; every
// barrier round of (channel block, tap) feeds MT x 2 MMAs from one A tile and
// one W tile).
// NB: accumulator buffers (2: the next tile's MMAs overlap this tile's
// epilogue; 1: they wait for it, which halves TMEM so two CTAs per SM fit).
template <int BN, int SA, int SB, int SE = 0, int MT = 1, int NB = 2>
struct VhShape {
  static_assert(BN % 32 == 0 && BN >= 32 && BN <= 256, "MMA N");
  static_assert(MT == 1 || MT == 2, "accumulators per tile");
  static constexpr int ROWS = MT * VC_BM + VH_HALO;           // frames staged per A tile
  static constexpr int A_BYTES = ROWS * VC_ROWB;               // 12 KB (MT 1) or 20 KB (MT 2)
  static constexpr int B_BYTES = BN * VC_ROWB;
  static constexpr int E_BYTES = MT * VC_BM * BN * 4;          // one tile's fp32 residual (128-byte swizzle)
  static_assert(A_BYTES % 1024 == 0 && B_BYTES % 1024 == 0, "swizzle atoms");
  static constexpr int SMEM = SA * A_BYTES + SB * B_BYTES + SE * E_BYTES + 1024 + 512;
  static_assert(SMEM <= 232448, "shared memory per CTA");
  static_assert(NB == 1 || NB == 2, "accumulator buffers");
  static constexpr int ACC_COLS = NB * MT * BN;
  static constexpr uint32_t TMEM_COLS = ACC_COLS <= 64 ? 64 : ACC_COLS <= 128 ? 128
                                        : ACC_COLS <= 256 ? 256 : 512;
};

// A row-shifted operand descriptor keeps the base-offset field 0: the MMA
// applies the swizzle to the address bits, as TMA wrote them (a start
// shifted by r rows reads rows r, r+1, ... of the tile; measured with the
// 128-byte swizzle, where setting the field to the row phase failed parity,
// and checked by the parity tests).
//
// SE > 0: the producer also loads each tile's residual rows (tmR, boxes of
// 32 channels x 128 frames) into SE shared-memory buffers while the mainloop
// runs, and the epilogue reads them there instead of from global memory.
// Tiles are ordered N fastest, so the N tiles of one M tile run on
// neighbouring CTAs at the same time and share its A rows in L2.
template <int BN, int SA, int SB, int SE, int MT, int NB>
__global__ void __launch_bounds__(VC_THREADS, 2)
    voc_conv_halo_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
                         const __grid_constant__ CUtensorMap tmR, VcArgs p, uint32_t* err) {
  using S = VhShape<BN, SA, SB, SE, MT, NB>;
  constexpr int TM = MT * VC_BM;        // frames per tile
  constexpr int SEN = SE > 0 ? SE : 1;  // residual buffers (1: none, never used)
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + SA * S::A_BYTES;
  uint8_t* sE = sB + SB * S::B_BYTES;
  uint64_t* a_full = reinterpret_cast<uint64_t*>(sE + SE * S::E_BYTES);
  uint64_t* a_empty = a_full + SA;
  uint64_t* b_full = a_empty + SA;
  uint64_t* b_empty = b_full + SB;
  uint64_t* tm_full = b_empty + SB;  // [2]
  uint64_t* tm_empty = tm_full + 2;  // [2]
  uint64_t* e_full = tm_empty + 2;   // [SE]
  uint64_t* e_empty = e_full + SEN;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(e_empty + SEN);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles_n = p.N / BN;
  const int total = p.tiles_m * tiles_n;
  const int nbox = (TM + (p.taps - 1) * p.dil + VH_BOX - 1) / VH_BOX;
  const bool eres = SE > 0 && p.res != nullptr;

  if (threadIdx.x == 0) {
    for (int s = 0; s < SA; ++s) {
      mbar_init(&a_full[s], 1);
      mbar_init(&a_empty[s], 1);
    }
    for (int s = 0; s < SB; ++s) {
      mbar_init(&b_full[s], 1);
      mbar_init(&b_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tm_full[b], 1);
      mbar_init(&tm_empty[b], 4);
    }
    for (int e = 0; e < SE; ++e) {
      mbar_init(&e_full[e], 1);
      mbar_init(&e_empty[e], 4);
    }
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch(&tmA);
    tma_prefetch(&tmW);
    if (SE > 0) tma_prefetch(&tmR);
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
      pdl_wait();
      int ga = 0, gb = 0, u = 0;
      bool ok = true;
#pragma unroll 1
      for (int t = blockIdx.x; ok && t < total; t += gridDim.x, ++u) {
        const int m = t / tiles_n, n0 = (t - m * tiles_n) * BN;
        const int b = m / p.tiles_t, f0 = (m - b * p.tiles_t) * TM;
        if (eres) {
          const int eb = u % SEN;
          if (u >= SEN && !mbar_wait(&e_empty[eb], ((u / SEN) & 1) ^ 1, abort_flag, err)) break;
          mbar_arrive_expect_tx(&e_full[eb], S::E_BYTES);
          for (int mt = 0; mt < MT; ++mt)
            for (int c = 0; c < BN / 32; ++c)
              tma_load_3d(sE + eb * S::E_BYTES + (mt * (BN / 32) + c) * VC_BM * 128, &tmR, &e_full[eb],
                          n0 + 32 * c, f0 + mt * VC_BM, b);
        }
#pragma unroll 1
        for (int cb = 0; ok && cb < p.nkb_c; ++cb, ++ga) {
          const int sa = ga % SA;
          if (ga >= SA && !mbar_wait(&a_empty[sa], ((ga / SA) & 1) ^ 1, abort_flag, err)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&a_full[sa], nbox * VH_BOX * VC_ROWB);
          for (int q = 0; q < nbox; ++q)
            tma_load_3d(sA + sa * S::A_BYTES + q * VH_BOX * VC_ROWB, &tmA, &a_full[sa], cb * VC_BK,
                        f0 + p.off0 + q * VH_BOX, b);
#pragma unroll 1
          for (int j = 0; j < p.taps; ++j, ++gb) {
            const int sb = gb % SB;
            if (gb >= SB && !mbar_wait(&b_empty[sb], ((gb / SB) & 1) ^ 1, abort_flag, err)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&b_full[sb], S::B_BYTES);
            tma_load_2d(sB + sb * S::B_BYTES, &tmW, &b_full[sb], (j * p.nkb_c + cb) * VC_BK, n0);
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_f16(VC_BM, BN);
      int ga = 0, gb = 0, u = 0;
      bool ok = true;
#pragma unroll 1
      for (int t = blockIdx.x; ok && t < total; t += gridDim.x, ++u) {
        const int buf = u % NB;
        if (u >= NB && !mbar_wait(&tm_empty[buf], ((u / NB) & 1) ^ 1, abort_flag, err)) break;
        tc_fence_after();
        const uint32_t acc = tmem + buf * MT * BN;
#pragma unroll 1
        for (int cb = 0; ok && cb < p.nkb_c; ++cb, ++ga) {
          const int sa = ga % SA;
          if (!mbar_wait(&a_full[sa], (ga / SA) & 1, abort_flag, err)) {
            ok = false;
            break;
          }
          const uint32_t a0 = smem_u32(sA + sa * S::A_BYTES);
#pragma unroll 1
          for (int j = 0; j < p.taps; ++j, ++gb) {
            const int sb = gb % SB;
            if (!mbar_wait(&b_full[sb], (gb / SB) & 1, abort_flag, err)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t bb = smem_u32(sB + sb * S::B_BYTES);
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
              const uint32_t a = a0 + static_cast<uint32_t>(mt * VC_BM + j * p.dil) * VC_ROWB;
#pragma unroll
              for (int kk = 0; kk < VC_BK / 16; ++kk)
                umma_bf16(acc + mt * BN, umma_desc_sw64(a + kk * 32), umma_desc_sw64(bb + kk * 32), idesc,
                          (cb | j | kk) != 0);
            }
            umma_commit(&b_empty[sb]);
          }
          if (ok) umma_commit(&a_empty[sa]);
        }
        if (ok) umma_commit(&tm_full[buf]);
      }
    }
  } else {
    pdl_wait();
    const int q = warp & 3;
    int u = 0;
#pragma unroll 1
    for (int t = blockIdx.x; t < total; t += gridDim.x, ++u) {
      const int buf = u % NB;
      const int m = t / tiles_n, n0 = (t - m * tiles_n) * BN;
      const int b = m / p.tiles_t;
      const int f0 = (m - b * p.tiles_t) * TM;
      VcPre pre;
      voc_conv_prefetch(p, b, f0 + q * 32 + lane, n0, pre, !eres);
      bool ready = mbar_wait(&tm_full[buf], (u / NB) & 1, abort_flag, err);
      const uint8_t* ebuf = nullptr;
      if (eres) {
        const int eb = u % SEN;
        ready = mbar_wait(&e_full[eb], (u / SEN) & 1, abort_flag, err) && ready;
        ebuf = sE + eb * S::E_BYTES;
      }
      if (!__all_sync(0xffffffffu, ready)) break;
      tc_fence_after();
#pragma unroll 1
      for (int mt = 0; mt < MT; ++mt) {
        const int row = q * 32 + lane;
        if (mt > 0) voc_conv_prefetch(p, b, f0 + mt * VC_BM + row, n0, pre, !eres);
        voc_conv_epilogue<BN>(p, tmem + (buf * MT + mt) * BN + (static_cast<uint32_t>(q * 32) << 16), b,
                              f0 + mt * VC_BM + row, n0, pre,
                              ebuf ? ebuf + mt * (BN / 32) * VC_BM * 128 : nullptr, row);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&tm_empty[buf]);
        if (eres) mbar_arrive(&e_empty[u % SEN]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, S::TMEM_COLS);
  }
}

// ---------------------------------------------------------------- activation
// Anti-aliased (Snake)Beta on [n][rows][cp] (``alias_free_act.py:43-48``,
// ``alias_free_resample.py:44-81``, causal, ratio 2, 12-tap filters):
//   u[2m+p] = 2 sum_{q<6} x[m-q] fu[2q+p]            (x[<0] = 0)
//   y = u + ib * sin(a u)^2                             (a = exp(alpha), ib = 1/(exp(beta)+1e-9))
//   out[m] = sum_{j<12} fd[j] y[max(2m+j-11, 0)]        (replicate padding on the left)
// Thread: one channel (lanes = 32 consecutive channels, coalesced rows) and
// VA_R consecutive output frames; it computes the 2 VA_R + 11 upsampled
// values those frames need from VA_R + 11 input frames.  The cost is the
// sines (two per output frame), so they use the hardware approximation.
constexpr int VA_R = 32;
constexpr int VA_WARPS = 4;

// rows must be a multiple of VA_R (every decoder tensor has a multiple of 128
// frames), so each thread's 32 outputs are all in range.
// kHalf: the output is a convolution operand (fp16); else fp32 (activation_post).
template <bool kHalf>
__global__ void __launch_bounds__(32 * VA_WARPS, 4)
    voc_act_kernel(const float* __restrict__ in, void* __restrict__ out, int rows, int cp,
                   const float* __restrict__ prm) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int c = blockIdx.x * 32 + lane;
  const int m0 = (blockIdx.y * VA_WARPS + warp) * VA_R;
  // parameters (constant) before the dependency wait; the filters as float4s
  const float a = __ldg(prm + c), ib = __ldg(prm + cp + c);
  float fu[12], fd[12];
  {
    const float4* u4 = reinterpret_cast<const float4*>(prm + 2 * cp + static_cast<size_t>(c) * 12);
    const float4* d4 = reinterpret_cast<const float4*>(prm + 14 * cp + static_cast<size_t>(c) * 12);
#pragma unroll
    for (int q = 0; q < 3; ++q) {
      const float4 uu = __ldg(u4 + q), dd = __ldg(d4 + q);
      fu[4 * q] = uu.x; fu[4 * q + 1] = uu.y; fu[4 * q + 2] = uu.z; fu[4 * q + 3] = uu.w;
      fd[4 * q] = dd.x; fd[4 * q + 1] = dd.y; fd[4 * q + 2] = dd.z; fd[4 * q + 3] = dd.w;
    }
  }
  pdl_wait();
  pdl_trigger();
  if (m0 >= rows) return;
  const float* ip = in + static_cast<size_t>(blockIdx.z) * rows * cp + c;
  float x[VA_R + 11];  // x[i] = in[m0 - 11 + i]
  if (m0 >= 11) {
    const float* p0 = ip + static_cast<size_t>(m0 - 11) * cp;
#pragma unroll
    for (int i = 0; i < VA_R + 11; ++i) {
      x[i] = *p0;
      p0 += cp;
    }
  } else {
#pragma unroll
    for (int i = 0; i < VA_R + 11; ++i) {
      const int m = m0 - 11 + i;
      x[i] = m >= 0 ? ip[static_cast<size_t>(m) * cp] : 0.0f;
    }
  }
  // y[i] = act(u[2 m0 - 11 + i]); q = 2 m0 - 11 + i = 2 mm + ph with
  // ph = (i + 1) & 1, and x[mm] is window entry (i - 11 - ph) / 2 + 11.  Each
  // output needs y[2k .. 2k+11]: the first 12 are computed up front, then two
  // more per output, so only a sliding window of y stays live.
  float y[2 * VA_R + 11];
  auto act = [&](int i) {
    const int ph = (i + 1) & 1;
    const int xi = (i - 11 - ph) / 2 + 11;
    float s = 0.0f;
#pragma unroll
    for (int qq = 0; qq < 6; ++qq) s += x[xi - qq] * fu[2 * qq + ph];
    const float uu = 2.0f * s;
    // the MUFU sine: absolute error ~1e-6 for the arguments seen here, far
    // below the fp16 rounding of the convolution operands
    const float sn = __sinf(uu * a);
    return uu + ib * (sn * sn);
  };
#pragma unroll
  for (int i = 0; i < 12; ++i) y[i] = act(i);
  if (m0 == 0) {  // frames before the first: the first upsampled value (q = 0 is i = 11)
#pragma unroll
    for (int i = 0; i < 11; ++i) y[i] = y[11];
  }
  const size_t o0 = static_cast<size_t>(blockIdx.z) * rows * cp + c + static_cast<size_t>(m0) * cp;
  __half* oh = static_cast<__half*>(out) + o0;
  float* of = static_cast<float*>(out) + o0;
#pragma unroll
  for (int k = 0; k < VA_R; ++k) {
    if (k > 0) {
      y[2 * k + 10] = act(2 * k + 10);
      y[2 * k + 11] = act(2 * k + 11);
    }
    float o = 0.0f;
#pragma unroll
    for (int j = 0; j < 12; ++j) o += fd[j] * y[2 * k + j];
    if constexpr (kHalf) {
      *oh = __float2half_rn(o);
      oh += cp;
    } else {
      *of = o;
      of += cp;
    }
  }
}

// The resblock activations (fixed filters, the same for every channel:
// ``Activation1d(..., fixed_filter=True)``, ``bigvgan.py:339-346``), two
// channels per thread on paired fp32 arithmetic (FFMA2): lanes 0-15 take the
// 32-channel block's channel pairs for frames [m0, m0+16), lanes 16-31 the
// same pairs for [m0+16, m0+32).  Same arithmetic as voc_act_kernel, with
// the upsampling filter pre-scaled by 2 (exact).  Input fp32 (the residual
// stream) or fp16 (a conv1 output); output fp16 (the next conv's operand).
constexpr int VB_R = 16;

DFM_DEV float2 ld2(const float* p) { return *reinterpret_cast<const float2*>(p); }
DFM_DEV float2 ld2(const __half* p) { return __half22float2(*reinterpret_cast<const __half2*>(p)); }

template <typename Tin>
__global__ void __launch_bounds__(32 * VA_WARPS, 4)
    voc_act2_kernel(const Tin* __restrict__ in, __half* __restrict__ out, int rows, int cp,
                    const float* __restrict__ prm) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int c = blockIdx.x * 32 + 2 * (lane & 15);
  const int m0 = ((blockIdx.y * VA_WARPS + warp) * 2 + (lane >> 4)) * VB_R;
  const float2 a = ld2(prm + c), ib = ld2(prm + cp + c);
  float fu[12], fd[12];
  {
    const float4* u4 = reinterpret_cast<const float4*>(prm + 2 * cp);   // channel 0's filters
    const float4* d4 = reinterpret_cast<const float4*>(prm + 14 * cp);
#pragma unroll
    for (int q = 0; q < 3; ++q) {
      const float4 uu = __ldg(u4 + q), dd = __ldg(d4 + q);
      fu[4 * q] = 2.0f * uu.x; fu[4 * q + 1] = 2.0f * uu.y; fu[4 * q + 2] = 2.0f * uu.z; fu[4 * q + 3] = 2.0f * uu.w;
      fd[4 * q] = dd.x; fd[4 * q + 1] = dd.y; fd[4 * q + 2] = dd.z; fd[4 * q + 3] = dd.w;
    }
  }
  pdl_wait();
  pdl_trigger();
  if (m0 >= rows) return;
  const Tin* ip = in + static_cast<size_t>(blockIdx.z) * rows * cp + c;
  float2 x[VB_R + 11];  // x[i] = in[m0 - 11 + i]
  if (m0 >= 11) {
    const Tin* p0 = ip + static_cast<size_t>(m0 - 11) * cp;
#pragma unroll
    for (int i = 0; i < VB_R + 11; ++i) {
      x[i] = ld2(p0);
      p0 += cp;
    }
  } else {
#pragma unroll
    for (int i = 0; i < VB_R + 11; ++i) {
      const int m = m0 - 11 + i;
      x[i] = m >= 0 ? ld2(ip + static_cast<size_t>(m) * cp) : make_float2(0.f, 0.f);
    }
  }
  float2 y[2 * VB_R + 11];
  auto act = [&](int i) {
    const int ph = (i + 1) & 1;
    const int xi = (i - 11 - ph) / 2 + 11;
    float2 s = make_float2(0.f, 0.f);
#pragma unroll
    for (int qq = 0; qq < 6; ++qq) {
      const float f = fu[2 * qq + ph];
      s = __ffma2_rn(x[xi - qq], make_float2(f, f), s);
    }
    const float2 t = __fmul2_rn(s, a);
    const float2 sn = make_float2(__sinf(t.x), __sinf(t.y));
    return __ffma2_rn(ib, __fmul2_rn(sn, sn), s);
  };
#pragma unroll
  for (int i = 0; i < 12; ++i) y[i] = act(i);
  if (m0 == 0) {
#pragma unroll
    for (int i = 0; i < 11; ++i) y[i] = y[11];
  }
  __half* op = out + static_cast<size_t>(blockIdx.z) * rows * cp + c + static_cast<size_t>(m0) * cp;
#pragma unroll
  for (int k = 0; k < VB_R; ++k) {
    if (k > 0) {
      y[2 * k + 10] = act(2 * k + 10);
      y[2 * k + 11] = act(2 * k + 11);
    }
    float2 o = make_float2(0.f, 0.f);
#pragma unroll
    for (int j = 0; j < 12; ++j) o = __ffma2_rn(make_float2(fd[j], fd[j]), y[2 * k + j], o);
    *reinterpret_cast<__half2*>(op) = __floats2half2_rn(o.x, o.y);
    op += cp;
  }
}

// ---------------------------------------------------------------- conv_post
// audio[b][t] = act(bias + sum_{j<7} sum_c w[j][c] a[b][t-6+j][c]) for t < n_out
// (a holds `rows` frames per request);
// act = tanh or clamp to [-1, 1] (``bigvgan.py:632-638``).  A block computes
// 256 frames from a shared-memory tile of 262 frames x 32 channels per pass.
constexpr int VP_T = 256;

__global__ void __launch_bounds__(VP_T)
    voc_post_kernel(const float* __restrict__ a, float* __restrict__ audio, int rows, int cp,
                    int n_out, long long audio_b, const float* __restrict__ w, const float* __restrict__ bias,
                    int use_tanh) {
  __shared__ float tile[VP_T + 6][33];
  const int t0 = blockIdx.x * VP_T, t = t0 + threadIdx.x;
  const size_t base = static_cast<size_t>(blockIdx.y) * rows * cp;
  const float b0 = bias ? __ldg(bias) : 0.0f;
  pdl_wait();
  pdl_trigger();
  float acc = 0.0f;
#pragma unroll 1
  for (int c0 = 0; c0 < cp; c0 += 32) {
    __syncthreads();
#pragma unroll 8   // independent loads: eight in flight per thread
    for (int i = threadIdx.x; i < (VP_T + 6) * 32; i += VP_T) {
      const int r = i >> 5, cc = i & 31;
      const int f = t0 - 6 + r;
      tile[r][cc] = (f >= 0 && f < rows) ? a[base + static_cast<size_t>(f) * cp + c0 + cc] : 0.0f;
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < 7; ++j) {
      const float* wj = w + static_cast<size_t>(j) * cp + c0;
#pragma unroll 8
      for (int cc = 0; cc < 32; ++cc) acc += __ldg(wj + cc) * tile[threadIdx.x + j][cc];
    }
  }
  if (t < n_out) {
    const float v = acc + b0;
    audio[static_cast<size_t>(blockIdx.y) * audio_b + t] =
        use_tanh ? tanhf(v) : fminf(fmaxf(v, -1.0f), 1.0f);
  }
}

// ---------------------------------------------------------------- front
// Y[orow(r)][j] = (b1[j] + sum_k X[r][k] W[j][k]) for r < M, j < N, with
// orow(r) = (r / rpg) * ostride + r % rpg.  64 x 64 output tiles, 4 x 4 per
// thread, fp32 FMA (the reference's fp32 nn.Linear).
constexpr int VL_T = 64, VL_K = 16;

__global__ void __launch_bounds__(256)
    voc_linear_kernel(const float* __restrict__ X, int ldx, const float* __restrict__ W,
                      const float* __restrict__ b1, float* __restrict__ Y, int ldy, int M, int N,
                      int K, int rpg, int ostride) {
  __shared__ float xs[VL_K][VL_T + 4];
  __shared__ float ws[VL_K][VL_T + 4];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int r0 = blockIdx.y * VL_T, j0 = blockIdx.x * VL_T;
  pdl_wait();
  pdl_trigger();
  float acc[4][4] = {};
#pragma unroll 1
  for (int k0 = 0; k0 < K; k0 += VL_K) {
#pragma unroll
    for (int i = threadIdx.x; i < VL_K * VL_T; i += 256) {
      const int rr = i / VL_K, kk = i % VL_K;
      const int r = r0 + rr, j = j0 + rr, k = k0 + kk;
      xs[kk][rr] = (r < M && k < K) ? X[static_cast<size_t>(r) * ldx + k] : 0.0f;
      ws[kk][rr] = (j < N && k < K) ? __ldg(W + static_cast<size_t>(j) * K + k) : 0.0f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < VL_K; ++kk) {
      float xv[4], wv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        xv[i] = xs[kk][ty * 4 + i];
        wv[i] = ws[kk][tx * 4 + i];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) acc[i][jj] += xv[i] * wv[jj];
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = r0 + ty * 4 + i;
    if (r >= M) continue;
    const size_t orow = static_cast<size_t>(r / rpg) * ostride + r % rpg;
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
      const int j = j0 + tx * 4 + jj;
      if (j < N) Y[orow * ldy + j] = acc[i][jj] + __ldg(b1 + j);
    }
  }
}

// One frame f of one LSTM layer for n requests (``SLSTM.stream_step``,
// ``bigvgan.py:170-214``; gate order i, f, g, o):
//   gates = (W_hh h_prev + b_hh) + gx[b][f]   (gx = W_ih x + b_ih)
//   c = sig(f) c + sig(i) tanh(g);  h = sig(o) tanh(c)
// h goes to h_next and to y[b][f] (plus skip[b][f] at the last layer).  A
// block takes 8 hidden units (one per warp) for 32 requests (one per lane):
// the 32 requests' h_prev sit transposed in shared memory, and the block's
// 32 rows of W_hh (4 gates x 8 units) are staged there too, so the inner
// loop reads only shared memory.
constexpr int VS_J = 8;

__global__ void __launch_bounds__(32 * VS_J)
    voc_lstm_step_kernel(const float* __restrict__ gx, int F, int f, const float* __restrict__ whh,
                         const float* __restrict__ bhh, const float* __restrict__ h_prev,
                         float* __restrict__ h_next, float* __restrict__ c, float* __restrict__ y,
                         const float* __restrict__ skip, int n, int Hm) {
  extern __shared__ float sm[];
  float* hs = sm;                  // [Hm][33]: h_prev of the block's 32 requests, transposed
  float* ws = sm + Hm * 33;        // [4][VS_J][Hm]: this block's rows of W_hh
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int j0 = blockIdx.x * VS_J, j = j0 + warp;
  const int b0 = blockIdx.y * 32, b = b0 + lane;
  // the weights are constant: stage them before the dependency wait
  for (int i = threadIdx.x * 4; i < 4 * VS_J * Hm; i += 32 * VS_J * 4) {
    const int row = i / Hm, k = i - row * Hm;          // row = g * VS_J + u
    const int g = row / VS_J, u = row - g * VS_J;
    *reinterpret_cast<float4*>(ws + i) =
        __ldg(reinterpret_cast<const float4*>(whh + (static_cast<size_t>(g) * Hm + j0 + u) * Hm + k));
  }
  pdl_wait();
  pdl_trigger();
  // h_prev of the 32 requests, 16 bytes per load and eight loads in flight
  // per thread (Hm is a multiple of 4); a misaligned state pointer takes
  // scalar loads
  if ((reinterpret_cast<uintptr_t>(h_prev) & 15) == 0) {
#pragma unroll 8
    for (int i = threadIdx.x * 4; i < 32 * Hm; i += 32 * VS_J * 4) {
      const int bl = i / Hm, k = i - bl * Hm;
      const float4 v = (b0 + bl < n)
                           ? __ldcg(reinterpret_cast<const float4*>(h_prev + static_cast<size_t>(b0 + bl) * Hm + k))
                           : make_float4(0.f, 0.f, 0.f, 0.f);
      hs[k * 33 + bl] = v.x;
      hs[(k + 1) * 33 + bl] = v.y;
      hs[(k + 2) * 33 + bl] = v.z;
      hs[(k + 3) * 33 + bl] = v.w;
    }
  } else {
#pragma unroll 8
    for (int i = threadIdx.x; i < 32 * Hm; i += 32 * VS_J) {
      const int bl = i / Hm, k = i - bl * Hm;
      hs[k * 33 + bl] = (b0 + bl < n) ? h_prev[static_cast<size_t>(b0 + bl) * Hm + k] : 0.0f;
    }
  }
  __syncthreads();
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
  for (int k = 0; k < Hm; k += 4) {
    float hv[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) hv[e] = hs[(k + e) * 33 + lane];
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      const float4 wv = *reinterpret_cast<const float4*>(ws + (g * VS_J + warp) * Hm + k);
      acc[g] += wv.x * hv[0];
      acc[g] += wv.y * hv[1];
      acc[g] += wv.z * hv[2];
      acc[g] += wv.w * hv[3];
    }
  }
  if (b >= n || j >= Hm) return;
  const float* gxr = gx + (static_cast<size_t>(b) * F + f) * 4 * Hm;
  float gate[4];
#pragma unroll
  for (int g = 0; g < 4; ++g) gate[g] = (acc[g] + __ldg(bhh + g * Hm + j)) + gxr[g * Hm + j];
  const float ig = 1.0f / (1.0f + expf(-gate[0]));
  const float fg = 1.0f / (1.0f + expf(-gate[1]));
  const float cg = tanhf(gate[2]);
  const float og = 1.0f / (1.0f + expf(-gate[3]));
  const size_t si = static_cast<size_t>(b) * Hm + j;
  const float cn = fg * c[si] + ig * cg;
  const float hn = og * tanhf(cn);
  c[si] = cn;
  h_next[si] = hn;
  const size_t yi = (static_cast<size_t>(b) * F + f) * Hm + j;
  y[yi] = skip ? hn + skip[yi] : hn;
}

// The decoder input [n][rows][lp] (``bigvgan.py:887-928`` for streams):
//   window > 0: the window after appending z[b] (F frames) behind valid[b]
//               frames (valid clamped to [0, W]); when the frames overflow W
//               the window keeps the last W; zeros past the valid frames;
//   window == 0: z[b][p] for p < len[b] (F when len is null), zeros elsewhere.
// Rows past W (or the length) and channels past L are zero.  dst is the
// fp16 operand of conv_pre; dst32 (optional) an fp32 copy for the window store.
__global__ void voc_pack_kernel(const float* __restrict__ z, const float* __restrict__ win,
                                const int* __restrict__ valid, const int* __restrict__ len,
                                __half* __restrict__ dst, float* __restrict__ dst32, int n, int F,
                                int W, int L, int lp, int rows) {
  pdl_wait();
  pdl_trigger();
  const size_t total = static_cast<size_t>(n) * rows * lp;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(i % lp);
    const size_t bp = i / lp;
    const int p = static_cast<int>(bp % rows), b = static_cast<int>(bp / rows);
    float v = 0.0f;
    if (c < L) {
      if (W > 0) {
        int vb = valid[b];
        vb = vb < 0 ? 0 : (vb > W ? W : vb);
        const int nv = vb + F < W ? vb + F : W;
        const int s = vb + F - W > 0 ? vb + F - W : 0;
        if (p < nv) {
          const int q = p + s;
          v = q < vb ? win[(static_cast<size_t>(b) * W + q) * L + c]
                     : z[(static_cast<size_t>(b) * F + (q - vb)) * L + c];
        }
      } else {
        const int lb = len ? len[b] : F;
        if (p < lb && p < F) v = z[(static_cast<size_t>(b) * F + p) * L + c];
      }
    }
    dst[i] = __float2half_rn(v);
    if (dst32) dst32[i] = v;
  }
}

// windows[b][p][c] = dinput[b][p][c] for p < W, c < L (the new stream windows,
// from the fp32 copy of the decoder input).
__global__ void voc_window_store_kernel(const float* __restrict__ din, float* __restrict__ win,
                                        int n, int W, int L, int lp, int rows) {
  pdl_wait();
  pdl_trigger();
  const size_t total = static_cast<size_t>(n) * W * L;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(i % L);
    const size_t bp = i / L;
    const int p = static_cast<int>(bp % W), b = static_cast<int>(bp / W);
    win[i] = din[(static_cast<size_t>(b) * rows + p) * lp + c];
  }
}

// dst[i] = src[i] (the LSTM state hand-back).
__global__ void voc_copy_kernel(const float* __restrict__ src, float* __restrict__ dst, size_t count) {
  pdl_wait();
  pdl_trigger();
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < count;
       i += static_cast<size_t>(gridDim.x) * blockDim.x)
    dst[i] = src[i];
}

}  // namespace dfm
