// Paged varlen attention of the FM head: each request's 34 query rows (17
// graduating + 17 active) over its own per-(layer, step) K/V prefix, which
// lives in 16-row pages of the pool.
//
// Semantics (the prefix-cache mask of the reference's cached FM head):
//   graduating row j (j < n_ext): keys [0, P + j + 1)   causal within the new rows
//   every other row:              keys [0, P + n_ext + 17)
// where P is the request's cache length before this tick.
//
// Pool layout: [plane][page][head][16 rows][64] bf16, plane = (layer*nfe +
// step)*2 + {0: K, 1: V}.  A (page, head) block is 2 KB contiguous; it is
// fetched with one TMA box {64, 16, 1, 1, 1} under the 128-byte swizzle.
//
// Work unit: (request, chunk of ATT_CH keys, head).  Warps 0..2 hold 16 query
// rows each (rows 34..47 are padding) and run bf16 mma.sync m16n8k16 with an
// online softmax in the exp2 domain; warp 3 is the TMA producer of a 4-stage
// ring of 64-key K and V tiles.  A request that fits in one chunk writes its
// normalised output directly; longer ones write (O, m, l) partials and the
// last chunk CTA of each (request, head), found with a completion counter,
// merges them.
#pragma once

#include "common.cuh"

namespace dfm {

constexpr int ATT_KT = 64;       // keys per tile
constexpr int ATT_STAGES = 3;
constexpr int ATT_CH = 1024;     // target keys per work unit (a request's keys are split
                                 // into ceil(total / ATT_CH) equal chunks of whole tiles)
constexpr int ATT_ROWS = 34;     // query rows per request
constexpr int ATT_THREADS = 128;
constexpr int ATT_TILE_BYTES = ATT_KT * 64 * 2;  // 8 KB per K (or V) tile
constexpr int ATT_SMEM = ATT_STAGES * 2 * ATT_TILE_BYTES + 1024 + 256;

struct AttnParams {
  const __nv_bfloat16* q;    // [n*34, H]
  __nv_bfloat16* out;        // [n*34, H]
  float* part_o;             // [n*MC*heads][34][64]
  float* part_ml;            // [n*MC*heads][34][2]
  int* sem;                  // [n*heads] chunk-completion counters (zero between launches)
  const int* cache_len;
  const int* n_ext;
  const int* block_table;
  int n, max_pages, num_pages, heads, H, MC;
  int plane_k, plane_v;
  int ext_slots;             // 17
  uint32_t* err;
};

DFM_DEV void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
DFM_DEV void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
DFM_DEV void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Byte offset of (row, 16-byte chunk) in a tile of 128-byte rows under the
// 128-byte TMA swizzle (chunk index XOR row mod 8).
DFM_DEV uint32_t sw128(int row, int chunk) {
  return static_cast<uint32_t>(row * 128 + ((chunk ^ (row & 7)) << 4));
}

__global__ void __launch_bounds__(ATT_THREADS, 4)
    attn_kernel(const __grid_constant__ CUtensorMap tm_pool, AttnParams p) {
  const int i = blockIdx.x / p.MC;
  const int c = blockIdx.x - i * p.MC;
  const int h = blockIdx.y;
  pdl_trigger();
  if (threadIdx.x == 0) tma_prefetch(&tm_pool);
  pdl_wait();
  if (i >= p.n) return;
  const int P = p.cache_len[i];
  const int ne = p.n_ext[i];
  const int total = P + ne + (ATT_ROWS - p.ext_slots);
  if (P < 0 || ne < 0 || ne > p.ext_slots || total > p.max_pages * 16) {
    if (c == 0 && h == 0 && threadIdx.x == 0) atomicOr(p.err, DFM_DEV_ERR_LEN);
    return;
  }
  const int nchunks = (total + ATT_CH - 1) / ATT_CH;
  if (c >= nchunks || nchunks > p.MC) return;
  const int tiles_all = (total + ATT_KT - 1) / ATT_KT;
  const int tiles_per = (tiles_all + nchunks - 1) / nchunks;
  const int k0 = c * tiles_per * ATT_KT;
  const int k1 = min(total, k0 + tiles_per * ATT_KT);
  const int ntiles = k1 > k0 ? (k1 - k0 + ATT_KT - 1) / ATT_KT : 0;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sK = smem;
  uint8_t* sV = smem + ATT_STAGES * ATT_TILE_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + 2 * ATT_STAGES * ATT_TILE_BYTES);
  uint64_t* empty = full + ATT_STAGES;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + ATT_STAGES);
  volatile int* last_flag = abort_flag + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < ATT_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 3);
    }
    *abort_flag = 0;
    *last_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();

  const size_t unit = (static_cast<size_t>(i) * p.MC + c) * p.heads + h;
  if (warp == 3) {
    // ------------------------------------------------------ TMA producer
    if (lane == 0) {
      const int* bt = p.block_table + static_cast<size_t>(i) * p.max_pages;
#pragma unroll 1
      for (int t = 0; t < ntiles; ++t) {
        const int s = t % ATT_STAGES;
        const uint32_t ph = (t / ATT_STAGES) & 1;
        if (t >= ATT_STAGES && !mbar_wait(&empty[s], ph ^ 1, abort_flag, p.err)) break;
        mbar_arrive_expect_tx(&full[s], 2 * ATT_TILE_BYTES);
#pragma unroll
        for (int pg = 0; pg < ATT_KT / 16; ++pg) {
          const int key = k0 + t * ATT_KT + pg * 16;
          // Pages past the request's keys, or invalid table entries, load from
          // an out-of-range page index so TMA fills the box with zeros.
          int page = p.num_pages;
          if (key < total) {
            const int pidx = key >> 4;
            const int e = pidx < p.max_pages ? bt[pidx] : -1;
            if (e >= 0 && e < p.num_pages) page = e;
            else atomicOr(p.err, DFM_DEV_ERR_PAGE);
          }
          tma_load_5d(sK + s * ATT_TILE_BYTES + pg * 2048, &tm_pool, &full[s], 0, 0, h, page,
                      p.plane_k);
          tma_load_5d(sV + s * ATT_TILE_BYTES + pg * 2048, &tm_pool, &full[s], 0, 0, h, page,
                      p.plane_v);
        }
      }
    }
  } else {
    // ------------------------------------------------------ compute warps
    const int g = lane >> 2, tq = lane & 3;
    const int r_lo = warp * 16 + g, r_hi = r_lo + 8;
    const int lim_lo = r_lo < ne ? P + r_lo + 1 : total;
    const int lim_hi = r_hi < ne ? P + r_hi + 1 : total;
    const float cexp = 0.125f * 1.4426950408889634f;  // 1/sqrt(64) * log2(e)

    uint32_t qa[4][4];
    {
      const __nv_bfloat16* qb = p.q + static_cast<size_t>(i) * ATT_ROWS * p.H + h * 64;
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        const int d0 = ks * 16 + tq * 2;
        auto ld = [&](int r, int d) -> uint32_t {
          if (r >= ATT_ROWS) return 0u;
          return *reinterpret_cast<const uint32_t*>(qb + static_cast<size_t>(r) * p.H + d);
        };
        qa[ks][0] = ld(r_lo, d0);
        qa[ks][1] = ld(r_hi, d0);
        qa[ks][2] = ld(r_lo, d0 + 8);
        qa[ks][3] = ld(r_hi, d0 + 8);
      }
    }

    float o[8][4];
#pragma unroll
    for (int a = 0; a < 8; ++a) o[a][0] = o[a][1] = o[a][2] = o[a][3] = 0.f;
    float m_lo = -INFINITY, m_hi = -INFINITY, l_lo = 0.f, l_hi = 0.f;

    // S = Q K^T of one 64-key tile (raw scores, fp32)
    auto qk = [&](uint32_t kbase, float (&sc)[8][4]) {
#pragma unroll
      for (int a = 0; a < 8; ++a) sc[a][0] = sc[a][1] = sc[a][2] = sc[a][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
#pragma unroll
        for (int nb = 0; nb < 8; nb += 2) {
          const int j = lane >> 3, rr = lane & 7;
          const int key = (nb + (j >> 1)) * 8 + rr;
          const int chunk = 2 * ks + (j & 1);
          uint32_t b0, b1, b2, b3;
          ldsm_x4(kbase + sw128(key, chunk), b0, b1, b2, b3);
          mma_bf16_16816(sc[nb], qa[ks], b0, b1);
          mma_bf16_16816(sc[nb + 1], qa[ks], b2, b3);
        }
      }
    };
    auto wait_tile = [&](int t) {
      return __all_sync(0xffffffffu, mbar_wait(&full[t % ATT_STAGES], (t / ATT_STAGES) & 1,
                                               abort_flag, p.err));
    };

    // Software pipeline: the QK^T of tile t+1 is issued before the PV of tile
    // t, so a warp always has independent tensor work while its softmax runs.
    float sc[8][4];
    bool ok = ntiles > 0 && wait_tile(0);
    if (ok) qk(smem_u32(sK), sc);
#pragma unroll 1
    for (int t = 0; ok && t < ntiles; ++t) {
      const int s = t % ATT_STAGES;
      const int kb = k0 + t * ATT_KT;
      // mask (only tiles reaching past the cached prefix need it), running max
      if (kb + ATT_KT > P) {
#pragma unroll
        for (int nb = 0; nb < 8; ++nb) {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int key = kb + nb * 8 + tq * 2 + (e & 1);
            if (key >= (e < 2 ? lim_lo : lim_hi)) sc[nb][e] = -INFINITY;
          }
        }
      }
      float mx_lo = -INFINITY, mx_hi = -INFINITY;
#pragma unroll
      for (int nb = 0; nb < 8; ++nb) {
        mx_lo = fmaxf(mx_lo, fmaxf(sc[nb][0], sc[nb][1]));
        mx_hi = fmaxf(mx_hi, fmaxf(sc[nb][2], sc[nb][3]));
      }
      mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffffu, mx_lo, 1));
      mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffffu, mx_lo, 2));
      mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffffu, mx_hi, 1));
      mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffffu, mx_hi, 2));
      const float mn_lo = fmaxf(m_lo, mx_lo), mn_hi = fmaxf(m_hi, mx_hi);
      // rescale the running sums only when some row's max moved
      if (!__all_sync(0xffffffffu, mn_lo == m_lo && mn_hi == m_hi)) {
        const float al_lo = mn_lo == -INFINITY ? 1.f : exp2f((m_lo - mn_lo) * cexp);
        const float al_hi = mn_hi == -INFINITY ? 1.f : exp2f((m_hi - mn_hi) * cexp);
        l_lo *= al_lo;
        l_hi *= al_hi;
#pragma unroll
        for (int a = 0; a < 8; ++a) {
          o[a][0] *= al_lo; o[a][1] *= al_lo;
          o[a][2] *= al_hi; o[a][3] *= al_hi;
        }
        m_lo = mn_lo;
        m_hi = mn_hi;
      }
      const float ms_lo = (m_lo == -INFINITY ? 0.f : m_lo) * cexp;
      const float ms_hi = (m_hi == -INFINITY ? 0.f : m_hi) * cexp;
      uint32_t pa[4][4];
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        float e[2][4];
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const int nb = 2 * kk + hh;
          e[hh][0] = exp2f(fmaf(sc[nb][0], cexp, -ms_lo));
          e[hh][1] = exp2f(fmaf(sc[nb][1], cexp, -ms_lo));
          e[hh][2] = exp2f(fmaf(sc[nb][2], cexp, -ms_hi));
          e[hh][3] = exp2f(fmaf(sc[nb][3], cexp, -ms_hi));
          l_lo += e[hh][0] + e[hh][1];
          l_hi += e[hh][2] + e[hh][3];
        }
        pa[kk][0] = pack_bf16(e[0][0], e[0][1]);
        pa[kk][1] = pack_bf16(e[0][2], e[0][3]);
        pa[kk][2] = pack_bf16(e[1][0], e[1][1]);
        pa[kk][3] = pack_bf16(e[1][2], e[1][3]);
      }
      // next tile's scores
      if (t + 1 < ntiles) {
        ok = wait_tile(t + 1);
        if (ok) qk(smem_u32(sK + ((t + 1) % ATT_STAGES) * ATT_TILE_BYTES), sc);
      }
      // O += P V
      const uint32_t vbase = smem_u32(sV + s * ATT_TILE_BYTES);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
        for (int db = 0; db < 8; db += 2) {
          const int j = lane >> 3, rr = lane & 7;
          const int key = kk * 16 + (j & 1) * 8 + rr;
          const int chunk = db + (j >> 1);
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(vbase + sw128(key, chunk), b0, b1, b2, b3);
          mma_bf16_16816(o[db], pa[kk], b0, b1);
          mma_bf16_16816(o[db + 1], pa[kk], b2, b3);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }

    l_lo += __shfl_xor_sync(0xffffffffu, l_lo, 1);
    l_lo += __shfl_xor_sync(0xffffffffu, l_lo, 2);
    l_hi += __shfl_xor_sync(0xffffffffu, l_hi, 1);
    l_hi += __shfl_xor_sync(0xffffffffu, l_hi, 2);

    if (nchunks == 1) {
      const float il_lo = l_lo > 0.f ? 1.f / l_lo : 0.f;
      const float il_hi = l_hi > 0.f ? 1.f / l_hi : 0.f;
      __nv_bfloat16* ob = p.out + static_cast<size_t>(i) * ATT_ROWS * p.H + h * 64;
#pragma unroll
      for (int db = 0; db < 8; ++db) {
        const int d = db * 8 + tq * 2;
        if (r_lo < ATT_ROWS)
          *reinterpret_cast<uint32_t*>(ob + static_cast<size_t>(r_lo) * p.H + d) =
              pack_bf16(o[db][0] * il_lo, o[db][1] * il_lo);
        if (r_hi < ATT_ROWS)
          *reinterpret_cast<uint32_t*>(ob + static_cast<size_t>(r_hi) * p.H + d) =
              pack_bf16(o[db][2] * il_hi, o[db][3] * il_hi);
      }
    } else {
      float* po = p.part_o + unit * ATT_ROWS * 64;
      float* pml = p.part_ml + unit * ATT_ROWS * 2;
#pragma unroll
      for (int db = 0; db < 8; ++db) {
        const int d = db * 8 + tq * 2;
        if (r_lo < ATT_ROWS)
          *reinterpret_cast<float2*>(po + r_lo * 64 + d) = make_float2(o[db][0], o[db][1]);
        if (r_hi < ATT_ROWS)
          *reinterpret_cast<float2*>(po + r_hi * 64 + d) = make_float2(o[db][2], o[db][3]);
      }
      if (tq == 0) {
        // m in the exp2 domain
        const float e_lo = m_lo == -INFINITY ? -INFINITY : m_lo * cexp;
        const float e_hi = m_hi == -INFINITY ? -INFINITY : m_hi * cexp;
        if (r_lo < ATT_ROWS) *reinterpret_cast<float2*>(pml + r_lo * 2) = make_float2(e_lo, l_lo);
        if (r_hi < ATT_ROWS) *reinterpret_cast<float2*>(pml + r_hi * 2) = make_float2(e_hi, l_hi);
      }
      __threadfence();
    }
  }

  if (nchunks == 1) return;   // CTA-uniform
  // ---------------------------------------------------------- split-key merge
  // The last chunk of (request, head) to finish merges every chunk's partial.
  __syncthreads();
  if (threadIdx.x == 0) {
    int* cnt = p.sem + static_cast<size_t>(i) * p.heads + h;
    const int prev = atomicAdd(cnt, 1);
    if (prev == nchunks - 1) {
      atomicExch(cnt, 0);
      *last_flag = 1;
    }
  }
  __syncthreads();
  if (!*last_flag) return;
  __threadfence();
  const size_t base = (static_cast<size_t>(i) * p.MC) * p.heads + h;
  for (int w = threadIdx.x; w < ATT_ROWS * 4; w += ATT_THREADS) {
    const int r = w >> 2, seg = (w & 3) * 16;
    float M = -INFINITY;
    for (int cc = 0; cc < nchunks; ++cc)
      M = fmaxf(M, p.part_ml[((base + static_cast<size_t>(cc) * p.heads) * ATT_ROWS + r) * 2]);
    float L = 0.f, acc[16];
#pragma unroll
    for (int d = 0; d < 16; ++d) acc[d] = 0.f;
    for (int cc = 0; cc < nchunks; ++cc) {
      const size_t u2 = base + static_cast<size_t>(cc) * p.heads;
      const float2 ml = *reinterpret_cast<const float2*>(p.part_ml + (u2 * ATT_ROWS + r) * 2);
      const float wgt = ml.x == -INFINITY ? 0.f : exp2f(ml.x - M);
      L += wgt * ml.y;
      const float4* src = reinterpret_cast<const float4*>(p.part_o + (u2 * ATT_ROWS + r) * 64 + seg);
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) {
        const float4 v = src[q4];
        acc[4 * q4] += wgt * v.x; acc[4 * q4 + 1] += wgt * v.y;
        acc[4 * q4 + 2] += wgt * v.z; acc[4 * q4 + 3] += wgt * v.w;
      }
    }
    const float il = L > 0.f ? 1.f / L : 0.f;
    uint4* dst = reinterpret_cast<uint4*>(p.out + (static_cast<size_t>(i) * ATT_ROWS + r) * p.H +
                                          h * 64 + seg);
    dst[0] = make_uint4(pack_bf16(acc[0] * il, acc[1] * il), pack_bf16(acc[2] * il, acc[3] * il),
                        pack_bf16(acc[4] * il, acc[5] * il), pack_bf16(acc[6] * il, acc[7] * il));
    dst[1] = make_uint4(pack_bf16(acc[8] * il, acc[9] * il), pack_bf16(acc[10] * il, acc[11] * il),
                        pack_bf16(acc[12] * il, acc[13] * il), pack_bf16(acc[14] * il, acc[15] * il));
  }
}

}  // namespace dfm
