// Paged prefix attention of the FM head on the tcgen05 tensor cores.
//
// Semantics (the prefix-cache mask of the reference's cached FM head,
// ``cached_fm.py:124-197``), per request with cache length P and n_ext
// graduating rows:
//   graduating row j (j < n_ext): keys [0, P + j + 1)
//   every other row:              keys [0, P + n_ext + 17)
// softmax(q k^T / 8) v in fp32 with bf16 operands.
//
// Work unit: one CTA per (request, chunk of up to 4096 keys, head), 192 threads:
//   warp 0     TMA: the 34 query rows (one 48-row box); per 128-key tile, 8 K
//              boxes and 8 V boxes (one 2 KB box per page, issued by 8 lanes)
//              into separate 2-deep K and V rings
//   warp 1     TMEM owner and the single MMA-issuing thread:
//                S^T[128 keys x 48 queries] = K . Q^T   (M=128, N=48, K=64)
//                O[128 x 64]               += P . V     (M=128, N=64, K=128, V MN-major)
//              each issued as soon as its own inputs are ready (polling)
//   warps 2-5  softmax: thread = one key row of S^T (TMEM lane); exponentials
//              against a running max per query, re-reduced across the 128 rows
//              only on the first tile or when a score exceeds it by 2^16;
//              probabilities written to shared memory as the bf16 A operand of
//              the PV product (MN-major: each thread stores its key row's 34
//              query values as five 16-byte chunks); per-query sums reduced
//              once at the end.
// S^T and P are double-buffered, so QK^T of tile t+1 and PV of tile t-1 overlap
// the softmax of tile t.  Units are launched longest request first.  A request
// split over several chunks writes (O, m, l) partials; the last chunk CTA of a
// (request, head) merges them (completion counter).  Every cross-role wait is
// bounded in time.
#pragma once

#include "common.cuh"

namespace dfm {

constexpr int TA_KT = 128;              // keys per tile = TMEM lanes of S^T
constexpr int TA_QN = 48;               // query columns of S^T (34 used)
constexpr int TA_ROWS = 34;             // query rows per request
constexpr int TA_CH = 4096;             // most keys one work unit takes (longer requests split)
constexpr int TA_THREADS = 192;
constexpr int TA_KV_BYTES = TA_KT * 128;           // 16 KB: 128 keys x 64 dims
constexpr int TA_Q_BYTES = TA_QN * 128;           // 48 rows x 128 B
// P (the bf16 A operand of O = P V) is stored MN-major: key k of the tile is
// the 128-byte row k of one 64-query swizzle atom (queries 0..33 used, 34..39
// zero).  The M=128 product reads a second 64-query atom TA_P_BUF bytes further
// on (the other P buffer, or the K ring after buffer 1): finite data that only
// feeds output rows 64..127, which are never read.
constexpr int TA_P_BUF = TA_KT * 128;              // 16 KB
constexpr int TA_OFF_P = 0;
constexpr int TA_OFF_K = TA_OFF_P + 2 * TA_P_BUF;
constexpr int TA_OFF_V = TA_OFF_K + 2 * TA_KV_BYTES;
constexpr int TA_OFF_Q = TA_OFF_V + 2 * TA_KV_BYTES;
constexpr int TA_OFF_MISC = TA_OFF_Q + TA_Q_BYTES;
constexpr int TA_MISC_BYTES = 6144;
constexpr int TA_SMEM = TA_OFF_MISC + TA_MISC_BYTES + 1024;
constexpr uint32_t TA_TMEM_COLS = 256;             // S^T buffers at 0 and 64, O at 128
constexpr uint32_t TA_O_COL = 128;
constexpr float TA_TAU = 16.0f;                    // lazy-rescale threshold, log2 units
constexpr float TA_M0 = 0.0f;                      // running-max start value (log2 units)
constexpr int TA_MAX_PAGES = (TA_CH / TA_KT + 1) * (TA_KT / 16);  // pages of one unit
constexpr int TA_MAX_ORDER = 256;                  // requests ordered longest-first

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

// Reduce-scatter of 32 per-lane values across a warp: afterwards lane l holds
// the reduction over all lanes of value l (31 shuffles instead of 32 x 5).
template <bool kMax>
DFM_DEV float warp_reduce_scatter32(float (&v)[32], int lane) {
#pragma unroll
  for (int step = 16; step >= 1; step >>= 1) {
    const bool upper = (lane & step) != 0;
#pragma unroll
    for (int k = 0; k < step; ++k) {
      const float send = upper ? v[k] : v[k + step];
      const float keep = upper ? v[k + step] : v[k];
      const float got = __shfl_xor_sync(0xffffffffu, send, step);
      v[k] = kMax ? fmaxf(keep, got) : keep + got;
    }
  }
  return v[0];
}

// Per-query reduction over this warp's 32 key rows of the 34 values x[j];
// the warp's result for query j goes to dst[sw * 34 + j].
template <bool kMax>
DFM_DEV void warp_reduce34(const float (&x)[TA_ROWS], float* dst, int sw, int lane) {
  float v[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = x[j];
  dst[sw * TA_ROWS + lane] = warp_reduce_scatter32<kMax>(v, lane);
  float a = x[32], b = x[33];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ao = __shfl_xor_sync(0xffffffffu, a, o);
    const float bo = __shfl_xor_sync(0xffffffffu, b, o);
    a = kMax ? fmaxf(a, ao) : a + ao;
    b = kMax ? fmaxf(b, bo) : b + bo;
  }
  if (lane == 0) {
    dst[sw * TA_ROWS + 32] = a;
    dst[sw * TA_ROWS + 33] = b;
  }
}

__global__ void __launch_bounds__(TA_THREADS, 2)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tm_pool,
                   const __grid_constant__ CUtensorMap tm_q, AttnParams p) {
  // Unit u = blockIdx.x: head fastest, then chunk, then the request of rank r
  // in the longest-first order (long units start in the first wave).
  const int h = blockIdx.x % p.heads;
  const int c = (blockIdx.x / p.heads) % p.MC;
  const int r = blockIdx.x / (p.heads * p.MC);
  pdl_trigger();
  if (threadIdx.x == 0) {
    tma_prefetch(&tm_pool);
    tma_prefetch(&tm_q);
  }
  pdl_wait();
  if (r >= p.n) return;
  int i = r;
  if (p.n <= TA_MAX_ORDER) {
    __shared__ int order_s[TA_MAX_ORDER];
    __shared__ int len_s[TA_MAX_ORDER];
    for (int x = threadIdx.x; x < p.n; x += blockDim.x) len_s[x] = p.cache_len[x] + p.n_ext[x];
    __syncthreads();
    for (int x = threadIdx.x; x < p.n; x += blockDim.x) {
      int rank = 0;
      for (int y = 0; y < p.n; ++y) rank += (len_s[y] > len_s[x]) || (len_s[y] == len_s[x] && y < x);
      order_s[rank] = x;
    }
    __syncthreads();
    i = order_s[r];
  }
  const int P = p.cache_len[i];
  const int ne = p.n_ext[i];
  const int total = P + ne + (TA_ROWS - p.ext_slots);
  if (P < 0 || ne < 0 || ne > p.ext_slots || total > p.max_pages * 16) {
    if (c == 0 && h == 0 && threadIdx.x == 0) atomicOr(p.err, DFM_DEV_ERR_LEN);
    return;
  }
  const int nchunks = (total + TA_CH - 1) / TA_CH;
  if (c >= nchunks || nchunks > p.MC) return;
  const int tiles_all = (total + TA_KT - 1) / TA_KT;
  const int tiles_per = (tiles_all + nchunks - 1) / nchunks;
  const int k0 = c * tiles_per * TA_KT;
  const int k1 = min(total, k0 + tiles_per * TA_KT);
  const int ntiles = k1 > k0 ? (k1 - k0 + TA_KT - 1) / TA_KT : 0;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sP = smem + TA_OFF_P;
  uint8_t* sK = smem + TA_OFF_K;
  uint8_t* sV = smem + TA_OFF_V;
  uint8_t* sQ = smem + TA_OFF_Q;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + TA_OFF_MISC);
  uint64_t* k_full = bars;         // [2]
  uint64_t* k_empty = bars + 2;    // [2]
  uint64_t* v_full = bars + 4;     // [2]
  uint64_t* v_empty = bars + 6;    // [2]
  uint64_t* s_full = bars + 8;     // [2]
  uint64_t* s_empty = bars + 10;   // [2]  arrivals of the 4 softmax warps
  uint64_t* q_full = bars + 12;
  uint64_t* p_full = bars + 13;    // [2]  arrivals of the 4 softmax warps
  uint64_t* p_empty = bars + 15;   // [2]
  uint64_t* team = bars + 17;      // the 4 softmax warps
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 18);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* last_flag = abort_flag + 1;
  volatile int* flags = abort_flag + 2;                              // [2][4]
  float* red = reinterpret_cast<float*>(smem + TA_OFF_MISC + 320);   // [3][4][34]
  float* vals = red + 3 * 4 * TA_ROWS;                               // [34]
  float* mfin = vals + TA_ROWS;                                      // [34]
  float* m_s = mfin + TA_ROWS;                                       // [2][34]
  int* page_s = reinterpret_cast<int*>(m_s + 2 * TA_ROWS);           // [TA_MAX_PAGES]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int b = 0; b < 2; ++b) {
      mbar_init(&k_full[b], 1);
      mbar_init(&k_empty[b], 1);
      mbar_init(&v_full[b], 1);
      mbar_init(&v_empty[b], 1);
      mbar_init(&s_full[b], 1);
      mbar_init(&s_empty[b], 4);
      mbar_init(&p_full[b], 4);
      mbar_init(&p_empty[b], 1);
    }
    mbar_init(q_full, 1);
    mbar_init(team, 4);
    *abort_flag = 0;
    *last_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TA_TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const size_t unit = (static_cast<size_t>(i) * p.MC + c) * p.heads + h;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    // The unit's page ids, read once by the whole warp: pages past the
    // request's keys, or invalid table entries, become an out-of-range page
    // index so TMA fills those boxes with zeros.
    {
      const int pg0 = k0 >> 4;
      const int npg = ntiles * (TA_KT / 16);
      const int* bt = p.block_table + static_cast<size_t>(i) * p.max_pages;
      for (int x = lane; x < npg && x < TA_MAX_PAGES; x += 32) {
        const int pidx = pg0 + x;
        int page = p.num_pages;
        if (pidx * 16 < total) {
          const int e = pidx < p.max_pages ? bt[pidx] : -1;
          if (e >= 0 && e < p.num_pages) page = e;
          else atomicOr(p.err, DFM_DEV_ERR_PAGE);
        }
        page_s[x] = page;
      }
      __syncwarp();
    }
    if (ntiles > 0) {
      if (lane == 0) {
        mbar_arrive_expect_tx(q_full, TA_QN * 128);
        tma_load_2d(sQ, &tm_q, q_full, h * 64, i * TA_ROWS);
      }
      // one tile = 8 page boxes, issued by lanes 0..7 after lane 0 armed the barrier
      auto load_tile = [&](uint8_t* dst, uint64_t* bar, int t, int plane) {
        if (lane == 0) mbar_arrive_expect_tx(bar, TA_KV_BYTES);
        __syncwarp();
        if (lane < TA_KT / 16) {
          const int x = t * (TA_KT / 16) + lane;
          const int page = x < TA_MAX_PAGES ? page_s[x] : p.num_pages;
          tma_load_5d(dst + lane * 2048, &tm_pool, bar, 0, 0, h, page, plane);
        }
      };
      // K(t) is released by QK^T(t), V(t) by PV(t): keys stream ahead of PV.
      int tk = 0, tv = 0;
      uint32_t spins = 0;
      uint64_t t_idle = 0;
      while (tk < ntiles || tv < ntiles) {
        int doK = 0, doV = 0, stop = 0;
        if (lane == 0) {
          doK = tk < ntiles && (tk < 2 || mbar_test(&k_empty[tk & 1], ((tk >> 1) & 1) ^ 1));
          doV = tv < tk + doK && (tv < 2 || mbar_test(&v_empty[tv & 1], ((tv >> 1) & 1) ^ 1));
          if (doK || doV) {
            spins = 0;
            t_idle = 0;
          } else if ((++spins & 255) == 0) {
            if (t_idle == 0) t_idle = globaltimer();
            else if (globaltimer() - t_idle > DFM_WAIT_LIMIT_NS) {
              *abort_flag = 1;
              atomicOr(p.err, DFM_DEV_ERR_TIMEOUT);
            }
          }
          stop = *abort_flag;
        }
        doK = __shfl_sync(0xffffffffu, doK, 0);
        doV = __shfl_sync(0xffffffffu, doV, 0);
        if (__shfl_sync(0xffffffffu, stop, 0)) break;
        if (doK) {
          load_tile(sK + (tk & 1) * TA_KV_BYTES, &k_full[tk & 1], tk, p.plane_k);
          ++tk;
        }
        if (doV) {
          load_tile(sV + (tv & 1) * TA_KV_BYTES, &v_full[tv & 1], tv, p.plane_v);
          ++tv;
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && ntiles > 0) {
      constexpr uint32_t idesc_s = umma_idesc_bf16(128, TA_QN);
      constexpr uint32_t idesc_o = umma_idesc_bf16_bmn(128, 64) | (1u << 15);  // A MN-major too
      const uint32_t q_addr = smem_u32(sQ);
      const uint32_t p_addr = smem_u32(sP);
      bool ok = mbar_wait(q_full, 0, abort_flag, p.err);
      int t1 = 0, t2 = 0;
      uint32_t spins = 0;
      uint64_t t_idle = 0;
      while (ok && t2 < ntiles && !*abort_flag) {
        bool prog = false;
        if (t1 < ntiles && t1 <= t2 + 1 && mbar_test(&k_full[t1 & 1], (t1 >> 1) & 1) &&
            (t1 < 2 || mbar_test(&s_empty[t1 & 1], ((t1 >> 1) & 1) ^ 1))) {
          tc_fence_after();
          const uint32_t k_addr = smem_u32(sK + (t1 & 1) * TA_KV_BYTES);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_bf16(tmem + (t1 & 1) * 64, umma_desc_sw128(k_addr + kk * 32),
                      umma_desc_sw128(q_addr + kk * 32), idesc_s, kk > 0);
          umma_commit(&s_full[t1 & 1]);
          umma_commit(&k_empty[t1 & 1]);
          ++t1;
          prog = true;
        }
        if (t2 < t1 && mbar_test(&p_full[t2 & 1], (t2 >> 1) & 1) &&
            mbar_test(&v_full[t2 & 1], (t2 >> 1) & 1)) {
          tc_fence_after();
          const uint32_t v_addr = smem_u32(sV + (t2 & 1) * TA_KV_BYTES);
          const uint32_t pb = p_addr + (t2 & 1) * TA_P_BUF;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            umma_bf16(tmem + TA_O_COL, umma_desc_sw128_mn(pb + kk * 2048, TA_P_BUF),
                      umma_desc_sw128(v_addr + kk * 2048), idesc_o, (t2 > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&v_empty[t2 & 1]);
          umma_commit(&p_empty[t2 & 1]);
          ++t2;
          prog = true;
        }
        if (prog) {
          spins = 0;
          t_idle = 0;
        } else if ((++spins & 255) == 0) {
          if (t_idle == 0) t_idle = globaltimer();
          else if (globaltimer() - t_idle > DFM_WAIT_LIMIT_NS) {
            *abort_flag = 1;
            atomicOr(p.err, DFM_DEV_ERR_TIMEOUT);
          }
        }
      }
    }
  } else {
    // ------------------------------------------------------------ softmax warps
    const int q4 = warp & 3;            // TMEM lane quadrant of this warp
    const int sw = warp - 2;            // 0..3
    const int row = q4 * 32 + lane;     // key row of the tile
    const uint32_t lane_off = static_cast<uint32_t>(q4 * 32) << 16;
    const float cexp = 0.125f * 1.4426950408889634f;  // 1/sqrt(64) * log2(e)
    // Running max per query in log2 units (score * cexp).  It starts at 0 so
    // that the first tile's x = score * cexp - max is exact; the first tile
    // always takes the update path, which replaces it with the tile's max.  A
    // query whose keys are all masked keeps max = -inf (its unmasked keys form
    // a prefix, so every later key is masked too) and x = -inf.
    if (sw == 0)
      for (int j = lane; j < TA_ROWS; j += 32) m_s[j] = TA_M0;
    int ver = 0;   // m_s[ver & 1] holds the running max (one writer per update)
    float l[TA_ROWS];
#pragma unroll
    for (int j = 0; j < TA_ROWS; ++j) l[j] = 0.f;
    uint32_t team_phase = 0;
    auto team_sync = [&]() -> bool {
      __syncwarp();
      if (lane == 0) mbar_arrive(team);
      const bool rr = __all_sync(0xffffffffu, mbar_wait(team, team_phase & 1, abort_flag, p.err));
      ++team_phase;
      return rr;
    };
    // the first tile's reduction reads m_s: make the initialisation visible
    bool ok = team_sync();
    const uint32_t prow = smem_u32(sP) + row * 128;   // this key's row of the P atom
    const int psw = row & 7;
#pragma unroll 1
    for (int t = 0; ok && t < ntiles; ++t) {
      const int sb = t & 1;
      ok = __all_sync(0xffffffffu, mbar_wait(&s_full[sb], (t >> 1) & 1, abort_flag, p.err));
      if (!ok) break;
      tc_fence_after();
      // x[j] = score * cexp - max_j   (log2 units, relative to the running max)
      float x[TA_ROWS];
      {
        uint32_t r32[32], r16[16];
        tmem_ld32(tmem + sb * 64 + lane_off, r32);
        tmem_ld16(tmem + sb * 64 + 32 + lane_off, r16);
        const float* mc = m_s + (ver & 1) * TA_ROWS;
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 32; ++j) x[j] = fmaf(__uint_as_float(r32[j]), cexp, -mc[j]);
        x[32] = fmaf(__uint_as_float(r16[0]), cexp, -mc[32]);
        x[33] = fmaf(__uint_as_float(r16[1]), cexp, -mc[33]);
      }
      if (k0 + t * TA_KT + TA_KT > P) {   // only tiles reaching past the cached prefix
        // key k is hidden from graduating rows j with P + j < k, and from all
        // rows beyond the request's keys
        const int key = k0 + t * TA_KT + row;
        const int d = key - P;
        const int jmask = key >= total ? TA_ROWS : (d <= 0 ? 0 : (d < ne ? d : ne));
#pragma unroll
        for (int j = 0; j < TA_ROWS; ++j)
          if (j < jmask) x[j] = -INFINITY;
      }
      bool over = (t == 0);
#pragma unroll
      for (int j = 0; j < TA_ROWS; ++j) over |= x[j] > TA_TAU;
      const bool any = __any_sync(0xffffffffu, over);
      if (lane == 0) flags[(t & 1) * 4 + sw] = any ? 1 : 0;
      // Releasing the S buffer doubles as the per-tile agreement of the four
      // softmax warps: each waits for the phase their four arrivals complete.
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_empty[sb]);
      ok = __all_sync(0xffffffffu, mbar_wait(&s_empty[sb], (t >> 1) & 1, abort_flag, p.err));
      if (!ok) break;
      const bool need = flags[(t & 1) * 4] | flags[(t & 1) * 4 + 1] | flags[(t & 1) * 4 + 2] |
                        flags[(t & 1) * 4 + 3];
      // the PV product two tiles back must be done before its P buffer is rewritten
      if (t >= 2) {
        ok = __all_sync(0xffffffffu,
                        mbar_wait(&p_empty[t & 1], ((t >> 1) & 1) ^ 1, abort_flag, p.err));
        if (!ok) break;
        tc_fence_after();
      }
      if (need) {
        // new running max: the old one raised by this tile's scores (x + max_old)
        const float* mc = m_s + (ver & 1) * TA_ROWS;
        float y[TA_ROWS];
#pragma unroll
        for (int j = 0; j < TA_ROWS; ++j) y[j] = x[j] + mc[j];
        float* rb = red + (t & 1) * 4 * TA_ROWS;
        warp_reduce34<true>(y, rb, sw, lane);
        ok = team_sync();
        if (!ok) break;
        if (sw == 0) {
          float* mn_s = m_s + ((ver + 1) & 1) * TA_ROWS;
          for (int j = lane; j < TA_ROWS; j += 32) {
            const float mt = fmaxf(fmaxf(rb[j], rb[TA_ROWS + j]),
                                   fmaxf(rb[2 * TA_ROWS + j], rb[3 * TA_ROWS + j]));
            const float mo = mc[j];
            const float mn = t == 0 ? mt : fmaxf(mo, mt);
            mn_s[j] = mn;
            vals[j] = (t == 0 || mn == -INFINITY) ? 1.f : fast_exp2(mo - mn);
          }
        }
        ok = team_sync();
        if (!ok) break;
        ++ver;
        const float* mn = m_s + (ver & 1) * TA_ROWS;
#pragma unroll
        for (int j = 0; j < TA_ROWS; ++j) {
          x[j] = mn[j] == -INFINITY ? -INFINITY : x[j] + (mc[j] - mn[j]);
          l[j] *= vals[j];
        }
        if (t >= 1) {
          // every earlier PV product must be done before O is rescaled
          ok = __all_sync(0xffffffffu, mbar_wait(&p_empty[(t - 1) & 1], ((t - 1) >> 1) & 1,
                                                 abort_flag, p.err));
          if (!ok) break;
          tc_fence_after();
          if (q4 <= 1) {
            // rescale the O rows (TMEM lane = query) by their query's factor
            const int qrow = q4 * 32 + lane;
            const float a = qrow < TA_ROWS ? vals[qrow] : 1.f;
            uint32_t o32[32];
#pragma unroll 1
            for (int half = 0; half < 2; ++half) {
              tmem_ld32(tmem + TA_O_COL + half * 32 + lane_off, o32);
              tmem_wait_ld();
#pragma unroll
              for (int e = 0; e < 32; ++e) o32[e] = __float_as_uint(__uint_as_float(o32[e]) * a);
              tmem_st32(tmem + TA_O_COL + half * 32 + lane_off, o32);
            }
            tmem_wait_st();
          }
        }
      }
      // probabilities: this key's row of P buffer t&1 (queries 0..39), row sums
      float e[40];
#pragma unroll
      for (int j = 0; j < TA_ROWS; ++j) {
        e[j] = fast_exp2(x[j]);
        l[j] += e[j];
      }
#pragma unroll
      for (int j = TA_ROWS; j < 40; ++j) e[j] = 0.f;
      const uint32_t pbase = prow + (t & 1) * TA_P_BUF;
#pragma unroll
      for (int c = 0; c < 5; ++c)
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(pbase + ((c ^ psw) << 4)),
                     "r"(pack_bf16(e[8 * c], e[8 * c + 1])), "r"(pack_bf16(e[8 * c + 2], e[8 * c + 3])),
                     "r"(pack_bf16(e[8 * c + 4], e[8 * c + 5])), "r"(pack_bf16(e[8 * c + 6], e[8 * c + 7]))
                     : "memory");
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[t & 1]);
    }
    if (ok && ntiles > 0) {
      ok = __all_sync(0xffffffffu, mbar_wait(&p_empty[(ntiles - 1) & 1], ((ntiles - 1) >> 1) & 1,
                                             abort_flag, p.err));
      tc_fence_after();
    }
    // per-query sums over the 128 key rows
    warp_reduce34<false>(l, red + 8 * TA_ROWS, sw, lane);
    if (ok) ok = team_sync();
    if (ok && sw == 0) {
      const float* rs = red + 8 * TA_ROWS;
      const float* mcur = m_s + (ver & 1) * TA_ROWS;
      for (int j = lane; j < TA_ROWS; j += 32) {
        vals[j] = rs[j] + rs[TA_ROWS + j] + rs[2 * TA_ROWS + j] + rs[3 * TA_ROWS + j];
        mfin[j] = mcur[j];
      }
    }
    if (ok) ok = team_sync();
    // O rows (TMEM lane = query) out
    if (ok && q4 <= 1) {
      const int qrow = q4 * 32 + lane;
      float o[64];
      if (ntiles > 0) {
        uint32_t o32[32];
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          tmem_ld32(tmem + TA_O_COL + half * 32 + lane_off, o32);
          tmem_wait_ld();
#pragma unroll
          for (int q = 0; q < 32; ++q) o[half * 32 + q] = __uint_as_float(o32[q]);
        }
      } else {
#pragma unroll
        for (int q = 0; q < 64; ++q) o[q] = 0.f;
      }
      if (qrow < TA_ROWS) {
        const float L = vals[qrow];
        if (nchunks == 1) {
          const float il = L > 0.f ? 1.f / L : 0.f;
          uint4* dst = reinterpret_cast<uint4*>(p.out + (static_cast<size_t>(i) * TA_ROWS + qrow) * p.H +
                                                h * 64);
#pragma unroll
          for (int q8 = 0; q8 < 8; ++q8)
            dst[q8] = make_uint4(pack_bf16(o[8 * q8] * il, o[8 * q8 + 1] * il),
                                 pack_bf16(o[8 * q8 + 2] * il, o[8 * q8 + 3] * il),
                                 pack_bf16(o[8 * q8 + 4] * il, o[8 * q8 + 5] * il),
                                 pack_bf16(o[8 * q8 + 6] * il, o[8 * q8 + 7] * il));
        } else {
          float4* po = reinterpret_cast<float4*>(p.part_o + (unit * TA_ROWS + qrow) * 64);
#pragma unroll
          for (int q4i = 0; q4i < 16; ++q4i)
            po[q4i] = make_float4(o[4 * q4i], o[4 * q4i + 1], o[4 * q4i + 2], o[4 * q4i + 3]);
          *reinterpret_cast<float2*>(p.part_ml + (unit * TA_ROWS + qrow) * 2) = make_float2(mfin[qrow], L);
          __threadfence();
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TA_TMEM_COLS);
  }
  if (nchunks == 1) return;   // CTA-uniform
  // ---------------------------------------------------------- split-key merge
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
  for (int w = threadIdx.x; w < TA_ROWS * 4; w += TA_THREADS) {
    const int rr = w >> 2, seg = (w & 3) * 16;
    float M = -INFINITY;
    for (int cc = 0; cc < nchunks; ++cc)
      M = fmaxf(M, p.part_ml[((base + static_cast<size_t>(cc) * p.heads) * TA_ROWS + rr) * 2]);
    float L = 0.f, acc[16];
#pragma unroll
    for (int d = 0; d < 16; ++d) acc[d] = 0.f;
    for (int cc = 0; cc < nchunks; ++cc) {
      const size_t u2 = base + static_cast<size_t>(cc) * p.heads;
      const float2 ml = *reinterpret_cast<const float2*>(p.part_ml + (u2 * TA_ROWS + rr) * 2);
      const float wgt = ml.x == -INFINITY ? 0.f : fast_exp2(ml.x - M);
      L += wgt * ml.y;
      const float4* src = reinterpret_cast<const float4*>(p.part_o + (u2 * TA_ROWS + rr) * 64 + seg);
#pragma unroll
      for (int q4i = 0; q4i < 4; ++q4i) {
        const float4 v = src[q4i];
        acc[4 * q4i] += wgt * v.x; acc[4 * q4i + 1] += wgt * v.y;
        acc[4 * q4i + 2] += wgt * v.z; acc[4 * q4i + 3] += wgt * v.w;
      }
    }
    const float il = L > 0.f ? 1.f / L : 0.f;
    uint4* dst = reinterpret_cast<uint4*>(p.out + (static_cast<size_t>(i) * TA_ROWS + rr) * p.H +
                                          h * 64 + seg);
    dst[0] = make_uint4(pack_bf16(acc[0] * il, acc[1] * il), pack_bf16(acc[2] * il, acc[3] * il),
                        pack_bf16(acc[4] * il, acc[5] * il), pack_bf16(acc[6] * il, acc[7] * il));
    dst[1] = make_uint4(pack_bf16(acc[8] * il, acc[9] * il), pack_bf16(acc[10] * il, acc[11] * il),
                        pack_bf16(acc[12] * il, acc[13] * il), pack_bf16(acc[14] * il, acc[15] * il));
  }
}

}  // namespace dfm
