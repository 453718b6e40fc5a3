// Paged prefix attention of the FM head on the tcgen05 tensor cores.
//
// Semantics (the prefix-cache mask of the reference's cached FM head,
// ``cached_fm.py:124-197``), per request with cache length P and n_ext
// graduating rows:
//   graduating row j (j < n_ext): keys [0, P + j + 1)
//   every other row:              keys [0, P + n_ext + 34 - ext_slots)
// softmax(q k^T / 8) v in fp32 with bf16 operands.  The FM head has
// ext_slots = 17 (the active block of 17 rows sees itself); the patch encoder
// (``layers.py:210-245``, a causal block of 8 new rows) passes ext_slots = 34
// and n_ext = 8, so every row is causal.
//
// Work unit: (request, chunk of up to 4096 keys, head), units ordered longest
// request first.  The kernel is persistent: a grid of two CTAs per SM, CTA b
// taking units b, 2G-1-b, 2G+b, ... (a snake over the ordered list, which
// evens out the per-CTA totals).  Each CTA streams the K/V tiles of its units
// back to back, so the next unit's loads overlap the current unit's tail.
// Roles (192 threads):
//   warp 0     TMA: per unit its page ids (into one of two buffers) and its 34
//              query rows (one 40-row box, two buffers); per 128-key tile 8 K
//              and 8 V boxes (one 2 KB box per page, issued by 8 lanes) into
//              a 2-deep K ring and a 3-deep V ring
//   warp 1     TMEM owner and the single MMA-issuing thread:
//                S^T[128 keys x 48 queries] = K . Q^T   (M=128, N=48, K=64)
//                O[128 x 64]               += P . V     (M=128, N=64, K=128, P and V MN-major)
//              each issued as soon as its own inputs are ready (polling); O
//              has one TMEM buffer per unit parity
//   warps 2-5  softmax: thread = one key row of S^T (TMEM lane); exponentials
//              against a running max per query, re-reduced across the 128 rows
//              only on a unit's first tile or when a score exceeds it by 2^16;
//              probabilities written to shared memory as the bf16 A operand of
//              the PV product (each thread stores its key row's 34 query values
//              as five 16-byte chunks); per-query sums reduced at the end of
//              each unit, when these warps also write the unit's output.
// A request split over several chunks writes (O, m, l) partials; the CTA that
// finishes its last chunk merges them (completion counter).  Every cross-role
// wait is bounded in time.
#pragma once

#include "common.cuh"

namespace dfm {

constexpr int TA_KT = 128;              // keys per tile = TMEM lanes of S^T
constexpr int TA_QN = 48;               // query columns of S^T (34 used)
constexpr int TA_QROWS = 40;            // query rows loaded per unit (34 used)
constexpr int TA_ROWS = 34;             // query rows per request
constexpr int TA_CH = 4096;             // most keys one work unit takes (longer requests split)
constexpr int TA_THREADS = 192;
constexpr int TA_KV_BYTES = TA_KT * 128;           // 16 KB: 128 keys x 64 dims
constexpr int TA_Q_BYTES = TA_QROWS * 128;         // 5 KB per query buffer
// P (the bf16 A operand of O = P V) is stored MN-major: key k of the tile is
// the 128-byte row k of one 64-query swizzle atom (queries 0..33 used, 34..39
// zero).  The M=128 product reads a second 64-query atom TA_P_BYTES further
// on (the K ring): finite data that only feeds output rows 64..127, which are
// never read.  Likewise the N=48 product of S^T reads query rows 40..47 past
// a query buffer (the other buffer or the barrier area); they only feed S^T
// columns 40..47, which are never read.
constexpr int TA_P_BYTES = TA_KT * 128;            // 16 KB
constexpr int TA_PSLOTS = 1;             // P buffers (2: the softmax of tile t+1 overlaps PV of tile t)
constexpr int TA_OFF_P = 0;
constexpr int TA_OFF_K = TA_OFF_P + TA_PSLOTS * TA_P_BYTES;
constexpr int TA_KSLOTS = 2;            // K ring: a slot is released as soon as QK^T has read it
constexpr int TA_VSLOTS = 3;            // V ring: a slot is held until PV, after the softmax
constexpr int TA_OFF_V = TA_OFF_K + TA_KSLOTS * TA_KV_BYTES;
constexpr int TA_OFF_Q = TA_OFF_V + TA_VSLOTS * TA_KV_BYTES;
constexpr int TA_OFF_MISC = TA_OFF_Q + 2 * TA_Q_BYTES;
constexpr int TA_MISC_BYTES = 6144;
constexpr int TA_MISC_RED = 512;         // barriers and flags first, then the float scratch
constexpr int TA_SMEM = TA_OFF_MISC + TA_MISC_BYTES + 1024;
constexpr int TA_CTAS_PER_SM = 2;
// dynamic shared memory + the 1 KB the runtime reserves per CTA
static_assert(TA_CTAS_PER_SM * (TA_SMEM + 1024) <= 233472, "two CTAs per SM");
constexpr uint32_t TA_TMEM_COLS = 256;             // S^T buffers at 0 and 64, O at 128 and 192
constexpr uint32_t TA_O_COL = 128;
constexpr float TA_TAU = 16.0f;                    // lazy-rescale threshold, log2 units
constexpr float TA_M0 = 0.0f;                      // running-max start value (log2 units)
constexpr int TA_MAX_PAGES = (TA_CH / TA_KT + 1) * (TA_KT / 16);  // pages of one unit
constexpr int TA_MAX_ORDER = 256;                  // requests ordered longest-first

struct AttnParams {
  const __nv_bfloat16* q;    // [n*q_rows, H]
  __nv_bfloat16* out;        // [n*q_rows, H]
  float* part_o;             // [n*MC*heads][34][64]
  float* part_ml;            // [n*MC*heads][34][2]
  int* sem;                  // [n*heads] chunk-completion counters (zero between launches)
  const int* cache_len;
  const int* n_ext;
  const int* block_table;
  int n, max_pages, num_pages, heads, H, MC;
  int plane_k, plane_v;
  int ext_slots;             // 17 (34: every row is causal, none sees a fixed block)
  int q_rows;                // rows per request in q and out: 34, or fewer (the patch
                             // encoder's 8); the 40-row query box then also carries
                             // the next requests' rows, whose outputs are not written
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

// One work unit of the attention, as every role derives it.
struct AttnUnit {
  int i, c, h;             // request, chunk, head
  int P, ne, total;        // cached keys, graduating rows, keys of the request
  int k0, ntiles, nchunks;
  bool bad;                // the request's lengths are invalid
};

DFM_DEV AttnUnit attn_unit(const AttnParams& p, const int* order_s, int u) {
  AttnUnit f;
  f.h = u % p.heads;
  f.c = (u / p.heads) % p.MC;
  const int r = u / (p.heads * p.MC);
  f.i = p.n <= TA_MAX_ORDER ? order_s[r] : r;
  f.P = p.cache_len[f.i];
  f.ne = p.n_ext[f.i];
  f.total = f.P + f.ne + (TA_ROWS - p.ext_slots);
  f.k0 = 0;
  f.ntiles = 0;
  f.nchunks = 0;
  f.bad = f.P < 0 || f.ne < 0 || f.ne > p.ext_slots || f.total > p.max_pages * 16;
  if (f.bad) return f;
  f.nchunks = (f.total + TA_CH - 1) / TA_CH;
  if (f.c >= f.nchunks || f.nchunks > p.MC) return f;
  const int tiles_all = (f.total + TA_KT - 1) / TA_KT;
  const int tiles_per = (tiles_all + f.nchunks - 1) / f.nchunks;
  f.k0 = f.c * tiles_per * TA_KT;
  const int k1 = min(f.total, f.k0 + tiles_per * TA_KT);
  f.ntiles = k1 > f.k0 ? (k1 - f.k0 + TA_KT - 1) / TA_KT : 0;
  return f;
}

// A role's position in this CTA's unit list: round k of the snake, the
// sequence number of the unit among those with work, and the tile within it.
struct AttnCursor {
  int k, seq, t;
  bool done;
  AttnUnit f;
};

// Advance `cu` to the next unit with work at round >= cu.k.
DFM_DEV void attn_seek(AttnCursor& cu, const AttnParams& p, const int* order_s, int U) {
  const int G = gridDim.x, b = blockIdx.x;
  while (true) {
    const int idx = cu.k * G + ((cu.k & 1) ? (G - 1 - b) : b);
    if (idx >= U) {
      cu.done = true;
      return;
    }
    cu.f = attn_unit(p, order_s, idx);
    if (cu.f.ntiles > 0) {
      cu.t = 0;
      return;
    }
    ++cu.k;
  }
}

DFM_DEV void attn_start(AttnCursor& cu, const AttnParams& p, const int* order_s, int U) {
  cu.k = 0;
  cu.seq = 0;
  cu.t = 0;
  cu.done = false;
  attn_seek(cu, p, order_s, U);
}

// Step to the next tile (and unit).
DFM_DEV void attn_step(AttnCursor& cu, const AttnParams& p, const int* order_s, int U) {
  if (++cu.t < cu.f.ntiles) return;
  ++cu.k;
  ++cu.seq;
  attn_seek(cu, p, order_s, U);
}

__global__ void __launch_bounds__(TA_THREADS, TA_CTAS_PER_SM)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tm_pool,
                   const __grid_constant__ CUtensorMap tm_q, AttnParams p) {
  pdl_trigger();
  if (threadIdx.x == 0) {
    tma_prefetch(&tm_pool);
    tma_prefetch(&tm_q);
  }
  pdl_wait();
  const int U = p.n * p.MC * p.heads;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sP = smem + TA_OFF_P;
  uint8_t* sK = smem + TA_OFF_K;
  uint8_t* sV = smem + TA_OFF_V;
  uint8_t* sQ = smem + TA_OFF_Q;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + TA_OFF_MISC);
  uint64_t* k_full = bars;                          // [TA_KSLOTS]
  uint64_t* k_empty = k_full + TA_KSLOTS;           // [TA_KSLOTS]
  uint64_t* v_full = k_empty + TA_KSLOTS;           // [TA_VSLOTS]
  uint64_t* v_empty = v_full + TA_VSLOTS;           // [TA_VSLOTS]
  uint64_t* s_full = v_empty + TA_VSLOTS;           // [2]
  uint64_t* s_empty = s_full + 2;   // [2]  arrivals of the 4 softmax warps
  uint64_t* q_full = s_empty + 2;   // [2]  per unit parity
  uint64_t* q_empty = q_full + 2;   // [2]
  uint64_t* p_full = q_empty + 2;   // [TA_PSLOTS]  arrivals of the 4 softmax warps
  uint64_t* p_empty = p_full + TA_PSLOTS;  // [TA_PSLOTS]
  uint64_t* o_empty = p_empty + TA_PSLOTS;  // [2]  per unit parity, arrivals of the 4 softmax warps
  uint64_t* team = o_empty + 2;     // the 4 softmax warps
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(team + 1);
  static_assert((2 * (TA_KSLOTS + TA_VSLOTS + TA_PSLOTS) + 11) * 8 + 44 <= TA_MISC_RED,
                "barrier area");
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* last_flag = abort_flag + 1;
  volatile int* flags = abort_flag + 2;                              // [2][4]
  float* red = reinterpret_cast<float*>(smem + TA_OFF_MISC + TA_MISC_RED);   // [3][4][34]
  float* vals = red + 3 * 4 * TA_ROWS;                               // [34]
  float* mfin = vals + TA_ROWS;                                      // [34]
  float* m_s = mfin + TA_ROWS;                                       // [2][34]
  int* page_s = reinterpret_cast<int*>(m_s + 2 * TA_ROWS);           // [2][TA_MAX_PAGES]
  int* order_s = page_s + 2 * TA_MAX_PAGES;                          // [TA_MAX_ORDER]
  static_assert(TA_MISC_RED + (3 * 4 + 5) * TA_ROWS * 4 + (2 * TA_MAX_PAGES + TA_MAX_ORDER) * 4 <=
                    TA_MISC_BYTES, "misc area");

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // requests in longest-first order (ties by index), once per CTA; the
  // lengths sit in the page-id buffer until the producer first uses it
  if (p.n <= TA_MAX_ORDER) {
    int* len_s = page_s;
    for (int x = threadIdx.x; x < p.n; x += blockDim.x) len_s[x] = p.cache_len[x] + p.n_ext[x];
    __syncthreads();
    for (int x = threadIdx.x; x < p.n; x += blockDim.x) {
      int rank = 0;
      for (int y = 0; y < p.n; ++y) rank += (len_s[y] > len_s[x]) || (len_s[y] == len_s[x] && y < x);
      order_s[rank] = x;
    }
  }
  // CTA 0 reports requests whose lengths no unit can serve (one thread per
  // request; the producer no longer walks its units' lengths before its first load)
  if (blockIdx.x == 0)
    for (int x = threadIdx.x; x < p.n; x += blockDim.x) {
      const int P = p.cache_len[x], ne = p.n_ext[x];
      if (P < 0 || ne < 0 || ne > p.ext_slots || P + ne + (TA_ROWS - p.ext_slots) > p.max_pages * 16)
        atomicOr(p.err, DFM_DEV_ERR_LEN);
    }
  if (threadIdx.x == 0) {
    for (int b = 0; b < TA_VSLOTS; ++b) {
      mbar_init(&v_full[b], 1);
      mbar_init(&v_empty[b], 1);
    }
    for (int b = 0; b < TA_KSLOTS; ++b) {
      mbar_init(&k_full[b], 1);
      mbar_init(&k_empty[b], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&s_empty[b], 4);
      mbar_init(&q_full[b], 1);
      mbar_init(&q_empty[b], 1);
      mbar_init(&o_empty[b], 4);
    }
    for (int b = 0; b < TA_PSLOTS; ++b) {
      mbar_init(&p_full[b], 4);
      mbar_init(&p_empty[b], 1);
    }
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

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    AttnCursor ck, cv;   // next K tile, next V tile
    attn_start(ck, p, order_s, U);
    attn_start(cv, p, order_s, U);
    // one tile = 8 page boxes, issued by lanes 0..7 after lane 0 armed the barrier
    auto load_tile = [&](uint8_t* dst, uint64_t* bar, const AttnCursor& cu, int plane) {
      if (lane == 0) mbar_arrive_expect_tx(bar, TA_KV_BYTES);
      __syncwarp();
      if (lane < TA_KT / 16) {
        const int x = cu.t * (TA_KT / 16) + lane;
        const int page = x < TA_MAX_PAGES ? page_s[(cu.seq & 1) * TA_MAX_PAGES + x] : p.num_pages;
        tma_load_5d(dst + lane * 2048, &tm_pool, bar, 0, 0, cu.f.h, page, plane);
      }
    };
    int gk = 0, gv = 0;   // K and V tiles issued so far (ring positions)
    uint32_t spins = 0;
    uint64_t t_idle = 0;
    while (!ck.done || !cv.done) {
      int doK = 0, doV = 0, stop = 0;
      if (lane == 0) {
        doK = !ck.done && (gk < TA_KSLOTS ||
                           mbar_test(&k_empty[gk % TA_KSLOTS], ((gk / TA_KSLOTS) & 1) ^ 1));
        if (doK && ck.t == 0)   // a new unit: its page ids and query buffer must be free
          doK = ck.seq <= cv.seq + 1 &&
                (ck.seq < 2 || mbar_test(&q_empty[ck.seq & 1], ((ck.seq >> 1) & 1) ^ 1));
        doV = !cv.done && gv < gk &&
              (gv < TA_VSLOTS ||
               mbar_test(&v_empty[gv % TA_VSLOTS], ((gv / TA_VSLOTS) & 1) ^ 1));
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
        if (ck.t == 0) {
          // The unit's page ids: pages past the request's keys, or invalid
          // table entries, become an out-of-range page index so TMA fills
          // those boxes with zeros.
          const int pg0 = ck.f.k0 >> 4;
          const int npg = ck.f.ntiles * (TA_KT / 16);
          const int* bt = p.block_table + static_cast<size_t>(ck.f.i) * p.max_pages;
          int* ps = page_s + (ck.seq & 1) * TA_MAX_PAGES;
          for (int x = lane; x < npg && x < TA_MAX_PAGES; x += 32) {
            const int pidx = pg0 + x;
            int page = p.num_pages;
            if (pidx * 16 < ck.f.total) {
              const int e = pidx < p.max_pages ? bt[pidx] : -1;
              if (e >= 0 && e < p.num_pages) page = e;
              else atomicOr(p.err, DFM_DEV_ERR_PAGE);
            }
            ps[x] = page;
          }
          __syncwarp();
          if (lane == 0) {
            mbar_arrive_expect_tx(&q_full[ck.seq & 1], TA_Q_BYTES);
            tma_load_2d(sQ + (ck.seq & 1) * TA_Q_BYTES, &tm_q, &q_full[ck.seq & 1], ck.f.h * 64,
                        ck.f.i * p.q_rows);
          }
        }
        load_tile(sK + (gk % TA_KSLOTS) * TA_KV_BYTES, &k_full[gk % TA_KSLOTS], ck, p.plane_k);
        ++gk;
        attn_step(ck, p, order_s, U);
      }
      if (doV) {
        load_tile(sV + (gv % TA_VSLOTS) * TA_KV_BYTES, &v_full[gv % TA_VSLOTS], cv, p.plane_v);
        ++gv;
        attn_step(cv, p, order_s, U);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_s = umma_idesc_bf16(128, TA_QN);
      constexpr uint32_t idesc_o = umma_idesc_bf16_bmn(128, 64) | (1u << 15);  // A MN-major too
      const uint32_t p_addr = smem_u32(sP);
      AttnCursor c1, c2;   // next QK^T tile, next PV tile
      attn_start(c1, p, order_s, U);
      attn_start(c2, p, order_s, U);
      int g1 = 0, g2 = 0;
      uint32_t spins = 0;
      uint64_t t_idle = 0;
      while (!c2.done && !*abort_flag) {
        bool prog = false;
        if (!c1.done && mbar_test(&k_full[g1 % TA_KSLOTS], (g1 / TA_KSLOTS) & 1) &&
            (g1 < 2 || mbar_test(&s_empty[g1 & 1], ((g1 >> 1) & 1) ^ 1)) &&
            (c1.t > 0 || mbar_test(&q_full[c1.seq & 1], (c1.seq >> 1) & 1))) {
          tc_fence_after();
          const uint32_t k_addr = smem_u32(sK + (g1 % TA_KSLOTS) * TA_KV_BYTES);
          const uint32_t q_addr = smem_u32(sQ + (c1.seq & 1) * TA_Q_BYTES);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_bf16(tmem + (g1 & 1) * 64, umma_desc_sw128(k_addr + kk * 32),
                      umma_desc_sw128(q_addr + kk * 32), idesc_s, kk > 0);
          umma_commit(&s_full[g1 & 1]);
          umma_commit(&k_empty[g1 % TA_KSLOTS]);
          if (c1.t == c1.f.ntiles - 1) umma_commit(&q_empty[c1.seq & 1]);
          ++g1;
          attn_step(c1, p, order_s, U);
          prog = true;
        }
        if (g2 < g1 && mbar_test(&p_full[g2 % TA_PSLOTS], (g2 / TA_PSLOTS) & 1) &&
            mbar_test(&v_full[g2 % TA_VSLOTS], (g2 / TA_VSLOTS) & 1) &&
            (c2.t > 0 || c2.seq < 2 || mbar_test(&o_empty[c2.seq & 1], ((c2.seq >> 1) & 1) ^ 1))) {
          tc_fence_after();
          const uint32_t v_addr = smem_u32(sV + (g2 % TA_VSLOTS) * TA_KV_BYTES);
          const uint32_t o_col = tmem + TA_O_COL + (c2.seq & 1) * 64;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            umma_bf16(o_col,
                      umma_desc_sw128_mn(p_addr + (g2 % TA_PSLOTS) * TA_P_BYTES + kk * 2048,
                                         TA_P_BYTES),
                      umma_desc_sw128(v_addr + kk * 2048), idesc_o, (c2.t > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&v_empty[g2 % TA_VSLOTS]);
          umma_commit(&p_empty[g2 % TA_PSLOTS]);
          ++g2;
          attn_step(c2, p, order_s, U);
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
    const uint32_t prow = smem_u32(sP) + row * 128;   // this key's row of the P atom
    const int psw = row & 7;
    uint32_t team_phase = 0;
    auto team_sync = [&]() -> bool {
      __syncwarp();
      if (lane == 0) mbar_arrive(team);
      const bool rr = __all_sync(0xffffffffu, mbar_wait(team, team_phase & 1, abort_flag, p.err));
      ++team_phase;
      return rr;
    };
    AttnCursor cu;
    attn_start(cu, p, order_s, U);
    int g = 0;   // tiles processed so far (S buffer and P phases)
    bool ok = true;
#pragma unroll 1
    while (ok && !cu.done) {
      const AttnUnit f = cu.f;
      const int seq = cu.seq;
      // Running max per query in log2 units (score * cexp).  It starts at 0 so
      // that the first tile's x = score * cexp - max is exact; the first tile
      // always takes the update path, which replaces it with the tile's max.
      // A query whose keys are all masked keeps max = -inf (its unmasked keys
      // form a prefix, so every later key is masked too) and x = -inf.
      if (sw == 0)
        for (int j = lane; j < TA_ROWS; j += 32) m_s[j] = TA_M0;
      int ver = 0;   // m_s[ver & 1] holds the running max (one writer per update)
      float l[TA_ROWS];
#pragma unroll
      for (int j = 0; j < TA_ROWS; ++j) l[j] = 0.f;
      // the initialisation is visible, and the previous unit's readers are done
      ok = team_sync();
#pragma unroll 1
      for (int t = 0; ok && t < f.ntiles; ++t, ++g) {
        const int sb = g & 1;
        ok = __all_sync(0xffffffffu, mbar_wait(&s_full[sb], (g >> 1) & 1, abort_flag, p.err));
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
        if (f.k0 + t * TA_KT + TA_KT > f.P) {   // only tiles reaching past the cached prefix
          // key k is hidden from graduating rows j with P + j < k, and from all
          // rows beyond the request's keys
          const int key = f.k0 + t * TA_KT + row;
          const int d = key - f.P;
          const int jmask = key >= f.total ? TA_ROWS : (d <= 0 ? 0 : (d < f.ne ? d : f.ne));
#pragma unroll
          for (int j = 0; j < TA_ROWS; ++j)
            if (j < jmask) x[j] = -INFINITY;
        }
        bool over = (t == 0);
#pragma unroll
        for (int j = 0; j < TA_ROWS; ++j) over |= x[j] > TA_TAU;
        const bool any = __any_sync(0xffffffffu, over);
        if (lane == 0) flags[sb * 4 + sw] = any ? 1 : 0;
        // Releasing the S buffer doubles as the per-tile agreement of the four
        // softmax warps: each waits for the phase their four arrivals complete.
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_empty[sb]);
        ok = __all_sync(0xffffffffu, mbar_wait(&s_empty[sb], (g >> 1) & 1, abort_flag, p.err));
        if (!ok) break;
        const bool need = flags[sb * 4] | flags[sb * 4 + 1] | flags[sb * 4 + 2] | flags[sb * 4 + 3];
        if (need) {
          // new running max: the old one raised by this tile's scores (x + max_old)
          const float* mc = m_s + (ver & 1) * TA_ROWS;
          float y[TA_ROWS];
#pragma unroll
          for (int j = 0; j < TA_ROWS; ++j) y[j] = x[j] + mc[j];
          float* rb = red + sb * 4 * TA_ROWS;
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
        }
        // probabilities: this key's row of P (queries 0..39), row sums.  They
        // depend only on S and the running max, so they are computed while the
        // previous tile's PV product may still be running.
        float e[40];
#pragma unroll
        for (int j = 0; j < TA_ROWS; ++j) {
          e[j] = fast_exp2(x[j]);
          l[j] += e[j];
        }
#pragma unroll
        for (int j = TA_ROWS; j < 40; ++j) e[j] = 0.f;
        // the PV product that last read this P buffer (and, for the rescale,
        // every earlier PV product of the unit) must be done before P is
        // rewritten and O rescaled
        if (g >= TA_PSLOTS) {
          ok = __all_sync(0xffffffffu, mbar_wait(&p_empty[g % TA_PSLOTS],
                                                 ((g / TA_PSLOTS) & 1) ^ 1, abort_flag, p.err));
          if (!ok) break;
          tc_fence_after();
        }
        if (need && TA_PSLOTS > 1 && t >= 1) {
          ok = __all_sync(0xffffffffu, mbar_wait(&p_empty[(g - 1) % TA_PSLOTS],
                                                 ((g - 1) / TA_PSLOTS) & 1, abort_flag, p.err));
          if (!ok) break;
          tc_fence_after();
        }
        if (need && t >= 1 && q4 <= 1) {
          // rescale this unit's O rows (TMEM lane = query) by their query's factor
          const int qrow = q4 * 32 + lane;
          const float a = qrow < TA_ROWS ? vals[qrow] : 1.f;
          const uint32_t oc = tmem + TA_O_COL + (seq & 1) * 64 + lane_off;
          uint32_t o32[32];
#pragma unroll 1
          for (int half = 0; half < 2; ++half) {
            tmem_ld32(oc + half * 32, o32);
            tmem_wait_ld();
#pragma unroll
            for (int ee = 0; ee < 32; ++ee) o32[ee] = __float_as_uint(__uint_as_float(o32[ee]) * a);
            tmem_st32(oc + half * 32, o32);
          }
          tmem_wait_st();
        }
#pragma unroll
        for (int c = 0; c < 5; ++c)
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(
                           prow + (g % TA_PSLOTS) * TA_P_BYTES + ((c ^ psw) << 4)),
                       "r"(pack_bf16(e[8 * c], e[8 * c + 1])), "r"(pack_bf16(e[8 * c + 2], e[8 * c + 3])),
                       "r"(pack_bf16(e[8 * c + 4], e[8 * c + 5])), "r"(pack_bf16(e[8 * c + 6], e[8 * c + 7]))
                       : "memory");
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[g % TA_PSLOTS]);
      }
      if (!ok) break;
      // the unit's last PV product
      ok = __all_sync(0xffffffffu, mbar_wait(&p_empty[(g - 1) % TA_PSLOTS],
                                             ((g - 1) / TA_PSLOTS) & 1, abort_flag, p.err));
      if (!ok) break;
      tc_fence_after();
      // per-query sums over the 128 key rows
      warp_reduce34<false>(l, red + 8 * TA_ROWS, sw, lane);
      ok = team_sync();
      if (!ok) break;
      if (sw == 0) {
        const float* rs = red + 8 * TA_ROWS;
        const float* mcur = m_s + (ver & 1) * TA_ROWS;
        for (int j = lane; j < TA_ROWS; j += 32) {
          vals[j] = rs[j] + rs[TA_ROWS + j] + rs[2 * TA_ROWS + j] + rs[3 * TA_ROWS + j];
          mfin[j] = mcur[j];
        }
      }
      ok = team_sync();
      if (!ok) break;
      const size_t unit = (static_cast<size_t>(f.i) * p.MC + f.c) * p.heads + f.h;
      // O rows (TMEM lane = query) out
      if (q4 <= 1) {
        const int qrow = q4 * 32 + lane;
        float o[64];
        uint32_t o32[32];
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          tmem_ld32(tmem + TA_O_COL + (seq & 1) * 64 + half * 32 + lane_off, o32);
          tmem_wait_ld();
#pragma unroll
          for (int q = 0; q < 32; ++q) o[half * 32 + q] = __uint_as_float(o32[q]);
        }
        if (qrow < TA_ROWS && qrow < p.q_rows) {
          const float L = vals[qrow];
          if (f.nchunks == 1) {
            const float il = L > 0.f ? 1.f / L : 0.f;
            uint4* dst = reinterpret_cast<uint4*>(
                p.out + (static_cast<size_t>(f.i) * p.q_rows + qrow) * p.H + f.h * 64);
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
            *reinterpret_cast<float2*>(p.part_ml + (unit * TA_ROWS + qrow) * 2) =
                make_float2(mfin[qrow], L);
            __threadfence();
          }
        }
      }
      // this unit's O buffer may be overwritten by the unit after next
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&o_empty[seq & 1]);
      if (f.nchunks > 1) {
        // ------------------------------------------------ split-key merge
        ok = team_sync();   // every partial of this chunk is written
        if (!ok) break;
        if (sw == 0 && lane == 0) {
          int* cnt = p.sem + static_cast<size_t>(f.i) * p.heads + f.h;
          const int prev = atomicAdd(cnt, 1);
          const bool last = prev == f.nchunks - 1;
          if (last) atomicExch(cnt, 0);
          *last_flag = last ? 1 : 0;
        }
        ok = team_sync();
        if (!ok) break;
        if (*last_flag) {
          __threadfence();
          const size_t base = (static_cast<size_t>(f.i) * p.MC) * p.heads + f.h;
          const int rows_out = p.q_rows < TA_ROWS ? p.q_rows : TA_ROWS;
          for (int w = sw * 32 + lane; w < rows_out * 4; w += 128) {
            const int rr = w >> 2, seg = (w & 3) * 16;
            float M = -INFINITY;
            for (int cc = 0; cc < f.nchunks; ++cc)
              M = fmaxf(M, p.part_ml[((base + static_cast<size_t>(cc) * p.heads) * TA_ROWS + rr) * 2]);
            float L = 0.f, acc[16];
#pragma unroll
            for (int d = 0; d < 16; ++d) acc[d] = 0.f;
            for (int cc = 0; cc < f.nchunks; ++cc) {
              const size_t u2 = base + static_cast<size_t>(cc) * p.heads;
              const float2 ml = *reinterpret_cast<const float2*>(p.part_ml + (u2 * TA_ROWS + rr) * 2);
              const float wgt = ml.x == -INFINITY ? 0.f : fast_exp2(ml.x - M);
              L += wgt * ml.y;
              const float4* src =
                  reinterpret_cast<const float4*>(p.part_o + (u2 * TA_ROWS + rr) * 64 + seg);
#pragma unroll
              for (int q4i = 0; q4i < 4; ++q4i) {
                const float4 v = src[q4i];
                acc[4 * q4i] += wgt * v.x; acc[4 * q4i + 1] += wgt * v.y;
                acc[4 * q4i + 2] += wgt * v.z; acc[4 * q4i + 3] += wgt * v.w;
              }
            }
            const float il = L > 0.f ? 1.f / L : 0.f;
            uint4* dst = reinterpret_cast<uint4*>(
                p.out + (static_cast<size_t>(f.i) * p.q_rows + rr) * p.H + f.h * 64 + seg);
            dst[0] = make_uint4(pack_bf16(acc[0] * il, acc[1] * il), pack_bf16(acc[2] * il, acc[3] * il),
                                pack_bf16(acc[4] * il, acc[5] * il), pack_bf16(acc[6] * il, acc[7] * il));
            dst[1] = make_uint4(pack_bf16(acc[8] * il, acc[9] * il), pack_bf16(acc[10] * il, acc[11] * il),
                                pack_bf16(acc[12] * il, acc[13] * il), pack_bf16(acc[14] * il, acc[15] * il));
          }
        }
      }
      cu.t = f.ntiles - 1;
      attn_step(cu, p, order_s, U);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TA_TMEM_COLS);
  }
}

}  // namespace dfm
