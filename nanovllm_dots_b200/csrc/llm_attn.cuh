// Paged GQA decode attention of the LLM backbone (one new token per sequence),
// the B200 replacement for the decode branch of the reference's Attention
// layer (``nanovllm_dots/layers/attention.py:60-97``): the token's K/V are
// stored into the paged cache at its slot (``store_kvcache``,
// ``attention.py:10-47``), then the token's query heads attend over the
// sequence's ``context_len`` cached positions (``flash_attn_with_kvcache`` with
// ``cache_seqlens``, ``block_table``, ``causal=True``: one query at the last
// position sees every cached key).
//
// Cache layout (the reference's, ``batched_llm.py:57-66``): k_cache / v_cache
// bf16 [num_blocks][block_size][kv_heads][D]; position p of sequence i lives at
// block block_table[i][p / block_size], row p % block_size.
//
// Work unit = (sequence, kv head, chunk of LA_CHUNK keys): the G = heads /
// kv_heads query heads that share the kv head are computed together, so every
// K/V byte is read once per step.  Decode is HBM-bound (6 FLOP per cache byte
// at G = 6), so the arithmetic runs on the CUDA cores; the data moves by TMA:
// 64-key sub-tiles of K and V (one 128-byte-swizzled box per 64 dims),
// double-buffered when a unit spans several, issued by one thread and completed
// on an mbarrier.  Per
// sub-tile the 128 threads
//   1. score: two threads per key, each over half the dims (16-byte swizzled
//      loads: 4 shared-memory wavefronts per warp, the minimum), all G queries;
//   2. online softmax: one warp per query (two when G > 4), lanes over keys;
//   3. PV: one thread per output dim (D = 128) or per dim and query parity
//      (D = 64), all queries, rescaling its accumulators by the max update.
// The unnormalised partial (acc, m, l) of each chunk goes to the workspace and
// llm_attn_combine_kernel merges a sequence's chunks.  Every wait is bounded.
#pragma once

#include "common.cuh"

namespace dfm {

constexpr int LA_SUB = 64;        // keys per sub-tile (TMA box rows)
constexpr int LA_CHUNK = 128;     // keys per work unit (measured best of 64, 128 and 512; merging
                                  // in the last unit instead of llm_attn_combine_kernel was slower)
constexpr int LA_NBUF = LA_CHUNK > LA_SUB ? 2 : 1;   // K/V sub-tile buffers
constexpr int LA_THREADS = 128;
constexpr int LA_MAXG = 8;        // query heads per kv head

template <int D>
struct LlmAttnSmem {
  static constexpr int BOXES = D / 64;                       // 64-dim boxes per key row
  static constexpr int TILE_BYTES = LA_SUB * D * 2;          // one K or V sub-tile
  static constexpr int OFF_K = 0;                            // [LA_NBUF] K buffers
  static constexpr int OFF_V = OFF_K + LA_NBUF * TILE_BYTES; // [LA_NBUF] V buffers
  static constexpr int OFF_Q = OFF_V + LA_NBUF * TILE_BYTES; // float [LA_MAXG][D]
  static constexpr int OFF_S = OFF_Q + LA_MAXG * D * 4;      // float [2][LA_MAXG][LA_SUB]
  // P [LA_MAXG][LA_SUB] overlays the first half of the score partials: each
  // softmax lane writes the probabilities of the keys whose scores it read
  static constexpr int OFF_P = OFF_S;
  static constexpr int OFF_ML = OFF_S + 2 * LA_MAXG * LA_SUB * 4; // float [3][LA_MAXG]: m, l, alpha
  static constexpr int OFF_BAR = OFF_ML + 3 * LA_MAXG * 4 + 32;   // uint64 [LA_NBUF] + abort flag
  static constexpr int BYTES = OFF_BAR + 64 + 1024;               // + 1 KB alignment slack
};
// three CTAs per SM at head_dim 128 (dynamic shared memory + the 1 KB the
// runtime reserves per CTA)
static_assert(3 * (LlmAttnSmem<128>::BYTES + 1024) <= 233472, "three decode CTAs per SM");

struct LlmAttnParams {
  const __nv_bfloat16* q;   // [n][H][D]
  const int* context_lens;  // [n]
  const int* block_table;   // [n][max_blocks]
  float* part_o;            // [n][H][max_chunks][D]
  float* part_ml;           // [n][H][max_chunks][2]
  int n, H, KVH, G, max_blocks, num_blocks, block_size, max_chunks;
  float scale_log2;         // softmax scale * log2(e)
  uint32_t* err;
};

// Store this step's K/V rows into the paged caches: one thread per 16 bytes.
// slot < 0 skips the row (the reference's -1 convention); a slot past the
// cache is reported and skipped.
__global__ void __launch_bounds__(256)
    llm_store_kv_kernel(const __nv_bfloat16* __restrict__ k, const __nv_bfloat16* __restrict__ v,
                        __nv_bfloat16* __restrict__ k_cache, __nv_bfloat16* __restrict__ v_cache,
                        const int* __restrict__ slot_mapping, int n, int row_elems,
                        long long num_slots, uint32_t* err) {
  const int per_row = row_elems / 8;
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  pdl_trigger();
  pdl_wait();
  if (idx >= 2 * n * per_row) return;
  const int kv = idx / (n * per_row);
  const int rem = idx - kv * n * per_row;
  const int i = rem / per_row, c = rem - i * per_row;
  const int slot = slot_mapping[i];
  if (slot < 0) return;
  if (slot >= num_slots) {
    if (c == 0) atomicOr(err, DFM_DEV_ERR_PAGE);
    return;
  }
  const __nv_bfloat16* src = (kv ? v : k) + static_cast<size_t>(i) * row_elems + c * 8;
  __nv_bfloat16* dst = (kv ? v_cache : k_cache) + static_cast<size_t>(slot) * row_elems + c * 8;
  *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(src);
}

template <int D>
__global__ void __launch_bounds__(LA_THREADS)
    llm_decode_attn_kernel(const __grid_constant__ CUtensorMap tm_k,
                           const __grid_constant__ CUtensorMap tm_v, LlmAttnParams p) {
  static_assert(D == 64 || D == 128, "head_dim 64 or 128");
  using S = LlmAttnSmem<D>;
  pdl_trigger();
  if (threadIdx.x == 0) {
    tma_prefetch(&tm_k);
    tma_prefetch(&tm_v);
  }
  pdl_wait();
  const int c = blockIdx.x, g = blockIdx.y, i = blockIdx.z;
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int k0 = c * LA_CHUNK;
  const int* bt = p.block_table + static_cast<size_t>(i) * p.max_blocks;
  // the block ids of the first sub-tiles depend only on the chunk: read them
  // together with the context length instead of after it
  int blk0[LA_NBUF];
  if (t == 0) {
#pragma unroll
    for (int j = 0; j < LA_NBUF; ++j) {
      const int bi = (k0 + j * LA_SUB) / p.block_size;
      blk0[j] = bi < p.max_blocks ? bt[bi] : -1;
    }
  }
  const int ctx = p.context_lens[i];
  if (ctx < 1 || ctx > p.max_blocks * p.block_size) {
    if (c == 0 && g == 0 && t == 0) atomicOr(p.err, DFM_DEV_ERR_LEN);
    return;
  }
  if (k0 >= ctx) return;   // this chunk lies past the sequence (uniform over the CTA)
  const int k1 = min(ctx, k0 + LA_CHUNK);
  const int nsub = (k1 - k0 + LA_SUB - 1) / LA_SUB;
  const int G = p.G;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sK = smem + S::OFF_K;
  uint8_t* sV = smem + S::OFF_V;
  float* sq = reinterpret_cast<float*>(smem + S::OFF_Q);
  float* s_part = reinterpret_cast<float*>(smem + S::OFF_S);
  float* s_p = reinterpret_cast<float*>(smem + S::OFF_P);
  float* m_s = reinterpret_cast<float*>(smem + S::OFF_ML);
  float* l_s = m_s + LA_MAXG;
  float* al_s = l_s + LA_MAXG;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::OFF_BAR);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(full + LA_NBUF);

  // one sub-tile: D / 64 boxes of K and of V for keys [kk, kk + 64) of this chunk
  auto issue = [&](int j, int blk) {
    const int key = k0 + j * LA_SUB;
    const int bi = key / p.block_size;
    if (blk < 0 || blk >= p.num_blocks) {
      atomicOr(p.err, DFM_DEV_ERR_PAGE);
      blk = p.num_blocks;   // out of range: TMA fills zeros
    }
    const int row = key - bi * p.block_size;
    const int buf = j % LA_NBUF;
    uint64_t* bar = &full[buf];
    mbar_arrive_expect_tx(bar, 2 * S::TILE_BYTES);
#pragma unroll
    for (int b = 0; b < S::BOXES; ++b) {
      tma_load_4d(sK + buf * S::TILE_BYTES + b * LA_SUB * 128, &tm_k, bar, b * 64, g, row, blk);
      tma_load_4d(sV + buf * S::TILE_BYTES + b * LA_SUB * 128, &tm_v, bar, b * 64, g, row, blk);
    }
  };
  if (t == 0) {
    for (int b = 0; b < LA_NBUF; ++b) mbar_init(&full[b], 1);
    *abort_flag = 0;
    fence_mbar_init();
#pragma unroll
    for (int j = 0; j < LA_NBUF; ++j)
      if (j < nsub) issue(j, blk0[j]);
  }
  // the group's queries, pre-scaled into log2 units
  const __nv_bfloat16* qg = p.q + (static_cast<size_t>(i) * p.H + g * G) * D;
  for (int x = t; x < G * D; x += LA_THREADS) sq[x] = __bfloat162float(qg[x]) * p.scale_log2;
  if (t < LA_MAXG) {
    m_s[t] = -INFINITY;
    l_s[t] = 0.f;
  }
  __syncthreads();

  // PV mapping: D = 128: dim t, every query; D = 64: dim t % 64, queries of parity t / 64
  const int pv_dim = t % D;
  const int pv_q0 = D == 128 ? 0 : t / 64;
  const int pv_qs = D == 128 ? 1 : 2;
  float acc[LA_MAXG];
#pragma unroll
  for (int q = 0; q < LA_MAXG; ++q) acc[q] = 0.f;

  // score mapping: key kk = t % 64, dims [half * D / 2, (half + 1) * D / 2)
  const int kk = t & (LA_SUB - 1), half = t >> 6;
  bool ok = true;
#pragma unroll 1
  for (int j = 0; j < nsub; ++j) {
    ok = mbar_wait(&full[j % LA_NBUF], (j / LA_NBUF) & 1, abort_flag, p.err);
    if (!ok) break;
    const uint8_t* kt = sK + (j % LA_NBUF) * S::TILE_BYTES;
    const uint8_t* vt = sV + (j % LA_NBUF) * S::TILE_BYTES;
    // ---- 1. scores
    {
      float sc[LA_MAXG];
#pragma unroll
      for (int q = 0; q < LA_MAXG; ++q) sc[q] = 0.f;
      constexpr int CH = D / 16;   // 16-byte chunks per half row
#pragma unroll
      for (int cc = 0; cc < CH; ++cc) {
        const int chunk = half * CH + cc;        // 0 .. D/8 - 1 over the whole row
        const int box = chunk >> 3, cin = chunk & 7;
        const uint4 kv = *reinterpret_cast<const uint4*>(kt + box * LA_SUB * 128 + kk * 128 +
                                                         ((cin ^ (kk & 7)) << 4));
        const __nv_bfloat162* k2 = reinterpret_cast<const __nv_bfloat162*>(&kv);
        float kf[8];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __bfloat1622float2(k2[e]);
          kf[2 * e] = f.x;
          kf[2 * e + 1] = f.y;
        }
        const int d0 = chunk * 8;
#pragma unroll
        for (int q = 0; q < LA_MAXG; ++q) {
          if (q < G) {
            const float4 qa = *reinterpret_cast<const float4*>(sq + q * D + d0);
            const float4 qb = *reinterpret_cast<const float4*>(sq + q * D + d0 + 4);
            sc[q] += kf[0] * qa.x + kf[1] * qa.y + kf[2] * qa.z + kf[3] * qa.w +
                     kf[4] * qb.x + kf[5] * qb.y + kf[6] * qb.z + kf[7] * qb.w;
          }
        }
      }
#pragma unroll
      for (int q = 0; q < LA_MAXG; ++q)
        if (q < G) s_part[(half * LA_MAXG + q) * LA_SUB + kk] = sc[q];
    }
    __syncthreads();
    // ---- 2. online softmax, one warp per query
    const int key_base = k0 + j * LA_SUB;
    for (int q = warp; q < G; q += LA_THREADS / 32) {
      float s0 = s_part[q * LA_SUB + lane] + s_part[(LA_MAXG + q) * LA_SUB + lane];
      float s1 = s_part[q * LA_SUB + lane + 32] + s_part[(LA_MAXG + q) * LA_SUB + lane + 32];
      if (key_base + lane >= k1) s0 = -INFINITY;
      if (key_base + lane + 32 >= k1) s1 = -INFINITY;
      const float m_old = m_s[q];
      const float m_new = fmaxf(m_old, warp_max(fmaxf(s0, s1)));
      // m_new is finite: every sub-tile holds at least one unmasked key
      const float p0 = fast_exp2(s0 - m_new), p1 = fast_exp2(s1 - m_new);
      const float alpha = fast_exp2(m_old - m_new);   // 0 on the first sub-tile
      const float ps = warp_sum(p0 + p1);
      s_p[q * LA_SUB + lane] = p0;
      s_p[q * LA_SUB + lane + 32] = p1;
      if (lane == 0) {
        m_s[q] = m_new;
        l_s[q] = l_s[q] * alpha + ps;
        al_s[q] = alpha;
      }
    }
    __syncthreads();
    // ---- 3. acc = acc * alpha + P V over the sub-tile's valid keys only: rows
    // past the sequence hold whatever the cache held (possibly not finite)
    {
      const int box = pv_dim >> 6, din = pv_dim & 63;
      const uint8_t* vcol = vt + box * LA_SUB * 128 + (din & 7) * 2;
      const int cin = din >> 3;
      const int kvalid = min(LA_SUB, k1 - key_base);
      float a[LA_MAXG];
#pragma unroll
      for (int q = 0; q < LA_MAXG; ++q) a[q] = 0.f;
#pragma unroll 4
      for (int k = 0; k < kvalid; ++k) {
        const float vv = __bfloat162float(
            *reinterpret_cast<const __nv_bfloat16*>(vcol + k * 128 + ((cin ^ (k & 7)) << 4)));
#pragma unroll
        for (int q = 0; q < LA_MAXG; ++q) {
          const int qq = pv_q0 + q * pv_qs;
          if (q * pv_qs < LA_MAXG && qq < G) a[q] += s_p[qq * LA_SUB + k] * vv;
        }
      }
#pragma unroll
      for (int q = 0; q < LA_MAXG; ++q) {
        const int qq = pv_q0 + q * pv_qs;
        if (q * pv_qs < LA_MAXG && qq < G) acc[q] = acc[q] * al_s[qq] + a[q];
      }
    }
    __syncthreads();   // buffer j % LA_NBUF, s_part and s_p are free again
    if (t == 0 && j + LA_NBUF < nsub)
      issue(j + LA_NBUF, bt[(k0 + (j + LA_NBUF) * LA_SUB) / p.block_size]);
  }
  if (!ok) return;
  // ---- unnormalised partial of this chunk
  const size_t row0 = static_cast<size_t>(i) * p.H + g * G;
#pragma unroll
  for (int q = 0; q < LA_MAXG; ++q) {
    const int qq = pv_q0 + q * pv_qs;
    if (q * pv_qs < LA_MAXG && qq < G)
      p.part_o[((row0 + qq) * p.max_chunks + c) * D + pv_dim] = acc[q];
  }
  if (t < G) {
    float* ml = p.part_ml + ((row0 + t) * p.max_chunks + c) * 2;
    ml[0] = m_s[t];
    ml[1] = l_s[t];
  }
}

// out[i][h] = sum_c 2^(m_c - M) acc_c / sum_c 2^(m_c - M) l_c over the chunks
// of sequence i; one block of D threads per (sequence, query head).  The
// chunks' partials are read eight at a time, every load of a batch in flight
// at once (one batch up to 1024 keys: the same sums, in the same order, as a
// single pass with M the maximum over all chunks).
template <int D>
__global__ void __launch_bounds__(D)
    llm_attn_combine_kernel(const float* __restrict__ part_o, const float* __restrict__ part_ml,
                            const int* __restrict__ context_lens, int H, int max_chunks,
                            int max_keys, __nv_bfloat16* __restrict__ out) {
  constexpr int CB = 8;
  const int row = blockIdx.x;            // i * H + h
  const int i = row / H;
  pdl_trigger();
  pdl_wait();
  const int ctx = context_lens[i];
  const int nch = (ctx < 1 || ctx > max_keys) ? 0 : (ctx + LA_CHUNK - 1) / LA_CHUNK;
  const float* ml = part_ml + static_cast<size_t>(row) * max_chunks * 2;
  const float* po = part_o + static_cast<size_t>(row) * max_chunks * D + threadIdx.x;
  float M = -INFINITY, L = 0.f, a = 0.f;
  for (int c0 = 0; c0 < nch; c0 += CB) {
    float m[CB], l[CB], o[CB];
#pragma unroll
    for (int j = 0; j < CB; ++j) {
      const bool v = c0 + j < nch;
      m[j] = v ? ml[2 * (c0 + j)] : -INFINITY;
      l[j] = v ? ml[2 * (c0 + j) + 1] : 0.f;
      o[j] = v ? po[static_cast<size_t>(c0 + j) * D] : 0.f;
    }
    float Mn = M;
#pragma unroll
    for (int j = 0; j < CB; ++j) Mn = fmaxf(Mn, m[j]);
    const float sc = M == -INFINITY ? 0.f : fast_exp2(M - Mn);
    L *= sc;
    a *= sc;
#pragma unroll
    for (int j = 0; j < CB; ++j) {
      const float w = fast_exp2(m[j] - Mn);
      L += w * l[j];
      a += w * o[j];
    }
    M = Mn;
  }
  out[static_cast<size_t>(row) * D + threadIdx.x] = __float2bfloat16(L > 0.f ? a / L : 0.f);
}

}  // namespace dfm
