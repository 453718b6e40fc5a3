// Row kernels of the patch encoder (``VAESemanticEncoder.decode_patch``,
// ``nanovllm_dots/models/dots/native/patch_encoder.py:202-235``): gathering a
// call's per-request state from its persistent cache rows, and the split-K sum
// of the output projection.
#pragma once

#include "common.cuh"

namespace dfm {

constexpr int PE_FRAMES = 16;   // latent frames per patch
constexpr int PE_LD = 64;       // latent channels
constexpr int PE_ROWS = 8;      // encoder rows per patch (stride-2 conv)

// One warp per encoder row (i, t) of the call, i < n, t < 8:
//   xc[i*8 + t] = [f(2t-1) | f(2t)]  (128 bf16: the two frames the stride-2
//   causal conv reads, ``patch_encoder.py:225-233``), where f(k) is frame k of
//   request i's patch and f(-1) the conv tail of its cache row (the previous
//   patch's last frame, zero after a reset).
// Warp (i, 0) also
//   - replaces the row's conv tail by the patch's last frame (after reading it),
//   - gathers the row's cached length: cache_len[i] = seqlens[row], n_new[i] = 8,
//     and advances seqlens[row] by 8 (``flash_patch_encoder.py:137``),
//   - writes the request's block-table line: cache row r owns pages
//     [r * pages_per_row, (r + 1) * pages_per_row) of the pool.
// A row outside [0, max_rows) or a full row is reported in err (DFM_DEVERR_PAGE /
// DFM_DEVERR_LEN); its block-table line is then -1, which every consumer
// checks, so nothing is written for it.
__global__ void __launch_bounds__(256)
    pe_prep_kernel(const __nv_bfloat16* __restrict__ patches, const int* __restrict__ rows, int n,
                   int* __restrict__ seqlens, __nv_bfloat16* __restrict__ conv_tail, int max_rows,
                   int pages_per_row, __nv_bfloat16* __restrict__ xc, int* __restrict__ cache_len,
                   int* __restrict__ n_new, int* __restrict__ block_table, uint32_t* err) {
  const int wid = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  pdl_trigger();
  pdl_wait();
  if (wid >= n * PE_ROWS) return;
  const int i = wid / PE_ROWS, t = wid - i * PE_ROWS;
  const int r = rows[i];
  const bool row_ok = r >= 0 && r < max_rows;
  // lane l: columns 4l .. 4l+3 of the 128-wide conv input row
  const int col = lane * 4;
  const int frame = 2 * t - 1 + (col >> 6);
  const int ch = col & 63;
  const __nv_bfloat16* patch = patches + static_cast<size_t>(i) * PE_FRAMES * PE_LD;
  uint2 v = make_uint2(0u, 0u);
  if (frame >= 0)
    v = *reinterpret_cast<const uint2*>(patch + frame * PE_LD + ch);
  else if (row_ok)
    v = *reinterpret_cast<const uint2*>(conv_tail + static_cast<size_t>(r) * PE_LD + ch);
  *reinterpret_cast<uint2*>(xc + static_cast<size_t>(wid) * 2 * PE_LD + col) = v;
  if (t != 0) return;
  __syncwarp();   // every lane has read the old tail
  int S = 0;
  bool ok = row_ok;
  if (row_ok) {
    if (lane < PE_LD / 4)
      *reinterpret_cast<uint2*>(conv_tail + static_cast<size_t>(r) * PE_LD + lane * 4) =
          *reinterpret_cast<const uint2*>(patch + (PE_FRAMES - 1) * PE_LD + lane * 4);
    S = seqlens[r];
    ok = S >= 0 && S + PE_ROWS <= pages_per_row * 16;
    if (!ok && lane == 0) atomicOr(err, DFM_DEV_ERR_LEN);
  } else if (lane == 0) {
    atomicOr(err, DFM_DEV_ERR_PAGE);
  }
  __syncwarp();
  if (lane == 0) {
    cache_len[i] = ok ? S : 0;
    n_new[i] = PE_ROWS;
    if (ok) seqlens[r] = S + PE_ROWS;
  }
  int* bt = block_table + static_cast<size_t>(i) * pages_per_row;
  for (int p = lane; p < pages_per_row; p += 32) bt[p] = ok ? r * pages_per_row + p : -1;
}

// out[i][c] = bf16(sum_s part[s][i][c]) over the ksplit partial planes of the
// output projection (the bias is in plane 0).  One thread per 4 columns.
__global__ void __launch_bounds__(256)
    pe_out_reduce_kernel(const float* __restrict__ part, int ksplit, size_t plane, int n, int cols,
                         __nv_bfloat16* __restrict__ out) {
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  pdl_trigger();
  pdl_wait();
  const int c4 = cols / 4;
  if (idx >= n * c4) return;
  const int i = idx / c4, c = (idx - i * c4) * 4;
  const size_t off = static_cast<size_t>(i) * cols + c;
  float4 a = *reinterpret_cast<const float4*>(part + off);
  for (int s = 1; s < ksplit; ++s) {
    const float4 b = *reinterpret_cast<const float4*>(part + s * plane + off);
    a.x += b.x; a.y += b.y; a.z += b.z; a.w += b.w;
  }
  *reinterpret_cast<uint2*>(out + off) = make_uint2(pack_bf16(a.x, a.y), pack_bf16(a.z, a.w));
}

}  // namespace dfm
