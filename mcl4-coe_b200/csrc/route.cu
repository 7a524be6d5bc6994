// Stable expert-major permutation with NVFP4 activation scatter, grouped-linear
// row layout, and the k-way combine.
//
// Restates the data-movement parts of SparseMoE.forward
// (src/mcl4_coe/backbone.py:895-911, loop branch :1017-1047):
//   perm   = argsort(sel.flatten(), stable=True)  -> expert-major, token order
//   out[t] = bf16(sum_j bf16(y[t, j] * bf16(w[t, j])))
// The permutation is a deterministic counting sort: the router ranks each
// chunk's slots per expert (router.cu), the scan turns per-chunk counts into
// offsets, and the scatter kernel writes every slot at
// pad_start[e] + (slots of e in earlier chunks) + rank.  Expert segments are
// padded to multiples of kSegRows rows (the GEMM's CTA-pair M tile).
#include "kernels.cuh"

namespace mcl4 {

// ---------------------------------------------------------------- permute + quantise

// Rows wider than 4096 elements.  Blocks [0, ceil(T/8)): one warp per token,
// quantise its row once and write it to its k slots, 32 blocks at a time.  Blocks after: one per expert, zero the scales of the
// padding rows of that expert's segment (zero scale => zero contribution).
__global__ void __launch_bounds__(256) permute_quant_kernel(
    const uint16_t* __restrict__ x, const uint8_t* __restrict__ valid, const int32_t* __restrict__ topk_idx,
    const float* __restrict__ topk_w, int T, int d, int E, int k, RouteWorkspace ws, int32_t* __restrict__ slot_pos,
    float* __restrict__ sorted_w, int32_t* __restrict__ perm, uint8_t* __restrict__ xq, uint8_t* __restrict__ xs) {
  __shared__ float inv_tab[128];
  fill_inverse_scale_table(inv_tab);
  __syncthreads();
  pdl_wait();     // routing and the expert layout are complete
  pdl_trigger();  // the gate/up GEMM may launch (it waits for this grid's writes)
  const int lane = threadIdx.x & 31;
  const int nblk = d / 16;
  const int token_blocks = (T + 7) / 8;
  if (int(blockIdx.x) >= token_blocks) {
    const int e = blockIdx.x - token_blocks;
    const int start = ws.pad_start[e] + ws.counts[e];
    const int end = ws.pad_start[e + 1];
    const int groups = nblk / 4;
    for (int i = threadIdx.x; i < (end - start) * groups; i += blockDim.x) {
      const int r = start + i / groups, g = i % groups;
      *reinterpret_cast<uint32_t*>(xs + rowmajor_scale_offset(uint64_t(r), uint32_t(4 * g), uint32_t(nblk))) = 0u;
    }
    return;
  }
  const int t = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (t >= T) return;
  if (valid != nullptr && valid[t] == 0) {
    if (lane < k) slot_pos[int64_t(t) * k + lane] = -1;
    return;
  }
  const int chunk = t / kRouteTokens;
  int my_pos = -1;  // slots with an expert id outside [0, E) (caller-supplied routing) are not routed
  if (lane < k) {
    const int e = topk_idx[int64_t(t) * k + lane];
    if (e >= 0 && e < E) {
      const int r = ws.local_rank[int64_t(t) * k + lane];
      const int base = ws.chunk_excl[int64_t(chunk) * E + e] + r;
      my_pos = ws.pad_start[e] + base;
      sorted_w[my_pos] = topk_w[int64_t(t) * k + lane];
      if (perm != nullptr) perm[ws.offs_start[e] + base] = t * k + lane;
    }
    slot_pos[int64_t(t) * k + lane] = my_pos;
  }
  for (int b0 = 0; b0 < nblk; b0 += 32) {
    const int b = b0 + lane;
    uint32_t s = 0;
    uint2 pk = make_uint2(0, 0);
    if (b < nblk) {
      const uint4* src = reinterpret_cast<const uint4*>(x + int64_t(t) * d + b * 16);
      uint4 u0 = __ldg(src), u1 = __ldg(src + 1);
      const uint32_t wds[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
      s = quantize_block16_bf16(wds, pk, inv_tab);
    }
    const int base_lane = lane & ~3;
    uint32_t word = 0;
#pragma unroll
    for (int q = 0; q < 4; ++q) word |= (__shfl_sync(0xffffffffu, s, base_lane + q) & 0xFFu) << (8 * q);
    for (int j = 0; j < k; ++j) {
      const int p = __shfl_sync(0xffffffffu, my_pos, j);
      if (b < nblk && p >= 0) {
        *reinterpret_cast<uint2*>(xq + int64_t(p) * (d / 2) + b * 8) = pk;
        if ((lane & 3) == 0)
          *reinterpret_cast<uint32_t*>(xs + rowmajor_scale_offset(uint64_t(p), uint32_t(b), uint32_t(nblk))) = word;
      }
    }
  }
}

// Rows of up to 32 * BPL 16-element blocks (d <= 512 * BPL): the same work as
// permute_quant_kernel with the token's whole row loaded before the routing
// lookups (which form a dependent chain of four loads) and every slot stored
// after quantising, so each warp keeps its row's loads in flight together.
template <int BPL>
__global__ void __launch_bounds__(256) permute_quant_row_kernel(
    const uint16_t* __restrict__ x, const uint8_t* __restrict__ valid, const int32_t* __restrict__ topk_idx,
    const float* __restrict__ topk_w, int T, int d, int E, int k, RouteWorkspace ws, int32_t* __restrict__ slot_pos,
    float* __restrict__ sorted_w, int32_t* __restrict__ perm, uint8_t* __restrict__ xq, uint8_t* __restrict__ xs,
    uint16_t* __restrict__ xg) {
  __shared__ float inv_tab[128];
  fill_inverse_scale_table(inv_tab);
  __syncthreads();
  pdl_wait();     // routing and the expert layout are complete
  pdl_trigger();  // the gate/up GEMM may launch (it waits for this grid's writes)
  const int lane = threadIdx.x & 31;
  const int nblk = d / 16;
  const int token_blocks = (T + 7) / 8;
  if (int(blockIdx.x) >= token_blocks) {  // zero the scales (and bf16 copies) of the expert's padding rows
    if (xs == nullptr) return;             // layout only
    const int e = blockIdx.x - token_blocks;
    const int start = ws.pad_start[e] + ws.counts[e];
    const int end = ws.pad_start[e + 1];
    const int groups = nblk / 4;
    for (int i = threadIdx.x; i < (end - start) * groups; i += blockDim.x) {
      const int r = start + i / groups, g = i % groups;
      *reinterpret_cast<uint32_t*>(xs + rowmajor_scale_offset(uint64_t(r), uint32_t(4 * g), uint32_t(nblk))) = 0u;
    }
    if (xg != nullptr) {
      const int64_t n16 = int64_t(end - start) * (d / 8);
      uint4* dst = reinterpret_cast<uint4*>(xg + int64_t(start) * d);
      for (int64_t i = threadIdx.x; i < n16; i += blockDim.x) dst[i] = make_uint4(0u, 0u, 0u, 0u);
    }
    return;
  }
  const int t = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (t >= T) return;
  if (valid != nullptr && valid[t] == 0) {
    if (lane < k) slot_pos[int64_t(t) * k + lane] = -1;
    return;
  }
  uint4 u[BPL][2];
#pragma unroll
  for (int i = 0; i < BPL; ++i) {
    const int b = lane + 32 * i;
    if (b < nblk && xq != nullptr) {
      const uint4* src = reinterpret_cast<const uint4*>(x + int64_t(t) * d + b * 16);
      u[i][0] = __ldg(src);
      u[i][1] = __ldg(src + 1);
    }
  }
  const int chunk = t / kRouteTokens;
  int my_pos = -1;  // slots with an expert id outside [0, E) (caller-supplied routing) are not routed
  if (lane < k) {
    const int e = topk_idx[int64_t(t) * k + lane];
    if (e >= 0 && e < E) {
      const int r = ws.local_rank[int64_t(t) * k + lane];
      const int base = ws.chunk_excl[int64_t(chunk) * E + e] + r;
      my_pos = ws.pad_start[e] + base;
      sorted_w[my_pos] = topk_w[int64_t(t) * k + lane];
      if (perm != nullptr) perm[ws.offs_start[e] + base] = t * k + lane;
    }
    slot_pos[int64_t(t) * k + lane] = my_pos;
  }
  if (xq == nullptr) return;  // layout only (slot positions, weights, permutation)
  uint2 pk[BPL];
  uint32_t word[BPL];
  const int base_lane = lane & ~3;
#pragma unroll
  for (int i = 0; i < BPL; ++i) {
    const int b = lane + 32 * i;
    uint32_t sc = 0;
    pk[i] = make_uint2(0, 0);
    if (b < nblk) {
      const uint32_t wds[8] = {u[i][0].x, u[i][0].y, u[i][0].z, u[i][0].w, u[i][1].x, u[i][1].y, u[i][1].z, u[i][1].w};
      sc = quantize_block16_bf16(wds, pk[i], inv_tab);
    }
    uint32_t wq = 0;
#pragma unroll
    for (int q = 0; q < 4; ++q) wq |= (__shfl_sync(0xffffffffu, sc, base_lane + q) & 0xFFu) << (8 * q);
    word[i] = wq;
  }
  for (int j = 0; j < k; ++j) {
    const int p = __shfl_sync(0xffffffffu, my_pos, j);
    if (p < 0) continue;
    uint8_t* row = xq + int64_t(p) * (d / 2);
#pragma unroll
    for (int i = 0; i < BPL; ++i) {
      const int b = lane + 32 * i;
      if (b < nblk) {
        *reinterpret_cast<uint2*>(row + b * 8) = pk[i];
        if ((lane & 3) == 0)
          *reinterpret_cast<uint32_t*>(xs + rowmajor_scale_offset(uint64_t(p), uint32_t(b), uint32_t(nblk))) =
              word[i];
        if (xg != nullptr) {  // training: the bf16 row for the weight gradient of the gate/up projection
          uint4* dst = reinterpret_cast<uint4*>(xg + int64_t(p) * d + b * 16);
          dst[0] = u[i][0];
          dst[1] = u[i][1];
        }
      }
    }
  }
}

int launch_permute_quantize(const uint16_t* x, const uint8_t* valid, const int32_t* topk_idx, const float* topk_w,
                            int T, int d, int E, int k, const RouteWorkspace& ws, int32_t* slot_pos, float* sorted_w,
                            int32_t* perm, uint8_t* xq, uint8_t* xs, cudaStream_t stream, uint16_t* xg) {
  const int blocks = (T + 7) / 8 + E;
  const int bpl = (d / 16 + 31) / 32;
  if (xg != nullptr && bpl > 8) return MCL4MOE_ERR_UNSUPPORTED;  // bf16 row copies: rows of up to 4096
  cudaError_t e;
  if (bpl <= 1)
    e = launch_pdl(permute_quant_row_kernel<1>, dim3(blocks), dim3(256), 0, stream, x, valid, topk_idx, topk_w, T, d,
                   E, k, ws, slot_pos, sorted_w, perm, xq, xs, xg);
  else if (bpl <= 2)
    e = launch_pdl(permute_quant_row_kernel<2>, dim3(blocks), dim3(256), 0, stream, x, valid, topk_idx, topk_w, T, d,
                   E, k, ws, slot_pos, sorted_w, perm, xq, xs, xg);
  else if (bpl <= 4)
    e = launch_pdl(permute_quant_row_kernel<4>, dim3(blocks), dim3(256), 0, stream, x, valid, topk_idx, topk_w, T, d,
                   E, k, ws, slot_pos, sorted_w, perm, xq, xs, xg);
  else if (bpl <= 8)
    e = launch_pdl(permute_quant_row_kernel<8>, dim3(blocks), dim3(256), 0, stream, x, valid, topk_idx, topk_w, T, d,
                   E, k, ws, slot_pos, sorted_w, perm, xq, xs, xg);
  else
    e = launch_pdl(permute_quant_kernel, dim3(blocks), dim3(256), 0, stream, x, valid, topk_idx, topk_w, T, d, E, k,
                   ws, slot_pos, sorted_w, perm, xq, xs);
  return e == cudaSuccess
             ? MCL4MOE_OK
             : MCL4MOE_ERR_CUDA;
}

// ---------------------------------------------------------------- grouped-linear helpers

__global__ void pad_from_offs_kernel(const int32_t* offs, int E, int32_t* pad_start, int32_t* offs_start,
                                     int32_t* counts) {
  if (threadIdx.x != 0) return;
  int32_t prev = 0, prun = 0;
  for (int e = 0; e < E; ++e) {
    const int32_t end = offs[e];
    const int32_t c = end - prev > 0 ? end - prev : 0;
    offs_start[e] = prev;
    counts[e] = c;
    pad_start[e] = prun;
    prun += (c + kSegRows - 1) / kSegRows * kSegRows;
    prev = end > prev ? end : prev;
  }
  pad_start[E] = prun;
}

int launch_pad_from_offs(const int32_t* offs, int E, int32_t* pad_start, int32_t* offs_start, int32_t* counts,
                         cudaStream_t stream) {
  pad_from_offs_kernel<<<1, 32, 0, stream>>>(offs, E, pad_start, offs_start, counts);
  return cudaGetLastError() == cudaSuccess ? MCL4MOE_OK : MCL4MOE_ERR_CUDA;
}

__global__ void __launch_bounds__(256) quant_grouped_rows_kernel(const uint16_t* __restrict__ x, int64_t M, int K,
                                                                 const int32_t* __restrict__ offs,
                                                                 const int32_t* __restrict__ pad_start,
                                                                 const int32_t* __restrict__ counts, int E,
                                                                 uint8_t* __restrict__ xq, uint8_t* __restrict__ xs) {
  __shared__ float inv_tab[128];
  fill_inverse_scale_table(inv_tab);
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int nblk = K / 16;
  const int64_t row_blocks = (M + 7) / 8;
  if (int64_t(blockIdx.x) >= row_blocks) {
    const int e = int(blockIdx.x - row_blocks);
    const int start = pad_start[e] + counts[e], end = pad_start[e + 1];
    const int groups = nblk / 4;
    for (int i = threadIdx.x; i < (end - start) * groups; i += blockDim.x) {
      const int r = start + i / groups, g = i % groups;
      *reinterpret_cast<uint32_t*>(xs + rowmajor_scale_offset(uint64_t(r), uint32_t(4 * g), uint32_t(nblk))) = 0u;
    }
    return;
  }
  const int64_t m = int64_t(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (m >= M) return;
  int lo = 0, hi = E;  // first e with offs[e] > m
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (offs[mid] > m) hi = mid;
    else lo = mid + 1;
  }
  if (lo >= E) return;  // row beyond the last segment
  const int e = lo;
  const int64_t start = e ? offs[e - 1] : 0;
  const int64_t p = pad_start[e] + (m - start);
  for (int b0 = 0; b0 < nblk; b0 += 32) {
    const int b = b0 + lane;
    uint32_t s = 0;
    uint2 pk = make_uint2(0, 0);
    if (b < nblk) {
      const uint4* src = reinterpret_cast<const uint4*>(x + m * K + b * 16);
      uint4 u0 = __ldg(src), u1 = __ldg(src + 1);
      const uint32_t wds[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
      s = quantize_block16_bf16(wds, pk, inv_tab);
      *reinterpret_cast<uint2*>(xq + p * (K / 2) + b * 8) = pk;
    }
    const int base_lane = lane & ~3;
    uint32_t word = 0;
#pragma unroll
    for (int q = 0; q < 4; ++q) word |= (__shfl_sync(0xffffffffu, s, base_lane + q) & 0xFFu) << (8 * q);
    if ((lane & 3) == 0 && b < nblk)
      *reinterpret_cast<uint32_t*>(xs + rowmajor_scale_offset(uint64_t(p), uint32_t(b), uint32_t(nblk))) = word;
  }
}

int launch_quantize_grouped_rows(const uint16_t* x, int64_t M, int K, const int32_t* offs, const int32_t* pad_start,
                                 const int32_t* counts, int E, uint8_t* xq, uint8_t* xs, cudaStream_t stream) {
  const int64_t blocks = (M + 7) / 8 + E;
  quant_grouped_rows_kernel<<<unsigned(blocks), 256, 0, stream>>>(x, M, K, offs, pad_start, counts, E, xq, xs);
  return cudaGetLastError() == cudaSuccess ? MCL4MOE_OK : MCL4MOE_ERR_CUDA;
}

// ---------------------------------------------------------------- combine

// One warp per token; lane handles 8 consecutive columns per step.  The k
// slot rows are summed in slot order in float32 and rounded once to bf16
// (src/mcl4_coe/backbone.py:1035-1041).
// out[t] = bf16(sum_j y[slot(t, j)]) with the k terms added in slot order in fp32
// (src/mcl4_coe/backbone.py:904-910; the routing weight is already in y).  One
// warp per token and column range: grid.y splits the row into ranges of
// cols_per_y columns, so a small batch still spreads over many warps.  BATCH
// slot pieces are loaded before they are added: 8 for small batches (few warps,
// latency-bound), 1 for large ones (bandwidth-bound; fewer registers, more warps).
// WEIGHTED: y holds unweighted rows and each slot's term is bf16(y * bf16(row_w[slot row]))
// (the training forward keeps the unweighted rows for the routing-weight gradient).
template <int BATCH, bool WEIGHTED>
__global__ void __launch_bounds__(256) combine_kernel(const uint16_t* __restrict__ y,
                                                      const int32_t* __restrict__ slot_pos,
                                                      const uint8_t* __restrict__ valid, int T, int k, int d,
                                                      int cols_per_y, uint16_t* __restrict__ out,
                                                      const float* __restrict__ row_w) {
  pdl_wait();  // the down projection's rows are complete
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (t >= T) return;
  const bool routed = valid == nullptr || valid[t] != 0;
  int my_pos = -1;
  if (routed && lane < k) my_pos = slot_pos[int64_t(t) * k + lane];
  const int c_end = min(d, int(blockIdx.y + 1) * cols_per_y);
  for (int c = int(blockIdx.y) * cols_per_y + lane * 8; c < c_end; c += 256) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (routed) {
      for (int j0 = 0; j0 < k; j0 += BATCH) {
        uint4 u[BATCH];
#pragma unroll
        for (int jj = 0; jj < BATCH; ++jj) {
          const int p = __shfl_sync(0xffffffffu, my_pos, (j0 + jj) & 31);
          u[jj] = (j0 + jj < k && p >= 0) ? __ldg(reinterpret_cast<const uint4*>(y + int64_t(p) * d + c))
                                          : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int jj = 0; jj < BATCH; ++jj) {
          if (j0 + jj >= k) break;
          const int p = __shfl_sync(0xffffffffu, my_pos, (j0 + jj) & 31);
          if (p < 0) continue;  // slot not routed (caller-supplied routing)
          uint32_t w4[4] = {u[jj].x, u[jj].y, u[jj].z, u[jj].w};
          if (WEIGHTED) {
            const float wb = round_bf16(__ldg(row_w + p));
            const uint32_t ww = pack_bf16x2(wb, wb);
#pragma unroll
            for (int i = 0; i < 4; ++i) w4[i] = bf16x2_mul(w4[i], ww);
          }
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            acc[2 * i] = __fadd_rn(acc[2 * i], bf16_to_f32(uint16_t(w4[i] & 0xFFFFu)));
            acc[2 * i + 1] = __fadd_rn(acc[2 * i + 1], bf16_to_f32(uint16_t(w4[i] >> 16)));
          }
        }
      }
    }
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
      o[i] = uint32_t(f32_to_bf16(acc[2 * i])) | (uint32_t(f32_to_bf16(acc[2 * i + 1])) << 16);
    *reinterpret_cast<uint4*>(out + int64_t(t) * d + c) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

int launch_combine(const uint16_t* y, const int32_t* slot_pos, const uint8_t* valid, int T, int k, int d, uint16_t* out,
                   cudaStream_t stream, const float* row_w) {
  if (T == 0) return MCL4MOE_OK;
  // enough warps to cover the SMs a few times: split each row into column ranges
  // (multiples of 256 columns) while the token warps alone are fewer than ~16 per SM
  const int chunks256 = d / 256;
  int split = 1;
  while (split < chunks256 && int64_t(T) * split < int64_t(16) * num_sms() && chunks256 % (2 * split) == 0) split *= 2;
  const int cols_per_y = d / split;
  const dim3 grid((T + 7) / 8, split);
  cudaError_t e;
  if (row_w != nullptr)
    e = split > 1 ? launch_pdl(combine_kernel<8, true>, grid, dim3(256), 0, stream, y, slot_pos, valid, T, k, d,
                               cols_per_y, out, row_w)
                  : launch_pdl(combine_kernel<1, true>, grid, dim3(256), 0, stream, y, slot_pos, valid, T, k, d,
                               cols_per_y, out, row_w);
  else
    e = split > 1 ? launch_pdl(combine_kernel<8, false>, grid, dim3(256), 0, stream, y, slot_pos, valid, T, k, d,
                               cols_per_y, out, row_w)
                  : launch_pdl(combine_kernel<1, false>, grid, dim3(256), 0, stream, y, slot_pos, valid, T, k, d,
                               cols_per_y, out, row_w);
  return e == cudaSuccess ? MCL4MOE_OK : MCL4MOE_ERR_CUDA;
}

}  // namespace mcl4
