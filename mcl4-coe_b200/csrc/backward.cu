// Backward of the MoE layer: the gradient kernels around the two grouped NVFP4
// input-gradient GEMMs (which run on the tcgen05 kernel of gemm_fp4.cu).
//
// Restates the reference's autograd path through SparseMoE.forward's grouped
// branch (src/mcl4_coe/backbone.py:853-911) and _NVFP4GroupedLinear.backward
// (src/mcl4_coe/nvfp4.py:1112-1216):
//   slot rows      d_y = bf16(d_out[t] * bf16(w)),  d_w = bf16(sum_c bf16(d_out[t,c] * y[c]))
//   quantisation   stochastic-rounded NVFP4 rows with a tensor-wise global scale
//                  (the STOCHASTIC branch of _nvfp4_quantize_1d_kernel, :735-790,
//                  launched at :1128-1151), noise = Philox4x32-10 as Triton's tl.rand
//   input grads    grouped NVFP4 GEMM on the transposed weight copy (:1152-1170)
//   SwiGLU         d_val = bf16(d_h * bf16(silu(g))), d_gate = silu'(g) * bf16(d_h * val)
//   router         softmax / top-k / renormalisation / auxiliary-loss / z-loss derivatives
//   input          d_x[t] = bf16(sum_j d_rows[slot(t, j)] + d_x_router[t])
// Rows are the padded expert-major rows of the forward (pad_start / counts);
// the noise of a row uses its index in the reference's unpadded layout
// (offs_start[e] + local), so the stochastic codes are the reference's.
#include "kernels.cuh"
#include "sr.cuh"

namespace mcl4 {

namespace {

// One 16-element block of bf16 values (8 packed words) quantised with stochastic
// rounding: scale byte returned, 8 packed bytes written.  off0: noise offset of
// the block's first element.
__device__ __forceinline__ uint32_t sr_block16(const uint32_t (&w)[8], float g, uint32_t k0, uint32_t k1,
                                               uint32_t off0, uint2& packed) {
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fmaxf(fabsf(bf16x2_lo(w[i])), fabsf(bf16x2_hi(w[i]))));
  const uint32_t s = f32_to_e4m3(fminf(__fdiv_rn(amax, __fmul_rn(6.0f, g)), 448.0f));
  const float dec = __fmul_rn(e4m3_to_f32(s), g);
  const float inv = dec > 0.f ? __fdiv_rn(1.0f, dec) : 0.f;
  uint32_t lo = 0u, hi = 0u;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const float x = __fmul_rn((i & 1) ? bf16x2_hi(w[i >> 1]) : bf16x2_lo(w[i >> 1]), inv);
    const float m = fminf(fabsf(x), 6.0f);
    const float u = m <= 2.0f ? __fmul_rn(m, 2.0f) : (m <= 4.0f ? __fadd_rn(m, 2.0f) : __fadd_rn(__fmul_rn(m, 0.5f), 4.0f));
    const float r = __fadd_rn(u, uniform_from_word(philox_word0(off0 + uint32_t(i), k0, k1)));
    uint32_t code = r >= 0.f ? static_cast<uint32_t>(r) : 0u;  // truncation, as the kernel's cast to uint8
    code = min(code, 7u) | (x < 0.f ? 8u : 0u);
    if (i < 8) lo |= code << (4 * i);
    else hi |= code << (4 * (i - 8));
  }
  packed = make_uint2(lo, hi);
  return s;
}

// Row of the padded expert-major layout -> (live, index in the reference's unpadded layout).
struct RowMap {
  const int32_t* pad_start;   // [E + 1], or nullptr: rows are the reference's rows
  const int32_t* counts;      // [E]
  const int32_t* offs_start;  // [E]
  int E;
};

__device__ __forceinline__ bool map_row(const RowMap& m, int64_t p, int64_t& ref_row) {
  if (m.pad_start == nullptr) {
    ref_row = p;
    return true;
  }
  int lo = 0, hi = m.E + 1;  // upper_bound(pad_start, p) - 1
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (m.pad_start[mid] <= p) lo = mid + 1;
    else hi = mid;
  }
  const int e = lo - 1;
  if (e < 0 || e >= m.E) return false;
  const int64_t local = p - m.pad_start[e];
  ref_row = int64_t(m.offs_start[e]) + local;
  return local < m.counts[e];
}

__device__ __forceinline__ float global_scale_from_amax(float a) {
  // src/mcl4_coe/nvfp4.py:1129-1134: max(amax > 0 ? amax / 2688 : 1, FLT_MIN)
  return fmaxf(a > 0.f ? __fdiv_rn(a, 2688.0f) : 1.0f, kFltMinNormal);
}

}  // namespace

// amax of a bf16 matrix (non-negative float bits order like integers).
__global__ void __launch_bounds__(256) bf16_amax_kernel(const uint16_t* __restrict__ x, int64_t n8, float* amax) {
  float m = 0.f;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n8; i += int64_t(gridDim.x) * blockDim.x) {
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(x) + i);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) m = fmaxf(m, fmaxf(fabsf(bf16x2_lo(w[j])), fabsf(bf16x2_hi(w[j]))));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) atomicMax(reinterpret_cast<unsigned int*>(amax), __float_as_uint(m));
}

// Stochastic-rounding NVFP4 rows: one warp per row, lanes over 16-element blocks.
// Writes packed [rows, cols/2], E4M3 scales row-major [rows, cols/16] and (block 0)
// the global scale.  Rows that are padding of an expert segment get zero codes and
// scales; rows at or beyond pad_start[E] are not touched.
__global__ void __launch_bounds__(256) sr_quant_kernel(const uint16_t* __restrict__ x, int64_t rows, int cols,
                                                       const float* __restrict__ amax, uint32_t k0, uint32_t k1,
                                                       RowMap map, uint8_t* __restrict__ packed,
                                                       uint8_t* __restrict__ scales, float* g_out) {
  const float g = global_scale_from_amax(*amax);
  if (blockIdx.x == 0 && threadIdx.x == 0 && g_out != nullptr) *g_out = g;
  const int lane = threadIdx.x & 31;
  const int64_t p = int64_t(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (p >= rows) return;
  if (map.pad_start != nullptr && p >= map.pad_start[map.E]) return;
  int64_t ref_row = 0;
  const bool live = map_row(map, p, ref_row);
  const int nblk = cols / 16;
  const uint32_t row_off = uint32_t(uint64_t(ref_row) * uint64_t(cols));  // 32-bit wrap, as the reference's int32
  for (int b = lane; b < nblk; b += 32) {
    uint2 pk = make_uint2(0u, 0u);
    uint32_t s = 0u;
    if (live) {
      const uint4* src = reinterpret_cast<const uint4*>(x + p * cols + b * 16);
      const uint4 u0 = __ldg(src), u1 = __ldg(src + 1);
      const uint32_t w[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
      s = sr_block16(w, g, k0, k1, row_off + uint32_t(b * 16), pk);
    }
    *reinterpret_cast<uint2*>(packed + p * (cols / 2) + b * 8) = pk;
    scales[p * nblk + b] = uint8_t(s);
  }
}

// Slot rows of the down projection's output gradient.  Blocks [0, ceil(T*k/8)):
// one warp per slot (t, j): d_y[p] = bf16(d_out[t] * bf16(w)) and the routing-weight
// gradient d_w = bf16(sum_c bf16(d_out[t, c] * y[p, c])) (float32 sum in a fixed
// order); the largest |d_y| goes to amax.  Blocks after: one per expert, zero
// d_y's padding rows.
__global__ void __launch_bounds__(256) slot_grad_kernel(const uint16_t* __restrict__ d_out,
                                                        const uint16_t* __restrict__ y,
                                                        const int32_t* __restrict__ slot_pos,
                                                        const float* __restrict__ topk_w, int T, int k, int d,
                                                        const int32_t* __restrict__ pad_start,
                                                        const int32_t* __restrict__ counts, uint16_t* __restrict__ d_y,
                                                        float* __restrict__ d_w, float* amax) {
  const int lane = threadIdx.x & 31;
  const int64_t slot_blocks = (int64_t(T) * k + 7) / 8;
  if (int64_t(blockIdx.x) >= slot_blocks) {
    const int e = int(blockIdx.x - slot_blocks);
    const int64_t start = pad_start[e] + counts[e], end = pad_start[e + 1];
    uint4* dst = reinterpret_cast<uint4*>(d_y + start * d);
    const int64_t n16 = (end - start) * (d / 8);
    for (int64_t i = threadIdx.x; i < n16; i += blockDim.x) dst[i] = make_uint4(0u, 0u, 0u, 0u);
    return;
  }
  const int64_t s = int64_t(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (s >= int64_t(T) * k) return;
  const int64_t t = s / k;
  const int p = slot_pos[s];
  if (p < 0) {
    if (lane == 0) d_w[s] = 0.f;
    return;
  }
  const float wb = round_bf16(topk_w[s]);
  const uint32_t ww = pack_bf16x2(wb, wb);
  float acc = 0.f, mx = 0.f;
  // four 256-column steps per pass: all eight 16-byte loads are in flight before the math
  for (int c0 = lane * 8; c0 < d; c0 += 1024) {
    uint4 g[4], yv[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int c = c0 + u * 256;
      if (c < d) {
        g[u] = __ldg(reinterpret_cast<const uint4*>(d_out + t * d + c));
        yv[u] = __ldg(reinterpret_cast<const uint4*>(y + int64_t(p) * d + c));
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int c = c0 + u * 256;
      if (c >= d) break;
      const uint32_t gw[4] = {g[u].x, g[u].y, g[u].z, g[u].w}, yw[4] = {yv[u].x, yv[u].y, yv[u].z, yv[u].w};
      uint32_t o[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        o[i] = bf16x2_mul(gw[i], ww);
        const uint32_t pr = bf16x2_mul(gw[i], yw[i]);
        acc = __fadd_rn(__fadd_rn(acc, bf16x2_lo(pr)), bf16x2_hi(pr));
        mx = fmaxf(mx, fmaxf(fabsf(bf16x2_lo(o[i])), fabsf(bf16x2_hi(o[i]))));
      }
      *reinterpret_cast<uint4*>(d_y + int64_t(p) * d + c) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, o));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  }
  if (lane == 0) {
    d_w[s] = round_bf16(acc);
    atomicMax(reinterpret_cast<unsigned int*>(amax), __float_as_uint(mx));
  }
}

// SwiGLU derivative (torch's silu backward: dy * s * (1 + x (1 - s)), s = sigmoid(x),
// in float32): one warp per padded row below pad_start[E], lanes over 8 columns.
// up holds [gate | value] (bf16), d_h the gradient of h = bf16(bf16(silu(gate)) * value).
__global__ void __launch_bounds__(256) swiglu_bwd_kernel(const uint16_t* __restrict__ d_h,
                                                         const uint16_t* __restrict__ up, int64_t rows_cap,
                                                         const int32_t* __restrict__ pad_end, int F,
                                                         uint16_t* __restrict__ d_up, float* amax) {
  const int lane = threadIdx.x & 31;
  const int64_t p = int64_t(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (p >= rows_cap || p >= *pad_end) return;
  float mx = 0.f;
  for (int c = lane * 8; c < F; c += 256) {
    const uint4 dh = __ldg(reinterpret_cast<const uint4*>(d_h + p * F + c));
    const uint4 gt = __ldg(reinterpret_cast<const uint4*>(up + p * 2 * F + c));
    const uint4 vl = __ldg(reinterpret_cast<const uint4*>(up + p * 2 * F + F + c));
    const uint32_t dw[4] = {dh.x, dh.y, dh.z, dh.w}, gw[4] = {gt.x, gt.y, gt.z, gt.w}, vw[4] = {vl.x, vl.y, vl.z, vl.w};
    uint32_t og[4], ov[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float dg[2], dv[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const float dhv = h ? bf16x2_hi(dw[i]) : bf16x2_lo(dw[i]);
        const float gv = h ? bf16x2_hi(gw[i]) : bf16x2_lo(gw[i]);
        const float vv = h ? bf16x2_hi(vw[i]) : bf16x2_lo(vw[i]);
        const float sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-gv)));
        const float silu = round_bf16(__fdiv_rn(gv, __fadd_rn(1.0f, expf(-gv))));
        const float d_silu = round_bf16(__fmul_rn(dhv, vv));
        dv[h] = round_bf16(__fmul_rn(dhv, silu));
        dg[h] = round_bf16(__fmul_rn(__fmul_rn(d_silu, sig), __fadd_rn(1.0f, __fmul_rn(gv, __fsub_rn(1.0f, sig)))));
        mx = fmaxf(mx, fmaxf(fabsf(dg[h]), fabsf(dv[h])));
      }
      og[i] = pack_bf16x2(dg[0], dg[1]);
      ov[i] = pack_bf16x2(dv[0], dv[1]);
    }
    *reinterpret_cast<uint4*>(d_up + p * 2 * F + c) = make_uint4(og[0], og[1], og[2], og[3]);
    *reinterpret_cast<uint4*>(d_up + p * 2 * F + F + c) = make_uint4(ov[0], ov[1], ov[2], ov[3]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) atomicMax(reinterpret_cast<unsigned int*>(amax), __float_as_uint(mx));
}

// Router derivative, one warp per token (E <= 256: lane l holds experts l + 32 i).
// src/mcl4_coe/backbone.py:787-883: probs = softmax(logits); weights = top-k probs,
// renormalised by max(sum, 1e-9) when norm; aux = E * sum_e counts_e * mean_t probs;
// z = mean_t logsumexp^2 (means over the n routed tokens; masked tokens get zeros).
template <int EW>
__global__ void __launch_bounds__(256) router_bwd_kernel(const float* __restrict__ logits,
                                                         const int32_t* __restrict__ topk_idx,
                                                         const float* __restrict__ topk_w,
                                                         const float* __restrict__ d_w,
                                                         const uint8_t* __restrict__ valid,
                                                         const float* __restrict__ stats, const float* d_aux,
                                                         const float* d_z, int T, int E, int k, int norm,
                                                         float* __restrict__ d_logits) {
  const int lane = threadIdx.x & 31;
  const int64_t t = int64_t(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (t >= T) return;
  float* out = d_logits + t * E;
  if (valid != nullptr && valid[t] == 0) {
    for (int e = lane; e < E; e += 32) out[e] = 0.f;
    return;
  }
  const float* row = logits + t * E;
  float l[EW], p[EW];
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < EW; ++i) {
    const int e = lane + 32 * i;
    l[i] = e < E ? row[e] : -INFINITY;
    mx = fmaxf(mx, l[i]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < EW; ++i) {
    p[i] = lane + 32 * i < E ? expf(__fsub_rn(l[i], mx)) : 0.f;
    sum = __fadd_rn(sum, p[i]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, o));
  const float inv = __fdiv_rn(1.0f, sum);
#pragma unroll
  for (int i = 0; i < EW; ++i) p[i] = __fmul_rn(p[i], inv);
  const float lse = __fadd_rn(mx, logf(sum));
  const float n = fmaxf(stats[2], 1.0f);
  const float da = d_aux != nullptr ? *d_aux : 0.f;
  const float dz = d_z != nullptr ? *d_z : 0.f;
  // slot j on lane j: top-k value v_j = probs[idx_j], weight w_j, upstream d_w_j
  int idx = -1;
  float v = 0.f, w = 0.f, dw = 0.f;
  if (lane < k) {
    idx = topk_idx[t * k + lane];
    w = topk_w[t * k + lane];
    dw = d_w[t * k + lane];
    if (idx >= 0 && idx < E) v = __fmul_rn(expf(__fsub_rn(row[idx], mx)), inv);
  }
  float dv = dw;
  if (norm) {
    float S = v, dot = __fmul_rn(dw, w);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      S = __fadd_rn(S, __shfl_xor_sync(0xffffffffu, S, o));
      dot = __fadd_rn(dot, __shfl_xor_sync(0xffffffffu, dot, o));
    }
    // w_j = v_j / max(S, 1e-9): below the clamp the denominator is a constant
    dv = S > 1e-9f ? __fdiv_rn(__fsub_rn(dw, dot), S) : __fdiv_rn(dw, 1e-9f);
  }
  float dp[EW];
  const float aux_scale = __fdiv_rn(__fmul_rn(da, float(E)), n);
#pragma unroll
  for (int i = 0; i < EW; ++i) {
    const int e = lane + 32 * i;
    dp[i] = e < E ? __fmul_rn(aux_scale, stats[3 + e]) : 0.f;
  }
  for (int j = 0; j < k; ++j) {
    const int ej = __shfl_sync(0xffffffffu, idx, j);
    const float dvj = __shfl_sync(0xffffffffu, dv, j);
#pragma unroll
    for (int i = 0; i < EW; ++i)
      if (ej == lane + 32 * i) dp[i] = __fadd_rn(dp[i], dvj);
  }
  float dot2 = 0.f;
#pragma unroll
  for (int i = 0; i < EW; ++i) dot2 = __fadd_rn(dot2, __fmul_rn(p[i], dp[i]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) dot2 = __fadd_rn(dot2, __shfl_xor_sync(0xffffffffu, dot2, o));
  const float zc = __fdiv_rn(__fmul_rn(__fmul_rn(dz, 2.0f), lse), n);
#pragma unroll
  for (int i = 0; i < EW; ++i) {
    const int e = lane + 32 * i;
    if (e < E) out[e] = __fadd_rn(__fmul_rn(p[i], __fsub_rn(dp[i], dot2)), __fmul_rn(zc, p[i]));
  }
}

// d_x[t] = bf16(sum_j d_rows[slot(t, j)] + d_x_router[t]) in float32, slots in order;
// masked tokens get bf16(d_x_router[t]).  One warp per token, lanes over 8 columns.
__global__ void __launch_bounds__(256) dx_combine_kernel(const uint16_t* __restrict__ d_rows,
                                                         const int32_t* __restrict__ slot_pos,
                                                         const float* __restrict__ dxr, int T, int k, int d,
                                                         uint16_t* __restrict__ d_x) {
  const int lane = threadIdx.x & 31;
  const int64_t t = int64_t(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (t >= T) return;
  int my_pos = lane < k ? slot_pos[t * k + lane] : -1;
  for (int c = lane * 8; c < d; c += 256) {
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.f;
    for (int j = 0; j < k; ++j) {
      const int p = __shfl_sync(0xffffffffu, my_pos, j);
      if (p < 0) continue;
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(d_rows + int64_t(p) * d + c));
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        acc[2 * i] = __fadd_rn(acc[2 * i], bf16x2_lo(w[i]));
        acc[2 * i + 1] = __fadd_rn(acc[2 * i + 1], bf16x2_hi(w[i]));
      }
    }
    if (dxr != nullptr) {
      const float4 a = __ldg(reinterpret_cast<const float4*>(dxr + t * d + c));
      const float4 b = __ldg(reinterpret_cast<const float4*>(dxr + t * d + c + 4));
      acc[0] = __fadd_rn(acc[0], a.x), acc[1] = __fadd_rn(acc[1], a.y), acc[2] = __fadd_rn(acc[2], a.z);
      acc[3] = __fadd_rn(acc[3], a.w), acc[4] = __fadd_rn(acc[4], b.x), acc[5] = __fadd_rn(acc[5], b.y);
      acc[6] = __fadd_rn(acc[6], b.z), acc[7] = __fadd_rn(acc[7], b.w);
    }
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) o[i] = pack_bf16x2(acc[2 * i], acc[2 * i + 1]);
    *reinterpret_cast<uint4*>(d_x + t * d + c) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// ---------------------------------------------------------------- launchers

int launch_sr_quant(const uint16_t* x, int64_t rows, int cols, const float* amax, uint64_t seed,
                    const int32_t* pad_start, const int32_t* counts, const int32_t* offs_start, int E,
                    uint8_t* packed, uint8_t* scales, float* g_out, cudaStream_t stream) {
  if (rows == 0) return MCL4MOE_OK;
  RowMap map{pad_start, counts, offs_start, E};
  const int64_t blocks = (rows + 7) / 8;
  sr_quant_kernel<<<unsigned(blocks), 256, 0, stream>>>(x, rows, cols, amax, uint32_t(seed & 0xFFFFFFFFu),
                                                         uint32_t(seed >> 32), map, packed, scales, g_out);
  return cudaGetLastError() == cudaSuccess ? MCL4MOE_OK : MCL4MOE_ERR_CUDA;
}

int launch_bf16_amax(const uint16_t* x, int64_t n, float* amax, cudaStream_t stream) {
  if (cudaMemsetAsync(amax, 0, sizeof(float), stream) != cudaSuccess) return MCL4MOE_ERR_CUDA;
  const int64_t n8 = n / 8;
  if (n8 == 0) return MCL4MOE_OK;
  int blocks = int((n8 + 255) / 256);
  if (blocks > 4 * num_sms()) blocks = 4 * num_sms();
  bf16_amax_kernel<<<blocks, 256, 0, stream>>>(x, n8, amax);
  return cudaGetLastError() == cudaSuccess ? MCL4MOE_OK : MCL4MOE_ERR_CUDA;
}

int launch_slot_grad(const uint16_t* d_out, const uint16_t* y, const int32_t* slot_pos, const float* topk_w, int T,
                     int k, int d, const int32_t* pad_start, const int32_t* counts, int E, uint16_t* d_y, float* d_w,
                     float* amax, cudaStream_t stream) {
  const int64_t blocks = (int64_t(T) * k + 7) / 8 + E;
  slot_grad_kernel<<<unsigned(blocks), 256, 0, stream>>>(d_out, y, slot_pos, topk_w, T, k, d, pad_start, counts, d_y,
                                                          d_w, amax);
  return cudaGetLastError() == cudaSuccess ? MCL4MOE_OK : MCL4MOE_ERR_CUDA;
}

int launch_swiglu_bwd(const uint16_t* d_h, const uint16_t* up, int64_t rows_cap, const int32_t* pad_end, int F,
                      uint16_t* d_up, float* amax, cudaStream_t stream) {
  if (rows_cap == 0) return MCL4MOE_OK;
  swiglu_bwd_kernel<<<unsigned((rows_cap + 7) / 8), 256, 0, stream>>>(d_h, up, rows_cap, pad_end, F, d_up, amax);
  return cudaGetLastError() == cudaSuccess ? MCL4MOE_OK : MCL4MOE_ERR_CUDA;
}

int launch_router_bwd(const float* logits, const int32_t* topk_idx, const float* topk_w, const float* d_w,
                      const uint8_t* valid, const float* stats, const float* d_aux, const float* d_z, int T, int E,
                      int k, int norm, float* d_logits, cudaStream_t stream) {
  if (T == 0) return MCL4MOE_OK;
  const unsigned blocks = unsigned((T + 7) / 8);
  if (E <= 32)
    router_bwd_kernel<1><<<blocks, 256, 0, stream>>>(logits, topk_idx, topk_w, d_w, valid, stats, d_aux, d_z, T, E,
                                                     k, norm, d_logits);
  else if (E <= 64)
    router_bwd_kernel<2><<<blocks, 256, 0, stream>>>(logits, topk_idx, topk_w, d_w, valid, stats, d_aux, d_z, T, E,
                                                     k, norm, d_logits);
  else if (E <= 128)
    router_bwd_kernel<4><<<blocks, 256, 0, stream>>>(logits, topk_idx, topk_w, d_w, valid, stats, d_aux, d_z, T, E,
                                                     k, norm, d_logits);
  else
    router_bwd_kernel<8><<<blocks, 256, 0, stream>>>(logits, topk_idx, topk_w, d_w, valid, stats, d_aux, d_z, T, E,
                                                     k, norm, d_logits);
  return cudaGetLastError() == cudaSuccess ? MCL4MOE_OK : MCL4MOE_ERR_CUDA;
}

int launch_dx_combine(const uint16_t* d_rows, const int32_t* slot_pos, const float* dxr, int T, int k, int d,
                      uint16_t* d_x, cudaStream_t stream) {
  if (T == 0) return MCL4MOE_OK;
  dx_combine_kernel<<<unsigned((T + 7) / 8), 256, 0, stream>>>(d_rows, slot_pos, dxr, T, k, d, d_x);
  return cudaGetLastError() == cudaSuccess ? MCL4MOE_OK : MCL4MOE_ERR_CUDA;
}

}  // namespace mcl4

// ---------------------------------------------------------------- C ABI

namespace {

using namespace mcl4;

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

struct BwdWorkspace {
  uint8_t* qa;    // stochastic-rounded NVFP4 rows of the gradient being fed to a GEMM [M_cap, Kmax/2]
  uint8_t* sa;    // their E4M3 scales, row-major [M_cap, Kmax/16]
  uint16_t* d_h;  // gradient of the SwiGLU output h, bf16 [M_cap, F]
  float* amax;    // [2]
  float* g;       // [2] global scales of d_y and d_up
  int32_t* err;
  size_t bytes;
};

BwdWorkspace bwd_workspace(void* base, int T, int d, int E, int k, int F) {
  BwdWorkspace w{};
  const int64_t mcap = padded_rows_cap(T, E, k);
  const int64_t kmax = d > 2 * F ? d : 2 * F;
  uint8_t* p = static_cast<uint8_t*>(base);
  size_t off = 0;
  auto take = [&](size_t bytes) {
    uint8_t* r = p ? p + off : nullptr;
    off += align256(bytes);
    return r;
  };
  w.qa = take(size_t(mcap) * kmax / 2);
  w.sa = take(size_t(mcap) * kmax / 16);
  w.d_h = reinterpret_cast<uint16_t*>(take(sizeof(uint16_t) * size_t(mcap) * F));
  w.amax = reinterpret_cast<float*>(take(2 * sizeof(float)));
  w.g = reinterpret_cast<float*>(take(2 * sizeof(float)));
  w.err = reinterpret_cast<int32_t*>(take(sizeof(int32_t)));
  w.bytes = off;
  return w;
}

int dgrad_gemm(const uint8_t* qa, const uint8_t* sa, int64_t mcap, int K, const uint8_t* bt, const uint8_t* bt_scales,
               const float* bg, const float* ag, int N, const int32_t* pad_start, const int32_t* counts, int E,
               uint16_t* out, int32_t* err, cudaStream_t s) {
  GemmArgs g{};
  g.pad_start = pad_start;
  g.row_count = counts;
  g.a_scales = sa;
  g.a_sf_rowmajor = 1;
  g.b_scales = bt_scales;
  g.b_g = bg;
  g.a_g = ag;
  g.E = E;
  g.K = K;
  g.N_total = N;
  g.n_tiles = N / 256;
  g.mode = 1;
  g.y = out;
  g.ldy = N;
  g.err = err;
  return launch_grouped_gemm(qa, mcap, bt, g, s);
}

}  // namespace

extern "C" {

int mcl4moe_quantize_rows_sr(const uint16_t* x, int64_t rows, int cols, uint64_t seed, uint8_t* packed,
                             uint8_t* scales, float* global_scale, float* amax_scratch, mcl4moe_stream_t stream) {
  if (rows < 0 || cols <= 0 || !packed || !scales || !global_scale || !amax_scratch || (rows > 0 && !x))
    return MCL4MOE_ERR_INVALID;
  if (cols % 16 != 0) return MCL4MOE_ERR_INVALID;
  if (!aligned16(x) || !aligned16(packed) || cols % 128 != 0) return MCL4MOE_ERR_UNSUPPORTED;
  cudaStream_t s = stream;
  int st = launch_bf16_amax(x, rows * cols, amax_scratch, s);
  if (st != MCL4MOE_OK) return st;
  if (rows == 0) {  // amax 0 -> g = 1, written by a kernel with no rows to quantise
    sr_quant_kernel<<<1, 32, 0, s>>>(x, 0, cols, amax_scratch, 0u, 0u, RowMap{nullptr, nullptr, nullptr, 0}, packed,
                                     scales, global_scale);
    return cudaGetLastError() == cudaSuccess ? MCL4MOE_OK : MCL4MOE_ERR_CUDA;
  }
  return launch_sr_quant(x, rows, cols, amax_scratch, seed, nullptr, nullptr, nullptr, 0, packed, scales,
                         global_scale, s);
}

size_t mcl4moe_moe_backward_workspace_size(int T, int d, int E, int k, int F) {
  if (T < 0 || d <= 0 || E <= 0 || k <= 0 || F <= 0) return 0;
  return bwd_workspace(nullptr, T, d, E, k, F).bytes;
}

int mcl4moe_moe_backward_experts(const mcl4moe_moe_bwd_args* a, mcl4moe_stream_t stream) {
  if (!a || a->T < 0 || a->d <= 0 || a->E <= 0 || a->k <= 0 || a->F <= 0 || a->k > a->E) return MCL4MOE_ERR_INVALID;
  if (a->E > kMaxExperts || a->k > kMaxTopK || a->d % 256 != 0 || a->F % 256 != 0) return MCL4MOE_ERR_UNSUPPORTED;
  if (int64_t(a->T) * a->k > kMaxRoutedSlots) return MCL4MOE_ERR_UNSUPPORTED;
  if (a->T == 0) return MCL4MOE_OK;
  if (!a->d_out || !a->slot_pos || !a->topk_w || !a->pad_start || !a->counts || !a->offs_start || !a->y_save ||
      !a->up_save || !a->w_up_t || !a->w_up_t_scales || !a->w_up_g || !a->w_dn_t || !a->w_dn_t_scales ||
      !a->w_dn_g || !a->d_y || !a->d_up || !a->d_rows || !a->d_w || !a->workspace)
    return MCL4MOE_ERR_INVALID;
  if (!aligned16(a->d_out) || !aligned16(a->y_save) || !aligned16(a->up_save) || !aligned16(a->d_y) ||
      !aligned16(a->d_up) || !aligned16(a->d_rows) || !aligned16(a->w_up_t) || !aligned16(a->w_dn_t) ||
      !aligned16(a->w_up_t_scales) || !aligned16(a->w_dn_t_scales))
    return MCL4MOE_ERR_INVALID;
  const BwdWorkspace w = bwd_workspace(a->workspace, a->T, a->d, a->E, a->k, a->F);
  if (a->workspace_bytes < w.bytes) return MCL4MOE_ERR_WORKSPACE;
  cudaStream_t s = stream;
  const int T = a->T, d = a->d, E = a->E, k = a->k, F = a->F;
  const int64_t mcap = padded_rows_cap(T, E, k);
  int32_t* err = a->error_word ? a->error_word : w.err;
  if (!a->error_word && cudaMemsetAsync(w.err, 0, sizeof(int32_t), s) != cudaSuccess) return MCL4MOE_ERR_CUDA;
  if (cudaMemsetAsync(w.amax, 0, 2 * sizeof(float), s) != cudaSuccess) return MCL4MOE_ERR_CUDA;
  // 1. slot rows: d_y and the routing-weight gradient
  int st = launch_slot_grad(a->d_out, a->y_save, a->slot_pos, a->topk_w, T, k, d, a->pad_start, a->counts, E, a->d_y,
                            a->d_w, w.amax, s);
  if (st != MCL4MOE_OK) return st;
  // 2. d_h = SR(d_y) x W_down (the down projection's input gradient, src/mcl4_coe/nvfp4.py:1128-1170)
  if ((st = launch_sr_quant(a->d_y, mcap, d, w.amax, a->seed_down, a->pad_start, a->counts, a->offs_start, E, w.qa,
                            w.sa, w.g, s)) != MCL4MOE_OK)
    return st;
  if ((st = dgrad_gemm(w.qa, w.sa, mcap, d, a->w_dn_t, a->w_dn_t_scales, a->w_dn_g, w.g, F, a->pad_start, a->counts, E,
                       w.d_h, err, s)) != MCL4MOE_OK)
    return st;
  // 3. SwiGLU derivative -> d_up = [d_gate | d_val]
  if ((st = launch_swiglu_bwd(w.d_h, a->up_save, mcap, a->pad_start + E, F, a->d_up, w.amax + 1, s)) != MCL4MOE_OK)
    return st;
  // 4. d_rows = SR(d_up) x W_up (the gate/up projection's input gradient)
  if ((st = launch_sr_quant(a->d_up, mcap, 2 * F, w.amax + 1, a->seed_up, a->pad_start, a->counts, a->offs_start, E,
                            w.qa, w.sa, w.g + 1, s)) != MCL4MOE_OK)
    return st;
  return dgrad_gemm(w.qa, w.sa, mcap, 2 * F, a->w_up_t, a->w_up_t_scales, a->w_up_g, w.g + 1, d, a->pad_start,
                    a->counts, E, a->d_rows, err, s);
}

int mcl4moe_moe_backward_wgrad(const uint16_t* g, const uint16_t* x, int64_t rows, int N, int K,
                               const int32_t* pad_start, int E, float* dw, int32_t* error_word,
                               mcl4moe_stream_t stream) {
  if (rows < 0 || N <= 0 || K <= 0 || E <= 0 || !pad_start || !dw || (rows > 0 && (!g || !x)))
    return MCL4MOE_ERR_INVALID;
  if (N % 128 != 0 || K % 256 != 0 || rows % 256 != 0 || E > kMaxExperts) return MCL4MOE_ERR_UNSUPPORTED;
  if (!aligned16(g) || !aligned16(x) || !aligned16(dw)) return MCL4MOE_ERR_INVALID;
  if (rows == 0) return cudaMemsetAsync(dw, 0, sizeof(float) * size_t(E) * N * K, stream) == cudaSuccess
                            ? MCL4MOE_OK
                            : MCL4MOE_ERR_CUDA;
  return launch_wgrad(g, x, rows, N, K, pad_start, E, dw, error_word, stream);
}

int mcl4moe_router_backward(const float* logits, const int32_t* topk_idx, const float* topk_w, const float* d_w,
                            const uint8_t* valid, const float* stats, const float* d_aux, const float* d_z, int T,
                            int E, int k, int norm_topk_prob, float* d_logits, mcl4moe_stream_t stream) {
  if (T < 0 || E <= 0 || k <= 0 || k > E) return MCL4MOE_ERR_INVALID;
  if (E > kMaxExperts || k > kMaxTopK) return MCL4MOE_ERR_UNSUPPORTED;
  if (T > 0 && (!logits || !topk_idx || !topk_w || !d_w || !stats || !d_logits)) return MCL4MOE_ERR_INVALID;
  return launch_router_bwd(logits, topk_idx, topk_w, d_w, valid, stats, d_aux, d_z, T, E, k, norm_topk_prob, d_logits,
                           stream);
}

int mcl4moe_moe_backward_dx(const uint16_t* d_rows, const int32_t* slot_pos, const float* d_x_router, int T, int k,
                            int d, uint16_t* d_x, mcl4moe_stream_t stream) {
  if (T < 0 || k <= 0 || d <= 0) return MCL4MOE_ERR_INVALID;
  if (k > kMaxTopK || d % 8 != 0) return MCL4MOE_ERR_UNSUPPORTED;
  if (T > 0 && (!d_rows || !slot_pos || !d_x)) return MCL4MOE_ERR_INVALID;
  if (!aligned16(d_rows) || !aligned16(d_x) || !aligned16(d_x_router)) return MCL4MOE_ERR_INVALID;
  return launch_dx_combine(d_rows, slot_pos, d_x_router, T, k, d, d_x, stream);
}

}  // extern "C"
