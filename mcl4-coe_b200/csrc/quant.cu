// NVFP4 quantisers: 16x16-tile weight quantisation (per-expert global scale)
// and 1x16 row activation quantisation (global scale 1).
//
// Weights restate _quantize_grouped_weights_core (src/mcl4_coe/nvfp4.py:923-952):
//   g   = max(amax(W) > 0 ? amax/2688 : 1, FLT_MIN)
//   s_t = e4m3(min(amax(tile) / (6 g), 448))          one per 16x16 tile
//   q   = e2m1(w * min(1/(s_t g), FLT_MAX))           packed along K
// Activations restate _quantize_nvfp4_core(two_dimensional=False,
// causal_row_scale=True) (src/mcl4_coe/nvfp4.py:197-225) with g = 1.
#include "kernels.cuh"

namespace mcl4 {

// ---------------------------------------------------------------- weights

struct WeightBatch {
  const float* w[kMaxWeightBatch];
  int32_t slot[kMaxWeightBatch];
};

// amax over each matrix: float bits of non-negative values order like ints.
__global__ void __launch_bounds__(256) weight_amax_kernel(WeightBatch batch, int64_t numel, float* amax) {
  const float* w = batch.w[blockIdx.y];
  float m = 0.f;
  const int64_t n4 = numel >> 2;
  const float4* w4 = reinterpret_cast<const float4*>(w);
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n4; i += int64_t(gridDim.x) * blockDim.x) {
    float4 v = __ldg(w4 + i);
    m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) atomicMax(reinterpret_cast<unsigned int*>(amax + blockIdx.y), __float_as_uint(m));
}

// One CTA = 16 rows x 1024 columns (64 tiles, two threads per tile, 8 columns each).
__global__ void __launch_bounds__(128) weight_quant_kernel(WeightBatch batch, int N, int K, const float* amax,
                                                           uint8_t* packed, uint8_t* scales, float* gscale,
                                                           uint8_t* ref_b_fwd, uint8_t* ref_bs_fwd,
                                                           uint8_t* ref_b_bwd, uint8_t* ref_bs_bwd) {
  const int i = blockIdx.z;
  const float* w = batch.w[i];
  const int slot = batch.slot[i];
  const int n0 = blockIdx.x * 16;
  const int c0 = blockIdx.y * 1024 + threadIdx.x * 8;
  const bool active = c0 < K;

  const float a = amax[i];
  float g = a > 0.f ? __fdiv_rn(a, 2688.0f) : 1.0f;  // src/mcl4_coe/nvfp4.py:928-929
  g = fmaxf(g, kFltMinNormal);
  if (blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) gscale[slot] = g;

  float v[16][8];
  float m = 0.f;
#pragma unroll
  for (int r = 0; r < 16; ++r) {
    if (active) {
      const float4* p = reinterpret_cast<const float4*>(w + int64_t(n0 + r) * K + c0);
      float4 x0 = __ldg(p), x1 = __ldg(p + 1);
      v[r][0] = x0.x; v[r][1] = x0.y; v[r][2] = x0.z; v[r][3] = x0.w;
      v[r][4] = x1.x; v[r][5] = x1.y; v[r][6] = x1.z; v[r][7] = x1.w;
    } else {
#pragma unroll
      for (int c = 0; c < 8; ++c) v[r][c] = 0.f;
    }
#pragma unroll
    for (int c = 0; c < 8; ++c) m = fmaxf(m, fabsf(v[r][c]));
  }
  m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));  // tile amax (pair of threads)
  if (!active) return;

  const uint32_t s = f32_to_e4m3(fminf(__fdiv_rn(m, __fmul_rn(6.0f, g)), 448.0f));  // :930-931
  const float inv = inverse_decoding(__fmul_rn(e4m3_to_f32(s), g));                 // :934-937
  const int kt = c0 >> 4;
  const size_t kh = size_t(K) / 2;
  uint8_t* pk = packed + size_t(slot) * N * kh;
  uint32_t codes[16];  // per row: 8 nibbles
#pragma unroll
  for (int r = 0; r < 16; ++r) {
    uint32_t word = 0;
#pragma unroll
    for (int c = 0; c < 8; ++c) word |= e2m1_code(__fmul_rn(v[r][c], inv)) << (4 * c);
    codes[r] = word;
    *reinterpret_cast<uint32_t*>(pk + size_t(n0 + r) * kh + (c0 >> 1)) = word;
  }
  if ((threadIdx.x & 1) == 0) {
    uint8_t* sc = scales + size_t(slot) * ((N + 127) / 128 * 128) * (K / 16);
#pragma unroll
    for (int r = 0; r < 16; ++r) sc[swizzled_scale_offset(n0 + r, kt, K / 16)] = uint8_t(s);
  }
  if (ref_b_fwd) {  // B_fwd [E, K/2, N]: byte (kp, n)
    uint8_t* b = ref_b_fwd + size_t(slot) * N * kh;
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      uint32_t bytes[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint32_t w4 = 0;
#pragma unroll
        for (int rr = 0; rr < 4; ++rr) w4 |= ((codes[q * 4 + rr] >> (8 * p)) & 0xFFu) << (8 * rr);
        bytes[q] = w4;
      }
      *reinterpret_cast<uint4*>(b + size_t((c0 >> 1) + p) * N + n0) = make_uint4(bytes[0], bytes[1], bytes[2], bytes[3]);
    }
  }
  if (ref_bs_fwd && (threadIdx.x & 1) == 0) {  // Bs_fwd [E, N, K/16]
    uint8_t* b = ref_bs_fwd + size_t(slot) * N * (K / 16);
#pragma unroll
    for (int r = 0; r < 16; ++r) b[size_t(n0 + r) * (K / 16) + kt] = uint8_t(s);
  }
  if (ref_b_bwd) {  // B_bwd [E, N/2, K]: byte (np, k) = code(2np, k) | code(2np+1, k) << 4
    uint8_t* b = ref_b_bwd + size_t(slot) * (N / 2) * K;
#pragma unroll
    for (int np = 0; np < 8; ++np) {
      uint32_t lo = 0, hi = 0;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        lo |= (((codes[2 * np] >> (4 * c)) & 0xFu) | (((codes[2 * np + 1] >> (4 * c)) & 0xFu) << 4)) << (8 * c);
        hi |= (((codes[2 * np] >> (4 * (c + 4))) & 0xFu) | (((codes[2 * np + 1] >> (4 * (c + 4))) & 0xFu) << 4)) << (8 * c);
      }
      *reinterpret_cast<uint2*>(b + size_t((n0 >> 1) + np) * K + c0) = make_uint2(lo, hi);
    }
  }
  if (ref_bs_bwd) {  // Bs_bwd [E, K, N/16]
    uint8_t* b = ref_bs_bwd + size_t(slot) * K * (N / 16);
#pragma unroll
    for (int c = 0; c < 8; ++c) b[size_t(c0 + c) * (N / 16) + (n0 >> 4)] = uint8_t(s);
  }
}

int launch_quantize_weights(const float* const* w_ptrs, const int32_t* slots, int n, int N, int K, uint8_t* packed,
                            uint8_t* scales, float* gscale, uint8_t* rb, uint8_t* rbs, uint8_t* rbb, uint8_t* rbbs,
                            float* amax, cudaStream_t stream) {
  for (int base = 0; base < n; base += kMaxWeightBatch) {
    const int cnt = n - base < kMaxWeightBatch ? n - base : kMaxWeightBatch;
    WeightBatch batch{};
    for (int i = 0; i < cnt; ++i) {
      batch.w[i] = w_ptrs[base + i];
      batch.slot[i] = slots[base + i];
    }
    if (cudaMemsetAsync(amax + base, 0, sizeof(float) * cnt, stream) != cudaSuccess) return MCL4MOE_ERR_CUDA;
    const int64_t numel = int64_t(N) * K;
    int gx = int((numel / 4 + 255) / 256);
    if (gx > 512) gx = 512;
    weight_amax_kernel<<<dim3(gx, cnt), 256, 0, stream>>>(batch, numel, amax + base);
    weight_quant_kernel<<<dim3(N / 16, (K + 1023) / 1024, cnt), 128, 0, stream>>>(batch, N, K, amax + base, packed,
                                                                                   scales, gscale, rb, rbs, rbb, rbbs);
    if (cudaGetLastError() != cudaSuccess) return MCL4MOE_ERR_CUDA;
  }
  return MCL4MOE_OK;
}

// ---------------------------------------------------------------- activations

// One warp per row; lane l handles 16-element blocks l, l+32, ...
__global__ void __launch_bounds__(256) act_quant_kernel(const uint16_t* __restrict__ x, int64_t rows, int cols,
                                                        int64_t ld_x, uint8_t* __restrict__ packed,
                                                        uint8_t* __restrict__ scales, int swizzled) {
  __shared__ float inv_tab[128];
  fill_inverse_scale_table(inv_tab);
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t row = int64_t(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int nblk = cols / 16;
  for (int b0 = 0; b0 < nblk; b0 += 32) {
    const int b = b0 + lane;
    uint32_t s = 0;
    if (b < nblk) {
      const uint4* src = reinterpret_cast<const uint4*>(x + row * ld_x + b * 16);
      uint4 u0 = __ldg(src), u1 = __ldg(src + 1);
      const uint32_t wds[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
      uint2 pk;
      s = quantize_block16_bf16(wds, pk, inv_tab);
      *reinterpret_cast<uint2*>(packed + row * (cols / 2) + b * 8) = pk;
    }
    if (!swizzled) {
      if (b < nblk) scales[row * nblk + b] = uint8_t(s);
    } else {
      // gather the 4 scale bytes of an aligned group of 4 blocks into one word
      const int base_lane = lane & ~3;
      uint32_t word = 0;
#pragma unroll
      for (int q = 0; q < 4; ++q) word |= (__shfl_sync(0xffffffffu, s, base_lane + q) & 0xFFu) << (8 * q);
      if ((lane & 3) == 0 && b < nblk)
        *reinterpret_cast<uint32_t*>(scales + swizzled_scale_offset(uint64_t(row), uint32_t(b), uint32_t(nblk))) = word;
    }
  }
}

int launch_quantize_activations(const uint16_t* x, int64_t rows, int cols, int64_t ld_x, uint8_t* packed,
                                uint8_t* scales, int swizzled, cudaStream_t stream) {
  if (rows == 0) return MCL4MOE_OK;
  act_quant_kernel<<<unsigned((rows + 7) / 8), 256, 0, stream>>>(x, rows, cols, ld_x, packed, scales, swizzled);
  return cudaGetLastError() == cudaSuccess ? MCL4MOE_OK : MCL4MOE_ERR_CUDA;
}

}  // namespace mcl4
