// NVFP4 quantisers: 16x16-tile weight quantisation (per-expert global scale)
// and 1x16 row activation quantisation (global scale 1).
//
// Weights restate _quantize_grouped_weights_core (src/mcl4_coe/nvfp4.py:923-952):
//   g   = max(amax(W) > 0 ? amax/2688 : 1, FLT_MIN)
//   s_t = e4m3(min(amax(tile) / (6 g), 448))          one per 16x16 tile
//   q   = e2m1(w * min(1/(s_t g), FLT_MAX))           packed along K
// Activations restate _quantize_nvfp4_core(two_dimensional=False,
// causal_row_scale=True) (src/mcl4_coe/nvfp4.py:197-225) with g = 1.
#include <algorithm>

#include "kernels.cuh"
#include "sr.cuh"

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
                                                           uint8_t* ref_b_bwd, uint8_t* ref_bs_bwd, uint8_t* t_packed,
                                                           uint8_t* t_scales) {
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
  if (t_packed) {  // W^T in the kernel layout [E, K, N/2]: row k packs (n, n+1) pairs, the bytes of B_bwd
    uint8_t* b = t_packed + size_t(slot) * K * (N / 2);
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      uint32_t lo = 0, hi = 0;
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        lo |= (((codes[2 * np] >> (4 * c)) & 0xFu) | (((codes[2 * np + 1] >> (4 * c)) & 0xFu) << 4)) << (8 * np);
        hi |= (((codes[2 * np + 8] >> (4 * c)) & 0xFu) | (((codes[2 * np + 9] >> (4 * c)) & 0xFu) << 4)) << (8 * np);
      }
      *reinterpret_cast<uint2*>(b + size_t(c0 + c) * (N / 2) + (n0 >> 1)) = make_uint2(lo, hi);
    }
  }
  if (t_scales) {  // the same 16x16 tile scale, swizzled for the K rows of W^T (N/16 blocks per row)
    uint8_t* b = t_scales + size_t(slot) * ((K + 127) / 128 * 128) * (N / 16);
#pragma unroll
    for (int c = 0; c < 8; ++c)
      b[swizzled_scale_offset(uint64_t(c0 + c), uint32_t(n0 >> 4), uint32_t(N / 16))] = uint8_t(s);
  }
}

int launch_quantize_weights(const float* const* w_ptrs, const int32_t* slots, int n, int N, int K, uint8_t* packed,
                            uint8_t* scales, float* gscale, uint8_t* rb, uint8_t* rbs, uint8_t* rbb, uint8_t* rbbs,
                            float* amax, cudaStream_t stream, uint8_t* t_packed, uint8_t* t_scales) {
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
                                                                                   scales, gscale, rb, rbs, rbb, rbbs,
                                                                                   t_packed, t_scales);
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

// ---------------------------------------------------------------- 1-D rows with a global scale

namespace {

template <typename InT>
__device__ __forceinline__ float load_f32(const InT* p);
template <>
__device__ __forceinline__ float load_f32<float>(const float* p) { return __ldg(p); }
template <>
__device__ __forceinline__ float load_f32<uint16_t>(const uint16_t* p) { return bf16_to_f32(__ldg(p)); }

// The 16 values of a block starting at p (16-byte aligned) with vector loads.
__device__ __forceinline__ void load_block16(const float* p, float (&v)[16]) {
  const float4* q = reinterpret_cast<const float4*>(p);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float4 f = __ldg(q + i);
    v[4 * i] = f.x, v[4 * i + 1] = f.y, v[4 * i + 2] = f.z, v[4 * i + 3] = f.w;
  }
}
__device__ __forceinline__ void load_block16(const uint16_t* p, float (&v)[16]) {
  const uint4* q = reinterpret_cast<const uint4*>(p);
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const uint4 u = __ldg(q + i);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      v[8 * i + 2 * j] = bf16_to_f32(uint16_t(w[j] & 0xFFFFu));
      v[8 * i + 2 * j + 1] = bf16_to_f32(uint16_t(w[j] >> 16));
    }
  }
}

// max |x| over a [rows, cols] matrix (row stride ld) into *amax (zeroed before):
// float bits of non-negative values order like unsigned ints.
template <typename InT>
__global__ void __launch_bounds__(256) rows_amax_kernel(const InT* __restrict__ x, int64_t rows, int cols, int64_t ld,
                                                        float* amax) {
  float m = 0.f;
  const int64_t n = rows * cols;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x)
    m = fmaxf(m, fabsf(load_f32(x + (i / cols) * ld + (i % cols))));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) atomicMax(reinterpret_cast<unsigned int*>(amax), __float_as_uint(m));
}

// g = 1 (causal row scales) or amax / 2688 clamped to the smallest normal
// (src/mcl4_coe/nvfp4.py:203-208); optionally g_ab = g * g_b (the GEMM's scale).
__global__ void rows_global_scale_kernel(const float* amax, int causal, float* g, const float* g_b, float* g_ab) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  float v = 1.f;
  if (!causal) {
    const float a = *amax;
    v = fmaxf(a > 0.f ? __fdiv_rn(a, 2688.0f) : 1.0f, kFltMinNormal);
  }
  *g = v;
  if (g_ab) *g_ab = __fmul_rn(v, *g_b);
}

// One warp per row, lane l takes 16-element blocks l, l+32, ...: scale
// e4m3(min(amax16 / (6 g), 448)), inverse 1 / (scale * g), E2M1 codes of x * inverse
// (src/mcl4_coe/nvfp4.py:209-225, one-dimensional mode); scales into the swizzled atoms
// (the reference's output layout) or row-major (the GEMM's A operand).  SR: stochastic
// rounding (the gradient quantisation of the backward), noise of element (row, col) the
// Philox draw at offset row * cols + col (32-bit wrap) under key (k0, k1).
template <typename InT, bool SR>
__global__ void __launch_bounds__(256) rows_quant_kernel(const InT* __restrict__ x, int64_t rows, int cols, int64_t ld,
                                                         const float* __restrict__ g_ptr, uint8_t* __restrict__ packed,
                                                         uint8_t* __restrict__ scales, int rowmajor, uint32_t k0,
                                                         uint32_t k1) {
  const int lane = threadIdx.x & 31;
  const int64_t row = int64_t(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (row >= rows) return;
  const float g = *g_ptr;
  const float six_g = __fmul_rn(6.0f, g);
  const int nblk = cols / 16;
  for (int b = lane; b < nblk; b += 32) {
    float v[16];
    float m = 0.f;
    load_block16(x + row * ld + b * 16, v);
#pragma unroll
    for (int j = 0; j < 16; ++j) m = fmaxf(m, fabsf(v[j]));
    const uint32_t sc = f32_to_e4m3(fminf(__fdiv_rn(m, six_g), 448.0f));
    const float inv = inverse_decoding(__fmul_rn(e4m3_to_f32(sc), g));
    uint32_t lo = 0, hi = 0;
    if constexpr (SR) {
      const uint32_t off0 = uint32_t(uint64_t(row) * uint64_t(cols)) + uint32_t(b * 16);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        lo |= e2m1_code_sr(__fmul_rn(v[j], inv), sr_uniform(off0 + j, k0, k1)) << (4 * j);
        hi |= e2m1_code_sr(__fmul_rn(v[8 + j], inv), sr_uniform(off0 + 8 + j, k0, k1)) << (4 * j);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        lo |= e2m1_code(__fmul_rn(v[j], inv)) << (4 * j);
        hi |= e2m1_code(__fmul_rn(v[8 + j], inv)) << (4 * j);
      }
    }
    *reinterpret_cast<uint2*>(packed + row * (cols / 2) + b * 8) = make_uint2(lo, hi);
    scales[rowmajor ? rowmajor_scale_offset(uint64_t(row), uint32_t(b), uint32_t(nblk))
                    : swizzled_scale_offset(uint64_t(row), uint32_t(b), uint32_t(nblk))] = uint8_t(sc);
  }
}

__global__ void single_segment_kernel(int64_t rows, int64_t rows_pad, int32_t* pad_start, int32_t* counts,
                                      int32_t* offs_start) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  pad_start[0] = 0;
  pad_start[1] = int32_t(rows_pad);
  counts[0] = int32_t(rows);
  offs_start[0] = 0;
}

}  // namespace

int launch_quantize_rows(const void* x, int dtype, int64_t rows, int cols, int64_t ld, int causal, uint8_t* packed,
                         uint8_t* scales, int64_t rows_pad, float* g, float* amax, const float* g_b, float* g_ab,
                         int rowmajor, cudaStream_t s, int stochastic, uint64_t seed) {
  const size_t scale_bytes = size_t(rows_pad) * size_t(cols / 16);
  if (cudaMemsetAsync(scales, 0, scale_bytes, s) != cudaSuccess) return MCL4MOE_ERR_CUDA;
  if (!causal) {
    if (cudaMemsetAsync(amax, 0, sizeof(float), s) != cudaSuccess) return MCL4MOE_ERR_CUDA;
    const int64_t n = rows * cols;
    const unsigned blocks = unsigned(std::min<int64_t>((n + 255) / 256, 4 * 148));
    if (blocks > 0) {
      if (dtype == 0)
        rows_amax_kernel<uint16_t><<<blocks, 256, 0, s>>>(static_cast<const uint16_t*>(x), rows, cols, ld, amax);
      else
        rows_amax_kernel<float><<<blocks, 256, 0, s>>>(static_cast<const float*>(x), rows, cols, ld, amax);
    }
  }
  rows_global_scale_kernel<<<1, 32, 0, s>>>(amax, causal, g, g_b, g_ab);
  if (rows > 0) {
    const unsigned blocks = unsigned((rows + 7) / 8);
    const uint32_t k0 = uint32_t(seed), k1 = uint32_t(seed >> 32);
    const uint16_t* xh = static_cast<const uint16_t*>(x);
    const float* xf = static_cast<const float*>(x);
    if (dtype == 0 && stochastic)
      rows_quant_kernel<uint16_t, true><<<blocks, 256, 0, s>>>(xh, rows, cols, ld, g, packed, scales, rowmajor, k0, k1);
    else if (dtype == 0)
      rows_quant_kernel<uint16_t, false><<<blocks, 256, 0, s>>>(xh, rows, cols, ld, g, packed, scales, rowmajor, k0, k1);
    else if (stochastic)
      rows_quant_kernel<float, true><<<blocks, 256, 0, s>>>(xf, rows, cols, ld, g, packed, scales, rowmajor, k0, k1);
    else
      rows_quant_kernel<float, false><<<blocks, 256, 0, s>>>(xf, rows, cols, ld, g, packed, scales, rowmajor, k0, k1);
  }
  return cudaGetLastError() == cudaSuccess ? MCL4MOE_OK : MCL4MOE_ERR_CUDA;
}

int launch_single_segment(int64_t rows, int64_t rows_pad, int32_t* pad_start, int32_t* counts, int32_t* offs_start,
                          cudaStream_t s) {
  single_segment_kernel<<<1, 32, 0, s>>>(rows, rows_pad, pad_start, counts, offs_start);
  return cudaGetLastError() == cudaSuccess ? MCL4MOE_OK : MCL4MOE_ERR_CUDA;
}

// ---------------------------------------------------------------- 2:4 sparsity masks

namespace {

// The 90 4x4 0/1 tiles with exactly two ones in every row and every column,
// in the enumeration order of the reference's catalog
// (src/mcl4_coe/nvfp4.py:50-67: rows r0..r3 each one of the six 2-of-4 row
// patterns in the listed order, nested r0 outermost), bit 4*row + col.  The
// order matters: the best pattern is the first maximum.
struct Catalog2to4 {
  uint16_t tile[90];
};

constexpr Catalog2to4 make_catalog_2to4() {
  constexpr uint8_t rows[6] = {0x3, 0x5, 0x9, 0x6, 0xA, 0xC};  // bit c = column c: 1100 1010 1001 0110 0101 0011
  Catalog2to4 c{};
  int n = 0;
  for (int a = 0; a < 6; ++a)
    for (int b = 0; b < 6; ++b)
      for (int e = 0; e < 6; ++e)
        for (int f = 0; f < 6; ++f) {
          bool ok = true;
          for (int col = 0; col < 4; ++col) {
            const int sum = ((rows[a] >> col) & 1) + ((rows[b] >> col) & 1) + ((rows[e] >> col) & 1) +
                            ((rows[f] >> col) & 1);
            ok = ok && sum == 2;
          }
          if (ok && n < 90)
            c.tile[n++] = uint16_t(rows[a] | (rows[b] << 4) | (rows[e] << 8) | (rows[f] << 12));
        }
  return c;
}

constexpr Catalog2to4 kCatalogHost = make_catalog_2to4();
static_assert(kCatalogHost.tile[89] != 0, "the doubly 2:4 catalog has 90 tiles");
__constant__ Catalog2to4 kCatalog = kCatalogHost;

// mode 2 (transposable): one thread per 4x4 tile of W [N, K]; the pattern with the
// largest sum of kept |w| (summed in fp32 over the tile's 16 positions in row-major
// order, dropped ones contributing +0), first maximum on ties
// (src/mcl4_coe/nvfp4.py:98-110).  mode 1 (row): one thread per 4 consecutive
// elements of a row, keeping the two largest |w| (lower index first on ties;
// :90-96).  w_masked = w * mask (a dropped negative weight becomes -0, as the
// reference's ``w * mask.float()``); mask (optional) 0/1 bytes [N, K].
__global__ void __launch_bounds__(256) mask_2to4_kernel(const float* __restrict__ w, int N, int K, int mode,
                                                        float* __restrict__ w_masked, uint8_t* __restrict__ mask) {
  const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (mode == 2) {
    const int tiles_k = K / 4;
    if (i >= int64_t(N / 4) * tiles_k) return;
    const int64_t r0 = (i / tiles_k) * 4, c0 = (i % tiles_k) * 4;
    float v[16], a[16];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const float4 q = *reinterpret_cast<const float4*>(w + (r0 + r) * K + c0);
      v[4 * r] = q.x, v[4 * r + 1] = q.y, v[4 * r + 2] = q.z, v[4 * r + 3] = q.w;
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) a[j] = fabsf(v[j]);
    int best = 0;
    float best_s = -1.f;
    for (int p = 0; p < 90; ++p) {
      const uint32_t m = kCatalog.tile[p];
      float sum = 0.f;
#pragma unroll
      for (int j = 0; j < 16; ++j) sum = __fadd_rn(sum, ((m >> j) & 1u) ? a[j] : 0.f);
      if (sum > best_s) best_s = sum, best = p;  // strict: the first maximum wins
    }
    const uint32_t m = kCatalog.tile[best];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      float4 o;
      o.x = __fmul_rn(v[4 * r], float((m >> (4 * r)) & 1u));
      o.y = __fmul_rn(v[4 * r + 1], float((m >> (4 * r + 1)) & 1u));
      o.z = __fmul_rn(v[4 * r + 2], float((m >> (4 * r + 2)) & 1u));
      o.w = __fmul_rn(v[4 * r + 3], float((m >> (4 * r + 3)) & 1u));
      *reinterpret_cast<float4*>(w_masked + (r0 + r) * K + c0) = o;
      if (mask)
        *reinterpret_cast<uint32_t*>(mask + (r0 + r) * K + c0) =
            ((m >> (4 * r)) & 1u) | (((m >> (4 * r + 1)) & 1u) << 8) | (((m >> (4 * r + 2)) & 1u) << 16) |
            (((m >> (4 * r + 3)) & 1u) << 24);
    }
  } else {
    const int groups = K / 4;
    if (i >= int64_t(N) * groups) return;
    const int64_t base = (i / groups) * K + (i % groups) * 4;
    const float4 q = *reinterpret_cast<const float4*>(w + base);
    const float v[4] = {q.x, q.y, q.z, q.w};
    int first = 0;
    for (int j = 1; j < 4; ++j)
      if (fabsf(v[j]) > fabsf(v[first])) first = j;
    int second = first == 0 ? 1 : 0;
    for (int j = 0; j < 4; ++j)
      if (j != first && fabsf(v[j]) > fabsf(v[second])) second = j;
    float o[4];
    uint32_t mb = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const bool keep = j == first || j == second;
      o[j] = __fmul_rn(v[j], keep ? 1.f : 0.f);
      mb |= uint32_t(keep) << (8 * j);
    }
    *reinterpret_cast<float4*>(w_masked + base) = make_float4(o[0], o[1], o[2], o[3]);
    if (mask) *reinterpret_cast<uint32_t*>(mask + base) = mb;
  }
}

}  // namespace

int launch_mask_2to4(const float* w, int N, int K, int mode, float* w_masked, uint8_t* mask, cudaStream_t stream) {
  const int64_t items = mode == 2 ? int64_t(N / 4) * (K / 4) : int64_t(N) * (K / 4);
  if (items == 0) return MCL4MOE_OK;
  const int64_t blocks = (items + 255) / 256;
  if (blocks > 0x7fffffff) return MCL4MOE_ERR_UNSUPPORTED;
  mask_2to4_kernel<<<dim3(unsigned(blocks)), 256, 0, stream>>>(w, N, K, mode, w_masked, mask);
  return cudaGetLastError() == cudaSuccess ? MCL4MOE_OK : MCL4MOE_ERR_CUDA;
}

}  // namespace mcl4
