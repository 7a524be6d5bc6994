// Backward of the single-matrix NVFP4 projection (_NVFP4Linear.backward,
// src/mcl4_coe/nvfp4.py:431-472): the weight gradient
//   dW = nvfp4_mm(H16(G^T), H16(X^T), stochastic_a=True)        (:454-459)
// with G = grad_output [M, N], X = inputs [M, K] and H16 the fixed-sign
// orthonormal Walsh-Hadamard transform over groups of 16 columns of the transposed
// matrices, i.e. over groups of 16 tokens (_hadamard16, :337-355).  Since H16 is
// orthonormal the product over the token dimension is G^T X; the transform spreads
// outliers across each 16-token block before the 1x16 quantisation.
//
// Each operand is written by one pass that reads its row-major source, transforms
// 16 tokens of one column in registers, quantises the block and stores it as row
// `column` of the transposed operand (the token index is the GEMM's K), after a pass
// that finds the transformed matrix's amax for the tensor-wise global scale
// (quantize_nvfp4's one-dimensional mode, :197-225: g = amax / 2688).  The GEMM is the
// tcgen05 block-scaled kernel of gemm_fp4.cu with one segment and an fp32 epilogue.
// The bias gradient (grad_output.float().sum(0), :468-469) comes out of G's amax
// pass as per-CTA column sums reduced in a fixed order.
#include "kernels.cuh"
#include "sr.cuh"

namespace mcl4 {

namespace {

template <typename InT>
__device__ __forceinline__ float ld_elem(const InT* p);
template <>
__device__ __forceinline__ float ld_elem<float>(const float* p) { return __ldg(p); }
template <>
__device__ __forceinline__ float ld_elem<uint16_t>(const uint16_t* p) { return bf16_to_f32(__ldg(p)); }

// Signs of the Hadamard rows (src/mcl4_coe/nvfp4.py:172-178): bit i set where sign i is -1.
constexpr uint32_t kHadamardNegative = 0xD7E8u;

// In-register transform of 16 values: v <- (v * signs) H / 4 with H the Sylvester
// Hadamard matrix, H[i][j] = (-1)^popcount(i & j): sign flips, four butterfly stages
// (pairs (i, i + w) within blocks of 2w, w = 1, 2, 4, 8), then the exact scale 1/4.
// The same operation order as the oracle, so results agree bit for bit.
__device__ __forceinline__ void hadamard16(float (&v)[16]) {
#pragma unroll
  for (int i = 0; i < 16; ++i)
    if ((kHadamardNegative >> i) & 1u) v[i] = -v[i];
#pragma unroll
  for (int w = 1; w < 16; w <<= 1) {
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      if (i & w) continue;
      const float a = v[i], b = v[i + w];
      v[i] = __fadd_rn(a, b);
      v[i + w] = __fsub_rn(a, b);
    }
  }
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __fmul_rn(v[i], 0.25f);
}

// Column c of tokens [t0, t0 + 16) of y [M, C] (row stride ld), zeros past M.
template <typename InT>
__device__ __forceinline__ void load_column16(const InT* __restrict__ y, int64_t M, int64_t ld, int64_t t0, int c,
                                              float (&v)[16]) {
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = t0 + i < M ? ld_elem(y + (t0 + i) * ld + c) : 0.f;
}

// amax of H16 over column blocks; CTA (32 columns, 8 token blocks), warp = token
// block, lane = column.  With col_part: the raw column sums of the CTA's 128 tokens
// into col_part[blockIdx.y * C + c].
template <typename InT>
__global__ void __launch_bounds__(256) ht_amax_kernel(const InT* __restrict__ y, int64_t M, int C, float* amax,
                                                      float* __restrict__ col_part) {
  __shared__ float sums[8][32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int c = blockIdx.x * 32 + lane;
  const int64_t t0 = (int64_t(blockIdx.y) * 8 + warp) * 16;
  float m = 0.f, sum = 0.f;
  if (c < C && t0 < M) {
    float v[16];
    load_column16(y, M, C, t0, c, v);
#pragma unroll
    for (int i = 0; i < 16; ++i) sum = __fadd_rn(sum, v[i]);
    hadamard16(v);
#pragma unroll
    for (int i = 0; i < 16; ++i) m = fmaxf(m, fabsf(v[i]));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (lane == 0) atomicMax(reinterpret_cast<unsigned int*>(amax), __float_as_uint(m));
  if (col_part == nullptr) return;
  sums[warp][lane] = sum;
  __syncthreads();
  if (warp == 0 && c < C) {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) s = __fadd_rn(s, sums[w][lane]);
    col_part[int64_t(blockIdx.y) * C + c] = s;
  }
}

// Fixed-order sum of the per-CTA column sums.
__global__ void __launch_bounds__(256) col_reduce_kernel(const float* __restrict__ col_part, int parts, int C,
                                                         float* __restrict__ out) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  float s = 0.f;
  for (int p = 0; p < parts; ++p) s = __fadd_rn(s, col_part[int64_t(p) * C + c]);
  out[c] = s;
}

// Quantised transposed operand: row r (< rows_out) of [rows_out, Kt] holds column r of
// y transformed over 16-token blocks (zeros for r >= C and tokens >= M); 1x16 blocks
// with scale e4m3(min(amax16 / (6 g), 448)) (row-major [rows_out, Kt/16] scales or the
// swizzled 128x4 atoms).  SR: stochastic codes, noise offset r * Kt + token.
template <typename InT, bool SR>
__global__ void __launch_bounds__(256) ht_quant_kernel(const InT* __restrict__ y, int64_t M, int C, int64_t Kt,
                                                       const float* __restrict__ g_ptr, uint32_t k0, uint32_t k1,
                                                       uint8_t* __restrict__ packed, uint8_t* __restrict__ scales,
                                                       int rowmajor) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int r = blockIdx.x * 32 + lane;
  const int64_t blk = int64_t(blockIdx.y) * 8 + warp;
  const int64_t t0 = blk * 16;
  const float g = *g_ptr;
  float v[16];
  if (r < C) load_column16(y, M, C, t0, r, v);
  else {
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = 0.f;
  }
  hadamard16(v);
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(v[i]));
  const uint32_t sc = f32_to_e4m3(fminf(__fdiv_rn(amax, __fmul_rn(6.0f, g)), 448.0f));
  const float inv = inverse_decoding(__fmul_rn(e4m3_to_f32(sc), g));
  uint32_t lo = 0, hi = 0;
  if constexpr (SR) {
    const uint32_t off0 = uint32_t(uint64_t(r) * uint64_t(Kt)) + uint32_t(t0);
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
  *reinterpret_cast<uint2*>(packed + int64_t(r) * (Kt / 2) + blk * 8) = make_uint2(lo, hi);
  const uint32_t nblk = uint32_t(Kt / 16);
  scales[rowmajor ? rowmajor_scale_offset(uint64_t(r), uint32_t(blk), nblk)
                  : swizzled_scale_offset(uint64_t(r), uint32_t(blk), nblk)] = uint8_t(sc);
}

// g = max(amax > 0 ? amax / 2688 : 1, FLT_MIN) for both operands and the product
// g_a * g_b the GEMM epilogue applies (src/mcl4_coe/nvfp4.py:203-208).
__global__ void wgrad_scales_kernel(const float* amax_a, const float* amax_b, float* g_a, float* g_b, float* g_ab) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  const float a = *amax_a, b = *amax_b;
  const float ga = fmaxf(a > 0.f ? __fdiv_rn(a, 2688.0f) : 1.0f, kFltMinNormal);
  const float gb = fmaxf(b > 0.f ? __fdiv_rn(b, 2688.0f) : 1.0f, kFltMinNormal);
  *g_a = ga;
  *g_b = gb;
  *g_ab = __fmul_rn(ga, gb);
}

__global__ void ht_global_scale_kernel(const float* amax, float* g) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  const float a = *amax;
  *g = fmaxf(a > 0.f ? __fdiv_rn(a, 2688.0f) : 1.0f, kFltMinNormal);
}

struct LinearWgradWorkspace {
  uint8_t* aq;  // [mp_a, Kt/2]   H16(G^T), stochastic
  uint8_t* as;  // [mp_a, Kt/16]  row-major
  uint8_t* bq;  // [Kp, Kt/2]     H16(X^T), round to nearest
  uint8_t* bs;  // [Kp * Kt/16]   swizzled
  int32_t* pad_start;
  int32_t* counts;
  int32_t* offs_start;
  float* amax;  // [2]
  float* g;     // [3]: g_a, g_b, g_a * g_b
  int32_t* err;
  float* col_part;  // [Kt / 128, N]
  size_t bytes;
};

LinearWgradWorkspace linear_wgrad_workspace(void* base, int64_t M, int N, int K) {
  LinearWgradWorkspace w{};
  const int64_t kt = (M + 255) / 256 * 256, mpa = (int64_t(N) + kSegRows - 1) / kSegRows * kSegRows;
  const int64_t kp = (int64_t(K) + 255) / 256 * 256;
  uint8_t* p = static_cast<uint8_t*>(base);
  size_t off = 0;
  auto take = [&](size_t bytes) {
    uint8_t* r = p ? p + off : nullptr;
    off += (bytes + 255) / 256 * 256;
    return r;
  };
  w.aq = take(size_t(mpa) * size_t(kt) / 2);
  w.as = take(size_t(mpa) * size_t(kt) / 16);
  w.bq = take(size_t(kp) * size_t(kt) / 2);
  w.bs = take(size_t(kp) * size_t(kt) / 16);
  w.pad_start = reinterpret_cast<int32_t*>(take(2 * sizeof(int32_t)));
  w.counts = reinterpret_cast<int32_t*>(take(sizeof(int32_t)));
  w.offs_start = reinterpret_cast<int32_t*>(take(sizeof(int32_t)));
  w.amax = reinterpret_cast<float*>(take(2 * sizeof(float)));
  w.g = reinterpret_cast<float*>(take(3 * sizeof(float)));
  w.err = reinterpret_cast<int32_t*>(take(sizeof(int32_t)));
  w.col_part = reinterpret_cast<float*>(take(size_t(kt / 128) * size_t(N) * sizeof(float)));
  w.bytes = off;
  return w;
}

template <typename InT>
void launch_ht_amax(const void* y, int64_t M, int C, float* amax, float* col_part, cudaStream_t s) {
  const dim3 grid(unsigned((C + 31) / 32), unsigned((M + 127) / 128));
  ht_amax_kernel<InT><<<grid, 256, 0, s>>>(static_cast<const InT*>(y), M, C, amax, col_part);
}

template <typename InT, bool SR>
void launch_ht_quant(const void* y, int64_t M, int C, int rows_out, int64_t Kt, const float* g, uint64_t seed,
                     uint8_t* packed, uint8_t* scales, int rowmajor, cudaStream_t s) {
  const dim3 grid(unsigned(rows_out / 32), unsigned(Kt / 128));
  ht_quant_kernel<InT, SR><<<grid, 256, 0, s>>>(static_cast<const InT*>(y), M, C, Kt, g, uint32_t(seed),
                                                 uint32_t(seed >> 32), packed, scales, rowmajor);
}

}  // namespace

}  // namespace mcl4

using namespace mcl4;

extern "C" {

int mcl4moe_quantize_hadamard_t(const void* y, int dtype, int64_t M, int C, int64_t kt, int rows_out, int stochastic,
                                uint64_t seed, uint8_t* packed, uint8_t* scales, int swizzled, float* global_scale,
                                float* amax_scratch, mcl4moe_stream_t stream) {
  if (M < 0 || C <= 0 || (dtype != 0 && dtype != 1) || !packed || !scales || !global_scale || !amax_scratch)
    return MCL4MOE_ERR_INVALID;
  if (M > 0 && !y) return MCL4MOE_ERR_INVALID;
  if (kt < M || kt % 128 != 0 || rows_out < C || rows_out % 32 != 0 || (swizzled && rows_out % 128 != 0))
    return MCL4MOE_ERR_INVALID;
  if (kt / 128 > 65535) return MCL4MOE_ERR_UNSUPPORTED;
  if (reinterpret_cast<uintptr_t>(packed) % 8 != 0) return MCL4MOE_ERR_INVALID;
  cudaStream_t s = stream;
  if (cudaMemsetAsync(amax_scratch, 0, sizeof(float), s) != cudaSuccess) return MCL4MOE_ERR_CUDA;
  if (M > 0) {
    if (dtype == 0) launch_ht_amax<uint16_t>(y, M, C, amax_scratch, nullptr, s);
    else launch_ht_amax<float>(y, M, C, amax_scratch, nullptr, s);
  }
  ht_global_scale_kernel<<<1, 32, 0, s>>>(amax_scratch, global_scale);
  if (kt > 0) {
    const int rm = swizzled ? 0 : 1;
    if (dtype == 0 && stochastic)
      launch_ht_quant<uint16_t, true>(y, M, C, rows_out, kt, global_scale, seed, packed, scales, rm, s);
    else if (dtype == 0)
      launch_ht_quant<uint16_t, false>(y, M, C, rows_out, kt, global_scale, seed, packed, scales, rm, s);
    else if (stochastic)
      launch_ht_quant<float, true>(y, M, C, rows_out, kt, global_scale, seed, packed, scales, rm, s);
    else
      launch_ht_quant<float, false>(y, M, C, rows_out, kt, global_scale, seed, packed, scales, rm, s);
  }
  return cudaGetLastError() == cudaSuccess ? MCL4MOE_OK : MCL4MOE_ERR_CUDA;
}

size_t mcl4moe_nvfp4_linear_wgrad_workspace_size(int64_t M, int N, int K) {
  if (M < 0 || N <= 0 || K <= 0) return 0;
  return linear_wgrad_workspace(nullptr, M, N, K).bytes;
}

int mcl4moe_nvfp4_linear_wgrad(const void* grad, int grad_dtype, const void* x, int x_dtype, int64_t M, int N, int K,
                               uint64_t seed, float* dw, float* d_bias, int32_t* error_word, void* workspace,
                               size_t workspace_bytes, mcl4moe_stream_t stream) {
  if (M < 0 || N <= 0 || K <= 0 || !dw || !workspace) return MCL4MOE_ERR_INVALID;
  if ((grad_dtype != 0 && grad_dtype != 1) || (x_dtype != 0 && x_dtype != 1)) return MCL4MOE_ERR_INVALID;
  if (M > 0 && (!grad || !x)) return MCL4MOE_ERR_INVALID;
  if ((M + 255) / 256 * 256 / 128 > 65535) return MCL4MOE_ERR_UNSUPPORTED;  // grid rows of the token blocks
  if (reinterpret_cast<uintptr_t>(dw) % 16 != 0) return MCL4MOE_ERR_INVALID;
  const LinearWgradWorkspace w = linear_wgrad_workspace(workspace, M, N, K);
  if (workspace_bytes < w.bytes) return MCL4MOE_ERR_WORKSPACE;
  cudaStream_t s = stream;
  const int64_t kt = (M + 255) / 256 * 256, kp = (int64_t(K) + 255) / 256 * 256;
  const int mpa = int((int64_t(N) + kSegRows - 1) / kSegRows * kSegRows);
  if (M == 0) {  // no tokens: zero gradients
    if (cudaMemsetAsync(dw, 0, size_t(N) * size_t(kp) * sizeof(float), s) != cudaSuccess) return MCL4MOE_ERR_CUDA;
    if (d_bias && cudaMemsetAsync(d_bias, 0, size_t(N) * sizeof(float), s) != cudaSuccess) return MCL4MOE_ERR_CUDA;
    return MCL4MOE_OK;
  }
  int32_t* err = error_word ? error_word : w.err;
  if (!error_word && cudaMemsetAsync(err, 0, sizeof(int32_t), s) != cudaSuccess) return MCL4MOE_ERR_CUDA;
  if (cudaMemsetAsync(w.amax, 0, 2 * sizeof(float), s) != cudaSuccess) return MCL4MOE_ERR_CUDA;
  float* part = d_bias ? w.col_part : nullptr;
  if (grad_dtype == 0) launch_ht_amax<uint16_t>(grad, M, N, w.amax, part, s);
  else launch_ht_amax<float>(grad, M, N, w.amax, part, s);
  if (x_dtype == 0) launch_ht_amax<uint16_t>(x, M, K, w.amax + 1, nullptr, s);
  else launch_ht_amax<float>(x, M, K, w.amax + 1, nullptr, s);
  if (d_bias) col_reduce_kernel<<<unsigned((N + 255) / 256), 256, 0, s>>>(w.col_part, int((M + 127) / 128), N, d_bias);
  wgrad_scales_kernel<<<1, 32, 0, s>>>(w.amax, w.amax + 1, w.g, w.g + 1, w.g + 2);
  if (grad_dtype == 0)
    launch_ht_quant<uint16_t, true>(grad, M, N, mpa, kt, w.g, seed, w.aq, w.as, 1, s);
  else
    launch_ht_quant<float, true>(grad, M, N, mpa, kt, w.g, seed, w.aq, w.as, 1, s);
  if (x_dtype == 0)
    launch_ht_quant<uint16_t, false>(x, M, K, int(kp), kt, w.g + 1, 0, w.bq, w.bs, 0, s);
  else
    launch_ht_quant<float, false>(x, M, K, int(kp), kt, w.g + 1, 0, w.bq, w.bs, 0, s);
  if (cudaGetLastError() != cudaSuccess) return MCL4MOE_ERR_CUDA;
  int st = launch_single_segment(N, mpa, w.pad_start, w.counts, w.offs_start, s);
  if (st != MCL4MOE_OK) return st;
  GemmArgs g{};
  g.pad_start = w.pad_start;
  g.row_count = w.counts;
  g.out_row_base = w.offs_start;
  g.a_scales = w.as;
  g.a_sf_rowmajor = 1;
  g.b_scales = w.bs;
  g.b_g = w.g + 2;
  g.E = 1;
  g.K = int(kt);
  g.N_total = int(kp);
  g.n_tiles = int(kp / 256);
  g.mode = 1;
  g.y32 = dw;
  g.bias = nullptr;
  g.ldy = kp;
  g.err = err;
  return launch_grouped_gemm(w.aq, mpa, w.bq, g, s);
}

}  // extern "C"
