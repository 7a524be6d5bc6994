// Internal launch interface shared by the kernel files and the C ABI (api.cu).
#pragma once

#include <atomic>
#include <utility>

#include "common.cuh"

namespace mcl4 {

constexpr int kMaxWeightBatch = 256;  // weight matrices per quantiser launch
constexpr int kMaxExperts = 256;
constexpr int kMaxTopK = 32;
constexpr int kRouteTokens = 128;     // tokens per router CTA (= permutation chunk)
// Routed slots per call (T * k): per-expert counts, offsets and slot ranks are int32.
constexpr int64_t kMaxRoutedSlots = int64_t(1) << 30;

// ---- workspace layout of the routing stage (all offsets 256-byte aligned)
struct RouteWorkspace {
  int32_t* local_rank;   // [T, k]  rank of slot (t, j) among its expert's slots in the chunk
  int32_t* chunk_excl;   // [C, E]  chunk counts, then (after the scan) exclusive prefix over chunks
  float* part_probs;     // [C, E]  per-chunk sum of routed probabilities
  float* part_misc;      // [C, 2]  per-chunk sum of lse^2 and routed-token count
  int32_t* pad_start;    // [E + 1] padded row start of each expert (multiple of kSegRows)
  int32_t* offs_start;   // [E]     unpadded row start of each expert
  int32_t* counts;       // [E]     routed slots per expert
  float* probs_sum;      // [E]     sum of routed probabilities per expert
  uint32_t* done;        // [1]     finished-expert counter of the scan (zeroed by the router)
  uint16_t* wsplit;      // [3][E_pad][d] bf16 parts of the router weight (hi, mid, lo)
  float* small_logits;   // [T, E] logits of small batches (T <= kRouteGemvMaxT), else null
  float* small_tok;      // [2][128] lse^2 and routed flag per token of a one-chunk batch (T <= 128),
                         // then 17 uint32 completion counters
  size_t bytes;
};

// Batches up to this many tokens compute their fp32 router logits on the CUDA cores
// (a few tokens leave the tensor-core router with one CTA walking d serially).
constexpr int kRouteGemvMaxT = 1024;
// ... and rows of at most kRouteGemvMaxSmem / 16 elements (8 staged bf16 rows per CTA).
constexpr size_t kRouteGemvMaxSmem = 200 * 1024;

inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

inline RouteWorkspace route_workspace(void* base, int T, int E, int k, int d) {
  RouteWorkspace w{};
  const int C = (T + kRouteTokens - 1) / kRouteTokens;
  uint8_t* p = static_cast<uint8_t*>(base);
  size_t off = 0;
  auto take = [&](size_t bytes) {
    uint8_t* r = p ? p + off : nullptr;
    off += align256(bytes);
    return r;
  };
  w.local_rank = reinterpret_cast<int32_t*>(take(sizeof(int32_t) * size_t(T) * k));
  w.chunk_excl = reinterpret_cast<int32_t*>(take(sizeof(int32_t) * size_t(C) * E));
  w.part_probs = reinterpret_cast<float*>(take(sizeof(float) * size_t(C) * E));
  w.part_misc = reinterpret_cast<float*>(take(sizeof(float) * size_t(C) * 2));
  w.pad_start = reinterpret_cast<int32_t*>(take(sizeof(int32_t) * (E + 1)));
  w.offs_start = reinterpret_cast<int32_t*>(take(sizeof(int32_t) * E));
  w.counts = reinterpret_cast<int32_t*>(take(sizeof(int32_t) * E));
  w.probs_sum = reinterpret_cast<float*>(take(sizeof(float) * E));
  w.done = reinterpret_cast<uint32_t*>(take(sizeof(uint32_t)));
  w.wsplit = reinterpret_cast<uint16_t*>(take(sizeof(uint16_t) * 3 * size_t((E + 15) / 16 * 16) * size_t(d)));
  w.small_logits = T <= kRouteGemvMaxT ? reinterpret_cast<float*>(take(sizeof(float) * size_t(T) * E)) : nullptr;
  w.small_tok = T <= kRouteTokens ? reinterpret_cast<float*>(take(sizeof(float) * 2 * kRouteTokens + 17 * 4)) : nullptr;
  w.bytes = off;
  return w;
}

// Block-wide exclusive scan of one int32 per thread (tmp: 64 ints of shared
// memory); ``total`` receives the block sum.  Every thread of the block calls it.
__device__ __forceinline__ int32_t block_exclusive_scan(int32_t v, int32_t* tmp, int32_t& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  int32_t x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int32_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) tmp[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int32_t w = lane < nw ? tmp[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int32_t y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    if (lane < nw) tmp[32 + lane] = w;
  }
  __syncthreads();
  total = tmp[32 + nw - 1];
  const int32_t before = warp ? tmp[32 + warp - 1] : 0;
  __syncthreads();
  return before + x - v;
}

// Deterministic block sum: fixed xor tree in each warp, warps added in order.
__device__ __forceinline__ float block_sum(float v, float* tmp) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  if (lane == 0) tmp[warp] = v;
  __syncthreads();
  float s = 0.f;
  for (int w = 0; w < nw; ++w) s = __fadd_rn(s, tmp[w]);
  __syncthreads();
  return s;
}


// Launch ``kernel`` with programmatic stream serialization: it may begin while the
// previous kernel on ``stream`` drains, and must pdl_wait() before reading that
// kernel's outputs.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                              Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Raise a kernel's dynamic shared-memory limit on the current device, once per
// device: the attribute belongs to the kernel's instance in each device's
// context, so a process that drives several GPUs sets it on every one.  ``done``
// is a bitmask of the devices (ordinal < 64) already configured.
template <typename... KArgs>
inline bool raise_smem_limit(void (*kernel)(KArgs...), int bytes, std::atomic<uint64_t>& done) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  const uint64_t bit = dev < 64 ? (uint64_t(1) << dev) : 0;
  if (bit != 0 && (done.load(std::memory_order_acquire) & bit) != 0) return true;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess) return false;
  done.fetch_or(bit, std::memory_order_release);
  return true;
}

// Expert segments of the grouped GEMMs start on multiples of kSegRows rows: a
// CTA pair computes 256-row tiles that must not straddle two experts.
constexpr int kSegRows = 256;

inline int64_t padded_rows_cap(int64_t T, int E, int k) {
  const int64_t m = T * k + int64_t(kSegRows - 1) * E;
  return (m + kSegRows - 1) / kSegRows * kSegRows;
}

// ---- launchers (return MCL4MOE_* status)
// t_packed / t_scales (nullable): W^T [K, N] in the kernel layout (packed [E, K, N/2], the 16x16 tile scales
// swizzled for K rows padded to 128), the B operand of the backward's input-gradient GEMM.
int launch_quantize_weights(const float* const* w_ptrs, const int32_t* slots, int n, int N, int K, uint8_t* packed,
                            uint8_t* scales, float* gscale, uint8_t* rb, uint8_t* rbs, uint8_t* rbb, uint8_t* rbbs,
                            float* amax, cudaStream_t stream, uint8_t* t_packed = nullptr,
                            uint8_t* t_scales = nullptr);

// One-dimensional NVFP4 rows (1x16 blocks) of a bf16 (dtype 0) or fp32 (dtype 1)
// matrix with global scale g = 1 (causal) or amax/2688; packed [rows, cols/2],
// scales for rows_pad rows (padding rows zero) in the 128x4 swizzled atoms or,
// with rowmajor, [rows_pad, cols/16]; g written to *g; with g_b, *g_ab = g * *g_b.
// amax: device scratch float.  cols % 64 == 0.  stochastic: stochastic rounding with
// noise seed `seed` (offsets row * cols + col).
int launch_quantize_rows(const void* x, int dtype, int64_t rows, int cols, int64_t ld, int causal, uint8_t* packed,
                         uint8_t* scales, int64_t rows_pad, float* g, float* amax, const float* g_b, float* g_ab,
                         int rowmajor, cudaStream_t s, int stochastic = 0, uint64_t seed = 0);

// pad_start = {0, rows_pad}, counts = {rows}, offs_start = {0}: one GEMM segment.
int launch_single_segment(int64_t rows, int64_t rows_pad, int32_t* pad_start, int32_t* counts, int32_t* offs_start,
                          cudaStream_t s);

// 2:4 sparsity mask of W [N, K] (mode 1: 2 of every 4 along K; mode 2: doubly 2:4
// per 4x4 tile) and the masked weights.
int launch_mask_2to4(const float* w, int N, int K, int mode, float* w_masked, uint8_t* mask, cudaStream_t stream);

int launch_quantize_activations(const uint16_t* x, int64_t rows, int cols, int64_t ld_x, uint8_t* packed,
                                uint8_t* scales, int swizzled, cudaStream_t stream);

// Router + top-k + chunk ranks + scan (+ statistics), writes topk/sel_mask/stats and fills ``ws``.
int launch_route(const uint16_t* x, const float* wr, const float* bias, const float* logits_in, const uint8_t* valid,
                 int T, int d, int E, int k, int norm_topk, int32_t* topk_idx, float* topk_w, float* logits_out,
                 float* sel_mask, int32_t* counts_out, float* stats, int32_t* offs_out, int32_t* err,
                 const RouteWorkspace& ws, cudaStream_t stream);

// Expert layout (ranks, chunk counts, segment starts) from caller-supplied
// expert ids [T, k] instead of the router; ids outside [0, E) are not routed.
int launch_route_from_indices(const int32_t* topk_idx, const uint8_t* valid, int T, int E, int k, int32_t* counts_out,
                              float* stats, int32_t* offs_out, const RouteWorkspace& ws, cudaStream_t stream);

// Scatter each routed token's NVFP4 row into its k padded expert-major slots.
int launch_permute_quantize(const uint16_t* x, const uint8_t* valid, const int32_t* topk_idx, const float* topk_w,
                            int T, int d, int E, int k, const RouteWorkspace& ws, int32_t* slot_pos, float* sorted_w,
                            int32_t* perm, uint8_t* xq, uint8_t* xs, cudaStream_t stream, uint16_t* xg = nullptr);

// Grouped-linear helpers: padded layout from inclusive ends, and row scatter.
int launch_pad_from_offs(const int32_t* offs, int E, int32_t* pad_start, int32_t* offs_start, int32_t* counts,
                         cudaStream_t stream);
int launch_quantize_grouped_rows(const uint16_t* x, int64_t M, int K, const int32_t* offs, const int32_t* pad_start,
                                 const int32_t* counts, int E, uint8_t* xq, uint8_t* xs, cudaStream_t stream);

// out[t] = bf16(sum_j y[slot_pos[t, j]]) for valid tokens, 0 otherwise.
// row_w (nullable): per padded row routing weight; y then holds unweighted rows, each weighted as bf16(y * bf16(w)).
int launch_combine(const uint16_t* y, const int32_t* slot_pos, const uint8_t* valid, int T, int k, int d, uint16_t* out,
                   cudaStream_t stream, const float* row_w = nullptr);

// ---- grouped block-scaled FP4 GEMM (tcgen05)
struct GemmArgs {
  const int32_t* pad_start;     // [E + 1]
  const int32_t* row_count;     // [E] valid rows per expert (stores of rows beyond are skipped)
  const int32_t* out_row_base;  // [E] destination row of an expert's first row (nullptr: padded row index)
  const uint8_t* a_scales;      // padded rows: row-major [rows, K/16] if a_sf_rowmajor, else 128x4 swizzled atoms
  int a_sf_rowmajor;
  const uint8_t* b_scales;      // [E, N_total*K/16] swizzled
  const float* b_g;             // [E]
  int E, K, N_total, n_tiles, mode;
  int F;                        // mode 0: columns of h (gate rows [0,F), value rows [F,2F) of B)
  uint8_t* hq;                  // mode 0: [M, F/2]
  uint8_t* hs;                  // mode 0: swizzled [M/128 * F/64 * 512]
  uint16_t* h_dbg;              // mode 0: bf16 [M, F] or nullptr
  uint16_t* up_save;            // mode 0: bf16 [M, 2F] gate | value rows bf16(acc * g) (training), or nullptr
  const float* a_g;             // modes 1/2: device scalar global scale of A (the output is acc * (a_g * b_g[e])),
                                // or nullptr for g_a = 1
  const float* row_w;           // mode 1: per padded row weight or nullptr
  uint16_t* y;                  // mode 1: bf16 output
  float* y32;                   // mode 2: fp32 output instead of y (acc * g [+ bias]), or nullptr
  const float* bias;            // mode 2 with y32: [N_total] added after the scale, or nullptr
  int64_t ldy;
  int32_t* err;
  int solo;                     // modes 0 (inference) / 1: single-CTA 128-row tiles that skip padding-only
                                // blocks (decode); mode 1 then writes valid rows only
  // mode 4 (gate/up for expert parallelism): row_w holds each valid row's h destination
  // (rank << 28 | row, as float bits); h codes / swizzled scales go to peer_hq / peer_hs[rank]
  uint8_t* peer_hq[8];
  uint8_t* peer_hs[8];
};

int launch_grouped_gemm(const uint8_t* a, int64_t a_rows, const uint8_t* b, const GemmArgs& args, cudaStream_t stream);

// ---- backward (backward.cu)
int launch_sr_quant(const uint16_t* x, int64_t rows, int cols, const float* amax, uint64_t seed,
                    const int32_t* pad_start, const int32_t* counts, const int32_t* offs_start, int E,
                    uint8_t* packed, uint8_t* scales, float* g_out, cudaStream_t stream);
int launch_bf16_amax(const uint16_t* x, int64_t n, float* amax, cudaStream_t stream);
int launch_slot_grad(const uint16_t* d_out, const uint16_t* y, const int32_t* slot_pos, const float* topk_w, int T,
                     int k, int d, const int32_t* pad_start, const int32_t* counts, int E, uint16_t* d_y, float* d_w,
                     float* amax, cudaStream_t stream);
int launch_swiglu_bwd(const uint16_t* d_h, const uint16_t* up, int64_t rows_cap, const int32_t* pad_end, int F,
                      uint16_t* d_up, float* amax, cudaStream_t stream);
int launch_router_bwd(const float* logits, const int32_t* topk_idx, const float* topk_w, const float* d_w,
                      const uint8_t* valid, const float* stats, const float* d_aux, const float* d_z, int T, int E,
                      int k, int norm, float* d_logits, cudaStream_t stream);
int launch_dx_combine(const uint16_t* d_rows, const int32_t* slot_pos, const float* dxr, int T, int k, int d,
                      uint16_t* d_x, cudaStream_t stream);
// dW[e] = G[seg e]^T X[seg e] (fp32 [E, N, K]) over the padded segments of pad_start (wgrad.cu).
int launch_wgrad(const uint16_t* g, const uint16_t* x, int64_t rows, int N, int K, const int32_t* pad_start, int E,
                 float* dw, int32_t* err, cudaStream_t stream);

int num_sms();

}  // namespace mcl4
