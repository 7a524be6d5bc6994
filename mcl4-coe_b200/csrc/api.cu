// extern "C" entry points of libmcl4moe (declared in include/mcl4moe.h).
// Host-side validation mirrors the reference's ValueError conditions
// (src/mcl4_coe/nvfp4.py:243-249, :297-304; src/mcl4_coe/backbone.py:95-112)
// and maps them to MCL4MOE_ERR_INVALID; shapes the kernels' tiling cannot
// serve return MCL4MOE_ERR_UNSUPPORTED.  Nothing here allocates memory.
#include <cstring>

#include <atomic>

#include "kernels.cuh"

using namespace mcl4;

namespace {

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

struct MoeWorkspace {
  RouteWorkspace route;
  int32_t* topk_idx;
  float* topk_w;
  int32_t* slot_pos;
  float* sorted_w;
  uint8_t* xq;
  uint8_t* xs;
  uint8_t* hq;
  uint8_t* hs;
  uint16_t* y;
  int32_t* counts;
  float* stats;
  int32_t* err;
  size_t bytes;
};

MoeWorkspace moe_workspace(void* base, int T, int d, int E, int k, int F) {
  MoeWorkspace w{};
  uint8_t* p = static_cast<uint8_t*>(base);
  w.route = route_workspace(base, T, E, k, d);
  size_t off = w.route.bytes;
  auto take = [&](size_t bytes) {
    uint8_t* r = p ? p + off : nullptr;
    off += align256(bytes);
    return r;
  };
  const int64_t mcap = padded_rows_cap(T, E, k);
  w.topk_idx = reinterpret_cast<int32_t*>(take(sizeof(int32_t) * size_t(T) * k));
  w.topk_w = reinterpret_cast<float*>(take(sizeof(float) * size_t(T) * k));
  w.slot_pos = reinterpret_cast<int32_t*>(take(sizeof(int32_t) * size_t(T) * k));
  w.sorted_w = reinterpret_cast<float*>(take(sizeof(float) * size_t(mcap)));
  w.xq = take(size_t(mcap) * d / 2);
  w.xs = take(size_t(mcap) * d / 16);
  w.hq = take(size_t(mcap) * F / 2);
  w.hs = take(size_t(mcap) * F / 16);
  w.y = reinterpret_cast<uint16_t*>(take(sizeof(uint16_t) * size_t(mcap) * d));
  w.counts = reinterpret_cast<int32_t*>(take(sizeof(int32_t) * E));
  w.stats = reinterpret_cast<float*>(take(sizeof(float) * (3 + E)));
  w.err = reinterpret_cast<int32_t*>(take(sizeof(int32_t)));
  w.bytes = off;
  return w;
}

int check_moe_shape(int T, int d, int E, int k, int F) {
  if (T < 0 || d <= 0 || E <= 0 || k <= 0 || F <= 0 || k > E) return MCL4MOE_ERR_INVALID;
  if (E > kMaxExperts || k > kMaxTopK) return MCL4MOE_ERR_UNSUPPORTED;
  if (d % 256 != 0 || F % 256 != 0) return MCL4MOE_ERR_UNSUPPORTED;
  if (int64_t(T) * k > kMaxRoutedSlots) return MCL4MOE_ERR_UNSUPPORTED;
  return MCL4MOE_OK;
}

}  // namespace

extern "C" {

const char* mcl4moe_status_string(int status) {
  switch (status) {
    case MCL4MOE_OK: return "ok";
    case MCL4MOE_ERR_INVALID: return "invalid argument";
    case MCL4MOE_ERR_UNSUPPORTED: return "unsupported device or shape";
    case MCL4MOE_ERR_CUDA: return "CUDA error";
    case MCL4MOE_ERR_TIMEOUT: return "device-side wait timed out";
    case MCL4MOE_ERR_WORKSPACE: return "workspace too small";
    default: return "unknown status";
  }
}

int mcl4moe_version(void) { return 100; }

int mcl4moe_device_supported(void) {
  int dev = 0, major = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return 0;
  return major == 10 ? 1 : 0;
}

int mcl4moe_read_error(int32_t* device_error_word, int32_t* host_value, mcl4moe_stream_t stream) {
  if (!device_error_word || !host_value) return MCL4MOE_ERR_INVALID;
  int32_t v = 0;
  if (cudaMemcpyAsync(&v, device_error_word, sizeof(v), cudaMemcpyDeviceToHost, stream) != cudaSuccess)
    return MCL4MOE_ERR_CUDA;
  if (cudaStreamSynchronize(stream) != cudaSuccess) return MCL4MOE_ERR_CUDA;
  *host_value = v;
  if (v != 0) {
    if (cudaMemsetAsync(device_error_word, 0, sizeof(int32_t), stream) != cudaSuccess) return MCL4MOE_ERR_CUDA;
    if (cudaStreamSynchronize(stream) != cudaSuccess) return MCL4MOE_ERR_CUDA;
    return MCL4MOE_ERR_TIMEOUT;
  }
  return MCL4MOE_OK;
}

int mcl4moe_quantize_weights(const float* const* w_ptrs, const int32_t* slots, int n, int N, int K, uint8_t* packed,
                             uint8_t* scales, float* global_scale, uint8_t* ref_b_fwd, uint8_t* ref_bs_fwd,
                             uint8_t* ref_b_bwd, uint8_t* ref_bs_bwd, float* amax_scratch, mcl4moe_stream_t stream) {
  if (n < 0 || N <= 0 || K <= 0 || !w_ptrs || !slots || !packed || !scales || !global_scale || !amax_scratch)
    return MCL4MOE_ERR_INVALID;
  if (N % 16 != 0 || K % 16 != 0) return MCL4MOE_ERR_INVALID;  // src/mcl4_coe/nvfp4.py:248-249
  if (K % 64 != 0) return MCL4MOE_ERR_UNSUPPORTED;
  for (int i = 0; i < n; ++i)
    if (!w_ptrs[i] || !aligned16(w_ptrs[i]) || slots[i] < 0) return MCL4MOE_ERR_INVALID;
  if (n == 0) return MCL4MOE_OK;
  return launch_quantize_weights(w_ptrs, slots, n, N, K, packed, scales, global_scale, ref_b_fwd, ref_bs_fwd,
                                 ref_b_bwd, ref_bs_bwd, amax_scratch, stream);
}

int mcl4moe_quantize_weights_t(const float* const* w_ptrs, const int32_t* slots, int n, int N, int K,
                               uint8_t* packed, uint8_t* scales, float* global_scale, uint8_t* packed_t,
                               uint8_t* scales_t, float* amax_scratch, mcl4moe_stream_t stream) {
  if (n < 0 || N <= 0 || K <= 0 || !w_ptrs || !slots || !packed || !scales || !global_scale || !amax_scratch ||
      !packed_t || !scales_t)
    return MCL4MOE_ERR_INVALID;
  if (N % 16 != 0 || K % 16 != 0) return MCL4MOE_ERR_INVALID;
  if (K % 128 != 0) return MCL4MOE_ERR_UNSUPPORTED;
  for (int i = 0; i < n; ++i)
    if (!w_ptrs[i] || !aligned16(w_ptrs[i]) || slots[i] < 0) return MCL4MOE_ERR_INVALID;
  if (n == 0) return MCL4MOE_OK;
  return launch_quantize_weights(w_ptrs, slots, n, N, K, packed, scales, global_scale, nullptr, nullptr, nullptr,
                                 nullptr, amax_scratch, stream, packed_t, scales_t);
}

int mcl4moe_mask_2to4(const float* w, int N, int K, int mode, float* w_masked, uint8_t* mask,
                      mcl4moe_stream_t stream) {
  if (N < 0 || K < 0 || (mode != 1 && mode != 2) || (int64_t(N) * K > 0 && (!w || !w_masked))) return MCL4MOE_ERR_INVALID;
  if (K % 4 != 0 || !aligned16(w) || !aligned16(w_masked) || (mask && reinterpret_cast<uintptr_t>(mask) % 4 != 0))
    return MCL4MOE_ERR_INVALID;
  if (mode == 2 && N % 4 != 0) mode = 1;  // src/mcl4_coe/nvfp4.py:90: tiles need both sides divisible by 4
  return launch_mask_2to4(w, N, K, mode, w_masked, mask, stream);
}

int mcl4moe_quantize_rows(const void* x, int dtype, int64_t rows, int cols, int64_t ld, int causal, uint8_t* packed,
                          uint8_t* scales, int64_t rows_pad, float* global_scale, float* amax_scratch,
                          mcl4moe_stream_t stream) {
  if (rows < 0 || cols <= 0 || (dtype != 0 && dtype != 1) || !packed || !scales || !global_scale || !amax_scratch)
    return MCL4MOE_ERR_INVALID;
  if (cols % 16 != 0) return MCL4MOE_ERR_INVALID;  // src/mcl4_coe/nvfp4.py:248-249
  if (cols % 64 != 0) return MCL4MOE_ERR_UNSUPPORTED;
  if (rows_pad < rows || rows_pad % 128 != 0 || ld < cols || (rows > 0 && !x)) return MCL4MOE_ERR_INVALID;
  if (!aligned16(x) || (ld * (dtype == 0 ? 2 : 4)) % 16 != 0) return MCL4MOE_ERR_INVALID;  // vector loads
  return launch_quantize_rows(x, dtype, rows, cols, ld, causal, packed, scales, rows_pad, global_scale, amax_scratch,
                              nullptr, nullptr, 0, stream);
}

int mcl4moe_quantize_rows_stochastic(const void* x, int dtype, int64_t rows, int cols, int64_t ld, int causal,
                                     uint64_t seed, uint8_t* packed, uint8_t* scales, int64_t rows_pad,
                                     float* global_scale, float* amax_scratch, mcl4moe_stream_t stream) {
  if (rows < 0 || cols <= 0 || (dtype != 0 && dtype != 1) || !packed || !scales || !global_scale || !amax_scratch)
    return MCL4MOE_ERR_INVALID;
  if (cols % 16 != 0) return MCL4MOE_ERR_INVALID;
  if (cols % 64 != 0) return MCL4MOE_ERR_UNSUPPORTED;
  if (rows_pad < rows || rows_pad % 128 != 0 || ld < cols || (rows > 0 && !x)) return MCL4MOE_ERR_INVALID;
  if (!aligned16(x) || (ld * (dtype == 0 ? 2 : 4)) % 16 != 0) return MCL4MOE_ERR_INVALID;
  return launch_quantize_rows(x, dtype, rows, cols, ld, causal, packed, scales, rows_pad, global_scale, amax_scratch,
                              nullptr, nullptr, 0, stream, 1, seed);
}

}  // extern "C"

namespace {

struct MmWorkspace {
  uint8_t* aq;
  uint8_t* as;
  int32_t* pad_start;
  int32_t* counts;
  int32_t* offs_start;
  float* g_a;
  float* g_ab;
  float* amax;
  int32_t* err;
  size_t bytes;
};

MmWorkspace mm_workspace(void* base, int64_t M, int K) {
  MmWorkspace w{};
  const int64_t mp = (M + kSegRows - 1) / kSegRows * kSegRows;
  uint8_t* p = static_cast<uint8_t*>(base);
  size_t off = 0;
  auto take = [&](size_t bytes) {
    uint8_t* r = p ? p + off : nullptr;
    off += align256(bytes);
    return r;
  };
  w.aq = take(size_t(mp) * K / 2);
  w.as = take(size_t(mp) * K / 16);
  w.pad_start = reinterpret_cast<int32_t*>(take(2 * sizeof(int32_t)));
  w.counts = reinterpret_cast<int32_t*>(take(sizeof(int32_t)));
  w.offs_start = reinterpret_cast<int32_t*>(take(sizeof(int32_t)));
  w.g_a = reinterpret_cast<float*>(take(sizeof(float)));
  w.g_ab = reinterpret_cast<float*>(take(sizeof(float)));
  w.amax = reinterpret_cast<float*>(take(sizeof(float)));
  w.err = reinterpret_cast<int32_t*>(take(sizeof(int32_t)));
  w.bytes = off;
  return w;
}

}  // namespace

extern "C" {

size_t mcl4moe_nvfp4_mm_workspace_size(int64_t M, int K) {
  if (M < 0 || K <= 0) return 0;
  return mm_workspace(nullptr, M, K).bytes;
}

}  // extern "C"

namespace {

// nvfp4_mm with A quantised here (round to nearest, or stochastic with `seed`).
int nvfp4_mm_impl(const void* x, int dtype, int64_t M, int K, int causal, int stochastic, uint64_t seed,
                  const uint8_t* b, const uint8_t* b_scales, const float* b_g, int N, const float* bias, float* out,
                  float* a_global_scale, int32_t* error_word, void* workspace, size_t workspace_bytes,
                  cudaStream_t stream) {
  if (M < 0 || K <= 0 || N <= 0 || (dtype != 0 && dtype != 1) || !b || !b_scales || !b_g || !out || !workspace)
    return MCL4MOE_ERR_INVALID;
  if (M > 0 && !x) return MCL4MOE_ERR_INVALID;
  if (K % 16 != 0) return MCL4MOE_ERR_INVALID;
  if (K % 256 != 0 || N % 256 != 0) return MCL4MOE_ERR_UNSUPPORTED;
  if (!aligned16(out) || !aligned16(b) || !aligned16(b_scales) || (bias && !aligned16(bias))) return MCL4MOE_ERR_INVALID;
  const MmWorkspace w = mm_workspace(workspace, M, K);
  if (workspace_bytes < w.bytes) return MCL4MOE_ERR_WORKSPACE;
  if (M == 0) return MCL4MOE_OK;
  const int64_t mp = (M + kSegRows - 1) / kSegRows * kSegRows;
  cudaStream_t s = stream;
  int32_t* err = error_word ? error_word : w.err;
  if (!error_word && cudaMemsetAsync(err, 0, sizeof(int32_t), s) != cudaSuccess) return MCL4MOE_ERR_CUDA;
  int st = launch_quantize_rows(x, dtype, M, K, K, causal, w.aq, w.as, mp, w.g_a, w.amax, b_g, w.g_ab, 1, s,
                                stochastic, seed);
  if (st != MCL4MOE_OK) return st;
  if (a_global_scale && cudaMemcpyAsync(a_global_scale, w.g_a, sizeof(float), cudaMemcpyDeviceToDevice, s) !=
                            cudaSuccess)
    return MCL4MOE_ERR_CUDA;
  if ((st = launch_single_segment(M, mp, w.pad_start, w.counts, w.offs_start, s)) != MCL4MOE_OK) return st;
  GemmArgs g{};
  g.pad_start = w.pad_start;
  g.row_count = w.counts;
  g.out_row_base = w.offs_start;
  g.a_scales = w.as;
  g.a_sf_rowmajor = 1;
  g.b_scales = b_scales;
  g.b_g = w.g_ab;
  g.E = 1;
  g.K = K;
  g.N_total = N;
  g.n_tiles = N / 256;
  g.mode = 1;
  g.y32 = out;
  g.bias = bias;
  g.ldy = N;
  g.err = err;
  return launch_grouped_gemm(w.aq, mp, b, g, s);
}

}  // namespace

extern "C" {

int mcl4moe_nvfp4_mm(const void* x, int dtype, int64_t M, int K, int causal, const uint8_t* b, const uint8_t* b_scales,
                     const float* b_g, int N, const float* bias, float* out, float* a_global_scale,
                     int32_t* error_word, void* workspace, size_t workspace_bytes, mcl4moe_stream_t stream) {
  return nvfp4_mm_impl(x, dtype, M, K, causal, 0, 0, b, b_scales, b_g, N, bias, out, a_global_scale, error_word,
                       workspace, workspace_bytes, stream);
}

int mcl4moe_nvfp4_mm_sr(const void* x, int dtype, int64_t M, int K, int causal, uint64_t seed, const uint8_t* b,
                        const uint8_t* b_scales, const float* b_g, int N, const float* bias, float* out,
                        float* a_global_scale, int32_t* error_word, void* workspace, size_t workspace_bytes,
                        mcl4moe_stream_t stream) {
  return nvfp4_mm_impl(x, dtype, M, K, causal, 1, seed, b, b_scales, b_g, N, bias, out, a_global_scale, error_word,
                       workspace, workspace_bytes, stream);
}

int mcl4moe_quantize_activations(const uint16_t* x, int64_t rows, int cols, int64_t ld_x, uint8_t* packed,
                                 uint8_t* scales, int swizzled, mcl4moe_stream_t stream) {
  if (rows < 0 || cols <= 0 || ld_x < cols || !x || !packed || !scales) return MCL4MOE_ERR_INVALID;
  if (cols % 16 != 0) return MCL4MOE_ERR_INVALID;
  if (cols % 64 != 0 || ld_x % 8 != 0 || !aligned16(x)) return MCL4MOE_ERR_UNSUPPORTED;
  return launch_quantize_activations(x, rows, cols, ld_x, packed, scales, swizzled, stream);
}

size_t mcl4moe_route_workspace_size(int T, int E, int k, int d) {
  if (T < 0 || E <= 0 || k <= 0 || int64_t(T) * k > kMaxRoutedSlots) return 0;
  return route_workspace(nullptr, T, E, k, d > 0 ? d : 0).bytes;
}

int mcl4moe_route(const uint16_t* x, const float* wr, const float* logit_bias, const float* logits_in,
                  const uint8_t* valid, int T, int d, int E, int k, int norm_topk_prob, int32_t* topk_idx,
                  float* topk_w, float* logits_out, float* sel_mask, int32_t* counts, float* stats, void* workspace,
                  size_t workspace_bytes, mcl4moe_stream_t stream) {
  if (T < 0 || E <= 0 || k <= 0 || k > E || !topk_idx || !topk_w || !workspace) return MCL4MOE_ERR_INVALID;
  if (E > kMaxExperts || k > kMaxTopK) return MCL4MOE_ERR_UNSUPPORTED;
  if (int64_t(T) * k > kMaxRoutedSlots) return MCL4MOE_ERR_UNSUPPORTED;  // int32 counts, offsets and ranks
  if (!logits_in) {
    if (!x || !wr || d <= 0) return MCL4MOE_ERR_INVALID;
    if (d % 64 != 0 || !aligned16(x) || !aligned16(wr)) return MCL4MOE_ERR_UNSUPPORTED;
  }
  const RouteWorkspace ws = route_workspace(workspace, T, E, k, d > 0 ? d : 0);
  if (workspace_bytes < ws.bytes) return MCL4MOE_ERR_WORKSPACE;
  return launch_route(x, wr, logit_bias, logits_in, valid, T, d, E, k, norm_topk_prob, topk_idx, topk_w, logits_out,
                      sel_mask, counts, stats, nullptr, nullptr, ws, stream);
}

int64_t mcl4moe_padded_rows(int T, int E, int k) { return padded_rows_cap(T, E, k); }

size_t mcl4moe_moe_workspace_size(int T, int d, int E, int k, int F) {
  if (check_moe_shape(T, d, E, k, F) != MCL4MOE_OK) return 0;
  return moe_workspace(nullptr, T, d, E, k, F).bytes;
}

void* mcl4moe_workspace_region(void* workspace, int region, int T, int d, int E, int k, int F) {
  const MoeWorkspace w = moe_workspace(workspace, T, d, E, k, F);
  switch (region) {
    case 0: return w.xq;
    case 1: return w.xs;
    case 2: return w.hq;
    case 3: return w.hs;
    case 4: return w.y;
    case 5: return w.route.pad_start;
    case 6: return w.slot_pos;
    case 7: return w.sorted_w;
    case 8: return w.err;
    case 9: return w.route.counts;
    case 10: return w.route.offs_start;
    default: return nullptr;
  }
}

}  // extern "C"

namespace {

// Checks shared by both forward entry points; `routed`: the caller supplies topk_idx / topk_w.
int check_forward_args(const mcl4moe_moe_args* a, bool routed) {
  if (!a) return MCL4MOE_ERR_INVALID;
  int st = check_moe_shape(a->T, a->d, a->E, a->k, a->F);
  if (st != MCL4MOE_OK) return st;
  if (!a->workspace || (a->T > 0 && (!a->x || !a->out))) return MCL4MOE_ERR_INVALID;
  if (routed ? (a->T > 0 && (!a->topk_idx || !a->topk_w)) : (!a->stats || (a->T > 0 && !a->router_w)))
    return MCL4MOE_ERR_INVALID;
  if (!a->w_up || !a->w_up_scales || !a->w_up_g || !a->w_dn || !a->w_dn_scales || !a->w_dn_g)
    return MCL4MOE_ERR_INVALID;
  if (!aligned16(a->x) || !aligned16(a->out) || !aligned16(a->w_up) || !aligned16(a->w_dn) ||
      !aligned16(a->w_up_scales) || !aligned16(a->w_dn_scales) || (!routed && !aligned16(a->router_w)) ||
      (a->h_debug && !aligned16(a->h_debug)) || !aligned16(a->up_save) || !aligned16(a->x_rows_save) ||
      !aligned16(a->y_save))
    return MCL4MOE_ERR_INVALID;
  if (a->x_rows_save && a->d > 4096) return MCL4MOE_ERR_UNSUPPORTED;  // training rows of up to 4096
  return MCL4MOE_OK;
}

// Expert GEMM tiling: 0 = by shape, 1 = CTA-pair 256-row tiles, 2 = single-CTA 128-row tiles.
std::atomic<int> g_expert_tiling{0};

// Single-CTA 128-row tiles for the inference forward when experts average at most 64
// routed rows (decode): a pair tile would multiply mostly padding rows, while a 128-row
// block without routed rows is skipped.  The training forward keeps the pair tiles
// (its saves and the backward read every padded row).
bool use_solo_tiles(const mcl4moe_moe_args* a) {
  const int policy = g_expert_tiling.load(std::memory_order_relaxed);
  if (policy == 1 || a->up_save != nullptr || a->y_save != nullptr) return false;
  if (policy == 2) return true;
  return int64_t(a->T) * a->k <= int64_t(a->E) * 64;
}

// Permutation + NVFP4 activation quantisation, gate/up GEMM with SwiGLU, down
// GEMM with the routing weight, combine: everything after the expert layout.
int forward_experts(const mcl4moe_moe_args* a, const MoeWorkspace& w, const int32_t* topk_idx, const float* topk_w,
                    int32_t* err, cudaStream_t s, int (*mark)(const mcl4moe_moe_args*, int, cudaStream_t)) {
  const int T = a->T, d = a->d, E = a->E, k = a->k, F = a->F;
  int st = launch_permute_quantize(a->x, a->valid, topk_idx, topk_w, T, d, E, k, w.route, w.slot_pos, w.sorted_w,
                                   a->perm, w.xq, w.xs, s, a->x_rows_save);
  if (st != MCL4MOE_OK) return st;
  if ((st = mark(a, 2, s)) != MCL4MOE_OK) return st;
  const int64_t mcap = padded_rows_cap(T, E, k);
  const int solo = use_solo_tiles(a) ? 1 : 0;

  GemmArgs g1{};
  g1.pad_start = w.route.pad_start;
  g1.row_count = w.route.counts;
  g1.a_scales = w.xs;
  g1.a_sf_rowmajor = 1;
  g1.b_scales = a->w_up_scales;
  g1.b_g = a->w_up_g;
  g1.E = E;
  g1.K = d;
  g1.N_total = 2 * F;
  g1.n_tiles = F / 128;
  g1.mode = 0;
  g1.F = F;
  g1.hq = w.hq;
  g1.hs = w.hs;
  g1.h_dbg = a->h_debug;
  g1.up_save = a->up_save;
  g1.err = err;
  g1.solo = solo;
  st = launch_grouped_gemm(w.xq, mcap, a->w_up, g1, s);
  if (st != MCL4MOE_OK) return st;
  if ((st = mark(a, 3, s)) != MCL4MOE_OK) return st;

  GemmArgs g2{};
  g2.pad_start = w.route.pad_start;
  g2.row_count = w.route.counts;
  g2.a_scales = w.hs;
  g2.b_scales = a->w_dn_scales;
  g2.b_g = a->w_dn_g;
  g2.E = E;
  g2.K = F;
  g2.N_total = d;
  g2.n_tiles = d / 256;
  g2.mode = 1;
  // training keeps the unweighted rows (the routing-weight gradient needs them) and weights in the combine
  g2.row_w = a->y_save ? nullptr : w.sorted_w;
  g2.y = a->y_save ? a->y_save : w.y;
  g2.ldy = d;
  g2.err = err;
  g2.solo = solo;
  st = launch_grouped_gemm(w.hq, mcap, a->w_dn, g2, s);
  if (st != MCL4MOE_OK) return st;
  if ((st = mark(a, 4, s)) != MCL4MOE_OK) return st;
  st = launch_combine(g2.y, w.slot_pos, a->valid, T, k, d, a->out, s, a->y_save ? w.sorted_w : nullptr);
  if (st != MCL4MOE_OK) return st;
  return mark(a, 5, s);
}

// Down projection with the routing weight and combine, on h rows already in the expert-major
// layout (hq codes [M_cap, F/2], swizzled hs scales) that the permute of this call laid out.
int experts_down(const mcl4moe_moe_args* a, const MoeWorkspace& w, const uint8_t* hq, const uint8_t* hs,
                 int32_t* err, cudaStream_t s) {
  const int T = a->T, d = a->d, E = a->E, k = a->k, F = a->F;
  const int64_t mcap = padded_rows_cap(T, E, k);
  GemmArgs g2{};
  g2.pad_start = w.route.pad_start;
  g2.row_count = w.route.counts;
  g2.a_scales = hs;
  g2.b_scales = a->w_dn_scales;
  g2.b_g = a->w_dn_g;
  g2.E = E;
  g2.K = F;
  g2.N_total = d;
  g2.n_tiles = d / 256;
  g2.mode = 1;
  g2.row_w = w.sorted_w;
  g2.y = w.y;
  g2.ldy = d;
  g2.err = err;
  g2.solo = use_solo_tiles(a) ? 1 : 0;
  int st = launch_grouped_gemm(hq, mcap, a->w_dn, g2, s);
  if (st != MCL4MOE_OK) return st;
  return launch_combine(w.y, w.slot_pos, a->valid, T, k, d, a->out, s, nullptr);
}

int mark_stage(const mcl4moe_moe_args* a, int i, cudaStream_t s) {
  if (a->stage_events == nullptr || a->stage_events[i] == nullptr) return MCL4MOE_OK;
  return cudaEventRecord(static_cast<cudaEvent_t>(a->stage_events[i]), s) == cudaSuccess ? MCL4MOE_OK
                                                                                          : MCL4MOE_ERR_CUDA;
}

// A caller-owned error word is sticky (kernels skip work while it is nonzero);
// the workspace's own word is cleared for every call.
int32_t* error_word(const mcl4moe_moe_args* a, const MoeWorkspace& w, cudaStream_t s, int* st) {
  *st = MCL4MOE_OK;
  if (a->error_word) return a->error_word;
  if (cudaMemsetAsync(w.err, 0, sizeof(int32_t), s) != cudaSuccess) *st = MCL4MOE_ERR_CUDA;
  return w.err;
}

}  // namespace

extern "C" {

int mcl4moe_set_expert_tiling(int mode) {
  if (mode < 0 || mode > 2) return -1;
  return g_expert_tiling.exchange(mode);
}

int mcl4moe_moe_forward(const mcl4moe_moe_args* a, mcl4moe_stream_t stream) {
  int st = check_forward_args(a, false);
  if (st != MCL4MOE_OK) return st;
  const MoeWorkspace w = moe_workspace(a->workspace, a->T, a->d, a->E, a->k, a->F);
  if (a->workspace_bytes < w.bytes) return MCL4MOE_ERR_WORKSPACE;
  cudaStream_t s = stream;
  const int T = a->T, d = a->d, E = a->E, k = a->k;
  int32_t* err = error_word(a, w, s, &st);
  if (st != MCL4MOE_OK) return st;
  int32_t* topk_idx = a->topk_idx ? a->topk_idx : w.topk_idx;
  float* topk_w = a->topk_w ? a->topk_w : w.topk_w;
  if ((st = mark_stage(a, 0, s)) != MCL4MOE_OK) return st;
  st = launch_route(a->x, a->router_w, a->logit_bias, nullptr, a->valid, T, d, E, k, a->norm_topk_prob, topk_idx,
                    topk_w, a->logits_out, a->sel_mask, w.counts, a->stats, a->offs, err, w.route, s);
  if (st != MCL4MOE_OK) return st;
  if ((st = mark_stage(a, 1, s)) != MCL4MOE_OK) return st;
  if (T == 0) {
    for (int i = 2; i < 6; ++i)
      if ((st = mark_stage(a, i, s)) != MCL4MOE_OK) return st;
    return MCL4MOE_OK;
  }
  return forward_experts(a, w, topk_idx, topk_w, err, s, mark_stage);
}

int mcl4moe_moe_forward_layout(const mcl4moe_moe_args* a, mcl4moe_stream_t stream) {
  if (!a) return MCL4MOE_ERR_INVALID;
  int st = check_moe_shape(a->T, a->d, a->E, a->k, a->F);
  if (st != MCL4MOE_OK) return st;
  if (!a->workspace || !a->stats || (a->T > 0 && (!a->x || !a->router_w))) return MCL4MOE_ERR_INVALID;
  if (!aligned16(a->x) || !aligned16(a->router_w)) return MCL4MOE_ERR_INVALID;
  const MoeWorkspace w = moe_workspace(a->workspace, a->T, a->d, a->E, a->k, a->F);
  if (a->workspace_bytes < w.bytes) return MCL4MOE_ERR_WORKSPACE;
  cudaStream_t s = stream;
  const int T = a->T, d = a->d, E = a->E, k = a->k;
  int32_t* err = error_word(a, w, s, &st);
  if (st != MCL4MOE_OK) return st;
  int32_t* topk_idx = a->topk_idx ? a->topk_idx : w.topk_idx;
  float* topk_w = a->topk_w ? a->topk_w : w.topk_w;
  st = launch_route(a->x, a->router_w, a->logit_bias, nullptr, a->valid, T, d, E, k, a->norm_topk_prob, topk_idx,
                    topk_w, a->logits_out, a->sel_mask, w.counts, a->stats, a->offs, err, w.route, s);
  if (st != MCL4MOE_OK || T == 0) return st;
  // the layout only: the dispatched rows carry the NVFP4 codes (rows of up to 4096 elements;
  // wider rows take the generic permute, which also writes the codes)
  const bool codes = d / 16 > 256;
  return launch_permute_quantize(a->x, a->valid, topk_idx, topk_w, T, d, E, k, w.route, w.slot_pos, w.sorted_w,
                                 a->perm, codes ? w.xq : nullptr, codes ? w.xs : nullptr, s, nullptr);
}

int mcl4moe_moe_forward_down(const mcl4moe_moe_args* a, const uint8_t* hq, const uint8_t* hs,
                             mcl4moe_stream_t stream) {
  if (!a) return MCL4MOE_ERR_INVALID;
  int st = check_moe_shape(a->T, a->d, a->E, a->k, a->F);
  if (st != MCL4MOE_OK) return st;
  if (!a->workspace || !a->w_dn || !a->w_dn_scales || !a->w_dn_g || (a->T > 0 && !a->out)) return MCL4MOE_ERR_INVALID;
  if (!aligned16(a->out) || !aligned16(a->w_dn) || !aligned16(a->w_dn_scales) || !aligned16(hq) || !aligned16(hs))
    return MCL4MOE_ERR_INVALID;
  const MoeWorkspace w = moe_workspace(a->workspace, a->T, a->d, a->E, a->k, a->F);
  if (a->workspace_bytes < w.bytes) return MCL4MOE_ERR_WORKSPACE;
  if (a->T == 0) return MCL4MOE_OK;
  cudaStream_t s = stream;
  int32_t* err = error_word(a, w, s, &st);
  if (st != MCL4MOE_OK) return st;
  return experts_down(a, w, hq ? hq : w.hq, hs ? hs : w.hs, err, s);
}

int mcl4moe_moe_forward_routed(const mcl4moe_moe_args* a, mcl4moe_stream_t stream) {
  int st = check_forward_args(a, true);
  if (st != MCL4MOE_OK) return st;
  const MoeWorkspace w = moe_workspace(a->workspace, a->T, a->d, a->E, a->k, a->F);
  if (a->workspace_bytes < w.bytes) return MCL4MOE_ERR_WORKSPACE;
  cudaStream_t s = stream;
  const int T = a->T, E = a->E, k = a->k;
  int32_t* err = error_word(a, w, s, &st);
  if (st != MCL4MOE_OK) return st;
  if ((st = mark_stage(a, 0, s)) != MCL4MOE_OK) return st;
  st = launch_route_from_indices(a->topk_idx, a->valid, T, E, k, w.counts, a->stats, a->offs, w.route, s);
  if (st != MCL4MOE_OK) return st;
  if ((st = mark_stage(a, 1, s)) != MCL4MOE_OK) return st;
  if (T == 0) {
    for (int i = 2; i < 6; ++i)
      if ((st = mark_stage(a, i, s)) != MCL4MOE_OK) return st;
    return MCL4MOE_OK;
  }
  return forward_experts(a, w, a->topk_idx, a->topk_w, err, s, mark_stage);
}

size_t mcl4moe_grouped_linear_workspace_size(int64_t M, int K, int E) {
  if (M < 0 || K <= 0 || E <= 0) return 0;
  const int64_t mcap = padded_rows_cap(M, E, 1);
  size_t off = 0;
  off += align256(sizeof(int32_t) * (E + 1));  // pad_start
  off += align256(sizeof(int32_t) * E);        // offs_start
  off += align256(sizeof(int32_t) * E);        // counts
  off += align256(size_t(mcap) * K / 2);       // xq
  off += align256(size_t(mcap) * K / 16);      // xs
  off += align256(sizeof(int32_t));            // error word
  return off;
}

int mcl4moe_grouped_linear(const uint16_t* x, int64_t M, int K, const int32_t* offs, int E, const uint8_t* w,
                           const uint8_t* w_scales, const float* w_g, int N, uint16_t* out, int32_t* error_word,
                           void* workspace, size_t workspace_bytes, mcl4moe_stream_t stream) {
  if (M < 0 || K <= 0 || N <= 0 || E <= 0 || !offs || !w || !w_scales || !w_g || !out || !workspace)
    return MCL4MOE_ERR_INVALID;
  if (M > 0 && !x) return MCL4MOE_ERR_INVALID;
  if (K % 16 != 0) return MCL4MOE_ERR_INVALID;
  if (K % 256 != 0 || N % 256 != 0 || E > kMaxExperts) return MCL4MOE_ERR_UNSUPPORTED;
  if (!aligned16(x) || !aligned16(out) || !aligned16(w) || !aligned16(w_scales)) return MCL4MOE_ERR_INVALID;
  if (workspace_bytes < mcl4moe_grouped_linear_workspace_size(M, K, E)) return MCL4MOE_ERR_WORKSPACE;
  if (M == 0) return MCL4MOE_OK;
  const int64_t mcap = padded_rows_cap(M, E, 1);
  uint8_t* p = static_cast<uint8_t*>(workspace);
  size_t off = 0;
  auto take = [&](size_t bytes) {
    uint8_t* r = p + off;
    off += align256(bytes);
    return r;
  };
  int32_t* pad_start = reinterpret_cast<int32_t*>(take(sizeof(int32_t) * (E + 1)));
  int32_t* offs_start = reinterpret_cast<int32_t*>(take(sizeof(int32_t) * E));
  int32_t* counts = reinterpret_cast<int32_t*>(take(sizeof(int32_t) * E));
  uint8_t* xq = take(size_t(mcap) * K / 2);
  uint8_t* xs = take(size_t(mcap) * K / 16);
  int32_t* err = error_word ? error_word : reinterpret_cast<int32_t*>(take(sizeof(int32_t)));
  cudaStream_t s = stream;
  if (!error_word && cudaMemsetAsync(err, 0, sizeof(int32_t), s) != cudaSuccess) return MCL4MOE_ERR_CUDA;
  int st = launch_pad_from_offs(offs, E, pad_start, offs_start, counts, s);
  if (st != MCL4MOE_OK) return st;
  st = launch_quantize_grouped_rows(x, M, K, offs, pad_start, counts, E, xq, xs, s);
  if (st != MCL4MOE_OK) return st;
  GemmArgs g{};
  g.pad_start = pad_start;
  g.row_count = counts;
  g.out_row_base = offs_start;
  g.a_scales = xs;
  g.a_sf_rowmajor = 1;
  g.b_scales = w_scales;
  g.b_g = w_g;
  g.E = E;
  g.K = K;
  g.N_total = N;
  g.n_tiles = N / 256;
  g.mode = 1;
  g.y = out;
  g.ldy = N;
  g.err = err;
  return launch_grouped_gemm(xq, mcap, w, g, s);
}

}  // extern "C"
