// Router / top-k / stable expert-major permutation / activation scatter / combine.
//
// Restates the routing and data-movement parts of SparseMoE.forward
// (src/mcl4_coe/backbone.py:787-911, loop branch :913-1047):
//   logits = x.float() @ Wr.float()^T (+ bias)   probs = softmax(logits)
//   w, sel = topk(probs, k)  (w /= max(sum w, 1e-9) when norm_topk_prob)
//   perm   = argsort(sel.flatten(), stable=True)  -> expert-major, token order
//   out[t] = bf16(sum_j bf16(y[t, j] * bf16(w[t, j])))
// The permutation is a deterministic counting sort: each router CTA ranks the
// slots of its 64 tokens per expert with warp ballots (token order), a
// single-CTA scan turns per-chunk counts into offsets, and the scatter kernel
// writes every slot at  pad_start[e] + (slots of e in earlier chunks) + rank.
// Expert segments are padded to multiples of 128 rows (the GEMM M tile).
#include "kernels.cuh"

namespace mcl4 {

namespace {

constexpr int kRouteThreads = 256;
constexpr int kKC = 32;  // K chunk of the router product

struct RouteSmem {
  float xs[kKC][kRouteTokens];  // x chunk, k-major
  float ws[kKC][64];            // router weight chunk, k-major
};

__device__ __forceinline__ unsigned long long warp_max_u64(unsigned long long v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    unsigned long long w = __shfl_xor_sync(0xffffffffu, v, o);
    v = w > v ? w : v;
  }
  return v;
}
__device__ __forceinline__ float warp_max_f(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum_f(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

}  // namespace

// One CTA routes 64 tokens: router product, softmax, top-k, statistics and
// per-chunk stable ranks.  Dynamic shared memory: logits [64][E] + selections.
template <int EW>  // experts per lane = ceil(E / 32) rounded up to the instantiation
__global__ void __launch_bounds__(kRouteThreads) router_kernel(
    const uint16_t* __restrict__ x, const float* __restrict__ wr, const float* __restrict__ bias,
    const float* __restrict__ logits_in, const uint8_t* __restrict__ valid, int T, int d, int E, int k, int norm_topk,
    int32_t* __restrict__ topk_idx, float* __restrict__ topk_w, float* __restrict__ logits_out,
    float* __restrict__ sel_mask, RouteWorkspace ws) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  float* logits_s = reinterpret_cast<float*>(smem_raw);                      // [64][E]
  int32_t* sel_s = reinterpret_cast<int32_t*>(logits_s + kRouteTokens * E);  // [64][k]
  int32_t* rank_s = sel_s + kRouteTokens * k;                                // [64][k]
  int32_t* gcount_s = rank_s + kRouteTokens * k;                             // [2][E]
  float* red_s = reinterpret_cast<float*>(gcount_s + 2 * E);                 // [8][E + 2]
  RouteSmem* gs = reinterpret_cast<RouteSmem*>((reinterpret_cast<uintptr_t>(red_s + 8 * (E + 2)) + 15) & ~uintptr_t(15));

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int chunk = blockIdx.x;
  const int t0 = chunk * kRouteTokens;
  if (chunk == 0 && tid == 0) *ws.done = 0u;  // the scan kernel runs after this one

  // ------------------------------------------------ logits
  if (logits_in != nullptr) {
    for (int i = tid; i < kRouteTokens * E; i += kRouteThreads) {
      const int tok = i / E, e = i - tok * E;
      logits_s[i] = (t0 + tok < T) ? logits_in[int64_t(t0 + tok) * E + e] : 0.f;
    }
  } else {
    const int ty = tid >> 4, tx = tid & 15;
    const int ld_tok = tid & 63, ld_part = tid >> 6;
    for (int ec = 0; ec < E; ec += 64) {
      float acc[4][4];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
      for (int k0 = 0; k0 < d; k0 += kKC) {
        {  // x chunk: token ld_tok, elements k0 + 8*ld_part .. +8
          float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
          if (t0 + ld_tok < T) {
            uint4 u = __ldg(reinterpret_cast<const uint4*>(x + int64_t(t0 + ld_tok) * d + k0 + ld_part * 8));
            const uint32_t w4[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              v[2 * i] = bf16_to_f32(uint16_t(w4[i] & 0xFFFFu));
              v[2 * i + 1] = bf16_to_f32(uint16_t(w4[i] >> 16));
            }
          }
#pragma unroll
          for (int i = 0; i < 8; ++i) gs->xs[ld_part * 8 + i][ld_tok] = v[i];
          float wv[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
          const int e = ec + ld_tok;
          if (e < E) {
            const float4* p = reinterpret_cast<const float4*>(wr + int64_t(e) * d + k0 + ld_part * 8);
            float4 a = __ldg(p), b = __ldg(p + 1);
            wv[0] = a.x; wv[1] = a.y; wv[2] = a.z; wv[3] = a.w; wv[4] = b.x; wv[5] = b.y; wv[6] = b.z; wv[7] = b.w;
          }
#pragma unroll
          for (int i = 0; i < 8; ++i) gs->ws[ld_part * 8 + i][ld_tok] = wv[i];
        }
        __syncthreads();
#pragma unroll 8
        for (int kk = 0; kk < kKC; ++kk) {
          const float4 a = *reinterpret_cast<const float4*>(&gs->xs[kk][ty * 4]);
          const float4 b = *reinterpret_cast<const float4*>(&gs->ws[kk][tx * 4]);
          const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
          for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
        }
        __syncthreads();
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int e = ec + tx * 4 + j;
          if (e < E) logits_s[(ty * 4 + i) * E + e] = bias ? __fadd_rn(acc[i][j], bias[e]) : acc[i][j];
        }
    }
  }
  __syncthreads();

  // ------------------------------------------------ softmax, top-k, statistics
  float prob_acc[EW];
#pragma unroll
  for (int i = 0; i < EW; ++i) prob_acc[i] = 0.f;
  float lse2_acc = 0.f, nval_acc = 0.f;
  for (int tok = warp * 8; tok < warp * 8 + 8; ++tok) {
    const int t = t0 + tok;
    if (t >= T) break;
    float l[EW];
#pragma unroll
    for (int i = 0; i < EW; ++i) {
      const int e = lane + 32 * i;
      l[i] = e < E ? logits_s[tok * E + e] : -INFINITY;
      if (logits_out != nullptr && e < E) logits_out[int64_t(t) * E + e] = l[i];
    }
    const bool routed = valid == nullptr || valid[t] != 0;
    if (!routed) {
      if (lane < k) {
        topk_idx[int64_t(t) * k + lane] = -1;
        topk_w[int64_t(t) * k + lane] = 0.f;
        sel_s[tok * k + lane] = -1;
      }
      if (sel_mask != nullptr)
#pragma unroll
        for (int i = 0; i < EW; ++i)
          if (lane + 32 * i < E) sel_mask[int64_t(t) * E + lane + 32 * i] = 0.f;
      continue;
    }
    float m = -INFINITY;
#pragma unroll
    for (int i = 0; i < EW; ++i) m = fmaxf(m, l[i]);
    m = warp_max_f(m);
    float p[EW], s = 0.f;
#pragma unroll
    for (int i = 0; i < EW; ++i) {
      p[i] = (lane + 32 * i < E) ? expf(__fsub_rn(l[i], m)) : 0.f;
      s = __fadd_rn(s, p[i]);
    }
    s = warp_sum_f(s);
    const float inv_s = __frcp_rn(s);
    const float lse = __fadd_rn(m, logf(s));
    lse2_acc = __fadd_rn(lse2_acc, __fmul_rn(lse, lse));
    nval_acc += 1.f;
#pragma unroll
    for (int i = 0; i < EW; ++i) {
      p[i] = __fmul_rn(p[i], inv_s);
      prob_acc[i] = __fadd_rn(prob_acc[i], p[i]);
    }
    // top-k: largest probability first, ties to the lower expert index
    uint32_t taken = 0;
    int my_e = -1;
    float my_p = 0.f;
    for (int j = 0; j < k; ++j) {
      unsigned long long best = 0;
#pragma unroll
      for (int i = 0; i < EW; ++i) {
        const int e = lane + 32 * i;
        if (e < E && !((taken >> i) & 1u)) {
          const unsigned long long key =
              (static_cast<unsigned long long>(__float_as_uint(p[i])) << 32) | (0xFFFFFFFFu - uint32_t(e));
          best = key > best ? key : best;
        }
      }
      best = warp_max_u64(best);
      const int e_star = int(0xFFFFFFFFu - uint32_t(best & 0xFFFFFFFFull));
      if ((e_star & 31) == lane) taken |= 1u << (e_star >> 5);
      if (lane == j) {
        my_e = e_star;
        my_p = __uint_as_float(uint32_t(best >> 32));
      }
    }
    float w = my_p;
    if (norm_topk) {
      float sum = 0.f;
      for (int j = 0; j < k; ++j) sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, my_p, j));
      w = __fdiv_rn(my_p, fmaxf(sum, 1e-9f));
    }
    if (lane < k) {
      topk_idx[int64_t(t) * k + lane] = my_e;
      topk_w[int64_t(t) * k + lane] = w;
      sel_s[tok * k + lane] = my_e;
    }
    if (sel_mask != nullptr)
#pragma unroll
      for (int i = 0; i < EW; ++i)
        if (lane + 32 * i < E) sel_mask[int64_t(t) * E + lane + 32 * i] = ((taken >> i) & 1u) ? 1.f : 0.f;
  }
  // tokens beyond T (last chunk) take no slot
  for (int i = tid; i < kRouteTokens * k; i += kRouteThreads)
    if (t0 + i / k >= T) sel_s[i] = -1;
#pragma unroll
  for (int i = 0; i < EW; ++i)
    if (lane + 32 * i < E) red_s[warp * (E + 2) + lane + 32 * i] = prob_acc[i];
  if (lane == 0) {
    red_s[warp * (E + 2) + E] = lse2_acc;
    red_s[warp * (E + 2) + E + 1] = nval_acc;
  }
  __syncthreads();

  // ------------------------------------------------ per-chunk statistics (fixed warp order)
  for (int e = tid; e < E + 2; e += kRouteThreads) {
    float a = 0.f;
    for (int w8 = 0; w8 < 8; ++w8) a = __fadd_rn(a, red_s[w8 * (E + 2) + e]);
    if (e < E) ws.part_probs[int64_t(chunk) * E + e] = a;
    else ws.part_misc[int64_t(chunk) * 2 + (e - E)] = a;
  }

  // ------------------------------------------------ stable ranks (warps 0, 1: 32 tokens each)
  if (warp < 2) {
    const int tok = warp * 32 + lane;
    uint32_t mw[EW];
#pragma unroll
    for (int i = 0; i < EW; ++i) mw[i] = 0;
    for (int j = 0; j < k; ++j) {
      const int e = sel_s[tok * k + j];
      if (e >= 0) {
#pragma unroll
        for (int i = 0; i < EW; ++i)
          if ((e >> 5) == i) mw[i] |= 1u << (e & 31);
      }
    }
    const uint32_t lt = (1u << lane) - 1u;
#pragma unroll
    for (int i = 0; i < EW; ++i) {
      for (int b = 0; b < 32; ++b) {
        const int e = i * 32 + b;
        if (e >= E) break;
        const bool has = (mw[i] >> b) & 1u;
        const uint32_t bal = __ballot_sync(0xffffffffu, has);
        if (has) {
          const int r = __popc(bal & lt);
          for (int j = 0; j < k; ++j)
            if (sel_s[tok * k + j] == e) rank_s[tok * k + j] = r;
        }
        if (lane == 0) gcount_s[warp * E + e] = __popc(bal);
      }
    }
  }
  __syncthreads();
  for (int e = tid; e < E; e += kRouteThreads)
    ws.chunk_excl[int64_t(chunk) * E + e] = gcount_s[e] + gcount_s[E + e];
  for (int i = tid; i < kRouteTokens * k; i += kRouteThreads) {
    const int tok = i / k;
    const int e = sel_s[i];
    if (t0 + tok < T) ws.local_rank[int64_t(t0) * k + i] = e < 0 ? 0 : rank_s[i] + (tok >= 32 ? gcount_s[e] : 0);
  }
}

// One CTA per expert: exclusive prefix of the expert's per-chunk slot counts
// (a block-wide scan over chunks) and its probability sum.  The last CTA to
// finish (counted with an atomic after a memory fence; no CTA waits on
// another) lays out the expert segments and finalises the statistics.
namespace {

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

}  // namespace

__global__ void __launch_bounds__(256) route_scan_kernel(int C, int E, int k, RouteWorkspace ws, int32_t* counts_out,
                                                         float* stats, int32_t* offs_out) {
  __shared__ int32_t itmp[64];
  __shared__ float ftmp[32];
  __shared__ bool is_last;
  const int tid = threadIdx.x;
  const int e = blockIdx.x;
  const int per = (C + blockDim.x - 1) / blockDim.x;
  const int c0 = tid * per, c1 = min(C, c0 + per);
  int32_t mine = 0;
  float ps = 0.f;
  for (int c = c0; c < c1; ++c) {
    mine += ws.chunk_excl[int64_t(c) * E + e];
    ps = __fadd_rn(ps, ws.part_probs[int64_t(c) * E + e]);
  }
  int32_t total;
  int32_t run = block_exclusive_scan(mine, itmp, total);
  for (int c = c0; c < c1; ++c) {
    const int32_t v = ws.chunk_excl[int64_t(c) * E + e];
    ws.chunk_excl[int64_t(c) * E + e] = run;
    run += v;
  }
  const float psum = block_sum(ps, ftmp);
  if (tid == 0) {
    ws.counts[e] = total;
    ws.probs_sum[e] = psum;
    __threadfence();
    is_last = atomicAdd(ws.done, 1u) == uint32_t(E - 1);
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();

  // ---- last CTA: expert layout and statistics
  float l2 = 0.f, nv = 0.f;
  for (int c = c0; c < c1; ++c) {
    l2 = __fadd_rn(l2, ws.part_misc[2 * c]);
    nv = __fadd_rn(nv, ws.part_misc[2 * c + 1]);
  }
  const float lse2 = block_sum(l2, ftmp);
  const float n = block_sum(nv, ftmp);
  if (tid == 0) {
    int32_t urun = 0, prun = 0;
    float aux = 0.f;
    const float denom = n * float(k);
    for (int x = 0; x < E; ++x) {
      const int32_t cnt = __ldcg(ws.counts + x);
      ws.offs_start[x] = urun;
      ws.pad_start[x] = prun;
      urun += cnt;
      prun += (cnt + 127) / 128 * 128;
      if (offs_out) offs_out[x] = urun;
      if (counts_out) counts_out[x] = cnt;
      if (stats) {
        const float cf = n > 0.f ? __fdiv_rn(float(cnt), denom) : 0.f;
        stats[3 + x] = cf;
        if (n > 0.f) aux = __fadd_rn(aux, __fmul_rn(cf, __fdiv_rn(__ldcg(ws.probs_sum + x), n)));
      }
    }
    ws.pad_start[E] = prun;
    if (stats) {
      stats[0] = n > 0.f ? __fmul_rn(float(E), aux) : 0.f;
      stats[1] = n > 0.f ? __fdiv_rn(lse2, n) : 0.f;
      stats[2] = n;
    }
  }
}

template <int EW>
static int launch_router_t(const uint16_t* x, const float* wr, const float* bias, const float* logits_in,
                           const uint8_t* valid, int T, int d, int E, int k, int norm_topk, int32_t* topk_idx,
                           float* topk_w, float* logits_out, float* sel_mask, const RouteWorkspace& ws,
                           cudaStream_t stream) {
  const size_t smem = sizeof(float) * kRouteTokens * E + sizeof(int32_t) * 2 * kRouteTokens * k +
                      sizeof(int32_t) * 2 * E + sizeof(float) * 8 * (E + 2) + sizeof(RouteSmem) + 16;
  static bool configured = false;
  if (!configured) {
    if (cudaFuncSetAttribute(router_kernel<EW>, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024) != cudaSuccess)
      return MCL4MOE_ERR_CUDA;
    configured = true;
  }
  const int C = (T + kRouteTokens - 1) / kRouteTokens;
  router_kernel<EW><<<C, kRouteThreads, smem, stream>>>(x, wr, bias, logits_in, valid, T, d, E, k, norm_topk, topk_idx,
                                                         topk_w, logits_out, sel_mask, ws);
  return cudaGetLastError() == cudaSuccess ? MCL4MOE_OK : MCL4MOE_ERR_CUDA;
}

int launch_route(const uint16_t* x, const float* wr, const float* bias, const float* logits_in, const uint8_t* valid,
                 int T, int d, int E, int k, int norm_topk, int32_t* topk_idx, float* topk_w, float* logits_out,
                 float* sel_mask, int32_t* counts_out, float* stats, int32_t* offs_out, const RouteWorkspace& ws,
                 cudaStream_t stream) {
  if (T > 0) {
    int st;
    if (E <= 32) st = launch_router_t<1>(x, wr, bias, logits_in, valid, T, d, E, k, norm_topk, topk_idx, topk_w,
                                         logits_out, sel_mask, ws, stream);
    else if (E <= 64) st = launch_router_t<2>(x, wr, bias, logits_in, valid, T, d, E, k, norm_topk, topk_idx, topk_w,
                                              logits_out, sel_mask, ws, stream);
    else if (E <= 128) st = launch_router_t<4>(x, wr, bias, logits_in, valid, T, d, E, k, norm_topk, topk_idx, topk_w,
                                               logits_out, sel_mask, ws, stream);
    else st = launch_router_t<8>(x, wr, bias, logits_in, valid, T, d, E, k, norm_topk, topk_idx, topk_w, logits_out,
                                 sel_mask, ws, stream);
    if (st != MCL4MOE_OK) return st;
  }
  const int C = (T + kRouteTokens - 1) / kRouteTokens;
  if (T == 0) {  // no router CTA ran: reset the finished-expert counter here
    if (cudaMemsetAsync(ws.done, 0, sizeof(uint32_t), stream) != cudaSuccess) return MCL4MOE_ERR_CUDA;
  }
  route_scan_kernel<<<E, 256, 0, stream>>>(C, E, k, ws, counts_out, stats, offs_out);
  return cudaGetLastError() == cudaSuccess ? MCL4MOE_OK : MCL4MOE_ERR_CUDA;
}

// ---------------------------------------------------------------- permute + quantise

// Blocks [0, ceil(T/8)): one warp per token, quantise its row once and write
// it to its k slots.  Blocks after: one per expert, zero the scales of the
// padding rows of that expert's segment (zero scale => zero contribution).
__global__ void __launch_bounds__(256) permute_quant_kernel(
    const uint16_t* __restrict__ x, const uint8_t* __restrict__ valid, const int32_t* __restrict__ topk_idx,
    const float* __restrict__ topk_w, int T, int d, int E, int k, RouteWorkspace ws, int32_t* __restrict__ slot_pos,
    float* __restrict__ sorted_w, int32_t* __restrict__ perm, uint8_t* __restrict__ xq, uint8_t* __restrict__ xs) {
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
      *reinterpret_cast<uint32_t*>(xs + swizzled_scale_offset(uint64_t(r), uint32_t(4 * g), uint32_t(nblk))) = 0u;
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
  int my_pos = 0;
  if (lane < k) {
    const int e = topk_idx[int64_t(t) * k + lane];
    const int r = ws.local_rank[int64_t(t) * k + lane];
    const int base = ws.chunk_excl[int64_t(chunk) * E + e] + r;
    my_pos = ws.pad_start[e] + base;
    slot_pos[int64_t(t) * k + lane] = my_pos;
    sorted_w[my_pos] = topk_w[int64_t(t) * k + lane];
    if (perm != nullptr) perm[ws.offs_start[e] + base] = t * k + lane;
  }
  for (int b0 = 0; b0 < nblk; b0 += 32) {
    const int b = b0 + lane;
    uint32_t s = 0;
    uint2 pk = make_uint2(0, 0);
    if (b < nblk) {
      const uint4* src = reinterpret_cast<const uint4*>(x + int64_t(t) * d + b * 16);
      uint4 u0 = __ldg(src), u1 = __ldg(src + 1);
      const uint32_t wds[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
      s = quantize_block16_bf16(wds, pk);
    }
    const int base_lane = lane & ~3;
    uint32_t word = 0;
#pragma unroll
    for (int q = 0; q < 4; ++q) word |= (__shfl_sync(0xffffffffu, s, base_lane + q) & 0xFFu) << (8 * q);
    for (int j = 0; j < k; ++j) {
      const int p = __shfl_sync(0xffffffffu, my_pos, j);
      if (b < nblk) {
        *reinterpret_cast<uint2*>(xq + int64_t(p) * (d / 2) + b * 8) = pk;
        if ((lane & 3) == 0)
          *reinterpret_cast<uint32_t*>(xs + swizzled_scale_offset(uint64_t(p), uint32_t(b), uint32_t(nblk))) = word;
      }
    }
  }
}

int launch_permute_quantize(const uint16_t* x, const uint8_t* valid, const int32_t* topk_idx, const float* topk_w,
                            int T, int d, int E, int k, const RouteWorkspace& ws, int32_t* slot_pos, float* sorted_w,
                            int32_t* perm, uint8_t* xq, uint8_t* xs, cudaStream_t stream) {
  const int blocks = (T + 7) / 8 + E;
  permute_quant_kernel<<<blocks, 256, 0, stream>>>(x, valid, topk_idx, topk_w, T, d, E, k, ws, slot_pos, sorted_w,
                                                   perm, xq, xs);
  return cudaGetLastError() == cudaSuccess ? MCL4MOE_OK : MCL4MOE_ERR_CUDA;
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
    prun += (c + 127) / 128 * 128;
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
  const int lane = threadIdx.x & 31;
  const int nblk = K / 16;
  const int64_t row_blocks = (M + 7) / 8;
  if (int64_t(blockIdx.x) >= row_blocks) {
    const int e = int(blockIdx.x - row_blocks);
    const int start = pad_start[e] + counts[e], end = pad_start[e + 1];
    const int groups = nblk / 4;
    for (int i = threadIdx.x; i < (end - start) * groups; i += blockDim.x) {
      const int r = start + i / groups, g = i % groups;
      *reinterpret_cast<uint32_t*>(xs + swizzled_scale_offset(uint64_t(r), uint32_t(4 * g), uint32_t(nblk))) = 0u;
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
      s = quantize_block16_bf16(wds, pk);
      *reinterpret_cast<uint2*>(xq + p * (K / 2) + b * 8) = pk;
    }
    const int base_lane = lane & ~3;
    uint32_t word = 0;
#pragma unroll
    for (int q = 0; q < 4; ++q) word |= (__shfl_sync(0xffffffffu, s, base_lane + q) & 0xFFu) << (8 * q);
    if ((lane & 3) == 0 && b < nblk)
      *reinterpret_cast<uint32_t*>(xs + swizzled_scale_offset(uint64_t(p), uint32_t(b), uint32_t(nblk))) = word;
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
__global__ void __launch_bounds__(256) combine_kernel(const uint16_t* __restrict__ y,
                                                      const int32_t* __restrict__ slot_pos,
                                                      const uint8_t* __restrict__ valid, int T, int k, int d,
                                                      uint16_t* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (t >= T) return;
  const bool routed = valid == nullptr || valid[t] != 0;
  int my_pos = 0;
  if (routed && lane < k) my_pos = slot_pos[int64_t(t) * k + lane];
  for (int c = lane * 8; c < d; c += 256) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (routed) {
      for (int j = 0; j < k; ++j) {
        const int p = __shfl_sync(0xffffffffu, my_pos, j);
        const uint4 u = __ldg(reinterpret_cast<const uint4*>(y + int64_t(p) * d + c));
        const uint32_t w4[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          acc[2 * i] = __fadd_rn(acc[2 * i], bf16_to_f32(uint16_t(w4[i] & 0xFFFFu)));
          acc[2 * i + 1] = __fadd_rn(acc[2 * i + 1], bf16_to_f32(uint16_t(w4[i] >> 16)));
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
                   cudaStream_t stream) {
  if (T == 0) return MCL4MOE_OK;
  combine_kernel<<<(T + 7) / 8, 256, 0, stream>>>(y, slot_pos, valid, T, k, d, out);
  return cudaGetLastError() == cudaSuccess ? MCL4MOE_OK : MCL4MOE_ERR_CUDA;
}

}  // namespace mcl4
