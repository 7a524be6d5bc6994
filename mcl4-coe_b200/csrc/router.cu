// Router: logits, softmax, top-k, routing statistics and per-chunk stable
// ranks; then the per-expert scan that lays out the expert segments.
//
// Restates the routing part of SparseMoE.forward
// (src/mcl4_coe/backbone.py:787-883, loop branch :913-1004):
//   logits = x.float() @ Wr.float()^T (+ bias)   probs = softmax(logits)
//   w, sel = topk(probs, k)  (w /= max(sum w, 1e-9) when norm_topk_prob)
//   counts, aux = E * sum(counts * mean probs), z = mean(logsumexp^2)
//
// Router product on the tensor cores: x is bf16, so x_k * w_k is exact in
// float32 when w is bf16.  The fp32 router weight is split exactly-enough
// into three bf16 parts (hi = bf16(w), mid = bf16(w - hi), lo = bf16(w - hi -
// mid), 24 mantissa bits in total) and the three products accumulate into
// one fp32 TMEM accumulator (tcgen05 kind::f16, M = 128 tokens, N = E padded
// to 16).  The result agrees with an fp32 SIMT / CPU product to ~1e-6
// relative, like any other fp32 summation order.
//
// Stable permutation: each CTA routes 128 consecutive tokens (a "chunk") and
// ranks the chunk's slots per expert in token order with warp ballots; the
// scan kernel turns per-chunk counts into per-expert prefixes (one CTA per
// expert) and the last CTA to finish lays out the padded expert segments.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "kernels.cuh"

namespace mcl4 {

namespace {

constexpr int kTailThreads = 512;   // 16 warps run the tail of the tensor-core router
constexpr int kTcThreads = 64 + kTailThreads;
constexpr int kLogitsThreads = 1024;  // the tail-only kernel (given logits): 32 warps

struct TailSmem {
  float* logits;   // [128][E + 1] logits (bias included), overwritten with the routed probabilities
  int32_t* sel;    // [128][k] selected experts (-1 for tokens that are not routed)
  float* selp;     // [128][k] their probabilities
  float* lse2;     // [128] lse^2 of routed tokens (0 otherwise)
  float* nval;     // [128] 1 for routed tokens
  uint32_t* bal;   // [4][E] per 32-token group: ballot of the tokens that selected expert e
  float* part;     // [4][E + 2] partial column sums (tails of more than 256 threads)
  int lds;
};

__host__ __device__ inline size_t tail_smem_bytes(int E, int k) {
  return sizeof(float) * kRouteTokens * (E + 1) + 2 * sizeof(int32_t) * kRouteTokens * k +
         2 * sizeof(float) * kRouteTokens + sizeof(uint32_t) * 4 * E + sizeof(float) * 4 * (E + 2) + 64;
}

__device__ inline TailSmem carve_tail(uint8_t* base, int E, int k) {
  TailSmem t;
  t.lds = E + 1;
  t.logits = reinterpret_cast<float*>(base);
  t.sel = reinterpret_cast<int32_t*>(t.logits + kRouteTokens * t.lds);
  t.selp = reinterpret_cast<float*>(t.sel + kRouteTokens * k);
  t.lse2 = t.selp + kRouteTokens * k;
  t.nval = t.lse2 + kRouteTokens;
  t.bal = reinterpret_cast<uint32_t*>(t.nval + kRouteTokens);
  t.part = reinterpret_cast<float*>(t.bal + 4 * E);
  return t;
}

// Softmax / top-k / statistics / stable ranks of one 128-token chunk whose
// logits (bias included) are in ``s.logits``.  Runs on NT threads (256, 512 or
// 1024) with ids ``g`` 0..NT-1; ``sync()`` is a barrier over exactly those threads.
//
// Token-parallel: a group of TPT adjacent threads owns one token and holds VPT of
// its logits each (experts h*VPT .. h*VPT+VPT-1 for member h); a pass covers
// NT/TPT tokens.  Softmax and top-k (largest probability first, ties to the lower
// expert index, as torch.topk on the reference's probabilities) combine across
// the group with xor shuffles.  Per-expert probability sums are column sums over
// the chunk's tokens in token order (in NT/256 consecutive token ranges added in
// order when NT > 256); stable ranks come from one ballot per expert and 32-token
// group.  Semantics: src/mcl4_coe/backbone.py:787-883.
template <int EW, int NT, class Sync>
__device__ void route_chunk_stats(const TailSmem& s, int g, int chunk, int T, int E, int k, const RouteWorkspace& ws,
                                  Sync sync);

template <int EW, int NT, class Sync>
__device__ void route_tail(const TailSmem& s, int g, int chunk, int T, int E, int k, int norm_topk,
                           const uint8_t* __restrict__ valid, int32_t* __restrict__ topk_idx,
                           float* __restrict__ topk_w, float* __restrict__ logits_out, float* __restrict__ sel_mask,
                           const RouteWorkspace& ws, Sync sync) {
  constexpr int kMinTpt = NT / kRouteTokens > 2 ? NT / kRouteTokens : 2;
  constexpr int TPT = EW > kMinTpt ? EW : kMinTpt;  // threads per token
  constexpr int VPT = 32 * EW / TPT;                // logits per thread (E <= 32 * EW)
  constexpr int kPass = NT / TPT;
  static_assert(TPT <= 32 && VPT >= 1 && VPT <= 32 && kRouteTokens % kPass == 0, "tail shape");
  const int h = g % TPT;
  const int t0 = chunk * kRouteTokens;
  for (int pass = 0; pass < kRouteTokens / kPass; ++pass) {
    const int tok = pass * kPass + g / TPT;
    const int t = t0 + tok;
    const bool in_range = t < T;
    const bool routed = in_range && (valid == nullptr || valid[t] != 0);
    float v[VPT];
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int e = h * VPT + i;
      v[i] = (e < E && in_range) ? s.logits[tok * s.lds + e] : -INFINITY;
      if (logits_out != nullptr && e < E && in_range) logits_out[int64_t(t) * E + e] = v[i];
    }
    float m = -INFINITY;
#pragma unroll
    for (int i = 0; i < VPT; ++i) m = fmaxf(m, v[i]);
#pragma unroll
    for (int o = 1; o < TPT; o <<= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (!in_range) m = 0.f;  // all -inf: keep the arithmetic finite, nothing is written
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      v[i] = (h * VPT + i < E && in_range) ? expf(__fsub_rn(v[i], m)) : 0.f;
      sum = __fadd_rn(sum, v[i]);
    }
#pragma unroll
    for (int o = 1; o < TPT; o <<= 1) sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, o));
    const float inv_s = in_range ? __frcp_rn(sum) : 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      v[i] = __fmul_rn(v[i], inv_s);
      const int e = h * VPT + i;
      if (e < E) s.logits[tok * s.lds + e] = routed ? v[i] : 0.f;  // column sums below
    }
    if (h == 0) {
      const float lse = routed ? __fadd_rn(m, logf(sum)) : 0.f;
      s.lse2[tok] = __fmul_rn(lse, lse);
      s.nval[tok] = routed ? 1.f : 0.f;
    }
    // top-k over the group: each member offers its best remaining candidate
    uint32_t taken = 0;
    float total = 0.f;
    for (int j = 0; j < k; ++j) {
      float bp = -1.f;
      int bi = 0;
#pragma unroll
      for (int i = 0; i < VPT; ++i)
        if (h * VPT + i < E && !((taken >> i) & 1u) && v[i] > bp) {
          bp = v[i];
          bi = i;
        }
      const uint32_t be = uint32_t(h * VPT + bi);
      unsigned long long best =
          bp >= 0.f ? (static_cast<unsigned long long>(__float_as_uint(bp)) << 32) | (0xFFFFFFFFu - be) : 0ull;
#pragma unroll
      for (int o = 1; o < TPT; o <<= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
        best = other > best ? other : best;
      }
      const int e_star = int(0xFFFFFFFFu - uint32_t(best & 0xFFFFFFFFull));
      const float p_star = __uint_as_float(uint32_t(best >> 32));
      if (e_star / VPT == h) taken |= 1u << (e_star % VPT);
      total = __fadd_rn(total, p_star);
      if (j % TPT == h) {
        s.sel[tok * k + j] = routed ? e_star : -1;
        s.selp[tok * k + j] = p_star;
      }
    }
    if (in_range) {
      for (int j = h; j < k; j += TPT) {
        const float w = norm_topk ? __fdiv_rn(s.selp[tok * k + j], fmaxf(total, 1e-9f)) : s.selp[tok * k + j];
        topk_idx[int64_t(t) * k + j] = routed ? s.sel[tok * k + j] : -1;
        topk_w[int64_t(t) * k + j] = routed ? w : 0.f;
      }
      if (sel_mask != nullptr)
#pragma unroll
        for (int i = 0; i < VPT; ++i) {
          const int e = h * VPT + i;
          if (e < E) sel_mask[int64_t(t) * E + e] = (routed && ((taken >> i) & 1u)) ? 1.f : 0.f;
        }
    }
  }
  sync();
  route_chunk_stats<EW, NT>(s, g, chunk, T, E, k, ws, sync);
}

// The chunk's statistics and stable ranks from its per-token results in shared memory
// (routed probabilities in ``s.logits``, selections in ``s.sel``, ``s.lse2``, ``s.nval``):
// per-expert probability sums and the lse^2 / routed-token sums (column sums in token
// order, in NT/256 consecutive token ranges added in order when NT > 256), per-expert
// chunk counts and each slot's rank among the chunk's slots of its expert.
template <int EW, int NT, class Sync>
__device__ void route_chunk_stats(const TailSmem& s, int g, int chunk, int T, int E, int k, const RouteWorkspace& ws,
                                  Sync sync) {
  const int t0 = chunk * kRouteTokens;
  // per-chunk statistics: column sums in token order (P consecutive token ranges)
  constexpr int P = NT / 256 > 0 ? NT / 256 : 1;
  constexpr int kRange = kRouteTokens / P;
  for (int idx = g; idx < (E + 2) * P; idx += NT) {
    const int c = idx % (E + 2), part = idx / (E + 2);
    const float* col = c < E ? s.logits + c : (c == E ? s.lse2 : s.nval);
    const int stride = c < E ? s.lds : 1;
    float acc = 0.f;
    for (int tok = part * kRange; tok < (part + 1) * kRange; ++tok) acc = __fadd_rn(acc, col[tok * stride]);
    if (P == 1) {
      if (c < E) ws.part_probs[int64_t(chunk) * E + c] = acc;
      else ws.part_misc[int64_t(chunk) * 2 + (c - E)] = acc;
    } else {
      s.part[part * (E + 2) + c] = acc;
    }
  }

  // stable ranks: warp w owns the 32 tokens of group w % 4 (lane = token) and the
  // experts e with e % (NT / 128) == w / 4; one ballot per expert
  const int lane = g & 31, warp = g >> 5;
  {
    constexpr int kSlices = NT / 128;
    const int grp = warp & 3, slice = warp >> 2;
    const int tok = grp * 32 + lane;
    uint32_t mw[EW];
#pragma unroll
    for (int i = 0; i < EW; ++i) mw[i] = 0;
    for (int j = 0; j < k; ++j) {
      const int e = s.sel[tok * k + j];
#pragma unroll
      for (int i = 0; i < EW; ++i)
        if (e >= 0 && (e >> 5) == i) mw[i] |= 1u << (e & 31);
    }
    for (int e = slice; e < E; e += kSlices) {
      uint32_t word = 0;
#pragma unroll
      for (int i = 0; i < EW; ++i)
        if ((e >> 5) == i) word = mw[i];
      const uint32_t bal = __ballot_sync(0xffffffffu, (word >> (e & 31)) & 1u);
      if (lane == 0) s.bal[grp * E + e] = bal;
    }
  }
  sync();
  if (P > 1) {
    for (int c = g; c < E + 2; c += NT) {
      float acc = s.part[c];
#pragma unroll
      for (int part = 1; part < P; ++part) acc = __fadd_rn(acc, s.part[part * (E + 2) + c]);
      if (c < E) ws.part_probs[int64_t(chunk) * E + c] = acc;
      else ws.part_misc[int64_t(chunk) * 2 + (c - E)] = acc;
    }
  }
  for (int e = g; e < E; e += NT)
    ws.chunk_excl[int64_t(chunk) * E + e] =
        __popc(s.bal[e]) + __popc(s.bal[E + e]) + __popc(s.bal[2 * E + e]) + __popc(s.bal[3 * E + e]);
  for (int i = g; i < kRouteTokens * k; i += NT) {
    const int tok = i / k;
    if (t0 + tok >= T) continue;
    const int e = s.sel[i];
    int r = 0;
    if (e >= 0) {
      const int grp = tok >> 5;
      r = __popc(s.bal[grp * E + e] & ((1u << (tok & 31)) - 1u));
      for (int gi = 0; gi < grp; ++gi) r += __popc(s.bal[gi * E + e]);
    }
    ws.local_rank[int64_t(t0) * k + i] = r;
  }
}

struct BlockSync {
  __device__ void operator()() const { __syncthreads(); }
};
struct TailBarrier {  // named barrier 1 over the tail threads of the tensor-core router
  __device__ void operator()() const { asm volatile("bar.sync 1, %0;" ::"n"(kTailThreads) : "memory"); }
};

}  // namespace

// ---------------------------------------------------------------- weight split

// Wr fp32 [E, d] -> three bf16 parts [3][E_pad][d]; rows E..E_pad-1 are zero.
__global__ void __launch_bounds__(256) router_split_kernel(const float* __restrict__ wr, int E, int E_pad, int d,
                                                           uint16_t* __restrict__ wsplit) {
  const int64_t n = int64_t(E_pad) * d;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
    const int e = int(i / d);
    const float w = e < E ? wr[i] : 0.f;
    const uint16_t hi = f32_to_bf16(w);
    const float r1 = __fsub_rn(w, bf16_to_f32(hi));
    const uint16_t mid = f32_to_bf16(r1);
    const float r2 = __fsub_rn(r1, bf16_to_f32(mid));
    wsplit[i] = hi;
    wsplit[n + i] = mid;
    wsplit[2 * n + i] = f32_to_bf16(r2);
  }
}

// ---------------------------------------------------------------- small-batch router

// fp32 logits of a small batch on the CUDA cores: CTA (token block of 8, expert
// block of 8); warp w owns expert e0 + w, lane l accumulates the 4-element groups
// 4l, 4l + 128, ... of d for the 8 tokens with fp32 fma (16-byte weight loads, eight
// groups in flight), then a fixed xor tree sums the lanes (deterministic).
// logits[t, e] = sum_k x[t, k] * Wr[e, k] (+ bias[e]).
__global__ void __launch_bounds__(256) router_gemv_kernel(const uint16_t* __restrict__ x,
                                                          const float* __restrict__ wr,
                                                          const float* __restrict__ bias, int T, int d, int E,
                                                          float* __restrict__ logits) {
  extern __shared__ uint16_t xs[];  // [8][d] bf16
  pdl_wait();  // x (and the router weight) are complete (PDL launch)
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int t0 = blockIdx.x * 8, e = blockIdx.y * 8 + warp;
  const int nt = min(8, T - t0);
  // the 8 token rows into shared memory in 16-byte chunks, 8 loads in flight per thread
  const int nchunk = 8 * d / 8;
  for (int base = threadIdx.x; base < nchunk; base += 8 * 256) {
    uint4 v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = base + u * 256;
      const int r = i / (d / 8), c = i - r * (d / 8);
      v[u] = make_uint4(0, 0, 0, 0);
      if (i < nchunk && r < nt) v[u] = __ldg(reinterpret_cast<const uint4*>(x + int64_t(t0 + r) * d) + c);
    }
#pragma unroll
    for (int u = 0; u < 8; ++u)
      if (base + u * 256 < nchunk) reinterpret_cast<uint4*>(xs)[base + u * 256] = v[u];
  }
  __syncthreads();
  pdl_trigger();
  if (e >= E) return;
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  const float4* wrow = reinterpret_cast<const float4*>(wr + int64_t(e) * d);
  const int groups = d / 4;  // d % 64 == 0
#pragma unroll 8
  for (int gq = lane; gq < groups; gq += 32) {
    const float4 wv = __ldg(wrow + gq);
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      const uint2 xv = *reinterpret_cast<const uint2*>(xs + r * d + 4 * gq);
      acc[r] = __fmaf_rn(bf16x2_lo(xv.x), wv.x, acc[r]);
      acc[r] = __fmaf_rn(bf16x2_hi(xv.x), wv.y, acc[r]);
      acc[r] = __fmaf_rn(bf16x2_lo(xv.y), wv.z, acc[r]);
      acc[r] = __fmaf_rn(bf16x2_hi(xv.y), wv.w, acc[r]);
    }
  }
#pragma unroll
  for (int r = 0; r < 8; ++r) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc[r] = __fadd_rn(acc[r], __shfl_xor_sync(0xffffffffu, acc[r], o));
  }
  if (lane < nt) {
    float v = acc[0];
#pragma unroll
    for (int r = 1; r < 8; ++r)
      if (lane == r) v = acc[r];
    logits[int64_t(t0 + lane) * E + e] = bias ? __fadd_rn(v, bias[e]) : v;
  }
}

// ---------------------------------------------------------------- tensor-core router

struct RouterTcArgs {
  const float* bias;
  const uint8_t* valid;
  int T, d, E, E_pad, k, norm_topk, stages;
  int fused;  // 3 * E_pad <= 256: the three weight parts form one N = 3 * E_pad operand
  uint32_t tmem_cols;
  int32_t* topk_idx;
  float* topk_w;
  float* logits_out;
  float* sel_mask;
  int32_t* err;
  // one chunk (T <= 128) on the logits path: the tail kernel also lays out the expert
  // segments and finalises the statistics (route_scan_kernel's work), so no scan launch
  int fuse_scan;
  int32_t* counts_out;
  float* stats;
  int32_t* offs_out;
};

template <int EW>
__global__ void __launch_bounds__(kTcThreads) router_tc_kernel(const __grid_constant__ CUtensorMap tmap_x,
                                                               const __grid_constant__ CUtensorMap tmap_w,
                                                               RouterTcArgs a, RouteWorkspace ws) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base - raw_addr);
  const uint32_t a_bytes = kRouteTokens * 128;            // 128 tokens x 64 bf16
  const uint32_t b_part = uint32_t(a.E_pad) * 128;        // E_pad rows x 64 bf16
  const uint32_t stage_bytes = a_bytes + 3 * b_part;
  const uint32_t region = uint32_t(a.stages) * stage_bytes;
  const size_t tail_bytes = tail_smem_bytes(a.E, a.k);
  const uint32_t bar_base = base + uint32_t(((region > tail_bytes ? region : tail_bytes) + 15) & ~size_t(15));
  auto full_bar = [&](int s) { return bar_base + 8u * s; };
  auto empty_bar = [&](int s) { return bar_base + 8u * (4 + s); };
  const uint32_t tfull_bar = bar_base + 64;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + (bar_base - base) + 72);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int chunk = blockIdx.x;
  const int t0 = chunk * kRouteTokens;
  if (tid == 0) {
    for (int s = 0; s < a.stages; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    mbar_init(tfull_bar, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), a.tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int kblocks = a.d / 64;
  pdl_wait();  // the router-weight split (previous kernel) has finished
  if (chunk == 0 && tid == 0) *ws.done = 0u;  // the scan kernel runs after this one

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&tmap_x);
      prefetch_tmap(&tmap_w);
      int stage = 0;
      uint32_t phase = 0;
      for (int kb = 0; kb < kblocks; ++kb) {
        if (!mbar_wait(empty_bar(stage), phase ^ 1u, a.err, 111)) break;
        const uint32_t st = base + stage * stage_bytes;
        mbar_arrive_expect_tx(full_bar(stage), stage_bytes);
        tma_load_2d(st, &tmap_x, kb * 64, t0, full_bar(stage));
        if (a.fused) {
          tma_load_2d(st + a_bytes, &tmap_w, kb * 64, 0, full_bar(stage));  // the three parts, stacked
        } else {
#pragma unroll
          for (int p = 0; p < 3; ++p)
            tma_load_2d(st + a_bytes + p * b_part, &tmap_w, kb * 64, p * a.E_pad, full_bar(stage));
        }
        if (++stage == a.stages) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      // kind::f16, bf16 x bf16 -> fp32, K-major A and B, M = 128, N = E_pad (or 3 * E_pad
      // when fused: one MMA per K step writes the three parts' products to columns
      // [0, E_pad), [E_pad, 2 E_pad), [2 E_pad, 3 E_pad))
      const uint32_t n_mma = a.fused ? 3u * uint32_t(a.E_pad) : uint32_t(a.E_pad);
      const uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((n_mma >> 3) << 17) | ((128u >> 4) << 24);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int kb = 0; kb < kblocks; ++kb) {
        if (!mbar_wait(full_bar(stage), phase, a.err, 211)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t st = base + stage * stage_bytes;
        if (a.fused) {
#pragma unroll
          for (int ks = 0; ks < 4; ++ks)
            tc_mma_f16(tmem_base, smem_desc(st + 32 * ks, 16, 1024, 2), smem_desc(st + a_bytes + 32 * ks, 16, 1024, 2),
                       idesc, (kb | ks) != 0 ? 1u : 0u);
        } else {
#pragma unroll
          for (int ks = 0; ks < 4; ++ks)
#pragma unroll
            for (int p = 0; p < 3; ++p)
              tc_mma_f16(tmem_base, smem_desc(st + 32 * ks, 16, 1024, 2),
                         smem_desc(st + a_bytes + p * b_part + 32 * ks, 16, 1024, 2), idesc,
                         (kb | ks | p) != 0 ? 1u : 0u);
        }
        tc_commit(empty_bar(stage));
        if (++stage == a.stages) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (ok) tc_commit(tfull_bar);
    }
    __syncwarp();
  } else {
    // tail warps: TMEM logits -> shared memory (+ bias), then softmax / top-k / ranks
    const int g = tid - 64;
    const int q = warp & 3, grp = (warp - 2) >> 2;  // TMEM lane quarter; column group
    const TailSmem s = carve_tail(smem, a.E, a.k);
    const bool ok = mbar_wait(tfull_bar, 0, a.err, 311);
    tc_fence_after();
    const int row = q * 32 + lane;
    const uint32_t lane_addr = tmem_base + (uint32_t(q * 32) << 16);
    auto ld8 = [&](uint32_t col, uint32_t (&v)[8]) {
      asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                   : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
                   : "r"(lane_addr + col)
                   : "memory");
    };
    for (int c0 = grp * 8; c0 < a.E_pad; c0 += (kTailThreads / 128) * 8) {  // E_pad: a multiple of 16
      uint32_t v[8], vm[8], vl[8];
      if (ok) {
        ld8(c0, v);
        if (a.fused) {
          ld8(c0 + a.E_pad, vm);
          ld8(c0 + 2 * a.E_pad, vl);
        }
        tmem_wait_ld();
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int e = c0 + j;
        if (e < a.E) {
          float lv = ok ? __uint_as_float(v[j]) : 0.f;
          // fused: hi + (mid + lo), the two small parts first
          if (ok && a.fused) lv = __fadd_rn(lv, __fadd_rn(__uint_as_float(vm[j]), __uint_as_float(vl[j])));
          s.logits[row * s.lds + e] = a.bias ? __fadd_rn(lv, a.bias[e]) : lv;
        }
      }
    }
    tc_fence_before();
    TailBarrier()();
    pdl_trigger();  // the scan kernel may launch; it waits for this grid's writes
    route_tail<EW, kTailThreads>(s, g, chunk, a.T, a.E, a.k, a.norm_topk, a.valid, a.topk_idx, a.topk_w,
                                 a.logits_out, a.sel_mask,
                   ws, TailBarrier());
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, a.tmem_cols);
  }
}

// route_scan_kernel's result for a single chunk, by the chunk's own CTA after its
// tail: the chunk counts are the expert totals (exclusive prefix 0), the chunk's
// probability and statistic sums are the totals.  Same arithmetic as the scan.
__device__ void finish_single_chunk(int E, int k, const RouteWorkspace& ws, int32_t* counts_out, float* stats,
                                    int32_t* offs_out) {
  __shared__ int32_t itmp[64];
  __shared__ float ftmp[32];
  const int tid = threadIdx.x;
  int32_t cnt = 0;
  float ps = 0.f;
  if (tid < E) {
    cnt = ws.chunk_excl[tid];
    ps = ws.part_probs[tid];
    ws.chunk_excl[tid] = 0;
    ws.counts[tid] = cnt;
    ws.probs_sum[tid] = ps;
  }
  const float lse2 = ws.part_misc[0], n = ws.part_misc[1];
  int32_t ignore;
  const int32_t ustart = block_exclusive_scan(cnt, itmp, ignore);
  const int32_t padded = (cnt + kSegRows - 1) / kSegRows * kSegRows;
  const int32_t pstart = block_exclusive_scan(padded, itmp, ignore);
  float term = 0.f;
  if (tid < E) {
    ws.offs_start[tid] = ustart;
    ws.pad_start[tid] = pstart;
    if (tid == E - 1) ws.pad_start[E] = pstart + padded;
    if (offs_out) offs_out[tid] = ustart + cnt;
    if (counts_out) counts_out[tid] = cnt;
    if (stats) {
      const float cf = n > 0.f ? __fdiv_rn(float(cnt), n * float(k)) : 0.f;
      stats[3 + tid] = cf;
      term = n > 0.f ? __fmul_rn(cf, __fdiv_rn(ps, n)) : 0.f;
    }
  }
  const float aux = block_sum(term, ftmp);
  if (tid == 0 && stats) {
    stats[0] = n > 0.f ? __fmul_rn(float(E), aux) : 0.f;
    stats[1] = n > 0.f ? __fdiv_rn(lse2, n) : 0.f;
    stats[2] = n;
  }
}

// Router tail on given logits (parity checks against recorded reference logits).
template <int EW>
__global__ void __launch_bounds__(kLogitsThreads) router_logits_kernel(const float* __restrict__ logits_in,
                                                                     const float* __restrict__ bias, RouterTcArgs a,
                                                                     RouteWorkspace ws) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const TailSmem s = carve_tail(smem_raw, a.E, a.k);
  const int chunk = blockIdx.x;
  const int t0 = chunk * kRouteTokens;
  pdl_wait();     // the logits are complete (PDL launch)
  pdl_trigger();  // the scan may launch; it waits for this grid's writes
  if (chunk == 0 && threadIdx.x == 0) *ws.done = 0u;
  // the chunk's logits into shared memory, 16 loads in flight per thread (a loop that
  // waits on each load before the next would pay one memory latency per element)
  constexpr int kBatch = 16;
  const int n = kRouteTokens * a.E;
  for (int base = threadIdx.x; base < n; base += kBatch * kLogitsThreads) {
    float lv[kBatch];
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const int i = base + u * kLogitsThreads;
      const int tok = i / a.E;
      lv[u] = (i < n && t0 + tok < a.T) ? __ldg(logits_in + int64_t(t0) * a.E + i) : 0.f;
    }
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const int i = base + u * kLogitsThreads;
      if (i < n) {
        const int tok = i / a.E, e = i - tok * a.E;
        s.logits[tok * s.lds + e] = bias ? __fadd_rn(lv[u], __ldg(bias + e)) : lv[u];
      }
    }
  }
  __syncthreads();
  route_tail<EW, kLogitsThreads>(s, threadIdx.x, chunk, a.T, a.E, a.k, a.norm_topk, a.valid, a.topk_idx, a.topk_w,
                                 a.logits_out,
                 a.sel_mask, ws, BlockSync());
  if (a.fuse_scan) {
    __syncthreads();  // the tail's chunk counts and sums (global memory of this block) are complete
    finish_single_chunk(a.E, a.k, ws, a.counts_out, a.stats, a.offs_out);
  }
}

// One-chunk batches (T <= 128) from x in one launch.  CTA (b, c) computes the fp32
// logits of tokens [8b, 8b + 8) and experts [8c, 8c + 8) exactly as the small-batch
// GEMV does (warp w owns expert 8c + w); the last CTA of token block b to finish runs
// one warp per token: softmax / top-k, the token's outputs and its per-token results
// (routed probabilities into the logits scratch, lse^2 and the routed flag); the last
// token block to finish gathers the chunk's results and computes its statistics, ranks
// and expert segments, as the tail-only kernel does for one chunk.  Completion
// counters (small_cnt: one per token block, then one for the chunk) are zeroed before
// the launch.  Semantics: src/mcl4_coe/backbone.py:787-883.
constexpr int kSmallTokPerCta = 8;

template <int EW>
__global__ void __launch_bounds__(256) router_small_kernel(const uint16_t* __restrict__ x,
                                                           const float* __restrict__ wr,
                                                           const float* __restrict__ bias, RouterTcArgs a,
                                                           RouteWorkspace ws) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const int d = a.d, E = a.E, k = a.k, T = a.T;
  uint16_t* xs = reinterpret_cast<uint16_t*>(smem_raw);  // [8][d] bf16
  float* lg = reinterpret_cast<float*>(smem_raw);         // [8][E] logits (after the GEMV part)
  __shared__ bool is_last;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int t0 = blockIdx.x * kSmallTokPerCta;
  uint32_t* cnt = reinterpret_cast<uint32_t*>(ws.small_tok + 2 * kRouteTokens);
  const int nt = min(kSmallTokPerCta, T - t0);
  pdl_wait();  // x and the router weight are complete (PDL launch)
  {
    const int nchunk = 8 * d / 8;  // 16-byte chunks of the 8 rows, 8 loads in flight per thread
    for (int base = threadIdx.x; base < nchunk; base += 8 * 256) {
      uint4 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int i = base + u * 256;
        const int r = i / (d / 8), c = i - r * (d / 8);
        v[u] = make_uint4(0, 0, 0, 0);
        if (i < nchunk && r < nt) v[u] = __ldg(reinterpret_cast<const uint4*>(x + int64_t(t0 + r) * d) + c);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (base + u * 256 < nchunk) reinterpret_cast<uint4*>(xs)[base + u * 256] = v[u];
    }
  }
  __syncthreads();
  pdl_trigger();
  // logits: the GEMV's per-lane fp32 fma order and xor tree, so the values are the GEMV's
  for (int e = blockIdx.y * 8 + warp; e < min(E, int(blockIdx.y) * 8 + 8); e += 8) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    const float4* wrow = reinterpret_cast<const float4*>(wr + int64_t(e) * d);
    const int groups = d / 4;
#pragma unroll 8
    for (int gq = lane; gq < groups; gq += 32) {
      const float4 wv = __ldg(wrow + gq);
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        const uint2 xv = *reinterpret_cast<const uint2*>(xs + r * d + 4 * gq);
        acc[r] = __fmaf_rn(bf16x2_lo(xv.x), wv.x, acc[r]);
        acc[r] = __fmaf_rn(bf16x2_hi(xv.x), wv.y, acc[r]);
        acc[r] = __fmaf_rn(bf16x2_lo(xv.y), wv.z, acc[r]);
        acc[r] = __fmaf_rn(bf16x2_hi(xv.y), wv.w, acc[r]);
      }
    }
#pragma unroll
    for (int r = 0; r < 8; ++r) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc[r] = __fadd_rn(acc[r], __shfl_xor_sync(0xffffffffu, acc[r], o));
    }
    if (lane < nt) {
      float v = acc[0];
#pragma unroll
      for (int r = 1; r < 8; ++r)
        if (lane == r) v = acc[r];
      ws.small_logits[int64_t(t0 + lane) * E + e] = bias ? __fadd_rn(v, __ldg(bias + e)) : v;
    }
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) is_last = atomicAdd(cnt + blockIdx.x, 1u) == gridDim.y - 1;
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  // the token block's logits (all experts) from the other CTAs of the block
  for (int i = threadIdx.x; i < nt * E; i += 256) lg[i] = __ldcg(ws.small_logits + int64_t(t0) * E + i);
  __syncthreads();
  // one warp per token: lane l holds experts l + 32 i
  if (warp < nt) {
    const int t = t0 + warp;
    const bool routed = a.valid == nullptr || a.valid[t] != 0;
    float v[EW];
#pragma unroll
    for (int i = 0; i < EW; ++i) {
      const int e = lane + 32 * i;
      v[i] = e < E ? lg[warp * E + e] : -INFINITY;
      if (a.logits_out != nullptr && e < E) a.logits_out[int64_t(t) * E + e] = v[i];
    }
    float m = -INFINITY;
#pragma unroll
    for (int i = 0; i < EW; ++i) m = fmaxf(m, v[i]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < EW; ++i) {
      v[i] = lane + 32 * i < E ? expf(__fsub_rn(v[i], m)) : 0.f;
      sum = __fadd_rn(sum, v[i]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, o));
    const float inv_s = __frcp_rn(sum);
#pragma unroll
    for (int i = 0; i < EW; ++i) {
      v[i] = __fmul_rn(v[i], inv_s);
      const int e = lane + 32 * i;
      if (e < E) ws.small_logits[int64_t(t) * E + e] = routed ? v[i] : 0.f;  // column sums of the last CTA
    }
    if (lane == 0) {
      const float lse = routed ? __fadd_rn(m, logf(sum)) : 0.f;
      ws.small_tok[t] = __fmul_rn(lse, lse);
      ws.small_tok[kRouteTokens + t] = routed ? 1.f : 0.f;
    }
    // top-k: largest probability first, ties to the lower expert index
    uint32_t taken = 0;
    float total = 0.f;
    int my_e = -1;
    float my_p = 0.f;
    for (int j = 0; j < k; ++j) {
      float bp = -1.f;
      int bi = 0;
#pragma unroll
      for (int i = 0; i < EW; ++i)
        if (lane + 32 * i < E && !((taken >> i) & 1u) && v[i] > bp) {
          bp = v[i];
          bi = i;
        }
      const uint32_t be = uint32_t(lane + 32 * bi);
      unsigned long long best =
          bp >= 0.f ? (static_cast<unsigned long long>(__float_as_uint(bp)) << 32) | (0xFFFFFFFFu - be) : 0ull;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
        best = other > best ? other : best;
      }
      const int e_star = int(0xFFFFFFFFu - uint32_t(best & 0xFFFFFFFFull));
      const float p_star = __uint_as_float(uint32_t(best >> 32));
      if ((e_star & 31) == lane) taken |= 1u << (e_star >> 5);
      total = __fadd_rn(total, p_star);
      if (lane == j) {
        my_e = e_star;
        my_p = p_star;
      }
    }
    if (lane < k) {
      const float w = a.norm_topk ? __fdiv_rn(my_p, fmaxf(total, 1e-9f)) : my_p;
      a.topk_idx[int64_t(t) * k + lane] = routed ? my_e : -1;
      a.topk_w[int64_t(t) * k + lane] = routed ? w : 0.f;
    }
    if (a.sel_mask != nullptr)
#pragma unroll
      for (int i = 0; i < EW; ++i) {
        const int e = lane + 32 * i;
        if (e < E) a.sel_mask[int64_t(t) * E + e] = (routed && ((taken >> i) & 1u)) ? 1.f : 0.f;
      }
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) is_last = atomicAdd(cnt + 16, 1u) == gridDim.x - 1;
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  // the last token block: the chunk's per-token results into the tail layout (tokens >= T empty)
  const TailSmem s = carve_tail(smem_raw, E, k);
  for (int i = threadIdx.x; i < kRouteTokens * E; i += 256) {
    const int tok = i / E, e = i - tok * E;
    s.logits[tok * s.lds + e] = tok < T ? __ldcg(ws.small_logits + i) : 0.f;
  }
  for (int i = threadIdx.x; i < kRouteTokens * k; i += 256) s.sel[i] = i < T * k ? __ldcg(a.topk_idx + i) : -1;
  for (int i = threadIdx.x; i < kRouteTokens; i += 256) {
    s.lse2[i] = i < T ? __ldcg(ws.small_tok + i) : 0.f;
    s.nval[i] = i < T ? __ldcg(ws.small_tok + kRouteTokens + i) : 0.f;
  }
  __syncthreads();
  route_chunk_stats<EW, 256>(s, threadIdx.x, 0, T, E, k, ws, BlockSync());
  __syncthreads();  // the chunk counts and sums (global memory of this block) are complete
  finish_single_chunk(E, k, ws, a.counts_out, a.stats, a.offs_out);
}

inline size_t small_router_smem(int d, int E, int k) {
  const size_t xrows = sizeof(uint16_t) * 8 * size_t(d), logits = sizeof(float) * 8 * size_t(E);
  const size_t own = xrows > logits ? xrows : logits;
  const size_t tail = tail_smem_bytes(E, k);
  return own > tail ? own : tail;
}

// ---------------------------------------------------------------- scan


// One CTA per expert: exclusive prefix of the expert's per-chunk slot counts
// and its probability sum.  The last CTA to finish (counted with an atomic
// after a memory fence; no CTA waits on another) lays out the expert segments
// and finalises the statistics.
__global__ void __launch_bounds__(256) route_scan_kernel(int C, int E, int k, RouteWorkspace ws, int32_t* counts_out,
                                                         float* stats, int32_t* offs_out) {
  __shared__ int32_t itmp[64];
  __shared__ float ftmp[32];
  __shared__ bool is_last;
  pdl_wait();
  pdl_trigger();
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

  float l2 = 0.f, nv = 0.f;
  for (int c = c0; c < c1; ++c) {
    l2 = __fadd_rn(l2, ws.part_misc[2 * c]);
    nv = __fadd_rn(nv, ws.part_misc[2 * c + 1]);
  }
  const float lse2 = block_sum(l2, ftmp);
  const float n = block_sum(nv, ftmp);
  // each thread takes one expert (E <= 256): counts -> segment starts by block scans
  const int32_t cnt = tid < E ? __ldcg(ws.counts + tid) : 0;
  int32_t ignore;
  const int32_t ustart = block_exclusive_scan(cnt, itmp, ignore);
  const int32_t pstart = block_exclusive_scan((cnt + kSegRows - 1) / kSegRows * kSegRows, itmp, ignore);
  float term = 0.f;
  if (tid < E) {
    ws.offs_start[tid] = ustart;
    ws.pad_start[tid] = pstart;
    if (tid == E - 1) ws.pad_start[E] = pstart + (cnt + kSegRows - 1) / kSegRows * kSegRows;
    if (offs_out) offs_out[tid] = ustart + cnt;
    if (counts_out) counts_out[tid] = cnt;
    if (stats) {
      const float cf = n > 0.f ? __fdiv_rn(float(cnt), n * float(k)) : 0.f;
      stats[3 + tid] = cf;
      term = n > 0.f ? __fmul_rn(cf, __fdiv_rn(__ldcg(ws.probs_sum + tid), n)) : 0.f;
    }
  }
  const float aux = block_sum(term, ftmp);
  if (tid == 0 && stats) {
    stats[0] = n > 0.f ? __fmul_rn(float(E), aux) : 0.f;
    stats[1] = n > 0.f ? __fdiv_rn(lse2, n) : 0.f;
    stats[2] = n;
  }
}

// ---------------------------------------------------------------- precomputed routing

// Chunk ranks of caller-supplied expert ids (one CTA per 128-token chunk, the
// router's chunking): slot (t, j) gets its rank among the chunk's slots of the
// same expert in flattened order t*k + j, the order of the reference's stable
// argsort of the selected experts (src/mcl4_coe/backbone.py:895-897).  Slots
// of masked tokens and ids outside [0, E) get rank -1 and are not routed.
// Each warp ranks 16 tokens (match_any per 32 slots), then the warps' counts
// are scanned per expert.  Writes the chunk's per-expert counts (the router's
// chunk counts) and zero probability sums; part_misc holds the chunk's routed
// token count for the scan's statistics.
__global__ void __launch_bounds__(256) route_ranks_kernel(const int32_t* __restrict__ topk_idx,
                                                          const uint8_t* __restrict__ valid, int T, int E, int k,
                                                          RouteWorkspace ws) {
  __shared__ int32_t cnt[8 * kMaxExperts];
  __shared__ int32_t n_tok;
  pdl_wait();
  pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = blockIdx.x;
  for (int i = threadIdx.x; i < 8 * E; i += blockDim.x) cnt[i] = 0;
  if (threadIdx.x == 0) n_tok = 0;
  if (c == 0 && threadIdx.x == 0) *ws.done = 0u;  // finished-expert counter of the scan
  __syncthreads();
  const int t0 = c * kRouteTokens + warp * 16;
  const int t1 = min(T, t0 + 16);
  const int64_t s0 = int64_t(t0) * k, s1 = t1 > t0 ? int64_t(t1) * k : s0;
  int32_t* my = cnt + warp * E;
  for (int64_t base = s0; base < s1; base += 32) {
    const int64_t sl = base + lane;
    int e = -1;
    if (sl < s1) {
      const int t = int(sl / k);
      const int v = topk_idx[sl];
      if ((valid == nullptr || valid[t] != 0) && v >= 0 && v < E) e = v;
    }
    const uint32_t peers = __match_any_sync(0xffffffffu, e);
    const int before = __popc(peers & ((1u << lane) - 1u));
    const int r = e >= 0 ? my[e] + before : -1;
    __syncwarp();
    if (e >= 0 && before == 0) my[e] += __popc(peers);
    __syncwarp();
    if (sl < s1) ws.local_rank[sl] = r;
  }
  if (lane < 16 && t0 + lane < t1 && (valid == nullptr || valid[t0 + lane] != 0)) atomicAdd(&n_tok, 1);
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int run = 0;
    for (int w = 0; w < 8; ++w) {
      const int v = cnt[w * E + e];
      cnt[w * E + e] = run;
      run += v;
    }
    ws.chunk_excl[int64_t(c) * E + e] = run;
    ws.part_probs[int64_t(c) * E + e] = 0.f;
  }
  if (threadIdx.x == 0) {
    ws.part_misc[2 * c] = 0.f;
    ws.part_misc[2 * c + 1] = float(n_tok);
  }
  __syncthreads();
  for (int64_t base = s0; base < s1; base += 32) {
    const int64_t sl = base + lane;
    if (sl >= s1) continue;
    const int t = int(sl / k);
    const int v = topk_idx[sl];
    if ((valid == nullptr || valid[t] != 0) && v >= 0 && v < E) ws.local_rank[sl] += my[v];
  }
}

// ---------------------------------------------------------------- host side

namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 2-D map over a bf16 [rows, cols] matrix, box 64 x box_rows, 128-byte swizzle; rows
// outside the matrix read as zero.
bool make_tmap_bf16(CUtensorMap* m, const void* ptr, uint64_t cols, uint64_t rows, uint32_t box_rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * 2};
  cuuint32_t box[2] = {64, box_rows};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int EW>
int launch_router_t(const uint16_t* x, const float* wr, const float* bias, const float* logits_in, RouterTcArgs a,
                    const RouteWorkspace& ws, cudaStream_t stream) {
  const int C = (a.T + kRouteTokens - 1) / kRouteTokens;
  if (logits_in != nullptr) {
    const size_t smem = tail_smem_bytes(a.E, a.k);
    static std::atomic<uint64_t> configured{0};
    if (!raise_smem_limit(router_logits_kernel<EW>, 200 * 1024, configured)) return MCL4MOE_ERR_CUDA;
    return launch_pdl(router_logits_kernel<EW>, dim3(C), dim3(kLogitsThreads), smem, stream, logits_in,
                      static_cast<const float*>(nullptr), a, ws) == cudaSuccess  // final logits
               ? MCL4MOE_OK
               : MCL4MOE_ERR_CUDA;
  }
  // split the router weight into three bf16 parts, then the tensor-core router
  const int64_t n = int64_t(a.E_pad) * a.d;
  int blocks = int((n + 255) / 256);
  if (blocks > 1024) blocks = 1024;
  router_split_kernel<<<blocks, 256, 0, stream>>>(wr, a.E, a.E_pad, a.d, ws.wsplit);
  CUtensorMap tx, tw;
  if (!make_tmap_bf16(&tx, x, uint64_t(a.d), uint64_t(a.T), kRouteTokens)) return MCL4MOE_ERR_CUDA;
  a.fused = 3 * a.E_pad <= 256 ? 1 : 0;
  if (!make_tmap_bf16(&tw, ws.wsplit, uint64_t(a.d), uint64_t(3) * a.E_pad, uint32_t(a.fused ? 3 * a.E_pad : a.E_pad)))
    return MCL4MOE_ERR_CUDA;
  const size_t stage_bytes = size_t(kRouteTokens) * 128 + 3 * size_t(a.E_pad) * 128;
  int stages = int((110 * 1024) / stage_bytes);
  stages = stages < 2 ? 2 : (stages > 4 ? 4 : stages);
  a.stages = stages;
  const size_t region = size_t(stages) * stage_bytes;
  const size_t tail = tail_smem_bytes(a.E, a.k);
  const size_t smem = 1024 + ((region > tail ? region : tail) + 15) / 16 * 16 + 128;
  uint32_t cols = 32;
  while (cols < uint32_t(a.fused ? 3 * a.E_pad : a.E_pad)) cols <<= 1;
  a.tmem_cols = cols;
  static std::atomic<uint64_t> configured{0};
  if (!raise_smem_limit(router_tc_kernel<EW>, 227 * 1024, configured)) return MCL4MOE_ERR_CUDA;
  if (smem > 227 * 1024) return MCL4MOE_ERR_UNSUPPORTED;
  if (launch_pdl(router_tc_kernel<EW>, dim3(C), dim3(kTcThreads), smem, stream, tx, tw, a, ws) != cudaSuccess)
    return MCL4MOE_ERR_CUDA;
  return cudaGetLastError() == cudaSuccess ? MCL4MOE_OK : MCL4MOE_ERR_CUDA;
}

}  // namespace

int launch_route(const uint16_t* x, const float* wr, const float* bias, const float* logits_in, const uint8_t* valid,
                 int T, int d, int E, int k, int norm_topk, int32_t* topk_idx, float* topk_w, float* logits_out,
                 float* sel_mask, int32_t* counts_out, float* stats, int32_t* offs_out, int32_t* err,
                 const RouteWorkspace& ws, cudaStream_t stream) {
  if (T > 0) {
    RouterTcArgs a{};
    a.bias = bias;
    a.valid = valid;
    a.T = T;
    a.d = d;
    a.E = E;
    a.E_pad = (E + 15) / 16 * 16;
    a.k = k;
    a.norm_topk = norm_topk;
    a.topk_idx = topk_idx;
    a.topk_w = topk_w;
    a.logits_out = logits_out;
    a.sel_mask = sel_mask;
    a.err = err;
    // The GEMV stages 8 bf16 token rows in shared memory (16 d bytes); wider rows take
    // the tensor-core router, which streams d in 64-column boxes at any width.
    const size_t gemv_smem = sizeof(uint16_t) * 8 * size_t(d);
    if (logits_in == nullptr && T <= kRouteTokens && ws.small_logits != nullptr && ws.small_tok != nullptr &&
        small_router_smem(d, E, k) <= kRouteGemvMaxSmem) {
      // one chunk from x: logits, per-token routing and the chunk's statistics in one launch
      a.counts_out = counts_out;
      a.stats = stats;
      a.offs_out = offs_out;
      if (cudaMemsetAsync(ws.small_tok + 2 * kRouteTokens, 0, 17 * sizeof(uint32_t), stream) != cudaSuccess)
        return MCL4MOE_ERR_CUDA;  // completion counters
      const size_t smem = small_router_smem(d, E, k);
      const dim3 grid((T + kSmallTokPerCta - 1) / kSmallTokPerCta, (E + 7) / 8);
      cudaError_t e;
      static std::atomic<uint64_t> c1{0}, c2{0}, c4{0}, c8{0};
      if (E <= 32) {
        if (!raise_smem_limit(router_small_kernel<1>, int(kRouteGemvMaxSmem), c1)) return MCL4MOE_ERR_CUDA;
        e = launch_pdl(router_small_kernel<1>, grid, dim3(256), smem, stream, x, wr, bias, a, ws);
      } else if (E <= 64) {
        if (!raise_smem_limit(router_small_kernel<2>, int(kRouteGemvMaxSmem), c2)) return MCL4MOE_ERR_CUDA;
        e = launch_pdl(router_small_kernel<2>, grid, dim3(256), smem, stream, x, wr, bias, a, ws);
      } else if (E <= 128) {
        if (!raise_smem_limit(router_small_kernel<4>, int(kRouteGemvMaxSmem), c4)) return MCL4MOE_ERR_CUDA;
        e = launch_pdl(router_small_kernel<4>, grid, dim3(256), smem, stream, x, wr, bias, a, ws);
      } else {
        if (!raise_smem_limit(router_small_kernel<8>, int(kRouteGemvMaxSmem), c8)) return MCL4MOE_ERR_CUDA;
        e = launch_pdl(router_small_kernel<8>, grid, dim3(256), smem, stream, x, wr, bias, a, ws);
      }
      return e == cudaSuccess && cudaGetLastError() == cudaSuccess ? MCL4MOE_OK : MCL4MOE_ERR_CUDA;
    }
    if (logits_in == nullptr && T <= kRouteGemvMaxT && ws.small_logits != nullptr && gemv_smem <= kRouteGemvMaxSmem) {
      const size_t smem = gemv_smem;
      if (smem > 48 * 1024) {
        static std::atomic<uint64_t> configured{0};
        if (!raise_smem_limit(router_gemv_kernel, int(kRouteGemvMaxSmem), configured)) return MCL4MOE_ERR_CUDA;
      }
      if (launch_pdl(router_gemv_kernel, dim3((T + 7) / 8, (E + 7) / 8), dim3(256), smem, stream, x, wr, bias, T, d,
                     E, ws.small_logits) != cudaSuccess)
        return MCL4MOE_ERR_CUDA;
      logits_in = ws.small_logits;  // final logits: the tail below adds no bias
    }
    int st;
    if (logits_in != nullptr && T <= kRouteTokens) {  // one chunk: the tail kernel finishes the scan
      a.fuse_scan = 1;
      a.counts_out = counts_out;
      a.stats = stats;
      a.offs_out = offs_out;
    }
    if (E <= 32) st = launch_router_t<1>(x, wr, bias, logits_in, a, ws, stream);
    else if (E <= 64) st = launch_router_t<2>(x, wr, bias, logits_in, a, ws, stream);
    else if (E <= 128) st = launch_router_t<4>(x, wr, bias, logits_in, a, ws, stream);
    else st = launch_router_t<8>(x, wr, bias, logits_in, a, ws, stream);
    if (st != MCL4MOE_OK) return st;
    if (a.fuse_scan) return cudaGetLastError() == cudaSuccess ? MCL4MOE_OK : MCL4MOE_ERR_CUDA;
  } else if (cudaMemsetAsync(ws.done, 0, sizeof(uint32_t), stream) != cudaSuccess) {
    return MCL4MOE_ERR_CUDA;  // no router CTA ran: reset the finished-expert counter here
  }
  const int C = (T + kRouteTokens - 1) / kRouteTokens;
  if (launch_pdl(route_scan_kernel, dim3(E), dim3(256), 0, stream, C, E, k, ws, counts_out, stats, offs_out) !=
      cudaSuccess)
    return MCL4MOE_ERR_CUDA;
  return cudaGetLastError() == cudaSuccess ? MCL4MOE_OK : MCL4MOE_ERR_CUDA;
}

int launch_route_from_indices(const int32_t* topk_idx, const uint8_t* valid, int T, int E, int k, int32_t* counts_out,
                              float* stats, int32_t* offs_out, const RouteWorkspace& ws, cudaStream_t stream) {
  const int C = (T + kRouteTokens - 1) / kRouteTokens;
  if (C > 0) {
    if (launch_pdl(route_ranks_kernel, dim3(C), dim3(256), 0, stream, topk_idx, valid, T, E, k, ws) != cudaSuccess)
      return MCL4MOE_ERR_CUDA;
  } else if (cudaMemsetAsync(ws.done, 0, sizeof(uint32_t), stream) != cudaSuccess) {
    return MCL4MOE_ERR_CUDA;
  }
  return launch_pdl(route_scan_kernel, dim3(E), dim3(256), 0, stream, C, E, k, ws, counts_out, stats, offs_out) ==
                 cudaSuccess
             ? MCL4MOE_OK
             : MCL4MOE_ERR_CUDA;
}

}  // namespace mcl4
