// Expert-parallel dispatch and combine around the grouped NVFP4 GEMMs.
//
// G ranks, rank g owns the contiguous experts [g*E_loc, (g+1)*E_loc).  Every
// rank routes its own tokens (weak scaling), then:
//   dispatch  (source)   one row per (token, destination rank) that holds at
//                        least one of the token's k experts, in token order per
//                        destination: the token's NVFP4 codes and 1x16 E4M3
//                        scales (quantised once, exactly as the single-GPU path
//                        does: activation scales are per row and do not depend on
//                        the expert), its k expert ids local to the destination
//                        (-1 where the expert lives elsewhere) and its k routing
//                        weights;
//   experts   (receiver) rows laid out expert-major in 256-row padded segments,
//                        gate/up + SwiGLU and down GEMMs, then one bf16 partial
//                        sum per received row over that row's local experts;
//   combine   (source)   out[t] = bf16(sum over destinations in rank order of the
//                        returned partials).
// The exchange itself (all-to-all of rows and of partials) is NCCL, driven by the
// host; the returned partials come back in the order the rows were sent, so a
// row's send position is also where its partial lands.
//
// Row format (bytes): [0, d/2) codes | [d/2, d/2 + d/16) scales, row-major |
// k int8 local expert ids, padded to 16 | k fp32 weights, padded to 16.
#include "kernels.cuh"

namespace mcl4 {

namespace {

constexpr int kMaxRanks = 8;

struct EpRow {
  int codes, scales, ids, weights, bytes;
};

__host__ __device__ inline EpRow ep_row(int d, int k) {
  EpRow r;
  r.codes = 0;
  r.scales = d / 2;
  r.ids = d / 2 + d / 16;
  r.weights = r.ids + (k + 15) / 16 * 16;
  r.bytes = r.weights + (4 * k + 15) / 16 * 16;
  return r;
}

// Destinations of one token as a bit mask (bit g: some expert of the token is on rank g).
__device__ __forceinline__ uint32_t dest_mask(const int32_t* topk_idx, const uint8_t* valid, int T, int k, int E_loc,
                                              int t) {
  uint32_t m = 0;
  if (t < T && (valid == nullptr || valid[t] != 0))
    for (int j = 0; j < k; ++j) {
      const int e = topk_idx[int64_t(t) * k + j];
      if (e >= 0) m |= 1u << (e / E_loc);
    }
  return m;
}

// Per 32-token group: rows and expert slots bound for each destination.
__global__ void __launch_bounds__(256) ep_count_kernel(const int32_t* __restrict__ topk_idx,
                                                       const uint8_t* __restrict__ valid, int T, int k, int G,
                                                       int E_loc, int32_t* __restrict__ grp_rows,
                                                       int32_t* __restrict__ send_slots) {
  pdl_wait();     // the previous kernel on the stream has completed (PDL launch)
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int w = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (w >= (T + 31) / 32) return;
  const int t = w * 32 + lane;
  const uint32_t m = dest_mask(topk_idx, valid, T, k, E_loc, t);
  int slots[kMaxRanks];
#pragma unroll
  for (int g = 0; g < kMaxRanks; ++g) slots[g] = 0;
  if (m != 0)
    for (int j = 0; j < k; ++j) {
      const int e = topk_idx[int64_t(t) * k + j];
#pragma unroll
      for (int g = 0; g < kMaxRanks; ++g)
        if (e >= 0 && e / E_loc == g) ++slots[g];
    }
#pragma unroll
  for (int g = 0; g < kMaxRanks; ++g) {
    if (g >= G) break;
    const int c = __popc(__ballot_sync(0xffffffffu, (m >> g) & 1u));
    int s = slots[g];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) {
      grp_rows[w * G + g] = c;
      if (s) atomicAdd(send_slots + g, s);  // integer sum: order does not matter
    }
  }
}

// One CTA per column: exclusive scan over groups in place; column total to ``totals``.
__global__ void __launch_bounds__(256) ep_column_scan_kernel(int32_t* __restrict__ grp, int W, int cols,
                                                             int32_t* __restrict__ totals) {
  pdl_wait();     // the previous kernel on the stream has completed (PDL launch)
  pdl_trigger();
  __shared__ int32_t tmp[64];
  const int c = blockIdx.x, tid = threadIdx.x;
  const int per = (W + blockDim.x - 1) / blockDim.x;
  const int w0 = tid * per, w1 = min(W, w0 + per);
  int32_t mine = 0;
  for (int w = w0; w < w1; ++w) mine += grp[int64_t(w) * cols + c];
  int32_t total;
  int32_t run = block_exclusive_scan(mine, tmp, total);
  for (int w = w0; w < w1; ++w) {
    const int32_t v = grp[int64_t(w) * cols + c];
    grp[int64_t(w) * cols + c] = run;
    run += v;
  }
  if (tid == 0) totals[c] = total;
}

// Quantise each token once and write its row to every destination that needs it.
// One CTA per 32-token group: warp 0 ranks the group's tokens per destination,
// then each warp packs 4 tokens.
__global__ void __launch_bounds__(256) ep_pack_kernel(const uint16_t* __restrict__ x,
                                                      const int32_t* __restrict__ topk_idx,
                                                      const float* __restrict__ topk_w,
                                                      const uint8_t* __restrict__ valid, int T, int d, int k, int G,
                                                      int E_loc, const int32_t* __restrict__ grp_offs,
                                                      const int32_t* __restrict__ send_rows,
                                                      uint8_t* __restrict__ send_buf,
                                                      int32_t* __restrict__ send_pos,
                                                      const int32_t* __restrict__ slot_src, int me) {
  __shared__ int32_t s_pos[32][kMaxRanks];
  __shared__ int32_t s_start[kMaxRanks];
  __shared__ float inv_tab[128];
  fill_inverse_scale_table(inv_tab);
  pdl_wait();     // the previous kernel on the stream has completed (PDL launch)
  pdl_trigger();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int w = blockIdx.x;
  const EpRow L = ep_row(d, k);
  if (threadIdx.x == 0) {
    int a = 0;
    for (int g = 0; g < G; ++g) {
      s_start[g] = a;
      a += send_rows[g];
    }
  }
  __syncthreads();
  if (warp == 0) {
    const int t = w * 32 + lane;
    const uint32_t m = dest_mask(topk_idx, valid, T, k, E_loc, t);
    const uint32_t lt = (1u << lane) - 1u;
    for (int g = 0; g < G; ++g) {
      const bool has = (m >> g) & 1u;
      const uint32_t bal = __ballot_sync(0xffffffffu, has);
      const int pos = has ? s_start[g] + grp_offs[w * G + g] + __popc(bal & lt) : -1;
      s_pos[lane][g] = pos;
      if (t < T) send_pos[int64_t(t) * G + g] = pos;
    }
  }
  __syncthreads();
  const int nblk = d / 16;
  for (int i = 0; i < 4; ++i) {
    const int tl = warp * 4 + i;
    const int t = w * 32 + tl;
    if (t >= T) break;
    bool any = false;
    for (int g = 0; g < G; ++g) any |= s_pos[tl][g] >= 0;
    if (!any) continue;
    // metadata: local ids on each destination and the k weights, or (slot_src) the k
    // destinations of the slots' h in this rank's expert-major layout (me << 28 | row)
    const int e = lane < k ? topk_idx[int64_t(t) * k + lane] : -1;
    const float wt = (lane < k && slot_src == nullptr) ? topk_w[int64_t(t) * k + lane] : 0.f;
    const int32_t code = (lane < k && slot_src != nullptr && e >= 0) ? ((me << 28) | slot_src[int64_t(t) * k + lane]) : -1;
    for (int g = 0; g < G; ++g) {
      const int p = s_pos[tl][g];
      if (p < 0) continue;
      uint8_t* row = send_buf + int64_t(p) * L.bytes;
      const bool here = lane < k && e >= 0 && e / E_loc == g;
      if (lane < (k + 15) / 16 * 16) row[L.ids + lane] = uint8_t(int8_t(here ? e - g * E_loc : -1));
      if (lane < k) {
        if (slot_src != nullptr) reinterpret_cast<int32_t*>(row + L.weights)[lane] = here ? code : -1;
        else reinterpret_cast<float*>(row + L.weights)[lane] = wt;
      }
    }
    // codes and scales (the activation quantiser of the single-GPU path); the row's loads
    // for up to four 32-block passes are issued together
    for (int b0 = 0; b0 < nblk; b0 += 128) {
      uint4 u[4][2];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int b = b0 + 32 * q + lane;
        if (b < nblk) {
          const uint4* src = reinterpret_cast<const uint4*>(x + int64_t(t) * d + b * 16);
          u[q][0] = __ldg(src);
          u[q][1] = __ldg(src + 1);
        }
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        if (b0 + 32 * q >= nblk) break;  // uniform over the warp
        const int b = b0 + 32 * q + lane;
        uint32_t s = 0;
        uint2 pk = make_uint2(0, 0);
        if (b < nblk) {
          const uint32_t wds[8] = {u[q][0].x, u[q][0].y, u[q][0].z, u[q][0].w,
                                   u[q][1].x, u[q][1].y, u[q][1].z, u[q][1].w};
          s = quantize_block16_bf16(wds, pk, inv_tab);
        }
        const int base_lane = lane & ~3;
        uint32_t word = 0;
#pragma unroll
        for (int j4 = 0; j4 < 4; ++j4) word |= (__shfl_sync(0xffffffffu, s, base_lane + j4) & 0xFFu) << (8 * j4);
        for (int g = 0; g < G; ++g) {
          const int p = s_pos[tl][g];
          if (p < 0 || b >= nblk) continue;
          uint8_t* row = send_buf + int64_t(p) * L.bytes;
          *reinterpret_cast<uint2*>(row + L.codes + b * 8) = pk;
          if ((lane & 3) == 0) *reinterpret_cast<uint32_t*>(row + L.scales + b) = word;
        }
      }
    }
  }
}

// Receiver: per 32-row group, slots of each local expert.
template <int EW>
__global__ void __launch_bounds__(256) ep_recv_count_kernel(const uint8_t* __restrict__ recv, int R, int d, int k,
                                                            int E_loc, int32_t* __restrict__ grp_cnt) {
  pdl_wait();     // the previous kernel on the stream has completed (PDL launch)
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int w = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (w >= (R + 31) / 32) return;
  const EpRow L = ep_row(d, k);
  const int r = w * 32 + lane;
  uint32_t mw[EW];
#pragma unroll
  for (int i = 0; i < EW; ++i) mw[i] = 0;
  if (r < R) {
    const int8_t* ids = reinterpret_cast<const int8_t*>(recv + int64_t(r) * L.bytes + L.ids);
    for (int j = 0; j < k; ++j) {
      const int e = ids[j] < E_loc ? ids[j] : -1;  // ids come from the pack kernel: always < E_loc
#pragma unroll
      for (int i = 0; i < EW; ++i)
        if (e >= 0 && (e >> 5) == i) mw[i] |= 1u << (e & 31);
    }
  }
#pragma unroll
  for (int i = 0; i < EW; ++i)
    for (int b = 0; b < 32; ++b) {
      const int e = i * 32 + b;
      const int c = __popc(__ballot_sync(0xffffffffu, (mw[i] >> b) & 1u));
      if (lane == b && e < E_loc) grp_cnt[int64_t(w) * E_loc + e] = c;
    }
}

// Segment starts of the local experts, each padded to kSegRows rows.
__global__ void __launch_bounds__(256) ep_pad_kernel(const int32_t* __restrict__ counts, int E_loc,
                                                     int32_t* __restrict__ pad_start) {
  pdl_wait();     // the previous kernel on the stream has completed (PDL launch)
  pdl_trigger();
  __shared__ int32_t tmp[64];
  const int e = threadIdx.x;
  const int c = e < E_loc ? counts[e] : 0;
  int32_t total;
  const int32_t start = block_exclusive_scan((c + kSegRows - 1) / kSegRows * kSegRows, tmp, total);
  if (e < E_loc) pad_start[e] = start;
  if (e == 0) pad_start[E_loc] = total;
}

// Receiver: copy each received row into the expert-major slots of its local
// experts (codes and scales as they are, into the row-major layout the GEMM reads),
// in received-row order within an expert.  Extra CTAs zero padding-row scales.
template <int EW>
__global__ void __launch_bounds__(256) ep_scatter_kernel(const uint8_t* __restrict__ recv, int R, int d, int k,
                                                         int E_loc, const int32_t* __restrict__ grp_offs,
                                                         const int32_t* __restrict__ counts,
                                                         const int32_t* __restrict__ pad_start,
                                                         uint8_t* __restrict__ xq, uint8_t* __restrict__ xs,
                                                         float* __restrict__ sorted_w,
                                                         int32_t* __restrict__ slot_pos) {
  pdl_wait();     // the previous kernel on the stream has completed (PDL launch)
  pdl_trigger();
  __shared__ uint32_t s_bal[32 * EW];
  __shared__ int32_t s_pos[32][32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int W = (R + 31) / 32;
  const int nblk = d / 16;
  const EpRow L = ep_row(d, k);
  if (int(blockIdx.x) >= W) {
    const int e = blockIdx.x - W;
    const int start = pad_start[e] + counts[e], end = pad_start[e + 1];
    const int groups = nblk / 4;
    for (int i = threadIdx.x; i < (end - start) * groups; i += blockDim.x) {
      const int r = start + i / groups, g = i % groups;
      *reinterpret_cast<uint32_t*>(xs + rowmajor_scale_offset(uint64_t(r), uint32_t(4 * g), uint32_t(nblk))) = 0u;
    }
    return;
  }
  const int w = blockIdx.x;
  if (warp == 0) {
    const int r = w * 32 + lane;
    // local expert id of slot j (ids from the pack kernel are always < E_loc)
    const int8_t* rid = reinterpret_cast<const int8_t*>(recv + int64_t(r) * L.bytes + L.ids);
    auto id_of = [&](int j) {
      const int e = r < R ? int(rid[j]) : -1;
      return e < E_loc ? e : -1;
    };
    uint32_t mw[EW];
#pragma unroll
    for (int i = 0; i < EW; ++i) mw[i] = 0;
    for (int j = 0; j < k; ++j) {
      const int e = id_of(j);
#pragma unroll
      for (int i = 0; i < EW; ++i)
        if (e >= 0 && (e >> 5) == i) mw[i] |= 1u << (e & 31);
    }
#pragma unroll
    for (int i = 0; i < EW; ++i)
      for (int b = 0; b < 32; ++b) {
        const uint32_t bal = __ballot_sync(0xffffffffu, (mw[i] >> b) & 1u);
        if (lane == b) s_bal[i * 32 + b] = bal;
      }
    __syncwarp();
    const uint32_t lt = (1u << lane) - 1u;
    for (int j = 0; j < k; ++j) {
      const int e = id_of(j);
      int pos = -1;
      if (e >= 0) pos = pad_start[e] + grp_offs[int64_t(w) * E_loc + e] + __popc(s_bal[e] & lt);
      s_pos[lane][j] = pos;
      if (r < R) slot_pos[int64_t(r) * k + j] = pos;
    }
  }
  __syncthreads();
  for (int i = 0; i < 4; ++i) {
    const int rl = warp * 4 + i;
    const int r = w * 32 + rl;
    if (r >= R) break;
    const uint8_t* row = recv + int64_t(r) * L.bytes;
    const float* wts = reinterpret_cast<const float*>(row + L.weights);
    for (int j = 0; j < k; ++j) {
      const int p = s_pos[rl][j];
      if (p < 0) continue;
      if (lane == 0) sorted_w[p] = wts[j];
      for (int c = lane; c < d / 32; c += 32)  // 16-byte chunks of codes
        *reinterpret_cast<uint4*>(xq + int64_t(p) * (d / 2) + c * 16) =
            *reinterpret_cast<const uint4*>(row + L.codes + c * 16);
      for (int q = lane; q < nblk / 4; q += 32)
        *reinterpret_cast<uint32_t*>(xs + rowmajor_scale_offset(uint64_t(p), uint32_t(4 * q), uint32_t(nblk))) =
            *reinterpret_cast<const uint32_t*>(row + L.scales + 4 * q);
    }
  }
}

// partial[r] = bf16(sum over the row's local slots, in slot order, of y) (fp32 sum).
__global__ void __launch_bounds__(256) ep_partial_kernel(const uint16_t* __restrict__ y,
                                                         const int32_t* __restrict__ slot_pos, int R, int k, int d,
                                                         uint16_t* __restrict__ partial) {
  pdl_wait();     // the previous kernel on the stream has completed (PDL launch)
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int r = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (r >= R) return;
  const int my_pos = lane < k ? slot_pos[int64_t(r) * k + lane] : -1;
  for (int c = lane * 8; c < d; c += 256) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int j = 0; j < k; ++j) {
      const int p = __shfl_sync(0xffffffffu, my_pos, j);
      if (p < 0) continue;
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(y + int64_t(p) * d + c));
      const uint32_t w4[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        acc[2 * i] = __fadd_rn(acc[2 * i], bf16_to_f32(uint16_t(w4[i] & 0xFFFFu)));
        acc[2 * i + 1] = __fadd_rn(acc[2 * i + 1], bf16_to_f32(uint16_t(w4[i] >> 16)));
      }
    }
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
      o[i] = uint32_t(f32_to_bf16(acc[2 * i])) | (uint32_t(f32_to_bf16(acc[2 * i + 1])) << 16);
    *reinterpret_cast<uint4*>(partial + int64_t(r) * d + c) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// Where the partial of received row r goes: rows of source s are
// [start[s], start[s+1]); row r of source s lands at addr[s] + (r - start[s]) * d
// bf16 elements.  addr[s] may map another GPU's memory (peer / IPC mapping).
struct EpDest {
  int G;
  int32_t start[kMaxRanks + 1];
  uint16_t* addr[kMaxRanks];
};

// ep_partial_kernel with the partial sums stored straight into their sources'
// receive buffers: over NVLink for other GPUs, so the return transfer overlaps
// this kernel's reads of y.
__global__ void __launch_bounds__(256) ep_partial_remote_kernel(const uint16_t* __restrict__ y,
                                                                const int32_t* __restrict__ slot_pos, int R, int k,
                                                                int d, EpDest dst) {
  pdl_wait();     // the previous kernel on the stream has completed (PDL launch)
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int r = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (r >= R) return;
  int s = 0;
  while (s + 1 < dst.G && r >= dst.start[s + 1]) ++s;
  uint16_t* out_row = dst.addr[s] + int64_t(r - dst.start[s]) * d;
  const int my_pos = lane < k ? slot_pos[int64_t(r) * k + lane] : -1;
  for (int c = lane * 8; c < d; c += 256) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int j = 0; j < k; ++j) {
      const int p = __shfl_sync(0xffffffffu, my_pos, j);
      if (p < 0) continue;
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(y + int64_t(p) * d + c));
      const uint32_t w4[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        acc[2 * i] = __fadd_rn(acc[2 * i], bf16_to_f32(uint16_t(w4[i] & 0xFFFFu)));
        acc[2 * i + 1] = __fadd_rn(acc[2 * i + 1], bf16_to_f32(uint16_t(w4[i] >> 16)));
      }
    }
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
      o[i] = uint32_t(f32_to_bf16(acc[2 * i])) | (uint32_t(f32_to_bf16(acc[2 * i + 1])) << 16);
    *reinterpret_cast<uint4*>(out_row + c) = make_uint4(o[0], o[1], o[2], o[3]);
  }
  __threadfence_system();  // the stores reach the peers before anyone is told the kernel is done
}

// out[t] = bf16(sum over destinations g = 0..G-1 of the partial returned for (t, g)).
__global__ void __launch_bounds__(256) ep_final_kernel(const uint16_t* __restrict__ back,
                                                       const int32_t* __restrict__ send_pos, int T, int d, int G,
                                                       uint16_t* __restrict__ out) {
  pdl_wait();     // the previous kernel on the stream has completed (PDL launch)
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (t >= T) return;
  const int my_pos = lane < G ? send_pos[int64_t(t) * G + lane] : -1;
  for (int c = lane * 8; c < d; c += 256) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int g = 0; g < G; ++g) {
      const int p = __shfl_sync(0xffffffffu, my_pos, g);
      if (p < 0) continue;
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(back + int64_t(p) * d + c));
      const uint32_t w4[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        acc[2 * i] = __fadd_rn(acc[2 * i], bf16_to_f32(uint16_t(w4[i] & 0xFFFFu)));
        acc[2 * i + 1] = __fadd_rn(acc[2 * i + 1], bf16_to_f32(uint16_t(w4[i] >> 16)));
      }
    }
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
      o[i] = uint32_t(f32_to_bf16(acc[2 * i])) | (uint32_t(f32_to_bf16(acc[2 * i + 1])) << 16);
    *reinterpret_cast<uint4*>(out + int64_t(t) * d + c) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// Source-side scratch: per-group row counts (scanned in place).
size_t dispatch_ws_bytes(int T, int G) { return align256(sizeof(int32_t) * size_t((T + 31) / 32) * G); }

struct ExpertsWs {
  int32_t* grp;        // [W_R, E_loc]
  int32_t* counts;     // [E_loc]
  int32_t* pad_start;  // [E_loc + 1]
  int32_t* slot_pos;   // [R, k]
  float* sorted_w;     // [mcap]
  uint8_t* xq;         // [mcap, d/2]
  uint8_t* xs;         // row-major [mcap, d/16]
  uint8_t* hq;         // [mcap, F/2]
  uint8_t* hs;         // swizzled [mcap * F/16]
  uint16_t* y;         // [mcap, d]
  int32_t* err;
  int64_t mcap;
  size_t bytes;
};

ExpertsWs experts_ws(void* base, int R, int slots, int d, int k, int E_loc, int F) {
  ExpertsWs w{};
  uint8_t* p = static_cast<uint8_t*>(base);
  size_t off = 0;
  auto take = [&](size_t bytes) {
    uint8_t* r = p ? p + off : nullptr;
    off += align256(bytes);
    return r;
  };
  w.mcap = padded_rows_cap(slots, E_loc, 1);
  w.grp = reinterpret_cast<int32_t*>(take(sizeof(int32_t) * size_t((R + 31) / 32) * E_loc));
  w.counts = reinterpret_cast<int32_t*>(take(sizeof(int32_t) * E_loc));
  w.pad_start = reinterpret_cast<int32_t*>(take(sizeof(int32_t) * (E_loc + 1)));
  w.slot_pos = reinterpret_cast<int32_t*>(take(sizeof(int32_t) * size_t(R) * k));
  w.sorted_w = reinterpret_cast<float*>(take(sizeof(float) * size_t(w.mcap)));
  w.xq = take(size_t(w.mcap) * d / 2);
  w.xs = take(size_t(w.mcap) * d / 16);
  w.hq = take(size_t(w.mcap) * F / 2);
  w.hs = take(size_t(w.mcap) * F / 16);
  w.y = reinterpret_cast<uint16_t*>(take(sizeof(uint16_t) * size_t(w.mcap) * d));
  w.err = reinterpret_cast<int32_t*>(take(sizeof(int32_t)));
  w.bytes = off;
  return w;
}

int check_ep_shape(int d, int k, int G, int E_loc, int F) {
  if (d <= 0 || k <= 0 || G <= 0 || E_loc <= 0 || F <= 0) return MCL4MOE_ERR_INVALID;
  if (G > kMaxRanks || E_loc > kMaxExperts || k > kMaxTopK || d % 256 != 0 || F % 256 != 0)
    return MCL4MOE_ERR_UNSUPPORTED;
  return MCL4MOE_OK;
}

template <int EW>
cudaError_t launch_recv_layout(const uint8_t* recv, int R, int d, int k, int E_loc, const ExpertsWs& w,
                               cudaStream_t s) {
  const int W = (R + 31) / 32;
  cudaError_t e = launch_pdl(ep_recv_count_kernel<EW>, dim3((W + 7) / 8), dim3(256), 0, s, recv, R, d, k, E_loc, w.grp);
  if (e == cudaSuccess) e = launch_pdl(ep_column_scan_kernel, dim3(E_loc), dim3(256), 0, s, w.grp, W, E_loc, w.counts);
  if (e == cudaSuccess) e = launch_pdl(ep_pad_kernel, dim3(1), dim3(256), 0, s, w.counts, E_loc, w.pad_start);
  if (e == cudaSuccess)
    e = launch_pdl(ep_scatter_kernel<EW>, dim3(W + E_loc), dim3(256), 0, s, recv, R, d, k, E_loc, w.grp, w.counts,
                   w.pad_start, w.xq, w.xs, w.sorted_w, w.slot_pos);
  return e;
}

}  // namespace

}  // namespace mcl4

using namespace mcl4;

extern "C" {

int mcl4moe_ep_row_bytes(int d, int k) {
  if (d <= 0 || d % 256 != 0 || k <= 0 || k > kMaxTopK) return 0;
  return ep_row(d, k).bytes;
}

size_t mcl4moe_ep_dispatch_workspace_size(int T, int G) {
  if (T < 0 || G <= 0 || G > kMaxRanks) return 0;
  return dispatch_ws_bytes(T, G);
}

int mcl4moe_ep_dispatch_count(const int32_t* topk_idx, const uint8_t* valid, int T, int k, int G, int E_loc,
                              int32_t* send_counts, void* workspace, size_t workspace_bytes,
                              mcl4moe_stream_t stream) {
  int st = check_ep_shape(256, k, G, E_loc, 256);
  if (st != MCL4MOE_OK) return st;
  if (T < 0 || !send_counts || !workspace || (T > 0 && !topk_idx)) return MCL4MOE_ERR_INVALID;
  if (workspace_bytes < dispatch_ws_bytes(T, G)) return MCL4MOE_ERR_WORKSPACE;
  cudaStream_t s = stream;
  if (cudaMemsetAsync(send_counts, 0, sizeof(int32_t) * 2 * G, s) != cudaSuccess) return MCL4MOE_ERR_CUDA;
  if (T == 0) return MCL4MOE_OK;
  int32_t* grp = static_cast<int32_t*>(workspace);
  const int W = (T + 31) / 32;
  cudaError_t e = launch_pdl(ep_count_kernel, dim3((W + 7) / 8), dim3(256), 0, s, topk_idx, valid, T, k, G, E_loc,
                             grp, send_counts + G);
  if (e == cudaSuccess) e = launch_pdl(ep_column_scan_kernel, dim3(G), dim3(256), 0, s, grp, W, G, send_counts);
  return e == cudaSuccess ? MCL4MOE_OK : MCL4MOE_ERR_CUDA;
}

int mcl4moe_ep_dispatch_pack(const uint16_t* x, const int32_t* topk_idx, const float* topk_w, const uint8_t* valid,
                             int T, int d, int k, int G, int E_loc, const int32_t* send_counts, int32_t* send_pos,
                             uint8_t* send_buf, void* workspace, size_t workspace_bytes, mcl4moe_stream_t stream) {
  int st = check_ep_shape(d, k, G, E_loc, 256);
  if (st != MCL4MOE_OK) return st;
  if (T < 0 || !send_counts || !workspace || (T > 0 && (!x || !topk_idx || !topk_w || !send_pos || !send_buf)))
    return MCL4MOE_ERR_INVALID;
  if (!aligned16(x) || !aligned16(send_buf)) return MCL4MOE_ERR_INVALID;
  if (workspace_bytes < dispatch_ws_bytes(T, G)) return MCL4MOE_ERR_WORKSPACE;
  if (T == 0) return MCL4MOE_OK;
  const int W = (T + 31) / 32;
  return launch_pdl(ep_pack_kernel, dim3(W), dim3(256), 0, stream, x, topk_idx, topk_w, valid, T, d, k, G, E_loc,
                    static_cast<const int32_t*>(workspace), send_counts, send_buf, send_pos,
                    static_cast<const int32_t*>(nullptr), 0) == cudaSuccess
             ? MCL4MOE_OK
             : MCL4MOE_ERR_CUDA;
}

int mcl4moe_ep_dispatch_pack_h(const uint16_t* x, const int32_t* topk_idx, const uint8_t* valid, int T, int d, int k,
                               int G, int E_loc, int rank, const int32_t* slot_pos, const int32_t* send_counts,
                               int32_t* send_pos, uint8_t* send_buf, void* workspace, size_t workspace_bytes,
                               mcl4moe_stream_t stream) {
  int st = check_ep_shape(d, k, G, E_loc, 256);
  if (st != MCL4MOE_OK) return st;
  if (T < 0 || rank < 0 || rank >= G || !send_counts || !workspace ||
      (T > 0 && (!x || !topk_idx || !slot_pos || !send_pos || !send_buf)))
    return MCL4MOE_ERR_INVALID;
  if (!aligned16(x) || !aligned16(send_buf)) return MCL4MOE_ERR_INVALID;
  if (workspace_bytes < dispatch_ws_bytes(T, G)) return MCL4MOE_ERR_WORKSPACE;
  if (T == 0) return MCL4MOE_OK;
  const int W = (T + 31) / 32;
  return launch_pdl(ep_pack_kernel, dim3(W), dim3(256), 0, stream, x, topk_idx, static_cast<const float*>(nullptr),
                    valid, T, d, k, G, E_loc, static_cast<const int32_t*>(workspace), send_counts, send_buf, send_pos,
                    slot_pos, rank) == cudaSuccess
             ? MCL4MOE_OK
             : MCL4MOE_ERR_CUDA;
}

int mcl4moe_ep_dispatch(const uint16_t* x, const int32_t* topk_idx, const float* topk_w, const uint8_t* valid, int T,
                        int d, int k, int G, int E_loc, int32_t* send_counts, int32_t* send_pos, uint8_t* send_buf,
                        void* workspace, size_t workspace_bytes, mcl4moe_stream_t stream) {
  int st = check_ep_shape(d, k, G, E_loc, 256);
  if (st != MCL4MOE_OK) return st;
  if (T < 0 || !send_counts || !workspace || (T > 0 && (!x || !topk_idx || !topk_w || !send_pos || !send_buf)))
    return MCL4MOE_ERR_INVALID;
  if (!aligned16(x) || !aligned16(send_buf)) return MCL4MOE_ERR_INVALID;
  if ((st = mcl4moe_ep_dispatch_count(topk_idx, valid, T, k, G, E_loc, send_counts, workspace, workspace_bytes,
                                      stream)) != MCL4MOE_OK)
    return st;
  return mcl4moe_ep_dispatch_pack(x, topk_idx, topk_w, valid, T, d, k, G, E_loc, send_counts, send_pos, send_buf,
                                  workspace, workspace_bytes, stream);
}

size_t mcl4moe_ep_experts_workspace_size(int R, int slots, int d, int k, int E_loc, int F) {
  if (R < 0 || slots < 0 || check_ep_shape(d, k, 1, E_loc, F) != MCL4MOE_OK) return 0;
  return experts_ws(nullptr, R, slots, d, k, E_loc, F).bytes;
}

}  // extern "C"

namespace {

int ep_experts_impl(const uint8_t* recv_buf, int R, int slots, int d, int k, int E_loc, int F, const uint8_t* w_up,
                    const uint8_t* w_up_scales, const float* w_up_g, const uint8_t* w_dn, const uint8_t* w_dn_scales,
                    const float* w_dn_g, uint16_t* partial, const EpDest* remote, int32_t* error_word,
                    void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  int st = check_ep_shape(d, k, 1, E_loc, F);
  if (st != MCL4MOE_OK) return st;
  if (R < 0 || slots < 0 || !workspace || (R > 0 && (!recv_buf || (!partial && !remote)))) return MCL4MOE_ERR_INVALID;
  if (!w_up || !w_up_scales || !w_up_g || !w_dn || !w_dn_scales || !w_dn_g) return MCL4MOE_ERR_INVALID;
  if (!aligned16(recv_buf) || !aligned16(partial) || !aligned16(w_up) || !aligned16(w_dn) ||
      !aligned16(w_up_scales) || !aligned16(w_dn_scales))
    return MCL4MOE_ERR_INVALID;
  const ExpertsWs w = experts_ws(workspace, R, slots, d, k, E_loc, F);
  if (workspace_bytes < w.bytes) return MCL4MOE_ERR_WORKSPACE;
  if (R == 0) return MCL4MOE_OK;
  cudaStream_t s = stream;
  int32_t* err = error_word ? error_word : w.err;
  if (!error_word && cudaMemsetAsync(w.err, 0, sizeof(int32_t), s) != cudaSuccess) return MCL4MOE_ERR_CUDA;
  const cudaError_t le = E_loc <= 32    ? launch_recv_layout<1>(recv_buf, R, d, k, E_loc, w, s)
                         : E_loc <= 64  ? launch_recv_layout<2>(recv_buf, R, d, k, E_loc, w, s)
                         : E_loc <= 128 ? launch_recv_layout<4>(recv_buf, R, d, k, E_loc, w, s)
                                        : launch_recv_layout<8>(recv_buf, R, d, k, E_loc, w, s);
  if (le != cudaSuccess) return MCL4MOE_ERR_CUDA;
  if (cudaGetLastError() != cudaSuccess) return MCL4MOE_ERR_CUDA;

  GemmArgs g1{};
  g1.pad_start = w.pad_start;
  g1.row_count = w.counts;
  g1.a_scales = w.xs;
  g1.a_sf_rowmajor = 1;
  g1.b_scales = w_up_scales;
  g1.b_g = w_up_g;
  g1.E = E_loc;
  g1.K = d;
  g1.N_total = 2 * F;
  g1.n_tiles = F / 128;
  g1.mode = 0;
  g1.F = F;
  g1.hq = w.hq;
  g1.hs = w.hs;
  g1.err = err;
  if ((st = launch_grouped_gemm(w.xq, w.mcap, w_up, g1, s)) != MCL4MOE_OK) return st;
  GemmArgs g2{};
  g2.pad_start = w.pad_start;
  g2.row_count = w.counts;
  g2.a_scales = w.hs;
  g2.b_scales = w_dn_scales;
  g2.b_g = w_dn_g;
  g2.E = E_loc;
  g2.K = F;
  g2.N_total = d;
  g2.n_tiles = d / 256;
  g2.mode = 1;
  g2.row_w = w.sorted_w;
  g2.y = w.y;
  g2.ldy = d;
  g2.err = err;
  if ((st = launch_grouped_gemm(w.hq, w.mcap, w_dn, g2, s)) != MCL4MOE_OK) return st;
  if (remote)
    return launch_pdl(ep_partial_remote_kernel, dim3((R + 7) / 8), dim3(256), 0, s, w.y, w.slot_pos, R, k, d,
                      *remote) == cudaSuccess
               ? MCL4MOE_OK
               : MCL4MOE_ERR_CUDA;
  return launch_pdl(ep_partial_kernel, dim3((R + 7) / 8), dim3(256), 0, s, w.y, w.slot_pos, R, k, d, partial) ==
                 cudaSuccess
             ? MCL4MOE_OK
             : MCL4MOE_ERR_CUDA;
}

}  // namespace

extern "C" {

int mcl4moe_ep_experts(const uint8_t* recv_buf, int R, int slots, int d, int k, int E_loc, int F,
                       const uint8_t* w_up, const uint8_t* w_up_scales, const float* w_up_g, const uint8_t* w_dn,
                       const uint8_t* w_dn_scales, const float* w_dn_g, uint16_t* partial, int32_t* error_word,
                       void* workspace, size_t workspace_bytes, mcl4moe_stream_t stream) {
  return ep_experts_impl(recv_buf, R, slots, d, k, E_loc, F, w_up, w_up_scales, w_up_g, w_dn, w_dn_scales, w_dn_g,
                         partial, nullptr, error_word, workspace, workspace_bytes, stream);
}

int mcl4moe_ep_experts_to_peers(const uint8_t* recv_buf, int R, int slots, int d, int k, int E_loc, int F,
                                const uint8_t* w_up, const uint8_t* w_up_scales, const float* w_up_g,
                                const uint8_t* w_dn, const uint8_t* w_dn_scales, const float* w_dn_g, int G,
                                const int32_t* seg_start, void* const* dst, int32_t* error_word, void* workspace,
                                size_t workspace_bytes, mcl4moe_stream_t stream) {
  if (G <= 0 || G > kMaxRanks || !seg_start || !dst) return MCL4MOE_ERR_INVALID;
  EpDest e{};
  e.G = G;
  for (int s = 0; s <= G; ++s) e.start[s] = seg_start[s];
  if (e.start[0] != 0 || e.start[G] != R) return MCL4MOE_ERR_INVALID;
  for (int s = 0; s < G; ++s) {
    if (e.start[s + 1] < e.start[s]) return MCL4MOE_ERR_INVALID;
    if (e.start[s + 1] > e.start[s] && (!dst[s] || !aligned16(dst[s]))) return MCL4MOE_ERR_INVALID;
    e.addr[s] = static_cast<uint16_t*>(dst[s]);
  }
  return ep_experts_impl(recv_buf, R, slots, d, k, E_loc, F, w_up, w_up_scales, w_up_g, w_dn, w_dn_scales, w_dn_g,
                         nullptr, &e, error_word, workspace, workspace_bytes, stream);
}

int mcl4moe_ep_gateup_to_peers(const uint8_t* recv_buf, int R, int slots, int d, int k, int E_loc, int F,
                               const uint8_t* w_up, const uint8_t* w_up_scales, const float* w_up_g, int G,
                               void* const* hq_dst, void* const* hs_dst, int32_t* error_word, void* workspace,
                               size_t workspace_bytes, mcl4moe_stream_t stream) {
  int st = check_ep_shape(d, k, G, E_loc, F);
  if (st != MCL4MOE_OK) return st;
  if (R < 0 || slots < 0 || !workspace || !hq_dst || !hs_dst || (R > 0 && !recv_buf)) return MCL4MOE_ERR_INVALID;
  if (!w_up || !w_up_scales || !w_up_g || !aligned16(recv_buf) || !aligned16(w_up) || !aligned16(w_up_scales))
    return MCL4MOE_ERR_INVALID;
  for (int g = 0; g < G; ++g)
    if (!hq_dst[g] || !hs_dst[g] || !aligned16(hq_dst[g]) || (reinterpret_cast<uintptr_t>(hs_dst[g]) & 1))
      return MCL4MOE_ERR_INVALID;
  const ExpertsWs w = experts_ws(workspace, R, slots, d, k, E_loc, F);
  if (workspace_bytes < w.bytes) return MCL4MOE_ERR_WORKSPACE;
  if (R == 0) return MCL4MOE_OK;
  cudaStream_t s = stream;
  int32_t* err = error_word ? error_word : w.err;
  if (!error_word && cudaMemsetAsync(w.err, 0, sizeof(int32_t), s) != cudaSuccess) return MCL4MOE_ERR_CUDA;
  const cudaError_t le = E_loc <= 32    ? launch_recv_layout<1>(recv_buf, R, d, k, E_loc, w, s)
                         : E_loc <= 64  ? launch_recv_layout<2>(recv_buf, R, d, k, E_loc, w, s)
                         : E_loc <= 128 ? launch_recv_layout<4>(recv_buf, R, d, k, E_loc, w, s)
                                        : launch_recv_layout<8>(recv_buf, R, d, k, E_loc, w, s);
  if (le != cudaSuccess || cudaGetLastError() != cudaSuccess) return MCL4MOE_ERR_CUDA;
  GemmArgs g1{};
  g1.pad_start = w.pad_start;
  g1.row_count = w.counts;
  g1.a_scales = w.xs;
  g1.a_sf_rowmajor = 1;
  g1.b_scales = w_up_scales;
  g1.b_g = w_up_g;
  g1.E = E_loc;
  g1.K = d;
  g1.N_total = 2 * F;
  g1.n_tiles = F / 128;
  g1.mode = 4;
  g1.F = F;
  g1.row_w = w.sorted_w;  // the rows' h destinations, from the dispatched rows
  g1.err = err;
  for (int g = 0; g < G; ++g) {
    g1.peer_hq[g] = static_cast<uint8_t*>(hq_dst[g]);
    g1.peer_hs[g] = static_cast<uint8_t*>(hs_dst[g]);
  }
  return launch_grouped_gemm(w.xq, w.mcap, w_up, g1, s);
}

int mcl4moe_ep_combine(const uint16_t* back_buf, const int32_t* send_pos, int T, int d, int G, uint16_t* out,
                       mcl4moe_stream_t stream) {
  if (T < 0 || d <= 0 || d % 256 != 0 || G <= 0 || G > kMaxRanks) return MCL4MOE_ERR_INVALID;
  if (T == 0) return MCL4MOE_OK;
  if (!send_pos || !out || !aligned16(out) || (back_buf && !aligned16(back_buf))) return MCL4MOE_ERR_INVALID;
  return launch_pdl(ep_final_kernel, dim3((T + 7) / 8), dim3(256), 0, stream, back_buf, send_pos, T, d, G, out) ==
                 cudaSuccess
             ? MCL4MOE_OK
             : MCL4MOE_ERR_CUDA;
}

}  // extern "C"
