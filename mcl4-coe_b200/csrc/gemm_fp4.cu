// Grouped NVFP4 x NVFP4 GEMM on the 5th-generation tensor cores (tcgen05,
// kind::mxf4nvf4, UE4M3 scale per 16 K), persistent over ragged expert
// segments.  Replaces the reference's Triton tl.dot_scaled kernel
// _nvfp4_grouped_mm_kernel (src/mcl4_coe/nvfp4.py:798-874):
//   out[m, n] = bf16( sum_k deq(A)[m, k] * deq(B_e)[n, k] * g_a * g_b[e] )
// for the rows m of expert e, with g_a = 1 (activations).
//
// Layout: A rows are grouped by expert and each expert segment is padded to a
// multiple of 128 rows (pad_start[E+1]); every 128-row M block therefore
// belongs to exactly one expert and its scales are whole 128x4 atoms.
// Tile 128 x 256, K step 256 (one 128-byte swizzle row of packed FP4).
//
// Warp roles (704 threads, one CTA per SM):
//   warp 0       TMA producer: A tile, two 128-row B halves, 3 scale bulk copies
//   warp 1       TMEM owner + single-thread MMA issuer (4 MMAs per stage)
//   warps 2..5   scale-factor writers, one per TMEM lane quarter: each scale
//                atom (128 rows x 4 scales, 512 B) is read from shared memory
//                into registers and written to its 4 TMEM columns with
//                tcgen05.st.  Every lane quarter writes the same 32-row data,
//                which is the 4x replicated layout the block-scaled MMA reads.
//                (tcgen05.cp would do the same but costs tensor-pipe time per
//                instruction comparable to an MMA, serialised with the MMAs.)
//   warps 6..21  epilogue: TMEM -> registers, then
//                mode 0 (gate/up): SwiGLU in bf16 and NVFP4 re-quantisation of h
//                                  (src/mcl4_coe/backbone.py:572-574)
//                mode 1 (down):    bf16(acc*g) [* bf16(routing weight)] to bf16 rows
//                                  (src/mcl4_coe/backbone.py:903)
// Pipelines: 4 smem stages (full / scales-full / empty mbarriers); one
// 256-column fp32 accumulator released by the epilogue right after it is
// read, so the next tile's MMAs overlap the epilogue math.  Scale factors live
// in a per-stage TMEM ring, overwritten only after the MMAs that read them
// completed.  Every wait is bounded (error word instead of a hang).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "kernels.cuh"

namespace mcl4 {

namespace {

constexpr int kBM = 128, kBN = 256, kBK = 256;
constexpr int kStages = 4;
constexpr uint32_t kATile = kBM * kBK / 2;   // 16384
constexpr uint32_t kBHalf = 128 * kBK / 2;    // 16384 (128 rows)
constexpr uint32_t kSFA = kBM * kBK / 16;      // 2048
constexpr uint32_t kSFBHalf = 128 * kBK / 16;  // 2048
constexpr uint32_t kStageBytes = kATile + 2 * kBHalf + kSFA + 2 * kSFBHalf;  // 55296
constexpr uint32_t kOffB = kATile, kOffSFA = kATile + 2 * kBHalf, kOffSFB = kOffSFA + kSFA;
constexpr int kSfWarps = 4;
constexpr int kEpiWarps = 16;
constexpr int kEpiWarp0 = 2 + kSfWarps;
constexpr int kThreads = 32 * (kEpiWarp0 + kEpiWarps);
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kSfCol0 = 256;          // accumulator uses columns [0, 256)
constexpr uint32_t kSfColsPerStage = 48;   // SFA 4 x 4 + SFB 4 x 8
constexpr uint32_t kIdesc = idesc_nvf4(128, 256);
constexpr uint32_t kBarBytes = 256;
constexpr size_t kSmemBytes = size_t(kStages) * kStageBytes + 1024 /*align*/ + kBarBytes +
                              sizeof(int32_t) * (kMaxExperts + 1);

static_assert(kSfCol0 + kStages * kSfColsPerStage <= kTmemCols, "TMEM budget");
static_assert(kStageBytes % 1024 == 0, "stage must keep 1024-byte alignment for 128B swizzle");

struct TileCoord {
  int e, mb, nt;
};

__device__ __forceinline__ int find_expert(const int32_t* pad_s, int E, int row) {
  int lo = 0, hi = E + 1;  // upper_bound(pad_s[0..E], row) - 1
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (pad_s[mid] <= row) lo = mid + 1;
    else hi = mid;
  }
  return lo - 1;
}

}  // namespace

__global__ void __launch_bounds__(kThreads, 1)
    grouped_gemm_fp4_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                            GemmArgs args) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base - raw_addr);
  const uint32_t bar_base = base + kStages * kStageBytes;
  auto full_bar = [&](int s) { return bar_base + 8u * s; };
  auto empty_bar = [&](int s) { return bar_base + 8u * (kStages + s); };
  auto sf_bar = [&](int s) { return bar_base + 8u * (2 * kStages + s); };
  const uint32_t tfull_bar = bar_base + 8u * (3 * kStages);
  const uint32_t tempty_bar = bar_base + 8u * (3 * kStages + 1);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kStages * kStageBytes + 8 * (3 * kStages + 2));
  int32_t* pad_s = reinterpret_cast<int32_t*>(smem + kStages * kStageBytes + kBarBytes);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int E = args.E;

  for (int i = tid; i <= E; i += kThreads) pad_s[i] = args.pad_start[i];
  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
      mbar_init(sf_bar(s), kSfWarps);
    }
    mbar_init(tfull_bar, 1);
    mbar_init(tempty_bar, kEpiWarps);
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmap_a);
    prefetch_tmap(&tmap_b);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int total_mb = pad_s[E] / kBM;
  const int n_tiles = args.n_tiles;
  const int total_tiles = total_mb * n_tiles;
  const int kblocks = args.K / kBK;
  const uint32_t sf_row_stride = uint32_t(args.K / 64) * 512u;  // bytes per 128-row scale block
  auto coord = [&](int t) {
    TileCoord c;
    c.mb = t / n_tiles;
    c.nt = t - c.mb * n_tiles;
    c.e = find_expert(pad_s, E, c.mb * kBM);
    return c;
  };
  auto b_rows = [&](const TileCoord& c, int& lr0, int& lr1) {  // local B rows of the two 128-row halves
    if (args.mode == 0) {
      lr0 = c.nt * 128;
      lr1 = args.F + c.nt * 128;
    } else {
      lr0 = c.nt * kBN;
      lr1 = lr0 + 128;
    }
  };

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x) {
        const TileCoord c = coord(t);
        int lr0, lr1;
        b_rows(c, lr0, lr1);
        const int brow = c.e * args.N_total;
        const uint8_t* bsc = args.b_scales + size_t(c.e) * (size_t(args.N_total) * args.K / 16);
        const uint8_t* asc = args.a_scales + size_t(c.mb) * sf_row_stride;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(empty_bar(stage), phase ^ 1u, args.err, 101)) {
            ok = false;
            break;
          }
          const uint32_t st = base + stage * kStageBytes;
          mbar_arrive_expect_tx(full_bar(stage), kStageBytes);
          tma_load_2d(st, &tmap_a, kb * (kBK / 2), c.mb * kBM, full_bar(stage));
          tma_load_2d(st + kOffB, &tmap_b, kb * (kBK / 2), brow + lr0, full_bar(stage));
          tma_load_2d(st + kOffB + kBHalf, &tmap_b, kb * (kBK / 2), brow + lr1, full_bar(stage));
          bulk_load(st + kOffSFA, asc + kb * 2048, kSFA, full_bar(stage));
          bulk_load(st + kOffSFB, bsc + size_t(lr0 / 128) * sf_row_stride + kb * 2048, kSFBHalf, full_bar(stage));
          bulk_load(st + kOffSFB + kSFBHalf, bsc + size_t(lr1 / 128) * sf_row_stride + kb * 2048, kSFBHalf,
                    full_bar(stage));
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x) {
        if (!mbar_wait(tempty_bar, acc_phase ^ 1u, args.err, 201)) break;
        tc_fence_after();
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(full_bar(stage), phase, args.err, 202) || !mbar_wait(sf_bar(stage), phase, args.err, 203)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t st = base + stage * kStageBytes;
          const uint32_t sf_col = tmem_base + kSfCol0 + stage * kSfColsPerStage;
#pragma unroll
          for (int ks = 0; ks < 4; ++ks) {
            const uint64_t adesc = smem_desc(st + 32 * ks, 16, 1024, 2);
            const uint64_t bdesc = smem_desc(st + kOffB + 32 * ks, 16, 1024, 2);
            tc_mma_nvf4(tmem_base, adesc, bdesc, kIdesc, sf_col + 4 * ks, sf_col + 16 + 8 * ks,
                        (kb | ks) != 0 ? 1u : 0u);
          }
          tc_commit(empty_bar(stage));
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        tc_commit(tfull_bar);
        acc_phase ^= 1u;
      }
    }
    __syncwarp();
  } else if (warp < kEpiWarp0) {
    // ------------------------------------------------------------ scale-factor writers
    // Lane l of quarter q copies bytes [16 l, 16 l + 16) of each 512-byte atom
    // (the 4 scales of rows l, l+32, l+64, l+96) to TMEM lane 32q + l, 4 columns.
    // A stage's TMEM slot is free once the stage is full again: the producer
    // only refills a stage after the MMAs that read it (and its scales) completed.
    const int q = warp & 3;
    const uint32_t lane_base = uint32_t(q * 32) << 16;
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x) {
      for (int kb = 0; kb < kblocks; ++kb) {
        if (!mbar_wait(full_bar(stage), phase, args.err, 121)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint8_t* st = smem + stage * kStageBytes;
        const uint32_t sf_col = tmem_base + lane_base + kSfCol0 + stage * kSfColsPerStage;
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
          tmem_st4(sf_col + 4 * ks, *reinterpret_cast<const uint4*>(st + kOffSFA + ks * 512 + lane * 16));
          tmem_st4(sf_col + 16 + 8 * ks, *reinterpret_cast<const uint4*>(st + kOffSFB + ks * 512 + lane * 16));
          tmem_st4(sf_col + 16 + 8 * ks + 4,
                   *reinterpret_cast<const uint4*>(st + kOffSFB + kSFBHalf + ks * 512 + lane * 16));
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(sf_bar(stage));
        if (++stage == kStages) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    // 16 warps: lane quarter q = warp % 4 (the TMEM lanes a warp may read),
    // column group sub = 0..3 (32 h columns in mode 0, 64 output columns in mode 1).
    const int q = warp & 3;
    const int sub = (warp - kEpiWarp0) >> 2;
    const int row_in_tile = q * 32 + lane;
    const uint32_t lane_addr = tmem_base + (uint32_t(q * 32) << 16);
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < total_tiles; t += gridDim.x) {
      const TileCoord c = coord(t);
      // per-tile scalars first: their load latency overlaps the MMAs of this tile
      const int64_t p = int64_t(c.mb) * kBM + row_in_tile;  // padded row
      const int local = int(p - pad_s[c.e]);
      const float gb = __ldg(args.b_g + c.e);
      const int rows_e = args.row_count ? __ldg(args.row_count + c.e) : (1 << 30);
      const float wrow = (args.mode == 1 && args.row_w && local < rows_e) ? __ldg(args.row_w + p) : 0.f;
      if (!mbar_wait(tfull_bar, acc_phase, args.err, 301)) break;
      acc_phase ^= 1u;
      tc_fence_after();
      uint32_t va[32], vb[32];
      if (args.mode == 0) {
        tmem_ld32(lane_addr + sub * 32, va);        // gate columns
        tmem_ld32(lane_addr + 128 + sub * 32, vb);  // value columns
      } else {
        tmem_ld32(lane_addr + sub * 64, va);
        tmem_ld32(lane_addr + sub * 64 + 32, vb);
      }
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty_bar);  // accumulator may be overwritten now

      const bool row_valid = local < rows_e;
      if (args.mode == 0) {
        // up = bf16(acc * g); h = bf16(bf16(silu(gate)) * value) (src/mcl4_coe/backbone.py:572-574),
        // then NVFP4 with 1x16 row scales (src/mcl4_coe/nvfp4.py:197-225).
        const int F = args.F;
        const int hb0 = c.nt * 8 + sub * 2;  // first 16-column block of h handled here
        uint32_t packed[4];
        uint32_t sword = 0;
#pragma unroll
        for (int blk = 0; blk < 2; ++blk) {
          uint32_t hh[8];
          uint32_t mx = 0;
#pragma unroll
          for (int pr = 0; pr < 8; ++pr) {
            const int j = blk * 16 + 2 * pr;
            const uint32_t gg = pack_bf16x2(__uint_as_float(va[j]) * gb, __uint_as_float(va[j + 1]) * gb);
            const uint32_t uu = pack_bf16x2(__uint_as_float(vb[j]) * gb, __uint_as_float(vb[j + 1]) * gb);
            const uint32_t ss = pack_bf16x2(silu_f32(bf16x2_lo(gg)), silu_f32(bf16x2_hi(gg)));
            hh[pr] = bf16x2_mul(ss, uu);
            mx = bf16x2_max(mx, hh[pr] & 0x7FFF7FFFu);
          }
          float inv;
          sword |= act_block_scale(fmaxf(bf16x2_lo(mx), bf16x2_hi(mx)), inv) << (8 * blk);
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            float n[8];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              n[2 * i] = __fmul_rn(bf16x2_lo(hh[half * 4 + i]), inv);
              n[2 * i + 1] = __fmul_rn(bf16x2_hi(hh[half * 4 + i]), inv);
            }
            packed[blk * 2 + half] = e2m1x8_act(n);
          }
          if (args.h_dbg != nullptr) {
            uint4* dst = reinterpret_cast<uint4*>(args.h_dbg + p * F + (hb0 + blk) * 16);
            dst[0] = make_uint4(hh[0], hh[1], hh[2], hh[3]);
            dst[1] = make_uint4(hh[4], hh[5], hh[6], hh[7]);
          }
        }
        *reinterpret_cast<uint4*>(args.hq + p * (F / 2) + hb0 * 8) =
            make_uint4(packed[0], packed[1], packed[2], packed[3]);
        *reinterpret_cast<uint16_t*>(args.hs +
                                     swizzled_scale_offset(uint64_t(p), uint32_t(hb0), uint32_t(F / 16))) =
            uint16_t(sword);
      } else if (row_valid) {
        // y = bf16(acc * g) [* bf16(routing weight), rounded to bf16] (src/mcl4_coe/backbone.py:903)
        const int64_t dst_row = args.out_row_base ? int64_t(args.out_row_base[c.e]) + local : p;
        const uint32_t ww = pack_bf16x2(wrow, wrow);
        uint4* dst = reinterpret_cast<uint4*>(args.y + dst_row * args.ldy + c.nt * kBN + sub * 64);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const uint32_t* src = i < 4 ? va + 8 * i : vb + 8 * (i - 4);
          uint32_t o[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint32_t yy = pack_bf16x2(__uint_as_float(src[2 * j]) * gb, __uint_as_float(src[2 * j + 1]) * gb);
            o[j] = args.row_w ? bf16x2_mul(yy, ww) : yy;
          }
          dst[i] = make_uint4(o[0], o[1], o[2], o[3]);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
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

// 2-D map over a [rows, row_bytes] uint8 matrix, box 128 bytes x 128 rows, 128B swizzle.
bool make_tmap(CUtensorMap* m, const void* base, uint64_t row_bytes, uint64_t rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {row_bytes, rows};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {128, 128};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

int num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

int launch_grouped_gemm(const uint8_t* a, int64_t a_rows, const uint8_t* b, const GemmArgs& args,
                        cudaStream_t stream) {
  if (args.K % kBK != 0 || args.E < 1 || args.E > kMaxExperts) return MCL4MOE_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) | reinterpret_cast<uintptr_t>(args.a_scales) |
       reinterpret_cast<uintptr_t>(args.b_scales)) & 15)
    return MCL4MOE_ERR_INVALID;
  CUtensorMap ta, tb;
  if (!make_tmap(&ta, a, uint64_t(args.K) / 2, uint64_t(a_rows))) return MCL4MOE_ERR_CUDA;
  if (!make_tmap(&tb, b, uint64_t(args.K) / 2, uint64_t(args.E) * args.N_total)) return MCL4MOE_ERR_CUDA;
  static bool configured = false;
  if (!configured) {
    if (cudaFuncSetAttribute(grouped_gemm_fp4_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kSmemBytes)) !=
        cudaSuccess)
      return MCL4MOE_ERR_CUDA;
    configured = true;
  }
  grouped_gemm_fp4_kernel<<<num_sms(), kThreads, kSmemBytes, stream>>>(ta, tb, args);
  return cudaGetLastError() == cudaSuccess ? MCL4MOE_OK : MCL4MOE_ERR_CUDA;
}

}  // namespace mcl4
