// Grouped NVFP4 x NVFP4 GEMM on the 5th-generation tensor cores (tcgen05,
// kind::mxf4nvf4, UE4M3 scale per 16 K), persistent over ragged expert
// segments.  Replaces the reference's Triton tl.dot_scaled kernel
// _nvfp4_grouped_mm_kernel (src/mcl4_coe/nvfp4.py:798-874):
//   out[m, n] = bf16( sum_k deq(A)[m, k] * deq(B_e)[n, k] * g_a * g_b[e] )
// for the rows m of expert e, with g_a = 1 (activations).
//
// Layout: A rows are grouped by expert and each expert segment is padded to a
// multiple of kSegRows = 256 rows (pad_start[E+1]); every 256-row block
// therefore belongs to exactly one expert and its scales are whole 128x4 atoms.
//
// CTA pairs.  The kernel runs as clusters of two CTAs on two SMs.  A pair
// computes a 256 x 256 output tile with one tcgen05.mma.cta_group::2 per K step
// of 64: each CTA stages its own 128 A rows and one 128-row half of the tile's
// 256 B rows, so a CTA streams 32 KB of operands per 256-deep K block instead
// of 48 KB for a single-SM 128 x 256 tile (the L2 -> SM traffic is what bounds
// the single-SM kernel).  Each CTA's TMEM receives its 128 accumulator rows,
// its own A scales and the full-N B scales (the layout the pair MMA reads).
// K step 256 per stage (one 128-byte swizzle row of packed FP4).
//
// Warp roles (704 threads per CTA, one CTA per SM):
//   warp 0       TMA producer: A tile and B half (completion counted on the
//                even CTA's barrier), 3 scale bulk copies (own barrier)
//   warp 1       TMEM owner; in the even CTA also the single-thread issuer of
//                the pair MMAs (4 per stage), committing to both CTAs' barriers
//   warps 2..5   scale-factor writers, one per TMEM lane quarter: each scale
//                atom (128 rows x 4 scales, 512 B) is read from shared memory
//                into registers and written to its 4 TMEM columns with
//                tcgen05.st.  Every lane quarter writes the same 32-row data,
//                which is the 4x replicated layout the block-scaled MMA reads.
//                (tcgen05.cp would do the same but costs tensor-pipe time per
//                instruction comparable to an MMA, serialised with the MMAs.)
//   warps 6..21  epilogue: TMEM -> registers, then
//                MODE 0 (gate/up): SwiGLU in bf16 and NVFP4 re-quantisation of h
//                                  (src/mcl4_coe/backbone.py:572-574)
//                MODE 1 (down):    bf16(acc*g) [* bf16(routing weight)] rows,
//                                  staged in 128B-swizzled shared memory and
//                                  written with TMA tile stores (full lines)
//                                  (src/mcl4_coe/backbone.py:903)
//                MODE 3 (gate/up, training): MODE 0 that also stores the bf16 gate and
//                                  value columns for the backward
//                MODE 2 (grouped linear): as MODE 1 into unpadded destination
//                                  rows with per-row stores of valid rows only
// Pipelines: smem stages with full (A/B bytes and TMEM scales of both CTAs,
// on the even CTA), scales-landed and empty mbarriers; one 256-column fp32
// accumulator released by both CTAs' epilogues right after it is read, so the
// next tile's MMAs overlap the epilogue math.  Scale factors live in a
// per-stage TMEM ring, overwritten only after the MMAs that read them
// completed.  Every mbarrier wait is bounded (error word instead of a hang).
// Every CTA fetches its own operand tiles with plain TMA loads (nothing is shared across the pair).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstring>
#include <mutex>

#include "kernels.cuh"

namespace mcl4 {

namespace {

constexpr int kBM = 128;  // rows per CTA; a pair covers kSegRows = 256
constexpr int kBN = 256, kBK = 256;
constexpr uint32_t kATile = kBM * kBK / 2;          // 16384
constexpr uint32_t kBHalf = 128 * kBK / 2;          // 16384: this CTA's 128 of the tile's 256 B rows
constexpr uint32_t kSFA = kBM * kBK / 16;           // 2048
constexpr uint32_t kSFBHalf = 128 * kBK / 16;       // 2048
constexpr uint32_t kABBytes = kATile + kBHalf;      // 32768 per CTA and stage
constexpr uint32_t kSFBytes = kSFA + 2 * kSFBHalf;  // 6144 per CTA and stage (full-N B scales)
constexpr uint32_t kStageBytes = kABBytes + kSFBytes;  // 38912 (pair); scale offsets per variant in Cfg
constexpr uint32_t kOffB = kATile;
constexpr int kSfWarps = 4;
constexpr int kEpiWarps = 16;
constexpr int kEpiWarp0 = 2 + kSfWarps;
constexpr int kThreads = 32 * (kEpiWarp0 + kEpiWarps);
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kSfCol0 = 256;         // accumulator uses columns [0, 256)
constexpr uint32_t kSfColsPerStage = 48;  // SFA 4 x 4 + SFB 4 x 8
constexpr uint32_t kIdesc = idesc_nvf4(256, 256);
constexpr uint32_t kIdescSolo = idesc_nvf4(128, 256);
constexpr uint32_t kBarBytes = 256;
constexpr uint32_t kWarpStoreBytes = 32 * 64 * 2;  // one epilogue warp's 32 rows x 64 bf16 (MODES 1, 3)
// MODE 4: per TMEM lane quarter, the tile's 32 rows of h assembled from its four column
// warps before they leave for the peers: codes 32 x 64 B, scales 32 x 8 B, destinations 32 x 4 B
constexpr uint32_t kH4Codes = 0, kH4Scales = 32 * 64, kH4Dst = kH4Scales + 32 * 8;
constexpr uint32_t kH4Quarter = kH4Dst + 32 * 4;

// SOLO: each CTA computes its own 128 x 256 tiles with cta_group::1 MMAs (M = 128),
// staging the full 256 B rows of the tile; used when experts hold few rows
// (decode), where a pair's 256-row tile would mostly multiply padding.
template <int MODE, bool SOLO = false>
struct Cfg {
  static constexpr uint32_t kAB = SOLO ? kATile + 2 * kBHalf : kABBytes;
  static constexpr uint32_t kStage = kAB + kSFBytes;
  static constexpr uint32_t kOffSfa = kAB, kOffSfb = kAB + kSFA;
  static constexpr int kStages = SOLO ? 4 : ((MODE == 0 || MODE == 4) ? 5 : 4);
  static constexpr uint32_t kStoreBytes = (!SOLO && (MODE == 1 || MODE == 3)) ? kEpiWarps * kWarpStoreBytes
                                          : (MODE == 4 ? 4 * kH4Quarter : 0);
  static constexpr size_t kSmem = 1024 /*align*/ + size_t(kStages) * kStage + kStoreBytes + kBarBytes +
                                  sizeof(int32_t) * (kMaxExperts + 1) + sizeof(float) * 128;
};

static_assert(kStageBytes % 1024 == 0, "stage must keep 1024-byte alignment for 128B swizzle");
static_assert(Cfg<0>::kSmem <= 232448 && Cfg<1>::kSmem <= 232448 && Cfg<2>::kSmem <= 232448 && Cfg<3>::kSmem <= 232448,
              "shared memory");
static_assert(Cfg<0, true>::kSmem <= 232448 && Cfg<1, true>::kSmem <= 232448, "shared memory (solo)");
static_assert(Cfg<4>::kSmem <= 232448, "shared memory (mode 4)");
static_assert(Cfg<0, true>::kStage % 1024 == 0, "solo stage alignment");
static_assert(kSfCol0 + Cfg<0, true>::kStages * kSfColsPerStage <= kTmemCols, "TMEM budget (solo)");
static_assert(kSfCol0 + Cfg<0>::kStages * kSfColsPerStage <= kTmemCols, "TMEM budget");
static_assert(8 * (3 * Cfg<0>::kStages + 2) + 4 <= kBarBytes, "barrier area");
static_assert(8 * (3 * Cfg<4>::kStages + 3) + 8 * 8 <= kBarBytes, "barrier area (mode 4 quarter barriers)");
static_assert(kSegRows == 2 * kBM, "a CTA pair covers one 256-row segment block");

struct TileCoord {
  int e, pm, nt;
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

template <int MODE, bool SOLO>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    grouped_gemm_fp4_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                            const __grid_constant__ CUtensorMap tmap_y, const __grid_constant__ CUtensorMap tmap_sfa,
                            GemmArgs args) {
  using C_ = Cfg<MODE, SOLO>;
  constexpr int S = C_::kStages;
  constexpr uint32_t kStageBytes = C_::kStage, kOffSFA = C_::kOffSfa, kOffSFB = C_::kOffSfb;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base - raw_addr);
  const uint32_t store_base = base + S * kStageBytes;  // MODE 1 / 3 output staging (1024-aligned)
  const uint32_t bar_base = store_base + C_::kStoreBytes;
  // full: even CTA only; A/B bytes of both CTAs plus the scale writers of both
  // CTAs (their TMEM scales are in place), so the MMA issuer waits once per stage.
  auto full_bar = [&](int s) { return bar_base + 8u * s; };
  auto sfull_bar = [&](int s) { return bar_base + 8u * (S + s); };       // own scale bytes landed
  auto empty_bar = [&](int s) { return bar_base + 8u * (2 * S + s); };   // stage consumed by the pair MMA
  const uint32_t tfull_bar = bar_base + 8u * (3 * S);       // accumulator ready (both CTAs)
  const uint32_t tempty_bar = bar_base + 8u * (3 * S + 1);  // even CTA: both epilogues read it
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + (bar_base - base) + 8 * (3 * S + 2));
  // MODE 4: per lane quarter, "the four column warps staged their h" and "... wrote it out"
  auto h4_staged = [&](int q) { return bar_base + 8u * (3 * S + 3 + q); };
  auto h4_drained = [&](int q) { return bar_base + 8u * (3 * S + 7 + q); };
  int32_t* pad_s = reinterpret_cast<int32_t*>(smem + (bar_base - base) + kBarBytes);
  float* s_inv = reinterpret_cast<float*>(pad_s + kMaxExperts + 1);  // 1/decoded scale per E4M3 code

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int E = args.E;
  const uint32_t rank = SOLO ? 0u : cluster_ctarank();
  const bool leader = rank == 0;
  // work unit: a CTA pair, or (SOLO) a single CTA
  const int pair = SOLO ? int(blockIdx.x) : int(cluster_id_x());
  const int npairs = SOLO ? int(gridDim.x) : int(cluster_count_x());

  constexpr bool kGateUp = MODE == 0 || MODE == 3 || MODE == 4;
  if (kGateUp && tid < 128) s_inv[tid] = inverse_decoding(e4m3_to_f32(uint32_t(tid)));
  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full_bar(s), 1 + (SOLO ? 1 : 2) * kSfWarps);
      mbar_init(sfull_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    mbar_init(tfull_bar, 1);
    mbar_init(tempty_bar, (SOLO ? 1 : 2) * kEpiWarps);
    if (MODE == 4)
      for (int q = 0; q < 4; ++q) {
        mbar_init(h4_staged(q), 4);
        mbar_init(h4_drained(q), 4);
      }
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmap_a);
    prefetch_tmap(&tmap_b);
    if (MODE == 1 || MODE == 3) prefetch_tmap(&tmap_y);
    if (args.a_sf_rowmajor) prefetch_tmap(&tmap_sfa);
  }
  if (warp == 1) {
    if (SOLO) {
      tmem_alloc(smem_u32(tmem_slot), kTmemCols);
      tmem_relinquish();
    } else {
      tmem_alloc_pair(smem_u32(tmem_slot), kTmemCols);
      tmem_relinquish_pair();
    }
  }
  // Everything above is independent of the previous kernel's output; from here on
  // its writes (expert layout, A operand) are read.
  pdl_wait();
  for (int i = tid; i <= E; i += kThreads) pad_s[i] = args.pad_start[i];
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // both CTAs' barriers exist before any cross-CTA arrive or transfer
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  // tile rows: 256-row pair blocks, or (SOLO) 128-row blocks
  const int total_pm = pad_s[E] / (SOLO ? kBM : kSegRows);
  const int n_tiles = args.n_tiles;
  const int total_tiles = total_pm * n_tiles;
  const int kblocks = args.K / kBK;
  const uint32_t sf_row_stride = uint32_t(args.K / 64) * 512u;  // bytes per 128-row scale block
  auto coord = [&](int t) {
    TileCoord c;
    c.pm = t / n_tiles;
    c.nt = t - c.pm * n_tiles;
    c.e = find_expert(pad_s, E, c.pm * (SOLO ? kBM : kSegRows));
    return c;
  };
  // first A row of this CTA's part of the tile
  auto tile_row0 = [&](const TileCoord& c) { return SOLO ? c.pm * kBM : c.pm * kSegRows + int(rank) * kBM; };
  // SOLO skips 128-row blocks that hold only padding rows (every role skips the same tiles)
  auto live = [&](const TileCoord& c) {
    return !SOLO || args.row_count == nullptr || c.pm * kBM - pad_s[c.e] < __ldg(args.row_count + c.e);
  };
  auto b_rows = [&](const TileCoord& c, int& lr0, int& lr1) {  // local B rows of the tile's two 128-row halves
    if (kGateUp) {
      lr0 = c.nt * 128;           // gate rows
      lr1 = args.F + c.nt * 128;  // value rows
    } else {
      lr0 = c.nt * kBN;
      lr1 = lr0 + 128;
    }
  };

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = pair; t < total_tiles && ok; t += npairs) {
        const TileCoord c = coord(t);
        if (!live(c)) continue;
        int lr0, lr1;
        b_rows(c, lr0, lr1);
        const int row0 = tile_row0(c);
        const int brow = c.e * args.N_total + (rank == 0 ? lr0 : lr1);
        const uint8_t* bsc = args.b_scales + size_t(c.e) * (size_t(args.N_total) * args.K / 16);
        const uint8_t* bsc0 = bsc + size_t(lr0 / 128) * sf_row_stride;
        const uint8_t* bsc1 = bsc + size_t(lr1 / 128) * sf_row_stride;
        const uint8_t* asc = args.a_scales + size_t(row0 / 128) * sf_row_stride;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(empty_bar(stage), phase ^ 1u, args.err, 101)) {
            ok = false;
            break;
          }
          const uint32_t st = base + stage * kStageBytes;
          mbar_arrive_expect_tx(sfull_bar(stage), kSFBytes);
          if (SOLO) {  // own A tile and both 128-row halves of the tile's B rows
            mbar_arrive_expect_tx(full_bar(stage), C_::kAB);
            tma_load_2d(st, &tmap_a, kb * (kBK / 2), row0, full_bar(stage));
            tma_load_2d(st + kOffB, &tmap_b, kb * (kBK / 2), c.e * args.N_total + lr0, full_bar(stage));
            tma_load_2d(st + kOffB + kBHalf, &tmap_b, kb * (kBK / 2), c.e * args.N_total + lr1, full_bar(stage));
          } else {
            if (leader) mbar_arrive_expect_tx(full_bar(stage), 2 * kABBytes);
            const uint32_t fb = map_shared_rank(full_bar(stage), 0);
            tma_load_2d_pair(st, &tmap_a, kb * (kBK / 2), row0, fb);
            tma_load_2d_pair(st + kOffB, &tmap_b, kb * (kBK / 2), brow, fb);
          }
          if (args.a_sf_rowmajor)  // this CTA's 128 rows x 16 scales of the K block, row-major
            tma_load_2d(st + kOffSFA, &tmap_sfa, kb * (kBK / 16), row0, sfull_bar(stage));
          else
            bulk_load(st + kOffSFA, asc + kb * 2048, kSFA, sfull_bar(stage));
          bulk_load(st + kOffSFB, bsc0 + kb * 2048, kSFBHalf, sfull_bar(stage));
          bulk_load(st + kOffSFB + kSFBHalf, bsc1 + kb * 2048, kSFBHalf, sfull_bar(stage));
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Drain: wait until the pair MMA released every stage, so that no MMA
      // completion is still on its way to this CTA's barriers at exit.
      for (int i = 0; i < S && ok; ++i) {
        ok = mbar_wait(empty_bar(stage), phase ^ 1u, args.err, 102);
        if (++stage == S) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ pair MMA issuer (even CTA)
    if (leader && lane == 0) {
      // Four epilogue warps share this warp's scheduler, so the issue loop is
      // kept short: descriptors, scale columns and barrier addresses of a stage
      // advance by fixed strides from precomputed stage-0 values.
      const uint64_t adesc0 = smem_desc(base, 16, 1024, 2);
      const uint64_t bdesc0 = smem_desc(base + kOffB, 16, 1024, 2);
      const uint32_t sf0 = tmem_base + kSfCol0;
      const uint32_t empty0_own = map_shared_rank(empty_bar(0), 0), empty0_peer = map_shared_rank(empty_bar(0), 1);
      const uint32_t tfull_own = map_shared_rank(tfull_bar, 0), tfull_peer = map_shared_rank(tfull_bar, 1);
      int stage = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true;
      for (int t = pair; t < total_tiles && ok; t += npairs) {
        if (SOLO && !live(coord(t))) continue;
        if (!mbar_wait(tempty_bar, acc_phase ^ 1u, args.err, 201)) break;
        tc_fence_after();
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(full_bar(stage), phase, args.err, 202)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t adesc = adesc0 + uint64_t(stage) * (kStageBytes >> 4);
          const uint64_t bdesc = bdesc0 + uint64_t(stage) * (kStageBytes >> 4);
          const uint32_t sf_col = sf0 + uint32_t(stage) * kSfColsPerStage;
          if (SOLO) {
#pragma unroll
            for (int ks = 0; ks < 4; ++ks)
              tc_mma_nvf4(tmem_base, adesc + 2 * ks, bdesc + 2 * ks, kIdescSolo, sf_col + 4 * ks, sf_col + 16 + 8 * ks,
                          (kb | ks) != 0 ? 1u : 0u);
            tc_commit(empty_bar(stage));
          } else {
#pragma unroll
            for (int ks = 0; ks < 4; ++ks)
              tc_mma_nvf4_pair(tmem_base, adesc + 2 * ks, bdesc + 2 * ks, kIdesc, sf_col + 4 * ks,
                               sf_col + 16 + 8 * ks, (kb | ks) != 0 ? 1u : 0u);
            tc_commit_pair(empty0_own + 8u * stage);
            tc_commit_pair(empty0_peer + 8u * stage);
          }
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        if (SOLO) {
          tc_commit(tfull_bar);
        } else {
          tc_commit_pair(tfull_own);
          tc_commit_pair(tfull_peer);
        }
        acc_phase ^= 1u;
      }
    }
    __syncwarp();
  } else if (warp < kEpiWarp0) {
    // ------------------------------------------------------------ scale-factor writers (both CTAs)
    // Lane l of quarter q copies bytes [16 l, 16 l + 16) of each 512-byte atom
    // (the 4 scales of rows l, l+32, l+64, l+96) to TMEM lane 32q + l, 4 columns.
    // A stage's TMEM slot is free once the stage's scales have landed again:
    // the producer refills a stage only after the pair MMAs that read it (and
    // its scales in both CTAs) completed.
    const int q = warp & 3;
    const uint32_t lane_base = uint32_t(q * 32) << 16;
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int t = pair; t < total_tiles && ok; t += npairs) {
      if (SOLO && !live(coord(t))) continue;
      for (int kb = 0; kb < kblocks; ++kb) {
        if (!mbar_wait(sfull_bar(stage), phase, args.err, 121)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint8_t* st = smem + stage * kStageBytes;
        const uint32_t sf_col = tmem_base + lane_base + kSfCol0 + stage * kSfColsPerStage;
        // columns [0,16): SFA of K steps 0..3; [16,48): per K step, SFB half 0 then half 1
        uint32_t va[16], vb[32];
        if (args.a_sf_rowmajor) {
          // row-major [128][16] bytes: row l + 32 j holds the 4 scale words of K steps 0..3
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint4 a = *reinterpret_cast<const uint4*>(st + kOffSFA + (lane + 32 * j) * 16);
            va[j] = a.x, va[4 + j] = a.y, va[8 + j] = a.z, va[12 + j] = a.w;
          }
        } else {
#pragma unroll
          for (int ks = 0; ks < 4; ++ks) {
            const uint4 a = *reinterpret_cast<const uint4*>(st + kOffSFA + ks * 512 + lane * 16);
            va[4 * ks] = a.x, va[4 * ks + 1] = a.y, va[4 * ks + 2] = a.z, va[4 * ks + 3] = a.w;
          }
        }
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
          const uint4 b0 = *reinterpret_cast<const uint4*>(st + kOffSFB + ks * 512 + lane * 16);
          const uint4 b1 = *reinterpret_cast<const uint4*>(st + kOffSFB + kSFBHalf + ks * 512 + lane * 16);
          vb[8 * ks] = b0.x, vb[8 * ks + 1] = b0.y, vb[8 * ks + 2] = b0.z, vb[8 * ks + 3] = b0.w;
          vb[8 * ks + 4] = b1.x, vb[8 * ks + 5] = b1.y, vb[8 * ks + 6] = b1.z, vb[8 * ks + 7] = b1.w;
        }
        tmem_st16(sf_col, va);
        tmem_st32(sf_col + 16, vb);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if (SOLO) mbar_arrive(full_bar(stage));
          else mbar_arrive_cluster(map_shared_rank(full_bar(stage), 0));
        }
        if (++stage == S) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    // 16 warps: lane quarter q = warp % 4 (the TMEM lanes a warp may read),
    // column group sub = 0..3 (32 h columns in MODE 0, 64 output columns otherwise).
    const int q = warp & 3;
    const int sub = (warp - kEpiWarp0) >> 2;
    const int row_in_tile = q * 32 + lane;
    const uint32_t lane_addr = tmem_base + (uint32_t(q * 32) << 16);
    const uint32_t tempty_leader = map_shared_rank(tempty_bar, 0);
    const uint32_t my_buf = store_base + uint32_t(warp - kEpiWarp0) * kWarpStoreBytes;
    uint8_t* const h4q = smem + (store_base - base) + uint32_t(q) * kH4Quarter;  // MODE 4 staging
    uint32_t acc_phase = 0, h4_phase = 0;
    bool h4_first = true;
    for (int t = pair; t < total_tiles; t += npairs) {
      const TileCoord c = coord(t);
      if (!live(c)) continue;
      // per-tile scalars first: their load latency overlaps the MMAs of this tile
      const int64_t p = int64_t(tile_row0(c)) + row_in_tile;  // padded row
      const int local = int(p - pad_s[c.e]);
      // acc * (g_a * g_b), the reference's order (src/mcl4_coe/nvfp4.py:869); g_a = 1 unless given
      const float gb = args.a_g != nullptr ? __fmul_rn(__ldg(args.a_g), __ldg(args.b_g + c.e)) : __ldg(args.b_g + c.e);
      const int rows_e = args.row_count ? __ldg(args.row_count + c.e) : (1 << 30);
      const float wrow = (!kGateUp && args.row_w && local < rows_e) ? __ldg(args.row_w + p) : 0.f;
      // MODE 4: destination (rank << 28 | row) of this row's h in its source's layout
      const int32_t hdst = (MODE == 4 && local < rows_e) ? __float_as_int(__ldg(args.row_w + p)) : -1;
      if (!mbar_wait(tfull_bar, acc_phase, args.err, 301)) break;
      acc_phase ^= 1u;
      tc_fence_after();
      uint32_t va[32], vb[32];
      if (kGateUp) {
        tmem_ld32(lane_addr + sub * 32, va);        // gate columns
        tmem_ld32(lane_addr + 128 + sub * 32, vb);  // value columns
      } else {
        tmem_ld32(lane_addr + sub * 64, va);
        tmem_ld32(lane_addr + sub * 64 + 32, vb);
      }
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {  // accumulator may be overwritten now
        if (SOLO) mbar_arrive(tempty_bar);
        else mbar_arrive_cluster(tempty_leader);
      }

      if (kGateUp) {
        // up = bf16(acc * g); h = bf16(bf16(silu(gate)) * value) (src/mcl4_coe/backbone.py:572-574),
        // then NVFP4 with 1x16 row scales (src/mcl4_coe/nvfp4.py:197-225).
        const int F = args.F;
        const int hb0 = c.nt * 8 + sub * 2;  // first 16-column block of h handled here
        uint32_t packed[4];
        uint32_t sword = 0;
        // MODE 3: the warp's 32 x 32 gate and value bf16 blocks go through two 64B-swizzled
        // smem tiles (row = lane, 16-byte chunk c at c ^ ((row >> 1) & 3)) and two TMA stores
        const uint32_t gate_buf = my_buf, val_buf = my_buf + kWarpStoreBytes / 2;
        if (MODE == 3) {
          if (lane == 0) bulk_wait_read_all();  // the previous tile's stores have read these tiles
          __syncwarp();
        }
#pragma unroll
        for (int blk = 0; blk < 2; ++blk) {
          uint32_t hh[8];
          uint32_t gq[4], uq[4];
          uint32_t mx = 0;
          const uint64_t gb2 = f2pack(gb, gb);
#pragma unroll
          for (int pr = 0; pr < 8; ++pr) {
            const int j = blk * 16 + 2 * pr;
            float a0, a1, b0, b1, s0, s1;
            f2unpack(fmul2(f2pack(__uint_as_float(va[j]), __uint_as_float(va[j + 1])), gb2), a0, a1);
            f2unpack(fmul2(f2pack(__uint_as_float(vb[j]), __uint_as_float(vb[j + 1])), gb2), b0, b1);
            const uint32_t gg = pack_bf16x2(a0, a1);
            const uint32_t uu = pack_bf16x2(b0, b1);
            if (MODE == 3) {  // training: the backward's SwiGLU derivative needs gate and value
              gq[pr & 3] = gg;
              uq[pr & 3] = uu;
              if ((pr & 3) == 3) {
                const uint32_t off = uint32_t(lane) * 64u + (uint32_t((blk * 2 + (pr >> 2)) ^ ((lane >> 1) & 3)) << 4);
                st_shared_v4(gate_buf + off, make_uint4(gq[0], gq[1], gq[2], gq[3]));
                st_shared_v4(val_buf + off, make_uint4(uq[0], uq[1], uq[2], uq[3]));
              }
            }
            silu_f32x2(bf16x2_lo(gg), bf16x2_hi(gg), s0, s1);
            hh[pr] = bf16x2_mul(pack_bf16x2(s0, s1), uu);
            mx = bf16x2_max(mx, hh[pr] & 0x7FFF7FFFu);
          }
          // scale = e4m3(min(amax/6, 448)), inv = 1/decoded scale (src/mcl4_coe/nvfp4.py:215-221)
          const uint32_t sc = f32_to_e4m3(fminf(div6_bf16_amax(fmaxf(bf16x2_lo(mx), bf16x2_hi(mx))), 448.0f));
          const float inv = s_inv[sc];
          sword |= sc << (8 * blk);
          const uint64_t inv2 = f2pack(inv, inv);
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            float n[8];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const uint32_t w = hh[half * 4 + i];
              f2unpack(fmul2(f2pack(bf16x2_lo(w), bf16x2_hi(w)), inv2), n[2 * i], n[2 * i + 1]);
            }
            packed[blk * 2 + half] = e2m1x8_act(n);
          }
          if (args.h_dbg != nullptr) {
            uint4* dst = reinterpret_cast<uint4*>(args.h_dbg + p * F + (hb0 + blk) * 16);
            dst[0] = make_uint4(hh[0], hh[1], hh[2], hh[3]);
            dst[1] = make_uint4(hh[4], hh[5], hh[6], hh[7]);
          }
        }
        if (MODE == 3) {
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {  // lane 0 holds the warp's first row
            tma_store_2d(&tmap_y, gate_buf, c.nt * 128 + sub * 32, int(p));
            tma_store_2d(&tmap_y, val_buf, F + c.nt * 128 + sub * 32, int(p));
            bulk_commit_group();
          }
        }
        if (MODE == 4) {
          // expert parallelism: h goes straight to the token's home GPU (peer stores over
          // NVLink into its expert-major layout), where the down projection runs.  The four
          // column warps of this lane quarter first assemble their rows in shared memory, so
          // that each row leaves as one 64-byte run of codes and two 4-byte scale words
          // instead of four 16-byte and four 2-byte stores.
          bool h4_ok = true;
          if (!h4_first) h4_ok = mbar_wait(h4_drained(q), h4_phase ^ 1u, args.err, 331);  // previous tile out
          *reinterpret_cast<uint4*>(h4q + kH4Codes + lane * 64 + sub * 16) =
              make_uint4(packed[0], packed[1], packed[2], packed[3]);
          *reinterpret_cast<uint16_t*>(h4q + kH4Scales + lane * 8 + sub * 2) = uint16_t(sword);
          if (sub == 0) *reinterpret_cast<int32_t*>(h4q + kH4Dst + lane * 4) = hdst;
          __syncwarp();
          if (lane == 0) mbar_arrive(h4_staged(q));
          h4_ok = mbar_wait(h4_staged(q), h4_phase, args.err, 332) && h4_ok;
          if (!h4_ok) break;
          {
            const int i = sub * 32 + lane;  // one 16-byte piece of the 32 rows' codes per thread
            const int r = i >> 2, ch = i & 3;
            const int32_t dst = *reinterpret_cast<const int32_t*>(h4q + kH4Dst + r * 4);
            if (dst >= 0)
              *reinterpret_cast<uint4*>(args.peer_hq[dst >> 28] + uint64_t(dst & 0x0FFFFFFF) * (F / 2) + c.nt * 64 +
                                        ch * 16) = *reinterpret_cast<const uint4*>(h4q + kH4Codes + r * 64 + ch * 16);
            if (i < 64) {  // the 8 scales of a row: blocks nt*8 .. nt*8+3 and nt*8+4 .. nt*8+7, one word each
              const int rr = i >> 1, w = i & 1;
              const int32_t d2 = *reinterpret_cast<const int32_t*>(h4q + kH4Dst + rr * 4);
              if (d2 >= 0)
                *reinterpret_cast<uint32_t*>(args.peer_hs[d2 >> 28] +
                                             swizzled_scale_offset(uint64_t(d2 & 0x0FFFFFFF), uint32_t(c.nt * 8 + 4 * w),
                                                                   uint32_t(F / 16))) =
                    *reinterpret_cast<const uint32_t*>(h4q + kH4Scales + rr * 8 + w * 4);
            }
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(h4_drained(q));
          h4_phase ^= 1u;
          h4_first = false;
        } else {
          *reinterpret_cast<uint4*>(args.hq + p * (F / 2) + hb0 * 8) =
              make_uint4(packed[0], packed[1], packed[2], packed[3]);
          *reinterpret_cast<uint16_t*>(args.hs +
                                       swizzled_scale_offset(uint64_t(p), uint32_t(hb0), uint32_t(F / 16))) =
              uint16_t(sword);
        }
      } else if (MODE == 1 && !SOLO) {
        // y = bf16(acc * g) [* bf16(routing weight), rounded to bf16] (src/mcl4_coe/backbone.py:903),
        // every padded row (padding rows hold zeros), through a 32 x 64 swizzled smem tile.
        const uint32_t ww = pack_bf16x2(wrow, wrow);
        if (lane == 0) bulk_wait_read_all();  // the previous tile's store has read this buffer
        __syncwarp();
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const uint32_t* src = i < 4 ? va + 8 * i : vb + 8 * (i - 4);
          uint32_t o[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint32_t yy = pack_bf16x2(__uint_as_float(src[2 * j]) * gb, __uint_as_float(src[2 * j + 1]) * gb);
            o[j] = args.row_w ? bf16x2_mul(yy, ww) : yy;
          }
          st_shared_v4(my_buf + uint32_t(lane) * 128u + (uint32_t(i ^ (lane & 7)) << 4),
                       make_uint4(o[0], o[1], o[2], o[3]));
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(&tmap_y, my_buf, c.nt * kBN + sub * 64, int(p));  // lane 0 holds the warp's first row
          bulk_commit_group();
        }
      } else if (local < rows_e && args.y32 != nullptr) {
        // fp32 rows acc * g [+ bias] into unpadded destination rows (single-matrix
        // NVFP4 GEMM, src/mcl4_coe/nvfp4.py:318-334 and :425-427): product and sum
        // rounded separately, as the reference's scaled_mm result + bias
        const int64_t dst_row = args.out_row_base ? int64_t(args.out_row_base[c.e]) + local : p;
        const int col0 = c.nt * kBN + sub * 64;
        float4* dst = reinterpret_cast<float4*>(args.y32 + dst_row * args.ldy + col0);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const uint32_t* src = i < 8 ? va + 4 * i : vb + 4 * (i - 8);
          float o[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            o[j] = __fmul_rn(__uint_as_float(src[j]), gb);
            if (args.bias) o[j] = __fadd_rn(o[j], __ldg(args.bias + col0 + 4 * i + j));
          }
          dst[i] = make_float4(o[0], o[1], o[2], o[3]);
        }
      } else if (local < rows_e) {
        // y rows into unpadded destination rows (or, SOLO, their padded rows), valid rows only
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
    if ((MODE == 1 || MODE == 3) && lane == 0) bulk_wait_all();
  }

  pdl_trigger();  // the next kernel may launch; it waits for this grid's writes
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // no pair MMA or peer access is outstanding past this point
  if (warp == 1) {
    tc_fence_after();
    if (SOLO) tmem_dealloc(tmem_base, kTmemCols);
    else tmem_dealloc_pair(tmem_base, kTmemCols);
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

// 2-D map over row-major A scales [rows, K/16] (bytes), box 16 scales (one K block) x 128 rows,
// no swizzle: the x coordinate is a multiple of 16 bytes and the row stride K/16 a multiple of 16.
bool make_tmap_scales(CUtensorMap* m, const void* base, uint64_t cols, uint64_t rows) {
  auto fn = encode_fn();
  if (!fn || cols % 16 != 0) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols};
  cuuint32_t box[2] = {16, 128};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 2-D map over a bf16 [rows, ld] matrix, box 64 columns (128 bytes) x 32 rows, 128B swizzle (tile stores).
bool make_tmap_store(CUtensorMap* m, const void* base, uint64_t ld, uint64_t rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {ld, rows};
  cuuint64_t strides[1] = {ld * 2};
  cuuint32_t box[2] = {64, 32};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 2-D map over the training save gate | value (bf16 [rows, 2F]), box 32 columns x 32 rows,
// 64B swizzle: one epilogue warp's gate or value block.
bool make_tmap_up_save(CUtensorMap* m, const void* base, uint64_t cols, uint64_t rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * 2};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Number of CTA pairs that can be resident at once (one CTA per SM).
template <int MODE, bool SOLO>
int resident_pairs() {
  static int n = 0;
  if (n == 0) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * 74);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = Cfg<MODE, SOLO>::kSmem;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, grouped_gemm_fp4_kernel<MODE, SOLO>, &cfg) != cudaSuccess ||
        clusters <= 0) {
      (void)cudaGetLastError();
      clusters = num_sms() / 2;
    }
    n = clusters;
  }
  return n;
}

template <int MODE, bool SOLO = false>
int launch_mode(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& ty, const CUtensorMap& tsa,
                const GemmArgs& args, cudaStream_t stream) {
  static std::atomic<uint64_t> configured{0};
  if (!raise_smem_limit(grouped_gemm_fp4_kernel<MODE, SOLO>, int(Cfg<MODE, SOLO>::kSmem), configured))
    return MCL4MOE_ERR_CUDA;
  const int pairs = resident_pairs<MODE, SOLO>();
  return launch_pdl(grouped_gemm_fp4_kernel<MODE, SOLO>, dim3(2 * pairs), dim3(kThreads), Cfg<MODE, SOLO>::kSmem,
                    stream, ta, tb, ty, tsa, args) == cudaSuccess
             ? MCL4MOE_OK
             : MCL4MOE_ERR_CUDA;
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
  if (a_rows % kSegRows != 0) return MCL4MOE_ERR_INVALID;
  if ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) | reinterpret_cast<uintptr_t>(args.a_scales) |
       reinterpret_cast<uintptr_t>(args.b_scales)) & 15)
    return MCL4MOE_ERR_INVALID;
  CUtensorMap ta, tb, ty, tsa;
  if (!make_tmap(&ta, a, uint64_t(args.K) / 2, uint64_t(a_rows))) return MCL4MOE_ERR_CUDA;
  if (!make_tmap(&tb, b, uint64_t(args.K) / 2, uint64_t(args.E) * args.N_total)) return MCL4MOE_ERR_CUDA;
  memset(&tsa, 0, sizeof(tsa));
  if (args.a_sf_rowmajor && !make_tmap_scales(&tsa, args.a_scales, uint64_t(args.K) / 16, uint64_t(a_rows)))
    return MCL4MOE_ERR_CUDA;
  if (args.mode == 4) {  // gate/up with h stored into the rows' home GPUs
    memset(&ty, 0, sizeof(ty));
    if (args.row_w == nullptr || args.row_count == nullptr || args.F % 128 != 0) return MCL4MOE_ERR_INVALID;
    return launch_mode<4>(ta, tb, ty, tsa, args, stream);
  }
  if (args.mode == 0) {
    memset(&ty, 0, sizeof(ty));
    if (args.up_save == nullptr)
      return args.solo ? launch_mode<0, true>(ta, tb, ty, tsa, args, stream) : launch_mode<0>(ta, tb, ty, tsa, args, stream);
    // MODE 3: the same gate/up kernel that also stores gate | value for the backward
    if ((reinterpret_cast<uintptr_t>(args.up_save) & 15) || args.F % 128 != 0) return MCL4MOE_ERR_INVALID;
    if (!make_tmap_up_save(&ty, args.up_save, 2 * uint64_t(args.F), uint64_t(a_rows))) return MCL4MOE_ERR_CUDA;
    return launch_mode<3>(ta, tb, ty, tsa, args, stream);
  }
  if (args.out_row_base == nullptr && args.solo && args.row_count != nullptr) {
    // SOLO: valid rows only, plain stores
    if ((reinterpret_cast<uintptr_t>(args.y) & 15) || (args.ldy * 2) % 16 != 0) return MCL4MOE_ERR_INVALID;
    memset(&ty, 0, sizeof(ty));
    return launch_mode<1, true>(ta, tb, ty, tsa, args, stream);
  }
  if (args.out_row_base == nullptr) {
    // Tile stores write every padded row: y holds a_rows rows of ldy elements.
    if ((reinterpret_cast<uintptr_t>(args.y) & 15) || (args.ldy * 2) % 16 != 0) return MCL4MOE_ERR_INVALID;
    if (!make_tmap_store(&ty, args.y, uint64_t(args.ldy), uint64_t(a_rows))) return MCL4MOE_ERR_CUDA;
    return launch_mode<1>(ta, tb, ty, tsa, args, stream);
  }
  memset(&ty, 0, sizeof(ty));
  return launch_mode<2>(ta, tb, ty, tsa, args, stream);
}

}  // namespace mcl4
