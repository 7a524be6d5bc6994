// Expert weight gradients of the grouped projections on the 5th-generation
// tensor cores: dW[e] = G[seg e]^T X[seg e] in float32, for every expert e, with
// G (the projection's output gradient) and X (its input) bf16 row-major over the
// padded expert-major rows of the forward.  Replaces the reference's Triton
// _grouped_wgrad_kernel (src/mcl4_coe/nvfp4.py:877-920: bf16 operands, fp32
// accumulation, one [N, K] result per expert, zero for an expert without rows).
//
// The reduction runs over rows, the row-major operands' strided dimension, so both
// operands enter the MMA "MN-major": a TMA box of 64 columns x 64 rows lands as
// 64 rows of 128 bytes (128-byte swizzle), which is the canonical MN-major SW128
// layout (64 contiguous M/N elements per row, 8-row groups 1024 bytes apart, the
// next 64 M/N elements one box further: LBO = box bytes, SBO = 1024).
//
// Tiles: 128 rows of dW (columns of G) x 256 columns (columns of X), one CTA per
// SM (tcgen05 kind::f16, M = 128, N = 256, K = 16 per MMA), persistent over
// (expert, row block, column block); each tile walks its expert's segment in
// 64-row stages (segments are multiples of 256 rows; their padding rows are zero
// in G, so they add nothing).  Warp 0: TMA producer; warp 1: TMEM owner and MMA
// issuer; warps 2..5: epilogue (TMEM -> fp32 rows of dW).  Every wait is bounded.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "kernels.cuh"

namespace mcl4 {

namespace {

constexpr int kWBM = 128;  // rows of dW per tile (columns of G)
constexpr int kWBN = 256;  // columns of dW per tile (columns of X)
constexpr int kWBR = 64;   // reduction rows per stage
constexpr uint32_t kWBox = 64 * kWBR * 2;             // one 64-column box: 8192 bytes
constexpr uint32_t kWABytes = (kWBM / 64) * kWBox;    // 16384
constexpr uint32_t kWBBytes = (kWBN / 64) * kWBox;    // 32768
constexpr uint32_t kWStage = kWABytes + kWBBytes;     // 49152
constexpr int kWStages = 4;
constexpr int kWThreads = 192;
constexpr size_t kWSmem = 1024 + size_t(kWStages) * kWStage + 256;
// kind::f16: fp32 accumulator, bf16 A and B, both MN-major, N = 256, M = 128
constexpr uint32_t kWIdesc =
    (1u << 4) | (1u << 7) | (1u << 10) | (1u << 15) | (1u << 16) | ((256u >> 3) << 17) | ((128u >> 4) << 24);
static_assert(kWStage % 1024 == 0, "stages keep the 1024-byte alignment of the 128-byte swizzle");

}  // namespace

struct WgradArgs {
  const int32_t* pad_start;  // [E + 1]
  int E, N, K;
  float* dw;                 // [E, N, K]
  int32_t* err;
};

__global__ void __launch_bounds__(kWThreads, 1)
    wgrad_kernel(const __grid_constant__ CUtensorMap tmap_g, const __grid_constant__ CUtensorMap tmap_x, WgradArgs a) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base - raw_addr);
  const uint32_t bar_base = base + kWStages * kWStage;
  auto full_bar = [&](int s) { return bar_base + 8u * s; };
  auto empty_bar = [&](int s) { return bar_base + 8u * (kWStages + s); };
  const uint32_t tfull_bar = bar_base + 8u * (2 * kWStages);
  const uint32_t tempty_bar = bar_base + 8u * (2 * kWStages + 1);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + (bar_base - base) + 8 * (2 * kWStages + 2));

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int s = 0; s < kWStages; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    mbar_init(tfull_bar, 1);
    mbar_init(tempty_bar, 4);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int nb_n = a.N / kWBM, nb_k = a.K / kWBN;
  const int per_e = nb_n * nb_k;
  const int total = a.E * per_e;
  auto tile = [&](int t, int& e, int& n0, int& k0, int& r0, int& steps) {
    e = t / per_e;
    const int r = t - e * per_e;
    n0 = (r / nb_k) * kWBM;
    k0 = (r % nb_k) * kWBN;
    r0 = __ldg(a.pad_start + e);
    steps = (__ldg(a.pad_start + e + 1) - r0) / kWBR;
  };

  if (warp == 0) {
    if (lane == 0) {  // ---------------------------------------------------- TMA producer
      prefetch_tmap(&tmap_g);
      prefetch_tmap(&tmap_x);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
        int e, n0, k0, r0, steps;
        tile(t, e, n0, k0, r0, steps);
        for (int s = 0; s < steps; ++s) {
          if (!mbar_wait(empty_bar(stage), phase ^ 1u, a.err, 131)) {
            ok = false;
            break;
          }
          const uint32_t st = base + stage * kWStage;
          mbar_arrive_expect_tx(full_bar(stage), kWStage);
#pragma unroll
          for (int j = 0; j < kWBM / 64; ++j)
            tma_load_2d(st + j * kWBox, &tmap_g, n0 + 64 * j, r0 + s * kWBR, full_bar(stage));
#pragma unroll
          for (int j = 0; j < kWBN / 64; ++j)
            tma_load_2d(st + kWABytes + j * kWBox, &tmap_x, k0 + 64 * j, r0 + s * kWBR, full_bar(stage));
          if (++stage == kWStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {  // ---------------------------------------------------- MMA issuer
      int stage = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
        int e, n0, k0, r0, steps;
        tile(t, e, n0, k0, r0, steps);
        if (!mbar_wait(tempty_bar, acc_phase ^ 1u, a.err, 231)) break;
        tc_fence_after();
        for (int s = 0; s < steps; ++s) {
          if (!mbar_wait(full_bar(stage), phase, a.err, 232)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t st = base + stage * kWStage;
#pragma unroll
          for (int ks = 0; ks < kWBR / 16; ++ks)  // 16 reduction rows per MMA = two 8-row groups
            tc_mma_f16(tmem_base, smem_desc(st + ks * 2048, kWBox, 1024, 2),
                       smem_desc(st + kWABytes + ks * 2048, kWBox, 1024, 2), kWIdesc, (s | ks) != 0 ? 1u : 0u);
          tc_commit(empty_bar(stage));
          if (++stage == kWStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        tc_commit(tfull_bar);  // with no MMA issued (an empty segment) it arrives at once
        acc_phase ^= 1u;
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ epilogue
    const int q = warp & 3;  // warps 2..5 -> TMEM lane quarters 2, 3, 0, 1
    const int row = q * 32 + lane;
    const uint32_t lane_addr = tmem_base + (uint32_t(q * 32) << 16);
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x) {
      int e, n0, k0, r0, steps;
      tile(t, e, n0, k0, r0, steps);
      if (!mbar_wait(tfull_bar, acc_phase, a.err, 331)) break;
      acc_phase ^= 1u;
      tc_fence_after();
      float* dst = a.dw + (int64_t(e) * a.N + n0 + row) * a.K + k0;
#pragma unroll 1
      for (int c = 0; c < kWBN / 32; ++c) {
        uint32_t v[32];
        tmem_ld32(lane_addr + c * 32, v);
        tmem_wait_ld();
        float4* d4 = reinterpret_cast<float4*>(dst + c * 32);
#pragma unroll
        for (int i = 0; i < 8; ++i)
          d4[i] = steps > 0 ? make_float4(__uint_as_float(v[4 * i]), __uint_as_float(v[4 * i + 1]),
                                          __uint_as_float(v[4 * i + 2]), __uint_as_float(v[4 * i + 3]))
                            : make_float4(0.f, 0.f, 0.f, 0.f);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty_bar);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 256);
  }
}

namespace {

PFN_cuTensorMapEncodeTiled_v12000 wgrad_encode_fn() {
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

// bf16 [rows, cols] row-major, box 64 columns (128 bytes) x 64 rows, 128-byte swizzle.
bool make_tmap_rows(CUtensorMap* m, const void* ptr, uint64_t cols, uint64_t rows) {
  auto fn = wgrad_encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * 2};
  cuuint32_t box[2] = {64, uint32_t(kWBR)};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

int launch_wgrad(const uint16_t* g, const uint16_t* x, int64_t rows, int N, int K, const int32_t* pad_start, int E,
                 float* dw, int32_t* err, cudaStream_t stream) {
  if (N % kWBM != 0 || K % kWBN != 0 || rows % kWBR != 0 || E < 1) return MCL4MOE_ERR_UNSUPPORTED;
  CUtensorMap tg, tx;
  if (!make_tmap_rows(&tg, g, uint64_t(N), uint64_t(rows)) || !make_tmap_rows(&tx, x, uint64_t(K), uint64_t(rows)))
    return MCL4MOE_ERR_CUDA;
  static std::atomic<uint64_t> configured{0};
  if (!raise_smem_limit(wgrad_kernel, int(kWSmem), configured)) return MCL4MOE_ERR_CUDA;
  const int64_t tiles = int64_t(E) * (N / kWBM) * (K / kWBN);
  const int grid = int(tiles < num_sms() ? tiles : num_sms());
  WgradArgs a{pad_start, E, N, K, dw, err};
  wgrad_kernel<<<grid, kWThreads, kWSmem, stream>>>(tg, tx, a);
  return cudaGetLastError() == cudaSuccess ? MCL4MOE_OK : MCL4MOE_ERR_CUDA;
}

}  // namespace mcl4
