// Shared device helpers for the NVFP4 MoE kernels (sm_100a only).
//
// Numerics follow the reference quantiser (src/mcl4_coe/nvfp4.py:186-225 and
// :923-952) operation by operation: every multiply / add / divide is an IEEE
// float32 round-to-nearest operation (explicit __fmul_rn / __fadd_rn /
// __fdiv_rn / __frcp_rn so the compiler cannot contract or approximate), and
// the library is built without fast-math so denormals are kept.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>

#include "../../include/mcl4moe.h"

namespace mcl4 {

constexpr float kFltMax = 3.402823466e38f;
constexpr float kFltMinNormal = 1.17549435e-38f;

// ---------------------------------------------------------------- numerics

__device__ __forceinline__ float bf16_to_f32(uint16_t b) {
  return __uint_as_float(static_cast<uint32_t>(b) << 16);
}

// float32 -> bfloat16 bits, round to nearest even (torch ``.to(bfloat16)``).
__device__ __forceinline__ uint16_t f32_to_bf16(float f) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}

__device__ __forceinline__ float round_bf16(float f) { return bf16_to_f32(f32_to_bf16(f)); }

// float32 in [0, 448] -> e4m3fn bits with round-to-nearest-even (the hardware
// cvt.rn.satfinite conversion; the callers clamp to 448 first, exactly as
// src/mcl4_coe/nvfp4.py:215 does, so saturation never differs from torch).
__device__ __forceinline__ uint32_t f32_to_e4m3(float v) {
  return static_cast<uint32_t>(__nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3));
}

// e4m3fn bits (sign bit clear) -> float32, exact.
__device__ __forceinline__ float e4m3_to_f32(uint32_t c) {
  uint32_t e = (c >> 3) & 0xF, m = c & 7;
  if (e == 0) return __fmul_rn(static_cast<float>(m), 0.001953125f);  // m * 2^-9
  return __uint_as_float(((e + 120u) << 23) | (m << 20));
}

// src/mcl4_coe/nvfp4.py:217-221 — 1/dec clamped to FLT_MAX, 0 when dec <= 0.
__device__ __forceinline__ float inverse_decoding(float dec) {
  return dec > 0.f ? fminf(__frcp_rn(dec), kFltMax) : 0.f;
}

// src/mcl4_coe/nvfp4.py:186-194 (deterministic branch): m = min(|v|, 6);
// u = 2m | m+2 | m/2+4 (each float32-rounded); code = rint(u) | signbit<<3.
__device__ __forceinline__ uint32_t e2m1_code(float v) {
  const float m = fminf(fabsf(v), 6.0f);
  float u;
  if (m <= 2.0f) u = __fmul_rn(m, 2.0f);
  else if (m <= 4.0f) u = __fadd_rn(m, 2.0f);
  else u = __fadd_rn(__fmul_rn(m, 0.5f), 4.0f);
  return static_cast<uint32_t>(__float2int_rn(u)) | ((__float_as_uint(v) >> 31) << 3);
}

// Quantise one 16-element row block with global scale 1 (the activation mode,
// src/mcl4_coe/nvfp4.py:204-224 with causal_row_scale=True):
// returns the e4m3 scale byte; writes the 8 packed bytes (low nibble = even).
__device__ __forceinline__ uint32_t quantize_block16(const float (&v)[16], uint2& packed) {
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(v[i]));
  const uint32_t s = f32_to_e4m3(fminf(__fdiv_rn(amax, 6.0f), 448.0f));
  const float inv = inverse_decoding(e4m3_to_f32(s));
  uint32_t lo = 0, hi = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) lo |= e2m1_code(__fmul_rn(v[i], inv)) << (4 * i);
#pragma unroll
  for (int i = 0; i < 8; ++i) hi |= e2m1_code(__fmul_rn(v[8 + i], inv)) << (4 * i);
  packed = make_uint2(lo, hi);
  return s;
}

// ---- packed bf16x2 helpers (low half = even element)
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ float bf16x2_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16x2_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
// Exact: the product of two bf16 values fits in float32, rounded once to bf16 (RN).
__device__ __forceinline__ uint32_t bf16x2_mul(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t bf16x2_max(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("max.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

// ---- packed float32 pairs (sm_100 f32x2: two independent IEEE round-to-nearest ops)
__device__ __forceinline__ uint64_t f2pack(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void f2unpack(uint64_t v, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t fmul2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}

// amax / 6 correctly rounded to float32 for any non-negative finite bfloat16
// amax: product with RN(1/6) followed by one Markstein correction step
// (remainder by fma, then fma with the reciprocal).  Checked exhaustively against
// the exact quotient over all 32640 such inputs.
__device__ __forceinline__ float div6_bf16_amax(float a) {
  const float r = 0.16666667163372039794921875f;  // RN(1/6)
  const float q0 = __fmul_rn(a, r);
  const float e = __fmaf_rn(-6.0f, q0, a);
  return __fmaf_rn(e, r, q0);
}

// SiLU of two bf16-rounded gate values, g / (1 + 2^(-g log2 e)), with the hardware
// exp2 and reciprocal approximations (a few float32 ulps); the multiplies and adds
// run as packed pairs.
__device__ __forceinline__ void silu_f32x2(float g0, float g1, float& s0, float& s1) {
  const uint64_t gg = f2pack(g0, g1);
  float t0, t1, e0, e1, d0, d1, r0, r1;
  f2unpack(fmul2(gg, f2pack(-1.4426950408889634f, -1.4426950408889634f)), t0, t1);
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e0) : "f"(t0));
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e1) : "f"(t1));
  f2unpack(fadd2(f2pack(e0, e1), f2pack(1.0f, 1.0f)), d0, d1);
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r0) : "f"(d0));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r1) : "f"(d1));
  f2unpack(fmul2(gg, f2pack(r0, r1)), s0, s1);
}

// 8 float32 values -> 8 E2M1 nibbles (element 0 in the low nibble) with the
// reference's rounding, for products of a bfloat16 value and a global-scale-1
// inverse block scale.  The hardware conversion rounds to nearest-even on the
// E2M1 grid; the reference (src/mcl4_coe/nvfp4.py:188-193) rounds u = m+2 or
// u = m/2+4 to float32 first, which differs only at |n| = 2.5+2^-22,
// 5+2^-21 (reference one code lower) and 3.5-2^-22 (one code higher).  The
// third value is not reachable from bf16 inputs (checked exhaustively over
// every bf16 value and e4m3 scale), the first two are corrected here.
__device__ __forceinline__ uint32_t e2m1x8_act(const float (&n)[8]) {
  uint32_t w;
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b0, %2, %1;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b1, %4, %3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b2, %6, %5;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b3, %8, %7;\n\t"
      "mov.b32 %0, {b0, b1, b2, b3};\n\t}"
      : "=r"(w)
      : "f"(n[0]), "f"(n[1]), "f"(n[2]), "f"(n[3]), "f"(n[4]), "f"(n[5]), "f"(n[6]), "f"(n[7]));
  // One test for all eight values first (the fix-up is rare): min over the XOR
  // with the pattern is zero exactly when some value matches.
  uint32_t hit = 0xFFFFFFFFu;
#pragma unroll
  for (int i = 0; i < 8; ++i) hit = min(hit, (__float_as_uint(n[i]) & 0x7F7FFFFFu) ^ 0x40200001u);
  if (hit != 0u) return w;
  uint32_t fix = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) fix |= ((__float_as_uint(n[i]) & 0x7F7FFFFFu) == 0x40200001u ? 1u : 0u) << (4 * i);
  return w - fix;
}

// 1 / decoded value of every non-negative E4M3 code (inverse_decoding of
// e4m3_to_f32), filled by the block's threads; callers sync before use.
__device__ __forceinline__ void fill_inverse_scale_table(float* t) {
  for (int i = threadIdx.x; i < 128; i += blockDim.x) t[i] = inverse_decoding(e4m3_to_f32(uint32_t(i)));
}

// Quantise 16 bf16 values (8 packed words) of one activation block; ``inv_tab``
// is a table from fill_inverse_scale_table.  Bytes of src/mcl4_coe/nvfp4.py:215-224
// (s = e4m3(min(amax/6, 448)), inv = min(1/dec, FLT_MAX), codes of x*inv): amax of
// bf16 values is itself a bf16 value, so div6_bf16_amax is the exact quotient, and
// the table holds the exact inverses.
__device__ __forceinline__ uint32_t quantize_block16_bf16(const uint32_t (&w)[8], uint2& packed,
                                                          const float* inv_tab) {
  uint32_t mx = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) mx = bf16x2_max(mx, w[i] & 0x7FFF7FFFu);
  const uint32_t s = f32_to_e4m3(fminf(div6_bf16_amax(fmaxf(bf16x2_lo(mx), bf16x2_hi(mx))), 448.0f));
  const float inv = inv_tab[s];
  const uint64_t inv2 = f2pack(inv, inv);
  float n[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) f2unpack(fmul2(f2pack(bf16x2_lo(w[i]), bf16x2_hi(w[i])), inv2), n[2 * i], n[2 * i + 1]);
  packed.x = e2m1x8_act(n);
#pragma unroll
  for (int i = 0; i < 4; ++i)
    f2unpack(fmul2(f2pack(bf16x2_lo(w[4 + i]), bf16x2_hi(w[4 + i])), inv2), n[2 * i], n[2 * i + 1]);
  packed.y = e2m1x8_act(n);
  return s;
}


// Byte offset of scale (row r, 16-block c) in the 128x4 scale atoms
// (src/mcl4_coe/nvfp4.py:131-144; the layout tcgen05 block-scaled MMA reads).
__device__ __host__ __forceinline__ uint64_t swizzled_scale_offset(uint64_t r, uint32_t c, uint32_t blocks_per_row) {
  const uint64_t atom = (r >> 7) * (blocks_per_row >> 2) + (c >> 2);
  return atom * 512 + (r & 31) * 16 + ((r >> 5) & 3) * 4 + (c & 3);
}

// Byte offset of scale (row r, 16-block c) in the row-major layout [rows, blocks_per_row]:
// the A-operand scales of the grouped GEMMs' first projection (a row's scales are
// contiguous, so a token's scatter writes them in whole sectors; the GEMM fetches a
// stage's 128 rows x 16 scales with one 2-D TMA load).
__device__ __host__ __forceinline__ uint64_t rowmajor_scale_offset(uint64_t r, uint32_t c, uint32_t blocks_per_row) {
  return r * blocks_per_row + c;
}

// ---------------------------------------------------------------- PTX wrappers

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(bar),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for phase ``parity`` of an mbarrier, giving up after ``kWaitLimitNs``:
// on time-out the error word gets ``code`` (first writer wins) and false is
// returned, so no kernel can spin forever on a barrier nobody completes.
constexpr uint64_t kWaitLimitNs = 1000ull * 1000ull * 1000ull;  // 1 s

__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, int32_t* err, int32_t code) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  uint32_t spins = 0;
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((++spins & 63u) == 0) {
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        if (err) atomicCAS(err, 0, code);
        return false;
      }
      if (err && *reinterpret_cast<volatile int32_t*>(err) != 0) return false;  // another role gave up
    }
  }
}

// 2-D TMA tile load into this CTA's shared memory, completion counted on ``bar``.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const void* tmap, int32_t x, int32_t y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(tmap), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// Plain bulk copy global -> shared (16-byte aligned, size % 16 == 0).
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}

// ---- tcgen05 (5th-generation tensor core, tensor memory)

__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Arrive on ``bar`` once every tcgen05 operation this thread issued so far has completed.
__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

// Copy one 128-row x 4-scale atom (512 B, no swizzle, 16-B rows, 8-row core
// matrices 128 B apart) from shared memory into 4 TMEM columns, replicated
// over the four 32-lane sub-partitions.
__device__ __forceinline__ void tc_copy_scales(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

// D(tmem) (+)= A(smem) * B(smem)^T with NVFP4 operands and UE4M3 scales per 16 K.
__device__ __forceinline__ void tc_mma_nvf4(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t sfa_tmem, uint32_t sfb_tmem, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.scale_vec::4X [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
      : "memory");
}

// D(tmem) (+)= A(smem) * B(smem)^T, 16-bit inputs (kind::f16), fp32 accumulate.
__device__ __forceinline__ void tc_mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns -> 32 registers per thread.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

// 32 lanes x 16 consecutive 32-bit columns -> 16 registers per thread.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 lanes x 4 consecutive 32-bit columns <- 4 registers per thread.
__device__ __forceinline__ void tmem_st4(uint32_t taddr, uint4 v) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %2, %3, %4};" ::"r"(taddr), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}
// 32 lanes x 16 consecutive 32-bit columns <- 16 registers per thread.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}
// 32 lanes x 32 consecutive 32-bit columns <- 32 registers per thread.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]),
      "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]),
      "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ uint4 ld_nc_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}

// ---- programmatic dependent launch: a kernel launched with launch_pdl may
// start while the previous kernel on the stream finishes; pdl_wait() blocks the
// calling thread until that kernel has completed and its writes are visible (a
// no-op for an ordinary launch); pdl_trigger() lets the next kernel launch early.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---- CTA pairs (cluster of 2): two SMs share one 256-row MMA
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_id_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_count_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}
// Address of the same shared-memory location in CTA ``rank`` of the cluster.
__device__ __forceinline__ uint32_t map_shared_rank(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
// All threads of both CTAs (hardware cluster barrier).
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Arrive on an mbarrier given by its cluster address (own CTA or the peer).
// Default (CTA-scope release) semantics: the barrier orders tcgen05 work through
// the tcgen05 fences around it; a cluster-scope acquire on the waiting side
// costs about half a microsecond per wait.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// 2-D TMA tile load into this CTA's shared memory whose completion is counted
// on an mbarrier of either CTA of the pair (``bar`` is a cluster address).
// Each CTA fetches its own tile.
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const void* tmap, int32_t x, int32_t y,
                                                 uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, "
      "%3}], [%4];" ::"r"(dst),
      "l"(tmap), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// Pair MMA (issued by the even CTA): D rows [0,128) in this CTA's TMEM from this
// CTA's A tile, rows [128,256) in the peer's TMEM from the peer's A tile; B's
// N columns come half from each CTA's B tile; each CTA's TMEM holds its own
// SFA and the full-N SFB at the given columns.
__device__ __forceinline__ void tc_mma_nvf4_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                                 uint32_t sfa_tmem, uint32_t sfb_tmem, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::mxf4nvf4.block_scale.scale_vec::4X [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
      : "memory");
}
// Arrive on the mbarrier at cluster address ``bar`` once the pair MMAs this
// thread issued so far have completed.
__device__ __forceinline__ void tc_commit_pair(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
// ---- TMA stores (shared -> global), bulk-group completion
__device__ __forceinline__ void tma_store_2d(const void* tmap, uint32_t src, int32_t x, int32_t y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%1, %2}], [%3];" ::"l"(tmap),
               "r"(x), "r"(y), "r"(src)
               : "memory");
}
__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

// Shared-memory matrix descriptor (tcgen05 format, version 1).
// layout: 0 = no swizzle, 2 = 128-byte swizzle.
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes, uint32_t layout) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFF);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFF) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFF) << 32;
  d |= 1ull << 46;  // descriptor version for sm_100
  d |= static_cast<uint64_t>(layout & 7) << 61;
  return d;
}

// Instruction descriptor of kind::mxf4nvf4: E2M1 A and B (format 1), K-major
// both, UE4M3 scales, fp32 accumulate, M x N, dense K = 64.
__host__ __device__ constexpr uint32_t idesc_nvf4(uint32_t m, uint32_t n) {
  return (1u << 7) | (1u << 10) | ((n >> 3) << 17) | (0u << 23) | ((m >> 4) << 24);
}

}  // namespace mcl4
