/*
 * mcl4moe — C ABI of the B200 (sm_100a) NVFP4 SwiGLU mixture-of-experts layer.
 *
 * Plain C: raw device pointers, sizes and a CUDA stream.  Nothing here
 * allocates device memory: every buffer, including scratch ("workspace"), is
 * owned and passed in by the caller.  Every function returns an int status
 * (MCL4MOE_OK == 0) and never aborts the process; kernels are launched on the
 * given stream and run asynchronously unless stated otherwise.
 *
 * Reference: mESmaC/MCL4-COE, src/mcl4_coe/nvfp4.py and
 * src/mcl4_coe/backbone.py.  Each entry point names the reference function it
 * replaces.
 *
 * Data formats (identical bytes to the reference quantiser):
 *   NVFP4 value  : E2M1 code, 4 bits; two per byte, even element in the low nibble.
 *   block scale  : float8 e4m3fn per 16 consecutive K elements (per 16x16 tile
 *                  for weights, repeated over the tile's 16 rows).
 *   global scale : float32; 1.0 for activations, amax/2688 per expert for weights.
 *   "swizzled" scales: the 128-row x 4-scale atoms of the reference's
 *                  _swizzle_scales (nvfp4.py:131-144): scale (r, c) of a matrix
 *                  with C scales per row sits at byte
 *                  ((r/128)*(C/4) + c/4)*512 + (r%32)*16 + ((r%128)/32)*4 + c%4.
 *   Weights, kernel layout: packed codes K-major [E, N, K/2] (the transpose of
 *                  the reference cache's B_fwd [E, K/2, N]) + swizzled scales
 *                  [E, N*K/16] + global scales [E].
 */
#ifndef MCL4MOE_H_
#define MCL4MOE_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same object as cudaStream_t / CUstream; NULL is the legacy default stream. */
typedef struct CUstream_st* mcl4moe_stream_t;

enum mcl4moe_status {
  MCL4MOE_OK = 0,
  MCL4MOE_ERR_INVALID = 1,      /* bad shape, null pointer or misalignment (the reference raises ValueError) */
  MCL4MOE_ERR_UNSUPPORTED = 2,  /* not an sm_100 device, or a shape outside the kernels' tiling */
  MCL4MOE_ERR_CUDA = 3,         /* a CUDA runtime call or kernel launch failed */
  MCL4MOE_ERR_TIMEOUT = 4,      /* a device-side wait gave up; see mcl4moe_read_error */
  MCL4MOE_ERR_WORKSPACE = 5     /* workspace smaller than the matching *_workspace_size */
};

/* Human-readable name of a status code (static storage). */
const char* mcl4moe_status_string(int status);

/* ABI version, major*10000 + minor*100 + patch. */
int mcl4moe_version(void);

/* 1 when the current CUDA device can run the kernels (compute capability 10.x). */
int mcl4moe_device_supported(void);

/* Synchronise ``stream`` and read then clear the device error word that the
 * kernels set when a bounded device-side wait gives up (0 = no error; 1xx =
 * TMA producer, 2xx = MMA issuer, 3xx = epilogue).  Blocking. */
int mcl4moe_read_error(int32_t* device_error_word, int32_t* host_value, mcl4moe_stream_t stream);

/* ------------------------------------------------------------------------
 * Replaces quantize_nvfp4 / _quantize_nvfp4_core in the one-dimensional modes
 * (src/mcl4_coe/nvfp4.py:197-259): 1x16 row blocks of a bf16 (dtype 0) or fp32
 * (dtype 1) matrix x [rows, cols] (row stride ld elements) with global scale
 * g = 1 (causal != 0, causal_row_scale=True) or g = max(amax/2688, FLT_MIN)
 * (amax > 0, else 1).  packed: [rows, cols/2]; scales: the swizzled 128x4-atom
 * layout of _swizzle_scales for rows_pad rows (multiple of 128, >= rows;
 * padding rows get zero scales); global_scale: device fp32 [1];
 * amax_scratch: device fp32 [1].  Requires cols % 64 == 0, x 16-byte aligned and
 * a row stride of a multiple of 16 bytes.
 * ------------------------------------------------------------------------ */
int mcl4moe_quantize_rows(const void* x, int dtype, int64_t rows, int cols, int64_t ld, int causal, uint8_t* packed,
                          uint8_t* scales, int64_t rows_pad, float* global_scale, float* amax_scratch,
                          mcl4moe_stream_t stream);

/* ------------------------------------------------------------------------
 * Replaces nvfp4_mm (src/mcl4_coe/nvfp4.py:285-334) with a prequantised B,
 * as _NVFP4Linear.forward calls it (:398-429): out (fp32 [M, N]) =
 * deq(A) @ deq(B).T * g_a * g_b (+ bias [N], added after the scaling), where A
 * is x (bf16 dtype 0 / fp32 dtype 1, [M, K] contiguous) quantised here in
 * one-dimensional mode (causal: g_a = 1, else tensor-wise g_a) and B is
 * packed [N, K/2] with swizzled scales for N rows and global scale b_g (device
 * fp32 [1]) — the output of mcl4moe_quantize_rows or, for a weight,
 * mcl4moe_quantize_weights with n = 1.  a_global_scale (device fp32 [1] or
 * NULL) receives g_a.  Requires K % 256 == 0, N % 256 == 0 (pad otherwise).
 * ------------------------------------------------------------------------ */
size_t mcl4moe_nvfp4_mm_workspace_size(int64_t M, int K);
int mcl4moe_nvfp4_mm(const void* x, int dtype, int64_t M, int K, int causal, const uint8_t* b, const uint8_t* b_scales,
                     const float* b_g, int N, const float* bias, float* out, float* a_global_scale,
                     int32_t* error_word, void* workspace, size_t workspace_bytes, mcl4moe_stream_t stream);

/* ------------------------------------------------------------------------
 * Stochastic rounding in the single-matrix operators (quantize_nvfp4 with
 * stochastic=True, nvfp4_mm with stochastic_a=True, src/mcl4_coe/nvfp4.py:186-194,
 * :285-334), as _NVFP4Linear.backward uses them (:431-472).  Codes are
 * min(trunc(u + U), 7) with u the scaled magnitude of the deterministic rule and
 * U in [0, 1) a Philox4x32-10 draw keyed by `seed` at offset row * cols + col
 * (the reference draws U with torch.rand_like: same distribution, different
 * stream).  Scales and global scales are those of the round-to-nearest mode.
 *
 * mcl4moe_quantize_rows_stochastic: mcl4moe_quantize_rows with stochastic codes.
 * mcl4moe_nvfp4_mm_sr: mcl4moe_nvfp4_mm with A quantised stochastically (the
 *   input gradient, grad_output x W: B = the weight's transposed 16x16-tile
 *   quantisation, mcl4moe_quantize_weights_t with n = 1).
 * mcl4moe_nvfp4_linear_wgrad: the weight gradient
 *   dW = nvfp4_mm(H16(G^T), H16(X^T), stochastic_a=True)  (:454-459)
 *   for grad_output G [M, N] and inputs X [M, K] (row-major, bf16 dtype 0 or
 *   fp32 dtype 1), H16 the fixed-sign orthonormal Walsh-Hadamard transform over
 *   groups of 16 tokens (_hadamard16, :337-355): H16(G^T) quantised
 *   stochastically (noise offset n * round_up(M, 256) + token), H16(X^T) to
 *   nearest, each with its tensor-wise global scale.  dw: fp32
 *   [N, round_up(K, 256)] (columns >= K are zero); d_bias (fp32 [N] or NULL):
 *   the column sums of G (:468-469).  M == 0 gives zeros.
 * ------------------------------------------------------------------------ */
int mcl4moe_quantize_rows_stochastic(const void* x, int dtype, int64_t rows, int cols, int64_t ld, int causal,
                                     uint64_t seed, uint8_t* packed, uint8_t* scales, int64_t rows_pad,
                                     float* global_scale, float* amax_scratch, mcl4moe_stream_t stream);
int mcl4moe_nvfp4_mm_sr(const void* x, int dtype, int64_t M, int K, int causal, uint64_t seed, const uint8_t* b,
                        const uint8_t* b_scales, const float* b_g, int N, const float* bias, float* out,
                        float* a_global_scale, int32_t* error_word, void* workspace, size_t workspace_bytes,
                        mcl4moe_stream_t stream);
/* mcl4moe_quantize_hadamard_t: one operand of that product on its own,
 * quantize_nvfp4(_hadamard16(y.t()), stochastic) for y [M, C] (row-major, bf16
 * dtype 0 or fp32 dtype 1) with the token dimension zero-padded to kt
 * (multiple of 128, >= M) and the rows to rows_out (multiple of 32, >= C; of 128
 * when swizzled): packed [rows_out, kt/2], scales row-major [rows_out, kt/16] or
 * the swizzled 128x4 atoms, global_scale = max(amax/2688 or 1, FLT_MIN) of the
 * transformed matrix (device fp32 [1]); amax_scratch device fp32 [1]. */
int mcl4moe_quantize_hadamard_t(const void* y, int dtype, int64_t M, int C, int64_t kt, int rows_out, int stochastic,
                                uint64_t seed, uint8_t* packed, uint8_t* scales, int swizzled, float* global_scale,
                                float* amax_scratch, mcl4moe_stream_t stream);
size_t mcl4moe_nvfp4_linear_wgrad_workspace_size(int64_t M, int N, int K);
int mcl4moe_nvfp4_linear_wgrad(const void* grad, int grad_dtype, const void* x, int x_dtype, int64_t M, int N, int K,
                               uint64_t seed, float* dw, float* d_bias, int32_t* error_word, void* workspace,
                               size_t workspace_bytes, mcl4moe_stream_t stream);

/* ------------------------------------------------------------------------
 * Replaces compute_2to4_mask (src/mcl4_coe/nvfp4.py:70-110), applied to a
 * weight before its NVFP4 quantisation when a layer's sparsity_mode is not
 * "none" (:1020-1023).  W fp32 [N, K] row-major; mode 1 = "2to4_row" (keep the
 * two largest |w| of every 4 consecutive elements along K), mode 2 =
 * "2to4_transposable" (per 4x4 tile the doubly 2:4 pattern of largest kept
 * L1, first maximum in the reference's catalog order; falls back to mode 1
 * when N % 4 != 0, as the reference does).  Writes w_masked = w * mask (fp32
 * [N, K]; may alias w) and, when non-NULL, mask as 0/1 bytes [N, K].
 * Requires K % 4 == 0 and 16-byte aligned w / w_masked.
 * ------------------------------------------------------------------------ */
int mcl4moe_mask_2to4(const float* w, int N, int K, int mode, float* w_masked, uint8_t* mask,
                      mcl4moe_stream_t stream);

/* ------------------------------------------------------------------------
 * Weight quantisation.
 * Replaces _quantize_grouped_weights_core (src/mcl4_coe/nvfp4.py:923-952)
 * and the dirty-expert refresh of _get_or_build_grouped_nvfp4_cache
 * (src/mcl4_coe/nvfp4.py:1010-1044).
 *
 * Quantises ``n`` fp32 weight matrices W_i [N, K] (host array of device
 * pointers; row-major, contiguous) into slots ``slots[i]`` (host array) of
 * the kernel-layout cache: packed [E, N, K/2], scales [E, Np*K/16] (swizzled,
 * Np = N rounded up to 128; the padding rows are not written), global_scale [E].  The optional ref_* outputs (NULL to skip) receive the
 * reference cache layout at the same slots: B_fwd [E, K/2, N],
 * Bs_fwd [E, N, K/16], B_bwd [E, N/2, K], Bs_bwd [E, K, N/16].
 * amax_scratch: device float32 [n].  Requires N % 16 == 0, K % 64 == 0.
 * ------------------------------------------------------------------------ */
int mcl4moe_quantize_weights(const float* const* w_ptrs, const int32_t* slots, int n, int N, int K,
                             uint8_t* packed, uint8_t* scales, float* global_scale, uint8_t* ref_b_fwd,
                             uint8_t* ref_bs_fwd, uint8_t* ref_b_bwd, uint8_t* ref_bs_bwd, float* amax_scratch,
                             mcl4moe_stream_t stream);

/* The same quantisation plus the transposed copy the backward's input-gradient
 * GEMM reads (the reference's B_bwd / Bs_bwd, src/mcl4_coe/nvfp4.py:947-951,
 * in the kernel layout): packed_t [E, K, N/2] (row k of W^T packs the (n, n+1)
 * pairs) and scales_t [E, K*N/16], the 16x16 tile scales swizzled for the K rows
 * of W^T.  Requires K % 128 == 0 in addition. */
int mcl4moe_quantize_weights_t(const float* const* w_ptrs, const int32_t* slots, int n, int N, int K,
                               uint8_t* packed, uint8_t* scales, float* global_scale, uint8_t* packed_t,
                               uint8_t* scales_t, float* amax_scratch, mcl4moe_stream_t stream);

/* ------------------------------------------------------------------------
 * Activation quantisation, 1x16 row blocks with global scale 1.
 * Replaces _quantize_nvfp4_core(x, two_dimensional=False,
 * stochastic=False, causal_row_scale=True) (src/mcl4_coe/nvfp4.py:197-225)
 * and its Triton launch _nvfp4_quantize_1d_kernel (src/mcl4_coe/nvfp4.py:735,
 * launched :1074-1086).
 * x: bf16 [rows, cols] with row stride ld_x (elements); packed [rows, cols/2];
 * scales [rows, cols/16] row-major when swizzled == 0, else the swizzled
 * atoms (rows padded to 128).  cols % 64 == 0.
 * ------------------------------------------------------------------------ */
int mcl4moe_quantize_activations(const uint16_t* x, int64_t rows, int cols, int64_t ld_x, uint8_t* packed,
                                 uint8_t* scales, int swizzled, mcl4moe_stream_t stream);

/* ------------------------------------------------------------------------
 * Router, top-k and routing statistics.
 * Replaces the routing part of SparseMoE.forward
 * (src/mcl4_coe/backbone.py:787-883, loop branch :913-1004):
 * fp32 logits x @ Wr^T (+ optional additive bias), softmax, top-k with
 * optional renormalisation, selection mask, counts, aux and z loss.
 * Tokens with valid[t] == 0 are not routed (loop-branch semantics).
 * logits_in (nullable) are final logits (any bias already added) that replace
 * the router product: then x, wr and logit_bias are unused.
 * Outputs: topk_idx int32 [T, k], topk_w fp32 [T, k] (0 for invalid tokens),
 * logits_out fp32 [T, E] (nullable), sel_mask fp32 [T, E] (nullable),
 * counts int32 [E], stats fp32 [3 + E]: {aux_loss, z_loss, n_routed,
 * counts_fraction[E]} (the layer's aux, router_z_loss and counts outputs).
 * Batches of up to 1024 tokens with d <= 12800 compute the logits on the CUDA
 * cores (fp32 FMA, fixed summation order); longer batches and wider rows run
 * the router product on the tensor cores with the fp32 weight split into
 * three bf16 parts (exact products, fp32 accumulation on the tensor pipe: the
 * logits' error grows with d, about 6.5e-5 at d = 12864).  Requires E <= 256,
 * k <= min(E, 32), d % 64 == 0, T * k <= 2^30 (counts, offsets and slot
 * ranks are int32; larger batches return MCL4MOE_ERR_UNSUPPORTED and a
 * workspace size of 0).
 * ------------------------------------------------------------------------ */
size_t mcl4moe_route_workspace_size(int T, int E, int k, int d);
int mcl4moe_route(const uint16_t* x, const float* wr, const float* logit_bias, const float* logits_in,
                  const uint8_t* valid, int T, int d, int E, int k, int norm_topk_prob, int32_t* topk_idx,
                  float* topk_w, float* logits_out, float* sel_mask, int32_t* counts, float* stats,
                  void* workspace, size_t workspace_bytes, mcl4moe_stream_t stream);

/* ------------------------------------------------------------------------
 * Routing without a caller workspace.  No counterpart in the reference: it
 * serves callers that cannot allocate device scratch (a C/cgo/JNI client
 * that owns only its input and output buffers, or a serving loop with a
 * fixed memory pool).  Same arguments, checks and results as mcl4moe_route,
 * but the scratch is a fixed device array inside this library of
 * mcl4moe_route_noalloc_scratch_bytes() bytes (8 MiB: enough for T = 131072
 * at E = 64, k = 8, d = 2048); a shape whose mcl4moe_route_workspace_size
 * exceeds it returns MCL4MOE_ERR_WORKSPACE.  The first call on a device (that
 * device current) does the set-up — it looks up the array's device address,
 * which may load the module — so make it before any stream capture; the
 * address is kept per device and CUDA context, and the first call in a new
 * context (after cudaDeviceReset) looks it up again.  Later calls allocate
 * nothing.  There is one array per device: calls on one device must not
 * overlap in time, or they race on the scratch.
 * ------------------------------------------------------------------------ */
size_t mcl4moe_route_noalloc_scratch_bytes(void);
int mcl4moe_route_noalloc(const uint16_t* x, const float* wr, const float* logit_bias, const float* logits_in,
                          const uint8_t* valid, int T, int d, int E, int k, int norm_topk_prob, int32_t* topk_idx,
                          float* topk_w, float* logits_out, float* sel_mask, int32_t* counts, float* stats,
                          mcl4moe_stream_t stream);

/* ------------------------------------------------------------------------
 * Full MoE layer forward.
 * Replaces SparseMoE.forward for the routing configuration without mitotic
 * pairs / lineage / coverage penalty / dense subset
 * (src/mcl4_coe/backbone.py:618-911): route -> stable expert-major permute
 * -> NVFP4 activation quantisation -> grouped gate/up GEMM with fused SwiGLU
 * and NVFP4 re-quantisation -> grouped down GEMM with the routing weight
 * -> k-way combine.  Shapes: d % 256 == 0, F % 256 == 0, E <= 256,
 * k <= min(E, 32).
 * ------------------------------------------------------------------------ */
typedef struct mcl4moe_moe_args {
  /* inputs */
  const uint16_t* x;          /* bf16 [T, d] */
  const float* router_w;      /* fp32 [E, d] */
  const float* logit_bias;    /* fp32 [E] or NULL */
  const uint8_t* valid;       /* uint8 [T] or NULL */
  const uint8_t* w_up;        /* kernel-layout NVFP4 up_proj [E, 2F, d/2] (gate rows first) */
  const uint8_t* w_up_scales; /* [E, 2F*d/16] swizzled */
  const float* w_up_g;        /* [E] */
  const uint8_t* w_dn;        /* kernel-layout NVFP4 down_proj [E, d, F/2] */
  const uint8_t* w_dn_scales; /* [E, d*F/16] swizzled */
  const float* w_dn_g;        /* [E] */
  int T, d, E, k, F;
  int norm_topk_prob;
  /* outputs */
  uint16_t* out;              /* bf16 [T, d] */
  float* stats;               /* fp32 [3 + E]: aux, z, n_routed, counts[E] */
  float* sel_mask;            /* fp32 [T, E] or NULL (last_selected_mask) */
  int32_t* topk_idx;          /* int32 [T, k] or NULL */
  float* topk_w;              /* fp32 [T, k] or NULL */
  int32_t* offs;              /* int32 [E] inclusive ends of the expert segments, or NULL */
  int32_t* perm;              /* int32 [T*k] stable argsort of the selected experts, or NULL */
  uint16_t* h_debug;          /* bf16 [M_cap, F] SwiGLU output in padded order, or NULL */
  int32_t* error_word;        /* device int32 set by a timed-out device wait, or NULL to use one inside the
                                 workspace (cleared on every call).  A caller-owned word is sticky: while it
                                 is nonzero the GEMM kernels skip their work. */
  void* workspace;
  size_t workspace_bytes;
  /* Optional cudaEvent_t[6] (NULL to skip): recorded on the stream before
   * routing and after routing, permutation, gate/up GEMM, down GEMM and combine. */
  void* const* stage_events;
  /* Training forward (all NULL for inference): what mcl4moe_moe_backward_experts
   * reads, in the padded expert-major rows (M_cap = mcl4moe_padded_rows(T, E, k)). */
  uint16_t* up_save;          /* bf16 [M_cap, 2F]: gate | value, bf16(acc * g) of the gate/up GEMM, or NULL */
  uint16_t* x_rows_save;      /* bf16 [M_cap, d]: the permuted input rows (padding rows zero), or NULL */
  uint16_t* y_save;           /* bf16 [M_cap, d]: unweighted down-projection rows bf16(acc * g); the combine then
                                 weights each slot as bf16(y * bf16(w)).  NULL: weighted rows stay internal */
  float* logits_out;          /* fp32 [T, E] router logits (mcl4moe_moe_forward only), or NULL */
} mcl4moe_moe_args;

size_t mcl4moe_moe_workspace_size(int T, int d, int E, int k, int F);
int mcl4moe_moe_forward(const mcl4moe_moe_args* args, mcl4moe_stream_t stream);

/* The layer forward from a routing the caller computed (replaces the grouped
 * dispatch after routing, src/mcl4_coe/backbone.py:893-911, for the routing
 * variants that feed it precomputed selections: mitotic twins :791-832,
 * lineage families :274-305, coverage penalty :843-851, dense subsets
 * :307-398).  Inputs topk_idx (int32 [T, k], expert ids; ids outside [0, E)
 * mark slots that are not routed) and topk_w (fp32 [T, k]); the stable
 * expert-major permutation, NVFP4 quantisation, grouped GEMMs and combine are
 * those of mcl4moe_moe_forward.  router_w, logit_bias and sel_mask are not
 * read; stats, when non-NULL, receives [0, 0, routed tokens, slot share per
 * expert] (the caller computes the variant's losses); offs / perm as in
 * mcl4moe_moe_forward.  Same workspace size. */
int mcl4moe_moe_forward_routed(const mcl4moe_moe_args* args, mcl4moe_stream_t stream);

/* ------------------------------------------------------------------------
 * Backward (training).  Replaces the autograd path of SparseMoE.forward's
 * grouped branch (src/mcl4_coe/backbone.py:853-911) through
 * _NVFP4GroupedLinear.backward (src/mcl4_coe/nvfp4.py:1112-1216).
 *
 * mcl4moe_quantize_rows_sr: the reference's stochastic-rounding gradient
 * quantiser (_nvfp4_quantize_1d_kernel with STOCHASTIC=True, :735-790, as the
 * backward launches it at :1128-1151): tensor-wise global scale
 * max(amax/2688 if amax > 0 else 1, FLT_MIN) written to global_scale, per 1x16
 * block s = e4m3(min(amax16 / (6 g), 448)), codes floor(u + U) clamped to 7 with
 * U the Philox4x32-10 draw of Triton's tl.rand(seed, row * cols + col).  x bf16
 * [rows, cols] contiguous; packed [rows, cols/2]; scales row-major
 * [rows, cols/16]; amax_scratch device fp32 [1].  cols % 128 == 0.
 *
 * mcl4moe_moe_backward_experts: from the gradient d_out of the layer output
 * and what the training forward saved (mcl4moe_moe_args' up_save / y_save and
 * the routing: slot_pos, topk_w and the expert layout pad_start / counts /
 * offs_start), computes in the padded expert-major rows:
 *   d_y    = bf16(d_out[t] * bf16(w))         (the down projection's output grad)
 *   d_w    = bf16(sum_c bf16(d_out[t,c] * y))  (routing-weight grad, [T, k])
 *   d_h    = SR(d_y) x W_down   (grouped NVFP4 GEMM on the transposed weights)
 *   d_up   = [d_gate | d_val] from the SwiGLU derivative
 *   d_rows = SR(d_up) x W_up
 * The weight gradients (d_y^T h, d_up^T x_rows per expert) and the router's
 * matrix products are the caller's.  seed_down / seed_up: the noise seeds of
 * the two quantisations.
 * mcl4moe_router_backward: d_logits [T, E] from d_w, the saved logits and
 * routing, the forward's stats and the upstream gradients of aux_loss / z_loss
 * (device fp32 scalars or NULL for 0).
 * mcl4moe_moe_backward_dx: d_x[t] = bf16(sum_j d_rows[slot(t, j)] +
 * d_x_router[t]) (fp32 d_x_router [T, d] or NULL).
 * ------------------------------------------------------------------------ */
typedef struct mcl4moe_moe_bwd_args {
  int T, d, E, k, F;
  const uint16_t* d_out;          /* bf16 [T, d] */
  const int32_t* slot_pos;        /* int32 [T, k]: padded row of slot (t, j), -1 when not routed */
  const float* topk_w;            /* fp32 [T, k] routing weights of the forward */
  const int32_t* pad_start;       /* int32 [E + 1] padded row start of each expert segment */
  const int32_t* counts;          /* int32 [E] routed rows per expert */
  const int32_t* offs_start;      /* int32 [E] first row of each expert in the unpadded order */
  const uint16_t* y_save;         /* bf16 [M_cap, d] unweighted down-projection rows */
  const uint16_t* up_save;        /* bf16 [M_cap, 2F] gate | value rows */
  const uint8_t* w_up_t;          /* up_proj^T in the kernel layout [E, d, F] bytes (2F codes per row) */
  const uint8_t* w_up_t_scales;   /* [E, d*2F/16] swizzled */
  const float* w_up_g;            /* [E] */
  const uint8_t* w_dn_t;          /* down_proj^T [E, F, d/2] */
  const uint8_t* w_dn_t_scales;   /* [E, F*d/16] swizzled */
  const float* w_dn_g;            /* [E] */
  uint64_t seed_down, seed_up;
  uint16_t* d_y;                  /* out bf16 [M_cap, d] (padding rows zero) */
  uint16_t* d_up;                 /* out bf16 [M_cap, 2F] */
  uint16_t* d_rows;               /* out bf16 [M_cap, d] gradient of the permuted input rows */
  float* d_w;                     /* out fp32 [T, k] */
  int32_t* error_word;            /* as in mcl4moe_moe_args */
  void* workspace;
  size_t workspace_bytes;
} mcl4moe_moe_bwd_args;

int mcl4moe_quantize_rows_sr(const uint16_t* x, int64_t rows, int cols, uint64_t seed, uint8_t* packed,
                             uint8_t* scales, float* global_scale, float* amax_scratch, mcl4moe_stream_t stream);
size_t mcl4moe_moe_backward_workspace_size(int T, int d, int E, int k, int F);
int mcl4moe_moe_backward_experts(const mcl4moe_moe_bwd_args* args, mcl4moe_stream_t stream);
/* Expert weight gradients: dW[e] = G[rows of e]^T X[rows of e] in fp32 ([E, N, K]) for
 * bf16 row-major G [rows, N] (d_y or d_up) and X [rows, K] (h or the permuted input
 * rows), the rows of expert e being [pad_start[e], pad_start[e+1]) (padding rows of G
 * zero); an expert without rows gets zeros.  Replaces _grouped_wgrad_kernel
 * (src/mcl4_coe/nvfp4.py:877-920).  Requires N % 128 == 0, K % 256 == 0,
 * rows % 256 == 0 (the padded row capacity). */
int mcl4moe_moe_backward_wgrad(const uint16_t* g, const uint16_t* x, int64_t rows, int N, int K,
                               const int32_t* pad_start, int E, float* dw, int32_t* error_word,
                               mcl4moe_stream_t stream);
int mcl4moe_router_backward(const float* logits, const int32_t* topk_idx, const float* topk_w, const float* d_w,
                            const uint8_t* valid, const float* stats, const float* d_aux, const float* d_z, int T,
                            int E, int k, int norm_topk_prob, float* d_logits, mcl4moe_stream_t stream);
int mcl4moe_moe_backward_dx(const uint16_t* d_rows, const int32_t* slot_pos, const float* d_x_router, int T, int k,
                            int d, uint16_t* d_x, mcl4moe_stream_t stream);

/* Capacity in rows of the padded, expert-major activation buffers
 * (sum over experts of count rounded up to 256, bounded by T*k + 255*E). */
int64_t mcl4moe_padded_rows(int T, int E, int k);

/* Expert GEMM tiling of mcl4moe_moe_forward / mcl4moe_moe_forward_routed (a tuning
 * knob with no counterpart in the reference; process-wide): 0 = chosen by shape (the
 * default: single-CTA 128-row tiles when an inference call averages at most 64 routed
 * rows per expert, CTA-pair 256-row tiles otherwise), 1 = always pair tiles, 2 =
 * single-CTA tiles for every inference call (training calls, which pass up_save /
 * y_save, always use pair tiles).  Both tilings give the same bytes.  Returns the
 * previous mode, or -1 for a mode outside [0, 2]. */
int mcl4moe_set_expert_tiling(int mode);

/* Device pointer of a named region inside a forward workspace (for tests,
 * debugging and the backward's inputs): 0 xq, 1 xs, 2 hq, 3 hs, 4 y,
 * 5 pad_start [E+1], 6 slot_pos [T, k], 7 sorted_w, 8 the int32 device error
 * word used when args.error_word is NULL, 9 counts [E] (routed rows per
 * expert), 10 offs_start [E] (first unpadded row of each expert). */
void* mcl4moe_workspace_region(void* workspace, int region, int T, int d, int E, int k, int F);

/* ------------------------------------------------------------------------
 * Grouped NVFP4 linear on rows already grouped by expert.
 * Replaces nvfp4_grouped_linear(inputs, experts, proj_name, offs)
 * (src/mcl4_coe/nvfp4.py:1219-1227 -> _NVFP4GroupedLinear.forward :1051-1110):
 * out[m, :] = bf16((quant(x[m]) . W_e^T) * g_e) for rows m of expert e, i.e.
 * rows [offs[e-1], offs[e]) (inclusive ends, int32 on the device).
 * x bf16 [M, K]; w kernel-layout [E, N, K/2] + scales + g; out bf16 [M, N].
 * K % 256 == 0, N % 256 == 0.
 * ------------------------------------------------------------------------ */
size_t mcl4moe_grouped_linear_workspace_size(int64_t M, int K, int E);
int mcl4moe_grouped_linear(const uint16_t* x, int64_t M, int K, const int32_t* offs, int E, const uint8_t* w,
                           const uint8_t* w_scales, const float* w_g, int N, uint16_t* out, int32_t* error_word,
                           void* workspace, size_t workspace_bytes, mcl4moe_stream_t stream);

/* ------------------------------------------------------------------------
 * Expert parallelism (G ranks, rank g owns experts [g*E_loc, (g+1)*E_loc)).
 * No counterpart in the reference, which runs the layer on one device: these
 * are the dispatch and combine steps around the grouped GEMMs when the experts
 * of SparseMoE (src/mcl4_coe/backbone.py:887-910) are sharded across GPUs.
 * The exchange between ranks (all-to-all of rows, then of partial sums) is
 * the caller's.  The shipped Python layer (ExpertParallelMoE) copies the
 * pieces with the copy engines straight into peer buffers mapped through CUDA
 * IPC (mcl4moe_ipc_import + mcl4moe_copy_list_async below), ordered by a
 * one-element NCCL all-reduce; over a non-NCCL process group (gloo) it uses
 * torch.distributed's all_to_all_single.
 *
 * Dispatch row (mcl4moe_ep_row_bytes(d, k) bytes): NVFP4 codes [d/2], 1x16
 * E4M3 scales row-major [d/16], k int8 expert ids local to the destination
 * (-1: expert on another rank) padded to 16, k fp32 routing weights padded to
 * 16.  Requires d % 256 == 0, G <= 8, E == G * E_loc.
 *
 * mcl4moe_ep_dispatch: from routing (topk_idx/topk_w of mcl4moe_route) builds
 * one row per (token, destination holding any of its experts), destinations
 * concatenated in rank order, tokens in index order within a destination.
 * send_counts (device int32 [2G]): rows then expert slots per destination;
 * send_pos (int32 [T, G]): row of (t, g) in send_buf or -1.  send_buf must hold
 * T * G rows (the worst case).
 * mcl4moe_ep_experts: on the receiving rank, R received rows holding `slots`
 * local expert slots in total -> partial (bf16 [R, d]): per row, the sum over
 * its local experts of bf16(bf16(acc * g) * bf16(w)), summed in fp32.
 * mcl4moe_ep_combine: out[t] = bf16(sum over g of back_buf[send_pos[t, g]]),
 * back_buf holding the partials returned in send order.
 * ------------------------------------------------------------------------ */
int mcl4moe_ep_row_bytes(int d, int k);
size_t mcl4moe_ep_dispatch_workspace_size(int T, int G);
int mcl4moe_ep_dispatch(const uint16_t* x, const int32_t* topk_idx, const float* topk_w, const uint8_t* valid, int T,
                        int d, int k, int G, int E_loc, int32_t* send_counts, int32_t* send_pos, uint8_t* send_buf,
                        void* workspace, size_t workspace_bytes, mcl4moe_stream_t stream);
/* mcl4moe_ep_dispatch in two calls on the same stream and workspace: _count
 * writes send_counts (and the per-group offsets _pack needs, in the workspace);
 * _pack writes send_pos and send_buf.  A caller exchanges the counts between
 * the two, so that reading them on the host overlaps the packing. */
int mcl4moe_ep_dispatch_count(const int32_t* topk_idx, const uint8_t* valid, int T, int k, int G, int E_loc,
                              int32_t* send_counts, void* workspace, size_t workspace_bytes,
                              mcl4moe_stream_t stream);
int mcl4moe_ep_dispatch_pack(const uint16_t* x, const int32_t* topk_idx, const float* topk_w, const uint8_t* valid,
                             int T, int d, int k, int G, int E_loc, const int32_t* send_counts, int32_t* send_pos,
                             uint8_t* send_buf, void* workspace, size_t workspace_bytes, mcl4moe_stream_t stream);
size_t mcl4moe_ep_experts_workspace_size(int R, int slots, int d, int k, int E_loc, int F);
int mcl4moe_ep_experts(const uint8_t* recv_buf, int R, int slots, int d, int k, int E_loc, int F,
                       const uint8_t* w_up, const uint8_t* w_up_scales, const float* w_up_g, const uint8_t* w_dn,
                       const uint8_t* w_dn_scales, const float* w_dn_g, uint16_t* partial, int32_t* error_word,
                       void* workspace, size_t workspace_bytes, mcl4moe_stream_t stream);
int mcl4moe_ep_combine(const uint16_t* back_buf, const int32_t* send_pos, int T, int d, int G, uint16_t* out,
                       mcl4moe_stream_t stream);
/* mcl4moe_ep_experts with the partial sums stored straight into their sources'
 * buffers (one kernel does the sums and the return transfer): received rows of
 * source s are [seg_start[s], seg_start[s+1]) (host int32 [G+1], seg_start[G]
 * == R) and row r of source s goes to dst[s] + (r - seg_start[s]) * d bf16
 * elements; dst[s] (host array of device pointers) may map another GPU's memory
 * (mcl4moe_ipc_import).  The stores are complete when the stream reaches the
 * end of the call. */
int mcl4moe_ep_experts_to_peers(const uint8_t* recv_buf, int R, int slots, int d, int k, int E_loc, int F,
                                const uint8_t* w_up, const uint8_t* w_up_scales, const float* w_up_g,
                                const uint8_t* w_dn, const uint8_t* w_dn_scales, const float* w_dn_g, int G,
                                const int32_t* seg_start, void* const* dst, int32_t* error_word, void* workspace,
                                size_t workspace_bytes, mcl4moe_stream_t stream);

/* ------------------------------------------------------------------------
 * Expert parallelism with the down projection at the token's home GPU ("h
 * back"; no counterpart in the reference).  The gate/up projections stay
 * sharded; the receiving GPU sends back each slot's NVFP4 h (F/2 codes + F/16
 * scales) instead of a bf16 partial sum (d values), and the source runs the
 * down projection (all E experts' down weights on every GPU) and the combine
 * of the single-device layer, so its output is the single-device output bit
 * for bit.
 *
 * mcl4moe_moe_forward_layout: the first half of mcl4moe_moe_forward (routing
 * and the expert-major layout of the call's slots, as mcl4moe_moe_args /
 * workspace); w_up / w_dn are not read.  The layout's slot_pos
 * (mcl4moe_workspace_region 6, int32 [T, k]) is what _dispatch_pack_h needs.
 * mcl4moe_ep_dispatch_pack_h: mcl4moe_ep_dispatch_pack whose rows carry, in
 * place of the k weights, the k destinations of the slots' h on this rank
 * (rank << 28 | slot_pos row; -1 for slots on other ranks).
 * mcl4moe_ep_gateup_to_peers: on the receiver, the gate/up GEMM with SwiGLU and
 * NVFP4 re-quantisation of the received slots, each slot's h stored into
 * hq_dst[rank] (codes [M_cap, F/2]) and hs_dst[rank] (128x4 swizzled scales for
 * M_cap rows) of its source; hq_dst / hs_dst (host arrays of G device
 * pointers) may map other GPUs' memory (mcl4moe_ipc_import).  The stores are
 * complete when the stream reaches the end of the call.
 * mcl4moe_moe_forward_down: the second half of mcl4moe_moe_forward on the same
 * args and workspace, the down projection reading h from hq / hs (NULL: the
 * workspace's own), then the combine into args->out.
 * ------------------------------------------------------------------------ */
int mcl4moe_moe_forward_layout(const mcl4moe_moe_args* args, mcl4moe_stream_t stream);
int mcl4moe_moe_forward_down(const mcl4moe_moe_args* args, const uint8_t* hq, const uint8_t* hs,
                             mcl4moe_stream_t stream);
int mcl4moe_ep_dispatch_pack_h(const uint16_t* x, const int32_t* topk_idx, const uint8_t* valid, int T, int d, int k,
                               int G, int E_loc, int rank, const int32_t* slot_pos, const int32_t* send_counts,
                               int32_t* send_pos, uint8_t* send_buf, void* workspace, size_t workspace_bytes,
                               mcl4moe_stream_t stream);
int mcl4moe_ep_gateup_to_peers(const uint8_t* recv_buf, int R, int slots, int d, int k, int E_loc, int F,
                               const uint8_t* w_up, const uint8_t* w_up_scales, const float* w_up_g, int G,
                               void* const* hq_dst, void* const* hs_dst, int32_t* error_word, void* workspace,
                               size_t workspace_bytes, mcl4moe_stream_t stream);

/* ------------------------------------------------------------------------
 * Peer-memory transport for the expert-parallel exchange (no counterpart in
 * the reference).  mcl4moe_ipc_export: CUDA IPC handle (64 bytes) of the
 * allocation holding ptr, and ptr's offset in it.  mcl4moe_ipc_import (another
 * process on the same node, any device with peer access): map that allocation,
 * returning its base; add the offset.  mcl4moe_ipc_close: unmap a base returned
 * by mcl4moe_ipc_import.  mcl4moe_copy_async: device-to-device copy on `stream`
 * (to a peer mapping it runs on the copy engines over NVLink).
 * ------------------------------------------------------------------------ */
int mcl4moe_ipc_export(const void* ptr, uint8_t* handle_out, uint64_t* offset_out);
int mcl4moe_ipc_import(const uint8_t* handle, void** base_out);
int mcl4moe_ipc_close(void* base);
int mcl4moe_copy_async(void* dst, const void* src, size_t bytes, mcl4moe_stream_t stream);
/* n device-to-device copies, copy i on streams[i % n_streams], in list order
 * (zero-byte entries are skipped); all arguments are host arrays. */
int mcl4moe_copy_list_async(void* const* dst, const void* const* src, const uint64_t* bytes, int n,
                            mcl4moe_stream_t const* streams, int n_streams);

#ifdef __cplusplus
}
#endif

#endif /* MCL4MOE_H_ */
