/*
 * kimi_b200.h - C ABI of the B200 (sm_100a) quantized decode hot path.
 *
 * Every entry point takes plain device pointers, element counts, element
 * strides and a CUDA stream passed as `void*` (a cudaStream_t; NULL is the
 * legacy default stream).  No torch or CUDA type appears in a signature.
 * Nothing here allocates device memory except where a function says so;
 * callers that need scratch memory pass it in and size it with the matching
 * *_workspace_size() function.
 *
 * Data formats follow the reference codec (engine/quant/w4a16.py:1-6, 98-99):
 *   - packed INT4 weights: uint8 [N, K/2] row-major (grouped banks: [E, N, K/2]);
 *     the code of the even reduction index k sits in the low nibble, the odd
 *     one in the high nibble; a nibble >= 8 decodes to nibble - 16.
 *   - scales: bf16 [N, K/group] (banks: [E, N, K/group]); group is 32 (the
 *     reference format) or 128 (the restated format); any group of 32 times a
 *     power of two that divides K is accepted.
 *   - decoded weight = bf16(float(code) * float(scale)), products and sums in
 *     fp32, every projection output rounded to bf16 (w4a16_gemv.py:146-158).
 *   - bf16 values travel as uint16_t bit patterns.
 *
 * Return value: KB_OK (0) or a kb_status code.  kb_last_error() returns a
 * human-readable message for the last failing call on the calling thread.
 * Arguments are validated before any launch; a failing call launches nothing.
 * No entry point throws, aborts or traps.
 */
#ifndef KIMI_B200_H
#define KIMI_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define KB_API __attribute__((visibility("default")))
#else
#define KB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum kb_status {
  KB_OK = 0,
  KB_ERR_NULL_POINTER = 1,     /* a required pointer is NULL                    */
  KB_ERR_BAD_SHAPE = 2,        /* a dimension is negative, zero or inconsistent */
  KB_ERR_BAD_GROUP = 3,        /* group size is not a multiple of 32 dividing K */
  KB_ERR_ALIGNMENT = 4,        /* a pointer or stride breaks the 16-byte rule   */
  KB_ERR_WORKSPACE = 5,        /* workspace missing or smaller than required    */
  KB_ERR_UNSUPPORTED = 6,      /* a size above a documented limit               */
  KB_ERR_LAUNCH = 7,           /* the CUDA runtime rejected a launch            */
  KB_ERR_DEVICE = 8            /* a device-side check recorded an error         */
} kb_status;

/* Library version, major*10000 + minor*100 + patch. */
KB_API int kb_version(void);

/* Message for the last failing call on this thread ("" after success). */
KB_API const char* kb_last_error(void);

/* Programmatic dependent launch: when enabled (the default), kernels are
 * launched with the programmatic-stream-serialization attribute so that a
 * kernel's prologue overlaps the tail of the kernel before it on the stream. */
KB_API void kb_set_pdl(int enabled);
KB_API int kb_get_pdl(void);

/* Device-side error word.  Kernels that meet an input they cannot process
 * safely (an expert index outside [0, E)) substitute a safe value (expert 0)
 * and set a bit here.
 * kb_device_errors() copies the word to the host (synchronizes the stream)
 * and clears it.  Bit 0: expert index out of range. */
KB_API int kb_device_errors(void* stream, uint32_t* out_bits);

/* ------------------------------------------------------------------------- */
/* Codec (engine/quant/w4a16.py:68-105 quantise).                              */
/* ------------------------------------------------------------------------- */

/* Quantise bf16 W[N,K] (row stride w_stride elements) into packed [N,K/2]
 * and scales [N,K/group]: scale = bf16(absmax/7) (1 for an all-zero group,
 * else clamped to the smallest normal bf16), code = clamp(rint(w/scale),-7,7).
 * Non-finite inputs set *nonfinite_flag (device int32, may be NULL) to 1. */
KB_API int kb_w4a16_quantise(const uint16_t* w, int64_t w_stride, int64_t N, int64_t K,
                      int64_t group, uint8_t* packed, uint16_t* scales,
                      int32_t* nonfinite_flag, void* stream);

/* ------------------------------------------------------------------------- */
/* Dense W4A16 projection.                                                     */
/* Replaces the registry op `w4a16_dense` (engine/kernels/__init__.py:92-125,  */
/* shipped variant engine/kernels/w4a16_dense_gemv.py:312-336, reference       */
/* engine/quant/triton_w4a16.py:151-188).  y[M,N] = x[M,K] . dequant(W)^T.     */
/* x: bf16 [M,K] with row stride x_stride (elements, unit stride along K);     */
/* y: bf16 [M,N] with row stride y_stride.  M == 0 is a no-op.                 */
/* ------------------------------------------------------------------------- */
KB_API int kb_w4a16_dense(const uint16_t* x, int64_t x_stride, int64_t M, int64_t K,
                   const uint8_t* packed, const uint16_t* scales, int64_t N,
                   int64_t group, uint16_t* y, int64_t y_stride, void* stream);

/* Up to KB_MAX_DENSE_PROBLEMS independent dense projections in one launch,
 * each with its own x, K, N, weights and output.  Replaces the unwired
 * `fused_qkv_w4a16` (engine/kernels/w4a16_fused_qkv.py:342-389), which is the
 * three-problem case with one shared x. */
#define KB_MAX_DENSE_PROBLEMS 8
typedef struct kb_dense_problem {
  const uint16_t* x; int64_t x_stride; int64_t M; int64_t K;
  const uint8_t* packed; const uint16_t* scales; int64_t N; int64_t group;
  uint16_t* y; int64_t y_stride;
} kb_dense_problem;
KB_API int kb_w4a16_dense_multi(const kb_dense_problem* problems, int count, void* stream);

/* ------------------------------------------------------------------------- */
/* Grouped (expert-indexed) W4A16 projection.                                  */
/* Replaces the registry op `w4a16_grouped` (engine/kernels/__init__.py:26-79; */
/* shipped engine/kernels/w4a16_gemv.py:610-635, reference                     */
/* engine/kernels/w4a16_grouped.py:121-194).                                   */
/* y[t,r,:] = x[t,:] . dequant(W[idx[t,r]])^T for every token t < T and route  */
/* r < R.  x: bf16 [T,K] (row stride x_stride); idx: int64 [T,R] contiguous;   */
/* packed: uint8 [E,N,K/2]; scales: bf16 [E,N,K/group]; y: bf16 [T,R,N]        */
/* contiguous.  Assignments sharing an expert read that expert's weights once. */
/* An index of -1 marks an empty slot: it is skipped (no output row written). */
/* Any other index outside [0,E) is computed as expert 0 (never read out of   */
/* bounds) and sets device error bit 0.  T*R must not exceed                  */
/* KB_MAX_ASSIGNMENTS.                                                         */
/* ------------------------------------------------------------------------- */
#define KB_MAX_ASSIGNMENTS 4096
KB_API int kb_w4a16_grouped(const uint16_t* x, int64_t x_stride, int64_t T, int64_t K,
                     const int64_t* idx, int64_t R, const uint8_t* packed,
                     const uint16_t* scales, int64_t E, int64_t N, int64_t group,
                     uint16_t* y, void* stream);

/* Fused gate/up + SwiGLU.  Replaces the registry op `w4a16_swiglu`
 * (engine/kernels/__init__.py:164-218; fused variant
 * engine/kernels/w4a16_gemv.py:772-790).  y[t,r,n] =
 * bf16( bf16(silu(bf16(g))) * bf16(u) ) with g = x[t].W1[e]^T, u = x[t].W3[e]^T
 * (the F.silu(gate)*up contract, w4a16_gemv.py:214-221). */
KB_API int kb_w4a16_swiglu(const uint16_t* x, int64_t x_stride, int64_t T, int64_t K,
                    const int64_t* idx, int64_t R, const uint8_t* w1_packed,
                    const uint16_t* w1_scales, const uint8_t* w3_packed,
                    const uint16_t* w3_scales, int64_t E, int64_t N, int64_t group,
                    uint16_t* y, void* stream);

/* ------------------------------------------------------------------------- */
/* Tensor-core (tcgen05/TMEM) forms of the projections for many tokens.        */
/* Replace the tensor-core W4A16 GEMM the reference falls back to for every    */
/* M > 1 dense call (engine/quant/triton_w4a16.py:44-124, dispatched at        */
/* engine/kernels/w4a16_dense_gemv.py:327-331) and, for expert groups of many  */
/* rows, the grouped/SwiGLU ops above (engine/kernels/w4a16_grouped.py:121-194,*/
/* engine/kernels/__init__.py:182-197).  Same arguments, layouts and results   */
/* as kb_w4a16_dense / kb_w4a16_grouped / kb_w4a16_swiglu (decoded weights     */
/* bf16(code*scale), fp32 accumulation, bf16 outputs); the reduction order     */
/* inside the tensor core differs, so outputs agree within rounding.           */
/* Limits: K % 128 == 0, N % 8 == 0, x row stride % 8 == 0, 16-byte aligned    */
/* pointers, K/group small enough for the per-CTA scale buffers (at most 81    */
/* groups per row), grouped T*R <= KB_MAX_ASSIGNMENTS and E <= 520; outside    */
/* them the call returns KB_ERR_UNSUPPORTED without launching.  y of the       */
/* grouped forms is bf16 [T*R, N] contiguous.                                  */
/* ------------------------------------------------------------------------- */
/* The dense form splits the reduction axis over several CTAs when the matrix
 * has too few 256-row tiles to fill the GPU; the splits' fp32 partials are
 * summed in split order by the last CTA of each tile (deterministic).  Its
 * workspace (kb_w4a16_dense_tc_workspace_size bytes, 0 when no split is
 * made) must be 256-byte aligned and zero-filled before its first use; every
 * launch leaves its counters at zero again.  Calls that share a workspace
 * must not overlap on the GPU. */
KB_API size_t kb_w4a16_dense_tc_workspace_size(int64_t M, int64_t K, int64_t N);
KB_API int kb_w4a16_dense_tc(const uint16_t* x, int64_t x_stride, int64_t M, int64_t K,
                             const uint8_t* packed, const uint16_t* scales, int64_t N,
                             int64_t group, uint16_t* y, int64_t y_stride, void* workspace,
                             size_t workspace_bytes, void* stream);
KB_API int kb_w4a16_grouped_tc(const uint16_t* x, int64_t x_stride, int64_t T, int64_t K,
                               const int64_t* idx, int64_t R, const uint8_t* packed,
                               const uint16_t* scales, int64_t E, int64_t N, int64_t group,
                               uint16_t* y, void* stream);
KB_API int kb_w4a16_swiglu_tc(const uint16_t* x, int64_t x_stride, int64_t T, int64_t K,
                              const int64_t* idx, int64_t R, const uint8_t* w1_packed,
                              const uint16_t* w1_scales, const uint8_t* w3_packed,
                              const uint16_t* w3_scales, int64_t E, int64_t N, int64_t group,
                              uint16_t* y, void* stream);

/* Down projection + routing-weighted combine.  Replaces `fused_w2_combine`
 * (engine/kernels/moe_combine.py:264-324; reference sequence
 * engine/klinear/moe.py:317-334 and moe_combine.py:209-261):
 *   o[t,r]  = bf16( activated[t,r,:] . dequant(W2[idx[t,r]])^T )
 *   out[t]  = bf16( sum_{r<R-1} float(o[t,r]) * weights[t,r] ) + o[t,R-1]
 * (bf16 add; the last route is the shared expert, weight 1, its weights entry
 * ignored).  activated: bf16 [T,R,K] contiguous; idx int64 [T,R]; weights fp32
 * [T,R] with row stride w_stride (>= R-1); out bf16 [T,N].  The per-route
 * outputs and arrival counters live in `workspace` (device memory of at least
 * kb_w4a16_w2_combine_workspace_size(T,R,N) bytes, zero-filled before its
 * first use; every call leaves its counters at zero again, so a buffer may be
 * reused for calls of the same (T,R,N) without clearing; where the counters
 * sit depends on (T,R,N), so zero the buffer again before using it for another
 * shape).  Calls that share a workspace must not overlap on the GPU. */
KB_API size_t kb_w4a16_w2_combine_workspace_size(int64_t T, int64_t R, int64_t N);
KB_API int kb_w4a16_w2_combine(const uint16_t* activated, int64_t T, int64_t R, int64_t K,
                        const int64_t* idx, const float* weights, int64_t w_stride,
                        const uint8_t* w2_packed, const uint16_t* w2_scales,
                        int64_t E, int64_t N, int64_t group, uint16_t* out,
                        void* workspace, size_t workspace_bytes, void* stream);

/* Routing-weighted combine of per-route outputs already in memory (the
 * combine half of moe_combine.py:209-261, for expert parallelism, where the
 * down projections run on the GPUs that own the experts):
 *   out[t,n] = bf16( bf16(sum_{r<R-1} float(routes[t,r,n]) * weights[t,r])
 *                    + routes[t,R-1,n] )
 * fp32 sum in route order, the last route the shared expert (weight 1).
 * routes bf16 [T,R,N] contiguous, 16-byte aligned; weights fp32 rows of
 * stride w_stride (>= R-1); out bf16 [T,N], 16-byte aligned; N % 8 == 0. */
KB_API int kb_moe_combine_routes(const uint16_t* routes, int64_t T, int64_t R, int64_t N,
                                 const float* weights, int64_t w_stride, uint16_t* out,
                                 void* stream);

/* ------------------------------------------------------------------------- */
/* KDA decode preparation (engine/klinear/attention.py:192-230; replaces the  */
/* reference's fused_short_conv_triple + fused_kda_gates,                      */
/* engine/kernels/kda_prepare.py:475-536, 618-665) in one launch.              */
/* q_in/k_in/v_in: bf16 [B, H*D] projections (row stride in_stride); states:  */
/* bf16 [B, H*D, 4] contiguous, updated in place (shift left, token last);    */
/* weights: bf16 [H*D, 4]; raw_decay bf16 [B, H*D]; dt_bias fp32 [H*D];       */
/* a_log fp32 [H]; raw_beta bf16 [B, H].  Outputs fp32: q, k (each head       */
/* normalised by rsqrt(sum of squares + eps)), v, decay [B, H, D], beta       */
/* [B, H] -- the inputs of kb_kda_decode_step.  D a multiple of 32, <= 256.   */
/* ------------------------------------------------------------------------- */
KB_API int kb_kda_prepare(const uint16_t* q_in, const uint16_t* k_in, const uint16_t* v_in,
                          int64_t in_stride, uint16_t* q_state, uint16_t* k_state,
                          uint16_t* v_state, const uint16_t* q_weight, const uint16_t* k_weight,
                          const uint16_t* v_weight, const uint16_t* raw_decay,
                          int64_t raw_decay_stride, const float* dt_bias, const float* a_log,
                          const uint16_t* raw_beta, int64_t raw_beta_stride, int64_t B,
                          int64_t H, int64_t D, float eps, float* q_out, float* k_out,
                          float* v_out, float* decay_out, float* beta_out, void* stream);

/* KDA decode preparation and step in one launch, for head_dim 128 with       */
/* contiguous state rows (state strides sb, sh, sk = 128): the arguments of   */
/* kb_kda_prepare (inputs, convolution states updated in place, gates, eps)  */
/* followed by kb_kda_decode_step's state, scale and outputs.  Each head's    */
/* preparation runs the operations of kb_kda_prepare in its order, so state, */
/* convolution states and outputs equal the two calls' bit for bit.          */
KB_API int kb_kda_prepare_step(const uint16_t* q_in, const uint16_t* k_in, const uint16_t* v_in,
                               int64_t in_stride, uint16_t* q_state, uint16_t* k_state,
                               uint16_t* v_state, const uint16_t* q_weight,
                               const uint16_t* k_weight, const uint16_t* v_weight,
                               const uint16_t* raw_decay, int64_t raw_decay_stride,
                               const float* dt_bias, const float* a_log,
                               const uint16_t* raw_beta, int64_t raw_beta_stride, float eps,
                               float* state, int64_t sb, int64_t sh, int64_t sk, int64_t B,
                               int64_t H, int64_t D, float scale, float* out, uint16_t* out_bf16,
                               void* stream);

/* ------------------------------------------------------------------------- */
/* Expert-parallel data plane (the layer of engine/klinear/moe.py:278-334 with */
/* its experts sharded over ranks: expert e on rank e / per_rank).  Fixed-     */
/* capacity exchange buffers, so no step needs a host-side count and the layer */
/* can be captured in a CUDA graph.                                            */
/*                                                                             */
/* kb_ep_dispatch: for the routed pairs idx[t, r] (int64, row stride           */
/* idx_stride, r < k) in token-major order, the destination rank d and the     */
/* pair's position p among the pairs bound for d (stable); copies hidden[t]    */
/* (bf16, row stride h_stride, H % 8 == 0) to payload row d * capacity + p of  */
/* send_rows, bf16 [world * capacity, H + 8]: H values, then the owner-local   */
/* expert id as an int64 (4 bf16 slots) and 4 bf16 of padding, so rows and ids */
/* travel in one exchange; unused slots carry id -1 (the grouped kernels skip  */
/* them).  slots[t * k + r] = d * capacity + p, int32 [T * k].                 */
/* capacity >= T * k (then nothing can overflow); T * k <= 8192, world <= 64.  */
/* shared_id >= 0: send_rows has T more rows after the world * capacity slots */
/* and row world * capacity + t receives hidden[t] with id shared_id (the     */
/* rank's own rows for its shared expert, processed with the received rows);  */
/* -1: no extra rows.                                                          */
/*                                                                             */
/* kb_ep_combine: out[t] = bf16( bf16(sum_{r<k} float(y[slots[t*k+r]]) *       */
/* weights[t, r]) + shared[t] ), fp32 sum in route order (the combine of       */
/* engine/kernels/moe_combine.py:209-261); y bf16 rows of width H.             */
/* ------------------------------------------------------------------------- */
KB_API int kb_ep_dispatch(const uint16_t* hidden, int64_t h_stride, int64_t T, int64_t H,
                          const int64_t* idx, int64_t idx_stride, int64_t k, int64_t per_rank,
                          int64_t world, int64_t capacity,
                          int64_t shared_id, uint16_t* send_rows,
                          int32_t* slots, void* stream);
KB_API int kb_ep_combine(const uint16_t* y, const int32_t* slots, int64_t T, int64_t k,
                         int64_t H, const float* weights, int64_t w_stride,
                         const uint16_t* shared, int64_t shared_stride, uint16_t* out,
                         int64_t out_stride, void* stream);

/* ------------------------------------------------------------------------- */
/* Router (engine/klinear/router.py:47-85, sigmoid path, one expert group).   */
/* logits = float(hidden) . float(W)^T; scores = sigmoid(logits);              */
/* choice = scores + bias; top_k by (choice desc, index asc);                  */
/* w = scores[idx] / (sum + 1e-20) (if renormalize) * scaling.                 */
/* hidden bf16 [T,K] (row stride h_stride); weight bf16 [E,K]; bias fp32 [E]   */
/* (NULL = zeros); w_out fp32 [T,top_k]; idx_out int64 [T,top_k], or           */
/* [T,top_k+1] with append_id in the last column when append_id >= 0 (the      */
/* shared-expert route of engine/klinear/moe.py:23-36).  The workspace         */
/* (kb_router_workspace_size bytes) holds logits and arrival counters: zero it */
/* before first use; every call leaves its counters at zero, so it may be      */
/* reused for the same (T,E) without clearing.  A NaN choice ranks below every */
/* number, so indices stay in [0,E).  Limits: E <= 1024, top_k <= 32.          */
/* ------------------------------------------------------------------------- */
KB_API size_t kb_router_workspace_size(int64_t T, int64_t E);
KB_API int kb_router_topk(const uint16_t* hidden, int64_t h_stride, int64_t T, int64_t K,
                   const uint16_t* weight, const float* bias, int64_t E,
                   int64_t top_k, int renormalize, float scaling,
                   int64_t* idx_out, int64_t append_id, float* w_out, void* workspace,
                   size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------- */
/* Router without a caller workspace.  No counterpart in the reference: this   */
/* is an addition of this library for callers that cannot allocate device      */
/* memory (a host binding the C ABI without a device allocator, or a serving   */
/* loop that must not call cudaMalloc between steps, since cudaMalloc can      */
/* synchronise the device and fail under memory pressure).  Same arguments and */
/* results as kb_router_topk minus the workspace; it allocates nothing.  Its   */
/* scratch is one fixed device array per device, kb_router_static_scratch_bytes*/
/* bytes (532,480), which limits T*E to 131072 (e.g. T <= 512 at E = 256);     */
/* larger calls return KB_ERR_WORKSPACE.  The first call on each device does a */
/* one-time set-up with that device current (symbol lookup, counter clear on   */
/* the given stream): make it before any stream capture.  Calls that overlap   */
/* in time on one device share the scratch and race: serialise them.          */
/* ------------------------------------------------------------------------- */
KB_API size_t kb_router_static_scratch_bytes(void);
KB_API int kb_router_topk_static(const uint16_t* hidden, int64_t h_stride, int64_t T, int64_t K,
                   const uint16_t* weight, const float* bias, int64_t E,
                   int64_t top_k, int renormalize, float scaling,
                   int64_t* idx_out, int64_t append_id, float* w_out, void* stream);

/* ------------------------------------------------------------------------- */
/* KDA recurrent decode step.  Replaces kda_decode_step                        */
/* (engine/kernels/kda_step.py:273-293, reference :173-196).  fp32 throughout: */
/*   S' = S * exp(decay)[:,None];  p = S'^T k;  d = v - p;                      */
/*   S  <- S' + (beta*k) d^T  (in place);  o = S^T (q*scale).                  */
/* state [B,H,Dk,Dv] with element strides (sb,sh,sk) and unit stride along Dv; */
/* q,k,decay [B,H,Dk], v [B,H,Dv], beta [B,H], out [B,H,Dv] contiguous.        */
/* out_bf16 (may be NULL) additionally receives bf16(o).  Dk,Dv <= 256.        */
/* ------------------------------------------------------------------------- */
KB_API int kb_kda_decode_step(float* state, int64_t sb, int64_t sh, int64_t sk,
                       const float* q, const float* k, const float* v,
                       const float* decay, const float* beta, int64_t B,
                       int64_t H, int64_t Dk, int64_t Dv, float scale,
                       float* out, uint16_t* out_bf16, void* stream);

/* ------------------------------------------------------------------------- */
/* Decode-step executor.  Runs a whole program of the operations above in one  */
/* persistent launch (one CTA per SM): the weight stream of every operation    */
/* runs ahead of the dependencies between operations, which are enforced with */
/* device completion counters.  It replaces the sequence of registry calls of  */
/* one decode step of the reference (engine/klinear/model.py:134-160 calling   */
/* the layers of engine/klinear/layers.py, captured as one CUDA graph by       */
/* engine/klinear/generate.py:226-276) for the operations of the hot path.     */
/* Every pointer is bound when the operation is added (the same static buffers */
/* a captured graph uses); each kb_step_launch runs the whole program.         */
/* An operation's consumers wait for the operations listed in deps before      */
/* they read their inputs; list every earlier operation that writes an input  */
/* or that reads a buffer the operation writes.  Results equal the            */
/* per-operation entry points up to fp32 summation order (router logits, KDA   */
/* partials).  Limits: 1 <= tokens <= KB_STEP_MAX_TOKENS, K % 128 == 0, E <=   */
/* 256, top_k <= 8, Dk <= 128.  kb_step_finalize uploads the program           */
/* (allocates device memory) on the current device.                           */
/* ------------------------------------------------------------------------- */
#define KB_STEP_MAX_TOKENS 8
#define KB_STEP_MAX_DEPS 4
typedef struct kb_step kb_step;
KB_API int kb_step_create(int64_t tokens, kb_step** out);
KB_API void kb_step_destroy(kb_step* step);
/* One to three INT4 projections of the same tokens (problem M == tokens). */
KB_API int kb_step_add_dense(kb_step* step, const kb_dense_problem* problems, int count,
                   const int* deps, int ndeps, int* op_out);
/* Dense gate/up + SwiGLU: y = bf16(silu(bf16 x.w1^T)) * bf16(x.w3^T).       */
KB_API int kb_step_add_swiglu(kb_step* step, const uint16_t* x, int64_t x_stride, int64_t K,
                   const uint8_t* w1_packed, const uint16_t* w1_scales,
                   const uint8_t* w3_packed, const uint16_t* w3_scales, int64_t N,
                   int64_t group, uint16_t* y, int64_t y_stride, const int* deps,
                   int ndeps, int* op_out);
/* Router logits; the selection runs in the expert operation that uses it.   */
/* scratch: 16*tokens*E bytes, 8-byte aligned, one per router of the program  */
/* and owned by it (zeroed by kb_step_finalize, not to be written between     */
/* launches): per launch parity and (token, expert) a 64-bit word holding the */
/* choice key + 1 and the fp32 sigmoid score.  idx_out int64                 */
/* [tokens, top_k+1] (shared expert id E appended), w_out fp32 [tokens, top_k]. */
KB_API int kb_step_add_router(kb_step* step, const uint16_t* hidden, int64_t h_stride,
                   int64_t K, const uint16_t* weight, const float* bias, int64_t E,
                   int64_t top_k, int renormalize, float scaling, void* scratch,
                   int64_t* idx_out, float* w_out, const int* deps, int ndeps,
                   int* op_out);
/* Expert block of one MoE layer on banks [E+1, ...] (slot E = shared expert):*/
/* gate/up + SwiGLU into activated [tokens*(top_k+1), I], down projection of  */
/* every route into routed_out [tokens*(top_k+1), H], combine into out        */
/* [tokens, H].  op_out receives the index of the down/combine operation,     */
/* the one later operations depend on.                                        */
KB_API int kb_step_add_moe(kb_step* step, int router_op, const uint16_t* hidden,
                   int64_t h_stride, int64_t H, const uint8_t* w1_packed,
                   const uint16_t* w1_scales, const uint8_t* w3_packed,
                   const uint16_t* w3_scales, const uint8_t* w2_packed,
                   const uint16_t* w2_scales, int64_t I, int64_t group,
                   uint16_t* activated, uint16_t* routed_out, uint16_t* out,
                   const int* deps, int ndeps, int* op_out);
KB_API int kb_step_add_kda(kb_step* step, float* state, int64_t sb, int64_t sh, int64_t sk,
                   const float* q, const float* k, const float* v, const float* decay,
                   const float* beta, int64_t B, int64_t H, int64_t Dk, int64_t Dv,
                   float scale, float* out, uint16_t* out_bf16, const int* deps,
                   int ndeps, int* op_out);
KB_API int kb_step_finalize(kb_step* step);
KB_API int kb_step_launch(kb_step* step, void* stream);
KB_API int kb_step_info(const kb_step* step, int* n_ops, int* stages, int* stage_bytes,
                   size_t* smem_bytes);
/* Optional timeline: with a device buffer of kb_step_trace_entries() int64   */
/* set, every launch records %globaltimer ns per (CTA, operation) in 8 fields: */
/* consumers start, inputs ready, routing built (expert blocks), end, producer */
/* done issuing the weights, reducers done, shared-expert items done (expert   */
/* gate/up), spare.  NULL switches it off.                                    */
KB_API int kb_step_set_trace(kb_step* step, int64_t* trace, int64_t entries);
KB_API int64_t kb_step_trace_entries(const kb_step* step);

#ifdef __cplusplus
}
#endif

#endif /* KIMI_B200_H */
