/*
 * godwit_cuda.h — C-ABI of the B200 (sm_100a) MoE expert hot path.
 *
 * This is the boundary Godwit's Swift engine binds in place of its Metal
 * expert kernels.  Every entry point takes plain pointers and sizes; nothing
 * in these signatures is a CUDA, PyTorch or Swift type (streams travel as
 * `void*`).  Each call returns a `gw_status`; on failure `gw_last_error()`
 * returns a thread-local message describing it.
 *
 * Reference interfaces replaced (paths inside rayl15/Godwit):
 *   - Router.logits / select / route        Sources/Godwit/Runtime/Router.swift:38-104
 *   - ExpertRunner.apply                    Sources/Godwit/Runtime/ExpertRunner.swift:275-331
 *   - ExpertRunner.applyBatch               Sources/Godwit/Runtime/ExpertRunner.swift:191-269
 *   - ExpertRunner.applyAssignments + the MoE half of TransformerLayer.forward
 *                                           Sources/Godwit/Runtime/ExpertRunner.swift:108-182,
 *                                           Sources/Godwit/Runtime/TransformerLayer.swift:150-238
 *   - ExpertCache / ModelReader.loadExpertStride (the slot cache becomes an
 *     HBM-resident bank)                    Sources/Godwit/Runtime/ExpertCache.swift:180-274,
 *                                           Sources/Godwit/Runtime/ModelReader.swift:73-76
 *   - mxfp4_gemv (benchmark GEMV)           Sources/Godwit/Metal/Quant/dequant_gemv.metal:37-67
 *   - MXFP4.decode (bit-exact dequant)      Sources/Godwit/Quant/MXFP4.swift:37-92
 *   - int8_affine_gemv / int8_affine_gemv_bias_batched (the trunk's int8
 *     projections: output head, attention q/k/v/o)
 *                                           Sources/Godwit/Metal/MoE/router.metal:65-141,
 *                                           Sources/Godwit/Runtime/ModelRunner.swift:165-190,
 *                                           Sources/Godwit/Runtime/Attention.swift:218-240
 *
 * Conventions:
 *   - Synchronous calls (no `_async` suffix) take HOST pointers, copy inputs to
 *     the device, run, copy results back and wait, mirroring the reference's
 *     commit-and-wait `MetalContext.run` (Infrastructure/Metal/MetalContext.swift:149-155).
 *   - `_async` calls take DEVICE pointers and are ordered on the context's
 *     stream (see gw_ctx_set_stream); they do not synchronise.
 *   - The library owns all device memory it allocates.  Host arrays are
 *     borrowed for the duration of a call only.
 *   - A gw_ctx is internally locked: calls on one context are serialised.
 *   - Shape misuse that the reference catches with `precondition` is
 *     reported as GW_E_ARG before any kernel launches.
 *   - Device activation and output buffers of the MoE `_async` calls
 *     (x_dev, out_dev, stream_dev) must be 16-byte aligned (any cudaMalloc
 *     or torch allocation is); an offset pointer that is not is rejected with
 *     GW_E_ARG before any launch.
 */
#ifndef GODWIT_CUDA_H
#define GODWIT_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__) || defined(__clang__)
#define GW_API __attribute__((visibility("default")))
#else
#define GW_API
#endif

typedef int32_t gw_status;

#define GW_OK             0
#define GW_E_ARG         (-1)  /* invalid argument (shape, index, null pointer) */
#define GW_E_CUDA        (-2)  /* CUDA runtime error                            */
#define GW_E_OOM         (-3)  /* device allocation failed                      */
#define GW_E_TIMEOUT     (-4)  /* a bounded device-side wait gave up            */
#define GW_E_STATE       (-5)  /* object used in the wrong state                */
#define GW_E_UNSUPPORTED (-6)  /* configuration this build does not implement   */

/* Activation input element type. The reference feeds Float16; the B200
 * configs feed bfloat16.  Both are accepted everywhere `x_dtype` appears. */
#define GW_DTYPE_F16   0
#define GW_DTYPE_BF16  1
/* Output element type of the int8 projections (y_dtype): fp32 as
 * int8_affine_gemv writes, or f16 as int8_affine_gemv_bias_batched does. */
#define GW_DTYPE_F32   2

/* Expert activation, mirroring FeedForwardActivation
 * (Sources/Godwit/Model/ArchitectureSpec.swift:15-39). */
#define GW_ACT_GPTOSS_CLAMPED 0  /* (clamp(up,±L)+1)·min(gate,L)·σ(α·min(gate,L)) — expert.metal:82-102 */
#define GW_ACT_SILU           1  /* silu(gate)·up                                  — expert.metal:380-393 */

/* Expert stride sections, in storage order (Install/InstallLayout.swift:18-25). */
#define GW_SEC_GATE_UP_BLOCKS 0
#define GW_SEC_GATE_UP_SCALES 1
#define GW_SEC_DOWN_BLOCKS    2
#define GW_SEC_DOWN_SCALES    3
#define GW_SEC_GATE_UP_BIAS   4
#define GW_SEC_DOWN_BIAS      5
#define GW_SEC_COUNT          6

typedef struct gw_ctx  gw_ctx;
typedef struct gw_bank gw_bank;

/* Bank description: the model dimensions of ArchitectureSpec plus the expert
 * stride and section spans of GodwitManifest.expertStride / expertSections
 * (Install/GodwitManifest.swift:47-51). */
typedef struct gw_bank_desc {
    int32_t hidden;            /* H: 2880 GPT-OSS, 2048 Qwen3                 */
    int32_t intermediate;      /* F: 2880 GPT-OSS, 768 Qwen3                  */
    int32_t experts;           /* E: routed experts per layer                 */
    int32_t layers;            /* L: MoE layers held by the bank              */
    int32_t top_k;             /* experts per token                           */
    int32_t activation;        /* GW_ACT_*                                    */
    float   limit;             /* swiglu_limit (7.0), GPT-OSS only            */
    float   alpha;             /* sigmoid steepness (1.702), GPT-OSS only     */
    int32_t has_router_bias;   /* 0: router bias treated as zeros             */
    int32_t shard_rank;        /* expert e is resident iff e % shard_count == shard_rank */
    int32_t shard_count;       /* 1 = the whole bank on this device           */
    int32_t reserved0;
    int64_t expert_stride;                  /* bytes per expert stride        */
    int64_t section_offset[GW_SEC_COUNT];   /* byte offset within the stride  */
    int64_t section_length[GW_SEC_COUNT];   /* byte length of the section     */
} gw_bank_desc;

/* ---- errors, version ---------------------------------------------------- */

/* Thread-local description of the last failure on this thread ("" if none). */
GW_API const char* gw_last_error(void);
/* ABI version, major*10000 + minor*100 + patch. */
GW_API int32_t gw_version(void);

/* ---- context ------------------------------------------------------------ */

/* Binds a context to CUDA device `device` (one process per GPU). */
GW_API gw_status gw_init(int32_t device, gw_ctx** out);
GW_API gw_status gw_shutdown(gw_ctx* ctx);
/* Orders subsequent `_async` work on `cuda_stream` (a cudaStream_t; NULL =
 * the context's own stream). */
GW_API gw_status gw_ctx_set_stream(gw_ctx* ctx, void* cuda_stream);
/* Waits for all work queued on the context's stream.  Returns GW_E_TIMEOUT
 * (and clears the record) when a bounded device-side wait inside one of the
 * context's kernels gave up since the last gw_sync; the kernel that gave up
 * wound down without faulting, so the context stays usable, but the results
 * of the work since the last gw_sync are not valid. */
GW_API gw_status gw_sync(gw_ctx* ctx);
/* Launches one kernel whose bounded wait, on a barrier that nothing ever
 * completes, gives up after `wait_cycles` SM clock cycles (0..1e8) and
 * records that the way the expert kernels do; the next gw_sync then returns
 * GW_E_TIMEOUT.  Lets a caller check its timeout handling end to end without
 * a GPU fault.  No counterpart in the reference. */
GW_API gw_status gw_selftest_wait_timeout(gw_ctx* ctx, int64_t wait_cycles);
/* Expert-path policy (no reference counterpart: the reference runs every
 * (expert, token) assignment as GEMVs, ExpertRunner.applyAssignments,
 * Runtime/ExpertRunner.swift:108-183).  A layer with T tokens runs its experts as tensor-core grouped GEMMs when
 * T * top_k >= min_avg * experts, else as the MXFP4 GEMV tiles; 0 = always
 * the GEMV tiles.  Default 8. */
GW_API gw_status gw_set_tensor_core_min_tokens(gw_ctx* ctx, int32_t min_avg);
/* Tensor-core expert path arithmetic: 0 (default) = exact f16 activations
 * (the reference's numerics, fp32 accumulation); 1 = tcgen05 block-scaled
 * MXFP4 x MXFP8 MMAs, the expert inputs and activations quantised to MXFP8
 * (E4M3 codes, one E8M0 scale per 32 values along K, scale = 2^(floor(log2
 * max|x|) - 8), nearest-even, saturating) — half the MMA instructions and no
 * weight widening, at ~6% relative (rel-L2) deviation from the f16 result. */
GW_API gw_status gw_set_block_scaled(gw_ctx* ctx, int32_t enable);

/* ---- layout (ExpertLayout.init, Install/InstallLayout.swift:50-92) ------ */

/* Fills `out` with the page-aligned stride and section spans the reference
 * installer writes, plus the dimensions given. */
GW_API gw_status gw_layout_default(int32_t hidden, int32_t intermediate, int32_t experts,
                            int32_t layers, int32_t top_k, int32_t activation,
                            gw_bank_desc* out);

/* ---- HBM-resident expert bank ------------------------------------------- */

GW_API gw_status gw_bank_create(gw_ctx* ctx, const gw_bank_desc* desc, gw_bank** out);
GW_API gw_status gw_bank_destroy(gw_bank* bank);
/* Copies one expert's stride — the bytes ModelReader.loadExpertStride returns
 * (Runtime/ModelReader.swift:73-76) — into HBM.  `len` must equal the stride.
 * Rejects experts not owned by this shard. */
GW_API gw_status gw_bank_upload_expert(gw_bank* bank, int32_t layer, int32_t expert,
                                const void* stride_bytes, size_t len);
/* Router weight bf16 [E, H] and bias bf16 [E] (may be NULL: zeros), the
 * tensors Router.logits binds (Runtime/Router.swift:38-66). */
GW_API gw_status gw_bank_upload_router(gw_bank* bank, int32_t layer,
                                const uint16_t* w_bf16, const uint16_t* b_bf16_or_null);
/* Fills every resident expert and the router of every layer on the device
 * with the seeded synthetic distribution (codes uniform 0..15, scales
 * uniform 118..124, biases and router weights ~N(0, 0.02) in bf16).  The
 * generator is a counter hash, reproducible on the host. */
GW_API gw_status gw_bank_fill_synthetic(gw_bank* bank, uint64_t seed);
/* Copies one resident expert's stride back to the host (`len` = stride). */
GW_API gw_status gw_bank_download_expert(gw_bank* bank, int32_t layer, int32_t expert,
                                  void* stride_bytes, size_t len);
/* Bytes of HBM the bank holds. */
GW_API gw_status gw_bank_bytes(gw_bank* bank, int64_t* out);

/* ---- synchronous host-pointer API --------------------------------------- */

/* Router.logits for T tokens: logits[T, E] (fp32). */
GW_API gw_status gw_router_logits(gw_ctx* ctx, gw_bank* bank, int32_t layer,
                           const void* x, int32_t x_dtype, int32_t T, float* logits);
/* Router.route for T tokens: experts[T, k] (highest logit first, the
 * selection-sort order of Router.select) and weights[T, k] (softmax over the
 * k selected logits). */
GW_API gw_status gw_route(gw_ctx* ctx, gw_bank* bank, int32_t layer,
                   const void* x, int32_t x_dtype, int32_t T,
                   int32_t* experts_out, float* weights_out);
/* ExpertRunner.apply: one expert on one token, y[H] before routing weight. */
GW_API gw_status gw_expert_apply(gw_ctx* ctx, gw_bank* bank, int32_t layer, int32_t expert,
                          const void* x, int32_t x_dtype, float* y);
/* ExpertRunner.applyBatch: y[H] = sum_i weights[i] * expert_i(x). */
GW_API gw_status gw_expert_apply_batch(gw_ctx* ctx, gw_bank* bank, int32_t layer,
                                const void* x, int32_t x_dtype, int32_t n,
                                const int32_t* experts, const float* weights, float* y);
/* MoE block for T tokens: out[T, H] = sum_k w[t,k] * expert_{e[t,k]}(x[t]).
 * If `experts_in`/`weights_in` are NULL the router runs on the device first
 * (and its decision is returned through `experts_out`/`weights_out` if those
 * are non-NULL); otherwise the given routing [T, k] is applied, which is
 * ExpertRunner.applyAssignments for the same assignment set. */
GW_API gw_status gw_moe_forward(gw_ctx* ctx, gw_bank* bank, int32_t layer,
                         const void* x, int32_t x_dtype, int32_t T,
                         const int32_t* experts_in, const float* weights_in,
                         float* out, int32_t* experts_out, float* weights_out);
/* mxfp4_gemv / mxfp4_gemv_bias on raw reference-layout arrays:
 * y[rows] = dequant(packed, scales) . x + bias.  cols % 32 == 0. */
GW_API gw_status gw_mxfp4_gemv(gw_ctx* ctx, const uint8_t* packed, const uint8_t* scales,
                        const uint16_t* bias_bf16_or_null, const void* x, int32_t x_dtype,
                        float* y, int32_t rows, int32_t cols);
/* MXFP4.decode on the device, fp32 out [rows, cols]; bit-exact with the
 * reference's CPU decoder (0xFF scale -> NaN). */
GW_API gw_status gw_mxfp4_dequant(gw_ctx* ctx, const uint8_t* packed, const uint8_t* scales,
                           int32_t rows, int32_t cols, float* w_out);

/* int8 affine projection on host arrays (Install/Int8Affine.swift format):
 * codes [rows][cols] uint8, meta [rows][cols/64][2] bf16 (scale, zero) pairs
 * — the two regions of an installed trunk tensor, codes first
 * (InstallLayout.swift:151-157) — bias [rows] bf16 or NULL, x [T][cols] f16;
 * y [T][rows] = sum over groups of scale*(codes.x) + zero*sum(x), + bias,
 * written as fp32 (y_dtype GW_DTYPE_F32, the head's int8_affine_gemv,
 * router.metal:65-98) or rounded to f16 (GW_DTYPE_F16,
 * int8_affine_gemv_bias_batched, router.metal:107-141).  cols % 64 == 0,
 * cols <= 16384. */
GW_API gw_status gw_int8_affine_gemv(gw_ctx* ctx, const uint8_t* codes, const uint16_t* meta,
                                     const uint16_t* bias_or_null, const uint16_t* x_f16, int32_t T,
                                     int32_t rows, int32_t cols, void* y, int32_t y_dtype);

/* ---- stream-ordered device-pointer API ---------------------------------- */

/* gw_int8_affine_gemv on device memory, ordered on the context's stream.
 * codes_dev and x_dev must be 16-byte aligned, meta_dev 4-byte aligned. */
GW_API gw_status gw_int8_affine_gemv_async(gw_ctx* ctx, const uint8_t* codes_dev,
                                           const uint16_t* meta_dev, const uint16_t* bias_dev_or_null,
                                           const uint16_t* x_dev, int32_t T, int32_t rows,
                                           int32_t cols, void* y_dev, int32_t y_dtype);

/* Batched GEMV over `count` independent matrices (device pointers, strides
 * in elements of each array's type).  x_stride may be 0 to share one x. */
GW_API gw_status gw_mxfp4_gemv_batched_async(gw_ctx* ctx, int32_t count,
                                      const uint8_t* packed, int64_t packed_stride,
                                      const uint8_t* scales, int64_t scale_stride,
                                      const uint16_t* bias_or_null, int64_t bias_stride,
                                      const void* x, int64_t x_stride, int32_t x_dtype,
                                      float* y, int64_t y_stride,
                                      int32_t rows, int32_t cols);
/* Router.route (Runtime/Router.swift:100-104) on device memory: x_dev [T, H]
 * -> experts_dev [T, k] int32, weights_dev [T, k] fp32, ordered on the
 * context's stream (gw_route's device twin; used by the all-to-all expert
 * parallelism to route a rank's own tokens before dispatching them). */
GW_API gw_status gw_route_async(gw_ctx* ctx, gw_bank* bank, int32_t layer, const void* x_dev,
                                int32_t x_dtype, int32_t T, int32_t* experts_dev, float* weights_dev);
/* One MoE layer on device memory: x_dev [T, H] (x_dtype), out_dev [T, H] fp32.
 * experts_dev/weights_dev: optional [T, k] outputs of the routing decision. */
GW_API gw_status gw_moe_forward_async(gw_ctx* ctx, gw_bank* bank, int32_t layer,
                               const void* x_dev, int32_t x_dtype, int32_t T,
                               float* out_dev, int32_t* experts_dev, float* weights_dev);
/* The whole layer stack with residual chaining and identity norm:
 * stream = x; for l: stream += moe_l(round_to_x_dtype(stream)).
 * x_dev [T, H] (x_dtype) in, stream_dev [T, H] fp32 out. */
GW_API gw_status gw_moe_stack_forward_async(gw_ctx* ctx, gw_bank* bank,
                                     const void* x_dev, int32_t x_dtype, int32_t T,
                                     float* stream_dev);
/* Applies a given routing [T, k] (device arrays) to x_dev: out_dev (=, or +=
 * when `accumulate` != 0) sum_k w * expert(x).  Expert ids this shard does
 * not own, or outside [0, E), contribute nothing — the per-rank half of
 * expert parallelism, whose rows carry one expert each: the expert path
 * (gw_set_tensor_core_min_tokens) is chosen as for T slots, not T * k. */
GW_API gw_status gw_moe_apply_async(gw_ctx* ctx, gw_bank* bank, int32_t layer,
                             const void* x_dev, int32_t x_dtype, int32_t T,
                             const int32_t* experts_dev, const float* weights_dev,
                             float* out_dev, int32_t accumulate);
/* stream_dev[i] += delta_dev[i] (delta may be NULL) and, if x_out_dev is not
 * NULL, x_out_dev[i] = round(stream_dev[i]) in x_dtype; n elements.  The
 * residual add of TransformerLayer.forward (Runtime/TransformerLayer.swift:232-238). */
GW_API gw_status gw_residual_round_async(gw_ctx* ctx, float* stream_dev, const float* delta_dev,
                                  void* x_out_dev, int32_t x_dtype, int64_t n);
/* RMSNorm ahead of the router (TransformerLayer.normalise,
 * Runtime/TransformerLayer.swift:265-285; Metal `rmsnorm`, Metal/MoE/router.metal:41-60):
 * out_dev[T, H] f16 = stream_dev[t, i] * (1 / sqrt(mean_i(stream_dev[t, i]^2) + eps)) * w[i],
 * fp32 arithmetic, bf16 weight [H].  The squares are summed as a tree, not in
 * index order, so an output can differ from the reference's by one f16 ulp.
 * H % 4 == 0; stream_dev 16-byte, weight_dev and out_dev 8-byte aligned. */
GW_API gw_status gw_rmsnorm_async(gw_ctx* ctx, const float* stream_dev, const uint16_t* weight_dev,
                                  float eps, int32_t T, int32_t H, void* out_dev);
/* The MoE half of TransformerLayer.forward (Runtime/TransformerLayer.swift:140-238)
 * on the device, with no host round trip between its steps: normed =
 * RMSNorm(stream, norm_w, eps) (the post-attention norm, :141-143), routing
 * and the experts on normed (as gw_moe_forward), then stream += the weighted
 * expert sum (:232-238).  stream [T, H] fp32 is updated in place; norm_w is
 * the layer's bf16 post-attention norm weight [H].  experts/weights: optional
 * [T, k] routing outputs.  gw_moe_block takes host pointers and returns when
 * done; gw_moe_block_async takes device pointers (stream 16-byte, norm_w
 * 8-byte aligned) and is ordered on the context's stream. */
GW_API gw_status gw_moe_block(gw_ctx* ctx, gw_bank* bank, int32_t layer, float* stream,
                              const uint16_t* norm_w, float eps, int32_t T, int32_t* experts_out,
                              float* weights_out);
GW_API gw_status gw_moe_block_async(gw_ctx* ctx, gw_bank* bank, int32_t layer, float* stream_dev,
                                    const uint16_t* norm_w_dev, float eps, int32_t T,
                                    int32_t* experts_dev, float* weights_dev);
/* One MoE layer that allocates no device memory, for callers that cannot
 * allocate while serving (memory planned up front, a hard memory cap, or no
 * tolerance for a first-call allocation).  No counterpart in the reference.
 * Same arguments and results as gw_moe_forward_async; the layer's scratch
 * lives in a fixed 4 MiB device array that every device loading this library
 * holds until the process exits, so the token count is limited to what fits
 * (up to T=55 at GPT-OSS shapes, 50 at Qwen3-30B-A3B shapes); larger T is
 * rejected with GW_E_ARG.  The first
 * call on a device resolves the array's address (cudaGetSymbolAddress); make
 * that first call before any stream capture.  The resolved address belongs
 * to the device's primary context: after a cudaDeviceReset of that device
 * this entry point must not be called again in the process.  All calls share
 * the array: calls that overlap on the GPU (other streams, other contexts of
 * the same device) race.  The experts always run on the persistent MXFP4
 * expert GEMV: the context's expert-path switches (gw_set_tensor_core_min_tokens,
 * gw_set_block_scaled) and the small-batch GEMV tiles do not apply here, so
 * its results equal gw_moe_forward_async's up to fp32 summation order
 * whenever that call runs a GEMV path too (always at decode sizes under the
 * default policy). */
GW_API gw_status gw_moe_forward_noalloc_async(gw_ctx* ctx, gw_bank* bank, int32_t layer,
                                              const void* x_dev, int32_t x_dtype, int32_t T,
                                              float* out_dev, int32_t* experts_dev,
                                              float* weights_dev);
/* Token-sliced expert parallelism, device side.  No counterpart in the
 * reference (it runs on one device); used by an engine that shards the
 * experts over `world` GPUs by index (rank e % world holds expert e).
 *
 * gw_ep_dispatch_async packs this rank's T routed tokens for one all-to-all:
 * send_dev holds world blocks of `capacity` rows, a row being H values of
 * x_dtype followed by four 16-bit words (the slot's expert id as int32,
 * -1 for an unused row, and its routing weight as fp32 bits); slot
 * t * top_k + j goes to row (e % world) * capacity + (the number of earlier
 * slots bound for the same rank), recorded in idx_dev [T * top_k].  A block
 * that needs more than `capacity` rows sets *overflow_dev (int32) to 1 (its
 * extra slots overwrite the block's last row); the caller checks it.
 * gw_ep_combine_async sums, per token, the returned weighted expert outputs
 * back_dev [world * capacity][H] fp32 at its slots' rows, in slot order,
 * into out_dev [T][H].  x_dev, send_dev, back_dev and out_dev 16-byte
 * aligned (send rows are then 8-byte aligned); world <= 64. */
GW_API gw_status gw_ep_dispatch_async(gw_ctx* ctx, gw_bank* bank, const void* x_dev, int32_t x_dtype,
                                      int32_t T, const int32_t* experts_dev, const float* weights_dev,
                                      int32_t world, int32_t capacity, void* send_dev, int32_t* idx_dev,
                                      int32_t* overflow_dev);
GW_API gw_status gw_ep_combine_async(gw_ctx* ctx, gw_bank* bank, const float* back_dev,
                                     const int32_t* idx_dev, int32_t T, float* out_dev);
/* Kernel timing recorded with CUDA events on the context's stream around
 * each expert GEMV launch while profiling is enabled. */
typedef struct gw_profile {
    int64_t gateup_launches;   /* gate_up GEMV + activation kernels           */
    int64_t down_launches;     /* down GEMV + routing-weight kernels          */
    int64_t gemv_launches;     /* plain batched GEMV kernels                  */
    double  gateup_ms;         /* summed device time of those launches        */
    double  down_ms;
    double  gemv_ms;
    int64_t expert_passes;     /* sum over profiled layers of experts streamed */
    int64_t gemv_matrices;     /* matrices processed by the profiled GEMVs    */
    int64_t router_launches;   /* router + top-k (or grouping) kernels        */
    int64_t combine_launches;  /* combine (+ residual) kernels                */
    double  router_ms;
    double  combine_ms;
} gw_profile;
/* Enables (1) or disables (0) kernel timing; enabling clears the counters. */
GW_API gw_status gw_profile_enable(gw_ctx* ctx, int32_t enable);
/* Waits for the stream, then reports the counters since profiling was enabled. */
GW_API gw_status gw_profile_read(gw_ctx* ctx, gw_profile* out);
/* Total number of this library's kernels launched through `ctx` so far. */
GW_API gw_status gw_last_launch_count(gw_ctx* ctx, int64_t* out);

#ifdef __cplusplus
}
#endif

#endif /* GODWIT_CUDA_H */
