/*
 * gtmoe.h -- C ABI of the B200 (sm_100a) MoE block of the Turbo-WinFare engine.
 *
 * Plain pointers and sizes only. Every pointer argument named *_dev is a CUDA device pointer;
 * `stream` is a cudaStream_t passed as void* (NULL = the legacy default stream). Calls are
 * asynchronous on `stream` unless stated otherwise. All functions return GTM_OK (0) or a
 * negative gtm_status; gtm_last_error() then holds a message for the calling thread (the
 * reference's convention, include/gturbo/c_api.h:74-78 and src/c_api.cpp:29-34).
 *
 * Replaces, for the MoE path:
 *   - ComputePipelineManager::dispatch (include/gturbo/pipeline.hpp:97-101, src/pipeline.cpp:409-518)
 *     for the kernels GemvInt4, GemvInt8, RouterTopK, GeGLU, ScaleAccum, MulBF16, RMSNormK,
 *     PostAttn and LayerTail: one entry each below, plus gtm_dispatch, which accepts the same
 *     16 root constants and byte-offset buffer bindings as the HLSL kernels;
 *   - the per-layer MoE sequence of ForwardRunner::produce_token (src/runner.cpp:549-716),
 *     i.e. ~48 dispatches and a CPU read-back of the router's top-K per layer, by one fused
 *     device-resident call (gtm_moe_decode) with all experts resident in HBM.
 */
#ifndef GTMOE_H
#define GTMOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GTM_API __attribute__((visibility("default")))

typedef enum gtm_status {
    GTM_OK = 0,
    GTM_ERR_INVALID = -1,      /* bad argument: null pointer, zero or inconsistent size     */
    GTM_ERR_UNSUPPORTED = -2,  /* shape the fused kernels are not built for                  */
    GTM_ERR_CUDA = -3,         /* a CUDA runtime call failed                                 */
    GTM_ERR_TIMEOUT = -4,      /* a bounded device-side wait gave up (see gtm_last_error)     */
    GTM_ERR_WORKSPACE = -5,    /* workspace missing or smaller than *_workspace_bytes()       */
    GTM_ERR_MISALIGNED = -6    /* pointer or byte offset without the alignment a kernel needs */
} gtm_status;

/* Message for the last failing call on this thread, "" after a successful one. The pointer
 * stays valid until the next failing call on the same thread. */
GTM_API const char* gtm_last_error(void);
GTM_API const char* gtm_version(void);

/* ---------------------------------------------------------------------------------------
 * Device context, buffers and fences (replaces the D3D12Context calls the MoE path makes,
 * include/gturbo/d3d12_context.hpp:22-54). One CUDA stream per context; not thread-safe per
 * context, as the reference runs one generation at a time.
 * ------------------------------------------------------------------------------------- */

/* D3D12Context construction: a context on CUDA device `device` with its own stream. */
GTM_API int gtm_ctx_create(int device, void** ctx_out);
GTM_API int gtm_ctx_destroy(void* ctx);
/* The context's cudaStream_t (pass it as `stream` to the calls below). */
GTM_API void* gtm_ctx_stream(void* ctx);
/* create_uma_buffer (d3d12_context.cpp:135-160): device memory, 64-bit addresses (no 4 GB
 * root-descriptor limit, runner.cpp:330-333). */
GTM_API int gtm_buffer_alloc(void* ctx, uint64_t bytes, void** dev_out);
GTM_API int gtm_buffer_free(void* ctx, void* dev);
/* Host <-> device copies on the context's stream, ordered with the kernels submitted there. */
GTM_API int gtm_buffer_upload(void* ctx, void* dev, uint64_t offset, const void* host, uint64_t bytes);
GTM_API int gtm_buffer_download(void* ctx, void* host, const void* dev, uint64_t offset, uint64_t bytes);
/* submit_command_list -> fence value (d3d12_context.cpp:100-114): a ticket for all work issued
 * on the context's stream so far. */
GTM_API int gtm_submit(void* ctx, uint64_t* ticket_out);
/* wait_for_fence (d3d12_context.cpp:122-127) with a bound instead of INFINITE: GTM_OK when the
 * work up to `ticket` is done, GTM_ERR_TIMEOUT after timeout_ms. */
GTM_API int gtm_wait(void* ctx, uint64_t ticket, uint32_t timeout_ms);

/* ---------------------------------------------------------------------------------------
 * Kernel entry points (the reference's compute kernels, same arithmetic contract).
 * Quantised matrices use MLX affine 4-/8-bit, group 64 along the input dimension, packed
 * low nibble first, with bf16 scales and biases laid out [rows][in_dim/64].
 * ------------------------------------------------------------------------------------- */

/* GemvInt4 (shaders/GemvInt4.hlsl:18-38): out[r] = sum_c (q[r][c]*s + b) * x[c].
 * Arithmetic is bit-identical to the reference CPU matvec (src/cpu_reference.cpp:55-83). */
GTM_API int gtm_gemv_q4(uint32_t rows, uint32_t in_dim, const void* w_dev, const uint16_t* s_dev,
                        const uint16_t* b_dev, const float* x_dev, float* out_dev, void* stream);
/* GemvInt8 (shaders/GemvInt8.hlsl:13-33), unsigned bytes; bit-identical to
 * src/cpu_reference.cpp:86-106. */
GTM_API int gtm_gemv_q8(uint32_t rows, uint32_t in_dim, const void* w_dev, const uint16_t* s_dev,
                        const uint16_t* b_dev, const float* x_dev, float* out_dev, void* stream);
/* RouterTopK (shaders/RouterTopK.hlsl:23-68): top-k by (logit desc, index asc), softmax over
 * the k selected, times bf16 per_expert_scale. k <= 32, num_experts <= 1024. */
GTM_API int gtm_router_topk(uint32_t num_experts, uint32_t k, const float* logits_dev,
                            const uint16_t* per_expert_scale_dev, uint32_t* idx_dev,
                            float* weights_dev, void* stream);
/* GeGLU (shaders/GeGLU.hlsl:15-28): act = gelu_tanh(gate) * up. */
GTM_API int gtm_geglu(uint32_t n, const float* gate_dev, const float* up_dev, float* act_dev, void* stream);
/* ScaleAccum (shaders/ScaleAccum.hlsl:20-35): out = (accumulate ? out : 0) + weights[w_index] * in. */
GTM_API int gtm_scale_accum(uint32_t n, const float* in_dev, const float* weights_dev, uint32_t w_index,
                            int accumulate, float* out_dev, void* stream);
/* MulBF16 (shaders/MulBF16.hlsl:17-30): out = in * bf16(w) * scale. */
GTM_API int gtm_mul_bf16(uint32_t n, const float* in_dev, const uint16_t* w_dev, float scale,
                         float* out_dev, void* stream);
/* RMSNormK (shaders/RMSNormK.hlsl:25-61): out = x / sqrt(mean(x^2) + eps) * [bf16 w].
 * w_dev may be NULL. The mean of squares is formed exactly as src/cpu_reference.cpp:43-52
 * (double accumulation), so results are bit-identical with the CPU reference. n <= 65536. */
GTM_API int gtm_rmsnorm(uint32_t n, const float* x_dev, const uint16_t* w_dev, float eps,
                        float* out_dev, void* stream);
/* PostAttn (shaders/PostAttn.hlsl:43-84): hidden_out = hidden + rms(attn)*w_post, then the
 * three views dense_x = h*w_pre, routed_x = h*w_pre2, router_x = h with h = rms(hidden_out). */
GTM_API int gtm_post_attn(uint32_t d, const float* attn_dev, const float* hidden_dev,
                          const uint16_t* w_post_dev, const uint16_t* w_pre_dev, const uint16_t* w_pre2_dev,
                          float eps, float* hidden_out_dev, float* dense_x_dev, float* routed_x_dev,
                          float* router_x_dev, void* stream);
/* LayerTail (shaders/LayerTail.hlsl:39-78):
 * hidden_out = (hidden + rms(rms(h2)*w_pf2 + h1) * w_pf) * layer_scalar. */
GTM_API int gtm_layer_tail(uint32_t d, const float* h2_dev, const float* h1_dev, const float* hidden_dev,
                           const uint16_t* w_pf2_dev, const uint16_t* w_pf_dev, float eps, float layer_scalar,
                           float* hidden_out_dev, void* stream);

/* The same kernels over n vectors at once (a batched decode step; the reference dispatches one
 * vector per call). Row i of each [n][...] array is vector i; every row's result is
 * bit-identical to the single-vector entry on it. n <= 512. */
/* GemvInt4 of x_dev row i ([n][in_dim]) into out_dev row i ([n][rows]). */
GTM_API int gtm_gemv_q4_rows(uint32_t rows, uint32_t in_dim, uint32_t n, const void* w_dev, const uint16_t* s_dev,
                             const uint16_t* b_dev, const float* x_dev, float* out_dev, void* stream);
/* RMSNormK of each of `rows` vectors of n elements ([rows][n]). */
GTM_API int gtm_rmsnorm_rows(uint32_t rows, uint32_t n, const float* x_dev, const uint16_t* w_dev, float eps,
                             float* out_dev, void* stream);
/* PostAttn of each of `rows` vectors of d elements; the three views may be NULL (not written). */
GTM_API int gtm_post_attn_rows(uint32_t rows, uint32_t d, const float* attn_dev, const float* hidden_dev,
                               const uint16_t* w_post_dev, const uint16_t* w_pre_dev, const uint16_t* w_pre2_dev,
                               float eps, float* hidden_out_dev, float* dense_x_dev, float* routed_x_dev,
                               float* router_x_dev, void* stream);

/* Kernel ids for gtm_dispatch, in the order of gturbo::KernelType (include/gturbo/pipeline.hpp:17-33). */
typedef enum gtm_kernel {
    GTM_KERNEL_RMSNORMK = 1, GTM_KERNEL_GEMV_INT4 = 2, GTM_KERNEL_GEMV_INT8 = 3,
    GTM_KERNEL_ROUTER_TOPK = 6, GTM_KERNEL_GEGLU = 7, GTM_KERNEL_POST_ATTN = 8,
    GTM_KERNEL_LAYER_TAIL = 9, GTM_KERNEL_SCALE_ACCUM = 11, GTM_KERNEL_MUL_BF16 = 12
} gtm_kernel;

/* Drop-in for ComputePipelineManager::dispatch (src/pipeline.cpp:409-518): the same 16 root
 * constants (gp0..gp3) each HLSL kernel reads, with srv/uav device buffers bound in the same
 * slots (t0..t5 / u0..u3) and addressed by the constants' BYTE offsets. grid_x is accepted
 * for signature parity; the CUDA launch shape is chosen internally. Kernels outside the MoE
 * path return GTM_ERR_UNSUPPORTED. */
GTM_API int gtm_dispatch(int kernel, const void* const* srv_dev, int n_srv, void* const* uav_dev, int n_uav,
                         const uint32_t constants[16], uint32_t grid_x, void* stream);

/* ---------------------------------------------------------------------------------------
 * Fused MoE block, batch-1 decode (one token through 1..GTM_MAX_LAYERS layers).
 * ------------------------------------------------------------------------------------- */

#define GTM_MAX_LAYERS 64

/* Byte offsets of one affine-quantised matrix (weight, bf16 scales, bf16 biases). */
typedef struct GtmQuant {
    uint64_t weight, scales, biases;
} GtmQuant;

/* One layer's MoE weights: a resident-tensor base with byte offsets (the resident index's
 * file_offset / scale_offset / bias_offset, include/gturbo/resident_index.hpp:17-27) and the
 * layer's packed expert image (packed_experts/layer_NN.bin) with the layout.json expertBlock
 * offsets (include/gturbo/packed_experts.hpp:34-59). Nothing is re-packed. */
typedef struct GtmLayer {
    const void* resident_dev;
    GtmQuant router;                 /* model.layers.L.router.proj.weight (8-bit)          */
    uint64_t router_scale;           /* router.scale, bf16[hidden]                          */
    uint64_t per_expert_scale;       /* router.per_expert_scale, bf16[experts]              */
    GtmQuant shared_gate, shared_up, shared_down;       /* mlp.{gate,up,down}_proj          */
    uint64_t pre_ffn_norm;           /* pre_feedforward_layernorm.weight    -> dense_x      */
    uint64_t pre_ffn_norm_2;         /* pre_feedforward_layernorm_2.weight  -> routed_x     */
    uint64_t post_ffn_norm_1;        /* post_feedforward_layernorm_1.weight -> h1           */
    uint64_t post_ffn_norm_2;        /* post_feedforward_layernorm_2.weight (tail, h2)      */
    uint64_t post_ffn_norm;          /* post_feedforward_layernorm.weight   (tail)          */
    uint64_t layer_scalar;           /* layer_scalar, bf16[1]                               */
    const void* experts_dev;         /* expert e at experts_dev + e * expert_stride         */
    uint64_t expert_stride;
    GtmQuant expert_gate, expert_up, expert_down;       /* layout.expertBlock offsets       */
} GtmLayer;

/* Model dimensions. The fused kernels are built for Gemma-4-26B-A4B's MoE shape:
 * hidden 2816, moe_intermediate 704, ffn_intermediate 2112, 128 experts, top-8, group 64. */
typedef struct GtmDims {
    uint32_t hidden, moe_inter, ffn_inter, num_experts, top_k;
    float eps;
} GtmDims;

enum {
    GTM_DECODE_NORM_BETWEEN_LAYERS = 1,  /* weightless RMSNorm on the residual after every layer but the last */
    /* Test hook for the bounded device-side waits: the launch's first grid-barrier wait waits for
     * an epoch no CTA arrives with, under a 2 ms limit instead of 2 s, so every CTA gives up,
     * records GTM_ERR_TIMEOUT (read by gtm_moe_decode_check) and returns; outputs are not
     * written. The workspace stays usable for the next launch. */
    GTM_DECODE_TEST_WAIT_RUNS_OUT = 0x100
};

typedef struct GtmDecodeIO {
    const float* hidden_in_dev;      /* [hidden] block input of layer 0                     */
    float* hidden_out_dev;           /* [hidden] output of the last layer                   */
    /* Optional per-layer outputs (NULL to skip): */
    uint32_t* topk_idx_dev;          /* [layers][top_k]                                     */
    float* topk_w_dev;               /* [layers][top_k]                                     */
    float* logits_dev;               /* [layers][experts] router logits                      */
    float* h1_dev;                   /* [layers][hidden] normed shared-expert output         */
    float* h2_dev;                   /* [layers][hidden] weighted routed-expert sum          */
    float* hidden_layers_dev;        /* [layers][hidden] residual after each layer (after the
                                        between-layer norm when that flag is set)            */
    const float* logit_bias_dev;     /* [layers][experts] added to the router logits before
                                        selection (benchmark skew knob; NULL = none)         */
    uint32_t flags;                  /* GTM_DECODE_* */
} GtmDecodeIO;

/* Workspace needed by gtm_moe_decode (device memory, 256-byte aligned, owned by the caller).
 * Zero it once before its first use (cudaMemset); calls keep it consistent afterwards. A
 * workspace serves one stream at a time. Returns 0 for unsupported dims. */
GTM_API size_t gtm_moe_decode_workspace_bytes(const GtmDims* dims);
/* One token through `num_layers` MoE blocks in a single persistent launch: fused router
 * (int8 GEMV + top-k + softmax, bit-identical logits and indices with the CPU reference),
 * shared expert, the top-k experts' int4 gate/up + GeGLU and down + weighted combine, and the
 * layer tail, with no host round trip. Asynchronous: the call validates, launches and returns.
 * Device-side waits are bounded (2 s per grid barrier); a wait that gives up leaves the
 * outputs undefined and is reported by the next gtm_moe_decode_check on the workspace. */
GTM_API int gtm_moe_decode(const GtmDims* dims, const GtmLayer* layers, int num_layers,
                           const GtmDecodeIO* io, void* workspace_dev, size_t workspace_bytes,
                           void* stream);
/* Reads back and clears the device-side error flag of a workspace after gtm_moe_decode
 * calls (synchronises `stream`). Returns GTM_OK or GTM_ERR_TIMEOUT. */
GTM_API int gtm_moe_decode_check(void* workspace_dev, void* stream);
/* gtm_moe_decode without a caller workspace. No counterpart in the reference. For callers that
 * cannot allocate device memory (a bare C/FFI host with no device allocator, or a process that
 * reserves all device memory at start-up and forbids later allocation): the scratch is a
 * statically sized array of the library, 256 KB per device, so the call allocates nothing. The
 * first call on each device looks that array up and should come before any stream capture; the
 * address it keeps is the primary context's, so call from the primary context and do not reset
 * the device after the first call.
 * Every call on a device shares the one array: calls that overlap on the GPU race. layers ==
 * NULL with num_layers == 0 reads and clears the array's device-side error word instead
 * (synchronises `stream`; returns GTM_OK or GTM_ERR_TIMEOUT). */
GTM_API int gtm_moe_decode_noalloc(const GtmDims* dims, const GtmLayer* layers, int num_layers,
                                   const GtmDecodeIO* io, void* stream);

/* ---------------------------------------------------------------------------------------
 * MoE block for T > 1 tokens (batched decode, prefill): one layer, tokens grouped by expert.
 * The reference has no batched path (prefill runs the per-token chain, src/runner.cpp:845-854);
 * this replaces that loop for one layer with routing, a tcgen05 grouped GEMM over the routed
 * and shared experts, and the combine + layer tail.
 * ------------------------------------------------------------------------------------- */

typedef struct GtmTokensIO {
    uint32_t num_tokens;             /* T >= 1                                              */
    const float* x_dev;              /* [T][hidden] fp32 block input, or NULL ...           */
    const uint16_t* x_bf16_dev;      /* ... [T][hidden] bf16 block input                    */
    float* hidden_out_dev;           /* [T][hidden]                                         */
    /* Optional outputs (NULL to skip): */
    uint32_t* topk_idx_dev;          /* [T][top_k]                                          */
    float* topk_w_dev;               /* [T][top_k]                                          */
    float* logits_dev;               /* [T][experts] router logits after the bias           */
    float* h1_dev;                   /* [T][hidden] normed shared-expert output             */
    float* h2_dev;                   /* [T][hidden] weighted routed-expert sum              */
    /* Optional inputs: */
    const float* logit_bias_dev;     /* [experts] added to every token's logits (NULL = none) */
    const float* route_logits_dev;   /* [T][experts] routing logits given by the caller; the
                                        router GEMV is skipped (NULL = compute them)        */
    uint32_t flags;                  /* 0, or GTM_TOKENS_TEST_WAIT_RUNS_OUT (gtm_moe_tokens) */
} GtmTokensIO;

enum {
    /* Test hook for the grouped GEMM's bounded pipeline waits (gtm_moe_tokens only): in the
     * gate/up GEMM the MMA warp of every CTA first waits on a barrier nothing arrives at, under a
     * 2 ms limit instead of 1 s, gives up and raises the CTA's abort flag, so every role leaves
     * its loop, the CTA frees its tensor memory and GTM_ERR_TIMEOUT is recorded (read by
     * gtm_moe_tokens_check); outputs are not written. The workspace stays usable. */
    GTM_TOKENS_TEST_WAIT_RUNS_OUT = 0x100
};

/* Workspace for gtm_moe_tokens with up to `max_tokens` tokens (0 for unsupported dims).
 * Zero it once before its first use; a workspace serves one stream at a time. */
GTM_API size_t gtm_moe_tokens_workspace_bytes(const GtmDims* dims, uint32_t max_tokens);
/* One layer for io->num_tokens tokens. Routing (router logits in the reference's exact order,
 * bit-identical top-k indices), grouped expert products on the tensor cores with int4 dequant in
 * the kernel, combine in router order and the layer tail. Asynchronous; pipeline waits on the
 * device are bounded (1 s) and reported by gtm_moe_tokens_check. */
GTM_API int gtm_moe_tokens(const GtmDims* dims, const GtmLayer* layer, const GtmTokensIO* io,
                           void* workspace_dev, size_t workspace_bytes, void* stream);
/* Reads back and clears the device-side error flag (synchronises `stream`). */
GTM_API int gtm_moe_tokens_check(void* workspace_dev, void* stream);

/* Stage timing of gtm_moe_tokens with device events, replacing the reference's wall-clock
 * PerformanceMetrics timers around its fences (include/gturbo/runner.hpp:87-106,
 * src/runner.cpp:396-421). `events` are n caller-owned cudaEvent_t handles (created, timing
 * enabled); the calling thread's next gtm_moe_tokens calls record events[i] on their stream at
 * stage boundary i (for i < n): 0 before the views and router, 1 before the routing tables,
 * 2 before the grouped gate/up GEMM, 3 before the grouped down GEMM, 4 before the combine,
 * 5 after it. The handles are kept (not owned) until the next call; n = 0 turns it off. */
enum { GTM_PHASE_EVENTS = 6 };
GTM_API int gtm_set_phase_events(void* const* events, int n);

/* ---------------------------------------------------------------------------------------
 * Tied LM head with greedy argmax: LMHeadGreedy + ArgmaxReduce (shaders/LMHeadGreedy.hlsl:1-73,
 * shaders/ArgmaxReduce.hlsl:1-62; runner.cpp:720-770). token = argmax_r logits[r], ties to the
 * lower row, over the int4 matvec of x (the final-normed hidden state) with the embedding
 * matrix (rows = vocab, in_dim = hidden; group-64 bf16 scales and biases). The winning logit
 * is bit-identical to the CPU reference's (cpu_reference.cpp:55-83 order), so the token is the
 * reference's: every row is first evaluated on the tensor cores with a rigorous error bound,
 * and every row whose bound interval reaches the best lower bound is recomputed in the exact
 * CPU order. Softcap is monotonic and, as in the reference's greedy path, not applied.
 * ------------------------------------------------------------------------------------- */
GTM_API size_t gtm_lm_head_workspace_bytes(uint32_t rows);
/* in_dim must be 2816; rows >= 1. token_dev: uint32 on the device; logit_dev (nullable): the
 * exact logit of the token. Asynchronous on `stream`; the workspace needs no initialisation. */
GTM_API int gtm_lm_head_greedy(uint32_t rows, uint32_t in_dim, const void* w_dev, const uint16_t* s_dev,
                               const uint16_t* b_dev, const float* x_dev, uint32_t* token_dev, float* logit_dev,
                               void* workspace_dev, size_t workspace_bytes, void* stream);
/* Rows the last call on this workspace recomputed exactly (synchronises `stream`). */
GTM_API int gtm_lm_head_candidates(void* workspace_dev, void* stream, int32_t* count_out);

/* ---------------------------------------------------------------------------------------
 * Expert-parallel MoE layer: rank r of `world` owns experts [r*E/world, (r+1)*E/world) and
 * its own tokens. No reference counterpart (the reference is single-GPU). The caller moves
 * rows between ranks (NCCL all-to-all over NVLink) between the phases:
 *   1. gtm_moe_ep_dispatch  own tokens: views, router, top-k; one routed_x row per (token,
 *                           slot), grouped by destination rank in (token, slot) order. A row
 *                           is `hidden` 32-bit words (4*hidden bytes) holding the fp16 high
 *                           part then the fp16 low part of routed_x; the caller moves it as
 *                           opaque bytes
 *   2. gtm_moe_ep_shared    own tokens: shared expert (independent of the exchange; it uses
 *                           its own part of the workspace, so it may run on a second stream
 *                           concurrently with phase 3 once phase 1 has completed; phase 4
 *                           must follow both)
 *      -- all-to-all of send_counts, then of rows and metadata --
 *   3. gtm_moe_ep_experts   received rows through this rank's experts; result rows (fp32
 *                           expert outputs, routing weight not applied) in the order the rows
 *                           were received
 *      -- all-to-all back, with the split sizes reversed --
 *   4. gtm_moe_ep_combine   own tokens: h2 = sum over the slots in router order of routing
 *                           weight x returned row, layer tail
 * With world = 1 the four phases compute what gtm_moe_tokens computes.
 * ------------------------------------------------------------------------------------- */

typedef struct GtmEpMeta {
    uint32_t expert;                 /* global expert id                                    */
    float weight;                    /* routing weight of the (token, slot)                 */
} GtmEpMeta;

#define GTM_EP_MAX_WORLD 64

/* One rank's view of the expert-parallel group. world divides the expert count; the rank
 * owns experts [rank*E/world, (rank+1)*E/world). Every phase of the rank gets the same
 * config and the same workspace. */
typedef struct GtmEpConfig {
    uint32_t world, rank;
    uint32_t max_tokens;             /* own tokens per call, at most                        */
    uint32_t max_recv_rows;          /* rows received for this rank's experts, at most      */
} GtmEpConfig;

/* Workspace for the EP phases of one rank (0 for unsupported dims or sizes). Zero it once
 * before its first use. */
GTM_API size_t gtm_moe_ep_workspace_bytes(const GtmDims* dims, const GtmEpConfig* ep);
/* send_rows_dev: [num_tokens * top_k][hidden] 32-bit words (see phase 1); send_meta_dev: [num_tokens * top_k];
 * send_counts_dev: [world] device int32, rows for each destination rank. */
GTM_API int gtm_moe_ep_dispatch(const GtmDims* dims, const GtmLayer* layer, const GtmTokensIO* io,
                                const GtmEpConfig* ep, float* send_rows_dev, GtmEpMeta* send_meta_dev,
                                int32_t* send_counts_dev, void* workspace_dev, size_t workspace_bytes, void* stream);
GTM_API int gtm_moe_ep_shared(const GtmDims* dims, const GtmLayer* layer, const GtmTokensIO* io,
                              const GtmEpConfig* ep, void* workspace_dev, size_t workspace_bytes, void* stream);
/* layer->experts_dev points at this rank's first expert (its slice of the expert image); every
 * received row names one of the rank's experts. ret_rows_dev: [n_recv][hidden] fp32, in the
 * order of recv_rows_dev. n_recv = 0 is a no-op. */
GTM_API int gtm_moe_ep_experts(const GtmDims* dims, const GtmLayer* layer, const GtmEpConfig* ep,
                               const float* recv_rows_dev, const GtmEpMeta* recv_meta_dev, uint32_t n_recv,
                               float* ret_rows_dev, void* workspace_dev, size_t workspace_bytes, void* stream);
/* ret_rows_dev: the returned rows in this rank's send order ([num_tokens * top_k][hidden]). */
GTM_API int gtm_moe_ep_combine(const GtmDims* dims, const GtmLayer* layer, const GtmTokensIO* io,
                               const GtmEpConfig* ep, const float* ret_rows_dev, void* workspace_dev,
                               size_t workspace_bytes, void* stream);
/* Reads back and clears the device-side error flag of an EP workspace (synchronises `stream`). */
GTM_API int gtm_moe_ep_check(void* workspace_dev, void* stream);

/* ---------------------------------------------------------------------------------------
 * Expert-parallel MoE layer over peer memory. No reference counterpart. The ranks of one
 * NVLink domain map each other's workspaces (gtm_ipc_* below, or any other peer mapping) and
 * the kernels move the data themselves with plain peer loads and stores; there is no
 * all-to-all and no host round trip. Every rank uses the same config (world, max_tokens;
 * max_recv_rows is ignored: room for world * max_tokens * top_k rows is always reserved),
 * so the workspaces have the same layout. One layer:
 *   1. gtm_moe_ep_peer_dispatch  own tokens: views, router, top-k; stores the top-8 ids and
 *                                the token count into every rank's workspace and each token's
 *                                routed view into the workspaces of the ranks that own one of
 *                                its experts (NVLink stores)
 *   2. gtm_moe_ep_peer_shared    own tokens: shared expert; may run on a second stream
 *                                concurrently with phase 3 once phase 1 has completed
 *      -- barrier: every rank has completed phase 1 --
 *   3. gtm_moe_ep_peer_experts   this rank's experts over every rank's (token, slot) entries,
 *                                read from the own workspace; each expert output row is stored
 *                                into its token's rank's workspace (routing weight not
 *                                applied); rows of one expert keep the source-rank-major entry
 *                                order, so the results match gtm_moe_tokens on the whole batch
 *      -- barrier: every rank has completed phase 3 --
 *   4. gtm_moe_ep_peer_combine   own tokens: h2 = sum over the slots in router order of
 *                                routing weight x expert output, layer tail (after phase 2)
 * The barriers are the caller's (a stream-ordered one-element all-reduce over NCCL is
 * enough: a kernel's peer stores are complete at system scope when it ends). The second
 * barrier also keeps the next layer's phase 1 from overwriting rows a peer still reads.
 * Phases 1 and 3 take every rank's workspace (GtmEpPeers); 2 and 4 only the own one.
 * ------------------------------------------------------------------------------------- */
#define GTM_EP_PEER_MAX_WORLD 8

/* Every rank's workspace, indexed by rank, as mapped in this process (own one included). */
typedef struct GtmEpPeers {
    void* workspace_dev[GTM_EP_PEER_MAX_WORLD];
} GtmEpPeers;

/* Workspace of one rank (0 for unsupported dims or config: world must divide 128 and be at
 * most GTM_EP_PEER_MAX_WORLD, world * max_tokens at most 65536). Zero it once before its first
 * use (gtm_ipc_alloc returns it zeroed). */
GTM_API size_t gtm_moe_ep_peer_workspace_bytes(const GtmDims* dims, const GtmEpConfig* ep);
/* peers->workspace_dev[ep->rank] is the own workspace. */
GTM_API int gtm_moe_ep_peer_dispatch(const GtmDims* dims, const GtmLayer* layer, const GtmTokensIO* io,
                                     const GtmEpConfig* ep, const GtmEpPeers* peers, size_t workspace_bytes,
                                     void* stream);
GTM_API int gtm_moe_ep_peer_shared(const GtmDims* dims, const GtmLayer* layer, const GtmTokensIO* io,
                                   const GtmEpConfig* ep, void* workspace_dev, size_t workspace_bytes,
                                   void* stream);
/* layer->experts_dev points at this rank's first expert; peers->workspace_dev[ep->rank] is the
 * own workspace. */
GTM_API int gtm_moe_ep_peer_experts(const GtmDims* dims, const GtmLayer* layer, const GtmEpConfig* ep,
                                    const GtmEpPeers* peers, size_t workspace_bytes, void* stream);
GTM_API int gtm_moe_ep_peer_combine(const GtmDims* dims, const GtmLayer* layer, const GtmTokensIO* io,
                                    const GtmEpConfig* ep, void* workspace_dev, size_t workspace_bytes,
                                    void* stream);

/* Device memory shared between the processes of one box (CUDA IPC; peer access is enabled
 * when a handle is opened). gtm_ipc_alloc returns zeroed memory and its 64-byte handle;
 * another process opens the handle to map the same memory. Close what was opened before the
 * owner frees it. */
#define GTM_IPC_HANDLE_BYTES 64
GTM_API int gtm_ipc_alloc(size_t bytes, void** dev_ptr, uint8_t handle_out[GTM_IPC_HANDLE_BYTES]);
GTM_API int gtm_ipc_open(const uint8_t handle[GTM_IPC_HANDLE_BYTES], void** dev_ptr);
GTM_API int gtm_ipc_close(void* dev_ptr);
GTM_API int gtm_ipc_free(void* dev_ptr);

#ifdef __cplusplus
}
#endif
#endif /* GTMOE_H */
