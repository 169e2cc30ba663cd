/*
 * moestream_cuda.h — C ABI of the moe-stream B200 (sm_100a) backend.
 *
 * This library replaces the Metal compute backend of moe-stream-core for the quantized
 * MoE decode step.  Each entry point names the reference function or call site it stands
 * in for (paths relative to the moe-stream repository, moe-stream-core/src/...).  All
 * arguments are plain pointers and sizes; "d_" pointers are device memory (allocate them
 * with ms_malloc or any CUDA allocator on the context's device), other pointers are host
 * memory.  Every call returns an ms_status; no C++ exception crosses this boundary.  A
 * context is not thread-safe: use it from one host thread, as the reference Engine is used
 * from its single engine thread (moe-stream-server/src/engine_handle.rs:88-93).
 */
#ifndef MOESTREAM_CUDA_H
#define MOESTREAM_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MS_ABI_VERSION 4

#if defined(__GNUC__)
#define MS_API __attribute__((visibility("default")))
#else
#define MS_API
#endif

/* Status codes (the Rust shim maps them to candle_core::Error::Msg with ms_last_error()). */
typedef enum ms_status {
  MS_OK = 0,
  MS_ERR_INVALID_ARG = 1,
  MS_ERR_OOM = 2,
  MS_ERR_CUDA = 3,
  MS_ERR_NCCL = 4,
  MS_ERR_TIMEOUT = 5,          /* a device-side bounded wait expired (see ms_ctx_error_flags) */
  MS_ERR_UNSUPPORTED_QTYPE = 6,
  MS_ERR_SHAPE = 7,
  MS_ERR_IO = 8,
  MS_ERR_FORMAT = 9,           /* malformed GGUF */
  MS_ERR_STATE = 10,           /* call out of order (e.g. step before finalize) */
  MS_ERR_DEVICE_INDEX = 11     /* a token / expert index outside its table was seen on the device */
} ms_status;

/* GGML tensor type ids, as gguf/reader.rs:38-65 (GgmlQuantType). */
typedef enum ms_qtype {
  MS_Q_F32 = 0,
  MS_Q_F16 = 1,
  MS_Q_Q8_0 = 8,
  MS_Q_Q4_K = 12,
  MS_Q_Q6_K = 14,
  MS_Q_MXFP4 = 39
} ms_qtype;

/* Architecture switches the reference derives from general.architecture (layer.rs:774). */
typedef enum ms_arch {
  MS_ARCH_GPT_OSS = 0,   /* OAI SwiGLU (clamp 7, alpha 1.702), softmax over the selected top-k */
  MS_ARCH_QWEN_MOE = 1   /* SiLU*up, softmax over all experts then top-k (+renormalise) */
} ms_arch;

typedef struct ms_ctx ms_ctx;
typedef struct ms_model ms_model;

MS_API int ms_abi_version(void);
MS_API const char* ms_status_string(ms_status s);

/* ---- context (replaces Device::new_metal, engine.rs:277-298) ---- */
MS_API ms_status ms_ctx_create(int device, ms_ctx** out);
/* Also destroys any model of this context that is still open (its handle becomes invalid). */
MS_API ms_status ms_ctx_destroy(ms_ctx* ctx);
/* Enqueue work on a caller-owned cudaStream_t (NULL = the legacy default stream). */
MS_API ms_status ms_ctx_set_stream(ms_ctx* ctx, void* cuda_stream);
/* Enqueue work on the context's own non-blocking stream (the default after ms_ctx_create). */
MS_API ms_status ms_ctx_use_own_stream(ms_ctx* ctx);
/* Wait for the stream; reports MS_ERR_TIMEOUT / MS_ERR_DEVICE_INDEX raised by device code. */
MS_API ms_status ms_sync(ms_ctx* ctx);
MS_API const char* ms_last_error(const ms_ctx* ctx);
/* Device error word (bit 0/1: wait timeouts, bit 2: bad index, bit 3: bad shape); clear if nonzero. */
MS_API ms_status ms_ctx_error_flags(ms_ctx* ctx, uint32_t* flags, int clear);
MS_API int ms_ctx_sm_count(const ms_ctx* ctx);

/* ---- device memory (so an FFI caller needs no CUDA runtime of its own) ---- */
MS_API ms_status ms_malloc(ms_ctx* ctx, size_t bytes, void** d_ptr);
MS_API ms_status ms_free(ms_ctx* ctx, void* d_ptr);
MS_API ms_status ms_memcpy_h2d(ms_ctx* ctx, void* d_dst, const void* src, size_t bytes);   /* synchronous */
MS_API ms_status ms_memcpy_d2h(ms_ctx* ctx, void* dst, const void* d_src, size_t bytes);   /* synchronous */

/* ---- kernels on device pointers (the metal/mod.rs seam, one entry per dispatch) ---- */

/* Block dequantization to f32, bit-exact with gguf/dequant.rs (dequantize_mxfp4 605-628,
 * dequantize_q4k 218-262, dequantize_q6k 335-378, dequantize_q80 511-531, f16 37-41). */
MS_API ms_status ms_dequantize(ms_ctx* ctx, int qtype, const void* d_blocks, int64_t n_elements, float* d_out);

/* y = x * rsqrt(mean(x^2) + eps) * w per row; replaces fused_rms_norm_metal (metal/mod.rs:290-371). */
MS_API ms_status ms_rms_norm(ms_ctx* ctx, const float* d_x, const float* d_w, float* d_y, int rows, int dim, float eps);

/* y = W x (+bias) for one token, W [rows, cols] in native blocks.  Replaces
 * mxfp4_matmul_metal_gpu (metal/mod.rs:896-962) for MXFP4 and the CPU QMatMul / dequant matmul
 * of Q4_K and Q6_K (model/layer.rs:1516-1748; W allocation padded to 16 rows),
 * quantized_attn_matmul_metal_gpu_batched (metal/mod.rs:1123-1141) for Q8_0 (activation quantized
 * to Q8_0 as the CPU QMatMul path does), and the dense f16/f32 matmuls. */
MS_API ms_status ms_gemv(ms_ctx* ctx, int qtype, const void* d_w, int rows, int cols, const float* d_x,
                  const float* d_bias, float* d_y);

/* RMSNorm + router GEMV + bias + dummy-expert mask + top-k + routing weights for one token.
 * Replaces softmax_topk_kernel's dispatch (metal/mod.rs:1560-1602) and layer.rs:806-837,
 * 1016-1027, 2346-2403.  d_mask may be NULL (1 = dummy expert).  Ties pick the lower index. */
MS_API ms_status ms_router_topk(ms_ctx* ctx, const float* d_h, const float* d_norm_w, float eps, const float* d_router_w,
                         const float* d_router_b, const uint8_t* d_mask, int hidden, int n_experts, int top_k,
                         int arch, int norm_topk_prob, float* d_xn, float* d_logits, int32_t* d_idx, float* d_wts);

/* RoPE, NeoX half-rotation of the first rot_dim dims of every head (dims beyond pass through):
 * y = rope(x), x / y [n_tokens][heads][head_dim] (y must not overlap x), per-token tables
 * cos / sin [n_tokens][rot_dim / 2] already sliced at each token's position.  Replaces
 * fused_rope_metal (metal/mod.rs:383-472) and rotary_embedding / partial_rotary_embedding
 * (ops/attention.rs:49-164). */
MS_API ms_status ms_rope(ms_ctx* ctx, const float* d_x, const float* d_cos, const float* d_sin, int n_tokens,
                         int heads, int head_dim, int rot_dim, float* d_y);

/* One token drawn from logits (SamplingParams::sample, engine.rs:124-208): d_logits [V] f32,
 * d_counts [V] times each token was generated (repetition penalty; NULL = none), r the uniform
 * draw in [0, 1), d_work [V] f32 scratch, *d_token the result (device memory).  Sums of
 * probabilities are exact to 2^-109 and rounded to f32 once, so the result does not depend on
 * summation order. */
MS_API ms_status ms_sample(ms_ctx* ctx, const float* d_logits, int V, const uint32_t* d_counts, float temperature,
                           float top_p, float repetition_penalty, float r, float* d_work, int32_t* d_token);

/* One attention half-layer in device memory (layer.rs:511-749 for a single decode token). */
typedef struct ms_attn_layer {
  int hidden, heads, kv_heads, head_dim, rot_dim;
  float eps;                  /* RMSNorm epsilon (attention norm and QK-norm) */
  int window;                 /* > 0: sliding window (the cache is a ring of `window` slots) */
  int cap;                    /* cache slots per kv head (== window for a sliding-window layer) */
  const float* attn_norm;     /* [hidden] */
  const void* wqkv;           /* Q8_0 [heads*hd + 2*kv_heads*hd, hidden]: q, k, v rows concatenated */
  const float* bqkv;          /* [heads*hd + 2*kv_heads*hd] or NULL */
  const void* wo;             /* Q8_0 [hidden, heads*hd] */
  const float* bo;            /* [hidden] or NULL */
  const float* sinks;         /* [heads] or NULL */
  const float* q_norm;        /* [head_dim] QK-RMSNorm weights, or NULL (both or neither) */
  const float* k_norm;
  float* k_cache;             /* f32 [kv_heads][cap][head_dim], updated in place */
  float* v_cache;
  const float* cos_t;         /* RoPE tables [max_seq][rot_dim / 2] */
  const float* sin_t;
  int q_gate;                 /* 1 (hybrid models, layer.rs:620-635, 699-705): wqkv's first 2*heads*hd rows
                                 (and bqkv's) hold [Q_h, gate_h] per head, and the attention output is
                                 multiplied by sigmoid(gate) before the O projection; 0 otherwise */
} ms_attn_layer;

/* h += O(SDPA(RoPE(QKV(RMSNorm(h))))) for one token at position pos, appending its K/V to the
 * cache (slot pos, or pos % window).  Q8_0 projections with the activation quantized to Q8_0
 * (candle QMatMul numerics), GQA, attention sinks, sliding window.  Replaces the per-layer attention
 * dispatch of the Metal decode path (quantized_attn_matmul_metal_gpu_batched, metal/mod.rs:1123,
 * fused_rope_metal 383, and LayerForward's attention branch, model/layer.rs:393-503, 511-749). */
MS_API ms_status ms_attn_layer_decode(ms_ctx* ctx, const ms_attn_layer* layer, int pos, float* d_h);

/* One-token MXFP4 expert FFN with weighted combine into the residual stream:
 * d_h += sum over selected experts e (ascending id) of w_e * (Wd_e act_e + bd_e),
 * act_e = SwiGLU(Wg_e x + bg_e, Wu_e x + bu_e).  Replaces gpu_routed_moe_forward_metal
 * (metal/mod.rs:1512-1677: mxfp4_fused_gate_up_swiglu_f32 + mxfp4_fused_down_accum_f32).
 * Weights are the stacked GGUF tensors blk.N.ffn_{gate,up,down}_exps in native layout;
 * biases may be NULL.  Uses device scratch owned by the context. */
MS_API ms_status ms_moe_mxfp4_decode(ms_ctx* ctx, const void* d_gate, const void* d_up, const void* d_down,
                              const float* d_gate_b, const float* d_up_b, const float* d_down_b, int hidden,
                              int inter, int n_experts, int top_k, int arch, const float* d_x, const int32_t* d_idx,
                              const float* d_wts, float* d_h);

/* Allocation-free variant of ms_moe_mxfp4_decode, for callers that cannot allocate device
 * memory when they run the MoE step (a fixed memory pool owns the whole budget, or the
 * step runs where cudaMalloc is not allowed).  No counterpart in the reference: the Metal
 * path allocates its routing buffers up front.  Same arguments and result as
 * ms_moe_mxfp4_decode; the scratch lives in one fixed device array of 512 KiB that every
 * GPU loading this library keeps until exit, so top_k <= 16, hidden <= 4096 and
 * inter <= 4096 (larger sizes return MS_ERR_SHAPE).  The first call on a device looks up
 * the array's device address; make that first call before any stream capture, and do not
 * use the entry point across a cudaDeviceReset (the looked-up address would be stale).
 * Every call shares the array: calls that overlap on the GPU (other streams or contexts on
 * the same device) race and must be serialised by the caller.  The calling thread's current
 * device is left as it was. */
MS_API ms_status ms_moe_mxfp4_decode_noalloc(ms_ctx* ctx, const void* d_gate, const void* d_up, const void* d_down,
                                             const float* d_gate_b, const float* d_up_b, const float* d_down_b,
                                             int hidden, int inter, int n_experts, int top_k, int arch,
                                             const float* d_x, const int32_t* d_idx, const float* d_wts, float* d_h);

/* ---- MXFP4 experts in the tensor-core layout ----
 * The model loader repacks MXFP4 experts into 128-row tiles that the 5th-generation tensor cores
 * read directly (block-scaled e2m1 x e2m1 MMA, ue8m0 scales; values unchanged).  These entry points
 * expose the same path for caller-owned buffers (replaces GpuExpertProjection / PackedMxfp4Layer
 * packing, metal/cache.rs:30-81, 289-308, and upload_mxfp4_weights, metal/mod.rs:1823).
 * Bytes of the packed gate+up and down stacks of n_experts experts (hidden, inter multiples of 64). */
MS_API ms_status ms_mxfp4_packed_bytes(int hidden, int inter, int n_experts, size_t* gate_up_bytes,
                                       size_t* down_bytes);
/* Repack device-resident native stacks (gate/up [E, inter, hidden], down [E, hidden, inter], GGUF
 * MXFP4 blocks) into device buffers sized by ms_mxfp4_packed_bytes.  Enqueued on the ctx stream. */
MS_API ms_status ms_mxfp4_pack_experts(ms_ctx* ctx, const void* gate, const void* up, const void* down, int hidden,
                                       int inter, int n_experts, void* gate_up_packed, void* down_packed);
/* ms_moe_mxfp4_decode over packed experts: h += sum_k w_k * FFN_{idx_k}(x) (ascending expert order). */
MS_API ms_status ms_moe_mxfp4_decode_packed(ms_ctx* ctx, const void* gate_up_packed, const void* down_packed,
                                            const float* gate_b, const float* up_b, const float* down_b, int hidden,
                                            int inter, int n_experts, int top_k, int arch, const float* x,
                                            const int32_t* idx, const float* wts, float* h);
/* Batched prefill of one MoE layer over T tokens (replaces the multi-token expert branches,
 * model/layer.rs:1316-1349, 1848-1894): tokens sorted by expert, a grouped GEMM on the tensor cores
 * with the MXFP4 weights expanded exactly to bf16 in shared memory and bf16 activations, f32
 * accumulation; out[t] = sum over the token's experts (ascending id) of w * FFN(x[t]).
 * x [T, hidden], idx / wts [T, top_k], out [T, hidden], device pointers; packed experts as above.
 * precise = 1 carries each activation as a bf16 hi + lo pair (two MMAs per K step, ~2^-18 relative
 * instead of bf16's 2^-9; about twice the tensor time). */
MS_API ms_status ms_moe_mxfp4_prefill_packed(ms_ctx* ctx, const void* gate_up_packed, const void* down_packed,
                                             const float* gate_b, const float* up_b, const float* down_b, int hidden,
                                             int inter, int n_experts, int top_k, int arch, const float* x,
                                             int n_tokens, const int32_t* idx, const float* wts, float* out,
                                             int precise);

/* ---- lockstep batch: B sequences at one shared position (Engine::forward over input_ids
 *      [B, T], engine.rs:1869-2006, KV rows per batch entry kv_cache.rs:37-60) ----
 * Every weight byte is streamed once per step for the whole batch: Q8_0 projections as int8 MMA
 * over the batch, experts grouped by id (each expert once per group of <= 4 tokens), LM head as
 * f16 MMA.  Needs native-layout experts (K-quants, or MXFP4 with MS_MOE_TC=0) and ep_size 1. */
MS_API ms_status ms_model_batch_open(ms_model* m, int batch);     /* allocates B KV caches, 1 <= B <= 32 */
MS_API ms_status ms_model_batch_close(ms_model* m);
MS_API ms_status ms_model_batch_clear(ms_model* m);               /* all sequences back to length 0 */
/* tokens [B][T] (row per sequence); next [B] = greedy token after the last position (or NULL) */
MS_API ms_status ms_model_batch_forward(ms_model* m, const int32_t* tokens, int n_tokens, int32_t* next);
/* n greedy steps, each step's argmax fed back on the device (no host sync) */
MS_API ms_status ms_model_batch_decode_steps_device(ms_model* m, int n_steps);
MS_API ms_status ms_model_batch_next_tokens(ms_model* m, int32_t* next);          /* [B] */
/* tokens fed per step, [rows][B] */
MS_API ms_status ms_model_batch_token_log(ms_model* m, int32_t* out, int max_rows, int* n_rows);
MS_API ms_status ms_model_batch_last_logits(ms_model* m, float* out);             /* [B][vocab] */
MS_API int ms_model_batch_kernels_per_step(const ms_model* m);
/* device microseconds per batch step of each launch class alone (step start, QKV, attention, O,
 * router, expert grouping, gate_up, down, residual, LM head) */
MS_API ms_status ms_model_batch_profile_step(ms_model* m, float* us, int max, int* n);

/* ---- hybrid (Qwen3.5 / Qwen3-Next) blocks ---- */
/* One Gated DeltaNet layer in device memory.  Projections are in native blocks (qtype as in
 * ms_gemv): qkv [2*n_k_heads*head_k_dim + n_v_heads*head_v_dim, hidden] (q, k, v rows),
 * gate (z) [n_v_heads*head_v_dim, hidden], ba [2*n_v_heads, hidden] (beta rows, then alpha rows),
 * out [hidden, n_v_heads*head_v_dim]; f32 conv1d [conv_dim, conv_kernel], ssm_a, dt_bias
 * [n_v_heads], norm [head_v_dim].  Mirrors the layer tensors deltanet.rs:204-260 reads. */
typedef struct ms_deltanet_layer {
  int hidden, n_k_heads, head_k_dim, n_v_heads, head_v_dim, conv_kernel;
  float eps;
  int qkv_q;  const void* qkv;
  int gate_q; const void* gate;
  int ba_q;   const void* ba;
  int out_q;  const void* out;
  const float *conv1d, *ssm_a, *dt_bias, *norm;
} ms_deltanet_layer;

/* One DeltaNet decode token (deltanet.rs:204-543): y = out(gated RMSNorm(delta-rule(conv(qkv x))))
 * with conv_state [conv_dim, conv_kernel-1] and rec_state [n_v_heads, head_k_dim, head_v_dim]
 * (f32, device) updated in place.  head_v_dim must be 128 and head_k_dim <= 128 (even). */
MS_API ms_status ms_deltanet_decode(ms_ctx* ctx, const ms_deltanet_layer* layer, const float* d_x,
                                    float* d_conv_state, float* d_rec_state, float* d_y);

/* y += sigmoid(x . gate_inp) * down(silu(gate x) * up x) for one token (layer.rs:2250-2293 and
 * its caller layer.rs:910-925).  gate_inp may be NULL (no scaling). */
MS_API ms_status ms_shared_expert(ms_ctx* ctx, int gate_up_qtype, const void* d_gate, const void* d_up,
                                  int down_qtype, const void* d_down, const float* d_gate_inp, int hidden,
                                  int inter, const float* d_x, float* d_y);

/* ---- model: the Engine surface (engine.rs open_with_device / preload_weights / forward /
 *      generate / clear_cache) ---- */
typedef struct ms_model_config {
  int arch;             /* ms_arch */
  int hidden, layers, heads, kv_heads, head_dim, rot_dim;
  int experts, top_k, inter, vocab;
  float rope_theta, eps;
  int sliding_window;   /* > 0: even layers attend to the last `sliding_window` positions */
  int norm_topk_prob;
  int max_seq_len;      /* RoPE table and KV capacity */
  int ep_rank, ep_size; /* expert parallel placement (single GPU: 0, 1) */
  int attn_splits;      /* split-K factor of decode attention, 0 = automatic */
  /* Gated DeltaNet hybrids (Qwen3-Next / Qwen3.5, config.rs:318-352, 446-494).  attn_interval > 0:
   * layer l is gated attention (Q projection [Q_h, gate_h] per head, output x sigmoid(gate),
   * layer.rs:620-635, 699-705) when (l + 1) % attn_interval == 0, else a Gated DeltaNet layer with
   * ssm_groups key heads of ssm_state dims, ssm_dt_rank value heads of ssm_inner / ssm_dt_rank (= 128)
   * dims and a causal conv of ssm_conv taps (tensors blk.N.attn_qkv / attn_gate / ssm_ba (or ssm_beta +
   * ssm_alpha) / ssm_out / ssm_conv1d / ssm_a / ssm_dt.bias / ssm_norm, deltanet.rs:101-137, 204-543).
   * 0: every layer is attention and the ssm fields are ignored.  Any model may also carry a shared
   * expert per layer (blk.N.ffn_{gate,up,down}_shexp, ffn_gate_inp_shexp; layer.rs:910-922). */
  int attn_interval;
  int ssm_groups, ssm_state, ssm_dt_rank, ssm_inner, ssm_conv;
} ms_model_config;

/* Create an empty model; then ms_model_set_tensor for every tensor and ms_model_finalize. */
MS_API ms_status ms_model_create(ms_ctx* ctx, const ms_model_config* cfg, ms_model** out);
/* Upload one GGUF-named tensor in its native block layout (no re-quantization).  dims are in
 * PyTorch order ([n_exp, rows, cols] for stacked experts).  Replaces preload_gates /
 * preload_attention / preload_experts_gpu (engine.rs:606-667, 674-921, 1079-1369). */
MS_API ms_status ms_model_set_tensor(ms_model* m, const char* name, int qtype, int n_dims, const int64_t* dims,
                              const void* host_data, size_t bytes);
MS_API ms_status ms_model_finalize(ms_model* m);
/* Expert parallelism (no counterpart in the reference, which runs on one device): a model
 * created with ep_size > 1 holds experts [ep_rank*E/ep_size, (ep_rank+1)*E/ep_size) and sums
 * each layer's MoE output over the group with an NCCL all-reduce inside the decode step.
 * Rank 0 calls ms_nccl_unique_id, the caller broadcasts the 128 bytes to every rank, and
 * each rank calls ms_model_init_ep before its first forward. */
MS_API ms_status ms_nccl_unique_id(ms_ctx* ctx, void* out, size_t bytes);
MS_API ms_status ms_model_init_ep(ms_model* m, const void* unique_id, size_t bytes);
/* Expert parallel over NVLink peer memory instead of NCCL: each rank gets its mailbox's CUDA IPC
 * handle (64 bytes), the caller gathers all ranks' handles in rank order (any host channel) and
 * passes them to ms_model_ep_connect.  Each layer's local MoE combine is then stored directly into
 * every rank's mailbox by one kernel, and the residual kernel sums the ranks' partials in rank
 * order after a bounded wait on their flags. */
MS_API ms_status ms_model_ep_handle(ms_model* m, void* out, size_t bytes);
MS_API ms_status ms_model_ep_connect(ms_model* m, const void* handles, size_t bytes);
/* Parse a GGUF file (reader.rs:259-368, config.rs:253-434) and upload everything. */
MS_API ms_status ms_model_open_gguf(ms_ctx* ctx, const char* path, int max_seq_len, int ep_rank, int ep_size,
                             ms_model** out);
/* Dynamic K (layer.rs:947-1011, entropy_to_k layer.rs:2329-2334; config.rs:183-192, 468-483): each
 * decode step's router computes the entropy H of softmax(router logits) per layer and routes
 * K = round(k_lo + clamp(H / ln E, 0, 1) (k_hi - k_lo)) experts, k_lo / k_hi = [k_min, k_max], or with
 * layer_adaptive the depth tier of LayerTierConfig::default_for_k(k_max) (first 15 % of layers
 * [k_max, k_max], up to 85 % [min(4, k_max), max(4, 2 k_max / 3)], then [max(4, 2 k_max / 3), k_max]).
 * 1 <= k_min <= k_max <= top_k; slots past K report expert id n_experts and weight 0.  Every prompt
 * token is then its own step (the reference takes one K per forward call from the mean entropy of
 * its tokens, which is the same for one-token calls).  Not with the lockstep batch. */
MS_API ms_status ms_model_set_dynamic_k(ms_model* m, int enable, int k_min, int k_max, int layer_adaptive);
/* Router statistics (the entropy_out / routing_stats_out of LayerForward::forward, layer.rs:393-503):
 * enable != 0 makes every later step record each layer's router entropy and the K it routed;
 * ms_model_router_stats reads those of the last step, entropy [layers] and k [layers] (either may be
 * NULL).  The routed ids and weights themselves come from ms_model_last_routing. */
MS_API ms_status ms_model_set_router_stats(ms_model* m, int enable);
MS_API ms_status ms_model_router_stats(ms_model* m, float* entropy, int32_t* k);
/* Running totals since router statistics were last enabled (RoutingStatsCollector and EntropyProfiler,
 * model/cache.rs:404-580, kept on the device and updated by every step's router): counts
 * [layers][n_experts] times each expert was routed, weight_sums [layers][n_experts] the sum of its
 * routing weights (f64, in step order), tokens [layers] steps seen, and entropy_log
 * [min(steps, max_steps)][layers] each step's router entropy (the log holds max_seq_len steps);
 * *n_steps = steps logged.  Any pointer may be NULL.  frequency = count / tokens, mean gate weight =
 * weight_sum / count and importance = frequency x mean gate weight follow on the host. */
MS_API ms_status ms_model_router_totals(ms_model* m, uint64_t* counts, double* weight_sums, uint64_t* tokens,
                                        float* entropy_log, int max_steps, int* n_steps);
/* Host-tier expert streaming (the reference's SSD / mmap streaming mode with its per-layer expert LRU,
 * gguf/reader.rs:631-858, model/layer.rs:1146-1152, 1777-1784, model/cache.rs:84-158).  Call after
 * ms_model_create and before the expert tensors are set: every layer's K-quant expert stacks (Q4_K /
 * Q6_K, still in their block format) are then kept in pinned host memory and HBM holds `slots`
 * experts per layer (slots >= top_k; 0 turns the tier off).  At each layer the step waits for the
 * router, copies the routed experts that are not cached into the least recently used slots not
 * routed this step, and runs the same expert kernels on the slots, so logits and tokens are the same
 * bits as with HBM-resident experts.  The step is then enqueued per call (no captured graph, one host
 * synchronisation per layer); prompts run one decode step per token; the lockstep batch path and
 * expert parallelism are not available.  Needs the order-independent numerics (ms_model_set_exact 1). */
MS_API ms_status ms_model_set_expert_tier(ms_model* m, int slots);
/* Expert-slot hits and misses since the model was created (ExpertCache::stats, cache.rs:144-158). */
MS_API ms_status ms_model_expert_tier_stats(const ms_model* m, uint64_t* hits, uint64_t* misses);
/* ms_model_open_gguf (one GPU) with host-tier experts of `expert_slots` HBM slots per layer. */
MS_API ms_status ms_model_open_gguf_tiered(ms_ctx* ctx, const char* path, int max_seq_len, int expert_slots,
                                           ms_model** out);
MS_API ms_status ms_model_get_config(const ms_model* m, ms_model_config* cfg);
MS_API ms_status ms_model_destroy(ms_model* m);

/* Run n tokens through the model at the current position (engine.rs:1869-2006); writes the
 * last position's logits [vocab] to host memory when logits != NULL. */
MS_API ms_status ms_model_forward(ms_model* m, const int32_t* tokens, int n_tokens, float* logits);
/* Decode numerics.  1 (default): every dot product and sum of the decode step (projections,
 * attention scores, softmax denominators, P*V, router, expert GEMVs, RMSNorm, LM head) is
 * accumulated in double and rounded to f32 once, and exp is the double exp rounded to f32; each
 * op's result is then its exact value correctly rounded, whatever the summation order, so greedy
 * tokens, routed experts and the Q8_0 activation codes are reproducible bit for bit against a CPU
 * evaluation of the reference's ops (engine.rs:1869-2118) that rounds the same way.  0: the
 * pipelined f32 kernels (tensor-core experts, split-K attention), results within ~1e-6 relative
 * of 1 per op but not bit-identical.  MXFP4 and K-quant experts and head dims 32/64/128 have
 * order-independent kernels. */
MS_API ms_status ms_model_set_exact(ms_model* m, int enable);
/* Sampled decoding (SamplingParams::sample, engine.rs:124-208, as generate_sampled drives it,
 * engine.rs:2222-2300).  enable != 0: from the next forward on, each step's token is drawn on the
 * device (repetition penalty over the tokens drawn since this call, greedy when temperature == 0,
 * temperature, softmax, top-p, then the draw) instead of the greedy argmax; the draws come from
 * SplitMix64(seed, n) for the n-th draw (24 bits, as rand builds an f32), so a seed reproduces a
 * sequence.  enable == 0 returns to greedy decoding.  temperature >= 0, 0 < top_p, penalty > 0. */
MS_API ms_status ms_model_set_sampling(ms_model* m, int enable, float temperature, float top_p,
                                       float repetition_penalty, uint64_t seed);
/* How ms_model_forward runs more than one token (a prompt).  1 (default): batched passes of up to
 * 2048 tokens -- Q8_0 projections of all tokens, QK-norm + RoPE at absolute positions, causal
 * attention with the sliding-window mask and sinks over the cache and the chunk, the router of
 * every token, and the experts as a grouped GEMM on the tensor cores (MXFP4 experts exact in bf16,
 * activations as bf16 hi + lo pairs, f32 accumulation: ~2^-18 relative); K-quant experts in groups
 * of 32 tokens.  2: the same with plain bf16 activations (fastest; ~1e-2 relative).  0: one decode
 * step per token.  Replaces the reference's multi-token forward (engine.rs:1869-2006;
 * layer.rs:1316-1349, 1848-1894; ops/attention.rs:210-244).  Expert-parallel models exchanging over
 * peer mailboxes fall back to mode 0; with NCCL the experts' output is all-reduced per layer. */
MS_API ms_status ms_model_set_prefill(ms_model* m, int mode);
/* One decode step with host buffers: token in, greedy next token out (argmax, lowest id on ties). */
MS_API ms_status ms_model_decode_step(ms_model* m, int32_t token, int32_t* next_token);
/* Greedy generation (engine.rs:2011-2118): clears the cache, prefill, max_new tokens out. */
MS_API ms_status ms_model_generate(ms_model* m, const int32_t* prompt, int n_prompt, int max_new, int32_t* out,
                            int* n_out);
/* n greedy steps entirely on the device, each feeding the previous argmax (no host copies). */
MS_API ms_status ms_model_decode_steps_device(ms_model* m, int n_steps);
/* tokens fed to the model since the last clear (device log), up to max */
MS_API ms_status ms_model_token_log(ms_model* m, int32_t* out, int max, int* n);
MS_API ms_status ms_model_clear_cache(ms_model* m);   /* engine.rs:2402-2408 */
MS_API ms_status ms_model_seq_len(const ms_model* m, int* n);
/* Diagnostics for parity tests: residual stream after the last layer of the last step [hidden],
 * routed experts of the last step for one layer [top_k], logits of the last step [vocab]. */
MS_API ms_status ms_model_last_hidden(ms_model* m, float* out);
MS_API ms_status ms_model_last_routing(ms_model* m, int layer, int32_t* idx, float* wts);
MS_API ms_status ms_model_last_logits(ms_model* m, float* out);
/* Layer trace for parity tests (single sequence): when enabled, every later step also copies the
 * residual stream after each layer and each layer's router logits (after bias and dummy mask) into
 * model buffers; ms_model_layer_trace reads those of the last step: hidden [layers][hidden],
 * logits [layers][experts] (either may be NULL).  Mirrors the per-layer dumps of the reference's
 * examples/full_compare.rs. */
MS_API ms_status ms_model_set_trace(ms_model* m, int enable);
MS_API ms_status ms_model_layer_trace(ms_model* m, float* hidden, float* logits);
/* 1 (default): replay each step as a captured CUDA graph; 0: plain stream launches. */
MS_API ms_status ms_model_set_graph(ms_model* m, int enable);
/* Tracing (single device, after at least one decode step): the decode step's launches grouped by
 * class -- 0 = embedding, 1..P = the P kernels of a layer by their position in it, P+1 = LM head --
 * and each class's launches of one step captured alone into a PDL-chained graph and timed over
 * ten launches: us[c] = device microseconds per step spent on class c.  The runs overwrite the
 * model's activations and KV cache: call ms_model_clear_cache before decoding again. */
MS_API ms_status ms_model_profile_step(ms_model* m, float* us, int max, int* n);
/* Kernel launches per decode step (for launch accounting). */
MS_API int ms_model_kernels_per_step(const ms_model* m);

#ifdef __cplusplus
}
#endif
#endif /* MOESTREAM_CUDA_H */
