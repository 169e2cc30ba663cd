/*
 * msoracle — CPU restatement of moe-stream's quantized MoE decode/prefill path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the CUDA
 * library in moe_stream_b200/csrc and the timed CPU baseline of bench.py.
 * Nothing in the product links or calls it.
 *
 * It restates the reference's default CPU path (SsdStreaming mode, no
 * QUANTIZED_MATMUL): dequantize experts to f32, f32 GEMVs, ascending-expert
 * accumulation, f32 KV cache, plain NeoX RoPE, SDPA with sinks and sliding
 * window, greedy argmax by stable sort.  Each function cites the reference
 * file:line it follows (paths relative to the moe-stream repository).
 *
 * Parity status: the block dequantizers, routing, RMSNorm, RoPE tables and the
 * combine order are restated exactly; the f32 matmul summation order of candle
 * (gemm crate) and candle's CPU QMatMul (Q8_0 attention) are third-party code
 * that is not in the reference tree, so those are pinned only by tolerance.
 */
#pragma once
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* GGML type ids (gguf/reader.rs:38-65). */
enum { ORC_F32 = 0, ORC_F16 = 1, ORC_Q8_0 = 8, ORC_Q4_K = 12, ORC_Q6_K = 14, ORC_MXFP4 = 39 };

/* ---- block formats (gguf/dequant.rs) ---- */
float orc_fp16_to_f32(uint16_t h);
float orc_e8m0_to_f32_half(uint8_t e);
/* returns 0 on success, -1 on unsupported type */
int orc_dequantize(int qtype, const void* blocks, int64_t n_elements, float* out);
/* dequant.rs:640-695 exact per-row sequential order (QUANTIZED_MATMUL=1 MXFP4 path) */
void orc_mxfp4_matvec_mul(const uint8_t* w, const float* x, int64_t rows, int64_t cols, float* y);
/* y = W x with W dequantized to f32 (default path): sequential f32 dot per row */
int orc_gemv(int qtype, const void* w, int64_t rows, int64_t cols, const float* x, float* y);
/* Q8_0 projection as candle CPU QMatMul computes it: activation quantized to Q8_0, integer
 * block dot, f32 block sum (mode 1); or exact f32 dequant-then-dot (mode 0). */
void orc_q8_0_gemv(const uint8_t* w, int64_t rows, int64_t cols, const float* x, float* y, int mode);
void orc_quantize_q8_0(const float* x, int64_t n, uint8_t* out);

/* ---- ops (ops/norm.rs, ops/attention.rs, ops/activation.rs) ---- */
void orc_rms_norm(const float* x, const float* w, float* y, int64_t rows, int64_t dim, float eps);
void orc_rope_tables(int rot_dim, int max_seq, double theta, float* cos_out, float* sin_out);
void orc_swiglu_oai(const float* g, const float* u, float* out, int64_t n, float alpha, float limit);
void orc_silu_and_mul(const float* g, const float* u, float* out, int64_t n);
/* ops/attention.rs:178-280; q [seq_q][nh][hd], k/v [nkv][seq_k][hd], out [seq_q][nh][hd] */
void orc_sdpa(const float* q, const float* k, const float* v, int nh, int nkv, int seq_q, int seq_k, int hd,
              double scale, int causal, const float* sinks, int sliding_window, float* out);
/* RoPE of x [n_tok][heads][hd] with per-token tables cos/sin [n_tok][rot/2] (ops/attention.rs:96-164) */
void orc_rope(const float* x, const float* cos_t, const float* sin_t, int n_tok, int heads, int hd, int rot, float* y);
/* SamplingParams::sample (engine.rs:124-208) of logits [V]: counts [V] = times each token was
 * generated (NULL: none), r = the uniform draw in [0, 1).  Sums of probabilities are exact to
 * 2^-109 and rounded to f32 once. */
int orc_sample(const float* logits, int V, const uint32_t* counts, float temperature, float top_p, float penalty,
               float r);
/* layer.rs:2346-2403; returns indices/weights [n_tok, k] */
void orc_top_k_routing(const float* logits, int n_tok, int n_exp, int k, int normalize, int softmax_weight,
                       int32_t* idx, float* w);

/* ---- one MoE FFN layer (layer.rs:756-1895 default CPU path, single or multi token) ----
 * x: [n_tok, hidden] (already RMS-normed); out: [n_tok, hidden] (overwritten). */
typedef struct {
  int hidden, inter, n_experts, top_k;
  int gate_q, up_q, down_q;          /* GGML ids */
  const void* gate; const void* up; const void* down;   /* stacked [E, rows, cols] native blocks */
  const float* gate_bias; const float* up_bias; const float* down_bias;  /* [E, rows] or NULL */
  const float* router_w;             /* [E, hidden] f32 */
  const float* router_b;             /* [E] or NULL */
  int oai_swiglu;                    /* GPT-OSS: OAI SwiGLU + softmax over top-k */
  int norm_topk_prob;
} orc_moe_layer;
int orc_moe_forward(const orc_moe_layer* L, const float* x, int n_tok, float* out,
                    int32_t* idx_out /* [n_tok*k] or NULL */, float* w_out /* or NULL */);

/* the same layer restricted to experts [e_begin, e_end) (routing over all experts) */
int orc_moe_forward_range(const orc_moe_layer* L, const float* x, int n_tok, float* out, int e_begin, int e_end);

/* ---- one attention half-layer for one decode token (layer.rs:511-749) ----
 * h += O(SDPA(RoPE(QKV(RMSNorm(h))))).  K, V: [kv_heads][pos+1][head_dim] f32 (the caller grows
 * them; rows < pos hold earlier tokens, row pos is written here).  Q8_0 projections. */
typedef struct {
  int hidden, heads, kv_heads, head_dim, rot_dim;
  float eps, rope_theta;
  int window;                        /* > 0: sliding window */
  int attn_mode;                     /* 1 = candle QMatMul (activation quantized), 0 = exact f32 */
  const float* attn_norm;
  const uint8_t *wq, *wk, *wv, *wo;  /* Q8_0 */
  const float *bq, *bk, *bv, *bo, *sinks, *q_norm, *k_norm;   /* or NULL */
  int q_gate;                        /* 1: wq rows (and bq) hold [Q_h, gate_h] per head (hybrid models,
                                        layer.rs:620-635); the output is multiplied by sigmoid(gate) */
} orc_attn_layer;
int orc_attn_decode(const orc_attn_layer* L, float* K, float* V, int pos, float* h);

/* ---- Gated DeltaNet decode step (model/deltanet.rs:204-543) ---- */
typedef struct {
  int hidden, n_k_heads, head_k_dim, n_v_heads, head_v_dim, conv_kernel;
  float eps;
  int qkv_q; const void* qkv;     /* [2*nk*hkd + nv*hvd, hidden] (flat Q, K, V rows) */
  int gate_q; const void* gate;   /* [nv*hvd, hidden] (z) */
  int ba_q; const void* ba;       /* [2*nv, hidden] (flat beta, alpha) */
  int out_q; const void* out;     /* [hidden, nv*hvd] */
  const float* conv1d;            /* [conv_dim, conv_kernel] */
  const float* ssm_a;             /* [nv] (-exp(A_log)) */
  const float* dt_bias;           /* [nv] */
  const float* norm;              /* [hvd] */
} orc_deltanet_layer;
/* one token: updates conv_state [conv_dim, k-1] and rec_state [nv, hkd, hvd]; y [hidden] */
int orc_deltanet_step(const orc_deltanet_layer* L, const float* x, float* conv_state, float* rec_state, float* y);
/* shared expert (layer.rs:1898-1953): y += sigmoid(x . gate_inp) * (silu(x Wg) * (x Wu)) Wd */
int orc_shared_expert(int gu_q, const void* gate, const void* up, int down_q, const void* down,
                      const float* gate_inp, int hidden, int inter, const float* x, float* y);

/* ---- whole model (engine.rs:1869-2118) ---- */
typedef struct orc_model orc_model;
/* open a GGUF file (reader.rs:259-368, config.rs:253-434) */
orc_model* orc_model_open(const char* path, int max_seq_len, char* err, int err_len);
/* attention projection numerics: 1 = candle QMatMul (activation quantized, default), 0 = exact f32 */
void orc_model_set_attn_mode(orc_model* m, int mode);
void orc_model_set_threads(orc_model* m, int n_threads);
/* forward a batch of tokens (one sequence, appended to the KV cache); writes the last
 * position's logits [vocab] if logits != NULL; returns 0 on success */
int orc_model_forward(orc_model* m, const int32_t* tokens, int n_tokens, float* logits);
/* greedy generate (engine.rs:2011-2118): clears cache, prefill, decode; returns #tokens written */
int orc_model_generate(orc_model* m, const int32_t* prompt, int n_prompt, int max_new, int32_t* out);
int orc_model_vocab(const orc_model* m);
int orc_model_hidden(const orc_model* m);
int orc_model_seq_len(const orc_model* m);
void orc_model_clear_cache(orc_model* m);
/* hidden state after the last forward (last position) [hidden] */
void orc_model_last_hidden(const orc_model* m, float* out);
/* routed experts of the last position per layer [layers*k] */
void orc_model_last_routing(const orc_model* m, int32_t* idx, float* w);
/* last forward, last position, every layer: residual stream after the layer [layers][hidden] and
 * router logits after bias and dummy mask [layers][n_experts]; either pointer may be NULL */
void orc_model_layer_trace(const orc_model* m, float* hidden, float* logits);
/* final norm + LM head of one hidden vector [hidden] -> logits [vocab] (timing / tests) */
void orc_model_lm_head(orc_model* m, const float* hidden, float* logits);
/* dynamic K (layer.rs:947-1011, config.rs:183-192, 468-483): per-token K from router entropy in
 * [k_min, k_max] (or the depth tier's range when layer_adaptive), k_max <= the model's top_k; slots
 * beyond K report expert id n_experts.  Returns 0, or -1 for an invalid range. */
int orc_model_set_dynamic_k(orc_model* m, int enable, int k_min, int k_max, int layer_adaptive);
/* router entropy and the K used per layer of the last forward [layers] (either may be NULL) */
void orc_model_router_stats(const orc_model* m, float* entropy, int32_t* k);
void orc_model_destroy(orc_model* m);

#ifdef __cplusplus
}
#endif
