// kernels.h — host-side launch interface of the moe-stream B200 kernels.
// Every argument is a plain device pointer or size; no torch types.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace ms {

// ---- device error word bits (the host reads them through ms_ctx_error_flags) ----
enum : uint32_t {
  EF_TIMEOUT_FULL = 1u << 0,    // consumer waited too long for a stage to land
  EF_TIMEOUT_EMPTY = 1u << 1,   // producer waited too long for a stage to drain
  EF_BAD_INDEX = 1u << 2,       // an expert / token index outside its table was skipped
  EF_BAD_SHAPE = 1u << 3,
};

enum QType : int { Q_F32 = 0, Q_F16 = 1, Q_Q8_0 = 8, Q_Q4_K = 12, Q_Q6_K = 14, Q_MXFP4 = 39,
                   // internal: Q6_K expert rows repacked at upload into 224-byte superblocks (the
                   // 210 bytes unchanged, then 14 bytes of padding) so every code word is aligned
                   Q_Q6_K_PAD = 1014 };
constexpr int kQ6PadBytes = 224;
cudaError_t launch_q6k_pad(const uint8_t* src, int64_t n_superblocks, uint8_t* dst, cudaStream_t s);

// bytes of one row of `cols` elements in GGML block layout; -1 when not representable
int64_t row_bytes(int qtype, int64_t cols);

struct DevCtx {
  int sm_count = 148;
  uint32_t* err = nullptr;  // device error word
};

// ---- generic / test ops ----
cudaError_t launch_dequantize(const DevCtx& c, int qtype, const void* blocks, int64_t n, float* out, cudaStream_t s);
cudaError_t launch_rms_norm(const DevCtx& c, const float* x, const float* w, float* y, int rows, int dim, float eps,
                            cudaStream_t s);
// RoPE (NeoX half-rotation of the first rot dims) of x [n_tok][heads][hd] with per-token tables
// cos/sin [n_tok][rot/2] -> y (y must not overlap x)
// gated attention of hybrid models (layer.rs:620-635, 699-705): y [2 Dq + 2 Dkv] with [Q_h, gate_h]
// per head -> qkv [Dq + 2 Dkv] and gate [Dq]; then att *= sigmoid(gate) and its Q8_0 blocks
cudaError_t launch_gate_split(const float* y, int nh, int hd, int Dkv, float* qkv, float* gate, cudaStream_t s);
cudaError_t launch_gate_apply_q8(float* att, const float* gate, int n, int8_t* oq, float* od, cudaStream_t s);
cudaError_t launch_rope(const float* x, const float* cs, const float* sn, float* y, int n_tok, int heads, int hd,
                        int rot, cudaStream_t s);
// *p = v on the stream (a capturable scalar upload)
cudaError_t launch_set_i32(int* p, int v, cudaStream_t s);

// A MoE combine not yet applied to the residual stream: the stream's value is
// h[r] + sum over local slots, in ascending expert id, of partial[slot][r] * wts[slot]
// (layer.rs:1797-1847 accumulation order; hidden = residual + moe_out, layer.rs:494),
// or h[r] + dense[r] when the expert-parallel all-reduce already summed it.
struct PendingCombine {
  const float* dense = nullptr;    // [H] summed MoE output, or null
  // [H] or null: added to the routed experts' combined output before the residual add (the shared
  // expert's output, layer.rs:910-922); read by the residual kernel only
  const float* extra = nullptr;
  const float* partial = nullptr;  // [K, H] per-slot expert outputs (bias included)
  // or, from the tensor-core down projection: per-range partial sums [items][kTcMaxSeg][128] of
  // item = local slot (ascending expert) x 128-row tile, tc_splits(items, seg_kw, seg_grid) ranges each
  const float* seg_part = nullptr;
  int seg_tiles = 0, seg_kw = 0, seg_grid = 0;
  const int* idx = nullptr;        // [K] expert ids
  const float* wts = nullptr;      // [K] routing weights
  int K = 0;
  int expert_base = 0, n_local = 0;
  // or, expert parallel over peer memory: every rank's partial MoE output in this rank's mailbox,
  // recv[parity][rank][H], complete once flags[parity][rank] >= *ep_seq (parity = *ep_seq & 1)
  const float* ep_recv = nullptr;
  const uint32_t* ep_flags = nullptr;
  const uint32_t* ep_seq = nullptr;
  int ep_n = 0;
  int ep_rows = 0;                 // mailbox rows per parity (max(ranks, slots))
  int ep_slots = 0;                // 1: the mailbox holds each slot's output [parity][slot][H] (from its
                                   // owner rank), combined here over all slots in ascending expert id
  __host__ __device__ bool active() const {
    return dense != nullptr || partial != nullptr || seg_part != nullptr || ep_recv != nullptr;
  }
};

// Expert-parallel exchange over NVLink peer memory (kernels_dense.cu): this rank's combined MoE
// output is stored into every rank's mailbox slot [parity][rank], then each rank's flag
// [parity][rank] is released with the step's sequence number.
constexpr int kMaxEp = 8;
struct EpSend {
  float* recv[kMaxEp];             // each rank's mailbox (peer pointers; own rank local)
  uint32_t* flags[kMaxEp];         // each rank's flag array [2][n]
  uint32_t* seq = nullptr;         // this rank's sequence counter (device)
  uint32_t* cnt = nullptr;         // CTA counter (device, zero, self-resetting)
  int rank = 0, n = 0;
  int rows = 0;                    // mailbox rows per parity
  int slots = 0;                   // 1: send each local slot's output to row [parity][slot] (else the combine)
};
cudaError_t launch_ep_send(const DevCtx& c, const PendingCombine& pc, int H, const EpSend& e, cudaStream_t s);

// y[r] = W[r,:] . x  (+bias[r]) (+residual: y[r] += y_in[r]);  MXFP4 / F16 / F32 weights.
struct GemvArgs {
  int qtype = Q_MXFP4;
  const void* w = nullptr;
  int rows = 0, cols = 0;
  const float* x = nullptr;
  const float* bias = nullptr;
  float* y = nullptr;
  int accumulate = 0;          // y[r] += result
};
cudaError_t launch_gemv(const DevCtx& c, const GemvArgs& a, cudaStream_t s);

// Q8_0 projection with the activation quantized to Q8_0 blocks (candle QMatMul numerics).
// Optional RMSNorm of x first (norm_w != null); optional residual add into `residual`.
struct Q8GemvArgs {
  const uint8_t* w = nullptr;  // [rows, cols] Q8_0
  int rows = 0, cols = 0;
  const float* x = nullptr;
  const float* norm_w = nullptr;
  float eps = 1e-5f;
  const float* bias = nullptr;
  float* y = nullptr;          // output (ignored when residual != null)
  float* residual = nullptr;   // residual[r] += W x + bias
  int exact = 0;               // 1: f32 activations (no quantization), for the exact-mode oracle
  const int8_t* xq_in = nullptr;  // activation already quantized by its producer: int8 codes [cols]
  const float* xd_in = nullptr;   // and block scales [cols / 32]; x / norm_w are then unused
};
cudaError_t launch_q8_gemv(const DevCtx& c, const Q8GemvArgs& a, cudaStream_t s);

// ---- MoE ----
// RMSNorm(h)*gamma -> xn, router logits = xn W^T + b (+ -inf mask) -> top-k + weights.
struct RouterArgs {
  const float* h = nullptr;       // [H] residual stream (nullptr: x is already normed, read xn)
  const float* norm_w = nullptr;  // [H]
  float eps = 1e-5f;
  float* xn = nullptr;            // [H] output (input when h == nullptr)
  const float* w = nullptr;       // [E, H] f32
  const float* b = nullptr;       // [E] or null
  const uint8_t* mask = nullptr;  // [E] 1 = dummy expert (masked to -inf) or null
  float* logits = nullptr;        // [E] scratch/output
  int* idx = nullptr;             // [K]
  float* wts = nullptr;           // [K]
  uint32_t* counter = nullptr;    // 1 word scratch, zero-initialised, self-resetting
  int H = 0, E = 0, K = 0;
  int softmax_weight = 1;         // GPT-OSS: softmax over the selected k logits
  int normalize = 0;              // renormalise top-k probabilities (norm_topk_prob)
  uint8_t* xterm = nullptr;       // optional: the normed x as MXFP4 B terms (tc_bterm_bytes(H/32))
  uint8_t* xbt = nullptr;         // optional: the normed x as exact B terms ([H/32][exact_term_block_bytes()],
  int* xfe = nullptr;             //   zeroed once) and their scale exponents [H/32]
  int batch = 1;                  // grid.y = tokens: h/xn + b*H, logits + b*E, idx/wts + b*K, counter + b
  // router statistics and dynamic K (layer.rs:947-1011, 2302-2334; one token, batch 1 only):
  // with `raw` set every CTA also stores its logit before the dummy mask, and the selecting warp
  // writes the entropy of softmax(raw) to *entropy; k_hi > 0 then routes only
  // K' = round(k_lo + clamp(H / ln E, 0, 1) (k_hi - k_lo)) experts (k_hi <= K), the other slots
  // get expert id E (none) and weight 0; *k_used = the K routed
  float* raw = nullptr;           // [E]
  float* entropy = nullptr;
  int* k_used = nullptr;
  int k_lo = 0, k_hi = 0;
  // running totals of this layer (RoutingStatsCollector::record / EntropyProfiler::record,
  // model/cache.rs:404-580), updated by the selecting lane once per step when cnt is set (needs raw):
  // per expert the times routed and the sum of its routing weights, the tokens seen, and the entropy
  // appended to a log of ent_cap entries with stride ent_stride
  unsigned long long* cnt = nullptr;   // [E]
  double* wsum = nullptr;              // [E]
  unsigned long long* tokens = nullptr;
  float* ent_log = nullptr;
  uint32_t* ent_n = nullptr;
  int ent_cap = 0, ent_stride = 1;
};
cudaError_t launch_router(const DevCtx& c, const RouterArgs& a, cudaStream_t s);

// Fused expert FFN for one token over MXFP4 experts: act = SwiGLU(Wg x + bg, Wu x + bu),
// y_e = Wd act + bd, h += sum over selected experts (ascending expert id) of w_e * y_e.
struct MoeArgs {
  const float* x = nullptr;        // [H] normed input
  const int* idx = nullptr;        // [K] selected expert ids
  const float* wts = nullptr;      // [K] routing weights
  int gate_q = Q_MXFP4;            // qtype of gate/up: MXFP4 or Q4_K
  int down_q = Q_MXFP4;            // qtype of down: MXFP4 or Q6_K (or Q4_K)
  const uint8_t* gate = nullptr;   // [E_local, I, H] native blocks
  const uint8_t* up = nullptr;     // [E_local, I, H]
  const uint8_t* down = nullptr;   // [E_local, H, I]
  const float* gate_b = nullptr;   // [E_local, I] or null
  const float* up_b = nullptr;
  const float* down_b = nullptr;   // [E_local, H] or null
  float* act = nullptr;            // [K, I] scratch
  float* partial = nullptr;        // [K, H] scratch
  uint32_t* tile_cnt = nullptr;    // reserved (no kernel reads it; may be null)
  float* h = nullptr;              // [H] residual stream: h += moe(x)   (when out == null)
  float* out = nullptr;            // [H] if set: out = moe(x) (no residual), for EP partial sums
  int H = 0, I = 0, K = 0;
  int expert_base = 0, n_local = 0;  // experts [base, base+n_local) live on this device
  int oai_swiglu = 1;
  int defer_combine = 0;           // 1: leave the combine pending (consumers apply it); no h / out update
};
cudaError_t launch_moe_mxfp4(const DevCtx& c, const MoeArgs& a, cudaStream_t s);
// the combine as its own kernel: h[r] += comb(r), or out[r] = comb(r) when out != null
cudaError_t launch_moe_combine(const DevCtx& c, const PendingCombine& pc, int H, float* h, float* out,
                               cudaStream_t s);
// plain MXFP4 / Q4_K / Q6_K GEMV through the same streaming machinery: y = W x (+bias) (+= when accumulate)
cudaError_t launch_block_gemv(const DevCtx& c, int qtype, const uint8_t* w, int rows, int cols, const float* x,
                              const float* bias, float* y, int accumulate, cudaStream_t s);

// ---- MXFP4 expert FFN on tcgen05 (repacked tiles; kernels_moe_tc.cu) ----
constexpr int kTcMaxSeg = 16;   // split-K ranges per item held in the partial-sum scratch
constexpr int kTcMaxTiles = 64; // down tiles a combine can read (hidden <= 8192)
int64_t tc_tile_bytes(int kc);            // one packed 128-row tile over kc chunk columns (K = 32 kc)
int64_t tc_bterm_bytes(int kc);           // one 16-term B operand over kc chunk columns (umma::bterm_bytes)
int tc_gu_tiles(int I);                   // gate_up tiles per expert (64 gate + 64 up rows each)
int tc_down_tiles(int H);                 // down tiles per expert (128 rows each, last zero-padded)
int tc_max_items(int H, int I, int K);    // items per projection (split-K scratch rows)
int tc_cnt_words(int H, int I, int K);    // counter words: 2 x items, per-slot ready counts, done
bool tc_supported(int H, int I);          // H % 64 == 0 && I % 64 == 0
struct TcMoeArgs {
  const uint8_t* gu = nullptr;      // [E_local][tc_gu_tiles(I)][tc_tile_bytes(H/32)]
  const uint8_t* down = nullptr;    // [E_local][tc_down_tiles(H)][tc_tile_bytes(I/32)]
  const float* gate_b = nullptr;    // [E_local, I] or null
  const float* up_b = nullptr;
  const float* down_b = nullptr;    // [E_local, H] or null
  const uint8_t* xterm = nullptr;   // B terms of the normed input (tc_bterm_bytes(H/32))
  uint8_t* act_terms = nullptr;     // scratch [K][tc_bterm_bytes(I/32)]
  float* act = nullptr;             // optional [K, I] f32 activations
  float* partial = nullptr;         // [K, H] per-slot expert outputs (bias included)
  float* part = nullptr;            // split-K scratch [2][tc_max_items][kTcMaxSeg][128]
  uint32_t* cnt = nullptr;          // [tc_cnt_words] zero-initialised, self-resetting
  const int* idx = nullptr;
  const float* wts = nullptr;
  int H = 0, I = 0, K = 0, expert_base = 0, n_local = 0, oai_swiglu = 1;
  float* h = nullptr;               // as MoeArgs: h += moe(x), or out = moe(x)
  float* out = nullptr;
  int defer_combine = 0;
};
cudaError_t launch_moe_tc(const DevCtx& c, const TcMoeArgs& a, cudaStream_t s);
// the pending combine of a launch_moe_tc call made with defer_combine (reads its down partials)
PendingCombine tc_pending_combine(const DevCtx& c, const TcMoeArgs& a);
// native GGUF MXFP4 [E][rows][cols] -> packed tiles: rows go to tile r / tile_rows_src at tile row
// row_off + r % tile_rows_src (gate: 64, 0; up: 64, 64; down: 128, 0)
cudaError_t launch_mxfp4_pack(const uint8_t* src, int E, int rows, int cols, int tile_rows_src, int row_off,
                              int tiles, uint8_t* dst, cudaStream_t s);
cudaError_t launch_xterms(const DevCtx& c, const float* x, int H, uint8_t* xterm, cudaStream_t s);

// ---- batched prefill: the expert FFN as a grouped bf16 GEMM on tcgen05 (kernels_prefill.cu) ----
struct PrefillArgs {
  const uint8_t* gu = nullptr;      // packed MXFP4 tiles, as TcMoeArgs
  const uint8_t* down = nullptr;
  const float* gate_b = nullptr;    // [E, I] or null
  const float* up_b = nullptr;
  const float* down_b = nullptr;    // [E, H] or null
  const float* x = nullptr;         // [T, H] normed inputs
  const int* idx = nullptr;         // [T, K] expert ids
  const float* wts = nullptr;       // [T, K] routing weights
  float* out = nullptr;             // [T, H]: = MoE(x), or += when accumulate
  void* scratch = nullptr;          // pf_scratch_bytes(H, I, E, T, K) bytes
  int H = 0, I = 0, E = 0, K = 0, T = 0, expert_base = 0, oai_swiglu = 1, accumulate = 0;
  int precise = 0;                  // 1: activations as bf16 hi + lo pairs (two MMAs per K step, ~2^-18 relative)
};
size_t pf_scratch_bytes(int H, int I, int E, int T, int K, int precise = 0);
cudaError_t launch_moe_prefill(const DevCtx& c, const PrefillArgs& a, cudaStream_t s);

// ---- multi-token forward (prompt prefill), kernels_prefill_attn.cu ----
// h[t] = embedding(tok[t]); xq/xd[t] = Q8_0(RMSNorm(h[t]) * norm_w)   (one CTA per token)
cudaError_t launch_pf_embed(const DevCtx& c, const int* tok, int T, const void* table, int q, int H, int vocab,
                            float* h, const float* norm_w, float eps, int8_t* xq, float* xd, cudaStream_t s);
// xq/xd[t] = Q8_0(RMSNorm(h[t]) * norm_w)
cudaError_t launch_pf_norm_q8(const float* h, int T, int H, const float* norm_w, float eps, int8_t* xq, float* xd,
                              cudaStream_t s);
// Q8_0 blocks of x[0..n) (n % 32 == 0)
cudaError_t launch_pf_quant(const float* x, int64_t n, int8_t* xq, float* xd, cudaStream_t s);
// h[i] += y[i]
cudaError_t launch_pf_add(float* h, const float* y, int64_t n, cudaStream_t s);
// QK-norm + RoPE of T tokens' projections, causal (sliding-window) attention with sinks over the
// cache (positions < pos0) and the chunk, then the chunk's K/V appended to the cache
struct PfAttnLaunch {
  const float* qkv = nullptr;      // [T][nh*hd + 2*nkv*hd]
  const float* q_norm = nullptr;   // [hd] or null (with k_norm)
  const float* k_norm = nullptr;
  float eps = 1e-6f;
  const float* cos_t = nullptr;    // [max_seq][rot/2]
  const float* sin_t = nullptr;
  int rot = 0, pos0 = 0, T = 0, nh = 0, nkv = 0, hd = 0;
  float* kc = nullptr;             // layer cache [nkv][cap][hd]
  float* vc = nullptr;
  int cap = 0, window = 0;
  const float* sinks = nullptr;
  float scale = 1.f;
  float* q = nullptr;              // scratch [T][nh][hd]
  float* kn = nullptr;             // scratch [T][nkv][hd]
  float* vn = nullptr;             // scratch [T][nkv][hd]
  float* out = nullptr;            // [T][nh*hd]
};
cudaError_t launch_pf_attention(const DevCtx& c, const PfAttnLaunch& L, cudaStream_t s);

// ---- attention (decode, one token) ----
struct AttnArgs {
  const float* qkv = nullptr;      // [nh*hd + 2*nkv*hd] projections (+bias), before RoPE
  const float* q_norm = nullptr;   // [hd] QK-RMSNorm weights or null
  const float* k_norm = nullptr;
  float eps = 1e-6f;
  const float* cos_t = nullptr;    // [max_seq][rot/2]
  const float* sin_t = nullptr;
  int rot = 0;                     // rotary dims (<= hd)
  const int* pos = nullptr;        // device: position of this token
  float* kc = nullptr;             // [nkv][cap][hd] f32 cache
  float* vc = nullptr;
  int cap = 0;                     // cache slots (== window for sliding-window layers: ring)
  int window = 0;                  // 0: full attention
  const float* sinks = nullptr;    // [nh] or null
  float* part = nullptr;           // scratch [nkv][S][rep][hd + 2]
  uint32_t* cnt = nullptr;         // [nkv] zero-initialised, self-resetting
  float* out = nullptr;            // [nh*hd]
  int8_t* oq = nullptr;            // optional Q8_0 codes of out [nh*hd] (for the O-projection)
  float* od = nullptr;             // and their block scales [nh*hd/32]
  int nh = 0, nkv = 0, hd = 0, S = 0;
  float scale = 1.0f;
  // batched decode (B sequences in lockstep, one position): grid.z = batch; sequence b reads
  // qkv + b*bs_qkv, its caches kc/vc + b*bs_kv, writes out/oq + b*bs_out, od + b*bs_out/32,
  // part + b*(nkv*S*REP*(hd+2)) and counters cnt + b*nkv
  int batch = 1;
  int64_t bs_qkv = 0, bs_kv = 0, bs_out = 0;
  int spl = 0;                     // streaming kernel: positions per split (a multiple of 32); 0: one-sequence tile kernel
  int head_split = 1;              // streaming kernel: CTAs sharing a kv head, each with nh/nkv/head_split query heads
};
cudaError_t launch_attention(const DevCtx& c, const AttnArgs& a, cudaStream_t s);
// tile-kernel splits (grid.x) needed to cover `range` attended positions
int attn_splits(int range, int hd);   // splits of a decode-attention launch covering `range` positions
// positions per split for `units` = kv_heads x sequences attending over `range` positions
int attn_split_positions(int range, int units, int sm_count);

// ---- order-independent decode kernels (kernels_exact.cu): f64 reductions rounded once ----
// decode attention for one token per sequence (AttnArgs as launch_attention; oq / od written when
// set); `range` = the most positions a sequence can attend to (cache slots, or the window)
cudaError_t launch_exact_attention(const DevCtx& c, const AttnArgs& a, int range, cudaStream_t s);
int exact_attn_cluster(int range, int units, int sm_count);
// the expert FFN of one token over packed MXFP4 tiles: f64 partial dots of gate/up rows per K
// segment (gp), the activations as exact digits, f64 partial dots of the down rows (dp), and each
// slot's output y = (segments summed in f64, rounded) + bias; the consumer (PendingCombine.partial
// = y) combines the slots in ascending expert id
struct ExactMoeArgs {
  const uint8_t* gu = nullptr;      // packed tiles, as TcMoeArgs
  const uint8_t* down = nullptr;
  const float* gate_b = nullptr;    // [E_local, I] or null
  const float* up_b = nullptr;
  const float* x = nullptr;         // [H] normed input
  const int* idx = nullptr;         // [K]
  int H = 0, I = 0, K = 0, expert_base = 0, n_local = 0, oai_swiglu = 1;
  double* gp = nullptr;             // [K][n_seg_gu][2 I]
  double* dp = nullptr;             // [K][n_seg_down][h_pad]
  int n_seg_gu = 0, n_seg_down = 0, h_pad = 0;
  const uint8_t* xbt = nullptr;     // [H/32][exact_term_block_bytes()] exact B terms of x (exact_bterm_warp), from the router
  const int* xfe = nullptr;         // [H/32 + 8] their scale exponents (+ padding for 32-byte copies)
  uint8_t* abt = nullptr;           // [K][I/32][exact_term_block_bytes()] B terms of the activations (from gate/up; zeroed once)
  int* afe = nullptr;               // [K][I/32 rounded up to 8] (32-byte copies of 8 chunks' exponents)
  uint32_t* cnt = nullptr;          // [K][gate/up tiles] + [K][down tiles], zero-initialised, self-resetting
  const float* down_b = nullptr;    // [E_local, H] or null
  float* y = nullptr;               // [K][H] each slot's output (the combine's PendingCombine.partial)
  int gu_tiles = 0, down_tiles = 0;           // filled by launch_exact_moe
  uint32_t* err = nullptr;                    // filled by launch_exact_moe
  int64_t gu_tile_bytes = 0, down_tile_bytes = 0;
};
int exact_seg_count(int kc);
int exact_term_block_bytes();     // bytes of one chunk's exact B-term block        // K segments over kc 32-element chunks
// the same for K-quant experts in native blocks (Q4_K, or Q6_K repacked to 224-byte superblocks):
// gate / up rows -> gu_out [K][2][I] (f32, rounded once, + bias), down rows -> y [K][H] (+ bias);
// the consumer combines y (PendingCombine.partial) in ascending expert id
struct ExactKqArgs {
  const uint8_t* gate = nullptr;    // [E_local, I, H]
  const uint8_t* up = nullptr;
  const uint8_t* down = nullptr;    // [E_local, H, I]
  int gate_fmt = Q_Q4_K, down_fmt = Q_Q6_K_PAD;
  const float *gate_b = nullptr, *up_b = nullptr, *down_b = nullptr;
  const float* x = nullptr;
  const int* idx = nullptr;
  int H = 0, I = 0, K = 0, expert_base = 0, n_local = 0, oai_swiglu = 0;
  int B = 1;                        // tokens: x [B][H], idx [B][K], gu_out [B K][2][I], y [B K][H]
  // [B K] or null: the weight slot of each (token, slot) in gate / up / down (host-tier expert
  // streaming keeps only a cache of slots in HBM); null: the expert's own position.  Biases and the
  // combine still follow idx.
  const int* wslot = nullptr;
  float* gu_out = nullptr;
  float* y = nullptr;
};
bool exact_kq_supported(int gate_q, int down_q, int H, int I);
// keys[b] = exact greedy token of sequence b: ids within a band of the approximate maximum of
// logits [B][V] re-scored with f64 dots of the f16 rows w [V][H] and the normed xf [B][H]
// (keys[b] must hold the approximate argmax key of logits b on entry; scratch: exact_refine_scratch_ints(B)
// ints, zero-initialised, self-resetting)
cudaError_t launch_exact_argmax_refine(const uint16_t* w, const float* xf, const float* bias, const float* logits,
                                       int V, int H, int B, unsigned long long* keys, int* scratch, const DevCtx& c,
                                       cudaStream_t s);
int exact_refine_scratch_ints(int B);
cudaError_t launch_exact_kq_moe(const DevCtx& c, const ExactKqArgs& a, cudaStream_t s);
cudaError_t launch_exact_moe(const DevCtx& c, const ExactMoeArgs& a, cudaStream_t s, int part = -1);

// ---- LM head / f16 GEMV ----
// logits = W (RMSNorm(h)*norm_w if norm_w) (+bias); argmax (lowest index on ties) into *key.
struct LmHeadArgs {
  const uint16_t* w = nullptr;     // [V, H] f16
  const float* x = nullptr;        // [H]
  const float* norm_w = nullptr;   // final norm weights or null (x used as is)
  float eps = 1e-5f;
  const float* bias = nullptr;
  float* logits = nullptr;         // [V] or null
  unsigned long long* key = nullptr;  // argmax key (value, index) or null; caller zeroes it
  int V = 0, H = 0;
  int accumulate = 0;
  float* x_out = nullptr;             // effective x (before the norm) written by CTA 0, or null
  float* xn_out = nullptr;            // x after the final norm (CTA 0), or null
};
cudaError_t launch_lmhead(const DevCtx& c, const LmHeadArgs& a, cudaStream_t s);
int argmax_from_key(unsigned long long key);

// f32 weights, y = W x (+bias)
cudaError_t launch_gemv_f32(const DevCtx& c, const float* w, int rows, int cols, const float* x,
                            const float* bias, float* y, int accumulate, cudaStream_t s);

// ---- batched decode: B sequences in lockstep at one position (kernels_batch.cu, kernels_moe.cu) ----
constexpr int kMaxBatch = 32;
struct BatchState {
  int pos;                 // position written this step (shared by the batch)
  int n_ctx;
  int max_seq;
  int use_argmax;          // 1: tokens from the previous step's argmax keys, else tok_in
  int n_log;               // steps appended to the token log
  int log_row;             // row of this step in the token log
};
// h[b] = embed(token b); xq/xd[b] = Q8_0(RMSNorm(h[b]) * norm_w); token log row n_log
// pos = n_ctx, n_ctx += 1, log row = n_log, n_log += 1 (one thread, before the step's kernels)
cudaError_t launch_batch_begin(const DevCtx& c, BatchState* st, cudaStream_t s);
cudaError_t launch_embed_batch(const DevCtx& c, BatchState* st, const int* tok_in, const unsigned long long* keys,
                               const void* table, int q, int H, int vocab, int B, float* h, int* log,
                               const float* norm_w, float eps, int8_t* xq, float* xd, cudaStream_t s);
// Q8_0 weights [rows, cols] x B Q8_0 activations (int8 MMA per 32-block, f32 block sums):
// y[b][r] = W x_b + bias, or residual[b][r] += W x_b + bias
struct Q8BatchArgs {
  const uint8_t* w = nullptr;
  int rows = 0, cols = 0, B = 0;
  const int8_t* xq = nullptr;      // [B][cols]
  const float* xd = nullptr;       // [B][cols / 32]
  const float* bias = nullptr;
  float* y = nullptr;              // [B][rows]
  float* residual = nullptr;       // [B][rows]
};
cudaError_t launch_q8_gemm_batch(const DevCtx& c, const Q8BatchArgs& a, cudaStream_t s);
// h[b] += sum over token b's local experts (ascending id) of w * y[entry]; then the next
// attention input (xq/xd: Q8_0 of RMSNorm(h[b]) * norm_w) or the LM head input (xf: f32)
struct BatchCombine {
  const float* y = nullptr;        // [B][K][H] expert outputs (bias included)
  const int* ent_of = nullptr;     // [B][K] entry of each (token, slot), -1 when not local
  const int* idx = nullptr;        // [B][K]
  const float* wts = nullptr;      // [B][K]
  int K = 0;
};
cudaError_t launch_resid_batch(const DevCtx& c, const BatchCombine& bc, float* h, int H, int B, const float* norm_w,
                               float eps, int8_t* xq, float* xd, float* xf, cudaStream_t s);
// logits[b] = W xf[b] (+bias), W f16 [V, H]; argmax keys[b] (lowest index on ties)
struct LmBatchArgs {
  const uint16_t* w = nullptr;
  const float* xf = nullptr;       // [B][H] normed
  int V = 0, H = 0, B = 0;
  const float* bias = nullptr;
  void* scratch = nullptr;         // lm_batch_scratch_bytes(V, H)
  float* logits = nullptr;         // [B][V] or null
  unsigned long long* keys = nullptr;  // [B]
};
int64_t lm_batch_scratch_bytes(int V, int H);
cudaError_t launch_lmhead_batch(const DevCtx& c, const LmBatchArgs& a, cudaStream_t s);
// expert FFN of a batch: tokens grouped by expert (each expert streamed once per group of <= 4
// tokens), K-quant / native MXFP4 experts
struct GroupMoeArgs {
  const float* x = nullptr;        // [B][H] normed MoE input
  const int* idx = nullptr;        // [B][K]
  int B = 0, K = 0, H = 0, I = 0;
  int gate_q = Q_Q4_K, down_q = Q_Q6_K;
  const uint8_t* gate = nullptr;   // [E_local, I, H]
  const uint8_t* up = nullptr;
  const uint8_t* down = nullptr;   // [E_local, H, I]
  const float *gate_b = nullptr, *up_b = nullptr, *down_b = nullptr;
  int expert_base = 0, n_local = 0;
  int oai_swiglu = 0;
  int* grp = nullptr;              // scratch: group_table_words(B, K, n_local)
  int* ent_slot = nullptr;         // [B*K] (token, slot) of each entry
  int* ent_of = nullptr;           // [B*K] entry of each (token, slot), -1 when not local
  float* act = nullptr;            // [B*K][I] by entry
  float* y = nullptr;              // [B][K][H] by (token, slot)
};
int group_table_words(int B, int K);
// part: 0 grouping (route), 1 gate_up + activation, 2 down -- launched in that order
cudaError_t launch_moe_group(const DevCtx& c, const GroupMoeArgs& a, int part, cudaStream_t s);

// ---- Gated DeltaNet / shared expert (kernels_ssm.cu) ----
struct DeltaNetStep {
  int nk = 0, hkd = 0, nv = 0, hvd = 0;
  float eps = 0.f, scale = 0.f;
  float* conv_out = nullptr;          // [2 nk hkd + nv hvd] after conv + SiLU
  const float* ba = nullptr;          // [2 nv]: beta logits, then alpha logits
  const float* z = nullptr;           // [nv hvd] output gate
  const float *ssm_a = nullptr, *dt_bias = nullptr, *norm = nullptr;
  float* state = nullptr;             // [nv, hkd, hvd]
  float* out = nullptr;               // [nv hvd]
};
cudaError_t launch_deltanet_core(const DevCtx& c, const DeltaNetStep& a, int conv_dim, int ks, const float* mixed,
                                 const float* conv_w, float* conv_state, cudaStream_t s);
cudaError_t launch_silu_mul(const float* g, const float* u, float* o, int n, cudaStream_t s);
// y += sigmoid(x . gate_inp) * v (assign: y = ...); gate_inp null: factor 1
cudaError_t launch_gated_accum(const float* x, const float* gate_inp, const float* v, float* y, int n, cudaStream_t s,
                               int assign = 0);

// ---- step plumbing ----
// ---- sampling (kernels_sample.cu): SamplingParams::sample (engine.rs:124-208) on the device ----
struct SampleArgs {
  const float* logits = nullptr;      // [V]
  int V = 0;
  const uint32_t* counts = nullptr;   // [V] times each token was generated (repetition penalty), or null
  float temperature = 1.0f, top_p = 1.0f, penalty = 1.0f;
  float r = 0.0f;                     // the draw in [0, 1) when rng is null
  unsigned long long* rng = nullptr;  // optional [seed, n]: draw = SplitMix64(seed, n); n advances per call
  float* work = nullptr;              // [V] scratch
  int* token_out = nullptr;           // optional
  unsigned long long* key_out = nullptr;   // optional: the token as a step key (StepState::key)
  uint32_t* counts_rw = nullptr;      // optional: counts[token] += 1 after the draw
  const int* draw = nullptr;          // optional: no draw at all while *draw == 0 (prompt positions)
};
cudaError_t launch_sample(const DevCtx& c, const SampleArgs& a, cudaStream_t s);

struct StepState {
  int token_in;            // host-provided token
  int use_argmax;          // 1: take the token from the previous step's argmax key
  int pos;                 // position being written this step
  int n_ctx;               // tokens in the cache
  int max_seq;
  int last_token;
  unsigned long long key;  // argmax of this step
  int n_log;               // tokens appended to the log
  int pad;
};
// token -> embedding row (f16 or f32 table) -> h; advances pos; resets the argmax key
cudaError_t launch_embed(const DevCtx& c, StepState* st, const void* table, int table_q, int H, int vocab,
                         float* h, int* token_log, cudaStream_t s, const float* norm_w = nullptr, float eps = 0.f,
                         int8_t* xq = nullptr, float* xd = nullptr);
// h += MoE output, then (norm_w set) RMSNorm + Q8_0 quantization of h for the next projection;
// cnt: one zero-initialised, self-resetting counter word
cudaError_t launch_resid_norm_q8(const DevCtx& c, const PendingCombine& pc, float* h, int H, const float* norm_w,
                                 float eps, int8_t* xq, float* xd, uint32_t* cnt, cudaStream_t s);

}  // namespace ms
