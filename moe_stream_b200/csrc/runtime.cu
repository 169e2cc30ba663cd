#include <algorithm>
// runtime.cu — host runtime and C ABI of the moe-stream B200 backend.
//
// Holds the context (device, stream, device error word, scratch), the model (weights
// uploaded in their native GGUF block layout, f32 KV cache, RoPE tables, per-step
// scratch), the GGUF loader, and the per-token decode step, which is captured once as a
// CUDA graph and replayed.  Reference call sites are cited per function.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <fcntl.h>
#include <nccl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cmath>
#include <cstdlib>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <set>
#include <string>
#include <vector>

#include "../../include/moestream_cuda.h"
#include "kernels.h"

using namespace ms;

struct ms_ctx {
  int device = 0;
  cudaStream_t own = nullptr, stream = nullptr;
  DevCtx dc;
  std::string err;
  // scratch for the standalone kernel entry points
  void* scratch = nullptr;
  size_t scratch_bytes = 0;
  uint32_t* counters = nullptr;   // zero-initialised, self-resetting
  size_t n_counters = 0;
  std::vector<ms_model*> models;  // live models; ms_ctx_destroy frees any still open
};

namespace {

ms_status fail(ms_ctx* c, ms_status s, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  if (c) c->err = buf;
  return s;
}

ms_status cuda_fail(ms_ctx* c, cudaError_t e, const char* what) {
  return fail(c, e == cudaErrorMemoryAllocation ? MS_ERR_OOM : MS_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

#define MS_CUDA(ctx, call)                                      \
  do {                                                          \
    cudaError_t e_ = (call);                                    \
    if (e_ != cudaSuccess) return cuda_fail((ctx), e_, #call);  \
  } while (0)

ms_status check_dev_flags(ms_ctx* c) {
  uint32_t f = 0;
  MS_CUDA(c, cudaMemcpy(&f, c->dc.err, 4, cudaMemcpyDeviceToHost));
  if (!f) return MS_OK;
  cudaMemset(c->dc.err, 0, 4);
  if (f & (EF_TIMEOUT_FULL | EF_TIMEOUT_EMPTY))
    return fail(c, MS_ERR_TIMEOUT, "device wait timed out (flags 0x%x)", f);
  return fail(c, MS_ERR_DEVICE_INDEX, "device saw an out-of-range index or shape (flags 0x%x)", f);
}

ms_status ensure_scratch(ms_ctx* c, size_t bytes, size_t counters) {
  if (bytes > c->scratch_bytes) {
    if (c->scratch) cudaFree(c->scratch);
    c->scratch = nullptr;
    c->scratch_bytes = 0;
    MS_CUDA(c, cudaMalloc(&c->scratch, bytes));
    c->scratch_bytes = bytes;
  }
  if (counters > c->n_counters) {
    if (c->counters) cudaFree(c->counters);
    c->counters = nullptr;
    c->n_counters = 0;
    MS_CUDA(c, cudaMalloc(&c->counters, counters * 4));
    // zeroed on the stream the kernels that use them are enqueued on (it may not synchronise
    // with the legacy stream)
    MS_CUDA(c, cudaMemsetAsync(c->counters, 0, counters * 4, c->stream));
    c->n_counters = counters;
  }
  return MS_OK;
}

int64_t raw_bytes(int q, int64_t n_elements) {
  switch (q) {
    case Q_F32: return n_elements * 4;
    case Q_F16: return n_elements * 2;
    case Q_Q8_0: return (n_elements + 31) / 32 * 34;
    case Q_Q4_K: return (n_elements + 255) / 256 * 144;
    case Q_Q6_K: return (n_elements + 255) / 256 * 210;
    case Q_MXFP4: return (n_elements + 31) / 32 * 17;
  }
  return -1;
}

}  // namespace

// =====================================================================================
// model
// =====================================================================================
struct LayerW {
  float* attn_norm = nullptr;
  float* post_norm = nullptr;
  uint8_t* wqkv = nullptr;
  float* bqkv = nullptr;
  uint8_t* wo = nullptr;
  float* bo = nullptr;
  float* sinks = nullptr;
  float* qn = nullptr;
  float* kn = nullptr;
  float* router_w = nullptr;
  float* router_b = nullptr;
  uint8_t* mask = nullptr;
  uint8_t* gate = nullptr;
  uint8_t* up = nullptr;
  uint8_t* down = nullptr;
  float* gate_b = nullptr;
  float* up_b = nullptr;
  float* down_b = nullptr;
  int gate_q = -1, up_q = -1, down_q = -1, attn_q = -1;
  float* kc = nullptr;
  float* vc = nullptr;
  int cap = 0, window = 0;
  int* idx = nullptr;
  float* wts = nullptr;
  int qkv_parts = 0, bqkv_parts = 0;
  // MXFP4 experts repacked for the tensor-core path (kernels_moe_tc.cu); native pointers stay null
  uint8_t* gu_tc = nullptr;
  uint8_t* down_tc = nullptr;
  bool have_gate = false, have_up = false, have_down = false;
  bool tc = false;
  // Gated DeltaNet layer of a hybrid model (deltanet.rs:204-543); attention fields stay null
  bool deltanet = false;
  uint8_t *dn_qkv = nullptr, *dn_z = nullptr, *dn_ba = nullptr, *dn_out = nullptr;
  int dn_qkv_q = -1, dn_z_q = -1, dn_ba_q = -1, dn_out_q = -1;
  int dn_ba_parts = 0;              // ssm_ba, or ssm_beta + ssm_alpha
  float *dn_conv_w = nullptr, *dn_a = nullptr, *dn_dt = nullptr, *dn_norm = nullptr;
  float *dn_conv_state = nullptr, *dn_state = nullptr;   // [conv_dim][taps - 1], [v heads][hkd][hvd]
  // shared expert (layer.rs:1898-1953, 2250-2293)
  uint8_t *sh_gate = nullptr, *sh_up = nullptr, *sh_down = nullptr;
  int sh_gate_q = -1, sh_up_q = -1, sh_down_q = -1;
  float* sh_gate_inp = nullptr;
  int sh_dims[3] = {0, 0, 0};       // gate rows, up rows, down cols (the shared expert's width)
  // one buffer for the DeltaNet input projections [qkv | z | ba rows] and one for the shared expert's
  // [gate | up rows] when their qtypes agree, so each group is a single GEMV launch
  uint8_t* dn_in = nullptr;
  int dn_in_q = -1;
  uint8_t* sh_gu = nullptr;
  int sh_gu_q = -1, sh_gu_rows = 0;
  int dk_lo = 0, dk_hi = 0;         // dynamic K range of this layer (ms_model_set_dynamic_k), 0: off
};

// NCCL is resolved at run time (dlopen), so a process that already loaded libnccl (torch does)
// shares that copy and single-GPU users need no NCCL at all.
struct NcclApi {
  bool ok = false;
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
};

static NcclApi* nccl_api() {
  static NcclApi api;
  static bool tried = false;
  if (tried) return api.ok ? &api : nullptr;
  tried = true;
  void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
  if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
  if (!h) return nullptr;
  api.get_unique_id = (decltype(api.get_unique_id))dlsym(h, "ncclGetUniqueId");
  api.comm_init_rank = (decltype(api.comm_init_rank))dlsym(h, "ncclCommInitRank");
  api.all_reduce = (decltype(api.all_reduce))dlsym(h, "ncclAllReduce");
  api.comm_destroy = (decltype(api.comm_destroy))dlsym(h, "ncclCommDestroy");
  api.error_string = (decltype(api.error_string))dlsym(h, "ncclGetErrorString");
  api.ok = api.get_unique_id && api.comm_init_rank && api.all_reduce && api.comm_destroy && api.error_string;
  return api.ok ? &api : nullptr;
}

// Lockstep batch of B sequences sharing one position (Engine::forward over input_ids [B, T]).
struct BatchRt {
  int B = 0;
  BatchState* st = nullptr;         // device
  BatchState* h_st = nullptr;       // pinned
  int* h_tok = nullptr;             // pinned token staging [max_seq][B] + constants 0, 1
  unsigned long long* h_keys = nullptr;   // pinned [B]
  int* tok_in = nullptr;            // [B]
  unsigned long long* keys = nullptr;     // [B] argmax keys of the last step
  int* log = nullptr;               // [max_seq][B] tokens fed per step
  float *h = nullptr, *qkv = nullptr, *attn = nullptr, *xn = nullptr, *rlog = nullptr, *wts = nullptr;
  float *act = nullptr, *y = nullptr, *xf = nullptr, *logits = nullptr, *part = nullptr;
  int8_t *xq_h = nullptr, *xq_a = nullptr;
  float *xd_h = nullptr, *xd_a = nullptr;
  int *idx = nullptr, *grp = nullptr, *ent_slot = nullptr, *ent_of = nullptr;
  int* ent_zero = nullptr;          // [B K] zeros: every (token, slot) entry local (exact experts)
  int* ref_scratch = nullptr;       // exact greedy re-scoring scratch
  uint32_t *attn_cnt = nullptr, *router_cnt = nullptr;
  std::vector<float*> kc, vc;
  void* lm_scratch = nullptr;
  int64_t bs_kv_full = 0;
  std::vector<void*> allocs;
  cudaGraphExec_t graph = nullptr;
  int seq = 0;
  int kernels_per_step = 0;
  int spl_full = 0, spl_swa = 0, S_full = 0, S_swa = 0;   // attention split sizes of the batch
};

struct ms_model {
  ms_ctx* ctx = nullptr;
  ncclComm_t comm = nullptr;        // expert-parallel communicator (ep_size > 1)
  // expert parallel over peer memory (ms_model_ep_connect): mailbox recv [2][n][H] floats then
  // flags [2][n]; peers' mailboxes opened through CUDA IPC
  float* ep_mail = nullptr;
  uint32_t *ep_seq = nullptr, *ep_cnt = nullptr;
  void* ep_peer[kMaxEp] = {};
  bool ep_p2p = false;
  float* moe_out = nullptr;         // [H] local MoE output, all-reduced across the EP group
  int8_t* xq_h = nullptr;           // Q8_0 codes of the next attention input [H]
  float* xd_h = nullptr;            // and block scales [H / 32]
  int8_t* xq_a = nullptr;           // Q8_0 codes of the attention output [Dq]
  float* xd_a = nullptr;
  ms_model_config cfg{};
  std::vector<LayerW> L;
  void* embd = nullptr;
  int embd_q = -1;
  uint16_t* out_w = nullptr;
  float* out_norm = nullptr;
  float* out_b = nullptr;
  float* cos_t = nullptr;
  float* sin_t = nullptr;
  // per-step scratch
  float *h = nullptr, *qkv = nullptr, *attn_out = nullptr, *xn = nullptr, *router_logits = nullptr;
  float *act = nullptr, *partial = nullptr, *logits = nullptr, *attn_part = nullptr, *h_last = nullptr;
  uint32_t *router_cnt = nullptr, *tile_cnt = nullptr, *attn_cnt = nullptr, *resid_cnt = nullptr;
  StepState* st = nullptr;
  int* token_log = nullptr;
  int expert_base = 0, n_local = 0;
  int splits_full = 0, splits_swa = 0;
  int attn_spl = 0;                 // single-sequence attention: 0 tile kernel, else streaming split length
  std::vector<void*> allocs;
  std::set<std::string> seen;
  cudaGraphExec_t graph = nullptr;
  bool use_graph = true;
  bool finalized = false;
  int seq = 0;
  int* h_tok = nullptr;             // pinned token staging [max_seq + 1]
  StepState* h_st = nullptr;        // pinned
  int kernels_per_step = 0;
  int prof_class = -1;   // >= 0: enqueue only the launches of this class (ms_model_profile_step)
  bool use_tc = true;    // repack MXFP4 experts for the tcgen05 path (MS_MOE_TC=0 keeps native blocks)
  uint8_t* xterm = nullptr;       // B terms of the MoE input (tensor-core path)
  uint8_t* act_terms = nullptr;   // [K] B terms of the expert activations
  float* tc_part = nullptr;       // split-K partial sums
  uint32_t* tc_cnt = nullptr;
  BatchRt* bt = nullptr;          // lockstep batch state (ms_model_batch_open)
  // layer trace (ms_model_set_trace): residual stream after each layer [layers][H] and router
  // logits per layer [layers][E] of the last step, copied inside the step when enabled
  float* trace_h = nullptr;
  float* trace_logits = nullptr;
  bool trace = false;
  // multi-token forward (prompt prefill): 0 = one decode step per token, 1 = batched with the
  // expert GEMM's activations as bf16 hi + lo pairs (default), 2 = batched with bf16 activations
  int prefill_mode = 1;
  // order-independent decode kernels (f64 reductions rounded once; bit-identical to the oracle):
  // attention and MXFP4 experts; ms_model_set_exact(m, 0) selects the pipelined f32 kernels
  bool exact = true;
  // sampled decoding (ms_model_set_sampling): each step's token drawn on the device
  bool sampling = false;
  float s_temp = 1.0f, s_top_p = 1.0f, s_pen = 1.0f;
  uint32_t* s_counts = nullptr;     // [V] times each token was drawn since sampling was enabled
  float* s_work = nullptr;          // [V] sampler scratch
  unsigned long long* s_rng = nullptr;   // [seed, n]
  int* s_draw = nullptr;            // 1: this step draws its token (0 on prompt positions before the last)
  double* ex_gp = nullptr;          // [K][segments][2 I] gate/up partial dots
  double* ex_dp = nullptr;          // [K][segments][h_pad] down partial dots
  uint8_t* ex_xbt = nullptr;        // [H/32][term block] exact B terms of the MoE input
  int* ex_xfe = nullptr;            // [H/32]
  uint8_t* ex_abt = nullptr;        // [K][I/32][term block] exact B terms of the activations
  int* ex_afe = nullptr;            // [K][I/32 rounded up to 8]
  uint32_t* ex_cnt = nullptr;       // [K][gate/up tiles] per-tile arrival counters
  int ex_seg_gu = 0, ex_seg_down = 0, ex_hpad = 0;
  float* ex_kgu = nullptr;          // K-quant experts: gate / up outputs [K][2][I]
  float* xn_final = nullptr;        // the LM head's input after the final norm [H]
  int head_start = 1;               // index of the step's first LM-head launch (profiling classes)
  int* ref_scratch = nullptr;       // exact greedy re-scoring: candidate ids, counters
  // hybrid models: DeltaNet step scratch, gated attention's raw Q/gate projection, shared expert
  float *dn_mixed = nullptr, *dn_conv = nullptr, *dn_zv = nullptr, *dn_bav = nullptr, *dn_o = nullptr;
  float *q_raw = nullptr, *q_gate = nullptr;
  float *sh_g = nullptr, *sh_a = nullptr, *sh_o = nullptr, *sh_y = nullptr;
  // host-tier expert streaming (ms_model_set_expert_tier): every layer's K-quant expert stacks live
  // in pinned host memory; HBM holds tier_slots experts per layer, least recently used evicted
  struct TierLayer {
    uint8_t* host[3] = {nullptr, nullptr, nullptr};   // gate, up, down stacks [E][rows][row bytes]
    int64_t stride[3] = {0, 0, 0};                   // bytes per expert (Q6_K padded to 224-byte blocks)
    std::vector<int> slot_expert;                     // expert held by each HBM slot (-1: empty)
    std::vector<uint64_t> slot_used;                  // step of the slot's last use
    int* wslot = nullptr;                             // device [16]: weight slot of each routed slot
  };
  int tier_slots = 0;
  std::vector<TierLayer> tier;
  uint64_t tier_hits = 0, tier_misses = 0, tier_clock = 0;
  int* h_wslot = nullptr;           // pinned [layers][16] staging of the slot tables
  int* h_tier_idx = nullptr;        // pinned [16] routed ids read back per layer
  // router statistics / dynamic K: unmasked logits [E], per-layer entropy and K of the last step
  bool router_stats = false, dyn_k = false;
  float* r_raw = nullptr;
  float* r_entropy = nullptr;
  int* r_k = nullptr;
  // running totals while router statistics are on: per layer and expert the times routed and the
  // sum of routing weights, tokens per layer, and the entropy log [max_seq_len][layers]
  unsigned long long* st_cnt = nullptr;
  double* st_wsum = nullptr;
  unsigned long long* st_tok = nullptr;
  float* st_log = nullptr;
  uint32_t* st_n = nullptr;
  int sh_max = 0;                   // widest shared expert (0: none)
  struct Prefill {
    int cap = 0;                       // tokens the buffers hold
    std::vector<void*> allocs;
    int* tok = nullptr;
    float *h = nullptr, *qkv = nullptr, *q = nullptr, *kn = nullptr, *vn = nullptr, *attn = nullptr;
    float *xn = nullptr, *rlog = nullptr, *wts = nullptr, *moe_y = nullptr, *gy = nullptr, *gact = nullptr;
    int8_t* xq = nullptr;
    float* xd = nullptr;
    int *idx = nullptr, *grp = nullptr, *ent_slot = nullptr, *ent_of = nullptr;
    uint32_t* rcnt = nullptr;
    void* moe_scratch = nullptr;
  } pf;

  template <class T>
  ms_status alloc(T** p, size_t bytes, bool zero = true) {
    void* q = nullptr;
    cudaError_t e = cudaMalloc(&q, bytes ? bytes : 16);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "cudaMalloc");
    if (zero) cudaMemset(q, 0, bytes ? bytes : 16);
    allocs.push_back(q);
    *p = reinterpret_cast<T*>(q);
    return MS_OK;
  }
};

namespace {

int q_dim(const ms_model_config& c) { return c.heads * c.head_dim; }
int kv_dim(const ms_model_config& c) { return c.kv_heads * c.head_dim; }
// DeltaNet hybrids (config.rs:446-458): gated attention every attn_interval-th layer, DeltaNet otherwise
bool is_hybrid(const ms_model_config& c) { return c.attn_interval > 0; }
bool is_attention_layer(const ms_model_config& c, int li) { return c.attn_interval <= 0 || (li + 1) % c.attn_interval == 0; }
// rows of the Q projection: [Q_h, gate_h] per head in hybrid models (layer.rs:620-635)
int q_rows(const ms_model_config& c) { return (is_hybrid(c) ? 2 : 1) * q_dim(c); }
int dn_conv_dim(const ms_model_config& c) { return 2 * c.ssm_groups * c.ssm_state + c.ssm_inner; }
int dn_hvd(const ms_model_config& c) { return c.ssm_dt_rank > 0 ? c.ssm_inner / c.ssm_dt_rank : 128; }

ms_status upload(ms_model* m, void* dst, const void* src, size_t bytes) {
  cudaError_t e = cudaMemcpy(dst, src, bytes, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return cuda_fail(m->ctx, e, "upload");
  return MS_OK;
}

// f32 vector tensor [n]
ms_status set_vec(ms_model* m, float** slot, const char* name, int q, int64_t n, int64_t want, const void* data) {
  if (q != Q_F32) return fail(m->ctx, MS_ERR_UNSUPPORTED_QTYPE, "%s: expected F32", name);
  if (n != want) return fail(m->ctx, MS_ERR_SHAPE, "%s: %lld elements, expected %lld", name, (long long)n, (long long)want);
  ms_status s = m->alloc(slot, (size_t)n * 4);
  if (s != MS_OK) return s;
  return upload(m, *slot, data, (size_t)n * 4);
}

// weight allocations are padded so 16-row streaming tiles never read past the end
size_t padded(size_t bytes) { return (bytes + 16 * 4352 + 255) & ~(size_t)255; }

// Host-tier expert stack (gate 0 / up 1 / down 2) of layer li: the native blocks into pinned host
// memory (Q6_K rows padded to 224-byte superblocks, as the HBM-resident layout), and an HBM cache of
// tier_slots experts.  The reference streams expert slices from the mmap'ed GGUF into an LRU of
// dequantized experts (gguf/reader.rs:631-858, model/cache.rs:84-158); here the slices stay in their
// block format and the cache is device memory.
ms_status tier_upload(ms_model* m, int li, int which, int q, int rows, int cols, const uint8_t* src, int64_t per,
                      uint8_t** dev, int* qt) {
  if (q != Q_Q4_K && q != Q_Q6_K)
    return fail(m->ctx, MS_ERR_UNSUPPORTED_QTYPE, "host-tier expert streaming covers Q4_K / Q6_K experts (qtype %d)", q);
  if (*dev) return fail(m->ctx, MS_ERR_STATE, "expert stack of layer %d set twice", li);
  const int E = m->n_local;
  const bool q6 = q == Q_Q6_K;
  const int64_t n_sb = (int64_t)rows * (cols / 256);
  const int64_t stride = q6 ? n_sb * kQ6PadBytes : per;
  ms_model::TierLayer& T = m->tier[li];
  void* host = nullptr;
  MS_CUDA(m->ctx, cudaHostAlloc(&host, (size_t)stride * E, cudaHostAllocDefault));
  T.host[which] = (uint8_t*)host;
  T.stride[which] = stride;
  if (q6) {
    for (int64_t b = 0; b < n_sb * E; ++b) {
      std::memcpy(T.host[which] + b * kQ6PadBytes, src + b * 210, 210);
      std::memset(T.host[which] + b * kQ6PadBytes + 210, 0, kQ6PadBytes - 210);
    }
  } else {
    std::memcpy(host, src, (size_t)per * E);
  }
  *qt = q6 ? Q_Q6_K_PAD : q;
  return m->alloc(dev, padded((size_t)stride * m->tier_slots));
}

// Before a host-tier layer's expert kernels: read the routed ids back (the router has run), bring
// every routed expert missing from the layer's HBM slots in from host memory (evicting the least
// recently used slot not routed this step), and upload the slot table the expert kernels read.
// Stream-ordered: the copies and the table precede the expert kernels on `s`.
ms_status tier_fetch(ms_model* m, int li, cudaStream_t s) {
  const ms_model_config& c = m->cfg;
  ms_model::TierLayer& T = m->tier[li];
  LayerW& Lw = m->L[li];
  const int K = c.top_k, C = m->tier_slots;
  MS_CUDA(m->ctx, cudaMemcpyAsync(m->h_tier_idx, Lw.idx, (size_t)K * 4, cudaMemcpyDeviceToHost, s));
  MS_CUDA(m->ctx, cudaStreamSynchronize(s));
  const uint64_t now = ++m->tier_clock;
  int* ws = m->h_wslot + (size_t)li * 16;
  bool hit[16];
  for (int k = 0; k < K; ++k) {
    const int e = m->h_tier_idx[k];
    if (e == c.experts) { hit[k] = true; ws[k] = 0; continue; }   // a slot past a dynamic K: no expert
    if (e < 0 || e >= m->n_local) return fail(m->ctx, MS_ERR_DEVICE_INDEX, "layer %d: routed expert %d out of range", li, e);
    hit[k] = false;
    for (int j = 0; j < C; ++j)
      if (T.slot_expert[j] == e) { ws[k] = j; T.slot_used[j] = now; hit[k] = true; ++m->tier_hits; break; }
  }
  uint8_t* dst[3] = {Lw.gate, Lw.up, Lw.down};
  for (int k = 0; k < K; ++k) {
    if (hit[k]) continue;
    int best = -1;   // an empty slot first, else the least recently used slot not routed this step
    for (int j = 0; j < C; ++j) {
      if (T.slot_expert[j] < 0) { best = j; break; }
      if (T.slot_used[j] != now && (best < 0 || T.slot_used[j] < T.slot_used[best])) best = j;
    }
    if (best < 0) return fail(m->ctx, MS_ERR_STATE, "layer %d: no free expert slot", li);
    const int e = m->h_tier_idx[k];
    for (int w = 0; w < 3; ++w)
      MS_CUDA(m->ctx, cudaMemcpyAsync(dst[w] + (size_t)best * T.stride[w], T.host[w] + (size_t)e * T.stride[w],
                                      (size_t)T.stride[w], cudaMemcpyHostToDevice, s));
    T.slot_expert[best] = e;
    T.slot_used[best] = now;
    ws[k] = best;
    ++m->tier_misses;
  }
  MS_CUDA(m->ctx, cudaMemcpyAsync(T.wslot, ws, (size_t)K * 4, cudaMemcpyHostToDevice, s));
  return MS_OK;
}

ms_status set_layer_tensor(ms_model* m, int li, const std::string& t, int q, const std::vector<int64_t>& dims,
                           const void* data, size_t bytes) {
  const ms_model_config& c = m->cfg;
  LayerW& Lw = m->L[li];
  const char* nm = t.c_str();
  int64_t n = 1;
  for (auto d : dims) n *= d;
  const int H = c.hidden, Dq = q_dim(c), Dkv = kv_dim(c);
  if (raw_bytes(q, n) < 0) return fail(m->ctx, MS_ERR_UNSUPPORTED_QTYPE, "%s: qtype %d", nm, q);
  if ((int64_t)bytes < raw_bytes(q, n)) return fail(m->ctx, MS_ERR_SHAPE, "%s: %zu bytes < %lld", nm, bytes, (long long)raw_bytes(q, n));
  if (t == "attn_norm.weight") return set_vec(m, &Lw.attn_norm, nm, q, n, H, data);
  if (t == "post_attention_norm.weight" || t == "ffn_norm.weight") return set_vec(m, &Lw.post_norm, nm, q, n, H, data);
  if (t == "attn_sinks.weight") return set_vec(m, &Lw.sinks, nm, q, n, c.heads, data);
  if (t == "attn_q_norm.weight") return set_vec(m, &Lw.qn, nm, q, n, c.head_dim, data);
  if (t == "attn_k_norm.weight") return set_vec(m, &Lw.kn, nm, q, n, c.head_dim, data);
  if (t == "attn_output.bias") return set_vec(m, &Lw.bo, nm, q, n, H, data);
  if (t == "ffn_gate_inp.bias") return set_vec(m, &Lw.router_b, nm, q, n, c.experts, data);
  if (t == "attn_q.weight" || t == "attn_k.weight" || t == "attn_v.weight") {
    // q, k, v rows are concatenated into one [Qr + 2 Dkv, H] projection (row layout unchanged);
    // Qr = Dq, or 2 Dq with [Q_h, gate_h] per head in hybrid models
    const int Qr = q_rows(c);
    const int rows = t == "attn_q.weight" ? Qr : Dkv;
    const int off = t == "attn_q.weight" ? 0 : (t == "attn_k.weight" ? Qr : Qr + Dkv);
    if (dims.size() != 2 || dims[0] != rows || dims[1] != H) return fail(m->ctx, MS_ERR_SHAPE, "%s: bad shape", nm);
    if (q != Q_Q8_0) return fail(m->ctx, MS_ERR_UNSUPPORTED_QTYPE, "%s: attention projections must be Q8_0", nm);
    if (Lw.attn_q >= 0 && Lw.attn_q != q) return fail(m->ctx, MS_ERR_UNSUPPORTED_QTYPE, "%s: mixed qtypes", nm);
    Lw.attn_q = q;
    const int64_t rb = row_bytes(q, H);
    if (!Lw.wqkv) {
      ms_status s = m->alloc(&Lw.wqkv, padded((size_t)(Qr + 2 * Dkv) * rb));
      if (s != MS_OK) return s;
    }
    ++Lw.qkv_parts;
    return upload(m, Lw.wqkv + (size_t)off * rb, data, (size_t)rows * rb);
  }
  if (t == "attn_q.bias" || t == "attn_k.bias" || t == "attn_v.bias") {
    const int Qr = q_rows(c);
    const int rows = t == "attn_q.bias" ? Qr : Dkv;
    const int off = t == "attn_q.bias" ? 0 : (t == "attn_k.bias" ? Qr : Qr + Dkv);
    if (q != Q_F32 || n != rows) return fail(m->ctx, MS_ERR_SHAPE, "%s: bad bias", nm);
    if (!Lw.bqkv) {
      ms_status s = m->alloc(&Lw.bqkv, (size_t)(Qr + 2 * Dkv) * 4);
      if (s != MS_OK) return s;
    }
    ++Lw.bqkv_parts;
    return upload(m, Lw.bqkv + off, data, (size_t)rows * 4);
  }
  if (t == "attn_output.weight") {
    if (dims.size() != 2 || dims[0] != H || dims[1] != Dq) return fail(m->ctx, MS_ERR_SHAPE, "%s: bad shape", nm);
    if (q != Q_Q8_0) return fail(m->ctx, MS_ERR_UNSUPPORTED_QTYPE, "%s: must be Q8_0", nm);
    ms_status s = m->alloc(&Lw.wo, padded(bytes));
    if (s != MS_OK) return s;
    return upload(m, Lw.wo, data, (size_t)raw_bytes(q, n));
  }
  // ---- Gated DeltaNet projections and tensors (deltanet.rs:101-137, 204-543) and the shared expert
  // (layer.rs:2250-2293).  Projections run as f32-activation GEMVs over the native blocks, the
  // reference's dequantize-then-matmul (Q8_0 would need the f32 activation too, so it is refused).
  {
    const int conv_dim = dn_conv_dim(c), vt = c.ssm_inner, nv = c.ssm_dt_rank;
    struct Proj { const char* name; uint8_t** w; int* qt; int rows, cols; bool dn; };
    const Proj projs[] = {
        {"attn_qkv.weight", &Lw.dn_qkv, &Lw.dn_qkv_q, conv_dim, H, true},
        {"attn_gate.weight", &Lw.dn_z, &Lw.dn_z_q, vt, H, true},
        {"ssm_ba.weight", &Lw.dn_ba, &Lw.dn_ba_q, 2 * nv, H, true},
        {"ssm_beta.weight", &Lw.dn_ba, &Lw.dn_ba_q, nv, H, true},
        {"ssm_alpha.weight", &Lw.dn_ba, &Lw.dn_ba_q, nv, H, true},
        {"ssm_out.weight", &Lw.dn_out, &Lw.dn_out_q, H, vt, true},
        {"ffn_gate_shexp.weight", &Lw.sh_gate, &Lw.sh_gate_q, -1, H, false},
        {"ffn_up_shexp.weight", &Lw.sh_up, &Lw.sh_up_q, -1, H, false},
        {"ffn_down_shexp.weight", &Lw.sh_down, &Lw.sh_down_q, H, -1, false}};
    for (const Proj& P : projs) {
      if (t != P.name) continue;
      if (P.dn && (!is_hybrid(c) || is_attention_layer(c, li)))
        return fail(m->ctx, MS_ERR_STATE, "%s: layer %d is not a DeltaNet layer", nm, li);
      if (q != Q_F32 && q != Q_Q4_K && q != Q_Q6_K && q != Q_MXFP4)
        return fail(m->ctx, MS_ERR_UNSUPPORTED_QTYPE, "%s: qtype %d (F32, Q4_K, Q6_K or MXFP4 required)", nm, q);
      if (dims.size() != 2) return fail(m->ctx, MS_ERR_SHAPE, "%s: 2-D tensor expected", nm);
      const int rows = P.rows > 0 ? P.rows : (int)dims[0], cols = P.cols > 0 ? P.cols : (int)dims[1];
      if (dims[0] != rows || dims[1] != cols || row_bytes(q, cols) <= 0)
        return fail(m->ctx, MS_ERR_SHAPE, "%s: expected [%d, %d]", nm, rows, cols);
      const int64_t rb = row_bytes(q, cols);
      const bool split_ba = t == "ssm_beta.weight" || t == "ssm_alpha.weight";
      if (*P.qt >= 0 && *P.qt != q) return fail(m->ctx, MS_ERR_UNSUPPORTED_QTYPE, "%s: mixed qtypes", nm);
      *P.qt = q;
      if (P.w == &Lw.sh_gate) Lw.sh_dims[0] = rows;
      if (P.w == &Lw.sh_up) Lw.sh_dims[1] = rows;
      if (P.w == &Lw.sh_down) Lw.sh_dims[2] = cols;
      if (*P.w && !split_ba) return fail(m->ctx, MS_ERR_STATE, "%s: set twice", nm);
      // beta rows first, then alpha rows (deltanet.rs:118-125)
      const size_t sub = t == "ssm_alpha.weight" ? (size_t)nv * rb : 0;
      if (t == "ssm_ba.weight" || split_ba) Lw.dn_ba_parts += split_ba ? 1 : 2;
      const bool dn_in = P.w == &Lw.dn_qkv || P.w == &Lw.dn_z || P.w == &Lw.dn_ba;
      const bool sh_in = P.w == &Lw.sh_gate || P.w == &Lw.sh_up;
      if (dn_in && !Lw.dn_in) {   // [qkv | z | ba] rows in one buffer, whole 16-row tiles
        ms_status s = m->alloc(&Lw.dn_in, padded((size_t)((conv_dim + vt + 2 * nv + 15) / 16 * 16) * rb));
        if (s != MS_OK) return s;
        Lw.dn_in_q = q;
      }
      if (sh_in && !Lw.sh_gu) {   // [gate | up] rows in one buffer
        ms_status s = m->alloc(&Lw.sh_gu, padded((size_t)((2 * rows + 15) / 16 * 16) * rb));
        if (s != MS_OK) return s;
        Lw.sh_gu_q = q;
        Lw.sh_gu_rows = rows;
      }
      if (!*P.w) {
        if (dn_in && Lw.dn_in_q == q) {
          const int r0 = P.w == &Lw.dn_qkv ? 0 : (P.w == &Lw.dn_z ? conv_dim : conv_dim + vt);
          *P.w = Lw.dn_in + (size_t)r0 * rb;
        } else if (sh_in && Lw.sh_gu_q == q && Lw.sh_gu_rows == rows) {
          *P.w = Lw.sh_gu + (P.w == &Lw.sh_up ? (size_t)rows * rb : 0);
        } else {   // own buffer, whole 16-row tiles for the GEMV's row streaming
          const int alloc_rows = split_ba ? 2 * nv : rows;
          ms_status s = m->alloc(P.w, padded((size_t)((alloc_rows + 15) / 16 * 16) * rb));
          if (s != MS_OK) return s;
        }
      }
      return upload(m, *P.w + sub, data, (size_t)rows * rb);
    }
    if (t == "ssm_conv1d.weight") {
      if (!is_hybrid(c) || is_attention_layer(c, li)) return fail(m->ctx, MS_ERR_STATE, "%s: not a DeltaNet layer", nm);
      if (q != Q_F32 || n != (int64_t)conv_dim * c.ssm_conv)
        return fail(m->ctx, MS_ERR_SHAPE, "%s: expected F32 [%d, %d]", nm, conv_dim, c.ssm_conv);
      return set_vec(m, &Lw.dn_conv_w, nm, q, n, n, data);
    }
    if (t == "ssm_a") return set_vec(m, &Lw.dn_a, nm, q, n, nv, data);
    if (t == "ssm_dt.bias") return set_vec(m, &Lw.dn_dt, nm, q, n, nv, data);
    if (t == "ssm_norm.weight") return set_vec(m, &Lw.dn_norm, nm, q, n, dn_hvd(c), data);
    if (t == "ffn_gate_inp_shexp.weight") return set_vec(m, &Lw.sh_gate_inp, nm, q, n, H, data);
  }
  if (t == "ffn_gate_inp.weight") {
    if (q != Q_F32 || dims.size() != 2 || dims[0] != c.experts || dims[1] != H)
      return fail(m->ctx, MS_ERR_SHAPE, "%s: expected F32 [%d, %d]", nm, c.experts, H);
    ms_status s = set_vec(m, &Lw.router_w, nm, q, n, (int64_t)c.experts * H, data);
    if (s != MS_OK) return s;
    // engine.rs:628-652: a router row constant within 1e-6 marks a dummy (padded) expert
    std::vector<uint8_t> mask(c.experts, 0);
    const float* w = (const float*)data;
    for (int e = 0; e < c.experts; ++e) {
      const float* r = w + (size_t)e * H;
      bool uni = true;
      for (int i = 0; i < H && uni; ++i) uni = std::fabs(r[i] - r[0]) < 1e-6f;
      mask[e] = uni ? 1 : 0;
    }
    s = m->alloc(&Lw.mask, c.experts);
    if (s != MS_OK) return s;
    return upload(m, Lw.mask, mask.data(), c.experts);
  }
  // stacked experts: keep only this rank's contiguous slice [base, base + n_local)
  struct { const char* name; uint8_t** w; float** b; int* qt; int rows, cols; } ex[3] = {
      {"ffn_gate_exps", &Lw.gate, &Lw.gate_b, &Lw.gate_q, c.inter, H},
      {"ffn_up_exps", &Lw.up, &Lw.up_b, &Lw.up_q, c.inter, H},
      {"ffn_down_exps", &Lw.down, &Lw.down_b, &Lw.down_q, H, c.inter}};
  for (auto& x : ex) {
    const std::string wn = std::string(x.name) + ".weight", bn = std::string(x.name) + ".bias";
    if (t == wn) {
      if (dims.size() != 3 || dims[0] != c.experts || dims[1] != x.rows || dims[2] != x.cols)
        return fail(m->ctx, MS_ERR_SHAPE, "%s: expected [%d, %d, %d]", nm, c.experts, x.rows, x.cols);
      if (q != Q_MXFP4 && q != Q_Q4_K && q != Q_Q6_K)
        return fail(m->ctx, MS_ERR_UNSUPPORTED_QTYPE, "%s: expert qtype %d not supported", nm, q);
      const int64_t per = raw_bytes(q, (int64_t)x.rows * x.cols);
      *x.qt = q;
      const bool is_down = x.w == &Lw.down;
      (is_down ? Lw.have_down : (x.w == &Lw.gate ? Lw.have_gate : Lw.have_up)) = true;
      if (m->tier_slots > 0)
        return tier_upload(m, li, is_down ? 2 : (x.w == &Lw.gate ? 0 : 1), q, x.rows, x.cols,
                           (const uint8_t*)data + per * m->expert_base, per, x.w, x.qt);
      if (q == Q_MXFP4 && m->use_tc && tc_supported(H, c.inter)) {
        // repack this rank's experts into tensor-core tiles (gate rows 0-63 and up rows 64-127 of a
        // gate_up tile; 128 hidden rows per down tile); the native blocks are not kept
        uint8_t** dst = is_down ? &Lw.down_tc : &Lw.gu_tc;
        const int tiles = is_down ? tc_down_tiles(H) : tc_gu_tiles(c.inter);
        const int64_t tbytes = tc_tile_bytes(x.cols / 32);
        // zeroing, upload and repack are ordered on the context's private stream (which does not
        // synchronise with the legacy stream), then waited for
        cudaStream_t os = m->ctx->own;
        const size_t pbytes = (size_t)m->n_local * tiles * tbytes;
        const bool fresh = *dst == nullptr;
        if (fresh) {
          ms_status s = m->alloc(dst, pbytes, false);
          if (s != MS_OK) return s;
        }
        void* tmp = nullptr;
        MS_CUDA(m->ctx, cudaMalloc(&tmp, (size_t)per * m->n_local));
        cudaError_t e = fresh ? cudaMemsetAsync(*dst, 0, pbytes, os) : cudaSuccess;
        if (e == cudaSuccess)
          e = cudaMemcpyAsync(tmp, (const uint8_t*)data + per * m->expert_base, (size_t)per * m->n_local,
                              cudaMemcpyHostToDevice, os);
        if (e == cudaSuccess)
          e = launch_mxfp4_pack((const uint8_t*)tmp, m->n_local, x.rows, x.cols, is_down ? 128 : 64,
                                x.w == &Lw.up ? 64 : 0, tiles, *dst, os);
        if (e == cudaSuccess) e = cudaStreamSynchronize(os);
        cudaFree(tmp);
        if (e != cudaSuccess) return cuda_fail(m->ctx, e, "mxfp4 repack");
        return MS_OK;
      }
      if (q == Q_Q6_K) {
        // Q6_K rows are repacked into 224-byte superblocks (same bytes + 14 bytes of padding) so
        // the expert kernels read aligned code words and copy rows into bank-padded stages
        const int64_t n_sb = (int64_t)m->n_local * x.rows * (x.cols / 256);
        ms_status s = m->alloc(x.w, padded((size_t)n_sb * kQ6PadBytes));
        if (s != MS_OK) return s;
        cudaStream_t os = m->ctx->own;
        void* tmp = nullptr;
        MS_CUDA(m->ctx, cudaMalloc(&tmp, (size_t)per * m->n_local));
        cudaError_t e = cudaMemcpyAsync(tmp, (const uint8_t*)data + per * m->expert_base, (size_t)per * m->n_local,
                                        cudaMemcpyHostToDevice, os);
        if (e == cudaSuccess) e = launch_q6k_pad((const uint8_t*)tmp, n_sb, *x.w, os);
        if (e == cudaSuccess) e = cudaStreamSynchronize(os);
        cudaFree(tmp);
        if (e != cudaSuccess) return cuda_fail(m->ctx, e, "q6_k repack");
        *x.qt = Q_Q6_K_PAD;
        return MS_OK;
      }
      ms_status s = m->alloc(x.w, padded((size_t)per * m->n_local));
      if (s != MS_OK) return s;
      return upload(m, *x.w, (const uint8_t*)data + per * m->expert_base, (size_t)per * m->n_local);
    }
    if (t == bn) {
      if (q != Q_F32 || n != (int64_t)c.experts * x.rows) return fail(m->ctx, MS_ERR_SHAPE, "%s: bad bias", nm);
      ms_status s = m->alloc(x.b, (size_t)x.rows * m->n_local * 4);
      if (s != MS_OK) return s;
      return upload(m, *x.b, (const float*)data + (size_t)x.rows * m->expert_base, (size_t)x.rows * m->n_local * 4);
    }
  }
  return MS_OK;   // tensors outside the decode path are ignored (as the reference ignores them)
}

// ops/attention.rs:9-34 evaluated on the host exactly as the reference does (f64 pow, f32 tables)
void rope_tables(int rot, int max_seq, double theta, std::vector<float>& cs, std::vector<float>& sn) {
  const int half = rot / 2;
  std::vector<float> inv(half);
  for (int i = 0; i < half; ++i) inv[i] = 1.0f / (float)std::pow(theta, 2.0 * (double)i / (double)rot);
  cs.resize((size_t)max_seq * half);
  sn.resize(cs.size());
  for (int p = 0; p < max_seq; ++p)
    for (int i = 0; i < half; ++i) {
      const float f = (float)p * inv[i];
      cs[(size_t)p * half + i] = std::cos(f);
      sn[(size_t)p * half + i] = std::sin(f);
    }
}

// launch i of a step: 0 = embed, the last = LM head, else 1 + its position within the layer
int launch_class(const ms_model* m, int i) {
  const int per_layer = (m->head_start - 1) / m->cfg.layers;
  if (i == 0) return 0;
  if (i >= m->head_start) return 1 + per_layer;
  return 1 + (i - 1) % per_layer;
}

// rows per parity of a peer mailbox: one per rank (combined outputs) or one per slot (exact mode)
int ep_rows(const ms_model* m) { return std::max(m->cfg.ep_size, m->cfg.top_k); }

// the order-independent attention covers head dims 32 / 64 / 128 and up to 32 query heads per kv head
bool exact_attn_ok(const ms_model* m) {
  const ms_model_config& c = m->cfg;
  const int rep = c.heads / c.kv_heads;
  return m->exact && (c.head_dim == 32 || c.head_dim == 64 || c.head_dim == 128) && 32 % rep == 0 &&
         (c.head_dim < 128 || rep <= 8);
}

SampleArgs sample_args(ms_model* m) {
  SampleArgs a;
  a.logits = m->logits; a.V = m->cfg.vocab; a.counts = m->s_counts; a.counts_rw = m->s_counts;
  a.temperature = m->s_temp; a.top_p = m->s_top_p; a.penalty = m->s_pen; a.rng = m->s_rng; a.work = m->s_work;
  a.key_out = &m->st->key; a.draw = m->s_draw;
  return a;
}

ms_status enqueue_step(ms_model* m, cudaStream_t s) {
  const ms_model_config& c = m->cfg;
  const DevCtx& dc = m->ctx->dc;
  const int H = c.hidden, Dq = q_dim(c), Dkv = kv_dim(c);
  int nk = 0;
#define LAUNCH(call)                                                       \
  do {                                                                     \
    if (m->prof_class < 0 || launch_class(m, nk) == m->prof_class) {       \
      cudaError_t e_ = (call);                                             \
      if (e_ != cudaSuccess) return cuda_fail(m->ctx, e_, #call);         \
    }                                                                      \
    ++nk;                                                                  \
  } while (0)
  // Every Q8_0 projection gets its activation already quantized by the kernel that produced it:
  // the embedding (layer 0), the residual-update kernel after each MoE (next layer's attention
  // input), and the attention merge (O-projection input).
  LAUNCH(launch_embed(dc, m->st, m->embd, m->embd_q, H, c.vocab, m->h, m->token_log, s, m->L[0].attn_norm, c.eps,
                      m->xq_h, m->xd_h));
  for (int li = 0; li < c.layers; ++li) {
    LayerW& Lw = m->L[li];
    if (Lw.deltanet) {
      // Gated DeltaNet mixer (deltanet.rs:204-543): h += out(gated RMSNorm(delta rule(conv(qkv x)))),
      // x = RMSNorm(h); f32-activation GEMVs over the native blocks, as the reference's dequantize + matmul
      const int conv_dim = dn_conv_dim(c), vt = c.ssm_inner, nv = c.ssm_dt_rank;
      LAUNCH(launch_rms_norm(dc, m->h, Lw.attn_norm, m->xn, 1, H, c.eps, s));
      GemvArgs g;
      g.qtype = Lw.dn_qkv_q; g.w = Lw.dn_qkv; g.rows = conv_dim; g.cols = H; g.x = m->xn; g.y = m->dn_mixed;
      const int64_t rb_in = row_bytes(Lw.dn_qkv_q, H);
      if (Lw.dn_z_q == Lw.dn_qkv_q && Lw.dn_ba_q == Lw.dn_qkv_q && Lw.dn_z == Lw.dn_qkv + (size_t)conv_dim * rb_in &&
          Lw.dn_ba == Lw.dn_z + (size_t)vt * rb_in) {
        g.rows = conv_dim + vt + 2 * nv;   // qkv, z, beta / alpha rows in one launch
        LAUNCH(launch_gemv(dc, g, s));
      } else {
        LAUNCH(launch_gemv(dc, g, s));
        g.qtype = Lw.dn_z_q; g.w = Lw.dn_z; g.rows = vt; g.y = m->dn_zv;
        LAUNCH(launch_gemv(dc, g, s));
        g.qtype = Lw.dn_ba_q; g.w = Lw.dn_ba; g.rows = 2 * nv; g.y = m->dn_bav;
        LAUNCH(launch_gemv(dc, g, s));
      }
      DeltaNetStep da;
      da.nk = c.ssm_groups; da.hkd = c.ssm_state; da.nv = nv; da.hvd = dn_hvd(c); da.eps = c.eps;
      da.scale = 1.0f / sqrtf((float)da.hvd); da.conv_out = m->dn_conv; da.ba = m->dn_bav; da.z = m->dn_zv;
      da.ssm_a = Lw.dn_a; da.dt_bias = Lw.dn_dt; da.norm = Lw.dn_norm; da.state = Lw.dn_state; da.out = m->dn_o;
      LAUNCH(launch_deltanet_core(dc, da, conv_dim, c.ssm_conv, m->dn_mixed, Lw.dn_conv_w, Lw.dn_conv_state, s));
      ++nk;   // conv + delta rule
      g.qtype = Lw.dn_out_q; g.w = Lw.dn_out; g.rows = H; g.cols = vt; g.x = m->dn_o; g.y = m->h; g.accumulate = 1;
      LAUNCH(launch_gemv(dc, g, s));   // h = h + out (the residual add, layer.rs:455)
    } else {
    const bool gated = is_hybrid(c);   // [Q_h, gate_h] per head, output x sigmoid(gate) (layer.rs:620-635, 699-705)
    Q8GemvArgs qa;
    qa.w = Lw.wqkv; qa.rows = q_rows(c) + 2 * Dkv; qa.cols = H; qa.xq_in = m->xq_h; qa.xd_in = m->xd_h;
    qa.bias = Lw.bqkv; qa.y = gated ? m->q_raw : m->qkv;
    LAUNCH(launch_q8_gemv(dc, qa, s));
    if (gated) LAUNCH(launch_gate_split(m->q_raw, c.heads, c.head_dim, Dkv, m->qkv, m->q_gate, s));
    AttnArgs aa;
    aa.qkv = m->qkv; aa.q_norm = Lw.qn; aa.k_norm = Lw.kn; aa.eps = c.eps; aa.cos_t = m->cos_t; aa.sin_t = m->sin_t;
    aa.rot = c.rot_dim; aa.pos = &m->st->pos; aa.kc = Lw.kc; aa.vc = Lw.vc; aa.cap = Lw.cap; aa.window = Lw.window;
    aa.sinks = Lw.sinks; aa.part = m->attn_part; aa.cnt = m->attn_cnt; aa.out = m->attn_out; aa.nh = c.heads;
    aa.nkv = c.kv_heads; aa.hd = c.head_dim; aa.S = Lw.window ? m->splits_swa : m->splits_full; aa.spl = m->attn_spl;
    // single sequence, streaming kernel: several CTAs per kv head (each a group of its query heads) fill the GPU
    if (m->attn_spl && (c.heads / c.kv_heads) % 4 == 0) aa.head_split = 4;
    else if (m->attn_spl && (c.heads / c.kv_heads) % 2 == 0 && c.heads / c.kv_heads >= 4) aa.head_split = 2;
    aa.scale = (float)(1.0 / std::sqrt((double)c.head_dim));
    // the O projection's Q8_0 activation comes from the attention kernel, or after the gate
    aa.oq = gated ? nullptr : m->xq_a;
    aa.od = gated ? nullptr : m->xd_a;
    if (exact_attn_ok(m)) LAUNCH(launch_exact_attention(dc, aa, Lw.window ? Lw.cap : c.max_seq_len, s));
    else LAUNCH(launch_attention(dc, aa, s));
    if (gated) LAUNCH(launch_gate_apply_q8(m->attn_out, m->q_gate, Dq, m->xq_a, m->xd_a, s));
    Q8GemvArgs oa;
    oa.w = Lw.wo; oa.rows = H; oa.cols = Dq; oa.xq_in = m->xq_a; oa.xd_in = m->xd_a; oa.bias = Lw.bo;
    oa.residual = m->h;
    LAUNCH(launch_q8_gemv(dc, oa, s));
    }
    RouterArgs ra;
    ra.h = m->h; ra.norm_w = Lw.post_norm; ra.eps = c.eps; ra.xn = m->xn; ra.w = Lw.router_w; ra.b = Lw.router_b;
    ra.mask = Lw.mask; ra.logits = m->router_logits; ra.idx = Lw.idx; ra.wts = Lw.wts; ra.counter = m->router_cnt;
    ra.H = H; ra.E = c.experts; ra.K = c.top_k; ra.softmax_weight = c.arch == MS_ARCH_GPT_OSS;
    ra.normalize = c.norm_topk_prob;
    if (m->router_stats || m->dyn_k) {   // entropy of the routing (and dynamic K), layer.rs:980-1011
      ra.raw = m->r_raw; ra.entropy = m->r_entropy + li; ra.k_used = m->r_k + li;
      if (m->dyn_k) { ra.k_lo = Lw.dk_lo; ra.k_hi = Lw.dk_hi; }
    }
    if (m->router_stats) {   // running totals (RoutingStatsCollector, EntropyProfiler)
      ra.cnt = m->st_cnt + (size_t)li * c.experts; ra.wsum = m->st_wsum + (size_t)li * c.experts;
      ra.tokens = m->st_tok + li; ra.ent_log = m->st_log + li; ra.ent_n = m->st_n + li;
      ra.ent_cap = c.max_seq_len; ra.ent_stride = c.layers;
    }
    if (Lw.tc && m->exact) {
      ra.xbt = m->ex_xbt;
      ra.xfe = m->ex_xfe;
    } else if (Lw.tc) {
      ra.xterm = m->xterm;
    }
    LAUNCH(launch_router(dc, ra, s));
    if (m->trace && m->prof_class < 0) {
      cudaError_t e_ = cudaMemcpyAsync(m->trace_logits + (size_t)li * c.experts, m->router_logits,
                                       (size_t)c.experts * 4, cudaMemcpyDeviceToDevice, s);
      if (e_ != cudaSuccess) return cuda_fail(m->ctx, e_, "trace copy");
    }
    TcMoeArgs ta;
    ta.gu = Lw.gu_tc; ta.down = Lw.down_tc; ta.gate_b = Lw.gate_b; ta.up_b = Lw.up_b; ta.down_b = Lw.down_b;
    ta.xterm = m->xterm; ta.act_terms = m->act_terms; ta.act = m->act; ta.partial = m->partial; ta.part = m->tc_part;
    ta.cnt = m->tc_cnt; ta.idx = Lw.idx; ta.wts = Lw.wts; ta.H = H; ta.I = c.inter; ta.K = c.top_k;
    ta.expert_base = m->expert_base; ta.n_local = m->n_local; ta.oai_swiglu = c.arch == MS_ARCH_GPT_OSS; ta.h = m->h;
    MoeArgs ma;
    ma.gate_q = Lw.gate_q; ma.down_q = Lw.down_q;
    ma.x = m->xn; ma.idx = Lw.idx; ma.wts = Lw.wts; ma.gate = Lw.gate; ma.up = Lw.up; ma.down = Lw.down;
    ma.gate_b = Lw.gate_b; ma.up_b = Lw.up_b; ma.down_b = Lw.down_b; ma.act = m->act; ma.partial = m->partial;
    ma.tile_cnt = m->tile_cnt; ma.h = m->h; ma.H = H; ma.I = c.inter; ma.K = c.top_k;
    ma.expert_base = m->expert_base; ma.n_local = m->n_local; ma.oai_swiglu = c.arch == MS_ARCH_GPT_OSS;
    PendingCombine pc;
    const bool exact_kq = m->exact && !Lw.tc && exact_kq_supported(Lw.gate_q, Lw.down_q, H, c.inter) &&
                          Lw.up_q == Lw.gate_q;
    if (m->tier_slots > 0 && !exact_kq)   // the slot table is read by the order-independent K-quant kernels only
      return fail(m->ctx, MS_ERR_STATE, "layer %d: host-tier experts need the order-independent K-quant kernels", li);
    if ((m->exact && Lw.tc) || exact_kq) {
      // order-independent experts: f64 partial dots; the combine (residual kernel, the peer-mailbox
      // send, or a combine kernel before the NCCL all-reduce) sums segments in ascending expert id
      PendingCombine lc;
      if (Lw.tc) {
        ExactMoeArgs ea;
        ea.gu = Lw.gu_tc; ea.down = Lw.down_tc; ea.gate_b = Lw.gate_b; ea.up_b = Lw.up_b; ea.x = m->xn; ea.idx = Lw.idx;
        ea.H = H; ea.I = c.inter; ea.K = c.top_k; ea.expert_base = m->expert_base; ea.n_local = m->n_local;
        ea.oai_swiglu = c.arch == MS_ARCH_GPT_OSS; ea.gp = m->ex_gp; ea.dp = m->ex_dp; ea.n_seg_gu = m->ex_seg_gu;
        ea.n_seg_down = m->ex_seg_down; ea.h_pad = m->ex_hpad;
        ea.xbt = m->ex_xbt; ea.xfe = m->ex_xfe; ea.abt = m->ex_abt; ea.afe = m->ex_afe; ea.cnt = m->ex_cnt;
        ea.down_b = Lw.down_b; ea.y = m->partial;
        LAUNCH(launch_exact_moe(dc, ea, s, 0));   // gate/up (+ activation digits)
        LAUNCH(launch_exact_moe(dc, ea, s, 1));   // down
        lc.partial = m->partial;
      } else {
        ExactKqArgs ka;
        ka.gate = Lw.gate; ka.up = Lw.up; ka.down = Lw.down; ka.gate_fmt = Lw.gate_q; ka.down_fmt = Lw.down_q;
        ka.gate_b = Lw.gate_b; ka.up_b = Lw.up_b; ka.down_b = Lw.down_b; ka.x = m->xn; ka.idx = Lw.idx; ka.H = H;
        ka.I = c.inter; ka.K = c.top_k; ka.expert_base = m->expert_base; ka.n_local = m->n_local;
        ka.oai_swiglu = c.arch == MS_ARCH_GPT_OSS; ka.gu_out = m->ex_kgu; ka.y = m->partial;
        if (m->tier_slots > 0) {   // host tier: routed experts into this layer's HBM slots first
          ms_status ts = tier_fetch(m, li, s);
          if (ts != MS_OK) return ts;
          ka.wslot = m->tier[li].wslot;
        }
        LAUNCH(launch_exact_kq_moe(dc, ka, s));
        ++nk;   // gate/up, down
        lc.partial = m->partial;
      }
      lc.idx = Lw.idx; lc.wts = Lw.wts; lc.K = c.top_k; lc.expert_base = m->expert_base; lc.n_local = m->n_local;
      if (c.ep_size > 1 && m->ep_p2p) {
        const int n = c.ep_size;
        EpSend e;
        for (int j = 0; j < n; ++j) {
          float* mb = j == c.ep_rank ? m->ep_mail : reinterpret_cast<float*>(m->ep_peer[j]);
          e.recv[j] = mb;
          e.flags[j] = reinterpret_cast<uint32_t*>(mb + (size_t)2 * ep_rows(m) * H);
        }
        e.seq = m->ep_seq; e.cnt = m->ep_cnt; e.rank = c.ep_rank; e.n = n; e.rows = ep_rows(m); e.slots = 1;
        LAUNCH(launch_ep_send(dc, lc, H, e, s));
        pc.ep_recv = m->ep_mail; pc.ep_flags = reinterpret_cast<const uint32_t*>(m->ep_mail + (size_t)2 * ep_rows(m) * H);
        pc.ep_seq = m->ep_seq; pc.ep_n = n; pc.ep_rows = ep_rows(m); pc.ep_slots = 1;
        // the receiving combine walks every slot (all experts), in ascending expert id
        pc.idx = Lw.idx; pc.wts = Lw.wts; pc.K = c.top_k; pc.expert_base = 0; pc.n_local = c.experts;
      } else if (c.ep_size > 1) {
        LAUNCH(launch_moe_combine(dc, lc, H, nullptr, m->moe_out, s));
        NcclApi* api = nccl_api();
        ncclResult_t r = api->all_reduce(m->moe_out, m->moe_out, (size_t)H, ncclFloat32, ncclSum, m->comm, s);
        if (r != ncclSuccess) return fail(m->ctx, MS_ERR_NCCL, "ncclAllReduce: %s", api->error_string(r));
        pc.dense = m->moe_out;
      } else {
        pc = lc;
      }
    } else if (c.ep_size > 1 && m->ep_p2p) {
      // expert parallel over peer memory: the local experts' combine goes straight into every
      // rank's mailbox (one kernel); the residual kernel waits for all ranks and sums them
      ma.defer_combine = 1;
      ta.defer_combine = 1;
      PendingCombine lc;
      if (Lw.tc) {
        LAUNCH(launch_moe_tc(dc, ta, s));
        lc = tc_pending_combine(dc, ta);
      } else {
        LAUNCH(launch_moe_mxfp4(dc, ma, s));
        ++nk;   // gate/up, down
        lc.partial = m->partial; lc.idx = Lw.idx; lc.wts = Lw.wts; lc.K = c.top_k;
        lc.expert_base = m->expert_base; lc.n_local = m->n_local;
      }
      const int n = c.ep_size;
      EpSend e;
      for (int j = 0; j < n; ++j) {
        float* mb = j == c.ep_rank ? m->ep_mail : reinterpret_cast<float*>(m->ep_peer[j]);
        e.recv[j] = mb;
        e.flags[j] = reinterpret_cast<uint32_t*>(mb + (size_t)2 * ep_rows(m) * H);
      }
      e.seq = m->ep_seq; e.cnt = m->ep_cnt; e.rank = c.ep_rank; e.n = n; e.rows = ep_rows(m);
      LAUNCH(launch_ep_send(dc, lc, H, e, s));
      pc.ep_recv = m->ep_mail; pc.ep_flags = reinterpret_cast<const uint32_t*>(m->ep_mail + (size_t)2 * ep_rows(m) * H);
      pc.ep_seq = m->ep_seq; pc.ep_n = n; pc.ep_rows = ep_rows(m);
    } else if (c.ep_size > 1) {
      // expert parallel: combine the local experts into moe_out, sum it over the EP group
      ma.defer_combine = 0; ma.out = m->moe_out;
      ta.defer_combine = 0; ta.out = m->moe_out;
      if (Lw.tc) {
        LAUNCH(launch_moe_tc(dc, ta, s));
        nk += 1;   // gate_up + down (one kernel), combine
      } else {
        LAUNCH(launch_moe_mxfp4(dc, ma, s));
        nk += 2;   // gate/up, down, combine
      }
      NcclApi* api = nccl_api();
      ncclResult_t r = api->all_reduce(m->moe_out, m->moe_out, (size_t)H, ncclFloat32, ncclSum, m->comm, s);
      if (r != ncclSuccess) return fail(m->ctx, MS_ERR_NCCL, "ncclAllReduce: %s", api->error_string(r));
      pc.dense = m->moe_out;
    } else {
      ma.defer_combine = 1;   // per-slot outputs stay in `partial`; the next kernel combines them
      ta.defer_combine = 1;
      if (Lw.tc) {
        LAUNCH(launch_moe_tc(dc, ta, s));   // gate_up + down in one kernel
        pc = tc_pending_combine(dc, ta);
      } else {
        // one token: the per-slot phase kernels (measured faster here than the grouped ones)
        LAUNCH(launch_moe_mxfp4(dc, ma, s));
        ++nk;   // gate/up, down
        pc.partial = m->partial; pc.idx = Lw.idx; pc.wts = Lw.wts; pc.K = c.top_k;
        pc.expert_base = m->expert_base; pc.n_local = m->n_local;
      }
    }
    if (Lw.sh_gate) {
      // shared expert (layer.rs:2250-2293): sigmoid(x . gate_inp) * down(silu(gate x) * up x) on the MoE
      // input; the residual kernel adds it to the routed output before the residual add (layer.rs:910-922)
      const int S = Lw.sh_dims[0];
      float* sh_u = m->sh_g + S;   // [gate | up] outputs back to back
      GemvArgs g;
      g.qtype = Lw.sh_gate_q; g.w = Lw.sh_gate; g.rows = S; g.cols = H; g.x = m->xn; g.y = m->sh_g;
      if (Lw.sh_gate == Lw.sh_gu && Lw.sh_up == Lw.sh_gu + (size_t)S * row_bytes(Lw.sh_gate_q, H)) {
        g.rows = 2 * S;   // gate and up rows in one launch
        LAUNCH(launch_gemv(dc, g, s));
      } else {
        LAUNCH(launch_gemv(dc, g, s));
        g.qtype = Lw.sh_up_q; g.w = Lw.sh_up; g.y = sh_u;
        LAUNCH(launch_gemv(dc, g, s));
      }
      LAUNCH(launch_silu_mul(m->sh_g, sh_u, m->sh_a, S, s));
      g.qtype = Lw.sh_down_q; g.w = Lw.sh_down; g.rows = H; g.cols = S; g.x = m->sh_a; g.y = m->sh_o;
      LAUNCH(launch_gemv(dc, g, s));
      LAUNCH(launch_gated_accum(m->xn, Lw.sh_gate_inp, m->sh_o, m->sh_y, H, s, 1));   // sh_y = sigmoid(.) * o
      pc.extra = m->sh_y;
    }
    // h += MoE (ascending expert order); quantize the next layer's attention input (none before a
    // DeltaNet layer, which normalises in f32)
    const float* next_norm = li + 1 < c.layers && !m->L[li + 1].deltanet ? m->L[li + 1].attn_norm : nullptr;
    LAUNCH(launch_resid_norm_q8(dc, pc, m->h, H, next_norm, c.eps, m->xq_h, m->xd_h, m->resid_cnt, s));
    if (m->trace && m->prof_class < 0) {
      cudaError_t e_ = cudaMemcpyAsync(m->trace_h + (size_t)li * H, m->h, (size_t)H * 4, cudaMemcpyDeviceToDevice, s);
      if (e_ != cudaSuccess) return cuda_fail(m->ctx, e_, "trace copy");
    }
  }
  m->head_start = nk;
  LmHeadArgs la;
  la.w = m->out_w; la.x = m->h; la.norm_w = m->out_norm; la.eps = c.eps; la.bias = m->out_b; la.logits = m->logits;
  la.key = &m->st->key; la.V = c.vocab; la.H = H; la.x_out = m->h_last;
  if (m->exact) la.xn_out = m->xn_final;
  LAUNCH(launch_lmhead(dc, la, s));
  if (m->sampling) {   // the step's token drawn from the logits (engine.rs:124-208)
    LAUNCH(launch_sample(dc, sample_args(m), s));
  } else if (m->exact) {   // the greedy token from exact re-scoring of the near-maximal ids
    LAUNCH(launch_exact_argmax_refine(m->out_w, m->xn_final, m->out_b, m->logits, c.vocab, H, 1, &m->st->key, m->ref_scratch, dc, s));
  }
#undef LAUNCH
  m->kernels_per_step = nk;
  return MS_OK;
}

ms_status run_step(ms_model* m) {
  cudaStream_t s = m->ctx->stream;
  if (m->cfg.ep_size > 1 && !m->comm && !m->ep_p2p)
    return fail(m->ctx, MS_ERR_STATE, "expert-parallel model: call ms_model_init_ep or ms_model_ep_connect first");
  // host-tier experts: the step stops at every layer's router for the host to fill the HBM slots,
  // so it is enqueued directly (a captured graph cannot contain the host's decisions)
  if (!m->use_graph || m->tier_slots > 0) return enqueue_step(m, s);
  if (!m->graph) {
    // capture on the context's private stream (the caller's stream may be the legacy default
    // stream, which cannot be captured); the graph is then launched on the caller's stream
    cudaGraph_t g = nullptr;
    cudaStream_t cs = m->ctx->own;
    MS_CUDA(m->ctx, cudaStreamSynchronize(s));
    MS_CUDA(m->ctx, cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal));
    ms_status st = enqueue_step(m, cs);
    cudaError_t e = cudaStreamEndCapture(cs, &g);
    if (st != MS_OK) { if (g) cudaGraphDestroy(g); return st; }
    if (e != cudaSuccess) return cuda_fail(m->ctx, e, "cudaStreamEndCapture");
    e = cudaGraphInstantiate(&m->graph, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) { m->graph = nullptr; return cuda_fail(m->ctx, e, "cudaGraphInstantiate"); }
  }
  MS_CUDA(m->ctx, cudaGraphLaunch(m->graph, s));
  return MS_OK;
}

// ---------------- multi-token forward (engine.rs:1869-2006 over a [1, T] prompt) ----------------
constexpr int kPrefillChunk = 2048;   // tokens per batched pass (bounds the scratch)

template <class T>
ms_status pf_alloc(ms_model* m, T** p, size_t bytes) {
  void* q = nullptr;
  cudaError_t e = cudaMalloc(&q, bytes ? bytes : 16);
  if (e != cudaSuccess) return cuda_fail(m->ctx, e, "cudaMalloc (prefill)");
  e = cudaMemset(q, 0, bytes ? bytes : 16);
  if (e != cudaSuccess) { cudaFree(q); return cuda_fail(m->ctx, e, "cudaMemset (prefill)"); }
  m->pf.allocs.push_back(q);
  *p = reinterpret_cast<T*>(q);
  return MS_OK;
}

ms_status pf_reserve(ms_model* m, int T) {
  auto& P = m->pf;
  if (P.cap >= T) return MS_OK;
  MS_CUDA(m->ctx, cudaStreamSynchronize(m->ctx->stream));
  for (void* q : P.allocs) cudaFree(q);
  P = ms_model::Prefill();
  const ms_model_config& c = m->cfg;
  const int H = c.hidden, Dq = q_dim(c), Dkv = kv_dim(c), K = c.top_k, E = c.experts;
  const int Wq = std::max(H, Dq);
  bool any_tc = false, any_native = false;
  for (auto& Lw : m->L) { any_tc = any_tc || Lw.tc; any_native = any_native || !Lw.tc; }
  ms_status s = MS_OK;
  s = s ? s : pf_alloc(m, &P.tok, (size_t)T * 4);
  s = s ? s : pf_alloc(m, &P.h, (size_t)T * H * 4);
  s = s ? s : pf_alloc(m, &P.xq, (size_t)T * Wq + 64);
  s = s ? s : pf_alloc(m, &P.xd, (size_t)T * Wq / 32 * 4 + 64);
  s = s ? s : pf_alloc(m, &P.qkv, (size_t)T * (Dq + 2 * Dkv) * 4);
  s = s ? s : pf_alloc(m, &P.q, (size_t)T * Dq * 4);
  s = s ? s : pf_alloc(m, &P.kn, (size_t)T * Dkv * 4);
  s = s ? s : pf_alloc(m, &P.vn, (size_t)T * Dkv * 4);
  s = s ? s : pf_alloc(m, &P.attn, (size_t)T * Dq * 4);
  s = s ? s : pf_alloc(m, &P.xn, (size_t)T * H * 4);
  s = s ? s : pf_alloc(m, &P.rlog, (size_t)T * E * 4);
  s = s ? s : pf_alloc(m, &P.idx, (size_t)T * K * 4);
  s = s ? s : pf_alloc(m, &P.wts, (size_t)T * K * 4);
  s = s ? s : pf_alloc(m, &P.rcnt, (size_t)(T + 16) * 4);
  if (c.ep_size > 1) s = s ? s : pf_alloc(m, &P.moe_y, (size_t)T * H * 4);
  if (any_tc) s = s ? s : pf_alloc(m, &P.moe_scratch, pf_scratch_bytes(H, c.inter, m->n_local, T, K, 1));
  if (any_native) {
    s = s ? s : pf_alloc(m, &P.grp, (size_t)group_table_words(kMaxBatch, K) * 4);
    s = s ? s : pf_alloc(m, &P.ent_slot, (size_t)kMaxBatch * K * 4);
    s = s ? s : pf_alloc(m, &P.ent_of, (size_t)kMaxBatch * K * 4);
    s = s ? s : pf_alloc(m, &P.gact, (size_t)kMaxBatch * K * c.inter * 4);
    s = s ? s : pf_alloc(m, &P.gy, (size_t)kMaxBatch * K * H * 4);
  }
  if (s != MS_OK) {
    for (void* q : P.allocs) cudaFree(q);
    P = ms_model::Prefill();
    return s;
  }
  P.cap = T;
  return MS_OK;
}

// whether the batched prefill covers this model (else the prompt runs one decode step per token)
bool pf_supported(const ms_model* m) {
  const ms_model_config& c = m->cfg;
  if (m->prefill_mode == 0) return false;
  if (c.ep_size > 1 && !m->comm) return false;   // the peer-mailbox exchange is sized for one token
  // DeltaNet layers run token by token (layer.rs:435-452) and shared experts have no batched path:
  // such models take one decode step per prompt token
  if (is_hybrid(c) || m->sh_max > 0) return false;
  if (m->tier_slots > 0) return false;   // host-tier experts: the expert kernels read HBM slots
  if (m->dyn_k || m->router_stats) return false;   // the batched router has no entropy / dynamic K
  if (c.hidden % 32 || (c.heads * c.head_dim) % 32 || c.head_dim % 32 || c.head_dim > 256) return false;
  return true;
}

// one batched pass over T <= kPrefillChunk tokens at positions [seq, seq + T)
ms_status pf_chunk(ms_model* m, const int32_t* tokens, int T, bool last_chunk) {
  const ms_model_config& c = m->cfg;
  const DevCtx& dc = m->ctx->dc;
  cudaStream_t s = m->ctx->stream;
  auto& P = m->pf;
  const int H = c.hidden, Dq = q_dim(c), Dkv = kv_dim(c), K = c.top_k, E = c.experts, pos0 = m->seq;
  for (int i = 0; i < T; ++i) m->h_tok[i] = tokens[i];
  MS_CUDA(m->ctx, cudaMemcpyAsync(P.tok, m->h_tok, (size_t)T * 4, cudaMemcpyHostToDevice, s));
#define PCALL(call)                                                    \
  do {                                                                 \
    cudaError_t e_ = (call);                                           \
    if (e_ != cudaSuccess) return cuda_fail(m->ctx, e_, #call);       \
  } while (0)
  PCALL(launch_pf_embed(dc, P.tok, T, m->embd, m->embd_q, H, c.vocab, P.h, m->L[0].attn_norm, c.eps, P.xq, P.xd, s));
  for (int li = 0; li < c.layers; ++li) {
    LayerW& Lw = m->L[li];
    // Q/K/V of all tokens (Q8_0 weights x Q8_0 activations, 32 tokens per pass)
    for (int c0 = 0; c0 < T; c0 += kMaxBatch) {
      Q8BatchArgs qa;
      qa.w = Lw.wqkv; qa.rows = Dq + 2 * Dkv; qa.cols = H; qa.B = std::min(kMaxBatch, T - c0);
      qa.xq = P.xq + (size_t)c0 * H; qa.xd = P.xd + (size_t)c0 * (H / 32); qa.bias = Lw.bqkv;
      qa.y = P.qkv + (size_t)c0 * (Dq + 2 * Dkv);
      PCALL(launch_q8_gemm_batch(dc, qa, s));
    }
    PfAttnLaunch al;
    al.qkv = P.qkv; al.q_norm = Lw.qn; al.k_norm = Lw.kn; al.eps = c.eps; al.cos_t = m->cos_t; al.sin_t = m->sin_t;
    al.rot = c.rot_dim; al.pos0 = pos0; al.T = T; al.nh = c.heads; al.nkv = c.kv_heads; al.hd = c.head_dim;
    al.kc = Lw.kc; al.vc = Lw.vc; al.cap = Lw.cap; al.window = Lw.window; al.sinks = Lw.sinks;
    al.scale = (float)(1.0 / std::sqrt((double)c.head_dim)); al.q = P.q; al.kn = P.kn; al.vn = P.vn; al.out = P.attn;
    PCALL(launch_pf_attention(dc, al, s));
    // O projection into the residual stream
    PCALL(launch_pf_quant(P.attn, (int64_t)T * Dq, P.xq, P.xd, s));
    for (int c0 = 0; c0 < T; c0 += kMaxBatch) {
      Q8BatchArgs oa;
      oa.w = Lw.wo; oa.rows = H; oa.cols = Dq; oa.B = std::min(kMaxBatch, T - c0);
      oa.xq = P.xq + (size_t)c0 * Dq; oa.xd = P.xd + (size_t)c0 * (Dq / 32); oa.bias = Lw.bo;
      oa.residual = P.h + (size_t)c0 * H;
      PCALL(launch_q8_gemm_batch(dc, oa, s));
    }
    // router of every token (RMSNorm, logits, dummy mask, top-k)
    RouterArgs ra;
    ra.h = P.h; ra.norm_w = Lw.post_norm; ra.eps = c.eps; ra.xn = P.xn; ra.w = Lw.router_w; ra.b = Lw.router_b;
    ra.mask = Lw.mask; ra.logits = P.rlog; ra.idx = P.idx; ra.wts = P.wts; ra.counter = P.rcnt; ra.H = H; ra.E = E;
    ra.K = K; ra.softmax_weight = c.arch == MS_ARCH_GPT_OSS; ra.normalize = c.norm_topk_prob; ra.batch = T;
    PCALL(launch_router(dc, ra, s));
    // experts: h += MoE(xn) (local experts; summed over the expert-parallel group by NCCL)
    float* moe_dst = c.ep_size > 1 ? P.moe_y : P.h;
    if (Lw.tc) {
      PrefillArgs pa;
      pa.gu = Lw.gu_tc; pa.down = Lw.down_tc; pa.gate_b = Lw.gate_b; pa.up_b = Lw.up_b; pa.down_b = Lw.down_b;
      pa.x = P.xn; pa.idx = P.idx; pa.wts = P.wts; pa.out = moe_dst; pa.scratch = P.moe_scratch; pa.H = H;
      pa.I = c.inter; pa.E = m->n_local; pa.K = K; pa.T = T; pa.expert_base = m->expert_base;
      pa.oai_swiglu = c.arch == MS_ARCH_GPT_OSS; pa.accumulate = c.ep_size > 1 ? 0 : 1;
      pa.precise = m->prefill_mode == 1;
      PCALL(launch_moe_prefill(dc, pa, s));
    } else {
      if (c.ep_size > 1) MS_CUDA(m->ctx, cudaMemsetAsync(P.moe_y, 0, (size_t)T * H * 4, s));
      for (int c0 = 0; c0 < T; c0 += kMaxBatch) {
        const int B = std::min(kMaxBatch, T - c0);
        GroupMoeArgs ga;
        ga.x = P.xn + (size_t)c0 * H; ga.idx = P.idx + (size_t)c0 * K; ga.B = B; ga.K = K; ga.H = H; ga.I = c.inter;
        ga.gate_q = Lw.gate_q; ga.down_q = Lw.down_q; ga.gate = Lw.gate; ga.up = Lw.up; ga.down = Lw.down;
        ga.gate_b = Lw.gate_b; ga.up_b = Lw.up_b; ga.down_b = Lw.down_b; ga.expert_base = m->expert_base;
        ga.n_local = m->n_local; ga.oai_swiglu = c.arch == MS_ARCH_GPT_OSS; ga.grp = P.grp; ga.ent_slot = P.ent_slot;
        ga.ent_of = P.ent_of; ga.act = P.gact; ga.y = P.gy;
        for (int part = 0; part < 3; ++part) PCALL(launch_moe_group(dc, ga, part, s));
        BatchCombine bc;
        bc.y = P.gy; bc.ent_of = P.ent_of; bc.idx = P.idx + (size_t)c0 * K; bc.wts = P.wts + (size_t)c0 * K; bc.K = K;
        PCALL(launch_resid_batch(dc, bc, moe_dst + (size_t)c0 * H, H, B, nullptr, c.eps, nullptr, nullptr, nullptr, s));
      }
    }
    if (c.ep_size > 1) {
      NcclApi* api = nccl_api();
      ncclResult_t r = api->all_reduce(P.moe_y, P.moe_y, (size_t)T * H, ncclFloat32, ncclSum, m->comm, s);
      if (r != ncclSuccess) return fail(m->ctx, MS_ERR_NCCL, "ncclAllReduce (prefill): %s", api->error_string(r));
      PCALL(launch_pf_add(P.h, P.moe_y, (int64_t)T * H, s));
    }
    if (m->trace) {   // the last token's residual stream and router logits after this layer
      MS_CUDA(m->ctx, cudaMemcpyAsync(m->trace_h + (size_t)li * H, P.h + (size_t)(T - 1) * H, (size_t)H * 4,
                                      cudaMemcpyDeviceToDevice, s));
      MS_CUDA(m->ctx, cudaMemcpyAsync(m->trace_logits + (size_t)li * E, P.rlog + (size_t)(T - 1) * E, (size_t)E * 4,
                                      cudaMemcpyDeviceToDevice, s));
    }
    if (last_chunk) {   // routing of the last position (ms_model_last_routing)
      MS_CUDA(m->ctx, cudaMemcpyAsync(Lw.idx, P.idx + (size_t)(T - 1) * K, (size_t)K * 4, cudaMemcpyDeviceToDevice, s));
      MS_CUDA(m->ctx, cudaMemcpyAsync(Lw.wts, P.wts + (size_t)(T - 1) * K, (size_t)K * 4, cudaMemcpyDeviceToDevice, s));
    }
    if (li + 1 < c.layers) PCALL(launch_pf_norm_q8(P.h, T, H, m->L[li + 1].attn_norm, c.eps, P.xq, P.xd, s));
  }
  if (last_chunk) {   // final norm + LM head of the last position (engine.rs:1963-1987, 2033)
    MS_CUDA(m->ctx, cudaMemsetAsync(&m->st->key, 0, sizeof(unsigned long long), s));
    LmHeadArgs la;
    la.w = m->out_w; la.x = P.h + (size_t)(T - 1) * H; la.norm_w = m->out_norm; la.eps = c.eps; la.bias = m->out_b;
    la.logits = m->logits; la.key = &m->st->key; la.V = c.vocab; la.H = H; la.x_out = m->h_last;
    if (m->exact) la.xn_out = m->xn_final;
    PCALL(launch_lmhead(dc, la, s));
    if (m->sampling)
      PCALL(launch_sample(dc, sample_args(m), s));
    else if (m->exact)
      PCALL(launch_exact_argmax_refine(m->out_w, m->xn_final, m->out_b, m->logits, c.vocab, H, 1, &m->st->key, m->ref_scratch, dc, s));
  }
#undef PCALL
  // the token log and the step state continue after the prompt
  MS_CUDA(m->ctx, cudaStreamSynchronize(s));
  StepState st;
  MS_CUDA(m->ctx, cudaMemcpy(&st, m->st, sizeof st, cudaMemcpyDeviceToHost));
  const int room = std::max(0, std::min(T, c.max_seq_len - st.n_log));
  if (room > 0) MS_CUDA(m->ctx, cudaMemcpy(m->token_log + st.n_log, tokens, (size_t)room * 4, cudaMemcpyHostToDevice));
  st.n_log += T;
  st.n_ctx = pos0 + T;
  st.pos = pos0 + T - 1;
  st.last_token = tokens[T - 1];
  MS_CUDA(m->ctx, cudaMemcpy(m->st, &st, sizeof st, cudaMemcpyHostToDevice));
  m->seq += T;
  return MS_OK;
}

ms_status pf_forward(ms_model* m, const int32_t* tokens, int n) {
  const int chunk = std::min(n, kPrefillChunk);
  ms_status st = pf_reserve(m, chunk);
  if (st != MS_OK) return st;
  for (int i = 0; i < n; i += kPrefillChunk) {
    const int t = std::min(kPrefillChunk, n - i);
    st = pf_chunk(m, tokens + i, t, i + t == n);
    if (st != MS_OK) return st;
  }
  return MS_OK;
}

// whether the next steps draw a token (sampled decoding): the same pinned 0 / 1 constants
ms_status set_draw(ms_model* m, int draw) {
  if (!m->s_draw) return MS_OK;
  const int* src = &m->h_tok[m->cfg.max_seq_len + 2 + (draw ? 1 : 0)];
  MS_CUDA(m->ctx, cudaMemcpyAsync(m->s_draw, src, sizeof(int), cudaMemcpyHostToDevice, m->ctx->stream));
  return MS_OK;
}

ms_status set_feed(ms_model* m, int use_argmax) {
  // StepState.use_argmax lives at a fixed offset; one small async copy from pinned memory
  // constants 0 / 1 live in the pinned staging tail, so pending copies never see a rewrite
  const int* src = &m->h_tok[m->cfg.max_seq_len + 2 + (use_argmax ? 1 : 0)];
  MS_CUDA(m->ctx, cudaMemcpyAsync(&m->st->use_argmax, src, sizeof(int), cudaMemcpyHostToDevice, m->ctx->stream));
  return MS_OK;
}

// ---------------- GGUF (reader.rs:259-368) ----------------
struct GgufMeta { int type = 0; int64_t i = 0; double f = 0; std::string s; };
struct GgufT { int q; std::vector<int64_t> shape; uint64_t off; int64_t nbytes; };

struct GgufParser {
  const uint8_t* b; size_t n, pos = 0; bool ok = true;
  bool need(size_t k) { if (pos + k > n) { ok = false; return false; } return true; }
  template <class T> T rd() { T v{}; if (need(sizeof(T))) { memcpy(&v, b + pos, sizeof(T)); pos += sizeof(T); } return v; }
  std::string str() { uint64_t k = rd<uint64_t>(); if (!need(k)) return {}; std::string s((const char*)b + pos, k); pos += k; return s; }
  void val(int t, GgufMeta* v, int depth = 0) {
    v->type = t;
    switch (t) {
      case 0: v->i = rd<uint8_t>(); break;
      case 1: v->i = rd<int8_t>(); break;
      case 2: v->i = rd<uint16_t>(); break;
      case 3: v->i = rd<int16_t>(); break;
      case 4: v->i = rd<uint32_t>(); break;
      case 5: v->i = rd<int32_t>(); break;
      case 6: v->f = rd<float>(); v->i = (int64_t)v->f; break;
      case 7: v->i = rd<uint8_t>(); break;
      case 8: v->s = str(); break;
      case 9: {
        int et = (int)rd<uint32_t>(); uint64_t k = rd<uint64_t>();
        if (depth > 4 || k > (1ull << 28)) { ok = false; return; }
        GgufMeta tmp;
        for (uint64_t j = 0; j < k && ok; ++j) val(et, &tmp, depth + 1);
        break;
      }
      case 10: v->i = (int64_t)rd<uint64_t>(); break;
      case 11: v->i = rd<int64_t>(); break;
      case 12: v->f = rd<double>(); v->i = (int64_t)v->f; break;
      default: ok = false;
    }
  }
};

}  // namespace

// lockstep batch helpers (the entry points are below)
namespace {

void batch_free(ms_model* m) {
  BatchRt* b = m->bt;
  if (!b) return;
  if (b->graph) cudaGraphExecDestroy(b->graph);
  for (void* p : b->allocs) cudaFree(p);
  if (b->h_st) cudaFreeHost(b->h_st);
  if (b->h_tok) cudaFreeHost(b->h_tok);
  if (b->h_keys) cudaFreeHost(b->h_keys);
  delete b;
  m->bt = nullptr;
}

template <class T>
ms_status balloc(ms_model* m, T** p, size_t bytes) {
  void* q = nullptr;
  cudaError_t e = cudaMalloc(&q, bytes ? bytes : 16);
  if (e != cudaSuccess) return cuda_fail(m->ctx, e, "cudaMalloc (batch)");
  e = cudaMemset(q, 0, bytes ? bytes : 16);
  if (e != cudaSuccess) { cudaFree(q); return cuda_fail(m->ctx, e, "cudaMemset (batch)"); }
  m->bt->allocs.push_back(q);
  *p = reinterpret_cast<T*>(q);
  return MS_OK;
}

// launch classes of the batch step (ms_model_batch_profile_step): 0 step start (begin, embed),
// 1 QKV, 2 attention, 3 O, 4 router, 5 expert grouping, 6 gate_up, 7 down, 8 residual, 9 LM head
constexpr int kBatchClasses = 10;

ms_status enqueue_batch_step(ms_model* m, cudaStream_t s) {
  const ms_model_config& c = m->cfg;
  const DevCtx& dc = m->ctx->dc;
  BatchRt& b = *m->bt;
  const int H = c.hidden, Dq = q_dim(c), Dkv = kv_dim(c), B = b.B;
  int nk = 0;
#define BLAUNCH(cls, n, call)                                          \
  do {                                                                 \
    if (m->prof_class < 0 || m->prof_class == (cls)) {                 \
      cudaError_t e_ = (call);                                         \
      if (e_ != cudaSuccess) return cuda_fail(m->ctx, e_, #call);      \
    }                                                                  \
    nk += (n);                                                         \
  } while (0)
  BLAUNCH(0, 1, launch_batch_begin(dc, b.st, s));
  BLAUNCH(0, 1, launch_embed_batch(dc, b.st, b.tok_in, b.keys, m->embd, m->embd_q, H, c.vocab, B, b.h, b.log,
                                   m->L[0].attn_norm, c.eps, b.xq_h, b.xd_h, s));
  for (int li = 0; li < c.layers; ++li) {
    LayerW& Lw = m->L[li];
    Q8BatchArgs qa;
    qa.w = Lw.wqkv; qa.rows = Dq + 2 * Dkv; qa.cols = H; qa.B = B; qa.xq = b.xq_h; qa.xd = b.xd_h; qa.bias = Lw.bqkv;
    qa.y = b.qkv;
    BLAUNCH(1, 1, launch_q8_gemm_batch(dc, qa, s));
    AttnArgs aa;
    aa.qkv = b.qkv; aa.q_norm = Lw.qn; aa.k_norm = Lw.kn; aa.eps = c.eps; aa.cos_t = m->cos_t; aa.sin_t = m->sin_t;
    aa.rot = c.rot_dim; aa.pos = &b.st->pos; aa.kc = b.kc[li]; aa.vc = b.vc[li]; aa.cap = Lw.cap; aa.window = Lw.window;
    aa.sinks = Lw.sinks; aa.part = b.part; aa.cnt = b.attn_cnt; aa.out = b.attn; aa.nh = c.heads; aa.nkv = c.kv_heads;
    aa.hd = c.head_dim; aa.S = Lw.window ? b.S_swa : b.S_full; aa.spl = Lw.window ? b.spl_swa : b.spl_full;
    aa.scale = (float)(1.0 / std::sqrt((double)c.head_dim)); aa.oq = b.xq_a; aa.od = b.xd_a;
    aa.batch = B; aa.bs_qkv = Dq + 2 * Dkv; aa.bs_kv = (int64_t)c.kv_heads * Lw.cap * c.head_dim; aa.bs_out = Dq;
    if (exact_attn_ok(m)) BLAUNCH(2, 1, launch_exact_attention(dc, aa, Lw.window ? Lw.cap : c.max_seq_len, s));
    else BLAUNCH(2, 1, launch_attention(dc, aa, s));
    Q8BatchArgs oa;
    oa.w = Lw.wo; oa.rows = H; oa.cols = Dq; oa.B = B; oa.xq = b.xq_a; oa.xd = b.xd_a; oa.bias = Lw.bo;
    oa.residual = b.h;
    BLAUNCH(3, 1, launch_q8_gemm_batch(dc, oa, s));
    RouterArgs ra;
    ra.h = b.h; ra.norm_w = Lw.post_norm; ra.eps = c.eps; ra.xn = b.xn; ra.w = Lw.router_w; ra.b = Lw.router_b;
    ra.mask = Lw.mask; ra.logits = b.rlog; ra.idx = b.idx; ra.wts = b.wts; ra.counter = b.router_cnt; ra.H = H;
    ra.E = c.experts; ra.K = c.top_k; ra.softmax_weight = c.arch == MS_ARCH_GPT_OSS; ra.normalize = c.norm_topk_prob;
    ra.batch = B;
    BLAUNCH(4, 1, launch_router(dc, ra, s));
    GroupMoeArgs ga;
    ga.x = b.xn; ga.idx = b.idx; ga.B = B; ga.K = c.top_k; ga.H = H; ga.I = c.inter; ga.gate_q = Lw.gate_q;
    ga.down_q = Lw.down_q; ga.gate = Lw.gate; ga.up = Lw.up; ga.down = Lw.down; ga.gate_b = Lw.gate_b;
    ga.up_b = Lw.up_b; ga.down_b = Lw.down_b; ga.expert_base = m->expert_base; ga.n_local = m->n_local;
    ga.oai_swiglu = c.arch == MS_ARCH_GPT_OSS; ga.grp = b.grp; ga.ent_slot = b.ent_slot; ga.ent_of = b.ent_of;
    ga.act = b.act; ga.y = b.y;
    BatchCombine bc;
    bc.y = b.y; bc.ent_of = b.ent_of; bc.idx = b.idx; bc.wts = b.wts; bc.K = c.top_k;
    if (m->exact && exact_kq_supported(Lw.gate_q, Lw.down_q, H, c.inter) && Lw.up_q == Lw.gate_q) {
      // order-independent experts per (token, slot): y [B][K][H] with the bias, every entry local
      ExactKqArgs ka;
      ka.gate = Lw.gate; ka.up = Lw.up; ka.down = Lw.down; ka.gate_fmt = Lw.gate_q; ka.down_fmt = Lw.down_q;
      ka.gate_b = Lw.gate_b; ka.up_b = Lw.up_b; ka.down_b = Lw.down_b; ka.x = b.xn; ka.idx = b.idx; ka.H = H;
      ka.I = c.inter; ka.K = c.top_k; ka.expert_base = m->expert_base; ka.n_local = m->n_local;
      ka.oai_swiglu = c.arch == MS_ARCH_GPT_OSS; ka.B = B; ka.gu_out = b.act; ka.y = b.y;
      BLAUNCH(6, 2, launch_exact_kq_moe(dc, ka, s));
      bc.ent_of = b.ent_zero;
    } else {
      BLAUNCH(5, 1, launch_moe_group(dc, ga, 0, s));
      BLAUNCH(6, 1, launch_moe_group(dc, ga, 1, s));
      BLAUNCH(7, 1, launch_moe_group(dc, ga, 2, s));
    }
    const bool last = li + 1 == c.layers;
    BLAUNCH(8, 1, launch_resid_batch(dc, bc, b.h, H, B, last ? m->out_norm : m->L[li + 1].attn_norm, c.eps,
                                     last ? nullptr : b.xq_h, last ? nullptr : b.xd_h, last ? b.xf : nullptr, s));
  }
  LmBatchArgs la;
  la.w = m->out_w; la.xf = b.xf; la.V = c.vocab; la.H = H; la.B = B; la.bias = m->out_b; la.scratch = b.lm_scratch;
  la.logits = b.logits; la.keys = b.keys;
  BLAUNCH(9, 3, launch_lmhead_batch(dc, la, s));   // prep, GEMM, key reduction
  if (m->exact)   // exact re-scoring of the near-maximal ids (the greedy token, bit for bit)
    BLAUNCH(9, 1, launch_exact_argmax_refine(m->out_w, b.xf, m->out_b, b.logits, c.vocab, H, B, b.keys, b.ref_scratch, dc, s));
#undef BLAUNCH
  b.kernels_per_step = nk;
  return MS_OK;
}

ms_status run_batch_step(ms_model* m) {
  BatchRt& b = *m->bt;
  cudaStream_t s = m->ctx->stream;
  if (!m->use_graph) return enqueue_batch_step(m, s);
  if (!b.graph) {
    cudaGraph_t g = nullptr;
    cudaStream_t cs = m->ctx->own;
    MS_CUDA(m->ctx, cudaStreamSynchronize(s));
    MS_CUDA(m->ctx, cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal));
    ms_status st = enqueue_batch_step(m, cs);
    cudaError_t e = cudaStreamEndCapture(cs, &g);
    if (st != MS_OK) { if (g) cudaGraphDestroy(g); return st; }
    if (e != cudaSuccess) return cuda_fail(m->ctx, e, "cudaStreamEndCapture");
    e = cudaGraphInstantiate(&b.graph, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) { b.graph = nullptr; return cuda_fail(m->ctx, e, "cudaGraphInstantiate"); }
  }
  MS_CUDA(m->ctx, cudaGraphLaunch(b.graph, s));
  return MS_OK;
}

ms_status batch_feed(ms_model* m, int use_argmax) {
  BatchRt& b = *m->bt;
  const int* src = &b.h_tok[(size_t)m->cfg.max_seq_len * b.B + (use_argmax ? 1 : 0)];
  MS_CUDA(m->ctx, cudaMemcpyAsync(&b.st->use_argmax, src, sizeof(int), cudaMemcpyHostToDevice, m->ctx->stream));
  return MS_OK;
}

ms_status batch_ready(ms_model* m, int n_steps) {
  if (!m) return MS_ERR_INVALID_ARG;
  if (!m->bt) return fail(m->ctx, MS_ERR_STATE, "no batch open (ms_model_batch_open)");
  if (m->bt->seq + n_steps > m->cfg.max_seq_len) return fail(m->ctx, MS_ERR_SHAPE, "batch sequence exceeds max_seq_len");
  cudaSetDevice(m->ctx->device);
  return MS_OK;
}

}  // namespace

extern "C" {

int ms_abi_version(void) { return MS_ABI_VERSION; }

const char* ms_status_string(ms_status s) {
  switch (s) {
    case MS_OK: return "ok";
    case MS_ERR_INVALID_ARG: return "invalid argument";
    case MS_ERR_OOM: return "out of device memory";
    case MS_ERR_CUDA: return "CUDA error";
    case MS_ERR_NCCL: return "NCCL error";
    case MS_ERR_TIMEOUT: return "device wait timed out";
    case MS_ERR_UNSUPPORTED_QTYPE: return "unsupported tensor type";
    case MS_ERR_SHAPE: return "shape mismatch";
    case MS_ERR_IO: return "I/O error";
    case MS_ERR_FORMAT: return "malformed GGUF";
    case MS_ERR_STATE: return "call out of order";
    case MS_ERR_DEVICE_INDEX: return "out-of-range index seen on the device";
  }
  return "unknown status";
}

ms_status ms_ctx_create(int device, ms_ctx** out) {
  if (!out) return MS_ERR_INVALID_ARG;
  *out = nullptr;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) return MS_ERR_INVALID_ARG;
  auto* c = new ms_ctx();
  c->device = device;
  cudaError_t e = cudaSetDevice(device);
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&c->own, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&c->dc.sm_count, cudaDevAttrMultiProcessorCount, device);
  if (e == cudaSuccess) e = cudaMalloc(&c->dc.err, 16);
  if (e == cudaSuccess) e = cudaMemset(c->dc.err, 0, 16);
  if (e != cudaSuccess) { delete c; return MS_ERR_CUDA; }
  c->stream = c->own;
  *out = c;
  return MS_OK;
}

ms_status ms_ctx_destroy(ms_ctx* c) {
  if (!c) return MS_ERR_INVALID_ARG;
  cudaSetDevice(c->device);
  cudaStreamSynchronize(c->stream);
  while (!c->models.empty()) ms_model_destroy(c->models.back());
  if (c->scratch) cudaFree(c->scratch);
  if (c->counters) cudaFree(c->counters);
  if (c->dc.err) cudaFree(c->dc.err);
  if (c->own) cudaStreamDestroy(c->own);
  delete c;
  return MS_OK;
}

ms_status ms_ctx_set_stream(ms_ctx* c, void* stream) {
  if (!c) return MS_ERR_INVALID_ARG;
  c->stream = stream ? (cudaStream_t)stream : cudaStreamLegacy;   // NULL: the legacy default stream
  return MS_OK;
}

ms_status ms_ctx_use_own_stream(ms_ctx* c) {
  if (!c) return MS_ERR_INVALID_ARG;
  c->stream = c->own;
  return MS_OK;
}

ms_status ms_sync(ms_ctx* c) {
  if (!c) return MS_ERR_INVALID_ARG;
  MS_CUDA(c, cudaStreamSynchronize(c->stream));
  return check_dev_flags(c);
}

const char* ms_last_error(const ms_ctx* c) { return c ? c->err.c_str() : "null context"; }

ms_status ms_ctx_error_flags(ms_ctx* c, uint32_t* flags, int clear) {
  if (!c || !flags) return MS_ERR_INVALID_ARG;
  MS_CUDA(c, cudaMemcpy(flags, c->dc.err, 4, cudaMemcpyDeviceToHost));
  if (clear && *flags) MS_CUDA(c, cudaMemset(c->dc.err, 0, 4));
  return MS_OK;
}

int ms_ctx_sm_count(const ms_ctx* c) { return c ? c->dc.sm_count : 0; }

ms_status ms_malloc(ms_ctx* c, size_t bytes, void** p) {
  if (!c || !p) return MS_ERR_INVALID_ARG;
  MS_CUDA(c, cudaMalloc(p, bytes ? bytes : 16));
  return MS_OK;
}
ms_status ms_free(ms_ctx* c, void* p) {
  if (!c) return MS_ERR_INVALID_ARG;
  MS_CUDA(c, cudaFree(p));
  return MS_OK;
}
ms_status ms_memcpy_h2d(ms_ctx* c, void* d, const void* s, size_t n) {
  if (!c) return MS_ERR_INVALID_ARG;
  MS_CUDA(c, cudaMemcpyAsync(d, s, n, cudaMemcpyHostToDevice, c->stream));
  MS_CUDA(c, cudaStreamSynchronize(c->stream));
  return MS_OK;
}
ms_status ms_memcpy_d2h(ms_ctx* c, void* d, const void* s, size_t n) {
  if (!c) return MS_ERR_INVALID_ARG;
  MS_CUDA(c, cudaMemcpyAsync(d, s, n, cudaMemcpyDeviceToHost, c->stream));
  MS_CUDA(c, cudaStreamSynchronize(c->stream));
  return MS_OK;
}

ms_status ms_dequantize(ms_ctx* c, int q, const void* d_blocks, int64_t n, float* d_out) {
  if (!c || !d_blocks || !d_out || n < 0) return MS_ERR_INVALID_ARG;
  if (raw_bytes(q, 1) < 0) return fail(c, MS_ERR_UNSUPPORTED_QTYPE, "qtype %d", q);
  MS_CUDA(c, launch_dequantize(c->dc, q, d_blocks, n, d_out, c->stream));
  return MS_OK;
}

ms_status ms_rms_norm(ms_ctx* c, const float* x, const float* w, float* y, int rows, int dim, float eps) {
  if (!c || !x || !w || !y || rows <= 0 || dim <= 0) return MS_ERR_INVALID_ARG;
  MS_CUDA(c, launch_rms_norm(c->dc, x, w, y, rows, dim, eps, c->stream));
  return MS_OK;
}

ms_status ms_gemv(ms_ctx* c, int q, const void* w, int rows, int cols, const float* x, const float* bias, float* y) {
  if (!c || !w || !x || !y || rows <= 0 || cols <= 0) return MS_ERR_INVALID_ARG;
  if (q != Q_MXFP4 && q != Q_Q8_0 && q != Q_F16 && q != Q_F32 && q != Q_Q4_K && q != Q_Q6_K)
    return fail(c, MS_ERR_UNSUPPORTED_QTYPE, "gemv qtype %d", q);
  if (row_bytes(q, cols) < 0) return fail(c, MS_ERR_SHAPE, "cols %d not a whole number of blocks", cols);
  GemvArgs a;
  a.qtype = q; a.w = w; a.rows = rows; a.cols = cols; a.x = x; a.bias = bias; a.y = y;
  cudaError_t e = launch_gemv(c->dc, a, c->stream);
  if (e == cudaErrorInvalidValue) return fail(c, MS_ERR_SHAPE, "gemv: unsupported shape %dx%d", rows, cols);
  if (e != cudaSuccess) return cuda_fail(c, e, "gemv");
  return MS_OK;
}

ms_status ms_router_topk(ms_ctx* c, const float* h, const float* nw, float eps, const float* rw, const float* rb,
                         const uint8_t* mask, int H, int E, int K, int arch, int norm_topk, float* xn, float* logits,
                         int32_t* idx, float* wts) {
  if (!c || !rw || !xn || !logits || !idx || !wts || (h && !nw) || H <= 0 || E <= 0 || K <= 0 || K > E || K > 16)
    return MS_ERR_INVALID_ARG;
  ms_status s = ensure_scratch(c, 16, 64);
  if (s != MS_OK) return s;
  RouterArgs a;
  a.h = h; a.norm_w = nw; a.eps = eps; a.xn = xn; a.w = rw; a.b = rb; a.mask = mask; a.logits = logits; a.idx = idx;
  a.wts = wts; a.counter = c->counters; a.H = H; a.E = E; a.K = K; a.softmax_weight = arch == MS_ARCH_GPT_OSS;
  a.normalize = norm_topk;
  MS_CUDA(c, launch_router(c->dc, a, c->stream));
  return MS_OK;
}

ms_status ms_moe_mxfp4_decode(ms_ctx* c, const void* gate, const void* up, const void* down, const float* gb,
                              const float* ub, const float* db, int H, int I, int E, int K, int arch, const float* x,
                              const int32_t* idx, const float* wts, float* h) {
  if (!c || !gate || !up || !down || !x || !idx || !wts || !h || K <= 0 || K > 16 || E <= 0) return MS_ERR_INVALID_ARG;
  if (H % 64 || I % 32) return fail(c, MS_ERR_SHAPE, "moe: hidden %% 64 and inter %% 32 required");
  const size_t act_b = (size_t)K * I * 4, part_b = (size_t)K * H * 4;
  ms_status s = ensure_scratch(c, act_b + part_b + 256, 64 + H / 16);
  if (s != MS_OK) return s;
  MoeArgs a;
  a.x = x; a.idx = idx; a.wts = wts; a.gate = (const uint8_t*)gate; a.up = (const uint8_t*)up;
  a.down = (const uint8_t*)down; a.gate_b = gb; a.up_b = ub; a.down_b = db;
  a.act = (float*)c->scratch; a.partial = (float*)((char*)c->scratch + ((act_b + 255) & ~(size_t)255));
  a.tile_cnt = c->counters + 64; a.h = h; a.H = H; a.I = I; a.K = K; a.expert_base = 0; a.n_local = E;
  a.oai_swiglu = arch == MS_ARCH_GPT_OSS;
  cudaError_t e = launch_moe_mxfp4(c->dc, a, c->stream);
  if (e != cudaSuccess) return cuda_fail(c, e, "moe_mxfp4");
  return MS_OK;
}

ms_status ms_mxfp4_packed_bytes(int H, int I, int E, size_t* gu_bytes, size_t* down_bytes) {
  if (!gu_bytes || !down_bytes || E <= 0 || H <= 0 || I <= 0) return MS_ERR_INVALID_ARG;
  if (!tc_supported(H, I)) return MS_ERR_SHAPE;
  *gu_bytes = (size_t)E * tc_gu_tiles(I) * tc_tile_bytes(H / 32);
  *down_bytes = (size_t)E * tc_down_tiles(H) * tc_tile_bytes(I / 32);
  return MS_OK;
}

ms_status ms_mxfp4_pack_experts(ms_ctx* c, const void* gate, const void* up, const void* down, int H, int I, int E,
                                void* gu_packed, void* down_packed) {
  if (!c || !gate || !up || !down || !gu_packed || !down_packed || E <= 0) return MS_ERR_INVALID_ARG;
  size_t gb = 0, db = 0;
  if (ms_mxfp4_packed_bytes(H, I, E, &gb, &db) != MS_OK) return fail(c, MS_ERR_SHAPE, "pack: hidden and inter must be multiples of 64");
  cudaSetDevice(c->device);
  MS_CUDA(c, cudaMemsetAsync(gu_packed, 0, gb, c->stream));
  MS_CUDA(c, cudaMemsetAsync(down_packed, 0, db, c->stream));
  MS_CUDA(c, launch_mxfp4_pack((const uint8_t*)gate, E, I, H, 64, 0, tc_gu_tiles(I), (uint8_t*)gu_packed, c->stream));
  MS_CUDA(c, launch_mxfp4_pack((const uint8_t*)up, E, I, H, 64, 64, tc_gu_tiles(I), (uint8_t*)gu_packed, c->stream));
  MS_CUDA(c, launch_mxfp4_pack((const uint8_t*)down, E, H, I, 128, 0, tc_down_tiles(H), (uint8_t*)down_packed,
                               c->stream));
  return MS_OK;
}

ms_status ms_moe_mxfp4_decode_packed(ms_ctx* c, const void* gu, const void* down, const float* gb, const float* ub,
                                     const float* db, int H, int I, int E, int K, int arch, const float* x,
                                     const int32_t* idx, const float* wts, float* h) {
  if (!c || !gu || !down || !x || !idx || !wts || !h || K <= 0 || K > 16 || E <= 0) return MS_ERR_INVALID_ARG;
  if (!tc_supported(H, I)) return fail(c, MS_ERR_SHAPE, "moe packed: hidden and inter must be multiples of 64");
  const size_t al = 256;
  auto up = [&](size_t b) { return (b + al - 1) & ~(al - 1); };
  const size_t xt_b = up((size_t)tc_bterm_bytes(H / 32)), at_b = up((size_t)K * tc_bterm_bytes(I / 32));
  const size_t act_b = up((size_t)K * I * 4), part_b = up((size_t)K * H * 4);
  const int items = tc_max_items(H, I, K);
  const size_t sp_b = up((size_t)2 * items * kTcMaxSeg * 128 * 4);
  ms_status s = ensure_scratch(c, xt_b + at_b + act_b + part_b + sp_b, 64 + 1024 + (size_t)tc_cnt_words(H, I, K));
  if (s != MS_OK) return s;
  uint8_t* base = (uint8_t*)c->scratch;
  TcMoeArgs a;
  a.gu = (const uint8_t*)gu; a.down = (const uint8_t*)down; a.gate_b = gb; a.up_b = ub; a.down_b = db;
  a.xterm = base; a.act_terms = base + xt_b; a.act = (float*)(base + xt_b + at_b);
  a.partial = (float*)(base + xt_b + at_b + act_b); a.part = (float*)(base + xt_b + at_b + act_b + part_b);
  a.cnt = c->counters + 64 + 1024; a.idx = idx; a.wts = wts; a.H = H; a.I = I; a.K = K; a.expert_base = 0;
  a.n_local = E; a.oai_swiglu = arch == MS_ARCH_GPT_OSS; a.h = h;
  MS_CUDA(c, launch_xterms(c->dc, x, H, base, c->stream));
  MS_CUDA(c, launch_moe_tc(c->dc, a, c->stream));
  return MS_OK;
}

ms_status ms_moe_mxfp4_prefill_packed(ms_ctx* c, const void* gu, const void* down, const float* gb, const float* ub,
                                      const float* db, int H, int I, int E, int K, int arch, const float* x, int T,
                                      const int32_t* idx, const float* wts, float* out, int precise) {
  if (!c || !gu || !down || !x || !idx || !wts || !out || K <= 0 || K > 16 || E <= 0 || E > 256 || T <= 0)
    return MS_ERR_INVALID_ARG;
  if (!tc_supported(H, I)) return fail(c, MS_ERR_SHAPE, "moe prefill: hidden and inter must be multiples of 64");
  if (precise != 0 && precise != 1) return MS_ERR_INVALID_ARG;
  ms_status s = ensure_scratch(c, pf_scratch_bytes(H, I, E, T, K, precise), 64);
  if (s != MS_OK) return s;
  PrefillArgs a;
  a.gu = (const uint8_t*)gu; a.down = (const uint8_t*)down; a.gate_b = gb; a.up_b = ub; a.down_b = db;
  a.x = x; a.idx = idx; a.wts = wts; a.out = out; a.scratch = c->scratch;
  a.H = H; a.I = I; a.E = E; a.K = K; a.T = T; a.expert_base = 0; a.oai_swiglu = arch == MS_ARCH_GPT_OSS;
  a.precise = precise;
  MS_CUDA(c, launch_moe_prefill(c->dc, a, c->stream));
  return MS_OK;
}

ms_status ms_rope(ms_ctx* c, const float* x, const float* cs, const float* sn, int n_tok, int heads, int hd, int rot,
                  float* y) {
  if (!c || !x || !cs || !sn || !y || n_tok <= 0 || heads <= 0 || hd <= 0) return MS_ERR_INVALID_ARG;
  if (rot <= 0 || rot > hd || rot % 2) return fail(c, MS_ERR_SHAPE, "rope: rot_dim %d must be even and <= head_dim %d", rot, hd);
  if (x == y) return fail(c, MS_ERR_INVALID_ARG, "rope: output must not overlap the input");
  MS_CUDA(c, launch_rope(x, cs, sn, y, n_tok, heads, hd, rot, c->stream));
  return MS_OK;
}

ms_status ms_sample(ms_ctx* c, const float* logits, int V, const uint32_t* counts, float temperature, float top_p,
                    float repetition_penalty, float r, float* work, int32_t* token) {
  if (!c || !logits || !work || !token || V <= 0) return MS_ERR_INVALID_ARG;
  if (!(temperature >= 0.0f) || !(top_p > 0.0f) || !(repetition_penalty > 0.0f) || !(r >= 0.0f && r < 1.0f))
    return fail(c, MS_ERR_INVALID_ARG, "sample: temperature >= 0, top_p > 0, penalty > 0 and 0 <= r < 1 required");
  SampleArgs a;
  a.logits = logits; a.V = V; a.counts = counts; a.temperature = temperature; a.top_p = top_p;
  a.penalty = repetition_penalty; a.r = r; a.work = work; a.token_out = token;
  MS_CUDA(c, launch_sample(c->dc, a, c->stream));
  return MS_OK;
}

ms_status ms_attn_layer_decode(ms_ctx* c, const ms_attn_layer* L, int pos, float* h) {
  if (!c || !L || !h || !L->attn_norm || !L->wqkv || !L->wo || !L->k_cache || !L->v_cache || !L->cos_t || !L->sin_t)
    return MS_ERR_INVALID_ARG;
  const int H = L->hidden, nh = L->heads, nkv = L->kv_heads, hd = L->head_dim;
  if (H <= 0 || nh <= 0 || nkv <= 0 || nh % nkv || hd <= 0 || L->cap <= 0 || pos < 0)
    return fail(c, MS_ERR_SHAPE, "attn layer: invalid shape");
  if (H % 32 || (nh * hd) % 32 || (hd != 32 && hd != 64 && hd != 128 && hd != 256) || L->rot_dim <= 0 ||
      L->rot_dim > hd || L->rot_dim % 2)
    return fail(c, MS_ERR_SHAPE, "attn layer: hidden and q_dim multiples of 32, head_dim 32/64/128/256 required");
  if ((L->q_norm == nullptr) != (L->k_norm == nullptr)) return fail(c, MS_ERR_INVALID_ARG, "attn layer: q_norm and k_norm go together");
  if (L->window <= 0 && pos >= L->cap) return fail(c, MS_ERR_SHAPE, "attn layer: position %d beyond the cache", pos);
  if (L->window > 0 && L->cap != L->window) return fail(c, MS_ERR_SHAPE, "attn layer: sliding-window cache must hold window slots");
  const int Dq = nh * hd, Dkv = nkv * hd, rep = nh / nkv;
  const int spl = hd <= 64 ? 0 : 256;
  const int range = L->cap;
  const int S = spl ? (range + spl - 1) / spl : attn_splits(range, hd);
  const int gated = L->q_gate ? 1 : 0;
  auto up = [](size_t b) { return (b + 255) & ~(size_t)255; };
  const size_t o_qkv = 0, o_att = o_qkv + up((size_t)(Dq + 2 * Dkv) * 4), o_oq = o_att + up((size_t)Dq * 4),
               o_od = o_oq + up((size_t)Dq + 64), o_part = o_od + up((size_t)Dq / 32 * 4 + 64),
               o_pos = o_part + up((size_t)nkv * S * rep * (hd + 2) * 4), o_raw = o_pos + 256,
               o_gate = o_raw + (gated ? up((size_t)(2 * Dq + 2 * Dkv) * 4) : 0),
               total = o_gate + (gated ? up((size_t)Dq * 4) : 0);
  // counter words [4096, 4096 + 4 nkv + 16) are this entry point's (self-resetting)
  ms_status st = ensure_scratch(c, total, 4096 + 4 * (size_t)nkv + 16);
  if (st != MS_OK) return st;
  uint8_t* base = (uint8_t*)c->scratch;
  int* d_pos = (int*)(base + o_pos);
  MS_CUDA(c, launch_set_i32(d_pos, pos, c->stream));
  Q8GemvArgs qa;
  qa.w = (const uint8_t*)L->wqkv; qa.rows = (gated ? 2 : 1) * Dq + 2 * Dkv; qa.cols = H; qa.x = h;
  qa.norm_w = L->attn_norm; qa.eps = L->eps; qa.bias = L->bqkv;
  qa.y = (float*)(base + (gated ? o_raw : o_qkv));
  MS_CUDA(c, launch_q8_gemv(c->dc, qa, c->stream));
  if (gated)   // [Q_h, gate_h] per head -> q rows, then k, v; and the gate
    MS_CUDA(c, launch_gate_split((const float*)(base + o_raw), nh, hd, Dkv, (float*)(base + o_qkv),
                                 (float*)(base + o_gate), c->stream));
  AttnArgs aa;
  aa.qkv = (const float*)(base + o_qkv); aa.q_norm = L->q_norm; aa.k_norm = L->k_norm; aa.eps = L->eps;
  aa.cos_t = L->cos_t; aa.sin_t = L->sin_t; aa.rot = L->rot_dim; aa.pos = d_pos; aa.kc = L->k_cache; aa.vc = L->v_cache;
  aa.cap = L->cap; aa.window = L->window > 0 ? L->window : 0; aa.sinks = L->sinks; aa.part = (float*)(base + o_part);
  aa.cnt = c->counters + 4096; aa.out = (float*)(base + o_att); aa.nh = nh; aa.nkv = nkv; aa.hd = hd; aa.S = S;
  aa.spl = spl; aa.scale = (float)(1.0 / std::sqrt((double)hd));
  // the O projection's Q8_0 activation comes from the attention kernel, or after the gate
  aa.oq = gated ? nullptr : (int8_t*)(base + o_oq);
  aa.od = gated ? nullptr : (float*)(base + o_od);
  if (spl && rep % 4 == 0) aa.head_split = 4;
  else if (spl && rep % 2 == 0 && rep >= 4) aa.head_split = 2;
  // order-independent attention (f64 reductions rounded once) where it has a kernel
  if ((hd == 32 || hd == 64 || (hd == 128 && rep <= 8)) && 32 % rep == 0)
    MS_CUDA(c, launch_exact_attention(c->dc, aa, range, c->stream));
  else
    MS_CUDA(c, launch_attention(c->dc, aa, c->stream));
  if (gated)   // attn_out *= sigmoid(gate) (layer.rs:699-705), then its Q8_0 blocks
    MS_CUDA(c, launch_gate_apply_q8((float*)(base + o_att), (const float*)(base + o_gate), Dq, (int8_t*)(base + o_oq),
                                    (float*)(base + o_od), c->stream));
  Q8GemvArgs oa;
  oa.w = (const uint8_t*)L->wo; oa.rows = H; oa.cols = Dq; oa.xq_in = (const int8_t*)(base + o_oq);
  oa.xd_in = (const float*)(base + o_od); oa.bias = L->bo;
  oa.residual = h;
  MS_CUDA(c, launch_q8_gemv(c->dc, oa, c->stream));
  return MS_OK;
}

// ---- hybrid blocks: Gated DeltaNet decode, shared expert ----
static bool gemv_qtype_ok(int q) {
  return q == Q_MXFP4 || q == Q_Q8_0 || q == Q_F16 || q == Q_F32 || q == Q_Q4_K || q == Q_Q6_K;
}

static ms_status gemv_into(ms_ctx* c, int q, const void* w, int rows, int cols, const float* x, float* y,
                           const char* what) {
  if (!w) return fail(c, MS_ERR_INVALID_ARG, "%s: null weight", what);
  if (!gemv_qtype_ok(q)) return fail(c, MS_ERR_UNSUPPORTED_QTYPE, "%s qtype %d", what, q);
  if (row_bytes(q, cols) < 0) return fail(c, MS_ERR_SHAPE, "%s: cols %d not a whole number of blocks", what, cols);
  GemvArgs a;
  a.qtype = q; a.w = w; a.rows = rows; a.cols = cols; a.x = x; a.y = y;
  cudaError_t e = launch_gemv(c->dc, a, c->stream);
  if (e == cudaErrorInvalidValue) return fail(c, MS_ERR_SHAPE, "%s: unsupported shape %dx%d", what, rows, cols);
  if (e != cudaSuccess) return cuda_fail(c, e, what);
  return MS_OK;
}

ms_status ms_deltanet_decode(ms_ctx* c, const ms_deltanet_layer* L, const float* x, float* conv_state, float* rec_state,
                             float* y) {
  if (!c || !L || !x || (!conv_state && L->conv_kernel > 1) || !rec_state || !y || !L->conv1d || !L->ssm_a || !L->dt_bias || !L->norm)
    return MS_ERR_INVALID_ARG;
  const int nk = L->n_k_heads, hkd = L->head_k_dim, nv = L->n_v_heads, hvd = L->head_v_dim, H = L->hidden;
  if (H <= 0 || nk <= 0 || nv <= 0 || L->conv_kernel < 1 || nv % nk) return MS_ERR_INVALID_ARG;
  if (hvd != 128 || hkd <= 0 || hkd > 128 || hkd % 2)
    return fail(c, MS_ERR_SHAPE, "deltanet: head_v_dim 128 and even head_k_dim <= 128 required");
  const int qt = nk * hkd, vt = nv * hvd, conv_dim = 2 * qt + vt;
  // scratch (floats): mixed, conv_out, z, ba, o — each 64-float aligned
  auto al = [](size_t n) { return (n + 63) & ~(size_t)63; };
  const size_t o_mixed = 0, o_conv = al(conv_dim), o_z = o_conv + al(conv_dim), o_ba = o_z + al(vt),
               o_o = o_ba + al(2 * nv), total = o_o + al(vt);
  ms_status s = ensure_scratch(c, total * 4, 64);
  if (s != MS_OK) return s;
  float* f = (float*)c->scratch;
  if ((s = gemv_into(c, L->qkv_q, L->qkv, conv_dim, H, x, f + o_mixed, "deltanet qkv")) != MS_OK) return s;
  if ((s = gemv_into(c, L->gate_q, L->gate, vt, H, x, f + o_z, "deltanet gate")) != MS_OK) return s;
  if ((s = gemv_into(c, L->ba_q, L->ba, 2 * nv, H, x, f + o_ba, "deltanet ba")) != MS_OK) return s;
  DeltaNetStep a;
  a.nk = nk; a.hkd = hkd; a.nv = nv; a.hvd = hvd; a.eps = L->eps; a.scale = 1.0f / sqrtf((float)hvd);
  a.conv_out = f + o_conv; a.ba = f + o_ba; a.z = f + o_z; a.ssm_a = L->ssm_a; a.dt_bias = L->dt_bias;
  a.norm = L->norm; a.state = rec_state; a.out = f + o_o;
  MS_CUDA(c, launch_deltanet_core(c->dc, a, conv_dim, L->conv_kernel, f + o_mixed, L->conv1d, conv_state, c->stream));
  return gemv_into(c, L->out_q, L->out, H, vt, f + o_o, y, "deltanet out");
}

ms_status ms_shared_expert(ms_ctx* c, int guq, const void* gate, const void* up, int dq, const void* down,
                           const float* gate_inp, int H, int I, const float* x, float* y) {
  if (!c || !gate || !up || !down || !x || !y || H <= 0 || I <= 0) return MS_ERR_INVALID_ARG;
  auto al = [](size_t n) { return (n + 63) & ~(size_t)63; };
  const size_t o_g = 0, o_u = al(I), o_a = o_u + al(I), o_o = o_a + al(I), total = o_o + al(H);
  ms_status s = ensure_scratch(c, total * 4, 64);
  if (s != MS_OK) return s;
  float* f = (float*)c->scratch;
  if ((s = gemv_into(c, guq, gate, I, H, x, f + o_g, "shared expert gate")) != MS_OK) return s;
  if ((s = gemv_into(c, guq, up, I, H, x, f + o_u, "shared expert up")) != MS_OK) return s;
  MS_CUDA(c, launch_silu_mul(f + o_g, f + o_u, f + o_a, I, c->stream));
  if ((s = gemv_into(c, dq, down, H, I, f + o_a, f + o_o, "shared expert down")) != MS_OK) return s;
  MS_CUDA(c, launch_gated_accum(x, gate_inp, f + o_o, y, H, c->stream));
  return MS_OK;
}

// ---------------------------------------------------------------------------------
ms_status ms_model_create(ms_ctx* c, const ms_model_config* cfg, ms_model** out) {
  if (!c || !cfg || !out) return MS_ERR_INVALID_ARG;
  *out = nullptr;
  const ms_model_config& k = *cfg;
  if (k.hidden <= 0 || k.layers <= 0 || k.heads <= 0 || k.kv_heads <= 0 || k.heads % k.kv_heads || k.head_dim <= 0 ||
      k.experts <= 0 || k.top_k <= 0 || k.top_k > 16 || k.top_k > k.experts || k.inter <= 0 || k.vocab <= 0 ||
      k.max_seq_len <= 0 || k.rot_dim <= 0 || k.rot_dim > k.head_dim || k.rot_dim % 2 || k.ep_size <= 0 ||
      k.ep_rank < 0 || k.ep_rank >= k.ep_size || k.experts % k.ep_size)
    return fail(c, MS_ERR_INVALID_ARG, "invalid model config");
  if (k.hidden % 64 || k.inter % 32) return fail(c, MS_ERR_SHAPE, "hidden %% 64 and inter %% 32 required");
  if (k.attn_interval < 0) return fail(c, MS_ERR_INVALID_ARG, "invalid model config: attn_interval < 0");
  if (k.attn_interval > 0 &&
      (k.ssm_groups <= 0 || k.ssm_state <= 0 || k.ssm_dt_rank <= 0 || k.ssm_inner <= 0 || k.ssm_conv < 1 ||
       k.ssm_conv > 16 || k.ssm_dt_rank % k.ssm_groups || k.ssm_inner % k.ssm_dt_rank))
    return fail(c, MS_ERR_INVALID_ARG, "invalid DeltaNet config (ssm fields)");
  if (k.attn_interval > 0 && (k.ssm_inner / k.ssm_dt_rank != 128 || k.ssm_state > 128 || k.ssm_state % 2))
    return fail(c, MS_ERR_SHAPE, "DeltaNet: value head dim 128 and an even key head dim <= 128 required");
  auto* m = new ms_model();
  m->ctx = c;
  c->models.push_back(m);
  m->cfg = k;
  m->L.resize(k.layers);
  m->n_local = k.experts / k.ep_size;
  if (const char* v = getenv("MS_MOE_TC")) m->use_tc = atoi(v) != 0;
  if (const char* v = getenv("MS_EXACT")) m->exact = atoi(v) != 0;
  m->expert_base = k.ep_rank * m->n_local;
  *out = m;
  return MS_OK;
}

ms_status ms_model_set_tensor(ms_model* m, const char* name, int q, int nd, const int64_t* dims, const void* data,
                              size_t bytes) {
  if (!m || !name || !dims || nd <= 0 || nd > 4 || !data) return MS_ERR_INVALID_ARG;
  if (m->finalized) return fail(m->ctx, MS_ERR_STATE, "set_tensor after finalize");
  cudaSetDevice(m->ctx->device);
  std::vector<int64_t> d(dims, dims + nd);
  int64_t n = 1;
  for (auto x : d) n *= x;
  const std::string nm(name);
  const ms_model_config& c = m->cfg;
  m->seen.insert(nm);
  if (raw_bytes(q, n) < 0) return fail(m->ctx, MS_ERR_UNSUPPORTED_QTYPE, "%s: qtype %d", name, q);
  if ((int64_t)bytes < raw_bytes(q, n)) return fail(m->ctx, MS_ERR_SHAPE, "%s: short buffer", name);
  if (nm == "token_embd.weight") {
    if (nd != 2 || d[0] != c.vocab || d[1] != c.hidden || (q != Q_F16 && q != Q_F32))
      return fail(m->ctx, MS_ERR_SHAPE, "%s: expected F16/F32 [%d, %d]", name, c.vocab, c.hidden);
    ms_status s = m->alloc(&m->embd, (size_t)raw_bytes(q, n), false);
    if (s != MS_OK) return s;
    m->embd_q = q;
    return upload(m, m->embd, data, (size_t)raw_bytes(q, n));
  }
  if (nm == "output.weight") {
    if (nd != 2 || d[0] != c.vocab || d[1] != c.hidden) return fail(m->ctx, MS_ERR_SHAPE, "%s: bad shape", name);
    if (q != Q_F16) return fail(m->ctx, MS_ERR_UNSUPPORTED_QTYPE, "%s: LM head must be F16", name);
    ms_status s = m->alloc(&m->out_w, (size_t)raw_bytes(q, n), false);
    if (s != MS_OK) return s;
    return upload(m, m->out_w, data, (size_t)raw_bytes(q, n));
  }
  if (nm == "output_norm.weight") return set_vec(m, &m->out_norm, name, q, n, c.hidden, data);
  if (nm == "output.bias") return set_vec(m, &m->out_b, name, q, n, c.vocab, data);
  int li = -1, off = 0;
  if (sscanf(name, "blk.%d.%n", &li, &off) == 1 && off > 0) {
    if (li < 0 || li >= c.layers) return fail(m->ctx, MS_ERR_SHAPE, "%s: layer out of range", name);
    return set_layer_tensor(m, li, std::string(name + off), q, d, data, bytes);
  }
  return MS_OK;
}

ms_status ms_model_finalize(ms_model* m) {
  if (!m) return MS_ERR_INVALID_ARG;
  if (m->finalized) return MS_OK;
  cudaSetDevice(m->ctx->device);
  const ms_model_config& c = m->cfg;
  if (!m->embd || !m->out_w || !m->out_norm) return fail(m->ctx, MS_ERR_STATE, "missing token_embd/output/output_norm");
  bool any_tc = false, any_dn = false;
  for (int li = 0; li < c.layers; ++li) {
    LayerW& Lw = m->L[li];
    Lw.deltanet = !is_attention_layer(c, li);
    if (!Lw.attn_norm || !Lw.post_norm || !Lw.router_w || !Lw.have_gate || !Lw.have_up || !Lw.have_down ||
        (!Lw.deltanet && (Lw.qkv_parts != 3 || !Lw.wo)))
      return fail(m->ctx, MS_ERR_STATE, "layer %d: missing tensors", li);
    if (Lw.deltanet && (!Lw.dn_qkv || !Lw.dn_z || Lw.dn_ba_parts != 2 || !Lw.dn_out || !Lw.dn_conv_w || !Lw.dn_a ||
                        !Lw.dn_dt || !Lw.dn_norm))
      return fail(m->ctx, MS_ERR_STATE, "layer %d: missing Gated DeltaNet tensors", li);
    if (Lw.sh_gate || Lw.sh_up || Lw.sh_down) {
      if (!Lw.sh_gate || !Lw.sh_up || !Lw.sh_down || Lw.sh_dims[0] != Lw.sh_dims[1] || Lw.sh_dims[0] != Lw.sh_dims[2] ||
          Lw.sh_gate_q != Lw.sh_up_q)
        return fail(m->ctx, MS_ERR_STATE, "layer %d: incomplete or inconsistent shared expert", li);
      m->sh_max = std::max(m->sh_max, Lw.sh_dims[0]);
    }
    Lw.tc = Lw.gu_tc && Lw.down_tc;
    if ((Lw.gu_tc || Lw.down_tc) && !Lw.tc)
      return fail(m->ctx, MS_ERR_UNSUPPORTED_QTYPE, "layer %d: MXFP4 and K-quant experts mixed in one layer", li);
    any_tc = any_tc || Lw.tc;
    if (Lw.bqkv_parts != 0 && Lw.bqkv_parts != 3) return fail(m->ctx, MS_ERR_STATE, "layer %d: partial qkv bias", li);
    if ((Lw.qn == nullptr) != (Lw.kn == nullptr)) return fail(m->ctx, MS_ERR_STATE, "layer %d: q/k norm mismatch", li);
    Lw.window = (c.sliding_window > 0 && li % 2 == 0) ? c.sliding_window : 0;   // config.rs:463-465
    Lw.cap = Lw.window ? std::min(Lw.window, c.max_seq_len) : c.max_seq_len;
    if (Lw.window) Lw.cap = Lw.window;
    ms_status s = MS_OK;
    if (Lw.deltanet) {   // DeltaNetState (deltanet.rs:139-196): zero at the start of a sequence
      s = m->alloc(&Lw.dn_conv_state, (size_t)dn_conv_dim(c) * std::max(c.ssm_conv - 1, 1) * 4);
      if (s == MS_OK) s = m->alloc(&Lw.dn_state, (size_t)c.ssm_dt_rank * c.ssm_state * dn_hvd(c) * 4);
      any_dn = true;
    } else {
      const size_t kvb = (size_t)c.kv_heads * Lw.cap * c.head_dim * 4;
      s = m->alloc(&Lw.kc, kvb, false);
      if (s == MS_OK) s = m->alloc(&Lw.vc, kvb, false);
    }
    if (s == MS_OK) s = m->alloc(&Lw.idx, 16 * 4);
    if (s == MS_OK) s = m->alloc(&Lw.wts, 16 * 4);
    if (s != MS_OK) return s;
  }
  if (m->tier_slots > 0) {
    for (int li = 0; li < c.layers; ++li) {
      ms_model::TierLayer& T = m->tier[li];
      if (!T.host[0] || !T.host[1] || !T.host[2])
        return fail(m->ctx, MS_ERR_STATE, "layer %d: host-tier expert stacks missing", li);
      if (!exact_kq_supported(m->L[li].gate_q, m->L[li].down_q, c.hidden, c.inter) || m->L[li].up_q != m->L[li].gate_q)
        return fail(m->ctx, MS_ERR_UNSUPPORTED_QTYPE, "layer %d: host-tier experts need Q4_K / Q6_K shapes the "
                    "order-independent kernels cover", li);
      T.slot_expert.assign(m->tier_slots, -1);
      T.slot_used.assign(m->tier_slots, 0);
      ms_status ts = m->alloc(&T.wslot, 16 * 4);
      if (ts != MS_OK) return ts;
    }
    MS_CUDA(m->ctx, cudaMallocHost(&m->h_wslot, (size_t)c.layers * 16 * 4));
    MS_CUDA(m->ctx, cudaMallocHost(&m->h_tier_idx, 16 * 4));
  }
  const int H = c.hidden, Dq = q_dim(c), Dkv = kv_dim(c), rep = c.heads / c.kv_heads;
  // decode attention splits: 128 positions each, sized for the longest attended range
  // decode attention splits sized for the longest attended range of each layer kind: head_dim <= 64
  // uses the tile kernel (whole K/V tiles staged before the wait), wider heads the streaming
  // kernel with 256-position splits (measured faster at 128)
  m->attn_spl = c.head_dim <= 64 ? 0 : 256;
  auto n_splits = [&](int range) { return m->attn_spl ? (range + m->attn_spl - 1) / m->attn_spl : attn_splits(range, c.head_dim); };
  const int S = n_splits(c.max_seq_len);
  m->splits_full = S;
  m->splits_swa = c.sliding_window > 0 ? n_splits(std::min(c.sliding_window, c.max_seq_len)) : S;
  ms_status s = MS_OK;
  s = s ? s : m->alloc(&m->h, (size_t)H * 4);
  s = s ? s : m->alloc(&m->h_last, (size_t)H * 4);
  s = s ? s : m->alloc(&m->moe_out, (size_t)H * 4);
  s = s ? s : m->alloc(&m->xq_h, (size_t)H + 64);
  s = s ? s : m->alloc(&m->xd_h, (size_t)H / 32 * 4 + 64);
  s = s ? s : m->alloc(&m->xq_a, (size_t)Dq + 64);
  s = s ? s : m->alloc(&m->xd_a, (size_t)Dq / 32 * 4 + 64);
  s = s ? s : m->alloc(&m->qkv, (size_t)(Dq + 2 * Dkv) * 4);
  s = s ? s : m->alloc(&m->attn_out, (size_t)Dq * 4);
  s = s ? s : m->alloc(&m->xn, (size_t)H * 4);
  s = s ? s : m->alloc(&m->router_logits, (size_t)c.experts * 4);
  s = s ? s : m->alloc(&m->act, (size_t)c.top_k * c.inter * 4);
  s = s ? s : m->alloc(&m->partial, (size_t)c.top_k * H * 4);
  s = s ? s : m->alloc(&m->logits, (size_t)c.vocab * 4);
  s = s ? s : m->alloc(&m->attn_part, (size_t)c.kv_heads * S * rep * (c.head_dim + 2) * 4);
  s = s ? s : m->alloc(&m->router_cnt, 16);
  s = s ? s : m->alloc(&m->resid_cnt, 16);
  s = s ? s : m->alloc(&m->tile_cnt, (size_t)(H / 16 + 16) * 4);
  s = s ? s : m->alloc(&m->attn_cnt, (size_t)(4 * c.kv_heads + 16) * 4);
  s = s ? s : m->alloc(&m->st, sizeof(StepState));
  s = s ? s : m->alloc(&m->token_log, (size_t)(c.max_seq_len + 1) * 4);
  s = s ? s : m->alloc(&m->ex_kgu, (size_t)c.top_k * 2 * c.inter * 4);
  s = s ? s : m->alloc(&m->xn_final, (size_t)H * 4);
  s = s ? s : m->alloc(&m->ref_scratch, (size_t)exact_refine_scratch_ints(1) * 4);
  s = s ? s : m->alloc(&m->r_raw, (size_t)c.experts * 4);
  s = s ? s : m->alloc(&m->r_entropy, (size_t)c.layers * 4);
  s = s ? s : m->alloc(&m->r_k, (size_t)c.layers * 4);
  s = s ? s : m->alloc(&m->st_cnt, (size_t)c.layers * c.experts * 8);
  s = s ? s : m->alloc(&m->st_wsum, (size_t)c.layers * c.experts * 8);
  s = s ? s : m->alloc(&m->st_tok, (size_t)c.layers * 8);
  s = s ? s : m->alloc(&m->st_log, (size_t)c.max_seq_len * c.layers * 4);
  s = s ? s : m->alloc(&m->st_n, (size_t)c.layers * 4);
  if (is_hybrid(c)) {   // gated attention: [Q_h, gate_h] projection, then the gate
    s = s ? s : m->alloc(&m->q_raw, (size_t)(q_rows(c) + 2 * Dkv) * 4);
    s = s ? s : m->alloc(&m->q_gate, (size_t)Dq * 4);
  }
  if (any_dn) {
    const int conv_dim = dn_conv_dim(c);
    // the input projections' outputs back to back [mixed qkv | z | beta, alpha] (one GEMV writes all)
    s = s ? s : m->alloc(&m->dn_mixed, ((size_t)conv_dim + c.ssm_inner + 2 * c.ssm_dt_rank) * 4);
    if (s == MS_OK) {
      m->dn_zv = m->dn_mixed + conv_dim;
      m->dn_bav = m->dn_zv + c.ssm_inner;
    }
    s = s ? s : m->alloc(&m->dn_conv, (size_t)conv_dim * 4);
    s = s ? s : m->alloc(&m->dn_o, (size_t)c.ssm_inner * 4);
  }
  if (m->sh_max > 0) {
    s = s ? s : m->alloc(&m->sh_g, (size_t)2 * m->sh_max * 4);   // [gate | up] outputs of one layer
    s = s ? s : m->alloc(&m->sh_a, (size_t)m->sh_max * 4);
    s = s ? s : m->alloc(&m->sh_o, (size_t)H * 4);
    s = s ? s : m->alloc(&m->sh_y, (size_t)H * 4);
  }
  if (any_tc) {
    m->ex_seg_gu = exact_seg_count(H / 32);
    m->ex_seg_down = exact_seg_count(c.inter / 32);
    m->ex_hpad = tc_down_tiles(H) * 128;
    s = s ? s : m->alloc(&m->ex_gp, (size_t)c.top_k * m->ex_seg_gu * 2 * c.inter * 8);
    s = s ? s : m->alloc(&m->ex_dp, (size_t)c.top_k * m->ex_seg_down * m->ex_hpad * 8);
    s = s ? s : m->alloc(&m->ex_xbt, (size_t)(H / 32) * exact_term_block_bytes());
    s = s ? s : m->alloc(&m->ex_xfe, (size_t)(H / 32 + 8) * 4);   // + the padding of a 32-byte copy
    s = s ? s : m->alloc(&m->ex_abt, (size_t)c.top_k * (c.inter / 32) * exact_term_block_bytes());
    s = s ? s : m->alloc(&m->ex_afe, (size_t)c.top_k * ((c.inter / 32 + 7) & ~7) * 4 + 32);   // rows of 8-aligned stride
    s = s ? s : m->alloc(&m->ex_cnt, (size_t)c.top_k * (tc_gu_tiles(c.inter) + tc_down_tiles(H)) * 4);
    s = s ? s : m->alloc(&m->xterm, (size_t)tc_bterm_bytes(H / 32));
    s = s ? s : m->alloc(&m->act_terms, (size_t)c.top_k * tc_bterm_bytes(c.inter / 32));
    s = s ? s : m->alloc(&m->tc_part, (size_t)2 * tc_max_items(H, c.inter, c.top_k) * kTcMaxSeg * 128 * 4);
    s = s ? s : m->alloc(&m->tc_cnt, (size_t)tc_cnt_words(H, c.inter, c.top_k) * 4);
  }
  if (s != MS_OK) return s;
  std::vector<float> cs, sn;
  rope_tables(c.rot_dim, c.max_seq_len, (double)c.rope_theta, cs, sn);
  s = m->alloc(&m->cos_t, cs.size() * 4, false);
  s = s ? s : m->alloc(&m->sin_t, sn.size() * 4, false);
  if (s != MS_OK) return s;
  s = upload(m, m->cos_t, cs.data(), cs.size() * 4);
  s = s ? s : upload(m, m->sin_t, sn.data(), sn.size() * 4);
  if (s != MS_OK) return s;
  MS_CUDA(m->ctx, cudaMallocHost(&m->h_tok, (size_t)(c.max_seq_len + 4) * 4));
  m->h_tok[c.max_seq_len + 2] = 0;
  m->h_tok[c.max_seq_len + 3] = 1;
  MS_CUDA(m->ctx, cudaMallocHost(&m->h_st, sizeof(StepState)));
  memset(m->h_st, 0, sizeof(StepState));
  m->h_st->max_seq = c.max_seq_len;
  MS_CUDA(m->ctx, cudaMemcpy(m->st, m->h_st, sizeof(StepState), cudaMemcpyHostToDevice));
  m->finalized = true;
  return MS_OK;
}

// ---------------- lockstep batch (Engine::forward over input_ids [B, T], engine.rs:1869-2006) ----------------

ms_status ms_model_batch_open(ms_model* m, int B) {
  if (!m || B < 1 || B > kMaxBatch) return MS_ERR_INVALID_ARG;
  if (!m->finalized) return fail(m->ctx, MS_ERR_STATE, "batch before finalize");
  const ms_model_config& c = m->cfg;
  if (c.ep_size > 1) return fail(m->ctx, MS_ERR_STATE, "batched decode runs on one GPU (ep_size 1)");
  if (is_hybrid(c) || m->sh_max > 0)
    return fail(m->ctx, MS_ERR_UNSUPPORTED_QTYPE, "batched decode covers attention + routed-expert layers only");
  if (m->tier_slots > 0) return fail(m->ctx, MS_ERR_STATE, "batched decode needs HBM-resident experts (no host tier)");
  if (m->dyn_k || m->router_stats) return fail(m->ctx, MS_ERR_STATE, "batched decode has no dynamic K / router statistics");
  for (int li = 0; li < c.layers; ++li)
    if (m->L[li].tc || !m->L[li].gate)
      return fail(m->ctx, MS_ERR_UNSUPPORTED_QTYPE,
                  "batched decode needs native-layout experts (K-quants, or MXFP4 with MS_MOE_TC=0)");
  const int H = c.hidden, Dq = q_dim(c), Dkv = kv_dim(c), rep = c.heads / c.kv_heads;
  if ((Dq + 2 * Dkv) % 16 || H % 16) return fail(m->ctx, MS_ERR_SHAPE, "batched projections need rows %% 16");
  cudaSetDevice(m->ctx->device);
  MS_CUDA(m->ctx, cudaStreamSynchronize(m->ctx->stream));
  batch_free(m);
  m->bt = new BatchRt();
  BatchRt& b = *m->bt;
  b.B = B;
  const int units = c.kv_heads * B, sms = m->ctx->dc.sm_count;
  b.spl_full = attn_split_positions(c.max_seq_len, units, sms);
  b.S_full = (c.max_seq_len + b.spl_full - 1) / b.spl_full;
  const int swa_range = c.sliding_window > 0 ? std::min(c.sliding_window, c.max_seq_len) : c.max_seq_len;
  b.spl_swa = attn_split_positions(swa_range, units, sms);
  b.S_swa = (swa_range + b.spl_swa - 1) / b.spl_swa;
  const int S = std::max(b.S_full, b.S_swa), EK = B * c.top_k;
  ms_status s = MS_OK;
  s = s ? s : balloc(m, &b.st, sizeof(BatchState));
  s = s ? s : balloc(m, &b.tok_in, (size_t)B * 4);
  s = s ? s : balloc(m, &b.keys, (size_t)B * 8);
  s = s ? s : balloc(m, &b.log, (size_t)(c.max_seq_len + 1) * B * 4);
  s = s ? s : balloc(m, &b.h, (size_t)B * H * 4);
  s = s ? s : balloc(m, &b.qkv, (size_t)B * (Dq + 2 * Dkv) * 4);
  s = s ? s : balloc(m, &b.attn, (size_t)B * Dq * 4);
  s = s ? s : balloc(m, &b.xn, (size_t)B * H * 4);
  s = s ? s : balloc(m, &b.rlog, (size_t)B * c.experts * 4);
  s = s ? s : balloc(m, &b.idx, (size_t)EK * 4);
  s = s ? s : balloc(m, &b.wts, (size_t)EK * 4);
  s = s ? s : balloc(m, &b.grp, (size_t)group_table_words(B, c.top_k) * 4);
  s = s ? s : balloc(m, &b.ent_slot, (size_t)EK * 4);
  s = s ? s : balloc(m, &b.ent_of, (size_t)EK * 4);
  s = s ? s : balloc(m, &b.ent_zero, (size_t)EK * 4);
  s = s ? s : balloc(m, &b.ref_scratch, (size_t)exact_refine_scratch_ints(B) * 4);
  s = s ? s : balloc(m, &b.act, (size_t)EK * 2 * c.inter * 4);
  s = s ? s : balloc(m, &b.y, (size_t)EK * H * 4);
  s = s ? s : balloc(m, &b.xf, (size_t)B * H * 4);
  s = s ? s : balloc(m, &b.logits, (size_t)B * c.vocab * 4);
  s = s ? s : balloc(m, &b.part, (size_t)B * c.kv_heads * S * rep * (c.head_dim + 2) * 4);
  s = s ? s : balloc(m, &b.xq_h, (size_t)B * H + 64);
  s = s ? s : balloc(m, &b.xd_h, (size_t)B * H / 32 * 4 + 64);
  s = s ? s : balloc(m, &b.xq_a, (size_t)B * Dq + 64);
  s = s ? s : balloc(m, &b.xd_a, (size_t)B * Dq / 32 * 4 + 64);
  s = s ? s : balloc(m, &b.attn_cnt, (size_t)(B * c.kv_heads + 16) * 4);
  s = s ? s : balloc(m, &b.router_cnt, (size_t)(B + 16) * 4);
  s = s ? s : balloc(m, &b.lm_scratch, (size_t)lm_batch_scratch_bytes(c.vocab, H));
  b.kc.resize(c.layers);
  b.vc.resize(c.layers);
  for (int li = 0; li < c.layers && s == MS_OK; ++li) {
    const size_t kvb = (size_t)B * c.kv_heads * m->L[li].cap * c.head_dim * 4;
    s = balloc(m, &b.kc[li], kvb);
    s = s ? s : balloc(m, &b.vc[li], kvb);
  }
  if (s != MS_OK) { batch_free(m); return s; }
  cudaError_t e = cudaMallocHost(&b.h_st, sizeof(BatchState));
  if (e == cudaSuccess) e = cudaMallocHost(&b.h_tok, ((size_t)c.max_seq_len * B + 4) * 4);
  if (e == cudaSuccess) e = cudaMallocHost(&b.h_keys, (size_t)B * 8);
  if (e != cudaSuccess) { batch_free(m); return cuda_fail(m->ctx, e, "cudaMallocHost (batch)"); }
  b.h_tok[(size_t)c.max_seq_len * B] = 0;
  b.h_tok[(size_t)c.max_seq_len * B + 1] = 1;
  memset(b.h_st, 0, sizeof(BatchState));
  b.h_st->max_seq = c.max_seq_len;
  MS_CUDA(m->ctx, cudaMemcpy(b.st, b.h_st, sizeof(BatchState), cudaMemcpyHostToDevice));
  return MS_OK;
}

ms_status ms_model_batch_close(ms_model* m) {
  if (!m) return MS_ERR_INVALID_ARG;
  cudaSetDevice(m->ctx->device);
  cudaStreamSynchronize(m->ctx->stream);
  batch_free(m);
  return MS_OK;
}

ms_status ms_model_batch_clear(ms_model* m) {
  ms_status st = batch_ready(m, 0);
  if (st != MS_OK) return st;
  BatchRt& b = *m->bt;
  MS_CUDA(m->ctx, cudaStreamSynchronize(m->ctx->stream));
  memset(b.h_st, 0, sizeof(BatchState));
  b.h_st->max_seq = m->cfg.max_seq_len;
  MS_CUDA(m->ctx, cudaMemcpy(b.st, b.h_st, sizeof(BatchState), cudaMemcpyHostToDevice));
  b.seq = 0;
  return MS_OK;
}

ms_status ms_model_batch_forward(ms_model* m, const int32_t* tokens, int T, int32_t* next) {
  if (!tokens || T <= 0) return MS_ERR_INVALID_ARG;
  ms_status st = batch_ready(m, T);
  if (st != MS_OK) return st;
  BatchRt& b = *m->bt;
  cudaStream_t s = m->ctx->stream;
  MS_CUDA(m->ctx, cudaStreamSynchronize(s));   // pinned staging is reused below
  for (int i = 0; i < b.B; ++i)
    for (int t = 0; t < T; ++t) {
      const int32_t tok = tokens[(size_t)i * T + t];
      if (tok < 0 || tok >= m->cfg.vocab) return fail(m->ctx, MS_ERR_INVALID_ARG, "token %d out of range", tok);
      b.h_tok[(size_t)t * b.B + i] = tok;
    }
  st = batch_feed(m, 0);
  if (st != MS_OK) return st;
  for (int t = 0; t < T; ++t) {
    MS_CUDA(m->ctx, cudaMemcpyAsync(b.tok_in, &b.h_tok[(size_t)t * b.B], (size_t)b.B * 4, cudaMemcpyHostToDevice, s));
    st = run_batch_step(m);
    if (st != MS_OK) return st;
  }
  b.seq += T;
  MS_CUDA(m->ctx, cudaMemcpyAsync(b.h_keys, b.keys, (size_t)b.B * 8, cudaMemcpyDeviceToHost, s));
  st = ms_sync(m->ctx);
  if (st != MS_OK) return st;
  if (next)
    for (int i = 0; i < b.B; ++i) next[i] = argmax_from_key(b.h_keys[i]);
  return MS_OK;
}

ms_status ms_model_batch_decode_steps_device(ms_model* m, int n) {
  if (n < 0) return MS_ERR_INVALID_ARG;
  ms_status st = batch_ready(m, n);
  if (st != MS_OK) return st;
  st = batch_feed(m, 1);
  if (st != MS_OK) return st;
  for (int i = 0; i < n; ++i) {
    st = run_batch_step(m);
    if (st != MS_OK) return st;
  }
  m->bt->seq += n;
  return MS_OK;
}

ms_status ms_model_batch_next_tokens(ms_model* m, int32_t* next) {
  if (!next) return MS_ERR_INVALID_ARG;
  ms_status st = batch_ready(m, 0);
  if (st != MS_OK) return st;
  BatchRt& b = *m->bt;
  MS_CUDA(m->ctx, cudaMemcpyAsync(b.h_keys, b.keys, (size_t)b.B * 8, cudaMemcpyDeviceToHost, m->ctx->stream));
  st = ms_sync(m->ctx);
  if (st != MS_OK) return st;
  for (int i = 0; i < b.B; ++i) next[i] = argmax_from_key(b.h_keys[i]);
  return MS_OK;
}

ms_status ms_model_batch_token_log(ms_model* m, int32_t* out, int max_rows, int* n_rows) {
  if (!out || !n_rows || max_rows < 0) return MS_ERR_INVALID_ARG;
  ms_status st = batch_ready(m, 0);
  if (st != MS_OK) return st;
  BatchRt& b = *m->bt;
  MS_CUDA(m->ctx, cudaStreamSynchronize(m->ctx->stream));
  BatchState h;
  MS_CUDA(m->ctx, cudaMemcpy(&h, b.st, sizeof h, cudaMemcpyDeviceToHost));
  const int k = std::min(std::min(h.n_log, max_rows), m->cfg.max_seq_len);
  if (k > 0) MS_CUDA(m->ctx, cudaMemcpy(out, b.log, (size_t)k * b.B * 4, cudaMemcpyDeviceToHost));
  *n_rows = k;
  return MS_OK;
}

ms_status ms_model_batch_last_logits(ms_model* m, float* out) {
  if (!out) return MS_ERR_INVALID_ARG;
  ms_status st = batch_ready(m, 0);
  if (st != MS_OK) return st;
  MS_CUDA(m->ctx, cudaStreamSynchronize(m->ctx->stream));
  MS_CUDA(m->ctx, cudaMemcpy(out, m->bt->logits, (size_t)m->bt->B * m->cfg.vocab * 4, cudaMemcpyDeviceToHost));
  return MS_OK;
}

ms_status ms_model_batch_profile_step(ms_model* m, float* us, int max, int* n) {
  if (!us || !n || max <= 0) return MS_ERR_INVALID_ARG;
  ms_status st = batch_ready(m, 0);
  if (st != MS_OK) return st;
  if (m->bt->kernels_per_step <= 0) return fail(m->ctx, MS_ERR_STATE, "profile after at least one batch step");
  cudaStream_t s = m->ctx->stream, cs = m->ctx->own;
  constexpr int kWarm = 3, kRuns = 10;
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  MS_CUDA(m->ctx, cudaEventCreate(&e0));
  MS_CUDA(m->ctx, cudaEventCreate(&e1));
  int k = 0;
  for (int c = 0; c < kBatchClasses && k < max && st == MS_OK; ++c) {
    // this class's launches of one batch step alone, PDL-chained as in the real step
    cudaGraph_t g = nullptr;
    cudaGraphExec_t ge = nullptr;
    st = ms_sync(m->ctx);
    if (st != MS_OK) break;
    MS_CUDA(m->ctx, cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal));
    m->prof_class = c;
    st = enqueue_batch_step(m, cs);
    m->prof_class = -1;
    cudaError_t e = cudaStreamEndCapture(cs, &g);
    if (st == MS_OK && e != cudaSuccess) st = cuda_fail(m->ctx, e, "cudaStreamEndCapture (batch profile)");
    if (st == MS_OK && (e = cudaGraphInstantiate(&ge, g, 0)) != cudaSuccess)
      st = cuda_fail(m->ctx, e, "cudaGraphInstantiate (batch profile)");
    for (int r = 0; r < kWarm + kRuns && st == MS_OK; ++r) {
      if (r == kWarm) cudaEventRecord(e0, s);
      if ((e = cudaGraphLaunch(ge, s)) != cudaSuccess) st = cuda_fail(m->ctx, e, "cudaGraphLaunch (batch profile)");
    }
    if (st == MS_OK) {
      cudaEventRecord(e1, s);
      st = ms_sync(m->ctx);
    }
    if (st == MS_OK) {
      float ms = 0.f;
      cudaEventElapsedTime(&ms, e0, e1);
      us[k++] = ms * 1000.f / kRuns;
    }
    if (ge) cudaGraphExecDestroy(ge);
    if (g) cudaGraphDestroy(g);
  }
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  *n = k;
  return st;
}

int ms_model_batch_kernels_per_step(const ms_model* m) { return m && m->bt ? m->bt->kernels_per_step : 0; }

ms_status ms_model_destroy(ms_model* m) {
  if (!m) return MS_ERR_INVALID_ARG;
  cudaSetDevice(m->ctx->device);
  cudaStreamSynchronize(m->ctx->stream);
  if (m->graph) cudaGraphExecDestroy(m->graph);
  if (m->comm) nccl_api()->comm_destroy(m->comm);
  for (void* p : m->ep_peer)
    if (p) cudaIpcCloseMemHandle(p);
  batch_free(m);
  for (void* p : m->pf.allocs) cudaFree(p);
  for (void* p : m->allocs) cudaFree(p);
  if (m->h_tok) cudaFreeHost(m->h_tok);
  if (m->h_st) cudaFreeHost(m->h_st);
  for (auto& T : m->tier)
    for (uint8_t* p : T.host)
      if (p) cudaFreeHost(p);
  if (m->h_wslot) cudaFreeHost(m->h_wslot);
  if (m->h_tier_idx) cudaFreeHost(m->h_tier_idx);
  auto& v = m->ctx->models;
  v.erase(std::remove(v.begin(), v.end(), m), v.end());
  delete m;
  return MS_OK;
}

ms_status ms_model_get_config(const ms_model* m, ms_model_config* cfg) {
  if (!m || !cfg) return MS_ERR_INVALID_ARG;
  *cfg = m->cfg;
  return MS_OK;
}

ms_status ms_model_set_graph(ms_model* m, int enable) {
  if (!m) return MS_ERR_INVALID_ARG;
  m->use_graph = enable != 0;
  return MS_OK;
}

int ms_model_kernels_per_step(const ms_model* m) { return m ? m->kernels_per_step : 0; }

ms_status ms_model_clear_cache(ms_model* m) {
  if (!m || !m->finalized) return MS_ERR_STATE;
  MS_CUDA(m->ctx, cudaStreamSynchronize(m->ctx->stream));
  // a new sequence: no token generated yet (the repetition penalty's list, engine.rs:2234)
  if (m->s_counts) MS_CUDA(m->ctx, cudaMemset(m->s_counts, 0, (size_t)m->cfg.vocab * 4));
  memset(m->h_st, 0, sizeof(StepState));
  m->h_st->max_seq = m->cfg.max_seq_len;
  MS_CUDA(m->ctx, cudaMemcpy(m->st, m->h_st, sizeof(StepState), cudaMemcpyHostToDevice));
  // DeltaNet recurrent and conv states start from zero for a new sequence (DeltaNetState::new)
  const ms_model_config& c = m->cfg;
  for (const LayerW& Lw : m->L)
    if (Lw.deltanet) {
      MS_CUDA(m->ctx, cudaMemsetAsync(Lw.dn_conv_state, 0, (size_t)dn_conv_dim(c) * std::max(c.ssm_conv - 1, 1) * 4,
                                      m->ctx->stream));
      MS_CUDA(m->ctx, cudaMemsetAsync(Lw.dn_state, 0, (size_t)c.ssm_dt_rank * c.ssm_state * dn_hvd(c) * 4,
                                      m->ctx->stream));
    }
  m->seq = 0;
  return MS_OK;
}

ms_status ms_model_seq_len(const ms_model* m, int* n) {
  if (!m || !n) return MS_ERR_INVALID_ARG;
  *n = m->seq;
  return MS_OK;
}

ms_status ms_model_forward(ms_model* m, const int32_t* tokens, int n, float* logits) {
  if (!m || !tokens || n <= 0) return MS_ERR_INVALID_ARG;
  if (!m->finalized) return fail(m->ctx, MS_ERR_STATE, "forward before finalize");
  if (m->seq + n > m->cfg.max_seq_len) return fail(m->ctx, MS_ERR_SHAPE, "sequence exceeds max_seq_len");
  cudaSetDevice(m->ctx->device);
  cudaStream_t s = m->ctx->stream;
  MS_CUDA(m->ctx, cudaStreamSynchronize(s));   // pinned staging is reused below
  for (int i = 0; i < n; ++i) {
    if (tokens[i] < 0 || tokens[i] >= m->cfg.vocab) return fail(m->ctx, MS_ERR_INVALID_ARG, "token %d out of range", tokens[i]);
    m->h_tok[i] = tokens[i];
  }
  if (n > 1 && pf_supported(m)) {
    // the whole prompt in batched passes (engine.rs:1869-2006 with seq_len > 1)
    ms_status st = set_feed(m, 0);
    if (st != MS_OK) return st;
    st = pf_forward(m, tokens, n);
    if (st != MS_OK) return st;
    if (logits) MS_CUDA(m->ctx, cudaMemcpyAsync(logits, m->logits, (size_t)m->cfg.vocab * 4, cudaMemcpyDeviceToHost, s));
    return ms_sync(m->ctx);
  }
  ms_status st = set_feed(m, 0);
  if (st != MS_OK) return st;
  for (int i = 0; i < n; ++i) {
    MS_CUDA(m->ctx, cudaMemcpyAsync(&m->st->token_in, &m->h_tok[i], 4, cudaMemcpyHostToDevice, s));
    if (m->sampling) {   // only the last prompt position draws the next token
      st = set_draw(m, i == n - 1);
      if (st != MS_OK) return st;
    }
    st = run_step(m);
    if (st != MS_OK) return st;
  }
  m->seq += n;
  if (logits) MS_CUDA(m->ctx, cudaMemcpyAsync(logits, m->logits, (size_t)m->cfg.vocab * 4, cudaMemcpyDeviceToHost, s));
  return ms_sync(m->ctx);
}

ms_status ms_model_decode_step(ms_model* m, int32_t token, int32_t* next) {
  if (!m || !next) return MS_ERR_INVALID_ARG;
  if (!m->finalized) return fail(m->ctx, MS_ERR_STATE, "decode before finalize");
  if (m->seq + 1 > m->cfg.max_seq_len) return fail(m->ctx, MS_ERR_SHAPE, "sequence exceeds max_seq_len");
  if (token < 0 || token >= m->cfg.vocab) return fail(m->ctx, MS_ERR_INVALID_ARG, "token out of range");
  cudaSetDevice(m->ctx->device);
  cudaStream_t s = m->ctx->stream;
  MS_CUDA(m->ctx, cudaStreamSynchronize(s));
  m->h_tok[0] = token;
  ms_status st = set_feed(m, 0);
  if (st != MS_OK) return st;
  MS_CUDA(m->ctx, cudaMemcpyAsync(&m->st->token_in, &m->h_tok[0], 4, cudaMemcpyHostToDevice, s));
  st = run_step(m);
  if (st != MS_OK) return st;
  MS_CUDA(m->ctx, cudaMemcpyAsync(&m->h_st->key, &m->st->key, 8, cudaMemcpyDeviceToHost, s));
  st = ms_sync(m->ctx);
  if (st != MS_OK) return st;
  m->seq += 1;
  *next = argmax_from_key(m->h_st->key);
  return MS_OK;
}

ms_status ms_model_decode_steps_device(ms_model* m, int n) {
  if (!m || n < 0) return MS_ERR_INVALID_ARG;
  if (!m->finalized) return fail(m->ctx, MS_ERR_STATE, "decode before finalize");
  if (m->seq + n > m->cfg.max_seq_len) return fail(m->ctx, MS_ERR_SHAPE, "sequence exceeds max_seq_len");
  cudaSetDevice(m->ctx->device);
  ms_status st = set_feed(m, 1);
  if (st != MS_OK) return st;
  for (int i = 0; i < n; ++i) {
    st = run_step(m);
    if (st != MS_OK) return st;
  }
  m->seq += n;
  return MS_OK;
}

ms_status ms_model_token_log(ms_model* m, int32_t* out, int max, int* n) {
  if (!m || !out || !n) return MS_ERR_INVALID_ARG;
  MS_CUDA(m->ctx, cudaStreamSynchronize(m->ctx->stream));
  StepState st;
  MS_CUDA(m->ctx, cudaMemcpy(&st, m->st, sizeof st, cudaMemcpyDeviceToHost));
  const int k = std::min(std::min(st.n_log, max), m->cfg.max_seq_len);
  if (k > 0) MS_CUDA(m->ctx, cudaMemcpy(out, m->token_log, (size_t)k * 4, cudaMemcpyDeviceToHost));
  *n = k;
  return MS_OK;
}

ms_status ms_model_generate(ms_model* m, const int32_t* prompt, int n_prompt, int max_new, int32_t* out, int* n_out) {
  if (!m || !prompt || n_prompt <= 0 || max_new <= 0 || !out) return MS_ERR_INVALID_ARG;
  if (n_prompt + max_new - 1 > m->cfg.max_seq_len) return fail(m->ctx, MS_ERR_SHAPE, "sequence exceeds max_seq_len");
  ms_status st = ms_model_clear_cache(m);
  if (st != MS_OK) return st;
  st = ms_model_forward(m, prompt, n_prompt, nullptr);   // prefill (engine.rs:2022-2025)
  if (st != MS_OK) return st;
  st = ms_model_decode_steps_device(m, max_new - 1);      // decode loop (engine.rs:2051-2096)
  if (st != MS_OK) return st;
  MS_CUDA(m->ctx, cudaMemcpyAsync(&m->h_st->key, &m->st->key, 8, cudaMemcpyDeviceToHost, m->ctx->stream));
  st = ms_sync(m->ctx);
  if (st != MS_OK) return st;
  std::vector<int32_t> log(n_prompt + max_new);
  int k = 0;
  st = ms_model_token_log(m, log.data(), (int)log.size(), &k);
  if (st != MS_OK) return st;
  int w = 0;
  for (int i = n_prompt; i < k && w < max_new - 1; ++i) out[w++] = log[i];
  out[w++] = argmax_from_key(m->h_st->key);
  if (n_out) *n_out = w;
  return MS_OK;
}

ms_status ms_model_last_hidden(ms_model* m, float* out) {
  if (!m || !out) return MS_ERR_INVALID_ARG;
  MS_CUDA(m->ctx, cudaStreamSynchronize(m->ctx->stream));
  MS_CUDA(m->ctx, cudaMemcpy(out, m->h_last, (size_t)m->cfg.hidden * 4, cudaMemcpyDeviceToHost));
  return MS_OK;
}

ms_status ms_model_last_routing(ms_model* m, int layer, int32_t* idx, float* wts) {
  if (!m || !idx || !wts || layer < 0 || layer >= m->cfg.layers) return MS_ERR_INVALID_ARG;
  MS_CUDA(m->ctx, cudaStreamSynchronize(m->ctx->stream));
  MS_CUDA(m->ctx, cudaMemcpy(idx, m->L[layer].idx, (size_t)m->cfg.top_k * 4, cudaMemcpyDeviceToHost));
  MS_CUDA(m->ctx, cudaMemcpy(wts, m->L[layer].wts, (size_t)m->cfg.top_k * 4, cudaMemcpyDeviceToHost));
  return MS_OK;
}

ms_status ms_model_set_exact(ms_model* m, int enable) {
  if (!m) return MS_ERR_INVALID_ARG;
  if (!enable && m->tier_slots > 0)
    return fail(m->ctx, MS_ERR_STATE, "host-tier experts run on the order-independent kernels only");
  cudaSetDevice(m->ctx->device);
  MS_CUDA(m->ctx, cudaStreamSynchronize(m->ctx->stream));
  m->exact = enable != 0;
  if (m->graph) { cudaGraphExecDestroy(m->graph); m->graph = nullptr; }
  if (m->bt && m->bt->graph) { cudaGraphExecDestroy(m->bt->graph); m->bt->graph = nullptr; }
  return MS_OK;
}

ms_status ms_model_set_sampling(ms_model* m, int enable, float temperature, float top_p, float repetition_penalty,
                                uint64_t seed) {
  if (!m) return MS_ERR_INVALID_ARG;
  if (!m->finalized) return fail(m->ctx, MS_ERR_STATE, "sampling before finalize");
  if (enable && (!(temperature >= 0.0f) || !(top_p > 0.0f) || !(repetition_penalty > 0.0f)))
    return fail(m->ctx, MS_ERR_INVALID_ARG, "sampling: temperature >= 0, top_p > 0 and penalty > 0 required");
  cudaSetDevice(m->ctx->device);
  MS_CUDA(m->ctx, cudaStreamSynchronize(m->ctx->stream));
  if (enable && !m->s_counts) {
    ms_status st = m->alloc(&m->s_counts, (size_t)m->cfg.vocab * 4);
    st = st ? st : m->alloc(&m->s_work, (size_t)m->cfg.vocab * 4);
    st = st ? st : m->alloc(&m->s_rng, 16);
    st = st ? st : m->alloc(&m->s_draw, 16);
    if (st != MS_OK) return st;
  }
  if (enable) {
    const unsigned long long rng[2] = {(unsigned long long)seed, 0ull};
    MS_CUDA(m->ctx, cudaMemcpy(m->s_rng, rng, sizeof rng, cudaMemcpyHostToDevice));
    MS_CUDA(m->ctx, cudaMemset(m->s_counts, 0, (size_t)m->cfg.vocab * 4));
    const int one = 1;
    MS_CUDA(m->ctx, cudaMemcpy(m->s_draw, &one, sizeof one, cudaMemcpyHostToDevice));
  }
  m->sampling = enable != 0;
  m->s_temp = temperature; m->s_top_p = top_p; m->s_pen = repetition_penalty;
  if (m->graph) { cudaGraphExecDestroy(m->graph); m->graph = nullptr; }   // recaptured with the sampler
  return MS_OK;
}

ms_status ms_model_set_prefill(ms_model* m, int mode) {
  if (!m || mode < 0 || mode > 2) return MS_ERR_INVALID_ARG;
  m->prefill_mode = mode;
  return MS_OK;
}

ms_status ms_model_set_trace(ms_model* m, int enable) {
  if (!m) return MS_ERR_INVALID_ARG;
  if (!m->finalized) return fail(m->ctx, MS_ERR_STATE, "trace before finalize");
  cudaSetDevice(m->ctx->device);
  if (enable && !m->trace_h) {
    ms_status s = m->alloc(&m->trace_h, (size_t)m->cfg.layers * m->cfg.hidden * 4);
    s = s ? s : m->alloc(&m->trace_logits, (size_t)m->cfg.layers * m->cfg.experts * 4);
    if (s != MS_OK) return s;
  }
  if (m->trace != (enable != 0)) {
    MS_CUDA(m->ctx, cudaStreamSynchronize(m->ctx->stream));
    m->trace = enable != 0;
    if (m->graph) { cudaGraphExecDestroy(m->graph); m->graph = nullptr; }   // re-captured with the copies
  }
  return MS_OK;
}

ms_status ms_model_layer_trace(ms_model* m, float* hidden, float* logits) {
  if (!m || (!hidden && !logits)) return MS_ERR_INVALID_ARG;
  if (!m->trace_h) return fail(m->ctx, MS_ERR_STATE, "enable the trace (ms_model_set_trace) before the step");
  MS_CUDA(m->ctx, cudaStreamSynchronize(m->ctx->stream));
  if (hidden) MS_CUDA(m->ctx, cudaMemcpy(hidden, m->trace_h, (size_t)m->cfg.layers * m->cfg.hidden * 4, cudaMemcpyDeviceToHost));
  if (logits) MS_CUDA(m->ctx, cudaMemcpy(logits, m->trace_logits, (size_t)m->cfg.layers * m->cfg.experts * 4, cudaMemcpyDeviceToHost));
  return MS_OK;
}

ms_status ms_model_last_logits(ms_model* m, float* out) {
  if (!m || !out) return MS_ERR_INVALID_ARG;
  MS_CUDA(m->ctx, cudaStreamSynchronize(m->ctx->stream));
  MS_CUDA(m->ctx, cudaMemcpy(out, m->logits, (size_t)m->cfg.vocab * 4, cudaMemcpyDeviceToHost));
  return MS_OK;
}

ms_status ms_nccl_unique_id(ms_ctx* c, void* out, size_t bytes) {
  if (!c || !out || bytes < sizeof(ncclUniqueId)) return MS_ERR_INVALID_ARG;
  NcclApi* api = nccl_api();
  if (!api) return fail(c, MS_ERR_NCCL, "libnccl.so.2 could not be loaded");
  ncclUniqueId id;
  ncclResult_t r = api->get_unique_id(&id);
  if (r != ncclSuccess) return fail(c, MS_ERR_NCCL, "ncclGetUniqueId: %s", api->error_string(r));
  memcpy(out, &id, sizeof id);
  return MS_OK;
}

ms_status ms_model_init_ep(ms_model* m, const void* unique_id, size_t bytes) {
  if (!m || !unique_id || bytes < sizeof(ncclUniqueId)) return MS_ERR_INVALID_ARG;
  if (m->cfg.ep_size <= 1) return MS_OK;
  if (m->comm) return fail(m->ctx, MS_ERR_STATE, "expert-parallel group already initialised");
  NcclApi* api = nccl_api();
  if (!api) return fail(m->ctx, MS_ERR_NCCL, "libnccl.so.2 could not be loaded");
  cudaSetDevice(m->ctx->device);
  ncclUniqueId id;
  memcpy(&id, unique_id, sizeof id);
  ncclResult_t r = api->comm_init_rank(&m->comm, m->cfg.ep_size, id, m->cfg.ep_rank);
  if (r != ncclSuccess) { m->comm = nullptr; return fail(m->ctx, MS_ERR_NCCL, "ncclCommInitRank: %s", api->error_string(r)); }
  if (m->graph) { cudaGraphExecDestroy(m->graph); m->graph = nullptr; }
  return MS_OK;
}

ms_status ms_model_ep_handle(ms_model* m, void* out, size_t bytes) {
  if (!m || !out || bytes < sizeof(cudaIpcMemHandle_t)) return MS_ERR_INVALID_ARG;
  if (!m->finalized || m->cfg.ep_size <= 1) return fail(m->ctx, MS_ERR_STATE, "needs a finalized expert-parallel model");
  if (m->cfg.ep_size > kMaxEp) return fail(m->ctx, MS_ERR_INVALID_ARG, "peer-memory exchange supports <= %d ranks", kMaxEp);
  cudaSetDevice(m->ctx->device);
  if (!m->ep_mail) {
    const size_t mb = (size_t)2 * ep_rows(m) * m->cfg.hidden * 4 + (size_t)2 * m->cfg.ep_size * 4;
    ms_status s = m->alloc(&m->ep_mail, mb);
    s = s ? s : m->alloc(&m->ep_seq, 16);
    s = s ? s : m->alloc(&m->ep_cnt, 16);
    if (s != MS_OK) return s;
    MS_CUDA(m->ctx, cudaDeviceSynchronize());
  }
  cudaIpcMemHandle_t h;
  MS_CUDA(m->ctx, cudaIpcGetMemHandle(&h, m->ep_mail));
  memcpy(out, &h, sizeof h);
  return MS_OK;
}

ms_status ms_model_ep_connect(ms_model* m, const void* handles, size_t bytes) {
  if (!m || !handles) return MS_ERR_INVALID_ARG;
  const int n = m->cfg.ep_size;
  if (!m->ep_mail) return fail(m->ctx, MS_ERR_STATE, "call ms_model_ep_handle first");
  if (bytes < (size_t)n * sizeof(cudaIpcMemHandle_t)) return MS_ERR_INVALID_ARG;
  if (m->ep_p2p) return fail(m->ctx, MS_ERR_STATE, "peer mailboxes already connected");
  cudaSetDevice(m->ctx->device);
  for (int j = 0; j < n; ++j) {
    if (j == m->cfg.ep_rank) continue;
    cudaIpcMemHandle_t h;
    memcpy(&h, static_cast<const uint8_t*>(handles) + (size_t)j * sizeof h, sizeof h);
    void* p = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      for (int q = 0; q < j; ++q)
        if (m->ep_peer[q]) { cudaIpcCloseMemHandle(m->ep_peer[q]); m->ep_peer[q] = nullptr; }
      return cuda_fail(m->ctx, e, "cudaIpcOpenMemHandle (peer mailbox)");
    }
    m->ep_peer[j] = p;
  }
  m->ep_p2p = true;
  if (m->graph) { cudaGraphExecDestroy(m->graph); m->graph = nullptr; }
  return MS_OK;
}

ms_status ms_model_profile_step(ms_model* m, float* us, int max, int* n) {
  if (!m || !us || !n || max <= 0) return MS_ERR_INVALID_ARG;
  if (!m->finalized || m->kernels_per_step <= 0)
    return fail(m->ctx, MS_ERR_STATE, "profile after finalize and at least one decode step");
  if (m->cfg.ep_size > 1) return fail(m->ctx, MS_ERR_STATE, "profiling is single-device only");
  if (m->tier_slots > 0) return fail(m->ctx, MS_ERR_STATE, "per-class profiling needs HBM-resident experts");
  if (is_hybrid(m->cfg) || m->sh_max > 0)   // the launch classes assume one launch pattern per layer
    return fail(m->ctx, MS_ERR_STATE, "per-class profiling covers uniform layer stacks (no DeltaNet / shared expert)");
  cudaSetDevice(m->ctx->device);
  cudaStream_t s = m->ctx->stream, cs = m->ctx->own;
  // a pass that launches nothing, so the launch layout (head_start) is the current mode's
  m->prof_class = 1 << 30;
  ms_status st0 = enqueue_step(m, cs);
  m->prof_class = -1;
  if (st0 != MS_OK) return st0;
  const int n_class = 2 + (m->head_start - 1) / m->cfg.layers;
  constexpr int kWarm = 3, kRuns = 10;
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  MS_CUDA(m->ctx, cudaEventCreate(&e0));
  MS_CUDA(m->ctx, cudaEventCreate(&e1));
  ms_status st = MS_OK;
  int k = 0;
  for (int c = 0; c < n_class && k < max && st == MS_OK; ++c) {
    // a graph holding only this class's launches of one step, chained with PDL like the real step
    cudaGraph_t g = nullptr;
    cudaGraphExec_t ge = nullptr;
    st = ms_sync(m->ctx);
    if (st != MS_OK) break;
    MS_CUDA(m->ctx, cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal));
    m->prof_class = c;
    st = enqueue_step(m, cs);
    m->prof_class = -1;
    cudaError_t e = cudaStreamEndCapture(cs, &g);
    if (st == MS_OK && e != cudaSuccess) st = cuda_fail(m->ctx, e, "cudaStreamEndCapture (profile)");
    if (st == MS_OK && (e = cudaGraphInstantiate(&ge, g, 0)) != cudaSuccess)
      st = cuda_fail(m->ctx, e, "cudaGraphInstantiate (profile)");
    for (int r = 0; r < kWarm + kRuns && st == MS_OK; ++r) {
      if (r == kWarm) cudaEventRecord(e0, s);
      if ((e = cudaGraphLaunch(ge, s)) != cudaSuccess) st = cuda_fail(m->ctx, e, "cudaGraphLaunch (profile)");
    }
    if (st == MS_OK) {
      cudaEventRecord(e1, s);
      st = ms_sync(m->ctx);
    }
    if (st == MS_OK) {
      float ms = 0.f;
      cudaEventElapsedTime(&ms, e0, e1);
      us[k++] = ms * 1000.f / kRuns;
    }
    if (ge) cudaGraphExecDestroy(ge);
    if (g) cudaGraphDestroy(g);
  }
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  *n = k;
  return st;
}

ms_status ms_model_set_expert_tier(ms_model* m, int slots) {
  if (!m || slots < 0) return MS_ERR_INVALID_ARG;
  const ms_model_config& c = m->cfg;
  if (m->finalized) return fail(m->ctx, MS_ERR_STATE, "expert tier after finalize");
  for (const LayerW& Lw : m->L)
    if (Lw.have_gate || Lw.have_up || Lw.have_down)
      return fail(m->ctx, MS_ERR_STATE, "expert tier must be chosen before the expert tensors are set");
  if (slots == 0) { m->tier_slots = 0; m->tier.clear(); return MS_OK; }
  if (c.ep_size > 1) return fail(m->ctx, MS_ERR_STATE, "host-tier experts run on one GPU (ep_size 1)");
  if (slots < c.top_k) return fail(m->ctx, MS_ERR_INVALID_ARG, "expert slots %d < top_k %d", slots, c.top_k);
  m->tier_slots = std::min(slots, m->n_local);
  m->tier.assign(c.layers, ms_model::TierLayer{});
  return MS_OK;
}

ms_status ms_model_set_dynamic_k(ms_model* m, int enable, int k_min, int k_max, int layer_adaptive) {
  if (!m) return MS_ERR_INVALID_ARG;
  const ms_model_config& c = m->cfg;
  if (!m->finalized) return fail(m->ctx, MS_ERR_STATE, "dynamic K after finalize");
  if (enable && (k_min < 1 || k_max < k_min || k_max > c.top_k))
    return fail(m->ctx, MS_ERR_INVALID_ARG, "dynamic K range [%d, %d] must lie in [1, top_k %d]", k_min, k_max, c.top_k);
  if (enable && m->bt) return fail(m->ctx, MS_ERR_STATE, "dynamic K with an open batch");
  MS_CUDA(m->ctx, cudaStreamSynchronize(m->ctx->stream));
  m->dyn_k = enable != 0;
  // LayerTierConfig::default_for_k (config.rs:86-106) and get_layer_k_range (config.rs:473-483)
  const int two_thirds = std::min(std::max(k_max * 2 / 3, 4), k_max);
  for (int li = 0; li < c.layers; ++li) {
    int lo = k_min, hi = k_max;
    if (layer_adaptive) {
      const float depth = (float)li / (float)c.layers;
      if (depth < 0.15f) { lo = k_max; hi = k_max; }
      else if (depth < 0.85f) { lo = std::min(4, k_max); hi = two_thirds; }
      else { lo = two_thirds; hi = k_max; }
    }
    m->L[li].dk_lo = enable ? lo : 0;
    m->L[li].dk_hi = enable ? hi : 0;
  }
  if (m->graph) { cudaGraphExecDestroy(m->graph); m->graph = nullptr; }
  return MS_OK;
}

ms_status ms_model_set_router_stats(ms_model* m, int enable) {
  if (!m) return MS_ERR_INVALID_ARG;
  if (!m->finalized) return fail(m->ctx, MS_ERR_STATE, "router statistics after finalize");
  if (enable && m->bt) return fail(m->ctx, MS_ERR_STATE, "router statistics with an open batch");
  MS_CUDA(m->ctx, cudaStreamSynchronize(m->ctx->stream));
  m->router_stats = enable != 0;
  if (enable) {   // the running totals start from zero
    const ms_model_config& c = m->cfg;
    cudaStream_t s = m->ctx->stream;
    MS_CUDA(m->ctx, cudaMemsetAsync(m->st_cnt, 0, (size_t)c.layers * c.experts * 8, s));
    MS_CUDA(m->ctx, cudaMemsetAsync(m->st_wsum, 0, (size_t)c.layers * c.experts * 8, s));
    MS_CUDA(m->ctx, cudaMemsetAsync(m->st_tok, 0, (size_t)c.layers * 8, s));
    MS_CUDA(m->ctx, cudaMemsetAsync(m->st_n, 0, (size_t)c.layers * 4, s));
  }
  if (m->graph) { cudaGraphExecDestroy(m->graph); m->graph = nullptr; }
  return MS_OK;
}

ms_status ms_model_router_totals(ms_model* m, uint64_t* counts, double* weight_sums, uint64_t* tokens,
                                 float* entropy_log, int max_steps, int* n_steps) {
  if (!m) return MS_ERR_INVALID_ARG;
  if (!m->router_stats) return fail(m->ctx, MS_ERR_STATE, "router statistics are off");
  const ms_model_config& c = m->cfg;
  cudaStream_t s = m->ctx->stream;
  const size_t le = (size_t)c.layers * c.experts;
  if (counts) MS_CUDA(m->ctx, cudaMemcpyAsync(counts, m->st_cnt, le * 8, cudaMemcpyDeviceToHost, s));
  if (weight_sums) MS_CUDA(m->ctx, cudaMemcpyAsync(weight_sums, m->st_wsum, le * 8, cudaMemcpyDeviceToHost, s));
  if (tokens) MS_CUDA(m->ctx, cudaMemcpyAsync(tokens, m->st_tok, (size_t)c.layers * 8, cudaMemcpyDeviceToHost, s));
  uint32_t n = 0;
  MS_CUDA(m->ctx, cudaMemcpyAsync(&n, m->st_n, 4, cudaMemcpyDeviceToHost, s));
  ms_status st = ms_sync(m->ctx);
  if (st != MS_OK) return st;
  const int rows = entropy_log ? std::min((int)n, std::max(max_steps, 0)) : 0;
  if (rows > 0) {
    MS_CUDA(m->ctx, cudaMemcpyAsync(entropy_log, m->st_log, (size_t)rows * c.layers * 4, cudaMemcpyDeviceToHost, s));
    st = ms_sync(m->ctx);
    if (st != MS_OK) return st;
  }
  if (n_steps) *n_steps = (int)n;
  return MS_OK;
}

ms_status ms_model_router_stats(ms_model* m, float* entropy, int32_t* k) {
  if (!m || (!entropy && !k)) return MS_ERR_INVALID_ARG;
  if (!m->router_stats && !m->dyn_k) return fail(m->ctx, MS_ERR_STATE, "router statistics are off");
  cudaStream_t s = m->ctx->stream;
  if (entropy) MS_CUDA(m->ctx, cudaMemcpyAsync(entropy, m->r_entropy, (size_t)m->cfg.layers * 4, cudaMemcpyDeviceToHost, s));
  if (k) MS_CUDA(m->ctx, cudaMemcpyAsync(k, m->r_k, (size_t)m->cfg.layers * 4, cudaMemcpyDeviceToHost, s));
  return ms_sync(m->ctx);
}

ms_status ms_model_expert_tier_stats(const ms_model* m, uint64_t* hits, uint64_t* misses) {
  if (!m || !hits || !misses) return MS_ERR_INVALID_ARG;
  *hits = m->tier_hits;
  *misses = m->tier_misses;
  return MS_OK;
}

static ms_status open_gguf(ms_ctx* c, const char* path, int max_seq_len, int ep_rank, int ep_size, int expert_slots,
                           ms_model** out);

ms_status ms_model_open_gguf(ms_ctx* c, const char* path, int max_seq_len, int ep_rank, int ep_size, ms_model** out) {
  return open_gguf(c, path, max_seq_len, ep_rank, ep_size, 0, out);
}

ms_status ms_model_open_gguf_tiered(ms_ctx* c, const char* path, int max_seq_len, int expert_slots, ms_model** out) {
  if (expert_slots <= 0) return MS_ERR_INVALID_ARG;
  return open_gguf(c, path, max_seq_len, 0, 1, expert_slots, out);
}

static ms_status open_gguf(ms_ctx* c, const char* path, int max_seq_len, int ep_rank, int ep_size, int expert_slots,
                           ms_model** out) {
  if (!c || !path || !out || max_seq_len <= 0) return MS_ERR_INVALID_ARG;
  *out = nullptr;
  int fd = ::open(path, O_RDONLY);
  if (fd < 0) return fail(c, MS_ERR_IO, "cannot open %s", path);
  struct stat sb;
  fstat(fd, &sb);
  const size_t size = (size_t)sb.st_size;
  void* map = mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
  ::close(fd);
  if (map == MAP_FAILED) return fail(c, MS_ERR_IO, "mmap failed");
  struct Unmap { void* p; size_t n; ~Unmap() { munmap(p, n); } } um{map, size};
  GgufParser P{(const uint8_t*)map, size};
  if (P.rd<uint32_t>() != 0x46554747u) return fail(c, MS_ERR_FORMAT, "invalid GGUF magic");
  const uint32_t ver = P.rd<uint32_t>();
  if (ver < 2 || ver > 3) return fail(c, MS_ERR_FORMAT, "unsupported GGUF version %u", ver);
  const uint64_t nt = P.rd<uint64_t>(), nm = P.rd<uint64_t>();
  if (nt > 1000000 || nm > 1000000) return fail(c, MS_ERR_FORMAT, "absurd tensor/metadata counts");
  std::map<std::string, GgufMeta> meta;
  for (uint64_t i = 0; i < nm && P.ok; ++i) {
    std::string k = P.str();
    GgufMeta v;
    P.val((int)P.rd<uint32_t>(), &v);
    meta[k] = v;
  }
  std::vector<std::pair<std::string, GgufT>> ts;
  for (uint64_t i = 0; i < nt && P.ok; ++i) {
    std::string name = P.str();
    const uint32_t nd = P.rd<uint32_t>();
    if (nd > 8) return fail(c, MS_ERR_FORMAT, "tensor %s: too many dims", name.c_str());
    GgufT t;
    std::vector<uint64_t> g(nd);
    for (uint32_t j = 0; j < nd; ++j) g[j] = P.rd<uint64_t>();
    for (int j = (int)nd - 1; j >= 0; --j) t.shape.push_back((int64_t)g[j]);   // TensorInfo::pt_shape
    t.q = (int)P.rd<uint32_t>();
    t.off = P.rd<uint64_t>();
    int64_t n = 1;
    for (auto x : t.shape) n *= x;
    t.nbytes = raw_bytes(t.q, n);
    ts.push_back({name, t});
  }
  if (!P.ok) return fail(c, MS_ERR_FORMAT, "truncated GGUF header");
  uint64_t align = 32;
  auto ai = meta.find("general.alignment");
  if (ai != meta.end() && ai->second.i > 0) align = (uint64_t)ai->second.i;
  const uint64_t start = (P.pos + align - 1) / align * align;
  auto gi = [&](const std::string& k, int64_t d) { auto it = meta.find(k); return it == meta.end() ? d : it->second.i; };
  auto gf = [&](const std::string& k, double d) {
    auto it = meta.find(k);
    if (it == meta.end()) return d;
    return (it->second.type == 6 || it->second.type == 12) ? it->second.f : (double)it->second.i;
  };
  auto gs = [&](const std::string& k, const std::string& d) { auto it = meta.find(k); return it == meta.end() ? d : it->second.s; };
  std::map<std::string, GgufT> tm(ts.begin(), ts.end());
  // config.rs:253-434 keys and defaults
  const std::string a = gs("general.architecture", "qwen2moe");
  ms_model_config cfg{};
  // config.rs:318-352: SSM tensors make a DeltaNet hybrid, every 4th layer attention unless the
  // file says otherwise; DeltaNet shape keys with the reference's defaults
  const bool has_ssm = tm.count("blk.0.ssm_a") || tm.count("blk.0.ssm_conv1d.weight");
  cfg.attn_interval = (int)gi(a + ".attention.full_attention_interval", has_ssm ? 4 : 0);
  cfg.ssm_groups = (int)gi(a + ".ssm.group_count", 16);
  cfg.ssm_state = (int)gi(a + ".ssm.state_size", 128);
  cfg.ssm_dt_rank = (int)gi(a + ".ssm.time_step_rank", gi(a + ".ssm.dt_rank", 32));
  cfg.ssm_inner = (int)gi(a + ".ssm.inner_size", 4096);
  cfg.ssm_conv = (int)gi(a + ".ssm.conv_kernel", 4);
  cfg.arch = a == "gpt-oss" ? MS_ARCH_GPT_OSS : MS_ARCH_QWEN_MOE;
  cfg.hidden = (int)gi(a + ".embedding_length", 2048);
  cfg.layers = (int)gi(a + ".block_count", 48);
  cfg.heads = (int)gi(a + ".attention.head_count", 16);
  cfg.kv_heads = (int)gi(a + ".attention.head_count_kv", 2);
  cfg.head_dim = (int)gi(a + ".attention.key_length", cfg.hidden / cfg.heads);
  cfg.experts = (int)gi(a + ".expert_count", 128);
  cfg.top_k = (int)gi(a + ".expert_used_count", 8);
  cfg.rope_theta = (float)gf(a + ".rope.freq_base", 1000000.0);
  cfg.eps = (float)gf(a + ".attention.layer_norm_rms_epsilon", 1e-6);
  auto te = tm.find("token_embd.weight");
  cfg.vocab = (int)gi(a + ".vocab_size", te != tm.end() ? te->second.shape[0] : 151936);
  auto ge = tm.find("blk.0.ffn_gate_exps.weight");
  cfg.inter = (int)gi(a + ".expert_feed_forward_length", ge != tm.end() && ge->second.shape.size() >= 3 ? ge->second.shape[1] : 768);
  cfg.sliding_window = (int)gi(a + ".attention.sliding_window", 0);
  double prf = gf(a + ".rope.partial_rotary_factor", -1.0);
  if (prf < 0) {
    const int64_t dc = gi(a + ".rope.dimension_count", -1);
    prf = dc >= 0 ? (double)((float)dc / (float)cfg.head_dim) : 1.0;
  }
  cfg.rot_dim = (int)((float)cfg.head_dim * (float)prf);
  const std::string name = gs("general.name", "");
  cfg.norm_topk_prob = !(name.find("Qwen1.5") != std::string::npos || name.find("Qwen2") != std::string::npos);
  cfg.max_seq_len = max_seq_len;
  cfg.ep_rank = ep_rank;
  cfg.ep_size = ep_size;
  ms_model* m = nullptr;
  ms_status s = ms_model_create(c, &cfg, &m);
  if (s != MS_OK) return s;
  if (expert_slots > 0 && (s = ms_model_set_expert_tier(m, expert_slots)) != MS_OK) { ms_model_destroy(m); return s; }
  for (auto& kv : ts) {
    const GgufT& t = kv.second;
    if (t.nbytes < 0) continue;   // types outside the decode path are not indexed
    if (start + t.off + (uint64_t)t.nbytes > size) { ms_model_destroy(m); return fail(c, MS_ERR_FORMAT, "%s: out of bounds", kv.first.c_str()); }
    s = ms_model_set_tensor(m, kv.first.c_str(), t.q, (int)t.shape.size(), t.shape.data(),
                            (const uint8_t*)map + start + t.off, (size_t)t.nbytes);
    if (s != MS_OK) { ms_model_destroy(m); return s; }
  }
  s = ms_model_finalize(m);
  if (s != MS_OK) { ms_model_destroy(m); return s; }
  *out = m;
  return MS_OK;
}

}  // extern "C"

// =====================================================================================
// Allocation-free variant of ms_moe_mxfp4_decode.
//
// Some callers cannot allocate device memory at the time they run the MoE step: a
// caller that has handed its whole memory budget to a fixed-size pool, a real-time
// loop that must not enter the CUDA allocator, or a host that replays the step from
// a context where cudaMalloc is forbidden.  For them this entry point keeps the FFN's
// scratch (per-slot activations and per-slot partial outputs) in one file-scope device array instead of context-owned cudaMalloc'd
// memory.  Every GPU that loads this library holds the array until the process exits.
// =====================================================================================
namespace {

constexpr int kNoAllocMaxTopK = 16;      // experts per token
constexpr int kNoAllocMaxDim = 4096;     // max hidden size and max expert intermediate size
constexpr size_t kNoAllocActFloats = (size_t)kNoAllocMaxTopK * kNoAllocMaxDim;
constexpr size_t kNoAllocPartFloats = (size_t)kNoAllocMaxTopK * kNoAllocMaxDim;
constexpr size_t kNoAllocFloats = kNoAllocActFloats + kNoAllocPartFloats;

// act [K*I] | partial [K*H]: 512 KiB per device.  Both slices are fully written by the
// kernels of each call before they are read, so no clearing is needed between calls.
static __device__ __align__(256) float g_moe_noalloc_scratch[kNoAllocFloats];

constexpr int kNoAllocMaxDevices = 64;
float* g_noalloc_addr[kNoAllocMaxDevices] = {};
std::mutex g_noalloc_mu;

// once per device, with that device current: the device address of the array (the
// array's name in host code is only a host-side stand-in and must not reach a kernel).
// The cached address belongs to the device's primary context: after a cudaDeviceReset in
// the same process it is stale, so the entry point must not be used across a reset.
ms_status noalloc_setup(ms_ctx* c, float** out) {
  if (c->device < 0 || c->device >= kNoAllocMaxDevices) return fail(c, MS_ERR_INVALID_ARG, "device index too large");
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_addr[c->device]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_moe_noalloc_scratch);
    if (e != cudaSuccess || !p) return cuda_fail(c, e == cudaSuccess ? cudaErrorInvalidSymbol : e, "cudaGetSymbolAddress");
    g_noalloc_addr[c->device] = (float*)p;
  }
  *out = g_noalloc_addr[c->device];
  return MS_OK;
}

}  // namespace

extern "C" ms_status ms_moe_mxfp4_decode_noalloc(ms_ctx* c, const void* gate, const void* up, const void* down,
                                                 const float* gb, const float* ub, const float* db, int H, int I,
                                                 int E, int K, int arch, const float* x, const int32_t* idx,
                                                 const float* wts, float* h) {
  if (!c || !gate || !up || !down || !x || !idx || !wts || !h || K <= 0 || E <= 0) return MS_ERR_INVALID_ARG;
  if (H <= 0 || I <= 0) return fail(c, MS_ERR_SHAPE, "moe noalloc: hidden and inter must be positive");
  if (K > kNoAllocMaxTopK || H > kNoAllocMaxDim || I > kNoAllocMaxDim)
    return fail(c, MS_ERR_SHAPE, "moe noalloc: top_k %d / hidden %d / inter %d exceed the fixed scratch "
                "(top_k <= %d, hidden <= %d, inter <= %d)", K, H, I, kNoAllocMaxTopK, kNoAllocMaxDim, kNoAllocMaxDim);
  if (H % 64 || I % 32) return fail(c, MS_ERR_SHAPE, "moe: hidden %% 64 and inter %% 32 required");
  // the caller's current device is restored on return
  int prev = -1;
  cudaError_t e = cudaGetDevice(&prev);
  if (e != cudaSuccess) return cuda_fail(c, e, "cudaGetDevice");
  struct Restore { int d; ~Restore() { if (d >= 0) cudaSetDevice(d); } } restore{prev != c->device ? prev : -1};
  e = cudaSetDevice(c->device);
  if (e != cudaSuccess) return cuda_fail(c, e, "cudaSetDevice");
  float* base = nullptr;
  ms_status s = noalloc_setup(c, &base);
  if (s != MS_OK) return s;
  MoeArgs a;
  a.x = x; a.idx = idx; a.wts = wts; a.gate = (const uint8_t*)gate; a.up = (const uint8_t*)up;
  a.down = (const uint8_t*)down; a.gate_b = gb; a.up_b = ub; a.down_b = db;
  a.act = base; a.partial = base + kNoAllocActFloats; a.tile_cnt = nullptr; a.h = h;
  a.H = H; a.I = I; a.K = K; a.expert_base = 0; a.n_local = E; a.oai_swiglu = arch == MS_ARCH_GPT_OSS;
  e = launch_moe_mxfp4(c->dc, a, c->stream);
  if (e != cudaSuccess) return cuda_fail(c, e, "moe_mxfp4 (noalloc)");
  return MS_OK;
}
