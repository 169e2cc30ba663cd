// kernels_moe_tc.cu — MXFP4 expert FFN for decode on the 5th-generation tensor cores (sm_100a).
//
// Reference semantics (moe-stream-core/src): expert FFN with OAI SwiGLU and per-expert biases,
// model/layer.rs:1797-1847 and ops/activation.rs:25-38; MXFP4 values gguf/dequant.rs:580-628
// (weight = e2m1 * 2^(E-127), i.e. the GGUF block's scale byte is the ue8m0 scale as is).
//
// Design.  The expert matrices are repacked once, at upload, into 128-row tiles laid out as the
// tensor core reads them (umma.cuh): a gate_up tile holds 64 gate rows and the 64 up rows of the
// same outputs; a down tile holds 128 rows of the hidden dimension (the last one zero-padded).
// A tile is stored as slabs of up to 8 chunk columns (K = 256), each slab's codes followed by
// its scale groups, so any K range of a tile is two contiguous byte ranges.  The activation is
// the B operand: 16 MXFP4 residual terms (N = 16), made by the producing kernel.  One
// tcgen05.mma.kind::mxf4.block_scale computes a 128 x 16 x 64 block-scaled product with f32
// accumulation in tensor memory; the row result is the sum of the 16 term columns.
//
// Work split.  The routed (slot, tile) items times K/64 MMA steps form one index space cut into
// equal contiguous ranges, one per CTA (split-K), so every SM streams the same number of bytes.
// A CTA writes the 128 per-row partial sums of each item range it covers; the last CTA to finish
// an item adds the partials in range order (deterministic), applies bias and activation (gate_up,
// which also quantizes its 64 activations into the down projection's B terms) or writes the
// per-slot expert output (down).  Warp roles: warp 0 streams stages with 1-D bulk copies, warp 1
// owns tensor memory and issues scale copies + MMAs (one elected thread), warps 2-5 drain the
// accumulators (double-buffered in tensor memory).  Every wait is bounded.
#include <cuda_fp16.h>

#include "common.cuh"
#include "kernels.h"
#include "umma.cuh"

namespace ms {

// Optional timeline (build with -DMS_TRACE): %globaltimer stamps per CTA in g_tc_trace[0][cta][k]:
// 0 entry, 1 slots known, 2 first gate_up copy issued, 3 down activation ready (producer),
// 4 last gate_up MMA committed, 5 last down MMA committed, 6 epilogue done, 7 kernel exit.
#ifdef MS_TRACE
__device__ unsigned long long g_tc_trace[2][1024][8];
#define TC_TRACE2(k)                                                                           \
  do {                                                                                         \
    unsigned long long t_;                                                                     \
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));                                     \
    g_tc_trace[1][blockIdx.x & 1023][(k)] = t_;                                                \
  } while (0)
#define TC_TRACE(k)                                                                            \
  do {                                                                                         \
    unsigned long long t_;                                                                     \
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));                                     \
    g_tc_trace[0][blockIdx.x & 1023][(k)] = t_;                                           \
  } while (0)
#else
#define TC_TRACE(k) ((void)0)
#define TC_TRACE2(k) ((void)0)
#endif

namespace {
// A slab is 16 chunk columns (K = 512, four K-words of 4 chunks); it is also the stage size.
constexpr int kCS = 16;
constexpr int kKW = kCS / 4;                 // K-words per slab
constexpr int kStA = kCS * 2048;             // A codes: 16 chunks x 128 rows x 16 B
constexpr int kStSFA = kKW * 512;            // A scale groups, one per K-word
constexpr int kStB = kCS * 256;              // B codes: 16 chunks x 16 terms x 16 B
constexpr int kStSFB = kKW * 512;            // B scale groups, one per K-word
constexpr int kStageBytes = kStA + kStSFA + kStB + kStSFB;
#ifndef MS_TC_CTAS_PER_SM
#define MS_TC_CTAS_PER_SM 2
#endif
constexpr int kCtasPerSm = MS_TC_CTAS_PER_SM;   // independent copy / MMA / epilogue pipelines per SM
constexpr int kStages = kCtasPerSm == 1 ? 4 : 2;
constexpr int kThreads = 192;
constexpr int kTmemCols = kCtasPerSm == 1 ? 256 : 128;
constexpr int kAccCols = 16;                 // one accumulator: 128 lanes x 16 f32 columns
constexpr int kSubAcc = 2;                   // consecutive MMAs alternate between 2 accumulators
constexpr int kAccSet = kSubAcc * kAccCols;  // columns of one (double-buffered) accumulator set
constexpr int kSlotCols = 8 * kKW;           // per stage: A and B scale groups, 4 columns each
constexpr int kMaxKSlots = 16;
static_assert(2 * kAccSet + kStages * kSlotCols <= kTmemCols, "tensor memory budget");

__host__ __device__ __forceinline__ int64_t slab_off(int s) { return (int64_t)s * (kCS * 2048 + kKW * 512); }
}  // namespace

int64_t tc_tile_bytes(int kc) {
  int64_t b = (int64_t)kc * 2048;
  for (int s = 0; s * kCS < kc; ++s) b += (int64_t)(((kc - s * kCS < kCS ? kc - s * kCS : kCS) + 3) / 4) * 512;
  return b;
}
int64_t tc_bterm_bytes(int kc) { return umma::bterm_bytes(kc); }
int tc_gu_tiles(int I) { return I / 64; }
int tc_down_tiles(int H) { return (H + 127) / 128; }
int tc_cnt_words(int H, int I, int K) { return 2 * tc_max_items(H, I, K) + 16 + 1; }
int tc_max_items(int H, int I, int K) { return K * (tc_gu_tiles(I) > tc_down_tiles(H) ? tc_gu_tiles(I) : tc_down_tiles(H)); }
bool tc_supported(int H, int I) { return H % 64 == 0 && I % 64 == 0; }

namespace {

// ---------------- repack: native GGUF MXFP4 rows -> tensor-core tiles ----------------
// src [E][rows][kc blocks of 17 B]; rows land in tile t = r / tile_rows_src at tile row
// row_off + r % tile_rows_src.  Rows past `rows` are written as zero codes with scale 0.
__global__ void mxfp4_pack_kernel(const uint8_t* __restrict__ src, int E, int rows, int kc, int tile_rows_src,
                                  int row_off, int tiles, uint8_t* __restrict__ dst, int64_t tile_bytes) {
  const int64_t n = (int64_t)E * tiles * tile_rows_src * kc;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int c = (int)(i % kc);
    int64_t q = i / kc;
    const int lr = (int)(q % tile_rows_src);
    q /= tile_rows_src;
    const int t = (int)(q % tiles);
    const int e = (int)(q / tiles);
    const int r = t * tile_rows_src + lr;
    uint32_t w[4] = {0u, 0u, 0u, 0u};
    uint8_t sc = 0;
    if (r < rows) {
      const uint8_t* b = src + ((int64_t)e * rows + r) * kc * 17 + (int64_t)c * 17;
      sc = b[0];
      // native byte j: low nibble = element j, high nibble = element j + 16 (dequant.rs:605-628);
      // packed byte i: element 2i (low nibble), element 2i + 1 (high nibble)
#pragma unroll
      for (int i2 = 0; i2 < 16; ++i2) {
        const uint32_t v = i2 < 8 ? ((b[1 + 2 * i2] & 0xFu) | ((b[2 + 2 * i2] & 0xFu) << 4))
                                  : ((b[1 + 2 * (i2 - 8)] >> 4) | (b[2 + 2 * (i2 - 8)] & 0xF0u));
        w[i2 >> 2] |= v << (8 * (i2 & 3));
      }
    }
    uint8_t* tile = dst + ((int64_t)e * tiles + t) * tile_bytes;
    const int slab = c / kCS, sl0 = slab * kCS, nch = min(kCS, kc - sl0);
    uint8_t* sb = tile + slab_off(slab);
    const int row = row_off + lr;
    *reinterpret_cast<uint4*>(sb + (int64_t)(c - sl0) * 2048 + row * 16) = make_uint4(w[0], w[1], w[2], w[3]);
    sb[(int64_t)nch * 2048 + ((c - sl0) >> 2) * 512 + 16 * (row & 31) + 4 * (row >> 5) + (c & 3)] = sc;
  }
}

// ---------------- x -> B terms (standalone entry points; the model's router does this) ----------------
__global__ void xterms_kernel(const float* __restrict__ x, int H, uint8_t* __restrict__ bt) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  pdl_wait_prior();
  pdl_launch_dependents();   // the next kernel may start its own (weight) prefetch now
  const int nb = H / 32;
  if (warp >= nb) return;
  umma::quantize_terms_warp(x[32 * warp + lane], lane, bt, nb, warp);
}

__device__ __forceinline__ float swiglu_oai_tc(float g, float u) {   // ops/activation.rs:25-45
  const float gc = fminf(g, 7.0f);
  const float uc = fminf(fmaxf(u, -7.0f), 7.0f);
  const float sig = 1.0f / (expf(-(gc * 1.702f)) + 1.0f);
  return (gc * sig) * (uc + 1.0f);
}

enum { TC_GATEUP = 0, TC_DOWN = 1 };

// one projection: packed weight tiles times B terms
struct TcPhase {
  const uint8_t* w;          // packed tiles [E_local][tiles][tile_bytes]
  int64_t tile_bytes;
  int tiles, kc;             // tiles per expert; chunk columns (reduction length / 32)
  const uint8_t* bterm;      // B terms: x (gate_up) or act_terms base (down)
  int64_t bterm_stride;      // per slot (down), 0 (gate_up)
  const float* bias0;        // gate_b (gate_up) / down_b (down)
  const float* bias1;        // up_b
  int rows;                  // rows per expert matrix of the output: I (gate_up) / H (down)
};

struct TcParams {
  TcPhase ph[2];             // [TC_GATEUP], [TC_DOWN]
  const int* idx;
  int K, expert_base, n_local;
  float* part;               // [2][max_items][kTcMaxSeg][128] split-K partials
  uint32_t* cnt;             // [2][max_items] item counters, then act_ready[kMaxK], then done: zeroed, self-resetting
  int max_items;
  float* act;                // [K][I] f32 activations (optional)
  uint8_t* act_terms;        // [K][bterm_bytes(I/32)]
  int oai;
  float* partial;            // [K][H] per-slot expert outputs
  uint32_t* err;
};

// This CTA's stages: its units of gate_up, then of down -- a unit is one of the S equal K ranges
// of an item -- each cut at slab boundaries.
struct Stage {
  int phase, item, seg, w0, w1;   // K-words [w0, w1) of item, within one slab; seg = the unit's range index
  bool seg_start, seg_end;        // first / last stage of the unit
};
struct StageWalk {   // two phases held as scalar pairs (no runtime-indexed arrays: registers only)
  int kw0, kw1, s0, s1, ua, ua1, ub, ub1, phase, item, seg, w, wend;
  __device__ void init(const int (&u0_)[2], const int (&u1_)[2], const int (&kw)[2], const int (&sp)[2]) {
    kw0 = kw[0]; kw1 = kw[1]; s0 = sp[0]; s1 = sp[1];
    ua = u0_[0]; ua1 = u1_[0]; ub = u0_[1]; ub1 = u1_[1];
    phase = 0; item = 0; seg = 0; w = wend = 0;
  }
  __device__ bool next(Stage& st) {
    st.seg_start = false;
    if (w >= wend) {
      if (phase == 0 && ua >= ua1) phase = 1;
      if (phase == 1 && ub >= ub1) return false;
      const int n = phase ? s1 : s0, kw = phase ? kw1 : kw0;
      const int u = phase ? ub : ua;
      item = u / n;
      seg = u - item * n;
      w = seg * kw / n;
      wend = (seg + 1) * kw / n;
      if (phase) ++ub; else ++ua;
      st.seg_start = true;
    }
    st.phase = phase;
    st.item = item;
    st.seg = seg;
    st.w0 = w;
    st.w1 = min(wend, (w / kKW + 1) * kKW);
    w = st.w1;
    st.seg_end = w >= wend;
    return true;
  }
};

__device__ __forceinline__ uint32_t ld_acquire_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// gate_up and down in one persistent launch.  A CTA runs its gate_up range, then its down
// range; the down producer issues each stage's weight copies at once and its activation-term
// copies only after every gate_up tile of that slot is finished (per-slot counter), so down's
// weight streaming overlaps gate_up's tail.  All CTAs are resident together (one per SM), and
// gate_up work waits on nothing but its own copies, so the counters always complete.
__global__ void __launch_bounds__(kThreads, kCtasPerSm) moe_tc_kernel(const __grid_constant__ TcParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ __align__(8) uint64_t full[kStages], empty[kStages], acc_full[2], acc_empty[2];
  __shared__ uint32_t tmem_base;
  __shared__ int s_slot[kMaxKSlots], s_exp[kMaxKSlots], s_n, s_last, s_abort;
  __shared__ float s_rows[128];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint32_t* act_ready = p.cnt + 2 * p.max_items;       // [kMaxKSlots]
  uint32_t* done = act_ready + kMaxKSlots;

  // barriers and tensor memory do not depend on the previous kernel: set them up before its wait
  if (threadIdx.x == 0) {
    TC_TRACE(0);
    for (int s = 0; s < kStages; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
    for (int a = 0; a < 2; ++a) { mbar_init(&acc_full[a], 1); mbar_init(&acc_empty[a], 128); }
    fence_mbar_init();
  }
  if (warp == 1) { umma::tmem_alloc(&tmem_base, kTmemCols); umma::tmem_relinquish(); }
  pdl_wait_prior();
  pdl_launch_dependents();   // the next kernel may start its own (weight) prefetch now
  if (threadIdx.x == 0) {
    // local slots in ascending expert order (layer.rs:1092-1106)
    int n = 0;
    for (int k = 0; k < p.K; ++k) {
      const int e = p.idx[k] - p.expert_base;
      if (e < 0 || e >= p.n_local) {
        if (p.n_local == 0 || p.idx[k] < 0) atomicOr(p.err, EF_BAD_INDEX);
        continue;
      }
      int j = n++;
      while (j > 0 && s_exp[j - 1] > e) { s_exp[j] = s_exp[j - 1]; s_slot[j] = s_slot[j - 1]; --j; }
      s_exp[j] = e;
      s_slot[j] = k;
    }
    s_n = n;
    s_abort = 0;
  }
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t tb = tmem_base;
  if (threadIdx.x == 0) TC_TRACE(1);
  int KW[2], S[2], u0[2], u1[2];
  for (int q = 0; q < 2; ++q) {
    KW[q] = (p.ph[q].kc + 3) / 4;                            // K-words per item (the last may hold 2 chunks)
    const int n_items = s_n * p.ph[q].tiles;
    S[q] = tc_splits(n_items, KW[q], (int)gridDim.x);
    const int U = n_items * S[q], G = min((int)gridDim.x, U);
    const bool on = U > 0 && (int)blockIdx.x < G;
    u0[q] = on ? (int)((int64_t)blockIdx.x * U / G) : 0;
    u1[q] = on ? (int)((int64_t)(blockIdx.x + 1) * U / G) : 0;
  }

  if (warp == 0) {
    // ---------------- producer ----------------
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      StageWalk it;
      it.init(u0, u1, KW, S);
      Stage st;
      int j = 0, ready_slot = -1;
      while (!*reinterpret_cast<volatile int*>(&s_abort) && it.next(st)) {
        const TcPhase& ph = p.ph[st.phase];
        const int ls = st.item / ph.tiles, t = st.item % ph.tiles;
        const uint8_t* tile = ph.w + ((int64_t)s_exp[ls] * ph.tiles + t) * ph.tile_bytes;
        const uint8_t* bt = ph.bterm + (int64_t)s_slot[ls] * ph.bterm_stride;
        const int slab = st.w0 / kKW, c0 = 4 * st.w0, c1 = min(ph.kc, 4 * st.w1), sl0 = slab * kCS;
        const int nch = min(kCS, ph.kc - sl0);
        const int s = j % kStages, n = j / kStages;
        if (n > 0 && !mbar_wait(&empty[s], (uint32_t)((n - 1) & 1), p.err, EF_TIMEOUT_EMPTY)) { s_abort = 1; break; }
        uint8_t* sp = smem + (size_t)s * kStageBytes;
        const uint32_t ab = (uint32_t)(c1 - c0) * 2048u, bb = (uint32_t)(c1 - c0) * 256u;
        const uint32_t gb = (uint32_t)(st.w1 - st.w0) * 512u;
        mbar_expect_tx(&full[s], ab + 2 * gb + bb);
        const uint8_t* sb = tile + slab_off(slab);
        bulk_g2s_stream(sp, sb + (int64_t)(c0 - sl0) * 2048, ab, &full[s], pol);
        bulk_g2s_stream(sp + kStA, sb + (int64_t)nch * 2048 + (st.w0 - slab * kKW) * 512, gb, &full[s], pol);
        if (st.phase == TC_DOWN && ready_slot != s_slot[ls]) {
          // this slot's activation terms are complete once all its gate_up tiles are finished
          const uint32_t target = (uint32_t)p.ph[TC_GATEUP].tiles;
          uint32_t it2 = 0;
          while (ld_acquire_u32(&act_ready[s_slot[ls]]) < target && ++it2 < kWaitLimit) __nanosleep(32);
          if (it2 >= kWaitLimit) { atomicOr(p.err, EF_TIMEOUT_FULL); s_abort = 1; }
          asm volatile("fence.proxy.async.global;" ::: "memory");   // generic-proxy writes -> bulk-copy reads
          ready_slot = s_slot[ls];
          TC_TRACE(3);
        }
        bulk_g2s(sp + kStA + kStSFA, bt + (int64_t)c0 * 256, bb, &full[s]);
        bulk_g2s(sp + kStA + kStSFA + kStB, bt + (int64_t)ph.kc * 256 + (int64_t)st.w0 * 512, gb, &full[s]);
        if (j == 0) TC_TRACE(2);
        ++j;
      }
      // no copy may still be landing in shared memory when the CTA exits
      for (int q = max(0, j - kStages); q < j; ++q)
        mbar_wait(&full[q % kStages], (uint32_t)((q / kStages) & 1), p.err, EF_TIMEOUT_FULL);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      StageWalk it;
      it.init(u0, u1, KW, S);
      Stage st;
      int j = 0, seg = 0, nmma = 0;
      while (!*reinterpret_cast<volatile int*>(&s_abort) && it.next(st)) {
        const int kc = p.ph[st.phase].kc;
        const int a = seg & 1;
        if (st.seg_start) {
          if (seg >= 2 && !mbar_wait(&acc_empty[a], (uint32_t)(((seg >> 1) - 1) & 1), p.err, EF_TIMEOUT_EMPTY)) {
            s_abort = 1;
            break;
          }
          nmma = 0;
        }
        const int s = j % kStages;
        if (!mbar_wait(&full[s], (uint32_t)((j / kStages) & 1), p.err, EF_TIMEOUT_FULL)) { s_abort = 1; break; }
        umma::fence_after_sync();
        const uint8_t* sp = smem + (size_t)s * kStageBytes;
        const uint32_t sfa_col = tb + (uint32_t)(2 * kAccSet + s * kSlotCols), sfb_col = sfa_col + 4 * kKW;
        const int nw = st.w1 - st.w0;
        for (int g = 0; g < nw; ++g) {
          umma::cp_sf_group(sfa_col + 4 * g, sp + kStA + g * 512);
          umma::cp_sf_group(sfb_col + 4 * g, sp + kStA + kStSFA + kStB + g * 512);
        }
        const uint32_t d_tmem = tb + (uint32_t)(a * kAccSet);
        const int c0 = 4 * st.w0, c1 = min(kc, 4 * st.w1);
        for (int cc = c0; cc < c1; cc += 2) {
          const uint64_t ad = umma::smem_desc(sp + (cc - c0) * 2048, 2048, 128);
          const uint64_t bd = umma::smem_desc(sp + kStA + kStSFA + (cc - c0) * 256, 256, 128);
          const int wl = (cc >> 2) - st.w0;            // K-word within the stage
          const uint32_t byte = (uint32_t)(cc & 3);    // the pair of blocks within the K-word
          umma::mma_mxf4(d_tmem + (uint32_t)((nmma % kSubAcc) * kAccCols), ad, bd,
                         umma::idesc_mxf4(128, 16, byte, byte), sfa_col + 4 * wl, sfb_col + 4 * wl,
                         nmma >= kSubAcc);
          ++nmma;
        }
        umma::commit(&empty[s]);   // the stage may be refilled once these MMAs have read it
        ++j;
        if (st.seg_end) {
          umma::commit(&acc_full[a]);
          TC_TRACE(4 + st.phase);
          ++seg;
        }
      }
    }
  } else {
    // ---------------- epilogue (warps 2-5: TMEM lane quadrants 2, 3, 0, 1) ----------------
    const int quad = warp & 3, row = 32 * quad + lane;
    const int et = threadIdx.x - 64;   // 0..127
    StageWalk it;
    it.init(u0, u1, KW, S);
    Stage st;
    int seg = 0, nmma = 0;
    while (it.next(st)) {
      const TcPhase& ph = p.ph[st.phase];
      if (st.seg_start) nmma = 0;
      nmma += (min(ph.kc, 4 * st.w1) - 4 * st.w0 + 1) / 2;
      if (!st.seg_end) continue;
      const int item = st.item, q0 = st.phase;
      const int ls = item / ph.tiles, t = item % ph.tiles;
      const int e = s_exp[ls], slot = s_slot[ls];
      const int nseg = q0 ? S[1] : S[0], segi = st.seg;
      // biases are read before the accumulator wait (they are off the critical path there)
      float b0 = 0.f, b1 = 0.f;
      if (q0 == TC_GATEUP) {
        if (et < 64) {
          if (ph.bias0) b0 = ph.bias0[(int64_t)e * ph.rows + t * 64 + et];
          if (ph.bias1) b1 = ph.bias1[(int64_t)e * ph.rows + t * 64 + et];
        }
      } else if (segi == 0 && ph.bias0 && t * 128 + row < ph.rows) {
        b0 = ph.bias0[(int64_t)e * ph.rows + t * 128 + row];
      }
      const int a = seg & 1;
      const bool ok = mbar_wait(&acc_full[a], (uint32_t)((seg >> 1) & 1), p.err, EF_TIMEOUT_FULL);
      if (et == 0 && q0 == TC_GATEUP) TC_TRACE2(0);
      umma::fence_after_sync();
      float sum = 0.f;
      const int nsub = min(kSubAcc, nmma);
      for (int q = 0; q < nsub; ++q) {
        float v[16];
        umma::ld_32x32b_x16(tb + ((uint32_t)(32 * quad) << 16) + (uint32_t)(a * kAccSet + q * kAccCols), v);
#pragma unroll
        for (int i = 0; i < 16; ++i) sum += v[i];   // term 0 (largest) first
      }
      umma::fence_before_sync();
      mbar_arrive(&acc_empty[a]);
      if (!ok) break;
      if (q0 == TC_DOWN) {
        // per-range partial sums; the consumer of the MoE output adds the ranges in K order
        p.part[(((int64_t)p.max_items + item) * kTcMaxSeg + segi) * 128 + row] = sum + b0;
        ++seg;
        continue;
      }
      // ---- gate_up: the item's 64 gate rows (TMEM rows 0-63) and up rows (64-127) ----
      bool finish = nseg == 1;
      const float* pp = s_rows;
      if (nseg == 1) {
        s_rows[row] = sum;
        named_bar(1, 128);
      } else {   // split item: the last range to finish adds the ranges in order
        const int64_t gitem = item;
        p.part[(gitem * kTcMaxSeg + segi) * 128 + row] = sum;
        named_bar(1, 128);
        if (et == 0) {
          __threadfence();   // this CTA's partials (ordered before by the barrier), then the count
          s_last = (atomicAdd(&p.cnt[gitem], 1u) == (uint32_t)nseg - 1) ? 1 : 0;
          if (s_last) {
            __threadfence();
            p.cnt[gitem] = 0u;
          }
        }
        named_bar(1, 128);
        finish = s_last != 0;
        pp = p.part + gitem * kTcMaxSeg * 128;
      }
      if (et == 0) TC_TRACE2(2);
      if (finish) {
        const int kc_out = p.ph[TC_DOWN].kc;
        if (et < 64) {
          float g = 0.f, up = 0.f;
          if (nseg == 1) { g = pp[et]; up = pp[64 + et]; }
          else for (int q = 0; q < nseg; ++q) { g += __ldcg(pp + q * 128 + et); up += __ldcg(pp + q * 128 + 64 + et); }
          g += b0;
          up += b1;
          const float av = p.oai ? swiglu_oai_tc(g, up) : (g / (1.0f + expf(-g))) * up;
          // this tile's 64 activations are chunk columns 2t, 2t+1 of the down projection's B terms
          umma::quantize_terms_warp(av, lane, p.act_terms + (int64_t)slot * umma::bterm_bytes(kc_out), kc_out,
                                    2 * t + (et >> 5));
          if (p.act) p.act[(int64_t)slot * ph.rows + t * 64 + et] = av;
        }
        if (et == 0) TC_TRACE2(3);
        named_bar(1, 128);
        if (et == 0) {
          __threadfence();   // the tile's activation terms, then the slot's ready count
          atomicAdd(&act_ready[slot], 1u);
          TC_TRACE2(5);
        }
      } else if (nseg == 1) {
        named_bar(1, 128);
      }
      ++seg;
    }
    if (et == 0) TC_TRACE(6);
  }
  umma::fence_before_sync();
  __syncthreads();
  if (warp == 1) umma::tmem_dealloc(tb, kTmemCols);
  if (threadIdx.x == 0) TC_TRACE(7);
  if (threadIdx.x == 0) {
    // the last CTA out clears the per-slot ready counts for the next call (every CTA has read
    // them by now: its producer finished)
    __threadfence();
    if (atomicAdd(done, 1u) == gridDim.x - 1) {
      for (int k = 0; k < kMaxKSlots; ++k) act_ready[k] = 0u;
      __threadfence();
      *done = 0u;
    }
  }
}

cudaError_t launch_tc(const DevCtx& c, const TcParams& p, cudaStream_t s) {
  const size_t smem = (size_t)kStages * kStageBytes;
  cudaError_t e = cudaFuncSetAttribute(moe_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(kCtasPerSm * c.sm_count));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, moe_tc_kernel, p);
}

}  // namespace

cudaError_t launch_mxfp4_pack(const uint8_t* src, int E, int rows, int cols, int tile_rows_src, int row_off,
                              int tiles, uint8_t* dst, cudaStream_t s) {
  if (cols % 64 || E <= 0 || rows <= 0 || tiles <= 0) return cudaErrorInvalidValue;
  const int kc = cols / 32;
  const int64_t n = (int64_t)E * tiles * tile_rows_src * kc;
  const int blocks = (int)((n + 255) / 256 < 65536 ? (n + 255) / 256 : 65536);
  mxfp4_pack_kernel<<<blocks, 256, 0, s>>>(src, E, rows, kc, tile_rows_src, row_off, tiles, dst, tc_tile_bytes(kc));
  return cudaGetLastError();
}

cudaError_t launch_xterms(const DevCtx& c, const float* x, int H, uint8_t* xterm, cudaStream_t s) {
  (void)c;
  const int nb = H / 32, blocks = (nb + 7) / 8;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)blocks);
  cfg.blockDim = dim3(256);
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, xterms_kernel, x, H, xterm);
}

PendingCombine tc_pending_combine(const DevCtx& c, const TcMoeArgs& a) {
  PendingCombine pc;
  pc.seg_part = a.part + (size_t)tc_max_items(a.H, a.I, a.K) * kTcMaxSeg * 128;
  pc.seg_tiles = tc_down_tiles(a.H);
  pc.seg_kw = (a.I / 32 + 3) / 4;                  // the kernel's split, recomputed from the routed slot count
  pc.seg_grid = kCtasPerSm * c.sm_count;

  pc.idx = a.idx; pc.wts = a.wts; pc.K = a.K; pc.expert_base = a.expert_base; pc.n_local = a.n_local;
  return pc;
}

cudaError_t launch_moe_tc(const DevCtx& c, const TcMoeArgs& a, cudaStream_t s) {
  if (a.K < 1 || a.K > kMaxKSlots || !tc_supported(a.H, a.I) || a.n_local < 0) return cudaErrorInvalidValue;
  TcParams p = {};
  p.idx = a.idx; p.K = a.K; p.expert_base = a.expert_base; p.n_local = a.n_local; p.err = c.err;
  p.part = a.part; p.cnt = a.cnt; p.max_items = tc_max_items(a.H, a.I, a.K);
  p.act = a.act; p.act_terms = a.act_terms; p.oai = a.oai_swiglu; p.partial = a.partial;
  TcPhase& g = p.ph[TC_GATEUP];   // gate + up (+ bias, activation, activation terms)
  g.w = a.gu; g.kc = a.H / 32; g.tile_bytes = tc_tile_bytes(g.kc); g.tiles = tc_gu_tiles(a.I);
  g.bterm = a.xterm; g.bterm_stride = 0; g.bias0 = a.gate_b; g.bias1 = a.up_b; g.rows = a.I;
  TcPhase& d = p.ph[TC_DOWN];     // down -> per-slot expert outputs
  d.w = a.down; d.kc = a.I / 32; d.tile_bytes = tc_tile_bytes(d.kc); d.tiles = tc_down_tiles(a.H);
  d.bterm = a.act_terms; d.bterm_stride = tc_bterm_bytes(a.I / 32); d.bias0 = a.down_b; d.bias1 = nullptr;
  d.rows = a.H;
  if (tc_down_tiles(a.H) > kTcMaxTiles) return cudaErrorInvalidValue;
  cudaError_t e = launch_tc(c, p, s);
  if (e != cudaSuccess || a.defer_combine) return e;
  return launch_moe_combine(c, tc_pending_combine(c, a), a.H, a.h, a.out, s);
}

}  // namespace ms
