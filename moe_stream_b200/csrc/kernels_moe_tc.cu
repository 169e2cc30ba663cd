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

// Optional timeline (build with -DMS_TRACE): %globaltimer stamps per CTA in g_tc_trace[mode][cta][k]:
// 0 entry, 1 tensor memory ready, 2 first copy issued, 3 first stage landed (MMA warp),
// 4 last MMA committed, 5 first accumulator ready (epilogue), 6 epilogue done, 7 last copy issued.
#ifdef MS_TRACE
__device__ unsigned long long g_tc_trace[2][1024][8];
#define TC_TRACE(k)                                                                            \
  do {                                                                                         \
    unsigned long long t_;                                                                     \
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));                                     \
    g_tc_trace[p.mode][blockIdx.x & 1023][(k)] = t_;                                           \
  } while (0)
#else
#define TC_TRACE(k) ((void)0)
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
constexpr int kStages = 4;
constexpr int kThreads = 192;
constexpr int kTmemCols = 256;
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

struct TcParams {
  int mode;
  const uint8_t* w;          // packed tiles [E_local][tiles][tile_bytes]
  int64_t tile_bytes;
  int tiles, kc;             // tiles per expert; chunk columns (reduction length / 32)
  const uint8_t* bterm;      // B terms: x (GATEUP) or act_terms base (DOWN)
  int64_t bterm_stride;      // per slot (DOWN), 0 (GATEUP)
  const int* idx;
  int K, expert_base, n_local;
  const float* bias0;        // gate_b (GATEUP) / down_b (DOWN)
  const float* bias1;        // up_b
  int rows;                  // rows per expert matrix of the output: I (GATEUP) / H (DOWN)
  float* part;               // [max_items][kTcMaxSeg][128] split-K partials
  uint32_t* cnt;             // [max_items] zero-initialised, self-resetting
  int max_items;
  float* act;                // GATEUP: [K][I] f32 activations (optional)
  uint8_t* act_terms;        // GATEUP: [K][tc_bterm_bytes(I/32)]
  int kc_out;                // GATEUP: I / 32
  int oai;
  float* partial;            // DOWN: [K][H] per-slot expert outputs
  uint32_t* err;
};

// first CTA whose unit range [b*T/G, (b+1)*T/G) contains unit x
__device__ __forceinline__ int cta_of_unit(int x, int T, int G) {
  int b = (int)((int64_t)x * G / T);
  while (b + 1 < G && (int)((int64_t)(b + 1) * T / G) <= x) ++b;
  while (b > 0 && (int)((int64_t)b * T / G) > x) --b;
  return b;
}

// This CTA's stages: its range of (item, K-word) units cut at slab boundaries.
struct Stage {
  int item, w0, w1;          // K-words [w0, w1) of item, within one slab
  bool seg_start, seg_end;   // first / last stage of this CTA's range of the item
};
struct StageWalk {
  int KW, u, u1, item, w, wend;
  __device__ void init(int u0, int u1_, int kw) { KW = kw; u = u0; u1 = u1_; item = 0; w = wend = 0; }
  __device__ bool next(Stage& st) {
    st.seg_start = false;
    if (w >= wend) {
      if (u >= u1) return false;
      item = u / KW;
      w = u - item * KW;
      wend = min(KW, u1 - item * KW);
      u = item * KW + wend;
      st.seg_start = true;
    }
    st.item = item;
    st.w0 = w;
    st.w1 = min(wend, (w / kKW + 1) * kKW);
    w = st.w1;
    st.seg_end = w >= wend;
    return true;
  }
};

__global__ void __launch_bounds__(kThreads, 1) moe_tc_kernel(TcParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ __align__(8) uint64_t full[kStages], empty[kStages], acc_full[2], acc_empty[2];
  __shared__ uint32_t tmem_base;
  __shared__ int s_slot[kMaxKSlots], s_exp[kMaxKSlots], s_n, s_last, s_abort;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) TC_TRACE(0);
  // barriers and tensor memory do not depend on the previous kernel: set them up before its wait
  if (threadIdx.x == 0) {
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
  const int KW = (p.kc + 3) / 4;                            // K-words per item (the last may hold 2 chunks)
  const int T = s_n * p.tiles * KW;
  int G = (int)gridDim.x;
  if (G > (T + 1) / 2) G = (T + 1) / 2;                      // at least ~2 K-words per CTA
  const bool active = T > 0 && (int)blockIdx.x < G;
  const int u0 = active ? (int)((int64_t)blockIdx.x * T / G) : 0;
  const int u1 = active ? (int)((int64_t)(blockIdx.x + 1) * T / G) : 0;

  if (warp == 0) {
    // ---------------- producer ----------------
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      StageWalk it;
      it.init(u0, u1, KW);
      Stage st;
      int j = 0;
      while (!*reinterpret_cast<volatile int*>(&s_abort) && it.next(st)) {
        const int ls = st.item / p.tiles, t = st.item % p.tiles;
        const uint8_t* tile = p.w + ((int64_t)s_exp[ls] * p.tiles + t) * p.tile_bytes;
        const uint8_t* bt = p.bterm + (int64_t)s_slot[ls] * p.bterm_stride;
        const int slab = st.w0 / kKW, c0 = 4 * st.w0, c1 = min(p.kc, 4 * st.w1), sl0 = slab * kCS;
        const int nch = min(kCS, p.kc - sl0);
        const int s = j % kStages, n = j / kStages;
        if (n > 0 && !mbar_wait(&empty[s], (uint32_t)((n - 1) & 1), p.err, EF_TIMEOUT_EMPTY)) { s_abort = 1; break; }
        uint8_t* sp = smem + (size_t)s * kStageBytes;
        const uint32_t ab = (uint32_t)(c1 - c0) * 2048u, bb = (uint32_t)(c1 - c0) * 256u;
        const uint32_t gb = (uint32_t)(st.w1 - st.w0) * 512u;
        mbar_expect_tx(&full[s], ab + 2 * gb + bb);
        const uint8_t* sb = tile + slab_off(slab);
        bulk_g2s_stream(sp, sb + (int64_t)(c0 - sl0) * 2048, ab, &full[s], pol);
        bulk_g2s_stream(sp + kStA, sb + (int64_t)nch * 2048 + (st.w0 - slab * kKW) * 512, gb, &full[s], pol);
        bulk_g2s(sp + kStA + kStSFA, bt + (int64_t)c0 * 256, bb, &full[s]);
        bulk_g2s(sp + kStA + kStSFA + kStB, bt + (int64_t)p.kc * 256 + (int64_t)st.w0 * 512, gb, &full[s]);
        if (j == 0) TC_TRACE(2);
        ++j;
      }
      TC_TRACE(7);
      // no copy may still be landing in shared memory when the CTA exits
      for (int q = max(0, j - kStages); q < j; ++q)
        mbar_wait(&full[q % kStages], (uint32_t)((q / kStages) & 1), p.err, EF_TIMEOUT_FULL);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      StageWalk it;
      it.init(u0, u1, KW);
      Stage st;
      int j = 0, seg = 0, nmma = 0;
      while (!*reinterpret_cast<volatile int*>(&s_abort) && it.next(st)) {
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
        if (j == 0) TC_TRACE(3);
        umma::fence_after_sync();
        const uint8_t* sp = smem + (size_t)s * kStageBytes;
        const uint32_t sfa_col = tb + (uint32_t)(2 * kAccSet + s * kSlotCols), sfb_col = sfa_col + 4 * kKW;
        const int nw = st.w1 - st.w0;
        for (int g = 0; g < nw; ++g) {
          umma::cp_sf_group(sfa_col + 4 * g, sp + kStA + g * 512);
          umma::cp_sf_group(sfb_col + 4 * g, sp + kStA + kStSFA + kStB + g * 512);
        }
        const uint32_t d_tmem = tb + (uint32_t)(a * kAccSet);
        const int c0 = 4 * st.w0, c1 = min(p.kc, 4 * st.w1);
        for (int cc = c0; cc < c1; cc += 2) {
          const uint64_t ad = umma::smem_desc(sp + (cc - c0) * 2048, 2048, 128);
          const uint64_t bd = umma::smem_desc(sp + kStA + kStSFA + (cc - c0) * 256, 256, 128);
          const int wl = (cc >> 2) - st.w0;            // K-word within the stage
          const uint32_t byte = (uint32_t)(cc & 3);    // the pair of blocks within the K-word
          umma::mma_mxf4(d_tmem + (uint32_t)((nmma % kSubAcc) * kAccCols), ad, bd,
                         umma::idesc_mxf4(128, 16, byte, byte), sfa_col + 4 * wl,
                         sfb_col + 4 * wl, nmma >= kSubAcc);
          ++nmma;
        }
        umma::commit(&empty[s]);   // the stage may be refilled once these MMAs have read it
        ++j;
        if (st.seg_end) {
          umma::commit(&acc_full[a]);
          TC_TRACE(4);
          ++seg;
        }
      }
    }
  } else {
    // ---------------- epilogue (warps 2-5: TMEM lane quadrants 2, 3, 0, 1) ----------------
    const int quad = warp & 3, row = 32 * quad + lane;
    const int et = threadIdx.x - 64;   // 0..127
    StageWalk it;
    it.init(u0, u1, KW);
    Stage st;
    int seg = 0, nmma = 0;
    while (it.next(st)) {
      if (st.seg_start) nmma = 0;
      nmma += (min(p.kc, 4 * st.w1) - 4 * st.w0 + 1) / 2;
      if (!st.seg_end) continue;
      const int item = st.item;
      const int a = seg & 1;
      const bool ok = mbar_wait(&acc_full[a], (uint32_t)((seg >> 1) & 1), p.err, EF_TIMEOUT_FULL);
      if (seg == 0 && et == 0) TC_TRACE(5);
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
      const int first = cta_of_unit(item * KW, T, G);
      const int nseg = cta_of_unit(item * KW + KW - 1, T, G) - first + 1;
      const int segi = (int)blockIdx.x - first;
      p.part[((int64_t)item * kTcMaxSeg + segi) * 128 + row] = sum;
      named_bar(1, 128);
      if (et == 0) {
        // release this CTA's partials (ordered before by the barrier) and count the range in
        __threadfence();
        s_last = (atomicAdd(&p.cnt[item], 1u) == (uint32_t)nseg - 1) ? 1 : 0;
        if (s_last) __threadfence();
      }
      named_bar(1, 128);
      if (s_last) {
        const int ls = item / p.tiles, t = item % p.tiles;
        const int e = s_exp[ls], slot = s_slot[ls];
        const float* pp = p.part + (int64_t)item * kTcMaxSeg * 128;
        if (p.mode == TC_GATEUP) {
          if (et < 64) {
            float g = 0.f, up = 0.f;
            for (int q = 0; q < nseg; ++q) { g += __ldcg(pp + q * 128 + et); up += __ldcg(pp + q * 128 + 64 + et); }
            const int r = t * 64 + et;
            if (p.bias0) g += p.bias0[(int64_t)e * p.rows + r];
            if (p.bias1) up += p.bias1[(int64_t)e * p.rows + r];
            const float av = p.oai ? swiglu_oai_tc(g, up) : (g / (1.0f + expf(-g))) * up;
            // this tile's 64 activations are chunk columns 2t, 2t+1 of the down projection's B terms
            umma::quantize_terms_warp(av, lane, p.act_terms + (int64_t)slot * umma::bterm_bytes(p.kc_out), p.kc_out,
                                      2 * t + (et >> 5));
            if (p.act) p.act[(int64_t)slot * p.rows + r] = av;
          }
        } else {
          const int r = t * 128 + et;
          if (r < p.rows) {
            float y = 0.f;
            for (int q = 0; q < nseg; ++q) y += __ldcg(pp + q * 128 + et);
            if (p.bias0) y += p.bias0[(int64_t)e * p.rows + r];
            p.partial[(int64_t)slot * p.rows + r] = y;
          }
        }
        if (et == 0) p.cnt[item] = 0u;
      }
      ++seg;
    }
    if (et == 0) TC_TRACE(6);
  }
  umma::fence_before_sync();
  __syncthreads();
  if (warp == 1) umma::tmem_dealloc(tb, kTmemCols);
}

cudaError_t launch_tc_phase(const DevCtx& c, const TcParams& p, cudaStream_t s) {
  const size_t smem = (size_t)kStages * kStageBytes;
  cudaError_t e = cudaFuncSetAttribute(moe_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)c.sm_count);
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

cudaError_t launch_moe_tc(const DevCtx& c, const TcMoeArgs& a, cudaStream_t s) {
  if (a.K < 1 || a.K > kMaxKSlots || !tc_supported(a.H, a.I) || a.n_local < 0) return cudaErrorInvalidValue;
  TcParams p = {};
  p.idx = a.idx; p.K = a.K; p.expert_base = a.expert_base; p.n_local = a.n_local; p.err = c.err;
  p.part = a.part; p.cnt = a.cnt; p.max_items = tc_max_items(a.H, a.I, a.K);
  // phase 1: gate + up (+ bias, activation, activation terms)
  p.mode = TC_GATEUP; p.w = a.gu; p.kc = a.H / 32; p.tile_bytes = tc_tile_bytes(p.kc); p.tiles = tc_gu_tiles(a.I);
  p.bterm = a.xterm; p.bterm_stride = 0; p.bias0 = a.gate_b; p.bias1 = a.up_b; p.rows = a.I; p.act = a.act;
  p.act_terms = a.act_terms; p.kc_out = a.I / 32; p.oai = a.oai_swiglu;
  cudaError_t e = launch_tc_phase(c, p, s);
  if (e != cudaSuccess) return e;
  // phase 2: down -> per-slot expert outputs
  p.mode = TC_DOWN; p.w = a.down; p.kc = a.I / 32; p.tile_bytes = tc_tile_bytes(p.kc); p.tiles = tc_down_tiles(a.H);
  p.bterm = a.act_terms; p.bterm_stride = tc_bterm_bytes(a.I / 32); p.bias0 = a.down_b; p.bias1 = nullptr;
  p.rows = a.H; p.act = nullptr; p.act_terms = nullptr; p.partial = a.partial;
  e = launch_tc_phase(c, p, s);
  if (e != cudaSuccess || a.defer_combine) return e;
  PendingCombine pc;
  pc.partial = a.partial; pc.idx = a.idx; pc.wts = a.wts; pc.K = a.K; pc.expert_base = a.expert_base;
  pc.n_local = a.n_local;
  return launch_moe_combine(c, pc, a.H, a.h, a.out, s);
}

}  // namespace ms
