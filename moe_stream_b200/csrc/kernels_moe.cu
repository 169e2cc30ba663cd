// kernels_moe.cu — router top-k and the fused MXFP4 expert FFN for decode (sm_100a).
//
// Reference semantics (moe-stream-core/src):
//   router + bias + dummy mask + top-k/softmax ... model/layer.rs:806-837, 1016-1027, 2346-2403
//   expert FFN, OAI SwiGLU, ascending-expert combine ... model/layer.rs:1797-1847, ops/activation.rs:25-38
//   MXFP4 block decode ... gguf/dequant.rs:580-628
//
// Expert FFN design (one token, memory bound): a persistent grid of one CTA per SM
// streams expert weight tiles in their native 17-byte MXFP4 blocks through a ring of
// shared-memory stages filled by 1-D bulk async copies (one producer thread, mbarrier
// completion).  Eight consumer warps decode the e2m1 codes in registers with
// cvt.rn.f16x2.e2m1x2 and feed mma.sync m16n8k16 (f16 in, f32 accumulate).  The
// activation vector is pre-split per 32-element block into f16 hi + lo parts after an
// exact power-of-two prescale, so each block dot is exact to ~2^-22 relative; the e8m0
// block scale and the prescale are re-applied in f32 per (row, block).  Column 0 of the
// MMA carries x_hi and column 1 carries x_lo.
#include <cuda_fp16.h>

#include "common.cuh"
#include "kernels.h"
#include "umma.cuh"

namespace ms {
namespace {

// Optional timeline of the phase kernel (build with -DMS_TRACE): %globaltimer stamps per CTA in
// g_phase_trace[mode][cta][slot] -- 0 entry, 1 prologue done, 2..9 warp 0's stage j ready,
// 10 warp 0 done, 11 producer's last copy issued.
#ifdef MS_TRACE
__device__ unsigned long long g_phase_trace[3][1024][16];
__device__ __forceinline__ unsigned long long gtimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
#define PHASE_TRACE(k) (g_phase_trace[p.mode][blockIdx.x & 1023][(k)] = gtimer())
#else
#define PHASE_TRACE(k) ((void)0)
#endif

constexpr int kCW = 16;                   // consumer warps
constexpr int kThreads = (kCW + 1) * 32;  // + one producer warp
constexpr int kMaxK = 16;                 // max experts per token
constexpr int kMaxStages = 8;
constexpr int kRedRows = 32;              // per-warp partial sums per item (RT=2 gate/up: 16 gate + 16 up)

enum { MODE_GATEUP = 0, MODE_DOWN = 1, MODE_PLAIN = 2 };
// weight block formats of the streamed matrix
enum { FMT_MXFP4 = 0, FMT_Q4K = 1, FMT_Q6K = 2, FMT_Q6KP = 3 };   // Q6KP: Q6_K in 224-byte superblocks

struct PhaseParams {
  int mode;
  int fmt;                 // FMT_*
  const uint8_t* w0;       // gate (GATEUP) or down (DOWN/PLAIN), stacked [E_local, rows, cols]
  const uint8_t* w1;       // up (GATEUP)
  int64_t expert_stride;   // bytes per expert matrix
  int rb;                  // bytes per streamed row
  int rs;                  // row stride in a shared-memory stage (rb, or rb + 16 to spread banks)
  int cols;                // reduction length (H for GATEUP, I for DOWN)
  int rows;                // rows per expert matrix (I for GATEUP, H for DOWN)
  int tile_rows;           // output rows per item (16)
  int n_tiles;
  int stage_bytes;
  int ns;
  const float* x;          // GATEUP: [cols] normed hidden; DOWN: act [K, cols]
  const int* idx;
  const float* wts;
  const float* bias0;      // gate_b or down_b
  const float* bias1;      // up_b
  float* act;              // GATEUP output [K, I]
  float* partial;          // DOWN scratch [K, H]
  uint32_t* tile_cnt;
  float* h;
  float* out;
  int K;
  int expert_base, n_local;
  int oai;
  int accumulate;          // PLAIN: y += W x
  uint32_t* err;
};

struct SlotInfo {
  int n;                   // local slots
  int slot[kMaxK];         // global slot index (0..K-1), ordered by ascending expert id
  int expert[kMaxK];       // local expert index
};

// One 32-column block of two MMA rows of this thread.  p0/p1: the rows' block starts in shared
// memory; w0/w1: 4-byte-aligned address of the word holding the thread's first code byte, with
// funnel shift sh0/sh1 (bits); the caller precomputes them so all loads use immediate offsets.
__device__ __forceinline__ void mx_block(const uint8_t* p0, const uint8_t* p1, const uint32_t* w0p,
                                         const uint32_t* w1p, uint32_t sh0, uint32_t sh1, const uint32_t (&bf)[4],
                                         int kbs, float& acc0, float& acc1) {
  const uint32_t w0 = __funnelshift_r(w0p[0], w0p[1], sh0);
  const uint32_t w1 = __funnelshift_r(w1p[0], w1p[1], sh1);
  const int e0 = *p0, e1 = *p1;
  uint32_t a0[4], a1[4];
  uint32_t g0, g1, g2, g3, u0, u1, u2, u3;
  e2m1x8_to_f16x2x4(w0, g0, g1, g2, g3);
  e2m1x8_to_f16x2x4(w1, u0, u1, u2, u3);
  a0[0] = g0; a0[1] = u0; a0[2] = g1; a0[3] = u1;
  a1[0] = g2; a1[1] = u2; a1[2] = g3; a1[3] = u3;
  float d[4] = {0.f, 0.f, 0.f, 0.f};
  mma_f16_16816(d, a0, bf[0], bf[1]);
  mma_f16_16816(d, a1, bf[2], bf[3]);
  // weight = e2m1 * 2^(E-127); x = x' * 2^kb: scale bits = (E + kb) << 23 (kbs = kb << 23)
  const float s0 = __int_as_float(max(e0 * 8388608 + kbs, 0));
  const float s1 = __int_as_float(max(e1 * 8388608 + kbs, 0));
  acc0 = fmaf(s0, d[0] + d[1], acc0);
  acc1 = fmaf(s1, d[2] + d[3], acc1);
}

// 4 unsigned 6-bit-or-less codes (one per byte) -> two f16x2 of (code - bias): bytes are placed
// under the f16 exponent of 1024 (0x64XX = 1024 + XX, exact) and the bias 1024 + b is subtracted.
__device__ __forceinline__ void codes4_to_f16x2(uint32_t q, uint32_t bias_h2, uint32_t& p0, uint32_t& p1) {
  const uint32_t t0 = __byte_perm(q, 0x64646464u, 0x4140u);   // [q0, 0x64, q1, 0x64]
  const uint32_t t1 = __byte_perm(q, 0x64646464u, 0x4342u);   // [q2, 0x64, q3, 0x64]
  const __half2 b = *reinterpret_cast<const __half2*>(&bias_h2);
  const __half2 r0 = __hsub2(*reinterpret_cast<const __half2*>(&t0), b);
  const __half2 r1 = __hsub2(*reinterpret_cast<const __half2*>(&t1), b);
  p0 = *reinterpret_cast<const uint32_t*>(&r0);
  p1 = *reinterpret_cast<const uint32_t*>(&r1);
}

// Q4_K sub-block j of one superblock for the thread's two MMA rows (gguf/dequant.rs:199-262):
// value = d*sc_j*q - dmin*m_j; the block dot is d*sc_j * sum(q x) - dmin*m_j * sum(x).
__device__ __forceinline__ void q4k_block(const uint8_t* sb0, const uint8_t* sb1, int j, int c, const uint32_t (&bf)[4],
                                          float xscale, float xsum, float& acc0, float& acc1) {
  const int jj = j & 3, nsh = (j & 1) * 4, qo = 16 + (j >> 1) * 32 + 4 * c;
  // the quad's four lanes decode one scale each -- lane c: row (c < 2 ? g : g + 8), d*sc (c even)
  // or dmin*m (c odd) -- and exchange them (the 6-bit fields of gguf/dequant.rs:199-208)
  const uint8_t* sbr = c < 2 ? sb0 : sb1;
  const int odd = c & 1;
  const uint32_t dm = *reinterpret_cast<const uint32_t*>(sbr);
  const uint32_t sa = *reinterpret_cast<const uint32_t*>(sbr + 4 + 4 * odd);   // scales (s0) or mins (s1)
  uint32_t v6;
  if (j < 4) {
    v6 = (sa >> (8 * jj)) & 63u;
  } else {
    const uint32_t s2 = *reinterpret_cast<const uint32_t*>(sbr + 12);
    v6 = ((s2 >> (8 * jj + 4 * odd)) & 0xFu) | (((sa >> (8 * jj + 6)) & 3u) << 4);
  }
  const float val = h2f_bits((uint16_t)((dm >> (16 * odd)) & 0xffffu)) * (float)v6;
  const float dsc0 = __shfl_sync(0xffffffffu, val, 0, 4) * xscale;
  const float dmn0 = __shfl_sync(0xffffffffu, val, 1, 4);
  const float dsc1 = __shfl_sync(0xffffffffu, val, 2, 4) * xscale;
  const float dmn1 = __shfl_sync(0xffffffffu, val, 3, 4);
  uint32_t p[2][2][2];   // [row][word][pair]
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const uint8_t* sb = r ? sb1 : sb0;
#pragma unroll
    for (int w = 0; w < 2; ++w) {
      const uint32_t q = (*reinterpret_cast<const uint32_t*>(sb + qo + 16 * w) >> nsh) & 0x0F0F0F0Fu;
      codes4_to_f16x2(q, 0x64006400u, p[r][w][0], p[r][w][1]);
    }
  }
  float dd[4] = {0.f, 0.f, 0.f, 0.f};
  uint32_t a[4];
  a[0] = p[0][0][0]; a[1] = p[1][0][0]; a[2] = p[0][0][1]; a[3] = p[1][0][1];
  mma_f16_16816(dd, a, bf[0], bf[1]);
  a[0] = p[0][1][0]; a[1] = p[1][1][0]; a[2] = p[0][1][1]; a[3] = p[1][1][1];
  mma_f16_16816(dd, a, bf[2], bf[3]);
  acc0 = fmaf(dsc0, dd[0] + dd[1], fmaf(-dmn0, xsum, acc0));
  acc1 = fmaf(dsc1, dd[2] + dd[3], fmaf(-dmn1, xsum, acc1));
}

// Q6_K elements (n, quad, l = 0..31) of one superblock for the thread's two rows
// (gguf/dequant.rs:335-378): q = (ql nibble | qh 2 bits << 4) - 32, scale d*sc[n*8 + l/16 + 2*quad].
// The two 16-element scale groups use separate MMAs.  ql/qh words are read at 2-byte alignment
// (rows of 210-byte blocks) through aligned loads and a funnel shift.
__device__ __forceinline__ uint32_t ld_u32_a2(const uint8_t* p) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  const uint32_t* w = reinterpret_cast<const uint32_t*>(a & ~(uintptr_t)3);
  return __funnelshift_r(w[0], w[1], (uint32_t)(a & 3) * 8u);
}
template <bool PAD>
__device__ __forceinline__ void q6k_block(const uint8_t* sb0, const uint8_t* sb1, int n, int quad, int c,
                                          const uint32_t (&bf)[4], float xscale, float& acc0, float& acc1) {
  const int qlo = n * 64 + (quad & 1) * 32 + 4 * c, qho = 128 + n * 32 + 4 * c;
  const int nsh = (quad >> 1) * 4, hsh = 2 * quad;
  uint32_t p[2][2][2];
  float s0[2], s1[2];
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const uint8_t* sb = r ? sb1 : sb0;
    const uint16_t scw = *reinterpret_cast<const uint16_t*>(sb + 192 + n * 8 + 2 * quad);
    const float d = h2f_bits(*reinterpret_cast<const uint16_t*>(sb + 208)) * xscale;
    s0[r] = d * (float)(int8_t)(scw & 0xff);
    s1[r] = d * (float)(int8_t)(scw >> 8);
#pragma unroll
    for (int w = 0; w < 2; ++w) {
      // padded superblocks start 16-byte aligned: aligned words; native 210-byte ones: funnel shift
      const uint32_t ql = PAD ? *reinterpret_cast<const uint32_t*>(sb + qlo + 16 * w) : ld_u32_a2(sb + qlo + 16 * w);
      const uint32_t qh = PAD ? *reinterpret_cast<const uint32_t*>(sb + qho + 16 * w) : ld_u32_a2(sb + qho + 16 * w);
      const uint32_t q = ((ql >> nsh) & 0x0F0F0F0Fu) | (((qh >> hsh) & 0x03030303u) << 4);
      codes4_to_f16x2(q, 0x64206420u, p[r][w][0], p[r][w][1]);   // 1024 + 32
    }
  }
  float da[4] = {0.f, 0.f, 0.f, 0.f}, db[4] = {0.f, 0.f, 0.f, 0.f};
  uint32_t a[4];
  a[0] = p[0][0][0]; a[1] = p[1][0][0]; a[2] = p[0][0][1]; a[3] = p[1][0][1];
  mma_f16_16816(da, a, bf[0], bf[1]);
  a[0] = p[0][1][0]; a[1] = p[1][1][0]; a[2] = p[0][1][1]; a[3] = p[1][1][1];
  mma_f16_16816(db, a, bf[2], bf[3]);
  acc0 = fmaf(s0[0], da[0] + da[1], fmaf(s1[0], db[0] + db[1], acc0));
  acc1 = fmaf(s0[1], da[2] + da[3], fmaf(s1[1], db[2] + db[3], acc1));
}

// B fragments of the activation vector for the K-blocks this warp owns.  MXFP4 pairs element
// 4c+q with 4c+16+q (the two nibbles of one code byte); the K-quants pair consecutive elements.
template <int FMT, int NBW>
__device__ __forceinline__ void build_bfrag(const float* __restrict__ x, int nb, int warp, int lane,
                                            uint32_t (&bf)[NBW][4], int (&kbs)[NBW], float (&xsum)[NBW]) {
  const int c = lane & 3, n = lane >> 2;
#pragma unroll
  for (int i = 0; i < NBW; ++i) {
    const int b = warp + kCW * i;
    bf[i][0] = bf[i][1] = bf[i][2] = bf[i][3] = 0u;
    kbs[i] = 0;
    xsum[i] = 0.f;
    if (b < nb) {
      const float v = x[32 * b + lane];
      if (FMT == FMT_Q4K) xsum[i] = warp_sum(v);
      const float m = warp_max(fabsf(v));
      const int ef = (int)((__float_as_uint(m) >> 23) & 0xffu);
      const int k = (m > 0.f) ? (ef - 126) : 0;              // m * 2^-k in [0.5, 1)
      kbs[i] = k * 8388608;
      const float sc = __uint_as_float((uint32_t)(127 - k) << 23);
      if (n < 2) {
        const float4 lo4 = *reinterpret_cast<const float4*>(x + 32 * b + 4 * c);
        const float4 hi4 = *reinterpret_cast<const float4*>(x + 32 * b + 16 + 4 * c);
        const float va[4] = {lo4.x, lo4.y, lo4.z, lo4.w};
        const float vb[4] = {hi4.x, hi4.y, hi4.z, hi4.w};
        __half hv[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const float a = (q < 4 ? va[q] : vb[q - 4]) * sc;
          __half ah = __float2half_rn(a);
          if (n == 1) ah = __float2half_rn(a - __half2float(ah));
          hv[q] = ah;
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          if (FMT == FMT_MXFP4) bf[i][q] = pack_half2(hv[q], hv[4 + q]);     // (4c+q, 4c+16+q)
          else bf[i][q] = pack_half2(hv[(q >> 1) * 4 + (q & 1) * 2], hv[(q >> 1) * 4 + (q & 1) * 2 + 1]);
        }
      }
    }
  }
}

__device__ __forceinline__ float swiglu_oai(float g, float u) {
  const float gc = fminf(g, 7.0f);
  const float uc = fminf(fmaxf(u, -7.0f), 7.0f);
  const float sig = 1.0f / (expf(-(gc * 1.702f)) + 1.0f);
  return (gc * sig) * (uc + 1.0f);
}
__device__ __forceinline__ float silu_mul(float g, float u) { return (g / (1.0f + expf(-g))) * u; }

// Epilogue of one item, run by the last consumer warp to finish it.
__device__ __forceinline__ void item_epilogue(const PhaseParams& p, const SlotInfo* si, const float* red, int ls,
                                              int t, int lane) {
  const int slot = si->slot[ls], e = si->expert[ls];
  if (p.mode == MODE_GATEUP) {
    // red[w][0..15] gate rows, red[w][16..31] up rows of output rows t*16 + 0..15
    const int r = t * 16 + (lane & 15);
    float sum = 0.f;
#pragma unroll
    for (int w = 0; w < kCW; ++w) sum += red[w * kRedRows + lane];
    const float* bias = lane < 16 ? p.bias0 : p.bias1;
    if (bias) sum += bias[(size_t)e * p.rows + r];
    const float up = __shfl_down_sync(0xffffffffu, sum, 16);
    if (lane < 16) p.act[(size_t)slot * p.rows + r] = p.oai ? swiglu_oai(sum, up) : silu_mul(sum, up);
    return;
  }
  float sum = 0.f;
  if (lane < 16) {
#pragma unroll
    for (int w = 0; w < kCW; ++w) sum += red[w * kRedRows + lane];
  }
  const int r = t * 16 + lane;
  if (p.mode == MODE_PLAIN) {
    if (lane < 16 && r < p.rows) {
      if (p.bias0) sum += p.bias0[r];
      p.out[r] = p.accumulate ? p.out[r] + sum : sum;
    }
    return;
  }
  // DOWN: per-slot expert output rows (bias included); the weighted combine in ascending expert
  // order happens in the consumer of the residual stream (PendingCombine) or moe_combine_kernel.
  if (lane < 16) {
    if (p.bias0) sum += p.bias0[(size_t)e * p.rows + r];
    p.partial[(size_t)slot * p.rows + r] = sum;
  }
}

// Shared-memory row stride of a stage: rows whose length is a multiple of 16 bytes but an even
// number of 16-byte units would put the eight rows of an MMA fragment on the same banks; they get
// 16 bytes of padding (copied row by row).  Other rows stay densely packed (one copy per matrix).
__host__ __device__ __forceinline__ int stage_row_stride(int rb) {
  return (rb % 16 == 0 && (rb / 16) % 2 == 0) ? rb + 16 : rb;
}

// Fills one stage (run by the whole producer warp): `tile_rows` rows of w0 (and of w1 after them
// when two) starting at byte `base`, rows at stride rs in shared memory.
__device__ __forceinline__ void issue_stage(uint8_t* dst, const uint8_t* w0, const uint8_t* w1, int64_t base, int rb,
                                            int rs, int tile_rows, bool two, uint64_t* bar, uint64_t pol, int lane) {
  const uint32_t part = (uint32_t)(tile_rows * rb);
  if (lane == 0) mbar_expect_tx(bar, (two ? 2u : 1u) * part);
  __syncwarp();
  if (rs == rb) {
    if (lane == 0) {
      bulk_g2s_stream(dst, w0 + base, part, bar, pol);
      if (two) bulk_g2s_stream(dst + part, w1 + base, part, bar, pol);
    }
  } else {
    const int nr = (two ? 2 : 1) * tile_rows;
    for (int r = lane; r < nr; r += 32) {
      const uint8_t* src = (r < tile_rows ? w0 : w1) + base + (int64_t)(r % tile_rows) * rb;
      bulk_g2s_stream(dst + (size_t)r * rs, src, (uint32_t)rb, bar, pol);
    }
  }
}

// RT = MMA row tiles per item: 2 for GATEUP (16 gate + 16 up rows), 1 for DOWN / PLAIN (16 rows).
template <int FMT, int NBW, int RT>
__global__ void __launch_bounds__(kThreads, 1) moe_mxfp4_phase_kernel(PhaseParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* stages = smem;
  const int nrb = p.ns + 1;   // reduction buffers: warps run at most ns items apart
  float* red = reinterpret_cast<float*>(smem + (size_t)p.ns * p.stage_bytes);       // [nrb][kCW][kRedRows]
  uint64_t* full = reinterpret_cast<uint64_t*>(red + (size_t)nrb * kCW * kRedRows);
  uint64_t* empty = full + kMaxStages;
  uint32_t* red_cnt = reinterpret_cast<uint32_t*>(empty + kMaxStages);                // [kMaxStages + 1]
  SlotInfo* si = reinterpret_cast<SlotInfo*>(red_cnt + kMaxStages + 1);
  int* abort_flag = reinterpret_cast<int*>(si + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) PHASE_TRACE(0);
  pdl_wait_prior();
  pdl_launch_dependents();   // the next kernel may start its own (weight) prefetch now
  if (threadIdx.x == 0) {
    // local slots ordered by ascending expert id (the reference's accumulation order)
    int n = 0;
    if (p.mode == MODE_PLAIN) { si->expert[0] = 0; si->slot[0] = 0; n = 1; }
    for (int k = 0; k < p.K && p.mode != MODE_PLAIN; ++k) {
      const int e = p.idx[k] - p.expert_base;
      if (e < 0 || e >= p.n_local) {
        if (p.n_local == 0 || p.idx[k] < 0) atomicOr(p.err, EF_BAD_INDEX);
        continue;
      }
      int j = n++;
      while (j > 0 && si->expert[j - 1] > e) {
        si->expert[j] = si->expert[j - 1];
        si->slot[j] = si->slot[j - 1];
        --j;
      }
      si->expert[j] = e;
      si->slot[j] = k;
    }
    si->n = n;
    *abort_flag = 0;
    for (int b = 0; b <= kMaxStages; ++b) red_cnt[b] = 0u;
    for (int s = 0; s < p.ns; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kCW);
    }
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) PHASE_TRACE(1);

  const int n_items = si->n * p.n_tiles;
  const int begin = (int)((int64_t)blockIdx.x * n_items / gridDim.x);
  const int end = (int)((int64_t)(blockIdx.x + 1) * n_items / gridDim.x);
  const int my_n = end - begin;
  if (my_n <= 0) return;

  if (warp == kCW) {
    // ---------------- producer (whole warp: per-row copies when rows are padded) ----------------
    const uint64_t pol = policy_evict_first();
    const uint32_t part_bytes = (uint32_t)(p.tile_rows * p.rb);
    int issued = 0;
    for (int j = 0; j < my_n; ++j) {
      const int s = j % p.ns, n = j / p.ns;
      if (n > 0 && !__all_sync(0xffffffffu, mbar_wait(&empty[s], (uint32_t)((n - 1) & 1), p.err, EF_TIMEOUT_EMPTY)))
        break;
      const int item = begin + j;
      const int ls = item / p.n_tiles, t = item % p.n_tiles;
      const int64_t base = (int64_t)si->expert[ls] * p.expert_stride + (int64_t)t * part_bytes;
      issue_stage(stages + (size_t)s * p.stage_bytes, p.w0, p.w1, base, p.rb, p.rs, p.tile_rows,
                  p.mode == MODE_GATEUP, &full[s], pol, lane);
      ++issued;
    }
    if (lane == 0) {
      PHASE_TRACE(11);
      // make sure no copy into this CTA's shared memory is still in flight at exit
      for (int j = max(0, issued - p.ns); j < issued; ++j)
        mbar_wait(&full[j % p.ns], (uint32_t)((j / p.ns) & 1), p.err, EF_TIMEOUT_FULL);
    }
    return;
  }

  // ---------------- consumers ----------------
  const int nb = p.cols / 32;
  const int c = lane & 3, g = lane >> 2;
  uint32_t bf[NBW][4];
  int kbs[NBW];
  float xsum[NBW];
  // this thread's two MMA rows per row tile (byte offsets of row starts in the stage)
  uint32_t off0[RT], off1[RT];
#pragma unroll
  for (int q = 0; q < RT; ++q) {
    if (p.mode == MODE_GATEUP) {
      off0[q] = (uint32_t)(8 * q + g) * p.rs;           // gate row
      off1[q] = (uint32_t)(16 + 8 * q + g) * p.rs;      // up row of the same output row
    } else {
      off0[q] = (uint32_t)(16 * q + g) * p.rs;
      off1[q] = (uint32_t)(16 * q + g + 8) * p.rs;
    }
  }
  // Block b = warp + kCW*i of a row starts at row + 17*b; kCW*17 = 272 bytes is a multiple of 4,
  // so the alignment of the thread's code bytes is the same for all its blocks.
  uint32_t bs0[RT], bs1[RT], wa0[RT], wa1[RT], sh0[RT], sh1[RT];
#pragma unroll
  for (int q = 0; q < RT; ++q) {
    bs0[q] = off0[q] + 17u * warp;
    bs1[q] = off1[q] + 17u * warp;
    const uint32_t c0 = bs0[q] + 1 + 4 * c, c1 = bs1[q] + 1 + 4 * c;
    wa0[q] = c0 & ~3u; sh0[q] = (c0 & 3u) * 8u;
    wa1[q] = c1 & ~3u; sh1[q] = (c1 & 3u) * 8u;
  }
  int cur_slot = -1;
  for (int j = 0; j < my_n; ++j) {
    if (*reinterpret_cast<volatile int*>(abort_flag)) break;
    const int s = j % p.ns, n = j / p.ns;
    const int item = begin + j;
    const int ls = item / p.n_tiles, t = item % p.n_tiles;
    const int x_slot = (p.mode == MODE_GATEUP) ? 0 : si->slot[ls];
    if (x_slot != cur_slot) {
      build_bfrag<FMT, NBW>(p.x + (size_t)x_slot * (p.mode == MODE_GATEUP ? 0 : p.cols), nb, warp, lane, bf, kbs,
                            xsum);
      cur_slot = x_slot;
    }
    float acc0[RT], acc1[RT];
#pragma unroll
    for (int q = 0; q < RT; ++q) acc0[q] = acc1[q] = 0.f;
    if (!mbar_wait(&full[s], (uint32_t)(n & 1), p.err, EF_TIMEOUT_FULL)) {
      if (lane == 0) atomicExch(abort_flag, 1);
      break;
    }
    if (warp == 0 && lane == 0 && j < 8) PHASE_TRACE(2 + j);
    const uint8_t* st = stages + (size_t)s * p.stage_bytes;
#pragma unroll
    for (int i = 0; i < NBW; ++i) {
      const int b = warp + kCW * i;
      if (b < nb) {
        if constexpr (FMT == FMT_MXFP4) {
#pragma unroll
          for (int q = 0; q < RT; ++q)
            mx_block(st + bs0[q] + kCW * 17 * i, st + bs1[q] + kCW * 17 * i,
                     reinterpret_cast<const uint32_t*>(st + wa0[q] + kCW * 17 * i),
                     reinterpret_cast<const uint32_t*>(st + wa1[q] + kCW * 17 * i), sh0[q], sh1[q], bf[i], kbs[i],
                     acc0[q], acc1[q]);
        } else {
          // 32-column block b = warp + 16 i lies in superblock b / 8 at sub-block warp % 8
          const float xscale = __int_as_float(max(127 * 8388608 + kbs[i], 0));   // 2^kb
          constexpr int kSb = FMT == FMT_Q6KP ? kQ6PadBytes : 210;                // Q6_K superblock stride
          const int sbk = b >> 3;
#pragma unroll
          for (int q = 0; q < RT; ++q) {
            if constexpr (FMT == FMT_Q4K)
              q4k_block(st + off0[q] + 144 * sbk, st + off1[q] + 144 * sbk, warp & 7, c, bf[i], xscale, xsum[i],
                        acc0[q], acc1[q]);
            else
              q6k_block<FMT == FMT_Q6KP>(st + off0[q] + kSb * sbk, st + off1[q] + kSb * sbk, (warp & 7) >> 2,
                                         warp & 3, c, bf[i], xscale, acc0[q], acc1[q]);
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);   // stage data no longer needed by this warp
    // partial sums -> reduction buffer; the last warp to arrive runs the item's epilogue
    const int rbuf = j % nrb;
    float* rw = red + ((size_t)rbuf * kCW + warp) * kRedRows;
    if (c == 0) {
#pragma unroll
      for (int q = 0; q < RT; ++q) {
        if (p.mode == MODE_GATEUP) { rw[8 * q + g] = acc0[q]; rw[16 + 8 * q + g] = acc1[q]; }
        else { rw[16 * q + g] = acc0[q]; rw[16 * q + g + 8] = acc1[q]; }
      }
    }
    __syncwarp();
    uint32_t old = 0;
    if (lane == 0) {
      __threadfence_block();
      old = atomicAdd(&red_cnt[rbuf], 1u);
    }
    old = __shfl_sync(0xffffffffu, old, 0);
    if (old == kCW - 1) {
      __threadfence_block();
      item_epilogue(p, si, red + (size_t)rbuf * kCW * kRedRows, ls, t, lane);
      __syncwarp();
      if (lane == 0) red_cnt[rbuf] = 0u;
    }
  }
  if (warp == 0 && lane == 0) PHASE_TRACE(10);
}

template <int FMT, int NBW, int RT>
cudaError_t launch_phase(const DevCtx& c, const PhaseParams& p, cudaStream_t s) {
  const size_t smem = (size_t)p.ns * p.stage_bytes + (size_t)(p.ns + 1) * kCW * kRedRows * sizeof(float) +
                      2 * kMaxStages * 8 + (kMaxStages + 1) * 4 + sizeof(SlotInfo) + 16;
  cudaError_t e = cudaFuncSetAttribute(moe_mxfp4_phase_kernel<FMT, NBW, RT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem);
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
  return cudaLaunchKernelEx(&cfg, moe_mxfp4_phase_kernel<FMT, NBW, RT>, p);
}

template <int FMT, int RT>
cudaError_t dispatch_nbw(const DevCtx& c, const PhaseParams& p, cudaStream_t s) {
  const int nbw = (p.cols / 32 + kCW - 1) / kCW;
  if (nbw <= 1) return launch_phase<FMT, 1, RT>(c, p, s);
  if (nbw <= 2) return launch_phase<FMT, 2, RT>(c, p, s);
  if (nbw <= 4) return launch_phase<FMT, 4, RT>(c, p, s);
  if (nbw <= 6) return launch_phase<FMT, 6, RT>(c, p, s);
  if (nbw <= 8) return launch_phase<FMT, 8, RT>(c, p, s);
  return cudaErrorInvalidValue;
}

cudaError_t dispatch_phase(const DevCtx& c, const PhaseParams& p, cudaStream_t s) {
  if (p.fmt == FMT_MXFP4) return p.mode == MODE_GATEUP ? dispatch_nbw<FMT_MXFP4, 2>(c, p, s) : dispatch_nbw<FMT_MXFP4, 1>(c, p, s);
  if (p.fmt == FMT_Q4K) return p.mode == MODE_GATEUP ? dispatch_nbw<FMT_Q4K, 2>(c, p, s) : dispatch_nbw<FMT_Q4K, 1>(c, p, s);
  if (p.fmt == FMT_Q6K) return p.mode == MODE_GATEUP ? dispatch_nbw<FMT_Q6K, 2>(c, p, s) : dispatch_nbw<FMT_Q6K, 1>(c, p, s);
  if (p.fmt == FMT_Q6KP) return p.mode == MODE_GATEUP ? dispatch_nbw<FMT_Q6KP, 2>(c, p, s) : dispatch_nbw<FMT_Q6KP, 1>(c, p, s);
  return cudaErrorInvalidValue;
}

int fmt_of(int qtype) {
  return qtype == Q_MXFP4 ? FMT_MXFP4 : qtype == Q_Q4_K ? FMT_Q4K : qtype == Q_Q6_K ? FMT_Q6K
       : qtype == Q_Q6_K_PAD ? FMT_Q6KP : -1;
}

int pick_stages(int stage_bytes) {
  int ns = (int)((192 * 1024) / stage_bytes);
  return ns < 2 ? 2 : (ns > 6 ? 6 : ns);
}

// ---------------- batched decode: tokens grouped by expert ----------------
// A batch's (token, slot) entries are sorted by local expert (then token) by group_route_kernel and
// cut into chunks of <= kGT tokens of one expert.  moe_group_kernel streams each chunk's expert
// tiles once, exactly like moe_mxfp4_phase_kernel, with B column 2t / 2t+1 carrying token t's
// x_hi / x_lo: MMA accumulator columns 2c, 2c+1 of lane (g, c) are token c, so each lane applies
// token c's prescale (and, for Q4_K, its block sum) in the per-block epilogue.
constexpr int kGT = 4;
constexpr int kRouteThreads = 1024;
constexpr int kGroupMaxStages = 16;
constexpr int kGroupRedCnt = 64;   // reduction counters: groups x buffers per group

struct GroupParams {
  int mode;                // MODE_GATEUP / MODE_DOWN
  int fmt;
  const uint8_t* w0;
  const uint8_t* w1;
  int64_t expert_stride;
  int rb, rs, cols, rows, n_tiles, stage_bytes, ns;
  const float* x;          // GATEUP: [B][cols] normed input; DOWN: act [entries][cols]
  const int* grp;          // [0] chunks, then (expert_local, entry_begin, n_tok) per chunk
  const int* ent_slot;     // flat (token, slot) index b * K + k of each entry
  int K;                   // slots per token
  const float* bias0;
  const float* bias1;
  float* out;              // GATEUP: act [entries][rows]; DOWN: y [entries][rows]
  int oai;
  uint32_t* err;
};

__device__ __forceinline__ int block_excl_scan(int v, int* wsum, int* total) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) wsum[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = lane < nw ? wsum[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    if (lane < nw) wsum[lane] = w;   // inclusive warp totals
    if (lane == nw - 1) *total = w;
  }
  __syncthreads();
  const int r = x - v + (warp > 0 ? wsum[warp - 1] : 0);
  __syncthreads();
  return r;
}

// One CTA: count entries per local expert, place them in (expert, token) order, emit the chunks.
__global__ void __launch_bounds__(kRouteThreads) group_route_kernel(const int* idx, int n_ent, int K, int expert_base,
                                                                    int n_local, int* grp, int* ent_slot, int* ent_of,
                                                                    uint32_t* err) {
  __shared__ int cnt[kRouteThreads];
  __shared__ int s_e[kMaxBatch * kMaxK];
  __shared__ int wsum[32], tot0, tot1;
  pdl_wait_prior();
  pdl_launch_dependents();
  const int t = threadIdx.x;
  cnt[t] = 0;
  for (int i = t; i < n_ent; i += blockDim.x) {
    const int id = idx[i], e = id - expert_base;
    if (id < 0) atomicOr(err, EF_BAD_INDEX);
    s_e[i] = (id >= 0 && e >= 0 && e < n_local) ? e : -1;
  }
  __syncthreads();
  for (int i = t; i < n_ent; i += blockDim.x)
    if (s_e[i] >= 0) atomicAdd(&cnt[s_e[i]], 1);
  __syncthreads();
  const int c = t < n_local ? cnt[t] : 0;
  const int off = block_excl_scan(c, wsum, &tot0);
  const int nch = (c + kGT - 1) / kGT;
  const int coff = block_excl_scan(nch, wsum, &tot1);
  for (int i = t; i < n_ent; i += blockDim.x) {
    const int e = s_e[i];
    if (e < 0) { ent_of[i] = -1; continue; }
    int rank = 0;
    for (int j = 0; j < i; ++j) rank += s_e[j] == e;
    // the entry's slot is its expert's offset (scanned counts, published below) + rank
    ent_of[i] = rank;   // provisional
  }
  __syncthreads();
  cnt[t] = off;   // expert offsets
  __syncthreads();
  for (int i = t; i < n_ent; i += blockDim.x) {
    const int e = s_e[i];
    if (e < 0) continue;
    const int pos = cnt[e] + ent_of[i];
    ent_of[i] = pos;
    ent_slot[pos] = i;
  }
  if (t < n_local)
    for (int q = 0; q < nch; ++q) {
      const int j = coff + q;
      grp[1 + 3 * j] = t;
      grp[2 + 3 * j] = off + kGT * q;
      grp[3 + 3 * j] = min(kGT, c - kGT * q);
    }
  if (t == 0) grp[0] = tot1;
}

// B fragments of up to kGT tokens for the K-blocks this warp owns (column 2t: token t's x_hi,
// 2t + 1: x_lo, each token prescaled by its own power of two); kbs / xsum: token c's (c = lane & 3)
template <int FMT, int NBW, int GW>
__device__ __forceinline__ void build_bfrag_group(const float* const (&xr)[kGT], int ntok, int nb, int wi, int lane,
                                                  uint32_t (&bf)[NBW][4], int (&kbs)[NBW], float (&xsum)[NBW]) {
  const int c = lane & 3, n = lane >> 2, tt = n >> 1, hl = n & 1;
#pragma unroll
  for (int i = 0; i < NBW; ++i) {
    const int b = wi + GW * i;
    bf[i][0] = bf[i][1] = bf[i][2] = bf[i][3] = 0u;
    kbs[i] = 0;
    xsum[i] = 0.f;
    if (b < nb) {
      int kt[kGT];
      float st = 1.f;
#pragma unroll
      for (int t = 0; t < kGT; ++t) {
        kt[t] = 0;
        if (t < ntok) {
          const float v = xr[t][32 * b + lane];
          if (FMT == FMT_Q4K) {
            const float xs = warp_sum(v);
            if (t == c) xsum[i] = xs;
          }
          const float m = warp_max(fabsf(v));
          const int ef = (int)((__float_as_uint(m) >> 23) & 0xffu);
          kt[t] = (m > 0.f) ? (ef - 126) : 0;
          if (t == tt) st = __uint_as_float((uint32_t)(127 - kt[t]) << 23);
        }
      }
#pragma unroll
      for (int t = 0; t < kGT; ++t)
        if (t == c) kbs[i] = kt[t] * 8388608;
      if (tt < ntok) {
        const float* x = xr[tt];
        const float4 lo4 = *reinterpret_cast<const float4*>(x + 32 * b + 4 * c);
        const float4 hi4 = *reinterpret_cast<const float4*>(x + 32 * b + 16 + 4 * c);
        const float va[4] = {lo4.x, lo4.y, lo4.z, lo4.w};
        const float vb[4] = {hi4.x, hi4.y, hi4.z, hi4.w};
        __half hv[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const float a = (q < 4 ? va[q] : vb[q - 4]) * st;
          __half ah = __float2half_rn(a);
          if (hl) ah = __float2half_rn(a - __half2float(ah));
          hv[q] = ah;
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          if (FMT == FMT_MXFP4) bf[i][q] = pack_half2(hv[q], hv[4 + q]);
          else bf[i][q] = pack_half2(hv[(q >> 1) * 4 + (q & 1) * 2], hv[(q >> 1) * 4 + (q & 1) * 2 + 1]);
        }
      }
    }
  }
}

// GW consumer warps share an item (split over its K blocks); the kCW / GW groups take items in turn.
template <int FMT, int NBW, int RT, int GW>
__global__ void __launch_bounds__(kThreads, 1) moe_group_kernel(GroupParams p) {
  constexpr int G = kCW / GW;             // items in flight at once
  constexpr int kGRed = kGT * kRedRows;   // per-warp partial sums per item
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* stages = smem;
  const int nrbg = (p.ns + G - 1) / G + 1;   // reduction buffers per group: its warps run < ns items apart
  float* red = reinterpret_cast<float*>(smem + (size_t)p.ns * p.stage_bytes);   // [G][nrbg][GW][kGRed]
  uint64_t* full = reinterpret_cast<uint64_t*>(red + (size_t)G * nrbg * GW * kGRed);
  uint64_t* empty = full + kGroupMaxStages;
  uint32_t* red_cnt = reinterpret_cast<uint32_t*>(empty + kGroupMaxStages);   // [G][nrbg]
  int* abort_flag = reinterpret_cast<int*>(red_cnt + kGroupRedCnt);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_wait_prior();
  pdl_launch_dependents();
  if (threadIdx.x == 0) {
    *abort_flag = 0;
    for (int b = 0; b < kGroupRedCnt; ++b) red_cnt[b] = 0u;
    for (int s = 0; s < p.ns; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], GW);
    }
    fence_mbar_init();
  }
  __syncthreads();
  const int n_items = p.grp[0] * p.n_tiles;
  const int begin = (int)((int64_t)blockIdx.x * n_items / gridDim.x);
  const int end = (int)((int64_t)(blockIdx.x + 1) * n_items / gridDim.x);
  const int my_n = end - begin;
  if (my_n <= 0) return;

  if (warp == kCW) {
    const uint64_t pol = policy_evict_first();
    const uint32_t part_bytes = (uint32_t)(16 * p.rb);
    int issued = 0;
    for (int j = 0; j < my_n; ++j) {
      const int s = j % p.ns, n = j / p.ns;
      if (n > 0 && !__all_sync(0xffffffffu, mbar_wait(&empty[s], (uint32_t)((n - 1) & 1), p.err, EF_TIMEOUT_EMPTY)))
        break;
      const int item = begin + j;
      const int ch = item / p.n_tiles, t = item % p.n_tiles;
      const int64_t base = (int64_t)p.grp[1 + 3 * ch] * p.expert_stride + (int64_t)t * part_bytes;
      issue_stage(stages + (size_t)s * p.stage_bytes, p.w0, p.w1, base, p.rb, p.rs, 16, p.mode == MODE_GATEUP,
                  &full[s], pol, lane);
      ++issued;
    }
    if (lane == 0)
      for (int j = max(0, issued - p.ns); j < issued; ++j)
        mbar_wait(&full[j % p.ns], (uint32_t)((j / p.ns) & 1), p.err, EF_TIMEOUT_FULL);
    return;
  }

  const int grp_i = warp / GW, wi = warp % GW;
  const int nb = p.cols / 32;
  const int c = lane & 3, g = lane >> 2;
  uint32_t bf[NBW][4];
  int kbs[NBW];
  float xsum[NBW];
  uint32_t off0[RT], off1[RT];
#pragma unroll
  for (int q = 0; q < RT; ++q) {
    if (p.mode == MODE_GATEUP) {
      off0[q] = (uint32_t)(8 * q + g) * p.rs;
      off1[q] = (uint32_t)(16 + 8 * q + g) * p.rs;
    } else {
      off0[q] = (uint32_t)(16 * q + g) * p.rs;
      off1[q] = (uint32_t)(16 * q + g + 8) * p.rs;
    }
  }
  uint32_t bs0[RT], bs1[RT], wa0[RT], wa1[RT], sh0[RT], sh1[RT];
#pragma unroll
  for (int q = 0; q < RT; ++q) {
    bs0[q] = off0[q] + 17u * wi;
    bs1[q] = off1[q] + 17u * wi;
    const uint32_t c0 = bs0[q] + 1 + 4 * c, c1 = bs1[q] + 1 + 4 * c;
    wa0[q] = c0 & ~3u; sh0[q] = (c0 & 3u) * 8u;
    wa1[q] = c1 & ~3u; sh1[q] = (c1 & 3u) * 8u;
  }
  int cur = -1, ntok = 0, ebeg = 0;
  for (int j = grp_i; j < my_n; j += G) {
    if (*reinterpret_cast<volatile int*>(abort_flag)) break;
    const int s = j % p.ns, n = j / p.ns;
    const int item = begin + j;
    const int ch = item / p.n_tiles, t = item % p.n_tiles;
    if (ch != cur) {
      ebeg = p.grp[2 + 3 * ch];
      ntok = p.grp[3 + 3 * ch];
      const float* xr[kGT];
#pragma unroll
      for (int q = 0; q < kGT; ++q) {
        const int ent = ebeg + min(q, ntok - 1);
        const int row = p.mode == MODE_GATEUP ? p.ent_slot[ent] / p.K : ent;
        xr[q] = p.x + (size_t)row * p.cols;
      }
      build_bfrag_group<FMT, NBW, GW>(xr, ntok, nb, wi, lane, bf, kbs, xsum);
      cur = ch;
    }
    float acc0[RT], acc1[RT];
#pragma unroll
    for (int q = 0; q < RT; ++q) acc0[q] = acc1[q] = 0.f;
    if (!mbar_wait(&full[s], (uint32_t)(n & 1), p.err, EF_TIMEOUT_FULL)) {
      if (lane == 0) atomicExch(abort_flag, 1);
      break;
    }
    const uint8_t* st = stages + (size_t)s * p.stage_bytes;
#pragma unroll
    for (int i = 0; i < NBW; ++i) {
      const int b = wi + GW * i;
      if (b < nb) {
        if constexpr (FMT == FMT_MXFP4) {
#pragma unroll
          for (int q = 0; q < RT; ++q)
            mx_block(st + bs0[q] + GW * 17 * i, st + bs1[q] + GW * 17 * i,
                     reinterpret_cast<const uint32_t*>(st + wa0[q] + GW * 17 * i),
                     reinterpret_cast<const uint32_t*>(st + wa1[q] + GW * 17 * i), sh0[q], sh1[q], bf[i], kbs[i],
                     acc0[q], acc1[q]);
        } else {
          const float xscale = __int_as_float(max(127 * 8388608 + kbs[i], 0));
          constexpr int kSb = FMT == FMT_Q6KP ? kQ6PadBytes : 210;   // Q6_K superblock stride
          const int sbk = b >> 3, sub = b & 7;
#pragma unroll
          for (int q = 0; q < RT; ++q) {
            if constexpr (FMT == FMT_Q4K)
              q4k_block(st + off0[q] + 144 * sbk, st + off1[q] + 144 * sbk, sub, c, bf[i], xscale, xsum[i],
                        acc0[q], acc1[q]);
            else
              q6k_block<FMT == FMT_Q6KP>(st + off0[q] + kSb * sbk, st + off1[q] + kSb * sbk, sub >> 2, sub & 3, c,
                                         bf[i], xscale, acc0[q], acc1[q]);
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
    const int rbuf = grp_i * nrbg + (j / G) % nrbg;
    float* rw = red + ((size_t)rbuf * GW + wi) * kGRed + c * kRedRows;   // token c's rows
#pragma unroll
    for (int q = 0; q < RT; ++q) {
      if (p.mode == MODE_GATEUP) { rw[8 * q + g] = acc0[q]; rw[16 + 8 * q + g] = acc1[q]; }
      else { rw[16 * q + g] = acc0[q]; rw[16 * q + g + 8] = acc1[q]; }
    }
    __syncwarp();
    uint32_t old = 0;
    if (lane == 0) {
      __threadfence_block();
      old = atomicAdd(&red_cnt[rbuf], 1u);
    }
    old = __shfl_sync(0xffffffffu, old, 0);
    if (old == GW - 1) {
      __threadfence_block();
      const float* rr = red + (size_t)rbuf * GW * kGRed;
      const int e = p.grp[1 + 3 * ch];
      for (int o = lane; o < kGT * 16; o += 32) {
        const int tk = o >> 4, r = o & 15, row = t * 16 + r;
        if (tk >= ntok) continue;
        float a0 = 0.f, a1 = 0.f;
#pragma unroll
        for (int w = 0; w < GW; ++w) {
          a0 += rr[w * kGRed + tk * kRedRows + r];
          if (p.mode == MODE_GATEUP) a1 += rr[w * kGRed + tk * kRedRows + 16 + r];
        }
        const size_t ent = (size_t)(ebeg + tk);
        if (p.bias0) a0 += p.bias0[(size_t)e * p.rows + row];
        if (p.mode == MODE_GATEUP) {   // activation rows by entry (the down phase's input order)
          if (p.bias1) a1 += p.bias1[(size_t)e * p.rows + row];
          p.out[ent * p.rows + row] = p.oai ? swiglu_oai(a0, a1) : silu_mul(a0, a1);
        } else {                       // expert outputs by (token, slot)
          p.out[(size_t)p.ent_slot[ent] * p.rows + row] = a0;
        }
      }
      __syncwarp();
      if (lane == 0) red_cnt[rbuf] = 0u;
    }
  }
}

size_t group_smem_bytes(int ns, int stage_bytes, int gw) {
  const int g = kCW / gw, nrbg = (ns + g - 1) / g + 1;
  return (size_t)ns * stage_bytes + (size_t)g * nrbg * gw * kGT * kRedRows * sizeof(float) + 2 * kGroupMaxStages * 8 +
         kGroupRedCnt * 4 + 16;
}

template <int FMT, int NBW, int RT, int GW>
cudaError_t launch_group(const DevCtx& c, const GroupParams& p, cudaStream_t s) {
  const size_t smem = group_smem_bytes(p.ns, p.stage_bytes, GW);
  cudaError_t e = cudaFuncSetAttribute(moe_group_kernel<FMT, NBW, RT, GW>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem);
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
  return cudaLaunchKernelEx(&cfg, moe_group_kernel<FMT, NBW, RT, GW>, p);
}

// gate_up (long K): all 16 warps on one item; down (short K): 4 items at once, 4 warps each
template <int FMT, int RT, int GW>
cudaError_t group_nbw(const DevCtx& c, const GroupParams& p, cudaStream_t s) {
  const int nbw = (p.cols / 32 + GW - 1) / GW;
  if (nbw <= 1) return launch_group<FMT, 1, RT, GW>(c, p, s);
  if (nbw <= 2) return launch_group<FMT, 2, RT, GW>(c, p, s);
  if (nbw <= 4) return launch_group<FMT, 4, RT, GW>(c, p, s);
  if (nbw <= 6) return launch_group<FMT, 6, RT, GW>(c, p, s);
  if (nbw <= 8) return launch_group<FMT, 8, RT, GW>(c, p, s);
  return cudaErrorInvalidValue;
}

int group_warps(const GroupParams& p) {   // measured: 16 for gate_up at hidden 2048, 4 for down at 768
  return (p.mode == MODE_DOWN && (p.cols / 32 + 3) / 4 <= 8) ? 4 : kCW;
}

cudaError_t dispatch_group(const DevCtx& c, const GroupParams& p, cudaStream_t s) {
  const bool gu = p.mode == MODE_GATEUP;
  if (!gu && group_warps(p) == 4) {
    if (p.fmt == FMT_MXFP4) return group_nbw<FMT_MXFP4, 1, 4>(c, p, s);
    if (p.fmt == FMT_Q4K) return group_nbw<FMT_Q4K, 1, 4>(c, p, s);
    if (p.fmt == FMT_Q6K) return group_nbw<FMT_Q6K, 1, 4>(c, p, s);
    if (p.fmt == FMT_Q6KP) return group_nbw<FMT_Q6KP, 1, 4>(c, p, s);
    return cudaErrorInvalidValue;
  }
  if (p.fmt == FMT_MXFP4) return gu ? group_nbw<FMT_MXFP4, 2, kCW>(c, p, s) : group_nbw<FMT_MXFP4, 1, kCW>(c, p, s);
  if (p.fmt == FMT_Q4K) return gu ? group_nbw<FMT_Q4K, 2, kCW>(c, p, s) : group_nbw<FMT_Q4K, 1, kCW>(c, p, s);
  if (p.fmt == FMT_Q6K) return gu ? group_nbw<FMT_Q6K, 2, kCW>(c, p, s) : group_nbw<FMT_Q6K, 1, kCW>(c, p, s);
  if (p.fmt == FMT_Q6KP) return gu ? group_nbw<FMT_Q6KP, 2, kCW>(c, p, s) : group_nbw<FMT_Q6KP, 1, kCW>(c, p, s);
  return cudaErrorInvalidValue;
}

// stages + the reduction buffers within ~220 KB
int pick_group_stages(int stage_bytes, int gw) {
  int ns = kGroupMaxStages;
  while (ns > 2 && group_smem_bytes(ns, stage_bytes, gw) > 220 * 1024) --ns;
  return ns;
}

// ---------------- router: RMSNorm + GEMV + bias + mask + top-k + softmax ----------------
// One CTA per expert row: each recomputes the RMSNorm of h (L2-resident), dots its router row
// and writes one logit; the last CTA to finish selects the top-k and the routing weights.
constexpr int kRouterThreads = 256;
constexpr int kRouterMaxE = 1024;

// Top-k selection and routing weights of one token by one warp, after every logit is written.
// Lane l holds logits l, l + 32, ... in registers (read once); ties go to the lower index, as a
// stable descending sort does (layer.rs:2346-2403).
template <int kPer>
__device__ __forceinline__ void router_select_t(const RouterArgs& a, uint32_t* err, int lane) {
  float lv[kPer];
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int i = lane + 32 * j;
    lv[j] = i < a.E ? __ldcg(&a.logits[i]) : -INFINITY;
  }
  // router entropy over the unmasked logits, and the dynamic K it selects (layer.rs:980-1011,
  // 2302-2334): exp and ln rounded from double, sums in double rounded once
  int K = a.K;
  float ent = 0.f;
  if (a.raw) {
    float rv[kPer];
    float rmx = -INFINITY;
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const int i = lane + 32 * j;
      rv[j] = i < a.E ? __ldcg(&a.raw[i]) : -INFINITY;
      rmx = fmaxf(rmx, rv[j]);
    }
    rmx = warp_max(rmx);
    double es = 0.0;
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      rv[j] = lane + 32 * j < a.E ? expcr(__fsub_rn(rv[j], rmx)) : 0.f;
      es += (double)rv[j];
    }
    const float s32 = (float)warp_sum_d(es);
    double hs = 0.0;
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const float p = __fdiv_rn(rv[j], s32);
      if (p > 0.f) hs += (double)__fmul_rn(p, (float)log((double)p));
    }
    ent = -(float)warp_sum_d(hs);
    if (a.k_hi > 0) {   // entropy_to_k
      const float hmax = (float)log((double)a.E);
      const float nrm = fminf(fmaxf(__fdiv_rn(ent, hmax), 0.f), 1.f);
      const float kf = __fadd_rn((float)a.k_lo, __fmul_rn(nrm, (float)(a.k_hi - a.k_lo)));
      K = min(max((int)roundf(kf), a.k_lo), a.k_hi);
    }
    if (lane == 0) {
      if (a.entropy) *a.entropy = ent;
      if (a.k_used) *a.k_used = K;
    }
  }
  uint32_t taken = 0u;
  float sel_v[kMaxK];
  int sel_i[kMaxK];
  for (int k = 0; k < K; ++k) {
    float best = -INFINITY;
    int bidx = 0x7fffffff;
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const int i = lane + 32 * j;
      if (i >= a.E || ((taken >> j) & 1u)) continue;
      const float v = lv[j];
      if (v > best || (v == best && i < bidx)) { best = v; bidx = i; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bidx, o);
      if (ov > best || (ov == best && oi < bidx)) { best = ov; bidx = oi; }
    }
    if (bidx == 0x7fffffff) {   // fewer selectable experts than k
      if (lane == 0) atomicOr(err, EF_BAD_INDEX);
      bidx = 0;
    }
    if ((bidx & 31) == lane) taken |= 1u << (bidx >> 5);
    sel_v[k] = best;
    sel_i[k] = bidx;
  }
  float w[kMaxK];
  if (a.softmax_weight) {              // layer.rs:2361-2372: softmax over the selected logits
    float mx = -INFINITY;
    for (int k = 0; k < K; ++k) mx = fmaxf(mx, sel_v[k]);
    double sum = 0.0;
    for (int k = 0; k < K; ++k) { w[k] = expcr(__fsub_rn(sel_v[k], mx)); }
    for (int k = 0; k < K; ++k) sum += (double)w[k];
    const float s32 = (float)sum;
    for (int k = 0; k < K; ++k) w[k] = __fdiv_rn(w[k], s32);
  } else {                              // layer.rs:2374-2394: softmax over all, then (re)normalise
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < kPer; ++j) mx = fmaxf(mx, lv[j]);
    mx = warp_max(mx);
    double sum = 0.0;
#pragma unroll
    for (int j = 0; j < kPer; ++j)
      if (lane + 32 * j < a.E) sum += (double)expcr(__fsub_rn(lv[j], mx));
    const float s32 = (float)warp_sum_d(sum);
    double ts = 0.0;
    for (int k = 0; k < K; ++k) { w[k] = __fdiv_rn(expcr(__fsub_rn(sel_v[k], mx)), s32); }
    for (int k = 0; k < K; ++k) ts += (double)w[k];
    const float t32 = (float)ts;
    if (a.normalize) for (int k = 0; k < K; ++k) w[k] = __fdiv_rn(w[k], t32);
  }
  if (lane == 0) {
    for (int k = 0; k < K; ++k) { a.idx[k] = sel_i[k]; a.wts[k] = w[k]; }
    for (int k = K; k < a.K; ++k) { a.idx[k] = a.E; a.wts[k] = 0.f; }   // slots past a dynamic K: none
    if (a.cnt) {   // running routing and entropy statistics, in step order (one thread)
      *a.tokens += 1ull;
      for (int k = 0; k < K; ++k) {
        a.cnt[sel_i[k]] += 1ull;
        a.wsum[sel_i[k]] += (double)w[k];
      }
      const uint32_t n = *a.ent_n;
      if ((int)n < a.ent_cap) {
        a.ent_log[(size_t)n * a.ent_stride] = ent;
        *a.ent_n = n + 1u;
      }
    }
    *a.counter = 0u;
  }
}

// logits per lane sized to the expert count
__device__ __forceinline__ void router_select(const RouterArgs& a, uint32_t* err, int lane) {
  const int per = (a.E + 31) / 32;
  if (per <= 1) router_select_t<1>(a, err, lane);
  else if (per <= 4) router_select_t<4>(a, err, lane);
  else if (per <= 8) router_select_t<8>(a, err, lane);
  else if (per <= 16) router_select_t<16>(a, err, lane);
  else router_select_t<kRouterMaxE / 32>(a, err, lane);
}

// One CTA per expert row.  Before waiting for the previous kernel the CTA starts a bulk copy of
// its router row into shared memory; then it normalises h (RMSNorm, h read twice, the second
// time from L1), dots its row and writes one logit; CTAs 0.. also write the normed x as the
// expert GEMVs' activation terms.  The last CTA to finish selects the top-k with one warp.
__global__ void __launch_bounds__(kRouterThreads) router_kernel(RouterArgs a, uint32_t* err, int row_async) {
  extern __shared__ __align__(16) float wrow[];   // [H] this expert's router row
  __shared__ __align__(8) uint64_t bar;
  __shared__ uint32_t last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int e = blockIdx.x;
  const float* wr = a.w + (size_t)e * a.H;
  if (row_async && threadIdx.x == 0) {   // weights do not depend on the previous kernel
    mbar_init(&bar, 1);
    fence_mbar_init();
    mbar_expect_tx(&bar, (uint32_t)a.H * 4u);
    bulk_g2s(wrow, wr, (uint32_t)a.H * 4u, &bar);
  }
  pdl_wait_prior();
  pdl_launch_dependents();   // the next kernel may start its own (weight) prefetch now
  double dot = 0.0;
  float inv = 1.f;
  // (the barriers of the RMSNorm also publish the mbarrier's initialisation)
  if (a.h) inv = rms_inv_cr(a.h, a.H, a.eps, threadIdx.x, kRouterThreads, [] { __syncthreads(); });
  else __syncthreads();
  bool row_ok = true;
  if (row_async) row_ok = mbar_wait(&bar, 0, err, EF_TIMEOUT_FULL);
  const float* wsrc = row_async ? wrow : wr;
  if (row_ok) {
    for (int i = threadIdx.x; i < a.H; i += kRouterThreads) {
      const float v = a.h ? __fmul_rn(__fmul_rn(a.h[i], inv), a.norm_w[i]) : a.xn[i];
      if (a.h && e == 0) a.xn[i] = v;
      dot = fma((double)v, (double)wsrc[i], dot);
    }
  }
  dot = warp_sum_d(dot);
  __shared__ double redd[kRouterThreads / 32];
  if (lane == 0) redd[warp] = dot;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int w = 0; w < kRouterThreads / 32; ++w) t += redd[w];
    float v = (float)t;
    if (a.b) v = __fadd_rn(v, a.b[e]);
    if (a.raw) a.raw[e] = v;   // before the dummy mask (the reference's entropy sees these)
    if (a.mask && a.mask[e]) v = -INFINITY;
    a.logits[e] = v;
    __threadfence();
    last = (atomicAdd(a.counter, 1u) == gridDim.x - 1) ? 1u : 0u;
  }
  if (a.xterm) {
    // the normed x as the expert GEMVs' B terms: warp w of CTA e takes 32-element blocks
    // e*8 + w, e*8 + w + 8*E, ... (same arithmetic as xn above, so the terms encode xn exactly)
    const int nb = a.H / 32, nw = kRouterThreads / 32;
    for (int b = e * nw + warp; b < nb; b += (int)gridDim.x * nw) {
      const int i = 32 * b + lane;
      const float v = a.h ? __fmul_rn(__fmul_rn(a.h[i], inv), a.norm_w[i]) : a.xn[i];
      umma::quantize_terms_warp(v, lane, a.xterm, nb, b);
    }
  }
  if (a.xbt) {   // the same blocks as exact B terms
    const int nb = a.H / 32, nw = kRouterThreads / 32;
    for (int b = e * nw + warp; b < nb; b += (int)gridDim.x * nw) {
      const int i = 32 * b + lane;
      const float v = a.h ? __fmul_rn(__fmul_rn(a.h[i], inv), a.norm_w[i]) : a.xn[i];
      exact_bterm_warp(v, lane, a.xbt + (size_t)b * kExactBlock, b & 1, a.xfe + b);
    }
  }
  __syncthreads();
  if (!last || warp != 0) return;
  __threadfence();
  router_select(a, err, lane);
}

// Batched router: grid (ceil(E / kRBRows), tokens).  Each CTA normalises its token's h into
// shared memory and dots kRBRows router rows (a warp per row, float4 loads); the last CTA of a
// token selects its top-k.
constexpr int kRBRows = 16;
__global__ void __launch_bounds__(kRouterThreads) router_batch_kernel(RouterArgs a, uint32_t* err) {
  extern __shared__ __align__(16) float xs[];   // [H] normed input
  __shared__ uint32_t last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.y;
  a.h += (size_t)b * a.H;
  a.xn += (size_t)b * a.H;
  a.logits += (size_t)b * a.E;
  a.idx += b * a.K;
  a.wts += b * a.K;
  a.counter += b;
  pdl_wait_prior();
  pdl_launch_dependents();
  const float inv = rms_inv_cr(a.h, a.H, a.eps, threadIdx.x, kRouterThreads, [] { __syncthreads(); });
  for (int i = threadIdx.x; i < a.H; i += kRouterThreads) {
    const float v = __fmul_rn(__fmul_rn(a.h[i], inv), a.norm_w[i]);
    xs[i] = v;
    if (blockIdx.x == 0) a.xn[i] = v;
  }
  __syncthreads();
  for (int r = warp; r < kRBRows; r += kRouterThreads / 32) {
    const int e = blockIdx.x * kRBRows + r;
    if (e >= a.E) break;
    const float4* w4 = reinterpret_cast<const float4*>(a.w + (size_t)e * a.H);
    const float4* x4 = reinterpret_cast<const float4*>(xs);
    double dot = 0.0;
    for (int i = lane; i < a.H / 4; i += 32) {
      const float4 w = __ldg(w4 + i), x = x4[i];
      dot = fma((double)x.x, (double)w.x, dot);
      dot = fma((double)x.y, (double)w.y, dot);
      dot = fma((double)x.z, (double)w.z, dot);
      dot = fma((double)x.w, (double)w.w, dot);
    }
    dot = warp_sum_d(dot);
    if (lane == 0) {
      float v = (float)dot;
      if (a.b) v = __fadd_rn(v, a.b[e]);
      if (a.mask && a.mask[e]) v = -INFINITY;
      a.logits[e] = v;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    last = (atomicAdd(a.counter, 1u) == gridDim.x - 1) ? 1u : 0u;
  }
  __syncthreads();
  if (!last || warp != 0) return;
  __threadfence();
  router_select(a, err, lane);
}

}  // namespace

cudaError_t launch_block_gemv(const DevCtx& c, int qtype, const uint8_t* w, int rows, int cols, const float* x,
                              const float* bias, float* y, int accumulate, cudaStream_t s) {
  // rows are streamed in 16-row tiles; the weight allocation must be padded to a whole tile
  const int fmt = fmt_of(qtype);
  const int rb = (int)row_bytes(qtype, cols);
  if (fmt < 0 || rb <= 0 || rows <= 0) return cudaErrorInvalidValue;
  if ((16 * rb) % 16) return cudaErrorInvalidValue;
  PhaseParams p = {};
  p.mode = MODE_PLAIN; p.fmt = fmt; p.w0 = w; p.expert_stride = 0; p.rb = rb; p.cols = cols; p.rows = rows;
  p.tile_rows = 16; p.n_tiles = (rows + 15) / 16; p.rs = stage_row_stride(rb); p.stage_bytes = 16 * p.rs;
  p.ns = pick_stages(p.stage_bytes);
  p.x = x; p.bias0 = bias; p.out = y; p.accumulate = accumulate; p.K = 1; p.err = c.err;
  return dispatch_phase(c, p, s);
}

size_t moe_mxfp4_smem_bytes(int H, int I) {
  const int rbg = H / 32 * 17;
  return (size_t)pick_stages(16 * rbg) * 16 * rbg;
}

__global__ void moe_combine_kernel(PendingCombine pc, int H, float* h, float* out) {
  __shared__ CombineOrder co;
  pdl_wait_prior();
  pdl_launch_dependents();   // the next kernel may start its own (weight) prefetch now
  if (threadIdx.x == 0) combine_order(pc, &co);
  __syncthreads();
  combine_prepare(pc, &co);
  __syncthreads();
  for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < H; r += gridDim.x * blockDim.x) {
    const float v = combine_at(pc, co, H, r);
    if (out) out[r] = v;
    else h[r] = h[r] + v;
  }
}

cudaError_t launch_moe_combine(const DevCtx& c, const PendingCombine& pc, int H, float* h, float* out,
                               cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((H + 255) / 256));
  cfg.blockDim = dim3(256);
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, moe_combine_kernel, pc, H, h, out);
}

cudaError_t launch_router(const DevCtx& c, const RouterArgs& a, cudaStream_t s) {
  if (a.raw && (a.batch != 1 || (a.k_hi > 0 && (a.k_lo < 1 || a.k_lo > a.k_hi || a.k_hi > a.K))))
    return cudaErrorInvalidValue;
  if (a.cnt && (!a.raw || !a.wsum || !a.tokens || !a.ent_log || !a.ent_n || a.ent_stride < 1))
    return cudaErrorInvalidValue;
  if (a.K < 1 || a.K > kMaxK || a.K > a.E || a.E > kRouterMaxE || !a.counter || a.batch < 1 ||
      (a.batch > 1 && (a.xterm || a.xbt)) || (a.xbt && (a.H % 32 || !a.xfe)))
    return cudaErrorInvalidValue;
  if (a.batch > 1) {
    if (a.H % 4 || !a.h || reinterpret_cast<uintptr_t>(a.w) % 16) return cudaErrorInvalidValue;
    const size_t smem = (size_t)a.H * 4;
    cudaError_t e = cudaFuncSetAttribute(router_batch_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((a.E + kRBRows - 1) / kRBRows), (unsigned)a.batch);
    cfg.blockDim = dim3(kRouterThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, router_batch_kernel, a, c.err);
  }
  cudaLaunchConfig_t cfg = {};
  // the router row goes to shared memory by a bulk copy when it is 16-byte aligned (all rows are
  // when the matrix is and H % 4 == 0)
  const int row_async = (reinterpret_cast<uintptr_t>(a.w) % 16 == 0 && a.H % 4 == 0 && a.H <= 12288) ? 1 : 0;
  const size_t smem = row_async ? (size_t)a.H * 4 : 0;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(router_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  cfg.gridDim = dim3((unsigned)a.E);
  cfg.blockDim = dim3(kRouterThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, router_kernel, a, c.err, row_async);
}

cudaError_t launch_moe_mxfp4(const DevCtx& c, const MoeArgs& a, cudaStream_t s) {
  if (a.K < 1 || a.K > kMaxK || a.H % 64 || a.I % 32 || a.n_local < 0) return cudaErrorInvalidValue;
  const int fg = fmt_of(a.gate_q), fd = fmt_of(a.down_q);
  if (fg < 0 || fd < 0) return cudaErrorInvalidValue;
  const int rbg = (int)row_bytes(a.gate_q, a.H);   // gate/up row bytes
  const int rbd = (int)row_bytes(a.down_q, a.I);   // down row bytes
  if (rbg <= 0 || rbd <= 0) return cudaErrorInvalidValue;
  PhaseParams p = {};
  p.K = a.K; p.idx = a.idx; p.wts = a.wts; p.expert_base = a.expert_base; p.n_local = a.n_local;
  p.oai = a.oai_swiglu; p.err = c.err;
  // phase 1: gate + up + activation
  p.mode = MODE_GATEUP; p.fmt = fg; p.w0 = a.gate; p.w1 = a.up; p.expert_stride = (int64_t)a.I * rbg; p.rb = rbg;
  p.cols = a.H; p.rows = a.I; p.tile_rows = 16; p.n_tiles = a.I / 16; p.rs = stage_row_stride(rbg);
  p.stage_bytes = 32 * p.rs;
  p.ns = pick_stages(p.stage_bytes); p.x = a.x; p.bias0 = a.gate_b; p.bias1 = a.up_b; p.act = a.act;
  if ((16 * rbg) % 16 || p.expert_stride % 16 || a.I % 16 || a.H % 16) return cudaErrorInvalidValue;
  cudaError_t e = dispatch_phase(c, p, s);
  if (e != cudaSuccess) return e;
  // phase 2: down -> per-slot partial rows
  p.mode = MODE_DOWN; p.fmt = fd; p.w0 = a.down; p.w1 = nullptr; p.expert_stride = (int64_t)a.H * rbd; p.rb = rbd;
  p.cols = a.I; p.rows = a.H; p.tile_rows = 16; p.n_tiles = a.H / 16; p.rs = stage_row_stride(rbd);
  p.stage_bytes = 16 * p.rs;
  p.ns = pick_stages(p.stage_bytes); p.x = a.act; p.bias0 = a.down_b; p.bias1 = nullptr;
  p.partial = a.partial; p.tile_cnt = a.tile_cnt; p.h = a.h; p.out = a.out;
  if ((16 * rbd) % 16 || p.expert_stride % 16) return cudaErrorInvalidValue;
  e = dispatch_phase(c, p, s);
  if (e != cudaSuccess || a.defer_combine) return e;
  PendingCombine pc;
  pc.partial = a.partial; pc.idx = a.idx; pc.wts = a.wts; pc.K = a.K; pc.expert_base = a.expert_base;
  pc.n_local = a.n_local;
  return launch_moe_combine(c, pc, a.H, a.h, a.out, s);
}

int group_table_words(int B, int K) { return 1 + 3 * B * K; }

cudaError_t launch_moe_group(const DevCtx& c, const GroupMoeArgs& a, int part, cudaStream_t s) {
  const int n_ent = a.B * a.K;
  if (a.B < 1 || a.B > kMaxBatch || a.K < 1 || a.K > kMaxK || a.n_local < 0 || a.n_local > kRouteThreads ||
      a.H % 64 || a.I % 32)
    return cudaErrorInvalidValue;
  const int fg = fmt_of(a.gate_q), fd = fmt_of(a.down_q);
  if (fg < 0 || fd < 0) return cudaErrorInvalidValue;
  const int rbg = (int)row_bytes(a.gate_q, a.H), rbd = (int)row_bytes(a.down_q, a.I);
  if (rbg <= 0 || rbd <= 0) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(kRouteThreads);
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  if (part == 0)
    return cudaLaunchKernelEx(&cfg, group_route_kernel, a.idx, n_ent, a.K, a.expert_base, a.n_local, a.grp,
                              a.ent_slot, a.ent_of, c.err);
  GroupParams p = {};
  p.grp = a.grp; p.ent_slot = a.ent_slot; p.K = a.K; p.oai = a.oai_swiglu; p.err = c.err;
  p.mode = MODE_GATEUP; p.fmt = fg; p.w0 = a.gate; p.w1 = a.up; p.expert_stride = (int64_t)a.I * rbg; p.rb = rbg;
  p.cols = a.H; p.rows = a.I; p.n_tiles = a.I / 16; p.rs = stage_row_stride(rbg); p.stage_bytes = 32 * p.rs;
  p.ns = pick_group_stages(p.stage_bytes, group_warps(p));
  p.x = a.x; p.bias0 = a.gate_b; p.bias1 = a.up_b; p.out = a.act;
  if ((16 * rbg) % 16 || p.expert_stride % 16 || a.I % 16) return cudaErrorInvalidValue;
  if (part == 1) return dispatch_group(c, p, s);
  p.mode = MODE_DOWN; p.fmt = fd; p.w0 = a.down; p.w1 = nullptr; p.expert_stride = (int64_t)a.H * rbd; p.rb = rbd;
  p.cols = a.I; p.rows = a.H; p.n_tiles = a.H / 16; p.rs = stage_row_stride(rbd); p.stage_bytes = 16 * p.rs;
  p.ns = pick_group_stages(p.stage_bytes, group_warps(p));
  p.x = a.act; p.bias0 = a.down_b; p.bias1 = nullptr; p.out = a.y;
  if ((16 * rbd) % 16 || p.expert_stride % 16) return cudaErrorInvalidValue;
  return dispatch_group(c, p, s);
}

}  // namespace ms
