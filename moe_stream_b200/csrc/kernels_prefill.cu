// kernels_prefill.cu — batched prefill: MXFP4 expert FFN as a grouped GEMM on the 5th-generation
// tensor cores (sm_100a), bf16 operands, f32 accumulation.
//
// Reference semantics (moe-stream-core/src): multi-token expert FFN, tokens grouped by expert and
// scattered back in ascending expert order (model/layer.rs:1316-1349, 1848-1894); OAI SwiGLU
// (ops/activation.rs:25-38); MXFP4 values (gguf/dequant.rs:580-628).  The reference runs a
// per-expert f32 matmul; here every step is a tensor-core GEMM whose only rounding is bf16 on the
// activations (the MXFP4 weights are exact in bf16).
//
// Flow (one MoE layer, T tokens, top-K):
//   pf_route_kernel    one CTA per local expert lists its (token, k) entries in token order
//   pf_gather_kernel   tokens of each expert -> bf16 in the operand layout, tiles of 256 tokens
//   pf_gemm_kernel<0>  gate_up: [128 weight rows] x [256 tokens] per item; SwiGLU epilogue writes
//                      the activation in the down GEMM's operand layout
//   pf_gemm_kernel<1>  down: routing-weighted expert outputs per (token, k)
//   pf_combine_kernel  out[t] = sum over k in ascending expert order
//
// Operand layout (K-major, no swizzle, as umma.cuh): a matrix of R rows is stored as K/8 chunk
// columns of R rows x 16 bytes (8 bf16).  Weights stay in the decode path's packed MXFP4 tiles;
// per K = 64 stage, 8 dequant warps expand the stage's codes to bf16 chunk columns in shared memory
// (value = e2m1 * 2^(E-127), exact in bf16) while the tensor core consumes the previous stage.
// Warp roles: 0 producer (1-D bulk copies), 1 MMA issuer + tensor-memory owner, 2-5 epilogue
// (double-buffered accumulators), 6-13 dequant.  Every wait is bounded.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "common.cuh"
#include "kernels.h"
#include "umma.cuh"

namespace ms {
namespace {

constexpr int kPfN = 256;                  // tokens per tile (MMA N)
constexpr int kPfCh = 2;                   // MXFP4 chunks per stage (K = 64)
constexpr int kPfStA = kPfCh * 2048;       // MXFP4 codes of a stage: 2 chunks x 128 rows x 16 B
constexpr int kPfStSF = 512;               // the scale group holding them
constexpr int kPfStB = 4 * kPfCh * kPfN * 16;   // tokens: 8 bf16 chunk columns x 256 rows x 16 B
constexpr int kPfABf = 4 * kPfCh * 128 * 16;    // dequantized weights of a stage
// PREC = 1 ("precise"): every token operand is a bf16 pair hi + lo (hi = bf16(x), lo = bf16(x - hi),
// |x - hi - lo| <= 2^-18 |x|) and each K step issues two MMAs into the same f32 accumulator, so the
// activations carry ~17 significant bits instead of 8 (the weights are exact in bf16 either way).
template <int PREC> struct PfCfg {
  static constexpr int kStage = kPfStA + kPfStSF + (PREC ? 2 : 1) * kPfStB;
  static constexpr int kStages = PREC ? 2 : 4;
};
constexpr int kPfUpLd = 33;                // padded row of the up-row exchange buffer (no bank conflicts)
constexpr int kPfThreads = 14 * 32;
constexpr int kPfDeqThreads = 8 * 32;
constexpr int kPfTmemCols = 512;           // two 256-column accumulators
constexpr int kPfMaxE = 256;
template <int PREC>
constexpr int pf_smem() { return PfCfg<PREC>::kStages * (PfCfg<PREC>::kStage + kPfABf) + 64 * kPfUpLd * 4; }

struct PfParams {
  int mode;                  // 0 gate_up, 1 down
  const uint8_t* w;          // packed MXFP4 tiles [E][tiles][tile_bytes]
  int64_t tile_bytes;
  int tiles, kc;             // weight tiles per expert; K / 32
  const uint8_t* b;          // token operand tiles: [tile][K / 8][256][16 B] bf16
  const uint8_t* b_lo;       // precise mode: the low bf16 halves, same layout
  const int* count;          // [E] tokens per expert
  const int* list;           // [E][T] (t * K + k) entries in token order
  int E, T, K, H, I;
  const float* bias0;        // gate_b / down_b
  const float* bias1;        // up_b
  const float* wts;          // [T * K] routing weights (down)
  uint8_t* act;              // gate_up output: token operand tiles of the activation
  uint8_t* act_lo;           // precise mode: their low halves
  float* y;                  // down output [T * K][H]
  int oai;
  uint32_t* err;
};

__device__ __forceinline__ float swiglu_pf(float g, float u) {   // ops/activation.rs:25-45
  const float gc = fminf(g, 7.0f);
  const float uc = fminf(fmaxf(u, -7.0f), 7.0f);
  const float sig = 1.0f / (expf(-(gc * 1.702f)) + 1.0f);
  return (gc * sig) * (uc + 1.0f);
}

// per-expert 256-token tile offsets, computed in shared memory by every CTA (E <= kPfMaxE)
__device__ __forceinline__ void pf_tile_offsets(const int* count, int E, int* off) {
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int e = 0; e < E; ++e) { off[e] = acc; acc += (count[e] + kPfN - 1) / kPfN; }
    off[E] = acc;
  }
  __syncthreads();
}

// ---------------- routing: one CTA per local expert, entries in token order ----------------
__global__ void __launch_bounds__(256) pf_route_kernel(const int* idx, int T, int K, int expert_base, int E,
                                                       int* count, int* list) {
  __shared__ int warp_cnt[8];
  __shared__ int base;
  const int e = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) base = 0;
  __syncthreads();
  const int n = T * K;
  for (int c0 = 0; c0 < n; c0 += 256) {
    const int i = c0 + threadIdx.x;
    const bool hit = i < n && idx[i] - expert_base == e;
    const unsigned m = __ballot_sync(0xffffffffu, hit);
    if (lane == 0) warp_cnt[warp] = __popc(m);
    __syncthreads();
    int before = base;
    for (int w = 0; w < warp; ++w) before += warp_cnt[w];
    if (hit) list[(size_t)e * T + before + __popc(m & ((1u << lane) - 1u))] = i;
    __syncthreads();
    if (threadIdx.x == 0) for (int w = 0; w < 8; ++w) base += warp_cnt[w];
    __syncthreads();
  }
  if (threadIdx.x == 0) count[e] = base;
}

// ---------------- gather: x [T][H] f32 -> bf16 token tiles [tile][H/8][256][8] ----------------
__global__ void pf_gather_kernel(const float* __restrict__ x, int H, int K, const int* count, const int* list, int E,
                                 int T, uint8_t* __restrict__ b, uint8_t* __restrict__ b_lo) {
  __shared__ int off[kPfMaxE + 1];
  pf_tile_offsets(count, E, off);
  const int nch = H / 8;
  const int64_t total = (int64_t)off[E] * nch * kPfN;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int row = (int)(i % kPfN);
    int64_t q = i / kPfN;
    const int ch = (int)(q % nch);
    const int tile = (int)(q / nch);
    int e = 0;
    while (e + 1 < E && off[e + 1] <= tile) ++e;
    const int pos = (tile - off[e]) * kPfN + row;
    uint4 v = make_uint4(0u, 0u, 0u, 0u), vl = v;
    if (pos < count[e]) {
      const int t = list[(size_t)e * T + pos] / K;
      const float4* src = reinterpret_cast<const float4*>(x + (size_t)t * H + 8 * ch);
      const float4 a = src[0], c = src[1];
      const float f[8] = {a.x, a.y, a.z, a.w, c.x, c.y, c.z, c.w};
      uint32_t hw[4], lw[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const __nv_bfloat162 hi = __floats2bfloat162_rn(f[2 * q], f[2 * q + 1]);
        const float2 hf = __bfloat1622float2(hi);
        const __nv_bfloat162 lo = __floats2bfloat162_rn(f[2 * q] - hf.x, f[2 * q + 1] - hf.y);
        hw[q] = *reinterpret_cast<const uint32_t*>(&hi);
        lw[q] = *reinterpret_cast<const uint32_t*>(&lo);
      }
      v = make_uint4(hw[0], hw[1], hw[2], hw[3]);
      vl = make_uint4(lw[0], lw[1], lw[2], lw[3]);
    }
    const int64_t o = ((int64_t)tile * nch + ch) * (kPfN * 16) + row * 16;
    *reinterpret_cast<uint4*>(b + o) = v;
    if (b_lo) *reinterpret_cast<uint4*>(b_lo + o) = vl;
  }
}

// ---------------- combine: out[t] = sum over k (ascending expert id) of y[t*K+k] ----------------
__global__ void pf_combine_kernel(const float* __restrict__ y, const int* idx, int K, int expert_base, int E, int H,
                                  float* __restrict__ out, int accumulate) {
  __shared__ int order[16];
  __shared__ int n;
  const int t = blockIdx.x;
  if (threadIdx.x == 0) {
    int m = 0;
    for (int k = 0; k < K; ++k) {
      const int e = idx[t * K + k] - expert_base;
      if (e < 0 || e >= E) continue;
      int j = m++;
      while (j > 0 && idx[t * K + order[j - 1]] > idx[t * K + k]) { order[j] = order[j - 1]; --j; }
      order[j] = k;
    }
    n = m;
  }
  __syncthreads();
  for (int h = threadIdx.x; h < H; h += blockDim.x) {
    float acc = 0.f;
    for (int j = 0; j < n; ++j) acc += y[((size_t)t * K + order[j]) * H + h];
    out[(size_t)t * H + h] = accumulate ? out[(size_t)t * H + h] + acc : acc;
  }
}

// ---------------- grouped GEMM ----------------
template <int MODE, int PREC>
__global__ void __launch_bounds__(kPfThreads, 1) pf_gemm_kernel(const __grid_constant__ PfParams p) {
  constexpr int kPfStages = PfCfg<PREC>::kStages, kPfStage = PfCfg<PREC>::kStage;
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t* stage_base = smem;                                   // [kPfStages][kPfStage]
  uint8_t* abf_base = smem + kPfStages * kPfStage;              // [kPfStages][kPfABf]
  float* s_up = reinterpret_cast<float*>(abf_base + kPfStages * kPfABf);   // [64][33] up rows of a column block
  __shared__ __align__(8) uint64_t full[kPfStages], empty[kPfStages], deq[kPfStages], acc_full[2], acc_empty[2];
  __shared__ uint32_t tmem_base;
  __shared__ int off[kPfMaxE + 1];
  __shared__ int s_abort;
  __shared__ int s_ent[kPfN];
  __shared__ float s_w[kPfN];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kPfStages; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); mbar_init(&deq[s], kPfDeqThreads); }
    for (int a = 0; a < 2; ++a) { mbar_init(&acc_full[a], 1); mbar_init(&acc_empty[a], 128); }
    fence_mbar_init();
    s_abort = 0;
  }
  if (warp == 1) { umma::tmem_alloc(&tmem_base, kPfTmemCols); umma::tmem_relinquish(); }
  umma::fence_before_sync();
  pf_tile_offsets(p.count, p.E, off);   // (contains the block barrier)
  umma::fence_after_sync();
  const uint32_t tb = tmem_base;
  const int n_items = off[p.E] * p.tiles;
  const int KW = (p.kc + kPfCh - 1) / kPfCh;   // stages per item
  const int nch_b = p.kc * 4;           // bf16 chunk columns of the token operand (K / 8)

  if (warp == 0) {
    // ---------------- producer ----------------
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      int j = 0;
      for (int it = blockIdx.x; it < n_items && !*reinterpret_cast<volatile int*>(&s_abort); it += gridDim.x) {
        const int tile = it / p.tiles, mt = it % p.tiles;
        int e = 0;
        while (e + 1 < p.E && off[e + 1] <= tile) ++e;
        const uint8_t* wt = p.w + ((int64_t)e * p.tiles + mt) * p.tile_bytes;
        const uint8_t* bt = p.b + (int64_t)tile * nch_b * (kPfN * 16);
        for (int w = 0; w < KW; ++w) {
          const int s = j % kPfStages, n = j / kPfStages;
          if (n > 0 && !mbar_wait(&empty[s], (uint32_t)((n - 1) & 1), p.err, EF_TIMEOUT_EMPTY)) { s_abort = 1; break; }
          const int c0 = kPfCh * w, c1 = min(p.kc, c0 + kPfCh), slab = c0 / 16, sl0 = slab * 16, nchs = min(16, p.kc - sl0);
          const uint8_t* sb = wt + (int64_t)slab * (16 * 2048 + 4 * 512);
          uint8_t* sp = stage_base + (size_t)s * kPfStage;
          const uint32_t ab = (uint32_t)(c1 - c0) * 2048u, bb = (uint32_t)(c1 - c0) * 4u * kPfN * 16u;
          mbar_expect_tx(&full[s], ab + 512u + (PREC ? 2u : 1u) * bb);
          bulk_g2s_stream(sp, sb + (int64_t)(c0 - sl0) * 2048, ab, &full[s], pol);
          bulk_g2s_stream(sp + kPfStA, sb + (int64_t)nchs * 2048 + ((c0 - sl0) >> 2) * 512, 512u, &full[s], pol);
          bulk_g2s(sp + kPfStA + kPfStSF, bt + (int64_t)(4 * c0) * (kPfN * 16), bb, &full[s]);
          if (PREC)
            bulk_g2s(sp + kPfStA + kPfStSF + kPfStB,
                     p.b_lo + (int64_t)tile * nch_b * (kPfN * 16) + (int64_t)(4 * c0) * (kPfN * 16), bb, &full[s]);
          ++j;
        }
      }
      for (int q = max(0, j - kPfStages); q < j; ++q)
        mbar_wait(&full[q % kPfStages], (uint32_t)((q / kPfStages) & 1), p.err, EF_TIMEOUT_FULL);
    }
  } else if (warp >= 6) {
    // ---------------- dequant: MXFP4 codes -> exact bf16 chunk columns ----------------
    const int dt = threadIdx.x - 6 * 32, r = dt & 127, half = dt >> 7;   // row, which of the 2 chunks
    int j = 0;
    for (int it = blockIdx.x; it < n_items; it += gridDim.x) {
      for (int w = 0; w < KW; ++w, ++j) {
        const int s = j % kPfStages;
        const bool ok = mbar_wait(&full[s], (uint32_t)((j / kPfStages) & 1), p.err, EF_TIMEOUT_FULL);
        const uint8_t* sp = stage_base + (size_t)s * kPfStage;
        uint8_t* ab = abf_base + (size_t)s * kPfABf;
        const int nchunk = min(p.kc - kPfCh * w, kPfCh);
        if (ok) {
          for (int cl = half; cl < half + 1 && cl < nchunk; ++cl) {
            const uint4 codes = *reinterpret_cast<const uint4*>(sp + cl * 2048 + r * 16);
            const uint32_t eb = sp[kPfStA + 16 * (r & 31) + 4 * (r >> 5) + ((kPfCh * w + cl) & 3)];
            const float sc = __uint_as_float(eb ? eb << 23 : 0x00400000u);   // 2^(E-127)
            const uint32_t cw[4] = {codes.x, codes.y, codes.z, codes.w};
#pragma unroll
            for (int q = 0; q < 4; ++q) {   // 4 bytes = 8 elements = one bf16 chunk column
              uint32_t o[4];
#pragma unroll
              for (int bi = 0; bi < 4; ++bi) {
                const uint32_t h2 = e2m1x2_to_f16x2((cw[q] >> (8 * bi)) & 0xFFu);
                const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&h2));
                const __nv_bfloat162 bv = __floats2bfloat162_rn(f.x * sc, f.y * sc);
                o[bi] = *reinterpret_cast<const uint32_t*>(&bv);
              }
              *reinterpret_cast<uint4*>(ab + (4 * cl + q) * 2048 + r * 16) = make_uint4(o[0], o[1], o[2], o[3]);
            }
          }
        }
        umma::fence_proxy_async_smem();   // these writes are read by the tensor core
        mbar_arrive(&deq[s]);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      int j = 0, seg = 0;
      const uint32_t idesc = umma::idesc_bf16(128, kPfN);
      for (int it = blockIdx.x; it < n_items && !*reinterpret_cast<volatile int*>(&s_abort); it += gridDim.x, ++seg) {
        const int a = seg & 1;
        if (seg >= 2 && !mbar_wait(&acc_empty[a], (uint32_t)(((seg >> 1) - 1) & 1), p.err, EF_TIMEOUT_EMPTY)) {
          s_abort = 1;
          break;
        }
        umma::fence_after_sync();
        const uint32_t d = tb + (uint32_t)(a * kPfN);
        int nmma = 0;
        for (int w = 0; w < KW; ++w, ++j) {
          const int s = j % kPfStages;
          if (!mbar_wait(&deq[s], (uint32_t)((j / kPfStages) & 1), p.err, EF_TIMEOUT_FULL)) { s_abort = 1; break; }
          umma::fence_after_sync();
          const uint8_t* ab = abf_base + (size_t)s * kPfABf;
          const uint8_t* bb = stage_base + (size_t)s * kPfStage + kPfStA + kPfStSF;
          const int nk = 2 * min(p.kc - kPfCh * w, kPfCh);   // MMAs of K = 16 (two bf16 chunk columns each)
          for (int k = 0; k < nk; ++k) {
            const uint64_t ad = umma::smem_desc(ab + 2 * k * 2048, 2048, 128);
            const uint64_t bd = umma::smem_desc(bb + 2 * k * (kPfN * 16), kPfN * 16, 128);
            umma::mma_bf16(d, ad, bd, idesc, nmma > 0);
            ++nmma;
            if (PREC) {   // the low halves of the same token columns, same weights
              const uint64_t bl = umma::smem_desc(bb + kPfStB + 2 * k * (kPfN * 16), kPfN * 16, 128);
              umma::mma_bf16(d, ad, bl, idesc, 1);
            }
          }
          umma::commit(&empty[s]);
        }
        umma::commit(&acc_full[a]);
      }
    }
  } else {
    // ---------------- epilogue (warps 2-5: TMEM lane quadrants 2, 3, 0, 1) ----------------
    const int quad = warp & 3, row = 32 * quad + lane;
    int seg = 0;
    for (int it = blockIdx.x; it < n_items; it += gridDim.x, ++seg) {
      const int tile = it / p.tiles, mt = it % p.tiles;
      int e = 0;
      while (e + 1 < p.E && off[e + 1] <= tile) ++e;
      const int tok0 = (tile - off[e]) * kPfN, cnt = p.count[e];
      const int a = seg & 1;
      const bool ok = mbar_wait(&acc_full[a], (uint32_t)((seg >> 1) & 1), p.err, EF_TIMEOUT_FULL);
      umma::fence_after_sync();
      if (MODE == 0) {
        const int r = row & 63;                         // activation row within the tile
        const int ai = mt * 64 + r;                     // activation index
        const float bg = p.bias0 ? p.bias0[(int64_t)e * p.I + ai] : 0.f;
        const float bu = p.bias1 ? p.bias1[(int64_t)e * p.I + ai] : 0.f;
        const int64_t ao = (int64_t)tile * (p.I / 8) * (kPfN * 16) + (int64_t)(ai >> 3) * (kPfN * 16) + (ai & 7) * 2;
        uint8_t* at = p.act + ao;
        uint8_t* atl = PREC ? p.act_lo + ao : nullptr;
        for (int cb = 0; cb < kPfN / 32; ++cb) {
          float v[32];
          umma::ld_32x32b_x32(tb + ((uint32_t)(32 * quad) << 16) + (uint32_t)(a * kPfN + cb * 32), v);
          if (row >= 64) {
#pragma unroll
            for (int n = 0; n < 32; ++n) s_up[r * kPfUpLd + n] = v[n];
          }
          named_bar(1, 128);
          if (row < 64 && ok) {
#pragma unroll
            for (int n = 0; n < 32; ++n) {
              const float av = p.oai ? swiglu_pf(v[n] + bg, s_up[r * kPfUpLd + n] + bu)
                                     : ((v[n] + bg) / (1.0f + expf(-(v[n] + bg)))) * (s_up[r * kPfUpLd + n] + bu);
              const __nv_bfloat16 hi = __float2bfloat16_rn(av);
              *reinterpret_cast<__nv_bfloat16*>(at + (cb * 32 + n) * 16) = hi;
              if (PREC) *reinterpret_cast<__nv_bfloat16*>(atl + (cb * 32 + n) * 16) = __float2bfloat16_rn(av - __bfloat162float(hi));
            }
          }
          named_bar(1, 128);
        }
      } else {
        // the tile's (token, k) entries and routing weights, read once
        named_bar(1, 128);
        for (int n = row; n < kPfN; n += 128) {
          const int pos = tok0 + n;
          const int ent = pos < cnt ? p.list[(size_t)e * p.T + pos] : -1;
          s_ent[n] = ent;
          s_w[n] = ent >= 0 ? p.wts[ent] : 0.f;
        }
        named_bar(1, 128);
        const int hr = mt * 128 + row;                  // hidden row
        const float bd = (p.bias0 && hr < p.H) ? p.bias0[(int64_t)e * p.H + hr] : 0.f;
        for (int cb = 0; cb < kPfN / 32; ++cb) {
          float v[32];
          umma::ld_32x32b_x32(tb + ((uint32_t)(32 * quad) << 16) + (uint32_t)(a * kPfN + cb * 32), v);
          if (ok && hr < p.H) {
            for (int n = 0; n < 32; ++n) {
              const int ent = s_ent[cb * 32 + n];
              if (ent < 0) break;
              p.y[(size_t)ent * p.H + hr] = (v[n] + bd) * s_w[cb * 32 + n];
            }
          }
        }
      }
      umma::fence_before_sync();
      mbar_arrive(&acc_empty[a]);
    }
  }
  umma::fence_before_sync();
  __syncthreads();
  if (warp == 1) umma::tmem_dealloc(tb, kPfTmemCols);
}

template <int MODE, int PREC>
cudaError_t launch_pf_gemm(const DevCtx& c, const PfParams& p, cudaStream_t s) {
  constexpr int smem = pf_smem<PREC>();
  cudaError_t e = cudaFuncSetAttribute(pf_gemm_kernel<MODE, PREC>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  pf_gemm_kernel<MODE, PREC><<<c.sm_count, kPfThreads, smem, s>>>(p);
  return cudaGetLastError();
}

}  // namespace

size_t pf_scratch_bytes(int H, int I, int E, int T, int K, int precise) {
  const size_t tiles = (size_t)(T * K) / kPfN + E + 1;   // upper bound on sum over experts of ceil(n_e / 256)
  const size_t m = precise ? 2 : 1;                       // token operands: hi (and lo) halves
  auto up = [](size_t b) { return (b + 255) & ~(size_t)255; };
  return up((size_t)E * 4) + up((size_t)E * T * 4) + m * up(tiles * H * kPfN * 2) + m * up(tiles * I * kPfN * 2) +
         up((size_t)T * K * H * 4);
}

cudaError_t launch_moe_prefill(const DevCtx& c, const PrefillArgs& a, cudaStream_t s) {
  if (a.E <= 0 || a.E > kPfMaxE || a.K < 1 || a.K > 16 || a.T <= 0 || !tc_supported(a.H, a.I))
    return cudaErrorInvalidValue;
  auto up = [](size_t b) { return (b + 255) & ~(size_t)255; };
  uint8_t* base = reinterpret_cast<uint8_t*>(a.scratch);
  const size_t tiles = (size_t)(a.T * a.K) / kPfN + a.E + 1;
  const size_t xb_b = up(tiles * a.H * kPfN * 2), act_b = up(tiles * a.I * kPfN * 2);
  int* count = reinterpret_cast<int*>(base);
  int* list = reinterpret_cast<int*>(base + up((size_t)a.E * 4));
  uint8_t* xb = base + up((size_t)a.E * 4) + up((size_t)a.E * a.T * 4);
  uint8_t* xb_lo = a.precise ? xb + xb_b : nullptr;
  uint8_t* act = xb + (a.precise ? 2 : 1) * xb_b;
  uint8_t* act_lo = a.precise ? act + act_b : nullptr;
  float* y = reinterpret_cast<float*>(act + (a.precise ? 2 : 1) * act_b);
  pf_route_kernel<<<a.E, 256, 0, s>>>(a.idx, a.T, a.K, a.expert_base, a.E, count, list);
  pf_gather_kernel<<<4 * c.sm_count, 256, 0, s>>>(a.x, a.H, a.K, count, list, a.E, a.T, xb, xb_lo);
  PfParams p = {};
  p.count = count; p.list = list; p.E = a.E; p.T = a.T; p.K = a.K; p.H = a.H; p.I = a.I; p.wts = a.wts;
  p.act = act; p.act_lo = act_lo; p.y = y; p.oai = a.oai_swiglu; p.err = c.err;
  p.mode = 0; p.w = a.gu; p.kc = a.H / 32; p.tile_bytes = tc_tile_bytes(p.kc); p.tiles = tc_gu_tiles(a.I);
  p.b = xb; p.b_lo = xb_lo; p.bias0 = a.gate_b; p.bias1 = a.up_b;
  cudaError_t e = a.precise ? launch_pf_gemm<0, 1>(c, p, s) : launch_pf_gemm<0, 0>(c, p, s);
  if (e != cudaSuccess) return e;
  p.mode = 1; p.w = a.down; p.kc = a.I / 32; p.tile_bytes = tc_tile_bytes(p.kc); p.tiles = tc_down_tiles(a.H);
  p.b = act; p.b_lo = act_lo; p.bias0 = a.down_b; p.bias1 = nullptr;
  e = a.precise ? launch_pf_gemm<1, 1>(c, p, s) : launch_pf_gemm<1, 0>(c, p, s);
  if (e != cudaSuccess) return e;
  pf_combine_kernel<<<a.T, 256, 0, s>>>(y, a.idx, a.K, a.expert_base, a.E, a.H, a.out, a.accumulate);
  return cudaGetLastError();
}

}  // namespace ms
