// kernels_batch.cu — dense kernels of the batched decode step (B sequences in lockstep, sm_100a).
//
// Reference semantics (moe-stream-core/src): Engine::forward over input_ids [B, 1] with a shared
// position (model/engine.rs:1869-2006, model/kv_cache.rs:37-60 concatenating along seq per batch
// row): embedding, Q8_0 projections through candle QMatMul (activation quantized to Q8_0, int8
// block dot, model/layer.rs:566-572, 722-730), residual + RMSNorm (ops/norm.rs:16-37), LM head
// and greedy argmax (engine.rs:1963-1987, 2069-2077).
//
// Every weight byte is read once per step for the whole batch:
//   q8_gemm_batch_kernel  one CTA per 16-row tile, the tile bulk-copied to shared memory; 8 warps
//                         split the 32-column blocks and run mma.sync m16n8k32 s8 per block (the
//                         exact int32 block dot of every token), folding d_w * d_x in f32.
//   lmhead_batch_kernel   f16 rows x per-token f16 hi/lo activation pieces (exact to ~2^-22 after a
//                         power-of-two prescale) on mma.sync m16n8k16, 4 tokens per MMA (columns
//                         2t, 2t+1 = token t's hi, lo); per-CTA argmax keys, then a final reduction.
#include <cuda_fp16.h>

#include "common.cuh"
#include "kernels.h"

namespace ms {
namespace {

__device__ __forceinline__ uint32_t lds_u32_a2(const uint8_t* p) {   // 2-byte aligned word
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  const uint32_t* w = reinterpret_cast<const uint32_t*>(a & ~(uintptr_t)3);
  return __funnelshift_r(w[0], w[1], (uint32_t)(a & 3) * 8u);
}

__device__ __forceinline__ void mma_s8_16832(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ unsigned long long key_of(float v, int idx) {   // larger key = larger v, lower idx
  uint32_t b = __float_as_uint(v);
  b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return ((unsigned long long)b << 32) | (uint32_t)(0xffffffffu - (uint32_t)idx);
}

__global__ void batch_begin_kernel(BatchState* st, uint32_t* err) {
  pdl_wait_prior();
  pdl_launch_dependents();
  int pos = st->n_ctx;
  if (pos >= st->max_seq) { atomicOr(err, EF_BAD_SHAPE); pos = st->max_seq - 1; }
  st->pos = pos;
  st->n_ctx = pos + 1;
  st->log_row = st->n_log;
  st->n_log = st->n_log + 1;
}

__global__ void __launch_bounds__(256) embed_batch_kernel(const BatchState* st, const int* tok_in,
                                                          const unsigned long long* keys, const void* table, int q,
                                                          int H, int vocab, int B, float* h, int* log, uint32_t* err,
                                                          const float* norm_w, float eps, int8_t* xq, float* xd) {
  extern __shared__ float es[];   // [H]
  __shared__ float red[256];
  __shared__ int tok_s;
  const int b = blockIdx.x;
  pdl_wait_prior();
  pdl_launch_dependents();
  if (threadIdx.x == 0) {
    int tok = tok_in[b];
    if (st->use_argmax) {
      const unsigned long long k = keys[b];
      tok = (int)(0xffffffffu - (uint32_t)(k & 0xffffffffull));
      if (k == 0ull) tok = 0;
    }
    if (tok < 0 || tok >= vocab) { atomicOr(err, EF_BAD_INDEX); tok = 0; }
    if (log && st->log_row < st->max_seq) log[(size_t)st->log_row * B + b] = tok;
    tok_s = tok;
  }
  __syncthreads();
  const int tok = tok_s;
  float* hb = h + (size_t)b * H;
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    const float v = (q == Q_F16) ? __half2float(reinterpret_cast<const __half*>(table)[(size_t)tok * H + i])
                                 : reinterpret_cast<const float*>(table)[(size_t)tok * H + i];
    hb[i] = v;
    es[i] = v;
  }
  __syncthreads();
  cta_rmsnorm_q8(es, H, norm_w, eps, xq + (size_t)b * H, xd + (size_t)b * (H / 32), red);
}

// ---------------- Q8_0 projection of a batch ----------------
constexpr int kQBWarps = 8;
constexpr int kQBChunk = 512;    // activation columns staged per pass (3 CTAs per SM)

__global__ void __launch_bounds__(kQBWarps * 32, 3) q8_gemm_batch_kernel(Q8BatchArgs a, int rb, int kc, uint32_t* err) {
  // shared memory: weight tile [16][rb] (+16) | codes [B][kc + 16] | scales [B][kc / 32 + 4], one
  // kc-column slice of the activations at a time
  extern __shared__ __align__(16) uint8_t sm[];
  __shared__ double red[kQBWarps][16][kMaxBatch + 1];
  __shared__ __align__(8) uint64_t bar;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
  const int tile = blockIdx.x;
  const int nb = a.cols / 32, B = a.B, NT = (B + 7) / 8;
  const int nbc = kc / 32;
  const int xs_stride = kc + 16, ds_stride = nbc + 4;
  const uint32_t bytes = (uint32_t)(16 * rb);
  uint8_t* wt = sm;
  int8_t* xs = reinterpret_cast<int8_t*>(sm + (((size_t)bytes + 16 + 15) & ~(size_t)15));
  float* ds = reinterpret_cast<float*>(xs + (size_t)B * xs_stride);
  if (threadIdx.x == 0) {   // weights do not depend on the previous kernel
    mbar_init(&bar, 1);
    fence_mbar_init();
    mbar_expect_tx(&bar, bytes);
    bulk_g2s_stream(wt, a.w + (size_t)tile * bytes, bytes, &bar, policy_evict_first());
  }
  pdl_wait_prior();
  pdl_launch_dependents();
  bool ok = true;
  double acc[kMaxBatch / 8][4];   // block terms (int32 dot x d_w x d_x) are exact in double
#pragma unroll
  for (int t = 0; t < kMaxBatch / 8; ++t) acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0.0;
  for (int k0 = 0; k0 < a.cols; k0 += kc) {
    // the batch's activation codes and block scales for columns [k0, k0 + kc) (L2-resident)
    if (k0) __syncthreads();
    const int vpr = kc / 16, b0k = k0 / 32;
    {
      // all of the slice's loads in flight before the shared-memory stores
      constexpr int kU = 8;
      for (int i0 = threadIdx.x; i0 < B * vpr; i0 += kU * blockDim.x) {
        uint4 v[kU];
#pragma unroll
        for (int u = 0; u < kU; ++u) {
          const int i = i0 + u * blockDim.x;
          if (i < B * vpr) {
            const int tb = i / vpr, q = i - tb * vpr;
            v[u] = __ldg(reinterpret_cast<const uint4*>(a.xq + (size_t)tb * a.cols + k0) + q);
          }
        }
#pragma unroll
        for (int u = 0; u < kU; ++u) {
          const int i = i0 + u * blockDim.x;
          if (i < B * vpr) {
            const int tb = i / vpr, q = i - tb * vpr;
            *reinterpret_cast<uint4*>(xs + (size_t)tb * xs_stride + 16 * q) = v[u];
          }
        }
      }
      for (int i0 = threadIdx.x; i0 < B * nbc; i0 += kU * blockDim.x) {
        float v[kU];
#pragma unroll
        for (int u = 0; u < kU; ++u) {
          const int i = i0 + u * blockDim.x;
          v[u] = i < B * nbc ? __ldg(a.xd + (size_t)(i / nbc) * nb + b0k + i % nbc) : 0.f;
        }
#pragma unroll
        for (int u = 0; u < kU; ++u) {
          const int i = i0 + u * blockDim.x;
          if (i < B * nbc) ds[(i / nbc) * ds_stride + i % nbc] = v[u];
        }
      }
    }
    __syncthreads();
    if (k0 == 0) ok = mbar_wait(&bar, 0, err, EF_TIMEOUT_FULL);
    if (!ok) continue;
    for (int bl = warp; bl < nbc; bl += kQBWarps) {
      const int blk = b0k + bl;
      const uint8_t* r0 = wt + (size_t)g * rb + 34 * blk;
      const uint8_t* r1 = r0 + (size_t)8 * rb;
      const uint32_t a0 = lds_u32_a2(r0 + 2 + 4 * c), a1 = lds_u32_a2(r1 + 2 + 4 * c);
      const uint32_t a2 = lds_u32_a2(r0 + 18 + 4 * c), a3 = lds_u32_a2(r1 + 18 + 4 * c);
      const float dw0 = h2f_bits(*reinterpret_cast<const uint16_t*>(r0));
      const float dw1 = h2f_bits(*reinterpret_cast<const uint16_t*>(r1));
#pragma unroll
      for (int t = 0; t < kMaxBatch / 8; ++t) {
        if (t < NT) {
          const int tb = 8 * t + g;   // this lane's B column
          uint32_t b0 = 0u, b1 = 0u;
          if (tb < B) {
            const int8_t* xr = xs + (size_t)tb * xs_stride + 32 * bl + 4 * c;
            b0 = *reinterpret_cast<const uint32_t*>(xr);
            b1 = *reinterpret_cast<const uint32_t*>(xr + 16);
          }
          int d[4] = {0, 0, 0, 0};
          mma_s8_16832(d, a0, a1, a2, a3, b0, b1);
          const int t0 = 8 * t + 2 * c;
          const float dx0 = t0 < B ? ds[t0 * ds_stride + bl] : 0.f;
          const float dx1 = t0 + 1 < B ? ds[(t0 + 1) * ds_stride + bl] : 0.f;
          acc[t][0] += (double)d[0] * (double)dw0 * (double)dx0;
          acc[t][1] += (double)d[1] * (double)dw0 * (double)dx1;
          acc[t][2] += (double)d[2] * (double)dw1 * (double)dx0;
          acc[t][3] += (double)d[3] * (double)dw1 * (double)dx1;
        }
      }
    }
  }
#pragma unroll
  for (int t = 0; t < kMaxBatch / 8; ++t) {
    if (t < NT) {
      const int t0 = 8 * t + 2 * c;
      red[warp][g][t0] = acc[t][0];
      red[warp][g][t0 + 1] = acc[t][1];
      red[warp][g + 8][t0] = acc[t][2];
      red[warp][g + 8][t0 + 1] = acc[t][3];
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 16 * B; i += blockDim.x) {
    const int r = i % 16, tb = i / 16;
    double vd = 0.0;
#pragma unroll
    for (int w = 0; w < kQBWarps; ++w) vd += red[w][r][tb];
    const int row = tile * 16 + r;
    float v = (float)vd;
    if (a.bias) v = __fadd_rn(v, a.bias[row]);
    if (!ok) v = 0.f;
    if (a.residual) a.residual[(size_t)tb * a.rows + row] = __fadd_rn(a.residual[(size_t)tb * a.rows + row], v);
    else a.y[(size_t)tb * a.rows + row] = v;
  }
}

// ---------------- residual update + next norm ----------------
__global__ void __launch_bounds__(256) resid_batch_kernel(BatchCombine bc, float* h, int H, const float* norm_w,
                                                          float eps, int8_t* xq, float* xd, float* xf) {
  extern __shared__ float hs[];   // [H]
  __shared__ int s_ent[16];
  __shared__ float s_w[16];
  __shared__ int s_n;
  __shared__ float red[256];
  const int b = blockIdx.x;
  pdl_wait_prior();
  pdl_launch_dependents();
  if (threadIdx.x == 0) {   // this token's local experts in ascending id (the reference's order)
    int n = 0, ids[16];
    for (int k = 0; k < bc.K; ++k) {
      if (bc.ent_of[b * bc.K + k] < 0) continue;
      const int e = bc.idx[b * bc.K + k];
      int j = n++;
      while (j > 0 && ids[j - 1] > e) { ids[j] = ids[j - 1]; s_ent[j] = s_ent[j - 1]; s_w[j] = s_w[j - 1]; --j; }
      ids[j] = e;
      s_ent[j] = b * bc.K + k;   // row of y
      s_w[j] = bc.wts[b * bc.K + k];
    }
    s_n = n;
  }
  __syncthreads();
  const int n = s_n;
  float* hb = h + (size_t)b * H;
  for (int r = threadIdx.x; r < H; r += blockDim.x) {
    float acc = 0.f;
    for (int q = 0; q < n; ++q) acc = __fadd_rn(acc, __fmul_rn(bc.y[(size_t)s_ent[q] * H + r], s_w[q]));
    const float v = __fadd_rn(hb[r], acc);
    hb[r] = v;
    hs[r] = v;
  }
  __syncthreads();
  if (xq) {
    cta_rmsnorm_q8(hs, H, norm_w, eps, xq + (size_t)b * H, xd + (size_t)b * (H / 32), red);
  } else if (xf) {
    const float inv = rms_inv_cr(hs, H, eps, threadIdx.x, blockDim.x, [] { __syncthreads(); });
    for (int i = threadIdx.x; i < H; i += blockDim.x)
      xf[(size_t)b * H + i] = norm_w ? __fmul_rn(__fmul_rn(hs[i], inv), norm_w[i]) : hs[i];
  }
}

// ---------------- LM head of a batch ----------------
constexpr int kLBWarps = 8;
constexpr int kLBRows = kLBWarps * 32;   // rows per CTA (2 MMA row tiles per warp)
constexpr int kLBChunk = 16;             // k-steps (16 columns each) per shared-memory chunk

// scratch: fragments [H/16][8 passes][32 lanes][2] u32 | scales [32] f32 | per-CTA keys [n_cta][32]
int64_t lm_frag_bytes(int H) { return (int64_t)(H / 16) * 8 * 32 * 8; }

// block b (one per token slot, a multiple of 4): power-of-two prescale of token b, its f16 hi/lo
// B-fragment entries; zero for slots >= B
__global__ void __launch_bounds__(256) lm_prep_kernel(LmBatchArgs a, uint32_t* frag, float* scale) {
  __shared__ float red[32];
  const int b = blockIdx.x, H = a.H;
  pdl_wait_prior();
  pdl_launch_dependents();
  const float* x = a.xf + (size_t)b * H;
  float m = 0.f;
  if (b < a.B)
    for (int i = threadIdx.x; i < H; i += blockDim.x) m = fmaxf(m, fabsf(x[i]));
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  m = 0.f;
  for (int k = 0; k < (int)(blockDim.x >> 5); ++k) m = fmaxf(m, red[k]);
  const int ef = (int)((__float_as_uint(m) >> 23) & 0xffu);
  const int e = (m > 0.f && ef > 0) ? ef - 126 : 0;              // m * 2^-e in [0.5, 1)
  const float sc = __uint_as_float((uint32_t)(127 - e) << 23);   // 2^-e
  if (threadIdx.x == 0 && b < a.B) { scale[b] = __uint_as_float((uint32_t)(127 + e) << 23); a.keys[b] = 0ull; }
  const int p = b >> 2, col = 2 * (b & 3);
  const int ns = H / 16;
  for (int i = threadIdx.x; i < ns * 2 * 4; i += blockDim.x) {
    const int s = i >> 3, hl = (i >> 2) & 1, c = i & 3;
    uint32_t w0 = 0u, w1 = 0u;
    if (b < a.B) {
      const float* xs = x + 16 * s + 2 * c;
      __half v[4];
      const float src[4] = {xs[0], xs[1], xs[8], xs[9]};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float y = src[q] * sc;
        __half hh = __float2half_rn(y);
        if (hl) hh = __float2half_rn(y - __half2float(hh));
        v[q] = hh;
      }
      w0 = pack_half2(v[0], v[1]);
      w1 = pack_half2(v[2], v[3]);
    }
    const int lane = ((col + hl) << 2) | c;
    uint32_t* dst = frag + (((size_t)s * 8 + p) * 32 + lane) * 2;
    dst[0] = w0;
    dst[1] = w1;
  }
}

__global__ void __launch_bounds__(kLBWarps * 32) lmhead_batch_kernel(LmBatchArgs a, const uint32_t* frag,
                                                                     const float* scale, unsigned long long* ckeys,
                                                                     uint32_t* err) {
  extern __shared__ __align__(16) uint32_t fs[];   // 2 x [kLBChunk][NP][32][2]
  __shared__ __align__(8) uint64_t bar[2];
  __shared__ unsigned long long kred[kLBWarps][kMaxBatch];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
  const int NP = (a.B + 3) / 4, ns = a.H / 16, nch = (ns + kLBChunk - 1) / kLBChunk;
  const uint32_t chunk_words = (uint32_t)kLBChunk * NP * 64;
  pdl_wait_prior();
  pdl_launch_dependents();
  if (threadIdx.x == 0) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    fence_mbar_init();
    for (int ci = 0; ci < 2 && ci < nch; ++ci) {
      const int s0 = ci * kLBChunk, nsk = min(kLBChunk, ns - s0);
      const uint32_t bytes = (uint32_t)nsk * NP * 256;
      mbar_expect_tx(&bar[ci], bytes);
      // the fragment rows of passes 0..NP-1 for k-steps s0.. are contiguous when NP == 8;
      // otherwise one copy per k-step
      if (NP == 8) bulk_g2s(fs + ci * chunk_words, frag + (size_t)s0 * 8 * 64, bytes, &bar[ci]);
      else
        for (int s = 0; s < nsk; ++s)
          bulk_g2s(fs + ci * chunk_words + s * NP * 64, frag + (size_t)(s0 + s) * 8 * 64, (uint32_t)NP * 256, &bar[ci]);
    }
  }
  __syncthreads();
  const int row0 = blockIdx.x * kLBRows + warp * 32;
  float acc[2][8][4];
#pragma unroll
  for (int t = 0; t < 2; ++t)
#pragma unroll
    for (int p = 0; p < 8; ++p) acc[t][p][0] = acc[t][p][1] = acc[t][p][2] = acc[t][p][3] = 0.f;
  const uint16_t* wr[2][2];
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    const int r0 = min(row0 + 16 * t + g, a.V - 1), r1 = min(row0 + 16 * t + g + 8, a.V - 1);
    wr[t][0] = a.w + (size_t)r0 * a.H + 2 * c;
    wr[t][1] = a.w + (size_t)r1 * a.H + 2 * c;
  }
  __shared__ int s_ok;
  int failed = -1;
  for (int ci = 0; ci < nch; ++ci) {
    const int buf = ci & 1;
    if (threadIdx.x == 0) s_ok = mbar_wait(&bar[buf], (uint32_t)((ci >> 1) & 1), err, EF_TIMEOUT_FULL) ? 1 : 0;
    __syncthreads();
    if (!s_ok) { failed = ci; break; }
    const uint32_t* fc = fs + buf * chunk_words;
    const int s0 = ci * kLBChunk, nsk = min(kLBChunk, ns - s0);
#pragma unroll 2
    for (int s = 0; s < nsk; ++s) {
      const int k0 = 16 * (s0 + s);
      uint32_t af[2][4];
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        af[t][0] = __ldg(reinterpret_cast<const uint32_t*>(wr[t][0] + k0));
        af[t][1] = __ldg(reinterpret_cast<const uint32_t*>(wr[t][1] + k0));
        af[t][2] = __ldg(reinterpret_cast<const uint32_t*>(wr[t][0] + k0 + 8));
        af[t][3] = __ldg(reinterpret_cast<const uint32_t*>(wr[t][1] + k0 + 8));
      }
#pragma unroll
      for (int p = 0; p < 8; ++p) {
        if (p < NP) {
          const uint2 bf = *reinterpret_cast<const uint2*>(fc + ((size_t)s * NP + p) * 64 + 2 * lane);
#pragma unroll
          for (int t = 0; t < 2; ++t) mma_f16_16816(acc[t][p], af[t], bf.x, bf.y);
        }
      }
    }
    __syncthreads();   // every warp is done with this buffer
    if (threadIdx.x == 0 && ci + 2 < nch) {
      const int s0n = (ci + 2) * kLBChunk, nskn = min(kLBChunk, ns - s0n);
      const uint32_t bytes = (uint32_t)nskn * NP * 256;
      mbar_expect_tx(&bar[buf], bytes);
      if (NP == 8) bulk_g2s(fs + buf * chunk_words, frag + (size_t)s0n * 8 * 64, bytes, &bar[buf]);
      else
        for (int s = 0; s < nskn; ++s)
          bulk_g2s(fs + buf * chunk_words + s * NP * 64, frag + (size_t)(s0n + s) * 8 * 64, (uint32_t)NP * 256,
                   &bar[buf]);
    }
  }
  if (failed >= 0) {   // a timed-out chunk: wait (bounded) for the other buffer's copy, contribute nothing
    const int ci = failed + 1;
    if (threadIdx.x == 0 && ci < nch) mbar_wait(&bar[ci & 1], (uint32_t)((ci >> 1) & 1), err, EF_TIMEOUT_FULL);
    return;
  }
  // epilogue: thread (g, c) holds token 4p + c at rows g, g + 8 of both tiles
#pragma unroll
  for (int p = 0; p < 8; ++p) {
    if (p < NP) {
      const int tb = 4 * p + c;
      unsigned long long best = 0ull;
      if (tb < a.B) {
        const float sc = scale[tb];
#pragma unroll
        for (int t = 0; t < 2; ++t)
#pragma unroll
          for (int hrow = 0; hrow < 2; ++hrow) {
            const int r = row0 + 16 * t + g + 8 * hrow;
            if (r < a.V) {
              float v = (acc[t][p][2 * hrow] + acc[t][p][2 * hrow + 1]) * sc;
              if (a.bias) v += a.bias[r];
              if (a.logits) a.logits[(size_t)tb * a.V + r] = v;
              const unsigned long long k = key_of(v, r);
              best = k > best ? k : best;
            }
          }
      }
      // reduce over the 8 lanes of this token (same c)
#pragma unroll
      for (int o = 4; o < 32; o <<= 1) {
        const unsigned long long ok2 = __shfl_xor_sync(0xffffffffu, best, o);
        best = ok2 > best ? ok2 : best;
      }
      if (g == 0 && tb < a.B) kred[warp][tb] = best;
    }
  }
  __syncthreads();
  for (int tb = threadIdx.x; tb < a.B; tb += blockDim.x) {
    unsigned long long best = 0ull;
    for (int w = 0; w < kLBWarps; ++w) best = kred[w][tb] > best ? kred[w][tb] : best;
    ckeys[(size_t)blockIdx.x * kMaxBatch + tb] = best;
  }
}

__global__ void __launch_bounds__(256) lm_keys_kernel(LmBatchArgs a, const unsigned long long* ckeys, int n_cta) {
  __shared__ unsigned long long r[256];
  const int tb = blockIdx.x;
  pdl_wait_prior();
  pdl_launch_dependents();
  unsigned long long best = 0ull;
  for (int i = threadIdx.x; i < n_cta; i += blockDim.x) {
    const unsigned long long k = ckeys[(size_t)i * kMaxBatch + tb];
    best = k > best ? k : best;
  }
  r[threadIdx.x] = best;
  __syncthreads();
  for (int o = 128; o > 0; o >>= 1) {
    if ((int)threadIdx.x < o) r[threadIdx.x] = r[threadIdx.x + o] > r[threadIdx.x] ? r[threadIdx.x + o] : r[threadIdx.x];
    __syncthreads();
  }
  if (threadIdx.x == 0) a.keys[tb] = r[0];
}

template <typename Kern, typename... Args>
cudaError_t launch_pdl_b(Kern k, dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k, args...);
}

// dynamic shared memory opt-in (static + dynamic may exceed the 48 KB default)
cudaError_t set_smem(const void* k, size_t smem) {
  return cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
}

}  // namespace

cudaError_t launch_batch_begin(const DevCtx& c, BatchState* st, cudaStream_t s) {
  return launch_pdl_b(batch_begin_kernel, dim3(1), dim3(1), 0, s, st, c.err);
}

cudaError_t launch_embed_batch(const DevCtx& c, BatchState* st, const int* tok_in, const unsigned long long* keys,
                               const void* table, int q, int H, int vocab, int B, float* h, int* log,
                               const float* norm_w, float eps, int8_t* xq, float* xd, cudaStream_t s) {
  if (B < 1 || B > kMaxBatch || H % 32 || !norm_w || (q != Q_F16 && q != Q_F32)) return cudaErrorInvalidValue;
  const size_t smem = (size_t)H * 4;
  cudaError_t e = set_smem((const void*)embed_batch_kernel, smem);
  if (e != cudaSuccess) return e;
  return launch_pdl_b(embed_batch_kernel, dim3((unsigned)B), dim3(256), smem, s, (const BatchState*)st, tok_in, keys,
                      table, q, H, vocab, B, h, log, c.err, norm_w, eps, xq, xd);
}

cudaError_t launch_q8_gemm_batch(const DevCtx& c, const Q8BatchArgs& a, cudaStream_t s) {
  if (a.B < 1 || a.B > kMaxBatch || a.rows % 16 || a.cols % 32 || a.rows <= 0 || (!a.y && !a.residual))
    return cudaErrorInvalidValue;
  if (reinterpret_cast<uintptr_t>(a.w) % 16 || reinterpret_cast<uintptr_t>(a.xq) % 4) return cudaErrorInvalidValue;
  const int rb = a.cols / 32 * 34;
  // activation slices (whole 32-column blocks): 512 columns keep 3 CTAs per SM when the grid
  // exceeds the SM count; a grid of at most one CTA per SM takes wider slices (fewer passes)
  const int chunk = a.rows / 16 > c.sm_count ? kQBChunk : 4 * kQBChunk;
  int np = (a.cols + chunk - 1) / chunk;
  while (a.cols % np || (a.cols / np) % 32) ++np;
  const int kc = a.cols / np;
  const size_t smem = (((size_t)16 * rb + 16 + 15) & ~(size_t)15) + (size_t)a.B * (kc + 16) +
                      (size_t)a.B * (kc / 32 + 4) * 4;
  if (smem > 200 * 1024) return cudaErrorInvalidValue;
  cudaError_t e = set_smem((const void*)q8_gemm_batch_kernel, smem);
  if (e != cudaSuccess) return e;
  return launch_pdl_b(q8_gemm_batch_kernel, dim3((unsigned)(a.rows / 16)), dim3(kQBWarps * 32), smem, s, a, rb, kc,
                      c.err);
}

cudaError_t launch_resid_batch(const DevCtx& c, const BatchCombine& bc, float* h, int H, int B, const float* norm_w,
                               float eps, int8_t* xq, float* xd, float* xf, cudaStream_t s) {
  (void)c;
  if (B < 1 || B > kMaxBatch || bc.K > 16 || (xq && (!norm_w || H % 32))) return cudaErrorInvalidValue;
  const size_t smem = (size_t)H * 4;
  cudaError_t e = set_smem((const void*)resid_batch_kernel, smem);
  if (e != cudaSuccess) return e;
  return launch_pdl_b(resid_batch_kernel, dim3((unsigned)B), dim3(256), smem, s, bc, h, H, norm_w, eps, xq, xd, xf);
}

int64_t lm_batch_scratch_bytes(int V, int H) {
  const int64_t n_cta = (V + kLBRows - 1) / kLBRows;
  return lm_frag_bytes(H) + kMaxBatch * 4 + n_cta * kMaxBatch * 8 + 256;
}

cudaError_t launch_lmhead_batch(const DevCtx& c, const LmBatchArgs& a, cudaStream_t s) {
  if (a.B < 1 || a.B > kMaxBatch || a.H % 16 || a.V <= 0 || !a.keys || !a.scratch) return cudaErrorInvalidValue;
  if (reinterpret_cast<uintptr_t>(a.w) % 4 || reinterpret_cast<uintptr_t>(a.scratch) % 16) return cudaErrorInvalidValue;
  uint32_t* frag = reinterpret_cast<uint32_t*>(a.scratch);
  float* scale = reinterpret_cast<float*>(reinterpret_cast<char*>(a.scratch) + lm_frag_bytes(a.H));
  unsigned long long* ckeys = reinterpret_cast<unsigned long long*>(
      reinterpret_cast<char*>(a.scratch) + ((lm_frag_bytes(a.H) + kMaxBatch * 4 + 15) & ~15ll));
  const int slots = (a.B + 3) / 4 * 4;
  cudaError_t e = launch_pdl_b(lm_prep_kernel, dim3((unsigned)slots), dim3(256), 0, s, a, frag, scale);
  if (e != cudaSuccess) return e;
  const int NP = slots / 4;
  const size_t smem = (size_t)2 * kLBChunk * NP * 256;
  e = set_smem((const void*)lmhead_batch_kernel, smem);
  if (e != cudaSuccess) return e;
  const int n_cta = (a.V + kLBRows - 1) / kLBRows;
  e = launch_pdl_b(lmhead_batch_kernel, dim3((unsigned)n_cta), dim3(kLBWarps * 32), smem, s, a,
                   (const uint32_t*)frag, (const float*)scale, ckeys, c.err);
  if (e != cudaSuccess) return e;
  return launch_pdl_b(lm_keys_kernel, dim3((unsigned)a.B), dim3(256), 0, s, a, (const unsigned long long*)ckeys, n_cta);
}

}  // namespace ms
