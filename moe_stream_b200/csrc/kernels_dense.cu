// kernels_dense.cu — Q8_0 projections, decode attention, LM head, norms, dequant (sm_100a).
//
// Reference semantics (moe-stream-core/src):
//   RMSNorm ......................... ops/norm.rs:16-37
//   Q8_0 projection on CPU (candle QMatMul: activation quantized to Q8_0, int8 block dot)
//                                     ... model/layer.rs:566-572, 722-730; block format gguf/dequant.rs:511-531
//   QK-norm, RoPE, KV append, SDPA with sinks / sliding window / GQA
//                                     ... model/layer.rs:643-692, ops/attention.rs:49-120, 178-280,
//                                         model/kv_cache.rs:37-60, config.rs:463-465
//   embedding + final norm + LM head + greedy argmax ... model/engine.rs:1877, 1963-1987, 2069-2077
#include <cuda_fp16.h>

#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace ms {

int64_t row_bytes(int q, int64_t cols) {
  switch (q) {
    case Q_F32: return cols * 4;
    case Q_F16: return cols * 2;
    case Q_Q8_0: return cols % 32 ? -1 : cols / 32 * 34;
    case Q_Q4_K: return cols % 256 ? -1 : cols / 256 * 144;
    case Q_Q6_K: return cols % 256 ? -1 : cols / 256 * 210;
    case Q_Q6_K_PAD: return cols % 256 ? -1 : cols / 256 * kQ6PadBytes;
    case Q_MXFP4: return cols % 32 ? -1 : cols / 32 * 17;
  }
  return -1;
}

namespace {

// ============================ dequant (bit-exact) ============================
__device__ __forceinline__ float e8m0_half(uint32_t e) {
  return e < 2 ? __uint_as_float(0x00200000u << e) : __uint_as_float((e - 1u) << 23);
}
__constant__ float kMx[16] = {0.0f, 1.0f, 2.0f, 3.0f, 4.0f, 6.0f, 8.0f, 12.0f,
                              -0.0f, -1.0f, -2.0f, -3.0f, -4.0f, -6.0f, -8.0f, -12.0f};

__global__ void dequant_kernel(int q, const uint8_t* __restrict__ src, int64_t n, float* __restrict__ out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  switch (q) {
    case Q_F32: out[i] = reinterpret_cast<const float*>(src)[i]; break;
    case Q_F16: out[i] = __half2float(reinterpret_cast<const __half*>(src)[i]); break;
    case Q_MXFP4: {   // dequant.rs:605-628
      const uint8_t* b = src + (i >> 5) * 17;
      const int j = (int)(i & 31);
      const uint8_t byte = b[1 + (j & 15)];
      out[i] = kMx[j < 16 ? (byte & 0xf) : (byte >> 4)] * e8m0_half(b[0]);
      break;
    }
    case Q_Q8_0: {    // dequant.rs:511-531
      const uint8_t* b = src + (i >> 5) * 34;
      const float d = __half2float(__ushort_as_half((uint16_t)(b[0] | (b[1] << 8))));
      out[i] = d * (float)(int8_t)b[2 + (i & 31)];
      break;
    }
    case Q_Q4_K: {    // dequant.rs:199-262
      const uint8_t* b = src + (i >> 8) * 144;
      const int e = (int)(i & 255), j = e >> 6, hi = (e >> 5) & 1, l = e & 31, is = 2 * j + hi;
      const float d = __half2float(__ushort_as_half((uint16_t)(b[0] | (b[1] << 8))));
      const float dmin = __half2float(__ushort_as_half((uint16_t)(b[2] | (b[3] << 8))));
      const uint8_t* sc = b + 4;
      uint32_t s, m;
      if (is < 4) { s = sc[is] & 63; m = sc[is + 4] & 63; }
      else { s = (sc[is + 4] & 0xf) | ((sc[is - 4] >> 6) << 4); m = (sc[is + 4] >> 4) | ((sc[is] >> 6) << 4); }
      const uint8_t qb = b[16 + j * 32 + l];
      const float qv = (float)(hi ? (qb >> 4) : (qb & 0xf));
      out[i] = __fsub_rn(__fmul_rn(__fmul_rn(d, (float)s), qv), __fmul_rn(dmin, (float)m));
      break;
    }
    case Q_Q6_K: {    // dequant.rs:335-378
      const uint8_t* b = src + (i >> 8) * 210;
      const int e = (int)(i & 255), half = e >> 7, r = e & 127, quad = r >> 5, l = r & 31;
      const uint8_t* ql = b + half * 64;
      const uint8_t* qh = b + 128 + half * 32;
      const int8_t* sc = reinterpret_cast<const int8_t*>(b + 192);
      const float d = __half2float(__ushort_as_half((uint16_t)(b[208] | (b[209] << 8))));
      int qv;
      if (quad == 0) qv = ((ql[l] & 0xf) | ((qh[l] & 3) << 4)) - 32;
      else if (quad == 1) qv = ((ql[l + 32] & 0xf) | (((qh[l] >> 2) & 3) << 4)) - 32;
      else if (quad == 2) qv = ((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
      else qv = ((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
      const int is = half * 8 + l / 16 + 2 * quad;
      out[i] = __fmul_rn(__fmul_rn(d, (float)sc[is]), (float)qv);
      break;
    }
  }
}

// ============================ RMSNorm ============================
__global__ void rms_norm_kernel(const float* __restrict__ x, const float* __restrict__ w, float* __restrict__ y,
                                int dim, float eps) {
  const float* xr = x + (size_t)blockIdx.x * dim;
  float* yr = y + (size_t)blockIdx.x * dim;
  const float inv = rms_inv_cr(xr, dim, eps, threadIdx.x, blockDim.x, [] { __syncthreads(); });
  for (int i = threadIdx.x; i < dim; i += blockDim.x) yr[i] = __fmul_rn(__fmul_rn(xr[i], inv), w[i]);
}

// ============================ Q8_0 projection ============================
// Persistent CTA per SM: one producer thread bulk-copies row groups (<= 8 rows, 16-byte
// aligned) into a ring of stages; 8 consumer warps each take one row of a stage.  Lane l
// owns activation blocks l, l+32, ... whose int8 codes stay in registers; a row block is
// 34 bytes (f16 d + 32 int8) at a 2-byte aligned offset, read with aligned words and a
// 16-bit funnel shift, dotted with __dp4a.  Block sums follow candle's Q8_0 vec_dot:
// (float)sum_i * d_w * d_x accumulated in f32.
constexpr int kQW = 8;
constexpr int kQThreads = (kQW + 1) * 32;
constexpr int kQMaxStages = 8;

struct Q8Params {
  const uint8_t* w;
  int rows, cols, rb, unit_rows, n_units, stage_rows, stage_bytes, ns;
  const float* x;
  const float* norm_w;
  float eps;
  const float* bias;
  float* y;
  float* residual;
  const int8_t* xq_in;
  const float* xd_in;
  uint32_t* err;
};

template <int NBL>
__global__ void __launch_bounds__(kQThreads, 1) q8_gemv_kernel(Q8Params p) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* stages = smem;
  int8_t* xq = reinterpret_cast<int8_t*>(smem + (size_t)p.ns * p.stage_bytes);   // [cols]
  float* xd = reinterpret_cast<float*>(xq + ((p.cols + 15) & ~15));                // [nb]
  float* xf = xd + ((p.cols / 32 + 3) & ~3);                                       // [cols]
  uint64_t* full = reinterpret_cast<uint64_t*>(xf + p.cols);
  uint64_t* empty = full + kQMaxStages;
  __shared__ int abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nb = p.cols / 32;
  // contiguous row range of this CTA, in units that keep every copy 16-byte aligned
  const int u0 = (int)((int64_t)blockIdx.x * p.n_units / gridDim.x);
  const int u1 = (int)((int64_t)(blockIdx.x + 1) * p.n_units / gridDim.x);
  const int r_begin = u0 * p.unit_rows, r_end = min(u1 * p.unit_rows, p.rows);
  const int n_stage = (r_end - r_begin + p.stage_rows - 1) / p.stage_rows;

  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < p.ns; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], kQW); }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == kQW) {
    // producer: weights do not depend on the previous kernel, start streaming before the wait
    if (lane == 0 && n_stage > 0) {
      const uint64_t pol = policy_evict_first();
      int issued = 0;
      for (int j = 0; j < n_stage; ++j) {
        const int s = j % p.ns, n = j / p.ns;
        if (j == p.ns) {   // ring full: the rest follows the consumers, which start after the wait
          pdl_wait_prior();
          pdl_launch_dependents();
        }
        if (n > 0 && !mbar_wait(&empty[s], (uint32_t)((n - 1) & 1), p.err, EF_TIMEOUT_EMPTY)) break;
        const int r0 = r_begin + j * p.stage_rows;
        const int nr = min(p.stage_rows, r_end - r0);
        const uint32_t bytes = (uint32_t)(((int64_t)nr * p.rb + 15) & ~15ll);
        mbar_expect_tx(&full[s], bytes);
        bulk_g2s_stream(stages + (size_t)s * p.stage_bytes, p.w + (int64_t)r0 * p.rb, bytes, &full[s], pol);
        ++issued;
      }
      for (int j = max(0, issued - p.ns); j < issued; ++j)
        mbar_wait(&full[j % p.ns], (uint32_t)((j / p.ns) & 1), p.err, EF_TIMEOUT_FULL);
    }
    // consumers use named barrier 1 only, so the producer warp may leave now
    return;
  }

  // ---- consumer prologue: the activation's Q8_0 blocks in registers.  They come quantized
  // from the producing kernel (xq_in / xd_in), or are made here: (RMSNorm) + Q8_0 quantization.
  pdl_wait_prior();
  pdl_launch_dependents();   // the next kernel may start its own (weight) prefetch now
  const int nct = kQW * 32;
  const int8_t* xqs = p.xq_in;
  const float* xds = p.xd_in;
  if (!xqs) {
    float inv = 1.f;
    if (p.norm_w) inv = rms_inv_cr(p.x, p.cols, p.eps, threadIdx.x, nct, [nct] { named_bar(1, nct); });
    for (int b = threadIdx.x; b < nb; b += nct) {
      float v[32];
      const float4* x4 = reinterpret_cast<const float4*>(p.x + 32 * b);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float4 t = x4[k];
        v[4 * k] = t.x; v[4 * k + 1] = t.y; v[4 * k + 2] = t.z; v[4 * k + 3] = t.w;
      }
      if (p.norm_w) {
        const float4* w4 = reinterpret_cast<const float4*>(p.norm_w + 32 * b);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const float4 t = w4[k];
          v[4 * k] = __fmul_rn(__fmul_rn(v[4 * k], inv), t.x);
          v[4 * k + 1] = __fmul_rn(__fmul_rn(v[4 * k + 1], inv), t.y);
          v[4 * k + 2] = __fmul_rn(__fmul_rn(v[4 * k + 2], inv), t.z);
          v[4 * k + 3] = __fmul_rn(__fmul_rn(v[4 * k + 3], inv), t.w);
        }
      }
      quantize_q8_block(v, xq + 32 * b, &xd[b]);
    }
    named_bar(1, nct);
    xqs = xq;
    xds = xd;
  }
  int xr[NBL][8];
  float xdr[NBL];
#pragma unroll
  for (int i = 0; i < NBL; ++i) {
    const int b = lane + 32 * i;
    xdr[i] = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) xr[i][k] = 0;
    if (b < nb) {
      const int4* q4 = reinterpret_cast<const int4*>(xqs + 32 * b);
      const int4 a0 = q4[0], a1 = q4[1];
      xr[i][0] = a0.x; xr[i][1] = a0.y; xr[i][2] = a0.z; xr[i][3] = a0.w;
      xr[i][4] = a1.x; xr[i][5] = a1.y; xr[i][6] = a1.z; xr[i][7] = a1.w;
      xdr[i] = xds[b];
    }
  }

  for (int j = 0; j < n_stage; ++j) {
    const int s = j % p.ns, n = j / p.ns;
    const int r0 = r_begin + j * p.stage_rows;
    const int nr = min(p.stage_rows, r_end - r0);
    const bool ok = mbar_wait(&full[s], (uint32_t)(n & 1), p.err, EF_TIMEOUT_FULL);
    if (!ok) { if (lane == 0) atomicExch(&abort_flag, 1); }
    double acc = 0.0;   // block terms sum_i * d_w * d_x are exact in double
    if (ok && warp < nr) {
      const uint8_t* row = stages + (size_t)s * p.stage_bytes + (size_t)warp * p.rb;
      // block b = lane + 32 i starts at 34 b; 34 * 32 = 1088 is a multiple of 4, so the
      // alignment of this lane's codes is the same for all of its blocks in the row
      const uint32_t off_l = (uint32_t)warp * p.rb + 34u * lane;
      const uint32_t qa_l = (off_l + 2) & ~3u, sh = ((off_l + 2) & 3u) * 8u;
      const uint8_t* sbase = stages + (size_t)s * p.stage_bytes;
#pragma unroll
      for (int i = 0; i < NBL; ++i) {
        const int b = lane + 32 * i;
        if (b < nb) {
          const uint16_t dw = *reinterpret_cast<const uint16_t*>(row + 34u * lane + 1088u * i);
          const uint32_t* wp = reinterpret_cast<const uint32_t*>(sbase + qa_l + 1088u * i);
          uint32_t wd[9];
#pragma unroll
          for (int k = 0; k < 9; ++k) wd[k] = wp[k];
          int sumi = 0;
#pragma unroll
          for (int k = 0; k < 8; ++k) sumi = __dp4a((int)__funnelshift_r(wd[k], wd[k + 1], sh), xr[i][k], sumi);
          acc += (double)sumi * (double)h2f_bits(dw) * (double)xdr[i];
        }
      }
    }
    __syncwarp();
    if (ok && lane == 0) mbar_arrive(&empty[s]);
    acc = warp_sum_d(acc);
    if (ok && warp < nr && lane == 0) {
      const int r = r0 + warp;
      float v = (float)acc;
      if (p.bias) v = __fadd_rn(v, p.bias[r]);
      if (p.residual) p.residual[r] = __fadd_rn(p.residual[r], v);
      else p.y[r] = v;
    }
    if (!ok) break;
  }
}

template <int NBL>
cudaError_t launch_q8(const DevCtx& c, const Q8Params& p, cudaStream_t s) {
  const size_t smem = (size_t)p.ns * p.stage_bytes + ((p.cols + 15) & ~15) + ((p.cols / 32 + 3) & ~3) * 4 +
                      (size_t)p.cols * 4 + 2 * kQMaxStages * 8 + 16;
  cudaError_t e = cudaFuncSetAttribute(q8_gemv_kernel<NBL>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)min(c.sm_count, p.n_units));
  cfg.blockDim = dim3(kQThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, q8_gemv_kernel<NBL>, p);
}

// ============================ attention (decode) ============================
// Grid (splits, kv_heads, batch), 8 warps per CTA; a split covers 256 consecutive positions and
// each warp 32 of them.  Lanes run over head dims (HD/32 each), so a cached K or V row is one
// coalesced load per warp straight from HBM (no shared-memory staging); before waiting for the
// projections each lane prefetches its part of the warp's rows into L2.  Scores: every lane forms
// the REP per-head partial dots of a position with the query heads held in registers, and a
// reduce-scatter over the warp (log2(REP) halving steps, then a full sum) leaves head h's score in
// lanes h*32/REP ..; each such lane keeps its head's 32 scores and softmax state.  P*V: the
// per-position weights are shuffled from those lanes and accumulated over the lane's dims.  The
// warps merge in shared memory; the last CTA of a kv group merges the splits, with the attention
// sink in the denominator (ops/attention.rs:178-280).
constexpr int kAWarps = 8;
constexpr int kAThreads = kAWarps * 32;
constexpr int kAChunk = 32;   // positions per warp

// positions per split
__host__ __device__ constexpr int attn_split_len(int) { return kAWarps * kAChunk; }

__device__ __forceinline__ void rope_inplace(float* v, int rot, const float* c, const float* s) {
  // ops/attention.rs:96-118: half-rotate over the first `rot` dims
  const int half = rot / 2;
  for (int i = threadIdx.x; i < half; i += blockDim.x) {
    const float x1 = v[i], x2 = v[i + half];
    v[i] = __fsub_rn(__fmul_rn(x1, c[i]), __fmul_rn(x2, s[i]));
    v[i + half] = __fadd_rn(__fmul_rn(x2, c[i]), __fmul_rn(x1, s[i]));
  }
}

// per-head RMSNorm over hd by one warp (layer.rs:643-650)
__device__ __forceinline__ void head_norm_warp(float* v, const float* w, int hd, float eps, int lane) {
  const float inv = rms_inv_cr_warp(v, hd, eps, lane);
  __syncwarp();
  for (int i = lane; i < hd; i += 32) v[i] = __fmul_rn(__fmul_rn(v[i], inv), w[i]);
  __syncwarp();
}

// ============================ attention (decode, one sequence) ============================
// Single-sequence decode (the lockstep batch uses attn_decode_kernel below).  Grid (splits, kv_heads), 4 warps per CTA.  A split covers attn_tile_len(HD) consecutive
// positions; right after the position is known, one thread issues bulk copies of the split's
// cached K and V rows (contiguous in the [kv_head][slot][hd] cache; two pieces where a
// sliding-window ring wraps) into shared memory, and the query load, QK-norm and RoPE run while
// they are in flight.  Scores: one position per lane, the K row's float4 chunks visited in a
// lane-rotated order so a quarter-warp touches distinct banks; each warp keeps its own softmax
// max/sum per query head; P*V with lanes over head dims from the staged V tile; the four warps
// merge in shared memory; the last CTA of a kv head merges the splits, with the attention sink
// in the denominator (ops/attention.rs:178-280).
constexpr int kTWarps = 4;
constexpr int kTThreads = kTWarps * 32;

// positions per split: K + V tiles of one split fill 64 KB of shared memory
__host__ __device__ constexpr int attn_tile_len(int hd) { return hd <= 64 ? 128 : 8192 / hd; }

template <int HD, int REP>
__global__ void __launch_bounds__(kTThreads) attn_tile_kernel(AttnArgs a, uint32_t* err) {
  constexpr int DL = HD / 32;                  // head dims per lane in P*V
  constexpr int SPL = attn_tile_len(HD);      // positions per split
  constexpr int PW = SPL / kTWarps;            // positions per warp (<= 32)
  constexpr int NC = HD / 4;                   // float4 chunks per row
  extern __shared__ __align__(128) float dyn[];
  float* Kt = dyn;                             // [SPL][HD] staged cache rows
  float* Vt = Kt + SPL * HD;
  float* wsm = Vt + SPL * HD;                  // [S][REP] split weights of the final merge
  __shared__ __align__(16) float qs[REP * HD];
  __shared__ __align__(16) float kn[HD];
  __shared__ __align__(16) float vn[HD];
  __shared__ float pw[kTWarps][REP][32];
  __shared__ float mw[kTWarps][REP], lw[kTWarps][REP];
  __shared__ __align__(16) float ow[kTWarps][REP][HD];
  __shared__ __align__(8) uint64_t bar;
  __shared__ uint32_t last;
  __shared__ int tile_ok;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kh = blockIdx.y, sidx = blockIdx.x, S = gridDim.x;
  // The position comes from the step's first kernel and the cached rows from earlier steps, both
  // complete before the previous kernel started (every kernel lets its dependents launch only after
  // its own wait), so the tile copies go out before this kernel waits for the projections.
  const int pos = *a.pos;
  const int lo = a.window ? max(0, pos - a.window + 1) : 0;
  const int p0 = lo + sidx * SPL, p1 = min(p0 + SPL, pos + 1);
  const bool active = p0 < p1;
  const bool has_new = active && p1 == pos + 1;
  const int pc1 = has_new ? pos : p1;          // cached rows [p0, pc1); the new row comes from qkv
  const int half = a.rot / 2;
  float* part = a.part + ((size_t)kh * S + sidx) * REP * (HD + 2);
  if (threadIdx.x == 0) {
    tile_ok = 1;
    if (active && pc1 > p0) {
      mbar_init(&bar, 1);
      fence_mbar_init();
      mbar_expect_tx(&bar, (uint32_t)(2 * (pc1 - p0) * HD * 4));
      const float* kbase = a.kc + (size_t)kh * a.cap * HD;
      const float* vbase = a.vc + (size_t)kh * a.cap * HD;
      for (int q = p0; q < pc1;) {   // kv_cache.rs:37-60 slot order (ring for sliding-window layers)
        const int slot = a.window ? q % a.cap : q;
        const int n = a.window ? min(pc1 - q, a.cap - slot) : pc1 - q;
        const uint32_t bytes = (uint32_t)(n * HD * 4);
        bulk_g2s(Kt + (size_t)(q - p0) * HD, kbase + (size_t)slot * HD, bytes, &bar);
        bulk_g2s(Vt + (size_t)(q - p0) * HD, vbase + (size_t)slot * HD, bytes, &bar);
        q += n;
      }
    }
  }
  pdl_wait_prior();
  pdl_launch_dependents();
  if (active) {
    const float* cs = a.cos_t + (size_t)pos * half;
    const float* sn = a.sin_t + (size_t)pos * half;
    for (int i = threadIdx.x; i < REP * HD; i += kTThreads) qs[i] = a.qkv[(size_t)kh * REP * HD + i];
    if (has_new) {
      const float* kq = a.qkv + (size_t)a.nh * HD + (size_t)kh * HD;
      const float* vq = kq + (size_t)a.nkv * HD;
      for (int i = threadIdx.x; i < HD; i += kTThreads) { kn[i] = kq[i]; vn[i] = vq[i]; }
    }
    __syncthreads();
    if (a.q_norm) {
      for (int h = warp; h < REP; h += kTWarps) head_norm_warp(qs + h * HD, a.q_norm, HD, a.eps, lane);
      if (has_new && warp == 0) head_norm_warp(kn, a.k_norm, HD, a.eps, lane);
      __syncthreads();
    }
    for (int h = 0; h < REP; ++h) rope_inplace(qs + h * HD, a.rot, cs, sn);
    if (has_new) rope_inplace(kn, a.rot, cs, sn);
    __syncthreads();
    if (has_new) {   // kv_cache.rs:37-60 append (ring slot for sliding-window layers)
      const int slot = a.window ? pos % a.cap : pos;
      float* kd = a.kc + ((size_t)kh * a.cap + slot) * HD;
      float* vd = a.vc + ((size_t)kh * a.cap + slot) * HD;
      for (int i = threadIdx.x; i < HD; i += kTThreads) { kd[i] = kn[i]; vd[i] = vn[i]; }
    }
    if (pc1 > p0 && !mbar_wait(&bar, 0, err, EF_TIMEOUT_FULL)) tile_ok = 0;
    // ---- scores: one position per lane ----
    const int i_loc = warp * PW + lane;
    const int p = p0 + i_loc;
    const bool valid = lane < PW && p < p1;
    const float* krow = (p == pos) ? kn : Kt + (size_t)i_loc * HD;
    float dot[REP];
#pragma unroll
    for (int h = 0; h < REP; ++h) dot[h] = 0.f;
    if (valid) {
#pragma unroll 4
      for (int k = 0; k < NC; ++k) {
        const int c = (k + lane) & (NC - 1);
        const float4 k4 = *reinterpret_cast<const float4*>(krow + 4 * c);
#pragma unroll
        for (int h = 0; h < REP; ++h) {
          const float4 q4 = *reinterpret_cast<const float4*>(qs + h * HD + 4 * c);
          dot[h] = fmaf(q4.x, k4.x, fmaf(q4.y, k4.y, fmaf(q4.z, k4.z, fmaf(q4.w, k4.w, dot[h]))));
        }
      }
    }
#pragma unroll
    for (int h = 0; h < REP; ++h) {
      const float sv = valid ? dot[h] * a.scale : -INFINITY;
      const float m = warp_max(sv);
      const float pe = (sv == -INFINITY) ? 0.f : expf(sv - m);
      const float l = warp_sum(pe);
      pw[warp][h][lane] = pe;
      if (lane == 0) { mw[warp][h] = m; lw[warp][h] = l; }
    }
    __syncwarp();
    // ---- P * V: lanes over head dims ----
    float o[REP][DL];
#pragma unroll
    for (int h = 0; h < REP; ++h)
#pragma unroll
      for (int t = 0; t < DL; ++t) o[h][t] = 0.f;
    const int nvalid = max(0, min(PW, p1 - (p0 + warp * PW)));
#pragma unroll 4
    for (int j = 0; j < nvalid; ++j) {
      const int jl = warp * PW + j;
      const float* vrow = (p0 + jl == pos) ? vn : Vt + (size_t)jl * HD;
      float v[DL];
#pragma unroll
      for (int t = 0; t < DL; ++t) v[t] = vrow[lane + 32 * t];
#pragma unroll
      for (int h = 0; h < REP; ++h) {
        const float pj_h = pw[warp][h][j];
#pragma unroll
        for (int t = 0; t < DL; ++t) o[h][t] = fmaf(pj_h, v[t], o[h][t]);
      }
    }
#pragma unroll
    for (int h = 0; h < REP; ++h)
#pragma unroll
      for (int t = 0; t < DL; ++t) ow[warp][h][lane + 32 * t] = o[h][t];
    __syncthreads();
    // ---- merge the four warps into this split's (m, l, o) ----
    for (int i = threadIdx.x; i < REP * HD; i += kTThreads) {
      const int h = i / HD, d = i - h * HD;
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < kTWarps; ++w) M = fmaxf(M, mw[w][h]);
      float L = 0.f, O = 0.f;
#pragma unroll
      for (int w = 0; w < kTWarps; ++w) {
        const float m = mw[w][h];
        if (m != -INFINITY) {
          const float f = expf(m - M);
          L = fmaf(lw[w][h], f, L);
          O = fmaf(ow[w][h][d], f, O);
        }
      }
      if (!tile_ok) { M = -INFINITY; L = 0.f; O = 0.f; }   // a timed-out copy contributes nothing
      part[h * (HD + 2) + 2 + d] = O;
      if (d == 0) { part[h * (HD + 2)] = M; part[h * (HD + 2) + 1] = L; }
    }
  } else {
    for (int h = threadIdx.x; h < REP; h += kTThreads) { part[h * (HD + 2)] = -INFINITY; part[h * (HD + 2) + 1] = 0.f; }
  }
  __syncthreads();   // every thread's stores, then (cumulative) thread 0's fence and count
  if (threadIdx.x == 0) {
    __threadfence();
    last = (atomicAdd(&a.cnt[kh], 1u) == (uint32_t)S - 1) ? 1u : 0u;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  // ---- merge the splits of this kv group (+ attention sink) ----
  const float* gp = a.part + (size_t)kh * S * REP * (HD + 2);
  float* hm = &mw[0][0];
  float* hinv = &lw[0][0];
  for (int i = threadIdx.x; i < S * REP; i += kTThreads) wsm[i] = __ldcg(&gp[(size_t)i * (HD + 2)]);
  __syncthreads();
  for (int h = threadIdx.x; h < REP; h += kTThreads) {
    float M = -INFINITY;
    for (int s = 0; s < S; ++s) M = fmaxf(M, wsm[s * REP + h]);
    float sink = 0.f;
    if (a.sinks) { sink = a.sinks[kh * REP + h]; M = 0.5f * ((M + sink) + fabsf(M - sink)); }
    float L = 0.f;
    for (int s = 0; s < S; ++s) {
      const float m = wsm[s * REP + h];
      if (m != -INFINITY) L += __ldcg(&gp[((size_t)s * REP + h) * (HD + 2) + 1]) * expf(m - M);
    }
    if (a.sinks) L += expf(sink - M);
    hm[h] = M;
    hinv[h] = 1.0f / L;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < S * REP; i += kTThreads) {
    const int h = i % REP;
    const float m = wsm[i];
    wsm[i] = (m == -INFINITY) ? 0.f : expf(m - hm[h]) * hinv[h];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < REP * HD; i += kTThreads) {
    const int h = i / HD, d = i - h * HD;
    const float* src = gp + (size_t)h * (HD + 2) + 2 + d;
    const size_t stride = (size_t)REP * (HD + 2);
    float o = 0.f;
    int s = 0;
    for (; s + 8 <= S; s += 8) {
      float v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = __ldcg(src + (size_t)(s + u) * stride);
#pragma unroll
      for (int u = 0; u < 8; ++u) o = fmaf(wsm[(s + u) * REP + h], v[u], o);
    }
    for (; s < S; ++s) o = fmaf(wsm[s * REP + h], __ldcg(src + (size_t)s * stride), o);
    a.out[(size_t)(kh * REP + h) * HD + d] = o;
    if (a.oq) ow[0][h][d] = o;
  }
  if (a.oq) {   // Q8_0 blocks of this group's output (the O-projection's activation)
    __syncthreads();
    const float* og = &ow[0][0][0];
    for (int bl = threadIdx.x; bl < REP * HD / 32; bl += kTThreads) {
      float v[32];
#pragma unroll
      for (int k = 0; k < 32; ++k) v[k] = og[32 * bl + k];
      const int gb = kh * REP * HD / 32 + bl;
      quantize_q8_block(v, a.oq + 32 * gb, &a.od[gb]);
    }
  }
  if (threadIdx.x == 0) a.cnt[kh] = 0u;
}

template <int HD, int REP, int PB, int MINB>
__global__ void __launch_bounds__(kAThreads, MINB) attn_decode_kernel(AttnArgs a, uint32_t* err) {
  constexpr int DPL = HD / 32;                 // head dims per lane
  constexpr int GL = 32 / REP;                 // lanes per head after the reduce-scatter
  extern __shared__ __align__(128) float dyn[];
  float* ow = dyn;                             // [kAWarps][REP][HD] per-warp outputs
  float* wsm = ow + kAWarps * REP * HD;        // [S][REP] split weights of the final merge
  __shared__ __align__(16) float qs[REP * HD];
  __shared__ __align__(16) float kn[HD];
  __shared__ __align__(16) float vn[HD];
  __shared__ float psm[kAWarps][REP][kAChunk];   // a chunk's scores, then its softmax weights
  __shared__ float mw[kAWarps][REP], lw[kAWarps][REP];
  __shared__ uint32_t last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int vh = blockIdx.y, kh = vh / a.head_split, sidx = blockIdx.x, S = gridDim.x;   // vh: kv head x query-head group
  if (blockIdx.z) {   // sequence b of a lockstep batch
    const int64_t b = blockIdx.z;
    a.qkv += b * a.bs_qkv;
    a.kc += b * a.bs_kv;
    a.vc += b * a.bs_kv;
    a.out += b * a.bs_out;
    if (a.oq) { a.oq += b * a.bs_out; a.od += b * a.bs_out / 32; }
    a.part += b * (int64_t)gridDim.y * S * REP * (HD + 2);
    a.cnt += b * gridDim.y;
  }
  // The position comes from the step's first kernel and the cached rows from earlier steps, both
  // complete before the previous kernel started (every kernel lets its dependents launch only after
  // its own wait), so the first chunk's rows can be prefetched before this kernel waits.
  const int spl = a.spl;
  const int pos = *a.pos;
  const int lo = a.window ? max(0, pos - a.window + 1) : 0;
  const int p0 = lo + sidx * spl, p1 = min(p0 + spl, pos + 1);
  const bool active = p0 < p1;
  const bool has_new = active && p1 == pos + 1;
  const float* kbase = a.kc + (size_t)kh * a.cap * HD;
  const float* vbase = a.vc + (size_t)kh * a.cap * HD;
  auto slot_of = [&](int q) { return a.window ? q % a.cap : q; };   // kv_cache.rs:37-60 (ring for SWA)
  // chunks of this warp: c0, c0 + kAWarps, ... (32 positions each)
  auto prefetch_chunk = [&](int cb) {
    constexpr int LPR = HD * 4 / 128;           // 128-byte lines per row
    for (int i = lane; i < 2 * kAChunk * LPR; i += 32) {
      const int r = i / (2 * LPR), pt = i % (2 * LPR), q = cb + r;
      if (q < min(p1, pos)) {
        const float* base = (pt < LPR ? kbase : vbase) + (size_t)slot_of(q) * HD + (pt % LPR) * 32;
        asm volatile("prefetch.global.L2 [%0];" ::"l"(base));
      }
    }
  };
  if (active && p0 + warp * kAChunk < p1) prefetch_chunk(p0 + warp * kAChunk);
  pdl_wait_prior();
  pdl_launch_dependents();
  const int half = a.rot / 2;
  float* part = a.part + ((size_t)vh * S + sidx) * REP * (HD + 2);
  if (active) {
    const float* cs = a.cos_t + (size_t)pos * half;
    const float* sn = a.sin_t + (size_t)pos * half;
    for (int i = threadIdx.x; i < REP * HD; i += kAThreads) qs[i] = a.qkv[(size_t)vh * REP * HD + i];
    if (has_new) {
      const float* kq = a.qkv + (size_t)a.nh * HD + (size_t)kh * HD;
      const float* vq = kq + (size_t)a.nkv * HD;
      for (int i = threadIdx.x; i < HD; i += kAThreads) { kn[i] = kq[i]; vn[i] = vq[i]; }
    }
    __syncthreads();
    if (a.q_norm) {
      for (int h = warp; h < REP; h += kAWarps) head_norm_warp(qs + h * HD, a.q_norm, HD, a.eps, lane);
      if (has_new && warp == 0) head_norm_warp(kn, a.k_norm, HD, a.eps, lane);
      __syncthreads();
    }
    for (int h = 0; h < REP; ++h) rope_inplace(qs + h * HD, a.rot, cs, sn);
    if (has_new) rope_inplace(kn, a.rot, cs, sn);
    __syncthreads();
    if (has_new && vh % a.head_split == 0) {   // kv_cache.rs:37-60 append (by the kv head's first query-head group)
      float* kd = a.kc + ((size_t)kh * a.cap + slot_of(pos)) * HD;
      float* vd = a.vc + ((size_t)kh * a.cap + slot_of(pos)) * HD;
      for (int i = threadIdx.x; i < HD; i += kAThreads) { kd[i] = kn[i]; vd[i] = vn[i]; }
    }
    const int my_h = lane / GL, gi = lane % GL;
    // query heads in lane order h ^ my_h: the reduce-scatter below then always keeps the lower half
    float qr[REP][DPL];
#pragma unroll
    for (int h = 0; h < REP; ++h)
#pragma unroll
      for (int d = 0; d < DPL; ++d) qr[h][d] = qs[(h ^ my_h) * HD + lane * DPL + d];
    float o[REP][DPL];
#pragma unroll
    for (int h = 0; h < REP; ++h)
#pragma unroll
      for (int d = 0; d < DPL; ++d) o[h][d] = 0.f;
    float M = -INFINITY, L = 0.f;   // softmax state of head my_h
    auto load_rows = [&](const float* base, const float* nrow, int q, int w1, float (&r)[DPL]) {
      if (q >= w1) {
#pragma unroll
        for (int d = 0; d < DPL; ++d) r[d] = 0.f;
      } else if (q == pos) {
#pragma unroll
        for (int d = 0; d < DPL; ++d) r[d] = nrow[lane * DPL + d];
      } else {
        const float* src = base + (size_t)slot_of(q) * HD + lane * DPL;
        if constexpr (DPL % 4 == 0) {
#pragma unroll
          for (int d = 0; d < DPL; d += 4) {
            const float4 v = __ldg(reinterpret_cast<const float4*>(src + d));
            r[d] = v.x; r[d + 1] = v.y; r[d + 2] = v.z; r[d + 3] = v.w;
          }
        } else if constexpr (DPL % 2 == 0) {
#pragma unroll
          for (int d = 0; d < DPL; d += 2) {
            const float2 v = __ldg(reinterpret_cast<const float2*>(src + d));
            r[d] = v.x; r[d + 1] = v.y;
          }
        } else {
#pragma unroll
          for (int d = 0; d < DPL; ++d) r[d] = __ldg(src + d);   // head_dim 32: one value per lane
        }
      }
    };
    for (int cb = p0 + warp * kAChunk; cb < p1; cb += kAWarps * kAChunk) {
      const int w1 = min(cb + kAChunk, p1);
      // a full chunk without the new row, contiguous in the cache: plain strided row loads
      const bool fast = w1 - cb == kAChunk && !(cb <= pos && pos < cb + kAChunk) &&
                        (!a.window || slot_of(cb) + kAChunk <= a.cap);
      const size_t row0 = (size_t)(fast ? slot_of(cb) : 0) * HD + lane * DPL;
      auto load_fast = [&](const float* base, int u, float (&r)[DPL]) {
        const float* src = base + row0 + (size_t)u * HD;
        if constexpr (DPL % 4 == 0) {
#pragma unroll
          for (int d = 0; d < DPL; d += 4) {
            const float4 v = __ldg(reinterpret_cast<const float4*>(src + d));
            r[d] = v.x; r[d + 1] = v.y; r[d + 2] = v.z; r[d + 3] = v.w;
          }
        } else if constexpr (DPL % 2 == 0) {
#pragma unroll
          for (int d = 0; d < DPL; d += 2) {
            const float2 v = __ldg(reinterpret_cast<const float2*>(src + d));
            r[d] = v.x; r[d + 1] = v.y;
          }
        } else {
#pragma unroll
          for (int d = 0; d < DPL; ++d) r[d] = __ldg(src + d);   // head_dim 32: one value per lane
        }
      };
      if (cb + kAWarps * kAChunk < p1) prefetch_chunk(cb + kAWarps * kAChunk);
      // ---- scores of the chunk's positions -> psm[warp][h][j] ----
#pragma unroll 1
      for (int jb = 0; jb < kAChunk; jb += PB) {
        float kr[PB][DPL];
#pragma unroll
        for (int u = 0; u < PB; ++u) {
          if (fast) load_fast(kbase, jb + u, kr[u]);
          else load_rows(kbase, kn, cb + jb + u, w1, kr[u]);
        }
#pragma unroll
        for (int u = 0; u < PB; ++u) {
          float v[REP];
#pragma unroll
          for (int h = 0; h < REP; ++h) {
            float t = 0.f;
#pragma unroll
            for (int d = 0; d < DPL; ++d) t = fmaf(qr[h][d], kr[u][d], t);
            v[h] = t;
          }
          // reduce-scatter: v[i] is head i ^ my_h, so each halving step keeps v[0 .. n/2) and adds the
          // partner's v[n/2 .. n) (the same heads in its order); v[0] ends as head my_h, then a sum
          // over its GL lanes
#pragma unroll
          for (int o2 = 16, n = REP; n > 1; o2 >>= 1, n >>= 1) {
#pragma unroll
            for (int i = 0; i < n / 2; ++i) v[i] += __shfl_xor_sync(0xffffffffu, v[i + n / 2], o2);
          }
#pragma unroll
          for (int o2 = GL / 2; o2 > 0; o2 >>= 1) v[0] += __shfl_xor_sync(0xffffffffu, v[0], o2);
          if (gi == 0) psm[warp][my_h][jb + u] = (cb + jb + u < w1) ? v[0] * a.scale : -INFINITY;
        }
      }
      __syncwarp();
      // ---- online softmax: lane (h, gi) owns positions gi, gi + GL, ... of head h ----
      float cm = -INFINITY;
      for (int j = gi; j < kAChunk; j += GL) cm = fmaxf(cm, psm[warp][my_h][j]);
#pragma unroll
      for (int o2 = GL / 2; o2 > 0; o2 >>= 1) cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, o2));
      const float Mn = fmaxf(M, cm);
      const float corr = (M == -INFINITY) ? 0.f : expf(M - Mn);
      float cl = 0.f;
      for (int j = gi; j < kAChunk; j += GL) {
        const float sv = psm[warp][my_h][j];
        const float pe = (sv == -INFINITY) ? 0.f : expf(sv - Mn);
        psm[warp][my_h][j] = pe;
        cl += pe;
      }
#pragma unroll
      for (int o2 = GL / 2; o2 > 0; o2 >>= 1) cl += __shfl_xor_sync(0xffffffffu, cl, o2);
      L = L * corr + cl;
      M = Mn;
      __syncwarp();
#pragma unroll
      for (int h = 0; h < REP; ++h) {
        const float ch = __shfl_sync(0xffffffffu, corr, h * GL);
#pragma unroll
        for (int d = 0; d < DPL; ++d) o[h][d] *= ch;
      }
      // ---- P * V over this lane's dims ----
#pragma unroll 1
      for (int jb = 0; jb < kAChunk; jb += PB) {
        float vr[PB][DPL];
#pragma unroll
        for (int u = 0; u < PB; ++u) {
          if (fast) load_fast(vbase, jb + u, vr[u]);
          else load_rows(vbase, vn, cb + jb + u, w1, vr[u]);
        }
#pragma unroll
        for (int u = 0; u < PB; ++u) {
#pragma unroll
          for (int h = 0; h < REP; ++h) {
            const float pj = psm[warp][h][jb + u];
#pragma unroll
            for (int d = 0; d < DPL; ++d) o[h][d] = fmaf(pj, vr[u][d], o[h][d]);
          }
        }
      }
      __syncwarp();
    }
    if (gi == 0) { mw[warp][my_h] = M; lw[warp][my_h] = L; }
#pragma unroll
    for (int h = 0; h < REP; ++h)
#pragma unroll
      for (int d = 0; d < DPL; ++d) ow[(warp * REP + h) * HD + lane * DPL + d] = o[h][d];
    __syncthreads();
    // ---- merge the warps into this split's (m, l, o) ----
    for (int i = threadIdx.x; i < REP * HD; i += kAThreads) {
      const int h = i / HD, d = i - h * HD;
      float Mx = -INFINITY;
#pragma unroll
      for (int w = 0; w < kAWarps; ++w) Mx = fmaxf(Mx, mw[w][h]);
      float Ls = 0.f, Os = 0.f;
#pragma unroll
      for (int w = 0; w < kAWarps; ++w) {
        const float mm = mw[w][h];
        if (mm != -INFINITY) {
          const float f = expf(mm - Mx);
          Ls = fmaf(lw[w][h], f, Ls);
          Os = fmaf(ow[(w * REP + h) * HD + d], f, Os);
        }
      }
      part[h * (HD + 2) + 2 + d] = Os;
      if (d == 0) { part[h * (HD + 2)] = Mx; part[h * (HD + 2) + 1] = Ls; }
    }
  } else {
    for (int h = threadIdx.x; h < REP; h += kAThreads) { part[h * (HD + 2)] = -INFINITY; part[h * (HD + 2) + 1] = 0.f; }
  }
  __syncthreads();   // every thread's stores, then (cumulative) thread 0's fence and count
  if (threadIdx.x == 0) {
    __threadfence();
    last = (atomicAdd(&a.cnt[vh], 1u) == (uint32_t)S - 1) ? 1u : 0u;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  // ---- merge the splits of this kv group (+ attention sink) ----
  const float* gp = a.part + (size_t)vh * S * REP * (HD + 2);
  float* hm = &mw[0][0];
  float* hinv = &lw[0][0];
  for (int i = threadIdx.x; i < S * REP; i += kAThreads) wsm[i] = __ldcg(&gp[(size_t)i * (HD + 2)]);
  __syncthreads();
  for (int h = threadIdx.x; h < REP; h += kAThreads) {
    float M = -INFINITY;
    for (int s = 0; s < S; ++s) M = fmaxf(M, wsm[s * REP + h]);
    float sink = 0.f;
    if (a.sinks) { sink = a.sinks[vh * REP + h]; M = 0.5f * ((M + sink) + fabsf(M - sink)); }
    float L = 0.f;
    for (int s = 0; s < S; ++s) {
      const float m = wsm[s * REP + h];
      if (m != -INFINITY) L += __ldcg(&gp[((size_t)s * REP + h) * (HD + 2) + 1]) * expf(m - M);
    }
    if (a.sinks) L += expf(sink - M);
    hm[h] = M;
    hinv[h] = 1.0f / L;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < S * REP; i += kAThreads) {
    const int h = i % REP;
    const float m = wsm[i];
    wsm[i] = (m == -INFINITY) ? 0.f : expf(m - hm[h]) * hinv[h];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < REP * HD; i += kAThreads) {
    const int h = i / HD, d = i - h * HD;
    const float* src = gp + (size_t)h * (HD + 2) + 2 + d;
    const size_t stride = (size_t)REP * (HD + 2);
    float o = 0.f;
    int s = 0;
    for (; s + 8 <= S; s += 8) {
      float v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = __ldcg(src + (size_t)(s + u) * stride);
#pragma unroll
      for (int u = 0; u < 8; ++u) o = fmaf(wsm[(s + u) * REP + h], v[u], o);
    }
    for (; s < S; ++s) o = fmaf(wsm[s * REP + h], __ldcg(src + (size_t)s * stride), o);
    a.out[(size_t)(vh * REP + h) * HD + d] = o;
    if (a.oq) ow[h * HD + d] = o;
  }
  if (a.oq) {   // Q8_0 blocks of this group's output (the O-projection's activation)
    __syncthreads();
    const float* og = ow;
    for (int bl = threadIdx.x; bl < REP * HD / 32; bl += kAThreads) {
      float v[32];
#pragma unroll
      for (int k = 0; k < 32; ++k) v[k] = og[32 * bl + k];
      const int gb = vh * REP * HD / 32 + bl;
      quantize_q8_block(v, a.oq + 32 * gb, &a.od[gb]);
    }
  }
  if (threadIdx.x == 0) a.cnt[vh] = 0u;
}

// ============================ gated attention (hybrid models, layer.rs:620-635, 699-705) ============================
// The Q projection of a hybrid attention layer holds [Q_h, gate_h] per head: y [2 Dq + 2 Dkv] ->
// the plain layout qkv [Dq + 2 Dkv] (q of every head, then k, v) and gate [Dq].
__global__ void gate_split_kernel(const float* __restrict__ y, int nh, int hd, int Dkv, float* __restrict__ qkv,
                                  float* __restrict__ gate) {
  pdl_wait_prior();
  pdl_launch_dependents();
  const int Dq = nh * hd;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < Dq + 2 * Dkv; i += gridDim.x * blockDim.x) {
    if (i < Dq) {
      const int h = i / hd, d = i - h * hd;
      qkv[i] = y[(size_t)h * 2 * hd + d];
      gate[i] = y[(size_t)h * 2 * hd + hd + d];
    } else {
      qkv[i] = y[Dq + i];   // k, v follow the 2 Dq gated query rows
    }
  }
}

// attn *= sigmoid(gate) with sigmoid = recip(exp(-x) + 1) (ops/activation.rs:41-45), then the
// O projection's Q8_0 activation: one thread per 32-element block
__global__ void gate_apply_q8_kernel(float* __restrict__ att, const float* __restrict__ gate, int n,
                                     int8_t* __restrict__ oq, float* __restrict__ od) {
  pdl_wait_prior();
  pdl_launch_dependents();
  for (int b = blockIdx.x * blockDim.x + threadIdx.x; b < n / 32; b += gridDim.x * blockDim.x) {
    float v[32];
#pragma unroll
    for (int k = 0; k < 32; ++k) {
      const int i = 32 * b + k;
      const float sg = __fdiv_rn(1.0f, __fadd_rn(expcr(-gate[i]), 1.0f));
      v[k] = __fmul_rn(att[i], sg);
      att[i] = v[k];
    }
    quantize_q8_block(v, oq + 32 * b, &od[b]);
  }
}

// ============================ LM head (f16) + argmax ============================
// Warp per row, 16-byte streaming loads; x (after the final RMSNorm) in registers.
constexpr int kLWarps = 8;
constexpr int kLMaxChunks = 16;   // H <= 16*32*8 = 4096

__device__ __forceinline__ unsigned long long argmax_key(float v, int idx) {
  uint32_t b = __float_as_uint(v);
  b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return ((unsigned long long)b << 32) | (uint32_t)(0xffffffffu - (uint32_t)idx);
}

template <int NCH>
__global__ void __launch_bounds__(kLWarps * 32, 1) lmhead_kernel(LmHeadArgs a) {
  extern __shared__ __align__(16) float xs[];
  __shared__ unsigned long long bestk[kLWarps];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_wait_prior();
  pdl_launch_dependents();   // the next kernel may start its own (weight) prefetch now
  for (int i = threadIdx.x; i < a.H; i += blockDim.x) {
    const float v = a.x[i];
    xs[i] = v;
    if (a.x_out && blockIdx.x == 0) a.x_out[i] = v;
  }
  __syncthreads();
  float inv = 1.f;
  if (a.norm_w) inv = rms_inv_cr(xs, a.H, a.eps, threadIdx.x, blockDim.x, [] { __syncthreads(); });
  __syncthreads();
  for (int i = threadIdx.x; i < a.H; i += blockDim.x) {
    xs[i] = a.norm_w ? __fmul_rn(__fmul_rn(xs[i], inv), a.norm_w[i]) : xs[i];
    if (a.xn_out && blockIdx.x == 0) a.xn_out[i] = xs[i];
  }
  __syncthreads();
  const int nch = a.H / 8;
  float xr[NCH][8];
#pragma unroll
  for (int i = 0; i < NCH; ++i) {
    const int ch = lane + 32 * i;
#pragma unroll
    for (int k = 0; k < 8; ++k) xr[i][k] = (ch < nch) ? xs[8 * ch + k] : 0.f;
  }
  const int rows_per = (a.V + gridDim.x - 1) / gridDim.x;
  const int rb = blockIdx.x * rows_per, re = min(a.V, rb + rows_per);
  unsigned long long best = 0ull;
  for (int r = rb + warp; r < re; r += kLWarps) {
    const uint4* wr = reinterpret_cast<const uint4*>(a.w + (size_t)r * a.H);
    uint4 wv[NCH];
#pragma unroll
    for (int i = 0; i < NCH; ++i) {
      const int ch = lane + 32 * i;
      if (ch < nch) wv[i] = __ldcs(wr + ch);
      else wv[i] = make_uint4(0, 0, 0, 0);
    }
    // f32 accumulation; with order-independent numerics the greedy token is then re-scored exactly
    // among the near-maximal ids (launch_exact_argmax_refine)
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < NCH; ++i) {
      const uint32_t u[4] = {wv[i].x, wv[i].y, wv[i].z, wv[i].w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&u[k]));
        acc = fmaf(f.x, xr[i][2 * k], acc);
        acc = fmaf(f.y, xr[i][2 * k + 1], acc);
      }
    }
    acc = warp_sum(acc);
    if (lane == 0) {
      float v = acc;
      if (a.bias) v = __fadd_rn(v, a.bias[r]);
      if (a.logits) { if (a.accumulate) v += a.logits[r]; a.logits[r] = v; }
      if (v == v) { const unsigned long long k = argmax_key(v, r); best = k > best ? k : best; }
    }
  }
  if (lane == 0) bestk[warp] = best;
  __syncthreads();
  if (threadIdx.x == 0 && a.key) {
    unsigned long long b = 0ull;
    for (int w = 0; w < kLWarps; ++w) b = bestk[w] > b ? bestk[w] : b;
    if (b) atomicMax(a.key, b);
  }
}

// ============================ f32 GEMV ============================
__global__ void gemv_f32_kernel(const float* __restrict__ w, int rows, int cols, const float* __restrict__ x,
                                const float* __restrict__ bias, float* __restrict__ y, int accumulate) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= rows) return;
  const float* wr = w + (size_t)warp * cols;
  float acc = 0.f;
  for (int i = lane; i < cols; i += 32) acc = fmaf(wr[i], x[i], acc);
  acc = warp_sum(acc);
  if (lane == 0) {
    float v = acc + (bias ? bias[warp] : 0.f);
    y[warp] = accumulate ? y[warp] + v : v;
  }
}

// ============================ embedding / step start ============================
__global__ void __launch_bounds__(1024) embed_kernel(StepState* st, const void* table, int q, int H, int vocab, float* h, int* log,
                             uint32_t* err, const float* norm_w, float eps, int8_t* xq, float* xd) {
  extern __shared__ float es[];   // [H]
  __shared__ int tok_s;
  __shared__ float red[256];
  pdl_wait_prior();
  pdl_launch_dependents();   // the next kernel may start its own (weight) prefetch now
  if (threadIdx.x == 0) {
    int tok = st->token_in;
    if (st->use_argmax) {
      const unsigned long long k = st->key;
      tok = (int)(0xffffffffu - (uint32_t)(k & 0xffffffffull));
      if (k == 0ull) tok = 0;
    }
    if (tok < 0 || tok >= vocab) { atomicOr(err, EF_BAD_INDEX); tok = 0; }
    int pos = st->n_ctx;
    if (pos >= st->max_seq) { atomicOr(err, EF_BAD_SHAPE); pos = st->max_seq - 1; }
    st->pos = pos;
    st->n_ctx = pos + 1;
    st->last_token = tok;
    st->key = 0ull;
    if (log && st->n_log < st->max_seq) log[st->n_log] = tok;
    st->n_log = st->n_log + 1;
    tok_s = tok;
  }
  __syncthreads();
  const int tok = tok_s;
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    const float v = (q == Q_F16) ? __half2float(reinterpret_cast<const __half*>(table)[(size_t)tok * H + i])
                                 : reinterpret_cast<const float*>(table)[(size_t)tok * H + i];
    h[i] = v;
    es[i] = v;
  }
  if (!norm_w) return;
  __syncthreads();
  cta_rmsnorm_q8(es, H, norm_w, eps, xq, xd, red);   // layer 0's attention input
}

// h += MoE output (slots in ascending expert order, or the expert-parallel sum), then the next
// layer's attention input: RMSNorm + Q8_0 quantization (when norm_w is set).  One CTA.
// h += the pending MoE combine, spread over ceil(H / 256) CTAs of 256 rows each; the last CTA to
// finish (counter) then normalises the whole h with the next layer's attention norm and writes
// its Q8_0 blocks.
constexpr int kResidRows = 256;
__global__ void __launch_bounds__(kResidRows) resid_norm_q8_kernel(PendingCombine pc, float* h, int H,
                                                                   const float* norm_w, float eps, int8_t* xq,
                                                                   float* xd, uint32_t* cnt, uint32_t* err) {
  extern __shared__ float hs[];   // [H] (last CTA)
  __shared__ CombineOrder co;
  __shared__ float red[256];
  __shared__ int s_idx[16];
  __shared__ float s_wts[16];
  __shared__ uint32_t last;
  pdl_wait_prior();
  pdl_launch_dependents();   // the next kernel may start its own (weight) prefetch now
  if (threadIdx.x < pc.K && threadIdx.x < 16 && pc.idx) {   // routing read in parallel, sorted by one thread
    s_idx[threadIdx.x] = pc.idx[threadIdx.x];
    s_wts[threadIdx.x] = pc.wts[threadIdx.x];
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    if (pc.ep_recv) ep_wait(pc, &co, err);   // the other ranks' partial outputs have landed
    combine_order(pc, &co, pc.idx ? s_idx : nullptr, pc.idx ? s_wts : nullptr);
  }
  __syncthreads();
  combine_prepare(pc, &co);
  __syncthreads();
  const int r = blockIdx.x * kResidRows + threadIdx.x;
  if (r < H) {
    const float moe = combine_at(pc, co, H, r);
    h[r] = h[r] + (pc.extra ? __fadd_rn(moe, pc.extra[r]) : moe);
  }
  if (!norm_w) return;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();   // this CTA's rows (ordered before by the barrier), then the count
    last = (atomicAdd(cnt, 1u) == gridDim.x - 1) ? 1u : 0u;
    if (last) __threadfence();
  }
  __syncthreads();
  if (!last) return;
  for (int i = threadIdx.x; i < H; i += blockDim.x) hs[i] = __ldcg(&h[i]);
  __syncthreads();
  cta_rmsnorm_q8(hs, H, norm_w, eps, xq, xd, red);
  if (threadIdx.x == 0) *cnt = 0u;
}

// Expert parallel over peer memory: this rank's MoE output (the pending combine of its local
// experts) is stored into slot [parity][rank] of every rank's mailbox over NVLink; the last CTA
// then releases flag [parity][rank] at every rank with the step's sequence number.  A mailbox slot
// of parity p is rewritten two steps later, after every rank has consumed it (the next step's
// combine needs every rank's release, which each rank issues after its own consumption).
__global__ void __launch_bounds__(256) ep_send_kernel(PendingCombine pc, int H, EpSend e) {
  __shared__ CombineOrder co;
  __shared__ uint32_t s_seq, last;
  pdl_wait_prior();
  pdl_launch_dependents();
  if (threadIdx.x == 0) {
    combine_order(pc, &co);
    s_seq = *reinterpret_cast<const volatile uint32_t*>(e.seq) + 1u;
  }
  __syncthreads();
  combine_prepare(pc, &co);
  __syncthreads();
  const uint32_t seq = s_seq, par = seq & 1u;
  for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < H; r += gridDim.x * blockDim.x) {
    if (e.slots) {   // each local slot's own output, so every rank combines all slots in one order
      for (int q = 0; q < co.n; ++q) {
        const int k = co.slot[q];
        const float v = slot_value(pc, k, H, r);
        for (int j = 0; j < e.n; ++j) e.recv[j][((size_t)par * e.rows + k) * H + r] = v;
      }
    } else {
      const float v = combine_at(pc, co, H, r);
      for (int j = 0; j < e.n; ++j) e.recv[j][((size_t)par * e.rows + e.rank) * H + r] = v;
    }
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) last = (atomicAdd(e.cnt, 1u) == gridDim.x - 1) ? 1u : 0u;
  __syncthreads();
  if (!last) return;
  __threadfence_system();
  if ((int)threadIdx.x < e.n) st_release_sys_u32(e.flags[threadIdx.x] + par * e.n + e.rank, seq);
  if (threadIdx.x == 0) {
    *e.seq = seq;
    *e.cnt = 0u;
  }
}

template <class Kern, class... Args>
cudaError_t launch_pdl(Kern k, dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args... args) {
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

}  // namespace

cudaError_t launch_dequantize(const DevCtx& c, int q, const void* blocks, int64_t n, float* out, cudaStream_t s) {
  if (n <= 0) return cudaSuccess;
  const int bs = 256;
  dequant_kernel<<<(unsigned)((n + bs - 1) / bs), bs, 0, s>>>(q, (const uint8_t*)blocks, n, out);
  return cudaGetLastError();
}

// NeoX half-rotation of the first `rot` dims of every head (ops/attention.rs:96-164): for i < rot/2,
// out[i] = x[i] c - x[i + rot/2] s and out[i + rot/2] = x[i + rot/2] c + x[i] s; dims >= rot pass
// through.  Products and sums are rounded separately (no fused multiply-add), as the reference's
// separate tensor ops round them.  One thread per (token, head, dim); cos/sin rows per token.
__global__ void rope_kernel(const float* __restrict__ x, const float* __restrict__ cs, const float* __restrict__ sn,
                            float* __restrict__ y, int n_tok, int heads, int hd, int rot) {
  const int64_t total = (int64_t)n_tok * heads * hd;
  const int half = rot / 2;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int d = (int)(i % hd);
    const int64_t t = i / ((int64_t)heads * hd);
    const float* xh = x + (i - d);
    float v;
    if (d < half) {
      const float c = cs[t * half + d], s = sn[t * half + d];
      v = __fsub_rn(__fmul_rn(xh[d], c), __fmul_rn(xh[d + half], s));
    } else if (d < rot) {
      const float c = cs[t * half + d - half], s = sn[t * half + d - half];
      v = __fadd_rn(__fmul_rn(xh[d], c), __fmul_rn(xh[d - half], s));
    } else {
      v = xh[d];
    }
    y[i] = v;
  }
}

cudaError_t launch_gate_split(const float* y, int nh, int hd, int Dkv, float* qkv, float* gate, cudaStream_t s) {
  const int n = nh * hd + 2 * Dkv;
  return launch_pdl(gate_split_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, s, y, nh, hd, Dkv, qkv, gate);
}

cudaError_t launch_gate_apply_q8(float* att, const float* gate, int n, int8_t* oq, float* od, cudaStream_t s) {
  if (n % 32) return cudaErrorInvalidValue;
  return launch_pdl(gate_apply_q8_kernel, dim3((unsigned)((n / 32 + 127) / 128)), dim3(128), 0, s, att, gate, n, oq,
                    od);
}

cudaError_t launch_rope(const float* x, const float* cs, const float* sn, float* y, int n_tok, int heads, int hd,
                        int rot, cudaStream_t s) {
  const int64_t total = (int64_t)n_tok * heads * hd;
  const int blocks = (int)std::min<int64_t>((total + 255) / 256, 4096);
  rope_kernel<<<blocks, 256, 0, s>>>(x, cs, sn, y, n_tok, heads, hd, rot);
  return cudaGetLastError();
}

__global__ void set_i32_kernel(int* p, int v) { *p = v; }
cudaError_t launch_set_i32(int* p, int v, cudaStream_t s) {
  set_i32_kernel<<<1, 1, 0, s>>>(p, v);
  return cudaGetLastError();
}

cudaError_t launch_rms_norm(const DevCtx& c, const float* x, const float* w, float* y, int rows, int dim, float eps,
                            cudaStream_t s) {
  rms_norm_kernel<<<rows, 256, 0, s>>>(x, w, y, dim, eps);
  return cudaGetLastError();
}

cudaError_t launch_q8_gemv(const DevCtx& c, const Q8GemvArgs& a, cudaStream_t s) {
  if (a.exact || a.cols % 32 || a.rows <= 0) return cudaErrorInvalidValue;
  Q8Params p = {};
  p.w = a.w; p.rows = a.rows; p.cols = a.cols; p.rb = a.cols / 32 * 34;
  int u = 1;
  while ((int64_t)u * p.rb % 16) u *= 2;
  p.unit_rows = u;                              // smallest row count whose bytes are a multiple of 16
  p.n_units = (a.rows + u - 1) / u;
  p.stage_rows = kQW;                           // one row per consumer warp
  if (p.stage_rows % u) p.stage_rows = u;       // (u <= 16; rows per stage must keep alignment)
  p.stage_bytes = (int)((((int64_t)p.stage_rows * p.rb) + 15) & ~15ll);
  // <= ~128 KB of stages, so the neighbouring kernels' CTAs (attention, MoE) fit beside this one
  p.ns = (int)((128 * 1024) / p.stage_bytes);
  p.ns = p.ns > 5 ? 5 : (p.ns < 2 ? 2 : p.ns);
  p.x = a.x; p.norm_w = a.norm_w; p.eps = a.eps; p.bias = a.bias; p.y = a.y; p.residual = a.residual;
  p.xq_in = a.xq_in; p.xd_in = a.xd_in;
  p.err = c.err;
  const int nbl = (a.cols / 32 + 31) / 32;
  if (p.stage_rows > kQW) return cudaErrorInvalidValue;
  if (nbl <= 1) return launch_q8<1>(c, p, s);
  if (nbl <= 2) return launch_q8<2>(c, p, s);
  if (nbl <= 3) return launch_q8<3>(c, p, s);
  if (nbl <= 4) return launch_q8<4>(c, p, s);
  if (nbl <= 8) return launch_q8<8>(c, p, s);
  return cudaErrorInvalidValue;
}

template <int HD, int REP>
cudaError_t launch_attn_k(const AttnArgs& a, const DevCtx& c, dim3 grid, cudaStream_t s) {
  if (a.spl == 0) {   // one sequence: K/V tiles staged in shared memory before the wait
    const size_t smem = ((size_t)2 * attn_tile_len(HD) * HD + (size_t)a.S * REP) * sizeof(float);
    cudaError_t e = cudaFuncSetAttribute(attn_tile_kernel<HD, REP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return e;
    return launch_pdl(attn_tile_kernel<HD, REP>, grid, dim3(kTThreads), smem, s, a, c.err);
  }
  const size_t smem = ((size_t)kAWarps * REP * HD + (size_t)a.S * REP) * sizeof(float);
  cudaError_t e = cudaFuncSetAttribute(attn_decode_kernel<HD, REP, 8, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem);
  if (e != cudaSuccess) return e;
  return launch_pdl(attn_decode_kernel<HD, REP, 8, 2>, grid, dim3(kAThreads), smem, s, a, c.err);
}

template <int HD>
cudaError_t launch_attn_hd(const AttnArgs& a, const DevCtx& c, int rep, dim3 grid, cudaStream_t s) {
  switch (rep) {
    case 1: return launch_attn_k<HD, 1>(a, c, grid, s);
    case 2: return launch_attn_k<HD, 2>(a, c, grid, s);
    case 4: return launch_attn_k<HD, 4>(a, c, grid, s);
    case 8: return launch_attn_k<HD, 8>(a, c, grid, s);
    case 16:
      if constexpr (HD <= 64) return launch_attn_k<HD, 16>(a, c, grid, s);
      break;
  }
  return cudaErrorInvalidValue;
}

int attn_splits(int range, int hd) { return (range + attn_tile_len(hd) - 1) / attn_tile_len(hd); }

int attn_split_positions(int range, int units, int sm_count) {
  const int full = attn_split_len(0);
  const int64_t target = 2LL * sm_count;   // CTAs: two resident per SM
  if ((int64_t)((range + full - 1) / full) * units < target) {
    // few sequences: shorter splits (whole 32-position chunks, >= 64) so the grid fills the GPU
    int spl = (int)(((int64_t)range * units + target - 1) / target);
    spl = (spl + kAChunk - 1) / kAChunk * kAChunk;
    return spl < 2 * kAChunk ? 2 * kAChunk : (spl > full ? full : spl);
  }
  // many: the fewest chunks per warp that keep the grid within ~4 waves
  const int chunks = (range + full - 1) / full;
  int cpw = 1;
  while (cpw < chunks && (int64_t)((chunks + cpw - 1) / cpw) * units > 4 * target) ++cpw;
  return cpw * full;
}

cudaError_t launch_attention(const DevCtx& c, const AttnArgs& a, cudaStream_t s) {
  if (a.nkv <= 0 || a.nh % a.nkv || a.S <= 0 || a.rot > a.hd || a.rot % 2) return cudaErrorInvalidValue;
  if (a.head_split < 1 || (a.nh / a.nkv) % a.head_split || (a.head_split > 1 && a.spl == 0)) return cudaErrorInvalidValue;
  const int rep = a.nh / a.nkv / a.head_split;   // query heads per CTA
  if ((size_t)a.S * rep > 8192) return cudaErrorInvalidValue;   // merge weights: <= 32 KB of shared memory
  if (a.batch < 1 || (a.batch > 1 && (a.bs_out % 32 || (a.oq && !a.od)))) return cudaErrorInvalidValue;
  // spl == 0: the single-sequence tile kernel (splits of attn_splits(range, hd) positions);
  // otherwise the streaming kernel with spl positions per split
  if (a.spl < 0 || a.spl % kAChunk || (a.spl == 0 && a.batch != 1)) return cudaErrorInvalidValue;
  const dim3 grid((unsigned)a.S, (unsigned)(a.nkv * a.head_split), (unsigned)a.batch);
  switch (a.hd) {
    case 32: return launch_attn_hd<32>(a, c, rep, grid, s);
    case 64: return launch_attn_hd<64>(a, c, rep, grid, s);
    case 128: return launch_attn_hd<128>(a, c, rep, grid, s);
    case 256: return launch_attn_hd<256>(a, c, rep, grid, s);
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_lmhead(const DevCtx& c, const LmHeadArgs& a, cudaStream_t s) {
  if (a.H % 8 || a.H > kLMaxChunks * 256) return cudaErrorInvalidValue;
  const int nch = (a.H / 8 + 31) / 32;
  const size_t smem = (size_t)a.H * sizeof(float);
  const dim3 grid((unsigned)min(2 * c.sm_count, (a.V + kLWarps - 1) / kLWarps)), block(kLWarps * 32);
  if (nch <= 4) return launch_pdl(lmhead_kernel<4>, grid, block, smem, s, a);
  if (nch <= 8) return launch_pdl(lmhead_kernel<8>, grid, block, smem, s, a);
  if (nch <= 12) return launch_pdl(lmhead_kernel<12>, grid, block, smem, s, a);
  return launch_pdl(lmhead_kernel<16>, grid, block, smem, s, a);
}

int argmax_from_key(unsigned long long key) { return (int)(0xffffffffu - (uint32_t)(key & 0xffffffffull)); }

cudaError_t launch_gemv_f32(const DevCtx& c, const float* w, int rows, int cols, const float* x, const float* bias,
                            float* y, int accumulate, cudaStream_t s) {
  const int warps_per = 8;
  gemv_f32_kernel<<<(rows + warps_per - 1) / warps_per, warps_per * 32, 0, s>>>(w, rows, cols, x, bias, y,
                                                                                accumulate);
  return cudaGetLastError();
}

cudaError_t launch_embed(const DevCtx& c, StepState* st, const void* table, int table_q, int H, int vocab, float* h,
                         int* token_log, cudaStream_t s, const float* norm_w, float eps, int8_t* xq, float* xd) {
  if (H % 32) return cudaErrorInvalidValue;
  const size_t smem = (size_t)H * sizeof(float);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(embed_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  return launch_pdl(embed_kernel, dim3(1), dim3(1024), smem, s, st, table, table_q, H, vocab, h, token_log, c.err,
                    norm_w, eps, xq, xd);
}

cudaError_t launch_resid_norm_q8(const DevCtx& c, const PendingCombine& pc, float* h, int H, const float* norm_w,
                                 float eps, int8_t* xq, float* xd, uint32_t* cnt, cudaStream_t s) {
  if (H % 32) return cudaErrorInvalidValue;
  const size_t smem = (size_t)H * sizeof(float);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(resid_norm_q8_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  return launch_pdl(resid_norm_q8_kernel, dim3((unsigned)((H + kResidRows - 1) / kResidRows)), dim3(kResidRows), smem, s,
                    pc, h, H, norm_w, eps, xq, xd, cnt, c.err);
}

cudaError_t launch_gemv(const DevCtx& c, const GemvArgs& a, cudaStream_t s) {
  switch (a.qtype) {
    case Q_MXFP4:
    case Q_Q4_K:
    case Q_Q6_K:
      return launch_block_gemv(c, a.qtype, (const uint8_t*)a.w, a.rows, a.cols, a.x, a.bias, a.y, a.accumulate, s);
    case Q_F16: {
      LmHeadArgs l;
      l.w = (const uint16_t*)a.w; l.x = a.x; l.bias = a.bias; l.logits = a.y; l.V = a.rows; l.H = a.cols;
      l.accumulate = a.accumulate;
      return launch_lmhead(c, l, s);
    }
    case Q_F32:
      return launch_gemv_f32(c, (const float*)a.w, a.rows, a.cols, a.x, a.bias, a.y, a.accumulate, s);
    case Q_Q8_0: {
      if (a.accumulate) return cudaErrorInvalidValue;
      Q8GemvArgs q;
      q.w = (const uint8_t*)a.w; q.rows = a.rows; q.cols = a.cols; q.x = a.x; q.bias = a.bias; q.y = a.y;
      return launch_q8_gemv(c, q, s);
    }
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_ep_send(const DevCtx& c, const PendingCombine& pc, int H, const EpSend& e, cudaStream_t s) {
  (void)c;
  if (e.n < 1 || e.n > kMaxEp || e.rank < 0 || e.rank >= e.n || !e.seq || !e.cnt) return cudaErrorInvalidValue;
  return launch_pdl(ep_send_kernel, dim3((unsigned)((H + 255) / 256)), dim3(256), 0, s, pc, H, e);
}

__global__ void q6k_pad_kernel(const uint16_t* __restrict__ src, int64_t n_sb, uint16_t* __restrict__ dst) {
  constexpr int kIn = 105, kOut = kQ6PadBytes / 2;   // 16-bit words per superblock
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n_sb * kOut; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t sb = i / kOut;
    const int w = (int)(i - sb * kOut);
    dst[i] = w < kIn ? src[sb * kIn + w] : (uint16_t)0;
  }
}

cudaError_t launch_q6k_pad(const uint8_t* src, int64_t n_sb, uint8_t* dst, cudaStream_t s) {
  if (n_sb <= 0) return cudaSuccess;
  if (reinterpret_cast<uintptr_t>(src) % 2 || reinterpret_cast<uintptr_t>(dst) % 16) return cudaErrorInvalidValue;
  q6k_pad_kernel<<<1184, 256, 0, s>>>(reinterpret_cast<const uint16_t*>(src), n_sb, reinterpret_cast<uint16_t*>(dst));
  return cudaGetLastError();
}

}  // namespace ms
