// kernels_prefill_attn.cu — the non-expert half of a multi-token forward (prompt prefill).
//
// Reference semantics (moe-stream-core/src): Engine::forward over a [1, T] prompt
// (model/engine.rs:1869-2006): embedding rows (1877), per layer RMSNorm (ops/norm.rs:16-37), the
// Q/K/V projections of all T tokens (model/layer.rs:566-584), QK-norm (643-650), RoPE at absolute
// positions (654-664, ops/attention.rs:49-164), K/V appended to the cache (model/kv_cache.rs:37-60),
// and causal multi-query SDPA with the sliding-window mask and attention sinks
// (ops/attention.rs:178-280: causal only when seq_q > 1; SWA masks q_abs - k >= window; sinks join
// the softmax denominator as exp(s - m')).
//
// Layout: token rows are [T][dim] f32.  The cache of a layer is [kv_heads][cap][hd] f32 (a ring of
// `window` slots on sliding-window layers).  The attention kernel reads keys before the chunk from
// the cache and the chunk's own keys from the chunk buffers, so a chunk longer than the window never
// reads a ring slot that the same chunk overwrote; the cache append runs after it.
#include <cuda_fp16.h>

#include "common.cuh"
#include "kernels.h"

namespace ms {
namespace {

// ---- rows: embedding + attention-norm quantization, norm quantization, plain quantization ----

__global__ void __launch_bounds__(256) pf_embed_kernel(const int* __restrict__ tok, const void* table, int q, int H,
                                                       int vocab, float* __restrict__ h, const float* norm_w,
                                                       float eps, int8_t* xq, float* xd, uint32_t* err) {
  extern __shared__ float es[];   // [H]
  __shared__ float red[256];
  const int t = blockIdx.x;
  int id = tok[t];
  if (id < 0 || id >= vocab) {
    if (threadIdx.x == 0) atomicOr(err, EF_BAD_INDEX);
    id = 0;
  }
  float* ht = h + (size_t)t * H;
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    const float v = (q == Q_F16) ? __half2float(reinterpret_cast<const __half*>(table)[(size_t)id * H + i])
                                 : reinterpret_cast<const float*>(table)[(size_t)id * H + i];
    ht[i] = v;
    es[i] = v;
  }
  __syncthreads();
  cta_rmsnorm_q8(es, H, norm_w, eps, xq + (size_t)t * H, xd + (size_t)t * (H / 32), red);
}

__global__ void __launch_bounds__(256) pf_norm_q8_kernel(const float* __restrict__ h, int H, const float* norm_w,
                                                         float eps, int8_t* xq, float* xd) {
  extern __shared__ float es[];
  __shared__ float red[256];
  const int t = blockIdx.x;
  for (int i = threadIdx.x; i < H; i += blockDim.x) es[i] = h[(size_t)t * H + i];
  __syncthreads();
  cta_rmsnorm_q8(es, H, norm_w, eps, xq + (size_t)t * H, xd + (size_t)t * (H / 32), red);
}

// Q8_0 blocks of rows x [T][cols] (the O projection's activation), one thread per 32-element block
__global__ void pf_quant_kernel(const float* __restrict__ x, int64_t n_blocks, int8_t* xq, float* xd) {
  for (int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; b < n_blocks; b += (int64_t)gridDim.x * blockDim.x) {
    float v[32];
    const float4* x4 = reinterpret_cast<const float4*>(x + 32 * b);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float4 t = x4[k];
      v[4 * k] = t.x; v[4 * k + 1] = t.y; v[4 * k + 2] = t.z; v[4 * k + 3] = t.w;
    }
    quantize_q8_block(v, xq + 32 * b, &xd[b]);
  }
}

// ---- Q/K/V preparation: QK-RMSNorm, RoPE at absolute positions, split into head rows ----

// RMSNorm of one head vector v[0..hd) (hd <= 256) held by a warp, in the same fixed order as
// canon_sumsq (256 strided partials -- single terms here -- then the pairwise tree)
__device__ __forceinline__ void warp_head_norm(float* v, const float* w, int hd, float eps, int lane) {
  float p[8];
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    const int j = lane + 32 * m;
    p[m] = j < hd ? fmaf(v[j], v[j], 0.f) : 0.f;
  }
#pragma unroll
  for (int m = 0; m < 4; ++m) p[m] = p[m] + p[m + 4];
#pragma unroll
  for (int m = 0; m < 2; ++m) p[m] = p[m] + p[m + 2];
  float t = p[0] + p[1];
#pragma unroll
  for (int s = 16; s >= 1; s >>= 1) t = t + __shfl_down_sync(0xffffffffu, t, s);
  t = __shfl_sync(0xffffffffu, t, 0);
  const float inv = 1.0f / sqrtf(t / (float)hd + eps);
  __syncwarp();
  for (int j = lane; j < hd; j += 32) v[j] = (v[j] * inv) * w[j];
  __syncwarp();
}

// NeoX rotation of the first rot dims of v (in shared memory, by one warp), products and sums
// rounded separately
__device__ __forceinline__ void warp_rope(float* v, const float* cs, const float* sn, int rot, int lane) {
  const int half = rot / 2;
  for (int i = lane; i < half; i += 32) {
    const float x1 = v[i], x2 = v[i + half], c = cs[i], s = sn[i];
    const float r1 = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s));
    const float r2 = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s));
    v[i] = r1;
    v[i + half] = r2;
  }
  __syncwarp();
}

struct PfPrepArgs {
  const float* qkv;        // [T][nh*hd + 2*nkv*hd] projections + bias
  const float* q_norm;     // [hd] or null
  const float* k_norm;
  float eps;
  const float* cos_t;      // [max_seq][rot/2]
  const float* sin_t;
  int rot, pos0, T, nh, nkv, hd;
  float* q;                // [T][nh][hd]
  float* k;                // [T][nkv][hd]
  float* v;                // [T][nkv][hd]
};

// one CTA per token; warps loop over the token's nh + nkv rotated heads
__global__ void __launch_bounds__(256) pf_qkv_prep_kernel(PfPrepArgs a) {
  extern __shared__ float hs[];   // [8 warps][hd]
  const int t = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31, hd = a.hd;
  const int Dq = a.nh * hd, Dkv = a.nkv * hd, W = Dq + 2 * Dkv;
  const float* row = a.qkv + (size_t)t * W;
  const int half = a.rot / 2, pos = a.pos0 + t;
  const float* cs = a.cos_t + (size_t)pos * half;
  const float* sn = a.sin_t + (size_t)pos * half;
  float* v = hs + warp * hd;
  for (int hh = warp; hh < a.nh + a.nkv; hh += 8) {
    const bool is_q = hh < a.nh;
    const float* src = row + (is_q ? hh * hd : Dq + (hh - a.nh) * hd);
    for (int j = lane; j < hd; j += 32) v[j] = src[j];
    __syncwarp();
    const float* nw = is_q ? a.q_norm : a.k_norm;
    if (nw) warp_head_norm(v, nw, hd, a.eps, lane);
    warp_rope(v, cs, sn, a.rot, lane);
    float* dst = is_q ? a.q + ((size_t)t * a.nh + hh) * hd : a.k + ((size_t)t * a.nkv + (hh - a.nh)) * hd;
    for (int j = lane; j < hd; j += 32) dst[j] = v[j];
    __syncwarp();
  }
  for (int j = threadIdx.x; j < Dkv; j += blockDim.x) a.v[(size_t)t * Dkv + j] = row[Dq + Dkv + j];
}

// ---- causal multi-query attention over the cache and the chunk ----

constexpr int kPaQ = 32;     // queries per CTA (8 warps x 4)
constexpr int kPaKT = 32;    // keys per shared-memory tile

struct PfAttnArgs {
  const float* q;          // [T][nh][hd] (normed, rotated)
  const float* kn;         // [T][nkv][hd] the chunk's keys (normed, rotated)
  const float* vn;         // [T][nkv][hd]
  const float* kc;         // cache [nkv][cap][hd]: positions < pos0
  const float* vc;
  int cap, window, pos0, T, nh, nkv;
  const float* sinks;      // [nh] or null
  float scale;
  float* out;              // [T][nh][hd]
};

template <int HD>
__global__ void __launch_bounds__(256) pf_attn_kernel(PfAttnArgs a) {
  extern __shared__ float sm[];
  float* qs = sm;                              // [kPaQ][HD]
  float* ks = qs + kPaQ * HD;                  // [kPaKT][HD + 1]
  float* vs = ks + kPaKT * (HD + 1);           // [kPaKT][HD]
  constexpr int DPL = HD / 32;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.y, g = h / (a.nh / a.nkv);
  const int t0 = blockIdx.x * kPaQ, t1 = min(a.T, t0 + kPaQ);
  for (int i = threadIdx.x; i < kPaQ * HD; i += blockDim.x) {
    const int qi = i / HD, d = i % HD;
    qs[i] = t0 + qi < a.T ? a.q[((size_t)(t0 + qi) * a.nh + h) * HD + d] : 0.f;
  }
  const int hi = a.pos0 + t1 - 1;
  const int lo = a.window > 0 ? max(0, a.pos0 + t0 - a.window + 1) : 0;
  float m[4], l[4], o[4][DPL];
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    m[r] = -INFINITY;
    l[r] = 0.f;
#pragma unroll
    for (int i = 0; i < DPL; ++i) o[r][i] = 0.f;
  }
  for (int kb = lo; kb <= hi; kb += kPaKT) {
    __syncthreads();   // previous tile consumed (and qs written, on the first pass)
    for (int i = threadIdx.x; i < kPaKT * HD; i += blockDim.x) {
      const int j = i / HD, d = i % HD, p = kb + j;
      float kv = 0.f, vv = 0.f;
      if (p <= hi) {
        if (p >= a.pos0) {
          const size_t o2 = ((size_t)(p - a.pos0) * a.nkv + g) * HD + d;
          kv = a.kn[o2];
          vv = a.vn[o2];
        } else {
          const int slot = a.window > 0 ? p % a.cap : p;
          const size_t o2 = ((size_t)g * a.cap + slot) * HD + d;
          kv = a.kc[o2];
          vv = a.vc[o2];
        }
      }
      ks[j * (HD + 1) + d] = kv;
      vs[j * HD + d] = vv;
    }
    __syncthreads();
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int qi = warp * 4 + r, t = t0 + qi;
      if (t >= a.T) break;
      const int qpos = a.pos0 + t, p = kb + lane;
      const bool valid = p <= qpos && p >= lo && (a.window <= 0 || qpos - p < a.window);
      float s = -INFINITY;
      if (valid) {
        const float* qv = qs + qi * HD;
        const float* kr = ks + lane * (HD + 1);
        float dot = 0.f;
#pragma unroll 16
        for (int d = 0; d < HD; ++d) dot = fmaf(qv[d], kr[d], dot);
        s = dot * a.scale;
      }
      const float tm = warp_max(s);
      if (tm == -INFINITY) continue;
      const float mn = fmaxf(m[r], tm);
      const float alpha = m[r] == -INFINITY ? 0.f : expf(m[r] - mn);
      const float pj = valid ? expf(s - mn) : 0.f;
      l[r] = l[r] * alpha + warp_sum(pj);
#pragma unroll
      for (int i = 0; i < DPL; ++i) o[r][i] *= alpha;
      for (int jj = 0; jj < kPaKT; ++jj) {
        const float pb = __shfl_sync(0xffffffffu, pj, jj);
        if (pb != 0.f) {
#pragma unroll
          for (int i = 0; i < DPL; ++i) o[r][i] = fmaf(pb, vs[jj * HD + lane + 32 * i], o[r][i]);
        }
      }
      m[r] = mn;
    }
  }
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int t = t0 + warp * 4 + r;
    if (t >= a.T) break;
    float mm = m[r], ll = l[r], sc = 1.f;
    if (a.sinks) {   // the sink joins the denominator only (ops/attention.rs:247-273)
      const float sk = a.sinks[h];
      const float mf = fmaxf(mm, sk);
      sc = expf(mm - mf);
      ll = ll * sc + expf(sk - mf);
    }
    const float inv = sc / ll;
    float* dst = a.out + ((size_t)t * a.nh + h) * HD;
#pragma unroll
    for (int i = 0; i < DPL; ++i) dst[lane + 32 * i] = o[r][i] * inv;
  }
}

// chunk K/V rows -> the cache (after the chunk's attention); on a ring only the last `window`
// positions of the chunk are kept
__global__ void pf_kv_append_kernel(const float* __restrict__ kn, const float* __restrict__ vn, float* kc, float* vc,
                                    int cap, int window, int pos0, int T, int nkv, int hd) {
  const int t = blockIdx.x, p = pos0 + t;
  if (window > 0 && t < T - window) return;
  const int slot = window > 0 ? p % cap : p;
  for (int i = threadIdx.x; i < nkv * hd; i += blockDim.x) {
    const int g = i / hd, d = i % hd;
    const size_t dst = ((size_t)g * cap + slot) * hd + d;
    kc[dst] = kn[((size_t)t * nkv + g) * hd + d];
    vc[dst] = vn[((size_t)t * nkv + g) * hd + d];
  }
}

// h[t] += y[t] (expert-parallel prefill: the all-reduced MoE output of every token)
__global__ void pf_add_kernel(float* __restrict__ h, const float* __restrict__ y, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    h[i] += y[i];
}

}  // namespace

cudaError_t launch_pf_embed(const DevCtx& c, const int* tok, int T, const void* table, int q, int H, int vocab,
                            float* h, const float* norm_w, float eps, int8_t* xq, float* xd, cudaStream_t s) {
  if (T <= 0 || H % 32 || !norm_w) return cudaErrorInvalidValue;
  const size_t smem = (size_t)H * 4;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(pf_embed_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  pf_embed_kernel<<<T, 256, smem, s>>>(tok, table, q, H, vocab, h, norm_w, eps, xq, xd, c.err);
  return cudaGetLastError();
}

cudaError_t launch_pf_norm_q8(const float* h, int T, int H, const float* norm_w, float eps, int8_t* xq, float* xd,
                              cudaStream_t s) {
  if (T <= 0 || H % 32 || !norm_w) return cudaErrorInvalidValue;
  const size_t smem = (size_t)H * 4;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(pf_norm_q8_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  pf_norm_q8_kernel<<<T, 256, smem, s>>>(h, H, norm_w, eps, xq, xd);
  return cudaGetLastError();
}

cudaError_t launch_pf_quant(const float* x, int64_t n, int8_t* xq, float* xd, cudaStream_t s) {
  if (n % 32) return cudaErrorInvalidValue;
  const int64_t nb = n / 32;
  pf_quant_kernel<<<(unsigned)std::min<int64_t>((nb + 255) / 256, 4096), 256, 0, s>>>(x, nb, xq, xd);
  return cudaGetLastError();
}

cudaError_t launch_pf_attention(const DevCtx& c, const PfAttnLaunch& L, cudaStream_t s) {
  (void)c;
  if (L.T <= 0 || L.nkv <= 0 || L.nh % L.nkv || L.hd > 256 || L.hd % 32 || L.rot > L.hd || L.rot % 2 ||
      (L.window > 0 && L.cap != L.window))
    return cudaErrorInvalidValue;
  PfPrepArgs p;
  p.qkv = L.qkv; p.q_norm = L.q_norm; p.k_norm = L.k_norm; p.eps = L.eps; p.cos_t = L.cos_t; p.sin_t = L.sin_t;
  p.rot = L.rot; p.pos0 = L.pos0; p.T = L.T; p.nh = L.nh; p.nkv = L.nkv; p.hd = L.hd; p.q = L.q; p.k = L.kn;
  p.v = L.vn;
  pf_qkv_prep_kernel<<<L.T, 256, (size_t)8 * L.hd * 4, s>>>(p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  PfAttnArgs a;
  a.q = L.q; a.kn = L.kn; a.vn = L.vn; a.kc = L.kc; a.vc = L.vc; a.cap = L.cap; a.window = L.window;
  a.pos0 = L.pos0; a.T = L.T; a.nh = L.nh; a.nkv = L.nkv; a.sinks = L.sinks; a.scale = L.scale; a.out = L.out;
  const dim3 grid((unsigned)((L.T + kPaQ - 1) / kPaQ), (unsigned)L.nh);
  auto go = [&](auto kern, int hd) {
    const size_t smem = ((size_t)kPaQ * hd + (size_t)kPaKT * (hd + 1) + (size_t)kPaKT * hd) * 4;
    cudaError_t r = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (r != cudaSuccess) return r;
    kern<<<grid, 256, smem, s>>>(a);
    return cudaGetLastError();
  };
  switch (L.hd) {
    case 32: e = go(pf_attn_kernel<32>, 32); break;
    case 64: e = go(pf_attn_kernel<64>, 64); break;
    case 128: e = go(pf_attn_kernel<128>, 128); break;
    case 256: e = go(pf_attn_kernel<256>, 256); break;
    default: return cudaErrorInvalidValue;
  }
  if (e != cudaSuccess) return e;
  pf_kv_append_kernel<<<L.T, 256, 0, s>>>(L.kn, L.vn, L.kc, L.vc, L.cap, L.window, L.pos0, L.T, L.nkv, L.hd);
  return cudaGetLastError();
}

cudaError_t launch_pf_add(float* h, const float* y, int64_t n, cudaStream_t s) {
  pf_add_kernel<<<(unsigned)std::min<int64_t>((n + 255) / 256, 8192), 256, 0, s>>>(h, y, n);
  return cudaGetLastError();
}

}  // namespace ms
