// kernels_exact.cu — decode-step kernels whose f32 results do not depend on summation order.
//
// Every dot product and sum is accumulated in double (f32 x f32 and MXFP4 x f32 products are exact
// in double) and rounded to f32 once; exp is the double exp rounded to f32.  The result of each
// reference op is then its exact value correctly rounded, so these kernels and the CPU oracle (which
// evaluates the reference ops the same way) agree bit for bit, and with them every downstream
// discrete decision: the Q8_0 codes of the next projection's activation, the routed experts and the
// greedy token.
//
//   exact_attn_kernel     decode attention (ops/attention.rs:178-280) for one token per sequence:
//                         a thread-block cluster per (kv head, sequence) splits the positions; the
//                         softmax needs the global max before any exp, so the CTAs exchange their
//                         maxima, then their f64 denominator sums, then their f64 P*V partials
//                         through distributed shared memory (three cluster barriers).  With 8
//                         queries per kv head the dots run on the f64 tensor cores.
//   exact_tc_kernel<0/1>  expert gate/up and down (model/layer.rs:1797-1847) over the packed MXFP4
//                         tiles on tcgen05: x (or the activation) as exact base-8 digit terms, unit
//                         block scales, f32 digit folds and f64 scaling in the epilogue; the last
//                         CTA of an item writes the activation terms (gate/up) or the slot's output
//                         row (down), which the residual kernel combines in ascending expert id.
//   exact_kq_*_kernel     K-quant experts (Q4_K / Q6_K), dequantized in the reference's f32 op
//                         order and dotted in double.
//   exact_argmax_refine   the greedy token: f64 re-scoring of the ids near the approximate maximum.
#include <cooperative_groups.h>
#include <cuda_fp16.h>

#include "common.cuh"
#include "kernels.h"
#include "umma.cuh"

namespace cg = cooperative_groups;

namespace ms {
namespace {

// ============================ attention ============================
constexpr int kXThreads = 256;
constexpr int kXWarps = kXThreads / 32;

// Reduce-scatter of 32 per-lane partials v[0..32) over a warp: afterwards lane L holds the sum
// over all lanes of v[L] (in v[0]).  Five halving rounds; double values.
__device__ __forceinline__ double warp_reduce_scatter32(double (&v)[32], int lane) {
#pragma unroll
  for (int o = 16, n = 32; o >= 1; o >>= 1, n >>= 1) {
    const bool up = (lane & o) != 0;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      if (i < n / 2) {
        const double send = up ? v[i] : v[i + n / 2];
        const double keep = up ? v[i + n / 2] : v[i];
        v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
      }
    }
  }
  return v[0];
}

// D += A B on the f64 tensor cores (m8n8k4): lane (g, t) = (lane >> 2, lane & 3) holds A[g][t],
// B[t][g] and D[g][2t], D[g][2t + 1]
__device__ __forceinline__ void dmma_884(double& d0, double& d1, double a, double b) {
  asm volatile("mma.sync.aligned.m8n8k4.row.col.f64.f64.f64.f64 {%0,%1}, {%2}, {%3}, {%0,%1};\n"
               : "+d"(d0), "+d"(d1)
               : "d"(a), "d"(b));
}

template <int HD, int REP>
__global__ void __launch_bounds__(kXThreads) exact_attn_kernel(AttnArgs a, uint32_t* err, int max_per_cta) {
  constexpr int DPL = HD / 32;
  constexpr int G = 32 / REP;              // positions per group (REP <= 32)
  extern __shared__ __align__(16) uint8_t xsm[];
  cg::cluster_group cl = cg::this_cluster();
  const int C = (int)cl.num_blocks(), rank = (int)cl.block_rank();
  float* qs = reinterpret_cast<float*>(xsm);                 // [REP][HD] normed, rotated queries
  float* kn = qs + REP * HD;                                  // [HD] new key
  float* vn = kn + HD;                                        // [HD] new value
  float* sc = vn + HD;                                        // [REP][max_per_cta] scores -> exp
  double* cl_max = reinterpret_cast<double*>(sc + (size_t)REP * max_per_cta);   // [C][REP] (as double)
  double* cl_sum = cl_max + 16 * REP;                          // [C][REP]
  double* wred = cl_sum + 16 * REP;                            // [kXWarps][REP][HD] warp partials
  double* cl_o = wred + (size_t)kXWarps * REP * HD;           // [C][slice] (slice owners)
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = blockIdx.y, b = blockIdx.z;
  const float* qkv = a.qkv + (size_t)b * a.bs_qkv;
  float* kc = a.kc + (size_t)b * a.bs_kv;
  float* vc = a.vc + (size_t)b * a.bs_kv;
  const int Dq = a.nh * HD, Dkv = a.nkv * HD;

  // the position comes from the step's first kernel (at least two launches back), so it and the
  // cached K/V rows of earlier positions may be read before waiting for the projections: this CTA's
  // rows are prefetched into L2 while the previous kernel runs
  const int pos = *a.pos;
  const int lo = a.window > 0 ? max(0, pos - a.window + 1) : 0;
  const int range = pos - lo + 1;
  const int per = (range + C - 1) / C;
  const int p0 = lo + rank * per, p1 = min(pos + 1, p0 + per);   // this CTA's positions [p0, p1)
  auto slot_of = [&](int p) { return a.window > 0 ? p % a.cap : p; };
  if (threadIdx.x < 2 && p1 - 1 > p0) {
    float* base = threadIdx.x == 0 ? kc : vc;
    const int s0 = slot_of(p0), s1 = slot_of(p1 - 2);   // rows before pos (pos itself is new)
    if (s1 >= s0) {
      bulk_prefetch_l2(base + ((size_t)g * a.cap + s0) * HD, (uint32_t)(s1 - s0 + 1) * HD * 4u);
    } else {   // the ring wraps
      bulk_prefetch_l2(base + ((size_t)g * a.cap + s0) * HD, (uint32_t)(a.cap - s0) * HD * 4u);
      bulk_prefetch_l2(base + (size_t)g * a.cap * HD, (uint32_t)(s1 + 1) * HD * 4u);
    }
  }
  pdl_wait_prior();
  pdl_launch_dependents();
  if (per > max_per_cta) {
    if (threadIdx.x == 0) atomicOr(err, EF_BAD_SHAPE);
  }
  // ---- queries, new key / value: QK-norm then RoPE at pos (layer.rs:643-664) ----
  for (int i = threadIdx.x; i < REP * HD; i += kXThreads) qs[i] = qkv[(size_t)(g * REP) * HD + i];
  for (int i = threadIdx.x; i < HD; i += kXThreads) {
    kn[i] = qkv[Dq + (size_t)g * HD + i];
    vn[i] = qkv[Dq + Dkv + (size_t)g * HD + i];
  }
  __syncthreads();
  const int half = a.rot / 2;
  const float* cs = a.cos_t + (size_t)pos * half;
  const float* sn = a.sin_t + (size_t)pos * half;
  for (int h = warp; h <= REP; h += kXWarps) {   // h == REP: the key
    float* v = h < REP ? qs + h * HD : kn;
    const float* nw = h < REP ? a.q_norm : a.k_norm;
    if (nw) {
      const float inv = rms_inv_cr_warp(v, HD, a.eps, lane);
      __syncwarp();
      for (int i = lane; i < HD; i += 32) v[i] = __fmul_rn(__fmul_rn(v[i], inv), nw[i]);
      __syncwarp();
    }
    for (int i = lane; i < half; i += 32) {
      const float x1 = v[i], x2 = v[i + half];
      v[i] = __fsub_rn(__fmul_rn(x1, cs[i]), __fmul_rn(x2, sn[i]));
      v[i + half] = __fadd_rn(__fmul_rn(x2, cs[i]), __fmul_rn(x1, sn[i]));
    }
    __syncwarp();
  }
  __syncthreads();
  // ---- scores: s = round(q . k) * scale (f64 dot) ----
  const int n_my = max(0, p1 - p0);
  if constexpr (REP == 8) {
    // f64 tensor cores: per 8 positions, A = K rows (8 x HD), B = the 8 queries; the k order is
    // permuted so lane (g, t) holds dims t*KQ .. t*KQ + KQ - 1 of position g and of query g
    constexpr int KQ = HD / 4;
    const int g8 = lane >> 2, t4 = lane & 3;
    double qf[KQ];
#pragma unroll
    for (int kk = 0; kk < KQ; ++kk) qf[kk] = (double)qs[g8 * HD + t4 * KQ + kk];
    auto load_k = [&](int pb, float (&kr)[KQ]) {
      const int p = p0 + pb + g8;
      if (pb + g8 < n_my) {
        const float* krow = (p == pos ? kn : kc + ((size_t)g * a.cap + slot_of(p)) * HD) + t4 * KQ;
#pragma unroll
        for (int kk = 0; kk < KQ; kk += 4) {
          const float4 v4 = *reinterpret_cast<const float4*>(krow + kk);
          kr[kk] = v4.x; kr[kk + 1] = v4.y; kr[kk + 2] = v4.z; kr[kk + 3] = v4.w;
        }
      } else {
#pragma unroll
        for (int kk = 0; kk < KQ; ++kk) kr[kk] = 0.f;
      }
    };
    float kcur[KQ];
    if (warp * 8 < n_my) load_k(warp * 8, kcur);
    for (int pb = warp * 8; pb < n_my; pb += kXWarps * 8) {
      float knext[KQ];
      if (pb + kXWarps * 8 < n_my) load_k(pb + kXWarps * 8, knext);
      double c0 = 0.0, c1 = 0.0, e0 = 0.0, e1 = 0.0;   // two accumulation chains
#pragma unroll
      for (int kk = 0; kk < KQ; kk += 2) {
        dmma_884(c0, c1, (double)kcur[kk], qf[kk]);
        dmma_884(e0, e1, (double)kcur[kk + 1], qf[kk + 1]);
      }
      if (pb + g8 < n_my) {   // D[position g][queries 2t, 2t + 1]
        sc[(size_t)(2 * t4) * max_per_cta + pb + g8] = __fmul_rn((float)(c0 + e0), a.scale);
        sc[(size_t)(2 * t4 + 1) * max_per_cta + pb + g8] = __fmul_rn((float)(c1 + e1), a.scale);
      }
#pragma unroll
      for (int kk = 0; kk < KQ; ++kk) kcur[kk] = knext[kk];
    }
  } else {
    double qd[REP][DPL];
#pragma unroll
    for (int h = 0; h < REP; ++h)
#pragma unroll
      for (int d = 0; d < DPL; ++d) qd[h][d] = (double)qs[h * HD + lane + 32 * d];
    // the group's K rows (G positions, DPL values per lane); the next group's are loaded before this
    // group's dots so the L2 reads overlap
    auto load_k = [&](int gb, float (&kr)[G][DPL]) {
#pragma unroll
      for (int u = 0; u < G; ++u) {
        const int p = p0 + gb + u;
        if (gb + u < n_my) {
          const float* krow = p == pos ? kn : kc + ((size_t)g * a.cap + slot_of(p)) * HD;
#pragma unroll
          for (int d = 0; d < DPL; ++d) kr[u][d] = krow[lane + 32 * d];
        } else {
#pragma unroll
          for (int d = 0; d < DPL; ++d) kr[u][d] = 0.f;
        }
      }
    };
    float kcur[G][DPL];
    if (warp * G < n_my) load_k(warp * G, kcur);
    for (int gb = warp * G; gb < n_my; gb += kXWarps * G) {
      float knext[G][DPL];
      if (gb + kXWarps * G < n_my) load_k(gb + kXWarps * G, knext);
      double v[32];
#pragma unroll
      for (int u = 0; u < G; ++u) {
#pragma unroll
        for (int h = 0; h < REP; ++h) {
          double t = 0.0;
#pragma unroll
          for (int d = 0; d < DPL; ++d) t = fma(qd[h][d], (double)kcur[u][d], t);
          v[u * REP + h] = t;
        }
      }
#pragma unroll
      for (int u = 0; u < G; ++u)
#pragma unroll
        for (int d = 0; d < DPL; ++d) kcur[u][d] = knext[u][d];
      const double dot = warp_reduce_scatter32(v, lane);   // lane = u * REP + h
      const int u = lane / REP, h = lane % REP;
      if (gb + u < n_my) {
        const float s = __fmul_rn((float)dot, a.scale);
        sc[(size_t)h * max_per_cta + gb + u] = s;
      }
    }
  }
  __syncthreads();
  // local maxima per head, then every CTA's maxima to every CTA of the cluster
  for (int h = warp; h < REP; h += kXWarps) {
    float m = -INFINITY;
    for (int j = lane; j < n_my; j += 32) m = fmaxf(m, sc[(size_t)h * max_per_cta + j]);
    m = warp_max(m);
    if (lane < C) {
      double* dst = cl.map_shared_rank(cl_max, lane);
      dst[rank * REP + h] = (double)m;
    }
  }
  cl.sync();
  // ---- exp(s - m') with the sink-aware max, f64 partial denominators ----
  __shared__ float s_mp[32];
  __shared__ float s_den[32];
  if (threadIdx.x < REP) {
    const int h = threadIdx.x;
    float m = -INFINITY;
    for (int r = 0; r < C; ++r) m = fmaxf(m, (float)cl_max[r * REP + h]);
    if (a.sinks) {
      const float sk = a.sinks[g * REP + h];
      m = __fmul_rn(__fadd_rn(__fadd_rn(m, sk), fabsf(__fsub_rn(m, sk))), 0.5f);
    }
    s_mp[h] = m;
  }
  __syncthreads();
  for (int h = warp; h < REP; h += kXWarps) {
    const float m = s_mp[h];
    double t = 0.0;
    for (int j = lane; j < n_my; j += 32) {
      const float e = expcr(__fsub_rn(sc[(size_t)h * max_per_cta + j], m));
      sc[(size_t)h * max_per_cta + j] = e;
      t += (double)e;
    }
    t = warp_sum_d(t);
    if (lane < C) {
      double* dst = cl.map_shared_rank(cl_sum, lane);
      dst[rank * REP + h] = t;
    }
  }
  cl.sync();
  if (threadIdx.x < REP) {
    const int h = threadIdx.x;
    double t = 0.0;
    for (int r = 0; r < C; ++r) t += cl_sum[r * REP + h];
    float den = (float)t;
    if (a.sinks) den = __fadd_rn(den, expcr(__fsub_rn(a.sinks[g * REP + h], s_mp[h])));
    s_den[h] = den;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < REP * n_my; i += kXThreads) {   // weights e / den (f32)
    const int h = i / n_my, j = i % n_my;
    sc[(size_t)h * max_per_cta + j] = __fdiv_rn(sc[(size_t)h * max_per_cta + j], s_den[h]);
  }
  __syncthreads();
  // ---- P*V: weights p = e / den (f32), f64 accumulation over positions ----
  if constexpr (REP == 8) {
    // f64 tensor cores: per 4 positions, A = V^T (8 dims x 4 positions), B = P^T (4 positions x 8
    // queries); lane (g, t) takes position t and dims g*MT .. g*MT + MT - 1 (m-tile mt = dim g*MT + mt)
    constexpr int MT = HD / 8;
    const int g8 = lane >> 2, t4 = lane & 3;
    double o[MT][2];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) o[mt][0] = o[mt][1] = 0.0;
    for (int j0 = warp * 8; j0 < n_my; j0 += kXWarps * 8) {   // two 4-position steps per round
      float vr[2][MT];
      double pw[2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int j = j0 + 4 * u + t4;
        if (j < n_my) {
          const int p = p0 + j;
          const float* vrow = (p == pos ? vn : vc + ((size_t)g * a.cap + slot_of(p)) * HD) + g8 * MT;
#pragma unroll
          for (int mt = 0; mt < MT; mt += 4) {
            const float4 v4 = *reinterpret_cast<const float4*>(vrow + mt);
            vr[u][mt] = v4.x; vr[u][mt + 1] = v4.y; vr[u][mt + 2] = v4.z; vr[u][mt + 3] = v4.w;
          }
          pw[u] = (double)sc[(size_t)g8 * max_per_cta + j];
        } else {
#pragma unroll
          for (int mt = 0; mt < MT; ++mt) vr[u][mt] = 0.f;
          pw[u] = 0.0;
        }
      }
#pragma unroll
      for (int u = 0; u < 2; ++u)
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) dmma_884(o[mt][0], o[mt][1], (double)vr[u][mt], pw[u]);
    }
    // D[dim g*MT + mt][queries 2t, 2t + 1]
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      wred[((size_t)warp * REP + 2 * t4) * HD + g8 * MT + mt] = o[mt][0];
      wred[((size_t)warp * REP + 2 * t4 + 1) * HD + g8 * MT + mt] = o[mt][1];
    }
  } else {
    double o[REP][DPL];
#pragma unroll
    for (int h = 0; h < REP; ++h)
#pragma unroll
      for (int d = 0; d < DPL; ++d) o[h][d] = 0.0;
    constexpr int U = DPL <= 2 ? 8 : 4;   // V rows per warp per round, loaded together
    for (int j0 = warp * U; j0 < n_my; j0 += kXWarps * U) {
      float vr[U][DPL];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int p = p0 + j0 + u;
        if (j0 + u < n_my) {
          const float* vrow = p == pos ? vn : vc + ((size_t)g * a.cap + slot_of(p)) * HD;
#pragma unroll
          for (int d = 0; d < DPL; ++d) vr[u][d] = vrow[lane + 32 * d];
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        if (j0 + u < n_my) {
#pragma unroll
          for (int h = 0; h < REP; ++h) {
            const float pw = sc[(size_t)h * max_per_cta + j0 + u];
#pragma unroll
            for (int d = 0; d < DPL; ++d) o[h][d] = fma((double)pw, (double)vr[u][d], o[h][d]);
          }
        }
      }
    }
#pragma unroll
    for (int h = 0; h < REP; ++h)
#pragma unroll
      for (int d = 0; d < DPL; ++d) wred[((size_t)warp * REP + h) * HD + lane + 32 * d] = o[h][d];
  }
  __syncthreads();
  // every CTA's partial P*V to the rank that owns its slice of the outputs (32-element multiples)
  const int NS = min(C, REP * HD / 32), SL = REP * HD / NS;
  for (int i = threadIdx.x; i < REP * HD; i += kXThreads) {
    double t = 0.0;
#pragma unroll
    for (int w = 0; w < kXWarps; ++w) t += wred[(size_t)w * REP * HD + i];
    double* dst = cl.map_shared_rank(cl_o, i / SL);
    dst[(size_t)rank * SL + i % SL] = t;
  }
  // the new key / value row goes to the cache once this CTA has read everything it needs
  if (p0 <= pos && pos < p1) {
    for (int i = threadIdx.x; i < HD; i += kXThreads) {
      kc[((size_t)g * a.cap + slot_of(pos)) * HD + i] = kn[i];
      vc[((size_t)g * a.cap + slot_of(pos)) * HD + i] = vn[i];
    }
  }
  cl.sync();
  if (rank >= NS) return;
  // ---- the outputs of this rank's slice (rounded once) and their Q8_0 blocks for the O projection ----
  const size_t o0 = (size_t)b * a.bs_out + (size_t)g * REP * HD + (size_t)rank * SL;
  for (int j = threadIdx.x; j < SL; j += kXThreads) {
    double t = 0.0;
    for (int r = 0; r < C; ++r) t += cl_o[(size_t)r * SL + j];
    const float v = (float)t;
    qs[j] = v;
    a.out[o0 + j] = v;
  }
  __syncthreads();
  if (a.oq) {
    for (int blk = threadIdx.x; blk < SL / 32; blk += kXThreads) {
      float v[32];
#pragma unroll
      for (int k = 0; k < 32; ++k) v[k] = qs[32 * blk + k];
      quantize_q8_block(v, a.oq + o0 + 32 * blk, &a.od[(o0 + 32 * blk) / 32]);
    }
  }
}

template <int HD, int REP>
cudaError_t launch_exact_attn_t(const AttnArgs& a, const DevCtx& c, int C, int max_per, cudaStream_t s) {
  const size_t smem = (size_t)(REP * HD + 2 * HD) * 4 + (size_t)REP * max_per * 4 + 2 * 16 * REP * 8 +
                      (size_t)kXWarps * REP * HD * 8 + (size_t)C * (REP * HD / std::min(C, REP * HD / 32)) * 8 + 64;
  if (smem > 227 * 1024) return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(exact_attn_kernel<HD, REP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem);
  if (e == cudaSuccess && C > 8)   // clusters of up to 16 CTAs (beyond the portable 8)
    e = cudaFuncSetAttribute(exact_attn_kernel<HD, REP>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)C, (unsigned)a.nkv, (unsigned)a.batch);
  cfg.blockDim = dim3(kXThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = (unsigned)C;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, exact_attn_kernel<HD, REP>, a, c.err, max_per);
}

template <int HD>
cudaError_t launch_exact_attn_hd(const AttnArgs& a, const DevCtx& c, int rep, int C, int max_per, cudaStream_t s) {
  switch (rep) {
    case 1: return launch_exact_attn_t<HD, 1>(a, c, C, max_per, s);
    case 2: return launch_exact_attn_t<HD, 2>(a, c, C, max_per, s);
    case 4: return launch_exact_attn_t<HD, 4>(a, c, C, max_per, s);
    case 8: return launch_exact_attn_t<HD, 8>(a, c, C, max_per, s);
    case 16:
      if constexpr (HD <= 64) return launch_exact_attn_t<HD, 16>(a, c, C, max_per, s);
      break;
  }
  return cudaErrorInvalidValue;
}

// ============================ experts (MXFP4 tiles on tcgen05) ============================
// The expert rows are the packed MXFP4 tiles of the tensor-core path (128 rows; slabs of 16 chunk
// columns, codes then 512-byte scale groups).  A unit is one K-word of one (slot, tile) item: 4
// chunk columns (the last unit of a row may hold 2) and their scale group.  Per K = 64 pair of
// chunks the tensor core computes, with every block scale set to 1,
// D[row][parity * 24 + t] = sum over the 32 elements of the pair's chunk `parity` of
// e2m1(w) * term_t(x) -- multiples of 1/2 below 2^10, exact in f32.  The epilogue folds 5 base-8
// digits at a time in f32 (still exact: below 2^23 halves), applies 2^(E_w - 127 - F + 15 g) and
// accumulates in f64.  A CTA runs two independent pipelines, each with its own warps: a producer
// (1-D bulk copies into 4 stages), an MMA issuer (one elected thread; two accumulators of 96 TMEM
// columns, so a unit's MMAs overlap the previous unit's drain) and 8 epilogue warps (two per TMEM
// lane quadrant, one chunk pair each).  The units of all (slot, tile) items are cut into equal
// contiguous ranges, one per pipeline; the last run of an item reduces the item's partials.
constexpr int kUC = 4;                          // chunk columns per unit (one K-word, one scale group)
constexpr int kUStA = kUC * 2048;               // A codes
constexpr int kUStS = 512;                      // A scale group
constexpr int kUStB = kUC * kExactBlock;        // B terms
constexpr int kUStF = 16;                       // the 4 chunks' scale exponents of B (x / activation)
constexpr int kUStage = kUStA + kUStS + kUStB + kUStF;
constexpr int kUPipes = 2;                      // independent copy / MMA / epilogue pipelines per CTA
constexpr int kUStages = 4;                     // stages per pipeline
constexpr int kUAcc = 2;                        // accumulators per pipeline (double-buffered)
constexpr int kUAccCols = (kUC / 2) * kExactCols;   // one accumulator: 2 pairs x 48 columns
constexpr int kUEpiWarps = 8;                   // epilogue warps per pipeline (two per TMEM lane quadrant)
constexpr int kUThreads = 32 * (2 * kUPipes + kUPipes * kUEpiWarps);
constexpr int kUTmemCols = 512;
constexpr uint32_t kUSfCol = kUPipes * kUAcc * kUAccCols;   // unit block scales: pipeline p's A at +8p, B at +8p+4
constexpr int kUMaxSlots = 16;
static_assert(kUSfCol + 8 * kUPipes <= kUTmemCols, "tensor memory budget");
static_assert(kUStage % 16 == 0, "bulk-copy alignment");

__host__ __device__ __forceinline__ int64_t ex_slab_off(int s) { return (int64_t)s * (16 * 2048 + 4 * 512); }

__device__ __forceinline__ float act_exact(float g, float u, int oai) {
  if (oai) {   // ops/activation.rs:25-45 (clamp 7, alpha 1.702)
    const float gc = fminf(g, 7.0f);
    const float uc = fminf(fmaxf(u, -7.0f), 7.0f);
    const float sg = __fdiv_rn(1.0f, __fadd_rn(expcr(-__fadd_rn(__fmul_rn(gc, 1.702f), 0.0f)), 1.0f));
    return __fmul_rn(__fmul_rn(gc, sg), __fadd_rn(uc, 1.0f));
  }
  // ops/activation.rs:13-15: silu(g) * u with silu(x) = x / (1 + exp(-x))
  return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expcr(-g))), u);
}

// position of a unit: slot list entry i, tile mt, unit u (chunk columns 8u ..); advanced in order
struct UnitCursor {
  int u, mt, i;
  __device__ void init(int q, int nu, int tiles) {
    u = q % nu;
    const int r = q / nu;
    mt = r % tiles;
    i = r / tiles;
  }
  __device__ void next(int nu, int tiles) {
    if (++u == nu) {
      u = 0;
      if (++mt == tiles) {
        mt = 0;
        ++i;
      }
    }
  }
};

// phase 0: gate/up (rows < 64 of a tile gate, >= 64 up; the last run of an item writes the
// activation terms); phase 1: down (the last run writes the slot's output rows).  Each CTA runs
// kUPipes independent pipelines, each over its own contiguous range of units (a "virtual CTA":
// the grid's unit sequence is cut into kUPipes x gridDim.x equal ranges).  A pipeline's
// consecutive units of one item form a run: its epilogue warps accumulate the run in registers
// and write one f64 partial per row at the run's first unit; the item's reducer finds the runs
// again from the range boundaries.  xres (gate/up): x's B terms stay in shared memory for the
// whole kernel, shared by the pipelines.
template <int PHASE>
__global__ void __launch_bounds__(kUThreads, 1) exact_tc_kernel(const __grid_constant__ ExactMoeArgs a, int xres) {
  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ __align__(8) uint64_t full[kUPipes][kUStages], empty[kUPipes][kUStages], acc_full[kUPipes][kUAcc],
      acc_empty[kUPipes][kUAcc], xb_full;
  __shared__ uint32_t tmem_base;
  __shared__ int s_slot[kUMaxSlots], s_exp[kUMaxSlots], s_n, s_abort, s_last[kUPipes];
  __shared__ double red[kUPipes][2][2][128];
  __shared__ __align__(16) uint8_t sf_one[512];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kc = PHASE ? a.I / 32 : a.H / 32;
  const int tiles = PHASE ? a.down_tiles : a.gu_tiles;
  const int nu = (kc + kUC - 1) / kUC;
  const int rows_out = PHASE ? a.h_pad : 2 * a.I;       // partial rows per (slot, run start)
  const uint8_t* wbase = PHASE ? a.down : a.gu;
  const int64_t tile_bytes = PHASE ? a.down_tile_bytes : a.gu_tile_bytes;
  double* part = PHASE ? a.dp : a.gp;                  // [K][nu][rows_out]
  uint32_t* err = a.err;

  // barriers and the unit scales do not depend on the previous kernel
  if (threadIdx.x == 0) {
    for (int p = 0; p < kUPipes; ++p) {
      for (int s = 0; s < kUStages; ++s) {
        mbar_init(&full[p][s], 1);
        mbar_init(&empty[p][s], 1 + kUEpiWarps);   // the MMA commit and every epilogue warp (stage bytes read)
      }
      for (int q = 0; q < kUAcc; ++q) {
        mbar_init(&acc_full[p][q], 1);
        mbar_init(&acc_empty[p][q], kUEpiWarps);
      }
    }
    mbar_init(&xb_full, 1);
    fence_mbar_init();
  }
  for (int i = threadIdx.x; i < 512; i += kUThreads) sf_one[i] = 127;   // ue8m0 1.0
  umma::fence_proxy_async_smem();
  pdl_wait_prior();
  pdl_launch_dependents();
  // all of tensor memory, taken only after the previous kernel has finished (so a kernel of the
  // same kind launched ahead of time never waits on a CTA that is waiting on it)
  if (warp == 2) {
    umma::tmem_alloc(&tmem_base, kUTmemCols);
    umma::tmem_relinquish();
  }
  if (threadIdx.x == 0) {
    int n = 0;
    for (int k = 0; k < a.K && n < kUMaxSlots; ++k) {
      const int e = a.idx[k] - a.expert_base;
      if (e < 0 || e >= a.n_local) continue;   // another rank's expert (or out of range: the combine skips it)
      s_slot[n] = k;
      s_exp[n] = e;
      ++n;
    }
    s_n = n;
    s_abort = 0;
  }
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t tb = tmem_base;
  const int U = s_n * tiles * nu, G = (int)gridDim.x * kUPipes;
  auto range_lo = [&](int b) { return (int)((int64_t)b * U / G); };
  const uint8_t* bt = PHASE ? a.abt : a.xbt;
  const int64_t bt_stride = PHASE ? (int64_t)kc * kExactBlock : 0;
  const int* fe_src = PHASE ? a.afe : a.xfe;
  const int64_t fe_stride = PHASE ? (int64_t)((kc + 7) & ~7) : 0;
  uint8_t* xb_s = smem + (size_t)kUPipes * kUStages * kUStage;   // xres: [kc][kExactBlock] terms, then exponents
  const int* xfe_s = reinterpret_cast<const int*>(xb_s + (size_t)kc * kExactBlock);
  const bool any = U > 0;

  if (warp < kUPipes) {
    // ---------------- producer of pipeline `warp` ----------------
    const int pp = warp;
    const int q0 = range_lo(kUPipes * blockIdx.x + pp), q1 = range_lo(kUPipes * blockIdx.x + pp + 1);
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      if (xres && pp == 0 && any) {
        const uint32_t fb = (uint32_t)((kc + 7) & ~7) * 4u;
        mbar_expect_tx(&xb_full, (uint32_t)kc * kExactBlock + fb);
        bulk_g2s(xb_s, bt, (uint32_t)kc * kExactBlock, &xb_full);
        bulk_g2s(xb_s + (size_t)kc * kExactBlock, fe_src, fb, &xb_full);
      }
      UnitCursor C;
      C.init(q0, nu, tiles);
      int j = 0;
      for (int q = q0; q < q1; ++q, ++j, C.next(nu, tiles)) {
        if (*reinterpret_cast<volatile int*>(&s_abort)) break;
        const int c0 = C.u * kUC, n = min(kUC, kc - c0);
        const int s = j % kUStages, use = j / kUStages;
        if (use > 0 && !mbar_wait(&empty[pp][s], (uint32_t)((use - 1) & 1), err, EF_TIMEOUT_EMPTY)) {
          s_abort = 1;
          break;
        }
        const int k = s_slot[C.i], e = s_exp[C.i];
        const int slab = c0 >> 4, sl0 = slab * 16, nch = min(16, kc - sl0);
        const uint8_t* sb = wbase + ((int64_t)e * tiles + C.mt) * tile_bytes + ex_slab_off(slab);
        uint8_t* st = smem + (size_t)(pp * kUStages + s) * kUStage;
        const uint32_t sbytes = 512u;   // the unit's scale group
        const uint32_t bytes = (uint32_t)n * 2048u + sbytes + (xres ? 0u : (uint32_t)n * kExactBlock + 16u);
        mbar_expect_tx(&full[pp][s], bytes);
        bulk_g2s_stream(st, sb + (int64_t)(c0 - sl0) * 2048, (uint32_t)n * 2048u, &full[pp][s], pol);
        bulk_g2s_stream(st + kUStA, sb + (int64_t)nch * 2048 + ((c0 - sl0) >> 2) * 512, sbytes, &full[pp][s], pol);
        if (!xres) {
          bulk_g2s(st + kUStA + kUStS, bt + (int64_t)k * bt_stride + (int64_t)c0 * kExactBlock,
                   (uint32_t)n * kExactBlock, &full[pp][s]);
          bulk_g2s(st + kUStA + kUStS + kUStB, fe_src + (int64_t)k * fe_stride + c0, 16u, &full[pp][s]);
        }
      }
      // no copy may still be landing in shared memory when the CTA exits
      for (int q = max(0, j - kUStages); q < j; ++q)
        mbar_wait(&full[pp][q % kUStages], (uint32_t)((q / kUStages) & 1), err, EF_TIMEOUT_FULL);
      if (xres && pp == 0 && any) mbar_wait(&xb_full, 0u, err, EF_TIMEOUT_FULL);
    }
  } else if (warp < 2 * kUPipes) {
    // ---------------- MMA issuer of pipeline `warp - kUPipes` ----------------
    const int pp = warp - kUPipes;
    const int q0 = range_lo(kUPipes * blockIdx.x + pp), q1 = range_lo(kUPipes * blockIdx.x + pp + 1);
    if (lane == 0) {
      const uint32_t sfa = tb + kUSfCol + 8u * pp, sfb = sfa + 4u;
      umma::cp_sf_group(sfa, sf_one);
      umma::cp_sf_group(sfb, sf_one);
      constexpr uint32_t idesc = umma::idesc_mxf4(128, kExactCols, 0, 0);
      if (xres && q1 > q0 && !mbar_wait(&xb_full, 0u, err, EF_TIMEOUT_FULL)) s_abort = 1;
      UnitCursor C;
      C.init(q0, nu, tiles);
      int j = 0;
      for (int q = q0; q < q1; ++q, ++j, C.next(nu, tiles)) {
        if (*reinterpret_cast<volatile int*>(&s_abort)) break;
        const int n = min(kUC, kc - C.u * kUC);
        const int s = j % kUStages, acc = j % kUAcc;
        if (!mbar_wait(&full[pp][s], (uint32_t)((j / kUStages) & 1), err, EF_TIMEOUT_FULL)) {
          s_abort = 1;
          break;
        }
        if (j >= kUAcc &&
            !mbar_wait(&acc_empty[pp][acc], (uint32_t)(((j / kUAcc) - 1) & 1), err, EF_TIMEOUT_EMPTY)) {
          s_abort = 1;
          break;
        }
        umma::fence_after_sync();
        const uint8_t* st = smem + (size_t)(pp * kUStages + s) * kUStage;
        const uint8_t* bsrc = xres ? xb_s + (size_t)C.u * kUC * kExactBlock : st + kUStA + kUStS;
        const uint64_t ad0 = umma::smem_desc(st, 2048, 128), bd0 = umma::smem_desc(bsrc, kExactBlock, 128);
        for (int p = 0; p < n / 2; ++p)   // descriptor start addresses in 16-byte units
          umma::mma_mxf4(tb + (uint32_t)((pp * kUAcc + acc) * kUAccCols + p * kExactCols),
                         ad0 + (uint64_t)(p * 4096 / 16), bd0 + (uint64_t)(p * 2 * kExactBlock / 16), idesc, sfa, sfb,
                         false);
        umma::commit(&empty[pp][s]);
        umma::commit(&acc_full[pp][acc]);
      }
    }
  } else {
    // ---------------- epilogue of pipeline (warp - 2 kUPipes) / kUEpiWarps ----------------
    const int ew = warp - 2 * kUPipes, pp = ew / kUEpiWarps, le = ew % kUEpiWarps;
    const int quad = warp & 3, pg = le >> 2;   // TMEM lane quadrant; chunk pair pg
    const int row = 32 * quad + lane;
    const int q0 = range_lo(kUPipes * blockIdx.x + pp), q1 = range_lo(kUPipes * blockIdx.x + pp + 1);
    UnitCursor C;
    C.init(q0, nu, tiles);
    int j = 0, run = 0, run_u0 = C.u, rp = 0;
    double racc = 0.0;
    if (xres && q1 > q0) mbar_wait_sleep(&xb_full, 0u, err, EF_TIMEOUT_FULL, 64);   // the resident scale exponents
    for (int q = q0; q < q1; ++q, ++j, C.next(nu, tiles)) {
      const int s = j % kUStages, acc = j % kUAcc;
      const int n = min(kUC, kc - C.u * kUC);
      bool ok = mbar_wait_sleep(&acc_full[pp][acc], (uint32_t)((j / kUAcc) & 1), err, EF_TIMEOUT_FULL, 64);
      ok = ok && mbar_wait(&full[pp][s], (uint32_t)((j / kUStages) & 1), err, EF_TIMEOUT_FULL);
      ok = __all_sync(0xffffffffu, ok);   // the accumulator loads below are warp-collective
      umma::fence_after_sync();
      const uint8_t* st = smem + (size_t)(pp * kUStages + s) * kUStage;
      uint32_t ews[2], fes[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int jc = 2 * pg + h;   // chunk within the unit: byte jc of the row's scale word
        ews[h] = st[kUStA + 16 * (row & 31) + 4 * (row >> 5) + jc];
        fes[h] = (uint32_t)(xres ? xfe_s[C.u * kUC + jc] : reinterpret_cast<const int*>(st + kUStA + kUStS + kUStB)[jc]);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[pp][s]);
      // the warp's chunk pair: 48 accumulator columns (chunk h: its 19 digit dots at h * 24 + t)
      float v[48];
      if (2 * pg < n && ok) {
        const uint32_t ta = tb + ((uint32_t)(32 * quad) << 16) + (uint32_t)((pp * kUAcc + acc) * kUAccCols + pg * kExactCols);
        umma::ld_32x32b_x32(ta, *reinterpret_cast<float(*)[32]>(&v[0]));
        umma::ld_32x32b_x16(ta + 32, *reinterpret_cast<float(*)[16]>(&v[32]));
      } else {
#pragma unroll
        for (int i = 0; i < 48; ++i) v[i] = 0.f;
      }
      umma::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[pp][acc]);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        if (2 * pg + h < n) {
          const float* vv = &v[h * 24];
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            const int t0 = 5 * g, t1 = min(kExactDigits, t0 + 5);
            float f = vv[t1 - 1];
#pragma unroll
            for (int t = t1 - 2; t >= t0; --t) f = fmaf(f, 8.0f, vv[t]);   // exact: halves below 2^23
            const double sc = __hiloint2double((int)((ews[h] + fes[h] + 15u * g) << 20), 0);
            racc = fma((double)f, sc, racc);
          }
        }
      }
      ++run;
      const bool run_end = q + 1 == q1 || C.u + 1 == nu;   // the next unit starts another item
      if (!run_end) continue;
      // ---- the run's partial: the two pair warps of each row summed, written at the run's first unit ----
      const int k = s_slot[C.i], e = s_exp[C.i], mt = C.mt;
      red[pp][rp][pg][row] = racc;
      racc = 0.0;
      named_bar(1 + pp, 32 * kUEpiWarps);
      const int nrun = run, u_start = run_u0;
      run = 0;
      run_u0 = 0;   // a later run of this pipeline starts an item at unit 0
      const int rb = rp;
      rp ^= 1;
      if (pg != 0) continue;
      const double t = red[pp][rb][0][row] + red[pp][rb][1][row];
      double* pk = part + (size_t)k * nu * rows_out;
      pk[(size_t)u_start * rows_out + (size_t)mt * 128 + row] = t;
      named_bar(3 + pp, 128);
      if (le == 0 && lane == 0) {
        __threadfence();   // the run's partials (ordered before by the barrier), then the count
        uint32_t* cnt = a.cnt + (PHASE ? (size_t)a.K * a.gu_tiles : 0) + (size_t)k * tiles + mt;
        s_last[pp] = atomicAdd(cnt, (uint32_t)nrun) + (uint32_t)nrun == (uint32_t)nu ? 1 : 0;
        if (s_last[pp]) {
          *cnt = 0u;
          __threadfence();
        }
      }
      named_bar(3 + pp, 128);
      if (!s_last[pp]) continue;
      // ---- the item's reduction: its runs in range order (the ranges cut the unit sequence) ----
      const int A0 = (C.i * tiles + mt) * nu;   // the item's first unit
      int bnext = max(0, (int)((int64_t)A0 * G / (U > 0 ? U : 1)) - 1);
      // up to 8 run starts at a time, so their loads are in flight together
      auto next_runs = [&](int (&runs)[8]) {
        int nr = 0;
        for (; bnext < G && nr < 8; ++bnext) {
          const int lo = range_lo(bnext), hi = range_lo(bnext + 1);
          if (lo >= A0 + nu) {
            bnext = G;
            break;
          }
          if (hi > lo && hi > A0) runs[nr++] = max(lo, A0) - A0;
        }
        return nr;
      };
      const double* base = pk + (size_t)mt * 128;
      int runs[8];
      if (PHASE == 0) {
        // the tile's 64 activations: gate row r and up row 64 + r, r = 32 * quad + lane for quads 0, 1
        if (quad < 2) {
          const int r = row, i = mt * 64 + r;
          double gs = 0.0, us = 0.0;
          for (int nr = next_runs(runs); nr > 0; nr = next_runs(runs)) {
            double gl[8], ul[8];
#pragma unroll
            for (int q2 = 0; q2 < 8; ++q2) {
              gl[q2] = q2 < nr ? __ldcg(base + (size_t)runs[q2] * rows_out + r) : 0.0;
              ul[q2] = q2 < nr ? __ldcg(base + (size_t)runs[q2] * rows_out + 64 + r) : 0.0;
            }
#pragma unroll
            for (int q2 = 0; q2 < 8; ++q2)
              if (q2 < nr) {
                gs += gl[q2];
                us += ul[q2];
              }
          }
          float gv = (float)gs, uv = (float)us;
          if (a.gate_b) gv = __fadd_rn(gv, a.gate_b[(size_t)e * a.I + i]);
          if (a.up_b) uv = __fadd_rn(uv, a.up_b[(size_t)e * a.I + i]);
          const int ch = 2 * mt + quad;   // the down projection's chunk column of these 32 activations
          const int kcd = a.I / 32;
          exact_bterm_warp(act_exact(gv, uv, a.oai_swiglu), lane, a.abt + ((int64_t)k * kcd + ch) * kExactBlock,
                           ch & 1, a.afe + (int64_t)k * ((kcd + 7) & ~7) + ch);
        }
      } else {
        const int r = mt * 128 + row;
        if (r < a.H) {
          double t2 = 0.0;
          for (int nr = next_runs(runs); nr > 0; nr = next_runs(runs)) {
            double vl[8];
#pragma unroll
            for (int q2 = 0; q2 < 8; ++q2) vl[q2] = q2 < nr ? __ldcg(base + (size_t)runs[q2] * rows_out + row) : 0.0;
#pragma unroll
            for (int q2 = 0; q2 < 8; ++q2)
              if (q2 < nr) t2 += vl[q2];
          }
          float y = (float)t2;
          if (a.down_b) y = __fadd_rn(y, a.down_b[(size_t)e * a.H + r]);
          a.y[(size_t)k * a.H + r] = y;
        }
      }
    }
  }
  umma::fence_before_sync();
  __syncthreads();
  if (warp == 2) umma::tmem_dealloc(tb, kUTmemCols);
}

// ============================ experts (K-quant native blocks) ============================
// A lane takes 64 elements of a row: group q (0..3) of a 256-element superblock -- Q4_K: the low
// and high nibbles of 32 code bytes (sub-blocks 2q, 2q+1); Q6_K: element runs l and l + 64 (q even)
// or l + 32 and l + 96 (q odd) of one half.  Element values are dequantized with the reference's
// f32 op order (dequant.rs:218-262, 335-378), then dotted with x in double.  x sits in shared memory
// as doubles with one padding double after every 64 elements (a superblock spans 260), so the 32
// lanes of a warp -- 32 groups at once -- read from different banks.
__device__ __forceinline__ double kq_group_dot(int fmt, const uint8_t* blk, int q, const double* xs) {
  double a0 = 0.0, a1 = 0.0;
  if (fmt == Q_Q4_K) {
    const float d = h2f_bits((uint16_t)(blk[0] | (blk[1] << 8)));
    const float dmin = h2f_bits((uint16_t)(blk[2] | (blk[3] << 8)));
    const uint8_t* sc = blk + 4;
    const int is0 = 2 * q, is1 = 2 * q + 1;
    uint32_t s0, m0, s1, m1;
    if (is0 < 4) { s0 = sc[is0] & 63; m0 = sc[is0 + 4] & 63; }
    else { s0 = (sc[is0 + 4] & 0xf) | ((sc[is0 - 4] >> 6) << 4); m0 = (sc[is0 + 4] >> 4) | ((sc[is0] >> 6) << 4); }
    if (is1 < 4) { s1 = sc[is1] & 63; m1 = sc[is1 + 4] & 63; }
    else { s1 = (sc[is1 + 4] & 0xf) | ((sc[is1 - 4] >> 6) << 4); m1 = (sc[is1 + 4] >> 4) | ((sc[is1] >> 6) << 4); }
    const float d1 = __fmul_rn(d, (float)s0), mf1 = __fmul_rn(dmin, (float)m0);
    const float d2 = __fmul_rn(d, (float)s1), mf2 = __fmul_rn(dmin, (float)m1);
    const uint4* qp = reinterpret_cast<const uint4*>(blk + 16 + 32 * q);
    const uint4 w0 = qp[0], w1 = qp[1];
    const uint32_t wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
    const double* xl = xs + 65 * q;   // 64-element group q (one padding double per group)
#pragma unroll
    for (int t = 0; t < 8; ++t) {
#pragma unroll
      for (int bi = 0; bi < 4; ++bi) {
        const uint32_t byte = (wv[t] >> (8 * bi)) & 0xFFu;
        const int l = 4 * t + bi;
        const float lo = __fsub_rn(__fmul_rn(d1, (float)(byte & 0xF)), mf1);
        const float hi = __fsub_rn(__fmul_rn(d2, (float)(byte >> 4)), mf2);
        a0 = fma((double)lo, xl[l], a0);
        a1 = fma((double)hi, xl[32 + l], a1);
      }
    }
  } else {   // Q6_K (224-byte padded superblocks)
    const float d = h2f_bits((uint16_t)(blk[208] | (blk[209] << 8)));
    const int8_t* scv = reinterpret_cast<const int8_t*>(blk + 192);
    const int half = q >> 1, sub = q & 1;
    const uint8_t* ql = blk + half * 64 + 32 * sub;
    const uint8_t* qh = blk + 128 + half * 32;
    const double* xl = xs + half * 130 + 32 * sub;   // padded: groups 2 half and 2 half + 1
#pragma unroll 8
    for (int l = 0; l < 32; ++l) {
      const uint32_t lb = ql[l], hb = qh[l];
      const int qa = (int)((lb & 0xF) | (((hb >> (2 * sub)) & 3) << 4)) - 32;
      const int qb = (int)((lb >> 4) | (((hb >> (4 + 2 * sub)) & 3) << 4)) - 32;
      const int isa = half * 8 + l / 16 + 2 * sub, isb = isa + 4;
      const float va = __fmul_rn(__fmul_rn(d, (float)scv[isa]), (float)qa);
      const float vb = __fmul_rn(__fmul_rn(d, (float)scv[isb]), (float)qb);
      a0 = fma((double)va, xl[l], a0);
      a1 = fma((double)vb, xl[65 + l], a1);
    }
  }
  return a0 + a1;
}

constexpr int kKThreads = 256;

// rows of one expert matrix (native K-quant blocks), G = cols / 64 lanes per row, 32 / G rows per
// warp (one row and several groups per lane when cols > 2048); y[row] = round(dot) (+ bias)
__device__ __forceinline__ void kq_rows(int fmt, const uint8_t* w, int64_t rb, int rows, int cols, const double* xs,
                                        int row0, const float* bias, float* y, double* red) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = cols / 64, R = G >= 32 ? 1 : 32 / G;
  const int sb_bytes = fmt == Q_Q4_K ? 144 : kQ6PadBytes;
  const int sub = lane / (G >= 32 ? 32 : G), grp0 = lane % (G >= 32 ? 32 : G);
  const int row = row0 + warp * R + sub;
  double part = 0.0;
  if (sub < R && row < rows) {
    const uint8_t* wr = w + (int64_t)row * rb;
    for (int gi = grp0; gi < G; gi += 32) part += kq_group_dot(fmt, wr + (gi >> 2) * sb_bytes, gi & 3, xs + 260 * (gi >> 2));
  }
  red[threadIdx.x] = part;
  __syncwarp();
  if (lane < R) {
    const int r2 = row0 + warp * R + lane;
    if (r2 < rows) {
      const int gw = G >= 32 ? 32 : G;
      double t = 0.0;
      for (int i = 0; i < gw; ++i) t += red[warp * 32 + lane * gw + i];
      float v = (float)t;
      if (bias) v = __fadd_rn(v, bias[r2]);
      y[r2] = v;
    }
  }
}

__global__ void __launch_bounds__(kKThreads) exact_kq_gu_kernel(ExactKqArgs a, uint32_t* err) {
  extern __shared__ double xk[];   // [H + H/64]: element e at e + e/64
  __shared__ double red[kKThreads];
  const int which = blockIdx.z & 1, b = blockIdx.z >> 1;   // 0 gate, 1 up; token b
  const int k = b * a.K + blockIdx.y;                       // (token, slot)
  pdl_wait_prior();
  pdl_launch_dependents();
  const int e = a.idx[k] - a.expert_base;
  if (e < 0 || e >= a.n_local) return;
  for (int i = threadIdx.x; i < a.H; i += kKThreads) xk[i + (i >> 6)] = (double)a.x[(size_t)b * a.H + i];
  __syncthreads();
  const int G = a.H / 64, R = G >= 32 ? 1 : 32 / G;
  const int64_t rb = (int64_t)(a.H / 256) * (a.gate_fmt == Q_Q4_K ? 144 : kQ6PadBytes);
  const int we = a.wslot ? a.wslot[k] : e;   // weight slot (host-tier cache) or the expert itself
  const uint8_t* w = (which ? a.up : a.gate) + (int64_t)we * a.I * rb;
  const float* bias = which ? (a.up_b ? a.up_b + (size_t)e * a.I : nullptr) : (a.gate_b ? a.gate_b + (size_t)e * a.I : nullptr);
  kq_rows(a.gate_fmt, w, rb, a.I, a.H, xk, blockIdx.x * (kKThreads / 32) * R, bias, a.gu_out + ((size_t)k * 2 + which) * a.I,
          red);
  (void)err;
}

__global__ void __launch_bounds__(kKThreads) exact_kq_down_kernel(ExactKqArgs a, uint32_t* err) {
  extern __shared__ double ak[];   // [I + I/64] activations, element e at e + e/64
  __shared__ double red[kKThreads];
  const int k = blockIdx.z * a.K + blockIdx.y;               // (token, slot)
  pdl_wait_prior();
  pdl_launch_dependents();
  const int e = a.idx[k] - a.expert_base;
  if (e < 0 || e >= a.n_local) return;
  const float* g = a.gu_out + (size_t)k * 2 * a.I;
  for (int i = threadIdx.x; i < a.I; i += kKThreads) ak[i + (i >> 6)] = (double)act_exact(g[i], g[a.I + i], a.oai_swiglu);
  __syncthreads();
  const int G = a.I / 64, R = G >= 32 ? 1 : 32 / G;
  const int64_t rb = (int64_t)(a.I / 256) * (a.down_fmt == Q_Q4_K ? 144 : kQ6PadBytes);
  const uint8_t* w = a.down + (int64_t)(a.wslot ? a.wslot[k] : e) * a.H * rb;
  kq_rows(a.down_fmt, w, rb, a.H, a.I, ak, blockIdx.x * (kKThreads / 32) * R,
          a.down_b ? a.down_b + (size_t)e * a.H : nullptr, a.y + (size_t)k * a.H, red);
  (void)err;
}

template <class Kern, class Args>
cudaError_t launch_pdl_x(Kern k, dim3 grid, dim3 block, size_t smem, cudaStream_t s, const Args& a, uint32_t* err) {
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
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
  return cudaLaunchKernelEx(&cfg, k, a, err);
}

}  // namespace

// CTAs per (kv head, sequence) cluster: a power of two (the output slices divide evenly), at most
// 16, at least 16 positions per CTA, and no more than needed for about two CTAs per SM over all
// (kv head, sequence) units
int exact_attn_cluster(int range, int units, int sm_count) {
  int C = 1;
  while (C < 16 && C * 16 < range && (long)units * C < 2L * sm_count) C *= 2;
  return C;
}

cudaError_t launch_exact_attention(const DevCtx& c, const AttnArgs& a, int range, cudaStream_t s) {
  if (a.nkv <= 0 || a.nh % a.nkv || a.rot > a.hd || a.rot % 2 || a.batch < 1 || range <= 0) return cudaErrorInvalidValue;
  if (a.batch > 1 && a.bs_out % 32) return cudaErrorInvalidValue;
  const int rep = a.nh / a.nkv;
  if (32 % rep) return cudaErrorInvalidValue;
  const int C = exact_attn_cluster(range, a.nkv * a.batch, c.sm_count);
  const int max_per = (range + C - 1) / C;
  switch (a.hd) {
    case 32: return launch_exact_attn_hd<32>(a, c, rep, C, max_per, s);
    case 64: return launch_exact_attn_hd<64>(a, c, rep, C, max_per, s);
    case 128: return launch_exact_attn_hd<128>(a, c, rep, C, max_per, s);
  }
  return cudaErrorInvalidValue;
}

int exact_seg_count(int kc) { return (kc + kUC - 1) / kUC; }
int exact_term_block_bytes() { return kExactBlock; }

cudaError_t launch_exact_moe(const DevCtx& c, const ExactMoeArgs& a0, cudaStream_t s, int part) {
  ExactMoeArgs a = a0;
  if (!tc_supported(a.H, a.I) || a.K < 1 || a.K > kUMaxSlots || !a.gp || !a.dp || !a.xbt || !a.xfe || !a.abt ||
      !a.afe || !a.cnt || !a.y || a.I % 64)
    return cudaErrorInvalidValue;
  a.gu_tiles = tc_gu_tiles(a.I);
  a.down_tiles = tc_down_tiles(a.H);
  a.gu_tile_bytes = tc_tile_bytes(a.H / 32);
  a.down_tile_bytes = tc_tile_bytes(a.I / 32);
  a.err = c.err;
  if (a.n_seg_gu != exact_seg_count(a.H / 32) || a.n_seg_down != exact_seg_count(a.I / 32) ||
      a.h_pad < tc_down_tiles(a.H) * 128)
    return cudaErrorInvalidValue;
  for (int ph = 0; ph < 2; ++ph) {
    if (part >= 0 && part != ph) continue;
    auto kern = ph ? exact_tc_kernel<1> : exact_tc_kernel<0>;
    // gate/up keeps x's B terms resident in shared memory when they fit beside the stages
    const int kc = ph ? a.I / 32 : a.H / 32;
    const size_t stages = (size_t)kUPipes * kUStages * kUStage;
    const size_t xb = (size_t)kc * kExactBlock + (size_t)((kc + 7) & ~7) * 4;
    const int xres = (ph == 0 && stages + xb <= 210 * 1024) ? 1 : 0;
    const size_t smem = stages + (xres ? xb : 0);
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)c.sm_count);
    cfg.blockDim = dim3(kUThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, kern, a, xres);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

namespace {
// Greedy token of each sequence from approximate logits: every id within `band` of the approximate
// maximum (already in keys[b], from the LM head) is re-scored exactly -- f64 dot of the f16 row with
// the normed x, rounded once, + bias -- and the best exact value wins, ties to the lower id.  The
// approximate logits carry errors far below `band`, so the exact maximum is among the candidates.
// Grid (slices, sequences): each CTA scans a slice of the logits; the last CTA of a sequence
// re-scores the candidates.  scratch per sequence: [kRefMaxCand] ids, count, CTA counter (zero,
// self-resetting).
constexpr int kRefMaxCand = 64;
__device__ __forceinline__ float key_value(unsigned long long key) {
  const uint32_t b = (uint32_t)(key >> 32);
  return __uint_as_float((b & 0x80000000u) ? (b & 0x7fffffffu) : ~b);
}
__global__ void __launch_bounds__(256) exact_argmax_refine_kernel(const uint16_t* __restrict__ w,
                                                                  const float* __restrict__ xf,
                                                                  const float* __restrict__ bias, const float* logits,
                                                                  int V, int H, unsigned long long* keys, int* scratch,
                                                                  uint32_t* err) {
  __shared__ uint32_t last;
  __shared__ unsigned long long s_best;
  const int b = blockIdx.y, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int* cand = scratch + (size_t)b * (kRefMaxCand + 2);
  int* cnt = cand + kRefMaxCand;
  uint32_t* done = reinterpret_cast<uint32_t*>(cnt + 1);
  const float* lg = logits + (size_t)b * V;
  pdl_wait_prior();
  pdl_launch_dependents();
  const float mx = key_value(keys[b]);
  const float band = 1e-4f * fabsf(mx) + 1e-5f;
  const int per = (V + gridDim.x - 1) / gridDim.x, i0 = blockIdx.x * per, i1 = min(V, i0 + per);
  for (int i = i0 + threadIdx.x; i < i1; i += blockDim.x) {
    if (__ldcg(lg + i) >= mx - band) {
      const int slot = atomicAdd(cnt, 1);
      if (slot < kRefMaxCand) cand[slot] = i;
      else atomicOr(err, EF_BAD_SHAPE);
    }
  }
  __syncthreads();   // every thread's stores, then (cumulative) thread 0's fence and count
  if (threadIdx.x == 0) {
    __threadfence();
    last = (atomicAdd(done, 1u) == gridDim.x - 1) ? 1u : 0u;
    s_best = 0ull;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  const int n = min(*reinterpret_cast<volatile int*>(cnt), kRefMaxCand);
  const float* x = xf + (size_t)b * H;
  for (int c = warp; c < n; c += blockDim.x / 32) {
    const int r = __ldcg(cand + c);
    const __half* row = reinterpret_cast<const __half*>(w) + (size_t)r * H;
    double acc = 0.0;
    for (int i = lane; i < H; i += 32) acc = fma((double)__half2float(row[i]), (double)x[i], acc);
    acc = warp_sum_d(acc);
    if (lane == 0) {
      float v = (float)acc;
      if (bias) v = __fadd_rn(v, bias[r]);
      uint32_t bits = __float_as_uint(v);
      bits = (bits & 0x80000000u) ? ~bits : (bits | 0x80000000u);
      const unsigned long long key = ((unsigned long long)bits << 32) | (uint32_t)(0xffffffffu - (uint32_t)r);
      atomicMax(&s_best, key);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    if (n > 0) keys[b] = s_best;
    *cnt = 0;
    *done = 0u;
  }
}
}  // namespace

int exact_refine_scratch_ints(int B) { return B * (kRefMaxCand + 2); }

cudaError_t launch_exact_argmax_refine(const uint16_t* w, const float* xf, const float* bias, const float* logits,
                                       int V, int H, int B, unsigned long long* keys, int* scratch, const DevCtx& c,
                                       cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)std::min(c.sm_count, (V + 255) / 256), (unsigned)B);
  cfg.blockDim = dim3(256);
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, exact_argmax_refine_kernel, w, xf, bias, logits, V, H, keys, scratch, c.err);
}

bool exact_kq_supported(int gate_q, int down_q, int H, int I) {
  auto ok = [](int q) { return q == Q_Q4_K || q == Q_Q6_K_PAD; };
  return ok(gate_q) && ok(down_q) && H % 256 == 0 && I % 256 == 0;
}

cudaError_t launch_exact_kq_moe(const DevCtx& c, const ExactKqArgs& a, cudaStream_t s) {
  if (!exact_kq_supported(a.gate_fmt, a.down_fmt, a.H, a.I) || a.K < 1 || a.K > 16 || !a.gu_out || !a.y)
    return cudaErrorInvalidValue;
  auto rows_per_cta = [](int cols) { const int G = cols / 64; return (kKThreads / 32) * (G >= 32 ? 1 : 32 / G); };
  const int rg = rows_per_cta(a.H), rd = rows_per_cta(a.I);
  if (a.B < 1) return cudaErrorInvalidValue;
  cudaError_t e = launch_pdl_x(exact_kq_gu_kernel, dim3((unsigned)((a.I + rg - 1) / rg), (unsigned)a.K, 2u * a.B),
                               dim3(kKThreads), (size_t)(a.H + a.H / 64) * 8, s, a, c.err);
  if (e != cudaSuccess) return e;
  return launch_pdl_x(exact_kq_down_kernel, dim3((unsigned)((a.H + rd - 1) / rd), (unsigned)a.K, (unsigned)a.B),
                      dim3(kKThreads), (size_t)(a.I + a.I / 64) * 8, s, a, c.err);
}

}  // namespace ms
