// kernels_ssm.cu — Gated DeltaNet decode step and the shared expert's elementwise parts (sm_100a).
//
// Reference semantics (moe-stream-core/src):
//   DeltaNet decode ... model/deltanet.rs:204-543 (conv1d + SiLU, repeat-interleave of q/k heads,
//                       L2 norms, S <- e^alpha S, delta = beta (v - S^T k), S += k delta^T,
//                       o = S^T q, per-head RMSNorm x weight x silu(z))
//   shared expert ..... model/layer.rs:2250-2293 (silu(g) * u, sigmoid(x . gate_inp) scaling)
//
// The projections are plain GEMVs (kernels_dense.cu / kernels_moe.cu).  dn_conv_kernel runs one
// thread per channel; dn_delta_kernel runs one CTA per value head with the head's
// [head_k_dim x head_v_dim] f32 state held column-wise in registers (thread j: column j, one half
// of the rows), so the state is read and written once per token.
#include "common.cuh"
#include "kernels.h"

namespace ms {
namespace {

constexpr int kDnMaxRows = 64;   // state rows per thread: head_k_dim <= 128 (two threads per column)

__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + expf(-x)); }

// depthwise causal conv over [state (k-1 values), x] per channel, state shift, SiLU
__global__ void dn_conv_kernel(const float* __restrict__ mixed, const float* __restrict__ w, float* conv_state,
                               int conv_dim, int ks, float* __restrict__ conv_out) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= conv_dim) return;
  float* st = conv_state + (size_t)c * (ks - 1);
  const float* wc = w + (size_t)c * ks;
  const float xin = mixed[c];
  float sum = 0.0f;
  for (int j = 0; j < ks - 1; ++j) sum = __fadd_rn(sum, __fmul_rn(st[j], wc[j]));   // deltanet.rs:351-355
  sum = __fadd_rn(sum, __fmul_rn(xin, wc[ks - 1]));
  for (int j = 0; j + 1 < ks - 1; ++j) st[j] = st[j + 1];
  if (ks > 1) st[ks - 2] = xin;
  conv_out[c] = silu_f(sum);
}

__device__ __forceinline__ float block_sum_2w(float v, float* red, int nw) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  v = warp_sum(v);
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.f;
  for (int w = 0; w < nw; ++w) t += red[w];
  __syncthreads();
  return t;
}

// one CTA per value head, 2 * hvd threads: thread (j, half) owns state column j, rows
// [half * hkd/2, (half + 1) * hkd/2)
__global__ void __launch_bounds__(256) dn_delta_kernel(DeltaNetStep a) {
  __shared__ float qs[128], ksh[128], red[8], part[2][128];
  const int h = blockIdx.x, hkd = a.hkd, hvd = a.hvd;
  const int j = threadIdx.x % hvd, half = threadIdx.x / hvd, rows = hkd / 2, r0 = half * rows;
  const int nw = (2 * hvd) / 32;
  const int g = h / (a.nv / a.nk), q_total = a.nk * hkd;
  // q, k of this head's key group (repeat-interleave, deltanet.rs:379-390) and their L2 norms
  float qv = 0.f, kv = 0.f;
  if (threadIdx.x < hkd) {
    qv = a.conv_out[(size_t)g * hkd + threadIdx.x];
    kv = a.conv_out[(size_t)q_total + g * hkd + threadIdx.x];
  }
  const float qn = fmaxf(sqrtf(block_sum_2w(qv * qv, red, nw)), a.eps);
  const float kn = fmaxf(sqrtf(block_sum_2w(kv * kv, red, nw)), a.eps);
  if (threadIdx.x < hkd) {
    qs[threadIdx.x] = qv / qn * a.scale;
    ksh[threadIdx.x] = kv / kn;
  }
  // gates (deltanet.rs:298-310)
  const float ab = a.ba[a.nv + h] + a.dt_bias[h];
  const float decay = expf(a.ssm_a[h] * logf(1.0f + expf(ab)));
  const float beta = 1.0f / (1.0f + expf(-a.ba[h]));
  __syncthreads();
  // decayed state column (registers), its read with k
  float* S = a.state + (size_t)h * hkd * hvd;
  float s[kDnMaxRows];
  float acc = 0.f;
#pragma unroll
  for (int i = 0; i < kDnMaxRows; ++i) {
    if (i < rows) {
      s[i] = S[(size_t)(r0 + i) * hvd + j] * decay;
      acc = fmaf(ksh[r0 + i], s[i], acc);
    }
  }
  part[half][j] = acc;
  __syncthreads();
  const float kvm = part[0][j] + part[1][j];
  const float delta = (a.conv_out[(size_t)2 * q_total + h * hvd + j] - kvm) * beta;
  __syncthreads();
  // write: S += k delta^T; query: o = S^T q
  acc = 0.f;
#pragma unroll
  for (int i = 0; i < kDnMaxRows; ++i) {
    if (i < rows) {
      s[i] = fmaf(ksh[r0 + i], delta, s[i]);
      S[(size_t)(r0 + i) * hvd + j] = s[i];
      acc = fmaf(qs[r0 + i], s[i], acc);
    }
  }
  part[half][j] = acc;
  __syncthreads();
  const float o = part[0][j] + part[1][j];
  // per-head RMSNorm x weight, x silu(z) (deltanet.rs:495-522)
  const float sq = block_sum_2w(half == 0 ? o * o : 0.f, red, nw);
  const float rms = sqrtf(sq / (float)hvd + a.eps);
  if (half == 0) {
    const float z = a.z[(size_t)h * hvd + j];
    a.out[(size_t)h * hvd + j] = (o / rms * a.norm[j]) * silu_f(z);
  }
}

__global__ void silu_mul_kernel(const float* __restrict__ g, const float* __restrict__ u, float* __restrict__ o, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) o[i] = silu_f(g[i]) * u[i];
}

// y += sigmoid(x . gate_inp) * v (every CTA recomputes the gate dot, deterministic)
__global__ void gated_accum_kernel(const float* __restrict__ x, const float* __restrict__ gate_inp,
                                   const float* __restrict__ v, float* __restrict__ y, int n, int assign) {
  __shared__ float red[8];
  float sig = 1.0f;
  if (gate_inp) {
    float d = 0.f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) d = fmaf(x[i], gate_inp[i], d);
    d = block_sum_2w(d, red, blockDim.x / 32);
    sig = 1.0f / (1.0f + expf(-d));
  }
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    y[i] = assign ? v[i] * sig : y[i] + v[i] * sig;
}

}  // namespace

cudaError_t launch_deltanet_core(const DevCtx& c, const DeltaNetStep& a, int conv_dim, int ks, const float* mixed,
                                 const float* conv_w, float* conv_state, cudaStream_t s) {
  (void)c;
  if (a.hvd != 128 || a.hkd % 2 || a.hkd > 2 * kDnMaxRows || a.hkd > 128 || a.nv % a.nk || ks < 1)
    return cudaErrorInvalidValue;
  dn_conv_kernel<<<(conv_dim + 255) / 256, 256, 0, s>>>(mixed, conv_w, conv_state, conv_dim, ks, a.conv_out);
  dn_delta_kernel<<<a.nv, 2 * a.hvd, 0, s>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_silu_mul(const float* g, const float* u, float* o, int n, cudaStream_t s) {
  silu_mul_kernel<<<(n + 255) / 256, 256, 0, s>>>(g, u, o, n);
  return cudaGetLastError();
}

cudaError_t launch_gated_accum(const float* x, const float* gate_inp, const float* v, float* y, int n, cudaStream_t s,
                               int assign) {
  gated_accum_kernel<<<(n + 255) / 256, 256, 0, s>>>(x, gate_inp, v, y, n, assign);
  return cudaGetLastError();
}

}  // namespace ms
