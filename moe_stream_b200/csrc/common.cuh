// common.cuh — device helpers shared by the moe-stream B200 kernels (sm_100a only).
//
// Weight streaming uses 1-D bulk async copies (cp.async.bulk, the TMA engine's
// untiled mode) into shared-memory stages guarded by mbarriers.  Every wait is
// bounded: on expiry the kernel records an error bit in the context's device
// error word and returns, so the context stays usable and the host reports
// MS_ERR_TIMEOUT instead of hanging the GPU.
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

#include "kernels.h"

#ifndef __CUDA_ARCH__
#define MS_HOST_ONLY 1
#endif

namespace ms {

// wait budget: ~2^22 try_wait probes (each may suspend up to the hardware hint) ≈ 1-2 s
constexpr uint32_t kWaitLimit = 1u << 22;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait.  Returns false (and sets `bit` in *err) when the budget runs out.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t* err, uint32_t bit) {
  for (uint32_t i = 0; i < kWaitLimit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  if (err) atomicOr(err, bit);
  return false;
}

// Bounded wait that sleeps between polls, for warps that would otherwise take issue slots from
// the producer / MMA threads of their SM sub-partition.
__device__ __forceinline__ bool mbar_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t* err, uint32_t bit,
                                                uint32_t ns) {
  for (uint32_t i = 0; i < kWaitLimit / 16; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    __nanosleep(ns);
  }
  if (err) atomicOr(err, bit);
  return false;
}

// 1-D bulk copy global -> this CTA's shared memory; bytes % 16 == 0, both addresses 16-aligned.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Same with an L2 evict-first hint: streamed weights should not displace activations / KV.
__device__ __forceinline__ void bulk_g2s_stream(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                                uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// prefetch [p, p + bytes) of global memory into L2 (bytes a multiple of 16, p 16-byte aligned)
__device__ __forceinline__ void bulk_prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// named barrier among `nthreads` threads (consumer warps only)
__device__ __forceinline__ void named_bar(uint32_t id, uint32_t nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ---- small math helpers ----
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float h2f_bits(uint16_t h) { return __half2float(__ushort_as_half(h)); }

// unaligned little-endian u32 / u16 read from shared memory via aligned loads + funnel shift
__device__ __forceinline__ uint32_t lds_u32_unaligned(const uint8_t* base, uint32_t off) {
  const uint32_t a = off & ~3u, sh = (off & 3u) * 8u;
  const uint32_t lo = *reinterpret_cast<const uint32_t*>(base + a);
  const uint32_t hi = *reinterpret_cast<const uint32_t*>(base + a + 4);
  return __funnelshift_r(lo, hi, sh);
}

// e2m1x2 (one byte: low nibble = first element) -> f16x2 (low half = low nibble); exact.
__device__ __forceinline__ uint32_t e2m1x2_to_f16x2(uint32_t byte) {
  uint32_t out;
  asm("{\n .reg .b8 b;\n cvt.u8.u32 b, %1;\n cvt.rn.f16x2.e2m1x2 %0, b;\n}\n" : "=r"(out) : "r"(byte));
  return out;
}

// the four bytes of w (byte i = e2m1 pair i) -> four f16x2 registers
__device__ __forceinline__ void e2m1x8_to_f16x2x4(uint32_t w, uint32_t& o0, uint32_t& o1, uint32_t& o2,
                                                  uint32_t& o3) {
  asm("{\n .reg .b8 b0, b1, b2, b3;\n mov.b32 {b0, b1, b2, b3}, %4;\n"
      " cvt.rn.f16x2.e2m1x2 %0, b0;\n cvt.rn.f16x2.e2m1x2 %1, b1;\n"
      " cvt.rn.f16x2.e2m1x2 %2, b2;\n cvt.rn.f16x2.e2m1x2 %3, b3;\n}\n"
      : "=r"(o0), "=r"(o1), "=r"(o2), "=r"(o3)
      : "r"(w));
}

__device__ __forceinline__ uint32_t pack_half2(__half lo, __half hi) {
  return (uint32_t)__half_as_ushort(lo) | ((uint32_t)__half_as_ushort(hi) << 16);
}

// D += A(16x16, f16, row) * B(16x8, f16, col); f32 accumulators.
__device__ __forceinline__ void mma_f16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// ---- pending MoE combine (see PendingCombine in kernels.h) ----
struct CombineOrder {
  int n;
  int slot[16];
  float w[16];
  uint32_t seq;   // expert-parallel mailbox: the step's sequence number
};

// The tensor-core MoE split: items (slot x tile) are cut into S equal K ranges (units), S the
// largest count that still gives every CTA at most one unit, capped by the K-words per item.
__host__ __device__ __forceinline__ int tc_splits(int n_items, int kw, int grid) {
  int S = n_items > 0 ? grid / n_items : 1;
  S = S < 1 ? 1 : S;
  S = S > kw ? kw : S;
  return S > kTcMaxSeg ? kTcMaxSeg : S;
}

// single thread: local slots ordered by ascending expert id.  ids / wts: the routing, either
// pc.idx / pc.wts or a shared-memory copy of them.
__device__ __forceinline__ void combine_order(const PendingCombine& pc, CombineOrder* co, const int* ids = nullptr,
                                              const float* wv = nullptr) {
  if (!ids) { ids = pc.idx; wv = pc.wts; }
  int n = 0;
  if (pc.partial || pc.seg_part || pc.ep_slots) {
    for (int k = 0; k < pc.K; ++k) {
      const int e = ids[k] - pc.expert_base;
      if (e < 0 || e >= pc.n_local) continue;
      int j = n++;
      while (j > 0 && ids[co->slot[j - 1]] - pc.expert_base > e) {
        co->slot[j] = co->slot[j - 1];
        co->w[j] = co->w[j - 1];
        --j;
      }
      co->slot[j] = k;
      co->w[j] = wv[k];
    }
  }
  co->n = n;
}

// all threads of the block, after combine_order and a barrier (nothing to prepare any more)
__device__ __forceinline__ void combine_prepare(const PendingCombine&, CombineOrder*) {}

// moe_out[r], accumulated from zero in ascending expert order as the reference does
// output row r of local slot k
__device__ __forceinline__ float slot_value(const PendingCombine& pc, int k, int H, int r) {
  (void)H;
  return pc.partial[(size_t)k * H + r];
}

__device__ __forceinline__ float combine_at(const PendingCombine& pc, const CombineOrder& co, int H, int r) {
  if (pc.dense) return pc.dense[r];
  if (pc.ep_recv && pc.ep_slots) {   // every slot's output from its owner rank: ascending expert id
    const float* rb = pc.ep_recv + (size_t)(co.seq & 1u) * pc.ep_rows * H + r;
    float acc = 0.f;
    for (int q = 0; q < co.n; ++q) acc = __fadd_rn(acc, __fmul_rn(__ldcg(rb + (size_t)co.slot[q] * H), co.w[q]));
    return acc;
  }
  if (pc.ep_recv) {   // the ranks' partial outputs, summed in rank order (written by peers: L2 loads)
    const float* rb = pc.ep_recv + (size_t)(co.seq & 1u) * pc.ep_rows * H + r;
    float acc = 0.f;
    for (int j = 0; j < pc.ep_n; ++j) acc += __ldcg(rb + (size_t)j * H);
    return acc;
  }
  float acc = 0.f;
  if (pc.seg_part) {
    const int t = r >> 7, ns = tc_splits(co.n * pc.seg_tiles, pc.seg_kw, pc.seg_grid);
    const size_t off = (size_t)t * kTcMaxSeg * 128 + (r & 127), qstride = (size_t)pc.seg_tiles * kTcMaxSeg * 128;
    if (co.n <= 8 && ns <= 4) {
      // up to 8 slots x 4 ranges as independent predicated loads, so they are in flight together
      float y[8][4];
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float* sp = pc.seg_part + q * qstride + off;
#pragma unroll
        for (int s2 = 0; s2 < 4; ++s2) y[q][s2] = (q < co.n && s2 < ns) ? __ldcg(sp + s2 * 128) : 0.f;
      }
#pragma unroll
      for (int q = 0; q < 8; ++q)
        if (q < co.n) acc += ((((y[q][0] + y[q][1]) + y[q][2]) + y[q][3])) * co.w[q];   // ranges in K order
      return acc;
    }
    for (int q = 0; q < co.n; ++q) {
      float v = 0.f;
      for (int s2 = 0; s2 < ns; ++s2) v += __ldcg(pc.seg_part + q * qstride + off + s2 * 128);
      acc += v * co.w[q];
    }
    return acc;
  }
  // ascending expert id, each product rounded before the sum (out += y * w, layer.rs:1845-1847)
  if (co.n <= 8) {   // the slots' loads in flight together
    float y[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) y[q] = q < co.n ? pc.partial[(size_t)co.slot[q] * H + r] : 0.f;
#pragma unroll
    for (int q = 0; q < 8; ++q)
      if (q < co.n) acc = __fadd_rn(acc, __fmul_rn(y[q], co.w[q]));
    return acc;
  }
  for (int q = 0; q < co.n; ++q) acc = __fadd_rn(acc, __fmul_rn(pc.partial[(size_t)co.slot[q] * H + r], co.w[q]));
  return acc;
}

// Q8_0 quantization of one 32-element block as candle's BlockQ8_0::from_float does:
// d = amax / 127 (stored as f16), q = roundf(x / d) with the unrounded f32 d.
__device__ __forceinline__ void quantize_q8_block(const float (&v)[32], int8_t* q, float* d_out) {
  float amax = 0.f;
#pragma unroll
  for (int k = 0; k < 32; ++k) amax = fmaxf(amax, fabsf(v[k]));
  const float d = amax / 127.0f;
  const float id = d != 0.0f ? 1.0f / d : 0.0f;
  int qw[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    uint32_t u = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) u |= ((uint32_t)(uint8_t)(int8_t)roundf(v[4 * k + j] * id)) << (8 * j);
    qw[k] = (int)u;
  }
  int4* dst = reinterpret_cast<int4*>(q);
  dst[0] = make_int4(qw[0], qw[1], qw[2], qw[3]);
  dst[1] = make_int4(qw[4], qw[5], qw[6], qw[7]);
  *d_out = __half2float(__float2half_rn(d));
}

// ---- order-independent f32 results ----
// Every reduction that produces an f32 value (dot products, sums, the RMSNorm mean) is taken in
// double and rounded once, and exp is the double exp rounded to f32: the f32 result is then the
// exact value correctly rounded (except when it lies within ~1e-16 relative of a rounding midpoint),
// whatever the summation order.  The CPU oracle evaluates the reference's ops the same way, so both
// produce the same bits -- including the Q8_0 codes and routing decisions that follow them.
__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float expcr(float x) { return (float)exp((double)x); }

// Exact base-8 terms of one 32-element f32 block (one element per lane), the B operand of the exact
// MXFP4 expert dots on the tensor cores: X_j = round(|x_j| 2^F) with F = 180 - (the block's largest
// biased exponent), so X_j < 2^54 and X keeps every bit of the block's larger elements.  X is written
// in kExactDigits = 19 balanced base-8 digits d in [-4, 3] (19 because balanced digits reach only
// 3/7 of 8^n), and term t of element j is the e2m1 code of sign(x_j) * d_t -- a value in [-4, 4],
// every one of which e2m1 holds exactly.  The chunk's 768-byte block holds 48 B columns of 32 codes
// (16 bytes, element 2i in the low nibble of byte i); the block's terms are columns parity * 24 + t,
// parity = the chunk index & 1, and every other column stays zero, so one K = 64 MMA over two
// chunks keeps the chunks' dots apart.  *fexp = 1023 - 127 - F, the block's part of the double
// scale exponent.
constexpr int kExactDigits = 19;
constexpr int kExactCols = 48;          // B columns per chunk block (two parities of 24)
constexpr int kExactBlock = kExactCols * 16;
__device__ __forceinline__ void exact_bterm_warp(float x, int lane, uint8_t* blk, int parity, int* fexp) {
  int eb = (int)((__float_as_uint(x) >> 23) & 0xFFu);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) eb = max(eb, __shfl_xor_sync(0xffffffffu, eb, o));
  const int F = 180 - eb;
  long long X = __double2ll_rn(fabs((double)x) * __longlong_as_double((long long)(F + 1023) << 52));
  const bool neg = (__float_as_uint(x) >> 31) != 0;
  uint32_t* col = reinterpret_cast<uint32_t*>(blk + parity * 24 * 16) + (lane >> 3);
#pragma unroll
  for (int t = 0; t < kExactDigits; ++t) {
    const int d = (int)((X + 4) & 7) - 4;   // balanced digit
    X = (X - d) >> 3;
    const int v = neg ? -d : d;             // in [-4, 4]
    const uint32_t mag = (uint32_t)(v < 0 ? -v : v);
    uint32_t code = (0x65420u >> (4 * mag)) & 0xFu;   // e2m1 of 0, 1, 2, 3, 4 (0x0, 0x2, 0x4, 0x5, 0x6)
    code |= v < 0 ? 8u : 0u;
    uint32_t w = code << (4 * (lane & 7));  // 8 lanes' codes -> one 32-bit word
    w |= __shfl_xor_sync(0xffffffffu, w, 1);
    w |= __shfl_xor_sync(0xffffffffu, w, 2);
    w |= __shfl_xor_sync(0xffffffffu, w, 4);
    if ((lane & 7) == 0) col[t * 4] = w;
  }
  if (lane == 0) *fexp = 1023 - 127 - F;
}

// inverse RMS with the reference's op sequence (ops/norm.rs:16-37): x.sqr() in f32, mean_keepdim =
// (sum rounded to f32) * f32(1/n) (candle's affine), + eps, sqrt, recip.  Threads tid in [0, nthr)
// (nthr a multiple of 32) take part; bar() synchronises them; every one gets the result.
template <class Bar>
__device__ __forceinline__ float rms_inv_cr(const float* x, int n, float eps, int tid, int nthr, Bar bar) {
  __shared__ double s_rms_red[33];
  double ss = 0.0;
  for (int i = tid; i < n; i += nthr) ss += (double)__fmul_rn(x[i], x[i]);
  ss = warp_sum_d(ss);
  if ((tid & 31) == 0) s_rms_red[tid >> 5] = ss;
  bar();
  double t = 0.0;
  for (int w = 0; w < (nthr >> 5); ++w) t += s_rms_red[w];
  bar();   // s_rms_red may be reused
  const float var = __fadd_rn(__fmul_rn((float)t, (float)(1.0 / (double)n)), 0.0f);
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
}

// the same for one vector held by one warp (per-head QK-norm)
__device__ __forceinline__ float rms_inv_cr_warp(const float* x, int n, float eps, int lane) {
  double ss = 0.0;
  for (int i = lane; i < n; i += 32) ss += (double)__fmul_rn(x[i], x[i]);
  ss = warp_sum_d(ss);
  const float var = __fadd_rn(__fmul_rn((float)ss, (float)(1.0 / (double)n)), 0.0f);
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
}

// Whole-CTA RMSNorm (weights w) of xs[0..H) in shared memory, then Q8_0 quantization into
// xq / xd (one thread per 32-element block).  red: >= 256 floats of shared scratch.
__device__ __forceinline__ void cta_rmsnorm_q8(const float* xs, int H, const float* w, float eps, int8_t* xq,
                                               float* xd, float* red) {
  (void)red;
  const int lane = threadIdx.x & 31;
  const float inv = rms_inv_cr(xs, H, eps, threadIdx.x, blockDim.x, [] { __syncthreads(); });
  for (int b = threadIdx.x; b < H / 32; b += blockDim.x) {
    float v[32];
#pragma unroll
    for (int k = 0; k < 32; ++k) {
      const int kk = (k + lane) & 31;   // rotate the start so lanes hit different banks
      v[kk] = __fmul_rn(__fmul_rn(xs[32 * b + kk], inv), w[32 * b + kk]);
    }
    quantize_q8_block(v, xq + 32 * b, &xd[b]);
  }
}

__device__ __forceinline__ uint32_t ld_acquire_sys_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys_u32(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Single thread: wait (bounded) until every rank's mailbox flag of this step is released; the
// sequence number goes to co->seq.  On expiry the error word gets EF_TIMEOUT_FULL.
__device__ __forceinline__ void ep_wait(const PendingCombine& pc, CombineOrder* co, uint32_t* err) {
  const uint32_t seq = *reinterpret_cast<const volatile uint32_t*>(pc.ep_seq);
  co->seq = seq;
  const uint32_t* f = pc.ep_flags + (size_t)(seq & 1u) * pc.ep_n;
  for (int j = 0; j < pc.ep_n; ++j) {
    uint32_t it = 0;
    while ((int32_t)(ld_acquire_sys_u32(f + j) - seq) < 0 && ++it < kWaitLimit) __nanosleep(64);
    if (it >= kWaitLimit) { atomicOr(err, EF_TIMEOUT_FULL); return; }
  }
}

// Programmatic dependent launch: let the next kernel start its prologue early /
// wait for the previous kernel's memory to be visible.
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait_prior() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

}  // namespace ms
