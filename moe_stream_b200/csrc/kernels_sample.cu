// kernels_sample.cu — the next token drawn from the logits on the device: SamplingParams::sample
// (model/engine.rs:124-208) with the order-independent reduction convention of the decode step.
//
// Steps, as the reference orders them: the repetition penalty over the generated tokens (a logit
// of a token generated n times is divided n times by the penalty when positive, else multiplied),
// greedy argmax when temperature == 0 (Iterator::max_by: the last index among equal maxima), else
// scaling by f32(1 / temperature), the stable softmax exp(v - max) / sum, the top-p nucleus when
// top_p < 1 (probabilities sorted descending with ties in index order, the shortest prefix whose
// running sum exceeds top_p, renormalised), and the first index whose running sum of the
// probabilities exceeds the draw r in [0, 1).
//
// Reductions.  Every sum of probabilities (the softmax denominator, the nucleus mass, the running
// sums compared with top_p and r) is accumulated as a 128-bit fixed-point integer with its least
// significant bit at 2^-109 -- integer addition is associative, so the result does not depend on
// order -- and rounded to f32 (nearest, ties to even) once where the reference holds an f32: a
// probability below 2^-85 loses the bits below 2^-109.  exp is the double exp rounded to f32.
//
// One CTA of 1024 threads runs every pass over the vocabulary in index order, so per-element ranks
// (ties at the nucleus boundary, the first crossing of r) come from block scans.  The nucleus
// boundary is found by a 3-pass radix select on the probabilities' f32 bit patterns (11 + 11 + 9
// bits), each pass a shared-memory histogram of counts and fixed-point masses.
#include "common.cuh"
#include "kernels.h"

namespace ms {
namespace {

constexpr int kSThreads = 1024;
constexpr int kSWarps = kSThreads / 32;
constexpr int kSBuckets = 2048;

struct U128 {
  unsigned long long lo, hi;
};
__device__ __forceinline__ U128 u128_add(U128 a, U128 b) {
  U128 r;
  r.lo = a.lo + b.lo;
  r.hi = a.hi + b.hi + (r.lo < a.lo ? 1ull : 0ull);
  return r;
}
__device__ __forceinline__ bool u128_zero(U128 a) { return (a.lo | a.hi) == 0ull; }

// a non-negative finite f32 as a multiple of 2^-109 (truncated below it)
__device__ __forceinline__ U128 fx_from_f32(float v) {
  const uint32_t b = __float_as_uint(v);
  const int E = (int)((b >> 23) & 0xFFu);
  U128 r = {0ull, 0ull};
  if (E == 0 || (b >> 31)) return r;   // zero, denormal (< 2^-126) or negative
  const unsigned long long M = (unsigned long long)((b & 0x7FFFFFu) | 0x800000u);
  const int sh = E - 41;                // v = M 2^(E-150) = M 2^(E-41) 2^-109
  if (sh >= 64) { r.hi = M << (sh - 64); }
  else if (sh > 40) { r.lo = M << sh; r.hi = M >> (64 - sh); }
  else if (sh >= 0) { r.lo = M << sh; }
  else if (sh > -24) { r.lo = M >> (-sh); }
  return r;
}

// a multiple of 2^-109 as a multiple of 2^-109 times m (m < 2^31): exact while it fits
__device__ __forceinline__ U128 u128_mul_small(U128 a, uint32_t m) {
  const unsigned long long lo_lo = (a.lo & 0xFFFFFFFFull) * m, lo_hi = (a.lo >> 32) * m;
  U128 r;
  const unsigned long long mid = (lo_lo >> 32) + lo_hi;
  r.lo = (lo_lo & 0xFFFFFFFFull) | (mid << 32);
  r.hi = a.hi * m + (mid >> 32);
  return r;
}

// round a multiple of 2^-109 to the nearest f32 (ties to even); values are below 2^18
__device__ __forceinline__ float fx_to_f32(U128 a) {
  if (u128_zero(a)) return 0.f;
  const int msb = a.hi ? 127 - __clzll((long long)a.hi) : 63 - __clzll((long long)a.lo);
  // the 24 bits below and including msb, the round bit and the sticky bits
  unsigned long long mant, rest_nonzero;
  int round_bit;
  const int lsb = msb - 23;   // bit index of the mantissa's last bit
  auto bit = [&](int i) -> int { return i >= 64 ? (int)((a.hi >> (i - 64)) & 1ull) : (int)((a.lo >> i) & 1ull); };
  if (lsb >= 0) {
    if (lsb >= 64) mant = a.hi >> (lsb - 64);
    else if (lsb == 0) mant = a.lo;
    else mant = (a.lo >> lsb) | (lsb > 0 ? (a.hi << (64 - lsb)) : 0ull);
    mant &= 0xFFFFFFull;
    round_bit = lsb >= 1 ? bit(lsb - 1) : 0;
    // sticky: any bit below lsb - 1
    if (lsb - 1 <= 0) rest_nonzero = 0ull;
    else if (lsb - 1 >= 64) rest_nonzero = a.lo | (a.hi & ((1ull << (lsb - 1 - 64)) - 1ull));
    else rest_nonzero = a.lo & ((1ull << (lsb - 1)) - 1ull);
  } else {
    mant = a.lo << (-lsb);
    round_bit = 0;
    rest_nonzero = 0ull;
  }
  int e = msb;   // value = mant * 2^(lsb - 109)
  if (round_bit && (rest_nonzero || (mant & 1ull))) {
    ++mant;
    if (mant == 0x1000000ull) {   // carried into a new bit
      mant >>= 1;
      ++e;
    }
  }
  // f32 with biased exponent (e - 109) + 127
  const uint32_t bits = ((uint32_t)(e - 109 + 127) << 23) | (uint32_t)(mant & 0x7FFFFFull);
  return __uint_as_float(bits);
}

struct ScanScratch {
  unsigned long long lo[kSWarps], hi[kSWarps];
  int cnt[kSWarps];
};

// inclusive block scan of a U128 (thread order); *total = the block's sum
__device__ __forceinline__ U128 block_scan_u128(U128 v, ScanScratch* sc, U128* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    U128 u;
    u.lo = __shfl_up_sync(0xffffffffu, v.lo, o);
    u.hi = __shfl_up_sync(0xffffffffu, v.hi, o);
    if (lane >= o) v = u128_add(v, u);
  }
  if (lane == 31) { sc->lo[warp] = v.lo; sc->hi[warp] = v.hi; }
  __syncthreads();
  if (warp == 0) {
    U128 w = {sc->lo[lane], sc->hi[lane]};
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      U128 u;
      u.lo = __shfl_up_sync(0xffffffffu, w.lo, o);
      u.hi = __shfl_up_sync(0xffffffffu, w.hi, o);
      if (lane >= o) w = u128_add(w, u);
    }
    sc->lo[lane] = w.lo;
    sc->hi[lane] = w.hi;
  }
  __syncthreads();
  if (warp > 0) v = u128_add(v, U128{sc->lo[warp - 1], sc->hi[warp - 1]});
  *total = U128{sc->lo[kSWarps - 1], sc->hi[kSWarps - 1]};
  __syncthreads();
  return v;
}

// exclusive block count of a predicate (thread order); *total = the block's count
__device__ __forceinline__ int block_rank(bool pred, ScanScratch* sc, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t bal = __ballot_sync(0xffffffffu, pred);
  if (lane == 0) sc->cnt[warp] = __popc(bal);
  __syncthreads();
  int before = 0, all = 0;
  for (int w = 0; w < kSWarps; ++w) {
    const int c = sc->cnt[w];
    if (w < warp) before += c;
    all += c;
  }
  __syncthreads();
  *total = all;
  return before + __popc(bal & ((1u << lane) - 1u));
}

__device__ __forceinline__ unsigned long long splitmix64(unsigned long long z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

__global__ void __launch_bounds__(kSThreads, 1) sample_kernel(SampleArgs a, uint32_t* err) {
  __shared__ unsigned int h_cnt[kSBuckets];
  __shared__ unsigned long long h_lo[kSBuckets], h_hi[kSBuckets];
  __shared__ ScanScratch sc;
  __shared__ float s_f[kSWarps];
  __shared__ int s_i[kSWarps];
  __shared__ U128 s_above;
  __shared__ uint32_t s_prefix, s_found;
  __shared__ int s_tok;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int V = a.V;
  pdl_wait_prior();
  pdl_launch_dependents();
  if (a.draw && *a.draw == 0) return;   // a prompt position that is not the last: no token is drawn

  float r = a.r;
  if (a.rng) {   // the step's draw: rand's f32 construction (24 random bits) from SplitMix64(seed, n)
    const unsigned long long z = splitmix64(a.rng[0] ^ (a.rng[1] * 0xD1B54A32D192ED03ull));
    r = (float)(uint32_t)(z >> 40) * (1.0f / 16777216.0f);
  }
  // ---- pass 1: penalty, greedy argmax or temperature, max ----
  const bool greedy = a.temperature == 0.0f;
  const float inv_t = __fdiv_rn(1.0f, a.temperature);
  float best = -INFINITY;
  int best_i = -1;
  for (int v = tid; v < V; v += kSThreads) {
    float x = a.logits[v];
    if (a.penalty != 1.0f && a.counts) {
      const uint32_t n = a.counts[v];
      for (uint32_t j = 0; j < n; ++j) x = x > 0.0f ? __fdiv_rn(x, a.penalty) : __fmul_rn(x, a.penalty);
    }
    if (!greedy && a.temperature != 1.0f) x = __fmul_rn(x, inv_t);
    a.work[v] = x;
    if (x > best || (greedy && x == best)) { best = x; best_i = v; }   // greedy: the last maximum
  }
  // block max (greedy: with the largest index among equal maxima)
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, best_i, o);
    if (ob > best || (ob == best && oi > best_i)) { best = ob; best_i = oi; }
  }
  if (lane == 0) { s_f[warp] = best; s_i[warp] = best_i; }
  __syncthreads();
  if (tid == 0) {
    float b = -INFINITY;
    int bi = -1;
    for (int w = 0; w < kSWarps; ++w)
      if (s_f[w] > b || (s_f[w] == b && s_i[w] > bi)) { b = s_f[w]; bi = s_i[w]; }
    s_f[0] = b;
    s_tok = bi < 0 ? 0 : bi;
  }
  __syncthreads();
  const float mx = s_f[0];
  if (!greedy) {
    // ---- pass 2: e = exp(x - max), the denominator ----
    U128 part = {0ull, 0ull};
    for (int v = tid; v < V; v += kSThreads) {
      const float e = expcr(__fsub_rn(a.work[v], mx));
      a.work[v] = e;
      part = u128_add(part, fx_from_f32(e));
    }
    U128 tot;
    block_scan_u128(part, &sc, &tot);
    const float S = fx_to_f32(tot);
    for (int v = tid; v < V; v += kSThreads) a.work[v] = __fdiv_rn(a.work[v], S);   // p
    __syncthreads();
    // ---- top-p: the nucleus boundary by radix select on p's bits ----
    bool cut = false;          // elements outside the nucleus are zeroed
    const bool renorm = a.top_p < 1.0f;   // the reference renormalises whenever top_p < 1
    uint32_t vstar = 0;        // boundary probability's bits
    uint32_t m_keep = 0;       // ties at vstar kept (in index order)
    float S2 = 1.0f;
    if (renorm) {
      if (tid == 0) { s_above = U128{0ull, 0ull}; s_prefix = 0u; s_found = 1u; }
      __syncthreads();
      const int shifts[3] = {20, 9, 0}, widths[3] = {11, 11, 9};
      uint32_t cstar = 0;
      for (int pass = 0; pass < 3; ++pass) {
        const int sh = shifts[pass], wd = widths[pass];
        const uint32_t hi_mask = pass == 0 ? 0u : (0x7FFFFFFFu >> (sh + wd)) << (sh + wd);
        for (int b = tid; b < kSBuckets; b += kSThreads) { h_cnt[b] = 0u; h_lo[b] = 0ull; h_hi[b] = 0ull; }
        __syncthreads();
        if (!s_found) break;
        const uint32_t prefix = s_prefix;
        for (int v = tid; v < V; v += kSThreads) {
          const uint32_t bits = __float_as_uint(a.work[v]);
          if ((bits & hi_mask) != prefix) continue;
          const int bk = (int)((bits >> sh) & ((1u << wd) - 1u));
          const U128 f = fx_from_f32(a.work[v]);
          atomicAdd(&h_cnt[bk], 1u);
          const unsigned long long old = atomicAdd(&h_lo[bk], f.lo);
          unsigned long long carry = (old + f.lo < old) ? 1ull : 0ull;
          if (f.hi + carry) atomicAdd(&h_hi[bk], f.hi + carry);
        }
        __syncthreads();
        // the first bucket (descending) where the running sum, rounded to f32, exceeds top_p:
        // warp 0, lane l takes buckets [64 l, 64 l + 64) read top down
        if (warp == 0) {
          const int nb = 1 << wd, per = nb / 32;
          const int b_top = nb - 1 - lane * per;   // this lane's buckets: b_top down to b_top - per + 1
          U128 lm = {0ull, 0ull};
          for (int q = 0; q < per; ++q) lm = u128_add(lm, U128{h_lo[b_top - q], h_hi[b_top - q]});
          // exclusive scan in lane order (lane 0 holds the largest buckets)
          U128 inc = lm;
#pragma unroll
          for (int o = 1; o < 32; o <<= 1) {
            U128 u;
            u.lo = __shfl_up_sync(0xffffffffu, inc.lo, o);
            u.hi = __shfl_up_sync(0xffffffffu, inc.hi, o);
            if (lane >= o) inc = u128_add(inc, u);
          }
          const U128 above = s_above;
          const U128 before = u128_add(above, U128{inc.lo - lm.lo - 0ull, inc.hi - lm.hi - (inc.lo < lm.lo ? 1ull : 0ull)});
          const bool crosses = fx_to_f32(u128_add(above, inc)) > a.top_p;
          const uint32_t cb = __ballot_sync(0xffffffffu, crosses);
          if (cb == 0u) {
            if (lane == 0) s_found = 0u;   // the whole remaining mass never exceeds top_p: keep all
          } else if (lane == __ffs(cb) - 1) {
            U128 run = before;
            for (int q = 0; q < per; ++q) {
              const int b = b_top - q;
              const U128 nx = u128_add(run, U128{h_lo[b], h_hi[b]});
              if (h_cnt[b] && fx_to_f32(nx) > a.top_p) {
                s_above = run;
                s_prefix = prefix | ((uint32_t)b << sh);
                s_i[0] = (int)h_cnt[b];
                break;
              }
              run = nx;
            }
          }
        }
        __syncthreads();
      }
      if (s_found) {
        cut = true;
        vstar = s_prefix;
        cstar = (uint32_t)s_i[0];
        // ties at the boundary: the fewest m >= 1 (in index order) whose running sum exceeds top_p
        const U128 above = s_above, fv = fx_from_f32(__uint_as_float(vstar));
        uint32_t lo_m = 1u, hi_m = cstar;
        while (lo_m < hi_m) {
          const uint32_t mid = (lo_m + hi_m) >> 1;
          if (fx_to_f32(u128_add(above, u128_mul_small(fv, mid))) > a.top_p) hi_m = mid;
          else lo_m = mid + 1u;
        }
        m_keep = lo_m;
        S2 = fx_to_f32(u128_add(above, u128_mul_small(fv, m_keep)));
      } else {
        // no prefix exceeds top_p: every token stays, renormalised by the sum of all p
        U128 part2 = {0ull, 0ull};
        for (int v = tid; v < V; v += kSThreads) part2 = u128_add(part2, fx_from_f32(a.work[v]));
        U128 tp;
        block_scan_u128(part2, &sc, &tp);
        S2 = fx_to_f32(tp);
      }
      __syncthreads();
    }
    // ---- the draw: the first index whose running sum of the (kept, renormalised) p exceeds r ----
    U128 run = {0ull, 0ull};
    int ties_before = 0;
    if (tid == 0) s_tok = 0x7FFFFFFF;
    __syncthreads();
    for (int base = 0; base < V; base += kSThreads) {
      const int v = base + tid;
      float q = 0.f;
      bool tie = false;
      if (v < V) {
        const float p = a.work[v];
        const uint32_t bits = __float_as_uint(p);
        tie = cut && bits == vstar;
        q = p;
        if (cut) q = bits > vstar ? __fdiv_rn(p, S2) : 0.f;
        else if (renorm) q = __fdiv_rn(p, S2);
      }
      if (cut) {
        int nt;
        const int rk = block_rank(tie, &sc, &nt);
        if (tie && (uint32_t)(ties_before + rk) < m_keep) q = __fdiv_rn(__uint_as_float(vstar), S2);
        ties_before += nt;
      }
      U128 tot2;
      const U128 inc = u128_add(run, block_scan_u128(fx_from_f32(q), &sc, &tot2));
      const bool hit = v < V && q > 0.f && fx_to_f32(inc) > r;
      const uint32_t hb = __ballot_sync(0xffffffffu, hit);
      if (hb && lane == __ffs(hb) - 1) atomicMin(&s_tok, v);
      __syncthreads();
      if (s_tok != 0x7FFFFFFF) break;
      run = u128_add(run, tot2);
    }
    if (tid == 0 && s_tok == 0x7FFFFFFF) s_tok = V - 1;   // rounding edge: the reference's fallback
    __syncthreads();
  }
  if (tid == 0) {
    const int tok = s_tok;
    if (a.token_out) *a.token_out = tok;
    if (a.key_out) *a.key_out = (1ull << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)tok);
    if (a.counts_rw && tok >= 0 && tok < V) a.counts_rw[tok] += 1u;
    if (a.rng) a.rng[1] += 1ull;
  }
  (void)err;
}

}  // namespace

cudaError_t launch_sample(const DevCtx& c, const SampleArgs& a, cudaStream_t s) {
  if (!a.logits || !a.work || a.V <= 0 || (!a.token_out && !a.key_out) || !(a.temperature >= 0.0f) ||
      !(a.top_p > 0.0f) || !(a.penalty > 0.0f))
    return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(kSThreads);
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, sample_kernel, a, c.err);
}

}  // namespace ms
