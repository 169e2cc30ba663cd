// msoracle.cpp — CPU restatement of moe-stream's default CPU inference path.
// TEST INFRASTRUCTURE ONLY: the parity checker and timed CPU baseline; never part of
// the product.  Build with -ffp-contract=off so a*b-c*d is evaluated as the
// reference's separate tensor ops evaluate it (no fused multiply-add).
// All file:line citations refer to the moe-stream repository (moe-stream-core/src/...).
#include "msoracle.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <functional>
#include <limits>
#include <map>
#include <string>
#include <thread>
#include <vector>

namespace {

// ---------------------------------------------------------------------------
// Numeric convention.  Every f32 tensor op of the reference is evaluated as IEEE f32 (elementwise
// add, mul, div, sqrt, min/max) and every reduction (matmul / dot, sum) and exp / log as the exact
// value rounded once to f32: summed in double (the f32 x f32 products are exact in double), then
// converted.  candle's own summation order is third-party and not pinned by any reference test;
// rounding the exact result makes the oracle's values independent of summation order, so the CUDA
// kernels (which also reduce in double) reproduce them bit for bit.
inline float round_f32(double v) { return (float)v; }
inline float expcr(float x) { return (float)std::exp((double)x); }
inline float logcr(float x) { return (float)std::log((double)x); }

// ---------------------------------------------------------------------------
// threading: static row chunking across hardware threads (dequant.rs:650-692 style)
int g_default_threads = 0;
int hw_threads() {
  if (g_default_threads > 0) return g_default_threads;
  unsigned n = std::thread::hardware_concurrency();
  return n ? (int)n : 1;
}
void parallel_for(int64_t n, int threads, const std::function<void(int64_t, int64_t)>& fn) {
  if (threads <= 1 || n < 2) { fn(0, n); return; }
  int t = (int)std::min<int64_t>(threads, n);
  int64_t chunk = (n + t - 1) / t;
  std::vector<std::thread> th;
  for (int i = 0; i < t; ++i) {
    int64_t b = i * chunk, e = std::min(n, b + chunk);
    if (b >= e) break;
    th.emplace_back([=, &fn] { fn(b, e); });
  }
  for (auto& x : th) x.join();
}

inline uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

// ---------------------------------------------------------------------------
// f16 -> f32, exact IEEE conversion (the `half` crate used at dequant.rs:37-41)
float h2f(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000) << 16;
  uint32_t exp = (h >> 10) & 0x1f, man = h & 0x3ff, bits;
  if (exp == 0) {
    if (man == 0) bits = sign;
    else {  // subnormal: normalise
      int e = -1;
      do { man <<= 1; ++e; } while (!(man & 0x400));
      bits = sign | ((uint32_t)(127 - 15 - e) << 23) | ((man & 0x3ff) << 13);
    }
  } else if (exp == 31) bits = sign | 0x7f800000u | (man << 13);
  else bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
  float f; std::memcpy(&f, &bits, 4); return f;
}

// f32 -> f16 round-to-nearest-even (the `half` crate's f16::from_f32)
uint16_t f2h(float f) {
  uint32_t x; std::memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000;
  uint32_t ax = x & 0x7fffffff;
  if (ax >= 0x7f800000) return (uint16_t)(sign | 0x7c00 | (ax > 0x7f800000 ? 0x200 | ((ax >> 13) & 0x3ff) : 0));
  if (ax >= 0x477ff000) return (uint16_t)(sign | 0x7c00);  // rounds to >= 65520 -> inf
  if (ax < 0x38800000) {  // result subnormal or zero
    if (ax < 0x33000000) return (uint16_t)sign;            // < 2^-25 rounds to 0
    uint32_t e = ax >> 23, m = (ax & 0x7fffff) | 0x800000;
    uint32_t shift = 126 - e;                               // 14 + (113 - e) ... bits to drop
    uint32_t half = m >> (shift - 1);
    uint32_t r = half >> 1;
    uint32_t rem = m & ((1u << (shift - 1)) - 1);
    if ((half & 1) && (rem || (r & 1))) r++;
    return (uint16_t)(sign | r);
  }
  uint32_t e = (ax >> 23) - 127 + 15, m = ax & 0x7fffff;
  uint32_t r = (e << 10) | (m >> 13);
  uint32_t rem = m & 0x1fff;
  if (rem > 0x1000 || (rem == 0x1000 && (r & 1))) r++;
  return (uint16_t)(sign | r);
}

float bits2f(uint32_t b) { float f; std::memcpy(&f, &b, 4); return f; }

// dequant.rs:580-583
const float kMxfp4Values[16] = {0.0f, 1.0f, 2.0f, 3.0f, 4.0f, 6.0f, 8.0f, 12.0f,
                                -0.0f, -1.0f, -2.0f, -3.0f, -4.0f, -6.0f, -8.0f, -12.0f};

// dequant.rs:589-597
float e8m0_half(uint8_t e) {
  if (e < 2) return bits2f(0x00200000u << e);
  return bits2f(((uint32_t)e - 1u) << 23);
}

// dequant.rs:605-628
void deq_mxfp4(const uint8_t* x, int64_t nb, float* y) {
  for (int64_t b = 0; b < nb; ++b, x += 17, y += 32) {
    float d = e8m0_half(x[0]);
    for (int j = 0; j < 16; ++j) {
      y[j] = kMxfp4Values[x[1 + j] & 0x0f] * d;
      y[j + 16] = kMxfp4Values[x[1 + j] >> 4] * d;
    }
  }
}

// dequant.rs:511-531
void deq_q8_0(const uint8_t* x, int64_t nb, float* y) {
  for (int64_t b = 0; b < nb; ++b, x += 34, y += 32) {
    float d = h2f(rd16(x));
    for (int i = 0; i < 32; ++i) y[i] = d * (float)(int8_t)x[2 + i];
  }
}

// dequant.rs:199-208
inline void scale_min_k4(int j, const uint8_t* q, uint8_t* sc, uint8_t* m) {
  if (j < 4) { *sc = q[j] & 63; *m = q[j + 4] & 63; }
  else {
    *sc = (uint8_t)((q[j + 4] & 0x0f) | ((q[j - 4] >> 6) << 4));
    *m = (uint8_t)((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
  }
}

// dequant.rs:218-262
void deq_q4_k(const uint8_t* x, int64_t nb, float* y) {
  for (int64_t b = 0; b < nb; ++b, x += 144, y += 256) {
    float d = h2f(rd16(x)), dmin = h2f(rd16(x + 2));
    const uint8_t* sc = x + 4; const uint8_t* qs = x + 16;
    int is = 0; float* o = y;
    for (int j = 0; j < 4; ++j) {
      uint8_t s0, m0, s1, m1;
      scale_min_k4(is, sc, &s0, &m0);
      float d1 = d * (float)s0, m1f = dmin * (float)m0;
      scale_min_k4(is + 1, sc, &s1, &m1);
      float d2 = d * (float)s1, m2f = dmin * (float)m1;
      for (int l = 0; l < 32; ++l) *o++ = d1 * (float)(qs[j * 32 + l] & 0x0f) - m1f;
      for (int l = 0; l < 32; ++l) *o++ = d2 * (float)(qs[j * 32 + l] >> 4) - m2f;
      is += 2;
    }
  }
}

// dequant.rs:335-378
void deq_q6_k(const uint8_t* x, int64_t nb, float* y) {
  for (int64_t b = 0; b < nb; ++b, x += 210, y += 256) {
    const uint8_t* ql = x; const uint8_t* qh = x + 128;
    const int8_t* sc = (const int8_t*)(x + 192);
    float d = h2f(rd16(x + 208));
    int yo = 0;
    for (int n = 0; n < 256; n += 128) {
      for (int l = 0; l < 32; ++l) {
        int is = n / 16 + l / 16;
        int q1 = ((ql[l] & 0x0f) | ((qh[l] & 3) << 4)) - 32;
        int q2 = ((ql[l + 32] & 0x0f) | (((qh[l] >> 2) & 3) << 4)) - 32;
        int q3 = ((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
        int q4 = ((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
        y[yo + l] = d * (float)sc[is] * (float)q1;
        y[yo + l + 32] = d * (float)sc[is + 2] * (float)q2;
        y[yo + l + 64] = d * (float)sc[is + 4] * (float)q3;
        y[yo + l + 96] = d * (float)sc[is + 6] * (float)q4;
      }
      yo += 128; ql += 64; qh += 32;
    }
  }
}

struct QInfo { int bytes, elems; };
bool qinfo(int q, QInfo* qi) {
  switch (q) {
    case ORC_F32: *qi = {4, 1}; return true;
    case ORC_F16: *qi = {2, 1}; return true;
    case ORC_Q8_0: *qi = {34, 32}; return true;
    case ORC_Q4_K: *qi = {144, 256}; return true;
    case ORC_Q6_K: *qi = {210, 256}; return true;
    case ORC_MXFP4: *qi = {17, 32}; return true;
  }
  return false;
}
int64_t raw_size(int q, int64_t n) {
  QInfo qi; if (!qinfo(q, &qi)) return -1;
  return (n + qi.elems - 1) / qi.elems * qi.bytes;
}

int dequant(int q, const void* src, int64_t n, float* out) {
  const uint8_t* p = (const uint8_t*)src;
  switch (q) {
    case ORC_F32: std::memcpy(out, src, n * 4); return 0;
    case ORC_F16: for (int64_t i = 0; i < n; ++i) out[i] = h2f(rd16(p + 2 * i)); return 0;
    case ORC_Q8_0: deq_q8_0(p, n / 32, out); return 0;
    case ORC_Q4_K: deq_q4_k(p, n / 256, out); return 0;
    case ORC_Q6_K: deq_q6_k(p, n / 256, out); return 0;
    case ORC_MXFP4: deq_mxfp4(p, n / 32, out); return 0;
  }
  return -1;
}

// f32 dequantize of a [rows, cols] matrix, rows split across threads
void dequant_matrix(int q, const void* src, int64_t rows, int64_t cols, float* out, int threads) {
  int64_t rb = raw_size(q, cols);
  parallel_for(rows, threads, [&](int64_t b, int64_t e) {
    for (int64_t r = b; r < e; ++r) dequant(q, (const uint8_t*)src + r * rb, cols, out + r * cols);
  });
}

// y[t, r] = sum_c x[t, c] * W[r, c]  (candle f32 matmul x.matmul(W.t()); sequential dot order)
void matmul_xwt(const float* x, int64_t n_tok, const float* W, int64_t rows, int64_t cols, float* y,
                int threads) {
  parallel_for(rows, threads, [&](int64_t b, int64_t e) {
    for (int64_t t = 0; t < n_tok; ++t) {
      const float* xt = x + t * cols;
      for (int64_t r = b; r < e; ++r) {
        const float* w = W + r * cols;
        double acc = 0.0;
        for (int64_t c = 0; c < cols; ++c) acc += (double)xt[c] * (double)w[c];
        y[t * rows + r] = round_f32(acc);
      }
    }
  });
}

// candle BlockQ8_0::from_float — the activation quantization used by QMatMul's vec_dot
void quantize_q8_0(const float* x, int64_t n, uint8_t* out) {
  for (int64_t b = 0; b < n / 32; ++b) {
    const float* xb = x + b * 32; uint8_t* o = out + b * 34;
    float amax = 0.0f;
    for (int i = 0; i < 32; ++i) amax = std::max(amax, std::fabs(xb[i]));
    float d = amax / 127.0f;
    float id = d != 0.0f ? 1.0f / d : 0.0f;
    uint16_t hd = f2h(d);
    o[0] = (uint8_t)(hd & 0xff); o[1] = (uint8_t)(hd >> 8);
    for (int i = 0; i < 32; ++i) o[2 + i] = (uint8_t)(int8_t)std::round(xb[i] * id);
  }
}

// QMatMul Q8_0 x Q8_0 vec_dot: sum_i over blocks (int dot) * d_w * d_x, f32 accumulation
void q8_0_gemv_actq(const uint8_t* w, int64_t rows, int64_t cols, const float* x, float* y, int threads,
                    int64_t n_tok = 1) {
  int64_t nb = cols / 32, rb = nb * 34;
  std::vector<uint8_t> xq(n_tok * rb);
  for (int64_t t = 0; t < n_tok; ++t) quantize_q8_0(x + t * cols, cols, xq.data() + t * rb);
  parallel_for(rows, threads, [&](int64_t b, int64_t e) {
    for (int64_t t = 0; t < n_tok; ++t) {
      const uint8_t* xt = xq.data() + t * rb;
      for (int64_t r = b; r < e; ++r) {
        const uint8_t* wr = w + r * rb;
        double sumf = 0.0;
        for (int64_t k = 0; k < nb; ++k) {
          const uint8_t* wb = wr + k * 34; const uint8_t* xb = xt + k * 34;
          int32_t sumi = 0;
          for (int i = 0; i < 32; ++i) sumi += (int32_t)(int8_t)wb[2 + i] * (int32_t)(int8_t)xb[2 + i];
          sumf += (double)sumi * (double)h2f(rd16(wb)) * (double)h2f(rd16(xb));   // exact in double
        }
        y[t * rows + r] = round_f32(sumf);
      }
    }
  });
}

// ops/norm.rs:16-37: x * recip(sqrt(mean(x^2) + eps)) * w
void rms_norm(const float* x, const float* w, float* y, int64_t rows, int64_t dim, float eps) {
  for (int64_t r = 0; r < rows; ++r) {
    const float* xr = x + r * dim; float* yr = y + r * dim;
    // x.sqr() (f32), mean_keepdim = sum * (1/n) (candle's affine), + eps, sqrt, recip
    double ss = 0.0;
    for (int64_t i = 0; i < dim; ++i) ss += (double)(xr[i] * xr[i]);
    const float var = round_f32(ss) * (float)(1.0 / (double)dim) + 0.0f;
    const float inv = 1.0f / std::sqrt(var + eps);
    for (int64_t i = 0; i < dim; ++i) yr[i] = (xr[i] * inv) * w[i];
  }
}

// ops/activation.rs:41-45
inline float sigmoid_ref(float x) { return 1.0f / (expcr(-x) + 1.0f); }

// ops/activation.rs:25-38
void swiglu_oai(const float* g, const float* u, float* out, int64_t n, float alpha, float limit) {
  for (int64_t i = 0; i < n; ++i) {
    float gc = std::min(g[i], limit);
    float uc = std::min(std::max(u[i], -limit), limit);
    float ga = gc * sigmoid_ref(gc * alpha + 0.0f);
    out[i] = ga * (uc + 1.0f);
  }
}

// ops/activation.rs:13-15 (candle_nn silu: x / (1 + exp(-x)))
void silu_and_mul(const float* g, const float* u, float* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = (g[i] / (1.0f + expcr(-g[i]))) * u[i];
}

// layer.rs:2346-2403 (stable descending sort, ties -> lower index first)
void top_k_routing(const float* logits, int n_tok, int n_exp, int k, bool normalize, bool softmax_weight,
                   int32_t* idx, float* wout) {
  std::vector<std::pair<int, float>> v(n_exp);
  auto desc = [](const std::pair<int, float>& a, const std::pair<int, float>& b) { return a.second > b.second; };
  for (int t = 0; t < n_tok; ++t) {
    const float* row = logits + (int64_t)t * n_exp;
    if (softmax_weight) {
      for (int e = 0; e < n_exp; ++e) v[e] = {e, row[e]};
      std::stable_sort(v.begin(), v.end(), desc);
      float mx = -std::numeric_limits<float>::infinity();
      for (int j = 0; j < k; ++j) mx = std::max(mx, v[j].second);
      std::vector<float> ex(k); double sum64 = 0.0;
      for (int j = 0; j < k; ++j) { ex[j] = expcr(v[j].second - mx); }
      for (int j = 0; j < k; ++j) sum64 += ex[j];
      const float sum = round_f32(sum64);
      for (int j = 0; j < k; ++j) { idx[t * k + j] = v[j].first; wout[t * k + j] = ex[j] / sum; }
    } else {
      float mx = -std::numeric_limits<float>::infinity();
      for (int e = 0; e < n_exp; ++e) mx = std::max(mx, row[e]);
      std::vector<float> ex(n_exp); double sum64 = 0.0;
      for (int e = 0; e < n_exp; ++e) ex[e] = expcr(row[e] - mx);
      for (int e = 0; e < n_exp; ++e) sum64 += ex[e];
      const float sum = round_f32(sum64);
      for (int e = 0; e < n_exp; ++e) v[e] = {e, ex[e] / sum};
      std::stable_sort(v.begin(), v.end(), desc);
      double ts64 = 0.0;
      for (int j = 0; j < k; ++j) ts64 += v[j].second;
      const float ts = round_f32(ts64);
      for (int j = 0; j < k; ++j) {
        idx[t * k + j] = v[j].first;
        wout[t * k + j] = normalize ? v[j].second / ts : v[j].second;
      }
    }
  }
}

// ops/attention.rs:9-34
void rope_tables(int rot_dim, int max_seq, double theta, float* cs, float* sn) {
  int half = rot_dim / 2;
  std::vector<float> inv(half);
  for (int i = 0; i < half; ++i) inv[i] = 1.0f / (float)std::pow(theta, 2.0 * (double)i / (double)rot_dim);
  for (int p = 0; p < max_seq; ++p)
    for (int i = 0; i < half; ++i) {
      float f = (float)p * inv[i];
      cs[(int64_t)p * half + i] = std::cos(f);
      sn[(int64_t)p * half + i] = std::sin(f);
    }
}

// ops/attention.rs:96-118: half-rotate RoPE of one head vector (first rot_dim dims)
void rope_apply(float* x, int rot_dim, const float* c, const float* s) {
  int half = rot_dim / 2;
  for (int i = 0; i < half; ++i) {
    float x1 = x[i], x2 = x[i + half];
    float r1 = x1 * c[i] - x2 * s[i];
    float r2 = x2 * c[i] + x1 * s[i];
    x[i] = r1; x[i + half] = r2;
  }
}

// ---------------------------------------------------------------------------
// MoE FFN (layer.rs:756-1895, default f32 path)
// Router entropy (layer.rs:2302-2325): Shannon entropy of softmax(logits) per token, averaged over
// the tokens of the call; exp and ln rounded from double, sums in double rounded once.
float router_entropy(const float* logits, int n_tok, int E) {
  double total = 0.0;
  for (int t = 0; t < n_tok; ++t) {
    const float* row = logits + (size_t)t * E;
    float mx = -INFINITY;
    for (int e = 0; e < E; ++e) mx = std::max(mx, row[e]);
    std::vector<float> ex(E);
    double s64 = 0.0;
    for (int e = 0; e < E; ++e) { ex[e] = expcr(row[e] - mx); s64 += ex[e]; }
    const float s = round_f32(s64);
    double h64 = 0.0;
    for (int e = 0; e < E; ++e) {
      const float p = ex[e] / s;
      if (p > 0.0f) h64 += (double)(p * (float)std::log((double)p));
    }
    total += (double)(-round_f32(h64));
  }
  return round_f32(total) / (float)n_tok;
}

// entropy_to_k (layer.rs:2329-2334): linear map of entropy / ln(E) onto [k_min, k_max], rounded
int entropy_to_k(float entropy, int E, int k_min, int k_max) {
  const float h_max = (float)std::log((double)E);
  const float norm = std::min(std::max(entropy / h_max, 0.0f), 1.0f);
  const float k = (float)k_min + norm * (float)(k_max - k_min);
  return std::min(std::max((int)std::round(k), k_min), k_max);
}

int moe_forward(const orc_moe_layer* L, const float* x, int n_tok, float* out, int32_t* idx_out, float* w_out,
                const std::vector<int>* dummies, int threads, int e_begin = 0, int e_end = 1 << 30,
                float* last_logits = nullptr, int dk_min = 0, int dk_max = 0, float* ent_out = nullptr,
                int* k_out = nullptr) {
  const int H = L->hidden, I = L->inter, E = L->n_experts, Kslots = L->top_k;
  std::vector<float> logits((size_t)n_tok * E);
  matmul_xwt(x, n_tok, L->router_w, E, H, logits.data(), threads);       // layer.rs:818-820
  if (L->router_b)                                                       // layer.rs:832-837
    for (int t = 0; t < n_tok; ++t) for (int e = 0; e < E; ++e) logits[(size_t)t * E + e] += L->router_b[e];
  // entropy before the dummy mask; dynamic K from it (layer.rs:980-1011): one K for the call
  int K = Kslots;
  if (ent_out || dk_max > 0) {
    const float ent = router_entropy(logits.data(), n_tok, E);
    if (ent_out) *ent_out = ent;
    if (dk_max > 0) K = entropy_to_k(ent, E, dk_min, dk_max);
  }
  if (k_out) *k_out = K;
  if (dummies)                                                           // layer.rs:1016-1026
    for (int t = 0; t < n_tok; ++t) for (int d : *dummies) logits[(size_t)t * E + d] += -INFINITY;
  if (last_logits) std::memcpy(last_logits, &logits[(size_t)(n_tok - 1) * E], (size_t)E * 4);
  std::vector<int32_t> idx((size_t)n_tok * K); std::vector<float> wts((size_t)n_tok * K);
  top_k_routing(logits.data(), n_tok, E, K, L->norm_topk_prob != 0, L->oai_swiglu != 0, idx.data(), wts.data());
  // [n_tok][slots] outputs; slots beyond a dynamic K hold expert id E (none) and weight 0
  for (int t = 0; t < n_tok; ++t)
    for (int j = 0; j < Kslots; ++j) {
      if (idx_out) idx_out[(size_t)t * Kslots + j] = j < K ? idx[(size_t)t * K + j] : E;
      if (w_out) w_out[(size_t)t * Kslots + j] = j < K ? wts[(size_t)t * K + j] : 0.0f;
    }
  // expert -> [(token, weight)] in (t, k) order; unique experts ascending (layer.rs:1092-1106)
  std::map<int, std::vector<std::pair<int, float>>> assign;
  for (int t = 0; t < n_tok; ++t)
    for (int j = 0; j < K; ++j) assign[idx[(size_t)t * K + j]].push_back({t, wts[(size_t)t * K + j]});
  std::memset(out, 0, sizeof(float) * (size_t)n_tok * H);
  const int64_t gsz = raw_size(L->gate_q, (int64_t)I * H), usz = raw_size(L->up_q, (int64_t)I * H),
                dsz = raw_size(L->down_q, (int64_t)H * I);
  std::vector<float> Wg((size_t)I * H), Wu((size_t)I * H), Wd((size_t)H * I);
  for (auto& kv : assign) {   // std::map iterates in ascending expert order (layer.rs:1797)
    const int e = kv.first; const auto& as = kv.second;
    if (e < e_begin || e >= e_end) continue;   // expert-parallel restriction (test decomposition)
    dequant_matrix(L->gate_q, (const uint8_t*)L->gate + e * gsz, I, H, Wg.data(), threads);  // layer.rs:1750-1762
    dequant_matrix(L->up_q, (const uint8_t*)L->up + e * usz, I, H, Wu.data(), threads);
    dequant_matrix(L->down_q, (const uint8_t*)L->down + e * dsz, H, I, Wd.data(), threads);
    const int n = (int)as.size();
    std::vector<float> xin((size_t)n * H);
    for (int i = 0; i < n; ++i) std::memcpy(&xin[(size_t)i * H], x + (size_t)as[i].first * H, H * 4);
    std::vector<float> g((size_t)n * I), u((size_t)n * I), a((size_t)n * I), o((size_t)n * H);
    matmul_xwt(xin.data(), n, Wg.data(), I, H, g.data(), threads);
    matmul_xwt(xin.data(), n, Wu.data(), I, H, u.data(), threads);
    for (int i = 0; i < n; ++i) for (int r = 0; r < I; ++r) {
      if (L->gate_bias) g[(size_t)i * I + r] += L->gate_bias[(size_t)e * I + r];
      if (L->up_bias) u[(size_t)i * I + r] += L->up_bias[(size_t)e * I + r];
    }
    if (L->oai_swiglu) swiglu_oai(g.data(), u.data(), a.data(), (int64_t)n * I, 1.702f, 7.0f);
    else silu_and_mul(g.data(), u.data(), a.data(), (int64_t)n * I);
    matmul_xwt(a.data(), n, Wd.data(), H, I, o.data(), threads);
    for (int i = 0; i < n; ++i) {
      float* oi = &o[(size_t)i * H];
      if (L->down_bias) for (int r = 0; r < H; ++r) oi[r] += L->down_bias[(size_t)e * H + r];
      float* dst = out + (size_t)as[i].first * H;
      const float w = as[i].second;   // single token: layer.rs:1816,1845; multi: 1883-1893
      for (int r = 0; r < H; ++r) dst[r] += oi[r] * w;
    }
  }
  return 0;
}

// ---------------------------------------------------------------------------
// GGUF (reader.rs:259-368)
struct GTensor { int qtype = 0; std::vector<int64_t> shape; const uint8_t* data = nullptr; int64_t nbytes = 0; };
struct MetaVal { int type = 0; uint64_t u = 0; int64_t i = 0; double f = 0; std::string s; };

struct Reader {
  const uint8_t* base = nullptr; size_t size = 0, pos = 0; bool ok = true;
  bool need(size_t n) { if (pos + n > size) { ok = false; return false; } return true; }
  template <class T> T rd() { T v{}; if (need(sizeof(T))) { std::memcpy(&v, base + pos, sizeof(T)); pos += sizeof(T); } return v; }
  std::string str() {
    uint64_t n = rd<uint64_t>();
    if (!need(n)) return {};
    std::string s((const char*)base + pos, n); pos += n; return s;
  }
  void value(int type, MetaVal* mv, int depth = 0) {
    mv->type = type;
    switch (type) {
      case 0: mv->u = rd<uint8_t>(); mv->i = (int64_t)mv->u; mv->f = (double)mv->u; break;
      case 1: mv->i = rd<int8_t>(); mv->u = (uint64_t)mv->i; mv->f = (double)mv->i; break;
      case 2: mv->u = rd<uint16_t>(); mv->i = (int64_t)mv->u; mv->f = (double)mv->u; break;
      case 3: mv->i = rd<int16_t>(); mv->u = (uint64_t)mv->i; mv->f = (double)mv->i; break;
      case 4: mv->u = rd<uint32_t>(); mv->i = (int64_t)mv->u; mv->f = (double)mv->u; break;
      case 5: mv->i = rd<int32_t>(); mv->u = (uint64_t)mv->i; mv->f = (double)mv->i; break;
      case 6: mv->f = rd<float>(); break;
      case 7: mv->u = rd<uint8_t>(); mv->i = (int64_t)mv->u; break;
      case 8: mv->s = str(); break;
      case 9: {
        int et = (int)rd<uint32_t>(); uint64_t n = rd<uint64_t>();
        if (depth > 4 || n > (1u << 28)) { ok = false; return; }
        MetaVal tmp;
        for (uint64_t k = 0; k < n && ok; ++k) value(et, &tmp, depth + 1);
        mv->u = n; break;
      }
      case 10: mv->u = rd<uint64_t>(); mv->i = (int64_t)mv->u; mv->f = (double)mv->u; break;
      case 11: mv->i = rd<int64_t>(); mv->u = (uint64_t)mv->i; mv->f = (double)mv->i; break;
      case 12: mv->f = rd<double>(); break;
      default: ok = false;
    }
  }
};

struct Gguf {
  void* map = nullptr; size_t size = 0;
  std::map<std::string, MetaVal> meta;
  std::map<std::string, GTensor> tensors;
  ~Gguf() { if (map) munmap(map, size); }
  bool open(const char* path, std::string* err) {
    int fd = ::open(path, O_RDONLY);
    if (fd < 0) { *err = std::string("cannot open ") + path; return false; }
    struct stat st; fstat(fd, &st); size = (size_t)st.st_size;
    map = mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0); ::close(fd);
    if (map == MAP_FAILED) { map = nullptr; *err = "mmap failed"; return false; }
    Reader r; r.base = (const uint8_t*)map; r.size = size;
    if (r.rd<uint32_t>() != 0x46554747u) { *err = "invalid GGUF magic"; return false; }
    uint32_t ver = r.rd<uint32_t>();
    if (ver < 2 || ver > 3) { *err = "unsupported GGUF version"; return false; }
    uint64_t nt = r.rd<uint64_t>(), nm = r.rd<uint64_t>();
    if (nt > 1000000 || nm > 1000000) { *err = "absurd counts"; return false; }
    for (uint64_t i = 0; i < nm && r.ok; ++i) {
      std::string k = r.str(); int t = (int)r.rd<uint32_t>(); MetaVal v; r.value(t, &v); meta[k] = v;
    }
    struct TI { std::string n; std::vector<uint64_t> d; int q; uint64_t off; };
    std::vector<TI> tis;
    for (uint64_t i = 0; i < nt && r.ok; ++i) {
      TI ti; ti.n = r.str(); uint32_t nd = r.rd<uint32_t>();
      if (nd > 8) { *err = "too many dims"; return false; }
      for (uint32_t j = 0; j < nd; ++j) ti.d.push_back(r.rd<uint64_t>());
      ti.q = (int)r.rd<uint32_t>(); ti.off = r.rd<uint64_t>(); tis.push_back(ti);
    }
    if (!r.ok) { *err = "truncated GGUF header"; return false; }
    uint64_t align = 32;
    auto it = meta.find("general.alignment");
    if (it != meta.end() && it->second.u) align = it->second.u;
    uint64_t start = (r.pos + align - 1) / align * align;
    for (auto& ti : tis) {
      GTensor t; t.qtype = ti.q;
      int64_t n = 1;
      for (auto it2 = ti.d.rbegin(); it2 != ti.d.rend(); ++it2) { t.shape.push_back((int64_t)*it2); n *= (int64_t)*it2; }
      t.nbytes = raw_size(ti.q, n);
      if (t.nbytes < 0) continue;   // unsupported types are simply not indexed here
      uint64_t off = start + ti.off;
      if (off + (uint64_t)t.nbytes > size) { *err = "tensor out of bounds: " + ti.n; return false; }
      t.data = (const uint8_t*)map + off;
      tensors[ti.n] = t;
    }
    return true;
  }
  const GTensor* get(const std::string& n) const { auto it = tensors.find(n); return it == tensors.end() ? nullptr : &it->second; }
  int64_t u32(const std::string& k, int64_t def) const { auto it = meta.find(k); return it == meta.end() ? def : it->second.i; }
  double f32(const std::string& k, double def) const {
    auto it = meta.find(k); if (it == meta.end()) return def;
    return (it->second.type == 6 || it->second.type == 12) ? it->second.f : (double)it->second.i;
  }
  std::string str(const std::string& k, const std::string& def) const { auto it = meta.find(k); return it == meta.end() ? def : it->second.s; }
};

}  // namespace

// ---------------------------------------------------------------------------
struct orc_model {
  Gguf g;
  std::string arch;
  int hidden = 0, layers = 0, heads = 0, kv_heads = 0, head_dim = 0, rot_dim = 0;
  int experts = 0, top_k = 0, inter = 0, vocab = 0, sliding_window = 0, max_seq = 0;
  float rope_theta = 0, eps = 0; bool norm_topk = true, oai = false;
  int attn_mode = 1, threads = 0;
  int attn_interval = 0;   // full_attention_interval; > 0 = DeltaNet hybrid with gated attention
  std::vector<float> cos_t, sin_t;
  struct Layer {
    const float* attn_norm = nullptr; const float* post_norm = nullptr;
    const GTensor *q = nullptr, *k = nullptr, *v = nullptr, *o = nullptr;
    const float *qb = nullptr, *kb = nullptr, *vb = nullptr, *ob = nullptr, *sinks = nullptr, *qn = nullptr, *kn = nullptr;
    orc_moe_layer moe{};
    std::vector<int> dummies;
    std::vector<float> K, V;   // [kv_heads][seq][hd] grown per step (kv_cache.rs:37-60)
    // hybrid models (config.rs:446-458): a layer is attention or Gated DeltaNet
    bool is_attn = true;
    orc_deltanet_layer dn{};
    std::vector<uint8_t> ba_cat;                     // split ssm_beta / ssm_alpha rows joined (beta first)
    std::vector<float> conv_state, rec_state;        // DeltaNetState (deltanet.rs:139-196), zero at start
    // shared expert (layer.rs:1898-1953, 2250-2293)
    const GTensor *sh_gate = nullptr, *sh_up = nullptr, *sh_down = nullptr;
    const float* sh_gate_inp = nullptr;
    int dk_lo = 0, dk_hi = 0;   // dynamic K range of this layer (0, 0: fixed top_k)
  };
  std::vector<Layer> L;
  const GTensor *embd = nullptr, *out = nullptr; const float* out_norm = nullptr; const float* out_bias = nullptr;
  int seq = 0;
  std::vector<float> last_hidden; std::vector<int32_t> last_idx; std::vector<float> last_w;
  // per layer, last position of the last forward: residual stream after the layer [layers][H]
  // and the router logits after bias and dummy mask [layers][E] (test diagnostics)
  std::vector<float> layer_hidden, layer_logits;
  // router entropy and the K used, per layer, of the last forward (layer.rs:980-1011)
  std::vector<float> last_entropy;
  std::vector<int> last_k;
};

namespace {
const float* f32p(const GTensor* t) { return t && t->qtype == ORC_F32 ? (const float*)t->data : nullptr; }

// one projection y = x W^T for n tokens, with the model's attention numerics
void project(orc_model* m, const GTensor* W, const float* x, int n, float* y) {
  int64_t rows = W->shape[0], cols = W->shape[1];
  int th = m->threads ? m->threads : hw_threads();
  if (W->qtype == ORC_Q8_0 && m->attn_mode == 1) { q8_0_gemv_actq(W->data, rows, cols, x, y, th, n); return; }
  std::vector<float> Wf((size_t)rows * cols);
  dequant_matrix(W->qtype, W->data, rows, cols, Wf.data(), th);
  matmul_xwt(x, n, Wf.data(), rows, cols, y, th);
}

// ops/attention.rs:178-280.  q: [seq_q][nh][hd]; K,V: [nkv][seq_k][hd]; out: [seq_q][nh][hd]
void sdpa(const float* q, const float* K, const float* V, int nh, int nkv, int n, int Lk, int hd, float scale,
          bool causal, const float* sinks, int sw, float* attn, int th) {
  const int rep = nh / nkv;
  parallel_for((int64_t)n * nh, th, [&](int64_t b, int64_t e) {
    std::vector<float> sc(Lk);
    for (int64_t id = b; id < e; ++id) {
      int t = (int)(id / nh), h = (int)(id % nh), kvh = h / rep;
      const float* qv = &q[((size_t)t * nh + h) * hd];
      const int qabs = (Lk - n) + t;
      float mx = -INFINITY;
      for (int j = 0; j < Lk; ++j) {
        const float* kv = &K[((size_t)kvh * Lk + j) * hd];
        double dot = 0.0;
        for (int d = 0; d < hd; ++d) dot += (double)qv[d] * (double)kv[d];
        float s = round_f32(dot) * scale + 0.0f;
        bool masked = (causal && j > qabs) || (sw > 0 && qabs - j >= sw);
        if (masked) s = -INFINITY;
        sc[j] = s; mx = std::max(mx, s);
      }
      float denom = 0.0f;
      double den64 = 0.0;
      if (sinks) {
        float sk = sinks[h];
        float mprime = ((mx + sk) + std::fabs(mx - sk)) * 0.5f;
        for (int j = 0; j < Lk; ++j) sc[j] = expcr(sc[j] - mprime);
        for (int j = 0; j < Lk; ++j) den64 += sc[j];
        denom = round_f32(den64) + expcr(sk - mprime);
      } else {
        for (int j = 0; j < Lk; ++j) sc[j] = expcr(sc[j] - mx);
        for (int j = 0; j < Lk; ++j) den64 += sc[j];
        denom = round_f32(den64);
      }
      std::vector<double> acc(hd, 0.0);
      for (int j = 0; j < Lk; ++j) {
        const float p = sc[j] / denom;
        if (p == 0.0f) continue;
        const float* vv = &V[((size_t)kvh * Lk + j) * hd];
        for (int d = 0; d < hd; ++d) acc[d] += (double)p * (double)vv[d];
      }
      float* o = &attn[((size_t)t * nh + h) * hd];
      for (int d = 0; d < hd; ++d) o[d] = round_f32(acc[d]);
    }
  });
}

// layer.rs:511-749 for n tokens at positions [seq, seq+n)
void attention(orc_model* m, orc_model::Layer& Ly, int li, const float* x, int n, float* out) {
  const int H = m->hidden, nh = m->heads, nkv = m->kv_heads, hd = m->head_dim;
  std::vector<float> q((size_t)n * nh * hd), k((size_t)n * nkv * hd), v((size_t)n * nkv * hd), gate;
  const bool gated = m->attn_interval > 0;   // hybrid models: Q projection = [Q_h, gate_h] per head
  if (gated) {                               // (layer.rs:620-635)
    const size_t Dq = (size_t)nh * hd;
    std::vector<float> qg((size_t)n * 2 * Dq);
    project(m, Ly.q, x, n, qg.data());
    if (Ly.qb) for (int t = 0; t < n; ++t) for (size_t i = 0; i < 2 * Dq; ++i) qg[t * 2 * Dq + i] += Ly.qb[i];
    gate.resize((size_t)n * Dq);
    for (int t = 0; t < n; ++t)
      for (int i = 0; i < nh; ++i)
        for (int d = 0; d < hd; ++d) {
          q[t * Dq + (size_t)i * hd + d] = qg[t * 2 * Dq + (size_t)i * 2 * hd + d];
          gate[t * Dq + (size_t)i * hd + d] = qg[t * 2 * Dq + (size_t)i * 2 * hd + hd + d];
        }
  } else {
    project(m, Ly.q, x, n, q.data());
  }
  project(m, Ly.k, x, n, k.data()); project(m, Ly.v, x, n, v.data());
  for (int t = 0; t < n; ++t) {
    if (Ly.qb && !gated) for (int i = 0; i < nh * hd; ++i) q[(size_t)t * nh * hd + i] += Ly.qb[i];
    if (Ly.kb) for (int i = 0; i < nkv * hd; ++i) k[(size_t)t * nkv * hd + i] += Ly.kb[i];
    if (Ly.vb) for (int i = 0; i < nkv * hd; ++i) v[(size_t)t * nkv * hd + i] += Ly.vb[i];
  }
  if (Ly.qn && Ly.kn) {    // layer.rs:643-650 QK-norm per head
    std::vector<float> tmp(hd);
    for (int t = 0; t < n * nh; ++t) { rms_norm(&q[(size_t)t * hd], Ly.qn, tmp.data(), 1, hd, m->eps); std::memcpy(&q[(size_t)t * hd], tmp.data(), hd * 4); }
    for (int t = 0; t < n * nkv; ++t) { rms_norm(&k[(size_t)t * hd], Ly.kn, tmp.data(), 1, hd, m->eps); std::memcpy(&k[(size_t)t * hd], tmp.data(), hd * 4); }
  }
  const int half = m->rot_dim / 2, p0 = m->seq;
  for (int t = 0; t < n; ++t) {      // layer.rs:654-664 RoPE at position_offset = cached length
    const float* c = &m->cos_t[(size_t)(p0 + t) * half]; const float* s = &m->sin_t[(size_t)(p0 + t) * half];
    for (int h = 0; h < nh; ++h) rope_apply(&q[((size_t)t * nh + h) * hd], m->rot_dim, c, s);
    for (int h = 0; h < nkv; ++h) rope_apply(&k[((size_t)t * nkv + h) * hd], m->rot_dim, c, s);
  }
  const int Lk = p0 + n;             // kv_cache.rs:37-60 append
  std::vector<float> K2((size_t)nkv * Lk * hd), V2((size_t)nkv * Lk * hd);
  for (int h = 0; h < nkv; ++h) {
    if (p0) {
      std::memcpy(&K2[(size_t)h * Lk * hd], &Ly.K[(size_t)h * p0 * hd], (size_t)p0 * hd * 4);
      std::memcpy(&V2[(size_t)h * Lk * hd], &Ly.V[(size_t)h * p0 * hd], (size_t)p0 * hd * 4);
    }
    for (int t = 0; t < n; ++t) {
      std::memcpy(&K2[((size_t)h * Lk + p0 + t) * hd], &k[((size_t)t * nkv + h) * hd], hd * 4);
      std::memcpy(&V2[((size_t)h * Lk + p0 + t) * hd], &v[((size_t)t * nkv + h) * hd], hd * 4);
    }
  }
  Ly.K.swap(K2); Ly.V.swap(V2);
  // ops/attention.rs:178-280
  const float scale = (float)(1.0 / std::sqrt((double)hd));
  const int sw = (m->sliding_window > 0 && li % 2 == 0) ? m->sliding_window : 0;   // config.rs:463-465
  std::vector<float> attn((size_t)n * nh * hd);
  sdpa(q.data(), Ly.K.data(), Ly.V.data(), nh, nkv, n, Lk, hd, scale, n > 1, Ly.sinks, sw, attn.data(),
       m->threads ? m->threads : hw_threads());
  if (gated)   // attn_out *= sigmoid(gate), sigmoid = recip(exp(-x) + 1) (layer.rs:699-705, activation.rs:41-45)
    for (size_t i = 0; i < attn.size(); ++i) attn[i] = attn[i] * (1.0f / (expcr(-gate[i]) + 1.0f));
  project(m, Ly.o, attn.data(), n, out);                     // layer.rs:709-730
  if (Ly.ob) for (int t = 0; t < n; ++t) for (int i = 0; i < H; ++i) out[(size_t)t * H + i] += Ly.ob[i];
}
}  // namespace

extern "C" {

float orc_fp16_to_f32(uint16_t h) { return h2f(h); }
float orc_e8m0_to_f32_half(uint8_t e) { return e8m0_half(e); }
int orc_dequantize(int qtype, const void* blocks, int64_t n, float* out) { return dequant(qtype, blocks, n, out); }

void orc_mxfp4_matvec_mul(const uint8_t* w, const float* x, int64_t rows, int64_t cols, float* y) {
  // dequant.rs:640-695: per row, sequential over blocks then j, lo then hi
  int64_t nb = cols / 32, rb = nb * 17;
  parallel_for(rows, hw_threads(), [&](int64_t b, int64_t e) {
    for (int64_t r = b; r < e; ++r) {
      float acc = 0.0f;
      for (int64_t k = 0; k < nb; ++k) {
        const uint8_t* blk = w + r * rb + k * 17;
        float d = e8m0_half(blk[0]);
        for (int j = 0; j < 16; ++j) {
          float lo = kMxfp4Values[blk[1 + j] & 0x0f], hi = kMxfp4Values[blk[1 + j] >> 4];
          acc += lo * d * x[k * 32 + j];
          acc += hi * d * x[k * 32 + j + 16];
        }
      }
      y[r] = acc;
    }
  });
}

int orc_gemv(int qtype, const void* w, int64_t rows, int64_t cols, const float* x, float* y) {
  QInfo qi; if (!qinfo(qtype, &qi)) return -1;
  std::vector<float> W((size_t)rows * cols);
  dequant_matrix(qtype, w, rows, cols, W.data(), hw_threads());
  matmul_xwt(x, 1, W.data(), rows, cols, y, hw_threads());
  return 0;
}

void orc_q8_0_gemv(const uint8_t* w, int64_t rows, int64_t cols, const float* x, float* y, int mode) {
  if (mode == 1) { q8_0_gemv_actq(w, rows, cols, x, y, hw_threads()); return; }
  orc_gemv(ORC_Q8_0, w, rows, cols, x, y);
}
int orc_moe_forward_range(const orc_moe_layer* L, const float* x, int n_tok, float* out, int e_begin, int e_end) {
  return moe_forward(L, x, n_tok, out, nullptr, nullptr, nullptr, hw_threads(), e_begin, e_end);
}
void orc_sdpa(const float* q, const float* k, const float* v, int nh, int nkv, int seq_q, int seq_k, int hd,
              double scale, int causal, const float* sinks, int sliding_window, float* out) {
  sdpa(q, k, v, nh, nkv, seq_q, seq_k, hd, (float)scale, causal != 0, sinks, sliding_window, out, 1);
}
void orc_quantize_q8_0(const float* x, int64_t n, uint8_t* out) { quantize_q8_0(x, n, out); }
void orc_rms_norm(const float* x, const float* w, float* y, int64_t rows, int64_t dim, float eps) { rms_norm(x, w, y, rows, dim, eps); }
void orc_rope_tables(int rot_dim, int max_seq, double theta, float* c, float* s) { rope_tables(rot_dim, max_seq, theta, c, s); }
void orc_swiglu_oai(const float* g, const float* u, float* out, int64_t n, float alpha, float limit) { swiglu_oai(g, u, out, n, alpha, limit); }
void orc_silu_and_mul(const float* g, const float* u, float* out, int64_t n) { silu_and_mul(g, u, out, n); }
void orc_top_k_routing(const float* logits, int n_tok, int n_exp, int k, int normalize, int softmax_weight, int32_t* idx, float* w) {
  top_k_routing(logits, n_tok, n_exp, k, normalize != 0, softmax_weight != 0, idx, w);
}
int orc_moe_forward(const orc_moe_layer* L, const float* x, int n_tok, float* out, int32_t* idx_out, float* w_out) {
  return moe_forward(L, x, n_tok, out, idx_out, w_out, nullptr, hw_threads());
}

void orc_rope(const float* x, const float* cs, const float* sn, int n_tok, int heads, int hd, int rot, float* y) {
  const int half = rot / 2;
  std::memcpy(y, x, sizeof(float) * (size_t)n_tok * heads * hd);
  for (int t = 0; t < n_tok; ++t)
    for (int h = 0; h < heads; ++h) rope_apply(&y[((size_t)t * heads + h) * hd], rot, &cs[(size_t)t * half], &sn[(size_t)t * half]);
}

// layer.rs:511-749 for one decode token, outside a model: the same steps as attention() above
int orc_attn_decode(const orc_attn_layer* L, float* K, float* V, int pos, float* h) {
  const int H = L->hidden, nh = L->heads, nkv = L->kv_heads, hd = L->head_dim, Dq = nh * hd, Dkv = nkv * hd;
  const int th = hw_threads();
  std::vector<float> xn(H), q(Dq), k(Dkv), v(Dkv), attn(Dq), o(H), gate;
  rms_norm(h, L->attn_norm, xn.data(), 1, H, L->eps);
  auto proj = [&](const uint8_t* w, int rows, int cols, const float* x, float* y) {
    if (L->attn_mode == 1) { q8_0_gemv_actq(w, rows, cols, x, y, th); return; }
    std::vector<float> Wf((size_t)rows * cols);
    dequant_matrix(ORC_Q8_0, w, rows, cols, Wf.data(), th);
    matmul_xwt(x, 1, Wf.data(), rows, cols, y, th);
  };
  if (L->q_gate) {   // hybrid models: per head [Q_h, gate_h] interleaved (layer.rs:620-635)
    std::vector<float> qg(2 * (size_t)Dq);
    proj(L->wq, 2 * Dq, H, xn.data(), qg.data());
    if (L->bq) for (int i = 0; i < 2 * Dq; ++i) qg[i] += L->bq[i];
    gate.resize(Dq);
    for (int i = 0; i < nh; ++i)
      for (int d = 0; d < hd; ++d) {
        q[(size_t)i * hd + d] = qg[(size_t)i * 2 * hd + d];
        gate[(size_t)i * hd + d] = qg[(size_t)i * 2 * hd + hd + d];
      }
  } else {
    proj(L->wq, Dq, H, xn.data(), q.data());
    if (L->bq) for (int i = 0; i < Dq; ++i) q[i] += L->bq[i];
  }
  proj(L->wk, Dkv, H, xn.data(), k.data()); proj(L->wv, Dkv, H, xn.data(), v.data());
  if (L->bk) for (int i = 0; i < Dkv; ++i) k[i] += L->bk[i];
  if (L->bv) for (int i = 0; i < Dkv; ++i) v[i] += L->bv[i];
  if (L->q_norm && L->k_norm) {
    std::vector<float> tmp(hd);
    for (int i = 0; i < nh; ++i) { rms_norm(&q[(size_t)i * hd], L->q_norm, tmp.data(), 1, hd, L->eps); std::memcpy(&q[(size_t)i * hd], tmp.data(), hd * 4); }
    for (int i = 0; i < nkv; ++i) { rms_norm(&k[(size_t)i * hd], L->k_norm, tmp.data(), 1, hd, L->eps); std::memcpy(&k[(size_t)i * hd], tmp.data(), hd * 4); }
  }
  const int half = L->rot_dim / 2;
  std::vector<float> cs((size_t)(pos + 1) * half), sn(cs.size());
  rope_tables(L->rot_dim, pos + 1, (double)L->rope_theta, cs.data(), sn.data());
  for (int i = 0; i < nh; ++i) rope_apply(&q[(size_t)i * hd], L->rot_dim, &cs[(size_t)pos * half], &sn[(size_t)pos * half]);
  for (int i = 0; i < nkv; ++i) rope_apply(&k[(size_t)i * hd], L->rot_dim, &cs[(size_t)pos * half], &sn[(size_t)pos * half]);
  const int Lk = pos + 1;   // caches hold [nkv][Lk][hd]; rows < pos were written by earlier calls
  for (int i = 0; i < nkv; ++i) {
    std::memcpy(&K[((size_t)i * Lk + pos) * hd], &k[(size_t)i * hd], hd * 4);
    std::memcpy(&V[((size_t)i * Lk + pos) * hd], &v[(size_t)i * hd], hd * 4);
  }
  const float scale = (float)(1.0 / std::sqrt((double)hd));
  sdpa(q.data(), K, V, nh, nkv, 1, Lk, hd, scale, false, L->sinks, L->window, attn.data(), th);
  if (L->q_gate)   // attn_out *= sigmoid(gate), sigmoid = recip(exp(-x) + 1) (layer.rs:699-705, activation.rs:41-45)
    for (int i = 0; i < Dq; ++i) attn[i] = attn[i] * (1.0f / (expcr(-gate[i]) + 1.0f));
  proj(L->wo, H, Dq, attn.data(), o.data());
  for (int i = 0; i < H; ++i) h[i] = h[i] + (L->bo ? o[i] + L->bo[i] : o[i]);
  return 0;
}

orc_model* orc_model_open(const char* path, int max_seq_len, char* err, int err_len) {
  auto* m = new orc_model();
  std::string e;
  auto fail = [&](const std::string& msg) -> orc_model* {
    if (err && err_len > 0) { std::snprintf(err, err_len, "%s", msg.c_str()); }
    delete m; return nullptr;
  };
  if (!m->g.open(path, &e)) return fail(e);
  Gguf& g = m->g;
  // config.rs:253-434 (keys and defaults)
  m->arch = g.str("general.architecture", "qwen2moe");
  const std::string a = m->arch;
  m->hidden = (int)g.u32(a + ".embedding_length", 2048);
  m->layers = (int)g.u32(a + ".block_count", 48);
  m->heads = (int)g.u32(a + ".attention.head_count", 16);
  m->kv_heads = (int)g.u32(a + ".attention.head_count_kv", 2);
  m->head_dim = (int)g.u32(a + ".attention.key_length", m->hidden / m->heads);
  m->experts = (int)g.u32(a + ".expert_count", 128);
  m->top_k = (int)g.u32(a + ".expert_used_count", 8);
  m->rope_theta = (float)g.f32(a + ".rope.freq_base", 1000000.0);
  m->eps = (float)g.f32(a + ".attention.layer_norm_rms_epsilon", 1e-6);
  const GTensor* te = g.get("token_embd.weight");
  m->vocab = (int)g.u32(a + ".vocab_size", te ? te->shape[0] : 151936);
  const GTensor* ge = g.get("blk.0.ffn_gate_exps.weight");
  m->inter = (int)g.u32(a + ".expert_feed_forward_length", ge && ge->shape.size() >= 3 ? ge->shape[1] : 768);
  m->sliding_window = (int)g.u32(a + ".attention.sliding_window", 0);
  double prf = g.f32(a + ".rope.partial_rotary_factor", -1.0);
  if (prf < 0) {
    int64_t dc = g.u32(a + ".rope.dimension_count", -1);
    prf = dc >= 0 ? (double)((float)dc / (float)m->head_dim) : 1.0;
  }
  m->rot_dim = (int)((float)m->head_dim * (float)prf);
  std::string name = g.str("general.name", "");
  m->norm_topk = !(name.find("Qwen1.5") != std::string::npos || name.find("Qwen2") != std::string::npos);
  m->oai = (a == "gpt-oss");
  // config.rs:318-352: SSM tensors make a DeltaNet hybrid (every attn_interval-th layer attention)
  const bool has_ssm = g.get("blk.0.ssm_a") || g.get("blk.0.ssm_conv1d.weight");
  m->attn_interval = (int)g.u32(a + ".attention.full_attention_interval", has_ssm ? 4 : 0);
  const int dn_nk = (int)g.u32(a + ".ssm.group_count", 16), dn_hkd = (int)g.u32(a + ".ssm.state_size", 128);
  int dn_nv = (int)g.u32(a + ".ssm.time_step_rank", -1);
  if (dn_nv < 0) dn_nv = (int)g.u32(a + ".ssm.dt_rank", 32);
  const int dn_inner = (int)g.u32(a + ".ssm.inner_size", 4096), dn_ks = (int)g.u32(a + ".ssm.conv_kernel", 4);
  const int dn_hvd = dn_nv == 0 ? 128 : dn_inner / dn_nv;   // config.rs:486-488
  m->max_seq = max_seq_len;
  m->cos_t.resize((size_t)max_seq_len * (m->rot_dim / 2)); m->sin_t.resize(m->cos_t.size());
  rope_tables(m->rot_dim, max_seq_len, (double)m->rope_theta, m->cos_t.data(), m->sin_t.data());
  m->embd = g.get("token_embd.weight"); m->out = g.get("output.weight");
  m->out_norm = f32p(g.get("output_norm.weight")); m->out_bias = f32p(g.get("output.bias"));
  if (!m->embd || !m->out || !m->out_norm) return fail("missing token_embd/output/output_norm");
  m->L.resize(m->layers);
  for (int li = 0; li < m->layers; ++li) {
    auto& Ly = m->L[li];
    std::string p = "blk." + std::to_string(li) + ".";
    Ly.attn_norm = f32p(g.get(p + "attn_norm.weight"));
    Ly.post_norm = f32p(g.get(p + "post_attention_norm.weight"));
    if (!Ly.post_norm) Ly.post_norm = f32p(g.get(p + "ffn_norm.weight"));
    if (!Ly.attn_norm || !Ly.post_norm) return fail("missing norm tensors in " + p);
    // config.rs:452-458: with an interval, layer li is attention when (li + 1) % interval == 0
    Ly.is_attn = m->attn_interval == 0 || (li + 1) % m->attn_interval == 0;
    if (!Ly.is_attn) {   // Gated DeltaNet layer, split (Unsloth) tensor format (deltanet.rs:101-137)
      auto& D = Ly.dn;
      D.hidden = m->hidden; D.n_k_heads = dn_nk; D.head_k_dim = dn_hkd; D.n_v_heads = dn_nv; D.head_v_dim = dn_hvd;
      D.conv_kernel = dn_ks; D.eps = m->eps;
      const GTensor *qkv = g.get(p + "attn_qkv.weight"), *z = g.get(p + "attn_gate.weight"),
                    *ba = g.get(p + "ssm_ba.weight"), *out = g.get(p + "ssm_out.weight");
      if (!qkv || !z || !out) return fail("missing DeltaNet projections in " + p + " (the split attn_qkv format is required)");
      D.qkv_q = qkv->qtype; D.qkv = qkv->data; D.gate_q = z->qtype; D.gate = z->data;
      D.out_q = out->qtype; D.out = out->data;
      if (ba) { D.ba_q = ba->qtype; D.ba = ba->data; }
      else {   // ssm_beta + ssm_alpha rows, beta first (deltanet.rs:118-125)
        const GTensor *bt = g.get(p + "ssm_beta.weight"), *at = g.get(p + "ssm_alpha.weight");
        if (!bt || !at || bt->qtype != at->qtype) return fail("missing ssm_ba / ssm_beta + ssm_alpha in " + p);
        Ly.ba_cat.assign(bt->data, bt->data + bt->nbytes);
        Ly.ba_cat.insert(Ly.ba_cat.end(), at->data, at->data + at->nbytes);
        D.ba_q = bt->qtype; D.ba = Ly.ba_cat.data();
      }
      D.conv1d = f32p(g.get(p + "ssm_conv1d.weight")); D.ssm_a = f32p(g.get(p + "ssm_a"));
      D.dt_bias = f32p(g.get(p + "ssm_dt.bias")); D.norm = f32p(g.get(p + "ssm_norm.weight"));
      if (!D.conv1d || !D.ssm_a || !D.dt_bias || !D.norm) return fail("missing DeltaNet f32 tensors in " + p);
      const int conv_dim = 2 * dn_nk * dn_hkd + dn_nv * dn_hvd;   // config.rs:492-494
      Ly.conv_state.assign((size_t)conv_dim * (dn_ks - 1), 0.0f);
      Ly.rec_state.assign((size_t)dn_nv * dn_hkd * dn_hvd, 0.0f);
    } else {
      Ly.q = g.get(p + "attn_q.weight"); Ly.k = g.get(p + "attn_k.weight");
      Ly.v = g.get(p + "attn_v.weight"); Ly.o = g.get(p + "attn_output.weight");
      if (!Ly.q || !Ly.k || !Ly.v || !Ly.o) return fail("missing attention tensors in " + p);
    }
    Ly.sh_gate = g.get(p + "ffn_gate_shexp.weight"); Ly.sh_up = g.get(p + "ffn_up_shexp.weight");
    Ly.sh_down = g.get(p + "ffn_down_shexp.weight"); Ly.sh_gate_inp = f32p(g.get(p + "ffn_gate_inp_shexp.weight"));
    if ((Ly.sh_gate || Ly.sh_up || Ly.sh_down) && !(Ly.sh_gate && Ly.sh_up && Ly.sh_down))
      return fail("incomplete shared expert in " + p);
    Ly.qb = f32p(g.get(p + "attn_q.bias")); Ly.kb = f32p(g.get(p + "attn_k.bias"));
    Ly.vb = f32p(g.get(p + "attn_v.bias")); Ly.ob = f32p(g.get(p + "attn_output.bias"));
    Ly.sinks = f32p(g.get(p + "attn_sinks.weight"));
    Ly.qn = f32p(g.get(p + "attn_q_norm.weight")); Ly.kn = f32p(g.get(p + "attn_k_norm.weight"));
    auto& M = Ly.moe;
    const GTensor *gt = g.get(p + "ffn_gate_exps.weight"), *ut = g.get(p + "ffn_up_exps.weight"),
                  *dt = g.get(p + "ffn_down_exps.weight"), *rw = g.get(p + "ffn_gate_inp.weight");
    if (!gt || !ut || !dt || !rw || rw->qtype != ORC_F32) return fail("missing MoE tensors in " + p);
    M.hidden = m->hidden; M.inter = (int)gt->shape[1]; M.n_experts = (int)rw->shape[0]; M.top_k = m->top_k;
    M.gate_q = gt->qtype; M.up_q = ut->qtype; M.down_q = dt->qtype;
    M.gate = gt->data; M.up = ut->data; M.down = dt->data;
    M.gate_bias = f32p(g.get(p + "ffn_gate_exps.bias")); M.up_bias = f32p(g.get(p + "ffn_up_exps.bias"));
    M.down_bias = f32p(g.get(p + "ffn_down_exps.bias"));
    M.router_w = (const float*)rw->data; M.router_b = f32p(g.get(p + "ffn_gate_inp.bias"));
    M.oai_swiglu = m->oai ? 1 : 0; M.norm_topk_prob = m->norm_topk ? 1 : 0;
    // engine.rs:628-652 dummy expert detection (constant router row within 1e-6)
    for (int e2 = 0; e2 < M.n_experts; ++e2) {
      const float* row = M.router_w + (size_t)e2 * m->hidden; bool uni = true;
      for (int i = 0; i < m->hidden && uni; ++i) uni = std::fabs(row[i] - row[0]) < 1e-6f;
      if (uni) Ly.dummies.push_back(e2);
    }
  }
  return m;
}

void orc_model_set_attn_mode(orc_model* m, int mode) { m->attn_mode = mode; }

// Dynamic K (config.rs:183-192, 468-483; LayerTierConfig::default_for_k, config.rs:86-106): per layer
// the range [k_min, k_max], or with layer_adaptive the depth tier's range for k_max.
int orc_model_set_dynamic_k(orc_model* m, int enable, int k_min, int k_max, int layer_adaptive) {
  if (!enable) { for (auto& l : m->L) l.dk_lo = l.dk_hi = 0; return 0; }
  if (k_min < 1 || k_max < k_min || k_max > m->top_k) return -1;
  const int two_thirds = std::min(std::max(k_max * 2 / 3, 4), k_max);
  for (int li = 0; li < m->layers; ++li) {
    int lo = k_min, hi = k_max;
    if (layer_adaptive) {
      const float depth = (float)li / (float)m->layers;
      if (depth < 0.15f) { lo = k_max; hi = k_max; }
      else if (depth < 0.85f) { lo = std::min(4, k_max); hi = two_thirds; }
      else { lo = two_thirds; hi = k_max; }
    }
    m->L[li].dk_lo = lo; m->L[li].dk_hi = hi;
  }
  return 0;
}

void orc_model_router_stats(const orc_model* m, float* entropy, int32_t* k) {
  for (int li = 0; li < m->layers; ++li) {
    if (entropy) entropy[li] = m->last_entropy.empty() ? 0.0f : m->last_entropy[li];
    if (k) k[li] = m->last_k.empty() ? 0 : m->last_k[li];
  }
}
void orc_model_set_threads(orc_model* m, int n) { m->threads = n; }
int orc_model_vocab(const orc_model* m) { return m->vocab; }
int orc_model_hidden(const orc_model* m) { return m->hidden; }
int orc_model_seq_len(const orc_model* m) { return m->seq; }
void orc_model_clear_cache(orc_model* m) {
  for (auto& l : m->L) {
    l.K.clear(); l.V.clear();
    std::fill(l.conv_state.begin(), l.conv_state.end(), 0.0f);
    std::fill(l.rec_state.begin(), l.rec_state.end(), 0.0f);
  }
  m->seq = 0;
}
void orc_model_destroy(orc_model* m) { delete m; }
void orc_model_last_hidden(const orc_model* m, float* o) { std::memcpy(o, m->last_hidden.data(), m->last_hidden.size() * 4); }
void orc_model_last_routing(const orc_model* m, int32_t* idx, float* w) {
  std::memcpy(idx, m->last_idx.data(), m->last_idx.size() * 4); std::memcpy(w, m->last_w.data(), m->last_w.size() * 4);
}

void orc_model_layer_trace(const orc_model* m, float* hidden, float* logits) {
  if (hidden) std::memcpy(hidden, m->layer_hidden.data(), m->layer_hidden.size() * 4);
  if (logits) std::memcpy(logits, m->layer_logits.data(), m->layer_logits.size() * 4);
}

// engine.rs:1963-1987: final RMSNorm + LM head (f16 weights converted exactly to f32)
static void lm_head(orc_model* m, const float* hidden, float* logits) {
  const int H = m->hidden;
  const int th = m->threads ? m->threads : hw_threads();
  std::vector<float> last(H);
  rms_norm(hidden, m->out_norm, last.data(), 1, H, m->eps);
  const int64_t rb = raw_size(m->out->qtype, H);
  parallel_for(m->vocab, th, [&](int64_t b, int64_t e) {
    std::vector<float> row(H);
    for (int64_t r = b; r < e; ++r) {
      dequant(m->out->qtype, m->out->data + r * rb, H, row.data());
      double acc = 0.0;
      for (int i = 0; i < H; ++i) acc += (double)last[i] * (double)row[i];
      logits[r] = m->out_bias ? round_f32(acc) + m->out_bias[r] : round_f32(acc);
    }
  });
}

void orc_model_lm_head(orc_model* m, const float* hidden, float* logits) { lm_head(m, hidden, logits); }

// engine.rs:1869-2006
int orc_model_forward(orc_model* m, const int32_t* tokens, int n, float* logits) {
  if (n <= 0 || m->seq + n > m->max_seq) return -1;
  const int H = m->hidden, K = m->top_k;
  const int th = m->threads ? m->threads : hw_threads();
  std::vector<float> h((size_t)n * H), xn((size_t)n * H), tmp((size_t)n * H);
  int64_t erb = raw_size(m->embd->qtype, H);
  for (int t = 0; t < n; ++t) {            // engine.rs:1877 index_select + to f32
    if (tokens[t] < 0 || tokens[t] >= m->vocab) return -2;
    dequant(m->embd->qtype, m->embd->data + (int64_t)tokens[t] * erb, H, &h[(size_t)t * H]);
  }
  m->last_idx.assign((size_t)m->layers * K, 0); m->last_w.assign((size_t)m->layers * K, 0.0f);
  const int E = m->experts;
  m->layer_hidden.assign((size_t)m->layers * H, 0.0f); m->layer_logits.assign((size_t)m->layers * E, 0.0f);
  m->last_entropy.assign(m->layers, 0.0f); m->last_k.assign(m->layers, 0);
  std::vector<int32_t> idx((size_t)n * K); std::vector<float> w((size_t)n * K);
  for (int li = 0; li < m->layers; ++li) {  // layer.rs:393-503
    auto& Ly = m->L[li];
    rms_norm(h.data(), Ly.attn_norm, xn.data(), n, H, m->eps);
    if (Ly.is_attn) {
      attention(m, Ly, li, xn.data(), n, tmp.data());
    } else {   // DeltaNet: one token after another through the recurrent state (layer.rs:435-452)
      for (int t = 0; t < n; ++t)
        if (orc_deltanet_step(&Ly.dn, &xn[(size_t)t * H], Ly.conv_state.data(), Ly.rec_state.data(),
                              &tmp[(size_t)t * H]) != 0)
          return -3;
    }
    for (size_t i = 0; i < h.size(); ++i) h[i] = h[i] + tmp[i];
    rms_norm(h.data(), Ly.post_norm, xn.data(), n, H, m->eps);
    moe_forward(&Ly.moe, xn.data(), n, tmp.data(), idx.data(), w.data(), &Ly.dummies, th, 0, 1 << 30,
                &m->layer_logits[(size_t)li * E], Ly.dk_lo, Ly.dk_hi, &m->last_entropy[li], &m->last_k[li]);
    if (Ly.sh_gate)   // routed output + shared expert output (layer.rs:910-922), per token
      for (int t = 0; t < n; ++t)
        if (orc_shared_expert(Ly.sh_gate->qtype, Ly.sh_gate->data, Ly.sh_up->data, Ly.sh_down->qtype, Ly.sh_down->data,
                              Ly.sh_gate_inp, H, (int)Ly.sh_gate->shape[0], &xn[(size_t)t * H], &tmp[(size_t)t * H]) != 0)
          return -3;
    for (size_t i = 0; i < h.size(); ++i) h[i] = h[i] + tmp[i];
    std::memcpy(&m->layer_hidden[(size_t)li * H], &h[(size_t)(n - 1) * H], (size_t)H * 4);
    std::memcpy(&m->last_idx[(size_t)li * K], &idx[(size_t)(n - 1) * K], K * 4);
    std::memcpy(&m->last_w[(size_t)li * K], &w[(size_t)(n - 1) * K], K * 4);
  }
  m->seq += n;
  m->last_hidden.assign(h.end() - H, h.end());
  if (logits) lm_head(m, m->last_hidden.data(), logits);
  return 0;
}

// engine.rs:2011-2118: greedy argmax by stable descending sort == lowest index among maxima
static int argmax_stable(const float* v, int n) {
  int best = 0;
  for (int i = 1; i < n; ++i) if (v[i] > v[best]) best = i;
  return best;
}

int orc_model_generate(orc_model* m, const int32_t* prompt, int n_prompt, int max_new, int32_t* out) {
  orc_model_clear_cache(m);
  std::vector<float> logits(m->vocab);
  if (orc_model_forward(m, prompt, n_prompt, logits.data()) != 0) return -1;
  int32_t next = argmax_stable(logits.data(), m->vocab);
  int n_out = 0; out[n_out++] = next;
  for (int s = 0; s + 1 < max_new; ++s) {
    if (orc_model_forward(m, &next, 1, logits.data()) != 0) return -1;
    next = argmax_stable(logits.data(), m->vocab);
    out[n_out++] = next;
  }
  return n_out;
}

// ---- Gated DeltaNet, one decode token (model/deltanet.rs:204-543) ----
int orc_deltanet_step(const orc_deltanet_layer* L, const float* x, float* conv_state, float* rec_state, float* y) {
  const int nk = L->n_k_heads, hkd = L->head_k_dim, nv = L->n_v_heads, hvd = L->head_v_dim, ks = L->conv_kernel;
  const int vpk = nv / nk, q_total = nk * hkd, v_total = nv * hvd, conv_dim = 2 * q_total + v_total, H = L->hidden;
  std::vector<float> mixed(conv_dim), z(v_total), ba(2 * nv);
  // 1-3. input projections (dequantized f32 weights, deltanet.rs:237-245)
  if (orc_gemv(L->qkv_q, L->qkv, conv_dim, H, x, mixed.data())) return -1;
  if (orc_gemv(L->gate_q, L->gate, v_total, H, x, z.data())) return -1;
  if (orc_gemv(L->ba_q, L->ba, 2 * nv, H, x, ba.data())) return -1;
  // gates (deltanet.rs:298-310): alpha = ssm_a * softplus(alpha_log + dt_bias), beta = sigmoid
  std::vector<float> alpha(nv), beta(nv);
  for (int h = 0; h < nv; ++h) {
    const float ab = ba[nv + h] + L->dt_bias[h];
    alpha[h] = L->ssm_a[h] * std::log(1.0f + std::exp(ab));
    beta[h] = 1.0f / (1.0f + std::exp(-ba[h]));
  }
  // 4. depthwise causal conv1d + state shift + SiLU (deltanet.rs:340-372)
  std::vector<float> conv(conv_dim);
  for (int c = 0; c < conv_dim; ++c) {
    float* st = conv_state + (size_t)c * (ks - 1);
    const float* w = L->conv1d + (size_t)c * ks;
    float sum = 0.0f;
    for (int j = 0; j < ks - 1; ++j) sum += st[j] * w[j];
    sum += mixed[c] * w[ks - 1];
    conv[c] = sum;
    for (int j = 0; j + 1 < ks - 1; ++j) st[j] = st[j + 1];
    if (ks > 1) st[ks - 2] = mixed[c];
  }
  for (int c = 0; c < conv_dim; ++c) conv[c] = conv[c] / (1.0f + std::exp(-conv[c]));
  // 5-6. repeat-interleave to value heads, L2 norm of q (x 1/sqrt(hvd)) and k (deltanet.rs:379-417)
  std::vector<float> q((size_t)nv * hkd), k((size_t)nv * hkd);
  for (int g = 0; g < nk; ++g)
    for (int r = 0; r < vpk; ++r)
      for (int i = 0; i < hkd; ++i) {
        q[(size_t)(g * vpk + r) * hkd + i] = conv[(size_t)g * hkd + i];
        k[(size_t)(g * vpk + r) * hkd + i] = conv[(size_t)q_total + g * hkd + i];
      }
  const float scale = 1.0f / std::sqrt((float)hvd);
  for (int h = 0; h < nv; ++h) {
    float qs = 0.f, kss = 0.f;
    for (int i = 0; i < hkd; ++i) qs += q[(size_t)h * hkd + i] * q[(size_t)h * hkd + i];
    const float qn = std::max(std::sqrt(qs), L->eps);
    for (int i = 0; i < hkd; ++i) q[(size_t)h * hkd + i] = q[(size_t)h * hkd + i] / qn * scale;
    for (int i = 0; i < hkd; ++i) kss += k[(size_t)h * hkd + i] * k[(size_t)h * hkd + i];
    const float kn = std::max(std::sqrt(kss), L->eps);
    for (int i = 0; i < hkd; ++i) k[(size_t)h * hkd + i] /= kn;
  }
  // 7. delta rule (deltanet.rs:434-489)
  std::vector<float> o(v_total, 0.0f);
  for (int h = 0; h < nv; ++h) {
    float* S = rec_state + (size_t)h * hkd * hvd;
    const float decay = std::exp(alpha[h]);
    for (int i = 0; i < hkd * hvd; ++i) S[i] *= decay;
    std::vector<float> kv(hvd, 0.0f);
    for (int i = 0; i < hkd; ++i)
      for (int j = 0; j < hvd; ++j) kv[j] += k[(size_t)h * hkd + i] * S[(size_t)i * hvd + j];
    std::vector<float> delta(hvd);
    for (int j = 0; j < hvd; ++j) delta[j] = (conv[(size_t)2 * q_total + h * hvd + j] - kv[j]) * beta[h];
    for (int i = 0; i < hkd; ++i)
      for (int j = 0; j < hvd; ++j) S[(size_t)i * hvd + j] += k[(size_t)h * hkd + i] * delta[j];
    for (int i = 0; i < hkd; ++i)
      for (int j = 0; j < hvd; ++j) o[(size_t)h * hvd + j] += q[(size_t)h * hkd + i] * S[(size_t)i * hvd + j];
  }
  // 8-9. per-head RMSNorm x weight, x silu(z) (deltanet.rs:495-522)
  for (int h = 0; h < nv; ++h) {
    float sq = 0.f;
    for (int j = 0; j < hvd; ++j) sq += o[(size_t)h * hvd + j] * o[(size_t)h * hvd + j];
    const float rms = std::sqrt(sq / (float)hvd + L->eps);
    for (int j = 0; j < hvd; ++j) o[(size_t)h * hvd + j] = o[(size_t)h * hvd + j] / rms * L->norm[j];
  }
  for (int i = 0; i < v_total; ++i) o[i] *= z[i] / (1.0f + std::exp(-z[i]));
  // 10. output projection (deltanet.rs:527-534)
  return orc_gemv(L->out_q, L->out, H, v_total, o.data(), y);
}

// ---- shared expert (model/layer.rs:2250-2293): y += sigmoid(x . gate_inp) * (silu(x Wg) * (x Wu)) Wd ----
int orc_shared_expert(int gu_q, const void* gate, const void* up, int down_q, const void* down,
                      const float* gate_inp, int hidden, int inter, const float* x, float* y) {
  std::vector<float> g(inter), u(inter), a(inter), o(hidden);
  if (orc_gemv(gu_q, gate, inter, hidden, x, g.data())) return -1;
  if (orc_gemv(gu_q, up, inter, hidden, x, u.data())) return -1;
  silu_and_mul(g.data(), u.data(), a.data(), inter);
  if (orc_gemv(down_q, down, hidden, inter, a.data(), o.data())) return -1;
  float sig = 1.0f;
  if (gate_inp) {
    float d = 0.f;
    for (int i = 0; i < hidden; ++i) d += x[i] * gate_inp[i];
    sig = 1.0f / (1.0f + std::exp(-d));
  }
  for (int i = 0; i < hidden; ++i) y[i] += o[i] * sig;
  return 0;
}

// SamplingParams::sample (engine.rs:124-208).  The reference's f32 running sums of probabilities
// become sums of 128-bit fixed-point integers (least significant bit 2^-109, probabilities below
// 2^-85 truncated there) rounded to f32 where the reference holds an f32, so the result does not
// depend on summation order; exp is the double exp rounded to f32.  r: the uniform draw in [0, 1).
namespace {
typedef unsigned __int128 u128;
u128 fx_from_f32(float v) {
  uint32_t b;
  std::memcpy(&b, &v, 4);
  const int E = (int)((b >> 23) & 0xFFu);
  if (E == 0 || (b >> 31)) return 0;
  const u128 M = (u128)((b & 0x7FFFFFu) | 0x800000u);
  const int sh = E - 41;
  if (sh >= 0) return M << sh;
  if (sh > -24) return M >> (-sh);
  return 0;
}
float fx_to_f32(u128 a) {   // nearest, ties to even (values below 2^18)
  if (a == 0) return 0.f;
  int msb = 127;
  while (!((a >> msb) & 1)) --msb;
  const int lsb = msb - 23;
  uint64_t mant;
  int round_bit = 0;
  bool sticky = false;
  if (lsb >= 0) {
    mant = (uint64_t)((a >> lsb) & 0xFFFFFFu);
    if (lsb >= 1) round_bit = (int)((a >> (lsb - 1)) & 1);
    if (lsb >= 2) sticky = (a & (((u128)1 << (lsb - 1)) - 1)) != 0;
  } else {
    mant = (uint64_t)(a << (-lsb));
  }
  int e = msb;
  if (round_bit && (sticky || (mant & 1))) {
    ++mant;
    if (mant == 0x1000000u) { mant >>= 1; ++e; }
  }
  const uint32_t bits = ((uint32_t)(e - 109 + 127) << 23) | (uint32_t)(mant & 0x7FFFFFu);
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}
}  // namespace

int orc_sample(const float* logits, int V, const uint32_t* counts, float temperature, float top_p, float penalty,
               float r) {
  std::vector<float> x(logits, logits + V);
  // repetition penalty over the generated tokens (engine.rs:129-141): once per occurrence
  if (penalty != 1.0f && counts)
    for (int v = 0; v < V; ++v)
      for (uint32_t j = 0; j < counts[v]; ++j) x[v] = x[v] > 0.0f ? x[v] / penalty : x[v] * penalty;
  if (temperature == 0.0f) {   // Iterator::max_by: the last of equal maxima (engine.rs:143-151)
    float best = -std::numeric_limits<float>::infinity();
    int bi = -1;
    for (int v = 0; v < V; ++v)
      if (x[v] >= best) { best = x[v]; bi = v; }
    return bi < 0 ? 0 : bi;
  }
  if (temperature != 1.0f) {   // engine.rs:154-159
    const float inv_t = 1.0f / temperature;
    for (float& v : x) v *= inv_t;
  }
  float mx = -std::numeric_limits<float>::infinity();   // engine.rs:162-168
  for (float v : x) mx = std::max(mx, v);
  std::vector<float> p(V);
  u128 tot = 0;
  for (int v = 0; v < V; ++v) {
    p[v] = expcr(x[v] - mx);
    tot += fx_from_f32(p[v]);
  }
  const float S = fx_to_f32(tot);
  for (float& v : p) v = v / S;
  if (top_p < 1.0f) {   // engine.rs:171-195: stable sort descending, shortest prefix exceeding top_p
    std::vector<int> ord(V);
    for (int v = 0; v < V; ++v) ord[v] = v;
    std::stable_sort(ord.begin(), ord.end(), [&](int a, int b) { return p[a] > p[b]; });
    u128 cum = 0;
    int cutoff = V;
    for (int i = 0; i < V; ++i) {
      cum += fx_from_f32(p[ord[i]]);
      if (fx_to_f32(cum) > top_p) { cutoff = i + 1; break; }
    }
    std::vector<char> keep(V, 0);
    for (int i = 0; i < cutoff; ++i) keep[ord[i]] = 1;
    u128 ks = 0;
    for (int v = 0; v < V; ++v) {
      if (!keep[v]) p[v] = 0.0f;
      ks += fx_from_f32(p[v]);
    }
    const float S2 = fx_to_f32(ks);
    if (S2 > 0.0f)
      for (float& v : p) v = v / S2;
  }
  u128 cum = 0;   // engine.rs:197-207
  for (int v = 0; v < V; ++v) {
    cum += fx_from_f32(p[v]);
    if (p[v] > 0.0f && r < fx_to_f32(cum)) return v;
  }
  return V - 1;
}

}  // extern "C"
