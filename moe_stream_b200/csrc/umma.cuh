// umma.cuh — 5th-generation tensor core (tcgen05) helpers for sm_100a: tensor-memory
// allocation, shared-memory matrix descriptors, block-scaled MXFP4 MMA, scale-factor copies
// into tensor memory, commit to an mbarrier and accumulator loads.
//
// Operand layout used throughout (K-major, no swizzle): a matrix of R rows x K fp4 elements
// is stored as K/32 "chunk columns" of R rows x 16 bytes (32 packed e2m1 codes, element 2i in
// the low nibble of byte i).  Chunk c, row r lives at c*R*16 + r*16.  For one MMA (K = 64 =
// two chunk columns) the descriptor's leading-byte offset is R*16 (next chunk column) and its
// stride-byte offset is 128 (next 8-row core matrix).
//
// Scale factors (ue8m0, one per row per 32-element block) are staged as 512-byte groups per
// four blocks ("K-word" w = blocks 4w..4w+3): byte 16*r0 + 4*r1 + j holds the scale of row
// r0 + 32*r1, block 4w + j.  tcgen05.cp .32x128b.warpx4 moves one group into four TMEM
// columns, replicated over the four 32-lane quadrants.  An MMA over blocks (2m, 2m+1) reads
// the group of word m/2 at byte offset 2*(m%2), selected by the scale-factor id.
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

namespace ms {
namespace umma {

// ---- tensor memory allocation (one full warp) ----
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   (uint32_t)__cvta_generic_to_shared(smem_dst)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void fence_before_sync() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// ---- shared-memory matrix descriptor (K-major, no swizzle) ----
__device__ __forceinline__ uint64_t smem_desc(const void* p, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  const uint32_t a = (uint32_t)__cvta_generic_to_shared(p);
  uint64_t d = 0;
  d |= (uint64_t)((a >> 4) & 0x3FFFu);                 // start address, bits [0,14)
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;   // leading-dimension byte offset, bits [16,30)
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;   // stride-dimension byte offset, bits [32,46)
  d |= (uint64_t)1 << 46;                              // descriptor version (sm_100)
  // base offset 0, absolute leading-offset mode 0, layout type 0 (no swizzle)
  return d;
}

// ---- instruction descriptor: kind::mxf4, ue8m0 scales, f32 accumulate, K-major A and B ----
__host__ __device__ constexpr uint32_t idesc_mxf4(int M, int N, uint32_t sfa_id, uint32_t sfb_id) {
  return (sfb_id & 3u) << 4 |        // B scale-factor id
         1u << 7 |                   // A format e2m1
         1u << 10 |                  // B format e2m1
         (uint32_t)(N >> 3) << 17 |  // N / 8
         1u << 23 |                  // scale format ue8m0
         (uint32_t)(M >> 4) << 24 |  // M / 16
         (sfa_id & 3u) << 29;        // A scale-factor id
}

// D[tmem] (+)= (A * sfa) x (B * sfb)^T over K = 64, issued by one thread.
__device__ __forceinline__ void mma_mxf4(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t sfa_tmem, uint32_t sfb_tmem, bool accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::mxf4.block_scale.block32 [%0], %1, %2, %3, [%5], [%6], p;\n}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"((uint32_t)accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
      : "memory");
}

// Copy a 32-row x 16-byte scale group from shared memory into 4 TMEM columns (all quadrants).
__device__ __forceinline__ void cp_sf_group(uint32_t taddr, const void* src) {
  const uint64_t d = smem_desc(src, 16, 128);
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(d) : "memory");
}

// Arrive on an mbarrier once all tcgen05 operations issued so far by this thread complete.
__device__ __forceinline__ void commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   (uint32_t)__cvta_generic_to_shared(bar))
               : "memory");
}

// 32 lanes x 16 consecutive f32 columns: thread t of the warp gets lane (quadrant base + t).
__device__ __forceinline__ void ld_32x32b_x16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// ---- dense bf16 MMA (kind::f16): D[tmem] (+)= A x B^T over K = 16, f32 accumulate, K-major A and B ----
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N) {
  return 1u << 4 |                   // D format f32
         1u << 7 |                   // A format bf16
         1u << 10 |                  // B format bf16
         (uint32_t)(N >> 3) << 17 |  // N / 8
         (uint32_t)(M >> 4) << 24;   // M / 16
}
__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         bool accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"((uint32_t)accumulate)
      : "memory");
}

// 32 lanes x 32 consecutive f32 columns
__device__ __forceinline__ void ld_32x32b_x32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// generic-proxy shared-memory writes become visible to tcgen05 / bulk-copy reads
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// ---- activation as MXFP4 terms (the B operand of the expert GEMVs) ----
// A 32-element block (one element per lane) with maximum |x| in [2^E, 2^(E+1)) is written in
// fixed point relative to its maximum, |x| = N * 2^(E-30) with N = RN(|x| 2^(30-E)) < 2^32, and
// N is cut into kTerms = 16 base-4 digits d_t = (N >> (30 - 2t)) & 3: term t is the e2m1 code of
// sign(x) * d_t (values 0, 1, 2, 3) under the ue8m0 scale 2^(E - 2t).  The terms are exact pieces
// of N, so the block is represented to 2^-31 of its maximum, and every term is computed
// independently (no residual chain).  Blocks below 2^-96 are written as zero.
//
// B matrix layout over kc chunk columns: term t is row t; the codes of chunk c at c*256 + t*16
// (element 2i in the low nibble of byte i); the scales after the codes (offset kc*256) in the
// same 512-byte groups as A's, one per K-word (4 chunks): byte 16*t + c%4 of group c/4.
// (An MMA's scale-factor address must be 4-column aligned, so a group serves one K-word.)
constexpr int kTerms = 16;

__host__ __device__ __forceinline__ int64_t bterm_bytes(int kc) { return (int64_t)kc * 256 + (int64_t)((kc + 3) / 4) * 512; }

__device__ __forceinline__ void quantize_terms_warp(float x, int lane, uint8_t* bt, int kc, int chunk) {
  float amax = fabsf(x);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const int eb = (int)(__float_as_uint(amax) >> 23);   // biased exponent of the block maximum
  const bool live = eb >= 31 && eb < 255;
  // 2^(30 - E) with E = eb - 127: biased exponent 284 - eb, in [30, 253] for live blocks
  const uint32_t N = live ? __float2uint_rn(fabsf(x) * __uint_as_float((uint32_t)(284 - eb) << 23)) : 0u;
  const uint32_t sgn = (__float_as_uint(x) >> 31) << 3;
  uint32_t lo = 0, hi = 0;   // nibbles of terms 0-7 and 8-15
#pragma unroll
  for (int t = 0; t < kTerms; ++t) {
    const uint32_t d = (N >> (30 - 2 * t)) & 3u;
    uint32_t code = (0x5420u >> (4 * d)) & 0xFu;   // e2m1 of 0, 1, 2, 3
    code |= code ? sgn : 0u;
    if (t < 8) lo |= code << (4 * t);
    else hi |= code << (4 * (t - 8));
  }
  const uint32_t plo = __shfl_xor_sync(0xffffffffu, lo, 1), phi = __shfl_xor_sync(0xffffffffu, hi, 1);
  if (!(lane & 1)) {
    uint8_t* cb = bt + (size_t)chunk * 256 + (lane >> 1);
#pragma unroll
    for (int t = 0; t < kTerms; ++t) {
      const uint32_t a = t < 8 ? lo >> (4 * t) : hi >> (4 * (t - 8));
      const uint32_t b = t < 8 ? plo >> (4 * t) : phi >> (4 * (t - 8));
      cb[t * 16] = (uint8_t)((a & 0xFu) | ((b & 0xFu) << 4));
    }
  }
  if (lane < kTerms)
    bt[(size_t)kc * 256 + (size_t)(chunk >> 2) * 512 + 16 * lane + (chunk & 3)] =
        (uint8_t)(live ? eb - 2 * lane : 0);
}

}  // namespace umma
}  // namespace ms
