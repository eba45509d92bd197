// Shared helpers for the libtsb kernels (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "../../include/tsb.h"

#define TSB_HD __device__ __forceinline__

namespace tsb {

// Returns TSB_ECUDA for any pending launch/runtime error of the last launch.
static inline int launch_status() {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? TSB_OK : TSB_ECUDA;
}

static inline bool aligned(const void *p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

static inline int ceil_div(int a, int b) { return (a + b - 1) / b; }

// Number of SMs of the current device (cached per device).
int sm_count();

// Peers of a gathered output (tsb_gather_t after checks): the kernel stores
// this rank's columns [col0, col0 + N) into y[p] for every rank p.
constexpr int kMaxGatherRanks = TSB_MAX_GATHER_RANKS;
struct GatherSpec {
  int world, rank, col0;
  void *y[kMaxGatherRanks];
  uint32_t *sig[kMaxGatherRanks];
};

TSB_HD float bf16_bits_to_float(uint16_t b) { return __uint_as_float(uint32_t(b) << 16); }

TSB_HD float bf16lo(uint32_t v) { return __uint_as_float(v << 16); }
TSB_HD float bf16hi(uint32_t v) { return __uint_as_float(v & 0xFFFF0000u); }

// Round-to-nearest-even float -> bf16 bits.
TSB_HD uint16_t float_to_bf16_bits(float f) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}

TSB_HD uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t *>(&h);
}

// d = (a & b) | c, one LOP3.
TSB_HD uint32_t lop3_and_or(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

TSB_HD uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

// D = A(16x16 bf16, row) * B(16x8 bf16, col) + C (f32), legacy warp MMA.
TSB_HD void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1, const float (&c)[4]) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1),
        "f"(c[0]), "f"(c[1]), "f"(c[2]), "f"(c[3]));
}

TSB_HD uint2 ldg_nc_v2(const void *p) {
  uint2 r;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
  return r;
}

TSB_HD uint4 ldg_nc_v4(const void *p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}

TSB_HD uint32_t bf2_as_u32(__nv_bfloat162 v) { return *reinterpret_cast<uint32_t *>(&v); }
TSB_HD __nv_bfloat162 u32_as_bf2(uint32_t v) { return *reinterpret_cast<__nv_bfloat162 *>(&v); }

// 8 codes of one MLX word -> 4 bf16x2 (natural order) of s*q + b. Two masks
// and a shift split the nibbles, byte permutes place (code | 0x4300) = bf16
// 128 + q, an exact bf16 subtract of 128 leaves q, and one bf16x2 fma rounds
// s*q + b once to bf16 (equal to bf16(fmaf(q, s, b)) whenever that float32
// sum is exact, as it is for quantizer-produced (s, b)).
TSB_HD void dequant_word(uint32_t w, __nv_bfloat162 s2, __nv_bfloat162 b2, uint32_t (&o)[4]) {
  const uint32_t t0 = w & 0x0F0F0F0Fu;          // codes 0,2,4,6
  const uint32_t t1 = (w >> 4) & 0x0F0F0F0Fu;   // codes 1,3,5,7
  const uint32_t u0 = prmt(t0, t1, 0x5140u);    // bytes: q0 q1 q2 q3
  const uint32_t u1 = prmt(t0, t1, 0x7362u);    // q4 q5 q6 q7
  const uint32_t magic = 0x43434343u;
  const __nv_bfloat162 k128 = __floats2bfloat162_rn(128.f, 128.f);
  const uint32_t v[4] = {prmt(u0, magic, 0x4140u), prmt(u0, magic, 0x4342u), prmt(u1, magic, 0x4140u),
                         prmt(u1, magic, 0x4342u)};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __nv_bfloat162 q = __hsub2(u32_as_bf2(v[i]), k128);
    o[i] = bf2_as_u32(__hfma2(q, s2, b2));
  }
}

// Scale pair for dequant_word_sub: (s * 2^133, s * 2^129) as bf16x2 bits, made
// by adding 133 and 129 to s's exponent field. Valid (true) when that is
// exact and finite, i.e. s is +-0 or a normal bf16 below 2^-5 in magnitude
// (exponent field 1..121); otherwise the caller uses dequant_word.
TSB_HD bool sub_scale_pair(uint32_t sb, uint32_t &s2) {
  const uint32_t mag = sb & 0x7FFFu;
  if (mag == 0u) {
    s2 = sb | (sb << 16);
    return true;
  }
  s2 = (sb + (133u << 7)) | ((sb + (129u << 7)) << 16);
  return mag >= 0x0080u && mag < (122u << 7);
}

// 8 codes of one MLX word -> 4 bf16x2 (natural order) of bf16(s*q + b) with
// one byte permute, one mask and one bf16x2 fma per pair (12 instructions per
// word against 17 for dequant_word). The permute copies byte j (codes 2j,
// 2j+1) into the low and the high half; the mask keeps code 2j in bits 0-3 of
// the low half and code 2j+1 in bits 4-7 of the high half. A bf16 whose bits
// 8-15 are zero is worth (bits 0-7 as an integer) * 2^-133 (the subnormals and
// the first binade share that spacing), so the halves hold q_even * 2^-133 and
// q_odd * 2^-129 exactly. With s2 = (s * 2^133, s * 2^129) from
// sub_scale_pair the fma's exact product is q*s, and the sum with b is rounded
// once: the same bf16 as dequant_word gives.
TSB_HD void dequant_word_sub(uint32_t w, __nv_bfloat162 s2, __nv_bfloat162 b2, uint32_t (&o)[4]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t t = prmt(w, 0u, 0x4040u | (uint32_t)j | ((uint32_t)j << 8)) & 0x00F0000Fu;
    o[j] = bf2_as_u32(__hfma2(u32_as_bf2(t), s2, b2));
  }
}

// 8 codes of one MLX word -> 4 bf16x2 (natural order) of bf16(s*q), without
// the bias: (code | 0x4300) is bf16 128 + q, and fma(128 + q, s, -128 s) =
// s*q rounded once (s and -128 s are exact bf16). The bias enters the matmul
// separately (sum_k b x_k per group), so the per-element work is one fma per
// pair after the byte shuffles.
TSB_HD void dequant_word_scaled(uint32_t w, __nv_bfloat162 s2, __nv_bfloat162 ns2, uint32_t (&o)[4]) {
  const uint32_t t0 = w & 0x0F0F0F0Fu;
  const uint32_t t1 = (w >> 4) & 0x0F0F0F0Fu;
  const uint32_t u0 = prmt(t0, t1, 0x5140u);
  const uint32_t u1 = prmt(t0, t1, 0x7362u);
  const uint32_t magic = 0x43434343u;
  const uint32_t v[4] = {prmt(u0, magic, 0x4140u), prmt(u0, magic, 0x4342u), prmt(u1, magic, 0x4140u),
                         prmt(u1, magic, 0x4342u)};
#pragma unroll
  for (int i = 0; i < 4; ++i) o[i] = bf2_as_u32(__hfma2(u32_as_bf2(v[i]), s2, ns2));
}

}  // namespace tsb
