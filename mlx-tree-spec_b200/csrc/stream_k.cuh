// Pieces of the verify-path matmul kernel (qmm_ts.cu): the persistent
// stream-K partition of (row tile, stage) units over the CTAs, ring positions,
// and the flag/partial helpers that join the parts of a split tile.
#pragma once

#include "gather.cuh"

namespace tsb {

// Advance a ring position (slot, phase bit) without divisions.
struct Ring {
  int slot = 0;
  uint32_t phase = 0;
  TSB_HD void next(int n) {
    if (++slot == n) { slot = 0; phase ^= 1u; }
  }
};

// Stream-K partition: CTA c of P owns units [U c / P, U (c+1) / P). The owners
// of tile t (units [t nst, (t+1) nst)) are CTAs c_lo(t) .. c_hi(t).
struct Part {
  long long U;
  int P, nst;
  TSB_HD long long start(int c) const { return U * c / P; }
  TSB_HD int c_lo(int t) const {
    const long long a = (long long)t * nst;
    return (int)(((a + 1) * P + U - 1) / U) - 1;
  }
  TSB_HD int c_hi(int t) const {
    const long long b = (long long)(t + 1) * nst;
    return (int)((b * P + U - 1) / U) - 1;
  }
};

TSB_HD uint32_t ld_acquire_gpu(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
TSB_HD void st_release_gpu(uint32_t *p, uint32_t v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// 16-byte global -> shared copy through L2 (cp.async.cg), completed by cp_async_wait_all.
TSB_HD void cp_async_cg16(uint32_t dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
TSB_HD void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

// The workspace of a verify-path call starts with a fixed flag region for
// every shape: partials of one call must never land where another shape's
// call keeps its flags (the region is only ever written with flag stores, so
// it stays zero between calls); the partials follow it.
constexpr size_t kFlagRegionBytes = 64 * 1024;

// Grid of a verify-path call, and the most parts any tile can be split into.
// P CTAs, at most one per SM and at least two stages each. Where the row
// tiles allow it, P makes every CTA's range one equal part of one tile or
// whole tiles (P a multiple of the tile count, or about tiles / ceil(tiles /
// #SM)), so that no CTA joins two tiles: measured faster on B200 for the
// 6144-row verify shapes (~5%) and for every M = 128 projection (4-23%).
// An aligned grid that would leave more than 15% of the SMs idle is kept only
// at M = 128 (`wide`); narrower calls then use P = #SM (5120x17408 at M <= 64:
// 120 aligned CTAs measured 3-5% slower than 148).
struct SkPlan {
  long long U;
  int P, nst, tiles, maxp;
};

inline SkPlan plan_stream_k(int N, int K, bool wide) {
  SkPlan p;
  p.tiles = N / 128;
  p.nst = (K / 64 + 3) / 4;
  p.U = (long long)p.tiles * p.nst;
  const long long sms = sm_count();
  long long P = sms, Pa;
  if (p.tiles <= sms) {
    long long k = sms / p.tiles;
    if (k > p.nst / 2) k = p.nst / 2;
    if (k < 1) k = 1;
    Pa = (long long)p.tiles * k;
  } else {
    const long long per_cta = (p.tiles + sms - 1) / sms;  // whole tiles per CTA
    Pa = (p.tiles + per_cta - 1) / per_cta;
  }
  if (wide || Pa * 100 >= 85 * sms) P = Pa;
  if (P > p.U / 2) P = p.U / 2;
  if (P < 1) P = 1;
  p.P = (int)P;
  const long long per = p.U / p.P;  // the shortest range
  p.maxp = (int)((p.nst + per - 1) / per) + 1;
  return p;
}

}  // namespace tsb
