// Output gathered over the GPUs of one node inside the matmul kernels
// (tsb_qmm_w4g64_gather): each rank's CTAs store the rank's columns into every
// rank's y over NVLink (plain peer stores), so no separate collective runs.
//
// Signal block of rank p (uint32, zero-filled once, then owned by these calls):
//   [0, world)               the epoch each rank last started
//   [world, 2 world)         CTAs of each rank that have finished writing their
//                            part of y here (cumulative over calls)
//   [2 world, 2 world + 3)   rank p's own counters: CTAs done in the current
//                            call, the epoch, the cumulative CTA total
// Start: one CTA of each rank tells every peer "started call e" (once the
// previous work on the rank's stream, including the readers of y, is done); a
// CTA waits for every peer's start word before its first remote store.
// Finish: every CTA, as it exits, adds 1 to its count in every peer's block
// with a system-scope release (cumulative: it orders the CTA's peer stores);
// the last CTA of a rank waits until each peer's count reaches this rank's own
// running total (every rank makes the same calls with the same grid), so y is
// complete on every rank when the grid completes. Every wait is bounded.
#pragma once

#include "sm100.cuh"

namespace tsb {

TSB_HD uint32_t ld_acquire_sys(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
TSB_HD void st_release_sys(uint32_t *p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
TSB_HD void red_add_release_sys(uint32_t *p, uint32_t v) {
  asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// Bounded wait until every other rank's word `base + p` has reached value ep
// (wrap-safe comparison); false (and TSB_ETIMEOUT recorded) if one does not.
TSB_HD bool wait_peers(const uint32_t *base, int world, int rank, uint32_t ep) {
  for (int p = 0; p < world; ++p) {
    if (p == rank) continue;
    const unsigned long long t0 = globaltimer_ns();
    while ((int)(ld_acquire_sys(base + p) - ep) < 0) {
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        record_status(TSB_ETIMEOUT);
        return false;
      }
    }
  }
  return true;
}

// Four floats read through L2 (written by another grid of the stream).
TSB_HD float4 ld_cg_v4(const float *p) {
  float4 v;
  asm volatile("ld.global.cg.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "l"(p)
               : "memory");
  return v;
}

// This call's epoch (read once the previous call on the stream has completed).
TSB_HD uint32_t gather_epoch(uint32_t *const *sig, int world, int rank) {
  return *reinterpret_cast<volatile uint32_t *>(sig[rank] + 2 * world + 1) + 1u;
}

// Tell every peer that this rank has started call ep (one thread of one CTA).
TSB_HD void gather_start(uint32_t *const *sig, int world, int rank, uint32_t ep) {
  for (int pp = 0; pp < world; ++pp)
    if (pp != rank) st_release_sys(sig[pp] + rank, ep);
}

// The finish handshake, by one thread per CTA after a CTA-wide barrier that
// ordered all of the CTA's peer stores before it; ctas = CTAs in the grid.
TSB_HD void gather_finish(uint32_t *const *sig, int world, int rank, uint32_t ctas) {
  uint32_t *own = sig[rank];
  for (int pp = 0; pp < world; ++pp)
    if (pp != rank) red_add_release_sys(sig[pp] + world + rank, 1u);
  if (atomicAdd(own + 2 * world, 1u) + 1u == ctas) {
    own[2 * world] = 0u;
    const uint32_t total = own[2 * world + 2] + ctas;
    wait_peers(own + world, world, rank, total);
    own[2 * world + 2] = total;
    own[2 * world + 1] += 1u;  // this call's epoch is complete on this rank
  }
}

}  // namespace tsb
