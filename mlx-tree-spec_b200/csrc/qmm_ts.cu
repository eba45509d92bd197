// Verify-pass 4-bit quantized matmul (M <= 128 tree tokens): tcgen05 MMA with
// the dequantized weight as the A operand in tensor memory ("TS" form) and the
// tokens as the MMA's N dimension. The B200 counterpart of the reference's
// small-M kernels on its MLX-format weights (mlx-tree-spec
// src/mlx_tree_spec/qmm_packed.py: nax_kernel 151-293 for M <= 16,
// nax_multi_kernel 300-394 for 17..63, the qmv GEMV 428-557 for M <= 4).
//
// Why TMEM for A: at small M every weight is used by only M tokens, so the
// kernel streams HBM at ~0.56 byte per weight while dequantizing. Writing the
// bf16 weights to shared memory and having the MMA read them back would cost
// 4 bytes of shared-memory traffic per weight; tcgen05.st into TMEM keeps the
// shared-memory path for the packed codes and x only.
//
// CTA: 128 weight rows (one TMEM lane each) x all tokens (NP = M rounded up
// to 16), a K range of whole stages (4 groups = 256 K each); one CTA per SM
// (all 512 TMEM columns); split-K CTAs of one row tile form a cluster and
// reduce through distributed shared memory. Warp roles:
//   warp 0    TMA producer of the codes ring: per stage the codes of the 128
//             rows (32 words each, 128-byte swizzle) and their scales and
//             biases (8-group boxes). A slot is refilled as soon as its
//             dequantizers have loaded its words into registers.
//   warp 2    TMA producer of the x ring: x for the stage (four 64-K boxes of
//             NP rows, 128-byte swizzle, rows >= M zero-filled by TMA); a slot
//             is refilled when the MMAs that read it have completed.
//   warps 1,3(,5) MMA issuers (one lane each, WGS of them): issuer u takes
//             the stages i = u (mod WGS): one wait, 16 tcgen05.mma (M=128,
//             N=NP, K=16) back to back and two commits per stage, into
//             accumulator u (summed in the epilogue). A = the dequantized
//             weights from TMEM, B = x from shared memory, f32 accumulators in
//             TMEM. Independent accumulators let the issuers' MMA streams
//             overlap; per-stage waits and commits are paid once per stage.
//   warps 8.. dequantizers, WGS warpgroups (3 for NP <= 32, else 2);
//             warpgroup u owns the same stages as issuer u, all four groups of
//             each (thread = weight row = TMEM lane): codes -> bf16(s*q + b) ->
//             tcgen05.st into its own stage slot of A in TMEM, handed to issuer
//             u once the stores have landed. Owning whole stages keeps the
//             dequantizer warps of a sub-partition at different stages, so one
//             warp's waits are covered by the others' arithmetic, and gives
//             every ring slot and barrier a single waiter that walks its
//             stages in order (no wait can run two phases ahead). Warpgroup 0
//             then runs the epilogue (TMEM -> registers -> bf16 y, or split-K
//             partials).
//
// Arithmetic: y = sum_k w_k x_k with w = bf16(fma(q, s, b)), the reference's
// dequantization rule (qmm_packed.py:200, 348, 635) exactly: (code | 0x4300)
// is bf16 128 + q, one bf16x2 subtract gives q exactly and one fused bf16x2
// fma rounds q*s + b once. At N = NP <= 64 an M=128 K=16 MMA costs about the
// same whatever N is (measured ~27 ns issued back to back), so the weights
// carry the bias and each group costs only its four K=16 MMAs.
#include "sm100.cuh"

#include <cooperative_groups.h>
#include <string.h>

namespace cg = cooperative_groups;

namespace tsb {

namespace {

template <int NP>
struct TsCfg {
  static constexpr int ROWS = 128;
  static constexpr int SG = 4;                     // groups per stage
  static constexpr int C_BYTES = ROWS * SG * 32;   // codes, 128 B per row
  static constexpr int SB_BYTES = ROWS * 8 * 2;    // 8 groups of scales (or biases) per row
  static constexpr int CSLOT_BYTES = C_BYTES + 2 * SB_BYTES;
  static constexpr int X_BOX_BYTES = NP * 128;     // one 64-K box of x
  static constexpr int XSLOT_BYTES = SG * X_BOX_BYTES;
  static constexpr int RING_BUDGET = 225 * 1024;   // shared memory for the two rings
  // WGS dequantizer warpgroups; warpgroup w owns the stages i = w (mod WGS)
  // and A stage slot w. NI MMA issuers; issuer u takes part u (SG/NI groups)
  // of every stage into accumulator u.
  static constexpr int WGS = 3;
  static constexpr int NI = NP <= 32 ? 4 : (NP <= 64 ? 2 : 1);  // MMA issuers, one accumulator each
  static constexpr int GPI = SG / NI;              // groups per issuer part
  static constexpr int NX = NP <= 32 ? 4 : (NP == 64 ? 3 : 2);  // x slots
  static constexpr int NC_FIT = (RING_BUDGET - NX * XSLOT_BYTES) / CSLOT_BYTES;
  static constexpr int NC = (NC_FIT > 12 ? 12 : NC_FIT) / WGS * WGS;          // codes slots, a multiple of WGS
  static constexpr int X_AREA = NC * CSLOT_BYTES;
  static constexpr int STAGE_AREA = X_AREA + NX * XSLOT_BYTES;
  static constexpr int A_COL0 = (NI * NP + 31) / 32 * 32;  // accumulators in [0, NI NP), A slots after
  static constexpr int GA = 32;                    // per group slot: 64 bf16 weights per row
  static constexpr int TMEM_COLS = 512;
  static constexpr int NAS = WGS;                  // stage slots of A in TMEM (4 groups each), one per warpgroup
  static constexpr int DQ_WARP0 = 8;               // first dequantizer warp (lane quarter = warp & 3)
  static constexpr int THREADS = (DQ_WARP0 + 4 * WGS) * 32;
  static constexpr size_t SMEM = (size_t)STAGE_AREA + 1024 + 1024;
  static_assert(NC >= WGS && A_COL0 + NAS * SG * GA <= TMEM_COLS, "ring depths and TMEM columns");
  static_assert(CSLOT_BYTES % 1024 == 0 && XSLOT_BYTES % 1024 == 0, "slot alignment (128-byte swizzle atoms)");
  static_assert(NP * 512 <= STAGE_AREA, "split-K partials fit in the stage area");
  static_assert(SMEM <= 227 * 1024, "shared memory per CTA");
};

// Advance a ring position (slot, phase bit) without divisions.
struct Ring {
  int slot = 0;
  uint32_t phase = 0;
  TSB_HD void next(int n) {
    if (++slot == n) { slot = 0; phase ^= 1u; }
  }
};

template <int NP>
__global__ void __launch_bounds__(TsCfg<NP>::THREADS, 1)
qmm_ts_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_w,
              const __grid_constant__ CUtensorMap tmap_s, const __grid_constant__ CUtensorMap tmap_b,
              const uint16_t *__restrict__ scales, const uint16_t *__restrict__ biases,
              uint16_t *__restrict__ y, int M, int N, int K, int ldy, int splits) {
  using C = TsCfg<NP>;
  extern __shared__ unsigned char smem_raw[];
  unsigned char *smem =
      reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::STAGE_AREA);
  uint64_t *full_c = bars;                       // [NC] codes + scales + biases landed
  uint64_t *free_c = bars + C::NC;               // [NC] dequantizers have loaded the slot
  uint64_t *full_x = bars + 2 * C::NC;           // [NX] x landed
  uint64_t *free_x = full_x + C::NX;             // [NX] MMAs that read the slot are done
  uint64_t *a_full = free_x + C::NX;             // [NAS] stage written into TMEM
  uint64_t *a_empty = a_full + C::NAS;           // [NAS] MMAs done with the stage slot
  uint64_t *acc_full = a_empty + C::NAS;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_full + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int n0 = blockIdx.x * C::ROWS;
  const int split = blockIdx.y;
  const int G = K / 64;
  const int nst_all = (G + C::SG - 1) / C::SG;
  const int st0 = (int)((long long)split * nst_all / splits);
  const int st1 = (int)((long long)(split + 1) * nst_all / splits);
  const int nst = st1 - st0;
  const int g0 = st0 * C::SG;
  const int g1 = min(G, st1 * C::SG);
  // G % 8 != 0: the scale rows' pitch (2G bytes) is not a multiple of 16, which
  // TMA tiles require; the dequantizers then load their row's scales and
  // biases directly (odd shapes only; model shapes have K % 512 == 0).
  const bool sb_direct = (G % 8) != 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::NC; ++s) {
      mbar_init(&full_c[s], 1);
      mbar_init(&free_c[s], 4);  // the 4 warps of the stage's warpgroup
    }
    for (int s = 0; s < C::NX; ++s) {
      mbar_init(&full_x[s], 1);
      mbar_init(&free_x[s], C::NI);  // every MMA issuer
    }
    for (int b = 0; b < C::NAS; ++b) {
      mbar_init(&a_full[b], 4);      // the 4 warps of the owning warpgroup
      mbar_init(&a_empty[b], C::NI);  // every MMA issuer
    }
    mbar_init(acc_full, C::NI);
    fence_mbar_init();
    fence_proxy_async_smem();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  auto cslot = [&](int s) { return smem + (size_t)s * C::CSLOT_BYTES; };
  auto xslot = [&](int s) { return smem + C::X_AREA + (size_t)s * C::XSLOT_BYTES; };

  if (warp == 0 || warp == 2) {
    // ---------------- TMA producers: warp 0 the codes ring, warp 2 the x ring
    const bool codes = warp == 0;
    const int nslots = codes ? C::NC : C::NX;
    uint64_t *full = codes ? full_c : full_x;
    uint64_t *freed = codes ? free_c : free_x;
    if (elect_one()) {
      if (codes) {
        tma_prefetch_desc(&tmap_w);
        if (!sb_direct) {
          tma_prefetch_desc(&tmap_s);
          tma_prefetch_desc(&tmap_b);
        }
      } else {
        tma_prefetch_desc(&tmap_x);
      }
      Ring ring;
      int issued = 0;
      for (int i = 0; i < nst; ++i, ring.next(nslots)) {
        if (i >= nslots && !mbar_wait(&freed[ring.slot], ring.phase ^ 1u)) break;
        const int gs = g0 + i * C::SG;
        if (codes) {
          unsigned char *st = cslot(ring.slot);
          mbar_arrive_expect_tx(&full[ring.slot], C::C_BYTES + (sb_direct ? 0 : 2 * C::SB_BYTES));
          tma_load_2d(st, &tmap_w, gs * 8, n0, &full[ring.slot]);
          if (!sb_direct) {
            const int gb = gs & ~7;  // 8-group box containing this stage's groups
            tma_load_2d(st + C::C_BYTES, &tmap_s, gb, n0, &full[ring.slot]);
            tma_load_2d(st + C::C_BYTES + C::SB_BYTES, &tmap_b, gb, n0, &full[ring.slot]);
          }
        } else {
          unsigned char *xt = xslot(ring.slot);
          mbar_arrive_expect_tx(&full[ring.slot], C::XSLOT_BYTES);
#pragma unroll
          for (int gl = 0; gl < C::SG; ++gl)
            tma_load_2d(xt + gl * C::X_BOX_BYTES, &tmap_x, (gs + gl) * 64, 0, &full[ring.slot]);
        }
        issued = i + 1;
      }
      // drain: every issued load has landed before the CTA can exit
      for (int i = (issued > nslots ? issued - nslots : 0); i < issued; ++i) {
        const unsigned long long t0 = globaltimer_ns();
        while (!mbar_try_wait(&full[i % nslots], (i / nslots) & 1)) {
          if (globaltimer_ns() - t0 > kWaitLimitNs) { record_status(TSB_ETIMEOUT); break; }
        }
      }
    }
  } else if ((warp & 1) && warp < 2 * C::NI) {
    // ---------------- MMA issuers: warp 2u+1 takes part u of every stage into
    // accumulator u; one lane each, descriptors built once per stage and
    // advanced by adding the 16-byte-unit offset of each 64-K box and 16-K slice
    const int u = warp >> 1;
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16_f32(128, NP);
      const uint32_t dacc = tmem_base + (uint32_t)(u * NP);
      bool ok = true, first = true;
      Ring ring, aring;
      for (int i = 0; i < nst && ok; ++i, ring.next(C::NX), aring.next(C::NAS)) {
        ok = mbar_wait(&full_x[ring.slot], ring.phase) &&
             mbar_wait(&a_full[aring.slot], aring.phase);
        if (!ok) break;
        tc_fence_after();
        const int gs = g0 + i * C::SG;
        const int gend = min(C::GPI * (u + 1), g1 - gs);
        const uint64_t xd = desc_kmajor_sw128(smem_addr(xslot(ring.slot)));
        const uint32_t a0 = tmem_base + C::A_COL0 + (uint32_t)(aring.slot * C::SG * C::GA);
        for (int gl = C::GPI * u; gl < gend; ++gl) {
          const uint32_t ag = a0 + gl * C::GA;
          const uint64_t bd = xd + (uint64_t)((gl * C::X_BOX_BYTES) >> 4);
          mma_ts_f16(dacc, ag, bd, idesc, first ? 0u : 1u);
          mma_ts_f16(dacc, ag + 8, bd + 2, idesc, 1u);  // +32 B: next 16 K
          mma_ts_f16(dacc, ag + 16, bd + 4, idesc, 1u);
          mma_ts_f16(dacc, ag + 24, bd + 6, idesc, 1u);
          first = false;
        }
        mma_commit(&a_empty[aring.slot]);
        mma_commit(&free_x[ring.slot]);
      }
      mma_commit(acc_full);  // every issuer arrives once, with or without groups
    }
    __syncwarp();
  } else if (warp >= C::DQ_WARP0) {
    // ---------------- dequantizers (thread = weight row = TMEM lane)
    const int q = warp & 3;
    const int wg = (warp - C::DQ_WARP0) >> 2;  // owns stages i = wg (mod WGS)
    const int r = q * 32 + lane;
    const int row = n0 + r;
    const uint32_t lane_base = tmem_base + ((uint32_t)(q * 32) << 16);
    bool ok = true;
    // Stage i lives in codes slot i % NC (NC % WGS == 0) and A stage slot
    // i % WGS = wg: every slot and every barrier has one owning warpgroup,
    // which walks its stages in order, so no wait can run two phases ahead.
    int cs = wg;
    uint32_t cphase = 0;
    int ai = 0;  // this warpgroup's stage count: phase of its A slot
    uint32_t a[32];
    for (int i = wg; i < nst && ok; i += C::WGS) {
      ok = warp_wait(&full_c[cs], cphase);
      if (!ok) break;
      const int gs = g0 + i * C::SG;
      const int ng = min(C::SG, g1 - gs);  // uniform
      const unsigned char *st = cslot(cs);
      // this row's scales and biases of the stage's four groups (8-byte loads)
      uint32_t s_w[2], b_w[2];
      if (sb_direct) {
#pragma unroll
        for (int hw = 0; hw < 2; ++hw) {
          const int ga = gs + 2 * hw;
          const size_t idx = (size_t)row * G + ga;
          const bool v0 = ga < g1, v1 = ga + 1 < g1;
          s_w[hw] = (v0 ? uint32_t(__ldg(scales + idx)) : 0u) | (v1 ? uint32_t(__ldg(scales + idx + 1)) << 16 : 0u);
          b_w[hw] = (v0 ? uint32_t(__ldg(biases + idx)) : 0u) | (v1 ? uint32_t(__ldg(biases + idx + 1)) << 16 : 0u);
        }
      } else {
        const int off = r * 16 + (gs & 7) * 2;  // (gs & 7) is 0 or 4: 8-byte aligned
        const uint2 sv = *reinterpret_cast<const uint2 *>(st + C::C_BYTES + off);
        const uint2 bv = *reinterpret_cast<const uint2 *>(st + C::C_BYTES + C::SB_BYTES + off);
        s_w[0] = sv.x; s_w[1] = sv.y; b_w[0] = bv.x; b_w[1] = bv.y;
      }
      // the stage's 32 packed words of this row, then release the codes slot
      uint32_t words[32];
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const int chunk = c ^ (r & 7);  // TMA 128-byte swizzle
        const uint4 v = *reinterpret_cast<const uint4 *>(st + r * 128 + chunk * 16);
        words[4 * c + 0] = v.x; words[4 * c + 1] = v.y; words[4 * c + 2] = v.z; words[4 * c + 3] = v.w;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&free_c[cs]);
      // the A slot is free once the MMAs of this warpgroup's previous stage completed
      if (ai > 0 && !warp_wait(&a_empty[wg], (uint32_t)((ai - 1) & 1))) {
        ok = false;
        break;
      }
      tc_fence_after();
#pragma unroll
      for (int gl = 0; gl < C::SG; ++gl) {
        if (gl >= ng) break;
        const uint32_t sb = (s_w[gl >> 1] >> (16 * (gl & 1))) & 0xFFFFu;
        const uint32_t bb = (b_w[gl >> 1] >> (16 * (gl & 1))) & 0xFFFFu;
        const __nv_bfloat162 s2 = u32_as_bf2(sb | (sb << 16));
        const __nv_bfloat162 b2 = u32_as_bf2(bb | (bb << 16));
#pragma unroll
        for (int wj = 0; wj < 8; ++wj) {
          uint32_t o[4];
          dequant_word(words[gl * 8 + wj], s2, b2, o);
          a[4 * wj + 0] = o[0]; a[4 * wj + 1] = o[1]; a[4 * wj + 2] = o[2]; a[4 * wj + 3] = o[3];
        }
        tmem_st32(lane_base + C::A_COL0 + (wg * C::SG + gl) * C::GA, a);
      }
      // tcgen05.st reads its source registers at issue (a is reused above); the
      // stores must only have reached TMEM before the issuers are told
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&a_full[wg]);
      if (!ok) break;
      ++ai;
      cs += C::WGS;
      if (cs >= C::NC) { cs -= C::NC; cphase ^= 1u; }
    }
    // ---------------- epilogue part 1: accumulator -> y or partials
    if (wg == 0 && ok && nst > 0 && warp_wait(acc_full, 0)) {
      tc_fence_after();
      float *red = reinterpret_cast<float *>(smem);  // [NP][128], the stage area is free now
      // accumulator u holds data once some stage has a group in its part
      int nacc = 1;
      while (nacc < C::NI && g1 - g0 > nacc * C::GPI) ++nacc;
#pragma unroll
      for (int c0 = 0; c0 < NP; c0 += 16) {
        uint32_t v[16];
        tmem_ld16(lane_base + c0, v);
        tmem_wait_ld();
        for (int u = 1; u < nacc; ++u) {
          uint32_t v1[16];
          tmem_ld16(lane_base + u * NP + c0, v1);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 16; ++e) v[e] = __float_as_uint(__uint_as_float(v[e]) + __uint_as_float(v1[e]));
        }
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const int t = c0 + e;
          if (splits == 1) {
            if (t < M) y[(size_t)t * ldy + row] = float_to_bf16_bits(__uint_as_float(v[e]));
          } else {
            red[t * 128 + r] = __uint_as_float(v[e]);
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
  if (splits > 1) {
    // ---------------- epilogue part 2: reduce the cluster's partials (DSMEM)
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();
    float *red = reinterpret_cast<float *>(smem);
    const int rank = (int)cluster.block_rank();
    const int total = NP * 128;
    const int per = (total + splits - 1) / splits;
    const int e0 = rank * per, e1 = min(total, e0 + per);
    for (int e = e0 + (int)threadIdx.x; e < e1; e += C::THREADS) {
      const int t = e >> 7;
      if (t >= M) continue;
      float acc = 0.f;
      for (int rr = 0; rr < splits; ++rr) acc += cluster.map_shared_rank(red, rr)[e];
      y[(size_t)t * ldy + n0 + (e & 127)] = float_to_bf16_bits(acc);
    }
    cluster.sync();
  }
}

template <int NP>
int launch_ts(const uint16_t *x, const uint32_t *w, const uint16_t *s, const uint16_t *b, uint16_t *y, int M, int N,
              int K, int ldy, cudaStream_t st) {
  using C = TsCfg<NP>;
  CUtensorMap tx, tw;
  if (make_tmap_2d(&tx, x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)K, (uint64_t)M, (uint64_t)K * 2, 64, NP,
                   CU_TENSOR_MAP_SWIZZLE_128B) != TSB_OK)
    return TSB_ECUDA;
  if (make_tmap_2d(&tw, w, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, (uint64_t)K / 8, (uint64_t)N, (uint64_t)K / 2, 32, 128,
                   CU_TENSOR_MAP_SWIZZLE_128B) != TSB_OK)
    return TSB_ECUDA;
  CUtensorMap tsc, tbi;
  const uint64_t G64 = (uint64_t)K / 64;
  memset(&tsc, 0, sizeof(tsc));
  memset(&tbi, 0, sizeof(tbi));
  if (G64 % 8 == 0) {  // else the kernel loads scales/biases directly
    if (!aligned(s, 16) || !aligned(b, 16)) return TSB_EINVAL;
    if (make_tmap_2d(&tsc, s, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, G64, (uint64_t)N, G64 * 2, 8, 128,
                     CU_TENSOR_MAP_SWIZZLE_NONE) != TSB_OK ||
        make_tmap_2d(&tbi, b, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, G64, (uint64_t)N, G64 * 2, 8, 128,
                     CU_TENSOR_MAP_SWIZZLE_NONE) != TSB_OK)
      return TSB_ECUDA;
  }
  static int attr_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (attr_dev != dev) {
    if (cudaFuncSetAttribute(qmm_ts_kernel<NP>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::SMEM) !=
        cudaSuccess)
      return TSB_ECUDA;
    attr_dev = dev;
  }
  const int tiles = N / 128;
  const int nst_all = (int)((G64 + C::SG - 1) / C::SG);
  // one CTA per SM (all of TMEM): split K so that the grid fills the SMs in one wave
  int splits = tiles >= sm_count() ? 1 : sm_count() / tiles;
  if (splits > 8) splits = 8;
  while (splits > 1 && nst_all / splits < 2) --splits;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(tiles, splits, 1);
  cfg.blockDim = dim3(C::THREADS, 1, 1);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = splits;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, qmm_ts_kernel<NP>, tx, tw, tsc, tbi, s, b, y, M, N, K, ldy, splits);
  return e == cudaSuccess ? TSB_OK : TSB_ECUDA;
}

}  // namespace

// M in [1, 128]: tokens padded to a multiple of 16 for the MMA's N.
int qmm_ts(const uint16_t *x, const uint32_t *w, const uint16_t *s, const uint16_t *b, uint16_t *y, int M, int N,
           int K, int ldy, cudaStream_t st) {
  if (M <= 16) return launch_ts<16>(x, w, s, b, y, M, N, K, ldy, st);
  if (M <= 32) return launch_ts<32>(x, w, s, b, y, M, N, K, ldy, st);
  if (M <= 64) return launch_ts<64>(x, w, s, b, y, M, N, K, ldy, st);
  return launch_ts<128>(x, w, s, b, y, M, N, K, ldy, st);
}

unsigned int status_ts(bool reset) {
  unsigned int v = 0;
  cudaMemcpyFromSymbol(&v, g_device_status, sizeof(v));
  if (reset && v) {
    const unsigned int z = 0;
    cudaMemcpyToSymbol(g_device_status, &z, sizeof(z));
  }
  return v;
}

}  // namespace tsb
