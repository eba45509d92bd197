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
// Schedule: a persistent, stream-K grid of P <= #SM CTAs (one per SM: all 512
// TMEM columns), launched as a programmatic dependent of the previous kernel on
// the stream: CTAs start as that kernel's CTAs exit and stream the (constant)
// weights at once; x, y and the workspace wait for the previous grid to
// complete (griddepcontrol.wait). The work is the list of (row tile of 128 weight
// rows, stage of 4 groups = 256 K) units, tile-major; CTA c takes the
// contiguous units [U c / P, U (c+1) / P). Its range crosses tile boundaries,
// so it works on a sequence of tile segments. A segment that covers a whole
// tile writes y directly. A tile split over CTAs c_lo < ... < c_hi: the parts
// of c_lo+1..c_hi (which end early in those CTAs' ranges) go to the workspace
// as float partials with a completion flag each; c_lo, whose part is the last
// segment of its range, waits for the flags, adds the partials, writes y and
// clears the flags (the workspace is left as it was found: flags zero).
//
// Warp roles (thread = weight row = TMEM lane wherever TMEM is touched):
//   warps 0-3  epilogue: per segment, accumulators -> registers -> y, partial
//              or fixup, 8 or 16 tokens at a time; y values are staged as bf16
//              in shared memory and written as 16-byte chunks of y rows;
//              warp 0 also allocates TMEM.
//   warp 4     TMA producer of the codes ring: per stage the codes of the 128
//              rows (32 words each, 128-byte swizzle) and their scales and
//              biases (8-group boxes). A slot is refilled as soon as its
//              dequantizers have loaded its words into registers.
//   warp 5     TMA producer of the x ring: x for the stage (four 64-K boxes of
//              NP rows, 128-byte swizzle, rows >= M zero-filled by TMA); a slot
//              is refilled when the MMAs that read it have completed.
//   warps 6,7,20,21  MMA issuers (NI of them, one lane each): issuer u takes
//              its share of every stage's groups into accumulator u (summed in
//              the epilogue); per stage one wait, the MMAs back to back and two
//              commits. A = the dequantized weights from TMEM, B = x from
//              shared memory, f32 accumulators in TMEM. One thread issues at
//              most one M=128 K=16 MMA every ~68 ns whatever N is, while four
//              issuing warps reach ~17 ns per MMA at N <= 32 (measured on
//              B200), so several issuers keep the tensor pipe busy.
//   warps 8-19 dequantizers, three warpgroups (two at NP = 128): warpgroup w
//              owns the stages i = w (mod WGS) of the CTA's range, all four groups:
//              codes -> bf16(s*q + b) -> tcgen05.st into its own stage slot of
//              A in TMEM, handed to the issuers once the stores have landed.
//              Owning whole stages keeps the dequantizer warps of a
//              sub-partition at different stages (one warp's waits are covered
//              by the others' arithmetic).
// Every ring slot and every mbarrier has waiters that walk their stages (or
// segments) in order, so no parity wait can run two phases ahead.
//
// Arithmetic: y = sum_k w_k x_k with w = bf16(q*s + b) rounded once (one bf16x2
// fma per pair of codes after a byte permute and a mask: dequant_word_sub; the
// magic-number form dequant_word for scales of 2^-5 and above). The reference
// rounds q*s + b to float32 first (qmm_packed.py:200, 348, 635); the two agree
// unless that float32 rounding lands exactly on a bf16 rounding midpoint, which
// needs |b| below half a float32 ulp of q*s and never happens for
// quantizer-made scales and biases. tsb_dequant_w4g64 follows the reference's
// two roundings bit for bit. The weights carry the bias, so each group costs
// only its four K=16 MMAs.
#include "stream_k.cuh"

#include <string.h>

namespace tsb {

namespace {

// Configuration variants (VAR), chosen per call by qmm_ts():
//   kTsDefault;
//   kTsWhole (NP = 64, the call's CTAs stream whole row tiles: more tiles than
//     SMs): four MMA issuers with two stage slots instead of two issuers with
//     three. Measured on B200 at M = 33-64: 8-10% faster on 34816x5120, but
//     3-11% slower on 6144x5120 and mixed on 5120x17408, which keep the default;
//   kTsShort (NP = 128, every CTA's range at most 10 stages): one issuer with
//     three stage slots instead of two with two: ~1 us faster on 6144x5120 and
//     5120x6144 (7-8 stages per CTA), 3-5 us slower on longer ranges.
constexpr int kTsDefault = 0, kTsWhole = 1, kTsShort = 2;

template <int NP, int VAR = kTsDefault>
struct TsCfg {
  static constexpr int ROWS = 128;
  static constexpr int SG = 4;                     // groups per stage
  static constexpr int C_BYTES = ROWS * SG * 32;   // codes, 128 B per row
  static constexpr int SB_BYTES = ROWS * 8 * 2;    // 8 groups of scales (or biases) per row
  static constexpr int CSLOT_BYTES = C_BYTES + 2 * SB_BYTES;
  static constexpr int X_BOX_BYTES = NP * 128;     // one 64-K box of x
  static constexpr int XSLOT_BYTES = SG * X_BOX_BYTES;
  static constexpr int RING_BUDGET = 225 * 1024;   // shared memory for the two rings
  // dequantizer warpgroups = A stage slots; at NP = 128 two, so that TMEM holds
  // a second accumulator: one thread issues at most one M=128 K=16 MMA per
  // ~68 ns whatever N is, so a single issuer would bound a stage at ~1.1 us
  static constexpr int WGS = NP == 128 ? (VAR == kTsShort ? 3 : 2) : (VAR == kTsWhole ? 2 : 3);
  static constexpr int NI = NP == 128 ? (VAR == kTsShort ? 1 : 2)                 // MMA issuers,
                                      : ((NP <= 32 || VAR == kTsWhole) ? 4 : 2);  // one accumulator each
  static constexpr int GPI = SG / NI;              // groups per issuer
  static constexpr int NX = NP <= 32 ? 4 : (NP == 64 ? 3 : 2);  // x slots
  static constexpr int NC_FIT = (RING_BUDGET - NX * XSLOT_BYTES) / CSLOT_BYTES;
  static constexpr int NC = (NC_FIT > 12 ? 12 : NC_FIT) / WGS * WGS;  // codes slots, a multiple of WGS
  static constexpr int X_AREA = NC * CSLOT_BYTES;
  static constexpr int STAGE_AREA = X_AREA + NX * XSLOT_BYTES;
  static constexpr int ACC_COLS = (NI * NP + 31) / 32 * 32;  // one set of NI accumulators
  // two accumulator sets when TMEM has room: segment k+1 accumulates while the
  // epilogue reads segment k
  static constexpr int NB = 2 * ACC_COLS + WGS * SG * 32 <= 512 ? 2 : 1;
  static constexpr int A_COL0 = NB * ACC_COLS;      // accumulators in [0, NB ACC_COLS), A slots after
  static constexpr int GA = 32;                    // per group: 64 bf16 weights per row
  static constexpr int TMEM_COLS = 512;
  static constexpr int CODES_WARP = 4, X_WARP = 5, DQ_WARP0 = 8;  // epilogue: warps 0-3
  static constexpr int THREADS = (NI > 2 ? 22 : 20) * 32;
  // epilogue: CW accumulator columns (tokens) per step; the step's bf16 outputs
  // are staged in shared memory and leave as 16-byte chunks of y rows
  static constexpr int CW = NI > 2 ? 8 : 16;
  static constexpr int Y_STAGE = CW * ROWS * 2;
  static constexpr size_t SMEM = (size_t)STAGE_AREA + 1024 + 1024 + Y_STAGE;
  static_assert(NC >= WGS && A_COL0 + WGS * SG * GA <= TMEM_COLS, "ring depths and TMEM columns");
  static_assert(CSLOT_BYTES % 1024 == 0 && XSLOT_BYTES % 1024 == 0, "slot alignment (128-byte swizzle atoms)");
  static_assert(SMEM <= 227 * 1024, "shared memory per CTA");
};

struct TsArgs {
  const uint16_t *scales, *biases;
  float *partials;     // [tiles][maxp][NP][128], part 0 unused
  uint32_t *flags;     // [tiles][maxp], zero between calls
  long long U;
  int M, N, K, ldy, P, nst, maxp;
  // Output over `world` GPUs: yp[p] is rank p's y at this rank's first column
  // (world 1: yp[0] is y); sig[p] is rank p's signal block (gather.cuh).
  int world, rank;
  uint16_t *yp[kMaxGatherRanks];
  uint32_t *sig[kMaxGatherRanks];
};

template <int NP, int VAR>
__global__ void __launch_bounds__(TsCfg<NP, VAR>::THREADS, 1)
qmm_ts_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_w,
              const __grid_constant__ CUtensorMap tmap_s, const __grid_constant__ CUtensorMap tmap_b, TsArgs a) {
  using C = TsCfg<NP, VAR>;
  extern __shared__ unsigned char smem_raw[];
  unsigned char *smem =
      reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::STAGE_AREA);
  uint16_t *ystage = reinterpret_cast<uint16_t *>(smem + C::STAGE_AREA + 1024);  // [CW][ROWS] bf16
  uint64_t *full_c = bars;                       // [NC] codes + scales + biases landed
  uint64_t *free_c = bars + C::NC;               // [NC] dequantizers have loaded the slot
  uint64_t *full_x = bars + 2 * C::NC;           // [NX] x landed
  uint64_t *free_x = full_x + C::NX;             // [NX] MMAs that read the slot are done
  uint64_t *a_full = free_x + C::NX;             // [WGS] stage written into TMEM
  uint64_t *a_empty = a_full + C::WGS;           // [WGS] MMAs done with the stage slot
  uint64_t *acc_full = a_empty + C::WGS;         // [NB] segment accumulated in set b
  uint64_t *acc_empty = acc_full + C::NB;        // [NB] set b read by the epilogue
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_empty + C::NB);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const Part part{a.U, a.P, a.nst};
  const int c = blockIdx.x;
  const long long u0 = part.start(c);
  const int L = (int)(part.start(c + 1) - u0);  // stages of this CTA
  const int G = a.K / 64;
  // G % 8 != 0: the scale rows' pitch (2G bytes) is not a multiple of 16, which
  // TMA tiles require; the dequantizers then load their row's scales and
  // biases directly (odd shapes only; model shapes have K % 512 == 0).
  const bool sb_direct = (G % 8) != 0;
  // (tile, stage within the tile) of local stage li; loops advance it with step()
  auto unit = [&](int li, int &tile, int &st) {
    const long long u = u0 + li;
    tile = (int)(u / a.nst);
    st = (int)(u - (long long)tile * a.nst);
  };
  auto step = [&](int &tile, int &st, int by) {
    st += by;
    while (st >= a.nst) { st -= a.nst; ++tile; }
  };

  auto cslot = [&](int s) { return smem + (size_t)s * C::CSLOT_BYTES; };
  auto xslot = [&](int s) { return smem + C::X_AREA + (size_t)s * C::XSLOT_BYTES; };
  // codes (and scales, biases) of local stage li into codes slot `slot`
  auto issue_codes = [&](int li, int slot) {
    int tile, st;
    unit(li, tile, st);
    const int gs = st * C::SG, n0 = tile * C::ROWS;
    unsigned char *cs = cslot(slot);
    mbar_arrive_expect_tx(&full_c[slot], C::C_BYTES + (sb_direct ? 0 : 2 * C::SB_BYTES));
    tma_load_2d(cs, &tmap_w, gs * 8, n0, &full_c[slot]);
    if (!sb_direct) {
      const int gb = gs & ~7;  // 8-group box containing this stage's groups
      tma_load_2d(cs + C::C_BYTES, &tmap_s, gb, n0, &full_c[slot]);
      tma_load_2d(cs + C::C_BYTES + C::SB_BYTES, &tmap_b, gb, n0, &full_c[slot]);
    }
  };
  const int first_loads = L < C::NC ? L : C::NC;

  if (warp == C::CODES_WARP && lane == 0) {
    for (int s = 0; s < C::NC; ++s) {
      mbar_init(&full_c[s], 1);
      mbar_init(&free_c[s], 4);  // the 4 warps of the stage's warpgroup
    }
    for (int s = 0; s < C::NX; ++s) {
      mbar_init(&full_x[s], 1);
      mbar_init(&free_x[s], C::NI);  // every MMA issuer
    }
    for (int b = 0; b < C::WGS; ++b) {
      mbar_init(&a_full[b], 4);      // the 4 warps of the owning warpgroup
      mbar_init(&a_empty[b], C::NI);  // every MMA issuer
    }
    for (int b = 0; b < C::NB; ++b) {
      mbar_init(&acc_full[b], C::NI);
      mbar_init(&acc_empty[b], 4);  // the epilogue warps
    }
    fence_mbar_init();
    fence_proxy_async_smem();
    // the weights, scales and biases are constant: the first ring's worth of
    // them streams while TMEM is allocated and the other roles start
    tma_prefetch_desc(&tmap_w);
    if (!sb_direct) {
      tma_prefetch_desc(&tmap_s);
      tma_prefetch_desc(&tmap_b);
    }
    for (int li = 0; li < first_loads; ++li) issue_codes(li, li);
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == C::CODES_WARP) {
    // ---------------- TMA producer of the codes ring (its first NC stages were
    // issued before the CTA-wide barrier)
    if (lane == 0) {
      Ring ring;
      ring.slot = first_loads % C::NC;
      ring.phase = first_loads == C::NC ? 1u : 0u;
      int issued = first_loads;
      for (int li = first_loads; li < L; ++li, ring.next(C::NC)) {
        if (!mbar_wait(&free_c[ring.slot], ring.phase ^ 1u)) break;
        issue_codes(li, ring.slot);
        issued = li + 1;
      }
      // the next kernel on the stream may start its CTAs once every CTA here
      // has issued its last weight load (it waits for this grid before
      // touching anything this grid writes); triggering at the start parked
      // the small decoder kernels' CTAs beside this one for its whole run
      griddep_launch_dependents();
      // drain: every issued load has landed before the CTA can exit
      for (int i = (issued > C::NC ? issued - C::NC : 0); i < issued; ++i) {
        const unsigned long long t0 = globaltimer_ns();
        while (!mbar_try_wait(&full_c[i % C::NC], (i / C::NC) & 1)) {
          if (globaltimer_ns() - t0 > kWaitLimitNs) { record_status(TSB_ETIMEOUT); break; }
        }
      }
    }
  } else if (warp == C::X_WARP) {
    // ---------------- TMA producer of the x ring; x may be the previous
    // kernel's output
    if (elect_one()) {
      tma_prefetch_desc(&tmap_x);
      Ring ring;
      int issued = 0;
      int tile, st;
      unit(0, tile, st);
      griddep_wait();
      for (int li = 0; li < L; ++li, ring.next(C::NX), step(tile, st, 1)) {
        if (li >= C::NX && !mbar_wait(&free_x[ring.slot], ring.phase ^ 1u)) break;
        const int gs = st * C::SG;
        unsigned char *xt = xslot(ring.slot);
        mbar_arrive_expect_tx(&full_x[ring.slot], C::XSLOT_BYTES);
#pragma unroll
        for (int gl = 0; gl < C::SG; ++gl)
          tma_load_2d(xt + gl * C::X_BOX_BYTES, &tmap_x, (gs + gl) * 64, 0, &full_x[ring.slot]);
        issued = li + 1;
      }
      for (int i = (issued > C::NX ? issued - C::NX : 0); i < issued; ++i) {
        const unsigned long long t0 = globaltimer_ns();
        while (!mbar_try_wait(&full_x[i % C::NX], (i / C::NX) & 1)) {
          if (globaltimer_ns() - t0 > kWaitLimitNs) { record_status(TSB_ETIMEOUT); break; }
        }
      }
    }
  } else if ((warp == 6 || warp == 7 || warp == 20 || warp == 21) &&
             (warp < 20 ? warp - 6 : warp - 18) < C::NI) {
    // ---------------- MMA issuers: issuer u takes groups [u, u+1) * GPI of every
    // stage into accumulator u; one lane each, descriptors built once per stage
    // and advanced by adding the 16-byte-unit offset of each 64-K box and 16-K slice
    const int u = warp < 20 ? warp - 6 : warp - 18;
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16_f32(128, NP);
      bool ok = true, first = true;
      int seg = 0;
      uint32_t dacc = tmem_base + (uint32_t)(u * NP);  // accumulator u of set seg % NB
      Ring ring, aring;
      int tile, st;
      unit(0, tile, st);
      for (int li = 0; li < L && ok; ++li, ring.next(C::NX), aring.next(C::WGS), step(tile, st, 1)) {
        if (li > 0 && st == 0) {
          // a new segment in set seg % NB: the epilogue must have read that set's
          // previous segment (seg - NB)
          if (seg >= C::NB) {
            ok = mbar_wait(&acc_empty[seg % C::NB], (uint32_t)(((seg / C::NB) - 1) & 1));
            if (!ok) break;
          }
          dacc = tmem_base + (uint32_t)((seg % C::NB) * C::ACC_COLS + u * NP);
          first = true;
        }
        ok = mbar_wait(&full_x[ring.slot], ring.phase) && mbar_wait(&a_full[aring.slot], aring.phase);
        if (!ok) break;
        tc_fence_after();
        const int gs = st * C::SG;
        const int gend = min(C::GPI * (u + 1), G - gs);
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
        if (li == L - 1 || st == a.nst - 1) {  // the segment's last stage
          mma_commit(&acc_full[seg % C::NB]);
          ++seg;
        }
      }
    }
    __syncwarp();
  } else if (warp >= C::DQ_WARP0 && warp < C::DQ_WARP0 + 4 * C::WGS) {
    // ---------------- dequantizers (thread = weight row = TMEM lane)
    const int q = warp & 3;
    const int wg = (warp - C::DQ_WARP0) >> 2;  // owns local stages li = wg (mod WGS)
    const int r = q * 32 + lane;
    const uint32_t lane_base = tmem_base + ((uint32_t)(q * 32) << 16);
    bool ok = true;
    // Stage li lives in codes slot li % NC (NC % WGS == 0) and A stage slot
    // li % WGS = wg, so this warpgroup is the only waiter of its slots.
    int cs = wg;
    uint32_t cphase = 0;
    int ai = 0;  // this warpgroup's stage count: phase of its A slot
    uint32_t wt[32];  // one group's 64 dequantized weights (bf16 pairs)
    int tile, st;
    unit(wg, tile, st);
    for (int li = wg; li < L && ok; li += C::WGS, step(tile, st, C::WGS)) {
      ok = warp_wait(&full_c[cs], cphase);
      if (!ok) break;
      const int row = tile * C::ROWS + r;
      const int gs = st * C::SG;
      const int ng = min(C::SG, G - gs);  // uniform
      const unsigned char *cb = cslot(cs);
      // this row's scales and biases of the stage's four groups (8-byte loads)
      uint32_t s_w[2], b_w[2];
      if (sb_direct) {
#pragma unroll
        for (int hw = 0; hw < 2; ++hw) {
          const int ga = gs + 2 * hw;
          const size_t idx = (size_t)row * G + ga;
          const bool v0 = ga < G, v1 = ga + 1 < G;
          s_w[hw] = (v0 ? uint32_t(__ldg(a.scales + idx)) : 0u) |
                    (v1 ? uint32_t(__ldg(a.scales + idx + 1)) << 16 : 0u);
          b_w[hw] = (v0 ? uint32_t(__ldg(a.biases + idx)) : 0u) |
                    (v1 ? uint32_t(__ldg(a.biases + idx + 1)) << 16 : 0u);
        }
      } else {
        const int off = r * 16 + (gs & 7) * 2;  // (gs & 7) is 0 or 4: 8-byte aligned
        const uint2 sv = *reinterpret_cast<const uint2 *>(cb + C::C_BYTES + off);
        const uint2 bv = *reinterpret_cast<const uint2 *>(cb + C::C_BYTES + C::SB_BYTES + off);
        s_w[0] = sv.x; s_w[1] = sv.y; b_w[0] = bv.x; b_w[1] = bv.y;
      }
      // the A slot is free once the MMAs of this warpgroup's previous stage completed
      if (ai > 0 && !warp_wait(&a_empty[wg], (uint32_t)((ai - 1) & 1))) {
        ok = false;
        break;
      }
      tc_fence_after();
      // one group at a time (a rolled loop keeps this role's code small next to
      // the other roles sharing the sub-partition's instruction cache): its
      // eight packed words, dequantized into 32 TMEM columns
      const uint64_t s64 = ((uint64_t)s_w[1] << 32) | s_w[0], b64 = ((uint64_t)b_w[1] << 32) | b_w[0];
#pragma unroll 1
      for (int gl = 0; gl < ng; ++gl) {
        const uint4 v0 = *reinterpret_cast<const uint4 *>(cb + r * 128 + (((2 * gl) ^ (r & 7)) << 4));
        const uint4 v1 = *reinterpret_cast<const uint4 *>(cb + r * 128 + (((2 * gl + 1) ^ (r & 7)) << 4));
        const uint32_t words[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
        const uint32_t sb = (uint32_t)(s64 >> (16 * gl)) & 0xFFFFu;
        const uint32_t bb = (uint32_t)(b64 >> (16 * gl)) & 0xFFFFu;
        const __nv_bfloat162 b2 = u32_as_bf2(bb | (bb << 16));
        uint32_t sp;
        if (sub_scale_pair(sb, sp)) {
#pragma unroll
          for (int wj = 0; wj < 8; ++wj) {
            uint32_t o[4];
            dequant_word_sub(words[wj], u32_as_bf2(sp), b2, o);
            wt[4 * wj + 0] = o[0]; wt[4 * wj + 1] = o[1]; wt[4 * wj + 2] = o[2]; wt[4 * wj + 3] = o[3];
          }
        } else {
          // scales of 2^-5 and above, subnormal, inf or nan: the exact slow form
          const __nv_bfloat162 s2 = u32_as_bf2(sb | (sb << 16));
#pragma unroll
          for (int wj = 0; wj < 8; ++wj) {
            uint32_t o[4];
            dequant_word(words[wj], s2, b2, o);
            wt[4 * wj + 0] = o[0]; wt[4 * wj + 1] = o[1]; wt[4 * wj + 2] = o[2]; wt[4 * wj + 3] = o[3];
          }
        }
        tmem_st32(lane_base + C::A_COL0 + (wg * C::SG + gl) * C::GA, wt);
      }
      // the codes slot is refilled by TMA (async proxy): order these generic-proxy
      // reads before that write, which the mbarrier release alone does not do
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&free_c[cs]);
      // tcgen05.st reads its source registers at issue (wt is reused above); the
      // stores must only have reached TMEM before the issuers are told
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&a_full[wg]);
      ++ai;
      cs += C::WGS;
      if (cs >= C::NC) { cs -= C::NC; cphase ^= 1u; }
    }
  } else if (warp < 4) {
    // ---------------- epilogue: one pass per segment of the CTA's range, 16
    // accumulator columns (tokens) at a time
    const int q = warp;
    const int r = q * 32 + lane;
    const uint32_t lane_base = tmem_base + ((uint32_t)(q * 32) << 16);
    griddep_wait();  // y and the workspace flags/partials are shared with the previous call
    // Gather over GPUs: this call's epoch (the previous call has completed, so
    // its epoch is final). CTA 0 tells every peer that this rank has started
    // it, i.e. that everything before it on this rank's stream (the readers of
    // the previous contents of y) has finished; remote stores into a peer's y
    // wait for that peer's word (once, before this CTA's first y store).
    uint32_t ep = 0;
    bool peers_started = a.world == 1;
    if (a.world > 1) {
      ep = gather_epoch(a.sig, a.world, a.rank);
      if (c == 0 && threadIdx.x == 0) gather_start(a.sig, a.world, a.rank, ep);
    }
    int li = 0, seg = 0;
    int tile, st0;
    unit(0, tile, st0);
    while (li < L) {
      const int seg_len = min(L - li, a.nst - st0);
      const bool whole = st0 == 0 && seg_len == a.nst;
      // issuer u accumulated iff some stage of the segment has a group in its share
      const int max_ng = min(C::SG, G - st0 * C::SG);
      int nacc = 1;
      while (nacc < C::NI && max_ng > nacc * C::GPI) ++nacc;
      int clo = c, parts = 1;
      if (!whole) {
        clo = part.c_lo(tile);
        parts = part.c_hi(tile) - clo + 1;
      }
      const int p = c - clo;  // this CTA's part of the tile
      float *pbase = a.partials + ((size_t)tile * a.maxp) * (NP * 128);
      uint32_t *fbase = a.flags + (size_t)tile * a.maxp;
      if (!warp_wait(&acc_full[seg % C::NB], (uint32_t)((seg / C::NB) & 1))) break;
      tc_fence_after();
      const uint32_t acc_base = lane_base + (uint32_t)((seg % C::NB) * C::ACC_COLS);
      // first part: wait for the later parts (one thread per flag, in parallel),
      // then pull all their partials into the stage area (idle once the last
      // segment is accumulated) with one round of cp.async
      bool staged = false;
      const float *sp = reinterpret_cast<const float *>(smem);
      if (!whole && p == 0) {
        if ((int)threadIdx.x < parts - 1) {
          const unsigned long long t0 = globaltimer_ns();
          while (ld_acquire_gpu(fbase + 1 + threadIdx.x) == 0u) {
            if (globaltimer_ns() - t0 > kWaitLimitNs) { record_status(TSB_ETIMEOUT); break; }
          }
        }
        named_barrier_sync(1, 128);
        __threadfence();
        const size_t bytes = (size_t)(parts - 1) * NP * 512;
        if (bytes <= (size_t)C::STAGE_AREA) {
          staged = true;
          const unsigned char *src = reinterpret_cast<const unsigned char *>(pbase + (size_t)NP * 128);
          const uint32_t dst = smem_addr(smem);
          for (size_t off = (size_t)threadIdx.x * 16; off < bytes; off += 128 * 16)
            cp_async_cg16(dst + (uint32_t)off, src + off);
          cp_async_wait_all();
          named_barrier_sync(1, 128);
        }
      }
      // CW accumulator columns (tokens) at a time, every accumulator's chunk in
      // flight at once behind one wait (8 columns with 4 accumulators keeps it
      // to 32 registers); columns at or past M (padding tokens) are skipped by
      // every part alike
      constexpr int CW = C::CW;
#pragma unroll 1
      for (int c0 = 0; c0 < NP && c0 < a.M; c0 += CW) {
        uint32_t tv[C::NI][CW];
#pragma unroll
        for (int uu = 0; uu < C::NI; ++uu)
          if (uu < nacc) {
            if constexpr (CW == 8) tmem_ld8(acc_base + uu * NP + c0, tv[uu]);
            else tmem_ld16(acc_base + uu * NP + c0, tv[uu]);
          }
        tmem_wait_ld();
        float v[CW];
#pragma unroll
        for (int e = 0; e < CW; ++e) v[e] = __uint_as_float(tv[0][e]);
#pragma unroll
        for (int uu = 1; uu < C::NI; ++uu)
          if (uu < nacc) {
#pragma unroll
            for (int e = 0; e < CW; ++e) v[e] += __uint_as_float(tv[uu][e]);
          }
        if (!whole && p > 0) {
          float *dst = pbase + (size_t)p * (NP * 128) + (size_t)c0 * 128 + r;
#pragma unroll
          for (int e = 0; e < CW; ++e) dst[e * 128] = v[e];
          continue;
        }
        if (staged) {
          for (int pp = 1; pp < parts; ++pp) {
            const float *src = sp + (size_t)(pp - 1) * (NP * 128) + (size_t)c0 * 128 + r;
#pragma unroll
            for (int e = 0; e < CW; ++e) v[e] += src[e * 128];
          }
        } else if (!whole) {
          // two parts' chunks in flight per round (L2 hits, one latency each)
          constexpr int PU = 2;
          for (int pp0 = 1; pp0 < parts; pp0 += PU) {
            float t[PU][CW];
#pragma unroll
            for (int q2 = 0; q2 < PU; ++q2)
              if (pp0 + q2 < parts) {
                const float *src = pbase + (size_t)(pp0 + q2) * (NP * 128) + (size_t)c0 * 128 + r;
#pragma unroll
                for (int e = 0; e < CW; ++e) t[q2][e] = __ldcg(src + e * 128);
              }
#pragma unroll
            for (int q2 = 0; q2 < PU; ++q2)
              if (pp0 + q2 < parts) {
#pragma unroll
                for (int e = 0; e < CW; ++e) v[e] += t[q2][e];
              }
          }
        }
        if (!peers_started) {
          if (threadIdx.x == 0) wait_peers(a.sig[a.rank], a.world, a.rank, ep);
          named_barrier_sync(1, 128);
          peers_started = true;
        }
        // bf16 outputs through shared memory: each thread holds one column of CW
        // tokens; y rows go out in 16-byte chunks (eight columns of a token),
        // to every rank's y
#pragma unroll
        for (int e = 0; e < CW; ++e) ystage[e * C::ROWS + r] = float_to_bf16_bits(v[e]);
        named_barrier_sync(1, 128);
        const int ntok = min(CW, a.M - c0);
        for (int i = threadIdx.x; i < ntok * (C::ROWS / 8); i += 128) {
          const int e = i / (C::ROWS / 8), ch = i % (C::ROWS / 8);
          const uint4 u = *reinterpret_cast<const uint4 *>(ystage + e * C::ROWS + ch * 8);
          for (int pp = 0; pp < a.world; ++pp)
            *reinterpret_cast<uint4 *>(a.yp[pp] + (size_t)(c0 + e) * a.ldy + (size_t)tile * C::ROWS + ch * 8) = u;
        }
        named_barrier_sync(1, 128);
      }
      // the accumulators are read: the issuers may start the next segment
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[seg % C::NB]);
      if (!whole && p > 0) {
        // publish this part: its partial above, then its flag
        __threadfence();
        named_barrier_sync(1, 128);
        if (threadIdx.x == 0) st_release_gpu(fbase + p, 1u);
      } else if (!whole) {
        // leave the flags clear for the next call
        named_barrier_sync(1, 128);
        for (int pp = 1 + (int)threadIdx.x; pp < parts; pp += 128) fbase[pp] = 0u;
      }
      li += seg_len;
      ++seg;
      step(tile, st0, seg_len);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
  if (a.world > 1 && threadIdx.x == 0) gather_finish(a.sig, a.world, a.rank, gridDim.x);
}

// Grid and workspace of one call.
struct TsPlan {
  long long U;
  int P, nst, tiles, maxp;
  size_t flag_bytes, part_bytes;
};

template <int NP>
TsPlan plan_ts(int M, int N, int K) {
  (void)M;
  const SkPlan sk = plan_stream_k(N, K, NP == 128);
  TsPlan p;
  p.U = sk.U;
  p.P = sk.P;
  p.nst = sk.nst;
  p.tiles = sk.tiles;
  p.maxp = sk.maxp;
  p.flag_bytes = kFlagRegionBytes;  // tiles * maxp flags must fit: checked at launch
  p.part_bytes = (size_t)p.tiles * p.maxp * NP * 128 * sizeof(float);
  return p;
}

template <int NP, int VAR = kTsDefault>
int launch_ts(const uint16_t *x, const uint32_t *w, const uint16_t *s, const uint16_t *b, uint16_t *y, int M, int N,
              int K, int ldy, void *ws, size_t ws_bytes, const GatherSpec *gs, cudaStream_t st) {
  using C = TsCfg<NP, VAR>;
  const TsPlan plan = plan_ts<NP>(M, N, K);
  if ((size_t)plan.tiles * plan.maxp * sizeof(uint32_t) > kFlagRegionBytes) return TSB_EUNSUPPORTED;
  if (!ws || ws_bytes < plan.flag_bytes + plan.part_bytes) return TSB_EWORKSPACE;
  if (!aligned(ws, 256)) return TSB_EINVAL;
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
    if (cudaFuncSetAttribute(qmm_ts_kernel<NP, VAR>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::SMEM) !=
        cudaSuccess)
      return TSB_ECUDA;
    attr_dev = dev;
  }
  TsArgs a;
  a.scales = s;
  a.biases = b;
  if (gs) {
    a.world = gs->world;
    a.rank = gs->rank;
    for (int p = 0; p < kMaxGatherRanks; ++p) {
      a.yp[p] = p < gs->world ? static_cast<uint16_t *>(gs->y[p]) + gs->col0 : nullptr;
      a.sig[p] = p < gs->world ? static_cast<uint32_t *>(gs->sig[p]) : nullptr;
    }
  } else {
    a.world = 1;
    a.rank = 0;
    for (int p = 0; p < kMaxGatherRanks; ++p) { a.yp[p] = nullptr; a.sig[p] = nullptr; }
    a.yp[0] = y;
  }
  a.flags = static_cast<uint32_t *>(ws);
  a.partials = reinterpret_cast<float *>(static_cast<unsigned char *>(ws) + plan.flag_bytes);
  a.U = plan.U;
  a.M = M; a.N = N; a.K = K; a.ldy = ldy;
  a.P = plan.P;
  a.nst = plan.nst;
  a.maxp = plan.maxp;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(plan.P, 1, 1);
  cfg.blockDim = dim3(C::THREADS, 1, 1);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = st;
  // Programmatic dependent launch: CTAs start on SMs as the previous kernel's
  // CTAs exit, and stream weights while it finishes. The first part of a split
  // tile waits for the later parts, which become resident as SMs free up (P <=
  // #SM, one CTA per SM; the previous kernel never waits on this one), so every
  // wait ends; a cooperative launch would hold the grid until all SMs are free.
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, qmm_ts_kernel<NP, VAR>, tx, tw, tsc, tbi, a);
  return e == cudaSuccess ? TSB_OK : TSB_ECUDA;
}

}  // namespace

// Workspace of the verify path: completion flags (zero between calls) and the
// float partials of split tiles.
size_t qmm_ts_workspace_bytes(int M, int N, int K) {
  TsPlan p;
  if (M <= 16) p = plan_ts<16>(M, N, K);
  else if (M <= 32) p = plan_ts<32>(M, N, K);
  else if (M <= 64) p = plan_ts<64>(M, N, K);
  else p = plan_ts<128>(M, N, K);
  return p.flag_bytes + p.part_bytes;
}

// M in [1, 128]: tokens padded to a multiple of 16 for the MMA's N.
int qmm_ts(const uint16_t *x, const uint32_t *w, const uint16_t *s, const uint16_t *b, uint16_t *y, int M, int N,
           int K, int ldy, void *ws, size_t ws_bytes, const GatherSpec *gs, cudaStream_t st) {
  if (M <= 16) return launch_ts<16>(x, w, s, b, y, M, N, K, ldy, ws, ws_bytes, gs, st);
  if (M <= 32) return launch_ts<32>(x, w, s, b, y, M, N, K, ldy, ws, ws_bytes, gs, st);
  if (M <= 64) {
    if (plan_ts<64>(M, N, K).tiles > sm_count())
      return launch_ts<64, kTsWhole>(x, w, s, b, y, M, N, K, ldy, ws, ws_bytes, gs, st);
    return launch_ts<64>(x, w, s, b, y, M, N, K, ldy, ws, ws_bytes, gs, st);
  }
  const TsPlan p = plan_ts<128>(M, N, K);
  if ((p.U + p.P - 1) / p.P <= 10) return launch_ts<128, kTsShort>(x, w, s, b, y, M, N, K, ldy, ws, ws_bytes, gs, st);
  return launch_ts<128>(x, w, s, b, y, M, N, K, ldy, ws, ws_bytes, gs, st);
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
