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
// to 16), a K range of whole stages; split-K CTAs of one row tile form a
// cluster and reduce through distributed shared memory. Warp roles:
//   warp 0    TMA producer of the codes ring: per stage (4 groups = 256 K)
//             the codes of the 128 rows (32 words each, 128-byte swizzle) and
//             their scales and biases (8-group boxes). A slot is refilled as
//             soon as the dequantizers have loaded its words into registers.
//   warp 10   TMA producer of the x ring: x for the stage (four 64-K boxes of
//             NP rows, 128-byte swizzle, rows >= M zero-filled by TMA); a slot
//             is refilled when the MMAs that read it have completed.
//   warp 1    MMA issuer: per group 4 tcgen05.mma (M=128, N=NP, K=16) on the
//             scaled codes plus 4 on the group's bias (below); A from TMEM,
//             B = x from shared memory, f32 accumulator in TMEM.
//   warps 2-9 dequantizers, two warpgroups (warpgroup w takes groups 2w and
//             2w+1 of each stage; thread = weight row = TMEM lane): codes ->
//             bf16(s*q) -> tcgen05.st into a ring of per-group A slots; the
//             store of one group drains while the next is dequantized. Then
//             the epilogue (TMEM -> registers -> bf16 y, or split-K partials).
//
// Arithmetic: y = sum_g [ sum_{k in g} bf16(s q_k) x_k + b sum_{k in g} x_k ].
// The first term needs one bf16x2 fma per pair of weights (fma(128+q, s,
// -128 s), exactly rounded). The second is the reference's `b * sum x` term
// (qmm_packed.py:14-16, 424-425) done on the tensor core: an 8-column TMEM
// block holding b in all 16 K positions multiplies each 16-wide K slice of x.
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
  // ring depths; two CTAs per SM up to NP = 64 (shared memory and 256 TMEM
  // columns each), one for NP = 128
  static constexpr int NC = NP == 64 ? 2 : 3;      // codes slots
  static constexpr int NX = NP == 16 ? 4 : 2;      // x slots
  static constexpr int X_AREA = NC * CSLOT_BYTES;
  static constexpr int STAGE_AREA = X_AREA + NX * XSLOT_BYTES;
  static constexpr int A_COL0 = NP < 32 ? 32 : NP; // D in columns [0, NP), A slots after
  static constexpr int GA = 40;                    // per group slot: 32 columns s*q, 8 columns bias
  static constexpr int TMEM_COLS = NP <= 64 ? 256 : 512;
  static constexpr int NAG_FIT = (TMEM_COLS - A_COL0) / GA;
  static constexpr int NAG = NAG_FIT > 8 ? 8 : NAG_FIT;  // ring of per-group A slots in TMEM
  static constexpr int THREADS = 352;
  static constexpr size_t SMEM = (size_t)STAGE_AREA + 1024 + 1024;
  static_assert(NAG >= 4, "A ring");
  static_assert(CSLOT_BYTES % 1024 == 0 && XSLOT_BYTES % 1024 == 0, "slot alignment (128-byte swizzle atoms)");
  static_assert(NP * 512 <= STAGE_AREA, "split-K partials fit in the stage area");
  static_assert(SMEM <= (NP <= 64 ? 112 * 1024 : 200 * 1024), "shared memory per CTA");
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
__global__ void __launch_bounds__(352, NP <= 64 ? 2 : 1)
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
  uint64_t *a_full = free_x + C::NX;             // [NAG] group written into TMEM
  uint64_t *a_empty = a_full + C::NAG;           // [NAG] MMA done with the slot
  uint64_t *acc_full = a_empty + C::NAG;
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
      mbar_init(&free_c[s], 8);  // every dequantizer warp
    }
    for (int s = 0; s < C::NX; ++s) {
      mbar_init(&full_x[s], 1);
      mbar_init(&free_x[s], 1);
    }
    for (int b = 0; b < C::NAG; ++b) {
      mbar_init(&a_full[b], 4);  // the 4 warps of the group's warpgroup
      mbar_init(&a_empty[b], 1);
    }
    mbar_init(acc_full, 1);
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

  if (warp == 0 || warp == 10) {
    // ---------------- TMA producers: warp 0 the codes ring, warp 10 the x ring
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
  } else if (warp == 1) {
    // ---------------- MMA issuer
    const uint32_t idesc = idesc_bf16_f32(128, NP);
    bool ok = true;
    Ring ring, aring;
    int gi = 0;
    for (int i = 0; i < nst && ok; ++i, ring.next(C::NX)) {
      ok = warp_wait(&full_x[ring.slot], ring.phase);
      if (!ok) break;
      const int gs = g0 + i * C::SG;
      const uint32_t xs = smem_addr(xslot(ring.slot));
      for (int gl = 0; gl < C::SG && gs + gl < g1; ++gl, ++gi, aring.next(C::NAG)) {
        ok = warp_wait(&a_full[aring.slot], aring.phase);
        if (!ok) break;
        tc_fence_after();
        if (elect_one()) {
          const uint32_t a_grp = tmem_base + C::A_COL0 + aring.slot * C::GA;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t bd = desc_kmajor_sw128(xs + gl * C::X_BOX_BYTES + kk * 32);
            mma_ts_f16(tmem_base, a_grp + kk * 8, bd, idesc, (gi > 0 || kk > 0) ? 1u : 0u);
            mma_ts_f16(tmem_base, a_grp + 32, bd, idesc, 1u);  // + b * (sum of this x slice)
          }
          mma_commit(&a_empty[aring.slot]);
        }
        __syncwarp();
      }
      if (!ok) break;
      if (elect_one()) {
        mma_commit(&free_x[ring.slot]);
        if (i == nst - 1) mma_commit(acc_full);
      }
      __syncwarp();
    }
  } else {
    // ---------------- dequantizers (thread = weight row = TMEM lane)
    const int q = warp & 3;
    const int wg = (warp - 2) >> 2;  // groups 2wg, 2wg+1 of each stage
    const int r = q * 32 + lane;
    const int row = n0 + r;
    const uint32_t lane_base = tmem_base + ((uint32_t)(q * 32) << 16);
    bool ok = true;
    int pend_slot = -1;  // A slot whose TMEM store is in flight
    auto flush = [&]() {
      if (pend_slot >= 0) {
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&a_full[pend_slot]);
        pend_slot = -1;
      }
    };
    // A slots: group gi of the CTA uses slot gi % NAG; this warpgroup's groups
    // are gi = 4i + 2wg + {0, 1}.
    Ring aring;
    aring.slot = (2 * wg) % C::NAG;
    aring.phase = (uint32_t)((2 * wg) / C::NAG) & 1u;
    uint32_t abuf[2][32];
    Ring ring;
    for (int i = 0; i < nst && ok; ++i, ring.next(C::NC)) {
      ok = warp_wait(&full_c[ring.slot], ring.phase);
      if (!ok) break;
      const int gs = g0 + i * C::SG;
      const unsigned char *st = cslot(ring.slot);
      // this row's scales and biases of the two groups (one 32-bit load each)
      uint32_t s_pair, b_pair;
      if (sb_direct) {
        const int ga = gs + 2 * wg;
        const size_t idx = (size_t)row * G + ga;
        const bool v0 = ga < g1, v1 = ga + 1 < g1;
        s_pair = (v0 ? uint32_t(__ldg(scales + idx)) : 0u) | (v1 ? uint32_t(__ldg(scales + idx + 1)) << 16 : 0u);
        b_pair = (v0 ? uint32_t(__ldg(biases + idx)) : 0u) | (v1 ? uint32_t(__ldg(biases + idx + 1)) << 16 : 0u);
      } else {
        const int off = r * 16 + ((gs & 7) + 2 * wg) * 2;
        s_pair = *reinterpret_cast<const uint32_t *>(st + C::C_BYTES + off);
        b_pair = *reinterpret_cast<const uint32_t *>(st + C::C_BYTES + C::SB_BYTES + off);
      }
      // both groups' packed words into registers, then release the codes slot
      uint32_t words2[2][8];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const int chunk = (2 * (2 * wg + h) + c) ^ (r & 7);  // TMA 128-byte swizzle
          const uint4 v = *reinterpret_cast<const uint4 *>(st + r * 128 + chunk * 16);
          words2[h][4 * c + 0] = v.x; words2[h][4 * c + 1] = v.y; words2[h][4 * c + 2] = v.z; words2[h][4 * c + 3] = v.w;
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&free_c[ring.slot]);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int gl = 2 * wg + h;
        const int gi = i * C::SG + gl;
        if (ok && gs + gl < g1) {  // uniform across the warpgroup
          const uint32_t(&words)[8] = words2[h];
          const uint32_t sbits = h ? (s_pair >> 16) : (s_pair & 0xFFFFu);
          const uint32_t bbits = h ? (b_pair >> 16) : (b_pair & 0xFFFFu);
          const uint16_t nsb = float_to_bf16_bits(bf16_bits_to_float((uint16_t)sbits) * -128.f);  // exact
          const __nv_bfloat162 s2 = u32_as_bf2(sbits | (sbits << 16));
          const __nv_bfloat162 ns2 = u32_as_bf2(uint32_t(nsb) | (uint32_t(nsb) << 16));
          uint32_t(&a)[32] = abuf[h];
#pragma unroll
          for (int wj = 0; wj < 8; ++wj) {
            uint32_t o[4];
            dequant_word_scaled(words[wj], s2, ns2, o);
            a[4 * wj + 0] = o[0]; a[4 * wj + 1] = o[1]; a[4 * wj + 2] = o[2]; a[4 * wj + 3] = o[3];
          }
          // hand the previous group to the MMA, then make sure this slot is free
          flush();
          if (gi >= C::NAG && !warp_wait(&a_empty[aring.slot], aring.phase ^ 1u)) {
            ok = false;
          } else {
            tc_fence_after();
            const uint32_t bb = bbits | (bbits << 16);
            const uint32_t bias_cols[8] = {bb, bb, bb, bb, bb, bb, bb, bb};
            const uint32_t a_grp = lane_base + C::A_COL0 + aring.slot * C::GA;
            tmem_st32(a_grp, a);
            tmem_st8(a_grp + 32, bias_cols);
            pend_slot = aring.slot;
          }
        }
        aring.next(C::NAG);
      }
      aring.next(C::NAG);  // the other warpgroup's two groups
      aring.next(C::NAG);
    }
    flush();
    // ---------------- epilogue part 1: accumulator -> y or partials
    if (wg == 0 && ok && nst > 0 && warp_wait(acc_full, 0)) {
      tc_fence_after();
      float *red = reinterpret_cast<float *>(smem);  // [NP][128], the stage area is free now
#pragma unroll
      for (int c0 = 0; c0 < NP; c0 += 16) {
        uint32_t v[16];
        tmem_ld16(lane_base + c0, v);
        tmem_wait_ld();
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
  const int per_sm = NP <= 64 ? 2 : 1;  // resident CTAs per SM (TMEM and shared memory)
  int splits = (per_sm * sm_count() + tiles / 2) / tiles;
  if (splits < 1) splits = 1;
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
