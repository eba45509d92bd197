// Prefill 4-bit quantized matmul (M >= a few hundred rows): tcgen05 GEMM with
// the weight dequantized into shared memory. B200 counterpart of the
// reference's prefill_kernel (mlx-tree-spec src/mlx_tree_spec/qmm_packed.py:
// 561-725), which dequantizes a BN x BK weight block into threadgroup memory
// per K step (`T(float(q) * s + b)`, :635) and runs MLX's NAX tiles on it.
//
// CTA tile: 256 x-rows (two M=128 MMAs) by BN weight rows, K step 64 (= one
// quantization group). Warp roles:
//   warp 0     TMA producer: x tiles (two 128x64 bf16 boxes, 128-byte swizzle)
//              and the packed codes of BN rows x 8 words per K step.
//   warp 1     MMA issuer: 2 x 4 tcgen05.mma (M=128, N=BN, K=16) per K step
//              into two TMEM accumulators (2*BN columns), commit frees the stage.
//   warps 2-9  dequantizers: codes (shared) -> bf16 s*q + b -> the B tile in
//              the K-major 128-byte-swizzle layout the MMA reads; then the
//              epilogue: TMEM -> registers -> bf16 -> y.
// Per stage the codes arrive with the x tile; the B tile of a stage is
// rewritten only after the MMA that read it committed (the producer waits on
// the stage's `empty` barrier before it refills the codes the dequantizers
// wait on).
//
// Dequantization per packed word (8 codes): two masks and one shift split the
// nibbles, byte permutes place code | 0x4300 (= bf16 128 + q) in natural order,
// an exact bf16 subtract of 128 gives q, and one bf16x2 fma rounds s*q + b once
// to bf16 (dequant_word). Here each thread dequantizes one word of each of its
// rows, so the per-group scale-pair form of the verify kernel (dequant_word_sub)
// would recompute its scale pair and branch per word; measured 23% slower at
// M = 4096. The reference rounds q*s + b to float32 first (qmm_packed.py:635);
// the two agree unless that float32 rounding lands exactly on a bf16 rounding
// midpoint, never for quantizer-produced weights.
#include "gather.cuh"

namespace tsb {

namespace {

// The split tail's float parts start this far into the qmm workspace (after the
// verify path's count region, which stays untouched and zero).
constexpr size_t kGemmPartOffset = 64 * 1024;

template <int BN>
struct GemmCfg {
  static constexpr int BM = 256;
  static constexpr int BK = 64;
  static constexpr int A_BYTES = 128 * BK * 2;  // one M half
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int C_BYTES = BN * 32;       // 8 words per row
  static constexpr int STAGE_BYTES = 2 * A_BYTES + B_BYTES + C_BYTES;
  static constexpr int STAGES = BN == 256 ? 3 : 4;
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int THREADS = 320;
  static constexpr int DQ_THREADS = 256;
  static constexpr int ROWS_PER_DQ = BN * 8 / DQ_THREADS;  // (row, word) items per dequant thread
  static constexpr size_t SMEM = (size_t)STAGES * STAGE_BYTES + 1024 /*barriers*/ + 1024 /*align*/;
};

// The output: yp[0] = y on one GPU; over `world` GPUs yp[p] is rank p's y at
// this rank's first column and sig[p] its signal block (gather.cuh): every tile
// is stored into every rank's y, so the N-sharded prefill needs no separate
// all-gather.
struct GemmOut {
  int world, rank;
  uint16_t *yp[kMaxGatherRanks];
  uint32_t *sig[kMaxGatherRanks];
};

// Which tiles a launch covers: CTA b takes linear tile tile0 + b / ksplit
// (M-tile fastest, so consecutive CTAs share a weight tile) and the K range
// [j num_k / ksplit, (j+1) num_k / ksplit) with j = b % ksplit. ksplit = 1: the
// whole tile, written to y (every rank's y when gathered). ksplit > 1: the
// range's float sums stored into part[b] ([256][BN] per CTA); the tail kernel
// below adds a tile's ksplit parts in a fixed order (deterministic results) and
// writes y. The workspace may hold anything on entry.
struct GemmTiles {
  int tile0, mtiles, ksplit;
  float *part;
};

template <int BN>
__global__ void __launch_bounds__(320, 1)
qmm_gemm_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_w,
                const uint16_t *__restrict__ scales, const uint16_t *__restrict__ biases,
                const GemmOut o, const GemmTiles tl, int M, int N, int K, int ldy) {
  using C = GemmCfg<BN>;
  extern __shared__ unsigned char smem_raw[];
  unsigned char *smem = reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::STAGES * C::STAGE_BYTES);
  uint64_t *full_x = bars;
  uint64_t *full_c = bars + C::STAGES;
  uint64_t *full_b = bars + 2 * C::STAGES;
  uint64_t *empty = bars + 3 * C::STAGES;
  uint64_t *acc_full = bars + 4 * C::STAGES;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 4 * C::STAGES + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int tidx = blockIdx.x / tl.ksplit, kpart = blockIdx.x % tl.ksplit;
  const int tile = tl.tile0 + tidx;
  const int m0 = (tile % tl.mtiles) * C::BM;
  const int n0 = (tile / tl.mtiles) * BN;
  const int G = K / 64;
  const int k0 = (int)((long long)G * kpart / tl.ksplit), k1 = (int)((long long)G * (kpart + 1) / tl.ksplit);
  const int num_k = k1 - k0;  // K steps of this CTA: i in [k0, k1), ring position i - k0
  const bool partial = tl.ksplit > 1;
  const bool gathered = o.world > 1 && !partial;

  // the next kernel of the call (the split tail) may start as this one's CTAs exit
  if (threadIdx.x == 0) griddep_launch_dependents();
  // gathered output: this call's epoch (the previous kernel on the stream has
  // completed); the first CTA tells the peers that this rank has started it
  const uint32_t ep = gathered ? gather_epoch(o.sig, o.world, o.rank) : 0u;
  if (gathered && blockIdx.x == 0 && threadIdx.x == 0) gather_start(o.sig, o.world, o.rank, ep);
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full_x[s], 1);
      mbar_init(&full_c[s], 1);
      mbar_init(&full_b[s], C::DQ_THREADS / 32);
      mbar_init(&empty[s], 1);
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

  auto stage_ptr = [&](int s) { return smem + (size_t)s * C::STAGE_BYTES; };

  if (warp == 0) {
    // ---------------- TMA producer
    if (elect_one()) {
      tma_prefetch_desc(&tmap_x);
      tma_prefetch_desc(&tmap_w);
      int issued = 0;
      for (int i = 0; i < num_k; ++i) {
        const int s = i % C::STAGES;
        if (i >= C::STAGES) {
          if (!mbar_wait(&empty[s], ((i / C::STAGES) - 1) & 1)) break;
        }
        unsigned char *st = stage_ptr(s);
        const int kc = (k0 + i) * C::BK;
        mbar_arrive_expect_tx(&full_x[s], 2 * C::A_BYTES);
        tma_load_2d(st, &tmap_x, kc, m0, &full_x[s]);
        tma_load_2d(st + C::A_BYTES, &tmap_x, kc, m0 + 128, &full_x[s]);
        mbar_arrive_expect_tx(&full_c[s], C::C_BYTES);
        tma_load_2d(st + 2 * C::A_BYTES + C::B_BYTES, &tmap_w, (k0 + i) * 8, n0, &full_c[s]);
        issued = i + 1;
      }
      // drain: every issued load has landed before the CTA can exit
      for (int i = (issued > C::STAGES ? issued - C::STAGES : 0); i < issued; ++i) {
        const int s = i % C::STAGES;
        const uint32_t par = (i / C::STAGES) & 1;
        const unsigned long long t0 = globaltimer_ns();
        while (!(mbar_try_wait(&full_x[s], par) && mbar_try_wait(&full_c[s], par))) {
          if (globaltimer_ns() - t0 > kWaitLimitNs) { record_status(TSB_ETIMEOUT); break; }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer
    const uint32_t idesc = idesc_bf16_f32(128, BN);
    bool ok = true;
    for (int i = 0; i < num_k && ok; ++i) {
      const int s = i % C::STAGES;
      const uint32_t par = (i / C::STAGES) & 1;
      ok = warp_wait(&full_x[s], par) && warp_wait(&full_b[s], par);
      if (!ok) break;
      tc_fence_after();
      if (elect_one()) {
        unsigned char *st = stage_ptr(s);
        const uint32_t a0 = smem_addr(st), a1 = smem_addr(st + C::A_BYTES), b = smem_addr(st + 2 * C::A_BYTES);
#pragma unroll
        for (int kk = 0; kk < C::BK / 16; ++kk) {
          const uint32_t acc = (i > 0 || kk > 0) ? 1u : 0u;
          const uint64_t bd = desc_kmajor_sw128(b + kk * 32);
          mma_ss_f16(tmem_base, desc_kmajor_sw128(a0 + kk * 32), bd, idesc, acc);
          mma_ss_f16(tmem_base + BN, desc_kmajor_sw128(a1 + kk * 32), bd, idesc, acc);
        }
        mma_commit(&empty[s]);
        if (i == num_k - 1) mma_commit(acc_full);
      }
      __syncwarp();
    }
  } else {
    // ---------------- dequantizers, then epilogue
    const int t = threadIdx.x - 64;  // 0..255
    const int j = t & 7;             // word within the group
    const int rsub = t >> 3;         // 0..31
    uint32_t sb_cur[C::ROWS_PER_DQ], sb_nxt[C::ROWS_PER_DQ];  // (s | b << 16)
    auto load_sb = [&](int g, uint32_t (&dst)[C::ROWS_PER_DQ]) {
#pragma unroll
      for (int it = 0; it < C::ROWS_PER_DQ; ++it) {
        const size_t idx = (size_t)(n0 + it * 32 + rsub) * G + g;
        dst[it] = uint32_t(__ldg(scales + idx)) | (uint32_t(__ldg(biases + idx)) << 16);
      }
    };
    load_sb(k0, sb_cur);
    bool ok = true;
    for (int i = 0; i < num_k; ++i) {
      const int s = i % C::STAGES;
      const uint32_t par = (i / C::STAGES) & 1;
      if (i + 1 < num_k) load_sb(k0 + i + 1, sb_nxt);
      if (!warp_wait(&full_c[s], par)) { ok = false; break; }
      unsigned char *st = stage_ptr(s);
      const uint32_t *codes = reinterpret_cast<const uint32_t *>(st + 2 * C::A_BYTES + C::B_BYTES);
      unsigned char *btile = st + 2 * C::A_BYTES;
#pragma unroll
      for (int it = 0; it < C::ROWS_PER_DQ; ++it) {
        const int r = it * 32 + rsub;
        const uint32_t w = codes[r * 8 + j];
        const uint32_t sbv = sb_cur[it];
        const __nv_bfloat162 b2 = u32_as_bf2((sbv >> 16) | (sbv & 0xFFFF0000u));
        uint32_t o[4];
        dequant_word(w, u32_as_bf2((sbv & 0xFFFFu) | (sbv << 16)), b2, o);
        const uint32_t off = (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((j ^ (r & 7)) << 4));
        *reinterpret_cast<uint4 *>(btile + off) = make_uint4(o[0], o[1], o[2], o[3]);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&full_b[s]);
#pragma unroll
      for (int it = 0; it < C::ROWS_PER_DQ; ++it) sb_cur[it] = sb_nxt[it];
    }
    // ---------------- epilogue. Every epilogue warp goes through it, even after
    // a failed (timed-out) wait, so that the named barrier below always
    // completes; only the stores depend on success.
    const bool good = warp_wait(acc_full, 0) && ok;
    tc_fence_after();
    // stores into a peer's y wait until that peer has started this call
    if (good && gathered) wait_peers(o.sig[o.rank], o.world, o.rank, ep);
    {
      const int q = warp & 3;                 // TMEM lane quadrant this warp may access
      const int half = (warp - 2) >> 2;       // which half of the columns
      if (partial && good) {
        // this K range's float sums, stored as they are read
        float *pt = tl.part + (size_t)blockIdx.x * C::BM * BN;
        for (int mh = 0; mh < 2; ++mh) {
          const int row = m0 + mh * 128 + q * 32 + lane;
          for (int c = half * (BN / 2); c < (half + 1) * (BN / 2); c += 16) {
            uint32_t r[16];
            tmem_ld16(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(mh * BN + c), r);
            tmem_wait_ld();
            if (row < M) {
              float4 *dst = reinterpret_cast<float4 *>(pt + (size_t)(row - m0) * BN + c);
#pragma unroll
              for (int e = 0; e < 4; ++e)
                dst[e] = make_float4(__uint_as_float(r[4 * e]), __uint_as_float(r[4 * e + 1]),
                                     __uint_as_float(r[4 * e + 2]), __uint_as_float(r[4 * e + 3]));
            }
          }
        }
      } else if (!partial) {
        // bf16 tile staged in shared memory (the pipeline's stages are free:
        // every MMA has completed), then written out as whole rows, 16 bytes a
        // thread, so that a warp's stores to y (a peer's y over NVLink) are
        // contiguous runs of 256 or 512 bytes
        constexpr int PITCH = BN * 2 + 16;    // staged row pitch: +16 B keeps 16-byte stores conflict-free
        static_assert(C::BM * PITCH <= C::STAGES * C::STAGE_BYTES, "staging tile");
        unsigned char *stg = smem;
        fence_proxy_async_smem();
        for (int mh = 0; mh < 2; ++mh) {
          const int rr = mh * 128 + q * 32 + lane;
          for (int c = half * (BN / 2); c < (half + 1) * (BN / 2); c += 16) {
            uint32_t r[16];
            tmem_ld16(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(mh * BN + c), r);
            tmem_wait_ld();
            uint32_t p[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) p[e] = pack_bf16x2(__uint_as_float(r[2 * e]), __uint_as_float(r[2 * e + 1]));
            uint4 *d = reinterpret_cast<uint4 *>(stg + rr * PITCH + c * 2);
            d[0] = make_uint4(p[0], p[1], p[2], p[3]);
            d[1] = make_uint4(p[4], p[5], p[6], p[7]);
          }
        }
        named_barrier_sync(1, C::DQ_THREADS);
        constexpr int CPR = BN / 8;           // 16-byte chunks per row
        for (int i = t; i < C::BM * CPR; i += C::DQ_THREADS) {
          const int rr = i / CPR, ch = i % CPR;
          const int row = m0 + rr;
          if (good && row < M) {
            const uint4 v = *reinterpret_cast<const uint4 *>(stg + rr * PITCH + ch * 16);
            for (int pp = 0; pp < o.world; ++pp)
              *reinterpret_cast<uint4 *>(o.yp[pp] + (size_t)row * ldy + n0 + ch * 8) = v;
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
  if (gathered && threadIdx.x == 0) gather_finish(o.sig, o.world, o.rank, gridDim.x);
  // a split launch starts before the whole-tile launch completes; it completes
  // only after it, so that the tail kernel (which waits for this grid) and its
  // gather handshakes come after both
  if (partial) griddep_wait();
}

// Finishes the tiles of a split tail: the ksplit float parts of each tile
// ([tiles][ksplit][256][BN]), added in order, -> bf16 y (every rank's y when
// gathered). Thread = 8 columns of one row: a warp reads and writes contiguous
// row segments; BN / 8 CTAs of 256 threads per tile.
template <int BN>
__global__ void __launch_bounds__(256)
qmm_gemm_tail_kernel(const float *part, int tile0, int mtiles, int ksplit, const GemmOut o, int M, int ldy) {
  griddep_wait();  // the parts written by the previous kernel are complete
  constexpr int CPR = BN / 8;  // 8-column chunks per row
  const int ti = blockIdx.x / CPR;
  const int i = (blockIdx.x % CPR) * 256 + threadIdx.x;  // (row, chunk) item of the tile
  const int rr = i / CPR, ch = i % CPR;
  const int tile = tile0 + ti;
  const int m0 = (tile % mtiles) * 256, n0 = (tile / mtiles) * BN;
  const int row = m0 + rr;
  const bool gathered = o.world > 1;
  const uint32_t ep = gathered ? gather_epoch(o.sig, o.world, o.rank) : 0u;
  if (gathered && blockIdx.x == 0 && threadIdx.x == 0) gather_start(o.sig, o.world, o.rank, ep);
  if (gathered) wait_peers(o.sig[o.rank], o.world, o.rank, ep);
  if (row < M) {
    const float *src = part + ((size_t)ti * ksplit * 256 + rr) * BN + ch * 8;
    float4 a = ld_cg_v4(src), b = ld_cg_v4(src + 4);
    for (int j = 1; j < ksplit; ++j) {
      const float *q = src + (size_t)j * 256 * BN;
      const float4 a2 = ld_cg_v4(q), b2 = ld_cg_v4(q + 4);
      a.x += a2.x; a.y += a2.y; a.z += a2.z; a.w += a2.w;
      b.x += b2.x; b.y += b2.y; b.z += b2.z; b.w += b2.w;
    }
    const uint4 v = make_uint4(pack_bf16x2(a.x, a.y), pack_bf16x2(a.z, a.w), pack_bf16x2(b.x, b.y),
                               pack_bf16x2(b.z, b.w));
    for (int pp = 0; pp < o.world; ++pp)
      *reinterpret_cast<uint4 *>(o.yp[pp] + (size_t)row * ldy + n0 + ch * 8) = v;
  }
  __syncthreads();
  if (gathered && threadIdx.x == 0) gather_finish(o.sig, o.world, o.rank, gridDim.x);
}

// The split tail: when the tiles fill the SMs' last wave poorly (e.g. 320 tiles of
// 256 x 256 at M = 4096, N = 5120 leave 24 tiles for a third wave of 148 SMs),
// the full waves run as usual and the remaining tiles are split along K over the
// SMs (float parts in the workspace), then finished by the tail kernel.
// tail = 0: one launch.
struct GemmPlan {
  int mtiles, tiles, full, tail, ksplit;
};

template <int BN>
GemmPlan plan_gemm(int M, int N, int K) {
  GemmPlan p;
  p.mtiles = (M + 255) / 256;
  p.tiles = p.mtiles * (N / BN);
  const int sms = sm_count();
  const int rem = p.tiles % sms;
  const int steps = K / 64;
  p.full = p.tiles;
  p.tail = 0;
  p.ksplit = 1;
  // the tiles left for a poorly filled last wave (all of them when there are
  // fewer tiles than SMs)
  const int left = p.tiles < sms ? p.tiles : rem;
  if (left > 0 && 2 * left <= sms) {
    int ks = sms / left;
    if (ks > 16) ks = 16;
    if (ks > steps / 4) ks = steps / 4;
    if (ks >= 3) {  // a 2-way split of a half-empty wave measured slower than none
      p.full = p.tiles - left;
      p.tail = left;
      p.ksplit = ks;
    }
  }
  return p;
}

template <int BN>
int launch_gemm(const uint16_t *x, const uint32_t *w, const uint16_t *s, const uint16_t *b, uint16_t *y, int M, int N,
                int K, int ldy, const GatherSpec *gs, void *ws, size_t ws_bytes, cudaStream_t st) {
  using C = GemmCfg<BN>;
  CUtensorMap tx, tw;
  if (make_tmap_2d(&tx, x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)K, (uint64_t)M, (uint64_t)K * 2, 64, 128,
                   CU_TENSOR_MAP_SWIZZLE_128B) != TSB_OK)
    return TSB_ECUDA;
  if (make_tmap_2d(&tw, w, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, (uint64_t)K / 8, (uint64_t)N, (uint64_t)K / 2, 8, BN,
                   CU_TENSOR_MAP_SWIZZLE_NONE) != TSB_OK)
    return TSB_ECUDA;
  static bool attr_set[2] = {false, false};
  bool &done = attr_set[BN == 256 ? 1 : 0];
  if (!done) {
    if (cudaFuncSetAttribute(qmm_gemm_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::SMEM) !=
        cudaSuccess)
      return TSB_ECUDA;
    done = true;
  }
  GemmOut o;
  for (int p = 0; p < kMaxGatherRanks; ++p) { o.yp[p] = nullptr; o.sig[p] = nullptr; }
  if (gs) {
    o.world = gs->world;
    o.rank = gs->rank;
    for (int p = 0; p < gs->world; ++p) {
      o.yp[p] = static_cast<uint16_t *>(gs->y[p]) + gs->col0;
      o.sig[p] = gs->sig[p];
    }
  } else {
    o.world = 1;
    o.rank = 0;
    o.yp[0] = y;
  }
  GemmPlan pl = plan_gemm<BN>(M, N, K);
  // the split tail keeps its parts in the workspace (after the verify path's
  // count region); without one, every tile runs whole
  float *part = nullptr;
  if (pl.tail) {
    const size_t need = kGemmPartOffset + (size_t)pl.tail * pl.ksplit * 256 * BN * sizeof(float);
    if (ws && ws_bytes >= need && aligned(ws, 256))
      part = reinterpret_cast<float *>(static_cast<unsigned char *>(ws) + kGemmPartOffset);
    else
      pl.full = pl.tiles, pl.tail = 0, pl.ksplit = 1;
  }
  GemmTiles whole{0, pl.mtiles, 1, nullptr};
  if (pl.full) {
    qmm_gemm_kernel<BN><<<pl.full, C::THREADS, C::SMEM, st>>>(tx, tw, s, b, o, whole, M, N, K, ldy);
    if (cudaGetLastError() != cudaSuccess) return TSB_ECUDA;
  }
  if (!pl.tail) return TSB_OK;
  // the split launch starts on SMs as the last full wave's CTAs exit (it
  // touches nothing the full tiles write); with no full tiles it is the call's
  // first kernel and waits for the previous work on the stream (x may be its
  // output). The tail kernel follows it either way.
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pl.full ? 1 : 0;
  cfg.stream = st;
  cfg.gridDim = dim3(pl.tail * pl.ksplit, 1, 1);
  cfg.blockDim = dim3(C::THREADS, 1, 1);
  cfg.dynamicSmemBytes = C::SMEM;
  GemmTiles split{pl.full, pl.mtiles, pl.ksplit, part};
  if (cudaLaunchKernelEx(&cfg, qmm_gemm_kernel<BN>, tx, tw, s, b, o, split, M, N, K, ldy) != cudaSuccess)
    return TSB_ECUDA;
  cfg.numAttrs = 1;
  cfg.gridDim = dim3(pl.tail * (BN / 8), 1, 1);
  cfg.blockDim = dim3(256, 1, 1);
  cfg.dynamicSmemBytes = 0;
  if (cudaLaunchKernelEx(&cfg, qmm_gemm_tail_kernel<BN>, (const float *)part, pl.full, pl.mtiles, pl.ksplit, o, M,
                         ldy) != cudaSuccess)
    return TSB_ECUDA;
  return TSB_OK;
}

}  // namespace

int qmm_gemm(const uint16_t *x, const uint32_t *w, const uint16_t *s, const uint16_t *b, uint16_t *y, int M, int N,
             int K, int ldy, const GatherSpec *gs, void *ws, size_t ws_bytes, cudaStream_t st) {
  if (N % 256 == 0) return launch_gemm<256>(x, w, s, b, y, M, N, K, ldy, gs, ws, ws_bytes, st);
  return launch_gemm<128>(x, w, s, b, y, M, N, K, ldy, gs, ws, ws_bytes, st);
}

// Workspace of the prefill path: the split tail's sums (0 when the tiles fill
// the last wave well).
size_t qmm_gemm_workspace_bytes(int M, int N, int K) {
  if (N % 256 == 0) {
    const GemmPlan p = plan_gemm<256>(M, N, K);
    return p.tail ? kGemmPartOffset + (size_t)p.tail * p.ksplit * 256 * 256 * sizeof(float) : 0;
  }
  const GemmPlan p = plan_gemm<128>(M, N, K);
  return p.tail ? kGemmPartOffset + (size_t)p.tail * p.ksplit * 256 * 128 * sizeof(float) : 0;
}

unsigned int status_gemm(bool reset) {
  unsigned int v = 0;
  cudaMemcpyFromSymbol(&v, g_device_status, sizeof(v));
  if (reset && v) {
    const unsigned int z = 0;
    cudaMemcpyToSymbol(g_device_status, &z, sizeof(z));
  }
  return v;
}

}  // namespace tsb
