// Tree-mask flash attention on tcgen05, for bf16 KV and both 8-bit KV formats.
// Same contract as the reference's tree_flash (mlx-tree-spec
// src/mlx_tree_spec/tree_flash.py:151-196; visibility at 40-45) and the same
// split-KV partial format and combine kernel as attn.cu.
//
// CTA = (request b, KV head, block of 128 packed query rows, key split). The
// G*T query rows of a KV head (row = head_local * T + node) are contiguous in
// q [B, Hq, T, D], so one 2D TMA box brings them; rows past the KV head's G*T
// are computed and dropped.
//   warp 0     TMA: Q once (four 64-wide D boxes, 128-byte swizzle, staged in
//              two V slots). bf16: K tiles of 64 keys through a three-stage
//              ring. 8-bit: the raw K and V tiles (codes, plus the MLX scales
//              and biases) through a five-stage ring of 1D bulk copies, in the
//              order the MMAs consume them (K0, then K_{j+1}, V_j).
//   warp 6     bf16: TMA of V tiles through a four-stage ring. K and V have
//              their own producers so a K load never queues behind a V slot
//              that waits for O += P V.
//   warps 6-13 8-bit: convert each raw tile into the same swizzled bf16 tile
//              the MMAs read (two-stage K and V rings): MLX s*q + b rounded to
//              bf16 (as mlx dequantize), reference int8 exact in bf16 with its
//              row scales applied outside the matmuls (tree_flash.py:14-19,
//              86-100); rows past n_kv are written as zeros.
//   warp 1     MMA: S_j = Q K_j^T with Q from TMEM (A operand) and K from shared
//              memory (K-major, M=128, N=64, K=256), so a tile reads only K from
//              shared memory; O += P_j V_j with P_j from TMEM and V_j from shared
//              memory as an MN-major operand (M=128, N=256, K=64). S_{j+1} is
//              issued before O += P_j V_j so scores overlap the softmax.
//   warps 2-5  copy Q into TMEM once; then softmax, one thread per query row
//              (= TMEM lane): scores -> scale, ancestor mask, online max/sum in
//              the exp2 domain -> P as bf16 written over the first 32 columns of
//              its own score buffer. O is rescaled in TMEM only when the running
//              max grows by more than 2^8 (values stay bounded in between),
//              after the previous P V has completed. Epilogue: O / l -> bf16
//              out, or normalised partials plus (max, sum) for the combine.
// TMEM (512 columns): O [0, 256), Q [256, 384), S0 [384, 448), S1 [448, 512);
// P_j lives in S_{j&1} [0, 32). S_{j+2} overwrites P_j only after O += P_j V_j:
// it is issued after that MMA, and tcgen05.mma operations of one thread run in
// issue order.
// Rows of the cache at or past n_kv never reach the output, whatever they hold
// (even NaN): their scores are masked and their V rows are zero in shared
// memory when O += P V reads them.
#include "sm100.cuh"

namespace tsb {

namespace {

constexpr int TC_KT = 64;                       // keys per tile
constexpr int TC_D = 256;
constexpr int TC_QBOX = 128 * 128;              // one 64-wide D box of 128 rows (bytes)
constexpr int TC_KVBOX = TC_KT * 128;           // one 64-wide D box of 64 keys
constexpr int TC_Q_BYTES = 4 * TC_QBOX;         // 64 KB
constexpr int TC_KV_BYTES = 4 * TC_KVBOX;       // 32 KB per bf16 K or V tile
constexpr uint32_t TC_O = 0, TC_Q = 256, TC_S0 = 384;
constexpr float TC_RESCALE_LOG2 = 8.f;
constexpr int TC_RAW_CODES = TC_KT * TC_D;      // 16 KB: one tile of 8-bit codes
constexpr int TC_NSC = 8;                       // reference-format row-scale ring (tiles)
constexpr int TC_NCONV = 8;                     // converter warps (8-bit formats): two per SM sub-partition
constexpr int TC_MAX_SMEM = 227 * 1024;

template <int FMT>
struct TcCfg {
  static constexpr bool Q8 = FMT != TSB_KV_BF16;
  static constexpr bool MLX = FMT == TSB_KV_MLX_Q8_G64;
  static constexpr bool REF = FMT == TSB_KV_REF_Q8_ROW;
  static constexpr int NK = Q8 ? 2 : 3;          // bf16 K tiles in flight
  static constexpr int NV = Q8 ? 2 : 4;          // bf16 V tiles in flight
  static constexpr int Q_SLOT = Q8 ? 0 : 2;      // V slots Q_SLOT, Q_SLOT+1 stage Q
  static constexpr int NR = Q8 ? 5 : 0;          // raw 8-bit tiles in flight
  // raw stage: codes [64][256] u8, then (MLX) scales [64][4] and biases [64][4] bf16
  static constexpr int RAW_STAGE = MLX ? TC_RAW_CODES + 2 * TC_KT * 8 : TC_RAW_CODES;
  // reference format: key and value row scales of TC_NSC tiles, [TC_NSC][2][64] float
  static constexpr int SC_BYTES = REF ? TC_NSC * 2 * TC_KT * 4 : 0;
  static constexpr int NBARS = 2 + 2 * NK + 2 * NV + 8 + 2 * NR + (REF ? TC_NSC : 0);
  static constexpr int CTRL = Q8 ? 2048 : 1024;  // barriers, TMEM address, masks, parents
  static constexpr int THREADS = Q8 ? (6 + TC_NCONV) * 32 : 224;
  static constexpr size_t SMEM = (size_t)(NK + NV) * TC_KV_BYTES + (size_t)NR * RAW_STAGE + SC_BYTES + CTRL + 1024;
  static_assert((NBARS + 1) * 8 + 64 * 8 + 64 * 4 <= CTRL, "control block");
  static_assert(SMEM <= TC_MAX_SMEM, "shared memory");
};

struct TcArgs {
  const int32_t *parents;
  const unsigned long long *bits;
  const unsigned char *kc, *vc;  // 8-bit codes, D bytes per cache row
  const void *ks, *kb, *vs, *vb; // MLX: bf16 [rows][4]; reference: float [rows] (ks, vs)
  int B, T, Hq, Hkv, n_kv, tail, cap;
  int row_blocks, splits, tiles_per_split;
  float scale_log2;
  uint16_t *out;
  float *lse;
  float *part_o;
  float *part_ml;
};

TSB_HD float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// MN-major operand, 128-byte swizzle: 64-element rows of 128 B along MN, 8-row
// K groups 1024 B apart (SBO), 64-element MN blocks `lbo` bytes apart (LBO).
TSB_HD uint64_t desc_mnmajor_sw128(uint32_t smem_byte_addr, uint32_t lbo) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_byte_addr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Byte k of w as the bits of float 2^23 + byte (exact): the byte becomes the
// low mantissa byte of 0x4B000000.
TSB_HD uint32_t byte_2p23(uint32_t w, uint32_t k) { return prmt(w, 0x4B000000u, 0x7540u | k); }

// 8 MLX codes (u8, low byte first) -> 8 bf16 of s*q + b: q exact in float,
// one float fma, round to nearest even (the dequantization of mlx
// dequantize and of the 8-bit staging in attn.cu).
TSB_HD uint4 dequant8_mlx(uint2 w, float s, float b) {
  uint32_t o[4];
  const uint32_t ws[2] = {w.x, w.y};
#pragma unroll
  for (int h = 0; h < 2; ++h) {
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const float q0 = __uint_as_float(byte_2p23(ws[h], 2 * e)) - 8388608.f;
      const float q1 = __uint_as_float(byte_2p23(ws[h], 2 * e + 1)) - 8388608.f;
      o[2 * h + e] = pack_bf16x2(__fmaf_rn(q0, s, b), __fmaf_rn(q1, s, b));
    }
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// 8 int8 codes -> 8 bf16 holding the same integers (exact): flipping the sign
// bit gives q + 128 as an unsigned byte.
TSB_HD uint4 convert8_s8(uint2 w) {
  uint32_t o[4];
  const uint32_t ws[2] = {w.x ^ 0x80808080u, w.y ^ 0x80808080u};
#pragma unroll
  for (int h = 0; h < 2; ++h) {
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const float q0 = __uint_as_float(byte_2p23(ws[h], 2 * e)) - 8388736.f;  // 2^23 + 128
      const float q1 = __uint_as_float(byte_2p23(ws[h], 2 * e + 1)) - 8388736.f;
      o[2 * h + e] = pack_bf16x2(q0, q1);
    }
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

template <int FMT>
__global__ void __launch_bounds__(TcCfg<FMT>::THREADS, 1)
tree_attn_tc_kernel(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_k,
                    const __grid_constant__ CUtensorMap tmap_v, TcArgs a) {
  using C = TcCfg<FMT>;
  constexpr int NK = C::NK, NV = C::NV, NR = C::NR;
  extern __shared__ unsigned char smem_raw[];
  unsigned char *smem =
      reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char *sK = smem;
  unsigned char *sV = sK + NK * TC_KV_BYTES;
  unsigned char *sQ = sV + C::Q_SLOT * TC_KV_BYTES;
  unsigned char *sRaw = sV + NV * TC_KV_BYTES;
  float *sSc = reinterpret_cast<float *>(sRaw + NR * C::RAW_STAGE);
  uint64_t *bars = reinterpret_cast<uint64_t *>(reinterpret_cast<unsigned char *>(sSc) + C::SC_BYTES);
  uint64_t *q_full = bars, *q_done = bars + 1;
  uint64_t *k_full = bars + 2, *k_free = k_full + NK;
  uint64_t *v_full = k_free + NK, *v_free = v_full + NV;
  uint64_t *s_full = v_free + NV, *s_free = s_full + 2;
  uint64_t *p_full = s_free + 2, *p_free = p_full + 2;
  uint64_t *raw_full = p_free + 2, *raw_free = raw_full + NR;  // 8-bit formats
  uint64_t *sc_full = raw_free + NR;                            // reference format, [TC_NSC]
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + C::NBARS);
  unsigned long long *sBits = reinterpret_cast<unsigned long long *>(bars + C::NBARS + 1);  // [T <= 64]
  int32_t *sPar = reinterpret_cast<int32_t *>(sBits + 64);                                 // [T <= 64]

  // Launched as a programmatic dependent: q and the new K/V rows are the
  // previous kernels'. Its own dependents (the split combine) launch as its
  // CTAs exit: an early trigger would park their CTAs beside this kernel's.
  griddep_wait();
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int G = a.Hq / a.Hkv;
  const int R = G * a.T;
  int unit = blockIdx.x;
  const int split = blockIdx.y;
  const int rb = unit % a.row_blocks;
  unit /= a.row_blocks;
  const int kh = unit % a.Hkv;
  const int b = unit / a.Hkv;
  const int n_tiles_total = (a.n_kv + TC_KT - 1) / TC_KT;
  const int j_begin = split * a.tiles_per_split;
  const int j_end = min(n_tiles_total, j_begin + a.tiles_per_split);
  const int nt = j_end - j_begin;
  const int tail_lo = a.n_kv - a.tail;

  if (threadIdx.x == 0) {
    // bf16 tiles are filled by a TMA transaction, 8-bit ones by the converter warps
    const uint32_t fill = C::Q8 ? TC_NCONV : 1;
    mbar_init(q_full, 1);
    mbar_init(q_done, 4);
    for (int i = 0; i < NK; ++i) { mbar_init(&k_full[i], fill); mbar_init(&k_free[i], 1); }
    for (int i = 0; i < NV; ++i) { mbar_init(&v_full[i], fill); mbar_init(&v_free[i], 1); }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 4);
      mbar_init(&p_full[i], 4);
      mbar_init(&p_free[i], 1);
    }
    for (int i = 0; i < NR; ++i) { mbar_init(&raw_full[i], 1); mbar_init(&raw_free[i], TC_NCONV); }
    if (C::REF)
      for (int i = 0; i < TC_NSC; ++i) mbar_init(&sc_full[i], TC_NCONV);
    fence_mbar_init();
    fence_proxy_async_smem();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const size_t kv_row0 = ((size_t)b * a.Hkv + kh) * (size_t)a.cap;

  if (warp == 0) {
    // ---------------- TMA producer
    if (elect_one()) {
      tma_prefetch_desc(&tmap_q);
      if (!C::Q8) {
        tma_prefetch_desc(&tmap_k);
        tma_prefetch_desc(&tmap_v);
      }
      const int qrow = ((b * a.Hq + kh * G) * a.T) + rb * 128;
      mbar_arrive_expect_tx(q_full, TC_Q_BYTES);
#pragma unroll
      for (int d = 0; d < 4; ++d) tma_load_2d(sQ + d * TC_QBOX, &tmap_q, d * 64, qrow, q_full);
      if constexpr (!C::Q8) {
        bool ok = true;
        int j = 0;
        for (; j < nt && ok; ++j) {
          const int key0 = (int)kv_row0 + (j_begin + j) * TC_KT;
          const int st = j % NK;
          if (j >= NK && !mbar_wait(&k_free[st], ((j / NK) - 1) & 1)) { ok = false; break; }
          mbar_arrive_expect_tx(&k_full[st], TC_KV_BYTES);
#pragma unroll
          for (int d = 0; d < 4; ++d)
            tma_load_2d(sK + st * TC_KV_BYTES + d * TC_KVBOX, &tmap_k, d * 64, key0, &k_full[st]);
        }
        // drain: the issued loads have landed before the CTA can exit
        const unsigned long long t0 = globaltimer_ns();
        while (!mbar_try_wait(q_full, 0)) {
          if (globaltimer_ns() - t0 > kWaitLimitNs) { record_status(TSB_ETIMEOUT); break; }
        }
        for (int i = (j > NK ? j - NK : 0); i < j; ++i) {
          const unsigned long long t1 = globaltimer_ns();
          while (!mbar_try_wait(&k_full[i % NK], (i / NK) & 1)) {
            if (globaltimer_ns() - t1 > kWaitLimitNs) { record_status(TSB_ETIMEOUT); break; }
          }
        }
      } else {
        // raw 8-bit tiles, rows [key0, min(key0 + 64, cap)) of this head's cache
        int seq = 0;
        auto load_raw = [&](bool isv, int j) -> bool {
          const int rs = seq % NR;
          if (seq >= NR && !mbar_wait(&raw_free[rs], ((seq / NR) - 1) & 1)) return false;
          const int key0 = (j_begin + j) * TC_KT;
          const int rows = min(TC_KT, a.cap - key0);
          const size_t r0 = kv_row0 + key0;
          unsigned char *dst = sRaw + rs * C::RAW_STAGE;
          const uint32_t bytes = (uint32_t)rows * TC_D + (C::MLX ? 2u * rows * 8u : 0u);
          mbar_arrive_expect_tx(&raw_full[rs], bytes);
          bulk_load(dst, (isv ? a.vc : a.kc) + r0 * TC_D, (uint32_t)rows * TC_D, &raw_full[rs]);
          if (C::MLX) {
            const uint16_t *sc = reinterpret_cast<const uint16_t *>(isv ? a.vs : a.ks);
            const uint16_t *bi = reinterpret_cast<const uint16_t *>(isv ? a.vb : a.kb);
            bulk_load(dst + TC_RAW_CODES, sc + r0 * 4, (uint32_t)rows * 8u, &raw_full[rs]);
            bulk_load(dst + TC_RAW_CODES + TC_KT * 8, bi + r0 * 4, (uint32_t)rows * 8u, &raw_full[rs]);
          }
          ++seq;
          return true;
        };
        bool ok = true;
        for (int j = 0; j < nt && ok; ++j) {
          if (j == 0) ok = load_raw(false, 0);
          if (ok && j + 1 < nt) ok = load_raw(false, j + 1);
          if (ok) ok = load_raw(true, j);
        }
        const unsigned long long t0 = globaltimer_ns();
        while (!mbar_try_wait(q_full, 0)) {
          if (globaltimer_ns() - t0 > kWaitLimitNs) { record_status(TSB_ETIMEOUT); break; }
        }
        for (int i = (seq > NR ? seq - NR : 0); i < seq; ++i) {
          const unsigned long long t1 = globaltimer_ns();
          while (!mbar_try_wait(&raw_full[i % NR], (i / NR) & 1)) {
            if (globaltimer_ns() - t1 > kWaitLimitNs) { record_status(TSB_ETIMEOUT); break; }
          }
        }
      }
    }
  } else if (warp >= 6) {
    if constexpr (!C::Q8) {
    // ---------------- V producer (bf16; warp 6 is the last warp)
    if (elect_one()) {
      bool ok = true;
      int j = 0;
      for (; j < nt && ok; ++j) {
        const int key0 = (int)kv_row0 + (j_begin + j) * TC_KT;
        const int st = j % NV;
        if (j == C::Q_SLOT && !mbar_wait(q_done, 0)) { ok = false; break; }
        if (j >= NV && !mbar_wait(&v_free[st], ((j / NV) - 1) & 1)) { ok = false; break; }
        mbar_arrive_expect_tx(&v_full[st], TC_KV_BYTES);
#pragma unroll
        for (int d = 0; d < 4; ++d)
          tma_load_2d(sV + st * TC_KV_BYTES + d * TC_KVBOX, &tmap_v, d * 64, key0, &v_full[st]);
      }
      for (int i = (j > NV ? j - NV : 0); i < j; ++i) {
        const unsigned long long t1 = globaltimer_ns();
        while (!mbar_try_wait(&v_full[i % NV], (i / NV) & 1)) {
          if (globaltimer_ns() - t1 > kWaitLimitNs) { record_status(TSB_ETIMEOUT); break; }
        }
      }
    }
    } else {
    // ---------------- converters (8-bit, warps 6-13): raw tile -> swizzled bf16 tile
    // Thread (warp w, lane l) writes 16-byte chunk l&7 of D box l>>3 (the MLX
    // group) of rows (w-6) + 8i: eight lanes fill one 128-byte row of a box.
    const int r_lo = warp - 6;
    const int grp = lane >> 3, ch = lane & 7;
    const int ct = threadIdx.x - 192;  // 0 .. 32 * TC_NCONV - 1
    int seq = 0;
    auto convert = [&](bool isv, int j) -> bool {
      const int rs = seq % NR;
      uint64_t *full;
      unsigned char *dst;
      if (!isv) {
        const int st = j % NK;
        if (j >= NK && !warp_wait(&k_free[st], ((j / NK) - 1) & 1)) return false;
        dst = sK + st * TC_KV_BYTES;
        full = &k_full[st];
      } else {
        const int st = j % NV;
        if (j == 0 && !warp_wait(q_done, 0)) return false;  // V slots 0-1 stage Q until it is in TMEM
        if (j >= NV && !warp_wait(&v_free[st], ((j / NV) - 1) & 1)) return false;
        dst = sV + st * TC_KV_BYTES;
        full = &v_full[st];
      }
      const int key0 = (j_begin + j) * TC_KT;
      const int nvalid = a.n_kv - key0;  // rows below this are keys
      // reference format: the tile's key (threads 0-63) and value (64-127) row
      // scales, fetched with the K tile, for the softmax warps
      float rsc = 0.f;
      if (C::REF && !isv && ct < 2 * TC_KT) {
        const int r = ct & 63;
        if (r < nvalid) rsc = reinterpret_cast<const float *>(ct < 64 ? a.ks : a.vs)[kv_row0 + key0 + r];
      }
      if (!warp_wait(&raw_full[rs], (seq / NR) & 1)) return false;
      const unsigned char *raw = sRaw + rs * C::RAW_STAGE;
      const uint16_t *rsb = reinterpret_cast<const uint16_t *>(raw + TC_RAW_CODES);
      // batches of CB rows: all loads of a batch first, then the conversions
      // and stores; the batch loop stays rolled (the instruction cache holds
      // the converter and softmax loops of the same sub-partition)
      constexpr int CB = 4, ROWS = TC_KT / TC_NCONV;
      static_assert(TC_KT % TC_NCONV == 0 && ROWS % CB == 0, "converter rows");
#pragma unroll 1
      for (int h = 0; h < ROWS / CB; ++h) {
        uint2 w[CB];
        uint32_t sb[CB], bb[CB];
#pragma unroll
        for (int i = 0; i < CB; ++i) {
          const int r = r_lo + TC_NCONV * (CB * h + i);
          w[i] = make_uint2(0u, 0u);
          sb[i] = 0u;
          bb[i] = 0u;
          if (r < nvalid) {
            w[i] = *reinterpret_cast<const uint2 *>(raw + r * TC_D + lane * 8);
            if (C::MLX) {
              sb[i] = rsb[r * 4 + grp];
              bb[i] = rsb[TC_KT * 4 + r * 4 + grp];
            }
          }
        }
#pragma unroll
        for (int i = 0; i < CB; ++i) {
          const int r = r_lo + TC_NCONV * (CB * h + i);
          uint4 o = make_uint4(0u, 0u, 0u, 0u);
          if (r < nvalid) {
            if (C::MLX)
              o = dequant8_mlx(w[i], __uint_as_float(sb[i] << 16), __uint_as_float(bb[i] << 16));
            else
              o = convert8_s8(w[i]);
          }
          *reinterpret_cast<uint4 *>(dst + grp * TC_KVBOX + r * 128 + ((ch ^ (r & 7)) << 4)) = o;
        }
      }
      if (C::REF && !isv && ct < 2 * TC_KT) sSc[(j % TC_NSC) * 2 * TC_KT + ct] = rsc;
      fence_proxy_async_smem();  // generic writes -> MMA reads; raw slot reads -> TMA refill
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&raw_free[rs]);
        mbar_arrive(full);
        if (C::REF && !isv) mbar_arrive(&sc_full[j % TC_NSC]);
      }
      ++seq;
      return true;
    };
    bool ok = true;
    for (int j = 0; j < nt && ok; ++j) {
      if (j == 0) ok = convert(false, 0);
      if (ok && j + 1 < nt) ok = convert(false, j + 1);
      if (ok) ok = convert(true, j);
    }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer
    const uint32_t idesc_s = idesc_bf16_f32(128, TC_KT);
    const uint32_t idesc_o = idesc_bf16_f32(128, TC_D) | (1u << 16);  // B (V) MN-major
    bool ok = warp_wait(q_done, 0);
    auto issue_s = [&](int j) -> bool {
      const int s = j % NK, sb = j & 1;
      if (!warp_wait(&k_full[s], (j / NK) & 1)) return false;
      if (j >= 2 && !warp_wait(&s_free[sb], ((j >> 1) - 1) & 1)) return false;
      tc_fence_after();
      if (elect_one()) {
        const uint32_t kb = smem_addr(sK + s * TC_KV_BYTES);
#pragma unroll
        for (int kk = 0; kk < 16; ++kk) {
          const uint32_t off_k = (kk >> 2) * TC_KVBOX + (kk & 3) * 32;
          mma_ts_f16(tmem + TC_S0 + sb * 64, tmem + TC_Q + kk * 8, desc_kmajor_sw128(kb + off_k), idesc_s,
                     kk > 0 ? 1u : 0u);
        }
        mma_commit(&s_full[sb]);
        mma_commit(&k_free[s]);
      }
      __syncwarp();
      return true;
    };
    auto issue_pv = [&](int j) -> bool {
      const int s = j % NV, pb = j & 1;
      if (!warp_wait(&v_full[s], (j / NV) & 1)) return false;
      if (!warp_wait(&p_full[pb], (j >> 1) & 1)) return false;
      tc_fence_after();
      if (!C::Q8) {
        // bf16: the TMA tile holds whatever follows row n_kv; zero those V rows
        // (their weights are 0, but 0 * NaN would not be)
        const int first = a.n_kv - (j_begin + j) * TC_KT;
        if (first < TC_KT) {
          unsigned char *vt = sV + s * TC_KV_BYTES;
          for (int i = lane; i < (TC_KT - first) * 32; i += 32) {
            const int r = first + (i >> 5), c = i & 31;
            *reinterpret_cast<uint4 *>(vt + (c >> 3) * TC_KVBOX + r * 128 + ((c & 7) << 4)) = make_uint4(0u, 0u, 0u, 0u);
          }
          fence_proxy_async_smem();
          __syncwarp();
        }
      }
      if (elect_one()) {
        const uint32_t vb = smem_addr(sV + s * TC_KV_BYTES);
#pragma unroll
        for (int kk = 0; kk < TC_KT / 16; ++kk) {
          mma_ts_f16(tmem + TC_O, tmem + TC_S0 + pb * 64 + kk * 8, desc_mnmajor_sw128(vb + kk * 2048, TC_KVBOX),
                     idesc_o, (j > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(&v_free[s]);
        mma_commit(&p_free[pb]);  // completes after this and every earlier MMA
      }
      __syncwarp();
      return true;
    };
    if (ok && nt > 0) ok = issue_s(0);
    for (int j = 0; j < nt && ok; ++j) {
      if (j + 1 < nt) ok = issue_s(j + 1);
      if (ok) ok = issue_pv(j);
    }
  } else if (warp >= 2 && warp <= 5) {
    // ---------------- softmax / epilogue (thread = query row = TMEM lane)
    // node masks, from the parent array (staged in shared memory) or given;
    // built here, off the producers' path, while the first scores compute
    {
      const int st = threadIdx.x - 64;  // 0..127
      if (st < a.T) sPar[st] = a.parents ? a.parents[(size_t)b * a.T + st] : 0;
      named_barrier_sync(1, 128);
      if (st < a.T) {
        unsigned long long m = 0;
        if (a.parents) {
          int j = st;
          bool okp = true;
          for (int steps = 0; steps <= a.T && j != -1; ++steps) {
            m |= 1ull << j;
            const int pj = sPar[j];
            if (!(pj == -1 || (pj >= 0 && pj < j))) { okp = false; break; }
            j = pj;
          }
          if (!okp) m = 0;
        } else {
          m = a.bits[(size_t)b * a.T + st];
        }
        sBits[st] = m;
      }
      named_barrier_sync(1, 128);
    }
    const int q = warp & 3;
    const int r = q * 32 + lane;
    const int gr = rb * 128 + r;
    const bool row_valid = gr < R;
    const int node = row_valid ? gr % a.T : 0;
    const unsigned long long mybits = sBits[node];
    const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16);
    const float sl2 = a.scale_log2;
    const int n_kv = a.n_kv;
    float m = -INFINITY, l = 0.f;  // running max (log2 domain) and sum
    // Q row r -> TMEM lane r, columns TC_Q + d/2 (the A-operand layout of a K-major
    // M=128 tile); the staging slots then go back to the V ring
    bool ok = warp_wait(q_full, 0);
    if (ok) {
#pragma unroll 1
      for (int bx = 0; bx < 4; ++bx) {
        const unsigned char *row = sQ + bx * TC_QBOX + r * 128;
        uint32_t qv[32];
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const uint4 u = *reinterpret_cast<const uint4 *>(row + ((c ^ (r & 7)) << 4));
          qv[4 * c] = u.x; qv[4 * c + 1] = u.y; qv[4 * c + 2] = u.z; qv[4 * c + 3] = u.w;
        }
        tmem_st32(lane_base + TC_Q + bx * 32, qv);
      }
      tmem_wait_st();
      tc_fence_before();
      fence_proxy_async_smem();  // the staging slots are refilled by TMA or the converters' generic stores
      __syncwarp();
      if (lane == 0) mbar_arrive(q_done);
    }
    for (int j = 0; j < nt && ok; ++j) {
      const int sb = j & 1;
      ok = warp_wait(&s_full[sb], (j >> 1) & 1);
      if (!ok) break;
      tc_fence_after();
      uint32_t sr[64];
      {
        uint32_t (&lo)[32] = *reinterpret_cast<uint32_t (*)[32]>(&sr[0]);
        uint32_t (&hi)[32] = *reinterpret_cast<uint32_t (*)[32]>(&sr[32]);
        tmem_ld32(lane_base + TC_S0 + sb * 64, lo);
        tmem_ld32(lane_base + TC_S0 + sb * 64 + 32, hi);
      }
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_free[sb]);
      const float *ksc = sSc + (j % TC_NSC) * 2 * TC_KT;  // reference format: key, then value scales
      if (C::REF) {
        // scores of int8 keys times the keys' row scales
        ok = warp_wait(&sc_full[j % TC_NSC], (j / TC_NSC) & 1);
        if (!ok) break;
#pragma unroll
        for (int e = 0; e < 64; e += 4) {
          const float4 k4 = *reinterpret_cast<const float4 *>(ksc + e);
          sr[e] = __float_as_uint(__uint_as_float(sr[e]) * k4.x);
          sr[e + 1] = __float_as_uint(__uint_as_float(sr[e + 1]) * k4.y);
          sr[e + 2] = __float_as_uint(__uint_as_float(sr[e + 2]) * k4.z);
          sr[e + 3] = __float_as_uint(__uint_as_float(sr[e + 3]) * k4.w);
        }
      }
      // mask (only the tail and the last tile need it), then the tile max of the
      // raw scores in eight independent chains; the scale is applied in the exp
      const int key0 = (j_begin + j) * TC_KT;
      if ((key0 + TC_KT > tail_lo) || (key0 + TC_KT > n_kv)) {
#pragma unroll
        for (int e = 0; e < 64; ++e) {
          const int key = key0 + e;
          bool vis = key < n_kv;
          if (vis && key >= tail_lo) vis = (mybits >> (key - tail_lo)) & 1ull;
          if (!vis) sr[e] = __float_as_uint(-INFINITY);
        }
      }
      float mx8[8];
#pragma unroll
      for (int c = 0; c < 8; ++c) mx8[c] = __uint_as_float(sr[c]);
#pragma unroll
      for (int e = 8; e < 64; ++e) mx8[e & 7] = fmaxf(mx8[e & 7], __uint_as_float(sr[e]));
      const float traw = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                               fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
      const float tmax = traw * sl2;  // scale > 0: max commutes with it
      // P V_{j-2} is done (S_j, written after it, is complete); waiting here
      // keeps every p_free wait below at most one phase behind.
      if (j >= 2) {
        ok = warp_wait(&p_free[sb], ((j >> 1) - 1) & 1);
        if (!ok) break;
      }
      // lazy rescale: move the reference max only when it grows by > 2^8
      const bool grow = tmax > m + TC_RESCALE_LOG2;
      if (__any_sync(0xffffffffu, grow)) {
        const float m_new = grow ? tmax : m;
        const float alpha = (m == -INFINITY) ? 0.f : ex2(m - m_new);
        if (j > 0) {  // O holds earlier tiles: wait for P V_{j-1} (and all before), then scale O in place
          ok = warp_wait(&p_free[sb ^ 1], ((j - 1) >> 1) & 1);
          if (!ok) break;
          tc_fence_after();
#pragma unroll 1
          for (int c = 0; c < TC_D; c += 32) {
            uint32_t o[32];
            tmem_ld32(lane_base + TC_O + c, o);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
            tmem_st32(lane_base + TC_O + c, o);
          }
          tmem_wait_st();
        }
        l *= alpha;
        m = m_new;
      }
      const float nbase = (m == -INFINITY) ? 0.f : -m;
      uint32_t pk[32];
      float ps[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        const float p0 = ex2(__fmaf_rn(__uint_as_float(sr[2 * e]), sl2, nbase));
        const float p1 = ex2(__fmaf_rn(__uint_as_float(sr[2 * e + 1]), sl2, nbase));
        ps[e & 3] += p0 + p1;
        if (C::REF) {
          // the value rows' scales weight P; the running sum keeps the plain weights
          const float2 v2 = *reinterpret_cast<const float2 *>(ksc + TC_KT + 2 * e);
          pk[e] = pack_bf16x2(p0 * v2.x, p1 * v2.y);
        } else {
          pk[e] = pack_bf16x2(p0, p1);
        }
      }
      l += (ps[0] + ps[1]) + (ps[2] + ps[3]);
      // P_j into TMEM, over the scores it was made from
      tc_fence_after();
      tmem_st32(lane_base + TC_S0 + sb * 64, pk);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[sb]);
    }
    // ---------------- epilogue
    if (ok && nt > 0 && warp_wait(&p_free[(nt - 1) & 1], ((nt - 1) >> 1) & 1)) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const int hl = gr / a.T;
      const size_t orow = ((size_t)b * a.Hq + (size_t)kh * G + hl) * a.T + node;
#pragma unroll 1
      for (int c = 0; c < TC_D; c += 32) {
        uint32_t o[32];
        tmem_ld32(lane_base + TC_O + c, o);
        tmem_wait_ld();
        if (!row_valid) continue;
        if (a.splits == 1) {
          uint32_t pkd[16];
#pragma unroll
          for (int e = 0; e < 16; ++e)
            pkd[e] = pack_bf16x2(__uint_as_float(o[2 * e]) * inv, __uint_as_float(o[2 * e + 1]) * inv);
          uint4 *dst = reinterpret_cast<uint4 *>(a.out + orow * TC_D + c);
          dst[0] = make_uint4(pkd[0], pkd[1], pkd[2], pkd[3]);
          dst[1] = make_uint4(pkd[4], pkd[5], pkd[6], pkd[7]);
          dst[2] = make_uint4(pkd[8], pkd[9], pkd[10], pkd[11]);
          dst[3] = make_uint4(pkd[12], pkd[13], pkd[14], pkd[15]);
        } else {
          const size_t prow = (size_t)split * a.B * a.Hq * a.T + orow;
          float4 *dst = reinterpret_cast<float4 *>(a.part_o + prow * TC_D + c);
#pragma unroll
          for (int e = 0; e < 8; ++e)
            dst[e] = make_float4(__uint_as_float(o[4 * e]) * inv, __uint_as_float(o[4 * e + 1]) * inv,
                                 __uint_as_float(o[4 * e + 2]) * inv, __uint_as_float(o[4 * e + 3]) * inv);
        }
      }
      if (row_valid) {
        if (a.splits == 1) {
          if (a.lse) a.lse[orow] = l > 0.f ? (m + log2f(l)) * 0.69314718055994531f : -INFINITY;
        } else {
          const size_t prow = (size_t)split * a.B * a.Hq * a.T + orow;
          a.part_ml[prow * 2 + 0] = m;
          a.part_ml[prow * 2 + 1] = l;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int FMT>
int launch_fmt(const CUtensorMap &tq, const CUtensorMap &tk, const CUtensorMap &tv, const TcArgs &a,
               cudaStream_t st) {
  using C = TcCfg<FMT>;
  static int attr_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (attr_dev != dev) {
    if (cudaFuncSetAttribute(tree_attn_tc_kernel<FMT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::SMEM) !=
        cudaSuccess)
      return TSB_ECUDA;
    attr_dev = dev;
  }
  const dim3 grid(a.B * a.Hkv * a.row_blocks, a.splits);
  const cudaError_t e = launch_pdl(tree_attn_tc_kernel<FMT>, grid, dim3(C::THREADS), (size_t)C::SMEM, st, tq, tk, tv, a);
  return e == cudaSuccess ? TSB_OK : TSB_ECUDA;
}

}  // namespace

// Plan of the tcgen05 path: row blocks of 128 packed query rows, tiles of 64
// keys, splits so that the grid covers the SMs about once.
void plan_attn_tc(int B, int T, int Hq, int Hkv, int n_kv, int &row_blocks, int &splits, int &tiles_per_split) {
  const int R = (Hq / Hkv) * T;
  row_blocks = (R + 127) / 128;
  const int units = B * Hkv * row_blocks;
  const int n_tiles = (n_kv + TC_KT - 1) / TC_KT;
  int s = sm_count() / units;  // one CTA per SM (TMEM 512 columns): stay within one wave
  if (s > n_tiles / 4) s = n_tiles / 4;
  if (s > 256) s = 256;  // the combine kernel holds at most 256 split weights per row
  if (s < 1) s = 1;
  tiles_per_split = (n_tiles + s - 1) / s;
  splits = (n_tiles + tiles_per_split - 1) / tiles_per_split;
}

// Whether a call can take the tcgen05 path. The MLX format's scales and biases
// arrive by 1D bulk copies of 8 bytes per row: they need 16-byte aligned bases
// and an even capacity (every tile then starts on a 16-byte boundary and holds
// an even number of rows).
bool attn_tc_supported(int kv_format, int cap, const void *ks, const void *kb, const void *vs, const void *vb) {
  if (kv_format == TSB_KV_BF16 || kv_format == TSB_KV_REF_Q8_ROW) return true;
  if (kv_format != TSB_KV_MLX_Q8_G64) return false;
  return cap % 2 == 0 && aligned(ks, 16) && aligned(kb, 16) && aligned(vs, 16) && aligned(vb, 16);
}

int launch_attn_tc(int kv_format, const uint16_t *q, const void *k, const void *ks, const void *kb, const void *v,
                   const void *vs, const void *vb, const int32_t *parents, const unsigned long long *bits, int B,
                   int T, int Hq, int Hkv, int n_kv, int tail, int cap, float scale, uint16_t *out, float *lse,
                   float *part_o, float *part_ml, cudaStream_t st) {
  TcArgs a;
  a.parents = parents;
  a.bits = bits;
  a.kc = reinterpret_cast<const unsigned char *>(k);
  a.vc = reinterpret_cast<const unsigned char *>(v);
  a.ks = ks; a.kb = kb; a.vs = vs; a.vb = vb;
  a.B = B; a.T = T; a.Hq = Hq; a.Hkv = Hkv; a.n_kv = n_kv; a.tail = tail; a.cap = cap;
  plan_attn_tc(B, T, Hq, Hkv, n_kv, a.row_blocks, a.splits, a.tiles_per_split);
  a.scale_log2 = scale * 1.4426950408889634f;
  a.out = out;
  a.lse = lse;
  a.part_o = part_o;
  a.part_ml = part_ml;
  CUtensorMap tq, tk, tv;
  if (make_tmap_2d(&tq, q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, TC_D, (uint64_t)B * Hq * T, TC_D * 2, 64, 128,
                   CU_TENSOR_MAP_SWIZZLE_128B) != TSB_OK)
    return TSB_ECUDA;
  if (kv_format == TSB_KV_BF16) {
    if (make_tmap_2d(&tk, k, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, TC_D, (uint64_t)B * Hkv * cap, TC_D * 2, 64, TC_KT,
                     CU_TENSOR_MAP_SWIZZLE_128B) != TSB_OK)
      return TSB_ECUDA;
    if (make_tmap_2d(&tv, v, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, TC_D, (uint64_t)B * Hkv * cap, TC_D * 2, 64, TC_KT,
                     CU_TENSOR_MAP_SWIZZLE_128B) != TSB_OK)
      return TSB_ECUDA;
    return launch_fmt<TSB_KV_BF16>(tq, tk, tv, a, st);
  }
  // the 8-bit kernels read K and V with 1D bulk copies; the maps are unused
  if (kv_format == TSB_KV_MLX_Q8_G64) return launch_fmt<TSB_KV_MLX_Q8_G64>(tq, tq, tq, a, st);
  if (kv_format == TSB_KV_REF_Q8_ROW) return launch_fmt<TSB_KV_REF_Q8_ROW>(tq, tq, tq, a, st);
  return TSB_EUNSUPPORTED;
}

unsigned int status_attn_tc(bool reset) {
  unsigned int v = 0;
  cudaMemcpyFromSymbol(&v, g_device_status, sizeof(v));
  if (reset && v) {
    const unsigned int z = 0;
    cudaMemcpyToSymbol(g_device_status, &z, sizeof(z));
  }
  return v;
}

}  // namespace tsb
