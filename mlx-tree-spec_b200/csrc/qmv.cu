// Verify-pass 4-bit quantized matrix-vector product for M <= 2 tokens on the
// CUDA cores: the B200 counterpart of the reference's packed GEMV (mlx-tree-spec
// src/mlx_tree_spec/qmv_packed in qmm_packed.py:428-557, chosen for M <= 4 by
// packed_linear.py:10-13), which factors the group affine out of the dot product:
//     sum_k (s q_k + b) x_k = s * sum_k q_k x_k + b * sum_k x_k   (per group of 64).
//
// Why not the tensor cores: at M = 1 the tcgen05 kernel pays a fixed cost of
// several microseconds per call (TMEM, barriers, pipeline fill, stream-K join),
// which dominates small weights. Here every weight byte is read once with
// 16-byte coalesced loads and consumed by integer dot products:
//   - codes: lo = w & 0x0F0F0F0F (codes 0,2,4,6 of the word), hi = (w >> 4) &
//     0x0F0F0F0F (codes 1,3,5,7), three instructions per 8 codes;
//   - x: per (token, 64-K group) a power-of-two c = 2^(5-e) brings the group's
//     largest finite |x| into [32, 64); x c = x1 + x2 / 128 with x1 = rint(x c)
//     and x2 = rint((x c - x1) 128), both in [-64, 64], so both fit int8 and
//     the split is off by at most 2^-13 of the group's largest value (exact for
//     one-hot rows). Made once per CTA into shared memory, permuted to match.
//   - dp4a.u32.s32 sums q x1 and q x2 exactly in int32 (four instructions per
//     8 codes per token), then per group: acc += (s 2^(e-5)) (S1 + S2/128) and,
//     once per group, acc += b X_g (X_g = float sum of the group's x).
// Under one integer-pipe instruction per code, so the kernel is bound by HBM,
// not by issue. Read back through one-hot x rows the result is bf16(f32(q*s +
// b)), the reference's dequantization rule (qmm_packed.py:200, 348, 635).
//
// Work: a persistent grid (one CTA of 16 warps per SM); each warp takes blocks
// of 4 weight rows (grid-stride), each lane 16 bytes (32 codes, half a
// group) of each row per step, x read from shared memory once per step for the
// block's rows; lanes reduce by shuffles at the end. The first steps' weight
// loads are issued before waiting for the previous kernel (weights are
// constant; x is not).
#include "gather.cuh"

namespace tsb {

namespace {

constexpr int kQmvWarps = 16;

// Where the outputs go: yp[p] is rank p's y at this rank's first column (world
// 1: yp[0] is y); sig[p] is rank p's signal block (the handshakes of
// gather.cuh, as in the tcgen05 kernels).
struct QmvOut {
  int world, rank;
  uint16_t *yp[kMaxGatherRanks];
  uint32_t *sig[kMaxGatherRanks];
};
constexpr int kQmvMaxSmem = 200 * 1024;

TSB_HD float pow2i(int k) { return __int_as_float((k + 127) << 23); }  // 2^k, k in [-126, 127]

TSB_HD int dp4a_us(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// Shared memory of a CTA: for each token t, the x pieces [t][piece][word] as
// uint2 {codes 0,2,4,6 ; codes 1,3,5,7} of x1 (piece 0) and x2 (piece 1), then
// per (t, group) the float pair {s-side factor 2^(e-5), X_g}.
template <int MT>
struct QmvSmem {
  static size_t bytes(int K) { return (size_t)MT * 2 * (K / 8) * 8 + (size_t)MT * (K / 64) * 8; }
};

// RW weight rows per warp block, PF 16-byte chunks of each row in flight per
// lane (RW * PF = 8: up to 64 KB of weights in flight per SM).
template <int MT, int RW>
__global__ void __launch_bounds__(kQmvWarps * 32, 1)
qmv_kernel(const uint16_t *__restrict__ x, const uint32_t *__restrict__ w, const uint16_t *__restrict__ scales,
           const uint16_t *__restrict__ biases, const QmvOut o, int N, int K, int ldy) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int W = K / 8, G = K / 64, V = K / 32;  // words, groups, 16-byte chunks per row
  uint2 *xp = reinterpret_cast<uint2 *>(smem);                                   // [MT][2][W]
  float2 *gf = reinterpret_cast<float2 *>(smem + (size_t)MT * 2 * W * 8);        // [MT][G]
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int nblk = N / RW;
  // warp w of CTA c takes the blocks w * gridDim + c + k * nw: consecutive
  // blocks go to different CTAs, so every SM streams even when there are fewer
  // blocks than warps
  const int gw = wid * gridDim.x + blockIdx.x, nw = gridDim.x * kQmvWarps;

  if (threadIdx.x == 0) griddep_launch_dependents();
  // the first block's first chunks in flight before x is ready
  constexpr int PF = 8 / RW;  // chunks per row kept in flight
  uint4 cur[PF][RW];
  int blk = gw;
  auto load_chunks = [&](int b, int v0, uint4 (&dst)[RW]) {
#pragma unroll
    for (int rr = 0; rr < RW; ++rr)
      dst[rr] = v0 < V ? ldg_nc_v4(w + ((size_t)(b * RW + rr) * W) + 4 * (size_t)v0) : make_uint4(0, 0, 0, 0);
  };
  if (blk < nblk) {
#pragma unroll
    for (int i = 0; i < PF; ++i) load_chunks(blk, lane + 32 * i, cur[i]);
  }

  griddep_wait();  // x may be the previous kernel's output
  // Gather over GPUs: this call's epoch (the previous call has completed). CTA 0
  // tells every peer that this rank has started it; stores into a peer's y
  // wait (below, once per CTA) until that peer has started it too.
  const uint32_t ep = o.world > 1 ? gather_epoch(o.sig, o.world, o.rank) : 0u;
  if (o.world > 1 && blockIdx.x == 0 && threadIdx.x == 0) gather_start(o.sig, o.world, o.rank, ep);
  // ---- x -> pieces: 8 threads per (token, group), one 8-element word each
  // (MT G 8 is a multiple of 8 and blockDim of 32: a group's threads are 8
  // consecutive lanes of one warp)
  for (int base = 0; base < MT * G * 8; base += blockDim.x) {
    const int i = base + (int)threadIdx.x;
    const bool ok = i < MT * G * 8;
    const int tg = i >> 3, wl = i & 7;
    const int t = tg / G, g = tg - t * G;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (ok) v = *reinterpret_cast<const uint4 *>(x + (size_t)t * K + 64 * (size_t)g + 8 * wl);
    const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
    float fv[8];
    float mx = 0.f, xs = 0.f;
    int bad = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      fv[2 * k] = __uint_as_float(wv[k] << 16);
      fv[2 * k + 1] = __uint_as_float(wv[k] & 0xFFFF0000u);
      const uint32_t m0 = wv[k] & 0x7FFFu, m1 = (wv[k] >> 16) & 0x7FFFu;
      bad |= (m0 >= 0x7F80u) | (m1 >= 0x7F80u);
      mx = fmaxf(mx, fmaxf(__uint_as_float(m0 << 16), __uint_as_float(m1 << 16)));
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) xs += fv[k];
    // the group's 8 threads: max, any non-finite, and the sum (fixed order)
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) {
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      bad |= __shfl_xor_sync(0xffffffffu, bad, o);
      xs += __shfl_xor_sync(0xffffffffu, xs, o);
    }
    if (!ok) continue;
    int e = 0;  // floor(log2(max |x|)), 0 for an all-zero group
    if (mx > 0.f) {
      const uint32_t bits = __float_as_uint(mx);
      const int ex = (int)(bits >> 23);
      e = ex ? ex - 127 : (31 - __clz((int)bits)) - 149;
    }
    const int a = 5 - e, a1 = a >> 1, a2 = a - a1;  // x c = (x 2^a1) 2^a2
    const float p1 = pow2i(a1), p2 = pow2i(a2);
    if (wl == 0) {
      const int f = e - 5, f1 = f >> 1, f2 = f - f1;  // 1 / c
      gf[t * G + g] = make_float2(bad ? __int_as_float(0x7FC00000) : pow2i(f1) * pow2i(f2), xs);
    }
    uint32_t q1[2] = {0u, 0u}, q2[2] = {0u, 0u};  // {even codes, odd codes}
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      float tv = (fv[k] * p1) * p2;
      if (!(fabsf(tv) <= 64.f)) tv = 0.f;  // inf and nan (the group is marked above)
      const float r1 = rintf(tv);
      const int i1 = (int)r1, i2 = (int)rintf((tv - r1) * 128.f);
      q1[k & 1] |= ((uint32_t)i1 & 0xFFu) << (8 * (k >> 1));
      q2[k & 1] |= ((uint32_t)i2 & 0xFFu) << (8 * (k >> 1));
    }
    const int wi = 8 * g + wl;
    xp[(t * 2 + 0) * W + wi] = make_uint2(q1[0], q1[1]);
    xp[(t * 2 + 1) * W + wi] = make_uint2(q2[0], q2[1]);
  }
  if (o.world > 1 && threadIdx.x == 0) wait_peers(o.sig[o.rank], o.world, o.rank, ep);
  __syncthreads();

  // ---- rows: RW per warp block, 16 bytes of each row per lane and step
  for (; blk < nblk; blk += nw) {
    float acc[RW][MT];
#pragma unroll
    for (int rr = 0; rr < RW; ++rr)
#pragma unroll
      for (int t = 0; t < MT; ++t) acc[rr][t] = 0.f;
    for (int v0 = lane; v0 < V; v0 += 32 * PF) {
#pragma unroll
      for (int i = 0; i < PF; ++i) {
        const int v = v0 + 32 * i;
        uint4 c[RW];
#pragma unroll
        for (int rr = 0; rr < RW; ++rr) c[rr] = cur[i][rr];
        // the chunk PF steps ahead (or the next block's first ones)
        int nb = blk, nv = v + 32 * PF;
        if (nv >= V) { nb = blk + nw; nv = lane + 32 * i; }
        if (nb < nblk) load_chunks(nb, nv, cur[i]);
        if (v >= V) continue;
        const int g = v >> 1;
        // x pieces of this chunk's 4 words, per token
        uint4 xa[MT][2][2];
#pragma unroll
        for (int t = 0; t < MT; ++t)
#pragma unroll
          for (int pc = 0; pc < 2; ++pc) {
            const uint4 *src = reinterpret_cast<const uint4 *>(xp + (t * 2 + pc) * W + 4 * v);
            xa[t][pc][0] = src[0];
            xa[t][pc][1] = src[1];
          }
        float2 gv[MT];
#pragma unroll
        for (int t = 0; t < MT; ++t) gv[t] = gf[t * G + g];
#pragma unroll
        for (int rr = 0; rr < RW; ++rr) {
          const int row = blk * RW + rr;
          const float s = bf16_bits_to_float(__ldg(scales + (size_t)row * G + g));
          const uint32_t cw[4] = {c[rr].x, c[rr].y, c[rr].z, c[rr].w};
          uint32_t lo[4], hi[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            lo[k] = cw[k] & 0x0F0F0F0Fu;
            hi[k] = (cw[k] >> 4) & 0x0F0F0F0Fu;
          }
#pragma unroll
          for (int t = 0; t < MT; ++t) {
            int s1 = 0, s2 = 0;
            const uint32_t x1[8] = {xa[t][0][0].x, xa[t][0][0].y, xa[t][0][0].z, xa[t][0][0].w,
                                    xa[t][0][1].x, xa[t][0][1].y, xa[t][0][1].z, xa[t][0][1].w};
            const uint32_t x2[8] = {xa[t][1][0].x, xa[t][1][0].y, xa[t][1][0].z, xa[t][1][0].w,
                                    xa[t][1][1].x, xa[t][1][1].y, xa[t][1][1].z, xa[t][1][1].w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              s1 = dp4a_us(lo[k], x1[2 * k], s1);
              s1 = dp4a_us(hi[k], x1[2 * k + 1], s1);
              s2 = dp4a_us(lo[k], x2[2 * k], s2);
              s2 = dp4a_us(hi[k], x2[2 * k + 1], s2);
            }
            const float d = (float)s1 + (float)s2 * 0.0078125f;  // exact: |s2| < 2^16
            float a2 = fmaf(s * gv[t].x, d, acc[rr][t]);
            if ((v & 1) == 0) a2 = fmaf(bf16_bits_to_float(__ldg(biases + (size_t)row * G + g)), gv[t].y, a2);
            acc[rr][t] = a2;
          }
        }
      }
    }
    // lanes -> row sums (fixed order), lane rr * MT + t writes
#pragma unroll
    for (int rr = 0; rr < RW; ++rr)
#pragma unroll
      for (int t = 0; t < MT; ++t)
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc[rr][t] += __shfl_xor_sync(0xffffffffu, acc[rr][t], o);
#pragma unroll
    for (int rr = 0; rr < RW; ++rr)
#pragma unroll
      for (int t = 0; t < MT; ++t)
        if (lane == rr * MT + t) {
          const uint16_t v = float_to_bf16_bits(acc[rr][t]);
          for (int p = 0; p < o.world; ++p) o.yp[p][(size_t)t * ldy + blk * RW + rr] = v;
        }
  }
  if (o.world > 1) {
    // every store of this CTA precedes the finish handshake's release
    __syncthreads();
    if (threadIdx.x == 0) gather_finish(o.sig, o.world, o.rank, gridDim.x);
  }
}

template <int MT, int RW>
int launch_qmv(const uint16_t *x, const uint32_t *w, const uint16_t *s, const uint16_t *b, const QmvOut &o, int N,
               int K, int ldy, cudaStream_t st) {
  const size_t smem = QmvSmem<MT>::bytes(K);
  if (smem > (size_t)kQmvMaxSmem) return TSB_EUNSUPPORTED;
  static int attr_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (attr_dev != dev) {
    if (cudaFuncSetAttribute(qmv_kernel<MT, RW>, cudaFuncAttributeMaxDynamicSharedMemorySize, kQmvMaxSmem) !=
        cudaSuccess)
      return TSB_ECUDA;
    attr_dev = dev;
  }
  int blocks = sm_count();
  const int nblk = N / RW;
  if (nblk < blocks) blocks = nblk;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(blocks, 1, 1);
  cfg.blockDim = dim3(kQmvWarps * 32, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, qmv_kernel<MT, RW>, x, w, s, b, o, N, K, ldy);
  return e == cudaSuccess ? TSB_OK : TSB_ECUDA;
}

}  // namespace

// M in {1, 2}, N % 4 == 0, K % 64 == 0 (callers check N % 128 and alignment).
// gs: the tensor-parallel form (this rank's N-shard, stored into every rank's
// y), else y alone.
int qmv(const uint16_t *x, const uint32_t *w, const uint16_t *s, const uint16_t *b, uint16_t *y, int M, int N, int K,
        int ldy, const GatherSpec *gs, cudaStream_t st) {
  QmvOut o;
  for (int p = 0; p < kMaxGatherRanks; ++p) { o.yp[p] = nullptr; o.sig[p] = nullptr; }
  if (gs) {
    o.world = gs->world;
    o.rank = gs->rank;
    for (int p = 0; p < gs->world; ++p) {
      o.yp[p] = static_cast<uint16_t *>(gs->y[p]) + gs->col0;
      o.sig[p] = static_cast<uint32_t *>(gs->sig[p]);
    }
  } else {
    o.world = 1;
    o.rank = 0;
    o.yp[0] = y;
  }
  // 4-row warp blocks: 2-row blocks (more warps streaming when N / 4 is below
  // the device's warp count) measured slower on B200 (5120x17408: 19.7 -> 28.2 us)
  if (M == 1) return launch_qmv<1, 4>(x, w, s, b, o, N, K, ldy, st);
  if (M == 2) return launch_qmv<2, 4>(x, w, s, b, o, N, K, ldy, st);
  return TSB_EINVAL;
}

}  // namespace tsb
