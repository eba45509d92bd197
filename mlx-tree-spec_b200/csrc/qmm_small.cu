// Small-M 4-bit quantized matmul on the MLX layout (verify pass, M <= 64 per
// token chunk), warp-level bf16 MMA with swap-AB: weight rows are the MMA's M
// dimension (16 per warp), tree tokens its N dimension (8 per token block).
//
// Arithmetic: per 64-group, the MMA multiplies the raw codes (held as the bf16
// value 128 + q, made with one LOP3 from the packed word) with x, and the group
// result is scaled in float32:
//   sum_k (s q_k + b) x_k = s * sum_k (128 + q_k) x_k + (b - 128 s) * sum_k x_k
// which is the reference's `s * sum q x + b * sum x` decomposition
// (mlx-tree-spec src/mlx_tree_spec/qmm_packed.py:14-16 and its _qmv kernel at
// 424-425), done on tensor cores.
//
// K permutation: within a group, lane c (0..3) of an MMA row quad owns words
// 2c and 2c+1 of the row (elements 16c..16c+15). For MMA step s (0..3) its A
// registers hold elements {16c+s, 16c+s+4} and {16c+8+s, 16c+12+s}, exactly the
// pairs `(word >> 4s) & 0x000F000F` extracts. The B operand (x) is prepared
// once per call in the same permuted order (qmm_prep_x_kernel), so the MMA's
// sum over k is unchanged.
#include "common.cuh"

#include <cooperative_groups.h>

namespace cg = cooperative_groups;

namespace tsb {

namespace {

constexpr int QS_ROWS = 128;   // weight rows per CTA (8 warps x 16)
constexpr int QS_THREADS = 256;
constexpr int QS_CHUNK_TOKENS = 64;
constexpr int QS_U = 4;        // groups per prefetch batch

// x [M, K] bf16 -> fragment-ordered x and per-group token sums (workspace).
//   xf[((tb * G + g) * 4 + s) * 32 + lane] = {b01, b23} of token tb*8 + lane/4
//   xs[(tb * G + g) * 8 + t]               = sum of the 64 x values of token tb*8+t, group g
// Tokens >= M are zero.
__global__ void qmm_prep_x_kernel(const uint16_t *__restrict__ x, int M, int K, int MTtot,
                                  uint2 *__restrict__ xf, float *__restrict__ xs) {
  const int G = K / 64;
  const long long total = (long long)MTtot * 8 * G * 4;
  const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  // Every lane stays to the end: the quad sum below is a full-warp shuffle.
  const bool live = i < total;
  const int c = int(i & 3);
  const long long r = live ? (i >> 2) : 0;
  const int g = int(r % G);
  const int tok = int(r / G);
  uint32_t p[8];
  if (live && tok < M) {
    const uint4 *src = reinterpret_cast<const uint4 *>(x + (size_t)tok * K + g * 64 + c * 16);
    const uint4 u0 = src[0], u1 = src[1];
    p[0] = u0.x; p[1] = u0.y; p[2] = u0.z; p[3] = u0.w;
    p[4] = u1.x; p[5] = u1.y; p[6] = u1.z; p[7] = u1.w;
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) p[j] = 0;
  }
  // p[j] holds elements 2j (low) and 2j+1 (high) of this lane's 16.
  float sum = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) sum += bf16lo(p[j]) + bf16hi(p[j]);
  sum += __shfl_xor_sync(0xffffffffu, sum, 1);
  sum += __shfl_xor_sync(0xffffffffu, sum, 2);
  if (!live) return;
  const int tb = tok / 8, n = tok % 8;
  const int lane = n * 4 + c;
#pragma unroll
  for (int s = 0; s < 4; ++s) {
    // element e lives in p[e/2], half e%2. b01 = {e=s, e=s+4}; b23 = {e=8+s, e=12+s}.
    const uint32_t b01 = prmt(p[s / 2], p[(s + 4) / 2], (s & 1) ? 0x7632u : 0x5410u);
    const uint32_t b23 = prmt(p[(8 + s) / 2], p[(12 + s) / 2], (s & 1) ? 0x7632u : 0x5410u);
    xf[(((long long)tb * G + g) * 4 + s) * 32 + lane] = make_uint2(b01, b23);
  }
  if (c == 0) xs[((long long)tb * G + g) * 8 + n] = sum;
}

template <int MT>
__global__ void __launch_bounds__(QS_THREADS, 2)
qmm_small_kernel(const uint32_t *__restrict__ w, const uint16_t *__restrict__ scales,
                 const uint16_t *__restrict__ biases, const uint2 *__restrict__ xf,
                 const float *__restrict__ xs, uint16_t *__restrict__ y, int M, int N, int K, int ldy,
                 int splits) {
  const int G = K / 64;
  const int KW = K / 8;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int quad = lane / 4, c = lane % 4;
  const int n0 = blockIdx.x * QS_ROWS;
  const int row_a = n0 + warp * 16 + quad;  // rows row_a and row_a + 8
  const int split = blockIdx.y;
  const int g0 = (int)((long long)split * G / splits);
  const int g1 = (int)((long long)(split + 1) * G / splits);
  const int chunk = blockIdx.z;  // token chunk of 64
  const int tb0 = chunk * (QS_CHUNK_TOKENS / 8);

  const uint32_t *wa = w + (size_t)row_a * KW + 2 * c;
  const uint32_t *wb = wa + (size_t)8 * KW;
  const uint16_t *sa = scales + (size_t)row_a * G;
  const uint16_t *sb = sa + (size_t)8 * G;
  const uint16_t *ba = biases + (size_t)row_a * G;
  const uint16_t *bb = ba + (size_t)8 * G;

  float acc[MT][4];
#pragma unroll
  for (int t = 0; t < MT; ++t)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[t][j] = 0.f;

  uint2 cw_a[QS_U], cw_b[QS_U];
  uint32_t csb[QS_U], cbb[QS_U];  // (scale_a | scale_b << 16), (bias_a | bias_b << 16)
  auto load_batch = [&](int gb, uint2 (&wa_)[QS_U], uint2 (&wb_)[QS_U], uint32_t (&s_)[QS_U],
                        uint32_t (&b_)[QS_U]) {
#pragma unroll
    for (int u = 0; u < QS_U; ++u) {
      const int g = gb + u;
      if (g < g1) {
        wa_[u] = ldg_nc_v2(wa + g * 8);
        wb_[u] = ldg_nc_v2(wb + g * 8);
        s_[u] = uint32_t(__ldg(sa + g)) | (uint32_t(__ldg(sb + g)) << 16);
        b_[u] = uint32_t(__ldg(ba + g)) | (uint32_t(__ldg(bb + g)) << 16);
      } else {
        wa_[u] = make_uint2(0, 0);
        wb_[u] = make_uint2(0, 0);
        s_[u] = 0;
        b_[u] = 0;
      }
    }
  };
  load_batch(g0, cw_a, cw_b, csb, cbb);

  for (int gb = g0; gb < g1; gb += QS_U) {
    uint2 nw_a[QS_U], nw_b[QS_U];
    uint32_t nsb[QS_U], nbb[QS_U];
    load_batch(gb + QS_U, nw_a, nw_b, nsb, nbb);
#pragma unroll
    for (int u = 0; u < QS_U; ++u) {
      const int g = gb + u;
      if (g < g1) {
        uint32_t a[4][4];
#pragma unroll
        for (int s = 0; s < 4; ++s) {
          a[s][0] = lop3_and_or(cw_a[u].x >> (4 * s), 0x000F000Fu, 0x43004300u);
          a[s][1] = lop3_and_or(cw_b[u].x >> (4 * s), 0x000F000Fu, 0x43004300u);
          a[s][2] = lop3_and_or(cw_a[u].y >> (4 * s), 0x000F000Fu, 0x43004300u);
          a[s][3] = lop3_and_or(cw_b[u].y >> (4 * s), 0x000F000Fu, 0x43004300u);
        }
        const float s_a = bf16lo(csb[u]), s_b = bf16hi(csb[u]);
        const float b_a = __fmaf_rn(-128.f, s_a, bf16lo(cbb[u]));
        const float b_b = __fmaf_rn(-128.f, s_b, bf16hi(cbb[u]));
        const uint2 *xg = xf + ((size_t)tb0 * G + g) * 128 + lane;
        const float *xsg = xs + ((size_t)tb0 * G + g) * 8 + 2 * c;
#pragma unroll
        for (int t = 0; t < MT; ++t) {
          float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int s = 0; s < 4; ++s) {
            const uint2 bx = __ldg(xg + ((size_t)t * G * 4 + s) * 32);
            mma_bf16_16816(d, a[s], bx.x, bx.y, d);
          }
          const float2 sx = __ldg(reinterpret_cast<const float2 *>(xsg + (size_t)t * G * 8));
          acc[t][0] = __fmaf_rn(s_a, d[0], __fmaf_rn(b_a, sx.x, acc[t][0]));
          acc[t][1] = __fmaf_rn(s_a, d[1], __fmaf_rn(b_a, sx.y, acc[t][1]));
          acc[t][2] = __fmaf_rn(s_b, d[2], __fmaf_rn(b_b, sx.x, acc[t][2]));
          acc[t][3] = __fmaf_rn(s_b, d[3], __fmaf_rn(b_b, sx.y, acc[t][3]));
        }
      }
    }
#pragma unroll
    for (int u = 0; u < QS_U; ++u) {
      cw_a[u] = nw_a[u];
      cw_b[u] = nw_b[u];
      csb[u] = nsb[u];
      cbb[u] = nbb[u];
    }
  }

  const int tok0 = chunk * QS_CHUNK_TOKENS;
  const int rl = warp * 16 + quad;  // local row
  if (splits == 1) {
#pragma unroll
    for (int t = 0; t < MT; ++t) {
      const int tk = tok0 + t * 8 + 2 * c;
      if (tk < M) {
        y[(size_t)tk * ldy + n0 + rl] = float_to_bf16_bits(acc[t][0]);
        y[(size_t)tk * ldy + n0 + rl + 8] = float_to_bf16_bits(acc[t][2]);
      }
      if (tk + 1 < M) {
        y[(size_t)(tk + 1) * ldy + n0 + rl] = float_to_bf16_bits(acc[t][1]);
        y[(size_t)(tk + 1) * ldy + n0 + rl + 8] = float_to_bf16_bits(acc[t][3]);
      }
    }
    return;
  }
  // Split-K: the CTAs of a cluster hold partial sums of the same output tile;
  // reduce them through distributed shared memory.
  __shared__ float red[MT * 8 * QS_ROWS];  // [token][row]
#pragma unroll
  for (int t = 0; t < MT; ++t) {
    const int tl = t * 8 + 2 * c;
    red[tl * QS_ROWS + rl] = acc[t][0];
    red[(tl + 1) * QS_ROWS + rl] = acc[t][1];
    red[tl * QS_ROWS + rl + 8] = acc[t][2];
    red[(tl + 1) * QS_ROWS + rl + 8] = acc[t][3];
  }
  cg::cluster_group cluster = cg::this_cluster();
  cluster.sync();
  const int rank = (int)cluster.block_rank();
  const int total = MT * 8 * QS_ROWS;
  const int per = (total + splits - 1) / splits;
  const int e0 = rank * per, e1 = min(total, e0 + per);
  for (int e = e0 + (int)threadIdx.x; e < e1; e += QS_THREADS) {
    float v = 0.f;
    for (int r = 0; r < splits; ++r) v += cluster.map_shared_rank(red, r)[e];
    const int tk = tok0 + e / QS_ROWS;
    if (tk < M) y[(size_t)tk * ldy + n0 + (e % QS_ROWS)] = float_to_bf16_bits(v);
  }
  cluster.sync();
}

template <int MT>
int launch_small(const uint32_t *w, const uint16_t *s, const uint16_t *b, const uint2 *xf, const float *xs,
                 uint16_t *y, int M, int N, int K, int ldy, int splits, int chunks, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(N / QS_ROWS, splits, chunks);
  cfg.blockDim = dim3(QS_THREADS, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = splits;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, qmm_small_kernel<MT>, w, s, b, xf, xs, y, M, N, K, ldy, splits);
  return e == cudaSuccess ? TSB_OK : TSB_ECUDA;
}

}  // namespace

// Workspace of the small-M path: fragment-ordered x plus group sums.
// Token blocks (of 8) the prep kernel fills: whole 64-token chunks when the
// call needs more than one chunk, since every chunk reads 8 blocks.
static int prep_token_blocks(int M) {
  return M > QS_CHUNK_TOKENS ? ((M + QS_CHUNK_TOKENS - 1) / QS_CHUNK_TOKENS) * (QS_CHUNK_TOKENS / 8) : (M + 7) / 8;
}

size_t qmm_small_workspace_bytes(int M, int K) {
  const size_t G = (size_t)K / 64;
  const size_t MTtot = (size_t)prep_token_blocks(M);
  return MTtot * G * 128 * sizeof(uint2) + MTtot * G * 8 * sizeof(float) + 256;
}

int qmm_small(const uint16_t *x, const uint32_t *w, const uint16_t *s, const uint16_t *b, uint16_t *y, int M,
              int N, int K, int ldy, void *ws, size_t ws_bytes, cudaStream_t st) {
  if (ws_bytes < qmm_small_workspace_bytes(M, K)) return TSB_EWORKSPACE;
  const int G = K / 64;
  const int MTtot = prep_token_blocks(M);
  uint2 *xf = reinterpret_cast<uint2 *>(ws);
  float *xs = reinterpret_cast<float *>(reinterpret_cast<char *>(ws) + (size_t)MTtot * G * 128 * sizeof(uint2));
  {
    const long long total = (long long)MTtot * 8 * G * 4;
    const int threads = 256;
    qmm_prep_x_kernel<<<(unsigned)((total + threads - 1) / threads), threads, 0, st>>>(x, M, K, MTtot, xf, xs);
    if (cudaGetLastError() != cudaSuccess) return TSB_ECUDA;
  }
  const int tiles = N / QS_ROWS;
  int splits = (2 * sm_count() + tiles / 2) / tiles;
  if (splits < 1) splits = 1;
  if (splits > 8) splits = 8;
  while (splits > 1 && G / splits < 4) --splits;
  const int chunks = (M + QS_CHUNK_TOKENS - 1) / QS_CHUNK_TOKENS;
  const int mt = chunks > 1 ? 8 : MTtot;
  switch (mt) {
    case 1: return launch_small<1>(w, s, b, xf, xs, y, M, N, K, ldy, splits, chunks, st);
    case 2: return launch_small<2>(w, s, b, xf, xs, y, M, N, K, ldy, splits, chunks, st);
    case 3: return launch_small<3>(w, s, b, xf, xs, y, M, N, K, ldy, splits, chunks, st);
    case 4: return launch_small<4>(w, s, b, xf, xs, y, M, N, K, ldy, splits, chunks, st);
    case 5: return launch_small<5>(w, s, b, xf, xs, y, M, N, K, ldy, splits, chunks, st);
    case 6: return launch_small<6>(w, s, b, xf, xs, y, M, N, K, ldy, splits, chunks, st);
    case 7: return launch_small<7>(w, s, b, xf, xs, y, M, N, K, ldy, splits, chunks, st);
    default: return launch_small<8>(w, s, b, xf, xs, y, M, N, K, ldy, splits, chunks, st);
  }
}

}  // namespace tsb
