// Public quantized-matmul entry point: argument checks and routing by M, the
// B200 counterpart of the reference's per-call router packed_linear._call
// (mlx-tree-spec src/mlx_tree_spec/packed_linear.py:83-104).
#include "common.cuh"

namespace tsb {
int qmm_ts(const uint16_t *x, const uint32_t *w, const uint16_t *s, const uint16_t *b, uint16_t *y, int M, int N,
           int K, int ldy, void *ws, size_t ws_bytes, const GatherSpec *gs, cudaStream_t st);
size_t qmm_ts_workspace_bytes(int M, int N, int K);
int qmm_gemm(const uint16_t *x, const uint32_t *w, const uint16_t *s, const uint16_t *b, uint16_t *y, int M, int N,
             int K, int ldy, const GatherSpec *gs, void *ws, size_t ws_bytes, cudaStream_t st);
size_t qmm_gemm_workspace_bytes(int M, int N, int K);
int qmv(const uint16_t *x, const uint32_t *w, const uint16_t *s, const uint16_t *b, uint16_t *y, int M, int N, int K,
        int ldy, const GatherSpec *gs, cudaStream_t st);

// Rows up to which the CUDA-core GEMV (qmv.cu) takes the call: it has no
// per-call pipeline to fill, which at M <= 2 costs more than it saves.
constexpr int kQmvMaxRows = 2;

// Rows above which the tcgen05 GEMM (dequantize into shared memory, 256-row
// tiles) takes over from the verify-pass kernel (weights dequantized into
// TMEM, tokens as the MMA's N <= 128).
constexpr int kTsMaxRows = 128;
}  // namespace tsb

using namespace tsb;

// The verify path (M <= 128) needs completion flags and the float partials of
// the row tiles it splits across CTAs; the prefill GEMM the float sums of its
// split tail, if it has one.
extern "C" size_t tsb_qmm_workspace_bytes(int M, int N, int K) {
  if (M <= 0 || N <= 0 || K <= 0 || N % 128 || K % 64) return 0;
  return M <= kTsMaxRows ? qmm_ts_workspace_bytes(M, N, K) : qmm_gemm_workspace_bytes(M, N, K);
}

extern "C" int tsb_qmm_w4g64(const void *x, const uint32_t *w, const void *scales, const void *biases, void *y,
                             int M, int N, int K, int ldy, void *ws, size_t ws_bytes, tsb_stream_t stream) {
  if (!x || !w || !scales || !biases || !y) return TSB_EINVAL;
  if (M <= 0 || N <= 0 || K <= 0 || ldy < N) return TSB_EINVAL;
  if (K % 64 || N % 128) return TSB_EUNSUPPORTED;
  if (ldy % 8) return TSB_EINVAL;
  if (!aligned(x, 16) || !aligned(w, 16) || !aligned(y, 16)) return TSB_EINVAL;
  if (M <= kQmvMaxRows) {
    const int r = qmv((const uint16_t *)x, w, (const uint16_t *)scales, (const uint16_t *)biases, (uint16_t *)y, M, N,
                      K, ldy, nullptr, (cudaStream_t)stream);
    if (r != TSB_EUNSUPPORTED) return r;  // else (x too long for shared memory) the verify kernel
  }
  if (M <= kTsMaxRows)
    return qmm_ts((const uint16_t *)x, w, (const uint16_t *)scales, (const uint16_t *)biases, (uint16_t *)y, M, N, K,
                  ldy, ws, ws_bytes, nullptr, (cudaStream_t)stream);
  return qmm_gemm((const uint16_t *)x, w, (const uint16_t *)scales, (const uint16_t *)biases, (uint16_t *)y, M, N, K,
                  ldy, nullptr, ws, ws_bytes, (cudaStream_t)stream);
}

// Tensor-parallel form: this rank's N-shard, its output columns stored into
// every rank's y by the kernel itself (no separate all-gather): the verify
// kernel at M <= 128, the prefill GEMM above.
extern "C" int tsb_qmm_w4g64_gather(const void *x, const uint32_t *w, const void *scales, const void *biases, int M,
                                    int Ns, int K, int ldy, const tsb_gather_t *g, void *ws, size_t ws_bytes,
                                    tsb_stream_t stream) {
  if (!x || !w || !scales || !biases || !g) return TSB_EINVAL;
  if (g->world < 1 || g->world > TSB_MAX_GATHER_RANKS || g->rank < 0 || g->rank >= g->world) return TSB_EINVAL;
  if (M <= 0 || Ns <= 0 || K <= 0) return TSB_EINVAL;
  if (K % 64 || Ns % 128) return TSB_EUNSUPPORTED;
  if ((long long)ldy < (long long)Ns * g->world || ldy % 8) return TSB_EINVAL;
  if (!aligned(x, 16) || !aligned(w, 16)) return TSB_EINVAL;
  GatherSpec gs;
  gs.world = g->world;
  gs.rank = g->rank;
  gs.col0 = g->rank * Ns;
  for (int p = 0; p < kMaxGatherRanks; ++p) {
    gs.y[p] = nullptr;
    gs.sig[p] = nullptr;
  }
  for (int p = 0; p < g->world; ++p) {
    if (!g->y[p] || !aligned(g->y[p], 16) || !g->sig[p] || !aligned(g->sig[p], 4)) return TSB_EINVAL;
    gs.y[p] = g->y[p];
    gs.sig[p] = g->sig[p];
  }
  uint16_t *y_own = (uint16_t *)g->y[g->rank] + gs.col0;
  if (M <= kQmvMaxRows) {
    const int r = qmv((const uint16_t *)x, w, (const uint16_t *)scales, (const uint16_t *)biases, y_own, M, Ns, K,
                      ldy, &gs, (cudaStream_t)stream);
    if (r != TSB_EUNSUPPORTED) return r;
  }
  if (M <= kTsMaxRows)
    return qmm_ts((const uint16_t *)x, w, (const uint16_t *)scales, (const uint16_t *)biases, y_own, M, Ns, K, ldy,
                  ws, ws_bytes, &gs, (cudaStream_t)stream);
  // prefill: the tcgen05 GEMM stores every tile into every rank's y
  return qmm_gemm((const uint16_t *)x, w, (const uint16_t *)scales, (const uint16_t *)biases, y_own, M, Ns, K, ldy,
                  &gs, ws, ws_bytes, (cudaStream_t)stream);
}
