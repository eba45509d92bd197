// Public quantized-matmul entry point: argument checks and routing by M, the
// B200 counterpart of the reference's per-call router packed_linear._call
// (mlx-tree-spec src/mlx_tree_spec/packed_linear.py:83-104).
#include "common.cuh"

namespace tsb {
size_t qmm_small_workspace_bytes(int M, int K);
int qmm_small(const uint16_t *x, const uint32_t *w, const uint16_t *s, const uint16_t *b, uint16_t *y, int M,
              int N, int K, int ldy, void *ws, size_t ws_bytes, cudaStream_t st);
int qmm_gemm(const uint16_t *x, const uint32_t *w, const uint16_t *s, const uint16_t *b, uint16_t *y, int M, int N,
             int K, int ldy, cudaStream_t st);

// Rows from which the tcgen05 GEMM (dequantize into shared memory, 256-row
// tiles) takes over from the small-M kernel.
constexpr int kGemmMinRows = 256;
}  // namespace tsb

using namespace tsb;

extern "C" size_t tsb_qmm_workspace_bytes(int M, int N, int K) {
  (void)N;
  if (M <= 0 || K <= 0) return 0;
  if (M >= kGemmMinRows) return 0;
  return qmm_small_workspace_bytes(M, K);
}

extern "C" int tsb_qmm_w4g64(const void *x, const uint32_t *w, const void *scales, const void *biases, void *y,
                             int M, int N, int K, int ldy, void *ws, size_t ws_bytes, tsb_stream_t stream) {
  if (!x || !w || !scales || !biases || !y) return TSB_EINVAL;
  if (M <= 0 || N <= 0 || K <= 0 || ldy < N) return TSB_EINVAL;
  if (K % 64 || N % 128) return TSB_EUNSUPPORTED;
  if (ldy % 8) return TSB_EINVAL;
  if (!aligned(x, 16) || !aligned(w, 16) || !aligned(y, 16)) return TSB_EINVAL;
  if (M >= kGemmMinRows)
    return qmm_gemm((const uint16_t *)x, w, (const uint16_t *)scales, (const uint16_t *)biases, (uint16_t *)y, M, N, K,
                    ldy, (cudaStream_t)stream);
  if (!ws || !aligned(ws, 16)) return TSB_EINVAL;
  return qmm_small((const uint16_t *)x, w, (const uint16_t *)scales, (const uint16_t *)biases, (uint16_t *)y, M,
                   N, K, ldy, ws, ws_bytes, (cudaStream_t)stream);
}
