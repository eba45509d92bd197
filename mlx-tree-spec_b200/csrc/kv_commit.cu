// Tree commit of the KV cache: after a verify pass, keep only the accepted
// root-to-node path of each request's tree nodes. The reference
// (mlx-tree-spec src/mlx_tree_spec/tree_verify.py:488-496, _keep_kv) gathers
// rows off0 + nodes of the cache and writes them to rows off0 .. off0 +
// len(nodes), for K and V (and the int8 caches' scales through
// Q8KVCache.take_rows, kv8.py:143-148), then sets the cache offset. The
// reference commits one request with one path; here each request of a batch
// has its own tree-region start and path.
//
// A destination row can be another copy's source (path [0, 2, 3] moves row 3
// to row 2 while row 2 moves to row 1), so one CTA per (request, KV head, K or
// V) first stages all of its accepted rows in shared memory, then writes them
// back. The accepted paths and every layer's cache pointers come as kernel
// parameters (at most 48 layers, 8 requests x 64 nodes), so a commit of a
// whole model is one launch with no device buffer and no host-to-device copy.
#include <cstring>

#include "common.cuh"

namespace tsb {
namespace {

constexpr int kMaxCommitRequests = 8;
constexpr int kMaxCommitNodes = 64;
constexpr int kMaxCommitLayers = 48;
constexpr int kRowVec = 256 * 2 / 16;  // 16-byte vectors in a bf16 row of 256 values

struct CommitPlanes {
  void *k, *v, *ks, *kb, *vs, *vb;
};

// ~2.9 KB of launch parameters: every layer's planes, every request's path.
struct CommitArgs {
  CommitPlanes layer[kMaxCommitLayers];
  int kv_format, B, Hkv, cap;
  int off0[kMaxCommitRequests];
  int n_keep[kMaxCommitRequests];
  uint8_t nodes[kMaxCommitRequests][kMaxCommitNodes];
};

// grid layers * B * Hkv * 2: one CTA per (layer, request, KV head, K or V)
__global__ void __launch_bounds__(256) kv_commit_kernel(const __grid_constant__ CommitArgs a) {
  __shared__ uint4 stage[kMaxCommitNodes * kRowVec];  // 32 KB: the accepted rows
  __shared__ uint2 aux[2][kMaxCommitNodes];           // their scales (and MLX biases)
  const int per_layer = a.B * a.Hkv * 2;
  const CommitPlanes &pl = a.layer[blockIdx.x / per_layer];
  const int rem0 = blockIdx.x % per_layer;
  const int b = rem0 / (2 * a.Hkv);
  const int rem = rem0 % (2 * a.Hkv);
  const int head = rem / 2;
  const bool isv = rem & 1;
  const int n = a.n_keep[b];
  if (n == 0) return;
  const size_t row0 = ((size_t)b * a.Hkv + head) * a.cap + a.off0[b];  // first row of the tree region
  // 16-byte vectors per row: bf16 32; both 8-bit formats 16
  const int vec = a.kv_format == TSB_KV_BF16 ? kRowVec : kRowVec / 2;
  uint4 *plane = static_cast<uint4 *>(isv ? pl.v : pl.k);
  for (int i = threadIdx.x; i < n * vec; i += blockDim.x) {
    const int r = i / vec, c = i % vec;
    stage[i] = plane[(row0 + a.nodes[b][r]) * vec + c];
  }
  if (a.kv_format == TSB_KV_REF_Q8_ROW) {
    const float *sc = static_cast<const float *>(isv ? pl.vs : pl.ks);
    for (int r = threadIdx.x; r < n; r += blockDim.x)
      aux[0][r].x = __float_as_uint(sc[row0 + a.nodes[b][r]]);
  } else if (a.kv_format == TSB_KV_MLX_Q8_G64) {
    const uint2 *sc = static_cast<const uint2 *>(isv ? pl.vs : pl.ks);  // 4 bf16 scales per row
    const uint2 *bi = static_cast<const uint2 *>(isv ? pl.vb : pl.kb);  // 4 bf16 biases per row
    for (int r = threadIdx.x; r < n; r += blockDim.x) {
      aux[0][r] = sc[row0 + a.nodes[b][r]];
      aux[1][r] = bi[row0 + a.nodes[b][r]];
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < n * vec; i += blockDim.x) {
    const int r = i / vec, c = i % vec;
    plane[(row0 + r) * vec + c] = stage[i];
  }
  if (a.kv_format == TSB_KV_REF_Q8_ROW) {
    float *sc = static_cast<float *>(isv ? pl.vs : pl.ks);
    for (int r = threadIdx.x; r < n; r += blockDim.x) sc[row0 + r] = __uint_as_float(aux[0][r].x);
  } else if (a.kv_format == TSB_KV_MLX_Q8_G64) {
    uint2 *sc = static_cast<uint2 *>(isv ? pl.vs : pl.ks);
    uint2 *bi = static_cast<uint2 *>(isv ? pl.vb : pl.kb);
    for (int r = threadIdx.x; r < n; r += blockDim.x) {
      sc[row0 + r] = aux[0][r];
      bi[row0 + r] = aux[1][r];
    }
  }
}

// Host-side checks of one layer's planes; returns TSB_OK or the status to report.
int check_planes(int kv_format, const CommitPlanes &p) {
  if (!p.k || !p.v) return TSB_EINVAL;
  if (kv_format == TSB_KV_MLX_Q8_G64 && (!p.ks || !p.kb || !p.vs || !p.vb)) return TSB_EINVAL;
  if (kv_format == TSB_KV_REF_Q8_ROW && (!p.ks || !p.vs)) return TSB_EINVAL;
  if (!aligned(p.k, 16) || !aligned(p.v, 16)) return TSB_EINVAL;
  if (kv_format == TSB_KV_MLX_Q8_G64 && (!aligned(p.ks, 8) || !aligned(p.kb, 8) || !aligned(p.vs, 8) || !aligned(p.vb, 8)))
    return TSB_EINVAL;
  return TSB_OK;
}

int launch_commit(int kv_format, int layers, const CommitPlanes *planes, int B, int Hkv, int D, int kv_capacity,
                  const int32_t *offsets, const int32_t *nodes, const int32_t *n_keep, int max_keep,
                  tsb_stream_t stream) {
  if (!planes || !offsets || !nodes || !n_keep) return TSB_EINVAL;
  if (layers <= 0 || B <= 0 || Hkv <= 0 || kv_capacity <= 0 || max_keep < 0) return TSB_EINVAL;
  if (D != 256) return TSB_EUNSUPPORTED;
  if (layers > kMaxCommitLayers || B > kMaxCommitRequests || max_keep > kMaxCommitNodes) return TSB_EUNSUPPORTED;
  if (kv_format < 0 || kv_format > 2) return TSB_EUNSUPPORTED;
  if ((long long)layers * B * Hkv * 2 > 0x7fffffffLL) return TSB_EUNSUPPORTED;
  CommitArgs a;
  memset(&a, 0, sizeof(a));
  for (int l = 0; l < layers; ++l) {
    const int st = check_planes(kv_format, planes[l]);
    if (st != TSB_OK) return st;
    a.layer[l] = planes[l];
  }
  a.kv_format = kv_format;
  a.B = B;
  a.Hkv = Hkv;
  a.cap = kv_capacity;
  for (int b = 0; b < B; ++b) {
    const int off = offsets[b], n = n_keep[b];
    if (off < 0 || n < 0 || n > max_keep || (long long)off + n > kv_capacity) return TSB_EINVAL;
    for (int i = 0; i < n; ++i) {
      const int node = nodes[(size_t)b * max_keep + i];
      if (node < 0 || node >= kMaxCommitNodes || (long long)off + node >= kv_capacity) return TSB_EINVAL;
      a.nodes[b][i] = (uint8_t)node;
    }
    a.off0[b] = off;
    a.n_keep[b] = n;
  }
  kv_commit_kernel<<<layers * B * Hkv * 2, 256, 0, (cudaStream_t)stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? TSB_OK : TSB_ECUDA;
}

}  // namespace
}  // namespace tsb

using namespace tsb;

extern "C" int tsb_kv_commit(int kv_format, void *k, void *k_scales, void *k_biases, void *v, void *v_scales,
                             void *v_biases, int B, int Hkv, int D, int kv_capacity, const int32_t *offsets,
                             const int32_t *nodes, const int32_t *n_keep, int max_keep, tsb_stream_t stream) {
  const CommitPlanes p{k, v, k_scales, k_biases, v_scales, v_biases};
  return launch_commit(kv_format, 1, &p, B, Hkv, D, kv_capacity, offsets, nodes, n_keep, max_keep, stream);
}

extern "C" int tsb_kv_commit_layers(int kv_format, int layers, void *const *k, void *const *k_scales,
                                    void *const *k_biases, void *const *v, void *const *v_scales,
                                    void *const *v_biases, int B, int Hkv, int D, int kv_capacity,
                                    const int32_t *offsets, const int32_t *nodes, const int32_t *n_keep, int max_keep,
                                    tsb_stream_t stream) {
  if (!k || !v || layers <= 0) return TSB_EINVAL;
  if (layers > kMaxCommitLayers) return TSB_EUNSUPPORTED;
  CommitPlanes p[kMaxCommitLayers];
  for (int l = 0; l < layers; ++l)
    p[l] = CommitPlanes{k[l], v[l], k_scales ? k_scales[l] : nullptr, k_biases ? k_biases[l] : nullptr,
                        v_scales ? v_scales[l] : nullptr, v_biases ? v_biases[l] : nullptr};
  return launch_commit(kv_format, layers, p, B, Hkv, D, kv_capacity, offsets, nodes, n_keep, max_keep, stream);
}
