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
// back. The accepted paths come as kernel parameters (at most 8 requests x 64
// nodes), so a commit needs no device buffer and no host-to-device copy.
#include "common.cuh"

namespace tsb {
namespace {

constexpr int kMaxCommitRequests = 8;
constexpr int kMaxCommitNodes = 64;
constexpr int kRowVec = 256 * 2 / 16;  // 16-byte vectors in a bf16 row of 256 values

struct CommitArgs {
  void *k, *v, *ks, *kb, *vs, *vb;
  int kv_format, Hkv, cap;
  int off0[kMaxCommitRequests];
  int n_keep[kMaxCommitRequests];
  uint8_t nodes[kMaxCommitRequests][kMaxCommitNodes];
};

__global__ void __launch_bounds__(256) kv_commit_kernel(CommitArgs a) {
  __shared__ uint4 stage[kMaxCommitNodes * kRowVec];  // 32 KB: the accepted rows
  __shared__ uint2 aux[2][kMaxCommitNodes];           // their scales (and MLX biases)
  const int b = blockIdx.x / (2 * a.Hkv);
  const int rem = blockIdx.x % (2 * a.Hkv);
  const int head = rem / 2;
  const bool isv = rem & 1;
  const int n = a.n_keep[b];
  if (n == 0) return;
  const size_t row0 = ((size_t)b * a.Hkv + head) * a.cap + a.off0[b];  // first row of the tree region
  // 16-byte vectors per row: bf16 32; both 8-bit formats 16
  const int vec = a.kv_format == TSB_KV_BF16 ? kRowVec : kRowVec / 2;
  uint4 *plane = static_cast<uint4 *>(isv ? a.v : a.k);
  for (int i = threadIdx.x; i < n * vec; i += blockDim.x) {
    const int r = i / vec, c = i % vec;
    stage[i] = plane[(row0 + a.nodes[b][r]) * vec + c];
  }
  if (a.kv_format == TSB_KV_REF_Q8_ROW) {
    const float *sc = static_cast<const float *>(isv ? a.vs : a.ks);
    for (int r = threadIdx.x; r < n; r += blockDim.x)
      aux[0][r].x = __float_as_uint(sc[row0 + a.nodes[b][r]]);
  } else if (a.kv_format == TSB_KV_MLX_Q8_G64) {
    const uint2 *sc = static_cast<const uint2 *>(isv ? a.vs : a.ks);  // 4 bf16 scales per row
    const uint2 *bi = static_cast<const uint2 *>(isv ? a.vb : a.kb);  // 4 bf16 biases per row
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
    float *sc = static_cast<float *>(isv ? a.vs : a.ks);
    for (int r = threadIdx.x; r < n; r += blockDim.x) sc[row0 + r] = __uint_as_float(aux[0][r].x);
  } else if (a.kv_format == TSB_KV_MLX_Q8_G64) {
    uint2 *sc = static_cast<uint2 *>(isv ? a.vs : a.ks);
    uint2 *bi = static_cast<uint2 *>(isv ? a.vb : a.kb);
    for (int r = threadIdx.x; r < n; r += blockDim.x) {
      sc[row0 + r] = aux[0][r];
      bi[row0 + r] = aux[1][r];
    }
  }
}

}  // namespace
}  // namespace tsb

using namespace tsb;

extern "C" int tsb_kv_commit(int kv_format, void *k, void *k_scales, void *k_biases, void *v, void *v_scales,
                             void *v_biases, int B, int Hkv, int D, int kv_capacity, const int32_t *offsets,
                             const int32_t *nodes, const int32_t *n_keep, int max_keep, tsb_stream_t stream) {
  if (!k || !v || !offsets || !nodes || !n_keep) return TSB_EINVAL;
  if (B <= 0 || Hkv <= 0 || kv_capacity <= 0 || max_keep < 0) return TSB_EINVAL;
  if (D != 256) return TSB_EUNSUPPORTED;
  if (B > kMaxCommitRequests || max_keep > kMaxCommitNodes) return TSB_EUNSUPPORTED;
  if (kv_format < 0 || kv_format > 2) return TSB_EUNSUPPORTED;
  if (kv_format == TSB_KV_MLX_Q8_G64 && (!k_scales || !k_biases || !v_scales || !v_biases)) return TSB_EINVAL;
  if (kv_format == TSB_KV_REF_Q8_ROW && (!k_scales || !v_scales)) return TSB_EINVAL;
  if (!aligned(k, 16) || !aligned(v, 16)) return TSB_EINVAL;
  if (kv_format == TSB_KV_MLX_Q8_G64 &&
      (!aligned(k_scales, 8) || !aligned(k_biases, 8) || !aligned(v_scales, 8) || !aligned(v_biases, 8)))
    return TSB_EINVAL;
  CommitArgs a;
  a.k = k; a.v = v; a.ks = k_scales; a.kb = k_biases; a.vs = v_scales; a.vb = v_biases;
  a.kv_format = kv_format;
  a.Hkv = Hkv;
  a.cap = kv_capacity;
  for (int b = 0; b < kMaxCommitRequests; ++b) {
    a.off0[b] = 0;
    a.n_keep[b] = 0;
    for (int i = 0; i < kMaxCommitNodes; ++i) a.nodes[b][i] = 0;
  }
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
  kv_commit_kernel<<<B * Hkv * 2, 256, 0, (cudaStream_t)stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? TSB_OK : TSB_ECUDA;
}
