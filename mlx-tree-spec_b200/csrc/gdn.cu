// GatedDeltaNet over tree nodes: the linear-attention half of the hybrid
// model's verify pass (mlx-tree-spec src/mlx_tree_spec/tree_verify.py:149-238
// tree_gated_delta, 251-271 batch_gdn; fused_ops.py:28-104 gdn_prep,
// 157-226 gdn_commit).
//
//   prep:   per node, the causal conv (kernel 4) over the node's window of 3
//           ancestors and itself (rows of concat(conv_state, qkv)), silu, the
//           per-head q/k RMS norms and scales, beta = sigmoid(b), the decay g.
//           One warp per (node, head slot): 4 channels per lane, the norm a
//           warp reduction.
//   tree:   each node's recurrence output along its own root path. A walk is a
//           root-to-leaf path; the host folds leaf siblings into walks as side
//           steps from the same state (no extra state read). A CTA per (walk,
//           value head, 32 dv rows) stages the walk's q/k/v/g/beta in shared
//           memory in one parallel phase; each warp then runs the walk for 4
//           state rows (4 x 128 floats in registers), its 4 dot products
//           reduced together so the shuffles overlap.
//   commit: the state after replaying the accepted path (nodes from the launch
//           parameters), and the new conv state (the last node's window). Each
//           lane reads its 4 state floats first and writes them last, so
//           state_out may be state_in.
//
// The walk arrays come from device memory, so every node index read there is
// checked against n before use (a bad index ends the walk / skips the entry).
#include "common.cuh"

namespace tsb {
namespace {

constexpr int kGdnD = 128;          // Dk = Dv = 128 (the reference's prep asserts it)
constexpr int kGdnWarps = 8;         // dv rows per CTA
constexpr int kGdnMaxPath = 64;

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

__device__ __forceinline__ float bf16r(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// 4 consecutive bf16 at p (8-byte aligned) -> floats
__device__ __forceinline__ void load4(const __nv_bfloat16 *p, float (&f)[4]) {
  const uint2 u = *reinterpret_cast<const uint2 *>(p);
  const __nv_bfloat162 lo = *reinterpret_cast<const __nv_bfloat162 *>(&u.x);
  const __nv_bfloat162 hi = *reinterpret_cast<const __nv_bfloat162 *>(&u.y);
  f[0] = __low2float(lo); f[1] = __high2float(lo); f[2] = __low2float(hi); f[3] = __high2float(hi);
}

__device__ __forceinline__ void store4(__nv_bfloat16 *p, const float (&f)[4]) {
  __nv_bfloat162 lo = __floats2bfloat162_rn(f[0], f[1]);
  __nv_bfloat162 hi = __floats2bfloat162_rn(f[2], f[3]);
  uint2 u;
  u.x = *reinterpret_cast<uint32_t *>(&lo);
  u.y = *reinterpret_cast<uint32_t *>(&hi);
  *reinterpret_cast<uint2 *>(p) = u;
}

struct PrepArgs {
  const __nv_bfloat16 *qkv, *conv_state, *conv_w, *a, *b;
  const int32_t *conv_idx;
  const float *a_log, *dt_bias;
  __nv_bfloat16 *q, *k, *v, *beta;
  float *g;
  int n, Hk, Hv;
};

// grid (ceil(slots / 4), n), 128 threads; slot = 2*Hk + Hv is the g/beta slot
__global__ void __launch_bounds__(128) gdn_prep_kernel(PrepArgs a) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int slot = blockIdx.x * 4 + warp;
  const int node = blockIdx.y;
  const int nslots = 2 * a.Hk + a.Hv;
  if (slot > nslots) return;
  if (slot == nslots) {
    for (int h = lane; h < a.Hv; h += 32) {
      const int i = node * a.Hv + h;
      const float ab = bf16r(__bfloat162float(a.a[i]) + a.dt_bias[h]);
      const float sp = ab > 20.0f ? ab : log1pf(expf(ab));
      a.g[i] = expf(-expf(a.a_log[h]) * bf16r(sp));
      a.beta[i] = __float2bfloat16_rn(1.0f / (1.0f + expf(-__bfloat162float(a.b[i]))));
    }
    return;
  }
  const int C = (2 * a.Hk + a.Hv) * kGdnD;
  const bool is_v = slot >= 2 * a.Hk;
  const int ch = slot * kGdnD + lane * 4;  // q heads, k heads, v heads are consecutive 128-column slots
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  // conv weights of the 4 channels: [ch][tap], 16 bf16 = 32 contiguous bytes
  float w[4][4];
  load4(a.conv_w + (size_t)ch * 4 + 0, w[0]);
  load4(a.conv_w + (size_t)ch * 4 + 4, w[1]);
  load4(a.conv_w + (size_t)ch * 4 + 8, w[2]);
  load4(a.conv_w + (size_t)ch * 4 + 12, w[3]);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int r = a.conv_idx[node * 4 + j];
    if (r < 0 || r >= 3 + a.n) continue;  // malformed window entry: contributes nothing
    const __nv_bfloat16 *src = r < 3 ? a.conv_state + (size_t)r * C : a.qkv + (size_t)(r - 3) * C;
    float x[4];
    load4(src + ch, x);
#pragma unroll
    for (int c = 0; c < 4; ++c) acc[c] += x[c] * w[c][j];
  }
  float s[4];
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const float cv = bf16r(acc[c]);
    s[c] = bf16r(cv / (1.0f + expf(-cv)));
  }
  if (is_v) {
    store4(a.v + ((size_t)node * a.Hv + (slot - 2 * a.Hk)) * kGdnD + lane * 4, s);
    return;
  }
  const float ss = warp_sum(s[0] * s[0] + s[1] * s[1] + s[2] * s[2] + s[3] * s[3]);
  const float inv = rsqrtf(ss / float(kGdnD) + 1e-6f);
  const bool is_q = slot < a.Hk;
  const float scale = is_q ? 1.0f / float(kGdnD) : 0.08838834764831845f;  // 1/Dk for q, Dk^-1/2 for k
  float o[4];
#pragma unroll
  for (int c = 0; c < 4; ++c) o[c] = bf16r(s[c] * inv) * scale;
  __nv_bfloat16 *dst = is_q ? a.q + ((size_t)node * a.Hk + slot) * kGdnD
                            : a.k + ((size_t)node * a.Hk + (slot - a.Hk)) * kGdnD;
  store4(dst + lane * 4, o);
}

struct TreeArgs {
  const __nv_bfloat16 *q, *k, *v, *beta;
  const float *g, *state;
  const int32_t *paths, *sibs, *owner;
  __nv_bfloat16 *y;
  int n, rows, lmax, Hk, Hv;
};

constexpr int kTreeRows = 4;                         // dv rows per warp
constexpr int kTreeDv = kGdnWarps * kTreeRows;        // 32 dv rows per CTA
constexpr int kStage = 32;                           // walk steps staged in shared memory

// Butterfly sum of 4 independent values across the warp (interleaved for ILP).
__device__ __forceinline__ void warp_sum4(float (&x)[kTreeRows]) {
#pragma unroll
  for (int o = 16; o; o >>= 1) {
#pragma unroll
    for (int r = 0; r < kTreeRows; ++r) x[r] += __shfl_xor_sync(0xffffffffu, x[r], o);
  }
}

__device__ __forceinline__ void unpack4(uint2 u, float (&f)[4]) {
  const __nv_bfloat162 lo = *reinterpret_cast<const __nv_bfloat162 *>(&u.x);
  const __nv_bfloat162 hi = *reinterpret_cast<const __nv_bfloat162 *>(&u.y);
  f[0] = __low2float(lo); f[1] = __high2float(lo); f[2] = __low2float(hi); f[3] = __high2float(hi);
}

// One walk step's inputs for this CTA: q/k of the node (and of its side leaf),
// g and beta, and v of the CTA's 32 dv rows.
struct StepIn {
  uint2 q[32], k[32], qs[32], ks[32];   // lane l holds dk 4l..4l+3
  __nv_bfloat16 v[kTreeDv], vs[kTreeDv];
  float g, gs, beta, betas;
  int node, sib;                        // -1: walk over / no side leaf
  int own, owns;                        // this walk writes the node's / side leaf's output
};

// grid (Dv / 32, Hv, rows), 256 threads. Warp w owns dv rows
// blockIdx.x * 32 + 4w .. +3 and keeps their state (4 x 4 floats per lane) in
// registers for the whole walk. The first kStage steps' inputs are staged in
// shared memory up front (all loads in flight at once); later steps load
// directly.
__global__ void __launch_bounds__(256) gdn_tree_kernel(TreeArgs a) {
  __shared__ StepIn s_in[kStage];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int dv_cta = blockIdx.x * kTreeDv;
  const int dv0 = dv_cta + warp * kTreeRows;
  const int hv = blockIdx.y, row = blockIdx.z;
  const int hk = hv / (a.Hv / a.Hk);
  const int staged = a.lmax < kStage ? a.lmax : kStage;

  // stage 1: node / side-leaf indices and their scalars
  for (int t = threadIdx.x; t < staged; t += blockDim.x) {
    int node = a.paths[row * a.lmax + t];
    int sib = a.sibs[row * a.lmax + t];
    if (node < 0 || node >= a.n) node = -1;
    if (sib < 0 || sib >= a.n || node < 0) sib = -1;
    StepIn &si = s_in[t];
    si.node = node;
    si.sib = sib;
    si.own = node >= 0 && a.owner[node] == row;
    si.owns = sib >= 0 && a.owner[sib] == row;
    if (node >= 0) {
      si.g = a.g[node * a.Hv + hv];
      si.beta = __bfloat162float(a.beta[node * a.Hv + hv]);
    }
    if (sib >= 0) {
      si.gs = a.g[sib * a.Hv + hv];
      si.betas = __bfloat162float(a.beta[sib * a.Hv + hv]);
    }
  }
  __syncthreads();
  // stage 2: vectors. Per step: 4 x 32 uint2 of q/k and 2 x 32 bf16 of v
  for (int i = threadIdx.x; i < staged * 32; i += blockDim.x) {
    const int t = i >> 5, l = i & 31;
    StepIn &si = s_in[t];
    if (si.node >= 0) {
      const size_t qk = ((size_t)si.node * a.Hk + hk) * kGdnD + l * 4;
      si.q[l] = *reinterpret_cast<const uint2 *>(a.q + qk);
      si.k[l] = *reinterpret_cast<const uint2 *>(a.k + qk);
      si.v[l] = a.v[((size_t)si.node * a.Hv + hv) * kGdnD + dv_cta + l];
    }
    if (si.sib >= 0) {
      const size_t qk = ((size_t)si.sib * a.Hk + hk) * kGdnD + l * 4;
      si.qs[l] = *reinterpret_cast<const uint2 *>(a.q + qk);
      si.ks[l] = *reinterpret_cast<const uint2 *>(a.k + qk);
      si.vs[l] = a.v[((size_t)si.sib * a.Hv + hv) * kGdnD + dv_cta + l];
    }
  }
  __syncthreads();

  float st[kTreeRows][4];
#pragma unroll
  for (int r = 0; r < kTreeRows; ++r) {
    const float4 s4 = *reinterpret_cast<const float4 *>(a.state + ((size_t)hv * kGdnD + dv0 + r) * kGdnD + lane * 4);
    st[r][0] = s4.x; st[r][1] = s4.y; st[r][2] = s4.z; st[r][3] = s4.w;
  }
  for (int t = 0; t < a.lmax; ++t) {
    int node, sib, own, owns;
    float g, beta, gs = 0.f, betas = 0.f;
    float qn[4], kn[4], qs[4], ks[4], vn[kTreeRows], vsv[kTreeRows];
    if (t < kStage) {
      const StepIn &si = s_in[t];
      node = si.node;
      if (node < 0) break;
      sib = si.sib; own = si.own; owns = si.owns;
      g = si.g; beta = si.beta;
      unpack4(si.q[lane], qn);
      unpack4(si.k[lane], kn);
#pragma unroll
      for (int r = 0; r < kTreeRows; ++r) vn[r] = __bfloat162float(si.v[warp * kTreeRows + r]);
      if (sib >= 0) {
        gs = si.gs; betas = si.betas;
        unpack4(si.qs[lane], qs);
        unpack4(si.ks[lane], ks);
#pragma unroll
        for (int r = 0; r < kTreeRows; ++r) vsv[r] = __bfloat162float(si.vs[warp * kTreeRows + r]);
      }
    } else {
      node = a.paths[row * a.lmax + t];
      if (node < 0 || node >= a.n) break;
      sib = a.sibs[row * a.lmax + t];
      if (sib >= a.n) sib = -1;
      own = a.owner[node] == row;
      owns = sib >= 0 && a.owner[sib] == row;
      g = a.g[node * a.Hv + hv];
      beta = __bfloat162float(a.beta[node * a.Hv + hv]);
      load4(a.q + ((size_t)node * a.Hk + hk) * kGdnD + lane * 4, qn);
      load4(a.k + ((size_t)node * a.Hk + hk) * kGdnD + lane * 4, kn);
#pragma unroll
      for (int r = 0; r < kTreeRows; ++r) vn[r] = __bfloat162float(a.v[((size_t)node * a.Hv + hv) * kGdnD + dv0 + r]);
      if (sib >= 0) {
        gs = a.g[sib * a.Hv + hv];
        betas = __bfloat162float(a.beta[sib * a.Hv + hv]);
        load4(a.q + ((size_t)sib * a.Hk + hk) * kGdnD + lane * 4, qs);
        load4(a.k + ((size_t)sib * a.Hk + hk) * kGdnD + lane * 4, ks);
#pragma unroll
        for (int r = 0; r < kTreeRows; ++r)
          vsv[r] = __bfloat162float(a.v[((size_t)sib * a.Hv + hv) * kGdnD + dv0 + r]);
      }
    }
    if (sib >= 0) {
      // a leaf sibling: one step from the same state, not kept
      float kv[kTreeRows], os[kTreeRows];
#pragma unroll
      for (int r = 0; r < kTreeRows; ++r) {
        kv[r] = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) kv[r] += st[r][i] * gs * ks[i];
      }
      warp_sum4(kv);
#pragma unroll
      for (int r = 0; r < kTreeRows; ++r) {
        const float ds = (vsv[r] - kv[r]) * betas;
        os[r] = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) os[r] += (st[r][i] * gs + ks[i] * ds) * qs[i];
      }
      warp_sum4(os);
      if (lane == 0 && owns) {
        const float o4[4] = {os[0], os[1], os[2], os[3]};
        store4(a.y + ((size_t)sib * a.Hv + hv) * kGdnD + dv0, o4);
      }
    }
    float kv[kTreeRows], out[kTreeRows];
#pragma unroll
    for (int r = 0; r < kTreeRows; ++r) {
      kv[r] = 0.f;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        st[r][i] *= g;
        kv[r] += st[r][i] * kn[i];
      }
    }
    warp_sum4(kv);
#pragma unroll
    for (int r = 0; r < kTreeRows; ++r) {
      const float delta = (vn[r] - kv[r]) * beta;
      out[r] = 0.f;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        st[r][i] += kn[i] * delta;
        out[r] += st[r][i] * qn[i];
      }
    }
    warp_sum4(out);
    // shared nodes are walked by several rows; the first row that has one writes it
    if (lane == 0 && own) {
      const float o4[4] = {out[0], out[1], out[2], out[3]};
      store4(a.y + ((size_t)node * a.Hv + hv) * kGdnD + dv0, o4);
    }
  }
}

struct CommitArgs {
  const __nv_bfloat16 *k, *v, *beta, *conv_state, *qkv;
  const float *g, *state_in;
  const int32_t *conv_idx;
  float *state_out;
  __nv_bfloat16 *conv_out;
  int n, Hk, Hv, m, last;
  uint8_t nodes[kGdnMaxPath];
};

// grid (Dv / 8, Hv + 1), 256 threads; blockIdx.y == Hv copies the conv window
__global__ void __launch_bounds__(256) gdn_commit_kernel(CommitArgs a) {
  const int C = (2 * a.Hk + a.Hv) * kGdnD;
  if ((int)blockIdx.y == a.Hv) {
    for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < 3 * C; e += gridDim.x * blockDim.x) {
      const int j = e / C, ch = e - j * C;
      const int r = a.conv_idx[a.last * 4 + 1 + j];
      __nv_bfloat16 val = __float2bfloat16_rn(0.f);
      if (r >= 0 && r < 3) val = a.conv_state[(size_t)r * C + ch];
      else if (r >= 3 && r < 3 + a.n) val = a.qkv[(size_t)(r - 3) * C + ch];
      a.conv_out[e] = val;
    }
    return;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int dv = blockIdx.x * kGdnWarps + warp, hv = blockIdx.y;
  const int hk = hv / (a.Hv / a.Hk);
  const size_t srow = ((size_t)hv * kGdnD + dv) * kGdnD + lane * 4;
  const float4 s4 = *reinterpret_cast<const float4 *>(a.state_in + srow);
  float st[4] = {s4.x, s4.y, s4.z, s4.w};
  for (int t = 0; t < a.m; ++t) {
    const int node = a.nodes[t];
    float kn[4];
    load4(a.k + ((size_t)node * a.Hk + hk) * kGdnD + lane * 4, kn);
    const float gv = a.g[node * a.Hv + hv];
    float kv = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      st[i] *= gv;
      kv += st[i] * kn[i];
    }
    kv = warp_sum(kv);
    const size_t vi = (size_t)node * a.Hv + hv;
    const float delta = (__bfloat162float(a.v[vi * kGdnD + dv]) - kv) * __bfloat162float(a.beta[vi]);
#pragma unroll
    for (int i = 0; i < 4; ++i) st[i] += kn[i] * delta;
  }
  *reinterpret_cast<float4 *>(a.state_out + srow) = make_float4(st[0], st[1], st[2], st[3]);
}

bool gdn_heads_ok(int Hk, int Dk, int Hv, int Dv) {
  return Dk == kGdnD && Dv == kGdnD && Hk > 0 && Hv > 0 && Hv % Hk == 0 && Hv <= 4096;
}

}  // namespace
}  // namespace tsb

using namespace tsb;

extern "C" int tsb_gdn_prep(const void *qkv, const void *conv_state, const int32_t *conv_idx, const void *conv_w,
                            const void *a, const void *b, const float *a_log, const float *dt_bias, void *q, void *k,
                            void *v, float *g, void *beta, int n, int Hk, int Dk, int Hv, int Dv,
                            tsb_stream_t stream) {
  if (!qkv || !conv_state || !conv_idx || !conv_w || !a || !b || !a_log || !dt_bias || !q || !k || !v || !g || !beta)
    return TSB_EINVAL;
  if (n <= 0) return TSB_EINVAL;
  if (!gdn_heads_ok(Hk, Dk, Hv, Dv)) return TSB_EUNSUPPORTED;
  if (n > 65535) return TSB_EUNSUPPORTED;  // one grid row per node
  if (!aligned(qkv, 8) || !aligned(conv_state, 8) || !aligned(conv_w, 8) || !aligned(q, 8) || !aligned(k, 8) ||
      !aligned(v, 8))
    return TSB_EINVAL;
  PrepArgs p{static_cast<const __nv_bfloat16 *>(qkv), static_cast<const __nv_bfloat16 *>(conv_state),
             static_cast<const __nv_bfloat16 *>(conv_w), static_cast<const __nv_bfloat16 *>(a),
             static_cast<const __nv_bfloat16 *>(b), conv_idx, a_log, dt_bias, static_cast<__nv_bfloat16 *>(q),
             static_cast<__nv_bfloat16 *>(k), static_cast<__nv_bfloat16 *>(v), static_cast<__nv_bfloat16 *>(beta),
             g, n, Hk, Hv};
  const int slots = 2 * Hk + Hv + 1;
  gdn_prep_kernel<<<dim3((slots + 3) / 4, n), 128, 0, (cudaStream_t)stream>>>(p);
  return cudaGetLastError() == cudaSuccess ? TSB_OK : TSB_ECUDA;
}

extern "C" int tsb_tree_gated_delta(const void *q, const void *k, const void *v, const float *g, const void *beta,
                                    const float *state, const int32_t *paths, const int32_t *sibs,
                                    const int32_t *owner, int rows, int lmax, int n, int Hk, int Dk, int Hv, int Dv,
                                    void *y, tsb_stream_t stream) {
  if (!q || !k || !v || !g || !beta || !state || !paths || !sibs || !owner || !y) return TSB_EINVAL;
  if (n <= 0 || rows <= 0 || lmax <= 0 || rows > 65535) return TSB_EINVAL;
  if (!gdn_heads_ok(Hk, Dk, Hv, Dv) || Hv > 65535) return TSB_EUNSUPPORTED;
  if (!aligned(q, 8) || !aligned(k, 8) || !aligned(y, 8) || !aligned(state, 16)) return TSB_EINVAL;
  TreeArgs t{static_cast<const __nv_bfloat16 *>(q), static_cast<const __nv_bfloat16 *>(k),
             static_cast<const __nv_bfloat16 *>(v), static_cast<const __nv_bfloat16 *>(beta), g, state, paths, sibs,
             owner, static_cast<__nv_bfloat16 *>(y), n, rows, lmax, Hk, Hv};
  gdn_tree_kernel<<<dim3(kGdnD / kTreeDv, Hv, rows), 256, 0, (cudaStream_t)stream>>>(t);
  return cudaGetLastError() == cudaSuccess ? TSB_OK : TSB_ECUDA;
}

extern "C" int tsb_gdn_commit(const void *k, const void *v, const float *g, const void *beta, const float *state_in,
                              const void *conv_state, const void *qkv, const int32_t *conv_idx, const int32_t *nodes,
                              int n_keep, int n, int Hk, int Dk, int Hv, int Dv, float *state_out, void *conv_out,
                              tsb_stream_t stream) {
  if (!k || !v || !g || !beta || !state_in || !conv_state || !qkv || !conv_idx || !nodes || !state_out || !conv_out)
    return TSB_EINVAL;
  if (n <= 0 || n_keep <= 0) return TSB_EINVAL;
  if (!gdn_heads_ok(Hk, Dk, Hv, Dv) || Hv + 1 > 65535) return TSB_EUNSUPPORTED;
  if (n_keep > kGdnMaxPath) return TSB_EUNSUPPORTED;
  if (!aligned(k, 8) || !aligned(state_in, 16) || !aligned(state_out, 16)) return TSB_EINVAL;
  {
    // conv_out is written by several CTAs while others still read conv_state:
    // the two [3, C] bf16 ranges must not overlap
    const size_t bytes = (size_t)3 * (2 * Hk + Hv) * kGdnD * 2;
    const uintptr_t s0 = reinterpret_cast<uintptr_t>(conv_state), o0 = reinterpret_cast<uintptr_t>(conv_out);
    if (s0 < o0 + bytes && o0 < s0 + bytes) return TSB_EINVAL;
  }
  CommitArgs c{};
  c.k = static_cast<const __nv_bfloat16 *>(k);
  c.v = static_cast<const __nv_bfloat16 *>(v);
  c.beta = static_cast<const __nv_bfloat16 *>(beta);
  c.conv_state = static_cast<const __nv_bfloat16 *>(conv_state);
  c.qkv = static_cast<const __nv_bfloat16 *>(qkv);
  c.g = g;
  c.state_in = state_in;
  c.conv_idx = conv_idx;
  c.state_out = state_out;
  c.conv_out = static_cast<__nv_bfloat16 *>(conv_out);
  c.n = n;
  c.Hk = Hk;
  c.Hv = Hv;
  c.m = n_keep;
  for (int i = 0; i < n_keep; ++i) {
    if (nodes[i] < 0 || nodes[i] >= n || nodes[i] >= kGdnMaxPath) return TSB_EINVAL;
    c.nodes[i] = (uint8_t)nodes[i];
  }
  c.last = nodes[n_keep - 1];
  gdn_commit_kernel<<<dim3(kGdnD / kGdnWarps, Hv + 1), 256, 0, (cudaStream_t)stream>>>(c);
  return cudaGetLastError() == cudaSuccess ? TSB_OK : TSB_ECUDA;
}
