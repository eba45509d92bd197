// Kernels of the verify-step decoder layer around the two hot ops (the 4-bit
// qmm and tree attention): the reference's fused residual add + RMS norm, the
// per-node preparation of q/k/v (per-head RMS norm, rope at the node's depth,
// K/V append into the cache, quantized on append for the 8-bit formats), the
// sigmoid output gate of gated-q attention and the SwiGLU activation.
//
// Reference: mlx-tree-spec src/mlx_tree_spec/fused_ops.py:107-154
// (add_rms_norm), src/mlx_tree_spec/tree_verify.py:311-367 (batch_attention /
// _attn_core: q_proj split into queries and gate, q_norm/k_norm, rope at depth,
// cache.update_and_fetch, o_proj(out * sigmoid(gate))), 414-447 (the layer
// loop), and the mlx-lm modules those call (nn.RMSNorm = mx.fast.rms_norm,
// mx.fast.rope, SwiGLU MLP down(silu(gate(x)) * up(x))). The 8-bit appends
// follow kv8.py:39-43 (reference rows) and the MLX g64 affine quantizer this
// library documents (tsb/quant.py).
//
// All of these move a few MB per layer at the verify step's M = B*T <= 128
// rows: HBM-bound, vectorised 16-byte loads and stores, one launch each.
#include "sm100.cuh"

namespace tsb {
namespace {

constexpr int NORM_MAX_THREADS = 1024;
constexpr int NORM_MAX_VEC = 2;  // 16-byte vectors per thread: D <= 16384

TSB_HD float bf16r(float v) { return bf16_bits_to_float(float_to_bf16_bits(v)); }

TSB_HD void unpack8(const uint4 u, float (&f)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}
TSB_HD uint4 pack8(const float (&f)[8]) {
  return make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]), pack_bf16x2(f[4], f[5]),
                    pack_bf16x2(f[6], f[7]));
}

// h = bf16(x + r) (or x), n = bf16(w * bf16(h * rsqrt(mean(h^2) + eps))) per
// row: fused_ops.py:107-129 (and mx.fast.rms_norm's rounding when r is null).
// One CTA per row, one thread per 16-byte vector (up to two): a row is one
// round of loads, a block reduction and one round of stores.
__global__ void __launch_bounds__(NORM_MAX_THREADS)
add_rms_norm_kernel(const uint16_t *x, const uint16_t *r, const uint16_t *w, uint16_t *h_out, uint16_t *n_out, int D,
                    float eps) {
  griddep_wait();  // launched as a programmatic dependent: inputs and outputs are the previous kernels'
  griddep_launch_dependents();
  const size_t base = (size_t)blockIdx.x * D;
  const int nv = D / 8;
  const int nt = blockDim.x;
  float vals[NORM_MAX_VEC][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < NORM_MAX_VEC; ++i) {
    const int c = threadIdx.x + i * nt;
    if (c < nv) {
      unpack8(*reinterpret_cast<const uint4 *>(x + base + 8 * c), vals[i]);
      if (r) {
        float rv[8];
        unpack8(*reinterpret_cast<const uint4 *>(r + base + 8 * c), rv);
#pragma unroll
        for (int e = 0; e < 8; ++e) vals[i][e] = bf16r(vals[i][e] + rv[e]);
        if (h_out) *reinterpret_cast<uint4 *>(h_out + base + 8 * c) = pack8(vals[i]);
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) ss = fmaf(vals[i][e], vals[i][e], ss);
    }
  }
  __shared__ float red[NORM_MAX_THREADS / 32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float total = 0.f;
  for (int i = 0; i < nt / 32; ++i) total += red[i];
  const float inv = rsqrtf(total / (float)D + eps);
#pragma unroll
  for (int i = 0; i < NORM_MAX_VEC; ++i) {
    const int c = threadIdx.x + i * nt;
    if (c < nv) {
      float wv[8], o[8];
      unpack8(*reinterpret_cast<const uint4 *>(w + 8 * c), wv);
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = wv[e] * bf16r(vals[i][e] * inv);
      *reinterpret_cast<uint4 *>(n_out + base + 8 * c) = pack8(o);
    }
  }
}

struct PrepArgs {
  const uint16_t *qkv;
  int ld;                       // row stride of qkv (elements)
  int B, T, Hq, Hkv;
  const uint16_t *q_norm, *k_norm;
  float eps;
  const int32_t *positions;     // [B*T]: rope position of each node (depth + prefix)
  int rope_dims;
  float rope_log2_base, rope_scale;
  uint16_t *q_out;              // [B, Hq, T, 256]
  int kv_format, cap;
  const int32_t *offsets;       // [B]: cache row of each request's first node
  void *k, *v;                  // caches [B, Hkv, cap, ...] in kv_format
  void *ks, *kb, *vs, *vb;      // their scales / biases (8-bit formats)
};

// One 256-wide head row held by a warp, 8 values per lane: RMS norm with
// weight w (fp32 sum of squares over the row, rounding as above).
TSB_HD void warp_rms_norm(float (&f)[8], const uint16_t *w, int lane, float eps) {
  float ss = 0.f;
#pragma unroll
  for (int e = 0; e < 8; ++e) ss = fmaf(f[e], f[e], ss);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float inv = rsqrtf(ss / 256.f + eps);
  float wv[8];
  unpack8(*reinterpret_cast<const uint4 *>(w + 8 * lane), wv);
#pragma unroll
  for (int e = 0; e < 8; ++e) f[e] = bf16r(wv[e] * bf16r(f[e] * inv));
}

// mx.fast.rope, non-traditional, at one position: for i < dims/2 the pair
// (x_i, x_{i+dims/2}) turns by pos * scale * base^(-2i/dims); dims..255 pass
// through. Values of the pair partner come from lane +- dims/16; cos and sin
// of the node's angles come from a table (cs, sn) the CTA builds once.
TSB_HD void warp_rope(float (&f)[8], int lane, int dims, const float *cs_t, const float *sn_t) {
  const int half = dims / 2;
  const int dl = half / 8;  // lane distance of a pair
  const bool lo = lane < dl, hi = lane >= dl && lane < 2 * dl;
  const int src = lo ? lane + dl : (hi ? lane - dl : lane);
  float p[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) p[e] = __shfl_sync(0xffffffffu, f[e], src);
  if (!(lo || hi)) return;
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const int j = (lo ? lane : lane - dl) * 8 + e;  // frequency index in [0, half)
    const float cs = cs_t[j], sn = sn_t[j];
    f[e] = lo ? bf16r(f[e] * cs - p[e] * sn) : bf16r(p[e] * sn + f[e] * cs);
  }
}

// Append one 256-value row (8 per lane) to a cache in its format.
TSB_HD void warp_append(const PrepArgs &a, void *cache, void *sc, void *bi, size_t row, const float (&f)[8],
                        int lane) {
  if (a.kv_format == TSB_KV_BF16) {
    reinterpret_cast<uint4 *>(static_cast<uint16_t *>(cache) + row * 256)[lane] = pack8(f);
  } else if (a.kv_format == TSB_KV_REF_Q8_ROW) {
    // kv8.quantize_rows: s = max(max|x| / 127, 1e-6), q = clip(rint(x / s), -127, 127)
    float amax = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) amax = fmaxf(amax, fabsf(f[e]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float s = fmaxf(__fdiv_rn(amax, 127.f), 1e-6f);
    uint32_t w[2] = {0u, 0u};
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float q = fminf(fmaxf(rintf(__fdiv_rn(f[e], s)), -127.f), 127.f);
      w[e >> 2] |= ((uint32_t)(int)q & 0xFFu) << (8 * (e & 3));
    }
    reinterpret_cast<uint2 *>(static_cast<int8_t *>(cache) + row * 256)[lane] = make_uint2(w[0], w[1]);
    if (lane == 0) static_cast<float *>(sc)[row] = s;
  } else {
    // MLX g64 affine: per 64 values (8 lanes) s = bf16((max - min) / 255),
    // b = bf16(min), q = clamp(rint((x - b) / s), 0, 255) (0 where s == 0)
    float mn = f[0], mx = f[0];
#pragma unroll
    for (int e = 1; e < 8; ++e) { mn = fminf(mn, f[e]); mx = fmaxf(mx, f[e]); }
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) {
      mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    }
    const uint16_t sb = float_to_bf16_bits(__fdiv_rn(mx - mn, 255.f));
    const uint16_t bb = float_to_bf16_bits(mn);
    const float s = bf16_bits_to_float(sb), b = bf16_bits_to_float(bb);
    uint32_t w[2] = {0u, 0u};
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float q = s == 0.f ? 0.f : fminf(fmaxf(rintf(__fdiv_rn(f[e] - b, s)), 0.f), 255.f);
      w[e >> 2] |= (uint32_t)q << (8 * (e & 3));
    }
    reinterpret_cast<uint2 *>(static_cast<uint32_t *>(cache) + row * 64)[lane] = make_uint2(w[0], w[1]);
    if ((lane & 7) == 0) {
      static_cast<uint16_t *>(sc)[row * 4 + lane / 8] = sb;
      static_cast<uint16_t *>(bi)[row * 4 + lane / 8] = bb;
    }
  }
}

constexpr int PREP_THREADS = 256;

// One CTA per node: each warp takes head rows (queries, keys, values) in turn.
__global__ void __launch_bounds__(PREP_THREADS) qkv_prep_kernel(PrepArgs a) {
  griddep_wait();  // launched as a programmatic dependent: inputs and outputs are the previous kernels'
  griddep_launch_dependents();
  const int m = blockIdx.x;  // node = request * T + t
  const int b = m / a.T, t = m - b * a.T;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int pos = a.positions[m];
  const size_t cache_row0 = (size_t)a.offsets[b] + t;
  const uint16_t *row = a.qkv + (size_t)m * a.ld;
  const int nh = a.Hq + 2 * a.Hkv;
  // the node's rope angles pos * scale * base^(-j/half), j < half, once
  __shared__ float cs_t[128], sn_t[128];
  const int half = a.rope_dims / 2;
  for (int j = threadIdx.x; j < half; j += PREP_THREADS) {
    const float inv_freq = exp2f(-((float)j / (float)half) * a.rope_log2_base);
    sincosf((float)pos * a.rope_scale * inv_freq, &sn_t[j], &cs_t[j]);
  }
  __syncthreads();
  for (int hv = warp; hv < nh; hv += PREP_THREADS / 32) {
    float f[8];
    if (hv < a.Hq) {
      // query half of head hv (the gate half follows it)
      unpack8(*reinterpret_cast<const uint4 *>(row + (size_t)hv * 512 + 8 * lane), f);
      warp_rms_norm(f, a.q_norm, lane, a.eps);
      warp_rope(f, lane, a.rope_dims, cs_t, sn_t);
      *reinterpret_cast<uint4 *>(a.q_out + (((size_t)b * a.Hq + hv) * a.T + t) * 256 + 8 * lane) = pack8(f);
    } else if (hv < a.Hq + a.Hkv) {
      const int g = hv - a.Hq;
      unpack8(*reinterpret_cast<const uint4 *>(row + (size_t)a.Hq * 512 + (size_t)g * 256 + 8 * lane), f);
      warp_rms_norm(f, a.k_norm, lane, a.eps);
      warp_rope(f, lane, a.rope_dims, cs_t, sn_t);
      warp_append(a, a.k, a.ks, a.kb, ((size_t)b * a.Hkv + g) * a.cap + cache_row0, f, lane);
    } else {
      const int g = hv - a.Hq - a.Hkv;
      unpack8(*reinterpret_cast<const uint4 *>(row + (size_t)a.Hq * 512 + (size_t)(a.Hkv + g) * 256 + 8 * lane),
              f);
      warp_append(a, a.v, a.vs, a.vb, ((size_t)b * a.Hkv + g) * a.cap + cache_row0, f, lane);
    }
  }
}

// y[b*T + t, h*256 + d] = bf16(out[b, h, t, d] * bf16(sigmoid(gate))), gate =
// qkv[b*T + t, h*512 + 256 + d]: o_proj's input (tree_verify.py:327).
__global__ void attn_gate_kernel(const uint16_t *out, const uint16_t *qkv, int ld, uint16_t *y, int T, int Hq,
                                 size_t n_vec) {
  griddep_wait();  // launched as a programmatic dependent: inputs and outputs are the previous kernels'
  griddep_launch_dependents();
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;  // 16-byte vector of y
  if (i >= n_vec) return;
  const int per_row = Hq * 32;  // vectors per y row
  const int m = (int)(i / per_row);
  const int c = (int)(i - (size_t)m * per_row);
  const int h = c / 32, d8 = c % 32;
  const int b = m / T, t = m - b * T;
  float o[8], g[8];
  unpack8(*reinterpret_cast<const uint4 *>(out + (((size_t)b * Hq + h) * T + t) * 256 + 8 * d8), o);
  unpack8(*reinterpret_cast<const uint4 *>(qkv + (size_t)m * ld + (size_t)h * 512 + 256 + 8 * d8), g);
#pragma unroll
  for (int e = 0; e < 8; ++e) o[e] = o[e] * bf16r(1.f / (1.f + expf(-g[e])));
  reinterpret_cast<uint4 *>(y)[i] = pack8(o);
}

// y[m, i] = bf16(bf16(g * bf16(sigmoid(g))) * u), g = gu[m, i], u = gu[m, I + i].
__global__ void swiglu_kernel(const uint16_t *gu, uint16_t *y, int I, size_t n_vec) {
  griddep_wait();  // launched as a programmatic dependent: inputs and outputs are the previous kernels'
  griddep_launch_dependents();
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n_vec) return;
  const int per_row = I / 8;
  const size_t m = i / per_row;
  const int c = (int)(i - m * per_row);
  float g[8], u[8];
  unpack8(*reinterpret_cast<const uint4 *>(gu + m * (size_t)(2 * I) + 8 * c), g);
  unpack8(*reinterpret_cast<const uint4 *>(gu + m * (size_t)(2 * I) + I + 8 * c), u);
#pragma unroll
  for (int e = 0; e < 8; ++e) g[e] = bf16r(g[e] * bf16r(1.f / (1.f + expf(-g[e])))) * u[e];
  reinterpret_cast<uint4 *>(y)[i] = pack8(g);
}

}  // namespace
}  // namespace tsb

using namespace tsb;

extern "C" int tsb_add_rms_norm(const void *x, const void *r, const void *w, void *h_out, void *n_out, int rows,
                                int D, float eps, tsb_stream_t stream) {
  if (!x || !w || !n_out) return TSB_EINVAL;
  if (rows <= 0 || D <= 0) return TSB_EINVAL;
  if (D % 8 || D > NORM_MAX_THREADS * NORM_MAX_VEC * 8) return TSB_EUNSUPPORTED;
  if (!aligned(x, 16) || !aligned(w, 16) || !aligned(n_out, 16) || (r && !aligned(r, 16)) ||
      (h_out && !aligned(h_out, 16)))
    return TSB_EINVAL;
  // one thread per 16-byte vector, in whole warps; beyond 1024 vectors, two each
  const int nv = D / 8;
  const int threads = nv <= NORM_MAX_THREADS ? (nv + 31) / 32 * 32 : NORM_MAX_THREADS;
  const cudaError_t e = launch_pdl(add_rms_norm_kernel, dim3(rows), dim3(threads), 0, (cudaStream_t)stream,
                                   (const uint16_t *)x, (const uint16_t *)r, (const uint16_t *)w, (uint16_t *)h_out,
                                   (uint16_t *)n_out, D, eps);
  return e == cudaSuccess ? TSB_OK : TSB_ECUDA;
}

extern "C" int tsb_qkv_prep(const void *qkv, int ld, int B, int T, int Hq, int Hkv, int D, const void *q_norm,
                            const void *k_norm, float eps, const int32_t *positions, int rope_dims, float rope_base,
                            float rope_scale, void *q_out, int kv_format, void *k, void *k_scales, void *k_biases,
                            void *v, void *v_scales, void *v_biases, int kv_capacity, const int32_t *offsets,
                            tsb_stream_t stream) {
  if (!qkv || !q_norm || !k_norm || !positions || !q_out || !k || !v || !offsets) return TSB_EINVAL;
  if (B <= 0 || T <= 0 || Hq <= 0 || Hkv <= 0 || kv_capacity <= 0) return TSB_EINVAL;
  if (D != 256) return TSB_EUNSUPPORTED;
  if (rope_dims < 16 || rope_dims > D || rope_dims % 16) return TSB_EUNSUPPORTED;
  if (!(rope_base > 0.f)) return TSB_EINVAL;
  if (kv_format < 0 || kv_format > 2) return TSB_EUNSUPPORTED;
  if (kv_format == TSB_KV_MLX_Q8_G64 && (!k_scales || !k_biases || !v_scales || !v_biases)) return TSB_EINVAL;
  if (kv_format == TSB_KV_REF_Q8_ROW && (!k_scales || !v_scales)) return TSB_EINVAL;
  if ((long long)ld < (long long)(2 * Hq + 2 * Hkv) * D || ld % 8) return TSB_EINVAL;
  if (!aligned(qkv, 16) || !aligned(q_norm, 16) || !aligned(k_norm, 16) || !aligned(q_out, 16) || !aligned(k, 16) ||
      !aligned(v, 16))
    return TSB_EINVAL;
  PrepArgs a;
  a.qkv = (const uint16_t *)qkv;
  a.ld = ld;
  a.B = B; a.T = T; a.Hq = Hq; a.Hkv = Hkv;
  a.q_norm = (const uint16_t *)q_norm;
  a.k_norm = (const uint16_t *)k_norm;
  a.eps = eps;
  a.positions = positions;
  a.rope_dims = rope_dims;
  a.rope_log2_base = log2f(rope_base);
  a.rope_scale = rope_scale;
  a.q_out = (uint16_t *)q_out;
  a.kv_format = kv_format;
  a.cap = kv_capacity;
  a.offsets = offsets;
  a.k = k; a.v = v;
  a.ks = k_scales; a.kb = k_biases; a.vs = v_scales; a.vb = v_biases;
  const cudaError_t e = launch_pdl(qkv_prep_kernel, dim3(B * T), dim3(PREP_THREADS), 0, (cudaStream_t)stream, a);
  return e == cudaSuccess ? TSB_OK : TSB_ECUDA;
}

extern "C" int tsb_attn_gate(const void *attn_out, const void *qkv, int ld, void *y, int B, int T, int Hq, int D,
                             tsb_stream_t stream) {
  if (!attn_out || !qkv || !y) return TSB_EINVAL;
  if (B <= 0 || T <= 0 || Hq <= 0) return TSB_EINVAL;
  if (D != 256) return TSB_EUNSUPPORTED;
  if ((long long)ld < (long long)2 * Hq * D || ld % 8) return TSB_EINVAL;
  if (!aligned(attn_out, 16) || !aligned(qkv, 16) || !aligned(y, 16)) return TSB_EINVAL;
  const size_t n_vec = (size_t)B * T * Hq * (D / 8);
  const cudaError_t e = launch_pdl(attn_gate_kernel, dim3((unsigned)((n_vec + 255) / 256)), dim3(256), 0,
                                   (cudaStream_t)stream, (const uint16_t *)attn_out, (const uint16_t *)qkv, ld,
                                   (uint16_t *)y, T, Hq, n_vec);
  return e == cudaSuccess ? TSB_OK : TSB_ECUDA;
}

extern "C" int tsb_swiglu(const void *gate_up, void *y, int M, int I, tsb_stream_t stream) {
  if (!gate_up || !y) return TSB_EINVAL;
  if (M <= 0 || I <= 0) return TSB_EINVAL;
  if (I % 8) return TSB_EUNSUPPORTED;
  if (!aligned(gate_up, 16) || !aligned(y, 16)) return TSB_EINVAL;
  const size_t n_vec = (size_t)M * (I / 8);
  const cudaError_t e = launch_pdl(swiglu_kernel, dim3((unsigned)((n_vec + 255) / 256)), dim3(256), 0,
                                   (cudaStream_t)stream, (const uint16_t *)gate_up, (uint16_t *)y, I, n_vec);
  return e == cudaSuccess ? TSB_OK : TSB_ECUDA;
}
