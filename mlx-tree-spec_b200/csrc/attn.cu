// Tree-mask flash attention: T tree-node queries of G = Hq/Hkv heads over one
// KV head's long prefix plus the nodes' own rows. Calls go to the tcgen05
// kernel (attn_tc.cu) whenever it takes them; the warp-MMA kernel below serves
// the rest (MLX 8-bit caches with an odd capacity or unaligned scale/bias
// rows) and owns the entry points, the plan and the split combine.
//
// Semantics follow mlx-tree-spec `tree_flash` (src/mlx_tree_spec/tree_flash.py:
// 151-196; visibility at 40-45): key row j < n_kv is visible to node t iff it
// lies before the tail or its tail bit is set in the node's mask. The masks
// come from the parent array (computed in the kernel prologue) or are given.
//
// Layout: one CTA owns (request b, KV head, a block of query rows, a key
// split). The G*T query rows of a KV head are packed (row = head_local * T +
// node), so each K/V tile is read once per row block for all of that KV head's
// query heads. Warps own 16 rows each; K/V tiles of 64 keys are staged in
// XOR-swizzled shared memory (cp.async for bf16; converted on the way in for
// the 8-bit formats) and double-buffered. Scores and PV use the warp MMA with
// fp32 accumulation; online softmax in registers (exp2 domain). With more than
// one key split, each split writes normalised partial outputs plus (max, sum)
// to the workspace and a combine kernel merges them (the reference's reduce
// kernel, tree_flash.py:187-194).
//
// 8-bit formats: REF_Q8_ROW keeps the int8 values exact in bf16 and applies the
// scales outside the matmuls as the reference's q8 kernel does
// (tree_flash.py:14-19,86-100): a key's scale multiplies its scores, a value's
// scale the softmax weight it meets; running sums use the unscaled weights.
// MLX_Q8_G64 rows are dequantized (s * q + b, rounded to bf16) into the tile.
#include "sm100.cuh"

#include <algorithm>
#include <mutex>

namespace tsb {

namespace {

constexpr int AT_D = 256;
constexpr int AT_KT = 64;          // keys per tile
constexpr int AT_MAXW = 8;         // warps per CTA (16 query rows each)
constexpr int AT_ROW_BYTES = AT_D * 2;
constexpr int AT_TILE_BYTES = AT_KT * AT_ROW_BYTES;  // 32 KB

TSB_HD uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

TSB_HD void cp_async16(uint32_t dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src));
}
TSB_HD void cp_async_commit() { asm volatile("cp.async.commit_group;"); }
TSB_HD void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

TSB_HD void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
TSB_HD void ldsm_x4_t(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}

// Byte offset of 16-byte chunk `ch` (0..31) of row `r` in a swizzled 512-byte-row tile.
TSB_HD uint32_t swz(int r, int ch) { return (uint32_t)(r * AT_ROW_BYTES + ((ch ^ (r & 7)) << 4)); }

struct AttnArgs {
  const uint16_t *q;
  const void *k, *ks, *kb, *v, *vs, *vb;
  const int32_t *parents;
  const unsigned long long *bits;
  int B, T, Hq, Hkv, n_kv, tail, cap;
  int rows_per_cta, row_blocks, splits, tiles_per_split;
  float scale_log2;  // scale * log2(e)
  uint16_t *out;
  float *lse;
  float *part_o;   // [splits][B][Hq][T][D]
  float *part_ml;  // [splits][B][Hq][T][2]
};

// Stage one K or V tile (keys j0 .. j0+63) into swizzled shared memory.
// bf16: cp.async. 8-bit formats: load, convert to bf16, store. Rows >= n_kv
// are zero-filled (they are masked anyway; zero keeps NaN/Inf garbage out).
template <int FMT>
TSB_HD void stage_tile(const AttnArgs &a, const void *base, const void *sc, const void *bi, size_t head_row0,
                       int j0, unsigned char *dst, float *rowscale, int tid, int nthreads) {
  if constexpr (FMT == TSB_KV_BF16) {
    const uint16_t *src = reinterpret_cast<const uint16_t *>(base);
    for (int i = tid; i < AT_KT * 32; i += nthreads) {
      const int r = i >> 5, ch = i & 31;
      const int j = j0 + r;
      const uint32_t d = smem_u32(dst + swz(r, ch));
      if (j < a.n_kv) {
        cp_async16(d, src + (head_row0 + j) * AT_D + ch * 8);
      } else {
        *reinterpret_cast<uint4 *>(dst + swz(r, ch)) = make_uint4(0, 0, 0, 0);
      }
    }
  } else if constexpr (FMT == TSB_KV_REF_Q8_ROW) {
    const int8_t *src = reinterpret_cast<const int8_t *>(base);
    const float *scp = reinterpret_cast<const float *>(sc);
    for (int i = tid; i < AT_KT * 16; i += nthreads) {  // 16 B of int8 = 16 values = 2 chunks
      const int r = i >> 4, c16 = i & 15;
      const int j = j0 + r;
      uint4 lo = make_uint4(0, 0, 0, 0), hi = lo;
      if (j < a.n_kv) {
        const uint4 raw = *reinterpret_cast<const uint4 *>(src + (head_row0 + j) * AT_D + c16 * 16);
        const uint32_t wv[4] = {raw.x, raw.y, raw.z, raw.w};
        uint32_t o[8];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float f0 = (float)(int8_t)(wv[e] & 0xFF), f1 = (float)(int8_t)((wv[e] >> 8) & 0xFF);
          const float f2 = (float)(int8_t)((wv[e] >> 16) & 0xFF), f3 = (float)(int8_t)(wv[e] >> 24);
          o[2 * e] = pack_bf16x2(f0, f1);
          o[2 * e + 1] = pack_bf16x2(f2, f3);
        }
        lo = make_uint4(o[0], o[1], o[2], o[3]);
        hi = make_uint4(o[4], o[5], o[6], o[7]);
      }
      *reinterpret_cast<uint4 *>(dst + swz(r, 2 * c16)) = lo;
      *reinterpret_cast<uint4 *>(dst + swz(r, 2 * c16 + 1)) = hi;
    }
    for (int r = tid; r < AT_KT; r += nthreads) {
      const int j = j0 + r;
      rowscale[r] = j < a.n_kv ? scp[head_row0 + j] : 0.f;
    }
  } else {  // TSB_KV_MLX_Q8_G64
    const uint32_t *src = reinterpret_cast<const uint32_t *>(base);
    const uint16_t *scp = reinterpret_cast<const uint16_t *>(sc);
    const uint16_t *bip = reinterpret_cast<const uint16_t *>(bi);
    for (int i = tid; i < AT_KT * 16; i += nthreads) {  // 4 words = 16 codes = 2 chunks
      const int r = i >> 4, c16 = i & 15;
      const int j = j0 + r;
      uint4 lo = make_uint4(0, 0, 0, 0), hi = lo;
      if (j < a.n_kv) {
        const uint4 raw = *reinterpret_cast<const uint4 *>(src + (head_row0 + j) * (AT_D / 4) + c16 * 4);
        const int g = c16 / 4;  // 64 values per group
        const float s = bf16_bits_to_float(scp[(head_row0 + j) * (AT_D / 64) + g]);
        const float b = bf16_bits_to_float(bip[(head_row0 + j) * (AT_D / 64) + g]);
        const uint32_t wv[4] = {raw.x, raw.y, raw.z, raw.w};
        uint32_t o[8];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float f0 = __fmaf_rn((float)(wv[e] & 0xFF), s, b);
          const float f1 = __fmaf_rn((float)((wv[e] >> 8) & 0xFF), s, b);
          const float f2 = __fmaf_rn((float)((wv[e] >> 16) & 0xFF), s, b);
          const float f3 = __fmaf_rn((float)(wv[e] >> 24), s, b);
          o[2 * e] = pack_bf16x2(f0, f1);
          o[2 * e + 1] = pack_bf16x2(f2, f3);
        }
        lo = make_uint4(o[0], o[1], o[2], o[3]);
        hi = make_uint4(o[4], o[5], o[6], o[7]);
      }
      *reinterpret_cast<uint4 *>(dst + swz(r, 2 * c16)) = lo;
      *reinterpret_cast<uint4 *>(dst + swz(r, 2 * c16 + 1)) = hi;
    }
  }
}

template <int FMT>
__global__ void __launch_bounds__(AT_MAXW * 32, 1) tree_attn_kernel(AttnArgs a) {
  extern __shared__ __align__(1024) unsigned char smem[];
  unsigned char *sQ = smem;                                   // rows_per_cta x 512 B
  unsigned char *sK0 = sQ + AT_MAXW * 16 * AT_ROW_BYTES;      // 2 x K tile
  unsigned char *sV0 = sK0 + 2 * AT_TILE_BYTES;               // 2 x V tile
  float *sKs = reinterpret_cast<float *>(sV0 + 2 * AT_TILE_BYTES);  // 2 x 64 key scales
  float *sVs = sKs + 2 * AT_KT;                                     // 2 x 64 value scales
  unsigned long long *sBits = reinterpret_cast<unsigned long long *>(sVs + 2 * AT_KT);  // T <= 64

  const int tid = threadIdx.x, nthreads = blockDim.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int gid = lane >> 2, c = lane & 3;
  const int G = a.Hq / a.Hkv;
  const int R = G * a.T;

  int unit = blockIdx.x;
  const int split = blockIdx.y;
  const int rb = unit % a.row_blocks;
  unit /= a.row_blocks;
  const int kh = unit % a.Hkv;
  const int b = unit / a.Hkv;
  const int row0 = rb * a.rows_per_cta;

  // ---- node masks (in-kernel from parents, or given) ----
  for (int node = tid; node < a.T; node += nthreads) {
    unsigned long long m = 0;
    if (a.parents) {
      const int32_t *p = a.parents + (size_t)b * a.T;
      int j = node;
      bool ok = true;
      for (int steps = 0; steps <= a.T && j != -1; ++steps) {
        m |= 1ull << j;
        const int pj = p[j];
        if (!(pj == -1 || (pj >= 0 && pj < j))) { ok = false; break; }
        j = pj;
      }
      if (!ok) m = 0;
    } else {
      m = a.bits[(size_t)b * a.T + node];
    }
    sBits[node] = m;
  }

  // ---- Q rows -> shared (zero rows past R) ----
  for (int i = tid; i < a.rows_per_cta * 32; i += nthreads) {
    const int r = i >> 5, ch = i & 31;
    const int gr = row0 + r;
    uint4 val = make_uint4(0, 0, 0, 0);
    if (gr < R) {
      const int hl = gr / a.T, t = gr % a.T;
      const int h = kh * G + hl;
      val = *reinterpret_cast<const uint4 *>(a.q + (((size_t)b * a.Hq + h) * a.T + t) * AT_D + ch * 8);
    }
    *reinterpret_cast<uint4 *>(sQ + swz(r, ch)) = val;
  }

  const size_t head_row0 = ((size_t)b * a.Hkv + kh) * (size_t)a.cap;
  const int tile_begin = split * a.tiles_per_split;
  const int n_tiles_total = (a.n_kv + AT_KT - 1) / AT_KT;
  const int tile_end = min(n_tiles_total, tile_begin + a.tiles_per_split);
  const int tail_lo = a.n_kv - a.tail;

  // per-thread rows: r_lo = warp*16 + gid, r_hi = r_lo + 8
  const int r_lo = warp * 16 + gid, r_hi = r_lo + 8;
  const bool warp_live = (row0 + warp * 16) < R;
  const int node_lo = (row0 + r_lo) % a.T, node_hi = (row0 + r_hi) % a.T;

  float o[32][4];
#pragma unroll
  for (int i = 0; i < 32; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_lo = -INFINITY, m_hi = -INFINITY, l_lo = 0.f, l_hi = 0.f;

  if (tile_begin < tile_end) {
    stage_tile<FMT>(a, a.k, a.ks, a.kb, head_row0, tile_begin * AT_KT, sK0, sKs, tid, nthreads);
    stage_tile<FMT>(a, a.v, a.vs, a.vb, head_row0, tile_begin * AT_KT, sV0, sVs, tid, nthreads);
    if constexpr (FMT == TSB_KV_BF16) cp_async_commit();
  }

  for (int it = tile_begin; it < tile_end; ++it) {
    const int buf = (it - tile_begin) & 1;
    if constexpr (FMT == TSB_KV_BF16) cp_async_wait_all();
    __syncthreads();
    // prefetch the next tile into the other buffer (its previous readers are done)
    if (it + 1 < tile_end) {
      stage_tile<FMT>(a, a.k, a.ks, a.kb, head_row0, (it + 1) * AT_KT, sK0 + (buf ^ 1) * AT_TILE_BYTES,
                      sKs + (buf ^ 1) * AT_KT, tid, nthreads);
      stage_tile<FMT>(a, a.v, a.vs, a.vb, head_row0, (it + 1) * AT_KT, sV0 + (buf ^ 1) * AT_TILE_BYTES,
                      sVs + (buf ^ 1) * AT_KT, tid, nthreads);
      if constexpr (FMT == TSB_KV_BF16) cp_async_commit();
    }
    if (!warp_live) continue;
    const unsigned char *sK = sK0 + buf * AT_TILE_BYTES;
    const unsigned char *sV = sV0 + buf * AT_TILE_BYTES;
    const int j0 = it * AT_KT;

    // ---- S = Q K^T (16 rows x 64 keys per warp) ----
    float s[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < 16; ++ks) {
      uint32_t qa[4];
      {
        const int mi = lane >> 3;
        const int r = warp * 16 + (lane & 7) + 8 * (mi & 1);
        ldsm_x4(smem_u32(sQ + swz(r, 2 * ks + (mi >> 1))), qa[0], qa[1], qa[2], qa[3]);
      }
#pragma unroll
      for (int n = 0; n < 8; n += 2) {
        uint32_t k0, k1, k2, k3;
        const int mi = lane >> 3;
        const int key = 8 * (n + (mi >> 1)) + (lane & 7);
        ldsm_x4(smem_u32(sK + swz(key, 2 * ks + (mi & 1))), k0, k1, k2, k3);
        mma_bf16_16816(s[n], qa, k0, k1, s[n]);
        mma_bf16_16816(s[n + 1], qa, k2, k3, s[n + 1]);
      }
    }

    // ---- scale, mask, online softmax ----
    const bool need_mask = (j0 + AT_KT > tail_lo) || (j0 + AT_KT > a.n_kv);
    const unsigned long long bl = sBits[node_lo], bh = sBits[node_hi];
    float mx_lo = -INFINITY, mx_hi = -INFINITY;
#pragma unroll
    for (int n = 0; n < 8; ++n) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int kl = 8 * n + 2 * c + e;
        float ksc = a.scale_log2;
        if constexpr (FMT == TSB_KV_REF_Q8_ROW) ksc *= sKs[buf * AT_KT + kl];
        float vlo = s[n][e] * ksc, vhi = s[n][2 + e] * ksc;
        if (need_mask) {
          const int j = j0 + kl;
          bool vis_lo = j < a.n_kv, vis_hi = vis_lo;
          if (vis_lo && j >= tail_lo) {
            const int tp = j - tail_lo;
            vis_lo = (bl >> tp) & 1ull;
            vis_hi = (bh >> tp) & 1ull;
          }
          if (!vis_lo) vlo = -INFINITY;
          if (!vis_hi) vhi = -INFINITY;
        }
        s[n][e] = vlo;
        s[n][2 + e] = vhi;
        mx_lo = fmaxf(mx_lo, vlo);
        mx_hi = fmaxf(mx_hi, vhi);
      }
    }
    mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffffu, mx_lo, 1));
    mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffffu, mx_lo, 2));
    mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffffu, mx_hi, 1));
    mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffffu, mx_hi, 2));
    const float mn_lo = fmaxf(m_lo, mx_lo), mn_hi = fmaxf(m_hi, mx_hi);
    // rows that have seen nothing yet keep a -inf max; use 0 as the exp base then
    const float base_lo = mn_lo == -INFINITY ? 0.f : mn_lo;
    const float base_hi = mn_hi == -INFINITY ? 0.f : mn_hi;
    const float alpha_lo = exp2f(m_lo - base_lo), alpha_hi = exp2f(m_hi - base_hi);
    m_lo = mn_lo;
    m_hi = mn_hi;
    float ps_lo = 0.f, ps_hi = 0.f;
    uint32_t pa[4][4];  // P as A fragments, 4 key steps of 16
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      const float p0 = exp2f(s[n][0] - base_lo), p1 = exp2f(s[n][1] - base_lo);
      const float p2 = exp2f(s[n][2] - base_hi), p3 = exp2f(s[n][3] - base_hi);
      ps_lo += p0 + p1;
      ps_hi += p2 + p3;
      float w0 = p0, w1 = p1, w2 = p2, w3 = p3;
      if constexpr (FMT == TSB_KV_REF_Q8_ROW) {
        const float v0 = sVs[buf * AT_KT + 8 * n + 2 * c], v1 = sVs[buf * AT_KT + 8 * n + 2 * c + 1];
        w0 *= v0; w1 *= v1; w2 *= v0; w3 *= v1;
      }
      const int kstep = n >> 1, half = n & 1;
      pa[kstep][2 * half + 0] = pack_bf16x2(w0, w1);  // row gid
      pa[kstep][2 * half + 1] = pack_bf16x2(w2, w3);  // row gid+8
    }
    l_lo = l_lo * alpha_lo + ps_lo;
    l_hi = l_hi * alpha_hi + ps_hi;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      o[i][0] *= alpha_lo; o[i][1] *= alpha_lo;
      o[i][2] *= alpha_hi; o[i][3] *= alpha_hi;
    }
    // ---- O += P V ----
#pragma unroll
    for (int kstep = 0; kstep < 4; ++kstep) {
      // A-fragment register order: {row gid, k 0-7}, {row gid+8, k 0-7}, {row gid, k 8-15}, {row gid+8, k 8-15}
      const uint32_t af[4] = {pa[kstep][0], pa[kstep][1], pa[kstep][2], pa[kstep][3]};
#pragma unroll
      for (int dt = 0; dt < 32; dt += 2) {
        uint32_t v0, v1, v2, v3;
        const int mi = lane >> 3;
        const int key = 16 * kstep + (lane & 7) + 8 * (mi & 1);
        ldsm_x4_t(smem_u32(sV + swz(key, dt + (mi >> 1))), v0, v1, v2, v3);
        mma_bf16_16816(o[dt], af, v0, v1, o[dt]);
        mma_bf16_16816(o[dt + 1], af, v2, v3, o[dt + 1]);
      }
    }
  }

  if (!warp_live) return;
  // row sums across the quad
  l_lo += __shfl_xor_sync(0xffffffffu, l_lo, 1);
  l_lo += __shfl_xor_sync(0xffffffffu, l_lo, 2);
  l_hi += __shfl_xor_sync(0xffffffffu, l_hi, 1);
  l_hi += __shfl_xor_sync(0xffffffffu, l_hi, 2);
  const float inv_lo = l_lo > 0.f ? 1.f / l_lo : 0.f;
  const float inv_hi = l_hi > 0.f ? 1.f / l_hi : 0.f;
  const int gr_lo = row0 + r_lo, gr_hi = row0 + r_hi;
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const int gr = half ? gr_hi : gr_lo;
    if (gr >= R) continue;
    const float inv = half ? inv_hi : inv_lo;
    const float mm = half ? m_hi : m_lo;
    const float ll = half ? l_hi : l_lo;
    const int hl = gr / a.T, t = gr % a.T;
    const int h = kh * G + hl;
    const size_t orow = ((size_t)b * a.Hq + h) * a.T + t;
    if (a.splits == 1) {
      uint16_t *dst = a.out + orow * AT_D;
#pragma unroll
      for (int dt = 0; dt < 32; ++dt) {
        const int d = dt * 8 + 2 * c;
        *reinterpret_cast<uint32_t *>(dst + d) = pack_bf16x2(o[dt][2 * half] * inv, o[dt][2 * half + 1] * inv);
      }
      if (a.lse && c == 0)
        a.lse[orow] = ll > 0.f ? (mm + log2f(ll)) * 0.69314718055994531f : -INFINITY;
    } else {
      const size_t prow = (size_t)split * a.B * a.Hq * a.T + orow;
      float *dst = a.part_o + prow * AT_D;
#pragma unroll
      for (int dt = 0; dt < 32; ++dt) {
        const int d = dt * 8 + 2 * c;
        *reinterpret_cast<float2 *>(dst + d) = make_float2(o[dt][2 * half] * inv, o[dt][2 * half + 1] * inv);
      }
      if (c == 0) {
        a.part_ml[prow * 2 + 0] = mm;
        a.part_ml[prow * 2 + 1] = ll;
      }
    }
  }
}

// Merge the key splits of each output row: weights l_s * 2^(m_s - m).
constexpr int CB_ROWS = 4;          // query rows per combine block
constexpr int CB_MAX_SPLITS = 256;  // split weights held in shared memory per row

// Merge split-KV partials (the reference's two-pass reduce, tree_flash.py:130-143):
// out = sum_s w_s * o_s with w_s = l_s * 2^(m_s - m) / sum_s l_s * 2^(m_s - m).
// One warp per row computes the split weights in parallel into shared memory;
// then 64 threads per row accumulate float4 slices with independent loads.
__global__ void __launch_bounds__(256) tree_attn_combine_kernel(const float *__restrict__ part_o,
                                                                const float *__restrict__ part_ml, int splits,
                                                                int rows, uint16_t *__restrict__ out,
                                                                float *__restrict__ lse) {
  griddep_wait();  // launched as a programmatic dependent: the partials are the attention kernel's
  griddep_launch_dependents();
  __shared__ float sw[CB_ROWS][CB_MAX_SPLITS];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = blockIdx.x * CB_ROWS;
  if (warp < CB_ROWS && row0 + warp < rows) {
    const int row = row0 + warp;
    float m = -INFINITY;
    for (int s = lane; s < splits; s += 32) {
      const float2 ml = __ldg(reinterpret_cast<const float2 *>(part_ml) + (size_t)s * rows + row);
      if (ml.y > 0.f) m = fmaxf(m, ml.x);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float den = 0.f;
    for (int s = lane; s < splits; s += 32) {
      const float2 ml = __ldg(reinterpret_cast<const float2 *>(part_ml) + (size_t)s * rows + row);
      const float w = ml.y > 0.f ? ml.y * exp2f(ml.x - m) : 0.f;
      sw[warp][s] = w;
      den += w;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) den += __shfl_xor_sync(0xffffffffu, den, o);
    const float inv = den > 0.f ? 1.f / den : 0.f;
    for (int s = lane; s < splits; s += 32) sw[warp][s] *= inv;
    if (lse && lane == 0) lse[row] = den > 0.f ? (m + log2f(den)) * 0.69314718055994531f : -INFINITY;
  }
  __syncthreads();
  const int r = threadIdx.x >> 6;
  const int row = row0 + r;
  if (row >= rows) return;
  const int c = (threadIdx.x & 63) * 4;
  const float4 *po = reinterpret_cast<const float4 *>(part_o + (size_t)row * AT_D + c);
  const size_t stride = (size_t)rows * (AT_D / 4);
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  int s = 0;
  for (; s + 4 <= splits; s += 4) {
    float4 v[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = __ldg(po + (size_t)(s + i) * stride);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float w = sw[r][s + i];
      acc.x = fmaf(w, v[i].x, acc.x);
      acc.y = fmaf(w, v[i].y, acc.y);
      acc.z = fmaf(w, v[i].z, acc.z);
      acc.w = fmaf(w, v[i].w, acc.w);
    }
  }
  for (; s < splits; ++s) {
    const float4 v = __ldg(po + (size_t)s * stride);
    const float w = sw[r][s];
    acc.x = fmaf(w, v.x, acc.x);
    acc.y = fmaf(w, v.y, acc.y);
    acc.z = fmaf(w, v.z, acc.z);
    acc.w = fmaf(w, v.w, acc.w);
  }
  *reinterpret_cast<uint2 *>(out + (size_t)row * AT_D + c) =
      make_uint2(pack_bf16x2(acc.x, acc.y), pack_bf16x2(acc.z, acc.w));
}

void launch_combine(const float *part_o, const float *part_ml, int splits, int rows, void *out, float *lse,
                    cudaStream_t st) {
  launch_pdl(tree_attn_combine_kernel, dim3((unsigned)((rows + CB_ROWS - 1) / CB_ROWS)), dim3(256), 0, st, part_o,
             part_ml, splits, rows, (uint16_t *)out, lse);
}

struct AttnPlan {
  int rows_per_cta, row_blocks, splits, tiles_per_split;
};

AttnPlan plan_attn(int B, int T, int Hq, int Hkv, int n_kv) {
  AttnPlan p;
  const int R = (Hq / Hkv) * T;
  p.row_blocks = (R + AT_MAXW * 16 - 1) / (AT_MAXW * 16);
  const int warps = (R + 16 * p.row_blocks - 1) / (16 * p.row_blocks);
  p.rows_per_cta = warps * 16;
  const int units = B * Hkv * p.row_blocks;
  const int n_tiles = (n_kv + AT_KT - 1) / AT_KT;
  int splits = (sm_count() + units - 1) / units;
  if (splits > n_tiles / 2) splits = n_tiles / 2;
  if (splits > CB_MAX_SPLITS) splits = CB_MAX_SPLITS;
  if (splits < 1) splits = 1;
  p.tiles_per_split = (n_tiles + splits - 1) / splits;
  p.splits = (n_tiles + p.tiles_per_split - 1) / p.tiles_per_split;
  return p;
}

size_t attn_smem_bytes() {
  return (size_t)AT_MAXW * 16 * AT_ROW_BYTES + 4 * (size_t)AT_TILE_BYTES + 4 * AT_KT * sizeof(float) +
         64 * sizeof(unsigned long long);
}

}  // namespace

void plan_attn_tc(int B, int T, int Hq, int Hkv, int n_kv, int &row_blocks, int &splits, int &tiles_per_split);
bool attn_tc_supported(int kv_format, int cap, const void *ks, const void *kb, const void *vs, const void *vb);
int launch_attn_tc(int kv_format, const uint16_t *q, const void *k, const void *ks, const void *kb, const void *v,
                   const void *vs, const void *vb, const int32_t *parents, const unsigned long long *bits, int B,
                   int T, int Hq, int Hkv, int n_kv, int tail, int cap, float scale, uint16_t *out, float *lse,
                   float *part_o, float *part_ml, cudaStream_t st);

}  // namespace tsb

using namespace tsb;

// Key splits of a call. bf16 and reference-int8 KV always run the tcgen05
// kernel; MLX 8-bit KV runs it when its scale/bias rows can be bulk-copied
// (attn_tc_supported) and the warp-MMA kernel otherwise, so its workspace
// covers whichever of the two plans splits more.
static int attn_splits(int B, int T, int Hq, int Hkv, int n_kv, int kv_format) {
  int rb, splits, tps;
  plan_attn_tc(B, T, Hq, Hkv, n_kv, rb, splits, tps);
  if (kv_format == TSB_KV_MLX_Q8_G64) splits = std::max(splits, plan_attn(B, T, Hq, Hkv, n_kv).splits);
  return splits;
}

extern "C" size_t tsb_tree_attn_workspace_bytes(int B, int T, int Hq, int Hkv, int D, int n_kv, int kv_format) {
  (void)D;
  if (B <= 0 || T <= 0 || Hq <= 0 || Hkv <= 0 || n_kv <= 0) return 0;
  const int splits = attn_splits(B, T, Hq, Hkv, n_kv, kv_format);
  if (splits <= 1) return 0;
  const size_t rows = (size_t)B * Hq * T;
  return (size_t)splits * rows * (AT_D + 2) * sizeof(float) + 256;
}

extern "C" int tsb_tree_attn(const void *q, const void *k, const void *k_scales, const void *k_biases,
                             const void *v, const void *v_scales, const void *v_biases, int kv_format,
                             const int32_t *parents, const uint64_t *bits, int B, int T, int Hq, int Hkv, int D,
                             int n_kv, int tail, int kv_capacity, float scale, void *out, float *lse, void *ws,
                             size_t ws_bytes, tsb_stream_t stream) {
  if (!q || !k || !v || !out) return TSB_EINVAL;
  if (B <= 0 || T <= 0 || Hq <= 0 || Hkv <= 0 || n_kv <= 0 || kv_capacity < n_kv) return TSB_EINVAL;
  if (D != AT_D) return TSB_EUNSUPPORTED;
  if (Hq % Hkv) return TSB_EUNSUPPORTED;
  if (T > 64) return TSB_EUNSUPPORTED;
  if (!parents && !bits) return TSB_EINVAL;
  if (parents) tail = T;
  if (tail < 0 || tail > 64 || tail > n_kv) return TSB_EUNSUPPORTED;
  if (kv_format == TSB_KV_MLX_Q8_G64 && (!k_scales || !k_biases || !v_scales || !v_biases)) return TSB_EINVAL;
  if (kv_format == TSB_KV_REF_Q8_ROW && (!k_scales || !v_scales)) return TSB_EINVAL;
  if (kv_format < 0 || kv_format > 2) return TSB_EUNSUPPORTED;
  if (!aligned(q, 16) || !aligned(k, 16) || !aligned(v, 16) || !aligned(out, 16)) return TSB_EINVAL;

  const size_t rows = (size_t)B * Hq * T;
  cudaStream_t st = (cudaStream_t)stream;
  if (attn_tc_supported(kv_format, kv_capacity, k_scales, k_biases, v_scales, v_biases)) {
    if (!(scale > 0.f)) return TSB_EUNSUPPORTED;  // the kernel takes row maxima of unscaled scores
    int rb, splits, tps;
    plan_attn_tc(B, T, Hq, Hkv, n_kv, rb, splits, tps);
    float *part_o = nullptr, *part_ml = nullptr;
    if (splits > 1) {
      const size_t need = tsb_tree_attn_workspace_bytes(B, T, Hq, Hkv, D, n_kv, kv_format);
      if (!ws || ws_bytes < need) return TSB_EWORKSPACE;
      if (!aligned(ws, 16)) return TSB_EINVAL;
      part_o = (float *)ws;
      part_ml = part_o + (size_t)splits * rows * AT_D;
    }
    int r = launch_attn_tc(kv_format, (const uint16_t *)q, k, k_scales, k_biases, v, v_scales, v_biases, parents,
                           (const unsigned long long *)bits, B, T, Hq, Hkv, n_kv, tail, kv_capacity, scale,
                           (uint16_t *)out, lse, part_o, part_ml, st);
    if (r != TSB_OK) return r;
    if (splits > 1) {
      launch_combine(part_o, part_ml, splits, (int)rows, out, lse, st);
      if (cudaGetLastError() != cudaSuccess) return TSB_ECUDA;
    }
    return TSB_OK;
  }
  const AttnPlan p = plan_attn(B, T, Hq, Hkv, n_kv);
  AttnArgs a;
  a.q = (const uint16_t *)q;
  a.k = k; a.ks = k_scales; a.kb = k_biases;
  a.v = v; a.vs = v_scales; a.vb = v_biases;
  a.parents = parents;
  a.bits = (const unsigned long long *)bits;
  a.B = B; a.T = T; a.Hq = Hq; a.Hkv = Hkv; a.n_kv = n_kv; a.tail = tail; a.cap = kv_capacity;
  a.rows_per_cta = p.rows_per_cta;
  a.row_blocks = p.row_blocks;
  a.splits = p.splits;
  a.tiles_per_split = p.tiles_per_split;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.out = (uint16_t *)out;
  a.lse = lse;
  a.part_o = nullptr;
  a.part_ml = nullptr;
  if (p.splits > 1) {
    const size_t need = tsb_tree_attn_workspace_bytes(B, T, Hq, Hkv, D, n_kv, kv_format);
    if (!ws || ws_bytes < need) return TSB_EWORKSPACE;
    if (!aligned(ws, 16)) return TSB_EINVAL;
    a.part_o = (float *)ws;
    a.part_ml = a.part_o + (size_t)p.splits * rows * AT_D;
  }
  const size_t smem = attn_smem_bytes();
  const dim3 grid(B * Hkv * p.row_blocks, p.splits);
  const dim3 block(p.rows_per_cta * 2);  // 32 threads per 16 rows
  cudaError_t e;
  switch (kv_format) {
    case TSB_KV_BF16:
      e = cudaFuncSetAttribute(tree_attn_kernel<TSB_KV_BF16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return TSB_ECUDA;
      tree_attn_kernel<TSB_KV_BF16><<<grid, block, smem, st>>>(a);
      break;
    case TSB_KV_MLX_Q8_G64:
      e = cudaFuncSetAttribute(tree_attn_kernel<TSB_KV_MLX_Q8_G64>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return TSB_ECUDA;
      tree_attn_kernel<TSB_KV_MLX_Q8_G64><<<grid, block, smem, st>>>(a);
      break;
    default:
      e = cudaFuncSetAttribute(tree_attn_kernel<TSB_KV_REF_Q8_ROW>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return TSB_ECUDA;
      tree_attn_kernel<TSB_KV_REF_Q8_ROW><<<grid, block, smem, st>>>(a);
      break;
  }
  if (cudaGetLastError() != cudaSuccess) return TSB_ECUDA;
  if (p.splits > 1) {
    launch_combine(a.part_o, a.part_ml, p.splits, (int)rows, out, lse, st);
    if (cudaGetLastError() != cudaSuccess) return TSB_ECUDA;
  }
  return TSB_OK;
}

// ---------------------------------------------------------------------------
// Allocation-free variant of tsb_tree_attn.
//
// Some callers cannot hand this library a workspace: a host whose device
// memory is owned by a pool allocator it cannot call into from the decode
// loop, a language binding (cgo, JNI, N-API) that has no device allocator of
// its own, or a serving loop that forbids any allocation once it is running.
// For them the split-KV partials live in a fixed array in the library's own
// device memory, reserved when the library is loaded on a device and held
// until the process exits (kAttnScratchBytes = 16 MiB per GPU). The first call
// on each device looks up that array's device address; make that first call
// before capturing a stream into a graph.
//
// The array is shared by every call on a device and keeps the last call's
// contents. Nothing in it must start at zero: each call's first kernel writes
// every partial that its combine kernel then reads. Calls whose GPU work can
// overlap (different streams, or graphs launched concurrently) race on it and
// must be serialized by the caller.
namespace tsb {
namespace {

constexpr size_t kAttnScratchBytes = 16u << 20;  // 16 MiB per device
static __device__ __align__(256) unsigned char g_attn_scratch[kAttnScratchBytes];

// Device address of g_attn_scratch on the current device. The host-side name
// of a __device__ array is only a stand-in, never a device address, so it is
// looked up once per device with cudaGetSymbolAddress (with that device
// current) and cached. nullptr if the lookup fails.
void *attn_scratch_ptr() {
  static std::mutex mu;
  static void *ptrs[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (!ptrs[dev]) {
    void *p = nullptr;
    if (cudaGetSymbolAddress(&p, g_attn_scratch) != cudaSuccess) return nullptr;
    ptrs[dev] = p;
  }
  return ptrs[dev];
}

}  // namespace
}  // namespace tsb

extern "C" int tsb_tree_attn_noalloc(const void *q, const void *k, const void *k_scales, const void *k_biases,
                                     const void *v, const void *v_scales, const void *v_biases, int kv_format,
                                     const int32_t *parents, const uint64_t *bits, int B, int T, int Hq, int Hkv,
                                     int D, int n_kv, int tail, int kv_capacity, float scale, void *out, float *lse,
                                     tsb_stream_t stream) {
  if (B <= 0 || T <= 0 || Hq <= 0 || Hkv <= 0 || n_kv <= 0) return TSB_EINVAL;
  const size_t need = tsb_tree_attn_workspace_bytes(B, T, Hq, Hkv, D, n_kv, kv_format);
  if (need > tsb::kAttnScratchBytes) return TSB_EWORKSPACE;  // beyond the fixed scratch: use tsb_tree_attn
  void *scratch = tsb::attn_scratch_ptr();
  if (!scratch) return TSB_ECUDA;
  return tsb_tree_attn(q, k, k_scales, k_biases, v, v_scales, v_biases, kv_format, parents, bits, B, T, Hq, Hkv, D,
                       n_kv, tail, kv_capacity, scale, out, lse, scratch, tsb::kAttnScratchBytes, stream);
}
