// Bit-exact 4-bit dequantization and tree ancestor masks.
//
// tsb_dequant_w4g64 follows the reference's dequant arithmetic
// `T(float((p >> (ki * 4)) & 0xF) * s + b)` (mlx-tree-spec
// src/mlx_tree_spec/qmm_packed.py:200,348,635) with the rounding fixed as
// bf16_rne(fmaf(q, s, b)).
// tsb_tree_ancestor_bits follows Tree.__init__ (tree_verify.py:66-121) and
// ancestor_bits (tree_flash.py:146-148), extended to forests.
// tsb_tree_mask_bits inverts Tree.mask (tree_verify.py:131-139): an SDPA mask
// whose columns before the tree rows are all visible becomes per-row bits.
#include "common.cuh"

namespace tsb {

// One thread per 4 words (32 elements of one row, inside one 64-group).
// HBM-bound: 16 B of codes in, 64 B of bf16 out per thread.
__global__ void __launch_bounds__(256) dequant_w4g64_kernel(const uint32_t *__restrict__ w,
                                                            const uint16_t *__restrict__ scales,
                                                            const uint16_t *__restrict__ biases,
                                                            uint16_t *__restrict__ out, long long n_quads,
                                                            int kw) {
  const int G = kw / 8;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n_quads;
       i += (long long)gridDim.x * blockDim.x) {
    const long long word0 = i * 4;
    const long long row = word0 / kw;
    const int c = int(word0 - row * kw);
    const int g = c / 8;
    const float s = bf16_bits_to_float(scales[row * G + g]);
    const float b = bf16_bits_to_float(biases[row * G + g]);
    const uint4 q4 = *reinterpret_cast<const uint4 *>(w + word0);
    const uint32_t qs[4] = {q4.x, q4.y, q4.z, q4.w};
    uint4 *dst = reinterpret_cast<uint4 *>(out + word0 * 8);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint32_t o[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float lo = __fmaf_rn(float((qs[j] >> (8 * e)) & 0xFu), s, b);
        const float hi = __fmaf_rn(float((qs[j] >> (8 * e + 4)) & 0xFu), s, b);
        o[e] = uint32_t(float_to_bf16_bits(lo)) | (uint32_t(float_to_bf16_bits(hi)) << 16);
      }
      dst[j] = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

// One thread per (request, node): walk to the root, setting one bit per node
// on the path. A parent that is neither -1 nor an earlier node stops the walk
// and marks the node invalid (bits 0, depth -1).
__global__ void ancestor_bits_kernel(const int32_t *__restrict__ parents, int B, int T,
                                     unsigned long long *__restrict__ bits, int32_t *__restrict__ depth) {
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= B * T) return;
  const int b = idx / T, i = idx % T;
  const int32_t *p = parents + (size_t)b * T;
  unsigned long long m = 0;
  int d = -1, j = i;
  bool ok = true;
  for (int steps = 0; steps <= T && j != -1; ++steps) {
    m |= 1ull << j;
    ++d;
    const int pj = p[j];
    if (!(pj == -1 || (pj >= 0 && pj < j))) {
      ok = false;
      break;
    }
    j = pj;
  }
  bits[idx] = ok ? m : 0ull;
  if (depth) depth[idx] = ok ? d : -1;
}

// Visibility of mask element c of a row: 1 visible, 0 hidden, -1 neither
// (an additive value other than +-0 and -inf).
__device__ __forceinline__ int mask_class(const unsigned char *row, int dt, long long c) {
  switch (dt) {
    case TSB_MASK_BOOL:
      return row[c] != 0;
    case TSB_MASK_BF16:
    case TSB_MASK_F16: {
      const uint16_t v = reinterpret_cast<const uint16_t *>(row)[c];
      if ((v & 0x7FFFu) == 0) return 1;
      return v == (dt == TSB_MASK_BF16 ? 0xFF80u : 0xFC00u) ? 0 : -1;
    }
    default: {
      const uint32_t v = reinterpret_cast<const uint32_t *>(row)[c];
      if ((v & 0x7FFFFFFFu) == 0) return 1;
      return v == 0xFF800000u ? 0 : -1;
    }
  }
}

// One CTA per mask row, threads striding over the columns (coalesced): the
// columns before the last `tail` must be visible, the tail columns give the
// row's bits. `bad` was zeroed on the stream before the launch.
__global__ void __launch_bounds__(256) mask_bits_kernel(const unsigned char *__restrict__ mask, int dt, int esize,
                                                        long long L, long long row_stride, int tail,
                                                        unsigned long long *__restrict__ bits,
                                                        int32_t *__restrict__ bad) {
  __shared__ unsigned long long s_bits;
  __shared__ int s_bad;
  if (threadIdx.x == 0) {
    s_bits = 0ull;
    s_bad = 0;
  }
  __syncthreads();
  const unsigned char *row = mask + (size_t)blockIdx.x * (size_t)row_stride * esize;
  const long long lo = L - tail;
  unsigned long long m = 0ull;
  int b = 0;
  for (long long c = threadIdx.x; c < L; c += blockDim.x) {
    const int k = mask_class(row, dt, c);
    if (k < 0 || (k == 0 && c < lo)) b = 1;
    else if (k == 1 && c >= lo) m |= 1ull << (c - lo);
  }
  if (m) atomicOr(&s_bits, m);
  if (b) atomicOr(&s_bad, 1);
  __syncthreads();
  if (threadIdx.x == 0) {
    bits[blockIdx.x] = s_bits;
    if (s_bad) atomicAdd(bad, 1);
  }
}

}  // namespace tsb

using namespace tsb;

extern "C" int tsb_dequant_w4g64(const uint32_t *w, const void *scales, const void *biases, void *out,
                                 int N, int K, tsb_stream_t stream) {
  if (!w || !scales || !biases || !out) return TSB_EINVAL;
  if (N <= 0 || K <= 0 || K % 64) return TSB_EINVAL;
  if (!aligned(w, 16) || !aligned(out, 16)) return TSB_EINVAL;
  const long long n_quads = (long long)N * (K / 8) / 4;
  const int threads = 256;
  long long blocks = (n_quads + threads - 1) / threads;
  const long long cap = (long long)sm_count() * 16;
  if (blocks > cap) blocks = cap;
  dequant_w4g64_kernel<<<(unsigned)blocks, threads, 0, (cudaStream_t)stream>>>(
      w, (const uint16_t *)scales, (const uint16_t *)biases, (uint16_t *)out, n_quads, K / 8);
  return launch_status();
}

extern "C" int tsb_tree_ancestor_bits(const int32_t *parents, int B, int T, uint64_t *bits, int32_t *depth,
                                      tsb_stream_t stream) {
  if (!parents || !bits) return TSB_EINVAL;
  if (B <= 0 || T <= 0) return TSB_EINVAL;
  if (T > 64) return TSB_EUNSUPPORTED;
  const int n = B * T;
  ancestor_bits_kernel<<<(n + 127) / 128, 128, 0, (cudaStream_t)stream>>>(parents, B, T,
                                                                          (unsigned long long *)bits, depth);
  return launch_status();
}

extern "C" int tsb_tree_mask_bits(const void *mask, int mask_dtype, int rows, long long L, long long row_stride,
                                  int tail, uint64_t *bits, int32_t *bad, tsb_stream_t stream) {
  if (!mask || !bits || !bad) return TSB_EINVAL;
  int esize = 0;
  switch (mask_dtype) {
    case TSB_MASK_BOOL: esize = 1; break;
    case TSB_MASK_BF16:
    case TSB_MASK_F16: esize = 2; break;
    case TSB_MASK_F32: esize = 4; break;
    default: return TSB_EINVAL;
  }
  if (rows <= 0 || L <= 0 || row_stride < L || tail < 0 || tail > L) return TSB_EINVAL;
  if (!aligned(mask, esize)) return TSB_EINVAL;
  if (tail > 64) return TSB_EUNSUPPORTED;
  const cudaStream_t st = (cudaStream_t)stream;
  if (cudaMemsetAsync(bad, 0, sizeof(int32_t), st) != cudaSuccess) return TSB_ECUDA;
  mask_bits_kernel<<<rows, 256, 0, st>>>(static_cast<const unsigned char *>(mask), mask_dtype, esize, L, row_stride,
                                         tail, (unsigned long long *)bits, bad);
  return launch_status();
}
