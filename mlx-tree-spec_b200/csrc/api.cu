// Library-wide entry points: status strings, version, device status, and the
// host-side helpers shared by the kernels (SM count, TMA tensor maps).
#include "sm100.cuh"

namespace tsb {

int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (dev < 0 || dev >= 64) return 148;
  if (!cached[dev]) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

int make_tmap_2d(CUtensorMap *map, const void *base, CUtensorMapDataType dtype, int elem_bytes, uint64_t cols,
                 uint64_t rows, uint64_t row_pitch_bytes, uint32_t box_cols, uint32_t box_rows,
                 CUtensorMapSwizzle swizzle) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return TSB_ECUDA;
  (void)elem_bytes;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {row_pitch_bytes};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dtype, 2, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? TSB_OK : TSB_ECUDA;
}

unsigned int status_gemm(bool reset);
unsigned int status_ts(bool reset);
unsigned int status_attn_tc(bool reset);

}  // namespace tsb

// Synchronizes `stream`, then reports the first device-side failure recorded
// by any kernel since the last reset (TSB_OK if none): a bounded wait that ran
// out (TSB_ETIMEOUT). reset != 0 clears the record.
extern "C" int tsb_device_status(tsb_stream_t stream, int reset) {
  if (cudaStreamSynchronize((cudaStream_t)stream) != cudaSuccess) return TSB_ECUDA;
  const unsigned int a = tsb::status_gemm(reset != 0);
  const unsigned int b = tsb::status_ts(reset != 0);
  const unsigned int c = tsb::status_attn_tc(reset != 0);
  return (int)(a ? a : (b ? b : c));
}

extern "C" const char *tsb_strerror(int status) {
  switch (status) {
    case TSB_OK: return "ok";
    case TSB_EUNSUPPORTED: return "unsupported shape or format (declined; caller falls back)";
    case TSB_EINVAL: return "invalid argument (null/misaligned pointer or inconsistent sizes)";
    case TSB_ECUDA: return "CUDA runtime or launch error";
    case TSB_ETIMEOUT: return "bounded device-side wait timed out";
    case TSB_EWORKSPACE: return "workspace too small";
    default: return "unknown status";
  }
}

extern "C" int tsb_version(void) { return (0 << 16) | (1 << 8) | 0; }
