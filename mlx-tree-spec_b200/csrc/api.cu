// Library-wide entry points: status strings, version, device facts.
#include "common.cuh"

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

}  // namespace tsb

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
