// Library identity and status text.
#include "common.cuh"

extern "C" int srswa_version(void) { return 100; }  // 0.1.0

extern "C" const char* srswa_status_string(int status) {
  switch (status) {
    case SRSWA_OK: return "ok";
    case SRSWA_EINVAL: return "invalid argument";
    case SRSWA_EUNSUPPORTED: return "unsupported shape or dtype";
    case SRSWA_EALIGN: return "pointer or stride not 16-byte aligned";
    case SRSWA_EWORKSPACE: return "workspace too small";
    case SRSWA_ETOOLARGE: return "size above a compiled-in maximum";
    default: break;
  }
  if (status > 0) return cudaGetErrorString(static_cast<cudaError_t>(status));
  return "unknown status";
}
