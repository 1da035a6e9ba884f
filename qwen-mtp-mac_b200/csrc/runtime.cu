// Library-wide runtime pieces: error text, version, the device error word, device properties.
#include <cstdlib>
#include <mutex>

#include "common.cuh"

namespace qmtp {

// One word per device that loads the library; kernels OR DEVERR_* bits into it.
static __device__ unsigned g_device_error;

static constexpr int kMaxDevices = 64;

unsigned* device_error_ptr() {
  static std::once_flag once[kMaxDevices];
  static unsigned* ptr[kMaxDevices];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::call_once(once[dev], [&] {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_error) == cudaSuccess) ptr[dev] = static_cast<unsigned*>(p);
  });
  return ptr[dev];
}

int sm_count() {
  static std::once_flag once[kMaxDevices];
  static int count[kMaxDevices];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 1;
  std::call_once(once[dev], [&] {
    int c = 0;
    cudaDeviceGetAttribute(&c, cudaDevAttrMultiProcessorCount, dev);
    count[dev] = c > 0 ? c : 1;
  });
  return count[dev];
}

bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("QMTP_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

}  // namespace qmtp

extern "C" const char* qmtp_strerror(int code) {
  switch (code) {
    case QMTP_OK: return "ok";
    case QMTP_ERR_SHAPE: return "unsupported or inconsistent sizes";
    case QMTP_ERR_ALIGN: return "pointer not 16-byte aligned";
    case QMTP_ERR_UNSUPPORTED: return "unsupported request";
    case QMTP_ERR_CUDA: return "CUDA launch or runtime error";
    case QMTP_ERR_ARG: return "invalid argument";
    default: return "unknown qmtp error";
  }
}

extern "C" int qmtp_version(void) { return 100; }

extern "C" int qmtp_device_error(unsigned* out, int clear) {
  if (!out) return QMTP_ERR_ARG;
  unsigned v = 0;
  if (cudaMemcpyFromSymbol(&v, qmtp::g_device_error, sizeof v) != cudaSuccess) return QMTP_ERR_CUDA;
  *out = v;
  if (clear) {
    const unsigned z = 0;
    if (cudaMemcpyToSymbol(qmtp::g_device_error, &z, sizeof z) != cudaSuccess) return QMTP_ERR_CUDA;
  }
  return QMTP_OK;
}
