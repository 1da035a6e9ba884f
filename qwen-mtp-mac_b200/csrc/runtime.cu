// Library-wide runtime pieces: error text, version, the device error word, device properties.
#include <cstdlib>
#include <mutex>

#include "common.cuh"

namespace qmtp {

// One word per device that loads the library; kernels OR DEVERR_* bits into it.
static __device__ unsigned g_device_error;

static constexpr int kMaxDevices = 64;

// The CUDA context current on this thread (driver entry point resolved once), or nullptr.
static CUcontext current_context() {
  using Fn = CUresult (*)(CUcontext*);
  static std::once_flag once;
  static Fn fn = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<Fn>(p);
  });
  CUcontext c = nullptr;
  if (!fn || fn(&c) != CUDA_SUCCESS) return nullptr;
  return c;
}

// Device addresses of __device__ symbols, cached per (context, symbol).  Keyed on the context, not
// the device ordinal, so a context created after cudaDeviceReset gets a fresh lookup instead of a
// stale address; failed lookups are not cached, so a call that failed (for example inside a stream
// capture) is retried by the next call.
int symbol_address(const void* symbol, void** out) {
  struct Entry {
    CUcontext ctx;
    const void* sym;
    void* addr;
  };
  static std::mutex mu;
  static Entry table[256];
  static int used = 0;
  CUcontext ctx = current_context();
  if (ctx) {
    std::lock_guard<std::mutex> lock(mu);
    for (int i = 0; i < used; ++i)
      if (table[i].ctx == ctx && table[i].sym == symbol) {
        *out = table[i].addr;
        return QMTP_OK;
      }
  }
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, symbol) != cudaSuccess || !p) {
    cudaGetLastError();  // the failed lookup leaves no sticky error behind
    return QMTP_ERR_CUDA;
  }
  if (!ctx) ctx = current_context();  // the lookup above may have created the primary context
  if (ctx) {
    std::lock_guard<std::mutex> lock(mu);
    if (used < 256) table[used++] = Entry{ctx, symbol, p};
  }
  *out = p;
  return QMTP_OK;
}

unsigned* device_error_ptr() {
  void* p = nullptr;
  return symbol_address(&g_device_error, &p) == QMTP_OK ? static_cast<unsigned*>(p) : nullptr;
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

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
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
