// Diagnostics of the library's own device building blocks, for its test suite:
//   * qmtp_math_eval evaluates the device exp / log and the bf16 activation formulas of
//     gdn_fused.py:22-41 (common.cuh) over caller-given inputs, so the tests can compare them with the
//     oracle on every bf16 value;
//   * qmtp_wait_selftest runs one bounded mbarrier wait that nothing completes, so the tests can see
//     the wait give up after its limit and record DEVERR_TIMEOUT in the device error word (no fault,
//     no hang: the wait is bounded and the kernel returns).
#include "common.cuh"

namespace qmtp {

__global__ void math_eval_kernel(int fn, const uint16_t* __restrict__ x, int n, float* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float v = bf2f(x[i]);
  float r;
  switch (fn) {
    case QMTP_MATH_EXP: r = q_expf(v); break;
    case QMTP_MATH_LOG: r = q_logf(v); break;
    case QMTP_MATH_SIGMOID_BF: r = sigmoid_bf(v); break;
    case QMTP_MATH_SILU_BF: r = silu_bf(v); break;
    case QMTP_MATH_SOFTPLUS_BF: r = softplus_bf(v); break;
    default: r = silu_f32(v); break;
  }
  out[i] = r;
}

__global__ void wait_selftest_kernel(unsigned limit, unsigned* err, int* result) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    // phase 0 never completes: nobody arrives
    const bool ok = mbar_wait_bounded(&bar, 0, err, limit);
    *result = ok ? 1 : 0;
  }
}

}  // namespace qmtp

using namespace qmtp;

extern "C" int qmtp_math_eval(int fn, const void* x, int n, float* out, void* stream) {
  if (!x || !out) return QMTP_ERR_ARG;
  if (fn < QMTP_MATH_EXP || fn > QMTP_MATH_SILU_F32) return QMTP_ERR_ARG;
  if (n < 1) return QMTP_ERR_SHAPE;
  launch_kernel(math_eval_kernel, dim3((n + 255) / 256), dim3(256), 0, static_cast<cudaStream_t>(stream), fn,
                static_cast<const uint16_t*>(x), n, out);
  return cudaGetLastError() == cudaSuccess ? QMTP_OK : QMTP_ERR_CUDA;
}

extern "C" int qmtp_wait_selftest(unsigned limit, int* result, void* stream) {
  if (!result) return QMTP_ERR_ARG;
  if (limit < 1 || limit > (1u << 20)) return QMTP_ERR_ARG;
  unsigned* err = device_error_ptr();
  if (!err) return QMTP_ERR_CUDA;
  wait_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(limit, err, result);
  return cudaGetLastError() == cudaSuccess ? QMTP_OK : QMTP_ERR_CUDA;
}
