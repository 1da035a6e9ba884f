// Shared device helpers for libqmtp (sm_100a only).
//
// Arithmetic rule for every kernel in this library: the fp32 operation sequence is fixed and
// written with explicit round-to-nearest intrinsics (__fmaf_rn, __fadd_rn, __fmul_rn, __fdiv_rn,
// __fsqrt_rn); the library is also built with -fmad=false so nothing is contracted behind our
// back.  The CPU oracle (oracle/qmtp_oracle.c) states the same sequences, so kernel results are
// bit-identical to it.  exp/log below are this library's own (Cody-Waite reduction, Taylor /
// atanh series), not CUDA's math library, for the same reason.
#pragma once
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/qmtp.h"

namespace qmtp {

// ----------------------------------------------------------------------------- launches
// Every kernel of the library is launched with programmatic stream serialisation (PDL): the next
// kernel in the stream may start while the previous one finishes.  Each kernel therefore calls
// pdl_wait() before it touches any memory an earlier kernel writes or reads (constant weights are
// the only exception: the qmv kernel prefetches them before the wait), and pdl_trigger() early so
// its own successor can start its prologue.  Calling pdl_wait() in every kernel keeps the chain
// transitive (a kernel finishing implies all earlier kernels finished).  QMTP_PDL=0 disables it.
// The 4-bit GEMV kernels trigger only after their own wait: a kernel launched behind one of them
// may start before it finishes, but never before the launch two back has finished, so data written
// two or more launches back may be read before the wait (qmtp_gdn_args.preload).
bool pdl_enabled();

template <typename... KArgs, typename... Args>
inline cudaError_t launch_kernel(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                                 Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// launch_kernel with a 1-D thread-block cluster of `cluster` CTAs (no cluster attribute when 1).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_kernel_cluster(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                                         int cluster, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = unsigned(cluster);
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = cluster > 1 ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

// ----------------------------------------------------------------------------- clusters
// Every thread of every CTA of the cluster arrives (release) and waits (acquire): the shared-memory
// stores of each CTA before it are visible to the others' distributed-shared-memory loads after it.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// L2 prefetch of `bytes` (a multiple of 16) at the 16-byte aligned address p.  A hint: no data
// comes back and no ordering is implied, and L2 is where every kernel's stores land, so it is safe
// before the dependency wait even for lines an earlier kernel is still writing.
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// 16-byte asynchronous global -> shared copy (both addresses 16-byte aligned), bypassing L1, and its
// group commit / wait: the thread's copies are in shared memory after cp_async_wait_all (other threads
// see them after a barrier).
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
  const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// The two halves of cluster_sync_all, for a barrier whose wait is deferred (e.g. "my peers may
// still read my shared memory": arrive after the last remote read, wait before exiting).
__device__ __forceinline__ void cluster_arrive_release() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_acquire() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// The float at the same shared-memory offset as `local` in CTA `rank` of this cluster.
__device__ __forceinline__ float ld_dsmem(const float* local, uint32_t rank) {
  uint32_t la = static_cast<uint32_t>(__cvta_generic_to_shared(local)), ra;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(la), "r"(rank));
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(ra) : "memory");
  return v;
}
// 16 aligned bytes at the same shared-memory offset as `local` in CTA `rank` of this cluster.
__device__ __forceinline__ float4 ld_dsmem_v4(const float* local, uint32_t rank) {
  uint32_t la = static_cast<uint32_t>(__cvta_generic_to_shared(local)), ra;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(la), "r"(rank));
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(ra)
               : "memory");
  return v;
}

// ----------------------------------------------------------------------------- errors
enum : unsigned { DEVERR_TIMEOUT = 1u, DEVERR_BADARG = 2u };
unsigned* device_error_ptr();  // per-device address of the library's device error word
// Device address of a __device__ symbol in the current context (cached per context; QMTP_ERR_CUDA if
// the lookup fails, which is not cached).
int symbol_address(const void* symbol, void** out);
int sm_count();                 // SMs of the current device (cached)
// cuTensorMapEncodeTiled from the driver (resolved once through the runtime; nullptr if unavailable).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();

#define QMTP_CUDA_TRY(expr)                          \
  do {                                               \
    cudaError_t e__ = (expr);                        \
    if (e__ != cudaSuccess) return QMTP_ERR_CUDA;    \
  } while (0)

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ----------------------------------------------------------------------------- bf16 bits
__device__ __forceinline__ float bf2f(uint16_t h) { return __uint_as_float(uint32_t(h) << 16); }
__device__ __forceinline__ float bflo(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float bfhi(uint32_t u) { return __uint_as_float(u & 0xFFFF0000u); }
// fp32 -> bf16 round-to-nearest-even; NaN -> 0x7FC0 (same rule as the oracle).
__device__ __forceinline__ uint16_t f2bf(float f) {
  uint32_t u = __float_as_uint(f);
  if ((u & 0x7FFFFFFFu) > 0x7F800000u) return 0x7FC0;
  u += 0x7FFFu + ((u >> 16) & 1u);
  return uint16_t(u >> 16);
}
__device__ __forceinline__ float R(float x) { return bf2f(f2bf(x)); }

// ----------------------------------------------------------------------------- exp / log
__device__ __forceinline__ float q_expf(float x) {
  if (x != x) return x;
  if (x > 88.72283935546875f) return __int_as_float(0x7F800000);
  if (x < -103.972084045410156f) return 0.0f;
  const float kf = rintf(__fmul_rn(x, 1.44269502162933349609375f));
  float r = __fmaf_rn(-kf, 0.693145751953125f, x);
  r = __fmaf_rn(-kf, 1.428606765330187045e-06f, r);
  float p = 1.98412701138295233249664e-04f;
  p = __fmaf_rn(p, r, 1.38888892251998186111450e-03f);
  p = __fmaf_rn(p, r, 8.33333376795053482055664e-03f);
  p = __fmaf_rn(p, r, 4.16666679084300994873047e-02f);
  p = __fmaf_rn(p, r, 1.66666671633720397949219e-01f);
  p = __fmaf_rn(p, r, 0.5f);
  p = __fmaf_rn(p, r, 1.0f);
  p = __fmaf_rn(p, r, 1.0f);
  const int k = int(kf);
  const int k1 = k / 2, k2 = k - k1;
  const float s1 = __uint_as_float(uint32_t(k1 + 127) << 23);
  const float s2 = __uint_as_float(uint32_t(k2 + 127) << 23);
  return __fmul_rn(__fmul_rn(p, s1), s2);
}

__device__ __forceinline__ float q_logf(float x) {
  if (x != x) return x;
  if (x < 0.0f) return __int_as_float(0x7FC00000);
  if (x == 0.0f) return __int_as_float(0xFF800000);
  if (x == __int_as_float(0x7F800000)) return x;
  int e = 0;
  uint32_t ix = __float_as_uint(x);
  if (ix < 0x00800000u) { x = __fmul_rn(x, 8388608.0f); ix = __float_as_uint(x); e = -23; }
  e += int(ix >> 23) - 127;
  float m = __uint_as_float((ix & 0x007FFFFFu) | 0x3F800000u);
  if (m > 1.41421353816986083984375f) { m = __fmul_rn(m, 0.5f); e += 1; }
  const float f = __fsub_rn(m, 1.0f);
  const float s = __fdiv_rn(f, __fadd_rn(2.0f, f));
  const float z = __fmul_rn(s, s);
  float p = 2.22222223877906799316406e-01f;
  p = __fmaf_rn(p, z, 2.85714298486709594726562e-01f);
  p = __fmaf_rn(p, z, 4.00000005960464477539062e-01f);
  p = __fmaf_rn(p, z, 6.66666686534881591796875e-01f);
  const float lm = __fmaf_rn(__fmul_rn(s, z), p, __fmul_rn(2.0f, s));
  const float ef = float(e);
  return __fmaf_rn(ef, 0.693145751953125f, __fmaf_rn(ef, 1.428606765330187045e-06f, lm));
}

// bf16 activation formulas of gdn_fused.py:22-41 (round after every op).
__device__ __forceinline__ float sigmoid_bf(float x) {
  const float y = R(__fdiv_rn(1.0f, R(__fadd_rn(1.0f, R(q_expf(fabsf(x)))))));
  return x < 0.0f ? y : R(__fsub_rn(1.0f, y));
}
__device__ __forceinline__ float silu_bf(float x) { return R(__fmul_rn(x, sigmoid_bf(x))); }
__device__ __forceinline__ float log1p_bf(float x) {
  const float xp1 = __fadd_rn(1.0f, x);
  if (xp1 == 1.0f) return x;
  const float t = __fdiv_rn(q_logf(xp1), __fsub_rn(xp1, 1.0f));
  return R(__fmul_rn(x, t));
}
__device__ __forceinline__ float softplus_bf(float x) {
  const float hi = x > 0.0f ? x : 0.0f, lo = x < 0.0f ? x : 0.0f;
  return R(__fadd_rn(hi, log1p_bf(R(q_expf(R(__fsub_rn(lo, hi)))))));
}
__device__ __forceinline__ float silu_f32(float x) {
  const float y = __fdiv_rn(1.0f, __fadd_rn(1.0f, q_expf(fabsf(x))));
  return __fmul_rn(x, x < 0.0f ? y : __fsub_rn(1.0f, y));
}
__device__ __forceinline__ float sigmoid_f32(float x) {
  const float y = __fdiv_rn(1.0f, __fadd_rn(1.0f, q_expf(fabsf(x))));
  return x < 0.0f ? y : __fsub_rn(1.0f, y);
}
// 1/sqrt(v) from two correctly rounded ops (identical to the oracle's 1.0f / sqrtf(v)).
__device__ __forceinline__ float rsqrt_rn(float v) { return __fdiv_rn(1.0f, __fsqrt_rn(v)); }

// ----------------------------------------------------------------------------- warp sums
// 32-lane xor butterfly (strides 16..1): every lane ends with the same bits.
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int d = 16; d >= 1; d >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xFFFFFFFFu, v, d));
  return v;
}

// Recursive-halving reduce-scatter of VP values (VP a power of two <= 32) across the warp.  For
// every value the additions form exactly the xor butterfly tree of warp_sum (fp add commutes), so
// the result is bit-identical to warp_sum applied value by value.  On return, v[0] holds value
// `idx`; `owner` is true for one lane per value.
template <int VP>
__device__ __forceinline__ void warp_reduce_scatter(float (&v)[VP], int lane, int& idx, bool& owner) {
  int n = VP;
  idx = 0;
  int rem_mask = 0;
#pragma unroll
  for (int d = 16; d >= 1; d >>= 1) {
    if (n > 1) {
      const int half = n >> 1;
      const bool up = (lane & d) != 0;
#pragma unroll
      for (int i = 0; i < VP / 2; ++i) {
        if (i < half) {
          const float send = up ? v[i] : v[i + half];
          const float keep = up ? v[i + half] : v[i];
          v[i] = __fadd_rn(keep, __shfl_xor_sync(0xFFFFFFFFu, send, d));
        }
      }
      if (up) idx += half;
      n = half;
    } else {
      v[0] = __fadd_rn(v[0], __shfl_xor_sync(0xFFFFFFFFu, v[0], d));
      rem_mask |= d;
    }
  }
  owner = (lane & rem_mask) == 0;
}

// Block-wide exclusive prefix sum of one int per thread (blockDim.x <= 1024, multiple of 32).
__device__ __forceinline__ int block_excl_scan(int v, int* s_warp, int& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  int x = v;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int o = __shfl_up_sync(0xFFFFFFFFu, x, d);
    if (lane >= d) x += o;
  }
  if (lane == 31) s_warp[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = lane < nw ? s_warp[lane] : 0;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int o = __shfl_up_sync(0xFFFFFFFFu, w, d);
      if (lane >= d) w += o;
    }
    if (lane < nw) s_warp[lane] = w;  // inclusive per warp
  }
  __syncthreads();
  total = s_warp[nw - 1];
  const int base = warp > 0 ? s_warp[warp - 1] : 0;
  __syncthreads();
  return base + x - v;
}

// ----------------------------------------------------------------------------- TMA / mbarrier
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
// 1-D bulk copy global -> shared, completion counted on `bar`.  dst/src 16-B aligned, bytes % 16 == 0.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                         uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: gives up after `limit` polls, records DEVERR_TIMEOUT and returns false.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, unsigned* err,
                                                  uint32_t limit = (1u << 24)) {
#pragma unroll 1  // a wait loop: unrolling only grows the code
  for (uint32_t it = 0; it < limit; ++it)
    if (mbar_try_wait(bar, parity)) return true;
  if (err) atomicOr(err, DEVERR_TIMEOUT);
  return false;
}

// try_wait with a suspend-time hint: the thread sleeps until the phase completes or about `ns`
// nanoseconds pass, so a waiting warp takes no issue slots from the warps doing the work.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(ns)
      : "memory");
  return ok != 0;
}
// Bounded sleeping wait: at most `limit` polls of up to 1 us each; on timeout records DEVERR_TIMEOUT.
__device__ __forceinline__ bool mbar_wait_sleep(uint64_t* bar, uint32_t parity, unsigned* err,
                                                uint32_t limit = (1u << 20)) {
#pragma unroll 1  // a wait loop: unrolling only grows the code
  for (uint32_t it = 0; it < limit; ++it)
    if (mbar_try_wait_sleep(bar, parity, 1000u)) return true;
  if (err) atomicOr(err, DEVERR_TIMEOUT);
  return false;
}

// Bounded wait with back-off: a failed poll puts the thread to sleep for about `ns` nanoseconds, so
// warps that run ahead of the critical one take no issue slots while they wait.
__device__ __forceinline__ bool mbar_wait_backoff(uint64_t* bar, uint32_t parity, unsigned* err, uint32_t ns,
                                                  uint32_t limit = (1u << 22)) {
#pragma unroll 1  // a wait loop: unrolling only grows the code
  for (uint32_t it = 0; it < limit; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    __nanosleep(ns);
  }
  if (err) atomicOr(err, DEVERR_TIMEOUT);
  return false;
}
// Bounded tight wait for the thread on the critical path (no sleep between polls).
__device__ __forceinline__ bool mbar_wait_spin(uint64_t* bar, uint32_t parity, unsigned* err,
                                               uint32_t limit = (1u << 26)) {
#pragma unroll 1  // a wait loop: unrolling only grows the code
  for (uint32_t it = 0; it < limit; ++it)
    if (mbar_try_wait(bar, parity)) return true;
  if (err) atomicOr(err, DEVERR_TIMEOUT);
  return false;
}

// ----------------------------------------------------------------------------- loads
__device__ __forceinline__ uint4 ldg_nc_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

}  // namespace qmtp

namespace qmtp {
// ----------------------------------------------------------------------------- tcgen05 (5th-gen tensor core)
// Shared-memory operand descriptor for the canonical SWIZZLE_NONE K-major layout: the tile is made of
// core matrices of 8 rows x 16 bytes (128 contiguous bytes); `lbo` is the byte distance between
// core matrices adjacent along K, `sbo` between core matrices adjacent along M (or N).
__device__ __forceinline__ uint64_t umma_desc(uint32_t smem_addr, uint32_t lbo, uint32_t sbo) {
  return uint64_t((smem_addr >> 4) & 0x3FFFu) | (uint64_t((lbo >> 4) & 0x3FFFu) << 16) |
         (uint64_t((sbo >> 4) & 0x3FFFu) << 32) | (uint64_t(1) << 46);
}
// Instruction descriptor, kind::f16 with bf16 A/B, fp32 accumulator, both operands K-major.
__host__ __device__ constexpr uint32_t umma_idesc_bf16(int M, int N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(N >> 3) << 17) | (uint32_t(M >> 4) << 24);
}
// Instruction descriptor, kind::f16 with f16 A/B, fp32 accumulator, both operands K-major.
__host__ __device__ constexpr uint32_t umma_idesc_f16(int M, int N) {
  return (1u << 4) | (uint32_t(N >> 3) << 17) | (uint32_t(M >> 4) << 24);
}
// Byte offset of element (r, k) in a [R x Kt] bf16 tile stored as SWIZZLE_NONE K-major core matrices,
// core matrices ordered K-chunk-major: (k/8) * (R/8) + r/8.  Then lbo = (R/8)*128, sbo = 128.
__host__ __device__ constexpr uint32_t cm_offset(int r, int k, int R) {
  return uint32_t(((k >> 3) * (R >> 3) + (r >> 3)) * 128 + (r & 7) * 16 + (k & 7) * 2);
}
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_dst)), "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// 32 lanes x 32 columns of fp32 accumulators: thread (warp w, lane l) gets row 32w + l.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
        "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
        "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
}  // namespace qmtp

namespace qmtp {
// D (TMEM) += A (TMEM, 128 lanes = rows, 32-bit columns = bf16 pairs, even k in the low half) x B (smem descriptor)
__device__ __forceinline__ void umma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// 2-D tiled TMA load (no multicast): box at element coordinates (x inner, y outer); x * elem size % 16 == 0.
__device__ __forceinline__ void tma_load_2d(void* dst, const void* tmap, int x, int y, uint64_t* bar,
                                            uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
      "l"(tmap), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}
__device__ __forceinline__ uint32_t mul_bf16x2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
}  // namespace qmtp
