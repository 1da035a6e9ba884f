// Multi-row 4-bit GEMV (qmv) for B200, NVFP4 group-16 (e2m1 nibbles, e4m3 scale per 16).
//
// Replaces qmv_kernel.py:14-101 (qmv_nvfp4_multi), the reference's own qmv format, for 1-4
// activation rows.  (The affine group-64 format runs on the tensor cores, csrc/qmv_tc.cu.)
// Design (HBM-bound streaming of the weights, each byte read once per call):
//   * one CTA per SM-slot, persistent over a contiguous range of output rows;
//   * the CTA's weight / scale rows arrive by 1-D TMA bulk copies (cp.async.bulk) into an NS-stage
//     shared-memory ring, completion tracked by mbarriers (bounded waits);
//   * "x-stationary": warp w, lane l owns K-chunk c = 32w + l (32 elements) for the whole kernel
//     and keeps those x values (all M rows) in registers, so x is read from HBM/L2 once per CTA;
//   * each byte of nibbles becomes two exact values with one hardware e2m1x2 conversion;
//   * the per-chunk partials of TR rows x M columns are reduced across the warp with a
//     reduce-scatter (one shuffle + add per value) and across warps in shared memory.
// The fp32 operation order is the one of oracle/qmtp_oracle.c:qo_qmv_nvfp4.
#include <algorithm>
#include <mutex>

#include "common.cuh"

namespace qmtp {

struct QmvParams {
  const uint16_t* x;
  const uint32_t* wq;
  const uint8_t* sc;
  uint16_t* y;
  const uint16_t* res;
  int N, ldy;
  unsigned* err;
};

template <int M, int W, int TR, int NS>
struct QmvCfg {
  static constexpr int K = W * 1024;
  static constexpr int WB = K / 2;   // weight bytes per row
  static constexpr int SB = K / 16;  // scale bytes per row
  static constexpr int NV = TR * M;
  static constexpr int VP = NV <= 1 ? 1 : NV <= 2 ? 2 : NV <= 4 ? 4 : NV <= 8 ? 8 : NV <= 16 ? 16 : 32;
  static_assert(NV <= 32, "TR*M must be <= 32");
  static constexpr int OFF_S = NS * TR * WB;
  static constexpr int OFF_RED = OFF_S + NS * TR * SB;
  static constexpr int OFF_BAR = OFF_RED + 2 * W * VP * 4;
  static constexpr int SMEM = OFF_BAR + NS * 8;
};

// (lo, hi) float pairs in one 64-bit register pair, for fma.rn.f32x2 (two IEEE fp32 fmas).
__device__ __forceinline__ uint64_t pack2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1,%2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void unpack2(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0,%1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}

// e2m1 nibble pairs -> exact fp32 values, unscaled: the hardware e2m1x2 -> f16x2 conversion of
// each byte (nibble 2b in the low half, 2b+1 in the high half; signed, zero exact), then f16 -> f32.
// p[b] = (nibble 2b, nibble 2b+1) as a (lo, hi) pair for fma.rn.f32x2.
__device__ __forceinline__ void e2m1_pairs(uint32_t w, uint64_t (&p)[4]) {
  uint32_t h[4];
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n\tcvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, b2;\n\tcvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
      : "=r"(h[0]), "=r"(h[1]), "=r"(h[2]), "=r"(h[3])
      : "r"(w));
#pragma unroll
  for (int b = 0; b < 4; ++b)
    p[b] = pack2(__half2float(__ushort_as_half(uint16_t(h[b] & 0xFFFFu))),
                 __half2float(__ushort_as_half(uint16_t(h[b] >> 16))));
}

__device__ __forceinline__ float e4m3_x16k(uint32_t s) {
  // e4m3 value * 2^14 (sign ignored): half bits (s & 0x7f) << 7 is value * 2^-8; times 2^22.
  return __fmul_rn(__half2float(__ushort_as_half(uint16_t((s & 0x7Fu) << 7))), 4194304.0f);
}

template <int M, int W, int TR, int NS>
__global__ void __launch_bounds__(W * 32, 1) qmv_kernel(const __grid_constant__ QmvParams p) {
  using C = QmvCfg<M, W, TR, NS>;
  const uint16_t* __restrict__ x = p.x;
  const uint32_t* __restrict__ wq = p.wq;
  const uint8_t* __restrict__ sc = p.sc;
  uint16_t* __restrict__ y = p.y;
  const uint16_t* __restrict__ res = p.res;
  const int N = p.N, ldy = p.ldy;
  unsigned* __restrict__ err = p.err;
  extern __shared__ __align__(128) unsigned char smem[];
  float* s_red = reinterpret_cast<float*>(smem + C::OFF_RED);
  uint64_t* s_bar = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int c = warp * 32 + lane;  // this thread's K-chunk
  // whole tiles per CTA (only the last tile of the matrix can be partial)
  const int ntot = (N + TR - 1) / TR;
  const int t0 = int((long long)blockIdx.x * ntot / gridDim.x);
  const int t1 = int((long long)(blockIdx.x + 1) * ntot / gridDim.x);
  const int r0 = t0 * TR;
  const int r1 = min(N, t1 * TR);
  const int nrows = max(0, r1 - r0);
  const int ntiles = (nrows + TR - 1) / TR;

  if (tid == 0) {
#pragma unroll
    for (int s = 0; s < NS; ++s) mbar_init(&s_bar[s], 1);
    fence_mbar_init();
  }
  __syncthreads();

  const uint64_t pol = policy_evict_first();
  auto issue = [&](int t) {
    const int s = t % NS;
    const int rows = min(TR, nrows - t * TR);
    const size_t row = size_t(r0) + size_t(t) * TR;
    mbar_expect_tx(&s_bar[s], uint32_t(rows * (C::WB + C::SB)));
    bulk_g2s(smem + s * TR * C::WB, reinterpret_cast<const uint8_t*>(wq) + row * C::WB, rows * C::WB, &s_bar[s], pol);
    bulk_g2s(smem + C::OFF_S + s * TR * C::SB, sc + row * C::SB, rows * C::SB, &s_bar[s], pol);
  };
  if (tid == 0) {
    const int pre = min(NS - 1, ntiles);
    for (int t = 0; t < pre; ++t) issue(t);
  }
  // The weights are constant: their first tiles are fetched while the previous kernel may still
  // run; everything below reads or writes activations and waits for it.  The trigger follows the
  // wait (a successor that starts implies the previous launch has finished).
  pdl_wait();
  pdl_trigger();

  // x prologue: this thread's 32 elements of every row as (even, odd) fp32 pairs times 2^-14.
  // The reference scales the weights (half-bit e2m1 decode = value * 2^-14, qmv_kernel.py:16-25);
  // here x carries the 2^-14 instead.  x * 2^-14 is exact for every bf16 x (its lowest set bit is
  // >= 2^-133, the scaled one >= 2^-147 > 2^-149), so e2m1 * (x * 2^-14) is the same exact product as
  // (e2m1 * 2^-14) * x and every fma rounds identically.
  uint64_t xp[M][16];
#pragma unroll
  for (int m = 0; m < M; ++m) {
    const uint16_t* xg = x + size_t(m) * size_t(C::K) + 32 * c;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint4 u = *reinterpret_cast<const uint4*>(xg + 8 * q);
      const uint32_t uu[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int h = 0; h < 4; ++h)
        xp[m][4 * q + h] = pack2(__fmul_rn(bflo(uu[h]), 0x1p-14f), __fmul_rn(bfhi(uu[h]), 0x1p-14f));
    }
  }

  bool abort = false;
  for (int t = 0; t < ntiles && !abort; ++t) {
    if (tid == 0 && t + NS - 1 < ntiles) {
      fence_proxy_async();
      issue(t + NS - 1);
    }
    const int s = t % NS;
    const bool ok = mbar_wait_bounded(&s_bar[s], uint32_t((t / NS) & 1), err);
    const int rows = min(TR, nrows - t * TR);

    float val[C::VP];
#pragma unroll
    for (int i = 0; i < C::VP; ++i) val[i] = 0.0f;
    if (ok) {
      const unsigned char* sw = smem + s * TR * C::WB;
      // All TR rows are computed (rows past the tile end read stale stage data and are dropped),
      // so the FMA chains of different rows interleave freely.
#pragma unroll
      for (int r = 0; r < TR; ++r) {
        const uint4 wv = *reinterpret_cast<const uint4*>(sw + r * C::WB + c * 16);
        const uint32_t wd[4] = {wv.x, wv.y, wv.z, wv.w};
        const uint8_t* ss = smem + C::OFF_S + s * TR * C::SB + r * C::SB;
        const float s0 = e4m3_x16k(ss[2 * c]), s1 = e4m3_x16k(ss[2 * c + 1]);
        float T[2][M];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          uint64_t acc[M];
#pragma unroll
          for (int m = 0; m < M; ++m) acc[m] = pack2(0.0f, 0.0f);
#pragma unroll
          for (int q = 0; q < 2; ++q) {
            uint64_t f[4];
            e2m1_pairs(wd[2 * h + q], f);  // f[b] = nibbles (2b, 2b+1) of the word
#pragma unroll
            for (int m = 0; m < M; ++m) {
#pragma unroll
              for (int b = 0; b < 4; ++b) acc[m] = ffma2(f[b], xp[m][8 * h + 4 * q + b], acc[m]);
            }
          }
#pragma unroll
          for (int m = 0; m < M; ++m) {
            float ae, ao;
            unpack2(acc[m], ae, ao);
            T[h][m] = __fadd_rn(ae, ao);
          }
        }
#pragma unroll
        for (int m = 0; m < M; ++m) val[r * M + m] = __fmaf_rn(s1, T[1][m], __fmul_rn(s0, T[0][m]));
      }
    }
    int idx;
    bool owner;
    warp_reduce_scatter<C::VP>(val, lane, idx, owner);
    float* red = s_red + (t & 1) * W * C::VP;
    if (owner) red[warp * C::VP + idx] = val[0];
    abort = __syncthreads_or(!ok) != 0;
    if (!abort && tid < rows * M) {
      float acc = red[tid];
#pragma unroll
      for (int w = 1; w < W; ++w) acc = __fadd_rn(acc, red[w * C::VP + tid]);
      const int r = tid / M, m = tid - (tid / M) * M;
      const size_t o = size_t(m) * ldy + r0 + t * TR + r;
      uint16_t out = f2bf(acc);
      if (res) out = f2bf(__fadd_rn(bf2f(res[o]), bf2f(out)));  // residual: R(res + R(x.W))
      y[o] = out;
    }
  }
}

// ----------------------------------------------------------------------------- launchers
template <int M, int W>
static int launch_qmv(const QmvParams& p, cudaStream_t st) {
  constexpr int TR = (W <= 4) ? 8 : 4;
  constexpr int NS = 3;
  using C = QmvCfg<M, W, TR, NS>;
  auto kern = qmv_kernel<M, W, TR, NS>;
  static int occ = -1;
  static std::once_flag once;
  std::call_once(once, [&] {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM) != cudaSuccess) return;
    cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    int o = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o, kern, W * 32, C::SMEM) != cudaSuccess) return;
    occ = o;
  });
  if (occ <= 0) return QMTP_ERR_CUDA;
  const int grid = std::max(1, std::min(p.N, sm_count() * occ));
  launch_kernel(kern, dim3(grid), dim3(W * 32), C::SMEM, st, p);
  return cudaGetLastError() == cudaSuccess ? QMTP_OK : QMTP_ERR_CUDA;
}

template <int M>
static int dispatch_w(int K, const QmvParams& p, cudaStream_t st) {
  switch (K) {
    case 1024: return launch_qmv<M, 1>(p, st);
    case 2048: return launch_qmv<M, 2>(p, st);
    case 4096: return launch_qmv<M, 4>(p, st);
    case 8192: return launch_qmv<M, 8>(p, st);
    case 12288: return launch_qmv<M, 12>(p, st);
    default: return QMTP_ERR_SHAPE;
  }
}

static int qmv_nvfp4_entry(const void* x, const void* w, const void* s, void* y, const void* res, int M, int N, int K,
                           int ldy, void* stream) {
  if (!x || !w || !s || !y) return QMTP_ERR_ARG;
  if (M < 1 || N < 1 || K < 1024 || K % 1024 != 0 || K > 12288 || ldy < N) return QMTP_ERR_SHAPE;
  if (!aligned16(x) || !aligned16(w) || !aligned16(s)) return QMTP_ERR_ALIGN;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  for (int m0 = 0; m0 < M; m0 += 4) {
    const int mm = std::min(4, M - m0);
    QmvParams p{};
    p.x = static_cast<const uint16_t*>(x) + size_t(m0) * size_t(K);
    p.wq = static_cast<const uint32_t*>(w);
    p.sc = static_cast<const uint8_t*>(s);
    p.y = static_cast<uint16_t*>(y) + size_t(m0) * ldy;
    p.res = res ? static_cast<const uint16_t*>(res) + size_t(m0) * ldy : nullptr;
    p.N = N;
    p.ldy = ldy;
    p.err = device_error_ptr();
    int rc;
    switch (mm) {
      case 1: rc = dispatch_w<1>(K, p, st); break;
      case 2: rc = dispatch_w<2>(K, p, st); break;
      case 3: rc = dispatch_w<3>(K, p, st); break;
      default: rc = dispatch_w<4>(K, p, st); break;
    }
    if (rc != QMTP_OK) return rc;
  }
  return QMTP_OK;
}

// ----------------------------------------------------------------------------- quantizer
// One warp per (row, group of 64): lane l holds elements 2l, 2l+1.  min/max are exact, so any
// reduction order gives the oracle's values; the rest is elementwise.
__global__ void quantize_affine_kernel(const uint16_t* __restrict__ w, uint32_t* __restrict__ wq,
                                       uint16_t* __restrict__ sc, uint16_t* __restrict__ bi, int N, int K) {
  pdl_trigger();
  pdl_wait();
  const int G = K / 64;
  const long long gid = (long long)blockIdx.x * (blockDim.x / 32) + (threadIdx.x / 32);
  if (gid >= (long long)N * G) return;
  const int lane = threadIdx.x & 31;
  const int n = int(gid / G), g = int(gid - (long long)n * G);
  const uint32_t pair = reinterpret_cast<const uint32_t*>(w + size_t(n) * K + size_t(g) * 64)[lane];
  const float v0 = bflo(pair), v1 = bfhi(pair);
  float mn = fminf(v0, v1), mx = fmaxf(v0, v1);
#pragma unroll
  for (int d = 16; d >= 1; d >>= 1) {
    mn = fminf(mn, __shfl_xor_sync(0xFFFFFFFFu, mn, d));
    mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, d));
  }
  uint16_t sb = f2bf(__fdiv_rn(__fsub_rn(mx, mn), 15.0f));
  if ((sb & 0x7FFFu) == 0) sb = 0x3F80;
  const uint16_t bb = f2bf(__fadd_rn(mn, 0.0f));  // -0 -> +0
  const float s = bf2f(sb), b = bf2f(bb);
  float q0 = rintf(__fdiv_rn(__fsub_rn(v0, b), s));
  float q1 = rintf(__fdiv_rn(__fsub_rn(v1, b), s));
  q0 = fminf(fmaxf(q0, 0.0f), 15.0f);
  q1 = fminf(fmaxf(q1, 0.0f), 15.0f);
  // lanes 4i..4i+3 hold the 8 nibbles of word i (low nibble first)
  uint32_t part = (uint32_t(q0) | (uint32_t(q1) << 4)) << (8 * (lane & 3));
  part |= __shfl_xor_sync(0xFFFFFFFFu, part, 1);
  part |= __shfl_xor_sync(0xFFFFFFFFu, part, 2);
  if ((lane & 3) == 0) wq[(size_t(n) * K + size_t(g) * 64) / 8 + (lane >> 2)] = part;
  if (lane == 0) {
    sc[size_t(n) * G + g] = sb;
    bi[size_t(n) * G + g] = bb;
  }
}

}  // namespace qmtp

using namespace qmtp;

extern "C" int qmtp_qmv_nvfp4_g16(const void* x, const void* w, const void* scales, void* y, int M, int N, int K,
                                  int ldy, void* stream) {
  return qmv_nvfp4_entry(x, w, scales, y, nullptr, M, N, K, ldy, stream);
}

extern "C" int qmtp_qmv_nvfp4_g16_res(const void* x, const void* w, const void* scales, void* y, const void* res,
                                      int M, int N, int K, int ldy, void* stream) {
  return qmv_nvfp4_entry(x, w, scales, y, res, M, N, K, ldy, stream);
}

extern "C" int qmtp_quantize_affine_g64(const void* w, void* wq, void* scales, void* biases, int N, int K,
                                        void* stream) {
  if (!w || !wq || !scales || !biases) return QMTP_ERR_ARG;
  if (N < 1 || K < 64 || K % 64 != 0) return QMTP_ERR_SHAPE;
  if (!aligned16(w) || !aligned16(wq)) return QMTP_ERR_ALIGN;
  const long long groups = (long long)N * (K / 64);
  const int wpb = 8;
  const long long blocks = (groups + wpb - 1) / wpb;
  if (blocks > 0x7FFFFFFFLL) return QMTP_ERR_SHAPE;
  launch_kernel(quantize_affine_kernel, dim3(unsigned(blocks)), dim3(wpb * 32), 0, static_cast<cudaStream_t>(stream), 
      static_cast<const uint16_t*>(w), static_cast<uint32_t*>(wq), static_cast<uint16_t*>(scales),
      static_cast<uint16_t*>(biases), N, K);
  return cudaGetLastError() == cudaSuccess ? QMTP_OK : QMTP_ERR_CUDA;
}
