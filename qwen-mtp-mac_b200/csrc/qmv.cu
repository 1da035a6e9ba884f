// Multi-row 4-bit GEMV (qmv) for B200: affine group-64 and NVFP4 group-16.
//
// Replaces qmv_kernel.py:14-101 (qmv_nvfp4_multi) and the MLX quantized_matmul route for 1-4
// activation rows.  Design (HBM-bound streaming of the weights, each byte read once per call):
//   * one CTA per SM-slot, persistent over a contiguous range of output rows;
//   * the CTA's weight / scale / bias rows arrive by 1-D TMA bulk copies (cp.async.bulk) into an
//     NS-stage shared-memory ring, completion tracked by mbarriers (bounded waits);
//   * "x-stationary": warp w, lane l owns K-chunk c = 32w + l (32 elements) for the whole kernel
//     and keeps those x values (all M rows) in registers, so x is read from HBM/L2 once per CTA;
//   * nibbles become exact floats with one AND/OR on a shifted word (2048+q / 128+q), the offsets
//     are removed through precomputed per-chunk x sums (see the oracle for the exact sequence);
//   * the per-chunk partials of TR rows x M columns are reduced across the warp with a
//     reduce-scatter (one shuffle + add per value) and across warps in shared memory.
// The fp32 operation order is the one of oracle/qmtp_oracle.c:qo_qmv_affine / qo_qmv_nvfp4.
#include <algorithm>
#include <mutex>
#include <type_traits>

#include "common.cuh"

namespace qmtp {

enum QFmt { FMT_AFFINE = 0, FMT_NVFP4 = 1 };
// x prologue applied while the x chunk is loaded (the op whose output the GEMV consumes, fused):
//   PRE_RMSNORM: x <- bf16(w * bf16(x * rsqrt(mean(x^2) + eps))) over the full row of K (decode.cu
//                rmsnorm_wide_kernel, same chunk ownership and reduction order, so bit-identical);
//   PRE_SWIGLU:  x <- bf16(silu_bf(gate) * up) with gate = x[:, 0:K], up = x[:, K:2K] (swiglu_kernel).
enum QPre { PRE_NONE = 0, PRE_RMSNORM = 1, PRE_SWIGLU = 2 };
// Epilogues (the op that consumes y, fused where it costs each output element once):
//   EPI_SWIGLU: the weight rows are [gate (N) | up (N)]; a CTA owns gate rows [r0, r1) and the up rows
//               N + [r0, r1), so y[m][j] = bf16(silu_bf(bf16(g)) * bf16(u)) (swiglu_kernel's sequence);
//   EPI_NORM:   after the last output is written, the CTA that finishes last RMS-normalises the M
//               rows of y into norm_y (rmsnorm_wide_kernel's chunk ownership and reduction order).
enum QEpi { EPI_NONE = 0, EPI_SWIGLU = 1, EPI_NORM = 2 };

// Up to four byte ranges that later kernels read, prefetched into L2 while this kernel streams
// its own weights (the CTAs split every range evenly).  Ranges are 16-byte aligned multiples of 16.
struct QPf {
  const uint8_t* p[4];
  unsigned long long n[4];
};

struct QmvParams {
  const uint16_t* x;
  long long ldx;
  const uint32_t* wq;
  const uint8_t* sc;
  const uint8_t* bi;
  uint16_t* y;
  const uint16_t* res;
  int N, ldy;
  unsigned* err;
  const uint16_t* pre_w;
  float eps;
  uint16_t* norm_y;        // EPI_NORM output rows (stride ldn), weight norm_w, epsilon norm_eps
  const uint16_t* norm_w;
  long long ldn;
  float norm_eps;
  unsigned* sync;          // EPI_NORM arrival counter: 0 before the launch, reset to 0 by the last CTA
  QPf pf;
};

template <int FMT, int M, int W, int TR, int NS>
struct QmvCfg {
  static constexpr int K = W * 1024;
  static constexpr int WB = K / 2;                               // weight bytes per row
  static constexpr int SB = (FMT == FMT_AFFINE) ? K / 32 : K / 16;  // scale bytes per row
  static constexpr int BB = (FMT == FMT_AFFINE) ? K / 32 : 0;       // bias bytes per row
  static constexpr int NV = TR * M;
  static constexpr int VP = NV <= 1 ? 1 : NV <= 2 ? 2 : NV <= 4 ? 4 : NV <= 8 ? 8 : NV <= 16 ? 16 : 32;
  static_assert(NV <= 32, "TR*M must be <= 32");
  static constexpr int OFF_S = NS * TR * WB;
  static constexpr int OFF_B = OFF_S + NS * TR * SB;
  static constexpr int OFF_RED = OFF_B + NS * TR * BB;
  static constexpr int OFF_BAR = OFF_RED + 2 * W * VP * 4;
  static constexpr int OFF_PRE = OFF_BAR + NS * 8;                 // per-(row, warp) sums of squares
  static constexpr int OFF_FLAG = OFF_PRE + 4 * 16 * 4;           // norm factors [4] + last-CTA flag
  static constexpr int SMEM = OFF_FLAG + 32;
};

__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// This CTA's share of the prefetch ranges (contiguous 16-byte-aligned slices, 64 KB per request).
__device__ __forceinline__ void issue_prefetch(const QPf& pf) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const unsigned long long n = pf.n[i];
    if (n == 0) continue;
    const unsigned long long per = ((n + gridDim.x - 1) / gridDim.x + 15) & ~15ull;
    const unsigned long long beg = per * blockIdx.x;
    const unsigned long long end = min(beg + per, n);
    for (unsigned long long o = beg; o < end; o += 65536ull)
      prefetch_l2(pf.p[i] + o, uint32_t(min(65536ull, end - o)));
  }
}

// (a & b) | c as one LOP3 (written out: the C++ form costs an extra logic op per value).
__device__ __forceinline__ uint32_t and_or(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
// acc = fma(a.lo, x.lo, acc); acc = fma(a.hi, x.hi, acc) with bf16 operands taken from the halves
// of 32-bit registers and an fp32 accumulator (fma.rn.f32.bf16: single rounding, = fmaf on the
// widened values).
__device__ __forceinline__ void fma_bf16x2(float& acc, uint32_t a, uint32_t x) {
  asm("{\n\t.reg .b16 a0, a1, x0, x1;\n\t"
      "mov.b32 {a0, a1}, %1;\n\t"
      "mov.b32 {x0, x1}, %2;\n\t"
      "fma.rn.f32.bf16 %0, a0, x0, %0;\n\t"
      "fma.rn.f32.bf16 %0, a1, x1, %0;\n\t}"
      : "+f"(acc)
      : "r"(a), "r"(x));
}

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

template <int FMT, int M, int W, int TR, int NS, int PRE, int EPI>
__global__ void __launch_bounds__(W * 32, 1) qmv_kernel(const __grid_constant__ QmvParams p) {
  using C = QmvCfg<FMT, M, W, TR, NS>;
  constexpr int K = C::K;
  // output rows per tile: with EPI_SWIGLU a tile holds HT gate rows (stage rows 0..HT-1) and the
  // matching HT up rows (stage rows HT..TR-1)
  constexpr int HT = EPI == EPI_SWIGLU ? TR / 2 : TR;
  static_assert(EPI != EPI_SWIGLU || TR % 2 == 0, "swiglu tiles pair rows");
  const uint16_t* __restrict__ x = p.x;
  const uint32_t* __restrict__ wq = p.wq;
  const uint8_t* __restrict__ sc = p.sc;
  const uint8_t* __restrict__ bi = p.bi;
  uint16_t* __restrict__ y = p.y;
  const uint16_t* __restrict__ res = p.res;
  const int N = p.N, ldy = p.ldy;
  unsigned* __restrict__ err = p.err;
  const long long ldx = p.ldx;
  const uint16_t* __restrict__ pre_w = p.pre_w;
  const float eps = p.eps;
  extern __shared__ __align__(128) unsigned char smem[];
  float* s_red = reinterpret_cast<float*>(smem + C::OFF_RED);
  uint64_t* s_bar = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int c = warp * 32 + lane;  // this thread's K-chunk
  // whole tiles per CTA (only the last tile of the matrix can be partial), so no CTA computes the
  // unused rows of a partial tile of its own
  const int ntot = (N + HT - 1) / HT;
  const int t0 = int((long long)blockIdx.x * ntot / gridDim.x);
  const int t1 = int((long long)(blockIdx.x + 1) * ntot / gridDim.x);
  const int r0 = t0 * HT;
  const int r1 = min(N, t1 * HT);
  const int nrows = max(0, r1 - r0);
  const int ntiles = (nrows + HT - 1) / HT;

  if (tid == 0) {
#pragma unroll
    for (int s = 0; s < NS; ++s) mbar_init(&s_bar[s], 1);
    fence_mbar_init();
  }
  __syncthreads();

  const uint64_t pol = policy_evict_first();
  auto issue_rows = [&](int s, int slot, size_t row, int rows) {
    bulk_g2s(smem + (s * TR + slot) * C::WB, reinterpret_cast<const uint8_t*>(wq) + row * C::WB, rows * C::WB,
             &s_bar[s], pol);
    bulk_g2s(smem + C::OFF_S + (s * TR + slot) * C::SB, sc + row * C::SB, rows * C::SB, &s_bar[s], pol);
    if constexpr (FMT == FMT_AFFINE)
      bulk_g2s(smem + C::OFF_B + (s * TR + slot) * C::BB, bi + row * C::BB, rows * C::BB, &s_bar[s], pol);
  };
  auto issue = [&](int t) {
    const int s = t % NS;
    const int rows = min(HT, nrows - t * HT);
    const size_t row = size_t(r0) + size_t(t) * HT;
    mbar_expect_tx(&s_bar[s], uint32_t((EPI == EPI_SWIGLU ? 2 : 1) * rows * (C::WB + C::SB + C::BB)));
    issue_rows(s, 0, row, rows);
    if constexpr (EPI == EPI_SWIGLU) issue_rows(s, HT, row + size_t(N), rows);
  };
  if (tid == 0) {
    const int pre = min(NS - 1, ntiles);
    for (int t = 0; t < pre; ++t) issue(t);
  }
  // The weights are constant: their first tiles are fetched while the previous kernel may still
  // run; everything below reads or writes activations and waits for it.
  pdl_trigger();
  pdl_wait();

  // x prologue (this thread's 32 elements of every row m).  Affine: bf16 pairs
  // xb[m][4q + j] = (x[8q + j], x[8q + j + 4]) matching the nibble pairs of word q, the lane sums
  // Sx_h, the initial accumulators -128*Sx_h and the chunk sum.  NVFP4: (even, odd) fp32 pairs times 2^-14.
  uint32_t xb[M][16];
  uint64_t xp[FMT == FMT_AFFINE ? 1 : M][16];
  float a0init[M][2];
  float xsum[M];
  // fused prologue ops: this thread's 32 x values of every row (row m at x + m * ldx)
  uint4 xin[M][4];
#pragma unroll
  for (int m = 0; m < M; ++m) {
    const uint16_t* xg = x + size_t(m) * size_t(ldx) + 32 * c;
#pragma unroll
    for (int q = 0; q < 4; ++q) xin[m][q] = *reinterpret_cast<const uint4*>(xg + 8 * q);
  }
  if constexpr (PRE == PRE_SWIGLU) {
#pragma unroll
    for (int m = 0; m < M; ++m) {
      const uint16_t* ug = x + size_t(m) * size_t(ldx) + K + 32 * c;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint4 uv = *reinterpret_cast<const uint4*>(ug + 8 * q);
        const uint32_t gg[4] = {xin[m][q].x, xin[m][q].y, xin[m][q].z, xin[m][q].w};
        const uint32_t uu[4] = {uv.x, uv.y, uv.z, uv.w};
        uint32_t o[4];
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          const uint16_t lo = f2bf(__fmul_rn(silu_bf(bflo(gg[h])), bflo(uu[h])));
          const uint16_t hi = f2bf(__fmul_rn(silu_bf(bfhi(gg[h])), bfhi(uu[h])));
          o[h] = lo | (uint32_t(hi) << 16);
        }
        xin[m][q] = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
  }
  if constexpr (PRE == PRE_RMSNORM) {
    float* s_pre = reinterpret_cast<float*>(smem + C::OFF_PRE);  // [M][W]
#pragma unroll
    for (int m = 0; m < M; ++m) {
      float ss = 0.0f;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint32_t uu[4] = {xin[m][q].x, xin[m][q].y, xin[m][q].z, xin[m][q].w};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          ss = __fmaf_rn(bflo(uu[h]), bflo(uu[h]), ss);
          ss = __fmaf_rn(bfhi(uu[h]), bfhi(uu[h]), ss);
        }
      }
      ss = warp_sum(ss);
      if (lane == 0) s_pre[m * W + warp] = ss;
    }
    __syncthreads();
#pragma unroll
    for (int m = 0; m < M; ++m) {
      float t = s_pre[m * W];
#pragma unroll
      for (int w = 1; w < W; ++w) t = __fadd_rn(t, s_pre[m * W + w]);
      const float r = rsqrt_rn(__fadd_rn(__fdiv_rn(t, float(K)), eps));
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint4 wu = *reinterpret_cast<const uint4*>(pre_w + 32 * c + 8 * q);
        const uint32_t ww[4] = {wu.x, wu.y, wu.z, wu.w};
        const uint32_t uu[4] = {xin[m][q].x, xin[m][q].y, xin[m][q].z, xin[m][q].w};
        uint32_t o[4];
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          const uint16_t lo = f2bf(__fmul_rn(bflo(ww[h]), R(__fmul_rn(bflo(uu[h]), r))));
          const uint16_t hi = f2bf(__fmul_rn(bfhi(ww[h]), R(__fmul_rn(bfhi(uu[h]), r))));
          o[h] = lo | (uint32_t(hi) << 16);
        }
        xin[m][q] = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
  }
#pragma unroll
  for (int m = 0; m < M; ++m) {
    uint4 u[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) u[q] = xin[m][q];
    if constexpr (FMT == FMT_AFFINE) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        xb[m][4 * q + 0] = __byte_perm(u[q].x, u[q].z, 0x5410);
        xb[m][4 * q + 1] = __byte_perm(u[q].x, u[q].z, 0x7632);
        xb[m][4 * q + 2] = __byte_perm(u[q].y, u[q].w, 0x5410);
        xb[m][4 * q + 3] = __byte_perm(u[q].y, u[q].w, 0x7632);
      }
      float sx[2] = {0.0f, 0.0f};
#pragma unroll
      for (int q = 0; q < 4; ++q)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          sx[q & 1] = __fadd_rn(sx[q & 1], bflo(xb[m][4 * q + j]));
          sx[q & 1] = __fadd_rn(sx[q & 1], bfhi(xb[m][4 * q + j]));
        }
      a0init[m][0] = -__fmul_rn(128.0f, sx[0]);
      a0init[m][1] = -__fmul_rn(128.0f, sx[1]);
      xsum[m] = __fadd_rn(sx[0], sx[1]);
    } else {
#pragma unroll
      // The reference scales the weights (half-bit e2m1 decode = value * 2^-14, qmv_kernel.py:16-25);
      // here x carries the 2^-14 instead.  x * 2^-14 is exact for every bf16 x (its lowest set bit
      // is >= 2^-133, the scaled one >= 2^-147 > 2^-149), so e2m1 * (x * 2^-14) is the same exact
      // product as (e2m1 * 2^-14) * x and every fma rounds identically.
      for (int q = 0; q < 4; ++q) {
        const uint32_t uu[4] = {u[q].x, u[q].y, u[q].z, u[q].w};
#pragma unroll
        for (int h = 0; h < 4; ++h)
          xp[m][4 * q + h] = pack2(__fmul_rn(bflo(uu[h]), 0x1p-14f), __fmul_rn(bfhi(uu[h]), 0x1p-14f));
      }
      a0init[m][0] = a0init[m][1] = 0.0f;
      xsum[m] = 0.0f;
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
    const int rows = min(HT, nrows - t * HT);
    // L2 prefetch for the following kernels once this CTA's own stream is flowing
    if (t == 0 && tid == 0) issue_prefetch(p.pf);

    float val[C::VP];
#pragma unroll
    for (int i = 0; i < C::VP; ++i) val[i] = 0.0f;
    if (ok) {
      const unsigned char* sw = smem + s * TR * C::WB;
      // All TR rows are computed (rows past the tile end read stale stage data and are dropped),
      // so the FMA chains of different rows interleave freely.
#pragma unroll
      for (int r = 0; r < TR; ++r) {
        if constexpr (FMT == FMT_AFFINE) {
          const uint4 wv = *reinterpret_cast<const uint4*>(sw + r * C::WB + c * 16);
          const uint32_t wd[4] = {wv.x, wv.y, wv.z, wv.w};
          const uint16_t* ss = reinterpret_cast<const uint16_t*>(smem + C::OFF_S + s * TR * C::SB + r * C::SB);
          const uint16_t* bb = reinterpret_cast<const uint16_t*>(smem + C::OFF_B + s * TR * C::BB + r * C::BB);
          const float sv = bf2f(ss[c >> 1]), bv = bf2f(bb[c >> 1]);
          float a[M][2];
#pragma unroll
          for (int m = 0; m < M; ++m) { a[m][0] = a0init[m][0]; a[m][1] = a0init[m][1]; }
#pragma unroll
          for (int q = 0; q < 4; ++q) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const uint32_t pr = and_or(wd[q] >> (4 * j), 0x000F000Fu, 0x43004300u);  // (128+q_j, 128+q_j+4)
#pragma unroll
              for (int m = 0; m < M; ++m) fma_bf16x2(a[m][q & 1], pr, xb[m][4 * q + j]);
            }
          }
#pragma unroll
          for (int m = 0; m < M; ++m)
            val[r * M + m] = __fmaf_rn(bv, xsum[m], __fmul_rn(sv, __fadd_rn(a[m][0], a[m][1])));
        } else {
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
      const size_t o = size_t(m) * ldy + r0 + t * HT + r;
      uint16_t out;
      if constexpr (EPI == EPI_SWIGLU) {
        const int tu = tid + HT * M;  // value (r + HT, m): the up row paired with gate row r
        float au = red[tu];
#pragma unroll
        for (int w = 1; w < W; ++w) au = __fadd_rn(au, red[w * C::VP + tu]);
        out = f2bf(__fmul_rn(silu_bf(bf2f(f2bf(acc))), bf2f(f2bf(au))));
      } else {
        out = f2bf(acc);
        if (res) out = f2bf(__fadd_rn(bf2f(res[o]), bf2f(out)));  // residual: R(res + R(x.W))
      }
      y[o] = out;
    }
  }

  if constexpr (EPI == EPI_NORM) {
    // Publish this CTA's outputs and count arrivals (threadfence-reduction pattern, no waiting):
    // the CTA that arrives last sees every row of y and normalises it.
    float* s_blk = reinterpret_cast<float*>(smem + C::OFF_PRE);  // [M][16] per-warp sums of squares
    unsigned* s_last = reinterpret_cast<unsigned*>(smem + C::OFF_FLAG + 16);
    __threadfence();
    __syncthreads();
    if (tid == 0) *s_last = (atomicAdd(p.sync, 1u) == gridDim.x - 1) ? 1u : 0u;
    __syncthreads();
    if (*s_last == 0u) return;
    __threadfence();
    // rmsnorm_wide_kernel over D = N features: thread c < D/32 owns elements [32c, 32c + 32).
    const int nthr = N / 32;
    uint32_t v[M][16];
    uint4 wn[4];
    if (tid < nthr) {
#pragma unroll
      for (int q = 0; q < 4; ++q) wn[q] = __ldg(reinterpret_cast<const uint4*>(p.norm_w + 32 * tid + 8 * q));
#pragma unroll
      for (int m = 0; m < M; ++m)
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint4 u = __ldcg(reinterpret_cast<const uint4*>(y + size_t(m) * ldy + 32 * tid + 8 * q));
          v[m][4 * q] = u.x; v[m][4 * q + 1] = u.y; v[m][4 * q + 2] = u.z; v[m][4 * q + 3] = u.w;
        }
#pragma unroll
      for (int m = 0; m < M; ++m) {
        float ss = 0.0f;
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          ss = __fmaf_rn(bflo(v[m][e]), bflo(v[m][e]), ss);
          ss = __fmaf_rn(bfhi(v[m][e]), bfhi(v[m][e]), ss);
        }
        ss = warp_sum(ss);
        if (lane == 0) s_blk[m * 16 + warp] = ss;
      }
    }
    __syncthreads();
    if (tid < nthr) {
#pragma unroll
      for (int m = 0; m < M; ++m) {
        // every thread forms the row factor itself (same sequence as the block's thread 0)
        float t = s_blk[m * 16];
        for (int i = 1; i < nthr / 32; ++i) t = __fadd_rn(t, s_blk[m * 16 + i]);
        const float r = rsqrt_rn(__fadd_rn(__fdiv_rn(t, float(N)), p.norm_eps));
        uint16_t* orow = p.norm_y + size_t(m) * size_t(p.ldn) + 32 * tid;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint32_t ww[4] = {wn[q].x, wn[q].y, wn[q].z, wn[q].w};
          uint32_t o[4];
#pragma unroll
          for (int h = 0; h < 4; ++h) {
            const uint16_t lo = f2bf(__fmul_rn(bflo(ww[h]), R(__fmul_rn(bflo(v[m][4 * q + h]), r))));
            const uint16_t hi = f2bf(__fmul_rn(bfhi(ww[h]), R(__fmul_rn(bfhi(v[m][4 * q + h]), r))));
            o[h] = lo | (uint32_t(hi) << 16);
          }
          *reinterpret_cast<uint4*>(orow + 8 * q) = make_uint4(o[0], o[1], o[2], o[3]);
        }
      }
    }
    if (tid == 0) *p.sync = 0u;  // ready for the next launch on this counter
  }
}

// ----------------------------------------------------------------------------- launchers
struct QmvLaunch {
  int grid_per_sm, block, smem, rows_per_tile, stages;
};

template <int FMT, int M, int W, int PRE, int EPI>
static int launch_qmv(const QmvParams& p, cudaStream_t st, QmvLaunch* info) {
  constexpr int TR = (W <= 4) ? 8 : 4;
  constexpr int NS = 3;
  using C = QmvCfg<FMT, M, W, TR, NS>;
  auto kern = qmv_kernel<FMT, M, W, TR, NS, PRE, EPI>;
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
  if (info) {
    *info = QmvLaunch{occ, W * 32, C::SMEM, TR, NS};
    return QMTP_OK;
  }
  const int grid = std::max(1, std::min(p.N, sm_count() * occ));
  launch_kernel(kern, dim3(grid), dim3(W * 32), C::SMEM, st, p);
  return cudaGetLastError() == cudaSuccess ? QMTP_OK : QMTP_ERR_CUDA;
}

template <int FMT, int M, int PRE, int EPI>
static int dispatch_w(int K, const QmvParams& p, cudaStream_t st, QmvLaunch* info = nullptr) {
  switch (K) {
    case 1024: return launch_qmv<FMT, M, 1, PRE, EPI>(p, st, info);
    case 2048: return launch_qmv<FMT, M, 2, PRE, EPI>(p, st, info);
    case 4096: return launch_qmv<FMT, M, 4, PRE, EPI>(p, st, info);
    case 8192: return launch_qmv<FMT, M, 8, PRE, EPI>(p, st, info);
    case 12288: return launch_qmv<FMT, M, 12, PRE, EPI>(p, st, info);
    default: return QMTP_ERR_SHAPE;
  }
}

template <int FMT, int PRE, int EPI>
static int dispatch_m(int M, int K, const QmvParams& p, cudaStream_t st, QmvLaunch* info = nullptr) {
  switch (M) {
    case 1: return dispatch_w<FMT, 1, PRE, EPI>(K, p, st, info);
    case 2: return dispatch_w<FMT, 2, PRE, EPI>(K, p, st, info);
    case 3: return dispatch_w<FMT, 3, PRE, EPI>(K, p, st, info);
    default: return dispatch_w<FMT, 4, PRE, EPI>(K, p, st, info);
  }
}

// All public qmv entry points land here.  N is the number of output columns (with EPI_SWIGLU the
// weight matrix holds 2N rows).
template <int FMT>
static int qmv_entry(const void* x, const void* w, const void* s, const void* b, void* y, const void* res, int M,
                     int N, int K, int ldy, void* stream, int pre = PRE_NONE, long long ldx = 0,
                     const void* pre_w = nullptr, float eps = 0.0f, int epi = EPI_NONE, void* norm_y = nullptr,
                     const void* norm_w = nullptr, long long ldn = 0, float norm_eps = 0.0f,
                     unsigned* sync = nullptr, const QPf* pf = nullptr) {
  if (!x || !w || !s || !y || (FMT == FMT_AFFINE && !b)) return QMTP_ERR_ARG;
  if (M < 1 || N < 1 || K < 1024 || K % 1024 != 0 || K > 12288 || ldy < N) return QMTP_ERR_SHAPE;
  if (ldx == 0) ldx = pre == PRE_SWIGLU ? 2LL * K : K;
  if (ldx < (pre == PRE_SWIGLU ? 2LL * K : K) || ldx % 8) return QMTP_ERR_SHAPE;
  if ((pre != PRE_NONE || epi != EPI_NONE) && FMT != FMT_AFFINE) return QMTP_ERR_UNSUPPORTED;
  if (pre != PRE_NONE && epi != EPI_NONE) return QMTP_ERR_UNSUPPORTED;
  if (pre == PRE_RMSNORM && !pre_w) return QMTP_ERR_ARG;
  if (epi == EPI_SWIGLU && res) return QMTP_ERR_UNSUPPORTED;
  if (epi == EPI_NORM) {
    if (!norm_y || !norm_w || !sync) return QMTP_ERR_ARG;
    // the normalising CTA has K/32 threads and covers D = N with N/32 of them
    if (N % 1024 != 0 || N > K || ldy % 8 || ldn < N || ldn % 8) return QMTP_ERR_SHAPE;
    if (!aligned16(y) || !aligned16(norm_y) || !aligned16(norm_w)) return QMTP_ERR_ALIGN;
  }
  if (!aligned16(x) || !aligned16(w) || !aligned16(s) || (b && !aligned16(b)) || (pre_w && !aligned16(pre_w)))
    return QMTP_ERR_ALIGN;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const uint16_t* xp = static_cast<const uint16_t*>(x);
  uint16_t* yp = static_cast<uint16_t*>(y);
  for (int m0 = 0; m0 < M; m0 += 4) {
    const int mm = std::min(4, M - m0);
    QmvParams p{};
    p.x = xp + size_t(m0) * size_t(ldx);
    p.ldx = ldx;
    p.wq = static_cast<const uint32_t*>(w);
    p.sc = static_cast<const uint8_t*>(s);
    p.bi = static_cast<const uint8_t*>(b);
    p.y = yp + size_t(m0) * ldy;
    p.res = res ? static_cast<const uint16_t*>(res) + size_t(m0) * ldy : nullptr;
    p.N = N;
    p.ldy = ldy;
    p.err = device_error_ptr();
    p.pre_w = static_cast<const uint16_t*>(pre_w);
    p.eps = eps;
    p.norm_y = norm_y ? static_cast<uint16_t*>(norm_y) + size_t(m0) * size_t(ldn) : nullptr;
    p.norm_w = static_cast<const uint16_t*>(norm_w);
    p.ldn = ldn;
    p.norm_eps = norm_eps;
    p.sync = sync;
    if (pf && m0 == 0) p.pf = *pf;
    int rc;
    if constexpr (FMT == FMT_AFFINE) {
      rc = pre == PRE_RMSNORM ? dispatch_m<FMT, PRE_RMSNORM, EPI_NONE>(mm, K, p, st)
         : pre == PRE_SWIGLU  ? dispatch_m<FMT, PRE_SWIGLU, EPI_NONE>(mm, K, p, st)
         : epi == EPI_SWIGLU  ? dispatch_m<FMT, PRE_NONE, EPI_SWIGLU>(mm, K, p, st)
         : epi == EPI_NORM    ? dispatch_m<FMT, PRE_NONE, EPI_NORM>(mm, K, p, st)
                              : dispatch_m<FMT, PRE_NONE, EPI_NONE>(mm, K, p, st);
    } else {
      rc = dispatch_m<FMT, PRE_NONE, EPI_NONE>(mm, K, p, st);
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

extern "C" int qmtp_qmv_affine_g64(const void* x, const void* w, const void* scales, const void* biases, void* y,
                                   int M, int N, int K, int ldy, void* stream) {
  return qmv_entry<FMT_AFFINE>(x, w, scales, biases, y, nullptr, M, N, K, ldy, stream);
}

extern "C" int qmtp_qmv_affine_g64_res(const void* x, const void* w, const void* scales, const void* biases, void* y,
                                       const void* res, int M, int N, int K, int ldy, void* stream) {
  if (!res) return QMTP_ERR_ARG;
  return qmv_entry<FMT_AFFINE>(x, w, scales, biases, y, res, M, N, K, ldy, stream);
}

extern "C" int qmtp_qmv_ex(const qmtp_qmv_args* a, void* stream) {
  if (!a) return QMTP_ERR_ARG;
  if (a->pre < PRE_NONE || a->pre > PRE_SWIGLU || a->epi < EPI_NONE || a->epi > EPI_NORM) return QMTP_ERR_ARG;
  QPf pf{};
  for (int i = 0; i < 4; ++i) {
    const long long n = a->prefetch_bytes[i] & ~15LL;
    if (a->prefetch[i] && n > 0 && aligned16(a->prefetch[i])) {
      pf.p[i] = static_cast<const uint8_t*>(a->prefetch[i]);
      pf.n[i] = static_cast<unsigned long long>(n);
    }
  }
  return qmv_entry<FMT_AFFINE>(a->x, a->w, a->scales, a->biases, a->y, a->res, a->M, a->N, a->K, a->ldy, stream,
                               a->pre, a->ldx, a->pre_w, a->pre_eps, a->epi, a->norm_y, a->norm_w, a->ld_norm,
                               a->norm_eps, a->sync, &pf);
}

extern "C" int qmtp_qmv_nvfp4_g16(const void* x, const void* w, const void* scales, void* y, int M, int N, int K,
                                  int ldy, void* stream) {
  return qmv_entry<FMT_NVFP4>(x, w, scales, nullptr, y, nullptr, M, N, K, ldy, stream);
}

extern "C" int qmtp_qmv_nvfp4_g16_res(const void* x, const void* w, const void* scales, void* y, const void* res,
                                      int M, int N, int K, int ldy, void* stream) {
  return qmv_entry<FMT_NVFP4>(x, w, scales, nullptr, y, res, M, N, K, ldy, stream);
}

extern "C" int qmtp_qmv_launch_info(int fmt, int M, int K, int* ctas_per_sm, int* threads, int* smem_bytes,
                                    int* rows_per_tile) {
  if (!ctas_per_sm || !threads || !smem_bytes || !rows_per_tile) return QMTP_ERR_ARG;
  if (M < 1 || M > 4 || (fmt != 0 && fmt != 1)) return QMTP_ERR_SHAPE;
  QmvLaunch info{};
  int rc;
  auto go = [&](auto fmtc) -> int {
    constexpr int F = decltype(fmtc)::value;
    QmvParams p{};
    p.N = 1;
    return dispatch_m<F, PRE_NONE, EPI_NONE>(M, K, p, 0, &info);
  };
  rc = fmt == 0 ? go(std::integral_constant<int, FMT_AFFINE>{}) : go(std::integral_constant<int, FMT_NVFP4>{});
  if (rc != QMTP_OK) return rc;
  *ctas_per_sm = info.grid_per_sm;
  *threads = info.block;
  *smem_bytes = info.smem;
  *rows_per_tile = info.rows_per_tile;
  return QMTP_OK;
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
