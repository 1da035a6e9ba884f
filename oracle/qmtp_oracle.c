/*
 * qmtp CPU oracle -- TEST INFRASTRUCTURE ONLY.
 *
 * This file is a plain-C restatement of the arithmetic of the qwen-mtp-mac decode hot path.
 * It is the checker for the CUDA library (tests/, __graft_entry__.smoke(), bench.py's
 * cpu_baseline leg); nothing in the product links or calls it.
 *
 * Parity status: UNPINNED against MLX.  The reference's arithmetic lives in MLX 0.31.2 /
 * mlx-lm 0.31.3 and in Metal kernels that need an Apple GPU; none of that is runnable here and
 * the reference ships no golden vectors.  What is pinned: the reference's own bit-level decoders
 * (qmv_kernel.py:16-29 deq8 / e4m3_scale, experiments/deepseek_moe/kernels.py:13-32 dot8 /
 * e8m0_scale) and its bf16 activation formulas (gdn_fused.py:22-41) are re-executed in numpy by
 * the tests and compared with the decoders and formulas below.
 *
 * Arithmetic contract.  Every function here fixes the exact IEEE-754 fp32 operation sequence
 * (explicit fmaf, no contraction: build with -ffp-contract=off).  The CUDA kernels implement the
 * same sequence, so results are bit-identical.  The sequences follow the reference where it fixes
 * them (per-lane sequential sums then a 32-lane reduction, as simd_sum in gdn_kernel.py:36-53)
 * and are chosen to be parallel-friendly where the reference leaves them to MLX:
 *   - a 32-lane reduction is the xor butterfly with strides 16, 8, 4, 2, 1;
 *   - exp / log are this file's own (Cody-Waite reduction + Taylor / atanh series), written from
 *     the mathematics and checked against libm to <= 2 ulp by the tests.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define QO_API __attribute__((visibility("default")))

/* ------------------------------------------------------------------ bf16 / bit helpers */

static inline float qo_asf(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint32_t qo_asu(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float qo_bf2f(uint16_t h) { return qo_asf((uint32_t)h << 16); }

/* fp32 -> bf16, round to nearest even; every NaN becomes 0x7FC0 (sign dropped). */
static inline uint16_t qo_f2bf(float f) {
  uint32_t u = qo_asu(f);
  if ((u & 0x7FFFFFFFu) > 0x7F800000u) return 0x7FC0;
  u += 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}
static inline float qo_R(float x) { return qo_bf2f(qo_f2bf(x)); }

/* 32-lane xor butterfly: v[l] <- v[l] + v[l ^ d] for d = 16, 8, 4, 2, 1.  All lanes end equal. */
static inline float qo_butterfly32(const float* in) {
  float v[32], t[32];
  memcpy(v, in, sizeof v);
  for (int d = 16; d >= 1; d >>= 1) {
    for (int l = 0; l < 32; ++l) t[l] = v[l] + v[l ^ d];
    memcpy(v, t, sizeof v);
  }
  return v[0];
}

/* ------------------------------------------------------------------ exp / log */

/* exp(x): k = rint(x*log2e); r = x - k*ln2 (two-constant Cody-Waite split);
 * e^r by the degree-7 Taylor polynomial (|r| <= ~0.35, truncation < 0.05 ulp);
 * result = p * 2^k1 * 2^k2 with k1 = k/2 (two exact-or-single-rounding scalings). */
static inline float qo_expf(float x) {
  if (x != x) return x;
  if (x > 88.72283935546875f) return INFINITY;
  if (x < -103.972084045410156f) return 0.0f;
  float kf = rintf(x * 1.44269502162933349609375f);
  float r = fmaf(-kf, 0.693145751953125f, x);
  r = fmaf(-kf, 1.428606765330187045e-06f, r);
  float p = 1.98412701138295233249664e-04f; /* 1/5040 */
  p = fmaf(p, r, 1.38888892251998186111450e-03f); /* 1/720 */
  p = fmaf(p, r, 8.33333376795053482055664e-03f); /* 1/120 */
  p = fmaf(p, r, 4.16666679084300994873047e-02f); /* 1/24 */
  p = fmaf(p, r, 1.66666671633720397949219e-01f); /* 1/6 */
  p = fmaf(p, r, 0.5f);
  p = fmaf(p, r, 1.0f);
  p = fmaf(p, r, 1.0f);
  int k = (int)kf;
  int k1 = k / 2, k2 = k - k1;
  float s1 = qo_asf((uint32_t)(k1 + 127) << 23), s2 = qo_asf((uint32_t)(k2 + 127) << 23);
  return (p * s1) * s2;
}

/* log(x): x = m * 2^e with m in [sqrt(1/2), sqrt(2)]; s = (m-1)/(m+1);
 * log(m) = 2 atanh(s) = 2s + s^3 (2/3 + s^2 (2/5 + s^2 (2/7 + s^2 2/9))); + e*ln2 (split). */
static inline float qo_logf(float x) {
  if (x != x) return x;
  if (x < 0.0f) return NAN;
  if (x == 0.0f) return -INFINITY;
  if (x == INFINITY) return x;
  int e = 0;
  uint32_t ix = qo_asu(x);
  if (ix < 0x00800000u) { x = x * 8388608.0f; ix = qo_asu(x); e = -23; }
  e += (int)(ix >> 23) - 127;
  float m = qo_asf((ix & 0x007FFFFFu) | 0x3F800000u);
  if (m > 1.41421353816986083984375f) { m = m * 0.5f; e += 1; }
  float f = m - 1.0f;
  float s = f / (2.0f + f);
  float z = s * s;
  float p = 2.22222223877906799316406e-01f;              /* 2/9 */
  p = fmaf(p, z, 2.85714298486709594726562e-01f);        /* 2/7 */
  p = fmaf(p, z, 4.00000005960464477539062e-01f);        /* 2/5 */
  p = fmaf(p, z, 6.66666686534881591796875e-01f);        /* 2/3 */
  float lm = fmaf(s * z, p, 2.0f * s);
  float ef = (float)e;
  return fmaf(ef, 0.693145751953125f, fmaf(ef, 1.428606765330187045e-06f, lm));
}

QO_API float qo_exp(float x) { return qo_expf(x); }
QO_API float qo_log(float x) { return qo_logf(x); }

/* ------------------------------------------------------------------ bf16 activation formulas
 * Restated from gdn_fused.py:22-41 (BF16_MATH): round to bf16 after every op, as MLX does for
 * bf16 tensors.  max/min with 0 are written as selects so that -0.0 behaves like +0.0. */

static inline float qo_sigmoid_bf(float x) {
  float y = qo_R(1.0f / qo_R(1.0f + qo_R(qo_expf(fabsf(x)))));
  return x < 0.0f ? y : qo_R(1.0f - y);
}
static inline float qo_silu_bf(float x) { return qo_R(x * qo_sigmoid_bf(x)); }
static inline float qo_log1p_bf(float x) {
  float xp1 = 1.0f + x;
  if (xp1 == 1.0f) return x;
  float t = qo_logf(xp1) / (xp1 - 1.0f);
  return qo_R(x * t);
}
static inline float qo_softplus_bf(float x) {
  float hi = x > 0.0f ? x : 0.0f, lo = x < 0.0f ? x : 0.0f;
  return qo_R(hi + qo_log1p_bf(qo_R(qo_expf(qo_R(lo - hi)))));
}
static inline float qo_silu_f32(float x) {
  float y = 1.0f / (1.0f + qo_expf(fabsf(x)));
  return x * (x < 0.0f ? y : 1.0f - y);
}
static inline float qo_sigmoid_f32(float x) {
  float y = 1.0f / (1.0f + qo_expf(fabsf(x)));
  return x < 0.0f ? y : 1.0f - y;
}

/* Elementwise evaluation over arrays of bf16 bit patterns (exhaustive tests). */
QO_API void qo_bf16_formulas(const uint16_t* x, int n, float* sg, float* sl, float* sp, float* s32) {
  for (int i = 0; i < n; ++i) {
    float v = qo_bf2f(x[i]);
    sg[i] = qo_sigmoid_bf(v);
    sl[i] = qo_silu_bf(v);
    sp[i] = qo_softplus_bf(v);
    s32[i] = qo_silu_f32(v);
  }
}

/* ------------------------------------------------------------------ 4-bit formats */

/* e2m1 nibble -> float (exact): magnitudes {0, .5, 1, 1.5, 2, 3, 4, 6}, bit 3 = sign. */
static inline float qo_e2m1(uint32_t nib) {
  static const float mag[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};
  float v = mag[nib & 7u];
  return (nib & 8u) ? -v : v;
}
/* e4m3 (fn) -> float (exact), sign ignored as in qmv_kernel.py:26-28. */
static inline float qo_e4m3(uint32_t s) {
  uint32_t e = (s >> 3) & 15u, m = s & 7u;
  if (e == 0) return (float)m * 0.001953125f; /* m/8 * 2^-6 */
  return ldexpf(1.0f + (float)m * 0.125f, (int)e - 7);
}
/* e8m0 -> 2^(s-127) (s = 255 is NaN in OCP MX; treated as 2^128 = inf here). */
static inline float qo_e8m0(uint32_t s) {
  if (s == 0) return qo_asf(0x00400000u); /* 2^-127 */
  if (s == 255) return INFINITY;
  return qo_asf(s << 23);
}
QO_API void qo_decode_tables(float* e2m1_16, float* e4m3_256, float* e8m0_256) {
  for (uint32_t i = 0; i < 16; ++i) e2m1_16[i] = qo_e2m1(i);
  for (uint32_t i = 0; i < 256; ++i) { e4m3_256[i] = qo_e4m3(i); e8m0_256[i] = qo_e8m0(i); }
}

/* ------------------------------------------------------------------ affine 4-bit quantizer
 * MLX affine convention (mx.quantize(w, group_size=64, bits=4)): per group of 64 along K,
 * w ~= scale*q + bias, q in [0,15], 8 nibbles per uint32 with the low nibble the lowest k
 * (qmv_kernel.py:8).  Restated as the plain min/max quantizer:
 *   scale = bf16((max-min)/15), bias = bf16(min), q = clamp(rint((w-bias)/scale), 0, 15);
 * a zero scale (constant group) is replaced by 1.  MLX's extra edge adjustment is not restated
 * (unpinned); every parity test feeds the same packed triple to both sides. */
QO_API void qo_quantize_affine(const uint16_t* w, uint32_t* wq, uint16_t* sc, uint16_t* bi,
                               int N, int K, int gs) {
  int G = K / gs;
#pragma omp parallel for schedule(static)
  for (int n = 0; n < N; ++n) {
    for (int g = 0; g < G; ++g) {
      const uint16_t* wg = w + (size_t)n * K + (size_t)g * gs;
      float mn = qo_bf2f(wg[0]), mx = mn;
      for (int j = 1; j < gs; ++j) {
        float v = qo_bf2f(wg[j]);
        mn = v < mn ? v : mn;
        mx = v > mx ? v : mx;
      }
      uint16_t sb = qo_f2bf((mx - mn) / 15.0f);
      if ((sb & 0x7FFFu) == 0) sb = 0x3F80; /* 1.0 */
      uint16_t bb = qo_f2bf(mn + 0.0f); /* -0 -> +0 */
      float s = qo_bf2f(sb), b = qo_bf2f(bb);
      sc[(size_t)n * G + g] = sb;
      bi[(size_t)n * G + g] = bb;
      for (int j = 0; j < gs; j += 8) {
        uint32_t word = 0;
        for (int i = 0; i < 8; ++i) {
          float q = rintf((qo_bf2f(wg[j + i]) - b) / s);
          q = q < 0.0f ? 0.0f : (q > 15.0f ? 15.0f : q);
          word |= (uint32_t)q << (4 * i);
        }
        wq[((size_t)n * K + (size_t)g * gs + j) / 8] = word;
      }
    }
  }
}

/* ------------------------------------------------------------------ qmv, affine 4-bit g64
 * y[m,n] = sum_k x[m,k] * (s[n,k/64] * q[n,k] + b[n,k/64]), K % 512 == 0.
 * Reference op: MLX quantized_matmul(x, w, s, b, transpose=True, group_size=64, bits=4) and the
 * multi-row GEMV of qmv_kernel.py:31-75 (same weight layout; that kernel is the NVFP4 variant).
 *
 * Exact sequence (block floating point per group of 64 activations, exact integer group sums):
 *   per token m and group g (k in [64g, 64g+64)):
 *     any x non-finite -> c = xf = NaN (the output row becomes NaN); all x zero -> c = xf = 0;
 *     else E = floor(log2(max|x|)), x_q = RNE(x * 2^(19-E)) (an integer, |x_q| < 2^20),
 *     c = 2^(E-19) as fp32 (0 below 2^-149), xf = float(sum_k x_q) * c;
 *   per row n:  S_g = sum_k q[n,k] * x_q[k]  (exact integer, |S_g| < 2^31);
 *     slice j = groups 8j..8j+7: H_0 = chain over groups 8j..8j+3, H_1 over 8j+4..8j+7, each from 0:
 *       H = fma(float(S_g), s_g * c_g, H);  H = fma(b_g, xf_g, H);
 *     P_j = H_0 + H_1;  y = ((P_0 + P_1) + P_2) + ...;  out = bf16(y).
 * The tensor-core kernel forms S_g from three signed byte limbs of x_q with kind::i8 MMAs; the
 * integer sums are exact, so their order does not matter.  Compared with MLX's fp32 sums this
 * rounds each group's dot product once instead of once per partial sum (x_q is exact for every
 * element >= 2^-12 of its group's maximum). */

static inline float qo_pow2(int k) {
  if (k >= -126) return qo_asf((uint32_t)(k + 127) << 23);
  if (k >= -149) return qo_asf(1u << (k + 149));
  return 0.0f;
}

/* |x| of bf16 magnitude bits a on the grid 2^(E-19), round half to even. */
static inline int32_t qo_grid_mag(uint32_t a, int E) {
  int ef = (int)(a >> 7);
  int sig = ef ? (int)(128u | (a & 127u)) : (int)(a & 127u);
  int ex = ef ? ef - 134 : -133;
  int sh = ex + 19 - E;
  if (sh >= 0) return sig << sh;
  int r = -sh;
  if (r > 8) return 0;
  int m = sig >> r, rem = sig & ((1 << r) - 1), half = 1 << (r - 1);
  if (rem > half || (rem == half && (m & 1))) ++m;
  return m;
}

/* One token row: x_q [K], c and xf per group [K/64]. */
static void qo_affine_xgroups(const uint16_t* x, int K, int32_t* xq, float* c, float* xf) {
  for (int g = 0; g < K / 64; ++g) {
    const uint16_t* xg = x + 64 * g;
    uint32_t amax = 0;
    int nf = 0;
    for (int e = 0; e < 64; ++e) {
      uint32_t a = xg[e] & 0x7FFFu;
      if (a >= 0x7F80u) nf = 1;
      if (a > amax) amax = a;
    }
    if (nf || amax == 0) {
      for (int e = 0; e < 64; ++e) xq[64 * g + e] = 0;
      c[g] = xf[g] = nf ? qo_asf(0x7FC00000u) : 0.0f;
      continue;
    }
    int ef = (int)(amax >> 7);
    int E;
    if (ef) {
      E = ef - 127;
    } else {
      int l = 0;
      while ((amax & 127u) >> (l + 1)) ++l;
      E = -133 + l;
    }
    int32_t sum = 0;
    for (int e = 0; e < 64; ++e) {
      int32_t mag = qo_grid_mag(xg[e] & 0x7FFFu, E);
      int32_t v = (xg[e] & 0x8000u) ? -mag : mag;
      xq[64 * g + e] = v;
      sum += v;
    }
    c[g] = qo_pow2(E - 19);
    xf[g] = (float)sum * c[g];
  }
}

static float qo_affine_row(const int32_t* xq, const float* c, const float* xf, const uint8_t* qrow,
                           const uint16_t* srow, const uint16_t* brow, int K) {
  int NSL = K / 512;
  float y = 0.0f;
  for (int sl = 0; sl < NSL; ++sl) {
    float H[2] = {0.0f, 0.0f};
    for (int h = 0; h < 2; ++h) {
      for (int gi = 0; gi < 4; ++gi) {
        int g = 8 * sl + 4 * h + gi;
        const uint8_t* qg = qrow + 64 * g;
        const int32_t* xg = xq + 64 * g;
        int32_t S = 0; /* exact: every partial sum is below 64 * 15 * 2^20 < 2^31 */
        for (int e = 0; e < 64; ++e) S += (int32_t)qg[e] * xg[e];
        float t = (float)S;
        float s = qo_bf2f(srow[g]), b = qo_bf2f(brow[g]);
        H[h] = fmaf(t, s * c[g], H[h]);
        H[h] = fmaf(b, xf[g], H[h]);
      }
    }
    float P = H[0] + H[1];
    y = (sl == 0) ? P : y + P;
  }
  return y;
}

QO_API int qo_qmv_affine(const uint16_t* x, const uint32_t* wq, const uint16_t* sc,
                         const uint16_t* bi, uint16_t* y, int M, int N, int K) {
  if (K % 512 != 0 || K < 512 || M < 1 || N < 1) return -1;
  int G = K / 64;
  int32_t* xq = (int32_t*)malloc(sizeof(int32_t) * (size_t)M * K);
  float* c = (float*)malloc(sizeof(float) * (size_t)M * G);
  float* xf = (float*)malloc(sizeof(float) * (size_t)M * G);
  for (int m = 0; m < M; ++m)
    qo_affine_xgroups(x + (size_t)m * K, K, xq + (size_t)m * K, c + (size_t)m * G, xf + (size_t)m * G);
#pragma omp parallel
  {
    uint8_t* qrow = (uint8_t*)malloc((size_t)K);
#pragma omp for schedule(static)
    for (int n = 0; n < N; ++n) {
      const uint32_t* wrow = wq + (size_t)n * (K / 8);
      for (int k = 0; k < K; ++k) qrow[k] = (uint8_t)((wrow[k >> 3] >> (4 * (k & 7))) & 15u);
      for (int m = 0; m < M; ++m) {
        float v = qo_affine_row(xq + (size_t)m * K, c + (size_t)m * G, xf + (size_t)m * G, qrow,
                                sc + (size_t)n * G, bi + (size_t)n * G, K);
        y[(size_t)m * N + n] = qo_f2bf(v);
      }
    }
    free(qrow);
  }
  free(xq);
  free(c);
  free(xf);
  return 0;
}

/* ------------------------------------------------------------------ qmv, NVFP4 (e2m1, e4m3 / 16)
 * y[m,n] = sum_g e4m3(s[n,g]) * sum_{i<16} e2m1(q[n,16g+i]) * x[m,16g+i]  (qmv_kernel.py:14-75,
 * MLX mode="nvfp4").  Same chunk / block / butterfly tree as the affine kernel; per chunk c the two
 * groups h = 0, 1 (16 elements each) are summed with an even/odd pair of sequential fmas:
 *   T_h = ae + ao;  P_c = fma(s_{2c+1}, T_1, s_{2c} * T_0).
 * As in qmv_kernel.py:16-28 the nibble values are carried as e2m1 * 2^-14 (exact half-precision
 * bit trick) and the 2^14 is folded into the scale, so the products are the ones the kernel forms. */
QO_API int qo_qmv_nvfp4(const uint16_t* x, const uint32_t* wq, const uint8_t* sc, uint16_t* y,
                        int M, int N, int K) {
  if (K % 1024 != 0 || M < 1 || N < 1) return -1;
  int NC = K / 32, G = K / 16;
#pragma omp parallel for schedule(static)
  for (int n = 0; n < N; ++n) {
    const uint32_t* wrow = wq + (size_t)n * (K / 8);
    const uint8_t* srow = sc + (size_t)n * G;
    for (int m = 0; m < M; ++m) {
      const uint16_t* xr = x + (size_t)m * K;
      float y_acc = 0.0f;
      for (int i = 0; i < NC / 32; ++i) {
        float P[32];
        for (int l = 0; l < 32; ++l) {
          int c = 32 * i + l;
          float T[2];
          for (int h = 0; h < 2; ++h) {
            float ae = 0.0f, ao = 0.0f;
            for (int wd = 0; wd < 2; ++wd) {
              uint32_t w = wrow[4 * c + 2 * h + wd];
              for (int jj = 0; jj < 8; jj += 2) {
                int k = 32 * c + 16 * h + 8 * wd + jj;
                ae = fmaf(qo_e2m1((w >> (4 * jj)) & 15u) * 6.103515625e-05f, qo_bf2f(xr[k]), ae);
                ao = fmaf(qo_e2m1((w >> (4 * jj + 4)) & 15u) * 6.103515625e-05f, qo_bf2f(xr[k + 1]), ao);
              }
            }
            T[h] = ae + ao;
          }
          float s0 = qo_e4m3(srow[2 * c]) * 16384.0f, s1 = qo_e4m3(srow[2 * c + 1]) * 16384.0f;
          P[l] = fmaf(s1, T[1], s0 * T[0]);
        }
        float B = qo_butterfly32(P);
        y_acc = (i == 0) ? B : y_acc + B;
      }
      y[(size_t)m * N + n] = qo_f2bf(y_acc);
    }
  }
  return 0;
}

/* ------------------------------------------------------------------ array helpers (tests) */
QO_API void qo_exp_arr(const float* x, float* y, long n) { for (long i = 0; i < n; ++i) y[i] = qo_expf(x[i]); }
QO_API void qo_log_arr(const float* x, float* y, long n) { for (long i = 0; i < n; ++i) y[i] = qo_logf(x[i]); }

/* ------------------------------------------------------------------ GatedDeltaNet
 * Lane structure of the reference kernels (gdn_kernel.py:11-64, gdn_fused.py:43-112): one
 * simdgroup per (batch, value head, dv row); lane l owns dk elements [NP*l, NP*l+NP) (NP = Dk/32),
 * sums its elements sequentially and the 32 lane partials are combined (here: xor butterfly). */

static inline float qo_lane_dot(const float* a, const float* b, int NP, int Dk) {
  /* sum over Dk of a*b: lane-sequential fmaf, then butterfly */
  float P[32];
  for (int l = 0; l < 32; ++l) {
    float acc = 0.0f;
    for (int i = 0; i < NP; ++i) acc = fmaf(a[NP * l + i], b[NP * l + i], acc);
    P[l] = acc;
  }
  (void)Dk;
  return qo_butterfly32(P);
}

/* One dv row of the delta rule over T tokens (state row st[Dk] updated in place).
 *   st *= g; kv = sum st*k; delta = (v - kv)*beta; st += k*delta; o = sum st*q.
 * Per lane and element i: st_i = st_i * g; kv = fma(st_i, k_i, kv) (interleaved, gdn_kernel.py:37-42);
 * then st_i = fma(k_i, delta, st_i); o = fma(st_i, q_i, o) (gdn_kernel.py:45-50). */
static void qo_gdn_row(float* st, int Dk, int T, const float* q, const float* k, int qk_stride,
                       const float* v, int v_stride, const float* g, const float* beta, int gb_stride,
                       float* y, int y_stride, float* mid, size_t mid_stride) {
  int NP = Dk / 32;
  for (int t = 0; t < T; ++t) {
    const float* qt = q + (size_t)t * qk_stride;
    const float* kt = k + (size_t)t * qk_stride;
    float gt = g[(size_t)t * gb_stride], bt = beta[(size_t)t * gb_stride];
    float P[32];
    for (int l = 0; l < 32; ++l) {
      float kv = 0.0f;
      for (int i = 0; i < NP; ++i) {
        int e = NP * l + i;
        st[e] = st[e] * gt;
        kv = fmaf(st[e], kt[e], kv);
      }
      P[l] = kv;
    }
    float kvm = qo_butterfly32(P);
    float delta = (v[(size_t)t * v_stride] - kvm) * bt;
    for (int l = 0; l < 32; ++l) {
      float o = 0.0f;
      for (int i = 0; i < NP; ++i) {
        int e = NP * l + i;
        st[e] = fmaf(kt[e], delta, st[e]);
        o = fmaf(st[e], qt[e], o);
      }
      P[l] = o;
    }
    y[(size_t)t * y_stride] = qo_butterfly32(P);
    if (mid && t < T - 1) memcpy(mid + (size_t)t * mid_stride, st, sizeof(float) * Dk);
  }
}

/* gated_delta_snapshot (gdn_kernel.py:75-88): q,k bf16 [B,T,Hk,Dk]; v bf16 [B,T,Hv,Dv];
 * g, beta fp32 [B,T,Hv]; state fp32 [B,Hv,Dv,Dk] -> y bf16 [B,T,Hv,Dv], state_out, state_mid
 * fp32 [T-1,B,Hv,Dv,Dk]. */
QO_API int qo_gdn_step(const uint16_t* q, const uint16_t* k, const uint16_t* v, const float* g,
                       const float* beta, const float* state_in, uint16_t* y, float* state_out,
                       float* state_mid, int B, int T, int Hk, int Hv, int Dk, int Dv) {
  if (Dk % 32 != 0 || Hv % Hk != 0 || T < 1) return -1;
  size_t per = (size_t)B * Hv * Dv * Dk;
#pragma omp parallel for collapse(2) schedule(static)
  for (int n = 0; n < B * Hv; ++n) {
    for (int dv = 0; dv < Dv; ++dv) {
      int b = n / Hv, hv = n % Hv, hk = hv / (Hv / Hk);
      float* qf = (float*)malloc(sizeof(float) * (size_t)T * Dk * 2);
      float* kf = qf + (size_t)T * Dk;
      float* vf = (float*)malloc(sizeof(float) * T);
      float* yf = (float*)malloc(sizeof(float) * T);
      float* gt = (float*)malloc(sizeof(float) * T * 2);
      float* bt = gt + T;
      for (int t = 0; t < T; ++t) {
        for (int e = 0; e < Dk; ++e) {
          size_t qi = (((size_t)b * T + t) * Hk + hk) * Dk + e;
          qf[(size_t)t * Dk + e] = qo_bf2f(q[qi]);
          kf[(size_t)t * Dk + e] = qo_bf2f(k[qi]);
        }
        vf[t] = qo_bf2f(v[(((size_t)b * T + t) * Hv + hv) * Dv + dv]);
        gt[t] = g[((size_t)b * T + t) * Hv + hv];
        bt[t] = beta[((size_t)b * T + t) * Hv + hv];
      }
      size_t row = ((size_t)n * Dv + dv) * Dk;
      float* st = state_out + row;
      memcpy(st, state_in + row, sizeof(float) * Dk);
      qo_gdn_row(st, Dk, T, qf, kf, Dk, vf, 1, gt, bt, 1, yf, 1, state_mid ? state_mid + row : NULL, per);
      for (int t = 0; t < T; ++t) y[(((size_t)b * T + t) * Hv + hv) * Dv + dv] = qo_f2bf(yf[t]);
      free(qf); free(vf); free(yf); free(gt);
    }
  }
  return 0;
}

/* gdn_core (gdn_fused.py:43-112), B = 1:
 *   win bf16 [S+KC-1, C] (C = 2*Hk*Dk + Hv*Dv), conv_w bf16 [C, KC], a, b bf16 [S, Hv] (row stride
 *   ld_ab), A_log fp32 [Hv], dt_bias bf16 [Hv], state fp32 [Hv, Dv, Dk]
 *   -> y fp32 [S, Hv, Dv] (bf16-rounded values), state_out, state_mid fp32 [S-1, Hv, Dv, Dk].
 * conv: acc = fma(w_j, win_{t+j}, acc) over taps j; q = silu_bf(R(acc)) ...
 * q/k rms: ss = lane-sequential fma(x,x) + butterfly; r = 1/sqrt(ss/Dk + 1e-6);
 * q = R(q*r)/Dk; k = R(R(k*r) * R(1/sqrt(Dk))); g = exp(-exp(A_log) * softplus_bf(R(a + dt_bias)));
 * beta = sigmoid_bf(b). */
static void qo_gdn_qk_prep(const float* xin /* [Dk] conv outputs (post silu) */, int Dk, int is_q, float* out) {
  int NP = Dk / 32;
  float P[32];
  for (int l = 0; l < 32; ++l) {
    float acc = 0.0f;
    for (int i = 0; i < NP; ++i) acc = fmaf(xin[NP * l + i], xin[NP * l + i], acc);
    P[l] = acc;
  }
  float ss = qo_butterfly32(P);
  float r = 1.0f / sqrtf(ss / (float)Dk + 1e-6f);
  float kscale = qo_R(1.0f / sqrtf((float)Dk));
  for (int e = 0; e < Dk; ++e) {
    if (is_q) out[e] = qo_R(xin[e] * r) / (float)Dk;
    else out[e] = qo_R(qo_R(xin[e] * r) * kscale);
  }
}

static inline float qo_conv_tap(const uint16_t* conv_w, const uint16_t* win, int C, int KC, int ch, int t) {
  float acc = 0.0f;
  for (int j = 0; j < KC; ++j) acc = fmaf(qo_bf2f(conv_w[(size_t)ch * KC + j]), qo_bf2f(win[(size_t)(t + j) * C + ch]), acc);
  return acc;
}

/* The elementwise half of gdn_core: qn, kn fp32 [S, Hk, Dk], vn fp32 [S, Hv*Dv], g, beta fp32
 * [S, Hv] (all values bf16-exact except g). */
QO_API int qo_gdn_fused_prep(const uint16_t* win, const uint16_t* conv_w, const uint16_t* a, const uint16_t* b,
                             int ld_ab, const float* A_log, const uint16_t* dt_bias, float* qn, float* kn,
                             float* vn, float* gt, float* bt, int S, int Hk, int Hv, int Dk, int Dv, int KC) {
  if (Dk % 32 != 0 || Hv % Hk != 0 || S < 1) return -1;
  int C = 2 * Hk * Dk + Hv * Dv;
  float* tmp = (float*)malloc(sizeof(float) * Dk);
  for (int t = 0; t < S; ++t) {
    for (int hk = 0; hk < Hk; ++hk) {
      for (int e = 0; e < Dk; ++e) tmp[e] = qo_silu_bf(qo_R(qo_conv_tap(conv_w, win, C, KC, hk * Dk + e, t)));
      qo_gdn_qk_prep(tmp, Dk, 1, qn + ((size_t)t * Hk + hk) * Dk);
      for (int e = 0; e < Dk; ++e) tmp[e] = qo_silu_bf(qo_R(qo_conv_tap(conv_w, win, C, KC, Hk * Dk + hk * Dk + e, t)));
      qo_gdn_qk_prep(tmp, Dk, 0, kn + ((size_t)t * Hk + hk) * Dk);
    }
    for (int cv = 0; cv < Hv * Dv; ++cv)
      vn[(size_t)t * Hv * Dv + cv] = qo_silu_bf(qo_R(qo_conv_tap(conv_w, win, C, KC, 2 * Hk * Dk + cv, t)));
    for (int hv = 0; hv < Hv; ++hv) {
      float A = -qo_expf(A_log[hv]);
      float sp = qo_softplus_bf(qo_R(qo_bf2f(a[(size_t)t * ld_ab + hv]) + qo_bf2f(dt_bias[hv])));
      gt[(size_t)t * Hv + hv] = qo_expf(A * sp);
      bt[(size_t)t * Hv + hv] = qo_sigmoid_bf(qo_bf2f(b[(size_t)t * ld_ab + hv]));
    }
  }
  free(tmp);
  return 0;
}

QO_API int qo_gdn_fused(const uint16_t* win, const uint16_t* conv_w, const uint16_t* a, const uint16_t* b,
                        int ld_ab, const float* A_log, const uint16_t* dt_bias, const float* state_in,
                        float* y, float* state_out, float* state_mid, int S, int Hk, int Hv, int Dk,
                        int Dv, int KC) {
  if (Dk % 32 != 0 || Hv % Hk != 0 || S < 1) return -1;
  float* qn = (float*)malloc(sizeof(float) * (size_t)S * Hk * Dk);
  float* kn = (float*)malloc(sizeof(float) * (size_t)S * Hk * Dk);
  float* vn = (float*)malloc(sizeof(float) * (size_t)S * Hv * Dv);
  float* gt = (float*)malloc(sizeof(float) * (size_t)S * Hv * 2);
  float* bt = gt + (size_t)S * Hv;
  qo_gdn_fused_prep(win, conv_w, a, b, ld_ab, A_log, dt_bias, qn, kn, vn, gt, bt, S, Hk, Hv, Dk, Dv, KC);
  size_t per = (size_t)Hv * Dv * Dk;
#pragma omp parallel for collapse(2) schedule(static)
  for (int hv = 0; hv < Hv; ++hv) {
    for (int dv = 0; dv < Dv; ++dv) {
      int hk = hv / (Hv / Hk);
      float* vf = (float*)malloc(sizeof(float) * (size_t)S * 4);
      float *yf = vf + S, *gg = vf + 2 * S, *bb = vf + 3 * S;
      for (int t = 0; t < S; ++t) {
        vf[t] = vn[(size_t)t * Hv * Dv + (size_t)hv * Dv + dv];
        gg[t] = gt[(size_t)t * Hv + hv];
        bb[t] = bt[(size_t)t * Hv + hv];
      }
      size_t row = ((size_t)hv * Dv + dv) * Dk;
      float* st = state_out + row;
      memcpy(st, state_in + row, sizeof(float) * Dk);
      qo_gdn_row(st, Dk, S, qn + (size_t)hk * Dk, kn + (size_t)hk * Dk, Hk * Dk, vf, 1, gg, bb, 1, yf, 1,
                 state_mid ? state_mid + row : NULL, per);
      for (int t = 0; t < S; ++t) y[((size_t)t * Hv + hv) * Dv + dv] = qo_R(yf[t]);
      free(vf);
    }
  }
  free(qn); free(kn); free(vn); free(gt);
  return 0;
}

/* gdn_norm_gate (gdn_fused.py:114-129): per (token, head) row of Dv:
 *   r = 1/sqrt(sum(y^2)/Dv + eps) (lane-sequential fma + butterfly); xn = R(w * R(y*r));
 *   out = bf16(xn * silu_f32(z)).  y fp32 [S, H, Dv], z bf16 [S, H*Dv] (row stride ld_z). */
QO_API void qo_gdn_norm_gate(const float* y, const uint16_t* z, int ld_z, const uint16_t* w, uint16_t* out,
                             int S, int H, int Dv, float eps) {
  int NP = Dv / 32;
  for (int t = 0; t < S; ++t)
    for (int h = 0; h < H; ++h) {
      const float* yr = y + ((size_t)t * H + h) * Dv;
      float P[32];
      for (int l = 0; l < 32; ++l) {
        float acc = 0.0f;
        for (int i = 0; i < NP; ++i) acc = fmaf(yr[NP * l + i], yr[NP * l + i], acc);
        P[l] = acc;
      }
      float r = 1.0f / sqrtf(qo_butterfly32(P) / (float)Dv + eps);
      for (int e = 0; e < Dv; ++e) {
        float xn = qo_R(qo_bf2f(w[e]) * qo_R(yr[e] * r));
        float zz = qo_bf2f(z[(size_t)t * ld_z + (size_t)h * Dv + e]);
        out[(size_t)t * H * Dv + (size_t)h * Dv + e] = qo_f2bf(xn * qo_silu_f32(zz));
      }
    }
}

/* ------------------------------------------------------------------ two-stage lm_head
 * lm_head2.py:23-29.  Stage 1 is qo_qmv_affine (coarse bf16 logits).  Selection: the topk entries
 * of a row under the total order (value descending, vocab index ascending), with bf16 values
 * compared through the order-preserving 16-bit key below (lm_head2.py:25 argpartition leaves ties
 * unspecified; this order resolves them).  Stage 2: fine = bf16(dot(W[idx], h)) with the dot
 * ordered as: lane l = 0..31 takes the 8-element chunks c = l, l+32, ... ascending, fmaf over the
 * chunk's elements ascending from 0, then the 32 lane sums are butterflied. */
static inline uint32_t qo_bf16_key(uint16_t b) { return (b & 0x8000u) ? (uint32_t)(~b & 0xFFFFu) : (uint32_t)(b | 0x8000u); }

typedef struct { uint32_t key; int32_t idx; } qo_cand;
static int qo_cand_cmp(const void* a, const void* b) {
  const qo_cand* x = (const qo_cand*)a; const qo_cand* y = (const qo_cand*)b;
  if (x->key != y->key) return x->key > y->key ? -1 : 1;
  return x->idx < y->idx ? -1 : (x->idx > y->idx ? 1 : 0);
}

QO_API int qo_topk_bf16(const uint16_t* vals, int M, int V, int ld, int k, int32_t* idx_out) {
  if (k < 1 || k > V) return -1;
  for (int m = 0; m < M; ++m) {
    qo_cand* c = (qo_cand*)malloc(sizeof(qo_cand) * (size_t)V);
    for (int i = 0; i < V; ++i) { c[i].key = qo_bf16_key(vals[(size_t)m * ld + i]); c[i].idx = i; }
    qsort(c, (size_t)V, sizeof(qo_cand), qo_cand_cmp);
    for (int j = 0; j < k; ++j) idx_out[(size_t)m * k + j] = c[j].idx;
    free(c);
  }
  return 0;
}

QO_API float qo_dot_bf16(const uint16_t* w, const uint16_t* h, int K) {
  float P[32];
  for (int l = 0; l < 32; ++l) {
    float acc = 0.0f;
    for (int c = l; c < K / 8; c += 32)
      for (int e = 0; e < 8; ++e) acc = fmaf(qo_bf2f(w[8 * c + e]), qo_bf2f(h[8 * c + e]), acc);
    P[l] = acc;
  }
  return qo_butterfly32(P);
}

/* fine[m][j] = bf16(dot(W[idx[m][j]], h[m])) and argmax[m] = the idx with the largest fine value
 * (ties: lowest vocab index), W bf16 [V, K]. */
QO_API int qo_rescore_bf16(const uint16_t* W, const uint16_t* h, const int32_t* idx, int M, int k, int K,
                           uint16_t* fine, int32_t* amax) {
  if (K % 256 != 0) return -1;
  for (int m = 0; m < M; ++m) {
    uint32_t bk = 0; int32_t bi = -1;
    for (int j = 0; j < k; ++j) {
      int32_t v = idx[(size_t)m * k + j];
      uint16_t f = qo_f2bf(qo_dot_bf16(W + (size_t)v * K, h + (size_t)m * K, K));
      fine[(size_t)m * k + j] = f;
      uint32_t key = qo_bf16_key(f);
      if (bi < 0 || key > bk || (key == bk && v < bi)) { bk = key; bi = v; }
    }
    amax[m] = bi;
  }
  return 0;
}

/* argmax over a bf16 row (ties: lowest index). */
QO_API int qo_argmax_bf16(const uint16_t* vals, int M, int V, int ld, int32_t* out) {
  for (int m = 0; m < M; ++m) {
    uint32_t bk = 0; int32_t bi = -1;
    for (int i = 0; i < V; ++i) {
      uint32_t key = qo_bf16_key(vals[(size_t)m * ld + i]);
      if (bi < 0 || key > bk) { bk = key; bi = i; }
    }
    out[m] = bi;
  }
  return 0;
}

/* ------------------------------------------------------------------ decoder ops
 * Sums of squares for RMS norms have two fixed trees:
 *   wide (D % 1024 == 0): 32-element contiguous chunk partials (fmaf from 0), butterfly over each
 *        block of 32 chunks, blocks added in order (the qmv reduction tree);
 *   head (D % 32 == 0, D <= 1024): lane l sums elements [l*D/32, (l+1)*D/32) (fmaf from 0), butterfly.
 * RMSNorm (mx.fast.rms_norm, as restated in gdn_fused.py:123-126): r = 1/sqrt(ss/D + eps),
 * y = R(w * R(x * r)). */
static float qo_sumsq_wide(const float* x, int D) {
  float y = 0.0f;
  for (int i = 0; i < D / 1024; ++i) {
    float P[32];
    for (int l = 0; l < 32; ++l) {
      float acc = 0.0f;
      for (int e = 0; e < 32; ++e) { float v = x[1024 * i + 32 * l + e]; acc = fmaf(v, v, acc); }
      P[l] = acc;
    }
    float B = qo_butterfly32(P);
    y = (i == 0) ? B : y + B;
  }
  return y;
}
static float qo_sumsq_head(const float* x, int D) {
  int NP = D / 32;
  float P[32];
  for (int l = 0; l < 32; ++l) {
    float acc = 0.0f;
    for (int e = 0; e < NP; ++e) { float v = x[NP * l + e]; acc = fmaf(v, v, acc); }
    P[l] = acc;
  }
  return qo_butterfly32(P);
}

/* x bf16 [M, D] (row stride ld_x) -> out bf16 [M, D] (row stride ld_o); wide tree if D % 1024 == 0
 * else head tree.  w bf16 [D]. */
QO_API void qo_rmsnorm(const uint16_t* x, int ld_x, const uint16_t* w, float eps, uint16_t* out, int ld_o, int M, int D) {
  float* xf = (float*)malloc(sizeof(float) * D);
  for (int m = 0; m < M; ++m) {
    for (int e = 0; e < D; ++e) xf[e] = qo_bf2f(x[(size_t)m * ld_x + e]);
    float ss = (D % 1024 == 0) ? qo_sumsq_wide(xf, D) : qo_sumsq_head(xf, D);
    float r = 1.0f / sqrtf(ss / (float)D + eps);
    for (int e = 0; e < D; ++e) out[(size_t)m * ld_o + e] = qo_f2bf(qo_bf2f(w[e]) * qo_R(xf[e] * r));
  }
  free(xf);
}

/* Quantized embedding gather (nn.QuantizedEmbedding): out[t] = bf16(fma(s, q, b)) of row tok[t]. */
QO_API void qo_embed(const int32_t* tok, int T, const uint32_t* wq, const uint16_t* sc, const uint16_t* bi, int D,
                     uint16_t* out) {
  int G = D / 64;
  for (int t = 0; t < T; ++t) {
    size_t r = (size_t)tok[t];
    for (int e = 0; e < D; ++e) {
      uint32_t q = (wq[(r * D + e) / 8] >> (4 * (e % 8))) & 15u;
      out[(size_t)t * D + e] = qo_f2bf(fmaf(qo_bf2f(sc[r * G + e / 64]), (float)q, qo_bf2f(bi[r * G + e / 64])));
    }
  }
}

/* NVFP4 embedding rows: bf16(e2m1(q) * e4m3(scale)), the product exact in fp32. */
QO_API void qo_embed_nvfp4(const int32_t* tok, int T, const uint32_t* wq, const uint8_t* sc, int D, uint16_t* out) {
  for (int t = 0; t < T; ++t) {
    size_t r = (size_t)tok[t];
    for (int e = 0; e < D; ++e) {
      uint32_t q = (wq[(r * D + e) / 8] >> (4 * (e % 8))) & 15u;
      out[(size_t)t * D + e] = qo_f2bf(qo_e2m1(q) * qo_e4m3(sc[r * (D / 16) + e / 16]));
    }
  }
}

/* Gated attention input prep (hf:modeling_qwen3_5.py:647-668 structure; MLX-style rounding):
 * for token s of the S rows of qkv (row stride ld): q heads [nq][2*Dh] (query then gate),
 * k [nkv][Dh], v [nkv][Dh] after the q part.  q, k: per-head RMS norm (head tree) with weights
 * qn_w / kn_w, then partial rotate-half RoPE on the first R dims with cos/sin tables [pos][R/2]:
 *   o_i = R(x_i*c - x_{i+R/2}*s),  o_{i+R/2} = R(x_{i+R/2}*c + x_i*s)   (products rounded, then sum).
 * Outputs: qo bf16 [S, nq, Dh], gate bf16 [S, nq, Dh], k/v written into the caches
 * kc/vc [nkv, max_pos, Dh] at position pos0 + s. */
QO_API void qo_attn_prep(const uint16_t* qkv, int ld, int S, int nq, int nkv, int Dh, int R, const uint16_t* qn_w,
                         const uint16_t* kn_w, float eps, const float* cos_t, const float* sin_t, int pos0,
                         uint16_t* qo, uint16_t* gate, uint16_t* kc, uint16_t* vc, int max_pos) {
  float* x = (float*)malloc(sizeof(float) * Dh);
  uint16_t* tmp = (uint16_t*)malloc(sizeof(uint16_t) * Dh);
  int half = R / 2;
  for (int s = 0; s < S; ++s) {
    const uint16_t* row = qkv + (size_t)s * ld;
    int pos = pos0 + s;
    const float* c = cos_t + (size_t)pos * half;
    const float* sn = sin_t + (size_t)pos * half;
    for (int hh = 0; hh < nq + nkv; ++hh) {
      int isq = hh < nq;
      const uint16_t* src = isq ? row + (size_t)hh * 2 * Dh : row + (size_t)nq * 2 * Dh + (size_t)(hh - nq) * Dh;
      for (int e = 0; e < Dh; ++e) x[e] = qo_bf2f(src[e]);
      float r = 1.0f / sqrtf(qo_sumsq_head(x, Dh) / (float)Dh + eps);
      const uint16_t* w = isq ? qn_w : kn_w;
      for (int e = 0; e < Dh; ++e) x[e] = qo_bf2f(qo_f2bf(qo_bf2f(w[e]) * qo_R(x[e] * r)));
      for (int e = 0; e < Dh; ++e) tmp[e] = qo_f2bf(x[e]);
      for (int i = 0; i < half; ++i) {
        float a = x[i] * c[i], b = x[i + half] * sn[i];
        float a2 = x[i + half] * c[i], b2 = x[i] * sn[i];
        tmp[i] = qo_f2bf(a - b);
        tmp[i + half] = qo_f2bf(a2 + b2);
      }
      if (isq) {
        memcpy(qo + ((size_t)s * nq + hh) * Dh, tmp, sizeof(uint16_t) * Dh);
        memcpy(gate + ((size_t)s * nq + hh) * Dh, src + Dh, sizeof(uint16_t) * Dh);
      } else {
        int kh = hh - nq;
        memcpy(kc + ((size_t)kh * max_pos + pos) * Dh, tmp, sizeof(uint16_t) * Dh);
        memcpy(vc + ((size_t)kh * max_pos + pos) * Dh, row + (size_t)nq * 2 * Dh + (size_t)nkv * Dh + (size_t)kh * Dh,
               sizeof(uint16_t) * Dh);
      }
    }
  }
  free(x); free(tmp);
}

/* Decode attention with the sigmoid output gate.  Query s (position pos0 + s) of head h attends
 * keys 0..pos0+s of kv head h / (nq/nkv).  Keys are dealt to NW = 8 splits (key j -> split j % 8):
 *   score_j = dot(q, k_j) (head tree: lane l takes Dh/32 contiguous dims, fmaf, butterfly) * Dh^-1/2
 *   per split w: m_w = max score; e_j = exp(score_j - m_w); den_w = sum e_j; num_w[d] = sum
 *   fma(e_j, v_jd, .) (keys ascending, from 0);
 *   M = max m_w; c_w = exp(m_w - M); den = sum_w fma(c_w, den_w, .); num_d likewise (w ascending);
 *   o_d = R(num_d / den); out_d = R(o_d * sigmoid_bf(gate_d)). */
QO_API void qo_attention(const uint16_t* q, const uint16_t* gate, const uint16_t* kc, const uint16_t* vc, int max_pos,
                         int S, int nq, int nkv, int Dh, int pos0, uint16_t* out) {
  const int NW = 8;
  float scale = 1.0f / sqrtf((float)Dh);
  int grp = nq / nkv;
  float* qf = (float*)malloc(sizeof(float) * Dh);
  float* kf = (float*)malloc(sizeof(float) * Dh);
  float* num = (float*)malloc(sizeof(float) * NW * Dh);
  float* acc = (float*)malloc(sizeof(float) * Dh);
  for (int s = 0; s < S; ++s)
    for (int h = 0; h < nq; ++h) {
      int L = pos0 + s + 1, kh = h / grp;
      for (int e = 0; e < Dh; ++e) qf[e] = qo_bf2f(q[((size_t)s * nq + h) * Dh + e]);
      float* sc = (float*)malloc(sizeof(float) * L);
      for (int j = 0; j < L; ++j) {
        const uint16_t* kr = kc + ((size_t)kh * max_pos + j) * Dh;
        int NP = Dh / 32;
        float P[32];
        for (int l = 0; l < 32; ++l) {
          float a = 0.0f;
          for (int e = 0; e < NP; ++e) a = fmaf(qf[NP * l + e], qo_bf2f(kr[NP * l + e]), a);
          P[l] = a;
        }
        sc[j] = qo_butterfly32(P) * scale;
      }
      float mw[8], den[8];
      int nonempty[8];
      for (int w = 0; w < NW; ++w) {
        nonempty[w] = w < L;
        mw[w] = -INFINITY; den[w] = 0.0f;
        for (int d = 0; d < Dh; ++d) num[w * Dh + d] = 0.0f;
        if (!nonempty[w]) continue;
        for (int j = w; j < L; j += NW) mw[w] = sc[j] > mw[w] ? sc[j] : mw[w];
        for (int j = w; j < L; j += NW) {
          float e = qo_expf(sc[j] - mw[w]);
          den[w] = den[w] + e;
          const uint16_t* vr = vc + ((size_t)kh * max_pos + j) * Dh;
          for (int d = 0; d < Dh; ++d) num[w * Dh + d] = fmaf(e, qo_bf2f(vr[d]), num[w * Dh + d]);
        }
      }
      float M = -INFINITY;
      for (int w = 0; w < NW; ++w) if (nonempty[w] && mw[w] > M) M = mw[w];
      float dsum = 0.0f;
      for (int d = 0; d < Dh; ++d) acc[d] = 0.0f;
      for (int w = 0; w < NW; ++w) {
        if (!nonempty[w]) continue;
        float cw = qo_expf(mw[w] - M);
        dsum = fmaf(cw, den[w], dsum);
        for (int d = 0; d < Dh; ++d) acc[d] = fmaf(cw, num[w * Dh + d], acc[d]);
      }
      for (int d = 0; d < Dh; ++d) {
        float o = qo_R(acc[d] / dsum);
        float gt = qo_bf2f(gate[((size_t)s * nq + h) * Dh + d]);
        out[(size_t)s * nq * Dh + (size_t)h * Dh + d] = qo_f2bf(o * qo_sigmoid_bf(gt));
      }
      free(sc);
    }
  free(qf); free(kf); free(num); free(acc);
}

/* Probability the draft head gives its argmax token (mtp.py:222-223, softmax(logits).max()) in the
 * reduction order of draft_prob_kernel: 1024 strided sequential partial sums of exp(l_j - l_token),
 * the xor butterfly over each 32 partials, the 32 group sums in order; 1 / total. */
QO_API float qo_draft_prob(const uint16_t* logits, int V, int token) {
  float part[1024], grp[32];
  float lmax = qo_bf2f(logits[token]);
  for (int t = 0; t < 1024; ++t) {
    float s = 0.0f;
    for (int j = t; j < V; j += 1024) s = s + qo_expf(qo_bf2f(logits[j]) - lmax);
    part[t] = s;
  }
  for (int w = 0; w < 32; ++w) {
    float v[32];
    for (int l = 0; l < 32; ++l) v[l] = part[32 * w + l];
    for (int d = 16; d >= 1; d >>= 1) {
      float nv[32];
      for (int l = 0; l < 32; ++l) nv[l] = v[l] + v[l ^ d];
      for (int l = 0; l < 32; ++l) v[l] = nv[l];
    }
    grp[w] = v[0];
  }
  float tot = grp[0];
  for (int w = 1; w < 32; ++w) tot = tot + grp[w];
  return 1.0f / tot;
}

/* SwiGLU (mlx-lm MLP: down(silu(gate(x)) * up(x))): act = R(silu_bf(g) * u); gu bf16 [S, 2I]
 * (gate columns then up columns, row stride ld) -> out bf16 [S, I]. */
QO_API void qo_swiglu(const uint16_t* gu, int ld, int S, int I, uint16_t* out) {
  for (int s = 0; s < S; ++s)
    for (int i = 0; i < I; ++i) {
      float g = qo_bf2f(gu[(size_t)s * ld + i]), u = qo_bf2f(gu[(size_t)s * ld + I + i]);
      out[(size_t)s * I + i] = qo_f2bf(qo_silu_bf(g) * u);
    }
}

/* bf16 residual add: out = R(a + b). */
QO_API void qo_add_bf16(const uint16_t* a, const uint16_t* b, uint16_t* out, long n) {
  for (long i = 0; i < n; ++i) out[i] = qo_f2bf(qo_bf2f(a[i]) + qo_bf2f(b[i]));
}

/* ------------------------------------------------------------------ MXFP4 / NVFP4 MoE
 * Weight format (experiments/deepseek_moe/kernels.py:3-5, qmv_kernel.py:7-9): uint32 [N, K/8],
 * 8 e2m1 nibbles per word, low nibble = lowest k; scales uint8 [N, K/G]:
 *   fmt 0 MXFP4: G = 32, e8m0 scale 2^(s-127)          (kernels.py:31-32 e8m0_scale)
 *   fmt 1 NVFP4: G = 16, e4m3 scale, sign bit ignored   (qmv_kernel.py:26-28 e4m3_scale)
 *
 * Quantizers.  The reference never quantizes (its bench draws random bits, bench_moe.py:24-31),
 * so the quantizer is this library's own, written from the OCP Microscaling spec v1.0 (sec. 6.3):
 *   MXFP4: s = clamp(floor(log2(amax)) - 2 + 127, 0, 254) (amax = 0 -> s = 0), v = w * 2^(127-s);
 *   NVFP4: scale = e4m3_rne(amax / 6) saturated to 448, v = w / scale (scale 0 -> all codes 0);
 *   code = e2m1 round-to-nearest-even of v, saturated at 6; a zero magnitude is coded +0.
 * NaN / Inf weights are not supported. */
static inline uint32_t qo_e2m1_code(float v) {
  float a = fabsf(v);
  uint32_t c = 0;
  if (a > 0.25f) c = 1;
  if (a >= 0.75f) c = 2;
  if (a > 1.25f) c = 3;
  if (a >= 1.75f) c = 4;
  if (a > 2.5f) c = 5;
  if (a >= 3.5f) c = 6;
  if (a > 5.0f) c = 7;
  if (c && signbit(v)) c |= 8u;
  return c;
}
static inline uint32_t qo_e4m3_code(float f) { /* f >= 0 */
  if (!(f > 0.0f)) return 0;
  if (f > 448.0f) return 0x7E;
  int e = ilogbf(f);
  if (e < -6) return (uint32_t)rintf(f * 512.0f); /* subnormal grid 2^-9 (8 -> code 8 = 2^-6) */
  uint32_t m = (uint32_t)rintf((ldexpf(f, -e) - 1.0f) * 8.0f);
  if (m == 8) { m = 0; e += 1; }
  uint32_t c = ((uint32_t)(e + 7) << 3) | m;
  return c > 0x7E ? 0x7E : c;
}
QO_API int qo_quantize_fp4(int fmt, const uint16_t* w, long N, int K, uint32_t* wq, uint8_t* sc) {
  const int G = fmt == 0 ? 32 : 16;
  if ((fmt != 0 && fmt != 1) || K % G) return -1;
  for (long n = 0; n < N; ++n)
    for (int g = 0; g < K / G; ++g) {
      const uint16_t* wr = w + n * K + (long)g * G;
      float amax = 0.0f;
      for (int i = 0; i < G; ++i) amax = fmaxf(amax, fabsf(qo_bf2f(wr[i])));
      uint32_t s;
      float mul = 0.0f, div = 0.0f;
      if (fmt == 0) {
        int se = amax > 0.0f ? ilogbf(amax) - 2 + 127 : 0;
        s = (uint32_t)(se < 0 ? 0 : se > 254 ? 254 : se);
        mul = s == 0 ? qo_asf(0x7F000000u) : qo_asf((254u - s) << 23); /* 2^(127-s) */
      } else {
        s = qo_e4m3_code(amax / 6.0f);
        div = qo_e4m3(s);
      }
      sc[n * (K / G) + g] = (uint8_t)s;
      for (int i = 0; i < G; i += 8) {
        uint32_t word = 0;
        for (int j = 0; j < 8; ++j) {
          float x = qo_bf2f(wr[i + j]);
          float v = fmt == 0 ? x * mul : (div > 0.0f ? x / div : 0.0f);
          word |= qo_e2m1_code(v) << (4 * j);
        }
        wq[n * (K / 8) + (g * G + i) / 8] = word;
      }
    }
  return 0;
}

/* Dequantize one row of K weights (exact in fp32). */
static void qo_fp4_row(int fmt, const uint32_t* wrow, const uint8_t* srow, int K, float* out) {
  const int G = fmt == 0 ? 32 : 16;
  for (int k = 0; k < K; ++k) {
    float s = fmt == 0 ? qo_e8m0(srow[k / G]) : qo_e4m3(srow[k / G]);
    out[k] = qo_e2m1((wrow[k / 8] >> (4 * (k % 8))) & 15u) * s;
  }
}
QO_API void qo_dequant_fp4(int fmt, const uint32_t* wq, const uint8_t* sc, long N, int K, float* out) {
  const int G = fmt == 0 ? 32 : 16;
  for (long n = 0; n < N; ++n) qo_fp4_row(fmt, wq + n * (K / 8), sc + n * (K / G), K, out + n * K);
}

/* Router: softmax over E routed logits, top-k, renormalised over the chosen k (DeepSeek
 * norm_topk_prob), times routed_scale; then n_shared shared experts (ids E .. E+n_shared-1) with
 * score 1.0, as bench_moe.py:41-42 builds idx / scores.  The renormalised weight of expert i is
 * exp(l_i - l_max) / sum_{j in topk} exp(l_j - l_max): the full softmax denominator cancels, so it
 * is computed that way.  Order of selection: larger logit first, ties to the lower expert id; a NaN
 * logit ranks below every number.  Fixed fp32 sequence: d_j = l_j - l_top (j in selection
 * order), e_j = exp(d_j), sum = ((e_0 + e_1) + e_2) ..., w_j = (e_j / sum) * routed_scale. */
static inline uint32_t qo_logit_key(float f) {
  if (f != f) return 0;
  uint32_t u = qo_asu(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
QO_API void qo_moe_route(const float* logits, int T, int E, int top_k, int n_shared, float routed_scale,
                         int32_t* idx, float* scores) {
  const int S = top_k + n_shared;
  for (int t = 0; t < T; ++t) {
    const float* l = logits + (long)t * E;
    int32_t* id = idx + (long)t * S;
    float* sc = scores + (long)t * S;
    for (int j = 0; j < top_k; ++j) {
      int best = -1;
      uint32_t bk = 0;
      for (int e = 0; e < E; ++e) {
        int taken = 0;
        for (int q = 0; q < j; ++q) taken |= id[q] == e;
        if (taken) continue;
        uint32_t k = qo_logit_key(l[e]);
        if (best < 0 || k > bk) { best = e; bk = k; }
      }
      id[j] = best;
    }
    float ex[64];
    float sum = 0.0f;
    for (int j = 0; j < top_k; ++j) {
      ex[j] = qo_expf(l[id[j]] - l[id[0]]);
      sum = j == 0 ? ex[0] : sum + ex[j];
    }
    for (int j = 0; j < top_k; ++j) sc[j] = (ex[j] / sum) * routed_scale;
    for (int j = 0; j < n_shared; ++j) { id[top_k + j] = E + j; sc[top_k + j] = 1.0f; }
  }
}

/* Expert FFN, restating experiments/deepseek_moe/kernels.py:35-107 for T tokens:
 *   h[t,j,i] = fp32( silu(min(g, L)) * clamp(u, -L, L) ),  g = Wg[e] x_t, u = Wu[e] x_t  (e = idx[t,j])
 *   y[t,n]   = sum_j scores[t,j] * (Wd[e] h[t,j])[n]
 * The dots and the weighted sum are evaluated in double (more accurate than the fp32 lane sums of
 * the reference); h is rounded to fp32 as the reference stores it (kernels.py:146).  limit = +inf
 * disables the clamp.  y_f32 gets the sum rounded to fp32, y_bf16 its RNE bf16.
 * Weights: wg, wu [E, I, H/8] / scales [E, I, H/G]; wd [E, H, I/8] / [E, H, I/G]. */
QO_API int qo_moe(int fmt, const uint16_t* x, const uint32_t* wg, const uint8_t* sg, const uint32_t* wu,
                  const uint8_t* su, const uint32_t* wd, const uint8_t* sd, const int32_t* idx, const float* scores,
                  int T, int S, int E, int H, int I, float limit, float* y_f32, uint16_t* y_bf16) {
  const int G = fmt == 0 ? 32 : 16;
  if (H % G || I % G || H % 8 || I % 8 || H > 8192 || I > 8192) return -1;
  for (long i = 0; i < (long)T * S; ++i)
    if (idx[i] < 0 || idx[i] >= E) return -2;
  double* yacc = (double*)calloc((size_t)T * H, sizeof(double));
  double* xd = (double*)malloc((size_t)T * H * sizeof(double));
  int* list = (int*)malloc((size_t)T * S * sizeof(int));
  float* h = (float*)malloc((size_t)T * S * I * sizeof(float));
  for (long i = 0; i < (long)T * H; ++i) xd[i] = qo_bf2f(x[i]);
  for (int e = 0; e < E; ++e) {
    int n = 0;
    for (int i = 0; i < T * S; ++i)
      if (idx[i] == e) list[n++] = i;
    if (!n) continue;
#pragma omp parallel for schedule(static)
    for (int r = 0; r < I; ++r) {
      float rg[8192], ru[8192];
      qo_fp4_row(fmt, wg + ((long)e * I + r) * (H / 8), sg + ((long)e * I + r) * (H / G), H, rg);
      qo_fp4_row(fmt, wu + ((long)e * I + r) * (H / 8), su + ((long)e * I + r) * (H / G), H, ru);
      for (int q = 0; q < n; ++q) {
        const double* xt = xd + (long)(list[q] / S) * H;
        double g = 0.0, u = 0.0;
        for (int k = 0; k < H; ++k) { g += rg[k] * xt[k]; u += ru[k] * xt[k]; }
        g = g < limit ? g : limit;
        u = u < -limit ? -limit : (u > limit ? limit : u);
        h[(long)q * I + r] = (float)(g / (1.0 + exp(-g)) * u);
      }
    }
#pragma omp parallel for schedule(static)
    for (int r = 0; r < H; ++r) {
      float rd[8192];
      qo_fp4_row(fmt, wd + ((long)e * H + r) * (I / 8), sd + ((long)e * H + r) * (I / G), I, rd);
      for (int q = 0; q < n; ++q) {
        double a = 0.0;
        const float* hq = h + (long)q * I;
        for (int k = 0; k < I; ++k) a += (double)rd[k] * hq[k];
        yacc[(long)(list[q] / S) * H + r] += (double)scores[list[q]] * a;
      }
    }
  }
  for (long i = 0; i < (long)T * H; ++i) {
    float f = (float)yacc[i];
    if (y_f32) y_f32[i] = f;
    if (y_bf16) y_bf16[i] = qo_f2bf(f);
  }
  free(yacc); free(xd); free(list); free(h);
  return 0;
}

/* ------------------------------------------------------------------ speculative sampling (T > 0)
 * engine.py:91-152 (Engine._dist / _sample_first / _verify) restated with a fixed operation order
 * and a counter-based generator, so the CUDA sampler (csrc/sample.cu) makes the same decisions.
 *
 * Random numbers: Philox4x32-10 (Salmon, Moraes, Dror, Shaw, "Parallel random numbers: as easy as
 * 1, 2, 3", SC 2011): 10 rounds of two 32x32->64 multiplies, Weyl key schedule.  A uniform is the
 * top 24 bits of output word 0 times 2^-24 (exact in fp32, in [0, 1)).  Counter = (call counter,
 * row, use (0: accept test, 1: categorical draw), 0), key = the 64-bit seed. */
QO_API void qo_philox4x32_10(const uint32_t* ctr_in, const uint32_t* key_in, uint32_t* out) {
  uint32_t c[4] = {ctr_in[0], ctr_in[1], ctr_in[2], ctr_in[3]}, k0 = key_in[0], k1 = key_in[1];
  for (int r = 0; r < 10; ++r) {
    if (r > 0) { k0 += 0x9E3779B9u; k1 += 0xBB67AE85u; }
    const uint64_t p0 = (uint64_t)0xD2511F53u * c[0], p1 = (uint64_t)0xCD9E8D57u * c[2];
    const uint32_t hi0 = (uint32_t)(p0 >> 32), lo0 = (uint32_t)p0, hi1 = (uint32_t)(p1 >> 32), lo1 = (uint32_t)p1;
    const uint32_t n0 = hi1 ^ c[1] ^ k0, n2 = hi0 ^ c[3] ^ k1;
    c[0] = n0; c[1] = lo1; c[2] = n2; c[3] = lo0;
  }
  memcpy(out, c, sizeof c);
}
static float qo_uniform(uint32_t seed_lo, uint32_t seed_hi, uint32_t ctr, uint32_t row, uint32_t use) {
  const uint32_t c[4] = {ctr, row, use, 0u}, k[2] = {seed_lo, seed_hi};
  uint32_t o[4];
  qo_philox4x32_10(c, k, o);
  return (float)(o[0] >> 8) * (1.0f / 16777216.0f);
}

typedef struct { float l; int32_t i; } qo_scand;
/* candidates ordered by exact logit descending, then vocabulary index ascending */
static int qo_scand_cmp(const void* a, const void* b) {
  const qo_scand *x = (const qo_scand*)a, *y = (const qo_scand*)b;
  if (x->l > y->l) return -1;
  if (x->l < y->l) return 1;
  return (x->i < y->i) ? -1 : (x->i > y->i);
}

/* Engine._dist (engine.py:92-108) over one row's K candidates (the two-stage head leaves every
 * other logit at -inf): temperature, top_k, log-softmax, top_p on the sorted exclusive cumsum,
 * min_p, renormalisation.  Leaves the kept candidates sorted in c[0..n) and p[0..n). */
static int qo_dist(const int32_t* idx, const uint16_t* fine, int K, float T, int top_k, float top_p, float min_p,
                   int V, qo_scand* c, float* p) {
  for (int j = 0; j < K; ++j) { c[j].l = qo_bf2f(fine[j]); c[j].i = idx[j]; }
  qsort(c, (size_t)K, sizeof(qo_scand), qo_scand_cmp);
  int n = K;
  if (top_k > 0 && top_k < V && top_k < n) n = top_k;
  float z[2048], lp[2048];
  for (int j = 0; j < n; ++j) z[j] = c[j].l / T;
  const float m = z[0];
  float s = 0.0f;
  for (int j = 0; j < n; ++j) s = s + qo_expf(z[j] - m);
  const float L = m + qo_logf(s);
  for (int j = 0; j < n; ++j) lp[j] = z[j] - L;
  if (top_p < 1.0f) {
    float acc = 0.0f;
    int np_ = n;
    for (int j = 0; j < n; ++j) {
      const float q = qo_expf(lp[j]);
      const float inc = acc + q;
      if (!(inc - q < top_p)) { np_ = j; break; }
      acc = inc;
    }
    n = np_;
  }
  if (min_p > 0.0f) {
    const float thr = lp[0] + qo_logf(min_p);
    int nm = n;
    for (int j = 0; j < n; ++j)
      if (!(lp[j] >= thr)) { nm = j; break; }
    n = nm;
  }
  float s2 = 0.0f;
  for (int j = 0; j < n; ++j) { p[j] = qo_expf(lp[j] - lp[0]); s2 = s2 + p[j]; }
  for (int j = 0; j < n; ++j) p[j] = p[j] / s2;
  return n;
}

/* categorical draw by inverse CDF over the kept candidates, skipping vocabulary id `excl` */
static int32_t qo_draw(const qo_scand* c, const float* p, int n, int32_t excl, float u) {
  float tot = 0.0f;
  for (int j = 0; j < n; ++j)
    if (c[j].i != excl) tot = tot + p[j];
  const float r = u * tot;
  float acc = 0.0f;
  int32_t last = c[0].i;
  for (int j = 0; j < n; ++j) {
    if (c[j].i == excl) continue;
    acc = acc + p[j];
    last = c[j].i;
    if (acc > r) return c[j].i;
  }
  return last;
}

/* mode verify (first_row < 0): rows 0..k of [*, ld] candidates against drafts[0..k) (engine.py:
 * 121-152): accept draft i with probability p_i(d_i), else draw from p_i without d_i and stop; all
 * accepted -> draw the bonus token from row k.  Writes the emitted tokens to out (n_acc + 1 of
 * them) and returns n_acc.  Mode first (first_row >= 0, engine.py:110-115): one draw from that row
 * into out[0] (its uniform uses counter row 0, wherever the row sits); returns 0.  K <= 2048; T > 0. */
QO_API int qo_sample(const int32_t* idx, const uint16_t* fine, int K, int ld, const int32_t* drafts, int k,
                     int first_row, float T, int top_k, float top_p, float min_p, int V, uint32_t seed_lo,
                     uint32_t seed_hi, uint32_t ctr, int32_t* out) {
  if (K < 1 || K > 2048 || !(T > 0.0f)) return -1;
  qo_scand c[2048];
  float p[2048];
  if (first_row >= 0) {
    const int n = qo_dist(idx + (size_t)first_row * ld, fine + (size_t)first_row * ld, K, T, top_k, top_p, min_p,
                          V, c, p);
    out[0] = qo_draw(c, p, n, -1, qo_uniform(seed_lo, seed_hi, ctr, 0u, 1u));  /* counter row 0 */
    return 0;
  }
  for (int i = 0; i <= k; ++i) {
    const int n = qo_dist(idx + (size_t)i * ld, fine + (size_t)i * ld, K, T, top_k, top_p, min_p, V, c, p);
    if (i == k) {
      out[k] = qo_draw(c, p, n, -1, qo_uniform(seed_lo, seed_hi, ctr, (uint32_t)k, 1u));
      return k;
    }
    float pd = 0.0f;
    for (int j = 0; j < n; ++j)
      if (c[j].i == drafts[i]) pd = p[j];
    if (qo_uniform(seed_lo, seed_hi, ctr, (uint32_t)i, 0u) < pd) {
      out[i] = drafts[i];
      continue;
    }
    out[i] = qo_draw(c, p, n, drafts[i], qo_uniform(seed_lo, seed_hi, ctr, (uint32_t)i, 1u));
    return i;
  }
  return k;
}

/* Engine._dist of one row for tests: the kept candidates (sorted) and their probabilities; returns n. */
QO_API int qo_sample_dist(const int32_t* idx, const uint16_t* fine, int K, float T, int top_k, float top_p,
                          float min_p, int V, int32_t* out_idx, float* out_p) {
  if (K < 1 || K > 2048 || !(T > 0.0f)) return -1;
  qo_scand c[2048];
  float p[2048];
  const int n = qo_dist(idx, fine, K, T, top_k, top_p, min_p, V, c, p);
  for (int j = 0; j < n; ++j) { out_idx[j] = c[j].i; out_p[j] = p[j]; }
  return n;
}
