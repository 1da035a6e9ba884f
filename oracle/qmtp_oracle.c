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
 * y[m,n] = sum_k x[m,k] * (s[n,k/64] * q[n,k] + b[n,k/64]), K % 1024 == 0.
 * Reference op: MLX quantized_matmul(x, w, s, b, transpose=True, group_size=64, bits=4) and the
 * multi-row GEMV of qmv_kernel.py:31-75 (same weight layout; that kernel is the NVFP4 variant).
 *
 * Exact sequence.  K is cut into chunks of 32 (c = k/32); block i = chunks 32i..32i+31.
 *   x side, per (m, c):  Xe = sum_{j even} x_j, Xo = sum_{j odd} x_j  (sequential, j ascending),
 *                        Ce = 2048*Xe, Co = 128*Xo, Xc = Xe + Xo.
 *   weight side: nibble j of the chunk is read as f_j = 2048 + q_j (j even) or 128 + q_j (j odd),
 *                both exact floats (the kernel builds them with one AND/OR on the shifted word).
 *   ae = -Ce, ao = -Co; for j = 0,2,..,30: ae = fma(f_j, x_j, ae); ao = fma(f_j+1, x_j+1, ao).
 *   T = ae + ao  (= sum q_j x_j up to rounding);  P_c = fma(b_g, Xc, s_g * T), g = c/2.
 *   B_i = butterfly32(P_{32i..32i+31});  y = ((B_0 + B_1) + B_2) + ...;  out = bf16(y). */

typedef struct { float ce, co, xc; } qo_xchunk;

static void qo_affine_xprep(const uint16_t* x, int K, float* xf, qo_xchunk* xc) {
  for (int k = 0; k < K; ++k) xf[k] = qo_bf2f(x[k]);
  for (int c = 0; c < K / 32; ++c) {
    const float* v = xf + 32 * c;
    float xe = 0.0f, xo = 0.0f;
    for (int j = 0; j < 32; j += 2) { xe = xe + v[j]; xo = xo + v[j + 1]; }
    xc[c].ce = 2048.0f * xe;
    xc[c].co = 128.0f * xo;
    xc[c].xc = xe + xo;
  }
}

static float qo_affine_row(const float* xf, const qo_xchunk* xc, const uint32_t* wrow,
                           const uint16_t* srow, const uint16_t* brow, int K) {
  int NC = K / 32;
  float y = 0.0f;
  for (int i = 0; i < NC / 32; ++i) {
    float P[32];
    for (int l = 0; l < 32; ++l) {
      int c = 32 * i + l;
      const float* v = xf + 32 * c;
      float ae = -xc[c].ce, ao = -xc[c].co;
      for (int wd = 0; wd < 4; ++wd) {
        uint32_t w = wrow[4 * c + wd];
        for (int jj = 0; jj < 8; jj += 2) {
          float fe = 2048.0f + (float)((w >> (4 * jj)) & 15u);
          float fo = 128.0f + (float)((w >> (4 * jj + 4)) & 15u);
          ae = fmaf(fe, v[8 * wd + jj], ae);
          ao = fmaf(fo, v[8 * wd + jj + 1], ao);
        }
      }
      float T = ae + ao;
      float s = qo_bf2f(srow[c >> 1]), b = qo_bf2f(brow[c >> 1]);
      P[l] = fmaf(b, xc[c].xc, s * T);
    }
    float B = qo_butterfly32(P);
    y = (i == 0) ? B : y + B;
  }
  return y;
}

QO_API int qo_qmv_affine(const uint16_t* x, const uint32_t* wq, const uint16_t* sc,
                         const uint16_t* bi, uint16_t* y, int M, int N, int K) {
  if (K % 1024 != 0 || M < 1 || N < 1) return -1;
  float* xf = (float*)malloc(sizeof(float) * (size_t)M * K);
  qo_xchunk* xc = (qo_xchunk*)malloc(sizeof(qo_xchunk) * (size_t)M * (K / 32));
  for (int m = 0; m < M; ++m) qo_affine_xprep(x + (size_t)m * K, K, xf + (size_t)m * K, xc + (size_t)m * (K / 32));
  int G = K / 64;
#pragma omp parallel for schedule(static)
  for (int n = 0; n < N; ++n) {
    for (int m = 0; m < M; ++m) {
      float v = qo_affine_row(xf + (size_t)m * K, xc + (size_t)m * (K / 32), wq + (size_t)n * (K / 8),
                              sc + (size_t)n * G, bi + (size_t)n * G, K);
      y[(size_t)m * N + n] = qo_f2bf(v);
    }
  }
  free(xf);
  free(xc);
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
