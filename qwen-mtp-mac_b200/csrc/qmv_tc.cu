// 4-bit affine group-64 GEMV (qmv) on the 5th-generation tensor cores (tcgen05.mma kind::i8).
//
// Replaces qmv_kernel.py:31-101 (qmv_nvfp4_multi) and the MLX quantized_matmul route of
// qmv_kernel.py:104-113 for the affine format: y[m, n] = sum_k x[m, k] * (s[n, k/64] * q[n, k] + b[n, k/64]).
//
// Arithmetic (the contract oracle/qmtp_oracle.c:qo_qmv_affine states):
//   * every group of 64 activations of a token is put on a block-floating-point grid: E = exponent of
//     the group's largest |x|, x_q = RNE(x * 2^(19-E)), an exact integer |x_q| < 2^20 (exact for every
//     element >= 2^-12 of the group's maximum);
//   * x_q is split into three signed bytes (x_q = l2*2^14 + l1*2^7 + l0) and the tensor core forms the
//     exact integer sums D_l = sum_k q_k * l_k (s8 x s8 -> s32), so S = sum_k q_k x_q,k is exact;
//   * per group: acc = fma(float(S), s * 2^(E-19), acc); acc = fma(b, float(sum x_q) * 2^(E-19), acc),
//     two chains of four groups per slice of 512 k, slices added in order.
// The per-group integer sums are exact, so the result does not depend on how the work is split: a
// launch may give a CTA whole tiles or slices of a tile, and every token row is independent of the
// others (batch-invariant).
//
// Design (one CTA of 20 warps per SM, 228 KB of shared memory, all 512 TMEM columns):
//   * a tile is R <= 128 weight rows (the MMA's M); a unit of work is (tile, slice of 512 k).  A CTA
//     takes whole tiles, or (cluster mode) the CTAs of a thread-block cluster share one tile: rank k
//     computes slices [k, k + 1) * NSL / cs, keeps each slice's partial in its shared memory, and rank
//     0 adds the other ranks' partials to its own running sum in slice order through distributed
//     shared memory (two cluster barriers; no global workspace, no atomics);
//   * warps 0, 2 and 12-19 first build the B operand of every slice the CTA needs (the three byte
//     limbs of every token, 16 x 64 bytes per group, canonical K-major layout) and the per-group
//     factors from x -- optionally RMS-normalising the token rows first (the NORM instantiation) --
//     while the first weight stages are in flight and already being unpacked;
//   * warp 0 is the TMA producer: per unit, two 128-byte-wide boxes of packed nibbles (128-byte swizzle)
//     and the unit's scales and biases land in a 4-stage ring;
//   * the two chains of a slice (groups 0-3 and 4-7) each have 4 unpacking warps (4-7, 8-11) and 4
//     epilogue warps (12-15, 16-19); warp w serves TMEM lane quarter w % 4 and a thread owns one
//     weight row.  An unpacking thread turns its row's nibbles into bytes (two LOP3s per word) and
//     stores them into TMEM as the A operand, and hands the unit's scales and biases to the epilogue
//     through a shared-memory side buffer; an epilogue thread reads the integer accumulators back and
//     runs the chain.  The chain-1 epilogue hands its partial to the chain-0 epilogue of the same row,
//     which adds the slices in order;
//   * warp 1 (chain 0) and warp 3 (chain 1) each issue the chain's 8 MMAs of a unit (M=128, N=16, K=32,
//     A from TMEM, B from shared memory) and one commit.  TMEM: A slots [0,256), accumulator slots
//     [256,512), two units in flight.
// The nibble-to-byte unpacking permutes k inside each word (bytes 0,2,4,6 then 1,3,5,7); the B operand
// is built with the same permutation, so every product pairs the right x with the right q.
#include <cuda.h>

#include <algorithm>
#include <atomic>
#include <mutex>

#include "common.cuh"

namespace qmtp {
namespace tq {

constexpr int kMaxRows = 128;                      // MMA M: rows of a tile
constexpr int kGpu = 8;                            // groups of 64 k per unit (one 512-k slice)
constexpr int kBox = 128;                          // inner bytes of a weight TMA box (4 groups)
constexpr int kWStage = 2 * kMaxRows * kBox;       // 32768: two boxes
constexpr int kSStage = kMaxRows * 16;             // 2048: 8 bf16 per row
constexpr int kStage = kWStage + 2 * kSStage;      // 36864
constexpr int kNS = 4;                             // weight ring stages
// B image of one group: 16 rows x 64 bytes as 4 x 2 core matrices (8 rows x 16 bytes each).  The
// four 16-byte k chunks sit kLbo = 272 bytes apart and the groups 1088 bytes apart (not multiples of
// 128), so the 32 lanes of a build store spread over all 32 banks (two wavefronts for 256 bytes);
// the 16-byte holes after chunks 0 and 1 hold the group's factors (c, xf) of tokens 0-1 and 2-3.
constexpr int kLbo = 272;
constexpr int kBGroup = 1088;
constexpr int kNB = 8;                             // B slots
constexpr int kBSlot = kGpu * kBGroup;             // 8704
constexpr int kMaxTok = 4;                         // tokens per launch (3 limbs each: 12 of 16 B rows)
constexpr int kOffB = kNS * kStage;                // 147456
constexpr int kOffH = kOffB + kNB * kBSlot;        // 217088: chain-1 partials [2][kMaxTok][128] fp32
constexpr int kOffSB = kOffH + 2 * kMaxTok * 128 * 4;  // 221184: scales | biases per unit [2][2][128] x 16 B
constexpr int kOffBar = kOffSB + 2 * 2 * 128 * 16;      // 229376
constexpr int kSmemUsed = kOffBar + 512;
constexpr int kSmem = kSmemUsed + 1024;            // slack for 1024-byte alignment of the base
constexpr int kThreads = 640;                      // 20 warps
constexpr int kTmemCols = 512;
constexpr int kABase = 0, kDBase = 256;
constexpr int kMinRows = 64;                       // smallest tile the planner picks
static_assert(kOffB % 1024 == 0 && kStage % 1024 == 0, "stage alignment");
static_assert(3 * kLbo + 2 * 128 <= kBGroup && kLbo - 256 >= 16 && kBGroup % 16 == 0, "B group layout");
// Byte offset of a group's (c, xf) float2 for token m inside its B image (the holes after chunks 0, 1).
__host__ __device__ constexpr int xs_offset(int g, int m) { return g * kBGroup + 256 + (m >> 1) * kLbo + (m & 1) * 8; }
static_assert(kSmem <= 232448, "shared memory per CTA");
// Cluster mode: a CTA holds at most this many slices of its tile, so that its per-slice partials
// ([unit][kMaxTok][128] fp32, 2 KB a unit) fit in the B slots it leaves free.
constexpr int kMaxClusterUnits = 6;
static_assert(kMaxClusterUnits * kMaxTok * 128 * 4 <= (kNB - kMaxClusterUnits) * kBSlot, "cluster partials");

// Barriers.  Per unit j: weight stage j % kNS (full / empty); A and accumulator slot a = j & 1 per
// chain h (afull / dfull / dempty [h][a]); activation operand slot (bfull / bempty); the chain-1 partial
// buffer j & 1 handed from the chain-1 workers to the chain-0 workers (hfull / hempty).
struct Bars {
  uint64_t full[kNS], empty[kNS];
  uint64_t afull[2][2], dfull[2][2], dempty[2][2];
  uint64_t bfull[kNB], bempty[kNB];
  uint64_t hfull[2], hempty[2];
  uint64_t drain[2];
  uint32_t tmem;
  int abort;
  int last;
  float rn[kMaxTok];  // RMSNorm prologue: 1 / rms per token
};
static_assert(sizeof(Bars) <= 512, "barrier block");

struct Params {
  const uint16_t* x;
  long long ldx;
  uint16_t* y;
  const uint16_t* res;
  unsigned* err;
  int ldy, N, K, NSL, R, ntiles;  // ntiles * (gridDim.x + 1) and ntiles * NSL < 2^31 (host-checked)
  int cs;             // cluster mode (> 1): CTAs per tile, one tile per cluster
  int pair;           // pair mode (cs == 2): a cluster owns a run of tiles and splits its units in two
  // activation prologue (template parameter PRO): kProRms: x = RMSNorm(x rows; nw, eps); kProSwiglu:
  // x = silu(g) * u with g = x[:, k] and u = x[:, K + k]; kProGated: x = bf16(RMSNorm_head(y; nw, eps)
  // * silu(z)), y fp32 rows at x (ldx in floats), z bf16 rows [ldz], heads of 128.
  const uint16_t* nw;
  float eps;
  const uint16_t* z;
  long long ldz;
};
enum : int { kProNone = 0, kProRms = 1, kProSwiglu = 2, kProGated = 3 };

// (tile, slice) of a CTA's units in processing order, advanced without divisions: `left` units of the
// current run, then (pair mode) one jump to a second run of `jl` units starting at (jt, js).
struct UnitCursor {
  int tile, sl, left, jt, js, jl;
  template <bool JUMP>
  __device__ __forceinline__ void next(int NSL) {
    if (JUMP && --left == 0 && jl > 0) {
      tile = jt;
      sl = js;
      left = jl;
      jl = 0;
      return;
    }
    if (++sl == NSL) {
      sl = 0;
      ++tile;
    }
  }
};

// D (TMEM, s32) (+)= A (TMEM, s8 rows) x B (shared memory, s8, K-major).  No "memory" clobber: the
// operands are ordered by the barrier waits and the tcgen05 fences around the issue loop.
__device__ __forceinline__ void umma_i8(uint32_t d, uint32_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d),
      "r"(a), "l"(b), "r"(idesc), "r"(acc));
}
// Instruction descriptor, kind::i8: s32 accumulator, s8 A and B, both K-major.
__host__ __device__ constexpr uint32_t idesc_i8(int M, int N) {
  return (2u << 4) | (1u << 7) | (1u << 10) | (uint32_t(N >> 3) << 17) | (uint32_t(M >> 4) << 24);
}
// 2^k as fp32 (exact for k >= -149, 0 below).
__device__ __forceinline__ float pow2f(int k) {
  if (k >= -126) return __uint_as_float(uint32_t(k + 127) << 23);
  if (k >= -149) return __uint_as_float(1u << (k + 149));
  return 0.0f;
}
// x * 2^(19-E) rounded to the nearest integer (ties to even).  The scaling is split into two powers
// of two that are normal fp32 numbers; bf16 x has 8 significant bits and |x| < 2^(E+1), so both
// products are exact whenever the result is at least 1/2 in magnitude (a product that underflows
// belongs to an element that rounds to 0 either way), and the conversion does the one rounding.
// The rounding is done by adding 1.5 * 2^23: every |x * 2^(19-E)| is below 2^20, so the sum lies in
// [2^23, 2^24), where the fp32 spacing is 1 and the addition rounds to the nearest integer, ties to
// even; the integer is the sum's low mantissa bits.
__device__ __forceinline__ int grid_value(float x, float s1, float s2) {
  return __float_as_int(__fadd_rn(__fmul_rn(__fmul_rn(x, s1), s2), 12582912.0f)) - 0x4B400000;
}
// The first NC (<= 12) accumulator columns of a lane quarter (32x32b shape): only the 3 * MT limb
// columns of a group are read.  Completion is awaited by the caller (tmem_ld_wait).
__device__ __forceinline__ void tmem_ld_x1(uint32_t taddr, uint32_t* v) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(v[0]) : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_x4(uint32_t taddr, uint32_t* v) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3])
               : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_x8(uint32_t taddr, uint32_t* v) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
               : "r"(taddr));
}
template <int NC>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, uint32_t* v) {
  static_assert(NC >= 1 && NC <= 12, "at most 12 accumulator columns");
  if constexpr (NC <= 4) {
    tmem_ld_x4(taddr, v);
  } else if constexpr (NC <= 8) {
    tmem_ld_x8(taddr, v);
  } else if constexpr (NC == 9) {
    tmem_ld_x8(taddr, v);
    tmem_ld_x1(taddr + 8u, v + 8);
  } else {
    tmem_ld_x8(taddr, v);
    tmem_ld_x4(taddr + 8u, v + 8);
  }
}

__device__ __forceinline__ void prefetch_tmap(const void* m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(m) : "memory");
}

// Two fp32 values rounded to nearest-even bf16 and packed (lo in bits 0-15), one conversion
// instruction.  Finite and infinite values round exactly as f2bf; a NaN may come out with another
// payload, which the activation grid treats like any NaN (the token row becomes NaN).
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t d;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}
// 8 normalised activations: bf16(w * bf16(x * r)) element by element (the RMSNorm of
// oracle qo_rmsnorm / rmsnorm_wide_kernel, r = 1 / rms of the token's row).
__device__ __forceinline__ uint4 rms_apply(uint4 xv, uint4 wv, float r) {
  const uint32_t xs[4] = {xv.x, xv.y, xv.z, xv.w}, ws[4] = {wv.x, wv.y, wv.z, wv.w};
  uint32_t o[4];
#pragma unroll
  for (int h = 0; h < 4; ++h) {
    const uint32_t t = pack_bf16x2(__fmul_rn(bflo(xs[h]), r), __fmul_rn(bfhi(xs[h]), r));
    o[h] = pack_bf16x2(__fmul_rn(bflo(ws[h]), bflo(t)), __fmul_rn(bfhi(ws[h]), bfhi(t)));
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// 8 SwiGLU activations: bf16(silu(g) * u) element by element (the decoder's swiglu_kernel).
__device__ __forceinline__ uint4 swiglu_apply(uint4 gv, uint4 uv) {
  const uint32_t gs[4] = {gv.x, gv.y, gv.z, gv.w}, us[4] = {uv.x, uv.y, uv.z, uv.w};
  uint32_t o[4];
#pragma unroll
  for (int h = 0; h < 4; ++h) {
    const uint32_t lo = f2bf(__fmul_rn(silu_bf(bflo(gs[h])), bflo(us[h])));
    const uint32_t hi = f2bf(__fmul_rn(silu_bf(bfhi(gs[h])), bfhi(us[h])));
    o[h] = lo | (hi << 16);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}
// 8 gated-norm activations of one head of 128 (gdn_norm_gate_kernel): this task holds elements
// [8i, 8i + 8) of the head, i = lane % 16, so the head's 16 tasks are 16 lanes of one warp.  The sum of
// squares is that kernel's: per 4 elements a sequential fma chain (norm lane 2i and 2i + 1), then the
// xor butterfly over the 32 chains -- done here on the pairs (lane xor 8, 4, 2, 1, then the pair).
// Every lane of the warp must call it.
__device__ __forceinline__ uint4 gated_apply(float4 y0, float4 y1, uint4 zv, uint4 wv, float eps) {
  float a = 0.0f, b = 0.0f;
  a = __fmaf_rn(y0.x, y0.x, a);
  a = __fmaf_rn(y0.y, y0.y, a);
  a = __fmaf_rn(y0.z, y0.z, a);
  a = __fmaf_rn(y0.w, y0.w, a);
  b = __fmaf_rn(y1.x, y1.x, b);
  b = __fmaf_rn(y1.y, y1.y, b);
  b = __fmaf_rn(y1.z, y1.z, b);
  b = __fmaf_rn(y1.w, y1.w, b);
#pragma unroll
  for (int d = 8; d >= 1; d >>= 1) {
    a = __fadd_rn(a, __shfl_xor_sync(0xFFFFFFFFu, a, d));
    b = __fadd_rn(b, __shfl_xor_sync(0xFFFFFFFFu, b, d));
  }
  const float r = rsqrt_rn(__fadd_rn(__fmul_rn(__fadd_rn(a, b), 1.0f / 128.0f), eps));
  const float yv[8] = {y0.x, y0.y, y0.z, y0.w, y1.x, y1.y, y1.z, y1.w};
  const uint32_t zs[4] = {zv.x, zv.y, zv.z, zv.w}, ws[4] = {wv.x, wv.y, wv.z, wv.w};
  uint32_t o[4];
#pragma unroll
  for (int h = 0; h < 4; ++h) {
    const float xl = R(__fmul_rn(bflo(ws[h]), R(__fmul_rn(yv[2 * h], r))));
    const float xh = R(__fmul_rn(bfhi(ws[h]), R(__fmul_rn(yv[2 * h + 1], r))));
    o[h] = uint32_t(f2bf(__fmul_rn(xl, silu_f32(bflo(zs[h]))))) |
           (uint32_t(f2bf(__fmul_rn(xh, silu_f32(bfhi(zs[h]))))) << 16);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// One activation task: 8 consecutive x of token m in group g (lane li of the group's 8 lanes) ->
// their three byte limbs in the B image of the slot (rows 3m..3m+2, permuted k: the even k of the
// 8 then the odd k, as the nibble unpacking orders the weights) and, from lane 0 of the group, the
// group factors (c, xf).  All 8 lanes of a group are in one warp.
__device__ __forceinline__ void prep_task(uint4 v, int m, int g, int li, uint8_t* bimg) {
  // largest magnitude of the group as a bf16 bit pattern (patterns order like magnitudes; an infinity
  // or NaN has a pattern >= 0x7F80, above every finite one)
  const uint32_t a2 = __vmaxu2(__vmaxu2(v.x & 0x7FFF7FFFu, v.y & 0x7FFF7FFFu), __vmaxu2(v.z & 0x7FFF7FFFu, v.w & 0x7FFF7FFFu));
  uint32_t amax = max(a2 & 0xFFFFu, a2 >> 16);
#pragma unroll
  for (int d = 1; d < 8; d <<= 1) amax = max(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, d));
  const bool nf = amax >= 0x7F80u;
  const int ef = int(amax >> 7);
  const int E = ef ? ef - 127 : -133 + (31 - __clz(int(amax & 127u) | 1));
  // k in [-109, 152]: both factors are normal fp32 powers of two.  An all-zero group gives x_q = 0; a
  // group with a non-finite element gets NaN factors below, whatever its x_q.
  const int k = 19 - E;
  const float s1 = pow2f(k >> 1), s2 = pow2f(k - (k >> 1));
  const float xv[8] = {bflo(v.x), bfhi(v.x), bflo(v.y), bfhi(v.y), bflo(v.z), bfhi(v.z), bflo(v.w), bfhi(v.w)};
  int xq[8];
  int xs = 0;
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    xq[e] = grid_value(xv[e], s1, s2);
    xs += xq[e];
  }
  // limb l of element e is byte 0 of (x_q >> 7l) (l0, l1 masked to 7 bits); the even elements fill the
  // low word of a limb's 8 bytes, the odd ones the high word
  auto pack4 = [](uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    return __byte_perm(__byte_perm(a, b, 0x0040), __byte_perm(c, d, 0x0040), 0x5410);
  };
  uint32_t lo[3], hi[3];
  lo[0] = pack4(xq[0], xq[2], xq[4], xq[6]) & 0x7F7F7F7Fu;
  hi[0] = pack4(xq[1], xq[3], xq[5], xq[7]) & 0x7F7F7F7Fu;
  lo[1] = pack4(xq[0] >> 7, xq[2] >> 7, xq[4] >> 7, xq[6] >> 7) & 0x7F7F7F7Fu;
  hi[1] = pack4(xq[1] >> 7, xq[3] >> 7, xq[5] >> 7, xq[7] >> 7) & 0x7F7F7F7Fu;
  lo[2] = pack4(xq[0] >> 14, xq[2] >> 14, xq[4] >> 14, xq[6] >> 14);
  hi[2] = pack4(xq[1] >> 14, xq[3] >> 14, xq[5] >> 14, xq[7] >> 14);
#pragma unroll
  for (int d = 1; d < 8; d <<= 1) xs += __shfl_xor_sync(0xFFFFFFFFu, xs, d);
  const int pb = 8 * li;
#pragma unroll
  for (int l = 0; l < 3; ++l) {
    const int j = 3 * m + l;
    const int off = g * kBGroup + (pb >> 4) * kLbo + (j >> 3) * 128 + (j & 7) * 16 + (pb & 15);
    *reinterpret_cast<uint2*>(bimg + off) = make_uint2(lo[l], hi[l]);
  }
  if (li == 0) {
    float c, xf;
    if (nf) {
      c = xf = __uint_as_float(0x7FC00000u);
    } else if (amax == 0) {
      c = xf = 0.0f;
    } else {
      c = pow2f(E - 19);
      xf = __fmul_rn(__int2float_rn(xs), c);
    }
    *reinterpret_cast<float2*>(bimg + xs_offset(g, m)) = make_float2(c, xf);
  }
}

// Warp roles (12 warps):
//   0      TMA producer (lane 0), after the activation build;
//   1, 3   MMA issuers of chain 0 (groups 0-3 of a unit) and chain 1 (groups 4-7), lane 0;
//   all    first build the activation operand of every slice the CTA needs (the first weight stages
//          are in flight meanwhile);
//   2      in stream mode (more than 8 slices and units), builds the later slices one unit at a time;
//   4-7    chain-0 workers, 8-11 chain-1 workers: warp w serves TMEM lane quarter w % 4, thread = row.
// PRO: the activation prologue (kProNone, kProRms, kProSwiglu, kProGated); PAIR: pair mode (2-CTA
// clusters owning tile runs).  A separate instantiation per variant keeps each kernel's code small.
template <int MT, int PRO, bool PAIR>
__global__ void __launch_bounds__(kThreads, 1)
    qmv_tc_kernel(const __grid_constant__ CUtensorMap tw, const __grid_constant__ CUtensorMap ts,
                  const __grid_constant__ CUtensorMap tb, const __grid_constant__ Params p) {
  extern __shared__ uint8_t smraw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smraw) + 1023) & ~uintptr_t(1023));
  Bars* bars = reinterpret_cast<Bars*>(sm + kOffBar);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int NSL = p.NSL, R = p.R;
  unsigned* err = p.err;

  int u0, u1;
  const int cs = p.cs;
  const uint32_t crank = cs > 1 ? cluster_rank() : 0u;
  // pair mode: rank 1's range may start with the last `tail` units of the tile rank 0 starts (rank 0's
  // "head"); rank 1 processes them last, so their weight stages are free for their slice partials
  int tail = 0, head = 0, n1 = 0;
  if (PAIR) {
    const int ncl = int(gridDim.x) / 2, c = int(blockIdx.x) / 2;
    const int t0 = c * p.ntiles / ncl, t1 = (c + 1) * p.ntiles / ncl;
    const int half = (t1 - t0) * NSL / 2;
    head = half % NSL;  // rank 0's last tile ends after `head` slices (0: tile-aligned split)
    tail = head ? NSL - head : 0;
    n1 = (t1 - t0) * NSL - half;  // units of rank 1
    u0 = t0 * NSL + (crank ? half : 0);
    u1 = crank ? t1 * NSL : t0 * NSL + half;
  } else if (cs > 1) {
    // cluster c = blockIdx.x / cs holds tile c; rank k takes slices [k, k + 1) * NSL / cs
    const int per = NSL / cs;
    u0 = int(blockIdx.x) / cs * NSL + int(crank) * per;
    u1 = u0 + per;
  } else {
    // whole tiles: CTA b takes tiles [b, b + 1) * ntiles / grid
    u0 = int(blockIdx.x) * p.ntiles / int(gridDim.x) * NSL;
    u1 = int(blockIdx.x + 1) * p.ntiles / int(gridDim.x) * NSL;
  }
  const int nun = u1 - u0;
  const int tl = crank ? tail : 0;  // this CTA's tail units (processed last)
  const int nA = nun - tl;          // units before them
  const UnitCursor first = nA > 0 && tl > 0 ? UnitCursor{(u0 + tl) / NSL, (u0 + tl) % NSL, nA, u0 / NSL, u0 % NSL, tl}
                                            : UnitCursor{u0 / NSL, u0 % NSL, nun, 0, 0, 0};
  // cache mode: every slice the CTA needs has its own B slot, built once up front; stream mode (more
  // than kNB distinct slices): slot j % kNB is rebuilt for each unit
  const bool cache = NSL <= kNB || nun <= kNB;
  // slots by slice when a CTA may revisit slices (several tiles), else by unit (cluster mode: one
  // tile, slots [0, nun); its slice partials go to the free slots after them)
  const bool by_slice = NSL <= kNB && (cs == 1 || PAIR);
  // B slot of unit j whose slice is sl
  auto slot_of = [&](int j, int sl) { return cache ? (by_slice ? sl : j) : (j & (kNB - 1)); };
  const int nbuild = cache ? min(nun, by_slice ? NSL : nun) : min(nun, kNB);
  // cluster mode: this CTA's slice partials, [unit][row][kMaxTok] fp32
  float* cpart = reinterpret_cast<float*>(sm + kOffB + nun * kBSlot);
  float Y[MT];  // chain-0 epilogue threads: running sum of the current tile's slices
#pragma unroll
  for (int m = 0; m < MT; ++m) Y[m] = 0.0f;

  if (tid == 0) {
    prefetch_tmap(&tw);
    prefetch_tmap(&ts);
    prefetch_tmap(&tb);
    for (int s = 0; s < kNS; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 8);
    }
    for (int h = 0; h < 2; ++h)
      for (int s = 0; s < 2; ++s) {
        mbar_init(&bars->afull[h][s], 4);   // the chain's workers have stored the unit's A
        mbar_init(&bars->dfull[h][s], 1);   // the chain's 8 MMAs of the unit are complete
        mbar_init(&bars->dempty[h][s], 4);  // the chain's workers have read the unit's accumulators
      }
    for (int s = 0; s < kNB; ++s) {
      mbar_init(&bars->bfull[s], 2 * MT);  // one arrival per warp batch of 32 tasks
      mbar_init(&bars->bempty[s], 8);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars->hfull[s], 4);
      mbar_init(&bars->hempty[s], 4);
      mbar_init(&bars->drain[s], 1);
    }
    bars->abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(&bars->tmem, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem;
  volatile int* abort_flag = &bars->abort;

  const uint64_t pol_w = policy_evict_first();
  auto issue = [&](int j, const UnitCursor& c) {
    const int sl = c.sl;
    const int row = c.tile * R;
    const int st = j % kNS;
    uint8_t* dst = sm + st * kStage;
    mbar_expect_tx(&bars->full[st], uint32_t(R * (2 * kBox + 32)));
    tma_load_2d(dst, &tw, sl * 256, row, &bars->full[st], pol_w);
    tma_load_2d(dst + kMaxRows * kBox, &tw, sl * 256 + kBox, row, &bars->full[st], pol_w);
    tma_load_2d(dst + kWStage, &ts, sl * 8, row, &bars->full[st], pol_w);
    tma_load_2d(dst + kWStage + kSStage, &tb, sl * 8, row, &bars->full[st], pol_w);
  };
  // The weights are constant: the first stages are requested before the dependency wait.
  const int pre = min(kNS, nun);
  UnitCursor pc = first;  // producer's cursor: the next unit to request
  if (warp == 0 && lane == 0)
    for (int j = 0; j < pre; ++j, pc.template next<PAIR>(NSL)) issue(j, pc);
  // trigger after the wait: a successor that starts implies the previous launch has finished (the
  // successor's CTAs still launch long before this kernel ends: its main loop follows)
  pdl_wait();
  pdl_trigger();

  // Builds the activation operand of units [j0, j0 + nb) (their slots) with `nthr` threads, this one
  // being number `me` of them: the tasks in slot order, each task's x loaded two tasks ahead, one
  // bfull arrival per warp batch.  The loop is not unrolled: the kernel's roles run different code at
  // the same time, and a small loop body keeps them in the instruction cache.
  constexpr int kBuilders = 320;  // up-front build: warps 0, 2 and 12-19
  const bool builder = warp == 0 || warp == 2 || warp >= 12;
  const int bme = warp == 0 ? lane : warp == 2 ? 32 + lane : tid - 320;  // builder index
  // RMSNorm prologue: 1 / rms per token in rn[m], over the whole row of every token, in the reduction
  // order of rmsnorm_wide_kernel: chains of 32 elements (fma), the xor butterfly over 32 chains, the
  // 1024-element group sums in order.  The group sums use the chain-1 partial buffer, which no
  // epilogue touches before the build has started (so not before both prologue barriers); rn itself
  // is read during the whole build and sits in the barrier block.
  float* rn = bars->rn;
  auto reduce_rows = [&](int me) {
    float* grp = reinterpret_cast<float*>(sm + kOffH);  // [kMaxTok][32] group sums
    const int C = p.K / 32;
    // chains are taken two per trip with all eight loads issued first (for K = 4096 and up to four
    // tokens, one trip)
#pragma unroll 1
    for (int v0 = me; v0 < MT * C; v0 += 2 * kBuilders) {  // warp-uniform: C is a multiple of 32
      uint4 u[2][4];
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int v = v0 + i * kBuilders;
        if (v < MT * C) {
          const int m = v / C, c = v - m * C;
          const uint16_t* src = p.x + (size_t)m * (size_t)p.ldx + 32 * c;
#pragma unroll
          for (int q = 0; q < 4; ++q) u[i][q] = *reinterpret_cast<const uint4*>(src + 8 * q);
        }
      }
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int v = v0 + i * kBuilders;
        if (v < MT * C) {  // warp-uniform
          const int m = v / C, c = v - m * C;
          float ss = 0.0f;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint32_t uu[4] = {u[i][q].x, u[i][q].y, u[i][q].z, u[i][q].w};
#pragma unroll
            for (int h = 0; h < 4; ++h) {
              ss = __fmaf_rn(bflo(uu[h]), bflo(uu[h]), ss);
              ss = __fmaf_rn(bfhi(uu[h]), bfhi(uu[h]), ss);
            }
          }
          ss = warp_sum(ss);
          if (lane == 0) grp[m * 32 + (c >> 5)] = ss;
        }
      }
    }
    asm volatile("bar.sync 2, 320;" ::: "memory");
    if (me < MT) {
      float t = grp[me * 32];
      for (int i = 1; i < p.K / 1024; ++i) t = __fadd_rn(t, grp[me * 32 + i]);
      rn[me] = rsqrt_rn(__fadd_rn(__fdiv_rn(t, float(p.K)), p.eps));
    }
    asm volatile("bar.sync 2, 320;" ::: "memory");
  };
  // reduce: the up-front build by all builders computes the RMSNorm factors first, with its own
  // first loads already in flight
  auto build = [&](int j0, int nb, int me, int nthr, bool reduce) {
    const int per_slot = 64 * MT;
    const int total = nb * per_slot;
    const int sbase = (first.sl + j0) % NSL;  // slice of unit j0
    auto kof = [&](int t) {  // k offset of task t
      const int jb = t / per_slot, r = t - jb * per_slot;
      const int sl = sbase + jb < NSL ? sbase + jb : sbase + jb - NSL;
      return sl * 512 + ((r >> 3) & 7) * 64 + (r & 7) * 8;
    };
    // a task's inputs: x (or y's first 4 / g), and per prologue the RMSNorm weights, u, or y's last 4,
    // z and the gated-norm weights
    struct In {
      uint4 a, b, c, d;
    };
    auto load = [&](int t) {
      const int m = (t % per_slot) >> 6;
      const int k = kof(t);
      In in;
      if (PRO == kProGated) {
        const float* yr = reinterpret_cast<const float*>(p.x) + (size_t)m * (size_t)p.ldx + k;
        in.a = *reinterpret_cast<const uint4*>(yr);
        in.b = *reinterpret_cast<const uint4*>(yr + 4);
        in.c = *reinterpret_cast<const uint4*>(p.z + (size_t)m * (size_t)p.ldz + k);
        in.d = *reinterpret_cast<const uint4*>(p.nw + (k & 127));
      } else {
        in.a = *reinterpret_cast<const uint4*>(p.x + (size_t)m * (size_t)p.ldx + k);
        if (PRO == kProRms) in.b = *reinterpret_cast<const uint4*>(p.nw + k);
        if (PRO == kProSwiglu) in.b = *reinterpret_cast<const uint4*>(p.x + (size_t)m * (size_t)p.ldx + p.K + k);
      }
      return in;
    };
    In va{}, vb{};
    if (me < total) va = load(me);
    if (me + nthr < total) vb = load(me + nthr);
    if (PRO == kProRms && reduce) reduce_rows(me);
    int cur_slot = -1;  // slot of this warp's open batch run (its bfull arrivals are owed)
    int batches = 0;
#pragma unroll 1
    for (int t = me; t < total; t += nthr) {  // warp-uniform: total and nthr are multiples of 32
      const In in = va;
      va = vb;
      if (t + 2 * nthr < total) vb = load(t + 2 * nthr);
      {
        const int jb = t / per_slot, r = t - jb * per_slot;
        uint4 v = in.a;
        if (PRO == kProRms) v = rms_apply(in.a, in.b, rn[r >> 6]);
        if (PRO == kProSwiglu) v = swiglu_apply(in.a, in.b);
        if (PRO == kProGated)
          v = gated_apply(make_float4(__uint_as_float(in.a.x), __uint_as_float(in.a.y), __uint_as_float(in.a.z),
                                      __uint_as_float(in.a.w)),
                          make_float4(__uint_as_float(in.b.x), __uint_as_float(in.b.y), __uint_as_float(in.b.z),
                                      __uint_as_float(in.b.w)),
                          in.c, in.d, p.eps);
        const int slot = slot_of(j0 + jb, sbase + jb < NSL ? sbase + jb : sbase + jb - NSL);
        if (slot != cur_slot && cur_slot >= 0) {
          fence_proxy_async();
          __syncwarp();
          if (lane == 0)
            for (int b = 0; b < batches; ++b) mbar_arrive(&bars->bfull[cur_slot]);
          batches = 0;
        }
        cur_slot = slot;
        ++batches;
        const int m = r >> 6, g = (r >> 3) & 7, li = r & 7;
        prep_task(v, m, g, li, sm + kOffB + slot * kBSlot);
      }
    }
    if (cur_slot >= 0) {
      fence_proxy_async();
      __syncwarp();
      if (lane == 0)
        for (int b = 0; b < batches; ++b) mbar_arrive(&bars->bfull[cur_slot]);
    }
  };

  // The activation operand is built up front by the producer warp (after its first requests), warp 2
  // and the epilogue warps (idle until the first accumulators are ready), while the unpacking warps
  // already turn the first weight stages into A operands and the MMA issuers wait for the first slot.
  // In stream mode warp 2 goes on building the later slots one unit at a time (one call site keeps a
  // single copy of the build code).
  if (builder) {
    int j = 0, nb = nbuild, me = bme, nthr = kBuilders;
    for (;;) {
      build(j, nb, me, nthr, j == 0);
      if (warp != 2 || cache) break;
      j = j == 0 ? kNB : j + 1;
      if (j >= nun) break;
      const int slot = j % kNB;
      if (*abort_flag || !mbar_wait_backoff(&bars->bempty[slot], uint32_t(((j / kNB) & 1) ^ 1), err, 64)) {
        *abort_flag = 1;
        break;
      }
      nb = 1;
      me = lane;
      nthr = 32;
    }
  }

  if (warp == 0) {
    // ------------------------------------------------------------------- TMA producer
    if (lane == 0) {
      int j = pre;
      for (; j < nun; ++j, pc.template next<PAIR>(NSL)) {
        const int st = j % kNS;
        if (*abort_flag || !mbar_wait_backoff(&bars->empty[st], ((j / kNS) & 1) ^ 1, err, 64)) break;
        fence_proxy_async();
        issue(j, pc);
      }
      if (j < nun) {
        *abort_flag = 1;
        // no copy may land after the CTA exits: wait for the stages still in flight
        for (int k = 1; k <= kNS && j - k >= 0; ++k) {
          const int jj = j - k;
          mbar_wait_backoff(&bars->full[jj % kNS], (jj / kNS) & 1, err, 64, 1u << 16);
        }
      }
    }
  } else if (warp == 1 || warp == 3) {
    // ------------------------------------------------------------------- MMA issuers (one per chain)
    // An MMA of this shape costs its issuing thread ~100 cycles; two issuing threads overlap on the
    // tensor core (one issuer for both chains measured 1.05-1.25x slower).
    if (lane == 0) {
      const int h = warp == 1 ? 0 : 1;
      constexpr uint32_t idesc = idesc_i8(128, 16);
      const uint32_t bsm = smem_u32(sm + kOffB);
      bool issued = false;
      UnitCursor c = first;
      for (int j = 0; j < nun; ++j, c.template next<PAIR>(NSL)) {
        const int a = j & 1;
        const int slot = slot_of(j, c.sl);
        const uint32_t bpar = cache ? 0u : uint32_t((j / kNB) & 1);
        if (*abort_flag || !mbar_wait_spin(&bars->bfull[slot], bpar, err) ||
            !mbar_wait_spin(&bars->afull[h][a], uint32_t((j >> 1) & 1), err) ||
            !mbar_wait_spin(&bars->dempty[h][a], uint32_t(((j >> 1) & 1) ^ 1), err)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d0 = tmem + uint32_t(kDBase + a * 128 + 64 * h);
        const uint32_t a0 = tmem + uint32_t(kABase + a * 128 + 64 * h);
        // descriptor of the chain's first group; group gi / k-half k2 start gi * kBGroup + k2 * 2 * kLbo
        // bytes later (the start-address field holds address / 16 and stays below 2^14)
        const uint64_t bd = umma_desc(bsm + uint32_t(slot * kBSlot + 4 * h * kBGroup), uint32_t(kLbo), 128u);
#pragma unroll
        for (int gi = 0; gi < 4; ++gi) {
#pragma unroll
          for (int k2 = 0; k2 < 2; ++k2)
            umma_i8(d0 + uint32_t(gi * 16), a0 + uint32_t(gi * 16 + 8 * k2),
                    bd + uint64_t((gi * kBGroup + k2 * 2 * kLbo) >> 4), idesc, uint32_t(k2));
        }
        umma_commit(&bars->dfull[h][a]);
        issued = true;
      }
      // every MMA issued has completed before the CTA releases TMEM
      if (issued) {
        umma_commit(&bars->drain[h]);
        mbar_wait_backoff(&bars->drain[h], 0, err, 64);
      }
    }
  } else if (warp == 2) {
    // (stream-mode operand builds: above)
  } else if (warp < 12) {
    // ------------------------------------------------------------------- unpacking warps
    const int h = warp < 8 ? 0 : 1;  // chain: groups 4h .. 4h+3 of every unit
    const int q = warp & 3;
    const int r = 32 * q + lane;
    const uint32_t tl = tmem + (uint32_t(32 * q) << 16);
    const int rsw = r & 7;
    bool ok = true;
    for (int j = 0; j < nun; ++j) {
      const int st = j % kNS;
      const int a = j & 1;
      // unit j reuses the A slot and the scale/bias slot of unit j-2: its epilogue (which waited for its
      // MMAs) must be done
      if (ok && !*abort_flag) {
        if (!mbar_wait_backoff(&bars->full[st], uint32_t((j / kNS) & 1), err, 32) ||
            !mbar_wait_backoff(&bars->dempty[h][a], uint32_t(((j >> 1) & 1) ^ 1), err, 32)) {
          ok = false;
          *abort_flag = 1;
        }
      } else {
        ok = false;
      }
      tc_fence_after();
      const uint8_t* sg = sm + st * kStage;
      const uint2 sv = *reinterpret_cast<const uint2*>(sg + kWStage + r * 16 + 8 * h);
      const uint2 bv = *reinterpret_cast<const uint2*>(sg + kWStage + kSStage + r * 16 + 8 * h);
      *reinterpret_cast<uint4*>(sm + kOffSB + ((a * 2 + h) * 128 + r) * 16) = make_uint4(sv.x, sv.y, bv.x, bv.y);
      const uint8_t* rowp = sg + h * (kMaxRows * kBox) + r * kBox;  // box h holds groups 4h .. 4h+3
#pragma unroll
      for (int gl = 0; gl < 4; ++gl) {
        const int c0 = 2 * gl;
        const uint4 w0 = *reinterpret_cast<const uint4*>(rowp + 16 * (c0 ^ rsw));
        const uint4 w1 = *reinterpret_cast<const uint4*>(rowp + 16 * ((c0 + 1) ^ rsw));
        const uint32_t wd[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
        uint32_t o[16];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          o[2 * i] = wd[i] & 0x0F0F0F0Fu;
          o[2 * i + 1] = (wd[i] >> 4) & 0x0F0F0F0Fu;
        }
        tmem_st16(tl + uint32_t(kABase + a * 128 + (4 * h + gl) * 16), o);
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0 && ok) {
        mbar_arrive(&bars->empty[st]);
        mbar_arrive(&bars->afull[h][a]);
      }
    }
  } else {
    // ------------------------------------------------------------------- epilogue warps
    const int h = warp < 16 ? 0 : 1;  // chain: groups 4h .. 4h+3 of every unit
    const int q = warp & 3;
    const int r = 32 * q + lane;
    const uint32_t tl = tmem + (uint32_t(32 * q) << 16);
    float* hx = reinterpret_cast<float*>(sm + kOffH);  // [2][kMaxTok][128] chain-1 partials
    bool ok = true;
    UnitCursor ec = first;  // unit of the next epilogue

    // Every epilogue warp runs the same sequence of epilogues and named barriers whatever happens: a
    // wait that gives up only sets `ok` false (and the CTA's abort flag), so no warp is left at a barrier.
    auto epilogue = [&](int jj) {
      const int a = jj & 1;
      const int tile = ec.tile, sl = ec.sl;
      ec.template next<PAIR>(NSL);
      const int slot = slot_of(jj, sl);
      const uint32_t bpar = cache ? 0u : uint32_t((jj / kNB) & 1);
      // dfull: the unit's MMAs are done; afull (already complete): orders the unpacking warp's scale /
      // bias stores before the reads below
      if (ok && !*abort_flag) {
        if (!mbar_wait_backoff(&bars->dfull[h][a], uint32_t((jj >> 1) & 1), err, 32) ||
            !mbar_wait_backoff(&bars->afull[h][a], uint32_t((jj >> 1) & 1), err, 32) ||
            !mbar_wait_backoff(&bars->bfull[slot], bpar, err, 32)) {
          ok = false;
          *abort_flag = 1;
        }
      } else {
        ok = false;
      }
      tc_fence_after();
      const uint8_t* bslot = sm + kOffB + slot * kBSlot;
      // this row's scales and biases of the chain's groups, left by the unpacking warp of the row
      const uint4 sbv = *reinterpret_cast<const uint4*>(sm + kOffSB + ((a * 2 + h) * 128 + r) * 16);
      const uint32_t sw[2] = {sbv.x, sbv.y}, bw[2] = {sbv.z, sbv.w};
      float H[MT];
#pragma unroll
      for (int m = 0; m < MT; ++m) H[m] = 0.0f;
      constexpr int NC = 3 * MT;
      constexpr int NCP = NC <= 4 ? 4 : NC <= 8 ? 8 : 12;
      uint32_t v[4][NCP];
#pragma unroll
      for (int gl = 0; gl < 4; ++gl) tmem_ld_cols<NC>(tl + uint32_t(kDBase + a * 128 + (4 * h + gl) * 16), v[gl]);
      tmem_ld_wait();
      // the accumulators and this unit's scales / biases are in registers: release the A, D and side
      // buffer slots of the chain to unit jj + 2
      tc_fence_before();
      __syncwarp();
      if (lane == 0 && ok) mbar_arrive(&bars->dempty[h][a]);
#pragma unroll
      for (int gl = 0; gl < 4; ++gl) {
        const int g = 4 * h + gl;
        const float s = (gl & 1) ? bfhi(sw[gl >> 1]) : bflo(sw[gl >> 1]);
        const float b = (gl & 1) ? bfhi(bw[gl >> 1]) : bflo(bw[gl >> 1]);
#pragma unroll
        for (int m = 0; m < MT; ++m) {
          const int S = int(v[gl][3 * m + 2]) * 16384 + int(v[gl][3 * m + 1]) * 128 + int(v[gl][3 * m]);
          const float2 cx = *reinterpret_cast<const float2*>(bslot + xs_offset(g, m));
          H[m] = __fmaf_rn(__int2float_rn(S), __fmul_rn(s, cx.x), H[m]);
          H[m] = __fmaf_rn(b, cx.y, H[m]);
        }
      }
      if (!cache) {
        __syncwarp();
        if (lane == 0 && ok) mbar_arrive(&bars->bempty[slot]);
      }
      float* hb = hx + (jj & 1) * (kMaxTok * 128);
      if (h == 1) {
        // hand chain 1 to the chain-0 worker of the same row
        if (ok && !*abort_flag) {
          if (!mbar_wait_backoff(&bars->hempty[jj & 1], uint32_t(((jj >> 1) & 1) ^ 1), err, 32)) {
            ok = false;
            *abort_flag = 1;
          }
        }
#pragma unroll
        for (int m = 0; m < MT; ++m) hb[m * 128 + r] = H[m];
        __syncwarp();
        if (lane == 0 && ok) mbar_arrive(&bars->hfull[jj & 1]);
        return;
      }
      if (ok && !*abort_flag) {
        if (!mbar_wait_backoff(&bars->hfull[jj & 1], uint32_t((jj >> 1) & 1), err, 32)) {
          ok = false;
          *abort_flag = 1;
        }
      }
      float P[MT];
#pragma unroll
      for (int m = 0; m < MT; ++m) P[m] = __fadd_rn(H[m], hb[m * 128 + r]);
      __syncwarp();
      if (lane == 0 && ok) mbar_arrive(&bars->hempty[jj & 1]);
      if (PAIR && jj >= nA) {
        // a tail unit: its partial waits for rank 0 in this unit's weight stage (the last kNS units
        // of a CTA leave their stages unused once unpacked)
        float pv[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int m = 0; m < MT; ++m) pv[m] = P[m];
        *reinterpret_cast<float4*>(sm + (jj % kNS) * kStage + size_t(r) * 16) = make_float4(pv[0], pv[1], pv[2], pv[3]);
        return;
      }
      if (!PAIR && cs > 1) {
        // cluster mode: rank 0 keeps the running sum of slices [0, NSL / cs); the other ranks leave
        // each slice's partial in shared memory for rank 0, which adds them in slice order at the end
        if (crank == 0) {
#pragma unroll
          for (int m = 0; m < MT; ++m) Y[m] = jj == 0 ? P[m] : __fadd_rn(Y[m], P[m]);
        } else {
          float pv[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
          for (int m = 0; m < MT; ++m) pv[m] = P[m];
          *reinterpret_cast<float4*>(cpart + ((size_t)jj * 128 + r) * kMaxTok) = make_float4(pv[0], pv[1], pv[2], pv[3]);
        }
        return;
      }
      // whole tiles: Y is the running sum of the tile's slices, in order
#pragma unroll
      for (int m = 0; m < MT; ++m) Y[m] = sl == 0 ? P[m] : __fadd_rn(Y[m], P[m]);
      if (sl != NSL - 1) return;
      const int row = tile * R + r;
      if (r < R && row < p.N) {
#pragma unroll
        for (int m = 0; m < MT; ++m) {
          uint16_t o = f2bf(Y[m]);
          const size_t oi = (size_t)m * p.ldy + row;
          if (p.res) o = f2bf(__fadd_rn(bf2f(p.res[oi]), bf2f(o)));
          p.y[oi] = o;
        }
      }
    };

    for (int j = 0; j < nun; ++j) epilogue(j);
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, kTmemCols);
  if (PAIR) {
    // Pair mode: rank 0 finishes its head tile with rank 1's tail partials, in slice order, between
    // two cluster barriers (the same rules as below).
    cluster_sync_all();
    if (crank == 0 && head > 0 && warp >= 12 && warp < 16) {
      const int r = 32 * (warp & 3) + lane;
      const int row = (u1 - 1) / NSL * R + r;
      if (r < R && row < p.N) {
        float4 v[kNS];
#pragma unroll
        for (int i = 0; i < kNS; ++i)
          if (i < tail)
            v[i] = ld_dsmem_v4(reinterpret_cast<const float*>(sm + ((n1 - tail + i) % kNS) * kStage + size_t(r) * 16),
                               1u);
#pragma unroll
        for (int i = 0; i < kNS; ++i) {
          if (i < tail) {
            const float pv[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
#pragma unroll
            for (int m = 0; m < MT; ++m) Y[m] = __fadd_rn(Y[m], pv[m]);
          }
        }
#pragma unroll
        for (int m = 0; m < MT; ++m) {
          uint16_t o = f2bf(Y[m]);
          const size_t oi = (size_t)m * p.ldy + row;
          if (p.res) o = f2bf(__fadd_rn(bf2f(p.res[oi]), bf2f(o)));
          p.y[oi] = o;
        }
      }
    }
    cluster_sync_all();
  } else if (cs > 1) {
    // Every thread of every CTA of the cluster passes both barriers (no path leaves the kernel early,
    // and every wait above is bounded).  The first makes the ranks' slice partials visible to rank 0,
    // the second keeps every rank's shared memory alive until rank 0 has read it.
    cluster_sync_all();
    if (crank == 0 && warp >= 12 && warp < 16) {
      const int r = 32 * (warp & 3) + lane;
      const int row = int(blockIdx.x) / cs * R + r;
      if (r < R && row < p.N) {
        const int per = NSL / cs;
        // the other ranks' slices in slice order: a rank's loads all in flight at once, then the adds
#pragma unroll 1
        for (int k = 1; k < cs; ++k) {
          float4 v[kMaxClusterUnits];
#pragma unroll
          for (int j = 0; j < kMaxClusterUnits; ++j)
            if (j < per) v[j] = ld_dsmem_v4(cpart + ((size_t)j * 128 + r) * kMaxTok, uint32_t(k));
#pragma unroll
          for (int j = 0; j < kMaxClusterUnits; ++j) {
            if (j < per) {
              const float pv[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
#pragma unroll
              for (int m = 0; m < MT; ++m) Y[m] = __fadd_rn(Y[m], pv[m]);
            }
          }
        }
#pragma unroll
        for (int m = 0; m < MT; ++m) {
          uint16_t o = f2bf(Y[m]);
          const size_t oi = (size_t)m * p.ldy + row;
          if (p.res) o = f2bf(__fadd_rn(bf2f(p.res[oi]), bf2f(o)));
          p.y[oi] = o;
        }
      }
    }
    cluster_sync_all();
  }
}

// ----------------------------------------------------------------------------- host side
struct Plan {
  int R, G, ntiles, NSL, cs, pair;
};
// Tile and unit indices are 32-bit in the kernel.
constexpr long long kMaxUnitProduct = (1LL << 31) - 1;

// Clusters of `cs` CTAs (228 KB of shared memory each) that can be resident at once on this device.
static int max_clusters(int cs);

// Planner override for tests and measurements (qmtp_qmv_set_mode): 0 = cost model, 1 = whole tiles
// only, 2 = cluster mode where the shape allows it.
static std::atomic<int> g_mode{0};

// Rows per tile, grid and mode, from a cost model of the slowest CTA, fitted to B200 timings of this
// kernel: about 2 us of setup and first weight latency, 0.45 us per activation slice built, about
// 1.05 us per unit (16 MMAs of ~98 issue cycles each over two issuers, plus the pipeline; the weight
// bytes of a 128-row unit stream in 0.84 us at the per-SM share of HBM bandwidth) and about 1.5 us to
// finish a tile shared inside a cluster.  Ties go to the larger tile and to cluster mode.
static Plan make_plan(int N, int K, int sms, bool allow_pair) {
  const int NSL = K / 512;
  Plan best{};
  double best_cost = 1e30;
  const int mode = g_mode.load(std::memory_order_relaxed);
  // cluster mode: one tile per cluster of cs CTAs, at most kMaxClusterUnits slices per CTA, all
  // clusters resident at once
  for (int cs = 2; cs <= 4 && mode != 1; cs *= 2) {
    if (NSL % cs || NSL / cs > kMaxClusterUnits) continue;
    const int mc = max_clusters(cs);
    for (int R = kMaxRows; R >= kMinRows; R -= 8) {
      const int T = (N + R - 1) / R;
      if (T > mc) continue;
      const int per = NSL / cs;
      const double unit_us = std::max(R * 288.0 / 44.0e3, 1.05);
      const double cost = 2.0 + 0.45 * per + per * unit_us + 1.5;
      if (cost < best_cost * 0.999) {
        best_cost = cost;
        best = Plan{R, T * cs, T, NSL, cs, 0};
      }
    }
  }
  // pair mode: every resident 2-CTA cluster owns a run of whole tiles and splits its units between its
  // two CTAs (a tile cut in the middle is finished by rank 0 from rank 1's partials)
  if (mode != 1 && NSL <= kNB && allow_pair) {
    const int ncl = max_clusters(2);
    for (int R = kMaxRows; R >= kMinRows && ncl > 0; R -= 8) {
      const int T = (N + R - 1) / R;
      // up to 4 tiles a cluster: beyond that whole tiles balance well and measured faster (head: 112
      // against 115 us at M = 3)
      if (T < ncl || T > 4 * ncl) continue;
      const int tpc = (T + ncl - 1) / ncl;  // most tiles a cluster owns
      const int per = (tpc * NSL + 1) / 2;
      const bool cut = (tpc * NSL / 2) % NSL != 0 || T % ncl != 0;
      const double unit_us = std::max(R * 288.0 / 44.0e3, 1.05);
      const double cost = 2.0 + 0.45 * std::min(NSL, kNB) + per * unit_us + (cut ? 1.5 : 0.5);
      if (cost < best_cost * 0.999) {
        best_cost = cost;
        best = Plan{R, 2 * ncl, T, NSL, 2, 1};
      }
    }
  }
  if (mode == 2 && best_cost < 1e30) return best;
  for (int R = kMaxRows; R >= kMinRows; R -= 8) {
    const int T = (N + R - 1) / R;
    const int G = std::min(sms, T);
    const long long per = (long long)((T + G - 1) / G) * NSL;
    const double unit_us = std::max(R * 288.0 / 44.0e3, 1.05);
    const double cost = 2.0 + 0.45 * std::min(NSL, kNB) + double(per) * unit_us;
    if (cost < best_cost * 0.999) {
      best_cost = cost;
      best = Plan{R, G, T, NSL, 1, 0};
    }
  }
  return best;
}

static bool encode_2d(CUtensorMap* m, CUtensorMapDataType dt, int esize, const void* base, long long inner,
                      long long rows, int box_inner, int box_rows, CUtensorMapSwizzle swz) {
  auto fn = tensor_map_encoder();
  if (!fn) return false;
  cuuint64_t dims[2] = {cuuint64_t(inner), cuuint64_t(rows)};
  cuuint64_t strides[1] = {cuuint64_t(inner * esize)};
  cuuint32_t box[2] = {uint32_t(box_inner), uint32_t(box_rows)};
  cuuint32_t es[2] = {1, 1};
  return fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int MT, int PRO, bool PAIR>
static bool prepare() {
  static std::once_flag once;
  static bool ok = false;
  std::call_once(once, [&] {
    ok = cudaFuncSetAttribute(qmv_tc_kernel<MT, PRO, PAIR>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem) ==
         cudaSuccess;
  });
  return ok;
}

template <int MT, int PRO, bool PAIR>
static int launch_variant(const CUtensorMap& tw, const CUtensorMap& ts, const CUtensorMap& tb, const Params& p, int G,
                          cudaStream_t st) {
  if (!prepare<MT, PRO, PAIR>()) return QMTP_ERR_CUDA;
  launch_kernel_cluster(qmv_tc_kernel<MT, PRO, PAIR>, dim3(G), dim3(kThreads), kSmem, st, p.cs, tw, ts, tb, p);
  return cudaGetLastError() == cudaSuccess ? QMTP_OK : QMTP_ERR_CUDA;
}

// Pair mode is instantiated for the plain and RMSNorm prologues only (the planner offers it to those).
template <int MT, int PRO>
static int launch_pro(const CUtensorMap& tw, const CUtensorMap& ts, const CUtensorMap& tb, const Params& p, int G,
                      cudaStream_t st) {
  if constexpr (PRO == kProNone || PRO == kProRms) {
    if (p.pair) return launch_variant<MT, PRO, true>(tw, ts, tb, p, G, st);
  } else {
    if (p.pair) return QMTP_ERR_UNSUPPORTED;
  }
  return launch_variant<MT, PRO, false>(tw, ts, tb, p, G, st);
}

template <int MT>
static int launch_mt(const CUtensorMap& tw, const CUtensorMap& ts, const CUtensorMap& tb, const Params& p, int pro,
                     int G, cudaStream_t st) {
  switch (pro) {
    case kProRms: return launch_pro<MT, kProRms>(tw, ts, tb, p, G, st);
    case kProSwiglu: return launch_pro<MT, kProSwiglu>(tw, ts, tb, p, G, st);
    case kProGated: return launch_pro<MT, kProGated>(tw, ts, tb, p, G, st);
    default: return launch_pro<MT, kProNone>(tw, ts, tb, p, G, st);
  }
}

static int max_clusters(int cs) {
  static std::mutex mu;
  static int cache[2][64] = {};  // [cs == 4][device]: clusters + 1, 0 = not queried
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  std::lock_guard<std::mutex> lk(mu);
  int& c = cache[cs == 4 ? 1 : 0][dev];
  if (c == 0) {
    int n = 0;
    if (prepare<1, kProNone, false>()) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(unsigned(cs));
      cfg.blockDim = dim3(kThreads);
      cfg.dynamicSmemBytes = kSmem;
      cudaLaunchAttribute at[1];
      at[0].id = cudaLaunchAttributeClusterDimension;
      at[0].val.clusterDim.x = unsigned(cs);
      at[0].val.clusterDim.y = 1;
      at[0].val.clusterDim.z = 1;
      cfg.attrs = at;
      cfg.numAttrs = 1;
      if (cudaOccupancyMaxActiveClusters(&n, qmv_tc_kernel<1, kProNone, false>, &cfg) != cudaSuccess) {
        cudaGetLastError();
        n = 0;
      }
    }
    c = n + 1;
  }
  return c - 1;
}

}  // namespace tq

// All affine qmv entry points land here.
// Activation prologue of a call: pro (tq::kPro*), the norm weight and eps, the gate rows (kProGated).
struct QmvPro {
  int pro;
  const void* nw;
  float eps;
  const void* z;
  long long ldz;
};

int qmv_tc(const void* x, long long ldx, const void* w, const void* s, const void* b, void* y, const void* res,
           int M, int N, int K, int ldy, void* stream, const QmvPro& pr) {
  using namespace tq;
  if (!x || !w || !s || !b || !y) return QMTP_ERR_ARG;
  if (M < 1 || N < 1 || K < 512 || K % 512 != 0 || ldy < N) return QMTP_ERR_SHAPE;
  if (ldx == 0) ldx = pr.pro == kProSwiglu ? 2LL * K : K;
  if (!aligned16(x) || !aligned16(w) || !aligned16(s) || !aligned16(b)) return QMTP_ERR_ALIGN;
  switch (pr.pro) {
    case kProNone:
      if (ldx < K || ldx % 8) return QMTP_ERR_SHAPE;
      break;
    case kProRms:
      if (ldx < K || ldx % 8 || K % 1024 != 0 || K > 32768) return QMTP_ERR_SHAPE;
      if (!pr.nw) return QMTP_ERR_ARG;
      if (!aligned16(pr.nw)) return QMTP_ERR_ALIGN;
      break;
    case kProSwiglu:
      if (ldx < 2LL * K || ldx % 8) return QMTP_ERR_SHAPE;
      break;
    case kProGated:  // x: fp32 rows, ldx in floats; heads of 128
      if (ldx < K || ldx % 4 || pr.ldz < K || pr.ldz % 8) return QMTP_ERR_SHAPE;
      if (!pr.nw || !pr.z) return QMTP_ERR_ARG;
      if (!aligned16(pr.nw) || !aligned16(pr.z)) return QMTP_ERR_ALIGN;
      break;
    default:
      return QMTP_ERR_ARG;
  }
  const Plan pl = make_plan(N, K, sm_count(), pr.pro == kProNone || pr.pro == kProRms);
  if ((long long)pl.ntiles * (pl.G + 1) > kMaxUnitProduct || (long long)pl.ntiles * pl.NSL > kMaxUnitProduct)
    return QMTP_ERR_SHAPE;
  CUtensorMap tw, ts, tb;
  if (!encode_2d(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, w, K / 2, N, kBox, pl.R, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_2d(&ts, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, s, K / 64, N, 8, pl.R, CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !encode_2d(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, b, K / 64, N, 8, pl.R, CU_TENSOR_MAP_SWIZZLE_NONE))
    return QMTP_ERR_CUDA;
  Params p{};
  p.ldx = ldx;
  p.ldy = ldy;
  p.N = N;
  p.K = K;
  p.NSL = pl.NSL;
  p.R = pl.R;
  p.ntiles = pl.ntiles;
  p.cs = pl.cs;
  p.pair = pl.pair;
  p.nw = static_cast<const uint16_t*>(pr.nw);
  p.eps = pr.eps;
  p.ldz = pr.ldz;
  p.err = device_error_ptr();
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  for (int m0 = 0; m0 < M; m0 += kMaxTok) {
    const int mm = std::min(kMaxTok, M - m0);
    p.x = pr.pro == kProGated
              ? reinterpret_cast<const uint16_t*>(static_cast<const float*>(x) + (size_t)m0 * (size_t)ldx)
              : static_cast<const uint16_t*>(x) + (size_t)m0 * (size_t)ldx;
    p.z = pr.z ? static_cast<const uint16_t*>(pr.z) + (size_t)m0 * (size_t)pr.ldz : nullptr;
    p.y = static_cast<uint16_t*>(y) + (size_t)m0 * (size_t)ldy;
    p.res = res ? static_cast<const uint16_t*>(res) + (size_t)m0 * (size_t)ldy : nullptr;
    int rc;
    switch (mm) {
      case 1: rc = launch_mt<1>(tw, ts, tb, p, pr.pro, pl.G, st); break;
      case 2: rc = launch_mt<2>(tw, ts, tb, p, pr.pro, pl.G, st); break;
      case 3: rc = launch_mt<3>(tw, ts, tb, p, pr.pro, pl.G, st); break;
      default: rc = launch_mt<4>(tw, ts, tb, p, pr.pro, pl.G, st); break;
    }
    if (rc != QMTP_OK) return rc;
  }
  return QMTP_OK;
}

int qmv_tc_plan(int N, int K, int* rows, int* grid, int* units, int* cluster) {
  const tq::Plan pl = tq::make_plan(N, K, sm_count(), true);
  if (rows) *rows = pl.R;
  if (grid) *grid = pl.G;
  if (units) *units = int((long long)pl.ntiles * pl.NSL);
  if (cluster) *cluster = pl.cs;
  return QMTP_OK;
}

}  // namespace qmtp

using namespace qmtp;

extern "C" int qmtp_qmv_affine_g64(const void* x, const void* w, const void* scales, const void* biases, void* y,
                                   int M, int N, int K, int ldy, void* stream) {
  return qmv_tc(x, 0, w, scales, biases, y, nullptr, M, N, K, ldy, stream, QmvPro{tq::kProNone, nullptr, 0.0f, nullptr, 0});
}

extern "C" int qmtp_qmv_affine_g64_res(const void* x, const void* w, const void* scales, const void* biases, void* y,
                                       const void* res, int M, int N, int K, int ldy, void* stream) {
  if (!res) return QMTP_ERR_ARG;
  return qmv_tc(x, 0, w, scales, biases, y, res, M, N, K, ldy, stream, QmvPro{tq::kProNone, nullptr, 0.0f, nullptr, 0});
}

// The workspace of the _split / _norm entry points is no longer used: a tile shared between CTAs is
// finished inside their thread-block cluster.  The query keeps answering 256 bytes for every valid
// shape so that callers which allocate it keep working.
extern "C" size_t qmtp_qmv_workspace(int N, int K) {
  if (N < 1 || K < 512 || K % 512) return 0;
  return 256;
}

extern "C" int qmtp_qmv_affine_g64_split(const void* x, long long ldx, const void* w, const void* scales,
                                         const void* biases, void* y, const void* res, int M, int N, int K, int ldy,
                                         void* workspace, size_t ws_bytes, void* stream) {
  (void)workspace;
  (void)ws_bytes;
  return qmv_tc(x, ldx, w, scales, biases, y, res, M, N, K, ldy, stream, QmvPro{tq::kProNone, nullptr, 0.0f, nullptr, 0});
}

extern "C" int qmtp_qmv_affine_g64_norm(const void* x, long long ldx, const void* norm_w, float eps, const void* w,
                                        const void* scales, const void* biases, void* y, const void* res, int M,
                                        int N, int K, int ldy, void* workspace, size_t ws_bytes, void* stream) {
  (void)workspace;
  (void)ws_bytes;
  if (!norm_w) return QMTP_ERR_ARG;
  return qmv_tc(x, ldx, w, scales, biases, y, res, M, N, K, ldy, stream, QmvPro{tq::kProRms, norm_w, eps, nullptr, 0});
}

extern "C" int qmtp_qmv_affine_g64_swiglu(const void* gu, long long ldgu, const void* w, const void* scales,
                                          const void* biases, void* y, const void* res, int M, int N, int K, int ldy,
                                          void* stream) {
  return qmv_tc(gu, ldgu, w, scales, biases, y, res, M, N, K, ldy, stream,
                QmvPro{tq::kProSwiglu, nullptr, 0.0f, nullptr, 0});
}

extern "C" int qmtp_qmv_affine_g64_gated(const float* yg, long long ldyg, const void* z, long long ldz,
                                         const void* norm_w, float eps, const void* w, const void* scales,
                                         const void* biases, void* y, const void* res, int M, int N, int K, int ldy,
                                         void* stream) {
  return qmv_tc(yg, ldyg, w, scales, biases, y, res, M, N, K, ldy, stream,
                QmvPro{tq::kProGated, norm_w, eps, z, ldz});
}

extern "C" int qmtp_qmv_set_mode(int mode) {
  if (mode < 0 || mode > 2) return QMTP_ERR_ARG;
  tq::g_mode.store(mode, std::memory_order_relaxed);
  return QMTP_OK;
}

extern "C" int qmtp_qmv_plan(int N, int K, int split, int* rows_per_tile, int* grid, int* units, int* cluster) {
  (void)split;
  if (N < 1 || K < 512 || K % 512) return QMTP_ERR_SHAPE;
  return qmv_tc_plan(N, K, rows_per_tile, grid, units, cluster);
}
