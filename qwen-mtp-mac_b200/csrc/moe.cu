// MXFP4 / NVFP4 mixture-of-experts decode on B200: the batched form of moe_decode
// (experiments/deepseek_moe/kernels.py:133-155) for T concurrent tokens.
//
//   h[t,j] = silu(min(Wg[e] x_t, L)) * clamp(Wu[e] x_t, -L, L)          e = idx[t,j]  (kernels.py:35-74)
//   y[t]   = sum_j scores[t,j] * Wd[e] h[t,j]                                          (kernels.py:76-107)
//
// Weights keep the reference layout: uint32 [E, N, K/8] (8 e2m1 nibbles, low nibble = lowest k) and
// uint8 scales [E, N, K/G] (MXFP4: e8m0, G = 32; NVFP4: e4m3 with the sign ignored, G = 16).
//
// Pipeline (one stream, each kernel a programmatic dependent of the previous one):
//   moe_group    one CTA: stable counting sort of the T*S (token, slot) entries by expert, cut into
//                token tiles of <= 64 entries; writes the tile table.
//   moe_gather   per tile row: the token's x as an f16 operand image (canonical K-major core-matrix
//                layout of the tensor core, 128 K per chunk), scaled by a per-token power of two.
//   moe_gemm<GU> persistent, one CTA per SM; a unit = (tile, 128 weight rows).  Warp roles:
//                  warp 0      TMA producer of the weight ring (2-D, 64-B swizzle) and the unit's scales;
//                  warp 2      producer of the operand-image ring (1-D bulk copies);
//                  warp 1      tcgen05.mma issuer (M = 128, N = tile tokens, K = 16 per instruction),
//                              A operand read from TMEM, B operand from shared memory;
//                  warps 4-19  dequantizers: packed e2m1 + scale -> f16 (gate/up) or bf16 (down) in
//                              registers, tcgen05.st into TMEM;
//                  warps 20-23 epilogue: accumulators -> SwiGLU h (gate/up) or fp32 partials (down).
//                gate/up writes h split as hi = bf16(h), lo = bf16(h - hi) (h to ~16 significant bits,
//                the reference keeps h in fp32, kernels.py:146) straight into the down operand image;
//                down multiplies the same weights by hi and lo and writes per-entry fp32 partials.
//   moe_combine  y[t] = sum_j scores[t,j] * partial[t,j] in slot order, rounded to bf16.
//
// Dequantization.  gate/up uses f16 operands: each byte of a word goes through the hardware
// e2m1x2 -> f16x2 conversion and one f16x2 multiply by the block factor (no integer bit work, which
// keeps the dequantizers off the integer pipe).  NVFP4 factors (e4m3 * 2^-8) are always exact in f16;
// MXFP4 factors are taken relative to the row's largest scale so they fit f16, and the epilogue
// restores the row's power of two.  down uses bf16 operands (h needs bf16's range): e2m1 magnitudes
// are placed as bf16 encodings of v * 2^-126 and multiplied by 2^126 * scale with one mul.rn.bf16x2
// per element pair (two multiplies when that factor exceeds bf16 range); its nibbles are laid out as
// pairs (0,4), (1,5), (2,6), (3,7), and the h operand image uses the same permutation of every 8 k.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"

namespace qmtp {
namespace moe {

constexpr int kRows = 128;                   // weight rows per unit (MMA M)
constexpr int kChunk = 128;                  // K per pipeline stage
constexpr int kMaxTok = 64;                  // entries per token tile (MMA N <= 64)
constexpr int kWBytes = kRows * kChunk / 2;  // packed bytes of one 128 x 128 weight tile
constexpr int kMaxW = 8;                     // weight ring stages (upper bound; chosen per launch)
constexpr int kNB = 4;                       // operand-image ring stages (= depth of the stage-done ring)
constexpr int kDQ = 4;                       // dequantizing warps per TMEM lane quarter
constexpr int kNDQ = 4 * kDQ;
constexpr int kWarps = 4 + kNDQ + 4;         // 4 control warps, dequantizers, 4 epilogue warps
constexpr int kThreads = kWarps * 32;
constexpr unsigned kTmemCols = 512;
constexpr uint32_t kWaitPolls = 1u << 20;    // bound of every mbarrier wait (normal waits end in microseconds)
constexpr int kSmemMax = 227 * 1024;

struct Tile {
  int expert, entry0, ntok, nt, row0, pad0, pad1, pad2;
};

template <bool GU>
struct Cfg {
  static constexpr int NMAT = GU ? 2 : 1;
  static constexpr int WSTAGE = NMAT * kWBytes;
  static constexpr int BSTAGE = GU ? kMaxTok * 256 : kMaxTok * 512;  // operand-image bytes per stage
  // TMEM: two accumulator buffers of 128 columns (gate | up, or the hi | lo halves of N = 2*nt for down),
  // then four A slots of 64 columns (gate/up: one half-chunk of K = 64 per slot, 32 columns per matrix;
  // down: one chunk of K = 128 per slot).
  static constexpr int NA = 4;
  static constexpr int ACOLS = 64;
  static constexpr int ACC_STRIDE = 128;
  static constexpr int A_BASE = 2 * ACC_STRIDE;
  static_assert(A_BASE + NA * ACOLS <= (int)kTmemCols, "TMEM budget");
};

// Shared-memory map of one GEMM CTA (host and device compute it the same way).
struct SmemMap {
  int w, b, s, rs, bars, total;
};
__host__ __device__ inline SmemMap smem_map(bool gu, int nw, int sbuf) {
  SmemMap m;
  int o = 0;
  m.w = o;
  o += nw * (gu ? 2 * kWBytes : kWBytes);
  m.b = o;
  o += kNB * (gu ? kMaxTok * 256 : kMaxTok * 512);
  m.s = o;
  o += 2 * sbuf;
  m.rs = o;
  o += 2 * 2 * kRows * 4;  // row exponents [unit parity][matrix][row]
  m.bars = o;
  o += 512;
  m.total = o + 1024;  // alignment slack
  return m;
}

// --------------------------------------------------------------------------- exact fp4 -> bf16
// Scale byte -> bf16x2 multipliers.  Fast path: mult = 2^126 * scale fits bf16.  Slow path (rare):
// multiply by 2^126 first, then by mult2 = scale.
struct Mult {
  uint32_t m, m2;
  bool slow;
};
__device__ __forceinline__ Mult mult_e8m0(uint32_t s) {
  Mult r;
  r.slow = s > 128u;
  r.m = ((s + 126u) << 7) * 0x00010001u;
  r.m2 = (s == 0 ? 0x0040u : s << 7) * 0x00010001u;  // 2^(s-127); s = 0 is the bf16 subnormal 2^-127
  return r;
}
__device__ __forceinline__ Mult mult_e4m3(uint32_t s) {
  const uint32_t c = s & 0x7Fu;
  const float f = c >= 8u ? __uint_as_float((c << 20) + (120u << 23)) : __fmul_rn(float(c), 0.001953125f);
  Mult r;
  r.slow = c >= 0x48u;  // e4m3 >= 4: 2^126 * scale overflows bf16
  r.m = (r.slow ? 0u : (__float_as_uint(__fmul_rn(f, 0x1p126f)) >> 16)) * 0x00010001u;
  r.m2 = (__float_as_uint(f) >> 16) * 0x00010001u;
  return r;
}
// One word (8 nibbles) -> 4 bf16x2: pairs (0,4), (1,5), (2,6), (3,7).  `fast`: one multiply by
// 2^126 * scale; `wide`: multiply by 2^126 first, then by the scale (every scale byte).
__device__ __forceinline__ void fp4_word_mags(uint32_t w, uint32_t (&m)[4]) {
  const uint32_t y = w >> 8;
  m[0] = ((w & 0x000F000Fu) * 0x1040u) & 0x81C081C0u;
  m[1] = ((w & 0x00F000F0u) * 0x0104u) & 0x81C081C0u;
  m[2] = ((y & 0x000F000Fu) * 0x1040u) & 0x81C081C0u;
  m[3] = ((y & 0x00F000F0u) * 0x0104u) & 0x81C081C0u;
}
__device__ __forceinline__ void fp4_word_fast(uint32_t w, uint32_t mult, uint32_t* r) {
  uint32_t m[4];
  fp4_word_mags(w, m);
#pragma unroll
  for (int i = 0; i < 4; ++i) r[i] = mul_bf16x2(m[i], mult);
}
__device__ __forceinline__ void fp4_word_wide(uint32_t w, uint32_t scale, uint32_t* r) {
  uint32_t m[4];
  fp4_word_mags(w, m);
#pragma unroll
  for (int i = 0; i < 4; ++i) r[i] = mul_bf16x2(mul_bf16x2(m[i], 0x7E807E80u), scale);
}
// f16 path (gate/up): hardware e2m1x2 -> f16x2 conversion of each byte (element pair (2b, 2b+1), low
// nibble in the low half), then one f16x2 multiply by the scale factor.  Natural k order.
__device__ __forceinline__ void fp4_word_f16(uint32_t w, uint32_t mult, uint32_t* r) {
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t.reg .b32 t0, t1, t2, t3;\n\t"
      "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
      "cvt.rn.f16x2.e2m1x2 t0, b0;\n\tcvt.rn.f16x2.e2m1x2 t1, b1;\n\t"
      "cvt.rn.f16x2.e2m1x2 t2, b2;\n\tcvt.rn.f16x2.e2m1x2 t3, b3;\n\t"
      "mul.rn.f16x2 %0, t0, %5;\n\tmul.rn.f16x2 %1, t1, %5;\n\t"
      "mul.rn.f16x2 %2, t2, %5;\n\tmul.rn.f16x2 %3, t3, %5;\n\t}"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
      : "r"(w), "r"(mult));
}
// f16 factor of an MXFP4 block (scale byte s) inside a row whose largest scale byte is smax:
// 2^(s - smax + 13), so |e2m1 * factor| <= 6 * 2^13 fits f16; the row's outputs are multiplied by
// 2^(smax - 140) in the epilogue.  Blocks 2^28 or more below the row's largest become f16 subnormal.
__device__ __forceinline__ uint32_t mult_mx_f16(uint32_t s, int smax) {
  const int me = int(s) - smax + 28;  // biased f16 exponent of the factor
  const uint32_t bits = me >= 1 ? uint32_t(me) << 10 : (me >= -9 ? 1u << (me + 9) : 0u);
  return bits * 0x00010001u;
}
// NVFP4 factor: e4m3 magnitude as f16 bits (s & 0x7f) << 7 = scale * 2^-8 (qmv_kernel.py:26-28 trick);
// outputs are multiplied by 2^8 in the epilogue.  e2m1 * e4m3 * 2^-8 is always exact in f16.
__device__ __forceinline__ uint32_t mult_nv_f16(uint32_t s) { return ((s & 0x7Fu) << 7) * 0x00010001u; }

// Position of element k (0..7) of a word inside its permuted 8-group.
__host__ __device__ __forceinline__ int perm8(int k) { return ((k & 3) << 1) | (k >> 2); }

// --------------------------------------------------------------------------- quantizer
// Bit-identical to the C oracle's qo_quantize_fp4 (OCP MX v1.0 sec. 6.3 for MXFP4; e4m3(amax/6)
// scale for NVFP4).  One thread per group.
__device__ __forceinline__ uint32_t e2m1_code(float v) {
  const float a = fabsf(v);
  uint32_t c = 0;
  if (a > 0.25f) c = 1;
  if (a >= 0.75f) c = 2;
  if (a > 1.25f) c = 3;
  if (a >= 1.75f) c = 4;
  if (a > 2.5f) c = 5;
  if (a >= 3.5f) c = 6;
  if (a > 5.0f) c = 7;
  if (c && (__float_as_uint(v) >> 31)) c |= 8u;
  return c;
}
__device__ __forceinline__ int ilogb_pos(float f) {  // f > 0, finite
  const uint32_t u = __float_as_uint(f);
  const int e = int((u >> 23) & 0xFFu);
  if (e) return e - 127;
  return (31 - __clz(int(u & 0x7FFFFFu))) - 149;
}
__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  return uint32_t(__half_as_ushort(__float2half_rn(lo))) | (uint32_t(__half_as_ushort(__float2half_rn(hi))) << 16);
}
__device__ __forceinline__ float e4m3_value(uint32_t s) {
  const uint32_t c = s & 0x7Fu;
  return c >= 8u ? __uint_as_float((c << 20) + (120u << 23)) : __fmul_rn(float(c), 0.001953125f);
}
__device__ __forceinline__ uint32_t e4m3_code(float f) {
  if (!(f > 0.0f)) return 0;
  if (f > 448.0f) return 0x7E;
  int e = ilogb_pos(f);
  if (e < -6) return uint32_t(rintf(__fmul_rn(f, 512.0f)));
  const float mant = __uint_as_float((__float_as_uint(f) & 0x7FFFFFu) | 0x3F800000u);
  uint32_t m = uint32_t(rintf(__fmul_rn(__fsub_rn(mant, 1.0f), 8.0f)));
  if (m == 8u) { m = 0; e += 1; }
  const uint32_t c = (uint32_t(e + 7) << 3) | m;
  return c > 0x7Eu ? 0x7Eu : c;
}
__global__ void quantize_fp4_kernel(int fmt, const uint16_t* __restrict__ w, long long N, int K,
                                    uint32_t* __restrict__ wq, uint8_t* __restrict__ sc) {
  pdl_wait();
  pdl_trigger();
  const int G = fmt == 0 ? 32 : 16;
  const int gpr = K / G;
  const long long gid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (gid >= N * gpr) return;
  const long long n = gid / gpr;
  const int g = int(gid % gpr);
  const uint16_t* wr = w + n * K + (long long)g * G;
  float v[32];
  float amax = 0.0f;
  for (int i = 0; i < G; ++i) {
    v[i] = bf2f(wr[i]);
    amax = fmaxf(amax, fabsf(v[i]));
  }
  uint32_t s;
  float mul = 0.0f, div = 0.0f;
  if (fmt == 0) {
    int se = amax > 0.0f ? ilogb_pos(amax) - 2 + 127 : 0;
    s = uint32_t(se < 0 ? 0 : se > 254 ? 254 : se);
    mul = s == 0 ? __uint_as_float(0x7F000000u) : __uint_as_float((254u - s) << 23);
  } else {
    s = e4m3_code(__fdiv_rn(amax, 6.0f));
    div = e4m3_value(s);
  }
  sc[n * gpr + g] = uint8_t(s);
  for (int i = 0; i < G; i += 8) {
    uint32_t word = 0;
    for (int j = 0; j < 8; ++j) {
      const float x = v[i + j];
      const float q = fmt == 0 ? __fmul_rn(x, mul) : (div > 0.0f ? __fdiv_rn(x, div) : 0.0f);
      word |= e2m1_code(q) << (4 * j);
    }
    wq[n * (K / 8) + (g * G + i) / 8] = word;
  }
}

// --------------------------------------------------------------------------- router
// One warp per token: top-k of E <= 1024 logits (larger first, ties to the lower id, NaN lowest),
// weights = softmax over the chosen k (the oracle's qo_moe_route sequence), then shared experts.
__device__ __forceinline__ uint32_t logit_key(float f) {
  if (f != f) return 0;
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__global__ void moe_route_kernel(const float* __restrict__ logits, int T, int E, int top_k, int n_shared,
                                 float routed_scale, int32_t* __restrict__ idx, float* __restrict__ scores) {
  pdl_wait();
  pdl_trigger();
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (t >= T) return;
  const float* l = logits + (long long)t * E;
  uint64_t cand[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const int e = lane + 32 * i;
    cand[i] = e < E ? (uint64_t(logit_key(l[e])) << 32) | uint64_t(0xFFFFFFFFu - uint32_t(e)) : 0ull;
  }
  const int S = top_k + n_shared;
  int sel[16];
  for (int j = 0; j < top_k; ++j) {
    uint64_t best = 0;
#pragma unroll
    for (int i = 0; i < 32; ++i) best = cand[i] > best ? cand[i] : best;
#pragma unroll
    for (int d = 16; d >= 1; d >>= 1) {
      const uint64_t o = __shfl_xor_sync(0xFFFFFFFFu, best, d);
      best = o > best ? o : best;
    }
    const int e = int(0xFFFFFFFFu - uint32_t(best & 0xFFFFFFFFu));
    sel[j] = e;
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (lane + 32 * i == e) cand[i] = 0ull;
  }
  if (lane == 0) {
    float ex[16];
    float sum = 0.0f;
    const float top = l[sel[0]];
    for (int j = 0; j < top_k; ++j) {
      ex[j] = q_expf(__fsub_rn(l[sel[j]], top));
      sum = j == 0 ? ex[0] : __fadd_rn(sum, ex[j]);
    }
    for (int j = 0; j < top_k; ++j) {
      idx[(long long)t * S + j] = sel[j];
      scores[(long long)t * S + j] = __fmul_rn(__fdiv_rn(ex[j], sum), routed_scale);
    }
    for (int j = 0; j < n_shared; ++j) {
      idx[(long long)t * S + top_k + j] = E + j;
      scores[(long long)t * S + top_k + j] = 1.0f;
    }
  }
}

// --------------------------------------------------------------------------- grouping
// One CTA of 1024 threads.  Entry i = t*S + j.  Warp w owns a contiguous segment of entries; within
// a warp, peers with the same expert are ranked by lane (match_any); a per-(warp, expert) count
// table turns that into a stable global order: pos = offset[e] + before[w][e] + rank.  So experts
// are laid out in id order and, within an expert, entries in (token, slot) order.
__global__ void __launch_bounds__(1024) moe_group_kernel(const int32_t* __restrict__ idx, int n, int S, int E,
                                                         int32_t* __restrict__ entry_pos,
                                                         int32_t* __restrict__ sorted_tok,
                                                         int32_t* __restrict__ rank_tmp, Tile* __restrict__ tiles,
                                                         int32_t* __restrict__ counters, unsigned* err) {
  extern __shared__ uint16_t cnt16[];  // [32][E]
  __shared__ int s_warp[32];
  __shared__ int s_eoff[1024];
  pdl_wait();
  pdl_trigger();
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  for (int i = tid; i < 32 * E; i += blockDim.x) cnt16[i] = 0;
  __syncthreads();
  const int L = (n + 31) / 32;
  const int seg0 = min(n, warp * L), seg1 = min(n, seg0 + L);
  for (int b = seg0; b < seg1; b += 32) {
    const int i = b + lane;
    int e = -1;
    if (i < seg1) {
      e = idx[i];
      if (e < -1 || e >= E) {  // -1: an empty row (padding of a fixed-capacity dispatch), skipped
        if (err) atomicOr(err, DEVERR_BADARG);
        e = -1;
      }
    }
    const unsigned peers = __match_any_sync(0xFFFFFFFFu, e);
    const int rank = __popc(peers & ((1u << lane) - 1u));
    int base = 0;
    if (e >= 0) base = cnt16[warp * E + e];
    __syncwarp();
    if (e >= 0 && rank == 0) cnt16[warp * E + e] = uint16_t(base + __popc(peers));
    __syncwarp();
    if (i < seg1) rank_tmp[i] = e >= 0 ? base + rank : -1;
  }
  __syncthreads();
  int cnt = 0;
  if (tid < E) {
    for (int w = 0; w < 32; ++w) {
      const int c = cnt16[w * E + tid];
      cnt16[w * E + tid] = uint16_t(cnt);
      cnt += c;
    }
  }
  const int ntile = (cnt + kMaxTok - 1) / kMaxTok;
  const int last = cnt - kMaxTok * (ntile - 1);
  const int prow = ntile ? kMaxTok * (ntile - 1) + ((last + 15) & ~15) : 0;
  int tot_e, tot_t, tot_r;
  const int eoff = block_excl_scan(cnt, s_warp, tot_e);
  const int etile = block_excl_scan(ntile, s_warp, tot_t);
  const int erow = block_excl_scan(prow, s_warp, tot_r);
  if (tid < E) {
    s_eoff[tid] = eoff;
    for (int j = 0; j < ntile; ++j) {
      Tile tl;
      tl.expert = tid;
      tl.entry0 = eoff + kMaxTok * j;
      tl.ntok = min(kMaxTok, cnt - kMaxTok * j);
      tl.nt = (tl.ntok + 15) & ~15;
      tl.row0 = erow + kMaxTok * j;
      tl.pad0 = tl.pad1 = tl.pad2 = 0;
      tiles[etile + j] = tl;
    }
  }
  if (tid == 0) {
    counters[0] = tot_t;
    counters[1] = tot_r;
    counters[2] = tot_e;
  }
  __syncthreads();
  for (int b = seg0; b < seg1; b += 32) {
    const int i = b + lane;
    if (i < seg1) {
      const int r = rank_tmp[i];
      if (r >= 0) {
        const int e = idx[i];
        const int pos = s_eoff[e] + cnt16[warp * E + e] + r;
        entry_pos[i] = pos;
        sorted_tok[pos] = i / S;
      } else {
        entry_pos[i] = -1;
      }
    }
  }
}

// --------------------------------------------------------------------------- operand image of x
// Tile image (f16, natural k order): K/128 chunks of nt x 128; inside a chunk, core matrix (k8, row8)
// at ((k8 * nt/8) + row8) * 128 bytes, row r & 7 at 16-B steps.  One warp per tile row.  Each token row
// is scaled by 2^-k (k = max(0, ilogb(max|x|) - 14)) so every value fits f16; k goes to xsh[entry]
// and the gate/up epilogue multiplies by 2^k.  bf16 -> f16 is exact for |x| >= 2^-17 after scaling.
__global__ void moe_gather_kernel(const uint16_t* __restrict__ x, int H, const Tile* __restrict__ tiles,
                                  const int32_t* __restrict__ counters, const int32_t* __restrict__ sorted_tok,
                                  uint8_t* __restrict__ ximg, int32_t* __restrict__ xsh) {
  pdl_wait();
  pdl_trigger();
  if (int(blockIdx.x) >= counters[0]) return;
  const Tile tl = tiles[blockIdx.x];
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.y * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= tl.nt) return;
  const int nt8 = tl.nt >> 3;
  uint8_t* base = ximg + (size_t)tl.row0 * H * 2 + (size_t)(row >> 3) * 128 + (row & 7) * 16;
  const int units = H >> 3;
  if (row >= tl.ntok) {
    for (int u = lane; u < units; u += 32)
      *reinterpret_cast<uint4*>(base + (size_t)u * nt8 * 128) = make_uint4(0u, 0u, 0u, 0u);
    return;
  }
  const uint4* xr = reinterpret_cast<const uint4*>(x + (size_t)sorted_tok[tl.entry0 + row] * H);
  float amax = 0.0f;
  for (int u = lane; u < units; u += 32) {
    const uint4 v = xr[u];
    amax = fmaxf(amax, fmaxf(fmaxf(fmaxf(fabsf(bflo(v.x)), fabsf(bfhi(v.x))), fmaxf(fabsf(bflo(v.y)), fabsf(bfhi(v.y)))),
                             fmaxf(fmaxf(fabsf(bflo(v.z)), fabsf(bfhi(v.z))), fmaxf(fabsf(bflo(v.w)), fabsf(bfhi(v.w))))));
  }
#pragma unroll
  for (int d = 16; d >= 1; d >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, d));
  const int k = (amax > 0.0f && amax <= 3.4e38f) ? max(0, ilogb_pos(amax) - 14) : 0;
  const float sc = __uint_as_float(uint32_t(127 - k) << 23);
  if (lane == 0) xsh[tl.entry0 + row] = k;
  for (int u = lane; u < units; u += 32) {
    const uint4 v = xr[u];
    uint4 o;
    o.x = pack_half2(__fmul_rn(bflo(v.x), sc), __fmul_rn(bfhi(v.x), sc));
    o.y = pack_half2(__fmul_rn(bflo(v.y), sc), __fmul_rn(bfhi(v.y), sc));
    o.z = pack_half2(__fmul_rn(bflo(v.z), sc), __fmul_rn(bfhi(v.z), sc));
    o.w = pack_half2(__fmul_rn(bflo(v.w), sc), __fmul_rn(bfhi(v.w), sc));
    *reinterpret_cast<uint4*>(base + (size_t)u * nt8 * 128) = o;
  }
}

// --------------------------------------------------------------------------- grouped GEMM
struct GemmArgs {
  const uint8_t* sa;      // scales of matrix 0 [E*R, KS] (1-D bulk copies when not staged by tensor maps)
  const uint8_t* sb;      // gate/up: scales of matrix 1
  const uint8_t* bimg;    // operand images: x (gate/up, f16) or h hi|lo (down, bf16)
  const Tile* tiles;
  const int32_t* counters;
  const int32_t* xsh;     // gate/up: per-entry exponent of the activation downscale
  uint8_t* himg;          // gate/up output: h operand images for down
  float* yp;              // down output: per-entry fp32 partials [n, R]
  const int32_t* out_row; // down: optional row of yp for each sorted entry (nullptr = the entry itself)
  int K;                  // reduction length
  int R;                  // weight rows per expert
  int KS;                 // scale bytes per weight row
  int fmt;                // 0 MXFP4, 1 NVFP4
  float limit;            // SwiGLU clamp (+inf = off)
  int h_rows;             // gate/up: K of the down GEMM (= R)
  int nw;                 // weight ring stages
  int sbuf;               // bytes of one scale buffer
  int sbox;               // gate/up: scales staged in 16-byte TMA boxes (KS % 16 == 0), else as rows
  unsigned* err;          // library device error word
};

struct Bars {
  uint64_t wfull[kMaxW], wempty[kMaxW];
  uint64_t bfull[kNB];
  uint64_t sdone[kNB];  // stage done: all MMAs of K-chunk `it` completed (frees its operand slot and A slots)
  uint64_t afull[4];
  uint64_t sfull[2], sempty[2];
  uint64_t accfull[2], accempty[2];
  uint64_t rsfull[2], rsempty[2];
  uint64_t drain;
  uint32_t tmem;
  int abort;
};
static_assert(sizeof(Bars) <= 512, "barrier block");

// MMA issue without a "memory" clobber: the operands are ordered by the barrier waits (volatile asm with
// clobbers) and tcgen05 fences around the issue loop; a clobber here would make the compiler reload
// values from memory between consecutive MMAs and roughly double the issue time.
__device__ __forceinline__ void umma_ts_first(uint32_t d, uint32_t a, uint64_t b, uint32_t idesc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, 0, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d),
      "r"(a), "l"(b), "r"(idesc));
}
__device__ __forceinline__ void umma_ts_acc(uint32_t d, uint32_t a, uint64_t b, uint32_t idesc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, 1, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d),
      "r"(a), "l"(b), "r"(idesc));
}

// Warp roles: 0 weight/scale producer, 1 and 3 MMA issuers, 2 operand-image producer,
// 4 .. 4+kNDQ-1 dequantizers (lane quarter dw & 3, sub-task dw >> 2), last 4 epilogue.
// Pacing: MMA issue is the critical resource (a kind::f16 MMA costs its issuing thread ~50 cycles for
// N <= 64, whatever the operand sizes; two issuing threads double the rate), so everything else runs
// ahead of it: the weight ring by up to nw chunks, the operand ring by kNB chunks,
// and the dequantizers by two chunks (gate/up: K-chunk `it` uses A slots 2*(it%2) + {0,1}, one per half
// of K, and is written once chunk it-2 is done; down: chunk `it` uses slot it%4, written once chunk it-4
// is done).  One commit per chunk and issuer (sdone, count 2) releases its operand slot and A slots.
// The issuer waits on one barrier per chunk (afull of the chunk's first A slot).  Timestamps of the
// issuing thread show each of its waits taking ~0.2 us in this kernel even when the phase has already
// completed, so each dequantizer warp announces its A share once per chunk (both K halves), and only
// after it has itself seen the chunk's operand image land (bfull): the operand-ring wait and the second
// A wait are off the issuer's path (gate/up 1.20 -> 1.08 us per chunk).
// Gate/up: f16 MMA, dequantizer sub-task = (matrix, chunk j of each K half).  Down: bf16 MMA with
// N = 2*nt (hi rows then lo rows of h), sub-task = one 32-element chunk.
template <bool GU>
__global__ void __launch_bounds__(kThreads, 1)
    moe_gemm_kernel(const __grid_constant__ CUtensorMap tw0, const __grid_constant__ CUtensorMap tw1,
                    const __grid_constant__ CUtensorMap ts0, const __grid_constant__ CUtensorMap ts1, GemmArgs a) {
  using C = Cfg<GU>;
  extern __shared__ uint8_t dsm_raw[];
  uint8_t* dsm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dsm_raw) + 1023) & ~uintptr_t(1023));
  const SmemMap map = smem_map(GU, a.nw, a.sbuf);
  uint8_t* wring = dsm + map.w;
  uint8_t* bring = dsm + map.b;
  uint8_t* sbufs = dsm + map.s;
  int* rsx = reinterpret_cast<int*>(dsm + map.rs);  // [2][2][128]
  Bars* bars = reinterpret_cast<Bars*>(dsm + map.bars);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  unsigned* err = a.err;
  const int NW = a.nw;

  if (tid == 0) {
    for (int s = 0; s < NW; ++s) {
      mbar_init(&bars->wfull[s], 1);
      mbar_init(&bars->wempty[s], kNDQ);
    }
    for (int s = 0; s < kNB; ++s) {
      mbar_init(&bars->bfull[s], 1);
      mbar_init(&bars->sdone[s], 2);  // one commit from each MMA issuer
    }
    for (int s = 0; s < C::NA; ++s) mbar_init(&bars->afull[s], kNDQ);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars->sfull[s], 1);
      mbar_init(&bars->sempty[s], kNDQ);
      mbar_init(&bars->accfull[s], 2);
      mbar_init(&bars->accempty[s], 4);
      mbar_init(&bars->rsfull[s], kNDQ);
      mbar_init(&bars->rsempty[s], 4);
    }
    mbar_init(&bars->drain, 2);
    bars->abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(&bars->tmem, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem;
  volatile int* abort_flag = &bars->abort;

  pdl_wait();
  pdl_trigger();
  const int RT = a.R / kRows;
  const int total = a.counters[0] * RT;
  const int nchunk = a.K / kChunk;
  const int KS = a.KS;
  // chunk j done <=> phase (j / kNB) of sdone[j % kNB] completed
  auto wait_done = [&](int j) -> bool {
    return j < 0 || mbar_wait_backoff(&bars->sdone[j % kNB], (j / kNB) & 1, err, 64);
  };

  if (warp == 0) {
    // ----------------------------------------------------------------- weight + scale producer
    if (lane == 0) {
      const uint64_t pol_w = policy_evict_first();
      int it = 0, lu = 0, ws = 0;
      uint32_t wph = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < total && ok; u += gridDim.x, ++lu) {
        const Tile tl = a.tiles[u / RT];
        const int row = tl.expert * a.R + (u % RT) * kRows;
        const int sb = lu & 1;
        if (*abort_flag || !(ok = mbar_wait_backoff(&bars->sempty[sb], ((lu >> 1) & 1) ^ 1, err, 128))) break;
        uint8_t* sdst = sbufs + sb * a.sbuf;
        if (GU) {
          mbar_expect_tx(&bars->sfull[sb], uint32_t(2 * kRows * KS));
          if (a.sbox) {
            for (int m = 0; m < 2; ++m)
              for (int bx = 0; bx < KS / 16; ++bx)
                tma_load_2d(sdst + m * kRows * KS + bx * (kRows * 16), m ? (const void*)&ts1 : (const void*)&ts0,
                            bx * 16, row, &bars->sfull[sb], pol_w);
          } else {
            bulk_g2s(sdst, a.sa + (size_t)row * KS, uint32_t(kRows * KS), &bars->sfull[sb], pol_w);
            bulk_g2s(sdst + kRows * KS, a.sb + (size_t)row * KS, uint32_t(kRows * KS), &bars->sfull[sb], pol_w);
          }
        } else {
          mbar_expect_tx(&bars->sfull[sb], uint32_t(kRows * KS));
          bulk_g2s(sdst, a.sa + (size_t)row * KS, uint32_t(kRows * KS), &bars->sfull[sb], pol_w);
        }
        for (int c = 0; c < nchunk; ++c, ++it, ws = ws + 1 == NW ? 0 : ws + 1, wph ^= ws == 0 ? 1u : 0u) {
          const int s = ws;  // it % NW, phase (it / NW) & 1, kept incrementally
          if (*abort_flag || !mbar_wait_backoff(&bars->wempty[s], wph ^ 1u, err, 128)) { ok = false; break; }
          uint8_t* st = wring + s * C::WSTAGE;
          mbar_expect_tx(&bars->wfull[s], uint32_t(C::WSTAGE));
          tma_load_2d(st, &tw0, c * (kChunk / 2), row, &bars->wfull[s], pol_w);
          if (GU) tma_load_2d(st + kWBytes, &tw1, c * (kChunk / 2), row, &bars->wfull[s], pol_w);
        }
      }
      if (!ok) {
        *abort_flag = 1;
        for (int k = 1; k <= NW && it - k >= 0; ++k) {
          const int j = it - k;
          mbar_wait_backoff(&bars->wfull[j % NW], (j / NW) & 1, err, 128);
        }
        for (int k = 1; k <= 2 && lu - k >= 0; ++k) {
          const int j = lu - k;
          mbar_wait_backoff(&bars->sfull[j & 1], (j >> 1) & 1, err, 128);
        }
      }
    }
  } else if (warp == 2) {
    // ----------------------------------------------------------------- operand-image producer
    if (lane == 0) {
      const uint64_t pol_b = policy_evict_last();
      int it = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < total && ok; u += gridDim.x) {
        const Tile tl = a.tiles[u / RT];
        const uint32_t bbytes = uint32_t(tl.nt * (GU ? 256 : 512));
        const uint8_t* bsrc = a.bimg + (size_t)tl.row0 * a.K * (GU ? 2 : 4);
        for (int c = 0; c < nchunk; ++c, ++it) {
          const int s = it % kNB;
          if (*abort_flag || !wait_done(it - kNB)) { ok = false; break; }
          mbar_expect_tx(&bars->bfull[s], bbytes);
          bulk_g2s(bring + s * C::BSTAGE, bsrc + (size_t)c * bbytes, bbytes, &bars->bfull[s], pol_b);
        }
      }
      if (!ok) {
        *abort_flag = 1;
        for (int k = 1; k <= kNB && it - k >= 0; ++k) {
          const int j = it - k;
          mbar_wait_backoff(&bars->bfull[j % kNB], (j / kNB) & 1, err, 128);
        }
      }
    }
  } else if (warp == 1 || warp == 3) {
    // ----------------------------------------------------------------- MMA issuers
    // A tcgen05.mma costs its issuing thread ~50 cycles, so two threads on different schedulers issue:
    // gate/up: issuer 0 the gate MMAs, issuer 1 the up MMAs; down: issuer 0 multiplies by the hi rows of
    // the operand chunk, issuer 1 by the lo rows, into the two halves of the accumulator.
    if (lane == 0) {
      const int iss = warp == 1 ? 0 : 1;
      int it = 0, lu = 0;
      bool ok = true, issued = false;
      for (int u = blockIdx.x; u < total && ok; u += gridDim.x, ++lu) {
        const Tile tl = a.tiles[u / RT];
        const int d = lu & 1;
        const int nt = tl.nt;
        const uint32_t idesc = GU ? umma_idesc_f16(128, nt) : umma_idesc_bf16(128, nt);
        // K-direction stride of the operand chunk: nt rows (gate/up) or 2*nt rows (down, hi then lo)
        const uint32_t lbo = uint32_t((GU ? nt : 2 * nt) / 8) * 128u;
        const uint32_t boff = GU ? 0u : uint32_t(iss * (nt / 8) * 128);
        if (*abort_flag || !(ok = mbar_wait_backoff(&bars->accempty[d], ((lu >> 1) & 1) ^ 1, err, 32))) break;
        tc_fence_after();
        const uint32_t dacc = tmem + uint32_t(d * C::ACC_STRIDE + (GU ? iss * 64 : iss * nt));
        for (int c = 0; c < nchunk; ++c, ++it) {
          const int s = it % kNB;
          // A of chunk `it` (gate/up: both K halves, slot pair 2*(it%2)) is announced only after the
          // dequantizers have also seen the operand chunk land, so this is the issuer's only wait
          const int ap = GU ? 2 * (it & 1) : it % C::NA;
          const uint32_t apar = GU ? uint32_t((it >> 1) & 1) : uint32_t((it / C::NA) & 1);
          if (*abort_flag || !mbar_wait_spin(&bars->afull[ap], apar, err)) { ok = false; break; }
          tc_fence_after();
          // descriptor of k-step 0 of this issuer's operand rows; k-step ks starts ks * 2 * lbo bytes later
          // (the start-address field holds address / 16 and stays below 2^14 for every smem address)
          const uint64_t bd0 = umma_desc(smem_u32(bring + s * C::BSTAGE) + boff, lbo, 128u);
          const uint64_t kstep = uint64_t((2u * lbo) >> 4);
          if (GU) {
            for (int h = 0; h < 2; ++h) {
              const uint32_t aA = tmem + uint32_t(C::A_BASE + (ap + h) * C::ACOLS + iss * 32);
              const uint64_t bh = bd0 + uint64_t(4 * h) * kstep;
              if (c == 0 && h == 0)
                umma_ts_first(dacc, aA, bh, idesc);
              else
                umma_ts_acc(dacc, aA, bh, idesc);
              umma_ts_acc(dacc, aA + 8, bh + kstep, idesc);
              umma_ts_acc(dacc, aA + 16, bh + 2 * kstep, idesc);
              umma_ts_acc(dacc, aA + 24, bh + 3 * kstep, idesc);
            }
          } else {
            const uint32_t aA = tmem + uint32_t(C::A_BASE + ap * C::ACOLS);
            if (c == 0)
              umma_ts_first(dacc, aA, bd0, idesc);
            else
              umma_ts_acc(dacc, aA, bd0, idesc);
#pragma unroll
            for (int ks = 1; ks < kChunk / 16; ++ks) umma_ts_acc(dacc, aA + ks * 8, bd0 + uint64_t(ks) * kstep, idesc);
          }
          issued = true;
          umma_commit(&bars->sdone[s]);
          if (c == nchunk - 1) umma_commit(&bars->accfull[d]);
        }
      }
      if (!ok) *abort_flag = 1;
      // every MMA issued has completed before TMEM is released (both issuers arrive on `drain`)
      if (issued) umma_commit(&bars->drain);
      else mbar_arrive(&bars->drain);
      mbar_wait_backoff(&bars->drain, 0, err, 64);
    }
  } else if (warp >= 4 && warp < 4 + kNDQ) {
    // ----------------------------------------------------------------- dequantizers
    const int dw = warp - 4, q = dw & 3, sub = dw >> 2;
    const int mat = GU ? sub >> 1 : 0;
    const int jj = sub & 1;  // gate/up: chunk jj of each K half (chunks jj and 2 + jj of the stage)
    const int r = q * 32 + lane;
    const int sw = (r >> 1) & 3;
    const uint32_t lane_base = tmem + (uint32_t(q * 32) << 16);
    int it = 0, lu = 0, ws = 0;
    uint32_t wph = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < total && ok; u += gridDim.x, ++lu) {
      const int sb = lu & 1, d = lu & 1;
      if (*abort_flag || !mbar_wait_backoff(&bars->sfull[sb], (lu >> 1) & 1, err, 64)) { ok = false; break; }
      const uint8_t* sbase = sbufs + sb * a.sbuf;
      int smax = 0;
      if (GU) {
        // this row's largest e8m0 byte (MXFP4), published with the NVFP4 constant for the epilogue
        int e_row = 8;
        if (a.fmt == 0) {
          uint32_t m = 0;
          if (a.sbox) {
            const uint8_t* rowp = sbase + mat * kRows * KS + r * 16;
            for (int bx = 0; bx < KS / 16; ++bx) {
              const uint4 v = *reinterpret_cast<const uint4*>(rowp + bx * (kRows * 16));
              m = __vmaxu4(m, __vmaxu4(__vmaxu4(v.x, v.y), __vmaxu4(v.z, v.w)));
            }
          } else {
            const uint8_t* rowp = sbase + mat * kRows * KS + r * KS;
            for (int j = 0; j < KS; j += 4) m = __vmaxu4(m, *reinterpret_cast<const uint32_t*>(rowp + j));
          }
          smax = int(max(max(m & 0xFFu, (m >> 8) & 0xFFu), max((m >> 16) & 0xFFu, m >> 24)));
          e_row = smax - 140;
        }
        if (!mbar_wait_backoff(&bars->rsempty[d], ((lu >> 1) & 1) ^ 1, err, 64)) { ok = false; break; }
        if (jj == 0) rsx[(d * 2 + mat) * kRows + r] = e_row;
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->rsfull[d]);
      }
      for (int c = 0; c < nchunk; ++c, ++it, ws = ws + 1 == NW ? 0 : ws + 1, wph ^= ws == 0 ? 1u : 0u) {
        const int s = ws;  // it % NW, phase (it / NW) & 1, kept incrementally
        if (*abort_flag || !mbar_wait_backoff(&bars->wfull[s], wph, err, 64)) { ok = false; break; }
        const uint8_t* wt = wring + s * C::WSTAGE + mat * kWBytes + r * 64;
        if (GU) {
          const uint4 w0 = *reinterpret_cast<const uint4*>(wt + 16 * (jj ^ sw));
          const uint4 w1 = *reinterpret_cast<const uint4*>(wt + 16 * ((2 + jj) ^ sw));
          // this row's scale bytes of the stage: MXFP4 4 (one per chunk), NVFP4 8 (two per chunk)
          const int j0 = a.fmt == 0 ? 4 * c : 8 * c;
          const uint8_t* sp = sbase + mat * kRows * KS + (a.sbox ? (j0 >> 4) * (kRows * 16) + r * 16 + (j0 & 15) : r * KS + j0);
          uint32_t s0, s1;
          if (a.fmt == 0) {
            s0 = *reinterpret_cast<const uint32_t*>(sp);
            s1 = 0;
          } else {
            const uint2 t2 = *reinterpret_cast<const uint2*>(sp);
            s0 = t2.x;
            s1 = t2.y;
          }
          __syncwarp();
          if (lane == 0) {
            mbar_arrive(&bars->wempty[s]);
            if (c == nchunk - 1) mbar_arrive(&bars->sempty[sb]);
          }
          if (!wait_done(it - 2)) { ok = false; break; }  // A slots of chunk it-2 are free again
          tc_fence_after();
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int ch = 2 * h + jj;
            const uint4 wv = h ? w1 : w0;
            uint32_t m0, m1;
            if (a.fmt == 0) {
              m0 = m1 = mult_mx_f16((s0 >> (8 * ch)) & 0xFFu, smax);
            } else {
              const uint32_t sw2 = ch < 2 ? s0 : s1;
              m0 = mult_nv_f16((sw2 >> (16 * (ch & 1))) & 0xFFu);
              m1 = mult_nv_f16((sw2 >> (16 * (ch & 1) + 8)) & 0xFFu);
            }
            uint32_t out[16];
            fp4_word_f16(wv.x, m0, out);
            fp4_word_f16(wv.y, m0, out + 4);
            fp4_word_f16(wv.z, m1, out + 8);
            fp4_word_f16(wv.w, m1, out + 12);
            const int ap = 2 * (it & 1) + h;
            tmem_st16(lane_base + uint32_t(C::A_BASE + ap * C::ACOLS + mat * 32 + jj * 16), out);
          }
          tmem_st_wait();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) {
            if (!mbar_wait_backoff(&bars->bfull[it % kNB], (it / kNB) & 1, err, 32)) *abort_flag = 1;
            mbar_arrive(&bars->afull[2 * (it & 1)]);
          }
        } else {
          const int ch = sub;
          const uint4 wv = *reinterpret_cast<const uint4*>(wt + 16 * (ch ^ sw));
          uint32_t sc;
          if (a.fmt == 0)
            sc = sbase[r * KS + 4 * c + ch];
          else
            sc = *reinterpret_cast<const uint16_t*>(sbase + r * KS + 8 * c + 2 * ch);
          __syncwarp();
          if (lane == 0) {
            mbar_arrive(&bars->wempty[s]);
            if (c == nchunk - 1) mbar_arrive(&bars->sempty[sb]);
          }
          if (!wait_done(it - C::NA)) { ok = false; break; }  // A slot of chunk it-4 is free again
          tc_fence_after();
          Mult m0, m1;
          if (a.fmt == 0) {
            m0 = m1 = mult_e8m0(sc & 0xFFu);
          } else {
            m0 = mult_e4m3(sc & 0xFFu);
            m1 = mult_e4m3((sc >> 8) & 0xFFu);
          }
          uint32_t out[16];
          if (!__any_sync(0xFFFFFFFFu, m0.slow || m1.slow)) {
            fp4_word_fast(wv.x, m0.m, out);
            fp4_word_fast(wv.y, m0.m, out + 4);
            fp4_word_fast(wv.z, m1.m, out + 8);
            fp4_word_fast(wv.w, m1.m, out + 12);
          } else {
            fp4_word_wide(wv.x, m0.m2, out);
            fp4_word_wide(wv.y, m0.m2, out + 4);
            fp4_word_wide(wv.z, m1.m2, out + 8);
            fp4_word_wide(wv.w, m1.m2, out + 12);
          }
          const int ap = it % C::NA;
          tmem_st16(lane_base + uint32_t(C::A_BASE + ap * C::ACOLS + ch * 16), out);
          tmem_st_wait();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) {
            if (!mbar_wait_backoff(&bars->bfull[it % kNB], (it / kNB) & 1, err, 32)) *abort_flag = 1;
            mbar_arrive(&bars->afull[ap]);
          }
        }
      }
    }
    if (!ok) *abort_flag = 1;
  } else if (warp >= 4 + kNDQ) {
    // ----------------------------------------------------------------- epilogue
    const int q = warp & 3, r = q * 32 + lane;
    const uint32_t lane_base = tmem + (uint32_t(q * 32) << 16);
    int lu = 0;
    for (int u = blockIdx.x; u < total; u += gridDim.x, ++lu) {
      const Tile tl = a.tiles[u / RT];
      const int rt = u % RT;
      const int d = lu & 1;
      if (*abort_flag || !mbar_wait_backoff(&bars->accfull[d], (lu >> 1) & 1, err, 256)) { *abort_flag = 1; break; }
      if (GU && !mbar_wait_backoff(&bars->rsfull[d], (lu >> 1) & 1, err, 256)) { *abort_flag = 1; break; }
      tc_fence_after();
      const uint32_t dacc = lane_base + uint32_t(d * C::ACC_STRIDE);
      if (GU) {
        const float fg = ldexpf(1.0f, rsx[(d * 2 + 0) * kRows + r]);
        const float fu = ldexpf(1.0f, rsx[(d * 2 + 1) * kRows + r]);
        // this row is k = rt*128 + r of the down GEMM: chunk rt, permuted position p; the down operand
        // chunk is [2*nt x 128]: rows 0..nt-1 carry hi(h), rows nt..2nt-1 carry lo(h)
        const int p = (r & ~7) | perm8(r & 7);
        const int n8 = (2 * tl.nt) >> 3;
        uint8_t* hb = a.himg + (size_t)tl.row0 * a.h_rows * 4 + (size_t)rt * tl.nt * 512 + (p >> 3) * n8 * 128 + (p & 7) * 2;
        for (int cg = 0; cg < tl.nt / 16; ++cg) {
          uint32_t g[16], v[16];
          tmem_ld16(dacc + uint32_t(cg * 16), g);
          tmem_ld16(dacc + 64u + uint32_t(cg * 16), v);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int n = cg * 16 + i;
            float hv = 0.0f;
            if (n < tl.ntok) {
              const float tf = ldexpf(1.0f, a.xsh[tl.entry0 + n]);
              const float gv = fminf(__fmul_rn(__fmul_rn(__uint_as_float(g[i]), fg), tf), a.limit);
              const float uv = fmaxf(fminf(__fmul_rn(__fmul_rn(__uint_as_float(v[i]), fu), tf), a.limit), -a.limit);
              hv = __fmul_rn(__fdiv_rn(gv, __fadd_rn(1.0f, q_expf(-gv))), uv);
            }
            const uint16_t hi = f2bf(hv);
            const uint16_t lo = f2bf(__fsub_rn(hv, bf2f(hi)));
            const int rl = n + tl.nt;
            *reinterpret_cast<uint16_t*>(hb + (n >> 3) * 128 + (n & 7) * 16) = hi;
            *reinterpret_cast<uint16_t*>(hb + (rl >> 3) * 128 + (rl & 7) * 16) = lo;
          }
        }
      } else {
        float* ycol = a.yp + rt * kRows + r;
        for (int cg = 0; cg < tl.nt / 16; ++cg) {
          uint32_t vh[16], vl[16];
          tmem_ld16(dacc + uint32_t(cg * 16), vh);
          tmem_ld16(dacc + uint32_t(tl.nt + cg * 16), vl);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int n = cg * 16 + i;
            if (n < tl.ntok) {
              const int e = tl.entry0 + n;
              const size_t row = size_t(a.out_row ? a.out_row[e] : e);
              ycol[row * a.R] = __fadd_rn(__uint_as_float(vh[i]), __uint_as_float(vl[i]));
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&bars->accempty[d]);
        if (GU) mbar_arrive(&bars->rsempty[d]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

// --------------------------------------------------------------------------- combine
__global__ void moe_combine_kernel(const float* __restrict__ yp, const int32_t* __restrict__ entry_pos,
                                   const float* __restrict__ scores, int S, int H, uint16_t* __restrict__ y) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x;
  int pos[16];
  float w[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    pos[j] = j < S ? entry_pos[(size_t)t * S + j] : -1;
    w[j] = j < S ? scores[(size_t)t * S + j] : 0.0f;
  }
  for (int n = (blockIdx.y * blockDim.x + threadIdx.x) * 4; n < H; n += blockDim.x * gridDim.y * 4) {
    float4 v[16];
#pragma unroll
    for (int j = 0; j < 16; ++j)
      v[j] = pos[j] >= 0 ? *reinterpret_cast<const float4*>(yp + (size_t)pos[j] * H + n) : make_float4(0.f, 0.f, 0.f, 0.f);
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      if (pos[j] < 0) continue;
      acc[0] = __fmaf_rn(w[j], v[j].x, acc[0]);
      acc[1] = __fmaf_rn(w[j], v[j].y, acc[1]);
      acc[2] = __fmaf_rn(w[j], v[j].z, acc[2]);
      acc[3] = __fmaf_rn(w[j], v[j].w, acc[3]);
    }
    uint2 o;
    o.x = uint32_t(f2bf(acc[0])) | (uint32_t(f2bf(acc[1])) << 16);
    o.y = uint32_t(f2bf(acc[2])) | (uint32_t(f2bf(acc[3])) << 16);
    *reinterpret_cast<uint2*>(y + (size_t)t * H + n) = o;
  }
}

// --------------------------------------------------------------------------- expert-parallel dispatch
// Plan (one CTA of 1024 threads): entry i = (t, j), expert e = idx[i].  A routed entry (e < n_routed) goes
// to rank d = e / per at slot p (its rank among d's entries in (t, j) order, from block scans, so the
// placement is deterministic); a shared entry takes the next local slot q in (t, j) order.
//   send_e[d * cap + p] = e - d * per (unused slots -1); sh_e[q] = per + e - n_routed (unused -1);
//   pos[i] = d * cap + p, or 2 * G * cap + q for a shared entry: the entry's row in the table
//   [partials back from the peers (G * cap rows) ; this rank's expert pass (G * cap received rows, then
//   the shared rows)];
//   counts[d] = entries to rank d, counts[G] = shared entries.  An entry beyond `cap` or with an invalid
//   expert id is dropped (pos = -1) and recorded in the device error word.
__global__ void __launch_bounds__(1024) moe_dispatch_plan_kernel(const int32_t* __restrict__ idx, int n,
                                                                 int n_routed, int n_exp, int per, int G, int cap,
                                                                 int32_t* __restrict__ send_e, int32_t* __restrict__ sh_e,
                                                                 int32_t* __restrict__ pos, int32_t* __restrict__ counts,
                                                                 unsigned* err) {
  __shared__ int s_warp[32];
  pdl_wait();
  pdl_trigger();
  const int tid = threadIdx.x;
  for (int i = tid; i < G * cap; i += blockDim.x) send_e[i] = -1;
  for (int i = tid; i < n; i += blockDim.x) {
    sh_e[i] = -1;
    pos[i] = -1;  // invalid expert ids keep -1 (recorded below)
  }
  auto cat = [&](int e) { return (e < 0 || e >= n_exp) ? -1 : (e < n_routed ? e / per : G); };
  const int per_thr = (n + blockDim.x - 1) / blockDim.x, i0 = min(n, tid * per_thr), i1 = min(n, i0 + per_thr);
  bool overflow = false;
  for (int c = 0; c <= G; ++c) {  // category c: rank c (routed) or G (shared)
    int mine = 0;
    for (int i = i0; i < i1; ++i) {
      const int e = idx[i];
      if (c == 0 && cat(e) < 0) overflow = true;
      mine += cat(e) == c;
    }
    int total;
    int slot = block_excl_scan(mine, s_warp, total);  // ends with a barrier: send_e / sh_e fills are done
    for (int i = i0; i < i1; ++i) {
      const int e = idx[i];
      if (cat(e) != c) continue;
      if (c < G) {
        if (slot < cap) {
          send_e[c * cap + slot] = e - c * per;
          pos[i] = c * cap + slot;
        } else {
          pos[i] = -1;
          overflow = true;
        }
      } else {
        sh_e[slot] = per + e - n_routed;
        pos[i] = 2 * G * cap + slot;
      }
      ++slot;
    }
    if (tid == 0) counts[c] = total;
  }
  if (overflow && err) atomicOr(err, DEVERR_BADARG);
}

// Row copies of the plan: x[t] of entry i to send_x (routed) or sh_x (shared); one CTA per entry.
__global__ void __launch_bounds__(256) moe_dispatch_rows_kernel(const uint16_t* __restrict__ x, int S, int H, int G,
                                                                int cap, const int32_t* __restrict__ pos,
                                                                uint16_t* __restrict__ send_x,
                                                                uint16_t* __restrict__ sh_x) {
  pdl_wait();
  pdl_trigger();
  const int i = blockIdx.x, p = pos[i];
  if (p < 0) return;
  const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)(i / S) * H);
  uint4* dst = reinterpret_cast<uint4*>(p < G * cap ? send_x + (size_t)p * H : sh_x + (size_t)(p - 2 * G * cap) * H);
  for (int k = threadIdx.x; k < H / 8; k += blockDim.x) dst[k] = src[k];
}

// --------------------------------------------------------------------------- host side
struct Workspace {
  size_t entry_pos, sorted_tok, rank_tmp, xsh, tiles, counters, ximg, himg, yp, total;
  int max_tiles, max_rows;
};
inline size_t up256(size_t v) { return (v + 255) & ~size_t(255); }
inline Workspace layout(int T, int S, int E, int H, int I) {
  Workspace w;
  const size_t n = size_t(T) * S;
  w.max_tiles = int(E + (n + kMaxTok - 1) / kMaxTok);
  w.max_rows = int(n + 15 * size_t(w.max_tiles));
  size_t o = 0;
  w.entry_pos = o; o = up256(o + n * 4);
  w.sorted_tok = o; o = up256(o + n * 4);
  w.rank_tmp = o; o = up256(o + n * 4);
  w.xsh = o; o = up256(o + n * 4);
  w.tiles = o; o = up256(o + size_t(w.max_tiles) * sizeof(Tile));
  w.counters = o; o = up256(o + 16);
  w.ximg = o; o = up256(o + size_t(w.max_rows) * H * 2);
  w.himg = o; o = up256(o + size_t(w.max_rows) * I * 4);
  w.yp = o; o = up256(o + n * H * 4);
  w.total = o;
  return w;
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
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
// uint8 2-D tensor [rows, cols] with row pitch `cols` bytes; box = bw bytes x 128 rows.
bool byte_map(CUtensorMap* m, const void* base, long long rows, long long cols, int bw, CUtensorMapSwizzle swz) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {cuuint64_t(cols), cuuint64_t(rows)};
  cuuint64_t strides[1] = {cuuint64_t(cols)};
  cuuint32_t box[2] = {uint32_t(bw), uint32_t(kRows)};
  cuuint32_t es[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
// Packed weights [rows, K/2 bytes]: box = 64 bytes (128 k) x 128 rows, 64-B swizzle.
bool weight_map(CUtensorMap* m, const void* base, long long rows, int K) {
  return byte_map(m, base, rows, K / 2, kChunk / 2, CU_TENSOR_MAP_SWIZZLE_64B);
}

// Weight-ring depth: as many stages as fit next to the operand ring and the two scale buffers.
template <bool GU>
int ring_stages(int sbuf) {
  for (int nw = kMaxW; nw >= 2; --nw)
    if (smem_map(GU, nw, sbuf).total <= kSmemMax) return nw;
  return 0;
}

template <bool GU>
cudaError_t launch_gemm(const CUtensorMap& w0, const CUtensorMap& w1, const CUtensorMap& s0, const CUtensorMap& s1,
                        const GemmArgs& a, int grid, cudaStream_t st) {
  static std::once_flag once;
  static cudaError_t attr = cudaSuccess;
  std::call_once(once, [] {
    attr = cudaFuncSetAttribute(moe_gemm_kernel<GU>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemMax);
  });
  if (attr != cudaSuccess) return attr;
  const size_t smem = size_t(smem_map(GU, a.nw, a.sbuf).total);
  return launch_kernel(moe_gemm_kernel<GU>, dim3(grid), dim3(kThreads), smem, st, w0, w1, s0, s1, a);
}

}  // namespace moe
}  // namespace qmtp

using namespace qmtp;
using namespace qmtp::moe;

extern "C" int qmtp_quantize_fp4(int fmt, const void* w, long long N, int K, void* wq, void* scales, void* stream) {
  if (fmt != 0 && fmt != 1) return QMTP_ERR_ARG;
  const int G = fmt == 0 ? 32 : 16;
  if (!w || !wq || !scales) return QMTP_ERR_ARG;
  if (N <= 0 || K <= 0 || K % G) return QMTP_ERR_SHAPE;
  const long long groups = N * (K / G);
  QMTP_CUDA_TRY(launch_kernel(quantize_fp4_kernel, dim3(unsigned((groups + 255) / 256)), dim3(256), 0,
                              static_cast<cudaStream_t>(stream), fmt, static_cast<const uint16_t*>(w), N, K,
                              static_cast<uint32_t*>(wq), static_cast<uint8_t*>(scales)));
  return QMTP_OK;
}

extern "C" int qmtp_moe_route(const void* logits, int T, int E, int top_k, int n_shared, float routed_scale, void* idx,
                              void* scores, void* stream) {
  if (!logits || !idx || !scores) return QMTP_ERR_ARG;
  if (T <= 0 || E <= 0 || E > 1024 || top_k <= 0 || top_k > E || n_shared < 0 || top_k + n_shared > 16)
    return QMTP_ERR_SHAPE;
  QMTP_CUDA_TRY(launch_kernel(moe_route_kernel, dim3(unsigned((T + 7) / 8)), dim3(256), 0,
                              static_cast<cudaStream_t>(stream), static_cast<const float*>(logits), T, E, top_k,
                              n_shared, routed_scale, static_cast<int32_t*>(idx), static_cast<float*>(scores)));
  return QMTP_OK;
}

extern "C" size_t qmtp_moe_workspace(int T, int S, int E, int H, int I) {
  if (T <= 0 || S <= 0 || E <= 0 || H <= 0 || I <= 0) return 0;
  return layout(T, S, E, H, I).total;
}

// Shared body of qmtp_moe (y = combined bf16 output) and qmtp_moe_experts (yp_out = fp32 partial of
// every (row, slot) entry with S == 1, written in input row order; no combine).
static int moe_run(int fmt, const void* x_, const void* wg, const void* sg_, const void* wu, const void* su_,
                   const void* wd, const void* sd_, const void* idx_, const void* scores_, void* y_, float* yp_out,
                   int T, int S, int E, int H, int I, float limit, void* workspace, size_t ws_bytes, void* stream_) {
  if (fmt != 0 && fmt != 1) return QMTP_ERR_ARG;
  if (!x_ || !wg || !sg_ || !wu || !su_ || !wd || !sd_ || !idx_ || !workspace) return QMTP_ERR_ARG;
  if (!yp_out && (!scores_ || !y_)) return QMTP_ERR_ARG;
  if (yp_out && S != 1) return QMTP_ERR_SHAPE;
  if (T <= 0 || S <= 0 || S > 16 || E <= 0 || E > 1024 || (long long)T * S > 65535) return QMTP_ERR_SHAPE;
  if (H <= 0 || I <= 0 || H % kRows || I % kRows) return QMTP_ERR_SHAPE;
  const int G = fmt == 0 ? 32 : 16;
  const int KS_gu = H / G, KS_dn = I / G;
  const int sbox = KS_gu % 16 == 0;  // gate/up scales in 16-byte TMA boxes (conflict-light reads), else rows
  const int sbuf_gu = (2 * kRows * KS_gu + 1023) & ~1023, sbuf_dn = (kRows * KS_dn + 1023) & ~1023;
  const int nw_gu = ring_stages<true>(sbuf_gu), nw_dn = ring_stages<false>(sbuf_dn);
  if (nw_gu < 2 || nw_dn < 2) return QMTP_ERR_UNSUPPORTED;
  if (!aligned16(x_) || !aligned16(wg) || !aligned16(wu) || !aligned16(wd) || !aligned16(sg_) || !aligned16(su_) ||
      !aligned16(sd_) || (y_ && !aligned16(y_)) || (yp_out && !aligned16(yp_out)) ||
      (reinterpret_cast<uintptr_t>(workspace) & 255u))
    return QMTP_ERR_ALIGN;
  const Workspace L = layout(T, S, E, H, I);
  if (ws_bytes < L.total) return QMTP_ERR_SHAPE;
  const auto* x = static_cast<const uint16_t*>(x_);
  const auto* sd = static_cast<const uint8_t*>(sd_);
  const auto* idx = static_cast<const int32_t*>(idx_);
  const auto* scores = static_cast<const float*>(scores_);
  auto* y = static_cast<uint16_t*>(y_);
  auto stream = static_cast<cudaStream_t>(stream_);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  auto* entry_pos = reinterpret_cast<int32_t*>(ws + L.entry_pos);
  auto* sorted_tok = reinterpret_cast<int32_t*>(ws + L.sorted_tok);
  auto* rank_tmp = reinterpret_cast<int32_t*>(ws + L.rank_tmp);
  auto* xsh = reinterpret_cast<int32_t*>(ws + L.xsh);
  auto* tiles = reinterpret_cast<Tile*>(ws + L.tiles);
  auto* counters = reinterpret_cast<int32_t*>(ws + L.counters);
  uint8_t* ximg = ws + L.ximg;
  uint8_t* himg = ws + L.himg;
  auto* yp = reinterpret_cast<float*>(ws + L.yp);

  CUtensorMap mg, mu, md, msg, msu;
  if (!weight_map(&mg, wg, (long long)E * I, H) || !weight_map(&mu, wu, (long long)E * I, H) ||
      !weight_map(&md, wd, (long long)E * H, I) ||
      (sbox && (!byte_map(&msg, sg_, (long long)E * I, KS_gu, 16, CU_TENSOR_MAP_SWIZZLE_NONE) ||
                !byte_map(&msu, su_, (long long)E * I, KS_gu, 16, CU_TENSOR_MAP_SWIZZLE_NONE))))
    return QMTP_ERR_CUDA;
  if (!sbox) msg = msu = mg;  // unused

  const int n = T * S;
  static std::once_flag once;
  static cudaError_t gattr = cudaSuccess;
  std::call_once(once, [] {
    gattr = cudaFuncSetAttribute(moe_group_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 32 * 1024 * 2);
  });
  QMTP_CUDA_TRY(gattr);
  unsigned* err = device_error_ptr();
  QMTP_CUDA_TRY(launch_kernel(moe_group_kernel, dim3(1), dim3(1024), size_t(32) * E * 2, stream, idx, n, S, E,
                              entry_pos, sorted_tok, rank_tmp, tiles, counters, err));
  QMTP_CUDA_TRY(launch_kernel(moe_gather_kernel, dim3(unsigned(L.max_tiles), kMaxTok / 8), dim3(256), 0, stream, x, H,
                              (const Tile*)tiles, (const int32_t*)counters, (const int32_t*)sorted_tok, ximg, xsh));
  const int grid = sm_count();
  GemmArgs gu{static_cast<const uint8_t*>(sg_), static_cast<const uint8_t*>(su_), ximg, tiles, counters, xsh, himg,
              nullptr, nullptr, H, I, KS_gu, fmt, limit, I, nw_gu, sbuf_gu, sbox, err};
  QMTP_CUDA_TRY(launch_gemm<true>(mg, mu, msg, msu, gu, grid, stream));
  GemmArgs dn{sd, nullptr, himg, tiles, counters, nullptr, nullptr, yp_out ? yp_out : yp,
              yp_out ? (const int32_t*)sorted_tok : nullptr, I, H, KS_dn, fmt, limit, 0, nw_dn, sbuf_dn, 0, err};
  QMTP_CUDA_TRY(launch_gemm<false>(md, md, md, md, dn, grid, stream));
  if (!yp_out)
    QMTP_CUDA_TRY(launch_kernel(moe_combine_kernel, dim3(unsigned(T), unsigned((H + 1023) / 1024)), dim3(256), 0,
                                stream, (const float*)yp, (const int32_t*)entry_pos, scores, S, H, y));
  return QMTP_OK;
}

extern "C" int qmtp_moe(int fmt, const void* x, const void* wg, const void* sg, const void* wu, const void* su,
                        const void* wd, const void* sd, const void* idx, const void* scores, void* y, int T, int S,
                        int E, int H, int I, float limit, void* workspace, size_t ws_bytes, void* stream) {
  return moe_run(fmt, x, wg, sg, wu, su, wd, sd, idx, scores, y, nullptr, T, S, E, H, I, limit, workspace, ws_bytes,
                 stream);
}

extern "C" int qmtp_moe_experts(int fmt, const void* x, const void* wg, const void* sg, const void* wu, const void* su,
                                const void* wd, const void* sd, const void* expert, void* partial, int n, int E, int H,
                                int I, float limit, void* workspace, size_t ws_bytes, void* stream) {
  if (!partial) return QMTP_ERR_ARG;
  return moe_run(fmt, x, wg, sg, wu, su, wd, sd, expert, nullptr, nullptr, static_cast<float*>(partial), n, 1, E, H, I,
                 limit, workspace, ws_bytes, stream);
}

extern "C" int qmtp_moe_dispatch(const void* idx, int T, int S, const void* x, int H, int n_routed, int n_shared,
                                 int world, int cap, void* send_x, void* send_e, void* sh_x, void* sh_e, void* pos,
                                 void* counts, void* stream) {
  if (!idx || !x || !send_x || !send_e || !sh_x || !sh_e || !pos || !counts) return QMTP_ERR_ARG;
  if (T <= 0 || S <= 0 || H <= 0 || H % 8 || world <= 0 || n_routed <= 0 || n_routed % world || n_shared < 0 ||
      cap <= 0 || (long long)T * S > (1 << 20) || (long long)world * cap > (1 << 24))
    return QMTP_ERR_SHAPE;
  if (!aligned16(x) || !aligned16(send_x) || !aligned16(sh_x)) return QMTP_ERR_ALIGN;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int n = T * S;
  QMTP_CUDA_TRY(launch_kernel(moe_dispatch_plan_kernel, dim3(1), dim3(1024), 0, st, static_cast<const int32_t*>(idx), n,
                              n_routed, n_routed + n_shared, n_routed / world, world, cap, static_cast<int32_t*>(send_e),
                              static_cast<int32_t*>(sh_e), static_cast<int32_t*>(pos), static_cast<int32_t*>(counts),
                              device_error_ptr()));
  QMTP_CUDA_TRY(launch_kernel(moe_dispatch_rows_kernel, dim3(unsigned(n)), dim3(256), 0, st,
                              static_cast<const uint16_t*>(x), S, H, world, cap, static_cast<const int32_t*>(pos),
                              static_cast<uint16_t*>(send_x), static_cast<uint16_t*>(sh_x)));
  return QMTP_OK;
}

extern "C" int qmtp_moe_combine(const void* partials, const void* row_of, const void* scores, int T, int S, int H,
                                void* y, void* stream) {
  if (!partials || !row_of || !scores || !y) return QMTP_ERR_ARG;
  if (T <= 0 || S <= 0 || S > 16 || H <= 0 || H % 4) return QMTP_ERR_SHAPE;
  if (!aligned16(partials) || (reinterpret_cast<uintptr_t>(y) & 7u)) return QMTP_ERR_ALIGN;
  QMTP_CUDA_TRY(launch_kernel(moe_combine_kernel, dim3(unsigned(T), unsigned((H + 1023) / 1024)), dim3(256), 0,
                              static_cast<cudaStream_t>(stream), static_cast<const float*>(partials),
                              static_cast<const int32_t*>(row_of), static_cast<const float*>(scores), S, H,
                              static_cast<uint16_t*>(y)));
  return QMTP_OK;
}
