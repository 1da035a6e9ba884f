// Decoder glue kernels for the synthetic Qwen3.5 model and the device-side speculative-decoding
// control of mtp.py:241-303.  Every position, length and rollback index is read from a device
// control block (qmtp_ctrl_*), so one verify + draft cycle can be captured once in a CUDA graph
// and replayed with one host read of the emitted tokens per cycle.
//
// Arithmetic (fixed fp32 sequences, bit-identical to oracle/qmtp_oracle.c):
//   rmsnorm     wide tree (D % 1024 == 0: thread c owns the 32-element chunk c) or head tree
//   attn_prep   q/k head RMS norm (head tree), partial rotate-half RoPE, KV-cache append
//   attention   keys dealt to 8 splits (one warp each), two-pass softmax per split, fixed merge,
//               output gate R(o * sigmoid_bf(gate))
//   swiglu      R(silu_bf(g) * u)
#include <algorithm>

#include "common.cuh"

namespace qmtp {

// ----------------------------------------------------------------------------- embedding
__global__ void embed_kernel(const int32_t* __restrict__ tok, const uint32_t* __restrict__ wq,
                             const uint16_t* __restrict__ sc, const uint16_t* __restrict__ bi, int D,
                             uint16_t* __restrict__ out, long long ld_out, int V, unsigned* err) {
  pdl_trigger();
  pdl_wait();
  const int t = blockIdx.x;
  const int r = tok[t];
  if (r < 0 || r >= V) {
    if (threadIdx.x == 0) atomicOr(err, DEVERR_BADARG);
    return;
  }
  const int G = D / 64;
  for (int w = threadIdx.x; w < D / 8; w += blockDim.x) {
    const uint32_t word = wq[size_t(r) * (D / 8) + w];
    const int g = (8 * w) / 64;
    const float s = bf2f(sc[size_t(r) * G + g]), b = bf2f(bi[size_t(r) * G + g]);
    uint16_t o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = f2bf(__fmaf_rn(s, float((word >> (4 * j)) & 15u), b));
    *reinterpret_cast<uint4*>(out + t * ld_out + 8 * w) =
        make_uint4(o[0] | (uint32_t(o[1]) << 16), o[2] | (uint32_t(o[3]) << 16), o[4] | (uint32_t(o[5]) << 16),
                   o[6] | (uint32_t(o[7]) << 16));
  }
}

// NVFP4 rows: out = bf16(e2m1(q) * e4m3(scale of 16)), the product exact in fp32 (2 x 4 significant bits);
// e4m3 is read as in qmv_kernel.py:26-28 (sign ignored; exponent 15 with mantissa 7 is 480).
__device__ __forceinline__ float e4m3_unsigned(uint32_t s) {
  const uint32_t e = (s >> 3) & 15u, m = s & 7u;
  if (e == 0) return __fmul_rn(float(m), 0.001953125f);
  return __uint_as_float((e + 120u) << 23 | (m << 20));
}
__global__ void embed_nvfp4_kernel(const int32_t* __restrict__ tok, const uint32_t* __restrict__ wq,
                                   const uint8_t* __restrict__ sc, int D, uint16_t* __restrict__ out,
                                   long long ld_out, int V, unsigned* err) {
  pdl_trigger();
  pdl_wait();
  const int t = blockIdx.x;
  const int r = tok[t];
  if (r < 0 || r >= V) {
    if (threadIdx.x == 0) atomicOr(err, DEVERR_BADARG);
    return;
  }
  for (int w = threadIdx.x; w < D / 8; w += blockDim.x) {
    const uint32_t word = wq[size_t(r) * (D / 8) + w];
    const float s = e4m3_unsigned(sc[size_t(r) * (D / 16) + w / 2]);
    uint16_t o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t q = (word >> (4 * j)) & 15u;
      const uint32_t mg = q & 7u;  // e2m1 magnitude: 0, .5, 1, 1.5, 2, 3, 4, 6
      const float v = mg < 2u ? 0.5f * float(mg) : __uint_as_float((((mg >> 1) + 126u) << 23) | ((mg & 1u) << 22));
      o[j] = f2bf(__fmul_rn(q & 8u ? -v : v, s));
    }
    *reinterpret_cast<uint4*>(out + t * ld_out + 8 * w) =
        make_uint4(o[0] | (uint32_t(o[1]) << 16), o[2] | (uint32_t(o[3]) << 16), o[4] | (uint32_t(o[5]) << 16),
                   o[6] | (uint32_t(o[7]) << 16));
  }
}

// ----------------------------------------------------------------------------- RMSNorm
// Wide tree: blockDim = D/32 threads, thread c owns elements [32c, 32c+32).
// RMS norm of one row of D = 32 * blockDim.x elements (thread c holds v = elements [32c, 32c + 32)):
// a 32-fma chain per thread, the warp butterfly, the warps' sums in order, then bf16(w * R(x * r)) into
// orow.  wq4: the thread's 32 weights.  Every thread of the block calls it.
__device__ __forceinline__ void rmsnorm_row(const float (&v)[32], const uint4 (&wq4)[4], float eps, int D,
                                            uint16_t* __restrict__ orow) {
  __shared__ float s_blk[32];
  __shared__ float s_r;
  const int c = threadIdx.x, lane = c & 31, warp = c >> 5;
  float ss = 0.0f;
#pragma unroll
  for (int e = 0; e < 32; ++e) ss = __fmaf_rn(v[e], v[e], ss);
  ss = warp_sum(ss);
  if (lane == 0) s_blk[warp] = ss;
  __syncthreads();
  if (c == 0) {
    float t = s_blk[0];
    for (int i = 1; i < int(blockDim.x >> 5); ++i) t = __fadd_rn(t, s_blk[i]);
    s_r = rsqrt_rn(__fadd_rn(__fdiv_rn(t, float(D)), eps));
  }
  __syncthreads();
  const float r = s_r;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const uint32_t ww[4] = {wq4[q].x, wq4[q].y, wq4[q].z, wq4[q].w};
    uint32_t o[4];
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      const uint16_t lo = f2bf(__fmul_rn(bflo(ww[h]), R(__fmul_rn(v[8 * q + 2 * h], r))));
      const uint16_t hi = f2bf(__fmul_rn(bfhi(ww[h]), R(__fmul_rn(v[8 * q + 2 * h + 1], r))));
      o[h] = lo | (uint32_t(hi) << 16);
    }
    *reinterpret_cast<uint4*>(orow + 32 * c + 8 * q) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

__device__ __forceinline__ void load_row32(const uint16_t* __restrict__ xr, float (&v)[32]) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const uint4 u = *reinterpret_cast<const uint4*>(xr + 8 * q);
    const uint32_t uu[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int h = 0; h < 4; ++h) { v[8 * q + 2 * h] = bflo(uu[h]); v[8 * q + 2 * h + 1] = bfhi(uu[h]); }
  }
}

__global__ void rmsnorm_wide_kernel(const uint16_t* __restrict__ x, long long ld_x, const int* __restrict__ row_sel,
                                    const uint16_t* __restrict__ w, float eps, uint16_t* __restrict__ out,
                                    long long ld_o, int D) {
  pdl_trigger();
  const int m = blockIdx.x, c = threadIdx.x;
  uint4 wq4[4];  // the norm weight is constant: fetched while the previous kernel may still run
#pragma unroll
  for (int q = 0; q < 4; ++q) wq4[q] = *reinterpret_cast<const uint4*>(w + 32 * c + 8 * q);
  pdl_wait();
  const long long row = row_sel ? (long long)(*row_sel) + m : m;
  float v[32];
  load_row32(x + row * ld_x + 32 * c, v);
  rmsnorm_row(v, wq4, eps, D, out + (long long)m * ld_o);
}

// Embedding rows and RMS norms in one launch, grid (M, jobs): job 0 dequantizes the embedding row of
// tok[m] (affine g64 table, embed_kernel's arithmetic), writes it to raw (if not null) and its RMS norm
// with w0 to out0; job 1 (x1 not null) is rmsnorm_wide_kernel on row row_sel1 + m of x1 with w1 into
// out1.  The verify step uses job 0 (the embedding and layer 0's input norm), an MTP step both (its
// two pre-fc norms).
__global__ void embed_rmsnorm_kernel(const int32_t* __restrict__ tok, const uint32_t* __restrict__ wq,
                                     const uint16_t* __restrict__ sc, const uint16_t* __restrict__ bi, int V,
                                     uint16_t* __restrict__ raw, long long ld_raw, const uint16_t* __restrict__ w0,
                                     uint16_t* __restrict__ out0, long long ld_o0, const uint16_t* __restrict__ x1,
                                     long long ld_x1, const int* __restrict__ row_sel1, const uint16_t* __restrict__ w1,
                                     uint16_t* __restrict__ out1, long long ld_o1, float eps, int D, unsigned* err) {
  pdl_trigger();
  const int m = blockIdx.x, job = blockIdx.y, c = threadIdx.x;
  const uint16_t* w = job == 0 ? w0 : w1;
  uint4 wq4[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) wq4[q] = *reinterpret_cast<const uint4*>(w + 32 * c + 8 * q);
  pdl_wait();
  float v[32];
  if (job == 0) {
    const int r = tok[m];
    if (r < 0 || r >= V) {  // uniform over the block: it leaves before any barrier
      if (c == 0) atomicOr(err, DEVERR_BADARG);
      return;
    }
    const int G = D / 64;
    const float s = bf2f(sc[size_t(r) * G + c / 2]), b = bf2f(bi[size_t(r) * G + c / 2]);  // elements 32c.. in group c/2
    uint32_t pk[16];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint32_t word = wq[size_t(r) * (D / 8) + 4 * c + q];
#pragma unroll
      for (int j = 0; j < 8; j += 2) {
        const uint16_t lo = f2bf(__fmaf_rn(s, float((word >> (4 * j)) & 15u), b));
        const uint16_t hi = f2bf(__fmaf_rn(s, float((word >> (4 * (j + 1))) & 15u), b));
        v[8 * q + j] = bf2f(lo);
        v[8 * q + j + 1] = bf2f(hi);
        pk[4 * q + j / 2] = lo | (uint32_t(hi) << 16);
      }
    }
    if (raw) {
#pragma unroll
      for (int q = 0; q < 4; ++q)
        *reinterpret_cast<uint4*>(raw + (long long)m * ld_raw + 32 * c + 8 * q) =
            make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
    }
    rmsnorm_row(v, wq4, eps, D, out0 + (long long)m * ld_o0);
  } else {
    const long long row = row_sel1 ? (long long)(*row_sel1) + m : m;
    load_row32(x1 + row * ld_x1 + 32 * c, v);
    rmsnorm_row(v, wq4, eps, D, out1 + (long long)m * ld_o1);
  }
}

// ----------------------------------------------------------------------------- attention prep
// One (token, head) row of q or k, Dh == 256, by one warp: RMS norm with the weight row (lane l owns
// dims [8l, 8l+8), wn4 its 8 weights), then rotate-half RoPE over dims [0, 64) at position pos (pairs
// (i, i + 32), lanes 0..7, lane l paired with lane l ^ 4).  Returns the lane's 8 bf16 results packed.
__device__ __forceinline__ uint4 prep_head_row(const uint16_t* __restrict__ src, uint4 wn4, float eps,
                                               const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                                               int pos, int lane) {
  constexpr int Dh = 256, NP = 8, RH = 32;  // rotary half
  float x[NP];
  {
    const uint4 u = *reinterpret_cast<const uint4*>(src + NP * lane);
    const uint32_t uu[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int h = 0; h < 4; ++h) { x[2 * h] = bflo(uu[h]); x[2 * h + 1] = bfhi(uu[h]); }
  }
  float ss = 0.0f;
#pragma unroll
  for (int e = 0; e < NP; ++e) ss = __fmaf_rn(x[e], x[e], ss);
  ss = warp_sum(ss);
  const float r = rsqrt_rn(__fadd_rn(__fdiv_rn(ss, float(Dh)), eps));
  {
    const uint32_t wv[4] = {wn4.x, wn4.y, wn4.z, wn4.w};
#pragma unroll
    for (int e = 0; e < NP; ++e)
      x[e] = R(__fmul_rn((e & 1) ? bfhi(wv[e >> 1]) : bflo(wv[e >> 1]), R(__fmul_rn(x[e], r))));
  }
  float o[NP];
#pragma unroll
  for (int e = 0; e < NP; ++e) {
    const float partner = __shfl_xor_sync(0xFFFFFFFFu, x[e], 4);
    o[e] = x[e];
    if (lane < 8) {
      const int d = NP * lane + e;          // this lane's dim
      const int i = d < RH ? d : d - RH;    // frequency index
      const float c = cos_t[(long long)pos * RH + i], sn = sin_t[(long long)pos * RH + i];
      if (d < RH) o[e] = __fsub_rn(__fmul_rn(x[e], c), __fmul_rn(partner, sn));
      else o[e] = __fadd_rn(__fmul_rn(x[e], c), __fmul_rn(partner, sn));
    }
  }
  uint32_t pk[4];
#pragma unroll
  for (int h = 0; h < 4; ++h) pk[h] = f2bf(o[2 * h]) | (uint32_t(f2bf(o[2 * h + 1])) << 16);
  return make_uint4(pk[0], pk[1], pk[2], pk[3]);
}

// One warp per (token s, head hh) with hh < nq query heads, then nkv key heads (prep_head_row); the
// gate and v rows are copied through.
__global__ void attn_prep_kernel(const uint16_t* __restrict__ qkv, long long ld, int S, int nq, int nkv,
                                 const uint16_t* __restrict__ qn_w, const uint16_t* __restrict__ kn_w, float eps,
                                 const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                                 const int* __restrict__ pos_ptr, int pos_add, uint16_t* __restrict__ qo,
                                 uint16_t* __restrict__ gate, uint16_t* __restrict__ kc, uint16_t* __restrict__ vc,
                                 int max_pos, unsigned* err) {
  pdl_trigger();
  constexpr int Dh = 256, NP = 8;
  const int lane = threadIdx.x & 31;
  const int wid = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  if (wid >= S * (nq + nkv)) return;
  const int s = wid / (nq + nkv), hh = wid - s * (nq + nkv);
  // the q / k norm weights are constant: fetched while the previous kernel may still run
  const uint4 wn4 = *reinterpret_cast<const uint4*>((hh < nq ? qn_w : kn_w) + NP * lane);
  pdl_wait();
  const int pos = (pos_ptr ? *pos_ptr : 0) + pos_add + s;
  if (pos < 0 || pos >= max_pos) {
    if (lane == 0) atomicOr(err, DEVERR_BADARG);
    return;
  }
  const bool isq = hh < nq;
  const uint16_t* row = qkv + (long long)s * ld;
  const uint16_t* src = isq ? row + (long long)hh * 2 * Dh : row + (long long)nq * 2 * Dh + (long long)(hh - nq) * Dh;
  const uint4 packed = prep_head_row(src, wn4, eps, cos_t, sin_t, pos, lane);
  if (isq) {
    *reinterpret_cast<uint4*>(qo + ((long long)s * nq + hh) * Dh + NP * lane) = packed;
    *reinterpret_cast<uint4*>(gate + ((long long)s * nq + hh) * Dh + NP * lane) =
        *reinterpret_cast<const uint4*>(src + Dh + NP * lane);
  } else {
    const int kh = hh - nq;
    *reinterpret_cast<uint4*>(kc + ((long long)kh * max_pos + pos) * Dh + NP * lane) = packed;
    *reinterpret_cast<uint4*>(vc + ((long long)kh * max_pos + pos) * Dh + NP * lane) =
        *reinterpret_cast<const uint4*>(row + (long long)nq * 2 * Dh + (long long)nkv * Dh + (long long)kh * Dh +
                                        NP * lane);
  }
}

// ----------------------------------------------------------------------------- attention
// One thread-block cluster of kAttnSplits CTAs per (query head, token); CTA rank w owns key split w
// (keys j = w, w + 8, ...).  Dh == 256.  Per CTA: scores (8 warps, lane owns 8 dims, warp_sum) ->
// split max -> exponentials -> den (one sequential chain) and num[d] (thread d, keys ascending) in
// shared memory.  Rank 0 then merges the 8 splits in order through distributed shared memory.
constexpr int kAttnSplits = 8;
constexpr int kAttnBatch = 8;   // keys a warp fetches at once in the score pass
constexpr int kAttnVStage = 128; // value rows of a split copied to shared memory while the scores run
                                 // (64 KB: three CTAs an SM still fit; contexts up to 1024 keys)

// FUSED: the kernel also does attn_prep_kernel's work for what it reads (qmtp_attention_fused).  Warp 0
// prepares this CTA's q row from the projection output, warp 1 the split's new key (of the S new
// positions at most one falls in a split, S <= 8) and copies its value row; the new key and value
// stand in for the cache rows wherever they are used, and one CTA per (kv head, new position) writes
// them to the caches.  The gate is read from the projection output.
struct AttnFuse {
  const uint16_t* qkv;   // bf16 [S, ld]: per query head (q, gate), then k heads, then v heads
  long long ld;
  const uint16_t* qn_w;  // bf16 [Dh] q / k RMS norm weights
  const uint16_t* kn_w;
  float eps;
  const float* cos_t;    // [max_pos, 32] RoPE tables
  const float* sin_t;
  int S;
};

template <bool FUSED>
__global__ void __launch_bounds__(256, 3)  // 3 CTAs an SM: the 8-CTA clusters of a launch fit in one wave
attention_kernel(const uint16_t* __restrict__ q, const uint16_t* __restrict__ gate, uint16_t* __restrict__ kc,
                 uint16_t* __restrict__ vc, int max_pos, int nq, int nkv, const int* __restrict__ pos_ptr,
                 int pos_add, uint16_t* __restrict__ out, unsigned* err, AttnFuse F) {
  pdl_trigger();
  __shared__ __align__(16) uint4 s_q[32], s_knew[32], s_vnew[32];  // FUSED: prepared q, new key and value rows
  uint4 wq4 = make_uint4(0, 0, 0, 0);  // FUSED: the lane's 8 norm weights (constants, fetched before the wait)
  if (FUSED) {
    const int wp = threadIdx.x >> 5;
    if (wp < 2) wq4 = *reinterpret_cast<const uint4*>((wp == 0 ? F.qn_w : F.kn_w) + 8 * (threadIdx.x & 31));
  }
  {
    // this split's key and value rows into L2 while the previous launches finish; the position is
    // read before the wait as an address hint only (a stale value prefetches other rows, no more)
    const int w = int(cluster_rank()), hq = blockIdx.x / kAttnSplits, s = blockIdx.y;
    int Lh = (pos_ptr ? *pos_ptr : 0) + pos_add + s + 1;
    Lh = Lh < 0 ? 0 : (Lh > max_pos ? max_pos : Lh);
    const int kh = hq / (nq / nkv);
    const int nk = w < Lh ? (Lh - w + kAttnSplits - 1) / kAttnSplits : 0;
    for (int n = threadIdx.x; n < nk; n += blockDim.x) {
      const long long r = ((long long)kh * max_pos + w + kAttnSplits * n) * 256;
      prefetch_l2(kc + r, 512);
      prefetch_l2(vc + r, 512);
    }
  }
  pdl_wait();
  constexpr int Dh = 256, NP = 8;
  extern __shared__ __align__(16) float sm[];
  float* s_num = sm;                 // [Dh] this split's numerator
  float* s_md = s_num + Dh;          // [2] split max, denominator
  float* s_red = s_md + 2;           // [8] per-warp maxima
  float* s_sc = s_red + 8;           // [max_pos / 8 + 1] scores, then exponentials
  // the first kAttnVStage value rows of the split: [kAttnVStage][Dh / 2] bf16 pairs, 16-byte aligned
  uint32_t* s_v = reinterpret_cast<uint32_t*>(sm + ((Dh + 10 + max_pos / kAttnSplits + 1 + 3) & ~3));
  const int w = int(cluster_rank());  // key split
  const int h = blockIdx.x / kAttnSplits, s = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int L = (pos_ptr ? *pos_ptr : 0) + pos_add + s + 1;
  if (L < 1 || L > max_pos) {  // uniform over the cluster: every CTA leaves before any barrier
    if (tid == 0 && w == 0) atomicOr(err, DEVERR_BADARG);
    return;
  }
  const int kh = h / (nq / nkv);
  const int nk = w < L ? (L - w + kAttnSplits - 1) / kAttnSplits : 0;  // keys of this split
  // FUSED: this split's new key, if any: position pos0 + t_new (t_new <= s) is key n_new of the split
  const int pos0 = L - s - 1;
  int t_new = -1, n_new = -1;
  if (FUSED) {
    const int t = ((w - pos0) % kAttnSplits + kAttnSplits) % kAttnSplits;
    if (t <= s) { t_new = t; n_new = (pos0 + t - w) / kAttnSplits; }
  }
  // loads that do not wait for q: the first kAttnVStage value rows of the split into shared memory
  // (asynchronous copies, 16 bytes a thread and step) and this warp's first round of key rows
  {
    const int nv = min(nk, kAttnVStage);
    for (int c = tid; c < nv * (Dh / 8); c += 256) {
      const int n = c / (Dh / 8), part = c - n * (Dh / 8);
      if (n != n_new)  // FUSED: the new row is written below from the projection output
        cp_async16(s_v + n * (Dh / 2) + part * 4, vc + ((long long)kh * max_pos + w + kAttnSplits * n) * Dh + part * 8);
    }
    cp_async_commit();
  }
  uint4 kr[kAttnBatch];
#pragma unroll
  for (int u = 0; u < kAttnBatch; ++u) {
    const int n = warp + 8 * u;
    if (n < nk) kr[u] = *reinterpret_cast<const uint4*>(kc + ((long long)kh * max_pos + w + kAttnSplits * n) * Dh + NP * lane);
  }
  if (FUSED) {
    if (warp == 0) {
      s_q[lane] = prep_head_row(F.qkv + (long long)s * F.ld + (long long)h * 2 * Dh, wq4, F.eps, F.cos_t, F.sin_t,
                                pos0 + s, lane);
    } else if (warp == 1 && t_new >= 0) {
      const uint16_t* row = F.qkv + (long long)t_new * F.ld + (long long)nq * 2 * Dh;
      const uint4 kk = prep_head_row(row + (long long)kh * Dh, wq4, F.eps, F.cos_t, F.sin_t, pos0 + t_new, lane);
      const uint4 vv = *reinterpret_cast<const uint4*>(row + (long long)nkv * Dh + (long long)kh * Dh + NP * lane);
      s_knew[lane] = kk;
      s_vnew[lane] = vv;
      if (n_new < kAttnVStage) *reinterpret_cast<uint4*>(s_v + n_new * (Dh / 2) + 4 * lane) = vv;
      // the caches: one CTA per (kv head, new position) -- the first query head of the group, last token
      if (h % (nq / nkv) == 0 && s == F.S - 1) {
        const long long r = ((long long)kh * max_pos + pos0 + t_new) * Dh + NP * lane;
        *reinterpret_cast<uint4*>(kc + r) = kk;
        *reinterpret_cast<uint4*>(vc + r) = vv;
      }
    }
    __syncthreads();
  }
  float qf[NP];
  {
    const uint4 u = FUSED ? s_q[lane] : *reinterpret_cast<const uint4*>(q + ((long long)s * nq + h) * Dh + NP * lane);
    const uint32_t uu[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) { qf[2 * e] = bflo(uu[e]); qf[2 * e + 1] = bfhi(uu[e]); }
  }
  const float scale = rsqrt_rn(float(Dh));
  // scores: warp `warp` takes split-local keys n = warp, warp + 8, ...; a score is lane-sequential
  // fmas over the lane's 8 dims + warp_sum (independent per key, so any distribution gives the
  // same values); the max is exact, hence order-free
  float mx = __int_as_float(0xFF800000);
  for (int n0 = warp; n0 < nk; n0 += 8 * kAttnBatch) {
    if (n0 != warp) {  // the first round was fetched above
#pragma unroll
      for (int u = 0; u < kAttnBatch; ++u) {
        const int n = n0 + 8 * u;
        if (n < nk)
          kr[u] = *reinterpret_cast<const uint4*>(kc + ((long long)kh * max_pos + w + kAttnSplits * n) * Dh + NP * lane);
      }
    }
    float acc[kAttnBatch];
#pragma unroll
    for (int u = 0; u < kAttnBatch; ++u) {
      const uint4 k4 = (FUSED && n0 + 8 * u == n_new) ? s_knew[lane] : kr[u];
      const uint32_t uu[4] = {k4.x, k4.y, k4.z, k4.w};
      acc[u] = 0.0f;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        acc[u] = __fmaf_rn(qf[2 * e], bflo(uu[e]), acc[u]);
        acc[u] = __fmaf_rn(qf[2 * e + 1], bfhi(uu[e]), acc[u]);
      }
    }
#pragma unroll
    for (int d = 16; d >= 1; d >>= 1)
#pragma unroll
      for (int u = 0; u < kAttnBatch; ++u) acc[u] = __fadd_rn(acc[u], __shfl_xor_sync(0xFFFFFFFFu, acc[u], d));
#pragma unroll
    for (int u = 0; u < kAttnBatch; ++u) {
      const int n = n0 + 8 * u;
      if (n < nk) {
        const float sc = __fmul_rn(acc[u], scale);
        if (lane == 0) s_sc[n] = sc;
        mx = sc > mx ? sc : mx;
      }
    }
  }
  if (lane == 0) s_red[warp] = mx;
  __syncthreads();
  float mw = s_red[0];
#pragma unroll
  for (int i = 1; i < 8; ++i) mw = s_red[i] > mw ? s_red[i] : mw;
  // exponentials (parallel), then the two sequential chains of the split
  for (int n = tid; n < nk; n += 256) s_sc[n] = q_expf(__fsub_rn(s_sc[n], mw));
  cp_async_wait_all();  // this thread's value-row copies; the barrier publishes everyone's
  __syncthreads();
  if (tid == Dh / 2) {  // warp 4: idle in the numerator pass below
    float den = 0.0f;
    for (int n = 0; n < nk; ++n) den = __fadd_rn(den, s_sc[n]);
    s_md[0] = mw;
    s_md[1] = den;
  }
  if (tid < Dh / 2) {
    // thread t owns dims 2t, 2t+1: one 32-bit word per key, keys ascending, 32 keys a batch; the
    // first kAttnVStage keys from shared memory, the rest from global memory
    float num0 = 0.0f, num1 = 0.0f;
    const uint32_t* vb = reinterpret_cast<const uint32_t*>(vc + ((long long)kh * max_pos + w) * Dh) + tid;
    for (int n0 = 0; n0 < nk; n0 += 32) {
      uint32_t v2[32];
      static_assert(kAttnVStage % 32 == 0, "a batch is staged whole or not at all");
      const bool staged = n0 < kAttnVStage;
#pragma unroll
      for (int u = 0; u < 32; ++u)
        if (n0 + u < nk)
          v2[u] = staged ? s_v[(n0 + u) * (Dh / 2) + tid]
                  : (FUSED && n0 + u == n_new) ? reinterpret_cast<const uint32_t*>(s_vnew)[tid]
                                               : vb[(long long)kAttnSplits * (n0 + u) * (Dh / 2)];
#pragma unroll
      for (int u = 0; u < 32; ++u)
        if (n0 + u < nk) {
          const float e = s_sc[n0 + u];
          num0 = __fmaf_rn(e, bflo(v2[u]), num0);
          num1 = __fmaf_rn(e, bfhi(v2[u]), num1);
        }
    }
    s_num[2 * tid] = num0;
    s_num[2 * tid + 1] = num1;
  }
  cluster_sync_all();  // every split's (max, den, num) is visible to rank 0
  if (w == 0) {
    const int d = tid;
    const int nsplit = L < kAttnSplits ? L : kAttnSplits;
    float mm[kAttnSplits], dd[kAttnSplits], nn[kAttnSplits];
#pragma unroll
    for (int ww = 0; ww < kAttnSplits; ++ww)
      if (ww < nsplit) {
        mm[ww] = ld_dsmem(s_md, ww);
        dd[ww] = ld_dsmem(s_md + 1, ww);
        nn[ww] = ld_dsmem(s_num + d, ww);
      }
    float M = __int_as_float(0xFF800000);
#pragma unroll
    for (int ww = 0; ww < kAttnSplits; ++ww)
      if (ww < nsplit && mm[ww] > M) M = mm[ww];
    float dsum = 0.0f, acc = 0.0f;
#pragma unroll
    for (int ww = 0; ww < kAttnSplits; ++ww)
      if (ww < nsplit) {
        const float cw = q_expf(__fsub_rn(mm[ww], M));
        dsum = __fmaf_rn(cw, dd[ww], dsum);
        acc = __fmaf_rn(cw, nn[ww], acc);
      }
    const float o = R(__fdiv_rn(acc, dsum));
    const float gt = bf2f(FUSED ? F.qkv[(long long)s * F.ld + (long long)h * 2 * Dh + Dh + d]
                                : gate[((long long)s * nq + h) * Dh + d]);
    out[(long long)s * nq * Dh + (long long)h * Dh + d] = f2bf(__fmul_rn(o, sigmoid_bf(gt)));
  }
  cluster_sync_all();  // rank 0 has read the other CTAs' shared memory before they exit
}

// ----------------------------------------------------------------------------- SwiGLU
__global__ void swiglu_kernel(const uint16_t* __restrict__ gu, long long ld, int I, uint16_t* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  const int s = blockIdx.y;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < I; i += gridDim.x * blockDim.x) {
    const float g = bf2f(gu[(long long)s * ld + i]), u = bf2f(gu[(long long)s * ld + I + i]);
    out[(long long)s * I + i] = f2bf(__fmul_rn(silu_bf(g), u));
  }
}

// ----------------------------------------------------------------------------- control
// Greedy acceptance (mtp.py:275-294 / engine.py:121-128): a = verify argmax [k+1], in = [t, d_1..d_k].
// keep = 1 + #leading drafts equal to a; emits a[0..keep); rollback bookkeeping for the next cycle.
__global__ void accept_kernel(const int32_t* __restrict__ a, const int32_t* __restrict__ in, int k,
                              int* __restrict__ ctrl, int32_t* __restrict__ out_tokens, int out_cap, int ring_slots,
                              int win_rows, int forced_keep) {
  pdl_trigger();
  pdl_wait();
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  int n_acc = 0;
  // adaptive k (mtp.py:229-238): only the first NUSE drafts are verified (0: all k)
  const int nuse = ctrl[QMTP_CTRL_NUSE];
  const int lim = nuse > 0 && nuse < k ? nuse : k;
  if (forced_keep > 0) {
    n_acc = forced_keep - 1;
  } else {
    while (n_acc < lim && a[n_acc] == in[1 + n_acc]) {
      ctrl[QMTP_CTRL_ACC0 + n_acc] += 1;
      ++n_acc;
    }
    ctrl[QMTP_CTRL_VERIFIED] += lim;
  }
  const int keep = n_acc + 1;
  int nout = ctrl[QMTP_CTRL_NOUT];
  if (forced_keep <= 0) {
    for (int i = 0; i < keep; ++i) {
      ctrl[QMTP_CTRL_EMIT0 + i] = a[i];
      if (nout < out_cap) out_tokens[nout++] = a[i];
    }
    ctrl[QMTP_CTRL_NOUT] = nout;
    ctrl[QMTP_CTRL_CYCLES] += 1;
  }
  ctrl[QMTP_CTRL_KEEP] = keep;
  ctrl[QMTP_CTRL_SEL] = keep - 1;
  ctrl[QMTP_CTRL_POS] += keep;
  ctrl[QMTP_CTRL_SLOT] = (ctrl[QMTP_CTRL_SLOT] + keep) % ring_slots;
  const int par = ctrl[QMTP_CTRL_WPAR] ^ 1;  // the window just written becomes the previous one
  ctrl[QMTP_CTRL_WPAR] = par;
  ctrl[QMTP_CTRL_CONV_ROW] = par * win_rows + keep;
  ctrl[QMTP_CTRL_WOUT_ROW] = (par ^ 1) * win_rows;
}

// Probability the draft head gives its argmax token (mtp.py:222-223: softmax(logits).max()): 1 / sum_j
// exp(l_j - l_max) over the vocabulary.  One CTA of 1024 threads; the sum is fixed in order: thread t
// adds the elements j = t, t + 1024, ... in order, the xor butterfly within each warp, then the 32
// warp sums in order (oracle qo_draft_prob).
constexpr int kProbThreads = 1024;
__global__ void __launch_bounds__(kProbThreads)
draft_prob_kernel(const uint16_t* __restrict__ logits, int V, const int32_t* __restrict__ token, float* __restrict__ prob,
                  unsigned* err) {
  pdl_trigger();
  pdl_wait();
  __shared__ float ws[kProbThreads / 32];
  const int tid = threadIdx.x;
  const int t = *token;
  if (t < 0 || t >= V) {  // uniform: every thread reads the same token
    if (tid == 0) {
      atomicOr(err, DEVERR_BADARG);
      *prob = 0.0f;
    }
    return;
  }
  const float lmax = bf2f(logits[t]);
  float s = 0.0f;
  for (int j = tid; j < V; j += kProbThreads) s = __fadd_rn(s, q_expf(__fsub_rn(bf2f(logits[j]), lmax)));
  s = warp_sum(s);
  if ((tid & 31) == 0) ws[tid >> 5] = s;
  __syncthreads();
  if (tid == 0) {
    float tot = ws[0];
    for (int w = 1; w < kProbThreads / 32; ++w) tot = __fadd_rn(tot, ws[w]);
    *prob = __fdiv_rn(1.0f, tot);
  }
}

// n_drafts (mtp.py:229-238): the drafts to verify next, from the chain's k probabilities -- keep
// multiplying while the running product stays >= tau (at least one draft); double precision like the
// reference's Python float product.
__global__ void mtp_nuse_kernel(const float* __restrict__ probs, int k, double tau, int* __restrict__ ctrl) {
  pdl_trigger();
  pdl_wait();
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  int n = 0;
  double acc = 1.0;
  for (int i = 0; i < k; ++i) {
    acc *= double(probs[i]);
    if (n && acc < tau) break;
    ++n;
  }
  ctrl[QMTP_CTRL_NUSE] = n;
}

// MTP cache bookkeeping between the two draft steps: MPOS += keep (mtp.py:291-294: the k-1 chained
// entries of the previous cycle are trimmed, the keep real pairs are committed).
__global__ void mtp_advance_kernel(int* __restrict__ ctrl) {
  pdl_trigger();
  pdl_wait();
  if (threadIdx.x == 0 && blockIdx.x == 0) ctrl[QMTP_CTRL_MPOS] += ctrl[QMTP_CTRL_KEEP];
}

// Next verify input [t, d1, d2]: t = a[keep-1].
__global__ void next_tokens_kernel(const int32_t* __restrict__ a, const int32_t* __restrict__ drafts, int k,
                                   const int* __restrict__ ctrl, int32_t* __restrict__ in) {
  pdl_trigger();
  pdl_wait();
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  in[0] = a[ctrl[QMTP_CTRL_SEL]];
  for (int i = 0; i < k; ++i) in[1 + i] = drafts[i];
}

}  // namespace qmtp

using namespace qmtp;

extern "C" int qmtp_embed(const int* tokens, int T, const void* wq, const void* scales, const void* biases, int V,
                          int D, void* out, int ld_out, void* stream) {
  if (!tokens || !wq || !scales || !biases || !out) return QMTP_ERR_ARG;
  if (T < 1 || D % 64 != 0 || ld_out < D || ld_out % 8 != 0) return QMTP_ERR_SHAPE;
  if (!aligned16(out)) return QMTP_ERR_ALIGN;
  // one packed word per thread (D / 8 threads up to 1024), so a row costs one round trip to memory
  const int threads = std::min(1024, std::max(32, ((D / 8 + 31) / 32) * 32));
  launch_kernel(embed_kernel, dim3(T), dim3(threads), 0, static_cast<cudaStream_t>(stream), 
      tokens, static_cast<const uint32_t*>(wq), static_cast<const uint16_t*>(scales),
      static_cast<const uint16_t*>(biases), D, static_cast<uint16_t*>(out), ld_out, V, device_error_ptr());
  return cudaGetLastError() == cudaSuccess ? QMTP_OK : QMTP_ERR_CUDA;
}

extern "C" int qmtp_embed_nvfp4(const int* tokens, int T, const void* wq, const void* scales, int V, int D, void* out,
                                int ld_out, void* stream) {
  if (!tokens || !wq || !scales || !out) return QMTP_ERR_ARG;
  if (T < 1 || D % 64 != 0 || ld_out < D || ld_out % 8 != 0) return QMTP_ERR_SHAPE;
  if (!aligned16(out)) return QMTP_ERR_ALIGN;
  const int threads = std::min(1024, std::max(32, ((D / 8 + 31) / 32) * 32));
  launch_kernel(embed_nvfp4_kernel, dim3(T), dim3(threads), 0, static_cast<cudaStream_t>(stream), tokens,
                static_cast<const uint32_t*>(wq), static_cast<const uint8_t*>(scales), D,
                static_cast<uint16_t*>(out), ld_out, V, device_error_ptr());
  return cudaGetLastError() == cudaSuccess ? QMTP_OK : QMTP_ERR_CUDA;
}

extern "C" int qmtp_rmsnorm(const void* x, int ld_x, const int* row_sel, const void* w, float eps, void* out,
                            int ld_out, int M, int D, void* stream) {
  if (!x || !w || !out) return QMTP_ERR_ARG;
  if (M < 1 || D % 1024 != 0 || D > 32768 || ld_x < D || ld_out < D || ld_x % 8 || ld_out % 8) return QMTP_ERR_SHAPE;
  if (!aligned16(x) || !aligned16(w) || !aligned16(out)) return QMTP_ERR_ALIGN;
  launch_kernel(rmsnorm_wide_kernel, dim3(M), dim3(D / 32), 0, static_cast<cudaStream_t>(stream), 
      static_cast<const uint16_t*>(x), ld_x, row_sel, static_cast<const uint16_t*>(w), eps,
      static_cast<uint16_t*>(out), ld_out, D);
  return cudaGetLastError() == cudaSuccess ? QMTP_OK : QMTP_ERR_CUDA;
}

extern "C" int qmtp_embed_rmsnorm(const int* tok, int M, const void* wq, const void* scales, const void* biases,
                                  int V, int D, void* raw, int ld_raw, const void* w0, void* out0, int ld_out0,
                                  const void* x1, int ld_x1, const int* row_sel1, const void* w1, void* out1,
                                  int ld_out1, float eps, void* stream) {
  if (!tok || !wq || !scales || !biases || !w0 || !out0) return QMTP_ERR_ARG;
  if (x1 && (!w1 || !out1)) return QMTP_ERR_ARG;
  if (M < 1 || V < 1 || D % 1024 != 0 || D > 32768 || ld_out0 < D || ld_out0 % 8) return QMTP_ERR_SHAPE;
  if (raw && (ld_raw < D || ld_raw % 8)) return QMTP_ERR_SHAPE;
  if (x1 && (ld_x1 < D || ld_out1 < D || ld_x1 % 8 || ld_out1 % 8)) return QMTP_ERR_SHAPE;
  const void* al[] = {w0, out0, raw, x1, w1, out1};
  for (const void* p : al)
    if (p && !aligned16(p)) return QMTP_ERR_ALIGN;
  launch_kernel(embed_rmsnorm_kernel, dim3(M, x1 ? 2 : 1), dim3(D / 32), 0, static_cast<cudaStream_t>(stream), tok,
                static_cast<const uint32_t*>(wq), static_cast<const uint16_t*>(scales),
                static_cast<const uint16_t*>(biases), V, static_cast<uint16_t*>(raw), (long long)ld_raw,
                static_cast<const uint16_t*>(w0), static_cast<uint16_t*>(out0), (long long)ld_out0,
                static_cast<const uint16_t*>(x1), (long long)ld_x1, row_sel1, static_cast<const uint16_t*>(w1),
                static_cast<uint16_t*>(out1), (long long)ld_out1, eps, D, device_error_ptr());
  return cudaGetLastError() == cudaSuccess ? QMTP_OK : QMTP_ERR_CUDA;
}

extern "C" int qmtp_attn_prep(const void* qkv, int ld, int S, int nq, int nkv, int Dh, int rotary, const void* qn_w,
                              const void* kn_w, float eps, const float* cos_t, const float* sin_t, const int* pos_ptr,
                              int pos_add, void* q_out, void* gate_out, void* k_cache, void* v_cache, int max_pos,
                              void* stream) {
  if (!qkv || !qn_w || !kn_w || !cos_t || !sin_t || !q_out || !gate_out || !k_cache || !v_cache) return QMTP_ERR_ARG;
  if (Dh != 256 || rotary != 64 || S < 1 || nq < 1 || nkv < 1 || nq % nkv || ld % 8) return QMTP_ERR_UNSUPPORTED;
  if (!aligned16(qkv) || !aligned16(qn_w) || !aligned16(kn_w)) return QMTP_ERR_ALIGN;
  const int warps = S * (nq + nkv), wpb = 8;
  launch_kernel(attn_prep_kernel, dim3((warps + wpb - 1) / wpb), dim3(wpb * 32), 0, static_cast<cudaStream_t>(stream), 
      static_cast<const uint16_t*>(qkv), ld, S, nq, nkv, static_cast<const uint16_t*>(qn_w),
      static_cast<const uint16_t*>(kn_w), eps, cos_t, sin_t, pos_ptr, pos_add, static_cast<uint16_t*>(q_out),
      static_cast<uint16_t*>(gate_out), static_cast<uint16_t*>(k_cache), static_cast<uint16_t*>(v_cache), max_pos,
      device_error_ptr());
  return cudaGetLastError() == cudaSuccess ? QMTP_OK : QMTP_ERR_CUDA;
}

static int attention_launch(bool fused, const void* q, const void* gate, void* k_cache, void* v_cache, int max_pos,
                            int S, int nq, int nkv, int Dh, const int* pos_ptr, int pos_add, void* out, const AttnFuse& F,
                            void* stream) {
  if (Dh != 256 || S < 1 || nq < 1 || nkv < 1 || nq % nkv || max_pos < 8) return QMTP_ERR_UNSUPPORTED;
  if (!aligned16(k_cache) || !aligned16(v_cache)) return QMTP_ERR_ALIGN;  // 16-byte rows
  // scores etc. (rounded up to 16 bytes), then the staged value rows
  const size_t smem = ((size_t(Dh) + 2 + 8 + size_t(max_pos / kAttnSplits + 1) + 3) & ~size_t(3)) * sizeof(float) +
                      size_t(kAttnVStage) * Dh * sizeof(uint16_t);
  if (smem > 200 * 1024) return QMTP_ERR_SHAPE;
  static const cudaError_t attr[2] = {
      cudaFuncSetAttribute(attention_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024),
      cudaFuncSetAttribute(attention_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024)};
  if (attr[0] != cudaSuccess || attr[1] != cudaSuccess) return QMTP_ERR_CUDA;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(nq * kAttnSplits), unsigned(S));
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = kAttnSplits;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[1].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = at;
  cfg.numAttrs = 2;
  cudaLaunchKernelEx(&cfg, fused ? attention_kernel<true> : attention_kernel<false>, static_cast<const uint16_t*>(q),
                     static_cast<const uint16_t*>(gate), static_cast<uint16_t*>(k_cache),
                     static_cast<uint16_t*>(v_cache), max_pos, nq, nkv, pos_ptr, pos_add, static_cast<uint16_t*>(out),
                     device_error_ptr(), F);
  return cudaGetLastError() == cudaSuccess ? QMTP_OK : QMTP_ERR_CUDA;
}

extern "C" int qmtp_attention(const void* q, const void* gate, const void* k_cache, const void* v_cache, int max_pos,
                              int S, int nq, int nkv, int Dh, const int* pos_ptr, int pos_add, void* out,
                              void* stream) {
  if (!q || !gate || !k_cache || !v_cache || !out) return QMTP_ERR_ARG;
  if (!aligned16(q)) return QMTP_ERR_ALIGN;
  return attention_launch(false, q, gate, const_cast<void*>(k_cache), const_cast<void*>(v_cache), max_pos, S, nq, nkv,
                          Dh, pos_ptr, pos_add, out, AttnFuse{}, stream);
}

extern "C" int qmtp_attention_fused(const void* qkv, int ld, int S, int nq, int nkv, int Dh, int rotary,
                                    const void* qn_w, const void* kn_w, float eps, const float* cos_t,
                                    const float* sin_t, const int* pos_ptr, int pos_add, void* k_cache, void* v_cache,
                                    int max_pos, void* out, void* stream) {
  if (!qkv || !qn_w || !kn_w || !cos_t || !sin_t || !k_cache || !v_cache || !out) return QMTP_ERR_ARG;
  if (Dh != 256 || rotary != 64 || S < 1 || S > kAttnSplits || ld % 8) return QMTP_ERR_UNSUPPORTED;
  if (!aligned16(qkv) || !aligned16(qn_w) || !aligned16(kn_w)) return QMTP_ERR_ALIGN;
  AttnFuse F{static_cast<const uint16_t*>(qkv), ld, static_cast<const uint16_t*>(qn_w),
             static_cast<const uint16_t*>(kn_w), eps, cos_t, sin_t, S};
  return attention_launch(true, nullptr, nullptr, k_cache, v_cache, max_pos, S, nq, nkv, Dh, pos_ptr, pos_add, out, F,
                          stream);
}

extern "C" int qmtp_swiglu(const void* gu, int ld, int S, int I, void* out, void* stream) {
  if (!gu || !out) return QMTP_ERR_ARG;
  if (S < 1 || I < 1 || ld < 2 * I) return QMTP_ERR_SHAPE;
  launch_kernel(swiglu_kernel, dim3(dim3(std::min((I + 255) / 256, 64), S)), dim3(256), 0, static_cast<cudaStream_t>(stream), 
      static_cast<const uint16_t*>(gu), ld, I, static_cast<uint16_t*>(out));
  return cudaGetLastError() == cudaSuccess ? QMTP_OK : QMTP_ERR_CUDA;
}

extern "C" int qmtp_mtp_accept(const int* a, const int* in, int k, int* ctrl, int* out_tokens, int out_cap,
                               int ring_slots, int win_rows, int forced_keep, void* stream) {
  if (!a || !in || !ctrl || !out_tokens) return QMTP_ERR_ARG;
  if (k < 1 || k > QMTP_CTRL_MAX_K || ring_slots < k + 2 || forced_keep > k + 1 || QMTP_CTRL_EMIT0 + k + 1 > QMTP_CTRL_SIZE)
    return QMTP_ERR_SHAPE;
  launch_kernel(accept_kernel, dim3(1), dim3(32), 0, static_cast<cudaStream_t>(stream), a, in, k, ctrl, out_tokens, out_cap, ring_slots,
                                                                  win_rows, forced_keep);
  return cudaGetLastError() == cudaSuccess ? QMTP_OK : QMTP_ERR_CUDA;
}

extern "C" int qmtp_draft_prob(const void* logits, int V, const int* token, float* prob, void* stream) {
  if (!logits || !token || !prob) return QMTP_ERR_ARG;
  if (V < 1) return QMTP_ERR_SHAPE;
  launch_kernel(draft_prob_kernel, dim3(1), dim3(kProbThreads), 0, static_cast<cudaStream_t>(stream),
                static_cast<const uint16_t*>(logits), V, token, prob, device_error_ptr());
  return cudaGetLastError() == cudaSuccess ? QMTP_OK : QMTP_ERR_CUDA;
}

extern "C" int qmtp_mtp_nuse(const float* probs, int k, double tau, int* ctrl, void* stream) {
  if (!probs || !ctrl) return QMTP_ERR_ARG;
  if (k < 1 || k > QMTP_CTRL_MAX_K) return QMTP_ERR_SHAPE;
  launch_kernel(mtp_nuse_kernel, dim3(1), dim3(32), 0, static_cast<cudaStream_t>(stream), probs, k, tau, ctrl);
  return cudaGetLastError() == cudaSuccess ? QMTP_OK : QMTP_ERR_CUDA;
}

extern "C" int qmtp_mtp_advance(int* ctrl, void* stream) {
  if (!ctrl) return QMTP_ERR_ARG;
  launch_kernel(mtp_advance_kernel, dim3(1), dim3(32), 0, static_cast<cudaStream_t>(stream), ctrl);
  return cudaGetLastError() == cudaSuccess ? QMTP_OK : QMTP_ERR_CUDA;
}

extern "C" int qmtp_next_tokens(const int* a, const int* drafts, int k, const int* ctrl, int* in, void* stream) {
  if (!a || !drafts || !ctrl || !in) return QMTP_ERR_ARG;
  launch_kernel(next_tokens_kernel, dim3(1), dim3(32), 0, static_cast<cudaStream_t>(stream), a, drafts, k, ctrl, in);
  return cudaGetLastError() == cudaSuccess ? QMTP_OK : QMTP_ERR_CUDA;
}
