// GatedDeltaNet decode/verify step on B200: the recurrent state of every (value head, dv row) stays
// in registers across the T verify tokens; the state after each token is written out as a rollback
// snapshot (gdn_kernel.py:11-88), and the fused variant also does the causal conv, silu, q/k RMS
// norms and the g / beta gates of gdn_fused.py:43-112 in the same launch.
//
// Work split: one warp per dv row; lane l owns dk elements [4l, 4l+4) of the row (the reference's
// lane layout, gdn_kernel.py:16,30); 32-lane sums are xor butterflies.  The fp32 sequence is the
// one of oracle/qmtp_oracle.c (qo_gdn_step / qo_gdn_fused / qo_gdn_norm_gate).
#include "common.cuh"

namespace qmtp {

// ----------------------------------------------------------------------------- snapshot step
template <int NP>
__global__ void __launch_bounds__(256)
gdn_step_kernel(const uint16_t* __restrict__ q, const uint16_t* __restrict__ k, const uint16_t* __restrict__ v,
                const float* __restrict__ g, const float* __restrict__ beta, const float* __restrict__ state_in,
                uint16_t* __restrict__ y, float* __restrict__ state_out, float* __restrict__ state_mid, int B,
                int T, int Hk, int Hv, int Dv) {
  pdl_trigger();
  pdl_wait();
  constexpr int Dk = NP * 32;
  const int lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;  // (b*Hv + hv)*Dv + dv
  if (row >= (long long)B * Hv * Dv) return;
  const int n = int(row / Dv), dv = int(row % Dv);
  const int b = n / Hv, hv = n % Hv, hk = hv / (Hv / Hk);
  const size_t srow = size_t(row) * Dk + NP * lane;
  const size_t per = size_t(B) * Hv * Dv * Dk;
  float st[NP];
#pragma unroll
  for (int i = 0; i < NP; ++i) st[i] = state_in[srow + i];
  for (int t = 0; t < T; ++t) {
    const size_t qo = ((size_t(b) * T + t) * Hk + hk) * Dk + NP * lane;
    float qf[NP], kf[NP];
#pragma unroll
    for (int i = 0; i < NP; ++i) { qf[i] = bf2f(q[qo + i]); kf[i] = bf2f(k[qo + i]); }
    const size_t gi = (size_t(b) * T + t) * Hv + hv;
    const float gt = g[gi], bt = beta[gi];
    float kv = 0.0f;
#pragma unroll
    for (int i = 0; i < NP; ++i) {
      st[i] = __fmul_rn(st[i], gt);
      kv = __fmaf_rn(st[i], kf[i], kv);
    }
    kv = warp_sum(kv);
    const float delta = __fmul_rn(__fsub_rn(bf2f(v[gi * Dv + dv]), kv), bt);
    float o = 0.0f;
#pragma unroll
    for (int i = 0; i < NP; ++i) {
      st[i] = __fmaf_rn(kf[i], delta, st[i]);
      o = __fmaf_rn(st[i], qf[i], o);
    }
    o = warp_sum(o);
    if (lane == 0) y[gi * Dv + dv] = f2bf(o);
    if (state_mid && t < T - 1) {
#pragma unroll
      for (int i = 0; i < NP; ++i) state_mid[size_t(t) * per + srow + i] = st[i];
    }
  }
#pragma unroll
  for (int i = 0; i < NP; ++i) state_out[srow + i] = st[i];
}

// ----------------------------------------------------------------------------- fused core
constexpr int kFusedWarps = 8;
constexpr int kFusedRPW = 2;                         // dv rows per warp
constexpr int kFusedDVB = kFusedWarps * kFusedRPW;   // dv rows per CTA

template <int NP>
__global__ void __launch_bounds__(kFusedWarps * 32)
gdn_fused_kernel(qmtp_gdn_args A, unsigned* __restrict__ err) {
  pdl_trigger();
  pdl_wait();
  constexpr int Dk = NP * 32;
  static_assert((Dk & (Dk - 1)) == 0, "the 1/Dk multiplications need a power of two");
  extern __shared__ __align__(16) float sm[];
  const int S = A.S, KC = A.KC, Hk = A.Hk, Hv = A.Hv, Dv = A.Dv;
  float* qk = sm;                          // [S][2][Dk]
  float* vs = qk + S * 2 * Dk;             // [S][DVB]
  float* gs = vs + S * kFusedDVB;          // [S]
  float* bs = gs + S;                      // [S]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int hv = blockIdx.x, dv0 = blockIdx.y * kFusedDVB, hk = hv / (Hv / Hk);
  const int C = 2 * Hk * Dk + Hv * Dv;
  const uint16_t* conv_src = static_cast<const uint16_t*>(A.conv_src);
  const uint16_t* qkv = static_cast<const uint16_t*>(A.qkv);
  const uint16_t* conv_w = static_cast<const uint16_t*>(A.conv_w);
  const int off = A.conv_row_off ? *A.conv_row_off : 0;
  auto win = [&](int r, int ch) -> uint16_t {
    return r < KC - 1 ? conv_src[(long long)(off + r) * A.ld_conv + ch] : qkv[(long long)(r - (KC - 1)) * A.ld_qkv + ch];
  };
  auto conv = [&](int t, int ch) -> float {
    float acc = 0.0f;
    for (int j = 0; j < KC; ++j) acc = __fmaf_rn(bf2f(conv_w[(long long)ch * KC + j]), bf2f(win(t + j, ch)), acc);
    return silu_bf(R(acc));
  };

  // The state rows of phase 3 do not depend on phases 1-2: fetch them first so their latency
  // overlaps the convolution.
  const size_t per = size_t(Hv) * Dv * Dk;
  const float* sin = A.state_in;
  int cur = 0;
  if (A.ring) {
    cur = *A.ring_cur;
    if (cur < 0 || cur >= A.ring_slots) {
      if (tid == 0) atomicOr(err, DEVERR_BADARG);
      return;
    }
    sin = A.ring + size_t(cur) * per;
  }
  float st[kFusedRPW][NP];
#pragma unroll
  for (int rr = 0; rr < kFusedRPW; ++rr) {
    const int dv = dv0 + warp * kFusedRPW + rr;
    if (dv < Dv) {
      const float4 s4 = *reinterpret_cast<const float4*>(sin + (size_t(hv) * Dv + dv) * Dk + NP * lane);
      st[rr][0] = s4.x; st[rr][1] = s4.y; st[rr][2] = s4.z; st[rr][3] = s4.w;
    }
  }

  // phase 1: conv + silu of this head's q / k channels and of the CTA's v channels; gates.
  // A thread takes a channel over all tokens.  For the decode shape (KC == 4, S <= 4) the channel's
  // window column and taps are fetched with independent loads first, then the S outputs are formed
  // from registers (same fma sequence as conv()).
  constexpr int kFastKC = 4, kFastS = 4;
  const bool fast = KC == kFastKC && S <= kFastS;
  auto conv_channel = [&](int ch, float* dst, int stride) {
    if (fast) {
      float wv[kFastKC - 1 + kFastS], cw[kFastKC];
#pragma unroll
      for (int r = 0; r < kFastKC - 1 + kFastS; ++r)
        if (r < kFastKC - 1 + S)
          wv[r] = bf2f(r < kFastKC - 1 ? conv_src[(long long)(off + r) * A.ld_conv + ch]
                                      : qkv[(long long)(r - (kFastKC - 1)) * A.ld_qkv + ch]);
#pragma unroll
      for (int j = 0; j < kFastKC; ++j) cw[j] = bf2f(conv_w[(long long)ch * kFastKC + j]);
#pragma unroll
      for (int t = 0; t < kFastS; ++t)
        if (t < S) {
          float acc = 0.0f;
#pragma unroll
          for (int j = 0; j < kFastKC; ++j) acc = __fmaf_rn(cw[j], wv[t + j], acc);
          dst[t * stride] = silu_bf(R(acc));
        }
    } else {
      for (int t = 0; t < S; ++t) dst[t * stride] = conv(t, ch);
    }
  };
  for (int cc = tid; cc < 2 * Dk; cc += blockDim.x) {
    const int isk = cc / Dk, e = cc - isk * Dk;
    conv_channel(isk * Hk * Dk + hk * Dk + e, qk + cc, 2 * Dk);
  }
  // v channels from the last warp and the gates from warp 5, so no warp carries all three parts
  for (int d = int(blockDim.x) - 1 - tid; d >= 0 && d < kFusedDVB; d += blockDim.x) {
    if (dv0 + d < Dv) {
      conv_channel(2 * Hk * Dk + hv * Dv + dv0 + d, vs + d, kFusedDVB);
    } else {
      for (int t = 0; t < S; ++t) vs[t * kFusedDVB + d] = 0.0f;
    }
  }
  const uint16_t* av = static_cast<const uint16_t*>(A.a);
  const uint16_t* bv = static_cast<const uint16_t*>(A.b);
  for (int t = tid - 160; t >= 0 && t < S; t += blockDim.x) {
    const float Aneg = -q_expf(A.A_log[hv]);
    const float dtb = bf2f(static_cast<const uint16_t*>(A.dt_bias)[hv]);
    const float sp = softplus_bf(R(__fadd_rn(bf2f(av[(long long)t * A.ld_ab + hv]), dtb)));
    gs[t] = q_expf(__fmul_rn(Aneg, sp));
    bs[t] = sigmoid_bf(bf2f(bv[(long long)t * A.ld_ab + hv]));
  }
  // window for the next step: q/k channels by the first CTA of their key head, v channels by owner
  if (A.win_out) {
    uint16_t* wo = static_cast<uint16_t*>(A.win_out) + (long long)(A.win_out_row_off ? *A.win_out_row_off : 0) * C;
    const int R_ = KC - 1 + S;
    {
      // the q/k channels of key head hk are shared by its rep x gridDim.y CTAs: each writes a slice
      const int rep = Hv / Hk, nsl = rep * int(gridDim.y), j = (hv - hk * rep) * int(gridDim.y) + int(blockIdx.y);
      const int E = R_ * 2 * Dk, per_sl = (E + nsl - 1) / nsl;
      const int i1 = min(E, (j + 1) * per_sl);
      for (int idx = j * per_sl + tid; idx < i1; idx += blockDim.x) {
        const int r = idx / (2 * Dk), rem = idx - r * 2 * Dk, isk = rem / Dk, e = rem - isk * Dk;
        const int ch = isk * Hk * Dk + hk * Dk + e;
        wo[(long long)r * C + ch] = win(r, ch);
      }
    }
    for (int idx = tid; idx < R_ * kFusedDVB; idx += blockDim.x) {
      const int r = idx / kFusedDVB, d = idx - r * kFusedDVB;
      if (dv0 + d < Dv) {
        const int ch = 2 * Hk * Dk + hv * Dv + dv0 + d;
        wo[(long long)r * C + ch] = win(r, ch);
      }
    }
  }
  __syncthreads();

  // phase 2: q = R(q * r_q) / Dk, k = R(R(k * r_k) * R(Dk^-1/2)) per token
  const float kscale = R(rsqrt_rn(float(Dk)));
  for (int p = warp; p < 2 * S; p += kFusedWarps) {
    float* xr = qk + p * Dk + NP * lane;
    float xv[NP];
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < NP; ++i) { xv[i] = xr[i]; ss = __fmaf_rn(xv[i], xv[i], ss); }
    ss = warp_sum(ss);
    // Dk is a power of two: x / Dk and x * (1 / Dk) are the same correctly rounded value
    const float r = rsqrt_rn(__fadd_rn(__fmul_rn(ss, 1.0f / float(Dk)), 1e-6f));
#pragma unroll
    for (int i = 0; i < NP; ++i)
      xr[i] = (p & 1) ? R(__fmul_rn(R(__fmul_rn(xv[i], r)), kscale)) : __fmul_rn(R(__fmul_rn(xv[i], r)), 1.0f / float(Dk));
  }
  __syncthreads();

  // phase 3: the delta rule for this warp's dv rows, states in registers
  auto snapshot_dst = [&](int t) -> float* {
    if (A.ring) return (A.snap || t == S - 1) ? A.ring + size_t((cur + t + 1) % A.ring_slots) * per : nullptr;
    if (t == S - 1) return A.state_out;
    return (A.snap && A.state_mid) ? A.state_mid + size_t(t) * per : nullptr;
  };
  if (S <= kFastS) {
    // decode shape: the tokens unrolled; only the k.state sums chain from token to token, the
    // q.state sums of all tokens are reduced together at the end (same operations, shorter chain)
    float op[kFastS][kFusedRPW];
#pragma unroll
    for (int t = 0; t < kFastS; ++t) {
      if (t >= S) break;
      const float4 q4 = *reinterpret_cast<const float4*>(qk + (t * 2 + 0) * Dk + NP * lane);
      const float4 k4 = *reinterpret_cast<const float4*>(qk + (t * 2 + 1) * Dk + NP * lane);
      const float qf[4] = {q4.x, q4.y, q4.z, q4.w}, kf[4] = {k4.x, k4.y, k4.z, k4.w};
      const float gt = gs[t], bt = bs[t];
      float* dst = snapshot_dst(t);
      float kv[kFusedRPW];
#pragma unroll
      for (int rr = 0; rr < kFusedRPW; ++rr) {
        kv[rr] = 0.0f;
#pragma unroll
        for (int i = 0; i < NP; ++i) {
          st[rr][i] = __fmul_rn(st[rr][i], gt);
          kv[rr] = __fmaf_rn(st[rr][i], kf[i], kv[rr]);
        }
      }
#pragma unroll
      for (int d = 16; d >= 1; d >>= 1)
#pragma unroll
        for (int rr = 0; rr < kFusedRPW; ++rr) kv[rr] = __fadd_rn(kv[rr], __shfl_xor_sync(0xFFFFFFFFu, kv[rr], d));
#pragma unroll
      for (int rr = 0; rr < kFusedRPW; ++rr) {
        const int dv = dv0 + warp * kFusedRPW + rr;
        const float delta = dv < Dv ? __fmul_rn(__fsub_rn(vs[t * kFusedDVB + dv - dv0], kv[rr]), bt) : 0.0f;
        op[t][rr] = 0.0f;
#pragma unroll
        for (int i = 0; i < NP; ++i) {
          st[rr][i] = __fmaf_rn(kf[i], delta, st[rr][i]);
          op[t][rr] = __fmaf_rn(st[rr][i], qf[i], op[t][rr]);
        }
        if (dst && dv < Dv)
          *reinterpret_cast<float4*>(dst + (size_t(hv) * Dv + dv) * Dk + NP * lane) =
              make_float4(st[rr][0], st[rr][1], st[rr][2], st[rr][3]);
      }
    }
#pragma unroll
    for (int d = 16; d >= 1; d >>= 1)
#pragma unroll
      for (int t = 0; t < kFastS; ++t)
#pragma unroll
        for (int rr = 0; rr < kFusedRPW; ++rr)
          if (t < S) op[t][rr] = __fadd_rn(op[t][rr], __shfl_xor_sync(0xFFFFFFFFu, op[t][rr], d));
    if (lane == 0) {
#pragma unroll
      for (int t = 0; t < kFastS; ++t)
#pragma unroll
        for (int rr = 0; rr < kFusedRPW; ++rr) {
          const int dv = dv0 + warp * kFusedRPW + rr;
          if (t < S && dv < Dv) A.y[(size_t(t) * Hv + hv) * Dv + dv] = R(op[t][rr]);
        }
    }
    return;
  }
  for (int t = 0; t < S; ++t) {
    const float4 q4 = *reinterpret_cast<const float4*>(qk + (t * 2 + 0) * Dk + NP * lane);
    const float4 k4 = *reinterpret_cast<const float4*>(qk + (t * 2 + 1) * Dk + NP * lane);
    const float qf[4] = {q4.x, q4.y, q4.z, q4.w}, kf[4] = {k4.x, k4.y, k4.z, k4.w};
    const float gt = gs[t], bt = bs[t];
    float* dst = snapshot_dst(t);
#pragma unroll
    for (int rr = 0; rr < kFusedRPW; ++rr) {
      const int dv = dv0 + warp * kFusedRPW + rr;
      if (dv >= Dv) continue;
      float kv = 0.0f;
#pragma unroll
      for (int i = 0; i < NP; ++i) {
        st[rr][i] = __fmul_rn(st[rr][i], gt);
        kv = __fmaf_rn(st[rr][i], kf[i], kv);
      }
      kv = warp_sum(kv);
      const float delta = __fmul_rn(__fsub_rn(vs[t * kFusedDVB + dv - dv0], kv), bt);
      float o = 0.0f;
#pragma unroll
      for (int i = 0; i < NP; ++i) {
        st[rr][i] = __fmaf_rn(kf[i], delta, st[rr][i]);
        o = __fmaf_rn(st[rr][i], qf[i], o);
      }
      o = warp_sum(o);
      if (lane == 0) A.y[(size_t(t) * Hv + hv) * Dv + dv] = R(o);
      if (dst)
        *reinterpret_cast<float4*>(dst + (size_t(hv) * Dv + dv) * Dk + NP * lane) =
            make_float4(st[rr][0], st[rr][1], st[rr][2], st[rr][3]);
    }
  }
}

// ----------------------------------------------------------------------------- gated norm
template <int NP>
__global__ void __launch_bounds__(256)
gdn_norm_gate_kernel(const float* __restrict__ y, const uint16_t* __restrict__ z, long long ld_z,
                     const uint16_t* __restrict__ w, uint16_t* __restrict__ out, long long ld_out, int S, int H,
                     float eps) {
  pdl_trigger();
  constexpr int Dv = NP * 32;
  static_assert((Dv & (Dv - 1)) == 0, "the 1/Dv multiplications need a power of two");
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;  // t*H + h
  if (row >= S * H) return;
  const int t = row / H, h = row - t * H;
  float wv[NP];  // the norm weight is constant: fetched while the previous kernel may still run
#pragma unroll
  for (int i = 0; i < NP; ++i) wv[i] = bf2f(w[NP * lane + i]);
  pdl_wait();
  const float* yr = y + size_t(row) * Dv + NP * lane;
  float yv[NP], zv[NP];
#pragma unroll
  for (int i = 0; i < NP; ++i) zv[i] = bf2f(z[(long long)t * ld_z + (long long)h * Dv + NP * lane + i]);
  float ss = 0.0f;
#pragma unroll
  for (int i = 0; i < NP; ++i) { yv[i] = yr[i]; ss = __fmaf_rn(yv[i], yv[i], ss); }
  ss = warp_sum(ss);
  const float r = rsqrt_rn(__fadd_rn(__fmul_rn(ss, 1.0f / float(Dv)), eps));  // Dv: a power of two
#pragma unroll
  for (int i = 0; i < NP; ++i) {
    const int e = NP * lane + i;
    const float xn = R(__fmul_rn(wv[i], R(__fmul_rn(yv[i], r))));
    out[(long long)t * ld_out + (long long)h * Dv + e] = f2bf(__fmul_rn(xn, silu_f32(zv[i])));
  }
}

// Four independent silu evaluations in one out-of-line call (the compiler interleaves them).  Each
// inlined silu carries a correctly rounded division; the decode-shape kernel runs once per layer with
// a cold instruction cache, so its roles share these single copies instead.
static __device__ __noinline__ float4 silu_bf4(float4 x) {
  return make_float4(silu_bf(x.x), silu_bf(x.y), silu_bf(x.z), silu_bf(x.w));
}
static __device__ __noinline__ float4 silu_f32x4(float4 x) {
  return make_float4(silu_f32(x.x), silu_f32(x.y), silu_f32(x.z), silu_f32(x.w));
}

// ----------------------------------------------------------------------------- decode shape
// The verify step of the decode loop: S <= 4 tokens, KC == 4 taps, Dk == Dv == 128.  Same
// arithmetic as gdn_fused_kernel (+ gdn_norm_gate_kernel with GATE), laid out for latency:
//  * constants (conv taps, A_log, dt_bias, the norm weight) are loaded before the dependency wait,
//    and with `preload` the previous step's state too (control words, state rows, old window rows);
//  * warps 0..2S-1 each own one (token, q|k) vector: lane l convolves channels 4l..4l+3 from 8-byte
//    window loads, then the warp applies the RMS norm itself (the fma chain over the lane's 4
//    channels and the xor butterfly of gdn_fused_kernel's phase 2), so no barrier separates conv
//    and norm;
//  * warp 8 convolves the CTA's 16 v channels, warp 9 computes the gates and warp 10 (GATE) silu(z)
//    of the gated norm's outputs: none of them sits on a q/k warp's path;
//  * the next conv window is written from the registers the convolution loaded (q/k channels by one
//    CTA of the key head, v channels by their owner);
//  * GATE: the 8 CTAs of a value head form a cluster; after the delta rule each holds its 16 rows of
//    y in shared memory, and a warp per token reads the head's 128 values over distributed shared
//    memory in gdn_norm_gate_kernel's lane order (lane l: rows 4l..4l+3).
// Grid (Dv / 16, Hv), 352 threads.
constexpr int kDecS = 4, kDecKC = 4, kDecRows = 16, kDecVWarp = 8, kDecGWarp = 9, kDecZWarp = 10;
constexpr int kDecWarps = 11;

template <bool GATE, int S>
__global__ void __launch_bounds__(kDecWarps * 32)
gdn_decode_kernel(qmtp_gdn_args A, unsigned* __restrict__ err) {
  static_assert(S >= 1 && S <= kDecS, "decode shape: 1..4 tokens");
  pdl_trigger();
  constexpr int Dk = 128, Dv = 128, NP = 4, KC = kDecKC;
  __shared__ __align__(16) float qk[2 * kDecS][Dk];  // [t][q|k][Dk], normalised
  __shared__ float vs[kDecS][kDecRows];
  __shared__ float gs[kDecS], bs[kDecS];
  __shared__ __align__(16) float ys[kDecS][kDecRows];
  __shared__ float gz[kDecS][kDecRows];
  __shared__ float rs[kDecS];
  const int Hk = A.Hk, Hv = A.Hv;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int hv = blockIdx.y, dv0 = blockIdx.x * kDecRows;
  const int rep = Hv / Hk, hk = hv / rep;
  const long long C = 2LL * Hk * Dk + (long long)Hv * Dv;
  const uint16_t* conv_src = static_cast<const uint16_t*>(A.conv_src);
  const uint16_t* qkv = static_cast<const uint16_t*>(A.qkv);
  const uint16_t* conv_w = static_cast<const uint16_t*>(A.conv_w);
  const bool vec = warp < 2 * S;
  const bool vwarp = warp == kDecVWarp && lane < kDecRows;
  const int tv = warp >> 1, isk = warp & 1;
  const long long chq = (long long)isk * Hk * Dk + (long long)hk * Dk + NP * lane;  // first of 4 channels
  const long long chv = 2LL * Hk * Dk + (long long)hv * Dv + dv0 + (lane & 15);

  // ---- constants (model weights; no kernel of the decode writes them)
  uint32_t cw[8] = {};  // vec: taps of channels chq..chq+3 (bf16 pairs); v warp: cw[0..1] = taps of chv
  float Aneg = 0.0f, dtb = 0.0f, nw = 0.0f;
  if (vec) {
    const uint4 c0 = *reinterpret_cast<const uint4*>(conv_w + chq * KC);
    const uint4 c1 = *reinterpret_cast<const uint4*>(conv_w + chq * KC + 8);
    cw[0] = c0.x; cw[1] = c0.y; cw[2] = c0.z; cw[3] = c0.w; cw[4] = c1.x; cw[5] = c1.y; cw[6] = c1.z; cw[7] = c1.w;
  } else if (vwarp) {
    const uint2 c = *reinterpret_cast<const uint2*>(conv_w + chv * KC);
    cw[0] = c.x; cw[1] = c.y;
  } else if (warp == kDecGWarp && lane < S) {
    Aneg = -q_expf(A.A_log[hv]);
    dtb = bf2f(static_cast<const uint16_t*>(A.dt_bias)[hv]);
  }
  if (GATE && tid < S * kDecRows) nw = bf2f(static_cast<const uint16_t*>(A.gate_w)[dv0 + (tid & 15)]);

  // ---- state of the previous step: control words, the state rows of phase 3 (warps 0..7, rows
  // dv0 + 2w, 2w + 1) and the window's conv rows (0..KC-2).  Before the dependency wait when the
  // caller says the launch just before wrote none of them (preload), else after it.
  int off = 0, wrow = 0, cur = 0;
  float st[2][NP];
  uint2 wr[KC];                    // vec: window rows tv..tv+KC-1 of channels chq..chq+3
  uint16_t wv[KC - 1 + kDecS];     // v warp: window rows 0..KC-2+S of channel chv
  auto load_prev = [&]() -> bool {
    off = A.conv_row_off ? *A.conv_row_off : 0;
    wrow = A.win_out_row_off ? *A.win_out_row_off : 0;
    const float* sin = A.state_in;
    if (A.ring) {
      cur = *A.ring_cur;
      if (cur < 0 || cur >= A.ring_slots) return false;  // uniform over the grid
      sin = A.ring + size_t(cur) * (size_t(Hv) * Dv * Dk);
    }
    if (warp < 8) {
#pragma unroll
      for (int rr = 0; rr < 2; ++rr) {
        const float4 s4 =
            *reinterpret_cast<const float4*>(sin + (size_t(hv) * Dv + dv0 + 2 * warp + rr) * Dk + NP * lane);
        st[rr][0] = s4.x; st[rr][1] = s4.y; st[rr][2] = s4.z; st[rr][3] = s4.w;
      }
    }
    if (vec) {
#pragma unroll
      for (int j = 0; j < KC; ++j)
        if (tv + j < KC - 1) wr[j] = *reinterpret_cast<const uint2*>(conv_src + (long long)(off + tv + j) * A.ld_conv + chq);
    } else if (vwarp) {
#pragma unroll
      for (int r = 0; r < KC - 1; ++r) wv[r] = conv_src[(long long)(off + r) * A.ld_conv + chv];
    }
    return true;
  };
  bool ok = true;
  if (A.preload) ok = load_prev();
  pdl_wait();
  if (!A.preload) ok = load_prev();
  if (!ok) {
    if (tid == 0) atomicOr(err, DEVERR_BADARG);
    return;
  }
  const size_t per = size_t(Hv) * Dv * Dk;
  uint16_t* wo = A.win_out ? static_cast<uint16_t*>(A.win_out) + (long long)wrow * C : nullptr;

  if (vec) {
    // ---- phase 1+2 for vector (tv, isk): the new rows of the window, then conv + silu + RMS norm
#pragma unroll
    for (int j = 0; j < KC; ++j)
      if (tv + j >= KC - 1) wr[j] = *reinterpret_cast<const uint2*>(qkv + (long long)(tv + j - (KC - 1)) * A.ld_qkv + chq);
    float acc[NP];
#pragma unroll
    for (int c = 0; c < NP; ++c) {
      acc[c] = 0.0f;
#pragma unroll
      for (int j = 0; j < KC; ++j) {
        const uint32_t tw = cw[2 * c + (j >> 1)];
        const float tap = (j & 1) ? bfhi(tw) : bflo(tw);
        const uint32_t ww = (c < 2) ? wr[j].x : wr[j].y;
        const float wvf = (c & 1) ? bfhi(ww) : bflo(ww);
        acc[c] = __fmaf_rn(tap, wvf, acc[c]);
      }
    }
    const float4 x4 = silu_bf4(make_float4(R(acc[0]), R(acc[1]), R(acc[2]), R(acc[3])));
    const float x[NP] = {x4.x, x4.y, x4.z, x4.w};
    float ss = 0.0f;
#pragma unroll
    for (int c = 0; c < NP; ++c) ss = __fmaf_rn(x[c], x[c], ss);
    ss = warp_sum(ss);
    const float r = rsqrt_rn(__fadd_rn(__fmul_rn(ss, 1.0f / float(Dk)), 1e-6f));
    static_assert(Dk == 128, "kscale below is R(1 / sqrt(128))");
    const float kscale = __uint_as_float(0x3DB50000u);  // R(rsqrt_rn(128.0f)): 0x3DB504F3 rounded to bf16
    float o[NP];
#pragma unroll
    for (int c = 0; c < NP; ++c)
      o[c] = isk ? R(__fmul_rn(R(__fmul_rn(x[c], r)), kscale)) : __fmul_rn(R(__fmul_rn(x[c], r)), 1.0f / float(Dk));
    *reinterpret_cast<float4*>(&qk[warp][NP * lane]) = make_float4(o[0], o[1], o[2], o[3]);
    // next window, q/k channels: written by the first CTA of the key head (token 0's warp the rows
    // 0..KC-1, token t's warp row t+KC-1)
    if (wo && hv == hk * rep && blockIdx.x == 0) {
      if (tv == 0) {
#pragma unroll
        for (int j = 0; j < KC; ++j) *reinterpret_cast<uint2*>(wo + j * C + chq) = wr[j];
      } else {
        *reinterpret_cast<uint2*>(wo + (tv + KC - 1) * C + chq) = wr[KC - 1];
      }
    }
  } else if (vwarp) {
    // ---- v channel chv over the S tokens (rows 0..KC-2+S of the window)
#pragma unroll
    for (int r = KC - 1; r < KC - 1 + S; ++r) wv[r] = qkv[(long long)(r - (KC - 1)) * A.ld_qkv + chv];
    float acc[kDecS] = {};
#pragma unroll
    for (int t = 0; t < S; ++t) {
#pragma unroll
      for (int j = 0; j < KC; ++j) {
        const float tap = (j & 1) ? bfhi(cw[j >> 1]) : bflo(cw[j >> 1]);
        acc[t] = __fmaf_rn(tap, bf2f(wv[t + j]), acc[t]);
      }
    }
    const float4 v4 = silu_bf4(make_float4(R(acc[0]), R(acc[1]), R(acc[2]), R(acc[3])));
    const float vv[kDecS] = {v4.x, v4.y, v4.z, v4.w};
#pragma unroll
    for (int t = 0; t < S; ++t) vs[t][lane] = vv[t];
    if (wo) {
#pragma unroll
      for (int r = 0; r < KC - 1 + S; ++r) wo[r * C + chv] = wv[r];
    }
  } else if (warp == kDecGWarp && lane < S) {
    // ---- gates of token t = lane
    const uint16_t* av = static_cast<const uint16_t*>(A.a);
    const uint16_t* bv = static_cast<const uint16_t*>(A.b);
    const float sp = softplus_bf(R(__fadd_rn(bf2f(av[(long long)lane * A.ld_ab + hv]), dtb)));
    gs[lane] = q_expf(__fmul_rn(Aneg, sp));
    bs[lane] = sigmoid_bf(bf2f(bv[(long long)lane * A.ld_ab + hv]));
  } else if (GATE && warp == kDecZWarp && lane < kDecRows) {
    // ---- silu(z) of the gated norm's outputs (token t, row dv0 + lane)
    const uint16_t* z = static_cast<const uint16_t*>(A.gate_z);
    float zv[kDecS] = {};
#pragma unroll
    for (int t = 0; t < S; ++t) zv[t] = bf2f(z[(long long)t * A.ld_gate_z + (long long)hv * Dv + dv0 + lane]);
    const float4 g4 = silu_f32x4(make_float4(zv[0], zv[1], zv[2], zv[3]));
    const float gv[kDecS] = {g4.x, g4.y, g4.z, g4.w};
#pragma unroll
    for (int t = 0; t < S; ++t) gz[t][lane] = gv[t];
  }
  __syncthreads();

  // ---- phase 3: delta rule for rows dv0 + 2w + rr (same sequence as gdn_fused_kernel's decode path)
  if (warp < 8) {
    float op[S][2];
#pragma unroll
    for (int t = 0; t < S; ++t) {
      const float4 q4 = *reinterpret_cast<const float4*>(&qk[2 * t][NP * lane]);
      const float4 k4 = *reinterpret_cast<const float4*>(&qk[2 * t + 1][NP * lane]);
      const float qf[4] = {q4.x, q4.y, q4.z, q4.w}, kf[4] = {k4.x, k4.y, k4.z, k4.w};
      const float gt = gs[t], bt = bs[t];
      float* dst = nullptr;
      if (A.ring) {
        int slot = cur + t + 1;  // cur < ring_slots and t + 1 <= S < ring_slots
        if (slot >= A.ring_slots) slot -= A.ring_slots;
        if (A.snap || t == S - 1) dst = A.ring + size_t(slot) * per;
      } else if (t == S - 1) {
        dst = A.state_out;
      } else if (A.snap && A.state_mid) {
        dst = A.state_mid + size_t(t) * per;
      }
      float kv[2];
#pragma unroll
      for (int rr = 0; rr < 2; ++rr) {
        kv[rr] = 0.0f;
#pragma unroll
        for (int i = 0; i < NP; ++i) {
          st[rr][i] = __fmul_rn(st[rr][i], gt);
          kv[rr] = __fmaf_rn(st[rr][i], kf[i], kv[rr]);
        }
      }
#pragma unroll
      for (int d = 16; d >= 1; d >>= 1)
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) kv[rr] = __fadd_rn(kv[rr], __shfl_xor_sync(0xFFFFFFFFu, kv[rr], d));
#pragma unroll
      for (int rr = 0; rr < 2; ++rr) {
        const int d = 2 * warp + rr;
        const float delta = __fmul_rn(__fsub_rn(vs[t][d], kv[rr]), bt);
        op[t][rr] = 0.0f;
#pragma unroll
        for (int i = 0; i < NP; ++i) {
          st[rr][i] = __fmaf_rn(kf[i], delta, st[rr][i]);
          op[t][rr] = __fmaf_rn(st[rr][i], qf[i], op[t][rr]);
        }
        if (dst)
          *reinterpret_cast<float4*>(dst + (size_t(hv) * Dv + dv0 + d) * Dk + NP * lane) =
              make_float4(st[rr][0], st[rr][1], st[rr][2], st[rr][3]);
      }
    }
#pragma unroll
    for (int d = 16; d >= 1; d >>= 1)
#pragma unroll
      for (int t = 0; t < S; ++t)
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) op[t][rr] = __fadd_rn(op[t][rr], __shfl_xor_sync(0xFFFFFFFFu, op[t][rr], d));
    if (lane == 0) {
#pragma unroll
      for (int t = 0; t < S; ++t)
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) {
          const float yv = R(op[t][rr]);
          A.y[(size_t(t) * Hv + hv) * Dv + dv0 + 2 * warp + rr] = yv;
          if (GATE) ys[t][2 * warp + rr] = yv;
        }
    }
  }
  if (GATE) {
    // ---- gated norm: r_t from the value head's 128 values of y, gathered over the cluster
    __syncwarp();
    cluster_sync_all();
    if (warp < S) {
      const float4 v = ld_dsmem_v4(&ys[warp][4 * (lane & 3)], uint32_t(lane >> 2));
      float ss = 0.0f;
      ss = __fmaf_rn(v.x, v.x, ss);
      ss = __fmaf_rn(v.y, v.y, ss);
      ss = __fmaf_rn(v.z, v.z, ss);
      ss = __fmaf_rn(v.w, v.w, ss);
      ss = warp_sum(ss);
      if (lane == 0) rs[warp] = rsqrt_rn(__fadd_rn(__fmul_rn(ss, 1.0f / float(Dv)), A.gate_eps));
    }
    __syncwarp();
    cluster_arrive_release();  // this CTA's remote reads are done
    __syncthreads();
    if (tid < S * kDecRows) {
      const int t = tid >> 4, d = tid & 15;
      const float xn = R(__fmul_rn(nw, R(__fmul_rn(ys[t][d], rs[t]))));
      static_cast<uint16_t*>(A.gate_out)[(long long)t * A.ld_gate_out + (long long)hv * Dv + dv0 + d] =
          f2bf(__fmul_rn(xn, gz[t][d]));
    }
    __syncwarp();
    cluster_wait_acquire();  // no CTA leaves while a peer may still read its ys
  }
}

static int g_gdn_mode = 0;

}  // namespace qmtp

using namespace qmtp;

extern "C" int qmtp_gdn_step(const void* q, const void* k, const void* v, const float* g, const float* beta,
                             const float* state_in, void* y, float* state_out, float* state_mid, int B, int T,
                             int Hk, int Hv, int Dk, int Dv, void* stream) {
  if (!q || !k || !v || !g || !beta || !state_in || !y || !state_out) return QMTP_ERR_ARG;
  if (B < 1 || T < 1 || Hk < 1 || Hv < 1 || Hv % Hk != 0 || Dv < 1 || Dk != 128) return QMTP_ERR_SHAPE;
  if (T > 1 && !state_mid) return QMTP_ERR_ARG;
  const long long rows = (long long)B * Hv * Dv;
  const int wpb = 8;
  const long long blocks = (rows + wpb - 1) / wpb;
  if (blocks > 0x7FFFFFFF) return QMTP_ERR_SHAPE;
  launch_kernel(gdn_step_kernel<4>, dim3(unsigned(blocks)), dim3(wpb * 32), 0, static_cast<cudaStream_t>(stream), 
      static_cast<const uint16_t*>(q), static_cast<const uint16_t*>(k), static_cast<const uint16_t*>(v), g, beta,
      state_in, static_cast<uint16_t*>(y), state_out, T > 1 ? state_mid : nullptr, B, T, Hk, Hv, Dv);
  return cudaGetLastError() == cudaSuccess ? QMTP_OK : QMTP_ERR_CUDA;
}

extern "C" int qmtp_gdn_fused_ex(const qmtp_gdn_args* args, void* stream) {
  if (!args) return QMTP_ERR_ARG;
  const qmtp_gdn_args& A = *args;
  if (!A.conv_src || !A.qkv || !A.conv_w || !A.a || !A.b || !A.A_log || !A.dt_bias || !A.y) return QMTP_ERR_ARG;
  if (A.Dk != 128 || A.S < 1 || A.S > 64 || A.KC < 1 || A.KC > 8 || A.Hk < 1 || A.Hv % A.Hk != 0 || A.Dv < 1)
    return QMTP_ERR_SHAPE;
  if (A.ring) {
    if (!A.ring_cur || A.ring_slots <= A.S) return QMTP_ERR_ARG;
  } else {
    if (!A.state_in || !A.state_out || (A.snap && A.S > 1 && !A.state_mid)) return QMTP_ERR_ARG;
  }
  const void* sp[] = {A.state_in, A.state_out, A.state_mid, A.ring};
  for (const void* p : sp)
    if (p && !aligned16(p)) return QMTP_ERR_ALIGN;
  const bool gate = A.gate_out != nullptr;
  if (gate && (!A.gate_z || !A.gate_w)) return QMTP_ERR_ARG;
  if (gate && (A.Dv != 128 || A.ld_gate_z < (long long)A.Hv * A.Dv || A.ld_gate_out < (long long)A.Hv * A.Dv))
    return QMTP_ERR_SHAPE;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto a8 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 7u) == 0; };
  const long long C = 2LL * A.Hk * A.Dk + (long long)A.Hv * A.Dv;
  const bool decode = g_gdn_mode == 0 && A.S <= kDecS && A.KC == kDecKC && A.Dv == 128 && aligned16(A.conv_w) &&
                      a8(A.conv_src) && a8(A.qkv) && A.ld_conv % 4 == 0 && A.ld_qkv % 4 == 0 && C % 4 == 0 &&
                      (!A.win_out || a8(A.win_out));
  if (decode) {
    const dim3 grid(128 / kDecRows, A.Hv), block(kDecWarps * 32);
    auto go = [&](auto kern_gate, auto kern_plain) {
      if (gate)
        launch_kernel_cluster(kern_gate, grid, block, 0, st, 128 / kDecRows, A, device_error_ptr());
      else
        launch_kernel(kern_plain, grid, block, 0, st, A, device_error_ptr());
    };
    switch (A.S) {
      case 1: go(gdn_decode_kernel<true, 1>, gdn_decode_kernel<false, 1>); break;
      case 2: go(gdn_decode_kernel<true, 2>, gdn_decode_kernel<false, 2>); break;
      case 3: go(gdn_decode_kernel<true, 3>, gdn_decode_kernel<false, 3>); break;
      default: go(gdn_decode_kernel<true, 4>, gdn_decode_kernel<false, 4>); break;
    }
    return cudaGetLastError() == cudaSuccess ? QMTP_OK : QMTP_ERR_CUDA;
  }
  const size_t smem = size_t(A.S) * (2 * 128 + kFusedDVB + 2) * sizeof(float);
  dim3 grid(A.Hv, (A.Dv + kFusedDVB - 1) / kFusedDVB);
  launch_kernel(gdn_fused_kernel<4>, dim3(grid), dim3(kFusedWarps * 32), smem, st, A, device_error_ptr());
  if (cudaGetLastError() != cudaSuccess) return QMTP_ERR_CUDA;
  if (!gate) return QMTP_OK;
  const int rows = A.S * A.Hv, wpb = 8;
  launch_kernel(gdn_norm_gate_kernel<4>, dim3((rows + wpb - 1) / wpb), dim3(wpb * 32), 0, st, static_cast<const float*>(A.y),
                static_cast<const uint16_t*>(A.gate_z), A.ld_gate_z, static_cast<const uint16_t*>(A.gate_w),
                static_cast<uint16_t*>(A.gate_out), A.ld_gate_out, A.S, A.Hv, A.gate_eps);
  return cudaGetLastError() == cudaSuccess ? QMTP_OK : QMTP_ERR_CUDA;
}

extern "C" int qmtp_gdn_set_mode(int mode) {
  const int prev = g_gdn_mode;
  if (mode == 0 || mode == 1) g_gdn_mode = mode;
  return prev;
}

extern "C" int qmtp_gdn_fused(const void* win, const void* conv_w, const void* a, const void* b, int ld_ab,
                              const float* A_log, const void* dt_bias, const float* state_in, float* y,
                              float* state_out, float* state_mid, int S, int Hk, int Hv, int Dk, int Dv, int KC,
                              int snap, void* stream) {
  if (!win) return QMTP_ERR_ARG;
  qmtp_gdn_args A{};
  const int C = 2 * Hk * Dk + Hv * Dv;
  A.conv_src = win;
  A.ld_conv = C;
  A.conv_row_off = nullptr;
  A.qkv = static_cast<const uint16_t*>(win) + (long long)(KC - 1) * C;
  A.ld_qkv = C;
  A.win_out = nullptr;
  A.win_out_row_off = nullptr;
  A.conv_w = conv_w;
  A.a = a;
  A.b = b;
  A.ld_ab = ld_ab;
  A.A_log = A_log;
  A.dt_bias = dt_bias;
  A.state_in = state_in;
  A.state_out = state_out;
  A.state_mid = state_mid;
  A.ring = nullptr;
  A.ring_cur = nullptr;
  A.ring_slots = 0;
  A.y = y;
  A.S = S;
  A.Hk = Hk;
  A.Hv = Hv;
  A.Dk = Dk;
  A.Dv = Dv;
  A.KC = KC;
  A.snap = snap;
  return qmtp_gdn_fused_ex(&A, stream);
}

extern "C" int qmtp_gdn_norm_gate(const float* y, const void* z, int ld_z, const void* w, void* out, int ld_out,
                                  int S, int H, int Dv, float eps, void* stream) {
  if (!y || !z || !w || !out) return QMTP_ERR_ARG;
  if (S < 1 || H < 1 || Dv != 128 || ld_z < H * Dv || ld_out < H * Dv) return QMTP_ERR_SHAPE;
  const int rows = S * H, wpb = 8;
  launch_kernel(gdn_norm_gate_kernel<4>, dim3((rows + wpb - 1) / wpb), dim3(wpb * 32), 0, static_cast<cudaStream_t>(stream), 
      y, static_cast<const uint16_t*>(z), ld_z, static_cast<const uint16_t*>(w), static_cast<uint16_t*>(out), ld_out,
      S, H, eps);
  return cudaGetLastError() == cudaSuccess ? QMTP_OK : QMTP_ERR_CUDA;
}
