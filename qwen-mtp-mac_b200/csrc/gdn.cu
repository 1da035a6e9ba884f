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
  const size_t smem = size_t(A.S) * (2 * 128 + kFusedDVB + 2) * sizeof(float);
  dim3 grid(A.Hv, (A.Dv + kFusedDVB - 1) / kFusedDVB);
  launch_kernel(gdn_fused_kernel<4>, dim3(grid), dim3(kFusedWarps * 32), smem, static_cast<cudaStream_t>(stream), A, device_error_ptr());
  return cudaGetLastError() == cudaSuccess ? QMTP_OK : QMTP_ERR_CUDA;
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
