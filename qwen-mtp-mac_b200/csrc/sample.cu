// Exact speculative sampling (temperature > 0) for the MTP verify loop: engine.py:91-152
// (Engine._dist, _sample_first, _verify).  The drafts are deterministic (MTP argmax), so draft i is
// accepted with probability p_i(d_i); on rejection the token is drawn from p_i without d_i and the
// cycle stops; if every draft is accepted a bonus token is drawn from row k.  The emitted tokens
// are written over the verify argmax rows, so the greedy bookkeeping that follows (qmtp_mtp_accept:
// counts a[i] == d_i, commits KEEP, rolls the state back) handles the sampled cycle unchanged.
//
// p_i is Engine._dist over the K candidates of the two-stage head (every other logit is -inf
// there): temperature, top_k, log-softmax, top_p on the sorted exclusive cumulative sum, min_p,
// renormalisation.  One CTA per call.  The candidates are sorted in shared memory (exact logit
// descending, vocabulary id ascending: a total order, so the sort network does not matter); the
// elementwise steps run across the threads and every sum and scan runs on thread 0 in index order.
// That fixed sequence is oracle/qmtp_oracle.c:qo_sample's, so the decisions are bit-identical.
//
// Random numbers: Philox4x32-10 (Salmon et al., SC 2011), key = the 64-bit seed in the control
// block, counter = (call counter, row, use, 0) with use 0 for the accept test and 1 for a draw; a
// uniform is the top 24 bits of word 0 times 2^-24.  Every call advances the call counter.
#include <climits>

#include "common.cuh"

namespace qmtp {
namespace {

constexpr int kSampMaxK = 2048;  // lm_head2.py:32-36: k_for returns at most 2048
constexpr int kSampThreads = 256;

__device__ __forceinline__ uint4 philox4x32_10(uint4 c, uint32_t k0, uint32_t k1) {
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    if (r > 0) {
      k0 += 0x9E3779B9u;
      k1 += 0xBB67AE85u;
    }
    const uint32_t lo0 = 0xD2511F53u * c.x, hi0 = __umulhi(0xD2511F53u, c.x);
    const uint32_t lo1 = 0xCD9E8D57u * c.z, hi1 = __umulhi(0xCD9E8D57u, c.z);
    c = make_uint4(hi1 ^ c.y ^ k0, lo1, hi0 ^ c.w ^ k1, lo0);
  }
  return c;
}

__device__ __forceinline__ float uniform01(uint32_t slo, uint32_t shi, uint32_t ctr, uint32_t row, uint32_t use) {
  const uint4 o = philox4x32_10(make_uint4(ctr, row, use, 0u), slo, shi);
  return __fmul_rn(__uint2float_rn(o.x >> 8), 1.0f / 16777216.0f);
}

// a before b: larger logit first, then smaller vocabulary id
__device__ __forceinline__ bool before(float la, int ia, float lb, int ib) {
  return la > lb || (la == lb && ia < ib);
}

// categorical draw by inverse CDF over the kept candidates, skipping vocabulary id excl (thread 0)
__device__ int draw(const int* si, const float* p, int n, int excl, float u) {
  float tot = 0.0f;
  for (int j = 0; j < n; ++j)
    if (si[j] != excl) tot = __fadd_rn(tot, p[j]);
  const float r = __fmul_rn(u, tot);
  float acc = 0.0f;
  int last = si[0];
  for (int j = 0; j < n; ++j) {
    if (si[j] == excl) continue;
    acc = __fadd_rn(acc, p[j]);
    last = si[j];
    if (acc > r) return si[j];
  }
  return last;
}

struct SampParams {
  float T, top_p, min_p;
  int top_k, V;
};

__global__ void __launch_bounds__(kSampThreads) sample_kernel(const int32_t* __restrict__ idx,
                                                              const uint16_t* __restrict__ fine, int K, int ld,
                                                              const int32_t* __restrict__ drafts, int k,
                                                              int first_row, SampParams sp, int* __restrict__ ctrl,
                                                              int32_t* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  __shared__ float sl[kSampMaxK];  // sorted logits, then z = l / T, then log-probabilities
  __shared__ int si[kSampMaxK];    // sorted vocabulary ids
  __shared__ float sp_[kSampMaxK]; // exponentials, then probabilities
  __shared__ float s_L, s_sum;
  __shared__ int s_n, s_stop;
  const int tid = threadIdx.x;
  const uint32_t ctr = uint32_t(ctrl[QMTP_CTRL_RNG]);
  const uint32_t slo = uint32_t(ctrl[QMTP_CTRL_SEED_LO]), shi = uint32_t(ctrl[QMTP_CTRL_SEED_HI]);
  int P = 1;
  while (P < K) P <<= 1;
  const int r0 = first_row >= 0 ? first_row : 0, r1 = first_row >= 0 ? first_row : k;
  for (int r = r0; r <= r1; ++r) {
    // ---- candidates of row r, sorted
    for (int j = tid; j < P; j += blockDim.x) {
      if (j < K) {
        sl[j] = bf2f(fine[size_t(r) * ld + j]);
        si[j] = idx[size_t(r) * ld + j];
      } else {
        sl[j] = __int_as_float(0xFF800000);
        si[j] = INT_MAX;
      }
    }
    __syncthreads();
    for (int size = 2; size <= P; size <<= 1) {
      for (int stride = size >> 1; stride > 0; stride >>= 1) {
        for (int t = tid; t < P / 2; t += blockDim.x) {
          const int i = 2 * t - (t & (stride - 1)), j = i + stride;
          const bool up = (i & size) == 0;
          const float li = sl[i], lj = sl[j];
          const int ii = si[i], ij = si[j];
          if (up ? before(lj, ij, li, ii) : before(li, ii, lj, ij)) {
            sl[i] = lj; sl[j] = li;
            si[i] = ij; si[j] = ii;
          }
        }
        __syncthreads();
      }
    }
    // ---- Engine._dist
    int n = K;
    if (sp.top_k > 0 && sp.top_k < sp.V && sp.top_k < n) n = sp.top_k;
    for (int j = tid; j < n; j += blockDim.x) sl[j] = __fdiv_rn(sl[j], sp.T);
    __syncthreads();
    const float m = sl[0];
    for (int j = tid; j < n; j += blockDim.x) sp_[j] = q_expf(__fsub_rn(sl[j], m));
    __syncthreads();
    if (tid == 0) {
      float s = 0.0f;
      for (int j = 0; j < n; ++j) s = __fadd_rn(s, sp_[j]);
      s_L = __fadd_rn(m, q_logf(s));
    }
    __syncthreads();
    const float L = s_L;
    for (int j = tid; j < n; j += blockDim.x) sl[j] = __fsub_rn(sl[j], L);
    __syncthreads();
    if (sp.top_p < 1.0f) {
      for (int j = tid; j < n; j += blockDim.x) sp_[j] = q_expf(sl[j]);
      __syncthreads();
      if (tid == 0) {
        float acc = 0.0f;
        int np_ = n;
        for (int j = 0; j < n; ++j) {
          const float inc = __fadd_rn(acc, sp_[j]);
          if (!(__fsub_rn(inc, sp_[j]) < sp.top_p)) { np_ = j; break; }
          acc = inc;
        }
        s_n = np_;
      }
      __syncthreads();
      n = s_n;
    }
    if (sp.min_p > 0.0f) {
      if (tid == 0) {
        const float thr = __fadd_rn(sl[0], q_logf(sp.min_p));
        int nm = n;
        for (int j = 0; j < n; ++j)
          if (!(sl[j] >= thr)) { nm = j; break; }
        s_n = nm;
      }
      __syncthreads();
      n = s_n;
    }
    const float l0 = sl[0];
    for (int j = tid; j < n; j += blockDim.x) sp_[j] = q_expf(__fsub_rn(sl[j], l0));
    __syncthreads();
    if (tid == 0) {
      float s2 = 0.0f;
      for (int j = 0; j < n; ++j) s2 = __fadd_rn(s2, sp_[j]);
      s_sum = s2;
    }
    __syncthreads();
    const float s2 = s_sum;
    for (int j = tid; j < n; j += blockDim.x) sp_[j] = __fdiv_rn(sp_[j], s2);
    __syncthreads();
    // ---- decision (thread 0)
    if (tid == 0) {
      int stop = 1;
      if (first_row >= 0) {
        out[r] = draw(si, sp_, n, -1, uniform01(slo, shi, ctr, 0u, 1u));
      } else if (r == k) {
        out[k] = draw(si, sp_, n, -1, uniform01(slo, shi, ctr, uint32_t(k), 1u));
      } else {
        const int d = drafts[r];
        float pd = 0.0f;
        for (int j = 0; j < n; ++j)
          if (si[j] == d) pd = sp_[j];
        if (uniform01(slo, shi, ctr, uint32_t(r), 0u) < pd) {
          out[r] = d;
          stop = 0;
        } else {
          out[r] = draw(si, sp_, n, d, uniform01(slo, shi, ctr, uint32_t(r), 1u));
        }
      }
      s_stop = stop;
    }
    __syncthreads();
    if (s_stop) break;
  }
  if (tid == 0) ctrl[QMTP_CTRL_RNG] = int(ctr + 1u);
}

}  // namespace
}  // namespace qmtp

using namespace qmtp;

extern "C" int qmtp_sample(const int* idx, const void* fine, int K, int ld, const int* drafts, int k, int first_row,
                           const qmtp_sampling* sp, int V, int* ctrl, int* out, void* stream) {
  if (!idx || !fine || !sp || !ctrl || !out || (first_row < 0 && !drafts)) return QMTP_ERR_ARG;
  if (K < 1 || K > kSampMaxK || ld < K || V < 1) return QMTP_ERR_SHAPE;
  if (first_row < 0 && (k < 1 || k > QMTP_CTRL_MAX_K)) return QMTP_ERR_SHAPE;
  if (!(sp->temperature > 0.0f) || !(sp->top_p > 0.0f) || sp->top_p > 1.0f || sp->min_p < 0.0f || sp->min_p > 1.0f ||
      sp->top_k < 0)
    return QMTP_ERR_ARG;
  const SampParams p{sp->temperature, sp->top_p, sp->min_p, sp->top_k, V};
  launch_kernel(sample_kernel, dim3(1), dim3(kSampThreads), 0, static_cast<cudaStream_t>(stream), idx,
                static_cast<const uint16_t*>(fine), K, ld, drafts, k, first_row, p, ctrl, out);
  return cudaGetLastError() == cudaSuccess ? QMTP_OK : QMTP_ERR_CUDA;
}
