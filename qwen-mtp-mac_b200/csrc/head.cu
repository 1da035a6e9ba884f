// Two-stage lm_head on B200 (lm_head2.py:14-29): coarse 4-bit logits over the full vocabulary (the
// qmv kernel), exact top-k selection, exact bf16 rescoring of the k candidate rows, argmax.
//
// Selection order: value descending, vocab index ascending (argpartition leaves ties open; this
// resolves them deterministically).  bf16 values are compared through the order-preserving 16-bit
// key `key16`; a candidate is the 64-bit word (key16 << 32) | (0xFFFFFFFF - index), so "larger
// word" means "better candidate" and any max/sort over these words is order-independent.
//
//   topk_partial  grid (G, M): block g of row m selects the top k of its slice of the row (the k-th
//                 largest key found bit by bit with block-wide counts) and writes k candidate words;
//   topk_merge    grid (M): bitonic-sorts the G*k candidate words, keeps the first k, rescoring
//                 each against the bf16 weight row (one warp per candidate, fixed reduction order
//                 of oracle qo_dot_bf16), and takes the argmax of the fine logits;
//   argmax        the same candidate words with k = 1 (draft head: argmax over the full vocab).
#include <algorithm>
#include <mutex>

#include "common.cuh"

namespace qmtp {

__device__ __forceinline__ uint32_t key16(uint16_t b) {
  return (b & 0x8000u) ? uint32_t(~b & 0xFFFFu) : uint32_t(b | 0x8000u);
}
__device__ __forceinline__ uint64_t cand_word(uint32_t key, uint32_t idx) {
  return (uint64_t(key) << 32) | uint64_t(0xFFFFFFFFu - idx);
}
__device__ __forceinline__ uint32_t cand_idx(uint64_t w) { return 0xFFFFFFFFu - uint32_t(w & 0xFFFFFFFFu); }

// Finds (within the bins above `base`) the bin b where the count from the top reaches k.
// hist[256]; warp 0 only.  Returns via s_res[0] = b, s_res[1] = count strictly above b.
__device__ void find_bin(const int* hist, int k, int base, int* s_res) {
  const int lane = threadIdx.x & 31;
  int local[8], s = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) { local[i] = hist[8 * lane + i]; s += local[i]; }
  int incl = s;  // suffix sum over lanes >= lane
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int o = __shfl_down_sync(0xFFFFFFFFu, incl, d);
    if (lane + d < 32) incl += o;
  }
  const int excl = incl - s;
  if (base + excl < k && base + incl >= k) {
    int cum = base + excl;
#pragma unroll
    for (int i = 7; i >= 0; --i) {
      if (cum + local[i] >= k) { s_res[0] = 8 * lane + i; s_res[1] = cum; break; }
      cum += local[i];
    }
  }
}

// Exact top-k of n (>= k) 16-bit keys in shared memory: T = the k-th largest key and g = #(key > T)
// (so g < k <= g + #(key == T)).  T is built from the top bit down, two bits a round: the largest
// candidate c with #(key >= T | c) >= k (the count only falls as the threshold rises).  Each thread
// holds its contiguous share of the keys in registers and a round is three block-wide counts; a
// histogram instead piles its shared-memory atomics onto the few bins logit keys occupy.
// blockDim.x == kTopkThreads, n <= kTopkThreads * 2 * kSelRegs; s_cnt: 3 * 32 ints.
constexpr int kTopkThreads = 256;
constexpr int kSelRegs = 24;  // 48 keys a thread: slices up to 12288 keys
__device__ void block_select16(const uint16_t* keys, int n, int k, int* s_cnt, int& T, int& g) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = int(blockDim.x) >> 5;
  const int per = (n + int(blockDim.x) - 1) / int(blockDim.x);
  const int a0 = min(n, tid * per), a1 = min(n, a0 + per);
  uint32_t kr[kSelRegs];  // key pairs; missing keys are 0, below every threshold asked (>= 1)
#pragma unroll
  for (int i = 0; i < kSelRegs; ++i) {
    const int e0 = a0 + 2 * i, e1 = e0 + 1;
    kr[i] = (e0 < a1 ? uint32_t(keys[e0]) : 0u) | ((e1 < a1 ? uint32_t(keys[e1]) : 0u) << 16);
  }
  auto count3 = [&](uint32_t t1, uint32_t t2, uint32_t t3, int (&c)[3]) {
    int c1 = 0, c2 = 0, c3 = 0;
#pragma unroll
    for (int i = 0; i < kSelRegs; ++i) {
      const uint32_t lo = kr[i] & 0xFFFFu, hi = kr[i] >> 16;
      c1 += int(lo >= t1) + int(hi >= t1);
      c2 += int(lo >= t2) + int(hi >= t2);
      c3 += int(lo >= t3) + int(hi >= t3);
    }
    c1 = __reduce_add_sync(0xFFFFFFFFu, c1);
    c2 = __reduce_add_sync(0xFFFFFFFFu, c2);
    c3 = __reduce_add_sync(0xFFFFFFFFu, c3);
    if (lane == 0) { s_cnt[warp] = c1; s_cnt[32 + warp] = c2; s_cnt[64 + warp] = c3; }
    __syncthreads();
    c[0] = c[1] = c[2] = 0;
    for (int w = 0; w < nw; ++w) { c[0] += s_cnt[w]; c[1] += s_cnt[32 + w]; c[2] += s_cnt[64 + w]; }
    __syncthreads();
  };
  uint32_t t = 0;
  for (int b = 14; b >= 0; b -= 2) {  // bits b+1, b
    int c[3];
    count3(t | (1u << b), t | (2u << b), t | (3u << b), c);
    t |= (c[2] >= k ? 3u : c[1] >= k ? 2u : c[0] >= k ? 1u : 0u) << b;
  }
  T = int(t);
  if (t == 0xFFFFu) {
    g = 0;
  } else {
    int c[3];
    count3(t + 1, t + 1, t + 1, c);
    g = c[0];
  }
}



__global__ void __launch_bounds__(kTopkThreads)
topk_partial_kernel(const uint16_t* __restrict__ vals, long long ld, int V, int k, uint64_t* __restrict__ cand) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ __align__(16) unsigned char sm_raw[];
  int* hist = reinterpret_cast<int*>(sm_raw);
  int* s_res = hist + 256;
  int* s_warp = s_res + 4;
  uint16_t* keys = reinterpret_cast<uint16_t*>(s_warp + 32);
  const int G = gridDim.x, blk = blockIdx.x, m = blockIdx.y, tid = threadIdx.x;
  const int i0 = int((long long)blk * V / G), i1 = int((long long)(blk + 1) * V / G), n = i1 - i0;
  const uint16_t* row = vals + (long long)m * ld + i0;
  {
    // 16-byte loads over the aligned middle of the slice, issued four at a time before any is used
    // (the slice is ~8K keys: a plain element loop would wait out one L2 round trip per element)
    const int mis = int((reinterpret_cast<uintptr_t>(row) >> 1) & 7u);
    const int head = min(n, mis ? 8 - mis : 0);
    const int nv = (n - head) / 8, tail0 = head + 8 * nv;
    for (int i = tid; i < head; i += blockDim.x) keys[i] = uint16_t(key16(row[i]));
    for (int i = tail0 + tid; i < n; i += blockDim.x) keys[i] = uint16_t(key16(row[i]));
    const uint4* v = reinterpret_cast<const uint4*>(row + head);
    constexpr int U = 4;
    for (int c0 = tid; c0 < nv; c0 += U * int(blockDim.x)) {
      uint4 u[U];
#pragma unroll
      for (int j = 0; j < U; ++j)
        if (c0 + j * int(blockDim.x) < nv) u[j] = v[c0 + j * blockDim.x];
#pragma unroll
      for (int j = 0; j < U; ++j) {
        const int c = c0 + j * int(blockDim.x);
        if (c < nv) {
          const uint32_t w[4] = {u[j].x, u[j].y, u[j].z, u[j].w};
          uint16_t* kd = keys + head + 8 * c;
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            kd[2 * e] = uint16_t(key16(uint16_t(w[e] & 0xFFFFu)));
            kd[2 * e + 1] = uint16_t(key16(uint16_t(w[e] >> 16)));
          }
        }
      }
    }
  }
  __syncthreads();
  int T, g;
  block_select16(keys, n, k, hist, T, g);
  // emit: every key > T, then the (k - g) lowest-index keys == T, each thread over a contiguous range
  const int per = (n + blockDim.x - 1) / blockDim.x;
  const int a0 = min(n, tid * per), a1 = min(n, a0 + per);
  int cgt = 0, ceq = 0;
  for (int i = a0; i < a1; ++i) {
    const int kk = keys[i];
    cgt += kk > T;
    ceq += kk == T;
  }
  int tot;
  int ogt = block_excl_scan(cgt, s_warp, tot);
  int oeq = block_excl_scan(ceq, s_warp, tot);
  uint64_t* out = cand + ((long long)m * G + blk) * k;
  for (int i = a0; i < a1; ++i) {
    const int kk = keys[i];
    if (kk > T) {
      out[ogt++] = cand_word(uint32_t(kk), uint32_t(i0 + i));
    } else if (kk == T) {
      if (oeq < k - g) out[g + oeq] = cand_word(uint32_t(kk), uint32_t(i0 + i));
      ++oeq;
    }
  }
}

constexpr int kMergeThreads = 1024;

// Sorts G*k candidate words of row m (descending), keeps k, rescoring + argmax.  W may be null
// (selection only).  out_words (may be null): the k kept words with their vocabulary index moved
// up by idx_base (a vocabulary shard's first row), the form qmtp_lmhead2_merge takes.
__global__ void __launch_bounds__(kMergeThreads)
topk_merge_kernel(const uint64_t* __restrict__ cand, int G, int k, int NP, const uint16_t* __restrict__ W,
                  const uint16_t* __restrict__ h, int K, int32_t* __restrict__ out_idx,
                  uint16_t* __restrict__ out_fine, int32_t* __restrict__ out_amax, uint32_t idx_base,
                  uint64_t* __restrict__ out_words) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ __align__(16) unsigned char sm_raw[];
  uint64_t* s = reinterpret_cast<uint64_t*>(sm_raw);  // [NP]
  uint64_t* fk = s + NP;                              // [k] fine candidate words
  const int m = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int n = G * k;
  for (int i = tid; i < NP; i += blockDim.x) s[i] = i < n ? cand[(long long)m * n + i] : 0ull;
  __syncthreads();
  for (int size = 2; size <= NP; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = tid; i < NP / 2; i += blockDim.x) {
        const int lo = 2 * i - (i & (stride - 1)), hi = lo + stride;
        const bool desc = (lo & size) == 0;
        const uint64_t a = s[lo], b = s[hi];
        if ((a < b) == desc) { s[lo] = b; s[hi] = a; }
      }
      __syncthreads();
    }
  }
  for (int j = tid; j < k; j += blockDim.x) {
    out_idx[(long long)m * k + j] = int32_t(cand_idx(s[j]));
    if (out_words) out_words[(long long)m * k + j] = cand_word(uint32_t(s[j] >> 32), cand_idx(s[j]) + idx_base);
  }
  if (!W) return;
  const uint16_t* hr = h + (long long)m * K;
  for (int j = warp; j < k; j += blockDim.x / 32) {
    const uint32_t v = cand_idx(s[j]);
    const uint16_t* wr = W + (long long)v * K;
    float acc = 0.0f;
    // the weight row's chunks of this lane (c = lane, lane + 32, ...) are fetched 8 at a time before
    // the fma chain consumes them in ascending order (h is small and stays in L1)
    constexpr int kB = 8;
    for (int c0 = lane; c0 < K / 8; c0 += 32 * kB) {
      uint4 w4[kB];
#pragma unroll
      for (int u = 0; u < kB; ++u)
        if (c0 + 32 * u < K / 8) w4[u] = ldg_nc_v4(wr + 8 * (c0 + 32 * u));
#pragma unroll
      for (int u = 0; u < kB; ++u) {
        if (c0 + 32 * u >= K / 8) break;
        const uint4 h4 = *reinterpret_cast<const uint4*>(hr + 8 * (c0 + 32 * u));
        const uint32_t ww[4] = {w4[u].x, w4[u].y, w4[u].z, w4[u].w}, hh[4] = {h4.x, h4.y, h4.z, h4.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          acc = __fmaf_rn(bflo(ww[e]), bflo(hh[e]), acc);
          acc = __fmaf_rn(bfhi(ww[e]), bfhi(hh[e]), acc);
        }
      }
    }
    acc = warp_sum(acc);
    const uint16_t f = f2bf(acc);
    if (lane == 0) {
      out_fine[(long long)m * k + j] = f;
      fk[j] = cand_word(key16(f), v);
    }
  }
  __syncthreads();
  if (warp == 0) {
    uint64_t best = 0;
    for (int j = lane; j < k; j += 32) best = max(best, fk[j]);
#pragma unroll
    for (int d = 16; d >= 1; d >>= 1) {
      const uint64_t o = __shfl_xor_sync(0xFFFFFFFFu, best, d);
      best = max(best, o);
    }
    if (lane == 0 && out_amax) out_amax[m] = int32_t(cand_idx(best));
  }
}

// Argmax over V (per row): block maxima of candidate words, then one block per row.
__global__ void __launch_bounds__(256)
argmax_partial_kernel(const uint16_t* __restrict__ vals, long long ld, int V, uint64_t* __restrict__ part) {
  pdl_trigger();
  pdl_wait();
  const int G = gridDim.x, blk = blockIdx.x, m = blockIdx.y, tid = threadIdx.x;
  const int i0 = int((long long)blk * V / G), i1 = int((long long)(blk + 1) * V / G);
  const uint16_t* row = vals + (long long)m * ld;
  uint64_t best = 0;
#pragma unroll 4
  for (int i = i0 + tid; i < i1; i += blockDim.x) best = max(best, cand_word(key16(row[i]), uint32_t(i)));
#pragma unroll
  for (int d = 16; d >= 1; d >>= 1) best = max(best, __shfl_xor_sync(0xFFFFFFFFu, best, d));
  __shared__ uint64_t sw[8];
  if ((tid & 31) == 0) sw[tid >> 5] = best;
  __syncthreads();
  if (tid == 0) {
    for (int w = 1; w < int(blockDim.x >> 5); ++w) best = max(best, sw[w]);
    part[(long long)m * G + blk] = best;
  }
}

// ids (may be null): the vocabulary id of every scored row (a draft head over a vocabulary subset,
// mtp.py:165-167 DraftHead.token); out gets ids[i] and out_local (may be null) the row i itself.
__global__ void argmax_final_kernel(const uint64_t* __restrict__ part, int G, const int32_t* __restrict__ ids,
                                    int32_t* __restrict__ out, int32_t* __restrict__ out_local) {
  pdl_trigger();
  pdl_wait();
  const int m = blockIdx.x, lane = threadIdx.x;
  uint64_t best = 0;
  for (int i = lane; i < G; i += 32) best = max(best, part[(long long)m * G + i]);
#pragma unroll
  for (int d = 16; d >= 1; d >>= 1) best = max(best, __shfl_xor_sync(0xFFFFFFFFu, best, d));
  if (lane == 0) {
    const int32_t i = int32_t(cand_idx(best));
    out[m] = ids ? ids[i] : i;
    if (out_local) out_local[m] = i;
  }
}

// ---- large candidate sets (k > 256, up to 2048: lm_head2.py:32-36 k_for with top_k up to 512)
// topk_select: per row, the k largest of the G*k candidate words (all distinct: the index is part of
// the word) by a most-significant-digit radix select over the six bytes that vary (the 16-bit key,
// then the index), then the k words compacted and bitonic-sorted in shared memory.  The same total
// order as topk_merge, so the same k candidates in the same order.
constexpr int kSelectThreads = 1024;
constexpr int kSelectMaxK = 2048;
__global__ void __launch_bounds__(kSelectThreads)
topk_select_kernel(const uint64_t* __restrict__ cand, int n, int k, int32_t* __restrict__ out_idx,
                   uint64_t* __restrict__ sel_words, uint32_t idx_base, uint64_t* __restrict__ out_words) {
  pdl_trigger();
  pdl_wait();
  __shared__ int hist[256];
  __shared__ int s_res[4];
  __shared__ int s_cnt;
  __shared__ uint64_t s[kSelectMaxK];
  const int m = blockIdx.x, tid = threadIdx.x;
  const uint64_t* row = cand + (long long)m * n;
  uint64_t prefix = 0, pmask = 0;
  int need = k;
  const int shifts[6] = {40, 32, 24, 16, 8, 0};
  for (int pass = 0; pass < 6; ++pass) {
    const int sh = shifts[pass];
    for (int i = tid; i < 256; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    for (int i = tid; i < n; i += blockDim.x) {
      const uint64_t w = row[i];
      if ((w & pmask) == prefix) atomicAdd(&hist[int((w >> sh) & 255u)], 1);
    }
    __syncthreads();
    if (tid < 32) find_bin(hist, need, 0, s_res);
    __syncthreads();
    const int b = s_res[0];
    need -= s_res[1];
    prefix |= uint64_t(b) << sh;
    pmask |= uint64_t(255) << sh;
    __syncthreads();
  }
  // prefix is now the k-th largest word (the top two bytes of every word are zero)
  if (tid == 0) s_cnt = 0;
  __syncthreads();
  for (int i = tid; i < n; i += blockDim.x) {
    const uint64_t w = row[i];
    if (w >= prefix) {
      const int pos = atomicAdd(&s_cnt, 1);
      if (pos < kSelectMaxK) s[pos] = w;  // exactly k words reach here (the words are distinct)
    }
  }
  int P = 1;
  while (P < k) P <<= 1;
  __syncthreads();
  for (int i = k + tid; i < P; i += blockDim.x) s[i] = 0ull;
  __syncthreads();
  for (int size = 2; size <= P; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = tid; i < P / 2; i += blockDim.x) {
        const int lo = 2 * i - (i & (stride - 1)), hi = lo + stride;
        const bool desc = (lo & size) == 0;
        const uint64_t a = s[lo], bb = s[hi];
        if ((a < bb) == desc) {
          s[lo] = bb;
          s[hi] = a;
        }
      }
      __syncthreads();
    }
  }
  for (int j = tid; j < k; j += blockDim.x) {
    const uint64_t w = s[j];
    out_idx[(long long)m * k + j] = int32_t(cand_idx(w));
    sel_words[(long long)m * k + j] = w;
    if (out_words) out_words[(long long)m * k + j] = cand_word(uint32_t(w >> 32), cand_idx(w) + idx_base);
  }
}

// Exact bf16 logits of selected candidates: one warp per (row, candidate), the reduction order of
// topk_merge_kernel's rescoring (qo_dot_bf16).
constexpr int kRescoreWarps = 8;
__global__ void __launch_bounds__(kRescoreWarps * 32)
rescore_kernel(const int32_t* __restrict__ idx, int k, const uint16_t* __restrict__ W, const uint16_t* __restrict__ h,
               int K, uint16_t* __restrict__ out_fine) {
  pdl_trigger();
  pdl_wait();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int m = blockIdx.y, j = blockIdx.x * kRescoreWarps + warp;
  if (j >= k) return;
  const uint32_t v = uint32_t(idx[(long long)m * k + j]);
  const uint16_t* hr = h + (long long)m * K;
  const uint16_t* wr = W + (long long)v * K;
  float acc = 0.0f;
  constexpr int kB = 8;
  for (int c0 = lane; c0 < K / 8; c0 += 32 * kB) {
    uint4 w4[kB];
#pragma unroll
    for (int u = 0; u < kB; ++u)
      if (c0 + 32 * u < K / 8) w4[u] = ldg_nc_v4(wr + 8 * (c0 + 32 * u));
#pragma unroll
    for (int u = 0; u < kB; ++u) {
      if (c0 + 32 * u >= K / 8) break;
      const uint4 h4 = *reinterpret_cast<const uint4*>(hr + 8 * (c0 + 32 * u));
      const uint32_t ww[4] = {w4[u].x, w4[u].y, w4[u].z, w4[u].w}, hh[4] = {h4.x, h4.y, h4.z, h4.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        acc = __fmaf_rn(bflo(ww[e]), bflo(hh[e]), acc);
        acc = __fmaf_rn(bfhi(ww[e]), bfhi(hh[e]), acc);
      }
    }
  }
  acc = warp_sum(acc);
  if (lane == 0) out_fine[(long long)m * k + j] = f2bf(acc);
}

// Argmax of the k exact logits of each row (ties to the lower vocabulary index): one warp per row.
__global__ void fine_argmax_kernel(const int32_t* __restrict__ idx, const uint16_t* __restrict__ fine, int k,
                                   int32_t* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  const int m = blockIdx.x, lane = threadIdx.x;
  uint64_t best = 0;
  for (int j = lane; j < k; j += 32)
    best = max(best, cand_word(key16(fine[(long long)m * k + j]), uint32_t(idx[(long long)m * k + j])));
#pragma unroll
  for (int d = 16; d >= 1; d >>= 1) best = max(best, __shfl_xor_sync(0xFFFFFFFFu, best, d));
  if (lane == 0) out[m] = int32_t(cand_idx(best));
}

// Merges the candidate lists of G vocabulary shards (words [G][M][k] with global indices, fine bf16
// logits alongside): per row the k best words over all shards, in order, their fine logits, and the
// argmax of those.  The best k of the union equal the best k of the whole vocabulary, because every
// shard's list holds its own best k under the same order.
constexpr int kShardMergeThreads = 512;
__global__ void __launch_bounds__(kShardMergeThreads)
lmhead2_merge_kernel(const uint64_t* __restrict__ words, const uint16_t* __restrict__ fine, int G, int M, int k,
                     int NP, int32_t* __restrict__ out_idx, uint16_t* __restrict__ out_fine,
                     int32_t* __restrict__ out_amax) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ __align__(16) unsigned char sm_raw[];
  uint64_t* s = reinterpret_cast<uint64_t*>(sm_raw);  // [NP] words
  int* pos = reinterpret_cast<int*>(s + NP);           // [NP] source position g * k + j
  uint64_t* fk = reinterpret_cast<uint64_t*>(pos + NP + (NP & 1));  // [k] fine candidate words
  const int m = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int n = G * k;
  for (int i = tid; i < NP; i += blockDim.x) {
    if (i < n) {
      const int g = i / k, j = i - g * k;
      s[i] = words[((long long)g * M + m) * k + j];
      pos[i] = i;
    } else {
      s[i] = 0ull;
      pos[i] = -1;
    }
  }
  __syncthreads();
  for (int size = 2; size <= NP; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = tid; i < NP / 2; i += blockDim.x) {
        const int lo = 2 * i - (i & (stride - 1)), hi = lo + stride;
        const bool desc = (lo & size) == 0;
        const uint64_t a = s[lo], b = s[hi];
        if ((a < b) == desc) {
          s[lo] = b;
          s[hi] = a;
          const int t = pos[lo];
          pos[lo] = pos[hi];
          pos[hi] = t;
        }
      }
      __syncthreads();
    }
  }
  for (int j = tid; j < k; j += blockDim.x) {
    const int p = pos[j], g = p / k, jj = p - g * k;
    const uint32_t v = cand_idx(s[j]);
    const uint16_t f = fine[((long long)g * M + m) * k + jj];
    out_idx[(long long)m * k + j] = int32_t(v);
    out_fine[(long long)m * k + j] = f;
    fk[j] = cand_word(key16(f), v);
  }
  __syncthreads();
  if (warp == 0) {
    uint64_t best = 0;
    for (int j = lane; j < k; j += 32) best = max(best, fk[j]);
#pragma unroll
    for (int d = 16; d >= 1; d >>= 1) best = max(best, __shfl_xor_sync(0xFFFFFFFFu, best, d));
    if (lane == 0 && out_amax) out_amax[m] = int32_t(cand_idx(best));
  }
}

static int topk_blocks(int V, int k) {
  // enough blocks to spread the selection, each slice >= k entries and <= 12288 keys (smem)
  int G = 32;
  while (G > 1 && V / G < k) G >>= 1;
  while ((V + G - 1) / G > 12288) G <<= 1;
  return G;
}
static int pow2_at_least(int n) {
  int p = 1;
  while (p < n) p <<= 1;
  return p;
}

}  // namespace qmtp

using namespace qmtp;

extern "C" size_t qmtp_topk_workspace(int M, int V, int k) {
  if (M < 1 || V < 1 || k < 1) return 0;
  const size_t cand = size_t(M) * topk_blocks(V, k) * k * sizeof(uint64_t);
  return k > 256 ? cand + size_t(M) * k * sizeof(uint64_t) : cand;  // k > 256: + the selected words
}

static int topk_rescore(const void* vals, int ld, int M, int V, int k, const void* w_fine, const void* h, int K,
                        int* out_idx, void* out_fine, int* out_argmax, void* workspace, size_t ws_bytes,
                        uint32_t idx_base, void* out_words, void* stream);

extern "C" int qmtp_topk_rescore(const void* vals, int ld, int M, int V, int k, const void* w_fine, const void* h,
                                 int K, int* out_idx, void* out_fine, int* out_argmax, void* workspace,
                                 size_t ws_bytes, void* stream) {
  return topk_rescore(vals, ld, M, V, k, w_fine, h, K, out_idx, out_fine, out_argmax, workspace, ws_bytes, 0u,
                      nullptr, stream);
}

static int topk_rescore(const void* vals, int ld, int M, int V, int k, const void* w_fine, const void* h, int K,
                        int* out_idx, void* out_fine, int* out_argmax, void* workspace, size_t ws_bytes,
                        uint32_t idx_base, void* out_words, void* stream) {
  if (!vals || !out_idx || !workspace) return QMTP_ERR_ARG;
  if (M < 1 || V < 1 || k < 1 || k > kSelectMaxK || k > V || ld < V) return QMTP_ERR_SHAPE;
  if (w_fine && (!h || !out_fine || K < 256 || K % 256 != 0)) return QMTP_ERR_SHAPE;
  if (w_fine && (!aligned16(w_fine) || !aligned16(h))) return QMTP_ERR_ALIGN;
  const int G = topk_blocks(V, k);
  if (ws_bytes < qmtp_topk_workspace(M, V, k) || !aligned16(workspace)) return QMTP_ERR_ARG;
  const int NP = pow2_at_least(G * k);
  if (k <= 256 && NP > 8192) return QMTP_ERR_UNSUPPORTED;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int slice = (V + G - 1) / G;
  const size_t smemA = (256 + 4 + 32) * sizeof(int) + size_t(slice) * sizeof(uint16_t);
  uint64_t* cand = static_cast<uint64_t*>(workspace);
  launch_kernel(topk_partial_kernel, dim3(dim3(G, M)), dim3(kTopkThreads), smemA, st, static_cast<const uint16_t*>(vals), ld, V, k, cand);
  if (k > 256) {
    // large k: radix select, then the rescoring spread over the SMs, then the argmax
    uint64_t* sel = cand + size_t(M) * G * k;
    launch_kernel(topk_select_kernel, dim3(M), dim3(kSelectThreads), 0, st, static_cast<const uint64_t*>(cand), G * k, k,
                  out_idx, sel, idx_base, static_cast<uint64_t*>(out_words));
    if (w_fine) {
      launch_kernel(rescore_kernel, dim3((k + kRescoreWarps - 1) / kRescoreWarps, M), dim3(kRescoreWarps * 32), 0, st,
                    static_cast<const int32_t*>(out_idx), k, static_cast<const uint16_t*>(w_fine),
                    static_cast<const uint16_t*>(h), K, static_cast<uint16_t*>(out_fine));
      if (out_argmax)
        launch_kernel(fine_argmax_kernel, dim3(M), dim3(32), 0, st, static_cast<const int32_t*>(out_idx),
                      static_cast<const uint16_t*>(out_fine), k, out_argmax);
    }
    return cudaGetLastError() == cudaSuccess ? QMTP_OK : QMTP_ERR_CUDA;
  }
  const size_t smemB = size_t(NP + k) * sizeof(uint64_t);
  static const cudaError_t attr =
      cudaFuncSetAttribute(topk_merge_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 80 * 1024);
  if (attr != cudaSuccess) return QMTP_ERR_CUDA;
  launch_kernel(topk_merge_kernel, dim3(M), dim3(kMergeThreads), smemB, st, cand, G, k, NP, static_cast<const uint16_t*>(w_fine),
                                                      static_cast<const uint16_t*>(h), K, out_idx,
                                                      static_cast<uint16_t*>(out_fine), out_argmax, idx_base,
                                                      static_cast<uint64_t*>(out_words));
  return cudaGetLastError() == cudaSuccess ? QMTP_OK : QMTP_ERR_CUDA;
}

extern "C" size_t qmtp_argmax_workspace(int M, int V) {
  if (M < 1 || V < 1) return 0;
  return size_t(M) * std::min(256, std::max(1, V / 1024)) * sizeof(uint64_t);
}

extern "C" int qmtp_argmax_bf16_ids(const void* vals, int ld, int M, int V, const int* ids, int* out, int* out_local,
                                    void* workspace, size_t ws_bytes, void* stream) {
  if (!vals || !out || !workspace) return QMTP_ERR_ARG;
  if (M < 1 || V < 1 || ld < V) return QMTP_ERR_SHAPE;
  if (ws_bytes < qmtp_argmax_workspace(M, V)) return QMTP_ERR_ARG;
  const int G = std::min(256, std::max(1, V / 1024));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint64_t* part = static_cast<uint64_t*>(workspace);
  launch_kernel(argmax_partial_kernel, dim3(dim3(G, M)), dim3(256), 0, st, static_cast<const uint16_t*>(vals), ld, V, part);
  launch_kernel(argmax_final_kernel, dim3(M), dim3(32), 0, st, static_cast<const uint64_t*>(part), G,
                static_cast<const int32_t*>(ids), out, out_local);
  return cudaGetLastError() == cudaSuccess ? QMTP_OK : QMTP_ERR_CUDA;
}

extern "C" int qmtp_argmax_bf16(const void* vals, int ld, int M, int V, int* out, void* workspace, size_t ws_bytes,
                                void* stream) {
  return qmtp_argmax_bf16_ids(vals, ld, M, V, nullptr, out, nullptr, workspace, ws_bytes, stream);
}

extern "C" size_t qmtp_lmhead2_workspace(int M, int V, int k) {
  const size_t coarse = (size_t(M) * V * sizeof(uint16_t) + 255) / 256 * 256;
  return coarse + qmtp_topk_workspace(M, V, k);
}

extern "C" int qmtp_lmhead2(const void* h, const void* wq, const void* scales, const void* biases, const void* w_fine,
                            int M, int V, int K, int k, int* out_idx, void* out_fine, int* out_argmax,
                            void* coarse_out, void* workspace, size_t ws_bytes, void* stream) {
  if (!h || !wq || !scales || !biases || !w_fine || !out_idx || !out_fine || !workspace) return QMTP_ERR_ARG;
  if (ws_bytes < qmtp_lmhead2_workspace(M, V, k)) return QMTP_ERR_ARG;
  unsigned char* ws = static_cast<unsigned char*>(workspace);
  const size_t coarse_bytes = (size_t(M) * V * sizeof(uint16_t) + 255) / 256 * 256;
  void* coarse = coarse_out ? coarse_out : ws;
  int rc = qmtp_qmv_affine_g64(h, wq, scales, biases, coarse, M, V, K, V, stream);
  if (rc != QMTP_OK) return rc;
  return qmtp_topk_rescore(coarse, V, M, V, k, w_fine, h, K, out_idx, out_fine, out_argmax, ws + coarse_bytes,
                           ws_bytes - coarse_bytes, stream);
}

// The reference's own head format (lm_head2.py:19: nn.QuantizedLinear.from_linear(lin, group_size=16,
// bits=4, mode="nvfp4")): the coarse logits from the NVFP4 g16 GEMV, the same selection and rescoring.
extern "C" int qmtp_lmhead2_nvfp4(const void* h, const void* wq, const void* scales, const void* w_fine, int M, int V,
                                  int K, int k, int* out_idx, void* out_fine, int* out_argmax, void* coarse_out,
                                  void* workspace, size_t ws_bytes, void* stream) {
  if (!h || !wq || !scales || !w_fine || !out_idx || !out_fine || !workspace) return QMTP_ERR_ARG;
  if (ws_bytes < qmtp_lmhead2_workspace(M, V, k)) return QMTP_ERR_ARG;
  unsigned char* ws = static_cast<unsigned char*>(workspace);
  const size_t coarse_bytes = (size_t(M) * V * sizeof(uint16_t) + 255) / 256 * 256;
  void* coarse = coarse_out ? coarse_out : ws;
  int rc = qmtp_qmv_nvfp4_g16(h, wq, scales, coarse, M, V, K, V, stream);
  if (rc != QMTP_OK) return rc;
  return qmtp_topk_rescore(coarse, V, M, V, k, w_fine, h, K, out_idx, out_fine, out_argmax, ws + coarse_bytes,
                           ws_bytes - coarse_bytes, stream);
}

// ----------------------------------------------------------------------------- vocabulary shards
extern "C" size_t qmtp_lmhead2_shard_workspace(int M, int Vs, int k) {
  const size_t head = qmtp_lmhead2_workspace(M, Vs, k);
  if (head == 0) return 0;
  return head + (size_t(M) * k * sizeof(int32_t) + 255) / 256 * 256;
}

extern "C" int qmtp_lmhead2_shard(const void* h, const void* wq, const void* scales, const void* biases,
                                  const void* w_fine, int M, int Vs, int K, int k, long long v0, void* out_words,
                                  void* out_fine, void* workspace, size_t ws_bytes, void* stream) {
  if (!h || !wq || !scales || !biases || !w_fine || !out_words || !out_fine || !workspace) return QMTP_ERR_ARG;
  if (M < 1 || Vs < 1 || k < 1 || k > Vs || v0 < 0 || v0 + Vs > 0x7FFFFFFFLL) return QMTP_ERR_SHAPE;
  const size_t need = qmtp_lmhead2_shard_workspace(M, Vs, k);
  if (need == 0 || ws_bytes < need) return QMTP_ERR_ARG;
  if (!aligned16(out_words) || !aligned16(workspace)) return QMTP_ERR_ALIGN;
  unsigned char* ws = static_cast<unsigned char*>(workspace);
  const size_t coarse_bytes = (size_t(M) * Vs * sizeof(uint16_t) + 255) / 256 * 256;
  const size_t topk_bytes = qmtp_topk_workspace(M, Vs, k);
  int* idx_local = reinterpret_cast<int*>(ws + coarse_bytes + (topk_bytes + 255) / 256 * 256);
  if (coarse_bytes + (topk_bytes + 255) / 256 * 256 + size_t(M) * k * sizeof(int32_t) > ws_bytes) return QMTP_ERR_ARG;
  int rc = qmtp_qmv_affine_g64(h, wq, scales, biases, ws, M, Vs, K, Vs, stream);
  if (rc != QMTP_OK) return rc;
  return topk_rescore(ws, Vs, M, Vs, k, w_fine, h, K, idx_local, out_fine, nullptr, ws + coarse_bytes, topk_bytes,
                      uint32_t(v0), out_words, stream);
}

extern "C" int qmtp_lmhead2_merge(const void* words, const void* fine, int G, int M, int k, int* out_idx,
                                  void* out_fine, int* out_argmax, void* stream) {
  if (!words || !fine || !out_idx || !out_fine) return QMTP_ERR_ARG;
  if (G < 1 || M < 1 || k < 1 || size_t(G) * k > 4096) return QMTP_ERR_SHAPE;
  const int NP = pow2_at_least(G * k);
  const size_t smem = size_t(NP) * (sizeof(uint64_t) + sizeof(int)) + (NP & 1) * sizeof(int) + size_t(k) * sizeof(uint64_t);
  static const cudaError_t attr =
      cudaFuncSetAttribute(lmhead2_merge_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 100 * 1024);
  if (attr != cudaSuccess) return QMTP_ERR_CUDA;
  launch_kernel(lmhead2_merge_kernel, dim3(M), dim3(kShardMergeThreads), smem, static_cast<cudaStream_t>(stream),
                static_cast<const uint64_t*>(words), static_cast<const uint16_t*>(fine), G, M, k, NP, out_idx,
                static_cast<uint16_t*>(out_fine), out_argmax);
  return cudaGetLastError() == cudaSuccess ? QMTP_OK : QMTP_ERR_CUDA;
}

// ----------------------------------------------------------------------------- no-allocation head
// Some callers cannot allocate device memory at all: a plugin whose host framework owns every byte
// of the GPU through its own pool (a cudaMalloc would go around that pool and its budget), a call
// site that may sit inside a stream capture (cudaMalloc is not allowed while a stream is being
// captured), or a serving loop that must not pay the device-wide synchronisation a cudaMalloc can
// cause.  qmtp_lmhead2_noalloc serves them with a scratch area that is part of the library image:
// the static array below, which every GPU that loads the library holds until the process exits.
namespace qmtp {
constexpr int kNoAllocMaxRows = 4;
constexpr int kNoAllocMaxVocab = 262144;
constexpr int kNoAllocMaxK = 64;
constexpr size_t kNoAllocBytes = size_t(kNoAllocMaxRows) * kNoAllocMaxVocab * sizeof(uint16_t)  // coarse logits
                                 + size_t(kNoAllocMaxRows) * 32 * kNoAllocMaxK * sizeof(uint64_t);  // candidates
static __device__ __align__(256) unsigned char g_lmhead2_scratch[kNoAllocBytes];

// Device address of the scratch in the current context.  The name g_lmhead2_scratch in host code
// is only a host-side stand-in, never a device address, so the address is looked up with the device
// current (cudaGetSymbolAddress) and cached per CUDA context: a context created after a
// cudaDeviceReset gets a fresh lookup, and a failed lookup is retried by the next call.
static int noalloc_scratch(void** out) { return symbol_address(g_lmhead2_scratch, out); }
}  // namespace qmtp

extern "C" int qmtp_lmhead2_noalloc(const void* h, const void* wq, const void* scales, const void* biases,
                                    const void* w_fine, int M, int V, int K, int k, int* out_idx, void* out_fine,
                                    int* out_argmax, void* stream) {
  if (M < 1 || M > kNoAllocMaxRows || V < 1 || V > kNoAllocMaxVocab || k < 1 || k > kNoAllocMaxK)
    return QMTP_ERR_SHAPE;
  const size_t need = qmtp_lmhead2_workspace(M, V, k);
  if (need == 0 || need > kNoAllocBytes) return QMTP_ERR_SHAPE;
  void* scratch = nullptr;
  const int rc = noalloc_scratch(&scratch);
  if (rc != QMTP_OK) return rc;
  // Nothing in the scratch has to start at zero: the coarse logits of all M rows and every
  // candidate slot are written before they are read, within the call.
  return qmtp_lmhead2(h, wq, scales, biases, w_fine, M, V, K, k, out_idx, out_fine, out_argmax, nullptr, scratch,
                      kNoAllocBytes, stream);
}
