// Top-k selection shared by the CSA scorers: largest scores first, equal
// scores by lower index, -1 past the valid count.  A 64-bit key
// (order-preserving bits of the score, ~index) makes every key distinct, so
// round r takes the largest key below round r-1's pick and nothing needs to be
// marked as taken.
#pragma once

#include <stdint.h>

#include "common.cuh"

namespace csahca {
namespace topk {

constexpr int kTopkRegs = 16;  // register path holds up to threads * kTopkRegs scores

__device__ __forceinline__ unsigned long long make_key(float score, int idx) {
  return (static_cast<unsigned long long>(float_order_key(score)) << 32) | static_cast<unsigned>(~idx);
}

// Top-k of scores[0, n) written to out[0, kout): largest first, equal scores by
// lower index, slots past min(kout, n) get -1.  Called by all threads of a CTA.
// Round r picks the largest composite key below round r-1's pick, so no element
// needs to be marked as taken.
template <int kThreads>
__device__ void block_topk(float* scores, int n, int kout, int32_t* out, unsigned long long* s_red) {
  constexpr int kWarps = kThreads / 32;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const bool in_regs = n <= kThreads * kTopkRegs;
  unsigned long long keys[kTopkRegs];
  if (in_regs) {
#pragma unroll
    for (int e = 0; e < kTopkRegs; ++e) {
      const int i = tid + e * kThreads;
      keys[e] = i < n ? make_key(__ldcg(scores + i), i) : 0ull;
    }
  }
  const int kvalid = min(kout, n);
  unsigned long long prev = ~0ull;
  for (int r = 0; r < kvalid; ++r) {
    unsigned long long best = 0ull;
    if (in_regs) {
#pragma unroll
      for (int e = 0; e < kTopkRegs; ++e)
        if (keys[e] < prev && keys[e] > best) best = keys[e];
    } else {
      for (int i = tid; i < n; i += kThreads) {
        const unsigned long long kk = make_key(__ldcg(scores + i), i);
        if (kk < prev && kk > best) best = kk;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
      best = other > best ? other : best;
    }
    if (lane == 0) s_red[warp] = best;
    __syncthreads();
    best = s_red[0];
#pragma unroll
    for (int w = 1; w < kWarps; ++w) best = s_red[w] > best ? s_red[w] : best;
    __syncthreads();
    if (tid == 0) out[r] = static_cast<int32_t>(~static_cast<unsigned>(best & 0xffffffffull));
    prev = best;
  }
  for (int r = kvalid + tid; r < kout; r += kThreads) out[r] = -1;
  __syncthreads();  // leave the workspace zero: a later call may put its counters here
  for (int i = tid; i < n; i += kThreads) scores[i] = 0.f;
}


}  // namespace topk
}  // namespace csahca

namespace csahca {
namespace topk {

// Top-k by radix selection, for kout <= kThreads.  Every element has the
// unique 64-bit key (order-preserving score bits, ~index), so the k largest
// keys are exactly the k largest scores with ties to the lower index.  The
// score halves are staged once in shared memory; the index half follows from
// the position.
//
//   1. Staging and the histogram of the top 12 score bits in one pass.
//   2. The bin holding the k-th largest key; if it is wanted whole, every key
//      of the bins at or above it is taken and the search ends.
//   3. Otherwise one pass splits the keys: those above the bin are taken,
//      those in it (a few hundred for real score distributions) become
//      candidates, and the remaining digits (12, 8 score bits, then 8-bit
//      digits of the index, reached only by equal scores) are resolved over
//      the candidates alone.  A bin with more than kRadixCand members is
//      resolved by passes over all keys instead.
//   4. Each taken key is written at its rank among the taken keys.
// Same results as block_topk.
constexpr int kRadixBins = 4096;
constexpr int kRadixCand = 2048;

template <int kThreads>
struct RadixSmem {
  unsigned hist[kRadixBins];
  unsigned wsum[32];
  unsigned misc[8];  // bin, need, whole, taken count, candidate count
  unsigned long long keys[kThreads];
  uint32_t cand[kRadixCand];
};

// The bin (of nb, from the top) that holds the need-th largest counted key.
// Each warp scans a contiguous run of bins, lanes on consecutive words.
// Writes misc[0] = bin, misc[1] = keys still wanted inside it, misc[2] = 1 if
// that is the whole bin.  Ends with a barrier.
template <int kThreads>
__device__ __forceinline__ void radix_find_bin(RadixSmem<kThreads>& sm, int nb, unsigned need) {
  constexpr int kWarps = kThreads / 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int seg = nb / kWarps;
  const int top = nb - 1 - warp * seg;  // this warp's bins: top, top-1, ..., top-seg+1
  unsigned t = 0;
  for (int r = lane; r < seg; r += 32) t += sm.hist[top - r];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
  if (lane == 0) sm.wsum[warp] = t;
  __syncthreads();
  if (warp == 0) {
    const unsigned w = lane < kWarps ? sm.wsum[lane] : 0u;
    unsigned wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const unsigned v = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += v;
    }
    __syncwarp();
    if (lane < kWarps) sm.wsum[lane] = wi - w;  // keys in the bins above each warp's run
  }
  __syncthreads();
  unsigned run = sm.wsum[warp];
  if (run < need && run + t >= need) {  // the target bin is in this warp's run
    for (int r0 = 0; r0 < seg; r0 += 32) {
      const int r = r0 + lane;
      const unsigned c = r < seg ? sm.hist[top - r] : 0u;
      unsigned incl = c;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const unsigned v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
      }
      const unsigned before = run + incl - c;
      if (r < seg && before < need && before + c >= need) {
        sm.misc[0] = unsigned(top - r);
        sm.misc[1] = need - before;
        sm.misc[2] = before + c == need ? 1u : 0u;
      }
      run += __shfl_sync(0xffffffffu, incl, 31);
    }
  }
  __syncthreads();
}

template <int kThreads>
__device__ void block_topk_radix(const float* scores, int n, int kout, int32_t* out, uint32_t* s_sk,
                                 RadixSmem<kThreads>& sm) {
  static_assert(kThreads % 32 == 0 && kThreads / 32 <= 32 && kRadixBins % (kThreads / 32) == 0 &&
                    256 % (kThreads / 32) == 0,
                "warp-segmented bin scan");
  const int tid = threadIdx.x;
  const int kvalid = min(kout, n);
  if (kvalid <= 0) {
    for (int r = tid; r < kout; r += kThreads) out[r] = -1;
    return;
  }
  // 1. Stage the order keys and count their top 12 bits.
  for (int b = tid; b < kRadixBins; b += kThreads) sm.hist[b] = 0u;
  if (tid == 0) sm.misc[3] = sm.misc[4] = 0u;
  __syncthreads();
  for (int base = 0; base < n; base += 8 * kThreads) {
    float v[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int i = base + e * kThreads + tid;
      v[e] = i < n ? __ldcg(scores + i) : 0.f;
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int i = base + e * kThreads + tid;
      if (i < n) {
        const uint32_t k = float_order_key(v[e]);
        s_sk[i] = k;
        atomicAdd(&sm.hist[k >> 20], 1u);
      }
    }
  }
  __syncthreads();
  // 2. The bin of the k-th largest key.
  radix_find_bin(sm, kRadixBins, unsigned(kvalid));
  const uint32_t bin0 = sm.misc[0];
  unsigned need = sm.misc[1];
  bool done = sm.misc[2] != 0u;
  const bool use_cand = !done && sm.hist[bin0] <= unsigned(kRadixCand);
  uint32_t pre_hi = bin0 << 20, msk_hi = 0xFFF00000u, pre_lo = 0u, msk_lo = 0u;
  // 3. Split: keys above the bin are taken, the bin's keys become candidates.
  if (use_cand) {
    for (int i = tid; i < n; i += kThreads) {
      const uint32_t k = s_sk[i];
      const uint32_t b = k >> 20;
      if (b > bin0)
        sm.keys[atomicAdd(&sm.misc[3], 1u)] = (static_cast<unsigned long long>(k) << 32) | ~static_cast<uint32_t>(i);
      else if (b == bin0)
        sm.cand[atomicAdd(&sm.misc[4], 1u)] = uint32_t(i);
    }
  }
  __syncthreads();
  const int m = use_cand ? int(sm.misc[4]) : n;  // elements the remaining passes visit
  for (int pass = 1; pass < 7 && !done; ++pass) {
    const bool hi = pass < 3;
    const int bits = pass == 1 ? 12 : 8;
    const int shift = pass == 1 ? 8 : pass == 2 ? 0 : 24 - 8 * (pass - 3);  // within its half
    const int nb = 1 << bits;
    for (int b = tid; b < nb; b += kThreads) sm.hist[b] = 0u;
    __syncthreads();
    for (int c = tid; c < m; c += kThreads) {
      const int i = use_cand ? int(sm.cand[c]) : c;
      const uint32_t k = s_sk[i], lo = ~static_cast<uint32_t>(i);
      if ((k & msk_hi) == pre_hi && (lo & msk_lo) == pre_lo)
        atomicAdd(&sm.hist[((hi ? k : lo) >> shift) & uint32_t(nb - 1)], 1u);
    }
    __syncthreads();
    radix_find_bin(sm, nb, need);
    if (hi) {
      pre_hi |= sm.misc[0] << shift;
      msk_hi |= uint32_t(nb - 1) << shift;
    } else {
      pre_lo |= sm.misc[0] << shift;
      msk_lo |= uint32_t(nb - 1) << shift;
    }
    need = sm.misc[1];
    done = sm.misc[2] != 0u;
  }
  // Every key >= the prefix (lower bits zero when the search ended early) is
  // taken: kvalid keys with those already taken in step 3.
  const unsigned long long prefix = (static_cast<unsigned long long>(pre_hi) << 32) | pre_lo;
  for (int c = tid; c < m; c += kThreads) {
    const int i = use_cand ? int(sm.cand[c]) : c;
    const unsigned long long k = (static_cast<unsigned long long>(s_sk[i]) << 32) | ~static_cast<uint32_t>(i);
    if (k >= prefix) sm.keys[atomicAdd(&sm.misc[3], 1u)] = k;
  }
  __syncthreads();
  // 4. Each taken key's output position is the number of taken keys above it.
  if (tid < kvalid) {
    const unsigned long long mine = sm.keys[tid];
    int rank = 0;
#pragma unroll 4
    for (int j = 0; j < kvalid; ++j) rank += sm.keys[j] > mine ? 1 : 0;
    out[rank] = static_cast<int32_t>(~static_cast<unsigned>(mine & 0xffffffffull));
  }
  for (int r = kvalid + tid; r < kout; r += kThreads) out[r] = -1;
}

}  // namespace topk
}  // namespace csahca
