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
// score halves are staged once in shared memory (s_sk, n words); the index
// half follows from the position.  Histogram passes over digits of 12, 12 and
// 8 bits (then 8-bit digits of the index, reached only by equal scores) narrow
// the key prefix; a pass whose chosen bin is wanted whole ends the search
// early, since every key in it is then taken.  The keys at or above the final
// prefix are compacted and each is written at its rank among them.  Same
// results as block_topk.
// Shared memory: s_sk n words, s_hist 4096 unsigned, s_wsum kThreads/32
// unsigned, s_keys kThreads unsigned long long, s_misc 4 unsigned.
template <int kThreads>
__device__ void block_topk_radix(const float* scores, int n, int kout, int32_t* out, uint32_t* s_sk,
                                 unsigned* s_hist, unsigned* s_wsum, unsigned long long* s_keys, unsigned* s_misc) {
  constexpr int kWarps = kThreads / 32;
  static_assert(kWarps <= 32 && kThreads % 32 == 0, "one warp scans the warp totals");
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int i = tid; i < n; i += kThreads) s_sk[i] = float_order_key(__ldcg(scores + i));
  const int kvalid = min(kout, n);
  // The key prefix found so far, as its score half and its ~index half.
  uint32_t pre_hi = 0u, msk_hi = 0u, pre_lo = 0u, msk_lo = 0u;
  int need = kvalid;  // keys still wanted from the keys that match the prefix
  bool done = kvalid <= 0;
  for (int pass = 0; pass < 7 && !done; ++pass) {
    const bool hi = pass < 3;
    const int bits = pass < 2 ? 12 : 8;
    const int shift = pass == 0 ? 20 : pass == 1 ? 8 : pass == 2 ? 0 : 24 - 8 * (pass - 3);  // within its half
    const int nb = 1 << bits;
    const int per = nb >= kThreads ? nb / kThreads : 1;
    for (int b = tid; b < nb; b += kThreads) s_hist[b] = 0u;
    __syncthreads();  // also orders the staging of s_sk before the first pass
    if (hi) {
      for (int i = tid; i < n; i += kThreads) {
        const uint32_t k = s_sk[i];
        if ((k & msk_hi) == pre_hi) atomicAdd(&s_hist[(k >> shift) & uint32_t(nb - 1)], 1u);
      }
    } else {  // the whole score half is fixed: only equal scores remain
      for (int i = tid; i < n; i += kThreads) {
        const uint32_t lo = ~static_cast<uint32_t>(i);
        if (s_sk[i] == pre_hi && (lo & msk_lo) == pre_lo) atomicAdd(&s_hist[(lo >> shift) & 0xFFu], 1u);
      }
    }
    __syncthreads();
    // Bins from the top: thread t owns bins nb-1-(t*per) down to nb-(t+1)*per.
    unsigned tot = 0;
    const bool owns = tid * per < nb;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (j < per && owns) tot += s_hist[nb - 1 - (tid * per + j)];
    unsigned incl = tot;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const unsigned v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    if (lane == 31) s_wsum[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      const unsigned w = lane < kWarps ? s_wsum[lane] : 0u;
      unsigned wi = w;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const unsigned v = __shfl_up_sync(0xffffffffu, wi, o);
        if (lane >= o) wi += v;
      }
      __syncwarp();
      if (lane < kWarps) s_wsum[lane] = wi - w;  // exclusive prefix of the warp totals
    }
    __syncthreads();
    unsigned run = s_wsum[warp] + incl - tot;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (!(j < per && owns)) continue;
      const unsigned c = s_hist[nb - 1 - (tid * per + j)];
      if (run < unsigned(need) && run + c >= unsigned(need)) {
        s_misc[0] = unsigned(nb - 1 - (tid * per + j));
        s_misc[1] = unsigned(need) - run;
        s_misc[3] = (run + c == unsigned(need)) ? 1u : 0u;
      }
      run += c;
    }
    __syncthreads();
    if (hi) {
      pre_hi |= s_misc[0] << shift;
      msk_hi |= uint32_t(nb - 1) << shift;
    } else {
      pre_lo |= s_misc[0] << shift;
      msk_lo |= uint32_t(nb - 1) << shift;
    }
    need = int(s_misc[1]);
    done = s_misc[3] != 0u;
  }
  // Exactly kvalid keys are >= the prefix (lower bits zero when the search ended early).
  const unsigned long long prefix = (static_cast<unsigned long long>(pre_hi) << 32) | pre_lo;
  if (tid == 0) s_misc[2] = 0u;
  __syncthreads();
  if (kvalid > 0) {
    for (int i = tid; i < n; i += kThreads) {
      const unsigned long long k = (static_cast<unsigned long long>(s_sk[i]) << 32) | ~static_cast<uint32_t>(i);
      if (k >= prefix) s_keys[atomicAdd(&s_misc[2], 1u)] = k;
    }
  }
  __syncthreads();
  // Each selected key's output position is the number of selected keys above
  // it (all keys are distinct): one pass over s_keys, read as broadcasts.
  if (tid < kvalid) {
    const unsigned long long mine = s_keys[tid];
    int rank = 0;
    for (int j = 0; j < kvalid; ++j) rank += s_keys[j] > mine ? 1 : 0;
    out[rank] = static_cast<int32_t>(~static_cast<unsigned>(mine & 0xffffffffull));
  }
  for (int r = kvalid + tid; r < kout; r += kThreads) out[r] = -1;
}

}  // namespace topk
}  // namespace csahca
