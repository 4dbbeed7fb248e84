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
