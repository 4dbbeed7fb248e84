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

// Top-k by radix selection, for n <= kThreads * kPer and kout <= kThreads:
// every element gets the unique 64-bit key (order-preserving score bits,
// ~index), so the k largest keys are exactly the k largest scores with ties
// to the lower index.  Eight passes of an 8-bit histogram (shared memory)
// narrow the key prefix to the k-th largest key; the elements at or above it
// are compacted and sorted descending by a bitonic network.  Same results as
// block_topk.  s_hist: 256 unsigned; s_keys: kThreads unsigned long long.
template <int kThreads, int kPer>
__device__ void block_topk_radix(const float* scores, int n, int kout, int32_t* out, unsigned* s_hist,
                                 unsigned long long* s_keys, unsigned* s_misc) {
  const int tid = threadIdx.x;
  unsigned long long keys[kPer];
#pragma unroll
  for (int e = 0; e < kPer; ++e) {
    const int i = tid * kPer + e;  // consecutive elements per thread: coalesced enough from L2
    keys[e] = i < n ? make_key(__ldcg(scores + i), i) : 0ull;
  }
  const int kvalid = min(kout, n);
  unsigned long long prefix = 0ull, mask = 0ull;
  int need = kvalid;  // how many keys >= the threshold remain to be found in the current bin
  for (int pass = 0; pass < 8 && kvalid > 0; ++pass) {
    const int shift = 56 - 8 * pass;
    for (int b = tid; b < 256; b += kThreads) s_hist[b] = 0u;
    __syncthreads();
#pragma unroll
    for (int e = 0; e < kPer; ++e)
      if (tid * kPer + e < n && (keys[e] & mask) == prefix) atomicAdd(&s_hist[(keys[e] >> shift) & 0xFF], 1u);
    __syncthreads();
    if (tid < 32) {
      // Bin holding the need-th largest key among the prefix matches, from the top.
      unsigned cnt[8];
      unsigned tot = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        cnt[j] = s_hist[255 - (8 * tid + j)];
        tot += cnt[j];
      }
      unsigned incl = tot;  // inclusive prefix over lanes (bins from the top)
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const unsigned v = __shfl_up_sync(0xffffffffu, incl, o);
        if (tid >= o) incl += v;
      }
      unsigned run = incl - tot;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (run < unsigned(need) && run + cnt[j] >= unsigned(need)) {
          s_misc[0] = unsigned(255 - (8 * tid + j));
          s_misc[1] = unsigned(need) - run;  // still needed inside this bin
        }
        run += cnt[j];
      }
    }
    __syncthreads();
    prefix |= static_cast<unsigned long long>(s_misc[0]) << shift;
    mask |= 0xFFull << shift;
    need = int(s_misc[1]);
    __syncthreads();
  }
  // prefix is now the kvalid-th largest key: compact every key >= it.
  if (tid == 0) s_misc[2] = 0u;
  __syncthreads();
#pragma unroll
  for (int e = 0; e < kPer; ++e)
    if (kvalid > 0 && tid * kPer + e < n && keys[e] >= prefix) s_keys[atomicAdd(&s_misc[2], 1u)] = keys[e];
  __syncthreads();
  int m = 1;
  while (m < kvalid) m <<= 1;
  for (int i = kvalid + tid; i < m; i += kThreads) s_keys[i] = 0ull;
  __syncthreads();
  // Bitonic sort of s_keys[0, m), descending.
  for (int size = 2; size <= m; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = tid; i < m; i += kThreads) {
        const int j = i ^ stride;
        if (j > i) {
          const bool desc = (i & size) == 0;
          const unsigned long long a = s_keys[i], b = s_keys[j];
          if (desc ? a < b : a > b) {
            s_keys[i] = b;
            s_keys[j] = a;
          }
        }
      }
      __syncthreads();
    }
  }
  for (int r = tid; r < kout; r += kThreads)
    out[r] = r < kvalid ? static_cast<int32_t>(~static_cast<unsigned>(s_keys[r] & 0xffffffffull)) : -1;
}

}  // namespace topk
}  // namespace csahca
