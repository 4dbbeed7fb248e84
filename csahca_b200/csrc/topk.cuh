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
//      candidates, and the remaining digits (8, 8 and 4 score bits, then
//      8-bit digits of the index, reached only by equal scores) are resolved
//      over the candidates alone.  A bin with more than kRadixCand members is
//      resolved by passes over all keys instead.
//   4. Each taken key is written at its rank among the taken keys.
// Same results as block_topk.  The passes over all keys are instruction-bound
// (two CTAs per SM, 16384 keys each), so they read shared memory four keys at
// a time and reject whole groups below the chosen bin with one comparison.
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
  const int seg = (nb + kWarps - 1) / kWarps;
  const int top = nb - 1 - warp * seg;  // this warp's bins: top, top-1, ..., down to 0 at most
  const int cnt = top < 0 ? 0 : min(seg, top + 1);
  unsigned t = 0;
  for (int r = lane; r < cnt; r += 32) t += sm.hist[top - r];
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
    for (int r0 = 0; r0 < cnt; r0 += 32) {
      const int r = r0 + lane;
      const unsigned c = r < cnt ? sm.hist[top - r] : 0u;
      unsigned incl = c;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const unsigned v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
      }
      const unsigned before = run + incl - c;
      if (r < cnt && before < need && before + c >= need) {
        sm.misc[0] = unsigned(top - r);
        sm.misc[1] = need - before;
        sm.misc[2] = before + c == need ? 1u : 0u;
      }
      run += __shfl_sync(0xffffffffu, incl, 31);
    }
  }
  __syncthreads();
}

// Slot for this lane's item in a shared list whose length is *count, one
// atomic per warp (all 32 lanes call it).
__device__ __forceinline__ unsigned radix_append(bool want, unsigned* count) {
  const unsigned mask = __ballot_sync(0xffffffffu, want);
  if (mask == 0u) return 0u;
  const int lane = threadIdx.x & 31, leader = __ffs(mask) - 1;
  unsigned base = 0;
  if (lane == leader) base = atomicAdd(count, unsigned(__popc(mask)));
  base = __shfl_sync(0xffffffffu, base, leader);
  return base + unsigned(__popc(mask & ((1u << lane) - 1u)));
}

__device__ __forceinline__ unsigned long long radix_key(uint32_t score_bits, int i) {
  return (static_cast<unsigned long long>(score_bits) << 32) | ~static_cast<uint32_t>(i);
}

// s_sk: n words of shared memory, 16-byte aligned.
template <int kThreads>
__device__ void block_topk_radix(const float* scores, int n, int kout, int32_t* out, uint32_t* s_sk,
                                 RadixSmem<kThreads>& sm) {
  static_assert(kThreads % 32 == 0 && kThreads / 32 <= 32, "one warp scans the warp totals");
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
  const int n4 = n >> 2;
  if ((reinterpret_cast<uintptr_t>(scores) & 15) == 0) {
    const float4* s4 = reinterpret_cast<const float4*>(scores);
    uint4* d4 = reinterpret_cast<uint4*>(s_sk);
    for (int base = 0; base < n4; base += 4 * kThreads) {
      float4 v[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int j = base + e * kThreads + tid;
        if (j < n4) v[e] = __ldcg(s4 + j);
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int j = base + e * kThreads + tid;
        if (j < n4) {
          const uint4 k = make_uint4(float_order_key(v[e].x), float_order_key(v[e].y), float_order_key(v[e].z),
                                     float_order_key(v[e].w));
          d4[j] = k;
          atomicAdd(&sm.hist[k.x >> 20], 1u);
          atomicAdd(&sm.hist[k.y >> 20], 1u);
          atomicAdd(&sm.hist[k.z >> 20], 1u);
          atomicAdd(&sm.hist[k.w >> 20], 1u);
        }
      }
    }
    for (int i = 4 * n4 + tid; i < n; i += kThreads) {
      const uint32_t k = float_order_key(__ldcg(scores + i));
      s_sk[i] = k;
      atomicAdd(&sm.hist[k >> 20], 1u);
    }
  } else {
    for (int i = tid; i < n; i += kThreads) {
      const uint32_t k = float_order_key(__ldcg(scores + i));
      s_sk[i] = k;
      atomicAdd(&sm.hist[k >> 20], 1u);
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
    // Atomic-free (appends to one shared counter serialise): each thread
    // marks its hits in two 32-bit masks over eight groups of four keys, a
    // block scan of the counts gives every thread its output offsets.
    constexpr int kWarps = kThreads / 32;
    const int lane = tid & 31, warp = tid >> 5;
    const uint4* k4 = reinterpret_cast<const uint4*>(s_sk);
    const uint32_t lo_edge = bin0 << 20;  // smallest key of the bin
    const int nv = (n + 3) >> 2;
    unsigned taken = 0, kept = 0;  // running list lengths, uniform
    for (int jb = 0; jb < nv; jb += 8 * kThreads) {
      uint32_t take_m = 0u, keep_m = 0u;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int j = jb + e * kThreads + tid;
        if (j >= nv) break;
        const uint4 q = k4[j];  // words past n are masked below
        if (max(max(q.x, q.y), max(q.z, q.w)) < lo_edge) continue;
        const uint32_t kk[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const uint32_t b = kk[c] >> 20;
          const bool ok = 4 * j + c < n;
          take_m |= (ok && b > bin0) ? 1u << (4 * e + c) : 0u;
          keep_m |= (ok && b == bin0) ? 1u << (4 * e + c) : 0u;
        }
      }
      // Counts packed as take << 16 | keep (each at most 16384 per round).
      const unsigned mine = (unsigned(__popc(take_m)) << 16) | unsigned(__popc(keep_m));
      unsigned incl = mine;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const unsigned v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
      }
      if (lane == 31) sm.wsum[warp] = incl;
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
        if (lane < kWarps) sm.wsum[lane] = wi - w;
        if (lane == 31) sm.misc[5] = wi;  // this round's totals
      }
      __syncthreads();
      const unsigned off = sm.wsum[warp] + incl - mine;
      unsigned at = taken + (off >> 16), ac = kept + (off & 0xFFFFu);
      while (take_m) {
        const int bit = __ffs(take_m) - 1;
        take_m &= take_m - 1;
        const int i = 4 * (jb + (bit >> 2) * kThreads + tid) + (bit & 3);
        sm.keys[at++] = radix_key(s_sk[i], i);
      }
      while (keep_m) {
        const int bit = __ffs(keep_m) - 1;
        keep_m &= keep_m - 1;
        sm.cand[ac++] = uint32_t(4 * (jb + (bit >> 2) * kThreads + tid) + (bit & 3));
      }
      const unsigned tot = sm.misc[5];
      taken += tot >> 16;
      kept += tot & 0xFFFFu;
      __syncthreads();  // wsum and misc[5] are rewritten by the next round
    }
    if (tid == 0) {
      sm.misc[3] = taken;
      sm.misc[4] = kept;
    }
  }
  __syncthreads();
  const int m = use_cand ? int(sm.misc[4]) : n;  // elements the remaining passes visit
  for (int pass = 1; pass < 8 && !done; ++pass) {
    const bool hi = pass < 4;
    const int bits = pass == 3 ? 4 : 8;
    const int shift = pass == 1 ? 12 : pass == 2 ? 4 : pass == 3 ? 0 : 24 - 8 * (pass - 4);  // within its half
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
    if (s_sk[i] < pre_hi) continue;
    const unsigned long long k = radix_key(s_sk[i], i);
    if (k >= prefix) sm.keys[atomicAdd(&sm.misc[3], 1u)] = k;
  }
  // 4. Rank of each taken key among the taken keys, counted by kThreads
  //    threads at once: key r = t % kvalid against one slice of the others.
  unsigned* rank = sm.hist;
  for (int r = tid; r < kvalid; r += kThreads) rank[r] = 0u;
  __syncthreads();
  {
    const int slices = max(1, kThreads / kvalid);
    const int r = tid % kvalid, sl = tid / kvalid;
    if (sl < slices) {
      const int len = (kvalid + slices - 1) / slices;
      const int j0 = sl * len, j1 = min(kvalid, j0 + len);
      for (int rr = r; rr < kvalid; rr += kThreads) {
        const unsigned long long mine = sm.keys[rr];
        unsigned above = 0;
        for (int j = j0; j < j1; ++j) above += sm.keys[j] > mine ? 1u : 0u;
        if (above) atomicAdd(&rank[rr], above);
      }
    }
  }
  __syncthreads();
  for (int r = tid; r < kvalid; r += kThreads)
    out[rank[r]] = static_cast<int32_t>(~static_cast<unsigned>(sm.keys[r] & 0xffffffffull));
  for (int r = kvalid + tid; r < kout; r += kThreads) out[r] = -1;
}

}  // namespace topk
}  // namespace csahca
