// CSA chunk scorer + per-(batch, head) top-k (sm_100a).
//
// Restates hybrid_attention/reference.py:40-56 (chunk_mean + select_topk_chunks)
// as one streaming pass over K: every valid K row is read once, each chunk is
// reduced to its fp32 mean, dotted with q and scaled; whoever scores the last
// chunk of a (batch, head) row then selects that row's top-k (ties: lower index).
//
// Two kernels, same results:
//  * csa_select_bulk_kernel (a chunk of at most 16 KB, the usual case): one
//    persistent CTA per SM; a producer thread streams whole chunks with
//    cp.async.bulk into a 12-stage shared-memory ring (192 KB in flight per SM,
//    no register cost), twelve consumer warps (one per stage) reduce one chunk each from shared
//    memory and a warp-level top-k runs in the warp that completes a row.
//  * csa_select_kernel (larger chunks): persistent CTAs, a warp per chunk with
//    16-byte non-allocating loads, a CTA-wide top-k.
//
// Work distribution: units of up to kMaxChunksPerUnit chunks of one row are
// taken from an atomic ticket, so ragged per-request lengths cost nothing for
// the chunks past a request's end.
//
// Workspace layout (zero on entry, zero on exit):
//   [0, 256)          ticket[0] = next unit, ticket[1] = retired CTAs
//   [256, 256+4BH)    per-row arrival counters (rounded up to 256 B)
//   [.., + 4*BH*C)    fp32 chunk scores
#include <algorithm>

#include "common.cuh"
#include "sm100.cuh"
#include "topk.cuh"

namespace csahca {
namespace {

constexpr int kSelThreads = 256;
constexpr int kSelWarps = kSelThreads / 32;
// Chunks per ticket unit: as large as keeps every SM busy.  Large units mean
// long contiguous reads and few counter updates (one fence per run of a row's
// chunks); small problems shrink the unit so all SMs still get work.
constexpr int kMaxChunksPerUnit = 64;
constexpr int kMinChunksPerUnit = 4;

struct SelectParams {
  const void* q;
  const void* k;
  const int32_t* seq_lens;
  int heads, seq_len, num_chunks, chunk, kout;
  int unit;           // chunks per ticket unit
  int units_per_row;  // ceil(num_chunks / unit)
  int total_units;
  float scale;
  unsigned* ticket;
  unsigned* counters;
  float* scores;
  int32_t* out;
};

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// Score of one chunk, computed by one warp; every lane returns the same value.
template <typename T, int D>
__device__ __forceinline__ float chunk_score(const T* rows, int chunk, const float* qf, int lane, float scale) {
  using G = RowGeom<T, D>;
  constexpr int kU = G::kVPL >= 8 ? 1 : 8 / G::kVPL;  // loads in flight per lane = 8
  const int tok_lane = lane / G::kLPT;
  const int vec_lane = lane % G::kLPT;
  const char* base = reinterpret_cast<const char*>(rows);
  constexpr int kRowBytes = D * sizeof(T);
  float acc[G::kFPL];
#pragma unroll
  for (int e = 0; e < G::kFPL; ++e) acc[e] = 0.f;

  const int steps = (chunk + G::kTPS - 1) / G::kTPS;
  for (int s0 = 0; s0 < steps; s0 += kU) {
    uint4 v[kU][G::kVPL];
#pragma unroll
    for (int i = 0; i < kU; ++i) {
      const int t = (s0 + i) * G::kTPS + tok_lane;
      const bool ok = t < chunk;
#pragma unroll
      for (int j = 0; j < G::kVPL; ++j)
        v[i][j] = ok ? ldg_stream(base + size_t(t) * kRowBytes + size_t(vec_lane + 32 * j) * 16) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int i = 0; i < kU; ++i)
#pragma unroll
      for (int j = 0; j < G::kVPL; ++j) {
        float f[G::kVec];
        Elem<T>::widen(v[i][j], f);
#pragma unroll
        for (int e = 0; e < G::kVec; ++e) acc[j * G::kVec + e] += f[e];
      }
  }
  // Sum the token lanes, then mean = sum / chunk (as torch's mean does).
  float dot = 0.f;
  const float count = float(chunk);
#pragma unroll
  for (int e = 0; e < G::kFPL; ++e) {
    float s = warp_sum_xor(acc[e], G::kLPT, 32);
    dot = fmaf(qf[e], __fdiv_rn(s, count), dot);
  }
  dot = warp_sum_xor(dot, 1, G::kLPT);
  return dot * scale;
}

using topk::make_key;

__device__ __forceinline__ void block_topk(float* scores, int n, int kout, int32_t* out, unsigned long long* s_red) {
  topk::block_topk<kSelThreads>(scores, n, kout, out, s_red);
}

template <typename T, int D>
__global__ void __launch_bounds__(kSelThreads) csa_select_kernel(SelectParams p) {
  using G = RowGeom<T, D>;
  __shared__ int s_unit;
  __shared__ int s_last;
  __shared__ unsigned long long s_red[kSelWarps];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int vec_lane = lane % G::kLPT;

  for (;;) {
    if (threadIdx.x == 0) s_unit = static_cast<int>(atomicAdd(p.ticket, 1u));
    __syncthreads();
    const int u = s_unit;
    __syncthreads();
    if (u >= p.total_units) break;
    const int row = u / p.units_per_row;  // b*H + h
    const int r = u - row * p.units_per_row;
    const int b = row / p.heads;
    int row_chunks = p.num_chunks;
    if (p.seq_lens != nullptr) {
      const int len = min(max(p.seq_lens[b], 0), p.seq_len);
      row_chunks = len / p.chunk;
    }
    const int units_b = max(1, (row_chunks + p.unit - 1) / p.unit);
    if (r >= units_b) continue;  // uniform across the CTA

    const T* qrow = static_cast<const T*>(p.q) + size_t(row) * D;
    float qf[G::kFPL];
#pragma unroll
    for (int j = 0; j < G::kVPL; ++j) {
      const uint4 v = *reinterpret_cast<const uint4*>(qrow + (vec_lane + 32 * j) * G::kVec);
      Elem<T>::widen(v, qf + j * G::kVec);
    }
    const T* krow = static_cast<const T*>(p.k) + size_t(row) * p.seq_len * D;
    const int c0 = r * p.unit;
    const int c1 = min(c0 + p.unit, row_chunks);
    for (int c = c0 + warp; c < c1; c += kSelWarps) {
      const float s = chunk_score<T, D>(krow + size_t(c) * p.chunk * D, p.chunk, qf, lane, p.scale);
      if (lane == 0) p.scores[size_t(row) * p.num_chunks + c] = s;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence();
      const unsigned old = atomicAdd(p.counters + row, 1u);
      s_last = old == static_cast<unsigned>(units_b - 1);
      if (s_last) p.counters[row] = 0u;  // every unit of this row has arrived
    }
    __syncthreads();
    if (s_last) {
      __threadfence();
      block_topk(p.scores + size_t(row) * p.num_chunks, row_chunks, p.kout, p.out + size_t(row) * p.kout, s_red);
    }
  }
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned done = atomicAdd(p.ticket + 1, 1u);
    if (done == gridDim.x - 1) {  // last CTA out restores the zero workspace
      p.ticket[0] = 0u;
      p.ticket[1] = 0u;
    }
  }
}

// ---------------------------------------------------------------------------------------------------
// Bulk-copy scorer (used when one chunk fits a 16 KB stage): one persistent CTA
// per SM.  A single producer thread takes 16-chunk units from the ticket and
// streams every chunk (chunk_size x D contiguous bytes) into a 12-stage shared
// memory ring with cp.async.bulk, so ~192 KB per SM are in flight without any
// register cost.  Twelve consumer warps (one per stage) each reduce a whole chunk from shared
// memory to its score; a per-row arrival counter hands the row to the warp that
// scores its last chunk, which runs a warp-level top-k.
constexpr int kBulkWarps = 12;                      // consumer warps
constexpr int kBulkThreads = (kBulkWarps + 1) * 32;  // + producer warp
constexpr int kStages = 12;
// Sequence number `it` goes to stage it % kStages and to consumer warp
// it % kBulkWarps.  Bulk copies may land out of order, so a warp must wait on
// every phase of its stages itself (a parity wait cannot tell phase k-1 from
// k+1): hence every stage is owned by exactly one warp.
static_assert(kStages % kBulkWarps == 0, "each ring stage must belong to a single consumer warp");
constexpr uint32_t kStageBytes = 16384;

struct StageMeta {
  int row;         // b*H + h, or -1 for the stop marker
  int chunk;
  int row_chunks;  // chunks of this row that will be scored
  int unit;        // unit-counter slot | (chunks in the unit << 8)
};

// Per-unit arrival counters in shared memory: the warp that scores a unit's
// last chunk publishes the whole unit to the row's global counter, so a row
// costs one global atomic (and one fence) per unit rather than per chunk.  A
// unit's slot is reused kUnitSlots units later; at most 2 x kStages chunks
// (issued but not yet counted) separate the producer from the consumers, so
// that unit has been fully counted by then.
constexpr int kUnitSlots = 32;
static_assert(kUnitSlots > 2 * kStages, "unit slots must outlast the chunks in flight");

constexpr uint32_t kBulkSmem =
    kStages * kStageBytes + 2 * kStages * 8 + kStages * sizeof(StageMeta) + 64 + kUnitSlots * 4 + 128;

__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst), "l"(src),
      "r"(bytes), "r"(sm100::smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                   sm100::smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

// Warp-level top-k of scores[0, n): largest first, ties to the lower index,
// -1 past min(kout, n).  Same selection rule as block_topk.
__device__ void warp_topk(float* scores, int n, int kout, int32_t* out) {
  const int lane = threadIdx.x & 31;
  constexpr int kRegs = 16;
  const bool in_regs = n <= 32 * kRegs;
  unsigned long long keys[kRegs];
  if (in_regs) {
#pragma unroll
    for (int e = 0; e < kRegs; ++e) {
      const int i = lane + 32 * e;
      keys[e] = i < n ? make_key(__ldcg(scores + i), i) : 0ull;
    }
  }
  const int kvalid = min(kout, n);
  unsigned long long prev = ~0ull;
  for (int r = 0; r < kvalid; ++r) {
    unsigned long long best = 0ull;
    if (in_regs) {
#pragma unroll
      for (int e = 0; e < kRegs; ++e)
        if (keys[e] < prev && keys[e] > best) best = keys[e];
    } else {
      for (int i = lane; i < n; i += 32) {
        const unsigned long long kk = make_key(__ldcg(scores + i), i);
        if (kk < prev && kk > best) best = kk;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
      best = other > best ? other : best;
    }
    if (lane == 0) out[r] = static_cast<int32_t>(~static_cast<unsigned>(best & 0xffffffffull));
    prev = best;
  }
  for (int r = kvalid + lane; r < kout; r += 32) out[r] = -1;
  // Leave the workspace zero: a later call with other shapes may place its
  // arrival counters where these scores lie.
  __syncwarp();
  for (int i = lane; i < n; i += 32) scores[i] = 0.f;
}

__device__ __forceinline__ unsigned atom_add_acq_rel_cta(unsigned* addr, unsigned v) {
  unsigned old;
  asm volatile("atom.acq_rel.cta.shared::cta.add.u32 %0, [%1], %2;"
               : "=r"(old)
               : "r"(static_cast<uint32_t>(__cvta_generic_to_shared(addr))), "r"(v)
               : "memory");
  return old;
}

// Counts `cnt` freshly stored scores of `row` (one fence for the batch); the
// warp whose count completes the row resets its counter and selects its top-k.
__device__ __noinline__ void publish_scores(const SelectParams& p, int row, int cnt, int total, int lane) {
  int last = 0;
  if (lane == 0) {
    asm volatile("fence.acq_rel.gpu;" ::: "memory");  // release the stored scores
    const unsigned old = atomicAdd(p.counters + row, unsigned(cnt));
    last = old + unsigned(cnt) == unsigned(total);
    if (last) p.counters[row] = 0u;  // every chunk of the row has been scored
  }
  last = __shfl_sync(0xffffffffu, last, 0);
  if (last) {
    __threadfence();
    warp_topk(p.scores + size_t(row) * p.num_chunks, total, p.kout, p.out + size_t(row) * p.kout);
  }
}

template <typename T, int D>
__global__ void __launch_bounds__(kBulkThreads, 1) csa_select_bulk_kernel(SelectParams p, int* err) {
  using G = RowGeom<T, D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  uint8_t* stages = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
  uint64_t* empty = full + kStages;
  StageMeta* meta = reinterpret_cast<StageMeta*>(empty + kStages);
  int* abort_flag = reinterpret_cast<int*>(meta + kStages);
  unsigned* unit_cnt = reinterpret_cast<unsigned*>(abort_flag + 16);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t chunk_bytes = uint32_t(p.chunk) * D * sizeof(T);

  if (threadIdx.x < kUnitSlots) unit_cnt[threadIdx.x] = 0u;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      sm100::mbar_init(&full[s], 1);
      sm100::mbar_init(&empty[s], 1);
    }
    *abort_flag = 0;
    sm100::fence_mbar_init();
  }
  __syncthreads();
  volatile int* abort_v = abort_flag;

  if (warp == kBulkWarps) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      bool ok = true;
      uint32_t it = 0;
      // The next ticket is taken while the current unit is issued, so the
      // atomic's round trip overlaps the copies instead of stalling the ring.
      int u_next = static_cast<int>(atomicAdd(p.ticket, 1u));
      int cached_b = -1, cached_chunks = 0;
      uint32_t units_issued = 0;
      for (;;) {
        const int u = u_next;
        if (u >= p.total_units) break;
        u_next = static_cast<int>(atomicAdd(p.ticket, 1u));
        const int row = u / p.units_per_row;
        const int r = u - row * p.units_per_row;
        const int b = row / p.heads;
        if (b != cached_b) {
          cached_b = b;
          cached_chunks = p.num_chunks;
          if (p.seq_lens != nullptr) cached_chunks = min(max(p.seq_lens[b], 0), p.seq_len) / p.chunk;
        }
        const int row_chunks = cached_chunks;
        const int units_b = max(1, (row_chunks + p.unit - 1) / p.unit);
        if (r >= units_b) continue;
        if (row_chunks == 0) {  // nothing to score: the row's selection is all -1
          for (int i = 0; i < p.kout; ++i) p.out[size_t(row) * p.kout + i] = -1;
          continue;
        }
        const char* src = static_cast<const char*>(p.k) + (size_t(row) * p.seq_len) * D * sizeof(T);
        const int c1 = min((r + 1) * p.unit, row_chunks);
        const int unit_tag = int(units_issued++ % kUnitSlots) | ((c1 - r * p.unit) << 8);
        for (int c = r * p.unit; c < c1 && ok; ++c, ++it) {
          const int s = it % kStages;
          if (it >= kStages) ok = sm100::mbar_wait(&empty[s], ((it / kStages) - 1) & 1, abort_v);
          if (!ok) break;
          meta[s] = StageMeta{row, c, row_chunks, unit_tag};
          mbar_arrive_expect_tx(&full[s], chunk_bytes);
          bulk_g2s(sm100::smem_u32(stages + s * kStageBytes), src + size_t(c) * chunk_bytes, chunk_bytes, &full[s]);
        }
        if (!ok) break;
      }
      // One stop marker per consumer warp (consecutive sequence numbers cover every warp).
      for (int w = 0; w < kBulkWarps && ok; ++w, ++it) {
        const int s = it % kStages;
        if (it >= kStages) ok = sm100::mbar_wait(&empty[s], ((it / kStages) - 1) & 1, abort_v);
        if (!ok) break;
        meta[s] = StageMeta{-1, 0, 0, 0};
        sm100::mbar_arrive(&full[s]);
      }
      if (!ok) {
        *abort_flag = 1;
        report_device_error(err, kErrWaitTimeout);
      }
      __threadfence();
      const unsigned done = atomicAdd(p.ticket + 1, 1u);
      if (done == gridDim.x - 1) {  // last CTA out restores the zero workspace
        p.ticket[0] = 0u;
        p.ticket[1] = 0u;
      }
    }
  } else {
    // ------------------------------------------------------------ consumers
    const int tok_lane = lane / G::kLPT, vec_lane = lane % G::kLPT;
    constexpr int kRowBytes = D * sizeof(T);
    int cached_row = -1;
    float qf[G::kFPL];
    for (uint32_t it = warp;; it += kBulkWarps) {
      const int s = it % kStages;
      if (!sm100::mbar_wait(&full[s], (it / kStages) & 1, abort_v)) {
        if (lane == 0) report_device_error(err, kErrWaitTimeout);
        break;
      }
      const StageMeta m = meta[s];
      if (m.row < 0) break;
      if (m.row != cached_row) {
        const T* qrow = static_cast<const T*>(p.q) + size_t(m.row) * D;
#pragma unroll
        for (int j = 0; j < G::kVPL; ++j)
          Elem<T>::widen(*reinterpret_cast<const uint4*>(qrow + (vec_lane + 32 * j) * G::kVec), qf + j * G::kVec);
        cached_row = m.row;
      }
      const uint8_t* base = stages + s * kStageBytes;
      float acc[G::kFPL];
#pragma unroll
      for (int e = 0; e < G::kFPL; ++e) acc[e] = 0.f;
      const int steps = (p.chunk + G::kTPS - 1) / G::kTPS;
#pragma unroll 4
      for (int st = 0; st < steps; ++st) {
        const int t = st * G::kTPS + tok_lane;
        if (t < p.chunk) {
#pragma unroll
          for (int j = 0; j < G::kVPL; ++j) {
            const uint4 v = *reinterpret_cast<const uint4*>(base + t * kRowBytes + (vec_lane + 32 * j) * 16);
            float f[G::kVec];
            Elem<T>::widen(v, f);
#pragma unroll
            for (int e = 0; e < G::kVec; ++e) acc[j * G::kVec + e] += f[e];
          }
        }
      }
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(&empty[s]);  // the stage is read; the producer may refill it
      float dot = 0.f;
      const float count = float(p.chunk);
#pragma unroll
      for (int e = 0; e < G::kFPL; ++e) {
        const float sum = warp_sum_xor(acc[e], G::kLPT, 32);
        dot = fmaf(qf[e], __fdiv_rn(sum, count), dot);
      }
      dot = warp_sum_xor(dot, 1, G::kLPT);
      int unit_done = 0;
      if (lane == 0) {
        p.scores[size_t(m.row) * p.num_chunks + m.chunk] = dot * p.scale;
        const int slot = m.unit & 0xFF, n = m.unit >> 8;
        // Release the score to the warp that finishes the unit (same CTA).
        unit_done = atom_add_acq_rel_cta(unit_cnt + slot, 1u) == unsigned(n - 1);
        if (unit_done) unit_cnt[slot] = 0u;
      }
      if (__shfl_sync(0xffffffffu, unit_done, 0)) publish_scores(p, m.row, m.unit >> 8, m.row_chunks, lane);
    }
  }
}

template <typename T, int D>
int launch_select(const SelectParams& p, cudaStream_t stream) {
  const size_t chunk_bytes = size_t(p.chunk) * D * sizeof(T);
  if (chunk_bytes <= kStageBytes && chunk_bytes % 16 == 0) {
    static bool configured[64] = {};
    int dev = 0;
    CSAHCA_RETURN_IF_CUDA(cudaGetDevice(&dev));
    if (dev < 64 && !configured[dev]) {
      CSAHCA_RETURN_IF_CUDA(cudaFuncSetAttribute(csa_select_bulk_kernel<T, D>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize, int(kBulkSmem)));
      configured[dev] = true;
    }
    const int grid = std::min(csahca_num_sms(), p.total_units);
    csa_select_bulk_kernel<T, D><<<grid, kBulkThreads, kBulkSmem, stream>>>(p, csahca_device_error_ptr());
    CSAHCA_RETURN_IF_CUDA(cudaGetLastError());
    return CSAHCA_OK;
  }
  int per_sm = 0;
  CSAHCA_RETURN_IF_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, csa_select_kernel<T, D>, kSelThreads, 0));
  int grid = std::max(1, per_sm) * csahca_num_sms();
  grid = std::min(grid, p.total_units);
  csa_select_kernel<T, D><<<grid, kSelThreads, 0, stream>>>(p);
  CSAHCA_RETURN_IF_CUDA(cudaGetLastError());
  return CSAHCA_OK;
}

template <typename T>
int dispatch_select_dim(int64_t head_dim, const SelectParams& p, cudaStream_t s) {
  switch (head_dim) {
    case 32: return launch_select<T, 32>(p, s);
    case 64: return launch_select<T, 64>(p, s);
    case 128: return launch_select<T, 128>(p, s);
    case 256: return launch_select<T, 256>(p, s);
    case 512: return launch_select<T, 512>(p, s);
    default: return csahca_set_unsupported("head_dim must be one of 32, 64, 128, 256, 512");
  }
}

}  // namespace
}  // namespace csahca

using namespace csahca;

extern "C" size_t csahca_csa_select_topk_workspace_size(int64_t batch, int64_t heads, int64_t seq_len,
                                                        int64_t chunk_size) {
  if (batch < 0 || heads < 0 || seq_len < 0 || chunk_size <= 0) return 0;
  const size_t rows = size_t(batch) * size_t(heads);
  const size_t chunks = size_t(seq_len / chunk_size);
  return 256 + align256(rows * 4) + align256(rows * chunks * 4);
}

extern "C" int csahca_csa_select_topk(const void* q, const void* k_cache, const int32_t* seq_lens, int dtype,
                                      int64_t batch, int64_t heads, int64_t seq_len, int64_t head_dim,
                                      int64_t chunk_size, int64_t top_k, int32_t* out_indices, void* workspace,
                                      size_t workspace_bytes, void* stream) {
  if (chunk_size <= 0) return csahca_set_arg_error("chunk_size must be positive");
  if (top_k <= 0) return csahca_set_arg_error("top_k must be positive");
  if (seq_len % chunk_size != 0) return csahca_set_arg_error("seq length must be divisible by chunk_size");
  if (batch < 0 || heads < 0 || seq_len < 0) return csahca_set_arg_error("sizes must be non-negative");
  const int64_t num_chunks = seq_len / chunk_size;
  const int64_t kout = std::min<int64_t>(top_k, num_chunks);
  const int64_t rows = batch * heads;
  if (rows == 0 || kout == 0) return CSAHCA_OK;
  if (seq_len * head_dim * rows > (int64_t(1) << 40) || num_chunks * rows > (int64_t(1) << 31))
    return csahca_set_unsupported("problem too large");
  if (workspace_bytes < csahca_csa_select_topk_workspace_size(batch, heads, seq_len, chunk_size))
    return csahca_set_arg_error("workspace too small");
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k_cache)) & 15)
    return csahca_set_arg_error("q and k_cache must be 16-byte aligned");
  SelectParams p;
  p.q = q;
  p.k = k_cache;
  p.seq_lens = seq_lens;
  p.heads = int(heads);
  p.seq_len = int(seq_len);
  p.num_chunks = int(num_chunks);
  p.chunk = int(chunk_size);
  p.kout = int(kout);
  p.unit = kMaxChunksPerUnit;
  while (p.unit > kMinChunksPerUnit && rows * ((num_chunks + p.unit - 1) / p.unit) < 4 * int64_t(csahca_num_sms()))
    p.unit /= 2;
  p.units_per_row = int((num_chunks + p.unit - 1) / p.unit);
  if (p.units_per_row == 0) p.units_per_row = 1;
  p.total_units = int(rows) * p.units_per_row;
  p.scale = float(1.0 / sqrt(double(head_dim)));
  char* ws = static_cast<char*>(workspace);
  p.ticket = reinterpret_cast<unsigned*>(ws);
  p.counters = reinterpret_cast<unsigned*>(ws + 256);
  p.scores = reinterpret_cast<float*>(ws + 256 + align256(size_t(rows) * 4));
  p.out = out_indices;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case CSAHCA_DTYPE_BF16: return dispatch_select_dim<__nv_bfloat16>(head_dim, p, s);
    case CSAHCA_DTYPE_F16: return dispatch_select_dim<__half>(head_dim, p, s);
    case CSAHCA_DTYPE_F32: return dispatch_select_dim<float>(head_dim, p, s);
    default: return csahca_set_arg_error("unsupported dtype");
  }
}
