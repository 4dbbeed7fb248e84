// CSA chunk scorer + per-(batch, head) top-k (sm_100a).
//
// Restates hybrid_attention/reference.py:40-56 (chunk_mean + select_topk_chunks)
// as one streaming kernel: K is read once at full HBM rate with 16-byte
// non-allocating loads, each warp reduces one chunk to its fp32 mean, dots it
// with q and stores the scaled score; the CTA that scores the last chunk range
// of a (batch, head) row then selects that row's top-k (ties: lower index).
//
// Work distribution: persistent CTAs (SM count x occupancy) take fixed-size
// units of kChunksPerUnit chunks from an atomic ticket, so ragged per-request
// lengths cost nothing for the chunks past a request's end.
//
// Workspace layout (zero on entry, zero on exit):
//   [0, 256)          ticket[0] = next unit, ticket[1] = retired CTAs
//   [256, 256+4BH)    per-row arrival counters (rounded up to 256 B)
//   [.., + 4*BH*C)    fp32 chunk scores
#include <algorithm>

#include "common.cuh"

namespace csahca {
namespace {

constexpr int kSelThreads = 256;
constexpr int kSelWarps = kSelThreads / 32;
constexpr int kChunksPerUnit = 16;
constexpr int kTopkRegs = 16;  // register path holds up to kSelThreads*kTopkRegs scores

struct SelectParams {
  const void* q;
  const void* k;
  const int32_t* seq_lens;
  int heads, seq_len, num_chunks, chunk, kout;
  int units_per_row;  // ceil(num_chunks / kChunksPerUnit)
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

__device__ __forceinline__ unsigned long long make_key(float score, int idx) {
  return (static_cast<unsigned long long>(float_order_key(score)) << 32) | static_cast<unsigned>(~idx);
}

// Top-k of scores[0, n) written to out[0, kout): largest first, equal scores by
// lower index, slots past min(kout, n) get -1.  Called by all threads of a CTA.
// Round r picks the largest composite key below round r-1's pick, so no element
// needs to be marked as taken.
__device__ void block_topk(const float* scores, int n, int kout, int32_t* out, unsigned long long* s_red) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const bool in_regs = n <= kSelThreads * kTopkRegs;
  unsigned long long keys[kTopkRegs];
  if (in_regs) {
#pragma unroll
    for (int e = 0; e < kTopkRegs; ++e) {
      const int i = tid + e * kSelThreads;
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
      for (int i = tid; i < n; i += kSelThreads) {
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
    for (int w = 1; w < kSelWarps; ++w) best = s_red[w] > best ? s_red[w] : best;
    __syncthreads();
    if (tid == 0) out[r] = static_cast<int32_t>(~static_cast<unsigned>(best & 0xffffffffull));
    prev = best;
  }
  for (int r = kvalid + tid; r < kout; r += kSelThreads) out[r] = -1;
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
    const int units_b = max(1, (row_chunks + kChunksPerUnit - 1) / kChunksPerUnit);
    if (r >= units_b) continue;  // uniform across the CTA

    const T* qrow = static_cast<const T*>(p.q) + size_t(row) * D;
    float qf[G::kFPL];
#pragma unroll
    for (int j = 0; j < G::kVPL; ++j) {
      const uint4 v = *reinterpret_cast<const uint4*>(qrow + (vec_lane + 32 * j) * G::kVec);
      Elem<T>::widen(v, qf + j * G::kVec);
    }
    const T* krow = static_cast<const T*>(p.k) + size_t(row) * p.seq_len * D;
    const int c0 = r * kChunksPerUnit;
    const int c1 = min(c0 + kChunksPerUnit, row_chunks);
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

template <typename T, int D>
int launch_select(const SelectParams& p, cudaStream_t stream) {
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
  p.units_per_row = int((num_chunks + kChunksPerUnit - 1) / kChunksPerUnit);
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
