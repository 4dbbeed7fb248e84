// Incremental chunk-sum cache for the CSA scorer (sm_100a).
//
// The scorer of hybrid_attention/reference.py:40-56 reads all of K every decode
// step to form per-chunk means.  During decoding a chunk's mean changes only
// while its tokens are being written, so a cache of fp32 chunk sums
// [B,H,S/chunk,D] (1/32 of a bf16 K cache at chunk 64) can stand in for K:
// scores become q . sum / chunk / sqrt(D), which ranks chunks exactly as
// q . mean / sqrt(D) up to fp32 rounding.  The scorer kernel runs on the sums
// with chunk = 1 (a "chunk" of one fp32 row is the row itself).
//
//   build:  sums[b,h,c,:] = sum_t K[b,h,c*chunk + t,:]          (fp32, token order)
//   append: sums[b,h,p/chunk,:] (+)= K[b,h,p,:] for p = positions[b]; the first
//           token of a chunk (p % chunk == 0) overwrites, so the cache needs no
//           clearing between requests.
//   select: one CTA per (b,h) row: warps take chunk rows of the sums (fp32
//           row-contiguous, 16-byte loads, eight rows in flight per warp), dot
//           them with q into the workspace scores, then the CTA's top-k.  The
//           cache is a dense [C, D] fp32 matrix per row, so this is a plain
//           GEMV-plus-select at HBM speed with no per-chunk bookkeeping.
#include <algorithm>
#include <cmath>

#include "common.cuh"
#include "topk.cuh"

namespace csahca {
namespace {

constexpr int kSumThreads = 256;

template <typename T>
__global__ void __launch_bounds__(kSumThreads) chunk_sums_build_kernel(const T* k, float* sums, int64_t rows,
                                                                       int seq_len, int dim, int chunk) {
  const int nchunks = seq_len / chunk;
  const int64_t total = rows * nchunks;
  const int warps = kSumThreads / 32;
  const int lane = threadIdx.x & 31;
  for (int64_t w = int64_t(blockIdx.x) * warps + (threadIdx.x >> 5); w < total; w += int64_t(gridDim.x) * warps) {
    const int64_t row = w / nchunks;
    const int c = int(w - row * nchunks);
    const T* src = k + (size_t(row) * seq_len + size_t(c) * chunk) * dim;
    float* dst = sums + size_t(w) * dim;
    for (int d = lane; d < dim; d += 32) {
      float acc = 0.f;
      for (int t = 0; t < chunk; ++t) acc += Elem<T>::to_f(src[size_t(t) * dim + d]);
      dst[d] = acc;
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(kSumThreads) chunk_sums_append_kernel(const T* k, const int32_t* positions,
                                                                        float* sums, int heads, int seq_len, int dim,
                                                                        int chunk, int64_t rows) {
  const int64_t i = int64_t(blockIdx.x) * kSumThreads + threadIdx.x;  // (row, dim)
  if (i >= rows * dim) return;
  const int64_t row = i / dim;
  const int d = int(i - row * dim);
  const int pos = positions[row / heads];
  if (pos < 0 || pos >= seq_len || pos / chunk >= seq_len / chunk) return;
  const float v = Elem<T>::to_f(k[(size_t(row) * seq_len + pos) * dim + d]);
  float* dst = sums + (size_t(row) * (seq_len / chunk) + pos / chunk) * dim + d;
  *dst = (pos % chunk == 0) ? v : *dst + v;
}

template <typename T>
int launch_build(const void* k, float* sums, int64_t rows, int64_t s, int64_t d, int64_t chunk, cudaStream_t st) {
  const int64_t warps_needed = rows * (s / chunk);
  const int64_t blocks = std::min<int64_t>((warps_needed + 7) / 8, int64_t(csahca_num_sms()) * 16);
  if (blocks == 0) return CSAHCA_OK;
  chunk_sums_build_kernel<T><<<unsigned(blocks), kSumThreads, 0, st>>>(static_cast<const T*>(k), sums, rows, int(s),
                                                                       int(d), int(chunk));
  CSAHCA_RETURN_IF_CUDA(cudaGetLastError());
  return CSAHCA_OK;
}

template <typename T>
int launch_append(const void* k, const int32_t* pos, float* sums, int64_t heads, int64_t rows, int64_t s, int64_t d,
                  int64_t chunk, cudaStream_t st) {
  const int64_t n = rows * d;
  if (n == 0) return CSAHCA_OK;
  chunk_sums_append_kernel<T><<<unsigned((n + kSumThreads - 1) / kSumThreads), kSumThreads, 0, st>>>(
      static_cast<const T*>(k), pos, sums, int(heads), int(s), int(d), int(chunk), rows);
  CSAHCA_RETURN_IF_CUDA(cudaGetLastError());
  return CSAHCA_OK;
}

// Few rows (fewer than SMs): 512 threads per row for more loads in flight;
// many rows: 256 threads and three CTAs per SM.
template <typename QT, int kSelSumThreads>
__global__ void __launch_bounds__(kSelSumThreads, 768 / kSelSumThreads) select_from_sums_kernel(const QT* q, const float* sums,
                                                                          const int32_t* seq_lens, int heads,
                                                                          int nchunks, int dim, int chunk, int kout,
                                                                          float scale, float* scores, int32_t* out) {
  __shared__ float s_q[1024];
  __shared__ unsigned long long s_red[kSelSumThreads / 32];
  const int row = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int d = threadIdx.x; d < dim; d += kSelSumThreads) s_q[d] = Elem<QT>::to_f(q[size_t(row) * dim + d]);
  int n = nchunks;
  if (seq_lens != nullptr) n = min(max(seq_lens[row / heads], 0) / chunk, nchunks);
  __syncthreads();
  const float* base = sums + size_t(row) * nchunks * dim;
  float* sc = scores + size_t(row) * nchunks;
  constexpr int kRows = 8;  // chunk rows in flight per warp
  for (int c0 = warp * kRows; c0 < n; c0 += (kSelSumThreads / 32) * kRows) {
    float acc[kRows];
#pragma unroll
    for (int i = 0; i < kRows; ++i) acc[i] = 0.f;
    for (int d = lane * 4; d < dim; d += 128) {
      float4 v[kRows];
#pragma unroll
      for (int i = 0; i < kRows; ++i)
        v[i] = c0 + i < n ? __ldcs(reinterpret_cast<const float4*>(base + size_t(c0 + i) * dim + d))
                          : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int i = 0; i < kRows; ++i)
        acc[i] = fmaf(v[i].x, s_q[d], fmaf(v[i].y, s_q[d + 1], fmaf(v[i].z, s_q[d + 2], fmaf(v[i].w, s_q[d + 3], acc[i]))));
    }
#pragma unroll
    for (int i = 0; i < kRows; ++i) {
      const float t = warp_sum_xor(acc[i], 1, 32);
      if (lane == 0 && c0 + i < n) sc[c0 + i] = t * scale;
    }
  }
  __syncthreads();
  topk::block_topk<kSelSumThreads>(sc, n, kout, out + size_t(row) * kout, s_red);
}

int check_shape(int64_t batch, int64_t heads, int64_t seq_len, int64_t head_dim, int64_t chunk) {
  if (chunk <= 0) return csahca_set_arg_error("chunk_size must be positive");
  if (batch < 0 || heads < 0 || seq_len < 0 || head_dim <= 0) return csahca_set_arg_error("sizes must be non-negative");
  if (seq_len % chunk != 0) return csahca_set_arg_error("seq length must be divisible by chunk_size");
  if (batch * heads * seq_len * head_dim >= (int64_t(1) << 40)) return csahca_set_unsupported("problem too large");
  return CSAHCA_OK;
}

}  // namespace
}  // namespace csahca

using namespace csahca;

extern "C" int csahca_csa_chunk_sums_build(const void* k_cache, int dtype, int64_t batch, int64_t heads,
                                           int64_t seq_len, int64_t head_dim, int64_t chunk_size, float* sums,
                                           void* stream) {
  if (int rc = check_shape(batch, heads, seq_len, head_dim, chunk_size)) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t rows = batch * heads;
  switch (dtype) {
    case CSAHCA_DTYPE_BF16: return launch_build<__nv_bfloat16>(k_cache, sums, rows, seq_len, head_dim, chunk_size, st);
    case CSAHCA_DTYPE_F16: return launch_build<__half>(k_cache, sums, rows, seq_len, head_dim, chunk_size, st);
    case CSAHCA_DTYPE_F32: return launch_build<float>(k_cache, sums, rows, seq_len, head_dim, chunk_size, st);
    default: return csahca_set_arg_error("unsupported dtype");
  }
}

extern "C" int csahca_csa_chunk_sums_append(const void* k_cache, int dtype, int64_t batch, int64_t heads,
                                            int64_t seq_len, int64_t head_dim, int64_t chunk_size,
                                            const int32_t* positions, float* sums, void* stream) {
  if (int rc = check_shape(batch, heads, seq_len, head_dim, chunk_size)) return rc;
  if (positions == nullptr) return csahca_set_arg_error("positions is required");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t rows = batch * heads;
  switch (dtype) {
    case CSAHCA_DTYPE_BF16:
      return launch_append<__nv_bfloat16>(k_cache, positions, sums, heads, rows, seq_len, head_dim, chunk_size, st);
    case CSAHCA_DTYPE_F16:
      return launch_append<__half>(k_cache, positions, sums, heads, rows, seq_len, head_dim, chunk_size, st);
    case CSAHCA_DTYPE_F32:
      return launch_append<float>(k_cache, positions, sums, heads, rows, seq_len, head_dim, chunk_size, st);
    default: return csahca_set_arg_error("unsupported dtype");
  }
}

extern "C" int csahca_csa_select_topk_from_sums(const void* q, int q_dtype, const float* sums,
                                                const int32_t* seq_lens, int64_t batch, int64_t heads,
                                                int64_t num_chunks, int64_t head_dim, int64_t chunk_size,
                                                int64_t top_k, int32_t* out_indices, void* workspace,
                                                size_t workspace_bytes, void* stream) {
  if (int rc = check_shape(batch, heads, num_chunks * chunk_size, head_dim, chunk_size)) return rc;
  if (top_k <= 0) return csahca_set_arg_error("top_k must be positive");
  if (head_dim % 4 != 0 || head_dim > 1024) return csahca_set_unsupported("head_dim must be a multiple of 4, <= 1024");
  if (reinterpret_cast<uintptr_t>(sums) & 15) return csahca_set_arg_error("sums must be 16-byte aligned");
  const int64_t rows = batch * heads;
  if (rows == 0 || num_chunks == 0) return CSAHCA_OK;
  if (workspace_bytes < csahca_csa_select_topk_workspace_size(batch, heads, num_chunks * chunk_size, chunk_size))
    return csahca_set_arg_error("workspace too small");
  // Same workspace layout as csahca_csa_select_topk: scores after the ticket and counters.
  float* scores = reinterpret_cast<float*>(static_cast<char*>(workspace) + 256 + ((size_t(rows) * 4 + 255) & ~size_t(255)));
  const int kout = int(std::min(top_k, num_chunks));
  const float scale = float(1.0 / (std::sqrt(double(head_dim)) * double(chunk_size)));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const dim3 grid{static_cast<unsigned>(rows)};
  const bool wide = rows < csahca_num_sms();
#define CSAHCA_SUMS_LAUNCH(QT)                                                                                    \
  do {                                                                                                           \
    if (wide)                                                                                                    \
      select_from_sums_kernel<QT, 512><<<grid, 512, 0, st>>>(static_cast<const QT*>(q), sums, seq_lens, int(heads), \
                                                              int(num_chunks), int(head_dim), int(chunk_size), kout, \
                                                              scale, scores, out_indices);                          \
    else                                                                                                         \
      select_from_sums_kernel<QT, 256><<<grid, 256, 0, st>>>(static_cast<const QT*>(q), sums, seq_lens, int(heads), \
                                                              int(num_chunks), int(head_dim), int(chunk_size), kout, \
                                                              scale, scores, out_indices);                          \
  } while (0)
  switch (q_dtype) {
    case CSAHCA_DTYPE_BF16: CSAHCA_SUMS_LAUNCH(__nv_bfloat16); break;
    case CSAHCA_DTYPE_F16: CSAHCA_SUMS_LAUNCH(__half); break;
    case CSAHCA_DTYPE_F32: CSAHCA_SUMS_LAUNCH(float); break;
    default: return csahca_set_arg_error("unsupported dtype");
  }
#undef CSAHCA_SUMS_LAUNCH
  CSAHCA_RETURN_IF_CUDA(cudaGetLastError());
  return CSAHCA_OK;
}
