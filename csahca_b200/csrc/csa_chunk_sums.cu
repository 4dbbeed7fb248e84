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
#include <algorithm>

#include "common.cuh"

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
