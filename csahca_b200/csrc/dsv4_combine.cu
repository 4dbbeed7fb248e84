// Log-sum-exp combine of DSV4 split-KV partials (sm_100a).
//
// Each of `parts` shards of a query's slot list produced, per (query, head), an
// output o_r normalised by its own softmax sum and lse_r = max + log2(sum) in
// log2 units (csahca_dsv4_decode_partial).  The full decode is
//   out = sum_r 2^(lse_r - M) o_r / (sum_r 2^(lse_r - M) + 2^(sink*log2e - M)),
// M = max(max_r lse_r, sink*log2e): the same sink-as-zero-valued-token rule as
// the single-shard kernel (dsv4_attention.cu:292-299 of the reference merge).
#include "common.cuh"

namespace csahca {
namespace {

constexpr int kDim = 512;
constexpr int kCombThreads = 128;
constexpr int kMaxParts = 64;

template <typename OT>
__global__ void __launch_bounds__(kCombThreads) dsv4_combine_kernel(const float* o, const float* lse, int parts,
                                                                    int rows, int heads, const float* sink, OT* out) {
  __shared__ float s_w[kMaxParts];
  __shared__ float s_inv;
  const int row = blockIdx.x;  // q * heads + h
  if (threadIdx.x == 0) {
    const float sk = sink != nullptr ? sink[row % heads] * kLog2e : -INFINITY;
    float m = sk;
    for (int r = 0; r < parts; ++r) m = fmaxf(m, lse[size_t(r) * rows + row]);
    float total = 0.f;
    for (int r = 0; r < parts; ++r) {
      const float l = lse[size_t(r) * rows + row];
      s_w[r] = (m == -INFINITY || l == -INFINITY) ? 0.f : exp2f(l - m);
      total += s_w[r];
    }
    if (m != -INFINITY && sk != -INFINITY) total += exp2f(sk - m);
    s_inv = total > 0.f ? 1.f / total : 0.f;
  }
  __syncthreads();
  for (int d = threadIdx.x; d < kDim; d += kCombThreads) {
    float a = 0.f;
    for (int r = 0; r < parts; ++r)
      if (s_w[r] != 0.f) a = fmaf(s_w[r], o[(size_t(r) * rows + row) * kDim + d], a);
    out[size_t(row) * kDim + d] = Elem<OT>::from_f(a * s_inv);
  }
}

}  // namespace
}  // namespace csahca

using namespace csahca;

extern "C" int csahca_dsv4_combine_partials(const float* o_parts, const float* lse_parts, int64_t parts,
                                            int64_t num_queries, int64_t heads, const float* attn_sink, void* out,
                                            int out_dtype, void* stream) {
  if (parts <= 0 || parts > kMaxParts) return csahca_set_arg_error("parts must be in [1, 64]");
  if (num_queries < 0 || heads < 0) return csahca_set_arg_error("sizes must be non-negative");
  const int64_t rows = num_queries * heads;
  if (rows == 0) return CSAHCA_OK;
  if (rows > (int64_t(1) << 30)) return csahca_set_unsupported("problem too large");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const dim3 grid{static_cast<unsigned>(rows)};
  switch (out_dtype) {
    case CSAHCA_DTYPE_BF16:
      dsv4_combine_kernel<__nv_bfloat16><<<grid, kCombThreads, 0, s>>>(
          o_parts, lse_parts, int(parts), int(rows), int(heads), attn_sink, static_cast<__nv_bfloat16*>(out));
      break;
    case CSAHCA_DTYPE_F16:
      dsv4_combine_kernel<__half><<<grid, kCombThreads, 0, s>>>(o_parts, lse_parts, int(parts), int(rows),
                                                                int(heads), attn_sink, static_cast<__half*>(out));
      break;
    case CSAHCA_DTYPE_F32:
      dsv4_combine_kernel<float><<<grid, kCombThreads, 0, s>>>(o_parts, lse_parts, int(parts), int(rows), int(heads),
                                                               attn_sink, static_cast<float*>(out));
      break;
    default:
      return csahca_set_arg_error("unsupported output dtype");
  }
  CSAHCA_RETURN_IF_CUDA(cudaGetLastError());
  return CSAHCA_OK;
}
