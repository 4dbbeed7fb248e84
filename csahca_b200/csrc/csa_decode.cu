// CSA split-K decode with in-kernel log-sum-exp combine (sm_100a).
//
// Replaces csrc/csa_attention.cu's three kernels (csa_decode_forward_kernel
// :10-91, csa_decode_tile_kernel :125-222, csa_decode_merge_kernel :225-274).
//
// One CTA = one unit of G selected chunks of one (batch, head) row.  Its 8 warps
// stream the unit's K and V rows with 16-byte non-allocating loads (a warp step
// covers 512 contiguous bytes: two 128-dim bf16 rows), keep an online softmax
// per token lane group in registers, and merge warp states through shared
// memory.  With 2..8 units per row and a small grid (at most kClusterGridMax
// CTAs), the row's CTAs form a thread-block cluster:
// each leaves its (max, sum, acc) partial in shared memory and rank 0 combines
// them through distributed shared memory.  With more units, each CTA stores its
// partial in the workspace and the last CTA of the row (atomic arrival
// counter) combines them.  Either way a decode is one launch.
//
// Token validity follows the reference: a slot with a negative chunk index is
// skipped (csa_attention.cu:176-179), and so is a token at or beyond seq_len
// (:181-184); a row with no token left yields zeros (:88).
//
// Workspace (used only on the counter path; any content on entry,
// the counters are cleared by a memset on the call's stream):
//   [0, 4*BH) arrival counters (rounded up to 256 B), then fp32 partials
//   [BH][U][D+2] = (acc[D], max, sum).
#include <algorithm>
#include <mutex>

#include <cooperative_groups.h>

#include "common.cuh"

namespace csahca {
namespace {

constexpr int kDecThreads = 256;
constexpr int kDecWarps = kDecThreads / 32;
constexpr int kMaxGroup = 16;      // selected chunks per CTA at most
// Split rows until at least this many CTAs: fewer, longer CTAs stream better.
// Measured on the config-2 distribution (decode only, back to back): 8 requests
// 47 -> 35 us, 16 requests 65 -> 54 us, 32 requests 107 -> 97 us going from a
// target of 2048 CTAs to 512; 64 requests and config 1 split the same either way.
constexpr int kTargetCtas = 512;

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

int pick_group(int64_t rows, int64_t top_k) {
  int g = int(std::min<int64_t>(top_k, kMaxGroup));
  while (g > 1 && rows * ((top_k + g - 1) / g) < kTargetCtas) g = (g + 1) / 2;
  return std::max(g, 1);
}

struct DecodeParams {
  const void* q;
  const void* k;
  const void* v;
  const void* idx;
  void* out;
  float* partial;
  unsigned* counters;
  int seq_len, top_k, chunk, group, units;
  float scale_log2;  // softmax scale * log2(e)
};

constexpr int kMaxClusterUnits = 8;  // portable cluster size
constexpr int64_t kClusterGridMax = 2048;

// kCluster: the row's `units` CTAs form one thread-block cluster and combine
// their partials through distributed shared memory (no workspace, no counters).
template <typename T, int D, typename IdxT, bool kCluster>
__global__ void __launch_bounds__(kDecThreads) csa_decode_kernel(DecodeParams p) {
  using G = RowGeom<T, D>;
  constexpr int kU = G::kVPL >= 4 ? 1 : 4 / G::kVPL;  // steps per batch (K+V loads in flight: 2*kU*kVPL)
  constexpr int kRowBytes = D * sizeof(T);

  __shared__ int s_chunk[kMaxGroup];
  __shared__ float s_m[kDecWarps], s_l[kDecWarps];
  __shared__ float s_acc[kDecWarps][D];
  __shared__ int s_last;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int tok_lane = lane / G::kLPT, vec_lane = lane % G::kLPT;
  const int row = blockIdx.x / p.units;
  const int unit = blockIdx.x - row * p.units;
  const int slot0 = unit * p.group;
  const int nslots = min(p.group, p.top_k - slot0);

  if (tid < nslots) {
    // A chunk that starts at or past seq_len holds no valid token: mapping it to
    // -1 here also keeps c * chunk below 2^31 in the token arithmetic below.
    const IdxT c = static_cast<const IdxT*>(p.idx)[size_t(row) * p.top_k + slot0 + tid];
    const IdxT nchunks = IdxT((p.seq_len + p.chunk - 1) / p.chunk);
    s_chunk[tid] = (c < 0 || c >= nchunks) ? -1 : int(c);
  }
  __syncthreads();

  float qf[G::kFPL];
  {
    const T* qrow = static_cast<const T*>(p.q) + size_t(row) * D;
#pragma unroll
    for (int j = 0; j < G::kVPL; ++j)
      Elem<T>::widen(*reinterpret_cast<const uint4*>(qrow + (vec_lane + 32 * j) * G::kVec), qf + j * G::kVec);
  }
  const char* kbase = static_cast<const char*>(p.k) + size_t(row) * p.seq_len * kRowBytes;
  const char* vbase = static_cast<const char*>(p.v) + size_t(row) * p.seq_len * kRowBytes;

  float m = -INFINITY, l = 0.f;
  float acc[G::kFPL];
#pragma unroll
  for (int e = 0; e < G::kFPL; ++e) acc[e] = 0.f;

  const int ntok = nslots * p.chunk;
  const int nsteps = (ntok + G::kTPS - 1) / G::kTPS;
  for (int sb = warp; sb < nsteps; sb += kDecWarps * kU) {
    uint4 kv[kU][G::kVPL], vv[kU][G::kVPL];
    bool ok[kU];
#pragma unroll
    for (int i = 0; i < kU; ++i) {
      const int s = sb + i * kDecWarps;
      const int t = s * G::kTPS + tok_lane;
      int token = -1;
      if (s < nsteps && t < ntok) {
        const int sl = t / p.chunk;
        const int c = s_chunk[sl];
        const int tk = c * p.chunk + (t - sl * p.chunk);
        if (c >= 0 && tk < p.seq_len) token = tk;
      }
      ok[i] = token >= 0;
#pragma unroll
      for (int j = 0; j < G::kVPL; ++j) {
        const size_t off = size_t(token) * kRowBytes + size_t(vec_lane + 32 * j) * 16;
        kv[i][j] = ok[i] ? ldg_stream(kbase + off) : make_uint4(0, 0, 0, 0);
        vv[i][j] = ok[i] ? ldg_stream(vbase + off) : make_uint4(0, 0, 0, 0);
      }
    }
    float sc[kU];
    float mx = m;
#pragma unroll
    for (int i = 0; i < kU; ++i) {
      float d = 0.f;
#pragma unroll
      for (int j = 0; j < G::kVPL; ++j) {
        float f[G::kVec];
        Elem<T>::widen(kv[i][j], f);
#pragma unroll
        for (int e = 0; e < G::kVec; ++e) d = fmaf(qf[j * G::kVec + e], f[e], d);
      }
      d = warp_sum_xor(d, 1, G::kLPT);
      sc[i] = ok[i] ? d * p.scale_log2 : -INFINITY;
      mx = fmaxf(mx, sc[i]);
    }
    if (mx == -INFINITY) continue;  // nothing valid yet for this lane group
    const float alpha = exp2f(m - mx);
    l *= alpha;
#pragma unroll
    for (int e = 0; e < G::kFPL; ++e) acc[e] *= alpha;
#pragma unroll
    for (int i = 0; i < kU; ++i) {
      const float pi = exp2f(sc[i] - mx);
      l += pi;
#pragma unroll
      for (int j = 0; j < G::kVPL; ++j) {
        float f[G::kVec];
        Elem<T>::widen(vv[i][j], f);
#pragma unroll
        for (int e = 0; e < G::kVec; ++e) acc[j * G::kVec + e] = fmaf(pi, f[e], acc[j * G::kVec + e]);
      }
    }
    m = mx;
  }

  // Merge the token lane groups of the warp (same vec_lane, different tokens).
#pragma unroll
  for (int o = G::kLPT; o < 32; o <<= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    const float l2 = __shfl_xor_sync(0xffffffffu, l, o);
    const float mm = fmaxf(m, m2);
    const float a1 = mm == -INFINITY ? 0.f : exp2f(m - mm);
    const float a2 = mm == -INFINITY ? 0.f : exp2f(m2 - mm);
    l = l * a1 + l2 * a2;
#pragma unroll
    for (int e = 0; e < G::kFPL; ++e) {
      const float x2 = __shfl_xor_sync(0xffffffffu, acc[e], o);
      acc[e] = acc[e] * a1 + x2 * a2;
    }
    m = mm;
  }
  if (tok_lane == 0) {
#pragma unroll
    for (int j = 0; j < G::kVPL; ++j)
#pragma unroll
      for (int e = 0; e < G::kVec; ++e) s_acc[warp][(vec_lane + 32 * j) * G::kVec + e] = acc[j * G::kVec + e];
    if (lane == 0) {
      s_m[warp] = m;
      s_l[warp] = l;
    }
  }
  __syncthreads();

  // Merge the warps.
  float mm = -INFINITY;
#pragma unroll
  for (int w = 0; w < kDecWarps; ++w) mm = fmaxf(mm, s_m[w]);
  float wgt[kDecWarps];
  float ll = 0.f;
#pragma unroll
  for (int w = 0; w < kDecWarps; ++w) {
    wgt[w] = mm == -INFINITY ? 0.f : exp2f(s_m[w] - mm);
    ll += s_l[w] * wgt[w];
  }
  T* out = static_cast<T*>(p.out) + size_t(row) * D;
  if (p.units == 1) {
    const float inv = ll > 0.f ? 1.f / ll : 0.f;
    for (int d = tid; d < D; d += kDecThreads) {
      float a = 0.f;
#pragma unroll
      for (int w = 0; w < kDecWarps; ++w) a = fmaf(s_acc[w][d], wgt[w], a);
      out[d] = Elem<T>::from_f(a * inv);
    }
    return;
  }

  if constexpr (kCluster) {
    namespace cg = cooperative_groups;
    __shared__ float s_part[D];
    __shared__ float s_ml[2];
    for (int d = tid; d < D; d += kDecThreads) {
      float a = 0.f;
#pragma unroll
      for (int w = 0; w < kDecWarps; ++w) a = fmaf(s_acc[w][d], wgt[w], a);
      s_part[d] = a;
    }
    if (tid == 0) {
      s_ml[0] = mm;
      s_ml[1] = ll;
    }
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();  // every CTA's partial is in its shared memory
    if (cluster.block_rank() == 0) {
      const int n = int(cluster.num_blocks());
      float gm = -INFINITY;
      for (int r = 0; r < n; ++r) gm = fmaxf(gm, cluster.map_shared_rank(s_ml, r)[0]);
      float gl = 0.f;
      for (int r = 0; r < n; ++r) {
        const float* ml = cluster.map_shared_rank(s_ml, r);
        if (ml[0] != -INFINITY) gl += ml[1] * exp2f(ml[0] - gm);
      }
      const float inv = gl > 0.f ? 1.f / gl : 0.f;
      for (int d = tid; d < D; d += kDecThreads) {
        float a = 0.f;
        for (int r = 0; r < n; ++r) {
          const float mu = cluster.map_shared_rank(s_ml, r)[0];
          if (mu != -INFINITY) a = fmaf(cluster.map_shared_rank(s_part, r)[d], exp2f(mu - gm), a);
        }
        out[d] = Elem<T>::from_f(a * inv);
      }
    }
    cluster.sync();  // peers keep their shared memory until rank 0 has read it
    return;
  }

  float* part = p.partial + (size_t(row) * p.units + unit) * (D + 2);
  for (int d = tid; d < D; d += kDecThreads) {
    float a = 0.f;
#pragma unroll
    for (int w = 0; w < kDecWarps; ++w) a = fmaf(s_acc[w][d], wgt[w], a);
    part[d] = a;
  }
  if (tid == 0) {
    part[D] = mm;
    part[D + 1] = ll;
  }
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    const unsigned old = atomicAdd(p.counters + row, 1u);
    s_last = old == unsigned(p.units - 1);
    if (s_last) p.counters[row] = 0u;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();

  // Last CTA of the row: log-sum-exp combine of the row's partials.
  const float* rp = p.partial + size_t(row) * p.units * (D + 2);
  float gm = -INFINITY;
  for (int u = 0; u < p.units; ++u) gm = fmaxf(gm, __ldcg(rp + size_t(u) * (D + 2) + D));
  float gl = 0.f;
  for (int u = 0; u < p.units; ++u) {
    const float mu = __ldcg(rp + size_t(u) * (D + 2) + D);
    if (mu != -INFINITY) gl += __ldcg(rp + size_t(u) * (D + 2) + D + 1) * exp2f(mu - gm);
  }
  const float inv = gl > 0.f ? 1.f / gl : 0.f;
  for (int d = tid; d < D; d += kDecThreads) {
    float a = 0.f;
    for (int u = 0; u < p.units; ++u) {
      const float mu = __ldcg(rp + size_t(u) * (D + 2) + D);
      if (mu != -INFINITY) a = fmaf(__ldcg(rp + size_t(u) * (D + 2) + d), exp2f(mu - gm), a);
    }
    out[d] = Elem<T>::from_f(a * inv);
  }
}

template <typename T, int D, typename IdxT>
int launch_decode_idx(const DecodeParams& p, int64_t rows, cudaStream_t s) {
  const dim3 grid(unsigned(rows * p.units));
  // Small grids (latency-bound decodes) combine inside a cluster; large grids
  // keep unconstrained CTA placement and combine through the workspace.
  if (p.units > 1 && p.units <= kMaxClusterUnits && rows * p.units <= kClusterGridMax) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kDecThreads);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = unsigned(p.units);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    CSAHCA_RETURN_IF_CUDA(cudaLaunchKernelEx(&cfg, csa_decode_kernel<T, D, IdxT, true>, p));
  } else {
    csa_decode_kernel<T, D, IdxT, false><<<grid, kDecThreads, 0, s>>>(p);
  }
  CSAHCA_RETURN_IF_CUDA(cudaGetLastError());
  return CSAHCA_OK;
}

template <typename T, int D>
int launch_decode(const DecodeParams& p, int64_t rows, int index_dtype, cudaStream_t s) {
  if (index_dtype == CSAHCA_INDEX_I32) return launch_decode_idx<T, D, int32_t>(p, rows, s);
  return launch_decode_idx<T, D, int64_t>(p, rows, s);
}

template <typename T>
int dispatch_decode_dim(int64_t head_dim, const DecodeParams& p, int64_t rows, int index_dtype, cudaStream_t s) {
  switch (head_dim) {
    case 32: return launch_decode<T, 32>(p, rows, index_dtype, s);
    case 64: return launch_decode<T, 64>(p, rows, index_dtype, s);
    case 128: return launch_decode<T, 128>(p, rows, index_dtype, s);
    case 256: return launch_decode<T, 256>(p, rows, index_dtype, s);
    case 512: return launch_decode<T, 512>(p, rows, index_dtype, s);
    default: return csahca_set_unsupported("head_dim must be one of 32, 64, 128, 256, 512");
  }
}

}  // namespace
}  // namespace csahca

using namespace csahca;

extern "C" size_t csahca_csa_decode_workspace_size(int64_t batch, int64_t heads, int64_t head_dim, int64_t top_k,
                                                   int64_t chunk_size) {
  (void)chunk_size;
  if (batch <= 0 || heads <= 0 || top_k <= 0 || head_dim <= 0) return 256;
  const int64_t rows = batch * heads;
  const int g = pick_group(rows, top_k);
  const int64_t units = (top_k + g - 1) / g;
  if (units == 1) return align256(size_t(rows) * 4);
  return align256(size_t(rows) * 4) + size_t(rows) * size_t(units) * size_t(head_dim + 2) * 4;
}

extern "C" int csahca_csa_decode(const void* q, const void* k_cache, const void* v_cache, const void* chunk_indices,
                                 int index_dtype, int dtype, int64_t batch, int64_t heads, int64_t seq_len,
                                 int64_t head_dim, int64_t top_k, int64_t chunk_size, void* out, void* workspace,
                                 size_t workspace_bytes, void* stream) {
  if (chunk_size <= 0) return csahca_set_arg_error("chunk_size must be positive");
  if (batch < 0 || heads < 0 || seq_len < 0 || top_k < 0) return csahca_set_arg_error("sizes must be non-negative");
  if (index_dtype != CSAHCA_INDEX_I32 && index_dtype != CSAHCA_INDEX_I64)
    return csahca_set_arg_error("chunk_indices must be int32 or int64");
  const int64_t rows = batch * heads;
  if (rows == 0) return CSAHCA_OK;
  const size_t esize = dtype == CSAHCA_DTYPE_F32 ? 4 : 2;
  if (top_k == 0) {  // no slot: every row is empty -> zeros
    CSAHCA_RETURN_IF_CUDA(
        cudaMemsetAsync(out, 0, size_t(rows) * size_t(head_dim) * esize, static_cast<cudaStream_t>(stream)));
    return CSAHCA_OK;
  }
  if (seq_len * head_dim > (int64_t(1) << 31) || chunk_size * top_k > (int64_t(1) << 30))
    return csahca_set_unsupported("problem too large");
  if (workspace_bytes < csahca_csa_decode_workspace_size(batch, heads, head_dim, top_k, chunk_size))
    return csahca_set_arg_error("workspace too small");
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache)) &
      15)
    return csahca_set_arg_error("q, k_cache and v_cache must be 16-byte aligned");
  DecodeParams p;
  p.q = q;
  p.k = k_cache;
  p.v = v_cache;
  p.idx = chunk_indices;
  p.out = out;
  p.seq_len = int(seq_len);
  p.top_k = int(top_k);
  p.chunk = int(chunk_size);
  p.group = pick_group(rows, top_k);
  p.units = int((top_k + p.group - 1) / p.group);
  p.counters = static_cast<unsigned*>(workspace);
  p.partial = reinterpret_cast<float*>(static_cast<char*>(workspace) + align256(size_t(rows) * 4));
  p.scale_log2 = float(1.0 / sqrt(double(head_dim))) * kLog2e;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // The arrival counters must start at zero.  Kernels reset them on exit, but
  // the partials of an earlier call with fewer rows may lie where this call's
  // counters are, so they are cleared here (a few KB) instead of having the
  // combine wipe every partial it read.
  if (p.units > 1 && !(p.units <= kMaxClusterUnits && rows * p.units <= kClusterGridMax))
    CSAHCA_RETURN_IF_CUDA(cudaMemsetAsync(p.counters, 0, size_t(rows) * 4, s));
  switch (dtype) {
    case CSAHCA_DTYPE_BF16: return dispatch_decode_dim<__nv_bfloat16>(head_dim, p, rows, index_dtype, s);
    case CSAHCA_DTYPE_F16: return dispatch_decode_dim<__half>(head_dim, p, rows, index_dtype, s);
    case CSAHCA_DTYPE_F32: return dispatch_decode_dim<float>(head_dim, p, rows, index_dtype, s);
    default: return csahca_set_arg_error("unsupported dtype");
  }
}

// ---------------------------------------------------------------------------------------------------
// Allocation-free variant of csahca_csa_decode.
//
// Some callers cannot hand us a workspace: a serving process that reserved all
// of HBM for its KV cache at start-up and forbids later cudaMalloc calls, code
// that must not trigger cudaMalloc's implicit device synchronisation in a
// latency-critical loop, or a foreign-language binding with no device
// allocator of its own.  This entry point keeps its scratch (the row arrival
// counters and the split partials) in a fixed array owned by the library, so
// the caller passes only inputs and outputs and no call allocates anything.
//
// Limits and rules:
//   * the array is 8 MiB and exists on every GPU that loads the library, until
//     the process exits; problems needing more scratch are rejected;
//   * the first call on a device looks the array's device address up
//     (cudaGetSymbolAddress) with that device current; make that first call
//     before any stream capture.  The address is kept for the life of the
//     process, so after cudaDeviceReset (or any reset of the primary context)
//     the process must be restarted before calling this entry point again;
//   * all calls share the one array and it keeps the previous call's contents:
//     each call clears the counters it needs at zero on its own stream, and two
//     calls whose kernels overlap on the GPU (different streams, or different
//     host threads without ordering) race on it.
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;  // 8 MiB on every device that loads the library
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mu;
void* g_noalloc_ptr[64] = {};

// Device address of g_noalloc_scratch on the current device (looked up once per device;
// the name itself is only a host-side stand-in and must never reach a kernel).
int noalloc_scratch(void** out) {
  int dev = 0;
  CSAHCA_RETURN_IF_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return csahca_set_unsupported("device index out of range");
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    CSAHCA_RETURN_IF_CUDA(cudaGetSymbolAddress(&p, g_noalloc_scratch));
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return CSAHCA_OK;
}

}  // namespace

extern "C" size_t csahca_csa_decode_noalloc_max_scratch_bytes(void) { return kNoAllocScratchBytes; }

extern "C" int csahca_csa_decode_noalloc(const void* q, const void* k_cache, const void* v_cache,
                                         const void* chunk_indices, int index_dtype, int dtype, int64_t batch,
                                         int64_t heads, int64_t seq_len, int64_t head_dim, int64_t top_k,
                                         int64_t chunk_size, void* out, void* stream) {
  if (batch < 0 || heads < 0 || top_k < 0) return csahca_set_arg_error("sizes must be non-negative");
  const size_t need = csahca_csa_decode_workspace_size(batch, heads, head_dim, top_k, chunk_size);
  if (need > kNoAllocScratchBytes)
    return csahca_set_arg_error(
        "csahca_csa_decode_noalloc: this problem needs more scratch than the library's fixed 8 MiB buffer; "
        "use csahca_csa_decode with a caller-provided workspace");
  void* scratch = nullptr;
  const int st = noalloc_scratch(&scratch);
  if (st != CSAHCA_OK) return st;
  // csahca_csa_decode clears the counters it uses on the caller's stream, so
  // the scratch needs no preparation here.
  return csahca_csa_decode(q, k_cache, v_cache, chunk_indices, index_dtype, dtype, batch, heads, seq_len, head_dim,
                           top_k, chunk_size, out, scratch, kNoAllocScratchBytes, stream);
}
