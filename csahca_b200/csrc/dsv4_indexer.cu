// DSV4 compressed-slot indexer: per-query index scores and top-k on device
// (sm_100a, tcgen05).
//
// The reference takes the compressed (C4 / C128) slot indices of its DSV4
// decode from its caller (integrations/sglang_dsv4/csahca_sglang_dsv4_patch/
// patch.py:336-341) and lists an on-device indexer as future work
// (docs/dsv4_abi_status.md:111-119).  This kernel computes them with the
// published lightning-indexer score of DeepSeek-V3.2 (its technical report,
// "DeepSeek Sparse Attention"):
//     I[t, s] = sum_j  w[t, j] * ReLU(q[t, j, :] . k[s, :])
// over H indexer heads j (q: [H, D] per query, w: [H] per query, k: one D-dim
// indexer key per compressed slot s), then the top-k slots by I (largest
// first, equal scores by lower slot, -1 past the valid count).
//
// Score kernel: persistent, two CTAs per SM, each streaming an equal share
// of all queries' 128-slot tiles.  Per tile,
//   S^T[slot, head] = K[slot, :] . Q[head, :]       (M=128 slots, N=H heads, K=D)
// runs as tcgen05.mma kind::f16 (bf16 in, fp32 accumulate in TMEM); each of
// 128 epilogue threads owns one slot (TMEM lane) and reduces its row with the
// weights and the ReLU.  Four producer warps copy the key tiles (rows of D
// bf16, 256 B for D = 128) into 128-byte-swizzled shared memory with cp.async,
// two tiles in flight.  Top-k kernel: one 512-thread CTA per query, radix
// selection over the stored scores (topk.cuh).
#include <algorithm>

#include "common.cuh"
#include "sm100.cuh"
#include "topk.cuh"

namespace csahca {
namespace {

using namespace sm100;

constexpr int kIdxHeads = 64;   // indexer heads (MMA N)
constexpr int kIdxDim = 128;    // indexer head dim (MMA K total)
constexpr int kTile = 128;      // slots per tile (MMA M)
constexpr int kEpiWarps = 4;
constexpr int kProdWarp0 = 4;
constexpr int kProdWarps = 4;
constexpr int kMmaWarp = kProdWarp0 + kProdWarps;
constexpr int kThreads = (kMmaWarp + 1) * 32;  // 288

constexpr uint32_t kSubBytes = kTile * 128;                 // 16 KB: 128 slots x 64 dims
constexpr uint32_t kKTileBytes = 2 * kSubBytes;             // 32 KB
constexpr uint32_t kQSubBytes = kIdxHeads * 128;            // 8 KB: 64 heads x 64 dims
constexpr uint32_t kQBytes = 2 * kQSubBytes;                // 16 KB: one query's indexer q
constexpr uint32_t kOffQ = 0;                               // two Q buffers
constexpr uint32_t kOffK = kOffQ + 2 * kQBytes;             // two key tiles
constexpr uint32_t kOffBar = kOffK + 2 * kKTileBytes;
constexpr uint32_t kSmemBytes = kOffBar + 2048 + 1024;      // barriers and weights + alignment slack
constexpr uint32_t kTmemCols = 128;                         // two S^T buffers of 64 columns
constexpr uint32_t kIdesc = idesc_bf16_f32(kTile, kIdxHeads, 0, 0);

struct IdxBars {
  uint64_t k_full[2], k_empty[2], s_full[2], s_empty[2], q_empty[2];
  uint32_t tmem_base;
  int abort_flag;
  float w[kEpiWarps][kIdxHeads];  // each epilogue warp's copy of the current query's weights
};
static_assert(sizeof(IdxBars) <= 2048, "barrier region");

struct IndexerParams {
  const __nv_bfloat16* q;  // [Q, H, D]
  const float* w;          // [Q, H]
  const __nv_bfloat16* k;  // [Q, N, D]
  const int32_t* lens;     // [Q] valid slots (nullptr: all N)
  float* scores;           // [Q, N]
  int num_queries, n_keys;
  int tiles_per_query;     // ceil(n_keys / 128)
  int* err;
};

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ uint32_t sw128(int row, int c16) {
  return uint32_t(row) * 128u + (uint32_t(c16 ^ (row & 7)) << 4);
}

__device__ __forceinline__ int valid_slots(const IndexerParams& p, int q) {
  return p.lens != nullptr ? max(0, min(__ldg(p.lens + q), p.n_keys)) : p.n_keys;
}

// The tiles of all queries in one sequence, query-major: tile g is tile
// g % T of query g / T.  A tile at or past the query's valid count holds no
// work; every role skips it the same way.
struct TileRef {
  int q, t, n;
};
__device__ __forceinline__ bool tile_at(const IndexerParams& p, int g, TileRef& r) {
  r.q = g / p.tiles_per_query;
  r.t = g - r.q * p.tiles_per_query;
  r.n = valid_slots(p, r.q);
  return r.t * kTile < r.n;
}

// Persistent: CTA c streams the tiles [total*c/G, total*(c+1)/G) of the
// sequence, so every CTA gets the same number of tiles whatever the number of
// queries (no partial last wave).  A range crosses query boundaries: each
// query it touches is a "visit" v, whose q goes to Q buffer v % 2, loaded in
// the same cp.async group as the visit's first key tile (so that tile's
// k_full also publishes q); the MMA thread frees the buffer with a commit
// after the visit's last tile.
__global__ void __launch_bounds__(kThreads, 2) indexer_score_kernel(IndexerParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  IdxBars* bars = reinterpret_cast<IdxBars*>(smem + kOffBar);
  const uint32_t q_base = smem_u32(smem + kOffQ), k_base = smem_u32(smem + kOffK);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  volatile int* abort_flag = &bars->abort_flag;
  // total fits an int: the host requires num_queries * n_keys < 2^31.
  const long long total = (long long)p.num_queries * p.tiles_per_query;
  const int g0 = int(total * blockIdx.x / gridDim.x), g1 = int(total * (blockIdx.x + 1) / gridDim.x);

  if (threadIdx.x == 0) {
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bars->k_full[b], kProdWarps * 32);
      mbar_init(&bars->k_empty[b], 1);
      mbar_init(&bars->s_full[b], 1);
      mbar_init(&bars->s_empty[b], kEpiWarps * 32);
      mbar_init(&bars->q_empty[b], 1);
    }
    bars->abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kMmaWarp) tmem_alloc(&bars->tmem_base, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  bool failed = false;

  if (warp >= kProdWarp0 && warp < kProdWarp0 + kProdWarps) {
    // ------------------------------------------------------------ producers
    // Key tiles: 16 consecutive threads copy one 256-byte row (chunk c = pt %
    // 16, sub-tile c / 8, swizzled chunk c % 8), so every warp instruction
    // reads 512 contiguous bytes; rows past the valid count are zero-filled.
    // q: thread pt copies head pt / 2, half pt % 2.
    const int pt = threadIdx.x - kProdWarp0 * 32;
    const int c = pt & 15, r0 = pt >> 4;  // rows r0, r0 + 8, ..., r0 + 120
    const uint32_t c_off = uint32_t(c >> 3) * kSubBytes;
    bool ok = true;
    int i = 0, v = -1, prev_q = -1;
    for (int g = g0; g < g1 && ok; ++g) {
      TileRef tr;
      if (!tile_at(p, g, tr)) continue;
      const int b = i & 1;
      if (i >= 2) ok = mbar_wait(&bars->k_empty[b], ((i >> 1) - 1) & 1, abort_flag);
      if (!ok) break;
      if (tr.q != prev_q) {
        ++v;
        prev_q = tr.q;
        if (v >= 2) ok = mbar_wait(&bars->q_empty[v & 1], ((v >> 1) - 1) & 1, abort_flag);
        if (!ok) break;
        const int head = pt >> 1, half = pt & 1;
        const __nv_bfloat16* src = p.q + (size_t(tr.q) * kIdxHeads + head) * kIdxDim + half * 64;
        const uint32_t qd = q_base + uint32_t(v & 1) * kQBytes + uint32_t(half) * kQSubBytes;
#pragma unroll
        for (int cc = 0; cc < 8; ++cc) cp_async16(qd + sw128(head, cc), src + cc * 8);
      }
      const __nv_bfloat16* kq = p.k + size_t(tr.q) * p.n_keys * kIdxDim;
      const int tile_slot = tr.t * kTile;
      const uint32_t dst = k_base + uint32_t(b) * kKTileBytes + c_off;
#pragma unroll
      for (int j = 0; j < kTile / 8; ++j) {
        const int row = r0 + 8 * j;
        const uint32_t a = dst + sw128(row, c & 7);
        if (tile_slot + row < tr.n)
          cp_async16(a, kq + size_t(tile_slot + row) * kIdxDim + c * 8);
        else
          asm volatile("st.shared.v4.u32 [%0], {%1,%1,%1,%1};" ::"r"(a), "r"(0u) : "memory");
      }
      cp_async_commit();
      // The previous tile (with its visit's q) has landed: publish it.
      if (i > 0) {
        cp_async_wait<1>();
        fence_proxy_async_smem();
        mbar_arrive(&bars->k_full[(i - 1) & 1]);
      }
      ++i;
    }
    if (ok && i > 0) {
      cp_async_wait<0>();
      fence_proxy_async_smem();
      mbar_arrive(&bars->k_full[(i - 1) & 1]);
    }
    if (!ok) failed = true;
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      bool ok = true;
      int i = 0, v = -1, prev_q = -1;
      for (int g = g0; g < g1 && ok; ++g) {
        TileRef tr;
        if (!tile_at(p, g, tr)) continue;
        if (tr.q != prev_q) {
          ++v;
          prev_q = tr.q;
        }
        const int b = i & 1;
        ok = mbar_wait(&bars->k_full[b], (i >> 1) & 1, abort_flag);
        if (ok && i >= 2) ok = mbar_wait(&bars->s_empty[b], ((i >> 1) - 1) & 1, abort_flag);
        if (!ok) break;
        tc_fence_after();
        const uint32_t kt = k_base + uint32_t(b) * kKTileBytes;
        const uint32_t qt = q_base + uint32_t(v & 1) * kQBytes;
#pragma unroll
        for (int kk = 0; kk < kIdxDim / 16; ++kk) {
          const uint32_t sub = uint32_t(kk >> 2), off = uint32_t(kk & 3) * 32u;
          mma_bf16_ss(tmem + 64 * b, smem_desc_sw128(kt + sub * kSubBytes + off, 16, 1024),
                      smem_desc_sw128(qt + sub * kQSubBytes + off, 16, 1024), kIdesc, kk != 0);
        }
        mma_commit(&bars->s_full[b]);
        mma_commit(&bars->k_empty[b]);
        // Last tile of this visit (the next tile with work is another query's,
        // or there is none): its q buffer is free once these MMAs complete.
        int gn = g + 1;
        TileRef tn;
        while (gn < g1 && !tile_at(p, gn, tn)) ++gn;
        if (gn >= g1 || tn.q != tr.q) mma_commit(&bars->q_empty[v & 1]);
        ++i;
      }
      if (!ok) failed = true;
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue: one slot per thread
    // At each visit's first tile every epilogue warp copies the query's
    // weights into its own buffer (no barrier across warps).
    const int t = threadIdx.x;
    const uint32_t t_lane = tmem + (uint32_t(warp * 32) << 16);
    float* w = bars->w[warp];
    int i = 0, prev_q = -1;
    for (int g = g0; g < g1; ++g) {
      TileRef tr;
      if (!tile_at(p, g, tr)) continue;
      if (tr.q != prev_q) {
        prev_q = tr.q;
        __syncwarp();  // every lane is done with the previous query's weights
        w[lane] = __ldg(p.w + size_t(tr.q) * kIdxHeads + lane);
        w[lane + 32] = __ldg(p.w + size_t(tr.q) * kIdxHeads + lane + 32);
        __syncwarp();
      }
      const int b = i & 1;
      const bool ok = mbar_wait(&bars->s_full[b], (i >> 1) & 1, abort_flag);
      if (!ok) {
        failed = true;
        break;
      }
      tc_fence_after();
      float sv[32];
      float acc = 0.f;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        tmem_ld32(t_lane + 64 * b + 32 * h, sv);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < 32; ++c) acc = fmaf(w[32 * h + c], fmaxf(sv[c], 0.f), acc);
      }
      tc_fence_before();
      mbar_arrive(&bars->s_empty[b]);
      const int slot = tr.t * kTile + t;
      if (slot < tr.n) p.scores[size_t(tr.q) * p.n_keys + slot] = acc;
      ++i;
    }
  }
  if (failed) {
    *abort_flag = 1;
    report_device_error(p.err, kErrWaitTimeout);
  }
  tc_fence_before();
  asm volatile("barrier.sync 0;" ::: "memory");
  tc_fence_after();
  if (warp == kMmaWarp) {
    __syncwarp();
    tmem_dealloc(tmem, kTmemCols);
  }
}

constexpr int kTopkThreads = 512;  // two CTAs per SM: 256 queries in one wave
constexpr int kTopkMaxSlots = 49152;  // radix path: the scores of one query staged in shared memory

// Top-k of query blockIdx.x's valid scores (largest first, ties to the lower
// slot, -1 past the valid count), by radix selection: n_keys <= 49152 and
// top_k <= 512.  Dynamic shared memory: n_keys words rounded up to a multiple of 4.
__global__ void __launch_bounds__(kTopkThreads, 2) indexer_topk_kernel(IndexerParams p, int kout, int32_t* out) {
  extern __shared__ __align__(16) uint32_t s_sk[];
  __shared__ topk::RadixSmem<kTopkThreads> sm;
  const int qi = blockIdx.x;
  topk::block_topk_radix<kTopkThreads>(p.scores + size_t(qi) * p.n_keys, valid_slots(p, qi), kout,
                                       out + size_t(qi) * kout, s_sk, sm);
}

// Same result for any n_keys and top_k, one selection round per output (leaves
// the scores zero; the score kernel rewrites them on every call).
__global__ void __launch_bounds__(kTopkThreads) indexer_topk_rounds_kernel(IndexerParams p, int kout, int32_t* out) {
  __shared__ unsigned long long s_red[kTopkThreads / 32];
  const int qi = blockIdx.x;
  topk::block_topk<kTopkThreads>(p.scores + size_t(qi) * p.n_keys, valid_slots(p, qi), kout,
                                 out + size_t(qi) * kout, s_red);
}

}  // namespace
}  // namespace csahca

using namespace csahca;

extern "C" size_t csahca_dsv4_indexer_workspace_size(int64_t num_queries, int64_t n_keys) {
  if (num_queries <= 0 || n_keys <= 0) return 256;
  return ((size_t(num_queries) * size_t(n_keys) * 4 + 255) & ~size_t(255));
}

extern "C" int csahca_dsv4_indexer_topk(const void* q, const float* weights, const void* keys,
                                        const int32_t* key_lens, int64_t num_queries, int64_t heads,
                                        int64_t n_keys, int64_t head_dim, int64_t top_k, int32_t* out_indices,
                                        void* workspace, size_t workspace_bytes, void* stream) {
  if (heads != kIdxHeads || head_dim != kIdxDim)
    return csahca_set_unsupported("the indexer supports 64 heads of dim 128");
  if (num_queries < 0 || n_keys < 0 || top_k <= 0) return csahca_set_arg_error("sizes must be non-negative, top_k positive");
  const int64_t kout = std::min<int64_t>(top_k, n_keys);
  if (num_queries == 0 || kout == 0) return CSAHCA_OK;
  if (n_keys * num_queries >= (int64_t(1) << 31)) return csahca_set_unsupported("problem too large");
  if (workspace_bytes < csahca_dsv4_indexer_workspace_size(num_queries, n_keys))
    return csahca_set_arg_error("workspace too small");
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(keys) | reinterpret_cast<uintptr_t>(weights)) & 15)
    return csahca_set_arg_error("q, weights and keys must be 16-byte aligned");
  IndexerParams p;
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.w = weights;
  p.k = static_cast<const __nv_bfloat16*>(keys);
  p.lens = key_lens;
  p.scores = static_cast<float*>(workspace);
  p.num_queries = int(num_queries);
  p.n_keys = int(n_keys);
  p.err = csahca_device_error_ptr();
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  static bool configured[64] = {};
  static int sm_count[64] = {};
  int dev = 0;
  CSAHCA_RETURN_IF_CUDA(cudaGetDevice(&dev));
  if (dev < 64 && !configured[dev]) {
    CSAHCA_RETURN_IF_CUDA(cudaDeviceGetAttribute(&sm_count[dev], cudaDevAttrMultiProcessorCount, dev));
    CSAHCA_RETURN_IF_CUDA(
        cudaFuncSetAttribute(indexer_score_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kSmemBytes)));
    CSAHCA_RETURN_IF_CUDA(cudaFuncSetAttribute(indexer_topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               kTopkMaxSlots * 4));
    configured[dev] = true;
  }
  p.tiles_per_query = int((n_keys + kTile - 1) / kTile);
  int sms = dev < 64 ? sm_count[dev] : 0;
  if (sms <= 0) CSAHCA_RETURN_IF_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  // Persistent: two CTAs per SM (96 registers, ~99 KB of shared memory each),
  // each streaming an equal share of all queries' tiles.
  const int64_t total_tiles = num_queries * int64_t(p.tiles_per_query);
  const unsigned grid = unsigned(std::min<int64_t>(total_tiles, int64_t(2) * sms));
  indexer_score_kernel<<<grid, kThreads, kSmemBytes, s>>>(p);
  CSAHCA_RETURN_IF_CUDA(cudaGetLastError());
  if (n_keys <= kTopkMaxSlots && kout <= kTopkThreads)
    indexer_topk_kernel<<<unsigned(num_queries), kTopkThreads, size_t((n_keys + 3) & ~int64_t(3)) * 4, s>>>(
        p, int(kout), out_indices);  // whole 16-byte groups: the split pass reads four keys at a time
  else
    indexer_topk_rounds_kernel<<<unsigned(num_queries), kTopkThreads, 0, s>>>(p, int(kout), out_indices);
  CSAHCA_RETURN_IF_CUDA(cudaGetLastError());
  return CSAHCA_OK;
}
