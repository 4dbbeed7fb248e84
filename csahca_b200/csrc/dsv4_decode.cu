// DeepSeek-V4 paged-FP8 latent-cache decode on tcgen05 tensor cores (sm_100a).
//
// Replaces csrc/dsv4_attention.cu (dsv4_swa_decode_forward_kernel :337-437,
// dsv4_decode_tile_kernel :144-271, dsv4_decode_merge_kernel :273-335).
//
// Per query all H heads share one 512-dim latent per slot, with V = K, so the
// decode is two dense contractions per block of 128 slots:
//   S^T[slot, head] = K[slot, :] . Q[head, :]          (M=128 slots, N=64 heads, K=512 dims)
//   O^T[dim,  head] += V^T[dim, slot] . P^T[slot, head]  (M=128 dims x 4, N=64, K=128 slots)
// Both run as tcgen05.mma kind::f16 (bf16 operands, fp32 accumulators in TMEM).
// The dequantised K tile in shared memory is written once in the 128-byte
// swizzled layout and read as a K-major A operand by the first MMA and as an
// MN-major A operand (V^T) by the second, so V needs no second copy.
//
// Warp roles (416 threads, one CTA per SM, persistent over (query, head group)):
//   warps 0-3   softmax + epilogue; thread t owns TMEM lane t (= slot row t of
//               S^T, = dim row t of each O^T block)
//   warp 4      TMEM allocator + single-thread MMA issuer
//   warps 5-12  producers: gather the block's cache rows (576 data bytes + scale
//               bytes) straight into registers, dequantise e4m3 x 2^(s-127) to
//               bf16 exactly, and store them into the swizzled K tile; also load Q
//
// Shared memory (1024-byte aligned):
//   Q      64 heads x 512 dims bf16, 8 K-major sub-tiles of [64 rows x 128 B]     64 KB
//   Kpair  4 x [2 sub-tiles of 128 slot rows x 128 B] (dims 128m .. 128m+127)  128 KB
//   P      128 slot rows x 64 heads bf16 (MN-major B of the PV MMA); also the
//          epilogue staging buffer                                               16 KB
// TMEM (512 columns): O^T blocks at columns 0/64/128/192, S^T at column 256.
//
// Slot semantics follow the reference: main slots [0, clamp(topk_lengths[q]))
// then extra slots [0, clamp(extra_topk_lengths[q])) (dsv4_attention.cu:185-225);
// negative indices are skipped; the sink is a virtual token of score sink[h]
// and value 0 (dsv4_attention.cu:292-299).  Softmax uses a lazily updated
// per-head running max (re-based only when the block max exceeds it by 2^8).
//
// Every wait on an mbarrier is bounded; on a timeout the CTA raises an abort
// flag, records kErrWaitTimeout in the device error word and all roles leave.
#include <algorithm>

#include "common.cuh"
#include "sm100.cuh"

namespace csahca {
namespace {

using namespace sm100;

constexpr int kNope = 448;
constexpr int kRope = 64;
constexpr int kDim = kNope + kRope;           // 512
constexpr int kRowBytes = kNope + 2 * kRope;  // 576 data bytes per slot
constexpr int kScaleBytes = 8;                // 7 UE8M0 scales + 1 pad per slot
constexpr int kSlots = 128;                   // slots per block (MMA M of S^T)
constexpr int kHeads = 64;                    // heads per CTA item (MMA N)

constexpr int kSoftWarps = 4;
constexpr int kMmaWarp = 4;
constexpr int kProdWarp0 = 5;
constexpr int kProdWarps = 8;
constexpr int kProdThreads = kProdWarps * 32;
constexpr int kThreads = (kProdWarp0 + kProdWarps) * 32;  // 416

constexpr uint32_t kQBytes = kHeads * kDim * 2;     // 65536
constexpr uint32_t kSubTileBytes = kSlots * 128;    // 16384
constexpr uint32_t kPairBytes = 2 * kSubTileBytes;  // 32768
constexpr uint32_t kPBytes = kSlots * kHeads * 2;   // 16384
constexpr uint32_t kOffQ = 0;
constexpr uint32_t kOffK = kOffQ + kQBytes;
constexpr uint32_t kOffP = kOffK + 4 * kPairBytes;
constexpr uint32_t kOffBar = kOffP + kPBytes;
constexpr uint32_t kSmemBytes = kOffBar + 2048 + 1024;  // + barriers/scratch + alignment slack

constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemS = 256;

constexpr uint32_t kIdescQK = idesc_bf16_f32(128, kHeads, 0, 0);
constexpr uint32_t kIdescPV = idesc_bf16_f32(128, kHeads, 1, 1);

struct Dsv4Params {
  const void* q;
  const uint8_t* cache;
  const int32_t* idx;
  const int32_t* lens;
  const uint8_t* xcache;
  const int32_t* xidx;
  const int32_t* xlens;
  const float* sink;
  void* out;
  int* err;
  int64_t bpp, xbpp;
  int64_t capacity, xcapacity;  // slots addressable in each cache
  int page, xpage;
  int nmain, nextra;  // slots per query in each index list
  int num_queries, heads, groups, num_items;
  float scale_log2;
};

// Barrier / scratch area (after the P buffer).
struct Bars {
  uint64_t q_full, q_empty;
  uint64_t k_full[4], k_empty[4];
  uint64_t s_full, p_full, o_full, o_empty;
  uint32_t tmem_base;
  int abort_flag;
  int any_rescale;
  int pad;
  float red[kSoftWarps][kHeads];  // per-warp column partials
  float m_use[kHeads];            // running max (log2 domain) used for P
  float alpha[kHeads];            // O/l rescale factors of the current block
  float inv_l[kHeads];            // final normalisers
};
static_assert(sizeof(Bars) <= 2048, "barrier area too large");

// Valid-slot space of a query: main slots then extra slots.
struct SlotSpace {
  int len_main, len_extra;
  __device__ __forceinline__ int total() const { return len_main + len_extra; }
  __device__ __forceinline__ int blocks() const { return (total() + kSlots - 1) / kSlots; }
};

__device__ __forceinline__ SlotSpace slot_space(const Dsv4Params& p, int q) {
  SlotSpace s;
  const int lm = p.lens != nullptr ? p.lens[q] : p.nmain;
  s.len_main = max(0, min(lm, p.nmain));
  int lx = 0;
  if (p.xcache != nullptr && p.xidx != nullptr && p.nextra > 0) {
    lx = p.xlens != nullptr ? p.xlens[q] : p.nextra;
    lx = max(0, min(lx, p.nextra));
  }
  s.len_extra = lx;
  return s;
}

struct SlotRef {
  const uint8_t* data;   // 576-byte row
  const uint8_t* scale;  // 8 scale bytes
};

// Resolve slot `gs` of query q to its row in a cache; false for skipped slots.
__device__ __forceinline__ bool resolve_slot(const Dsv4Params& p, const SlotSpace& sp, int q, int gs, SlotRef& r,
                                             bool report) {
  if (gs >= sp.total()) return false;
  const bool main = gs < sp.len_main;
  const int loc = main ? __ldg(p.idx + size_t(q) * p.nmain + gs)
                       : __ldg(p.xidx + size_t(q) * p.nextra + (gs - sp.len_main));
  if (loc < 0) return false;
  const int64_t cap = main ? p.capacity : p.xcapacity;
  if (loc >= cap) {
    if (report) report_device_error(p.err, kErrSlotOutOfRange);
    return false;
  }
  const int page_size = main ? p.page : p.xpage;
  const int64_t bpp = main ? p.bpp : p.xbpp;
  const uint8_t* base = main ? p.cache : p.xcache;
  const int64_t page = loc / page_size;
  const int in_page = int(loc - page * page_size);
  const uint8_t* pb = base + page * bpp;
  r.data = pb + int64_t(in_page) * kRowBytes;
  r.scale = pb + int64_t(page_size) * kRowBytes + int64_t(in_page) * kScaleBytes;
  return true;
}

// 16 e4m3 bytes x 2^(s-127) -> 16 bf16 (exact).  The e4m3 exponent/mantissa
// bits are placed into a bf16 pattern (value x 2^-120, subnormals included) and
// one bf16x2 multiply by 2^(s-7) restores the magnitude and applies the scale.
__device__ __forceinline__ uint32_t e4m3x2_bits_to_bf16x2(uint32_t w, int hi) {
  const uint32_t mag = w & 0x7F7F7F7Fu;
  const uint32_t m = __byte_perm(mag, 0u, hi ? 0x4342u : 0x4140u) << 4;
  const uint32_t s = __byte_perm(w, 0u, hi ? 0x3424u : 0x1404u) & 0x80008000u;
  return m | s;
}

__device__ __forceinline__ uint32_t bf16x2_mul(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

__device__ __forceinline__ void dequant16(const uint4& raw, int scale_u8, uint4& lo, uint4& hi) {
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
  uint32_t o[8];
  if (scale_u8 <= 134) {
    const uint32_t f = uint32_t(scale_u8 + 120) << 7;  // bf16 2^(s-7)
    const uint32_t f2 = f | (f << 16);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      o[2 * i] = bf16x2_mul(e4m3x2_bits_to_bf16x2(w[i], 0), f2);
      o[2 * i + 1] = bf16x2_mul(e4m3x2_bits_to_bf16x2(w[i], 1), f2);
    }
  } else {
    // 2^(s-7) overflows bf16: apply 2^120 and 2^(s-127) separately.
    const uint32_t f1 = (uint32_t(247) << 7) | (uint32_t(247) << 23);
    const uint32_t e2 = uint32_t(scale_u8) << 7;
    const uint32_t f2 = e2 | (e2 << 16);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      o[2 * i] = bf16x2_mul(bf16x2_mul(e4m3x2_bits_to_bf16x2(w[i], 0), f1), f2);
      o[2 * i + 1] = bf16x2_mul(bf16x2_mul(e4m3x2_bits_to_bf16x2(w[i], 1), f1), f2);
    }
  }
  lo = make_uint4(o[0], o[1], o[2], o[3]);
  hi = make_uint4(o[4], o[5], o[6], o[7]);
}

// Byte offset of 16-byte chunk `c16` (0..7) of row `row` in a 128B-swizzled tile.
__device__ __forceinline__ uint32_t sw128(int row, int c16) {
  return uint32_t(row) * 128u + (uint32_t(c16 ^ (row & 7)) << 4);
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, const uint4& v) {
  asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

// Store chunk `c` (0..35: 28 nope chunks of 16 dims, then 8 rope chunks of 8
// dims) of slot row `slot` into the K pair tiles.
__device__ __forceinline__ void store_k_chunk(uint32_t k_base, int slot, int c, const uint4& raw, int scale_u8) {
  if (c < 28) {
    const int d0 = c * 16;           // first dim
    const int sub = d0 >> 6;         // 0..6
    const int c16 = (d0 & 63) >> 3;  // 0,2,4,6
    uint4 lo, hi;
    dequant16(raw, scale_u8, lo, hi);
    const uint32_t t = k_base + uint32_t(sub) * kSubTileBytes;
    st_shared_v4(t + sw128(slot, c16), lo);
    st_shared_v4(t + sw128(slot, c16 + 1), hi);
  } else {
    const uint32_t t = k_base + 7u * kSubTileBytes;
    st_shared_v4(t + sw128(slot, c - 28), raw);
  }
}

__device__ __forceinline__ void zero_k_chunk(uint32_t k_base, int slot, int c) {
  const uint4 z = make_uint4(0, 0, 0, 0);
  if (c < 28) {
    const int d0 = c * 16;
    const uint32_t t = k_base + uint32_t(d0 >> 6) * kSubTileBytes;
    st_shared_v4(t + sw128(slot, (d0 & 63) >> 3), z);
    st_shared_v4(t + sw128(slot, ((d0 & 63) >> 3) + 1), z);
  } else {
    st_shared_v4(k_base + 7u * kSubTileBytes + sw128(slot, c - 28), z);
  }
}

// 8 q elements -> 8 bf16 packed in a uint4.
template <typename QT>
__device__ __forceinline__ uint4 load_q8_bf16(const QT* src);
template <>
__device__ __forceinline__ uint4 load_q8_bf16<__nv_bfloat16>(const __nv_bfloat16* src) {
  return __ldg(reinterpret_cast<const uint4*>(src));
}
template <>
__device__ __forceinline__ uint4 load_q8_bf16<__half>(const __half* src) {
  const uint4 v = __ldg(reinterpret_cast<const uint4*>(src));
  const __half2* h = reinterpret_cast<const __half2*>(&v);
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(h[i]);
    const __nv_bfloat162 b = __floats2bfloat162_rn(f.x, f.y);
    o[i] = *reinterpret_cast<const uint32_t*>(&b);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}
template <>
__device__ __forceinline__ uint4 load_q8_bf16<float>(const float* src) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(src));
  const float4 b = __ldg(reinterpret_cast<const float4*>(src) + 1);
  const __nv_bfloat162 o0 = __floats2bfloat162_rn(a.x, a.y), o1 = __floats2bfloat162_rn(a.z, a.w);
  const __nv_bfloat162 o2 = __floats2bfloat162_rn(b.x, b.y), o3 = __floats2bfloat162_rn(b.z, b.w);
  return make_uint4(*reinterpret_cast<const uint32_t*>(&o0), *reinterpret_cast<const uint32_t*>(&o1),
                    *reinterpret_cast<const uint32_t*>(&o2), *reinterpret_cast<const uint32_t*>(&o3));
}

// Column reduce-scatter over the 32 lanes of a warp: v[64] per lane -> lane L
// returns the reduction of columns 2L and 2L+1 over all lanes.  Destroys v.
template <bool kMax>
__device__ __forceinline__ float2 warp_colreduce64(float* v) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int width = 32, bit = 16; bit >= 1; width >>= 1, bit >>= 1) {
    const bool upper = (lane & bit) != 0;
#pragma unroll
    for (int j = 0; j < width; ++j) {
      const float send = upper ? v[j] : v[j + width];
      const float keep = upper ? v[j + width] : v[j];
      const float recv = __shfl_xor_sync(0xffffffffu, send, bit);
      v[j] = kMax ? fmaxf(keep, recv) : keep + recv;
    }
  }
  return make_float2(v[0], v[1]);
}

// Barrier of the 128 softmax threads that also ANDs a predicate across them.
__device__ __forceinline__ bool soft_sync_and(bool ok) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, 1, 128, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(uint32_t(ok))
      : "memory");
  return r != 0;
}

template <typename QT>
__global__ void __launch_bounds__(kThreads, 1) dsv4_decode_kernel(Dsv4Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Bars* bars = reinterpret_cast<Bars*>(smem + kOffBar);
  const uint32_t q_base = smem_u32(smem + kOffQ);
  const uint32_t k_base = smem_u32(smem + kOffK);
  const uint32_t p_base = smem_u32(smem + kOffP);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  volatile int* abort_flag = &bars->abort_flag;

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, kProdThreads);
    mbar_init(&bars->q_empty, 1);
    for (int m = 0; m < 4; ++m) {
      mbar_init(&bars->k_full[m], kProdThreads);
      mbar_init(&bars->k_empty[m], 1);
    }
    mbar_init(&bars->s_full, 1);
    mbar_init(&bars->p_full, kSoftWarps * 32);
    mbar_init(&bars->o_full, 1);
    mbar_init(&bars->o_empty, kSoftWarps * 32);
    bars->abort_flag = 0;
    bars->any_rescale = 0;
    fence_mbar_init();
  }
  if (threadIdx.x < kHeads) bars->m_use[threadIdx.x] = -INFINITY;
  if (warp == kMmaWarp) tmem_alloc(&bars->tmem_base, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  bool failed = false;

  if (warp >= kProdWarp0) {
    // ------------------------------------------------------------ producers
    const int ptid = threadIdx.x - kProdWarp0 * 32;
    uint32_t items_done = 0, blocks_done = 0;
    for (int item = blockIdx.x; item < p.num_items; item += gridDim.x) {
      const int q = item / p.groups, hg = item - q * p.groups;
      const SlotSpace sp = slot_space(p, q);
      const int nblk = sp.blocks();
      if (nblk == 0) continue;
      if (items_done > 0 && !mbar_wait(&bars->q_empty, (items_done - 1) & 1, abort_flag)) goto prod_fail;
      {
        const QT* qsrc = static_cast<const QT*>(p.q) + size_t(q) * p.heads * kDim;
#pragma unroll 4
        for (int k = 0; k < 16; ++k) {
          const int i = ptid + kProdThreads * k;
          const int row = i >> 6, c = i & 63;
          const int head = hg * kHeads + row;
          uint4 v = make_uint4(0, 0, 0, 0);
          if (head < p.heads) v = load_q8_bf16<QT>(qsrc + size_t(head) * kDim + c * 8);
          st_shared_v4(q_base + uint32_t(c >> 3) * (kHeads * 128) + sw128(row, c & 7), v);
        }
      }
      fence_proxy_async_smem();
      mbar_arrive(&bars->q_full);

      for (int blk = 0; blk < nblk; ++blk, ++blocks_done) {
        // Gather this block's rows into registers (the loads overlap the MMAs
        // and softmax of the previous block).
        uint4 raw[18];
        int scl[18];
        {
          const int cA = ptid & 7;
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const int slot = (ptid >> 3) + 32 * k;
            SlotRef r;
            const bool ok = resolve_slot(p, sp, q, blk * kSlots + slot, r, true);
#pragma unroll
            for (int m = 0; m < 3; ++m) {
              const int c = 8 * m + cA;
              raw[m * 4 + k] = ok ? ldg_stream(r.data + c * 16) : make_uint4(0, 0, 0, 0);
              scl[m * 4 + k] = ok ? int(__ldg(r.scale + (c >> 2))) : -1;
            }
          }
#pragma unroll
          for (int k = 0; k < 6; ++k) {
            const int i = ptid + kProdThreads * k;
            const int slot = i / 12, c = 24 + i % 12;
            SlotRef r;
            const bool ok = resolve_slot(p, sp, q, blk * kSlots + slot, r, false);
            raw[12 + k] = ok ? ldg_stream(r.data + c * 16) : make_uint4(0, 0, 0, 0);
            scl[12 + k] = ok ? (c < 28 ? int(__ldg(r.scale + (c >> 2))) : 0) : -1;
          }
        }
        // Dequantise into the K pairs as they free up.
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          if (blocks_done > 0 && !mbar_wait(&bars->k_empty[m], (blocks_done - 1) & 1, abort_flag)) goto prod_fail;
          if (m < 3) {
            const int c = 8 * m + (ptid & 7);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const int slot = (ptid >> 3) + 32 * k;
              if (scl[m * 4 + k] >= 0)
                store_k_chunk(k_base, slot, c, raw[m * 4 + k], scl[m * 4 + k]);
              else
                zero_k_chunk(k_base, slot, c);
            }
          } else {
#pragma unroll
            for (int k = 0; k < 6; ++k) {
              const int i = ptid + kProdThreads * k;
              const int slot = i / 12, c = 24 + i % 12;
              if (scl[12 + k] >= 0)
                store_k_chunk(k_base, slot, c, raw[12 + k], scl[12 + k]);
              else
                zero_k_chunk(k_base, slot, c);
            }
          }
          fence_proxy_async_smem();
          mbar_arrive(&bars->k_full[m]);
        }
      }
      ++items_done;
    }
    if (false) {
    prod_fail:
      failed = true;
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      uint32_t items_done = 0, blocks_done = 0;
      for (int item = blockIdx.x; item < p.num_items; item += gridDim.x) {
        const int q = item / p.groups;
        const SlotSpace sp = slot_space(p, q);
        const int nblk = sp.blocks();
        if (nblk == 0) continue;
        if (!mbar_wait(&bars->q_full, items_done & 1, abort_flag)) goto mma_fail;
        for (int blk = 0; blk < nblk; ++blk, ++blocks_done) {
          const uint32_t par = blocks_done & 1;
          // S^T = K . Q^T over the 512 dims, pair by pair as the producers fill them.
          for (int m = 0; m < 4; ++m) {
            if (!mbar_wait(&bars->k_full[m], par, abort_flag)) goto mma_fail;
            tc_fence_after();
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int sub = 2 * m + h;
#pragma unroll
              for (int kk = 0; kk < 4; ++kk) {
                const uint64_t a = smem_desc_sw128(k_base + sub * kSubTileBytes + kk * 32, 16, 1024);
                const uint64_t b = smem_desc_sw128(q_base + sub * (kHeads * 128) + kk * 32, 16, 1024);
                mma_bf16_ss(tmem + kTmemS, a, b, kIdescQK, (sub | kk) != 0);
              }
            }
          }
          mma_commit(&bars->s_full);
          if (blk == nblk - 1) mma_commit(&bars->q_empty);
          if (!mbar_wait(&bars->p_full, par, abort_flag)) goto mma_fail;
          if (blk == 0 && items_done > 0 && !mbar_wait(&bars->o_empty, (items_done - 1) & 1, abort_flag))
            goto mma_fail;
          tc_fence_after();
          // O^T[m] += V^T[m] . P^T, V^T read MN-major from the same K pair tile.
          for (int m = 0; m < 4; ++m) {
#pragma unroll
            for (int kk = 0; kk < kSlots / 16; ++kk) {
              const uint64_t a = smem_desc_sw128(k_base + m * kPairBytes + kk * 2048, kSubTileBytes, 1024);
              const uint64_t b = smem_desc_sw128(p_base + kk * 2048, kSubTileBytes, 1024);
              mma_bf16_ss(tmem + 64 * m, a, b, kIdescPV, (blk | kk) != 0);
            }
            mma_commit(&bars->k_empty[m]);
          }
          if (blk == nblk - 1) mma_commit(&bars->o_full);
        }
        ++items_done;
      }
      if (false) {
      mma_fail:
        failed = true;
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ softmax + epilogue
    const int t = threadIdx.x;  // TMEM lane
    const uint32_t t_lane = tmem + (uint32_t(warp * 32) << 16);
    float lsum = 0.f;  // running sum of head t (threads 0..63)
    uint32_t items_done = 0, blocks_done = 0;
    constexpr int esz = sizeof(QT);
    for (int item = blockIdx.x; item < p.num_items; item += gridDim.x) {
      const int q = item / p.groups, hg = item - q * p.groups;
      const SlotSpace sp = slot_space(p, q);
      const int nblk = sp.blocks();
      const int hcount = min(kHeads, p.heads - hg * kHeads);
      uint8_t* out_q = static_cast<uint8_t*>(p.out) + (size_t(q) * p.heads + size_t(hg) * kHeads) * kDim * esz;
      if (nblk == 0) {
        const int nvec = hcount * kDim * esz / 16;
        for (int i = t; i < nvec; i += 128) reinterpret_cast<uint4*>(out_q)[i] = make_uint4(0, 0, 0, 0);
        continue;
      }
      for (int blk = 0; blk < nblk; ++blk, ++blocks_done) {
        const bool okw = mbar_wait(&bars->s_full, blocks_done & 1, abort_flag);
        if (!soft_sync_and(okw)) goto soft_fail;
        tc_fence_after();
        SlotRef r;
        const bool valid = resolve_slot(p, sp, q, blk * kSlots + t, r, false);
        float v[64];
        tmem_ld32(t_lane + kTmemS, v);
        tmem_ld32(t_lane + kTmemS + 32, v + 32);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < 64; ++c) v[c] = valid ? v[c] * p.scale_log2 : -INFINITY;
        {
          const float2 mx = warp_colreduce64<true>(v);
          bars->red[warp][2 * lane] = mx.x;
          bars->red[warp][2 * lane + 1] = mx.y;
        }
        named_bar_sync(1, 128);
        if (t < kHeads) {
          float bm = bars->red[0][t];
#pragma unroll
          for (int w = 1; w < kSoftWarps; ++w) bm = fmaxf(bm, bars->red[w][t]);
          const float mo = bars->m_use[t];
          float alpha = 1.f;
          if (mo == -INFINITY) {
            bars->m_use[t] = bm;
          } else if (bm > mo + 8.f) {
            alpha = exp2f(mo - bm);
            bars->m_use[t] = bm;
            bars->any_rescale = 1;
          }
          bars->alpha[t] = alpha;
          lsum *= alpha;
        }
        named_bar_sync(1, 128);
        // P^T row t = exp2(s - m_use), written as bf16 in the swizzled MN-major layout.
        tmem_ld32(t_lane + kTmemS, v);
        tmem_ld32(t_lane + kTmemS + 32, v + 32);
        tmem_wait_ld();
#pragma unroll
        for (int cc = 0; cc < 8; ++cc) {
          uint32_t w4[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int c = cc * 8 + 2 * j;
            const float m0 = bars->m_use[c], m1 = bars->m_use[c + 1];
            const float p0 = (valid && m0 != -INFINITY) ? exp2f(fmaf(v[c], p.scale_log2, -m0)) : 0.f;
            const float p1 = (valid && m1 != -INFINITY) ? exp2f(fmaf(v[c + 1], p.scale_log2, -m1)) : 0.f;
            v[c] = p0;
            v[c + 1] = p1;
            const __nv_bfloat162 b2 = __floats2bfloat162_rn(p0, p1);
            w4[j] = *reinterpret_cast<const uint32_t*>(&b2);
          }
          st_shared_v4(p_base + sw128(t, cc), make_uint4(w4[0], w4[1], w4[2], w4[3]));
        }
        {
          const float2 sm = warp_colreduce64<false>(v);
          bars->red[warp][2 * lane] = sm.x;  // the max partials were consumed before the last barrier
          bars->red[warp][2 * lane + 1] = sm.y;
        }
        const bool rescale = bars->any_rescale != 0;
        named_bar_sync(1, 128);
        if (t < kHeads) {
#pragma unroll
          for (int w = 0; w < kSoftWarps; ++w) lsum += bars->red[w][t];
        }
        if (rescale && blk > 0) {
          // Re-base the O^T accumulators of the heads whose max moved (columns = heads).
#pragma unroll 1
          for (int m = 0; m < 4; ++m)
#pragma unroll 1
            for (int hh = 0; hh < 2; ++hh) {
              tmem_ld32(t_lane + 64 * m + 32 * hh, v);
              tmem_wait_ld();
#pragma unroll
              for (int c = 0; c < 32; ++c) v[c] *= bars->alpha[32 * hh + c];
              tmem_st32(t_lane + 64 * m + 32 * hh, v);
            }
          tmem_wait_st();
        }
        named_bar_sync(1, 128);  // red / alpha / any_rescale consumed
        if (t == 0) bars->any_rescale = 0;
        fence_proxy_async_smem();
        tc_fence_before();
        mbar_arrive(&bars->p_full);
      }
      // -------------------------------------------------------------- epilogue
      {
        const bool okw = mbar_wait(&bars->o_full, items_done & 1, abort_flag);
        if (!soft_sync_and(okw)) goto soft_fail;
      }
      tc_fence_after();
      if (t < kHeads) {
        float total = lsum;
        const float mu = bars->m_use[t];
        if (p.sink != nullptr && hg * kHeads + t < p.heads) {
          const float sk = p.sink[hg * kHeads + t] * kLog2e;
          total += (mu == -INFINITY) ? (sk == -INFINITY ? 0.f : INFINITY) : exp2f(sk - mu);
        }
        bars->inv_l[t] = (total > 0.f && total != INFINITY) ? 1.f / total : 0.f;
        bars->m_use[t] = -INFINITY;
        lsum = 0.f;
      }
      named_bar_sync(1, 128);
      {
        constexpr int rows_per_pass = int(kPBytes / (128 * esz));  // heads staged per pass
        constexpr int vec_per_row = 128 * esz / 16;
        uint8_t* stage = smem + kOffP;
        float v[64];
        for (int m = 0; m < 4; ++m) {
          tmem_ld32(t_lane + 64 * m, v);
          tmem_ld32(t_lane + 64 * m + 32, v + 32);
          tmem_wait_ld();
          for (int h0 = 0; h0 < kHeads; h0 += rows_per_pass) {
#pragma unroll
            for (int c = 0; c < 64; ++c) {
              if (c >= h0 && c < h0 + rows_per_pass)
                reinterpret_cast<QT*>(stage)[(c - h0) * 128 + t] = Elem<QT>::from_f(v[c] * bars->inv_l[c]);
            }
            named_bar_sync(1, 128);
            const int rows = min(rows_per_pass, hcount - h0);
            for (int i = t; i < rows * vec_per_row; i += 128) {
              const int h = i / vec_per_row, vv = i - h * vec_per_row;
              uint4* dst = reinterpret_cast<uint4*>(out_q + (size_t(h0 + h) * kDim + 128 * m) * esz) + vv;
              *dst = reinterpret_cast<const uint4*>(stage)[h * vec_per_row + vv];
            }
            named_bar_sync(1, 128);
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&bars->o_empty);
      ++items_done;
    }
    if (false) {
    soft_fail:
      failed = true;
    }
  }
  if (failed) {
    *abort_flag = 1;
    report_device_error(p.err, kErrWaitTimeout);
  }
  // Threads may arrive here from divergent paths after a timeout: use the
  // non-aligned CTA barrier, then reconverge warp 4 before it frees TMEM.
  tc_fence_before();
  asm volatile("barrier.sync 0;" ::: "memory");
  tc_fence_after();
  if (warp == kMmaWarp) {
    __syncwarp();
    tmem_dealloc(tmem, kTmemCols);
  }
}

template <typename QT>
int launch_dsv4(const Dsv4Params& p, cudaStream_t stream) {
  static bool configured[64] = {};
  int dev = 0;
  CSAHCA_RETURN_IF_CUDA(cudaGetDevice(&dev));
  if (dev < 64 && !configured[dev]) {
    CSAHCA_RETURN_IF_CUDA(
        cudaFuncSetAttribute(dsv4_decode_kernel<QT>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kSmemBytes)));
    configured[dev] = true;
  }
  const int grid = std::min(p.num_items, csahca_num_sms());
  dsv4_decode_kernel<QT><<<grid, kThreads, kSmemBytes, stream>>>(p);
  CSAHCA_RETURN_IF_CUDA(cudaGetLastError());
  return CSAHCA_OK;
}

}  // namespace
}  // namespace csahca

using namespace csahca;

extern "C" int csahca_dsv4_decode(const void* q, int q_dtype, int64_t num_queries, int64_t heads, const uint8_t* cache,
                                  int64_t num_pages, int64_t bytes_per_page, int64_t page_size,
                                  const int32_t* token_indices, int64_t topk_slots, const int32_t* topk_lengths,
                                  const uint8_t* extra_cache, int64_t extra_num_pages, int64_t extra_bytes_per_page,
                                  int64_t extra_page_size, const int32_t* extra_token_indices,
                                  int64_t extra_topk_slots, const int32_t* extra_topk_lengths, const float* attn_sink,
                                  float softmax_scale, void* out, void* stream) {
  if (page_size <= 0) return csahca_set_arg_error("page_size must be positive");
  if (num_queries < 0 || heads < 0 || topk_slots < 0 || num_pages < 0)
    return csahca_set_arg_error("sizes must be non-negative");
  if (bytes_per_page < page_size * (kRowBytes + kScaleBytes))
    return csahca_set_arg_error("bytes_per_page is too small for DSV4 page layout");
  const bool has_extra =
      extra_cache != nullptr && extra_token_indices != nullptr && extra_topk_slots > 0 && extra_num_pages > 0;
  if (has_extra) {
    if (extra_page_size <= 0) return csahca_set_arg_error("extra_page_size must be positive");
    if (extra_bytes_per_page < extra_page_size * (kRowBytes + kScaleBytes))
      return csahca_set_arg_error("extra_bytes_per_page is too small for DSV4 page layout");
  }
  if (num_queries == 0 || heads == 0) return CSAHCA_OK;
  if ((reinterpret_cast<uintptr_t>(cache) | uintptr_t(bytes_per_page)) & 15)
    return csahca_set_unsupported("paged cache base and bytes_per_page must be multiples of 16 bytes");
  if (has_extra && ((reinterpret_cast<uintptr_t>(extra_cache) | uintptr_t(extra_bytes_per_page)) & 15))
    return csahca_set_unsupported("extra paged cache base and bytes_per_page must be multiples of 16 bytes");
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(out)) & 15)
    return csahca_set_arg_error("q and out must be 16-byte aligned");
  if (num_queries * heads > (int64_t(1) << 30)) return csahca_set_unsupported("problem too large");

  Dsv4Params p;
  p.q = q;
  p.cache = cache;
  p.idx = token_indices;
  p.lens = topk_lengths;
  p.xcache = has_extra ? extra_cache : nullptr;
  p.xidx = has_extra ? extra_token_indices : nullptr;
  p.xlens = has_extra ? extra_topk_lengths : nullptr;
  p.sink = attn_sink;
  p.out = out;
  p.err = csahca_device_error_ptr();
  p.bpp = bytes_per_page;
  p.xbpp = has_extra ? extra_bytes_per_page : 0;
  p.capacity = std::min<int64_t>(num_pages * page_size, int64_t(1) << 31);
  p.xcapacity = has_extra ? std::min<int64_t>(extra_num_pages * extra_page_size, int64_t(1) << 31) : 0;
  p.page = int(page_size);
  p.xpage = has_extra ? int(extra_page_size) : 1;
  p.nmain = int(topk_slots);
  p.nextra = has_extra ? int(extra_topk_slots) : 0;
  p.num_queries = int(num_queries);
  p.heads = int(heads);
  p.groups = int((heads + kHeads - 1) / kHeads);
  p.num_items = p.num_queries * p.groups;
  p.scale_log2 = softmax_scale * kLog2e;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (q_dtype) {
    case CSAHCA_DTYPE_BF16: return launch_dsv4<__nv_bfloat16>(p, s);
    case CSAHCA_DTYPE_F16: return launch_dsv4<__half>(p, s);
    case CSAHCA_DTYPE_F32: return launch_dsv4<float>(p, s);
    default: return csahca_set_arg_error("unsupported q dtype");
  }
}
