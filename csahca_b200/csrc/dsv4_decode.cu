// DeepSeek-V4 paged-FP8 latent-cache decode on tcgen05 tensor cores (sm_100a).
//
// Replaces csrc/dsv4_attention.cu (dsv4_swa_decode_forward_kernel :337-437,
// dsv4_decode_tile_kernel :144-271, dsv4_decode_merge_kernel :273-335).
//
// Per query all H heads share one 512-dim latent per slot, with V = K, so the
// decode is two dense contractions per block of 64 slots:
//   S^T[slot, head] = K[slot, :] . Q[head, :]          (K = 512 dims)
//   O^T[dim,  head] += V^T[dim, slot] . P^T[slot, head]  (M=128 dims x 4, N=64, K=64 slots)
// The first runs as M=128 x N=128 MMAs that stack the two 256-dim halves of
// K (rows) and of Q (columns), 16 per block; the diagonal quadrants of the
// result are the two halves' partial scores, added by the softmax warps.
// Both run as tcgen05.mma kind::f16 (bf16 operands, fp32 accumulators in TMEM).
// The dequantised K tile in shared memory is written once in the 128-byte
// swizzled layout and read as a K-major A operand by the first MMA and as an
// MN-major A operand (V^T) by the second, so V needs no second copy.
//
// Warp roles (512 threads, one CTA per SM, persistent over (query, head group)):
//   warps 0-3   softmax + epilogue (TMEM lanes 32w..32w+31)
//   warp 4      TMEM allocator + single-thread, event-driven MMA issuer
//   warps 5-12  producers: 4 threads per slot row load its 576 data bytes into
//               registers a block ahead, dequantise e4m3 x 2^(s-127) to bf16
//               exactly and store them into the swizzled K tile
//   warps 13-14 slot-table resolvers (index -> row address, scale bytes, L2
//               prefetch), up to kTabBufs blocks ahead
//   warp 15     Q loader
//
// Shared memory (1024-byte aligned):
//   Q      64 heads x 512 dims bf16, 8 K-major sub-tiles of [64 rows x 128 B]     64 KB
//   K      2 buffers x 8 sub-tiles of [64 slot rows x 128 B]                     128 KB
//          (sub-tiles in the order 0,4,1,5,2,6,3,7 in both Q and K)
//   P      2 buffers x 64 slot rows x 64 heads bf16 (MN-major B of the PV MMA)    16 KB
//   barriers, softmax scratch, slot tables, score exchange                      ~14 KB
// TMEM (512 columns): O^T blocks at columns 0/64/128/192, S buffers (128
// columns each) at 256/384.
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
#include <type_traits>

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
constexpr int kSlots = 64;                    // slots per block (MMA M of S^T)
constexpr int kHeads = 64;                    // heads per CTA item (MMA N)

constexpr int kSoftWarps = 4;
constexpr int kMmaWarp = 4;
constexpr int kProdWarp0 = 5;   // dequantising producers: 4 threads per slot row
constexpr int kProdWarps = 8;
constexpr int kProdThreads = kProdWarps * 32;  // 256 = kSlots x 4
constexpr int kResWarp0 = kProdWarp0 + kProdWarps;  // slot-table resolvers: one thread per slot
constexpr int kResWarps = 2;
constexpr int kResThreads = kResWarps * 32;  // 64 = kSlots
constexpr int kQWarp = kResWarp0 + kResWarps;  // Q loader
constexpr int kThreads = (kQWarp + 1) * 32;    // 512 (4 warps per sub-partition, 128 registers)

constexpr int kKBufs = 2;                             // K tiles (and S / P buffers) in flight
constexpr uint32_t kQBytes = kHeads * kDim * 2;      // 65536
constexpr uint32_t kSubTileBytes = kSlots * 128;     // 8192: 64 slot rows x 64 dims bf16
constexpr uint32_t kPairBytes = 2 * kSubTileBytes;   // 16384: dims 128m .. 128m+127
constexpr uint32_t kBlockBytes = 4 * kPairBytes;     // 65536: one block's K tile
constexpr uint32_t kPBytes = kSlots * kHeads * 2;    // 8192 per buffer
constexpr uint32_t kOffQ = 0;
constexpr uint32_t kOffK = kOffQ + kQBytes;
constexpr uint32_t kOffP = kOffK + kKBufs * kBlockBytes;
constexpr uint32_t kOffBar = kOffP + kKBufs * kPBytes;
constexpr int kTabBufs = 4;                                  // slot tables in flight (see resolvers)
constexpr uint32_t kBarBytes = 2304;
constexpr uint32_t kOffTab = kOffBar + kBarBytes;
constexpr uint32_t kTabBytes = kTabBufs * kSlots * 16;      // 4 KB
// Score exchange between the two softmax warps of a slot row: 64 slots x 32
// fp32 partial scores.
constexpr uint32_t kOffX = kOffTab + kTabBytes;
constexpr uint32_t kXBytes = kSlots * 32 * 4;                // 8 KB
constexpr uint32_t kSmemBytes = kOffX + kXBytes + 1024;      // + alignment slack
static_assert(kSmemBytes <= 232448, "shared memory budget");

constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemS = 256;  // S buffers (128 columns each) at columns 256 and 384

// Optional stage timestamps of CTA 0 (build with -DCSAHCA_DSV4_TRACE; diagnosis only).
#ifdef CSAHCA_DSV4_TRACE
__device__ long long g_dsv4_trace[2 * 8 * 16];
#define DSV4_TRACE(item_no, blk, ev)                                                      \
  do {                                                                                    \
    if (blockIdx.x == 0 && (item_no) < 2 && (blk) < 8)                                    \
      g_dsv4_trace[((item_no) * 8 + (blk)) * 16 + (ev)] = clock64();                      \
  } while (0)
#else
#define DSV4_TRACE(item_no, blk, ev) \
  do {                               \
  } while (0)
#endif

constexpr uint32_t kIdescQK = idesc_bf16_f32(2 * kSlots, 2 * kHeads, 0, 0);

// K and Q tiles keep their eight 64-dim sub-tiles in the order 0,4,1,5,2,6,3,7,
// so sub-tiles k and k+4 are adjacent: one M=128 operand holds the same 64
// slots for dims 64k.. (rows 0-63) and 64(k+4).. (rows 64-127), one N=128
// operand Q's 64 heads for the same two dim ranges.  The split-K MMA then adds
// two useful quadrants per instruction (rows 0-63 x columns 0-63 and rows
// 64-127 x columns 64-127), and every V^T block (dims 128m.., sub-tiles 2m and
// 2m+1) lies at a fixed 16 KB stride.
__host__ __device__ constexpr uint32_t sub_pos(int k) { return uint32_t(k < 4 ? 2 * k : 2 * (k - 4) + 1); }
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
  float* lse;  // non-null: split-KV partial mode (fp32 o normalised by its own sum, lse in log2 units, no sink)
  int* err;
  int64_t bpp, xbpp;
  int64_t capacity, xcapacity;  // slots addressable in each cache
  int page, xpage;
  int nmain, nextra;  // slots per query in each index list
  int num_queries, heads, groups, num_items;
  // Slot-list sharding (split-KV): this launch decodes shards split0 ..
  // split0+splits-1 of split_total equal ranges of every query's main and
  // extra slot lists; work row qs = s * num_queries + q (s local), and the
  // outputs are indexed by qs.  splits = split_total = 1 for a plain decode.
  int splits, split0, split_total;
  float scale_log2;
};

// Barrier / scratch area (after the P buffer).
struct Bars {
  uint64_t q_full, q_empty;
  uint64_t k_full[kKBufs][4], k_empty[kKBufs][4];
  uint64_t s_full[kKBufs], p_full[kKBufs];
  uint64_t o_full, o_empty, pv_done;
  uint64_t tab_full[kTabBufs], tab_empty[kTabBufs];
  uint32_t tmem_base;
  int abort_flag;
  float red[kSoftWarps][kHeads];  // per-warp column partials
  float m_use[kHeads];            // running max (log2 domain) used for P
  float alpha[kHeads];            // O/l rescale factors of the current block
  float inv_l[kHeads];            // final normalisers
};
static_assert(sizeof(Bars) <= kBarBytes, "barrier area too large");

// Valid-slot space of one work row (a query, or one shard of a query's slot
// lists): main slots then extra slots, starting at main_off / extra_off of the
// query's index lists.
struct SlotSpace {
  int q;  // the query
  int len_main, len_extra, main_off, extra_off;
  __device__ __forceinline__ int total() const { return len_main + len_extra; }
  __device__ __forceinline__ int blocks() const { return (total() + kSlots - 1) / kSlots; }
};

__device__ __forceinline__ SlotSpace slot_space(const Dsv4Params& p, int qs) {
  SlotSpace s;
  s.q = qs % p.num_queries;
  const int sg = p.split0 + qs / p.num_queries;
  const int lm = max(0, min(p.lens != nullptr ? p.lens[s.q] : p.nmain, p.nmain));
  const int lo_m = int((int64_t(p.nmain) * sg) / p.split_total);
  const int hi_m = int((int64_t(p.nmain) * (sg + 1)) / p.split_total);
  s.main_off = lo_m;
  s.len_main = max(0, min(lm - lo_m, hi_m - lo_m));
  s.len_extra = 0;
  s.extra_off = 0;
  if (p.xcache != nullptr && p.xidx != nullptr && p.nextra > 0) {
    const int lx = max(0, min(p.xlens != nullptr ? p.xlens[s.q] : p.nextra, p.nextra));
    const int lo_x = int((int64_t(p.nextra) * sg) / p.split_total);
    const int hi_x = int((int64_t(p.nextra) * (sg + 1)) / p.split_total);
    s.extra_off = lo_x;
    s.len_extra = max(0, min(lx - lo_x, hi_x - lo_x));
  }
  return s;
}

// One resolved slot of a block: its 576-byte row (nullptr = skipped) and the
// address of its 8 scale bytes.  The producers load the scale bytes together
// with the row, so a table costs the resolvers no dependent load.
struct SlotEntry {
  const uint8_t* row;
  const uint2* scales;
};
static_assert(sizeof(SlotEntry) == 16, "slot table entry is 16 bytes");

// Slot resolution in two steps for the resolver pipeline: slot_loc() issues the
// index load, finish_slot() turns the index into the row and scale addresses
// (and prefetches the row into L2); the caller stores the entry one step later.
struct PendingSlot {
  int loc;
  bool main;
};

__device__ __forceinline__ PendingSlot slot_loc(const Dsv4Params& p, const SlotSpace& sp, int blk, int tid) {
  const int q = sp.q;
  PendingSlot r;
  r.loc = -1;
  r.main = true;
  const int gs = blk * kSlots + tid;
  if (tid >= 0 && tid < kSlots && gs < sp.total()) {
    r.main = gs < sp.len_main;
    r.loc = r.main ? __ldg(p.idx + size_t(q) * p.nmain + sp.main_off + gs)
                   : __ldg(p.xidx + size_t(q) * p.nextra + sp.extra_off + (gs - sp.len_main));
  }
  return r;
}

__device__ __forceinline__ SlotEntry finish_slot(const Dsv4Params& p, const PendingSlot& ps) {
  SlotEntry e;
  e.row = nullptr;
  e.scales = nullptr;
  const int64_t cap = ps.main ? p.capacity : p.xcapacity;
  if (ps.loc >= 0 && ps.loc < cap) {
    const unsigned page_size = unsigned(ps.main ? p.page : p.xpage);
    const unsigned page = unsigned(ps.loc) / page_size;
    const unsigned in_page = unsigned(ps.loc) - page * page_size;
    const uint8_t* pb = (ps.main ? p.cache : p.xcache) + int64_t(page) * (ps.main ? p.bpp : p.xbpp);
    e.row = pb + int64_t(in_page) * kRowBytes;
    e.scales = reinterpret_cast<const uint2*>(pb + int64_t(page_size) * kRowBytes + int64_t(in_page) * kScaleBytes);
    // Pull the row into L2 now (two blocks ahead of its register loads): the
    // gather is latency-bound, and this keeps many rows in flight without
    // registers or shared memory.
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(e.row), "r"(uint32_t(kRowBytes)) : "memory");
  } else if (ps.loc >= cap) {
    report_device_error(p.err, kErrSlotOutOfRange);
  }
  return e;
}

__device__ __forceinline__ int scale_byte(const uint2& s, int group) {
  const uint32_t w = group < 4 ? s.x : s.y;
  return int((w >> (8 * (group & 3))) & 0xFFu);
}

// Next (item, block) this CTA works on after (item, blk); false when none is left.
__device__ __forceinline__ bool next_work(const Dsv4Params& p, int item, int blk, int nblk, int& nitem, int& nblk_out,
                                          SlotSpace& nsp) {
  if (blk + 1 < nblk) {
    nitem = item;
    nblk_out = blk + 1;
    nsp = slot_space(p, item / p.groups);
    return true;
  }
  for (int it = item + gridDim.x; it < p.num_items; it += gridDim.x) {
    nsp = slot_space(p, it / p.groups);
    if (nsp.blocks() > 0) {
      nitem = it;
      nblk_out = 0;
      return true;
    }
  }
  return false;
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// 16 e4m3 bytes x 2^(s-127) -> 16 bf16 (exact).  Each e4m3 byte's magnitude
// bits are moved to bits 4..10 of a bf16 lane and its sign to bit 15, which
// reads as value x 2^-120 (e4m3 subnormals included); one bf16x2 multiply by
// 2^(s-7) then restores the magnitude and applies the scale.
__device__ __forceinline__ uint32_t bf16x2_mul(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// Bytes 2k, 2k+1 of a word (magnitudes in `mag`, signs in `sgn`) -> bf16x2 bits.
template <int K>
__device__ __forceinline__ uint32_t e4m3_pair_bits(uint32_t mag, uint32_t sgn) {
  const uint32_t m = __byte_perm(mag, 0u, K == 0 ? 0x4140u : 0x4342u);  // bytes to lane bits 0..7
  const uint32_t sg = __byte_perm(sgn, 0u, K == 0 ? 0x1404u : 0x3424u);  // signs to lane bit 15
  return (m << 4) + sg;
}

__device__ __forceinline__ void dequant16(const uint4& raw, int scale_u8, uint4& lo, uint4& hi) {
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
  uint32_t o[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t mag = w[i] & 0x7F7F7F7Fu, sgn = w[i] & 0x80808080u;
    o[2 * i] = e4m3_pair_bits<0>(mag, sgn);
    o[2 * i + 1] = e4m3_pair_bits<1>(mag, sgn);
  }
  if (scale_u8 <= 134) {
    const uint32_t f = uint32_t(scale_u8 + 120) << 7;  // bf16 2^(s-7)
    const uint32_t f2 = f | (f << 16);
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = bf16x2_mul(o[i], f2);
  } else {
    // 2^(s-7) overflows bf16: apply 2^120 and 2^(s-127) separately.
    const uint32_t f1 = (uint32_t(247) << 7) | (uint32_t(247) << 23);
    const uint32_t e2 = uint32_t(scale_u8) << 7;
    const uint32_t f2 = e2 | (e2 << 16);
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = bf16x2_mul(bf16x2_mul(o[i], f1), f2);
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

// Column reduce-scatter over a full warp: v[32] per lane -> lane L returns the
// max (or sum) of column L over the 32 lanes.  Destroys v.
template <bool kMax>
__device__ __forceinline__ float warp_colreduce32(float* v) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int width = 16; width >= 1; width >>= 1) {
    const bool upper = (lane & width) != 0;
#pragma unroll
    for (int j = 0; j < width; ++j) {
      const float send = upper ? v[j] : v[j + width];
      const float keep = upper ? v[j + width] : v[j];
      const float recv = __shfl_xor_sync(0xffffffffu, send, width);
      v[j] = kMax ? fmaxf(keep, recv) : keep + recv;
    }
  }
  return v[0];
}

// Named barrier `id` over `n` threads that also ANDs a predicate across them, so
// a group leaves together when any member's bounded wait gave up.
__device__ __forceinline__ bool group_sync_and(int id, int n, bool ok) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %3, 0;\n\t"
      "bar.red.and.pred q, %1, %2, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(id), "r"(n), "r"(uint32_t(ok))
      : "memory");
  return r != 0;
}
__device__ __forceinline__ bool soft_sync_and(bool ok) { return group_sync_and(1, 128, ok); }

__device__ __forceinline__ bool group_sync_or(int id, int n, bool x) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %3, 0;\n\t"
      "bar.red.or.pred q, %1, %2, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(id), "r"(n), "r"(uint32_t(x))
      : "memory");
  return r != 0;
}

// 2^x with the hardware approximation (about 2 ulp; inputs here are <= 8).
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// log2(x) and 1/x with the hardware approximations (relative error ~2^-22),
// used once per query for the normalisers.
__device__ __forceinline__ float fast_log2(float x) {
  float y;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float fast_rcp(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Two adjacent output elements (4 or 8 bytes, aligned) in one store.
__device__ __forceinline__ void store_pair(__nv_bfloat16* dst, float a, float b) {
  *reinterpret_cast<__nv_bfloat162*>(dst) = __floats2bfloat162_rn(a, b);
}
__device__ __forceinline__ void store_pair(__half* dst, float a, float b) {
  *reinterpret_cast<__half2*>(dst) = __floats2half2_rn(a, b);
}
__device__ __forceinline__ void store_pair(float* dst, float a, float b) {
  *reinterpret_cast<float2*>(dst) = make_float2(a, b);
}

// Position in the CTA's sequence of (item, block) work units; empty items are skipped.
struct Cursor {
  bool valid;
  int item, blk, nblk;
  SlotSpace sp;
};

__device__ __forceinline__ Cursor first_cursor(const Dsv4Params& p) {
  Cursor c;
  c.valid = false;
  for (int it = blockIdx.x; it < p.num_items; it += gridDim.x) {
    const SlotSpace sp = slot_space(p, it / p.groups);
    if (sp.blocks() > 0) {
      c.valid = true;
      c.item = it;
      c.blk = 0;
      c.nblk = sp.blocks();
      c.sp = sp;
      break;
    }
  }
  return c;
}

__device__ __forceinline__ Cursor next_cursor(const Dsv4Params& p, const Cursor& c) {
  Cursor n = c;
  if (!c.valid) return n;
  if (c.blk + 1 < c.nblk) {  // same item: no memory access
    n.blk = c.blk + 1;
    return n;
  }
  n.valid = false;
  int ni, nb;
  SlotSpace nsp;
  if (next_work(p, c.item, c.blk, c.nblk, ni, nb, nsp)) {
    n.valid = true;
    n.item = ni;
    n.blk = nb;
    n.nblk = nsp.blocks();
    n.sp = nsp;
  }
  return n;
}

template <typename QT>
__global__ void __launch_bounds__(kThreads, 1) dsv4_decode_kernel(Dsv4Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Bars* bars = reinterpret_cast<Bars*>(smem + kOffBar);
  const uint32_t q_base = smem_u32(smem + kOffQ);
  const uint32_t k_base = smem_u32(smem + kOffK);
  const uint32_t p_base = smem_u32(smem + kOffP);
  SlotEntry* tabs = reinterpret_cast<SlotEntry*>(smem + kOffTab);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  volatile int* abort_flag = &bars->abort_flag;

  if (threadIdx.x == 0) DSV4_TRACE(0, 0, 1);  // kernel entry (exit: item 1, block 0)
  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 32);
    mbar_init(&bars->q_empty, 1);
    for (int b = 0; b < kKBufs; ++b) {
      for (int m = 0; m < 4; ++m) {
        mbar_init(&bars->k_full[b][m], kProdThreads);
        mbar_init(&bars->k_empty[b][m], 1);
      }
      mbar_init(&bars->s_full[b], 1);
      mbar_init(&bars->p_full[b], kSoftWarps * 32);
    }
    mbar_init(&bars->o_full, 1);
    mbar_init(&bars->o_empty, kSoftWarps * 32);
    mbar_init(&bars->pv_done, 1);
    for (int t = 0; t < kTabBufs; ++t) {
      mbar_init(&bars->tab_full[t], kResThreads);
      mbar_init(&bars->tab_empty[t], kProdThreads + kSoftWarps * 32);
    }
    bars->abort_flag = 0;
    fence_mbar_init();
  }
  if (threadIdx.x < kHeads) bars->m_use[threadIdx.x] = -INFINITY;
  if (warp == kMmaWarp) tmem_alloc(&bars->tmem_base, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  bool failed = false;

  if (warp >= kProdWarp0 && warp < kProdWarp0 + kProdWarps) {
    // ------------------------------------------------------------ producers
    // Thread (slot s, quarter r) owns 16-byte chunks c = 4i + r (i = 0..8) of
    // slot row s in every block: chunks 0..27 are e4m3 (chunk 4i + r is dims
    // 64i + 16r .. +15, scale group i, K sub-tile i), chunks 28..35 are the
    // bf16 rope dims (K sub-tile 7).  The shared-memory offsets are therefore
    // fixed per thread, and four threads read 64 contiguous bytes of a row.
    // Sub-tile k is stored at position sub_pos(k) of the tile.  Block g goes to
    // K buffer g%2, in four groups m = {sub-tiles m, m+4} (the operands of one
    // QK group).  One register set rotates group by group: right after the
    // stores of group m of block g, the loads of group m of block g+1 go out
    // into the same registers, so every row load has a block period to land.
    // Invalid slots load nothing and store zeros.
    const int pt = threadIdx.x - kProdWarp0 * 32;
    const int s = pt >> 2, r = pt & 3;
    const uint32_t x7 = uint32_t(s & 7), row_off = uint32_t(s) * 128u;
    const uint32_t off_lo = row_off + ((uint32_t(2 * r) ^ x7) << 4);
    const uint32_t off_hi = row_off + ((uint32_t(2 * r + 1) ^ x7) << 4);
    const uint32_t off_r0 = sub_pos(7) * kSubTileBytes + row_off + ((uint32_t(r) ^ x7) << 4);
    const uint32_t off_r1 = sub_pos(7) * kSubTileBytes + row_off + ((uint32_t(r + 4) ^ x7) << 4);
    uint4 raw[9];
    uint2 sc = make_uint2(0, 0);
    bool ok = true;
    uint32_t g = 0;
    Cursor cur = first_cursor(p);
#define DSV4_LOAD(I, C)                                                                        \
  raw[I] = rowp != nullptr ? ldg_stream(rowp + (C) * 16) : make_uint4(0, 0, 0, 0)
#define DSV4_LOAD_PAIR(M)                      \
  do {                                         \
    if ((M) < 3) {                             \
      DSV4_LOAD((M), 4 * (M) + r);             \
      DSV4_LOAD((M) + 4, 4 * (M) + 16 + r);    \
    } else {                                   \
      DSV4_LOAD(3, 12 + r);                    \
      DSV4_LOAD(7, 28 + r);                    \
      DSV4_LOAD(8, 32 + r);                    \
    }                                          \
  } while (0)
#define DSV4_STORE_NOPE(I)                                         \
  do {                                                             \
    uint4 lo, hi;                                                  \
    dequant16(raw[I], scale_byte(sc, I), lo, hi);                  \
    st_shared_v4(kbuf + sub_pos(I) * kSubTileBytes + off_lo, lo);  \
    st_shared_v4(kbuf + sub_pos(I) * kSubTileBytes + off_hi, hi);  \
  } while (0)
    if (cur.valid) {
      ok = mbar_wait(&bars->tab_full[0], 0, abort_flag);
      const SlotEntry e = tabs[s];
      mbar_arrive(&bars->tab_empty[0]);
      const uint8_t* rowp = e.row;
      sc = e.row != nullptr ? __ldg(e.scales) : make_uint2(0, 0);
      DSV4_LOAD_PAIR(0);
      DSV4_LOAD_PAIR(1);
      DSV4_LOAD_PAIR(2);
      DSV4_LOAD_PAIR(3);
    }
#ifdef CSAHCA_DSV4_TRACE
    uint32_t p_items = 0;
#endif
    while (ok && cur.valid) {
#ifdef CSAHCA_DSV4_TRACE
      if (pt == 0 && p_items == 0 && cur.blk < 8) DSV4_TRACE(0, cur.blk, 0);
#endif
      const Cursor nxt = next_cursor(p, cur);
      const uint8_t* rowp = nullptr;
      uint2 sc_next = make_uint2(0, 0);
      if (nxt.valid) {
        const int tb = (g + 1) % kTabBufs;
        ok = mbar_wait(&bars->tab_full[tb], ((g + 1) / kTabBufs) & 1, abort_flag);
        const SlotEntry e = tabs[tb * kSlots + s];
        mbar_arrive(&bars->tab_empty[tb]);
        rowp = e.row;
        sc_next = e.row != nullptr ? __ldg(e.scales) : make_uint2(0, 0);
      }
      const int b = g % kKBufs;
      const uint32_t kbuf = k_base + uint32_t(b) * kBlockBytes;
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        if (g >= kKBufs) ok = ok && mbar_wait(&bars->k_empty[b][m], ((g / kKBufs) - 1) & 1, abort_flag);
#ifdef CSAHCA_DSV4_TRACE
        if (pt == 0 && m == 0 && p_items == 0 && cur.blk < 8) DSV4_TRACE(0, cur.blk, 12);
#endif
        if (m < 3) {
          DSV4_STORE_NOPE(m);
          DSV4_STORE_NOPE(m + 4);
        } else {
          DSV4_STORE_NOPE(3);
          st_shared_v4(kbuf + off_r0, raw[7]);
          st_shared_v4(kbuf + off_r1, raw[8]);
        }
        fence_proxy_async_smem();
        mbar_arrive(&bars->k_full[b][m]);
        if (nxt.valid) DSV4_LOAD_PAIR(m);
      }
#undef DSV4_STORE_NOPE
#ifdef CSAHCA_DSV4_TRACE
      if (pt == 0 && p_items == 0 && cur.blk < 8) DSV4_TRACE(0, cur.blk, 2);
      if (cur.blk == cur.nblk - 1) ++p_items;
#endif
      sc = sc_next;
      ++g;
      cur = nxt;
    }
#undef DSV4_LOAD_PAIR
#undef DSV4_LOAD
    if (!ok) failed = true;
  } else if (warp >= kResWarp0 && warp < kResWarp0 + kResWarps) {
    // ------------------------------------------------------------ slot-table resolvers
    // Thread rs resolves slot rs of every block into tabs[j % kTabBufs]: the
    // index load runs two blocks ahead, the row address, scale-byte load and L2
    // prefetch of the row one block ahead, and the entry is published when the
    // table buffer is free (every producer and softmax thread has read it).
    // The resolvers thus run up to kTabBufs blocks ahead of the producers, and
    // the row prefetches reach L2 long before the producers' register loads.
    const int rs = threadIdx.x - kResWarp0 * 32;
    bool ok = true;
    uint32_t j = 0;
    // The first item's first main index is loaded before its lengths are known
    // (the load does not depend on them), and its extra indices are pulled into
    // L2, so the first slot table waits on one DRAM round trip less.
    int spec_loc = -1, spec_off = -1;
    if (blockIdx.x < p.num_items) {
      const int qs = blockIdx.x / p.groups;
      const int q = qs % p.num_queries, sg = p.split0 + qs / p.num_queries;
      const int lo_m = int((int64_t(p.nmain) * sg) / p.split_total);
      if (lo_m + rs < p.nmain) {
        spec_off = lo_m;
        spec_loc = __ldg(p.idx + size_t(q) * p.nmain + lo_m + rs);
      }
      if (p.xidx != nullptr && p.nextra > 0) {
        const int lo_x = int((int64_t(p.nextra) * sg) / p.split_total);
        if (lo_x + rs < p.nextra)
          asm volatile("prefetch.global.L2 [%0];" ::"l"(p.xidx + size_t(q) * p.nextra + lo_x + rs) : "memory");
      }
    }
    Cursor c0 = first_cursor(p);
    Cursor c1 = next_cursor(p, c0);
    Cursor c2 = next_cursor(p, c1);
    SlotEntry e0, e1;
    e0.row = e1.row = nullptr;
    e0.scales = e1.scales = nullptr;
    PendingSlot ps;
    ps.loc = -1;
    ps.main = true;
    {
      // The index loads of the first three blocks go out together, then the
      // scale loads of the first two: two round trips to the first table
      // instead of five.
      PendingSlot p0, p1;
      p0.loc = p1.loc = -1;
      p0.main = p1.main = true;
      if (c0.valid && c0.item == int(blockIdx.x) && c0.blk == 0 && c0.sp.main_off == spec_off &&
          rs < c0.sp.len_main) {
        p0.loc = spec_loc;  // the speculative load above is this slot's index
      } else if (c0.valid) {
        p0 = slot_loc(p, c0.sp, c0.blk, rs);
      }
      if (c1.valid) p1 = slot_loc(p, c1.sp, c1.blk, rs);
      if (c2.valid) ps = slot_loc(p, c2.sp, c2.blk, rs);
      if (c0.valid) e0 = finish_slot(p, p0);
      if (c1.valid) e1 = finish_slot(p, p1);
    }
    while (c0.valid) {
      const int tb = j % kTabBufs;
      if (j >= kTabBufs && !(ok = mbar_wait(&bars->tab_empty[tb], ((j / kTabBufs) - 1) & 1, abort_flag))) break;
      tabs[tb * kSlots + rs] = e0;
      mbar_arrive(&bars->tab_full[tb]);
      const Cursor c3 = next_cursor(p, c2);
      e0 = e1;
      if (c2.valid) e1 = finish_slot(p, ps);
      if (c3.valid) ps = slot_loc(p, c3.sp, c3.blk, rs);
      c0 = c1;
      c1 = c2;
      c2 = c3;
      ++j;
    }
    if (!ok) failed = true;
  } else if (warp == kQWarp) {
    // ------------------------------------------------------------ Q loader
    // Q of an item goes into the swizzled K-major Q tile once the last QK of the
    // previous item has read it (q_empty).
    bool ok = true;
    uint32_t items = 0;
    for (int it = blockIdx.x; it < p.num_items && ok; it += gridDim.x) {
      const int qs = it / p.groups, hg = it - qs * p.groups;
      const SlotSpace sp = slot_space(p, qs);
      if (sp.blocks() == 0) continue;
      const int q = sp.q;
      if (items > 0 && !(ok = mbar_wait(&bars->q_empty, (items - 1) & 1, abort_flag))) break;
      const QT* qsrc = static_cast<const QT*>(p.q) + size_t(q) * p.heads * kDim;
#pragma unroll 4
      for (int i = lane; i < kHeads * 64; i += 32) {
        const int row = i >> 6, c = i & 63;
        const int head = hg * kHeads + row;
        const uint32_t dst = q_base + sub_pos(c >> 3) * (kHeads * 128) + sw128(row, c & 7);
        if (head >= p.heads) {
          st_shared_v4(dst, make_uint4(0, 0, 0, 0));
        } else if constexpr (std::is_same<QT, __nv_bfloat16>::value) {
          cp_async16(dst, qsrc + size_t(head) * kDim + c * 8);
        } else {
          st_shared_v4(dst, load_q8_bf16<QT>(qsrc + size_t(head) * kDim + c * 8));
        }
      }
      cp_async_wait_all();
      fence_proxy_async_smem();
      mbar_arrive(&bars->q_full);
      ++items;
    }
    if (!ok) failed = true;
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA issuer
    // Event-driven issue: PV(g) goes out as soon as the softmax has published
    // P(g); QK(g+1) goes out pair by pair as the producers finish each K pair,
    // every consecutive ready pair in one go.  Readiness is polled with the
    // non-blocking test_wait, so a barrier that is not complete yet never holds
    // the issuing thread back from another that is.
    // QK(g) may start only once PV(g-2) is issued (that PV's p_full wait proves
    // the softmax has finished reading S buffer g%2).  PV has priority, since it
    // frees K pairs for the producers.
    if (lane == 0) {
      uint32_t gq = 0, gp = 0, q_items = 0, pv_items = 0;
      int mq = 0;            // next K pair of QK(gq)
      bool q_ready = false;  // Q of the item of QK(gq) has been waited for
      Cursor qk = first_cursor(p);
      Cursor pv = qk;
      bool ok = true;
      long long idle_since = -1;
      while (ok && pv.valid) {
        bool progressed = false;
        if (gp < gq) {
          const int b = gp % kKBufs;
          bool ready = mbar_test_wait(&bars->p_full[b], (gp / kKBufs) & 1);
          if (ready && pv.blk == 0 && pv_items > 0) ready = mbar_test_wait(&bars->o_empty, (pv_items - 1) & 1);
          if (ready) {
            DSV4_TRACE(pv_items, pv.blk, 5);
            tc_fence_after();
            // O^T[m] += V^T[m] . P^T, V^T read MN-major from the same K tile.
            const uint32_t kbuf = k_base + uint32_t(b) * kBlockBytes;
            const uint32_t pbuf = p_base + uint32_t(b) * kPBytes;
            // Descriptors are built once; every further MMA only moves the start
            // address field (bits 0..13, in 16-byte units), which keeps the single
            // issuing thread at a few instructions per MMA.
            // V^T block m (dims 128m..): sub-tiles 2m and 2m+1, two positions apart.
            const uint64_t a_pv = smem_desc_sw128(kbuf, 2 * kSubTileBytes, 1024);
            const uint64_t b_pv = smem_desc_sw128(pbuf, kPBytes, 1024);
            const uint32_t acc_first = pv.blk != 0;
            // V^T blocks 0 and 2 first (sub-tiles 0,1,4,5: K groups 0 and 1, which
            // the producers may refill as soon as these MMAs complete), then
            // blocks 1 and 3 (groups 2 and 3).  Within each half the two blocks
            // alternate k-step by k-step, so no MMA waits on the accumulation
            // of the one before it.
#pragma unroll
            for (int half = 0; half < 2; ++half) {
#pragma unroll
              for (int kk = 0; kk < kSlots / 16; ++kk)
#pragma unroll
                for (int mm = 0; mm < 2; ++mm) {
                  const int m = half + 2 * mm;
                  mma_bf16_ss(tmem + 64 * m, a_pv + uint64_t((sub_pos(2 * m) * kSubTileBytes + kk * 2048) >> 4),
                              b_pv + uint64_t((kk * 2048) >> 4), kIdescPV, kk == 0 ? acc_first : 1u);
                }
              mma_commit(&bars->k_empty[b][2 * half]);
              mma_commit(&bars->k_empty[b][2 * half + 1]);
            }
            mma_commit(&bars->pv_done);
            DSV4_TRACE(pv_items, pv.blk, 6);
            if (pv.blk == pv.nblk - 1) {
              mma_commit(&bars->o_full);
              ++pv_items;
            }
            ++gp;
            pv = next_cursor(p, pv);
            progressed = true;
          }
        }
        if (!progressed && qk.valid && gq <= gp + 1) {
          const int bq = gq % kKBufs;
          bool ready = true;
          if (qk.blk == 0 && !q_ready) {
            ready = q_ready = mbar_test_wait(&bars->q_full, q_items & 1);
            if (q_ready) ++q_items;
          }
          if (ready) ready = mbar_test_wait(&bars->k_full[bq][mq], (gq / kKBufs) & 1);
          while (ready) {
            if (mq == 0) DSV4_TRACE(q_items - 1, qk.blk, 3);
            if (mq == 3) DSV4_TRACE(q_items - 1, qk.blk, 14);
            tc_fence_after();
            const uint64_t a_qk = smem_desc_sw128(k_base + uint32_t(bq) * kBlockBytes + 2 * mq * kSubTileBytes, 16, 1024);
            const uint64_t b_qk = smem_desc_sw128(q_base + 2 * mq * (kHeads * 128), 16, 1024);
            const uint32_t acc_first = mq != 0;
            // Group mq: sub-tiles mq and mq+4 of K (rows) and Q (columns) at once.
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              mma_bf16_ss(tmem + kTmemS + 128 * bq, a_qk + uint64_t((kk * 32) >> 4), b_qk + uint64_t((kk * 32) >> 4),
                          kIdescQK, kk == 0 ? acc_first : 1u);
            if (++mq == 4) {
              mma_commit(&bars->s_full[bq]);
              if (qk.blk == qk.nblk - 1) mma_commit(&bars->q_empty);
              DSV4_TRACE(q_items - 1, qk.blk, 4);
              mq = 0;
              q_ready = false;
              ++gq;
              qk = next_cursor(p, qk);
              progressed = true;
              break;
            }
            progressed = true;
            ready = mbar_test_wait(&bars->k_full[bq][mq], (gq / kKBufs) & 1);
          }
        }
        if (progressed) {
          idle_since = -1;
        } else {
          // Nothing ready: sleep briefly on the barrier that is due next.
          if (gp < gq)
            mbar_try_wait_sleep(&bars->p_full[gp % kKBufs], (gp / kKBufs) & 1, 200u);
          else if (qk.valid)
            mbar_try_wait_sleep(&bars->k_full[gq % kKBufs][mq], (gq / kKBufs) & 1, 200u);
          if (idle_since < 0)
            idle_since = clock64();
          else if (*abort_flag || clock64() - idle_since > 4000000000ll)
            ok = false;
        }
      }
      if (!ok) failed = true;
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ softmax + epilogue
    // S buffer b (128 columns) holds, for slot s, the partial scores over dims
    // of sub-tiles 0-3 in lane s, columns 0-63 (heads) and those over sub-tiles
    // 4-7 in lane 64 + s, columns 64-127.  Warps 0/2 take slots 0-31, warps 1/3
    // slots 32-63; warps 0-1 own heads 0-31, warps 2-3 heads 32-63.  Each
    // thread hands the partials of the other half of the heads to its partner
    // (same slot, other warp pair) through shared memory and adds the
    // partner's to its own, then works on 32 heads of one slot.
    // The per-head running max m_use only moves when some score of the block
    // exceeds it by more than 2^8 (block-wide vote; the column-max reduction runs
    // only then); each thread keeps its slot's partial sums of P per head in
    // registers until the query ends.
    const int t = threadIdx.x;
    const int hh = warp >> 1;                 // head half owned by this thread
    const int slot = 32 * (warp & 1) + lane;  // slot row of this thread
    const int h_lo = 32 * hh;                 // first head of this thread's half
    const uint32_t t_lane = tmem + (uint32_t(warp * 32) << 16);
    const uint32_t x_row = smem_u32(smem + kOffX) + uint32_t(slot) * 128u;
    const uint32_t x_sw = uint32_t(slot & 7);
    const float sl2 = p.scale_log2;
    constexpr int esz = sizeof(QT);
    // Items without any valid slot: zeros (the sink alone gives a zero output).
    for (int item = blockIdx.x; item < p.num_items; item += gridDim.x) {
      const int q = item / p.groups, hg = item - q * p.groups;  // q: work row (query-shard)
      if (slot_space(p, q).blocks() != 0) continue;
      const int hcount = min(kHeads, p.heads - hg * kHeads);
      const int oesz = p.lse != nullptr ? 4 : esz;
      uint8_t* out_q = static_cast<uint8_t*>(p.out) + (size_t(q) * p.heads + size_t(hg) * kHeads) * kDim * oesz;
      const int nvec = hcount * kDim * oesz / 16;
      for (int i = t; i < nvec; i += 128) reinterpret_cast<uint4*>(out_q)[i] = make_uint4(0, 0, 0, 0);
      if (p.lse != nullptr && t < hcount) p.lse[size_t(q) * p.heads + hg * kHeads + t] = -INFINITY;
    }
    float la[32];  // this slot's partial sums of P per head of this half (m_use frame)
#pragma unroll
    for (int c = 0; c < 32; ++c) la[c] = 0.f;
    uint32_t g = 0, items_done = 0;
    float sink_l2 = -INFINITY;  // sink logit (log2 units) of head t of the current item, t < kHeads
    for (Cursor cur = first_cursor(p); cur.valid; cur = next_cursor(p, cur), ++g) {
      const int b = g % kKBufs;
      const bool okw = mbar_wait(&bars->s_full[b], (g / kKBufs) & 1, abort_flag);
      if (!soft_sync_and(okw)) goto soft_fail;
      if (t == 0) DSV4_TRACE(items_done, cur.blk, 7);
      if (cur.blk == 0 && t < kHeads && p.sink != nullptr) {
        // The sink logit of this thread's head, fetched now so the epilogue does not wait on it.
        const int hsink = (cur.item % p.groups) * kHeads + t;
        sink_l2 = hsink < p.heads ? __ldg(p.sink + hsink) * kLog2e : -INFINITY;
      }
      tc_fence_after();
      const bool valid = tabs[(g % kTabBufs) * kSlots + slot].row != nullptr;
      mbar_arrive(&bars->tab_empty[g % kTabBufs]);
      const uint32_t s_col = kTmemS + 128 * b;
      float v[32];  // scores of this thread's slot, heads h_lo .. h_lo+31
      {
        float w[32];  // the partner's heads, from this thread's dims
        tmem_ld32(t_lane + s_col + (hh ? 96 : 0), v);
        tmem_ld32(t_lane + s_col + (hh ? 64 : 32), w);
        tmem_wait_ld();
        // Heads 32-63 of dims 0-255 go from warps 0-1 to warps 2-3, then heads
        // 0-31 of dims 256-511 back, through one 8 KB buffer.
#pragma unroll
        for (int round = 0; round < 2; ++round) {
          if (hh == round) {
#pragma unroll
            for (int j = 0; j < 8; ++j)
              st_shared_v4(x_row + ((uint32_t(j) ^ x_sw) << 4),
                           make_uint4(__float_as_uint(w[4 * j]), __float_as_uint(w[4 * j + 1]),
                                      __float_as_uint(w[4 * j + 2]), __float_as_uint(w[4 * j + 3])));
          }
          named_bar_sync(1, 128);
          if (hh != round) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              uint4 x4;
              asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                           : "=r"(x4.x), "=r"(x4.y), "=r"(x4.z), "=r"(x4.w)
                           : "r"(x_row + ((uint32_t(j) ^ x_sw) << 4)));
              v[4 * j] += __uint_as_float(x4.x);
              v[4 * j + 1] += __uint_as_float(x4.y);
              v[4 * j + 2] += __uint_as_float(x4.z);
              v[4 * j + 3] += __uint_as_float(x4.w);
            }
          }
          if (round == 0) named_bar_sync(1, 128);  // the buffer is read before round 1 writes it
        }
      }
      bool over = false;
#pragma unroll
      for (int c = 0; c < 32; ++c) over |= fmaf(v[c], sl2, -bars->m_use[h_lo + c]) > 8.f;
      const bool rebase = group_sync_or(1, 128, valid && over);
      if (rebase) {
        {
          float w[32];
#pragma unroll
          for (int c = 0; c < 32; ++c) w[c] = valid ? v[c] * sl2 : -INFINITY;
          bars->red[warp][lane] = warp_colreduce32<true>(w);  // head h_lo + lane over this warp's 32 slots
        }
        named_bar_sync(1, 128);
        if (t < kHeads) {
          const int w0 = 2 * (t >> 5);
          const float bm = fmaxf(bars->red[w0][t & 31], bars->red[w0 + 1][t & 31]);
          const float mo = bars->m_use[t];
          float alpha = 1.f;
          if (bm > mo + 8.f || (mo == -INFINITY && bm != -INFINITY)) {
            alpha = mo == -INFINITY ? 0.f : fast_exp2(mo - bm);
            bars->m_use[t] = bm;
          }
          bars->alpha[t] = alpha;
        }
        named_bar_sync(1, 128);
#pragma unroll
        for (int c = 0; c < 32; ++c) la[c] *= bars->alpha[h_lo + c];
        if (cur.blk > 0) {
          // O must hold PV of the previous block before it is re-based.
          const bool okp = mbar_wait(&bars->pv_done, (g - 1) & 1, abort_flag);
          if (!soft_sync_and(okp)) goto soft_fail;
          tc_fence_after();
#pragma unroll 1
          for (int m = 0; m < 4; ++m)
#pragma unroll 1
            for (int oh = 0; oh < 2; ++oh) {
              float o[32];
              tmem_ld32(t_lane + 64 * m + 32 * oh, o);
              tmem_wait_ld();
#pragma unroll
              for (int c = 0; c < 32; ++c) o[c] *= bars->alpha[32 * oh + c];
              tmem_st32(t_lane + 64 * m + 32 * oh, o);
            }
          tmem_wait_st();
        }
        named_bar_sync(1, 128);  // alpha consumed before the next re-base writes it
      }
      if (t == 0) DSV4_TRACE(items_done, cur.blk, 8);
      // P^T row = 2^(s*scale - m_use) in bf16, swizzled MN-major; sums in registers.
      const uint32_t pbuf = p_base + uint32_t(b) * kPBytes;
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        uint32_t w4[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int c = 8 * cc + 2 * j;
          const float p0 = valid ? fast_exp2(fmaf(v[c], sl2, -bars->m_use[h_lo + c])) : 0.f;
          const float p1 = valid ? fast_exp2(fmaf(v[c + 1], sl2, -bars->m_use[h_lo + c + 1])) : 0.f;
          la[c] += p0;
          la[c + 1] += p1;
          const __nv_bfloat162 b2 = __floats2bfloat162_rn(p0, p1);
          w4[j] = *reinterpret_cast<const uint32_t*>(&b2);
        }
        st_shared_v4(pbuf + sw128(slot, 4 * hh + cc), make_uint4(w4[0], w4[1], w4[2], w4[3]));
      }
      fence_proxy_async_smem();
      tc_fence_before();
      if (t == 0) DSV4_TRACE(items_done, cur.blk, 9);
      mbar_arrive(&bars->p_full[b]);
      if (cur.blk != cur.nblk - 1) continue;

      // -------------------------------------------------------------- epilogue
      const int q = cur.item / p.groups, hg = cur.item - q * p.groups;  // q: work row (query-shard)
      const int hcount = min(kHeads, p.heads - hg * kHeads);
      const int oesz = p.lse != nullptr ? 4 : esz;
      uint8_t* out_q = static_cast<uint8_t*>(p.out) + (size_t(q) * p.heads + size_t(hg) * kHeads) * kDim * oesz;
      {
        // Per-head sums: reduce the slots' partials once per query.
        float tmp[32];
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          tmp[c] = la[c];
          la[c] = 0.f;
        }
        bars->red[warp][lane] = warp_colreduce32<false>(tmp);
        const bool okw2 = mbar_wait(&bars->o_full, items_done & 1, abort_flag);
        if (!soft_sync_and(okw2)) goto soft_fail;
      }
      if (t == 0) DSV4_TRACE(items_done, 0, 10);
      tc_fence_after();
      if (t < kHeads) {
        const int w0 = 2 * (t >> 5);
        float total = bars->red[w0][t & 31] + bars->red[w0 + 1][t & 31];
        const float mu = bars->m_use[t];
        if (p.lse != nullptr) {
          if (hg * kHeads + t < p.heads)
            p.lse[size_t(q) * p.heads + hg * kHeads + t] = (total > 0.f && mu != -INFINITY) ? mu + fast_log2(total) : -INFINITY;
        } else if (p.sink != nullptr && hg * kHeads + t < p.heads) {
          total += (mu == -INFINITY) ? (sink_l2 == -INFINITY ? 0.f : INFINITY) : fast_exp2(sink_l2 - mu);
        }
        bars->inv_l[t] = (total > 0.f && total != INFINITY) ? fast_rcp(total) : 0.f;
        bars->m_use[t] = -INFINITY;
      }
      named_bar_sync(1, 128);
      {
        // Stage rounds of heads in the (free) P buffers as [head][512] rows of
        // the output type -- each thread owns one dim of each O^T block -- and
        // send every round to global memory with one bulk store.  After the
        // CTA's last block the K buffers are idle (every PV has completed and
        // the producers are done), so each round gets its own 16 KB there and
        // no round waits for the previous round's store.
        const bool f32out = p.lse != nullptr || esz == 4;
        const int per_round = f32out ? 8 : 16;  // 16 KB of staging per round
        const int oes = f32out ? 4 : esz;
        const bool spread = !next_cursor(p, cur).valid;
        static_assert(kKBufs * kBlockBytes >= 8 * 16384, "K buffers hold every staging round");
        if (t == 0) DSV4_TRACE(1, 1, 10);
        for (int h0 = 0; h0 < hcount; h0 += per_round) {
          if (t == 0) DSV4_TRACE(1, 2 + h0 / per_round, 10);
          const uint32_t stage = spread ? k_base + uint32_t(h0 / per_round) * 16384u : p_base;
          if (h0 > 0 && !spread) {
            if (t == 0) bulk_wait_read_all();
            named_bar_sync(1, 128);  // the previous round's bulk store has read the staging
          }
          // One O^T block at a time and no unrolling across blocks: this code runs
          // once per query, so its size (instruction-cache misses) matters more
          // than its loop overhead.
          float inv[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) inv[i] = i < per_round ? bars->inv_l[h0 + i] : 0.f;
#pragma unroll 1
          for (int m = 0; m < 4; ++m) {
            float o[16];
            tmem_ld16(t_lane + 64 * m + h0, o);
            tmem_wait_ld();
            if (m == 3 && h0 + per_round >= hcount) {
              // Every O value has been read: the next query's PV may start now.
              tc_fence_before();
              mbar_arrive(&bars->o_empty);
            }
            const uint32_t a0 = stage + uint32_t((128 * m + t) * oes);
            if (f32out) {
#pragma unroll
              for (int i = 0; i < 8; ++i)
                asm volatile("st.shared.f32 [%0], %1;" ::"r"(a0 + uint32_t(i * kDim * 4)), "f"(o[i] * inv[i]) : "memory");
            } else {
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                const QT x = Elem<QT>::from_f(o[i] * inv[i]);
                asm volatile("st.shared.u16 [%0], %1;" ::"r"(a0 + uint32_t(i * kDim * 2)),
                             "h"(*reinterpret_cast<const unsigned short*>(&x))
                             : "memory");
              }
            }
          }
          if (t == 0) DSV4_TRACE(1, 2 + h0 / per_round, 11);
          fence_proxy_async_smem();
          named_bar_sync(1, 128);
          if (t == 0) {
            const int nh = min(per_round, hcount - h0);
            bulk_store_s2g(out_q + size_t(h0) * kDim * oes, stage, uint32_t(nh * kDim * oes));
            bulk_commit();
          }
        }
        if (t == 0) bulk_wait_read_all();  // the P buffers are free again for the next query
      }
      if (t == 0) DSV4_TRACE(items_done, 0, 11);
      named_bar_sync(1, 128);  // inv_l / red consumed before the next query reuses them
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
  if (threadIdx.x == 0) DSV4_TRACE(1, 0, 1);
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

static int dsv4_entry(const void* q, int q_dtype, int64_t num_queries, int64_t heads, const uint8_t* cache,
                      int64_t num_pages, int64_t bytes_per_page, int64_t page_size, const int32_t* token_indices,
                      int64_t topk_slots, const int32_t* topk_lengths, const uint8_t* extra_cache,
                      int64_t extra_num_pages, int64_t extra_bytes_per_page, int64_t extra_page_size,
                      const int32_t* extra_token_indices, int64_t extra_topk_slots,
                      const int32_t* extra_topk_lengths, const float* attn_sink, float softmax_scale, void* out,
                      float* lse, int64_t shard0, int64_t shards, int64_t shards_total, void* stream) {
  if (shards < 1 || shards_total < 1 || shard0 < 0 || shard0 + shards > shards_total)
    return csahca_set_arg_error("invalid shard range");
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
  if (num_queries * shards * heads > (int64_t(1) << 30)) return csahca_set_unsupported("problem too large");

  Dsv4Params p;
  p.q = q;
  p.cache = cache;
  p.idx = token_indices;
  p.lens = topk_lengths;
  p.xcache = has_extra ? extra_cache : nullptr;
  p.xidx = has_extra ? extra_token_indices : nullptr;
  p.xlens = has_extra ? extra_topk_lengths : nullptr;
  p.sink = lse != nullptr ? nullptr : attn_sink;
  p.out = out;
  p.lse = lse;
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
  p.splits = int(shards);
  p.split0 = int(shard0);
  p.split_total = int(shards_total);
  p.num_items = p.num_queries * p.splits * p.groups;
  p.scale_log2 = softmax_scale * kLog2e;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (q_dtype) {
    case CSAHCA_DTYPE_BF16: return launch_dsv4<__nv_bfloat16>(p, s);
    case CSAHCA_DTYPE_F16: return launch_dsv4<__half>(p, s);
    case CSAHCA_DTYPE_F32: return launch_dsv4<float>(p, s);
    default: return csahca_set_arg_error("unsupported q dtype");
  }
}

extern "C" int csahca_dsv4_decode(const void* q, int q_dtype, int64_t num_queries, int64_t heads, const uint8_t* cache,
                                  int64_t num_pages, int64_t bytes_per_page, int64_t page_size,
                                  const int32_t* token_indices, int64_t topk_slots, const int32_t* topk_lengths,
                                  const uint8_t* extra_cache, int64_t extra_num_pages, int64_t extra_bytes_per_page,
                                  int64_t extra_page_size, const int32_t* extra_token_indices,
                                  int64_t extra_topk_slots, const int32_t* extra_topk_lengths, const float* attn_sink,
                                  float softmax_scale, void* out, void* stream) {
  return dsv4_entry(q, q_dtype, num_queries, heads, cache, num_pages, bytes_per_page, page_size, token_indices,
                    topk_slots, topk_lengths, extra_cache, extra_num_pages, extra_bytes_per_page, extra_page_size,
                    extra_token_indices, extra_topk_slots, extra_topk_lengths, attn_sink, softmax_scale, out, nullptr,
                    0, 1, 1, stream);
}

extern "C" int csahca_dsv4_decode_partial(const void* q, int q_dtype, int64_t num_queries, int64_t heads,
                                          const uint8_t* cache, int64_t num_pages, int64_t bytes_per_page,
                                          int64_t page_size, const int32_t* token_indices, int64_t topk_slots,
                                          const int32_t* topk_lengths, const uint8_t* extra_cache,
                                          int64_t extra_num_pages, int64_t extra_bytes_per_page,
                                          int64_t extra_page_size, const int32_t* extra_token_indices,
                                          int64_t extra_topk_slots, const int32_t* extra_topk_lengths,
                                          float softmax_scale, int64_t shard0, int64_t shards, int64_t shards_total,
                                          float* o_partial, float* lse_partial, void* stream) {
  if (lse_partial == nullptr || o_partial == nullptr) return csahca_set_arg_error("o_partial and lse_partial are required");
  return dsv4_entry(q, q_dtype, num_queries, heads, cache, num_pages, bytes_per_page, page_size, token_indices,
                    topk_slots, topk_lengths, extra_cache, extra_num_pages, extra_bytes_per_page, extra_page_size,
                    extra_token_indices, extra_topk_slots, extra_topk_lengths, nullptr, softmax_scale, o_partial,
                    lse_partial, shard0, shards, shards_total, stream);
}

#ifdef CSAHCA_DSV4_TRACE
extern "C" __attribute__((visibility("default"))) int csahca_dsv4_trace_read(long long* host, int n) {
  if (n > 2 * 8 * 16) n = 2 * 8 * 16;
  CSAHCA_RETURN_IF_CUDA(cudaDeviceSynchronize());
  CSAHCA_RETURN_IF_CUDA(cudaMemcpyFromSymbol(host, csahca::g_dsv4_trace, sizeof(long long) * n));
  return CSAHCA_OK;
}
extern "C" __attribute__((visibility("default"))) int csahca_dsv4_trace_reset(void) {
  static long long zeros[2 * 8 * 16] = {};
  CSAHCA_RETURN_IF_CUDA(cudaMemcpyToSymbol(csahca::g_dsv4_trace, zeros, sizeof(zeros)));
  return CSAHCA_OK;
}
#endif
