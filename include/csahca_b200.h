/*
 * csahca_b200 — C ABI of the B200 (sm_100a) compressed-sparse-attention decode kernels.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream
 * (cudaStream_t passed as void*), enqueues its kernels on that stream and
 * returns without synchronising.  Nothing here allocates device memory: outputs
 * and workspaces are supplied by the caller.
 *
 * Return value: CSAHCA_OK (0) on success, otherwise a CSAHCA_E* code; the
 * message of the last failure on the calling thread is csahca_last_error().
 * Argument checks mirror the TORCH_CHECK conditions of the reference host code
 * and return CSAHCA_EINVAL with the same message text.
 *
 * Reference: ypd666/CSAHCA (hybrid_attention/, csrc/).  Each declaration names
 * the reference interface it replaces.
 */
#ifndef CSAHCA_B200_H_
#define CSAHCA_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

/* Element types of q / K / V / outputs. */
#define CSAHCA_DTYPE_F32 0
#define CSAHCA_DTYPE_F16 1
#define CSAHCA_DTYPE_BF16 2

/* Element types of CSA chunk-index tensors. */
#define CSAHCA_INDEX_I32 0
#define CSAHCA_INDEX_I64 1

/* Status codes. */
#define CSAHCA_OK 0
#define CSAHCA_EINVAL 1       /* argument rejected (message in csahca_last_error) */
#define CSAHCA_ECUDA 2        /* a CUDA runtime call failed */
#define CSAHCA_EUNSUPPORTED 3 /* valid for the reference, not supported by these kernels */

/* Message of the last non-zero status returned on the calling thread. */
const char* csahca_last_error(void);

/* Library version string. */
const char* csahca_version(void);

/*
 * Reads and clears the device error word of the current device.  Kernels set it
 * (instead of trapping) when a bounded wait gives up or a slot index falls
 * outside its cache.  Synchronises the current device.  *code = 0 means no error.
 */
int csahca_read_device_error(int* code);

/* ------------------------------------------------------------------ CSA scorer
 * Chunk scorer + per-(batch, head) top-k.
 * Replaces hybrid_attention/reference.py:40-56 (chunk_mean + select_topk_chunks),
 * called by hybrid_attention/benchmark.py:97 and model_inference.py:53,183.
 *
 *   score[b,h,c] = (q[b,h,:] . mean_t K[b,h,c*chunk + t,:]) / sqrt(head_dim)   (fp32)
 *   out[b,h,:]   = indices of the min(top_k, S/chunk) largest scores, largest
 *                  first, equal scores ordered by lower chunk index.
 *
 * q [B,H,D], k_cache [B,H,S,D] of `dtype`; S % chunk_size == 0.
 * seq_lens: NULL, or int32 [B] per-request valid lengths (each a multiple of
 *   chunk_size, <= S).  Request b then only scores its first seq_lens[b]/chunk
 *   chunks, and slots past that count are written as -1.
 * out_indices: int32 [B,H,min(top_k, S/chunk_size)].
 * workspace: csahca_csa_select_topk_workspace_size() bytes, zero-filled before
 *   its first use; every call leaves it zero-filled again.  Calls that may run
 *   concurrently must not share a workspace.
 * head_dim in {32, 64, 128, 256, 512}.
 */
size_t csahca_csa_select_topk_workspace_size(int64_t batch, int64_t heads, int64_t seq_len, int64_t chunk_size);
int csahca_csa_select_topk(const void* q, const void* k_cache, const int32_t* seq_lens, int dtype, int64_t batch,
                           int64_t heads, int64_t seq_len, int64_t head_dim, int64_t chunk_size, int64_t top_k,
                           int32_t* out_indices, void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------ CSA chunk-sum cache
 * An incremental stand-in for the scorer's read of all of K (the scorer of
 * hybrid_attention/reference.py:40-56 recomputes every chunk mean each step;
 * the reference lists caching them as future work).  sums is fp32
 * [B,H,S/chunk_size,D]: build fills it from k_cache; append adds, for each
 * request b, the K row at positions[b] (int32 [B]; out-of-range positions are
 * ignored) into its chunk, the first token of a chunk overwriting.
 * csahca_csa_select_topk_from_sums selects on the cache exactly as
 * csahca_csa_select_topk does on k_cache (scores q . sum / chunk / sqrt(D);
 * same index order, ties and -1 fill; seq_lens in tokens as there; workspace of
 * csahca_csa_select_topk_workspace_size(B, H, num_chunks * chunk_size,
 * chunk_size) bytes with the same zero-fill contract).  q of q_dtype, head_dim
 * a multiple of 4 up to 1024, sums 16-byte aligned.
 */
int csahca_csa_chunk_sums_build(const void* k_cache, int dtype, int64_t batch, int64_t heads, int64_t seq_len,
                                int64_t head_dim, int64_t chunk_size, float* sums, void* stream);
int csahca_csa_select_topk_from_sums(const void* q, int q_dtype, const float* sums, const int32_t* seq_lens,
                                     int64_t batch, int64_t heads, int64_t num_chunks, int64_t head_dim,
                                     int64_t chunk_size, int64_t top_k, int32_t* out_indices, void* workspace,
                                     size_t workspace_bytes, void* stream);
int csahca_csa_chunk_sums_append(const void* k_cache, int dtype, int64_t batch, int64_t heads, int64_t seq_len,
                                 int64_t head_dim, int64_t chunk_size, const int32_t* positions, float* sums,
                                 void* stream);

/* ------------------------------------------------------------------ CSA decode
 * Split-K decode over the selected chunks with an in-kernel log-sum-exp combine.
 * Replaces csrc/csa_attention.cu:330-385 (csa_decode_forward_cuda) and
 * csrc/csa_attention.cu:387-452 (csa_decode_forward_tiled_cuda), i.e. the
 * pybind symbols csa_decode_forward / csa_decode_forward_tiled
 * (csrc/bindings.cpp:54-77,158-160).
 *
 * q [B,H,D], k_cache / v_cache [B,H,S,D] of `dtype`, chunk_indices [B,H,top_k]
 * (int32 or int64); out [B,H,D] of `dtype`.  Slots with a negative chunk index
 * and tokens at or beyond S are skipped; a (b,h) with no token left gets zeros.
 * The tile size of the reference is a tuning knob only and has no counterpart:
 * results do not depend on it.
 * workspace: csahca_csa_decode_workspace_size() bytes of any content (the call
 *   clears the part it needs with a memset on `stream`); calls that may run
 *   concurrently must not share it.  head_dim in {32, 64, 128, 256, 512}.
 */
size_t csahca_csa_decode_workspace_size(int64_t batch, int64_t heads, int64_t head_dim, int64_t top_k,
                                        int64_t chunk_size);
int csahca_csa_decode(const void* q, const void* k_cache, const void* v_cache, const void* chunk_indices,
                      int index_dtype, int dtype, int64_t batch, int64_t heads, int64_t seq_len, int64_t head_dim,
                      int64_t top_k, int64_t chunk_size, void* out, void* workspace, size_t workspace_bytes,
                      void* stream);

/*
 * Allocation-free CSA decode (no counterpart in the reference).
 * Same computation and arguments as csahca_csa_decode minus the workspace: the
 * scratch is a fixed 8 MiB array inside the library (one per GPU, held until
 * process exit), for callers that cannot allocate device memory at call time --
 * e.g. a server that pre-reserved all HBM, a latency-critical loop that must
 * avoid cudaMalloc's implicit synchronisation, or a foreign-language binding
 * without a device allocator.  Problems whose scratch would exceed
 * csahca_csa_decode_noalloc_max_scratch_bytes() return CSAHCA_EINVAL.  The first
 * call on a device resolves the array's device address; make it before any
 * stream capture.  The address is kept for the life of the process: after
 * cudaDeviceReset (or any primary-context reset) restart the process before
 * calling this again.  All calls share the array: calls that overlap on the
 * GPU race.
 */
size_t csahca_csa_decode_noalloc_max_scratch_bytes(void);
int csahca_csa_decode_noalloc(const void* q, const void* k_cache, const void* v_cache, const void* chunk_indices,
                              int index_dtype, int dtype, int64_t batch, int64_t heads, int64_t seq_len,
                              int64_t head_dim, int64_t top_k, int64_t chunk_size, void* out, void* stream);

/* ------------------------------------------------------------------ DSV4 indexer
 * Compressed-slot selection on device: per query, index scores
 *   I[s] = sum_j w[j] * max(0, q[j, :] . k[s, :])
 * over its indexer heads j and key slots s (the lightning-indexer score of
 * the DeepSeek-V3.2 technical report), then the top_k slots by I, largest
 * first, equal scores by lower slot, -1 past min(top_k, valid slots).  The
 * reference has no counterpart: its DSV4 path receives these indices from its
 * caller (integrations/sglang_dsv4/csahca_sglang_dsv4_patch/patch.py:336-341)
 * and lists an on-device indexer as future work (docs/dsv4_abi_status.md:111-119).
 *
 * q [Q, 64, 128] bf16, weights [Q, 64] fp32, keys [Q, n_keys, 128] bf16 (each
 * query's compressed-slot keys), key_lens [Q] int32 valid slots (NULL: all);
 * out_indices [Q, min(top_k, n_keys)] int32.  workspace:
 * csahca_dsv4_indexer_workspace_size() bytes of any content.  q, weights and
 * keys must be 16-byte aligned (CSAHCA_EINVAL otherwise); 64 heads of dim
 * 128 only, num_queries * n_keys < 2^31
 * (CSAHCA_EUNSUPPORTED otherwise).
 */
size_t csahca_dsv4_indexer_workspace_size(int64_t num_queries, int64_t n_keys);
int csahca_dsv4_indexer_topk(const void* q, const float* weights, const void* keys, const int32_t* key_lens,
                             int64_t num_queries, int64_t heads, int64_t n_keys, int64_t head_dim, int64_t top_k,
                             int32_t* out_indices, void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------ DSV4 decode
 * DeepSeek-V4 paged FP8 latent-cache decode (compress ratio 0 / 4 / 128).
 * Replaces csrc/dsv4_attention.cu:585-657 (dsv4_swa_decode_forward_cuda),
 * :659-760 (dsv4_sparse_decode_forward_cuda) and :762-909
 * (dsv4_decode_forward_tiled_cuda), i.e. the pybind symbols
 * dsv4_swa_decode_forward / dsv4_sparse_decode_forward /
 * dsv4_decode_forward_tiled (csrc/bindings.cpp:79-164).
 *
 * Cache rows: 448 e4m3 + 64 bf16 dims (576 bytes) at page*bytes_per_page +
 * (loc%page_size)*576, UE8M0 scales at page*bytes_per_page + page_size*576 +
 * (loc%page_size)*8, page = loc/page_size.
 * q [Q,H,512] of q_dtype; out [Q,H,512] of q_dtype.
 * token_indices int32 [Q,topk_slots]; topk_lengths NULL or int32 [Q] (clamped
 * to [0,topk_slots]); the extra (compressed) cache arguments may be NULL /
 * zero-sized.  Negative slot indices are skipped.  attn_sink NULL or fp32 [H]
 * (a virtual token with score sink[h] and value 0).  The tile size of the
 * reference is a tuning knob with no counterpart here.
 * Slot indices at or beyond num_pages*page_size are skipped and flag the device
 * error word (the reference reads out of bounds there).
 */
int csahca_dsv4_decode(const void* q, int q_dtype, int64_t num_queries, int64_t heads, const uint8_t* cache,
                       int64_t num_pages, int64_t bytes_per_page, int64_t page_size, const int32_t* token_indices,
                       int64_t topk_slots, const int32_t* topk_lengths, const uint8_t* extra_cache,
                       int64_t extra_num_pages, int64_t extra_bytes_per_page, int64_t extra_page_size,
                       const int32_t* extra_token_indices, int64_t extra_topk_slots,
                       const int32_t* extra_topk_lengths, const float* attn_sink, float softmax_scale, void* out,
                       void* stream);

/* ------------------------------------------------------------------ DSV4 split-KV
 * One shard of a long request's slot list, and the merge of all shards.
 * The reference has no host entry for this (its single-GPU merge is
 * csrc/dsv4_attention.cu:273-335, dsv4_decode_merge_kernel, whose rule the
 * combine follows); it serves the split-KV decode of one long request across
 * GPUs, where each GPU decodes a contiguous range of the main and extra slots
 * and the shards' (o, lse) are all-gathered and merged.
 *
 * csahca_dsv4_decode_partial: arguments as csahca_dsv4_decode without the
 * sink, plus a shard range: every query's main and extra slot lists are cut
 * into shards_total equal contiguous ranges (range s of n slots is
 * [n*s/shards_total, n*(s+1)/shards_total), lengths clamped into it) and this
 * call decodes shards shard0 .. shard0+shards-1, all in one launch.
 * o_partial fp32 [shards,Q,H,512] = each shard's output normalised by its own
 * softmax sum; lse_partial fp32 [shards,Q,H] = max score + log2(sum), in log2
 * units (scores already scaled by softmax_scale), -inf for an empty shard.
 *
 * csahca_dsv4_combine_partials: o_parts [parts,Q,H,512] and lse_parts
 * [parts,Q,H] (fp32, shard-major) -> out [Q,H,512] of out_dtype; attn_sink NULL
 * or fp32 [H], counted once as a zero-valued token.  1 <= parts <= 64.
 */
int csahca_dsv4_decode_partial(const void* q, int q_dtype, int64_t num_queries, int64_t heads, const uint8_t* cache,
                               int64_t num_pages, int64_t bytes_per_page, int64_t page_size,
                               const int32_t* token_indices, int64_t topk_slots, const int32_t* topk_lengths,
                               const uint8_t* extra_cache, int64_t extra_num_pages, int64_t extra_bytes_per_page,
                               int64_t extra_page_size, const int32_t* extra_token_indices, int64_t extra_topk_slots,
                               const int32_t* extra_topk_lengths, float softmax_scale, int64_t shard0,
                               int64_t shards, int64_t shards_total, float* o_partial, float* lse_partial,
                               void* stream);
int csahca_dsv4_combine_partials(const float* o_parts, const float* lse_parts, int64_t parts, int64_t num_queries,
                                 int64_t heads, const float* attn_sink, void* out, int out_dtype, void* stream);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif

#endif /* CSAHCA_B200_H_ */
