/*
 * shadowkv_b200.h -- C ABI of the B200 (sm_100a) ShadowKV packed-KV data plane.
 *
 * Every entry point takes DEVICE pointers, plain sizes and a cudaStream_t
 * (passed as void*), enqueues its kernels on that stream and returns an int
 * status (SKV_OK == 0).  Nothing here allocates memory: outputs, and the
 * scratch buffers whose sizes the *_scratch_bytes queries return, belong to the
 * caller.  Functions are reentrant; the only process-wide state is the
 * thread-local last-error message returned by skv_last_error().
 *
 * Layouts (reference schema of shadowinfer/shadowkv/packed_kv_cache.py):
 *   K, V        float32 [B, H, S, D], contiguous
 *   codes       int8    [S, H]   0=fp32 1=fp16 2=int8 3=int4 4=evicted
 *   masks       uint8   [S, H]   0/1 (reuse / protected / evict sets)
 *   slot        int32   [S, H]   (pos << 2) | code for a stored entry, -1 if absent
 *   bucket fp32 k/v float[N,B,D]; fp16 half[N,B,D];
 *          int8 k/v int8[N,B,D] + scale float[N,B];
 *          int4 k/v uint8[N*rb], rb = ceil(B*D/2), scale float[N*B*G]
 *   flat        int64   h*S + t of each bucket entry, in bucket order
 *
 * The entry each declaration replaces is cited as reference-file:line.
 */
#ifndef SHADOWKV_B200_H
#define SHADOWKV_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
    SKV_OK = 0,
    SKV_ERR_INVALID_ARGUMENT = 1, /* null pointer, non-positive size */
    SKV_ERR_SHAPE = 2,            /* shape mismatch between operands */
    SKV_ERR_GROUP_SIZE = 3,       /* int4 group size mismatch / invalid */
    SKV_ERR_SCRATCH = 4,          /* scratch buffer smaller than required */
    SKV_ERR_TOO_LARGE = 5,        /* size beyond a documented limit */
    SKV_ERR_CUDA = 6,             /* a CUDA launch or runtime call failed */
    SKV_ERR_UNSUPPORTED = 7       /* configuration the kernels do not cover */
};

/* One precision bucket (fp32, fp16, int8 or int4) of a packed cache. */
typedef struct skv_bucket {
    void* k;          /* payload of K (layout per precision, see above) */
    void* v;          /* payload of V */
    float* scale_k;   /* int8/int4 scales of K, NULL for fp32/fp16 */
    float* scale_v;   /* int8/int4 scales of V */
    int64_t* flat;    /* [count] h*S+t of every entry, bucket order */
    int64_t count;    /* number of entries */
} skv_bucket;

/* Library identification and error reporting. */
const char* skv_version(void);
const char* skv_status_string(int status);
const char* skv_last_error(void);
/* Number of kernels this library has launched in the process (all threads). */
int64_t skv_launch_count(void);

/* ShadowKVAgent.allocate_precision_codes  (shadowinfer/shadowkv/shadowkv_agent.py:1028-1059)
 * mode: 0 aggressive, 1 balanced, 2 conservative, other -> no adjustment. */
int skv_allocate_codes(const float* importance, int64_t n, int mode, int8_t* codes, void* stream);

/* kv_sensitivity  (shadowinfer/shadowkv/rd_allocator.py:47-61) -> float32 [S,H] */
int skv_kv_sensitivity(const float* k, const float* v, int B, int H, int S, int D,
                       float* sensitivity, void* stream);

/* predict_codes_bytes  (shadowinfer/shadowkv/rd_allocator.py:170-187) -> *out (device int64) */
int skv_predict_codes_bytes(const int8_t* codes, int64_t n, int batch, int head_dim,
                            int group_size, int64_t* out, void* stream);

/* admit_codes  (shadowinfer/shadowkv/rd_allocator.py:190-318)
 * sensitivity may be NULL (treated as ones), protected_mask may be NULL.
 * budget_bytes < 0 means "no budget".  result[0] = predicted bytes,
 * result[1] = evicted count (device int64[2]).  codes_in is not modified. */
size_t skv_admit_scratch_bytes(int S, int H);
int skv_admit_codes(const int8_t* codes_in, int8_t* codes_out, const float* importance,
                    const float* sensitivity, const uint8_t* protected_mask, int S, int H,
                    int64_t budget_bytes, int batch, int head_dim, int group_size,
                    int sink_tokens, int rd_allocation, int allow_eviction,
                    void* scratch, size_t scratch_bytes, int64_t* result, void* stream);

/* PrecisionPlan.from_codes  (shadowinfer/shadowkv/precision_plan.py:113-177)
 * flat_out  int64[S*H]: entries of codes 0,1,2,3,4 concatenated, each token-major
 * slot_out  int32[S*H]; reuse_flat_out int64[S*H] (may be NULL with reuse_mask NULL)
 * counts    int64[6] (device): entries per code 0..4, then reuse entries. */
size_t skv_plan_scratch_bytes(int S, int H);
int skv_plan_bucket(const int8_t* codes, const uint8_t* reuse_mask, int S, int H,
                    int64_t* flat_out, int32_t* slot_out, int64_t* reuse_flat_out,
                    int64_t* counts, void* scratch, size_t scratch_bytes, void* stream);

/* Allocation-free skv_plan_bucket (no counterpart in the reference).
 * For callers that cannot allocate device memory -- e.g. a host runtime that has handed the
 * whole device pool to its own allocator, or code that must not call into the CUDA
 * allocator between launches -- and so cannot provide the scratch buffer skv_plan_bucket
 * needs.  Outputs are identical to skv_plan_bucket; the tile counts live in a 64 KiB array in
 * the library's device memory, held on every device that loads the library until exit.
 * Limit: S*H <= skv_plan_static_max_entries() (4,194,304); larger sizes return
 * SKV_ERR_TOO_LARGE without launching.  The first call on a device looks up the array's
 * device address (cudaGetSymbolAddress); make that first call outside any stream capture.
 * All calls share the array: calls that overlap on the GPU (other streams, other threads)
 * race and must be serialised by the caller. */
int64_t skv_plan_static_max_entries(void);
int skv_plan_bucket_static(const int8_t* codes, const uint8_t* reuse_mask, int S, int H,
                           int64_t* flat_out, int32_t* slot_out, int64_t* reuse_flat_out,
                           int64_t* counts, void* stream);

/* PackedKVCache._do_pack_with_plan / _pack_int4_rows
 * (shadowinfer/shadowkv/packed_kv_cache.py:222-388) fused with the dense working
 * copy of ShadowKVAgent._compress_kv_with_plan (shadowkv_agent.py:1698-1809):
 * dense_k/dense_v (nullable) receive the compress_kv "k"/"v" tensors; rows with
 * reuse_mask set are taken from k_prev/v_prev when those are given. */
int skv_pack(const float* k, const float* v, int B, int H, int S, int D, int group_size,
             const int32_t* slot, const skv_bucket* buckets /* [4] */,
             float* dense_k, float* dense_v, const float* k_prev, const float* v_prev,
             const uint8_t* reuse_mask, void* stream);
/* skv_pack with the buckets laid out in ONE allocation on the device, so that the launch needs
 * no host copy of the plan's counts (the host reads them afterwards, while the kernel runs):
 * a one-thread kernel writes the skv_bucket[4] of `slab` for the DEVICE counts[0..3] (the
 * plan's, skv_plan_bucket) into `desc` (device, 192 bytes, 16-byte aligned) -- per precision
 * in code order its k, v (scale_k, scale_v) tensors in the reference layout, each at a 256-byte
 * boundary; bucket c's flat indices are flat_all[sum(counts[:c]) ...] -- and the pack kernel
 * reads them there.  If the layout needs more than slab_bytes, the descriptors are empty and
 * nothing is written (the caller packs again into a larger slab).  skv_pack_slab_bytes: the
 * bytes that layout needs, for HOST counts.  D in {64, 128, 256}, int4 group a multiple of 16,
 * K/V 16-byte and the slab 256-byte aligned (else SKV_ERR_UNSUPPORTED); no dense copy. */
int64_t skv_pack_slab_bytes(const int64_t* counts, int B, int D, int group_size);
int skv_pack_slab(const float* k, const float* v, int B, int H, int S, int D, int group_size, const int32_t* slot,
                  const int64_t* counts, const int64_t* flat_all, void* slab, int64_t slab_bytes, void* desc,
                  void* stream);

/* PackedKVCache.unpack / _dequantize_int4_bucket
 * (shadowinfer/shadowkv/packed_kv_cache.py:535-577, :636-656) -> zero-filled
 * float32 [B,H,S,D] K and V.  int4_group is the int4 bucket's group_size. */
int skv_unpack(const skv_bucket* buckets /* [4] */, const int32_t* slot, int B, int H, int S,
               int D, int int4_group, float* k_out, float* v_out, void* stream);

/* PackedKVCache.apply_reuse_mask  (shadowinfer/shadowkv/packed_kv_cache.py:753-854)
 * stats[0] = applied, stats[1] = skipped_precision (device int64[2], overwritten), or NULL
 * when the counts are not wanted. */
int skv_apply_reuse(const skv_bucket* cur /* [4] */, const int32_t* cur_slot, int S,
                    const skv_bucket* prev /* [4] */, const int32_t* prev_slot, int S_prev,
                    const uint8_t* reuse_mask, int B, int H, int D, int int4_group,
                    int64_t* stats, void* stream);

/* PackedKVCache.evict  (shadowinfer/shadowkv/packed_kv_cache.py:666-740), two steps:
 * skv_evict_count: kept[p] (device int64[4]) = entries of bucket p not in evict_mask,
 *   kept[4] = removed total.
 * skv_evict_compact: stable compaction of every bucket into dst (sized kept[p]),
 *   slot rewritten in place (removed -> -1, kept -> new position).  Pass the same src
 *   array to both calls; a bucket with dst[p].count == src[p].count is left untouched. */
size_t skv_evict_scratch_bytes(int64_t max_bucket_entries);
int skv_evict_count(const skv_bucket* src /* [4] */, const uint8_t* evict_mask, int S, int H,
                    int64_t* kept, void* scratch, size_t scratch_bytes, void* stream);
int skv_evict_compact(const skv_bucket* src /* [4] */, const skv_bucket* dst /* [4] */,
                      const uint8_t* evict_mask, int32_t* slot, int B, int S, int H, int D,
                      int int4_group, void* scratch, size_t scratch_bytes, void* stream);

/* Per-head KV row lists for skv_packed_attention: rows int32[H*S] (slot encoding, stored
 * entries of head h grouped by precision fp32, fp16, int8, int4, token order inside a group),
 * counts int32[H*5] (stored entries per precision, evicted entries).  Derived from the cache's
 * slot map; no reference counterpart (the reference never attends over the packed form). */
int skv_head_index(const int32_t* slot, int S, int H, int32_t* rows, int32_t* counts, void* stream);

/* Attention over the packed cache: O = softmax(Q K^T * scale) V, non-causal, with evicted
 * entries as zero K/V rows -- the result of PackedKVCache.unpack()
 * (shadowinfer/shadowkv/packed_kv_cache.py:535-577) fed to SimpleDiffusionLLM._compute_block's
 * attention (shadowinfer/models/simple_diffusion_llm.py:165-169), without materialising the
 * dense fp32 K/V.  The packed rows of each head are dequantised once into fp16 tensor-core tiles
 * in `scratch` (at least skv_packed_attention_scratch_bytes bytes, 16-byte aligned), which
 * every query tile of the head then reads: K and V in fp16, plus, for the 16 channels of
 * largest max |K| in each KV head, lo = RNE(k - RNE(k)) in a tile of its own, which one extra
 * MMA (K = 16) contracts with the same channels of Q -- channel outliers of K would otherwise
 * make fp16's 2^-11 rounding of K the dominant error (tiles of fp16 entries only are exact and
 * skip it).  The scratch also holds the per-head channel maxima and selection.
 * q fp16 [B,H,S_q,D], out fp32 [B,H,S_q,D]; D = 64 or 128; error_flag (device int32) is cleared
 * and set non-zero if a pipeline wait timed out (results then invalid). */
size_t skv_packed_attention_scratch_bytes(int B, int H, int S_kv, int D);
int skv_packed_attention(const void* q, int B, int H, int S_q, int D, const skv_bucket* buckets /* [4] */,
                         int S_kv, int int4_group, const int32_t* rows, const int32_t* counts, float scale,
                         void* scratch, size_t scratch_bytes, float* out, int32_t* error_flag, void* stream);

/* The two halves of skv_packed_attention, for callers that attend several query blocks over
 * one unchanged cache (stage once, attend many times) or time the halves separately.
 * skv_stage_kv_tiles: dequantises every stored row into the fp16 tiles in `scratch`.
 * skv_attend_kv_tiles: the tensor-core attention over tiles staged for the same rows/counts. */
int skv_stage_kv_tiles(const skv_bucket* buckets /* [4] */, int B, int H, int S_kv, int D, int int4_group,
                       const int32_t* rows, const int32_t* counts, void* scratch, size_t scratch_bytes, void* stream);
int skv_attend_kv_tiles(const void* q, int B, int H, int S_q, int D, int S_kv, const int32_t* rows,
                        const int32_t* counts, float scale, const void* scratch, size_t scratch_bytes, float* out,
                        int32_t* error_flag, void* stream);

/* Grouped-query attention over a packed cache plus this step's own dense K/V: the attention
 * of shadowinfer/models/diffusion_llama.py:376-390 and simple_diffusion_llm.py:160-169
 * (cat(past, new) -> repeat_kv -> softmax(q k^T * scale) v) with the past read from the packed
 * buckets.  q fp16 [B, H_q, S_q, D]; the cache has H_kv heads (H_q % H_kv == 0, query head h
 * reads KV head h / (H_q / H_kv)); rows/counts from skv_head_index over the cache's S_kv
 * tokens; k_new / v_new float [B, H_kv, S_new, D] (16-byte aligned; NULL when S_new == 0).
 * Scratch: skv_packed_attention_scratch_bytes(B, H_kv, S_kv + S_new, D). */
int skv_stage_kv_tiles_gqa(const skv_bucket* buckets, int B, int H_kv, int S_kv, int D, int int4_group,
                           const int32_t* rows, const int32_t* counts, const float* k_new, const float* v_new,
                           int S_new, void* scratch, size_t scratch_bytes, int flags, void* stream);
int skv_attend_kv_tiles_gqa(const void* q, int B, int H_q, int S_q, int D, int H_kv, int S_kv, const int32_t* rows,
                            const int32_t* counts, int S_new, float scale, const void* scratch, size_t scratch_bytes,
                            float* out, int32_t* error_flag, int max_ctas, int flags, void* stream);
/* The attention with its outputs stored into n_peers buffers [B, H_out, S_q, D] (device array of
 * device pointers: every rank's output buffer, mapped into this process), this call's query heads
 * at [head_offset, head_offset + H_q): the head-sharded all-gather of the outputs fused into the
 * epilogue (plain stores over NVLink; no multicast).  The buffers are complete once every
 * rank's call has finished. */
int skv_attend_kv_tiles_peers(const void* q, int B, int H_q, int S_q, int D, int H_kv, int S_kv, const int32_t* rows,
                              const int32_t* counts, int S_new, float scale, const void* scratch,
                              size_t scratch_bytes, float* const* out_peers, int n_peers, int head_offset,
                              int H_out, int32_t* error_flag, int max_ctas, int flags, void* stream);
/* Peer mappings for out_peers (CUDA IPC between the processes of one node).  export: the
 * skv_ipc_handle_bytes() handle of the allocation holding ptr and ptr's byte offset in it.
 * open (on the device that will launch the kernel): maps another process's exported buffer
 * with peer access from the current device; *ptr = mapping + offset, *base is what
 * skv_ipc_close takes.  A process opens each peer allocation once. */
int skv_ipc_handle_bytes(void);
int skv_ipc_export(const void* ptr, void* handle, int64_t* offset);
int skv_ipc_open(const void* handle, int64_t offset, void** base, void** ptr);
int skv_ipc_close(void* base);
/* The plain exchange, for measuring the fused epilogue against it: bytes of src (device, this
 * rank's share) stored at byte offset dst_offset of each of the n_dst buffers whose addresses
 * dst_ptrs (device int64[n_dst], e.g. a PeerOutputs' ptrs) holds -- this rank's own buffer and
 * its peers' over NVLink.  Every 16-byte chunk is loaded once; no load reads peer memory.
 * src, bytes and dst_offset 16-byte multiples; the destinations 16-byte aligned. */
int skv_peer_store(const void* src, int64_t bytes, const int64_t* dst_ptrs, int n_dst, int64_t dst_offset,
                   void* stream);
/* max_ctas: CTAs of the persistent attention kernel (0 = one per SM); fewer leave SMs free for
 * work that should run beside it (e.g. the NCCL all-gather of the previous layer's outputs).
 * flags (the _gqa / _peers entry points; staging and attention take the same flags):
 *   0                -- the default: the 16 largest channels of K per KV head also contribute their
 *                       fp16 lo part (one extra K = 16 MMA per score tile), which keeps relative L2
 *                       within 1e-3 of the fp32 reference also with channel outliers in K;
 *   SKV_ATTN_FAST_K  -- K in fp16 only: no channel selection and no extra MMA, but K enters the
 *                       scores with fp16's 2^-11 relative error, which outlier channels of K turn
 *                       into ~2e-3 relative L2 on the long-context workload. */
#define SKV_ATTN_FAST_K 1
/*   SKV_ATTN_ONE_TILE -- the single-query-tile pipeline (units of 128 queries, two score buffers,
 *                       the next step's scores computed during this step's softmax) instead of the
 *                       default two-tile one (units of 256 queries, one score buffer per tile):
 *                       slower on long sequences (twice the K/V tile traffic), slightly faster on
 *                       short query blocks. */
#define SKV_ATTN_ONE_TILE 2
/*   SKV_ATTN_FMA_EXP  -- two-tile pipeline: one column pair in four computes its softmax
 *                       exponentials with a polynomial on the FMA pipe (relative error <= 7.5e-5)
 *                       instead of the MUFU. */
#define SKV_ATTN_FMA_EXP 4
/*   SKV_ATTN_PAIR     -- head_dim 128: the CTA-pair pipeline.  Two CTAs (one cluster) take a unit of
 *                       256 queries, one 128-row query tile each; the tensor-core MMAs are issued for
 *                       both at once (M = 256), each CTA loading half of every staged K and V tile,
 *                       so a CTA's TMEM holds two score buffers and the scores run two KV steps ahead
 *                       of the P V products; the tile's softmax is split over eight warps.  Takes no
 *                       other pipeline flag (FAST_K and OUT_F16 may be combined); slower than the
 *                       default on B200 (its M = 256 MMAs of N = 128 are issue-bound). */
#define SKV_ATTN_PAIR 8
/*   SKV_ATTN_OUT_F16  -- the output (`out`, and with peers every rank's buffer) is written as fp16,
 *                       each value rounded to nearest even from the fp32 result: half the bytes
 *                       to store and, head-sharded, to send over NVLink.  The pointers keep their
 *                       float* type in the signatures; the buffers must hold B*H*S_q*D halves. */
#define SKV_ATTN_OUT_F16 16
int skv_packed_attention_gqa(const void* q, int B, int H_q, int S_q, int D, const skv_bucket* buckets, int H_kv,
                             int S_kv, int int4_group, const int32_t* rows, const int32_t* counts,
                             const float* k_new, const float* v_new, int S_new, float scale, void* scratch,
                             size_t scratch_bytes, float* out, int32_t* error_flag, int max_ctas, int flags,
                             void* stream);

/* ---- cross-layer budget: KVCacheManager.enforce_global_budget
 * (shadowinfer/shadowkv/kv_cache_manager.py:129-200).  The reference sorts every non-sink
 * (layer, token, head) by importance and evicts from the front in batches, re-reading usage
 * after each batch; these three calls give the bytes freed by the first k candidates and the
 * candidates themselves without a sort. */

/* One layer's candidates, tokens sink..S_m-1 (token-major, then head) of an importance matrix
 * float [S_m, H_m]: score[i] = importance, weight[i] = entry_cost[code] of the cache entry in
 * slot int32 [S_c, H_c] (slot may be NULL; 0 when absent or outside the cache).  Writes
 * (S_m - sink) * H_m values (nothing when sink >= S_m). */
int skv_budget_candidates(const float* importance, int S_m, int H_m, const int32_t* slot, int S_c, int H_c,
                          int sink_tokens, const int64_t* entry_cost /* host [4] */, float* score,
                          int64_t* weight, void* stream);
/* k-th smallest key (score, position) of n candidates (1 <= k <= n, n < 2^31) and the summed
 * weight of the k smallest: result int64[2] (device) = {weight sum, key}; -1 on an internal
 * timeout.  Ties in score keep list order, as the reference's stable sort does. */
size_t skv_rank_select_scratch_bytes(int64_t n);
int skv_rank_select(const float* score, const int64_t* weight, int64_t n, int64_t k, void* scratch,
                    size_t scratch_bytes, int64_t* result, void* stream);
/* mask[i] = 1 for the candidates at or below the key in result (from skv_rank_select). */
int skv_mark_smallest(const float* score, int64_t n, const int64_t* result, uint8_t* mask, void* stream);

/* ---------------------------------------------------------------------------------------
 * Paged KV store  (shadowinfer/shadowkv/paged_kv_store.py)
 *
 * A page holds the rows of one precision for consecutive tokens.  Payload slab
 * [B, H, cap, row]: row = D float | D half | D int8 | ceil(D/2) int4 bytes ((q+8) high nibble
 * first, a zero nibble after an odd last value); scales float [B, H, cap] (int8) or
 * [B, H, cap, D/G] (int4, G the effective group of packed_kv_cache.py:307).
 * ------------------------------------------------------------------------------------- */
/* Page payload pointers should be 16-byte aligned and scale pointers 4-byte aligned (the
 * kernels use 16-byte vectors then, value-by-value access otherwise). */
typedef struct skv_page_desc {
    void* k;              /* payload row of the page's first token in block (b, h) = (0, 0) */
    void* v;
    float* scale_k;       /* scale row of that token (NULL for fp32 / fp16 pages) */
    float* scale_v;
    int64_t start_token;  /* global position of the page's first token */
    int32_t num_tokens;   /* tokens in the page */
    int32_t row_stride;   /* rows from one (b, h) block to the next (the slab's cap) */
    int32_t precision;    /* 0 fp32, 1 fp16, 2 int8, 3 int4 */
    int32_t reserved[3];
} skv_page_desc;          /* 64 bytes */

typedef struct skv_page_write {
    skv_page_desc page;   /* destination page, num_tokens as after the write */
    int64_t src_token;    /* first source token of the run */
    int32_t dst_row;      /* first row inside the page */
    int32_t rows;         /* rows to write (>= 1) */
    int32_t table_pos;    /* page-table entry that receives `page` after the launch, or -1 */
    int32_t reserved;
} skv_page_write;         /* 88 bytes */

/* PagedKVStore._quantize_chunk + the page merge of append / the row copy of rewrite_tokens
 * (paged_kv_store.py:189-224, :248-307, :408-448): quantises K/V float [B, H, T_src, D] rows
 * [src_token, src_token + rows) of every write into its page's rows [dst_row, dst_row + rows),
 * bit-identical to Quantizer.quantize_int8 / quantize_int4 per (b, h, token) row.  `writes` is
 * HOST memory, read during the call; `table` (device, may be NULL) receives each write's
 * page descriptor at table_pos. */
int skv_paged_write(const float* k, const float* v, int B, int H, int64_t T_src, int D, int int4_group_size,
                    const skv_page_write* writes, int n_writes, skv_page_desc* table, void* stream);

/* PagedKVStore.gather  (paged_kv_store.py:326-402): dense float K/V [B, H, s_out, D] from the
 * n_pages descriptors of `table` (device, token order, non-overlapping); tokens no page holds
 * are zero.  max_span_tokens >= max over pages j of (start_j - end_{j-1}) + num_tokens_j and
 * >= s_out - end_last. */
int skv_paged_gather(const skv_page_desc* table, int n_pages, int B, int H, int D, int int4_group_size,
                     int64_t s_out, int64_t max_span_tokens, float* k_out, float* v_out, void* stream);

/* The head-row zeroing of PagedKVStore._plan_eviction  (paged_kv_store.py:662-672):
 * items int32 [n_items, 3] (device) = {table entry, row inside the page, head}; zeroes that
 * row of K and V in every batch (0x88 bytes for int4 pages).  *error_flag (device int32) is
 * set to 1 if an item lies outside the table or its page. */
int skv_paged_clear_heads(const skv_page_desc* table, int n_pages, const int32_t* items, int64_t n_items, int B,
                          int H, int D, int* error_flag, void* stream);

/* ---------------------------------------------------------------------------------------
 * Decision inputs of the agent
 * ------------------------------------------------------------------------------------- */
/* ShadowKVAgent.decide_reuse_per_token  (shadowinfer/shadowkv/shadowkv_agent.py:1165-1256):
 * K/V float [B,H,S,D] of the current and previous step, importance float [S,H];
 * effective_threshold = base(mode) * (1 - 0.5*progress) * (1 - 0.3*qdrift) as the reference
 * computes it on the host.  mask uint8 [S,H] = drift < max(thr * (1 - 0.3*clamp(imp,0,1)), 1e-5);
 * drift float [S,H] (may be NULL); counts int64[4] (device) = {full-reuse tokens, partial,
 * none, reused entries}. */
int skv_reuse_decide(const float* k_cur, const float* v_cur, const float* k_prev, const float* v_prev, int B, int H,
                     int S, int D, const float* importance, double effective_threshold, uint8_t* mask, float* drift,
                     int64_t* counts, void* stream);

/* compute_irap_importance  (shadowinfer/shadowkv/importance_model.py:37-134) with the agent's input
 * contract (shadowkv_agent.py:894-965): scores float [B,H,Sq,Sk]; input_mode 0 = probabilities
 * used as given, 1 = logits (softmax of the NaN-cleaned rows), 2 = probabilities divided by
 * their row sum clamped to 1e-10.  ema_prev float [S_prev,H] or NULL (cold start).
 * importance, ema float [Sk,H]; delta_parts double[2] (device) = {sum (ema - prev)^2,
 * sum prev^2} for delta_a.  Ties in the EMA rank by token index. */
size_t skv_irap_scratch_bytes(int B, int H, int Sq, int Sk);
int skv_irap_importance(const float* scores, int B, int H, int Sq, int Sk, int input_mode, const float* ema_prev,
                        int S_prev, double irap_decay, double entropy_weight, int sink_tokens, double layer_factor,
                        void* scratch, size_t scratch_bytes, float* importance, float* ema, double* delta_parts,
                        void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SHADOWKV_B200_H */
