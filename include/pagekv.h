/*
 * pagekv.h - C ABI of libpagekv, a B200 (sm_100a) implementation of pagellm's paged
 * KV-cache hot path (pagellm: src/pagellm/cache/paged.py).
 *
 * Conventions
 *   - Every entry point returns an int status (PK_OK = 0). On failure a message is
 *     available from pk_last_error() (thread-local, valid until the next failing call).
 *   - "dev" pointers are CUDA device pointers on the pool's device; "host" pointers are
 *     ordinary host memory (pinned memory makes the copies asynchronous).
 *   - stream is a cudaStream_t passed as void* (NULL = legacy default stream).
 *     Calls are asynchronous with respect to the host unless stated otherwise.
 *   - Query / key / value / output rows are float32, row-major:
 *       q, out: [rows][n_heads][head_dim]     k, v: [rows][n_kv_heads][head_dim]
 *   - The pool stores K and V as [layers][num_blocks][block_size][n_kv_heads][head_dim]
 *     in float32 or bfloat16; a token's slot is block * block_size + offset.
 *   - Global state: the thread-local error message, the one-shot test hook
 *     pk_test_inject_launch_failure, and the device array (and its per-device address
 *     cache) of pk_decode_attend_static. Pools, batches and block managers are independent
 *     objects; none needs locking for the single-engine-thread use pagellm makes of its
 *     cache.
 */
#ifndef PAGEKV_H
#define PAGEKV_H

#include <stddef.h>
#include <stdint.h>

#if defined(PK_BUILD)
#define PK_API __attribute__((visibility("default")))
#else
#define PK_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum pk_status {
    PK_OK = 0,
    PK_ERR_INVALID_ARG = 1,   /* bad shape / dtype / pointer: pagellm raises ValueError   */
    PK_ERR_OUT_OF_RANGE = 2,  /* block id, slot or position outside the pool or table     */
    PK_ERR_CUDA = 3,          /* a CUDA runtime call failed                                 */
    PK_ERR_OUT_OF_BLOCKS = 4, /* free list and evictable set empty: pagellm's OutOfBlocks   */
    PK_ERR_DOUBLE_FREE = 5,   /* decref of a block whose ref count is 0                     */
    PK_ERR_TIMEOUT = 6,       /* a bounded device-side wait gave up (kernel returned early) */
    PK_ERR_DUPLICATE = 7,     /* sequence id already has a table                            */
    PK_ERR_NOT_FOUND = 8,     /* unknown sequence id                                        */
    PK_ERR_UNSUPPORTED = 9    /* configuration this build does not handle                   */
};

enum pk_dtype { PK_F32 = 0, PK_BF16 = 1 };

typedef struct pk_pool pk_pool;
typedef struct pk_batch pk_batch;
typedef struct pk_block_manager pk_block_manager;

/* Message of the last failing call on this thread ("" if none). */
PK_API const char* pk_last_error(void);
/* ABI version: bumped on any incompatible change. */
PK_API int pk_abi_version(void);

/* ---------------------------------------------------------------- pool
 * Replaces PagedKVPool (cache/paged.py:282-300). K and V are allocated on `device`
 * and zero-filled, as pagellm's np.zeros pool is. */
PK_API int pk_pool_create(int n_layers, int64_t num_blocks, int block_size, int n_kv_heads,
                   int head_dim, int dtype, int device, pk_pool** out);
PK_API int pk_pool_destroy(pk_pool* pool);
/* Device base pointers of K and V and the total bytes (PagedKVPool.nbytes, :298-300). */
PK_API int pk_pool_buffers(const pk_pool* pool, void** k_dev, void** v_dev, int64_t* nbytes);
/* Whether the tensor-core attention kernel serves this pool (bf16, head_dim 64/128/256,
 * block_size a multiple of 16, <= 8 KV heads), its shared-memory layout and pipeline depth,
 * and why not when it does not. */
PK_API int pk_pool_tc_info(const pk_pool* pool, int* enabled, int* per_head_layout, int* stages,
                    const char** why);
/* Copy-on-write block copies over all layers (PagedKVPool.copy_block, :294-296, driven by
 * engine/llm_engine.py:205-206). pairs_host: npairs (src, dst) int64 pairs, applied as if
 * in list order. Ids are checked on the host before anything is launched. */
PK_API int pk_pool_copy_blocks(pk_pool* pool, const int64_t* pairs_host, int64_t npairs, void* stream);
/* Same, with the pairs already on the device (no validation beyond npairs >= 0;
 * every id must be in [0, num_blocks) and no dst may also be a src). */
PK_API int pk_pool_copy_blocks_dev(pk_pool* pool, const int64_t* pairs_dev, int64_t npairs,
                            void* stream);
/* Scatter rows into one layer at the given slots (PagedBatch.write_and_attend,
 * :443-444): pool.k_flat[layer, slots] = k. k_dev/v_dev float32 [n][n_kv_heads][head_dim];
 * slots_dev int64. Slots are not range-checked here (pk_batch_plan checks its own). */
PK_API int pk_pool_append(pk_pool* pool, int layer, const float* k_dev, const float* v_dev,
                   const int64_t* slots_dev, int64_t n, void* stream);

/* slot_mapping (cache/paged.py:303-306): slots[i] = table[p / bs] * bs + p % bs for
 * p = positions[i]. Device arrays. A position outside [0, table_len * bs) yields slot
 * -1 and, if err_dev is not NULL, sets *err_dev to 1. */
PK_API int pk_slot_mapping(const int32_t* table_dev, int64_t table_len, const int64_t* positions_dev,
                    int64_t n, int block_size, int64_t* slots_dev, int32_t* err_dev,
                    void* stream);

/* ---------------------------------------------------------------- batch
 * Replaces PagedBatch (cache/paged.py:383-464): the per-step view of a set of sequences.
 * A batch object is reusable across steps; its device buffers only grow. */
PK_API int pk_batch_create(pk_pool* pool, pk_batch** out);
PK_API int pk_batch_destroy(pk_batch* batch);
/* PagedBatch.__init__ (:397-439). Host arrays: block tables in CSR form
 * (table_indptr[nseq+1] int64, table_ids int32), starts[nseq], n_new[nseq] (int64).
 * Sequence i owns rows offsets[i] .. offsets[i]+n_new[i]-1 at positions starts[i]...
 * Validates every table (ids in range, long enough for starts[i]+n_new[i] tokens), uploads
 * it, computes positions and slots on the device and plans the attention kernels.
 * Returns the number of rows in *n_rows. */
PK_API int pk_batch_plan(pk_batch* batch, int nseq, const int64_t* table_indptr,
                  const int32_t* table_ids, const int64_t* starts, const int64_t* n_new,
                  int64_t* n_rows, void* stream);
/* Device pointers of the step's int64 positions and slots (valid until the next plan). */
PK_API int pk_batch_rows(const pk_batch* batch, const int64_t** positions_dev, const int64_t** slots_dev);
/* PagedBatch.write_and_attend (:441-464) for one layer: append k/v at the step's slots,
 * then causal GQA attention of every row over its sequence's cached prefix plus the
 * step's own rows. q_dev/out_dev [rows][n_heads][head_dim], k_dev/v_dev
 * [rows][n_kv_heads][head_dim], float32, device. */
PK_API int pk_batch_write_and_attend(pk_batch* batch, int layer, int n_heads, const float* q_dev,
                              const float* k_dev, const float* v_dev, float* out_dev,
                              void* stream);
/* Attention only (no append): the read half of write_and_attend. */
PK_API int pk_batch_attend(pk_batch* batch, int layer, int n_heads, const float* q_dev, float* out_dev,
                    void* stream);
/* write_and_attend from HOST buffers: uploads q/k/v, runs the layer and downloads out,
 * all on `stream`; returns after `out_host` is filled (synchronous). When `out_host` lies
 * wholly inside one page-locked allocation the device can address (cudaMallocHost,
 * cudaHostAlloc, cudaHostRegister), the kernels store the result into it directly, so the
 * transfer overlaps the attention; steps with a shared-prefix pass, and pageable buffers,
 * get a device-to-host copy after the kernels. */
PK_API int pk_batch_write_and_attend_host(pk_batch* batch, int layer, int n_heads, const float* q_host,
                                   const float* k_host, const float* v_host, float* out_host,
                                   void* stream);
/* Reads (and clears) the device error word that bounded waits set on timeout.
 * Synchronises `stream`. Returns PK_ERR_TIMEOUT if any kernel of this batch gave up. */
PK_API int pk_batch_check(pk_batch* batch, void* stream);
/* Planning statistics of the last plan: [0] rows, [1] units on the tensor-core split-KV
 * kernel, [2] its CTAs, [3] its total K/V blocks, [4] units split across CTAs (merged),
 * [5] rows on the CUDA-core kernel, [6] kernels launched by the last call, [7] wide-tile
 * work items (128 query rows each) on the tcgen05 kernel. */
PK_API int pk_batch_stats(const pk_batch* batch, int64_t* stats8);
/* Bytes moved by the last pk_batch_write_and_attend_host: [0] host to device, [1] device to
 * host by a copy after the kernels, [2] stored by the kernels straight into the caller's
 * page-locked result buffer. */
PK_API int pk_batch_io_stats(const pk_batch* batch, int64_t* stats3);
/* Shared-prefix (cascade) attention - no counterpart in pagellm, whose attention reads every
 * sequence's keys separately (cache/paged.py:454-463): sequences of a step whose block
 * tables begin with the same block ids (forks, prefix-cache hits) have the shared keys
 * attended once per 128 query rows on the tcgen05 kernel, merged with the split-KV result
 * for the rest of each sequence. `mode`: 0 off, 1 (default) where a cost estimate says it
 * is faster than reading the prefix once per sequence, 2 for every eligible group; it
 * applies from the next plan. pk_batch_prefix_stats: [0] prefix groups, [1] shared-prefix
 * work items, [2] shared keys summed over the groups, [3] sum over the groups of
 * (query tokens x shared keys), the work the shared-prefix pass does per query head. */
PK_API int pk_batch_set_prefix_sharing(pk_batch* batch, int mode);
PK_API int pk_batch_prefix_stats(const pk_batch* batch, int64_t* stats4);

/* Per-kernel timing of this batch's own launches: with profiling on, CUDA events are
 * recorded on the launching stream around every kernel. pk_batch_profile_read synchronises
 * them and returns, per kind [0 append, 1 split-KV tensor-core attention, 2 partial merge,
 * 3 CUDA-core attention, 4 wide-tile tcgen05 attention], the summed milliseconds and launch
 * counts, then resets. */
PK_API int pk_batch_profile(pk_batch* batch, int enable);
PK_API int pk_batch_profile_read(pk_batch* batch, double* ms5, int64_t* count5);
/* Self-test of the bounded device waits (no counterpart in pagellm): launches a kernel
 * that waits on a barrier phase nothing completes; the wait gives up after limit_ns
 * (<= 2 s) and the kernel reports it. *timed_out = 1 when that happened as designed.
 * Synchronises the device. */
PK_API int pk_selftest_bounded_wait(int device, int64_t limit_ns, int* timed_out);
/* Host-side fault injection for tests (no counterpart in pagellm): the next attention call
 * (write_and_attend / attend, any batch) returns PK_ERR_CUDA before launching anything, as
 * a failed launch would; later calls run normally. No GPU fault is involved. */
PK_API int pk_test_inject_launch_failure(void);
/* Host-only dry run of the split-KV planner (no device needed). The units' blocks, end to
 * end, are cut into contiguous CTA ranges; a range costs its blocks plus
 * `unit_switch_blocks` per unit boundary inside it (a CTA that crosses into another unit
 * reloads queries, publishes a partial and usually merges the unit it ends in); the cut
 * minimises the largest cost over at most n = max(1, min(max_ctas, total, max(total / 16,
 * ceil(n_units / 3)))) CTAs. Writes *ncta (<= n) and, if cta_first_block is not NULL, the
 * first block of each CTA [*ncta + 1] (the caller provides n + 1 entries). */
PK_API int pk_plan_partition(const int64_t* unit_blocks, int64_t n_units, int max_ctas, int unit_switch_blocks,
                             int64_t* cta_first_block, int* ncta);


/* Head-sharded output gather (no counterpart in pagellm, which runs in one process): every
 * rank of `world` computed the query heads [r*H/world, (r+1)*H/world) of all `rows` rows;
 * after an all-gather of those [rows][H/world][head_dim] slices into src_dev
 * [world][rows][row_floats] (row_floats = H/world * head_dim), dst_dev receives the
 * [rows][H][head_dim] output PagedBatch.write_and_attend (cache/paged.py:441-464) returns.
 * float32 device buffers, 16-byte aligned, row_floats a multiple of 4. */
PK_API int pk_gather_interleave(const float* src_dev, float* dst_dev, int world, int64_t rows,
                                int64_t row_floats, void* stream);

/* Head-sharded output exchange over peer memory (no counterpart in pagellm, which runs in one
 * process). Each of `world` ranks (one process per GPU, GPUs with peer access over NVLink)
 * creates one on its device with room for a [rows][H][head_dim] float32 result (`bytes`,
 * a multiple of 16), passes the 64-byte IPC handle from pk_peer_gather_handle to every other
 * rank (any host-side channel), and calls pk_peer_gather_open with all `world` handles in
 * rank order. pk_peer_gather_heads then runs one launch per step: this rank's slice
 * [rows][row_floats] (row_floats = H/world * head_dim, a multiple of 4) is stored into every
 * rank's result buffer at head offset rank * H/world, and the launch completes once every
 * rank's slice has landed here, so *result_dev ([rows][H][head_dim], the output of
 * PagedBatch.write_and_attend, cache/paged.py:441-464) is complete in stream order. The two
 * result buffers alternate by step; every rank calls it for every step, in the same order.
 * A peer that does not signal within 1 s makes the launch record a timeout, reported by
 * pk_peer_gather_check (which synchronises the stream). */
typedef struct pk_peer_gather pk_peer_gather;
PK_API int pk_peer_gather_create(int device, int world, int rank, int64_t bytes, pk_peer_gather** out);
PK_API int pk_peer_gather_handle(const pk_peer_gather* gather, uint8_t* handle64);
PK_API int pk_peer_gather_open(pk_peer_gather* gather, const uint8_t* handles);
PK_API int pk_peer_gather_heads(pk_peer_gather* gather, const float* slice_dev, int64_t rows, int64_t row_floats,
                                float** result_dev, void* stream);
PK_API int pk_peer_gather_check(pk_peer_gather* gather, void* stream);
PK_API int pk_peer_gather_destroy(pk_peer_gather* gather);
/* The head-sharded step with the exchange fused into the attention: this rank's
 * pk_batch_write_and_attend (PagedBatch.write_and_attend, cache/paged.py:441-464, over the
 * rank's n_heads = H/world query heads) whose kernel stores every output row straight into
 * every rank's result buffer at head offset rank * n_heads and, once all its rows are stored,
 * exchanges the step's completion flags with the other ranks - one launch per step instead of
 * attention + pk_peer_gather_heads. A step the split-KV kernel does not compute alone (chunks,
 * shared prefixes, fp32 pools) computes the slice into batch scratch and then exchanges it with
 * pk_peer_gather_heads. *result_dev, the timeout report and the calling rules are those of
 * pk_peer_gather_heads; at most 8 ranks. */
PK_API int pk_peer_gather_write_and_attend(pk_peer_gather* gather, pk_batch* batch, int layer, int n_heads,
                                           const float* q_dev, const float* k_dev, const float* v_dev,
                                           float** result_dev, void* stream);

/* Decode attention that allocates nothing. No counterpart in the reference: pagellm has no
 * device memory at all. For callers that cannot call cudaMalloc - a serving framework that
 * hands out all of HBM through its own caching allocator, or a plugin host that forbids
 * cudaMalloc/cudaFree on the request path because cudaFree synchronises the device.
 * Sequence i has ctx_lens[i] tokens in the pool (its table: table_ids[table_indptr[i] ..],
 * host arrays); its one query row q_dev[i] sits at position ctx_lens[i]-1 and attends over
 * positions 0..ctx_lens[i]-1 (no append); out_dev[i] receives the result. Requires a pool
 * the tensor-core kernel serves and at most 8 query heads per KV head.
 * All scratch (tables, plan, partial results) lives in a 16 MiB array that every GPU
 * loading this library holds until exit; a call that needs more, or has more than 512
 * sequences, fails with PK_ERR_INVALID_ARG before launching anything. Every call on a device
 * shares that array and leaves it dirty (the error word is cleared per call): calls that
 * overlap on the GPU race. The call uploads from host memory of the call itself, so it cannot be
 * captured into a CUDA graph: on a capturing stream it returns PK_ERR_UNSUPPORTED before doing
 * anything. err_dev (required, a device int the caller owns and clears):
 * set to 1 if a bounded device wait gave up, so a timeout is never lost.
 * Pageable table_ids / ctx arrays are copied before return; pinned ones must stay valid until
 * the stream has run the call. */
PK_API int pk_decode_attend_static(const pk_pool* pool, int layer, int n_heads, int nseq,
                                   const int64_t* table_indptr, const int32_t* table_ids,
                                   const int64_t* ctx_lens, const float* q_dev, float* out_dev,
                                   int32_t* err_dev, void* stream);

/* ---------------------------------------------------------------- block bookkeeping
 * Host-side replacement of BlockAllocator and BlockManager (cache/paged.py:47-274): FIFO
 * free list, int64 ref counts, LRU set of evictable cached blocks, hash -> block map and
 * per-sequence tables, in C++. Hashing (block_hash chains, paged.py:120-131) stays with the
 * caller, which passes digests as (bytes, length). No CUDA involved; messages of failing
 * calls come from pk_bm_last_error(). */
PK_API const char* pk_bm_last_error(void);
PK_API int pk_bm_create(int64_t num_blocks, int block_size, int enable_prefix_caching,
                        pk_block_manager** out);
PK_API int pk_bm_destroy(pk_block_manager* m);
/* BlockAllocator.allocate / incref / decref / lookup / register (paged.py:73-117).
 * allocate -> PK_ERR_OUT_OF_BLOCKS when nothing is free or evictable; decref of a block with
 * ref 0 -> PK_ERR_DOUBLE_FREE; incref of an unreferenced block that is not cached ->
 * PK_ERR_NOT_FOUND; lookup writes -1 when the hash is unknown or caching is off. */
PK_API int pk_bm_allocate_block(pk_block_manager* m, int32_t* block);
PK_API int pk_bm_incref(pk_block_manager* m, int32_t block);
PK_API int pk_bm_decref(pk_block_manager* m, int32_t block);
PK_API int pk_bm_lookup(pk_block_manager* m, const uint8_t* hash, int64_t len, int32_t* block);
PK_API int pk_bm_register(pk_block_manager* m, int32_t block, const uint8_t* hash, int64_t len);
/* [0] num_free (paged.py:63-66), [1] free-list length, [2] evictable, [3] cached hashes,
 * [4] prefix_hits, [5] prefix_queries, [6] sequences with a table. */
PK_API int pk_bm_counts(const pk_block_manager* m, int64_t* counts7);
/* Live pointer to the int64 ref counts (BlockAllocator.ref, paged.py:54). */
PK_API int pk_bm_refcounts(pk_block_manager* m, int64_t** ref);
/* Free list in FIFO order (paged.py:53) / evictable blocks oldest first (paged.py:57). */
PK_API int pk_bm_free_list(const pk_block_manager* m, int32_t* out, int64_t cap, int64_t* n);
PK_API int pk_bm_evictable_list(const pk_block_manager* m, int32_t* out, int64_t cap, int64_t* n);
/* Hash a block is published under (BlockAllocator.block_hash, paged.py:55); *len = -1 if none. */
PK_API int pk_bm_block_hash(const pk_block_manager* m, int32_t block, uint8_t* out, int64_t cap,
                            int64_t* len);
PK_API int pk_bm_add_prefix_stats(pk_block_manager* m, int64_t hits, int64_t queries);
/* BlockManager.allocate (paged.py:187-203) given the caller's plan_prefix result. */
PK_API int pk_bm_seq_allocate(pk_block_manager* m, int64_t seq, int64_t n_tokens,
                              const int32_t* hits, int64_t n_hits, const uint8_t* hashes,
                              int64_t hash_len, int64_t* cached_tokens);
/* BlockManager.can_append (paged.py:206-213). */
PK_API int pk_bm_can_append(pk_block_manager* m, int64_t seq, int64_t n_tokens, int* ok);
/* BlockManager.ensure_capacity (paged.py:215-239): (src, dst) copy pairs into pairs_out. */
PK_API int pk_bm_ensure_capacity(pk_block_manager* m, int64_t seq, int64_t n_tokens,
                                 int64_t write_from, int64_t* pairs_out, int64_t cap,
                                 int64_t* npairs);
/* A sequence's hash chain (BlockTable.hashes, paged.py:142-144): length and last digest,
 * or the digest at position i. */
PK_API int pk_bm_seq_hashes(pk_block_manager* m, int64_t seq, int64_t* n, uint8_t* last,
                            int64_t cap, int64_t* last_len);
PK_API int pk_bm_seq_hash_at(pk_block_manager* m, int64_t seq, int64_t i, uint8_t* out,
                             int64_t cap, int64_t* len);
/* BlockManager.mark_computed's bookkeeping (paged.py:251-254): append digests, register. */
PK_API int pk_bm_seq_push_hashes(pk_block_manager* m, int64_t seq, const uint8_t* hashes,
                                 int64_t hash_len, int64_t count);
/* BlockManager.fork (paged.py:257-263) and free (paged.py:265-271). */
PK_API int pk_bm_fork(pk_block_manager* m, int64_t parent, int64_t child);
/* Paged speculative rollback (no counterpart in pagellm's paged cache; pagellm rolls back
 * contiguous caches only: cache/contiguous.py:33-38 truncate, engine/speculative.py:136-137;
 * paged rollback is on its roadmap, README.md:370): keep the first n_tokens of a sequence.
 * Blocks past them are released last block first (as free, cache/paged.py:265-271); the
 * hash chain keeps the remaining full blocks; a kept partial last block published in the
 * prefix cache and held by this sequence alone is unpublished (its next writes change it).
 * n_tokens outside [0, blocks * block_size] -> PK_ERR_INVALID_ARG. */
PK_API int pk_bm_truncate(pk_block_manager* m, int64_t seq, int64_t n_tokens);
PK_API int pk_bm_free_seq(pk_block_manager* m, int64_t seq);
/* BlockManager.block_table (paged.py:273-274); sequence ids with a table. */
PK_API int pk_bm_table(const pk_block_manager* m, int64_t seq, int32_t* out, int64_t cap,
                       int64_t* n);
PK_API int pk_bm_seq_ids(const pk_block_manager* m, int64_t* out, int64_t cap, int64_t* n);
/* Tables of `nseq` sequences as CSR (the input of pk_batch_plan), without a detour through
 * Python lists. ids = NULL sizes the call (*total). */
PK_API int pk_bm_tables_csr(const pk_block_manager* m, const int64_t* seqs, int64_t nseq,
                            int64_t* indptr, int32_t* ids, int64_t cap, int64_t* total);

#ifdef __cplusplus
}
#endif
#endif /* PAGEKV_H */
