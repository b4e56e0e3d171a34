// Internal declarations shared by the libpagekv translation units.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace pk {

// Most query columns (query token x head-in-group) one tensor-core warp carries.
constexpr int kMaxCols = 16;
// Largest number of KV heads the tensor-core kernel maps to warps of one CTA.
constexpr int kTcMaxKvHeads = 8;
constexpr int kWideKeys = 128;  // keys per tile of the wide-tile kernel (a multiple of block_size)

// Parameters of the split-KV tensor-core attention kernel (bf16 pool).
// Head-sharded output exchange fused into the split-KV kernel (n > 0): every output row goes
// to out[0..n) - each rank's result buffer, already offset to this rank's first query head,
// rows out_H heads apart - and when every consumer warp of the launch has stored its rows
// (a system-scope fence, then a count in `done`), the last one writes `epoch` into flag word
// `rank` of every rank (flag_of) and waits, for at most the wait limit, until every rank's
// flag word here (flags) holds it; a timeout sets *err.
constexpr int kMaxOutPeers = 8;
struct PeerOut {
    int n;
    int out_H;
    int rank;
    unsigned int epoch;
    float* out[kMaxOutPeers];
    unsigned int* flag_of[kMaxOutPeers];
    unsigned int* flags;
    unsigned int* done;  // zero between launches; the last warp resets it
    int* err;
};

// A "unit" is a window of at most kMaxCols / g query tokens of one sequence; every unit
// reads the blocks holding positions 0 .. unit_ctx-1 of its sequence. Units' blocks are
// laid end to end and cut into ncta equal ranges, one per CTA.
struct TcParams {
    const float* q;        // [rows][H][D]
    float* out;            // [rows][H][D]
    // [segments][kvh] blocks of kMaxCols * D floats: un-normalised partial sums in fragment
    // order interleaved by lane (accumulator quad j = mt * NT + nt of lane L is float4
    // j * 32 + L of the block)
    float* part_o;
    float* part_ml;        // [segments][kvh][kMaxCols][2]  (running max, sum), log2 domain
    int* err;              // device error word
    const int32_t* indptr;  // [nseq+1] block-table CSR
    const int32_t* ids;     // block ids
    const int32_t* starts;  // [nseq]
    const int32_t* offsets; // [nseq+1] first row of each sequence
    const int32_t* u_seq;   // [nu] sequence of each unit
    const int32_t* u_t0;    // [nu] first query token of the unit within its sequence
    const int32_t* u_n;     // [nu] query tokens in the unit
    const int32_t* u_blk;   // [nu+1] prefix sum of the units' block counts
    // [nu] first block of the sequence the unit reads (blocks before it - a prefix shared
    // with other sequences - are attended by the wide-tile kernel); NULL = all 0.
    const int32_t* u_kb0;
    // [rows][H] log2-domain log-sum-exp of each output row (max + log2(sum)); NULL = not
    // written. The shared-prefix pass merges its partial with the row through it.
    float* lse;
    // [ncta + 1] first block of each CTA's range; NULL = equal ranges [c*T/ncta, (c+1)*T/ncta)
    const int32_t* cta_blk;
    // [nu][2] first and last CTA whose range holds blocks of each unit; NULL = searched in
    // cta_blk (read only by the in-kernel merge)
    const int32_t* u_cta;
    // [nu] packed unit records, two int4 each: {t0, n, kb0, row0}, {qpos0, blk0, blk1, tbase}
    // (row0 = offsets[seq] + t0, qpos0 = starts[seq] + t0, blk0/blk1 = u_blk[u]/u_blk[u + 1],
    // tbase = indptr[seq] + kb0 - blk0, so that block j's id is ids[tbase + j]); NULL =
    // gathered from the arrays above
    const int4* u_meta;
    int nu;
    int total_blocks;
    int ncta;
    int kvh;
    int g;
    int H;
    int bs;
    int stages;
    int virt;              // virtual CTAs per CTA (0 or 1: one); kvh * virt <= kTcMaxKvHeads
    int per_head_layout;   // 0: one TMA box per K/V block, 1: one box per (block, head)
    int64_t layer_slot0;   // first slot of the layer in the flat [layers*num_blocks*bs] axis
    float qscale;          // log2(e) / sqrt(D)
    // In-kernel merge (NULL counters: leave the partials to merge_kernel): zero-initialised
    // counters per (partial slot, KV head) for the first-level groups of a unit's CTAs, and per
    // (unit, KV head) for the second level; both left at zero by the kernel.
    int* counters;
    int* unit_counters;
    // Fused append: fp32 rows [rows][kvh][D] of this step and the layer's bf16 pool bases;
    // NULL k_new = attention only.
    const float* k_new;
    const float* v_new;
    __nv_bfloat16* pool_k;
    __nv_bfloat16* pool_v;
    PeerOut peer;  // n == 0: rows go to `out` (H heads per row)
};

struct MergeParams {
    float* out;
    const float* part_o;
    const float* part_ml;
    const int32_t* offsets;
    const int32_t* u_seq;
    const int32_t* u_t0;
    const int32_t* u_n;
    const int32_t* split_u;   // [nsplit] unit of each split entry
    const int32_t* split_c0;  // first CTA that worked on it
    const int32_t* split_c1;  // last CTA that worked on it
    int kvh;
    int g;
    int H;
    int D;
    int nt;  // n8 tiles of the attention launch that wrote the partials (fragment layout)
};

// CUDA-core attention for any pool dtype / head_dim (float32 pools, odd shapes).
struct GenericParams {
    const float* q;
    float* out;
    const void* pool_k;  // layer base
    const void* pool_v;
    const int32_t* row_seq;
    const int32_t* indptr;
    const int32_t* ids;
    const int32_t* starts;
    const int32_t* offsets;
    const int32_t* rows;  // rows to process (indices into q/out)
    // Fused append (NULL: off): keys at positions >= the sequence's start are read from these
    // fp32 rows [step rows][kvh][D] (rounded to the pool type), and the CTA of (row, first
    // query head of a KV head) stores its row to the pool (pool_k / pool_v layer bases).
    const float* k_new;
    const float* v_new;
    int nrows;
    int H;
    int kvh;
    int D;
    int bs;
    float scale;  // 1/sqrt(D)
};

// Tensor-core (tcgen05) wide-tile attention: one CTA per (work item, KV head); a work
// item is 128 query rows (= 128/g tokens) of one sequence.
struct WideParams {
    const float* q;
    float* out;
    int* err;
    const int32_t* indptr;
    const int32_t* ids;
    const int32_t* w_seq;   // [nitems] sequence whose block table the item reads
    const int32_t* w_tok0;  // [nitems] first entry of the item's query tokens in tok_row/tok_pos
    const int32_t* w_ntok;  // [nitems] query tokens in the item (<= 128/g)
    const int32_t* w_kend;  // [nitems] keys 0..kend-1 of the table are attended
    const int32_t* tok_row; // query/output row of each token
    const int32_t* tok_pos; // absolute position of each token (causal limit)
    // Shared-prefix pass: NULL = write the normalised output; else merge this partial with
    // the output row already written (and its log2-domain log-sum-exp [rows][H] here).
    const float* lse;
    const int32_t* w_pair;     // [pairs][2] items of a pair (second = -1: none), same table
    const int32_t* pair_kend;  // [pairs] keys of the pair (the larger kend of its items)
    const int32_t* cta_seg;    // [nctas+1] this launch's CTAs: segment ranges
    const int32_t* seg;        // [segments][6] pair, head, first/end key tile, slot (-1 whole), pair-head
    float* part_o;             // [slots][2][128][128] un-normalised partial O
    float* part_ml;            // [slots][2][128][2] (max, sum), log2 domain
    // [items * kvh + 1][32 KB] query tiles packed by launch_wide_q_pack (bf16, scaled,
    // in the shared-memory image the MMA reads); tile item * kvh + head, the last all zero
    const uint8_t* qpk;
    int q_zero_tile;
    int nctas;
    int H;
    int kvh;
    int g;
    int bs;
    int64_t layer_slot0;
    float qscale;
};

// Read-only view of a pool's fields for entry points outside pk_api.cu.
struct PoolView {
    int device;
    int n_layers;
    int64_t num_blocks;
    int block_size;
    int kvh;
    int d;
    int dtype;
    int num_sms;
    bool tc_ok;
    int tc_per_head;
    int tc_stages;
    int tc_virt;
    size_t tc_smem;
    const CUtensorMap* tmk;
    const CUtensorMap* tmv;
};

cudaError_t launch_tc_attention(int D, int NT, const CUtensorMap* tmk, const CUtensorMap* tmv,
                                const TcParams& p, size_t smem, cudaStream_t st);
size_t tc_smem_bytes(int D, int bs, int kvh, int stages, int virt);
// Shared memory a launch with the fused head exchange needs beyond tc_smem_bytes (each consumer
// warp's staging of 4 output rows, and alignment slack).
size_t tc_peer_stage_bytes(int D);
cudaError_t launch_merge(const MergeParams& p, int nsplit, cudaStream_t st);
size_t wide_smem_bytes();
cudaError_t launch_wide_attention(const CUtensorMap* tmk1, const CUtensorMap* tmv1, const WideParams& p,
                                  cudaStream_t st);
// Bytes of one packed query tile of the wide-tile kernel (128 rows x 128 dims, bf16).
constexpr int kWideQTileBytes = 128 * 128 * 2;
// Packs the query tiles of `nitems` wide-tile items (all KV heads) plus the zero tile into
// p.qpk-sized memory at `qpk`.
cudaError_t launch_wide_q_pack(const WideParams& p, int nitems, uint8_t* qpk, cudaStream_t st);
// Append of chunk rows into a bf16 pool, slots resolved from the block table.
struct WideAppend {
    __nv_bfloat16* pool_k;
    __nv_bfloat16* pool_v;
    const float* k;
    const float* v;
    const int32_t *row_seq, *offsets, *starts, *indptr, *ids;
    const int32_t* rows;  // [n] the step rows to append
    const int64_t* slots; // [n] their pool slots (layer 0); NULL = looked up from the tables
    int64_t n;
    int rowlen;           // kvh * head_dim
    int bs;
};
// launch_wide_q_pack and the append of `a` in one launch (a.n == 0: pack only).
cudaError_t launch_wide_prep(const WideParams& p, int nitems, uint8_t* qpk, const WideAppend& a, cudaStream_t st);
// Combines the partial slots of (pair, head)s cut between wide-kernel CTAs:
// split = [nsplit][4] pair, head, first slot, slots.
cudaError_t launch_wide_merge(const WideParams& p, const int32_t* split, int nsplit, cudaStream_t st);
cudaError_t launch_generic_attention(int dtype, const GenericParams& p, cudaStream_t st);
cudaError_t launch_plan_rows(const int32_t* row_seq, const int32_t* offsets, const int32_t* starts,
                             const int32_t* indptr, const int32_t* ids, int bs, int64_t nrows,
                             int64_t* positions, int64_t* slots, cudaStream_t st);
cudaError_t launch_append(int dtype, void* pool_k_layer, void* pool_v_layer, const float* k,
                          const float* v, const int64_t* slots, const int32_t* rows, int64_t n,
                          int rowlen, cudaStream_t st);
// The same with each row's slot resolved from the block table (row -> sequence -> position
// -> block id), with no per-row slots array.
cudaError_t launch_append_table(int dtype, void* pool_k_layer, void* pool_v_layer, const float* k,
                                const float* v, const int32_t* row_seq, const int32_t* offsets,
                                const int32_t* starts, const int32_t* indptr, const int32_t* ids, int bs,
                                const int32_t* rows, int64_t n, int rowlen, cudaStream_t st);
cudaError_t launch_copy_blocks(void* k, void* v, const int64_t* pairs, int64_t npairs, int layers,
                               int64_t layer_bytes, int64_t block_bytes, cudaStream_t st);
cudaError_t launch_bounded_wait_selftest(int* err, unsigned long long limit_ns, cudaStream_t st);
// Three device-addressable host arrays (float counts multiples of 4, 16-byte aligned) into
// device buffers, one launch.
cudaError_t launch_h2d_gather(const float* a_src, float* a_dst, int64_t a_floats, const float* b_src, float* b_dst,
                              int64_t b_floats, const float* c_src, float* c_dst, int64_t c_floats, cudaStream_t st);
// src [world][rows][row_floats] -> dst [rows][world][row_floats]; row_floats % 4 == 0, both
// pointers 16-byte aligned.
cudaError_t launch_interleave_heads(const float* src, float* dst, int world, int64_t rows, int64_t row_floats,
                                    cudaStream_t st);
cudaError_t launch_slot_mapping(const int32_t* table, int64_t table_len, const int64_t* positions,
                                int64_t n, int bs, int64_t* slots, int32_t* err, cudaStream_t st);

}  // namespace pk

struct pk_pool;
// Fills *out from `pool`; false if pool is NULL.
bool pk_pool_view(const pk_pool* pool, pk::PoolView* out);
struct pk_peer_gather;
// The exchange of the next step of `g` for slices of [rows][row_floats] floats (row_floats =
// heads x d of one rank): bumps the step epoch and fills *po (d: floats per head); *result is
// this rank's [rows][world * row_floats] result buffer of that step. PK_OK or an error code.
int pk_peer_gather_step(pk_peer_gather* g, int64_t rows, int64_t row_floats, int d, pk::PeerOut* po,
                        float** result);
// Sets the message pk_last_error() returns on this thread.
void pk_set_last_error(const char* msg);
