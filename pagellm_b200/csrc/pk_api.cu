// libpagekv C ABI: pool, per-step batch planning and kernel orchestration.
// The entry points mirror pagellm's cache/paged.py (PagedKVPool, slot_mapping, PagedBatch);
// the declarations and their reference citations are in include/pagekv.h.

#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <queue>
#include <array>
#include <string>
#include <unordered_map>
#include <vector>

#include "pagekv.h"
#include "pk_internal.h"
#include "pk_device.cuh"

namespace {

thread_local std::string g_err;

int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_err = buf;
    return code;
}

#define PK_CUDA(call)                                                                      \
    do {                                                                                   \
        cudaError_t e_ = (call);                                                           \
        if (e_ != cudaSuccess)                                                             \
            return fail(PK_ERR_CUDA, "%s failed: %s", #call, cudaGetErrorString(e_));      \
    } while (0)

// Makes `dev` current for the scope, restoring the caller's device afterwards.
struct DeviceScope {
    int prev = -1;
    cudaError_t err = cudaSuccess;
    explicit DeviceScope(int dev) {
        cudaGetDevice(&prev);
        if (prev != dev) err = cudaSetDevice(dev);
    }
    ~DeviceScope() {
        int cur = -1;
        cudaGetDevice(&cur);
        if (prev >= 0 && cur != prev) cudaSetDevice(prev);
    }
};

// Grow-only device allocation.
struct DevBuf {
    void* ptr = nullptr;
    size_t cap = 0;
    cudaError_t reserve(size_t bytes) {
        if (bytes <= cap) return cudaSuccess;
        if (ptr) {
            cudaError_t e = cudaFree(ptr);
            if (e != cudaSuccess) return e;
            ptr = nullptr;
            cap = 0;
        }
        size_t want = std::max<size_t>(bytes, 4096);
        want = want + want / 4;
        cudaError_t e = cudaMalloc(&ptr, want);
        if (e == cudaSuccess) cap = want;
        return e;
    }
    void release() {
        if (ptr) cudaFree(ptr);
        ptr = nullptr;
        cap = 0;
    }
};

// Packs several host arrays into one pinned buffer and ships them with a single copy.
// The pinned buffer is reused only after the previous copy out of it has finished.
struct Uploader {
    void* host = nullptr;
    size_t host_cap = 0;
    DevBuf dev;
    cudaEvent_t done = nullptr;
    bool pending = false;
    std::vector<std::pair<const void*, size_t>> parts;
    std::vector<size_t> offs;

    static size_t up256(size_t x) { return (x + 255) & ~size_t(255); }
    void begin() {
        parts.clear();
        offs.clear();
    }
    size_t add(const void* src, size_t bytes) {
        size_t off = parts.empty() ? 0 : up256(offs.back() + parts.back().second);
        parts.emplace_back(src, bytes);
        offs.push_back(off);
        return off;
    }
    int commit(cudaStream_t st) {
        size_t total = parts.empty() ? 0 : offs.back() + parts.back().second;
        if (total == 0) return PK_OK;
        if (!done) PK_CUDA(cudaEventCreateWithFlags(&done, cudaEventDisableTiming));
        if (pending) {
            PK_CUDA(cudaEventSynchronize(done));
            pending = false;
        }
        if (total > host_cap) {
            if (host) PK_CUDA(cudaFreeHost(host));
            host = nullptr;
            host_cap = 0;
            size_t want = std::max<size_t>(total + total / 4, 4096);
            PK_CUDA(cudaMallocHost(&host, want));
            host_cap = want;
        }
        PK_CUDA(dev.reserve(total));
        for (size_t i = 0; i < parts.size(); ++i)
            if (parts[i].second) std::memcpy(static_cast<char*>(host) + offs[i], parts[i].first, parts[i].second);
        PK_CUDA(cudaMemcpyAsync(dev.ptr, host, total, cudaMemcpyHostToDevice, st));
        PK_CUDA(cudaEventRecord(done, st));
        pending = true;
        return PK_OK;
    }
    template <typename T>
    T* at(size_t i) const {
        return reinterpret_cast<T*>(static_cast<char*>(dev.ptr) + offs[i]);
    }
    void release() {
        if (pending && done) cudaEventSynchronize(done);
        if (host) cudaFreeHost(host);
        host = nullptr;
        host_cap = 0;
        dev.release();
        if (done) cudaEventDestroy(done);
        done = nullptr;
    }
};

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

PFN_cuPointerGetAttributes_v7000 pointer_attributes_fn() {
    static PFN_cuPointerGetAttributes_v7000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuPointerGetAttributes", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuPointerGetAttributes_v7000>(p);
    });
    return fn;
}

// Device address of the host range [p, p + bytes) when all of it lies inside one
// page-locked allocation that the current device can address (cudaMallocHost, cudaHostAlloc
// and cudaHostRegister ranges are mapped under unified addressing), else nullptr. The
// allocation's extent comes from the driver, so a kernel never stores past the end of a
// buffer shorter than `bytes`: such a buffer, and pageable memory, get nullptr.
void* mapped_host_range(const void* p, size_t bytes) {
    PFN_cuPointerGetAttributes_v7000 fn = pointer_attributes_fn();
    if (!fn || !p || bytes == 0) return nullptr;
    const CUdeviceptr a = reinterpret_cast<CUdeviceptr>(p);
    // one driver query for all four attributes (pageable memory reports no memory type)
    unsigned int mtype = 0;
    CUdeviceptr start = 0, dptr = 0;
    size_t size = 0;
    CUpointer_attribute attrs[4] = {CU_POINTER_ATTRIBUTE_MEMORY_TYPE, CU_POINTER_ATTRIBUTE_RANGE_START_ADDR,
                                    CU_POINTER_ATTRIBUTE_RANGE_SIZE, CU_POINTER_ATTRIBUTE_DEVICE_POINTER};
    void* data[4] = {&mtype, &start, &size, &dptr};
    if (fn(4, attrs, data, a) != CUDA_SUCCESS || mtype != CU_MEMORYTYPE_HOST) return nullptr;
    if (a < start || a - start > size || bytes > size - (a - start)) return nullptr;
    if (dptr == 0 || dptr % 16 != 0) return nullptr;
    return reinterpret_cast<void*>(dptr);
}

}  // namespace

struct pk_pool {
    int device = 0;
    int n_layers = 0;
    int64_t num_blocks = 0;
    int block_size = 0;
    int kvh = 0;
    int d = 0;
    int dtype = 0;
    int esize = 0;
    void* k = nullptr;
    void* v = nullptr;
    int64_t layer_elems = 0;
    int num_sms = 0;
    // tensor-core path
    bool tc_ok = false;
    int tc_per_head = 0;
    int tc_stages = 0;
    size_t tc_smem = 0;
    int tc_virt = 1;  // virtual split-KV CTAs per CTA (8 / kvh for pools of few KV heads)
    int smem_optin = 0;  // largest dynamic shared memory a CTA may opt in to
    std::string tc_why;
    CUtensorMap tmk{};
    CUtensorMap tmv{};
    // wide-tile (tcgen05) kernel: one (block, head, 64-dim chunk) per TMA box
    bool wide_ok = false;
    CUtensorMap tmk1{};
    CUtensorMap tmv1{};
    Uploader pairs_up;

    size_t layer_bytes() const { return static_cast<size_t>(layer_elems) * esize; }
    size_t block_bytes() const { return static_cast<size_t>(block_size) * kvh * d * esize; }
    char* k_layer(int layer) const { return static_cast<char*>(k) + layer * layer_bytes(); }
    char* v_layer(int layer) const { return static_cast<char*>(v) + layer * layer_bytes(); }
};

struct pk_batch {
    pk_pool* pool = nullptr;
    int nseq = 0;
    int64_t nrows = 0;
    std::vector<int32_t> indptr, ids, starts, nnew, offsets, row_seq;
    Uploader meta;  // 0 indptr, 1 ids, 2 starts, 3 offsets, 4 row_seq, 5 append rows
    // Fused append is exact only if every slot written this step is read by nobody but the
    // writing row's own unit; otherwise (shared or repeated blocks, duplicate slots) the
    // step appends first with a separate kernel, last writer per slot, as pagellm does.
    bool fuse_append_ok = true;
    std::vector<int32_t> app_rows;  // winner rows when slots repeat (else empty = all rows)
    std::vector<int32_t> writer_seq, writer_idx;  // per block id, scratch of the check
    std::vector<uint64_t> written;                // bit per block id: written this step
    // positions / slots of the step's rows (rows buffer) not built yet; the plan's stream
    mutable bool rows_pending = false;
    cudaStream_t rows_stream = nullptr;
    // merge counters, zero between launches: uploaded as zeros with every attention plan
    // (plan part 22), left at zero by the kernel, reset by pk_batch_check after a timeout
    std::vector<int32_t> ctr_zero;
    // Wide-tile work runs on a side stream, forked from and joined back into the caller's
    // stream with events, so it overlaps the split-KV kernel.
    cudaStream_t side = nullptr;
    cudaEvent_t ev_fork = nullptr, ev_join = nullptr, ev_pack = nullptr;
    DevBuf rows;    // positions [nrows] then slots [nrows]
    DevBuf err;     // one int
    // attention plan for plan_H query heads
    int plan_H = -1;
    bool use_tc = false;
    int nu = 0, total_blocks = 0, ncta = 0, nt = 1, nsplit = 0;
    int ngeneric = 0;
    std::vector<int32_t> u_seq, u_t0, u_n, u_blk, sp_u, sp_c0, sp_c1, gen_rows;
    std::vector<int32_t> cta_blk;  // [ncta + 1] first block of each split-KV CTA
    // Wide-tile work items: [0, nwide) chunk items (side stream), then [nwide, nwide +
    // nprefix) shared-prefix items (after the split-KV kernel, merged into its rows).
    int nwide = 0, nprefix = 0, nprefix_groups = 0;
    int64_t prefix_keys = 0;  // shared keys summed over the prefix groups
    int64_t prefix_token_keys = 0;  // sum over the groups of query tokens x shared keys
    int prefix_sharing = 1;   // 0 off, 1 where the cost estimate favours it, 2 always
    std::vector<int32_t> w_seq, w_tok0, w_ntok, w_kend, tok_row, tok_pos;
    std::vector<int32_t> w_rows;   // rows of chunk items (appended separately)
    std::vector<int32_t> w_pair;   // item pairs: chunk pairs, then prefix pairs
    int npair_chunk = 0, npair_prefix = 0;
    // wide-kernel schedule: per CTA a range of segments (pair, head, key tiles, slot, ph)
    std::vector<int32_t> pair_kend, cta_seg, seg, ph_info, split;
    int ncta_chunk = 0, ncta_prefix = 0, nslots = 0, nph = 0, nwsplit = 0;
    int nwsplit_chunk = 0;  // the first nwsplit_chunk entries of split belong to chunk pairs
    int tc_per_sm = 1;      // split-KV CTAs that share an SM in the current plan
    DevBuf wpart;  // partial O and (max, sum) of pair-heads cut between CTAs
    DevBuf qpk;    // packed bf16 query tiles of the wide-tile items (+1 zero tile)
    std::vector<int32_t> u_kb0;    // per unit: first block read (after a shared prefix)
    std::vector<int32_t> u_cta;    // per unit: first and last split-KV CTA of its blocks
    std::vector<int32_t> u_meta;   // per unit: packed record (TcParams::u_meta)
    std::vector<int64_t> w_slots;  // per wide-item row (w_rows): its pool slot
    std::vector<int32_t> seq_kb0;  // scratch: per sequence
    int tc_max_new = 0;            // most new tokens of a sequence on the split-KV kernel
    DevBuf lse;                    // [rows][H] when shared-prefix items exist
    Uploader plan;  // 0 u_seq 1 u_t0 2 u_n 3 u_blk 4 sp_u 5 sp_c0 6 sp_c1 7 gen_rows 8 w_seq
                    // 9 w_tok0 10 w_rows 11 w_ntok 12 w_kend 13 tok_row 14 tok_pos 15 u_kb0
                    // 16 w_pair 17 pair_kend 18 cta_seg 19 seg 20 split 21 cta_blk
                    // 22 merge counters (zeros) 23 u_cta 24 u_meta 25 w_slots
    DevBuf ws;
    size_t ws_part_o_floats = 0;
    DevBuf io;  // q | k | v | out for the host-buffer entry point
    // Head-sharded exchange fused into the split-KV launch of the current call (n == 0: off),
    // and the slice the exchange sends when the step cannot fuse it
    pk::PeerOut peer_out{};
    DevBuf peer_slice;
    int launches = 0;
    // bytes the last pk_batch_write_and_attend_host moved: host to device, device to host
    // by a copy after the kernels, stored by the kernels straight into the caller's
    // page-locked result buffer
    int64_t io_h2d = 0, io_d2h = 0, io_direct = 0;
    // Optional per-kernel timing: events recorded on the launching stream around each
    // launch, resolved by pk_batch_profile_read.
    bool profiling = false;
    std::vector<cudaEvent_t> ev_pool;
    size_t ev_used = 0;
    std::vector<int> ev_kind;  // kind of each recorded (start, end) pair

    const int64_t* positions() const { return static_cast<const int64_t*>(rows.ptr); }
    const int64_t* slots() const { return static_cast<const int64_t*>(rows.ptr) + nrows; }
};

// Positions and slots of the step's rows (paged.py:412-424) on the device, built on first
// use: a decode step with the fused append never reads them.
static cudaError_t ensure_rows(const pk_batch* B, cudaStream_t st) {
    if (!B->rows_pending) return cudaSuccess;
    B->rows_pending = false;
    return pk::launch_plan_rows(B->meta.at<int32_t>(4), B->meta.at<int32_t>(3), B->meta.at<int32_t>(2),
                                B->meta.at<int32_t>(0), B->meta.at<int32_t>(1), B->pool->block_size,
                                B->nrows, static_cast<int64_t*>(B->rows.ptr),
                                static_cast<int64_t*>(B->rows.ptr) + B->nrows, st);
}

namespace {

// Encode the two tensor maps of the tensor-core kernel. Layout 0 views a layer-stacked
// pool as [chunk of 64 dims][kv head][slot][64 dims] so that one box = one whole K (or V)
// block with each (head, chunk) slice's tokens on consecutive 128-byte rows; layout 1
// is the natural order, one box per (block, head).
// One (block, head, 64-dim chunk) per box over the layout-0 view: the wide kernel's tiles.
bool encode_chunk_maps(pk_pool* P, std::string* why) {
    auto enc = tensor_map_encoder();
    if (!enc) {
        *why = "cuTensorMapEncodeTiled unavailable";
        return false;
    }
    const cuuint64_t slots = static_cast<cuuint64_t>(P->n_layers) * P->num_blocks * P->block_size;
    cuuint64_t dims[4] = {64, slots, static_cast<cuuint64_t>(P->kvh), static_cast<cuuint64_t>(P->d / 64)};
    cuuint64_t strides[3] = {static_cast<cuuint64_t>(P->kvh) * P->d * 2, static_cast<cuuint64_t>(P->d) * 2, 128};
    // one 64-dim chunk of one block per box, for K and V alike
    const cuuint32_t box_k[4] = {64, static_cast<cuuint32_t>(P->block_size), 1, 1};
    const cuuint32_t box_v[4] = {64, static_cast<cuuint32_t>(P->block_size), 1, 1};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    for (int t = 0; t < 2; ++t) {
        CUresult r = enc(t == 0 ? &P->tmk1 : &P->tmv1, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4,
                         t == 0 ? P->k : P->v, dims, strides, t == 0 ? box_k : box_v, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) {
            *why = "cuTensorMapEncodeTiled(chunk box) failed";
            return false;
        }
    }
    return true;
}

bool encode_pool_maps(pk_pool* P, int layout, std::string* why) {
    auto enc = tensor_map_encoder();
    if (!enc) {
        *why = "cuTensorMapEncodeTiled unavailable";
        return false;
    }
    const cuuint64_t slots = static_cast<cuuint64_t>(P->n_layers) * P->num_blocks * P->block_size;
    const int chunks = P->d / 64;
    cuuint64_t dims[4];
    cuuint64_t strides[3];
    cuuint32_t box[4];
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    if (layout == 0) {
        dims[0] = 64; dims[1] = slots; dims[2] = P->kvh; dims[3] = chunks;
        strides[0] = static_cast<cuuint64_t>(P->kvh) * P->d * 2;
        strides[1] = static_cast<cuuint64_t>(P->d) * 2;
        strides[2] = 128;
        box[0] = 64; box[1] = P->block_size; box[2] = P->kvh; box[3] = chunks;
    } else {
        dims[0] = 64; dims[1] = chunks; dims[2] = P->kvh; dims[3] = slots;
        strides[0] = 128;
        strides[1] = static_cast<cuuint64_t>(P->d) * 2;
        strides[2] = static_cast<cuuint64_t>(P->kvh) * P->d * 2;
        box[0] = 64; box[1] = chunks; box[2] = 1; box[3] = P->block_size;
    }
    for (int t = 0; t < 2; ++t) {
        CUresult r = enc(t == 0 ? &P->tmk : &P->tmv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4,
                         t == 0 ? P->k : P->v, dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) {
            char b[96];
            snprintf(b, sizeof(b), "cuTensorMapEncodeTiled(layout %d) returned %d", layout, (int)r);
            *why = b;
            return false;
        }
    }
    return true;
}

void setup_tc(pk_pool* P) {
    P->tc_ok = false;
    auto no = [&](const char* w) { P->tc_why = w; };
    if (P->dtype != PK_BF16) return no("pool is not bf16");
    // only these head sizes have a compiled instance (launch_tc_attention)
    if (P->d != 64 && P->d != 128 && P->d != 256) return no("head_dim not in {64,128,256}");
    if (P->block_size % 16 != 0 || P->block_size > 256) return no("block_size not a multiple of 16 (<=256)");
    if (P->kvh > pk::kTcMaxKvHeads) return no("more than 8 KV heads");
    const int64_t slots = static_cast<int64_t>(P->n_layers) * P->num_blocks * P->block_size;
    if (slots >= (int64_t(1) << 31)) return no("pool has 2^31 slots or more");
    int optin = 0;
    cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, P->device);
    P->smem_optin = optin;
    const size_t stage = static_cast<size_t>(2) * P->block_size * P->kvh * P->d * 2;
    // A CTA has one consumer warp per KV head of each of its V virtual CTAs. With few KV heads
    // (the head-sharded layout gives 1-4 per GPU) V = 8 / kvh virtual CTAs - each its own block
    // range, stage ring and barriers - keep 8 consumer warps per SM under one producer warp
    // (several 2-warp CTAs per SM would spend half the register file on producers). Stages: as
    // many as fit (at most 8); V is lowered while fewer than 3 fit.
    int stages = 0;
    for (int v = std::max(1, pk::kTcMaxKvHeads / P->kvh); v >= 1; --v) {
        const size_t budget = std::min<size_t>(static_cast<size_t>(optin), size_t(200) << 10);
        stages = 8;
        while (stages >= 2 && pk::tc_smem_bytes(P->d, P->block_size, P->kvh, stages, v) > budget) --stages;
        P->tc_virt = v;
        if (stages >= 3 || v == 1) break;
    }
    (void)stage;
    if (stages < 2) return no("K/V block too large for two shared-memory stages");
    std::string why;
    if (encode_pool_maps(P, 0, &why)) {
        P->tc_per_head = 0;
    } else if (encode_pool_maps(P, 1, &why)) {
        P->tc_per_head = 1;
    } else {
        P->tc_why = why;
        return;
    }
    P->tc_stages = stages;
    P->tc_smem = pk::tc_smem_bytes(P->d, P->block_size, P->kvh, stages, P->tc_virt);
    P->tc_ok = true;
    P->tc_why.clear();
    // wide tiles: head_dim 128, 128-key tiles made of whole blocks, the layout-0 view
    std::string why2;
    P->wide_ok = P->d == 128 && pk::kWideKeys % P->block_size == 0 && P->tc_per_head == 0 &&
                 static_cast<size_t>(optin) >= pk::wide_smem_bytes() && encode_chunk_maps(P, &why2);
}

int ceil_div(int64_t a, int64_t b) { return static_cast<int>((a + b - 1) / b); }

// Split-KV CTA count: one per SM at most; at least kMinBlocksPerCta blocks each, unless
// the step has many short units (each unit costs a query load, a fill of the pipeline and
// a store on top of its blocks), which are then spread kUnitsPerCta per CTA; never more
// CTAs than blocks.
constexpr int64_t kMinBlocksPerCta = 16;
constexpr int64_t kUnitsPerCta = 3;
constexpr int kFuseMaxNew = 1;  // fuse the append only when split-KV sequences add <= 1 token

int64_t split_kv_ctas(int64_t T, int64_t nu, int64_t max_ctas) {
    if (T <= 0) return 0;
    const int64_t want = std::max(T / kMinBlocksPerCta, (nu + kUnitsPerCta - 1) / kUnitsPerCta);
    return std::max<int64_t>(1, std::min({max_ctas, T, want}));
}

// Sequences with at least this many new query rows (tokens x heads per KV head) go to the
// wide-tile tensor-core kernel; fewer rows stay on the split-KV kernel's units.
constexpr int64_t kWideMinRows = 64;

// Time a split-KV CTA loses per unit boundary inside its block range (B200, C2 decode
// shape): it reloads queries, publishes a partial for the unit it leaves, and the unit it
// ends in it usually finishes last of that unit's CTAs, so it merges the unit's partials at
// the end of its run. Per-CTA globaltimer traces first showed ~9.5 us (112 us against 102.6 us
// at equal block counts). Sweeps of the cost (6 / 9 / 11 / 14 / 18 us, three C2 batches and
// the C5 8- and 4-way shards) put the fastest steps at 11 us once merges had become cheap
// (C2 98.3 against 99.8 us at 14); pools split into virtual CTAs (few KV heads) were fastest
// at 14 us (the 8-way head shard of C5: 125.2 against 129.3 us at 11).
constexpr double kUnitSwitchUs = 11.0;
constexpr double kUnitSwitchUsVirtual = 14.0;

// The units' blocks (in unit order, prefix sums ub[0..nu]) cut into contiguous CTA ranges,
// at most n of them. A range costs its blocks plus `switch_cost` blocks per unit boundary
// inside it; the cut minimises the largest cost: bisection on the bound, each CTA filled
// greedily up to it. Returns the CTAs used; first[0..count] are their first blocks.
template <typename I>
int partition_blocks(const I* ub, int64_t nu, int64_t n, int64_t switch_cost, std::vector<int32_t>& first) {
    const int64_t T = nu > 0 ? static_cast<int64_t>(ub[nu]) : 0;
    first.assign(1, 0);
    if (T <= 0 || n <= 0) return 0;
    auto fill = [&](int64_t X, bool keep) -> int64_t {
        int64_t b = 0, count = 0, u = 0;
        while (b < T) {
            while (static_cast<int64_t>(ub[u + 1]) <= b) ++u;
            int64_t R = X, e = b, uu = u;
            for (;;) {
                const int64_t take = std::min<int64_t>(static_cast<int64_t>(ub[uu + 1]) - e, R);
                e += take;
                R -= take;
                if (e < static_cast<int64_t>(ub[uu + 1]) || uu + 1 >= nu || R < switch_cost + 1) break;
                R -= switch_cost;
                ++uu;
            }
            if (e == b) e = b + 1;
            b = e;
            ++count;
            if (keep) first.push_back(static_cast<int32_t>(b));
        }
        return count;
    };
    int64_t lo = (T + n - 1) / n, hi = T + switch_cost * nu;  // hi: one CTA always fits
    while (lo < hi) {
        const int64_t mid = lo + (hi - lo) / 2;
        if (fill(mid, false) <= n) hi = mid;
        else lo = mid + 1;
    }
    return static_cast<int>(fill(lo, true));
}

// CTA of block j under the partition `first` (count + 1 entries).
int cta_of_block(const std::vector<int32_t>& first, int64_t j) {
    return static_cast<int>(std::upper_bound(first.begin(), first.end(), static_cast<int32_t>(j)) - first.begin()) - 1;
}


// Shared prefixes (cascade attention). Sequences whose block tables begin with the same
// block ids - forks and prefix-cache hits in pagellm (cache/paged.py:187-203, :257-263) -
// hold bit-identical K/V there. For a group of them, the wide-tile kernel attends every
// group token to the shared keys once per 128 rows, and the split-KV units start after the
// prefix; the two partials are merged per row. A group is the sequences with the same first
// block id; its prefix is the common run of ids, cut to whole blocks before every member's
// first new token (so no key of it is written this step and every query sees all of it).
// In mode 1 it is taken only where a cost estimate says reading the prefix once per
// sequence (the split-KV path) would take longer than the wide-tile CTAs over it.
constexpr int64_t kPrefixMinKeys = 64;
constexpr double kWideUsPerKeyTile = 2.5;     // one CTA (256 rows) over one 128-key tile
constexpr double kWideFixedUs = 5.0;          // launch, Q load, epilogue
constexpr int64_t kWideMinTilesPerCta = 4;    // stream-K shares smaller than this cost more than they save
constexpr double kSplitKvBytesPerUs = 6.0e6;  // split-KV streaming rate (HBM / L2)

// Unit-boundary cost in blocks for a pool: kUnitSwitchUs (kUnitSwitchUsVirtual for pools in
// virtual CTAs) of one CTA's share of the split-KV streaming rate (`ctas` CTAs sharing it),
// over the K+V bytes of one block.
int64_t unit_switch_blocks(const pk_pool* P, int64_t ctas) {
    const double cta_rate = kSplitKvBytesPerUs / static_cast<double>(std::max<int64_t>(1, ctas));
    const double blk = static_cast<double>(P->block_bytes()) * 2.0;
    const double us = P->tc_virt > 1 ? kUnitSwitchUsVirtual : kUnitSwitchUs;
    return std::max<int64_t>(0, std::llround(us * cta_rate / blk));
}

void plan_shared_prefixes(pk_batch* B, int qmax, int tpt, const std::vector<int>& tc_seqs) {
    pk_pool* P = B->pool;
    std::vector<std::pair<int32_t, int>> keyed;
    for (int i : tc_seqs)
        if (B->indptr[i + 1] > B->indptr[i]) keyed.emplace_back(B->ids[B->indptr[i]], i);
    std::stable_sort(keyed.begin(), keyed.end(),
                     [](const std::pair<int32_t, int>& a, const std::pair<int32_t, int>& b) { return a.first < b.first; });
    const double blk_bytes = static_cast<double>(P->block_bytes()) * 2.0;  // K + V, all heads
    for (size_t a = 0; a < keyed.size();) {
        size_t b = a + 1;
        while (b < keyed.size() && keyed[b].first == keyed[a].first) ++b;
        if (b - a >= 2) {
            const int ref = keyed[a].second;
            const int32_t* rt = B->ids.data() + B->indptr[ref];
            int64_t pb = std::min<int64_t>(B->indptr[ref + 1] - B->indptr[ref], B->starts[ref] / P->block_size);
            int64_t toks = 0, units = 0;
            for (size_t x = a; x < b && pb > 0; ++x) {
                const int s = keyed[x].second;
                const int32_t* stb = B->ids.data() + B->indptr[s];
                const int64_t lim = std::min<int64_t>({pb, B->indptr[s + 1] - B->indptr[s],
                                                       B->starts[s] / P->block_size});
                int64_t k = 0;
                while (k < lim && stb[k] == rt[k]) ++k;
                pb = k;
                toks += B->nnew[s];
                units += ceil_div(B->nnew[s], qmax);
            }
            const int64_t keys = pb * P->block_size;
            if (keys >= kPrefixMinKeys) {
                // stream-K over (pair-head, key tile): the work W in equal shares over <= one wave
                const int64_t work = ceil_div(ceil_div(toks, tpt), 2) * P->kvh * ceil_div(keys, pk::kWideKeys);
                const int64_t g = std::max<int64_t>(1, std::min<int64_t>(P->num_sms, work / kWideMinTilesPerCta));
                const double est_wide = static_cast<double>(ceil_div(work, g)) * kWideUsPerKeyTile + kWideFixedUs;
                const double est_split = static_cast<double>(units) * pb * blk_bytes / kSplitKvBytesPerUs;
                if (B->prefix_sharing == 2 || est_wide < est_split) {
                    // the group's tokens, member by member, cut into items of tpt tokens
                    int fill = 0;
                    auto close_item = [&]() {
                        B->w_seq.push_back(ref);
                        B->w_tok0.push_back(static_cast<int32_t>(B->tok_row.size()) - fill);
                        B->w_ntok.push_back(fill);
                        B->w_kend.push_back(static_cast<int32_t>(keys));
                        fill = 0;
                    };
                    for (size_t x = a; x < b; ++x) {
                        const int s = keyed[x].second;
                        B->seq_kb0[s] = static_cast<int32_t>(pb);
                        for (int t = 0; t < B->nnew[s]; ++t) {
                            B->tok_row.push_back(B->offsets[s] + t);
                            B->tok_pos.push_back(B->starts[s] + t);
                            if (++fill == tpt) close_item();
                        }
                    }
                    if (fill > 0) close_item();
                    B->nprefix_groups++;
                    B->prefix_keys += keys;
                    B->prefix_token_keys += toks * keys;
                }
            }
        }
        a = b;
    }
}

// Wide-kernel schedule: the (pair-head, key tile) work of the chunk pairs, then of the
// shared-prefix pairs, each cut over G CTAs with a makespan of ceil(W / G) tiles (W the
// kind's tiles). Whole pair-heads first, longest first, each to the least-loaded CTA that
// stays within the makespan (a whole pair-head needs no partial and no merge); the
// pair-heads that fit nowhere are cut into pieces that fill the CTAs' spare capacity in CTA
// order, so only those few leave partial slots (one per piece) for wide_merge_kernel.
// Chunk pair-heads (run beside the split-KV kernel on a second stream) are never cut: one CTA
// each. Shared-prefix work (after the split-KV kernel) gets all SMs, fewer when shares would
// be under kWideMinTilesPerCta tiles.
void build_wide_schedule(pk_batch* B, int64_t chunk_ctas) {
    pk_pool* P = B->pool;
    const int kvh = P->kvh;
    const int npairs = B->npair_chunk + B->npair_prefix;
    B->pair_kend.resize(npairs);
    for (int x = 0; x < npairs; ++x) {
        const int i0 = B->w_pair[2 * x], i1 = B->w_pair[2 * x + 1];
        B->pair_kend[x] = std::max(B->w_kend[i0], i1 >= 0 ? B->w_kend[i1] : 0);
    }
    B->cta_seg.assign(1, 0);
    B->seg.clear();
    B->ph_info.clear();
    B->split.clear();
    B->nslots = B->nwsplit = B->nwsplit_chunk = 0;
    auto tiles = [&](int x) { return static_cast<int64_t>(ceil_div(B->pair_kend[x], pk::kWideKeys)); };
    // Schedules the pair-heads of pairs [x0, x1) over at most G CTAs; returns the CTAs used.
    // whole_only: no pair-head is cut (the makespan is at least the longest pair-head).
    auto stream_k = [&](int x0, int x1, int64_t G, bool whole_only) -> int {
        const int nph = (x1 - x0) * kvh;
        if (nph <= 0) return 0;
        auto ph_tiles = [&](int q) { return tiles(x0 + q / kvh); };
        int64_t W = 0;
        for (int q = 0; q < nph; ++q) W += ph_tiles(q);
        G = std::max<int64_t>(1, std::min(G, W));
        int64_t longest = 0;
        for (int q = 0; q < nph; ++q) longest = std::max(longest, ph_tiles(q));
        const int64_t target = whole_only ? std::max((W + G - 1) / G, longest) : (W + G - 1) / G;
        std::vector<int> order(nph);
        for (int q = 0; q < nph; ++q) order[q] = q;
        std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return ph_tiles(a) > ph_tiles(b); });
        std::vector<int64_t> load(G, 0);
        std::vector<std::vector<std::array<int64_t, 3>>> segs_of(G);  // {q, t0, t1}
        using LoadCta = std::pair<int64_t, int64_t>;                   // (load, cta), min-heap
        std::priority_queue<LoadCta, std::vector<LoadCta>, std::greater<LoadCta>> heap;
        for (int64_t c = 0; c < G; ++c) heap.push({0, c});
        std::vector<int> rest;
        for (int q : order) {
            const LoadCta top = heap.top();
            if (top.first + ph_tiles(q) <= target) {
                heap.pop();
                segs_of[top.second].push_back({q, 0, ph_tiles(q)});
                load[top.second] = top.first + ph_tiles(q);
                heap.push({load[top.second], top.second});
            } else {
                rest.push_back(q);
            }
        }
        std::sort(rest.begin(), rest.end());
        int64_t c = 0;
        for (int q : rest) {
            int64_t t = 0;
            const int64_t T = ph_tiles(q);
            while (t < T) {
                while (c + 1 < G && load[c] >= target) ++c;  // the last CTA takes any rounding rest
                const int64_t take = std::max<int64_t>(1, std::min<int64_t>(T - t, target - load[c]));
                segs_of[c].push_back({q, t, t + take});
                load[c] += take;
                t += take;
            }
        }
        // a pair-head cut into several segments gets one partial slot per segment
        std::vector<int32_t> count(nph, 0), next(nph, -1);
        for (int64_t cc = 0; cc < G; ++cc)
            for (const auto& sg : segs_of[cc]) count[sg[0]]++;
        for (int q = 0; q < nph; ++q) {
            if (count[q] > 1) {
                B->split.insert(B->split.end(), {x0 + q / kvh, q % kvh, B->nslots, count[q]});
                next[q] = B->nslots;
                B->nslots += count[q];
            }
        }
        int used = 0;
        for (int64_t cc = 0; cc < G; ++cc) {
            if (segs_of[cc].empty()) continue;
            for (const auto& sg : segs_of[cc]) {
                const int q = static_cast<int>(sg[0]);
                const int slot = next[q] >= 0 ? next[q]++ : -1;
                B->seg.insert(B->seg.end(), {x0 + q / kvh, q % kvh, static_cast<int32_t>(sg[1]),
                                             static_cast<int32_t>(sg[2]), slot, 0});
            }
            B->cta_seg.push_back(static_cast<int32_t>(B->seg.size() / 6));
            ++used;
        }
        return used;
    };
    int64_t Wc = 0, Wp = 0;
    for (int x = 0; x < B->npair_chunk; ++x) Wc += tiles(x) * kvh;
    for (int x = B->npair_chunk; x < npairs; ++x) Wp += tiles(x) * kvh;
    const int64_t nph_chunk = static_cast<int64_t>(B->npair_chunk) * kvh;
    // Chunk pair-heads stay whole, one per CTA: cut into pieces (measured on C3: 64 pair-heads
    // of 9-12 tiles over the 76 SMs the split-KV kernel leaves), each piece's query-tile load,
    // 128 KB partial and merge cost more than the balance gains.
    (void)chunk_ctas;
    (void)Wc;
    B->ncta_chunk = stream_k(0, B->npair_chunk, nph_chunk, true);
    B->nwsplit_chunk = static_cast<int>(B->split.size() / 4);
    B->ncta_prefix = stream_k(B->npair_chunk, npairs,
                              std::min<int64_t>(P->num_sms, std::max<int64_t>(1, Wp / kWideMinTilesPerCta)), false);
    B->nph = 0;
    B->nwsplit = static_cast<int>(B->split.size() / 4);
}

int build_attention_plan(pk_batch* B, int H, cudaStream_t st) {
    pk_pool* P = B->pool;
    const int g = H / P->kvh;
    B->plan_H = -1;
    B->u_seq.clear(); B->u_t0.clear(); B->u_n.clear(); B->u_blk.assign(1, 0);
    B->sp_u.clear(); B->sp_c0.clear(); B->sp_c1.clear(); B->gen_rows.clear();
    B->cta_blk.assign(1, 0);
    B->use_tc = false;
    B->nu = B->total_blocks = B->ncta = B->nsplit = B->ngeneric = 0;
    B->nt = 1;
    int qmax = 0;
    if (P->tc_ok && g <= pk::kMaxCols) {
        qmax = std::max(1, pk::kMaxCols / g);
        if (P->d == 256) qmax = g <= 8 ? std::max(1, 8 / g) : 0;  // one n8 tile only at D=256
    }
    B->w_seq.clear(); B->w_tok0.clear(); B->w_ntok.clear(); B->w_kend.clear();
    B->tok_row.clear(); B->tok_pos.clear(); B->w_rows.clear(); B->u_kb0.clear(); B->u_cta.clear();
    B->nwide = B->nprefix = B->nprefix_groups = 0;
    B->prefix_keys = B->prefix_token_keys = 0;
    B->seq_kb0.assign(B->nseq, 0);
    const bool wide_ok = P->wide_ok && g <= 128 && 128 % g == 0;
    const int tpt = wide_ok ? 128 / g : 0;  // query tokens per wide item
    std::vector<int> tc_seqs;
    for (int i = 0; i < B->nseq; ++i) {
        const int n = B->nnew[i];
        if (n <= 0) continue;
        if (wide_ok && static_cast<int64_t>(n) * g >= kWideMinRows) {
            // chunk items: 128 query rows (128/g consecutive tokens) each
            for (int t0 = 0; t0 < n; t0 += tpt) {
                const int nt = std::min(tpt, n - t0);
                for (int t = t0; t < t0 + nt; ++t) {
                    B->tok_row.push_back(B->offsets[i] + t);
                    B->tok_pos.push_back(B->starts[i] + t);
                }
                B->w_seq.push_back(i);
                B->w_tok0.push_back(static_cast<int32_t>(B->tok_row.size()) - nt);
                B->w_ntok.push_back(nt);
                B->w_kend.push_back(B->starts[i] + t0 + nt);
            }
            for (int r = 0; r < n; ++r) B->w_rows.push_back(B->offsets[i] + r);
            continue;
        }
        if (qmax == 0) {
            for (int r = 0; r < n; ++r) B->gen_rows.push_back(B->offsets[i] + r);
            continue;
        }
        tc_seqs.push_back(i);
    }
    B->nwide = static_cast<int>(B->w_seq.size());
    B->tc_max_new = 0;
    for (int i : tc_seqs) B->tc_max_new = std::max(B->tc_max_new, B->nnew[i]);
    if (wide_ok && B->prefix_sharing != 0 && tc_seqs.size() >= 2) plan_shared_prefixes(B, qmax, tpt, tc_seqs);
    B->nprefix = static_cast<int>(B->w_seq.size()) - B->nwide;
    int64_t T = 0;
    for (int i : tc_seqs) {
        const int n = B->nnew[i];
        const int kb0 = B->seq_kb0[i];
        for (int t0 = 0; t0 < n; t0 += qmax) {
            const int nu = std::min(qmax, n - t0);
            const int64_t ctx = static_cast<int64_t>(B->starts[i]) + t0 + nu;
            T += ceil_div(ctx, P->block_size) - kb0;
            B->u_seq.push_back(i);
            B->u_t0.push_back(t0);
            B->u_n.push_back(nu);
            B->u_blk.push_back(static_cast<int32_t>(T));
            B->u_kb0.push_back(kb0);
            B->nt = std::max(B->nt, ceil_div(static_cast<int64_t>(nu) * g, 8));
        }
    }
    if (T >= (int64_t(1) << 31)) return fail(PK_ERR_UNSUPPORTED, "step reads 2^31 blocks or more");
    // Wide CTAs take two items each: neighbouring items of one sequence (chunk) or of one
    // prefix group, which read the same block table. Within each kind the pairs with the
    // most keys go first, so the longest CTAs start in the first wave.
    B->w_pair.clear();
    auto make_pairs = [&](int a0, int a1) {
        std::vector<std::pair<int32_t, int32_t>> pr;
        for (int x = a0; x < a1;) {
            if (x + 1 < a1 && B->w_seq[x + 1] == B->w_seq[x]) {
                pr.emplace_back(x, x + 1);
                x += 2;
            } else {
                pr.emplace_back(x, -1);
                x += 1;
            }
        }
        auto keys = [&](const std::pair<int32_t, int32_t>& q) {
            return std::max(B->w_kend[q.first], q.second >= 0 ? B->w_kend[q.second] : 0);
        };
        std::stable_sort(pr.begin(), pr.end(), [&](const std::pair<int32_t, int32_t>& x, const std::pair<int32_t, int32_t>& y) {
            return keys(x) > keys(y);
        });
        for (const auto& q : pr) {
            B->w_pair.push_back(q.first);
            B->w_pair.push_back(q.second);
        }
        return static_cast<int>(pr.size());
    };
    B->npair_chunk = make_pairs(0, B->nwide);
    B->npair_prefix = make_pairs(B->nwide, B->nwide + B->nprefix);
    B->nu = static_cast<int>(B->u_seq.size());
    B->ngeneric = static_cast<int>(B->gen_rows.size());
    if (B->nu > 0) {
        B->use_tc = true;
        B->total_blocks = static_cast<int>(T);
        // On small steps more CTAs would cut every unit into many partials whose merge
        // outweighs the bandwidth the extra SMs add.
        // (virtual) split-KV CTAs per SM: one CTA (its shared memory fills the SM) of tc_virt
        const int per_sm = P->tc_virt;
        B->tc_per_sm = per_sm;
        const int64_t nmax = split_kv_ctas(T, B->nu, static_cast<int64_t>(P->num_sms) * per_sm);
        B->ncta = partition_blocks(B->u_blk.data(), B->nu, nmax,
                                   unit_switch_blocks(P, static_cast<int64_t>(P->num_sms) * per_sm), B->cta_blk);
        B->u_cta.resize(2 * static_cast<size_t>(B->nu));
        for (int u = 0; u < B->nu; ++u) {
            const int c0 = cta_of_block(B->cta_blk, B->u_blk[u]);
            const int c1 = cta_of_block(B->cta_blk, B->u_blk[u + 1] - 1);
            B->u_cta[2 * u] = c0;
            B->u_cta[2 * u + 1] = c1;
            if (c0 != c1) {
                B->sp_u.push_back(u);
                B->sp_c0.push_back(c0);
                B->sp_c1.push_back(c1);
            }
        }
        B->nsplit = static_cast<int>(B->sp_u.size());
        const size_t segs = static_cast<size_t>(B->nu) + B->ncta;
        B->ws_part_o_floats = segs * P->kvh * pk::kMaxCols * P->d;
        const size_t ws_bytes = (B->ws_part_o_floats + segs * P->kvh * pk::kMaxCols * 2) * sizeof(float);
        PK_CUDA(B->ws.reserve(ws_bytes));
        // merge counters: per (partial slot, KV head) for the first level, then per (unit, KV
        // head) for the second; they travel as zeros with the plan's upload
        B->ctr_zero.assign((segs + static_cast<size_t>(B->nu)) * P->kvh, 0);
    }
    // chunk work shares the GPU with the split-KV CTAs: it gets the SMs they leave free
    build_wide_schedule(B, B->use_tc ? std::max<int64_t>(1, P->num_sms - ceil_div(B->ncta, B->tc_per_sm))
                                     : P->num_sms);
    B->plan.begin();
    B->plan.add(B->u_seq.data(), B->u_seq.size() * 4);
    B->plan.add(B->u_t0.data(), B->u_t0.size() * 4);
    B->plan.add(B->u_n.data(), B->u_n.size() * 4);
    B->plan.add(B->u_blk.data(), B->u_blk.size() * 4);
    B->plan.add(B->sp_u.data(), B->sp_u.size() * 4);
    B->plan.add(B->sp_c0.data(), B->sp_c0.size() * 4);
    B->plan.add(B->sp_c1.data(), B->sp_c1.size() * 4);
    B->plan.add(B->gen_rows.data(), B->gen_rows.size() * 4);
    B->plan.add(B->w_seq.data(), B->w_seq.size() * 4);
    B->plan.add(B->w_tok0.data(), B->w_tok0.size() * 4);
    B->plan.add(B->w_rows.data(), B->w_rows.size() * 4);
    B->plan.add(B->w_ntok.data(), B->w_ntok.size() * 4);
    B->plan.add(B->w_kend.data(), B->w_kend.size() * 4);
    B->plan.add(B->tok_row.data(), B->tok_row.size() * 4);
    B->plan.add(B->tok_pos.data(), B->tok_pos.size() * 4);
    B->plan.add(B->u_kb0.data(), B->u_kb0.size() * 4);
    B->plan.add(B->w_pair.data(), B->w_pair.size() * 4);
    B->plan.add(B->pair_kend.data(), B->pair_kend.size() * 4);
    B->plan.add(B->cta_seg.data(), B->cta_seg.size() * 4);
    B->plan.add(B->seg.data(), B->seg.size() * 4);
    B->plan.add(B->split.data(), B->split.size() * 4);
    B->plan.add(B->cta_blk.data(), B->cta_blk.size() * 4);
    if (!B->use_tc) B->ctr_zero.clear();
    B->plan.add(B->ctr_zero.data(), B->ctr_zero.size() * 4);  // 22
    if (!B->use_tc) B->u_cta.clear();
    B->plan.add(B->u_cta.data(), B->u_cta.size() * 4);  // 23
    // packed unit records: {t0, n, kb0, row0}, {qpos0, blk0, blk1, tbase}
    B->u_meta.resize(8 * static_cast<size_t>(B->nu));
    for (int u = 0; u < B->nu; ++u) {
        const int i = B->u_seq[u];
        int32_t* r = B->u_meta.data() + 8 * static_cast<size_t>(u);
        r[0] = B->u_t0[u];
        r[1] = B->u_n[u];
        r[2] = B->u_kb0[u];
        r[3] = B->offsets[i] + B->u_t0[u];
        r[4] = B->starts[i] + B->u_t0[u];
        r[5] = B->u_blk[u];
        r[6] = B->u_blk[u + 1];
        r[7] = B->indptr[i] + B->u_kb0[u] - B->u_blk[u];
    }
    B->plan.add(B->u_meta.data(), B->u_meta.size() * 4);  // 24
    // pool slots of the wide-item rows, for their append
    B->w_slots.resize(B->w_rows.size());
    for (size_t x = 0; x < B->w_rows.size(); ++x) {
        const int r = B->w_rows[x];
        const int i = B->row_seq[r];
        const int64_t pos = static_cast<int64_t>(B->starts[i]) + (r - B->offsets[i]);
        const int64_t blk = pos / P->block_size;
        B->w_slots[x] = static_cast<int64_t>(B->ids[B->indptr[i] + blk]) * P->block_size + (pos - blk * P->block_size);
    }
    B->plan.add(B->w_slots.data(), B->w_slots.size() * 8);  // 25
    if (B->nslots > 0)
        PK_CUDA(B->wpart.reserve(static_cast<size_t>(B->nslots) * 2 * 128 * (128 + 2) * sizeof(float)));
    if (!B->w_seq.empty())
        PK_CUDA(B->qpk.reserve((B->w_seq.size() * P->kvh + 1) * static_cast<size_t>(pk::kWideQTileBytes)));
    if (B->nprefix > 0) PK_CUDA(B->lse.reserve(static_cast<size_t>(B->nrows) * H * sizeof(float)));
    int rc = B->plan.commit(st);
    if (rc != PK_OK) return rc;
    B->plan_H = H;
    return PK_OK;
}

// Kinds reported by pk_batch_profile_read.
enum ProfKind { kProfAppend = 0, kProfTc = 1, kProfMerge = 2, kProfGeneric = 3, kProfWide = 4, kProfKinds = 5 };

cudaError_t prof_mark(pk_batch* B, cudaStream_t st) {
    if (!B->profiling) return cudaSuccess;
    if (B->ev_used == B->ev_pool.size()) {
        cudaEvent_t e;
        cudaError_t r = cudaEventCreate(&e);
        if (r != cudaSuccess) return r;
        B->ev_pool.push_back(e);
    }
    return cudaEventRecord(B->ev_pool[B->ev_used++], st);
}

cudaError_t prof_begin(pk_batch* B, cudaStream_t st) { return prof_mark(B, st); }

cudaError_t prof_end(pk_batch* B, int kind, cudaStream_t st) {
    if (!B->profiling) return cudaSuccess;
    B->ev_kind.push_back(kind);
    return prof_mark(B, st);
}

// Row buffers must be 16-byte aligned: the kernels read them with 8- and 16-byte loads.
int check_aligned(const void* p, const char* what) {
    if ((reinterpret_cast<uintptr_t>(p) & 15u) != 0)
        return fail(PK_ERR_INVALID_ARG, "%s is not 16-byte aligned", what);
    return PK_OK;
}

int check_heads(const pk_batch* B, int H) {
    if (H <= 0 || H % B->pool->kvh != 0)
        return fail(PK_ERR_INVALID_ARG, "n_heads=%d is not a positive multiple of n_kv_heads=%d", H,
                    B->pool->kvh);
    return PK_OK;
}

// Wide-tile launch parameters for CTAs [first, first + n) of the plan's schedule.
pk::WideParams wide_params(pk_batch* B, int layer, int H, const float* q, float* out, int first, int n,
                           const float* lse) {
    pk_pool* P = B->pool;
    pk::WideParams w{};
    w.q = q;
    w.out = out;
    w.err = static_cast<int*>(B->err.ptr);
    w.indptr = B->meta.at<int32_t>(0);
    w.ids = B->meta.at<int32_t>(1);
    w.w_seq = B->plan.at<int32_t>(8);
    w.w_tok0 = B->plan.at<int32_t>(9);
    w.w_ntok = B->plan.at<int32_t>(11);
    w.w_kend = B->plan.at<int32_t>(12);
    w.w_pair = B->plan.at<int32_t>(16);
    w.pair_kend = B->plan.at<int32_t>(17);
    w.cta_seg = B->plan.at<int32_t>(18) + first;
    w.seg = B->plan.at<int32_t>(19);
    w.qpk = static_cast<const uint8_t*>(B->qpk.ptr);
    w.q_zero_tile = static_cast<int>(B->w_seq.size()) * P->kvh;
    w.part_o = static_cast<float*>(B->wpart.ptr);
    w.part_ml = static_cast<float*>(B->wpart.ptr) + static_cast<size_t>(B->nslots) * 2 * 128 * 128;
    w.tok_row = B->plan.at<int32_t>(13);
    w.tok_pos = B->plan.at<int32_t>(14);
    w.lse = lse;
    w.nctas = n;
    w.H = H;
    w.kvh = P->kvh;
    w.g = H / P->kvh;
    w.bs = P->block_size;
    w.layer_slot0 = static_cast<int64_t>(layer) * P->num_blocks * P->block_size;
    w.qscale = static_cast<float>(1.4426950408889634 / std::sqrt(static_cast<double>(P->d)));
    return w;
}

// Host-side fault injection for tests: the next attention call of any batch fails as a
// launch error would, before it launches anything.
std::atomic<int> g_inject_launch_failure{0};

int attend_impl(pk_batch* B, int layer, int H, const float* q, float* out, cudaStream_t st,
                const float* k_new = nullptr, const float* v_new = nullptr) {
    // k_new set: fused append - the split-KV kernel appends its units' rows, and the rows
    // of wide-tile sequences are appended just before the wide kernel, on its stream.
    pk_pool* P = B->pool;
    if (g_inject_launch_failure.exchange(0) != 0)
        return fail(PK_ERR_CUDA, "injected launch failure (pk_test_inject_launch_failure)");
    if (B->plan_H != H) {
        int rc = build_attention_plan(B, H, st);
        if (rc != PK_OK) return rc;
    }
    if (B->nrows == 0) return PK_OK;
    const int g = H / P->kvh;
    // ---- wide-tile part (side stream when split-KV work runs beside it)
    cudaStream_t ws = st;
    const int nitems = B->nwide + B->nprefix;
    const bool fork = (B->nwide > 0 || B->nprefix > 0) && B->use_tc;
    if (fork) {
        if (!B->side) PK_CUDA(cudaStreamCreateWithFlags(&B->side, cudaStreamNonBlocking));
        if (!B->ev_fork) PK_CUDA(cudaEventCreateWithFlags(&B->ev_fork, cudaEventDisableTiming));
        if (!B->ev_join) PK_CUDA(cudaEventCreateWithFlags(&B->ev_join, cudaEventDisableTiming));
        if (!B->ev_pack) PK_CUDA(cudaEventCreateWithFlags(&B->ev_pack, cudaEventDisableTiming));
        PK_CUDA(cudaEventRecord(B->ev_fork, st));
        PK_CUDA(cudaStreamWaitEvent(B->side, B->ev_fork, 0));
        if (B->nwide > 0) ws = B->side;
    }
    // Query tiles of every wide item are packed once (bf16 shared-memory images the wide
    // kernel fetches with one bulk copy). With chunk items that happens in the same launch
    // as the chunk rows' append, on the wide stream; with only a shared-prefix pass the pack
    // runs on the side stream beside the split-KV kernel (or first, without one).
    bool pack_on_side = false;
    if (B->nwide == 0 && B->nprefix > 0) {
        const pk::WideParams wp = wide_params(B, layer, H, q, out, 0, 0, nullptr);
        cudaStream_t ps = fork ? B->side : st;
        PK_CUDA(pk::launch_wide_q_pack(wp, nitems, static_cast<uint8_t*>(B->qpk.ptr), ps));
        B->launches++;
        if (ps != st) {
            PK_CUDA(cudaEventRecord(B->ev_pack, ps));
            pack_on_side = true;
        }
    }
    if (B->nwide > 0) {
        const pk::WideParams wp = wide_params(B, layer, H, q, out, 0, 0, nullptr);
        pk::WideAppend a{};
        if (k_new != nullptr) {
            a.pool_k = reinterpret_cast<__nv_bfloat16*>(P->k_layer(layer));
            a.pool_v = reinterpret_cast<__nv_bfloat16*>(P->v_layer(layer));
            a.k = k_new;
            a.v = v_new;
            a.row_seq = B->meta.at<int32_t>(4);
            a.offsets = B->meta.at<int32_t>(3);
            a.starts = B->meta.at<int32_t>(2);
            a.indptr = B->meta.at<int32_t>(0);
            a.ids = B->meta.at<int32_t>(1);
            a.rows = B->plan.at<int32_t>(10);
            a.slots = B->plan.at<int64_t>(25);
            a.n = static_cast<int64_t>(B->w_rows.size());
            a.rowlen = P->kvh * P->d;
            a.bs = P->block_size;
        }
        PK_CUDA(prof_begin(B, ws));
        PK_CUDA(pk::launch_wide_prep(wp, nitems, static_cast<uint8_t*>(B->qpk.ptr), a, ws));
        PK_CUDA(prof_end(B, kProfAppend, ws));
        B->launches++;
        if (B->nprefix > 0 && ws != st) {
            PK_CUDA(cudaEventRecord(B->ev_pack, ws));
            pack_on_side = true;
        }
        const pk::WideParams w = wide_params(B, layer, H, q, out, 0, B->ncta_chunk, nullptr);
        PK_CUDA(prof_begin(B, ws));
        PK_CUDA(pk::launch_wide_attention(&P->tmk1, &P->tmv1, w, ws));
        B->launches++;
        if (B->nwsplit_chunk > 0) {  // chunk pair-heads cut between CTAs: normalised merge
            PK_CUDA(pk::launch_wide_merge(w, B->plan.at<int32_t>(20), B->nwsplit_chunk, ws));
            B->launches++;
        }
        PK_CUDA(prof_end(B, kProfWide, ws));
    }
    if (B->use_tc) {
        pk::TcParams p{};
        p.q = q;
        p.out = out;
        p.part_o = static_cast<float*>(B->ws.ptr);
        p.part_ml = static_cast<float*>(B->ws.ptr) + B->ws_part_o_floats;
        p.err = static_cast<int*>(B->err.ptr);
        p.indptr = B->meta.at<int32_t>(0);
        p.ids = B->meta.at<int32_t>(1);
        p.starts = B->meta.at<int32_t>(2);
        p.offsets = B->meta.at<int32_t>(3);
        p.u_seq = B->plan.at<int32_t>(0);
        p.u_t0 = B->plan.at<int32_t>(1);
        p.u_n = B->plan.at<int32_t>(2);
        p.u_blk = B->plan.at<int32_t>(3);
        p.u_kb0 = B->nprefix > 0 ? B->plan.at<int32_t>(15) : nullptr;
        p.lse = B->nprefix > 0 ? static_cast<float*>(B->lse.ptr) : nullptr;
        p.nu = B->nu;
        p.total_blocks = B->total_blocks;
        p.ncta = B->ncta;
        p.cta_blk = B->plan.at<int32_t>(21);
        p.u_cta = B->plan.at<int32_t>(23);
        p.u_meta = B->nu > 0 ? B->plan.at<int4>(24) : nullptr;
        p.kvh = P->kvh;
        p.g = g;
        p.H = H;
        p.bs = P->block_size;
        p.stages = P->tc_stages;
        p.virt = P->tc_virt;
        p.per_head_layout = P->tc_per_head;
        p.layer_slot0 = static_cast<int64_t>(layer) * P->num_blocks * P->block_size;
        p.qscale = static_cast<float>(1.4426950408889634 / std::sqrt(static_cast<double>(P->d)));
        p.counters = B->plan.at<int>(22);
        p.unit_counters = p.counters + (static_cast<size_t>(B->nu) + B->ncta) * P->kvh;
        p.k_new = k_new;
        p.v_new = v_new;
        p.pool_k = reinterpret_cast<__nv_bfloat16*>(P->k_layer(layer));
        p.pool_v = reinterpret_cast<__nv_bfloat16*>(P->v_layer(layer));
        p.peer = B->peer_out;
        const size_t smem = P->tc_smem + (p.peer.n > 0 ? pk::tc_peer_stage_bytes(P->d) : 0);
        PK_CUDA(prof_begin(B, st));
        PK_CUDA(pk::launch_tc_attention(P->d, B->nt, &P->tmk, &P->tmv, p, smem, st));
        PK_CUDA(prof_end(B, kProfTc, st));
        B->launches++;
        if (B->nsplit > 0 && p.counters == nullptr) {
            pk::MergeParams m{};
            m.out = out;
            m.part_o = p.part_o;
            m.part_ml = p.part_ml;
            m.offsets = p.offsets;
            m.u_seq = p.u_seq;
            m.u_t0 = p.u_t0;
            m.u_n = p.u_n;
            m.split_u = B->plan.at<int32_t>(4);
            m.split_c0 = B->plan.at<int32_t>(5);
            m.split_c1 = B->plan.at<int32_t>(6);
            m.kvh = P->kvh;
            m.g = g;
            m.H = H;
            m.D = P->d;
            m.nt = B->nt;
            PK_CUDA(prof_begin(B, st));
            PK_CUDA(pk::launch_merge(m, B->nsplit, st));
            PK_CUDA(prof_end(B, kProfMerge, st));
            B->launches++;
        }
    }
    if (B->nprefix > 0) {
        // shared-prefix items: after the split-KV kernel has written the rows they merge into
        const pk::WideParams w = wide_params(B, layer, H, q, out, B->ncta_chunk, B->ncta_prefix,
                                             static_cast<const float*>(B->lse.ptr));
        if (pack_on_side) PK_CUDA(cudaStreamWaitEvent(st, B->ev_pack, 0));
        PK_CUDA(prof_begin(B, st));
        PK_CUDA(pk::launch_wide_attention(&P->tmk1, &P->tmv1, w, st));
        if (B->nwsplit > B->nwsplit_chunk) {
            PK_CUDA(pk::launch_wide_merge(w, B->plan.at<int32_t>(20) + 4 * B->nwsplit_chunk,
                                          B->nwsplit - B->nwsplit_chunk, st));
            B->launches++;
        }
        PK_CUDA(prof_end(B, kProfWide, st));
        B->launches++;
    }
    if (fork) {
        // everything issued on the side stream (append, chunk tiles, or the pack) before the
        // caller's stream moves on
        PK_CUDA(cudaEventRecord(B->ev_join, B->side));
        PK_CUDA(cudaStreamWaitEvent(st, B->ev_join, 0));
    }
    if (B->ngeneric > 0) {
        if (P->d > 512) return fail(PK_ERR_UNSUPPORTED, "head_dim %d > 512", P->d);
        pk::GenericParams p{};
        p.q = q;
        p.out = out;
        p.pool_k = P->k_layer(layer);
        p.pool_v = P->v_layer(layer);
        p.row_seq = B->meta.at<int32_t>(4);
        p.indptr = B->meta.at<int32_t>(0);
        p.ids = B->meta.at<int32_t>(1);
        p.starts = B->meta.at<int32_t>(2);
        p.offsets = B->meta.at<int32_t>(3);
        p.rows = B->plan.at<int32_t>(7);
        p.nrows = B->ngeneric;
        p.H = H;
        p.kvh = P->kvh;
        p.D = P->d;
        p.bs = P->block_size;
        p.scale = static_cast<float>(1.0 / std::sqrt(static_cast<double>(P->d)));
        p.k_new = k_new;  // fused calls only (then every row of the step is on this kernel)
        p.v_new = v_new;
        PK_CUDA(prof_begin(B, st));
        PK_CUDA(pk::launch_generic_attention(P->dtype, p, st));
        PK_CUDA(prof_end(B, kProfGeneric, st));
        B->launches++;
    }
    return PK_OK;
}

}  // namespace

void pk_set_last_error(const char* msg) { g_err = msg ? msg : ""; }

bool pk_pool_view(const pk_pool* P, pk::PoolView* v) {
    if (!P || !v) return false;
    v->device = P->device;
    v->n_layers = P->n_layers;
    v->num_blocks = P->num_blocks;
    v->block_size = P->block_size;
    v->kvh = P->kvh;
    v->d = P->d;
    v->dtype = P->dtype;
    v->num_sms = P->num_sms;
    v->tc_ok = P->tc_ok;
    v->tc_per_head = P->tc_per_head;
    v->tc_stages = P->tc_stages;
    v->tc_virt = P->tc_virt;
    v->tc_smem = P->tc_smem;
    v->tmk = &P->tmk;
    v->tmv = &P->tmv;
    return true;
}

extern "C" {

const char* pk_last_error(void) { return g_err.c_str(); }

int pk_abi_version(void) { return 1; }

int pk_pool_create(int n_layers, int64_t num_blocks, int block_size, int n_kv_heads, int head_dim,
                   int dtype, int device, pk_pool** out) {
    if (!out) return fail(PK_ERR_INVALID_ARG, "out is NULL");
    *out = nullptr;
    if (n_layers <= 0 || num_blocks <= 0 || block_size <= 0 || n_kv_heads <= 0 || head_dim <= 0)
        return fail(PK_ERR_INVALID_ARG, "pool dimensions must be positive");
    if (dtype != PK_F32 && dtype != PK_BF16) return fail(PK_ERR_INVALID_ARG, "unknown dtype %d", dtype);
    if (num_blocks >= (int64_t(1) << 31)) return fail(PK_ERR_INVALID_ARG, "num_blocks must be < 2^31");
    DeviceScope ds(device);
    if (ds.err != cudaSuccess) return fail(PK_ERR_CUDA, "cudaSetDevice(%d): %s", device, cudaGetErrorString(ds.err));
    auto* P = new pk_pool();
    P->device = device;
    P->n_layers = n_layers;
    P->num_blocks = num_blocks;
    P->block_size = block_size;
    P->kvh = n_kv_heads;
    P->d = head_dim;
    P->dtype = dtype;
    P->esize = dtype == PK_F32 ? 4 : 2;
    P->layer_elems = num_blocks * block_size * static_cast<int64_t>(n_kv_heads) * head_dim;
    const size_t bytes = static_cast<size_t>(n_layers) * P->layer_bytes();
    cudaError_t e = cudaMalloc(&P->k, bytes);
    if (e == cudaSuccess) e = cudaMalloc(&P->v, bytes);
    if (e == cudaSuccess) e = cudaMemset(P->k, 0, bytes);
    if (e == cudaSuccess) e = cudaMemset(P->v, 0, bytes);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&P->num_sms, cudaDevAttrMultiProcessorCount, device);
    if (e != cudaSuccess) {
        if (P->k) cudaFree(P->k);
        if (P->v) cudaFree(P->v);
        delete P;
        return fail(PK_ERR_CUDA, "pool allocation of 2 x %zu bytes: %s", bytes, cudaGetErrorString(e));
    }
    setup_tc(P);
    *out = P;
    return PK_OK;
}

int pk_pool_destroy(pk_pool* pool) {
    if (!pool) return PK_OK;
    DeviceScope ds(pool->device);
    pool->pairs_up.release();
    if (pool->k) cudaFree(pool->k);
    if (pool->v) cudaFree(pool->v);
    delete pool;
    return PK_OK;
}

int pk_pool_buffers(const pk_pool* pool, void** k_dev, void** v_dev, int64_t* nbytes) {
    if (!pool) return fail(PK_ERR_INVALID_ARG, "pool is NULL");
    if (k_dev) *k_dev = pool->k;
    if (v_dev) *v_dev = pool->v;
    if (nbytes) *nbytes = 2 * static_cast<int64_t>(pool->n_layers) * pool->layer_bytes();
    return PK_OK;
}

int pk_pool_tc_info(const pk_pool* pool, int* enabled, int* per_head_layout, int* stages,
                    const char** why) {
    if (!pool) return fail(PK_ERR_INVALID_ARG, "pool is NULL");
    if (enabled) *enabled = pool->tc_ok ? 1 : 0;
    if (per_head_layout) *per_head_layout = pool->tc_per_head;
    if (stages) *stages = pool->tc_stages;
    if (why) *why = pool->tc_why.c_str();
    return PK_OK;
}

int pk_pool_copy_blocks_dev(pk_pool* pool, const int64_t* pairs_dev, int64_t npairs, void* stream) {
    if (!pool) return fail(PK_ERR_INVALID_ARG, "pool is NULL");
    if (npairs < 0) return fail(PK_ERR_INVALID_ARG, "npairs < 0");
    if (npairs == 0) return PK_OK;
    if (!pairs_dev) return fail(PK_ERR_INVALID_ARG, "pairs is NULL");
    DeviceScope ds(pool->device);
    PK_CUDA(pk::launch_copy_blocks(pool->k, pool->v, pairs_dev, npairs, pool->n_layers,
                                   static_cast<int64_t>(pool->layer_bytes()),
                                   static_cast<int64_t>(pool->block_bytes()),
                                   static_cast<cudaStream_t>(stream)));
    return PK_OK;
}

int pk_pool_copy_blocks(pk_pool* pool, const int64_t* pairs_host, int64_t npairs, void* stream) {
    if (!pool) return fail(PK_ERR_INVALID_ARG, "pool is NULL");
    if (npairs < 0) return fail(PK_ERR_INVALID_ARG, "npairs < 0");
    if (npairs == 0) return PK_OK;
    if (!pairs_host) return fail(PK_ERR_INVALID_ARG, "pairs is NULL");
    for (int64_t i = 0; i < 2 * npairs; ++i)
        if (pairs_host[i] < 0 || pairs_host[i] >= pool->num_blocks)
            return fail(PK_ERR_OUT_OF_RANGE, "copy pair %lld: block id %lld outside [0, %lld)",
                        (long long)(i / 2), (long long)pairs_host[i], (long long)pool->num_blocks);
    DeviceScope ds(pool->device);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    // Pairs run as one launch when no copy reads or overwrites another's destination;
    // otherwise they are cut into consecutive groups that keep list order.
    std::vector<int64_t> group_start{0};
    {
        std::vector<char> is_dst(static_cast<size_t>(pool->num_blocks), 0);
        std::vector<char> is_src(static_cast<size_t>(pool->num_blocks), 0);
        std::vector<int64_t> touched;
        for (int64_t i = 0; i < npairs; ++i) {
            const int64_t s = pairs_host[2 * i], d = pairs_host[2 * i + 1];
            if (is_dst[s] || is_dst[d] || is_src[d]) {
                for (int64_t b : touched) is_dst[b] = is_src[b] = 0;
                touched.clear();
                group_start.push_back(i);
            }
            is_src[s] = 1;
            is_dst[d] = 1;
            touched.push_back(s);
            touched.push_back(d);
        }
    }
    group_start.push_back(npairs);
    Uploader& up = pool->pairs_up;
    up.begin();
    up.add(pairs_host, static_cast<size_t>(npairs) * 16);
    int rc = up.commit(st);
    if (rc != PK_OK) return rc;
    const int64_t* dev = up.at<int64_t>(0);
    for (size_t gi = 0; gi + 1 < group_start.size(); ++gi) {
        const int64_t a = group_start[gi], b = group_start[gi + 1];
        PK_CUDA(pk::launch_copy_blocks(pool->k, pool->v, dev + 2 * a, b - a, pool->n_layers,
                                       static_cast<int64_t>(pool->layer_bytes()),
                                       static_cast<int64_t>(pool->block_bytes()), st));
    }
    return PK_OK;
}

int pk_pool_append(pk_pool* pool, int layer, const float* k_dev, const float* v_dev,
                   const int64_t* slots_dev, int64_t n, void* stream) {
    if (!pool) return fail(PK_ERR_INVALID_ARG, "pool is NULL");
    if (layer < 0 || layer >= pool->n_layers) return fail(PK_ERR_OUT_OF_RANGE, "layer %d", layer);
    if (n < 0) return fail(PK_ERR_INVALID_ARG, "n < 0");
    if (n == 0) return PK_OK;
    if (!k_dev || !v_dev || !slots_dev) return fail(PK_ERR_INVALID_ARG, "NULL pointer");
    DeviceScope ds(pool->device);
    PK_CUDA(pk::launch_append(pool->dtype, pool->k_layer(layer), pool->v_layer(layer), k_dev, v_dev,
                              slots_dev, nullptr, n, pool->kvh * pool->d, static_cast<cudaStream_t>(stream)));
    return PK_OK;
}

int pk_slot_mapping(const int32_t* table_dev, int64_t table_len, const int64_t* positions_dev,
                    int64_t n, int block_size, int64_t* slots_dev, int32_t* err_dev, void* stream) {
    if (n < 0 || table_len < 0 || block_size <= 0) return fail(PK_ERR_INVALID_ARG, "bad sizes");
    if (n == 0) return PK_OK;
    if (!positions_dev || !slots_dev || (!table_dev && table_len > 0))
        return fail(PK_ERR_INVALID_ARG, "NULL pointer");
    PK_CUDA(pk::launch_slot_mapping(table_dev, table_len, positions_dev, n, block_size, slots_dev,
                                    err_dev, static_cast<cudaStream_t>(stream)));
    return PK_OK;
}

int pk_batch_create(pk_pool* pool, pk_batch** out) {
    if (!pool || !out) return fail(PK_ERR_INVALID_ARG, "NULL pointer");
    DeviceScope ds(pool->device);
    auto* B = new pk_batch();
    B->pool = pool;
    cudaError_t e = B->err.reserve(sizeof(int));
    if (e == cudaSuccess) e = cudaMemset(B->err.ptr, 0, sizeof(int));
    if (e != cudaSuccess) {
        delete B;
        return fail(PK_ERR_CUDA, "batch error word: %s", cudaGetErrorString(e));
    }
    *out = B;
    return PK_OK;
}

int pk_batch_destroy(pk_batch* B) {
    if (!B) return PK_OK;
    DeviceScope ds(B->pool->device);
    B->meta.release();
    B->plan.release();
    B->rows.release();
    B->err.release();
    B->ws.release();
    B->io.release();
    B->lse.release();
    B->wpart.release();
    B->qpk.release();
    for (cudaEvent_t e : B->ev_pool) cudaEventDestroy(e);
    if (B->ev_fork) cudaEventDestroy(B->ev_fork);
    if (B->ev_join) cudaEventDestroy(B->ev_join);
    if (B->ev_pack) cudaEventDestroy(B->ev_pack);
    if (B->side) cudaStreamDestroy(B->side);
    delete B;
    return PK_OK;
}

int pk_batch_plan(pk_batch* B, int nseq, const int64_t* table_indptr, const int32_t* table_ids,
                  const int64_t* starts, const int64_t* n_new, int64_t* n_rows, void* stream) {
    if (!B) return fail(PK_ERR_INVALID_ARG, "batch is NULL");
    if (nseq < 0) return fail(PK_ERR_INVALID_ARG, "nseq < 0");
    if (nseq > 0 && (!table_indptr || !starts || !n_new))
        return fail(PK_ERR_INVALID_ARG, "NULL pointer");
    pk_pool* P = B->pool;
    const int bs = P->block_size;
    B->plan_H = -1;
    B->nseq = 0;
    B->nrows = 0;
    B->indptr.assign(1, 0);
    B->ids.clear();
    B->starts.clear();
    B->nnew.clear();
    B->offsets.assign(1, 0);
    B->row_seq.clear();
    if (nseq > 0 && table_indptr[0] != 0) return fail(PK_ERR_INVALID_ARG, "table_indptr[0] != 0");
    int64_t rows = 0;
    for (int i = 0; i < nseq; ++i) {
        const int64_t s = starts[i], n = n_new[i];
        const int64_t tb = table_indptr[i], te = table_indptr[i + 1];
        if (s < 0 || n < 0) return fail(PK_ERR_INVALID_ARG, "seq %d: start %lld / n_new %lld negative", i, (long long)s, (long long)n);
        if (te < tb) return fail(PK_ERR_INVALID_ARG, "table_indptr not non-decreasing at seq %d", i);
        const int64_t ctx = s + n;
        if (ctx >= (int64_t(1) << 31)) return fail(PK_ERR_UNSUPPORTED, "seq %d: context %lld too long", i, (long long)ctx);
        const int64_t need = (ctx + bs - 1) / bs;
        if (need > te - tb)
            return fail(PK_ERR_OUT_OF_RANGE, "seq %d: positions up to %lld need %lld blocks, table has %lld",
                        i, (long long)(ctx - 1), (long long)need, (long long)(te - tb));
        if (need > 0 && !table_ids) return fail(PK_ERR_INVALID_ARG, "table_ids is NULL");
        // range check as a min / max reduction (vectorised); the offender only on failure
        int32_t lo = 0, hi = 0;
        if (need > 0) {
            lo = hi = table_ids[tb];
            for (int64_t j = tb + 1; j < tb + need; ++j) {
                lo = std::min(lo, table_ids[j]);
                hi = std::max(hi, table_ids[j]);
            }
        }
        if (lo < 0 || hi >= P->num_blocks) {
            for (int64_t j = tb; j < tb + need; ++j) {
                const int32_t b = table_ids[j];
                if (b < 0 || b >= P->num_blocks)
                    return fail(PK_ERR_OUT_OF_RANGE, "seq %d: block id %d outside [0, %lld)", i, b,
                                (long long)P->num_blocks);
            }
        }
        // Only the referenced prefix of each table is uploaded.
        B->ids.insert(B->ids.end(), table_ids + tb, table_ids + tb + need);
        if (B->ids.size() >= (size_t(1) << 31)) return fail(PK_ERR_UNSUPPORTED, "too many table entries");
        B->indptr.push_back(static_cast<int32_t>(B->ids.size()));
        B->starts.push_back(static_cast<int32_t>(s));
        B->nnew.push_back(static_cast<int32_t>(n));
        rows += n;
        if (rows >= (int64_t(1) << 31)) return fail(PK_ERR_UNSUPPORTED, "too many rows");
        B->offsets.push_back(static_cast<int32_t>(rows));
        for (int64_t r = 0; r < n; ++r) B->row_seq.push_back(i);
    }
    // Written blocks: which (sequence, table index) writes each; any other reference to
    // such a block, or two writers, rules the fused append out for this step.
    B->fuse_append_ok = true;
    B->app_rows.clear();
    if (B->writer_seq.size() != static_cast<size_t>(P->num_blocks)) {
        B->writer_seq.assign(P->num_blocks, -1);
        B->writer_idx.assign(P->num_blocks, -1);
        B->written.assign((P->num_blocks + 63) / 64, 0);
    }
    std::vector<int32_t> touched;
    bool dup_slot = false;
    for (int i = 0; i < nseq && B->fuse_append_ok; ++i) {
        for (int64_t pos = B->starts[i]; pos < static_cast<int64_t>(B->starts[i]) + B->nnew[i]; ++pos) {
            const int32_t j = static_cast<int32_t>(pos / bs);
            const int32_t b = B->ids[B->indptr[i] + j];
            if (B->writer_seq[b] < 0) {
                B->writer_seq[b] = i;
                B->writer_idx[b] = j;
                B->written[b >> 6] |= uint64_t(1) << (b & 63);
                touched.push_back(b);
            } else if (B->writer_seq[b] != i || B->writer_idx[b] != j) {
                B->fuse_append_ok = false;
                dup_slot = true;  // may share a slot: resolve last writers below
                break;
            }
        }
    }
    // every table entry against the written set: a bitmap (one bit per block, L1-resident)
    // first, the writer's (sequence, index) only for written blocks
    const uint64_t* wbits = B->written.data();
    for (int i = 0; i < nseq && B->fuse_append_ok; ++i) {
        const int32_t* t = B->ids.data() + B->indptr[i];
        const int32_t n = B->indptr[i + 1] - B->indptr[i];
        for (int32_t j = 0; j < n; ++j) {
            const int32_t b = t[j];
            if (((wbits[b >> 6] >> (b & 63)) & 1) && (B->writer_seq[b] != i || B->writer_idx[b] != j)) {
                B->fuse_append_ok = false;
                break;
            }
        }
    }
    for (int32_t b : touched) {
        B->writer_seq[b] = B->writer_idx[b] = -1;
        B->written[b >> 6] = 0;
    }
    if (dup_slot) {
        // last row wins per slot (numpy fancy assignment order)
        std::unordered_map<int64_t, int32_t> last;
        last.reserve(static_cast<size_t>(rows) * 2);
        int32_t r = 0;
        for (int i = 0; i < nseq; ++i)
            for (int64_t pos = B->starts[i]; pos < static_cast<int64_t>(B->starts[i]) + B->nnew[i]; ++pos, ++r) {
                const int64_t slot = static_cast<int64_t>(B->ids[B->indptr[i] + pos / bs]) * bs + pos % bs;
                last[slot] = r;
            }
        r = 0;
        for (int i = 0; i < nseq; ++i)
            for (int64_t pos = B->starts[i]; pos < static_cast<int64_t>(B->starts[i]) + B->nnew[i]; ++pos, ++r) {
                const int64_t slot = static_cast<int64_t>(B->ids[B->indptr[i] + pos / bs]) * bs + pos % bs;
                if (last[slot] == r) B->app_rows.push_back(r);
            }
    }
    B->nseq = nseq;
    B->nrows = rows;
    if (n_rows) *n_rows = rows;
    DeviceScope ds(P->device);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    B->meta.begin();
    B->meta.add(B->indptr.data(), B->indptr.size() * 4);
    B->meta.add(B->ids.data(), B->ids.size() * 4);
    B->meta.add(B->starts.data(), B->starts.size() * 4);
    B->meta.add(B->offsets.data(), B->offsets.size() * 4);
    B->meta.add(B->row_seq.data(), B->row_seq.size() * 4);
    B->meta.add(B->app_rows.data(), B->app_rows.size() * 4);
    int rc = B->meta.commit(st);
    if (rc != PK_OK) return rc;
    PK_CUDA(B->rows.reserve(static_cast<size_t>(std::max<int64_t>(rows, 1)) * 16));
    B->rows_pending = rows > 0;  // built by the first reader (ensure_rows)
    B->rows_stream = st;
    return PK_OK;
}

int pk_batch_rows(const pk_batch* B, const int64_t** positions_dev, const int64_t** slots_dev) {
    if (!B) return fail(PK_ERR_INVALID_ARG, "batch is NULL");
    DeviceScope ds(B->pool->device);
    PK_CUDA(ensure_rows(B, B->rows_stream));
    if (positions_dev) *positions_dev = B->positions();
    if (slots_dev) *slots_dev = B->slots();
    return PK_OK;
}

int pk_batch_attend(pk_batch* B, int layer, int n_heads, const float* q_dev, float* out_dev,
                    void* stream) {
    if (!B) return fail(PK_ERR_INVALID_ARG, "batch is NULL");
    int rc = check_heads(B, n_heads);
    if (rc != PK_OK) return rc;
    if (layer < 0 || layer >= B->pool->n_layers) return fail(PK_ERR_OUT_OF_RANGE, "layer %d", layer);
    if (B->nrows > 0 && (!q_dev || !out_dev)) return fail(PK_ERR_INVALID_ARG, "NULL pointer");
    if ((rc = check_aligned(q_dev, "q")) || (rc = check_aligned(out_dev, "out"))) return rc;
    DeviceScope ds(B->pool->device);
    B->launches = 0;
    return attend_impl(B, layer, n_heads, q_dev, out_dev, static_cast<cudaStream_t>(stream));
}

int pk_batch_write_and_attend(pk_batch* B, int layer, int n_heads, const float* q_dev,
                              const float* k_dev, const float* v_dev, float* out_dev, void* stream) {
    if (!B) return fail(PK_ERR_INVALID_ARG, "batch is NULL");
    int rc = check_heads(B, n_heads);
    if (rc != PK_OK) return rc;
    pk_pool* P = B->pool;
    if (layer < 0 || layer >= P->n_layers) return fail(PK_ERR_OUT_OF_RANGE, "layer %d", layer);
    if (B->nrows > 0 && (!q_dev || !k_dev || !v_dev || !out_dev))
        return fail(PK_ERR_INVALID_ARG, "NULL pointer");
    if ((rc = check_aligned(q_dev, "q")) || (rc = check_aligned(k_dev, "k")) ||
        (rc = check_aligned(v_dev, "v")) || (rc = check_aligned(out_dev, "out")))
        return rc;
    DeviceScope ds(P->device);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    B->launches = 0;
    if (B->plan_H != n_heads) {
        rc = build_attention_plan(B, n_heads, st);
        if (rc != PK_OK) return rc;
    }
    // Fused append (rows patched into the attention kernels' shared memory) pays off for
    // decode steps; with several new tokens per sequence one scatter kernel first is faster
    // than each unit fetching its rows on its critical path.
    if (B->ngeneric == 0 && B->fuse_append_ok && (B->use_tc || B->nwide > 0) && B->tc_max_new <= kFuseMaxNew)
        return attend_impl(B, layer, n_heads, q_dev, out_dev, st, k_dev, v_dev);
    // A step wholly on the CUDA-core kernel appends inside it as well: its CTAs read the
    // step's rows from the inputs and one CTA per (row, KV head) stores each to the pool.
    if (B->ngeneric > 0 && !B->use_tc && B->nwide == 0 && B->fuse_append_ok)
        return attend_impl(B, layer, n_heads, q_dev, out_dev, st, k_dev, v_dev);
    if (B->nrows > 0) {
        const bool listed = !B->app_rows.empty();
        PK_CUDA(prof_begin(B, st));
        PK_CUDA(pk::launch_append_table(P->dtype, P->k_layer(layer), P->v_layer(layer), k_dev, v_dev,
                                        B->meta.at<int32_t>(4), B->meta.at<int32_t>(3), B->meta.at<int32_t>(2),
                                        B->meta.at<int32_t>(0), B->meta.at<int32_t>(1), P->block_size,
                                        listed ? B->meta.at<int32_t>(5) : nullptr,
                                        listed ? static_cast<int64_t>(B->app_rows.size()) : B->nrows,
                                        P->kvh * P->d, st));
        PK_CUDA(prof_end(B, kProfAppend, st));
        B->launches++;
    }
    return attend_impl(B, layer, n_heads, q_dev, out_dev, st);
}

int pk_peer_gather_write_and_attend(pk_peer_gather* g, pk_batch* B, int layer, int n_heads,
                                    const float* q_dev, const float* k_dev, const float* v_dev,
                                    float** result_dev, void* stream) {
    if (!g || !B || !result_dev) return fail(PK_ERR_INVALID_ARG, "NULL pointer");
    int rc = check_heads(B, n_heads);
    if (rc != PK_OK) return rc;
    pk_pool* P = B->pool;
    if (layer < 0 || layer >= P->n_layers) return fail(PK_ERR_OUT_OF_RANGE, "layer %d", layer);
    if (B->nrows > 0 && (!q_dev || !k_dev || !v_dev)) return fail(PK_ERR_INVALID_ARG, "NULL pointer");
    if ((rc = check_aligned(q_dev, "q")) || (rc = check_aligned(k_dev, "k")) || (rc = check_aligned(v_dev, "v")))
        return rc;
    DeviceScope ds(P->device);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (B->plan_H != n_heads) {
        rc = build_attention_plan(B, n_heads, st);
        if (rc != PK_OK) return rc;
    }
    const int64_t row_floats = static_cast<int64_t>(n_heads) * P->d;
    // One split-KV launch writes every output row of such a step: the exchange rides on it
    // (if the launch's shared memory has room for the rows' staging).
    if (B->nrows > 0 && B->use_tc && B->nwide == 0 && B->nprefix == 0 && B->ngeneric == 0 &&
        P->tc_smem + pk::tc_peer_stage_bytes(P->d) <= static_cast<size_t>(P->smem_optin)) {
        float* res = nullptr;
        rc = pk_peer_gather_step(g, B->nrows, row_floats, P->d, &B->peer_out, &res);
        if (rc != PK_OK) return rc;
        rc = pk_batch_write_and_attend(B, layer, n_heads, q_dev, k_dev, v_dev, res, stream);
        B->peer_out = pk::PeerOut{};
        if (rc != PK_OK) return rc;
        *result_dev = res;
        return PK_OK;
    }
    // Otherwise the attention writes this rank's slice, and one push launch exchanges it.
    const float* slice = nullptr;
    if (B->nrows > 0) {
        PK_CUDA(B->peer_slice.reserve(static_cast<size_t>(B->nrows) * row_floats * sizeof(float)));
        rc = pk_batch_write_and_attend(B, layer, n_heads, q_dev, k_dev, v_dev, static_cast<float*>(B->peer_slice.ptr),
                                       stream);
        if (rc != PK_OK) return rc;
        slice = static_cast<const float*>(B->peer_slice.ptr);
    }
    return pk_peer_gather_heads(g, slice, B->nrows, row_floats, result_dev, stream);
}

int pk_batch_write_and_attend_host(pk_batch* B, int layer, int n_heads, const float* q_host,
                                   const float* k_host, const float* v_host, float* out_host,
                                   void* stream) {
    if (!B) return fail(PK_ERR_INVALID_ARG, "batch is NULL");
    int rc = check_heads(B, n_heads);
    if (rc != PK_OK) return rc;
    pk_pool* P = B->pool;
    if (B->nrows > 0 && (!q_host || !k_host || !v_host || !out_host))
        return fail(PK_ERR_INVALID_ARG, "NULL pointer");
    DeviceScope ds(P->device);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const size_t qn = static_cast<size_t>(B->nrows) * n_heads * P->d;
    const size_t kn = static_cast<size_t>(B->nrows) * P->kvh * P->d;
    const auto up = [](size_t floats) { return (floats + 63) & ~size_t(63); };  // 256 B
    PK_CUDA(B->io.reserve((2 * up(qn) + 2 * up(kn)) * sizeof(float)));
    float* qd = static_cast<float*>(B->io.ptr);
    float* kd = qd + up(qn);
    float* vd = kd + up(kn);
    float* od = vd + up(kn);
    B->io_h2d = B->io_d2h = B->io_direct = 0;
    if (B->nrows > 0) {
        // Inputs in page-locked memory the device can address come over in one launch that
        // reads all three (many reads in flight on the host link at once); other memory by the
        // copy engine, one copy each.
        const float* qm = static_cast<const float*>(mapped_host_range(q_host, qn * sizeof(float)));
        const float* km = qm ? static_cast<const float*>(mapped_host_range(k_host, kn * sizeof(float))) : nullptr;
        const float* vm = km ? static_cast<const float*>(mapped_host_range(v_host, kn * sizeof(float))) : nullptr;
        if (vm && qn % 4 == 0 && kn % 4 == 0) {
            PK_CUDA(pk::launch_h2d_gather(qm, qd, static_cast<int64_t>(qn), km, kd, static_cast<int64_t>(kn), vm, vd,
                                          static_cast<int64_t>(kn), st));
        } else {
            PK_CUDA(cudaMemcpyAsync(qd, q_host, qn * sizeof(float), cudaMemcpyHostToDevice, st));
            PK_CUDA(cudaMemcpyAsync(kd, k_host, kn * sizeof(float), cudaMemcpyHostToDevice, st));
            PK_CUDA(cudaMemcpyAsync(vd, v_host, kn * sizeof(float), cudaMemcpyHostToDevice, st));
        }
        B->io_h2d = static_cast<int64_t>(qn + 2 * kn) * sizeof(float);
        // the attention plan now, while the copies run (pk_batch_write_and_attend reuses it)
        if (layer >= 0 && layer < P->n_layers && B->plan_H != n_heads) {
            rc = build_attention_plan(B, n_heads, st);
            if (rc != PK_OK) return rc;
        }
        // A page-locked result buffer is stored into by the kernels themselves: the result
        // crosses PCIe while the attention runs instead of in a copy after it. Not with a
        // shared-prefix pass, which reads the split-KV rows back from the output.
        if (B->plan_H == n_heads && B->nprefix == 0) {
            if (float* direct = static_cast<float*>(mapped_host_range(out_host, qn * sizeof(float)))) {
                od = direct;
                B->io_direct = static_cast<int64_t>(qn) * sizeof(float);
            }
        }
    }
    rc = pk_batch_write_and_attend(B, layer, n_heads, qd, kd, vd, od, stream);
    if (rc != PK_OK) return rc;
    if (B->nrows > 0 && B->io_direct == 0) {
        PK_CUDA(cudaMemcpyAsync(out_host, od, qn * sizeof(float), cudaMemcpyDeviceToHost, st));
        B->io_d2h = static_cast<int64_t>(qn) * sizeof(float);
    }
    PK_CUDA(cudaStreamSynchronize(st));
    return PK_OK;
}

int pk_batch_io_stats(const pk_batch* B, int64_t* s) {
    if (!B || !s) return fail(PK_ERR_INVALID_ARG, "NULL pointer");
    s[0] = B->io_h2d;
    s[1] = B->io_d2h;
    s[2] = B->io_direct;
    return PK_OK;
}

int pk_batch_check(pk_batch* B, void* stream) {
    if (!B) return fail(PK_ERR_INVALID_ARG, "batch is NULL");
    DeviceScope ds(B->pool->device);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    PK_CUDA(cudaStreamSynchronize(st));
    int word = 0;
    PK_CUDA(cudaMemcpy(&word, B->err.ptr, sizeof(int), cudaMemcpyDeviceToHost));
    if (word != 0) {
        PK_CUDA(cudaMemset(B->err.ptr, 0, sizeof(int)));
        if (B->plan_H >= 0 && !B->ctr_zero.empty())
            PK_CUDA(cudaMemset(B->plan.at<int>(22), 0, B->ctr_zero.size() * sizeof(int)));
        return fail(PK_ERR_TIMEOUT, "a bounded device wait timed out (error word %d)", word);
    }
    return PK_OK;
}

int pk_batch_stats(const pk_batch* B, int64_t* s) {
    if (!B || !s) return fail(PK_ERR_INVALID_ARG, "NULL pointer");
    s[7] = B->nwide;
    s[0] = B->nrows;
    s[1] = B->nu;
    s[2] = B->ncta;
    s[3] = B->total_blocks;
    s[4] = B->nsplit;
    s[5] = B->ngeneric;
    s[6] = B->launches;
    return PK_OK;
}

int pk_test_inject_launch_failure(void) {
    g_inject_launch_failure.store(1);
    return PK_OK;
}

int pk_batch_set_prefix_sharing(pk_batch* B, int mode) {
    if (!B) return fail(PK_ERR_INVALID_ARG, "batch is NULL");
    if (mode < 0 || mode > 2) return fail(PK_ERR_INVALID_ARG, "prefix sharing mode %d not in 0..2", mode);
    if (B->prefix_sharing != mode) {
        B->prefix_sharing = mode;
        B->plan_H = -1;
    }
    return PK_OK;
}

int pk_batch_prefix_stats(const pk_batch* B, int64_t* s) {
    if (!B || !s) return fail(PK_ERR_INVALID_ARG, "NULL pointer");
    s[0] = B->nprefix_groups;
    s[1] = B->nprefix;
    s[2] = B->prefix_keys;
    s[3] = B->prefix_token_keys;
    return PK_OK;
}

int pk_batch_profile(pk_batch* B, int enable) {
    if (!B) return fail(PK_ERR_INVALID_ARG, "batch is NULL");
    B->profiling = enable != 0;
    B->ev_used = 0;
    B->ev_kind.clear();
    return PK_OK;
}

int pk_batch_profile_read(pk_batch* B, double* ms5, int64_t* count5) {
    double* ms4 = ms5;
    int64_t* count4 = count5;
    if (!B || !ms4 || !count4) return fail(PK_ERR_INVALID_ARG, "NULL pointer");
    DeviceScope ds(B->pool->device);
    for (int k = 0; k < kProfKinds; ++k) {
        ms4[k] = 0.0;
        count4[k] = 0;
    }
    for (size_t i = 0; i < B->ev_kind.size(); ++i) {
        PK_CUDA(cudaEventSynchronize(B->ev_pool[2 * i + 1]));
        float ms = 0.f;
        PK_CUDA(cudaEventElapsedTime(&ms, B->ev_pool[2 * i], B->ev_pool[2 * i + 1]));
        ms4[B->ev_kind[i]] += ms;
        count4[B->ev_kind[i]] += 1;
    }
    B->ev_used = 0;
    B->ev_kind.clear();
    return PK_OK;
}

int pk_selftest_bounded_wait(int device, int64_t limit_ns, int* timed_out) {
    if (!timed_out || limit_ns <= 0 || limit_ns > 2000000000LL)
        return fail(PK_ERR_INVALID_ARG, "limit_ns must be in (0, 2e9]");
    DeviceScope ds(device);
    if (ds.err != cudaSuccess) return fail(PK_ERR_CUDA, "cudaSetDevice(%d)", device);
    int* word = nullptr;
    PK_CUDA(cudaMalloc(&word, sizeof(int)));
    cudaError_t e = cudaMemset(word, 0, sizeof(int));
    if (e == cudaSuccess) e = pk::launch_bounded_wait_selftest(word, static_cast<unsigned long long>(limit_ns), nullptr);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    int v = 0;
    if (e == cudaSuccess) e = cudaMemcpy(&v, word, sizeof(int), cudaMemcpyDeviceToHost);
    cudaFree(word);
    if (e != cudaSuccess) return fail(PK_ERR_CUDA, "bounded-wait self-test: %s", cudaGetErrorString(e));
    *timed_out = v == pk::kErrTimeout ? 1 : 0;
    return PK_OK;
}

int pk_gather_interleave(const float* src_dev, float* dst_dev, int world, int64_t rows, int64_t row_floats,
                         void* stream) {
    if (world <= 0 || rows < 0 || row_floats < 0) return fail(PK_ERR_INVALID_ARG, "bad sizes");
    if (rows == 0 || row_floats == 0) return PK_OK;
    if (!src_dev || !dst_dev) return fail(PK_ERR_INVALID_ARG, "NULL pointer");
    if (row_floats % 4 != 0) return fail(PK_ERR_INVALID_ARG, "row_floats %lld is not a multiple of 4", (long long)row_floats);
    int rc;
    if ((rc = check_aligned(src_dev, "src")) || (rc = check_aligned(dst_dev, "dst"))) return rc;
    PK_CUDA(pk::launch_interleave_heads(src_dev, dst_dev, world, rows, row_floats, static_cast<cudaStream_t>(stream)));
    return PK_OK;
}

int pk_plan_partition(const int64_t* unit_blocks, int64_t n_units, int max_ctas, int unit_switch_blocks,
                      int64_t* cta_first_block, int* ncta) {
    if (n_units < 0 || max_ctas <= 0 || unit_switch_blocks < 0 || !ncta || (n_units > 0 && !unit_blocks))
        return fail(PK_ERR_INVALID_ARG, "bad arguments");
    std::vector<int64_t> ub(static_cast<size_t>(n_units) + 1, 0);
    for (int64_t i = 0; i < n_units; ++i) {
        if (unit_blocks[i] <= 0) return fail(PK_ERR_INVALID_ARG, "unit %lld has no blocks", (long long)i);
        ub[i + 1] = ub[i] + unit_blocks[i];
        if (ub[i + 1] >= (int64_t(1) << 31)) return fail(PK_ERR_UNSUPPORTED, "too many blocks");
    }
    const int64_t n = split_kv_ctas(ub[n_units], n_units, max_ctas);
    std::vector<int32_t> first;
    *ncta = partition_blocks(ub.data(), n_units, n, unit_switch_blocks, first);
    if (cta_first_block)
        for (int c = 0; c <= *ncta; ++c) cta_first_block[c] = first[c];
    return PK_OK;
}

}  // extern "C"
