// Decode attention that allocates nothing: the split-KV tensor-core attention of
// pk_attn_tc.cu, with every piece of scratch it needs (the step's block tables and plan,
// the per-CTA partial results of split sequences) held in one file-scope device array
// instead of memory from cudaMalloc.
//
// Who needs this: a caller that runs under an allocator it does not own - a serving
// framework that hands out every byte of HBM through its own caching allocator, or a
// plugin host that forbids cudaMalloc / cudaFree on the request path because cudaFree
// synchronises the whole device - can still call the fast decode kernel: it passes inputs
// and outputs only.
//
// Limits and sharing:
// * The array is kStaticScratchBytes (16 MiB) on every GPU that loads the library, held
//   until the process exits. A call whose plan does not fit is rejected with
//   PK_ERR_INVALID_ARG before anything is launched (at most kStaticMaxSeqs sequences).
// * Every call on a device uses the same array and leaves its contents behind. Calls whose
//   work overlaps on the GPU (two streams, or two host threads) race on the array.
// * A bounded device wait that gives up is reported through the caller's error word
//   (err_dev, required): the array holds no error state that a later call would have to
//   read back.
// * The first call on a device looks the array's device address up
//   (cudaGetSymbolAddress) with that device current and caches it; make that first call
//   before any stream capture.

#include <cstdarg>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "pagekv.h"
#include "pk_internal.h"

namespace {

constexpr size_t kStaticScratchBytes = size_t(16) << 20;
constexpr int kStaticMaxSeqs = 512;
constexpr int kMaxDevices = 64;

__device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

// Failing calls leave their message where pk_last_error() reads it.
int sfail(int code, const char* fmt, ...) {
    char buf[320];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    pk_set_last_error(buf);
    return code;
}

std::mutex g_addr_mu;
unsigned char* g_addr[kMaxDevices] = {};

// Device address of g_static_scratch on `device` (which must be current).
int scratch_address(int device, unsigned char** out) {
    if (device < 0 || device >= kMaxDevices) return sfail(PK_ERR_INVALID_ARG, "device %d out of range", device);
    std::lock_guard<std::mutex> lock(g_addr_mu);
    if (!g_addr[device]) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);
        if (e != cudaSuccess)
            return sfail(PK_ERR_CUDA, "cudaGetSymbolAddress(scratch) on device %d: %s", device,
                         cudaGetErrorString(e));
        g_addr[device] = static_cast<unsigned char*>(p);
    }
    *out = g_addr[device];
    return PK_OK;
}

size_t up256(size_t x) { return (x + 255) & ~size_t(255); }

int cta_of(int64_t j, int64_t T, int64_t n) {
    int64_t c = j * n / T;
    while (c + 1 < n && (c + 1) * T / n <= j) ++c;
    while (c > 0 && c * T / n > j) --c;
    return static_cast<int>(c);
}

}  // namespace

extern "C" PK_API int pk_decode_attend_static(const pk_pool* pool, int layer, int n_heads, int nseq,
                                              const int64_t* table_indptr, const int32_t* table_ids,
                                              const int64_t* ctx_lens, const float* q_dev,
                                              float* out_dev, int32_t* err_dev, void* stream) {
    pk::PoolView P;
    if (!pk_pool_view(pool, &P)) return sfail(PK_ERR_INVALID_ARG, "pool is NULL");
    if (!P.tc_ok) return sfail(PK_ERR_UNSUPPORTED, "the tensor-core kernel does not serve this pool");
    if (layer < 0 || layer >= P.n_layers) return sfail(PK_ERR_OUT_OF_RANGE, "layer %d", layer);
    if (n_heads <= 0 || n_heads % P.kvh != 0)
        return sfail(PK_ERR_INVALID_ARG, "n_heads=%d is not a positive multiple of %d", n_heads, P.kvh);
    const int g = n_heads / P.kvh;
    if (g > 8) return sfail(PK_ERR_UNSUPPORTED, "more than 8 query heads per KV head");
    if (nseq < 0 || nseq > kStaticMaxSeqs)
        return sfail(PK_ERR_INVALID_ARG, "nseq=%d outside [0, %d] (static scratch limit)", nseq, kStaticMaxSeqs);
    if (nseq == 0) return PK_OK;
    if (!table_indptr || !table_ids || !ctx_lens || !q_dev || !out_dev)
        return sfail(PK_ERR_INVALID_ARG, "NULL pointer");
    if (!err_dev) return sfail(PK_ERR_INVALID_ARG, "err_dev is NULL (a timed-out wait would go unreported)");
    if ((reinterpret_cast<uintptr_t>(q_dev) | reinterpret_cast<uintptr_t>(out_dev)) & 15u)
        return sfail(PK_ERR_INVALID_ARG, "q and out must be 16-byte aligned");
    {
        // its uploads read host memory of this call (the plan is on the stack), which a
        // captured graph would read again at replay, after it is gone
        cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
        if (cudaStreamIsCapturing(static_cast<cudaStream_t>(stream), &cs) != cudaSuccess)
            return sfail(PK_ERR_CUDA, "cudaStreamIsCapturing failed");
        if (cs != cudaStreamCaptureStatusNone)
            return sfail(PK_ERR_UNSUPPORTED, "pk_decode_attend_static cannot be captured into a CUDA graph");
    }
    const int bs = P.block_size;

    // Host-side plan in fixed-size stack arrays: one unit (= one decode row) per sequence.
    int32_t indptr[kStaticMaxSeqs + 1], starts[kStaticMaxSeqs], offsets[kStaticMaxSeqs + 1];
    int32_t useq[kStaticMaxSeqs], ut0[kStaticMaxSeqs], un[kStaticMaxSeqs], ublk[kStaticMaxSeqs + 1];
    int32_t su[kStaticMaxSeqs], sc0[kStaticMaxSeqs], sc1[kStaticMaxSeqs];
    if (table_indptr[0] != 0) return sfail(PK_ERR_INVALID_ARG, "table_indptr[0] != 0");
    const int64_t n_ids = table_indptr[nseq];
    if (n_ids < 0 || n_ids >= (int64_t(1) << 31)) return sfail(PK_ERR_INVALID_ARG, "bad table_indptr");
    int64_t T = 0;
    ublk[0] = 0;
    offsets[0] = 0;
    for (int i = 0; i < nseq; ++i) {
        const int64_t L = ctx_lens[i], tb = table_indptr[i], te = table_indptr[i + 1];
        if (L < 1 || L >= (int64_t(1) << 31)) return sfail(PK_ERR_INVALID_ARG, "seq %d: context length %lld", i, (long long)L);
        if (te < tb) return sfail(PK_ERR_INVALID_ARG, "table_indptr decreases at seq %d", i);
        const int64_t need = (L + bs - 1) / bs;
        if (need > te - tb)
            return sfail(PK_ERR_OUT_OF_RANGE, "seq %d: %lld tokens need %lld blocks, table has %lld", i,
                         (long long)L, (long long)need, (long long)(te - tb));
        for (int64_t j = tb; j < tb + need; ++j)
            if (table_ids[j] < 0 || table_ids[j] >= P.num_blocks)
                return sfail(PK_ERR_OUT_OF_RANGE, "seq %d: block id %d outside the pool", i, table_ids[j]);
        indptr[i] = static_cast<int32_t>(tb);
        starts[i] = static_cast<int32_t>(L - 1);
        offsets[i + 1] = i + 1;
        useq[i] = i;
        ut0[i] = 0;
        un[i] = 1;
        T += need;
        ublk[i + 1] = static_cast<int32_t>(T);
    }
    indptr[nseq] = static_cast<int32_t>(n_ids);
    if (T >= (int64_t(1) << 31)) return sfail(PK_ERR_UNSUPPORTED, "too many blocks");
    const int64_t nv = static_cast<int64_t>(P.num_sms) * (P.tc_virt > 1 ? P.tc_virt : 1);  // (virtual) CTAs
    const int ncta = static_cast<int>(T < nv ? T : nv);
    int nsplit = 0;
    for (int u = 0; u < nseq; ++u) {
        const int c0 = cta_of(ublk[u], T, ncta), c1 = cta_of(ublk[u + 1] - 1, T, ncta);
        if (c0 != c1) {
            su[nsplit] = u;
            sc0[nsplit] = c0;
            sc1[nsplit] = c1;
            ++nsplit;
        }
    }

    // Scratch layout (256-byte aligned pieces).
    const size_t segs = static_cast<size_t>(nseq) + ncta;
    const size_t o_part = 0;
    const size_t n_part_o = segs * P.kvh * pk::kMaxCols * P.d;
    const size_t o_ml = up256(o_part + n_part_o * sizeof(float));
    const size_t o_ids = up256(o_ml + segs * P.kvh * pk::kMaxCols * 2 * sizeof(float));
    const size_t o_meta = up256(o_ids + static_cast<size_t>(n_ids) * sizeof(int32_t));
    // meta = indptr | starts | offsets | useq | ut0 | un | ublk | su | sc0 | sc1
    int32_t pack[10 * (kStaticMaxSeqs + 1)];
    size_t m = 0;
    size_t off[10];
    const auto put = [&](const int32_t* a, size_t n) {
        std::memcpy(pack + m, a, n * sizeof(int32_t));
        const size_t at = m;
        m += n;
        return at;
    };
    off[0] = put(indptr, nseq + 1);
    off[1] = put(starts, nseq);
    off[2] = put(offsets, nseq + 1);
    off[3] = put(useq, nseq);
    off[4] = put(ut0, nseq);
    off[5] = put(un, nseq);
    off[6] = put(ublk, nseq + 1);
    off[7] = put(su, nsplit);
    off[8] = put(sc0, nsplit);
    off[9] = put(sc1, nsplit);
    const size_t total = o_meta + m * sizeof(int32_t);
    if (total > kStaticScratchBytes)
        return sfail(PK_ERR_INVALID_ARG,
                     "this step needs %zu bytes of scratch; the static scratch holds %zu "
                     "(fewer sequences, shorter tables or fewer KV heads fit)",
                     total, kStaticScratchBytes);

    int prev = -1;
    cudaGetDevice(&prev);
    if (prev != P.device && cudaSetDevice(P.device) != cudaSuccess)
        return sfail(PK_ERR_CUDA, "cudaSetDevice(%d) failed", P.device);
    struct Restore {
        int dev;
        ~Restore() {
            int cur = -1;
            cudaGetDevice(&cur);
            if (dev >= 0 && cur != dev) cudaSetDevice(dev);
        }
    } restore{prev};
    unsigned char* base = nullptr;
    int rc = scratch_address(P.device, &base);
    if (rc != PK_OK) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaMemcpyAsync(base + o_ids, table_ids, static_cast<size_t>(n_ids) * sizeof(int32_t),
                                    cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(base + o_meta, pack, m * sizeof(int32_t), cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess) return sfail(PK_ERR_CUDA, "scratch upload: %s", cudaGetErrorString(e));
    const int32_t* meta = reinterpret_cast<const int32_t*>(base + o_meta);

    pk::TcParams p{};
    p.q = q_dev;
    p.out = out_dev;
    p.part_o = reinterpret_cast<float*>(base + o_part);
    p.part_ml = reinterpret_cast<float*>(base + o_ml);
    p.err = reinterpret_cast<int*>(err_dev);
    p.indptr = meta + off[0];
    p.ids = reinterpret_cast<const int32_t*>(base + o_ids);
    p.starts = meta + off[1];
    p.offsets = meta + off[2];
    p.u_seq = meta + off[3];
    p.u_t0 = meta + off[4];
    p.u_n = meta + off[5];
    p.u_blk = meta + off[6];
    p.nu = nseq;
    p.total_blocks = static_cast<int>(T);
    p.ncta = ncta;
    p.kvh = P.kvh;
    p.g = g;
    p.H = n_heads;
    p.bs = bs;
    p.stages = P.tc_stages;
    p.virt = P.tc_virt;
    p.per_head_layout = P.tc_per_head;
    p.layer_slot0 = static_cast<int64_t>(layer) * P.num_blocks * bs;
    p.qscale = static_cast<float>(1.4426950408889634 / std::sqrt(static_cast<double>(P.d)));
    e = pk::launch_tc_attention(P.d, 1, P.tmk, P.tmv, p, P.tc_smem, st);
    if (e != cudaSuccess) return sfail(PK_ERR_CUDA, "attention launch: %s", cudaGetErrorString(e));
    if (nsplit > 0) {
        pk::MergeParams mp{};
        mp.out = out_dev;
        mp.part_o = p.part_o;
        mp.part_ml = p.part_ml;
        mp.offsets = p.offsets;
        mp.u_seq = p.u_seq;
        mp.u_t0 = p.u_t0;
        mp.u_n = p.u_n;
        mp.split_u = meta + off[7];
        mp.split_c0 = meta + off[8];
        mp.split_c1 = meta + off[9];
        mp.kvh = P.kvh;
        mp.g = g;
        mp.H = n_heads;
        mp.D = P.d;
        mp.nt = 1;
        e = pk::launch_merge(mp, nsplit, st);
        if (e != cudaSuccess) return sfail(PK_ERR_CUDA, "merge launch: %s", cudaGetErrorString(e));
    }
    return PK_OK;
}
