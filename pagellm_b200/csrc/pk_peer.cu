// Head-sharded output exchange over peer memory (NVLink / NVSwitch), one kernel per step.
//
// In the head-sharded layout every rank (one process per GPU) computes the attention output
// of its query heads [r*H/N, (r+1)*H/N) for all rows. Each rank owns one device allocation,
// exported by IPC handle and mapped by every peer: two result buffers [rows][H][D] (alternating
// by step, so a fast rank writing step s+1 never overwrites what a slow rank still reads of
// step s) and a flag word per sender. One launch per step:
//   * every thread stores 16-byte pieces of this rank's slice into every rank's current result
//     buffer, at this rank's head offset (plain peer stores, no multicast);
//   * each CTA counts itself done (acquire-release increment, system scope); the last CTA
//     writes the step's epoch into this rank's flag word in every rank's allocation (release,
//     system scope, one lane per destination), then waits until every rank's flag word here
//     holds the epoch (acquire, one lane per sender), for at most 1 s of %globaltimer - after
//     that it records a timeout in the error word and returns.
// When the launch completes, the local result buffer holds every rank's slice.

#include <algorithm>
#include <cstring>
#include <vector>

#include "pagekv.h"
#include "pk_device.cuh"
#include "pk_internal.h"

namespace {

constexpr int kMaxRanks = 64;
constexpr size_t kFlagBytes = 256;  // one uint32 per sender, then padding

struct PeerParams {
    const float4* src;               // [rows][s4] this rank's slice
    float4* dst[kMaxRanks];          // every rank's current result buffer [rows][world][s4]
    unsigned int* flag_of[kMaxRanks];  // every rank's flag words; this rank writes [rank]
    unsigned int* flags;             // this rank's flag words (read)
    unsigned int* done;              // CTA completion counter, zero between launches
    int* err;
    int64_t rows;
    int64_t s4;
    int world;
    int rank;
    unsigned int epoch;
};

__global__ void __launch_bounds__(256) peer_push_kernel(const PeerParams p) {
    const int64_t total = p.rows * p.s4;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t row = i / p.s4;
        const int64_t c = i - row * p.s4;
        const float4 v = p.src[i];
        const int64_t o = (row * p.world + p.rank) * p.s4 + c;
        // every rank starts with a different destination, so the senders spread over the
        // switch ports instead of all storing into the same peer first
        for (int k = 0; k < p.world; ++k) {
            int r = p.rank + k;
            if (r >= p.world) r -= p.world;
            p.dst[r][o] = v;
        }
    }
    __shared__ int last;
    __syncthreads();
    if (threadIdx.x == 0)  // this CTA's stores before its count (acquire-release, system scope)
        last = pk::atom_add_acq_rel_sys(p.done, 1u) == gridDim.x - 1;
    __syncthreads();
    if (!last || threadIdx.x >= 32) return;
    // The last CTA's first warp: every CTA's stores are ordered before its count, which this
    // CTA has acquired, so before the flags - one release store per destination, each on its
    // own lane.
    const int lane = threadIdx.x;
    if (lane == 0) *p.done = 0;
    __syncwarp();
    for (int r = lane; r < p.world; r += 32) pk::st_release_sys(p.flag_of[r] + p.rank, p.epoch);
    // Lane r watches sender r's flag word here; the warp leaves once all have the epoch, or
    // records a timeout after kWaitLimitNs.
    const unsigned long long t0 = pk::global_ns();
    for (int r0 = 0; r0 < p.world; r0 += 32) {
        const int r = r0 + lane;
        for (;;) {
            const bool arrived = r >= p.world || static_cast<int>(pk::ld_acquire_sys(p.flags + r) - p.epoch) >= 0;
            if (__all_sync(0xffffffffu, arrived)) break;
            if (pk::global_ns() - t0 > pk::kWaitLimitNs) {
                if (lane == 0) atomicExch(p.err, pk::kErrTimeout);
                return;
            }
        }
    }
}

int pfail(int code, const char* msg) {
    pk_set_last_error(msg);
    return code;
}

}  // namespace

struct pk_peer_gather {
    int device = 0, world = 0, rank = 0;
    int64_t bytes = 0;               // one result buffer
    char* base = nullptr;            // this rank's allocation: 2 buffers + flags
    std::vector<char*> peer_base;    // every rank's allocation as mapped here (own: base)
    unsigned int* done = nullptr;    // local CTA counter
    int* err = nullptr;              // local error word
    unsigned int epoch = 0;
    bool open = false;
};

int pk_peer_gather_step(pk_peer_gather* g, int64_t rows, int64_t row_floats, int d, pk::PeerOut* po,
                        float** result) {
    if (!g || !po || !result) return pfail(PK_ERR_INVALID_ARG, "NULL pointer");
    if (!g->open) return pfail(PK_ERR_INVALID_ARG, "peer gather not opened (pk_peer_gather_open)");
    if (g->world > pk::kMaxOutPeers) return pfail(PK_ERR_UNSUPPORTED, "fused exchange: at most 8 ranks");
    if (rows < 0 || d <= 0 || row_floats <= 0 || row_floats % d)
        return pfail(PK_ERR_INVALID_ARG, "rows >= 0 and row_floats a positive multiple of d");
    if (rows * row_floats * g->world * 4 > g->bytes)
        return pfail(PK_ERR_INVALID_ARG, "result larger than the peer gather's buffers");
    const unsigned int epoch = ++g->epoch;
    const int64_t buf = (epoch & 1u) * g->bytes;
    *po = pk::PeerOut{};
    po->n = g->world;
    po->out_H = static_cast<int>(row_floats / d) * g->world;
    po->rank = g->rank;
    po->epoch = epoch;
    for (int r = 0; r < g->world; ++r) {
        po->out[r] = reinterpret_cast<float*>(g->peer_base[r] + buf) + g->rank * row_floats;
        po->flag_of[r] = reinterpret_cast<unsigned int*>(g->peer_base[r] + 2 * g->bytes);
    }
    po->flags = reinterpret_cast<unsigned int*>(g->base + 2 * g->bytes);
    po->done = g->done;
    po->err = g->err;
    *result = reinterpret_cast<float*>(g->base + buf);
    return PK_OK;
}

extern "C" {

PK_API int pk_peer_gather_create(int device, int world, int rank, int64_t bytes, pk_peer_gather** out) {
    if (!out) return pfail(PK_ERR_INVALID_ARG, "out is NULL");
    *out = nullptr;
    if (world < 1 || world > kMaxRanks || rank < 0 || rank >= world || bytes <= 0 || bytes % 16)
        return pfail(PK_ERR_INVALID_ARG, "peer gather: world in 1..64, rank < world, bytes > 0 and a multiple of 16");
    int prev = -1;
    cudaGetDevice(&prev);
    if (cudaSetDevice(device) != cudaSuccess) return pfail(PK_ERR_CUDA, "cudaSetDevice failed");
    auto* g = new pk_peer_gather();
    g->device = device;
    g->world = world;
    g->rank = rank;
    g->bytes = bytes;
    cudaError_t e = cudaMalloc(&g->base, 2 * static_cast<size_t>(bytes) + kFlagBytes);
    if (e == cudaSuccess) e = cudaMemset(g->base + 2 * bytes, 0, kFlagBytes);
    if (e == cudaSuccess) e = cudaMalloc(&g->done, sizeof(unsigned int) + sizeof(int));
    if (e == cudaSuccess) e = cudaMemset(g->done, 0, sizeof(unsigned int) + sizeof(int));
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (prev >= 0) cudaSetDevice(prev);
    if (e != cudaSuccess) {
        if (g->base) cudaFree(g->base);
        if (g->done) cudaFree(g->done);
        delete g;
        return pfail(PK_ERR_CUDA, "peer gather: device allocation failed");
    }
    g->err = reinterpret_cast<int*>(g->done + 1);
    *out = g;
    return PK_OK;
}

PK_API int pk_peer_gather_handle(const pk_peer_gather* g, uint8_t* handle64) {
    if (!g || !handle64) return pfail(PK_ERR_INVALID_ARG, "NULL pointer");
    static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(g->device);
    cudaIpcMemHandle_t h;
    const cudaError_t e = cudaIpcGetMemHandle(&h, g->base);
    if (prev >= 0) cudaSetDevice(prev);
    if (e != cudaSuccess) return pfail(PK_ERR_CUDA, "cudaIpcGetMemHandle failed");
    std::memcpy(handle64, &h, 64);
    return PK_OK;
}

PK_API int pk_peer_gather_open(pk_peer_gather* g, const uint8_t* handles) {
    if (!g || !handles) return pfail(PK_ERR_INVALID_ARG, "NULL pointer");
    if (g->open) return pfail(PK_ERR_INVALID_ARG, "peer gather already opened");
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(g->device);
    g->peer_base.assign(g->world, nullptr);
    int rc = PK_OK;
    for (int r = 0; r < g->world; ++r) {
        if (r == g->rank) {
            g->peer_base[r] = g->base;
            continue;
        }
        cudaIpcMemHandle_t h;
        std::memcpy(&h, handles + 64 * r, 64);
        void* p = nullptr;
        if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            rc = pfail(PK_ERR_CUDA, "cudaIpcOpenMemHandle failed (no peer access between these GPUs?)");
            break;
        }
        g->peer_base[r] = static_cast<char*>(p);
    }
    if (rc != PK_OK) {
        for (int r = 0; r < g->world; ++r)
            if (r != g->rank && g->peer_base[r]) cudaIpcCloseMemHandle(g->peer_base[r]);
        g->peer_base.clear();
    } else {
        g->open = true;
    }
    if (prev >= 0) cudaSetDevice(prev);
    return rc;
}

PK_API int pk_peer_gather_heads(pk_peer_gather* g, const float* slice_dev, int64_t rows, int64_t row_floats,
                                float** result_dev, void* stream) {
    if (!g || !result_dev) return pfail(PK_ERR_INVALID_ARG, "NULL pointer");
    if (!g->open) return pfail(PK_ERR_INVALID_ARG, "peer gather not opened (pk_peer_gather_open)");
    if (rows < 0 || row_floats <= 0 || row_floats % 4)
        return pfail(PK_ERR_INVALID_ARG, "rows >= 0 and row_floats a positive multiple of 4");
    if (rows * row_floats * g->world * 4 > g->bytes)
        return pfail(PK_ERR_INVALID_ARG, "result larger than the peer gather's buffers");
    if (rows > 0 && (!slice_dev || reinterpret_cast<uintptr_t>(slice_dev) % 16))
        return pfail(PK_ERR_INVALID_ARG, "slice must be a 16-byte aligned device pointer");
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(g->device);
    const unsigned int epoch = ++g->epoch;
    const int64_t buf = (epoch & 1u) * g->bytes;
    PeerParams p{};
    p.src = reinterpret_cast<const float4*>(slice_dev);
    for (int r = 0; r < g->world; ++r) {
        p.dst[r] = reinterpret_cast<float4*>(g->peer_base[r] + buf);
        p.flag_of[r] = reinterpret_cast<unsigned int*>(g->peer_base[r] + 2 * g->bytes);
    }
    p.flags = reinterpret_cast<unsigned int*>(g->base + 2 * g->bytes);
    p.done = g->done;
    p.err = g->err;
    p.rows = rows;
    p.s4 = row_floats / 4;
    p.world = g->world;
    p.rank = g->rank;
    p.epoch = epoch;
    const int64_t total = rows * p.s4;
    const int blocks = static_cast<int>(std::min<int64_t>(std::max<int64_t>((total + 255) / 256, 1), 148 * 4));
    peer_push_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(p);
    const cudaError_t e = cudaGetLastError();
    if (prev >= 0) cudaSetDevice(prev);
    if (e != cudaSuccess) return pfail(PK_ERR_CUDA, "peer push launch failed");
    *result_dev = reinterpret_cast<float*>(g->base + buf);
    return PK_OK;
}

PK_API int pk_peer_gather_check(pk_peer_gather* g, void* stream) {
    if (!g) return pfail(PK_ERR_INVALID_ARG, "NULL pointer");
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(g->device);
    int word = 0;
    cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
    if (e == cudaSuccess) e = cudaMemcpy(&word, g->err, sizeof(int), cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && word) e = cudaMemset(g->err, 0, sizeof(int));
    if (prev >= 0) cudaSetDevice(prev);
    if (e != cudaSuccess) return pfail(PK_ERR_CUDA, "peer gather check failed");
    return word ? pfail(PK_ERR_TIMEOUT, "a peer did not signal its slice within the wait limit") : PK_OK;
}

PK_API int pk_peer_gather_destroy(pk_peer_gather* g) {
    if (!g) return PK_OK;
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(g->device);
    cudaDeviceSynchronize();
    for (int r = 0; r < static_cast<int>(g->peer_base.size()); ++r)
        if (r != g->rank && g->peer_base[r]) cudaIpcCloseMemHandle(g->peer_base[r]);
    if (g->base) cudaFree(g->base);
    if (g->done) cudaFree(g->done);
    if (prev >= 0) cudaSetDevice(prev);
    delete g;
    return PK_OK;
}

}  // extern "C"
