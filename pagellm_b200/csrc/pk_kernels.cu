// CUDA-core kernels of libpagekv: per-step row planning (positions + slot mapping),
// K/V append through the slot mapping, copy-on-write block copies, and the generic
// attention kernel used for float32 pools and for shapes the tensor-core kernel does not
// take.

#include <cuda_bf16.h>

#include <algorithm>

#include "pk_device.cuh"
#include "pk_internal.h"

namespace pk {

namespace {

// ------------------------------------------------------------------ rows of a step
// PagedBatch.__init__ (pagellm cache/paged.py:410-420): position and slot of every row.
__global__ void plan_rows_kernel(const int32_t* __restrict__ row_seq,
                                 const int32_t* __restrict__ offsets,
                                 const int32_t* __restrict__ starts,
                                 const int32_t* __restrict__ indptr,
                                 const int32_t* __restrict__ ids, int bs, int64_t nrows,
                                 int64_t* __restrict__ positions, int64_t* __restrict__ slots) {
    for (int64_t r = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; r < nrows;
         r += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int s = row_seq[r];
        const int64_t pos = static_cast<int64_t>(starts[s]) + (r - offsets[s]);
        const int64_t blk = pos / bs;
        positions[r] = pos;
        slots[r] = static_cast<int64_t>(ids[indptr[s] + blk]) * bs + (pos - blk * bs);
    }
}

// slot_mapping (cache/paged.py:303-306) over device arrays, with a range check.
__global__ void slot_mapping_kernel(const int32_t* __restrict__ table, int64_t table_len,
                                    const int64_t* __restrict__ positions, int64_t n, int bs,
                                    int64_t* __restrict__ slots, int32_t* err) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t pos = positions[i];
        const int64_t blk = pos >= 0 ? pos / bs : -1;
        if (blk < 0 || blk >= table_len) {
            slots[i] = -1;
            if (err) atomicExch(err, 1);
        } else {
            slots[i] = static_cast<int64_t>(table[blk]) * bs + (pos - blk * bs);
        }
    }
}

// ------------------------------------------------------------------ append
// pool_flat[layer, slots[r]] = rows[r] (cache/paged.py:443-444). One thread per 4 values.
__device__ __forceinline__ void store4(float* dst, float4 x) { *reinterpret_cast<float4*>(dst) = x; }
__device__ __forceinline__ void store4(__nv_bfloat16* dst, float4 x) {
    uint2 w;
    w.x = pack_bf16(x.x, x.y);
    w.y = pack_bf16(x.z, x.w);
    *reinterpret_cast<uint2*>(dst) = w;
}
__device__ __forceinline__ void store1(float* dst, float x) { *dst = x; }
__device__ __forceinline__ void store1(__nv_bfloat16* dst, float x) { *dst = __float2bfloat16_rn(x); }

// Where row r of the step goes: its slot from the per-row slots array, or resolved from the
// block table (position starts[s] + r - offsets[s] of its sequence s, paged.py:412-424), so
// that the append needs no separate per-row planning launch.
struct SlotsArray {
    const int64_t* slots;
    __device__ __forceinline__ int64_t operator()(int64_t r) const { return slots[r]; }
};
struct SlotsTable {
    const int32_t *row_seq, *offsets, *starts, *indptr, *ids;
    int bs;
    __device__ __forceinline__ int64_t operator()(int64_t r) const {
        const int s = row_seq[r];
        const int64_t pos = static_cast<int64_t>(starts[s]) + (r - offsets[s]);
        const int64_t blk = pos / bs;
        return static_cast<int64_t>(ids[indptr[s] + blk]) * bs + (pos - blk * bs);
    }
};

// rows == NULL: rows 0..n-1; otherwise only the listed rows (used when several rows of a
// step share a slot: the list then holds the last writer of each slot).
template <typename T, typename Slot>
__global__ void append_vec4_kernel(T* __restrict__ pk_, T* __restrict__ pv_,
                                   const float* __restrict__ k, const float* __restrict__ v,
                                   const Slot slot, const int32_t* __restrict__ rows,
                                   int64_t n, int rowlen) {
    const int per_row = rowlen / 4;
    const int64_t total = n * per_row;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t ri = i / per_row;
        const int c = static_cast<int>(i - ri * per_row) * 4;
        const int64_t r = rows ? rows[ri] : ri;
        const float4 kx = *reinterpret_cast<const float4*>(k + r * rowlen + c);
        const float4 vx = *reinterpret_cast<const float4*>(v + r * rowlen + c);
        const int64_t dst = slot(r) * rowlen + c;
        store4(pk_ + dst, kx);
        store4(pv_ + dst, vx);
    }
}

template <typename T, typename Slot>
__global__ void append_scalar_kernel(T* __restrict__ pk_, T* __restrict__ pv_,
                                     const float* __restrict__ k, const float* __restrict__ v,
                                     const Slot slot, const int32_t* __restrict__ rows,
                                     int64_t n, int rowlen) {
    const int64_t total = n * rowlen;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t ri = i / rowlen;
        const int c = static_cast<int>(i - ri * rowlen);
        const int64_t r = rows ? rows[ri] : ri;
        const int64_t dst = slot(r) * rowlen + c;
        store1(pk_ + dst, k[r * rowlen + c]);
        store1(pv_ + dst, v[r * rowlen + c]);
    }
}

// ------------------------------------------------------------------ copy-on-write
// k[:, dst] = k[:, src]; v[:, dst] = v[:, src] (cache/paged.py:294-296).
// grid = (pairs, layers, 2 tensors); W = widest word dividing the block size.
template <typename W>
__global__ void copy_blocks_kernel(uint8_t* __restrict__ k, uint8_t* __restrict__ v,
                                   const int64_t* __restrict__ pairs, int64_t layer_bytes,
                                   int64_t block_bytes) {
    const int64_t src = pairs[2 * blockIdx.x];
    const int64_t dst = pairs[2 * blockIdx.x + 1];
    uint8_t* base = (blockIdx.z == 0 ? k : v) + blockIdx.y * layer_bytes;
    const W* s = reinterpret_cast<const W*>(base + src * block_bytes);
    W* d = reinterpret_cast<W*>(base + dst * block_bytes);
    const int64_t words = block_bytes / static_cast<int64_t>(sizeof(W));
    for (int64_t i = threadIdx.x; i < words; i += blockDim.x) d[i] = s[i];
}

// ------------------------------------------------------------------ head-sharded output
// src [world][rows][S] (an all-gather of every rank's [rows][H/world][D] slice, S floats per
// row) -> dst [rows][world][S]: rank r's query heads land at [r*H/world, (r+1)*H/world).
// One thread per 16 bytes; consecutive threads walk one destination row, so both the reads
// (a run of S floats) and the writes are contiguous.
__global__ void interleave_heads_kernel(const float4* __restrict__ src, float4* __restrict__ dst,
                                        int world, int64_t rows, int64_t s4) {
    const int64_t total = static_cast<int64_t>(world) * rows * s4;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t row = i / (world * s4);
        const int64_t rem = i - row * world * s4;
        const int64_t r = rem / s4;
        const int64_t c = rem - r * s4;
        dst[i] = src[(r * rows + row) * s4 + c];
    }
}

// ------------------------------------------------------------------ host -> device gather
// Up to three page-locked host arrays (device-addressable: mapped pinned memory) copied into
// device buffers by one launch: each thread moves several independent 16-byte pieces, so many
// reads are in flight over the host link at once.
struct H2DPart {
    const float4* src;
    float4* dst;
    int64_t n;  // 16-byte pieces
};

__global__ void __launch_bounds__(256) h2d_gather_kernel(H2DPart a, H2DPart b, H2DPart c) {
    const int64_t total = a.n + b.n + c.n;
    constexpr int kPer = 4;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t i0 = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i0 < total; i0 += stride * kPer) {
        float4 v[kPer];
#pragma unroll
        for (int k = 0; k < kPer; ++k) {
            const int64_t i = i0 + k * stride;
            if (i < a.n) v[k] = a.src[i];
            else if (i < a.n + b.n) v[k] = b.src[i - a.n];
            else if (i < total) v[k] = c.src[i - a.n - b.n];
        }
#pragma unroll
        for (int k = 0; k < kPer; ++k) {
            const int64_t i = i0 + k * stride;
            if (i < a.n) a.dst[i] = v[k];
            else if (i < a.n + b.n) b.dst[i - a.n] = v[k];
            else if (i < total) c.dst[i - a.n - b.n] = v[k];
        }
    }
}

// ------------------------------------------------------------------ generic attention
// One CTA (4 warps) per (row, query head). Keys are dealt to warps one at a time; each
// warp keeps a running max / sum / output (the online softmax of cache/paged.py:309-352),
// and the four warps are merged at the end. Lanes hold DPL dims of the head each.
__device__ __forceinline__ float load_f(const float* p) { return *p; }
__device__ __forceinline__ float load_f(const __nv_bfloat16* p) { return __bfloat162float(*p); }

// x as the pool would hold it (bf16 pools round to nearest even).
__device__ __forceinline__ float as_pool(float x, const float*) { return x; }
__device__ __forceinline__ float as_pool(float x, const __nv_bfloat16*) { return __bfloat162float(__float2bfloat16_rn(x)); }

// Fused append for the CUDA-core kernels: the CTA of (row r, first query head of KV head kh)
// stores the step's row r (fp32 inputs) to its pool slot; other CTAs read new keys from the
// inputs, so nothing in the launch reads those slots.
template <typename T>
__device__ __forceinline__ void generic_store_new_row(const GenericParams& p, int r, int seq, int kh) {
    const int64_t pos = static_cast<int64_t>(p.starts[seq]) + (r - p.offsets[seq]);
    const int64_t blk = pos / p.bs;
    const int64_t slot = static_cast<int64_t>(p.ids[p.indptr[seq] + blk]) * p.bs + (pos - blk * p.bs);
    T* pk_ = const_cast<T*>(static_cast<const T*>(p.pool_k)) + (slot * p.kvh + kh) * p.D;
    T* pv_ = const_cast<T*>(static_cast<const T*>(p.pool_v)) + (slot * p.kvh + kh) * p.D;
    const float* kr = p.k_new + (static_cast<size_t>(r) * p.kvh + kh) * p.D;
    const float* vr = p.v_new + (static_cast<size_t>(r) * p.kvh + kh) * p.D;
    for (int d = threadIdx.x; d < p.D; d += blockDim.x) {
        store1(pk_ + d, kr[d]);
        store1(pv_ + d, vr[d]);
    }
}

template <typename T, int DPL>
__global__ void __launch_bounds__(128) generic_attn_kernel(const GenericParams p) {
    constexpr int NW = 4;
    __shared__ float sm_m[NW], sm_l[NW];
    extern __shared__ float sm_acc[];  // [NW][D]
    const int r = p.rows[blockIdx.x];
    const int head = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int seq = p.row_seq[r];
    const int pos = p.starts[seq] + (r - p.offsets[seq]);  // sees keys 0..pos
    const int g = p.H / p.kvh;
    const int kh = head / g;
    const T* kpool = static_cast<const T*>(p.pool_k);
    const T* vpool = static_cast<const T*>(p.pool_v);
    const int32_t* tbl = p.ids + p.indptr[seq];

    float qv[DPL], acc[DPL];
    const float* qp = p.q + (static_cast<size_t>(r) * p.H + head) * p.D;
#pragma unroll
    for (int i = 0; i < DPL; ++i) {
        const int d = lane + 32 * i;
        qv[i] = d < p.D ? qp[d] : 0.f;
        acc[i] = 0.f;
    }
    float m = -INFINITY, l = 0.f;
    for (int j = warp; j <= pos; j += NW) {
        // a row of this step (fused append): from the inputs, as the pool will hold it
        const bool fresh = p.k_new != nullptr && j >= p.starts[seq];
        const size_t src = fresh ? (static_cast<size_t>(p.offsets[seq] + j - p.starts[seq]) * p.kvh + kh) * p.D : 0;
        const int64_t slot = static_cast<int64_t>(tbl[j / p.bs]) * p.bs + (j % p.bs);
        const size_t off = (static_cast<size_t>(slot) * p.kvh + kh) * p.D;
        float dot = 0.f;
#pragma unroll
        for (int i = 0; i < DPL; ++i) {
            const int d = lane + 32 * i;
            if (d < p.D) dot = fmaf(qv[i], fresh ? as_pool(p.k_new[src + d], kpool) : load_f(kpool + off + d), dot);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
        const float s = dot * p.scale;
        const float mnew = fmaxf(m, s);
        const float corr = expf(m - mnew);
        const float w = expf(s - mnew);
        l = l * corr + w;
#pragma unroll
        for (int i = 0; i < DPL; ++i) {
            const int d = lane + 32 * i;
            const float vv = d < p.D ? (fresh ? as_pool(p.v_new[src + d], vpool) : load_f(vpool + off + d)) : 0.f;
            acc[i] = fmaf(w, vv, acc[i] * corr);
        }
        m = mnew;
    }
    if (lane == 0) {
        sm_m[warp] = m;
        sm_l[warp] = l;
    }
#pragma unroll
    for (int i = 0; i < DPL; ++i) {
        const int d = lane + 32 * i;
        if (d < p.D) sm_acc[warp * p.D + d] = acc[i];
    }
    if (p.k_new != nullptr && head % g == 0) generic_store_new_row<T>(p, r, seq, kh);
    __syncthreads();
    float mx = -INFINITY;
    for (int w = 0; w < NW; ++w) mx = fmaxf(mx, sm_m[w]);
    float den = 0.f;
    float wt[NW];
    for (int w = 0; w < NW; ++w) {
        wt[w] = sm_m[w] == -INFINITY ? 0.f : expf(sm_m[w] - mx);
        den += wt[w] * sm_l[w];
    }
    float* op = p.out + (static_cast<size_t>(r) * p.H + head) * p.D;
    for (int d = threadIdx.x; d < p.D; d += blockDim.x) {
        float num = 0.f;
        for (int w = 0; w < NW; ++w) num += wt[w] * sm_acc[w * p.D + d];
        op[d] = num / den;
    }
}

// Key-parallel variant for head_dim <= 32: lane = key. Each lane scores one key of a
// round of 32 per warp against the whole q row held in registers, the warp makes one
// online-softmax update per round, and the lanes' partial outputs are summed once at the
// end. At these head sizes generic_attn_kernel's one-key-per-warp loop is a chain of
// dependent loads per key; here a chain serves 32 keys.
// One key's row (head_dim <= 32) into registers; head_dim 32 rows (16-byte aligned: the row
// starts at a multiple of 32 elements) as vector loads, others element by element.
__device__ __forceinline__ void load_row32(const float* src, int D, float (&x)[32]) {
    if (D == 32) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float4 v = reinterpret_cast<const float4*>(src)[i];
            x[4 * i] = v.x;
            x[4 * i + 1] = v.y;
            x[4 * i + 2] = v.z;
            x[4 * i + 3] = v.w;
        }
    } else {
#pragma unroll
        for (int d = 0; d < 32; ++d) x[d] = d < D ? src[d] : 0.f;
    }
}
__device__ __forceinline__ void load_row32(const __nv_bfloat16* src, int D, float (&x)[32]) {
    if (D == 32) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint4 v = reinterpret_cast<const uint4*>(src)[i];
            const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                x[8 * i + 2 * k] = __uint_as_float(w[k] << 16);
                x[8 * i + 2 * k + 1] = __uint_as_float(w[k] & 0xFFFF0000u);
            }
        }
    } else {
#pragma unroll
        for (int d = 0; d < 32; ++d) x[d] = d < D ? __bfloat162float(src[d]) : 0.f;
    }
}

template <typename T>
__global__ void __launch_bounds__(128) generic_attn_small_kernel(const GenericParams p) {
    constexpr int NW = 4, DM = 32;
    __shared__ float sm_m[NW], sm_l[NW];
    __shared__ float sm_acc[NW][DM];
    const int r = p.rows[blockIdx.x];
    const int head = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int seq = p.row_seq[r];
    const int pos = p.starts[seq] + (r - p.offsets[seq]);  // sees keys 0..pos
    const int g = p.H / p.kvh;
    const int kh = head / g;
    const T* kpool = static_cast<const T*>(p.pool_k);
    const T* vpool = static_cast<const T*>(p.pool_v);
    const int32_t* tbl = p.ids + p.indptr[seq];
    const float* qp = p.q + (static_cast<size_t>(r) * p.H + head) * p.D;
    float qv[DM], acc[DM];
#pragma unroll
    for (int d = 0; d < DM; ++d) {
        qv[d] = d < p.D ? qp[d] : 0.f;
        acc[d] = 0.f;
    }
    float m = -INFINITY, l = 0.f;
    for (int j0 = warp * 32; j0 <= pos; j0 += NW * 32) {
        const int j = j0 + lane;
        const bool live = j <= pos;  // lane 0 always is: every round has a finite max
        size_t off = 0;
        if (live) {
            const int64_t slot = static_cast<int64_t>(tbl[j / p.bs]) * p.bs + (j % p.bs);
            off = (static_cast<size_t>(slot) * p.kvh + kh) * p.D;
        }
        float s = -INFINITY;
        float kv[DM], vv[DM];
        if (live && p.k_new != nullptr && j >= p.starts[seq]) {
            // a row of this step: from the inputs, as the pool will hold it
            const size_t src = (static_cast<size_t>(p.offsets[seq] + j - p.starts[seq]) * p.kvh + kh) * p.D;
            float dot = 0.f;
#pragma unroll
            for (int d = 0; d < DM; ++d) {
                kv[d] = d < p.D ? as_pool(p.k_new[src + d], kpool) : 0.f;
                vv[d] = d < p.D ? as_pool(p.v_new[src + d], vpool) : 0.f;
                dot = fmaf(qv[d], kv[d], dot);
            }
            s = dot * p.scale;
        } else if (live) {
            load_row32(kpool + off, p.D, kv);
            load_row32(vpool + off, p.D, vv);
            float dot = 0.f;
#pragma unroll
            for (int d = 0; d < DM; ++d) dot = fmaf(qv[d], kv[d], dot);
            s = dot * p.scale;
        } else {
#pragma unroll
            for (int d = 0; d < DM; ++d) vv[d] = 0.f;
        }
        float rmax = s;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) rmax = fmaxf(rmax, __shfl_xor_sync(0xffffffffu, rmax, o));
        const float mnew = fmaxf(m, rmax);
        const float corr = expf(m - mnew);
        const float w = live ? expf(s - mnew) : 0.f;
        float wsum = w;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) wsum += __shfl_xor_sync(0xffffffffu, wsum, o);
        l = l * corr + wsum;
#pragma unroll
        for (int d = 0; d < DM; ++d) acc[d] = fmaf(w, vv[d], acc[d] * corr);
        m = mnew;
    }
#pragma unroll
    for (int d = 0; d < DM; ++d) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc[d] += __shfl_xor_sync(0xffffffffu, acc[d], o);
        if (lane == d) sm_acc[warp][d] = acc[d];
    }
    if (lane == 0) {
        sm_m[warp] = m;
        sm_l[warp] = l;
    }
    if (p.k_new != nullptr && head % g == 0) generic_store_new_row<T>(p, r, seq, kh);
    __syncthreads();
    if (threadIdx.x < p.D) {
        float mx = -INFINITY;
        for (int w = 0; w < NW; ++w) mx = fmaxf(mx, sm_m[w]);
        float den = 0.f, num = 0.f;
        for (int w = 0; w < NW; ++w) {
            const float wt = sm_m[w] == -INFINITY ? 0.f : expf(sm_m[w] - mx);
            den += wt * sm_l[w];
            num += wt * sm_acc[w][threadIdx.x];
        }
        p.out[(static_cast<size_t>(r) * p.H + head) * p.D + threadIdx.x] = num / den;
    }
}

template <typename T>
cudaError_t launch_generic_t(const GenericParams& p, cudaStream_t st) {
    const int dpl = (p.D + 31) / 32;
    const dim3 grid(p.nrows, p.H);
    const size_t smem = 4 * p.D * sizeof(float);
    if (p.D <= 32) generic_attn_small_kernel<T><<<grid, 128, 0, st>>>(p);
    else if (dpl <= 1) generic_attn_kernel<T, 1><<<grid, 128, smem, st>>>(p);
    else if (dpl <= 2) generic_attn_kernel<T, 2><<<grid, 128, smem, st>>>(p);
    else if (dpl <= 4) generic_attn_kernel<T, 4><<<grid, 128, smem, st>>>(p);
    else if (dpl <= 8) generic_attn_kernel<T, 8><<<grid, 128, smem, st>>>(p);
    else if (dpl <= 16) generic_attn_kernel<T, 16><<<grid, 128, smem, st>>>(p);
    else return cudaErrorInvalidValue;
    return cudaGetLastError();
}

// Self-test of the bounded wait every pipeline uses: wait on an mbarrier phase that nothing
// completes; the wait must give up after limit_ns and report through the error word.
__global__ void bounded_wait_selftest_kernel(int* err, unsigned long long limit_ns) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    const bool done = mbar_wait_bounded(&bar, 0u, limit_ns);
    if (!done && threadIdx.x == 0) atomicExch(err, kErrTimeout);
}

int grid_for(int64_t work, int threads) {
    int64_t b = (work + threads - 1) / threads;
    if (b < 1) b = 1;
    if (b > 148 * 16) b = 148 * 16;
    return static_cast<int>(b);
}

}  // namespace

cudaError_t launch_plan_rows(const int32_t* row_seq, const int32_t* offsets, const int32_t* starts,
                             const int32_t* indptr, const int32_t* ids, int bs, int64_t nrows,
                             int64_t* positions, int64_t* slots, cudaStream_t st) {
    if (nrows <= 0) return cudaSuccess;
    plan_rows_kernel<<<grid_for(nrows, 256), 256, 0, st>>>(row_seq, offsets, starts, indptr, ids,
                                                           bs, nrows, positions, slots);
    return cudaGetLastError();
}

cudaError_t launch_slot_mapping(const int32_t* table, int64_t table_len, const int64_t* positions,
                                int64_t n, int bs, int64_t* slots, int32_t* err, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    slot_mapping_kernel<<<grid_for(n, 256), 256, 0, st>>>(table, table_len, positions, n, bs, slots,
                                                          err);
    return cudaGetLastError();
}

template <typename Slot>
cudaError_t launch_append_t(int dtype, void* pool_k_layer, void* pool_v_layer, const float* k, const float* v,
                            const Slot& slot, const int32_t* rows, int64_t n, int rowlen, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    // 4-wide path only when every row start is 16-byte aligned on both sides.
    const auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
    const bool vec = rowlen % 4 == 0 && a16(k) && a16(v) && a16(pool_k_layer) && a16(pool_v_layer);
    const int64_t work = vec ? n * (rowlen / 4) : n * rowlen;
    const int grid = grid_for(work, 256);
    if (dtype == 0) {
        float* pk_ = static_cast<float*>(pool_k_layer);
        float* pv_ = static_cast<float*>(pool_v_layer);
        if (vec) append_vec4_kernel<float, Slot><<<grid, 256, 0, st>>>(pk_, pv_, k, v, slot, rows, n, rowlen);
        else append_scalar_kernel<float, Slot><<<grid, 256, 0, st>>>(pk_, pv_, k, v, slot, rows, n, rowlen);
    } else {
        auto* pk_ = static_cast<__nv_bfloat16*>(pool_k_layer);
        auto* pv_ = static_cast<__nv_bfloat16*>(pool_v_layer);
        if (vec) append_vec4_kernel<__nv_bfloat16, Slot><<<grid, 256, 0, st>>>(pk_, pv_, k, v, slot, rows, n, rowlen);
        else append_scalar_kernel<__nv_bfloat16, Slot><<<grid, 256, 0, st>>>(pk_, pv_, k, v, slot, rows, n, rowlen);
    }
    return cudaGetLastError();
}

cudaError_t launch_append(int dtype, void* pool_k_layer, void* pool_v_layer, const float* k,
                          const float* v, const int64_t* slots, const int32_t* rows, int64_t n,
                          int rowlen, cudaStream_t st) {
    return launch_append_t(dtype, pool_k_layer, pool_v_layer, k, v, SlotsArray{slots}, rows, n, rowlen, st);
}

cudaError_t launch_append_table(int dtype, void* pool_k_layer, void* pool_v_layer, const float* k,
                                const float* v, const int32_t* row_seq, const int32_t* offsets,
                                const int32_t* starts, const int32_t* indptr, const int32_t* ids, int bs,
                                const int32_t* rows, int64_t n, int rowlen, cudaStream_t st) {
    return launch_append_t(dtype, pool_k_layer, pool_v_layer, k, v,
                           SlotsTable{row_seq, offsets, starts, indptr, ids, bs}, rows, n, rowlen, st);
}

cudaError_t launch_copy_blocks(void* k, void* v, const int64_t* pairs, int64_t npairs, int layers,
                               int64_t layer_bytes, int64_t block_bytes, cudaStream_t st) {
    if (npairs <= 0) return cudaSuccess;
    const dim3 grid(static_cast<unsigned>(npairs), layers, 2);
    auto* kb = static_cast<uint8_t*>(k);
    auto* vb = static_cast<uint8_t*>(v);
    if (block_bytes % 16 == 0)
        copy_blocks_kernel<uint4><<<grid, 256, 0, st>>>(kb, vb, pairs, layer_bytes, block_bytes);
    else if (block_bytes % 8 == 0)
        copy_blocks_kernel<uint2><<<grid, 256, 0, st>>>(kb, vb, pairs, layer_bytes, block_bytes);
    else if (block_bytes % 4 == 0)
        copy_blocks_kernel<uint32_t><<<grid, 256, 0, st>>>(kb, vb, pairs, layer_bytes, block_bytes);
    else
        copy_blocks_kernel<uint16_t><<<grid, 256, 0, st>>>(kb, vb, pairs, layer_bytes, block_bytes);
    return cudaGetLastError();
}

cudaError_t launch_interleave_heads(const float* src, float* dst, int world, int64_t rows, int64_t row_floats,
                                    cudaStream_t st) {
    const int64_t s4 = row_floats / 4;
    const int64_t total = static_cast<int64_t>(world) * rows * s4;
    if (total <= 0) return cudaSuccess;
    const int threads = 256;
    const int64_t blocks = std::min<int64_t>((total + threads - 1) / threads, 148 * 8);
    interleave_heads_kernel<<<static_cast<int>(blocks), threads, 0, st>>>(
        reinterpret_cast<const float4*>(src), reinterpret_cast<float4*>(dst), world, rows, s4);
    return cudaGetLastError();
}

cudaError_t launch_h2d_gather(const float* a_src, float* a_dst, int64_t a_floats, const float* b_src, float* b_dst,
                              int64_t b_floats, const float* c_src, float* c_dst, int64_t c_floats, cudaStream_t st) {
    H2DPart a{reinterpret_cast<const float4*>(a_src), reinterpret_cast<float4*>(a_dst), a_floats / 4};
    H2DPart b{reinterpret_cast<const float4*>(b_src), reinterpret_cast<float4*>(b_dst), b_floats / 4};
    H2DPart c{reinterpret_cast<const float4*>(c_src), reinterpret_cast<float4*>(c_dst), c_floats / 4};
    const int64_t total = a.n + b.n + c.n;
    if (total <= 0) return cudaSuccess;
    const int64_t blocks = std::min<int64_t>((total + 4 * 256 - 1) / (4 * 256), 148 * 4);
    h2d_gather_kernel<<<static_cast<int>(blocks), 256, 0, st>>>(a, b, c);
    return cudaGetLastError();
}

cudaError_t launch_bounded_wait_selftest(int* err, unsigned long long limit_ns, cudaStream_t st) {
    bounded_wait_selftest_kernel<<<1, 32, 0, st>>>(err, limit_ns);
    return cudaGetLastError();
}

cudaError_t launch_generic_attention(int dtype, const GenericParams& p, cudaStream_t st) {
    if (p.nrows <= 0) return cudaSuccess;
    return dtype == 0 ? launch_generic_t<float>(p, st) : launch_generic_t<__nv_bfloat16>(p, st);
}

}  // namespace pk
