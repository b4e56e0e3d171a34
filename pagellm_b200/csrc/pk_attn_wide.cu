// Causal chunked-prefill / speculative-verify attention over the paged cache on the
// 5th-generation tensor cores (tcgen05 + TMEM), bf16 pools, head_dim 128.
//
// Semantics: pagellm cache/paged.py:454-463 -> model/transformer.py:116-146: the query at
// absolute position p sees keys 0..p of its sequence, keys read through the block table.
//
// Work: a work item is one query tile, up to 128/g query tokens read through one block
// table; rows are (token, head-in-group) pairs, row r = t*g + j, so the g heads of a token
// share every K/V tile. Items come in pairs that read the same block table, so every K/V
// tile brought into shared memory serves 256 query rows (half the L2 -> SM traffic of one
// tile per CTA, which is what bounded that design). Keys 0..kend-1 of a pair stream in tiles
// of 128 (128/bs blocks). Two kinds of item:
//   chunk   consecutive tokens of one sequence (a prefill chunk or a wide verify window);
//           causal by absolute position.
//   prefix  tokens of several sequences whose block tables begin with the same blocks
//           (forks / prefix-cache hits); kend = the shared blocks' keys, all before every
//           token's position. Each such K/V tile is read once per 256 rows instead of once
//           per sequence; the partial is merged into the row that the split-KV kernel wrote
//           for the rest of the sequence (cascade attention).
// Schedule: each CTA walks a list of segments = key-tile ranges of (item pair, KV head).
// For chunk items a segment is a whole pair-head; shared-prefix work is cut stream-K style:
// the launch's (pair-head, key tile) space is split into equal shares, one per CTA (at most
// one wave), and a pair-head cut between CTAs leaves a partial (un-normalised O, max, sum)
// per CTA that the last CTA to finish it merges in slot order (per pair-head counters,
// left at zero).
//
// Warp roles (320 threads):
//   warp 0  producer: one lane fills a 3-slot K ring and a 2-slot V ring with TMA loads (no
//           multicast), one copy per (block, 64-dim chunk); mbarrier completion.
//   warp 1  TMEM owner (alloc/dealloc, 512 columns) and, on one lane, the MMA issuer:
//           S_t = Q_t . K^T  (M=128, N=128, K=128; bf16 -> fp32 in TMEM)
//           O_t += P_t . V   (M=128, N=128, K=128; P_t from TMEM, V MN-major from smem)
//   warps 2-5 / 6-9  softmax of query tile 0 / 1: thread = row. Loads all 128 scores of S_t
//           from TMEM with one wait (a few registers spill; re-reading S in 32-column passes
//           to avoid that serialises four TMEM round trips per pass and measured slower),
//           masks by absolute position, online max/sum in the exp2 domain (the base moves only
//           when a tile's max exceeds it by 2^8, and only then is O_t in TMEM rescaled),
//           writes P_t (bf16) over S_t's first 64 columns, and finally O_t / l to global.
// Q is rounded to bf16 once (scaled by log2(e)/sqrt(d)); P to bf16; accumulation is fp32.
// Every wait is bounded; on a timeout the CTA records the error, unwinds and frees TMEM.

#include "pk_device.cuh"
#include "pk_internal.h"

namespace pk {

namespace {

constexpr int kWRows = 128;        // query rows per tile (UMMA M); two tiles per CTA
constexpr int kWKeys = kWideKeys;  // keys per tile (UMMA N of S, K of P.V)
constexpr int kWD = 128;           // head dim
constexpr int kKStages = 3;        // K ring: a slot frees when S of both query tiles completes
constexpr int kVStages = 2;        // V ring: a slot frees when P.V of both query tiles completes
constexpr int kWThreads = 320;
constexpr uint32_t kTmemCols = 512;
// TMEM columns: S_0 [0,128), S_1 [128,256) (P_t written over the first 64 columns of S_t),
// O_0 [256,384), O_1 [384,512).
constexpr uint32_t kColO = 2 * kWKeys;
static_assert(kColO + 2 * kWD <= kTmemCols, "TMEM budget");
static_assert(kWideQTileBytes == kWRows * kWD * 2, "packed query tile size");

// shared memory carve-up (bytes from a 1024-aligned base)
constexpr int kQBytes = kWRows * kWD * 2;   // 32 KB per query tile (bf16): [chunk][row][64]
constexpr int kKVBytes = kWKeys * kWD * 2;  // 32 KB per K or V tile: [chunk][key][64]
constexpr int kOffQ = 0;
constexpr int kOffK = kOffQ + 2 * kQBytes;
constexpr int kOffV = kOffK + kKStages * kKVBytes;
constexpr int kOffBar = kOffV + kVStages * kKVBytes;
constexpr int kSmemBytes = kOffBar + 256 + 1024;

// ---------------------------------------------------------------- tcgen05 wrappers
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                 "r"(ncols));
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// A operand from TMEM (rows = lanes, K packed two bf16 per 32-bit column).
__device__ __forceinline__ void umma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
          "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
          "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
          "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float* v) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]), "f"(v[8]),
        "f"(v[9]), "f"(v[10]), "f"(v[11]), "f"(v[12]), "f"(v[13]), "f"(v[14]), "f"(v[15]), "f"(v[16]),
        "f"(v[17]), "f"(v[18]), "f"(v[19]), "f"(v[20]), "f"(v[21]), "f"(v[22]), "f"(v[23]), "f"(v[24]),
        "f"(v[25]), "f"(v[26]), "f"(v[27]), "f"(v[28]), "f"(v[29]), "f"(v[30]), "f"(v[31])
        : "memory");
}
__device__ __forceinline__ void tmem_st32u(uint32_t taddr, const uint32_t* v) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
        "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]),
        "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]),
        "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
        : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 2^x on the special-function unit (approximate, flush-to-zero; 2^-inf = 0).
__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Shared-memory matrix descriptor, 128-byte swizzle (sm_100 format: version 1).
// lbo / sbo in bytes (multiples of 16).
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((addr >> 4) & 0x3FFF);
    d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFF) << 16;
    d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFF) << 32;
    d |= static_cast<uint64_t>(1) << 46;  // version
    d |= static_cast<uint64_t>(2) << 61;  // SWIZZLE_128B
    return d;
}

// Instruction descriptor, kind::f16: bf16 x bf16 -> fp32, M = 128.
__host__ __device__ constexpr uint32_t idesc_bf16(int n, bool b_mn_major) {
    return (1u << 4)                  // D format f32
           | (1u << 7)                // A bf16
           | (1u << 10)               // B bf16
           | (0u << 15)               // A K-major
           | ((b_mn_major ? 1u : 0u) << 16)
           | (static_cast<uint32_t>(n >> 3) << 17)
           | (static_cast<uint32_t>(kWRows >> 4) << 24);
}

constexpr uint32_t kIdescS = idesc_bf16(kWKeys, false);
constexpr uint32_t kIdescO = idesc_bf16(kWD, true);

// Offset of 16-byte unit u of row r in a [rows][128 B] tile with the 128-byte swizzle.
__device__ __forceinline__ uint32_t sw128(int r, int u) {
    return static_cast<uint32_t>(r * 128 + ((u ^ (r & 7)) << 4));
}

// Per-CTA segment list: a segment is key tiles [t0, t1) of one (item pair, KV head).
struct Seg {
    int pair, head, t0, t1, slot, ph;  // slot < 0: the segment covers the whole pair-head
};
__device__ __forceinline__ Seg load_seg(const int32_t* s, int i) {
    const int32_t* e = s + 6 * i;
    return Seg{e[0], e[1], e[2], e[3], e[4], e[5]};
}

__global__ void __launch_bounds__(kWThreads, 1)
    wide_attn_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                     const WideParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~uintptr_t(1023));
    uint64_t* kfull = reinterpret_cast<uint64_t*>(smem + kOffBar);
    uint64_t* kempty = kfull + kKStages;
    uint64_t* vfull = kempty + kKStages;
    uint64_t* vempty = vfull + kVStages;
    uint64_t* sfull = vempty + kVStages;  // [tile]
    uint64_t* pfull = sfull + 2;          // [tile], one arrival per softmax warp
    uint64_t* pvdone = pfull + 2;         // [tile]
    uint64_t* qfull = pvdone + 2;         // [tile], Q of the next segment in shared memory (bulk copy)
    uint64_t* ofree = qfull + 2;          // [tile], O of the last segment read out of TMEM
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ofree + 2);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int g = p.g;
    const int s_begin = p.cta_seg[blockIdx.x], s_end = p.cta_seg[blockIdx.x + 1];

    if (threadIdx.x == 0) {
        for (int s = 0; s < kKStages; ++s) {
            mbar_init(&kfull[s], 1);
            mbar_init(&kempty[s], 1);
        }
        for (int s = 0; s < kVStages; ++s) {
            mbar_init(&vfull[s], 1);
            mbar_init(&vempty[s], 1);
        }
        for (int t = 0; t < 2; ++t) {
            mbar_init(&sfull[t], 1);
            mbar_init(&pfull[t], 4);
            mbar_init(&pvdone[t], 1);
            mbar_init(&qfull[t], 1);
            mbar_init(&ofree[t], 4);
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t smem_base = smem_u32(smem);

    if (warp == 0) {
        // ------------------------------------------------------------ producer
        // One lane fills both rings over the CTA's segments in order, polling without
        // blocking: K tile n as soon as its slot is free (S of both query tiles done with the
        // slot's previous tile), V tile n once K tile n is issued and its slot is free.
        if (lane == 0) {
            prefetch_tensormap(&tmk);
            prefetch_tensormap(&tmv);
            const int per_tile = kWKeys / p.bs;
            // cursors: segment, tile within the pair's key tiles, running tile count
            int ks = s_begin, vs = s_begin, nk = 0, nv = 0;
            Seg sk = ks < s_end ? load_seg(p.seg, ks) : Seg{}, sv = sk;
            int kt = sk.t0, vt = sv.t0;
            auto issue = [&](const CUtensorMap* map, uint8_t* dst, uint64_t* bar, const Seg& sg, int jt) {
                const int i0 = p.w_pair[2 * sg.pair];
                const int32_t* tbl = p.ids + p.indptr[p.w_seq[i0]];
                const int kv_end = p.pair_kend[sg.pair];
                const int nblk = (kv_end + p.bs - 1) / p.bs;
                // the tile's block ids first, as independent loads: one load latency per tile
                int idv[kWKeys / 16];
#pragma unroll
                for (int b = 0; b < kWKeys / 16; ++b)
                    if (b < per_tile) idv[b] = __ldg(tbl + min(jt * per_tile + b, nblk - 1));  // past the end: valid, masked
                mbar_arrive_expect_tx(bar, kKVBytes);
#pragma unroll
                for (int b = 0; b < kWKeys / 16; ++b) {
                    if (b >= per_tile) break;
                    const int slot0 = static_cast<int>(p.layer_slot0 + static_cast<int64_t>(idv[b]) * p.bs);
                    for (int c = 0; c < 2; ++c)
                        tma_load_4d(dst + c * (kWKeys * 128) + b * p.bs * 128, map, 0, slot0, sg.head, c, bar);
                }
            };
            // Q tiles of segment k: one bulk copy per query tile from the packed tiles, issued
            // once the epilogue of segment k-1 has left that buffer (ofree of both tiles)
            auto issue_q = [&](int k) {
                const Seg sg = load_seg(p.seg, s_begin + k);
#pragma unroll
                for (int t = 0; t < 2; ++t) {
                    const int item = p.w_pair[2 * sg.pair + t];
                    const int qt = item >= 0 ? item * p.kvh + sg.head : p.q_zero_tile;
                    mbar_arrive_expect_tx(&qfull[t], kQBytes);
                    bulk_load(smem + kOffQ + t * kQBytes, p.qpk + static_cast<size_t>(qt) * kQBytes, kQBytes, &qfull[t]);
                }
            };
            int nq = 0;  // segments whose Q has been issued
            if (s_begin < s_end) {
                issue_q(0);
                nq = 1;
            }
            unsigned long long idle_since = global_ns();
            while (vs < s_end || s_begin + nq < s_end) {
                bool progressed = false;
                if (s_begin + nq < s_end && mbar_test_wait(&ofree[0], static_cast<uint32_t>((nq - 1) & 1)) &&
                    mbar_test_wait(&ofree[1], static_cast<uint32_t>((nq - 1) & 1))) {
                    issue_q(nq);
                    ++nq;
                    progressed = true;
                }
                if (ks < s_end && mbar_test_wait(&kempty[nk % kKStages], ((nk / kKStages) & 1u) ^ 1u)) {
                    issue(&tmk, smem + kOffK + (nk % kKStages) * kKVBytes, &kfull[nk % kKStages], sk, kt);
                    ++nk;
                    if (++kt == sk.t1 && ++ks < s_end) {
                        sk = load_seg(p.seg, ks);
                        kt = sk.t0;
                    }
                    progressed = true;
                }
                if (nv < nk && mbar_test_wait(&vempty[nv % kVStages], ((nv / kVStages) & 1u) ^ 1u)) {
                    issue(&tmv, smem + kOffV + (nv % kVStages) * kKVBytes, &vfull[nv % kVStages], sv, vt);
                    ++nv;
                    if (++vt == sv.t1 && ++vs < s_end) {
                        sv = load_seg(p.seg, vs);
                        vt = sv.t0;
                    }
                    progressed = true;
                }
                if (progressed) {
                    idle_since = global_ns();
                } else if (*abort_flag || global_ns() - idle_since > kWaitLimitNs) {
                    *abort_flag = 1;
                    atomicExch(p.err, kErrTimeout);
                    break;
                }
            }
            // never leave the CTA with copies still landing in its shared memory
            if (nq > 0)
                for (int t = 0; t < 2; ++t) mbar_wait_bounded(&qfull[t], static_cast<uint32_t>((nq - 1) & 1));
            for (int t = max(0, nk - kKStages); t < nk; ++t)
                mbar_wait_bounded(&kfull[t % kKStages], static_cast<uint32_t>(t / kKStages) & 1u);
            for (int t = max(0, nv - kVStages); t < nv; ++t)
                mbar_wait_bounded(&vfull[t % kVStages], static_cast<uint32_t>(t / kVStages) & 1u);
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        // Per segment, after S_0(first), S_1(first), for each key tile j:
        // P_0.V(j), S_0(j+1), P_1.V(j), S_1(j+1). Each query tile's S(j+1) overwrites its P(j)
        // in TMEM, so it is issued right after that tile's P.V(j) (tcgen05 MMAs of one thread
        // execute in issue order); softmax of one tile overlaps the other tile's MMAs. A
        // segment's first S_t waits for its Q_t in shared memory, its first P_t.V for the
        // previous segment's O_t to have been read out.
        if (lane == 0) {
            uint64_t qd[2][kWD / 16];
#pragma unroll
            for (int t = 0; t < 2; ++t)
#pragma unroll
                for (int kk = 0; kk < kWD / 16; ++kk)
                    qd[t][kk] = smem_desc(smem_base + kOffQ + t * kQBytes + (kk >> 2) * (kWRows * 128) + (kk & 3) * 32,
                                          16, 1024);
            const uint64_t kd0 = smem_desc(smem_base + kOffK, 16, 1024);
            const uint64_t vd0 = smem_desc(smem_base + kOffV, kWKeys * 128, 1024);
            bool ok = true;
            auto wait = [&](uint64_t* bar, uint32_t parity) {
                if (ok && (!mbar_wait_bounded(bar, parity) || *abort_flag)) ok = false;
                return ok;
            };
            auto issue_s = [&](int t, int n) {  // n: the CTA's running key-tile count
                const uint32_t kb = static_cast<uint32_t>((n % kKStages) * kKVBytes);
#pragma unroll
                for (int kk = 0; kk < kWD / 16; ++kk) {
                    // A = Q_t [128 rows][128 dims] K-major, B = K [128 keys][128 dims] K-major
                    const uint64_t bd = kd0 + ((kb + (kk >> 2) * (kWKeys * 128) + (kk & 3) * 32) >> 4);
                    umma_bf16(tmem + t * kWKeys, qd[t][kk], bd, kIdescS, kk > 0 ? 1u : 0u);
                }
                umma_commit(&sfull[t]);
            };
            auto issue_pv = [&](int t, int n, bool first) {
                const uint32_t vb = static_cast<uint32_t>((n % kVStages) * kKVBytes);
#pragma unroll
                for (int kk = 0; kk < kWKeys / 16; ++kk) {
                    // A = P_t in TMEM (16 keys = 8 columns per step); B = V [key][128 dims] MN-major
                    const uint64_t bd = vd0 + ((vb + kk * 16 * 128) >> 4);
                    umma_bf16_ts(tmem + kColO + t * kWD, tmem + t * kWKeys + kk * 8, bd, kIdescO,
                                 (!first || kk > 0) ? 1u : 0u);
                }
                umma_commit(&pvdone[t]);
            };
            int n = 0;  // running key-tile count (ring and barrier phases)
            for (int si = s_begin; si < s_end && ok; ++si) {
                const Seg sg = load_seg(p.seg, si);
                const int k = si - s_begin;  // segment count (qfull / ofree phases)
                const int nt = sg.t1 - sg.t0;
                if (!wait(&kfull[n % kKStages], static_cast<uint32_t>(n / kKStages) & 1u)) break;
                if (!wait(&qfull[0], static_cast<uint32_t>(k & 1))) break;
                tc_fence_after();
                issue_s(0, n);
                if (!wait(&qfull[1], static_cast<uint32_t>(k & 1))) break;
                tc_fence_after();
                issue_s(1, n);
                umma_commit(&kempty[n % kKStages]);
                for (int j = 0; j < nt && ok; ++j, ++n) {
                    const bool more = j + 1 < nt;
                    if (!wait(&vfull[n % kVStages], static_cast<uint32_t>(n / kVStages) & 1u)) break;
                    if (!wait(&pfull[0], static_cast<uint32_t>(n & 1))) break;
                    if (j == 0 && k > 0 && !wait(&ofree[0], static_cast<uint32_t>((k - 1) & 1))) break;
                    tc_fence_after();
                    issue_pv(0, n, j == 0);
                    if (more) {
                        if (!wait(&kfull[(n + 1) % kKStages], static_cast<uint32_t>((n + 1) / kKStages) & 1u)) break;
                        tc_fence_after();
                        issue_s(0, n + 1);
                    }
                    if (!wait(&pfull[1], static_cast<uint32_t>(n & 1))) break;
                    if (j == 0 && k > 0 && !wait(&ofree[1], static_cast<uint32_t>((k - 1) & 1))) break;
                    tc_fence_after();
                    issue_pv(1, n, j == 0);
                    umma_commit(&vempty[n % kVStages]);
                    if (more) {
                        issue_s(1, n + 1);
                        umma_commit(&kempty[(n + 1) % kKStages]);
                    }
                }
            }
            if (!ok) {
                *abort_flag = 1;
                atomicExch(p.err, kErrTimeout);
            }
        }
    } else {
        // ------------------------------------------------------------ softmax warpgroups
        // warps 2-5: query tile 0, warps 6-9: query tile 1; thread = row (TMEM lane).
        const int tile = warp >= 6 ? 1 : 0;
        const int q4 = warp & 3;
        const int r = 32 * q4 + lane;
        const int t_row = r / g, jh = r % g;
        const uint32_t trow = tmem + (static_cast<uint32_t>(32 * q4) << 16);
        const uint32_t tS = trow + tile * kWKeys;      // S_t, and P_t in its first 64 columns
        const uint32_t tO = trow + kColO + tile * kWD;  // O_t
        bool ok = true;
        int n = 0;  // running key-tile count
        for (int si = s_begin; si < s_end; ++si) {
            const Seg sg = load_seg(p.seg, si);
            const int h = sg.head;
            const int item = p.w_pair[2 * sg.pair + tile];
            const int ntok = item >= 0 ? p.w_ntok[item] : 0;
            const int tok0 = item >= 0 ? p.w_tok0[item] : 0;
            const int kend_t = item >= 0 ? p.w_kend[item] : 0;
            const int kv_end = p.pair_kend[sg.pair];
            const int last_tile = (kv_end + kWKeys - 1) / kWKeys - 1;
            const bool live = t_row < ntok;
            // last visible key: the row's own position, and never past its item's key range
            const int qlim = live ? min(p.tok_pos[tok0 + t_row], kend_t - 1) : -1;
            const int orow = p.tok_row[tok0 + (live ? t_row : 0)];
            const size_t oidx = static_cast<size_t>(orow) * p.H + h * g + jh;
            float m = -INFINITY, l = 0.f;
            for (int jt = sg.t0; jt < sg.t1 && ok; ++jt, ++n) {
                const int kbase = jt * kWKeys;
                const bool got = mbar_wait_bounded(&sfull[tile], static_cast<uint32_t>(n & 1));
                if (!__all_sync(0xffffffffu, got) || *abort_flag) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                // all 128 scores of the row, one TMEM wait; mask by absolute position only on
                // tiles that reach past this row's limit (earlier tiles are fully visible; dead
                // rows mask everything)
                const bool masked = kbase + kWKeys - 1 > qlim;
                float sv[kWKeys];
#pragma unroll
                for (int c = 0; c < kWKeys / 32; ++c) tmem_ld32(tS + c * 32, sv + c * 32);
                tmem_wait_ld();
                if (masked) {
#pragma unroll
                    for (int i = 0; i < kWKeys; ++i)
                        if (kbase + i > qlim) sv[i] = -INFINITY;
                }
                // row max as 8 independent chains
                float mx8[8];
#pragma unroll
                for (int kq = 0; kq < 8; ++kq) {
                    mx8[kq] = sv[kq];
#pragma unroll
                    for (int i = kq + 8; i < kWKeys; i += 8) mx8[kq] = fmaxf(mx8[kq], sv[i]);
                }
                const float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                                       fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
                // Lazy rescale: keep the exponent base of earlier tiles unless this tile's max
                // exceeds it by more than 8 (P stays <= 2^8 in bf16, l and O in fp32), so O in
                // TMEM is rescaled only when the base actually moves.
                const float mnew = (m == -INFINITY || mx > m + 8.f) ? mx : m;
                const float base = mnew == -INFINITY ? 0.f : mnew;
                const float corr = m == -INFINITY ? 0.f : ex2_approx(m - base);
                // P = 2^(S - base) as bf16 pairs over S's first 64 columns, 64 keys at a time
                float sum8[8];
#pragma unroll
                for (int kq = 0; kq < 8; ++kq) sum8[kq] = 0.f;
#pragma unroll
                for (int half = 0; half < kWKeys / 64; ++half) {
                    uint32_t pk[32];
#pragma unroll
                    for (int i = 0; i < 32; ++i) {
                        const float a = ex2_approx(sv[half * 64 + 2 * i] - base);
                        const float b = ex2_approx(sv[half * 64 + 2 * i + 1] - base);
                        sum8[i & 7] += a + b;
                        pk[i] = pack_bf16(a, b);
                    }
                    tmem_st32u(tS + half * 32, pk);
                }
                tmem_wait_st();
                l = l * corr + (((sum8[0] + sum8[1]) + (sum8[2] + sum8[3])) + ((sum8[4] + sum8[5]) + (sum8[6] + sum8[7])));
                m = mnew;
                // O is rescaled to the new base after P is written and before P.V of this tile
                // may start (pfull below). O already holds P.V of the previous tile: that MMA
                // was issued before this tile's S MMA, so it completed before sfull fired; the
                // pvdone wait only confirms it.
                if (jt > sg.t0 && __any_sync(0xffffffffu, corr != 1.f)) {
                    const bool done = mbar_wait_bounded(&pvdone[tile], static_cast<uint32_t>((n - 1) & 1));
                    if (!__all_sync(0xffffffffu, done) || *abort_flag) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
#pragma unroll 1
                    for (int c = 0; c < kWD / 32; ++c) {
                        float o[32];
                        tmem_ld32(tO + c * 32, o);
                        tmem_wait_ld();
#pragma unroll
                        for (int i = 0; i < 32; ++i) o[i] *= corr;
                        tmem_st32(tO + c * 32, o);
                    }
                    tmem_wait_st();
                }
                if (tile == 0 && jt == last_tile && kv_end < kbase + kWKeys) {
                    // keys past the context in the last tile: zero their V rows so P = 0 meets 0
                    // (tile 0's P.V is issued first, so tile 1's sees the zeros too)
                    const int s = n % kVStages;
                    const bool landed = mbar_wait_bounded(&vfull[s], static_cast<uint32_t>(n / kVStages) & 1u);
                    if (!__all_sync(0xffffffffu, landed)) {
                        ok = false;
                        break;
                    }
                    uint8_t* vd = smem + kOffV + s * kKVBytes;
                    const int first = kv_end - kbase;
                    const int units = (kWKeys - first) * 2 * 8;
                    for (int x = threadIdx.x - 64; x < units; x += 128) {
                        const int key = first + x / 16;
                        const int c = (x / 8) & 1;
                        *reinterpret_cast<uint4*>(vd + c * (kWKeys * 128) + sw128(key, x & 7)) = make_uint4(0, 0, 0, 0);
                    }
                    fence_proxy_async_smem();  // the zeroed V rows (generic writes) before the MMA reads them
                }
                tc_fence_before();
                // one arrival per warp (count 4): the MMA starts once all rows of P_t are written
                __syncwarp();
                if (lane == 0) mbar_arrive(&pfull[tile]);
            }
            if (ok) {
                const bool done = mbar_wait_bounded(&pvdone[tile], static_cast<uint32_t>((n - 1) & 1));
                ok = __all_sync(0xffffffffu, done) && !*abort_flag;
            }
            // ---- epilogue
            // O leaves TMEM one row per thread; the rows go to global memory through the 4 KB
            // of the tile's Q buffer that hold this warp's own 32 Q rows (dimensions 0-63):
            // every S MMA that read Q_t has completed, and this warp writes its next Q rows
            // only after this. 32 columns at a time, so that each store (and, in the
            // shared-prefix pass, each load of the split-KV row) covers 128 contiguous bytes
            // of 4 rows instead of 16 bytes of 32 rows. float4 slot i of staging row r sits at
            // slot i ^ (r & 7): conflict-free both ways.
            if (ok) tc_fence_after();
            float* stg = reinterpret_cast<float*>(smem + kOffQ + tile * kQBytes + q4 * 4096);
            auto stg4 = [&](int row, int i) { return reinterpret_cast<float4*>(stg + row * 32 + 4 * (i ^ (row & 7))); };
            const int sub = lane >> 3, cq = lane & 7;  // transposed: row 4*kk + sub, 4 columns at 4*cq
            if (sg.slot < 0) {
                // Final rows: o / l, or, in the shared-prefix pass, merged with the row the
                // split-KV kernel wrote (normalised, log-sum-exp lse_s):
                //   (o * 2^(m-M) + out * 2^(lse_s-M)) / (l * 2^(m-M) + 2^(lse_s-M)).
                float wo = l > 0.f ? 1.f / l : 0.f, wr = 0.f;
                if (ok && p.lse != nullptr && live) {
                    const float ls = p.lse[oidx];
                    const float mm = fmaxf(l > 0.f ? m : -INFINITY, ls);
                    const float a = l > 0.f ? exp2f(m - mm) : 0.f;
                    const float b = exp2f(ls - mm);
                    const float inv = 1.f / (l * a + b);
                    wo = a * inv;
                    wr = b * inv;
                }
                // the rows this lane stores in the transposed pass: their output offsets,
                // liveness and split-KV weights, from the lanes that own them
                const unsigned long long oidx64 = oidx;
                float* orow[8];
                float wrr[8];
                bool liv[8];
#pragma unroll
                for (int kk = 0; kk < 8; ++kk) {
                    const int src = 4 * kk + sub;
                    const unsigned long long oi = __shfl_sync(0xffffffffu, oidx64, src);
                    orow[kk] = p.out + static_cast<size_t>(oi) * kWD + 4 * cq;
                    wrr[kk] = __shfl_sync(0xffffffffu, wr, src);
                    liv[kk] = __shfl_sync(0xffffffffu, live ? 1 : 0, src) != 0;
                }
#pragma unroll 1
                for (int c = 0; c < kWD / 32 && ok; ++c) {
                    float o[32];
                    tmem_ld32(tO + c * 32, o);
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 8; ++i)
                        *stg4(lane, i) = make_float4(o[4 * i] * wo, o[4 * i + 1] * wo, o[4 * i + 2] * wo, o[4 * i + 3] * wo);
                    __syncwarp();
                    float4 y[8];
                    if (p.lse != nullptr) {
#pragma unroll
                        for (int kk = 0; kk < 8; ++kk)
                            y[kk] = liv[kk] ? *reinterpret_cast<const float4*>(orow[kk] + c * 32) : make_float4(0.f, 0.f, 0.f, 0.f);
                    }
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk) {
                        float4 x = *stg4(4 * kk + sub, cq);
                        if (p.lse != nullptr) {
                            x.x += y[kk].x * wrr[kk];
                            x.y += y[kk].y * wrr[kk];
                            x.z += y[kk].z * wrr[kk];
                            x.w += y[kk].w * wrr[kk];
                        }
                        if (liv[kk]) *reinterpret_cast<float4*>(orow[kk] + c * 32) = x;
                    }
                    __syncwarp();
                }
            } else if (ok) {
                // Partial: un-normalised O and (max, sum) of this row into the pair-head's
                // slot; wide_merge_kernel combines the slots afterwards. The warp's 32 slot
                // rows are consecutive.
                const size_t prow0 = (static_cast<size_t>(sg.slot) * 2 + tile) * kWRows + 32 * q4;
                float* po = p.part_o + prow0 * kWD + 4 * cq;
#pragma unroll 1
                for (int c = 0; c < kWD / 32; ++c) {
                    float o[32];
                    tmem_ld32(tO + c * 32, o);
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 8; ++i)
                        *stg4(lane, i) = make_float4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
                    __syncwarp();
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk)
                        *reinterpret_cast<float4*>(po + static_cast<size_t>(4 * kk + sub) * kWD + c * 32) =
                            *stg4(4 * kk + sub, cq);
                    __syncwarp();
                }
                p.part_ml[(prow0 + lane) * 2] = m;
                p.part_ml[(prow0 + lane) * 2 + 1] = l;
            }
            // the staging writes (generic proxy) before the next Q bulk copy into this buffer
            fence_proxy_async_smem();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&ofree[tile]);
        }
        if (!ok) {
            *abort_flag = 1;
            if (lane == 0) atomicExch(p.err, kErrTimeout);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

// One warp per row of a (pair, KV head) cut between CTAs: combines the row's partial slots
// (slot order, so the result does not depend on which CTA finished first) and, in the
// shared-prefix pass, the row the split-KV kernel wrote. Lane = 4 dims: coalesced.
__global__ void __launch_bounds__(256) wide_merge_kernel(const WideParams p, const int32_t* split, int nsplit) {
    const int wid = blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    const int e = wid / (2 * kWRows);
    if (e >= nsplit) return;
    const int tile = (wid / kWRows) & 1, r = wid % kWRows;
    const int pair = split[4 * e], h = split[4 * e + 1], s0 = split[4 * e + 2], ns = split[4 * e + 3];
    const int item = p.w_pair[2 * pair + tile];
    if (item < 0) return;
    const int g = p.g;
    const int t = r / g, j = r % g;
    if (t >= p.w_ntok[item]) return;
    const size_t oidx = static_cast<size_t>(p.tok_row[p.w_tok0[item] + t]) * p.H + h * g + j;
    auto ml = [&](int s) { return p.part_ml + ((static_cast<size_t>(s) * 2 + tile) * kWRows + r) * 2; };
    float4* op = reinterpret_cast<float4*>(p.out + oidx * kWD) + lane;
    // the split-KV row and its log-sum-exp, loaded up front (independent of the slots)
    float4 y = make_float4(0.f, 0.f, 0.f, 0.f);
    float ls = -INFINITY;
    if (p.lse != nullptr) {
        ls = p.lse[oidx];
        y = *op;
    }
    // slots' (max, sum) spread over the lanes (slot s0 + 32i + lane), then the max
    float mx = -INFINITY;
    for (int s = s0 + lane; s < s0 + ns; s += 32) mx = fmaxf(mx, ml(s)[0]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float L = 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int b0 = s0; b0 < s0 + ns; b0 += 32) {
        // this lane's slot weight, then every slot of the batch broadcast by shuffles; the
        // row loads of a batch are independent of each other
        const int sl = b0 + lane;
        float w = 0.f, lw = 0.f;
        if (sl < s0 + ns) {
            const float ms = ml(sl)[0];
            w = ms == -INFINITY ? 0.f : exp2f(ms - mx);
            lw = w * ml(sl)[1];
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) lw += __shfl_xor_sync(0xffffffffu, lw, o);
        L += lw;
        const int nb = min(32, s0 + ns - b0);
#pragma unroll 4
        for (int i = 0; i < nb; ++i) {
            const float wi = __shfl_sync(0xffffffffu, w, i);
            const float4 x = reinterpret_cast<const float4*>(p.part_o + ((static_cast<size_t>(b0 + i) * 2 + tile) * kWRows + r) * kWD)[lane];
            acc.x += wi * x.x;
            acc.y += wi * x.y;
            acc.z += wi * x.z;
            acc.w += wi * x.w;
        }
    }
    float wo = L > 0.f ? 1.f / L : 0.f, wr = 0.f;
    if (p.lse != nullptr) {
        // merge with the split-KV result: (acc * 2^(mx-M) + y * 2^(lse_s-M)) / (L * 2^(mx-M) + 2^(lse_s-M))
        const float mm = fmaxf(L > 0.f ? mx : -INFINITY, ls);
        const float a = L > 0.f ? exp2f(mx - mm) : 0.f;
        const float b = exp2f(ls - mm);
        const float inv = 1.f / (L * a + b);
        wo = a * inv;
        wr = b * inv;
    }
    *op = make_float4(acc.x * wo + y.x * wr, acc.y * wo + y.y * wr, acc.z * wo + y.z * wr, acc.w * wo + y.w * wr);
}

}  // namespace

size_t wide_smem_bytes() { return kSmemBytes; }

cudaError_t launch_wide_merge(const WideParams& p, const int32_t* split, int nsplit, cudaStream_t st) {
    if (nsplit <= 0) return cudaSuccess;
    const int warps = nsplit * 2 * kWRows;
    wide_merge_kernel<<<(warps + 7) / 8, 256, 0, st>>>(p, split, nsplit);
    return cudaGetLastError();
}

// Query tiles for the wide-tile kernel, packed once per call: tile item * kvh + h holds the
// item's 128 rows (token r / g, query head h * g + r % g), scaled into the exp2 domain and
// rounded to bf16, in the exact shared-memory image the S MMA reads ([64-dim chunk][row]
// [64], 128-byte swizzle), so that a CTA fetches it with one 32 KB bulk copy. Rows past the
// item's tokens are zero, and so is the extra last tile (the empty half of a pair).
__device__ __forceinline__ void pack_q_tile(const WideParams& p, int ntiles, uint8_t* __restrict__ qpk, int b) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint8_t* dst = qpk + static_cast<size_t>(b) * kQBytes;
    const bool real = b < ntiles;
    const int item = real ? b / p.kvh : 0, h = real ? b % p.kvh : 0;
    const int ntok = real ? p.w_ntok[item] : 0;
    const int tok0 = real ? p.w_tok0[item] : 0;
    const int g = p.g;
    const int c = lane >> 4, u = (lane & 15) >> 1, half = lane & 1;
#pragma unroll 1
    for (int i0 = 0; i0 < 32; i0 += 16) {
        float4 x[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const int r = 32 * warp + i0 + i;
            x[i] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (r / g < ntok) {
                const int row = p.tok_row[tok0 + r / g];
                const float* qp = p.q + (static_cast<size_t>(row) * p.H + h * g + r % g) * kWD;
                x[i] = __ldg(reinterpret_cast<const float4*>(qp) + lane);
            }
        }
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const int r = 32 * warp + i0 + i;
            const uint2 v = make_uint2(pack_bf16(x[i].x * p.qscale, x[i].y * p.qscale),
                                       pack_bf16(x[i].z * p.qscale, x[i].w * p.qscale));
            *reinterpret_cast<uint2*>(dst + c * (kWRows * 128) + sw128(r, u) + half * 8) = v;
        }
    }
}

__global__ void __launch_bounds__(128) wide_q_pack_kernel(const WideParams p, int ntiles, uint8_t* __restrict__ qpk) {
    pack_q_tile(p, ntiles, qpk, blockIdx.x);
}

// The pack and the append of the chunk rows (rows[0..n) of the step, fp32 -> the bf16
// pool, slot from the block table: sequence row_seq[r], position starts[s] + r - offsets[s])
// in one launch: CTAs 0..ntiles pack, the rest append 4 dims per thread.
__global__ void __launch_bounds__(128) wide_prep_kernel(const WideParams p, int ntiles, uint8_t* __restrict__ qpk,
                                                        const WideAppend a) {
    if (static_cast<int>(blockIdx.x) <= ntiles) {
        pack_q_tile(p, ntiles, qpk, blockIdx.x);
        return;
    }
    const int per_row = a.rowlen / 4;
    const int64_t total = a.n * per_row;
    for (int64_t i = (blockIdx.x - ntiles - 1) * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x - ntiles - 1) * blockDim.x) {
        const int64_t ri = i / per_row;
        const int c = static_cast<int>(i - ri * per_row) * 4;
        const int64_t r = a.rows[ri];
        const float4 kx = *reinterpret_cast<const float4*>(a.k + r * a.rowlen + c);
        const float4 vx = *reinterpret_cast<const float4*>(a.v + r * a.rowlen + c);
        int64_t slot;
        if (a.slots != nullptr) {
            slot = a.slots[ri];  // from the plan: one load instead of a chain of five
        } else {
            const int sq = a.row_seq[r];
            const int64_t pos = static_cast<int64_t>(a.starts[sq]) + (r - a.offsets[sq]);
            const int64_t blk = pos / a.bs;
            slot = static_cast<int64_t>(a.ids[a.indptr[sq] + blk]) * a.bs + (pos - blk * a.bs);
        }
        const int64_t dst = slot * a.rowlen + c;
        *reinterpret_cast<uint2*>(a.pool_k + dst) = make_uint2(pack_bf16(kx.x, kx.y), pack_bf16(kx.z, kx.w));
        *reinterpret_cast<uint2*>(a.pool_v + dst) = make_uint2(pack_bf16(vx.x, vx.y), pack_bf16(vx.z, vx.w));
    }
}

cudaError_t launch_wide_q_pack(const WideParams& p, int nitems, uint8_t* qpk, cudaStream_t st) {
    if (nitems <= 0) return cudaSuccess;
    const int ntiles = nitems * p.kvh;
    wide_q_pack_kernel<<<ntiles + 1, 128, 0, st>>>(p, ntiles, qpk);
    return cudaGetLastError();
}

cudaError_t launch_wide_prep(const WideParams& p, int nitems, uint8_t* qpk, const WideAppend& a, cudaStream_t st) {
    if (nitems <= 0) return cudaSuccess;
    const int ntiles = nitems * p.kvh;
    const int64_t items = a.n * (a.rowlen / 4);
    const int64_t ablocks = std::min<int64_t>((items + 127) / 128, 148 * 16);
    wide_prep_kernel<<<static_cast<unsigned>(ntiles + 1 + std::max<int64_t>(ablocks, 1)), 128, 0, st>>>(p, ntiles, qpk, a);
    return cudaGetLastError();
}

cudaError_t launch_wide_attention(const CUtensorMap* tmk1, const CUtensorMap* tmv1, const WideParams& p,
                                  cudaStream_t st) {
    if (p.nctas <= 0) return cudaSuccess;
    cudaError_t e = cudaFuncSetAttribute(wide_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e != cudaSuccess) return e;
    wide_attn_kernel<<<p.nctas, kWThreads, kSmemBytes, st>>>(*tmk1, *tmv1, p);
    return cudaGetLastError();
}

}  // namespace pk
