// Split-KV paged attention on the tensor cores for bf16 pools (decode rows, speculative
// verify windows, and prefill chunks cut into windows).
//
// Semantics: pagellm cache/paged.py:441-464 (write_and_attend's read half) with the
// causal rule of model/transformer.py:116-146 - the query at absolute position p sees
// keys 0..p of its sequence, read through the block table (cache/paged.py:309-352 is the
// block-at-a-time structure followed here).
//
// Work split. Every sequence's query rows are cut into "units" of at most 16/g query
// tokens (g = query heads per KV head), so one unit's (token, head) columns fit one or two
// n8 MMA tiles. A unit reads the blocks that hold positions 0..unit_ctx-1 (from block
// u_kb0 on when a shared prefix is attended by the wide-tile kernel instead). All units'
// blocks are laid end to end and the total is cut into `ncta` contiguous ranges: CTA c owns
// blocks [cta_blk[c], cta_blk[c+1]) (the planner's cut, which charges every unit boundary
// inside a range), or [c*T/ncta, (c+1)*T/ncta) without cta_blk. A unit inside one CTA is finished there;
// a unit cut by CTA boundaries leaves one partial (max, sum, un-normalised output) per
// CTA; the last CTA to finish a (unit, KV head) merges them in place (per-unit counters),
// or, without counters, merge_kernel does it in a second launch.
//
// Fused append: with k_new / v_new set, rows written in this step are taken from the fp32
// inputs (rounded to bf16) when their block is consumed, and stored to the pool by the unit
// that owns them, so no separate append launch is needed.
//
// CTA = 1 producer warp + one consumer warp per KV head. The producer streams each K/V
// block of the layer into a ring of shared-memory stages with TMA bulk tensor loads (no
// multicast) signalling mbarriers; consumers wait, compute, and release the stage.
//
// Per consumer warp and 16-token tile, with the transposed formulation (tokens as MMA rows):
//   S^T[16 x 8*NT] = K[16 x D] . Q^T[D x 8*NT]     (Q split as bf16 hi + lo for accuracy
//                                                   where registers allow: NT=1, D<=128)
//   online softmax down the columns (exp2 domain, scale folded into Q)
//   P^T -> bf16, transposed in registers with movmatrix into the B operand
//   O^T[D x 8*NT] += V^T[D x 16] . P^T[16 x 8*NT]  (V^T read with ldmatrix.trans)
// Shared-memory tiles use the TMA 128-byte swizzle, so the eight 16-byte rows of every
// ldmatrix phase land in distinct bank groups.

#include "pk_device.cuh"
#include "pk_internal.h"

namespace pk {

namespace {

__device__ __forceinline__ int upper_bound_i32(const int32_t* a, int n, int x) {
    int lo = 0, hi = n;
    while (lo < hi) {
        int mid = (lo + hi) >> 1;
        if (a[mid] <= x) lo = mid + 1; else hi = mid;
    }
    return lo;
}

// CTA whose block range holds block j: the planner's ranges (first blocks cta_blk[0..n]),
// else the equal ranges [c*T/n, (c+1)*T/n).
__device__ __forceinline__ int cta_of_block(int j, int T, int n, const int32_t* cta_blk) {
    if (cta_blk != nullptr) return upper_bound_i32(cta_blk, n + 1, j) - 1;
    int c = static_cast<int>(static_cast<int64_t>(j) * n / T);
    while (c + 1 < n && static_cast<int64_t>(c + 1) * T / n <= j) ++c;
    while (c > 0 && static_cast<int64_t>(c) * T / n > j) --c;
    return c;
}

// Normalised output of the columns a lane holds (C-fragment layout of O^T: dims
// mt*16 + grp (+8), columns nt*8 + 2*quad + e) for the live query tokens of a unit.
// With `lse` set, also the row's log2-domain log-sum-exp m + log2(l) ([rows][H]). With the
// fused head exchange on (po.n > 0) every row goes to each rank's result buffer instead.
template <int D, int NT>
__device__ __forceinline__ void store_rows(float* out, const float (&acc)[D / 16][NT][4],
                                           const float (&m)[NT][2], const float (&l)[NT][2],
                                           float* lse, int nq, int g, int H, int row0, int h,
                                           int quad, int grp, const PeerOut& po) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            const int col = nt * 8 + 2 * quad + e;
            const int tq = col / g;
            if (tq >= nq) continue;
            const float inv = 1.f / l[nt][e];
            if (po.n == 0) {
                const size_t orow = static_cast<size_t>(row0 + tq) * H + h * g + col % g;
                if (lse != nullptr && grp == 0) lse[orow] = m[nt][e] + log2f(l[nt][e]);
                float* op = out + orow * D;
#pragma unroll
                for (int mt = 0; mt < D / 16; ++mt) {
                    op[mt * 16 + grp] = acc[mt][nt][e] * inv;
                    op[mt * 16 + grp + 8] = acc[mt][nt][2 + e] * inv;
                }
            } else {
                const size_t orow = static_cast<size_t>(row0 + tq) * po.out_H + h * g + col % g;
                for (int r = 0; r < po.n; ++r) {
                    float* op = po.out[r] + orow * D;
#pragma unroll
                    for (int mt = 0; mt < D / 16; ++mt) {
                        op[mt * 16 + grp] = acc[mt][nt][e] * inv;
                        op[mt * 16 + grp + 8] = acc[mt][nt][2 + e] * inv;
                    }
                }
            }
        }
}

template <int D>
struct TileGeom {
    static constexpr int kChunks = D / 64;  // 128-byte swizzle rows per token and head
};

// Byte offset inside a swizzled K/V stage tile of the 16-byte unit holding
// dims [8*u, 8*u+8) of (head h, token t).
__device__ __forceinline__ uint32_t tile_off(int chunk, int h, int t, int u16, int kvh, int bs,
                                             int chunks, int per_head) {
    const int row = per_head ? ((h * bs + t) * chunks + chunk) : ((chunk * kvh + h) * bs + t);
    return static_cast<uint32_t>(row * 128 + ((u16 ^ (row & 7)) << 4));
}

// One unit's metadata: the plan's packed record (two 16-byte loads, one round trip) when
// present, else gathered from the per-unit and per-sequence arrays (a chain of dependent
// loads: unit -> sequence -> its start, row offset and table).
struct UnitInfo {
    int t0, n, kb0, row0, qpos0, blk0, blk1, tbase;
};
__device__ __forceinline__ UnitInfo load_unit(const TcParams& p, int u) {
    UnitInfo x;
    if (p.u_meta != nullptr) {
        const int4 a = __ldg(p.u_meta + 2 * u);
        const int4 b = __ldg(p.u_meta + 2 * u + 1);
        x.t0 = a.x;
        x.n = a.y;
        x.kb0 = a.z;
        x.row0 = a.w;
        x.qpos0 = b.x;
        x.blk0 = b.y;
        x.blk1 = b.z;
        x.tbase = b.w;
        return x;
    }
    const int seq = p.u_seq[u];
    x.t0 = p.u_t0[u];
    x.n = p.u_n[u];
    x.kb0 = p.u_kb0 != nullptr ? p.u_kb0[u] : 0;
    x.row0 = p.offsets[seq] + x.t0;
    x.qpos0 = p.starts[seq] + x.t0;
    x.blk0 = p.u_blk[u];
    x.blk1 = p.u_blk[u + 1];
    x.tbase = p.indptr[seq] + x.kb0 - x.blk0;
    return x;
}

// CTAs per first-level group of the two-level merge of a unit's partials.
constexpr int kMergeGroup = 6;

template <int D, int NT>
__global__ void __launch_bounds__((kTcMaxKvHeads + 1) * 32, 1)
    tc_attn_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                   const __grid_constant__ TcParams p) {
    constexpr int KS = D / 16;  // k-steps over the head dim / m-tiles of O^T
    constexpr int CH = TileGeom<D>::kChunks;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~uintptr_t(1023));
    // A CTA hosts V virtual CTAs (V > 1 for pools of few KV heads): each has its own block
    // range (partition entry blockIdx.x * V + v), stage ring, barriers and kvh consumer warps,
    // so that an SM runs up to 8 consumer warps under one producer warp whatever kvh is.
    const int V = p.virt > 1 ? p.virt : 1;
    const int tile_bytes = p.bs * p.kvh * D * 2;
    const int ring_bytes = p.stages * 2 * tile_bytes;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + V * ring_bytes);
    uint64_t* empty = full + V * p.stages;
    // each virtual CTA's end of work (one arrival per consumer warp of it), then one barrier
    // per consumer warp for the bulk copies of its end-of-range merge
    uint64_t* endbar = empty + V * p.stages;
    uint64_t* mbar_m = endbar + V;
    // with the fused head exchange on: each consumer warp's 4-row staging area for the rows it
    // stores to every rank (tc_peer_stage_bytes beyond the pool's usual shared memory)
    float* peer_stage = reinterpret_cast<float*>(
        (reinterpret_cast<uintptr_t>(mbar_m + kTcMaxKvHeads) + 15) & ~uintptr_t(15));

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int nwc = p.kvh * V;  // consumer warps

    if (threadIdx.x == 0) {
        for (int s = 0; s < V * p.stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], p.kvh);
        }
        for (int v = 0; v < V; ++v) mbar_init(&endbar[v], p.kvh);
        for (int w = 0; w < nwc; ++w) mbar_init(&mbar_m[w], 1);
        fence_mbar_init();
    }
    __syncthreads();

    // block range [lo, hi) of virtual CTA cv (empty past the partition)
    auto range_of = [&](int cv, int& lo_, int& hi_) {
        if (cv >= p.ncta) {
            lo_ = hi_ = p.total_blocks;
            return;
        }
        lo_ = p.cta_blk ? p.cta_blk[cv] : static_cast<int>(static_cast<int64_t>(cv) * p.total_blocks / p.ncta);
        hi_ = p.cta_blk ? p.cta_blk[cv + 1] : static_cast<int>(static_cast<int64_t>(cv + 1) * p.total_blocks / p.ncta);
    };
    const int vme = warp < nwc ? warp / p.kvh : 0;  // this warp's virtual CTA (the producer: 0)
    const int c = blockIdx.x * V + vme;             // its partition entry
    int lo, hi;
    range_of(c, lo, hi);
    const int u_first = upper_bound_i32(p.u_blk, p.nu + 1, lo) - 1;
    uint8_t* ring = smem + vme * ring_bytes;
    uint64_t* vfull = full + vme * p.stages;
    uint64_t* vempty = empty + vme * p.stages;
    uint64_t* vend = endbar + vme;

    if (warp == nwc) {
        // ------------------------------------------------------------ producer
        if (lane == 0 && V == 1) {
            prefetch_tensormap(&tmk);
            prefetch_tensormap(&tmv);
            // K/V blocks are read once per launch: first out of L2, so that what is read again
            // (queries, block tables, the partials the merges fetch) stays there
            const uint64_t evict_first = l2_policy_evict_first();
            int it = 0;
            bool ok = true;
            for (int j = lo, u = u_first; j < hi && ok; ++u) {
                const UnitInfo ui = load_unit(p, u);
                const int uend = min(hi, ui.blk1);
                const int tbase = ui.tbase;
                // the unit's query rows into L2 while its first blocks stream in
                prefetch_l2_bulk(p.q + static_cast<size_t>(ui.row0) * p.H * D,
                                 static_cast<uint32_t>(ui.n) * p.H * D * 4u);
                for (; j < uend; ++j, ++it) {
                    const int s = it % p.stages;
                    const uint32_t k = static_cast<uint32_t>(it / p.stages);
                    if (!mbar_wait_bounded(&vempty[s], (k & 1u) ^ 1u)) {
                        atomicExch(p.err, kErrTimeout);
                        ok = false;
                        break;
                    }
                    const int phys = p.ids[tbase + j];
                    const int slot0 = static_cast<int>(p.layer_slot0 + static_cast<int64_t>(phys) * p.bs);
                    uint8_t* kd = ring + s * 2 * tile_bytes;
                    uint8_t* vd = kd + tile_bytes;
                    mbar_arrive_expect_tx(&vfull[s], 2u * tile_bytes);
                    if (!p.per_head_layout) {
                        tma_load_4d_hint(kd, &tmk, 0, slot0, 0, 0, &vfull[s], evict_first);
                        tma_load_4d_hint(vd, &tmv, 0, slot0, 0, 0, &vfull[s], evict_first);
                    } else {
                        const int hb = p.bs * CH * 128;
                        for (int h = 0; h < p.kvh; ++h) {
                            tma_load_4d_hint(kd + h * hb, &tmk, 0, 0, h, slot0, &vfull[s], evict_first);
                            tma_load_4d_hint(vd + h * hb, &tmv, 0, 0, h, slot0, &vfull[s], evict_first);
                        }
                    }
                }
            }
            // Never leave the CTA with copies still landing in its shared memory.
            for (int t = max(0, it - p.stages); t < it; ++t) {
                mbar_wait_bounded(&vfull[t % p.stages], static_cast<uint32_t>(t / p.stages) & 1u);
            }
        } else if (V > 1) {
            // Lane v feeds virtual CTA v. The lanes advance in warp-uniform rounds: each issues
            // its next block once that stage of its ring is free (non-blocking test), and the
            // warp gives up after kWaitLimitNs without any lane making progress.
            const bool has = lane < V;
            int vlo = 0, vhi = 0;
            if (has) range_of(blockIdx.x * V + lane, vlo, vhi);
            uint8_t* vr = smem + (has ? lane : 0) * ring_bytes;
            uint64_t* pf = full + (has ? lane : 0) * p.stages;
            uint64_t* pe = empty + (has ? lane : 0) * p.stages;
            if (lane == 0) {
                prefetch_tensormap(&tmk);
                prefetch_tensormap(&tmv);
            }
            const uint64_t evict_first = l2_policy_evict_first();
            int j = vlo, it = 0, uend = 0, tbase = 0;
            int u = has ? upper_bound_i32(p.u_blk, p.nu + 1, vlo) - 1 : 0;
            bool active = has && j < vhi, fresh = true;
            unsigned long long t_last = global_ns();
            while (__any_sync(0xffffffffu, active)) {
                bool issued = false;
                if (active) {
                    if (fresh) {
                        const UnitInfo ui = load_unit(p, u);
                        uend = min(vhi, ui.blk1);
                        tbase = ui.tbase;
                        prefetch_l2_bulk(p.q + static_cast<size_t>(ui.row0) * p.H * D,
                                         static_cast<uint32_t>(ui.n) * p.H * D * 4u);
                        fresh = false;
                    }
                    const int s = it % p.stages;
                    const uint32_t k = static_cast<uint32_t>(it / p.stages);
                    if (mbar_test_wait(&pe[s], (k & 1u) ^ 1u)) {
                        const int phys = p.ids[tbase + j];
                        const int slot0 = static_cast<int>(p.layer_slot0 + static_cast<int64_t>(phys) * p.bs);
                        uint8_t* kd = vr + s * 2 * tile_bytes;
                        uint8_t* vd = kd + tile_bytes;
                        mbar_arrive_expect_tx(&pf[s], 2u * tile_bytes);
                        if (!p.per_head_layout) {
                            tma_load_4d_hint(kd, &tmk, 0, slot0, 0, 0, &pf[s], evict_first);
                            tma_load_4d_hint(vd, &tmv, 0, slot0, 0, 0, &pf[s], evict_first);
                        } else {
                            const int hb = p.bs * CH * 128;
                            for (int h = 0; h < p.kvh; ++h) {
                                tma_load_4d_hint(kd + h * hb, &tmk, 0, 0, h, slot0, &pf[s], evict_first);
                                tma_load_4d_hint(vd + h * hb, &tmv, 0, 0, h, slot0, &pf[s], evict_first);
                            }
                        }
                        ++j;
                        ++it;
                        issued = true;
                        if (j >= uend) {
                            ++u;
                            fresh = true;
                        }
                        active = j < vhi;
                    }
                }
                if (__any_sync(0xffffffffu, issued)) {
                    t_last = global_ns();
                } else if (global_ns() - t_last > kWaitLimitNs) {
                    if (lane == 0) atomicExch(p.err, kErrTimeout);
                    break;
                }
            }
            // Never leave the CTA with copies still landing in its shared memory.
            if (has)
                for (int t = max(0, it - p.stages); t < it; ++t)
                    mbar_wait_bounded(&pf[t % p.stages], static_cast<uint32_t>(t / p.stages) & 1u);
        }
        return;
    }

    // ---------------------------------------------------------------- consumers
    const int h = warp - vme * p.kvh;  // KV head within virtual CTA vme
    const int g = p.g;
    const int quad = lane & 3;   // column pair within an n8 tile
    const int grp = lane >> 2;   // row within an 8-row group
    int it = 0;
    bool alive = true;
    for (int j = lo, u = u_first; j < hi && alive; ++u) {
        const UnitInfo ui = load_unit(p, u);
        const int ublk1 = ui.blk1;             // the unit's blocks end here (this range may end first)
        const int uend = min(hi, ublk1);
        const int ublk0 = ui.blk0;
        const int t0 = ui.t0;
        const int nq = ui.n;
        const int qpos0 = ui.qpos0;            // absolute position of the unit's first query
        const int uctx = qpos0 + nq;           // keys kb0*bs..uctx-1 are read
        const int kb0 = ui.kb0;
        const int row0 = ui.row0;

        // Q^T as the B operand: column n = lane/4 of each n8 tile, dims 2*quad(+1), +8.
        // Q's low half (q - bf16(q)) only where registers allow it: with two n8 tiles or
        // head_dim 256 the 168-register cap of a 9-warp CTA would spill it, so there Q is
        // used at bf16 (the precision the wide-tile kernel uses throughout).
        constexpr bool kLo = NT == 1 && D <= 128;
        uint32_t qh[KS][NT][2], ql[kLo ? KS : 1][NT][2];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const int col = nt * 8 + grp;
            const int tq = col / g;
            const bool live = tq < nq;
            const float* qp = p.q + (static_cast<size_t>(row0 + (live ? tq : 0)) * p.H + h * g +
                                     col % g) * D;
#pragma unroll
            for (int ks = 0; ks < KS; ++ks) {
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    float2 x = make_float2(0.f, 0.f);
                    if (live) x = *reinterpret_cast<const float2*>(qp + ks * 16 + half * 8 + 2 * quad);
                    x.x *= p.qscale;
                    x.y *= p.qscale;
                    const uint32_t hb = pack_bf16(x.x, x.y);
                    qh[ks][nt][half] = hb;
                    if constexpr (kLo) ql[ks][nt][half] = pack_bf16(x.x - bf16_lo_f(hb), x.y - bf16_hi_f(hb));
                }
            }
        }
        // Causal limit of the C-fragment columns this lane holds (2*quad, 2*quad+1).
        int lim[NT][2];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int tq = (nt * 8 + 2 * quad + e) / g;
                lim[nt][e] = tq < nq ? qpos0 + tq : -1;
            }

        float m[NT][2], l[NT][2];
        float acc[KS][NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            m[nt][0] = m[nt][1] = -INFINITY;
            l[nt][0] = l[nt][1] = 0.f;
#pragma unroll
            for (int mt = 0; mt < KS; ++mt)
#pragma unroll
                for (int i = 0; i < 4; ++i) acc[mt][nt][i] = 0.f;
        }

        for (; j < uend; ++j, ++it) {
            const int s = it % p.stages;
            // Every lane waits; the verdict is made warp-uniform (and the warp reconverged)
            // before the .sync.aligned matrix instructions below.
            const bool got = mbar_wait_bounded(&vfull[s], static_cast<uint32_t>(it / p.stages) & 1u);
            if (!__all_sync(0xffffffffu, got)) {
                if (lane == 0) {
                    atomicExch(p.err, kErrTimeout);
                    mbar_arrive(vend);  // the other warps' end-of-work wait does not hang on this one
                }
                alive = false;
                break;
            }
            const uint32_t kst = smem_u32(ring + s * 2 * tile_bytes);
            const uint32_t vst = kst + tile_bytes;
            const int kpos0 = (j - ublk0 + kb0) * p.bs;
            const int nvalid = min(p.bs, uctx - kpos0);
            if (nvalid < p.bs) {
                // Slots past the context may hold anything; zero this head's V rows there so
                // that 0 * V stays 0 in the P.V product.
                uint8_t* vgen = ring + s * 2 * tile_bytes + tile_bytes;
                const int units = (p.bs - nvalid) * CH * 8;
                for (int x = lane; x < units; x += 32) {
                    const int t = nvalid + x / (CH * 8);
                    const int ch = (x / 8) % CH;
                    const int u16 = x % 8;
                    *reinterpret_cast<uint4*>(vgen + tile_off(ch, h, t, u16, p.kvh, p.bs, CH,
                                                              p.per_head_layout)) =
                        make_uint4(0, 0, 0, 0);
                }
                __syncwarp();
            }
            // Rows appended in this step (positions >= the sequence's start) come from the
            // fp32 inputs, rounded to bf16, instead of from the pool; the unit whose own
            // query rows they are also stores them to the pool (the fused append).
            bool patched = false;
            if (p.k_new != nullptr) {
                const int s_start = qpos0 - t0;  // the sequence's first new position
                const int lo_pos = max(kpos0, s_start);
                const int hi_pos = min(kpos0 + p.bs, uctx);
                if (lo_pos < hi_pos) {
                    patched = true;
                    uint8_t* kgen = ring + s * 2 * tile_bytes;
                    uint8_t* vgen = kgen + tile_bytes;
                    const int phys = p.ids[ui.tbase + j];
                    const int row_base = row0 - qpos0;  // row of position pos: row_base + pos
                    // (position, 4-dim) items, lane-strided; each batch issues all its loads
                    // (read-only inputs) before any store, so the rows' latencies overlap.
                    constexpr int kPerRow = D / 4;
                    constexpr int kBatch = (NT == 1 && D <= 128) ? 2 : 1;  // register budget
                    const int items = (hi_pos - lo_pos) * kPerRow;
                    for (int base = 0; base < items; base += 32 * kBatch) {
                        float4 kx[kBatch], vx[kBatch];
#pragma unroll
                        for (int e = 0; e < kBatch; ++e) {
                            const int it = base + e * 32 + lane;
                            if (it < items) {
                                const size_t src = (static_cast<size_t>(row_base + lo_pos + it / kPerRow) * p.kvh + h) * D +
                                                   (it % kPerRow) * 4;
                                kx[e] = __ldg(reinterpret_cast<const float4*>(p.k_new + src));
                                vx[e] = __ldg(reinterpret_cast<const float4*>(p.v_new + src));
                            }
                        }
#pragma unroll
                        for (int e = 0; e < kBatch; ++e) {
                            const int it = base + e * 32 + lane;
                            if (it >= items) continue;
                            const int pos = lo_pos + it / kPerRow;
                            const int d0 = (it % kPerRow) * 4;
                            const int t = pos - kpos0;
                            const uint2 kb = make_uint2(pack_bf16(kx[e].x, kx[e].y), pack_bf16(kx[e].z, kx[e].w));
                            const uint2 vb = make_uint2(pack_bf16(vx[e].x, vx[e].y), pack_bf16(vx[e].z, vx[e].w));
                            const uint32_t off = tile_off(d0 >> 6, h, t, (d0 & 63) >> 3, p.kvh, p.bs, CH,
                                                          p.per_head_layout) + ((d0 & 7) ? 8u : 0u);
                            *reinterpret_cast<uint2*>(kgen + off) = kb;
                            *reinterpret_cast<uint2*>(vgen + off) = vb;
                            if (pos >= qpos0) {
                                const size_t dst = (static_cast<size_t>(phys) * p.bs + t) * p.kvh * D + h * D + d0;
                                *reinterpret_cast<uint2*>(p.pool_k + dst) = kb;
                                *reinterpret_cast<uint2*>(p.pool_v + dst) = vb;
                            }
                        }
                    }
                    __syncwarp();
                }
            }
            for (int mtile = 0; mtile < p.bs / 16; ++mtile) {
                // ---- S^T = K . Q^T
                float sacc[NT][4];
#pragma unroll
                for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                    for (int i = 0; i < 4; ++i) sacc[nt][i] = 0.f;
                {
                    const int tk = mtile * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
                    for (int ks = 0; ks < KS; ++ks) {
                        const int u16 = (ks & 3) * 2 + (lane >> 4);
                        uint32_t a[4];
                        ldmatrix_x4(a, kst + tile_off(ks >> 2, h, tk, u16, p.kvh, p.bs, CH,
                                                      p.per_head_layout));
#pragma unroll
                        for (int nt = 0; nt < NT; ++nt) {
                            mma_bf16_16816(sacc[nt], a, qh[ks][nt][0], qh[ks][nt][1]);
                            if constexpr (kLo) mma_bf16_16816(sacc[nt], a, ql[ks][nt][0], ql[ks][nt][1]);
                        }
                    }
                }
                // ---- mask + online softmax down each column
                const int kp_a = kpos0 + mtile * 16 + grp;  // rows held: grp and grp + 8
                const int kp_b = kp_a + 8;
                uint32_t pb[NT][2];
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    float pr[4];
#pragma unroll
                    for (int e = 0; e < 2; ++e) {
                        const float xa = (kp_a <= lim[nt][e] && kp_a < uctx) ? sacc[nt][e] : -INFINITY;
                        const float xb = (kp_b <= lim[nt][e] && kp_b < uctx) ? sacc[nt][2 + e] : -INFINITY;
                        float mx = fmaxf(xa, xb);
                        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
                        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
                        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
                        const float mnew = fmaxf(m[nt][e], mx);
                        const float base = (mnew == -INFINITY) ? 0.f : mnew;
                        const float corr = exp2f(m[nt][e] - base);
                        const float pa = exp2f(xa - base);
                        const float pbv = exp2f(xb - base);
                        l[nt][e] = l[nt][e] * corr + pa + pbv;
                        m[nt][e] = mnew;
#pragma unroll
                        for (int mt = 0; mt < KS; ++mt) {
                            acc[mt][nt][e] *= corr;
                            acc[mt][nt][2 + e] *= corr;
                        }
                        pr[e] = pa;
                        pr[2 + e] = pbv;
                    }
                    // P^T C-fragment rows grp / grp+8 -> B operand (k = token, n = column)
                    pb[nt][0] = movmatrix_trans(pack_bf16(pr[0], pr[1]));
                    pb[nt][1] = movmatrix_trans(pack_bf16(pr[2], pr[3]));
                }
                // ---- O^T += V^T . P^T
                {
                    const int tv = mtile * 16 + (lane & 7) + (lane >> 4) * 8;
#pragma unroll
                    for (int mt = 0; mt < KS; ++mt) {
                        const int u16 = (mt & 3) * 2 + ((lane >> 3) & 1);
                        uint32_t a[4];
                        ldmatrix_x4_trans(a, vst + tile_off(mt >> 2, h, tv, u16, p.kvh, p.bs, CH,
                                                            p.per_head_layout));
#pragma unroll
                        for (int nt = 0; nt < NT; ++nt) mma_bf16_16816(acc[mt][nt], a, pb[nt][0], pb[nt][1]);
                    }
                }
            }
            // Generic-proxy writes into the stage must be ordered before the next TMA fill.
            if (nvalid < p.bs || patched) fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(&vempty[s]);
        }
        if (!alive) break;

        // ---- finish the unit's segment
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                float t = l[nt][e];
                t += __shfl_xor_sync(0xffffffffu, t, 4);
                t += __shfl_xor_sync(0xffffffffu, t, 8);
                t += __shfl_xor_sync(0xffffffffu, t, 16);
                l[nt][e] = t;
            }
        // The last unit of the range: once every consumer warp of the (virtual) CTA is here, no
        // stage of its ring is read or filled any more, and its warps may stage a merge there.
        bool at_end = false;
        if (ublk1 >= hi) {
            __syncwarp();
            if (lane == 0) mbar_arrive(vend);
            at_end = __all_sync(0xffffffffu, mbar_wait_bounded(vend, 0u));
        }
        // The unit's output rows. With the fused head exchange at the end of the range they go
        // through this warp's share of the idle stage ring, so that every rank receives them as
        // 16-byte stores in 512-byte runs (rows of a token's g heads are contiguous there);
        // elsewhere store_rows.
        auto store_out = [&](const float (&o)[KS][NT][4], const float (&mm)[NT][2], const float (&ll)[NT][2]) {
            if (p.peer.n == 0) {
                store_rows<D, NT>(p.out, o, mm, ll, p.lse, nq, g, p.H, row0, h, quad, grp, p.peer);
                return;
            }
            // Every rank receives the rows as whole 512-byte runs of 16-byte stores: 4 rows at a
            // time go through this warp's staging area (rows padded to D + 4 floats, so that a
            // warp's column groups hit different banks), then each row leaves contiguously.
            constexpr int Dp = D + 4;
            float* tile = peer_stage + static_cast<size_t>(warp) * 4 * Dp;
            const int ncol = nq * g;
            for (int c0 = 0; c0 < ncol; c0 += 4) {
#pragma unroll
                for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                    for (int e = 0; e < 2; ++e) {
                        const int col = nt * 8 + 2 * quad + e;
                        if (col < c0 || col >= c0 + 4 || col >= ncol) continue;
                        const float inv = 1.f / ll[nt][e];
#pragma unroll
                        for (int mt = 0; mt < KS; ++mt) {
                            tile[(col - c0) * Dp + mt * 16 + grp] = o[mt][nt][e] * inv;
                            tile[(col - c0) * Dp + mt * 16 + grp + 8] = o[mt][nt][2 + e] * inv;
                        }
                    }
                __syncwarp();
                const int n4 = min(4, ncol - c0) * (D / 4);
                for (int i = lane; i < n4; i += 32) {
                    const int lc = i / (D / 4);
                    const int d4 = i - lc * (D / 4);
                    const int col = c0 + lc;
                    const float4 v = *reinterpret_cast<const float4*>(tile + lc * Dp + d4 * 4);
                    const size_t orow = static_cast<size_t>(row0 + col / g) * p.peer.out_H + h * g + col % g;
                    for (int r = 0; r < p.peer.n; ++r) reinterpret_cast<float4*>(p.peer.out[r] + orow * D)[d4] = v;
                }
                __syncwarp();
            }
        };
        const bool whole = ublk0 >= lo && ublk1 <= hi;
        if (whole) {
            store_out(acc, m, l);
        } else {
            // The partial of (unit u, CTA c, head h): (max, sum) per live column at
            // part_ml[slot][h][col], and the un-normalised O in fragment order interleaved by
            // lane - accumulator quad j = mt * NT + nt of lane L is float4 j * 32 + L of
            // part_o[slot][h] - so each of the KS * NT 16-byte accesses of a warp covers 512
            // contiguous bytes, in global memory and (conflict-free) in shared memory.
            constexpr int kFrag = KS * NT * 4;  // floats per lane
            const size_t seg = static_cast<size_t>(u) + c;
            const size_t base = (seg * p.kvh + h) * kMaxCols;
            bool lane_live = false;
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const int col = nt * 8 + 2 * quad + e;
                    if (col / g >= nq) continue;
                    lane_live = true;
                    if (grp == 0) {
                        p.part_ml[(base + col) * 2] = m[nt][e];
                        p.part_ml[(base + col) * 2 + 1] = l[nt][e];
                    }
                }
            if (lane_live) {
                float4* po = reinterpret_cast<float4*>(p.part_o + base * D) + lane;
#pragma unroll
                for (int mt = 0; mt < KS; ++mt)
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt)
                        po[(mt * NT + nt) * 32] = make_float4(acc[mt][nt][0], acc[mt][nt][1], acc[mt][nt][2], acc[mt][nt][3]);
            }
            if (p.counters != nullptr) {
                // Two-level merge in fixed order. The unit's CTAs cf..cl form groups of
                // kMergeGroup consecutive CTAs; the last CTA of a group to finish head h merges
                // the group's partials (in parallel with the other groups); with several
                // groups it stores the group's partial in the slot of the group's first CTA,
                // and the last group to finish merges the group partials. A unit spread over
                // many CTAs (a long sequence) then costs two short merges at the end of the
                // launch instead of one long one. Counters are left at zero for the next launch.
                // the unit's first and last CTA, from the plan (one round trip, no search)
                const int cf = p.u_cta != nullptr ? p.u_cta[2 * u] : cta_of_block(ublk0, p.total_blocks, p.ncta, p.cta_blk);
                const int cl = p.u_cta != nullptr ? p.u_cta[2 * u + 1]
                                                  : cta_of_block(ublk1 - 1, p.total_blocks, p.ncta, p.cta_blk);
                const int ngr = (cl - cf + kMergeGroup) / kMergeGroup;
                const int g0 = cf + (c - cf) / kMergeGroup * kMergeGroup;
                const int g1 = min(cl, g0 + kMergeGroup - 1);
                auto arrive_last = [&](int* ctr, int count) {
                    __syncwarp();
                    int last = 0;
                    if (lane == 0) {
                        __threadfence();  // release the warp's partial (ordered by __syncwarp)
                        last = atomicAdd(ctr, 1) == count - 1;
                        if (last) *ctr = 0;
                    }
                    last = __shfl_sync(0xffffffffu, last, 0);
                    if (last) __threadfence();
                    return last != 0;
                };
                float mx[NT][2], den[NT][2];
                float num[KS][NT][4];
                auto reset = [&]() {
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                        for (int e = 0; e < 2; ++e) {
                            mx[nt][e] = -INFINITY;
                            den[nt][e] = 0.f;
                        }
#pragma unroll
                    for (int mt = 0; mt < KS; ++mt)
#pragma unroll
                        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                            for (int i = 0; i < 4; ++i) num[mt][nt][i] = 0.f;
                };
                // folds one partial into (mx, den, num): ml = its (max, sum) row, fr = the
                // partial's O plus this lane (quad j at fr[j * 32]); an online softmax merge, so
                // the order of folds fixes the bits
                auto fold = [&](const float* ml, const float4* fr, bool from_global) {
                    float a[NT][2], b[NT][2];
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                        for (int e = 0; e < 2; ++e) {
                            const int col = nt * 8 + 2 * quad + e;
                            const bool live = col / g < nq;
                            const float mc = live ? (from_global ? __ldcg(ml + 2 * col) : ml[2 * col]) : -INFINITY;
                            const float lc = live ? (from_global ? __ldcg(ml + 2 * col + 1) : ml[2 * col + 1]) : 0.f;
                            const float mn = fmaxf(mx[nt][e], mc);
                            a[nt][e] = mx[nt][e] == -INFINITY ? 0.f : exp2f(mx[nt][e] - mn);
                            b[nt][e] = mc == -INFINITY ? 0.f : exp2f(mc - mn);
                            mx[nt][e] = mn;
                            den[nt][e] = den[nt][e] * a[nt][e] + lc * b[nt][e];
                        }
#pragma unroll
                    for (int mt = 0; mt < KS; ++mt)
#pragma unroll
                        for (int nt = 0; nt < NT; ++nt) {
                            float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
                            if (lane_live) x = from_global ? __ldcg(fr + (mt * NT + nt) * 32) : fr[(mt * NT + nt) * 32];
                            num[mt][nt][0] = num[mt][nt][0] * a[nt][0] + x.x * b[nt][0];
                            num[mt][nt][1] = num[mt][nt][1] * a[nt][1] + x.y * b[nt][1];
                            num[mt][nt][2] = num[mt][nt][2] * a[nt][0] + x.z * b[nt][0];
                            num[mt][nt][3] = num[mt][nt][3] * a[nt][1] + x.w * b[nt][1];
                        }
                };
                // Merges the partials in the slots of CTAs first, first + stride, ... (count of
                // them) into (mx, den, num), every one read as stored. At the end of the CTA's
                // range they are staged in this warp's share of the idle stage ring, several per
                // bulk-copy round trip; elsewhere (a merge mid-range, rare) register loads are
                // used, two partials per round trip. Returns false if a wait timed out.
                constexpr uint32_t kFragBytes = 32u * kFrag * 4u;  // all lanes' fragments
                constexpr uint32_t kMlBytes = kMaxCols * 2u * 4u;  // (max, sum) of every column
                constexpr uint32_t kPieceBytes = kFragBytes + kMlBytes;
                const uint32_t region_bytes = (static_cast<uint32_t>(p.stages) * 2u * tile_bytes / p.kvh) & ~127u;
                const int per_batch = static_cast<int>(region_bytes / kPieceBytes);
                int batches = 0;  // this warp's merge barrier phases used so far
                auto merge = [&](int first, int count, int stride) {
                    reset();
                    auto seg_of = [&](int i) { return (static_cast<size_t>(u) + first + i * stride) * p.kvh + h; };
                    if (at_end && per_batch >= 2) {
                        uint8_t* region = ring + static_cast<size_t>(h) * region_bytes;
                        uint64_t* mb = &mbar_m[warp];
                        if (lane == 0) fence_proxy_async_global();
                        for (int i0 = 0; i0 < count; i0 += per_batch) {
                            const int nb = min(per_batch, count - i0);
                            if (lane == 0) {
                                mbar_arrive_expect_tx(mb, static_cast<uint32_t>(nb) * kPieceBytes);
                                for (int i = 0; i < nb; ++i) {
                                    const size_t sg2 = seg_of(i0 + i);
                                    bulk_load(region + i * kPieceBytes, p.part_o + sg2 * kMaxCols * D, kFragBytes, mb);
                                    bulk_load(region + i * kPieceBytes + kFragBytes, p.part_ml + sg2 * kMaxCols * 2,
                                              kMlBytes, mb);
                                }
                            }
                            const bool got = mbar_wait_bounded(mb, static_cast<uint32_t>(batches & 1));
                            ++batches;
                            if (!__all_sync(0xffffffffu, got)) {
                                if (lane == 0) atomicExch(p.err, kErrTimeout);
                                return false;
                            }
                            for (int i = 0; i < nb; ++i)
                                fold(reinterpret_cast<const float*>(region + i * kPieceBytes + kFragBytes),
                                     reinterpret_cast<const float4*>(region + i * kPieceBytes) + lane, false);
                            __syncwarp();  // every lane is done with the batch before the next lands
                        }
                        return true;
                    }
                    auto fold_at = [&](int i) {
                        const size_t sg2 = seg_of(i);
                        fold(p.part_ml + sg2 * kMaxCols * 2,
                             reinterpret_cast<const float4*>(p.part_o + sg2 * kMaxCols * D) + lane, true);
                    };
                    if constexpr (NT == 1 && D <= 128) {
#pragma unroll 2
                        for (int i = 0; i < count; ++i) fold_at(i);
                    } else {
#pragma unroll 1
                        for (int i = 0; i < count; ++i) fold_at(i);
                    }
                    return true;
                };
                if (arrive_last(p.counters + (static_cast<size_t>(u) + g0) * p.kvh + h, g1 - g0 + 1) &&
                    merge(g0, g1 - g0 + 1, 1)) {
                    if (ngr == 1) {
                        store_out(num, mx, den);
                    } else {
                        // the group's partial, in the slot of its first CTA (whose partial the
                        // merge has consumed)
                        const size_t gb = ((static_cast<size_t>(u) + g0) * p.kvh + h) * kMaxCols;
#pragma unroll
                        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                            for (int e = 0; e < 2; ++e) {
                                const int col = nt * 8 + 2 * quad + e;
                                if (col / g < nq && grp == 0) {
                                    p.part_ml[(gb + col) * 2] = mx[nt][e];
                                    p.part_ml[(gb + col) * 2 + 1] = den[nt][e];
                                }
                            }
                        if (lane_live) {
                            float4* po = reinterpret_cast<float4*>(p.part_o + gb * D) + lane;
#pragma unroll
                            for (int mt = 0; mt < KS; ++mt)
#pragma unroll
                                for (int nt = 0; nt < NT; ++nt)
                                    po[(mt * NT + nt) * 32] =
                                        make_float4(num[mt][nt][0], num[mt][nt][1], num[mt][nt][2], num[mt][nt][3]);
                        }
                        if (arrive_last(p.unit_counters + static_cast<size_t>(u) * p.kvh + h, ngr) &&
                            merge(cf, ngr, kMergeGroup))
                            store_out(num, mx, den);
                    }
                }
            }
        }
    }
    if (p.peer.n > 0) {
        // Fused head exchange: every consumer warp (with work or not, timed out or not) counts
        // itself done with an acquire-release increment at system scope, which orders its rows'
        // stores before the count; the last of the launch, which has acquired every other
        // warp's, publishes the step's epoch to every rank (release stores, one lane per rank)
        // and waits until every rank's epoch has arrived here (one lane per sender), for at
        // most kWaitLimitNs.
        __syncwarp();
        int last = 0;
        if (lane == 0)
            last = atom_add_acq_rel_sys(p.peer.done, 1u) == gridDim.x * static_cast<unsigned int>(nwc) - 1u;
        last = __shfl_sync(0xffffffffu, last, 0);
        if (last) {
            if (lane == 0) *p.peer.done = 0;
            __syncwarp();
            if (lane < p.peer.n) st_release_sys(p.peer.flag_of[lane] + p.peer.rank, p.peer.epoch);
            const unsigned long long t0 = global_ns();
            for (;;) {
                const bool arrived =
                    lane >= p.peer.n || static_cast<int>(ld_acquire_sys(p.peer.flags + lane) - p.peer.epoch) >= 0;
                if (__all_sync(0xffffffffu, arrived)) break;
                if (global_ns() - t0 > kWaitLimitNs) {
                    if (lane == 0) atomicExch(p.peer.err, kErrTimeout);
                    break;
                }
            }
        }
    }
}

// One CTA per (split unit, KV head): combine the partials of every CTA that worked on it
// (the separate-launch merge; partials in tc_attn_kernel's lane-interleaved fragment order).
__global__ void merge_kernel(const MergeParams p) {
    const int e = blockIdx.x;
    const int h = blockIdx.y;
    const int u = p.split_u[e];
    const int c0 = p.split_c0[e];
    const int c1 = p.split_c1[e];
    const int seq = p.u_seq[u];
    const int row0 = p.offsets[seq] + p.u_t0[u];
    const int ncols = p.u_n[u] * p.g;
    for (int col = 0; col < ncols; ++col) {
        float mmax = -INFINITY;
        for (int c = c0; c <= c1; ++c) {
            const size_t idx = ((static_cast<size_t>(u) + c) * p.kvh + h) * kMaxCols + col;
            mmax = fmaxf(mmax, p.part_ml[idx * 2]);
        }
        float den = 0.f;
        for (int c = c0; c <= c1; ++c) {
            const size_t idx = ((static_cast<size_t>(u) + c) * p.kvh + h) * kMaxCols + col;
            den += exp2f(p.part_ml[idx * 2] - mmax) * p.part_ml[idx * 2 + 1];
        }
        const float inv = 1.f / den;
        float* op = p.out + (static_cast<size_t>(row0 + col / p.g) * p.H + h * p.g + col % p.g) * p.D;
        // column col, dim d: lane quad + 4 * grp, quad j = mt * NT + nt, element 2 * hi + e,
        // at float (j * 32 + lane) * 4 + element of the partial
        const int nt = col / 8, quad = (col % 8) / 2, ce = col & 1;
        for (int d = threadIdx.x; d < p.D; d += blockDim.x) {
            const int mt = d / 16, r = d % 16, grp = r & 7, hi = r >> 3;
            const int lane = quad + 4 * grp;
            const int vi = ((mt * p.nt + nt) * 32 + lane) * 4 + 2 * hi + ce;
            float num = 0.f;
            for (int c = c0; c <= c1; ++c) {
                const size_t sg = (static_cast<size_t>(u) + c) * p.kvh + h;
                const size_t idx = sg * kMaxCols + col;
                num += exp2f(p.part_ml[idx * 2] - mmax) * p.part_o[sg * kMaxCols * p.D + vi];
            }
            op[d] = num * inv;
        }
    }
}

template <int D, int NT>
cudaError_t launch_tc_t(const CUtensorMap* tmk, const CUtensorMap* tmv, const TcParams& p,
                        size_t smem, cudaStream_t st) {
    auto kern = tc_attn_kernel<D, NT>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    const int V = p.virt > 1 ? p.virt : 1;
    kern<<<(p.ncta + V - 1) / V, (p.kvh * V + 1) * 32, smem, st>>>(*tmk, *tmv, p);
    return cudaGetLastError();
}

}  // namespace

size_t tc_peer_stage_bytes(int D) {
    return 16 + static_cast<size_t>(kTcMaxKvHeads) * 4 * (D + 4) * sizeof(float);
}

size_t tc_smem_bytes(int D, int bs, int kvh, int stages, int virt) {
    // per virtual CTA: stages of K + V blocks, a full and an empty barrier per stage and the
    // end-of-work barrier; one merge barrier per consumer warp; the slack that aligns the base
    // to 1024 bytes
    return static_cast<size_t>(virt) * (static_cast<size_t>(stages) * 2 * bs * kvh * D * 2 +
                                         (2 * stages + 1) * sizeof(uint64_t)) +
           kTcMaxKvHeads * sizeof(uint64_t) + 1024;
}

cudaError_t launch_tc_attention(int D, int NT, const CUtensorMap* tmk, const CUtensorMap* tmv,
                                const TcParams& p, size_t smem, cudaStream_t st) {
    if (D == 64 && NT == 1) return launch_tc_t<64, 1>(tmk, tmv, p, smem, st);
    if (D == 64 && NT == 2) return launch_tc_t<64, 2>(tmk, tmv, p, smem, st);
    if (D == 128 && NT == 1) return launch_tc_t<128, 1>(tmk, tmv, p, smem, st);
    if (D == 128 && NT == 2) return launch_tc_t<128, 2>(tmk, tmv, p, smem, st);
    if (D == 256 && NT == 1) return launch_tc_t<256, 1>(tmk, tmv, p, smem, st);
    return cudaErrorInvalidValue;
}

cudaError_t launch_merge(const MergeParams& p, int nsplit, cudaStream_t st) {
    if (nsplit <= 0) return cudaSuccess;
    merge_kernel<<<dim3(nsplit, p.kvh), 128, 0, st>>>(p);
    return cudaGetLastError();
}

}  // namespace pk
