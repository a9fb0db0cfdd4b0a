// exact_tc.cu -- exact uint8 fine search on the tensor cores (tcgen05.mma
// kind::i8).
//
// The same work as exact_group_kernel (exact.cu): one CTA takes a list and up
// to 127 queries that probe it (a group of the work list), and every query
// keeps the k smallest keys (distance, original id) of the list.  q.x comes
// from the tensor cores: u8 x u8 products accumulated in s32 in tensor memory,
// exact (a row of d <= 256 bytes sums at most 256 * 255^2 < 2^31), so
// |q|^2 + |x|^2 - 2 q.x is the reference's integer sum of squared differences
// (updates/exact_update.cu:632-666, cpu_fine_kernels_v3_u8.cpp:356-595).
//
// The MMA has the group's queries as M (128 rows of A, in shared memory) and
// a tile of 128 list rows as N (B), so accumulator lane i holds query i's dot
// products with the tile's rows: each epilogue thread owns one query and half
// of the tile's columns and keeps that query's k smallest keys in registers,
// with no exchange between threads until the list is done.
//
// A CTA is 10 warps, working on up to two groups at once (two query slots):
//   warp 0             claims the next group, stages its queries (the MMA's
//                      A operand), their norms and bounds into a free slot
//                      while the epilogue still works on the previous group;
//                      one lane issues the tensor copies: tiles of 128 list
//                      rows (d bytes each)
//                      into a ring of stages, 128-byte swizzled, through a
//                      tensor map over the index's rows in this GPU's memory
//                      (no multicast); rows past the list belong to the next
//                      list or lie past the tensor (read as zeros) and are
//                      masked by the epilogue;
//   warp 1             allocates tensor memory; one lane issues, per tile,
//                      d / 32 MMAs (M = 128 queries, N = 128 rows, K = 32)
//                      into one of 2 accumulators of 128 columns;
//   warps 2..9         epilogue: warp w reads lanes 32 (w % 4) .. + 31
//                      (queries) and columns 64 ((w - 2) / 4) .. + 63 (tile
//                      rows); a row whose distance is at most the query's
//                      running k-th (or its bound from lists done before) is
//                      kept in the thread's slots in shared memory, and the
//                      slots are then inserted into the thread's sorted k
//                      smallest (a compare-exchange chain in registers).
// After the list's last tile the two threads of a query merge their k
// smallest and append them to the query's candidate buffer.  Keys are ranked
// by (distance, position) while scanning: a list's rows are stored in
// increasing original id, so within a list that is the (distance, id) order.
// Every wait is bounded; a wait that gives up sets the error flag, the CTA
// drains its own copies and MMAs and returns.
#include <cstring>
#include <mutex>

#include "launch.h"
#include "tc.cuh"

namespace isb {

namespace {

constexpr int kTQ = 128;               // queries per group (MMA M; groups hold up to 127)
constexpr int kTN = 128;               // list rows per tile (MMA N)
constexpr int kTAcc = 2;               // tensor-memory accumulators of kTN columns
constexpr int kTWarps = 10;
constexpr int kTThreads = 32 * kTWarps;
constexpr int kTEpi = 256;             // epilogue threads (warps 2..9)
constexpr int kTKMax = 16;             // largest k
constexpr int kTSlots = 32;            // kept rows per thread between insertions
constexpr int kTMaxStages = 6;

__host__ __device__ constexpr size_t exact_tc_fixed(int d) {
    return 2 * (size_t)kTQ * d                          // queries of two groups (A operand)
           + sizeof(uint32_t) * kTSlots * kTEpi         // kept rows (also the final exchange)
           + sizeof(uint2) * 8 * 64;                    // per epilogue warp: its rows' |x|^2 and position
}

// stages of list tiles that fit beside the fixed arrays (1 KB kept for
// aligning the base to the swizzle atom, 4 KB for static shared memory)
__host__ __device__ inline int exact_tc_stages(int d) {
    const size_t cap = 227 * 1024 - 1024 - 4096;
    const int st = (int)((cap - exact_tc_fixed(d)) / ((size_t)kTN * d));
    return st > kTMaxStages ? kTMaxStages : st;
}

__host__ __device__ inline size_t exact_tc_smem(int d) {
    return (size_t)exact_tc_stages(d) * kTN * d + exact_tc_fixed(d) + 1024;
}

// barrier of the 8 epilogue warps (named barrier 1)
__device__ __forceinline__ void epi_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kTEpi) : "memory"); }

// the same barrier, returning whether any epilogue thread passed v = true
// (so that all epilogue warps take the same branch after a bounded wait)
__device__ __forceinline__ bool epi_sync_any(bool v) {
    uint32_t r;
    asm volatile(
        "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred q, 1, %2, p;\n selp.u32 %0, 1, 0, q;\n}"
        : "=r"(r)
        : "r"((uint32_t)v), "n"(kTEpi)
        : "memory");
    return r != 0;
}

// inserts key into the ascending list lv (one compare-exchange per slot; the
// list's first kTKMax - k slots hold 0 and never move)
__device__ __forceinline__ void topk_insert(uint64_t (&lv)[kTKMax], uint64_t key) {
#pragma unroll
    for (int e = 0; e < kTKMax; ++e) {
        const uint64_t a = lv[e];
        const bool lt = key < a;
        lv[e] = lt ? key : a;
        key = lt ? a : key;
    }
}

// One group in flight per slot (two slots): what the copy warp decoded and
// staged for it, read by the MMA thread and the epilogue.
struct TcGroup {
    int64_t off;     // first position of the list
    int count;       // rows of the list
    int nqg;         // queries of the group (0: no more groups)
};

template <int NKB>   // 128-byte K blocks per row: d = 128 NKB
__global__ void __launch_bounds__(kTThreads, 1)
    exact_tc_kernel(const __grid_constant__ CUtensorMap tmap, const uint8_t* __restrict__ q_u8, ListStore ls,
                    WorkList wl, CandBuf cb, int k, int stages, int* counter, int* flag) {
    constexpr int d = 128 * NKB;
    extern __shared__ unsigned char sm_raw[];
    unsigned char* sm =
        reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(sm_raw) + 1023) & ~uintptr_t(1023));
    __shared__ __align__(8) uint64_t bar_full[kTMaxStages];
    __shared__ __align__(8) uint64_t bar_empty[kTMaxStages];
    __shared__ __align__(8) uint64_t bar_af[kTAcc];
    __shared__ __align__(8) uint64_t bar_ae[kTAcc];
    __shared__ __align__(8) uint64_t bar_qready[2];   // a slot's queries and descriptor are staged
    __shared__ __align__(8) uint64_t bar_qfree[2];    // the MMAs and the epilogue are done with a slot
    __shared__ uint32_t s_tmem;
    __shared__ int s_fail;
    __shared__ TcGroup s_grp[2];
    __shared__ int s_qn[2][kTQ], s_qid[2][kTQ];
    __shared__ uint32_t s_tau[2][kTQ];
    const size_t tile_bytes = (size_t)kTN * d;
    const size_t a_bytes = (size_t)kTQ * d;
    unsigned char* sA0 = sm + (size_t)stages * tile_bytes;                      // queries [2][kTQ][d], swizzled
    uint32_t* sSlot = reinterpret_cast<uint32_t*>(sA0 + 2 * a_bytes);           // [kTSlots][kTEpi]
    uint2* sRow = reinterpret_cast<uint2*>(sSlot + kTSlots * kTEpi);            // [8 warps][64]
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const volatile int* vfail = &s_fail;

    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                     "r"(kTAcc * kTN)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (tid == 0) {
        for (int s = 0; s < stages; ++s) {
            mbar_init(&bar_full[s], 1);
            mbar_init(&bar_empty[s], 1);
        }
        for (int a = 0; a < kTAcc; ++a) {
            mbar_init(&bar_af[a], 1);
            mbar_init(&bar_ae[a], kTEpi / 32);     // one arrival per epilogue warp
        }
        for (int q = 0; q < 2; ++q) {
            mbar_init(&bar_qready[q], 1);
            mbar_init(&bar_qfree[q], 1 + kTEpi / 32);   // the MMA thread's commit + each epilogue warp
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        s_fail = 0;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;
    const int NG = *wl.n_groups;

    if (warp == 0) {
        // ---- copy warp: claims the groups, stages their queries (all lanes), and
        // issues the list tiles (lane 0) ----
        int64_t gt = 0;          // tiles issued so far
        for (int gi = 0;; ++gi) {
            const int slot = gi & 1;
            if (gi >= 2 && !mbar_wait_timed(&bar_qfree[slot], (uint32_t)(((gi >> 1) - 1) & 1), vfail)) {
                if (lane == 0) s_fail = 1;
                break;
            }
            int it = 0;
            if (lane == 0) it = *vfail ? NG : atomicAdd(counter, 1);
            it = __shfl_sync(0xffffffffu, it, 0);
            TcGroup grp{0, 0, 0};
            int p0 = 0;
            if (it < NG) {
                const int64_t pk = wl.groups[it];
                const int l = (int)(pk >> 32);
                p0 = (int)((pk >> 7) & 0x1FFFFFF);
                grp.nqg = (int)(pk & 127);
                grp.count = ls.counts[l];
                grp.off = ls.offsets[l];
            }
            unsigned char* sA = sA0 + (size_t)slot * a_bytes;
            if (grp.nqg > 0) {
                // the group's queries in the swizzled A layout by asynchronous 16-byte
                // copies, all in flight at once (rows past nqg are zero); lane L
                // stages rows L, L + 32, ... and keeps their query ids
                int qids[kTQ / 32];
#pragma unroll
                for (int i = 0; i < kTQ / 32; ++i) {
                    const int r = lane + 32 * i;
                    qids[i] = r < grp.nqg ? wl.pair_q[p0 + r] : -1;
                }
#pragma unroll
                for (int i = 0; i < kTQ / 32; ++i) {
                    const int r = lane + 32 * i;
#pragma unroll
                    for (int c = 0; c < 8 * NKB; ++c) {
                        unsigned char* dst = sA + (size_t)(c >> 3) * kTQ * 128 + r * 128 + (((c & 7) ^ (r & 7)) << 4);
                        if (qids[i] >= 0)
                            asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)),
                                         "l"(q_u8 + (size_t)qids[i] * d + 16 * c)
                                         : "memory");
                        else
                            *reinterpret_cast<uint4*>(dst) = make_uint4(0u, 0u, 0u, 0u);
                    }
                }
                // the bounds over the lists done before (a key above the bound cannot be
                // among the query's k smallest), read while the copies land
                uint32_t taus[kTQ / 32];
#pragma unroll
                for (int i = 0; i < kTQ / 32; ++i)
                    taus[i] = qids[i] >= 0 ? (uint32_t)(*((volatile unsigned long long*)(cb.thr + qids[i])) >> 32)
                                           : 0xFFFFFFFFu;
                asm volatile("cp.async.wait_all;" ::: "memory");
                // |q|^2 of this lane's rows, from the staged copy
#pragma unroll
                for (int i = 0; i < kTQ / 32; ++i) {
                    const int r = lane + 32 * i;
                    uint32_t n2 = 0;
#pragma unroll
                    for (int c = 0; c < 8 * NKB; ++c) {
                        const uint4 v = *reinterpret_cast<const uint4*>(sA + (size_t)(c >> 3) * kTQ * 128 + r * 128 +
                                                                       (((c & 7) ^ (r & 7)) << 4));
                        n2 = __dp4a(v.x, v.x, n2);
                        n2 = __dp4a(v.y, v.y, n2);
                        n2 = __dp4a(v.z, v.z, n2);
                        n2 = __dp4a(v.w, v.w, n2);
                    }
                    s_qn[slot][r] = (int)n2;
                    s_qid[slot][r] = qids[i];
                    s_tau[slot][r] = taus[i];
                }
            }
            if (lane == 0) s_grp[slot] = grp;
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(&bar_qready[slot]);
            if (grp.nqg == 0) break;
            if (lane == 0) {
                const int ntiles = (grp.count + kTN - 1) / kTN;
                for (int t = 0; t < ntiles; ++t, ++gt) {
                    const int s = (int)(gt % stages);
                    if (gt >= stages && !mbar_wait_timed(&bar_empty[s], (uint32_t)(((gt / stages) - 1) & 1), vfail)) {
                        s_fail = 1;
                        break;
                    }
                    mbar_arrive_expect(&bar_full[s], (uint32_t)tile_bytes);
                    const int y = (int)(grp.off + (int64_t)t * kTN);
#pragma unroll
                    for (int kb = 0; kb < NKB; ++kb)
                        tma_load_2d(sm + (size_t)s * tile_bytes + (size_t)kb * kTN * 128, &tmap, 128 * kb, y,
                                    &bar_full[s]);
                }
            }
            __syncwarp();
            if (*vfail) break;
        }
        // the copies in flight land before the CTA's shared memory is released
        if (lane == 0)
            for (int64_t g = gt - stages > 0 ? gt - stages : 0; g < gt; ++g)
                mbar_wait_timed(&bar_full[g % stages], (uint32_t)((g / stages) & 1), nullptr);
    } else if (warp == 1) {
        // ---- MMA thread ----
        if (lane == 0) {
            constexpr uint32_t idesc = umma_idesc_u8(kTQ, kTN);
            int64_t gt = 0;
            for (int gi = 0;; ++gi) {
                const int slot = gi & 1;
                if (!mbar_wait_timed(&bar_qready[slot], (uint32_t)((gi >> 1) & 1), vfail)) {
                    s_fail = 1;
                    break;
                }
                const TcGroup grp = s_grp[slot];
                if (grp.nqg == 0) break;
                const uint32_t a_addr = smem_u32(sA0 + (size_t)slot * a_bytes);
                const int ntiles = (grp.count + kTN - 1) / kTN;
                bool ok = true;
                for (int t = 0; t < ntiles; ++t, ++gt) {
                    const int s = (int)(gt % stages), a = (int)(gt % kTAcc);
                    if ((gt >= kTAcc && !mbar_wait_timed(&bar_ae[a], (uint32_t)(((gt / kTAcc) - 1) & 1), vfail)) ||
                        !mbar_wait_timed(&bar_full[s], (uint32_t)((gt / stages) & 1), vfail)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t b_addr = smem_u32(sm + (size_t)s * tile_bytes);
                    const uint32_t dacc = tmem + (uint32_t)(a * kTN);
#pragma unroll
                    for (int kk = 0; kk < 4 * NKB; ++kk) {
                        // K block kk / 4, 32 bytes kk % 4 inside its swizzled 128
                        const uint32_t ka = (uint32_t)(kk >> 2) * (kTQ * 128) + (uint32_t)(kk & 3) * 32;
                        const uint32_t kr = (uint32_t)(kk >> 2) * (kTN * 128) + (uint32_t)(kk & 3) * 32;
                        const uint64_t ad = umma_smem_desc_sw128(a_addr + ka);
                        const uint64_t bd = umma_smem_desc_sw128(b_addr + kr);
                        const uint32_t acc = kk ? 1u : 0u;
                        asm volatile(
                            "{\n .reg .pred pa;\n setp.ne.b32 pa, %4, 0;\n"
                            " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, pa;\n}" ::"r"(dacc),
                            "l"(ad), "l"(bd), "r"(idesc), "r"(acc)
                            : "memory");
                    }
                    tc_commit(&bar_empty[s]);
                    tc_commit(&bar_af[a]);
                }
                if (!ok) {
                    s_fail = 1;
                    break;
                }
                tc_commit(&bar_qfree[slot]);      // the slot's queries are no longer read
            }
            // the MMAs in flight are done before tensor memory is released
            if (gt > 0) mbar_wait_timed(&bar_af[(gt - 1) % kTAcc], (uint32_t)(((gt - 1) / kTAcc) & 1), nullptr);
        }
        __syncwarp();
    } else {
        // ---- epilogue ----
        const int ew = warp - 2, quarter = warp & 3, half = ew >> 2;
        const int qi = quarter * 32 + lane;               // TMEM lane = the thread's query
        uint2* myrows = sRow + ew * 64;
        uint32_t* myslot = sSlot + (tid - 64);             // slot c at [c][kTEpi]
        int64_t gt = 0;
        for (int gi = 0;; ++gi) {
            const int slot = gi & 1;
            const bool ready = mbar_wait_timed(&bar_qready[slot], (uint32_t)((gi >> 1) & 1), vfail);
            if (epi_sync_any(!ready)) {                    // every epilogue warp leaves together
                if (tid == 64) s_fail = 1;
                break;
            }
            const TcGroup grp = s_grp[slot];
            if (grp.nqg == 0) break;
            const int count = grp.count;
            const int64_t off = grp.off;
            const int ntiles = (count + kTN - 1) / kTN;
            const bool live = qi < grp.nqg;
            const int q = s_qid[slot][qi];
            const uint32_t qn = (uint32_t)s_qn[slot][qi];
            const uint32_t tau = s_tau[slot][qi];
            uint64_t lv[kTKMax];
#pragma unroll
            for (int i = 0; i < kTKMax; ++i) lv[i] = i < kTKMax - k ? 0ull : kKeyNone;
            uint32_t lim = tau;                                // distances above it are not kept
            // |x|^2 and position of this warp's 64 rows of tile t (0xFFFFFFFF: past the
            // list or deleted), read one tile ahead
            auto row_info = [&](int t, int h) {
                const int v = t * kTN + half * 64 + 32 * h + lane;
                uint2 rw = make_uint2(0u, 0xFFFFFFFFu);
                if (v < count) {
                    const int64_t pos = off + v;
                    if (!(ls.deleted && ls.deleted[pos])) rw = make_uint2((uint32_t)ls.sqnorm[pos], (uint32_t)pos);
                }
                return rw;
            };
            // a warp none of whose 32 queries is in the group only hands the
            // accumulators back (after they are written, to keep the phases)
            const bool warp_live = __any_sync(0xffffffffu, live);
            uint2 nrw0 = make_uint2(0u, 0xFFFFFFFFu), nrw1 = nrw0;
            if (warp_live) {
                nrw0 = row_info(0, 0);
                nrw1 = row_info(0, 1);
            }
            bool ok = true;
            for (int t = 0; t < ntiles; ++t, ++gt) {
                const int a = (int)(gt % kTAcc);
                const bool got = mbar_wait_timed(&bar_af[a], (uint32_t)((gt / kTAcc) & 1), vfail);
                if (!__all_sync(0xffffffffu, got)) {
                    ok = false;
                    break;
                }
                if (!warp_live) {
                    tc_fence_after();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&bar_ae[a]);
                    continue;
                }
                myrows[lane] = nrw0;
                myrows[32 + lane] = nrw1;
                if (t + 1 < ntiles) {
                    nrw0 = row_info(t + 1, 0);
                    nrw1 = row_info(t + 1, 1);
                }
                tc_fence_after();
                uint32_t dot[2][32];
                const uint32_t ta = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(a * kTN + half * 64);
                tmem_ld32(ta, dot[0]);
                tmem_ld32(ta + 32, dot[1]);
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&bar_ae[a]);
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    // rows within the limit go to the slots, then into the k smallest
                    int nk = 0;
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        const uint2 rw = myrows[32 * h + j];
                        const uint32_t dist = qn + rw.x - 2u * dot[h][j];
                        if (live && rw.y != 0xFFFFFFFFu && dist <= lim) {
                            myslot[nk * kTEpi] = (dist << 6) | (uint32_t)(32 * h + j);
                            ++nk;
                        }
                    }
                    for (int c = 0; c < nk; ++c) {
                        const uint32_t e = myslot[c * kTEpi];
                        const uint64_t key = make_key(e >> 6, myrows[e & 63].y);
                        if (key < lv[kTKMax - 1]) topk_insert(lv, key);
                    }
                    const uint32_t kd = (uint32_t)(lv[kTKMax - 1] >> 32);
                    lim = kd < tau ? kd : tau;
                }
                __syncwarp();                              // the rows of the next tile overwrite myrows
            }
            if (!ok) {
                if (lane == 0) s_fail = 1;
            }
            // the two threads of a query: half 1 hands its k smallest to half 0,
            // which merges them and appends the result to the query's buffer
            epi_sync();
            uint64_t* xch = reinterpret_cast<uint64_t*>(sSlot);      // [kTQ][kTKMax]
            if (half == 1) {
#pragma unroll
                for (int i = 0; i < kTKMax; ++i) xch[qi * kTKMax + i] = lv[i];
            }
            epi_sync();
            if (half == 0 && live && !*vfail) {
                for (int i = kTKMax - k; i < kTKMax; ++i) {
                    const uint64_t o = xch[qi * kTKMax + i];
                    if (o >= lv[kTKMax - 1]) break;              // the other list is ascending
                    topk_insert(lv, o);
                }
                // the list's keys are slots kTKMax - k .. kTKMax - k + nk - 1 (ascending);
                // the slots are indexed statically so that lv stays in registers
                int nk = 0;
#pragma unroll
                for (int i = 0; i < kTKMax; ++i) nk += (i >= kTKMax - k && lv[i] != kKeyNone) ? 1 : 0;
                if (nk > 0) {
                    const int base = atomicAdd(cb.cnt + q, nk);
#pragma unroll
                    for (int i = 0; i < kTKMax; ++i) {
                        const int r = i - (kTKMax - k);
                        if (r < 0 || r >= nk) continue;
                        const uint64_t kp = lv[i];
                        const uint32_t pos = (uint32_t)kp;
                        const uint64_t key = make_key((uint32_t)(kp >> 32), ls.ids ? (uint32_t)ls.ids[pos] : pos);
                        if (base + r < cb.cap) cb.keys[(size_t)q * cb.cap + base + r] = key;
                        else atomicExch(cb.overflow, 1);
                        // k keys of this list: their k-th bounds the query's k smallest
                        if (r == k - 1) atomicMin(cb.thr + q, (unsigned long long)key);
                    }
                }
            }
            epi_sync();                                    // xch is free for the next group
            if (lane == 0) mbar_arrive(&bar_qfree[slot]);
            // (a failure seen now ends the loop at the next group's collective check)
        }
    }

    __syncthreads();
    if (s_fail && tid == 0) atomicOr(flag, 4);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTAcc * kTN)
                     : "memory");
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link
// against the driver library)
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
        else
            cudaGetLastError();
    });
    return fn;
}

}  // namespace

bool exact_tc_usable(int d, int k) { return (d == 128 || d == 256) && k > 0 && k <= kTKMax; }

cudaError_t exact_tc_map(const uint8_t* rows, int64_t n, int d, void* map_out) {
    if (!rows || n <= 0 || n >= ((int64_t)1 << 31) - kTN || (d != 128 && d != 256) ||
        (reinterpret_cast<uintptr_t>(rows) & 15))
        return cudaErrorInvalidValue;
    EncodeTiledFn fn = encode_fn();
    if (!fn) return cudaErrorNotSupported;
    const cuuint64_t dims[2] = {(cuuint64_t)d, (cuuint64_t)n};
    const cuuint64_t strides[1] = {(cuuint64_t)d};
    const cuuint32_t box[2] = {128, (cuuint32_t)kTN};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = fn(static_cast<CUtensorMap*>(map_out), CU_TENSOR_MAP_DATA_TYPE_UINT8, 2,
                          const_cast<uint8_t*>(rows), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

cudaError_t exact_tc_scan(const void* map, const uint8_t* q_u8, int d, int k, ListStore ls, WorkList wl,
                          int max_groups, CandBuf cb, int* work_counter, int* flag, cudaStream_t st) {
    if (!exact_tc_usable(d, k) || !wl.groups || !ls.sqnorm || !map) return cudaErrorInvalidValue;
    if (max_groups <= 0) return cudaSuccess;
    cudaError_t e = cudaMemsetAsync(work_counter, 0, sizeof(int), st);
    if (e) return e;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int stages = exact_tc_stages(d);
    const size_t smem = exact_tc_smem(d);
    if (stages < 2) return cudaErrorInvalidConfiguration;
    CUtensorMap tmap;
    memcpy(&tmap, map, sizeof(tmap));
    auto go = [&](auto kern) {
        cudaError_t e2 = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e2) return e2;
        const int grid = sms < max_groups ? sms : max_groups;
        note_launch();
        kern<<<grid, kTThreads, smem, st>>>(tmap, q_u8, ls, wl, cb, k, stages, work_counter, flag);
        return cudaGetLastError();
    };
    return d == 128 ? go(exact_tc_kernel<1>) : go(exact_tc_kernel<2>);
}

}  // namespace isb
