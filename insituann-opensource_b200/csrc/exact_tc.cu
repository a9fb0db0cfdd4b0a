// exact_tc.cu -- exact uint8 fine search on the tensor cores (tcgen05.mma
// kind::i8).
//
// The same work as exact_group_kernel (exact.cu): one CTA takes a list and up
// to 64 queries that probe it (a group of the work list), and every query
// keeps the k smallest keys (distance, original id) of the list.  q.x comes
// from the tensor cores: u8 x u8 products accumulated in s32 in tensor memory,
// exact (a row of d <= 256 bytes sums at most 256 * 255^2 < 2^31), so
// |q|^2 + |x|^2 - 2 q.x is the reference's integer sum of squared differences
// (updates/exact_update.cu:632-666, cpu_fine_kernels_v3_u8.cpp:356-595).
//
// A CTA is 10 warps:
//   warp 0, one lane   tensor copies: tiles of 128 list rows (d bytes each)
//                      into a ring of stages, 128-byte swizzled, through a
//                      tensor map over the index's rows in this GPU's memory
//                      (no multicast); rows past the list belong to the next
//                      list or lie past the tensor (read as zeros) and are
//                      masked by the epilogue;
//   warp 1             allocates tensor memory; one lane issues, per tile,
//                      d / 32 MMAs (M = 128 rows, N = 64 queries, K = 32)
//                      into one of 4 accumulators of 64 columns;
//   warps 2..9         epilogue: warp w reads the accumulator's lanes
//                      32 (w % 4) .. + 31 (tile rows) and columns
//                      32 ((w - 2) / 4) .. + 31 (queries); a key below its
//                      query's running k-th is staged in shared memory (one
//                      atomic per warp and query); a query whose staging area
//                      may not hold another tile, and every query after the
//                      list's last tile, merges its staged keys into its k
//                      smallest (one warp per 8 queries).
// The queries of a group sit in shared memory in the same swizzled layout
// (the MMA's B operand).  Every wait is bounded; a wait that gives up sets
// the error flag, the CTA drains its own copies and MMAs and returns.
#include <cstring>
#include <mutex>

#include "launch.h"
#include "tc.cuh"

namespace isb {

namespace {

constexpr int kTM = 128;               // list rows per tile (MMA M)
constexpr int kTQ = 64;                // queries per group (MMA N)
constexpr int kTAcc = 4;               // tensor-memory accumulators
constexpr int kTWarps = 10;
constexpr int kTThreads = 32 * kTWarps;
constexpr int kTEpi = 256;             // epilogue threads (warps 2..9)
constexpr int kTKMax = 16;             // largest k
constexpr int kTCap = 160;             // staged keys per query (>= 128 + 32)
constexpr int kTMaxStages = 6;

__host__ __device__ constexpr size_t exact_tc_fixed(int d) {
    return (size_t)kTQ * d                              // queries (B operand)
           + sizeof(uint64_t) * kTQ * kTKMax            // k smallest per query
           + sizeof(uint64_t) * kTQ * kTCap;            // staged keys
}

// stages of list tiles that fit beside the fixed arrays (1 KB kept for
// aligning the base to the swizzle atom)
__host__ __device__ inline int exact_tc_stages(int d) {
    const size_t cap = 227 * 1024 - 1024 - 2048;       // 2 KB of static shared memory aside
    const int st = (int)((cap - exact_tc_fixed(d)) / ((size_t)kTM * d));
    return st > kTMaxStages ? kTMaxStages : st;
}

__host__ __device__ inline size_t exact_tc_smem(int d) {
    return (size_t)exact_tc_stages(d) * kTM * d + exact_tc_fixed(d) + 1024;
}

// barrier of the 8 epilogue warps (named barrier 1)
__device__ __forceinline__ void epi_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kTEpi) : "memory"); }

// the same barrier, returning whether any epilogue thread passed v = true
__device__ __forceinline__ bool epi_sync_any(bool v) {
    uint32_t r;
    asm volatile(
        "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred q, 1, %2, p;\n selp.u32 %0, 1, 0, q;\n}"
        : "=r"(r)
        : "r"((uint32_t)v), "n"(kTEpi)
        : "memory");
    return r != 0;
}

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
    __shared__ uint32_t s_tmem;
    __shared__ int s_fail, s_item;
    __shared__ unsigned long long s_tau[kTQ];
    __shared__ int s_cnt[kTQ], s_qn[kTQ], s_qid[kTQ];
    const size_t tile_bytes = (size_t)kTM * d;
    unsigned char* sA = sm;
    unsigned char* sB = sm + (size_t)stages * tile_bytes;
    uint64_t* sTop = reinterpret_cast<uint64_t*>(sB + (size_t)kTQ * d);     // [kTQ][kTKMax]
    uint64_t* sStage = sTop + kTQ * kTKMax;                                  // [kTQ][kTCap]
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const volatile int* vfail = &s_fail;

    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                     "r"(kTAcc * kTQ)
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
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        s_fail = 0;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;
    const int NG = *wl.n_groups;
    int64_t gt = 0;             // tiles this CTA has started so far (mbarrier phases)
    int64_t issued = 0;         // warp 0: tiles whose copies were issued
    int64_t mma_done = 0;       // warp 1: tiles whose MMAs were issued

    for (;;) {
        if (tid == 0) s_item = s_fail ? NG : atomicAdd(counter, 1);
        __syncthreads();
        const int it = s_item;
        if (it >= NG) break;
        const int64_t pk = wl.groups[it];
        const int l = (int)(pk >> 32), p0 = (int)((pk >> 7) & 0x1FFFFFF), nqg = (int)(pk & 127);
        const int count = ls.counts[l];
        const int64_t off = ls.offsets[l];
        const int ntiles = (count + kTM - 1) / kTM;
        // the group's queries in the swizzled B layout (rows past nqg are zero)
        for (int e = tid; e < kTQ * 8 * NKB; e += kTThreads) {
            const int r = e / (8 * NKB), c = e % (8 * NKB), kb = c >> 3, cc = c & 7;
            uint4 v = make_uint4(0u, 0u, 0u, 0u);
            if (r < nqg) v = __ldg(reinterpret_cast<const uint4*>(q_u8 + (size_t)wl.pair_q[p0 + r] * d) + c);
            *reinterpret_cast<uint4*>(sB + (size_t)kb * kTQ * 128 + r * 128 + ((cc ^ (r & 7)) << 4)) = v;
        }
        if (tid < kTQ) {
            const int r = tid;
            const int q = r < nqg ? wl.pair_q[p0 + r] : -1;
            uint32_t n2 = 0;
            if (q >= 0) {
                const uint4* qr = reinterpret_cast<const uint4*>(q_u8 + (size_t)q * d);
#pragma unroll
                for (int c = 0; c < 8 * NKB; ++c) {
                    const uint4 v = __ldg(qr + c);
                    n2 = __dp4a(v.x, v.x, n2);
                    n2 = __dp4a(v.y, v.y, n2);
                    n2 = __dp4a(v.z, v.z, n2);
                    n2 = __dp4a(v.w, v.w, n2);
                }
            }
            s_qn[r] = (int)n2;
            s_qid[r] = q;
            s_cnt[r] = 0;
            // a query starts from its bound over the lists done so far (the k-th
            // of k keys already in its buffer): a key at or above it cannot be
            // among the query's k smallest
            s_tau[r] = q >= 0 ? *((volatile unsigned long long*)(cb.thr + q)) : kKeyNone;
        }
        for (int e = tid; e < kTQ * kTKMax; e += kTThreads) sTop[e] = kKeyNone;
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        tc_fence_before();
        __syncthreads();
        tc_fence_after();

        if (warp == 0) {
            if (lane == 0) {
                for (int t = 0; t < ntiles; ++t) {
                    const int64_t g = gt + t;
                    const int s = (int)(g % stages);
                    if (g >= stages && !mbar_wait_or(&bar_empty[s], (uint32_t)(((g / stages) - 1) & 1), vfail)) {
                        s_fail = 1;
                        break;
                    }
                    mbar_arrive_expect(&bar_full[s], (uint32_t)tile_bytes);
                    const int y = (int)(off + (int64_t)t * kTM);
#pragma unroll
                    for (int kb = 0; kb < NKB; ++kb)
                        tma_load_2d(sA + (size_t)s * tile_bytes + (size_t)kb * kTM * 128, &tmap, 128 * kb, y,
                                    &bar_full[s]);
                    issued = g + 1;
                }
            }
            __syncwarp();
        } else if (warp == 1) {
            if (lane == 0) {
                constexpr uint32_t idesc = umma_idesc_u8(kTM, kTQ);
                const uint32_t b_addr = smem_u32(sB);
                for (int t = 0; t < ntiles; ++t) {
                    const int64_t g = gt + t;
                    const int s = (int)(g % stages), a = (int)(g % kTAcc);
                    if (g >= kTAcc && !mbar_wait_or(&bar_ae[a], (uint32_t)(((g / kTAcc) - 1) & 1), vfail)) {
                        s_fail = 1;
                        break;
                    }
                    if (!mbar_wait_or(&bar_full[s], (uint32_t)((g / stages) & 1), vfail)) {
                        s_fail = 1;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(sA + (size_t)s * tile_bytes);
                    const uint32_t dacc = tmem + (uint32_t)(a * kTQ);
#pragma unroll
                    for (int kk = 0; kk < 4 * NKB; ++kk) {
                        // K block kk / 4 of the rows, 32 bytes kk % 4 inside its swizzled 128
                        const uint32_t ko = (uint32_t)(kk >> 2) * (kTM * 128) + (uint32_t)(kk & 3) * 32;
                        const uint32_t kq = (uint32_t)(kk >> 2) * (kTQ * 128) + (uint32_t)(kk & 3) * 32;
                        const uint64_t ad = umma_smem_desc_sw128(a_addr + ko);
                        const uint64_t bd = umma_smem_desc_sw128(b_addr + kq);
                        const uint32_t acc = kk ? 1u : 0u;
                        asm volatile(
                            "{\n .reg .pred pa;\n setp.ne.b32 pa, %4, 0;\n"
                            " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, pa;\n}" ::"r"(dacc),
                            "l"(ad), "l"(bd), "r"(idesc), "r"(acc)
                            : "memory");
                    }
                    tc_commit(&bar_empty[s]);
                    tc_commit(&bar_af[a]);
                    mma_done = g + 1;
                }
            }
            __syncwarp();
        } else {
            const int ew = warp - 2, quarter = warp & 3, half = ew >> 2;
            const int trow = quarter * 32 + lane;             // TMEM lane = tile row
            for (int t = 0; t < ntiles; ++t) {
                const int64_t g = gt + t;
                const int a = (int)(g % kTAcc);
                // this row's id and |x|^2 (a deleted position has id 0xFFFFFFFF: skipped)
                const int v = t * kTM + trow;
                uint32_t id = 0xFFFFFFFFu;
                int xn = 0;
                if (v < count) {
                    const int64_t pos = off + v;
                    if (!(ls.deleted && ls.deleted[pos])) id = ls.ids ? (uint32_t)ls.ids[pos] : (uint32_t)pos;
                    xn = ls.sqnorm[pos];
                }
                // a wait that gave up is acted on at the barrier after the filter,
                // which all epilogue warps reach (the values read are then discarded)
                const bool got = mbar_wait_or(&bar_af[a], (uint32_t)((g / kTAcc) & 1), vfail);
                tc_fence_after();
                uint32_t dot[32];
                tmem_ld32(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(a * kTQ + half * 32), dot);
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&bar_ae[a]);
                // keys below their query's k-th go to its staging area
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    const int r = half * 32 + i;
                    if (r >= nqg) break;
                    const uint32_t dist = (uint32_t)(s_qn[r] + xn) - 2u * dot[i];
                    const uint64_t key = make_key(dist, id);
                    const bool pass = id != 0xFFFFFFFFu && key < s_tau[r];
                    const unsigned ball = __ballot_sync(0xffffffffu, pass);
                    if (ball) {
                        int base = 0;
                        if (lane == 0) base = atomicAdd(&s_cnt[r], __popc(ball));
                        base = __shfl_sync(0xffffffffu, base, 0);
                        if (pass) sStage[r * kTCap + base + __popc(ball & ((1u << lane) - 1u))] = key;
                    }
                }
                if (epi_sync_any(!got)) {
                    if (tid == 64) s_fail = 1;
                    break;
                }
                // merges: a query whose staging area could overflow in the next
                // tile, and every query after the last tile
                const bool last = t == ntiles - 1;
                for (int rr = 0; rr < 8; ++rr) {
                    const int r = 8 * ew + rr;
                    if (r >= nqg) break;
                    const int ns = s_cnt[r];
                    if (ns == 0 || (!last && ns <= kTCap - kTM)) continue;
                    const int m = k + ns;
                    if (m <= 32) {
                        // lane i takes element i of (k smallest, staged) and writes it
                        // at its rank among all m, ties by element index
                        const uint64_t mine = lane < k ? sTop[r * kTKMax + lane]
                                                       : (lane < m ? sStage[r * kTCap + (lane - k)] : kKeyNone);
                        int rank = 0;
                        for (int j = 0; j < m; ++j) {
                            const uint64_t o = __shfl_sync(0xffffffffu, mine, j);
                            rank += (o < mine || (o == mine && j < lane)) ? 1 : 0;
                        }
                        __syncwarp();
                        if (lane < m && rank < k) sTop[r * kTKMax + rank] = mine;
                        if (lane < m && rank == k - 1 && mine != kKeyNone && mine < s_tau[r]) s_tau[r] = mine;
                    } else {
                        constexpr int E = (kTKMax + kTCap + 31) / 32;
                        uint64_t v6[E];
#pragma unroll
                        for (int e = 0; e < E; ++e) {
                            const int i = e * 32 + lane;
                            v6[e] = i < k ? sTop[r * kTKMax + i]
                                          : (i - k < ns ? sStage[r * kTCap + (i - k)] : kKeyNone);
                        }
                        uint64_t kth = kKeyNone;
                        for (int o = 0; o < k; ++o) {
                            const uint64_t mm = warp_take_min<E>(v6);
                            if (lane == o) sTop[r * kTKMax + o] = mm;
                            kth = mm;
                        }
                        __syncwarp();
                        if (lane == 0 && kth != kKeyNone && kth < s_tau[r]) s_tau[r] = kth;
                    }
                    __syncwarp();
                    if (lane == 0) s_cnt[r] = 0;
                }
                epi_sync();
            }
            // every query's k smallest keys of this list into its candidate buffer
            if (!*vfail) {
                for (int rr = 0; rr < 8; ++rr) {
                    const int r = 8 * ew + rr;
                    if (r >= nqg) break;
                    const uint64_t key = lane < k ? sTop[r * kTKMax + lane] : kKeyNone;
                    const bool ok = key != kKeyNone;
                    const unsigned ball = __ballot_sync(0xffffffffu, ok);
                    if (!ball) continue;
                    const int q = s_qid[r];
                    int base = 0;
                    if (lane == 0) {
                        base = atomicAdd(cb.cnt + q, __popc(ball));
                        const uint64_t kth = sTop[r * kTKMax + k - 1];
                        if (kth != kKeyNone) atomicMin(cb.thr + q, (unsigned long long)kth);
                    }
                    base = __shfl_sync(0xffffffffu, base, 0);
                    if (ok) {
                        const int at = base + __popc(ball & ((1u << lane) - 1u));
                        if (at < cb.cap) cb.keys[(size_t)q * cb.cap + at] = key;
                        else atomicExch(cb.overflow, 1);
                    }
                }
            }
        }
        gt += ntiles;
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        if (s_fail) break;
    }

    // drain: the copies and MMAs this CTA issued are complete before its shared
    // and tensor memory are released (only a wait that gave up leaves any)
    if (s_fail) {
        if (warp == 0 && lane == 0) {
            for (int64_t g = issued - stages > 0 ? issued - stages : 0; g < issued; ++g)
                mbar_wait(&bar_full[g % stages], (uint32_t)((g / stages) & 1));
        }
        if (warp == 1 && lane == 0 && mma_done > 0) {
            const int64_t g = mma_done - 1;
            mbar_wait(&bar_af[g % kTAcc], (uint32_t)((g / kTAcc) & 1));
        }
        if (tid == 0) atomicOr(flag, 4);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTAcc * kTQ)
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
    if (!rows || n <= 0 || n >= ((int64_t)1 << 31) - kTM || (d != 128 && d != 256) ||
        (reinterpret_cast<uintptr_t>(rows) & 15))
        return cudaErrorInvalidValue;
    EncodeTiledFn fn = encode_fn();
    if (!fn) return cudaErrorNotSupported;
    const cuuint64_t dims[2] = {(cuuint64_t)d, (cuuint64_t)n};
    const cuuint64_t strides[1] = {(cuuint64_t)d};
    const cuuint32_t box[2] = {128, (cuuint32_t)kTM};
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
