// route_tc.cu -- coarse routing on the tensor cores (tcgen05) with exact rescoring.
//
// The routing result is defined by the exact fp32 direct-difference distance
// sum_j (q_j - c_j)^2 (route.cu).  This file gets the same top-nprobe lists
// faster in two steps:
//
//  1. route_tc_kernel: an approximate distance of every (query, centroid)
//     pair, D~ = ||q||^2 + ||c||^2 - 2 q.c, with q.c from one tcgen05 GEMM.
//     Each fp32 value x is split into bf16 parts hi = bf16(x), lo =
//     bf16(x - hi); the GEMM runs over K' = 3d with A = [q_hi | q_hi | q_lo]
//     and B = [c_hi | c_lo | c_hi], i.e. q_hi.c_hi + q_hi.c_lo + q_lo.c_hi,
//     accumulated in fp32 in tensor memory.  A CTA owns 128 queries (the MMA
//     M), stages their operand once, streams 64-centroid operand tiles into
//     shared memory with bulk async copies (two buffers), issues the MMAs
//     from one thread into two alternating accumulators, and its 4 warps read
//     each accumulator back (one query row per TMEM lane) and write D~ bits.
//  2. route_rescore_kernel: per query, the nprobe-th smallest D~ (T~), every
//     centroid with D~ <= T~ + 2 eps is a candidate, where eps = 2^-11
//     (||q||^2 + max ||c||^2) bounds |D~ - D| for every centroid (the split
//     leaves a relative error near 2^-16 in q.c, the fp32 accumulation of 3d
//     products less than 2^-14; the bound keeps a factor 4 of margin).  The
//     candidates are rescored with the exact distance and their top-nprobe
//     by (distance, list id) is the result -- the same set as the exact
//     routing, because every centroid of the exact top-nprobe has
//     D~ <= T~ + 2 eps.  A query with more candidates than fit is rescored
//     over all centroids.
//
// Shared-memory operands use the canonical K-major layout without swizzle:
// 8-row x 16-byte core matrices, the two 8-element halves of one MMA's K = 16
// 128 bytes apart (LBO), consecutive 8-row groups 256 bytes apart (SBO), and
// the K blocks of 16 one after another.
#include <cuda_bf16.h>

#include "launch.h"
#include "tc.cuh"

namespace isb {

namespace {

constexpr int kTCM = 128;                 // queries per CTA (MMA M)
constexpr int kTCN = 64;                  // centroids per tile (MMA N)
constexpr int kTCThreads = 128;           // 4 warps: one TMEM lane (query row) per thread
constexpr int kPMaxRouteD = 512;          // largest d of the fallback rows

__device__ __forceinline__ uint32_t bf16_bits(__nv_bfloat16 h) { return (uint32_t)__bfloat16_as_ushort(h); }

// the 8 bf16 of chunk k8 of the split row [x_hi | x_hi | x_lo] (hi_lo_hi = false)
// or [x_hi | x_lo | x_hi] (hi_lo_hi = true) of the fp32 row x[d]; d % 16 == 0,
// so a chunk never straddles two parts
__device__ __forceinline__ uint4 split_chunk(const float* x, int d, int k8, bool valid_row, bool hi_lo_hi) {
    const int k = 8 * k8, part = k / d, j0 = k - part * d;
    const bool lo = hi_lo_hi ? part == 1 : part == 2;
    uint32_t w[4];
#pragma unroll
    for (int e = 0; e < 8; e += 2) {
        uint32_t pair = 0;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const float v = valid_row ? x[j0 + e + h] : 0.f;
            const __nv_bfloat16 hi = __float2bfloat16_rn(v);
            const __nv_bfloat16 out = lo ? __float2bfloat16_rn(v - __bfloat162float(hi)) : hi;
            pair |= bf16_bits(out) << (16 * h);
        }
        w[e / 2] = pair;
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
}

// centroid operand tiles [ntiles][64 x 3d] in the canonical layout, split
// [hi | lo | hi]; squared norms cn, and cne = cn for valid lists, +inf for
// invalid lists and the padding rows of the last tile
__global__ void route_tc_prepare_kernel(const float* __restrict__ cent, const uint8_t* __restrict__ valid, int nlist,
                                        int d, uint16_t* __restrict__ ops, float* __restrict__ cn,
                                        float* __restrict__ cne) {
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    const size_t t0 = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
    const int NT = kTCN, K8 = 3 * d / 8;
    const int ntiles = (nlist + NT - 1) / NT;
    const size_t tile_bytes = (size_t)NT * 3 * d * 2;
    for (size_t e = t0; e < (size_t)ntiles * NT * K8; e += stride) {
        const int t = (int)(e / ((size_t)NT * K8));
        const int r = (int)((e / K8) % NT), k8 = (int)(e % K8);
        const int c = t * NT + r;
        const bool ok = c < nlist && valid[c];
        const uint4 v = split_chunk(cent + (size_t)(ok ? c : 0) * d, d, k8, ok, true);
        *reinterpret_cast<uint4*>(reinterpret_cast<unsigned char*>(ops) + (size_t)t * tile_bytes +
                                  tc_chunk_off(r, k8, NT)) = v;
    }
    for (size_t c = t0; c < (size_t)ntiles * NT; c += stride) {
        float s = __int_as_float(0x7f800000);
        if (c < (size_t)nlist) {
            s = 0.f;
            for (int j = 0; j < d; ++j) s = __fadd_rn(s, __fmul_rn(cent[c * d + j], cent[c * d + j]));
            cn[c] = s;
        }
        cne[c] = c < (size_t)nlist && valid[c] ? s : __int_as_float(0x7f800000);   // +inf: never a candidate
    }
}

__global__ void route_tc_cnmax_kernel(const float* __restrict__ cn, const uint8_t* __restrict__ valid, int nlist,
                                      float* __restrict__ cn_max) {
    __shared__ float red[256];
    float m = 0.f;
    for (int c = threadIdx.x; c < nlist; c += blockDim.x)
        if (valid[c]) m = fmaxf(m, cn[c]);
    red[threadIdx.x] = m;
    __syncthreads();
    for (int s = blockDim.x / 2; s > 0; s >>= 1) {
        if (threadIdx.x < s) red[threadIdx.x] = fmaxf(red[threadIdx.x], red[threadIdx.x + s]);
        __syncthreads();
    }
    if (threadIdx.x == 0) *cn_max = red[0];
}

// One CTA: 128 queries x a range of 64-centroid tiles.  Tensor memory holds
// two 128 x 64 fp32 accumulators: the MMAs of tile t+1 run while the 4 warps
// read tile t back.  Each warp moves its 32 rows x 32 columns through a
// padded shared-memory square so that the distance stores are 128-byte rows
// (one query, 32 consecutive lists per warp store).
constexpr int kTCStage = 32 * 33;         // floats of one warp's transpose square

__host__ __device__ constexpr size_t route_tc_smem(int d) {
    return (size_t)kTCM * 3 * d * 2 + 2 * (size_t)kTCN * 3 * d * 2 + sizeof(float) * (4 * kTCStage + kTCM);
}

__global__ void __launch_bounds__(kTCThreads, 1)
    route_tc_kernel(const float* __restrict__ q, int nq, int d, const uint16_t* __restrict__ ops,
                    const float* __restrict__ cn, const uint8_t* __restrict__ valid, int nlist, int tiles_per_cta,
                    uint32_t* __restrict__ out, int* flag) {
    extern __shared__ __align__(1024) unsigned char sm[];
    __shared__ __align__(8) uint64_t bar_b[2];
    __shared__ __align__(8) uint64_t bar_mma[2];
    __shared__ uint32_t s_tmem;
    __shared__ int s_fail;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int K = 3 * d, K8 = K / 8;
    const uint32_t a_bytes = (uint32_t)kTCM * K * 2, b_bytes = (uint32_t)kTCN * K * 2;
    unsigned char* sA = sm;
    unsigned char* sB = sm + a_bytes;                                      // [2][b_bytes]
    float* stage = reinterpret_cast<float*>(sB + 2 * (size_t)b_bytes);      // [4][32][33]
    float* s_qn = stage + 4 * kTCStage;                                    // [128]
    const int q0 = blockIdx.x * kTCM;
    const int ntiles = (nlist + kTCN - 1) / kTCN;
    const int t_begin = blockIdx.y * tiles_per_cta;
    const int t_end = min(ntiles, t_begin + tiles_per_cta);
    const int n = t_end - t_begin;
    if (n <= 0) return;                                    // the whole CTA leaves together

    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                     "r"(2 * kTCN)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (tid == 0) {
        mbar_init(&bar_b[0], 1);
        mbar_init(&bar_b[1], 1);
        mbar_init(&bar_mma[0], 1);
        mbar_init(&bar_mma[1], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        s_fail = 0;
    }
    // this thread's query row of A and its squared norm (used by D~ only)
    const int qi = q0 + tid;
    const bool qok = qi < nq;
    const float* qr = q + (size_t)(qok ? qi : 0) * d;
    float qn = 0.f;
    if (qok)
        for (int j = 0; j < d; ++j) qn = __fadd_rn(qn, __fmul_rn(qr[j], qr[j]));
    s_qn[tid] = qn;
    for (int k8 = 0; k8 < K8; ++k8)
        *reinterpret_cast<uint4*>(sA + tc_chunk_off(tid, k8, kTCM)) = split_chunk(qr, d, k8, qok, false);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = s_tmem;
    const unsigned char* gops = reinterpret_cast<const unsigned char*>(ops);
    constexpr uint32_t idesc = umma_idesc_bf16(kTCM, kTCN);
    const uint32_t a_addr = smem_u32(sA);
    // thread 0: copy tile i of this CTA into buffer i & 1
    auto copy_tile = [&](int i) {
        mbar_arrive_expect(&bar_b[i & 1], b_bytes);
        bulk_g2s(sB + (size_t)(i & 1) * b_bytes, gops + (size_t)(t_begin + i) * b_bytes, b_bytes, &bar_b[i & 1]);
    };
    // thread 0: MMAs of tile i into accumulator i & 1; false when its copy did not land
    auto mma_tile = [&](int i) -> bool {
        if (!mbar_wait_timed(&bar_b[i & 1], (uint32_t)((i >> 1) & 1), nullptr)) return false;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t b_addr = smem_u32(sB + (size_t)(i & 1) * b_bytes);
        const uint32_t dacc = tmem + (uint32_t)((i & 1) * kTCN);
        for (int kb = 0; kb < K / 16; ++kb) {
            const uint64_t ad = umma_smem_desc(a_addr + (uint32_t)kb * (kTCM * 32));
            const uint64_t bd = umma_smem_desc(b_addr + (uint32_t)kb * (kTCN * 32));
            const uint32_t acc = kb > 0 ? 1u : 0u;
            asm volatile(
                "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(dacc),
                "l"(ad), "l"(bd), "r"(idesc), "r"(acc)
                : "memory");
        }
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                         smem_u32(&bar_mma[i & 1]))
                     : "memory");
        return true;
    };
    if (tid == 0) {
        copy_tile(0);
        if (n > 1) copy_tile(1);
        if (!mma_tile(0)) s_fail = 1;
    }
    float* st = stage + warp * kTCStage;
    int it = 0;
    for (; it < n; ++it) {
        // the next tile's MMAs go to the other accumulator while this one is read
        if (tid == 0 && it + 1 < n && !s_fail && !mma_tile(it + 1)) s_fail = 1;
        __syncthreads();
        if (s_fail) break;
        const bool done = mbar_wait_timed(&bar_mma[it & 1], (uint32_t)((it >> 1) & 1), nullptr);
        if (__syncthreads_or(!done)) {
            if (tid == 0) s_fail = 1;
            break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        // tile it's MMAs are complete: its buffer takes tile it + 2
        if (tid == 0 && it + 2 < n) copy_tile(it + 2);
        const int cbase = (t_begin + it) * kTCN;
        const uint32_t tacc = tmem + (uint32_t)((it & 1) * kTCN) + ((uint32_t)(warp * 32) << 16);
        for (int c0 = 0; c0 < kTCN; c0 += 32) {
            uint32_t r[32];
            asm volatile(
                "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "
                "%13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, "
                "[%32];"
                : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                  "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
                  "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
                  "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
                  "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
                : "r"(tacc + (uint32_t)c0)
                : "memory");
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
            // row = this lane's query, column j: st[lane][j]; read back transposed
#pragma unroll
            for (int j = 0; j < 32; ++j) st[lane * 33 + j] = __uint_as_float(r[j]);
            __syncwarp();
            const int c = cbase + c0 + lane;
            const bool cok = c < nlist;
            const float cnc = cok ? __ldg(cn + c) : 0.f;
            const bool vc = cok && __ldg(valid + c);
#pragma unroll 4
            for (int j = 0; j < 32; ++j) {
                const int row = warp * 32 + j, qj = q0 + row;
                if (cok && qj < nq) {
                    const float dt = fmaxf(s_qn[row] + cnc - 2.f * st[j * 33 + lane], 0.f);
                    out[(size_t)qj * nlist + c] = vc ? __float_as_uint(dt) : 0xFFFFFFFFu;
                }
            }
            __syncwarp();
        }
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncthreads();                      // accumulator it & 1 read before tile it + 2's MMAs reuse it
    }
    if (s_fail) {
        // a wait gave up: report it, give copies and MMAs in flight a last
        // bounded chance to land, then release the tensor memory
        if (tid == 0) {
            atomicOr(flag, 4);
            for (int b = 0; b < 2; ++b) {
                mbar_wait_timed(&bar_mma[b], 0, nullptr);
                mbar_wait_timed(&bar_b[b], 0, nullptr);
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * kTCN)
                     : "memory");
}

constexpr int kRsT = 256;                 // threads of the rescoring CTA
constexpr int kRsItems = 16;              // approximate keys per thread in registers
constexpr int kRsCap = 2048;              // candidates rescored from shared memory

__device__ __forceinline__ float exact_route_dist(const float* __restrict__ sq, const float* __restrict__ c, int d) {
    float s = 0.f;
    for (int j = 0; j < d; ++j) {
        const float x = __fsub_rn(sq[j], __ldg(c + j));
        s = __fadd_rn(s, __fmul_rn(x, x));
    }
    return s;
}

// one CTA per query: candidates from the approximate distances, exact
// rescoring, top-L by (exact distance, list id)
__global__ void __launch_bounds__(kRsT) route_rescore_kernel(const uint32_t* __restrict__ approx,
                                                             const float* __restrict__ q, const float* __restrict__ cent,
                                                             const float* __restrict__ cn_max,
                                                             const uint8_t* __restrict__ valid, int nlist, int d, int L,
                                                             const int32_t* __restrict__ id_map, int32_t* out_ids,
                                                             float* out_dist, uint64_t* out_keys) {
    extern __shared__ __align__(16) unsigned char rs_sm[];
    float* sq = reinterpret_cast<float*>(rs_sm);                                    // [d]
    uint64_t* ck = reinterpret_cast<uint64_t*>(rs_sm + sizeof(float) * ((d + 3) & ~3));  // [kRsCap]
    __shared__ int hist[256];
    __shared__ int bc[4];
    __shared__ unsigned long long mm[64];
    __shared__ int s_cnt;
    __shared__ float s_qn;
    const int row = blockIdx.x, tid = threadIdx.x;
    const uint32_t* ar = approx + (size_t)row * nlist;
    for (int j = tid; j < d; j += kRsT) sq[j] = q[(size_t)row * d + j];
    if (tid == 0) s_cnt = 0;
    __syncthreads();
    if (tid == 0) {
        float s = 0.f;
        for (int j = 0; j < d; ++j) s = __fadd_rn(s, __fmul_rn(sq[j], sq[j]));
        s_qn = s;
    }
    // T~: the L-th smallest approximate key (bits << 32 | local list), or for
    // L <= 32 an upper bound of it: the smallest over the warps of each warp's
    // L-th smallest value (that warp alone has L values at or below it)
    uint64_t tkey;
    if (L <= 32 && nlist <= kRsT * kRsItems) {
        float v[kRsItems];
#pragma unroll
        for (int e = 0; e < kRsItems; ++e) {
            const int i = tid + kRsT * e;
            const uint32_t a = i < nlist ? ar[i] : 0xFFFFFFFFu;
            v[e] = a != 0xFFFFFFFFu ? __uint_as_float(a) : __int_as_float(0x7f800000);
        }
        // sort the lane's values (bitonic network on registers)
#pragma unroll
        for (int size = 2; size <= kRsItems; size <<= 1)
#pragma unroll
            for (int stride = size >> 1; stride > 0; stride >>= 1)
#pragma unroll
                for (int i = 0; i < kRsItems; ++i) {
                    const int jx = i ^ stride;
                    if (jx > i) {
                        const bool up = (i & size) == 0;
                        const float a = v[i], b = v[jx];
                        if ((a > b) == up) {
                            v[i] = b;
                            v[jx] = a;
                        }
                    }
                }
        // L rounds of the warp minimum over the lanes' heads
        float lth = __int_as_float(0x7f800000);
        for (int r = 0; r < L; ++r) {
            float m = v[0];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) m = fminf(m, __shfl_xor_sync(0xffffffffu, m, o));
            const unsigned who = __ballot_sync(0xffffffffu, v[0] == m);
            if ((int)(tid & 31) == __ffs(who) - 1) {
#pragma unroll
                for (int e = 0; e + 1 < kRsItems; ++e) v[e] = v[e + 1];
                v[kRsItems - 1] = __int_as_float(0x7f800000);
            }
            lth = m;
        }
        if (tid == 0) s_cnt = 0x7f800000;
        __syncthreads();
        if ((tid & 31) == 0) atomicMin(&s_cnt, (int)__float_as_uint(lth));   // non-negative: bits order as values
        __syncthreads();
        const uint32_t tb = (uint32_t)s_cnt;
        tkey = tb >= 0x7f800000u ? kKeyNone - 1 : ((uint64_t)tb << 32);
        __syncthreads();
        if (tid == 0) s_cnt = 0;
    } else if (nlist <= kRsT * kRsItems) {
        uint64_t v[kRsItems];
#pragma unroll
        for (int e = 0; e < kRsItems; ++e) {
            const int i = tid + kRsT * e;
            v[e] = i < nlist ? make_key(ar[i], (uint32_t)i) : kKeyNone;
        }
        tkey = nlist > L ? block_kth_items<kRsT, kRsItems>([&](int e) { return v[e]; }, L, kKeyNone - 1, hist, bc, mm)
                         : kKeyNone - 1;
    } else {
        tkey = block_kth_key<kRsT>([&](int i) -> uint64_t { return make_key(ar[i], (uint32_t)i); }, nlist, L,
                                   kKeyNone - 1, hist, bc);
    }
    __syncthreads();
    const uint32_t thi = key_hi(tkey);
    // every list whose approximate distance is within 2 eps of T~ (all valid
    // lists when fewer than L have a distance)
    const float eps = ldexpf(s_qn + *cn_max, -11);
    const float lim = thi == 0xFFFFFFFFu ? __int_as_float(0x7f800000) : __uint_as_float(thi) + 2.f * eps;
    for (int i = tid; i < nlist; i += kRsT) {
        const uint32_t a = ar[i];
        if (a != 0xFFFFFFFFu && __uint_as_float(a) <= lim) {
            const int at = atomicAdd(&s_cnt, 1);
            if (at < kRsCap) ck[at] = (uint64_t)i;
        }
    }
    __syncthreads();
    const int ncand = s_cnt;
    int Lp = 1;
    while (Lp < L) Lp <<= 1;
    if (ncand <= kRsCap) {
        int np = 1;
        while (np < ncand) np <<= 1;
        if (np < Lp) np = Lp;
        for (int i = tid; i < np; i += kRsT) {     // each thread rewrites only its own entries
            uint64_t key = kKeyNone;
            if (i < ncand) {
                const int c = (int)ck[i];
                const float dd = exact_route_dist(sq, cent + (size_t)c * d, d);
                key = make_key(__float_as_uint(dd), id_map ? (uint32_t)id_map[c] : (uint32_t)c);
            }
            ck[i] = key;
        }
        __syncthreads();
        block_bitonic_sort<kRsT>(ck, np);
    } else {
        // too many near-ties: rescore every valid list
        auto keyf = [&](int i) -> uint64_t {
            if (!valid[i]) return kKeyNone;
            const float dd = exact_route_dist(sq, cent + (size_t)i * d, d);
            return make_key(__float_as_uint(dd), id_map ? (uint32_t)id_map[i] : (uint32_t)i);
        };
        const uint64_t kap = block_kth_key<kRsT>(keyf, nlist, L, kKeyNone - 1, hist, bc);
        if (tid == 0) s_cnt = 0;
        __syncthreads();
        for (int i = tid; i < nlist; i += kRsT) {
            const uint64_t k = keyf(i);
            if (k < kap) ck[atomicAdd(&s_cnt, 1)] = k;
        }
        __syncthreads();
        const int cl = s_cnt;
        for (int i = cl + tid; i < Lp; i += kRsT) ck[i] = i < L ? kap : kKeyNone;
        block_bitonic_sort<kRsT>(ck, Lp);
    }
    for (int i = tid; i < L; i += kRsT) {
        const uint64_t k = ck[i];
        const bool ok = k != kKeyNone && key_hi(k) != 0xFFFFFFFFu;
        if (out_ids) out_ids[(size_t)row * L + i] = ok ? (int32_t)key_lo(k) : -1;
        if (out_dist) out_dist[(size_t)row * L + i] = ok ? __uint_as_float(key_hi(k)) : __int_as_float(0x7f800000);
        if (out_keys) out_keys[(size_t)row * L + i] = k;
    }
}

// ---------------------------------------------------------------------------
// Fused routing for nprobe <= 32: one sweep, no distance matrix leaves the SM.
// ---------------------------------------------------------------------------
// The split operands of route_tc_kernel (64-centroid tiles, parts
// [c_hi | c_lo | c_hi]), so the same eps = 2^-11 (|q|^2 + max |c|^2) bounds
// |D~ - D|.  The query operand holds [q_hi | q_lo] once; the MMAs of parts 0
// and 1 both read q_hi.  A CTA whose 128 queries all have q_lo = 0 (queries
// that bf16 holds exactly, e.g. integer values below 256) runs parts 0 and 1
// only: q.c = q_hi.c_hi + q_hi.c_lo then misses only q.(c - c_hi - c_lo).
//
// Grid: (query blocks of 128, column splits); CTA (x, y) sweeps the tiles
// [y * tiles_per_cta, ...) and produces, per query row, the exact top-L of
// its columns; the splits are merged afterwards (route_split_merge_kernel).
// The top-L of a union is the top-L of the parts' top-L, so the merged lists
// equal the exact routing.
//
// Warp roles (320 threads, no block-wide barrier inside the sweep):
//   warp 8  (one thread): bulk async copies of operand tiles into a ring of
//           stages (as many as fit: 2-5), each stage freed by the commit of
//           the MMAs that read it;
//   warp 9  (one thread): tcgen05 MMAs of tile g into one of 4 TMEM
//           accumulators, committed to the accumulator's "full" barrier;
//   warps 0-7: TMEM lane quarter w % 4 (rows 32 (w % 4) .. +31), columns
//           32 (w / 4) .. +31 of every tile (each row is shared by two
//           threads, "halves"); each reads its 32 values with tcgen05.ld,
//           frees the accumulator, then filters.
// While the tiles stream by, each epilogue thread keeps
//   * lv: the L smallest D~ it has seen (ascending), lmax = lv[L-1];
//   * a list of (D~, column) with D~ <= lmax + 2 eps at the time it was seen,
//     pruned to the current bound before a piece of columns could overflow it
//     (a prune that does not make room gives up on the row).
// The filter tests c_n - 2 q.c <= lmax + 2 eps - |q|^2 (+ a rounding slack)
// on column pairs with packed fp32 arithmetic; only a pair some lane of the
// warp keeps takes the append branch.  lmax only decreases and each half's
// lmax is at least the row's final L-th smallest D~ (T~), so every column
// with D~ <= T~ + 2 eps -- a superset of the exact top-L -- is in one of the
// two lists.  The candidates are rescored exactly and the row's top-L of this
// split is written; a row whose list overflowed is handed to
// route_exact_rows_kernel.  Every wait is bounded and also gives up once
// another role has failed.
constexpr int kFT = 256;                  // epilogue threads
constexpr int kFBlock = 320;              // + the copy warp and the MMA warp
constexpr int kFLMax = 32;                // largest L of the fused path
constexpr int kFN = kTCN;                 // centroids per tile (MMA N)
constexpr int kFAcc = 4;                  // TMEM accumulators
constexpr int kFMaxStages = 8;
constexpr int kFMaxSplits = 32;           // column splits per query block (one lane each in the merge)

// candidate slots per (row, half): the L smallest, one piece of kFW columns and a
// band of near-ties above the running bound
constexpr int kFW = 8;
__host__ __device__ constexpr int fused_list(int lmax) { return lmax <= 16 ? lmax + 24 : 48; }

// shared memory besides the stage region: A, candidate lists, qn / T~ / counts
__host__ __device__ constexpr size_t route_fused_fixed(int d, int list) {
    return (size_t)kTCM * 2 * d * 2 + (sizeof(float) + sizeof(uint16_t)) * kFT * (size_t)list +
           sizeof(float) * 2 * kTCM + sizeof(int) * kFBlock;
}
// the stage region must hold two 2-part tiles (queries bf16 holds exactly)
// and one 3-part tile (a single stage serialises copy and MMA but works), and
// after the sweep the halves' L-lists and the rescoring's pair list
__host__ __device__ constexpr size_t route_fused_region_min(int d, int list) {
    const size_t part = (size_t)kFN * d * 2;
    const size_t tiles = 4 * part > 3 * part ? 4 * part : 3 * part;
    const size_t after = sizeof(float) * kTCM * kFLMax + sizeof(uint16_t) * kFT * (size_t)list;
    return tiles > after ? tiles : after;
}
constexpr size_t kFSmemCap = 227 * 1024 - 4608;  // dynamic shared memory of one CTA (4.5 KB static aside)

__host__ __device__ constexpr size_t route_fused_region(int d, int list) {
    return ((kFSmemCap - route_fused_fixed(d, list)) / 128) * 128;
}

template <int LMAX, int LIST>
__global__ void __launch_bounds__(kFBlock, 1)
    route_tc_fused_kernel(const float* __restrict__ q, int nq, int d, const uint16_t* __restrict__ ops,
                          const float* __restrict__ cne, const float* __restrict__ cn_max,
                          const uint8_t* __restrict__ valid, int nlist, const float* __restrict__ cent, int L,
                          const int32_t* __restrict__ id_map, int tiles_per_cta, int region, int32_t* out_ids,
                          uint64_t* out_keys, uint64_t* split_keys, uint32_t* row_bound,
                          int32_t* __restrict__ row_fallback, int* flag) {
    extern __shared__ __align__(1024) unsigned char sm[];
    __shared__ __align__(8) uint64_t bar_full[kFMaxStages];
    __shared__ __align__(8) uint64_t bar_empty[kFMaxStages];
    __shared__ __align__(8) uint64_t bar_af[kFAcc];
    __shared__ __align__(8) uint64_t bar_ae[kFAcc];
    __shared__ uint32_t s_tmem;
    __shared__ int s_fail;
    __shared__ int s_scan[33];
    __shared__ float s_halfb[2][kTCM];     // each half's running (L/2)-th smallest D~ (L == LMAX)
    __shared__ __align__(16) float s_cn[8][2][32];   // per epilogue warp: its columns' norms, two tiles
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const bool epi = warp < 8;
    const int quarter = warp & 3, half = (warp >> 2) & 1;
    const int row = quarter * 32 + lane;                  // TMEM lane = query row of an epilogue thread
    const uint32_t part_bytes = (uint32_t)kFN * d * 2;    // one part of one tile
    const uint32_t a_bytes = (uint32_t)kTCM * 2 * d * 2;
    unsigned char* sA = sm;
    unsigned char* sB = sm + a_bytes;                                             // stage region
    float* s_lval = reinterpret_cast<float*>(sB + region);                       // [LIST][kFT]
    uint16_t* s_lcol = reinterpret_cast<uint16_t*>(s_lval + kFT * LIST);          // [LIST][kFT]
    float* s_qn = reinterpret_cast<float*>(s_lcol + kFT * LIST);                  // [128]
    float* s_T = s_qn + kTCM;                                                     // [128]
    int* s_nc = reinterpret_cast<int*>(s_T + kTCM);                               // [kFBlock]
    // after the sweep the stage region holds the halves' L-lists, then the rescored keys
    float* s_lv = reinterpret_cast<float*>(sB);                                   // [LMAX][128] (half 1)
    const int q0 = blockIdx.x * kTCM;
    const int ntiles_all = (nlist + kFN - 1) / kFN;
    const int t_begin = blockIdx.y * tiles_per_cta;
    const int nt = min(ntiles_all, t_begin + tiles_per_cta) - t_begin;           // >= 1 (launch)
    const int c_begin = t_begin * kFN;
    const float INF = __int_as_float(0x7f800000);

    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                     "r"(kFAcc * kFN)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (tid == 0) {
        for (int b = 0; b < kFMaxStages; ++b) {
            mbar_init(&bar_full[b], 1);
            mbar_init(&bar_empty[b], 1);
        }
        for (int a = 0; a < kFAcc; ++a) {
            mbar_init(&bar_af[a], 1);
            mbar_init(&bar_ae[a], 8);         // one arrival per epilogue warp
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        s_fail = 0;
    }
    if (tid < 2 * kTCM) s_halfb[tid >> 7][tid & (kTCM - 1)] = INF;
    // A operand [q_hi | q_lo]: epilogue thread t builds row t % 128, the 8-element
    // groups g of its half (two 16-byte loads per group)
    int has_lo = 0;
    if (epi) {
        const int r = tid & (kTCM - 1), qi = q0 + r;
        const bool qok = qi < nq;
        const float4* qr4 = reinterpret_cast<const float4*>(q + (size_t)(qok ? qi : 0) * d);
        const int G = d / 8;
        for (int g = tid >> 7; g < G; g += kFT / kTCM) {
            const float4 va = qok ? __ldg(qr4 + 2 * g) : make_float4(0.f, 0.f, 0.f, 0.f);
            const float4 vb = qok ? __ldg(qr4 + 2 * g + 1) : make_float4(0.f, 0.f, 0.f, 0.f);
            auto split2 = [](float x0, float x1, uint32_t& whi, uint32_t& wlo) {
                const __nv_bfloat16 h0 = __float2bfloat16_rn(x0), h1 = __float2bfloat16_rn(x1);
                const __nv_bfloat16 l0 = __float2bfloat16_rn(x0 - __bfloat162float(h0));
                const __nv_bfloat16 l1 = __float2bfloat16_rn(x1 - __bfloat162float(h1));
                whi = bf16_bits(h0) | (bf16_bits(h1) << 16);
                wlo = bf16_bits(l0) | (bf16_bits(l1) << 16);
            };
            uint4 hi4, lo4;
            split2(va.x, va.y, hi4.x, lo4.x);
            split2(va.z, va.w, hi4.y, lo4.y);
            split2(vb.x, vb.y, hi4.z, lo4.z);
            split2(vb.z, vb.w, hi4.w, lo4.w);
            *reinterpret_cast<uint4*>(sA + tc_chunk_off(r, g, kTCM)) = hi4;
            *reinterpret_cast<uint4*>(sA + tc_chunk_off(r, G + g, kTCM)) = lo4;
            has_lo |= (lo4.x | lo4.y | lo4.z | lo4.w) != 0u;
        }
        if (tid < kTCM) {
            float qn = 0.f;
            if (qok)
                for (int w = 0; w < d / 4; ++w) {
                    const float4 a = __ldg(qr4 + w);
                    qn = __fadd_rn(qn, __fmul_rn(a.x, a.x));
                    qn = __fadd_rn(qn, __fmul_rn(a.y, a.y));
                    qn = __fadd_rn(qn, __fmul_rn(a.z, a.z));
                    qn = __fadd_rn(qn, __fmul_rn(a.w, a.w));
                }
            s_qn[tid] = qn;
        }
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    const int nparts = __syncthreads_or(has_lo) ? 3 : 2;
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = s_tmem;
    const uint32_t stage_bytes = (uint32_t)nparts * part_bytes;
    int nst = (int)((uint32_t)region / stage_bytes);
    if (nst > kFMaxStages) nst = kFMaxStages;
    const volatile int* vfail = &s_fail;
    int issued = 0, mma_issued = 0;

    // the L smallest, ascending, in the last L slots; the slots before them hold
    // -inf and never change, so lmax = lv[LMAX - 1] needs no runtime index
    float lv[LMAX];
#pragma unroll
    for (int i = 0; i < LMAX; ++i) lv[i] = i < LMAX - L ? -INF : INF;
    float lmax = INF;
    float ub = INF;                        // the row's shared bound as last read
    int nc = 0;                            // entries in this thread's list
    bool over = false;                     // the list overflowed within the bound
    const float qn = epi ? s_qn[row] : 0.f;
    // |D~ - D| <= eps = 2^-13 (|q|^2 + max |c|^2): the split leaves q.c with an
    // error below 2^-17 sum |q_j c_j| (each bf16 rounding is within 2^-9, so
    // c - c_hi - c_lo is within 2^-18 |c| and q_lo c_lo within 2^-18 |q| |c|),
    // the tensor cores' fp32 accumulation of at most 3d <= 384 exact bf16
    // products adds at most 2 * 384 * 2^-24 sum |q_j c_j| (allowing truncating
    // adds), the fp32 norms 2^-17 of each, the final fma and add 2^-22 of the
    // total: with 2 |q| |c| <= |q|^2 + |c|^2, about 2^-14.9 (|q|^2 + |c|^2),
    // a quarter of eps
    const float eps2 = 2.f * ldexpf(qn + *cn_max, -13);
    float* myval = s_lval + tid;           // entry i at [i][tid]: a warp's stores hit 32 banks
    uint16_t* mycol = s_lcol + tid;

    if (warp == 8) {
        if (lane == 0) {
            // copies: tile g into stage g % nst once the MMAs of tile g - nst are done
            const unsigned char* gops = reinterpret_cast<const unsigned char*>(ops);
            const size_t tile_stride = (size_t)3 * part_bytes;
            for (int g = 0; g < nt; ++g) {
                const int s = g % nst;
                if (g >= nst && !mbar_wait_timed(&bar_empty[s], (uint32_t)(((g / nst) - 1) & 1), vfail)) {
                    s_fail = 1;
                    break;
                }
                mbar_arrive_expect(&bar_full[s], stage_bytes);
                bulk_g2s(sB + (size_t)s * stage_bytes, gops + (size_t)(t_begin + g) * tile_stride, stage_bytes,
                         &bar_full[s]);
                issued = g + 1;
            }
        }
        __syncwarp();
    } else if (warp == 9) {
        if (lane == 0) {
            constexpr uint32_t idesc = umma_idesc_bf16(kTCM, kFN);
            const uint32_t a_addr = smem_u32(sA);
            const int kbp = d / 16;                  // K blocks of 16 per part
            for (int g = 0; g < nt; ++g) {
                const int s = g % nst, a = g % kFAcc;
                if (g >= kFAcc && !mbar_wait_timed(&bar_ae[a], (uint32_t)(((g / kFAcc) - 1) & 1), vfail)) {
                    s_fail = 1;
                    break;
                }
                if (!mbar_wait_timed(&bar_full[s], (uint32_t)((g / nst) & 1), vfail)) {
                    s_fail = 1;
                    break;
                }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t b_addr = smem_u32(sB + (size_t)s * stage_bytes);
                const uint32_t dacc = tmem + (uint32_t)(a * kFN);
                for (int p = 0; p < nparts; ++p) {
                    const int ap = p == 2 ? 1 : 0;      // parts 0 and 1 read q_hi, part 2 reads q_lo
                    for (int kb = 0; kb < kbp; ++kb) {
                        const uint64_t ad = umma_smem_desc(a_addr + (uint32_t)(ap * kbp + kb) * (kTCM * 32));
                        const uint64_t bd = umma_smem_desc(b_addr + (uint32_t)(p * kbp + kb) * (kFN * 32));
                        const uint32_t acc = (p | kb) ? 1u : 0u;
                        asm volatile(
                            "{\n .reg .pred pa;\n setp.ne.b32 pa, %4, 0;\n"
                            " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, pa;\n}" ::"r"(dacc),
                            "l"(ad), "l"(bd), "r"(idesc), "r"(acc)
                            : "memory");
                    }
                }
                asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                                 smem_u32(&bar_empty[s]))
                             : "memory");
                asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                                 smem_u32(&bar_af[a]))
                             : "memory");
                mma_issued = g + 1;
            }
        }
        __syncwarp();
    } else {
        // candidate test on (c_n - 2 q.c) against lim - |q|^2, widened by a slack
        // that covers the rounding of the shifted comparison (far below eps)
        const float slack = ldexpf(qn + *cn_max, -19);
        float lq = INF;                    // min(lmax, ub) + 2 eps - |q|^2 + slack
        constexpr int kW = kFW;
        // the row's bound shared by all CTAs (and both halves) of this query: the
        // smallest running L-th D~ any of them has published; any such value is
        // >= the row's final L-th smallest D~, so it is a valid filter bound
        volatile uint32_t* rb = (row_bound && q0 + row < nq) ? row_bound + (q0 + row) : nullptr;
        uint32_t ub_next = rb ? *rb : 0x7f800000u;
        float pub = INF;                   // the last bound this thread published
        // the column norms of this warp's 32 columns of a tile: one coalesced load
        // per lane (issued a tile ahead) into the warp's buffer, read back as
        // broadcasts
        float cnn = __ldg(cne + c_begin + half * 32 + lane);
        for (int g = 0; g < nt; ++g) {
            const int a = g % kFAcc;
            const bool got = mbar_wait_timed(&bar_af[a], (uint32_t)((g / kFAcc) & 1), vfail);
            if (!__all_sync(0xffffffffu, got)) {
                if (lane == 0) s_fail = 1;
                break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            uint32_t r[32];
            asm volatile(
                "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
                "%12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, "
                "%30, %31}, [%32];"
                : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
                  "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
                  "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]),
                  "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]),
                  "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
                : "r"(tmem + (uint32_t)(a * kFN + half * 32) + ((uint32_t)(quarter * 32) << 16))
                : "memory");
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(&bar_ae[a]);          // the accumulator may be refilled
            ub = fminf(ub, __uint_as_float(ub_next));
            if (rb) ub_next = *rb;                            // for the next tile
            lq = fminf(lmax, ub) + eps2 - qn + slack;
            const int rel0 = g * kFN + half * 32;            // column of r[0], relative to c_begin
            s_cn[warp][g & 1][lane] = cnn;
            __syncwarp();
            if (g + 1 < nt) cnn = __ldg(cne + c_begin + rel0 + kFN + lane);
            float4 cn4[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) cn4[i] = reinterpret_cast<const float4*>(s_cn[warp][g & 1])[i];
#pragma unroll
            for (int j0 = 0; j0 < 32; j0 += kW) {
                if (!over && nc > LIST - kW) {
                    const float lim = fminf(lmax, ub) + eps2;
                    int k2 = 0;
                    for (int i = 0; i < nc; ++i) {
                        const float v = myval[i * kFT];
                        if (v <= lim) {
                            myval[k2 * kFT] = v;
                            mycol[k2 * kFT] = mycol[i * kFT];
                            ++k2;
                        }
                    }
                    nc = k2;
                    if (nc > LIST - kW) over = true;
                }
                const int nc0 = nc;
#pragma unroll
                for (int j = j0; j < j0 + kW; j += 4) {
                    const float4 c4 = cn4[j / 4];
                    const float2 m2 = make_float2(-2.f, -2.f);
                    const float2 x01 = __ffma2_rn(make_float2(__uint_as_float(r[j]), __uint_as_float(r[j + 1])), m2,
                                                  make_float2(c4.x, c4.y));
                    const float2 x23 = __ffma2_rn(make_float2(__uint_as_float(r[j + 2]), __uint_as_float(r[j + 3])),
                                                  m2, make_float2(c4.z, c4.w));
                    const bool p0 = x01.x <= lq, p1 = x01.y <= lq, p2 = x23.x <= lq, p3 = x23.y <= lq;
                    if (__any_sync(0xffffffffu, p0 | p1 | p2 | p3) && !over) {
                        if (p0) {
                            myval[nc * kFT] = fmaxf(x01.x + qn, 0.f);
                            mycol[nc * kFT] = (uint16_t)(rel0 + j);
                            ++nc;
                        }
                        if (p1) {
                            myval[nc * kFT] = fmaxf(x01.y + qn, 0.f);
                            mycol[nc * kFT] = (uint16_t)(rel0 + j + 1);
                            ++nc;
                        }
                        if (p2) {
                            myval[nc * kFT] = fmaxf(x23.x + qn, 0.f);
                            mycol[nc * kFT] = (uint16_t)(rel0 + j + 2);
                            ++nc;
                        }
                        if (p3) {
                            myval[nc * kFT] = fmaxf(x23.y + qn, 0.f);
                            mycol[nc * kFT] = (uint16_t)(rel0 + j + 3);
                            ++nc;
                        }
                    }
                }
                // the L smallest: only this thread's new entries
                for (int i = nc0; i < nc; ++i) {
                    float v = myval[i * kFT];
                    if (v < lmax) {
#pragma unroll
                        for (int e = 0; e < LMAX; ++e) {
                            const float a2 = lv[e];
                            lv[e] = fminf(a2, v);
                            v = fmaxf(a2, v);
                        }
                        lmax = lv[LMAX - 1];
                    }
                }
                lq = fminf(lmax, ub) + eps2 - qn + slack;
            }
            // the two halves of a row: L/2 values of each at or below max(A[L/2-1],
            // B[L/2-1]) make L values at or below it, so it bounds the row's L-th
            float bnd = lmax;
            if (L == LMAX) {
                s_halfb[half][row] = lv[LMAX / 2 - 1];
                bnd = fminf(bnd, fmaxf(lv[LMAX / 2 - 1], s_halfb[half ^ 1][row]));
                ub = fminf(ub, bnd);
                lq = fminf(lmax, ub) + eps2 - qn + slack;
            }
            if (rb && bnd < pub) {
                atomicMin(const_cast<uint32_t*>(rb), __float_as_uint(bnd));    // non-negative: bits order as values
                pub = bnd;
            }
        }
    }
    __syncthreads();
    const bool failed = s_fail != 0;
    if (failed) {
        // a wait gave up: report it, give copies and MMAs in flight a last
        // bounded chance to land, then release the tensor memory
        if (tid == 8 * 32) {
            atomicOr(flag, 4);
            for (int g = issued - nst < 0 ? 0 : issued - nst; g < issued; ++g)
                mbar_wait_timed(&bar_full[g % nst], (uint32_t)((g / nst) & 1), nullptr);
        }
        if (tid == 9 * 32 && mma_issued > 0) {
            const int g = mma_issued - 1;
            mbar_wait_timed(&bar_af[g % kFAcc], (uint32_t)((g / kFAcc) & 1), nullptr);
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kFAcc * kFN)
                     : "memory");
    // T~ of the row: the L-th smallest of the two halves' ascending L smallest
    // A (this thread's lv, half 0) and B (half 1's, through s_lv, entry-major
    // [i][row]: the lanes of a warp read 32 different banks), as
    // min over i = 0..L of max(A[i-1], B[L-1-i]) with A[-1] = B[-1] = -inf;
    // in the arrays A[i] is slot LMAX - L + i (slot ip = LMAX - L + i - 1 below)
    if (epi && half == 1) {
#pragma unroll
        for (int i = 0; i < LMAX; ++i) s_lv[i * kTCM + row] = lv[i];
    }
    __syncthreads();
    if (epi && half == 0) {
        float T = INF;
#pragma unroll
        for (int ip = -1; ip < LMAX; ++ip) {
            if (ip < LMAX - L - 1) continue;
            const float a = ip < 0 ? -INF : lv[ip < 0 ? 0 : ip];
            const int jb = 2 * LMAX - L - 2 - ip;
            const float b = jb < LMAX - L ? -INF : s_lv[jb * kTCM + row];
            T = fminf(T, fmaxf(a, b));
        }
        s_T[row] = T;
        // the split's L-th smallest D~ bounds the row for the CTAs that follow
        if (row_bound && q0 + row < nq && T < INF) atomicMin(row_bound + q0 + row, __float_as_uint(T));
    }
    __syncthreads();
    // this thread's candidates: list entries within T~ + 2 eps, moved to the
    // front of its list and rescored in place (the exact distance replaces D~)
    const float T = epi ? s_T[row] : INF;
    // candidates: D~ <= min(T~ of this split's lists, the shared bound) + 2 eps,
    // both >= the row's global L-th smallest D~
    const float tb = fminf(T, ub);
    const float climit = tb + eps2;
    const int qi = q0 + row;
    int nk = 0;
    const bool big = !epi || over || !(tb < 3.0e38f);
    if (epi && qi < nq && !failed && !big) {
        for (int i = 0; i < nc; ++i) {
            if (myval[i * kFT] > climit) continue;
            mycol[nk * kFT] = mycol[i * kFT];
            ++nk;
        }
    }
    // Balanced rescoring: every (thread, slot) candidate of the CTA goes into
    // one pair list (after the halves' L-lists in the stage region), which all
    // threads work through two at a time (two independent exact sums, their
    // loads in flight together)
    uint16_t* s_pair = reinterpret_cast<uint16_t*>(s_lv + LMAX * kTCM);     // [kFT * LIST]
    {
        const int mine = (epi && qi < nq && !failed && !big) ? nk : 0;
        int total;
        const int off = block_excl_scan<kFBlock>(mine, s_scan, &total);
        for (int i = 0; i < mine; ++i) s_pair[off + i] = (uint16_t)((i << 8) | tid);
        __syncthreads();
        for (int p = tid; p < total; p += 2 * kFBlock) {
            const int e0 = s_pair[p], e1 = p + kFBlock < total ? s_pair[p + kFBlock] : e0;
            const int t0 = e0 & 255, i0 = e0 >> 8, t1 = e1 & 255, i1 = e1 >> 8;
            const int c0 = c_begin + s_lcol[i0 * kFT + t0], c1 = c_begin + s_lcol[i1 * kFT + t1];
            const float4* qa = reinterpret_cast<const float4*>(q + (size_t)(q0 + (t0 & (kTCM - 1))) * d);
            const float4* qb = reinterpret_cast<const float4*>(q + (size_t)(q0 + (t1 & (kTCM - 1))) * d);
            const float4* r0 = reinterpret_cast<const float4*>(cent + (size_t)c0 * d);
            const float4* r1 = reinterpret_cast<const float4*>(cent + (size_t)c1 * d);
            float s0 = 0.f, s1 = 0.f;
#pragma unroll 4
            for (int j = 0; j < d / 4; ++j) {
                const float4 a0 = __ldg(qa + j), b0 = __ldg(r0 + j), a1 = __ldg(qb + j), b1 = __ldg(r1 + j);
                float x = __fsub_rn(a0.x, b0.x), y = __fsub_rn(a1.x, b1.x);
                s0 = __fadd_rn(s0, __fmul_rn(x, x));
                s1 = __fadd_rn(s1, __fmul_rn(y, y));
                x = __fsub_rn(a0.y, b0.y);
                y = __fsub_rn(a1.y, b1.y);
                s0 = __fadd_rn(s0, __fmul_rn(x, x));
                s1 = __fadd_rn(s1, __fmul_rn(y, y));
                x = __fsub_rn(a0.z, b0.z);
                y = __fsub_rn(a1.z, b1.z);
                s0 = __fadd_rn(s0, __fmul_rn(x, x));
                s1 = __fadd_rn(s1, __fmul_rn(y, y));
                x = __fsub_rn(a0.w, b0.w);
                y = __fsub_rn(a1.w, b1.w);
                s0 = __fadd_rn(s0, __fmul_rn(x, x));
                s1 = __fadd_rn(s1, __fmul_rn(y, y));
            }
            s_lval[i0 * kFT + t0] = s0;
            if (p + kFBlock < total) s_lval[i1 * kFT + t1] = s1;
        }
    }
    s_nc[tid] = big ? -1 : nk;
    __syncthreads();
    if (epi && half == 0 && qi < nq) {
        const int na = s_nc[tid], nb = s_nc[tid + kTCM];
        const bool fall = failed || na < 0 || nb < 0;
        if (fall) row_fallback[qi] = 1;
        // top-L of the row's candidates by (exact distance, list): repeated
        // minimum over the two halves' lists; local columns order as the
        // global ids do (id_map is increasing), so (distance bits, column) keys
        // rank them and the output keys carry the global ids
        const float* va = s_lval + tid;
        const float* vb = s_lval + tid + kTCM;
        const uint16_t* ca = s_lcol + tid;
        const uint16_t* cb = s_lcol + tid + kTCM;
        uint64_t last = 0;
        for (int o = 0; o < L; ++o) {
            uint64_t best = kKeyNone;
            if (!fall) {
                for (int i = 0; i < na; ++i) {
                    const uint64_t kk = make_key(__float_as_uint(va[i * kFT]), (uint32_t)ca[i * kFT]);
                    if ((o == 0 || kk > last) && kk < best) best = kk;
                }
                for (int i = 0; i < nb; ++i) {
                    const uint64_t kk = make_key(__float_as_uint(vb[i * kFT]), (uint32_t)cb[i * kFT]);
                    if ((o == 0 || kk > last) && kk < best) best = kk;
                }
            }
            last = best;
            uint64_t outk = kKeyNone;
            if (best != kKeyNone) {
                const int c = c_begin + (int)key_lo(best);
                outk = make_key(key_hi(best), id_map ? (uint32_t)id_map[c] : (uint32_t)c);
            }
            if (split_keys) {
                split_keys[((size_t)blockIdx.y * nq + qi) * L + o] = outk;
            } else if (!fall) {
                const bool ok = outk != kKeyNone;
                if (out_ids) out_ids[(size_t)qi * L + o] = ok ? (int32_t)key_lo(outk) : -1;
                if (out_keys) out_keys[(size_t)qi * L + o] = outk;
            }
        }
    }
}

// Top-L per query of the column splits' sorted top-L keys [S][nq][L]: one
// warp per query, lane s walks split s's list, L rounds of the warp minimum.
__global__ void __launch_bounds__(256) route_split_merge_kernel(const uint64_t* __restrict__ keys, int S, int nq,
                                                                int L, int32_t* out_ids, uint64_t* out_keys) {
    const int qi = (int)((blockIdx.x * (size_t)blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
    if (qi >= nq) return;                  // whole warps only
    const uint64_t* mine = keys + ((size_t)lane * nq + qi) * L;
    int pos = 0;
    for (int o = 0; o < L; ++o) {
        const uint64_t h = (lane < S && pos < L) ? mine[pos] : kKeyNone;
        uint64_t m = h;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            const uint64_t t = __shfl_xor_sync(0xffffffffu, m, off);
            m = t < m ? t : m;
        }
        if (h == m && m != kKeyNone) ++pos;   // keys are distinct: one lane advances
        if (lane == 0) {
            const bool ok = m != kKeyNone && key_hi(m) != 0xFFFFFFFFu;
            if (out_ids) out_ids[(size_t)qi * L + o] = ok ? (int32_t)key_lo(m) : -1;
            if (out_keys) out_keys[(size_t)qi * L + o] = m;
        }
    }
}

// Rows the fused kernel marked: exact distances to every list, top-L.
__global__ void __launch_bounds__(kRsT) route_exact_rows_kernel(const int32_t* __restrict__ row_fallback,
                                                                const float* __restrict__ q,
                                                                const float* __restrict__ cent,
                                                                const uint8_t* __restrict__ valid, int nlist, int d,
                                                                int L, const int32_t* __restrict__ id_map,
                                                                int32_t* out_ids, uint64_t* out_keys) {
    const int row = blockIdx.x, tid = threadIdx.x;
    if (!row_fallback[row]) return;
    __shared__ float sq[kPMaxRouteD];
    __shared__ uint64_t sk[64];
    __shared__ int hist[256];
    __shared__ int bc[4];
    __shared__ int s_cnt;
    for (int j = tid; j < d; j += kRsT) sq[j] = q[(size_t)row * d + j];
    if (tid == 0) s_cnt = 0;
    __syncthreads();
    auto keyf = [&](int i) -> uint64_t {
        if (!valid[i]) return kKeyNone;
        const float dd = exact_route_dist(sq, cent + (size_t)i * d, d);
        return make_key(__float_as_uint(dd), id_map ? (uint32_t)id_map[i] : (uint32_t)i);
    };
    int nvalid = 0;
    for (int i = tid; i < nlist; i += kRsT) nvalid += valid[i] ? 1 : 0;
    nvalid = block_sum<kRsT>(nvalid, hist);
    const int take = nvalid < L ? nvalid : L;
    uint64_t kap = kKeyNone;
    if (take > 0) kap = block_kth_key<kRsT>(keyf, nlist, take, kKeyNone - 1, hist, bc);
    __syncthreads();
    for (int i = tid; i < nlist; i += kRsT) {
        const uint64_t k = keyf(i);
        if (k < kap) sk[atomicAdd(&s_cnt, 1)] = k;
    }
    __syncthreads();
    const int cl = s_cnt;
    for (int i = cl + tid; i < 64; i += kRsT) sk[i] = i < take ? kap : kKeyNone;
    block_bitonic_sort<kRsT>(sk, 64);
    for (int i = tid; i < L; i += kRsT) {
        const uint64_t k = sk[i];
        const bool ok = k != kKeyNone;
        if (out_ids) out_ids[(size_t)row * L + i] = ok ? (int32_t)key_lo(k) : -1;
        if (out_keys) out_keys[(size_t)row * L + i] = k;
    }
}

}  // namespace

bool route_tc_usable(int d, int nlist) {
    return d > 0 && d % 16 == 0 && nlist > 0 && route_tc_smem(d) <= 227 * 1024;
}

int route_tc_tile(int) { return kTCN; }

size_t route_tc_ops_elems(int nlist, int d) { return (size_t)((nlist + kTCN - 1) / kTCN) * kTCN * 3 * d; }

size_t route_tc_cne_len(int nlist) { return (size_t)((nlist + kTCN - 1) / kTCN) * kTCN; }

cudaError_t route_tc_prepare(const float* cent, const uint8_t* valid, int nlist, int d, uint16_t* ops, float* cn,
                             float* cne, float* cn_max, cudaStream_t st) {
    if (!route_tc_usable(d, nlist)) return cudaErrorInvalidValue;
    note_launch();
    route_tc_prepare_kernel<<<512, 256, 0, st>>>(cent, valid, nlist, d, ops, cn, cne);
    cudaError_t e = cudaGetLastError();
    if (e) return e;
    note_launch();
    route_tc_cnmax_kernel<<<1, 256, 0, st>>>(cn, valid, nlist, cn_max);
    return cudaGetLastError();
}

cudaError_t route_tc(const float* q, int nq, const uint16_t* ops, const float* cn, const uint8_t* valid, int nlist,
                     int d, uint32_t* out, int* flag, cudaStream_t st) {
    if (nq <= 0) return cudaSuccess;
    if (!route_tc_usable(d, nlist)) return cudaErrorInvalidValue;
    const size_t smem = route_tc_smem(d);
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int gx = (nq + kTCM - 1) / kTCM, ntiles = (nlist + kTCN - 1) / kTCN;
    int gy = sms / gx;
    if (gy < 1) gy = 1;
    if (gy > ntiles) gy = ntiles;
    const int per = (ntiles + gy - 1) / gy;
    gy = (ntiles + per - 1) / per;
    cudaError_t e = cudaFuncSetAttribute(route_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e) return e;
    note_launch();
    route_tc_kernel<<<dim3(gx, gy), kTCThreads, smem, st>>>(q, nq, d, ops, cn, valid, nlist, per, out, flag);
    return cudaGetLastError();
}

namespace {
int fused_lmax(int L) { return L <= 8 ? 8 : (L <= 16 ? 16 : 32); }
}  // namespace

bool route_tc_fused_usable(int d, int nlist, int L) {
    if (!route_tc_usable(d, nlist) || L < 1 || L > kFLMax || d > kPMaxRouteD) return false;
    const int list = fused_list(fused_lmax(L));
    if (route_fused_fixed(d, list) + 1024 >= kFSmemCap) return false;
    if (route_fused_region(d, list) < route_fused_region_min(d, list)) return false;
    // at most kFMaxSplits column splits of at most 65536 columns (16-bit list entries)
    const int ntiles = (nlist + kFN - 1) / kFN;
    return (ntiles + kFMaxSplits - 1) / kFMaxSplits <= 65536 / kFN;
}

int route_tc_fused_splits(int nq, int nlist) {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int ntiles = (nlist + kFN - 1) / kFN, qb = (nq + kTCM - 1) / kTCM;
    int best = 1;
    double best_cost = 1e300;
    // one CTA per SM (shared memory); a CTA costs its tiles plus about 6 tiles
    // of fixed work (operand build, rescoring), a split launch one merge
    for (int S = 1; S <= kFMaxSplits && S <= ntiles; ++S) {
        const int per = (ntiles + S - 1) / S;
        if (per * kFN > 65536) continue;
        const int Sr = (ntiles + per - 1) / per;
        const long long waves = ((long long)qb * Sr + sms - 1) / sms;
        const double cost = (double)waves * (per + 6) + (Sr > 1 ? 2.0 : 0.0);
        if (cost < best_cost) {
            best_cost = cost;
            best = Sr;
        }
    }
    return best;
}

cudaError_t route_tc_fused(const float* q, int nq, const uint16_t* ops, const float* cne, const float* cn_max,
                           const uint8_t* valid, int nlist, int d, const float* cent, int L, const int32_t* id_map,
                           int32_t* out_ids, uint64_t* out_keys, int32_t* row_fallback, uint64_t* split_keys,
                           uint32_t* row_bound, int splits, int* flag, cudaStream_t st) {
    if (nq <= 0) return cudaSuccess;
    if (!route_tc_fused_usable(d, nlist, L)) return cudaErrorInvalidValue;
    const int ntiles = (nlist + kFN - 1) / kFN;
    if (splits < 1) splits = 1;
    const int per = (ntiles + splits - 1) / splits;
    const int S = (ntiles + per - 1) / per;
    if (S > kFMaxSplits || per * kFN > 65536 || (S > 1 && !split_keys)) return cudaErrorInvalidValue;
    cudaError_t e = cudaMemsetAsync(row_fallback, 0, sizeof(int32_t) * (size_t)nq, st);
    if (e) return e;
    // 0x7f7f7f7f: a float above any distance, "no bound yet"
    if (row_bound && (e = cudaMemsetAsync(row_bound, 0x7f, sizeof(uint32_t) * (size_t)nq, st))) return e;
    const int lmax = fused_lmax(L), list = fused_list(lmax);
    const size_t region = route_fused_region(d, list);
    const size_t smem = route_fused_fixed(d, list) + region;
    const dim3 grid((unsigned)((nq + kTCM - 1) / kTCM), (unsigned)S);
    uint64_t* sk = S > 1 ? split_keys : nullptr;
    note_launch();
#define ISB_FUSED(LM)                                                                                            \
    {                                                                                                            \
        constexpr int LI = fused_list(LM);                                                                       \
        e = cudaFuncSetAttribute(route_tc_fused_kernel<LM, LI>, cudaFuncAttributeMaxDynamicSharedMemorySize,     \
                                 (int)smem);                                                                     \
        if (e) return e;                                                                                         \
        route_tc_fused_kernel<LM, LI><<<grid, kFBlock, smem, st>>>(q, nq, d, ops, cne, cn_max, valid, nlist,     \
                                                                    cent, L, id_map, per, (int)region, out_ids,  \
                                                                    out_keys, sk, row_bound, row_fallback, flag); \
    }
    if (lmax == 8) ISB_FUSED(8) else if (lmax == 16) ISB_FUSED(16) else ISB_FUSED(32)
#undef ISB_FUSED
    if ((e = cudaGetLastError())) return e;
    if (S > 1) {
        note_launch();
        route_split_merge_kernel<<<(unsigned)(((size_t)nq * 32 + 255) / 256), 256, 0, st>>>(sk, S, nq, L, out_ids,
                                                                                              out_keys);
        if ((e = cudaGetLastError())) return e;
    }
    note_launch();
    route_exact_rows_kernel<<<nq, kRsT, 0, st>>>(row_fallback, q, cent, valid, nlist, d, L, id_map, out_ids,
                                                 out_keys);
    return cudaGetLastError();
}

cudaError_t route_rescore(const uint32_t* approx, const float* q, int nq, const float* cent, const float* cn_max,
                          const uint8_t* valid, int nlist, int d, int L, const int32_t* id_map, int32_t* out_ids,
                          float* out_dist, uint64_t* out_keys, cudaStream_t st) {
    if (nq <= 0) return cudaSuccess;
    if (L <= 0 || L > kRsCap) return cudaErrorInvalidValue;
    const size_t smem = sizeof(float) * ((d + 3) & ~3) + sizeof(uint64_t) * kRsCap;
    cudaError_t e = cudaFuncSetAttribute(route_rescore_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e) return e;
    note_launch();
    route_rescore_kernel<<<nq, kRsT, smem, st>>>(approx, q, cent, cn_max, valid, nlist, d, L, id_map, out_ids,
                                                  out_dist, out_keys);
    return cudaGetLastError();
}

}  // namespace isb
