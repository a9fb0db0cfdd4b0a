// pq.cu -- residual-PQ ADC scan (with the update overlay) and exact rerank.
//
// Semantics (the reference's CPU statement of the math,
// cuda/search/cpu_fine/cpu_fine_kernels_pq_resid.cpp):
//   LUT[m][c] = sum_j ((q_j - cent_j) - cb[m][c][j])^2 in j order     (:176-189)
//   ADC(v)    = sum_m LUT[m][code_v[m]] in m order                     (:200-213)
//   stage 1   = the rerank_n best (ADC, position) of every probed list (:300-423)
//   stage 2   = unique candidates reranked exactly, top-k              (:431-519)
// and the overlay of updates/pq_update.cu:975-1055: published delta segments
// are scanned with the same LUTs and their best DELTA_TOPK candidates are
// reranked together with the main ones.
//
// Differences in design from the reference GPU runner (pq_update.cu:117-171):
//   * one CTA per (query, list) pair builds that pair's LUT once and scans the
//     whole list in chunks (the reference rebuilds the LUT per 2048-vector
//     chunk and lets only 256 of 1024 threads scan);
//   * selection is exact: the per-chunk keep-the-single-best-of-8 step of the
//     reference is replaced by the shared block filter, which keeps every key
//     that can still reach the query's top-R;
//   * main and delta pairs are work items of the same persistent launch, so
//     the overlay costs no extra launches or host round trips;
//   * the rerank runs on the device, not on host threads.
// Every sum uses __fadd_rn/__fmul_rn so no multiply-add is contracted and the
// results equal the CPU restatement bit for bit.
#include "emit.cuh"
#include "launch.h"

namespace isb {

namespace {

constexpr int kPT = 256;       // threads of the scan CTA
constexpr int kPChunk = kPQScanChunk;
constexpr int kPMaxD = 512;

template <int M>
__device__ __forceinline__ float adc_sum(const uint8_t* __restrict__ code, const float* __restrict__ lut) {
    float s = 0.f;
    if constexpr (M % 16 == 0) {
        const uint4* c4 = reinterpret_cast<const uint4*>(code);
        uint4 w[M / 16];
#pragma unroll
        for (int i = 0; i < M / 16; ++i) w[i] = __ldg(c4 + i);
#pragma unroll
        for (int i = 0; i < M / 16; ++i) {
            const uint32_t ww[4] = {w[i].x, w[i].y, w[i].z, w[i].w};
#pragma unroll
            for (int b = 0; b < 16; ++b) {
                const int m = i * 16 + b;
                const uint32_t c = (ww[b >> 2] >> (8 * (b & 3))) & 0xFFu;
                s = __fadd_rn(s, lut[m * kCodes + c]);
            }
        }
    } else {
        const uint2* c2 = reinterpret_cast<const uint2*>(code);
        uint2 w[M / 8];
#pragma unroll
        for (int i = 0; i < M / 8; ++i) w[i] = __ldg(c2 + i);
#pragma unroll
        for (int i = 0; i < M / 8; ++i) {
            const uint32_t ww[2] = {w[i].x, w[i].y};
#pragma unroll
            for (int b = 0; b < 8; ++b) {
                const int m = i * 8 + b;
                const uint32_t c = (ww[b >> 2] >> (8 * (b & 3))) & 0xFFu;
                s = __fadd_rn(s, lut[m * kCodes + c]);
            }
        }
    }
    return s;
}

template <int M>
__global__ void __launch_bounds__(kPT) pq_scan_kernel(PQParams p, WorkList wl, CandBuf cm, CandBuf cd,
                                                      int* counter) {
    extern __shared__ __align__(16) float smf[];
    float* lut = smf;                    // [M][256]
    float* resid = lut + M * kCodes;     // [d]
    float* dist = resid + kPMaxD;        // [kPChunk]
    __shared__ EmitSmem esm;
    __shared__ int s_item;
    const int tid = threadIdx.x;
    const int d = p.d, dsub = p.dsub;
    const int P = *wl.n_pairs;
    const int total = p.has_delta ? 2 * P : P;
    for (;;) {
        const int it = next_item(counter, total, &s_item);
        if (it < 0) break;
        const bool seg_delta = it >= P;
        const int pi = seg_delta ? it - P : it;
        const int q = wl.pair_q[pi], l = wl.pair_l[pi];
        const ListStore& S = seg_delta ? p.delta : p.main;
        const CandBuf& cb = seg_delta ? cd : cm;
        const int count = S.counts[l];
        if (count <= 0) continue;
        const int64_t off = S.offsets[l];
        const int64_t koff = S.key_off ? S.key_off[l] : off;
        const float* qv = p.q + (size_t)q * d;
        const float* cv = p.cent + (size_t)l * d;
        for (int j = tid; j < d; j += kPT) resid[j] = __fsub_rn(qv[j], cv[j]);
        __syncthreads();
        for (int e = tid; e < M * kCodes; e += kPT) {
            const int m = e >> 8;
            const float* cbv = p.codebook + (size_t)e * dsub;
            const float* rv = resid + m * dsub;
            float s = 0.f;
            for (int j = 0; j < dsub; ++j) {
                const float x = __fsub_rn(rv[j], __ldg(cbv + j));
                s = __fadd_rn(s, __fmul_rn(x, x));
            }
            lut[e] = s;
        }
        __syncthreads();
        for (int cs = 0; cs < count; cs += kPChunk) {
            const int len = min(kPChunk, count - cs);
            const uint8_t* codes = S.data + (size_t)(off + cs) * M;
            for (int v = tid; v < len; v += kPT) dist[v] = adc_sum<M>(codes + (size_t)v * M, lut);
            __syncthreads();
            const uint32_t kbase = (uint32_t)(koff + cs);
            auto keyf = [&](int i) -> uint64_t { return make_key(__float_as_uint(dist[i]), kbase + (uint32_t)i); };
            block_filter_emit<kPT>(keyf, len, cb, q, esm);
        }
    }
}


constexpr int kGQ = 4;      // queries per group

// ---------------------------------------------------------------------------
// Grouped phase-staggered ADC scan (M = 16, 32, 48 with dsub = 2, 4 or 8):
// the kernel the search uses for these shapes.
//
// A CTA takes one list and up to 4 probing queries (a group of the work list)
// and the four queries' LUTs are interleaved as float4 (a group of two or one
// query uses bank-shifted copies of a float2 or float table instead, so its
// gathers move only the entries it sums; see stagger_tile).  The M sub-quantizers
// form 8 blocks of MPL = M/8.  A warp is four groups of 8 lanes; lane j of a
// group sums the vectors 8k + j of its stripe, one block per step, blocks in
// order, so a vector takes 8 steps and is started at step 8k + j: at step x
// lane j works on block (x - j) mod 8, the 8 lanes of a group always on 8
// different blocks, and the lane whose block is 7 finishes vector x - 7.  A
// sum never leaves its lane (no shuffles), and every distance is the sum over
// m in m order.
//
// LUT row c holds entry m at float4 position p(m) = m/MPL + 8*(m%MPL): block
// b lies in the 16-byte bank group b of every row, so the 8 lanes of a group
// (one quarter-warp) read 8 distinct bank groups and each gather is
// conflict-free whatever the code values.
//
// Codes are re-laid out once per index (pq_build_gring) into tiles of 16
// steps.  Lane j's stream of tile T is the 16*MPL bytes b = i*MPL + s (step i,
// sub-quantizer s of the block) holding code[v][MPL*blk + s] with
// g = 16T + i - j, v = 8*floor(g/8) + j, blk = g mod 8 (0 outside the list);
// its 16-byte piece u = b/16 sits at tile offset (8u + j)*16, so each of a
// group's MPL 16-byte loads reads one whole 128-byte line, and the lane
// indexes the bytes statically.  A stripe starts on a multiple of 8 rows, on
// a tile or half way into one (load_tile takes half-tile indices).  With a
// published delta the scan may read a combined stream instead (mix_stripes):
// the same layout over positions that interleave each stripe's main and
// delta rows.
//
// The sums of queries (0,1) and (2,3) are float2 pairs added with the packed
// fp32x2 instructions (__fadd2_rn: two independent round-to-nearest adds).  A
// lane starts a vector with an FMA by 0 of its previous sum, which assumes
// finite LUT entries (an entry overflows only for |q - c| above 1e19).
// ---------------------------------------------------------------------------
constexpr int kRW = 8;                 // warps per CTA
constexpr int kRT = 32 * kRW;          // threads per CTA
constexpr int kRChunk = 2048;          // vectors per filtered chunk
constexpr int kRRings = 4 * kRW;       // 8-lane groups (stripes) per CTA
constexpr int kRSteps = kRChunk / kRRings;   // steps per filtered chunk (a multiple of 16)
static_assert(kRSteps % 16 == 0, "a chunk is whole tiles");

__host__ __device__ inline int64_t gring_tiles(int count) { return (int64_t)(count + 7) / 16 + 3; }
// vectors per stripe: count / kRRings rounded up to a multiple of 8 (half a tile)
__host__ __device__ inline int gring_stripe(int count) {
    return (int)(((int64_t)count + 8 * kRRings - 1) / (8 * kRRings)) * 8;
}
// The combined main + delta tile stream of a list (PQParams::mix): stripe r
// holds the main rows r*Sm .. r*Sm + Sm - 1 at its steps 0 .. Sm - 1 and the
// delta rows r*Sd .. r*Sd + Sd - 1 at its steps Sm .. Sm + Sd - 1 (each part
// only below its count), S = Sm + Sd rounded up to 8, kRRings * S positions in
// all: every warp takes a share of the delta rows in the same steps.
struct MixStripes {
    int Sm, Sd, S;
};
__host__ __device__ inline MixStripes mix_stripes(int cm, int cd) {
    MixStripes m;
    m.Sm = (cm + kRRings - 1) / kRRings;
    m.Sd = (cd + kRRings - 1) / kRRings;
    m.S = (m.Sm + m.Sd + 7) / 8 * 8;
    return m;
}
// filtered chunks of one list: stripe 0 takes min(S, count) + 7 steps
__host__ __device__ inline int gring_chunks(int count) {
    if (count <= 0) return 0;
    const int S = gring_stripe(count);
    return ((S < count ? S : count) + 7 + kRSteps - 1) / kRSteps;
}

template <int M>
struct GRing {
    static constexpr int MPL = M / 8;
    __host__ __device__ static constexpr int pos(int m) { return m / MPL + 8 * (m % MPL); }
    __host__ __device__ static constexpr int inv(int p) { return MPL * (p % 8) + p / 8; }
    static constexpr size_t smem_bytes() { return sizeof(float4) * ((size_t)256 * M + kRChunk); }
};

// NST steps (NST = 16: a whole tile; otherwise the first nst < 16) of one
// lane: at step i of the tile the lane is on block (i - j) mod 8 (tiles start
// on multiples of 16 steps).  In each window of 8 steps every lane finishes
// exactly one vector, at step 8w + ((j + 7) mod 8); the lane keeps its sums
// and at the window's end (or the tile's last step) all lanes store together,
// lane j to out[its finishing step]: one 16-byte store per lane per 8 steps.
// A stored sum at or below query k's bound thf sets bit k of maybe (a superset
// of the keys the chunk's filter can admit), except at the steps from xdr on
// (the delta rows of a combined main + delta stream, which the warp filters
// itself; xdr past the tile: none).
//
// Q = queries per LUT entry.  Q = 4: one table of float4 entries; a
// quarter-warp (one lane group) reads 8 distinct 16-byte bank groups.  Q = 2
// (M a multiple of 16): two copies of a float2 table, copy 1 with entry
// position p XOR 8; lane group g reads copy g & 1, so the two groups of a
// half-warp read disjoint halves of the banks.  Q = 1 (M = 32): four copies
// of a float table, copy g with position p XOR 8g; the four groups of a warp
// read four disjoint bank octets.  Each layout is conflict-free, and a gather
// costs 4, 2 or 1 wavefronts per warp.  In copy x entry m = MPL*blk + s sits
// at (blk + 8s) XOR 8x = blk + 8 (s XOR x).
template <int M, int NST, int Q>
__device__ __forceinline__ void stagger_tile(const float* __restrict__ lutf, const uint32_t (&w)[M / 2], int nst,
                                             int j, int g, float2& s01, float2& s23, float4* out, float4 thf,
                                             int xdr, uint32_t& maybe) {
    constexpr int MPL = M / 8;
    static_assert(Q == 4 || (Q == 2 && M % 16 == 0) || (Q == 1 && M == 32), "LUT layout");
    float4 fin = make_float4(0.f, 0.f, 0.f, 0.f);
    const int cp = Q == 4 ? 0 : (Q == 2 ? (g & 1) : g);             // the copy this lane group reads
#pragma unroll
    for (int i = 0; i < NST; ++i) {
        if (NST < 16 && i >= nst) break;
        const int blk = (i - j) & 7;
        const float2 k2 = blk == 0 ? make_float2(0.f, 0.f) : make_float2(1.f, 1.f);
#pragma unroll
        for (int s = 0; s < MPL; ++s) {
            const int byte = i * MPL + s;
            const uint32_t c = (w[byte >> 2] >> (8 * (byte & 3))) & 0xFFu;
            if constexpr (Q == 4) {
                const float4 f = reinterpret_cast<const float4*>(lutf)[c * M + blk + 8 * s];
                if (s == 0) {
                    s01 = __ffma2_rn(s01, k2, make_float2(f.x, f.y));
                    s23 = __ffma2_rn(s23, k2, make_float2(f.z, f.w));
                } else {
                    s01 = __fadd2_rn(s01, make_float2(f.x, f.y));
                    s23 = __fadd2_rn(s23, make_float2(f.z, f.w));
                }
            } else if constexpr (Q == 2) {
                const float2 f = reinterpret_cast<const float2*>(lutf)[(cp * 256 + c) * M + blk + 8 * (s ^ cp)];
                s01 = s == 0 ? __ffma2_rn(s01, k2, f) : __fadd2_rn(s01, f);
            } else {
                const float f = lutf[(cp * 256 + c) * M + blk + 8 * (s ^ cp)];
                s01.x = s == 0 ? __fmaf_rn(s01.x, k2.x, f) : __fadd_rn(s01.x, f);
            }
        }
        if (blk == 7) fin = make_float4(s01.x, Q >= 2 ? s01.y : 0.f, Q == 4 ? s23.x : 0.f, Q == 4 ? s23.y : 0.f);
        if ((i & 7) == 7 || (NST < 16 && i == nst - 1)) {
            const int fstep = (i & ~7) + ((j + 7) & 7);
            if (fstep <= i) {
                out[fstep] = fin;
                if (fstep < xdr) {
                    maybe |= (fin.x <= thf.x ? 1u : 0u);
                    if (Q >= 2) maybe |= (fin.y <= thf.y ? 2u : 0u);
                    if (Q == 4) maybe |= (fin.z <= thf.z ? 4u : 0u) | (fin.w <= thf.w ? 8u : 0u);
                }
            }
        }
    }
}

// 16-byte read-only load issued where it stands: the tile prefetch must leave
// a whole tile of steps between its issue and its use, so it is not left to
// the compiler to move it next to the use.
__device__ __forceinline__ uint4 ldg_v4_here(const uint4* ptr) {
    uint4 r;
    asm volatile("ld.global.nc.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(ptr)
                 : "memory");
    return r;
}

// The 16 steps of a lane from half-tile H on (tile H/2, or the second half of
// tile (H-1)/2 and the first half of the next for odd H): a tile's bytes are
// its lanes' 16-byte pieces u = 0..MPL-1 one after another (steps 8u/MPL ..
// of the lane in piece u), so the pieces from half a tile on are the same
// pieces 64*MPL bytes further, read with the same static byte indexing.
template <int MPL>
__device__ __forceinline__ void load_tile(const uint4* lanebase, int64_t H, uint32_t (&w)[4 * MPL]) {
    const uint4* tp = lanebase + H * (4 * MPL);   // half a tile is 64*MPL bytes = 4*MPL uint4
#pragma unroll
    for (int u = 0; u < MPL; ++u) {
        const uint4 x = ldg_v4_here(tp + 8 * u);
        w[4 * u] = x.x; w[4 * u + 1] = x.y; w[4 * u + 2] = x.z; w[4 * u + 3] = x.w;
    }
}

// small asynchronous global -> shared copies (sizes 4 and 8, naturally aligned)
__device__ __forceinline__ void cp_async_4(void* dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_async_8(void* dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// Shared-memory descriptor of the group a CTA takes next, fetched by thread 0
// while the current group runs: the packed group word first (stage A), then
// what it points to (stage B): the list's count, key offset and tile offset
// and the group's query ids (-1 past its size).
struct GroupDesc {
    int64_t pk, koff, goff;
    int count, q[kGQ];
    int64_t dkoff, dgoff;    // the same list's delta segment (when one is published)
    int64_t mgoff;           // the list's main and delta rows in one tile stream (PQParams::mix)
    int dcount;
};

__device__ __forceinline__ void desc_stage_a(GroupDesc& g, const WorkList& wl, int it, int NG) {
    cp_async_8(&g.pk, wl.groups + (it >= NG ? it - NG : it));
}

__device__ __forceinline__ void desc_stage_b(GroupDesc& g, const PQParams& p, const WorkList& wl, int it, int NG) {
    const int64_t pk = g.pk;
    const int l = (int)(pk >> 32), p0 = ((int)pk) >> 3, nqg = ((int)pk) & 7;
    const ListStore& S = it >= NG ? p.delta : p.main;
    cp_async_4(&g.count, S.counts + l);
    cp_async_8(&g.koff, (S.key_off ? S.key_off : S.offsets) + l);
    cp_async_8(&g.goff, S.gring_off + l);
    if (p.has_delta) {
        const ListStore& D = p.delta;
        cp_async_4(&g.dcount, D.counts + l);
        cp_async_8(&g.dkoff, (D.key_off ? D.key_off : D.offsets) + l);
        if (p.mix) cp_async_8(&g.mgoff, p.mix_off + l);
        else cp_async_8(&g.dgoff, D.gring_off + l);
    } else {
        g.dcount = 0;
    }
#pragma unroll
    for (int k = 0; k < kGQ; ++k) {
        if (k < nqg) cp_async_4(&g.q[k], wl.pair_q + p0 + k);
        else g.q[k] = -1;
    }
}

// Persistent CTA loop over the work list's groups.  Latency that does not
// depend on the group is taken off the group's critical path:
//   * the next group's descriptor is fetched into shared memory during this group;
//   * the next work item is claimed (atomic) while this group runs;
//   * the codebook rows a thread needs for its LUT column are requested
//     before the group is even decoded (they are the same for every group);
//   * the first code tile is requested before the LUT is built, each next
//     tile one tile ahead, and each chunk's query bounds before its steps.
template <int M, int DSUB, int DM>
__global__ void __launch_bounds__(kRT, 1) pq_stagger_kernel(PQParams p, WorkList wl, CandBuf cm, CandBuf cd,
                                                          int* counter) {
    using RG = GRing<M>;
    constexpr int MPL = RG::MPL;
    constexpr int d = M * DSUB;
    constexpr int kCStep = kRT / M;                              // codes a LUT builder thread strides by
    constexpr int kNC = (256 + kCStep - 1) / kCStep;             // codes per LUT builder thread, at most
    constexpr int kLB = kNC < 64 / DSUB ? kNC : 64 / DSUB;       // codebook rows in flight per thread
    extern __shared__ __align__(16) float smf[];
    float4* lut = reinterpret_cast<float4*>(smf);          // [256][M], entry m at pos(m)
    float4* dist4 = lut + 256 * M;                          // [kRChunk] four queries per vector
    float* resid = reinterpret_cast<float*>(dist4);         // [kGQ][d] while the LUT is built
    __shared__ EmitSmem esm;
    __shared__ int s_item;
    __shared__ __align__(8) GroupDesc s_gd;     // the group this CTA starts next
    // the current group's main and delta list (count, key offset, tile offset),
    // kept past the next group's descriptor fetch
    // [0] main rows, [1] delta rows, [2] both in one tile stream (PQParams::mix)
    __shared__ int64_t s_skoff[3], s_sgoff[3];
    __shared__ int s_scount[3];
    __shared__ unsigned long long s_thr1[kGQ];   // the second segment's bounds, read before the LUT build
    __shared__ unsigned long long s_thd[3][kGQ]; // each chunk's delta bounds (combined stream), buffers as s_cnt
    // per-chunk totals and "some sum may pass" bits of the 4 queries, three
    // buffers in rotation: chunk c adds into buffer c % 3 and, after its first
    // barrier, clears buffer (c + 2) % 3 -- last read in chunk c - 1 (done
    // before this barrier), next written in chunk c + 2 (after the next one)
    __shared__ int s_cnt[3][kGQ];
    __shared__ uint32_t s_any[3];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, grp = lane >> 3, j = lane & 7;
    // LUT builders: thread t owns LUT column ps = t % M (sub-quantizer inv(ps)) for codes t / M + kCStep * i
    const bool builder = tid < kCStep * M;
    const int ps = tid % M, mcol = RG::inv(ps), c0 = tid / M;
    const int NG = *wl.n_groups;
    const int total = NG;                    // a group scans its list's main and delta rows
    const int rid = warp * 4 + grp;          // stripe of this lane group
    if (tid < 3 * kGQ) s_cnt[tid / kGQ][tid % kGQ] = 0;
    if (tid < 3) s_any[tid] = 0;
    if (tid == 0) {
        s_item = atomicAdd(counter, 1);
        if (s_item < total) {
            desc_stage_a(s_gd, wl, s_item, NG);
            cp_async_wait_all();
            desc_stage_b(s_gd, p, wl, s_item, NG);
            cp_async_wait_all();
        }
    }
    __syncthreads();
    int cpar = 0;                       // buffer of s_cnt / s_any the next chunk adds into
    float cbv[kLB][DSUB];
    auto load_cb = [&](int cbase) {
#pragma unroll
        for (int b = 0; b < kLB; ++b) {
            const int c = min(cbase + b * kCStep, 255);
            const float* src = p.codebook_t + ((size_t)c * M + mcol) * DSUB;
            if constexpr (DSUB % 4 == 0) {
#pragma unroll
                for (int u = 0; u < DSUB; u += 4) {
                    const float4 t4 = __ldg(reinterpret_cast<const float4*>(src + u));
                    cbv[b][u] = t4.x; cbv[b][u + 1] = t4.y; cbv[b][u + 2] = t4.z; cbv[b][u + 3] = t4.w;
                }
            } else {
#pragma unroll
                for (int u = 0; u < DSUB; u += 2) {
                    const float2 t2 = __ldg(reinterpret_cast<const float2*>(src + u));
                    cbv[b][u] = t2.x; cbv[b][u + 1] = t2.y;
                }
            }
        }
    };
    for (;;) {
        const int it = s_item;
        if (it >= total) break;
        int nxt = 0;
        if (tid == 0) nxt = atomicAdd(counter, 1);       // used at the end of this group
        if (builder) load_cb(c0);
        const int64_t packed = s_gd.pk;
        const int l = (int)(packed >> 32), nqg = ((int)packed) & 7;
        // queries per LUT entry for this group (stagger_tile): 4, or 2 / 1 for
        // groups of two / one query (1 needs M = 32, else 2)
        const int qmode = nqg >= 3 ? 4 : (nqg == 2 || M != 32) ? 2 : 1;
        // the group's list in the main segment and, with the overlay, the same
        // list's delta rows: both are scanned here with the one LUT (read out of
        // s_gd before the next group's descriptor rewrites it)
        const int count_m = s_gd.count, count_d = DM ? s_gd.dcount : 0;
        if (tid == 0) {
            s_scount[0] = count_m;
            s_scount[1] = count_d;
            s_skoff[0] = s_gd.koff;
            s_sgoff[0] = s_gd.goff;
            s_skoff[1] = s_gd.dkoff;
            s_sgoff[1] = s_gd.dgoff;
            s_scount[2] = kRRings * mix_stripes(count_m, count_d).S;
            s_skoff[2] = s_gd.koff;
            s_sgoff[2] = DM == 2 ? s_gd.mgoff : 0;
        }
        bool fetched = false;            // thread 0: stage A of the next descriptor issued
        bool staged = false;             // thread 0: its stage B issued
        if (count_m > 0 || count_d > 0) {
            uint32_t w[4 * MPL], wn[4 * MPL];
            // segment seg's stripes and tiles (from s_gd for the first segment,
            // before the barrier that publishes the shared copies)
            auto seg_setup = [&](int seg, bool from_desc, const uint4*& lanebase, int64_t& hmax, int& S,
                                 int64_t& H0, int& wsteps, int& nchunks) {
                const int count = seg == 2 ? kRRings * mix_stripes(count_m, count_d).S : (seg ? count_d : count_m);
                const int64_t goff =
                    from_desc ? (seg == 2 ? s_gd.mgoff : (seg ? s_gd.dgoff : s_gd.goff)) : s_sgoff[seg];
                const uint8_t* tiles = (seg == 2 ? p.mix : (seg ? p.delta.gring : p.main.gring)) + goff;
                hmax = 2 * gring_tiles(count) - 2;    // last half tile a 16-step load may start on
                // Lane group r owns the stripe [r*S, r*S + S) of the list (S a
                // multiple of 8, so a stripe starts on a tile or half way into
                // one: half tile H0) and runs through it without draining: it
                // finishes vector r*S + x - 7 at step x.
                // Steps are cut into chunks of kRSteps; after each chunk the CTA
                // filters the kRRings * kRSteps finished slots.  The longest
                // stripe (group 0) takes min(S, count) + 7 steps.
                S = gring_stripe(count);
                const int a = rid * S < count ? rid * S : count;
                const int wa = warp * 4 * S;
                wsteps = wa < count ? min(S, count - wa) + 7 : 0;    // steps of this warp (its group 0)
                nchunks = gring_chunks(count);
                lanebase = reinterpret_cast<const uint4*>(tiles) + j;
                H0 = a / 8;
            };
            const uint4* lanebase;
            int64_t hmax, H0;
            int S, wsteps, nchunks;
            // With a delta segment the (short) delta rows go first and the
            // main rows second: the second segment's first tile is then
            // prefetched during the first segment's last tile (or, for a warp
            // with no steps in the first segment, right away), and its bounds
            // are read before the LUT build, so switching segments exposes no
            // global-memory latency.
            // With the combined tile stream of a list's main and delta rows
            // (built when the delta is published) both are scanned in one pass,
            // over stripes of the combined list: positions below the main count
            // are main rows, the others delta rows (segment 2).
            const int seg0 = DM == 2 ? 2 : DM == 1 && count_d > 0 ? 1 : 0;
            const int seg1 = DM == 1 && seg0 == 1 && count_m > 0 ? 0 : -1;
            seg_setup(seg0, true, lanebase, hmax, S, H0, wsteps, nchunks);
            const uint4* pre1 = nullptr;     // first tile of seg1 for this lane (null: none)
            if (DM == 1 && seg1 >= 0) {
                const uint4* lb1;
                int64_t hm1, H01;
                int S1, ws1, nc1;
                seg_setup(seg1, true, lb1, hm1, S1, H01, ws1, nc1);
                pre1 = lb1 + min(H01, hm1) * (4 * MPL);
            }
            bool have1 = false;              // w already holds seg1's first tile
            if (DM == 1 && pre1 && wsteps == 0) {
                load_tile<MPL>(pre1, 0, w);
                have1 = true;
            } else {
                load_tile<MPL>(lanebase, min(H0, hmax), w);
            }
            {
                const float* cv = p.cent + (size_t)l * d;
                for (int e = tid; e < kGQ * d; e += kRT) {
                    const int k = e / d, x = e - k * d;
                    const int qk = s_gd.q[k];
                    resid[e] = qk >= 0 ? __fsub_rn(p.q[(size_t)qk * d + x], cv[x]) : 0.f;
                }
            }
            // the group's bounds, requested before the LUT build and used after it
            // (the second segment's into shared memory, read when it starts)
            uint64_t thr0[kGQ];
            {
                const CandBuf& cb0 = seg0 == 1 ? cd : cm;
#pragma unroll
                for (int k = 0; k < kGQ; ++k)
                    thr0[k] = k < nqg ? *((volatile unsigned long long*)(cb0.thr + s_gd.q[k])) : 0ull;
                if (DM == 1 && seg1 >= 0 && tid < nqg)
                    s_thr1[tid] = *((volatile unsigned long long*)(cm.thr + s_gd.q[tid]));
            }
            __syncthreads();
            if (builder) {
                float2 r01[DSUB], r23[DSUB];
#pragma unroll
                for (int u = 0; u < DSUB; ++u) {
                    r01[u] = make_float2(resid[mcol * DSUB + u], resid[d + mcol * DSUB + u]);
                    r23[u] = make_float2(resid[2 * d + mcol * DSUB + u], resid[3 * d + mcol * DSUB + u]);
                }
                for (int cb0 = c0;; cb0 += kLB * kCStep) {
#pragma unroll
                    for (int b = 0; b < kLB; ++b) {
                        const int c = cb0 + b * kCStep;
                        if (c >= 256) break;
                        // scalar round-to-nearest operations: a packed fp32x2 multiply
                        // feeding a packed add was measured not to reproduce the
                        // separately rounded x*x + a of the CPU statement
                        // entries of the group's absent queries are left 0 (their
                        // sums are never compared): a group of one or two queries
                        // builds a quarter or half of the table
                        float acc[kGQ];
#pragma unroll
                        for (int kq = 0; kq < kGQ; ++kq) {
                            float a = 0.f;
                            if (kq > 0 && kq >= nqg) {
                                acc[kq] = 0.f;
                                continue;
                            }
#pragma unroll
                            for (int u = 0; u < DSUB; ++u) {
                                const float r = kq == 0 ? r01[u].x : kq == 1 ? r01[u].y : kq == 2 ? r23[u].x : r23[u].y;
                                const float x = __fsub_rn(r, cbv[b][u]);
                                a = u == 0 ? __fmul_rn(x, x) : __fadd_rn(a, __fmul_rn(x, x));
                            }
                            acc[kq] = a;
                        }
                        if (qmode == 4) {
                            lut[c * M + ps] = make_float4(acc[0], acc[1], acc[2], acc[3]);
                        } else if (qmode == 2) {        // copies 0 and 1 (position XOR 8)
                            float2* l2 = reinterpret_cast<float2*>(smf);
                            const float2 v = make_float2(acc[0], acc[1]);
                            l2[c * M + ps] = v;
                            l2[(256 + c) * M + (ps ^ 8)] = v;
                        } else if constexpr (M == 32) {  // copies 0..3 (position XOR 8x)
#pragma unroll
                            for (int x = 0; x < 4; ++x) smf[(256 * x + c) * M + (ps ^ (8 * x))] = acc[0];
                        }
                    }
                    if (cb0 + kLB * kCStep >= 256) break;
                    load_cb(cb0 + kLB * kCStep);
                }
            }
            __syncthreads();
            // the query ids are read before the next group's fetch rewrites them
            // (its stage B starts after the first chunk's barrier)
            int qid[kGQ];
#pragma unroll
            for (int k = 0; k < kGQ; ++k) qid[k] = s_gd.q[k];
            if (tid == 0 && nxt < total) {
                desc_stage_a(s_gd, wl, nxt, NG);
                fetched = true;
            }
            float2 s01 = make_float2(0.f, 0.f), s23 = make_float2(0.f, 0.f);
            // float form of the bounds for the stores' pass test, taken from bounds
            // already in registers (the group's first, then each chunk's cut): a
            // bound only decreases, so an older one only sets more bits.  A bound
            // at or above +inf bits admits everything: its bit is forced on.
            float4 thf;
            uint32_t force;
            auto set_thf = [&](const uint64_t (&b)[kGQ]) {
                float tf[kGQ];
                force = 0;
#pragma unroll
                for (int k = 0; k < kGQ; ++k) {
                    const uint32_t hi = (uint32_t)(b[k] >> 32);
                    tf[k] = k < nqg && hi < 0x7f800000u ? __uint_as_float(hi) : -1.f;
                    if (k < nqg && hi >= 0x7f800000u) force |= 1u << k;
                }
                thf = make_float4(tf[0], tf[1], tf[2], tf[3]);
            };
            for (int si = 0; si < (DM == 1 ? 2 : 1); ++si) {
            const int seg = si == 0 ? seg0 : seg1;
            if (seg < 0) break;
            const int count = s_scount[seg];
            if (count == 0) continue;
            const CandBuf& cb = seg == 1 ? cd : cm;
            const uint32_t kbase = (uint32_t)s_skoff[seg];
            // combined stream: each stripe's main rows, then its delta rows (key base dkbase)
            const MixStripes ms = mix_stripes(DM == 2 ? count_m : 0, DM == 2 ? count_d : 0);
            const uint32_t dkbase = (uint32_t)s_skoff[1];
            if (si == 1) {                     // the main rows after the delta rows: same LUT
                seg_setup(seg, false, lanebase, hmax, S, H0, wsteps, nchunks);
                if (!have1) load_tile<MPL>(lanebase, min(H0, hmax), w);
                pre1 = nullptr;
#pragma unroll
                for (int k = 0; k < kGQ; ++k) thr0[k] = k < nqg ? s_thr1[k] : 0ull;
                s01 = make_float2(0.f, 0.f);
                s23 = make_float2(0.f, 0.f);
            }
            set_thf(thr0);
            // first step at which a lane group finishes a delta row of the
            // combined stream (stripe step Sm, finished 7 steps later)
            const int xd = DM == 2 ? ms.Sm + 7 : 0x7FFFFFFF;
            for (int t = 0; t < nchunks; ++t) {
                uint64_t thr[kGQ];    // read now, used after the steps: a bound only ever decreases
#pragma unroll
                for (int k = 0; k < kGQ; ++k)
                    thr[k] = k < nqg ? *((volatile unsigned long long*)(cb.thr + qid[k])) : 0ull;
                // the delta bounds land in shared memory during the steps (an older
                // copy of a bound is only a looser one)
                if (DM == 2 && warp == 1 && lane < nqg) cp_async_8(&s_thd[cpar][lane], cd.thr + (lane == 0 ? qid[0] : lane == 1 ? qid[1] : lane == 2 ? qid[2] : qid[3]));
                uint32_t maybe = 0;
#pragma unroll 1
                for (int tl = 0; tl < kRSteps / 16; ++tl) {
                    const int x0 = t * kRSteps + 16 * tl;
                    if (x0 >= wsteps) break;
                    if (DM == 1 && pre1 && x0 + 16 >= wsteps) {     // this warp's last tile of seg0
                        load_tile<MPL>(pre1, 0, wn);
                        have1 = true;
                    } else {
                        load_tile<MPL>(lanebase, min(H0 + 2 * (x0 / 16 + 1), hmax), wn);
                    }
                    // slot of (group r, step s of the chunk) = r * kRSteps + s
                    float4* out = dist4 + rid * kRSteps + 16 * tl;
                    const bool full = wsteps - x0 >= 16;
                    if (qmode == 4) {
                        if (full) stagger_tile<M, 16, 4>(smf, w, 16, j, grp, s01, s23, out, thf, xd - x0, maybe);
                        else stagger_tile<M, 15, 4>(smf, w, wsteps - x0, j, grp, s01, s23, out, thf, xd - x0, maybe);
                    } else if (M != 32 || qmode == 2) {
                        if (full) stagger_tile<M, 16, 2>(smf, w, 16, j, grp, s01, s23, out, thf, xd - x0, maybe);
                        else stagger_tile<M, 15, 2>(smf, w, wsteps - x0, j, grp, s01, s23, out, thf, xd - x0, maybe);
                    } else {
                        if (full) stagger_tile<M, 16, (M == 32 ? 1 : 2)>(smf, w, 16, j, grp, s01, s23, out, thf, xd - x0, maybe);
                        else stagger_tile<M, 15, (M == 32 ? 1 : 2)>(smf, w, wsteps - x0, j, grp, s01, s23, out, thf,
                                                                   xd - x0, maybe);
                    }
#pragma unroll
                    for (int u = 0; u < 4 * MPL; ++u) w[u] = wn[u];
                }
                maybe = __reduce_or_sync(0xffffffffu, maybe);
                if (lane == 0 && (maybe | force)) atomicOr(&s_any[cpar], maybe | force);
                if (DM == 2 && warp == 1) cp_async_wait_all();
                __syncthreads();
                if (DM == 2) {
                    // The delta rows of the combined stream that this warp's stripes
                    // finished in the chunk, against the delta bounds.  The warp
                    // wrote their slots itself (no block barrier is needed to read
                    // them, and the next writes to them are its own); lane i takes
                    // the warp's i-th such row (each stripe holds about 1/32 of the
                    // list's delta rows, so usually one pass of 32).  A query with
                    // more passing keys than the delta rank Rd gets a new bound: the
                    // Rd-th smallest of any Rd or more existing keys bounds the
                    // rank-Rd key from above.
                    const int va = t * kRSteps >= 7 ? t * kRSteps - 7 : 0, vb = min(S, t * kRSteps + kRSteps - 7);
                    int lo[4], ln[4], m = 0;
#pragma unroll
                    for (int g4 = 0; g4 < 4; ++g4) {
                        const int r = 4 * warp + g4;
                        const int dl = min(ms.Sd, max(0, count_d - r * ms.Sd));     // delta rows of stripe r
                        const int a = max(ms.Sm, va), b = min(ms.Sm + dl, vb);     // stripe steps, less 7
                        lo[g4] = a;
                        ln[g4] = b > a ? b - a : 0;
                        m += ln[g4];
                    }
                    if (m > 0) {
                        // item i of the warp's rows: its four sums and delta position
                        auto item = [&](int i, float4& fv, uint32_t& dp) -> bool {
                            if (i >= m) return false;
                            int g4 = 0, a = lo[0];
                            if (i >= ln[0]) {
                                i -= ln[0]; g4 = 1; a = lo[1];
                                if (i >= ln[1]) {
                                    i -= ln[1]; g4 = 2; a = lo[2];
                                    if (i >= ln[2]) { i -= ln[2]; g4 = 3; a = lo[3]; }
                                }
                            }
                            const int xs = a + i, r = 4 * warp + g4;
                            fv = dist4[r * kRSteps + (xs + 7 - t * kRSteps)];
                            dp = (uint32_t)(r * ms.Sd + xs - ms.Sm);
                            return true;
                        };
                        auto dkey = [&](bool ok, const float4& fv, uint32_t dp, int k) -> uint64_t {
                            const float dk = k == 0 ? fv.x : k == 1 ? fv.y : k == 2 ? fv.z : fv.w;
                            return ok ? make_key(__float_as_uint(dk), dkbase + dp) : kKeyNone;
                        };
                        uint64_t bnd[kGQ];
                        int nk[kGQ];
                        auto count_pass = [&]() {
#pragma unroll
                            for (int k = 0; k < kGQ; ++k) nk[k] = 0;
                            for (int i0 = 0; i0 < m; i0 += 32) {
                                float4 fv;
                                uint32_t dp;
                                const bool ok = item(i0 + lane, fv, dp);
#pragma unroll
                                for (int k = 0; k < kGQ; ++k)
                                    if (k < nqg) nk[k] += __popc(__ballot_sync(0xffffffffu, dkey(ok, fv, dp, k) <= bnd[k]));
                            }
                        };
#pragma unroll
                        for (int k = 0; k < kGQ; ++k) {
                            const unsigned long long b = k < nqg ? s_thd[cpar][k] : 0ull;
                            bnd[k] = b < kKeyNone - 1 ? b : kKeyNone - 1;
                        }
                        count_pass();
                        if (cd.R <= 32) {
                            float4 fv;
                            uint32_t dp;
                            const bool ok = item(lane, fv, dp);
                            bool cut = false;
#pragma unroll
                            for (int k = 0; k < kGQ; ++k) {
                                if (k >= nqg || nk[k] <= cd.R) continue;
                                const uint64_t kk = dkey(ok, fv, dp, k);
                                const bool pass = kk <= bnd[k];
                                if (__popc(__ballot_sync(0xffffffffu, pass)) < cd.R) continue;
                                const uint64_t mk = warp_sort32(pass ? kk : kKeyNone);
                                const uint64_t c = __shfl_sync(0xffffffffu, mk, cd.R - 1);
                                if (c < bnd[k]) {
                                    bnd[k] = c;
                                    cut = true;
                                    if (lane == 0) atomicMin(cd.thr + qid[k], (unsigned long long)c);
                                }
                            }
                            if (cut) count_pass();
                        }
                        // one atomic per query, the queries' in flight together
                        const int myn = lane == 0 ? nk[0] : lane == 1 ? nk[1] : lane == 2 ? nk[2] : nk[3];
                        const int myq = lane == 0 ? qid[0] : lane == 1 ? qid[1] : lane == 2 ? qid[2] : qid[3];
                        int mybase = 0;
                        if (lane < nqg && myn > 0) mybase = atomicAdd(cd.cnt + myq, myn);
                        int at[kGQ];
#pragma unroll
                        for (int k = 0; k < kGQ; ++k) at[k] = __shfl_sync(0xffffffffu, mybase, k);
                        for (int i0 = 0; i0 < m; i0 += 32) {
                            float4 fv;
                            uint32_t dp;
                            const bool ok = item(i0 + lane, fv, dp);
#pragma unroll
                            for (int k = 0; k < kGQ; ++k) {
                                if (k >= nqg || nk[k] == 0) continue;
                                const uint64_t kk = dkey(ok, fv, dp, k);
                                const bool pass = kk <= bnd[k];
                                const unsigned ball = __ballot_sync(0xffffffffu, pass);
                                if (pass) {
                                    const int i = at[k] + __popc(ball & ((1u << lane) - 1u));
                                    if (i < cd.cap) cd.keys[(size_t)qid[k] * cd.cap + i] = kk;
                                    else atomicExch(cd.overflow, 1);
                                }
                                at[k] += __popc(ball);
                            }
                        }
                    }
                }
                if (tid == 0 && fetched && !staged) {         // stage A landed long ago
                    cp_async_wait_all();
                    desc_stage_b(s_gd, p, wl, nxt, NG);
                    staged = true;
                }
                const int cfree = cpar == 0 ? 2 : cpar - 1;      // (cpar + 2) % 3
                if (tid < kGQ) s_cnt[cfree][tid] = 0;
                if (tid == 0) s_any[cfree] = 0;
                if (s_any[cpar] == 0) {          // no sum of the chunk can pass any bound
                    cpar = cpar == 2 ? 0 : cpar + 1;
                    set_thf(thr);
                    continue;
                }
                // thread t reads the slots t + kRT*e: group t/64 + 4e, chunk step
                // t % 64, i.e. vectors (t/64 + 4e)*S + t*kRSteps + t%64 - 7.
                // All of them are read into registers before the totals'
                // barrier, so the next chunk may overwrite the slots as soon as
                // that has passed.
                constexpr int kE = kRRings * kRSteps / kRT;
                float4 f[kE];
                uint32_t vid[kE];     // list position, or 0xFFFFFFFF for no vector
#pragma unroll
                for (int e = 0; e < kE; ++e) {
                    const int x = t * kRSteps + (tid % kRSteps), rr = tid / kRSteps + (kRT / kRSteps) * e;
                    if (DM == 2) {           // the main rows of the combined stream
                        const int mi = rr * ms.Sm + x - 7;
                        vid[e] = (x >= 7 && x - 7 < ms.Sm && mi < count_m) ? (uint32_t)mi : 0xFFFFFFFFu;
                    } else {
                        const int v = rr * S + x - 7;
                        vid[e] = (x >= 7 && x - 7 < S && v < count) ? (uint32_t)v : 0xFFFFFFFFu;
                    }
                    f[e] = vid[e] != 0xFFFFFFFFu ? dist4[tid + kRT * e] : make_float4(0.f, 0.f, 0.f, 0.f);
                }
                int cnt4[kGQ];
#pragma unroll
                for (int k = 0; k < kGQ; ++k) {
                    thr[k] = thr[k] < kKeyNone - 1 ? thr[k] : kKeyNone - 1;    // never admits kKeyNone
                    cnt4[k] = 0;
                }
                auto key_of = [&](int e, int k) -> uint64_t {
                    const float dk = k == 0 ? f[e].x : k == 1 ? f[e].y : k == 2 ? f[e].z : f[e].w;
                    return vid[e] != 0xFFFFFFFFu ? make_key(__float_as_uint(dk), kbase + vid[e]) : kKeyNone;
                };
#pragma unroll
                for (int e = 0; e < kE; ++e)
#pragma unroll
                    for (int k = 0; k < kGQ; ++k) cnt4[k] += (k < nqg && key_of(e, k) <= thr[k]) ? 1 : 0;
                const int4 tot = block_sum4_once<kRT>(make_int4(cnt4[0], cnt4[1], cnt4[2], cnt4[3]), s_cnt[cpar]);
                cpar = cpar == 2 ? 0 : cpar + 1;
                const int totk[kGQ] = {tot.x, tot.y, tot.z, tot.w};
                // queries with more than R keys under their bound get a new
                // bound that admits R .. R + slack of them (one shared descent
                // whose histograms use the slots, already in registers)
                unsigned sel = 0;
                uint64_t cut[kGQ];
#pragma unroll
                for (int k = 0; k < kGQ; ++k) {
                    cut[k] = thr[k];
                    if (k < nqg && totk[k] > cb.R) sel |= 1u << k;
                }
                if (sel) {
                    uint64_t cs[kGQ];
                    block_cut_items<kRT, kE, kGQ>(key_of, sel, cb.R, cb.slack, thr, reinterpret_cast<int*>(dist4),
                                                  esm.bc, esm.mm, cs);
#pragma unroll
                    for (int k = 0; k < kGQ; ++k) {
                        if (!((sel >> k) & 1u)) continue;
                        cut[k] = cs[k] < thr[k] ? cs[k] : thr[k];
                        if (tid == 0) atomicMin(cb.thr + qid[k], (unsigned long long)cut[k]);
                    }
                }
#pragma unroll
                for (int k = 0; k < kGQ; ++k)
                    if (k < nqg && totk[k] > 0)
                        warp_append_items<kE>([&](int e) { return key_of(e, k); }, cut[k], cb, qid[k]);
                if (sel) __syncthreads();     // the histograms lived in the slots
                set_thf(cut);
            }
            }
        }
        if (tid == 0) {
            if (fetched && !staged) {          // lists too short for a chunk barrier after the fetch
                cp_async_wait_all();
                desc_stage_b(s_gd, p, wl, nxt, NG);
            }
            if (nxt < total && !fetched) {    // an empty list: fetch the next descriptor now
                desc_stage_a(s_gd, wl, nxt, NG);
                cp_async_wait_all();
                desc_stage_b(s_gd, p, wl, nxt, NG);
            }
            cp_async_wait_all();
            s_item = nxt;
        }
        __syncthreads();
    }
}

// one launch per search pass: with a published delta segment every group also
// scans its list's delta rows, in the combined tile stream (DM = 2) or after
// the main rows from the delta's own tiles (DM = 1)
template <int M, int DSUB, int DM>
cudaError_t launch_gring_seg(const PQParams& p, WorkList wl, int max_groups, CandBuf cm, CandBuf cd, int* counter,
                             cudaStream_t st) {
    const size_t smem = GRing<M>::smem_bytes();
    cudaError_t e = cudaFuncSetAttribute(pq_stagger_kernel<M, DSUB, DM>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e) return e;
    int dev = 0, sms = 148, per_sm = 1;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, pq_stagger_kernel<M, DSUB, DM>, kRT, smem);
    if (per_sm < 1) return cudaErrorInvalidConfiguration;
    long long items = (long long)max_groups;
    long long grid = (long long)sms * per_sm;
    if (grid > items) grid = items;
    if (grid < 1) grid = 1;
    note_launch();
    pq_stagger_kernel<M, DSUB, DM><<<(int)grid, kRT, smem, st>>>(p, wl, cm, cd, counter);
    return cudaGetLastError();
}

template <int M, int DSUB>
cudaError_t launch_gring(const PQParams& p, WorkList wl, int max_groups, CandBuf cm, CandBuf cd, int* counter,
                         cudaStream_t st) {
    if (p.has_delta && p.mix) return launch_gring_seg<M, DSUB, 2>(p, wl, max_groups, cm, cd, counter, st);
    if (p.has_delta) return launch_gring_seg<M, DSUB, 1>(p, wl, max_groups, cm, cd, counter, st);
    return launch_gring_seg<M, DSUB, 0>(p, wl, max_groups, cm, cd, counter, st);
}

template <int MPL>
__global__ void gring_layout_kernel(const uint8_t* __restrict__ codes, const int64_t* __restrict__ offsets,
                                    const int32_t* __restrict__ counts, const int64_t* __restrict__ tile_off,
                                    int nlist, int M, uint8_t* __restrict__ out) {
    for (int l = blockIdx.x; l < nlist; l += gridDim.x) {
        const int cnt = counts[l];
        const int64_t off = offsets[l];
        const int64_t total = gring_tiles(cnt) * 128 * MPL;
        uint8_t* dst = out + tile_off[l];
        for (int64_t e = threadIdx.x; e < total; e += blockDim.x) {
            const int64_t T = e / (128 * MPL);
            const int r = (int)(e % (128 * MPL));
            const int u = r / 128, jj = (r % 128) / 16, b = 16 * u + r % 16, i = b / MPL, s = b % MPL;
            const int64_t g = 16 * T + i - jj;
            const int64_t g8 = g >= 0 ? g / 8 : -((7 - g) / 8);      // floor(g / 8)
            const int blk = (int)(g - 8 * g8);
            const int64_t v = 8 * g8 + jj;
            dst[e] = (v >= 0 && v < cnt) ? codes[(size_t)(off + v) * M + MPL * blk + s] : (uint8_t)0;
        }
    }
}

// byte offset, inside a list's tiles, of sub-quantizer byte s of block b of
// vector v (the inverse of gring_layout_kernel's mapping; v >= 0)
template <int MPL>
__device__ __forceinline__ int64_t gring_byte(int64_t v, int b, int s) {
    const int j = (int)(v & 7);
    const int64_t g = (v - j) + b + j;          // 16T + i
    const int64_t T = g / 16;
    const int i = (int)(g % 16), byte = i * MPL + s;
    return T * 128 * MPL + (int64_t)(8 * (byte / 16) + j) * 16 + byte % 16;
}

// combined tiles of list l (mix_stripes): position p = r*S + x of stripe r
// holds main row r*Sm + x for x < Sm, delta row r*Sd + x - Sm for Sm <= x <
// Sm + Sd (each below its count), zeros otherwise; bytes come from the main
// and delta grouped-ring tiles
template <int MPL>
__global__ void gring_mix_kernel(const uint8_t* __restrict__ mt, const int64_t* __restrict__ moff,
                                 const int32_t* __restrict__ mcnt, const uint8_t* __restrict__ dt,
                                 const int64_t* __restrict__ doff, const int32_t* __restrict__ dcnt,
                                 const int64_t* __restrict__ xoff, int nlist, uint8_t* __restrict__ out) {
    for (int l = blockIdx.x; l < nlist; l += gridDim.x) {
        const int cm = mcnt[l], cdl = dcnt[l];
        const MixStripes ms = mix_stripes(cm, cdl);
        const int64_t np = (int64_t)kRRings * ms.S;
        const int64_t total = gring_tiles((int)np) * 128 * MPL;
        const uint8_t* src_m = mt + moff[l];
        const uint8_t* src_d = dt + doff[l];
        uint8_t* dst = out + xoff[l];
        for (int64_t e = threadIdx.x; e < total; e += blockDim.x) {
            const int64_t T = e / (128 * MPL);
            const int r = (int)(e % (128 * MPL));
            const int u = r / 128, jj = (r % 128) / 16, b = 16 * u + r % 16, i = b / MPL, s = b % MPL;
            const int64_t g = 16 * T + i - jj;
            const int64_t g8 = g >= 0 ? g / 8 : -((7 - g) / 8);      // floor(g / 8)
            const int blk = (int)(g - 8 * g8);
            const int64_t v = 8 * g8 + jj;
            uint8_t val = 0;
            if (v >= 0 && v < np) {
                const int st = (int)(v / ms.S), x = (int)(v % ms.S);
                if (x < ms.Sm) {
                    const int64_t mi = (int64_t)st * ms.Sm + x;
                    if (mi < cm) val = src_m[gring_byte<MPL>(mi, blk, s)];
                } else if (x < ms.Sm + ms.Sd) {
                    const int64_t di = (int64_t)st * ms.Sd + (x - ms.Sm);
                    if (di < cdl) val = src_d[gring_byte<MPL>(di, blk, s)];
                }
            }
            dst[e] = val;
        }
    }
}

template <int M>
cudaError_t launch_scan(const PQParams& p, WorkList wl, int max_pairs, CandBuf cm, CandBuf cd, int* counter,
                        cudaStream_t st) {
    size_t smem = sizeof(float) * ((size_t)M * kCodes + kPMaxD + kPChunk);
    cudaError_t e = cudaFuncSetAttribute(pq_scan_kernel<M>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e) return e;
    int dev = 0, sms = 148, per_sm = 1;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, pq_scan_kernel<M>, kPT, smem);
    if (per_sm < 1) per_sm = 1;
    long long items = (long long)max_pairs * (p.has_delta ? 2 : 1);
    long long grid = (long long)sms * per_sm;
    if (grid > items) grid = items;
    if (grid < 1) grid = 1;
    note_launch();
    pq_scan_kernel<M><<<(int)grid, kPT, smem, st>>>(p, wl, cm, cd, counter);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// rerank
// ---------------------------------------------------------------------------
constexpr int kRRT = 256;
// slots of the rerank's repeat table for np candidates: at least twice np and
// room for the per-warp top-k lists (8 warps x 16)
__host__ __device__ constexpr int rr_table(int np) { return 2 * np > 256 ? 2 * np : 256; }
constexpr int kRRMax = 4096;  // R + Rd candidates per query

// local position of a ranking-key position (shards rank by global positions)
__device__ __forceinline__ int64_t local_pos(const ListStore& S, uint32_t kpos, int nlist) {
    if (!S.key_off) return (int64_t)kpos;
    int lo = 0, hi = nlist - 1;
    while (lo < hi) {  // last list whose key_off <= kpos
        int mid = (lo + hi + 1) >> 1;
        if (S.key_off[mid] <= (int64_t)kpos) lo = mid; else hi = mid - 1;
    }
    return S.offsets[lo] + ((int64_t)kpos - S.key_off[lo]);
}

__device__ __forceinline__ uint8_t to_u8(float x) {  // updates/exact_update.cu:410-418
    x = fminf(fmaxf(x, 0.f), 255.f);
    return (uint8_t)lroundf(x);
}

// Inserts key into an open-addressing table of mask + 1 slots (empty =
// kKeyNone); true for the first insertion of a key, false for a repeat.  The
// table has at least twice as many slots as keys, so the probe loop ends.
__device__ __forceinline__ bool hash_first(unsigned long long* tab, int mask, uint64_t key) {
    int h = (int)((key * 0x9E3779B97F4A7C15ull) >> 40) & mask;
    for (int probe = 0; probe <= mask; ++probe) {
        const unsigned long long old = atomicCAS(&tab[h], (unsigned long long)kKeyNone, (unsigned long long)key);
        if (old == kKeyNone) return true;
        if (old == key) return false;
        h = (h + 1) & mask;
    }
    return false;
}

// Exact rerank of one query's stage-1 candidates (CTA per query).  Four threads
// share a candidate row: for the fp32 distance thread `sub` owns the lanes
// 4 sub .. 4 sub + 3 of the reference's 16-lane AVX-512 arithmetic
// (cuda/search/cpu_fine/cpu_fine_kernels_pq_resid.cpp:106-131: per block of 16
// dimensions acc[l] = fma(q - v, q - v, acc[l]), then the 512-bit horizontal
// add, a pairwise tree l + 8, + 4, + 2, + 1), so its 16-byte loads of a block
// are one coalesced 64-byte piece of the row and the tree's first two levels
// are shuffles inside the group of four.  The u8 distance is an exact int32
// sum, split the same way.  NB = d / 16 when the row length is a template
// constant (all loads of a row issued before the arithmetic), 0 for any d.
template <int NB>
__global__ void __launch_bounds__(kRRT) pq_rerank_kernel(PQParams p, int nlist, const uint64_t* __restrict__ s1m,
                                                         int R, const uint64_t* __restrict__ s1d, int Rd, int k,
                                                         int32_t* out_ids, float* out_dist, uint64_t* out_exm,
                                                         uint64_t* out_exd, const uint64_t* __restrict__ kmax,
                                                         uint64_t* out_topk) {
    extern __shared__ uint64_t sk[];            // [np] exact keys, [np] stage-1 keys, a table of rr_table(np) slots
    __shared__ __align__(16) float sq[kPMaxD];
    __shared__ int s_live;
    __shared__ __align__(16) uint8_t squ[kPMaxD];
    const int q = blockIdx.x, tid = threadIdx.x, lane = tid & 31, d = p.d;
    const int nb = NB ? NB : d / 16;
    const bool f32 = p.main.rr_f32 != nullptr;
    const int nc = R + Rd;
    const uint64_t km = kmax ? kmax[q] : kKeyNone;   // main keys above it are not candidates (a shard's part)
    int np = 1;
    while (np < nc) np <<= 1;
    uint64_t* s1 = sk + np;
    unsigned long long* tab = reinterpret_cast<unsigned long long*>(sk + 2 * np);
    const int tmask = rr_table(np) - 1;
    for (int j = tid; j < d; j += kRRT) {
        float x = p.q[(size_t)q * d + j];
        sq[j] = x;
        squ[j] = to_u8(x);
    }
    if (tid == 0) s_live = 0;
    if (!out_exm)
        for (int i = tid; i <= tmask; i += kRRT) tab[i] = kKeyNone;
    __syncthreads();
    // every candidate's stage-1 key in one coalesced pass (kKeyNone above the
    // query's key limit and past the end).  The per-candidate keys of a
    // cross-shard merge keep their slots; the final top-k path packs the live
    // keys to the front (one shared add per warp), delta keys tagged by bit 63
    // (a distance's sign bit, always clear in a key), and works only on those.
    for (int c0 = 0; c0 < np; c0 += kRRT) {
        const int c = c0 + tid;
        uint64_t key = kKeyNone;
        if (c < R) {
            const uint64_t km1 = s1m[(size_t)q * R + c];
            key = km1 <= km ? km1 : kKeyNone;
        } else if (c < nc) {
            key = s1d[(size_t)q * Rd + (c - R)];
            if (!out_exm && key != kKeyNone) key |= 1ull << 63;
        }
        if (out_exm) {
            if (c < np) s1[c] = key;
            continue;
        }
        const bool ok = key != kKeyNone;
        const unsigned ball = __ballot_sync(0xffffffffu, ok);
        int base = 0;
        if (lane == 0 && ball) base = atomicAdd(&s_live, __popc(ball));
        base = __shfl_sync(0xffffffffu, base, 0);
        if (ok) s1[base + __popc(ball & ((1u << lane) - 1u))] = key;
    }
    __syncthreads();
    const int nlive = out_exm ? np : s_live;
    const int grp = tid >> 2, sub = tid & 3;
    for (int c0 = 0; c0 < nlive; c0 += kRRT / 4) {
        const int c = c0 + grp;
        bool live = false, dl = false;
        uint64_t key = kKeyNone;
        if (c < nlive) {
            key = s1[c];
            if (out_exm) {
                dl = c >= R;
                live = key != kKeyNone;
            } else {
                dl = (key >> 63) != 0;
                // the final top-k reranks each position once (a list probed
                // twice repeats its keys in stage 1)
                if (sub == 0) live = hash_first(tab, tmask, key);
                key &= ~(1ull << 63);
            }
        }
        if (!out_exm) live = __shfl_sync(0xffffffffu, live, lane & ~3);
        const ListStore& S = dl ? p.delta : p.main;
        int64_t lp = live ? local_pos(S, key_lo(key), nlist) : 0;
        // a deleted position keeps its stage-1 slot but is not reranked (pq_update.cu:503-523)
        if (live && S.deleted && S.deleted[lp]) live = false;
        uint32_t hi;
        if (f32) {
            float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
            if (live) {
                const float4* row = reinterpret_cast<const float4*>(S.rr_f32 + (size_t)lp * d) + sub;
                const float4* qv = reinterpret_cast<const float4*>(sq) + sub;
                auto step = [&](const float4 v, const float4 u) {
                    const float x0 = __fsub_rn(u.x, v.x), x1 = __fsub_rn(u.y, v.y);
                    const float x2 = __fsub_rn(u.z, v.z), x3 = __fsub_rn(u.w, v.w);
                    a0 = __fmaf_rn(x0, x0, a0);
                    a1 = __fmaf_rn(x1, x1, a1);
                    a2 = __fmaf_rn(x2, x2, a2);
                    a3 = __fmaf_rn(x3, x3, a3);
                };
                if constexpr (NB > 0) {
                    float4 v[NB];
#pragma unroll
                    for (int t = 0; t < NB; ++t) v[t] = __ldg(row + 4 * t);
#pragma unroll
                    for (int t = 0; t < NB; ++t) step(v[t], qv[4 * t]);
                } else {
                    for (int t = 0; t < nb; ++t) step(__ldg(row + 4 * t), qv[4 * t]);
                }
            }
            // lanes l and l + 8 are threads sub and sub ^ 2; l and l + 4 are sub and sub ^ 1
            a0 = __fadd_rn(a0, __shfl_xor_sync(0xffffffffu, a0, 2));
            a1 = __fadd_rn(a1, __shfl_xor_sync(0xffffffffu, a1, 2));
            a2 = __fadd_rn(a2, __shfl_xor_sync(0xffffffffu, a2, 2));
            a3 = __fadd_rn(a3, __shfl_xor_sync(0xffffffffu, a3, 2));
            a0 = __fadd_rn(a0, __shfl_xor_sync(0xffffffffu, a0, 1));
            a1 = __fadd_rn(a1, __shfl_xor_sync(0xffffffffu, a1, 1));
            a2 = __fadd_rn(a2, __shfl_xor_sync(0xffffffffu, a2, 1));
            a3 = __fadd_rn(a3, __shfl_xor_sync(0xffffffffu, a3, 1));
            hi = __float_as_uint(__fadd_rn(__fadd_rn(a0, a2), __fadd_rn(a1, a3)));
        } else {
            uint32_t acc = 0;
            if (live) {
                const uint4* row = reinterpret_cast<const uint4*>(S.rr_u8 + (size_t)lp * d);
                const uint4* qq = reinterpret_cast<const uint4*>(squ);
                for (int w = sub; w < nb; w += 4) {
                    const uint4 v = __ldg(row + w), u = qq[w];
                    uint32_t a;
                    a = __vabsdiffu4(v.x, u.x); acc = __dp4a(a, a, acc);
                    a = __vabsdiffu4(v.y, u.y); acc = __dp4a(a, a, acc);
                    a = __vabsdiffu4(v.z, u.z); acc = __dp4a(a, a, acc);
                    a = __vabsdiffu4(v.w, u.w); acc = __dp4a(a, a, acc);
                }
            }
            acc += __shfl_xor_sync(0xffffffffu, acc, 2);
            acc += __shfl_xor_sync(0xffffffffu, acc, 1);
            hi = acc;
        }
        if (sub == 0 && c < np) {
            uint64_t ek = kKeyNone;
            if (live) ek = make_key(hi, S.ids ? (uint32_t)S.ids[lp] : key_lo(key));
            if (c < nc && out_exm) {
                if (c < R) out_exm[(size_t)q * R + c] = ek;
                else out_exd[(size_t)q * Rd + (c - R)] = ek;
            }
            sk[c] = ek;
        }
    }
    if (!out_exm)
        for (int c = nlive + tid; c < np; c += kRRT) sk[c] = kKeyNone;
    __syncthreads();
    if (out_exm) return;
    if (k <= 16 && nlive <= (kRRT / 32) * 128) {
        // each warp's k smallest of its slice of the live keys (at most 128; into
        // the table region, free now), then warp 0's k smallest of those (at most 128)
        uint64_t* cand = reinterpret_cast<uint64_t*>(tab);
        const int w = tid >> 5, per = (nlive + kRRT / 32 - 1) / (kRRT / 32);
        const int lo = w * per, nw = lo < nlive ? min(per, nlive - lo) : 0;
        warp_smallest_k_dispatch(sk + lo, nw, k, cand + w * k);
        __syncthreads();
        if (w == 0) {
            warp_smallest_k_dispatch(cand, (kRRT / 32) * k, k, sk);
            __syncwarp();
            if (lane < k) {
                const uint64_t ek = sk[lane];
                const bool ok = ek != kKeyNone;
                if (out_topk) {
                    out_topk[(size_t)q * k + lane] = ek;
                } else {
                    out_ids[(size_t)q * k + lane] = ok ? (int32_t)key_lo(ek) : -1;
                    out_dist[(size_t)q * k + lane] =
                        ok ? (f32 ? __uint_as_float(key_hi(ek)) : (float)key_hi(ek)) : __int_as_float(0x7f800000);
                }
            }
        }
        return;
    }
    block_bitonic_sort<kRRT>(sk, np);
    for (int j = tid; j < k; j += kRRT) {
        const uint64_t ek = j < np ? sk[j] : kKeyNone;
        const bool ok = ek != kKeyNone;
        if (out_topk) {
            out_topk[(size_t)q * k + j] = ek;
            continue;
        }
        out_ids[(size_t)q * k + j] = ok ? (int32_t)key_lo(ek) : -1;
        out_dist[(size_t)q * k + j] =
            ok ? (f32 ? __uint_as_float(key_hi(ek)) : (float)key_hi(ek)) : __int_as_float(0x7f800000);
    }
}

// ---------------------------------------------------------------------------
// merge of per-shard (ADC key, exact key) lists
// ---------------------------------------------------------------------------
constexpr int kMT = 256;
constexpr int kMMax = 8192;

// sorts (key, payload) pairs ascending by key; n power of two
__device__ void bitonic_pairs(uint64_t* k, int* v, int n) {
    for (int size = 2; size <= n; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            __syncthreads();
            for (int i = threadIdx.x; i < n / 2; i += kMT) {
                int lo = 2 * i - (i & (stride - 1)), hi = lo + stride;
                bool asc = ((lo & size) == 0);
                uint64_t a = k[lo], b = k[hi];
                if ((a > b) == asc) {
                    k[lo] = b; k[hi] = a;
                    int t = v[lo]; v[lo] = v[hi]; v[hi] = t;
                }
            }
        }
    }
    __syncthreads();
}

__global__ void __launch_bounds__(kMT) merge_shards_kernel(const uint64_t* adc_m, const uint64_t* ex_m, int n_m, int R,
                                                           const uint64_t* adc_d, const uint64_t* ex_d, int n_d,
                                                           int Rd, int k, int exact_is_int, int32_t* out_ids,
                                                           float* out_dist) {
    extern __shared__ uint64_t smk[];                 // [npmax] keys, then [npmax] payloads
    __shared__ uint64_t fin[2048];
    int npmax = 1;
    while (npmax < (n_m > n_d ? n_m : n_d)) npmax <<= 1;
    int* smv = reinterpret_cast<int*>(smk + npmax);
    const int q = blockIdx.x, tid = threadIdx.x;
    int nf = 0;
    for (int seg = 0; seg < 2; ++seg) {
        const int n = seg ? n_d : n_m, take = seg ? Rd : R;
        if (n == 0 || take == 0) continue;
        const uint64_t* a = (seg ? adc_d : adc_m) + (size_t)q * n;
        const uint64_t* ex = (seg ? ex_d : ex_m) + (size_t)q * n;
        int np = 1;
        while (np < n) np <<= 1;
        for (int i = tid; i < np; i += kMT) {
            smk[i] = i < n ? a[i] : kKeyNone;
            smv[i] = i;
        }
        bitonic_pairs(smk, smv, np);
        const int lim = take < n ? take : n;
        for (int i = tid; i < lim; i += kMT) {
            uint64_t e = kKeyNone;
            if (smk[i] != kKeyNone && !(i > 0 && smk[i - 1] == smk[i])) e = ex[smv[i]];
            fin[nf + i] = e;
        }
        nf += lim;
        __syncthreads();
    }
    int np = 1;
    while (np < nf) np <<= 1;
    for (int i = nf + tid; i < np; i += kMT) fin[i] = kKeyNone;
    block_bitonic_sort<kMT>(fin, np);
    for (int j = tid; j < k; j += kMT) {
        const uint64_t ek = j < np ? fin[j] : kKeyNone;
        const bool ok = ek != kKeyNone;
        out_ids[(size_t)q * k + j] = ok ? (int32_t)key_lo(ek) : -1;
        out_dist[(size_t)q * k + j] =
            ok ? (exact_is_int ? (float)key_hi(ek) : __uint_as_float(key_hi(ek))) : __int_as_float(0x7f800000);
    }
}

// ---------------------------------------------------------------------------
// sharded search, owner side
// ---------------------------------------------------------------------------
// Each of the G shards sent its stage-1 list of the query: R keys in any
// order, kKeyNone-padded.  The query's stage 1 over the whole index is every
// distinct key <= kappa, the R-th smallest of the union (with multiplicity,
// as a single stage-1 selection counts a repeated position), so every shard
// reranks its keys <= kappa.  One CTA per owned query.
constexpr int kShT = 256;

__global__ void __launch_bounds__(kShT) shard_kappa_kernel(const uint64_t* __restrict__ adc, int G, int qo, int R,
                                                           uint64_t* __restrict__ kappa) {
    __shared__ int hist[256];
    __shared__ int bc[4];
    __shared__ int s_valid;
    const int q = blockIdx.x, tid = threadIdx.x;
    const int n = G * R;
    // element i of the union: shard i / R, entry i % R
    auto keyf = [&](int i) -> uint64_t { return adc[((size_t)(i / R) * qo + q) * R + (i % R)]; };
    if (tid == 0) s_valid = 0;
    __syncthreads();
    int v = 0;
    for (int i = tid; i < n; i += kShT) v += keyf(i) != kKeyNone ? 1 : 0;
    if (v) atomicAdd(&s_valid, v);
    __syncthreads();
    const int valid = s_valid;
    uint64_t kap = kKeyNone - 1;                   // fewer than R keys: every key is in stage 1
    if (valid > R) kap = block_kth_key<kShT>(keyf, n, R, kKeyNone - 1, hist, bc);
    if (tid == 0) kappa[q] = kap;
}

// Final top-k of an owned query from the G shards' exact top-k lists (keys of
// distinct positions), one warp per query: L rounds of the warp minimum.
template <int E>
__global__ void __launch_bounds__(256) shard_final_kernel(const uint64_t* __restrict__ top, int G, int qo, int k,
                                                          int exact_is_int, int32_t* out_ids, float* out_dist) {
    const int q = (int)((blockIdx.x * (size_t)blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
    if (q >= qo) return;                           // whole warps only
    const int n = G * k;
    uint64_t v[E];
#pragma unroll
    for (int e = 0; e < E; ++e) {
        const int i = e * 32 + lane;
        v[e] = i < n ? top[((size_t)(i / k) * qo + q) * k + (i % k)] : kKeyNone;
    }
    uint64_t mine = kKeyNone;
    for (int it = 0; it < k; ++it) {
        const uint64_t wm = warp_take_min<E>(v);
        if (lane == it) mine = wm;
    }
    if (lane < k) {
        const bool ok = mine != kKeyNone;
        out_ids[(size_t)q * k + lane] = ok ? (int32_t)key_lo(mine) : -1;
        out_dist[(size_t)q * k + lane] =
            ok ? (exact_is_int ? (float)key_hi(mine) : __uint_as_float(key_hi(mine))) : __int_as_float(0x7f800000);
    }
}

}  // namespace

bool pq_supported_m(int M) { return M > 0 && M <= 64 && M % 8 == 0; }

int pq_scan_chunks(int M, int d, int count) {
    if (count <= 0) return 0;
    return pq_group_usable(M, d) ? gring_chunks(count) : (count + kPChunk - 1) / kPChunk;
}

int pq_scan_chunk_items(int M, int d) { return pq_group_usable(M, d) ? kRRings * kRSteps : kPChunk; }

int pq_chunk_slack(int M, int d, int R) { return pq_group_usable(M, d) ? R / 4 : 0; }

int64_t pq_gring_list_bytes(int count, int M) { return gring_tiles(count) * 128 * (M / 8); }

int64_t pq_mix_list_bytes(int count_main, int count_delta, int M) {
    return gring_tiles(kRRings * mix_stripes(count_main, count_delta).S) * 128 * (M / 8);
}

cudaError_t pq_build_gring(const uint8_t* codes, const int64_t* offsets, const int32_t* counts,
                           const int64_t* tile_off, int nlist, int M, uint8_t* out, cudaStream_t st) {
    if (M != 16 && M != 32 && M != 48) return cudaErrorInvalidValue;
    if (nlist <= 0) return cudaSuccess;
    const int grid = nlist < 4096 ? nlist : 4096;
    note_launch();
    switch (M / 8) {
        case 2: gring_layout_kernel<2><<<grid, 256, 0, st>>>(codes, offsets, counts, tile_off, nlist, M, out); break;
        case 4: gring_layout_kernel<4><<<grid, 256, 0, st>>>(codes, offsets, counts, tile_off, nlist, M, out); break;
        default: gring_layout_kernel<6><<<grid, 256, 0, st>>>(codes, offsets, counts, tile_off, nlist, M, out); break;
    }
    return cudaGetLastError();
}

cudaError_t pq_build_gring_mix(const uint8_t* main_tiles, const int64_t* main_off, const int32_t* main_counts,
                               const uint8_t* delta_tiles, const int64_t* delta_off, const int32_t* delta_counts,
                               const int64_t* mix_off, int nlist, int M, uint8_t* out, cudaStream_t st) {
    if (M != 16 && M != 32 && M != 48) return cudaErrorInvalidValue;
    if (nlist <= 0) return cudaSuccess;
    const int grid = nlist < 4096 ? nlist : 4096;
    note_launch();
#define ISB_MIX(MPL)                                                                                           \
    gring_mix_kernel<MPL><<<grid, 256, 0, st>>>(main_tiles, main_off, main_counts, delta_tiles, delta_off,      \
                                                 delta_counts, mix_off, nlist, out)
    switch (M / 8) {
        case 2: ISB_MIX(2); break;
        case 4: ISB_MIX(4); break;
        default: ISB_MIX(6); break;
    }
#undef ISB_MIX
    return cudaGetLastError();
}

namespace {

constexpr int kDW = 8;      // warps per CTA of the direct delta kernel

// The delta rows of every list a query probes, scanned without LUTs: each
// lane takes one row and computes its ADC distance from the residual and the
// codebook with the operations of the LUT build and the stagger sum in their
// order (entry m = sum over u of (r_u - c_u)^2, products and sums rounded
// separately; distance = entries added in m order), so every key equals the
// one the LUT scan would form.  A warp keeps its 32 smallest keys (one per
// lane, ascending) and merges each batch of 32 rows into them only when some
// row beats its largest; the CTA (one query) merges its warps' lists and
// writes the Rd <= 32 smallest, sorted, kKeyNone past the available keys.  A
// repeated probe scans its list again (its keys count twice, as in the
// candidate-buffer path).  Replaces, for small deltas, the per-list delta
// scan of build_delta_pq_mutable_publish / the overlay search
// (updates/pq_update.cu:448-523).
template <int M, int DSUB>
__global__ void __launch_bounds__(kDW * 32, 1) delta_direct_kernel(PQParams p, const int32_t* __restrict__ probes,
                                                               int nprobe, int nlist_global,
                                                               const int32_t* __restrict__ list_map, int Rd,
                                                               uint64_t* __restrict__ out) {
    constexpr int d = M * DSUB;
    __shared__ float s_res[kDW][d];
    __shared__ uint64_t s_top[kDW * 32];
    const int q = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const ListStore& D = p.delta;
    uint64_t top = kKeyNone;
    for (int c = warp; c < nprobe; c += kDW) {
        const int g = probes[(size_t)q * nprobe + c];
        if (g < 0 || g >= nlist_global) continue;
        const int l = list_map ? list_map[g] : g;
        if (l < 0) continue;
        const int cnt = D.counts[l];
        if (cnt <= 0) continue;
        const int64_t off = D.offsets[l];
        const uint32_t kb = (uint32_t)(D.key_off ? D.key_off[l] : off);
        const float* cv = p.cent + (size_t)l * d;
        for (int x = lane; x < d; x += 32) s_res[warp][x] = __fsub_rn(p.q[(size_t)q * d + x], cv[x]);
        __syncwarp();
        for (int r0 = 0; r0 < cnt; r0 += 32) {
            const int r = r0 + lane;
            uint64_t key = kKeyNone;
            if (r < cnt) {
                const uint4* cp = reinterpret_cast<const uint4*>(D.data + (size_t)(off + r) * M);
                float dist = 0.f;
#pragma unroll
                for (int h = 0; h < M / 16; ++h) {
                    const uint4 w4 = __ldg(cp + h);
                    const uint32_t w[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
                    for (int b = 0; b < 16; ++b) {
                        const int m = 16 * h + b;
                        const uint32_t code = (w[b >> 2] >> (8 * (b & 3))) & 0xFFu;
                        const float* cb = p.codebook_t + ((size_t)code * M + m) * DSUB;
                        float cbv[DSUB];
                        if constexpr (DSUB % 4 == 0) {
#pragma unroll
                            for (int u = 0; u < DSUB; u += 4) {
                                const float4 t4 = __ldg(reinterpret_cast<const float4*>(cb + u));
                                cbv[u] = t4.x; cbv[u + 1] = t4.y; cbv[u + 2] = t4.z; cbv[u + 3] = t4.w;
                            }
                        } else {
                            const float2 t2 = __ldg(reinterpret_cast<const float2*>(cb));
                            cbv[0] = t2.x; cbv[1] = t2.y;
                        }
                        float a = 0.f;
#pragma unroll
                        for (int u = 0; u < DSUB; ++u) {
                            const float x = __fsub_rn(s_res[warp][m * DSUB + u], cbv[u]);
                            a = u == 0 ? __fmul_rn(x, x) : __fadd_rn(a, __fmul_rn(x, x));
                        }
                        dist = m == 0 ? a : __fadd_rn(dist, a);
                    }
                }
                key = make_key(__float_as_uint(dist), kb + (uint32_t)r);
            }
            const uint64_t worst = __shfl_sync(0xffffffffu, top, 31);
            if (__any_sync(0xffffffffu, key < worst)) {
                // the batch sorted and reversed against the ascending list: their
                // lane-wise minima are the 32 smallest of both, a bitonic sequence
                uint64_t b = warp_sort32(key);
                b = __shfl_sync(0xffffffffu, b, 31 - lane);
                uint64_t v = b < top ? b : top;
#pragma unroll
                for (int j = 16; j > 0; j >>= 1) {
                    const uint64_t o = __shfl_xor_sync(0xffffffffu, v, j);
                    v = (lane & j) == 0 ? (o < v ? o : v) : (o > v ? o : v);
                }
                top = v;
            }
        }
        __syncwarp();     // the residual is rewritten for the next probe
    }
    s_top[warp * 32 + lane] = top;
    block_bitonic_sort<kDW * 32>(s_top, kDW * 32);
    for (int i = threadIdx.x; i < Rd; i += kDW * 32) out[(size_t)q * Rd + i] = s_top[i];
}

// The same search with the codebook staged in shared memory, sub-quantizer
// major ([m][c][u]: a warp's 32 gathers of one sub-quantizer fall on 32
// random 16-byte slots of one 4 KB row instead of 32 L1 lines), by persistent
// CTAs of kDW2 warps, each CTA taking queries q = blockIdx.x + i * gridDim.x.
constexpr int kDW2 = 16;
template <int M, int DSUB>
constexpr size_t delta_smem_bytes() {
    return sizeof(float) * ((size_t)M * 256 * DSUB + (size_t)kDW2 * M * DSUB) + sizeof(uint64_t) * kDW2 * 32;
}

template <int M, int DSUB>
__global__ void __launch_bounds__(kDW2 * 32, 1) delta_direct_smem_kernel(PQParams p, const int32_t* __restrict__ probes,
                                                                    int nq, int nprobe, int nlist_global,
                                                                    const int32_t* __restrict__ list_map, int Rd,
                                                                    uint64_t* __restrict__ out) {
    constexpr int d = M * DSUB;
    extern __shared__ __align__(16) float smd[];
    float* s_cb = smd;                                   // [M][256][DSUB]
    float* s_res = s_cb + (size_t)M * 256 * DSUB;        // [kDW2][d]
    uint64_t* s_top = reinterpret_cast<uint64_t*>(s_res + kDW2 * d);   // [kDW2 * 32]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int i = threadIdx.x; i < M * 256 * DSUB; i += kDW2 * 32) {
        const int c = i / (M * DSUB), m = (i / DSUB) % M, u = i % DSUB;
        s_cb[((size_t)m * 256 + c) * DSUB + u] = p.codebook_t[i];
    }
    __syncthreads();
    const ListStore& D = p.delta;
    float* res = s_res + warp * d;
    for (int q = blockIdx.x; q < nq; q += gridDim.x) {
        uint64_t top = kKeyNone;
        for (int c = warp; c < nprobe; c += kDW2) {
            const int g = probes[(size_t)q * nprobe + c];
            if (g < 0 || g >= nlist_global) continue;
            const int l = list_map ? list_map[g] : g;
            if (l < 0) continue;
            const int cnt = D.counts[l];
            if (cnt <= 0) continue;
            const int64_t off = D.offsets[l];
            const uint32_t kb = (uint32_t)(D.key_off ? D.key_off[l] : off);
            const float* cv = p.cent + (size_t)l * d;
            for (int x = lane; x < d; x += 32) res[x] = __fsub_rn(p.q[(size_t)q * d + x], cv[x]);
            __syncwarp();
            for (int r0 = 0; r0 < cnt; r0 += 32) {
                const int r = r0 + lane;
                uint64_t key = kKeyNone;
                if (r < cnt) {
                    const uint4* cp = reinterpret_cast<const uint4*>(D.data + (size_t)(off + r) * M);
                    float dist = 0.f;
#pragma unroll
                    for (int h = 0; h < M / 16; ++h) {
                        const uint4 w4 = __ldg(cp + h);
                        const uint32_t w[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
                        for (int b = 0; b < 16; ++b) {
                            const int m = 16 * h + b;
                            const uint32_t code = (w[b >> 2] >> (8 * (b & 3))) & 0xFFu;
                            const float* cb = s_cb + ((size_t)m * 256 + code) * DSUB;
                            float cbv[DSUB];
                            if constexpr (DSUB % 4 == 0) {
#pragma unroll
                                for (int u = 0; u < DSUB; u += 4) {
                                    const float4 t4 = *reinterpret_cast<const float4*>(cb + u);
                                    cbv[u] = t4.x; cbv[u + 1] = t4.y; cbv[u + 2] = t4.z; cbv[u + 3] = t4.w;
                                }
                            } else {
                                const float2 t2 = *reinterpret_cast<const float2*>(cb);
                                cbv[0] = t2.x; cbv[1] = t2.y;
                            }
                            float a = 0.f;
#pragma unroll
                            for (int u = 0; u < DSUB; ++u) {
                                const float x = __fsub_rn(res[m * DSUB + u], cbv[u]);
                                a = u == 0 ? __fmul_rn(x, x) : __fadd_rn(a, __fmul_rn(x, x));
                            }
                            dist = m == 0 ? a : __fadd_rn(dist, a);
                        }
                    }
                    key = make_key(__float_as_uint(dist), kb + (uint32_t)r);
                }
                const uint64_t worst = __shfl_sync(0xffffffffu, top, 31);
                if (__any_sync(0xffffffffu, key < worst)) {
                    uint64_t b = warp_sort32(key);
                    b = __shfl_sync(0xffffffffu, b, 31 - lane);
                    uint64_t v = b < top ? b : top;
#pragma unroll
                    for (int j = 16; j > 0; j >>= 1) {
                        const uint64_t o = __shfl_xor_sync(0xffffffffu, v, j);
                        v = (lane & j) == 0 ? (o < v ? o : v) : (o > v ? o : v);
                    }
                    top = v;
                }
            }
            __syncwarp();
        }
        s_top[warp * 32 + lane] = top;
        block_bitonic_sort<kDW2 * 32>(s_top, kDW2 * 32);
        for (int i = threadIdx.x; i < Rd; i += kDW2 * 32) out[(size_t)q * Rd + i] = s_top[i];
        __syncthreads();      // s_top is rewritten for the next query
    }
}

}  // namespace

bool pq_delta_direct_usable(int M, int d, int Rd) {
    return Rd >= 1 && Rd <= 32 && pq_group_usable(M, d) && d <= kPMaxD;
}

namespace {

// the shared-memory codebook where it fits in one CTA, else the codebook
// gathered through L1
template <int MM, int DS>
cudaError_t launch_delta_direct(const PQParams& p, const int32_t* probes, int nq, int nprobe, int nlist_global,
                                const int32_t* list_map, int Rd, uint64_t* out, int sms, cudaStream_t st) {
    constexpr size_t smem = delta_smem_bytes<MM, DS>();
    if constexpr (smem <= 220 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(delta_direct_smem_kernel<MM, DS>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e) return e;
        const int grid = nq < sms ? nq : sms;
        delta_direct_smem_kernel<MM, DS><<<grid, kDW2 * 32, smem, st>>>(p, probes, nq, nprobe, nlist_global,
                                                                        list_map, Rd, out);
    } else {
        delta_direct_kernel<MM, DS><<<nq, kDW * 32, 0, st>>>(p, probes, nprobe, nlist_global, list_map, Rd, out);
    }
    return cudaGetLastError();
}

}  // namespace

cudaError_t pq_delta_direct(const PQParams& p, const int32_t* probes, int nq, int nprobe, int nlist_global,
                            const int32_t* list_map, int Rd, uint64_t* out, cudaStream_t st) {
    if (!pq_delta_direct_usable(p.M, p.d, Rd) || !p.delta.data || !p.codebook_t) return cudaErrorInvalidValue;
    if (nq <= 0) return cudaSuccess;
    const int ds = p.d / p.M;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    note_launch();
#define ISB_DIRECT(MM, DS) \
    if (p.M == MM && ds == DS) return launch_delta_direct<MM, DS>(p, probes, nq, nprobe, nlist_global, list_map, Rd, out, sms, st);
    ISB_DIRECT(16, 2) ISB_DIRECT(16, 4) ISB_DIRECT(16, 8)
    ISB_DIRECT(32, 2) ISB_DIRECT(32, 4) ISB_DIRECT(32, 8)
    ISB_DIRECT(48, 2) ISB_DIRECT(48, 4)
#undef ISB_DIRECT
    return cudaErrorInvalidValue;
}

bool pq_group_usable(int M, int d) {
    if (M <= 0 || d % M != 0) return false;
    const int dsub = d / M;
    return (M == 16 || M == 32 || M == 48) && (dsub == 2 || dsub == 4 || dsub == 8);
}

cudaError_t pq_scan(const PQParams& p, WorkList wl, int max_pairs, CandBuf cm, CandBuf cd, int* counter,
                    cudaStream_t st) {
    if (p.d > kPMaxD || !pq_supported_m(p.M)) return cudaErrorInvalidValue;
    if (max_pairs <= 0) return cudaSuccess;
    cudaError_t e = cudaMemsetAsync(counter, 0, sizeof(int), st);
    if (e) return e;
    if (pq_group_usable(p.M, p.d) && wl.groups && p.codebook_t) {
        const int ds = p.d / p.M;
        if (!p.main.gring || (p.has_delta && !p.delta.gring)) return cudaErrorInvalidValue;
#define ISB_GROUP(MM, DS) \
    if (p.M == MM && ds == DS) return launch_gring<MM, DS>(p, wl, max_pairs, cm, cd, counter, st);
        ISB_GROUP(16, 2) ISB_GROUP(16, 4) ISB_GROUP(16, 8)
        ISB_GROUP(32, 2) ISB_GROUP(32, 4) ISB_GROUP(32, 8)
        ISB_GROUP(48, 2) ISB_GROUP(48, 4)
#undef ISB_GROUP
    }
    switch (p.M) {
        case 8: return launch_scan<8>(p, wl, max_pairs, cm, cd, counter, st);
        case 16: return launch_scan<16>(p, wl, max_pairs, cm, cd, counter, st);
        case 24: return launch_scan<24>(p, wl, max_pairs, cm, cd, counter, st);
        case 32: return launch_scan<32>(p, wl, max_pairs, cm, cd, counter, st);
        case 40: return launch_scan<40>(p, wl, max_pairs, cm, cd, counter, st);
        case 48: return launch_scan<48>(p, wl, max_pairs, cm, cd, counter, st);
        case 56: return launch_scan<56>(p, wl, max_pairs, cm, cd, counter, st);
        case 64: return launch_scan<64>(p, wl, max_pairs, cm, cd, counter, st);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t pq_rerank(const PQParams& p, int nlist, const uint64_t* s1_main, int R, const uint64_t* s1_delta,
                      int Rd, int nq, int k, int32_t* out_ids, float* out_dist, uint64_t* out_exact_main,
                      uint64_t* out_exact_delta, cudaStream_t st, const uint64_t* kmax, uint64_t* out_topk) {
    if (nq <= 0) return cudaSuccess;
    const int nc = R + Rd;
    if (nc > kRRMax || p.d > kPMaxD || (p.d % 16) != 0) return cudaErrorInvalidValue;
    int np = 1;
    while (np < nc) np <<= 1;
    if (!out_exact_main && np < k) return cudaErrorInvalidValue;
    const size_t smem = sizeof(uint64_t) * (2 * (size_t)np + (out_exact_main ? 0 : rr_table(np)));
    auto go = [&](auto kern) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 136 * 1024);
        if (e) return e;
        note_launch();
        kern<<<nq, kRRT, smem, st>>>(p, nlist, s1_main, R, s1_delta, Rd, k, out_ids, out_dist, out_exact_main,
                                     out_exact_delta, kmax, out_topk);
        return cudaGetLastError();
    };
    switch (p.main.rr_f32 ? p.d / 16 : 0) {
        case 2: return go(pq_rerank_kernel<2>);
        case 3: return go(pq_rerank_kernel<3>);
        case 4: return go(pq_rerank_kernel<4>);
        case 6: return go(pq_rerank_kernel<6>);
        case 8: return go(pq_rerank_kernel<8>);
        default: return go(pq_rerank_kernel<0>);
    }
}

cudaError_t pq_merge_shards(const uint64_t* adc_main, const uint64_t* exact_main, int n_main, int R,
                            const uint64_t* adc_delta, const uint64_t* exact_delta, int n_delta, int Rd, int nq,
                            int k, int exact_is_int, int32_t* out_ids, float* out_dist, cudaStream_t st) {
    if (nq <= 0) return cudaSuccess;
    if (n_main > kMMax || n_delta > kMMax || R + Rd > 2048 || k > 2048) return cudaErrorInvalidValue;
    int npmax = 1;
    while (npmax < (n_main > n_delta ? n_main : n_delta)) npmax <<= 1;
    size_t smem = (sizeof(uint64_t) + sizeof(int)) * npmax;
    cudaError_t e = cudaFuncSetAttribute(merge_shards_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e) return e;
    note_launch();
    merge_shards_kernel<<<nq, kMT, smem, st>>>(adc_main, exact_main, n_main, R, adc_delta, exact_delta, n_delta, Rd,
                                               k, exact_is_int, out_ids, out_dist);
    return cudaGetLastError();
}

cudaError_t pq_shard_kappa(const uint64_t* adc_all, int G, int qo, int R, uint64_t* kappa, cudaStream_t st) {
    if (qo <= 0) return cudaSuccess;
    note_launch();
    shard_kappa_kernel<<<qo, kShT, 0, st>>>(adc_all, G, qo, R, kappa);
    return cudaGetLastError();
}

cudaError_t pq_shard_final(const uint64_t* top_all, int G, int qo, int k, int exact_is_int, int32_t* out_ids,
                           float* out_dist, cudaStream_t st) {
    if (G <= 0 || k <= 0 || k > 32 || G * k > 256) return cudaErrorInvalidValue;
    if (qo <= 0) return cudaSuccess;
    const int n = G * k;
    const unsigned blocks = (unsigned)(((size_t)qo * 32 + 255) / 256);
    note_launch();
    if (n <= 32) shard_final_kernel<1><<<blocks, 256, 0, st>>>(top_all, G, qo, k, exact_is_int, out_ids, out_dist);
    else if (n <= 64) shard_final_kernel<2><<<blocks, 256, 0, st>>>(top_all, G, qo, k, exact_is_int, out_ids, out_dist);
    else if (n <= 128) shard_final_kernel<4><<<blocks, 256, 0, st>>>(top_all, G, qo, k, exact_is_int, out_ids, out_dist);
    else shard_final_kernel<8><<<blocks, 256, 0, st>>>(top_all, G, qo, k, exact_is_int, out_ids, out_dist);
    return cudaGetLastError();
}

}  // namespace isb
