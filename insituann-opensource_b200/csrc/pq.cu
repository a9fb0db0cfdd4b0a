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
// Grouped ring ADC scan (M = 16, 32, 48 with dsub = 2, 4 or 8): the kernel the
// search uses for these shapes.
//
// As in pq_group_kernel, a CTA takes one list and up to 4 probing queries and
// the four LUTs are interleaved as float4.  Instead of one thread summing a
// whole vector, a warp runs four systolic rings of 8 lanes: lane j of a ring
// owns the MPL = M/8 consecutive sub-quantizers m = MPL*j .. MPL*j+MPL-1.  At
// step x it receives the four partial sums of vector x-j from lane j-1
// (shuffles), adds its MPL entries in m order and passes them on; lane 7
// finishes vector x-7.  The distance of every query is therefore still the
// sum over m in m order.
//
// LUT row c holds entry m at float4 position p(m) = m/MPL + 8*(m%MPL), so in
// every gather lane j of a ring reads bank group j: each quarter-warp (one
// ring) touches 8 distinct 16-byte bank groups and the gather is
// conflict-free whatever the code values.
//
// Codes are re-laid out once per index (pq_build_gring) into tiles of 16
// steps: tile T of a list holds, for lane j, step i and sub-quantizer s, the
// byte code[16T+i-j][MPL*j+s] (0 outside the list), so a lane reads its
// 16*MPL bytes of a tile with MPL coalesced 16-byte loads and indexes them
// statically.
// ---------------------------------------------------------------------------
constexpr int kRW = 8;                 // warps per CTA
constexpr int kRT = 32 * kRW;          // threads per CTA
constexpr int kRChunk = 2048;          // vectors per filtered chunk
constexpr int kRRings = 4 * kRW;       // 8-lane rings per CTA

__host__ __device__ inline int64_t gring_tiles(int count) { return (int64_t)(count + 7) / 16 + 3; }

template <int M>
struct GRing {
    static constexpr int MPL = M / 8;
    static constexpr int kTileBytes = 128 * MPL;
    __host__ __device__ static constexpr int pos(int m) { return m / MPL + 8 * (m % MPL); }
    __host__ __device__ static constexpr int inv(int p) { return MPL * (p % 8) + p / 8; }
    static constexpr size_t smem_bytes() { return sizeof(float4) * ((size_t)256 * M + kRChunk); }
};

template <int M, int DSUB>
__global__ void __launch_bounds__(kRT, 1) pq_gring_kernel(PQParams p, WorkList wl, CandBuf cm, CandBuf cd,
                                                          int* counter) {
    using RG = GRing<M>;
    constexpr int MPL = RG::MPL;
    constexpr int d = M * DSUB;
    extern __shared__ __align__(16) float smf[];
    float4* lut = reinterpret_cast<float4*>(smf);          // [256][M], entry m at pos(m)
    float4* dist4 = lut + 256 * M;                          // [kRChunk] four queries per vector
    float* resid = reinterpret_cast<float*>(dist4);         // [kGQ][d] while the LUT is built
    __shared__ EmitSmem esm;
    __shared__ int s_item, s_q[kGQ];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, ring = lane >> 3, j = lane & 7;
    const float keep = j == 0 ? 0.f : 1.f;
    const int NG = *wl.n_groups;
    const int total = p.has_delta ? 2 * NG : NG;
    for (;;) {
        const int it = next_item(counter, total, &s_item);
        if (it < 0) break;
        const bool seg_delta = it >= NG;
        const int gi = seg_delta ? it - NG : it;
        const int packed = wl.groups[gi];
        const int p0 = packed >> 3, nqg = packed & 7;
        const int l = wl.pair_l[p0];
        const ListStore& SG = seg_delta ? p.delta : p.main;
        const CandBuf& cb = seg_delta ? cd : cm;
        const int count = SG.counts[l];
        if (count <= 0) continue;
        const int64_t koff = SG.key_off ? SG.key_off[l] : SG.offsets[l];
        const uint8_t* tiles = SG.gring + SG.gring_off[l];
        const int64_t ntiles = gring_tiles(count);
        if (tid < kGQ) s_q[tid] = tid < nqg ? wl.pair_q[p0 + tid] : -1;
        __syncthreads();
        {
            const float* cv = p.cent + (size_t)l * d;
            for (int e = tid; e < kGQ * d; e += kRT) {
                const int k = e / d, x = e - k * d;
                const int qk = s_q[k];
                resid[e] = qk >= 0 ? __fsub_rn(p.q[(size_t)qk * d + x], cv[x]) : 0.f;
            }
            __syncthreads();
            // thread t owns LUT column pos = t % M (sub-quantizer inv(pos)) for codes c = t / M + kRT / M * i
            constexpr int kCStep = kRT / M > 0 ? kRT / M : 1;
            if (tid < kCStep * M) {
                const int ps = tid % M, m = RG::inv(ps), c0 = tid / M;
                float r[kGQ][DSUB];
#pragma unroll
                for (int k = 0; k < kGQ; ++k)
#pragma unroll
                    for (int u = 0; u < DSUB; ++u) r[k][u] = resid[k * d + m * DSUB + u];
                for (int c = c0; c < 256; c += kCStep) {
                    float cbv[DSUB];
                    const float* src = p.codebook_t + ((size_t)c * M + m) * DSUB;
                    if constexpr (DSUB % 4 == 0) {
#pragma unroll
                        for (int u = 0; u < DSUB; u += 4) {
                            const float4 t4 = __ldg(reinterpret_cast<const float4*>(src + u));
                            cbv[u] = t4.x; cbv[u + 1] = t4.y; cbv[u + 2] = t4.z; cbv[u + 3] = t4.w;
                        }
                    } else {
#pragma unroll
                        for (int u = 0; u < DSUB; u += 2) {
                            const float2 t2 = __ldg(reinterpret_cast<const float2*>(src + u));
                            cbv[u] = t2.x; cbv[u + 1] = t2.y;
                        }
                    }
                    float acc[kGQ];
#pragma unroll
                    for (int k = 0; k < kGQ; ++k) {
                        const float x0 = __fsub_rn(r[k][0], cbv[0]);
                        float a = __fmul_rn(x0, x0);
#pragma unroll
                        for (int u = 1; u < DSUB; ++u) {
                            const float x = __fsub_rn(r[k][u], cbv[u]);
                            a = __fadd_rn(a, __fmul_rn(x, x));
                        }
                        acc[k] = a;
                    }
                    lut[c * M + ps] = make_float4(acc[0], acc[1], acc[2], acc[3]);
                }
            }
            __syncthreads();
        }
        // this lane's LUT columns: pos(MPL*j + s) = j + 8*s
        const float4* lutj = lut + j;
        for (int cs = 0; cs < count; cs += kRChunk) {
            const int len = min(kRChunk, count - cs);
            const int Lr = (((len + kRRings - 1) / kRRings) + 15) & ~15;   // vectors per ring, multiple of 16
            const int a = cs + (warp * 4 + ring) * Lr;                      // list-relative range [a, b)
            const int b = min(a + Lr, cs + len);
            if (cs + warp * 4 * Lr < cs + len) {                            // ring 0 of this warp has work
                float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
                const int T0 = a / 16;
                const int ntr = Lr / 16 + 1;
                const uint8_t* lanebase = tiles + j * 16 * MPL;
                uint32_t w[4 * MPL], wn[4 * MPL];
                {
                    const int64_t T = min((int64_t)T0, ntiles - 1);
                    const uint4* tp = reinterpret_cast<const uint4*>(lanebase + T * RG::kTileBytes);
#pragma unroll
                    for (int u = 0; u < MPL; ++u) {
                        const uint4 x = __ldg(tp + u);
                        w[4 * u] = x.x; w[4 * u + 1] = x.y; w[4 * u + 2] = x.z; w[4 * u + 3] = x.w;
                    }
                }
                for (int tt = 0; tt < ntr; ++tt) {
                    {
                        const int64_t T = min((int64_t)(T0 + tt + 1), ntiles - 1);
                        const uint4* tp = reinterpret_cast<const uint4*>(lanebase + T * RG::kTileBytes);
#pragma unroll
                        for (int u = 0; u < MPL; ++u) {
                            const uint4 x = __ldg(tp + u);
                            wn[4 * u] = x.x; wn[4 * u + 1] = x.y; wn[4 * u + 2] = x.z; wn[4 * u + 3] = x.w;
                        }
                    }
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const float i0 = __shfl_up_sync(0xffffffffu, s0, 1, 8);
                        const float i1 = __shfl_up_sync(0xffffffffu, s1, 1, 8);
                        const float i2 = __shfl_up_sync(0xffffffffu, s2, 1, 8);
                        const float i3 = __shfl_up_sync(0xffffffffu, s3, 1, 8);
#pragma unroll
                        for (int s = 0; s < MPL; ++s) {
                            const int byte = i * MPL + s;
                            const uint32_t c = (w[byte >> 2] >> (8 * (byte & 3))) & 0xFFu;
                            const float4 f = lutj[c * M + 8 * s];
                            if (s == 0) {
                                s0 = fmaf(i0, keep, f.x);
                                s1 = fmaf(i1, keep, f.y);
                                s2 = fmaf(i2, keep, f.z);
                                s3 = fmaf(i3, keep, f.w);
                            } else {
                                s0 = __fadd_rn(s0, f.x);
                                s1 = __fadd_rn(s1, f.y);
                                s2 = __fadd_rn(s2, f.z);
                                s3 = __fadd_rn(s3, f.w);
                            }
                        }
                        const int v = 16 * (T0 + tt) + i - 7;   // vector finished by lane 7 at this step
                        if (j == 7 && v >= a && v < b) dist4[v - cs] = make_float4(s0, s1, s2, s3);
                    }
#pragma unroll
                    for (int u = 0; u < 4 * MPL; ++u) w[u] = wn[u];
                }
            }
            __syncthreads();
            const uint32_t kbase = (uint32_t)(koff + cs);
            uint64_t thr[kGQ];
            int cnt4[kGQ];
#pragma unroll
            for (int k = 0; k < kGQ; ++k) {
                thr[k] = k < nqg ? *((volatile unsigned long long*)(cb.thr + s_q[k])) : 0ull;
                cnt4[k] = 0;
            }
            for (int i = tid; i < len; i += kRT) {
                const float4 f = dist4[i];
                const float fk[kGQ] = {f.x, f.y, f.z, f.w};
#pragma unroll
                for (int k = 0; k < kGQ; ++k)
                    cnt4[k] += (k < nqg && make_key(__float_as_uint(fk[k]), kbase + (uint32_t)i) <= thr[k]) ? 1 : 0;
            }
            const int4 tot = block_sum4<kRT>(make_int4(cnt4[0], cnt4[1], cnt4[2], cnt4[3]), esm.scratch);
            const int totk[kGQ] = {tot.x, tot.y, tot.z, tot.w};
            const float* dflat = reinterpret_cast<const float*>(dist4);
#pragma unroll
            for (int k = 0; k < kGQ; ++k) {
                if (k >= nqg || totk[k] == 0) continue;
                auto keyf = [&](int i) -> uint64_t {
                    return make_key(__float_as_uint(dflat[4 * i + k]), kbase + (uint32_t)i);
                };
                uint64_t cut = thr[k];
                if (totk[k] > cb.R) {
                    const uint64_t kap = block_kth_key<kRT>(keyf, len, cb.R, thr[k], esm.hist, esm.bc);
                    cut = kap < thr[k] ? kap : thr[k];
                    if (tid == 0) atomicMin(cb.thr + s_q[k], (unsigned long long)cut);
                }
                warp_append<kRT, kRChunk / kRT>(keyf, len, cut, cb, s_q[k]);
            }
            __syncthreads();
        }
    }
}

template <int M, int DSUB>
cudaError_t launch_gring(const PQParams& p, WorkList wl, int max_groups, CandBuf cm, CandBuf cd, int* counter,
                         cudaStream_t st) {
    const size_t smem = GRing<M>::smem_bytes();
    cudaError_t e =
        cudaFuncSetAttribute(pq_gring_kernel<M, DSUB>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e) return e;
    int dev = 0, sms = 148, per_sm = 1;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, pq_gring_kernel<M, DSUB>, kRT, smem);
    if (per_sm < 1) return cudaErrorInvalidConfiguration;
    long long items = (long long)max_groups * (p.has_delta ? 2 : 1);
    long long grid = (long long)sms * per_sm;
    if (grid > items) grid = items;
    if (grid < 1) grid = 1;
    note_launch();
    pq_gring_kernel<M, DSUB><<<(int)grid, kRT, smem, st>>>(p, wl, cm, cd, counter);
    return cudaGetLastError();
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
            const int jj = r / (16 * MPL), r2 = r % (16 * MPL), i = r2 / MPL, s = r2 % MPL;
            const int64_t v = 16 * T + i - jj;
            dst[e] = (v >= 0 && v < cnt) ? codes[(size_t)(off + v) * M + MPL * jj + s] : (uint8_t)0;
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

__global__ void __launch_bounds__(kRRT) pq_rerank_kernel(PQParams p, int nlist, const uint64_t* __restrict__ s1m,
                                                         int R, const uint64_t* __restrict__ s1d, int Rd, int k,
                                                         int32_t* out_ids, float* out_dist, uint64_t* out_exm,
                                                         uint64_t* out_exd) {
    extern __shared__ uint64_t sk[];
    __shared__ float sq[kPMaxD];
    __shared__ __align__(16) uint8_t squ[kPMaxD];
    const int q = blockIdx.x, tid = threadIdx.x, d = p.d;
    const bool f32 = p.main.rr_f32 != nullptr;
    for (int j = tid; j < d; j += kRRT) {
        float x = p.q[(size_t)q * d + j];
        sq[j] = x;
        squ[j] = to_u8(x);
    }
    __syncthreads();
    const int nc = R + Rd;
    int np = 1;
    while (np < nc) np <<= 1;
    for (int c = tid; c < np; c += kRRT) {
        uint64_t ek = kKeyNone;
        if (c < nc) {
            const bool dl = c >= R;
            const uint64_t* src = dl ? s1d + (size_t)q * Rd : s1m + (size_t)q * R;
            const int j = dl ? c - R : c;
            const uint64_t key = src[j];
            // a list probed twice repeats its keys: rerank each position once,
            // except when the per-candidate keys go to a cross-shard merge
            if (key != kKeyNone && (out_exm || !(j > 0 && src[j - 1] == key))) {
                const ListStore& S = dl ? p.delta : p.main;
                const int64_t lp = local_pos(S, key_lo(key), nlist);
                uint32_t hi;
                if (f32) {
                    const float4* row = reinterpret_cast<const float4*>(S.rr_f32 + (size_t)lp * d);
                    float s = 0.f;
                    for (int w = 0; w < d / 4; ++w) {
                        float4 v = __ldg(row + w);
                        float x0 = __fsub_rn(sq[4 * w + 0], v.x);
                        s = __fadd_rn(s, __fmul_rn(x0, x0));
                        float x1 = __fsub_rn(sq[4 * w + 1], v.y);
                        s = __fadd_rn(s, __fmul_rn(x1, x1));
                        float x2 = __fsub_rn(sq[4 * w + 2], v.z);
                        s = __fadd_rn(s, __fmul_rn(x2, x2));
                        float x3 = __fsub_rn(sq[4 * w + 3], v.w);
                        s = __fadd_rn(s, __fmul_rn(x3, x3));
                    }
                    hi = __float_as_uint(s);
                } else {
                    const uint4* row = reinterpret_cast<const uint4*>(S.rr_u8 + (size_t)lp * d);
                    const uint4* qq = reinterpret_cast<const uint4*>(squ);
                    uint32_t acc = 0;
                    for (int w = 0; w < d / 16; ++w) {
                        uint4 v = __ldg(row + w), u = qq[w];
                        uint32_t a;
                        a = __vabsdiffu4(v.x, u.x); acc = __dp4a(a, a, acc);
                        a = __vabsdiffu4(v.y, u.y); acc = __dp4a(a, a, acc);
                        a = __vabsdiffu4(v.z, u.z); acc = __dp4a(a, a, acc);
                        a = __vabsdiffu4(v.w, u.w); acc = __dp4a(a, a, acc);
                    }
                    hi = acc;
                }
                const uint32_t id = S.ids ? (uint32_t)S.ids[lp] : key_lo(key);
                ek = make_key(hi, id);
            }
        }
        if (c < nc && out_exm) {
            if (c < R) out_exm[(size_t)q * R + c] = ek;
            else out_exd[(size_t)q * Rd + (c - R)] = ek;
        }
        sk[c] = ek;
    }
    if (out_exm) return;
    block_bitonic_sort<kRRT>(sk, np);
    for (int j = tid; j < k; j += kRRT) {
        const uint64_t ek = j < np ? sk[j] : kKeyNone;
        const bool ok = ek != kKeyNone;
        out_ids[(size_t)q * k + j] = ok ? (int32_t)key_lo(ek) : -1;
        out_dist[(size_t)q * k + j] =
            ok ? (f32 ? __uint_as_float(key_hi(ek)) : (float)key_hi(ek)) : __int_as_float(0x7f800000);
    }
}

// ---------------------------------------------------------------------------
// merge of per-shard (ADC key, exact key) lists
// ---------------------------------------------------------------------------
constexpr int kMT = 512;
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
    extern __shared__ uint64_t smk[];
    int* smv = reinterpret_cast<int*>(smk + kMMax);
    __shared__ uint64_t fin[2048];
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

}  // namespace

bool pq_supported_m(int M) { return M > 0 && M <= 64 && M % 8 == 0; }

int pq_scan_chunk(int M, int d) { return pq_group_usable(M, d) ? kRChunk : kPChunk; }

int64_t pq_gring_list_bytes(int count, int M) { return gring_tiles(count) * 128 * (M / 8); }

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
                      uint64_t* out_exact_delta, cudaStream_t st) {
    if (nq <= 0) return cudaSuccess;
    const int nc = R + Rd;
    if (nc > kRRMax || p.d > kPMaxD || (p.d % 16) != 0) return cudaErrorInvalidValue;
    int np = 1;
    while (np < nc) np <<= 1;
    if (!out_exact_main && np < k) return cudaErrorInvalidValue;
    size_t smem = sizeof(uint64_t) * np;
    cudaError_t e = cudaFuncSetAttribute(pq_rerank_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 64 * 1024);
    if (e) return e;
    note_launch();
    pq_rerank_kernel<<<nq, kRRT, smem, st>>>(p, nlist, s1_main, R, s1_delta, Rd, k, out_ids, out_dist,
                                             out_exact_main, out_exact_delta);
    return cudaGetLastError();
}

cudaError_t pq_merge_shards(const uint64_t* adc_main, const uint64_t* exact_main, int n_main, int R,
                            const uint64_t* adc_delta, const uint64_t* exact_delta, int n_delta, int Rd, int nq,
                            int k, int exact_is_int, int32_t* out_ids, float* out_dist, cudaStream_t st) {
    if (nq <= 0) return cudaSuccess;
    if (n_main > kMMax || n_delta > kMMax || R + Rd > 2048 || k > 2048) return cudaErrorInvalidValue;
    size_t smem = (sizeof(uint64_t) + sizeof(int)) * kMMax;
    cudaError_t e = cudaFuncSetAttribute(merge_shards_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e) return e;
    note_launch();
    merge_shards_kernel<<<nq, kMT, smem, st>>>(adc_main, exact_main, n_main, R, adc_delta, exact_delta, n_delta, Rd,
                                               k, exact_is_int, out_ids, out_dist);
    return cudaGetLastError();
}

}  // namespace isb
