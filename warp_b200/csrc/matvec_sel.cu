/*
 * matvec_sel.cu — the VQ3R matvec with NC interleaved copies of each
 * table, for fewer shared-memory bank conflicts (sm_100a).
 *
 * Same arithmetic as matvec_rows_kernel (src/model.c:1956-2024: per 64-row
 * block, per position ascending, t = (L0[i0] + L1[i1]) + L2[i2], acc += t;
 * the same thread/row/position mapping, so the same sums bit for bit). The
 * difference is where a lookup reads: a warp's 32 lookups of one
 * instruction hit uniformly random banks (about 3.5 shared-memory
 * wavefronts instead of 1). Here the table of every (position, stage)
 * holds each entry NC times side by side (entry c at words NC*c .. NC*c +
 * NC - 1, i.e. bank (NC*c + r) % 32), and every lookup carries a copy
 * number r. The copy numbers are chosen once per matrix, offline
 * (sel_build_kernel): among the lanes of one instruction whose index falls
 * in the same bank class (c % (32/NC)), they take copies 0, 1, ..., NC-1 in
 * lane order, so no bank holds more than ceil(n/NC) of them — about 2.6
 * wavefronts with 2 copies and 2.1 with 4 for uniform indices.
 *
 * The copy-select stream: per (64-row block, position, quarter) one record
 * of SW 32-bit words, lookup j = k*ST + s (k the row slot of the quarter,
 * s the stage) at bits [j*lg, j*lg + lg), lg = log2(NC).
 */
#include "vq3r_common.cuh"
#include "wc_launch.h"

#include <cuda_runtime.h>
#include <stdint.h>

using namespace wc;

namespace {

template <int NC> struct SelFmt;
template <> struct SelFmt<2> { static constexpr int LG = 1, SW = 2; };
template <> struct SelFmt<4> { static constexpr int LG = 2, SW = 4; };

/* Copy number of lookup J (compile time) from the record's words. */
template <int NC, int J>
__device__ __forceinline__ uint32_t sel_at(const uint32_t *sw)
{
    constexpr int LG = SelFmt<NC>::LG;
    constexpr int bit = J * LG;
    return (sw[bit >> 5] >> (bit & 31)) & (NC - 1);
}

template <int ST, int NC, int K>
struct RowStepSel {
    static __device__ __forceinline__ void run(float *acc, const uint32_t *w, const uint32_t *sw,
                                               const float *L)
    {
        constexpr int T = kEntries * NC;           /* words per (position, stage) table */
        float t = L[NC * byte_at<K * ST>(w) + sel_at<NC, K * ST>(sw)];
        if (ST > 1)
            t += L[T + NC * byte_at<K * ST + (ST > 1 ? 1 : 0)>(w) +
                   sel_at<NC, K * ST + (ST > 1 ? 1 : 0)>(sw)];
        if (ST > 2)
            t += L[2 * T + NC * byte_at<K * ST + (ST > 2 ? 2 : 0)>(w) +
                   sel_at<NC, K * ST + (ST > 2 ? 2 : 0)>(sw)];
        acc[K] += t;
        RowStepSel<ST, NC, K + 1>::run(acc, w, sw, L);
    }
};
template <int ST, int NC>
struct RowStepSel<ST, NC, kRowsPerThread> {
    static __device__ __forceinline__ void run(float *, const uint32_t *, const uint32_t *,
                                               const float *) {}
};

/* The index words and copy-select record of one position for 16 rows,
 * two positions in flight (as Gather16). */
template <int ST, int NC>
struct GatherSel {
    static constexpr int W = 4 * ST, SW = SelFmt<NC>::SW;
    uint32_t b0[W], b1[W], s0[SW], s1[SW];
    const uint8_t *p;
    const uint32_t *ps;
    int n;

    __device__ __forceinline__ void load(uint32_t *dst, uint32_t *sdst, int v) const
    {
        const uint64_t pol = l2_evict_first();
        const uint8_t *src = p + (size_t)v * kBlock * ST;
#pragma unroll
        for (int i = 0; i < ST; i++) {
            const uint4 q = ld_stream16(src + 16 * i, pol);
            dst[4 * i] = q.x; dst[4 * i + 1] = q.y; dst[4 * i + 2] = q.z; dst[4 * i + 3] = q.w;
        }
        /* a position's records are 4 quarters x SW words apart */
        const uint32_t *ss = ps + (size_t)v * 4 * SW;
        if (SW == 4) {
            const uint4 q = ld_stream16(ss, pol);
            sdst[0] = q.x; sdst[1] = q.y; sdst[2] = q.z; sdst[3] = q.w;
        } else {
            uint32_t x0, x1;
            asm("ld.global.nc.L2::cache_hint.v2.u32 {%0, %1}, [%2], %3;"
                : "=r"(x0), "=r"(x1) : "l"(ss), "l"(pol));
            sdst[0] = x0; sdst[1] = x1;
        }
    }

    __device__ __forceinline__ void begin(const uint8_t *p0, const uint32_t *ps0, int nvv)
    {
        p = p0;
        ps = ps0;
        n = nvv;
        if (n > 0) load(b0, s0, 0);
        if (n > 1) load(b1, s1, 1);
    }

    __device__ __forceinline__ void run(float *acc, const float *L)
    {
        constexpr int PT = ST * kEntries * NC;     /* words per position */
        int v = 0;
#pragma unroll 1
        for (; v + 1 < n; v += 2) {
            RowStepSel<ST, NC, 0>::run(acc, b0, s0, L + (size_t)v * PT);
            if (v + 2 < n) load(b0, s0, v + 2);
            RowStepSel<ST, NC, 0>::run(acc, b1, s1, L + (size_t)(v + 1) * PT);
            if (v + 3 < n) load(b1, s1, v + 3);
        }
        if (v < n) RowStepSel<ST, NC, 0>::run(acc, b0, s0, L + (size_t)v * PT);
    }
};

/* Tile = (matrix, kVsM positions, every row): thread t owns row block
 * t / 4, quarter t % 4 (M > 2048 rows: one lane of quarter blocks covers
 * the tile, as in matvec_rows_kernel). */
template <int ST, int NC, int MAXT, int kVsM>
__global__ void __launch_bounds__(MAXT)
matvec_sel_kernel(int ns, const wc_matvec_args a)
{
    extern __shared__ __align__(16) unsigned char smraw[];
    constexpr int SW = SelFmt<NC>::SW;
    float *xs = reinterpret_cast<float *>(smraw);
    float *lut = xs + kVsM * kVecDim;
    const int gi = blockIdx.x / ns, slice = blockIdx.x % ns;
    const int nv = a.N / kVecDim, nrb = (a.M + kBlock - 1) / kBlock;
    const int rb = threadIdx.x >> 2, q = threadIdx.x & 3;
    const int v0 = slice * kVsM, nvs = min(kVsM, nv - v0);
    const bool active = rb < nrb;
    GatherSel<ST, NC> gat;
    if (active)
        gat.begin(a.idx[gi] + (((size_t)rb * nv + v0) * kBlock + q * 16) * ST,
                  a.sel[gi] + (((size_t)rb * nv + v0) * 4 + q) * SW, nvs);
    else
        gat.n = 0;
    const float *xg = a.x[gi] + (size_t)v0 * kVecDim;
    for (int i = threadIdx.x; i < nvs * kVecDim; i += blockDim.x) xs[i] = xg[i];
    __syncthreads();
    /* the table: entry (v, s, c) = FMA chain over d from 0 (bit-identical
     * to build_lut_slice), stored NC times at words NC*c .. NC*c+NC-1 */
    for (int i = threadIdx.x; i < ST * kEntries; i += blockDim.x) {
        const int s = i / kEntries, c = i % kEntries;
        const float4 *src = reinterpret_cast<const float4 *>(
            a.books + ((size_t)(a.cb_base + s) * kEntries + c) * kVecDim);
        const float4 b0 = __ldg(src), b1 = __ldg(src + 1);
        for (int v = 0; v < nvs; v++) {
            const float4 x0 = *reinterpret_cast<const float4 *>(xs + v * kVecDim);
            const float4 x1 = *reinterpret_cast<const float4 *>(xs + v * kVecDim + 4);
            float acc = 0.0f;
            acc = __fmaf_rn(x0.x, b0.x, acc); acc = __fmaf_rn(x0.y, b0.y, acc);
            acc = __fmaf_rn(x0.z, b0.z, acc); acc = __fmaf_rn(x0.w, b0.w, acc);
            acc = __fmaf_rn(x1.x, b1.x, acc); acc = __fmaf_rn(x1.y, b1.y, acc);
            acc = __fmaf_rn(x1.z, b1.z, acc); acc = __fmaf_rn(x1.w, b1.w, acc);
            float *dst = lut + ((size_t)(v * ST + s) * kEntries + c) * NC;
            if (NC == 4)
                *reinterpret_cast<float4 *>(dst) = make_float4(acc, acc, acc, acc);
            else
                *reinterpret_cast<float2 *>(dst) = make_float2(acc, acc);
        }
    }
    __syncthreads();
    if (!active) return;
    float acc[kRowsPerThread];
#pragma unroll
    for (int k = 0; k < kRowsPerThread; k++) acc[k] = 0.0f;
    gat.run(acc, lut);
    const int row0 = rb * kBlock + q * 16;
    float *dst = a.part + ((size_t)gi * ns + slice) * a.M + row0;
    if (row0 + 16 <= a.M && ((reinterpret_cast<uintptr_t>(dst) & 15) == 0)) {
#pragma unroll
        for (int k = 0; k < kRowsPerThread; k += 4)
            *reinterpret_cast<float4 *>(dst + k) = make_float4(acc[k], acc[k + 1], acc[k + 2], acc[k + 3]);
    } else {
#pragma unroll
        for (int k = 0; k < kRowsPerThread; k++)
            if (row0 + k < a.M) dst[k] = acc[k];
    }
}

/* The copy numbers of one matrix, one block per (group of 8 row blocks —
 * one warp of the matvec — , position): thread t < 16*ST takes lookup
 * j = t (row slot k = t / ST, stage s = t % ST) of the 32 lanes, counts the
 * lanes per bank class in lane order and gives the n-th of a class copy
 * n % NC; then each lane packs its record. */
template <int ST, int NC>
__global__ void __launch_bounds__(64) sel_build_kernel(const uint8_t *__restrict__ idx,
                                                       uint32_t *__restrict__ sel, int nrb, int nv)
{
    constexpr int LG = SelFmt<NC>::LG, SW = SelFmt<NC>::SW, NCLS = 32 / NC;
    __shared__ uint8_t sb[32][kRowsPerThread * ST];
    const int wg = blockIdx.x, v = blockIdx.y;
    for (int j = threadIdx.x; j < kRowsPerThread * ST; j += blockDim.x) {
        const int k = j / ST, s = j % ST;
        uint8_t cnt[NCLS];
#pragma unroll
        for (int c = 0; c < NCLS; c++) cnt[c] = 0;
        for (int l = 0; l < 32; l++) {
            const int rb = wg * 8 + (l >> 2), q = l & 3;
            uint8_t r = 0;
            if (rb < nrb) {
                const int i = idx[(((size_t)rb * nv + v) * kBlock + q * 16 + k) * ST + s];
                const int c = i % NCLS;
#pragma unroll
                for (int cc = 0; cc < NCLS; cc++)            /* registers, not a local array */
                    if (cc == c) { r = cnt[cc] % NC; cnt[cc]++; }
            }
            sb[l][j] = r;
        }
    }
    __syncthreads();
    for (int l = threadIdx.x; l < 32; l += blockDim.x) {
        const int rb = wg * 8 + (l >> 2), q = l & 3;
        if (rb >= nrb) continue;
        uint32_t w[SW];
#pragma unroll
        for (int i = 0; i < SW; i++) w[i] = 0;
        for (int j = 0; j < kRowsPerThread * ST; j++) {
            const int bit = j * LG;
            w[bit >> 5] |= (uint32_t)sb[l][j] << (bit & 31);
        }
        uint32_t *dst = sel + (((size_t)rb * nv + v) * 4 + q) * SW;
#pragma unroll
        for (int i = 0; i < SW; i++) dst[i] = w[i];
    }
}

constexpr int kVsSel = 8;      /* positions per tile, as the plain matvec */

template <int ST, int NC>
int sel_launch(const wc_matvec_args *a, cudaStream_t s)
{
    const int nv = a->N / kVecDim, nrb = (a->M + kBlock - 1) / kBlock;
    const int ns = (nv + kVsSel - 1) / kVsSel;
    const int threads = ((nrb * 4 + 31) / 32) * 32;
    const size_t smem = ((size_t)kVsSel * kVecDim + (size_t)kVsSel * ST * kEntries * NC) * 4;
    const auto k = threads <= 256 ? matvec_sel_kernel<ST, NC, 256, kVsSel>
                                  : matvec_sel_kernel<ST, NC, 512, kVsSel>;
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return (int)cudaErrorInvalidValue;
    k<<<a->G * ns, threads, smem, s>>>(ns, *a);
    wc_count_launches(1);
    return (int)cudaGetLastError();
}

} /* namespace */

extern "C" size_t wc_sel_words(int M, int N, int copies)
{
    const int nrb = (M + kBlock - 1) / kBlock, nv = N / kVecDim;
    const int sw = copies == 4 ? SelFmt<4>::SW : SelFmt<2>::SW;
    return (size_t)nrb * nv * 4 * sw;
}

extern "C" int wc_sel_build_launch(const uint8_t *idx, uint32_t *sel, int M, int N, int stages,
                                   int copies, void *stream)
{
    cudaStream_t s = (cudaStream_t)stream;
    const int nrb = (M + kBlock - 1) / kBlock, nv = N / kVecDim;
    const dim3 grid((nrb + 7) / 8, nv);
    if (stages == 3 && copies == 2) sel_build_kernel<3, 2><<<grid, 64, 0, s>>>(idx, sel, nrb, nv);
    else if (stages == 3 && copies == 4) sel_build_kernel<3, 4><<<grid, 64, 0, s>>>(idx, sel, nrb, nv);
    else return (int)cudaErrorInvalidValue;
    wc_count_launches(1);
    return (int)cudaGetLastError();
}

/* The copy-select matvec: the gather launch, then the plain matvec's
 * reduce (partial sums in slice order, times the row scales). */
extern "C" int wc_matvec_sel_launch(const wc_matvec_args *a, int copies, void *stream)
{
    cudaStream_t s = (cudaStream_t)stream;
    if (a->stages != 3) return (int)cudaErrorInvalidValue;
    const int rc = copies == 2 ? sel_launch<3, 2>(a, s)
                 : copies == 4 ? sel_launch<3, 4>(a, s) : (int)cudaErrorInvalidValue;
    if (rc) return rc;
    const int nv = a->N / kVecDim;
    return wc_matvec_reduce_launch(a, (nv + kVsSel - 1) / kVsSel, stream);
}
