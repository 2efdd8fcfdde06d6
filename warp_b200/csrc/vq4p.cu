/*
 * vq4p.cu — the VQ4P expert format on sm_100a: WQ_VQ4P matrices
 * (src/waste_format.h:57), their int8 lookup tables and the expert loop over
 * them (src/model.c:2026-2229 vq_quant_range / vq_rows_p6, used by
 * moe_layer :2873-2911 and moe_chunk :3585-3659).
 *
 * Format: four residual stages of 64-entry, 8-dim codebooks. Per row and
 * vector position, three bytes hold four 6-bit indices, little-endian:
 * p = b0 | b1 << 8 | b2 << 16, j_s = (p >> 6s) & 63 (tools/convert.py:315-337).
 * The bytes are in the blocked layout [M/64][N/8][64][3].
 *
 * Arithmetic, all of it the reference's, so results are bit-identical:
 *   lut[v][s][c] = sum_d x[8v+d] * C_{cb+s}[c][d]  FMA chain from 0, d ascending
 *   per block of 32 positions: mx = max |lut| (the strict > scan), ls = mx / 127,
 *     inv = mx > 0 ? 127 / mx : 0, q = clamp(rint(lut * inv), -127, 127)
 *   per row and block: sum = sum_v sum_s q[v][s][j_s]   integers, exact
 *   acc = acc + ls * (float)sum over blocks ascending (rounded multiply, then
 *     rounded add: the reference's x86 build has no FMA contraction), and
 *   y = acc * f16(scale) with the scale's subnormals kept.
 *
 * B200 mapping. One CTA per (block of 32 positions, 1024 rows, problem).
 * It builds its block's fp32 table in registers (128 threads, two (stage,
 * entry) pairs each, 32 positions), reduces the block maximum, and writes
 * the int8 table to shared memory as [32][4][64] bytes. A 64-byte stage
 * table is 16 words in 16 different banks, so a warp whose 32 lanes look up
 * the same stage at the same position never conflicts: one wavefront per 32
 * lookups, where VQ3R's 256-entry fp32 tables average about 3.5. Each
 * thread owns 8 consecutive rows of a 64-row block (24 index bytes per
 * position: three 8-byte loads) and keeps their integer sums in registers.
 * The sums go to an int32 array [problem][block][M]; a fold kernel adds
 * them up in block order (and, in the expert loop, applies the gated
 * activation or the weighted reduce on the way).
 */
#include "vq3r_common.cuh"
#include "wc_launch.h"

#include <cuda_runtime.h>
#include <stdint.h>

using namespace wc;

namespace {

constexpr int kP6Threads = 128;
constexpr int kP6Blk = 32;                       /* WASTE_VQ_LUT_BLK, src/model.h:60 */
constexpr int kP6St = 4, kP6En = 64;
constexpr int kP6RowsT = 8;                      /* rows per thread                  */
constexpr int kP6RowsCta = kP6Threads / (kBlock / kP6RowsT) * kBlock;  /* 1024 rows  */
constexpr int kBookStride = kEntries * kVecDim;  /* books are held 256 entries apart */
constexpr int kFoldThreads = 256;

enum { P6_LIST = 0, P6_GATEUP = 1, P6_DOWN = 2 };

struct P6Prob {
    const uint8_t *idx;
    const float *x;
    const float *book;      /* stage 0 of this matrix's four books */
    int *part;              /* [blocks][M]                          */
    float *ls;              /* [blocks]                             */
    bool ok;
};

__device__ __forceinline__ const uint8_t *p6_record(const wc_p6_args &a, int pair, bool *ok)
{
    const int e = a.route[pair] - a.bank.first;
    if (e < 0 || e >= a.bank.n_experts) {
        *ok = false;
        return nullptr;
    }
    *ok = true;
    return a.bank.base + (size_t)e * a.bank.rec_bytes;
}

template <int MODE>
__device__ __forceinline__ P6Prob p6_resolve(const wc_p6_args &a, int z, int M, int N, int nblk)
{
    P6Prob p;
    p.part = a.part + (size_t)z * nblk * M;
    p.ls = a.ls + (size_t)z * nblk;
    p.ok = true;
    if (MODE == P6_LIST) {
        p.idx = a.idx[z];
        p.x = a.x[z];
        p.book = a.books + (size_t)a.cb[z] * kBookStride;
    } else if (MODE == P6_GATEUP) {
        const int pair = z >> 1, kind = z & 1;
        const uint8_t *rec = p6_record(a, pair, &p.ok);
        p.idx = p.ok ? rec + (kind ? a.bank.up_off : a.bank.gate_off) : nullptr;
        p.x = a.x_in + (size_t)(pair / a.K) * N;
        p.book = a.books + (size_t)(a.bank.cb_base + kind * kP6St) * kBookStride;
    } else {
        const uint8_t *rec = p6_record(a, z, &p.ok);
        p.idx = p.ok ? rec + a.bank.down_off : nullptr;
        p.x = a.h + (size_t)z * N;
        p.book = a.books + (size_t)(a.bank.cb_base + 2 * kP6St) * kBookStride;
    }
    return p;
}

/* Writes the block's int8 table [32][4][64] into T and returns its scale
 * to every thread. Thread t owns (stage, entry) pairs t and t + 128. */
__device__ __forceinline__ float p6_build_table(int8_t *T, const float *xs, const float *book,
                                                int nvb, uint32_t *red)
{
    const int tid = threadIdx.x;
    float cb[2][kVecDim];
#pragma unroll
    for (int k = 0; k < 2; k++) {
        const int q = tid + k * kP6Threads;
        const float4 *row =
            reinterpret_cast<const float4 *>(book + (size_t)(q >> 6) * kBookStride + (q & 63) * kVecDim);
        const float4 lo = __ldg(row), hi = __ldg(row + 1);
        cb[k][0] = lo.x; cb[k][1] = lo.y; cb[k][2] = lo.z; cb[k][3] = lo.w;
        cb[k][4] = hi.x; cb[k][5] = hi.y; cb[k][6] = hi.z; cb[k][7] = hi.w;
    }
    float val[2][kP6Blk];
    float mx = 0.0f;
#pragma unroll
    for (int v = 0; v < kP6Blk; v++) {
#pragma unroll
        for (int k = 0; k < 2; k++) {
            float t = 0.0f;
            if (v < nvb) {
#pragma unroll
                for (int d = 0; d < kVecDim; d++) t = __fmaf_rn(xs[v * kVecDim + d], cb[k][d], t);
                const float f = fabsf(t);
                if (f > mx) mx = f;             /* NaN never wins, as in the reference */
            }
            val[k][v] = t;
        }
    }
    /* non-negative floats order like their bit patterns */
    const uint32_t wm = __reduce_max_sync(0xffffffffu, __float_as_uint(mx));
    if ((tid & 31) == 0) red[tid >> 5] = wm;
    __syncthreads();
    uint32_t bm = red[0];
#pragma unroll
    for (int w = 1; w < kP6Threads / 32; w++) bm = max(bm, red[w]);
    mx = __uint_as_float(bm);
    const float inv = mx > 0.0f ? __fdiv_rn(127.0f, mx) : 0.0f;
#pragma unroll
    for (int v = 0; v < kP6Blk; v++) {
        if (v < nvb) {
#pragma unroll
            for (int k = 0; k < 2; k++) {
                int q = __float2int_rn(__fmul_rn(val[k][v], inv));
                q = q > 127 ? 127 : (q < -127 ? -127 : q);
                T[v * (kP6St * kP6En) + k * kP6Threads + tid] = (int8_t)q;
            }
        }
    }
    return __fdiv_rn(mx, 127.0f);
}

/* The 24-bit field of row r among 8 rows packed in six little-endian words. */
__device__ __forceinline__ uint32_t p6_field(const uint32_t *w, int r)
{
    switch (r) {
    case 0: return w[0] & 0xffffffu;
    case 1: return __funnelshift_r(w[0], w[1], 24) & 0xffffffu;
    case 2: return __funnelshift_r(w[1], w[2], 16) & 0xffffffu;
    case 3: return w[2] >> 8;
    case 4: return w[3] & 0xffffffu;
    case 5: return __funnelshift_r(w[3], w[4], 24) & 0xffffffu;
    case 6: return __funnelshift_r(w[4], w[5], 16) & 0xffffffu;
    default: return w[5] >> 8;
    }
}

template <int MODE>
__global__ void __launch_bounds__(kP6Threads) p6_rows_kernel(const __grid_constant__ wc_p6_args a,
                                                             int M, int N)
{
    __shared__ float xs[kP6Blk * kVecDim];
    __shared__ __align__(16) int8_t T[kP6Blk * kP6St * kP6En];
    __shared__ uint32_t red[kP6Threads / 32];
    const int nv = N / kVecDim, nblk = (nv + kP6Blk - 1) / kP6Blk;
    const int blk = blockIdx.x, v0 = blk * kP6Blk, nvb = min(kP6Blk, nv - v0);
    const P6Prob p = p6_resolve<MODE>(a, blockIdx.z, M, N, nblk);
    if (!p.ok) {
        if (threadIdx.x == 0 && blockIdx.x == 0 && blockIdx.y == 0) atomicOr(a.err, WC_ERR_BAD_EXPERT);
        return;
    }
    const int tid = threadIdx.x;
    for (int i = tid; i < nvb * kVecDim; i += kP6Threads) xs[i] = p.x[v0 * kVecDim + i];
    __syncthreads();
    const float ls = p6_build_table(T, xs, p.book, nvb, red);
    if (blockIdx.y == 0 && tid == 0) p.ls[blk] = ls;
    __syncthreads();

    const int rb = blockIdx.y * (kP6RowsCta / kBlock) + (tid >> 3);    /* 64-row block    */
    const int r0 = rb * kBlock + (tid & 7) * kP6RowsT;                 /* first row owned */
    if (r0 >= M) return;
    const uint8_t *src = p.idx + ((size_t)rb * nv + v0) * (kBlock * 3) + (tid & 7) * (kP6RowsT * 3);
    int sum[kP6RowsT];
#pragma unroll
    for (int r = 0; r < kP6RowsT; r++) sum[r] = 0;
#pragma unroll 4
    for (int v = 0; v < nvb; v++) {
        const uint2 *s2 = reinterpret_cast<const uint2 *>(src + (size_t)v * (kBlock * 3));
        const uint2 q0 = __ldg(s2), q1 = __ldg(s2 + 1), q2 = __ldg(s2 + 2);
        const uint32_t w[6] = { q0.x, q0.y, q1.x, q1.y, q2.x, q2.y };
        const int8_t *Tv = T + v * (kP6St * kP6En);
#pragma unroll
        for (int r = 0; r < kP6RowsT; r++) {
            const uint32_t f = p6_field(w, r);
            sum[r] += (int)Tv[f & 63] + (int)Tv[kP6En + ((f >> 6) & 63)] +
                      (int)Tv[2 * kP6En + ((f >> 12) & 63)] + (int)Tv[3 * kP6En + (f >> 18)];
        }
    }
    int *dst = p.part + (size_t)blk * M + r0;
    if (r0 + kP6RowsT <= M && (M & 3) == 0) {
        reinterpret_cast<int4 *>(dst)[0] = make_int4(sum[0], sum[1], sum[2], sum[3]);
        reinterpret_cast<int4 *>(dst)[1] = make_int4(sum[4], sum[5], sum[6], sum[7]);
    } else {
#pragma unroll
        for (int r = 0; r < kP6RowsT; r++)
            if (r0 + r < M) dst[r] = sum[r];
    }
}

/* acc over the blocks in order, then times the row's scale. */
__device__ __forceinline__ float p6_fold(const int *part, const float *ls, int nblk, int M, int r,
                                         uint16_t scale)
{
    float acc = 0.0f;
    for (int b = 0; b < nblk; b++)
        acc = __fadd_rn(acc, __fmul_rn(ls[b], (float)part[(size_t)b * M + r]));
    return __fmul_rn(acc, f16_keep(scale));
}

__global__ void __launch_bounds__(kFoldThreads) p6_fold_list_kernel(const __grid_constant__ wc_p6_args a)
{
    const int g = blockIdx.y, r = blockIdx.x * kFoldThreads + threadIdx.x;
    if (r >= a.M) return;
    const int nblk = (a.N / kVecDim + kP6Blk - 1) / kP6Blk;
    a.y[g][r] = p6_fold(a.part + (size_t)g * nblk * a.M, a.ls + (size_t)g * nblk, nblk, a.M, r,
                        a.scale[g][r]);
}

/* Gate and up of one (token, expert) pair, folded, then the gated activation
 * (src/model.c:2898-2903) into h[pair][inter]. */
__global__ void __launch_bounds__(kFoldThreads) p6_fold_act_kernel(const __grid_constant__ wc_p6_args a)
{
    const int pair = blockIdx.y, i = blockIdx.x * kFoldThreads + threadIdx.x;
    const int inter = a.bank.inter, lat = a.bank.lat;
    if (i >= inter) return;
    bool ok;
    const uint8_t *rec = p6_record(a, pair, &ok);
    if (!ok) return;
    const int nblk = (lat / kVecDim + kP6Blk - 1) / kP6Blk;
    const uint16_t *sc = reinterpret_cast<const uint16_t *>(rec + a.bank.scale_off);
    const size_t stride = (size_t)nblk * inter;
    const float g = p6_fold(a.part + (2 * pair) * stride, a.ls + (size_t)(2 * pair) * nblk, nblk,
                            inter, i, sc[i]);
    const float u = p6_fold(a.part + (2 * pair + 1) * stride, a.ls + (size_t)(2 * pair + 1) * nblk,
                            nblk, inter, i, sc[inter + i]);
    a.h[(size_t)pair * inter + i] = act_pair_cr(a.act, g, u, a.situ_beta, a.situ_lbeta);
}

/* Down of every pair of token t, folded, and the weighted reduce into
 * ysum[t]: router order (src/model.c:2909-2910, ysum += w[j]*acc from 0), or
 * ascending expert id with zero weights skipped and each expert once, at
 * the first slot naming it (src/model.c:3626-3656). */
__global__ void __launch_bounds__(kFoldThreads) p6_fold_combine_kernel(const __grid_constant__ wc_p6_args a)
{
    const int t = blockIdx.y, i = blockIdx.x * kFoldThreads + threadIdx.x;
    const int inter = a.bank.inter, lat = a.bank.lat, K = a.K;
    if (i >= lat) return;
    const int nblk = (inter / kVecDim + kP6Blk - 1) / kP6Blk;
    const size_t stride = (size_t)nblk * lat;
    const int *route = a.route + (size_t)t * K;
    const float *rw = a.rw + (size_t)t * K;
    float y = 0.0f;
    int last = -1;
    for (int n = 0; n < K; n++) {
        int j = n;
        if (a.order_by_id) {
            /* the smallest id above the last one taken, at its first slot */
            j = -1;
            for (int k = 0; k < K; k++)
                if (route[k] > last && (j < 0 || route[k] < route[j])) j = k;
            if (j < 0) break;
            last = route[j];
            if (rw[j] == 0.0f) continue;
        }
        const int pair = t * K + j;
        bool ok;
        const uint8_t *rec = p6_record(a, pair, &ok);
        if (!ok) continue;
        const uint16_t *sc = reinterpret_cast<const uint16_t *>(rec + a.bank.scale_off);
        const float d = p6_fold(a.part + pair * stride, a.ls + (size_t)pair * nblk, nblk, lat, i,
                                sc[2 * inter + i]);
        y = __fadd_rn(y, __fmul_rn(rw[j], d));
    }
    a.ysum[(size_t)t * lat + i] = y;
}

/* The int8 table of every block of x against books cb..cb+3 (the
 * reference's vq_build_lut + vq_quant_lut): q [nv][4][64], qs [blocks]. */
__global__ void __launch_bounds__(kP6Threads) p6_table_kernel(int8_t *q, float *qs, const float *x,
                                                              const float *book, int nv)
{
    __shared__ float xs[kP6Blk * kVecDim];
    __shared__ __align__(16) int8_t T[kP6Blk * kP6St * kP6En];
    __shared__ uint32_t red[kP6Threads / 32];
    const int blk = blockIdx.x, v0 = blk * kP6Blk, nvb = min(kP6Blk, nv - v0);
    for (int i = threadIdx.x; i < nvb * kVecDim; i += kP6Threads) xs[i] = x[v0 * kVecDim + i];
    __syncthreads();
    const float ls = p6_build_table(T, xs, book, nvb, red);
    __syncthreads();
    if (threadIdx.x == 0) qs[blk] = ls;
    for (int i = threadIdx.x; i < nvb * kP6St * kP6En; i += kP6Threads)
        q[(size_t)v0 * kP6St * kP6En + i] = T[i];
}

} /* namespace */

extern "C" {

size_t wc_p6_part_ints(int G, int M, int N)
{
    const int nblk = (N / kVecDim + kP6Blk - 1) / kP6Blk;
    return (size_t)G * nblk * M;
}

size_t wc_p6_ls_floats(int G, int N)
{
    return (size_t)G * ((N / kVecDim + kP6Blk - 1) / kP6Blk);
}

int wc_p6_matvec_launch(const wc_p6_args *a, void *stream)
{
    cudaStream_t st = (cudaStream_t)stream;
    const int nblk = (a->N / kVecDim + kP6Blk - 1) / kP6Blk;
    const dim3 grid(nblk, (a->M + kP6RowsCta - 1) / kP6RowsCta, a->G);
    p6_rows_kernel<P6_LIST><<<grid, kP6Threads, 0, st>>>(*a, a->M, a->N);
    const dim3 fg((a->M + kFoldThreads - 1) / kFoldThreads, a->G);
    p6_fold_list_kernel<<<fg, kFoldThreads, 0, st>>>(*a);
    wc_count_launches(2);
    return (int)cudaGetLastError();
}

int wc_p6_moe_launch(const wc_p6_args *a, void *stream)
{
    cudaStream_t st = (cudaStream_t)stream;
    const int inter = a->bank.inter, lat = a->bank.lat, pairs = a->T * a->K;
    const int nb_gu = (lat / kVecDim + kP6Blk - 1) / kP6Blk;
    const int nb_d = (inter / kVecDim + kP6Blk - 1) / kP6Blk;
    p6_rows_kernel<P6_GATEUP><<<dim3(nb_gu, (inter + kP6RowsCta - 1) / kP6RowsCta, 2 * pairs),
                                kP6Threads, 0, st>>>(*a, inter, lat);
    p6_fold_act_kernel<<<dim3((inter + kFoldThreads - 1) / kFoldThreads, pairs), kFoldThreads, 0,
                         st>>>(*a);
    p6_rows_kernel<P6_DOWN><<<dim3(nb_d, (lat + kP6RowsCta - 1) / kP6RowsCta, pairs), kP6Threads,
                              0, st>>>(*a, lat, inter);
    p6_fold_combine_kernel<<<dim3((lat + kFoldThreads - 1) / kFoldThreads, a->T), kFoldThreads, 0,
                             st>>>(*a);
    wc_count_launches(4);
    return (int)cudaGetLastError();
}

int wc_p6_table_launch(int8_t *q, float *qs, const float *x, const float *books, int cb, int nv,
                       void *stream)
{
    p6_table_kernel<<<(nv + kP6Blk - 1) / kP6Blk, kP6Threads, 0, (cudaStream_t)stream>>>(
        q, qs, x, books + (size_t)cb * kBookStride, nv);
    wc_count_launches(1);
    return (int)cudaGetLastError();
}

} /* extern "C" */
