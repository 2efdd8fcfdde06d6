/*
 * vq3r_kernels.cu — sm_100a kernels for the VQ3R routed-expert FFN.
 *
 * The arithmetic is the reference's fused VQ matvec (sqliteai/warp
 * src/model.c:1843-2289): per token a table LUT[v][s][c] = <x_v, C_s[c]>,
 * then y[r] = f16(scale[r]) * sum_v sum_s LUT[v][s][idx[r][v][s]]. The
 * weights are never materialised.
 *
 * B200 mapping (memory-bound decode):
 *   - a tile is (matrix family, vector slice [v0, v0+Vs), row range); the
 *     CTA builds its slice of the table in shared memory from x and the
 *     codebooks (FMA chain, bit-identical to the AVX kernels), so no table
 *     ever goes to HBM;
 *   - each thread owns 16 rows (a quarter of a 64-row index block) and
 *     streams their indices with 16-byte loads, one position ahead;
 *   - the gather is 3 shared-memory lookups + 3 fp32 adds per (row, v);
 *   - lanes that split a slice's positions are reduced in shared memory in
 *     a fixed order, and slices are reduced by the consumer in slice order,
 *     so results are deterministic run to run.
 */
#include "vq3r_common.cuh"
#include "wc_launch.h"

#include <cuda_runtime.h>
#include <stdint.h>

using namespace wc;

static unsigned long long g_launches = 0;

extern "C" uint64_t wc_launches(void) { return g_launches; }

/* ---- phase timers --------------------------------------------------------
 * The device analogue of the reference's WASTE_PROFILE buckets
 * (src/model.c:37-52): when on, every kernel launch is bracketed by a pair
 * of CUDA events on its own stream, and wc_prof_read sums the elapsed
 * times per phase. Off by default; never used inside graph capture. */
namespace {
constexpr int kProfPairs = 4096;
struct Prof {
    int on, n;
    cudaEvent_t ev[kProfPairs][2];
    int phase[kProfPairs];
    int created;
    double ms[WC_PH_COUNT];
    unsigned long long cnt[WC_PH_COUNT];
} P;

void prof_drain()
{
    for (int i = 0; i < P.n; i++) {
        float t = 0.0f;
        cudaEventSynchronize(P.ev[i][1]);
        if (cudaEventElapsedTime(&t, P.ev[i][0], P.ev[i][1]) == cudaSuccess) {
            P.ms[P.phase[i]] += t;
            P.cnt[P.phase[i]]++;
        }
    }
    P.n = 0;
}

int prof_begin(int phase, cudaStream_t s)
{
    if (!P.on) return -1;
    if (P.n == kProfPairs) prof_drain();
    const int i = P.n++;
    P.phase[i] = phase;
    cudaEventRecord(P.ev[i][0], s);
    return i;
}

void prof_end(int i, cudaStream_t s)
{
    if (i >= 0) cudaEventRecord(P.ev[i][1], s);
}
} /* namespace */

extern "C" int wc_prof_enable(int on)
{
    if (on && !P.created) {
        for (int i = 0; i < kProfPairs; i++)
            for (int k = 0; k < 2; k++)
                if (cudaEventCreate(&P.ev[i][k]) != cudaSuccess) return -1;
        P.created = 1;
    }
    if (!on && P.on) prof_drain();
    P.on = on;
    return 0;
}

extern "C" void wc_prof_read(double *ms, unsigned long long *cnt, int nphase)
{
    prof_drain();
    for (int i = 0; i < nphase && i < WC_PH_COUNT; i++) {
        if (ms) ms[i] = P.ms[i];
        if (cnt) cnt[i] = P.cnt[i];
        P.ms[i] = 0;
        P.cnt[i] = 0;
    }
}

namespace {

/* ---- tile geometry ------------------------------------------------------ */

struct TileGeom {
    int nrb;        /* 64-row blocks in the matrix                          */
    int nrb_tile;   /* blocks per tile                                      */
    int nchunk;     /* row chunks                                           */
    int Q;          /* quarter-blocks (threads per lane) per tile           */
    int nlanes;     /* lanes splitting the slice's positions                */
    int nv, Vs, ns; /* positions, positions per slice, slices               */
    int threads;
    size_t smem;    /* bytes                                                */
};

TileGeom make_geom(int M, int N, int Vs, int stages)
{
    TileGeom g;
    g.nrb = (M + kBlock - 1) / kBlock;
    g.nrb_tile = g.nrb < 64 ? g.nrb : 64;
    g.nchunk = (g.nrb + g.nrb_tile - 1) / g.nrb_tile;
    g.nrb_tile = (g.nrb + g.nchunk - 1) / g.nchunk;
    g.Q = g.nrb_tile * 4;
    g.nv = N / kVecDim;
    g.Vs = Vs < g.nv ? Vs : g.nv;
    g.ns = (g.nv + g.Vs - 1) / g.Vs;
    int nl = 320 / g.Q;
    if (nl < 1) nl = 1;
    if (nl > g.Vs) nl = g.Vs;
    g.nlanes = nl;
    g.threads = g.Q * nl;
    const size_t lut = (size_t)g.Vs * stages * kEntries;
    const size_t red = (size_t)nl * g.nrb_tile * kBlock;
    g.smem = ((size_t)g.Vs * kVecDim + (lut > red ? lut : red)) * sizeof(float);
    return g;
}

/* The body every gather tile runs once xs (the slice's inputs, Vs*8 floats)
 * is in shared memory. Writes one partial sum per valid row to out[row]. */
template <int ST>
__device__ __forceinline__ void tile_gather(const uint8_t *__restrict__ mat,
                                            const TileGeom &g, int chunk,
                                            int slice, const float *xs,
                                            float *lut, const float *books,
                                            int cb, int M, float *out)
{
    const int v0 = slice * g.Vs;
    const int nvs = min(g.Vs, g.nv - v0);
    build_lut_slice<ST>(lut, xs, books, cb, nvs);
    __syncthreads();

    const int tid = threadIdx.x;
    const int lane = tid / g.Q, qi = tid % g.Q;
    const int rbl = qi >> 2, q = qi & 3;
    const int rb = chunk * g.nrb_tile + rbl;
    float acc[kRowsPerThread];
#pragma unroll
    for (int k = 0; k < kRowsPerThread; k++) acc[k] = 0.0f;
    const bool active = lane < g.nlanes && rbl < g.nrb_tile && rb < g.nrb;
    if (active) {
        const int vl0 = lane * nvs / g.nlanes, vl1 = (lane + 1) * nvs / g.nlanes;
        const uint8_t *p = mat + (((size_t)rb * g.nv + v0 + vl0) * kBlock + q * 16) * ST;
        gather16<ST>(acc, p, lut + (size_t)vl0 * ST * kEntries, vl1 - vl0);
    }
    __syncthreads();             /* the table is dead; reuse it for lanes */
    float *red = lut;
    const int R = g.nrb_tile * kBlock;
    if (active) {
#pragma unroll
        for (int k = 0; k < kRowsPerThread; k++)
            red[lane * R + rbl * kBlock + q * 16 + k] = acc[k];
    }
    __syncthreads();
    const int row0 = chunk * g.nrb_tile * kBlock;
    for (int r = tid; r < R; r += blockDim.x) {
        if (row0 + r >= M) break;
        float s = red[r];
        for (int l = 1; l < g.nlanes; l++) s += red[l * R + r];
        out[row0 + r] = s;
    }
}

/* ---- batched matvec (independent matrices, each with its own x) --------- */

template <int ST>
__global__ void __launch_bounds__(512)
matvec_tiles_kernel(TileGeom g, const wc_matvec_args a)
{
    const float *books = a.books;
    const int cb = a.cb_base, M = a.M;
    float *part = a.part;
    extern __shared__ float smem[];
    float *xs = smem, *lut = smem + g.Vs * kVecDim;
    const int per_g = g.ns * g.nchunk;
    const int gi = blockIdx.x / per_g, rem = blockIdx.x % per_g;
    const int slice = rem / g.nchunk, chunk = rem % g.nchunk;
    const int v0 = slice * g.Vs, nvs = min(g.Vs, g.nv - v0);
    const float *xg = a.x[gi] + (size_t)v0 * kVecDim;
    for (int i = threadIdx.x; i < nvs * kVecDim; i += blockDim.x) xs[i] = xg[i];
    __syncthreads();
    tile_gather<ST>(a.idx[gi], g, chunk, slice, xs, lut, books, cb, M,
                    part + ((size_t)gi * g.ns + slice) * M);
}

__global__ void matvec_reduce_kernel(int ns, const wc_matvec_args a)
{
    const int M = a.M;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= a.G * M) return;
    const int gi = i / M, r = i % M;
    const float *p = a.part + (size_t)gi * ns * M + r;
    float s = 0.0f;
    for (int k = 0; k < ns; k++) s += p[(size_t)k * M];
    a.y[gi][r] = s * f16_keep(a.scale[gi][r]);
}

/* ---- table build and dequantise (single kernels, for parity) ----------- */

template <int ST>
__global__ void lutb_kernel(float *lut, const float *x, const float *books,
                            int cb, int nv)
{
    /* one block per position */
    __shared__ float xs[kVecDim];
    const int v = blockIdx.x;
    if (threadIdx.x < kVecDim) xs[threadIdx.x] = x[(size_t)v * kVecDim + threadIdx.x];
    __syncthreads();
    build_lut_slice<ST>(lut + (size_t)v * ST * kEntries, xs, books, cb, 1);
}

template <int ST>
__global__ void dequant_kernel(float *W, const uint8_t *idx, const uint16_t *scale,
                               int M, int N, const float *books, int cb)
{
    const int nv = N / kVecDim;
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (size_t)M * nv) return;
    const int r = (int)(i / nv), v = (int)(i % nv);
    const uint8_t *ix = idx + (((size_t)(r / kBlock) * nv + v) * kBlock + r % kBlock) * ST;
    const float sc = f16_keep(scale[r]);
    float rec[kVecDim];
#pragma unroll
    for (int d = 0; d < kVecDim; d++) rec[d] = 0.0f;
#pragma unroll
    for (int s = 0; s < ST; s++) {
        const float *C = books + ((size_t)(cb + s) * kEntries + ix[s]) * kVecDim;
#pragma unroll
        for (int d = 0; d < kVecDim; d++) rec[d] = __fadd_rn(rec[d], C[d]);
    }
    float4 *dst = reinterpret_cast<float4 *>(W + (size_t)r * N + (size_t)v * kVecDim);
    dst[0] = make_float4(__fmul_rn(rec[0], sc), __fmul_rn(rec[1], sc),
                         __fmul_rn(rec[2], sc), __fmul_rn(rec[3], sc));
    dst[1] = make_float4(__fmul_rn(rec[4], sc), __fmul_rn(rec[5], sc),
                         __fmul_rn(rec[6], sc), __fmul_rn(rec[7], sc));
}

/* ---- MoE layer ------------------------------------------------------------ */

/* Warp-per-row dot products: the router (fp32 rows) and the shared expert's
 * gate/up (Q8G rows, src/model.c:265-320 layout), all reading x. */
__device__ __forceinline__ float warp_sum(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ float dot_f32_row(const float *__restrict__ w, const float *__restrict__ x,
                             int n, int lane)
{
    float acc = 0.0f;
    if ((n & 3) == 0) {
        const float4 *w4 = reinterpret_cast<const float4 *>(w);
        const float4 *x4 = reinterpret_cast<const float4 *>(x);
        for (int i = lane; i < n / 4; i += 32) {
            const float4 a = __ldg(w4 + i), b = __ldg(x4 + i);
            acc = fmaf(a.x, b.x, acc); acc = fmaf(a.y, b.y, acc);
            acc = fmaf(a.z, b.z, acc); acc = fmaf(a.w, b.w, acc);
        }
    } else {
        for (int i = lane; i < n; i += 32) acc = fmaf(w[i], x[i], acc);
    }
    return warp_sum(acc);
}

/* Q8G row: 16-byte chunks; chunk c covers inputs [16c, 16c+16) of group
 * c*16/128. Inputs at or past n (a partly filled last group) are skipped. */
__device__ float dot_q8g_row(const int8_t *__restrict__ row,
                             const uint16_t *__restrict__ ws,
                             const float *__restrict__ x, int n, int lane)
{
    float acc = 0.0f;
    const int nchunk = (n + 15) / 16;
    for (int c = lane; c < nchunk; c += 32) {
        const uint4 q = ldg16(row + (size_t)c * 16);
        const uint32_t wv[4] = { q.x, q.y, q.z, q.w };
        float part = 0.0f;
        const int base = c * 16;
#pragma unroll
        for (int i = 0; i < 16; i++) {
            if (base + i < n) {
                const int8_t b = (int8_t)((wv[i >> 2] >> (8 * (i & 3))) & 0xff);
                part = fmaf((float)b, x[base + i], part);
            }
        }
        acc = fmaf(f16_keep(ws[base / 128]), part, acc);
    }
    return warp_sum(acc);
}

__global__ void router_shared_kernel(wc_moe_args a)
{
    const int warps = blockDim.x / 32;
    const int row = blockIdx.x * warps + threadIdx.x / 32, lane = threadIdx.x % 32;
    const int lat = a.bank.lat;
    const int per_t = a.E + 2 * a.si;
    const int t = row / per_t, r = row % per_t;
    if (t >= a.T) return;
    const float *x = a.x + (size_t)t * lat;
    if (r < a.E) {
        const float v = dot_f32_row(a.router + (size_t)r * lat, x, lat, lane);
        if (lane == 0) a.ws.logits[(size_t)t * a.E + r] = v;
        return;
    }
    const int rr = r - a.E;
    const int kind = rr / a.si, o = rr % a.si;
    const int ng = (lat + 127) / 128;
    const size_t rowbytes = (size_t)ng * 128;
    const int8_t *W = kind ? a.shu : a.shg;
    const uint16_t *S = kind ? a.shu_s : a.shg_s;
    const float v = dot_q8g_row(W + (size_t)o * rowbytes, S + (size_t)o * ng, x, lat, lane);
    if (lane == 0) (kind ? a.ws.sh_u : a.ws.sh_g)[(size_t)t * a.si + o] = v;
}

/* Routing, src/model.c:2724-2747: score = 1/(1+expf(-logit)); K rounds of
 * argmax over score + bias (0.0f when there is no bias) with a strict >,
 * so the lowest index wins a tie and a NaN never wins; w = score[best];
 * optional renorm by (sum + 1e-20f) in j order; times routed_scale.
 * One warp per token. Also forms the shared expert's SiLU(g)*u. */
__global__ void route_kernel(wc_moe_args a)
{
    extern __shared__ float sm[];
    const int t = blockIdx.x;
    float *score = sm;
    const int E = a.E, K = a.K;
    const float *lg = a.ws.logits + (size_t)t * E;
    for (int e = threadIdx.x; e < E; e += blockDim.x)
        score[e] = 1.0f / (1.0f + expf(-lg[e]));
    if (a.si > 0) {
        for (int i = threadIdx.x; i < a.si; i += blockDim.x) {
            const size_t o = (size_t)t * a.si + i;
            a.ws.sh_h[o] = silu_ref(a.ws.sh_g[o]) * a.ws.sh_u[o];
        }
    }
    __syncthreads();
    if (threadIdx.x >= 32) return;
    const int lane = threadIdx.x;
    __shared__ int chosen[64];
    __shared__ float wsel[64];
    for (int j = 0; j < K; j++) {
        float bv = -1e30f;
        int best = -1;
        for (int e = lane; e < E; e += 32) {
            bool taken = false;
            for (int p = 0; p < j; p++) taken |= (chosen[p] == e);
            if (taken) continue;
            const float v = score[e] + (a.bias ? a.bias[e] : 0.0f);
            if (v > bv) { bv = v; best = e; }   /* e ascending per lane */
        }
        /* combine lanes: larger value wins; equal values -> lower index */
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, best, o);
            const bool take = (oi >= 0) && (best < 0 || ov > bv || (ov == bv && oi < best));
            if (take) { bv = ov; best = oi; }
        }
        if (lane == 0) {
            chosen[j] = best;
            wsel[j] = best >= 0 ? score[best] : 0.0f;
        }
        __syncwarp();
    }
    if (lane == 0) {
        if (a.renorm && K > 1) {
            float s = 0;
            for (int j = 0; j < K; j++) s += wsel[j];
            for (int j = 0; j < K; j++) wsel[j] /= (s + 1e-20f);
        }
        for (int j = 0; j < K; j++) {
            a.idx_out[(size_t)t * K + j] = chosen[j];
            a.w_out[(size_t)t * K + j] = wsel[j] * a.routed_scale;
        }
    }
}

struct MoeGeom {
    TileGeom gu, d;
    int gu_tiles, d_tiles, sh_blocks;
};

/* gate/up tiles: (t, kind, slice, j, chunk). */
template <int ST>
__global__ void __launch_bounds__(512)
gateup_kernel(wc_moe_args a, TileGeom g, const int *idx)
{
    extern __shared__ float smem[];
    float *xs = smem, *lut = smem + g.Vs * kVecDim;
    int b = blockIdx.x;
    const int chunk = b % g.nchunk; b /= g.nchunk;
    const int j = b % a.K; b /= a.K;
    const int slice = b % g.ns; b /= g.ns;
    const int kind = b % 2; const int t = b / 2;
    const wc_bank &bk = a.bank;
    const int v0 = slice * g.Vs, nvs = min(g.Vs, g.nv - v0);
    const float *xt = a.x + (size_t)t * bk.lat + (size_t)v0 * kVecDim;
    for (int i = threadIdx.x; i < nvs * kVecDim; i += blockDim.x) xs[i] = xt[i];
    __syncthreads();
    const int e = idx[(size_t)t * a.K + j] - bk.first;
    const uint8_t *rec = bk.base + (size_t)e * bk.rec_bytes;
    const uint8_t *mat = rec + (kind ? bk.up_off : bk.gate_off);
    float *out = a.ws.p_gu + ((((size_t)t * 2 + kind) * g.ns + slice) * a.K + j) * bk.inter;
    tile_gather<ST>(mat, g, chunk, slice, xs, lut, a.books, bk.cb_base + kind * ST,
                    bk.inter, out);
}

/* down tiles: (t, j, slice, chunk) with the SiLU(g)*u prologue; then the
 * shared expert's down rows (warp per row) in the trailing blocks. */
template <int ST>
__global__ void __launch_bounds__(512)
down_kernel(wc_moe_args a, TileGeom gu, TileGeom g, int d_tiles, const int *idx)
{
    extern __shared__ float smem[];
    const wc_bank &bk = a.bank;
    if ((int)blockIdx.x >= d_tiles) {
        /* shared expert down: [lat][si] Q8G, input sh_h */
        const int warps = blockDim.x / 32;
        const int row = (blockIdx.x - d_tiles) * warps + threadIdx.x / 32;
        const int lane = threadIdx.x % 32;
        const int t = row / bk.lat, o = row % bk.lat;
        if (t >= a.T) return;
        const int ng = (a.si + 127) / 128;
        const size_t rowbytes = (size_t)ng * 128;
        const float v = dot_q8g_row(a.shd + (size_t)o * rowbytes, a.shd_s + (size_t)o * ng,
                                    a.ws.sh_h + (size_t)t * a.si, a.si, lane);
        if (lane == 0) a.ws.sh_out[(size_t)t * bk.lat + o] = v;
        return;
    }
    float *xs = smem, *lut = smem + g.Vs * kVecDim;
    int b = blockIdx.x;
    const int chunk = b % g.nchunk; b /= g.nchunk;
    const int slice = b % g.ns; b /= g.ns;
    const int j = b % a.K; const int t = b / a.K;
    const int v0 = slice * g.Vs, nvs = min(g.Vs, g.nv - v0);
    const int e = idx[(size_t)t * a.K + j] - bk.first;
    const uint8_t *rec = bk.base + (size_t)e * bk.rec_bytes;
    const uint16_t *sc = reinterpret_cast<const uint16_t *>(rec + bk.scale_off);
    const int inter = bk.inter;
    const float *pg = a.ws.p_gu + (((size_t)t * 2 + 0) * gu.ns) * a.K * inter + (size_t)j * inter;
    const float *pu = a.ws.p_gu + (((size_t)t * 2 + 1) * gu.ns) * a.K * inter + (size_t)j * inter;
    const size_t sstride = (size_t)a.K * inter;
    for (int i = threadIdx.x; i < nvs * kVecDim; i += blockDim.x) {
        const int n = v0 * kVecDim + i;
        float sg = 0.0f, su = 0.0f;
        for (int s = 0; s < gu.ns; s++) {
            sg += pg[(size_t)s * sstride + n];
            su += pu[(size_t)s * sstride + n];
        }
        const float gv = sg * f16_keep(sc[n]);
        const float uv = su * f16_keep(sc[inter + n]);
        xs[i] = silu_ref(gv) * uv;
    }
    __syncthreads();
    float *out = a.ws.p_d + (((size_t)t * a.K + j) * g.ns + slice) * bk.lat;
    tile_gather<ST>(rec + bk.down_off, g, chunk, slice, xs, lut, a.books,
                    bk.cb_base + 2 * ST, bk.lat, out);
}

/* out[t][i] = sum_j w[j] * (f16(scale_down_j[i]) * sum_s P_d[t][j][s][i]),
 * j in router order (src/model.c:2908-2909) — or in ascending expert id
 * when order_by_id (moe_chunk, src/model.c:3632-3656) — then + shared. */
__global__ void combine_kernel(wc_moe_args a, TileGeom g, const int *idx,
                               const float *w)
{
    const wc_bank &bk = a.bank;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    const int t = blockIdx.y;
    if (i >= bk.lat) return;
    const int K = a.K;
    const int *it = idx + (size_t)t * K;
    const float *wt = w + (size_t)t * K;
    float y = 0.0f;
    int last = -1;
    for (int n = 0; n < K; n++) {
        int j = n;
        if (a.order_by_id) {          /* next larger id after `last` */
            int bj = -1;
            for (int q = 0; q < K; q++)
                if (it[q] > last && (bj < 0 || it[q] < it[bj])) bj = q;
            if (bj < 0) break;
            j = bj;
            last = it[bj];
            /* the reference takes the first j routed to this id */
            for (int q = 0; q < bj; q++) if (it[q] == it[bj]) { j = q; break; }
        }
        const float wj = wt[j];
        if (a.order_by_id && wj == 0.0f) continue;
        const int e = it[j] - bk.first;
        const uint16_t *sc = reinterpret_cast<const uint16_t *>(
            bk.base + (size_t)e * bk.rec_bytes + bk.scale_off) + 2 * bk.inter;
        const float *p = a.ws.p_d + (((size_t)t * K + j) * g.ns) * bk.lat + i;
        float s = 0.0f;
        for (int k = 0; k < g.ns; k++) s += p[(size_t)k * bk.lat];
        const float acc = s * f16_keep(sc[i]);
        y = __fadd_rn(y, __fmul_rn(wj, acc));
    }
    if (a.si > 0) y = __fadd_rn(y, a.ws.sh_out[(size_t)t * bk.lat + i]);
    a.out[(size_t)t * bk.lat + i] = y;
}

constexpr int kVsGateUp = 12;
constexpr int kVsDown = 8;

MoeGeom moe_geom(const wc_moe_args *a)
{
    MoeGeom m;
    const wc_bank &b = a->bank;
    m.gu = make_geom(b.inter, b.lat, kVsGateUp, b.stages);
    m.d = make_geom(b.lat, b.inter, kVsDown, b.stages);
    m.gu_tiles = a->T * 2 * m.gu.ns * a->K * m.gu.nchunk;
    m.d_tiles = a->T * a->K * m.d.ns * m.d.nchunk;
    const int warps = m.d.threads / 32;
    m.sh_blocks = a->si > 0 ? (a->T * b.lat + warps - 1) / warps : 0;
    return m;
}

template <int ST>
int moe_launch_st(const wc_moe_args *a, cudaStream_t s)
{
    const MoeGeom m = moe_geom(a);
    if (m.d.threads < 32 || m.d.threads % 32) { /* shared rows use whole warps */ }
    const int *idx = a->idx;
    const float *w = a->w;
    if (a->router) {
        const int rows = a->T * (a->E + 2 * a->si);
        int pe = prof_begin(WC_PH_ROUTER, s);
        router_shared_kernel<<<(rows + 7) / 8, 256, 0, s>>>(*a);
        prof_end(pe, s);
        pe = prof_begin(WC_PH_ROUTE, s);
        route_kernel<<<a->T, 256, (size_t)a->E * sizeof(float), s>>>(*a);
        prof_end(pe, s);
        g_launches += 2;
        idx = a->idx_out;
        w = a->w_out;
    }
    cudaFuncSetAttribute(gateup_kernel<ST>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)m.gu.smem);
    int pe = prof_begin(WC_PH_GATEUP, s);
    gateup_kernel<ST><<<m.gu_tiles, m.gu.threads, m.gu.smem, s>>>(*a, m.gu, idx);
    prof_end(pe, s);
    cudaFuncSetAttribute(down_kernel<ST>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)m.d.smem);
    const int dthreads = ((m.d.threads + 31) / 32) * 32;
    pe = prof_begin(WC_PH_DOWN, s);
    down_kernel<ST><<<m.d_tiles + (a->router ? m.sh_blocks : 0), dthreads, m.d.smem, s>>>(
        *a, m.gu, m.d, m.d_tiles, idx);
    prof_end(pe, s);
    dim3 cg((a->bank.lat + 255) / 256, a->T);
    wc_moe_args ca = *a;
    if (!a->router) ca.si = 0;
    pe = prof_begin(WC_PH_COMBINE, s);
    combine_kernel<<<cg, 256, 0, s>>>(ca, m.d, idx, w);
    prof_end(pe, s);
    g_launches += 3;
    return (int)cudaGetLastError();
}

} /* namespace */

extern "C" size_t wc_moe_ws_floats(int T, int K, int E, int lat, int inter, int si,
                                   int stages)
{
    const TileGeom gu = make_geom(inter, lat, kVsGateUp, stages);
    const TileGeom d = make_geom(lat, inter, kVsDown, stages);
    size_t n = 0;
    n += (size_t)T * 2 * gu.ns * K * inter;
    n += (size_t)T * K * d.ns * lat;
    n += (size_t)T * E;
    n += (size_t)T * si * 3 + (size_t)T * lat;
    return n + 64;
}

extern "C" void wc_moe_ws_carve(wc_moe_ws *ws, float *base, int T, int K, int E,
                                int lat, int inter, int si, int stages)
{
    const TileGeom gu = make_geom(inter, lat, kVsGateUp, stages);
    const TileGeom d = make_geom(lat, inter, kVsDown, stages);
    float *p = base;
    ws->p_gu = p; p += (size_t)T * 2 * gu.ns * K * inter;
    ws->p_d = p; p += (size_t)T * K * d.ns * lat;
    ws->logits = p; p += (size_t)T * E;
    ws->sh_g = p; p += (size_t)T * si;
    ws->sh_u = p; p += (size_t)T * si;
    ws->sh_h = p; p += (size_t)T * si;
    ws->sh_out = p;
}

extern "C" int wc_moe_launch(const wc_moe_args *a, void *stream)
{
    cudaStream_t s = (cudaStream_t)stream;
    switch (a->bank.stages) {
    case 3: return moe_launch_st<3>(a, s);
    case 2: return moe_launch_st<2>(a, s);
    default: return (int)cudaErrorInvalidValue;
    }
}

static constexpr int kVsMatvec = 16;

extern "C" size_t wc_matvec_part_floats(int G, int M, int N)
{
    const TileGeom g = make_geom(M, N, kVsMatvec, 3);
    return (size_t)G * g.ns * M;
}

template <int ST>
static int matvec_launch_st(const wc_matvec_args *a, cudaStream_t s)
{
    const TileGeom g = make_geom(a->M, a->N, kVsMatvec, ST);
    cudaFuncSetAttribute(matvec_tiles_kernel<ST>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)g.smem);
    const int tiles = a->G * g.ns * g.nchunk;
    int pe = prof_begin(WC_PH_MATVEC, s);
    matvec_tiles_kernel<ST><<<tiles, g.threads, g.smem, s>>>(g, *a);
    prof_end(pe, s);
    const int n = a->G * a->M;
    pe = prof_begin(WC_PH_MATVEC_REDUCE, s);
    matvec_reduce_kernel<<<(n + 255) / 256, 256, 0, s>>>(g.ns, *a);
    prof_end(pe, s);
    g_launches += 2;
    return (int)cudaGetLastError();
}

extern "C" int wc_matvec_launch(const wc_matvec_args *a, void *stream)
{
    cudaStream_t s = (cudaStream_t)stream;
    switch (a->stages) {
    case 3: return matvec_launch_st<3>(a, s);
    case 2: return matvec_launch_st<2>(a, s);
    default: return (int)cudaErrorInvalidValue;
    }
}

extern "C" int wc_lutb_launch(float *lut, const float *x, const float *books, int cb,
                              int nv, int stages, void *stream)
{
    cudaStream_t s = (cudaStream_t)stream;
    if (stages == 3) lutb_kernel<3><<<nv, 256, 0, s>>>(lut, x, books, cb, nv);
    else if (stages == 2) lutb_kernel<2><<<nv, 256, 0, s>>>(lut, x, books, cb, nv);
    else return (int)cudaErrorInvalidValue;
    g_launches += 1;
    return (int)cudaGetLastError();
}

extern "C" int wc_dequant_launch(float *W, const uint8_t *idx, const uint16_t *scale,
                                 int M, int N, const float *books, int cb, int stages,
                                 void *stream)
{
    cudaStream_t s = (cudaStream_t)stream;
    const size_t n = (size_t)M * (N / kVecDim);
    const unsigned blocks = (unsigned)((n + 255) / 256);
    if (stages == 3) dequant_kernel<3><<<blocks, 256, 0, s>>>(W, idx, scale, M, N, books, cb);
    else if (stages == 2) dequant_kernel<2><<<blocks, 256, 0, s>>>(W, idx, scale, M, N, books, cb);
    else return (int)cudaErrorInvalidValue;
    g_launches += 1;
    return (int)cudaGetLastError();
}
