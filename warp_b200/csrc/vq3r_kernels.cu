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

extern "C" int wc_profiling(void) { return P.on; }

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

constexpr int kMaxTopK = 64;

/* ---- tile geometry ------------------------------------------------------
 * A tile is (group of matrices that share one table slice, slice of vector
 * positions). Every thread owns 16 rows (a quarter of a 64-row index block)
 * of one matrix of the group and a contiguous run of the slice's positions
 * (its lane); lanes of the same rows are summed in shared memory in lane
 * order. */

struct TileGeom {
    int M, nrb;       /* rows per matrix, 64-row blocks per matrix           */
    int EG, groups;   /* matrices per tile, tiles along the matrix axis      */
    int nv, Vs, ns;   /* positions, positions per slice, slices              */
    int Q;            /* quarter-blocks per tile (threads per lane)          */
    int nlanes;
    int threads;
    size_t region;    /* floats: max(table, lane reduction), 16-byte multiple */
    size_t stage;     /* bytes of TMA-staged index streams (0: streamed)     */
    size_t smem;      /* bytes: barriers + xs + region + stage               */
};

/* Shared-memory carve-up of a tile: two mbarriers, the slice's inputs, the
 * table / lane-reduction region, then the staged index streams. */
struct TileSmem {
    uint64_t *bars;
    float *xs, *lut;
    uint8_t *stage;
    __device__ __forceinline__ TileSmem(unsigned char *raw, const TileGeom &g)
    {
        bars = reinterpret_cast<uint64_t *>(raw);
        xs = reinterpret_cast<float *>(raw + 16);
        lut = xs + ((g.Vs * kVecDim + 3) & ~3);
        /* TMA tensor copies land on 128-byte boundaries */
        const uintptr_t st = reinterpret_cast<uintptr_t>(lut + g.region);
        stage = reinterpret_cast<uint8_t *>((st + 127) & ~(uintptr_t)127);
    }
};

constexpr int kMaxTileRows = 8192;

TileGeom make_geom(int M, int N, int nmat, int Vs, int stages, int target_threads)
{
    TileGeom g;
    g.M = M;
    g.nrb = (M + kBlock - 1) / kBlock;
    int eg = kMaxTileRows / (g.nrb * kBlock);
    if (eg < 1) eg = 1;
    if (eg > nmat) eg = nmat;
    g.groups = (nmat + eg - 1) / eg;
    g.EG = (nmat + g.groups - 1) / g.groups;     /* balance the groups */
    g.Q = g.EG * g.nrb * 4;
    g.nv = N / kVecDim;
    g.Vs = Vs < g.nv ? Vs : g.nv;
    g.ns = (g.nv + g.Vs - 1) / g.Vs;
    int nl = target_threads / g.Q;
    if (nl < 1) nl = 1;
    if (nl > g.Vs) nl = g.Vs;
    while (g.Q * nl > 512 && nl > 1) nl--;
    g.nlanes = nl;
    g.threads = ((g.Q * nl + 31) / 32) * 32;
    const size_t lut = (size_t)g.Vs * stages * kEntries;
    /* the lane reduction reuses the table region; one lane needs none */
    const size_t red = nl > 1 ? (size_t)nl * g.EG * g.nrb * kBlock : 0;
    size_t region = lut > red ? lut : red;
    if (region < (size_t)2 * g.threads) region = (size_t)2 * g.threads;  /* down prologue */
    g.region = (region + 3) & ~(size_t)3;
    g.stage = 0;
    g.smem = 16 + (((size_t)g.Vs * kVecDim + 3) & ~(size_t)3) * sizeof(float) +
             g.region * sizeof(float);
    return g;
}

/* The same tile with its index streams staged in shared memory by TMA:
 * every (matrix, row block) of the group, the slice's positions. */
TileGeom with_stage(TileGeom g, int stages)
{
    g.stage = (size_t)g.EG * g.nrb * g.Vs * kBlock * stages;
    g.smem += g.stage + 128;       /* + the stage's 128-byte alignment */
    return g;
}

/* Per-thread part of a tile: which rows, which positions, and the index
 * stream, whose first loads are issued at construction. */
template <int ST, typename Gat = Gather16<ST>>
struct TileThread {
    int lane, m, rbl, q, vl0, vl1;
    bool active;
    Gat G;

    /* The matrix this thread's rows belong to (0 .. EG-1). */
    static __device__ __forceinline__ int matrix_of_thread(const TileGeom &g)
    {
        return (threadIdx.x % g.Q) / (g.nrb * 4);
    }

    TileThread() = default;

    /* mat: the index stream of matrix matrix_of_thread(g) (may be anything
     * when that matrix is past nm: the thread is then inactive). */
    __device__ __forceinline__ TileThread(const TileGeom &g, int slice, int nm,
                                          const uint8_t *mat)
    {
        const int tid = threadIdx.x;
        lane = tid / g.Q;
        const int qi = tid % g.Q;
        m = qi / (g.nrb * 4);
        const int rem = qi % (g.nrb * 4);
        rbl = rem >> 2;
        q = rem & 3;
        const int v0 = slice * g.Vs, nvs = min(g.Vs, g.nv - v0);
        active = lane < g.nlanes && m < nm;
        vl0 = lane * nvs / g.nlanes;
        vl1 = (lane + 1) * nvs / g.nlanes;
        if (active) {
            const uint8_t *p = mat + (((size_t)rbl * g.nv + v0 + vl0) * kBlock + q * 16) * ST;
            G.begin(p, vl1 - vl0);
        } else {
            G.n = 0;
        }
    }

    /* After the table is built: gather, reduce the lanes, and write one
     * partial sum per valid row to out[m * mstride + row]. */
    __device__ __forceinline__ void finish(const TileGeom &g, float *lut, float *out,
                                           size_t mstride, int nm, const int *slots = nullptr)
    {
        float acc[kRowsPerThread];
#pragma unroll
        for (int k = 0; k < kRowsPerThread; k++) acc[k] = 0.0f;
        if (active) G.run(acc, lut + (size_t)vl0 * ST * kEntries);
        if (g.nlanes == 1) {             /* the thread owns its rows outright */
            if (!active) return;
            const int row0 = rbl * kBlock + q * 16;
            float *dst = out + (size_t)(slots ? slots[m] : m) * mstride + row0;
            if (row0 + 16 <= g.M && ((reinterpret_cast<uintptr_t>(dst) & 15) == 0)) {
#pragma unroll
                for (int k = 0; k < kRowsPerThread; k += 4)
                    *reinterpret_cast<float4 *>(dst + k) =
                        make_float4(acc[k], acc[k + 1], acc[k + 2], acc[k + 3]);
            } else {
#pragma unroll
                for (int k = 0; k < kRowsPerThread; k++)
                    if (row0 + k < g.M) dst[k] = acc[k];
            }
            return;
        }
        __syncthreads();                 /* the table is dead; reuse it */
        float *red = lut;
        const int R = g.EG * g.nrb * kBlock;
        if (active) {
            float *dst = red + (size_t)lane * R + (size_t)m * g.nrb * kBlock + rbl * kBlock + q * 16;
#pragma unroll
            for (int k = 0; k < kRowsPerThread; k += 4)
                *reinterpret_cast<float4 *>(dst + k) =
                    make_float4(acc[k], acc[k + 1], acc[k + 2], acc[k + 3]);
        }
        __syncthreads();
        const int rows_pm = g.nrb * kBlock;
        for (int r = threadIdx.x; r < nm * rows_pm; r += blockDim.x) {
            const int mm = r / rows_pm, row = r % rows_pm;
            if (row >= g.M) continue;
            float s = red[r];
            for (int l = 1; l < g.nlanes; l++) s += red[(size_t)l * R + r];
            out[(size_t)(slots ? slots[mm] : mm) * mstride + row] = s;
        }
    }
};

/* ---- batched matvec (independent matrices, each with its own x) --------- */

template <int ST, int MAXT>
__global__ void __launch_bounds__(MAXT, 2)
matvec_tiles_kernel(TileGeom g, const wc_matvec_args a)
{
    extern __shared__ __align__(16) unsigned char smraw[];
    TileSmem sm(smraw, g);
    float *xs = sm.xs, *lut = sm.lut;
    const int gi = blockIdx.x / g.ns, slice = blockIdx.x % g.ns;
    TileThread<ST> th(g, slice, 1, a.idx[gi]);
    const int v0 = slice * g.Vs, nvs = min(g.Vs, g.nv - v0);
    const float *xg = a.x[gi] + (size_t)v0 * kVecDim;
    for (int i = threadIdx.x; i < nvs * kVecDim; i += blockDim.x) xs[i] = xg[i];
    __syncthreads();
    build_lut_slice<ST>(lut, xs, a.books, a.cb_base, nvs);
    __syncthreads();
    th.finish(g, lut, a.part + ((size_t)gi * g.ns + slice) * a.M, 0, 1);
}

/* The same tile for matrices of more than 2048 rows, where one lane of
 * quarter blocks covers the tile (thread t: row block t/4, quarter t%4) and
 * no lane reduction is needed: the mapping is fixed, the index words of two
 * positions are in flight before the table is built, and the partial sums
 * go straight from registers to memory. Vs = kVsM positions per tile. */
template <int ST, int MAXT, int kVsM>
__global__ void __launch_bounds__(MAXT)
matvec_rows_kernel(int ns, const wc_matvec_args a)
{
    extern __shared__ __align__(16) unsigned char smraw[];
    float *xs = reinterpret_cast<float *>(smraw);
    float *lut = xs + kVsM * kVecDim;
    const int gi = blockIdx.x / ns, slice = blockIdx.x % ns;
    const int nv = a.N / kVecDim, nrb = (a.M + kBlock - 1) / kBlock;
    const int rb = threadIdx.x >> 2, q = threadIdx.x & 3;
    const int v0 = slice * kVsM, nvs = min(kVsM, nv - v0);
    const bool active = rb < nrb;
    Gather16<ST> gat;
    const uint8_t *p = a.idx[gi] + (((size_t)rb * nv + v0) * kBlock + q * 16) * ST;
    if (active) gat.begin(p, nvs);
    else gat.n = 0;
    const float *xg = a.x[gi] + (size_t)v0 * kVecDim;
    for (int i = threadIdx.x; i < nvs * kVecDim; i += blockDim.x) xs[i] = xg[i];
    __syncthreads();
    build_lut_slice<ST>(lut, xs, a.books, a.cb_base, nvs);
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
    /* one block per position; build_lut_slice reads xs as float4 */
    __shared__ __align__(16) float xs[kVecDim];
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

/* ---- MoE layer ------------------------------------------------------------
 * Four launches per layer, chained with programmatic dependent launch (PDL)
 * so that each kernel's routing-independent prologue overlaps its
 * predecessor:
 *   1. router_kernel   router logits (fp32 rows, split in quarters) and the
 *                      shared expert's gate/up (Q8G rows); the last block to
 *                      finish runs the top-K and the shared SiLU(g)*u;
 *   2. gateup_kernel   [before the wait] stage x and build the gate or up
 *                      table slice — it depends on x and the codebooks only;
 *                      [after] gather the routed experts' gate/up rows, then
 *                      a share of the shared expert's down rows;
 *   3. down_kernel     [before] issue the routed expert's down index loads;
 *                      [after] SiLU(g)*u from the gate/up partials, table,
 *                      gather;
 *   4. combine_kernel  [before] row scales; [after] slice sums, the
 *                      router-order weighted reduce, + shared.
 * griddepcontrol.wait is a no-op for a kernel launched without PDL, so the
 * same kernels run unchanged behind a host copy. */

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;"); }

/* Ask L2 to fetch [p, p+bytes) from HBM (no registers, no shared memory:
 * cp.async.bulk.prefetch.L2). p 16-byte aligned, bytes a multiple of 16. */
__device__ __forceinline__ void l2_prefetch(const void *p, size_t bytes)
{
    const char *c = static_cast<const char *>(p);
    constexpr size_t kChunk = 64 * 1024;
    for (size_t off = 0; off < bytes; off += kChunk) {
        const uint32_t n = (uint32_t)(bytes - off < kChunk ? bytes - off : kChunk);
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(c + off), "r"(n) : "memory");
    }
}

__device__ __forceinline__ void st_release(unsigned int *p, unsigned int v)
{
    asm volatile("st.release.gpu.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned int ld_acquire(const unsigned int *p)
{
    unsigned int v;
    asm volatile("ld.acquire.gpu.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

/* Spins on a flag another CTA of an earlier kernel publishes. The kernels
 * that wait are launched only after every CTA of the publisher has started
 * (programmatic launch), so the publisher never waits for a slot they hold.
 * Bounded: after kSpinLimit polls (well over a second) the wait gives up,
 * records WC_ERR_ROUTE_WAIT and reports failure. */
constexpr long long kSpinLimit = 1ll << 24;

__device__ __forceinline__ bool wait_flag(const unsigned int *flag, unsigned int *err)
{
    /* the first polls back to back (the flag is usually a few hundred
     * nanoseconds away), then with a pause between them */
    for (long long i = 0; i < kSpinLimit; i++) {
        if (ld_acquire(flag)) return true;
        if (i >= 64) __nanosleep(64);
    }
    atomicOr(err, WC_ERR_ROUTE_WAIT);
    return false;
}

/* fetch-and-add with acquire-release semantics at GPU scope */
__device__ __forceinline__ unsigned int atomic_add_acq_rel(unsigned int *p, unsigned int v)
{
    unsigned int old;
    asm volatile("atom.add.acq_rel.gpu.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

/* ---- the expert-parallel exchange through peer memory --------------------
 * Flags are written by another GPU over NVLink: release/acquire at system
 * scope, and every wait is bounded (WC_ERR_PEER_WAIT, work skipped). */
__device__ __forceinline__ void st_release_sys(unsigned int *p, unsigned int v)
{
    asm volatile("st.release.sys.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned int ld_acquire_sys(const unsigned int *p)
{
    unsigned int v;
    asm volatile("ld.acquire.sys.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ unsigned int *ep_xflags(const wc_ep_link &l, int r)
{
    return reinterpret_cast<unsigned int *>(l.mail[r]);
}
__device__ __forceinline__ unsigned int *ep_pflags(const wc_ep_link &l, int r)
{
    return reinterpret_cast<unsigned int *>(l.mail[r] + 256);
}
__device__ __forceinline__ unsigned int *ep_ticket(const wc_ep_link &l)
{
    return reinterpret_cast<unsigned int *>(l.mail[l.rank] + 512);
}
__device__ __forceinline__ unsigned int *ep_epoch(const wc_ep_link &l)
{
    return reinterpret_cast<unsigned int *>(l.mail[l.rank] + 640);
}
/* rank r's mailbox: x [world][T][hidden], then part [world][T][hidden] */
__device__ __forceinline__ float *ep_x(const wc_ep_link &l, int r)
{
    return reinterpret_cast<float *>(l.mail[r] + WC_EP_MAIL_HDR);
}
__device__ __forceinline__ float *ep_part(const wc_ep_link &l, int r)
{
    return ep_x(l, r) + (size_t)l.world * l.T * l.hidden;
}

/* Rank r's poison word: set by any rank whose wait on a peer gave up. The
 * ranks' epochs are out of step from then on (the rank that called alone is
 * ahead), so a later wait could pass on a stale flag and read a mailbox that
 * another rank is rewriting; every wait checks this word first and fails
 * instead. Only new mailboxes (ep_init after ep_shutdown) clear it. */
__device__ __forceinline__ unsigned int *ep_poison(const wc_ep_link &l, int r)
{
    return reinterpret_cast<unsigned int *>(l.mail[r] + 768);
}

/* A wait that ran out: the error bit here, and the poison word in every
 * rank's mailbox, so every rank's next exchange fails too. */
__device__ __forceinline__ void ep_give_up(const wc_ep_link &l, unsigned int *err)
{
    atomicOr(err, WC_ERR_PEER_WAIT);
    for (int r = 0; r < l.world; r++) st_release_sys(ep_poison(l, r), 1u);
}

/* Until every rank's flag (in this rank's mailbox) reaches epoch e, or the
 * exchange is poisoned, or the poll limit runs out (false on either). */
__device__ __forceinline__ bool ep_wait_all(const wc_ep_link &l, const unsigned int *flags,
                                            unsigned int e, unsigned int *err)
{
    const unsigned int *poison = ep_poison(l, l.rank);
    if (ld_acquire_sys(poison)) {
        atomicOr(err, WC_ERR_PEER_WAIT);
        return false;
    }
    for (int r = 0; r < l.world; r++) {
        long long i = 0;
        while ((int)(ld_acquire_sys(flags + r) - e) < 0) {
            if (++i >= l.wait_polls || ((i & 255) == 0 && ld_acquire_sys(poison))) {
                ep_give_up(l, err);
                return false;
            }
            __nanosleep(64);
        }
    }
    return true;
}

/* Layer start: this rank's T tokens into every rank's mailbox (not with
 * rep: every rank has them already), then the x flag of this rank, at the
 * new epoch, in every mailbox. One block. */
__global__ void __launch_bounds__(256) ep_publish_kernel(wc_ep_link l, const float *x)
{
    __shared__ unsigned int e;
    pdl_trigger();                   /* the router may start staging its rows */
    pdl_wait();                      /* x: the previous kernel's output */
    if (threadIdx.x == 0) e = *ep_epoch(l) + 1;
    __syncthreads();
    const size_t n4 = (size_t)l.T * l.hidden / 4, off = (size_t)l.rank * l.T * l.hidden;
    const float4 *src = reinterpret_cast<const float4 *>(x);
    for (size_t i = threadIdx.x; i < (l.rep ? 0 : n4); i += blockDim.x) {
        const float4 v = src[i];
        for (int r = 0; r < l.world; r++) reinterpret_cast<float4 *>(ep_x(l, r) + off)[i] = v;
    }
    __syncthreads();                 /* every thread's stores before the releases */
    if ((int)threadIdx.x < l.world) st_release_sys(ep_xflags(l, threadIdx.x) + l.rank, e);
    if (threadIdx.x == 0) *ep_epoch(l) = e;       /* later kernels of this call read it */
}

/* Layer end: once every rank's partial sums of this rank's tokens are in,
 * out[t] = the sum over ranks in rank order. grid (ceil(hidden/256), T). */
__global__ void __launch_bounds__(256) ep_finalize_kernel(wc_ep_link l, float *out,
                                                         const float *resid, unsigned int *err)
{
    __shared__ int ok;
    /* launched programmatically behind the combine: nothing here reads what
     * the combine writes before the partial-sum flags say it is in (the
     * combine's last block releases this rank's flag after every block's
     * stores), so the grid-dependency wait is not needed; the next kernel
     * may start its own prologue at once */
    pdl_trigger();
    const unsigned int e = *ep_epoch(l);
    if (threadIdx.x == 0) ok = ep_wait_all(l, ep_pflags(l, l.rank), e, err);
    __syncthreads();
    if (!ok) return;
    for (int r = 0; r < l.world; r++) (void)ld_acquire_sys(ep_pflags(l, l.rank) + r);
    const int t = blockIdx.y, i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= l.hidden) return;
    const float *part = ep_part(l, l.rank);
    float y = 0.0f;
    for (int r = 0; r < l.world; r++)
        y = __fadd_rn(y, __ldcv(part + ((size_t)r * l.T + t) * l.hidden + i));
    if (resid) y = __fadd_rn(resid[(size_t)t * l.hidden + i], y);   /* the block's h + moe */
    out[(size_t)t * l.hidden + i] = y;
}

/* dst[0..n) = src[0..n) (global, written by an earlier phase) into shared
 * memory: every thread's loads issued before any store. n <= 8*blockDim. */
__device__ __forceinline__ void stage_floats(float *dst, const float *src, int n)
{
    constexpr int U = 8;
    float v[U];
#pragma unroll
    for (int k = 0; k < U; k++) {
        const int i = threadIdx.x + k * blockDim.x;
        v[k] = i < n ? __ldcg(src + i) : 0.0f;
    }
#pragma unroll
    for (int k = 0; k < U; k++) {
        const int i = threadIdx.x + k * blockDim.x;
        if (i < n) dst[i] = v[k];
    }
}

__device__ __forceinline__ float warp_sum(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

/* The reference's rmsnorm (src/model.c:132-138) of x[0..n) in shared
 * memory, in place: r = 1 / sqrtf(sum(x*x) / n + eps), x[i] = (x[i]*r)*w[i].
 * The sum of squares is a fixed tree (thread strides, warp shuffles, warps
 * in order), so every block that normalises the same x gets the same bits.
 * w: the weights, staged in shared memory with x (a global read per element
 * here would be a dependent round trip per loop step). red: blockDim/32 + 1
 * floats of shared memory. Every thread must call it. */
__device__ __forceinline__ void block_rmsnorm(float *x, int n, const float *w, float eps,
                                              float *red)
{
    float s = 0.0f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) s = __fadd_rn(s, __fmul_rn(x[i], x[i]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        float t = 0.0f;
        for (int k = 0; k < (int)(blockDim.x >> 5); k++) t = __fadd_rn(t, red[k]);
        red[32] = 1.0f / sqrtf(t / (float)n + eps);
    }
    __syncthreads();
    const float r = red[32];
    for (int i = threadIdx.x; i < n; i += blockDim.x) x[i] = __fmul_rn(__fmul_rn(x[i], r), w[i]);
    __syncthreads();
}

/* fp32 dot of w[0..n) with xs (shared memory), every load issued first.
 * n4 = n/4 must be <= 32*U4. */
template <int U4>
__device__ __forceinline__ float dot_f32_span(const float *__restrict__ w, const float *xs,
                                              int n4, int lane)
{
    const float4 *w4 = reinterpret_cast<const float4 *>(w);
    const float4 *x4 = reinterpret_cast<const float4 *>(xs);
    float4 a[U4];
#pragma unroll
    for (int u = 0; u < U4; u++) {
        const int i = u * 32 + lane;
        a[u] = i < n4 ? __ldg(w4 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float acc = 0.0f;
#pragma unroll
    for (int u = 0; u < U4; u++) {
        const int i = u * 32 + lane;
        if (i < n4) {
            const float4 b = x4[i];
            acc = fmaf(a[u].x, b.x, acc); acc = fmaf(a[u].y, b.y, acc);
            acc = fmaf(a[u].z, b.z, acc); acc = fmaf(a[u].w, b.w, acc);
        }
    }
    return warp_sum(acc);
}

/* Q8G row (src/model.c:265-320 layout: int8 rows padded to whole groups of
 * 128, one f16 scale per group) . x, with the row and its group scales in
 * shared memory. Step s
 * covers group s: lane l takes weights [128s + 4l, 128s + 4l + 4) (one
 * 32-bit word) and the matching float4 of x, so a warp step reads 128
 * contiguous weight bytes and 512 contiguous x bytes — no bank conflicts.
 * n must be a multiple of 4. */
__device__ __forceinline__ float dot_q8g_smem(const uint8_t *row, const float *gsc,
                                              const float *xs, int n, int lane)
{
    const int ng = (n + 127) / 128;
    float acc = 0.0f;
    for (int s = 0; s < ng; s++) {
        const int i = s * 128 + lane * 4;
        if (i < n) {
            const float4 wf = s8x4_to_f32(*reinterpret_cast<const uint32_t *>(row + i));
            const float4 xv = *reinterpret_cast<const float4 *>(xs + i);
            float part = wf.x * xv.x;
            part = fmaf(wf.y, xv.y, part);
            part = fmaf(wf.z, xv.z, part);
            part = fmaf(wf.w, xv.w, part);
            acc = fmaf(gsc[s], part, acc);
        }
    }
    return warp_sum(acc);
}

/* ---- 1. router (+ top-K in the last block) --------------------------------
 * Blocks of 8 warps: router blocks hold 2 rows, a quarter row per warp;
 * shared blocks hold 8 shared gate/up rows, a row per warp. Each thread
 * issues its weight loads and its share of x first, so a block costs one
 * DRAM round trip. The last block of a token (ticket) routes it. */
constexpr int kRouterBlock = 256;
constexpr int kRouterSplit = 4;        /* warps per router row              */
constexpr int kMaxPerLane = 32;        /* E <= 1024 (one live bit per lane entry) */
constexpr int kRouteMaxK = 32;         /* route_warp: lane j keeps choice j */
constexpr int kSiluU = 8;              /* shared SiLU inputs per thread held in registers */

struct RouterGeom {
    int rblocks;       /* blocks for the router rows (2 rows per block)      */
    int sblocks;       /* blocks for the shared gate/up rows (8 per block)   */
    int sblocks_base;  /* = rblocks                                          */
};

/* Shared rows go 8 to a block and never straddle the gate/up boundary
 * (si % 8 == 0, checked by the host), so each block's rows are one
 * contiguous run for TMA. */
__host__ __device__ inline RouterGeom router_geom(int E, int si)
{
    RouterGeom g;
    const int rows_pb = (kRouterBlock / 32) / kRouterSplit;
    g.rblocks = (E + rows_pb - 1) / rows_pb;
    g.sblocks = 2 * ((si + (kRouterBlock / 32) - 1) / (kRouterBlock / 32));
    g.sblocks_base = g.rblocks;
    return g;
}

/* Routing, src/model.c:2724-2747, by one warp, everything in registers:
 * lane l holds ids l, l+32, ... (NK of them): score = 1/(1+expf(-logit)),
 * v = score + bias (or + 0.0f when there is none). K rounds of argmax:
 * within a lane the ids ascend and the comparison is a strict >, across
 * lanes the larger value wins and equal values go to the lower id — so the
 * lowest id wins a tie and a NaN never wins, exactly as the sequential scan
 * from -1e30f does. w = score[best]; renorm by (sum + 1e-20f) accumulated in
 * j order; times routed_scale. */
/* A float as an unsigned key with the same order (-0 taken as +0): larger
 * float, larger key. Only finite values above -1e30 are keyed here (the
 * candidates the reference's scan can select), and their keys are nonzero. */
__device__ __forceinline__ uint32_t order_key(float f)
{
    const uint32_t u = __float_as_uint(f + 0.0f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

template <int NK>
__device__ void route_warp(const wc_moe_args &a, int t, int lane)
{
    const int E = a.E, K = a.K;
    const float *lg = a.ws.logits + (size_t)t * E;
    float sc[NK], v[NK];
#pragma unroll
    for (int k = 0; k < NK; k++) {
        const int e = lane + 32 * k;
        sc[k] = e < E ? __ldcg(lg + e) : 0.0f;
        v[k] = (e < E && a.bias) ? __ldg(a.bias + e) : 0.0f;
    }
    uint32_t live = 0;
#pragma unroll
    for (int k = 0; k < NK; k++) {
        const int e = lane + 32 * k;
        sc[k] = 1.0f / (1.0f + expf(-sc[k]));
        v[k] = sc[k] + v[k];
        if (e < E) live |= 1u << k;
    }
    float wsel = 0.0f, wsum = 0.0f;
    int mine = -1;                      /* lane j keeps the j-th choice */
    for (int j = 0; j < K; j++) {
        /* this lane's best: ids ascend within a lane, strict > from -1e30 */
        float bv = -1e30f, bsc = 0.0f;
        int bk = -1;
#pragma unroll
        for (int k = 0; k < NK; k++)
            if (((live >> k) & 1) && v[k] > bv) { bv = v[k]; bsc = sc[k]; bk = k; }
        /* the warp's largest value, then the lowest id holding it: the
         * reference's ascending scan with a strict > picks exactly that */
        const uint32_t key = bk >= 0 ? order_key(bv) : 0u;
        const uint32_t kmax = __reduce_max_sync(0xffffffffu, key);
        int best = -1;
        float wb = 0.0f;
        if (kmax != 0u) {                                    /* warp-uniform */
            const uint32_t cand = (bk >= 0 && key == kmax) ? (uint32_t)(lane + 32 * bk)
                                                           : 0xffffffffu;
            best = (int)__reduce_min_sync(0xffffffffu, cand);
            wb = __shfl_sync(0xffffffffu, bsc, best & 31);
            if ((best & 31) == lane) live &= ~(1u << (best >> 5));
        }
        if (lane == j) { mine = best; wsel = wb; }
        wsum += wb;                     /* the same j-order sum in every lane */
    }
    if (lane < K) {
        float w = wsel;
        if (a.renorm && K > 1) w /= (wsum + 1e-20f);
        a.idx_out[(size_t)t * K + lane] = mine;
        a.w_out[(size_t)t * K + lane] = w * a.routed_scale;
    }
}

template <int NK>
__global__ void __launch_bounds__(kRouterBlock) router_kernel(wc_moe_args a, RouterGeom rg)
{
    /* shared memory: barrier | x [lat] | staged weight rows | staged scales */
    extern __shared__ __align__(16) unsigned char smraw[];
    __shared__ float part[kRouterBlock / 32];
    __shared__ float nred[33];
    __shared__ unsigned int ticket;
    __shared__ int ep_fail;
    if (threadIdx.x == 0) ep_fail = 0;
    pdl_trigger();                   /* let gate/up start its table build */
    const int lat = a.bank.lat, n4 = lat / 4;
    const int t = blockIdx.y;
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int b = blockIdx.x;
    const bool is_router = b < rg.rblocks;
    const bool sh_here = t >= a.sh_t0 && t < a.sh_t1;     /* this token's shared rows */
    const int ng = (lat + 127) / 128;
    uint64_t *bar = reinterpret_cast<uint64_t *>(smraw);
    float *xs = reinterpret_cast<float *>(smraw + 16);
    uint8_t *wst = reinterpret_cast<uint8_t *>(xs + lat);
    const int rows_pb = (kRouterBlock / 32) / kRouterSplit;
    /* this block's rows: router rows [r0, r0+nr) or shared rows of one kind */
    int r0 = 0, nr = 0, kind = 0, o0 = 0;
    const uint8_t *wsrc = nullptr;
    uint32_t wbytes = 0;
    if (is_router) {
        r0 = b * rows_pb;
        nr = max(0, min(rows_pb, a.E - r0));
        wsrc = reinterpret_cast<const uint8_t *>(a.router + (size_t)r0 * lat);
        wbytes = (uint32_t)nr * lat * 4;
    } else {
        const int rr0 = (b - rg.sblocks_base) * (kRouterBlock / 32);
        kind = rr0 / a.si;
        o0 = rr0 % a.si;
        nr = sh_here ? max(0, min(kRouterBlock / 32, a.si - o0)) : 0;
        wsrc = reinterpret_cast<const uint8_t *>(kind ? a.shu : a.shg) + (size_t)o0 * ng * 128;
        wbytes = (uint32_t)nr * ng * 128;
    }
    uint16_t *sst = reinterpret_cast<uint16_t *>(wst + (size_t)(kRouterBlock / 32) * ng * 128);
    float *nws = reinterpret_cast<float *>(sst + (size_t)(kRouterBlock / 32) * ng);
    /* The weight rows (and the block's rmsnorm weights) depend on nothing
     * earlier in the stream: their copies are issued before the
     * grid-dependency wait, so they overlap the end of the previous kernel.
     * x, and every write this kernel makes, come after it. */
    if (threadIdx.x == 0) {
        mbar_init(bar, 1);
        mbar_fence_init();
        uint32_t tx = (uint32_t)lat * 4 + wbytes;
        const uint32_t sbytes = is_router ? 0u : (uint32_t)nr * ng * 2;
        const uint32_t nbytes = a.norm_w ? (uint32_t)lat * 4 : 0u;
        tx += sbytes + nbytes;
        mbar_expect_tx(bar, tx);
        if (wbytes) bulk_g2s(wst, wsrc, wbytes, bar);
        if (sbytes)
            bulk_g2s(sst, (kind ? a.shu_s : a.shg_s) + (size_t)o0 * ng, sbytes, bar);
        if (nbytes) bulk_g2s(nws, a.norm_w, nbytes, bar);
    }
    pdl_wait();
    if (threadIdx.x == 0) {
        if (a.ep.on) {            /* every rank's tokens are in this mailbox */
            if (!ep_wait_all(a.ep, ep_xflags(a.ep, a.ep.rank), *ep_epoch(a.ep), a.ws.err))
                ep_fail = 1;
            asm volatile("fence.proxy.async.global;" ::: "memory");   /* for the bulk copy */
        }
        /* x is complete: gate/up may build its tables (released even when a
         * peer wait failed, so no tile waits for it in vain). With the
         * rmsnorm in front, block 0 releases it once the normalised x is
         * written (below). */
        if (b == 0 && !a.norm_w) st_release(a.ws.x_flag + t, 1u);
        bulk_g2s(xs, a.x + (size_t)t * lat, (uint32_t)lat * 4, bar);
    }
    __syncthreads();
    /* block-uniform (the rmsnorm below synchronises the block) */
    const bool ok = __syncthreads_and(mbar_wait(bar, 0) && !ep_fail);   /* a missing peer: no dot products */
    if (!ok && !ep_fail && threadIdx.x == 0) atomicOr(a.ws.err, WC_ERR_TMA_WAIT);
    if (a.norm_w) {                  /* the MoE block: route and run on rmsnorm(x) */
        if (ok) block_rmsnorm(xs, lat, nws, a.norm_eps, nred);
        if (b == 0) {
            for (int i = threadIdx.x; ok && i < lat; i += blockDim.x)
                a.ws.xn[(size_t)t * lat + i] = xs[i];
            __syncthreads();
            if (threadIdx.x == 0) st_release(a.ws.x_flag + t, 1u);
        }
    }
    if (is_router) {
        const int lr = warp / kRouterSplit, qtr = warp % kRouterSplit;
        const int per = (n4 + kRouterSplit - 1) / kRouterSplit;
        const int q0 = qtr * per, q1 = min(n4, q0 + per);
        const float4 *w4 = reinterpret_cast<const float4 *>(wst) + (size_t)lr * n4;
        const float4 *x4 = reinterpret_cast<const float4 *>(xs);
        float acc = 0.0f;
        if (ok && lr < nr)
            for (int i = q0 + lane; i < q1; i += 32) {
                const float4 w = w4[i], xv = x4[i];
                acc = fmaf(w.x, xv.x, acc); acc = fmaf(w.y, xv.y, acc);
                acc = fmaf(w.z, xv.z, acc); acc = fmaf(w.w, xv.w, acc);
            }
        acc = warp_sum(acc);
        if (lane == 0) part[warp] = acc;
        __syncthreads();
        if ((int)threadIdx.x < nr) {
            const float *p = part + threadIdx.x * kRouterSplit;
            a.ws.logits[(size_t)t * a.E + r0 + threadIdx.x] = ((p[0] + p[1]) + p[2]) + p[3];
        }
    } else if (ok && warp < nr) {
        const uint8_t *row = wst + (size_t)warp * ng * 128;
        const uint16_t *srow = sst + (size_t)warp * ng;
        float acc = 0.0f;
        for (int gi = 0; gi < ng; gi++) {
            const int i = gi * 128 + lane * 4;
            if (i < lat) {
                const float4 wf = s8x4_to_f32(*reinterpret_cast<const uint32_t *>(row + i));
                const float4 xv = *reinterpret_cast<const float4 *>(xs + i);
                float part = wf.x * xv.x;
                part = fmaf(wf.y, xv.y, part);
                part = fmaf(wf.z, xv.z, part);
                part = fmaf(wf.w, xv.w, part);
                acc = fmaf(f16_keep(srow[gi]), part, acc);
            }
        }
        acc = warp_sum(acc);
        if (lane == 0) (kind ? a.ws.sh_u : a.ws.sh_g)[(size_t)t * a.si + o0 + warp] = acc;
    }
    /* the last block of this token routes it: the block's writes are
     * ordered before thread 0's release; its acquire orders the other
     * blocks' writes before the routing reads (all through L2) */
    /* Two tickets: the route waits only for the router blocks; the shared
     * expert's activation only for the shared blocks (its consumer, the
     * down kernel's shared blocks, waits on the shared flag). */
    unsigned int *tk = is_router ? a.ws.tickets + t : a.ws.sh_ticket + t;
    const unsigned int nblk = is_router ? (unsigned)rg.rblocks : (unsigned)rg.sblocks;
    __syncthreads();
    if (threadIdx.x == 0) ticket = atomic_add_acq_rel(tk, 1u);
    __syncthreads();
    if (ticket != nblk - 1) return;
    if (is_router) {
        if (warp == 0) route_warp<NK>(a, t, lane);
        __syncthreads();
        if (threadIdx.x == 0) {
            *tk = 0;                                   /* ready for the next launch */
            st_release(a.ws.route_flag + t, 1u);       /* gate/up may go */
        }
        return;
    }
    if (!sh_here) {
        if (threadIdx.x == 0) *tk = 0;
        return;
    }
    {
        float g[kSiluU], u[kSiluU];
        const int nt = blockDim.x;
#pragma unroll
        for (int k = 0; k < kSiluU; k++) {
            const int i = threadIdx.x + k * nt;
            g[k] = i < a.si ? __ldcg(a.ws.sh_g + (size_t)t * a.si + i) : 0.0f;
            u[k] = i < a.si ? __ldcg(a.ws.sh_u + (size_t)t * a.si + i) : 0.0f;
        }
#pragma unroll
        for (int k = 0; k < kSiluU; k++) {
            const int i = threadIdx.x + k * nt;
            if (i < a.si)
                a.ws.sh_h[(size_t)t * a.si + i] = act_pair(a.act, g[k], u[k], a.situ_beta,
                                                           a.situ_lbeta);
        }
        for (int i = threadIdx.x + kSiluU * nt; i < a.si; i += nt)   /* si > 2048 */
            a.ws.sh_h[(size_t)t * a.si + i] =
                act_pair(a.act, __ldcg(a.ws.sh_g + (size_t)t * a.si + i),
                         __ldcg(a.ws.sh_u + (size_t)t * a.si + i), a.situ_beta, a.situ_lbeta);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        *tk = 0;
        st_release(a.ws.sh_flag + t, 1u);              /* the shared down rows may go */
    }
}

/* The router for many tokens (T >= 16): a block holds TB tokens' x in
 * shared memory and streams its weight rows once for all of them (the
 * single-token kernel re-reads every row per token). Router blocks take rw
 * rows per warp, shared blocks 2*rw Q8G rows per warp. Each dot product
 * keeps the single-token kernel's order (four quarter rows, lane-strided
 * FMA chains, warp sums, then ((q0+q1)+q2)+q3; per Q8G group the scale
 * times the group's products), so both kernels give the same logits. The
 * last block of a token group routes its tokens, one warp each. */
constexpr int kRouterTB = 8;           /* tokens per block, at most */
/* Calls of at least this many tokens take the batched forms (the many-token
 * router, gate/up tiles that take further expert groups in rounds, the
 * separate SiLU kernel); smaller ones keep the latency forms of decode. */
constexpr int kBatchedT = 16;
constexpr int kRouterTokensMin = kBatchedT;
constexpr int kRtChunk = 8;            /* router weight float4 loads in flight per lane */
constexpr int kShChunk = 16;           /* shared-expert weight words in flight per lane */

struct RouterTGeom {
    int rblocks, sblocks, rw, TB;
};

__host__ inline RouterTGeom router_t_geom(int E, int si, int T, int lat)
{
    RouterTGeom g;
    int tb = (int)((112 * 1024) / ((size_t)lat * 4));
    tb = tb < 1 ? 1 : (tb > kRouterTB ? kRouterTB : tb);
    g.TB = tb < T ? tb : T;
    const int groups = (T + g.TB - 1) / g.TB;
    const int warps = kRouterBlock / 32;
    g.rw = 1;
    for (int rw = 4; rw > 1; rw /= 2) {     /* fewer, longer blocks while >= 4 per SM */
        const int rb = (E + warps * rw - 1) / (warps * rw);
        const int sb = (2 * si + warps * 2 * rw - 1) / (warps * 2 * rw);
        if ((rb + sb) * groups >= 4 * 148) { g.rw = rw; break; }
    }
    g.rblocks = (E + warps * g.rw - 1) / (warps * g.rw);
    g.sblocks = (2 * si + warps * 2 * g.rw - 1) / (warps * 2 * g.rw);
    return g;
}

template <int NK>
__global__ void __launch_bounds__(kRouterBlock) router_tokens_kernel(wc_moe_args a, RouterTGeom rg)
{
    extern __shared__ __align__(16) unsigned char smraw[];
    __shared__ float nred[33];
    __shared__ unsigned int ticket;
    __shared__ int ep_fail;
    if (threadIdx.x == 0) ep_fail = 0;
    pdl_trigger();
    const int lat = a.bank.lat, n4 = lat / 4, ng = (lat + 127) / 128;
    const int t0 = blockIdx.y * rg.TB, nt = min(rg.TB, a.T - t0);
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int warps = kRouterBlock / 32;
    const int b = blockIdx.x;
    const bool is_router = b < rg.rblocks;
    uint64_t *bar = reinterpret_cast<uint64_t *>(smraw);
    float *xs = reinterpret_cast<float *>(smraw + 16);
    /* this warp's rows: router rows [r0, r1) or shared rows [r0, r1) of the
     * 2*si gate-then-up rows */
    const int rpw = is_router ? rg.rw : 2 * rg.rw;
    const int nrows = is_router ? a.E : 2 * a.si;
    const int rb0 = (is_router ? b : b - rg.rblocks) * warps * rpw;
    const int r0 = min(nrows, rb0 + warp * rpw), r1 = min(nrows, r0 + rpw);
    /* tokens of the group that get the shared expert here */
    const int ts0 = max(0, a.sh_t0 - t0), ts1 = min(nt, a.sh_t1 - t0);
    float *nws = xs + (size_t)rg.TB * lat;          /* rmsnorm weights */
    if (threadIdx.x == 0) {
        mbar_init(bar, 1);
        mbar_fence_init();
        /* one arrival for every byte this block stages: the group's x (its
         * copy is issued after the dependency wait) and the rmsnorm
         * weights (constants: copied now) */
        mbar_expect_tx(bar, (uint32_t)(nt + (a.norm_w ? 1 : 0)) * lat * 4);
        if (a.norm_w) bulk_g2s(nws, a.norm_w, (uint32_t)lat * 4, bar);
    }
    /* the block's weight rows into L2 while the previous kernel finishes */
    if (lane == 0 && r1 > r0) {
        if (is_router) {
            l2_prefetch(a.router + (size_t)r0 * lat, (size_t)(r1 - r0) * lat * 4);
        } else if (ts1 > ts0) {
            for (int r = r0; r < r1; r++)
                l2_prefetch((r < a.si ? a.shg + (size_t)r * ng * 128
                                      : a.shu + (size_t)(r - a.si) * ng * 128), (size_t)ng * 128);
        }
    }
    pdl_wait();
    if (threadIdx.x == 0) {
        if (a.ep.on) {            /* every rank's tokens are in this mailbox */
            if (!ep_wait_all(a.ep, ep_xflags(a.ep, a.ep.rank), *ep_epoch(a.ep), a.ws.err))
                ep_fail = 1;
            asm volatile("fence.proxy.async.global;" ::: "memory");   /* for the bulk copy */
        }
        if (b == 0 && !a.norm_w)  /* the group's x is complete (see router_kernel) */
            for (int k = 0; k < nt; k++) st_release(a.ws.x_flag + t0 + k, 1u);
        bulk_g2s(xs, a.x + (size_t)t0 * lat, (uint32_t)nt * lat * 4, bar);
    }
    __syncthreads();
    const bool ok = __syncthreads_and(mbar_wait(bar, 0) && !ep_fail);
    if (!ok && !ep_fail && threadIdx.x == 0) atomicOr(a.ws.err, WC_ERR_TMA_WAIT);
    if (a.norm_w) {                  /* rmsnorm of each token, as in router_kernel */
        for (int k = 0; k < nt && ok; k++) block_rmsnorm(xs + (size_t)k * lat, lat, nws,
                                                         a.norm_eps, nred);
        if (b == 0) {
            for (int i = threadIdx.x; ok && i < nt * lat; i += blockDim.x)
                a.ws.xn[(size_t)t0 * lat + i] = xs[i];
            __syncthreads();
            if (threadIdx.x == 0)
                for (int k = 0; k < nt; k++) st_release(a.ws.x_flag + t0 + k, 1u);
        }
    }
    const float4 *x4 = reinterpret_cast<const float4 *>(xs);
    if (ok && is_router) {
        const int per = (n4 + kRouterSplit - 1) / kRouterSplit;
        for (int r = r0; r < r1; r++) {
            const float4 *w4 = reinterpret_cast<const float4 *>(a.router + (size_t)r * lat);
            float res[kRouterTB];
#pragma unroll
            for (int k = 0; k < kRouterTB; k++) res[k] = 0.0f;
            for (int qtr = 0; qtr < kRouterSplit; qtr++) {
                const int q0 = qtr * per, q1 = min(n4, q0 + per);
                float acc[kRouterTB];
#pragma unroll
                for (int k = 0; k < kRouterTB; k++) acc[k] = 0.0f;
                /* chunks of kRtChunk weight loads in flight at once; the
                 * FMA chain still runs over i ascending */
                for (int base = q0 + lane; base < q1; base += 32 * kRtChunk) {
                    float4 wv[kRtChunk];
#pragma unroll
                    for (int c = 0; c < kRtChunk; c++) {
                        const int i = base + 32 * c;
                        wv[c] = i < q1 ? __ldg(w4 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
                    }
#pragma unroll
                    for (int c = 0; c < kRtChunk; c++) {
                        const int i = base + 32 * c;
                        if (i >= q1) break;
                        const float4 w = wv[c];
#pragma unroll
                        for (int k = 0; k < kRouterTB; k++) {
                            if (k < nt) {
                                const float4 xv = x4[(size_t)k * n4 + i];
                                acc[k] = fmaf(w.x, xv.x, acc[k]); acc[k] = fmaf(w.y, xv.y, acc[k]);
                                acc[k] = fmaf(w.z, xv.z, acc[k]); acc[k] = fmaf(w.w, xv.w, acc[k]);
                            }
                        }
                    }
                }
#pragma unroll
                for (int k = 0; k < kRouterTB; k++) {
                    if (k < nt) {             /* block-uniform */
                        const float q = warp_sum(acc[k]);
                        res[k] = qtr == 0 ? q : res[k] + q;
                    }
                }
            }
            if (lane == 0)
                for (int k = 0; k < nt; k++) a.ws.logits[(size_t)(t0 + k) * a.E + r] = res[k];
        }
    } else if (ok && ts1 > ts0) {
        for (int r = r0; r < r1; r++) {
            const int kind = r >= a.si, o = kind ? r - a.si : r;
            const uint8_t *row = reinterpret_cast<const uint8_t *>(kind ? a.shu : a.shg) +
                                 (size_t)o * ng * 128;
            const uint16_t *srow = (kind ? a.shu_s : a.shg_s) + (size_t)o * ng;
            float acc[kRouterTB];
#pragma unroll
            for (int k = 0; k < kRouterTB; k++) acc[k] = 0.0f;
            for (int gb = 0; gb < ng; gb += kShChunk) {
                uint32_t wv[kShChunk];
                uint16_t sv[kShChunk];
#pragma unroll
                for (int c = 0; c < kShChunk; c++) {
                    const int gi = gb + c, i = gi * 128 + lane * 4;
                    wv[c] = (gi < ng && i < lat)
                                ? __ldg(reinterpret_cast<const unsigned int *>(row + i)) : 0u;
                    sv[c] = gi < ng ? __ldg(srow + gi) : (uint16_t)0;
                }
#pragma unroll
                for (int c = 0; c < kShChunk; c++) {
                    const int gi = gb + c, i = gi * 128 + lane * 4;
                    if (gi >= ng) break;
                    if (i >= lat) continue;
                    const float sc = f16_keep(sv[c]);
                    const float4 wf = s8x4_to_f32(wv[c]);
                    const float w0 = wf.x, w1 = wf.y, w2 = wf.z, w3 = wf.w;
#pragma unroll
                    for (int k = 0; k < kRouterTB; k++) {
                        if (k >= ts0 && k < ts1) {
                            const float4 xv = *reinterpret_cast<const float4 *>(xs + (size_t)k * lat + i);
                            float part = w0 * xv.x;
                            part = fmaf(w1, xv.y, part);
                            part = fmaf(w2, xv.z, part);
                            part = fmaf(w3, xv.w, part);
                            acc[k] = fmaf(sc, part, acc[k]);
                        }
                    }
                }
            }
#pragma unroll
            for (int k = 0; k < kRouterTB; k++) {
                if (k >= ts0 && k < ts1) {    /* block-uniform */
                    const float v = warp_sum(acc[k]);
                    if (lane == 0) (kind ? a.ws.sh_u : a.ws.sh_g)[(size_t)(t0 + k) * a.si + o] = v;
                }
            }
        }
    }
    /* the last block of this token group routes it (ordering as in the
     * single-token kernel: writes, barrier, acq_rel ticket) */
    /* two tickets, as in router_kernel: the group's route after its router
     * blocks, the shared activation after its shared blocks */
    unsigned int *tk = is_router ? a.ws.tickets + t0 : a.ws.sh_ticket + t0;
    const unsigned int nblk = is_router ? (unsigned)rg.rblocks : (unsigned)rg.sblocks;
    __syncthreads();
    if (threadIdx.x == 0) ticket = atomic_add_acq_rel(tk, 1u);
    __syncthreads();
    if (ticket != nblk - 1) return;
    if (is_router) {
        if (warp < nt) route_warp<NK>(a, t0 + warp, lane);
        __syncthreads();
        if (threadIdx.x == 0) {
            *tk = 0;                                   /* ready for the next launch */
            for (int k = 0; k < nt; k++) st_release(a.ws.route_flag + t0 + k, 1u);
        }
        return;
    }
    for (int k = ts0; k < ts1; k++) {
        const size_t tb = (size_t)(t0 + k) * a.si;
        for (int i = threadIdx.x; i < a.si; i += blockDim.x)
            a.ws.sh_h[tb + i] = act_pair(a.act, __ldcg(a.ws.sh_g + tb + i),
                                         __ldcg(a.ws.sh_u + tb + i), a.situ_beta, a.situ_lbeta);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        *tk = 0;
        for (int k = ts0; k < ts1; k++) st_release(a.ws.sh_flag + t0 + k, 1u);
    }
}

/* The record of routed expert j of token t (ids are global; a bank may hold
 * a contiguous subset starting at `first`). */
__device__ __forceinline__ const uint8_t *expert_rec(const wc_bank &bk, const int *idx,
                                                     int K, int t, int j)
{
    return bk.base + (size_t)(__ldcg(idx + (size_t)t * K + j) - bk.first) * bk.rec_bytes;
}

/* Whether routed expert j of token t is held by this bank. With expert
 * parallelism a rank's bank holds only its own range of ids; the others'
 * records are not in this GPU's memory, so no address is formed for them:
 * their tiles skip, and their contributions come from the owning rank. */
__device__ __forceinline__ bool expert_here(const wc_moe_args &a, const int *idx, int K, int t, int j)
{
    if (!a.partial_bank) return true;        /* every routed expert is held here */
    const int e = __ldcg(idx + (size_t)t * K + j) - a.bank.first;
    return e >= 0 && e < a.bank.n_experts;
}

/* ---- 2. gate/up ------------------------------------------------------------
 * tile = (token, kind, slice, expert group): one table slice shared by the
 * rows of every expert in the group. Before routing is known: x, the
 * codebook rows and the table. Then the wait — on the router's published
 * flag when the router runs in the same chain (no kernel-completion
 * latency), else the programmatic dependency — and the routed experts' index
 * streams come in by TMA in two halves; the gather starts on the first half
 * while the second lands. */
constexpr int kGuBooks = 2;            /* codebook rows per thread (768/512) */

template <int ST>
__global__ void __launch_bounds__(512, 1)
gateup_kernel(const __grid_constant__ wc_moe_args a, TileGeom g, const int *idx)
{
    extern __shared__ __align__(16) unsigned char smraw[];
    __shared__ int go, s_nloc;
    __shared__ int s_slot[kMaxTopK];
    TileSmem sm(smraw, g);
    int b = blockIdx.x;
    const int grp = b % g.groups; b /= g.groups;
    const int slice = b % g.ns; b /= g.ns;
    const int kind = b % 2; const int t = b / 2;
    const wc_bank &bk = a.bank;
    const int v0 = slice * g.Vs, nvs = min(g.Vs, g.nv - v0);
    if (threadIdx.x == 0) {
        mbar_init(&sm.bars[0], 1);
        mbar_init(&sm.bars[1], 1);
        mbar_fence_init();
    }
    /* routing-independent: x slice, codebook rows, the table — built while
     * the route is computed, unless this device holds so few of the experts
     * (gu_eg > 0) that most tiles find no work: then the route comes first.
     * With the router in the chain this grid starts while the router runs,
     * and the router itself may still be waiting on whatever wrote x (the
     * previous layer's combine, when layers are chained on one stream): x
     * is read only after the router's x flag, which the router releases once
     * its own grid-dependency wait has passed. The codebook rows are
     * constants and come first. Without the router this grid is launched in
     * stream order, after x is complete. */
    const bool route_first = a.partial_bank && a.gu_eg > 0;
    const float *xsrc = a.norm_w ? a.ws.xn : a.x;   /* the block: the router's rmsnorm(x) */
    BookRows<ST, kGuBooks> books;
    if (!route_first) {
        books.load(a.books, bk.cb_base + kind * ST);
        if (a.router) {
            if (threadIdx.x == 0) go = wait_flag(a.ws.x_flag + t, a.ws.err);
            __syncthreads();
            if (!go) return;
        }
        if ((int)threadIdx.x < nvs * kVecDim)
            sm.xs[threadIdx.x] = ld_pin_f32(xsrc + (size_t)t * bk.lat + (size_t)v0 * kVecDim + threadIdx.x);
        __syncthreads();
        books.build(sm.lut, sm.xs, nvs);
    }
    if (a.router) {
        if (threadIdx.x == 0) {
            go = wait_flag(a.ws.route_flag + t, a.ws.err);
            /* the last tile of this token to pass clears both flags (every
             * tile passed the x flag before the route flag) */
            const int per_t = 2 * g.ns * g.groups;
            if (atomicAdd(a.ws.route_pass + t, 1u) == (unsigned)per_t - 1) {
                a.ws.route_pass[t] = 0;
                a.ws.route_flag[t] = 0;
                a.ws.x_flag[t] = 0;
            }
        }
        __syncthreads();
        if (!go) return;
    } else {
        pdl_wait();
    }
    pdl_trigger();
    /* the group's route slots: slots j0.. of the token, or, with a partial
     * bank, the token's slots whose experts are held here, compacted; then
     * the tile takes groups grp, grp + groups, ... of them in rounds, with
     * one table (one lane of threads: the table is never reused as the lane
     * reduction) */
    int j0 = grp * g.EG;
    int nm;
    if (route_first) {
        if (threadIdx.x < 32) {                 /* one warp reads the routes at once */
            int n = 0;
            for (int jb = 0; jb < a.K; jb += 32) {
                const int j = jb + (int)threadIdx.x;
                const bool hj = j < a.K && expert_here(a, idx, a.K, t, j);
                const unsigned mk = __ballot_sync(0xffffffffu, hj);
                if (hj) s_slot[n + __popc(mk & ((1u << threadIdx.x) - 1u))] = j;
                n += __popc(mk);
            }
            if (threadIdx.x == 0) s_nloc = n;
        }
        __syncthreads();
        if (j0 >= s_nloc) return;               /* uniform: no local expert left */
        nm = min(g.EG, s_nloc - j0);
        books.load(a.books, bk.cb_base + kind * ST);
        if ((int)threadIdx.x < nvs * kVecDim)
            sm.xs[threadIdx.x] = ld_pin_f32(xsrc + (size_t)t * bk.lat + (size_t)v0 * kVecDim + threadIdx.x);
        __syncthreads();
        books.build(sm.lut, sm.xs, nvs);
    } else {
        nm = min(g.EG, a.K - j0);
        if ((int)threadIdx.x < nm) s_slot[j0 + threadIdx.x] = j0 + threadIdx.x;
        __syncthreads();
    }
    for (uint32_t round = 0;; round++) {
    const int *slot = s_slot + j0;              /* matrix m is route slot slot[m] */
    /* stage the group's index streams for this slice: (matrix, row block)
     * runs of nvs positions, in halves [0,h) and [h,nvs); matrices of
     * experts held by another rank are neither staged nor gathered
     * (route-first groups hold only local slots) */
    uint32_t here = 0;
    for (int mm = 0; mm < nm; mm++)
        if (route_first || expert_here(a, idx, a.K, t, slot[mm])) here |= 1u << mm;
    const uint32_t psz = kBlock * ST;
    const int h = (nvs + 1) / 2;
    const int ncopy = nm * g.nrb;
    const int nhere = __popc(here) * g.nrb;
    /* with the layer's tensor maps: two boxes per expert (the halves of its
     * row blocks), each half on its own barrier */
    const bool use_map = bk.tmap_ok;
    if (threadIdx.x == 0) {
        if (use_map) {
            const uint32_t box = (uint32_t)(g.nrb / 2) * nvs * psz;
            if (nhere) {
                mbar_expect_tx(&sm.bars[0], (uint32_t)__popc(here) * box);
                mbar_expect_tx(&sm.bars[1], (uint32_t)__popc(here) * box);
            }
        } else {
            if (nhere) mbar_expect_tx(&sm.bars[0], (uint32_t)nhere * h * psz);
            if (nhere && nvs > h) mbar_expect_tx(&sm.bars[1], (uint32_t)nhere * (nvs - h) * psz);
        }
    }
    __syncthreads();
    if (use_map && (int)threadIdx.x < nm && ((here >> threadIdx.x) & 1u)) {
        /* thread m issues expert m's two boxes: the route reads run in parallel */
        const int mm = threadIdx.x;
        const uint32_t box = (uint32_t)(g.nrb / 2) * nvs * psz;
        const int e = __ldcg(idx + (size_t)t * a.K + slot[mm]) - bk.first;
        uint8_t *dst = sm.stage + (size_t)mm * g.nrb * nvs * psz;
        tma_load_3d(dst, &bk.tmap[kind], v0 * 24, 0, e, &sm.bars[0]);
        tma_load_3d(dst + box, &bk.tmap[kind], v0 * 24, g.nrb / 2, e, &sm.bars[1]);
    }
    for (int c = threadIdx.x; c < ncopy && !use_map; c += blockDim.x) {
        const int m = c / g.nrb, rbl = c % g.nrb;
        if (!((here >> m) & 1u)) continue;
        const uint8_t *src = expert_rec(bk, idx, a.K, t, slot[m]) + (kind ? bk.up_off : bk.gate_off) +
                             ((size_t)rbl * g.nv + v0) * psz;
        uint8_t *dst = sm.stage + (size_t)(m * g.nrb + rbl) * nvs * psz;
        bulk_g2s(dst, src, h * psz, &sm.bars[0]);
        if (nvs > h) bulk_g2s(dst + (size_t)h * psz, src + (size_t)h * psz, (nvs - h) * psz, &sm.bars[1]);
    }
    if (threadIdx.x == 0 && t == 0 && round == 0 && a.prefetch_down) {
        /* this block's share of the routed experts' down index streams:
         * L2 fetches them while the gathers below keep HBM idle. Issued
         * once this tile's own streams have landed, so the prefetch does
         * not compete with them for HBM (bounded waits; a failure shows
         * again, and is reported, in the gather's own wait) */
        if (nhere) {
            mbar_wait(&sm.bars[0], round & 1u);
            if (use_map || nvs > h) mbar_wait(&sm.bars[1], round & 1u);
        }
        const size_t per = bk.scale_off - bk.down_off;
        const size_t total = per * (size_t)a.K * a.T;
        const int nb = gridDim.x;
        const size_t share = ((total + nb - 1) / nb + 15) & ~(size_t)15;
        size_t lo = (size_t)blockIdx.x * share, hi = min(total, lo + share);
        while (lo < hi) {
            const size_t jt = lo / per, off = lo % per;
            const size_t n = min(hi - lo, per - off) & ~(size_t)15;
            if (n == 0) break;
            const int e = __ldcg(idx + jt) - bk.first;
            if (e >= 0 && e < bk.n_experts)
                l2_prefetch(bk.base + (size_t)e * bk.rec_bytes + bk.down_off + off, n);
            lo += per - off;
        }
    }
    TileGeom gs = g;                 /* the staged view: positions [0, nvs) */
    gs.nv = nvs;
    gs.Vs = nvs;
    const int m = min(TileThread<ST, GatherSmem<ST>>::matrix_of_thread(g), nm - 1);
    TileThread<ST, GatherSmem<ST>> th(gs, 0, nm, sm.stage + (size_t)m * g.nrb * nvs * psz);
    th.active = th.active && ((here >> m) & 1u);
    th.G.first = th.vl0;
    if (use_map) {                   /* this thread's rows arrive with one box */
        th.G.bar0 = th.rbl < g.nrb / 2 ? &sm.bars[0] : &sm.bars[1];
        th.G.bar1 = nullptr;
    } else {
        th.G.bar0 = &sm.bars[0];
        th.G.bar1 = nvs > h ? &sm.bars[1] : nullptr;
    }
    th.G.split = h;
    th.G.par = round & 1u;
    __syncthreads();                 /* the table */
    float *out = a.ws.p_gu + ((((size_t)t * 2 + kind) * g.ns + slice) * a.K) * bk.inter;
    th.finish(gs, sm.lut, out, bk.inter, nm, slot);
    if (th.active && !th.G.ok) atomicOr(a.ws.err, WC_ERR_TMA_WAIT);
    if (!route_first || g.nlanes != 1) break;
    j0 += g.groups * g.EG;
    if (j0 >= s_nloc) break;         /* uniform */
    nm = min(g.EG, s_nloc - j0);
    __syncthreads();                 /* every gather is done with the staged streams */
    }
}

/* The down tile's gathers once its table is built: one partial sum per
 * output row of the slice. */
template <int ST>
__device__ __forceinline__ void down_gather(const wc_moe_args &a, const TileGeom &g, TileSmem &sm,
                                            int t, int j, int slice, int nvs)
{
    TileGeom gs = g;                 /* the staged view: positions [0, nvs) */
    gs.nv = nvs;
    gs.Vs = nvs;
    TileThread<ST, GatherSmem<ST>> th(gs, 0, 1, sm.stage);
    th.G.first = th.vl0;
    th.G.bar0 = &sm.bars[0];
    th.G.bar1 = nullptr;
    th.G.split = nvs;
    float *out = a.ws.p_d + (((size_t)t * a.K + j) * g.ns + slice) * a.bank.lat;
    th.finish(gs, sm.lut, out, 0, 1);
    if (th.active && !th.G.ok) atomicOr(a.ws.err, WC_ERR_TMA_WAIT);
}

/* ---- 3. down ---------------------------------------------------------------
 * tile = (token, expert j, slice). Before the wait (the route is known:
 * gate/up passed it before letting this kernel start): TMA stages the
 * expert's down index stream for the slice, and the gate/up row scales for
 * the slice's inputs and the codebook rows are loaded. After: the gate/up
 * slice sums (every load issued at once), SiLU(g)*u, the table, the gather
 * from shared memory. Blocks past d_tiles compute the shared expert's down
 * rows ([lat][si] Q8G, sh_rows_pw rows per warp, weights staged by TMA
 * before the wait). */
constexpr int kDnBooks = 2;            /* codebook rows per thread (768/432) */
constexpr int kDnSlices = 12;          /* gate/up slices summed per thread  */
constexpr int kShRowsMax = 12;         /* shared down rows per warp (shared memory) */

__device__ __forceinline__ void shared_down_block(const wc_moe_args &a, unsigned char *raw,
                                                  int sb, int rows_pw, int d_tiles)
{
    const wc_bank &bk = a.bank;
    const int warps = blockDim.x / 32, warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int ngs = (a.si + 127) / 128;
    const size_t rowb = (size_t)ngs * 128;
    const int row0 = sb * warps * rows_pw;
    const int nrows = max(0, min(warps * rows_pw, bk.lat - row0));
    uint64_t *bar = reinterpret_cast<uint64_t *>(raw);
    float *hs = reinterpret_cast<float *>(raw + 16);
    float *scs = hs + ((a.si + 3) & ~3);                   /* [nrows][ngs] scales */
    uint8_t *wst = reinterpret_cast<uint8_t *>(scs + ((warps * rows_pw * ngs + 3) & ~3));
    if (threadIdx.x == 0) {
        mbar_init(bar, 1);
        mbar_fence_init();
        if (nrows > 0) {
            mbar_expect_tx(bar, (uint32_t)(nrows * rowb));
            bulk_g2s(wst, a.shd + (size_t)row0 * rowb, (uint32_t)(nrows * rowb), bar);
        }
    }
    /* the rows' group scales, every load issued before any store */
    {
        constexpr int U = 4;
        const int n = nrows * ngs;
        uint16_t v[U];
#pragma unroll
        for (int k = 0; k < U; k++) {
            const int i = threadIdx.x + k * blockDim.x;
            v[k] = i < n ? ld_pin_u16(a.shd_s + (size_t)row0 * ngs + i) : (uint16_t)0;
        }
#pragma unroll
        for (int k = 0; k < U; k++) {
            const int i = threadIdx.x + k * blockDim.x;
            if (i < n) scs[i] = f16_keep(v[k]);
        }
        for (int i = threadIdx.x + U * blockDim.x; i < n; i += blockDim.x)
            scs[i] = f16_keep(ld_pin_u16(a.shd_s + (size_t)row0 * ngs + i));
    }
    pdl_trigger();
    pdl_wait();
    /* the shared activation of each token: the router's last shared block
     * raises its flag (every block of the router grid has started before
     * this grid launched, so the wait ends); the last of these blocks to
     * pass a token's flag clears it */
    __shared__ int sgo;
    if (threadIdx.x == 0) {
        sgo = 1;
        for (int tt = a.sh_t0; tt < a.sh_t1; tt++) {
            if (!wait_flag(a.ws.sh_flag + tt, a.ws.err)) { sgo = 0; break; }
            if (atomicAdd(a.ws.sh_pass + tt, 1u) == gridDim.x - (unsigned)d_tiles - 1) {
                a.ws.sh_pass[tt] = 0;
                a.ws.sh_flag[tt] = 0;
            }
        }
    }
    __syncthreads();
    const bool ok = sgo && (nrows == 0 || mbar_wait(bar, 0));
    if (!ok) {
        if (threadIdx.x == 0 && sgo) atomicOr(a.ws.err, WC_ERR_TMA_WAIT);
        return;
    }
    for (int tt = a.sh_t0; tt < a.sh_t1; tt++) {
        __syncthreads();
        stage_floats(hs, a.ws.sh_h + (size_t)tt * a.si, a.si);
        __syncthreads();
        for (int r = 0; r < rows_pw; r++) {
            const int lr = warp * rows_pw + r, o = row0 + lr;
            if (o >= bk.lat) break;
            const float acc = dot_q8g_smem(wst + (size_t)lr * rowb, scs + (size_t)lr * ngs, hs,
                                           a.si, lane);
            if (lane == 0) a.ws.sh_out[(size_t)tt * bk.lat + o] = acc;
        }
    }
}

template <int ST>
__global__ void __launch_bounds__(512, 1)
down_kernel(const __grid_constant__ wc_moe_args a, TileGeom gu, TileGeom g, int d_tiles,
            int sh_rows_pw, const int *idx)
{
    extern __shared__ __align__(16) unsigned char smraw[];
    const wc_bank &bk = a.bank;
    if ((int)blockIdx.x >= d_tiles) {
        shared_down_block(a, smraw, blockIdx.x - d_tiles, sh_rows_pw, d_tiles);
        return;
    }
    TileSmem sm(smraw, g);
    float *xs = sm.xs, *lut = sm.lut;
    int b = blockIdx.x;
    const int slice = b % g.ns; b /= g.ns;
    const int j = b % a.K; const int t = b / a.K;
    if (!expert_here(a, idx, a.K, t, j)) return;        /* another rank's expert */
    const int v0 = slice * g.Vs, nvs = min(g.Vs, g.nv - v0);
    const uint32_t psz = kBlock * ST;
    const uint8_t *rec = expert_rec(bk, idx, a.K, t, j);
    if (threadIdx.x == 0) {
        mbar_init(&sm.bars[0], 1);
        mbar_fence_init();
        mbar_expect_tx(&sm.bars[0], (uint32_t)g.nrb * nvs * psz);
        if (bk.tmap_ok)              /* the whole slice of the stream: one box */
            tma_load_3d(sm.stage, &bk.tmap[2], v0 * 24, 0,
                        __ldcg(idx + (size_t)t * a.K + j) - bk.first, &sm.bars[0]);
    }
    __syncthreads();
    for (int rbl = threadIdx.x; rbl < g.nrb && !bk.tmap_ok; rbl += blockDim.x)
        bulk_g2s(sm.stage + (size_t)rbl * nvs * psz,
                 rec + bk.down_off + ((size_t)rbl * g.nv + v0) * psz, nvs * psz, &sm.bars[0]);
    BookRows<ST, kDnBooks> books;
    books.load(a.books, bk.cb_base + 2 * ST);
    const int nin = nvs * kVecDim;
    const int inter = bk.inter;
    const uint16_t *sc = reinterpret_cast<const uint16_t *>(rec + bk.scale_off);
    float sg_scale = 0.0f, su_scale = 0.0f;
    if ((int)threadIdx.x < nin && !a.act_pre) {
        const int n = v0 * kVecDim + threadIdx.x;
        sg_scale = f16_keep(ld_pin_u16(sc + n));
        su_scale = f16_keep(ld_pin_u16(sc + inter + n));
    }
    pdl_trigger();
    pdl_wait();                      /* gate/up partials (or h) are complete */
    if (a.act_pre) {                 /* SiLU(g)*u of this slice, computed once */
        if ((int)threadIdx.x < nin)
            xs[threadIdx.x] = __ldcg(a.ws.h + ((size_t)t * a.K + j) * inter + v0 * kVecDim +
                                     threadIdx.x);
        __syncthreads();
        books.build(lut, xs, nvs);
        __syncthreads();
        down_gather<ST>(a, g, sm, t, j, slice, nvs);
        return;
    }
    const size_t sstride = (size_t)a.K * inter;
    const float *pg = a.ws.p_gu + (((size_t)t * 2 + 0) * gu.ns) * sstride + (size_t)j * inter;
    const float *pu = a.ws.p_gu + (((size_t)t * 2 + 1) * gu.ns) * sstride + (size_t)j * inter;
    /* part p of P sums slices p, p+P, ... (at most kDnSlices of them, all
     * loads issued at once); parts are then added in order */
    const int P = max(1, (int)blockDim.x / nin);
    float *red2 = lut;                         /* [P][2][nin], before the table */
    if ((int)threadIdx.x < P * nin) {
        const int i = threadIdx.x % nin, p = threadIdx.x / nin;
        const int n = v0 * kVecDim + i;
        float vg[kDnSlices], vu[kDnSlices];
#pragma unroll
        for (int k = 0; k < kDnSlices; k++) {
            const int s2 = p + k * P;
            vg[k] = s2 < gu.ns ? __ldcg(pg + (size_t)s2 * sstride + n) : 0.0f;
            vu[k] = s2 < gu.ns ? __ldcg(pu + (size_t)s2 * sstride + n) : 0.0f;
        }
        float sg = 0.0f, su = 0.0f;
#pragma unroll
        for (int k = 0; k < kDnSlices; k++) { sg += vg[k]; su += vu[k]; }
        for (int s2 = p + kDnSlices * P; s2 < gu.ns; s2 += P) {       /* not at our shapes */
            sg += __ldcg(pg + (size_t)s2 * sstride + n);
            su += __ldcg(pu + (size_t)s2 * sstride + n);
        }
        red2[(p * 2 + 0) * nin + i] = sg;
        red2[(p * 2 + 1) * nin + i] = su;
    }
    __syncthreads();
    if ((int)threadIdx.x < nin) {
        const int i = threadIdx.x;
        float sg = 0.0f, su = 0.0f;
        for (int p = 0; p < P; p++) {
            sg += red2[(p * 2 + 0) * nin + i];
            su += red2[(p * 2 + 1) * nin + i];
        }
        xs[i] = act_pair(a.act, sg * sg_scale, su * su_scale, a.situ_beta, a.situ_lbeta);
    }
    __syncthreads();
    books.build(lut, xs, nvs);
    __syncthreads();
    down_gather<ST>(a, g, sm, t, j, slice, nvs);
}

/* SiLU(g)*u for every (token, routed expert) of a batched call, once, in
 * the down tiles' arithmetic: the gate/up slice sums in P parts (part p:
 * slices p, p+P, ... ascending, the first kDnSlices of them padded with
 * zeros), the parts in order, then the f16 row scales. P is what the down
 * tile holding input n uses: its threads over its inputs. grid
 * (ceil(inter/256), T*K). */
template <int ST>
__global__ void __launch_bounds__(256) act_kernel(const __grid_constant__ wc_moe_args a,
                                                  TileGeom gu, TileGeom d, const int *idx)
{
    pdl_trigger();                   /* the down tiles stage their streams meanwhile */
    const wc_bank &bk = a.bank;
    const int pair = blockIdx.y, t = pair / a.K, j = pair % a.K;
    const int n = blockIdx.x * blockDim.x + threadIdx.x;
    const int inter = bk.inter;
    pdl_wait();                      /* gate/up partials are complete */
    if (n >= inter || !expert_here(a, idx, a.K, t, j)) return;
    const int dsl = n / (d.Vs * kVecDim);
    const int nin = min(d.Vs, d.nv - dsl * d.Vs) * kVecDim;
    const int P = max(1, d.threads / nin);
    const size_t sstride = (size_t)a.K * inter;
    const float *pg = a.ws.p_gu + (((size_t)t * 2 + 0) * gu.ns) * sstride + (size_t)j * inter + n;
    const float *pu = a.ws.p_gu + (((size_t)t * 2 + 1) * gu.ns) * sstride + (size_t)j * inter + n;
    float sg = 0.0f, su = 0.0f;
    for (int p = 0; p < P; p++) {
        float vg[kDnSlices], vu[kDnSlices];
#pragma unroll
        for (int k = 0; k < kDnSlices; k++) {
            const int s2 = p + k * P;
            vg[k] = s2 < gu.ns ? __ldcg(pg + (size_t)s2 * sstride) : 0.0f;
            vu[k] = s2 < gu.ns ? __ldcg(pu + (size_t)s2 * sstride) : 0.0f;
        }
        float g = 0.0f, u = 0.0f;
#pragma unroll
        for (int k = 0; k < kDnSlices; k++) { g += vg[k]; u += vu[k]; }
        for (int s2 = p + kDnSlices * P; s2 < gu.ns; s2 += P) {
            g += __ldcg(pg + (size_t)s2 * sstride);
            u += __ldcg(pu + (size_t)s2 * sstride);
        }
        sg += g;
        su += u;
    }
    const uint16_t *sc = reinterpret_cast<const uint16_t *>(expert_rec(bk, idx, a.K, t, j) +
                                                           bk.scale_off);
    const float gs = f16_keep(ld_pin_u16(sc + n)), us = f16_keep(ld_pin_u16(sc + inter + n));
    a.ws.h[(size_t)pair * inter + n] = act_pair(a.act, sg * gs, su * us, a.situ_beta,
                                                a.situ_lbeta);
}

/* ---- 4. combine --------------------------------------------------------------
 * out[t][i] = sum_j w[j] * (f16(scale_down_j[i]) * sum_s P_d[t][j][s][i]),
 * j in router order (src/model.c:2908-2909) — or in ascending expert id
 * when order_by_id (moe_chunk, src/model.c:3632-3656) — then + shared.
 * Block: 32 outputs x 8 expert lanes; every load issued up front. */
constexpr int kMaxSlicesReg = 16;

__global__ void __launch_bounds__(256) combine_kernel(wc_moe_args a, TileGeom g,
                                                      const int *idx, const float *w)
{
    __shared__ float accj[kMaxTopK][32];
    __shared__ int order[kMaxTopK];
    __shared__ float wsm[kMaxTopK];
    const wc_bank &bk = a.bank;
    const int t = blockIdx.y, K = a.K;
    const int il = threadIdx.x % 32, jl = threadIdx.x / 32;
    const int i = blockIdx.x * 32 + il;
    const int *it = idx + (size_t)t * K;
    const bool ok = i < bk.lat;
    /* before the wait: the row scales (the route is complete by now) */
    constexpr int kJ = kMaxTopK / 8;
    float scl[kJ];
#pragma unroll
    for (int n = 0; n < kJ; n++) {
        const int j = jl + 8 * n;
        scl[n] = 0.0f;
        if (j < K && ok && expert_here(a, it, K, 0, j)) {
            const uint16_t *sc = reinterpret_cast<const uint16_t *>(
                bk.base + (size_t)(__ldcg(it + j) - bk.first) * bk.rec_bytes + bk.scale_off) +
                2 * bk.inter;
            scl[n] = f16_keep(ld_pin_u16(sc + i));
        }
    }
    if (threadIdx.x == 0 && t == 0) {
        /* ranges the caller wants in L2 for what follows (the next layer's
         * router and shared expert), split over the blocks */
        for (int r = 0; r < 4; r++) {
            const size_t n = a.pf_bytes[r];
            if (!a.pf_ptr[r] || n == 0) continue;
            const size_t share = ((n + gridDim.x - 1) / gridDim.x + 15) & ~(size_t)15;
            const size_t lo = (size_t)blockIdx.x * share;
            if (lo < n) l2_prefetch(static_cast<const char *>(a.pf_ptr[r]) + lo,
                                    (min(n, lo + share) - lo) & ~(size_t)15);
        }
    }
    /* the route weights and the residual input are complete before this
     * layer's first kernel ran its own wait (the router wrote the weights;
     * the residual is the layer's input): read them before the wait */
    if (threadIdx.x < K) wsm[threadIdx.x] = __ldcg(w + (size_t)t * K + threadIdx.x);
    const float hres = (a.resid && !a.ep.on && jl == 0 && ok)
                           ? __ldcg(a.resid + (size_t)t * bk.lat + i) : 0.0f;
    pdl_wait();
    pdl_trigger();         /* down is done: the next layer's router may prefetch its rows */
    const bool sh_here = a.si > 0 && t >= a.sh_t0 && t < a.sh_t1;
    const float shv = (sh_here && jl == 0 && ok) ? __ldcg(a.ws.sh_out + (size_t)t * bk.lat + i)
                                                 : 0.0f;
#pragma unroll
    for (int n = 0; n < kJ; n++) {
        const int j = jl + 8 * n;
        if (j >= K) break;
        float s = 0.0f;
        if (ok && expert_here(a, it, K, 0, j)) {
            const float *p = a.ws.p_d + (((size_t)t * K + j) * g.ns) * bk.lat + i;
            float v[kMaxSlicesReg];
#pragma unroll
            for (int k = 0; k < kMaxSlicesReg; k++)
                v[k] = k < g.ns ? __ldcg(p + (size_t)k * bk.lat) : 0.0f;
#pragma unroll
            for (int k = 0; k < kMaxSlicesReg; k++) s += v[k];
            for (int k = kMaxSlicesReg; k < g.ns; k++) s += __ldcg(p + (size_t)k * bk.lat);
            s *= scl[n];
        }
        accj[j][il] = s;
    }
    if (threadIdx.x == 0) {
        int last = -1, nn = 0;
        for (int n = 0; n < K; n++) {
            int jj = n;
            if (a.order_by_id) {          /* next larger id, first j routed to it */
                jj = -1;
                for (int q = 0; q < K; q++) {
                    const int e = __ldcg(it + q);
                    if (e > last && (jj < 0 || e < __ldcg(it + jj))) jj = q;
                }
                if (jj >= 0) last = __ldcg(it + jj);
            }
            if (jj >= 0 && !expert_here(a, it, K, 0, jj)) continue;   /* held elsewhere */
            order[nn++] = jj;
        }
        for (; nn < K; nn++) order[nn] = -1;
    }
    __syncthreads();
    if (jl == 0 && ok) {
        float y = 0.0f;
        for (int n = 0; n < K; n++) {
            const int j = order[n];
            if (j < 0) break;
            const float wj = wsm[j];
            if (a.order_by_id && wj == 0.0f) continue;
            y = __fadd_rn(y, __fmul_rn(wj, accj[j][il]));
        }
        if (sh_here) y = __fadd_rn(y, shv);
        if (!a.ep.on) {
            /* the block's residual add, h + moe (src/model.c:3945) */
            if (a.resid) y = __fadd_rn(hres, y);
            a.out[(size_t)t * bk.lat + i] = y;
        } else if (!a.ep.rep) {   /* straight into the token's rank, over NVLink */
            const int owner = t / a.ep.T, tl = t % a.ep.T;
            ep_part(a.ep, owner)[((size_t)a.ep.rank * a.ep.T + tl) * a.ep.hidden + i] = y;
        } else {                  /* every rank holds the token: to all of them */
            for (int r = 0; r < a.ep.world; r++)
                ep_part(a.ep, r)[((size_t)a.ep.rank * a.ep.T + t) * a.ep.hidden + i] = y;
        }
    }
    if (!a.ep.on) return;
    /* the last block of this rank's combine tells every rank its partial
     * sums are in */
    __shared__ unsigned int last;
    __syncthreads();                 /* the block's stores happen before thread 0's fence */
    if (threadIdx.x == 0) {
        __threadfence_system();
        last = atomic_add_acq_rel(ep_ticket(a.ep), 1u) == gridDim.x * gridDim.y - 1;
    }
    __syncthreads();
    if (!last) return;
    if (threadIdx.x == 0) *ep_ticket(a.ep) = 0;
    __threadfence_system();
    if ((int)threadIdx.x < a.ep.world)
        st_release_sys(ep_pflags(a.ep, threadIdx.x) + a.ep.rank, *ep_epoch(a.ep));
}

/* Positions per gate/up tile: each slice's partial sums are written and
 * summed again by the down tiles, so wide experts take longer slices. */
extern "C" int wc_vs_gateup(int lat, int inter)
{
    /* 7168-wide experts: 224 slices of 4 positions would write and re-read
     * 3.7 MB of partial sums per (token, expert); 8 positions halve that
     * and the staged streams still fit while a tile holds at most 128 row
     * blocks (kMaxTileRows), i.e. while inter <= 8192 */
    return (lat >= 4096 && inter <= kMaxTileRows) ? 2 * WC_VS_GATEUP : WC_VS_GATEUP;
}
constexpr int kVsDown = WC_VS_DOWN;

struct MoeGeom {
    TileGeom gu, d;
    int gu_tiles, d_tiles, sh_blocks, sh_rows_pw;
};

constexpr int kSMs = 148;              /* B200 */

/* dynamic shared memory of a router block: barrier | x | the larger of two
 * router rows (fp32) and eight shared rows (Q8G) | their group scales */
size_t router_smem(int lat)
{
    const size_t ngr = ((size_t)lat + 127) / 128;
    size_t wmax = (size_t)((kRouterBlock / 32) / kRouterSplit) * lat * 4;
    const size_t wsh = (size_t)(kRouterBlock / 32) * ngr * 128;
    if (wsh > wmax) wmax = wsh;
    /* barrier | x | rows | scales | rmsnorm weights */
    return 16 + (size_t)lat * 4 + wmax + (size_t)(kRouterBlock / 32) * ngr * 2 + (size_t)lat * 4 + 16;
}

/* dynamic shared memory of a shared-down block: barrier | h | scales | rows */
size_t shared_down_smem(int threads, int rows_pw, int si)
{
    const size_t rows = (size_t)(threads / 32) * rows_pw, ngs = ((size_t)si + 127) / 128;
    return 16 + (((size_t)si + 3) & ~(size_t)3) * 4 + ((rows * ngs + 3) & ~(size_t)3) * 4 +
           rows * ngs * 128;
}

MoeGeom moe_geom(const wc_moe_args *a)
{
    MoeGeom m;
    const wc_bank &b = a->bank;
    if (a->partial_bank && a->gu_eg > 0) {
        /* experts spread over devices: tiles of the expected local count,
         * enough groups for the case where every routed expert is local */
        /* one lane per quarter block: small tiles, many per SM, and the
         * empty ones retire right after the route */
        const int q = a->gu_eg * ((b.inter + kBlock - 1) / kBlock) * 4;
        m.gu = with_stage(make_geom(b.inter, b.lat, a->gu_eg, wc_vs_gateup(b.lat, b.inter), b.stages, q), b.stages);
        /* decode-sized calls: every group its own tile (latency); batched
         * calls: tiles for the expected local count, each taking further
         * groups in rounds when a token has more (one lane: the table
         * survives) */
        const int full = (a->K + m.gu.EG - 1) / m.gu.EG;
        m.gu.groups = (m.gu.nlanes == 1 && a->T >= kBatchedT)
                          ? (a->gu_eg + m.gu.EG - 1) / m.gu.EG : full;
    } else {
        m.gu = with_stage(make_geom(b.inter, b.lat, a->K, wc_vs_gateup(b.lat, b.inter), b.stages, 512), b.stages);
    }
    m.d = with_stage(make_geom(b.lat, b.inter, 1, kVsDown, b.stages, 448), b.stages);
    m.gu_tiles = a->T * 2 * m.gu.ns * m.gu.groups;
    m.d_tiles = a->T * a->K * m.d.ns;
    /* the shared expert's down rows take the SMs the down tiles leave free
     * (one down block per SM), or a few more when there are none */
    const int warps = m.d.threads / 32;
    int free_sms = kSMs - m.d_tiles % kSMs;
    if (free_sms < 8) free_sms = 8;
    m.sh_rows_pw = (b.lat + free_sms * warps - 1) / (free_sms * warps);
    if (m.sh_rows_pw > kShRowsMax) m.sh_rows_pw = kShRowsMax;
    while (m.sh_rows_pw > 1 && shared_down_smem(m.d.threads, m.sh_rows_pw, a->si) > 227 * 1024)
        m.sh_rows_pw--;
    const int rows_pb = warps * m.sh_rows_pw;
    m.sh_blocks = a->si > 0 ? (b.lat + rows_pb - 1) / rows_pb : 0;
    return m;
}

/* The register-resident forms hold a fixed number of positions per thread;
 * shapes outside these bounds are refused by the host. */
bool moe_geom_ok(const MoeGeom &m, const wc_moe_args *a)
{
    if (!a->router) {   /* router/shared limits only apply to the whole layer */
        return a->K <= kMaxTopK && m.gu.smem <= 227 * 1024 && m.d.smem <= 227 * 1024;
    }

    if (router_smem(a->bank.lat) > 227 * 1024 || a->K > kRouteMaxK) return false;
    if (a->E > 32 * kMaxPerLane) return false;
    if (a->si > 0 && shared_down_smem(m.d.threads, m.sh_rows_pw, a->si) > 227 * 1024) return false;
    if (a->si % (kRouterBlock / 32) || a->bank.lat % 4 || a->si % 4) return false;
    if (m.gu.smem > 227 * 1024 || m.d.smem > 227 * 1024) return false;
    if (m.d.ns > kMaxSlicesReg * 8 || a->K > kMaxTopK) return false;
    return true;
}

template <typename... KArgs, typename... Args>
cudaError_t launch(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                   bool pdl, Args... args)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, args...);
}

template <int ST>
int moe_launch_st(const wc_moe_args *a, cudaStream_t s)
{
    const MoeGeom m = moe_geom(a);
    if (!moe_geom_ok(m, a)) return (int)cudaErrorInvalidValue;
    const int *idx = a->idx;
    const float *w = a->w;
    bool pdl = false;
    cudaError_t e = cudaSuccess;
    if (a->router) {
        if (a->E > 32 * kMaxPerLane) return (int)cudaErrorInvalidValue;
        const RouterGeom rg = router_geom(a->E, a->si);
        const int pe = prof_begin(WC_PH_ROUTER, s);
        const size_t rsm = router_smem(a->bank.lat);
        cudaFuncSetAttribute(router_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)rsm);
        cudaFuncSetAttribute(router_kernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)rsm);
        cudaFuncSetAttribute(router_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)rsm);
        const dim3 rgrid(rg.rblocks + rg.sblocks, a->T);
        /* programmatic launch: the router's weight copies overlap whatever
         * kernel precedes it in the stream (the previous layer's combine) */
        const bool rpdl = !P.on;
        if (a->T >= kRouterTokensMin) {   /* weights read once per token group */
            const RouterTGeom tg = router_t_geom(a->E, a->si, a->T, a->bank.lat);
            /* barrier | x of the group | rmsnorm weights */
            const size_t tsm = 16 + (size_t)(tg.TB + 1) * a->bank.lat * 4;
            const dim3 tgrid(tg.rblocks + tg.sblocks, (a->T + tg.TB - 1) / tg.TB);
            cudaFuncSetAttribute(router_tokens_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tsm);
            cudaFuncSetAttribute(router_tokens_kernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tsm);
            cudaFuncSetAttribute(router_tokens_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tsm);
            if (a->E <= 256)
                e = launch(router_tokens_kernel<8>, tgrid, dim3(kRouterBlock), tsm, s, rpdl, *a, tg);
            else if (a->E <= 512)
                e = launch(router_tokens_kernel<16>, tgrid, dim3(kRouterBlock), tsm, s, rpdl, *a, tg);
            else
                e = launch(router_tokens_kernel<32>, tgrid, dim3(kRouterBlock), tsm, s, rpdl, *a, tg);
        } else if (a->E <= 256)
            e = launch(router_kernel<8>, rgrid, dim3(kRouterBlock), rsm, s, rpdl, *a, rg);
        else if (a->E <= 512)
            e = launch(router_kernel<16>, rgrid, dim3(kRouterBlock), rsm, s, rpdl, *a, rg);
        else
            e = launch(router_kernel<32>, rgrid, dim3(kRouterBlock), rsm, s, rpdl, *a, rg);
        prof_end(pe, s);
        g_launches += 1;
        idx = a->idx_out;
        w = a->w_out;
        pdl = true;
        if (e != cudaSuccess) return (int)e;
    }
    const int prof = P.on;             /* events between kernels defeat PDL */
    cudaFuncSetAttribute(gateup_kernel<ST>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)m.gu.smem);
    int pe = prof_begin(WC_PH_GATEUP, s);
    e = launch(gateup_kernel<ST>, dim3(m.gu_tiles), dim3(m.gu.threads), m.gu.smem, s,
               pdl && !prof, *a, m.gu, idx);
    prof_end(pe, s);
    if (e != cudaSuccess) return (int)e;
    /* batched calls: SiLU(g)*u once per (token, expert) instead of in
     * every down tile, whose prologue would otherwise wait on ns_gu
     * partial sums per input */
    wc_moe_args da = *a;
    da.act_pre = a->T >= kBatchedT;
    if (da.act_pre) {
        pe = prof_begin(WC_PH_ACT, s);
        e = launch(act_kernel<ST>, dim3((a->bank.inter + 255) / 256, a->T * a->K), dim3(256), 0,
                   s, !prof, da, m.gu, m.d, idx);
        prof_end(pe, s);
        g_launches += 1;
        if (e != cudaSuccess) return (int)e;
    }
    size_t dsm = m.d.smem;
    if (a->router && a->si > 0) {
        const size_t shm = shared_down_smem(m.d.threads, m.sh_rows_pw, a->si);
        if (shm > dsm) dsm = shm;
    }
    cudaFuncSetAttribute(down_kernel<ST>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dsm);
    pe = prof_begin(WC_PH_DOWN, s);
    e = launch(down_kernel<ST>, dim3(m.d_tiles + (a->router ? m.sh_blocks : 0)),
               dim3(m.d.threads), dsm, s, !prof, da, m.gu, m.d, m.d_tiles, m.sh_rows_pw, idx);
    prof_end(pe, s);
    if (e != cudaSuccess) return (int)e;
    wc_moe_args ca = *a;
    if (!a->router) ca.si = 0;
    pe = prof_begin(WC_PH_COMBINE, s);
    e = launch(combine_kernel, dim3((a->bank.lat + 31) / 32, a->T), dim3(256), 0, s, !prof,
               ca, m.d, idx, w);
    prof_end(pe, s);
    g_launches += 3;
    if (e != cudaSuccess) return (int)e;
    return (int)cudaGetLastError();
}

} /* namespace */

extern "C" size_t wc_moe_ws_floats(int T, int K, int E, int lat, int inter, int si,
                                   int stages)
{
    const TileGeom gu = make_geom(inter, lat, K, wc_vs_gateup(lat, inter), stages, 512);
    const TileGeom d = make_geom(lat, inter, 1, kVsDown, stages, 448);
    size_t n = 0;
    n += (size_t)T * 2 * gu.ns * K * inter;
    n += (size_t)T * K * d.ns * lat;
    n += (size_t)T * E;
    n += (size_t)T * si * 3 + (size_t)T * lat;
    n += (size_t)T * K * inter;              /* h */
    n += (size_t)T * lat;                    /* xn */
    return n + WC_WS_CONTROL_WORDS + 64;     /* + control words */
}

extern "C" void wc_moe_ws_carve(wc_moe_ws *ws, float *base, int T, int K, int E,
                                int lat, int inter, int si, int stages)
{
    const TileGeom gu = make_geom(inter, lat, K, wc_vs_gateup(lat, inter), stages, 512);
    const TileGeom d = make_geom(lat, inter, 1, kVsDown, stages, 448);
    float *p = base;
    /* control words first (zeroed once at allocation, self-resetting):
     * tickets [0,64), route flags [64,128), pass counters [128,192), err
     * 192, x flags [256,320), shared tickets [320,384), shared flags
     * [384,448), shared pass counters [448,512) */
    ws->tickets = reinterpret_cast<unsigned int *>(p);
    ws->route_flag = ws->tickets + 64;
    ws->route_pass = ws->tickets + 128;
    ws->err = ws->tickets + 192;
    ws->x_flag = ws->tickets + 256;
    ws->sh_ticket = ws->tickets + 320;
    ws->sh_flag = ws->tickets + 384;
    ws->sh_pass = ws->tickets + 448;
    p += WC_WS_CONTROL_WORDS;
    ws->p_gu = p; p += (size_t)T * 2 * gu.ns * K * inter;
    ws->p_d = p; p += (size_t)T * K * d.ns * lat;
    ws->logits = p; p += (size_t)T * E;
    ws->sh_g = p; p += (size_t)T * si;
    ws->sh_u = p; p += (size_t)T * si;
    ws->sh_h = p; p += (size_t)T * si;
    ws->sh_out = p; p += (size_t)T * lat;
    ws->h = p; p += (size_t)T * K * inter;
    ws->xn = p;
}

extern "C" int wc_moe_supported(const wc_moe_args *a)
{
    const MoeGeom m = moe_geom(a);
    return moe_geom_ok(m, a) ? 0 : -1;
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

/* 8 positions per tile and a 256-thread target (one lane per quarter
 * block at M = 4096): four tiles per SM, each with a 24 KB table — the
 * shape that keeps the shared-memory pipe busiest (measured against 16/32
 * positions, 128-512 threads, and cluster-reduced slices). */
static constexpr int kVsMatvec = 8;

/* The allocation-free matvec's partial sums live here instead of in
 * cudaMalloc'd scratch: the array is part of this module's image, so it
 * exists on a device as soon as the module is loaded there. */
static __device__ __align__(256) float g_noalloc_part[WC_NOALLOC_PART_FLOATS];

extern "C" int wc_noalloc_part(float **ptr)
{
    return (int)cudaGetSymbolAddress((void **)ptr, g_noalloc_part);
}

/* Set-up of the allocation-free matvec on the current device: the array's
 * address, and the kernels that entry point launches, loaded now. Under
 * lazy module loading the module (and with it the 32 MiB array) and each
 * kernel's code are otherwise brought onto the device at their first use,
 * which would make that first call allocate. */
extern "C" int wc_noalloc_setup(float **ptr)
{
    cudaFuncAttributes fa;
    cudaError_t e = cudaGetSymbolAddress((void **)ptr, g_noalloc_part);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, matvec_rows_kernel<3, 256, kVsMatvec>);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, matvec_rows_kernel<3, 512, kVsMatvec>);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, matvec_rows_kernel<2, 256, kVsMatvec>);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, matvec_rows_kernel<2, 512, kVsMatvec>);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, matvec_tiles_kernel<3, 512>);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, matvec_tiles_kernel<2, 512>);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, matvec_reduce_kernel);
    return (int)e;
}

/* The architecture the loaded kernels were compiled for (100 = sm_100). */
extern "C" int wc_binary_version(void)
{
    cudaFuncAttributes fa;
    if (cudaFuncGetAttributes(&fa, matvec_reduce_kernel) != cudaSuccess) return -1;
    return fa.binaryVersion;
}

extern "C" void wc_count_launches(int n) { g_launches += (uint64_t)n; }

extern "C" size_t wc_matvec_part_floats(int G, int M, int N)
{
    const TileGeom g = make_geom(M, N, 1, kVsMatvec, 3, 256);
    return (size_t)G * g.ns * M;
}

template <int ST>
static int matvec_launch_st(const wc_matvec_args *a, cudaStream_t s)
{
    const TileGeom g = make_geom(a->M, a->N, 1, kVsMatvec, ST, 256);
    const int tiles = a->G * g.ns;
    int pe;
    if (g.nlanes == 1) {           /* M > 2048: one thread per quarter block */
        const int threads = ((g.nrb * 4 + 31) / 32) * 32;
        const size_t smem = ((size_t)kVsMatvec * kVecDim + (size_t)kVsMatvec * ST * kEntries) * 4;
        const auto k = threads <= 256 ? matvec_rows_kernel<ST, 256, kVsMatvec>
                                      : matvec_rows_kernel<ST, 512, kVsMatvec>;
        cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        pe = prof_begin(WC_PH_MATVEC, s);
        k<<<tiles, threads, smem, s>>>(g.ns, *a);
    } else {
        const auto k = matvec_tiles_kernel<ST, 512>;
        cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)g.smem);
        pe = prof_begin(WC_PH_MATVEC, s);
        k<<<tiles, g.threads, g.smem, s>>>(g, *a);
    }
    prof_end(pe, s);
    const int n = a->G * a->M;
    pe = prof_begin(WC_PH_MATVEC_REDUCE, s);
    matvec_reduce_kernel<<<(n + 255) / 256, 256, 0, s>>>(g.ns, *a);
    prof_end(pe, s);
    g_launches += 2;
    return (int)cudaGetLastError();
}

extern "C" int wc_matvec_reduce_launch(const wc_matvec_args *a, int ns, void *stream)
{
    const int n = a->G * a->M;
    const int pe = prof_begin(WC_PH_MATVEC_REDUCE, (cudaStream_t)stream);
    matvec_reduce_kernel<<<(n + 255) / 256, 256, 0, (cudaStream_t)stream>>>(ns, *a);
    prof_end(pe, (cudaStream_t)stream);
    g_launches += 1;
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

/* out[i] = resid[i] + y[i] (the block's residual add where no kernel of
 * the layer can do it: after an NCCL reduction). out may alias y. */
__global__ void resid_add_kernel(float *out, const float *resid, const float *y, size_t n)
{
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = __fadd_rn(resid[i], y[i]);
}

/* blockIdx.y = copy; every thread's loads issued before its stores. */
__global__ void __launch_bounds__(256) copy_words_kernel(const wc_copy_args c)
{
    pdl_trigger();                   /* the next kernel may stage its constants */
    pdl_wait();                      /* src: complete */
    const int k = blockIdx.y;
    if (k >= c.n) return;
    const uint32_t *src = static_cast<const uint32_t *>(c.src[k]);
    uint32_t *dst = static_cast<uint32_t *>(c.dst[k]);
    const size_t n = c.bytes[k] / 4, stride = (size_t)gridDim.x * blockDim.x;
    constexpr int U = 8;
    for (size_t base = (size_t)blockIdx.x * blockDim.x + threadIdx.x; base < n; base += U * stride) {
        uint32_t v[U];
#pragma unroll
        for (int u = 0; u < U; u++) {
            const size_t i = base + u * stride;
            v[u] = i < n ? __ldcv(src + i) : 0u;
        }
#pragma unroll
        for (int u = 0; u < U; u++) {
            const size_t i = base + u * stride;
            if (i < n) __stcs(dst + i, v[u]);
        }
    }
}

extern "C" int wc_copy_launch(const wc_copy_args *c, void *stream)
{
    size_t most = 0;
    for (int k = 0; k < c->n && k < WC_COPY_MAX; k++)
        if (c->bytes[k] > most) most = c->bytes[k];
    if (c->n <= 0 || c->n > WC_COPY_MAX || most == 0) return (int)cudaErrorInvalidValue;
    const size_t words = most / 4;
    unsigned blocks = (unsigned)((words + 256 * 8 - 1) / (256 * 8));
    if (blocks > 64) blocks = 64;
    const cudaError_t e = launch(copy_words_kernel, dim3(blocks, c->n), dim3(256), 0,
                                 (cudaStream_t)stream, c->pdl && !P.on, *c);
    g_launches += 1;
    return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

extern "C" int wc_resid_add_launch(float *out, const float *resid, const float *y, size_t n,
                                   void *stream)
{
    resid_add_kernel<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>(out, resid,
                                                                                 y, n);
    g_launches += 1;
    return (int)cudaGetLastError();
}

extern "C" int wc_ep_publish_launch(const wc_ep_link *l, const float *x, unsigned int *err,
                                    void *stream)
{
    (void)err;
    const int pe = prof_begin(WC_PH_EP_PUBLISH, (cudaStream_t)stream);
    const cudaError_t e = launch(ep_publish_kernel, dim3(1), dim3(256), 0, (cudaStream_t)stream,
                                 !P.on, *l, x);
    prof_end(pe, (cudaStream_t)stream);
    if (e != cudaSuccess) return (int)e;
    g_launches += 1;
    return (int)cudaGetLastError();
}

extern "C" int wc_ep_finalize_launch(const wc_ep_link *l, float *out, const float *resid,
                                     unsigned int *err, void *stream)
{
    const int pe = prof_begin(WC_PH_EP_FINALIZE, (cudaStream_t)stream);
    const cudaError_t e = launch(ep_finalize_kernel, dim3((l->hidden + 255) / 256, l->T),
                                 dim3(256), 0, (cudaStream_t)stream, !P.on, *l, out, resid, err);
    prof_end(pe, (cudaStream_t)stream);
    if (e != cudaSuccess) return (int)e;
    g_launches += 1;
    return (int)cudaGetLastError();
}
