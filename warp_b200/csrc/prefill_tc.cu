/*
 * prefill_tc.cu — the batched (prefill) routed-expert path on the 5th-
 * generation tensor cores (sm_100a tcgen05).
 *
 * What it computes is moe_chunk's expert loop (src/model.c:3585-3659): for
 * every token t and each of its K routed experts e (weights rw[t][j]),
 *   h = SiLU(G_e x_t) * (U_e x_t),   y = D_e h,
 *   out[t] = sum over its experts in ascending id of rw[t][j] * y.
 * With many tokens per expert this is a set of dense contractions, so
 * instead of per-token lookup tables (the decode path) each expert's
 * weights are dequantised into shared memory once per 128 tokens and fed
 * to tcgen05.mma with the tokens routed to it as the N dimension.
 *
 * Precision (results must stay within 2e-5 relative L2 of the fp32
 * reference): operands are split into fp16 hi + lo (x = hi + lo exactly to
 * ~22 bits) after an exact power-of-two pre-scale that keeps both halves in
 * fp16's normal range (per layer for the weights, per token for the
 * activations), and each K=16 step issues hi*hi + hi*lo + lo*hi. The
 * tensor core's fp32 accumulation loses ~2^-24 per accumulate, so the K
 * loop is spread round-robin over four TMEM accumulators and their sums
 * are added in registers in the epilogue: ~1e-6 per contraction.
 *
 * Pipeline for one call (one layer, T tokens):
 *   pf_bucket   routed (token, slot) pairs grouped by expert; tiles of at
 *               most 128 pairs per expert
 *   pf_split_x  x -> fp16 hi/lo with a per-token scale
 *   pf_gemm<0>  gate and up rows: tile (pairs, kind, 128 rows), K = hidden
 *   pf_split_h  h = SiLU(g) * u -> fp16 hi/lo with a per-pair scale
 *   pf_gemm<1>  down rows: tile (pairs, 128 rows), K = expert inter
 *   pf_combine  per token, experts in ascending id, weighted sum
 *
 * Every wait is bounded (mbarrier polls), sets an error bit on timeout,
 * and TMEM is freed on every path. No multicast, no clusters.
 */
#include "vq3r_common.cuh"
#include "wc_launch.h"

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

using namespace wc;

namespace {

constexpr int kPfRows = 128;          /* MMA M: weight rows per tile              */
constexpr int kPfTok = 128;           /* MMA N: routed pairs per tile             */
constexpr int kPfKs = 64;             /* K elements per step (8 vector positions) */
constexpr int kPfAcc = 4;             /* TMEM accumulators, round robin by step   */
constexpr int kPfThreads = 256;       /* two threads per weight row (4 positions each) */
constexpr int kPfMaxE = 1024;

/* shared memory of a GEMM tile. Operands use the K-major no-swizzle
 * core-matrix layout, [8 chunks][128 rows][16 bytes] per 64-wide K step:
 *   A  (dequantised weights, hi and lo): 2 stages            64 KB
 *   B  (token operand, hi and lo):       ring of 4 steps    128 KB
 *   indices of the step's weight rows:   ring of 4 steps     12 KB
 *   the kind's codebooks in fp16                             12 KB
 * The B and index rings are filled by cp.async two steps ahead, so their
 * global-memory latency hides behind the current step's dequantisation
 * and MMAs. */
constexpr int kPfOpBytes = 8 * 128 * 16;                      /* 16 KB */
constexpr int kPfAOff = 0;
constexpr int kPfBOff = kPfAOff + 2 * 2 * kPfOpBytes;
constexpr int kPfIdxBytes = 2 * 8 * 192;                       /* 3 KB  */
constexpr int kPfIdxOff = kPfBOff + 4 * 2 * kPfOpBytes;
constexpr int kPfBookOff = kPfIdxOff + 4 * kPfIdxBytes;
constexpr int kPfBookBytes = 3 * 256 * 8 * 2;                  /* 12 KB */
constexpr int kPfSmem = kPfBookOff + kPfBookBytes;              /* 216 KB */
static_assert(kPfSmem + 4096 <= 227 * 1024, "prefill tile exceeds shared memory");

/* 16-byte asynchronous copy global -> shared (zero-filled when !valid) */
__device__ __forceinline__ void cp_async16(void *dst, const void *src, bool valid)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;"
                 ::"r"(smem_u32(dst)), "l"(src), "r"(valid ? 16 : 0) : "memory");
}
__device__ __forceinline__ void cp_async_commit()
{
    asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait()
{
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ uint64_t sm_desc(uint32_t addr, uint32_t lbo, uint32_t sbo)
{
    /* tcgen05 shared-memory descriptor: start, leading and stride byte
     * offsets in 16-byte units, version 1, no swizzle */
    uint64_t d = (uint64_t)((addr >> 4) & 0x3FFF);
    d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
    d |= (uint64_t)1 << 46;
    return d;
}

/* kind::f16 instruction descriptor: fp32 accumulator, fp16 A and B, both
 * K-major, M = 128, N = kPfTok */
__device__ __forceinline__ uint32_t mma_idesc()
{
    return (1u << 4) | (0u << 7) | (0u << 10) | ((uint32_t)(kPfTok >> 3) << 17) |
           ((uint32_t)(kPfRows >> 4) << 24);
}

__device__ __forceinline__ void mma_f16(uint32_t tmem, uint64_t a, uint64_t b, uint32_t idesc,
                                        uint32_t accumulate)
{
    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n"
                 ::"r"(tmem), "l"(a), "l"(b), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0),
                   "r"(0));
}

__device__ __forceinline__ void mma_commit(uint64_t *bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 ::"r"(smem_u32(bar)) : "memory");
}

/* v = hi + lo in fp16 (hi the nearest fp16, lo the nearest fp16 to the rest) */
__device__ __forceinline__ void split_f16(float v, uint16_t &hi, uint16_t &lo)
{
    const __half h = __float2half_rn(v);
    hi = __half_as_ushort(h);
    lo = __half_as_ushort(__float2half_rn(v - __half2float(h)));
}

/* the same for two values at once, with packed conversions */
__device__ __forceinline__ void split_f16x2(float a, float b, __half2 &hi, __half2 &lo)
{
    hi = __floats2half2_rn(a, b);
    const float2 back = __half22float2(hi);
    lo = __floats2half2_rn(a - back.x, b - back.y);
}

/* 2^(14 - e) for the largest |value| m = f * 2^e (0.5 <= f < 1): scaled
 * values stay below 2^14, far from fp16's limit, and their low halves
 * stay normal for all but the smallest values. */
__device__ __forceinline__ float pow2_scale(float m)
{
    if (!(m > 0.0f) || !isfinite(m)) return 1.0f;
    int e;
    frexpf(m, &e);
    e = 14 - e;
    e = e > 100 ? 100 : (e < -100 ? -100 : e);
    return ldexpf(1.0f, e);
}

__device__ __forceinline__ float block_max(float v, float *red)
{
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    const int w = threadIdx.x / 32, l = threadIdx.x % 32, nw = blockDim.x / 32;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    float m = 0.0f;
    for (int i = 0; i < nw; i++) m = fmaxf(m, red[i]);
    return m;
}

/* ---- 1. pairs grouped by expert ------------------------------------------ */
__global__ void __launch_bounds__(1024) pf_bucket(wc_pf_args a)
{
    __shared__ int cnt[kPfMaxE], off[kPfMaxE];
    const int nb = a.bank.n_experts, np = a.T * a.K;
    for (int e = threadIdx.x; e < nb; e += blockDim.x) cnt[e] = 0;
    __syncthreads();
    for (int p = threadIdx.x; p < np; p += blockDim.x) {
        const int e = a.route[p] - a.bank.first;
        if (e >= 0 && e < nb) atomicAdd(&cnt[e], 1);
        else atomicOr(a.err, WC_ERR_BAD_EXPERT);      /* skipped: not held here */
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int o = 0, nt = 0;
        for (int e = 0; e < nb; e++) {
            off[e] = o;
            for (int s = 0; s < cnt[e]; s += kPfTok) {
                a.tile_e[nt] = e;
                a.tile_s[nt] = o + s;
                a.tile_n[nt] = min(kPfTok, cnt[e] - s);
                nt++;
            }
            o += cnt[e];
        }
        *a.ntiles = nt;
    }
    __syncthreads();
    for (int e = threadIdx.x; e < nb; e += blockDim.x) cnt[e] = 0;
    __syncthreads();
    for (int p = threadIdx.x; p < np; p += blockDim.x) {
        const int e = a.route[p] - a.bank.first;
        if (e >= 0 && e < nb) a.pairs[off[e] + atomicAdd(&cnt[e], 1)] = p;
    }
}

/* ---- 2/4. operands to fp16 hi/lo with a per-row power-of-two scale -------- */
__global__ void __launch_bounds__(256) pf_split_x(wc_pf_args a)
{
    __shared__ float red[8];
    const int t = blockIdx.x, n = a.bank.lat;
    const float *x = a.x + (size_t)t * n;
    float m = 0.0f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) m = fmaxf(m, fabsf(x[i]));
    const float s = pow2_scale(block_max(m, red));
    for (int i = threadIdx.x; i < n; i += blockDim.x)
        split_f16(x[i] * s, a.xh[(size_t)t * n + i], a.xl[(size_t)t * n + i]);
    if (threadIdx.x == 0) a.xinv[t] = 1.0f / s;
}

/* h = SiLU(g) * u (src/model.c:501, 2898), or SiTU (:505, :3646-3648), for
 * one routed pair */
__global__ void __launch_bounds__(256) pf_split_h(wc_pf_args a)
{
    __shared__ float red[8];
    const int i = blockIdx.x, n = a.bank.inter;
    const float *g = a.gu + (size_t)i * 2 * n, *u = g + n;
    float m = 0.0f;
    for (int k = threadIdx.x; k < n; k += blockDim.x)
        m = fmaxf(m, fabsf(act_pair(a.act, g[k], u[k], a.situ_beta, a.situ_lbeta)));
    const float s = pow2_scale(block_max(m, red));
    for (int k = threadIdx.x; k < n; k += blockDim.x)
        split_f16(act_pair(a.act, g[k], u[k], a.situ_beta, a.situ_lbeta) * s,
                  a.hh[(size_t)i * n + k], a.hl[(size_t)i * n + k]);
    if (threadIdx.x == 0) a.hinv[i] = 1.0f / s;
}

/* ---- 3/5. the tensor-core tile ---------------------------------------------
 * DOWN = 0: grid (tile, 2 * inter/128): gate or up rows [128 mb, 128 mb + 128)
 *           of expert tile_e over the tile's pairs, K = hidden.
 * DOWN = 1: grid (tile, hidden/128): down rows, K = inter.
 * Thread r owns weight row r: it dequantises that row for each K step
 * (((0 + C0[i0]) + C1[i1]) + C2[i2], times the kind's pre-scale) and, in
 * the epilogue, reads TMEM lane r. */
template <int DOWN>
__global__ void __launch_bounds__(kPfThreads, 1) pf_gemm(wc_pf_args a)
{
    extern __shared__ __align__(1024) unsigned char smraw[];
    __shared__ uint64_t bars[2];
    __shared__ uint32_t tmem_base;
    __shared__ int s_pair[kPfTok];
    __shared__ float s_inv[kPfTok];

    const int tile = blockIdx.x;
    if (tile >= *a.ntiles) return;                    /* uniform: before any TMEM use */
    const wc_bank &bk = a.bank;
    const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
    const int e = a.tile_e[tile], s0 = a.tile_s[tile], n = a.tile_n[tile];
    const int mb = blockIdx.y;
    int kind, m0, Kin, Mrows;
    if (!DOWN) {
        const int per = bk.inter / kPfRows;
        kind = mb / per;
        m0 = (mb % per) * kPfRows;
        Kin = bk.lat;
        Mrows = bk.inter;
    } else {
        kind = 2;
        m0 = mb * kPfRows;
        Kin = bk.inter;
        Mrows = bk.lat;
    }
    const int nv = Kin / kVecDim, nks = Kin / kPfKs;
    const uint8_t *rec = bk.base + (size_t)e * bk.rec_bytes;
    const uint32_t moff = kind == 0 ? bk.gate_off : (kind == 1 ? bk.up_off : bk.down_off);
    const uint8_t *mat = rec + moff;
    const uint16_t *rscale = reinterpret_cast<const uint16_t *>(rec + bk.scale_off) +
                             (kind == 0 ? 0 : (kind == 1 ? bk.inter : 2 * bk.inter));
    const float wsc = a.wscale[kind];

    uint16_t *cb = reinterpret_cast<uint16_t *>(smraw + kPfBookOff);

    /* TMEM: four accumulators of kPfTok fp32 columns */
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(smem_u32(&tmem_base)), "r"(kPfAcc * kPfTok));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    if (tid == 0) {
        mbar_init(&bars[0], 1);
        mbar_init(&bars[1], 1);
        mbar_fence_init();
    }
    /* the kind's codebooks as fp16 (exact: they were fp16 with subnormals
     * flushed), and the tile's pairs */
    {
        const float *src = a.books + (size_t)(bk.cb_base + kind * 3) * 256 * 8;
        for (int i = tid; i < 3 * 256 * 8; i += kPfThreads)
            cb[i] = __half_as_ushort(__float2half_rn(src[i]));
    }
    for (int j = tid; j < kPfTok; j += kPfThreads) {
        const int p = j < n ? a.pairs[s0 + j] : -1;
        s_pair[j] = p;
        s_inv[j] = j < n ? (DOWN ? a.hinv[s0 + j] : a.xinv[p / a.K]) : 0.0f;
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;");
    const uint32_t tmem = tmem_base;
    const uint32_t idesc = mma_idesc();
    const int rb0 = m0 / kBlock;

    /* this thread's B row (pair jb) and half of its 8 chunks: x of the
     * pair's token, or its h */
    const int jb = tid % kPfTok, chalf = tid / kPfTok;
    const bool jvalid = jb < n;
    const size_t brow = !jvalid ? 0 : (DOWN ? (size_t)(s0 + jb) : (size_t)(s_pair[jb] / a.K));
    const uint16_t *bh_src = (DOWN ? a.hh : a.xh) + brow * Kin;
    const uint16_t *bl_src = (DOWN ? a.hl : a.xl) + brow * Kin;

    /* step k's indices and B rows into ring slot k & 3 (one group per step,
     * empty past the end so the group count stays uniform) */
    auto issue = [&](int k) {
        if (k < nks) {
            const int slot = k & 3;
            uint8_t *six = smraw + kPfIdxOff + slot * kPfIdxBytes;
            const int v0 = k * (kPfKs / kVecDim);
            for (int c = tid; c < 2 * 96; c += kPfThreads) {
                const int r = c / 96, q = c % 96;
                cp_async16(six + r * 1536 + q * 16,
                           mat + ((size_t)(rb0 + r) * nv + v0) * kBlock * 3 + (size_t)q * 16, true);
            }
            unsigned char *bh = smraw + kPfBOff + slot * 2 * kPfOpBytes, *bl = bh + kPfOpBytes;
#pragma unroll
            for (int cc = 0; cc < 4; cc++) {
                const int c = chalf * 4 + cc;
                const int o = c * (kPfTok * 16) + (jb / 8) * 128 + (jb % 8) * 16;
                cp_async16(bh + o, bh_src + (size_t)k * kPfKs + c * 8, jvalid);
                cp_async16(bl + o, bl_src + (size_t)k * kPfKs + c * 8, jvalid);
            }
        }
        cp_async_commit();
    };

    bool ok = true;
    issue(0);
    issue(1);
    for (int ks = 0; ks < nks; ks++) {
        const int st = ks & 1, slot = ks & 3;
        /* A stage st and ring slot (ks+2)&3 were read by step ks-2's MMAs */
        if (ks >= 2) ok = mbar_wait(&bars[st], ((ks - 2) >> 1) & 1);
        if (!ok) break;
        issue(ks + 2);
        cp_async_wait<2>();                              /* step ks's group landed */
        __syncthreads();
        unsigned char *sa_hi = smraw + kPfAOff + st * 2 * kPfOpBytes;
        unsigned char *sa_lo = sa_hi + kPfOpBytes;
        unsigned char *sb_hi = smraw + kPfBOff + slot * 2 * kPfOpBytes;
        unsigned char *sb_lo = sb_hi + kPfOpBytes;
        const uint8_t *six = smraw + kPfIdxOff + slot * kPfIdxBytes;
        /* A: row m0 + r, positions 4*vh .. 4*vh+3 of the step's 8 */
        {
            const int r = tid % kPfRows, vh = tid / kPfRows, rbl = r / kBlock, rr = r % kBlock;
#pragma unroll 2
            for (int v = 4 * vh; v < 4 * vh + 4; v++) {
                const uint8_t *ib = six + rbl * 1536 + v * 192 + rr * 3;
                const uint4 c0 = *reinterpret_cast<const uint4 *>(cb + ((0 * 256 + ib[0]) << 3));
                const uint4 c1 = *reinterpret_cast<const uint4 *>(cb + ((1 * 256 + ib[1]) << 3));
                const uint4 c2 = *reinterpret_cast<const uint4 *>(cb + ((2 * 256 + ib[2]) << 3));
                const __half2 *h0 = reinterpret_cast<const __half2 *>(&c0);
                const __half2 *h1 = reinterpret_cast<const __half2 *>(&c1);
                const __half2 *h2 = reinterpret_cast<const __half2 *>(&c2);
                __align__(16) __half2 hi[4], lo[4];
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    const float2 f0 = __half22float2(h0[q]), f1 = __half22float2(h1[q]),
                                 f2 = __half22float2(h2[q]);
                    const float wa = ((0.0f + f0.x) + f1.x) + f2.x;
                    const float wb = ((0.0f + f0.y) + f1.y) + f2.y;
                    split_f16x2(wa * wsc, wb * wsc, hi[q], lo[q]);
                }
                const int o = v * (kPfRows * 16) + (r / 8) * 128 + (r % 8) * 16;
                *reinterpret_cast<uint4 *>(sa_hi + o) = *reinterpret_cast<const uint4 *>(hi);
                *reinterpret_cast<uint4 *>(sa_lo + o) = *reinterpret_cast<const uint4 *>(lo);
            }
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  /* visible to the MMA */
        __syncthreads();
        if (tid == 0) {
            asm volatile("tcgen05.fence::after_thread_sync;");
            const uint32_t acc = tmem + (uint32_t)((ks % kPfAcc) * kPfTok);
#pragma unroll
            for (int sub = 0; sub < 4; sub++) {
                const uint32_t ao = sub * 2 * (kPfRows * 16), bo = sub * 2 * (kPfTok * 16);
                const uint64_t ah = sm_desc(smem_u32(sa_hi) + ao, kPfRows * 16, 128);
                const uint64_t al = sm_desc(smem_u32(sa_lo) + ao, kPfRows * 16, 128);
                const uint64_t bh = sm_desc(smem_u32(sb_hi) + bo, kPfTok * 16, 128);
                const uint64_t bl = sm_desc(smem_u32(sb_lo) + bo, kPfTok * 16, 128);
                mma_f16(acc, ah, bh, idesc, (ks >= kPfAcc || sub > 0) ? 1u : 0u);
                mma_f16(acc, ah, bl, idesc, 1u);
                mma_f16(acc, al, bh, idesc, 1u);
            }
            mma_commit(&bars[st]);
        }
    }
    cp_async_wait<0>();                                  /* no copy outlives the tile */
    /* the last step's commit covers every MMA issued before it */
    if (ok) ok = mbar_wait(&bars[(nks - 1) & 1], ((nks - 1) >> 1) & 1);
    if (!ok) {
        if (tid == 0) atomicOr(a.err, WC_ERR_TMA_WAIT);
        /* let the tensor core drain before TMEM is released */
        mbar_wait(&bars[(nks - 1) & 1], ((nks - 1) >> 1) & 1);
    }
    asm volatile("tcgen05.fence::after_thread_sync;");
    if (ok) {
        /* warp w reads TMEM lanes 32*(w%4).. (its lane quarter) = weight rows,
         * columns (pairs) [64*(w/4), 64*(w/4) + 64) */
        const int quarter = warp % 4, chw = warp / 4;
        const int r = quarter * 32 + lane;
        const float rs = f16_keep(rscale[m0 + r]) / wsc;
        const int cend = min(n, chw * (kPfTok / 2) + kPfTok / 2);
        for (int c0 = chw * (kPfTok / 2); c0 < cend; c0 += 16) {
            float sum[16];
#pragma unroll
            for (int j = 0; j < 16; j++) sum[j] = 0.0f;
#pragma unroll
            for (int q = 0; q < kPfAcc; q++) {
                uint32_t v[16];
                const uint32_t ta = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(q * kPfTok + c0);
                asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 "
                             "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
                             : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]),
                               "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]), "=r"(v[9]),
                               "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]),
                               "=r"(v[15])
                             : "r"(ta));
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                if (q < nks) {                          /* accumulators never written stay out */
#pragma unroll
                    for (int j = 0; j < 16; j++) sum[j] += __uint_as_float(v[j]);
                }
            }
#pragma unroll
            for (int j = 0; j < 16; j++) {
                const int jj = c0 + j;
                if (jj >= n) break;
                const float val = (sum[j] * s_inv[jj]) * rs;
                if (!DOWN)
                    a.gu[((size_t)(s0 + jj) * 2 + kind) * bk.inter + m0 + r] = val;
                else
                    a.y[(size_t)s_pair[jj] * bk.lat + m0 + r] = val;
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;"
                     ::"r"(tmem), "r"(kPfAcc * kPfTok));
    (void)Mrows;
}

/* ---- 6. per token, experts in ascending id (src/model.c:3632-3656) -------- */
__global__ void __launch_bounds__(256) pf_combine(wc_pf_args a)
{
    __shared__ int ord[64];
    __shared__ float wj[64];
    const int t = blockIdx.y, K = a.K;
    if (threadIdx.x == 0) {
        /* insertion order by (id, slot): the reference's ascending scan */
        int n = 0;
        for (int j = 0; j < K; j++) {
            const int e = a.route[t * K + j];
            int q = n++;
            while (q > 0 && a.route[t * K + ord[q - 1]] > e) { ord[q] = ord[q - 1]; q--; }
            ord[q] = j;
        }
    }
    if (threadIdx.x < K) wj[threadIdx.x] = a.rw[t * K + threadIdx.x];
    __syncthreads();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= a.bank.lat) return;
    float y = 0.0f;
    for (int q = 0; q < K; q++) {
        const int j = ord[q];
        const int e = a.route[t * K + j] - a.bank.first;
        const float w = wj[j];
        if (w == 0.0f || e < 0 || e >= a.bank.n_experts) continue;
        y = __fadd_rn(y, __fmul_rn(w, a.y[((size_t)t * K + j) * a.bank.lat + i]));
    }
    a.out[(size_t)t * a.bank.lat + i] = y;
}

}  // namespace

extern "C" int wc_pf_supported(const wc_bank *b, int T, int K)
{
    if (b->stages != 3 || b->inter % kPfRows || b->lat % kPfRows) return -1;
    if (b->lat % kPfKs || b->inter % kPfKs || K > 64 || T <= 0 || T * K > WC_PF_MAX_PAIRS)
        return -1;
    if (b->n_experts > kPfMaxE) return -1;
    return 0;
}

extern "C" size_t wc_pf_max_tiles(int T, int K, int n_experts)
{
    return (size_t)(T * K + kPfTok - 1) / kPfTok + (size_t)n_experts;
}

extern "C" int wc_pf_launch(const wc_pf_args *a, void *stream)
{
    cudaStream_t s = (cudaStream_t)stream;
    const wc_bank &b = a->bank;
    const int np = a->T * a->K;
    const int max_tiles = (int)wc_pf_max_tiles(a->T, a->K, b.n_experts);
    pf_bucket<<<1, 1024, 0, s>>>(*a);
    pf_split_x<<<a->T, 256, 0, s>>>(*a);
    cudaFuncSetAttribute(pf_gemm<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, kPfSmem);
    cudaFuncSetAttribute(pf_gemm<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, kPfSmem);
    pf_gemm<0><<<dim3(max_tiles, 2 * b.inter / kPfRows), kPfThreads, kPfSmem, s>>>(*a);
    pf_split_h<<<np, 256, 0, s>>>(*a);
    pf_gemm<1><<<dim3(max_tiles, b.lat / kPfRows), kPfThreads, kPfSmem, s>>>(*a);
    pf_combine<<<dim3((b.lat + 255) / 256, a->T), 256, 0, s>>>(*a);
    wc_count_launches(6);
    return (int)cudaGetLastError();
}
