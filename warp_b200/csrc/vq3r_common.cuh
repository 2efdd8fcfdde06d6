/*
 * vq3r_common.cuh — device helpers shared by the VQ3R kernels (sm_100a).
 *
 * Index layout (the reference's blocked layout, docs/FORMAT.md:194-208,
 * tools/convert.py:297-312): [M/64][N/8][64][stages] bytes, one byte per
 * stage. For a fixed (row block, vector position) the 64 rows' indices are
 * 64*stages contiguous bytes, so a quarter of a block (16 rows) is exactly
 * `stages` 16-byte words — one LDG.128 per stage.
 */
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace wc {

constexpr int kVecDim = 8;      /* docs/FORMAT.md expert_quant.vec_dim */
constexpr int kEntries = 256;   /* entries per stage codebook          */
constexpr int kBlock = 64;      /* index_block == VQ_TILE              */
constexpr int kRowsPerThread = 16;

/* f16 -> f32 exactly as src/simd.h:49-67 (subnormals kept, exponent 31 not
 * special-cased). Used for row scales and Q8G group scales. */
__device__ __forceinline__ float f16_keep(uint16_t h)
{
    const uint32_t sign = (uint32_t)(h >> 15) << 31;
    const uint32_t e = (h >> 10) & 0x1f, mn = h & 0x3ff;
    if (e == 0) {
        const float f = (float)mn * 5.9604644775390625e-08f;
        return sign ? -f : f;
    }
    return __uint_as_float(sign | ((e + 112u) << 23) | (mn << 13));
}

/* The four signed bytes of w (byte 0 first) as exact floats, without
 * integer-to-float conversions, whose issue rate is a small fraction of the
 * FMA pipe's: each byte, offset by 128, becomes the low mantissa bits of
 * 2^23 (a byte permute), and 2^23 + 128 is subtracted in float — exact, so
 * the values are those of (float)(int8_t)byte. */
__device__ __forceinline__ float4 s8x4_to_f32(uint32_t w)
{
    const uint32_t u = w ^ 0x80808080u;
    const float bias = 8388736.0f;                       /* 2^23 + 128 */
    return make_float4(__int_as_float(__byte_perm(u, 0x4B000000u, 0x7440)) - bias,
                       __int_as_float(__byte_perm(u, 0x4B000000u, 0x7441)) - bias,
                       __int_as_float(__byte_perm(u, 0x4B000000u, 0x7442)) - bias,
                       __int_as_float(__byte_perm(u, 0x4B000000u, 0x7443)) - bias);
}

/* The four 4-bit codes of the low 16 bits of w (low nibble first) minus 8,
 * as exact floats, the same way (2^23 + code - (2^23 + 8)). */
__device__ __forceinline__ float4 u4x4_to_f32(uint32_t w)
{
    const float bias = 8388616.0f;                       /* 2^23 + 8 */
    return make_float4(__int_as_float(0x4B000000u | (w & 0xfu)) - bias,
                       __int_as_float(0x4B000000u | ((w >> 4) & 0xfu)) - bias,
                       __int_as_float(0x4B000000u | ((w >> 8) & 0xfu)) - bias,
                       __int_as_float(0x4B000000u | ((w >> 12) & 0xfu)) - bias);
}

/* Byte `p` (compile-time) of a little-endian run of 32-bit words. */
template <int P>
__device__ __forceinline__ uint32_t byte_at(const uint32_t *w)
{
    return (w[P >> 2] >> (8 * (P & 3))) & 0xffu;
}

/* 16-byte global load through the read-only path. */
__device__ __forceinline__ uint4 ldg16(const void *p)
{
    return __ldg(reinterpret_cast<const uint4 *>(p));
}

/* Loads that must be ISSUED where they are written: a prefetch into
 * registers ahead of a barrier or a grid-dependency wait. A read-only (.nc)
 * load may legally be sunk to its first use or issued again there, which
 * turns the prefetch into a stall; a volatile coherent load is neither. */
__device__ __forceinline__ uint4 ld_pin16(const void *p)
{
    uint4 v;
    asm volatile("ld.global.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}

__device__ __forceinline__ float4 ld_pin_f4(const void *p)
{
    float4 v;
    asm volatile("ld.global.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "l"(p));
    return v;
}

__device__ __forceinline__ uint16_t ld_pin_u16(const void *p)
{
    unsigned short v;
    asm volatile("ld.global.u16 %0, [%1];" : "=h"(v) : "l"(p));
    return v;
}

/* Streaming 16-byte load for data read once: an L2 evict-first policy, so
 * a long index stream does not push out what the kernel wrote (partial
 * sums that a reduction reads back). */
__device__ __forceinline__ uint64_t l2_evict_first()
{
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

__device__ __forceinline__ uint4 ld_stream16(const void *ptr, uint64_t pol)
{
    uint4 v;
    asm("ld.global.nc.L2::cache_hint.v4.u32 {%0, %1, %2, %3}, [%4], %5;"
        : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(ptr), "l"(pol));
    return v;
}

__device__ __forceinline__ float ld_pin_f32(const void *p)
{
    float v;
    asm volatile("ld.global.f32 %0, [%1];" : "=f"(v) : "l"(p));
    return v;
}

/* Builds the table slice for vector positions [v0, v0+nvs) of one matrix
 * family into shared memory:
 *   lut[(v - v0)*ST*256 + s*256 + c] = fma chain over d of x[8v+d]*C[cb+s][c][d]
 * from 0, d ascending — bit-identical to src/simd_avx512.c:104-112.
 * xs: nvs*8 floats already in shared memory, 16-byte aligned (read as
 * float4 broadcasts). books: [n_books][256][8]. */
template <int ST>
__device__ __forceinline__ void build_lut_slice(float *lut, const float *xs,
                                                const float *__restrict__ books,
                                                int cb, int nvs)
{
    for (int i = threadIdx.x; i < ST * kEntries; i += blockDim.x) {
        const int s = i / kEntries, c = i % kEntries;
        const float4 *src = reinterpret_cast<const float4 *>(
            books + ((size_t)(cb + s) * kEntries + c) * kVecDim);
        const float4 a = __ldg(src), b = __ldg(src + 1);
        for (int v = 0; v < nvs; v++) {
            const float4 x0 = *reinterpret_cast<const float4 *>(xs + v * kVecDim);
            const float4 x1 = *reinterpret_cast<const float4 *>(xs + v * kVecDim + 4);
            float acc = 0.0f;
            acc = __fmaf_rn(x0.x, a.x, acc); acc = __fmaf_rn(x0.y, a.y, acc);
            acc = __fmaf_rn(x0.z, a.z, acc); acc = __fmaf_rn(x0.w, a.w, acc);
            acc = __fmaf_rn(x1.x, b.x, acc); acc = __fmaf_rn(x1.y, b.y, acc);
            acc = __fmaf_rn(x1.z, b.z, acc); acc = __fmaf_rn(x1.w, b.w, acc);
            lut[(v * ST + s) * kEntries + c] = acc;
        }
    }
}

/* One vector position for 16 rows: add sum_s L_s[idx] to acc[k]. The 16*ST
 * index bytes of this quarter-block are in w[0 .. 4*ST). */
template <int ST, int K>
struct RowStep {
    static __device__ __forceinline__ void run(float *acc, const uint32_t *w,
                                               const float *L)
    {
        float t = L[byte_at<K * ST>(w)];
        if (ST > 1) t += L[kEntries + byte_at<K * ST + (ST > 1 ? 1 : 0)>(w)];
        if (ST > 2) t += L[2 * kEntries + byte_at<K * ST + (ST > 2 ? 2 : 0)>(w)];
        acc[K] += t;
        RowStep<ST, K + 1>::run(acc, w, L);
    }
};
template <int ST>
struct RowStep<ST, kRowsPerThread> {
    static __device__ __forceinline__ void run(float *, const uint32_t *, const float *) {}
};

/* Streams the index words of one quarter-block (16 rows) over nvv
 * consecutive vector positions and adds their lookups into acc[16].
 * begin() issues the loads of the first two positions, so a kernel can call
 * it before building its table and have the DRAM latency overlap the build;
 * run() keeps two positions in flight ahead of the arithmetic. Positions are
 * 64*ST bytes apart; L is the table at the first position. */
template <int ST>
struct Gather16 {
    static constexpr int W = 4 * ST;       /* 32-bit words per position */
    uint32_t b0[W], b1[W];
    const uint8_t *p;
    int n;

    __device__ __forceinline__ void load(uint32_t *dst, const uint8_t *src) const
    {
        const uint64_t pol = l2_evict_first();   /* one instruction; not kept live */
#pragma unroll
        for (int i = 0; i < ST; i++) {
            const uint4 q = ld_stream16(src + 16 * i, pol);
            dst[4 * i] = q.x; dst[4 * i + 1] = q.y; dst[4 * i + 2] = q.z; dst[4 * i + 3] = q.w;
        }
    }

    __device__ __forceinline__ void begin(const uint8_t *p0, int nvv)
    {
        p = p0;
        n = nvv;
        if (n > 0) load(b0, p);
        if (n > 1) load(b1, p + (size_t)kBlock * ST);
    }

    __device__ __forceinline__ void run(float *acc, const float *L)
    {
        const size_t stride = (size_t)kBlock * ST;
        int v = 0;
#pragma unroll 1
        for (; v + 1 < n; v += 2) {
            RowStep<ST, 0>::run(acc, b0, L + (size_t)v * ST * kEntries);
            if (v + 2 < n) load(b0, p + (size_t)(v + 2) * stride);
            RowStep<ST, 0>::run(acc, b1, L + (size_t)(v + 1) * ST * kEntries);
            if (v + 3 < n) load(b1, p + (size_t)(v + 3) * stride);
        }
        if (v < n) RowStep<ST, 0>::run(acc, b0, L + (size_t)v * ST * kEntries);
    }
};

/* Codebook rows for the table build, loaded ahead of time: entry i of the
 * thread's share (i = threadIdx.x + k*blockDim.x, k < NE) of the ST*256
 * (stage, code) pairs of book group cb. */
template <int ST, int NE>
struct BookRows {
    float4 c[NE][2];
    bool all;                 /* the block's NE rows per thread cover every entry */
    const float *src_books;
    int src_cb;

    __device__ __forceinline__ void load(const float *__restrict__ books, int cb)
    {
        all = (int)blockDim.x * NE >= ST * kEntries;
        src_books = books;
        src_cb = cb;
        if (!all) return;     /* small blocks build from global memory instead */
#pragma unroll
        for (int k = 0; k < NE; k++) {
            const int i = threadIdx.x + k * blockDim.x;
            if (i < ST * kEntries) {
                const int s = i / kEntries, code = i % kEntries;
                const float4 *src = reinterpret_cast<const float4 *>(
                    books + ((size_t)(cb + s) * kEntries + code) * kVecDim);
                c[k][0] = ld_pin_f4(src);
                c[k][1] = ld_pin_f4(src + 1);
            }
        }
    }

    /* lut[(v*ST + s)*256 + code] = FMA chain over d from 0, d ascending —
     * the same arithmetic as build_lut_slice, from the prefetched rows.
     * xs 16-byte aligned. */
    __device__ __forceinline__ void build(float *lut, const float *xs, int nvs) const
    {
        if (!all) {
            build_lut_slice<ST>(lut, xs, src_books, src_cb, nvs);
            return;
        }
#pragma unroll
        for (int k = 0; k < NE; k++) {
            const int i = threadIdx.x + k * blockDim.x;
            if (i >= ST * kEntries) continue;
            const int s = i / kEntries, code = i % kEntries;
            const float4 a = c[k][0], b = c[k][1];
            for (int v = 0; v < nvs; v++) {
                const float4 x0 = *reinterpret_cast<const float4 *>(xs + v * kVecDim);
                const float4 x1 = *reinterpret_cast<const float4 *>(xs + v * kVecDim + 4);
                float acc = 0.0f;
                acc = __fmaf_rn(x0.x, a.x, acc); acc = __fmaf_rn(x0.y, a.y, acc);
                acc = __fmaf_rn(x0.z, a.z, acc); acc = __fmaf_rn(x0.w, a.w, acc);
                acc = __fmaf_rn(x1.x, b.x, acc); acc = __fmaf_rn(x1.y, b.y, acc);
                acc = __fmaf_rn(x1.z, b.z, acc); acc = __fmaf_rn(x1.w, b.w, acc);
                lut[(v * ST + s) * kEntries + code] = acc;
            }
        }
    }
};

/* ---- TMA bulk copies into shared memory ----------------------------------
 * cp.async.bulk (the untiled TMA form) moves a contiguous run of global
 * memory into this CTA's shared memory and signals an mbarrier with the byte
 * count; both addresses 16-byte aligned, the size a multiple of 16. The
 * copy is issued where it is written and holds no registers, which is what
 * a prefetch ahead of a grid-dependency wait needs. No multicast. */
__device__ __forceinline__ uint32_t smem_u32(const void *p)
{
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

/* Make the initialised barrier visible to the async (TMA) proxy. */
__device__ __forceinline__ void mbar_fence_init()
{
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;"
                 ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar)
{
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}

/* Tiled TMA load of a 3-D box at {x, y, z} (x in elements of the map,
 * x * element size a multiple of 16 bytes) into shared memory (128-byte
 * aligned), signalling `bar` with the box's bytes. The map is a kernel
 * parameter (__grid_constant__). No multicast. */
__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, int x, int y, int z,
                                            uint64_t *bar)
{
    asm volatile("cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
                 " [%0], [%1, {%2, %3, %4}], [%5];"
                 ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z),
                   "r"(smem_u32(bar)) : "memory");
}

/* Bounded wait for phase `parity` of the barrier: false after kMbarLimit
 * polls (each try_wait also suspends for a while), so a copy that never
 * lands ends the wait instead of the kernel. */
constexpr int kMbarLimit = 1 << 22;

__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity)
{
    for (int i = 0; i < kMbarLimit; i++) {
        uint32_t done;
        asm volatile("{\n\t.reg .pred p;\n\t"
                     "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                     "selp.u32 %0, 1, 0, p;\n\t}"
                     : "=r"(done) : "r"(smem_u32(bar)), "r"(parity) : "memory");
        if (done) return true;
    }
    return false;
}

/* The index stream of one quarter-block staged in shared memory:
 * base points at the quarter's 16*ST bytes of its first position,
 * consecutive positions `pstride` bytes apart. */
template <int ST>
__device__ __forceinline__ void gather_smem(float *acc, const uint8_t *base, int pstride,
                                            const float *L, int nvv)
{
    constexpr int W = 4 * ST;
    for (int v = 0; v < nvv; v++) {
        uint32_t w[W];
        const uint4 *src = reinterpret_cast<const uint4 *>(base + (size_t)v * pstride);
#pragma unroll
        for (int i = 0; i < ST; i++) {
            const uint4 q = src[i];
            w[4 * i] = q.x; w[4 * i + 1] = q.y; w[4 * i + 2] = q.z; w[4 * i + 3] = q.w;
        }
        RowStep<ST, 0>::run(acc, w, L + (size_t)v * ST * kEntries);
    }
}

/* Gather policy for index streams staged in shared memory by TMA (layout
 * [row block][position][64][ST], i.e. positions 64*ST bytes apart). The
 * positions before `split` land on bar0, the rest on bar1 (bar1 may be
 * null when there is one phase); each wait is bounded and a failure is
 * reported through `ok`. */
template <int ST>
struct GatherSmem {
    const uint8_t *p;
    int n, first;             /* positions [first, first+n) of the slice */
    uint64_t *bar0, *bar1;
    int split;
    uint32_t par;             /* barrier phase parity of this staging round */
    bool ok;

    __device__ __forceinline__ void begin(const uint8_t *p0, int nvv)
    {
        p = p0;
        n = nvv;
        par = 0;
        ok = true;
    }

    __device__ __forceinline__ void run(float *acc, const float *L)
    {
        const int stride = kBlock * ST;
        if (bar1 == nullptr) {
            ok = mbar_wait(bar0, par);
            if (ok) gather_smem<ST>(acc, p, stride, L, n);
            return;
        }
        const int n0 = max(0, min(n, split - first));
        if (n0 > 0) {
            ok = mbar_wait(bar0, par);
            if (!ok) return;
            gather_smem<ST>(acc, p, stride, L, n0);
        }
        if (n0 < n) {
            ok = mbar_wait(bar1, par);
            if (!ok) return;
            gather_smem<ST>(acc, p + (size_t)n0 * stride, stride, L + (size_t)n0 * ST * kEntries,
                            n - n0);
        }
    }
};

__device__ __forceinline__ float silu_ref(float v)
{
    /* src/model.c:501: v / (1 + expf(-v)). */
    return v / (1.0f + expf(-v));
}

/* src/model.c:505-509 waste_situ_pair, K3's SiTU: beta*tanh(g/beta)*sigmoid(g)
 * times lbeta*tanh(u/lbeta) (u itself when lbeta <= 0). */
__device__ __forceinline__ float situ_ref(float g, float u, float beta, float lbeta)
{
    const float a = beta * tanhf(g / beta) / (1.0f + expf(-g));
    return a * (lbeta > 0.0f ? lbeta * tanhf(u / lbeta) : u);
}

/* exp(x) rounded once to float, for the VQ4P expert loop (whose int8
 * re-quantisation of the down table turns a one-ulp difference in an
 * activation into a whole table step, about 1e-4 relative on a layer) and
 * for KDA. Method: Cody and Waite's reduction x = k*ln2 + r with
 * k = rint(x/ln2) (two fused multiply-adds against ln2 split into a double
 * and its remainder), exp(r) by its Taylor series to r^13 in double
 * (|r| <= 0.347, truncation below 1e-17), scaled by 2^k and converted to
 * float in one rounding. The result is the correctly rounded exp(x) except
 * within about 1e-16 relative of a rounding midpoint; glibc's expf (within
 * 0.502 ulp) returns the same float for all but a few inputs in 10^4. */
__host__ __device__ __forceinline__ float expf_cr(float x)
{
    if (x != x) return x;
    if (x < -104.0f) return 0.0f;                        /* below half the least subnormal */
    if (x > 89.0f) return (float)(1e300 * 1e300);        /* above FLT_MAX: +inf */
    const double xd = (double)x;
    const double k = rint(xd * 1.4426950408889634);
    double r = fma(-k, 0.6931471805599453, xd);
    r = fma(-k, 2.3190468138462996e-17, r);
    double p = 1.0 / 6227020800.0;                       /* 1/13! */
    p = fma(p, r, 1.0 / 479001600.0);
    p = fma(p, r, 1.0 / 39916800.0);
    p = fma(p, r, 1.0 / 3628800.0);
    p = fma(p, r, 1.0 / 362880.0);
    p = fma(p, r, 1.0 / 40320.0);
    p = fma(p, r, 1.0 / 5040.0);
    p = fma(p, r, 1.0 / 720.0);
    p = fma(p, r, 1.0 / 120.0);
    p = fma(p, r, 1.0 / 24.0);
    p = fma(p, r, 1.0 / 6.0);
    p = fma(p, r, 0.5);
    p = fma(p, r, 1.0);
    p = fma(p, r, 1.0);
    return (float)scalbn(p, (int)k);
}

/* tanh(x) rounded once to float: CUDA's double tanh (an error of a few
 * double ulps) converted in one rounding, so correctly rounded except
 * within about 1e-15 relative of a rounding midpoint. */
__device__ __forceinline__ float tanhf_cr(float x)
{
    return (float)tanh((double)x);
}

/* The activations of the VQ4P loop with those functions: SiLU as
 * src/model.c:501 (v / (1 + expf(-v)), IEEE division), SiTU as :505-509. */
__device__ __forceinline__ float act_pair_cr(int act, float g, float u, float beta, float lbeta)
{
    const float sg = __fadd_rn(1.0f, expf_cr(-g));
    if (!act) return __fmul_rn(__fdiv_rn(g, sg), u);
    const float a = __fdiv_rn(__fmul_rn(beta, tanhf_cr(__fdiv_rn(g, beta))), sg);
    return __fmul_rn(a, lbeta > 0.0f ? __fmul_rn(lbeta, tanhf_cr(__fdiv_rn(u, lbeta))) : u);
}

/* The gated activation of a layer: SiLU(g)*u (act 0) or SiTU (act 1). */
__device__ __forceinline__ float act_pair(int act, float g, float u, float beta, float lbeta)
{
    return act ? situ_ref(g, u, beta, lbeta) : silu_ref(g) * u;
}

} /* namespace wc */
