/*
 * trunk_mvq.cu — the engine's quantised trunk matvec on sm_100a: the
 * mvq_rows_f32 slot of the reference's dispatch table
 * (src/waste_backend.h:81; arithmetic src/model.c:265-320).
 *
 * y[o] = sum_k f16(ws[o][k]) * (sum_{i<g} w[o][k*g+i] * x[k*g+i]) for
 * Q8G (int8), Q4G (two signed nibbles per byte, low first, value - 8) and
 * Q3G (a 3-bit bitstream, value - 4) rows of `rowbytes` bytes, with one f16
 * scale per group of g weights (subnormal scales kept, src/simd.h:49-67).
 *
 * B200 mapping: HBM-bound GEMV (one byte or less per weight, read once).
 * Q8G/Q4G rows with 128-weight groups stream through shared memory by bulk
 * copy (mvq_tma_kernel); Q3G and other group sizes take a per-weight path
 * (mvq_kernel). x sits in shared memory, zero past `in`, so the padded tail
 * of the last group adds nothing. The sum order differs from the CPU's
 * serial one, within fp32 rounding.
 */
#include "vq3r_common.cuh"
#include "wc_launch.h"

#include <cuda_runtime.h>
#include <stdint.h>

using namespace wc;

namespace {

constexpr int kMvqThreads = 256;

/* Programmatic dependent launch (a no-op for a kernel launched without it):
 * the next kernel may start its prologue; and the wait for the previous
 * kernel's results. */
__device__ __forceinline__ void pdl_trigger_m() { asm volatile("griddepcontrol.launch_dependents;"); }
__device__ __forceinline__ void pdl_wait_m() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

template <typename... KArgs, typename... Args>
cudaError_t launch_m(void (*kern)(KArgs...), unsigned blocks, size_t smem, cudaStream_t s, bool pdl,
                     Args... args)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(blocks);
    cfg.blockDim = dim3(kMvqThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, args...);
}
constexpr int kMvqStages = 2;            /* bulk-copy ring depth of the tile kernel */

__device__ __forceinline__ float warp_sum_f(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

/* xs[0..n) = x[0..in), zero past in. Each thread issues up to kXBatch of
 * its loads before storing any, so the copy costs one memory round trip per
 * kXBatch * blockDim values instead of one per blockDim. */
constexpr int kXBatch = 16;

__device__ __forceinline__ void stage_x(float *xs, const float *__restrict__ x, int in, int n)
{
    for (int base = threadIdx.x; base < n; base += kXBatch * blockDim.x) {
        float v[kXBatch];
#pragma unroll
        for (int j = 0; j < kXBatch; j++) {
            const int i = base + j * blockDim.x;
            v[j] = i < in ? x[i] : 0.0f;
        }
#pragma unroll
        for (int j = 0; j < kXBatch; j++) {
            const int i = base + j * blockDim.x;
            if (i < n) xs[i] = v[j];
        }
    }
}

/* src/simd.h:69-74 waste_q3_at: signed 3-bit code i of a packed row. */
__device__ __forceinline__ int q3_at(const uint8_t *p, long i)
{
    const long off = i * 3;
    const int v = (p[off >> 3] >> (off & 7)) | (p[(off >> 3) + 1] << (8 - (off & 7)));
    return (v & 7) - 4;
}

/* Q3G, or a group size other than 128: warp per row, per-weight decode. */
template <int BITS>
__global__ void __launch_bounds__(kMvqThreads)
mvq_kernel(float *__restrict__ y, const uint8_t *__restrict__ W, const uint16_t *__restrict__ ws,
           const float *__restrict__ x, int r0, int r1, int in, int ng, int g, size_t rowbytes)
{
    extern __shared__ __align__(16) float xs[];
    const int n = ng * g;
    pdl_trigger_m();
    pdl_wait_m();                            /* x: the previous kernel's output */
    stage_x(xs, x, in, n);
    __syncthreads();
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int wpb = blockDim.x / 32;
    for (int o = r0 + blockIdx.x * wpb + warp; o < r1; o += gridDim.x * wpb) {
        const uint8_t *row = W + (size_t)o * rowbytes;
        const uint16_t *sr = ws + (size_t)o * ng;
        float acc = 0.0f;
        for (int k = 0; k < ng; k++) {
            float p = 0.0f;
            for (int i = lane; i < g; i += 32) {
                const long e = (long)k * g + i;
                int wv;
                if (BITS == 8) wv = (int8_t)row[e];
                else if (BITS == 4) {
                    const uint8_t b = row[e >> 1];
                    wv = (int)((e & 1) ? (b >> 4) : (b & 0x0f)) - 8;
                } else {
                    wv = q3_at(row, e);
                }
                p = fmaf((float)wv, xs[e], p);
            }
            acc = fmaf(f16_keep(__ldg(sr + k)), p, acc);
        }
        acc = warp_sum_f(acc);
        if (lane == 0) y[o] = acc;
    }
}

/* Q8G / Q4G rows of 128-weight groups: a persistent block streams tiles of
 * R consecutive rows (R * rowbytes contiguous bytes, and their scales)
 * into a kMvqStages-deep shared-memory ring with bulk copies (cp.async.bulk, no
 * registers held by bytes in flight), and computes one tile while the next ones
 * lands. A warp takes two rows of a tile at a time, a group per step (lane
 * l: weights [4l, 4l+4) of each row against one float4 of x), and
 * accumulates scale * partial per lane; one warp sum per row. Waits are
 * bounded: a tile whose copy never lands is written as NaN. */
struct MvqTile {
    int R;                 /* rows per tile; R * ng * 2 a multiple of 16      */
    uint32_t wbytes;       /* R * rowbytes, a multiple of 16                  */
    uint32_t sbytes;       /* R * ng * 2                                      */
};

template <int BITS>
__global__ void __launch_bounds__(kMvqThreads)
mvq_tma_kernel(float *__restrict__ y, const uint8_t *__restrict__ W,
               const uint16_t *__restrict__ ws, const float *__restrict__ x, int r0, int r1,
               int in, int ng, size_t rowbytes, MvqTile tl)
{
    extern __shared__ __align__(128) unsigned char sm[];
    uint64_t *bars = reinterpret_cast<uint64_t *>(sm);  /* [kMvqStages] */
    float *xs = reinterpret_cast<float *>(sm + 128);
    const int n = ng * 128;
    uint8_t *stage0 = sm + 128 + (((size_t)n * 4 + 127) & ~(size_t)127);
    const size_t sstride = ((size_t)tl.wbytes + tl.sbytes + 127) & ~(size_t)127;
    const int rows = r1 - r0;
    const int ntiles = (rows + tl.R - 1) / tl.R;
    /* tile i's rows and bytes (the last tile may be short: its copy is too) */
    /* the scales of a short last tile whose byte count is not a multiple
     * of 16 are copied up to the last 16-byte boundary and the rest read
     * from global memory (no copy reads past the tensor) */
    auto issue = [&](int i, int st) {
        const int t0 = r0 + i * tl.R, nr = min(tl.R, r1 - t0);
        const uint32_t wb = (uint32_t)nr * (uint32_t)rowbytes;
        const uint32_t sb = ((uint32_t)nr * ng * 2) & ~15u;
        uint8_t *dst = stage0 + st * sstride;
        mbar_expect_tx(&bars[st], wb + sb);
        bulk_g2s(dst, W + (size_t)t0 * rowbytes, wb, &bars[st]);
        if (sb) bulk_g2s(dst + tl.wbytes, ws + (size_t)t0 * ng, sb, &bars[st]);
    };
    if (threadIdx.x == 0) {
        for (int q = 0; q < kMvqStages; q++) mbar_init(&bars[q], 1);
        mbar_fence_init();
        for (int q = 0; q < kMvqStages; q++)
            if ((int)(blockIdx.x + q * gridDim.x) < ntiles) issue(blockIdx.x + q * gridDim.x, q);
    }
    pdl_trigger_m();
    pdl_wait_m();                            /* the weights are constants: only x waits */
    stage_x(xs, x, in, n);
    __syncthreads();
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    int it = 0;
    for (int i = blockIdx.x; i < ntiles; i += gridDim.x, it++) {
        const int st = it % kMvqStages;                         /* stage    */
        const uint32_t par = (uint32_t)(it / kMvqStages) & 1u;  /* its phase */
        const int t0 = r0 + i * tl.R, nr = min(tl.R, r1 - t0);
        const bool ok = mbar_wait(&bars[st], par);
        const uint8_t *wt = stage0 + st * sstride;
        const uint16_t *stl = reinterpret_cast<const uint16_t *>(wt + tl.wbytes);
        const int sstaged = (nr * ng * 2 & ~15) / 2;            /* scales staged */
        /* a warp takes two rows at a time; per group step, lane l reads
         * weights [4l, 4l+4) of the group of both rows (one 32-bit (Q8G) or
         * 16-bit (Q4G) word each) and the matching float4 of x once: every
         * shared-memory read of the step is conflict-free */
        for (int r2 = 2 * warp; r2 < nr; r2 += 2 * (kMvqThreads / 32)) {
            const bool two = r2 + 1 < nr;
            const uint8_t *rowa = wt + (size_t)r2 * rowbytes;
            const uint8_t *rowb = rowa + (two ? rowbytes : 0);
            float acca = 0.0f, accb = 0.0f;
            for (int k = 0; k < ng; k++) {
                const float4 xv = *reinterpret_cast<const float4 *>(xs + k * 128 + 4 * lane);
                float pa, pb;
                float4 fa, fb;
                if (BITS == 8) {
                    fa = s8x4_to_f32(*reinterpret_cast<const uint32_t *>(rowa + k * 128 + 4 * lane));
                    fb = s8x4_to_f32(*reinterpret_cast<const uint32_t *>(rowb + k * 128 + 4 * lane));
                } else {
                    fa = u4x4_to_f32(*reinterpret_cast<const uint16_t *>(rowa + k * 64 + 2 * lane));
                    fb = u4x4_to_f32(*reinterpret_cast<const uint16_t *>(rowb + k * 64 + 2 * lane));
                }
                pa = fa.x * xv.x;
                pa = fmaf(fa.y, xv.y, pa);
                pa = fmaf(fa.z, xv.z, pa);
                pa = fmaf(fa.w, xv.w, pa);
                pb = fb.x * xv.x;
                pb = fmaf(fb.y, xv.y, pb);
                pb = fmaf(fb.z, xv.z, pb);
                pb = fmaf(fb.w, xv.w, pb);
                const int qa = r2 * ng + k, qb = qa + ng;
                const uint16_t sa = qa < sstaged ? stl[qa] : __ldg(ws + (size_t)t0 * ng + qa);
                const uint16_t sb = !two ? (uint16_t)0
                                  : (qb < sstaged ? stl[qb] : __ldg(ws + (size_t)t0 * ng + qb));
                acca = fmaf(f16_keep(sa), pa, acca);
                accb = fmaf(f16_keep(sb), pb, accb);
            }
            acca = warp_sum_f(acca);
            accb = warp_sum_f(accb);
            if (lane == 0) {
                y[t0 + r2] = ok ? acca : __int_as_float(0x7fc00000);
                if (two) y[t0 + r2 + 1] = ok ? accb : __int_as_float(0x7fc00000);
            }
        }
        __syncthreads();                     /* every warp is done with this stage */
        if (threadIdx.x == 0 && i + kMvqStages * (int)gridDim.x < ntiles)
            issue(i + kMvqStages * gridDim.x, st);
    }
}

template <int BITS>
int mvq_go(const wc_mvq_args *a, cudaStream_t s)
{
    const size_t smem = (size_t)a->ng * a->group * sizeof(float);
    const auto k = mvq_kernel<BITS>;
    if (smem > 48 * 1024 &&
        cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return (int)cudaErrorInvalidValue;
    const int rows = a->r1 - a->r0;
    const int wpb = kMvqThreads / 32;
    int blocks = (rows + wpb - 1) / wpb;
    const int cap = 148 * 8;                 /* 8 resident blocks per SM */
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    const cudaError_t e = launch_m(k, (unsigned)blocks, smem, s, a->pdl != 0, a->y, a->W, a->ws,
                                   a->x, a->r0, a->r1, a->in, a->ng, a->group, a->rowbytes);
    wc_count_launches(1);
    return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

template <int BITS>
int mvq_tma_go(const wc_mvq_args *a, cudaStream_t s)
{
    /* tiles of up to 16 rows and about 40 KB, kMvqStages stages, two blocks
     * per SM; every tile's scales must start on a 16-byte boundary */
    MvqTile tl;
    tl.R = 0;
    for (int R = 16; R >= 1; R--)
        if ((size_t)R * a->rowbytes <= (40u << 10) && ((size_t)R * a->ng * 2) % 16 == 0) {
            tl.R = R;
            break;
        }
    if (tl.R == 0 || ((size_t)a->r0 * a->ng * 2) % 16) return mvq_go<BITS>(a, s);
    tl.wbytes = (uint32_t)(tl.R * a->rowbytes);
    tl.sbytes = (uint32_t)tl.R * a->ng * 2;
    const size_t sstride = ((size_t)tl.wbytes + tl.sbytes + 127) & ~(size_t)127;
    const size_t smem = 128 + (((size_t)a->ng * 128 * 4 + 127) & ~(size_t)127) +
                        kMvqStages * sstride;
    if (smem > 220 * 1024) return mvq_go<BITS>(a, s);
    const auto k = mvq_tma_kernel<BITS>;
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return (int)cudaErrorInvalidValue;
    const int ntiles = (a->r1 - a->r0 + tl.R - 1) / tl.R;
    int blocks = 148 * 2;
    if (blocks > ntiles) blocks = ntiles;
    const cudaError_t e = launch_m(k, (unsigned)blocks, smem, s, a->pdl != 0, a->y, a->W, a->ws,
                                   a->x, a->r0, a->r1, a->in, a->ng, a->rowbytes, tl);
    wc_count_launches(1);
    return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

} /* namespace */

extern "C" int wc_mvq_launch(const wc_mvq_args *a, void *stream)
{
    cudaStream_t s = (cudaStream_t)stream;
    if ((size_t)a->ng * a->group * sizeof(float) > 200 * 1024) return (int)cudaErrorInvalidValue;
    /* the bulk-copy form: 128-weight groups, rows a multiple of 16 bytes,
     * 16-byte aligned tensors */
    const bool tma = a->group == 128 &&
                     ((a->bits == 8 && a->rowbytes == (size_t)a->ng * 128) ||
                      (a->bits == 4 && a->rowbytes == (size_t)a->ng * 64)) &&
                     ((uintptr_t)a->W & 15) == 0 && ((uintptr_t)a->ws & 15) == 0;
    switch (a->bits) {
    case 8: return tma ? mvq_tma_go<8>(a, s) : mvq_go<8>(a, s);
    case 4: return tma ? mvq_tma_go<4>(a, s) : mvq_go<4>(a, s);
    case 3: return mvq_go<3>(a, s);
    default: return (int)cudaErrorInvalidValue;
    }
}
