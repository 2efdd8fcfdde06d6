/*
 * vq_encode.cu — the residual-VQ encoder of the container converter on
 * sm_100a: waste_vq_encode and waste_vq_lloyd (src/vq.c:50-136), which
 * tools/convert.py calls through ctypes to quantise every expert matrix.
 *
 *   encode  per vector, per stage: the entry nearest under squared
 *           Euclidean distance (sum over d of (v_d - C_d)^2 in d order, a
 *           rounded multiply then a rounded add; the first index wins ties,
 *           NaN never wins), its index written, the entry subtracted
 *   lloyd   one Lloyd iteration: assign (one stage), then every non-empty
 *           cluster's centroid = (float)(sum in double of its members, in
 *           vector order / count); empty clusters keep their centroid
 *
 * B200 mapping. Encoding is arithmetic (stages x entries x dim x 3 flops a
 * vector) on a codebook that every vector reads: all stages' books sit in
 * shared memory, one thread per vector walks the entries in order, and a
 * warp's 32 lanes read the same entry at the same time (a broadcast). The
 * distances never leave registers and only the winning byte is written.
 * The Lloyd update keeps the reference's summation order exactly (a double
 * sum is not associative): a stable counting sort by cluster (per-block
 * counts, a scan, then one warp per block placing its members in vector
 * order with match-any ranks) gathers the vectors cluster by cluster, and
 * one thread per (cluster, dimension) adds its column serially.
 */
#include "vq3r_common.cuh"
#include "wc_launch.h"

#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

namespace {

constexpr int kEncThreads = 256;
constexpr int kLloydBlock = 4096;       /* vectors a block counts and places */

/* The nearest entry of C (entries x DIM) to cur, and cur minus it. */
template <int DIM>
__device__ __forceinline__ int vq_step(float *cur, const float *C, int entries, int dim)
{
    const int D = DIM > 0 ? DIM : dim;
    int best = 0;
    float bestd = __int_as_float(0x7f800000);
    for (int c = 0; c < entries; c++) {
        const float *e = C + (size_t)c * D;
        float d = 0.0f;
#pragma unroll
        for (int j = 0; j < (DIM > 0 ? DIM : 64); j++) {
            if (DIM == 0 && j >= D) break;
            const float t = __fsub_rn(cur[j], e[j]);
            d = __fadd_rn(d, __fmul_rn(t, t));
        }
        if (d < bestd) {
            bestd = d;
            best = c;
        }
    }
    const float *e = C + (size_t)best * D;
#pragma unroll
    for (int j = 0; j < (DIM > 0 ? DIM : 64); j++) {
        if (DIM == 0 && j >= D) break;
        cur[j] = __fsub_rn(cur[j], e[j]);
    }
    return best;
}

/* One thread per vector; every stage's book in shared memory. */
template <int DIM>
__global__ void __launch_bounds__(kEncThreads) vq_encode_kernel(const float *__restrict__ X, int n,
                                                                const float *__restrict__ books,
                                                                int stages, int entries, int dim,
                                                                uint8_t *__restrict__ out)
{
    extern __shared__ float sb[];
    const int D = DIM > 0 ? DIM : dim;
    const int nb = stages * entries * D;
    for (int i = threadIdx.x; i < nb; i += blockDim.x) sb[i] = books[i];
    __syncthreads();
    const size_t v = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (v >= (size_t)n) return;
    float cur[DIM > 0 ? DIM : 64];
#pragma unroll
    for (int j = 0; j < (DIM > 0 ? DIM : 64); j++) {
        if (DIM == 0 && j >= D) break;
        cur[j] = X[v * D + j];
    }
    for (int s = 0; s < stages; s++)
        out[v * stages + s] = (uint8_t)vq_step<DIM>(cur, sb + (size_t)s * entries * D, entries, D);
}

/* Per block of kLloydBlock vectors: how many fall in each cluster. */
__global__ void __launch_bounds__(256) lloyd_count_kernel(const uint8_t *asg, int n, int entries,
                                                          int *bc)
{
    __shared__ int cnt[256];
    for (int c = threadIdx.x; c < entries; c += blockDim.x) cnt[c] = 0;
    __syncthreads();
    const size_t i0 = (size_t)blockIdx.x * kLloydBlock;
    for (int k = threadIdx.x; k < kLloydBlock; k += blockDim.x)
        if (i0 + k < (size_t)n) atomicAdd(&cnt[asg[i0 + k]], 1);
    __syncthreads();
    for (int c = threadIdx.x; c < entries; c += blockDim.x)
        bc[(size_t)blockIdx.x * entries + c] = cnt[c];
}

/* One block: per cluster, the offset of each block's members (over blocks)
 * and the count; then each cluster's start (over clusters). */
__global__ void __launch_bounds__(256) lloyd_scan_kernel(const int *bc, int nblk, int entries,
                                                         int *off, int *cnt, int *start)
{
    const int c = threadIdx.x;
    if (c < entries) {
        int run = 0;
        for (int b = 0; b < nblk; b++) {
            off[(size_t)b * entries + c] = run;
            run += bc[(size_t)b * entries + c];
        }
        cnt[c] = run;
    }
    __syncthreads();
    if (c == 0) {
        int run = 0;
        for (int k = 0; k < entries; k++) {
            start[k] = run;
            run += cnt[k];
        }
    }
}

/* One warp per block: its vectors placed in vector order within each
 * cluster (lanes of the same cluster ranked by lane, then the running count
 * of earlier steps), copied into Xs at their sorted position. */
__global__ void __launch_bounds__(32) lloyd_place_kernel(const float *X, const uint8_t *asg, int n,
                                                         int entries, int dim, const int *off,
                                                         const int *start, float *Xs)
{
    __shared__ int run[256];
    const int lane = threadIdx.x;
    for (int c = lane; c < entries; c += 32) run[c] = 0;
    __syncwarp();
    const size_t i0 = (size_t)blockIdx.x * kLloydBlock;
    for (int k = 0; k < kLloydBlock; k += 32) {
        const size_t i = i0 + k + lane;
        const bool ok = i < (size_t)n;
        const unsigned act = __ballot_sync(0xffffffffu, ok);
        if (!act) break;
        const int a = ok ? asg[i] : -1;
        const unsigned peers = __match_any_sync(0xffffffffu, a);
        if (ok) {
            const int rank = __popc(peers & ((1u << lane) - 1u));
            const size_t pos = (size_t)start[a] + off[(size_t)blockIdx.x * entries + a] + run[a] +
                               rank;
            for (int d = 0; d < dim; d++) Xs[pos * dim + d] = X[i * dim + d];
        }
        __syncwarp();
        if (ok && (peers & ((1u << lane) - 1u)) == 0) run[a] += __popc(peers);
        __syncwarp();
    }
}

/* One thread per (cluster, dimension): the column's double sum in vector
 * order, then the centroid (src/vq.c:124-132); counts the live clusters. */
__global__ void __launch_bounds__(256) lloyd_mean_kernel(const float *Xs, const int *cnt,
                                                         const int *start, int entries, int dim,
                                                         float *C, int *live)
{
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= entries * dim) return;
    const int c = t / dim, d = t % dim;
    const int m = cnt[c];
    if (m == 0) return;
    const float *p = Xs + (size_t)start[c] * dim + d;
    double s = 0.0;
    int j = 0;
    for (; j + 4 <= m; j += 4) {
        const float a0 = p[(size_t)j * dim], a1 = p[(size_t)(j + 1) * dim];
        const float a2 = p[(size_t)(j + 2) * dim], a3 = p[(size_t)(j + 3) * dim];
        s = __dadd_rn(s, (double)a0);
        s = __dadd_rn(s, (double)a1);
        s = __dadd_rn(s, (double)a2);
        s = __dadd_rn(s, (double)a3);
    }
    for (; j < m; j++) s = __dadd_rn(s, (double)p[(size_t)j * dim]);
    C[(size_t)c * dim + d] = (float)__ddiv_rn(s, (double)m);
    if (d == 0) atomicAdd(live, 1);
}

} /* namespace */

extern "C" {

size_t wc_vq_encode_smem(int stages, int entries, int dim)
{
    return (size_t)stages * entries * dim * sizeof(float);
}

int wc_vq_encode_launch(const float *X, int n, const float *books, int stages, int entries,
                        int dim, uint8_t *out, void *stream)
{
    const size_t smem = wc_vq_encode_smem(stages, entries, dim);
    const unsigned grid = (unsigned)(((size_t)n + kEncThreads - 1) / kEncThreads);
    cudaError_t e;
    if (dim == 8) {
        e = cudaFuncSetAttribute(vq_encode_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)smem);
        if (e != cudaSuccess) return (int)e;
        vq_encode_kernel<8><<<grid, kEncThreads, smem, (cudaStream_t)stream>>>(
            X, n, books, stages, entries, dim, out);
    } else {
        e = cudaFuncSetAttribute(vq_encode_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)smem);
        if (e != cudaSuccess) return (int)e;
        vq_encode_kernel<0><<<grid, kEncThreads, smem, (cudaStream_t)stream>>>(
            X, n, books, stages, entries, dim, out);
    }
    wc_count_launches(1);
    return (int)cudaGetLastError();
}

size_t wc_vq_lloyd_scratch(int n, int entries, int dim)
{
    const size_t nblk = ((size_t)n + kLloydBlock - 1) / kLloydBlock;
    const auto al = [](size_t b) { return (b + 255) & ~(size_t)255; };
    return al((size_t)n) + 2 * al(nblk * entries * sizeof(int)) + 2 * al(entries * sizeof(int)) +
           al(sizeof(int)) + al((size_t)n * dim * sizeof(float));
}

int wc_vq_lloyd_launch(const float *X, int n, float *C, int entries, int dim, void *scratch,
                       int *d_live, void *stream)
{
    cudaStream_t st = (cudaStream_t)stream;
    const int nblk = (int)(((size_t)n + kLloydBlock - 1) / kLloydBlock);
    const auto al = [](size_t b) { return (b + 255) & ~(size_t)255; };
    char *p = (char *)scratch;
    uint8_t *asg = (uint8_t *)p;            p += al((size_t)n);
    int *bc = (int *)p;                     p += al((size_t)nblk * entries * sizeof(int));
    int *off = (int *)p;                    p += al((size_t)nblk * entries * sizeof(int));
    int *cnt = (int *)p;                    p += al(entries * sizeof(int));
    int *start = (int *)p;                  p += al(entries * sizeof(int));
    p += al(sizeof(int));
    float *Xs = (float *)p;
    cudaError_t e = cudaMemsetAsync(d_live, 0, sizeof(int), st);
    if (e != cudaSuccess) return (int)e;
    int rc = wc_vq_encode_launch(X, n, C, 1, entries, dim, asg, stream);
    if (rc) return rc;
    lloyd_count_kernel<<<nblk, 256, 0, st>>>(asg, n, entries, bc);
    lloyd_scan_kernel<<<1, 256, 0, st>>>(bc, nblk, entries, off, cnt, start);
    lloyd_place_kernel<<<nblk, 32, 0, st>>>(X, asg, n, entries, dim, off, start, Xs);
    lloyd_mean_kernel<<<(entries * dim + 255) / 256, 256, 0, st>>>(Xs, cnt, start, entries, dim,
                                                                    C, d_live);
    wc_count_launches(4);
    return (int)cudaGetLastError();
}

} /* extern "C" */
