/*
 * kda.cu — Kimi Delta Attention's decode-time kernels on sm_100a: the
 * kda_step, short_conv_step and rmsnorm_gated slots of the reference's
 * dispatch table (src/waste_backend.h:69-76; arithmetic src/kda.c:19-111).
 *
 *   kda_step       per head: q, k L2-normalised (q also by K^-0.5); the state
 *                  rows decayed by exp(g) and u = S'^T k (pass A); the delta
 *                  d = beta (v - u); S += k d^T and o = S^T q (pass B)
 *   short_conv     per channel: a causal depthwise conv over a ring of the
 *                  previous KS-1 inputs, the ring shifted, then SiLU
 *   rmsnorm_gated  per head: x * r * w * sigmoid(gate), r = 1/sqrt(mean x^2 + eps)
 *
 * B200 mapping. The recurrent state (K x V floats a head, 64 KB at 128 x 128)
 * stays in HBM between tokens. One warp per (head, 32 columns), lane l
 * owning one column of the head's state: the column is copied into shared
 * memory with all its rows in flight at once (cp.async), decayed and
 * reduced into u (pass A), then updated, reduced into o and written once
 * (pass B) — the state crosses HBM twice a token (a read and a write,
 * 128-byte row segments), where the CPU streams it through cache four
 * times. kv = k*kn and qv = q*qn are
 * recomputed per use, which gives the same floats as the CPU's.
 *
 * Arithmetic follows the reference's x86 build term for term (rounded
 * multiply, then rounded add: no contraction), the serial sums in the same
 * order, sqrtf and the divisions IEEE, and exp rounded once (expf_cr), so
 * the device matches the CPU bit for bit except where glibc's expf is not
 * correctly rounded (a few inputs in 10^4).
 */
#include "vq3r_common.cuh"
#include "wc_launch.h"
#include "pdl.cuh"

#include <cuda_runtime.h>
#include <stdint.h>

using namespace wc;

namespace {

/* src/kda.c:19-24: serial sum of squares, 1 / sqrtf(s + 1e-12). N is a
 * compile-time length, so the loads are issued well ahead of the (serial)
 * adds. */
template <int N>
__device__ __forceinline__ float l2_rnorm_serial(const float *x)
{
    float s = 0.0f;
#pragma unroll 32
    for (int i = 0; i < N; i++) s = __fadd_rn(s, __fmul_rn(x[i], x[i]));
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(s, 1e-12f)));
}

/* 4-byte asynchronous copy global -> shared (cp.async), so that all K rows
 * of a lane's column are in flight at once. */
__device__ __forceinline__ void cp_async4(float *dst, const float *src)
{
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;"
                 ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(dst))), "l"(src) : "memory");
}

/* grid (H, ceil(V/32)), one warp: lane l owns column c = 32*blockIdx.y + l
 * of head blockIdx.x. The column is copied into shared memory first, all
 * K rows at once (one memory round trip instead of one per few rows), and
 * both passes work on it there. The state is the previous token's, final
 * before this layer began, so its copies are issued before the wait on the
 * kernel that produced q, k, v, g and beta. */
template <int K>
__global__ void __launch_bounds__(32) kda_step_kernel(int V, const float *__restrict__ q,
                                                      const float *__restrict__ k,
                                                      const float *__restrict__ v,
                                                      const float *__restrict__ g_log,
                                                      const float *__restrict__ beta, float *S,
                                                      float *__restrict__ o)
{
    __shared__ float qs[K], ks[K], dec[K];
    __shared__ float col[K][32];
    __shared__ float norms[2];
    const int h = blockIdx.x, lane = threadIdx.x;
    const int c = blockIdx.y * 32 + lane;
    float *Sc = S + (size_t)h * K * V + c;
    if (c < V) {
#pragma unroll 16
        for (int kk = 0; kk < K; kk++) cp_async4(&col[kk][lane], Sc + (size_t)kk * V);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    wc_pdl::trigger();
    wc_pdl::wait();
    for (int i = lane; i < K; i += 32) {
        qs[i] = q[(size_t)h * K + i];
        ks[i] = k[(size_t)h * K + i];
        dec[i] = expf_cr(g_log[(size_t)h * K + i]);
    }
    __syncwarp();
    if (lane == 0) {
        const float qscale = __fdiv_rn(1.0f, __fsqrt_rn((float)K));
        norms[0] = __fmul_rn(l2_rnorm_serial<K>(qs), qscale);
    } else if (lane == 16) {
        norms[1] = l2_rnorm_serial<K>(ks);
    }
    __syncwarp();
    const float qn = norms[0], kn = norms[1];
    asm volatile("cp.async.wait_group 0;" ::: "memory");   /* this lane's own column */
    if (c >= V) return;
    float u = 0.0f;
#pragma unroll 32
    for (int kk = 0; kk < K; kk++) {
        const float r = __fmul_rn(col[kk][lane], dec[kk]);
        col[kk][lane] = r;
        u = __fadd_rn(u, __fmul_rn(r, __fmul_rn(ks[kk], kn)));
    }
    const float d = __fmul_rn(beta[h], __fsub_rn(v[(size_t)h * V + c], u));
    float acc = 0.0f;
#pragma unroll 32
    for (int kk = 0; kk < K; kk++) {
        const float r = __fadd_rn(col[kk][lane], __fmul_rn(d, __fmul_rn(ks[kk], kn)));
        acc = __fadd_rn(acc, __fmul_rn(r, __fmul_rn(qs[kk], qn)));
        Sc[(size_t)kk * V] = r;
    }
    o[(size_t)h * V + c] = acc;
}

__global__ void __launch_bounds__(256) short_conv_kernel(int C, int KS, const float *__restrict__ w,
                                                         const float *__restrict__ bias,
                                                         float *ring, const float *x, float *y)
{
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= C) return;
    const int R = KS - 1;
    const float *wc = w + (size_t)c * KS;
    float *rc = ring + (size_t)c * R;
    const float xc = x[c];
    float acc = bias ? bias[c] : 0.0f;
    for (int j = 0; j < R; j++) acc = __fadd_rn(acc, __fmul_rn(rc[j], wc[j]));
    acc = __fadd_rn(acc, __fmul_rn(xc, wc[R]));
    for (int j = 0; j + 1 < R; j++) rc[j] = rc[j + 1];
    if (R > 0) rc[R - 1] = xc;
    y[c] = __fdiv_rn(acc, __fadd_rn(1.0f, expf_cr(-acc)));
}

/* nh heads of C channels, one CTA each (one weight vector for all). */
__global__ void __launch_bounds__(128) rmsnorm_gated_kernel(int C, const float *x, const float *gate,
                                                            const float *__restrict__ weight,
                                                            float eps, float *y)
{
    extern __shared__ float xs[];
    __shared__ float rr;
    const size_t base = (size_t)blockIdx.x * C;
    wc_pdl::trigger();          /* the projection behind may stage its weights */
    wc_pdl::wait();             /* x: the step's output */
    for (int i = threadIdx.x; i < C; i += blockDim.x) xs[i] = x[base + i];
    __syncthreads();
    if (threadIdx.x == 0) {
        float s = 0.0f;
        for (int i = 0; i < C; i++) s = __fadd_rn(s, __fmul_rn(xs[i], xs[i]));
        rr = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(s, (float)C), eps)));
    }
    __syncthreads();
    const float r = rr;
    for (int i = threadIdx.x; i < C; i += blockDim.x) {
        const float g = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf_cr(-gate[base + i])));
        y[base + i] = __fmul_rn(__fmul_rn(__fmul_rn(xs[i], r), weight[i]), g);
    }
}

/* The decay gate in place (src/model.c:2374-2391, per head): with
 * lower_bound < 0, g = lb / (1 + exp(-ea * z)); else g = -ea * softplus(z)
 * (z itself above 20), z = g + dt_bias, ea = exp(A_log[h]); and beta =
 * sigmoid(beta) (src/model.c:2447). exp and log1p rounded once. */
__global__ void __launch_bounds__(256) kda_gate_kernel(float *g, const float *A_log,
                                                       const float *dt_bias, int H, int D,
                                                       float lower_bound, float *beta)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    wc_pdl::trigger();          /* the step behind may fetch its state meanwhile */
    if (i < H) beta[i] = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf_cr(-beta[i])));
    if (i >= H * D) return;
    const float ea = expf_cr(A_log[i / D]);
    const float z = __fadd_rn(g[i], dt_bias ? dt_bias[i] : 0.0f);
    if (lower_bound < 0.0f) {
        g[i] = __fdiv_rn(lower_bound, __fadd_rn(1.0f, expf_cr(-__fmul_rn(ea, z))));
    } else {
        const float sp = z > 20.0f ? z : (float)log1p((double)expf_cr(z));
        g[i] = __fmul_rn(-ea, sp);
    }
}

} /* namespace */

extern "C" {

int wc_kda_gate_launch(float *g, const float *A_log, const float *dt_bias, int H, int D,
                       float lower_bound, float *beta, void *stream)
{
    kda_gate_kernel<<<(H * D + 255) / 256, 256, 0, (cudaStream_t)stream>>>(g, A_log, dt_bias, H,
                                                                            D, lower_bound, beta);
    wc_count_launches(1);
    return (int)cudaGetLastError();
}

int wc_kda_supported(int K, int V)
{
    return (K == 128 || K == 64 || K == 32) && V > 0 ? 0 : -1;
}

int wc_kda_step_launch(int H, int K, int V, const float *q, const float *k, const float *v,
                       const float *g_log, const float *beta, float *S, float *o, void *stream,
                       int pdl)
{
    cudaStream_t st = (cudaStream_t)stream;
    const dim3 grid(H, (V + 31) / 32);
    cudaError_t e;
    if (K == 128)
        e = wc_pdl::launch(kda_step_kernel<128>, grid, dim3(32), 0, st, pdl != 0, V, q, k, v,
                           g_log, beta, S, o);
    else if (K == 64)
        e = wc_pdl::launch(kda_step_kernel<64>, grid, dim3(32), 0, st, pdl != 0, V, q, k, v,
                           g_log, beta, S, o);
    else if (K == 32)
        e = wc_pdl::launch(kda_step_kernel<32>, grid, dim3(32), 0, st, pdl != 0, V, q, k, v,
                           g_log, beta, S, o);
    else
        return (int)cudaErrorInvalidValue;
    wc_count_launches(1);
    return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

int wc_short_conv_launch(int C, int KS, const float *w, const float *bias, float *ring,
                         const float *x, float *y, void *stream)
{
    short_conv_kernel<<<(C + 255) / 256, 256, 0, (cudaStream_t)stream>>>(C, KS, w, bias, ring, x,
                                                                          y);
    wc_count_launches(1);
    return (int)cudaGetLastError();
}

int wc_rmsnorm_gated_launch(int nh, int C, const float *x, const float *gate, const float *weight,
                            float eps, float *y, void *stream, int pdl)
{
    const cudaError_t e = wc_pdl::launch(rmsnorm_gated_kernel, dim3(nh), dim3(128),
                                         (size_t)C * sizeof(float), (cudaStream_t)stream,
                                         pdl != 0, C, x, gate, weight, eps, y);
    wc_count_launches(1);
    return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

} /* extern "C" */
