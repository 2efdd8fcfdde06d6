/*
 * mla.cu — the MLA attention layer's decode-time kernels on sm_100a, for the
 * whole-layer slot (the reference's mla_layer, src/model.c:2577-2649, with
 * the absorbed head loop mla_head_range, :2530-2575).
 *
 *   mla_prep_kernel  the latent c = kv_a_proj(x) normalised (rmsnorm with
 *                    kv_a_layernorm over its first kv_lora values), the
 *                    rotary pairs applied to it and to every head's query
 *                    (unless the model is NoPE), the latent stored at its
 *                    position in the cache and in the result block; or, for
 *                    the LoRA'd query, the plain rmsnorm of q_a
 *   mla_head_kernel  per head: q~ = W_kb^T q_nope (rows of kv_b_proj scaled
 *                    by the query and summed, the reference's order), the
 *                    scores against every cached latent (times the scale),
 *                    softmax, the context c~ = sum_s p_s c_s, and o = W_vb c~
 *   mla_gate_kernel  the optional sigmoid output gate
 *
 * B200 mapping. Decode attention over a short latent cache is latency work:
 * one CTA per head (512 threads, one per latent dimension), the query, the
 * absorbed query, the scores and the context in shared memory; kv_b_proj's
 * rows are read once per token with coalesced byte loads (8- or 4-bit
 * groups of 128, the engine's layout) and the latents once per phase. The
 * projections around it run through the trunk matvec (trunk_mvq.cu).
 * Sums keep the reference's orders where it has one (q~ over the query's
 * dimensions ascending, the context over positions ascending, the softmax
 * sum ascending); the dot products are lane-strided with warp reductions.
 */
#include "vq3r_common.cuh"
#include "wc_launch.h"
#include "pdl.cuh"

#include <cuda_runtime.h>
#include <stdint.h>

using namespace wc;

namespace {

constexpr int kMlaThreads = 512;
constexpr int kLatBatch = 16;        /* cached-latent loads a thread has in flight */

/* Value j of row r of a quantised trunk tensor (groups of `group`, one f16
 * scale per group): 8-bit signed bytes, or 4-bit codes minus 8 (low nibble
 * first), times the group's scale — src/model.c:407-440. W and ws are the
 * head's rows staged in shared memory (r counted from the head's first).
 * Column j's place in a row is the same for every row (its group gj, the
 * byte holding it and, at 4 bits, which nibble), so DeqCol computes it once
 * and steps it along a lane's columns without a division. */
struct DeqCol {
    int gj, jin;                     /* group, index inside it */
    __device__ __forceinline__ DeqCol(int j, int group) : gj(j / group), jin(j - gj * group) {}
    __device__ __forceinline__ void advance(int step, int group)
    {
        jin += step;
        while (jin >= group) { jin -= group; gj++; }
    }
};

template <int BITS>
__device__ __forceinline__ float deq_col(const uint8_t *W, const uint16_t *ws, size_t rowbytes,
                                         int ng, int group, int r, const DeqCol &c)
{
    const float s = f16_keep(ws[(size_t)r * ng + c.gj]);
    const uint8_t *row = W + (size_t)r * rowbytes;
    if (BITS == 8) return s * (float)(int8_t)row[c.gj * group + c.jin];
    const uint8_t byte = row[(c.gj * group) / 2 + (c.jin >> 1)];
    const int v = (c.jin & 1) ? (byte >> 4) - 8 : (byte & 0x0F) - 8;
    return s * (float)v;
}

__device__ __forceinline__ float block_sum(float v, float *red)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[w] = v;
    __syncthreads();
    float t = 0.0f;
    for (int k = 0; k < nw; k++) t += red[k];
    return t;
}

/* One block. x[0..n) normalised in place by weight w (rmsnorm; n <= 8 *
 * blockDim). With rope (cs/sn, half pairs) the pairs of rot[0..2*half) are
 * rotated; with q (nh heads of qd, rope part at qk_nope) every head's rope
 * pairs too. lat_dst / lat_out: where the latent (x then rot, latd values)
 * is stored (the cache row and the result block). */
__global__ void __launch_bounds__(kMlaThreads) mla_prep_kernel(
    float *x, int n, const float *w, float eps, float *rot, const float *cs, const float *sn,
    int half, float *q, int nh, int qd, int qk_nope, float *lat, const int *pos_p,
    float *lat_out, int latd)
{
    /* the cache row of this token's position (read from device memory, so
     * one launch serves every position) */
    float *lat_dst = lat && pos_p ? lat + (size_t)(*pos_p) * latd : nullptr;
    wc_pdl::trigger();               /* the head kernel behind may stage its rows */
    __shared__ float red[32];
    float v[8];
    float s = 0.0f;
#pragma unroll
    for (int k = 0; k < 8; k++) {
        const int i = threadIdx.x + k * blockDim.x;
        v[k] = i < n ? x[i] : 0.0f;
        s = __fadd_rn(s, __fmul_rn(v[k], v[k]));
    }
    s = block_sum(s, red);
    const float r = 1.0f / sqrtf(s / (float)n + eps);
#pragma unroll
    for (int k = 0; k < 8; k++) {
        const int i = threadIdx.x + k * blockDim.x;
        if (i < n) x[i] = __fmul_rn(__fmul_rn(v[k], r), w[i]);
    }
    if (half > 0) {                  /* src/model.c:2512-2519 */
        for (int j = threadIdx.x; j < half; j += blockDim.x) {
            const float e = rot[2 * j], o = rot[2 * j + 1];
            rot[2 * j] = __fsub_rn(__fmul_rn(e, cs[j]), __fmul_rn(o, sn[j]));
            rot[2 * j + 1] = __fadd_rn(__fmul_rn(e, sn[j]), __fmul_rn(o, cs[j]));
        }
        for (int t = threadIdx.x; t < nh * half; t += blockDim.x) {
            const int h = t / half, j = t % half;
            float *qr = q + (size_t)h * qd + qk_nope;
            const float e = qr[2 * j], o = qr[2 * j + 1];
            qr[2 * j] = __fsub_rn(__fmul_rn(e, cs[j]), __fmul_rn(o, sn[j]));
            qr[2 * j + 1] = __fadd_rn(__fmul_rn(e, sn[j]), __fmul_rn(o, cs[j]));
        }
    }
    __syncthreads();
    for (int i = threadIdx.x; lat_dst && i < latd; i += blockDim.x) {
        lat_dst[i] = x[i];
        if (lat_out) lat_out[i] = x[i];
    }
}

/* grid nh: head h, over cache rows 0..*pos_p. Shared memory: the head's
 * kv_b_proj rows (nope + vh rows, staged by one bulk copy at the start) and
 * their scales | q (qd) | q~ (kl) | c~ (kl) | scores (up to the cache's
 * rows). */
template <int BITS>
__global__ void __launch_bounds__(kMlaThreads, 1) mla_head_kernel(
    const float *__restrict__ q, const float *__restrict__ lat, const int *pos_p, int latd, int kl,
    int qd, int nope, int rope, int vh, const uint8_t *__restrict__ W,
    const uint16_t *__restrict__ ws, size_t rowbytes, int ng, int group, float scale,
    float *__restrict__ o)
{
    extern __shared__ __align__(16) unsigned char smb[];
    __shared__ float red[32];
    __shared__ __align__(8) uint64_t bar;
    __shared__ int okw;
    const int h = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int nw = blockDim.x >> 5, wrows = nope + vh;
    const uint32_t wb = (uint32_t)((size_t)wrows * rowbytes), sb = (uint32_t)wrows * ng * 2;
    uint8_t *Ws = smb;
    uint16_t *wss = reinterpret_cast<uint16_t *>(smb + wb);
    float *qs = reinterpret_cast<float *>(smb + wb + ((sb + 15) & ~15u));
    float *qa = qs + ((qd + 3) & ~3), *ca = qa + ((kl + 3) & ~3), *sc = ca + ((kl + 3) & ~3);
    if (tid == 0) {                  /* the head's rows: constants, before the wait */
        mbar_init(&bar, 1);
        mbar_fence_init();
        mbar_expect_tx(&bar, wb + sb);
        bulk_g2s(Ws, W + (size_t)h * wrows * rowbytes, wb, &bar);
        bulk_g2s(wss, ws + (size_t)h * wrows * ng, sb, &bar);
    }
    wc_pdl::trigger();
    wc_pdl::wait();                  /* q, the cache row and the position: the prep's */
    const int S = *pos_p + 1;
    for (int i = tid; i < qd; i += blockDim.x) qs[i] = q[(size_t)h * qd + i];
    if (tid == 0) okw = mbar_wait(&bar, 0);
    __syncthreads();
    if (!okw) {                      /* the copy never landed: the head's output is NaN */
        for (int i = tid; i < vh; i += blockDim.x) o[(size_t)h * vh + i] = __int_as_float(0x7fc00000);
        return;
    }
    /* q~[j] = sum over i ascending of q_i * W_kb[h*wrows + i][j] (exact
     * zeros skipped, as the reference does) */
    for (int j = tid; j < kl; j += blockDim.x) {
        const DeqCol col(j, group);
        float acc = 0.0f;
#pragma unroll 8
        for (int i = 0; i < nope; i++) {
            const float qi = qs[i];
            if (qi == 0.0f) continue;
            acc = __fadd_rn(acc, __fmul_rn(qi, deq_col<BITS>(Ws, wss, rowbytes, ng, group, i, col)));
        }
        qa[j] = acc;
    }
    __syncthreads();
    /* scores: one warp per position. The cached latents are read through L2
     * (the prep kernel ahead wrote this token's row), each lane's loads
     * batched ahead of its sums, which keep their order. */
    for (int s = warp; s < S; s += nw) {
        const float *cs = lat + (size_t)s * latd;
        float a = 0.0f, b = 0.0f;
        float rv[2];
#pragma unroll
        for (int u = 0; u < 2; u++)
            rv[u] = lane + 32 * u < rope ? __ldcg(cs + kl + lane + 32 * u) : 0.0f;
        for (int j0 = lane; j0 < kl; j0 += 32 * kLatBatch) {
            float v[kLatBatch];
#pragma unroll
            for (int u = 0; u < kLatBatch; u++)
                v[u] = j0 + 32 * u < kl ? __ldcg(cs + j0 + 32 * u) : 0.0f;
#pragma unroll
            for (int u = 0; u < kLatBatch; u++)
                if (j0 + 32 * u < kl) a = fmaf(qa[j0 + 32 * u], v[u], a);
        }
#pragma unroll
        for (int u = 0; u < 2; u++)
            if (lane + 32 * u < rope) b = fmaf(qs[nope + lane + 32 * u], rv[u], b);
        for (int j = lane + 64; j < rope; j += 32) b = fmaf(qs[nope + j], __ldcg(cs + kl + j), b);
#pragma unroll
        for (int k = 16; k > 0; k >>= 1) {
            a += __shfl_xor_sync(0xffffffffu, a, k);
            b += __shfl_xor_sync(0xffffffffu, b, k);
        }
        if (lane == 0) sc[s] = __fmul_rn(__fadd_rn(a, b), scale);
    }
    __syncthreads();
    /* softmax (src/model.c:511-518): max, exp(x - max), sum, divide */
    float mx = -3.402823466e38f;
    for (int s = tid; s < S; s += blockDim.x) mx = fmaxf(mx, sc[s]);
#pragma unroll
    for (int k = 16; k > 0; k >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, k));
    if (lane == 0) red[warp] = mx;
    __syncthreads();
    mx = red[0];
    for (int k = 1; k < nw; k++) mx = fmaxf(mx, red[k]);
    __syncthreads();
    for (int s = tid; s < S; s += blockDim.x) sc[s] = expf_cr(__fsub_rn(sc[s], mx));
    __syncthreads();
    if (tid == 0) {                  /* the sum in position order */
        float t = 0.0f;
        for (int s = 0; s < S; s++) t = __fadd_rn(t, sc[s]);
        red[0] = t;
    }
    __syncthreads();
    const float sum = red[0];
    __syncthreads();
    for (int s = tid; s < S; s += blockDim.x) sc[s] = __fdiv_rn(sc[s], sum);
    __syncthreads();
    /* c~[j] = sum over positions ascending of p_s * c_s[j] */
    for (int j = tid; j < kl; j += blockDim.x) {
        float acc = 0.0f;
        for (int s0 = 0; s0 < S; s0 += kLatBatch) {
            float v[kLatBatch];
#pragma unroll
            for (int u = 0; u < kLatBatch; u++)
                v[u] = s0 + u < S ? __ldcg(lat + (size_t)(s0 + u) * latd + j) : 0.0f;
#pragma unroll
            for (int u = 0; u < kLatBatch; u++)
                if (s0 + u < S) acc = __fadd_rn(acc, __fmul_rn(sc[s0 + u], v[u]));
        }
        ca[j] = acc;
    }
    __syncthreads();
    /* o[i] = W_vb[h*wrows + nope + i] . c~, one warp per row */
    for (int i = warp; i < vh; i += nw) {
        const int r = nope + i;
        float a = 0.0f;
        DeqCol col(lane, group);
        for (int j = lane; j < kl; j += 32, col.advance(32, group))
            a = fmaf(deq_col<BITS>(Ws, wss, rowbytes, ng, group, r, col), ca[j], a);
#pragma unroll
        for (int k = 16; k > 0; k >>= 1) a += __shfl_xor_sync(0xffffffffu, a, k);
        if (lane == 0) o[(size_t)h * vh + i] = a;
    }
}

__global__ void __launch_bounds__(256) mla_gate_kernel(float *o, const float *g, int n)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    wc_pdl::trigger();               /* the output projection may stage its weights */
    wc_pdl::wait();                  /* o: the head kernel's */
    if (i < n) o[i] = __fmul_rn(o[i], __fdiv_rn(1.0f, __fadd_rn(1.0f, expf_cr(-g[i]))));
}

} /* namespace */

extern "C" {

size_t wc_mla_head_smem(int qd, int kl, int S, int wrows, size_t rowbytes, int ng)
{
    const size_t wb = (size_t)wrows * rowbytes, sb = ((size_t)wrows * ng * 2 + 15) & ~(size_t)15;
    return wb + sb + (size_t)(((qd + 3) & ~3) + 2 * ((kl + 3) & ~3) + S) * sizeof(float);
}

int wc_mla_prep_launch(float *x, int n, const float *w, float eps, float *rot, const float *cs,
                       const float *sn, int half, float *q, int nh, int qd, int qk_nope,
                       float *lat, const int *pos_p, float *lat_out, int latd, void *stream)
{
    if (n > 8 * kMlaThreads) return (int)cudaErrorInvalidValue;
    mla_prep_kernel<<<1, kMlaThreads, 0, (cudaStream_t)stream>>>(
        x, n, w, eps, rot, cs, sn, half, q, nh, qd, qk_nope, lat, pos_p, lat_out, latd);
    wc_count_launches(1);
    return (int)cudaGetLastError();
}

int wc_mla_head_launch(const float *q, const float *lat, const int *pos_p, int S_max, int latd,
                       int kl, int qd, int nope, int rope, int vh, int nh, const uint8_t *W,
                       const uint16_t *ws, size_t rowbytes, int ng, int group, int bits,
                       float scale, float *o, void *stream, int pdl)
{
    /* the bulk copies want 16-byte sizes and addresses */
    if ((((size_t)(nope + vh) * rowbytes) & 15) || (((size_t)(nope + vh) * ng * 2) & 15) ||
        ((uintptr_t)W & 15) || ((uintptr_t)ws & 15))
        return (int)cudaErrorInvalidValue;
    const size_t smem = wc_mla_head_smem(qd, kl, S_max, nope + vh, rowbytes, ng);
    cudaError_t e;
    if (bits == 8) {
        e = cudaFuncSetAttribute(mla_head_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)smem);
        if (e != cudaSuccess) return (int)e;
        e = wc_pdl::launch(mla_head_kernel<8>, dim3(nh), dim3(kMlaThreads), smem,
                           (cudaStream_t)stream, pdl != 0, q, lat, pos_p, latd, kl, qd, nope,
                           rope, vh, W, ws, rowbytes, ng, group, scale, o);
    } else if (bits == 4) {
        e = cudaFuncSetAttribute(mla_head_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)smem);
        if (e != cudaSuccess) return (int)e;
        e = wc_pdl::launch(mla_head_kernel<4>, dim3(nh), dim3(kMlaThreads), smem,
                           (cudaStream_t)stream, pdl != 0, q, lat, pos_p, latd, kl, qd, nope,
                           rope, vh, W, ws, rowbytes, ng, group, scale, o);
    } else {
        return (int)cudaErrorInvalidValue;
    }
    wc_count_launches(1);
    return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

int wc_mla_gate_launch(float *o, const float *g, int n, void *stream, int pdl)
{
    const cudaError_t e = wc_pdl::launch(mla_gate_kernel, dim3((n + 255) / 256), dim3(256), 0,
                                         (cudaStream_t)stream, pdl != 0, o, g, n);
    wc_count_launches(1);
    return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

} /* extern "C" */
