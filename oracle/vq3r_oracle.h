/*
 * vq3r_oracle.h — CPU restatement of WARP's routed-expert FFN path, used as
 * the parity checker for the CUDA backend.
 *
 * TEST INFRASTRUCTURE ONLY. Nothing in the product (libwaste_cuda.so, the
 * warp_b200 package's compute path) links, loads or calls this code. Only
 * tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg use it,
 * and only as the checker or the timed CPU baseline.
 *
 * Every function restates one piece of the reference engine (paths are
 * relative to the sqliteai/warp source tree) and follows its arithmetic
 * order exactly, so that on x86 it reproduces the reference bit for bit:
 *
 *   orc_f16_flush      src/model.c:1278-1287   codebook f16->f32, subnormals -> signed 0
 *   orc_f16            src/simd.h:49-67        row/group scale f16->f32, subnormals kept
 *   orc_lut_build      src/simd_avx512.c:90-123 (FMA chain from 0, d ascending;
 *                      identical to src/simd_avx2.c:100-133), or with fma=0
 *                      the portable src/model.c:1862-1901 (mul then add)
 *   orc_vq_rows        src/model.c:1956-2024   blocked-index gather, t=(L0+L1)+L2
 *   orc_vq_matvec      src/model.c:2282-2289   lut build + gather
 *   orc_vq4p_quant     src/model.c:2049-2114   VQ4P: int8 table, one scale per 32 positions
 *   orc_vq4p_rows      src/model.c:2129-2229   VQ4P: 6-bit unpack, int16 block sums, fp32 fold
 *   orc_vq4p_matvec    src/model.c:2282-2289   VQ4P table + quantise + gather
 *   orc_dequant        tools/verify_container.py:51-88 with the loader's flush
 *   orc_dotf           src/model.c:155-160     x86 dot product (serial)
 *   orc_route          src/model.c:2720-2747   sigmoid + bias, iterative argmax,
 *                                              renorm (+1e-20), routed scale
 *   orc_mvq_rows       src/model.c:265-320     Q8G/Q4G/Q3G matvec, portable order
 *   orc_moe_layer      src/model.c:2713-2939   one token through router, K experts
 *                                              (router-order reduce) and shared FFN
 *   orc_moe_chunk      src/model.c:3512-3693   prefill chunk: ascending expert-id
 *                                              accumulation per token
 *   orc_situ_pair      src/model.c:505-509     K3's SiTU activation (act_situ)
 *   orc_rmsnorm        src/model.c:132-138     serial sum of squares, x*r*w
 *   orc_moe_block      src/model.c:3927-3945   h + moe_layer(rmsnorm(h)): the MoE
 *                                              half of a decoder layer
 *   orc_kda_step       src/kda.c:26-68         Kimi Delta Attention decode step
 *   orc_vq_encode      src/vq.c:50-105         the converter's RVQ encoder
 *   orc_vq_lloyd       src/vq.c:107-136        one Lloyd iteration
 *   orc_short_conv_step src/kda.c:84-99        causal depthwise conv + SiLU
 *   orc_rmsnorm_gated  src/kda.c:101-111       rmsnorm times sigmoid(gate)
 *
 * Parity is pinned against the reference compiled from its own sources
 * (oracle/Makefile -> oracle/_ref/libwaste_ref.so); see tests/golden/.
 */
#ifndef VQ3R_ORACLE_H
#define VQ3R_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

float orc_f16_flush(uint16_t h);
float orc_f16(uint16_t h);

/* books: [n_books][entries][vec_dim] fp32 (already flushed). */
void orc_lut_build(float *lut, const float *books, int cb_base, const float *x,
                   int nv, int stages, int entries, int vec_dim, int fma);

void orc_vq_rows(float *y, const uint8_t *idx, const uint16_t *scale,
                 const float *lut, int M, int nv, int stages, int entries);

void orc_vq_matvec(float *y, const uint8_t *idx, const uint16_t *scale,
                   const float *x, int M, int N, const float *books, int cb_base,
                   int stages, int entries, int vec_dim, float *lut_scratch,
                   int fma);

void orc_dequant(float *W, const uint8_t *idx, const uint16_t *scale, int M,
                 int N, const float *books, int cb_base, int stages,
                 int entries, int vec_dim, int index_block);

float orc_dotf(const float *a, const float *b, int n);
/* VQ4P: lut [nv][4][64] -> q [nv][4][64], qs [ceil(nv/32)]; rows over the
 * packed blocked layout [M/64][nv][64][3]; books [n_books][64][8]. */
void orc_vq4p_quant(const float *lut, int nv, int8_t *q, float *qs);
void orc_vq4p_rows(float *y, const uint8_t *idx, const uint16_t *scale, const int8_t *q,
                   const float *qs, int M, int nv);
void orc_vq4p_matvec(float *y, const uint8_t *idx, const uint16_t *scale, const float *x,
                     int M, int N, const float *books, int cb_base, float *lut, int8_t *q,
                     float *qs, int fma);

/* logits: [E]; writes idx[K], w[K]. bias may be NULL. */
void orc_route(const float *logits, const float *bias, int E, int K, int renorm,
               float routed_scale, int *idx, float *w);

/* Q8G (bits=8), Q4G (bits=4) or Q3G (bits=3) row matvec, group `group`,
 * rowbytes stride. */
void orc_mvq_rows(float *y, const int8_t *W, const uint16_t *ws, const float *x,
                  int rows, int in, int group, int bits, size_t rowbytes);

/* One MoE layer's weights, as the engine holds them. */
typedef struct {
    int hidden, inter, n_experts, top_k;
    int renorm;
    float routed_scale;
    int stages, entries, vec_dim, index_block;
    const float *router;        /* [E][hidden] f32                           */
    const float *bias;          /* [E] f32 or NULL                           */
    const float *books;         /* [n_books][entries][vec_dim], flushed      */
    int n_books;
    const uint8_t *bank;        /* E records of rec_bytes each               */
    size_t rec_bytes;
    int shared_inter;           /* 0 = no shared expert                      */
    const int8_t *sh_gate, *sh_up, *sh_down;       /* Q8G rows               */
    const uint16_t *sh_gate_s, *sh_up_s, *sh_down_s;
    int sh_bits, sh_group;
    int act_situ;               /* 0: SiLU(g)*u; 1: SiTU (K3)               */
    float situ_beta, situ_lbeta;
    int index_bits;             /* 8: VQ3R/VQ2R; 6: VQ4P (4 stages of 64)    */
} orc_moe;

float orc_situ_pair(float g, float u, float beta, float lbeta);
/* 1: the activations' (and KDA's) exp/tanh correctly rounded (the device's
 * arithmetic) instead of libm's expf/tanhf (the reference's); 0 (default). */
void orc_set_exact_math(int on);

/* Returns 0, or -1 when a record header does not describe the record. */
int orc_record_check(const orc_moe *L, int layer, int expert);

/* out[hidden] = routed (router order) + shared. idx/w may be NULL. */
int orc_moe_layer(const orc_moe *L, int layer, const float *x, float *out,
                  int *idx_out, float *w_out, int fma);

/* Routed experts only, given a route: ysum[lat] = sum_j w[j]*expert_j(x). */
int orc_moe_experts(const orc_moe *L, const int *idx, const float *w, int K,
                    const float *x, float *ysum, int fma);

/* nT tokens [nT][hidden] -> out [nT][hidden]; route/rw may be NULL. */
int orc_moe_chunk(const orc_moe *L, int layer, const float *x, int nT,
                  float *out, int *route, float *rw, int fma);

void orc_rmsnorm(float *o, const float *x, const float *w, int n, float eps);

/* h_out[hidden] = h + moe_layer(rmsnorm(h, norm_w, eps)). */
int orc_moe_block(const orc_moe *L, int layer, const float *h, const float *norm_w,
                  float eps, float *h_out, int *idx_out, float *w_out, int fma);

/* KDA: q, k, g_log [H][K]; v, o [H][V]; beta [H]; S [H][K][V] updated in
 * place; u scratch of V floats. */
void orc_kda_step(int H, int K, int V, const float *q, const float *k, const float *v,
                  const float *g_log, const float *beta, float *S, float *o, float *u);
void orc_short_conv_step(int C, int KS, const float *w, const float *bias, float *ring,
                         const float *x, float *y);
void orc_rmsnorm_gated(int C, const float *x, const float *gate, const float *weight,
                       float eps, float *y);
/* The converter's encoder: X [n][dim], books [stages][entries][dim],
 * out [n][stages]; Lloyd updates C [entries][dim] and returns the number of
 * non-empty clusters. */
void orc_vq_encode(const float *X, int n, const float *books, int stages, int entries, int dim,
                   uint8_t *out);
int orc_vq_lloyd(const float *X, int n, float *C, int entries, int dim);
#ifdef __cplusplus
}
#endif
#endif
