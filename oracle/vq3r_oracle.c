/*
 * vq3r_oracle.c — CPU restatement of the reference's routed-expert FFN path.
 *
 * TEST INFRASTRUCTURE ONLY: the checker for the CUDA backend, never part of
 * the product path (see vq3r_oracle.h). Build with -ffp-contract=off so that
 * every `a += b * c` below stays a rounded multiply followed by a rounded
 * add, which is what the reference's x86 build (-O2, no -mfma) executes.
 * The FMA chains that the reference's AVX2/AVX-512 kernels execute are
 * written as explicit fmaf() calls.
 *
 * Parity is pinned: tests/golden/ holds vectors produced by the reference
 * compiled from its own sources (oracle/Makefile), and tests/test_golden.py
 * checks this file against them bit for bit.
 */
#include "vq3r_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* Expert record header: the reference's 48-byte waste_expert_hdr
 * (src/waste_format.h:98-132). The layout is the on-disk format, so it has
 * to be the same field for field. */
typedef struct {
    uint32_t magic;
    uint16_t layer, expert_id;
    uint8_t fmt, flags;
    uint16_t codebook_id, lowrank_id, reserved0;
    uint32_t rec_4k_blocks;
    uint32_t gate_off, up_off, down_off, chan_corr_off;
    uint32_t crc32;
    uint32_t reserved1[2];
} orc_hdr;

#define ORC_MAGIC_EXPERT 0x50584557u /* src/waste_format.h:33 */
#define ORC_WQ_VQ3R 4                /* src/waste_format.h:51 */
#define ORC_WQ_VQ2R 5                /* src/waste_format.h:52 */
#define ORC_WQ_VQ4P 8                /* src/waste_format.h:57 */
#define ORC_LUT_BLK 32               /* WASTE_VQ_LUT_BLK, src/model.h:60 */
#define ORC_ALIGN 4096u              /* src/waste_format.h:42 */

/* src/model.c:1278-1287: sign kept, exponent 0 (zero or subnormal) -> 0.
 * Exponent 31 is not special-cased there, so it is not here either. */
float orc_f16_flush(uint16_t v)
{
    const uint32_t sign = (uint32_t)(v >> 15) << 31;
    const uint32_t e = (v >> 10) & 0x1f, man = v & 0x3ff;
    const uint32_t bits = e ? (sign | ((e + 112u) << 23) | (man << 13)) : sign;
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* src/simd.h:49-67: subnormals are mantissa * 2^-24, not zero. */
float orc_f16(uint16_t h)
{
    const uint32_t sign = (uint32_t)(h >> 15) << 31;
    const uint32_t e = (h >> 10) & 0x1f, mn = h & 0x3ff;
    if (e == 0) {
        const float f = (float)mn * 5.9604644775390625e-08f;
        return sign ? -f : f;
    }
    const uint32_t bits = sign | ((e + 112u) << 23) | (mn << 13);
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* lut[(v*stages + s)*entries + c] = sum_d x[v*vd + d] * C_{cb_base+s}[c][d].
 * fma=1: acc = fma(x_d, C, acc) from acc = 0, d ascending — the order of
 *        src/simd_avx512.c:104-112 and src/simd_avx2.c:114-122.
 * fma=0: t += x_d * C — src/model.c:1893-1897 on x86 (no contraction). */
void orc_lut_build(float *lut, const float *books, int cb_base, const float *x,
                   int nv, int stages, int entries, int vd, int fma)
{
    for (int v = 0; v < nv; v++) {
        const float *xv = x + (size_t)v * vd;
        for (int s = 0; s < stages; s++) {
            const float *C = books + (size_t)(cb_base + s) * entries * vd;
            float *dst = lut + ((size_t)v * stages + s) * entries;
            for (int c = 0; c < entries; c++) {
                float t = 0.0f;
                if (fma)
                    for (int d = 0; d < vd; d++)
                        t = fmaf(xv[d], C[(size_t)c * vd + d], t);
                else
                    for (int d = 0; d < vd; d++)
                        t += xv[d] * C[(size_t)c * vd + d];
                dst[c] = t;
            }
        }
    }
}

/* src/model.c:1956-2024. Index layout [M/64][nv][64][stages]; per row the
 * sum runs over v ascending and each term is (L0 + L1) + L2, which is what
 * both the eight-row unrolled body and the remainder loop evaluate. */
void orc_vq_rows(float *y, const uint8_t *idx, const uint16_t *scale,
                 const float *lut, int M, int nv, int st, int en)
{
    const int B = 64; /* VQ_TILE == index_block, src/model.c:1937 */
    for (int r = 0; r < M; r++) {
        const int rb = r / B, ri = r % B;
        float acc = 0.0f;
        for (int v = 0; v < nv; v++) {
            const float *blk = lut + (size_t)v * st * en;
            const uint8_t *ix = idx + (((size_t)rb * nv + v) * B + ri) * st;
            float t = blk[ix[0]];
            for (int s = 1; s < st; s++) t += blk[(size_t)s * en + ix[s]];
            acc += t;
        }
        y[r] = acc * orc_f16(scale[r]);
    }
}

/* src/model.c:2282-2289: build the table for this x, then gather. */
void orc_vq_matvec(float *y, const uint8_t *idx, const uint16_t *scale,
                   const float *x, int M, int N, const float *books, int cb_base,
                   int stages, int entries, int vd, float *lut, int fma)
{
    orc_lut_build(lut, books, cb_base, x, N / vd, stages, entries, vd, fma);
    orc_vq_rows(y, idx, scale, lut, M, N / vd, stages, entries);
}

/* src/model.c:2049-2114 vq_quant_range, the portable loop: per block of 32
 * positions (4 stages x 64 entries each), mx = max |lut| by a strict >
 * scan, scale mx / 127, and q = clamp(lrintf(lut * (127 / mx)), -127, 127)
 * (inv = 0 when mx is 0). */
void orc_vq4p_quant(const float *lut, int nv, int8_t *q, float *qs)
{
    const int per = 4 * 64;
    for (int blk = 0; blk * ORC_LUT_BLK < nv; blk++) {
        const int v0 = blk * ORC_LUT_BLK;
        const int v1 = v0 + ORC_LUT_BLK < nv ? v0 + ORC_LUT_BLK : nv;
        const size_t n = (size_t)(v1 - v0) * per;
        const float *src = lut + (size_t)v0 * per;
        float mx = 0.0f;
        for (size_t i = 0; i < n; i++) {
            const float f = fabsf(src[i]);
            if (f > mx) mx = f;
        }
        qs[blk] = mx / 127.0f;
        const float inv = mx > 0 ? 127.0f / mx : 0.0f;
        for (size_t i = 0; i < n; i++) {
            int t = (int)lrintf(src[i] * inv);
            if (t > 127) t = 127;
            else if (t < -127) t = -127;
            q[(size_t)v0 * per + i] = (int8_t)t;
        }
    }
}

/* src/model.c:2129-2229 vq_rows_p6, the portable loop: per row and block of
 * 32 positions an int16 sum of the four stages' table bytes (indices
 * unpacked from three little-endian bytes, 6 bits each), folded into
 * acc += scale_blk * (float)sum; y = acc * f16(row scale). */
void orc_vq4p_rows(float *y, const uint8_t *idx, const uint16_t *scale, const int8_t *q,
                   const float *qs, int M, int nv)
{
    const int B = 64, en = 64;
    for (int r = 0; r < M; r++) {
        const int rb = r / B, ri = r % B;
        float acc = 0.0f;
        for (int v0 = 0; v0 < nv; v0 += ORC_LUT_BLK) {
            const int v1 = v0 + ORC_LUT_BLK < nv ? v0 + ORC_LUT_BLK : nv;
            int16_t sum = 0;
            for (int v = v0; v < v1; v++) {
                const int8_t *T = q + (size_t)v * 4 * en;
                const uint8_t *ix = idx + (((size_t)rb * nv + v) * B + ri) * 3;
                const unsigned b0 = ix[0], b1 = ix[1], b2 = ix[2];
                const unsigned j0 = b0 & 0x3f, j1 = ((b0 >> 6) | (b1 << 2)) & 0x3f;
                const unsigned j2 = ((b1 >> 4) | (b2 << 4)) & 0x3f, j3 = (b2 >> 2) & 0x3f;
                sum = (int16_t)(sum + T[j0] + T[en + j1] + T[2 * en + j2] + T[3 * en + j3]);
            }
            acc += qs[v0 / ORC_LUT_BLK] * (float)sum;
        }
        y[r] = acc * orc_f16(scale[r]);
    }
}

/* src/model.c:2282-2289 vq_matvec for a VQ4P matrix: the fp32 table (books
 * [n][64][8]), its int8 quantisation, then the packed-index gather. */
void orc_vq4p_matvec(float *y, const uint8_t *idx, const uint16_t *scale, const float *x,
                     int M, int N, const float *books, int cb_base, float *lut, int8_t *q,
                     float *qs, int fma)
{
    orc_lut_build(lut, books, cb_base, x, N / 8, 4, 64, 8, fma);
    orc_vq4p_quant(lut, N / 8, q, qs);
    orc_vq4p_rows(y, idx, scale, q, qs, M, N / 8);
}

/* tools/verify_container.py:73-84 (un-block, recon = sum_s C_s[idx_s] from a
 * zero vector, times the row scale), with the codebooks decoded the way the
 * engine decodes them (flushed, src/model.c:1278-1287). W is [M][N]. */
void orc_dequant(float *W, const uint8_t *idx, const uint16_t *scale, int M,
                 int N, const float *books, int cb_base, int st, int en,
                 int vd, int B)
{
    const int nv = N / vd;
    for (int r = 0; r < M; r++) {
        const float sc = orc_f16(scale[r]);
        for (int v = 0; v < nv; v++) {
            const uint8_t *ix = idx + (((size_t)(r / B) * nv + v) * B + r % B) * st;
            for (int d = 0; d < vd; d++) {
                float rec = 0.0f;
                for (int s = 0; s < st; s++)
                    rec += books[((size_t)(cb_base + s) * en + ix[s]) * vd + d];
                W[(size_t)r * N + (size_t)v * vd + d] = rec * sc;
            }
        }
    }
}

/* src/model.c:155-160 (the x86 build). */
float orc_dotf(const float *a, const float *b, int n)
{
    float acc = 0;
    for (int i = 0; i < n; i++) acc += a[i] * b[i];
    return acc;
}

/* exp and tanh of the activations (and of KDA): libm's expf / tanhf (what
 * the reference calls), or — with orc_set_exact_math(1) — the correctly
 * rounded values, computed in double and rounded once. The second mode is
 * the device's arithmetic where its exp and tanh are correctly rounded, so
 * the two differ only where libm's float functions are not. The router's
 * sigmoid always uses expf. */
static int orc_exact_math;
void orc_set_exact_math(int on) { orc_exact_math = on; }
static float orc_expf(float x) { return orc_exact_math ? (float)exp((double)x) : expf(x); }
static float orc_tanhf(float x) { return orc_exact_math ? (float)tanh((double)x) : tanhf(x); }

static float orc_sigmoid(float v) { return 1.0f / (1.0f + expf(-v)); }
static float orc_silu(float v) { return v / (1.0f + orc_expf(-v)); } /* src/model.c:501 */

/* src/model.c:505-509 waste_situ_pair (K3's SiTU): beta*tanh(g/beta)*sigmoid(g),
 * times lbeta*tanh(u/lbeta) (or u when lbeta <= 0). */
float orc_situ_pair(float g, float u, float beta, float lbeta)
{
    const float a = beta * orc_tanhf(g / beta) / (1.0f + orc_expf(-g));
    return a * (lbeta > 0.0f ? lbeta * orc_tanhf(u / lbeta) : u);
}

/* The layer's gated activation: SiLU(g)*u, or SiTU when the model sets
 * act_situ (src/model.c:2900-2904, :2658-2660, :3646-3650, :3687). */
static float orc_act(const orc_moe *L, float g, float u)
{
    return L->act_situ ? orc_situ_pair(g, u, L->situ_beta, L->situ_lbeta) : orc_silu(g) * u;
}

/* src/model.c:2724-2747. */
void orc_route(const float *sc, const float *bias, int E, int K, int renorm,
               float routed_scale, int *idx, float *w)
{
    float *score = (float *)malloc((size_t)E * sizeof(float));
    for (int e = 0; e < E; e++) score[e] = orc_sigmoid(sc[e]);
    for (int j = 0; j < K; j++) {
        int best = -1;
        float bv = -1e30f;
        for (int e = 0; e < E; e++) {
            int taken = 0;
            for (int p = 0; p < j; p++)
                if (idx[p] == e) { taken = 1; break; }
            if (taken) continue;
            const float v = score[e] + (bias ? bias[e] : 0.0f);
            if (v > bv) { bv = v; best = e; }
        }
        idx[j] = best;
        w[j] = score[best];
    }
    if (renorm && K > 1) {
        float s = 0;
        for (int j = 0; j < K; j++) s += w[j];
        for (int j = 0; j < K; j++) w[j] /= (s + 1e-20f);
    }
    for (int j = 0; j < K; j++) w[j] *= routed_scale;
    free(score);
}

/* src/model.c:265-320, portable branch: per group, part = sum w*x in index
 * order, then acc += f16(scale) * part. */
void orc_mvq_rows(float *y, const int8_t *W, const uint16_t *ws, const float *x,
                  int rows, int in, int g, int bits, size_t rowbytes)
{
    const int ng = (in + g - 1) / g;
    int8_t *unp = (int8_t *)malloc((size_t)g);
    for (int o = 0; o < rows; o++) {
        const int8_t *row = W + (size_t)o * rowbytes;
        const uint16_t *s = ws + (size_t)o * ng;
        float acc = 0;
        for (int k = 0; k < ng; k++) {
            const int8_t *w;
            if (bits == 3) {
                /* src/simd.h:69-74 waste_q3_at over the row's bitstream */
                const uint8_t *p3 = (const uint8_t *)row;
                for (int i = 0; i < g; i++) {
                    const long off = ((long)k * g + i) * 3;
                    const int v = (p3[off >> 3] >> (off & 7)) | (p3[(off >> 3) + 1] << (8 - (off & 7)));
                    unp[i] = (int8_t)((v & 7) - 4);
                }
                w = unp;
            } else if (bits == 4) {
                const uint8_t *p4 = (const uint8_t *)row + (size_t)k * g / 2;
                for (int i = 0; i < g / 2; i++) {
                    unp[2 * i] = (int8_t)((p4[i] & 0x0F) - 8);
                    unp[2 * i + 1] = (int8_t)((p4[i] >> 4) - 8);
                }
                w = unp;
            } else {
                w = row + (size_t)k * g;
            }
            const float *xx = x + (size_t)k * g;
            const int lim = (k * g + g <= in) ? g : in - k * g;
            float part = 0;
            for (int i = 0; i < lim; i++) part += (float)w[i] * xx[i];
            acc += orc_f16(s[k]) * part;
        }
        y[o] = acc;
    }
    free(unp);
}

/* src/model.c:3366-3398 (mmq_rows, Q8G): dequantize the row, then dotf. */
static void orc_mmq_rows(float *Y, const int8_t *W, const uint16_t *ws,
                         const float *X, int out, int in, int T, int g,
                         size_t rowbytes)
{
    const int ng = (in + g - 1) / g;
    float *row = (float *)malloc((size_t)in * sizeof(float));
    for (int o = 0; o < out; o++) {
        const int8_t *q = W + (size_t)o * rowbytes;
        const uint16_t *sc = ws + (size_t)o * ng;
        for (int k = 0; k < ng; k++) {
            const float s = orc_f16(sc[k]);
            const int lim = (k * g + g <= in) ? g : in - k * g;
            for (int i = 0; i < lim; i++)
                row[k * g + i] = (float)q[(size_t)k * g + i] * s;
        }
        for (int t = 0; t < T; t++)
            Y[(size_t)t * out + o] = orc_dotf(row, X + (size_t)t * in, in);
    }
    free(row);
}

static const orc_hdr *rec_hdr(const orc_moe *L, int e)
{
    return (const orc_hdr *)(L->bank + (size_t)e * L->rec_bytes);
}

/* src/model.c:1698-1745 without the optional crc32. */
int orc_record_check(const orc_moe *L, int layer, int expert)
{
    const orc_hdr *h = rec_hdr(L, expert);
    const size_t rb = L->rec_bytes;
    if (rb < sizeof *h || h->magic != ORC_MAGIC_EXPERT) return -1;
    if (h->layer != (uint16_t)layer || h->expert_id != (uint16_t)expert) return -1;
    if ((size_t)h->rec_4k_blocks * ORC_ALIGN != rb) return -1;
    if (L->index_bits == 6 ? h->fmt != ORC_WQ_VQ4P
                           : (h->fmt != ORC_WQ_VQ3R && h->fmt != ORC_WQ_VQ2R))
        return -1;
    if (h->lowrank_id != 0) return -1;
    if ((long)h->codebook_id + 3L * L->stages > L->n_books) return -1;
    if (!(h->gate_off == sizeof *h && h->gate_off < h->up_off &&
          h->up_off < h->down_off && h->down_off < h->chan_corr_off &&
          h->chan_corr_off <= rb))
        return -1;
    const size_t scales = 2u * (size_t)(2 * L->inter + L->hidden);
    if (scales > rb - h->chan_corr_off) return -1;
    return 0;
}

/* src/model.c:2264-2280 vq_apply in the layer's format. For VQ4P the table
 * is quantised here; the engine quantises once when it builds the table
 * (vq_build_lut), which gives the same bytes. */
static void orc_apply(const orc_moe *L, float *y, const uint8_t *idx, const uint16_t *sc,
                      const float *lut, int M, int nv)
{
    if (L->index_bits == 6) {
        int8_t *q = (int8_t *)malloc((size_t)nv * 4 * 64);
        float *qs = (float *)malloc((size_t)(nv / ORC_LUT_BLK + 2) * sizeof(float));
        orc_vq4p_quant(lut, nv, q, qs);
        orc_vq4p_rows(y, idx, sc, q, qs, M, nv);
        free(q);
        free(qs);
    } else {
        orc_vq_rows(y, idx, sc, lut, M, nv, L->stages, L->entries);
    }
}

/* The serial expert loop of src/model.c:2873-2911: gate/up tables built
 * once from the first routed expert's codebook_id, then per expert gate,
 * up, SiLU(g)*u, down (its own table), and ysum += w[j]*acc in j order. */
int orc_moe_experts(const orc_moe *L, const int *idx, const float *w, int K,
                    const float *x, float *ysum, int fma)
{
    const int lat = L->hidden, inter = L->inter, st = L->stages;
    const int en = L->entries, vd = L->vec_dim;
    const size_t lut_sz = (size_t)((lat > inter ? lat : inter) / vd) * st * en;
    float *lut_g = (float *)malloc(lut_sz * sizeof(float));
    float *lut_u = (float *)malloc(lut_sz * sizeof(float));
    float *lut_d = (float *)malloc(lut_sz * sizeof(float));
    float *ga = (float *)malloc((size_t)inter * sizeof(float));
    float *ub = (float *)malloc((size_t)inter * sizeof(float));
    float *acc = (float *)malloc((size_t)lat * sizeof(float));
    memset(ysum, 0, (size_t)lat * sizeof(float));
    int lut_ready = 0;
    for (int j = 0; j < K; j++) {
        const uint8_t *rec = L->bank + (size_t)idx[j] * L->rec_bytes;
        const orc_hdr *h = (const orc_hdr *)rec;
        const uint16_t *sc = (const uint16_t *)(rec + h->chan_corr_off);
        if (!lut_ready) {
            orc_lut_build(lut_g, L->books, h->codebook_id + 0 * st, x, lat / vd,
                          st, en, vd, fma);
            orc_lut_build(lut_u, L->books, h->codebook_id + 1 * st, x, lat / vd,
                          st, en, vd, fma);
            lut_ready = 1;
        }
        orc_apply(L, ga, rec + h->gate_off, sc, lut_g, inter, lat / vd);
        orc_apply(L, ub, rec + h->up_off, sc + inter, lut_u, inter, lat / vd);
        for (int i = 0; i < inter; i++) ga[i] = orc_act(L, ga[i], ub[i]);
        orc_lut_build(lut_d, L->books, h->codebook_id + 2 * st, ga, inter / vd, st, en, vd,
                      fma);
        orc_apply(L, acc, rec + h->down_off, sc + 2 * inter, lut_d, lat, inter / vd);
        const float wj = w[j];
        for (int i = 0; i < lat; i++) ysum[i] += wj * acc[i];
    }
    free(lut_g); free(lut_u); free(lut_d); free(ga); free(ub); free(acc);
    return 0;
}

/* src/model.c:2651-2666 with accum=0, then src/model.c:2939 out += tmp. */
static void orc_shared_ffn(const orc_moe *L, const float *x, float *out)
{
    const int si = L->shared_inter, hid = L->hidden, g = L->sh_group;
    float *a = (float *)malloc((size_t)si * sizeof(float));
    float *b = (float *)malloc((size_t)si * sizeof(float));
    float *tmp = (float *)malloc((size_t)hid * sizeof(float));
    const size_t rb_in = (size_t)((hid + g - 1) / g) * g * (L->sh_bits == 4 ? 1 : 2) / 2;
    const size_t rb_si = (size_t)((si + g - 1) / g) * g * (L->sh_bits == 4 ? 1 : 2) / 2;
    orc_mvq_rows(a, L->sh_gate, L->sh_gate_s, x, si, hid, g, L->sh_bits, rb_in);
    orc_mvq_rows(b, L->sh_up, L->sh_up_s, x, si, hid, g, L->sh_bits, rb_in);
    for (int i = 0; i < si; i++) a[i] = orc_act(L, a[i], b[i]);
    orc_mvq_rows(tmp, L->sh_down, L->sh_down_s, a, hid, si, g, L->sh_bits, rb_si);
    for (int i = 0; i < hid; i++) out[i] += tmp[i];
    free(a); free(b); free(tmp);
}

/* src/model.c:2713-2939 for a model without a latent projection. */
int orc_moe_layer(const orc_moe *L, int layer, const float *x, float *out,
                  int *idx_out, float *w_out, int fma)
{
    const int E = L->n_experts, K = L->top_k, hid = L->hidden;
    float *logits = (float *)malloc((size_t)E * sizeof(float));
    int idx[64];
    float w[64];
    (void)layer;
    for (int e = 0; e < E; e++)
        logits[e] = orc_dotf(L->router + (size_t)e * hid, x, hid);
    orc_route(logits, L->bias, E, K, L->renorm, L->routed_scale, idx, w);
    free(logits);
    for (int j = 0; j < K; j++)
        if (orc_record_check(L, layer, idx[j])) return -1;
    orc_moe_experts(L, idx, w, K, x, out, fma);
    if (idx_out) memcpy(idx_out, idx, (size_t)K * sizeof(int));
    if (w_out) memcpy(w_out, w, (size_t)K * sizeof(float));
    if (L->shared_inter > 0) orc_shared_ffn(L, x, out);
    return 0;
}

/* src/model.c:3512-3693 for a model without a latent projection: route every
 * token, visit the distinct experts in ascending id, and add each (token,
 * expert) contribution as it comes; the shared FFN is the batched
 * dequantize-then-dot of mmq_rows (Q8G). */
int orc_moe_chunk(const orc_moe *L, int layer, const float *x, int nT,
                  float *out, int *route_out, float *rw_out, int fma)
{
    const int E = L->n_experts, K = L->top_k, hid = L->hidden, lat = hid;
    const int inter = L->inter, st = L->stages, en = L->entries, vd = L->vec_dim;
    int *route = (int *)malloc((size_t)nT * K * sizeof(int));
    float *rw = (float *)malloc((size_t)nT * K * sizeof(float));
    float *logits = (float *)malloc((size_t)E * sizeof(float));
    for (int t = 0; t < nT; t++) {
        for (int e = 0; e < E; e++)
            logits[e] = orc_dotf(L->router + (size_t)e * hid, x + (size_t)t * hid, hid);
        orc_route(logits, L->bias, E, K, L->renorm, L->routed_scale,
                  route + (size_t)t * K, rw + (size_t)t * K);
    }
    free(logits);
    const size_t lut_sz = (size_t)((hid > inter ? hid : inter) / vd) * st * en;
    float *lut_gu = (float *)malloc((size_t)nT * 2 * lut_sz * sizeof(float));
    float *lut_d = (float *)malloc(lut_sz * sizeof(float));
    float *ga = (float *)malloc((size_t)inter * sizeof(float));
    float *ub = (float *)malloc((size_t)inter * sizeof(float));
    float *acc = (float *)malloc((size_t)lat * sizeof(float));
    float *ysum = (float *)calloc((size_t)nT * lat, sizeof(float));
    int lut_ready = 0, rc = 0;
    for (int e = 0; e < E; e++) {
        int used = 0;
        for (int i = 0; i < nT * K; i++)
            if (route[i] == e) { used = 1; break; }
        if (!used) continue;
        if (orc_record_check(L, layer, e)) { rc = -1; break; }
        const uint8_t *rec = L->bank + (size_t)e * L->rec_bytes;
        const orc_hdr *h = (const orc_hdr *)rec;
        const uint16_t *s16 = (const uint16_t *)(rec + h->chan_corr_off);
        if (!lut_ready) {
            for (int t = 0; t < nT; t++) {
                orc_lut_build(lut_gu + (size_t)(2 * t) * lut_sz, L->books,
                              h->codebook_id + 0 * st, x + (size_t)t * lat,
                              lat / vd, st, en, vd, fma);
                orc_lut_build(lut_gu + (size_t)(2 * t + 1) * lut_sz, L->books,
                              h->codebook_id + 1 * st, x + (size_t)t * lat,
                              lat / vd, st, en, vd, fma);
            }
            lut_ready = 1;
        }
        for (int t = 0; t < nT; t++) {
            float wj = 0;
            for (int j = 0; j < K; j++)
                if (route[(size_t)t * K + j] == e) { wj = rw[(size_t)t * K + j]; break; }
            if (wj == 0.0f) continue;
            orc_apply(L, ga, rec + h->gate_off, s16, lut_gu + (size_t)(2 * t) * lut_sz, inter,
                      lat / vd);
            orc_apply(L, ub, rec + h->up_off, s16 + inter,
                      lut_gu + (size_t)(2 * t + 1) * lut_sz, inter, lat / vd);
            for (int i = 0; i < inter; i++) ga[i] = orc_act(L, ga[i], ub[i]);
            orc_lut_build(lut_d, L->books, h->codebook_id + 2 * st, ga, inter / vd, st, en,
                          vd, fma);
            orc_apply(L, acc, rec + h->down_off, s16 + 2 * inter, lut_d, lat, inter / vd);
            float *dst = ysum + (size_t)t * lat;
            for (int i = 0; i < lat; i++) dst[i] += wj * acc[i];
        }
    }
    memcpy(out, ysum, (size_t)nT * hid * sizeof(float));
    if (L->shared_inter > 0 && L->sh_bits == 8) {
        const int si = L->shared_inter, g = L->sh_group;
        float *sa = (float *)malloc((size_t)nT * si * sizeof(float));
        float *sb = (float *)malloc((size_t)nT * si * sizeof(float));
        float *sh = (float *)malloc((size_t)nT * hid * sizeof(float));
        const size_t rb_in = (size_t)((hid + g - 1) / g) * g;
        const size_t rb_si = (size_t)((si + g - 1) / g) * g;
        orc_mmq_rows(sa, L->sh_gate, L->sh_gate_s, x, si, hid, nT, g, rb_in);
        orc_mmq_rows(sb, L->sh_up, L->sh_up_s, x, si, hid, nT, g, rb_in);
        for (int i = 0; i < nT * si; i++) sa[i] = orc_act(L, sa[i], sb[i]);
        orc_mmq_rows(sh, L->sh_down, L->sh_down_s, sa, hid, si, nT, g, rb_si);
        for (int i = 0; i < nT * hid; i++) out[i] += sh[i];
        free(sa); free(sb); free(sh);
    }
    if (route_out) memcpy(route_out, route, (size_t)nT * K * sizeof(int));
    if (rw_out) memcpy(rw_out, rw, (size_t)nT * K * sizeof(float));
    free(route); free(rw); free(lut_gu); free(lut_d); free(ga); free(ub);
    free(acc); free(ysum);
    return rc;
}

/* src/model.c:132-138 waste_rmsnorm: s accumulated serially in fp32, then
 * r = 1 / sqrtf(s / n + eps), o[i] = (x[i] * r) * w[i]. */
void orc_rmsnorm(float *o, const float *x, const float *w, int n, float eps)
{
    float s = 0.0f;
    for (int i = 0; i < n; i++) s += x[i] * x[i];
    const float r = 1.0f / sqrtf(s / (float)n + eps);
    for (int i = 0; i < n; i++) o[i] = x[i] * r * w[i];
}

/* The MoE half of a decoder layer, src/model.c:3927-3945 (no attention
 * residuals): norm = rmsnorm(h, post_attention_layernorm), resid =
 * moe_layer(norm), h_out[i] = h[i] + resid[i]. */
int orc_moe_block(const orc_moe *L, int layer, const float *h, const float *norm_w,
                  float eps, float *h_out, int *idx_out, float *w_out, int fma)
{
    const int hid = L->hidden;
    float *norm = (float *)malloc((size_t)hid * sizeof(float));
    float *resid = (float *)malloc((size_t)hid * sizeof(float));
    orc_rmsnorm(norm, h, norm_w, hid, eps);
    const int rc = orc_moe_layer(L, layer, norm, resid, idx_out, w_out, fma);
    if (!rc)
        for (int i = 0; i < hid; i++) h_out[i] = h[i] + resid[i];
    free(norm);
    free(resid);
    return rc;
}

/* ---- KDA (src/kda.c, the x86 scalar kernels; -ffp-contract=off keeps
 * every a += b * c a rounded multiply then a rounded add) ---------------- */

/* src/kda.c:19-24 l2_rnorm */
static float orc_l2_rnorm(const float *x, int n)
{
    float s = 0.0f;
    for (int i = 0; i < n; i++) s += x[i] * x[i];
    return 1.0f / sqrtf(s + 1e-12f);
}

/* src/kda.c:26-68 waste_kda_step: per head, q and k L2-normalised (q also
 * by K^-0.5); pass A decays the rows by exp(g) and forms u = S'^T k; the
 * delta d = beta (v - u); pass B adds k d^T and forms o = S^T q. */
void orc_kda_step(int H, int K, int V, const float *q, const float *k, const float *v,
                  const float *g_log, const float *beta, float *S, float *o, float *u)
{
    const float qscale = 1.0f / sqrtf((float)K);
    for (int h = 0; h < H; h++) {
        const float *qh = q + (size_t)h * K, *kh = k + (size_t)h * K;
        const float *vh = v + (size_t)h * V, *gh = g_log + (size_t)h * K;
        float *Sh = S + (size_t)h * K * V, *oh = o + (size_t)h * V;
        const float b = beta[h];
        const float qn = orc_l2_rnorm(qh, K) * qscale;
        const float kn = orc_l2_rnorm(kh, K);
        memset(u, 0, (size_t)V * sizeof(float));
        for (int kk = 0; kk < K; kk++) {
            float *row = Sh + (size_t)kk * V;
            const float d = orc_expf(gh[kk]);
            const float kv = kh[kk] * kn;
            for (int i = 0; i < V; i++) {
                row[i] *= d;
                u[i] += row[i] * kv;
            }
        }
        for (int i = 0; i < V; i++) u[i] = b * (vh[i] - u[i]);
        memset(oh, 0, (size_t)V * sizeof(float));
        for (int kk = 0; kk < K; kk++) {
            float *row = Sh + (size_t)kk * V;
            const float kv = kh[kk] * kn;
            const float qv = qh[kk] * qn;
            for (int i = 0; i < V; i++) {
                row[i] += u[i] * kv;
                oh[i] += row[i] * qv;
            }
        }
    }
}

/* src/kda.c:84-99 waste_short_conv_step: a causal depthwise conv over the
 * ring of the previous KS-1 inputs (oldest first) and this one, the ring
 * shifted, then SiLU. */
void orc_short_conv_step(int C, int KS, const float *w, const float *bias, float *ring,
                         const float *x, float *y)
{
    const int R = KS - 1;
    for (int c = 0; c < C; c++) {
        const float *wc = w + (size_t)c * KS;
        float *rc = ring + (size_t)c * R;
        float acc = bias ? bias[c] : 0.0f;
        for (int j = 0; j < R; j++) acc += rc[j] * wc[j];
        acc += x[c] * wc[R];
        for (int j = 0; j + 1 < R; j++) rc[j] = rc[j + 1];
        if (R > 0) rc[R - 1] = x[c];
        y[c] = acc / (1.0f + orc_expf(-acc));
    }
}

/* src/kda.c:101-111 waste_rmsnorm_gated: y = x * r * w * sigmoid(gate),
 * r = 1 / sqrt(mean(x^2) + eps), the sum serial. */
void orc_rmsnorm_gated(int C, const float *x, const float *gate, const float *weight, float eps,
                       float *y)
{
    float s = 0.0f;
    for (int i = 0; i < C; i++) s += x[i] * x[i];
    const float r = 1.0f / sqrtf(s / (float)C + eps);
    for (int i = 0; i < C; i++) {
        const float g = 1.0f / (1.0f + orc_expf(-gate[i]));
        y[i] = x[i] * r * weight[i] * g;
    }
}

/* ---- the converter's RVQ encoder (src/vq.c, the portable loops) ---------- */

/* src/vq.c:51-82 vq_step: the nearest entry (d = sum (v_j - e_j)^2 in j
 * order, strict <, first index wins), and the residual. */
static int orc_vq_step(const float *v, const float *C, int entries, int dim, float *resid)
{
    int best = 0;
    float bestd = INFINITY;
    for (int c = 0; c < entries; c++) {
        const float *e = C + (size_t)c * dim;
        float d = 0;
        for (int j = 0; j < dim; j++) {
            const float t = v[j] - e[j];
            d += t * t;
        }
        if (d < bestd) {
            bestd = d;
            best = c;
        }
    }
    for (int j = 0; j < dim; j++) resid[j] = v[j] - C[(size_t)best * dim + j];
    return best;
}

/* src/vq.c:84-105 vq_range / waste_vq_encode: every stage of every vector. */
void orc_vq_encode(const float *X, int n, const float *books, int stages, int entries, int dim,
                   uint8_t *out)
{
    float cur[64], nxt[64];
    for (int i = 0; i < n; i++) {
        for (int d = 0; d < dim; d++) cur[d] = X[(size_t)i * dim + d];
        for (int s = 0; s < stages; s++) {
            out[(size_t)i * stages + s] = (uint8_t)orc_vq_step(
                cur, books + (size_t)s * entries * dim, entries, dim, nxt);
            for (int d = 0; d < dim; d++) cur[d] = nxt[d];
        }
    }
}

/* src/vq.c:107-136 waste_vq_lloyd: assign, then double sums in vector
 * order and centroid = (float)(sum / count) for the non-empty clusters.
 * Returns their number (or -1 when out of memory). */
int orc_vq_lloyd(const float *X, int n, float *C, int entries, int dim)
{
    uint8_t *asg = (uint8_t *)malloc((size_t)n);
    double *sum = (double *)calloc((size_t)entries * dim, sizeof(double));
    long *cnt = (long *)calloc((size_t)entries, sizeof(long));
    if (!asg || !sum || !cnt) { free(asg); free(sum); free(cnt); return -1; }
    orc_vq_encode(X, n, C, 1, entries, dim, asg);
    for (int i = 0; i < n; i++) {
        const int a = asg[i];
        cnt[a]++;
        for (int d = 0; d < dim; d++) sum[(size_t)a * dim + d] += X[(size_t)i * dim + d];
    }
    int live = 0;
    for (int c = 0; c < entries; c++)
        if (cnt[c]) {
            live++;
            for (int d = 0; d < dim; d++)
                C[(size_t)c * dim + d] = (float)(sum[(size_t)c * dim + d] / (double)cnt[c]);
        }
    free(asg); free(sum); free(cnt);
    return live;
}
