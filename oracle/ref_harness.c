/*
 * ref_harness.c — exposes the reference engine's static hot-path functions
 * (vq_build_lut, vq_matvec, moe_layer, moe_chunk; sqliteai/warp
 * src/model.c) so that tests can pin the CPU restatement in vq3r_oracle.c
 * against the real thing, and bench.py can time the reference CPU path.
 *
 * TEST INFRASTRUCTURE ONLY. This translation unit #includes the reference's
 * own src/model.c, found through -I on the reference tree (oracle/Makefile);
 * nothing from the reference is copied into this repository. The build goes
 * to oracle/_ref/, which is never committed.
 *
 * The model struct is filled in by hand with exactly the fields the MoE
 * path reads (src/model.c:2713-2939 and 3512-3693); expert records are read
 * by the reference's own bank_fetch/record_check from a memfd.
 */
#include "model.c"

#include <sys/mman.h>

#include "waste.h"      /* waste_version */

/* Registration functions of the reference's backends (defined in
 * src/kda.c, src/simd_avx2.c, src/simd_avx512.c; declared only inside
 * src/backend.c, so declared again here). */
const char *waste_kda_register_cpu(waste_kernels *t);
const char *waste_register_avx2(waste_kernels *t);
const char *waste_register_avx512(waste_kernels *t);

/* Backend selection. 0: the portable slots (what WASTE_BACKEND=cpu runs,
 * src/kda.c:118-128). 1: AVX-512 (src/simd_avx512.c:125-130). 2: AVX2. */
const char *refh_set_backend(int which)
{
    waste_backend_init(WASTE_BE_FORCE_CPU | WASTE_BE_NO_DEVICE);
    const char *n = waste_kda_register_cpu(&waste_k);
#if defined(__x86_64__)
    const uint32_t f = waste_cpu_features();
    if (which == 1 && (f & WASTE_CPU_AVX512F) && (f & WASTE_CPU_AVX512BW))
        n = waste_register_avx512(&waste_k);
    else if (which == 2 && (f & WASTE_CPU_AVX2) && (f & WASTE_CPU_FMA))
        n = waste_register_avx2(&waste_k);
    else if (which != 0)
        return NULL;
#else
    if (which != 0) return NULL;
#endif
    return n;
}

/* The best backend waste_backend_init would pick here, as an int for
 * refh_set_backend: 1 when AVX-512 is usable, 2 for AVX2, else 0. */
int refh_best_backend(void)
{
#if defined(__x86_64__)
    const uint32_t f = waste_cpu_features();
    if ((f & WASTE_CPU_AVX512F) && (f & WASTE_CPU_AVX512BW)) return 1;
    if ((f & WASTE_CPU_AVX2) && (f & WASTE_CPU_FMA)) return 2;
#endif
    return 0;
}

void refh_pool_init(int nthreads) { waste_pool_init(nthreads, NULL); }
int refh_pool_threads(void) { return waste_pool_threads(); }
const char *refh_version(void) { return waste_version(); }

/* The engine's codebook decode (src/model.c:1269-1304) runs inside
 * waste_model_load, so it is reached by loading a container: these load
 * one, hand back the decoded codebooks (m->codebooks, [n_books][256][8]),
 * and free it. */
void *refh_load(const char *dir)
{
    waste_model *m = (waste_model *)calloc(1, sizeof *m);
    waste_load_opts o;
    memset(&o, 0, sizeof o);
    o.n_threads = 1;
    if (waste_model_load(m, dir, 64, &o)) { free(m); return NULL; }
    return m;
}

const float *refh_codebooks(void *p, int *n_books)
{
    const waste_model *m = (const waste_model *)p;
    if (n_books) *n_books = m->n_books;
    return m->codebooks;
}

void refh_free(void *p)
{
    waste_model_free((waste_model *)p);
    free(p);
}

static float *transpose_books(const float *books, int n_books, int en, int vd)
{
    float *T = (float *)malloc((size_t)n_books * en * vd * sizeof(float));
    for (int b = 0; b < n_books; b++)
        for (int c = 0; c < en; c++)
            for (int d = 0; d < vd; d++)
                T[((size_t)b * vd + d) * en + c] = books[((size_t)b * en + c) * vd + d];
    return T;
}

/* lut[nv][stages][entries] through the live waste_k.lutb_range slot. */
void refh_lutb(float *lut, const float *books, int n_books, int cb_base,
               const float *x, int nv, int stages, int entries, int vd)
{
    float *T = transpose_books(books, n_books, entries, vd);
    lutb_arg a = { lut, T, x, cb_base, stages, entries, vd };
    waste_k.lutb_range(0, nv, &a);
    free(T);
}

static waste_model *mk_model(const float *books, int n_books, int stages,
                             int entries, int vd)
{
    waste_model *m = (waste_model *)calloc(1, sizeof *m);
    m->codebooks = (float *)malloc((size_t)n_books * entries * vd * sizeof(float));
    memcpy(m->codebooks, books, (size_t)n_books * entries * vd * sizeof(float));
    m->codebooksT = transpose_books(books, n_books, entries, vd);
    m->n_books = n_books;
    m->vec_dim = vd;
    m->cb_entries = entries;
    m->stages = stages;
    m->index_bits = 8;
    pthread_mutex_init(&m->fetch_mu, NULL);
    return m;
}

/* src/model.c:2282 vq_matvec, through the thread pool. */
void refh_vq_matvec(float *y, const uint8_t *idx, const uint16_t *scale,
                    const float *x, int M, int N, const float *books,
                    int n_books, int cb_base, int stages, int entries, int vd)
{
    waste_model *m = mk_model(books, n_books, stages, entries, vd);
    float *lut = (float *)malloc((size_t)(N / vd) * stages * entries * sizeof(float));
    vq_matvec(m, y, idx, scale, x, M, N, cb_base, lut, NULL, NULL);
    free(lut);
    free(m->codebooks); free(m->codebooksT); free(m);
}

/* src/model.c:2282 vq_matvec on a VQ4P matrix (index_bits 6: four stages of
 * 64 entries, packed indices): books [n_books][64][8]. */
void refh_vq4p_matvec(float *y, const uint8_t *idx, const uint16_t *scale,
                      const float *x, int M, int N, const float *books,
                      int n_books, int cb_base)
{
    waste_model *m = mk_model(books, n_books, 4, 64, 8);
    m->index_bits = 6;
    const int nv = N / 8;
    float *lut = (float *)malloc((size_t)nv * 4 * 64 * sizeof(float));
    int8_t *q = (int8_t *)malloc((size_t)nv * 4 * 64);
    float *qs = (float *)malloc((size_t)(nv / WASTE_VQ_LUT_BLK + 2) * sizeof(float));
    vq_matvec(m, y, idx, scale, x, M, N, cb_base, lut, q, qs);
    free(lut); free(q); free(qs);
    free(m->codebooks); free(m->codebooksT); free(m);
}

/* src/model.c:1911-1923 vq_build_lut with the int8 shadow (vq_quant_lut):
 * q [N/8][4][64], qs [ceil(N/256)]. */
void refh_vq4p_table(int8_t *q, float *qs, const float *x, int N, const float *books,
                     int n_books, int cb_base)
{
    waste_model *m = mk_model(books, n_books, 4, 64, 8);
    m->index_bits = 6;
    float *lut = (float *)malloc((size_t)(N / 8) * 4 * 64 * sizeof(float));
    vq_build_lut(m, lut, cb_base, x, N, 4, 64, 8, q, qs);
    free(lut);
    free(m->codebooks); free(m->codebooksT); free(m);
}

/* A reusable handle for repeated matvec timing: same as refh_vq_matvec but
 * with the model and table allocated once. */
typedef struct { waste_model *m; float *lut; int N; } refh_mv;

void *refh_mv_open(const float *books, int n_books, int stages, int entries,
                   int vd, int Nmax)
{
    refh_mv *h = (refh_mv *)calloc(1, sizeof *h);
    h->m = mk_model(books, n_books, stages, entries, vd);
    h->lut = (float *)malloc((size_t)(Nmax / vd) * stages * entries * sizeof(float));
    h->N = Nmax;
    return h;
}

void refh_mv_run(void *p, float *y, const uint8_t *idx, const uint16_t *scale,
                 const float *x, int M, int N, int cb_base)
{
    refh_mv *h = (refh_mv *)p;
    vq_matvec(h->m, y, idx, scale, x, M, N, cb_base, h->lut, NULL, NULL);
}

void refh_mv_close(void *p)
{
    refh_mv *h = (refh_mv *)p;
    free(h->lut); free(h->m->codebooks); free(h->m->codebooksT); free(h->m);
    free(h);
}

/* ---- one MoE layer ------------------------------------------------------ */

typedef struct {
    waste_model *m;
    int layer;
} refh_moe;

static void add_tensor(waste_model *m, int *n, const char *name)
{
    snprintf(m->t[*n].name, sizeof m->t[*n].name, "%s", name);
    (*n)++;
}

/* Builds a model holding one MoE layer `layer` (Kimi-Linear form: no
 * latent projection, SiLU, sigmoid router with optional bias, renorm and
 * routed scale), whose bank is `n_experts` records of rec_bytes copied into
 * a memfd and read back by the reference's bank_fetch. The shared expert is
 * Q8G (group 128) when sh_inter > 0. Chunk scratch for up to max_tokens. */
void *refh_moe_open(int layer, int hidden, int inter, int n_experts, int top_k,
                    int renorm, float routed_scale, const float *router,
                    const float *bias, const float *books, int n_books,
                    int cb_base, const void *bank, size_t rec_bytes,
                    int sh_inter, const int8_t *shg, const uint16_t *shg_s,
                    const int8_t *shu, const uint16_t *shu_s,
                    const int8_t *shd, const uint16_t *shd_s, int max_tokens,
                    int index_bits)
{
    /* index_bits 6: a VQ4P bank (four stages of 64-entry books) */
    const int st = index_bits == 6 ? 4 : 3, en = index_bits == 6 ? 64 : 256, vd = 8, g = 128;
    waste_model *m = mk_model(books, n_books, st, en, vd);
    m->index_bits = index_bits == 6 ? 6 : 8;
    waste_config *c = &m->cfg;
    c->n_layers = layer + 1;
    c->hidden = hidden;
    c->n_experts = n_experts;
    c->top_k = top_k;
    c->moe_inter = inter;
    /* the engine sizes the shared FFN as moe_inter * n_shared
     * (src/model.c:2938), so the shared width must be a multiple of it */
    if (sh_inter > 0 && sh_inter % inter) return NULL;
    c->n_shared = sh_inter > 0 ? sh_inter / inter : 1;
    c->first_dense = layer;
    c->renorm = renorm;
    c->routed_scale = routed_scale;
    c->eps = 1e-5f;

    m->t = (waste_tensor *)calloc(8, sizeof(waste_tensor));
    int n = 0;
    char nm[160];
    snprintf(nm, sizeof nm, "model.layers.%d.block_sparse_moe.gate.weight", layer);
    m->t[n].data = (float *)router;
    m->t[n].shape[0] = n_experts; m->t[n].shape[1] = hidden; m->t[n].ndim = 2;
    add_tensor(m, &n, nm);
    if (bias) {
        snprintf(nm, sizeof nm,
                 "model.layers.%d.block_sparse_moe.gate.e_score_correction_bias", layer);
        m->t[n].data = (float *)bias;
        m->t[n].shape[0] = n_experts; m->t[n].ndim = 1;
        add_tensor(m, &n, nm);
    }
    if (sh_inter > 0) {
        const char *kinds[3] = { "gate_proj", "up_proj", "down_proj" };
        const int8_t *q[3] = { shg, shu, shd };
        const uint16_t *qs[3] = { shg_s, shu_s, shd_s };
        const int rows[3] = { sh_inter, sh_inter, hidden };
        const int cols[3] = { hidden, hidden, sh_inter };
        for (int k = 0; k < 3; k++) {
            snprintf(nm, sizeof nm,
                     "model.layers.%d.block_sparse_moe.shared_experts.%s.weight",
                     layer, kinds[k]);
            waste_tensor *t = &m->t[n];
            t->q = (int8_t *)q[k];
            t->qs = (uint16_t *)qs[k];
            t->group = g;
            t->bits = 8;
            t->rowbytes = (size_t)((cols[k] + g - 1) / g) * g;
            t->shape[0] = rows[k]; t->shape[1] = cols[k]; t->ndim = 2;
            add_tensor(m, &n, nm);
        }
    }
    m->n_tensors = n;

    const int fd = memfd_create("refh_bank", 0);
    const size_t total = rec_bytes * (size_t)n_experts;
    size_t off = 0;
    while (off < total) {
        const ssize_t w = write(fd, (const char *)bank + off, total - off);
        if (w <= 0) return NULL;
        off += (size_t)w;
    }
    m->bank[layer].fd = fd;
    m->bank[layer].rec_bytes = (int64_t)rec_bytes;
    m->bank[layer].n_experts = n_experts;
    m->bank[layer].cb_base = cb_base;
    m->expert_m[0] = m->expert_m[1] = inter;
    m->expert_n[0] = m->expert_n[1] = hidden;
    m->expert_m[2] = hidden;
    m->expert_n[2] = inter;
    m->miss_buf = (uint8_t *)malloc(rec_bytes);

    const int si = sh_inter > inter ? sh_inter : inter;
    const int nmax = hidden > inter ? hidden : inter;
    const size_t lut_sz = (size_t)(nmax / vd + 1) * st * en;
    m->att = (float *)calloc((size_t)WASTE_ATT_ROUTER_OFF + 2 * n_experts + 64, sizeof(float));
    m->ff = (float *)calloc((size_t)2 * si, sizeof(float));
    m->e_gate = (float *)calloc((size_t)hidden, sizeof(float));
    m->h = (float *)calloc((size_t)hidden, sizeof(float));
    m->ares = (float *)calloc((size_t)4 * hidden, sizeof(float));
    m->lut = (float *)malloc(3 * lut_sz * sizeof(float));

    const int T = max_tokens > 0 ? max_tokens : 1;
    m->croute = (int *)calloc((size_t)T * top_k, sizeof(int));
    m->crw = (float *)calloc((size_t)T * top_k, sizeof(float));
    m->cused = (int *)calloc((size_t)T * 64 + n_experts, sizeof(int));
    m->cq = (float *)malloc((size_t)(2 * T + 1) * lut_sz * sizeof(float));
    m->cff = (float *)calloc((size_t)2 * inter + hidden, sizeof(float));
    if (m->index_bits == 6) {
        /* the int8 shadows of m->lut and m->cq, region for region */
        const size_t nsc = (size_t)(nmax / vd + 1) / WASTE_VQ_LUT_BLK + 2;
        m->lut8 = (int8_t *)malloc(3 * lut_sz);
        m->lut8_scale = (float *)malloc(3 * nsc * sizeof(float));
        m->cq8 = (int8_t *)malloc((size_t)(2 * T + 1) * lut_sz);
        m->cq8_scale = (float *)malloc((size_t)(2 * T + 1) * nsc * sizeof(float));
    }
    m->clat = (float *)calloc((size_t)2 * T * hidden, sizeof(float));
    m->ckv = (float *)calloc((size_t)T * (2 * si + hidden), sizeof(float));
    m->chunk_cap = T;

    refh_moe *h = (refh_moe *)calloc(1, sizeof *h);
    h->m = m;
    h->layer = layer;
    return h;
}

/* The model's gated activation (src/model.c:987-990): act_situ selects
 * waste_situ_pair (K3) in place of SiLU, with its two betas. */
void refh_moe_set_act(void *p, int act_situ, float beta, float linear_beta)
{
    refh_moe *h = (refh_moe *)p;
    h->m->cfg.act_situ = act_situ;
    h->m->cfg.situ_beta = beta;
    h->m->cfg.situ_linear_beta = linear_beta;
}

/* src/model.c:2713 moe_layer. Returns 0, or the sticky read error code. */
int refh_moe_layer(void *p, const float *x, float *out, int *routed)
{
    refh_moe *h = (refh_moe *)p;
    h->m->read_error = 0;
    moe_layer(h->m, h->layer, x, out, routed);
    return h->m->read_error;
}

/* src/model.c:3512 moe_chunk; route/rw receive croute/crw ([nT][K]). */
int refh_moe_chunk(void *p, const float *x, int nT, float *out, int *route,
                   float *rw)
{
    refh_moe *h = (refh_moe *)p;
    if (nT > h->m->chunk_cap) return -1;
    h->m->read_error = 0;
    moe_chunk(h->m, h->layer, x, out, nT);
    const int K = h->m->cfg.top_k;
    if (route) memcpy(route, h->m->croute, (size_t)nT * K * sizeof(int));
    if (rw) memcpy(rw, h->m->crw, (size_t)nT * K * sizeof(float));
    return h->m->read_error;
}

#if defined(WASTE_ENABLE_CUDA)
/* Built against the engine patched with this repository's CUDA backend
 * (integration/): the engine's own backend choice (src/backend.c:168-212)
 * with the CUDA backend compiled in, which registers it when an sm_100
 * device is present and fills the expert-path slots. */
const char *refh_backend_auto(void)
{
    waste_backend_init(WASTE_BE_AUTO);
    return waste_backend_name();
}

/* The patched loader's upload (wcu_upload) for a layer built here: the
 * codebooks and the bank go to HBM. Returns 1 when the expert-path slots
 * are live afterwards (moe_layer / moe_chunk run their experts on the
 * device), 0 when the backend declined. */
int refh_moe_upload(void *p)
{
    refh_moe *h = (refh_moe *)p;
    wcu_upload(h->m);
    return waste_vq.moe_experts != NULL;
}
#endif

void refh_moe_close(void *p)
{
    refh_moe *h = (refh_moe *)p;
    waste_model *m = h->m;
#if defined(WASTE_ENABLE_CUDA)
    wcu_release(m);
#endif
    close(m->bank[h->layer].fd);
    free(m->t); free(m->miss_buf); free(m->att); free(m->ff); free(m->e_gate);
    free(m->h); free(m->ares); free(m->lut); free(m->croute); free(m->crw);
    free(m->cused); free(m->cq); free(m->cff); free(m->clat); free(m->ckv);
    free(m->codebooks); free(m->codebooksT);
    free(m->lut8); free(m->lut8_scale); free(m->cq8); free(m->cq8_scale);
    pthread_mutex_destroy(&m->fetch_mu);
    free(m); free(h);
}
