/*
 * wc_launch.h — the shim between the plain-C host layer (waste_cuda.c) and
 * the CUDA kernels (vq3r_kernels.cu). Plain C structs of device pointers and
 * sizes; every launcher returns a cudaError_t as int (0 = launched).
 */
#ifndef WC_LAUNCH_H
#define WC_LAUNCH_H

#include <cuda.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Vector positions per gate/up and per down tile of the decode kernels.
 * The gate/up count depends on the expert width (wc_vs_gateup). */
#define WC_VS_GATEUP 4
#define WC_VS_DOWN   8
int wc_vs_gateup(int lat, int inter);

/* One layer's bank as the kernels see it: E records of rec_bytes each,
 * all with the same payload offsets (checked at load). tmap: TMA tensor
 * maps of the gate, up and down index streams over the bank, 8-byte
 * elements, dims {positions * 24, 64-row blocks, experts}; boxes of one
 * tile's positions by half the row blocks (gate/up) or all of them (down).
 * tmap_ok = 0 when the shapes do not fit the boxes (per-row-block copies
 * are used instead). */
typedef struct {
    CUtensorMap tmap[3];
    int tmap_ok;
    const uint8_t *base;
    size_t rec_bytes;
    uint32_t gate_off, up_off, down_off, scale_off;
    int n_experts, first;     /* records held: global ids [first, first+n) */
    int cb_base;              /* codebook_id shared by every record         */
    int inter, lat, stages;
} wc_bank;

/* The workspace a MoE launch writes; sized by wc_moe_ws_bytes. */
typedef struct {
    float *p_gu;       /* [T][2][ns_gu][K][inter] partial gate/up sums      */
    float *p_d;        /* [T][K][ns_d][lat] partial down sums               */
    float *logits;     /* [T][E]                                            */
    float *sh_g, *sh_u, *sh_h, *sh_out;   /* shared expert [T][si] / [T][hid] */
    float *h;          /* [T][K][inter] SiLU(g)*u, batched calls only        */
    float *xn;         /* [T][lat] rmsnorm(x), the MoE block only            */
    unsigned int *tickets;  /* [T] router blocks done; zero between launches   */
    unsigned int *route_flag;  /* [T] 1 once routing is published            */
    unsigned int *route_pass;  /* [T] gate/up tiles that have seen the flag   */
    unsigned int *x_flag;      /* [T] 1 once the router's dependency wait has
                                  passed: x is complete                        */
    unsigned int *sh_ticket;   /* [T] router blocks of the shared expert done */
    unsigned int *sh_flag;     /* [T] 1 once the shared activation is written */
    unsigned int *sh_pass;     /* [T] shared down blocks that have seen it     */
    unsigned int *err;         /* sticky device error bits (WC_ERR_*)         */
} wc_moe_ws;

/* Device error bits: a bounded wait that ran out, or a route naming an
 * expert the bank does not hold (skipped). */
#define WC_ERR_ROUTE_WAIT 1u
#define WC_ERR_TMA_WAIT   2u
#define WC_ERR_BAD_EXPERT 4u
#define WC_ERR_PEER_WAIT  8u          /* a peer's flag did not arrive in time */

/* Expert-parallel exchange through peer memory (NVLink). Every rank has a
 * mailbox of the same layout, mapped into every other rank's address
 * space:
 *   +0     x flags     [WC_EP_MAX] : epoch of rank r's tokens, set by r
 *   +256   part flags  [WC_EP_MAX] : epoch of rank r's partial sums, set by r
 *   +512   combine ticket (local use)
 *   +640   epoch counter (local use: bumped once per layer call)
 *   +768   poison word: set in every mailbox by a rank whose peer wait
 *          gave up; every later wait fails at once (ep_init clears it)
 *   +1024  x   [world][T][hidden]  : every rank's tokens
 *   then   part[world][T][hidden]  : every rank's partial sums of this
 *                                    rank's tokens
 * Flags only grow (epochs), so nothing is reset between calls.
 * With rep set, every rank holds the same T tokens: x is not copied (the x
 * flags still order one call after the last), and each rank's partial sums
 * go to every rank, so all of them finish with the full outputs. */
#define WC_EP_MAX 8
#define WC_EP_MAIL_HDR 1024
typedef struct {
    int on, rank, world, T, hidden, rep;
    int wait_polls;                   /* polls before a peer wait gives up  */
    unsigned char *mail[WC_EP_MAX];   /* every rank's mailbox as mapped here */
} wc_ep_link;

int wc_ep_publish_launch(const wc_ep_link *l, const float *x, unsigned int *err, void *stream);
int wc_ep_finalize_launch(const wc_ep_link *l, float *out, const float *resid,
                          unsigned int *err, void *stream);
/* out[i] = resid[i] + y[i], i < n (out may alias y). */
int wc_resid_add_launch(float *out, const float *resid, const float *y, size_t n, void *stream);

/* Up to four copies of 4-byte words in one launch, for the small per-call
 * transfers between pinned host memory (mapped into the device's address
 * space) and device buffers: a kernel's loads and stores cross the bus in
 * one round trip, where each copy-engine transfer costs its own setup.
 * Pointers 4-byte aligned, sizes multiples of 4. */
#define WC_COPY_MAX 4
typedef struct {
    void *dst[WC_COPY_MAX];
    const void *src[WC_COPY_MAX];
    size_t bytes[WC_COPY_MAX];
    int n;
    int pdl;           /* 1: launched programmatically behind the kernel that
                          wrote src (it waits for that kernel, not for the
                          launch boundary) */
} wc_copy_args;
int wc_copy_launch(const wc_copy_args *c, void *stream);

typedef struct {
    wc_bank bank;
    const float *books;       /* [n_books][256][8] fp32                      */
    int T, K;
    const float *x;           /* [T][lat]                                    */
    const int *idx;           /* [T][K] global expert ids                    */
    const float *w;           /* [T][K]                                      */
    float *out;               /* [T][lat]                                    */
    int order_by_id;          /* 1: per token, add experts in ascending id   */
    /* router + shared expert; router == NULL means idx/w are given */
    const float *router, *bias;
    int E, renorm;
    float routed_scale;
    int *idx_out;             /* written by the router when router != NULL   */
    float *w_out;
    int si;                   /* shared intermediate; 0 = no shared expert   */
    int sh_t0, sh_t1;         /* tokens [sh_t0, sh_t1) get the shared expert
                                 (all of them, unless expert parallel)       */
    int partial_bank;         /* 1: the bank holds only some experts; routes
                                 to the others are skipped, not computed      */
    int gu_eg;                /* gate/up experts per tile with a partial bank
                                 (0: all K of a token)                        */
    int act_pre;              /* set by the launcher: SiLU(g)*u computed once
                                 per (token, expert) before the down tiles    */
    wc_ep_link ep;            /* on: x comes from the mailbox, partial sums go
                                 to the tokens' ranks through peer memory    */
    const int8_t *shg, *shu, *shd;
    const uint16_t *shg_s, *shu_s, *shd_s;
    wc_moe_ws ws;
    /* The MoE half of a decoder layer (src/model.c:3927-3945): with norm_w
     * set, the router normalises x (rmsnorm, eps) and every kernel of the
     * layer works on that; with resid set, out = resid + the layer's output
     * (the residual add). */
    const float *norm_w;
    float norm_eps;
    const float *resid;
    /* the gated activation: 0 SiLU(g)*u, 1 SiTU with its two betas
     * (src/model.c:505-509) */
    int act;
    float situ_beta, situ_lbeta;
    /* L2 prefetching: the routed experts' down streams during gate/up, and
     * up to four caller ranges (16-byte aligned) during combine */
    int prefetch_down;
    const void *pf_ptr[4];
    size_t pf_bytes[4];
} wc_moe_args;

/* The workspace starts with this many control words (tickets, flags, pass
 * counters, the error word at 192), then the float arrays. */
#define WC_WS_CONTROL_WORDS 512

/* Floats of workspace for T tokens. The region must be zeroed once when it
 * is allocated (the ticket counters reset themselves after every launch). */
size_t wc_moe_ws_floats(int T, int K, int E, int lat, int inter, int si,
                        int stages);
void   wc_moe_ws_carve(wc_moe_ws *ws, float *base, int T, int K, int E, int lat,
                       int inter, int si, int stages);
int    wc_moe_launch(const wc_moe_args *a, void *stream);
/* 0 when the shapes in `a` are within the kernels' register-resident
 * bounds: every tile within 227 KB of shared memory, and for the whole layer
 * (device router) top-K <= 32 and experts <= 1024. */
int    wc_moe_supported(const wc_moe_args *a);

/* Batched matvec: G <= WC_MAX_G matrices of [M][N]. The pointer tables go
 * by value in the kernel parameters (4 KiB), so a launch needs no upload
 * and can be captured in a CUDA graph. */
#define WC_MAX_G 120
typedef struct {
    int G, M, N, stages, cb_base;
    const uint8_t *idx[WC_MAX_G];
    const uint16_t *scale[WC_MAX_G];
    const float *x[WC_MAX_G];
    float *y[WC_MAX_G];
    const float *books;
    float *part;              /* [G][ns][M] workspace                         */
    const uint32_t *sel[WC_MAX_G];   /* copy-select streams (matvec_sel.cu)   */
} wc_matvec_args;

size_t wc_matvec_part_floats(int G, int M, int N);
int    wc_matvec_launch(const wc_matvec_args *a, void *stream);
/* The reduce step alone: y[g][r] = f16(scale) * sum of the ns partials. */
int    wc_matvec_reduce_launch(const wc_matvec_args *a, int ns, void *stream);

/* The matvec with interleaved table copies (matvec_sel.cu): copies 2 or 4,
 * stages 3, rows 2049..8192 (one lane of quarter blocks per tile). The
 * copy-select stream of a matrix has wc_sel_words(M, N, copies) 32-bit
 * words and is written once by wc_sel_build_launch from its index stream. */
size_t wc_sel_words(int M, int N, int copies);
int    wc_sel_build_launch(const uint8_t *idx, uint32_t *sel, int M, int N, int stages,
                           int copies, void *stream);
int    wc_matvec_sel_launch(const wc_matvec_args *a, int copies, void *stream);

/* Fixed partial-sum scratch of the allocation-free matvec: a module-scope
 * device array of WC_NOALLOC_PART_FLOATS floats (32 MiB). wc_noalloc_part
 * looks up its address on the current device (cudaGetSymbolAddress; the
 * return is a cudaError_t). */
#define WC_NOALLOC_PART_FLOATS ((size_t)8 << 20)
int    wc_noalloc_part(float **ptr);
/* The same lookup plus loading the kernels the allocation-free matvec
 * launches, so a later call needs nothing brought onto the device. */
int    wc_noalloc_setup(float **ptr);
int    wc_binary_version(void);

/* VQ4P (vq4p.cu): four 64-entry stages, 6-bit indices packed four to three
 * bytes, int8 tables with one scale per 32 positions. The list form runs
 * G <= WC_MAX_G independent matvecs y[g] = VQ4P(idx[g], scale[g]) . x[g]
 * (book base cb[g]); the expert form runs the expert loop of T tokens over
 * a VQ4P bank: gate/up of every (token, slot) pair, the gated activation
 * into h, down, and the weighted reduce into ysum (router order, or
 * ascending expert id when order_by_id). part/ls are scratch of
 * wc_p6_part_ints / wc_p6_ls_floats elements for the larger of the two
 * phases (G = 2*T*K pairs of [inter][lat], or T*K of [lat][inter]). */
typedef struct {
    int G, M, N;
    const uint8_t *idx[WC_MAX_G];
    const uint16_t *scale[WC_MAX_G];
    const float *x[WC_MAX_G];
    float *y[WC_MAX_G];
    int cb[WC_MAX_G];
    const float *books;        /* [n_books][256][8] f32; a VQ4P book fills entries 0..63 */
    int *part;                 /* [problem][block][M] integer block sums             */
    float *ls;                 /* [problem][block] table scales                      */
    wc_bank bank;
    int T, K, order_by_id, act;
    float situ_beta, situ_lbeta;
    const int *route;          /* [T][K] global expert ids                           */
    const float *rw;           /* [T][K]                                             */
    const float *x_in;         /* [T][lat]                                           */
    float *h;                  /* [T*K][inter] activations                           */
    float *ysum;               /* [T][lat]                                           */
    unsigned int *err;
} wc_p6_args;

size_t wc_p6_part_ints(int G, int M, int N);
size_t wc_p6_ls_floats(int G, int N);
int    wc_p6_matvec_launch(const wc_p6_args *a, void *stream);
int    wc_p6_moe_launch(const wc_p6_args *a, void *stream);
/* The int8 tables of x against books cb..cb+3: q [nv][4][64], qs [blocks]. */
int    wc_p6_table_launch(int8_t *q, float *qs, const float *x, const float *books, int cb,
                          int nv, void *stream);

/* KDA (kda.cu): decode step, causal conv, gated rmsnorm (src/kda.c). With
 * pdl set, the step and the norm launch programmatically behind the kernel
 * before them on the stream: the step fetches its state before waiting on
 * that kernel; the norm lets the kernel behind it start at once. */
int wc_kda_supported(int K, int V);
int wc_kda_step_launch(int H, int K, int V, const float *q, const float *k, const float *v,
                       const float *g_log, const float *beta, float *S, float *o, void *stream,
                       int pdl);
int wc_short_conv_launch(int C, int KS, const float *w, const float *bias, float *ring,
                         const float *x, float *y, void *stream);
int wc_rmsnorm_gated_launch(int nh, int C, const float *x, const float *gate, const float *weight,
                            float eps, float *y, void *stream, int pdl);
/* The decay gate of H*D channels in place and beta = sigmoid(beta) [H]. */
int wc_kda_gate_launch(float *g, const float *A_log, const float *dt_bias, int H, int D,
                       float lower_bound, float *beta, void *stream);

/* The converter's residual-VQ encoder (vq_encode.cu, src/vq.c:50-136):
 * encode n vectors of dim against `stages` books of `entries` each (the
 * books in shared memory: wc_vq_encode_smem bytes); one Lloyd iteration
 * over n vectors with scratch of wc_vq_lloyd_scratch bytes, C updated in
 * place and the number of non-empty clusters written to d_live. */
size_t wc_vq_encode_smem(int stages, int entries, int dim);
int    wc_vq_encode_launch(const float *X, int n, const float *books, int stages, int entries,
                           int dim, uint8_t *out, void *stream);
size_t wc_vq_lloyd_scratch(int n, int entries, int dim);
int    wc_vq_lloyd_launch(const float *X, int n, float *C, int entries, int dim, void *scratch,
                          int *d_live, void *stream);

int wc_lutb_launch(float *lut, const float *x, const float *books, int cb_base,
                   int nv, int stages, void *stream);
int wc_dequant_launch(float *W, const uint8_t *idx, const uint16_t *scale,
                      int M, int N, const float *books, int cb_base, int stages,
                      void *stream);

/* Batched (prefill) expert path on the tensor cores (prefill_tc.cu): T
 * tokens, K routed experts each, route/rw [T][K], x/out [T][lat]; the
 * workspace arrays are sized by the host (wc_pf_max_tiles). */
#define WC_PF_MAX_PAIRS 65536
typedef struct {
    wc_bank bank;
    const float *books;
    int T, K;
    const int *route;
    const float *rw;
    const float *x;
    float *out;
    float wscale[3];          /* power-of-two pre-scales of gate, up, down weights */
    int *pairs;               /* [T*K] pair ids (t*K + j) grouped by expert      */
    int *tile_e, *tile_s, *tile_n, *ntiles;
    uint16_t *xh, *xl;        /* [T][lat] fp16 halves of x * 1/xinv              */
    float *xinv;              /* [T]                                             */
    float *gu;                /* [pairs][2][inter] gate, up (list order)         */
    uint16_t *hh, *hl;        /* [pairs][inter] fp16 halves of h * 1/hinv        */
    float *hinv;              /* [pairs]                                         */
    float *y;                 /* [T*K][lat] per pair, unweighted                 */
    unsigned int *err;
    int act;                  /* 0 SiLU(g)*u, 1 SiTU                             */
    float situ_beta, situ_lbeta;
} wc_pf_args;

int    wc_pf_supported(const wc_bank *b, int T, int K);
size_t wc_pf_max_tiles(int T, int K, int n_experts);
int    wc_pf_launch(const wc_pf_args *a, void *stream);

/* The trunk matvec (trunk_mvq.cu): rows [r0, r1) of a Q8G / Q4G / Q3G
 * tensor (bits 8 / 4 / 3), `rowbytes` bytes per row, one f16 scale per
 * group of `group` weights (ng groups per row), against x[in] fp32; all
 * device pointers. y[r] for r in [r0, r1). */
typedef struct {
    float *y;
    const uint8_t *W;
    const uint16_t *ws;
    const float *x;
    int r0, r1, in, ng, group, bits;
    size_t rowbytes;
    int pdl;           /* 1: launched programmatically behind the previous
                          kernel; the weight copies start before its end
                          and x is read only after the dependency wait   */
} wc_mvq_args;

int wc_mvq_launch(const wc_mvq_args *a, void *stream);

/* Kernels launched by this library since load. */
uint64_t wc_launches(void);
void     wc_count_launches(int n);

/* MLA attention (mla.cu). */
size_t wc_mla_head_smem(int qd, int kl, int S, int wrows, size_t rowbytes, int ng);
/* pos_p: the token's position in device memory (the cache row written,
 * rows 0..pos attended); S_max: the rows the head kernel's shared memory
 * is sized for (> pos). */
int wc_mla_prep_launch(float *x, int n, const float *w, float eps, float *rot, const float *cs,
                       const float *sn, int half, float *q, int nh, int qd, int qk_nope,
                       float *lat, const int *pos_p, float *lat_out, int latd, void *stream);
int wc_mla_head_launch(const float *q, const float *lat, const int *pos_p, int S_max, int latd,
                       int kl, int qd, int nope, int rope, int vh, int nh, const uint8_t *W,
                       const uint16_t *ws, size_t rowbytes, int ng, int group, int bits,
                       float scale, float *o, void *stream, int pdl);
int wc_mla_gate_launch(float *o, const float *g, int n, void *stream, int pdl);
/* With pdl set, the head and the gate launch programmatically behind the
 * kernel before them: the head stages its kv_b_proj rows (constants) while
 * the prep runs. */

/* Phase timers (see waste_cuda_profile in include/waste_cuda.h). */
enum { WC_PH_ROUTER, WC_PH_ACT, WC_PH_GATEUP, WC_PH_DOWN, WC_PH_COMBINE,
       WC_PH_MATVEC, WC_PH_MATVEC_REDUCE, WC_PH_EP_PUBLISH, WC_PH_EP_FINALIZE, WC_PH_COUNT };
int  wc_prof_enable(int on);
int  wc_profiling(void);      /* 1 while the phase timers are on */
void wc_prof_read(double *ms, unsigned long long *cnt, int nphase);

#ifdef __cplusplus
}
#endif
#endif
