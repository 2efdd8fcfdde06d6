/*
 * waste_cuda.c — host side of the B200 backend, plain C over the CUDA
 * runtime. Implements include/waste_cuda.h: device selection and the plugin
 * registration (src/backend.c:57-59,202-204 in the reference), codebooks and
 * expert banks resident in HBM (what src/ecache.c does for RAM), and the
 * expert-loop slots, which copy the engine's host buffers in and out around
 * the kernels in vq3r_kernels.cu.
 *
 * State is per process: one device, one stream, one set of layers — the
 * reference's dispatch table is a process global too (src/backend.c:38).
 * Calls are serialised by a mutex; the engine calls the slots from the
 * thread running waste_model_step.
 */
#include "../../include/waste_cuda.h"
#include "wc_launch.h"

#include <cuda_runtime_api.h>
#include <dlfcn.h>
#include <nccl.h>
#include <pthread.h>
#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

#define WC_MAX_LAYERS 128          /* WASTE_MAX_LAYERS, src/model.h:44 */
#define WC_MAX_TOPK 64             /* src/model.c:814-815 bounds top_k */
#define WC_CHUNK_MAX 64            /* WASTE_CHUNK_MAX, src/model.h:285 */

/* Expert record header, the reference's waste_expert_hdr
 * (src/waste_format.h:98-132): an on-disk format, kept field for field. */
typedef struct {
    uint32_t magic;
    uint16_t layer, expert_id;
    uint8_t fmt, flags;
    uint16_t codebook_id, lowrank_id, reserved0;
    uint32_t rec_4k_blocks;
    uint32_t gate_off, up_off, down_off, chan_corr_off;
    uint32_t crc32;
    uint32_t reserved1[2];
} wc_hdr;

#define WC_MAGIC_EXPERT 0x50584557u   /* src/waste_format.h:33 */
#define WC_WQ_VQ3R 4                  /* src/waste_format.h:51 */
#define WC_WQ_VQ2R 5                  /* src/waste_format.h:52 */
#define WC_WQ_VQ4P 8                  /* src/waste_format.h:57: 4 stages of 64, 6-bit indices packed 4-in-3 */
#define WC_ALIGN 4096u                /* src/waste_format.h:42 */

typedef struct {
    int loaded;
    wc_bank kb;                  /* device view                              */
    uint8_t *d_base;
    int n_total;                 /* experts in the layer                      */
    uint8_t *present;            /* host: which records have been loaded      */
    int n_present;
    int have_hdr;                /* offsets/codebook fixed by the first record */
    /* trunk */
    int trunk;
    float *d_router, *d_bias;
    int E, hidden, top_k, renorm;
    float routed_scale;
    int si;
    int8_t *d_shg, *d_shu, *d_shd;
    uint16_t *d_shg_s, *d_shu_s, *d_shd_s;
    /* the MoE block's rmsnorm (post_attention_layernorm) */
    float *d_norm;
    float norm_eps;
    /* the gated activation of the device-routed paths: 0 SiLU, 1 SiTU */
    int act;
    float situ_beta, situ_lbeta;
    /* the host-buffer layer and block calls as one CUDA graph each (copies
     * in, kernels, copies out), rebuilt when anything they point at may
     * have moved */
    cudaGraphExec_t gx, gxb;
    unsigned gx_epoch, gxb_epoch;
} wc_layer;

static struct {
    int inited, device;
    cudaStream_t stream;
    char name[300];
    float *d_books;
    int n_books;
    int cb_entries;              /* 256 (VQ3R/VQ2R) or 64 (VQ4P); books sit 256 entries apart */
    float *book_absmax;          /* host: max |entry| of each book               */
    int books_f16;               /* every entry an fp16 normal or zero (exact in fp16) */
    /* batched (prefill) path on the tensor cores */
    void *d_pf;
    size_t pf_bytes;
    wc_layer layer[WC_MAX_LAYERS];
    /* workspace for one launch of up to WC_CHUNK_MAX tokens */
    float *d_ws;
    size_t ws_floats;
    float *d_x, *d_out;
    int *d_idx;
    float *d_w;
    size_t io_floats;
    /* pinned staging */
    float *h_x, *h_out;
    int *h_idx;
    float *h_w;
    /* single-kernel parity APIs */
    void *d_tmp;
    size_t tmp_bytes;
    /* fetch layer+1's router and shared expert into L2 during layer */
    int prefetch_next;
    /* pinned host buffers are mapped at their own addresses: the host
     * calls move their small inputs and results with one copy kernel */
    int host_direct;
    /* the host layer call's results in one block, so one copy brings them
     * back: out [res_lat] | route [WC_MAX_TOPK] | weights [WC_MAX_TOPK] | err */
    float *d_res, *h_res;
    int res_lat;
    /* VQ4P scratch: integer block sums, table scales, activations */
    void *d_p6;
    size_t p6_bytes;
    /* the encoder's buffers (host-pointer forms) and the Lloyd scratch */
    void *d_enc;
    size_t enc_bytes;
} S;

/* Bumped by every call that allocates, frees or reloads what a cached
 * layer graph points at (workspace, banks, trunks, codebooks, the expert
 * split); a graph built under another epoch is rebuilt before use. */
static unsigned g_epoch = 1;

/* Expert parallelism: this process's rank among `world` processes (one GPU
 * each) that share every MoE layer, each holding a contiguous range of the
 * experts. NCCL is resolved at run time (dlopen), so the library loads and
 * runs single-GPU without it. Kept outside S: shutdown tears it down first. */
static struct {
    int active, rank, world;
    void *lib;
    ncclComm_t comm;
    ncclResult_t (*get_unique_id)(ncclUniqueId *);
    ncclResult_t (*comm_init_rank)(ncclComm_t *, int, ncclUniqueId, int);
    ncclResult_t (*comm_destroy)(ncclComm_t);
    ncclResult_t (*all_gather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t,
                               cudaStream_t);
    ncclResult_t (*reduce_scatter)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t,
                                   ncclComm_t, cudaStream_t);
    const char *(*error_string)(ncclResult_t);
    ncclResult_t (*all_reduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t,
                               ncclComm_t, cudaStream_t);
    float *d_xall, *d_outall;     /* [world*T][hidden] gathered tokens and partials */
    size_t all_floats;
    /* the exchange through peer memory: every rank's mailbox mapped here */
    int p2p;                      /* 1 once every rank mapped every mailbox */
    unsigned char *mail[WC_EP_MAX];
    int mail_T, mail_hidden;
    int wait_polls;               /* peer-wait limit, WASTE_CUDA_EP_WAIT_POLLS */
    int poisoned;                 /* a peer wait gave up: layer calls refused until
                                     ep_shutdown + ep_init build new mailboxes */
} EP;

/* The allocation-free matvec's fixed partial-sum array on the bound device
 * (set by init, cleared by shutdown). */
_Static_assert(WASTE_CUDA_NOALLOC_SCRATCH_BYTES == WC_NOALLOC_PART_FLOATS * sizeof(float),
               "header and kernel disagree on the fixed scratch size");
static float *g_noalloc_part;

/* Two pinned staging buffers for loading banks from files: while one is
 * copied to HBM, the next range is read into the other. */
#define WC_STAGE_BYTES ((size_t)64 << 20)
static struct {
    uint8_t *buf[2];
    size_t bytes;
    cudaEvent_t done[2];
    int ev;
} g_stage;

static pthread_mutex_t g_mu = PTHREAD_MUTEX_INITIALIZER;

/* Uploads and clears issued outside the library's streams. Those streams
 * are non-blocking, so nothing orders them after the default stream, and a
 * cudaMemcpy from pageable memory (or a cudaMemset) may return before the
 * device holds the bytes: each of these returns only once it does, so a
 * kernel on any stream launched afterwards reads them. */
static cudaError_t h2d_now(void *d, const void *h, size_t n)
{
    const cudaError_t e = cudaMemcpy(d, h, n, cudaMemcpyHostToDevice);
    return e != cudaSuccess ? e : cudaStreamSynchronize(0);
}

static cudaError_t memset_now(void *d, int v, size_t n)
{
    const cudaError_t e = cudaMemset(d, v, n);
    return e != cudaSuccess ? e : cudaStreamSynchronize(0);
}
static void ep_shutdown_locked(void);
static void mirrors_free(void);
/* the engine's KDA slot signatures (src/waste_backend.h:69-76) */
typedef void (*wc_kda_fn)(int H, int K, int V, const float *q, const float *k, const float *v,
                          const float *g_log, const float *beta, float *S, float *o,
                          float *scratch);
typedef void (*wc_conv_fn)(int C, int KS, const float *w, const float *bias, float *ring,
                           const float *x, float *y);
typedef void (*wc_rmsg_fn)(int C, const float *x, const float *gate, const float *weight,
                           float eps, float *y);
static void states_free(void);
static void branches_free(void);
static void kda_slot(int H, int K, int V, const float *q, const float *k, const float *v,
                     const float *g_log, const float *beta, float *S, float *o, float *scratch);
static void conv_slot(int C, int KS, const float *w, const float *bias, float *ring,
                      const float *x, float *y);
static void rmsg_slot(int C, const float *x, const float *gate, const float *weight, float eps,
                      float *y);
static wc_kda_fn g_kda_cpu;
static wc_conv_fn g_conv_cpu;
static wc_rmsg_fn g_rmsg_cpu;
static int pf_wanted(const wc_layer *L, int T, int K);
static int p6_experts(const wc_layer *L, int T, int K, int act, float situ_beta,
                      float situ_lbeta, int order_by_id);
static int pf_args(const wc_layer *L, int T, int K, wc_pf_args *a);
static _Thread_local char g_err[256];
static char g_err_global[256];

static int fail(int code, const char *fmt, ...)
{
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof g_err, fmt, ap);
    va_end(ap);
    memcpy(g_err_global, g_err, sizeof g_err);
    return code;
}

static int cuda_fail(cudaError_t e, const char *what)
{
    if (e == cudaErrorMemoryAllocation)
        return fail(WASTE_CUDA_E_NOMEM, "%s: %s", what, cudaGetErrorString(e));
    return fail(WASTE_CUDA_E_DEVICE, "%s: %s", what, cudaGetErrorString(e));
}

#define CK(call, what) do { cudaError_t e_ = (call); if (e_ != cudaSuccess) { \
    rc = cuda_fail(e_, what); goto out; } } while (0)

const char *waste_cuda_last_error(void)
{
    return g_err[0] ? g_err : (g_err_global[0] ? g_err_global : NULL);
}

uint64_t waste_cuda_launch_count(void) { return wc_launches(); }

/* The workspace's control words (wc_moe_ws_carve): err sits 192 words in. */
static unsigned read_device_errors(int clear)
{
    if (!S.d_ws) return 0;
    unsigned int *err = (unsigned int *)S.d_ws + 192, v = 0;
    if (cudaStreamSynchronize(S.stream) != cudaSuccess) return ~0u;
    if (cudaMemcpy(&v, err, sizeof v, cudaMemcpyDeviceToHost) != cudaSuccess) return ~0u;
    /* a wait that gave up leaves tickets, flags and pass counters of that
     * launch half-set: the whole control block (the error word included)
     * starts again from zero */
    if (v && clear) memset_now(S.d_ws, 0, WC_WS_CONTROL_WORDS * sizeof(unsigned int));
    if ((v & WC_ERR_PEER_WAIT) && EP.active) EP.poisoned = 1;
    return v;
}

unsigned waste_cuda_device_errors(void)
{
    pthread_mutex_lock(&g_mu);
    const unsigned v = S.inited ? read_device_errors(1) : 0;
    pthread_mutex_unlock(&g_mu);
    return v;
}

int waste_cuda_profile(int on)
{
    pthread_mutex_lock(&g_mu);
    const int rc = wc_prof_enable(on) ? fail(WASTE_CUDA_E_DEVICE, "profile events") : 0;
    pthread_mutex_unlock(&g_mu);
    return rc;
}

int waste_cuda_profile_read(double *ms, uint64_t *launches, int nphase)
{
    if (nphase < 0) return fail(WASTE_CUDA_E_ARG, "nphase < 0");
    pthread_mutex_lock(&g_mu);
    unsigned long long c[WC_PH_COUNT];
    double t[WC_PH_COUNT];
    wc_prof_read(t, c, WC_PH_COUNT);
    for (int i = 0; i < nphase && i < WC_PH_COUNT; i++) {
        if (ms) ms[i] = t[i];
        if (launches) launches[i] = c[i];
    }
    pthread_mutex_unlock(&g_mu);
    return 0;
}

static int getenv_flag(const char *name, int dflt)
{
    const char *e = getenv(name);
    return (e && *e) ? (*e != '0') : dflt;
}

static int pick_device(int requested)
{
    if (requested >= 0) return requested;
    const char *e = getenv("WASTE_CUDA_DEVICE");
    return e ? atoi(e) : 0;
}

/* Workspace for T tokens at the largest shapes loaded so far. */
/* The small copies of one host call between pinned host buffers and device
 * buffers (at most WC_COPY_MAX, 256 KB in all): one copy kernel, whose
 * loads and stores cross the bus in one round trip, when the pinned
 * buffers are mapped at their own addresses; else one copy-engine transfer
 * each (the copy engine pays a setup of several microseconds per transfer). */
static cudaError_t small_copies(const wc_copy_args *c, enum cudaMemcpyKind kind)
{
    size_t total = 0;
    for (int k = 0; k < c->n; k++) total += c->bytes[k];
    if (S.host_direct && total <= (256u << 10)) return (cudaError_t)wc_copy_launch(c, S.stream);
    for (int k = 0; k < c->n; k++) {
        const cudaError_t e = cudaMemcpyAsync(c->dst[k], c->src[k], c->bytes[k], kind, S.stream);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

static int ensure_ws(int T, int K, int E, int lat, int inter, int si, int stages)
{
    const size_t need = wc_moe_ws_floats(T, K, E, lat, inter, si, stages);
    const size_t io = (size_t)T * (lat > 0 ? lat : 1);
    if (need > S.ws_floats) {
        if (S.d_ws) cudaFree(S.d_ws);
        S.d_ws = NULL;
        S.ws_floats = 0;
        g_epoch++;
        cudaError_t e = cudaMalloc((void **)&S.d_ws, need * sizeof(float));
        if (e != cudaSuccess) return cuda_fail(e, "workspace");
        /* the router's ticket counters live here and must start at zero */
        e = memset_now(S.d_ws, 0, need * sizeof(float));
        if (e != cudaSuccess) return cuda_fail(e, "workspace clear");
        S.ws_floats = need;
    }
    if (io > S.io_floats) {
        g_epoch++;
        if (S.d_x) cudaFree(S.d_x);
        if (S.d_out) cudaFree(S.d_out);
        if (S.h_x) cudaFreeHost(S.h_x);
        if (S.h_out) cudaFreeHost(S.h_out);
        S.d_x = S.d_out = S.h_x = S.h_out = NULL;
        S.io_floats = 0;
        if (cudaMalloc((void **)&S.d_x, io * sizeof(float)) ||
            cudaMalloc((void **)&S.d_out, io * sizeof(float)) ||
            cudaMallocHost((void **)&S.h_x, io * sizeof(float)) ||
            cudaMallocHost((void **)&S.h_out, io * sizeof(float)))
            return fail(WASTE_CUDA_E_NOMEM, "io buffers for %d tokens", T);
        S.io_floats = io;
    }
    return 0;
}

static int init_locked(int device)
{
    int rc = 0;
    const int dev = pick_device(device);
    if (S.inited) {
        if (dev == S.device) return 0;
        return fail(WASTE_CUDA_E_ARG, "already bound to device %d", S.device);
    }
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n <= 0)
        return fail(WASTE_CUDA_E_NODEV, "no CUDA device");
    if (dev < 0 || dev >= n) return fail(WASTE_CUDA_E_NODEV, "device %d of %d", dev, n);
    struct cudaDeviceProp p;
    CK(cudaGetDeviceProperties(&p, dev), "cudaGetDeviceProperties");
    if (p.major != 10) return fail(WASTE_CUDA_E_NODEV, "device %d is sm_%d%d, not sm_100", dev,
                                   p.major, p.minor);
    CK(cudaSetDevice(dev), "cudaSetDevice");
    CK(cudaStreamCreateWithFlags(&S.stream, cudaStreamNonBlocking), "cudaStreamCreate");
    /* the allocation-free matvec's array and kernels, on the device now */
    CK((cudaError_t)wc_noalloc_setup(&g_noalloc_part), "fixed scratch set-up");
    if (!g_noalloc_part) return fail(WASTE_CUDA_E_DEVICE, "fixed scratch address: NULL");
    CK(cudaMalloc((void **)&S.d_idx, (size_t)WC_CHUNK_MAX * WC_MAX_TOPK * sizeof(int)), "idx");
    CK(cudaMalloc((void **)&S.d_w, (size_t)WC_CHUNK_MAX * WC_MAX_TOPK * sizeof(float)), "w");
    CK(cudaMallocHost((void **)&S.h_idx, (size_t)WC_CHUNK_MAX * WC_MAX_TOPK * sizeof(int)), "h_idx");
    CK(cudaMallocHost((void **)&S.h_w, (size_t)WC_CHUNK_MAX * WC_MAX_TOPK * sizeof(float)), "h_w");
    {
        void *dp = NULL;
        S.host_direct = getenv_flag("WASTE_CUDA_HOST_COPY_KERNEL", 1) &&
                        cudaHostGetDevicePointer(&dp, S.h_idx, 0) == cudaSuccess &&
                        dp == (void *)S.h_idx;
        cudaGetLastError();
    }
    snprintf(S.name, sizeof S.name, "CUDA sm_100a (%s)", p.name);
    {
        const char *pe = getenv("WASTE_CUDA_PREFETCH");
        S.prefetch_next = !(pe && *pe == '0');
    }
    S.device = dev;
    S.inited = 1;
out:
    return rc;
}

int waste_cuda_init(int device)
{
    pthread_mutex_lock(&g_mu);
    const int rc = init_locked(device);
    pthread_mutex_unlock(&g_mu);
    return rc;
}

int waste_cuda_device(void) { return S.inited ? S.device : -1; }

const char *waste_cuda_backend_name(void) { return S.inited ? S.name : NULL; }

static void free_layer(wc_layer *L)
{
    if (L->gx) cudaGraphExecDestroy(L->gx);
    if (L->gxb) cudaGraphExecDestroy(L->gxb);
    cudaFree(L->d_norm);
    cudaFree(L->d_base);
    cudaFree(L->d_router); cudaFree(L->d_bias);
    cudaFree(L->d_shg); cudaFree(L->d_shu); cudaFree(L->d_shd);
    cudaFree(L->d_shg_s); cudaFree(L->d_shu_s); cudaFree(L->d_shd_s);
    free(L->present);
    memset(L, 0, sizeof *L);
}

void waste_cuda_shutdown(void)
{
    pthread_mutex_lock(&g_mu);
    ep_shutdown_locked();
    if (S.inited) {
        cudaStreamSynchronize(S.stream);
        for (int i = 0; i < WC_MAX_LAYERS; i++) free_layer(&S.layer[i]);
        cudaFree(S.d_books); cudaFree(S.d_ws); cudaFree(S.d_x); cudaFree(S.d_out);
        cudaFree(S.d_idx); cudaFree(S.d_w); cudaFree(S.d_tmp); cudaFree(S.d_pf);
        free(S.book_absmax);
        cudaFreeHost(S.h_x); cudaFreeHost(S.h_out); cudaFreeHost(S.h_idx);
        cudaFreeHost(S.h_w);
        cudaFree(S.d_res); cudaFreeHost(S.h_res);
        cudaFree(S.d_p6);
        cudaFree(S.d_enc);
        mirrors_free();
        states_free();
        for (int b = 0; b < 2; b++) {
            cudaFreeHost(g_stage.buf[b]);
            if (g_stage.ev) cudaEventDestroy(g_stage.done[b]);
        }
        memset(&g_stage, 0, sizeof g_stage);
        branches_free();
        cudaStreamDestroy(S.stream);
        memset(&S, 0, sizeof S);
        g_noalloc_part = NULL;
    }
    pthread_mutex_unlock(&g_mu);
}

/* ---- registration ---------------------------------------------------- */

/* ---- the trunk matvec slot ---------------------------------------------
 * The engine's dispatch table (src/waste_backend.h:67-90) and the argument
 * of its mvq_rows_f32 slot (src/simd.h:35-39), restated field for field:
 * the slot is called with a pointer to the table at registration and with
 * a pointer to the argument on every trunk matvec. */
typedef struct {
    wc_kda_fn kda_step;
    wc_conv_fn short_conv_step;
    wc_rmsg_fn rmsnorm_gated;
    void (*mvq_rows_f32)(int b, int e, void *arg);
    void (*lutb_range)(int lo, int hi, void *arg);
    int on_device;
} wc_kernels_table;

typedef struct {
    float *y;
    const int8_t *W;
    const uint16_t *ws;
    const int8_t *xq;
    const float *xs;
    int in, ng, group, bits;
    size_t rowbytes;
} wc_mvq_arg;

/* Device copies of the engine's trunk tensors, keyed by the host address
 * of their weights (the engine keeps them resident and passes the same
 * pointers on every call), open addressing. */
#define WC_MIRRORS 4096
static struct {
    const void *key;
    uint8_t *d_W;
    uint16_t *d_ws;
    size_t rows, rowbytes;
    int ng;
} g_mirror[WC_MIRRORS];
static float *g_mvq_x, *g_mvq_y;
static size_t g_mvq_xcap, g_mvq_ycap;
static float *g_mvq_hx, *g_mvq_hy;                  /* pinned staging of x and y */
static size_t g_mvq_hxcap, g_mvq_hycap;
static void (*g_mvq_cpu)(int b, int e, void *arg);   /* the slot's previous occupant */
static size_t g_trunk_min = (size_t)1 << 20;         /* WASTE_CUDA_TRUNK_MIN bytes */

static size_t mirror_hash(const void *p)
{
    uint64_t x = (uint64_t)(uintptr_t)p;
    x ^= x >> 33; x *= 0xff51afd7ed558ccdULL; x ^= x >> 33;
    return (size_t)(x & (WC_MIRRORS - 1));
}

/* The tensor's device copy holding at least `rows` rows, made (or grown)
 * now when it is not there yet. NULL when it cannot be. Under g_mu. */
static int mirror_get(const wc_mvq_arg *a, size_t rows, uint8_t **dW, uint16_t **dws)
{
    size_t i = mirror_hash(a->W);
    for (int probe = 0; probe < WC_MIRRORS; probe++, i = (i + 1) & (WC_MIRRORS - 1)) {
        if (g_mirror[i].key == a->W) {
            if (g_mirror[i].rows >= rows && g_mirror[i].rowbytes == a->rowbytes &&
                g_mirror[i].ng == a->ng) {
                *dW = g_mirror[i].d_W;
                *dws = g_mirror[i].d_ws;
                return 0;
            }
            cudaFree(g_mirror[i].d_W);
            cudaFree(g_mirror[i].d_ws);
            g_epoch++;                  /* graphs holding the old copy are stale */
            break;
        }
        if (!g_mirror[i].key) break;
    }
    if (g_mirror[i].key && g_mirror[i].key != a->W) return -1;   /* table full */
    const size_t wb = rows * a->rowbytes, sb = rows * (size_t)a->ng * sizeof(uint16_t);
    uint8_t *w = NULL;
    uint16_t *s = NULL;
    if (cudaMalloc((void **)&w, wb) != cudaSuccess || cudaMalloc((void **)&s, sb) != cudaSuccess ||
        h2d_now(w, a->W, wb) != cudaSuccess || h2d_now(s, a->ws, sb) != cudaSuccess) {
        cudaFree(w);
        cudaFree(s);
        cudaGetLastError();
        memset(&g_mirror[i], 0, sizeof g_mirror[i]);
        return -1;
    }
    g_mirror[i].key = a->W;
    g_mirror[i].d_W = w;
    g_mirror[i].d_ws = s;
    g_mirror[i].rows = rows;
    g_mirror[i].rowbytes = a->rowbytes;
    g_mirror[i].ng = a->ng;
    *dW = w;
    *dws = s;
    return 0;
}

static void mirrors_free(void)
{
    g_epoch++;
    for (int i = 0; i < WC_MIRRORS; i++) {
        if (!g_mirror[i].key) continue;
        cudaFree(g_mirror[i].d_W);
        cudaFree(g_mirror[i].d_ws);
    }
    memset(g_mirror, 0, sizeof g_mirror);
    cudaFree(g_mvq_x);
    cudaFree(g_mvq_y);
    g_mvq_x = g_mvq_y = NULL;
    g_mvq_xcap = g_mvq_ycap = 0;
    cudaFreeHost(g_mvq_hx);
    cudaFreeHost(g_mvq_hy);
    g_mvq_hx = g_mvq_hy = NULL;
    g_mvq_hxcap = g_mvq_hycap = 0;
}

/* A pinned host buffer of at least `bytes` (grown, never shrunk). */
static int pinned_at_least(float **p, size_t *cap, size_t bytes)
{
    if (bytes <= *cap) return 0;
    cudaFreeHost(*p);
    *p = NULL;
    *cap = 0;
    if (cudaMallocHost((void **)p, bytes) != cudaSuccess) {
        cudaGetLastError();
        return -1;
    }
    *cap = bytes;
    return 0;
}

/* The device side of one slot call, under g_mu: 0, or -1 (the caller
 * computes the rows on the CPU instead). */
static int mvq_device(int b, int e, const wc_mvq_arg *a)
{
    uint8_t *dW;
    uint16_t *dws;
    if (!S.inited || mirror_get(a, (size_t)e, &dW, &dws)) return -1;
    const size_t xb = (size_t)a->in * sizeof(float), yb = (size_t)e * sizeof(float);
    if (xb > g_mvq_xcap) {
        cudaFree(g_mvq_x);
        g_mvq_x = NULL;
        g_mvq_xcap = 0;
        if (cudaMalloc((void **)&g_mvq_x, xb) != cudaSuccess) return -1;
        g_mvq_xcap = xb;
    }
    if (yb > g_mvq_ycap) {
        cudaFree(g_mvq_y);
        g_mvq_y = NULL;
        g_mvq_ycap = 0;
        if (cudaMalloc((void **)&g_mvq_y, yb) != cudaSuccess) return -1;
        g_mvq_ycap = yb;
    }
    wc_mvq_args k = { g_mvq_y, dW, dws, g_mvq_x, b, e, a->in, a->ng, a->group, a->bits,
                      a->rowbytes, 0 };
    /* x and (up to 256 KB of) y through pinned staging and the copy
     * kernel; a longer y range (lm_head) straight into the caller's memory */
    const size_t yr = (size_t)(e - b) * sizeof(float);
    const int stage_y = S.host_direct && yr <= (256u << 10) &&
                        !pinned_at_least(&g_mvq_hy, &g_mvq_hycap, yr);
    if (pinned_at_least(&g_mvq_hx, &g_mvq_hxcap, xb)) return -1;
    memcpy(g_mvq_hx, a->xs, xb);
    const wc_copy_args cin = { { g_mvq_x }, { g_mvq_hx }, { xb }, 1, 0 };
    const wc_copy_args cout = { { g_mvq_hy }, { g_mvq_y + b }, { yr }, 1, 0 };
    if (small_copies(&cin, cudaMemcpyHostToDevice) != cudaSuccess ||
        wc_mvq_launch(&k, S.stream) != 0 ||
        (stage_y ? small_copies(&cout, cudaMemcpyDeviceToHost)
                 : cudaMemcpyAsync(a->y + b, g_mvq_y + b, yr, cudaMemcpyDeviceToHost,
                                   S.stream)) != cudaSuccess ||
        cudaStreamSynchronize(S.stream) != cudaSuccess) {
        cudaGetLastError();
        return -1;
    }
    if (stage_y) memcpy(a->y + b, g_mvq_hy, yr);
    return 0;
}

/* The engine's mvq_rows_f32 slot (src/model.c:397, run on the calling
 * thread with the whole row range: on_device). Tensors of at least
 * WASTE_CUDA_TRUNK_MIN bytes (default 1 MiB) run on the device from their
 * HBM copy; smaller ones, the quantised-activation form (xq set) and any
 * device failure run on the CPU kernel the slot held before (the slot has
 * no error channel, as the Metal backend does it). */
static void mvq_slot(int b, int e, void *arg)
{
    const wc_mvq_arg *a = (const wc_mvq_arg *)arg;
    int done = -1;
    if (!a->xq && a->xs && (a->bits == 8 || a->bits == 4 || a->bits == 3) && e > b &&
        (size_t)e * a->rowbytes >= g_trunk_min) {
        pthread_mutex_lock(&g_mu);
        done = mvq_device(b, e, a);
        pthread_mutex_unlock(&g_mu);
    }
    if (done != 0 && g_mvq_cpu) g_mvq_cpu(b, e, arg);
}

const char *waste_register_cuda(void *table)
{
    const char *e = getenv("WASTE_CUDA");
    if (e && *e == '0') return NULL;
    if (waste_cuda_init(-1) != 0) return NULL;
    wc_kernels_table *t = (wc_kernels_table *)table;
    if (t && t->mvq_rows_f32 && getenv_flag("WASTE_CUDA_TRUNK", 1)) {
        const char *m = getenv("WASTE_CUDA_TRUNK_MIN");
        if (m && *m) g_trunk_min = (size_t)strtoull(m, NULL, 10);
        if (t->mvq_rows_f32 != mvq_slot) g_mvq_cpu = t->mvq_rows_f32;
        t->mvq_rows_f32 = mvq_slot;
        t->on_device = 1;
    }
    /* KDA: the decode step (recurrent state kept in HBM) by default; the
     * conv and the gated norm on request, since each of their calls is a
     * few KB whose host round trip costs more than the CPU's arithmetic */
    if (t && t->kda_step && getenv_flag("WASTE_CUDA_KDA", 1)) {
        if (t->kda_step != kda_slot) g_kda_cpu = t->kda_step;
        t->kda_step = kda_slot;
        t->on_device = 1;
    }
    if (t && t->short_conv_step && getenv_flag("WASTE_CUDA_KDA_CONV", 0)) {
        if (t->short_conv_step != conv_slot) g_conv_cpu = t->short_conv_step;
        t->short_conv_step = conv_slot;
    }
    if (t && t->rmsnorm_gated && getenv_flag("WASTE_CUDA_KDA_NORM", 0)) {
        if (t->rmsnorm_gated != rmsg_slot) g_rmsg_cpu = t->rmsnorm_gated;
        t->rmsnorm_gated = rmsg_slot;
    }
    return S.name;
}

void waste_cuda_release_host_buffers(void)
{
    pthread_mutex_lock(&g_mu);
    if (S.inited) {
        cudaStreamSynchronize(S.stream);
        mirrors_free();
        states_free();
    }
    pthread_mutex_unlock(&g_mu);
}

/* ---- KDA: recurrent state resident in HBM -----------------------------
 * The engine's KDA state (m->S[L], [H][K][V]) and conv rings (m->conv[L])
 * move to HBM the first time a slot sees them, keyed by host address, as
 * do the conv and norm weights; from then on the device copy is the state
 * and the host copy is stale. waste_cuda_state_pull brings a range back to
 * the host (before the engine reads it: a snapshot save) and
 * waste_cuda_state_push reloads it from the host (after the engine writes
 * it: a reset, a snapshot load). */
#define WC_STATES 1024
static struct {
    const uint8_t *host;
    size_t bytes;
    uint8_t *dev;
} g_rs[WC_STATES];
static int g_nrs;
static float *g_kda_pin, *g_kda_dev;     /* pinned and device staging, floats */
static size_t g_kda_cap;
static float *g_mla_pin, *g_mla_dev;     /* the MLA layer's staging */
static size_t g_mla_cap;

/* The device address of host range [h, h + bytes): inside a held copy, or
 * a copy made now from the host bytes. NULL when it partly overlaps a held
 * copy or cannot be made. Under g_mu. */
static void *rs_get(const void *h, size_t bytes)
{
    const uint8_t *p = (const uint8_t *)h;
    for (int i = 0; i < g_nrs; i++)
        if (p >= g_rs[i].host && p + bytes <= g_rs[i].host + g_rs[i].bytes)
            return g_rs[i].dev + (p - g_rs[i].host);
    for (int i = 0; i < g_nrs; i++)
        if (p < g_rs[i].host + g_rs[i].bytes && g_rs[i].host < p + bytes) return NULL;
    if (g_nrs == WC_STATES) return NULL;
    uint8_t *d = NULL;
    if (cudaMalloc((void **)&d, bytes) != cudaSuccess ||
        h2d_now(d, h, bytes) != cudaSuccess) {
        cudaFree(d);
        cudaGetLastError();
        return NULL;
    }
    g_rs[g_nrs].host = p;
    g_rs[g_nrs].bytes = bytes;
    g_rs[g_nrs].dev = d;
    g_nrs++;
    return d;
}

static void layer_graphs_free(void);
static void states_free(void)
{
    g_epoch++;
    layer_graphs_free();
    for (int i = 0; i < g_nrs; i++) cudaFree(g_rs[i].dev);
    memset(g_rs, 0, sizeof g_rs);
    g_nrs = 0;
    cudaFreeHost(g_kda_pin);
    cudaFree(g_kda_dev);
    g_kda_pin = g_kda_dev = NULL;
    g_kda_cap = 0;
    cudaFreeHost(g_mla_pin);
    cudaFree(g_mla_dev);
    g_mla_pin = g_mla_dev = NULL;
    g_mla_cap = 0;
}

/* Copies the parts of [h, h + bytes) held in HBM one way or the other. */
static int rs_sync(const void *h, size_t bytes, int to_host)
{
    int rc = 0;
    const uint8_t *p = (const uint8_t *)h;
    for (int i = 0; i < g_nrs; i++) {
        const uint8_t *lo = p > g_rs[i].host ? p : g_rs[i].host;
        const uint8_t *e0 = p + bytes, *e1 = g_rs[i].host + g_rs[i].bytes;
        const uint8_t *hi = e0 < e1 ? e0 : e1;
        if (lo >= hi) continue;
        uint8_t *d = g_rs[i].dev + (lo - g_rs[i].host);
        if (to_host)
            CK(cudaMemcpy((void *)lo, d, (size_t)(hi - lo), cudaMemcpyDeviceToHost), "state D2H");
        else
            CK(h2d_now(d, lo, (size_t)(hi - lo)), "state H2D");
    }
out:
    return rc;
}

int waste_cuda_state_pull(void *host, size_t bytes)
{
    if (!host) return fail(WASTE_CUDA_E_ARG, "NULL pointer");
    pthread_mutex_lock(&g_mu);
    int rc = 0;
    if (S.inited) {
        cudaStreamSynchronize(S.stream);
        rc = rs_sync(host, bytes, 1);
    }
    pthread_mutex_unlock(&g_mu);
    return rc;
}

int waste_cuda_state_push(const void *host, size_t bytes)
{
    if (!host) return fail(WASTE_CUDA_E_ARG, "NULL pointer");
    pthread_mutex_lock(&g_mu);
    int rc = 0;
    if (S.inited) {
        cudaStreamSynchronize(S.stream);
        rc = rs_sync(host, bytes, 0);
    }
    pthread_mutex_unlock(&g_mu);
    return rc;
}

static int kda_stage(size_t floats)
{
    if (floats <= g_kda_cap) return 0;
    g_epoch++;
    cudaFreeHost(g_kda_pin);
    cudaFree(g_kda_dev);
    g_kda_pin = g_kda_dev = NULL;
    g_kda_cap = 0;
    if (cudaMallocHost((void **)&g_kda_pin, floats * sizeof(float)) != cudaSuccess ||
        cudaMalloc((void **)&g_kda_dev, floats * sizeof(float)) != cudaSuccess) {
        cudaGetLastError();
        return fail(WASTE_CUDA_E_NOMEM, "KDA staging");
    }
    g_kda_cap = floats;
    return 0;
}

int waste_cuda_kda_step(int H, int K, int V, const float *q, const float *k, const float *v,
                        const float *g_log, const float *beta, float *S_, float *o)
{
    int rc = 0;
    if (H <= 0 || !q || !k || !v || !g_log || !beta || !S_ || !o || wc_kda_supported(K, V))
        return fail(WASTE_CUDA_E_ARG, "kda_step: bad arguments (K 32, 64 or 128)");
    pthread_mutex_lock(&g_mu);
    if (!S.inited && (rc = init_locked(-1))) goto out;
    float *dS = (float *)rs_get(S_, (size_t)H * K * V * sizeof(float));
    if (!dS) { rc = fail(WASTE_CUDA_E_NOMEM, "kda_step: state copy"); goto out; }
    const size_t hk = (size_t)H * K, hv = (size_t)H * V, n_in = 3 * hk + hv + H;
    if ((rc = kda_stage(n_in + hv))) goto out;
    float *p = g_kda_pin;
    memcpy(p, q, hk * 4);
    memcpy(p + hk, k, hk * 4);
    memcpy(p + 2 * hk, g_log, hk * 4);
    memcpy(p + 3 * hk, v, hv * 4);
    memcpy(p + 3 * hk + hv, beta, (size_t)H * 4);
    float *d = g_kda_dev;
    CK(cudaMemcpyAsync(d, p, n_in * 4, cudaMemcpyHostToDevice, S.stream), "KDA inputs H2D");
    CK((cudaError_t)wc_kda_step_launch(H, K, V, d, d + hk, d + 3 * hk, d + 2 * hk,
                                       d + 3 * hk + hv, dS, d + n_in, S.stream, 0), "KDA step");
    CK(cudaMemcpyAsync(p + n_in, d + n_in, hv * 4, cudaMemcpyDeviceToHost, S.stream), "o D2H");
    CK(cudaStreamSynchronize(S.stream), "KDA step");
    memcpy(o, p + n_in, hv * 4);
out:
    pthread_mutex_unlock(&g_mu);
    return rc;
}

int waste_cuda_short_conv_step(int C, int KS, const float *w, const float *bias, float *ring,
                               const float *x, float *y)
{
    int rc = 0;
    if (C <= 0 || KS < 1 || !w || !ring || !x || !y)
        return fail(WASTE_CUDA_E_ARG, "short_conv_step: bad arguments");
    pthread_mutex_lock(&g_mu);
    if (!S.inited && (rc = init_locked(-1))) goto out;
    float *dr = KS > 1 ? (float *)rs_get(ring, (size_t)C * (KS - 1) * sizeof(float)) : NULL;
    float *dw = (float *)rs_get(w, (size_t)C * KS * sizeof(float));
    float *db = bias ? (float *)rs_get(bias, (size_t)C * sizeof(float)) : NULL;
    if ((KS > 1 && !dr) || !dw || (bias && !db)) {
        rc = fail(WASTE_CUDA_E_NOMEM, "short_conv_step: device copies");
        goto out;
    }
    if ((rc = kda_stage(2 * (size_t)C))) goto out;
    memcpy(g_kda_pin, x, (size_t)C * 4);
    CK(cudaMemcpyAsync(g_kda_dev, g_kda_pin, (size_t)C * 4, cudaMemcpyHostToDevice, S.stream),
       "conv x H2D");
    CK((cudaError_t)wc_short_conv_launch(C, KS, dw, db, dr, g_kda_dev, g_kda_dev + C, S.stream),
       "short conv");
    CK(cudaMemcpyAsync(g_kda_pin + C, g_kda_dev + C, (size_t)C * 4, cudaMemcpyDeviceToHost,
                       S.stream), "conv y D2H");
    CK(cudaStreamSynchronize(S.stream), "short conv");
    memcpy(y, g_kda_pin + C, (size_t)C * 4);
out:
    pthread_mutex_unlock(&g_mu);
    return rc;
}

int waste_cuda_rmsnorm_gated_heads(int nh, int C, const float *x, const float *gate,
                                   const float *weight, float eps, float *y)
{
    int rc = 0;
    if (nh <= 0 || C <= 0 || C > 8192 || !x || !gate || !weight || !y)
        return fail(WASTE_CUDA_E_ARG, "rmsnorm_gated: bad arguments");
    pthread_mutex_lock(&g_mu);
    if (!S.inited && (rc = init_locked(-1))) goto out;
    float *dw = (float *)rs_get(weight, (size_t)C * sizeof(float));
    if (!dw) { rc = fail(WASTE_CUDA_E_NOMEM, "rmsnorm_gated: weight copy"); goto out; }
    const size_t n = (size_t)nh * C;
    if ((rc = kda_stage(3 * n))) goto out;
    memcpy(g_kda_pin, x, n * 4);
    memcpy(g_kda_pin + n, gate, n * 4);
    CK(cudaMemcpyAsync(g_kda_dev, g_kda_pin, 2 * n * 4, cudaMemcpyHostToDevice, S.stream),
       "norm inputs H2D");
    CK((cudaError_t)wc_rmsnorm_gated_launch(nh, C, g_kda_dev, g_kda_dev + n, dw, eps,
                                            g_kda_dev + 2 * n, S.stream, 0), "gated norm");
    CK(cudaMemcpyAsync(g_kda_pin + 2 * n, g_kda_dev + 2 * n, n * 4, cudaMemcpyDeviceToHost,
                       S.stream), "norm y D2H");
    CK(cudaStreamSynchronize(S.stream), "gated norm");
    memcpy(y, g_kda_pin + 2 * n, n * 4);
out:
    pthread_mutex_unlock(&g_mu);
    return rc;
}

int waste_cuda_kda_step_dev(int H, int K, int V, const float *q, const float *k, const float *v,
                            const float *g_log, const float *beta, float *S_, float *o,
                            void *stream)
{
    int rc = 0;
    if (H <= 0 || !q || !k || !v || !g_log || !beta || !S_ || !o || wc_kda_supported(K, V))
        return fail(WASTE_CUDA_E_ARG, "kda_step_dev: bad arguments (K 32, 64 or 128)");
    pthread_mutex_lock(&g_mu);
    if (!S.inited) { rc = fail(WASTE_CUDA_E_NODEV, "kda_step_dev before waste_cuda_init"); goto out; }
    CK((cudaError_t)wc_kda_step_launch(H, K, V, q, k, v, g_log, beta, S_, o,
                                       stream ? stream : (void *)S.stream, 0), "KDA step");
out:
    pthread_mutex_unlock(&g_mu);
    return rc;
}

int waste_cuda_short_conv_dev(int C, int KS, const float *w, const float *bias, float *ring,
                              const float *x, float *y, void *stream)
{
    int rc = 0;
    if (C <= 0 || KS < 1 || !w || (KS > 1 && !ring) || !x || !y)
        return fail(WASTE_CUDA_E_ARG, "short_conv_dev: bad arguments");
    pthread_mutex_lock(&g_mu);
    if (!S.inited) { rc = fail(WASTE_CUDA_E_NODEV, "short_conv_dev before waste_cuda_init"); goto out; }
    CK((cudaError_t)wc_short_conv_launch(C, KS, w, bias, ring, x, y,
                                         stream ? stream : (void *)S.stream), "short conv");
out:
    pthread_mutex_unlock(&g_mu);
    return rc;
}

int waste_cuda_rmsnorm_gated_dev(int nh, int C, const float *x, const float *gate,
                                 const float *weight, float eps, float *y, void *stream)
{
    int rc = 0;
    if (nh <= 0 || C <= 0 || C > 8192 || !x || !gate || !weight || !y)
        return fail(WASTE_CUDA_E_ARG, "rmsnorm_gated_dev: bad arguments");
    pthread_mutex_lock(&g_mu);
    if (!S.inited) { rc = fail(WASTE_CUDA_E_NODEV, "rmsnorm_gated_dev before waste_cuda_init"); goto out; }
    CK((cudaError_t)wc_rmsnorm_gated_launch(nh, C, x, gate, weight, eps, y,
                                            stream ? stream : (void *)S.stream, 0), "gated norm");
out:
    pthread_mutex_unlock(&g_mu);
    return rc;
}

/* The device copy of a trunk tensor (a mirror, made at first use). */
static int qt_dev(const waste_cuda_qtensor *t, uint8_t **dW, uint16_t **dws, int *ng)
{
    if (!t->W || !t->ws || t->rows <= 0 || t->cols <= 0 || t->group <= 0 ||
        (t->bits != 8 && t->bits != 4 && t->bits != 3) || t->rowbytes == 0)
        return -1;
    *ng = (t->cols + t->group - 1) / t->group;
    const wc_mvq_arg a = { NULL, (const int8_t *)t->W, t->ws, NULL, NULL, t->cols, *ng, t->group,
                           t->bits, t->rowbytes };
    return mirror_get(&a, (size_t)t->rows, dW, dws);
}

static int qt_launch_on(const waste_cuda_qtensor *t, const float *x, float *y, cudaStream_t st,
                        int pdl)
{
    uint8_t *dW;
    uint16_t *dws;
    int ng;
    if (qt_dev(t, &dW, &dws, &ng)) return -1;
    wc_mvq_args k = { y, dW, dws, x, 0, t->rows, t->cols, ng, t->group, t->bits, t->rowbytes,
                      pdl };
    return wc_mvq_launch(&k, st);
}

/* On the library's stream, launched programmatically: the weight copies
 * overlap the kernel before (not while the phase timers put events between
 * kernels). */
static int qt_launch(const waste_cuda_qtensor *t, const float *x, float *y)
{
    return qt_launch_on(t, x, y, S.stream, !wc_profiling());
}

/* Side streams and events for the independent branches of a layer (its
 * projections of the same input): forked from the library's stream and
 * joined back, so they run side by side — and become parallel branches of
 * a layer's graph when captured. Created outside any capture. */
#define WC_BRANCHES 6
static cudaStream_t g_side[WC_BRANCHES];
static cudaEvent_t g_fork, g_join[WC_BRANCHES];
static int g_branches_ok;

static int branches_ready(void)
{
    if (g_branches_ok) return 0;
    if (cudaEventCreateWithFlags(&g_fork, cudaEventDisableTiming) != cudaSuccess) return -1;
    for (int i = 0; i < WC_BRANCHES; i++)
        if (cudaStreamCreateWithFlags(&g_side[i], cudaStreamNonBlocking) != cudaSuccess ||
            cudaEventCreateWithFlags(&g_join[i], cudaEventDisableTiming) != cudaSuccess)
            return -1;
    g_branches_ok = 1;
    return 0;
}

static void branches_free(void)
{
    if (!g_branches_ok) return;
    for (int i = 0; i < WC_BRANCHES; i++) {
        cudaStreamDestroy(g_side[i]);
        cudaEventDestroy(g_join[i]);
    }
    cudaEventDestroy(g_fork);
    g_branches_ok = 0;
}

static int fork_branches(int n)
{
    if (cudaEventRecord(g_fork, S.stream) != cudaSuccess) return -1;
    for (int i = 0; i < n; i++)
        if (cudaStreamWaitEvent(g_side[i], g_fork, 0) != cudaSuccess) return -1;
    return 0;
}

static int join_branches(int n)
{
    for (int i = 0; i < n; i++)
        if (cudaEventRecord(g_join[i], g_side[i]) != cudaSuccess ||
            cudaStreamWaitEvent(S.stream, g_join[i], 0) != cudaSuccess)
            return -1;
    return 0;
}

/* ---- per-layer CUDA graphs of the whole-layer slots ---------------------
 * A whole-layer call is a dozen kernels (projections, convolutions, the
 * step, norms) plus the copies in and out; launched one by one from the
 * host, the launches cost more than the kernels. Each layer's sequence is
 * captured once into a graph, keyed by the caller's descriptor (the engine
 * keeps one per layer), at the descriptor's second call: its first call
 * makes the device copies of the layer's tensors and state, which a capture
 * cannot. A graph is rebuilt when g_epoch has moved (staging, mirrors or
 * states reallocated or freed). WASTE_CUDA_LAYER_GRAPHS=0 launches directly. */
#define WC_LGRAPHS 256
static struct {
    const void *key;
    int seen;
    unsigned epoch;
    cudaGraphExec_t gx;
} g_lg[WC_LGRAPHS];
static int g_nlg;
static int g_lg_on = -1;

static void layer_graphs_free(void)
{
    for (int i = 0; i < g_nlg; i++)
        if (g_lg[i].gx) cudaGraphExecDestroy(g_lg[i].gx);
    memset(g_lg, 0, sizeof g_lg);
    g_nlg = 0;
}

/* Runs fn(ctx) on S.stream: from the key's graph, or captured into one, or
 * directly. 0 or -1. Under g_mu. */
static int run_layer(const void *key, int (*fn)(void *), void *ctx)
{
    if (g_lg_on < 0) g_lg_on = getenv_flag("WASTE_CUDA_LAYER_GRAPHS", 1);
    int e = -1;
    for (int i = 0; i < g_nlg; i++)
        if (g_lg[i].key == key) { e = i; break; }
    if (e < 0 && g_nlg < WC_LGRAPHS && g_lg_on) {
        e = g_nlg++;
        g_lg[e].key = key;
    }
    if (e >= 0 && g_lg[e].gx && g_lg[e].epoch == g_epoch)
        return cudaGraphLaunch(g_lg[e].gx, S.stream) == cudaSuccess ? 0 : -1;
    if (e >= 0 && g_lg[e].seen) {
        if (g_lg[e].gx) { cudaGraphExecDestroy(g_lg[e].gx); g_lg[e].gx = NULL; }
        cudaGraph_t g = NULL;
        if (cudaStreamBeginCapture(S.stream, cudaStreamCaptureModeThreadLocal) == cudaSuccess) {
            const int r = fn(ctx);
            const cudaError_t ee = cudaStreamEndCapture(S.stream, &g);   /* always end it */
            if (!r && ee == cudaSuccess && g &&
                cudaGraphInstantiate(&g_lg[e].gx, g, 0) == cudaSuccess) {
                cudaGraphDestroy(g);
                g_lg[e].epoch = g_epoch;
                return cudaGraphLaunch(g_lg[e].gx, S.stream) == cudaSuccess ? 0 : -1;
            }
            if (g) cudaGraphDestroy(g);
            g_lg[e].gx = NULL;
        }
        cudaGetLastError();             /* a failed capture: launch directly */
    }
    if (e >= 0) g_lg[e].seen = 1;
    return fn(ctx);
}

struct kda_ctx {
    const waste_cuda_kda_layer_desc *d;
    float *dS, *dA, *dB, *dN, *dw[3], *dr[3];
};

/* The layer's device work on S.stream: x in from the pinned staging, the
 * kernels, y out to it. */
static int kda_enqueue(void *p)
{
    const struct kda_ctx *k = (const struct kda_ctx *)p;
    const waste_cuda_kda_layer_desc *d = k->d;
    const int H = d->H, D = d->D, C = H * D, hid = d->hidden, KS = d->conv_k;
    const int full_gate = d->g_full.W != NULL;
    /* staging: in | q k v g o gate | beta | lo_f lo_g | out */
    float *x = g_kda_dev, *q = x + hid, *kk = q + C, *v = kk + C, *g = v + C, *o = g + C;
    float *gate = o + C, *beta = gate + C, *lf = beta + H, *lg = lf + D, *y = lg + D;
    const wc_copy_args cin = { { x }, { g_kda_pin }, { (size_t)hid * 4 }, 1, 0 };
    if (small_copies(&cin, cudaMemcpyHostToDevice) != cudaSuccess) return -1;
    /* the branches that read only x, side by side: q, k and v each through
     * its short conv; the f path (f_a, f_b); beta's projection; the g path */
    const waste_cuda_qtensor *qkv[3] = { &d->q, &d->k, &d->v };
    float *dst[3] = { q, kk, v };
    int lrc = fork_branches(WC_BRANCHES);
    for (int i = 0; i < 3 && !lrc; i++) {
        lrc = qt_launch_on(qkv[i], x, dst[i], g_side[i], 0);
        if (!lrc) lrc = wc_short_conv_launch(C, KS, k->dw[i], NULL, k->dr[i], dst[i], dst[i],
                                             g_side[i]);
    }
    if (!lrc) lrc = qt_launch_on(&d->f_a, x, lf, g_side[3], 0);
    if (!lrc) lrc = qt_launch_on(&d->f_b, lf, g, g_side[3], 0);
    if (!lrc) lrc = qt_launch_on(&d->b, x, beta, g_side[4], 0);
    if (!lrc && full_gate) lrc = qt_launch_on(&d->g_full, x, gate, g_side[5], 0);
    if (!lrc && !full_gate) lrc = qt_launch_on(&d->g_a, x, lg, g_side[5], 0);
    if (!lrc && !full_gate) lrc = qt_launch_on(&d->g_b, lg, gate, g_side[5], 0);
    if (!lrc) lrc = join_branches(WC_BRANCHES);
    if (!lrc) lrc = wc_kda_gate_launch(g, k->dA, k->dB, H, D, d->lower_bound, beta, S.stream);
    /* gate → step → norm → o_proj programmatically (not while the phase
     * timers put events between kernels): the step's state fetch and the
     * projection's weight copies overlap the kernel before each */
    const int pdl = !wc_profiling();
    if (!lrc) lrc = wc_kda_step_launch(H, D, D, q, kk, v, g, beta, k->dS, o, S.stream, pdl);
    if (!lrc) lrc = wc_rmsnorm_gated_launch(H, D, o, gate, k->dN, d->eps, o, S.stream, pdl);
    if (!lrc) lrc = qt_launch(&d->o, o, y);
    if (lrc) return -1;
    const wc_copy_args cout = { { g_kda_pin }, { y }, { (size_t)hid * 4 }, 1, 1 };
    return small_copies(&cout, cudaMemcpyDeviceToHost) == cudaSuccess ? 0 : -1;
}

int waste_cuda_kda_layer(const waste_cuda_kda_layer_desc *d, const float *in, float *out)
{
    int rc = 0;
    if (!d || !in || !out || d->H <= 0 || d->hidden <= 0 || d->conv_k < 1 ||
        wc_kda_supported(d->D, d->D) || !d->S || !d->A_log || !d->o_norm)
        return fail(WASTE_CUDA_E_ARG, "kda_layer: bad descriptor (D 32, 64 or 128)");
    const int H = d->H, D = d->D, C = H * D, hid = d->hidden, KS = d->conv_k;
    pthread_mutex_lock(&g_mu);
    if (!S.inited && (rc = init_locked(-1))) goto out;
    {
        struct kda_ctx k;
        k.d = d;
        k.dS = (float *)rs_get(d->S, (size_t)H * D * D * sizeof(float));
        k.dA = (float *)rs_get(d->A_log, (size_t)H * sizeof(float));
        k.dB = d->dt_bias ? (float *)rs_get(d->dt_bias, (size_t)C * sizeof(float)) : NULL;
        k.dN = (float *)rs_get(d->o_norm, (size_t)D * sizeof(float));
        int ok = k.dS && k.dA && k.dN && (!d->dt_bias || k.dB);
        for (int i = 0; i < 3 && ok; i++) {
            k.dw[i] = d->conv_w[i] ? (float *)rs_get(d->conv_w[i], (size_t)C * KS * sizeof(float))
                                   : NULL;
            k.dr[i] = KS > 1 && d->conv_ring[i]
                          ? (float *)rs_get(d->conv_ring[i], (size_t)C * (KS - 1) * sizeof(float))
                          : NULL;
            ok = k.dw[i] && (KS == 1 || k.dr[i]);
        }
        if (!ok) { rc = fail(WASTE_CUDA_E_NOMEM, "kda_layer: device copies"); goto out; }
        const size_t n = (size_t)hid + 6 * (size_t)C + H + 2 * (size_t)D + hid;
        if ((rc = kda_stage(n))) goto out;
        if (branches_ready()) { rc = fail(WASTE_CUDA_E_DEVICE, "kda_layer: side streams"); goto out; }
        memcpy(g_kda_pin, in, (size_t)hid * 4);
        if (run_layer(d, kda_enqueue, &k)) {
            rc = fail(WASTE_CUDA_E_DEVICE, "kda_layer: a launch or a tensor copy failed");
            goto out;
        }
        CK(cudaStreamSynchronize(S.stream), "kda_layer");
        memcpy(out, g_kda_pin, (size_t)hid * 4);
    }
out:
    pthread_mutex_unlock(&g_mu);
    return rc;
}

/* ---- MLA: the whole attention layer, its latent cache in HBM ------------- */

static int mla_stage(size_t floats)
{
    if (floats <= g_mla_cap) return 0;
    g_epoch++;
    cudaFreeHost(g_mla_pin);
    cudaFree(g_mla_dev);
    g_mla_pin = g_mla_dev = NULL;
    g_mla_cap = 0;
    if (cudaMallocHost((void **)&g_mla_pin, floats * sizeof(float)) != cudaSuccess ||
        cudaMalloc((void **)&g_mla_dev, floats * sizeof(float)) != cudaSuccess) {
        cudaGetLastError();
        return fail(WASTE_CUDA_E_NOMEM, "MLA staging");
    }
    g_mla_cap = floats;
    return 0;
}

struct mla_ctx {
    const waste_cuda_mla_layer_desc *d;
    float *dlat, *dkvn, *dqan;
    uint8_t *kW;
    uint16_t *kws;
    int kng, S_max;
    size_t n_in, n_out;
};

/* The layer's device work on S.stream: x, the rope tables and the
 * position in from the pinned staging, the kernels, y and the new latent
 * row out to it. Nothing here depends on the position except through the
 * staged word, so one graph serves every position. */
static int mla_enqueue(void *p)
{
    const struct mla_ctx *k = (const struct mla_ctx *)p;
    const waste_cuda_mla_layer_desc *d = k->d;
    const int nh = d->heads, qd = d->qk_nope + d->qk_rope, vh = d->v_head, kl = d->kv_lora;
    const int latd = kl + d->qk_rope, hid = d->hidden, half = d->nope ? 0 : d->qk_rope / 2;
    /* staging: in x | cs | sn | pos ; out y | latent row ; work q | c | q_a | o | g */
    float *x = g_mla_dev, *cs = x + hid, *sn = cs + half;
    const int *pos_d = (const int *)(sn + half);
    float *y = x + k->n_in, *lrow = y + hid;
    float *q = lrow + latd, *ckv = q + (size_t)nh * qd, *qa = ckv + latd;
    float *o = qa + d->q_lora, *g = o + (size_t)nh * vh;
    const wc_copy_args cin = { { x }, { g_mla_pin }, { k->n_in * 4 }, 1, 0 };
    if (small_copies(&cin, cudaMemcpyHostToDevice) != cudaSuccess) return -1;
    /* the query, the latent and the gate read only x: side by side */
    int lrc = fork_branches(3);
    if (!lrc && d->q_lora > 0) {
        lrc = qt_launch_on(&d->q_a, x, qa, g_side[0], 0);
        if (!lrc) lrc = wc_mla_prep_launch(qa, d->q_lora, k->dqan, d->eps, NULL, NULL, NULL, 0,
                                           NULL, 0, 0, 0, NULL, NULL, NULL, 0, g_side[0]);
        if (!lrc) lrc = qt_launch_on(&d->q_b, qa, q, g_side[0], 0);
    } else if (!lrc) {
        lrc = qt_launch_on(&d->q, x, q, g_side[0], 0);
    }
    if (!lrc) lrc = qt_launch_on(&d->kv_a, x, ckv, g_side[1], 0);
    if (!lrc && d->g.W) lrc = qt_launch_on(&d->g, x, g, g_side[2], 0);
    if (!lrc) lrc = join_branches(3);
    if (!lrc) lrc = wc_mla_prep_launch(ckv, kl, k->dkvn, d->eps, ckv + kl, cs, sn, half, q, nh, qd,
                                       d->qk_nope, k->dlat, pos_d, lrow, latd, S.stream);
    /* prep → head → gate → o_proj programmatically (not under the phase
     * timers): the head's row staging and the projection's weight copies
     * overlap the kernel before each */
    const int pdl = !wc_profiling();
    if (!lrc) lrc = wc_mla_head_launch(q, k->dlat, pos_d, k->S_max, latd, kl, qd, d->qk_nope,
                                       d->qk_rope, vh, nh, k->kW, k->kws, d->kv_b.rowbytes, k->kng,
                                       d->kv_b.group, d->kv_b.bits, d->scale, o, S.stream, pdl);
    if (!lrc && d->g.W) lrc = wc_mla_gate_launch(o, g, nh * vh, S.stream, pdl);
    if (!lrc) lrc = qt_launch(&d->o, o, y);
    if (lrc) return -1;
    const wc_copy_args cout = { { g_mla_pin + k->n_in }, { y }, { k->n_out * 4 }, 1, 1 };
    return small_copies(&cout, cudaMemcpyDeviceToHost) == cudaSuccess ? 0 : -1;
}

int waste_cuda_mla_layer(const waste_cuda_mla_layer_desc *d, int pos, const float *in, float *out)
{
    int rc = 0;
    if (!d || !in || !out || d->heads <= 0 || d->hidden <= 0 || d->kv_lora <= 0 ||
        d->kv_lora > 4096 || d->qk_nope <= 0 || d->qk_rope < 0 || (d->qk_rope & 1) ||
        d->v_head <= 0 || !d->latcache || !d->kv_a_norm || pos < 0 || pos >= d->kv_cap ||
        !d->kv_b.W || (d->kv_b.bits != 8 && d->kv_b.bits != 4) || d->kv_b.cols != d->kv_lora ||
        d->kv_b.rows != d->heads * (d->qk_nope + d->v_head) || !d->kv_a.W || !d->o.W ||
        (d->q_lora > 0 ? (!d->q_a.W || !d->q_b.W || !d->q_a_norm || d->q_lora > 4096) : !d->q.W) ||
        (!d->nope && d->qk_rope > 0 && !d->rope_inv_freq))
        return fail(WASTE_CUDA_E_ARG, "mla_layer: bad descriptor or position");
    const int nh = d->heads, qd = d->qk_nope + d->qk_rope, vh = d->v_head, kl = d->kv_lora;
    const int latd = kl + d->qk_rope, hid = d->hidden, half = d->nope ? 0 : d->qk_rope / 2;
    /* the head kernel's shared memory sized for the whole cache (one graph
     * for every position), or else for this call's rows (launched directly) */
    const int wrows = d->qk_nope + vh, kng_ = (kl + d->kv_b.group - 1) / d->kv_b.group;
    const int whole = wc_mla_head_smem(qd, kl, d->kv_cap, wrows, d->kv_b.rowbytes, kng_) <= 200u * 1024;
    const int S_max = whole ? d->kv_cap : pos + 1;
    if (wc_mla_head_smem(qd, kl, S_max, wrows, d->kv_b.rowbytes, kng_) > 200u * 1024)
        return fail(WASTE_CUDA_E_ARG, "mla_layer: %d positions exceed the head kernel's "
                    "shared memory", pos + 1);
    pthread_mutex_lock(&g_mu);
    if (!S.inited && (rc = init_locked(-1))) goto out;
    {
        struct mla_ctx k;
        k.d = d;
        k.S_max = S_max;
        k.dlat = (float *)rs_get(d->latcache, (size_t)d->kv_cap * latd * sizeof(float));
        k.dkvn = (float *)rs_get(d->kv_a_norm, (size_t)kl * sizeof(float));
        k.dqan = d->q_lora > 0 ? (float *)rs_get(d->q_a_norm, (size_t)d->q_lora * 4) : NULL;
        if (!k.dlat || !k.dkvn || (d->q_lora > 0 && !k.dqan) ||
            qt_dev(&d->kv_b, &k.kW, &k.kws, &k.kng)) {
            rc = fail(WASTE_CUDA_E_NOMEM, "mla_layer: device copies");
            goto out;
        }
        k.n_in = (size_t)hid + 2 * (size_t)half + 1;
        k.n_out = (size_t)hid + latd;
        const size_t n = k.n_in + k.n_out + (size_t)nh * qd + latd + (size_t)d->q_lora +
                         2 * (size_t)nh * vh;
        if ((rc = mla_stage(n))) goto out;
        if (branches_ready()) { rc = fail(WASTE_CUDA_E_DEVICE, "mla_layer: side streams"); goto out; }
        memcpy(g_mla_pin, in, (size_t)hid * 4);
        for (int j = 0; j < half; j++) {        /* src/model.c:2502-2510, on the host's libm */
            const float a = (float)pos * d->rope_inv_freq[j];
            g_mla_pin[hid + j] = cosf(a);
            g_mla_pin[hid + half + j] = sinf(a);
        }
        memcpy(g_mla_pin + hid + 2 * half, &pos, sizeof(int));
        if (whole ? run_layer(d, mla_enqueue, &k) : mla_enqueue(&k)) {
            rc = fail(WASTE_CUDA_E_DEVICE, "mla_layer: a launch or a tensor copy failed");
            goto out;
        }
        CK(cudaStreamSynchronize(S.stream), "mla_layer");
        memcpy(out, g_mla_pin + k.n_in, (size_t)hid * 4);
        /* the engine's own copy of the cache row (its snapshot save reads it) */
        memcpy(d->latcache + (size_t)pos * latd, g_mla_pin + k.n_in + hid, (size_t)latd * 4);
    }
out:
    pthread_mutex_unlock(&g_mu);
    return rc;
}

/* The slots: the device, or — when it cannot take the call — the CPU
 * kernel the slot held before, on the host copy brought up to date first
 * and pushed back after. */
static void kda_slot(int H, int K, int V, const float *q, const float *k, const float *v,
                     const float *g_log, const float *beta, float *S_, float *o, float *scratch)
{
    if (waste_cuda_kda_step(H, K, V, q, k, v, g_log, beta, S_, o) == 0) return;
    const size_t b = (size_t)H * K * V * sizeof(float);
    waste_cuda_state_pull(S_, b);
    g_kda_cpu(H, K, V, q, k, v, g_log, beta, S_, o, scratch);
    waste_cuda_state_push(S_, b);
}

static void conv_slot(int C, int KS, const float *w, const float *bias, float *ring,
                      const float *x, float *y)
{
    if (waste_cuda_short_conv_step(C, KS, w, bias, ring, x, y) == 0) return;
    const size_t b = (size_t)C * (KS > 1 ? KS - 1 : 0) * sizeof(float);
    if (b) waste_cuda_state_pull(ring, b);
    g_conv_cpu(C, KS, w, bias, ring, x, y);
    if (b) waste_cuda_state_push(ring, b);
}

static void rmsg_slot(int C, const float *x, const float *gate, const float *weight, float eps,
                      float *y)
{
    if (waste_cuda_rmsnorm_gated_heads(1, C, x, gate, weight, eps, y) == 0) return;
    g_rmsg_cpu(C, x, gate, weight, eps, y);
}

/* The engine's per-layer loop of rmsnorm_gated over its heads as one call
 * (a slot of waste_vq_slots, used when WASTE_CUDA_KDA_NORM is set). */
static void rmsg_heads_slot(int nh, int C, const float *x, const float *gate,
                            const float *weight, float eps, float *y)
{
    if (waste_cuda_rmsnorm_gated_heads(nh, C, x, gate, weight, eps, y) == 0) return;
    for (int h = 0; h < nh; h++)
        g_rmsg_cpu(C, x + (size_t)h * C, gate + (size_t)h * C, weight, eps, y + (size_t)h * C);
}

static void state_push_slot(const void *host, size_t bytes) { waste_cuda_state_push(host, bytes); }

/* The whole-layer slot: moe_layer on the device for one token. */
static int moe_layer_slot(int layer, const float *x, float *out, int *routed)
{
    return waste_cuda_moe_layer(layer, x, out, routed, NULL);
}
static void state_pull_slot(void *host, size_t bytes) { waste_cuda_state_pull(host, bytes); }


int waste_cuda_mvq_rows_dev(float *d_y, const void *d_W, const uint16_t *d_ws, const float *d_x,
                            int r0, int r1, int in, int group, int bits, size_t rowbytes,
                            void *stream)
{
    if (!d_y || !d_W || !d_ws || !d_x || r0 < 0 || r1 <= r0 || in <= 0 || group <= 0 ||
        (bits != 8 && bits != 4 && bits != 3) || rowbytes == 0)
        return fail(WASTE_CUDA_E_ARG, "mvq_rows_dev: bad arguments");
    int rc = 0;
    pthread_mutex_lock(&g_mu);
    if (!S.inited) { rc = fail(WASTE_CUDA_E_NODEV, "mvq_rows_dev before waste_cuda_init"); goto out; }
    {
        const int ng = (in + group - 1) / group;
        wc_mvq_args k = { d_y, (const uint8_t *)d_W, d_ws, d_x, r0, r1, in, ng, group, bits,
                          rowbytes, 0 };
        CK((cudaError_t)wc_mvq_launch(&k, stream ? stream : (void *)S.stream), "trunk matvec");
    }
out:
    pthread_mutex_unlock(&g_mu);
    return rc;
}

static int slot_bank_load(int layer, int n_experts, size_t rec_bytes, int first,
                          int count, const void *records, int inter, int lat,
                          int stages)
{
    return waste_cuda_vq_bank_load(layer, n_experts, rec_bytes, first, count,
                                   records, inter, lat, stages);
}

int waste_register_cuda_vq(waste_vq_slots *s)
{
    if (!s) return WASTE_CUDA_E_ARG;
    memset(s, 0, sizeof *s);
    if (!S.inited && waste_cuda_init(-1) != 0) return WASTE_CUDA_E_NODEV;
    s->codebooks_load = waste_cuda_codebooks_load;
    s->vq_bank_load = slot_bank_load;
    s->vq_bank_free = waste_cuda_vq_bank_free;
    s->moe_experts = waste_cuda_moe_experts;
    s->moe_chunk_experts = waste_cuda_moe_chunk_experts;
    s->vq_bank_load_file = waste_cuda_vq_bank_load_file;
    s->state_push = state_push_slot;
    s->state_pull = state_pull_slot;
    s->moe_trunk_load = waste_cuda_moe_trunk_load;
    s->moe_activation = waste_cuda_moe_activation;
    if (getenv_flag("WASTE_CUDA_MOE_LAYER", 1)) s->moe_layer = moe_layer_slot;
    if (getenv_flag("WASTE_CUDA_KDA", 1) && getenv_flag("WASTE_CUDA_KDA_LAYER", 1))
        s->kda_layer = waste_cuda_kda_layer;
    if (getenv_flag("WASTE_CUDA_MLA_LAYER", 1)) s->mla_layer = waste_cuda_mla_layer;
    if (g_rmsg_cpu && getenv_flag("WASTE_CUDA_KDA_NORM", 0)) s->rmsnorm_gated_heads = rmsg_heads_slot;
    return 0;
}

/* ---- codebooks --------------------------------------------------------- */

static int books_upload(const float *books, int n_books, int entries)
{
    int rc = 0;
    float *pad = NULL;
    g_epoch++;
    const size_t bytes = (size_t)n_books * 256 * 8 * sizeof(float);
    if (S.d_books) { cudaFree(S.d_books); S.d_books = NULL; S.n_books = 0; }
    if (entries != 256) {
        /* every book keeps a 256-entry slot; a 64-entry book fills the
         * first 64 and the rest stays zero */
        pad = (float *)calloc((size_t)n_books * 256 * 8, sizeof(float));
        if (!pad) return fail(WASTE_CUDA_E_NOMEM, "codebook staging");
        for (int b = 0; b < n_books; b++)
            memcpy(pad + (size_t)b * 256 * 8, books + (size_t)b * entries * 8,
                   (size_t)entries * 8 * sizeof(float));
        books = pad;
    }
    free(S.book_absmax);
    S.book_absmax = (float *)calloc((size_t)n_books, sizeof(float));
    if (!S.book_absmax) { rc = fail(WASTE_CUDA_E_NOMEM, "codebook maxima"); goto out; }
    /* per-book maxima (the tensor-core path's weight pre-scale), and whether
     * every entry is exact in fp16 (normal or zero), which that path needs */
    S.books_f16 = 1;
    for (int b = 0; b < n_books; b++)
        for (size_t i = 0; i < 256 * 8; i++) {
            const float v = books[(size_t)b * 256 * 8 + i];
            uint32_t bits;
            memcpy(&bits, &v, 4);
            const uint32_t ex = (bits >> 23) & 0xff;
            if (v != 0.0f && (ex < 113 || ex > 142 || (bits & 0x1fff))) S.books_f16 = 0;
            const float m = v < 0 ? -v : v;
            if (m > S.book_absmax[b]) S.book_absmax[b] = m;
        }
    CK(cudaMalloc((void **)&S.d_books, bytes), "codebooks");
    CK(h2d_now(S.d_books, books, bytes), "codebooks H2D");
    S.n_books = n_books;
    S.cb_entries = entries;
out:
    free(pad);
    return rc;
}

int waste_cuda_codebooks_load(const float *books, int n_books, int entries, int vec_dim)
{
    if (!books || n_books <= 0 || (entries != 256 && entries != 64) || vec_dim != 8)
        return fail(WASTE_CUDA_E_ARG, "codebooks: need entries 256 (VQ3R) or 64 (VQ4P), "
                    "vec_dim 8");
    pthread_mutex_lock(&g_mu);
    int rc = S.inited ? 0 : init_locked(-1);
    if (!rc) rc = books_upload(books, n_books, entries);
    pthread_mutex_unlock(&g_mu);
    return rc;
}

/* The loader's decode, src/model.c:1278-1287: f16 -> f32 keeping the sign,
 * with exponent 0 (zero and every subnormal) flushed to zero. */
static float f16_flush(uint16_t v)
{
    const uint32_t sign = (uint32_t)(v >> 15) << 31;
    const uint32_t e = (v >> 10) & 0x1f, man = v & 0x3ff;
    const uint32_t bits = e ? (sign | ((e + 112u) << 23) | (man << 13)) : sign;
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

int waste_cuda_codebooks_load_f16(const uint16_t *raw, int n_books, int entries, int vec_dim)
{
    if (!raw || n_books <= 0 || (entries != 256 && entries != 64) || vec_dim != 8)
        return fail(WASTE_CUDA_E_ARG, "codebooks: need entries 256 (VQ3R) or 64 (VQ4P), "
                    "vec_dim 8");
    const size_t n = (size_t)n_books * entries * vec_dim;
    float *f = (float *)malloc(n * sizeof(float));
    if (!f) return fail(WASTE_CUDA_E_NOMEM, "codebook staging");
    for (size_t i = 0; i < n; i++) f[i] = f16_flush(raw[i]);
    const int rc = waste_cuda_codebooks_load(f, n_books, entries, vec_dim);
    free(f);
    return rc;
}

/* ---- expert banks ------------------------------------------------------- */

/* src/model.c:1698-1745 record_check, without the optional crc32. */
static int check_record(const wc_hdr *h, int layer, int expert, size_t rec_bytes,
                        int stages, int inter, int lat)
{
    if (rec_bytes < sizeof *h || h->magic != WC_MAGIC_EXPERT) return -1;
    if (h->layer != (uint16_t)layer || h->expert_id != (uint16_t)expert) return -1;
    if ((size_t)h->rec_4k_blocks * WC_ALIGN != rec_bytes) return -1;
    /* the fmt byte and the layer's format agree (src/model.c:1713-1719):
     * VQ4P with four stages of 64-entry books, else VQ3R/VQ2R with 256 */
    if (stages == 4 ? (h->fmt != WC_WQ_VQ4P || S.cb_entries != 64)
                    : ((h->fmt != WC_WQ_VQ3R && h->fmt != WC_WQ_VQ2R) || S.cb_entries != 256))
        return -1;
    if (h->lowrank_id != 0) return -1;
    if ((long)h->codebook_id + 3L * stages > S.n_books) return -1;
    if (!(h->gate_off == sizeof *h && h->gate_off < h->up_off &&
          h->up_off < h->down_off && h->down_off < h->chan_corr_off &&
          h->chan_corr_off <= rec_bytes))
        return -1;
    const size_t scales = 2u * (size_t)(2 * inter + lat);
    if (scales > rec_bytes - h->chan_corr_off) return -1;
    /* the index streams must fit before the next section */
    const size_t nrb_i = (size_t)(inter + 63) / 64, nrb_l = (size_t)(lat + 63) / 64;
    const size_t per = stages == 4 ? 3 : (size_t)stages;   /* index bytes per row and position */
    const size_t gate_b = nrb_i * 64 * (lat / 8) * per;
    const size_t down_b = nrb_l * 64 * (inter / 8) * per;
    if (h->up_off - h->gate_off < gate_b || h->down_off - h->up_off < gate_b ||
        h->chan_corr_off - h->down_off < down_b)
        return -1;
    /* 16-byte loads of the index streams */
    if ((h->gate_off | h->up_off | h->down_off) & 15) return -1;
    return 0;
}

/* Contiguous split of n experts over `world` ranks: rank r holds
 * [r*n/world, (r+1)*n/world). */
static void split_range(int n, int rank, int world, int *first, int *count)
{
    const int lo = (int)((long long)rank * n / world);
    const int hi = (int)((long long)(rank + 1) * n / world);
    *first = lo;
    *count = hi - lo;
}

int waste_cuda_ep_range(int n_experts, int rank, int world, int *first, int *count)
{
    if (n_experts <= 0 || world <= 0 || rank < 0 || rank >= world || !first || !count)
        return fail(WASTE_CUDA_E_ARG, "ep_range: bad arguments");
    split_range(n_experts, rank, world, first, count);
    return 0;
}

/* cuTensorMapEncodeTiled, reached through the runtime (no -lcuda). */
typedef CUresult (*wc_encode_tiled_fn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                       const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                       const cuuint32_t *, CUtensorMapInterleave,
                                       CUtensorMapSwizzle, CUtensorMapL2promotion,
                                       CUtensorMapFloatOOBfill);

static wc_encode_tiled_fn encode_tiled(void)
{
    static wc_encode_tiled_fn fn;
    static int tried;
    if (!tried) {
        tried = 1;
        void *p = NULL;
        enum cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess && q == cudaDriverEntryPointSuccess)
            fn = (wc_encode_tiled_fn)p;
    }
    return fn;
}

/* The bank's index streams as 3-D tensors of 8-byte elements: {positions of
 * a row block * 24, 64-row blocks, experts held}, strides {row block,
 * record}. Box: one decode tile's positions by half the row blocks
 * (gate/up) or all of them (down). Leaves tmap_ok = 0 when a shape does not
 * fit (the kernels then copy row block by row block). */
static void bank_tensor_maps(wc_bank *kb)
{
    kb->tmap_ok = 0;
    wc_encode_tiled_fn enc = encode_tiled();
    if (!enc) return;
    const int nv_gu = kb->lat / 8, nrb_gu = (kb->inter + 63) / 64;
    const int nv_d = kb->inter / 8, nrb_d = (kb->lat + 63) / 64;
    const int vs_gu = wc_vs_gateup(kb->lat, kb->inter);
    if (nv_gu % vs_gu || nv_d % WC_VS_DOWN || nrb_gu % 2 || nrb_gu / 2 > 256 ||
        nrb_d > 256 || WC_VS_DOWN * 24 > 256 || vs_gu * 24 > 256 || kb->stages != 3)
        return;
    const uint32_t off[3] = { kb->gate_off, kb->up_off, kb->down_off };
    for (int k = 0; k < 3; k++) {
        const int nv = k < 2 ? nv_gu : nv_d, nrb = k < 2 ? nrb_gu : nrb_d;
        const cuuint64_t dims[3] = { (cuuint64_t)nv * 24, (cuuint64_t)nrb,
                                     (cuuint64_t)kb->n_experts };
        const cuuint64_t strides[2] = { (cuuint64_t)nv * 192, (cuuint64_t)kb->rec_bytes };
        const cuuint32_t box[3] = { (cuuint32_t)(k < 2 ? vs_gu : WC_VS_DOWN) * 24,
                                    (cuuint32_t)(k < 2 ? nrb / 2 : nrb), 1 };
        const cuuint32_t estr[3] = { 1, 1, 1 };
        void *base = (void *)(kb->base + off[k]);
        if (((uintptr_t)base & 15) ||
            enc(&kb->tmap[k], CU_TENSOR_MAP_DATA_TYPE_UINT64, 3, base, dims, strides, box, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) !=
                CUDA_SUCCESS)
            return;
    }
    kb->tmap_ok = 1;
}

/* HBM for records [first, first+count) of a layer of n_experts; the caller
 * holds g_mu and has checked the shape arguments. */
static int reserve_locked(int layer, int n_experts, size_t rec_bytes, int first, int count,
                          int inter, int lat, int stages)
{
    int rc = 0;
    g_epoch++;
    wc_layer *L = &S.layer[layer];
    if (L->d_base) {
        if (L->n_total != n_experts || L->kb.rec_bytes != rec_bytes || L->kb.inter != inter ||
            L->kb.lat != lat || L->kb.stages != stages || L->kb.first != first ||
            L->kb.n_experts != count)
            return fail(WASTE_CUDA_E_ARG, "layer %d: bank shape or range differs from the "
                        "first reservation", layer);
        return 0;
    }
    free(L->present);
    L->present = (uint8_t *)calloc((size_t)count, 1);
    L->n_present = 0;
    if (!L->present) return fail(WASTE_CUDA_E_NOMEM, "bank index");
    CK(cudaMalloc((void **)&L->d_base, rec_bytes * (size_t)count), "bank");
    L->n_total = n_experts;
    L->kb.rec_bytes = rec_bytes;
    L->kb.inter = inter;
    L->kb.lat = lat;
    L->kb.stages = stages;
    L->kb.n_experts = count;
    L->kb.first = first;
    L->kb.base = L->d_base;
out:
    return rc;
}

static int bank_args_ok(int layer, int n_experts, size_t rec_bytes, int first, int count,
                        int inter, int lat, int stages)
{
    return layer >= 0 && layer < WC_MAX_LAYERS && n_experts > 0 && first >= 0 && count > 0 &&
           first + count <= n_experts && rec_bytes > 0 && rec_bytes % WC_ALIGN == 0 &&
           inter > 0 && lat > 0 && inter % 8 == 0 && lat % 8 == 0 &&
           (stages == 2 || stages == 3 || stages == 4);
}

int waste_cuda_vq_bank_reserve(int layer, int n_experts, size_t rec_bytes, int first,
                               int count, int inter, int lat, int stages)
{
    int rc = 0;
    if (!bank_args_ok(layer, n_experts, rec_bytes, first, count, inter, lat, stages))
        return fail(WASTE_CUDA_E_ARG, "vq_bank_reserve: bad arguments");
    pthread_mutex_lock(&g_mu);
    if (!S.inited && (rc = init_locked(-1))) goto out;
    rc = reserve_locked(layer, n_experts, rec_bytes, first, count, inter, lat, stages);
out:
    pthread_mutex_unlock(&g_mu);
    return rc;
}

/* Records [first, first+count) of a layer from host memory: every header
 * checked, the layer's bank reserved at its first load, then one copy —
 * synchronous, or (copy_stream set: records in pinned memory) ordered on
 * copy_stream. Under g_mu. */
static int bank_load_locked(int layer, int n_experts, size_t rec_bytes, int first, int count,
                            const void *records, int inter, int lat, int stages,
                            cudaStream_t copy_stream)
{
    int rc = 0;
    if (!S.inited && (rc = init_locked(-1))) goto out;
    if (!S.d_books) { rc = fail(WASTE_CUDA_E_ARG, "load codebooks before banks"); goto out; }
    wc_layer *L = &S.layer[layer];
    /* check every header before anything is reserved or copied */
    for (int i = 0; i < count; i++) {
        const wc_hdr *h = (const wc_hdr *)((const uint8_t *)records + (size_t)i * rec_bytes);
        if (check_record(h, layer, first + i, rec_bytes, stages, inter, lat)) {
            rc = fail(WASTE_CUDA_E_RECORD, "layer %d expert %d: record header is not "
                      "what the bank index describes", layer, first + i);
            goto out;
        }
        const wc_hdr *h0 = L->have_hdr ? NULL : (const wc_hdr *)records;
        const uint32_t go = h0 ? h0->gate_off : L->kb.gate_off;
        const uint32_t uo = h0 ? h0->up_off : L->kb.up_off;
        const uint32_t dof = h0 ? h0->down_off : L->kb.down_off;
        const uint32_t so = h0 ? h0->chan_corr_off : L->kb.scale_off;
        const int cb = h0 ? h0->codebook_id : L->kb.cb_base;
        if (h->gate_off != go || h->up_off != uo || h->down_off != dof ||
            h->chan_corr_off != so || h->codebook_id != cb) {
            rc = fail(WASTE_CUDA_E_RECORD, "layer %d expert %d: payload offsets or "
                      "codebook_id differ from the layer's first record", layer, first + i);
            goto out;
        }
    }
    if (!L->d_base) {
        /* first load of the layer: the whole layer, or this rank's range */
        int r0 = 0, rn = n_experts;
        if (EP.active) split_range(n_experts, EP.rank, EP.world, &r0, &rn);
        if ((rc = reserve_locked(layer, n_experts, rec_bytes, r0, rn, inter, lat, stages)))
            goto out;
    } else if (L->n_total != n_experts || L->kb.rec_bytes != rec_bytes ||
               L->kb.inter != inter || L->kb.lat != lat || L->kb.stages != stages) {
        rc = fail(WASTE_CUDA_E_ARG, "layer %d: bank shape differs from the first load", layer);
        goto out;
    }
    if (first < L->kb.first || first + count > L->kb.first + L->kb.n_experts) {
        rc = fail(WASTE_CUDA_E_ARG, "layer %d: records [%d, %d) fall outside the experts "
                  "this bank holds, [%d, %d)", layer, first, first + count, L->kb.first,
                  L->kb.first + L->kb.n_experts);
        goto out;
    }
    if (!L->have_hdr) {
        const wc_hdr *h0 = (const wc_hdr *)records;
        L->kb.gate_off = h0->gate_off;
        L->kb.up_off = h0->up_off;
        L->kb.down_off = h0->down_off;
        L->kb.scale_off = h0->chan_corr_off;
        L->kb.cb_base = h0->codebook_id;
        L->have_hdr = 1;
        bank_tensor_maps(&L->kb);
    }
    const int at = first - L->kb.first;
    if (copy_stream)
        CK(cudaMemcpyAsync(L->d_base + (size_t)at * rec_bytes, records, rec_bytes * (size_t)count,
                           cudaMemcpyHostToDevice, copy_stream), "bank H2D");
    else
        CK(h2d_now(L->d_base + (size_t)at * rec_bytes, records, rec_bytes * (size_t)count),
           "bank H2D");
    for (int i = at; i < at + count; i++) {
        L->n_present += !L->present[i];
        L->present[i] = 1;
    }
    L->loaded = 1;
out:
    return rc;
}

int waste_cuda_vq_bank_load(int layer, int n_experts, size_t rec_bytes, int first,
                            int count, const void *records, int inter, int lat,
                            int stages)
{
    if (!records || !bank_args_ok(layer, n_experts, rec_bytes, first, count, inter, lat, stages))
        return fail(WASTE_CUDA_E_ARG, "vq_bank_load: bad arguments");
    pthread_mutex_lock(&g_mu);
    const int rc = bank_load_locked(layer, n_experts, rec_bytes, first, count, records, inter,
                                    lat, stages, NULL);
    pthread_mutex_unlock(&g_mu);
    return rc;
}

int waste_cuda_vq_bank_load_file(int layer, int fd, int64_t offset, int n_experts,
                                 size_t rec_bytes, int first, int count, int inter, int lat,
                                 int stages)
{
    int rc = 0;
    if (fd < 0 || offset < 0 || !bank_args_ok(layer, n_experts, rec_bytes, first, count, inter,
                                                lat, stages))
        return fail(WASTE_CUDA_E_ARG, "vq_bank_load_file: bad arguments");
    pthread_mutex_lock(&g_mu);
    if (!S.inited && (rc = init_locked(-1))) goto out;
    /* whole records per range, at least one; the buffers are page aligned
     * (pinned allocations), so files opened for direct I/O read too */
    size_t per = WC_STAGE_BYTES / rec_bytes;
    if (per < 1) per = 1;
    const size_t need = per * rec_bytes;
    if (need > g_stage.bytes) {
        for (int b = 0; b < 2; b++) {
            if (g_stage.ev) cudaEventSynchronize(g_stage.done[b]);
            cudaFreeHost(g_stage.buf[b]);
            g_stage.buf[b] = NULL;
        }
        g_stage.bytes = 0;
        for (int b = 0; b < 2; b++)
            CK(cudaMallocHost((void **)&g_stage.buf[b], need), "bank staging");
        g_stage.bytes = need;
    }
    if (!g_stage.ev) {
        for (int b = 0; b < 2; b++)
            CK(cudaEventCreateWithFlags(&g_stage.done[b], cudaEventDisableTiming), "staging event");
        g_stage.ev = 1;
    }
    for (int e0 = 0, k = 0; e0 < count; e0 += (int)per, k++) {
        const int n = count - e0 < (int)per ? count - e0 : (int)per;
        const int b = k & 1;
        CK(cudaEventSynchronize(g_stage.done[b]), "staging reuse");   /* its last copy is done */
        size_t got = 0;
        const size_t want = (size_t)n * rec_bytes;
        const int64_t at = offset + (int64_t)(first + e0) * (int64_t)rec_bytes;
        while (got < want) {
            const ssize_t r = pread(fd, g_stage.buf[b] + got, want - got, (off_t)(at + (int64_t)got));
            if (r <= 0) {
                rc = fail(WASTE_CUDA_E_ARG, "vq_bank_load_file: layer %d: short read at byte %lld",
                          layer, (long long)(at + (int64_t)got));
                goto drain;
            }
            got += (size_t)r;
        }
        if ((rc = bank_load_locked(layer, n_experts, rec_bytes, first + e0, n, g_stage.buf[b],
                                   inter, lat, stages, S.stream)))
            goto drain;
        CK(cudaEventRecord(g_stage.done[b], S.stream), "staging event");
    }
drain:
    cudaStreamSynchronize(S.stream);
out:
    pthread_mutex_unlock(&g_mu);
    return rc;
}

void waste_cuda_vq_bank_free(int layer)
{
    if (layer < 0 || layer >= WC_MAX_LAYERS) return;
    pthread_mutex_lock(&g_mu);
    if (S.inited) {
        cudaStreamSynchronize(S.stream);
        wc_layer *L = &S.layer[layer];
        g_epoch++;
        cudaFree(L->d_base);
        L->d_base = NULL;
        free(L->present);
        L->present = NULL;
        L->n_present = 0;
        L->loaded = L->have_hdr = 0;
        memset(&L->kb, 0, sizeof L->kb);
    }
    pthread_mutex_unlock(&g_mu);
}

int waste_cuda_moe_trunk_load(int layer, int n_experts, int hidden, int top_k,
                              int renorm, float routed_scale, const float *router,
                              const float *bias, int sh_inter, const int8_t *sh_gate,
                              const uint16_t *sh_gate_s, const int8_t *sh_up,
                              const uint16_t *sh_up_s, const int8_t *sh_down,
                              const uint16_t *sh_down_s)
{
    int rc = 0;
    if (layer < 0 || layer >= WC_MAX_LAYERS || n_experts <= 0 || n_experts > 4096 ||
        top_k < 1 || top_k > WC_MAX_TOPK || top_k > n_experts || hidden <= 0 ||
        !router || sh_inter < 0 ||
        (sh_inter > 0 && (!sh_gate || !sh_gate_s || !sh_up || !sh_up_s || !sh_down || !sh_down_s)))
        return fail(WASTE_CUDA_E_ARG, "moe_trunk_load: bad arguments");
    pthread_mutex_lock(&g_mu);
    if (!S.inited && (rc = init_locked(-1))) goto out;
    g_epoch++;
    wc_layer *L = &S.layer[layer];
    cudaFree(L->d_router); cudaFree(L->d_bias);
    cudaFree(L->d_shg); cudaFree(L->d_shu); cudaFree(L->d_shd);
    cudaFree(L->d_shg_s); cudaFree(L->d_shu_s); cudaFree(L->d_shd_s);
    L->d_router = L->d_bias = NULL;
    L->d_shg = L->d_shu = L->d_shd = NULL;
    L->d_shg_s = L->d_shu_s = L->d_shd_s = NULL;
    const size_t rb = (size_t)n_experts * hidden * sizeof(float);
    CK(cudaMalloc((void **)&L->d_router, rb), "router");
    CK(h2d_now(L->d_router, router, rb), "router H2D");
    if (bias) {
        CK(cudaMalloc((void **)&L->d_bias, (size_t)n_experts * sizeof(float)), "bias");
        CK(h2d_now(L->d_bias, bias, (size_t)n_experts * sizeof(float)), "bias H2D");
    }
    if (sh_inter > 0) {
        const int g = 128;
        const size_t ng_h = (size_t)(hidden + g - 1) / g, ng_s = (size_t)(sh_inter + g - 1) / g;
        const size_t gb = (size_t)sh_inter * ng_h * g, db = (size_t)hidden * ng_s * g;
        const size_t gs = (size_t)sh_inter * ng_h * 2, ds = (size_t)hidden * ng_s * 2;
        CK(cudaMalloc((void **)&L->d_shg, gb), "shared gate");
        CK(cudaMalloc((void **)&L->d_shu, gb), "shared up");
        CK(cudaMalloc((void **)&L->d_shd, db), "shared down");
        CK(cudaMalloc((void **)&L->d_shg_s, gs), "shared gate scales");
        CK(cudaMalloc((void **)&L->d_shu_s, gs), "shared up scales");
        CK(cudaMalloc((void **)&L->d_shd_s, ds), "shared down scales");
        CK(h2d_now(L->d_shg, sh_gate, gb), "H2D");
        CK(h2d_now(L->d_shu, sh_up, gb), "H2D");
        CK(h2d_now(L->d_shd, sh_down, db), "H2D");
        CK(h2d_now(L->d_shg_s, sh_gate_s, gs), "H2D");
        CK(h2d_now(L->d_shu_s, sh_up_s, gs), "H2D");
        CK(h2d_now(L->d_shd_s, sh_down_s, ds), "H2D");
    }
    L->trunk = 1;
    L->E = n_experts;
    L->hidden = hidden;
    L->top_k = top_k;
    L->renorm = renorm;
    L->routed_scale = routed_scale;
    L->si = sh_inter;
out:
    pthread_mutex_unlock(&g_mu);
    return rc;
}

int waste_cuda_moe_activation(int layer, int act, float situ_beta, float situ_linear_beta)
{
    if (layer < 0 || layer >= WC_MAX_LAYERS || (act != 0 && act != 1) ||
        (act == 1 && !(situ_beta > 0.0f)))
        return fail(WASTE_CUDA_E_ARG, "moe_activation: layer %d, act %d (0 SiLU, 1 SiTU with "
                    "beta > 0)", layer, act);
    pthread_mutex_lock(&g_mu);
    wc_layer *L = &S.layer[layer];
    g_epoch++;
    L->act = act;
    L->situ_beta = act ? situ_beta : 0.0f;
    L->situ_lbeta = act ? situ_linear_beta : 0.0f;
    pthread_mutex_unlock(&g_mu);
    return 0;
}

int waste_cuda_moe_norm_load(int layer, int hidden, const float *norm_w, float eps)
{
    int rc = 0;
    if (layer < 0 || layer >= WC_MAX_LAYERS || hidden <= 0 || !norm_w || !(eps >= 0.0f))
        return fail(WASTE_CUDA_E_ARG, "moe_norm_load: bad arguments");
    pthread_mutex_lock(&g_mu);
    if (!S.inited && (rc = init_locked(-1))) goto out;
    wc_layer *L = &S.layer[layer];
    if (!L->trunk || L->hidden != hidden) {
        rc = fail(WASTE_CUDA_E_ARG, "moe_norm_load: layer %d's trunk (width %d) is not "
                  "loaded, or its width is not %d", layer, L->hidden, hidden);
        goto out;
    }
    g_epoch++;
    cudaFree(L->d_norm);
    L->d_norm = NULL;
    CK(cudaMalloc((void **)&L->d_norm, (size_t)hidden * sizeof(float)), "norm weight");
    CK(h2d_now(L->d_norm, norm_w, (size_t)hidden * sizeof(float)), "norm weight H2D");
    L->norm_eps = eps;
out:
    pthread_mutex_unlock(&g_mu);
    return rc;
}

/* ---- expert loop ------------------------------------------------------- */

static int layer_ready(int layer, int lat, int inter, wc_layer **out)
{
    if (layer < 0 || layer >= WC_MAX_LAYERS || !S.layer[layer].loaded)
        return fail(WASTE_CUDA_E_NOBANK, "layer %d has no bank in HBM", layer);
    wc_layer *L = &S.layer[layer];
    if (lat != L->kb.lat || inter != L->kb.inter)
        return fail(WASTE_CUDA_E_ARG, "layer %d: call shape %dx%d, bank %dx%d", layer,
                    lat, inter, L->kb.lat, L->kb.inter);
    *out = L;
    return 0;
}

static int check_route(const wc_layer *L, const int *idx, int n)
{
    for (int i = 0; i < n; i++)
    {
        if (idx[i] < L->kb.first || idx[i] >= L->kb.first + L->kb.n_experts)
            return fail(WASTE_CUDA_E_ARG, "expert id %d outside the bank", idx[i]);
        if (!L->present[idx[i] - L->kb.first])
            return fail(WASTE_CUDA_E_ARG, "expert %d's record was not loaded here", idx[i]);
    }
    return 0;
}

static void fill_args(wc_moe_args *a, const wc_layer *L, int T, int K, int E, int si)
{
    memset(a, 0, sizeof *a);
    a->bank = L->kb;
    a->books = S.d_books;
    a->T = T;
    a->K = K;
    a->E = E;
    a->si = si;
    a->sh_t0 = 0;
    a->sh_t1 = T;
    a->partial_bank = L->kb.first != 0 || L->kb.n_experts != L->n_total;
    if (a->partial_bank && L->n_total > 0) {
        /* routed experts of a token expected here; at two or fewer most
         * gate/up tiles would be empty, so they become route-first tiles of
         * that many experts */
        const int eg = (int)(((long)K * L->kb.n_experts + L->n_total - 1) / L->n_total);
        a->gu_eg = eg <= 4 ? eg : 0;
    }
    wc_moe_ws_carve(&a->ws, S.d_ws, T, K, E, L->kb.lat, L->kb.inter, si, L->kb.stages);
}

static int run_experts(int layer, int T, int K, const int *idx, const float *w,
                       const float *x, float *ysum, int lat, int inter, int act,
                       float situ_beta, float situ_lbeta, int order_by_id)
{
    int rc = 0;
    wc_layer *L = NULL;
    if (T <= 0 || T > WC_CHUNK_MAX || K <= 0 || K > WC_MAX_TOPK || !idx || !w || !x || !ysum)
        return fail(WASTE_CUDA_E_ARG, "moe call: bad arguments");
    if (act != 0 && act != 1)
        return fail(WASTE_CUDA_E_ARG, "moe call: act %d (0 SiLU, 1 SiTU)", act);
    pthread_mutex_lock(&g_mu);
    if ((rc = layer_ready(layer, lat, inter, &L))) goto out;
    if ((rc = check_route(L, idx, T * K))) goto out;
    /* a VQ4P bank uses the io buffers and the error word, not the fused
     * kernels' workspace layout, which is sized here as for VQ3R */
    if ((rc = ensure_ws(T, K, 1, lat, inter, 0, L->kb.stages == 4 ? 3 : L->kb.stages))) goto out;
    const size_t xb = (size_t)T * lat * sizeof(float);
    memcpy(S.h_x, x, xb);
    memcpy(S.h_idx, idx, (size_t)T * K * sizeof(int));
    memcpy(S.h_w, w, (size_t)T * K * sizeof(float));
    {
        const wc_copy_args cin = { { S.d_x, S.d_idx, S.d_w, NULL }, { S.h_x, S.h_idx, S.h_w, NULL },
                                   { xb, (size_t)T * K * sizeof(int), (size_t)T * K * sizeof(float), 0 },
                                   3, 0 };
        CK(small_copies(&cin, cudaMemcpyHostToDevice), "x, route, weights in");
    }
    if (L->kb.stages == 4) {
        if ((rc = p6_experts(L, T, K, act, situ_beta, situ_lbeta, order_by_id))) goto out;
    } else if (order_by_id && pf_wanted(L, T, K)) {
        /* a chunk with enough tokens per expert: dense tiles on the tensor cores */
        wc_pf_args pa;
        if ((rc = pf_args(L, T, K, &pa))) goto out;
        pa.act = act;
        pa.situ_beta = situ_beta;
        pa.situ_lbeta = situ_lbeta;
        pa.route = S.d_idx;
        pa.rw = S.d_w;
        pa.x = S.d_x;
        pa.out = S.d_out;
        CK((cudaError_t)wc_pf_launch(&pa, S.stream), "prefill kernels");
    } else {
        wc_moe_args a;
        fill_args(&a, L, T, K, 1, 0);
        a.x = S.d_x;
        a.idx = S.d_idx;
        a.w = S.d_w;
        a.out = S.d_out;
        a.order_by_id = order_by_id;
        a.act = act;
        a.situ_beta = situ_beta;
        a.situ_lbeta = situ_lbeta;
        a.prefetch_down = 1;
        if (wc_moe_supported(&a)) { rc = fail(WASTE_CUDA_E_ARG, "expert shape outside the kernels' bounds"); goto out; }
        CK((cudaError_t)wc_moe_launch(&a, S.stream), "expert kernels");
    }
    {
        const wc_copy_args cout = { { S.h_out }, { S.d_out }, { xb }, 1, 0 };
        CK(small_copies(&cout, cudaMemcpyDeviceToHost), "ysum out");
    }
    CK(cudaStreamSynchronize(S.stream), "expert loop");
    if (read_device_errors(1)) {
        rc = fail(WASTE_CUDA_E_DEVICE, "layer %d: a bounded device wait gave up", layer);
        goto out;
    }
    memcpy(ysum, S.h_out, xb);
out:
    pthread_mutex_unlock(&g_mu);
    return rc;
}

int waste_cuda_moe_experts(const waste_moe_call *c)
{
    if (!c) return fail(WASTE_CUDA_E_ARG, "NULL call");
    return run_experts(c->layer, 1, c->K, c->idx, c->w, c->x, c->ysum, c->lat, c->inter,
                       c->act, c->situ_beta, c->situ_linear_beta, 0);
}

int waste_cuda_moe_chunk_experts(const waste_moe_chunk_call *c)
{
    if (!c) return fail(WASTE_CUDA_E_ARG, "NULL call");
    return run_experts(c->layer, c->nT, c->K, c->route, c->rw, c->x, c->ysum, c->lat,
                       c->inter, c->act, c->situ_beta, c->situ_linear_beta, 1);
}

/* ---- whole layer ----------------------------------------------------------- */

/* Arguments for T tokens through the device router. part = 0: the whole
 * layer, every expert held here. part = 1: the experts this bank holds (all
 * of its range loaded), the rest left to the ranks that hold them. */
static int layer_args(int layer, int T, int part, wc_moe_args *a, wc_layer **Lp)
{
    int rc;
    if (layer < 0 || layer >= WC_MAX_LAYERS || !S.layer[layer].loaded || !S.layer[layer].trunk)
        return fail(WASTE_CUDA_E_NOBANK, "layer %d: bank or trunk not loaded", layer);
    wc_layer *L = &S.layer[layer];
    if (L->kb.stages == 4)
        return fail(WASTE_CUDA_E_ARG, "layer %d: a VQ4P bank runs through moe_experts / "
                    "moe_chunk_experts only", layer);
    if (T <= 0 || T > WC_CHUNK_MAX)
        return fail(WASTE_CUDA_E_ARG, "layer %d: %d tokens, 1..%d per call", layer, T,
                    WC_CHUNK_MAX);
    if (L->hidden != L->kb.lat)
        return fail(WASTE_CUDA_E_ARG, "layer %d: router width %d != expert width %d", layer,
                    L->hidden, L->kb.lat);
    if (L->n_total != L->E)
        return fail(WASTE_CUDA_E_ARG, "layer %d: router has %d experts, bank %d", layer, L->E,
                    L->n_total);
    if (part ? L->n_present != L->kb.n_experts
             : (L->kb.first != 0 || L->kb.n_experts != L->E || L->n_present != L->E))
        return fail(WASTE_CUDA_E_ARG, part ? "layer %d: not every record of the bank's range "
                    "is loaded" : "layer %d: the whole-layer path needs every expert", layer);
    if ((rc = ensure_ws(T, L->top_k, L->E, L->kb.lat, L->kb.inter, L->si, L->kb.stages)))
        return rc;
    fill_args(a, L, T, L->top_k, L->E, L->si);
    a->router = L->d_router;
    a->bias = L->d_bias;
    a->renorm = L->renorm;
    a->routed_scale = L->routed_scale;
    a->shg = L->d_shg; a->shu = L->d_shu; a->shd = L->d_shd;
    a->shg_s = L->d_shg_s; a->shu_s = L->d_shu_s; a->shd_s = L->d_shd_s;
    a->act = L->act;
    a->situ_beta = L->situ_beta;
    a->situ_lbeta = L->situ_lbeta;
    a->prefetch_down = 1;
    if (S.prefetch_next && layer + 1 < WC_MAX_LAYERS && S.layer[layer + 1].trunk) {
        /* the next layer's router and shared expert, fetched into L2 while
         * this layer's gathers keep HBM idle */
        const wc_layer *N = &S.layer[layer + 1];
        const int g = 128;
        const size_t ng_h = (size_t)(N->hidden + g - 1) / g, ng_s = (size_t)(N->si + g - 1) / g;
        a->pf_ptr[0] = N->d_router;
        a->pf_bytes[0] = (size_t)N->E * N->hidden * sizeof(float);
        if (N->si > 0) {
            a->pf_ptr[1] = N->d_shg;
            a->pf_bytes[1] = (size_t)N->si * ng_h * g;
            a->pf_ptr[2] = N->d_shu;
            a->pf_bytes[2] = (size_t)N->si * ng_h * g;
            a->pf_ptr[3] = N->d_shd;
            a->pf_bytes[3] = (size_t)N->hidden * ng_s * g;
        }
    }
    if (wc_moe_supported(a))
        return fail(WASTE_CUDA_E_ARG, "layer %d: shape outside the kernels' bounds "
                    "(top-K <= 32, experts <= 1024, tiles within 227 KB of shared memory)",
                    layer);
    *Lp = L;
    return 0;
}

int waste_cuda_moe_layer_dev(int layer, const float *d_x, float *d_out, int *d_idx,
                             float *d_w, void *stream)
{
    int rc = 0;
    wc_moe_args a;
    wc_layer *L = NULL;
    if (!d_x || !d_out || !d_idx || !d_w) return fail(WASTE_CUDA_E_ARG, "NULL pointer");
    pthread_mutex_lock(&g_mu);
    if ((rc = layer_args(layer, 1, 0, &a, &L))) goto out;
    a.x = d_x;
    a.out = d_out;
    a.idx_out = d_idx;
    a.w_out = d_w;
    CK((cudaError_t)wc_moe_launch(&a, stream ? stream : (void *)S.stream), "layer kernels");
out:
    pthread_mutex_unlock(&g_mu);
    return rc;
}

/* The block's extra arguments: the rmsnorm in front and the residual add. */
static int block_args(wc_moe_args *a, const wc_layer *L, int layer, const float *d_h)
{
    if (!L->d_norm)
        return fail(WASTE_CUDA_E_NOBANK, "layer %d: no norm weight (waste_cuda_moe_norm_load)",
                    layer);
    a->norm_w = L->d_norm;
    a->norm_eps = L->norm_eps;
    a->resid = d_h;
    return 0;
}

int waste_cuda_moe_block_dev(int layer, int T, const float *d_h, float *d_h_out, int *d_idx,
                             float *d_w, void *stream)
{
    int rc = 0;
    wc_moe_args a;
    wc_layer *L = NULL;
    if (!d_h || !d_h_out || !d_idx || !d_w) return fail(WASTE_CUDA_E_ARG, "NULL pointer");
    pthread_mutex_lock(&g_mu);
    if ((rc = layer_args(layer, T, 0, &a, &L))) goto out;
    if ((rc = block_args(&a, L, layer, d_h))) goto out;
    a.x = d_h;
    a.out = d_h_out;
    a.idx_out = d_idx;
    a.w_out = d_w;
    CK((cudaError_t)wc_moe_launch(&a, stream ? stream : (void *)S.stream), "block kernels");
out:
    pthread_mutex_unlock(&g_mu);
    return rc;
}

int waste_cuda_moe_layer_part_dev(int layer, int T, const float *d_x, float *d_out,
                                  int sh_t0, int sh_t1, int *d_idx, float *d_w, void *stream)
{
    int rc = 0;
    wc_moe_args a;
    wc_layer *L = NULL;
    if (!d_x || !d_out || !d_idx || !d_w || sh_t0 < 0 || sh_t1 < sh_t0 || sh_t1 > T)
        return fail(WASTE_CUDA_E_ARG, "moe_layer_part: bad arguments");
    pthread_mutex_lock(&g_mu);
    if ((rc = layer_args(layer, T, 1, &a, &L))) goto out;
    a.x = d_x;
    a.out = d_out;
    a.idx_out = d_idx;
    a.w_out = d_w;
    a.sh_t0 = sh_t0;
    a.sh_t1 = sh_t1;
    CK((cudaError_t)wc_moe_launch(&a, stream ? stream : (void *)S.stream), "layer kernels");
out:
    pthread_mutex_unlock(&g_mu);
    return rc;
}

/* ---- batched (prefill) experts on the tensor cores -------------------------- */

static size_t al256z(size_t n) { return (n + 255) & ~(size_t)255; }

/* Carves the prefill workspace for T tokens x K experts (grown on demand). */
static int pf_args(const wc_layer *L, int T, int K, wc_pf_args *a)
{
    const size_t np = (size_t)T * K, lat = L->kb.lat, inter = L->kb.inter;
    const size_t nt = wc_pf_max_tiles(T, K, L->kb.n_experts);
    size_t sz[13], need = 0;
    sz[0] = np * 4;                         /* pairs            */
    sz[1] = sz[2] = sz[3] = nt * 4;         /* tile_e, _s, _n   */
    sz[4] = 4;                              /* ntiles           */
    sz[5] = sz[6] = (size_t)T * lat * 2;    /* xh, xl           */
    sz[7] = (size_t)T * 4;                  /* xinv             */
    sz[8] = np * 2 * inter * 4;             /* gu               */
    sz[9] = sz[10] = np * inter * 2;        /* hh, hl           */
    sz[11] = np * 4;                        /* hinv             */
    sz[12] = np * lat * 4;                  /* y                */
    for (int i = 0; i < 13; i++) need += al256z(sz[i]);
    if (need > S.pf_bytes) {
        cudaFree(S.d_pf);
        S.d_pf = NULL;
        S.pf_bytes = 0;
        const cudaError_t e = cudaMalloc(&S.d_pf, need);
        if (e != cudaSuccess) return cuda_fail(e, "prefill workspace");
        S.pf_bytes = need;
    }
    char *p = (char *)S.d_pf;
    void *ptr[13];
    for (int i = 0; i < 13; i++) { ptr[i] = p; p += al256z(sz[i]); }
    memset(a, 0, sizeof *a);
    a->bank = L->kb;
    a->books = S.d_books;
    a->T = T;
    a->K = K;
    a->pairs = (int *)ptr[0];
    a->tile_e = (int *)ptr[1]; a->tile_s = (int *)ptr[2]; a->tile_n = (int *)ptr[3];
    a->ntiles = (int *)ptr[4];
    a->xh = (uint16_t *)ptr[5]; a->xl = (uint16_t *)ptr[6]; a->xinv = (float *)ptr[7];
    a->gu = (float *)ptr[8];
    a->hh = (uint16_t *)ptr[9]; a->hl = (uint16_t *)ptr[10]; a->hinv = (float *)ptr[11];
    a->y = (float *)ptr[12];
    a->err = (unsigned int *)S.d_ws + 192;
    for (int k = 0; k < 3; k++) {
        float bound = 0.0f;
        for (int st = 0; st < 3; st++) bound += S.book_absmax[L->kb.cb_base + 3 * k + st];
        int ex = 0;
        frexpf(bound > 0.0f ? bound : 1.0f, &ex);
        ex = 14 - ex;                                  /* |w * scale| < 2^14 */
        ex = ex > 40 ? 40 : (ex < -40 ? -40 : ex);
        a->wscale[k] = ldexpf(1.0f, ex);
    }
    return 0;
}

/* Whether the tensor-core path takes this call: its shape bounds, fp16-exact
 * codebooks, and enough pairs per expert for dense tiles to beat lookups. */
static int pf_wanted(const wc_layer *L, int T, int K)
{
    return S.books_f16 && L->kb.stages == 3 && wc_pf_supported(&L->kb, T, K) == 0 &&
           (long)T * K >= 2L * L->kb.n_experts && getenv_flag("WASTE_CUDA_PREFILL_TC", 1);
}

int waste_cuda_moe_prefill_dev(int layer, int T, int K, const int *d_route, const float *d_rw,
                               const float *d_x, float *d_out, void *stream)
{
    int rc = 0;
    wc_layer *L = NULL;
    wc_pf_args a;
    if (T <= 0 || K <= 0 || !d_route || !d_rw || !d_x || !d_out)
        return fail(WASTE_CUDA_E_ARG, "moe_prefill: bad arguments");
    pthread_mutex_lock(&g_mu);
    if (layer < 0 || layer >= WC_MAX_LAYERS || !S.layer[layer].loaded) {
        rc = fail(WASTE_CUDA_E_NOBANK, "layer %d has no bank in HBM", layer);
        goto out;
    }
    L = &S.layer[layer];
    if (L->n_present != L->kb.n_experts) {
        rc = fail(WASTE_CUDA_E_ARG, "layer %d: not every record of the bank is loaded", layer);
        goto out;
    }
    if (!S.books_f16 || L->kb.stages != 3 || wc_pf_supported(&L->kb, T, K)) {
        rc = fail(WASTE_CUDA_E_ARG, "layer %d: outside the tensor-core path's bounds (3 stages, "
                  "rows multiples of 128, T*K <= %d, K <= 64, fp16-exact codebooks)", layer,
                  WC_PF_MAX_PAIRS);
        goto out;
    }
    if ((rc = ensure_ws(1, K, 1, L->kb.lat, L->kb.inter, 0, L->kb.stages))) goto out;
    if ((rc = pf_args(L, T, K, &a))) goto out;
    a.act = L->act;
    a.situ_beta = L->situ_beta;
    a.situ_lbeta = L->situ_lbeta;
    a.route = d_route;
    a.rw = d_rw;
    a.x = d_x;
    a.out = d_out;
    CK((cudaError_t)wc_pf_launch(&a, stream ? stream : (void *)S.stream), "prefill kernels");
out:
    pthread_mutex_unlock(&g_mu);
    return rc;
}

/* ---- expert parallelism over NCCL ------------------------------------------ */

static int nccl_fail(ncclResult_t r, const char *what)
{
    return fail(WASTE_CUDA_E_DEVICE, "%s: %s", what,
                EP.error_string ? EP.error_string(r) : "NCCL error");
}

static int nccl_load(void)
{
    if (EP.lib) return 0;
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return fail(WASTE_CUDA_E_NODEV, "expert parallelism needs libnccl.so.2: %s",
                        dlerror());
    *(void **)&EP.get_unique_id = dlsym(h, "ncclGetUniqueId");
    *(void **)&EP.comm_init_rank = dlsym(h, "ncclCommInitRank");
    *(void **)&EP.comm_destroy = dlsym(h, "ncclCommDestroy");
    *(void **)&EP.all_gather = dlsym(h, "ncclAllGather");
    *(void **)&EP.reduce_scatter = dlsym(h, "ncclReduceScatter");
    *(void **)&EP.error_string = dlsym(h, "ncclGetErrorString");
    *(void **)&EP.all_reduce = dlsym(h, "ncclAllReduce");
    if (!EP.get_unique_id || !EP.comm_init_rank || !EP.comm_destroy || !EP.all_gather ||
        !EP.reduce_scatter || !EP.error_string || !EP.all_reduce) {
        dlclose(h);
        return fail(WASTE_CUDA_E_NODEV, "libnccl.so.2 lacks an entry point this library uses");
    }
    EP.lib = h;
    return 0;
}

int waste_cuda_ep_unique_id(void *id, size_t bytes)
{
    if (!id || bytes < sizeof(ncclUniqueId))
        return fail(WASTE_CUDA_E_ARG, "ep_unique_id: need %zu bytes", sizeof(ncclUniqueId));
    pthread_mutex_lock(&g_mu);
    int rc = nccl_load();
    if (!rc) {
        ncclUniqueId u;
        const ncclResult_t r = EP.get_unique_id(&u);
        if (r != ncclSuccess) rc = nccl_fail(r, "ncclGetUniqueId");
        else memcpy(id, &u, sizeof u);
    }
    pthread_mutex_unlock(&g_mu);
    return rc;
}

int waste_cuda_ep_init(int rank, int world, const void *id, size_t bytes)
{
    int rc = 0;
    if (world <= 0 || rank < 0 || rank >= world || !id || bytes < sizeof(ncclUniqueId))
        return fail(WASTE_CUDA_E_ARG, "ep_init: bad arguments");
    pthread_mutex_lock(&g_mu);
    if (EP.active) { rc = fail(WASTE_CUDA_E_ARG, "expert parallelism already initialised"); goto out; }
    if (!S.inited) { rc = fail(WASTE_CUDA_E_NODEV, "ep_init before waste_cuda_init"); goto out; }
    if ((rc = nccl_load())) goto out;
    CK(cudaSetDevice(S.device), "cudaSetDevice");
    ncclUniqueId u;
    memcpy(&u, id, sizeof u);
    const ncclResult_t r = EP.comm_init_rank(&EP.comm, world, u, rank);
    if (r != ncclSuccess) { rc = nccl_fail(r, "ncclCommInitRank"); goto out; }
    EP.rank = rank;
    EP.world = world;
    {
        const char *wp = getenv("WASTE_CUDA_EP_WAIT_POLLS");
        const long v = (wp && *wp) ? strtol(wp, NULL, 10) : 0;
        EP.wait_polls = (v > 0 && v <= (1L << 30)) ? (int)v : (1 << 24);
    }
    EP.active = 1;
    g_epoch++;
out:
    pthread_mutex_unlock(&g_mu);
    return rc;
}

/* Every rank's agreement on an int (min over ranks), through NCCL. */
static int ep_agree_min(int v, int *out)
{
    int rc = 0;
    int *d = NULL;
    CK(cudaMalloc((void **)&d, sizeof(int)), "agreement word");
    CK(h2d_now(d, &v, sizeof(int)), "agreement H2D");
    const ncclResult_t r = EP.all_reduce(d, d, 1, ncclInt32, ncclMin, EP.comm, S.stream);
    if (r != ncclSuccess) { rc = nccl_fail(r, "ncclAllReduce"); goto out; }
    CK(cudaStreamSynchronize(S.stream), "agreement");
    CK(cudaMemcpy(out, d, sizeof(int), cudaMemcpyDeviceToHost), "agreement D2H");
out:
    cudaFree(d);
    return rc;
}

/* Unmaps the peers' mailboxes and, once every rank has, frees this one. */
static void ep_mail_free(void)
{
    if (!EP.mail[EP.rank]) return;
    for (int r = 0; r < EP.world; r++)
        if (r != EP.rank && EP.mail[r]) cudaIpcCloseMemHandle(EP.mail[r]);
    int dummy = 0;
    ep_agree_min(0, &dummy);                 /* nobody maps this one any more */
    cudaFree(EP.mail[EP.rank]);
    memset(EP.mail, 0, sizeof EP.mail);
    EP.p2p = 0;
    EP.mail_T = EP.mail_hidden = 0;
}

/* Collective: mailboxes for T tokens per rank of `hidden` floats, mapped on
 * every rank, or EP.p2p = 0 on every rank when any mapping fails. */
static int ep_mail_setup(int T, int hidden)
{
    int rc = 0;
    if (EP.mail[EP.rank] && T <= EP.mail_T && hidden <= EP.mail_hidden) return 0;
    if (EP.mail[EP.rank]) ep_mail_free();
    g_epoch++;
    const int Tm = T > WC_CHUNK_MAX / EP.world ? T : WC_CHUNK_MAX / EP.world;
    const size_t bytes = WC_EP_MAIL_HDR + 2 * (size_t)EP.world * Tm * hidden * sizeof(float);
    unsigned char *mine = NULL, *dh = NULL;
    cudaIpcMemHandle_t hs[WC_EP_MAX];
    int ok = 1;
    CK(cudaMalloc((void **)&mine, bytes), "mailbox");
    CK(memset_now(mine, 0, bytes), "mailbox clear");
    CK(cudaDeviceSynchronize(), "mailbox clear");
    if (cudaIpcGetMemHandle(&hs[EP.rank], mine) != cudaSuccess) ok = 0;
    CK(cudaMalloc((void **)&dh, sizeof hs), "handle exchange");
    CK(h2d_now(dh + EP.rank * sizeof(cudaIpcMemHandle_t), &hs[EP.rank],
               sizeof(cudaIpcMemHandle_t)), "handle H2D");
    {
        const ncclResult_t r = EP.all_gather(dh + EP.rank * sizeof(cudaIpcMemHandle_t), dh,
                                             sizeof(cudaIpcMemHandle_t), ncclUint8, EP.comm,
                                             S.stream);
        if (r != ncclSuccess) { rc = nccl_fail(r, "ncclAllGather"); goto out; }
    }
    CK(cudaStreamSynchronize(S.stream), "handle exchange");
    CK(cudaMemcpy(hs, dh, (size_t)EP.world * sizeof(cudaIpcMemHandle_t),
                  cudaMemcpyDeviceToHost), "handles D2H");
    EP.mail[EP.rank] = mine;
    for (int r = 0; r < EP.world && ok; r++) {
        if (r == EP.rank) continue;
        void *p = NULL;
        if (cudaIpcOpenMemHandle(&p, hs[r], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            cudaGetLastError();
            ok = 0;
        } else {
            EP.mail[r] = (unsigned char *)p;
        }
    }
    int all = 0;
    if ((rc = ep_agree_min(ok, &all))) goto out;
    EP.mail_T = Tm;
    EP.mail_hidden = hidden;
    EP.p2p = all;
    if (!all) ep_mail_free();                /* every rank falls back to NCCL */
out:
    cudaFree(dh);
    return rc;
}

static void ep_shutdown_locked(void)
{
    if (!EP.active) return;
    if (S.inited) cudaStreamSynchronize(S.stream);
    ep_mail_free();
    EP.comm_destroy(EP.comm);
    cudaFree(EP.d_xall);
    cudaFree(EP.d_outall);
    EP.comm = NULL;
    EP.d_xall = EP.d_outall = NULL;
    EP.all_floats = 0;
    EP.active = EP.rank = EP.world = 0;
    EP.poisoned = 0;
    g_epoch++;
}

void waste_cuda_ep_shutdown(void)
{
    pthread_mutex_lock(&g_mu);
    ep_shutdown_locked();
    pthread_mutex_unlock(&g_mu);
}

/* Both expert-parallel layer calls. rep = 0: each rank brings its own T
 * tokens and receives their outputs. rep = 1: every rank brings the same T
 * tokens and receives all of their outputs. */
static int ep_layer(int layer, int T, const float *d_x, float *d_out, int *d_idx, float *d_w,
                    void *stream, int rep, int block)
{
    int rc = 0;
    wc_moe_args a;
    wc_layer *L = NULL;
    if (!d_x || !d_out || T <= 0) return fail(WASTE_CUDA_E_ARG, "ep_moe_layer: bad arguments");
    pthread_mutex_lock(&g_mu);
    if (!EP.active) { rc = fail(WASTE_CUDA_E_ARG, "ep_moe_layer before ep_init"); goto out; }
    if (EP.poisoned) {
        rc = fail(WASTE_CUDA_E_DEVICE, "ep_moe_layer: an earlier call gave up waiting on a "
                  "peer; the ranks' exchange is out of step until waste_cuda_ep_shutdown and "
                  "waste_cuda_ep_init");
        goto out;
    }
    const int Ta = rep ? T : T * EP.world;
    const int tr = rep ? 0 : EP.rank;            /* this rank's tokens in the routes */
    if ((rc = layer_args(layer, Ta, 1, &a, &L))) goto out;
    /* the block: every rank normalises the tokens it routes; the residual
     * is added once, where the token's output is finished (the finalize of
     * the peer exchange, or after the NCCL reduction) */
    if (block && (rc = block_args(&a, L, layer, NULL))) goto out;
    {
        int r0, rn;
        split_range(L->E, EP.rank, EP.world, &r0, &rn);
        if (L->kb.first != r0 || L->kb.n_experts != rn) {
            rc = fail(WASTE_CUDA_E_ARG, "layer %d: bank holds [%d, %d), rank %d of %d owns "
                      "[%d, %d)", layer, L->kb.first, L->kb.first + L->kb.n_experts, EP.rank,
                      EP.world, r0, r0 + rn);
            goto out;
        }
    }
    const size_t need = (size_t)Ta * L->hidden;
    if (need > EP.all_floats) {
        cudaFree(EP.d_xall);
        cudaFree(EP.d_outall);
        EP.d_xall = EP.d_outall = NULL;
        EP.all_floats = 0;
        CK(cudaMalloc((void **)&EP.d_xall, need * sizeof(float)), "ep tokens");
        CK(cudaMalloc((void **)&EP.d_outall, need * sizeof(float)), "ep partials");
        EP.all_floats = need;
    }
    cudaStream_t st = stream ? (cudaStream_t)stream : S.stream;
    const size_t per = (size_t)T * L->hidden;
    const size_t kb = (size_t)T * L->top_k;
    if (getenv_flag("WASTE_CUDA_EP_P2P", 1) && (rc = ep_mail_setup(T, L->hidden))) goto out;
    if (EP.p2p && T <= EP.mail_T && L->hidden <= EP.mail_hidden) {
        /* tokens out to every mailbox, the layer on all of them, partial
         * sums straight into the tokens' ranks, sum in rank order */
        wc_ep_link lk;
        memset(&lk, 0, sizeof lk);
        lk.on = 1;
        lk.rank = EP.rank;
        lk.world = EP.world;
        lk.T = T;
        lk.hidden = L->hidden;
        lk.rep = rep;
        lk.wait_polls = EP.wait_polls;
        memcpy(lk.mail, EP.mail, sizeof lk.mail);
        CK((cudaError_t)wc_ep_publish_launch(&lk, d_x, a.ws.err, st), "ep publish");
        a.x = rep ? d_x : (const float *)(EP.mail[EP.rank] + WC_EP_MAIL_HDR);
        a.out = EP.d_outall;
        a.idx_out = S.d_idx;
        a.w_out = S.d_w;
        a.ep = lk;
        if (a.gu_eg == 0)     /* route-first (x arrives with the route), tiles
                                 for the expected local count */
            a.gu_eg = (int)(((long)L->top_k * L->kb.n_experts + L->n_total - 1) / L->n_total);
    } else if (!rep) {
        const ncclResult_t r = EP.all_gather(d_x, EP.d_xall, per, ncclFloat32, EP.comm, st);
        if (r != ncclSuccess) { rc = nccl_fail(r, "ncclAllGather"); goto out; }
        a.x = EP.d_xall;
        a.out = EP.d_outall;
        a.idx_out = S.d_idx;
        a.w_out = S.d_w;
    } else {
        a.x = d_x;
        a.out = EP.d_outall;
        a.idx_out = S.d_idx;
        a.w_out = S.d_w;
    }
    /* the shared expert once per token: on the token's rank, or (rep) on
     * one rank of a split of the tokens */
    a.sh_t0 = rep ? EP.rank * T / EP.world : EP.rank * T;
    a.sh_t1 = rep ? (EP.rank + 1) * T / EP.world : EP.rank * T + T;
    CK((cudaError_t)wc_moe_launch(&a, st), "layer kernels");
    if (a.ep.on) {
        CK((cudaError_t)wc_ep_finalize_launch(&a.ep, d_out, block ? d_x : NULL, a.ws.err, st),
           "ep finalize");
    } else if (!rep) {
        const ncclResult_t r = EP.reduce_scatter(EP.d_outall, d_out, per, ncclFloat32, ncclSum,
                                                 EP.comm, st);
        if (r != ncclSuccess) { rc = nccl_fail(r, "ncclReduceScatter"); goto out; }
    } else {
        const ncclResult_t r = EP.all_reduce(EP.d_outall, d_out, per, ncclFloat32, ncclSum,
                                             EP.comm, st);
        if (r != ncclSuccess) { rc = nccl_fail(r, "ncclAllReduce"); goto out; }
    }
    if (block && !a.ep.on)
        CK((cudaError_t)wc_resid_add_launch(d_out, d_x, d_out, per, st), "residual add");
    if (d_idx) CK(cudaMemcpyAsync(d_idx, S.d_idx + (size_t)tr * kb, kb * sizeof(int),
                                  cudaMemcpyDeviceToDevice, st), "route copy");
    if (d_w) CK(cudaMemcpyAsync(d_w, S.d_w + (size_t)tr * kb, kb * sizeof(float),
                                cudaMemcpyDeviceToDevice, st), "weight copy");
out:
    pthread_mutex_unlock(&g_mu);
    return rc;
}

int waste_cuda_ep_moe_layer_dev(int layer, int T, const float *d_x, float *d_out, int *d_idx,
                                float *d_w, void *stream)
{
    return ep_layer(layer, T, d_x, d_out, d_idx, d_w, stream, 0, 0);
}

int waste_cuda_ep_moe_layer_rep_dev(int layer, int T, const float *d_x, float *d_out,
                                    int *d_idx, float *d_w, void *stream)
{
    return ep_layer(layer, T, d_x, d_out, d_idx, d_w, stream, 1, 0);
}

int waste_cuda_ep_moe_block_dev(int layer, int T, const float *d_h, float *d_h_out, int *d_idx,
                                float *d_w, void *stream)
{
    return ep_layer(layer, T, d_h, d_h_out, d_idx, d_w, stream, 0, 1);
}

int waste_cuda_ep_moe_block_rep_dev(int layer, int T, const float *d_h, float *d_h_out,
                                    int *d_idx, float *d_w, void *stream)
{
    return ep_layer(layer, T, d_h, d_h_out, d_idx, d_w, stream, 1, 1);
}

/* The host-buffer layer call captured once: H2D of x, the kernel chain,
 * D2H of the output, route, weights and error word. Rebuilt when the
 * epoch moved since it was made. */
static size_t res_floats(int lat) { return (size_t)lat + 2 * WC_MAX_TOPK + 4; }

static int ensure_res(int lat)
{
    if (lat <= S.res_lat) return 0;
    g_epoch++;
    cudaFree(S.d_res);
    cudaFreeHost(S.h_res);
    S.d_res = S.h_res = NULL;
    S.res_lat = 0;
    if (cudaMalloc((void **)&S.d_res, res_floats(lat) * sizeof(float)) != cudaSuccess ||
        cudaMallocHost((void **)&S.h_res, res_floats(lat) * sizeof(float)) != cudaSuccess ||
        memset_now(S.d_res, 0, res_floats(lat) * sizeof(float)) != cudaSuccess)
        return fail(WASTE_CUDA_E_NOMEM, "layer result block");
    S.res_lat = lat;
    return 0;
}

static int layer_graph(cudaGraphExec_t *gx, unsigned *gx_epoch, const wc_moe_args *a,
                       size_t xb)
{
    int rc = 0;
    if (*gx && *gx_epoch == g_epoch) return 0;
    if (*gx) { cudaGraphExecDestroy(*gx); *gx = NULL; }
    cudaGraph_t g = NULL;
    CK(cudaStreamBeginCapture(S.stream, cudaStreamCaptureModeThreadLocal), "graph capture");
    const wc_copy_args cin = { { S.d_x }, { S.h_x }, { xb }, 1, 0 };
    const wc_copy_args cout = { { S.h_res }, { S.d_res },
                                { res_floats(S.res_lat) * sizeof(float) }, 1, 1 };
    cudaError_t e = small_copies(&cin, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = (cudaError_t)wc_moe_launch(a, S.stream);
    if (e == cudaSuccess) e = small_copies(&cout, cudaMemcpyDeviceToHost);
    const cudaError_t ee = cudaStreamEndCapture(S.stream, &g);   /* always end it */
    if (e == cudaSuccess) e = ee;
    if (e == cudaSuccess) e = cudaGraphInstantiate(gx, g, 0);
    if (g) cudaGraphDestroy(g);
    if (e != cudaSuccess) {
        *gx = NULL;
        cudaGetLastError();
        rc = cuda_fail(e, "layer graph");
        goto out;
    }
    *gx_epoch = g_epoch;
out:
    return rc;
}

/* The host-buffer layer call (block = 0) and block call (block = 1). */
static int host_layer(int layer, const float *x, float *out, int *routed, float *weights,
                      int block)
{
    int rc = 0;
    wc_moe_args a;
    wc_layer *L = NULL;
    if (!x || !out) return fail(WASTE_CUDA_E_ARG, "NULL pointer");
    pthread_mutex_lock(&g_mu);
    if ((rc = layer_args(layer, 1, 0, &a, &L))) goto out;
    if (block && (rc = block_args(&a, L, layer, S.d_x))) goto out;
    const size_t xb = (size_t)L->hidden * sizeof(float);
    a.x = S.d_x;
    a.out = S.d_out;
    a.idx_out = S.d_idx;
    a.w_out = S.d_w;
    memcpy(S.h_x, x, xb);
    if (!wc_profiling()) {
        /* one graph launch per call: x in, the kernel chain, and one copy of
         * the result block (output, route, weights, error word) out */
        if ((rc = ensure_res(L->hidden))) goto out;
        const int lat = S.res_lat;
        a.out = S.d_res;
        a.idx_out = (int *)(S.d_res + lat);
        a.w_out = S.d_res + lat + WC_MAX_TOPK;
        a.ws.err = (unsigned int *)(S.d_res + lat + 2 * WC_MAX_TOPK);
        if ((rc = block ? layer_graph(&L->gxb, &L->gxb_epoch, &a, xb)
                        : layer_graph(&L->gx, &L->gx_epoch, &a, xb))) goto out;
        CK(cudaGraphLaunch(block ? L->gxb : L->gx, S.stream), "layer graph");
        CK(cudaStreamSynchronize(S.stream), "moe layer");
        const unsigned int err = *(const unsigned int *)(S.h_res + lat + 2 * WC_MAX_TOPK);
        if (err) {
            memset_now(S.d_res + lat + 2 * WC_MAX_TOPK, 0, sizeof(unsigned int));
            memset_now(S.d_ws, 0, WC_WS_CONTROL_WORDS * sizeof(unsigned int));
            rc = fail(WASTE_CUDA_E_DEVICE, "layer %d: a bounded device wait gave up", layer);
            goto out;
        }
        memcpy(out, S.h_res, xb);
        if (routed) memcpy(routed, S.h_res + lat, (size_t)L->top_k * sizeof(int));
        if (weights) memcpy(weights, S.h_res + lat + WC_MAX_TOPK, (size_t)L->top_k * sizeof(float));
        goto out;
    } else {                        /* phase timers: events between the kernels */
        CK(cudaMemcpyAsync(S.d_x, S.h_x, xb, cudaMemcpyHostToDevice, S.stream), "x H2D");
        CK((cudaError_t)wc_moe_launch(&a, S.stream), "layer kernels");
        CK(cudaMemcpyAsync(S.h_out, S.d_out, xb, cudaMemcpyDeviceToHost, S.stream), "out D2H");
        CK(cudaMemcpyAsync(S.h_idx, S.d_idx, (size_t)L->top_k * sizeof(int),
                           cudaMemcpyDeviceToHost, S.stream), "idx D2H");
        CK(cudaMemcpyAsync(S.h_w, S.d_w, (size_t)L->top_k * sizeof(float),
                           cudaMemcpyDeviceToHost, S.stream), "w D2H");
        CK(cudaStreamSynchronize(S.stream), "moe layer");
        if (read_device_errors(1)) {
            rc = fail(WASTE_CUDA_E_DEVICE, "layer %d: a bounded device wait gave up", layer);
            goto out;
        }
    }
    memcpy(out, S.h_out, xb);
    if (routed) memcpy(routed, S.h_idx, (size_t)L->top_k * sizeof(int));
    if (weights) memcpy(weights, S.h_w, (size_t)L->top_k * sizeof(float));
out:
    pthread_mutex_unlock(&g_mu);
    return rc;
}

int waste_cuda_moe_layer(int layer, const float *x, float *out, int *routed, float *weights)
{
    return host_layer(layer, x, out, routed, weights, 0);
}

int waste_cuda_moe_block(int layer, const float *h, float *h_out, int *routed, float *weights)
{
    return host_layer(layer, h, h_out, routed, weights, 1);
}

/* ---- single kernels (host buffers) -------------------------------------- */

static int tmp_reserve(size_t bytes)
{
    if (bytes <= S.tmp_bytes) return 0;
    cudaFree(S.d_tmp);
    S.d_tmp = NULL;
    S.tmp_bytes = 0;
    cudaError_t e = cudaMalloc(&S.d_tmp, bytes);
    if (e != cudaSuccess) return cuda_fail(e, "scratch");
    S.tmp_bytes = bytes;
    return 0;
}

static size_t al256(size_t n) { return (n + 255) & ~(size_t)255; }

/* ---- VQ4P ------------------------------------------------------------------ */

/* Scratch for a VQ4P launch: integer block sums and table scales for the
 * larger of two phases (G problems of [M][N] each), then `h_floats` floats
 * of activations. */
static int p6_reserve(int G0, int M0, int N0, int G1, int M1, int N1, size_t h_floats,
                      int **part, float **ls, float **h)
{
    size_t pi = wc_p6_part_ints(G0, M0, N0), lf = wc_p6_ls_floats(G0, N0);
    if (G1 > 0) {
        const size_t pi1 = wc_p6_part_ints(G1, M1, N1), lf1 = wc_p6_ls_floats(G1, N1);
        if (pi1 > pi) pi = pi1;
        if (lf1 > lf) lf = lf1;
    }
    const size_t need = al256(pi * sizeof(int)) + al256(lf * sizeof(float)) +
                        al256(h_floats * sizeof(float));
    if (need > S.p6_bytes) {
        g_epoch++;
        cudaFree(S.d_p6);
        S.d_p6 = NULL;
        S.p6_bytes = 0;
        const cudaError_t e = cudaMalloc(&S.d_p6, need);
        if (e != cudaSuccess) return cuda_fail(e, "VQ4P scratch");
        S.p6_bytes = need;
    }
    char *b = (char *)S.d_p6;
    *part = (int *)b;
    *ls = (float *)(b + al256(pi * sizeof(int)));
    if (h) *h = (float *)(b + al256(pi * sizeof(int)) + al256(lf * sizeof(float)));
    return 0;
}

/* The expert loop over a VQ4P bank for the T tokens staged in S.d_x /
 * S.d_idx / S.d_w; ysum into S.d_out. The caller holds g_mu. */
static int p6_experts(const wc_layer *L, int T, int K, int act, float situ_beta,
                      float situ_lbeta, int order_by_id)
{
    int rc = 0;
    const int pairs = T * K, lat = L->kb.lat, inter = L->kb.inter;
    wc_p6_args *a = (wc_p6_args *)calloc(1, sizeof *a);
    if (!a) return fail(WASTE_CUDA_E_NOMEM, "VQ4P arguments");
    if ((rc = p6_reserve(2 * pairs, inter, lat, pairs, lat, inter, (size_t)pairs * inter,
                         &a->part, &a->ls, &a->h)))
        goto out;
    a->books = S.d_books;
    a->bank = L->kb;
    a->T = T;
    a->K = K;
    a->order_by_id = order_by_id;
    a->act = act;
    a->situ_beta = situ_beta;
    a->situ_lbeta = situ_lbeta;
    a->route = S.d_idx;
    a->rw = S.d_w;
    a->x_in = S.d_x;
    a->ysum = S.d_out;
    a->err = (unsigned int *)S.d_ws + 192;
    CK((cudaError_t)wc_p6_moe_launch(a, S.stream), "VQ4P expert kernels");
out:
    free(a);
    return rc;
}

static int check_p6(int M, int N, int cb_base)
{
    if (M <= 0 || N <= 0 || N % 8 || cb_base < 0)
        return fail(WASTE_CUDA_E_ARG, "VQ4P matrix: bad shape");
    if (!S.d_books || S.cb_entries != 64 || cb_base + 4 > S.n_books)
        return fail(WASTE_CUDA_E_ARG, "VQ4P: 64-entry codebooks not loaded or cb_base out of "
                    "range");
    return 0;
}

int waste_cuda_vq4p_matvec_dev(int G, const uint8_t *const *idx, const uint16_t *const *scale,
                               const float *const *x, float *const *y, int M, int N,
                               int cb_base, void *stream)
{
    int rc = 0;
    wc_p6_args *a = NULL;
    if (G <= 0 || G > WC_MAX_G || !idx || !scale || !x || !y)
        return fail(WASTE_CUDA_E_ARG, "vq4p_matvec_dev: bad arguments");
    for (int g = 0; g < G; g++)
        if (!idx[g] || !scale[g] || !x[g] || !y[g] || ((uintptr_t)idx[g] & 7))
            return fail(WASTE_CUDA_E_ARG, "vq4p_matvec_dev: matrix %d: NULL or idx not "
                        "8-byte aligned", g);
    pthread_mutex_lock(&g_mu);
    if (!S.inited && (rc = init_locked(-1))) goto out;
    if ((rc = check_p6(M, N, cb_base))) goto out;
    a = (wc_p6_args *)calloc(1, sizeof *a);
    if (!a) { rc = fail(WASTE_CUDA_E_NOMEM, "VQ4P arguments"); goto out; }
    if ((rc = p6_reserve(G, M, N, 0, 0, 0, 0, &a->part, &a->ls, NULL))) goto out;
    a->G = G;
    a->M = M;
    a->N = N;
    a->books = S.d_books;
    for (int g = 0; g < G; g++) {
        a->idx[g] = idx[g];
        a->scale[g] = scale[g];
        a->x[g] = x[g];
        a->y[g] = y[g];
        a->cb[g] = cb_base;
    }
    CK((cudaError_t)wc_p6_matvec_launch(a, stream ? stream : (void *)S.stream), "VQ4P matvec");
out:
    free(a);
    pthread_mutex_unlock(&g_mu);
    return rc;
}

int waste_cuda_vq4p_matvec(float *y, const uint8_t *idx, const uint16_t *scale, const float *x,
                           int M, int N, int cb_base)
{
    int rc = 0;
    wc_p6_args *a = NULL;
    if (!y || !idx || !scale || !x) return fail(WASTE_CUDA_E_ARG, "NULL pointer");
    pthread_mutex_lock(&g_mu);
    if (!S.inited && (rc = init_locked(-1))) goto out;
    if ((rc = check_p6(M, N, cb_base))) goto out;
    const size_t ib = (size_t)((M + 63) / 64) * 64 * (N / 8) * 3;
    const size_t o_sc = al256(ib), o_x = o_sc + al256((size_t)M * 2),
                 o_y = o_x + al256((size_t)N * 4), tot = o_y + (size_t)M * 4;
    if ((rc = tmp_reserve(tot))) goto out;
    char *t = (char *)S.d_tmp;
    CK(cudaMemcpyAsync(t, idx, ib, cudaMemcpyHostToDevice, S.stream), "idx H2D");
    CK(cudaMemcpyAsync(t + o_sc, scale, (size_t)M * 2, cudaMemcpyHostToDevice, S.stream),
       "scale H2D");
    CK(cudaMemcpyAsync(t + o_x, x, (size_t)N * 4, cudaMemcpyHostToDevice, S.stream), "x H2D");
    a = (wc_p6_args *)calloc(1, sizeof *a);
    if (!a) { rc = fail(WASTE_CUDA_E_NOMEM, "VQ4P arguments"); goto out; }
    if ((rc = p6_reserve(1, M, N, 0, 0, 0, 0, &a->part, &a->ls, NULL))) goto out;
    a->G = 1;
    a->M = M;
    a->N = N;
    a->books = S.d_books;
    a->idx[0] = (const uint8_t *)t;
    a->scale[0] = (const uint16_t *)(t + o_sc);
    a->x[0] = (const float *)(t + o_x);
    a->y[0] = (float *)(t + o_y);
    a->cb[0] = cb_base;
    CK((cudaError_t)wc_p6_matvec_launch(a, S.stream), "VQ4P matvec");
    CK(cudaMemcpyAsync(y, t + o_y, (size_t)M * 4, cudaMemcpyDeviceToHost, S.stream), "y D2H");
    CK(cudaStreamSynchronize(S.stream), "VQ4P matvec");
out:
    free(a);
    pthread_mutex_unlock(&g_mu);
    return rc;
}

int waste_cuda_vq4p_table(int8_t *q, float *qs, const float *x, int N, int cb_base)
{
    int rc = 0;
    if (!q || !qs || !x) return fail(WASTE_CUDA_E_ARG, "NULL pointer");
    pthread_mutex_lock(&g_mu);
    if (!S.inited && (rc = init_locked(-1))) goto out;
    if ((rc = check_p6(1, N, cb_base))) goto out;
    const int nv = N / 8, nb = (nv + 31) / 32;
    const size_t qb = (size_t)nv * 256, o_qs = al256(qb), o_x = o_qs + al256((size_t)nb * 4);
    if ((rc = tmp_reserve(o_x + (size_t)N * 4))) goto out;
    char *t = (char *)S.d_tmp;
    CK(cudaMemcpyAsync(t + o_x, x, (size_t)N * 4, cudaMemcpyHostToDevice, S.stream), "x H2D");
    CK((cudaError_t)wc_p6_table_launch((int8_t *)t, (float *)(t + o_qs), (const float *)(t + o_x),
                                       S.d_books, cb_base, nv, S.stream), "VQ4P table");
    CK(cudaMemcpyAsync(q, t, qb, cudaMemcpyDeviceToHost, S.stream), "table D2H");
    CK(cudaMemcpyAsync(qs, t + o_qs, (size_t)nb * 4, cudaMemcpyDeviceToHost, S.stream),
       "scales D2H");
    CK(cudaStreamSynchronize(S.stream), "VQ4P table");
out:
    pthread_mutex_unlock(&g_mu);
    return rc;
}

/* ---- the converter's RVQ encoder --------------------------------------------- */

#define WC_ENC_SMEM_MAX 232448      /* 227 KB of shared memory a block */

static int enc_args(int n, int stages, int entries, int dim)
{
    if (n <= 0 || stages <= 0 || entries <= 0 || entries > 256 || dim <= 0 || dim > 64)
        return fail(WASTE_CUDA_E_ARG, "vq_encode: n > 0, stages > 0, entries 1..256, dim 1..64");
    if (wc_vq_encode_smem(stages, entries, dim) > WC_ENC_SMEM_MAX)
        return fail(WASTE_CUDA_E_ARG, "vq_encode: %d stages x %d entries x %d dims of codebook "
                    "exceed 227 KB of shared memory", stages, entries, dim);
    return 0;
}

static int enc_reserve(size_t bytes)
{
    if (bytes <= S.enc_bytes) return 0;
    cudaFree(S.d_enc);
    S.d_enc = NULL;
    S.enc_bytes = 0;
    const cudaError_t e = cudaMalloc(&S.d_enc, bytes);
    if (e != cudaSuccess) return cuda_fail(e, "encoder buffers");
    S.enc_bytes = bytes;
    return 0;
}

int waste_cuda_vq_encode_dev(const float *d_X, int n, const float *d_books, int stages,
                             int entries, int dim, uint8_t *d_out, void *stream)
{
    int rc;
    if (!d_X || !d_books || !d_out) return fail(WASTE_CUDA_E_ARG, "NULL pointer");
    if ((rc = enc_args(n, stages, entries, dim))) return rc;
    pthread_mutex_lock(&g_mu);
    if (!S.inited) { rc = fail(WASTE_CUDA_E_NODEV, "vq_encode_dev before waste_cuda_init"); goto out; }
    CK((cudaError_t)wc_vq_encode_launch(d_X, n, d_books, stages, entries, dim, d_out,
                                        stream ? stream : (void *)S.stream), "vq encode");
out:
    pthread_mutex_unlock(&g_mu);
    return rc;
}

int waste_cuda_vq_encode(const float *X, int n, const float *books, int stages, int entries,
                         int dim, uint8_t *out)
{
    int rc;
    if (!X || !books || !out) return fail(WASTE_CUDA_E_ARG, "NULL pointer");
    if ((rc = enc_args(n, stages, entries, dim))) return rc;
    pthread_mutex_lock(&g_mu);
    if (!S.inited && (rc = init_locked(-1))) goto out;
    {
        const size_t xb = (size_t)n * dim * sizeof(float);
        const size_t bb = (size_t)stages * entries * dim * sizeof(float);
        const size_t ob = (size_t)n * stages;
        const size_t o_b = al256(xb), o_o = o_b + al256(bb);
        if ((rc = enc_reserve(o_o + ob))) goto out;
        char *d = (char *)S.d_enc;
        CK(cudaMemcpyAsync(d, X, xb, cudaMemcpyHostToDevice, S.stream), "X H2D");
        CK(cudaMemcpyAsync(d + o_b, books, bb, cudaMemcpyHostToDevice, S.stream), "books H2D");
        CK((cudaError_t)wc_vq_encode_launch((const float *)d, n, (const float *)(d + o_b), stages,
                                            entries, dim, (uint8_t *)(d + o_o), S.stream),
           "vq encode");
        CK(cudaMemcpyAsync(out, d + o_o, ob, cudaMemcpyDeviceToHost, S.stream), "codes D2H");
        CK(cudaStreamSynchronize(S.stream), "vq encode");
    }
out:
    pthread_mutex_unlock(&g_mu);
    return rc;
}

int waste_cuda_vq_lloyd_dev(const float *d_X, int n, float *d_C, int entries, int dim,
                            int *d_live, void *stream)
{
    int rc;
    if (!d_X || !d_C || !d_live) return fail(WASTE_CUDA_E_ARG, "NULL pointer");
    if ((rc = enc_args(n, 1, entries, dim))) return rc;
    pthread_mutex_lock(&g_mu);
    if (!S.inited) { rc = fail(WASTE_CUDA_E_NODEV, "vq_lloyd_dev before waste_cuda_init"); goto out; }
    if ((rc = enc_reserve(wc_vq_lloyd_scratch(n, entries, dim)))) goto out;
    CK((cudaError_t)wc_vq_lloyd_launch(d_X, n, d_C, entries, dim, S.d_enc, d_live,
                                       stream ? stream : (void *)S.stream), "lloyd");
out:
    pthread_mutex_unlock(&g_mu);
    return rc;
}

int waste_cuda_vq_lloyd(const float *X, int n, float *C, int entries, int dim)
{
    int rc;
    if (!X || !C) return fail(WASTE_CUDA_E_ARG, "NULL pointer");
    if ((rc = enc_args(n, 1, entries, dim))) return rc;
    pthread_mutex_lock(&g_mu);
    if (!S.inited && (rc = init_locked(-1))) goto out;
    {
        const size_t xb = (size_t)n * dim * sizeof(float);
        const size_t cb = (size_t)entries * dim * sizeof(float);
        const size_t o_c = al256(xb), o_l = o_c + al256(cb), o_s = o_l + 256;
        if ((rc = enc_reserve(o_s + wc_vq_lloyd_scratch(n, entries, dim)))) goto out;
        char *d = (char *)S.d_enc;
        int live = 0;
        CK(cudaMemcpyAsync(d, X, xb, cudaMemcpyHostToDevice, S.stream), "X H2D");
        CK(cudaMemcpyAsync(d + o_c, C, cb, cudaMemcpyHostToDevice, S.stream), "C H2D");
        CK((cudaError_t)wc_vq_lloyd_launch((const float *)d, n, (float *)(d + o_c), entries, dim,
                                           d + o_s, (int *)(d + o_l), S.stream), "lloyd");
        CK(cudaMemcpyAsync(C, d + o_c, cb, cudaMemcpyDeviceToHost, S.stream), "C D2H");
        CK(cudaMemcpyAsync(&live, d + o_l, sizeof live, cudaMemcpyDeviceToHost, S.stream),
           "live D2H");
        CK(cudaStreamSynchronize(S.stream), "lloyd");
        rc = live;
    }
out:
    pthread_mutex_unlock(&g_mu);
    return rc;
}

int waste_cuda_lutb(float *lut, const float *x, int cb_base, int nv, int stages)
{
    int rc = 0;
    if (!lut || !x || nv <= 0 || (stages != 2 && stages != 3) || cb_base < 0)
        return fail(WASTE_CUDA_E_ARG, "lutb: bad arguments");
    pthread_mutex_lock(&g_mu);
    if (!S.d_books || cb_base + stages > S.n_books) {
        rc = fail(WASTE_CUDA_E_ARG, "lutb: codebooks not loaded or cb_base out of range");
        goto out;
    }
    const size_t xb = (size_t)nv * 8 * sizeof(float), lb = (size_t)nv * stages * 256 * sizeof(float);
    if ((rc = tmp_reserve(al256(xb) + lb))) goto out;
    float *dx = (float *)S.d_tmp, *dl = (float *)((char *)S.d_tmp + al256(xb));
    CK(cudaMemcpyAsync(dx, x, xb, cudaMemcpyHostToDevice, S.stream), "x H2D");
    CK((cudaError_t)wc_lutb_launch(dl, dx, S.d_books, cb_base, nv, stages, S.stream), "lutb");
    CK(cudaMemcpyAsync(lut, dl, lb, cudaMemcpyDeviceToHost, S.stream), "lut D2H");
    CK(cudaStreamSynchronize(S.stream), "lutb");
out:
    pthread_mutex_unlock(&g_mu);
    return rc;
}

static int check_mat(int M, int N, int cb_base, int stages)
{
    if (M <= 0 || N <= 0 || N % 8 || (stages != 2 && stages != 3) || cb_base < 0)
        return fail(WASTE_CUDA_E_ARG, "matrix: bad shape");
    if (M > 8192)      /* one tile holds every row of its matrix: 512 threads */
        return fail(WASTE_CUDA_E_ARG, "matrix: M = %d rows, at most 8192", M);
    if (!S.d_books || cb_base + stages > S.n_books)
        return fail(WASTE_CUDA_E_ARG, "codebooks not loaded or cb_base out of range");
    return 0;
}

int waste_cuda_vq_matvec(float *y, const uint8_t *idx, const uint16_t *scale,
                         const float *x, int M, int N, int cb_base, int stages)
{
    int rc = 0;
    if (!y || !idx || !scale || !x) return fail(WASTE_CUDA_E_ARG, "NULL pointer");
    pthread_mutex_lock(&g_mu);
    if ((rc = check_mat(M, N, cb_base, stages))) goto out;
    const size_t nrb = (size_t)(M + 63) / 64;
    const size_t ib = nrb * 64 * (N / 8) * stages, sb = (size_t)M * 2;
    const size_t xb = (size_t)N * 4, yb = (size_t)M * 4;
    const size_t pb = wc_matvec_part_floats(1, M, N) * 4;
    if ((rc = tmp_reserve(al256(ib) + al256(sb) + al256(xb) + al256(yb) + al256(pb)))) goto out;
    char *p = (char *)S.d_tmp;
    uint8_t *d_idx = (uint8_t *)p; p += al256(ib);
    uint16_t *d_sc = (uint16_t *)p; p += al256(sb);
    float *d_x = (float *)p; p += al256(xb);
    float *d_y = (float *)p; p += al256(yb);
    float *d_part = (float *)p;
    CK(cudaMemcpyAsync(d_idx, idx, ib, cudaMemcpyHostToDevice, S.stream), "idx H2D");
    CK(cudaMemcpyAsync(d_sc, scale, sb, cudaMemcpyHostToDevice, S.stream), "scale H2D");
    CK(cudaMemcpyAsync(d_x, x, xb, cudaMemcpyHostToDevice, S.stream), "x H2D");
    static wc_matvec_args a;          /* 4 KiB: kept off the stack */
    memset(&a, 0, sizeof a);
    a.G = 1; a.M = M; a.N = N; a.stages = stages; a.cb_base = cb_base;
    a.idx[0] = d_idx; a.scale[0] = d_sc; a.x[0] = d_x; a.y[0] = d_y;
    a.books = S.d_books;
    a.part = d_part;
    CK((cudaError_t)wc_matvec_launch(&a, S.stream), "matvec");
    CK(cudaMemcpyAsync(y, d_y, yb, cudaMemcpyDeviceToHost, S.stream), "y D2H");
    CK(cudaStreamSynchronize(S.stream), "matvec");
out:
    pthread_mutex_unlock(&g_mu);
    return rc;
}

int waste_cuda_vq_matvec_dev(int G, const uint8_t *const *idx, const uint16_t *const *scale,
                             const float *const *x, float *const *y, int M, int N,
                             int cb_base, int stages, void *stream)
{
    int rc = 0;
    if (G <= 0 || G > WC_MAX_G || !idx || !scale || !x || !y)
        return fail(WASTE_CUDA_E_ARG, "matvec_dev: G must be 1..%d, pointers non-NULL", WC_MAX_G);
    for (int g = 0; g < G; g++)
        if (((uintptr_t)idx[g] & 15) || ((uintptr_t)x[g] & 15))
            return fail(WASTE_CUDA_E_ARG, "matrix %d: index or x pointer not 16-byte aligned", g);
    pthread_mutex_lock(&g_mu);
    if ((rc = check_mat(M, N, cb_base, stages))) goto out;
    if ((rc = tmp_reserve(wc_matvec_part_floats(G, M, N) * 4))) goto out;
    static wc_matvec_args a;
    memset(&a, 0, sizeof a);
    a.G = G; a.M = M; a.N = N; a.stages = stages; a.cb_base = cb_base;
    for (int g = 0; g < G; g++) {
        a.idx[g] = idx[g]; a.scale[g] = scale[g]; a.x[g] = x[g]; a.y[g] = y[g];
    }
    a.books = S.d_books;
    a.part = (float *)S.d_tmp;
    CK((cudaError_t)wc_matvec_launch(&a, stream ? stream : (void *)S.stream), "matvec");
out:
    pthread_mutex_unlock(&g_mu);
    return rc;
}

/* Allocation-free form of vq_matvec_dev. The partial sums go to the fixed
 * device array behind wc_noalloc_setup instead of the growable scratch, so
 * no call makes cudaMalloc or cudaFree (whose implicit device-wide
 * synchronisation a running decode loop cannot afford, and which can fail
 * once the caller has reserved the device's memory). The array's address
 * is looked up, and its module and kernels loaded, when init binds the
 * device; shutdown forgets it, and the next init looks it up again. Every
 * partial a call reads back is written earlier in the same call, so
 * nothing has to start at zero. */

int waste_cuda_vq_matvec_dev_noalloc(int G, const uint8_t *const *idx,
                                     const uint16_t *const *scale, const float *const *x,
                                     float *const *y, int M, int N, int cb_base, int stages,
                                     void *stream)
{
    int rc = 0;
    if (G <= 0 || G > WC_MAX_G || !idx || !scale || !x || !y)
        return fail(WASTE_CUDA_E_ARG, "matvec_dev_noalloc: G must be 1..%d, pointers non-NULL",
                    WC_MAX_G);
    for (int g = 0; g < G; g++)
        if (((uintptr_t)idx[g] & 15) || ((uintptr_t)x[g] & 15))
            return fail(WASTE_CUDA_E_ARG, "matrix %d: index or x pointer not 16-byte aligned", g);
    pthread_mutex_lock(&g_mu);
    if ((rc = check_mat(M, N, cb_base, stages))) goto out;
    const size_t need = wc_matvec_part_floats(G, M, N) * sizeof(float);
    if (need > WASTE_CUDA_NOALLOC_SCRATCH_BYTES) {
        rc = fail(WASTE_CUDA_E_ARG,
                  "matvec_dev_noalloc: G=%d of %dx%d needs %zu bytes of partial sums, more than "
                  "the fixed %zu-byte scratch (G * ceil(N/64) * M * 4 must not exceed it)",
                  G, M, N, need, (size_t)WASTE_CUDA_NOALLOC_SCRATCH_BYTES);
        goto out;
    }
    int cur = -1;
    CK(cudaGetDevice(&cur), "cudaGetDevice");
    if (!S.inited || cur != S.device || !g_noalloc_part) {
        rc = fail(WASTE_CUDA_E_ARG, "matvec_dev_noalloc: current device %d is not the "
                  "library's device %d (waste_cuda_init binds it)", cur,
                  S.inited ? S.device : -1);
        goto out;
    }
    static wc_matvec_args a;
    memset(&a, 0, sizeof a);
    a.G = G; a.M = M; a.N = N; a.stages = stages; a.cb_base = cb_base;
    for (int g = 0; g < G; g++) {
        a.idx[g] = idx[g]; a.scale[g] = scale[g]; a.x[g] = x[g]; a.y[g] = y[g];
    }
    a.books = S.d_books;
    a.part = g_noalloc_part;
    CK((cudaError_t)wc_matvec_launch(&a, stream ? stream : (void *)S.stream), "matvec");
out:
    pthread_mutex_unlock(&g_mu);
    return rc;
}

/* ---- the matvec with interleaved table copies (matvec_sel.cu) ------------ */

static int sel_shape_ok(int M, int N, int stages, int copies)
{
    if ((copies != 2 && copies != 4) || stages != 3 || N <= 0 || N % 8 || M <= 2048 || M > 8192)
        return fail(WASTE_CUDA_E_ARG, "vq_sel: copies 2 or 4, 3 stages, 2048 < M <= 8192, "
                    "N a multiple of 8 (got copies %d, stages %d, %dx%d)", copies, stages, M, N);
    return 0;
}

size_t waste_cuda_vq_sel_bytes(int M, int N, int stages, int copies)
{
    if (sel_shape_ok(M, N, stages, copies)) return 0;
    return wc_sel_words(M, N, copies) * sizeof(uint32_t);
}

int waste_cuda_vq_sel_build_dev(const uint8_t *d_idx, void *d_sel, int M, int N, int stages,
                                int copies, void *stream)
{
    int rc = 0;
    if (!d_idx || !d_sel || ((uintptr_t)d_sel & 15))
        return fail(WASTE_CUDA_E_ARG, "vq_sel_build: NULL or unaligned (16 bytes) pointer");
    if ((rc = sel_shape_ok(M, N, stages, copies))) return rc;
    pthread_mutex_lock(&g_mu);
    if (!S.inited) { rc = fail(WASTE_CUDA_E_NODEV, "vq_sel_build before waste_cuda_init"); goto out; }
    CK((cudaError_t)wc_sel_build_launch(d_idx, (uint32_t *)d_sel, M, N, stages, copies,
                                        stream ? stream : (void *)S.stream), "copy-select build");
out:
    pthread_mutex_unlock(&g_mu);
    return rc;
}

int waste_cuda_vq_matvec_sel_dev(int G, const uint8_t *const *idx, const void *const *sel,
                                 const uint16_t *const *scale, const float *const *x,
                                 float *const *y, int M, int N, int cb_base, int stages,
                                 int copies, void *stream)
{
    int rc = 0;
    if (G <= 0 || G > WC_MAX_G || !idx || !sel || !scale || !x || !y)
        return fail(WASTE_CUDA_E_ARG, "matvec_sel_dev: G must be 1..%d, pointers non-NULL", WC_MAX_G);
    if ((rc = sel_shape_ok(M, N, stages, copies))) return rc;
    for (int g = 0; g < G; g++)
        if (((uintptr_t)idx[g] & 15) || ((uintptr_t)x[g] & 15) || ((uintptr_t)sel[g] & 15))
            return fail(WASTE_CUDA_E_ARG, "matrix %d: index, select or x pointer not 16-byte "
                        "aligned", g);
    pthread_mutex_lock(&g_mu);
    if ((rc = check_mat(M, N, cb_base, stages))) goto out;
    if ((rc = tmp_reserve(wc_matvec_part_floats(G, M, N) * 4))) goto out;
    static wc_matvec_args a;
    memset(&a, 0, sizeof a);
    a.G = G; a.M = M; a.N = N; a.stages = stages; a.cb_base = cb_base;
    for (int g = 0; g < G; g++) {
        a.idx[g] = idx[g]; a.scale[g] = scale[g]; a.x[g] = x[g]; a.y[g] = y[g];
        a.sel[g] = (const uint32_t *)sel[g];
    }
    a.books = S.d_books;
    a.part = (float *)S.d_tmp;
    CK((cudaError_t)wc_matvec_sel_launch(&a, copies, stream ? stream : (void *)S.stream),
       "matvec_sel");
out:
    pthread_mutex_unlock(&g_mu);
    return rc;
}

int waste_cuda_vq_dequant(float *W, const uint8_t *idx, const uint16_t *scale, int M, int N,
                          int cb_base, int stages)
{
    int rc = 0;
    if (!W || !idx || !scale) return fail(WASTE_CUDA_E_ARG, "NULL pointer");
    pthread_mutex_lock(&g_mu);
    if ((rc = check_mat(M, N, cb_base, stages))) goto out;
    const size_t nrb = (size_t)(M + 63) / 64;
    const size_t ib = nrb * 64 * (N / 8) * stages, sb = (size_t)M * 2, wb = (size_t)M * N * 4;
    if ((rc = tmp_reserve(al256(ib) + al256(sb) + wb))) goto out;
    uint8_t *d_idx = (uint8_t *)S.d_tmp;
    uint16_t *d_sc = (uint16_t *)((char *)S.d_tmp + al256(ib));
    float *d_W = (float *)((char *)S.d_tmp + al256(ib) + al256(sb));
    CK(cudaMemcpyAsync(d_idx, idx, ib, cudaMemcpyHostToDevice, S.stream), "idx H2D");
    CK(cudaMemcpyAsync(d_sc, scale, sb, cudaMemcpyHostToDevice, S.stream), "scale H2D");
    CK((cudaError_t)wc_dequant_launch(d_W, d_idx, d_sc, M, N, S.d_books, cb_base, stages,
                                      S.stream), "dequant");
    CK(cudaMemcpyAsync(W, d_W, wb, cudaMemcpyDeviceToHost, S.stream), "W D2H");
    CK(cudaStreamSynchronize(S.stream), "dequant");
out:
    pthread_mutex_unlock(&g_mu);
    return rc;
}
