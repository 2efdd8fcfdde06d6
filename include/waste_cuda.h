/*
 * waste_cuda.h — C ABI of the B200 (sm_100a) backend for WARP's routed-expert
 * FFN: 3-bit residual-VQ ("VQ3R") expert weights held resident in HBM, the
 * fused LUT matvec, and the MoE expert loop, behind the reference engine's
 * backend plugin interface (sqliteai/warp src/waste_backend.h).
 *
 * Every entry point is `extern "C"`, takes plain pointers and sizes, returns
 * an int status (0 = done; negative = the caller falls back or reports, as
 * the reference's slot contract asks) and hands the caller no memory to
 * free: what it allocates (banks, trunks, workspace, scratch) is its own and
 * goes with vq_bank_free / shutdown. Host-pointer entry points are synchronous: inputs are read and
 * outputs written before they return. `_dev` entry points take device
 * pointers and a cudaStream_t (as void*), and are ordered on that stream.
 *
 * Reference interfaces replaced (paths in the sqliteai/warp tree):
 *   waste_register_cuda          src/backend.c:57-59 (decl), :202-204 (call)
 *   waste_cuda_vq_bank_load      the expert cache: src/ecache.c:596
 *                                waste_ecache_get + src/model.c:1767 bank_fetch
 *   waste_cuda_codebooks_load*   src/model.c:1269-1304 codebook decode/transpose
 *   waste_cuda_lutb              src/model.c:1911-1923 vq_build_lut
 *                                (slot lutb_range, src/waste_backend.h:82)
 *   waste_cuda_vq_matvec(_dev)   src/model.c:2282-2289 vq_matvec
 *   waste_cuda_vq_dequant        tools/verify_container.py:73-84 (dequantised W)
 *   waste_cuda_vq4p_*            src/model.c:2026-2229 vq_quant_range / vq_rows_p6
 *                                (the WQ_VQ4P format, src/waste_format.h:57)
 *   waste_cuda_moe_experts       src/model.c:2873-2911 moe_layer's expert loop
 *   waste_cuda_moe_chunk_experts src/model.c:3585-3659 moe_chunk's expert loop
 *   waste_cuda_moe_layer(_dev)   src/model.c:2713-2939 moe_layer (router,
 *                                experts, shared expert) for a device-resident
 *                                hidden state
 *   waste_cuda_kda_step(_dev)    src/kda.c:26-68 waste_kda_step (slot kda_step,
 *                                src/waste_backend.h:69-72)
 *   waste_cuda_short_conv_*      src/kda.c:84-99 (slot short_conv_step)
 *   waste_cuda_kda_layer         src/model.c:2417-2472 kda_layer (whole layer)
 *   waste_cuda_mla_layer         src/model.c:2577-2649 mla_layer with its absorbed
 *                                head loop mla_head_range (:2530-2575)
 *   waste_cuda_rmsnorm_gated_*   src/kda.c:101-111 (slot rmsnorm_gated)
 *   waste_cuda_vq_encode(_dev)   src/vq.c:50-105 waste_vq_encode (the converter's
 *                                RVQ encoder, tools/convert.py:349-363)
 *   waste_cuda_vq_lloyd(_dev)    src/vq.c:107-136 waste_vq_lloyd
 *   waste_cuda_moe_block(_dev)   src/model.c:3927-3945 the MoE half of a
 *                                decoder layer: rmsnorm (:132-138), moe_layer,
 *                                residual add
 */
#ifndef WASTE_CUDA_H
#define WASTE_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define WASTE_CUDA_OK          0
#define WASTE_CUDA_E_ARG      -1  /* shape or argument outside what is supported */
#define WASTE_CUDA_E_DEVICE   -2  /* a CUDA call failed; see waste_cuda_last_error */
#define WASTE_CUDA_E_RECORD   -3  /* an expert record header failed its check      */
#define WASTE_CUDA_E_NOBANK   -4  /* the layer's bank (or trunk) is not loaded     */
#define WASTE_CUDA_E_NOMEM    -5  /* device memory exhausted                       */
#define WASTE_CUDA_E_NODEV    -6  /* no usable sm_100 device                       */

/* ---- plugin registration ----------------------------------------------
 * Replaces the missing src/cuda.cu that src/backend.c:57-59 declares and
 * src/backend.c:202-204 calls, once, under g_init_mu. Probes for an sm_100
 * device (WASTE_CUDA=0 declines; WASTE_CUDA_DEVICE picks one) and returns
 * the backend name, or NULL to decline so the previous backend stays
 * (src/waste_backend.h:116-120). A translation unit that includes the
 * engine's waste_backend.h first sees the engine's own prototype (a pointer
 * to its waste_kernels table); anywhere else the table is an opaque
 * pointer. Of that table it fills mvq_rows_f32 (the trunk matvec, see
 * waste_cuda_mvq_rows_dev; WASTE_CUDA_TRUNK=0 leaves it alone), kda_step
 * (WASTE_CUDA_KDA=0 leaves it), short_conv_step and rmsnorm_gated (only
 * with WASTE_CUDA_KDA_CONV=1 / WASTE_CUDA_KDA_NORM=1: their calls carry a
 * few KB each, and the host round trip costs more than the CPU's work),
 * and sets on_device, so the engine hands it whole row ranges — and the
 * whole head range of a KDA step — on the calling thread. The expert
 * path's slots are waste_vq_slots below. */
#ifdef WASTE_BACKEND_H
const char *waste_register_cuda(waste_kernels *t);
#else
const char *waste_register_cuda(void *waste_kernels_table);
#endif

/* The expert-path slots an engine adds next to waste_kernels: its
 * moe_layer and moe_chunk call them before their CPU expert loops, and its
 * loader uploads the banks through them. Filled by waste_register_cuda_vq;
 * a NULL slot means the engine keeps its CPU loop. */
typedef struct waste_moe_call waste_moe_call;
typedef struct waste_moe_chunk_call waste_moe_chunk_call;
typedef struct waste_cuda_kda_layer_desc waste_cuda_kda_layer_desc;
typedef struct waste_cuda_mla_layer_desc waste_cuda_mla_layer_desc;
typedef struct {
    int  (*codebooks_load)(const float *books, int n_books, int entries, int vec_dim);
    int  (*vq_bank_load)(int layer, int n_experts, size_t rec_bytes, int first,
                         int count, const void *records, int inter, int lat,
                         int stages);
    void (*vq_bank_free)(int layer);
    int  (*moe_experts)(const waste_moe_call *c);
    int  (*moe_chunk_experts)(const waste_moe_chunk_call *c);
    int  (*vq_bank_load_file)(int layer, int fd, int64_t offset, int n_experts,
                              size_t rec_bytes, int first, int count, int inter,
                              int lat, int stages);
    /* KDA recurrent state held in HBM (see waste_cuda_state_push/pull): the
     * engine pushes a state range after writing it on the host (reset,
     * snapshot load) and pulls it before reading it (snapshot save). */
    void (*state_push)(const void *host, size_t bytes);
    void (*state_pull)(void *host, size_t bytes);
    /* rmsnorm_gated over nh heads of C channels with one weight vector, in
     * one call (NULL unless WASTE_CUDA_KDA_NORM=1; the engine then loops
     * over heads through waste_kernels.rmsnorm_gated). */
    void (*rmsnorm_gated_heads)(int nh, int C, const float *x, const float *gate,
                                const float *weight, float eps, float *y);
    /* A whole moe_layer on the device for a layer whose trunk (F32 router,
     * optional bias, Q8G shared expert of group 128) the engine handed over
     * with moe_trunk_load and moe_activation: one token, out[hidden] =
     * routed experts (router order) + shared expert, routed[K] the chosen
     * ids (NULL allowed). A negative return leaves the engine's own path.
     * WASTE_CUDA_MOE_LAYER=0 leaves moe_layer NULL. */
    int  (*moe_trunk_load)(int layer, int n_experts, int hidden, int top_k, int renorm,
                           float routed_scale, const float *router, const float *bias,
                           int sh_inter, const int8_t *sh_gate, const uint16_t *sh_gate_s,
                           const int8_t *sh_up, const uint16_t *sh_up_s,
                           const int8_t *sh_down, const uint16_t *sh_down_s);
    int  (*moe_activation)(int layer, int act, float situ_beta, float situ_linear_beta);
    int  (*moe_layer)(int layer, const float *x, float *out, int *routed);
    /* A whole KDA attention layer on the device (see waste_cuda_kda_layer);
     * a negative return leaves the engine's own path. WASTE_CUDA_KDA_LAYER=0
     * or WASTE_CUDA_KDA=0 leaves it NULL. */
    int  (*kda_layer)(const waste_cuda_kda_layer_desc *d, const float *in, float *out);
    /* A whole MLA attention layer on the device (see waste_cuda_mla_layer);
     * a negative return leaves the engine's own path. WASTE_CUDA_MLA_LAYER=0
     * leaves it NULL. */
    int  (*mla_layer)(const waste_cuda_mla_layer_desc *d, int pos, const float *in, float *out);
} waste_vq_slots;

/* Fills `s` and returns 0, or returns WASTE_CUDA_E_NODEV (slots left NULL). */
int waste_register_cuda_vq(waste_vq_slots *s);

/* ---- device and lifetime ------------------------------------------------ */
/* Binds the calling process to `device` (-1: WASTE_CUDA_DEVICE or 0) and
 * allocates the workspace. Idempotent for the same device. */
int         waste_cuda_init(int device);
void        waste_cuda_shutdown(void);
int         waste_cuda_device(void);
const char *waste_cuda_last_error(void);
/* "CUDA sm_100a (<device name>)" once initialised, else NULL. */
const char *waste_cuda_backend_name(void);

/* ---- codebooks ---------------------------------------------------------
 * books: [n_books][entries][vec_dim] fp32, as the engine holds them after
 * load (m->codebooks, src/model.c:1275-1288 — subnormals already flushed).
 * The _f16 form takes the raw codebooks.bin entries and decodes them the
 * way the engine's loader does (src/model.c:1278-1287: f16 -> f32 with
 * subnormals flushed to signed zero). entries 256 (VQ3R, VQ2R) or 64
 * (VQ4P); vec_dim 8. */
int waste_cuda_codebooks_load(const float *books, int n_books, int entries,
                              int vec_dim);
int waste_cuda_codebooks_load_f16(const uint16_t *raw, int n_books, int entries,
                                  int vec_dim);

/* ---- expert banks resident in HBM ---------------------------------------
 * Uploads records [first, first+count) of layer `layer`'s bank (records are
 * the on-disk waste_expert_hdr + payload, src/waste_format.h:98-132, each
 * rec_bytes long). Every header is checked the way src/model.c:1698-1745
 * record_check does (magic, identity, size, fmt, lowrank, codebook range,
 * offset order, room for the scales) before anything is copied. The first
 * call for a layer sizes its bank for n_experts records; the shapes are
 * gate/up [inter][lat] and down [lat][inter]. stages 2 or 3: VQ2R/VQ3R
 * records (256-entry codebooks); stages 4: VQ4P records (64-entry
 * codebooks, see below). A caller that shards the experts loads only the
 * records it owns (first/count); the others stay absent and a call that
 * names one fails with WASTE_CUDA_E_ARG. */
int  waste_cuda_vq_bank_load(int layer, int n_experts, size_t rec_bytes,
                             int first, int count, const void *records,
                             int inter, int lat, int stages);
void waste_cuda_vq_bank_free(int layer);

/* The same records read straight from a bank file: record e of the layer
 * at byte offset + e * rec_bytes of `fd` (src/model.c:1767-1795 bank_fetch
 * reads them there, offset 0). Ranges of whole records (up to 64 MB) are
 * read with pread into two pinned staging buffers, and each range's upload
 * overlaps the read of the next; every header is checked before its range
 * is copied. The buffers are page aligned, so a file opened for direct I/O
 * (O_DIRECT) reads too. Replaces, for a bank resident in HBM, the engine's
 * expert cache (src/ecache.c) and its per-record reads. Returns once the
 * records are in HBM. */
int  waste_cuda_vq_bank_load_file(int layer, int fd, int64_t offset, int n_experts,
                                  size_t rec_bytes, int first, int count, int inter,
                                  int lat, int stages);

/* Reserves HBM for records [first, first+count) of a layer of n_experts
 * ahead of loading, for a caller that holds only part of the experts. Later
 * loads must fall inside the range. Without it, a layer's first
 * vq_bank_load reserves the whole layer (or, after waste_cuda_ep_init, this
 * rank's range). No counterpart in the reference, which reads every expert
 * from disk on one host. */
int  waste_cuda_vq_bank_reserve(int layer, int n_experts, size_t rec_bytes,
                                int first, int count, int inter, int lat,
                                int stages);

/* Trunk tensors of one MoE layer for the device-resident layer path:
 * router [n_experts][hidden] fp32 (F32 per docs/FORMAT.md), its score
 * correction bias (NULL = none), the routing constants, and the shared
 * expert as Q8G rows (group 128, rows padded to whole groups, one f16 scale
 * per group; src/model.c:265-320 layout). sh_inter 0 = no shared expert. */
int waste_cuda_moe_trunk_load(int layer, int n_experts, int hidden, int top_k,
                              int renorm, float routed_scale,
                              const float *router, const float *bias,
                              int sh_inter, const int8_t *sh_gate,
                              const uint16_t *sh_gate_s, const int8_t *sh_up,
                              const uint16_t *sh_up_s, const int8_t *sh_down,
                              const uint16_t *sh_down_s);

/* The gated activation the device-routed paths of a layer use (the whole
 * layer, the block, expert parallel, prefill_dev) for its routed and shared
 * experts: act 0 = SiLU(g)*u (the default), act 1 = SiTU with situ_beta > 0
 * and situ_linear_beta (<= 0: u unsquashed) — the model's act_situ,
 * activation_situ_beta and activation_situ_linear_beta
 * (src/model.c:987-990). The expert-loop slots take it per call instead. */
int waste_cuda_moe_activation(int layer, int act, float situ_beta,
                              float situ_linear_beta);

/* ---- the expert loop (decode) ------------------------------------------
 * What moe_layer's serial loop computes (src/model.c:2873-2911) for one
 * token: gate/up tables built once from x, then per routed expert j in
 * router order gate, up, the gated activation, down, and ysum = sum_j
 * w[j]*acc_j accumulated in j order. idx/w/x/ysum are host pointers owned
 * by the caller (m->... in the engine). act 0 = SiLU(g)*u (src/model.c:501);
 * act 1 = K3's SiTU, waste_situ_pair(g, u, situ_beta, situ_linear_beta)
 * (src/model.c:505-509, the model's act_situ). */
struct waste_moe_call {
    int layer, K;
    const int *idx;
    const float *w;
    const float *x;      /* [lat]  */
    float *ysum;         /* [lat]  */
    int lat, inter;
    int act;
    float situ_beta, situ_linear_beta;
};
int waste_cuda_moe_experts(const waste_moe_call *c);

/* ---- the expert loop (prefill chunk) ------------------------------------
 * moe_chunk's loop (src/model.c:3585-3659): nT tokens, route/rw [nT][K]
 * (router order per token), x and ysum [nT][lat]. Per token the expert
 * contributions are added in ascending expert id, as the reference does. */
struct waste_moe_chunk_call {
    int layer, nT, K;
    const int *route;
    const float *rw;
    const float *x;      /* [nT][lat] */
    float *ysum;         /* [nT][lat] */
    int lat, inter;
    int act;
    float situ_beta, situ_linear_beta;
};
int waste_cuda_moe_chunk_experts(const waste_moe_chunk_call *c);

/* The prefill expert loop on the tensor cores, device pointers: T tokens
 * (T*K <= 65536), route/rw [T][K] (router order), x/out [T][lat]. Computes
 * what moe_chunk_experts does (per token, experts added in ascending id) as
 * dense tiles: each expert's weights are dequantised into shared memory
 * once per 128 routed tokens and multiplied on the tensor cores (tcgen05)
 * with split-fp16 operands, within 2e-5 of the fp32 loop. Needs 3-stage
 * codebooks that are exact in fp16 (as loaded from codebooks.bin), rows in
 * multiples of 128, and every record of the layer's bank range loaded;
 * experts outside the bank are skipped and flagged
 * (WASTE_CUDA_DERR_BAD_EXPERT). moe_chunk_experts takes this path itself
 * when a chunk has at least two routed tokens per expert on average
 * (WASTE_CUDA_PREFILL_TC=0 keeps it on the lookup path). Ordered on
 * `stream`. */
int waste_cuda_moe_prefill_dev(int layer, int T, int K, const int *d_route,
                               const float *d_rw, const float *d_x,
                               float *d_out, void *stream);

/* ---- the whole MoE layer -------------------------------------------------
 * moe_layer (src/model.c:2713-2939) for a Kimi-Linear-shaped layer: router
 * matvec, sigmoid + bias top-K (strict >, lowest index wins ties), renorm
 * (+1e-20) and routed scale, the routed experts, and the shared expert.
 * Host form: x/out [hidden] and optional routed idx / weights [K] are host
 * pointers. _dev form: device pointers, ordered on `stream`, nothing copied. */
int waste_cuda_moe_layer(int layer, const float *x, float *out, int *routed,
                         float *weights);
int waste_cuda_moe_layer_dev(int layer, const float *d_x, float *d_out,
                             int *d_idx, float *d_w, void *stream);

/* ---- the MoE block: the MoE half of a decoder layer ----------------------
 * What the decode step does around moe_layer (src/model.c:3927-3945, a model
 * without attention residuals): norm = rmsnorm(h) with the layer's
 * post_attention_layernorm weight (src/model.c:132-138: r = 1/sqrtf(sum
 * h*h / n + eps), norm = h*r*w), resid = moe_layer(norm), h_out = h + resid.
 * The router normalises h on the device and every kernel of the layer
 * works on that; the combine adds h. So the output of one layer's block is
 * the next layer's input on the same stream, with no host step between.
 * waste_cuda_moe_norm_load gives a layer (whose trunk is loaded) its norm
 * weight [hidden] and eps. _dev: T (1..64) tokens, device pointers, every
 * expert held here; d_h_out may equal d_h. Host form: one token, host
 * buffers, like waste_cuda_moe_layer. */
int waste_cuda_moe_norm_load(int layer, int hidden, const float *norm_w, float eps);
int waste_cuda_moe_block(int layer, const float *h, float *h_out, int *routed,
                         float *weights);
int waste_cuda_moe_block_dev(int layer, int T, const float *d_h, float *d_h_out,
                             int *d_idx, float *d_w, void *stream);

/* The local part of a layer whose experts are spread over several devices:
 * T (1..64) tokens through the device router (the same routes on every
 * device), the routed experts THIS bank holds (all of its range loaded) in
 * router order, and the shared expert for tokens [sh_t0, sh_t1) only.
 * d_out[T][hidden] receives these partial sums; a token's output is the sum
 * of the partials over the devices, which hold disjoint ranges and add the
 * shared expert once. d_idx/d_w [T][K] receive the routes. For callers
 * that run their own exchange; waste_cuda_ep_moe_layer_dev and _rep_dev
 * wrap it with the library's own. Ordered on `stream`. */
int waste_cuda_moe_layer_part_dev(int layer, int T, const float *d_x,
                                  float *d_out, int sh_t0, int sh_t1,
                                  int *d_idx, float *d_w, void *stream);

/* ---- expert parallelism (one process per GPU, NVLink peer memory) --------
 * `world` processes share every MoE layer; rank r holds the contiguous
 * expert range [r*E/world, (r+1)*E/world) (waste_cuda_ep_range), and the
 * trunk (router, bias, shared expert) is replicated. Sequence per process:
 * waste_cuda_init(device); rank 0 calls waste_cuda_ep_unique_id and hands
 * the bytes to every rank over any channel; every rank calls
 * waste_cuda_ep_init (it returns once all have joined); then codebooks,
 * banks (each rank uploads only its own records: a layer's first
 * vq_bank_load after ep_init reserves the rank's range; a layer call
 * refuses a bank whose range is not the rank's) and trunks.
 * waste_cuda_ep_moe_layer_dev: every rank passes its own T tokens (the same
 * T everywhere, world*T <= 64). Every rank's tokens reach every rank, each
 * routes all of them, runs its own experts for every token routed there,
 * adds the shared expert for its own tokens, and sends each token's partial
 * sum to the token's rank, which adds them in rank order: each rank
 * receives its own tokens' outputs d_out[T][hidden]. d_idx/d_w (optional,
 * [T][K]) receive its tokens' routes. The exchange runs inside the layer's
 * kernels through every rank's mailbox, mapped into every other rank's
 * address space over NVLink (CUDA IPC, set up by the first call, which is
 * collective); where a mapping fails on any rank, every rank uses NCCL
 * instead (all-gather, reduce-scatter), as it does with
 * WASTE_CUDA_EP_P2P=0. Ordered on `stream`; every rank must make the same
 * calls in the same order. NCCL (for set-up and the fallback) is loaded at
 * run time (libnccl.so.2); without it these return WASTE_CUDA_E_NODEV. No
 * counterpart in the reference, which runs on one host.
 * A wait on a peer's flag gives up after WASTE_CUDA_EP_WAIT_POLLS polls
 * (environment, read by ep_init; default 2^24, several seconds) and sets
 * WASTE_CUDA_DERR_PEER_WAIT, so a rank that never makes its call costs the
 * others an error, not a hang. After that the ranks' exchange is out of
 * step: the rank that gave up also marks every rank's mailbox, so every
 * rank's later layer calls fail on the device (PEER_WAIT again, outputs not
 * valid), and once waste_cuda_device_errors has reported the bit, the
 * library refuses further ep layer calls with WASTE_CUDA_E_DEVICE. Recovery:
 * every rank calls waste_cuda_ep_shutdown and then waste_cuda_ep_init with a
 * new id, which builds new mailboxes. */
int  waste_cuda_ep_range(int n_experts, int rank, int world, int *first,
                         int *count);
int  waste_cuda_ep_unique_id(void *id, size_t bytes);   /* >= 128 bytes */
int  waste_cuda_ep_init(int rank, int world, const void *id, size_t bytes);
void waste_cuda_ep_shutdown(void);
int  waste_cuda_ep_moe_layer_dev(int layer, int T, const float *d_x,
                                 float *d_out, int *d_idx, float *d_w,
                                 void *stream);
/* The same layer for a batch that every rank holds (replicated trunk, e.g.
 * a batch of one): every rank passes the SAME T tokens (1..64), runs its
 * own experts for all of them, and every rank receives all T outputs, each
 * the sum of the ranks' partial sums in rank order (NCCL all-reduce on the
 * fallback path). The shared expert runs once per token, on one rank of a
 * split of the tokens. d_idx/d_w receive all T routes. */
int  waste_cuda_ep_moe_layer_rep_dev(int layer, int T, const float *d_x,
                                     float *d_out, int *d_idx, float *d_w,
                                     void *stream);
/* The MoE block (see waste_cuda_moe_block) over the same exchange: every
 * rank normalises the tokens it routes, and each token's h is added once,
 * on the rank that receives its output. Same call rules as ep_moe_layer_dev
 * and _rep_dev. */
int  waste_cuda_ep_moe_block_dev(int layer, int T, const float *d_h,
                                 float *d_h_out, int *d_idx, float *d_w,
                                 void *stream);
int  waste_cuda_ep_moe_block_rep_dev(int layer, int T, const float *d_h,
                                     float *d_h_out, int *d_idx, float *d_w,
                                     void *stream);

/* Sticky error bits raised on the device. Every wait inside a kernel is
 * bounded; when one runs out, the kernel sets a bit and skips its work
 * instead of hanging:
 *   WASTE_CUDA_DERR_ROUTE_WAIT  the gate/up kernel waited too long for the
 *                               router kernel's route flag;
 *   WASTE_CUDA_DERR_TMA_WAIT    a bulk copy into shared memory did not
 *                               complete in time.
 * The host forms check these themselves and return WASTE_CUDA_E_DEVICE;
 * callers of the _dev forms call this after synchronising. Waits for the
 * library's stream; reading clears the bits. */
#define WASTE_CUDA_DERR_ROUTE_WAIT 1u
#define WASTE_CUDA_DERR_TMA_WAIT   2u   /* also: a tensor-core commit that never came */
#define WASTE_CUDA_DERR_BAD_EXPERT 4u   /* a device-side route named an expert not held */
#define WASTE_CUDA_DERR_PEER_WAIT  8u   /* expert parallel: a peer's token or partial-sum
                                           flag did not arrive (a rank that did not make
                                           the call); the layer's outputs are not valid */
unsigned waste_cuda_device_errors(void);

/* ---- single VQ3R kernels ---------------------------------------------------
 * lutb: lut[nv][stages][entries] = sum_d x[8v+d] * C_{cb_base+s}[c][d], an
 * FMA chain from 0 in d order — bit-identical to the reference's AVX2 and
 * AVX-512 lutb_range (src/simd_avx2.c:100-133, src/simd_avx512.c:90-123).
 * vq_matvec: y[M] = f16(scale[r]) * sum_v (L0[i0]+L1[i1]+L2[i2]) over the
 * blocked index layout [M/64][N/8][64][stages] (src/model.c:1956-2024).
 * vq_dequant: W[M][N] = (((0 + C0[i0]) + C1[i1]) + C2[i2]) * f16(scale[r]).
 * Shapes: N a multiple of 8, M at most 8192 for the matvecs. */
int waste_cuda_lutb(float *lut, const float *x, int cb_base, int nv, int stages);
int waste_cuda_vq_matvec(float *y, const uint8_t *idx, const uint16_t *scale,
                         const float *x, int M, int N, int cb_base, int stages);
int waste_cuda_vq_dequant(float *W, const uint8_t *idx, const uint16_t *scale,
                          int M, int N, int cb_base, int stages);

/* ---- VQ4P ----------------------------------------------------------------
 * The engine's other 3-bit expert format (WQ_VQ4P, src/waste_format.h:57):
 * four residual stages of 64-entry codebooks, the four 6-bit indices of a
 * row and position packed little-endian into three bytes
 * (tools/convert.py:315-337), in the same blocked layout [M/64][N/8][64][3].
 * The fp32 table is quantised to int8 with one scale per 32 positions and
 * the sums stay integers until a per-block fold (src/model.c:2026-2229
 * vq_quant_range / vq_rows_p6), so results are bit-identical to the CPU's.
 * Needs codebooks loaded with entries = 64. A bank loaded with stages = 4
 * holds VQ4P records (fmt 8); moe_experts and moe_chunk_experts run it, and
 * the device-routed layer, block, prefill and expert-parallel entry points
 * (VQ3R only) return WASTE_CUDA_E_ARG for it. Its gated activation uses
 * correctly rounded exp and tanh (libm's float versions miss the correct
 * rounding on a few inputs, which the int8 re-quantisation of the down
 * table can turn into a whole table step).
 * vq4p_matvec(_dev): y = VQ4P(idx, scale) . x, any M, N a multiple of 8;
 * the _dev form runs G (1..120) matrices of one shape, idx[g] 8-byte
 * aligned. vq4p_table: the int8 tables q[N/8][4][64] and scales
 * qs[ceil(N/256)] of x against books cb_base..cb_base+3 (vq_build_lut then
 * vq_quant_lut). */
int waste_cuda_vq4p_matvec(float *y, const uint8_t *idx, const uint16_t *scale,
                           const float *x, int M, int N, int cb_base);
int waste_cuda_vq4p_matvec_dev(int G, const uint8_t *const *idx,
                               const uint16_t *const *scale,
                               const float *const *x, float *const *y, int M,
                               int N, int cb_base, void *stream);
int waste_cuda_vq4p_table(int8_t *q, float *qs, const float *x, int N, int cb_base);

/* Batched independent matvecs on device pointers: for g < G (1..120),
 * y[g][M] = VQ(idx[g], scale[g]) . x[g][N]. idx/scale/x/y are arrays of G
 * device pointers held in HOST memory; idx[g] and x[g] 16-byte aligned.
 * One gather launch for all G, then one reduce launch. */
int waste_cuda_vq_matvec_dev(int G, const uint8_t *const *idx,
                             const uint16_t *const *scale,
                             const float *const *x, float *const *y, int M,
                             int N, int cb_base, int stages, void *stream);

/* vq_matvec_dev for callers that cannot allocate device memory once they
 * run: a decode loop that reserved the device's memory for weights and
 * state at load time (a late cudaMalloc can then fail), or one that cannot
 * take the device-wide synchronisation of cudaFree while other streams
 * work. vq_matvec_dev grows its partial-sum scratch with cudaFree and
 * cudaMalloc; this entry point allocates nothing and keeps the partial
 * sums in a fixed array of WASTE_CUDA_NOALLOC_SCRATCH_BYTES (32 MiB)
 * compiled into the library. It has no counterpart in the reference.
 *  - Limit: G * ceil(N/64) * M * 4 bytes must fit the array (G = 32
 *    matrices of 4096 x 4096 fill it exactly); larger calls return
 *    WASTE_CUDA_E_ARG with the sizes in waste_cuda_last_error().
 *  - The array is taken on the device when waste_cuda_init binds it (the
 *    library's module is loaded there then, and the array's address looked
 *    up), so every call after init allocates nothing, the first included.
 *    Every GPU the library is bound to holds the 32 MiB until the process
 *    exits. After waste_cuda_shutdown the next init looks the address up
 *    again.
 *  - The calling thread's current device must be the library's device.
 *  - Nothing in the array has to start at zero: each call writes every
 *    partial sum it reads back.
 *  - There is one array per device: calls whose kernels overlap on the GPU
 *    (different streams, or different host threads without ordering
 *    between their streams) race on it. Order them on one stream.
 * Arguments, alignment rules and results are those of vq_matvec_dev. */
#define WASTE_CUDA_NOALLOC_SCRATCH_BYTES ((size_t)32 << 20)
int waste_cuda_vq_matvec_dev_noalloc(int G, const uint8_t *const *idx,
                                     const uint16_t *const *scale,
                                     const float *const *x, float *const *y,
                                     int M, int N, int cb_base, int stages,
                                     void *stream);

/* ---- KDA (Kimi Delta Attention) decode step -----------------------------
 * src/kda.c:19-111 on the device, bit for bit except where glibc's expf is
 * not correctly rounded (the device's exp is; a few inputs in 10^4).
 * kda_step: q, k, g_log [H][K]; v, o [H][V]; beta [H]; S [H][K][V] updated
 * in place; K 32, 64 or 128. short_conv_step: C channels, kernel KS, w
 * [C][KS], bias [C] or NULL, ring [C][KS-1] (oldest first) updated,
 * y = SiLU(conv) (y may be x). rmsnorm_gated_heads: nh heads of C
 * channels, one weight vector, y = x * r * w * sigmoid(gate) per head (y
 * may be x).
 * Host-pointer forms (the slots): the state (S, ring) and the weights are
 * kept in HBM from the first call that names them, keyed by host address:
 * the host copy of a state is stale from then on — waste_cuda_state_pull
 * copies a range back, waste_cuda_state_push reloads it after the caller
 * wrote it (both cover every held copy that overlaps the range; ranges
 * nothing holds are left alone). A call whose state range partly overlaps
 * a held one fails with WASTE_CUDA_E_NOMEM. waste_cuda_release_host_buffers
 * drops every held copy. _dev forms: device pointers, ordered on `stream`. */
/* A whole KDA attention layer for one token (src/model.c:2417-2472
 * kda_layer): q/k/v projections each through its short conv, the f
 * low-rank path and the decay gate, beta = sigmoid(b_proj x), the KDA step
 * on the layer's state, the g path (low-rank, or full when g_full.W is
 * set), the gated rmsnorm per head and o_proj: out[hidden] from in[hidden]
 * in one call. Trunk tensors as the engine holds them (Q8G or Q4G rows of
 * `rowbytes`, f16 group scales), copied to HBM at first use and keyed by
 * host address like the trunk slot's; S and the three conv rings are the
 * engine's state, held in HBM like the kda_step slot's (state_push /
 * state_pull keep them coherent). */
typedef struct {
    const void *W;             /* rows x rowbytes quantised weights        */
    const uint16_t *ws;        /* rows x ceil(cols/group) f16 scales       */
    int rows, cols, bits, group;
    size_t rowbytes;
} waste_cuda_qtensor;
struct waste_cuda_kda_layer_desc {
    int H, D, conv_k, hidden;                   /* C = H * D channels      */
    waste_cuda_qtensor q, k, v, o, f_a, f_b, g_a, g_b, b, g_full;
    const float *conv_w[3];                     /* [C][conv_k] each        */
    const float *A_log;                         /* [H]                     */
    const float *dt_bias;                       /* [C] or NULL             */
    const float *o_norm;                        /* [D]                     */
    float lower_bound, eps;
    float *S;                                   /* [H][D][D]               */
    float *conv_ring[3];                        /* [C][conv_k - 1] each    */
};
int waste_cuda_kda_layer(const waste_cuda_kda_layer_desc *d, const float *in, float *out);

/* A whole MLA attention layer for one token at position `pos`
 * (src/model.c:2577-2649 mla_layer): the query (q_proj, or q_a_proj ->
 * rmsnorm -> q_b_proj when q_lora > 0), the latent kv_a_proj_with_mqa(in)
 * with kv_a_layernorm over its first kv_lora values, the rotary pairs
 * (skipped when nope is set), the latent stored at row pos of the layer's
 * cache, the absorbed attention of every head over rows 0..pos (q~ =
 * W_kb^T q_nope, scores times `scale`, softmax, context, W_vb), the optional
 * sigmoid output gate (g.W set), and o_proj: out[hidden] in one call. The
 * cache is the engine's latcache[L] ([kv_cap][kv_lora + qk_rope] floats):
 * held in HBM from the first call, keyed by host address; every call also
 * writes its new row into the host copy, so the engine's own reads of the
 * cache (a snapshot save) see it, and state_push after the engine writes
 * rows (a snapshot load) updates the HBM copy. kv_b_proj in 8- or 4-bit
 * groups; pos < kv_cap. Sums in the reference's order where it fixes one
 * (q~, the context, the softmax sum); the dot products lane-strided. */
struct waste_cuda_mla_layer_desc {
    int heads, qk_nope, qk_rope, v_head, kv_lora, q_lora, hidden, kv_cap;
    int nope;                                   /* 1: no rotary pairs      */
    waste_cuda_qtensor q, q_a, q_b, kv_a, kv_b, o, g;
    const float *q_a_norm;                      /* [q_lora], with q_lora   */
    const float *kv_a_norm;                     /* [kv_lora]               */
    const float *rope_inv_freq;                 /* [qk_rope / 2]           */
    float eps, scale;
    float *latcache;                            /* [kv_cap][kv_lora + qk_rope] */
};
int waste_cuda_mla_layer(const waste_cuda_mla_layer_desc *d, int pos, const float *in,
                         float *out);
int waste_cuda_kda_step(int H, int K, int V, const float *q, const float *k,
                        const float *v, const float *g_log, const float *beta,
                        float *S, float *o);
int waste_cuda_short_conv_step(int C, int KS, const float *w, const float *bias,
                               float *ring, const float *x, float *y);
int waste_cuda_rmsnorm_gated_heads(int nh, int C, const float *x, const float *gate,
                                   const float *weight, float eps, float *y);
int waste_cuda_state_push(const void *host, size_t bytes);
int waste_cuda_state_pull(void *host, size_t bytes);
int waste_cuda_kda_step_dev(int H, int K, int V, const float *q, const float *k,
                            const float *v, const float *g_log, const float *beta,
                            float *S, float *o, void *stream);
int waste_cuda_short_conv_dev(int C, int KS, const float *w, const float *bias,
                              float *ring, const float *x, float *y, void *stream);
int waste_cuda_rmsnorm_gated_dev(int nh, int C, const float *x, const float *gate,
                                 const float *weight, float eps, float *y, void *stream);

/* ---- the converter's residual-VQ encoder ----------------------------------
 * vq_encode: for each of n vectors X[n][dim] and each stage s, the index of
 * the entry of books[s] ([stages][entries][dim]) nearest to the residual
 * (squared Euclidean distance summed in dim order; the first index wins a
 * tie), written to out[n][stages], then subtracted — src/vq.c:50-105,
 * bit for bit. vq_lloyd: one Lloyd iteration of C [entries][dim] over X:
 * assign, then each non-empty cluster's centroid becomes the double sum of
 * its members in vector order over their count, rounded to float (empty
 * clusters keep theirs) — src/vq.c:107-136, bit for bit; returns the number
 * of non-empty clusters (host form) or writes it to *d_live (device form).
 * entries 1..256, dim 1..64, stages * entries * dim * 4 bytes <= 227 KB.
 * The host forms take the converter's buffers (its nthreads argument has
 * no counterpart); the _dev forms take device pointers and `stream`. */
int waste_cuda_vq_encode(const float *X, int n, const float *books, int stages,
                         int entries, int dim, uint8_t *out);
int waste_cuda_vq_encode_dev(const float *X, int n, const float *books, int stages,
                             int entries, int dim, uint8_t *out, void *stream);
int waste_cuda_vq_lloyd(const float *X, int n, float *C, int entries, int dim);
int waste_cuda_vq_lloyd_dev(const float *X, int n, float *C, int entries, int dim,
                            int *d_live, void *stream);

/* ---- the trunk matvec (the mvq_rows_f32 slot) ---------------------------
 * src/model.c:265-320 waste_mvq_rows_f32 on the device: y[r] for r in
 * [r0, r1) = sum over groups k of f16(ws[r][k]) * (sum over the group's
 * weights w*x), for Q8G (bits 8), Q4G (bits 4: two signed nibbles per byte,
 * low first, minus 8) and Q3G (bits 3: a 3-bit bitstream, minus 4) rows of
 * `rowbytes` bytes with `group` weights per f16 scale. Device pointers,
 * ordered on `stream`; within 2e-5 of the CPU kernel (sum order).
 * The slot waste_register_cuda installs does the same from the engine's
 * host tensors: it keeps an HBM copy of each tensor it sees (keyed by the
 * host address of its weights, made at first use), copies x in and y out,
 * and runs tensors below WASTE_CUDA_TRUNK_MIN bytes (default 1 MiB) — and
 * anything the device path cannot take — on the CPU kernel the slot held
 * before. waste_cuda_release_host_buffers drops those copies, and the KDA
 * state copies below (the engine calls it before freeing a model:
 * src/backend.c:223-229, waste_backend_release_host_buffers). */
int  waste_cuda_mvq_rows_dev(float *d_y, const void *d_W, const uint16_t *d_ws,
                             const float *d_x, int r0, int r1, int in, int group,
                             int bits, size_t rowbytes, void *stream);
void waste_cuda_release_host_buffers(void);

/* ---- the matvec with interleaved table copies ----------------------------
 * vq_matvec_dev with fewer shared-memory bank conflicts: every table entry
 * is held `copies` (2 or 4) times side by side, and each lookup reads the
 * copy a per-matrix copy-select stream names, chosen once so that the 32
 * lookups of a warp instruction spread over the banks. The sums are the
 * ones vq_matvec_dev computes, bit for bit (same order, same table values).
 * vq_sel_bytes: the stream's size for an M x N matrix (0 for shapes outside
 * 2048 < M <= 8192, N a multiple of 8, 3 stages). vq_sel_build_dev writes
 * the stream of one matrix from its index stream (device pointers, 16-byte
 * aligned; once per matrix, e.g. at load). No counterpart in the reference
 * (a CPU has no bank conflicts to avoid). */
size_t waste_cuda_vq_sel_bytes(int M, int N, int stages, int copies);
int    waste_cuda_vq_sel_build_dev(const uint8_t *d_idx, void *d_sel, int M, int N,
                                   int stages, int copies, void *stream);
int    waste_cuda_vq_matvec_sel_dev(int G, const uint8_t *const *idx,
                                    const void *const *sel, const uint16_t *const *scale,
                                    const float *const *x, float *const *y, int M, int N,
                                    int cb_base, int stages, int copies, void *stream);

/* Kernels this library launched since load (a running count, for
 * benchmarks that report how many of their launches were this library's). */
uint64_t waste_cuda_launch_count(void);

/* Phase timers: the device counterpart of the reference's WASTE_PROFILE
 * buckets (src/model.c:37-52, printed by tests/test_forward.c:118-134).
 * While on, each kernel is bracketed by CUDA events on its stream;
 * waste_cuda_profile_read waits for them, writes the summed milliseconds
 * and launch counts of up to nphase phases (order below), and resets. Not
 * for use while a stream is being captured into a CUDA graph. */
enum {
    WASTE_CUDA_PH_ROUTER = 0,   /* router logits + shared gate/up + top-K */
    WASTE_CUDA_PH_ACT,          /* SiLU(g)*u of batched calls            */
    WASTE_CUDA_PH_GATEUP,       /* routed gate/up gathers               */
    WASTE_CUDA_PH_DOWN,         /* SiLU(g)*u, down gathers, shared down */
    WASTE_CUDA_PH_COMBINE,      /* router-order reduce (+ shared)       */
    WASTE_CUDA_PH_MATVEC,       /* batched matvec gathers               */
    WASTE_CUDA_PH_MATVEC_REDUCE,
    WASTE_CUDA_PH_EP_PUBLISH,   /* expert parallel: tokens into the mailboxes */
    WASTE_CUDA_PH_EP_FINALIZE,  /* expert parallel: partial sums in rank order */
    WASTE_CUDA_PH_COUNT
};
int waste_cuda_profile(int on);
int waste_cuda_profile_read(double *ms, uint64_t *launches, int nphase);

#ifdef __cplusplus
}
#endif
#endif /* WASTE_CUDA_H */
