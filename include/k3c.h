/* k3c.h -- C ABI of libk3cuda.so, the B200 (sm_100a) routed-expert hot path.
 *
 * Two layers:
 *
 *   1. DROP-IN entry points with the reference's exact names, signatures and semantics
 *      (host pointers in, host pointers out, void return, abort on a precondition
 *      violation). Linking libk3cuda.so in place of the reference's k3_ops.o routes these
 *      calls through the GPU. Each cites the declaration it replaces in the reference's
 *      include/k3/k3.h.
 *
 *   2. DEVICE entry points (k3c_*): device pointers, an explicit CUDA stream, an int
 *      status (K3C_OK or a negative K3C_E* code, message in k3c_last_error()). These are
 *      the performance path; nothing in them synchronises the host unless stated.
 *
 * Reference types (K3ExpertQ, K3ExpertSrc) are mirrored field-for-field so the ABI is the
 * reference's; when the reference's k3.h is included first its definitions are used.
 */
#ifndef K3C_H
#define K3C_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------- mirrored types ---- */
#ifndef K3_H
#define K3_MXFP4_GROUP 32   /* include/k3/k3.h:548 */
#define K3_MAX_TOPK 64      /* include/k3/k3.h:557 */
enum { K3_WF32 = 0, K3_WBF16 = 1, K3_WI8 = 2 };   /* include/k3/k3.h:270 */

/* One expert as three (packed, scale) pairs: include/k3/k3.h:323-327. In the k3c_* API
 * these are DEVICE addresses. */
typedef struct {
    const unsigned char *p1, *s1;   /* w1 gate */
    const unsigned char *p3, *s3;   /* w3 up   */
    const unsigned char *p2, *s2;   /* w2 down */
} K3ExpertQ;

/* Expert source vtable: include/k3/k3.h:332-355. */
typedef struct K3ExpertSrc {
    int (*get)(struct K3ExpertSrc *self, int layer, int expert, K3ExpertQ *out);
    int (*getmany)(struct K3ExpertSrc *self, int layer, const int *experts, int n);
    int (*resident)(struct K3ExpertSrc *self, int layer, int expert, K3ExpertQ *out);
    void *ctx;
} K3ExpertSrc;

/* Model configuration, include/k3/k3.h:73-116, field for field (k3_moe reads hidden,
 * rms_eps, n_experts, topk, n_shared, latent, moe_inter, routed_scale, moe_renorm,
 * latent_norm, situ_b1, situ_b2). */
typedef struct {
    int hidden;
    int n_layers;
    int vocab;
    float rms_eps;
    int kda_heads;
    int kda_head_dim;
    int conv_k;
    float gate_lb;
    int n_heads;
    int q_lora;
    int kv_lora;
    int qk_nope;
    int qk_rope;
    int v_head;
    int mla_out_gate;
    int n_experts;
    int topk;
    int n_shared;
    int latent;
    int moe_inter;
    float routed_scale;
    int moe_renorm;
    int latent_norm;
    int first_dense;
    int dense_inter;
    int attn_res_block;
    float situ_b1;
    float situ_b2;
    int n_full_attn;
    int *full_attn;
} K3Cfg;

/* Latent MoE layer weights, include/k3/k3.h:357-380, field for field. HOST addresses.
 * gate/bias fp32; w1/w3/w2 the fp32 resident bank ([e][moe_inter][latent] gate and up,
 * [e][latent][moe_inter] down), used when src is NULL; down/up/sh1/sh3/sh2 tagged by wdt. */
typedef struct {
    const float *gate, *bias;
    const float *w1, *w3, *w2;
    const float *latent_norm;
    const void *down, *up;
    const void *sh1, *sh3, *sh2;
    int wdt;
    struct K3ExpertSrc *src;
    int layer;
    int cache_only;
} K3MoeW;
#endif /* K3_H */

/* Binary-compatible with cudaStream_t; NULL is the legacy default stream. */
typedef struct CUstream_st *k3c_stream_t;

/* --------------------------------------------------------------- status codes ---- */
enum {
    K3C_OK = 0,
    K3C_EINVAL = -1,     /* bad argument (shape, alignment, range)          */
    K3C_ECUDA = -2,      /* a CUDA call failed                              */
    K3C_ENOMEM = -3,     /* device or pinned allocation failed              */
    K3C_ETIMEOUT = -4,   /* a bounded device wait gave up                   */
    K3C_ENOTFOUND = -5,  /* expert not resident / not registered            */
    K3C_EFULL = -6       /* every pool slot is pinned or in flight          */
};
/* Message for the last failing k3c_* call on this host thread ("" if none). */
const char *k3c_last_error(void);
/* Library version string and the compiled device architecture ("sm_100a"). */
const char *k3c_version(void);

/* Instrumentation (no reference counterpart; the reference times its stages with wall
 * clocks, src/cache/k3_cache.c:90-102). k3c_launch_count: kernels this library has
 * launched since load. k3c_timing_enable(1) makes the k3c_* entry points record CUDA
 * events around their stages on the launching stream; k3c_timing_read sums and resets
 * the elapsed milliseconds and call counts per stage, in the order
 * {experts, router, combine, q8, dispatch} (dispatch: the prefill's token quantisation into
 * its pairs' rows, which under expert parallelism reads the tokens of other ranks). */
long long k3c_launch_count(void);
void k3c_timing_enable(int on);
int k3c_timing_read(double *ms, long long *count, int nstage);
/* No reference counterpart (the reference has no device waits). Runs the bounded-wait helpers
 * every pipelined kernel here uses on a wait nothing satisfies -- kind 0: an mbarrier phase,
 * kind 1: a release/acquire counter -- with a limit of limit_ms (<= 2000; the kernels use
 * 2000): returns K3C_ETIMEOUT and the context stays usable. kind 2 (a satisfied counter)
 * returns K3C_OK. Synchronises `stream`. */
int k3c_selftest_wait(int kind, double limit_ms, k3c_stream_t stream);

/* Activation / weight element types used by the k3c_* entry points. */
enum { K3C_F32 = 0, K3C_BF16 = 1 };
/* Expert activation functions. */
enum { K3C_ACT_SWIGLU = 0, K3C_ACT_SITU = 1 };
/* Trunk weight types, the reference's K3_WF32 / K3_WBF16 / K3_WI8 (include/k3/k3.h:270). */
enum { K3C_WF32 = 0, K3C_WBF16 = 1, K3C_WI8 = 2 };
/* A per-row int8 trunk matrix in the layout k3c_q8_pack makes (device arrays): the draft
 * model's K3_WI8 weights (rows [f32 scale][int8 * in] in its files, tools/int8_trunk.py:33-45). */
typedef struct {
    const int8_t *wq;       /* [out][ldw] */
    const float *wscale;    /* [out] */
    int ldw;
} k3c_q8_mat;

/* ====================================================================================
 * 1. DROP-IN ENTRY POINTS (host pointers)
 * ==================================================================================== */

/* include/k3/k3.h:559-560. out[rows][2*pcols] = E2M1(nibble) * 2^(scale-127); the LOW nibble
 * is the EVEN element; scale 255 gives 0. Bit-exact with the reference. */
void k3_mxfp4_dequant(float *out, const unsigned char *packed,
                      const unsigned char *scales, int rows, int pcols, int group);

/* include/k3/k3.h:565-566. y[rows] = W[rows][in] . x[in] with W read as MXFP4 (packed
 * [rows][in/2], scales [rows][ceil(in/group)]). Aborts on odd `in` or group > 64, as the
 * reference does (src/core/k3_ops.c:1366-1384). */
void k3_matmul_mxfp4(float *y, const float *x, const unsigned char *packed,
                     const unsigned char *scales, int in, int rows, int group);

/* include/k3/k3.h:285. W is `out` rows of [f32 scale][int8 * in] (row stride 4+in). */
void k3_matmul_q8(float *y, const float *x, const void *W, int in, int out);

/* src/core/k3_ops.c:265 and include/k3/k3.h:281. y[out] = W[out][in] . x[in], fp32 or bf16
 * weights, bit-exact with the reference: its fixed order (16 double accumulators over
 * i%16 by fused multiply-adds, a fixed combining tree, the in%16 tail fused in order, one
 * rounding to float). */
void k3_matmul(float *y, const float *x, const float *W, int in, int out);
void k3_matmul_bf16(float *y, const float *x, const uint16_t *W, int in, int out);

/* include/k3/k3.h:241-243. Sigmoid scores, selection on score+bias, weights from the
 * unbiased score, optional renorm, times routed_scale; idx/w in descending order. */
void k3_router(int *idx, float *w, const float *x, const float *W,
               const float *bias, int hidden, int n_experts, int topk,
               int renorm, float routed_scale);

/* include/k3/k3.h:388: routed experts dropped from a sum because they failed to load. */
extern long k3_expert_drops;

/* include/k3/k3.h:382, src/core/k3_ops.c:556-656. The K3 latent MoE layer for T tokens:
 * out[T][hidden] from x[T][hidden] (host fp32). Per token: route on the full width
 * (w->gate, w->bias); with w->cache_only and w->src->resident, keep only the resident top-k
 * experts and renormalise their weights; z = down x; the selected experts on z at the latent
 * width (from w->src: getmany of the top-k, then get() -- or resident() when cache_only --
 * for each; a failed get is counted in k3_expert_drops with the reference's message and
 * skipped; without a source, the fp32 bank w->w1/w3/w2), summed with their weights in top-k
 * order; RMSNorm of the sum (c->latent_norm); up; plus the full-width shared expert
 * unweighted. idx/wt (host, topk entries) are left as the reference leaves them: the last
 * token's routing. scratch is accepted and not used (the work space is on the GPU), so
 * callers size it with k3_moe_scratch exactly as before.
 *
 * Experts run on the tcgen05 tensor cores (the routed-expert kernels of the k3c_* layer:
 * activations as three E4M3 terms up to 32 tokens, two above) when the latent width and
 * moe_inter are multiples of 128 (the latent width of 256 above 32 tokens) and SiTU has the
 * K3 bounds 4 and 25: within 2e-2 of the reference's output (measured ~1e-5 up to 32 tokens).
 * Otherwise, for the fp32 bank, or with K3C_DROPIN_FP32=1 in the environment, they run as
 * fp32 GEMVs (k3_matmul's order for the bank, 1e-5 for MXFP4). Trunk matrices always run
 * bit-exact (k3_matmul / k3_matmul_bf16 order) or, for K3_WI8, as exact int32 sums.
 *
 * Experts from a source other than k3c_pool_source are copied (host or device memory) into
 * device staging right after each get(), within the reference's validity window; experts
 * from a k3c_pool_source are used in their pool slots (no copy) and released once the call's
 * kernels are enqueued. Weights are uploaded on every call unless
 * k3c_dropin_keep_weights(1) promises that weight arrays do not change at a given address.
 * Aborts, as the reference does, on a precondition violation or a CUDA failure. */
void k3_moe(float *out, const float *x, const K3MoeW *w, const K3Cfg *c, int T, int *idx,
            float *wt, float *scratch);
/* include/k3/k3.h:418-426, src/core/k3_ops.c:689-808. Same outputs as k3_moe; with a source,
 * more than one token, no cache_only and K3_NO_BATCH_PREFILL unset, the source sees the
 * reference's batched pattern: per 64-token chunk, getmany of the chunk's distinct experts
 * in first-seen order, then one get() per distinct expert (a failure drops that expert for the
 * whole chunk: one k3_expert_drops count, "this chunk is CORRUPT"); idx/wt are written only by
 * a final one-token chunk, as in the reference. Otherwise it is k3_moe. */
void k3_moe_prefill(float *out, const float *x, const K3MoeW *w, const K3Cfg *c, int T,
                    int *idx, float *wt, float *scratch);
/* include/k3/k3.h:381, src/core/k3_ops.c:658-666: the reference's scratch size in floats. */
size_t k3_moe_scratch(const K3Cfg *c);
/* No counterpart in the reference. 1: the drop-ins above keep a device copy of each weight
 * array (router, norm, trunk matrices, fp32 bank) keyed by its host address and size, so a
 * weight is uploaded once per process -- for callers whose weights stay put (the engine);
 * 0 (the default): every call uploads what it reads. k3c_dropin_forget_weights() frees the
 * kept copies. */
void k3c_dropin_keep_weights(int on);
void k3c_dropin_forget_weights(void);

/* ====================================================================================
 * 2. DEVICE ENTRY POINTS (device pointers, explicit stream)
 * ==================================================================================== */

/* Device form of k3_mxfp4_dequant (same layout and semantics). */
int k3c_mxfp4_dequant(float *out, const uint8_t *packed, const uint8_t *scales,
                      int rows, int pcols, int group, k3c_stream_t stream);

/* Batched MXFP4 GEMV: y[t*ldy + r] = sum_k W[r][k] * x[t*ldx + k] for t < ntok (fp32 x,
 * fp32 accumulate). Device form of k3_matmul_mxfp4 for ntok tokens at once. */
int k3c_mxfp4_gemv(float *y, int ldy, const float *x, int ldx, int ntok,
                   const uint8_t *packed, const uint8_t *scales, int in, int rows,
                   int group, k3c_stream_t stream);

/* INT8 per-row trunk projection, pool layout: wq [out][ldw] int8 (ldw >= in, a multiple of
 * 32, zero-padded) and wscale [out] fp32. k3c_q8_pack converts the reference's inline row layout
 * ([f32 scale][int8*in], stride 4+in, include/k3/k3.h:265-303), already on the device,
 * into that layout. k3c_q8_gemv: y[t*ldy + o] = wscale[o] * sum_i wq[o][i] * x[t][i], x of
 * type x_dtype (K3C_F32 or K3C_BF16) with row stride ldx elements. */
int k3c_q8_pack(int8_t *wq, float *wscale, int ldw, const void *w_rows, int in, int out,
                k3c_stream_t stream);
int k3c_q8_gemv(float *y, int ldy, const void *x, int x_dtype, int ldx, int ntok,
                const int8_t *wq, const float *wscale, int ldw, int in, int out,
                k3c_stream_t stream);
/* k3c_q8_gemv with caller-owned device scratch (k3c_q8_gemv_scratch bytes; depends on ntok,
 * in and out) instead of a stream-ordered allocation per call: K3C_EINVAL when too small. */
size_t k3c_q8_gemv_scratch(int ntok, int in, int out);
int k3c_q8_gemv_ws(float *y, int ldy, const void *x, int x_dtype, int ldx, int ntok,
                   const int8_t *wq, const float *wscale, int ldw, int in, int out,
                   void *scratch, size_t scratch_bytes, k3c_stream_t stream);

/* Router for ntok tokens: logits W.x accumulated in double, sigmoid as in the reference,
 * top-k selection on score+bias with strict-greater first-index ties, renorm, scale.
 * x: [ntok][hidden] of x_dtype; W: [n_experts][hidden] of w_dtype; bias fp32 or NULL.
 * idx/w: [ntok][topk]. scores (optional, may be NULL): [ntok][n_experts] fp32. */
int k3c_router(int *idx, float *w, float *scores, const void *x, int x_dtype,
               const void *W, int w_dtype, const float *bias, int hidden, int n_experts,
               int topk, int renorm, float routed_scale, int ntok, k3c_stream_t stream);
/* k3c_router with caller-owned device scratch (k3c_router_scratch bytes) instead of a
 * stream-ordered allocation per call. */
size_t k3c_router_scratch(int hidden, int n_experts, int ntok);
int k3c_router_ws(int *idx, float *w, float *scores, const void *x, int x_dtype,
                  const void *W, int w_dtype, const float *bias, int hidden, int n_experts,
                  int topk, int renorm, float routed_scale, int ntok, void *scratch,
                  size_t scratch_bytes, k3c_stream_t stream);
/* The draft model's cache-only routing (src/core/k3_ops.c:580-593), on the device: for each
 * token of idx/wt [ntok][topk] (as a router wrote them), keep the entries whose expert has a
 * resident run (0 <= run_of[e] < n_runs, run_of device [n_experts]: the test the expert
 * kernels apply) in their top-k order, divide the kept weights by their float sum when it is
 * positive, and set the remaining entries to expert -1 with weight 0. Run the layer with that
 * routing through a routed entry point (k3c_moe_decode_tc_routed, k3c_moe_prefill_tc_routed,
 * k3c_moe_latent_decode_routed) with drops = NULL: the emptied entries are skipped, and the
 * reference counts no drops in this mode. The run table of resident experts comes from
 * k3c_pool_acquire_resident (pinned, copies complete on the stream). */
int k3c_route_cache_only(int *idx, float *wt, int ntok, int topk, const int *run_of, int n_experts,
                         int n_runs, k3c_stream_t stream);
/* Selection stage alone, on given fp32 scores [ntok][n_experts]: the parity boundary at
 * which indices must match the reference bit-exactly. */
int k3c_router_select(int *idx, float *w, const float *scores, const float *bias,
                      int n_experts, int topk, int renorm, float routed_scale, int ntok,
                      k3c_stream_t stream);

/* One expert FFN for ntok tokens: y[t] = down(act(gate x[t], up x[t])), x fp32
 * [ntok][hidden], y fp32 [ntok][hidden]; e holds device addresses. scratch: device bytes,
 * at least k3c_expert_ffn_scratch(ntok, hidden, inter). */
size_t k3c_expert_ffn_scratch(int ntok, int hidden, int inter);
int k3c_expert_ffn(float *y, const float *x, int ntok, const K3ExpertQ *e, int hidden,
                   int inter, int act, void *scratch, size_t scratch_bytes,
                   k3c_stream_t stream);

/* A non-latent MoE layer (router + routed experts + unweighted shared expert).
 * `experts` is a DEVICE array [n_experts] of K3ExpertQ holding device addresses; an
 * entry whose p1 is NULL is not resident and is counted as a drop if selected.
 * `shared` is a DEVICE pointer to one K3ExpertQ, or NULL. */
typedef struct {
    int hidden, inter, n_experts, topk, renorm, act;
    float routed_scale;
    const void *router_w;       /* [n_experts][hidden], router_dtype */
    int router_dtype;           /* K3C_F32 or K3C_BF16 */
    const float *router_bias;   /* [n_experts] or NULL */
    const K3ExpertQ *experts;   /* device array [n_experts] */
    const K3ExpertQ *shared;    /* device pointer or NULL */
} k3c_moe_layer;

/* Scratch (device bytes) k3c_moe_decode needs for ntok tokens. */
size_t k3c_moe_decode_scratch(const k3c_moe_layer *L, int ntok);
/* out[ntok][hidden] fp32 = MoE(x); x [ntok][hidden] of x_dtype. idx/wt (device, may be
 * NULL) receive the routing [ntok][topk]. drops (device int, may be NULL) is incremented
 * by the number of selected experts that were not resident. */
int k3c_moe_decode(float *out, const void *x, int x_dtype, int ntok, const k3c_moe_layer *L,
                   int *idx, float *wt, int *drops, void *scratch, size_t scratch_bytes,
                   k3c_stream_t stream);

/* No counterpart in the reference. k3c_moe_decode without caller scratch, for callers that
 * cannot allocate device memory: an engine that owns all device memory and gives this
 * library no allocator, or a decode loop whose host code must not call cudaMalloc. The
 * scratch is a fixed device array inside the library, K3C_NOALLOC_SCRATCH_BYTES (8 MiB)
 * per GPU that loads it, held until the process exits; that covers the BASELINE decode
 * batch (hidden 7168, inter 2048, top-8 + shared, 16 tokens: ~5.8 MB). A call whose
 * k3c_moe_decode_scratch(L, ntok) exceeds the maximum returns K3C_EINVAL without touching
 * the GPU. The call itself allocates nothing; inputs and outputs are the caller's. The
 * first call on each device looks up the array's device address (cudaGetSymbolAddress)
 * with that device current: make that first call before any stream capture begins. All
 * calls on a device share the array and leave the last call's contents in it (none is read
 * before being written), so calls whose kernels overlap on the GPU race. */
#define K3C_NOALLOC_SCRATCH_BYTES (8u << 20)
int k3c_moe_decode_noalloc(float *out, const void *x, int x_dtype, int ntok,
                           const k3c_moe_layer *L, int *idx, float *wt, int *drops,
                           k3c_stream_t stream);

/* ------------------------------------------------------------------------------------
 * Tensor-core path (tcgen05 block-scaled MMA, kind::mxf8f6f4).
 *
 * Experts live in an HBM arena of "pool-format" runs (no reference counterpart; the
 * reference's cache holds the checkpoint's byte run, src/cache/k3_cache.c:24-261): the same
 * bytes as the checkpoint's w1/w2/w3 packed nibbles and E8M0 scales, re-ordered so the
 * tensor core can read them -- gate and up rows interleaved in blocks of 64 and the scales
 * in 512-byte 128-row x 4-group atoms. k3c_pool_pack_expert converts one expert given in the
 * reference layout (device addresses) into a run of k3c_pool_run_bytes bytes (256-byte
 * aligned). hidden and inter must be multiples of 128.
 * ------------------------------------------------------------------------------------ */
size_t k3c_pool_run_bytes(int hidden, int inter);
int k3c_pool_pack_expert(uint8_t *run, const K3ExpertQ *src, int hidden, int inter,
                         k3c_stream_t stream);

typedef struct {
    int hidden, inter, n_experts, topk, renorm, act;
    float routed_scale;
    const void *router_w;       /* [n_experts][hidden], router_dtype */
    int router_dtype;
    const float *router_bias;   /* [n_experts] or NULL */
    const uint8_t *arena;       /* device: n_runs pool-format runs, run_stride bytes apart */
    size_t run_stride;          /* multiple of 256, >= k3c_pool_run_bytes */
    int n_runs;
    const int *run_of;          /* device [n_experts]: run index, -1 = not resident (drop) */
    int shared_run;             /* run index of the shared expert, -1 = none */
    int terms;                  /* E4M3 terms per activation (1..3): ~4 bits each */
} k3c_moe_pool_layer;

/* Same contract as k3c_moe_decode (non-latent MoE layer, drops counted), computed with
 * tcgen05 block-scaled MMAs on pool-format experts; ntok <= 32. */
size_t k3c_moe_decode_tc_scratch(const k3c_moe_pool_layer *L, int ntok);
int k3c_moe_decode_tc(float *out, const void *x, int x_dtype, int ntok,
                      const k3c_moe_pool_layer *L, int *idx, float *wt, int *drops,
                      void *scratch, size_t scratch_bytes, k3c_stream_t stream);

/* Same as k3c_moe_decode_tc with the routing given: idx/wt [ntok][topk] on the device (top-k
 * expert ids and their weights, as k3c_router writes them); the router is not run. Used when
 * routing comes from elsewhere (the streamed-expert stack, replays of recorded routing). */
int k3c_moe_decode_tc_routed(float *out, const void *x, int x_dtype, int ntok,
                             const k3c_moe_pool_layer *L, const int *idx, const float *wt,
                             int *drops, void *scratch, size_t scratch_bytes, k3c_stream_t stream);

/* ------------------------------------------------------------------------------------
 * Routed experts from the checkpoint's safetensors shards (src/io/k3_st.h, src/io/k3_load.h).
 * Host functions except k3c_expert_upload; none of them allocates device memory.
 * ------------------------------------------------------------------------------------ */
/* Tensor element types of a shard (the reference's K3Dtype values, src/io/k3_st.h:35). */
enum { K3C_DT_U8 = 1, K3C_DT_BF16 = 2, K3C_DT_F16 = 3, K3C_DT_F32 = 4,
       /* K3_DT_I8R: the draft trunk's per-row int8 rows [f32 scale][int8 * cols]; only in a
        * packed trunk (below), never in a safetensors shard */
       K3C_DT_I8R = 5 };
typedef struct {
    int shard, dtype, ndim;
    int64_t off;          /* absolute byte offset in its shard file */
    int64_t nbytes;
    int64_t shape[4];
} k3c_tensor;
typedef struct k3c_ckpt k3c_ckpt;   /* the indexed shards of one checkpoint directory */
/* k3_st_open / k3_st_close (src/io/k3_st.h:70-71): index every *.safetensors file of dir
 * (shard i is the i-th name in sorted order). NULL on failure, k3c_last_error() says why:
 * an impossible header length, a tensor whose byte span is not its shape's, a span past the
 * end of the file, an unsupported dtype (U8, BF16, F16, F32 are read), a name twice. */
k3c_ckpt *k3c_ckpt_open(const char *dir);
void k3c_ckpt_close(k3c_ckpt *c);
/* A packed trunk directory (src/io/k3_trunk.c:98-200; written by the reference's
 * tools/pack_trunk.py, and as the draft model's int8 trunk by tools/int8_trunk.py): trunk.json
 * lists per layer its run's file_off / nbytes in trunk.bin and its tensors (off within the run,
 * nbytes, dtype, shape); dtypes BF16, F32, U8, F16 and I8R. k3c_trunk_open refuses a manifest
 * whose tensor spans leave their run or the file, whose I8R tensor is not rows * (4 + cols)
 * bytes for its shape [rows, cols], or whose other tensors' spans are not their shape's bytes.
 * k3c_trunk_find: tensor `name` of `layer` with off made absolute in trunk.bin (shard 0).
 * k3c_trunk_read: that tensor's bytes (one O_DIRECT read widened to 4096-byte boundaries when
 * buf is page aligned and the manifest's align is 4096, as k3_trunk_open decides; a buffered
 * read otherwise); the payload starts at buf + *payload_off. An I8R tensor feeds the draft
 * model's K3C_WI8 trunk: copy its rows to the device and k3c_q8_pack them (in = cols,
 * out = rows) into the k3c_q8_mat of a k3c_moe_latent_layer. */
typedef struct k3c_trunk k3c_trunk;
k3c_trunk *k3c_trunk_open(const char *dir);
void k3c_trunk_close(k3c_trunk *tr);
int k3c_trunk_layers(const k3c_trunk *tr);
int k3c_trunk_find(const k3c_trunk *tr, int layer, const char *name, k3c_tensor *t);
int64_t k3c_trunk_read(const k3c_trunk *tr, const k3c_tensor *t, void *buf, int64_t bufcap,
                       int64_t *payload_off);
int k3c_ckpt_shards(const k3c_ckpt *c);
/* 1 when the shard could be opened for O_DIRECT reads (expert reads then bypass the page
 * cache); 0 when reads fall back to the buffered descriptor. */
int k3c_ckpt_direct(const k3c_ckpt *c, int shard);
/* k3_st_find (src/io/k3_st.h:76): K3C_ENOTFOUND when absent. */
int k3c_ckpt_find(const k3c_ckpt *c, const char *name, k3c_tensor *t);

/* K3QMat / K3ExpertRef (src/io/k3_load.h:29-45), same fields in the same order. */
typedef struct {
    int64_t p_off, p_bytes;   /* packed nibbles, offset within the run */
    int64_t s_off, s_bytes;   /* E8M0 scales, offset within the run */
    int rows, pcols, scols;
} k3c_qmat;
typedef struct {
    int layer, expert, shard;
    int64_t off, nbytes;      /* run start in the shard, run bytes */
    int contiguous;           /* 1: the six tensors tile one span, read with one call */
    k3c_qmat m[3];            /* w1, w2, w3 */
} k3c_expert_run;
/* k3_expert_ref (src/io/k3_load.c:15-105): resolve the six tensors of
 * "language_model.model.layers.L.block_sparse_moe.experts.E.{w1,w2,w3}.{weight_packed,
 * weight_scale}" and check them: U8, 2-D, equal row counts, one scale per 32 elements, one
 * shard. A contiguous run keeps the file's offsets; otherwise the run is assembled in the
 * order w1.packed w1.scale w2.packed w2.scale w3.packed w3.scale. */
int k3c_expert_ref(const k3c_ckpt *c, int layer, int expert, k3c_expert_run *r);
/* k3_expert_load_direct (src/io/k3_load.c:137-145): a contiguous run is one O_DIRECT read
 * widened to 4096-byte boundaries, so buf must be page aligned and hold nbytes + 8192; the run
 * then starts at buf + *payload_off (0, by a buffered read, when the shard has no O_DIRECT
 * descriptor or buf is not page aligned). Scattered
 * tensors are six buffered reads into the canonical order at buf. Returns payload bytes. */
int64_t k3c_expert_read(const k3c_ckpt *c, const k3c_expert_run *r, void *buf, int64_t bufcap,
                        int64_t *payload_off);
/* Copy a run read by k3c_expert_read (payload = buf + payload_off; pinned memory makes the
 * copy asynchronous) into dev_staging (r->nbytes device bytes) and pack it into the
 * pool-format device run dev_run (k3c_pool_pack_expert): one routed expert from the
 * checkpoint into an HBM pool slot or arena run. The tensors' offsets within the run must be
 * multiples of 16 bytes, as they are for every K3 shape. */
int k3c_expert_upload(uint8_t *dev_run, const k3c_expert_run *r, const void *payload,
                      uint8_t *dev_staging, k3c_stream_t stream);

/* ------------------------------------------------------------------------------------
 * The K3 latent MoE layer (src/core/k3_ops.c:556-656) and its trunk operations.
 * ------------------------------------------------------------------------------------ */

/* Device form of k3_mmw (include/k3/k3.h:289-296) for ntok <= 32 tokens:
 * y[t*ldy + o] = sum_i W[o][i] x[t*ldx + i] (accumulate != 0: y += that, one float add),
 * W [out][in] of type wdt (K3C_WF32 or K3C_WBF16), fp32 x. Bit-exact with k3_matmul /
 * k3_matmul_bf16 token by token. Int8 trunk rows run through k3c_q8_pack / k3c_q8_gemv. */
int k3c_mmw(float *y, int ldy, const float *x, int ldx, int ntok, const void *W, int wdt,
            int in, int out, int accumulate, k3c_stream_t stream);
/* The same product for many tokens on the tensor cores (tcgen05 kind::f16), bf16 W only: x
 * enters as two bf16 terms (hi = bf16(x), lo = bf16(x - hi)), products accumulate in fp32.
 * Not bit-exact with k3_matmul_bf16 (k3c_mmw is); error ~1e-6 of max|y|. in a multiple of 8,
 * W 16-byte aligned; any ntok and out. scratch: k3c_mmw_tc_scratch(ntok, in) bytes of device
 * memory for the activation terms. The latent layer takes this path for more than 32 tokens
 * with a bf16 trunk (K3C_TRUNK_EXACT=1 keeps it on k3c_mmw). */
size_t k3c_mmw_tc_scratch(int ntok, int in);
int k3c_mmw_tc(float *y, int ldy, const float *x, int ldx, int ntok, const void *W, int in, int out,
               int accumulate, void *scratch, size_t scratch_bytes, k3c_stream_t stream);
/* k3_situ_glu (src/core/k3_ops.c:110-122) on ntok rows: gu [ntok][2n] (gate | up),
 * y [ntok][n]. */
int k3c_situ_glu(float *y, const float *gu, int n, int ntok, float b1, float b2,
                 k3c_stream_t stream);
/* k3_rmsnorm (src/core/k3_ops.c:94-102) on ntok rows of n: y may alias x. */
int k3c_rmsnorm(float *y, const float *x, const float *w, int n, int ntok, float eps,
                k3c_stream_t stream);

/* One latent MoE layer (the K3MoeW / K3Cfg fields of include/k3/k3.h:94-113, 357-380).
 * Routing runs on the full-width input with router_w; the routed experts are pool-format
 * runs at the latent width, described by `experts` (experts.hidden = latent,
 * experts.inter = moe_inter; its n_experts, topk, renorm, routed_scale, act and terms apply;
 * its router fields are not used; shared_run must be -1). The trunk matrices have type
 * wdt: down [latent][hidden], up [hidden][latent], sh1/sh3 [inter*n_shared][hidden],
 * sh2 [hidden][inter*n_shared]; device addresses for K3C_WF32 / K3C_WBF16 (matmuls in the
 * reference's order, bit-exact), and for K3C_WI8 (the draft model) each is the address of a
 * host k3c_q8_mat (the int8 tensor-core GEMV, exact int32 sums, one scale per row). */
typedef struct {
    int hidden;
    k3c_moe_pool_layer experts;
    const float *router_w;        /* [experts.n_experts][hidden] fp32 */
    const float *router_bias;     /* [experts.n_experts] or NULL */
    const void *down, *up;
    const void *sh1, *sh3, *sh2;
    const float *latent_norm;     /* [latent] (used when latent_norm_on) */
    int wdt, n_shared, latent_norm_on;
    float rms_eps, situ_b1, situ_b2;
    /* The draft model's K3MoeW.cache_only (src/core/k3_ops.c:580-593): route among the experts
     * with a run in experts.run_of only (k3c_route_cache_only after the router) and count no
     * drops. experts.run_of must then hold only runs that are pinned and filled on the stream
     * (k3c_pool_acquire_resident). */
    int cache_only;
} k3c_moe_latent_layer;

/* k3_moe (src/core/k3_ops.c:556-656) for ntok <= 65535 tokens: out [ntok][hidden] fp32 from
 * x [ntok][hidden] fp32. Per token: route on x; z = down x; the top-k experts on z at the
 * latent width, summed with their weights in top-k order; RMSNorm of the sum; out = up sum;
 * plus the shared expert sh2(SiTU(sh1 x, sh3 x)) unweighted. Up to 32 tokens the experts run
 * on the tensor-core decode kernels (the activation as experts.terms E4M3 terms); more tokens
 * run them on the prefill kernels (two E4M3 terms; the latent width must then be a multiple of
 * 256) and the trunk matrices 32 tokens at a time. idx/wt (device, may be NULL) receive the
 * routing [ntok][topk]; drops counts selected experts without a resident run. */
size_t k3c_moe_latent_scratch(const k3c_moe_latent_layer *L, int ntok);
int k3c_moe_latent_decode(float *out, const float *x, int ntok, const k3c_moe_latent_layer *L,
                          int *idx, float *wt, int *drops, void *scratch, size_t scratch_bytes,
                          k3c_stream_t stream);
/* The same layer with the routing given: idx/wt [ntok][topk] on the device are used as they are
 * (the router and L->cache_only are not applied; entries < 0 or without a run are skipped and
 * counted in drops when it is not NULL). The k3_moe drop-in runs this after the expert source
 * has been asked for every selected expert. */
int k3c_moe_latent_decode_routed(float *out, const float *x, int ntok, const k3c_moe_latent_layer *L,
                                 const int *idx, const float *wt, int *drops, void *scratch,
                                 size_t scratch_bytes, k3c_stream_t stream);

/* MoE prefill over ntok tokens: the reference's k3_moe_prefill / moe_prefill_chunk
 * (src/core/k3_ops.c:689-808) for the non-latent shape -- route, group the (token, expert)
 * pairs by expert, run each expert's FFN over its group as tcgen05 block-scaled MMAs, combine
 * in each token's top-k order (k3_ops.c:641-642) plus the shared expert. Activations enter
 * the MMAs as two E4M3 terms per element (the layer's `terms` field is not used). Same
 * outputs, drop counting and error behaviour as k3c_moe_decode_tc; hidden must be a multiple
 * of 256, inter of 128, x 16-byte aligned, ntok <= 65535. */
size_t k3c_moe_prefill_tc_scratch(const k3c_moe_pool_layer *L, int ntok);
/* Prefill with the routing given (idx/wt [ntok][topk] on the device); ids that are negative
 * or not resident are skipped (counted in drops if drops is not NULL). With shared_run < 0
 * the output is the routed experts' weighted sum only. Expert parallelism runs each GPU's
 * received tokens through this with the experts of other GPUs marked -1. */
int k3c_moe_prefill_tc_routed(float *out, const void *x, int x_dtype, int ntok,
                              const k3c_moe_pool_layer *L, const int *idx, const float *wt,
                              int *drops, void *scratch, size_t scratch_bytes, k3c_stream_t stream);
int k3c_moe_prefill_tc(float *out, const void *x, int x_dtype, int ntok,
                       const k3c_moe_pool_layer *L, int *idx, float *wt, int *drops,
                       void *scratch, size_t scratch_bytes, k3c_stream_t stream);

/* The combine alone (k3_ops.c:641-642): out[t] = sum_j wt[t][j] * contrib[t][j] in top-k order,
 * plus contrib[t][topk] when has_shared; contrib [ntok][topk+1][hidden] fp32. Pairs whose id
 * (idx, may be NULL) lies outside [0, n_experts) are skipped. */
int k3c_moe_combine(float *out, const float *contrib, const float *wt, const int *idx, int n_experts,
                    int ntok, int topk, int hidden, int has_shared, k3c_stream_t stream);

/* ---- Expert-parallel prefill over peer memory (no reference counterpart: the reference is
 * a single-process CPU engine). The ranks of one node each own a set of routed experts (the
 * layer's run table marks the others -1) and their own tokens. Per layer, with a cross-rank
 * barrier (a one-element NCCL all-reduce on the stream) between the steps:
 *   1. each rank writes its tokens' bf16 or fp32 activations into its x buffer and their
 *      top-k ids and weights into its idx and wt buffers (k3c_router_ws);  -- barrier
 *   2. k3c_moe_prefill_ep_experts on every rank: plans over all ranks' pairs (reading the
 *      peers' idx), quantises the tokens it needs straight out of the peers' x buffers
 *      (loads over NVLink), runs its own experts over them and its own tokens' shared expert;
 *      the down-projection epilogue stores each pair's output as a bf16 row at [t][k] of the
 *      token owner's receive buffer (stores over NVLink, overlapping the MMAs of the next
 *      tiles; the shared expert's row at [t][topk]);                          -- barrier
 *   3. k3c_moe_ep_combine on every rank: its tokens' rows added in top-k order with its own
 *      weights, then the shared row -- the single-GPU combine, so the result equals
 *      k3c_moe_prefill_tc of the same layer bit for bit. A pair whose expert no rank holds
 *      (expert_rank[e] < 0) is skipped.
 * Buffers are exchanged once per process: k3c_ep_alloc gives device memory and its IPC
 * handle, k3c_ep_open maps a peer's handle (same node). The receive buffer holds
 * [t_max][topk+1][hidden] bf16 (2 bytes each). ---- */
#define K3C_EP_MAX 8
typedef struct {
    unsigned char bytes[64];
} k3c_ipc_handle;
int k3c_ep_alloc(void **ptr, size_t bytes, k3c_ipc_handle *handle);
int k3c_ep_free(void *ptr);
int k3c_ep_open(void **ptr, const k3c_ipc_handle *handle);
int k3c_ep_close(void *peer_ptr);

typedef struct {
    int world, rank;              /* ranks sharing the layer, this process's rank */
    int t_max;                    /* token rows of every rank's buffers */
    int x_dtype;                  /* K3C_BF16 or K3C_F32 */
    int ntok[K3C_EP_MAX];         /* each rank's token count (<= t_max) */
    const void *x[K3C_EP_MAX];    /* each rank's activations [t_max][hidden] */
    const int *idx[K3C_EP_MAX];   /* each rank's top-k ids [t_max][topk] */
    const float *wt[K3C_EP_MAX];  /* each rank's top-k weights [t_max][topk] */
    uint16_t *recv[K3C_EP_MAX];   /* each rank's pair rows [t_max][topk+1][hidden], bf16 */
    /* Device [n_experts] or NULL. 1: every rank holds the expert (a hot expert replicated to
     * spread its load) and each rank runs only its own tokens' pairs of it, so those pair rows
     * never cross NVLink; 0: the pairs of all ranks' tokens run wherever the expert is
     * resident. */
    const unsigned char *local_only;
    /* A cudaEvent_t or NULL: when the x[q] of other ranks are filled by a copy still in flight
     * on another stream (an all-gather of the token rows), the event recorded after it; step 2
     * plans first and makes the stream wait for it only before it reads those rows. */
    void *x_ready;
} k3c_ep_peers;
size_t k3c_moe_prefill_ep_scratch(const k3c_moe_pool_layer *L, const k3c_ep_peers *peers);
int k3c_moe_prefill_ep_experts(const k3c_moe_pool_layer *L, const k3c_ep_peers *peers,
                               void *scratch, size_t scratch_bytes, k3c_stream_t stream);
/* Step 3: out [ntok of this rank][hidden] fp32; expert_rank (device, n_experts ints): the rank
 * holding each expert, -1 for none; has_shared: the layer has a shared expert. */
int k3c_moe_ep_combine(float *out, const k3c_ep_peers *peers, int hidden, int topk,
                       const int *expert_rank, int n_experts, int has_shared, k3c_stream_t stream);

/* ---- HBM expert pool: the reference's expert cache (src/cache/k3_cache.c:24-261) with
 * experts streamed from pinned host memory. A slot holds one pool-format run
 * (k3c_pool_run_bytes). Keys are layer*n_experts + expert; victim choice, hit/miss/eviction
 * and batch-prefetch accounting follow the reference (pick_victim k3_cache.c:46-57, getmany
 * :131-234, report :416-425). Not thread-safe across pools' shared streams (one pool per
 * caller, as the reference). ---- */
enum { K3C_SLOT_EMPTY = -1, K3C_SLOT_INFLIGHT = -2 };
/* Where the host bytes of (layer, expert) live: a pool-format run in pinned host memory, or
 * NULL if there are none (the request then fails with K3C_ENOTFOUND). */
typedef const void *(*k3c_pool_src_fn)(void *ctx, int layer, int expert);
typedef struct {
    long long hits, misses, evictions, prefetch_reads, bytes_h2d;
} k3c_pool_stats_t;
typedef struct k3c_expert_pool k3c_expert_pool;

/* Allocates n_slots slots in HBM and the pool's copy stream; NULL on failure
 * (k3c_last_error says why). */
k3c_expert_pool *k3c_pool_create(int hidden, int inter, int n_layers, int n_experts, int n_slots,
                                 k3c_pool_src_fn src, void *ctx);
void k3c_pool_destroy(k3c_expert_pool *pool);
uint8_t *k3c_pool_arena(k3c_expert_pool *pool);            /* slot s at arena + s*stride */
size_t k3c_pool_slot_stride(const k3c_expert_pool *pool);
int k3c_pool_slots(const k3c_expert_pool *pool);
/* The expert shape the pool's runs hold (hidden = the experts' input width). */
int k3c_pool_shape(const k3c_expert_pool *pool, int *hidden, int *inter);
/* Slot holding (layer, expert) -- possibly still filling -- or -1. A query only: it pins
 * nothing and orders nothing, so a kernel must not read the slot on its word; use
 * k3c_pool_acquire_resident (or a k3c_pool_source's resident()) for that. */
int k3c_pool_resident(k3c_expert_pool *pool, int layer, int expert);
/* The draft model's resident set (reference: K3ExpertSrc.resident, src/cache/k3_cache.c:239-250,
 * used by k3_moe's cache-only routing, src/core/k3_ops.c:580-593): every expert of `layer`
 * that has a slot, pinned until k3c_pool_release, with `stream` made to wait for any of their
 * copies still in flight (no new copy is issued and no hit or miss is counted). ids (host, may
 * be NULL, cap entries) receives the pinned expert ids -- pass them to k3c_pool_release;
 * dev_run_of (device, n_experts ints, may be NULL) receives run_of[e] = slot for those and -1
 * elsewhere, ordered on `stream`: the run table for k3c_route_cache_only and the routed entry
 * points. Returns the count (>= 0; K3C_EFULL if it exceeds cap, nothing pinned) or a status. */
int k3c_pool_acquire_resident(k3c_expert_pool *pool, int layer, int *ids, int cap, int *dev_run_of,
                              k3c_stream_t stream);
/* Batch hint (reference: getmany): start the copies of the ids not resident; returns how
 * many were started. Counted as prefetch reads, not as hits or misses. */
int k3c_pool_getmany(k3c_expert_pool *pool, int layer, const int *ids, int n);
/* get() for each id (hits and misses counted per request): copies the misses, pins every
 * slot until k3c_pool_release, and makes `stream` wait for any copy still in flight.
 * slots (host, may be NULL) receives the slot of each id; dev_run_of (device, may be NULL,
 * n_experts ints) receives -1 everywhere except run_of[ids[i]] = slot, ordered on `stream`:
 * the run table of k3c_moe_pool_layer. */
int k3c_pool_acquire(k3c_expert_pool *pool, int layer, const int *ids, int n, int *slots,
                     int *dev_run_of, k3c_stream_t stream);
/* Unpins; the slots may be overwritten once the work enqueued on `stream` so far is done. */
int k3c_pool_release(k3c_expert_pool *pool, int layer, const int *ids, int n, k3c_stream_t stream);
/* Acquire that is never released (shared experts); returns the slot or a negative status. */
int k3c_pool_pin(k3c_expert_pool *pool, int layer, int expert, k3c_stream_t stream);
int k3c_pool_stats(k3c_expert_pool *pool, k3c_pool_stats_t *out);
int k3c_pool_sync(k3c_expert_pool *pool);                  /* waits for the copy stream */
/* The reference cache's bookkeeping around the counters (src/cache/k3_cache.c:235-261, 355-455):
 * every get request (k3c_pool_acquire, a pool source's get) appends (layer, expert) to an
 * access trace of int32 pairs and counts it in a per-key request histogram, both recording
 * what was asked for, hit or miss.
 *   k3c_pool_trace: copies up to cap int32 values (pairs) of the trace into out (may be NULL)
 *     and returns the trace's length in int32 values;
 *   k3c_pool_hist: copies the histogram [n_layers * n_experts] (uint32) into out;
 *   k3c_pool_dump_trace: the trace as a flat binary file of int32 pairs, the format
 *     k3_cache_dump_trace writes and tools/sim_cache.py replays (-1 if there is none);
 *   k3c_pool_dump_hist: the histogram as JSON {"n_layers","n_experts","counts":{"L,e":n}},
 *     nonzero entries only, as k3_cache_dump_hist;
 *   k3c_pool_set_pin: k3_cache_pin -- pin (1) or unpin (0) the slot of a resident expert so
 *     eviction skips it (the payoff of the histogram); 0 if the expert is not resident;
 *   k3c_pool_reset_stats: k3_cache_reset_stats (hits, misses, evictions, bytes and
 *     prefetch reads together);
 *   k3c_pool_report: k3_cache_report's summary on stdout, host bytes in place of disk. */
int64_t k3c_pool_trace(k3c_expert_pool *pool, int32_t *out, int64_t cap);
int k3c_pool_hist(k3c_expert_pool *pool, uint32_t *out);
int k3c_pool_dump_trace(k3c_expert_pool *pool, const char *path);
int k3c_pool_dump_hist(k3c_expert_pool *pool, const char *path);
int k3c_pool_set_pin(k3c_expert_pool *pool, int layer, int expert, int pin);
void k3c_pool_reset_stats(k3c_expert_pool *pool);
void k3c_pool_report(k3c_expert_pool *pool, const char *label);

/* ---- The pool as the reference's K3ExpertSrc (include/k3/k3.h:332-355), for the k3_moe /
 * k3_moe_prefill drop-ins and any caller of the reference's interface.
 *   get(layer, e, q)      = k3c_pool_acquire of one expert (hit/miss counted, trace, copy on a
 *                           miss): pins its slot and makes the source's stream wait for the
 *                           copy; q receives DEVICE addresses into the slot's pool-format run:
 *                           p1/s1 = the interleaved gate/up matrix and its scale atoms, p2/s2 =
 *                           down and its atoms, p3 = s3 = NULL (up lives inside p1). 0 or -1.
 *   getmany(layer, ids, n)= k3c_pool_getmany (prefetch copies; returns the count started).
 *   resident(layer, e, q) = 1 if e has a slot; with q non-NULL the slot is also pinned and the
 *                           stream made to wait for its copy, as get() but without counting.
 * Pins taken by get/resident hold until k3c_pool_source_release, which orders the slots'
 * reuse after the work enqueued on the source's stream so far -- the reference's "valid until
 * the caller finishes the token" made explicit for asynchronous consumers. A kernel reading
 * the slots must run on k3c_pool_source_stream. Not thread-safe (as the reference's cache). */
K3ExpertSrc *k3c_pool_source_create(k3c_expert_pool *pool, k3c_stream_t stream);
void k3c_pool_source_destroy(K3ExpertSrc *src);     /* releases its pins first */
int k3c_pool_source_release(K3ExpertSrc *src);
k3c_stream_t k3c_pool_source_stream(const K3ExpertSrc *src);
k3c_expert_pool *k3c_pool_source_pool(const K3ExpertSrc *src);   /* NULL: not a pool source */
/* Slot of a q that this source's get/resident returned, or -1. */
int k3c_pool_source_slot(const K3ExpertSrc *src, const K3ExpertQ *q);

#ifdef __cplusplus
}
#endif

#endif /* K3C_H */
