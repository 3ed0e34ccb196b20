/* ref_harness.c -- composes the reference's OWN kernels into the BASELINE workloads.
 *
 * TEST AND BASELINE INFRASTRUCTURE ONLY. oracle/Makefile compiles this file together with
 * the reference's sources (src/core/k3_ops.c and, for the cache oracle, src/cache/k3_cache.c,
 * src/io/k3_load.c, src/io/k3_st.c), taken where they lie in the reference tree, into
 * oracle/_ref/libk3ref.so. Nothing here re-implements a reference kernel: every matmul and
 * the router are the reference's own k3_matmul_mxfp4, k3_matmul_q8 and k3_router. Only the
 * glue the reference does not ship is written here:
 *   - SwiGLU, which the reference does not have (the BASELINE configs use it), written as
 *     (g*sigmoid(g))*u with the reference's sigmoid (src/core/k3_ops.c:105);
 *   - the non-latent layer composition of the BASELINE configs, i.e. k3_moe
 *     (src/core/k3_ops.c:556-656) without the latent down/up/norm steps;
 *   - for the latent layer, only the K3Cfg/K3MoeW set-up and an in-memory expert source
 *     around the reference's own k3_moe.
 *
 * bench.py times refh_moe_layer as the reference arm (cpu_baseline kind "reference").
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "k3.h"
#include "k3_cache.h"
#include "k3_load.h"

static float refh_sigmoid(float v) { return 1.0f / (1.0f + expf(-v)); }

/* One expert for one token through the reference's k3_matmul_mxfp4: the
 * src/core/k3_ops.c:628-631 sequence with SwiGLU (act=0) or the reference's SiTU (act=1).
 * scratch holds 3*inter floats. */
static void refh_ffn1(float *y, const float *x, const K3ExpertQ *q, int hidden, int inter,
                      int act, float *scratch)
{
    float *gu = scratch, *a = scratch + 2 * inter;
    k3_matmul_mxfp4(gu, x, q->p1, q->s1, hidden, inter, K3_MXFP4_GROUP);
    k3_matmul_mxfp4(gu + inter, x, q->p3, q->s3, hidden, inter, K3_MXFP4_GROUP);
    if (act == 1) {
        k3_situ_glu(a, gu, inter, 4.0f, 25.0f);
    } else {
        for (int i = 0; i < inter; i++) {
            const float g = gu[i];
            a[i] = (g * refh_sigmoid(g)) * gu[inter + i];
        }
    }
    k3_matmul_mxfp4(y, a, q->p2, q->s2, inter, hidden, K3_MXFP4_GROUP);
}

/* BASELINE config[0]: one expert FFN for ntok tokens. */
int refh_expert_ffn(float *y, const float *x, int ntok, const K3ExpertQ *q, int hidden,
                    int inter, int act)
{
    float *s = (float *)malloc((size_t)3 * inter * sizeof(float));
    if (!s) return -1;
    for (int t = 0; t < ntok; t++)
        refh_ffn1(y + (size_t)t * hidden, x + (size_t)t * hidden, q, hidden, inter, act, s);
    free(s);
    return 0;
}

/* BASELINE config[1]/[2]: a non-latent MoE layer over ntok tokens with the reference's
 * k3_router, k3_matmul_mxfp4 experts, the float top-k-order combine of
 * src/core/k3_ops.c:599,641-642 and the unweighted shared expert of :650-654.
 * experts[] is indexed by expert id; router_w is fp32 [n_experts][hidden]. */
int refh_moe_layer(float *out, const float *x, int ntok, const float *router_w,
                   const float *router_bias, const K3ExpertQ *experts,
                   const K3ExpertQ *shared, int hidden, int inter, int n_experts, int topk,
                   int renorm, float routed_scale, int act, int *idx_out, float *wt_out)
{
    int *idx = (int *)malloc((size_t)topk * sizeof(int));
    float *wt = (float *)malloc((size_t)topk * sizeof(float));
    float *edn = (float *)malloc((size_t)hidden * sizeof(float));
    float *s = (float *)malloc((size_t)3 * inter * sizeof(float));
    if (!idx || !wt || !edn || !s) { free(idx); free(wt); free(edn); free(s); return -1; }
    for (int t = 0; t < ntok; t++) {
        const float *xt = x + (size_t)t * hidden;
        float *ot = out + (size_t)t * hidden;
        k3_router(idx, wt, xt, router_w, router_bias, hidden, n_experts, topk, renorm,
                  routed_scale);
        for (int i = 0; i < hidden; i++) ot[i] = 0.0f;
        for (int j = 0; j < topk; j++) {
            refh_ffn1(edn, xt, &experts[idx[j]], hidden, inter, act, s);
            const float wj = wt[j];
            for (int i = 0; i < hidden; i++) ot[i] += wj * edn[i];
        }
        if (shared) {
            refh_ffn1(edn, xt, shared, hidden, inter, act, s);
            for (int i = 0; i < hidden; i++) ot[i] += edn[i];
        }
        if (idx_out) memcpy(idx_out + (size_t)t * topk, idx, (size_t)topk * sizeof(int));
        if (wt_out) memcpy(wt_out + (size_t)t * topk, wt, (size_t)topk * sizeof(float));
    }
    free(idx); free(wt); free(edn); free(s);
    return 0;
}

/* An in-memory expert source for k3_moe: get() hands out experts[expert] (MXFP4). */
static int refh_src_get(struct K3ExpertSrc *self, int layer, int expert, K3ExpertQ *out)
{
    (void)layer;
    *out = ((const K3ExpertQ *)self->ctx)[expert];
    return 0;
}

/* The K3 latent MoE layer run by the reference's OWN k3_moe (src/core/k3_ops.c:556-656):
 * this function only fills a K3Cfg and a K3MoeW (zeroed first, as include/k3/k3.h:305-313
 * requires) and, for MXFP4 experts, an in-memory K3ExpertSrc. experts != NULL streams
 * MXFP4 experts through the source; otherwise the fp32 bank w1/w3/w2 is used. k3_moe runs
 * one token per call so that each token's routing can be returned. */
int refh_moe_latent(float *out, const float *x, int ntok, const float *router_w,
                    const float *router_bias, const K3ExpertQ *experts, const float *w1,
                    const float *w3, const float *w2, const float *latent_norm,
                    const void *down, const void *up, const void *sh1, const void *sh3,
                    const void *sh2, int wdt, int hidden, int latent, int inter, int n_shared,
                    int n_experts, int topk, int renorm, float routed_scale,
                    int latent_norm_on, float rms_eps, float situ_b1, float situ_b2,
                    int *idx_out, float *wt_out)
{
    K3Cfg c;
    memset(&c, 0, sizeof(c));
    c.hidden = hidden;
    c.rms_eps = rms_eps;
    c.n_experts = n_experts;
    c.topk = topk;
    c.n_shared = n_shared;
    c.latent = latent;
    c.moe_inter = inter;
    c.routed_scale = routed_scale;
    c.moe_renorm = renorm;
    c.latent_norm = latent_norm_on;
    c.situ_b1 = situ_b1;
    c.situ_b2 = situ_b2;
    K3ExpertSrc src;
    memset(&src, 0, sizeof(src));
    src.get = refh_src_get;
    src.ctx = (void *)experts;
    K3MoeW w;
    memset(&w, 0, sizeof(w));
    w.gate = router_w;
    w.bias = router_bias;
    w.w1 = w1;
    w.w3 = w3;
    w.w2 = w2;
    w.latent_norm = latent_norm;
    w.down = down;
    w.up = up;
    w.sh1 = sh1;
    w.sh3 = sh3;
    w.sh2 = sh2;
    w.wdt = wdt;
    w.src = experts ? &src : NULL;
    int *idx = (int *)malloc((size_t)topk * sizeof(int));
    float *wt = (float *)malloc((size_t)topk * sizeof(float));
    float *scratch = (float *)malloc(k3_moe_scratch(&c) * sizeof(float));
    if (!idx || !wt || !scratch) { free(idx); free(wt); free(scratch); return -1; }
    for (int t = 0; t < ntok; t++) {
        k3_moe(out + (size_t)t * hidden, x + (size_t)t * hidden, &w, &c, 1, idx, wt, scratch);
        if (idx_out) memcpy(idx_out + (size_t)t * topk, idx, (size_t)topk * sizeof(int));
        if (wt_out) memcpy(wt_out + (size_t)t * topk, wt, (size_t)topk * sizeof(float));
    }
    free(idx); free(wt); free(scratch);
    return 0;
}

/* The reference's own shard index and expert loader on a checkpoint directory: k3_st_open,
 * k3_expert_ref and k3_expert_load_direct (src/io/k3_st.c, src/io/k3_load.c). Returns the
 * payload bytes read, -1 when k3_st_open fails, -2 when k3_expert_ref rejects the expert. */
long long refh_expert_read(const char *dir, int layer, int expert, unsigned char *buf, long long cap,
                           K3ExpertRef *ref_out, long long *payload_off)
{
    K3St s;
    memset(&s, 0, sizeof s);
    if (k3_st_open(&s, dir) != 0) return -1;
    K3ExpertRef r;
    if (k3_expert_ref(&s, layer, expert, &r) != 0) { k3_st_close(&s); return -2; }
    if (ref_out) *ref_out = r;
    int64_t po = 0;
    const int64_t n = k3_expert_load_direct(&s, &r, buf, cap, &po);
    if (payload_off) *payload_off = po;
    k3_st_close(&s);
    return (long long)n;
}

/* The reference's own shard index: k3_st_open then k3_st_find for each of n names. For name
 * i, info[8*i .. 8*i+7] = found, shard, dtype, ndim, offset, nbytes, shape[0], shape[1].
 * Returns 0, or -1 when k3_st_open fails. */
int refh_st_find(const char *dir, const char *const *names, int n, long long *info)
{
    K3St s;
    memset(&s, 0, sizeof s);
    if (k3_st_open(&s, dir) != 0) return -1;
    for (int i = 0; i < n; i++) {
        long long *o = info + 8 * (size_t)i;
        const K3Tensor *t = k3_st_find(&s, names[i]);
        memset(o, 0, 8 * sizeof(long long));
        if (!t) continue;
        o[0] = 1; o[1] = t->shard; o[2] = t->dtype; o[3] = t->ndim; o[4] = t->off; o[5] = t->nbytes;
        o[6] = t->ndim > 0 ? t->shape[0] : 0; o[7] = t->ndim > 1 ? t->shape[1] : 0;
    }
    k3_st_close(&s);
    return 0;
}

/* Thread count the reference's OpenMP loops will use, for the cpu_baseline record.
 * refh_set_threads sets it for this process (a launcher such as torch.distributed.run exports
 * OMP_NUM_THREADS=1 to every rank; the baseline runs on rank 0 alone and may use the host). */
#ifdef _OPENMP
#include <omp.h>
int refh_threads(void) { return omp_get_max_threads(); }
void refh_set_threads(int n) { if (n > 0) omp_set_num_threads(n); }
#else
int refh_threads(void) { return 1; }
void refh_set_threads(int n) { (void)n; }
#endif

/* The reference's OWN k3_moe (prefill = 0) or k3_moe_prefill (prefill = 1) on caller-built
 * K3MoeW / K3Cfg (the test builds them through the mirrored layouts of include/k3c.h, which is
 * itself an ABI check) and the caller's expert source; scratch sized by k3_moe_scratch. Returns
 * the reference's k3_expert_drops counted during the call, or -1 on allocation failure. */
long refh_moe_call(int prefill, float *out, const float *x, int T, const K3MoeW *w, const K3Cfg *c,
                   int *idx, float *wt)
{
    float *scratch = (float *)malloc(k3_moe_scratch(c) * sizeof(float));
    if (!scratch) return -1;
    const long d0 = k3_expert_drops;
    if (prefill) k3_moe_prefill(out, x, w, c, T, idx, wt, scratch);
    else         k3_moe(out, x, w, c, T, idx, wt, scratch);
    free(scratch);
    return k3_expert_drops - d0;
}

/* The reference's OWN expert cache (src/cache/k3_cache.c) replaying a request sequence, for
 * pinning the bookkeeping restatement oracle/cache_model.py. The cache is built by
 * k3_cache_init over the checkpoint in dir with room for exactly nslot slots. ops is a flat
 * stream of records [kind, layer, n, ids[n]]: kind 0 = src.get of ids[0], 1 = src.getmany of
 * the n ids, 2 = k3_cache_pin(ids[0], 1), 3 = k3_cache_pin(ids[0], 0). After record i,
 * key_of[i*nslot .. +nslot) receives the cache's key_of table and rc[i] the call's return
 * value. stats = {hits, misses, evictions, prefetch_reads}; trace (cap trace_cap int32) and
 * hist (n_layers*n_experts) are the cache's own records; *ntrace their int32 count.
 * Returns the number of records replayed, or -1 (checkpoint), -2 (cache init), -3 (ops). */
int refh_cache_replay(const char *dir, const K3Cfg *cfg, int nslot, const int *ops, int n_ops, int n_rec,
                      int *key_of, int *rc, unsigned long long *stats, int *trace, long long trace_cap,
                      long long *ntrace, unsigned *hist)
{
    K3St st;
    memset(&st, 0, sizeof st);
    if (k3_st_open(&st, dir) != 0) return -1;
    K3ExpertRef probe;
    if (k3_expert_ref(&st, cfg->first_dense, 0, &probe) != 0) { k3_st_close(&st); return -1; }
    int64_t slot_bytes = probe.nbytes + 2 * K3_ST_ALIGN;          /* the init's own sizing rule */
    slot_bytes = (slot_bytes + K3_ST_ALIGN - 1) & ~(int64_t)(K3_ST_ALIGN - 1);
    K3Cache c;
    if (k3_cache_init(&c, &st, cfg, (int64_t)nslot * slot_bytes) != 0 || c.nslot != nslot) {
        k3_st_close(&st);
        return -2;
    }
    int pos = 0, i = 0;
    for (; i < n_rec && pos + 3 <= n_ops; i++) {
        const int kind = ops[pos], layer = ops[pos + 1], n = ops[pos + 2];
        const int *ids = ops + pos + 3;
        if (n < 1 || pos + 3 + n > n_ops) { i = -3; break; }
        K3ExpertQ q;
        if (kind == 0) rc[i] = c.src.get(&c.src, layer, ids[0], &q);
        else if (kind == 1) rc[i] = c.src.getmany ? c.src.getmany(&c.src, layer, ids, n) : -1;
        else rc[i] = k3_cache_pin(&c, layer, ids[0], kind == 2);
        memcpy(key_of + (size_t)i * nslot, c.key_of, (size_t)nslot * sizeof(int));
        pos += 3 + n;
    }
    stats[0] = c.hits;
    stats[1] = c.misses;
    stats[2] = c.evictions;
    stats[3] = c.prefetch_reads;
    *ntrace = c.ntrace;
    if (trace && c.trace) memcpy(trace, c.trace, (size_t)(c.ntrace < trace_cap ? c.ntrace : trace_cap) * 4);
    if (hist) memcpy(hist, c.hist, (size_t)c.n_layers * c.n_experts * sizeof(unsigned));
    k3_cache_free(&c);
    k3_st_close(&st);
    return i;
}
