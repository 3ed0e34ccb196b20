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
 *     (src/core/k3_ops.c:556-656) without the latent down/up/norm steps.
 *
 * bench.py times refh_moe_layer as the reference arm (cpu_baseline kind "reference").
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "k3.h"

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

/* Thread count the reference's OpenMP loops will use, for the cpu_baseline record. */
#ifdef _OPENMP
#include <omp.h>
int refh_threads(void) { return omp_get_max_threads(); }
#else
int refh_threads(void) { return 1; }
#endif
