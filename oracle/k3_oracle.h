/* k3_oracle.h -- CPU restatement of the reference's routed-expert hot path.
 *
 * TEST INFRASTRUCTURE ONLY. Nothing in the product library links or calls this code; it
 * exists so that the test-suite, __graft_entry__.smoke() and the cpu_baseline leg of
 * bench.py have an independent CPU answer to compare the CUDA path against.
 *
 * Every function cites the reference file:line whose algorithm it restates (paths are
 * relative to the jaylauffer/kimi-k3-in-rust tree). Parity of this restatement is pinned
 * two ways by tests/test_oracle.py:
 *   - against the reference's own golden vectors (tests/golden/, converted from
 *     tests/fixtures/mxfp4.json and tests/fixtures/ops/router.json), and
 *   - against the reference's own kernels compiled from its sources into
 *     oracle/_ref/libk3ref.so (see oracle/Makefile), when that library is present.
 */
#ifndef K3_ORACLE_H
#define K3_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* One expert as three (packed, scale) pairs, gate/up/down; the K3ExpertQ field order
 * (include/k3/k3.h:323-327). */
typedef struct {
    const unsigned char *p1, *s1;   /* gate [inter][hidden/2], [inter][hidden/32] */
    const unsigned char *p3, *s3;   /* up   [inter][hidden/2], [inter][hidden/32] */
    const unsigned char *p2, *s2;   /* down [hidden][inter/2], [hidden][inter/32] */
} ora_expert;

enum { ORA_ACT_SWIGLU = 0, ORA_ACT_SITU = 1 };

float ora_e2m1(unsigned code);
float ora_e8m0(unsigned char b);

void ora_mxfp4_dequant(float *out, const unsigned char *packed, const unsigned char *scales,
                       int rows, int pcols, int group);
void ora_matmul_mxfp4(float *y, const float *x, const unsigned char *packed,
                      const unsigned char *scales, int in, int rows, int group);
void ora_matmul_f32(float *y, const float *x, const float *W, int in, int out);
void ora_matmul_q8(float *y, const float *x, const void *W, int in, int out);
void ora_router(int *idx, float *w, const float *x, const float *W, const float *bias,
                int hidden, int n_experts, int topk, int renorm, float routed_scale);
void ora_router_select(int *idx, float *w, const float *score, const float *bias,
                       int n_experts, int topk, int renorm, float routed_scale);
void ora_router_scores(float *score, const float *x, const float *W, int hidden, int n_experts);
void ora_swiglu(float *y, const float *gu, int n);
void ora_situ_glu(float *y, const float *gu, int n, float b1, float b2);
void ora_rmsnorm(float *y, const float *x, const float *w, int n, float eps);

/* One expert FFN for ntok tokens: y[t] = down(act(gate x[t], up x[t])). */
void ora_expert_ffn(float *y, const float *x, int ntok, const ora_expert *e,
                    int hidden, int inter, int act);

/* One non-latent MoE layer (BASELINE config shape) for ntok tokens:
 *   route on x, run the top-k experts, sum weight*expert in top-k order, add the shared
 *   expert unweighted. experts[] is indexed by expert id. idx/wt receive the routing
 *   ([ntok][topk]) when non-NULL. Router W is fp32 [n_experts][hidden]. */
void ora_moe_layer(float *out, const float *x, int ntok, const float *router_w,
                   const float *router_bias, const ora_expert *experts,
                   const ora_expert *shared, int hidden, int inter, int n_experts,
                   int topk, int renorm, float routed_scale, int act,
                   int *idx, float *wt);

#ifdef __cplusplus
}
#endif

#endif /* K3_ORACLE_H */
