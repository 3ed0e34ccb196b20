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
/* Trunk weight types, the reference's K3_WF32 / K3_WBF16 / K3_WI8 (include/k3/k3.h:270). */
enum { ORA_WF32 = 0, ORA_WBF16 = 1, ORA_WI8 = 2 };

float ora_e2m1(unsigned code);
float ora_e8m0(unsigned char b);

void ora_mxfp4_dequant(float *out, const unsigned char *packed, const unsigned char *scales,
                       int rows, int pcols, int group);
void ora_matmul_mxfp4(float *y, const float *x, const unsigned char *packed,
                      const unsigned char *scales, int in, int rows, int group);
void ora_matmul_f32(float *y, const float *x, const float *W, int in, int out);
void ora_matmul_bf16(float *y, const float *x, const uint16_t *W, int in, int out);
void ora_mmw(float *y, const float *x, const void *W, int wdt, int in, int out);
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

/* A latent MoE layer of the K3 model (the K3MoeW fields of include/k3/k3.h:357-380 and
 * the K3Cfg fields the layer reads, :94-113). Routed experts live at the latent width:
 * either the fp32 bank w1/w3 [n_experts][inter][latent], w2 [n_experts][latent][inter]
 * (the reference's fixtures), or, when w1 is NULL, experts[] in MXFP4. The trunk matrices
 * down [latent][hidden], up [hidden][latent], sh1/sh3 [inter*n_shared][hidden],
 * sh2 [hidden][inter*n_shared] have type wdt. */
typedef struct {
    const float *router_w, *router_bias;
    const float *w1, *w3, *w2;
    const ora_expert *experts;
    const float *latent_norm;
    const void *down, *up, *sh1, *sh3, *sh2;
    int wdt;
    int hidden, latent, inter, n_shared, n_experts, topk, renorm, latent_norm_on;
    float routed_scale, rms_eps, situ_b1, situ_b2;
} ora_latent;

void ora_moe_latent(float *out, const float *x, int ntok, const ora_latent *L, int *idx,
                    float *wt);

#ifdef __cplusplus
}
#endif

#endif /* K3_ORACLE_H */
