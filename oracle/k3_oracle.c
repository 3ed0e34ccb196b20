/* k3_oracle.c -- CPU restatement of the reference's routed-expert hot path.
 *
 * TEST INFRASTRUCTURE ONLY (see k3_oracle.h). The product is libk3cuda.so; nothing in it
 * links this file. Built with -ffp-contract=off and without -ffast-math, the same
 * floating-point contract the reference states at src/core/k3_ops.c:8-29, so that every
 * float operation written here is the operation that runs.
 *
 * Row loops are OpenMP-parallel over independent output rows only; each row is summed by
 * one thread in a fixed order, so results do not depend on the thread count (the same
 * property the reference relies on, src/core/k3_ops.c:249-252).
 */
#include "k3_oracle.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

static void ora_fatal(const char *msg, long v)
{
    fprintf(stderr, "k3_oracle: FATAL, %s (%ld)\n", msg, v);
    abort();
}

/* E2M1 code -> value. Bit 3 is the sign, bits 0-2 index the eight magnitudes
 * {0, .5, 1, 1.5, 2, 3, 4, 6}; code 8 is -0.0. Restates K3_E2M1, src/core/k3_ops.c:1049-1052. */
float ora_e2m1(unsigned code)
{
    static const float mag[8] = { 0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f };
    const float m = mag[code & 7u];
    return (code & 8u) ? -m : m;
}

/* E8M0 byte -> 2^(b-127); 255 (NaN by the OCP MX spec) is zero.
 * Restates k3_e8m0_init, src/core/k3_ops.c:1315-1322, and the dequant's own mapping at
 * :1784-1785. ldexpf is exact for a power of two, including the subnormal 2^-127. */
float ora_e8m0(unsigned char b)
{
    return b == 255 ? 0.0f : ldexpf(1.0f, (int)b - 127);
}

/* out[r][i] = E2M1(nibble(r,i)) * E8M0(scale(r, i/group)); the LOW nibble of a byte is the
 * EVEN element. Restates k3_mxfp4_dequant, src/core/k3_ops.c:1770-1800. */
void ora_mxfp4_dequant(float *out, const unsigned char *packed, const unsigned char *scales,
                       int rows, int pcols, int group)
{
    const int width = pcols * 2;
    const int ngrp = (width + group - 1) / group;
    for (int r = 0; r < rows; r++) {
        const unsigned char *pr = packed + (size_t)r * pcols;
        const unsigned char *sr = scales + (size_t)r * ngrp;
        float *o = out + (size_t)r * width;
        for (int i = 0; i < width; i++) {
            const unsigned char byte = pr[i >> 1];
            const unsigned nib = (i & 1) ? (unsigned)(byte >> 4) : (unsigned)(byte & 0x0F);
            o[i] = ora_e2m1(nib) * ora_e8m0(sr[i / group]);
        }
    }
}

/* y[r] = sum_i W[r][i] x[i] with W read as MXFP4. Restates k3_matmul_mxfp4,
 * src/core/k3_ops.c:1363-1768: preconditions `in` even and group <= 64 abort
 * (:1366-1384); ngrp = ceil(in/group) (:1387); a 255 scale skips its whole group
 * (:1519); accumulation in double, output rounded once to float (:1764).
 * Each weight is formed as the fp32 product E2M1 * 2^(s-127), exactly as the reference's
 * flat row path folds the scale into the weight (:1420-1427, :1463-1464): exact, except
 * that s >= 252 with a large code overflows to +-inf, which then propagates (inf, or NaN
 * when both signs occur), the dequantise-then-matmul semantics. Products are exact in
 * double; each group is summed in element order and added to the row total. The
 * reference's 16-lane order reassociates the same exact products; the two agree to
 * ~1e-16 relative, the bound the reference documents at :1347-1361. */
void ora_matmul_mxfp4(float *y, const float *x, const unsigned char *packed,
                      const unsigned char *scales, int in, int rows, int group)
{
    if (in & 1) ora_fatal("ora_matmul_mxfp4: odd `in`", in);
    if (group > 64 || group <= 0) ora_fatal("ora_matmul_mxfp4: group outside 1..64", group);
    const int pcols = in / 2;
    const int ngrp = (in + group - 1) / group;
#pragma omp parallel for schedule(static) if (rows > 64)
    for (int r = 0; r < rows; r++) {
        const unsigned char *pr = packed + (size_t)r * pcols;
        const unsigned char *sr = scales + (size_t)r * ngrp;
        double acc = 0.0;
        for (int g = 0; g < ngrp; g++) {
            if (sr[g] == 255) continue;
            const int lo = g * group;
            const int hi = lo + group < in ? lo + group : in;
            const float sc = ora_e8m0(sr[g]);
            double sub = 0.0;
            for (int i = lo; i < hi; i++) {
                const unsigned char byte = pr[i >> 1];
                const unsigned nib = (i & 1) ? (unsigned)(byte >> 4) : (unsigned)(byte & 0x0F);
                const float wv = ora_e2m1(nib) * sc;
                sub += (double)wv * (double)x[i];
            }
            acc += sub;
        }
        y[r] = (float)acc;
    }
}

/* y[o] = sum_i W[o][i] x[i], fp32 weights, double accumulator, one rounding at the end.
 * The reference's k3_matmul (src/core/k3_ops.c:265-291) splits the sum over 16 lanes;
 * this sums in element order. Used only to build dequantise-then-matmul comparisons,
 * the check the reference itself makes at tests/unit/test_expert.c:192-238. */
void ora_matmul_f32(float *y, const float *x, const float *W, int in, int out)
{
#pragma omp parallel for schedule(static) if (out > 64)
    for (int o = 0; o < out; o++) {
        const float *row = W + (size_t)o * in;
        double acc = 0.0;
        for (int i = 0; i < in; i++) acc += (double)row[i] * (double)x[i];
        y[o] = (float)acc;
    }
}

/* Per-row int8 matmul over the reference's inline row layout [f32 scale][int8 * in],
 * row stride 4+in bytes (include/k3/k3.h:265-303). y[o] = scale_o * sum_i w[o][i] x[i].
 * Restates k3_matmul_q8, src/core/k3_ops.c:1204-1272. The reference accumulates in float
 * and states no determinism contract for this kernel (:1198-1203); the oracle sums in
 * double so that it is the more accurate of the two and the comparison tolerance bounds
 * the device kernel's float rounding. */
void ora_matmul_q8(float *y, const float *x, const void *W, int in, int out)
{
    const unsigned char *base = (const unsigned char *)W;
    const size_t rowb = (size_t)4 + (size_t)in;
#pragma omp parallel for schedule(static) if (out > 64)
    for (int o = 0; o < out; o++) {
        const unsigned char *row = base + (size_t)o * rowb;
        float scale;
        memcpy(&scale, row, 4);
        const signed char *w = (const signed char *)(row + 4);
        double acc = 0.0;
        for (int i = 0; i < in; i++) acc += (double)w[i] * (double)x[i];
        y[o] = (float)acc * scale;
    }
}

/* score[e] = sigmoid(W[e] . x): double accumulator in element order, the logit rounded to
 * float, then 1/(1+expf(-logit)) in float. Restates src/core/k3_ops.c:447-451. */
void ora_router_scores(float *score, const float *x, const float *W, int hidden, int n_experts)
{
#pragma omp parallel for schedule(static) if (n_experts > 64)
    for (int e = 0; e < n_experts; e++) {
        const float *row = W + (size_t)e * hidden;
        double acc = 0.0;
        for (int i = 0; i < hidden; i++) acc += (double)row[i] * (double)x[i];
        score[e] = 1.0f / (1.0f + expf(-(float)acc));
    }
}

/* Top-k selection on score+bias with the weights gathered from the UNBIASED score.
 * Restates src/core/k3_ops.c:452-475: repeated strict-greater argmax from -INFINITY (so
 * ties go to the lowest index and NaN is never chosen), a taken entry becomes -INFINITY,
 * an exhausted search writes (0, 0.0f); renormalisation, when renorm && topk > 1, sums the
 * weights in double, takes inv = (float)(1/(sum+1e-20)) and multiplies in float; finally
 * every weight is multiplied by routed_scale. idx/w come out in descending choice order. */
void ora_router_select(int *idx, float *w, const float *score, const float *bias,
                       int n_experts, int topk, int renorm, float routed_scale)
{
    float *choice = (float *)malloc((size_t)n_experts * sizeof(float));
    if (!choice) ora_fatal("ora_router_select: out of memory", n_experts);
    for (int e = 0; e < n_experts; e++) choice[e] = score[e] + (bias ? bias[e] : 0.0f);
    for (int j = 0; j < topk; j++) {
        int best = -1;
        float bv = -INFINITY;
        for (int e = 0; e < n_experts; e++)
            if (choice[e] > bv) { bv = choice[e]; best = e; }
        if (best < 0) { idx[j] = 0; w[j] = 0.0f; continue; }
        idx[j] = best;
        w[j] = score[best];
        choice[best] = -INFINITY;
    }
    if (renorm && topk > 1) {
        double s = 0.0;
        for (int j = 0; j < topk; j++) s += (double)w[j];
        const float inv = (float)(1.0 / (s + 1e-20));
        for (int j = 0; j < topk; j++) w[j] *= inv;
    }
    for (int j = 0; j < topk; j++) w[j] *= routed_scale;
    free(choice);
}

/* The whole router, src/core/k3_ops.c:419-478. */
void ora_router(int *idx, float *w, const float *x, const float *W, const float *bias,
                int hidden, int n_experts, int topk, int renorm, float routed_scale)
{
    float *score = (float *)malloc((size_t)n_experts * sizeof(float));
    if (!score) ora_fatal("ora_router: out of memory", n_experts);
    ora_router_scores(score, x, W, hidden, n_experts);
    ora_router_select(idx, w, score, bias, n_experts, topk, renorm, routed_scale);
    free(score);
}

static float ora_sigmoidf(float v) { return 1.0f / (1.0f + expf(-v)); }

/* SwiGLU over gu = [gate | up] (n each): y = (g * sigmoid(g)) * u in float, with the
 * sigmoid written as at src/core/k3_ops.c:105. The reference ships no SwiGLU; the
 * BASELINE configs use it, so it is restated from its definition silu(g) * u. */
void ora_swiglu(float *y, const float *gu, int n)
{
    for (int i = 0; i < n; i++) {
        const float g = gu[i];
        y[i] = (g * ora_sigmoidf(g)) * gu[n + i];
    }
}

/* SiTU-GLU, src/core/k3_ops.c:110-123: a = b1*tanh(g/b1)*sigmoid(g) (the sigmoid sees the
 * UNCAPPED gate), u = b2*tanh(up/b2), y = a*u. */
void ora_situ_glu(float *y, const float *gu, int n, float b1, float b2)
{
    for (int i = 0; i < n; i++) {
        const float g = gu[i];
        const float a = b1 * tanhf(g / b1) * ora_sigmoidf(g);
        const float u = b2 * tanhf(gu[n + i] / b2);
        y[i] = a * u;
    }
}

/* RMSNorm with a double sum of squares and eps inside the root, src/core/k3_ops.c:94-102. */
void ora_rmsnorm(float *y, const float *x, const float *w, int n, float eps)
{
    double ss = 0.0;
    for (int i = 0; i < n; i++) ss += (double)x[i] * (double)x[i];
    const float inv = (float)(1.0 / sqrt(ss / (double)n + (double)eps));
    for (int i = 0; i < n; i++) y[i] = w[i] * x[i] * inv;
}

/* One expert for ntok tokens: the src/core/k3_ops.c:628-631 sequence (gate, up, activation,
 * down) at the expert's own width, with the activation selectable (SiTU is the reference's,
 * SwiGLU the BASELINE configs'). SiTU uses the K3 constants b1=4, b2=25 (k3.h:111-113). */
void ora_expert_ffn(float *y, const float *x, int ntok, const ora_expert *e,
                    int hidden, int inter, int act)
{
    float *gu = (float *)malloc((size_t)3 * inter * sizeof(float));
    if (!gu) ora_fatal("ora_expert_ffn: out of memory", inter);
    float *a = gu + 2 * inter;
    for (int t = 0; t < ntok; t++) {
        const float *xt = x + (size_t)t * hidden;
        ora_matmul_mxfp4(gu, xt, e->p1, e->s1, hidden, inter, 32);
        ora_matmul_mxfp4(gu + inter, xt, e->p3, e->s3, hidden, inter, 32);
        if (act == ORA_ACT_SITU) ora_situ_glu(a, gu, inter, 4.0f, 25.0f);
        else ora_swiglu(a, gu, inter);
        ora_matmul_mxfp4(y + (size_t)t * hidden, a, e->p2, e->s2, inter, hidden, 32);
    }
    free(gu);
}

/* Non-latent MoE layer (BASELINE config[1]/[2] shape). Per token: route on the full input
 * (src/core/k3_ops.c:576), run the selected experts, accumulate acc += w_j * expert_j in
 * float and in top-k order starting from zero (:599, :641-642), then add the shared expert
 * computed on the same input with no weight (:650-654). The latent down/up projection and
 * aggregate RMSNorm of the K3 model (:596, :646-647) are absent in these configs. The
 * prefill chunk-union schedule (:717-808) produces per-token results identical to this
 * per-token loop by construction (:677-681), so this one function is the oracle for both. */
void ora_moe_layer(float *out, const float *x, int ntok, const float *router_w,
                   const float *router_bias, const ora_expert *experts,
                   const ora_expert *shared, int hidden, int inter, int n_experts,
                   int topk, int renorm, float routed_scale, int act,
                   int *idx, float *wt)
{
    int *li = (int *)malloc((size_t)topk * sizeof(int));
    float *lw = (float *)malloc((size_t)topk * sizeof(float));
    float *edn = (float *)malloc((size_t)hidden * sizeof(float));
    float *sdn = (float *)malloc((size_t)hidden * sizeof(float));
    if (!li || !lw || !edn || !sdn) ora_fatal("ora_moe_layer: out of memory", hidden);
    for (int t = 0; t < ntok; t++) {
        const float *xt = x + (size_t)t * hidden;
        float *ot = out + (size_t)t * hidden;
        ora_router(li, lw, xt, router_w, router_bias, hidden, n_experts, topk, renorm,
                   routed_scale);
        for (int i = 0; i < hidden; i++) ot[i] = 0.0f;
        for (int j = 0; j < topk; j++) {
            ora_expert_ffn(edn, xt, 1, &experts[li[j]], hidden, inter, act);
            const float wj = lw[j];
            for (int i = 0; i < hidden; i++) ot[i] += wj * edn[i];
        }
        if (shared) {
            ora_expert_ffn(sdn, xt, 1, shared, hidden, inter, act);
            for (int i = 0; i < hidden; i++) ot[i] += sdn[i];
        }
        if (idx) memcpy(idx + (size_t)t * topk, li, (size_t)topk * sizeof(int));
        if (wt) memcpy(wt + (size_t)t * topk, lw, (size_t)topk * sizeof(float));
    }
    free(li); free(lw); free(edn); free(sdn);
}
