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

/* bf16 bit pattern -> fp32: the pattern is the top half of the float (include/k3/k3.h:274-279). */
static float ora_bf16f(uint16_t h)
{
    union { uint32_t u; float f; } v;
    v.u = (uint32_t)h << 16;
    return v.f;
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

/* One output of the trunk matmuls in the reference's fixed summation order: element i of
 * the first in - in%16 feeds double accumulator i%16 by a fused multiply-add in element
 * order; the sixteen are combined as b_l = (a_l + a_{l+4}) + (a_{l+8} + a_{l+12}) for
 * l = 0..3 and then (b0 + b1) + (b2 + b3); the in%16 tail is fused onto that total in
 * element order; the result is rounded once to float. Restates k3_matmul,
 * src/core/k3_ops.c:265-291. k3_matmul_bf16 (:1091-1196) keeps the same partition and
 * tree in each of its paths (the bf16 value is its bit pattern shifted into an fp32), so
 * both are bit-exact against this. bf16 != 0 selects uint16 weights. */
static float ora_dot_tree(const void *row, int bf16, const float *x, int in)
{
    const float *rf = (const float *)row;
    const uint16_t *rh = (const uint16_t *)row;
#define ORA_W(i) (bf16 ? ora_bf16f(rh[(i)]) : rf[(i)])
    double a[16] = { 0 };
    int i = 0;
    for (; i + 15 < in; i += 16)
        for (int l = 0; l < 16; l++) a[l] = fma((double)ORA_W(i + l), (double)x[i + l], a[l]);
    const double b0 = (a[0] + a[4]) + (a[8] + a[12]);
    const double b1 = (a[1] + a[5]) + (a[9] + a[13]);
    const double b2 = (a[2] + a[6]) + (a[10] + a[14]);
    const double b3 = (a[3] + a[7]) + (a[11] + a[15]);
    double acc = (b0 + b1) + (b2 + b3);
    for (; i < in; i++) acc = fma((double)ORA_W(i), (double)x[i], acc);
#undef ORA_W
    return (float)acc;
}

/* y[o] = sum_i W[o][i] x[i], fp32 weights [out][in], k3_matmul's order (above). */
void ora_matmul_f32(float *y, const float *x, const float *W, int in, int out)
{
#pragma omp parallel for schedule(static) if (out > 64)
    for (int o = 0; o < out; o++) y[o] = ora_dot_tree(W + (size_t)o * in, 0, x, in);
}

/* The same with bf16 weights (uint16 bit patterns [out][in]): k3_matmul_bf16,
 * src/core/k3_ops.c:1091-1196. */
void ora_matmul_bf16(float *y, const float *x, const uint16_t *W, int in, int out)
{
#pragma omp parallel for schedule(static) if (out > 64)
    for (int o = 0; o < out; o++) y[o] = ora_dot_tree(W + (size_t)o * in, 1, x, in);
}

/* The trunk matmul dispatch on the weight type, include/k3/k3.h:289-296. */
void ora_mmw(float *y, const float *x, const void *W, int wdt, int in, int out)
{
    if (wdt == ORA_WBF16) ora_matmul_bf16(y, x, (const uint16_t *)W, in, out);
    else if (wdt == ORA_WI8) ora_matmul_q8(y, x, W, in, out);
    else ora_matmul_f32(y, x, (const float *)W, in, out);
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

/* The latent MoE layer of the K3 model, src/core/k3_ops.c:556-656, per token:
 *   1. route on the full-width input (:576);
 *   2. z = down x, the trunk matmul into the latent width (:596);
 *   3. accL = sum over the top-k of w_j * expert_j(z), in float, in top-k order, from zero,
 *      each expert gate/up -> SiTU-GLU -> down at the latent width (:599-642); the experts
 *      come from the fp32 bank w1/w3/w2 through k3_matmul (:635-638) or, when w1 is NULL,
 *      from MXFP4 experts through k3_matmul_mxfp4 (:628-631);
 *   4. RMSNorm of the aggregate when latent_norm_on (:646);
 *   5. out = up accL (:647);
 *   6. the shared expert at full width (sh1/sh3 -> SiTU-GLU -> sh2, intermediate
 *      inter*n_shared) on the original input, added with no weight (:650-654).
 * idx/wt ([ntok][topk]) receive the routing when non-NULL. The draft-only cache_only mode
 * (:580-593) is not part of this path. */
void ora_moe_latent(float *out, const float *x, int ntok, const ora_latent *L, int *idx,
                    float *wt)
{
    const int E = L->hidden, Lw = L->latent, I = L->inter, SI = L->inter * L->n_shared;
    const int K = L->topk;
    int *li = (int *)malloc((size_t)K * sizeof(int));
    float *lw = (float *)malloc((size_t)K * sizeof(float));
    float *z = (float *)malloc((size_t)Lw * sizeof(float));
    float *acc = (float *)malloc((size_t)Lw * sizeof(float));
    float *gu = (float *)malloc((size_t)3 * I * sizeof(float));
    float *edn = (float *)malloc((size_t)Lw * sizeof(float));
    float *sgu = (float *)malloc((size_t)3 * SI * sizeof(float));
    float *sdn = (float *)malloc((size_t)E * sizeof(float));
    if (!li || !lw || !z || !acc || !gu || !edn || !sgu || !sdn)
        ora_fatal("ora_moe_latent: out of memory", E);
    float *act = gu + 2 * I, *sact = sgu + 2 * SI;
    for (int t = 0; t < ntok; t++) {
        const float *xt = x + (size_t)t * E;
        float *ot = out + (size_t)t * E;
        ora_router(li, lw, xt, L->router_w, L->router_bias, E, L->n_experts, K, L->renorm,
                   L->routed_scale);
        ora_mmw(z, xt, L->down, L->wdt, E, Lw);
        for (int i = 0; i < Lw; i++) acc[i] = 0.0f;
        for (int j = 0; j < K; j++) {
            const int e = li[j];
            if (L->w1) {
                ora_matmul_f32(gu, z, L->w1 + (size_t)e * I * Lw, Lw, I);
                ora_matmul_f32(gu + I, z, L->w3 + (size_t)e * I * Lw, Lw, I);
                ora_situ_glu(act, gu, I, L->situ_b1, L->situ_b2);
                ora_matmul_f32(edn, act, L->w2 + (size_t)e * Lw * I, I, Lw);
            } else {
                const ora_expert *q = &L->experts[e];
                ora_matmul_mxfp4(gu, z, q->p1, q->s1, Lw, I, 32);
                ora_matmul_mxfp4(gu + I, z, q->p3, q->s3, Lw, I, 32);
                ora_situ_glu(act, gu, I, L->situ_b1, L->situ_b2);
                ora_matmul_mxfp4(edn, act, q->p2, q->s2, I, Lw, 32);
            }
            const float wj = lw[j];
            for (int i = 0; i < Lw; i++) acc[i] += wj * edn[i];
        }
        if (L->latent_norm_on) ora_rmsnorm(acc, acc, L->latent_norm, Lw, L->rms_eps);
        ora_mmw(ot, acc, L->up, L->wdt, Lw, E);
        ora_mmw(sgu, xt, L->sh1, L->wdt, E, SI);
        ora_mmw(sgu + SI, xt, L->sh3, L->wdt, E, SI);
        ora_situ_glu(sact, sgu, SI, L->situ_b1, L->situ_b2);
        ora_mmw(sdn, sact, L->sh2, L->wdt, SI, E);
        for (int i = 0; i < E; i++) ot[i] += sdn[i];
        if (idx) memcpy(idx + (size_t)t * K, li, (size_t)K * sizeof(int));
        if (wt) memcpy(wt + (size_t)t * K, lw, (size_t)K * sizeof(float));
    }
    free(li); free(lw); free(z); free(acc); free(gu); free(edn); free(sgu); free(sdn);
}
