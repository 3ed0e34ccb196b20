// router.cu -- sigmoid top-k router (src/core/k3_ops.c:419-478 of the reference).
//
// logits  W.x with every product exact in double (bf16 and fp32 operands widen exactly) and
//         the sum in double, rounded once to float: the reference's double accumulator
//         (:447-450). Lane-strided summation reassociates exact products, which moves the
//         double sum by ~1e-16 relative; the float rounding absorbs it.
// score   1/(1+e) in float with e = exp(-logit) rounded once from double, i.e. a correctly
//         rounded expf; the reference calls libm expf (:451).
// select  repeated strict-greater argmax on score+bias from -INFINITY, lowest index on
//         ties, NaN never chosen, (0, 0.0f) when nothing qualifies (:459-467); renorm with
//         a double sum and a float inverse (:469-474); times routed_scale (:475).
#include <cuda_runtime.h>
#include <math.h>

#include "common.cuh"

namespace k3c {

template <typename T>
__device__ __forceinline__ double widen(const T *p, size_t i);
template <>
__device__ __forceinline__ double widen<float>(const float *p, size_t i) { return (double)p[i]; }
template <>
__device__ __forceinline__ double widen<uint16_t>(const uint16_t *p, size_t i) {
    return (double)bf16_bits_to_f32(p[i]);
}

// Eight W elements of row `row` from element k (k a multiple of 8, rows 16-byte aligned
// when vec): exact widening to double.
template <typename WT>
__device__ __forceinline__ void load_w8(const WT *row, int k, int hidden, bool vec, double (&w)[8]) {
    if (vec && k + 8 <= hidden) {
        if constexpr (sizeof(WT) == 2) {
            const uint4 u = *reinterpret_cast<const uint4 *>(row + k);
            const uint32_t p[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
            for (int q = 0; q < 4; q++) {
                w[2 * q] = (double)__uint_as_float(p[q] << 16);
                w[2 * q + 1] = (double)__uint_as_float(p[q] & 0xFFFF0000u);
            }
        } else {
            const float4 a = *reinterpret_cast<const float4 *>(row + k);
            const float4 b = *reinterpret_cast<const float4 *>(row + k + 4);
            w[0] = a.x; w[1] = a.y; w[2] = a.z; w[3] = a.w;
            w[4] = b.x; w[5] = b.y; w[6] = b.z; w[7] = b.w;
        }
    } else {
#pragma unroll
        for (int q = 0; q < 8; q++) w[q] = k + q < hidden ? widen<WT>(row, k + q) : 0.0;
    }
}

// grid (ceil(E/8), ceil(ntok/4)): warp w owns expert row 8*bx + w and the block's 4 tokens.
// x is staged in chunks of 2048 elements (fp32, exact) and reused by the 8 rows; each lane
// owns 8-element segments; products and sums in double, lane partials reduced by a fixed
// shuffle tree.
template <typename WT, typename XT>
__global__ void __launch_bounds__(256) k_router_scores(float *__restrict__ scores,
                                                       const XT *__restrict__ x,
                                                       const WT *__restrict__ W, int hidden,
                                                       int n_experts, int ntok, int vec) {
    constexpr int TCH = 4, KC = 2048;
    __shared__ __align__(16) float xs[TCH * KC];  // 32 KB
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int e = blockIdx.x * 8 + warp;
    const int t0 = blockIdx.y * TCH;
    const int nt = ntok - t0 < TCH ? ntok - t0 : TCH;
    double acc[TCH] = {0.0, 0.0, 0.0, 0.0};
    const WT *row = W + (size_t)(e < n_experts ? e : 0) * hidden;
    for (int k0 = 0; k0 < hidden; k0 += KC) {
        __syncthreads();
        for (int i = threadIdx.x; i < TCH * KC; i += blockDim.x) {
            const int t = i / KC, k = k0 + i % KC;
            xs[i] = (t < nt && k < hidden) ? (float)widen<XT>(x, (size_t)(t0 + t) * hidden + k) : 0.0f;
        }
        __syncthreads();
        if (e >= n_experts) continue;
        for (int seg = lane; seg < KC / 8 && k0 + 8 * seg < hidden; seg += 32) {
            double w[8];
            load_w8<WT>(row, k0 + 8 * seg, hidden, vec != 0, w);
#pragma unroll
            for (int t = 0; t < TCH; t++) {
                const float4 a = *reinterpret_cast<const float4 *>(xs + t * KC + 8 * seg);
                const float4 b = *reinterpret_cast<const float4 *>(xs + t * KC + 8 * seg + 4);
                acc[t] = fma(w[0], (double)a.x, acc[t]);
                acc[t] = fma(w[1], (double)a.y, acc[t]);
                acc[t] = fma(w[2], (double)a.z, acc[t]);
                acc[t] = fma(w[3], (double)a.w, acc[t]);
                acc[t] = fma(w[4], (double)b.x, acc[t]);
                acc[t] = fma(w[5], (double)b.y, acc[t]);
                acc[t] = fma(w[6], (double)b.z, acc[t]);
                acc[t] = fma(w[7], (double)b.w, acc[t]);
            }
        }
    }
    if (e >= n_experts) return;
#pragma unroll
    for (int t = 0; t < TCH; t++) {
        const double a = warp_sum_d(acc[t]);
        if (lane == 0 && t < nt) {
            const float logit = (float)a;
            const float ex = (float)exp(-(double)logit);
            scores[(size_t)(t0 + t) * n_experts + e] = __fdiv_rn(1.0f, __fadd_rn(1.0f, ex));
        }
    }
}

// One warp per token: top-k by repeated warp argmax over score+bias.
__global__ void __launch_bounds__(256) k_router_select(int *__restrict__ idx, float *__restrict__ w,
                                                       const float *__restrict__ scores,
                                                       const float *__restrict__ bias,
                                                       int n_experts, int topk, int renorm,
                                                       float routed_scale, int ntok) {
    extern __shared__ float ch[];  // [8 warps][n_experts] choice values
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = blockIdx.x * 8 + warp;
    if (t >= ntok) return;
    float *c = ch + (size_t)warp * n_experts;
    const float *s = scores + (size_t)t * n_experts;
    for (int e = lane; e < n_experts; e += 32) c[e] = __fadd_rn(s[e], bias ? bias[e] : 0.0f);
    __syncwarp();
    int *it = idx + (size_t)t * topk;
    float *wt = w + (size_t)t * topk;
    for (int j = 0; j < topk; j++) {
        float bv = -INFINITY;
        int bi = -1;
        for (int e = lane; e < n_experts; e += 32) {
            const float v = c[e];
            if (v > bv) { bv = v; bi = e; }  // ascending e per lane: first index wins
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (oi >= 0 && (bi < 0 || ov > bv || (ov == bv && oi < bi))) { bv = ov; bi = oi; }
        }
        if (lane == 0) {
            if (bi < 0) { it[j] = 0; wt[j] = 0.0f; }
            else { it[j] = bi; wt[j] = s[bi]; c[bi] = -INFINITY; }
        }
        __syncwarp();
    }
    if (lane == 0) {
        if (renorm && topk > 1) {
            double sum = 0.0;
            for (int j = 0; j < topk; j++) sum += (double)wt[j];
            const float inv = (float)(1.0 / (sum + 1e-20));
            for (int j = 0; j < topk; j++) wt[j] = __fmul_rn(wt[j], inv);
        }
        for (int j = 0; j < topk; j++) wt[j] = __fmul_rn(wt[j], routed_scale);
    }
}

int launch_router_select(int *idx, float *w, const float *scores, const float *bias,
                         int n_experts, int topk, int renorm, float routed_scale, int ntok,
                         cudaStream_t s) {
    if (n_experts <= 0 || topk <= 0 || topk > K3_MAX_TOPK || ntok < 0)
        return set_error(K3C_EINVAL, "router_select: n_experts=%d topk=%d ntok=%d", n_experts,
                         topk, ntok);
    if (ntok == 0) return K3C_OK;
    const size_t smem = (size_t)8 * n_experts * sizeof(float);
    if (smem > 200 * 1024) return set_error(K3C_EINVAL, "router_select: n_experts=%d too large", n_experts);
    if (smem > 48 * 1024)
        K3C_TRY_CUDA(cudaFuncSetAttribute(k_router_select, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    k_router_select<<<(ntok + 7) / 8, 256, smem, s>>>(idx, w, scores, bias, n_experts, topk,
                                                      renorm, routed_scale, ntok);
    K3C_CHECK_LAUNCH();
    return K3C_OK;
}

template <typename WT, typename XT>
static int launch_scores_t(float *scores, const void *x, const void *W, int hidden,
                           int n_experts, int ntok, cudaStream_t s) {
    const int vec = ((uintptr_t)W % 16 == 0) && ((hidden * (int)sizeof(WT)) % 16 == 0);
    k_router_scores<WT, XT><<<dim3((n_experts + 7) / 8, (ntok + 3) / 4), 256, 0, s>>>(
        scores, (const XT *)x, (const WT *)W, hidden, n_experts, ntok, vec);
    K3C_CHECK_LAUNCH();
    return K3C_OK;
}

int launch_router_scores(float *scores, const void *x, int x_dtype, const void *W, int w_dtype,
                         int hidden, int n_experts, int ntok, cudaStream_t s) {
    if (hidden <= 0 || n_experts <= 0) return set_error(K3C_EINVAL, "router: hidden=%d n_experts=%d", hidden, n_experts);
    if (ntok == 0) return K3C_OK;
    if (w_dtype == K3C_BF16 && x_dtype == K3C_BF16) return launch_scores_t<uint16_t, uint16_t>(scores, x, W, hidden, n_experts, ntok, s);
    if (w_dtype == K3C_BF16 && x_dtype == K3C_F32) return launch_scores_t<uint16_t, float>(scores, x, W, hidden, n_experts, ntok, s);
    if (w_dtype == K3C_F32 && x_dtype == K3C_BF16) return launch_scores_t<float, uint16_t>(scores, x, W, hidden, n_experts, ntok, s);
    if (w_dtype == K3C_F32 && x_dtype == K3C_F32) return launch_scores_t<float, float>(scores, x, W, hidden, n_experts, ntok, s);
    return set_error(K3C_EINVAL, "router: dtypes x=%d W=%d", x_dtype, w_dtype);
}

}  // namespace k3c

extern "C" int k3c_router_select(int *idx, float *w, const float *scores, const float *bias,
                                 int n_experts, int topk, int renorm, float routed_scale,
                                 int ntok, k3c_stream_t stream) {
    k3c::clear_error();
    return k3c::launch_router_select(idx, w, scores, bias, n_experts, topk, renorm,
                                     routed_scale, ntok, (cudaStream_t)stream);
}

extern "C" int k3c_router(int *idx, float *w, float *scores, const void *x, int x_dtype,
                          const void *W, int w_dtype, const float *bias, int hidden,
                          int n_experts, int topk, int renorm, float routed_scale, int ntok,
                          k3c_stream_t stream) {
    k3c::clear_error();
    cudaStream_t s = (cudaStream_t)stream;
    float *sc = scores;
    if (!sc) {
        K3C_TRY_CUDA(cudaMallocAsync((void **)&sc, (size_t)ntok * n_experts * sizeof(float), s));
    }
    int rc = k3c::launch_router_scores(sc, x, x_dtype, W, w_dtype, hidden, n_experts, ntok, s);
    if (rc == K3C_OK)
        rc = k3c::launch_router_select(idx, w, sc, bias, n_experts, topk, renorm, routed_scale,
                                       ntok, s);
    if (!scores) cudaFreeAsync(sc, s);
    return rc;
}
