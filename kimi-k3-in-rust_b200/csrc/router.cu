// router.cu -- sigmoid top-k router (src/core/k3_ops.c:419-478 of the reference).
//
// logits  W.x with every product exact in double (bf16 and fp32 operands widen exactly) and
//         the sum in double, rounded once to float: the reference's double accumulator
//         (:447-450). The sum runs in K chunks of 256 (one kernel, partials in double) that
//         the select kernel adds in chunk order; the chunked, lane-strided order reassociates
//         exact products, which moves the double sum by ~1e-16 relative; the float rounding
//         absorbs it.
// score   1/(1+e) in float with e = exp(-logit) rounded once from double, i.e. a correctly
//         rounded expf; the reference calls libm expf (:451).
// select  repeated strict-greater argmax on score+bias from -INFINITY, lowest index on
//         ties, NaN never chosen, (0, 0.0f) when nothing qualifies (:459-467); renorm with
//         a double sum and a float inverse (:469-474); times routed_scale (:475).
#include <cuda_runtime.h>
#include <math.h>
#include <stdlib.h>

#include <type_traits>

#include "common.cuh"
#include "rt_tc.cuh"

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

// Logits in K chunks of RT_KC = 256: grid (ceil(E/32), ceil(hidden/RT_KC), ceil(ntok/NT)),
// 256 threads. The block stages x[chunk][NT tokens] in shared memory as double (exact,
// converted once per block). Lane l of every warp takes expert 32*bx + l and streams its own
// W row, warp w the K slice [32w, 32w+32) of the chunk, so every shared-memory read of x is
// a broadcast feeding 32 FMAs (one per lane). The eight slice sums are added in warp order
// and part[chunk][t][e] receives the chunk's double sum; the select kernel adds the chunks
// in order. NT (1..16 tokens per block) keeps small batches from computing empty slots.
constexpr int RT_KC = 256;
constexpr int RT_KW = RT_KC / 8;   // K per warp

template <typename XT>
__device__ __forceinline__ void load_x8(const XT *p, int n, bool vec, float (&v)[8]);
template <>
__device__ __forceinline__ void load_x8<uint16_t>(const uint16_t *p, int n, bool vec, float (&v)[8]) {
    if (vec && n >= 8) {
        const uint4 u = *reinterpret_cast<const uint4 *>(p);
        const uint32_t q[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            v[2 * i] = __uint_as_float(q[i] << 16);
            v[2 * i + 1] = __uint_as_float(q[i] & 0xFFFF0000u);
        }
    } else {
#pragma unroll
        for (int i = 0; i < 8; i++) v[i] = i < n ? bf16_bits_to_f32(p[i]) : 0.0f;
    }
}
template <>
__device__ __forceinline__ void load_x8<float>(const float *p, int n, bool vec, float (&v)[8]) {
    if (vec && n >= 8) {
        const float4 a = *reinterpret_cast<const float4 *>(p);
        const float4 b = *reinterpret_cast<const float4 *>(p + 4);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
        v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    } else {
#pragma unroll
        for (int i = 0; i < 8; i++) v[i] = i < n ? p[i] : 0.0f;
    }
}

__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// A lane's whole RT_KW-element W slice as raw 16-byte vectors, all requested at once.
template <typename WT>
struct WSlice {
    static constexpr int V = RT_KW * (int)sizeof(WT) / 16;
    uint4 raw[V];
    __device__ __forceinline__ void load(const WT *row) {
#pragma unroll
        for (int i = 0; i < V; i++) raw[i] = *reinterpret_cast<const uint4 *>(row + i * (16 / sizeof(WT)));
    }
    // elements [8g, 8g+8) widened to double (exact)
    __device__ __forceinline__ void get(int g, double (&w)[8]) const {
        if constexpr (sizeof(WT) == 2) {
            const uint4 u = raw[g];
            const uint32_t q[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
            for (int i = 0; i < 4; i++) {
                w[2 * i] = (double)__uint_as_float(q[i] << 16);
                w[2 * i + 1] = (double)__uint_as_float(q[i] & 0xFFFF0000u);
            }
        } else {
            const uint4 a = raw[2 * g], b = raw[2 * g + 1];
            w[0] = __uint_as_float(a.x); w[1] = __uint_as_float(a.y);
            w[2] = __uint_as_float(a.z); w[3] = __uint_as_float(a.w);
            w[4] = __uint_as_float(b.x); w[5] = __uint_as_float(b.y);
            w[6] = __uint_as_float(b.z); w[7] = __uint_as_float(b.w);
        }
    }
};

// EPT experts per lane (lane l of block b takes experts 32*EPT*b + l + 32*u, u < EPT): every
// activation read from shared memory then feeds EPT x 2 FMAs, which keeps the FP64 pipe rather
// than the shared-memory pipe the limit at 16 tokens per block. Each expert's sum keeps its
// order (its own K slice per warp, warps in order, chunks in order), whatever EPT is.
template <typename WT, typename XT, int NT, int EPT>
__global__ void __launch_bounds__(256, EPT == 1 ? 2 : 1) k_router_partial(double *__restrict__ part,
                                                                      const XT *__restrict__ x,
                                                                      const WT *__restrict__ W, int hidden,
                                                                      int n_experts, int ntok, int vec_w, int vec_x,
                                                                      int cpb) {
    extern __shared__ __align__(16) double rsm[];   // xs [RT_KC][NT], then red [8][NT][32*EPT]
    double *xs = rsm;
    double *red = rsm + RT_KC * NT;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    grid_dep_launch();   // the select kernel may be scheduled; it waits for this grid's end
    grid_dep_wait();     // x may come from the previous kernel
    const int t0 = blockIdx.z * NT, nt = min(NT, ntok - t0);
    int e[EPT];
#pragma unroll
    for (int u = 0; u < EPT; u++) e[u] = blockIdx.x * 32 * EPT + 32 * u + lane;
    double acc[EPT][NT];
#pragma unroll
    for (int u = 0; u < EPT; u++)
#pragma unroll
        for (int t = 0; t < NT; t++) acc[u][t] = 0.0;
    // this block adds chunks [cpb*y, cpb*y + cpb) in order; chunk c+1's activations and W
    // slices are loaded into registers while chunk c is multiplied
    const int nchunk = (hidden + RT_KC - 1) / RT_KC;
    const int c_begin = blockIdx.y * cpb, c_end = min(nchunk, c_begin + cpb);
    constexpr int NG = NT * (RT_KC / 8);                 // 8-element groups per chunk
    constexpr int XR = NG >= 256 ? NG / 256 : 1;         // groups per thread
    float xv[XR][8];
    auto load_chunk = [&](int c) {
        const int k0 = c * RT_KC, kn = min(RT_KC, hidden - k0);
#pragma unroll
        for (int r = 0; r < XR; r++) {
            const int i = threadIdx.x + 256 * r;
            // consecutive threads take consecutive tokens, so stores of one k row are contiguous
            const int t = i % NT, kk = (i / NT) * 8;
            if (i < NG && t < nt) load_x8<XT>(x + (size_t)(t0 + t) * hidden + k0 + kk, kn - kk, vec_x != 0, xv[r]);
            else
#pragma unroll
                for (int q = 0; q < 8; q++) xv[r][q] = 0.0f;
        }
    };
    auto store_chunk = [&]() {
#pragma unroll
        for (int r = 0; r < XR; r++) {
            const int i = threadIdx.x + 256 * r;
            if (i >= NG) continue;
            const int t = i % NT, kk = (i / NT) * 8;
#pragma unroll
            for (int q = 0; q < 8; q++) xs[(kk + q) * NT + t] = (double)xv[r][q];
        }
    };
    // every chunk full and rows 16-byte aligned: whole W slices, one round trip each
    const bool wfast = vec_w && hidden % RT_KC == 0;
    const WT *wbase[EPT];
#pragma unroll
    for (int u = 0; u < EPT; u++) wbase[u] = W + (size_t)(e[u] < n_experts ? e[u] : 0) * hidden + warp * RT_KW;
    WSlice<WT> wnext[EPT];
    load_chunk(c_begin);
    if (wfast)
#pragma unroll
        for (int u = 0; u < EPT; u++) wnext[u].load(wbase[u] + (size_t)c_begin * RT_KC);
    for (int c = c_begin; c < c_end; c++) {
        const int k0 = c * RT_KC, kn = min(RT_KC, hidden - k0);
        if (c > c_begin) __syncthreads();   // every warp is done with the previous chunk
        store_chunk();
        __syncthreads();
        WSlice<WT> wcur[EPT];
#pragma unroll
        for (int u = 0; u < EPT; u++) wcur[u] = wnext[u];
        if (c + 1 < c_end) {
            load_chunk(c + 1);
            if (wfast)
#pragma unroll
                for (int u = 0; u < EPT; u++) wnext[u].load(wbase[u] + (size_t)(c + 1) * RT_KC);
        }
        const int kw = warp * RT_KW, kwn = min(RT_KW, kn - kw);   // this warp's slice
        // acc[u][t] += w[u][0..8) . x[kw+k .. kw+k+8)[t]
        auto step = [&](const double (&w)[EPT][8], int k) {
#pragma unroll
            for (int q = 0; q < 8; q++) {
                const double *xp = xs + (kw + k + q) * NT;   // same address in every lane: broadcast
                if constexpr (NT % 2 == 0) {
#pragma unroll
                    for (int t2 = 0; t2 < NT / 2; t2++) {
                        const double2 xq = reinterpret_cast<const double2 *>(xp)[t2];
#pragma unroll
                        for (int u = 0; u < EPT; u++) {
                            acc[u][2 * t2] = fma(w[u][q], xq.x, acc[u][2 * t2]);
                            acc[u][2 * t2 + 1] = fma(w[u][q], xq.y, acc[u][2 * t2 + 1]);
                        }
                    }
                } else {
#pragma unroll
                    for (int t = 0; t < NT; t++)
#pragma unroll
                        for (int u = 0; u < EPT; u++) acc[u][t] = fma(w[u][q], xp[t], acc[u][t]);
                }
            }
        };
        if (wfast) {
#pragma unroll
            for (int g = 0; g < RT_KW / 8; g++) {
                double w[EPT][8];
#pragma unroll
                for (int u = 0; u < EPT; u++) wcur[u].get(g, w[u]);
                step(w, 8 * g);
            }
        } else {
            for (int k = 0; k < kwn; k += 8) {
                double w[EPT][8];
#pragma unroll
                for (int u = 0; u < EPT; u++)
                    load_w8<WT>(W + (size_t)(e[u] < n_experts ? e[u] : 0) * hidden + k0 + kw, k, kwn, vec_w != 0,
                                w[u]);
                step(w, k);
            }
        }
    }
    constexpr int EW = 32 * EPT;   // experts per block
#pragma unroll
    for (int u = 0; u < EPT; u++)
#pragma unroll
        for (int t = 0; t < NT; t++) red[(warp * NT + t) * EW + 32 * u + lane] = acc[u][t];
    __syncthreads();
    for (int i = threadIdx.x; i < NT * EW; i += 256) {
        const int t = i / EW, l = i % EW, ee = blockIdx.x * EW + l;
        double sum = red[t * EW + l];
#pragma unroll
        for (int w = 1; w < 8; w++) sum += red[(w * NT + t) * EW + l];
        if (t < nt && ee < n_experts) part[((size_t)blockIdx.y * ntok + t0 + t) * n_experts + ee] = sum;
    }
}

__device__ __forceinline__ float sigmoid_score(double logit_d) {
    const float logit = (float)logit_d;
    const float ex = (float)exp(-(double)logit);
    return __fdiv_rn(1.0f, __fadd_rn(1.0f, ex));
}

// The plain double dot product of token row x and expert row w (the reference's own order),
// for a row whose residual list overflowed or that holds a NaN or an infinity.
__device__ __noinline__ double rt_plain(const uint16_t *wrow, const uint16_t *xrow, int H) {
    double acc = 0.0;
    for (int k = 0; k < H; k++) acc += (double)bf16_bits_to_f32(wrow[k]) * (double)bf16_bits_to_f32(xrow[k]);
    return acc;
}

// The tensor-core logits lg[u] of RU (token, expert) items completed with their residual
// terms: c = sum_i rx_i * w[k_i] over the token's list, then + sum_j (x[k_j] - rx(x[k_j])) *
// rw_j over the expert's list, in list order, and lg + c -- each item's own order, with the
// items' loads interleaved so that their round trips overlap. Items with ok[u] false are
// skipped; an item whose list overflowed gets the plain double dot product.
template <int RU>
__device__ __forceinline__ void rt_finish(const RtFix &fix, double (&lg)[RU], const bool (&ok)[RU],
                                          const int (&tt)[RU], const int (&t)[RU], const int (&e)[RU],
                                          const int *s_nx, const int *s_ex, const int (*s_xk)[RT_CAP],
                                          const float (*s_xr)[RT_CAP], int n_experts) {
    int nx[RU], nw[RU];
    int nxm = 0, nwm = 0;
#pragma unroll
    for (int u = 0; u < RU; u++) {
        nx[u] = ok[u] ? s_nx[tt[u]] : 0;
        nw[u] = ok[u] ? fix.wcnt[e[u]] : 0;
    }
    bool plain[RU];
    double c[RU];
#pragma unroll
    for (int u = 0; u < RU; u++) {
        plain[u] = ok[u] && (nx[u] > fix.cap || nw[u] > fix.cap);
        if (plain[u] || !ok[u]) nx[u] = nw[u] = 0;
        nxm = max(nxm, nx[u]);
        nwm = max(nwm, nw[u]);
        c[u] = 0.0;
    }
    for (int i = 0; i < nxm; i++) {
        float wv[RU];
#pragma unroll
        for (int u = 0; u < RU; u++)
            wv[u] = i < nx[u] ? bf16_bits_to_f32(fix.W[(size_t)e[u] * fix.H + s_xk[tt[u]][i]]) : 0.0f;
#pragma unroll
        for (int u = 0; u < RU; u++)
            if (i < nx[u]) c[u] += (double)s_xr[tt[u]][i] * (double)wv[u];
    }
    for (int j = 0; j < nwm; j++) {
        int k[RU];
        float r[RU], xv[RU];
#pragma unroll
        for (int u = 0; u < RU; u++) {
            k[u] = j < nw[u] ? fix.wk[(size_t)j * n_experts + e[u]] : 0;
            r[u] = j < nw[u] ? fix.wr[(size_t)j * n_experts + e[u]] : 0.0f;
        }
#pragma unroll
        for (int u = 0; u < RU; u++) xv[u] = j < nw[u] ? bf16_bits_to_f32(fix.x[(size_t)t[u] * fix.H + k[u]]) : 0.0f;
#pragma unroll
        for (int u = 0; u < RU; u++)
            if (j < nw[u]) {
                int q0, q1, q2;
                const float rx = rt_split(xv[u], s_ex[tt[u]], q0, q1, q2);
                c[u] += (double)(xv[u] - rx) * (double)r[u];
            }
    }
#pragma unroll
    for (int u = 0; u < RU; u++) {
        if (plain[u]) lg[u] = rt_plain(fix.W + (size_t)e[u] * fix.H, fix.x + (size_t)t[u] * fix.H, fix.H);
        else if (ok[u]) lg[u] = lg[u] + c[u];
    }
}

// TPB tokens per block (1 for small batches, 8 for large ones). With `part`, all threads
// first form the scores from the logit chunks (added in chunk order) and write them to
// `scores` if that is not null; otherwise `scores` holds them on entry. Warp tt then takes
// token tt's top-k by repeated warp argmax over score+bias.
template <int TPB>
__global__ void __launch_bounds__(256) k_router_select(int *__restrict__ idx, float *__restrict__ w,
                                                       float *__restrict__ scores,
                                                       const double *__restrict__ part, int nchunk,
                                                       const float *__restrict__ bias,
                                                       int n_experts, int topk, int renorm,
                                                       float routed_scale, int ntok, RtFix fix) {
    extern __shared__ float ch[];  // [TPB][2][n_experts]: choice values, scores
    __shared__ int s_xk[TPB][RT_CAP];
    __shared__ float s_xr[TPB][RT_CAP];
    __shared__ int s_nx[TPB], s_ex[TPB];
    __shared__ int s_idx[TPB][K3_MAX_TOPK];
    __shared__ float s_w[TPB][K3_MAX_TOPK];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t0 = blockIdx.x * TPB;
    const int nt = ntok - t0 < TPB ? ntok - t0 : TPB;
    grid_dep_wait();   // the logit chunks come from the partial kernel
    if (fix.x) {   // the tokens' residual lists, for the tensor-core logits
        for (int i = threadIdx.x; i < nt; i += blockDim.x) {
            s_nx[i] = fix.xcnt[t0 + i];
            s_ex[i] = fix.xexp[t0 + i];
        }
        __syncthreads();
        for (int i = threadIdx.x; i < nt * RT_CAP; i += blockDim.x) {
            const int tt = i / RT_CAP, k = i % RT_CAP;
            if (k < s_nx[tt] && k < fix.cap) {
                s_xk[tt][k] = fix.xk[(size_t)(t0 + tt) * fix.cap + k];
                s_xr[tt][k] = fix.xr[(size_t)(t0 + tt) * fix.cap + k];
            }
        }
        __syncthreads();
    }
    // RU items per thread per pass, KL chunk loads of each in flight: the tensor-core logits
    // (one or a few K slices, residual gathers) interleave four items; the CUDA-core logits
    // (dozens of K chunks) keep sixteen chunk loads of one item in flight.
    auto logits = [&](auto ru, auto kl) {
        constexpr int RU = decltype(ru)::value, KL = decltype(kl)::value;
        const int nitems = nt * n_experts;
        for (int i0 = threadIdx.x; i0 < nitems; i0 += blockDim.x * RU) {
            bool ok[RU];
            int tt[RU], e[RU], t[RU];
#pragma unroll
            for (int u = 0; u < RU; u++) {
                const int i = i0 + u * (int)blockDim.x;
                ok[u] = i < nitems;
                tt[u] = ok[u] ? i / n_experts : 0;
                e[u] = ok[u] ? i % n_experts : 0;
                t[u] = t0 + tt[u];
            }
            float v[RU];
            if (part) {
                // chunks in order, KL loads of each item in flight per pass
                double lg[RU];
#pragma unroll
                for (int u = 0; u < RU; u++) lg[u] = 0.0;
                for (int k0 = 0; k0 < nchunk; k0 += KL) {
                    double vk[RU][KL];
#pragma unroll
                    for (int u = 0; u < RU; u++)
#pragma unroll
                        for (int k = 0; k < KL; k++)
                            vk[u][k] = ok[u] && k0 + k < nchunk
                                           ? part[((size_t)(k0 + k) * ntok + t[u]) * n_experts + e[u]] : 0.0;
#pragma unroll
                    for (int u = 0; u < RU; u++)
#pragma unroll
                        for (int k = 0; k < KL; k++)
                            if (k0 + k < nchunk) lg[u] += vk[u][k];
                }
                if (fix.x) rt_finish<RU>(fix, lg, ok, tt, t, e, s_nx, s_ex, s_xk, s_xr, n_experts);
#pragma unroll
                for (int u = 0; u < RU; u++) {
                    v[u] = sigmoid_score(lg[u]);
                    if (ok[u] && scores) scores[(size_t)t[u] * n_experts + e[u]] = v[u];
                }
            } else {
#pragma unroll
                for (int u = 0; u < RU; u++) v[u] = ok[u] ? scores[(size_t)t[u] * n_experts + e[u]] : 0.0f;
            }
#pragma unroll
            for (int u = 0; u < RU; u++) {
                if (!ok[u]) continue;
                ch[(size_t)(2 * tt[u] + 1) * n_experts + e[u]] = v[u];
                ch[(size_t)(2 * tt[u]) * n_experts + e[u]] = __fadd_rn(v[u], bias ? bias[e[u]] : 0.0f);
            }
        }
    };
    if (nchunk > 4) logits(std::integral_constant<int, 1>{}, std::integral_constant<int, 16>{});
    else logits(std::integral_constant<int, 4>{}, std::integral_constant<int, 4>{});
    __syncthreads();
    if (warp >= nt) return;
    const int t = t0 + warp;
    float *c = ch + (size_t)(2 * warp) * n_experts;
    const float *sc = c + n_experts;
    int *sidx = s_idx[warp];
    float *sw = s_w[warp];
    // warp argmax of (value, index) pairs: largest value, lowest index on ties, -1 if none
    auto warp_best = [&](float bv, int bi) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (oi >= 0 && (bi < 0 || ov > bv || (ov == bv && oi < bi))) { bv = ov; bi = oi; }
        }
        return bi;
    };
    constexpr int RMAX = 16;   // candidates per lane held in registers (n_experts <= 512)
    if (n_experts <= 32 * RMAX) {
        float v[RMAX];
#pragma unroll
        for (int j = 0; j < RMAX; j++) v[j] = lane + 32 * j < n_experts ? c[lane + 32 * j] : -INFINITY;
        for (int j = 0; j < topk; j++) {
            float bv = -INFINITY;
            int bj = -1;
#pragma unroll
            for (int q = 0; q < RMAX; q++)
                if (v[q] > bv) { bv = v[q]; bj = q; }   // ascending e per lane: first index wins
            const int bi = warp_best(bv, bj >= 0 ? lane + 32 * bj : -1);
            if (bi >= 0 && (bi & 31) == lane) {
#pragma unroll
                for (int q = 0; q < RMAX; q++)
                    if (q == (bi >> 5)) v[q] = -INFINITY;
            }
            if (lane == 0) {
                sidx[j] = bi < 0 ? 0 : bi;
                sw[j] = bi < 0 ? 0.0f : sc[bi];
            }
        }
    } else {
        for (int j = 0; j < topk; j++) {
            float bv = -INFINITY;
            int bi = -1;
            for (int e = lane; e < n_experts; e += 32) {
                const float v = c[e];
                if (v > bv) { bv = v; bi = e; }  // ascending e per lane: first index wins
            }
            bi = warp_best(bv, bi);
            if (lane == 0) {
                if (bi < 0) { sidx[j] = 0; sw[j] = 0.0f; }
                else { sidx[j] = bi; sw[j] = sc[bi]; c[bi] = -INFINITY; }
            }
            __syncwarp();
        }
    }
    __syncwarp();
    if (lane == 0) {
        if (renorm && topk > 1) {
            double sum = 0.0;
            for (int j = 0; j < topk; j++) sum += (double)sw[j];
            const float inv = (float)(1.0 / (sum + 1e-20));
            for (int j = 0; j < topk; j++) sw[j] = __fmul_rn(sw[j], inv);
        }
        for (int j = 0; j < topk; j++) sw[j] = __fmul_rn(sw[j], routed_scale);
    }
    __syncwarp();
    for (int j = lane; j < topk; j += 32) {
        idx[(size_t)t * topk + j] = sidx[j];
        w[(size_t)t * topk + j] = sw[j];
    }
}

static int sm_count_rt() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
    }
    return n;
}

static int launch_select(int *idx, float *w, float *scores, const double *part, int nchunk,
                         const float *bias, int n_experts, int topk, int renorm, float routed_scale,
                         int ntok, cudaStream_t s, RtFix fix = RtFix{}) {
    if (n_experts <= 0 || topk <= 0 || topk > K3_MAX_TOPK || ntok < 0)
        return set_error(K3C_EINVAL, "router_select: n_experts=%d topk=%d ntok=%d", n_experts,
                         topk, ntok);
    if (ntok == 0) return K3C_OK;
    const size_t smem1 = (size_t)2 * n_experts * sizeof(float);
    if (smem1 > 200 * 1024) return set_error(K3C_EINVAL, "router_select: n_experts=%d too large", n_experts);
    // Tokens per block (the top-k of each runs in its own warp): the most that still gives every
    // SM about six blocks, so that the logit phase's loads from many blocks overlap.
    auto go = [&](auto kern, int tpb) -> int {
        const size_t smem = (size_t)tpb * smem1;
        if (smem > 48 * 1024)
            K3C_TRY_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        count_launch();
        K3C_TRY_CUDA(launch_pdl(kern, dim3((ntok + tpb - 1) / tpb), dim3(256), smem, s, idx, w, scores, part,
                                nchunk, bias, n_experts, topk, renorm, routed_scale, ntok, fix));
        return K3C_OK;
    };
    const long want = 6L * sm_count_rt();
    if (ntok >= 8 * want && 8 * smem1 <= 200 * 1024) return go(k_router_select<8>, 8);
    if (ntok >= 4 * want && 4 * smem1 <= 200 * 1024) return go(k_router_select<4>, 4);
    if (ntok >= 2 * want && 2 * smem1 <= 200 * 1024) return go(k_router_select<2>, 2);
    return go(k_router_select<1>, 1);
}

int launch_router_select(int *idx, float *w, const float *scores, const float *bias,
                         int n_experts, int topk, int renorm, float routed_scale, int ntok,
                         cudaStream_t s) {
    return launch_select(idx, w, const_cast<float *>(scores), nullptr, 0, bias, n_experts, topk, renorm,
                         routed_scale, ntok, s);
}

static int router_nparts(int hidden, int n_experts, int ntok);

// Enough for either logit path (the operand dtypes are not known here).
size_t router_scratch_bytes(int hidden, int n_experts, int ntok) {
    size_t b = (size_t)router_nparts(hidden, n_experts, ntok) * ntok * n_experts * sizeof(double);
    if (router_tc_applies(K3C_BF16, K3C_BF16, hidden, ntok)) {
        const size_t t = router_tc_scratch_bytes(hidden, n_experts, ntok);
        if (t > b) b = t;
    }
    return b;
}

// Experts per lane: two for many tokens (the grid has blocks to spare and the FP64 pipe, not
// shared memory, should be the limit), one for small batches (twice the blocks fill the SMs).
static int router_ept(int ntok) { return ntok >= 64 ? 2 : 1; }

// K chunks per block: 1 (most parallel) unless the grid would exceed about three waves,
// in which case blocks take several chunks and the partial array shrinks accordingly.
static int router_cpb(int hidden, int n_experts, int ntok) {
    const int nchunk = (hidden + RT_KC - 1) / RT_KC;
    const int ew = 32 * router_ept(ntok);
    const long long blocks = (long long)((n_experts + ew - 1) / ew) * nchunk * ((ntok + 15) / 16);
    const long long cap = 3LL * 3 * sm_count_rt();
    int cpb = (int)((blocks + cap - 1) / cap);
    return cpb < 1 ? 1 : (cpb > nchunk ? nchunk : cpb);
}
static int router_nparts(int hidden, int n_experts, int ntok) {
    const int nchunk = (hidden + RT_KC - 1) / RT_KC, cpb = router_cpb(hidden, n_experts, ntok);
    return (nchunk + cpb - 1) / cpb;
}

template <typename WT, typename XT, int NT, int EPT>
static int launch_partial_ept(double *part, const void *x, const void *W, int hidden, int n_experts, int ntok,
                              int vec_w, int vec_x, cudaStream_t s) {
    const int smem = (RT_KC * NT + 8 * NT * 32 * EPT) * (int)sizeof(double);
    auto kern = k_router_partial<WT, XT, NT, EPT>;
    if (smem > 48 * 1024)
        K3C_TRY_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    const int cpb = router_cpb(hidden, n_experts, ntok);
    const dim3 grid((n_experts + 32 * EPT - 1) / (32 * EPT), router_nparts(hidden, n_experts, ntok),
                    (ntok + NT - 1) / NT);
    count_launch();
    K3C_TRY_CUDA(launch_pdl(kern, grid, dim3(256), smem, s, part, (const XT *)x, (const WT *)W, hidden, n_experts,
                            ntok, vec_w, vec_x, cpb));
    return K3C_OK;
}

template <typename WT, typename XT, int NT>
static int launch_partial_nt(double *part, const void *x, const void *W, int hidden, int n_experts, int ntok,
                             int vec_w, int vec_x, cudaStream_t s) {
    if constexpr (NT == 16)
        if (router_ept(ntok) == 2)
            return launch_partial_ept<WT, XT, NT, 2>(part, x, W, hidden, n_experts, ntok, vec_w, vec_x, s);
    return launch_partial_ept<WT, XT, NT, 1>(part, x, W, hidden, n_experts, ntok, vec_w, vec_x, s);
}

template <typename WT, typename XT>
static int launch_partial_t(double *part, const void *x, const void *W, int hidden, int n_experts, int ntok,
                            cudaStream_t s) {
    const int vec_w = ((uintptr_t)W % 16 == 0) && ((hidden * (int)sizeof(WT)) % 16 == 0);
    const int vec_x = ((uintptr_t)x % 16 == 0) && ((hidden * (int)sizeof(XT)) % 16 == 0);
    if (ntok <= 1) return launch_partial_nt<WT, XT, 1>(part, x, W, hidden, n_experts, ntok, vec_w, vec_x, s);
    if (ntok <= 2) return launch_partial_nt<WT, XT, 2>(part, x, W, hidden, n_experts, ntok, vec_w, vec_x, s);
    if (ntok <= 4) return launch_partial_nt<WT, XT, 4>(part, x, W, hidden, n_experts, ntok, vec_w, vec_x, s);
    if (ntok <= 8) return launch_partial_nt<WT, XT, 8>(part, x, W, hidden, n_experts, ntok, vec_w, vec_x, s);
    return launch_partial_nt<WT, XT, 16>(part, x, W, hidden, n_experts, ntok, vec_w, vec_x, s);
}

int launch_router(int *idx, float *w, float *scores, const void *x, int x_dtype, const void *W, int w_dtype,
                  const float *bias, int hidden, int n_experts, int topk, int renorm, float routed_scale,
                  int ntok, double *part, cudaStream_t s) {
    if (hidden <= 0 || n_experts <= 0) return set_error(K3C_EINVAL, "router: hidden=%d n_experts=%d", hidden, n_experts);
    if (ntok == 0) return K3C_OK;
    int rc;
    if (router_tc_applies(x_dtype, w_dtype, hidden, ntok) && ((uintptr_t)x % 16) == 0 && ((uintptr_t)W % 16) == 0) {
        RtFix fix;
        double *tpart = nullptr;
        int S = 1;
        K3C_TRY(launch_router_tc(&fix, &tpart, &S, x, W, hidden, n_experts, ntok, part, s));
        K3C_TRY(launch_select(idx, w, scores, tpart, S, bias, n_experts, topk, renorm, routed_scale, ntok, s, fix));
        static const int sync_check = getenv("K3C_SYNC_CHECK") ? 1 : 0;
        return sync_check ? router_tc_check(s) : K3C_OK;
    }
    if (w_dtype == K3C_BF16 && x_dtype == K3C_BF16) rc = launch_partial_t<uint16_t, uint16_t>(part, x, W, hidden, n_experts, ntok, s);
    else if (w_dtype == K3C_BF16 && x_dtype == K3C_F32) rc = launch_partial_t<uint16_t, float>(part, x, W, hidden, n_experts, ntok, s);
    else if (w_dtype == K3C_F32 && x_dtype == K3C_BF16) rc = launch_partial_t<float, uint16_t>(part, x, W, hidden, n_experts, ntok, s);
    else if (w_dtype == K3C_F32 && x_dtype == K3C_F32) rc = launch_partial_t<float, float>(part, x, W, hidden, n_experts, ntok, s);
    else return set_error(K3C_EINVAL, "router: dtypes x=%d W=%d", x_dtype, w_dtype);
    if (rc) return rc;
    return launch_select(idx, w, scores, part, router_nparts(hidden, n_experts, ntok), bias, n_experts, topk, renorm,
                         routed_scale, ntok, s);
}

}  // namespace k3c

namespace k3c {
// The draft model's cache-only routing (src/core/k3_ops.c:580-593), one warp per token (lane
// 0 works, in top-k order): keep the entries whose expert has a run (run_of[e] in [0, n_runs),
// the test the expert kernels apply), divide their weights by the float sum of the kept
// weights when it is positive, and empty the remaining entries (expert -1, weight 0).
__global__ void __launch_bounds__(128) k_route_cache_only(int *__restrict__ idx, float *__restrict__ wt, int ntok,
                                                          int topk, const int *__restrict__ run_of, int n_experts,
                                                          int n_runs) {
    __shared__ int si[4][K3_MAX_TOPK];
    __shared__ float sw[4][K3_MAX_TOPK];
    const int wl = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = blockIdx.x * 4 + wl;
    if (t >= ntok || lane != 0) return;
    int *ti = idx + (size_t)t * topk;
    float *tw = wt + (size_t)t * topk;
    int m = 0;
    float wsum = 0.0f;
    for (int j = 0; j < topk; j++) {
        const int e = ti[j];
        const int r = e >= 0 && e < n_experts ? run_of[e] : -1;
        if (r >= 0 && r < n_runs) {
            si[wl][m] = e;
            sw[wl][m] = tw[j];
            wsum = __fadd_rn(wsum, tw[j]);
            m++;
        }
    }
    for (int j = 0; j < topk; j++) {
        ti[j] = j < m ? si[wl][j] : -1;
        tw[j] = j < m ? (wsum > 0.0f ? __fdiv_rn(sw[wl][j], wsum) : sw[wl][j]) : 0.0f;
    }
}

int launch_route_cache_only(int *idx, float *wt, int ntok, int topk, const int *run_of, int n_experts, int n_runs,
                            cudaStream_t s) {
    if (ntok < 0 || topk <= 0 || topk > K3_MAX_TOPK || n_experts <= 0 || n_runs < 0)
        return set_error(K3C_EINVAL, "route_cache_only: ntok=%d topk=%d n_experts=%d n_runs=%d", ntok, topk,
                         n_experts, n_runs);
    if (ntok == 0) return K3C_OK;
    if (!idx || !wt || !run_of) return set_error(K3C_EINVAL, "route_cache_only: null pointer");
    k_route_cache_only<<<(ntok + 3) / 4, 128, 0, s>>>(idx, wt, ntok, topk, run_of, n_experts, n_runs);
    K3C_CHECK_LAUNCH();
    return K3C_OK;
}
}  // namespace k3c

extern "C" int k3c_route_cache_only(int *idx, float *wt, int ntok, int topk, const int *run_of, int n_experts,
                                    int n_runs, k3c_stream_t stream) {
    k3c::clear_error();
    return k3c::launch_route_cache_only(idx, wt, ntok, topk, run_of, n_experts, n_runs, (cudaStream_t)stream);
}

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
    if (ntok <= 0 || hidden <= 0 || n_experts <= 0)
        return k3c::launch_router(idx, w, scores, x, x_dtype, W, w_dtype, bias, hidden, n_experts, topk, renorm,
                                  routed_scale, ntok, nullptr, s);
    double *part = nullptr;
    k3c::keep_async_pool();
    K3C_TRY_CUDA(cudaMallocAsync((void **)&part, k3c::router_scratch_bytes(hidden, n_experts, ntok), s));
    const int rc = k3c::launch_router(idx, w, scores, x, x_dtype, W, w_dtype, bias, hidden, n_experts, topk,
                                      renorm, routed_scale, ntok, part, s);
    cudaFreeAsync(part, s);
    return rc;
}

extern "C" size_t k3c_router_scratch(int hidden, int n_experts, int ntok) {
    if (hidden <= 0 || n_experts <= 0 || ntok <= 0) return 0;
    return k3c::router_scratch_bytes(hidden, n_experts, ntok) + 256;
}

extern "C" int k3c_router_ws(int *idx, float *w, float *scores, const void *x, int x_dtype, const void *W,
                             int w_dtype, const float *bias, int hidden, int n_experts, int topk, int renorm,
                             float routed_scale, int ntok, void *scratch, size_t scratch_bytes,
                             k3c_stream_t stream) {
    k3c::clear_error();
    cudaStream_t s = (cudaStream_t)stream;
    if (ntok <= 0 || hidden <= 0 || n_experts <= 0)
        return k3c::launch_router(idx, w, scores, x, x_dtype, W, w_dtype, bias, hidden, n_experts, topk, renorm,
                                  routed_scale, ntok, nullptr, s);
    const size_t need = k3c::router_scratch_bytes(hidden, n_experts, ntok);
    char *base = reinterpret_cast<char *>(((uintptr_t)scratch + 255) & ~(uintptr_t)255);
    if (!scratch || (size_t)(base - (char *)scratch) + need > scratch_bytes)
        return k3c::set_error(K3C_EINVAL, "router: scratch of %zu bytes, %zu needed", scratch_bytes, need + 256);
    k3c::stage_begin(k3c::STAGE_ROUTER, s);
    const int rc = k3c::launch_router(idx, w, scores, x, x_dtype, W, w_dtype, bias, hidden, n_experts, topk, renorm,
                                      routed_scale, ntok, reinterpret_cast<double *>(base), s);
    k3c::stage_end(k3c::STAGE_ROUTER, s);
    return rc;
}
