// moe.cu -- expert FFN and the non-latent MoE layer for decode-sized batches.
//
// Reference semantics (src/core/k3_ops.c:556-656, restated for the BASELINE shapes):
//   route each token on its full input; run each selected expert as gate/up GEMV, the
//   activation, and the down GEMV; accumulate acc += w_j * expert_j in float, in top-k
//   order, from zero; add the shared expert unweighted. A selected expert that is not
//   resident is skipped and counted as a drop (:616-626).
//
// Device schedule (one stream, no host round trip):
//   plan     group the (token, slot) pairs by expert, deterministically (pairs of one
//            expert keep token order), so each expert's weights stream from HBM once for
//            all of its tokens; the shared expert is one more slot holding every token.
//   gateup   per (slot, 8 rows): gate and up rows read once, SwiGLU/SiTU fused in the
//            epilogue; act[pair][inter] fp32.
//   down     per (slot, 16 rows): down rows read once; unweighted expert output written
//            to contrib[token][k][hidden] (k = topk for the shared expert).
//   combine  out[t] = sum_j w[t][j] * contrib[t][j] in j order (separately rounded multiply
//            and add, as the reference compiles with -ffp-contract=off) + contrib[t][topk].
#include <cuda_runtime.h>

#include "common.cuh"
#include "gemv_core.cuh"

namespace k3c {

int launch_router(int *idx, float *w, float *scores, const void *x, int x_dtype, const void *W, int w_dtype,
                  const float *bias, int hidden, int n_experts, int topk, int renorm, float routed_scale,
                  int ntok, double *part, cudaStream_t s);
size_t router_scratch_bytes(int hidden, int n_experts, int ntok);

struct Slot {
    K3ExpertQ q;
    int ntok;       // pairs in this slot
    int pair_base;  // first pair index
};

struct Plan {
    int *n_slots;     // [1]
    Slot *slots;      // [max_slots]
    int *pair_tok;    // [max_pairs]
    int *pair_k;      // [max_pairs]
    uint8_t *dropped; // [ntok*topk]
};

__device__ __forceinline__ float sigmoid_ref(float v) {
    return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-v)));
}

__device__ __forceinline__ float act_fn(float g, float u, int act) {
    if (act == K3C_ACT_SITU) {  // src/core/k3_ops.c:110-123, b1=4, b2=25
        const float a = __fmul_rn(__fmul_rn(4.0f, tanhf(__fdiv_rn(g, 4.0f))), sigmoid_ref(g));
        const float uu = __fmul_rn(25.0f, tanhf(__fdiv_rn(u, 25.0f)));
        return __fmul_rn(a, uu);
    }
    return __fmul_rn(__fmul_rn(g, sigmoid_ref(g)), u);  // silu(g) * u
}

// ------------------------------------------------------------------------- plan
// One block. Pairs (t, j) -> slot of expert idx[t][j]; rank within the slot = number of
// earlier pairs (row-major) with the same expert, so the layout is deterministic.
__global__ void __launch_bounds__(1024) k_moe_plan(Plan p, const int *__restrict__ idx, int ntok,
                                                   int topk, const K3ExpertQ *__restrict__ experts,
                                                   int n_experts, const K3ExpertQ *__restrict__ shared,
                                                   int *__restrict__ drops) {
    extern __shared__ int sm[];
    int *cnt = sm;                 // [n_experts]
    int *slot_of = sm + n_experts; // [n_experts]
    __shared__ int s_npairs;
    const int P = ntok * topk;
    for (int e = threadIdx.x; e < n_experts; e += blockDim.x) cnt[e] = 0;
    __syncthreads();
    for (int i = threadIdx.x; i < P; i += blockDim.x) {
        const int e = idx[i];
        const bool ok = e >= 0 && e < n_experts && experts[e].p1 != nullptr;
        p.dropped[i] = ok ? 0 : 1;
        if (ok) atomicAdd(&cnt[e], 1);
        else if (drops) atomicAdd(drops, 1);
    }
    __syncthreads();
    if (threadIdx.x == 0) {  // n_experts is small (hundreds); a serial scan is cheapest here
        int ns = 0, base = 0;
        for (int e = 0; e < n_experts; e++) {
            if (cnt[e] > 0) {
                slot_of[e] = ns;
                p.slots[ns].q = experts[e];
                p.slots[ns].ntok = cnt[e];
                p.slots[ns].pair_base = base;
                base += cnt[e];
                ns++;
            } else {
                slot_of[e] = -1;
            }
        }
        if (shared) {
            p.slots[ns].q = *shared;
            p.slots[ns].ntok = ntok;
            p.slots[ns].pair_base = base;
            ns++;
        }
        s_npairs = base;
        *p.n_slots = ns;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < P; i += blockDim.x) {
        if (p.dropped[i]) continue;
        const int e = idx[i];
        int rank = 0;
        for (int k = 0; k < i; k++) rank += (idx[k] == e && !p.dropped[k]);
        const int pos = p.slots[slot_of[e]].pair_base + rank;
        p.pair_tok[pos] = i / topk;
        p.pair_k[pos] = i % topk;
    }
    if (shared) {
        for (int t = threadIdx.x; t < ntok; t += blockDim.x) {
            p.pair_tok[s_npairs + t] = t;
            p.pair_k[s_npairs + t] = topk;
        }
    }
}

// ------------------------------------------------------- single expert (k3c_expert_ffn)
// gate/up + activation: grid ceil(inter/8), warp w takes gate row and up row r = 8*bx + w,
// CPL weight chunks per lane requested at once (the first ones before the activations are
// staged); the NT token rows sit in shared memory in the x_swz order. Dynamic shared memory:
// NT * hidden floats.
template <int NT, int CPL>
__global__ void __launch_bounds__(256) k_ffn_gateup(K3ExpertQ q, const float *__restrict__ x, int ntok,
                                                    int hidden, int inter, int act, float *__restrict__ actbuf) {
    extern __shared__ __align__(16) float ffn_sx[];
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");   // the down kernel may start fetching
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r = blockIdx.x * 8 + warp;
    const bool live = r < inter;
    const size_t pitch = (size_t)hidden / 2, spitch = (size_t)hidden / 32;
    const int nchunk = hidden / 32;
    const uint8_t *prow[2] = {q.p1 + (size_t)(live ? r : 0) * pitch, q.p3 + (size_t)(live ? r : 0) * pitch};
    const uint8_t *srow[2] = {q.s1 + (size_t)(live ? r : 0) * spitch, q.s3 + (size_t)(live ? r : 0) * spitch};
    MxChunks<2, CPL> ch;
    if (live) ch.load(prow, srow, 0, nchunk);
    for (int t0 = 0; t0 < ntok; t0 += NT) {
        const int nt = ntok - t0 < NT ? ntok - t0 : NT;
        if (t0) __syncthreads();                  // every warp is done with the previous rows
        for (int t = 0; t < nt; t++) stage_x_swz(ffn_sx + t * hidden, x + (size_t)(t0 + t) * hidden, hidden);
        __syncthreads();
        float acc[2][NT];
#pragma unroll
        for (int i = 0; i < 2; i++)
#pragma unroll
            for (int t = 0; t < NT; t++) acc[i][t] = 0.f;
        for (int c0 = 0; c0 < nchunk; c0 += 32 * CPL) {
            if (!live) break;
            if (c0 > 0 || t0 > 0) ch.load(prow, srow, c0, nchunk);
            ch.template fma_smem<NT>(ffn_sx, hidden, nt, c0, nchunk, acc);
        }
#pragma unroll
        for (int t = 0; t < NT; t++) {
            const float g = warp_sum(acc[0][t]);
            const float u = warp_sum(acc[1][t]);
            if (live && lane == 0 && t < nt) actbuf[(size_t)(t0 + t) * inter + r] = act_fn(g, u, act);
        }
    }
}

// down: grid ceil(hidden/32), warp w takes rows 4*(8*bx+w)+{0..3} (one wave of blocks on
// 148 SMs at hidden 7168). Launched as a programmatic dependent of k_ffn_gateup: the first
// weight chunks are requested before the wait for the activations, which are then staged
// like k_ffn_gateup's (NT * inter floats).
template <int NT, int CPL>
__global__ void __launch_bounds__(256) k_ffn_down(K3ExpertQ q, const float *__restrict__ actbuf, int ntok,
                                                  int hidden, int inter, float *__restrict__ y) {
    extern __shared__ __align__(16) float ffn_sa[];
    constexpr int RD = 4;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rb = (blockIdx.x * 8 + warp) * RD;
    const bool live = rb < hidden;
    const size_t pitch = (size_t)inter / 2, spitch = (size_t)inter / 32;
    const int nchunk = inter / 32;
    const uint8_t *prow[RD], *srow[RD];
#pragma unroll
    for (int i = 0; i < RD; i++) {
        const int r = live && rb + i < hidden ? rb + i : 0;
        prow[i] = q.p2 + (size_t)r * pitch;
        srow[i] = q.s2 + (size_t)r * spitch;
    }
    MxChunks<RD, CPL> ch;
    if (live) ch.load(prow, srow, 0, nchunk);
    asm volatile("griddepcontrol.wait;" ::: "memory");   // actbuf is complete
    for (int t0 = 0; t0 < ntok; t0 += NT) {
        const int nt = ntok - t0 < NT ? ntok - t0 : NT;
        if (t0) __syncthreads();
        for (int t = 0; t < nt; t++) stage_x_swz(ffn_sa + t * inter, actbuf + (size_t)(t0 + t) * inter, inter);
        __syncthreads();
        float acc[RD][NT];
#pragma unroll
        for (int i = 0; i < RD; i++)
#pragma unroll
            for (int t = 0; t < NT; t++) acc[i][t] = 0.f;
        for (int c0 = 0; c0 < nchunk; c0 += 32 * CPL) {
            if (!live) break;
            if (c0 > 0 || t0 > 0) ch.load(prow, srow, c0, nchunk);
            ch.template fma_smem<NT>(ffn_sa, inter, nt, c0, nchunk, acc);
        }
#pragma unroll
        for (int t = 0; t < NT; t++) {
#pragma unroll
            for (int i = 0; i < RD; i++) {
                const float v = warp_sum(acc[i][t]);
                if (live && lane == 0 && t < nt && rb + i < hidden) y[(size_t)(t0 + t) * hidden + rb + i] = v;
            }
        }
    }
}

template <int NT>
static int launch_ffn_pair(const K3ExpertQ &e, const float *x, int ntok, int hidden, int inter, int act,
                           float *actbuf, float *y, cudaStream_t s) {
    constexpr int CG = NT == 1 ? 8 : 4;
    const size_t sg = (size_t)NT * hidden * sizeof(float), sd = (size_t)NT * inter * sizeof(float);
    static bool attr_of[64] = {};
    bool &attr = attr_of[cur_dev()];
    if (!attr) {
        K3C_TRY_CUDA(cudaFuncSetAttribute(k_ffn_gateup<NT, CG>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
        K3C_TRY_CUDA(cudaFuncSetAttribute(k_ffn_down<NT, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
        attr = true;
    }
    k_ffn_gateup<NT, CG><<<(inter + 7) / 8, 256, sg, s>>>(e, x, ntok, hidden, inter, act, actbuf);
    K3C_CHECK_LAUNCH();
    K3C_TRY_CUDA(launch_pdl(k_ffn_down<NT, 2>, dim3((hidden + 31) / 32), dim3(256), sd, s, e, (const float *)actbuf,
                            ntok, hidden, inter, y));
    count_launch();
    return K3C_OK;
}

// ---------------------------------------------------------------- gate/up + act
// grid (inter/8, max_slots): warp w computes gate row r and up row r (r = 8*bx + w) for all
// tokens of the slot, NT at a time.
template <int NT>
__global__ void __launch_bounds__(256) k_moe_gateup(Plan p, const float *__restrict__ xf,
                                                    int hidden, int inter, int act,
                                                    float *__restrict__ actbuf) {
    const int s = blockIdx.y;
    if (s >= *p.n_slots) return;
    const Slot sl = p.slots[s];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r = blockIdx.x * 8 + warp;
    if (r >= inter) return;
    const size_t pitch = (size_t)hidden / 2, spitch = (size_t)hidden / 32;
    const uint8_t *prow[2] = {sl.q.p1 + r * pitch, sl.q.p3 + r * pitch};
    const uint8_t *srow[2] = {sl.q.s1 + r * spitch, sl.q.s3 + r * spitch};
    for (int t0 = 0; t0 < sl.ntok; t0 += NT) {
        const int nt = sl.ntok - t0 < NT ? sl.ntok - t0 : NT;
        const float *xrow[NT];
#pragma unroll
        for (int t = 0; t < NT; t++)
            xrow[t] = xf + (size_t)p.pair_tok[sl.pair_base + t0 + (t < nt ? t : 0)] * hidden;
        float acc[2][NT];
        mx_dot_rows<2, NT>(prow, srow, xrow, nt, hidden / 32, acc);
#pragma unroll
        for (int t = 0; t < NT; t++) {
            const float g = warp_sum(acc[0][t]);
            const float u = warp_sum(acc[1][t]);
            if (lane == 0 && t < nt)
                actbuf[(size_t)(sl.pair_base + t0 + t) * inter + r] = act_fn(g, u, act);
        }
    }
}

// -------------------------------------------------------------------------- down
// grid (hidden/16, max_slots): warp w computes down rows 2*(8*bx+w)+{0,1}.
template <int NT>
__global__ void __launch_bounds__(256) k_moe_down(Plan p, const float *__restrict__ actbuf,
                                                  int hidden, int inter, int kstride,
                                                  float *__restrict__ contrib) {
    const int s = blockIdx.y;
    if (s >= *p.n_slots) return;
    const Slot sl = p.slots[s];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r0 = (blockIdx.x * 8 + warp) * 2;
    if (r0 >= hidden) return;
    const int r1 = r0 + 1 < hidden ? r0 + 1 : r0;
    const size_t pitch = (size_t)inter / 2, spitch = (size_t)inter / 32;
    const uint8_t *prow[2] = {sl.q.p2 + r0 * pitch, sl.q.p2 + r1 * pitch};
    const uint8_t *srow[2] = {sl.q.s2 + r0 * spitch, sl.q.s2 + r1 * spitch};
    for (int t0 = 0; t0 < sl.ntok; t0 += NT) {
        const int nt = sl.ntok - t0 < NT ? sl.ntok - t0 : NT;
        const float *xrow[NT];
#pragma unroll
        for (int t = 0; t < NT; t++)
            xrow[t] = actbuf + (size_t)(sl.pair_base + t0 + (t < nt ? t : 0)) * inter;
        float acc[2][NT];
        mx_dot_rows<2, NT>(prow, srow, xrow, nt, inter / 32, acc);
#pragma unroll
        for (int t = 0; t < NT; t++) {
            const float a0 = warp_sum(acc[0][t]);
            const float a1 = warp_sum(acc[1][t]);
            if (lane == 0 && t < nt) {
                const int pr = sl.pair_base + t0 + t;
                float *o = contrib + ((size_t)p.pair_tok[pr] * kstride + p.pair_k[pr]) * hidden;
                o[r0] = a0;
                if (r1 != r0) o[r1] = a1;
            }
        }
    }
}

// ----------------------------------------------------------------------- combine
// A pair is skipped when dropped[t*topk+j] is set (if given) or its id is outside
// [0, n_experts) (if ids is given).
__device__ __forceinline__ bool pair_skipped(const uint8_t *dropped, const int *ids, int n_experts, int i) {
    return (dropped && dropped[i]) || (ids && (unsigned)ids[i] >= (unsigned)n_experts);
}

__global__ void k_moe_combine(float *__restrict__ out, const float *__restrict__ contrib,
                              const float *__restrict__ wt, const uint8_t *__restrict__ dropped,
                              const int *__restrict__ ids, int n_experts,
                              int ntok, int topk, int hidden, int has_shared) {
    const int t = blockIdx.y;
    const int ks = topk + 1;
    for (int h = blockIdx.x * blockDim.x + threadIdx.x; h < hidden; h += gridDim.x * blockDim.x) {
        float acc = 0.0f;
        for (int j = 0; j < topk; j++) {
            if (pair_skipped(dropped, ids, n_experts, t * topk + j)) continue;
            acc = __fadd_rn(acc, __fmul_rn(wt[t * topk + j], contrib[((size_t)t * ks + j) * hidden + h]));
        }
        if (has_shared) acc = __fadd_rn(acc, contrib[((size_t)t * ks + topk) * hidden + h]);
        out[(size_t)t * hidden + h] = acc;
    }
}

// Four consecutive outputs per thread (hidden % 4 == 0, 16-byte aligned rows): the same
// per-element operations in the same order, with every one of a thread's topk+1 16-byte
// loads in flight at once.
__global__ void k_moe_combine4(float4 *__restrict__ out, const float4 *__restrict__ contrib,
                               const float *__restrict__ wt, const uint8_t *__restrict__ dropped,
                               const int *__restrict__ ids, int n_experts,
                               int ntok, int topk, int h4, int has_shared) {
    const int t = blockIdx.y;
    const int ks = topk + 1;
    const int h = blockIdx.x * blockDim.x + threadIdx.x;
    if (h >= h4) return;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    constexpr int JM = 8;                       // rows loaded ahead of their use
    for (int j0 = 0; j0 < topk; j0 += JM) {
        float4 cj[JM];
#pragma unroll
        for (int i = 0; i < JM; i++)
            if (j0 + i < topk) cj[i] = contrib[((size_t)t * ks + j0 + i) * h4 + h];
#pragma unroll
        for (int i = 0; i < JM; i++) {
            const int j = j0 + i;
            if (j >= topk || pair_skipped(dropped, ids, n_experts, t * topk + j)) continue;
            const float w = wt[t * topk + j];
            const float4 c = cj[i];
            acc.x = __fadd_rn(acc.x, __fmul_rn(w, c.x));
            acc.y = __fadd_rn(acc.y, __fmul_rn(w, c.y));
            acc.z = __fadd_rn(acc.z, __fmul_rn(w, c.z));
            acc.w = __fadd_rn(acc.w, __fmul_rn(w, c.w));
        }
    }
    if (has_shared) {
        const float4 c = contrib[((size_t)t * ks + topk) * h4 + h];
        acc.x = __fadd_rn(acc.x, c.x);
        acc.y = __fadd_rn(acc.y, c.y);
        acc.z = __fadd_rn(acc.z, c.z);
        acc.w = __fadd_rn(acc.w, c.w);
    }
    out[(size_t)t * h4 + h] = acc;
}

int launch_moe_combine_ids(float *out, const float *contrib, const float *wt, const uint8_t *dropped,
                           const int *ids, int n_experts, int ntok, int topk, int hidden, int has_shared,
                           cudaStream_t s) {
    if (ntok <= 0) return K3C_OK;
    if (hidden % 4 == 0 && ((uintptr_t)out & 15) == 0 && ((uintptr_t)contrib & 15) == 0) {
        const int h4 = hidden / 4;
        k_moe_combine4<<<dim3((h4 + 127) / 128, ntok), 128, 0, s>>>(
            reinterpret_cast<float4 *>(out), reinterpret_cast<const float4 *>(contrib), wt, dropped, ids, n_experts,
            ntok, topk, h4, has_shared);
    } else {
        k_moe_combine<<<dim3((hidden + 255) / 256, ntok), 256, 0, s>>>(out, contrib, wt, dropped, ids, n_experts,
                                                                      ntok, topk, hidden, has_shared);
    }
    K3C_CHECK_LAUNCH();
    return K3C_OK;
}

int launch_moe_combine(float *out, const float *contrib, const float *wt, const uint8_t *dropped,
                       int ntok, int topk, int hidden, int has_shared, cudaStream_t s) {
    return launch_moe_combine_ids(out, contrib, wt, dropped, nullptr, 0, ntok, topk, hidden, has_shared, s);
}

template <typename XT>
__global__ void k_to_f32(float *__restrict__ y, const XT *__restrict__ x, size_t n) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        if constexpr (sizeof(XT) == 2) y[i] = bf16_bits_to_f32(x[i]);
        else y[i] = x[i];
    }
}

// ------------------------------------------------------------------- launchers
static int check_dims(int hidden, int inter) {
    if (hidden <= 0 || inter <= 0 || hidden % 32 || inter % 32)
        return set_error(K3C_EINVAL, "moe: hidden=%d inter=%d must be positive multiples of 32", hidden, inter);
    return K3C_OK;
}

static int launch_ffn_kernels(const Plan &p, int max_slots, const float *xf, int hidden,
                              int inter, int act, float *actbuf, int kstride, float *contrib,
                              int max_tok_per_slot, cudaStream_t s) {
    dim3 ga((inter + 7) / 8, max_slots), gd((hidden + 15) / 16, max_slots);
    if (max_tok_per_slot <= 1) {
        k_moe_gateup<1><<<ga, 256, 0, s>>>(p, xf, hidden, inter, act, actbuf);
        K3C_CHECK_LAUNCH();
        k_moe_down<1><<<gd, 256, 0, s>>>(p, actbuf, hidden, inter, kstride, contrib);
    } else if (max_tok_per_slot <= 2) {
        k_moe_gateup<2><<<ga, 256, 0, s>>>(p, xf, hidden, inter, act, actbuf);
        K3C_CHECK_LAUNCH();
        k_moe_down<2><<<gd, 256, 0, s>>>(p, actbuf, hidden, inter, kstride, contrib);
    } else {
        k_moe_gateup<4><<<ga, 256, 0, s>>>(p, xf, hidden, inter, act, actbuf);
        K3C_CHECK_LAUNCH();
        k_moe_down<4><<<gd, 256, 0, s>>>(p, actbuf, hidden, inter, kstride, contrib);
    }
    K3C_CHECK_LAUNCH();
    return K3C_OK;
}

static bool carve_plan(Carve &cv, Plan &p, int max_slots, int max_pairs, int ntok_topk) {
    p.n_slots = cv.take<int>(1);
    p.slots = cv.take<Slot>(max_slots);
    p.pair_tok = cv.take<int>(max_pairs);
    p.pair_k = cv.take<int>(max_pairs);
    p.dropped = cv.take<uint8_t>(ntok_topk > 0 ? ntok_topk : 1);
    return p.n_slots && p.slots && p.pair_tok && p.pair_k && p.dropped;
}

// Sizing passes carve from a dummy non-null base: only the offsets matter.
static char *const kSizingBase = reinterpret_cast<char *>(4096);

size_t ffn_scratch(int ntok, int hidden, int inter) {
    Carve cv{kSizingBase, (size_t)-1 / 2, 0};
    cv.take<float>((size_t)(ntok > 0 ? ntok : 1) * inter);
    return cv.used + 256;
}

int launch_expert_ffn(float *y, const float *x, int ntok, const K3ExpertQ *e, int hidden,
                      int inter, int act, void *scratch, size_t scratch_bytes, cudaStream_t s) {
    K3C_TRY(check_dims(hidden, inter));
    if (!e || !e->p1 || !e->p2 || !e->p3) return set_error(K3C_EINVAL, "expert_ffn: null expert");
    if (ntok <= 0) return K3C_OK;
    if (((uintptr_t)x & 15) != 0) return set_error(K3C_EINVAL, "expert_ffn: x not 16-byte aligned");
    Carve cv{(char *)scratch, scratch_bytes, 0};
    float *actbuf = cv.take<float>((size_t)ntok * inter);
    if (!actbuf) return set_error(K3C_EINVAL, "expert_ffn: scratch too small (%zu)", scratch_bytes);
    if ((size_t)(hidden > inter ? hidden : inter) * 4 * 4 > 200 * 1024)
        return set_error(K3C_EINVAL, "expert_ffn: hidden=%d inter=%d too large (12800 at most)", hidden, inter);
    return ntok <= 1 ? launch_ffn_pair<1>(*e, x, ntok, hidden, inter, act, actbuf, y, s)
                     : launch_ffn_pair<4>(*e, x, ntok, hidden, inter, act, actbuf, y, s);
}

struct DecodeBufs {
    Plan p;
    float *xf, *wt, *actbuf, *contrib;
    int *idx;
};

static bool carve_decode(Carve &cv, DecodeBufs &b, const k3c_moe_layer *L, int ntok) {
    const int P = ntok * L->topk;
    const int max_slots = (P < L->n_experts ? P : L->n_experts) + 1;
    const int max_pairs = P + ntok;
    if (!carve_plan(cv, b.p, max_slots, max_pairs, P)) return false;
    b.xf = cv.take<float>((size_t)ntok * L->hidden);
    b.idx = cv.take<int>(P);
    b.wt = cv.take<float>(P);
    b.actbuf = cv.take<float>((size_t)max_pairs * L->inter);
    // contrib is first written by the down kernels, after routing: the router's logit
    // chunks share its space
    const size_t nc = (size_t)ntok * (L->topk + 1) * L->hidden;
    const size_t np = router_scratch_bytes(L->hidden, L->n_experts, ntok) / sizeof(float);
    b.contrib = cv.take<float>(nc > np ? nc : np);
    return b.xf && b.idx && b.wt && b.actbuf && b.contrib;
}

size_t moe_decode_scratch(const k3c_moe_layer *L, int ntok) {
    Carve cv{kSizingBase, (size_t)-1 / 2, 0};
    DecodeBufs b;
    carve_decode(cv, b, L, ntok);
    return cv.used + 256;
}

int launch_moe_decode(float *out, const void *x, int x_dtype, int ntok, const k3c_moe_layer *L,
                      int *idx_out, float *wt_out, int *drops, void *scratch,
                      size_t scratch_bytes, cudaStream_t s) {
    if (!L) return set_error(K3C_EINVAL, "moe_decode: null layer");
    K3C_TRY(check_dims(L->hidden, L->inter));
    if (L->n_experts <= 0 || L->topk <= 0 || L->topk > K3_MAX_TOPK || L->topk > L->n_experts)
        return set_error(K3C_EINVAL, "moe_decode: n_experts=%d topk=%d", L->n_experts, L->topk);
    if (!L->experts || !L->router_w) return set_error(K3C_EINVAL, "moe_decode: null experts/router");
    if (ntok <= 0) return K3C_OK;
    if (ntok * L->topk > 4096) return set_error(K3C_EINVAL, "moe_decode: ntok*topk=%d > 4096 (use prefill)", ntok * L->topk);
    if ((size_t)L->n_experts * 2 * sizeof(int) > 96 * 1024) return set_error(K3C_EINVAL, "moe_decode: n_experts too large");
    Carve cv{(char *)scratch, scratch_bytes, 0};
    DecodeBufs b;
    if (!carve_decode(cv, b, L, ntok)) return set_error(K3C_EINVAL, "moe_decode: scratch too small (%zu)", scratch_bytes);
    int *idx = idx_out ? idx_out : b.idx;
    float *wt = wt_out ? wt_out : b.wt;
    const size_t nx = (size_t)ntok * L->hidden;
    if (x_dtype == K3C_BF16) k_to_f32<uint16_t><<<(unsigned)((nx + 255) / 256 < 1184 ? (nx + 255) / 256 : 1184), 256, 0, s>>>(b.xf, (const uint16_t *)x, nx);
    else if (x_dtype == K3C_F32) k_to_f32<float><<<(unsigned)((nx + 255) / 256 < 1184 ? (nx + 255) / 256 : 1184), 256, 0, s>>>(b.xf, (const float *)x, nx);
    else return set_error(K3C_EINVAL, "moe_decode: x_dtype=%d", x_dtype);
    K3C_CHECK_LAUNCH();
    stage_begin(STAGE_ROUTER, s);
    K3C_TRY(launch_router(idx, wt, nullptr, x, x_dtype, L->router_w, L->router_dtype, L->router_bias, L->hidden,
                          L->n_experts, L->topk, L->renorm, L->routed_scale, ntok,
                          reinterpret_cast<double *>(b.contrib), s));
    stage_end(STAGE_ROUTER, s);
    const int P = ntok * L->topk;
    const int max_slots = (P < L->n_experts ? P : L->n_experts) + (L->shared ? 1 : 0);
    const size_t psmem = (size_t)L->n_experts * 2 * sizeof(int);
    if (psmem > 48 * 1024) K3C_TRY_CUDA(cudaFuncSetAttribute(k_moe_plan, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)psmem));
    k_moe_plan<<<1, 1024, psmem, s>>>(b.p, idx, ntok, L->topk, L->experts, L->n_experts, L->shared, drops);
    K3C_CHECK_LAUNCH();
    stage_begin(STAGE_EXPERTS, s);
    K3C_TRY(launch_ffn_kernels(b.p, max_slots, b.xf, L->hidden, L->inter, L->act, b.actbuf,
                               L->topk + 1, b.contrib, ntok, s));
    stage_end(STAGE_EXPERTS, s);
    k_moe_combine<<<dim3((L->hidden + 255) / 256, ntok), 256, 0, s>>>(out, b.contrib, wt, b.p.dropped, nullptr, 0,
                                                                       ntok, L->topk, L->hidden, L->shared ? 1 : 0);
    K3C_CHECK_LAUNCH();
    return K3C_OK;
}

}  // namespace k3c

extern "C" size_t k3c_expert_ffn_scratch(int ntok, int hidden, int inter) {
    return k3c::ffn_scratch(ntok, hidden, inter);
}

extern "C" int k3c_expert_ffn(float *y, const float *x, int ntok, const K3ExpertQ *e,
                              int hidden, int inter, int act, void *scratch,
                              size_t scratch_bytes, k3c_stream_t stream) {
    k3c::clear_error();
    k3c::stage_begin(k3c::STAGE_EXPERTS, (cudaStream_t)stream);
    int rc = k3c::launch_expert_ffn(y, x, ntok, e, hidden, inter, act, scratch, scratch_bytes,
                                    (cudaStream_t)stream);
    k3c::stage_end(k3c::STAGE_EXPERTS, (cudaStream_t)stream);
    return rc;
}

extern "C" size_t k3c_moe_decode_scratch(const k3c_moe_layer *L, int ntok) {
    return L ? k3c::moe_decode_scratch(L, ntok) : 0;
}

extern "C" int k3c_moe_decode(float *out, const void *x, int x_dtype, int ntok,
                              const k3c_moe_layer *L, int *idx, float *wt, int *drops,
                              void *scratch, size_t scratch_bytes, k3c_stream_t stream) {
    k3c::clear_error();
    return k3c::launch_moe_decode(out, x, x_dtype, ntok, L, idx, wt, drops, scratch,
                                  scratch_bytes, (cudaStream_t)stream);
}
