// latent.cu -- the K3 latent MoE layer (src/core/k3_ops.c:556-656) on the GPU, and the
// trunk matmuls it runs (k3_mmw, include/k3/k3.h:289-296: k3_matmul and k3_matmul_bf16,
// src/core/k3_ops.c:265-291 and 1091-1196).
//
// Trunk matmuls are bit-exact with the reference. The reference fixes the summation order
// of every output: element i of the first in - in%16 goes to double accumulator i%16 by a
// fused multiply-add in element order, the sixteen accumulators are combined as
// b_l = (a_l + a_{l+4}) + (a_{l+8} + a_{l+12}), l = 0..3, then (b0 + b1) + (b2 + b3), the
// in%16 tail is fused onto the total in element order and the result is rounded once to
// float. Here each output row belongs to 16 threads: thread l owns accumulator l and runs
// its chain over the row in element order (double FMAs, exact widening of the fp32 or bf16
// weight and the fp32 activation), and the row's threads combine the sixteen with width-16
// shuffles in the same tree. The activations of up to NT tokens are staged in shared
// memory as doubles, chunk by chunk, and every weight a thread loads is used for all of
// them.
//
// The layer: route on the full-width input (the router of router.cu); one trunk launch for
// z = down x and the shared expert's sh1 x, sh3 x (same input), then SiTU; the routed experts
// at the latent width through the tensor-core decode kernels with the routing given
// (moe_pool.cu; their weighted top-k-order sum is the aggregate); RMSNorm of the aggregate;
// one trunk launch for sdn = sh2 SiTU(...) and out = up aggregate; out += sdn, one float add
// per element. The shared branch depends only on x, so computing it early changes no bit of
// the result against the reference's order of steps.
#include <cuda_runtime.h>
#include <math.h>

#include <type_traits>

#include "common.cuh"

namespace k3c {

size_t mmw_tc_terms_bytes(int ntok, int in);
bool mmw_tc_applies(const void *W, int in);
int launch_mmw_tc_split(void *terms, const float *x, int ldx, int ntok, int in, cudaStream_t s);
int launch_mmw_tc_gemm(float *y, int ldy, const void *terms, int ntok, const void *W, int in, int out,
                       int accumulate, cudaStream_t s);
int launch_router(int *idx, float *w, float *scores, const void *x, int x_dtype, const void *W, int w_dtype,
                  const float *bias, int hidden, int n_experts, int topk, int renorm, float routed_scale,
                  int ntok, double *part, cudaStream_t s);
size_t router_scratch_bytes(int hidden, int n_experts, int ntok);
size_t moe_decode_tc_scratch(const k3c_moe_pool_layer *L, int ntok);
int launch_moe_decode_tc(float *out, const void *x, int x_dtype, int ntok, const k3c_moe_pool_layer *L,
                         int *idx_out, float *wt_out, int *drops, void *scratch, size_t scratch_bytes,
                         cudaStream_t s, bool routed);
size_t moe_prefill_tc_scratch(const k3c_moe_pool_layer *L, int T, bool own_contrib);
int launch_route_cache_only(int *idx, float *wt, int ntok, int topk, const int *run_of, int n_experts, int n_runs,
                            cudaStream_t s);
int launch_q8_gemv(float *y, int ldy, const void *x, int x_dtype, int ldx, int ntok, const int8_t *wq,
                   const float *wscale, int ldw, int in, int out, cudaStream_t s);
int launch_moe_prefill_tc(float *out, const void *x, int x_dtype, int T, const k3c_moe_pool_layer *L,
                          int *idx_out, float *wt_out, int *drops, void *scratch, size_t scratch_bytes,
                          cudaStream_t s, bool routed, const k3c_ep_peers *ep);

// ------------------------------------------------------------------ trunk matmul
// Pipeline: the activations of a chunk of KC elements (all tokens) sit in shared memory as
// doubles, two buffers, the next chunk's values held in registers while the current chunk
// runs; weights are loaded in blocks of 8 K-steps of 16 elements, the next block while the
// current one is multiplied (across chunk boundaries too). None of this changes the order
// in which any accumulator sees its elements.
constexpr int MW_THREADS = 256;
constexpr int MW_GROUPS = MW_THREADS / 16;   // 16-thread groups per block
constexpr int MW_UNROLL = 8;                 // K steps of 16 per weight block
constexpr int MW_UB = 16 * MW_UNROLL;        // elements per weight block
constexpr int MW_XBUF = 4096;                // doubles per activation buffer (two buffers)

// Each 16-thread group owns R rows and NTT of the NT tokens. From 16 tokens up the two
// groups of a warp share their rows and split the tokens (TS = 2), so an activation read
// from shared memory feeds R rows' FMAs in both halves of the warp; below that the two groups
// take different rows (TS = 1).
template <int NT>
struct MwCfg {
    static constexpr int TS = NT >= 16 ? 2 : 1;         // token split across a warp's groups
    static constexpr int NTT = NT / TS;                 // tokens per group
    static constexpr int R = NTT >= 16 ? 1 : 2;         // rows per group
    static constexpr int KC = MW_XBUF / NT;             // activation chunk (elements)
    static constexpr int ROWS = MW_GROUPS * R / TS;     // rows per block
    static constexpr int XPT = MW_XBUF / MW_THREADS;    // activations each thread stages per chunk
    static constexpr size_t SMEM = 2 * (size_t)MW_XBUF * sizeof(double);
    static_assert(KC % MW_UB == 0, "a chunk holds whole weight blocks");
};

template <bool BF16>
using mw_raw_t = typename std::conditional<BF16, unsigned short, float>::type;

template <bool BF16>
__device__ __forceinline__ mw_raw_t<BF16> mw_raw(const char *row, int i) {
    return __ldg(reinterpret_cast<const mw_raw_t<BF16> *>(row) + i);
}
template <bool BF16>
__device__ __forceinline__ double mw_wide(mw_raw_t<BF16> v) {
    if constexpr (BF16) return (double)__uint_as_float((uint32_t)v << 16);
    else return (double)v;
}

// One matrix of a launch: y[t*ldy + o] = sum_i W[o][i] x[t*ldx + i] (accumulate: y += that,
// one float addition) for o < out, t < ntok.
struct MwSeg {
    const float *x;
    const void *W;
    float *y;
    int ldx, ldy, in, out, accumulate, blocks;
};
constexpr int MW_MAXSEG = 3;
// Up to three matrices of the same weight type and token count run as one grid (blocks of
// segment 0 first): the blocks of several small launches fill the SMs' slots together
// instead of each launch ending in its own partial wave.
struct MwSegs {
    MwSeg s[MW_MAXSEG];
    int n;
};

// Each segment's products for t < ntok <= NT, in the reference's order (file comment).
template <int NT, bool BF16>
__global__ void __launch_bounds__(MW_THREADS, 2) k_mmw(const MwSegs segs, int ntok) {
    int blk = blockIdx.x;
    MwSeg sg = segs.s[0];
    if (segs.n > 1 && blk >= segs.s[0].blocks) {
        blk -= segs.s[0].blocks;
        sg = segs.s[1];
        if (segs.n > 2 && blk >= segs.s[1].blocks) {
            blk -= segs.s[1].blocks;
            sg = segs.s[2];
        }
    }
    const float *__restrict__ x = sg.x;
    const void *__restrict__ W = sg.W;
    float *__restrict__ y = sg.y;
    const int ldx = sg.ldx, ldy = sg.ldy, in = sg.in, out = sg.out, accumulate = sg.accumulate;
    using Cfg = MwCfg<NT>;
    using raw_t = mw_raw_t<BF16>;
    constexpr int R = Cfg::R, KC = Cfg::KC, NTT = Cfg::NTT;
    extern __shared__ double xs[];   // [2][NT][KC]
    const int l = threadIdx.x & 15, grp = threadIdx.x >> 4;
    const int row0 = blk * Cfg::ROWS + (Cfg::TS == 2 ? (grp >> 1) : grp) * R;
    const int tok0 = Cfg::TS == 2 ? (grp & 1) * NTT : 0;
    const char *wrow[R];
#pragma unroll
    for (int r = 0; r < R; r++) {
        const int o = row0 + r < out ? row0 + r : out - 1;   // rows past the end load row out-1
        wrow[r] = reinterpret_cast<const char *>(W) + (size_t)o * in * sizeof(raw_t);
    }
    double a[R][NTT];
#pragma unroll
    for (int r = 0; r < R; r++)
#pragma unroll
        for (int t = 0; t < NTT; t++) a[r][t] = 0.0;

    // this thread's share of a chunk: buffer element e = threadIdx.x + 256 j is (t, k) =
    // (e / KC, e % KC), the layout of the [NT][KC] buffer
    float xr[Cfg::XPT];
    auto fetch_x = [&](int kb, int kcn) {
#pragma unroll
        for (int j = 0; j < Cfg::XPT; j++) {
            const int e = threadIdx.x + MW_THREADS * j, t = e / KC, k = e - t * KC;
            xr[j] = (t < ntok && k < kcn) ? x[(size_t)t * ldx + kb + k] : 0.0f;
        }
    };
    auto store_x = [&](double *buf) {
#pragma unroll
        for (int j = 0; j < Cfg::XPT; j++) buf[threadIdx.x + MW_THREADS * j] = (double)xr[j];
    };
    auto load_block = [&](raw_t (&w)[MW_UNROLL][R], int kb) {
#pragma unroll
        for (int u = 0; u < MW_UNROLL; u++)
#pragma unroll
            for (int r = 0; r < R; r++) w[u][r] = mw_raw<BF16>(wrow[r], kb + 16 * u + l);
    };

    const int in16 = in & ~15;
    const int nchunk = (in16 + KC - 1) / KC;
    raw_t wc[MW_UNROLL][R];
    if (in16 > 0) {
        const int kc0 = in16 < KC ? in16 : KC;
        fetch_x(0, kc0);
        if (kc0 >= MW_UB) load_block(wc, 0);
        store_x(xs);
    }
    __syncthreads();
    for (int c = 0; c < nchunk; c++) {
        const int k0 = c * KC;
        const int kc = in16 - k0 < KC ? in16 - k0 : KC;
        const double *xb = xs + (c & 1) * MW_XBUF;
        const bool more = c + 1 < nchunk;
        const int k0n = k0 + KC;
        const int kcn = more ? (in16 - k0n < KC ? in16 - k0n : KC) : 0;
        if (more) fetch_x(k0n, kcn);   // consumed after this chunk's products
        const int nb = kc / MW_UB;
        for (int b = 0; b < nb; b++) {
            raw_t wn[MW_UNROLL][R];
            const bool next_here = b + 1 < nb;
            const bool next_there = !next_here && kcn >= MW_UB;
            if (next_here) load_block(wn, k0 + (b + 1) * MW_UB);
            else if (next_there) load_block(wn, k0n);
#pragma unroll
            for (int u = 0; u < MW_UNROLL; u++) {
                const int k = b * MW_UB + 16 * u + l;
                double wd[R];
#pragma unroll
                for (int r = 0; r < R; r++) wd[r] = mw_wide<BF16>(wc[u][r]);
#pragma unroll
                for (int t = 0; t < NTT; t++) {
                    const double xv = xb[(tok0 + t) * KC + k];
#pragma unroll
                    for (int r = 0; r < R; r++) a[r][t] = fma(wd[r], xv, a[r][t]);
                }
            }
            if (next_here || next_there) {
#pragma unroll
                for (int u = 0; u < MW_UNROLL; u++)
#pragma unroll
                    for (int r = 0; r < R; r++) wc[u][r] = wn[u][r];
            }
        }
        // the last chunk's K steps past its whole weight blocks
        for (int m = nb * MW_UB; m < kc; m += 16) {
            const int k = m + l;
            double wd[R];
#pragma unroll
            for (int r = 0; r < R; r++) wd[r] = mw_wide<BF16>(mw_raw<BF16>(wrow[r], k0 + k));
#pragma unroll
            for (int t = 0; t < NTT; t++) {
                const double xv = xb[(tok0 + t) * KC + k];
#pragma unroll
                for (int r = 0; r < R; r++) a[r][t] = fma(wd[r], xv, a[r][t]);
            }
        }
        // the other buffer was last read in chunk c-1, which every thread has left
        if (more) store_x(xs + ((c + 1) & 1) * MW_XBUF);
        __syncthreads();
    }
    // (a_l + a_{l+4}) + (a_{l+8} + a_{l+12}) at lanes 0..3, then (b0 + b1) + (b2 + b3) at lane 0
#pragma unroll
    for (int r = 0; r < R; r++) {
        const int o = row0 + r;
#pragma unroll
        for (int tt = 0; tt < NTT; tt++) {
            const int t = tok0 + tt;
            double v = a[r][tt];
            v += __shfl_down_sync(0xffffffffu, v, 4, 16);
            v += __shfl_down_sync(0xffffffffu, v, 8, 16);
            v += __shfl_down_sync(0xffffffffu, v, 1, 16);
            v += __shfl_down_sync(0xffffffffu, v, 2, 16);
            if (l == 0 && o < out && t < ntok) {
                const float *xt = x + (size_t)t * ldx;
                for (int i = in16; i < in; i++) v = fma(mw_wide<BF16>(mw_raw<BF16>(wrow[r], i)), (double)xt[i], v);
                const float f = __double2float_rn(v);
                float *dst = y + (size_t)t * ldy + o;
                *dst = accumulate ? __fadd_rn(*dst, f) : f;
            }
        }
    }
}

template <int NT, bool BF16>
static int launch_mmw_nt(MwSegs segs, int ntok, cudaStream_t s) {
    using Cfg = MwCfg<NT>;
    auto k = k_mmw<NT, BF16>;
    static bool attr_done[64] = {};
    const int dev = cur_dev();
    if (!attr_done[dev]) {
        K3C_TRY_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Cfg::SMEM));
        attr_done[dev] = true;
    }
    int grid = 0;
    for (int i = 0; i < segs.n; i++) {
        segs.s[i].blocks = (segs.s[i].out + Cfg::ROWS - 1) / Cfg::ROWS;
        grid += segs.s[i].blocks;
    }
    k<<<grid, MW_THREADS, Cfg::SMEM, s>>>(segs, ntok);
    K3C_CHECK_LAUNCH();
    return K3C_OK;
}

template <bool BF16>
static int launch_mmw_t(const MwSegs &segs, int ntok, cudaStream_t s) {
    if (ntok <= 1) return launch_mmw_nt<1, BF16>(segs, ntok, s);
    if (ntok <= 2) return launch_mmw_nt<2, BF16>(segs, ntok, s);
    if (ntok <= 4) return launch_mmw_nt<4, BF16>(segs, ntok, s);
    if (ntok <= 8) return launch_mmw_nt<8, BF16>(segs, ntok, s);
    if (ntok <= 16) return launch_mmw_nt<16, BF16>(segs, ntok, s);
    return launch_mmw_nt<32, BF16>(segs, ntok, s);
}

// Matrices with out == 0 are dropped; every other one is checked before anything launches.
static int launch_mmw_segs(const MwSeg *list, int n, int ntok, int wdt, cudaStream_t s) {
    if (ntok <= 0) return K3C_OK;
    if (ntok > 32) return set_error(K3C_EINVAL, "mmw: ntok=%d > 32", ntok);
    if (wdt != K3C_WBF16 && wdt != K3C_WF32)
        return set_error(K3C_EINVAL, "mmw: wdt=%d (int8 trunk rows run through k3c_q8_pack/k3c_q8_gemv)", wdt);
    MwSegs segs = {};
    for (int i = 0; i < n; i++) {
        const MwSeg &g = list[i];
        if (g.out <= 0) continue;
        if (g.in <= 0 || !g.y || !g.x || !g.W || g.ldy < g.out || g.ldx < g.in)
            return set_error(K3C_EINVAL, "mmw: bad arguments (in=%d out=%d ldx=%d ldy=%d)", g.in, g.out, g.ldx,
                             g.ldy);
        if (segs.n == MW_MAXSEG) return set_error(K3C_EINVAL, "mmw: more than %d matrices", MW_MAXSEG);
        segs.s[segs.n++] = g;
    }
    if (segs.n == 0) return K3C_OK;
    return wdt == K3C_WBF16 ? launch_mmw_t<true>(segs, ntok, s) : launch_mmw_t<false>(segs, ntok, s);
}

int launch_mmw(float *y, int ldy, const float *x, int ldx, int ntok, const void *W, int wdt, int in, int out,
               int accumulate, cudaStream_t s) {
    const MwSeg g = {x, W, y, ldx, ldy, in, out, accumulate, 0};
    return launch_mmw_segs(&g, 1, ntok, wdt, s);
}

// ------------------------------------------------------------------ RMSNorm, SiTU-GLU
// y[t] = w * x[t] * inv, inv = 1/sqrt(mean(x[t]^2) + eps) computed in double and rounded to
// float once (src/core/k3_ops.c:94-102). One block per token; the sum of squares is a block
// reduction in double (the reference sums in element order: the two totals agree to a few
// units of 2^-53 relative, which reaches the float inv only at a rounding boundary). y may
// alias x.
__global__ void __launch_bounds__(256) k_rmsnorm_rows(float *y, const float *x, const float *__restrict__ w,
                                                      int n, float eps) {
    __shared__ double part[8];
    const float *xt = x + (size_t)blockIdx.x * n;
    float *yt = y + (size_t)blockIdx.x * n;
    double ss = 0.0;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const double v = (double)xt[i];
        ss = __dadd_rn(ss, __dmul_rn(v, v));
    }
    ss = warp_sum_d(ss);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
    __syncthreads();
    double tot = 0.0;
#pragma unroll
    for (int i = 0; i < 8; i++) tot = __dadd_rn(tot, part[i]);
    const float inv = __double2float_rn(1.0 / sqrt(tot / (double)n + (double)eps));
    for (int i = threadIdx.x; i < n; i += blockDim.x) yt[i] = __fmul_rn(__fmul_rn(w[i], xt[i]), inv);
}

// y[t][i] = (b1 tanh(g/b1) sigmoid(g)) * (b2 tanh(u/b2)), g = gu[t][i], u = gu[t][n + i]
// (src/core/k3_ops.c:110-122; the sigmoid takes the uncapped gate).
__global__ void __launch_bounds__(256) k_situ_rows(float *__restrict__ y, const float *__restrict__ gu, int n,
                                                   float b1, float b2) {
    const float *g = gu + (size_t)blockIdx.y * 2 * n;
    float *yt = y + (size_t)blockIdx.y * n;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const float gv = g[i], uv = g[n + i];
        const float sg = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-gv)));
        const float a = __fmul_rn(__fmul_rn(b1, tanhf(__fdiv_rn(gv, b1))), sg);
        yt[i] = __fmul_rn(a, __fmul_rn(b2, tanhf(__fdiv_rn(uv, b2))));
    }
}

// The trunk matrices of one step: fp32 / bf16 through the batched k_mmw grid; int8 rows (the
// draft model) one k3c_q8_gemv each, W being the address of a host k3c_q8_mat.
static int trunk_segs(const MwSeg *list, int n, int ntok, int wdt, cudaStream_t s) {
    if (wdt != K3C_WI8) return launch_mmw_segs(list, n, ntok, wdt, s);
    for (int i = 0; i < n; i++) {
        const MwSeg &g = list[i];
        if (g.out <= 0) continue;
        const k3c_q8_mat *m = static_cast<const k3c_q8_mat *>(g.W);
        if (!m || !m->wq || !m->wscale || g.accumulate)
            return set_error(K3C_EINVAL, "moe_latent: int8 trunk matrix %d is not a k3c_q8_mat", i);
        K3C_TRY(launch_q8_gemv(g.y, g.ldy, g.x, K3C_F32, g.ldx, ntok, m->wq, m->wscale, m->ldw, g.in, g.out, s));
    }
    return K3C_OK;
}

// y[i] = y[i] + d[i] (one float addition each), n elements.
__global__ void __launch_bounds__(256) k_add_f32(float *__restrict__ y, const float *__restrict__ d, size_t n) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        y[i] = __fadd_rn(y[i], d[i]);
}

// ------------------------------------------------------------------ the layer
// Up to LAT_CHUNK tokens go through the decode kernels and one trunk launch per step; more
// tokens run the trunk matrices LAT_CHUNK tokens at a time and the routed experts through the
// prefill kernels (each expert read once for all of its tokens).
constexpr int LAT_CHUNK = 32;
// trunk launches of the many-token path: at 16 tokens the two 16-lane groups of a warp share
// two rows (each shared-memory read of an activation feeds two rows' FMAs); at 32 they take one
// row each. Re-reading the weights per launch costs far less than that difference.
constexpr int LAT_TRUNK_CHUNK = 16;
constexpr int LAT_MAX_TOKENS = 65535;
// bf16 trunk matrices for many tokens run on the tensor cores (trunk_tc.cu), this many tokens
// per pass (bounds the shared branch's scratch; each pass reads every trunk matrix once)
constexpr int LAT_TC_CHUNK = 2048;

struct LatentBufs {
    double *rpart;     // router logit chunks
    float *z;          // [ntok][latent]
    float *agg;        // [ntok][latent] weighted expert sum, then normalised
    float *sgu;        // [chunk][2*SI]
    float *sact;       // [chunk][SI]
    float *sdn;        // [ntok][hidden] shared expert output
    int *idx;          // [ntok][topk] when the caller passes none
    float *wt;
    void *tc;          // tensor-core decode scratch
    size_t tc_bytes;
    void *terms;       // bf16 activation terms of the tensor-core trunk (many tokens, bf16 trunk)
};

static bool carve_latent(Carve &cv, LatentBufs &b, const k3c_moe_latent_layer *L, int ntok) {
    const int SI = L->experts.inter * L->n_shared;
    const int Lw = L->experts.hidden;
    const bool tc_trunk = ntok > LAT_CHUNK && L->wdt == K3C_WBF16;
    const int C = tc_trunk ? (ntok < LAT_TC_CHUNK ? ntok : LAT_TC_CHUNK) : (ntok < LAT_CHUNK ? ntok : LAT_CHUNK);
    const int kmax = L->hidden > SI ? (L->hidden > Lw ? L->hidden : Lw) : (SI > Lw ? SI : Lw);
    b.rpart = cv.take<double>(router_scratch_bytes(L->hidden, L->experts.n_experts, ntok) / sizeof(double) + 1);
    b.z = cv.take<float>((size_t)ntok * Lw);
    b.agg = cv.take<float>((size_t)ntok * Lw);
    b.sgu = cv.take<float>((size_t)C * 2 * SI);
    b.sact = cv.take<float>((size_t)C * SI);
    b.sdn = cv.take<float>((size_t)ntok * L->hidden);
    b.idx = cv.take<int>((size_t)ntok * L->experts.topk);
    b.wt = cv.take<float>((size_t)ntok * L->experts.topk);
    b.tc_bytes = ntok <= LAT_CHUNK ? moe_decode_tc_scratch(&L->experts, ntok)
                                   : moe_prefill_tc_scratch(&L->experts, ntok, true);
    b.tc = cv.take<char>(b.tc_bytes, 1024);
    b.terms = tc_trunk ? cv.take<char>(mmw_tc_terms_bytes(C, kmax), 256) : nullptr;
    return b.rpart && b.z && b.agg && b.sgu && b.sact && b.sdn && b.idx && b.wt && b.tc && (b.terms || !tc_trunk);
}

static int check_latent(const k3c_moe_latent_layer *L, int ntok) {
    if (!L) return set_error(K3C_EINVAL, "moe_latent: null layer");
    const k3c_moe_pool_layer &X = L->experts;
    if (ntok > LAT_MAX_TOKENS) return set_error(K3C_EINVAL, "moe_latent: ntok=%d > %d", ntok, LAT_MAX_TOKENS);
    if (L->hidden <= 0 || X.hidden <= 0 || X.inter <= 0 || L->n_shared < 0)
        return set_error(K3C_EINVAL, "moe_latent: hidden=%d latent=%d inter=%d n_shared=%d", L->hidden, X.hidden,
                         X.inter, L->n_shared);
    if (L->wdt != K3C_WF32 && L->wdt != K3C_WBF16 && L->wdt != K3C_WI8)
        return set_error(K3C_EINVAL, "moe_latent: wdt=%d", L->wdt);
    if (!L->router_w || !L->down || !L->up || (L->n_shared > 0 && (!L->sh1 || !L->sh3 || !L->sh2)) ||
        (L->latent_norm_on && !L->latent_norm))
        return set_error(K3C_EINVAL, "moe_latent: missing weights");
    if (X.shared_run >= 0)
        return set_error(K3C_EINVAL, "moe_latent: the latent layer's shared expert is the full-width trunk MLP; "
                                     "experts.shared_run must be -1");
    // the expert kernels apply SiTU with the K3 constants
    if (X.act == K3C_ACT_SITU && (L->situ_b1 != 4.0f || L->situ_b2 != 25.0f))
        return set_error(K3C_EINVAL, "moe_latent: expert SiTU runs with b1=4, b2=25 (got %g, %g)",
                         (double)L->situ_b1, (double)L->situ_b2);
    return K3C_OK;
}

size_t moe_latent_scratch(const k3c_moe_latent_layer *L, int ntok) {
    Carve cv{reinterpret_cast<char *>(4096), (size_t)-1 / 2, 0};
    LatentBufs b;
    carve_latent(cv, b, L, ntok);
    return cv.used + 1024;
}

int launch_moe_latent(float *out, const float *x, int ntok, const k3c_moe_latent_layer *L, int *idx_out,
                      float *wt_out, int *drops, void *scratch, size_t scratch_bytes, cudaStream_t s,
                      bool routed = false) {
    K3C_TRY(check_latent(L, ntok));
    if (ntok <= 0) return K3C_OK;
    Carve cv{(char *)scratch, scratch_bytes, 0};
    LatentBufs b;
    if (!carve_latent(cv, b, L, ntok))
        return set_error(K3C_EINVAL, "moe_latent: scratch too small (%zu)", scratch_bytes);
    const k3c_moe_pool_layer &X = L->experts;
    const int H = L->hidden, Lw = X.hidden, SI = X.inter * L->n_shared, K = X.topk;
    if (routed && (!idx_out || !wt_out)) return set_error(K3C_EINVAL, "moe_latent_routed: null routing");
    int *idx = idx_out ? idx_out : b.idx;
    float *wt = wt_out ? wt_out : b.wt;
    if (!routed) {
        // 1. route on the full width
        stage_begin(STAGE_ROUTER, s);
        K3C_TRY(launch_router(idx, wt, nullptr, x, K3C_F32, L->router_w, K3C_F32, L->router_bias, H, X.n_experts,
                              K, X.renorm, X.routed_scale, ntok, b.rpart, s));
        if (L->cache_only) {
            // the draft model: keep the resident experts, renormalise, count no drops
            K3C_TRY(launch_route_cache_only(idx, wt, ntok, K, X.run_of, X.n_experts, X.n_runs, s));
            drops = nullptr;
        }
        stage_end(STAGE_ROUTER, s);
    }
    const bool sh = L->n_shared > 0;
    if (b.terms && mmw_tc_applies(L->down, H) && mmw_tc_applies(L->up, Lw) &&
        (!sh || (mmw_tc_applies(L->sh1, H) && mmw_tc_applies(L->sh3, H) && mmw_tc_applies(L->sh2, SI)))) {
        // many tokens, bf16 trunk: every trunk matrix on the tensor cores, LAT_TC_CHUNK tokens
        // per pass (the activations of a pass split once into their two bf16 terms and shared
        // by the matrices that read them: down, sh1 and sh3 read x)
        stage_begin(STAGE_Q8, s);
        for (int t0 = 0; t0 < ntok; t0 += LAT_TC_CHUNK) {
            const int c = ntok - t0 < LAT_TC_CHUNK ? ntok - t0 : LAT_TC_CHUNK;
            K3C_TRY(launch_mmw_tc_split(b.terms, x + (size_t)t0 * H, H, c, H, s));
            K3C_TRY(launch_mmw_tc_gemm(b.z + (size_t)t0 * Lw, Lw, b.terms, c, L->down, H, Lw, 0, s));
            if (sh) {
                K3C_TRY(launch_mmw_tc_gemm(b.sgu, 2 * SI, b.terms, c, L->sh1, H, SI, 0, s));
                K3C_TRY(launch_mmw_tc_gemm(b.sgu + SI, 2 * SI, b.terms, c, L->sh3, H, SI, 0, s));
                dim3 gs((SI + 255) / 256 < 148 ? (SI + 255) / 256 : 148, c);
                k_situ_rows<<<gs, 256, 0, s>>>(b.sact, b.sgu, SI, L->situ_b1, L->situ_b2);
                K3C_CHECK_LAUNCH();
                K3C_TRY(launch_mmw_tc_split(b.terms, b.sact, SI, c, SI, s));
                K3C_TRY(launch_mmw_tc_gemm(b.sdn + (size_t)t0 * H, H, b.terms, c, L->sh2, SI, H, 0, s));
            }
        }
        stage_end(STAGE_Q8, s);
        K3C_TRY(launch_moe_prefill_tc(b.agg, b.z, K3C_F32, ntok, &X, idx, wt, drops, b.tc, b.tc_bytes, s, true,
                                      nullptr));
        stage_begin(STAGE_Q8, s);
        if (L->latent_norm_on) {
            k_rmsnorm_rows<<<ntok, 256, 0, s>>>(b.agg, b.agg, L->latent_norm, Lw, L->rms_eps);
            K3C_CHECK_LAUNCH();
        }
        for (int t0 = 0; t0 < ntok; t0 += LAT_TC_CHUNK) {
            const int c = ntok - t0 < LAT_TC_CHUNK ? ntok - t0 : LAT_TC_CHUNK;
            K3C_TRY(launch_mmw_tc_split(b.terms, b.agg + (size_t)t0 * Lw, Lw, c, Lw, s));
            K3C_TRY(launch_mmw_tc_gemm(out + (size_t)t0 * H, H, b.terms, c, L->up, Lw, H, 0, s));
        }
        if (sh) {
            const size_t n = (size_t)ntok * H;
            k_add_f32<<<(unsigned)((n + 255) / 256 < 1184 ? (n + 255) / 256 : 1184), 256, 0, s>>>(out, b.sdn, n);
            K3C_CHECK_LAUNCH();
        }
        stage_end(STAGE_Q8, s);
        return K3C_OK;
    }
    if (ntok > LAT_CHUNK) {
        // the same steps for many tokens: trunk matrices (and the shared branch) 16 tokens at
        // a time, the routed experts through the prefill kernels
        stage_begin(STAGE_Q8, s);
        for (int t0 = 0; t0 < ntok; t0 += LAT_TRUNK_CHUNK) {
            const int c = ntok - t0 < LAT_TRUNK_CHUNK ? ntok - t0 : LAT_TRUNK_CHUNK;
            const float *xc = x + (size_t)t0 * H;
            const MwSeg first[3] = {{xc, L->down, b.z + (size_t)t0 * Lw, H, Lw, H, Lw, 0, 0},
                                    {xc, L->sh1, b.sgu, H, 2 * SI, H, sh ? SI : 0, 0, 0},
                                    {xc, L->sh3, b.sgu + SI, H, 2 * SI, H, sh ? SI : 0, 0, 0}};
            K3C_TRY(trunk_segs(first, 3, c, L->wdt, s));
            if (sh) {
                dim3 gs((SI + 255) / 256 < 148 ? (SI + 255) / 256 : 148, c);
                k_situ_rows<<<gs, 256, 0, s>>>(b.sact, b.sgu, SI, L->situ_b1, L->situ_b2);
                K3C_CHECK_LAUNCH();
                const MwSeg down2 = {b.sact, L->sh2, b.sdn + (size_t)t0 * H, SI, H, SI, H, 0, 0};
                K3C_TRY(trunk_segs(&down2, 1, c, L->wdt, s));
            }
        }
        stage_end(STAGE_Q8, s);
        K3C_TRY(launch_moe_prefill_tc(b.agg, b.z, K3C_F32, ntok, &X, idx, wt, drops, b.tc, b.tc_bytes, s, true,
                                      nullptr));
        stage_begin(STAGE_Q8, s);
        if (L->latent_norm_on) {
            k_rmsnorm_rows<<<ntok, 256, 0, s>>>(b.agg, b.agg, L->latent_norm, Lw, L->rms_eps);
            K3C_CHECK_LAUNCH();
        }
        for (int t0 = 0; t0 < ntok; t0 += LAT_TRUNK_CHUNK) {
            const int c = ntok - t0 < LAT_TRUNK_CHUNK ? ntok - t0 : LAT_TRUNK_CHUNK;
            const MwSeg up = {b.agg + (size_t)t0 * Lw, L->up, out + (size_t)t0 * H, Lw, H, Lw, H, 0, 0};
            K3C_TRY(trunk_segs(&up, 1, c, L->wdt, s));
        }
        if (sh) {
            const size_t n = (size_t)ntok * H;
            k_add_f32<<<(unsigned)((n + 255) / 256 < 1184 ? (n + 255) / 256 : 1184), 256, 0, s>>>(out, b.sdn, n);
            K3C_CHECK_LAUNCH();
        }
        stage_end(STAGE_Q8, s);
        return K3C_OK;
    }
    stage_begin(STAGE_Q8, s);   // trunk projections are reported with the trunk stage
    // 2. z = down x, and the shared expert's gate and up projections of the same x in the same
    //    launch (the shared branch depends on nothing else, so computing it first changes no
    //    result)
    const MwSeg first[3] = {{x, L->down, b.z, H, Lw, H, Lw, 0, 0},
                            {x, L->sh1, b.sgu, H, 2 * SI, H, sh ? SI : 0, 0, 0},
                            {x, L->sh3, b.sgu + SI, H, 2 * SI, H, sh ? SI : 0, 0, 0}};
    K3C_TRY(trunk_segs(first, 3, ntok, L->wdt, s));
    if (sh) {
        dim3 gs((SI + 255) / 256 < 148 ? (SI + 255) / 256 : 148, ntok);
        k_situ_rows<<<gs, 256, 0, s>>>(b.sact, b.sgu, SI, L->situ_b1, L->situ_b2);
        K3C_CHECK_LAUNCH();
    }
    stage_end(STAGE_Q8, s);
    // 3. routed experts at the latent width, weighted top-k-order sum
    K3C_TRY(launch_moe_decode_tc(b.agg, b.z, K3C_F32, ntok, &X, idx, wt, drops, b.tc, b.tc_bytes, s, true));
    stage_begin(STAGE_Q8, s);
    // 4. RMSNorm of the aggregate
    if (L->latent_norm_on) {
        k_rmsnorm_rows<<<ntok, 256, 0, s>>>(b.agg, b.agg, L->latent_norm, Lw, L->rms_eps);
        K3C_CHECK_LAUNCH();
    }
    // 5. out = up aggregate, and the shared expert's down projection in the same launch (its
    //    longer rows first); 6. out += shared output, one float addition per element, the
    //    reference's `ot[i] += sdn[i]`
    const MwSeg second[2] = {{b.sact, L->sh2, b.sdn, SI, H, SI, sh ? H : 0, 0, 0},
                             {b.agg, L->up, out, Lw, H, Lw, H, 0, 0}};
    K3C_TRY(trunk_segs(second, 2, ntok, L->wdt, s));
    if (sh) {
        const size_t n = (size_t)ntok * H;
        k_add_f32<<<(unsigned)((n + 255) / 256 < 296 ? (n + 255) / 256 : 296), 256, 0, s>>>(out, b.sdn, n);
        K3C_CHECK_LAUNCH();
    }
    stage_end(STAGE_Q8, s);
    return K3C_OK;
}

}  // namespace k3c

extern "C" int k3c_mmw(float *y, int ldy, const float *x, int ldx, int ntok, const void *W, int wdt, int in,
                       int out, int accumulate, k3c_stream_t stream) {
    k3c::clear_error();
    return k3c::launch_mmw(y, ldy, x, ldx, ntok, W, wdt, in, out, accumulate, (cudaStream_t)stream);
}

extern "C" int k3c_situ_glu(float *y, const float *gu, int n, int ntok, float b1, float b2,
                            k3c_stream_t stream) {
    k3c::clear_error();
    if (n <= 0 || ntok <= 0) return K3C_OK;
    if (!y || !gu) return k3c::set_error(K3C_EINVAL, "situ_glu: null pointer");
    dim3 gs((n + 255) / 256 < 148 ? (n + 255) / 256 : 148, ntok);
    k3c::k_situ_rows<<<gs, 256, 0, (cudaStream_t)stream>>>(y, gu, n, b1, b2);
    K3C_CHECK_LAUNCH();
    return K3C_OK;
}

extern "C" int k3c_rmsnorm(float *y, const float *x, const float *w, int n, int ntok, float eps,
                           k3c_stream_t stream) {
    k3c::clear_error();
    if (n <= 0 || ntok <= 0) return K3C_OK;
    if (!y || !x || !w) return k3c::set_error(K3C_EINVAL, "rmsnorm: null pointer");
    k3c::k_rmsnorm_rows<<<ntok, 256, 0, (cudaStream_t)stream>>>(y, x, w, n, eps);
    K3C_CHECK_LAUNCH();
    return K3C_OK;
}

extern "C" size_t k3c_moe_latent_scratch(const k3c_moe_latent_layer *L, int ntok) {
    return L ? k3c::moe_latent_scratch(L, ntok) : 0;
}

extern "C" int k3c_moe_latent_decode(float *out, const float *x, int ntok, const k3c_moe_latent_layer *L,
                                     int *idx, float *wt, int *drops, void *scratch, size_t scratch_bytes,
                                     k3c_stream_t stream) {
    k3c::clear_error();
    return k3c::launch_moe_latent(out, x, ntok, L, idx, wt, drops, scratch, scratch_bytes, (cudaStream_t)stream);
}

extern "C" int k3c_moe_latent_decode_routed(float *out, const float *x, int ntok, const k3c_moe_latent_layer *L,
                                            const int *idx, const float *wt, int *drops, void *scratch,
                                            size_t scratch_bytes, k3c_stream_t stream) {
    k3c::clear_error();
    return k3c::launch_moe_latent(out, x, ntok, L, const_cast<int *>(idx), const_cast<float *>(wt), drops, scratch,
                                  scratch_bytes, (cudaStream_t)stream, true);
}
