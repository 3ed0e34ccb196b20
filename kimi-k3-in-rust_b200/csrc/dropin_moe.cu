// dropin_moe.cu -- the reference's MoE layer entry points over host pointers: k3_moe
// (src/core/k3_ops.c:556-656), k3_moe_prefill (:668-808) and k3_moe_scratch (:658-666), declared
// at include/k3/k3.h:381-426, with the K3Cfg / K3MoeW / K3ExpertSrc types of include/k3/k3.h.
//
// A call runs in three phases:
//   1. route: the tokens and the router weights go to the device, the router runs there and the
//      top-k lists come back to the host;
//   2. experts, on the host, in the reference's call pattern on the expert source: for k3_moe,
//      token by token, the cache-only filter (resident() of each top-k entry, the kept weights
//      divided by their float sum), getmany of the top-k, then get() -- or resident() in
//      cache-only mode -- of each; for the batched k3_moe_prefill, per 64-token chunk, getmany
//      of the chunk's distinct experts in first-seen order and one get() per distinct expert. A
//      failed get is counted in k3_expert_drops with the reference's message and its pairs are
//      skipped. Experts from a k3c_pool_source stay in their pool slots; experts from any other
//      source are copied (from host or device memory) into device staging right after get() and
//      the copies complete before the source is called again, so its pointers are only used
//      inside the reference's validity window ("until the caller finishes the token");
//   3. compute: the layer with that routing, on the tensor-core latent kernels
//      (launch_moe_latent with the routing given) or, for the fp32 resident bank and for shapes
//      those kernels do not take, on fp32 GEMVs (the bank in k3_matmul's order, MXFP4 through the
//      CUDA-core GEMV) followed by the same trunk steps; the output comes back to the host.
// Tokens are processed in contiguous groups whose distinct experts fit the staging (or, for a
// pool source, leave slots free); per-token results do not depend on the grouping.
#include <cuda_runtime.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <mutex>
#include <vector>

#include "common.cuh"
#include "pool_common.cuh"

namespace k3c {
int launch_router(int *idx, float *w, float *scores, const void *x, int x_dtype, const void *W, int w_dtype,
                  const float *bias, int hidden, int n_experts, int topk, int renorm, float routed_scale,
                  int ntok, double *part, cudaStream_t s);
size_t router_scratch_bytes(int hidden, int n_experts, int ntok);
int launch_mmw(float *y, int ldy, const float *x, int ldx, int ntok, const void *W, int wdt, int in, int out,
               int accumulate, cudaStream_t s);
int launch_mx_exact(float *y, int ldy, const float *x, int ldx, int ntok, const uint8_t *packed,
                    const uint8_t *scales, int in, int rows, int group, cudaStream_t s);
int launch_q8_pack(int8_t *wq, float *wscale, int ldw, const void *rows, int in, int out, cudaStream_t s);
int launch_q8_gemv(float *y, int ldy, const void *x, int x_dtype, int ldx, int ntok, const int8_t *wq,
                   const float *wscale, int ldw, int in, int out, cudaStream_t s);
size_t moe_latent_scratch(const k3c_moe_latent_layer *L, int ntok);
int launch_moe_latent(float *out, const float *x, int ntok, const k3c_moe_latent_layer *L, int *idx_out,
                      float *wt_out, int *drops, void *scratch, size_t scratch_bytes, cudaStream_t s, bool routed);

namespace {

[[noreturn]] void mfatal(const char *what, const char *detail) {
    fprintf(stderr, "k3c: FATAL, %s: %s\n    Aborting rather than returning with the output buffer unwritten.\n",
            what, detail);
    abort();
}
void mcuda(cudaError_t e, const char *what) {
    if (e != cudaSuccess) mfatal(what, cudaGetErrorString(e));
}
void mrc(int rc, const char *what) {
    if (rc != K3C_OK) mfatal(what, k3c_last_error());
}

// Growable device buffer (contents are not kept when it grows).
struct DBuf {
    char *p = nullptr;
    size_t cap = 0;
    char *get(size_t n, const char *what) {
        if (n > cap) {
            if (p) cudaFree(p);
            p = nullptr;
            cap = 0;
            const size_t want = align_up(n < 256 ? 256 : n, (size_t)1 << 20);
            if (cudaMalloc((void **)&p, want) != cudaSuccess) mfatal(what, "cudaMalloc of the work space failed");
            cap = want;
        }
        return p;
    }
};

// A bump allocator over one DBuf (256-byte aligned pieces).
struct Bump {
    size_t used = 0;
    size_t take(size_t n) {
        const size_t o = used;
        used = align_up(used + n, 256);
        return o;
    }
};

// A weight array kept on the device across calls (k3c_dropin_keep_weights).
struct Kept {
    const void *host;
    size_t bytes;
    int q8_in;          // > 0: a K3_WI8 matrix packed as q8 (wq, ws)
    char *dev;
    k3c_q8_mat q8;
};

struct Ctx {
    std::mutex mu;
    cudaStream_t own = nullptr;
    DBuf io, wts, route, table, ring, stage, tc, work;
    std::vector<Kept> kept;
};
Ctx g_ctx[64];
bool g_keep = false;

// One weight the call reads: a host array (fp32 / bf16 as is, or K3_WI8 rows packed to q8).
struct Need {
    const void *h;
    size_t bytes;
    int q8_in, q8_out;   // K3_WI8 rows: in, out
    const void *dev;     // device copy (fp32/bf16) or nullptr
    k3c_q8_mat q8;       // packed rows (K3_WI8)
};

size_t q8_ldw(int in) { return align_up((size_t)in, 32); }

// Device copies of every Need: from the kept set (uploading what is missing) or into this
// call's weight arena.
void materialize(Ctx &c, std::vector<Need> &need, cudaStream_t s, const char *what) {
    if (g_keep) {
        for (Need &n : need) {
            if (!n.h) continue;
            Kept *hit = nullptr;
            for (Kept &k : c.kept)
                if (k.host == n.h && k.bytes == n.bytes && k.q8_in == n.q8_in) hit = &k;
            if (!hit) {
                Kept k{n.h, n.bytes, n.q8_in, nullptr, {}};
                if (n.q8_in > 0) {
                    const size_t ldw = q8_ldw(n.q8_in);
                    const size_t wq = align_up((size_t)n.q8_out * ldw, 256);
                    if (cudaMalloc((void **)&k.dev, wq + (size_t)n.q8_out * 4) != cudaSuccess)
                        mfatal(what, "cudaMalloc of a kept weight failed");
                    char *rows = nullptr;
                    mcuda(cudaMallocAsync((void **)&rows, n.bytes, s), what);
                    mcuda(cudaMemcpyAsync(rows, n.h, n.bytes, cudaMemcpyDefault, s), what);
                    mrc(launch_q8_pack((int8_t *)k.dev, (float *)(k.dev + wq), (int)ldw, rows, n.q8_in, n.q8_out, s),
                        what);
                    mcuda(cudaFreeAsync(rows, s), what);
                    k.q8 = {(const int8_t *)k.dev, (const float *)(k.dev + wq), (int)ldw};
                } else {
                    if (cudaMalloc((void **)&k.dev, n.bytes) != cudaSuccess)
                        mfatal(what, "cudaMalloc of a kept weight failed");
                    mcuda(cudaMemcpyAsync(k.dev, n.h, n.bytes, cudaMemcpyDefault, s), what);
                }
                c.kept.push_back(k);
                hit = &c.kept.back();
            }
            n.dev = hit->dev;
            n.q8 = hit->q8;
        }
        return;
    }
    Bump b;
    std::vector<size_t> off(need.size()), off2(need.size());
    for (size_t i = 0; i < need.size(); i++) {
        if (!need[i].h) continue;
        off[i] = b.take(need[i].bytes);
        if (need[i].q8_in > 0)
            off2[i] = b.take(align_up((size_t)need[i].q8_out * q8_ldw(need[i].q8_in), 256) + (size_t)need[i].q8_out * 4);
    }
    char *base = c.wts.get(b.used, what);
    for (size_t i = 0; i < need.size(); i++) {
        Need &n = need[i];
        if (!n.h) continue;
        mcuda(cudaMemcpyAsync(base + off[i], n.h, n.bytes, cudaMemcpyDefault, s), what);
        n.dev = base + off[i];
        if (n.q8_in > 0) {
            const size_t ldw = q8_ldw(n.q8_in);
            char *wq = base + off2[i];
            float *ws = (float *)(wq + align_up((size_t)n.q8_out * ldw, 256));
            mrc(launch_q8_pack((int8_t *)wq, ws, (int)ldw, n.dev, n.q8_in, n.q8_out, s), what);
            n.q8 = {(const int8_t *)wq, ws, (int)ldw};
        }
    }
}

// y[t*ldy + o] (+)= W x[t*ldx + .] for ntok tokens, W of type wdt (for K3_WI8, `W` is a host
// k3c_q8_mat): the trunk matmul of the fp32 engine.
int trunk_mm(float *y, int ldy, const float *x, int ldx, int ntok, const void *W, int wdt, int in, int out,
             cudaStream_t s) {
    if (wdt == K3C_WI8) {
        const k3c_q8_mat *q = (const k3c_q8_mat *)W;
        return launch_q8_gemv(y, ldy, x, K3C_F32, ldx, ntok, q->wq, q->wscale, q->ldw, in, out, s);
    }
    for (int t0 = 0; t0 < ntok; t0 += 32) {
        const int n = ntok - t0 < 32 ? ntok - t0 : 32;
        K3C_TRY(launch_mmw(y + (size_t)t0 * ldy, ldy, x + (size_t)t0 * ldx, ldx, n, W, wdt, in, out, 0, s));
    }
    return K3C_OK;
}

__global__ void k_rows_gather(float *__restrict__ dst, const float *__restrict__ src, const int *__restrict__ rows,
                              int n, int width) {
    const size_t total = (size_t)n * width;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x)
        dst[i] = src[(size_t)rows[i / width] * width + i % width];
}

__global__ void k_rows_scatter(float *__restrict__ dst, const float *__restrict__ src, const int *__restrict__ rows,
                               int n, int width) {
    const size_t total = (size_t)n * width;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x)
        dst[(size_t)rows[i / width] * width + i % width] = src[i];
}

// agg[t][i] = sum over j in top-k order of wt[t][j] * contrib[t][j][i], entries with idx < 0
// skipped, each product and sum rounded to float (k3_ops.c:641-642 with -ffp-contract=off).
__global__ void k_combine_latent(float *__restrict__ agg, const float *__restrict__ contrib, const int *__restrict__ idx,
                                 const float *__restrict__ wt, int ntok, int topk, int width) {
    const size_t total = (size_t)ntok * width;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const int t = (int)(i / width), c = (int)(i % width);
        float acc = 0.0f;
        for (int j = 0; j < topk; j++) {
            if (idx[(size_t)t * topk + j] < 0) continue;
            acc = __fadd_rn(acc, __fmul_rn(wt[(size_t)t * topk + j], contrib[((size_t)t * topk + j) * width + c]));
        }
        agg[i] = acc;
    }
}

__global__ void k_add_rows(float *__restrict__ y, const float *__restrict__ d, size_t n) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        y[i] = __fadd_rn(y[i], d[i]);
}

unsigned grid_for(size_t n) {
    const size_t b = (n + 255) / 256;
    return (unsigned)(b < 1184 ? (b ? b : 1) : 1184);
}

// Byte layout of one expert in the reference's run order (src/io/k3_load.c:82-105), at the
// latent width: gate / up [inter][latent] and down [latent][inter], MXFP4 with group 32.
struct RefRun {
    size_t gp, gs, dp, ds, up, us, bytes;
    size_t n_gp, n_gs, n_dp, n_ds;
};
RefRun ref_run(int L, int I) {
    RefRun r;
    r.n_gp = (size_t)I * (L / 2);
    r.n_gs = (size_t)I * ((L + K3_MXFP4_GROUP - 1) / K3_MXFP4_GROUP);
    r.n_dp = (size_t)L * (I / 2);
    r.n_ds = (size_t)L * ((I + K3_MXFP4_GROUP - 1) / K3_MXFP4_GROUP);
    r.gp = 0;
    r.gs = align_up(r.gp + r.n_gp, 256);
    r.dp = align_up(r.gs + r.n_gs, 256);
    r.ds = align_up(r.dp + r.n_dp, 256);
    r.up = align_up(r.ds + r.n_ds, 256);
    r.us = align_up(r.up + r.n_gp, 256);
    r.bytes = align_up(r.us + r.n_gs, 256);
    return r;
}

struct Layer {
    // from K3Cfg
    int H, L, I, E, K, SI, renorm, latent_norm;
    float routed_scale, eps, b1, b2;
    // device weights
    const float *gate, *bias, *norm, *w1, *w3, *w2;
    const void *down, *up, *sh1, *sh3, *sh2;   // device, or host k3c_q8_mat (K3_WI8)
    int wdt;
    k3c_q8_mat q8[5];
};

// The experts a group of tokens uses and where they are.
struct Staged {
    std::vector<int> run_of;          // expert -> run (pool slot, staging slot) or -1
    std::vector<K3ExpertQ> q;         // fp32 engine, MXFP4: device addresses per staged expert
    int n = 0;                        // staged experts
    int slots = 0;                    // room in this group
    bool any_copy = false;
};

class MoeCall {
  public:
    MoeCall(Ctx &c, const K3MoeW *w, const K3Cfg *cfg, int T, const char *what)
        : c_(c), w_(w), T_(T), what_(what) {
        l_.H = cfg->hidden;
        l_.L = cfg->latent;
        l_.I = cfg->moe_inter;
        l_.E = cfg->n_experts;
        l_.K = cfg->topk;
        l_.SI = cfg->moe_inter * cfg->n_shared;
        l_.renorm = cfg->moe_renorm;
        l_.latent_norm = cfg->latent_norm;
        l_.routed_scale = cfg->routed_scale;
        l_.eps = cfg->rms_eps;
        l_.b1 = cfg->situ_b1;
        l_.b2 = cfg->situ_b2;
        l_.wdt = w->wdt;
        check(cfg);
        pool_ = w->src ? k3c_pool_source_pool(w->src) : nullptr;
        if (pool_) {
            s_ = (cudaStream_t)k3c_pool_source_stream(w->src);
        } else {
            if (!c.own) mcuda(cudaStreamCreateWithFlags(&c.own, cudaStreamNonBlocking), what);
            s_ = c.own;
        }
        const int force32 = getenv("K3C_DROPIN_FP32") ? atoi(getenv("K3C_DROPIN_FP32")) : 0;
        // the tensor-core latent kernels: MXFP4 experts in pool format, SiTU with K3's bounds
        tc_ = w->src && !force32 && l_.L % 128 == 0 && l_.I % 128 == 0 && (T <= 32 || l_.L % 256 == 0) &&
              l_.b1 == 4.0f && l_.b2 == 25.0f && T <= 65535;
        if (pool_ && !tc_)
            mfatal(what, "a k3c_pool_source serves pool-format runs, which run on the tensor-core kernels only: "
                         "latent and moe_inter must be multiples of 128 (latent of 256 above 32 tokens), SiTU "
                         "bounds 4 and 25, and K3C_DROPIN_FP32 unset");
        if (pool_) {
            int ph = 0, pi = 0;
            k3c_pool_shape(pool_, &ph, &pi);
            if (ph != l_.L || pi != l_.I) mfatal(what, "the pool's expert shape is not (latent, moe_inter)");
        }
        rr_ = ref_run(l_.L, l_.I);
        cap_ = group_cap();
    }

    // Phase 1: tokens and weights up, routing on the device, top-k lists down.
    void route(const float *x) {
        const int H = l_.H, E = l_.E, K = l_.K, T = T_;
        need_.clear();
        const int wdt = l_.wdt;
        auto trunk_need = [&](const void *h, int in, int out) {
            Need n{};
            n.h = h;
            if (h) {
                if (wdt == K3C_WI8) {
                    n.bytes = (size_t)out * (4 + (size_t)in);
                    n.q8_in = in;
                    n.q8_out = out;
                } else {
                    n.bytes = (size_t)out * in * (wdt == K3C_WBF16 ? 2 : 4);
                }
            }
            need_.push_back(n);
        };
        auto plain = [&](const void *h, size_t bytes) {
            Need n{};
            n.h = h;
            n.bytes = h ? bytes : 0;
            need_.push_back(n);
        };
        plain(w_->gate, (size_t)E * H * 4);                                   // 0
        plain(w_->bias, (size_t)E * 4);                                       // 1
        plain(l_.latent_norm ? w_->latent_norm : nullptr, (size_t)l_.L * 4);  // 2
        trunk_need(w_->down, H, l_.L);                                        // 3
        trunk_need(w_->up, l_.L, H);                                          // 4
        trunk_need(l_.SI ? w_->sh1 : nullptr, H, l_.SI);                      // 5
        trunk_need(l_.SI ? w_->sh3 : nullptr, H, l_.SI);                      // 6
        trunk_need(l_.SI ? w_->sh2 : nullptr, l_.SI, H);                      // 7
        const bool bank = !w_->src;
        const size_t per = (size_t)l_.I * l_.L * 4;
        plain(bank ? w_->w1 : nullptr, per * E);                              // 8
        plain(bank ? w_->w3 : nullptr, per * E);                              // 9
        plain(bank ? w_->w2 : nullptr, per * E);                              // 10
        materialize(c_, need_, s_, what_);
        l_.gate = (const float *)need_[0].dev;
        l_.bias = (const float *)need_[1].dev;
        l_.norm = (const float *)need_[2].dev;
        const void **tr[5] = {&l_.down, &l_.up, &l_.sh1, &l_.sh3, &l_.sh2};
        for (int i = 0; i < 5; i++) {
            Need &n = need_[3 + i];
            l_.q8[i] = n.q8;
            *tr[i] = !n.h ? nullptr : (wdt == K3C_WI8 ? (const void *)&l_.q8[i] : n.dev);
        }
        l_.w1 = (const float *)need_[8].dev;
        l_.w3 = (const float *)need_[9].dev;
        l_.w2 = (const float *)need_[10].dev;
        // tokens in, routing
        Bump b;
        const size_t o_x = b.take((size_t)T * H * 4), o_o = b.take((size_t)T * H * 4);
        const size_t o_i = b.take((size_t)T * K * 4), o_w = b.take((size_t)T * K * 4);
        const size_t o_p = b.take(router_scratch_bytes(H, E, T));
        char *io = c_.io.get(b.used, what_);
        dx_ = (float *)(io + o_x);
        dout_ = (float *)(io + o_o);
        didx_ = (int *)(io + o_i);
        dwt_ = (float *)(io + o_w);
        mcuda(cudaMemcpyAsync(dx_, x, (size_t)T * H * 4, cudaMemcpyHostToDevice, s_), what_);
        mrc(launch_router(didx_, dwt_, nullptr, dx_, K3C_F32, l_.gate, K3C_F32, l_.bias, H, E, K, l_.renorm,
                          l_.routed_scale, T, (double *)(io + o_p), s_),
            what_);
        ridx_.resize((size_t)T * K);
        rwt_.resize((size_t)T * K);
        mcuda(cudaMemcpyAsync(ridx_.data(), didx_, (size_t)T * K * 4, cudaMemcpyDeviceToHost, s_), what_);
        mcuda(cudaMemcpyAsync(rwt_.data(), dwt_, (size_t)T * K * 4, cudaMemcpyDeviceToHost, s_), what_);
        mcuda(cudaStreamSynchronize(s_), what_);
        hidx_ = ridx_;
        hwt_ = rwt_;
    }

    // k3_moe: phase 2 token by token, phase 3 per group of tokens. last_idx/last_wt (host,
    // may be NULL) receive the lists the reference leaves in idx/wt: the last token's router
    // output, compacted and renormalised in cache-only mode.
    void run_per_token(int t0, int t1, int *last_idx, float *last_wt) {
        const int K = l_.K;
        K3ExpertSrc *src = w_->src;
        int g0 = t0;
        Staged st;
        reset(st, cap_);
        for (int t = t0; t < t1; t++) {
            int *it = &hidx_[(size_t)t * K];
            float *wtt = &hwt_[(size_t)t * K];
            // the reference's idx/wt for this token (entries past nk keep the router's values)
            std::vector<int> ci(it, it + K);
            std::vector<float> cw(wtt, wtt + K);
            int nk = K;
            if (w_->cache_only && src->resident) {
                int m = 0;
                float wsum = 0.0f;
                for (int j = 0; j < K; j++)
                    if (src->resident(src, w_->layer, ci[j], nullptr)) {
                        ci[m] = ci[j];
                        cw[m] = cw[j];
                        wsum += cw[j];
                        m++;
                    }
                nk = m;
                if (wsum > 0.0f)
                    for (int j = 0; j < nk; j++) cw[j] /= wsum;
            }
            if (group_full(st, ci.data(), nk)) {   // compute what is staged, then start afresh
                compute(st, g0, t);
                g0 = t;
                reset(st, cap_);
            }
            std::vector<int> use(ci.begin(), ci.begin() + nk);
            if (!w_->cache_only && src->getmany) src->getmany(src, w_->layer, ci.data(), nk);
            for (int j = 0; j < nk; j++) {
                K3ExpertQ q;
                const int miss = w_->cache_only ? !src->resident(src, w_->layer, ci[j], &q)
                                                : (src->get(src, w_->layer, ci[j], &q) != 0);
                if (miss) {
                    if (!w_->cache_only) {
                        k3_expert_drops++;
                        fprintf(stderr, "EXPERT DROP: layer %d expert %d failed to load; this token is CORRUPT\n",
                                w_->layer, ci[j]);
                    }
                    use[j] = -1;   // skipped
                    continue;
                }
                stage(st, ci[j], q);
            }
            sync_copies(st);
            for (int j = 0; j < K; j++) {   // the device lists: the used entries in order, -1 elsewhere
                it[j] = j < nk ? use[j] : -1;
                wtt[j] = j < nk ? cw[j] : 0.0f;
            }
            if (t == t1 - 1 && last_idx) {
                memcpy(last_idx, ci.data(), (size_t)K * sizeof(int));
                memcpy(last_wt, cw.data(), (size_t)K * sizeof(float));
            }
        }
        compute(st, g0, t1);
    }

    // k3_moe_prefill's batched path for tokens [t0, t1) of one chunk (more than one token).
    void run_chunk(int t0, int t1) {
        const int K = l_.K, E = l_.E;
        K3ExpertSrc *src = w_->src;
        std::vector<int> uniq;
        std::vector<char> seen(E, 0);
        for (int t = t0; t < t1; t++)
            for (int j = 0; j < K; j++) {
                const int e = hidx_[(size_t)t * K + j];
                if (e >= 0 && e < E && !seen[e]) {
                    seen[e] = 1;
                    uniq.push_back(e);
                }
            }
        Staged st;
        reset(st, (int)uniq.size());
        if (src->getmany) src->getmany(src, w_->layer, uniq.data(), (int)uniq.size());
        std::vector<char> failed(E, 0);
        for (int e : uniq) {
            K3ExpertQ q;
            if (src->get(src, w_->layer, e, &q) != 0) {
                k3_expert_drops++;
                fprintf(stderr, "EXPERT DROP: layer %d expert %d failed to load; this chunk is CORRUPT\n", w_->layer,
                        e);
                failed[e] = 1;
                continue;
            }
            stage(st, e, q);
            sync_copies(st);   // the source's pointers are read before the next get()
        }
        for (int t = t0; t < t1; t++)
            for (int j = 0; j < K; j++) {
                int &e = hidx_[(size_t)t * K + j];
                if (e >= 0 && e < E && failed[e]) e = -1;
            }
        compute(st, t0, t1);
    }

    // The fp32 bank (no source): every token at once.
    void run_bank(int *last_idx, float *last_wt) {
        Staged st;
        reset(st, 0);
        compute(st, 0, T_);
        if (last_idx) {
            const int K = l_.K;
            memcpy(last_idx, &ridx_[(size_t)(T_ - 1) * K], (size_t)K * 4);
            memcpy(last_wt, &rwt_[(size_t)(T_ - 1) * K], (size_t)K * 4);
        }
    }

    void finish(float *out) {
        mcuda(cudaMemcpyAsync(out, dout_, (size_t)T_ * l_.H * 4, cudaMemcpyDeviceToHost, s_), what_);
        mcuda(cudaStreamSynchronize(s_), what_);
    }

    bool has_src() const { return w_->src != nullptr; }

  private:
    Ctx &c_;
    const K3MoeW *w_;
    int T_;
    const char *what_;
    Layer l_{};
    k3c_expert_pool *pool_ = nullptr;
    cudaStream_t s_ = nullptr;
    bool tc_ = false;
    RefRun rr_{};
    std::vector<Need> need_;
    float *dx_ = nullptr, *dout_ = nullptr, *dwt_ = nullptr;
    int *didx_ = nullptr;
    std::vector<int> ridx_, hidx_;
    std::vector<float> rwt_, hwt_;
    int cap_ = 0;   // experts one group may stage (foreign source) or pin (pool source)

    void check(const K3Cfg *cfg) {
        char d[160];
        if (!w_ || !cfg) mfatal(what_, "null weights or config");
        if (T_ < 0 || T_ > 65535) {
            snprintf(d, sizeof d, "T=%d outside 0..65535", T_);
            mfatal(what_, d);
        }
        if (l_.H <= 0 || l_.L <= 0 || l_.I <= 0 || l_.E <= 0 || l_.K <= 0 || l_.K > K3_MAX_TOPK || l_.K > l_.E ||
            cfg->n_shared < 0) {
            snprintf(d, sizeof d, "hidden=%d latent=%d moe_inter=%d n_experts=%d topk=%d n_shared=%d", l_.H, l_.L,
                     l_.I, l_.E, l_.K, cfg->n_shared);
            mfatal(what_, d);
        }
        if (l_.wdt != K3C_WF32 && l_.wdt != K3C_WBF16 && l_.wdt != K3C_WI8) mfatal(what_, "unknown wdt");
        if (!w_->gate || !w_->down || !w_->up || (l_.SI && (!w_->sh1 || !w_->sh3 || !w_->sh2)) ||
            (l_.latent_norm && !w_->latent_norm))
            mfatal(what_, "a weight the layer reads is NULL");
        if (!w_->src && (!w_->w1 || !w_->w3 || !w_->w2)) mfatal(what_, "no expert source and no resident bank");
        if (w_->src && !w_->src->get) mfatal(what_, "expert source without get()");
        if (w_->src && w_->cache_only && !w_->src->resident)
            mfatal(what_, "cache_only needs an expert source with resident()");
        if (w_->src && (l_.L % 2 || l_.I % 2)) mfatal(what_, "MXFP4 experts need even latent and moe_inter");
    }

    // A fresh group that can stage `slots` experts (foreign sources: device staging sized for
    // them now, so nothing moves while the group fills).
    void reset(Staged &st, int slots) {
        st.run_of.assign(l_.E, -1);
        st.q.clear();
        st.n = 0;
        st.any_copy = false;
        st.slots = slots;
        if (!w_->src || pool_ || slots <= 0) return;
        const size_t ring = (size_t)(tc_ ? l_.K + 1 : slots) * rr_.bytes;
        ring_ = c_.ring.get(ring, what_);
        if (tc_) arena_ = c_.stage.get((size_t)slots * pool_stride(), what_);
    }

    size_t pool_stride() const { return align_up(pool_geom(l_.L, l_.I).run, 256); }

    // Experts one group of k3_moe tokens may stage: for a pool source, the slots less room for
    // two tokens' pins; otherwise 8 GB of staged runs, at least two tokens' worth.
    int group_cap() const {
        if (pool_) {
            const int ns = k3c_pool_slots(pool_);
            return ns - 2 * l_.K > l_.K ? ns - 2 * l_.K : l_.K;
        }
        const size_t per = tc_ ? pool_stride() : rr_.bytes;
        size_t n = ((size_t)8 << 30) / (per ? per : 1);
        if (n < (size_t)2 * l_.K) n = 2 * l_.K;
        return (int)(n < (size_t)l_.E ? n : (size_t)l_.E);
    }

    // Would staging these nk experts overflow the group?
    bool group_full(const Staged &st, const int *ids, int nk) const {
        int add = 0;
        for (int j = 0; j < nk; j++)
            if (ids[j] >= 0 && ids[j] < l_.E && st.run_of[ids[j]] < 0) add++;
        return st.n + add > st.slots && st.n > 0;
    }

    // Expert e (from get/resident) into this group's run table.
    void stage(Staged &st, int e, const K3ExpertQ &q) {
        if (st.run_of[e] >= 0) return;
        if (pool_) {
            const int slot = k3c_pool_source_slot(w_->src, &q);
            if (slot < 0) mfatal(what_, "a pool source returned an expert outside its arena");
            st.run_of[e] = slot;
            st.n++;
            return;
        }
        if (st.n >= st.slots) mfatal(what_, "more distinct experts than the group's staging");
        if (!q.p1 || !q.s1 || !q.p3 || !q.s3 || !q.p2 || !q.s2) mfatal(what_, "the source returned a NULL matrix");
        const int u = st.n++;
        // the six matrices of the reference layout, from host or device memory
        char *r = ring_ + (size_t)(tc_ ? u % (l_.K + 1) : u) * rr_.bytes;
        mcuda(cudaMemcpyAsync(r + rr_.gp, q.p1, rr_.n_gp, cudaMemcpyDefault, s_), what_);
        mcuda(cudaMemcpyAsync(r + rr_.gs, q.s1, rr_.n_gs, cudaMemcpyDefault, s_), what_);
        mcuda(cudaMemcpyAsync(r + rr_.up, q.p3, rr_.n_gp, cudaMemcpyDefault, s_), what_);
        mcuda(cudaMemcpyAsync(r + rr_.us, q.s3, rr_.n_gs, cudaMemcpyDefault, s_), what_);
        mcuda(cudaMemcpyAsync(r + rr_.dp, q.p2, rr_.n_dp, cudaMemcpyDefault, s_), what_);
        mcuda(cudaMemcpyAsync(r + rr_.ds, q.s2, rr_.n_ds, cudaMemcpyDefault, s_), what_);
        st.any_copy = true;
        K3ExpertQ dq;
        dq.p1 = (const unsigned char *)(r + rr_.gp);
        dq.s1 = (const unsigned char *)(r + rr_.gs);
        dq.p3 = (const unsigned char *)(r + rr_.up);
        dq.s3 = (const unsigned char *)(r + rr_.us);
        dq.p2 = (const unsigned char *)(r + rr_.dp);
        dq.s2 = (const unsigned char *)(r + rr_.ds);
        if (tc_)   // into this group's pool-format run u (the ring slot is reused after a sync)
            mrc(k3c_pool_pack_expert((uint8_t *)arena_ + (size_t)u * pool_stride(), &dq, l_.L, l_.I,
                                     (k3c_stream_t)s_),
                what_);
        st.q.push_back(dq);
        st.run_of[e] = u;
    }

    // The copies read the source's memory before it is called again (and before a ring slot
    // is written a second time).
    void sync_copies(Staged &st) {
        if (st.any_copy) mcuda(cudaStreamSynchronize(s_), what_);
        st.any_copy = false;
    }

    char *ring_ = nullptr, *arena_ = nullptr;

    // Phase 3 for tokens [t0, t1) with the experts of `st`; a pool source's pins are released
    // once the kernels reading the slots are enqueued.
    void compute(Staged &st, int t0, int t1) {
        const int n = t1 - t0;
        if (n <= 0) return;
        const int K = l_.K, H = l_.H;
        int *didx = didx_ + (size_t)t0 * K;
        float *dwt = dwt_ + (size_t)t0 * K;
        mcuda(cudaMemcpyAsync(didx, &hidx_[(size_t)t0 * K], (size_t)n * K * 4, cudaMemcpyHostToDevice, s_), what_);
        mcuda(cudaMemcpyAsync(dwt, &hwt_[(size_t)t0 * K], (size_t)n * K * 4, cudaMemcpyHostToDevice, s_), what_);
        const float *x = dx_ + (size_t)t0 * H;
        float *out = dout_ + (size_t)t0 * H;
        if (tc_)
            compute_tc(st, x, out, n, didx, dwt);
        else
            compute_fp32(st, t0, x, out, n, didx, dwt);
        if (pool_) mrc(k3c_pool_source_release(w_->src), what_);
        // the host lists and run table went up from pageable memory; the next group rewrites them
        mcuda(cudaStreamSynchronize(s_), what_);
    }

    void compute_tc(Staged &st, const float *x, float *out, int n, int *didx, float *dwt) {
        int *table = (int *)c_.table.get((size_t)l_.E * 4, what_);
        mcuda(cudaMemcpyAsync(table, st.run_of.data(), (size_t)l_.E * 4, cudaMemcpyHostToDevice, s_), what_);
        k3c_moe_latent_layer M;
        memset(&M, 0, sizeof M);
        M.hidden = l_.H;
        k3c_moe_pool_layer &X = M.experts;
        X.hidden = l_.L;
        X.inter = l_.I;
        X.n_experts = l_.E;
        X.topk = l_.K;
        X.renorm = l_.renorm;
        X.act = K3C_ACT_SITU;
        X.routed_scale = l_.routed_scale;
        X.router_w = l_.gate;
        X.router_dtype = K3C_F32;
        X.router_bias = l_.bias;
        if (pool_) {
            X.arena = k3c_pool_arena(pool_);
            X.run_stride = k3c_pool_slot_stride(pool_);
            X.n_runs = k3c_pool_slots(pool_);
        } else {
            X.run_stride = pool_stride();
            X.n_runs = st.n > 0 ? st.n : 1;
            X.arena = (const uint8_t *)(arena_ ? arena_ : c_.stage.get(X.run_stride, what_));
        }
        X.run_of = table;
        X.shared_run = -1;
        X.terms = 3;
        M.router_w = l_.gate;
        M.router_bias = l_.bias;
        M.down = l_.down;
        M.up = l_.up;
        M.sh1 = l_.sh1;
        M.sh3 = l_.sh3;
        M.sh2 = l_.sh2;
        M.latent_norm = l_.norm;
        M.wdt = l_.wdt;
        M.n_shared = l_.SI ? l_.SI / l_.I : 0;
        M.latent_norm_on = l_.latent_norm;
        M.rms_eps = l_.eps;
        M.situ_b1 = l_.b1;
        M.situ_b2 = l_.b2;
        const size_t need = moe_latent_scratch(&M, n);
        char *scr = c_.tc.get(need, what_);
        mrc(launch_moe_latent(out, x, n, &M, didx, dwt, nullptr, scr, need, s_, true), what_);
    }

    void compute_fp32(Staged &st, int t0, const float *x, float *out, int n, const int *didx, const float *dwt) {
        const int H = l_.H, L = l_.L, I = l_.I, K = l_.K, SI = l_.SI, E = l_.E;
        // pairs grouped by expert (token-major within an expert)
        std::vector<std::vector<int>> by(E);
        for (int t = 0; t < n; t++)
            for (int j = 0; j < K; j++) {
                const int e = hidx_[(size_t)(t0 + t) * K + j];
                if (e >= 0) by[e].push_back(t * K + j);
            }
        int nmax = 0, npairs = 0;
        for (int e = 0; e < E; e++) {
            nmax = (int)by[e].size() > nmax ? (int)by[e].size() : nmax;
            npairs += (int)by[e].size();
        }
        Bump b;
        const size_t o_z = b.take((size_t)n * L * 4), o_agg = b.take((size_t)n * L * 4);
        const size_t o_c = b.take((size_t)n * K * L * 4), o_sgu = b.take((size_t)n * 2 * SI * 4);
        const size_t o_sa = b.take((size_t)n * SI * 4), o_sd = b.take((size_t)n * H * 4);
        const size_t o_zg = b.take((size_t)nmax * L * 4), o_gu = b.take((size_t)nmax * 2 * I * 4);
        const size_t o_ac = b.take((size_t)nmax * I * 4), o_ed = b.take((size_t)nmax * L * 4);
        const size_t o_pl = b.take((size_t)(2 * npairs + 1) * 4);
        char *wk = c_.work.get(b.used, what_);
        float *z = (float *)(wk + o_z), *agg = (float *)(wk + o_agg), *contrib = (float *)(wk + o_c);
        float *sgu = (float *)(wk + o_sgu), *sact = (float *)(wk + o_sa), *sdn = (float *)(wk + o_sd);
        float *zg = (float *)(wk + o_zg), *gu = (float *)(wk + o_gu), *act = (float *)(wk + o_ac);
        float *edn = (float *)(wk + o_ed);
        int *plist = (int *)(wk + o_pl);
        // pair lists on the device: per expert, its tokens then its (t*K + j) slots
        std::vector<int> hl;
        std::vector<size_t> off(E, 0);
        for (int e = 0; e < E; e++) {
            off[e] = hl.size();
            for (int p : by[e]) hl.push_back(p / K);
            for (int p : by[e]) hl.push_back(p);
        }
        if (!hl.empty())
            mcuda(cudaMemcpyAsync(plist, hl.data(), hl.size() * 4, cudaMemcpyHostToDevice, s_), what_);
        mcuda(cudaMemsetAsync(contrib, 0, (size_t)n * K * L * 4, s_), what_);
        // z = down x; the shared expert's gate/up and its SiTU and down projection
        mrc(trunk_mm(z, L, x, H, n, l_.down, l_.wdt, H, L, s_), what_);
        if (SI) {
            mrc(trunk_mm(sgu, 2 * SI, x, H, n, l_.sh1, l_.wdt, H, SI, s_), what_);
            mrc(trunk_mm(sgu + SI, 2 * SI, x, H, n, l_.sh3, l_.wdt, H, SI, s_), what_);
            mrc(k3c_situ_glu(sact, sgu, SI, n, l_.b1, l_.b2, (k3c_stream_t)s_), what_);
            mrc(trunk_mm(sdn, H, sact, SI, n, l_.sh2, l_.wdt, SI, H, s_), what_);
        }
        // the routed experts, one distinct expert at a time over its pairs
        for (int e = 0; e < E; e++) {
            const int m = (int)by[e].size();
            if (!m) continue;
            const int *toks = plist + off[e], *slots = plist + off[e] + m;
            k_rows_gather<<<grid_for((size_t)m * L), 256, 0, s_>>>(zg, z, toks, m, L);
            mrc(cudaGetLastError() == cudaSuccess ? K3C_OK : K3C_ECUDA, what_);
            count_launch();
            if (!w_->src) {   // the fp32 bank in k3_matmul's order
                const float *e1 = l_.w1 + (size_t)e * I * L, *e3 = l_.w3 + (size_t)e * I * L;
                const float *e2 = l_.w2 + (size_t)e * L * I;
                mrc(trunk_mm(gu, 2 * I, zg, L, m, e1, K3C_WF32, L, I, s_), what_);
                mrc(trunk_mm(gu + I, 2 * I, zg, L, m, e3, K3C_WF32, L, I, s_), what_);
                mrc(k3c_situ_glu(act, gu, I, m, l_.b1, l_.b2, (k3c_stream_t)s_), what_);
                mrc(trunk_mm(edn, L, act, I, m, e2, K3C_WF32, I, L, s_), what_);
            } else {           // MXFP4 from the staged reference-layout copy
                const K3ExpertQ &q = st.q[st.run_of[e]];
                mrc(launch_mx_exact(gu, 2 * I, zg, L, m, q.p1, q.s1, L, I, K3_MXFP4_GROUP, s_), what_);
                mrc(launch_mx_exact(gu + I, 2 * I, zg, L, m, q.p3, q.s3, L, I, K3_MXFP4_GROUP, s_), what_);
                mrc(k3c_situ_glu(act, gu, I, m, l_.b1, l_.b2, (k3c_stream_t)s_), what_);
                mrc(launch_mx_exact(edn, L, act, I, m, q.p2, q.s2, I, L, K3_MXFP4_GROUP, s_), what_);
            }
            k_rows_scatter<<<grid_for((size_t)m * L), 256, 0, s_>>>(contrib, edn, slots, m, L);
            mrc(cudaGetLastError() == cudaSuccess ? K3C_OK : K3C_ECUDA, what_);
            count_launch();
        }
        k_combine_latent<<<grid_for((size_t)n * L), 256, 0, s_>>>(agg, contrib, didx, dwt, n, K, L);
        mrc(cudaGetLastError() == cudaSuccess ? K3C_OK : K3C_ECUDA, what_);
        count_launch();
        if (l_.latent_norm) mrc(k3c_rmsnorm(agg, agg, l_.norm, L, n, l_.eps, (k3c_stream_t)s_), what_);
        mrc(trunk_mm(out, H, agg, L, n, l_.up, l_.wdt, L, H, s_), what_);
        if (SI) {
            k_add_rows<<<grid_for((size_t)n * H), 256, 0, s_>>>(out, sdn, (size_t)n * H);
            mrc(cudaGetLastError() == cudaSuccess ? K3C_OK : K3C_ECUDA, what_);
            count_launch();
        }
    }

};

Ctx &ctx_for(const char *what) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) mfatal(what, "no CUDA device");
    return g_ctx[dev];
}

void moe_call(float *out, const float *x, const K3MoeW *w, const K3Cfg *c, int T, int *idx, float *wt, bool prefill) {
    const char *what = prefill ? "k3_moe_prefill" : "k3_moe";
    if (!w || !c) mfatal(what, "null weights or config");
    if (T <= 0) return;
    Ctx &ctx = ctx_for(what);
    std::lock_guard<std::mutex> lk(ctx.mu);
    MoeCall call(ctx, w, c, T, what);
    call.route(x);
    static const int no_batch = getenv("K3_NO_BATCH_PREFILL") ? 1 : 0;
    if (!call.has_src()) {
        call.run_bank(idx, wt);
    } else if (!prefill || T <= 1 || no_batch || w->cache_only) {
        call.run_per_token(0, T, idx, wt);
    } else {
        const int CHUNK = 64;   // the reference's fixed sub-chunk (k3_ops.c:705-713)
        for (int t0 = 0; t0 < T; t0 += CHUNK) {
            const int n = T - t0 < CHUNK ? T - t0 : CHUNK;
            if (n == 1)
                call.run_per_token(t0, t0 + 1, idx, wt);
            else
                call.run_chunk(t0, t0 + n);
        }
    }
    call.finish(out);
}

}  // namespace
}  // namespace k3c

extern "C" {

size_t k3_moe_scratch(const K3Cfg *c) {
    const size_t SI = (size_t)c->moe_inter * c->n_shared;
    return (size_t)2 * c->latent + (size_t)3 * c->moe_inter + (size_t)c->latent + 3 * SI + (size_t)c->hidden;
}

void k3_moe(float *out, const float *x, const K3MoeW *w, const K3Cfg *c, int T, int *idx, float *wt,
            float *scratch) {
    (void)scratch;
    k3c::moe_call(out, x, w, c, T, idx, wt, false);
}

void k3_moe_prefill(float *out, const float *x, const K3MoeW *w, const K3Cfg *c, int T, int *idx, float *wt,
                    float *scratch) {
    (void)scratch;
    k3c::moe_call(out, x, w, c, T, idx, wt, true);
}

void k3c_dropin_keep_weights(int on) { k3c::g_keep = on != 0; }

void k3c_dropin_forget_weights(void) {
    for (int d = 0; d < 64; d++) {
        k3c::Ctx &c = k3c::g_ctx[d];
        std::lock_guard<std::mutex> lk(c.mu);
        if (c.kept.empty()) continue;
        int cur = 0;
        cudaGetDevice(&cur);
        cudaSetDevice(d);
        cudaDeviceSynchronize();
        for (auto &k : c.kept) cudaFree(k.dev);
        c.kept.clear();
        cudaSetDevice(cur);
    }
}

}  // extern "C"
