// moe_prefill.cu -- MoE prefill on the tcgen05 tensor cores: the reference's
// k3_moe_prefill / moe_prefill_chunk (src/core/k3_ops.c:689-808) for the non-latent BASELINE
// shape: route every token, group the (token, expert) pairs by expert, run each expert's
// SwiGLU FFN over its group, and combine the outputs in each token's top-k order.
//
// Layout of the work:
//   pairs   T*topk (token, k) pairs are counting-sorted by expert (stable: pair index order
//           within an expert). Rows: expert e's pairs occupy compact rows [eoff_e, eoff_e+n_e),
//           the shared expert's T rows follow; slots of up to 128 consecutive rows, one
//           expert owning ceil(n_e/128) of them.
//   x       each row's token is quantised into J = 2 E4M3 terms per element with one UE8M0
//           scale per 32 elements (the decode path's term split), in row order, so a slot's
//           A tile is one TMA box of 128 rows starting at its first row. Rows past the slot's
//           pairs belong to the next slot: they only feed accumulator rows that are never read.
//   GU      per work item (slot, 256 gate/up rows): the slot's 128 pair rows are the MMA's M
//           side, 256 pool-format gate/up weight rows are N. Both terms accumulate into one
//           TMEM accumulator (each MMA applies its own block scales). The epilogue (one thread
//           per pair row) forms SwiGLU for 128 intermediate columns and requantises each
//           32-column block, which lies inside one thread, into the down stage's operand
//           (same compact rows).
//   D       per work item (slot, 256 hidden rows): the same MMA over the requantised
//           activations; the epilogue writes each pair's unweighted expert output as a bf16
//           row (rounded to nearest) into the token's [topk+1][H] pair rows -- in the token
//           owner's receive buffer, over NVLink, under expert parallelism.
//   combine the decode path's fixed-order weighted sum (k3_ops.c:641-642, fp32 products and
//           sums of the bf16 rows) plus the shared expert.
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdlib.h>

#include "common.cuh"
#include "pool_common.cuh"
#include "tc_common.cuh"
#include "tc_host.cuh"

namespace k3c {

int launch_router(int *idx, float *w, float *scores, const void *x, int x_dtype, const void *W, int w_dtype,
                  const float *bias, int hidden, int n_experts, int topk, int renorm, float routed_scale,
                  int ntok, double *part, cudaStream_t s);
size_t router_scratch_bytes(int hidden, int n_experts, int ntok);
int launch_moe_combine(float *out, const float *contrib, const float *wt, const uint8_t *dropped,
                       int ntok, int topk, int hidden, int has_shared, cudaStream_t s);
int launch_moe_combine_ids(float *out, const float *contrib, const float *wt, const uint8_t *dropped,
                           const int *ids, int n_experts, int ntok, int topk, int hidden, int has_shared,
                           cudaStream_t s);

namespace {
constexpr int PF_J = 2;                       // E4M3 terms per activation
constexpr int PF_M = 128;                     // pair rows per slot (MMA M)
constexpr int PF_N = 256;                     // weight rows per work item (MMA N)
constexpr int PF_CHUNK = 1024;                // pairs per planning block
constexpr int PF_A = PF_M * 128;              // one term's A tile: 16 KB
constexpr int PF_B = PF_N * 128;              // padded E2M1 B tile: 32 KB
constexpr int PF_SF = (PF_J + 2) * 512;       // SFA per term + two SFB atoms
constexpr int PF_STAGE = PF_J * PF_A + PF_B + PF_SF;
constexpr int PF_STAGES = 3;
constexpr int PF_EPI_WARPS = 8;               // two per TMEM lane quadrant, each half the columns
constexpr int PF_THREADS = 64 + 32 * PF_EPI_WARPS;
constexpr int PF_STG = 32 * 64;                // D epilogue: a warp's 32 rows x 32 bf16 columns
constexpr int PF_BYTES = 1024 + PF_STAGES * PF_STAGE + 256 + PF_EPI_WARPS * PF_STG;
constexpr uint32_t PF_TMEM = 512;             // accumulator 256 columns + scale factors
constexpr uint32_t PF_SF_COL = 256;
constexpr uint32_t PF_TX = PF_J * PF_A + PF_N * 64 + PF_SF;   // E2M1 moves 4 bits per element
static_assert(PF_STAGE % 1024 == 0, "stage bases stay 1024-byte aligned");
static_assert(8 * (2 * PF_STAGES + 2) + 4 <= 256, "barrier area");
static_assert(PF_BYTES <= 227 * 1024, "fits one CTA per SM");
}  // namespace

struct SlotPf {
    int run, ntok, row0;   // pool run, pairs in the slot, first compact row
};

// ------------------------------------------------------------------ planning
// Per chunk of 1024 pairs: the pair's expert (-1 when the expert is not resident, counted as
// a drop), the chunk's per-expert counts, and each pair's rank among the chunk's earlier
// pairs of the same expert.
__global__ void __launch_bounds__(1024) k_pf_count(int *__restrict__ pe_out, int *__restrict__ rank_out,
                                                   int *__restrict__ cnt, uint8_t *__restrict__ dropped,
                                                   int *__restrict__ drops, const int *__restrict__ idx, int P,
                                                   const int *__restrict__ run_of, int n_experts, int n_runs) {
    extern __shared__ int pfs[];
    int *hist = pfs, *pe = pfs + n_experts;
    const int i0 = blockIdx.x * PF_CHUNK, n = min(PF_CHUNK, P - i0);
    for (int e = threadIdx.x; e < n_experts; e += blockDim.x) hist[e] = 0;
    __syncthreads();
    const int i = threadIdx.x;
    int e = -1;
    if (i < n) {
        e = idx[i0 + i];
        // a run index outside the arena is treated as not resident: the kernels form raw
        // addresses from it
        const bool ok = e >= 0 && e < n_experts && run_of[e] >= 0 && run_of[e] < n_runs;
        dropped[i0 + i] = ok ? 0 : 1;
        if (ok) atomicAdd(&hist[e], 1);
        else {
            if (drops) atomicAdd(drops, 1);
            e = -1;
        }
        pe_out[i0 + i] = e;
    }
    pe[i] = e;
    __syncthreads();
    if (i < n && e >= 0) {
        int r = 0;
        for (int k = 0; k < i; k++) r += pe[k] == e;
        rank_out[i0 + i] = r;
    }
    for (int x = threadIdx.x; x < n_experts; x += blockDim.x) cnt[(size_t)blockIdx.x * n_experts + x] = hist[x];
}

// Block-wide exclusive prefix sums of (a, b) over the threads' values; *ta, *tb get the totals.
__device__ __forceinline__ void block_scan2(int a, int b, int &xa, int &xb, int &ta, int &tb, int2 *warp_sum) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarp = blockDim.x >> 5;
    int ia = a, ib = b;   // inclusive warp scans
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int va = __shfl_up_sync(0xffffffffu, ia, o), vb = __shfl_up_sync(0xffffffffu, ib, o);
        if (lane >= o) {
            ia += va;
            ib += vb;
        }
    }
    if (lane == 31) warp_sum[warp] = make_int2(ia, ib);
    __syncthreads();
    int pa = 0, pb = 0;
    ta = tb = 0;
    for (int w = 0; w < nwarp; w++) {
        const int2 v = warp_sum[w];
        if (w < warp) {
            pa += v.x;
            pb += v.y;
        }
        ta += v.x;
        tb += v.y;
    }
    xa = pa + ia - a;
    xb = pb + ib - b;
    __syncthreads();   // warp_sum may be rewritten by the caller's next scan
}

// One block: each expert's per-chunk bases, its first compact row (eoff) and first slot
// (slot_base) by block-wide prefix sums of n_e and ceil(n_e/128), the slot table, and the
// shared expert's rows and slots after all routed pairs (tokens sh_base .. sh_base+sh_n-1).
__global__ void __launch_bounds__(1024) k_pf_slots(int *__restrict__ n_slots, SlotPf *__restrict__ slots,
                                                   int *__restrict__ pair_tok, int *__restrict__ pair_k,
                                                   int *__restrict__ row_tok, int *__restrict__ n_rows,
                                                   int *__restrict__ chunk_base, int *__restrict__ slot_base,
                                                   int *__restrict__ eoff, const int *__restrict__ cnt,
                                                   int nchunk, const int *__restrict__ run_of, int n_experts,
                                                   int sh_base, int sh_n, int topk, int shared_run,
                                                   int *__restrict__ sh_row0) {
    __shared__ int2 warp_sum[32];
    int sbase = 0, rbase = 0;
    for (int e0 = 0; e0 < n_experts; e0 += blockDim.x) {
        const int e = e0 + threadIdx.x;
        int ne = 0;
        if (e < n_experts)
            for (int c = 0; c < nchunk; c++) {
                chunk_base[(size_t)c * n_experts + e] = ne;
                ne += cnt[(size_t)c * n_experts + e];
            }
        const int nsl = (ne + PF_M - 1) / PF_M;
        int xs, xr, ts, tr;
        block_scan2(nsl, ne, xs, xr, ts, tr, warp_sum);
        if (e < n_experts) {
            slot_base[e] = sbase + xs;
            eoff[e] = rbase + xr;
            for (int q = 0; q < nsl; q++) {
                SlotPf &sl = slots[sbase + xs + q];
                sl.run = run_of[e];
                sl.ntok = min(PF_M, ne - PF_M * q);
                sl.row0 = rbase + xr + PF_M * q;
            }
        }
        sbase += ts;
        rbase += tr;
    }
    if (threadIdx.x == 0) *sh_row0 = shared_run >= 0 ? rbase : -1;   // the shared rows follow the routed ones
    if (shared_run >= 0) {
        for (int t = threadIdx.x; t < sh_n; t += blockDim.x) {
            const size_t pos = (size_t)(sbase + t / PF_M) * PF_M + t % PF_M;
            pair_tok[pos] = sh_base + t;
            pair_k[pos] = topk;
            row_tok[rbase + t] = sh_base + t;
        }
        const int nsh = (sh_n + PF_M - 1) / PF_M;
        for (int q = threadIdx.x; q < nsh; q += blockDim.x) {
            slots[sbase + q].run = shared_run;
            slots[sbase + q].ntok = min(PF_M, sh_n - PF_M * q);
            slots[sbase + q].row0 = rbase + PF_M * q;
        }
        sbase += nsh;
        rbase += sh_n;
    }
    if (threadIdx.x == 0) {
        *n_slots = sbase;
        *n_rows = rbase;
    }
}

// Pair i of expert e goes to row r % 128 of slot slot_base[e] + r / 128, r its rank among all
// pairs of e (chunk base + rank within the chunk); its compact A row is eoff[e] + r
// (pair_row[i]; pairs that run nowhere here keep -1).
__global__ void __launch_bounds__(1024) k_pf_scatter(int *__restrict__ pair_tok, int *__restrict__ pair_k,
                                                     int *__restrict__ row_tok, int *__restrict__ pair_row,
                                                     const int *__restrict__ pe,
                                                     const int *__restrict__ rank, const int *__restrict__ chunk_base,
                                                     const int *__restrict__ slot_base, const int *__restrict__ eoff,
                                                     int P, int n_experts, int topk) {
    const int i = blockIdx.x * PF_CHUNK + threadIdx.x;
    if (i >= P) return;
    const int e = pe[i];
    if (e < 0) return;
    const int r = chunk_base[(size_t)blockIdx.x * n_experts + e] + rank[i];
    const size_t pos = (size_t)(slot_base[e] + r / PF_M) * PF_M + r % PF_M;
    pair_tok[pos] = i / topk;
    pair_k[pos] = i % topk;
    row_tok[eoff[e] + r] = i / topk;
    pair_row[i] = eoff[e] + r;
}

// Scale atoms of the A operand per slot: sfa [slot][J][H/128][512] from the per-token scales
// tsf [J][T][H/32] of each row's token (rows past the last row repeat the slot's first row;
// their products are never read).
__global__ void __launch_bounds__(256) k_pf_slot_sf(uint8_t *__restrict__ sfa, const uint8_t *__restrict__ tsf,
                                                    const int *__restrict__ row_tok,
                                                    const int *__restrict__ n_slots, const SlotPf *__restrict__ slots,
                                                    const int *__restrict__ n_rows, int T, int H) {
    const int s = blockIdx.x, j = blockIdx.y;
    if (s >= *n_slots) return;
    const int KT = H / 128, row0 = slots[s].row0, nr = *n_rows;
    for (int i = threadIdx.x; i < PF_M * KT; i += blockDim.x) {
        const int m = i % PF_M, kt = i / PF_M;
        const int r = row0 + m < nr ? row0 + m : row0;
        const int tok = row_tok[r];
        const uint32_t w = *reinterpret_cast<const uint32_t *>(tsf + ((size_t)j * T + tok) * (H / 32) + 4 * kt);
        *reinterpret_cast<uint32_t *>(sfa + (((size_t)s * PF_J + j) * KT + kt) * 512 + 16 * (m % 32) + 4 * (m / 32)) = w;
    }
}

// ------------------------------------------------------------------ persistent tcgen05 kernel
struct PfArgs {
    const int *n_list;        // slots this launch runs: list[0 .. *n_list)
    const int *list;
    const SlotPf *slots;
    const uint8_t *sfb;       // tail kernel: token scale atoms [slot][J][KT][512]
    const int *pair_tok, *pair_k;
    const uint8_t *arena;
    size_t run_stride;
    const uint8_t *sfa;       // A scale atoms [slot][J][KT][512]
    uint8_t *act_q;           // GU out: [J][rows_cap][I] E4M3, compact rows
    uint8_t *act_sf;          // GU out: [slot][J][I/128][512]
    uint16_t *contrib[K3C_EP_MAX];   // D out, bf16: rank q's [tmax][topk+1][H] (one rank: [0] = [T][..])
    int tmax;                     // pair token g lives on rank g / tmax, row g % tmax
    int kstride, T, H, I, act, rows_cap;
    int *err;
};

// 32 values of one thread -> J E4M3 terms (32 bytes each) and J UE8M0 scales, the split of
// quantize_block with the block held by one thread.
__device__ __forceinline__ void quant_row32(float (&a)[32], uint4 (&q)[PF_J][2], uint32_t (&sf)[PF_J]) {
#pragma unroll
    for (int j = 0; j < PF_J; j++) {
        float amax = 0.0f;
#pragma unroll
        for (int i = 0; i < 32; i++) amax = fmaxf(amax, fabsf(a[i]));
        const int e = block_exp(amax);
        sf[j] = (uint32_t)(e + 127);
        const float inv = exp2i(-e);
        uint32_t w[8];
#pragma unroll
        for (int i = 0; i < 8; i++) w[i] = 0u;
#pragma unroll
        for (int i = 0; i < 32; i++) {
            const uint32_t b = tc::f32_to_e4m3(a[i] * inv);
            w[i >> 2] |= b << (8 * (i & 3));
            const float back = tc::e4m3_to_f32(b);
            a[i] = a[i] - (e >= -126 ? back * exp2i(e) : (back * exp2i(-126)) * 0.5f);
        }
        q[j][0] = make_uint4(w[0], w[1], w[2], w[3]);
        q[j][1] = make_uint4(w[4], w[5], w[6], w[7]);
    }
}

// Where token g's activations are: rank g / tmax's buffer x[rank], row g % tmax (a peer's
// memory under expert parallelism, read with plain loads over NVLink); rows at or past that
// rank's ntok are quantised as zeros.
struct XSrc {
    const void *x[K3C_EP_MAX];
    int ntok[K3C_EP_MAX];
    int tmax;
    const uint8_t *need;   // tokens to quantise (NULL: all)
};

// Token g's J terms written straight into the compact A rows of its pairs (pair_row[g*topk+k],
// and its shared-expert row sh_row0 + g - sh_base when g is one of the shared tokens), and its
// block scales into xsf [J][T][H/32] (the slot scale atoms are built from them): every token
// read and quantised once, no per-token staging copy. One thread per 32-element block.
template <typename XT>
__global__ void __launch_bounds__(256) k_pf_quant_pairs(uint8_t *__restrict__ xq, uint8_t *__restrict__ xsf,
                                                        const XSrc src_x, const int *__restrict__ pair_row,
                                                        const int *__restrict__ sh_row0, int sh_base, int sh_n,
                                                        int T, int H, int topk, int rows_cap) {
    const int nb = H / 32;
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int r = (int)(i / nb), blk = (int)(i % nb);
    if (r >= T) return;
    if (src_x.need && !src_x.need[r]) return;   // no pair of this token runs here
    const int rq = r / src_x.tmax, tr = r % src_x.tmax;
    const bool live = tr < src_x.ntok[rq];
    const XT *src = reinterpret_cast<const XT *>(src_x.x[rq]) + (size_t)(live ? tr : 0) * H + blk * 32;
    float a[32];
    if constexpr (sizeof(XT) == 2) {
#pragma unroll
        for (int v = 0; v < 4; v++) {
            const uint4 u = reinterpret_cast<const uint4 *>(src)[v];
            const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
            for (int h = 0; h < 4; h++) {
                a[8 * v + 2 * h] = __uint_as_float(w[h] << 16);
                a[8 * v + 2 * h + 1] = __uint_as_float(w[h] & 0xFFFF0000u);
            }
        }
    } else {
#pragma unroll
        for (int v = 0; v < 8; v++) {
            const float4 f = reinterpret_cast<const float4 *>(src)[v];
            a[4 * v] = f.x;
            a[4 * v + 1] = f.y;
            a[4 * v + 2] = f.z;
            a[4 * v + 3] = f.w;
        }
    }
    if (!live)
#pragma unroll
        for (int v = 0; v < 32; v++) a[v] = 0.0f;
    uint4 q[PF_J][2];
    uint32_t sf[PF_J];
    quant_row32(a, q, sf);
#pragma unroll
    for (int j = 0; j < PF_J; j++) xsf[((size_t)j * T + r) * nb + blk] = (uint8_t)sf[j];
    const int sr0 = *sh_row0;
    for (int k = 0; k <= topk; k++) {
        int row;
        if (k < topk) row = pair_row[(size_t)r * topk + k];
        else row = (sr0 >= 0 && r >= sh_base && r < sh_base + sh_n) ? sr0 + (r - sh_base) : -1;
        if (row < 0) continue;
#pragma unroll
        for (int j = 0; j < PF_J; j++) {
            uint4 *d = reinterpret_cast<uint4 *>(xq + ((size_t)j * rows_cap + row) * H + blk * 32);
            d[0] = q[j][0];
            d[1] = q[j][1];
        }
    }
}

// The activation with the hardware exponential and divide: its result is requantised to two
// E4M3 terms right away, so the last-bit differences from act_apply do not survive.
__device__ __forceinline__ float act_fast(float g, float u, int act) {
    if (act == K3C_ACT_SWIGLU) return __fdividef(g, 1.0f + __expf(-g)) * u;
    return act_apply(g, u, act);
}

template <bool GU>
__global__ void __launch_bounds__(PF_THREADS) k_pf_moe(const __grid_constant__ CUtensorMap tmA,
                                                       const __grid_constant__ CUtensorMap tmW, PfArgs p) {
    extern __shared__ uint8_t pf_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(((uintptr_t)pf_raw + 1023) & ~(uintptr_t)1023);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + PF_STAGES * PF_STAGE);   // 256 bytes, then staging
    uint64_t *full = bars, *empty = bars + PF_STAGES, *tfull = bars + 2 * PF_STAGES, *tempty = tfull + 1;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(tempty + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int i = 0; i < PF_STAGES; i++) {
            tc::mbar_init(&full[i], 1);
            tc::mbar_init(&empty[i], 1);
        }
        tc::mbar_init(tfull, 1);
        tc::mbar_init(tempty, PF_EPI_WARPS);
        tc::fence_mbar_init();
    }
    if (warp == 1) tc::tmem_alloc(tmem_slot, PF_TMEM);
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    const int n_slots = *p.n_list;
    const int KT = GU ? p.H / 128 : p.I / 128;           // K tiles per item
    const int NTL = GU ? (2 * p.I) / PF_N : p.H / PF_N;  // N tiles per slot
    const int n_items = n_slots * NTL;
    const PoolGeom g = pool_geom(p.H, p.I);
    const size_t sf_off = GU ? g.gu_s : g.d_s;

    if (warp == 0) {
        // ---------------------------------------------------------------- producer
        if (lane == 0) {
            bool ok = tc::tc_check((tc::smem_u32(smem) & 1023) == 0, p.err, 40);
            tc::prefetch_tmap(&tmA);
            tc::prefetch_tmap(&tmW);
            uint32_t kiter = 0;
            for (int it = blockIdx.x; ok && it < n_items; it += gridDim.x) {
                const int s = p.list[it / NTL], nt = it % NTL;
                const SlotPf sl = p.slots[s];
                const uint8_t *wsf = p.arena + (size_t)sl.run * p.run_stride + sf_off;
                for (int kt = 0; kt < KT; kt++, kiter++) {
                    const int st = kiter % PF_STAGES;
                    const uint32_t ph = (kiter / PF_STAGES) & 1u;
                    if (kiter >= PF_STAGES && !tc::mbar_wait(&empty[st], ph ^ 1u, p.err, 41)) { ok = false; break; }
                    uint8_t *sa = smem + st * PF_STAGE;
                    uint8_t *sb = sa + PF_J * PF_A;
                    uint8_t *ssf = sb + PF_B;
                    tc::mbar_expect_tx(&full[st], PF_TX);
#pragma unroll
                    for (int j = 0; j < PF_J; j++) {
                        tc::tma_load_3d(sa + j * PF_A, &tmA, &full[st], kt * 128, sl.row0, j);
                        tc::bulk_load(ssf + j * 512, p.sfa + (((size_t)s * PF_J + j) * KT + kt) * 512, 512, &full[st]);
                    }
                    tc::tma_load_3d(sb, &tmW, &full[st], kt * 128, nt * PF_N, sl.run);
                    tc::bulk_load(ssf + PF_J * 512, wsf + ((size_t)(2 * nt) * KT + kt) * 512, 512, &full[st]);
                    tc::bulk_load(ssf + (PF_J + 1) * 512, wsf + ((size_t)(2 * nt + 1) * KT + kt) * 512, 512, &full[st]);
                }
            }
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------------- MMA issuer
        if (lane == 0) {
            uint32_t kiter = 0, li = 0;
            bool ok = true;
            const uint32_t idesc0 = tc::idesc_mxf8f6f4(tc::FMT_E4M3, tc::FMT_E2M1, PF_N, 0, 0);
            for (int it = blockIdx.x; ok && it < n_items; it += gridDim.x, li++) {
                if (li >= 1 && !tc::mbar_wait(tempty, (li - 1) & 1u, p.err, 44)) { ok = false; break; }
                tc::tc_fence_after();
                for (int kt = 0; kt < KT; kt++, kiter++) {
                    const int st = kiter % PF_STAGES;
                    const uint32_t ph = (kiter / PF_STAGES) & 1u;
                    if (!tc::mbar_wait(&full[st], ph, p.err, 42)) { ok = false; break; }
                    tc::tc_fence_after();
                    uint8_t *sa = smem + st * PF_STAGE;
                    uint8_t *sb = sa + PF_J * PF_A;
                    uint8_t *ssf = sb + PF_B;
                    const uint32_t sfc = tmem + PF_SF_COL + 16u * (kiter & 1u);
#pragma unroll
                    for (int j = 0; j < PF_J; j++) tc::tc_cp_sf(sfc + 4 * j, tc::desc_sf_atom(tc::smem_u32(ssf + j * 512)));
                    tc::tc_cp_sf(sfc + 8, tc::desc_sf_atom(tc::smem_u32(ssf + PF_J * 512)));
                    tc::tc_cp_sf(sfc + 12, tc::desc_sf_atom(tc::smem_u32(ssf + (PF_J + 1) * 512)));
#pragma unroll
                    for (int kb = 0; kb < 4; kb++) {
                        const uint64_t db = tc::desc_kmajor_sw128(tc::smem_u32(sb) + 32 * kb);
                        const uint32_t id = idesc0 | ((uint32_t)kb << 4) | ((uint32_t)kb << 29);
#pragma unroll
                        for (int j = 0; j < PF_J; j++) {
                            const uint64_t da = tc::desc_kmajor_sw128(tc::smem_u32(sa + j * PF_A) + 32 * kb);
                            tc::tc_mma_mx(tmem, da, db, id, (sfc + 4 * j) | ((uint32_t)kb << 30),
                                          (sfc + 8) | ((uint32_t)kb << 30), (kt | kb | j) != 0);
                        }
                    }
                    tc::tc_commit(&empty[st]);
                }
                if (ok) tc::tc_commit(tfull);
            }
        }
    } else {
        // ---------------------------------------------------------------- epilogue
        const int q = warp & 3;                 // TMEM lane quadrant
        const int half = (warp - 2) >> 2;       // which half of the item's columns
        const int m = 32 * q + lane;            // pair row of the slot
        const uint32_t lane_base = (uint32_t)(32 * q) << 16;
        uint32_t li = 0;
        for (int it = blockIdx.x; it < n_items; it += gridDim.x, li++) {
            const int s = p.list[it / NTL], nt = it % NTL;
            const bool ok = *(volatile int *)p.err == 0 && tc::mbar_wait(tfull, li & 1u, p.err, 43);
            __syncwarp();
            tc::tc_fence_after();
            const SlotPf sl = p.slots[s];
            // The whole accumulator slice of this thread goes to registers first and the
            // accumulator is released, so the next item's MMAs overlap the arithmetic and the
            // stores below.
            if (GU) {
                uint32_t vg[2][32], vu[2][32];
#pragma unroll
                for (int cc = 0; cc < 2; cc++) {
                    const int c = 2 * half + cc;
                    // gate columns of intermediate block c and the matching up columns
                    const uint32_t gcol = 128u * (c >> 1) + 32u * (c & 1);
                    tc::tmem_ld32(tmem + lane_base + gcol, vg[cc]);
                    tc::tmem_ld32(tmem + lane_base + gcol + 64, vu[cc]);
                }
                tc::tmem_ld_wait();
                tc::tc_fence_before();
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(tempty);
                const int KTd = p.I / 128;
#pragma unroll
                for (int cc = 0; cc < 2; cc++) {
                    const int c = 2 * half + cc;
                    if (!ok) continue;
                    float a[32];
#pragma unroll
                    for (int i = 0; i < 32; i++)
                        a[i] = act_fast(__uint_as_float(vg[cc][i]), __uint_as_float(vu[cc][i]), p.act);
                    uint4 qv[PF_J][2];
                    uint32_t sf[PF_J];
                    quant_row32(a, qv, sf);
                    if (m >= sl.ntok) continue;   // that row belongs to the next slot
                    const int col = 128 * nt + 64 * (c >> 1) + 32 * (c & 1);   // intermediate index
#pragma unroll
                    for (int j = 0; j < PF_J; j++) {
                        uint4 *dst = reinterpret_cast<uint4 *>(p.act_q + ((size_t)j * p.rows_cap + sl.row0 + m) * p.I + col);
                        dst[0] = qv[j][0];
                        dst[1] = qv[j][1];
                        p.act_sf[(((size_t)s * PF_J + j) * KTd + col / 128) * 512 + atom_byte(m, (col % 128) / 32)] =
                            (uint8_t)sf[j];
                    }
                }
            } else {
                constexpr int NC = PF_N / 64;   // 32-column chunks per half
                uint32_t v[NC][32];
#pragma unroll
                for (int cc = 0; cc < NC; cc++) tc::tmem_ld32(tmem + lane_base + 32u * (half * NC + cc), v[cc]);
                tc::tmem_ld_wait();
                tc::tc_fence_before();
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(tempty);
                // This thread's row goes to its pair's row of the token owner's buffer (NULL: the
                // row is past the slot's pairs). Each 32-column chunk is staged in shared memory
                // and stored by four lanes per row, so a warp's store covers 8 rows x 64
                // contiguous bytes instead of 32 rows x 16 bytes: the rows of a peer's buffer
                // cross NVLink in 64-byte writes.
                uint16_t *dst = nullptr;
                if (ok && m < sl.ntok) {
                    const size_t pr = (size_t)s * PF_M + m;
                    const int g = p.pair_tok[pr];
                    dst = p.contrib[g / p.tmax] + ((size_t)(g % p.tmax) * p.kstride + p.pair_k[pr]) * p.H +
                          (size_t)nt * PF_N + 32 * half * NC;
                }
                uint8_t *stg = smem + PF_STAGES * PF_STAGE + 256 + (warp - 2) * PF_STG;
                const uint32_t sw = (lane >> 1) & 3;   // 16-byte chunk swizzle of this lane's row
#pragma unroll
                for (int cc = 0; cc < NC; cc++) {
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        uint32_t w[4];
#pragma unroll
                        for (int k = 0; k < 4; k++)
                            w[k] = f32x2_to_bf16x2(__uint_as_float(v[cc][8 * i + 2 * k]),
                                                   __uint_as_float(v[cc][8 * i + 2 * k + 1]));
                        *reinterpret_cast<uint4 *>(stg + lane * 64 + 16 * (i ^ sw)) = make_uint4(w[0], w[1], w[2], w[3]);
                    }
                    __syncwarp();
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        const int r = (lane >> 2) + 8 * i, c = lane & 3;
                        const unsigned long long rd =
                            __shfl_sync(0xffffffffu, (unsigned long long)(uintptr_t)dst, r);
                        const uint4 val =
                            *reinterpret_cast<const uint4 *>(stg + r * 64 + 16 * (c ^ ((r >> 1) & 3)));
                        if (rd) *reinterpret_cast<uint4 *>(reinterpret_cast<uint8_t *>(rd) + cc * 64 + c * 16) = val;
                    }
                    __syncwarp();
                }
            }
        }
    }
    if constexpr (!GU) __threadfence_system();   // pair outputs may live in a peer's memory
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    if (warp == 1) tc::tmem_dealloc(tmem, PF_TMEM);
}

constexpr int PT_NMAX = 64;                     // pairs per tail slot at most (MMA N <= 64)

// ------------------------------------------------------------------ slot lists
// One block: slots of at most PT_NMAX pairs (an expert's last, partial slot) go to `tail`
// (k_pf_tail), the others to `full` (the kernel above), both in slot order. all_full: every
// slot to full.
__global__ void __launch_bounds__(1024) k_pf_split(int *__restrict__ full, int *__restrict__ n_full,
                                                   int *__restrict__ tail, int *__restrict__ n_tail,
                                                   const int *__restrict__ n_slots, const SlotPf *__restrict__ slots,
                                                   int all_full) {
    __shared__ int2 warp_sum[32];
    const int ns = *n_slots;
    int bf = 0, bt = 0;
    for (int s0 = 0; s0 < ns; s0 += blockDim.x) {
        const int s = s0 + threadIdx.x;
        const int f = s < ns && (all_full || slots[s].ntok > PT_NMAX);
        const int t = s < ns && !f;
        int xf, xt, tf, tt;
        block_scan2(f, t, xf, xt, tf, tt, warp_sum);
        if (f) full[bf + xf] = s;
        if (t) tail[bt + xt] = s;
        bf += tf;
        bt += tt;
    }
    if (threadIdx.x == 0) {
        *n_full = bf;
        *n_tail = bt;
    }
}

// ------------------------------------------------------------------ tail slots (swap A/B)
// A slot with n < 128 pairs wastes 128 - n rows of the kernel above. For n <= 64 the roles swap:
// the MMA's M side is 128 pool-format weight rows (GU: 64 gate + 64 up rows of one
// intermediate block of 64; D: 128 hidden rows) and N is the slot's pairs rounded up to 16,
// both E4M3 terms accumulating into one accumulator (two MMAs per K step, each with its own
// token scales). Work item = (tail slot, weight row tile). GU epilogue: the up rows' values
// go through shared memory to the gate rows' threads, which form SwiGLU and requantise each
// 32-column block across the warp (lane = intermediate column) into the same compact rows
// and slot scale atoms the D stages read. D epilogue: lane = hidden row, one coalesced store
// per pair.
// The kernel streams every tail expert's weights once with little math per byte, so the
// stages are small (8 KB of packed weights each) and many (six) to keep ~48 KB per SM in
// flight.
constexpr int PT_STAGES = 6;
constexpr int PT_A = 128 * 128;                 // padded E2M1 weight tile
constexpr int PT_BJ = PT_NMAX * 128;            // one term's token rows
constexpr int PT_STAGE = PT_A + PF_J * PT_BJ + 2048;   // + SFA and J SFB atoms (1024-aligned)
constexpr int PT_TILE = 64 * (PT_NMAX + 1) * 4; // up rows [64][PT_NMAX + 1] fp32
constexpr int PT_THREADS = 192;                 // producer, MMA, four epilogue warps
constexpr int PT_BYTES = 1024 + PT_STAGES * PT_STAGE + PT_TILE + 256;
constexpr uint32_t PT_TMEM = 256;               // two accumulators of PT_NMAX columns + scale factors
constexpr uint32_t PT_SF_COL = 2 * PT_NMAX;
static_assert(PT_BYTES <= 227 * 1024, "fits one CTA per SM");
static_assert(PT_STAGE % 1024 == 0, "stage bases stay 1024-byte aligned");

template <bool GU>
__global__ void __launch_bounds__(PT_THREADS) k_pf_tail(const __grid_constant__ CUtensorMap tmW,
                                                        const __grid_constant__ CUtensorMap tmB, PfArgs p) {
    extern __shared__ uint8_t pt_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(((uintptr_t)pt_raw + 1023) & ~(uintptr_t)1023);
    float *tile = reinterpret_cast<float *>(smem + PT_STAGES * PT_STAGE);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + PT_STAGES * PT_STAGE + PT_TILE);
    uint64_t *full = bars, *empty = bars + PT_STAGES, *tfull = bars + 2 * PT_STAGES, *tempty = tfull + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(tempty + 2);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int i = 0; i < 2 * PT_STAGES; i++) tc::mbar_init(&bars[i], 1);
        tc::mbar_init(&tfull[0], 1);
        tc::mbar_init(&tfull[1], 1);
        tc::mbar_init(&tempty[0], 4);
        tc::mbar_init(&tempty[1], 4);
        tc::fence_mbar_init();
    }
    if (warp == 1) tc::tmem_alloc(tmem_slot, PT_TMEM);
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    const int n_list = *p.n_list;
    const int KT = GU ? p.H / 128 : p.I / 128;         // K tiles per item
    const int RT = GU ? (2 * p.I) / 128 : p.H / 128;   // weight row tiles per slot
    const int n_items = n_list * RT;
    const PoolGeom g = pool_geom(p.H, p.I);
    const size_t sf_off = GU ? g.gu_s : g.d_s;

    if (warp == 0 && lane == 0) {
        // ------------------------------------------------------------ producer
        bool ok = tc::tc_check((tc::smem_u32(smem) & 1023) == 0, p.err, 50);
        tc::prefetch_tmap(&tmW);
        tc::prefetch_tmap(&tmB);
        uint32_t kiter = 0;
        for (int it = blockIdx.x; ok && it < n_items; it += gridDim.x) {
            const int s = p.list[it / RT], rt = it % RT;
            const SlotPf sl = p.slots[s];
            const int nb = (sl.ntok + 15) / 16;           // 16-row token boxes
            const uint8_t *wsf = p.arena + (size_t)sl.run * p.run_stride + sf_off + (size_t)rt * KT * 512;
            for (int kt = 0; kt < KT; kt++, kiter++) {
                const int st = kiter % PT_STAGES;
                const uint32_t ph = (kiter / PT_STAGES) & 1u;
                if (kiter >= PT_STAGES && !tc::mbar_wait(&empty[st], ph ^ 1u, p.err, 51)) { ok = false; break; }
                uint8_t *sa = smem + st * PT_STAGE;
                uint8_t *sb = sa + PT_A;
                uint8_t *ssf = sb + PF_J * PT_BJ;
                tc::mbar_expect_tx(&full[st], PT_A / 2 + PF_J * nb * 16 * 128 + (1 + PF_J) * 512);
                tc::tma_load_3d(sa, &tmW, &full[st], kt * 128, rt * 128, sl.run);
#pragma unroll
                for (int j = 0; j < PF_J; j++) {
                    for (int b = 0; b < nb; b++)
                        tc::tma_load_3d(sb + j * PT_BJ + b * 2048, &tmB, &full[st], kt * 128, sl.row0 + 16 * b, j);
                    tc::bulk_load(ssf + 512 * (1 + j), p.sfb + (((size_t)s * PF_J + j) * KT + kt) * 512, 512, &full[st]);
                }
                tc::bulk_load(ssf, wsf + (size_t)kt * 512, 512, &full[st]);
            }
        }
    } else if (warp == 1 && lane == 0) {
        // ------------------------------------------------------------ MMA issuer
        uint32_t kiter = 0, li = 0;
        bool ok = true;
        for (int it = blockIdx.x; ok && it < n_items; it += gridDim.x, li++) {
            const int s = p.list[it / RT];
            const uint32_t npad = (uint32_t)((p.slots[s].ntok + 15) & ~15);
            const uint32_t idesc0 = tc::idesc_mxf8f6f4(tc::FMT_E2M1, tc::FMT_E4M3, npad, 0, 0);
            const uint32_t a = li & 1u, use = li >> 1;
            if (use >= 1 && !tc::mbar_wait(&tempty[a], (use - 1) & 1u, p.err, 54)) { ok = false; break; }
            tc::tc_fence_after();
            const uint32_t d = tmem + a * PT_NMAX;
            for (int kt = 0; kt < KT; kt++, kiter++) {
                const int st = kiter % PT_STAGES;
                const uint32_t ph = (kiter / PT_STAGES) & 1u;
                if (!tc::mbar_wait(&full[st], ph, p.err, 52)) { ok = false; break; }
                tc::tc_fence_after();
                uint8_t *sa = smem + st * PT_STAGE;
                uint8_t *sb = sa + PT_A;
                uint8_t *ssf = sb + PF_J * PT_BJ;
                const uint32_t sfc = tmem + PT_SF_COL + 16u * (kiter & 1u);
                tc::tc_cp_sf(sfc, tc::desc_sf_atom(tc::smem_u32(ssf)));
#pragma unroll
                for (int j = 0; j < PF_J; j++)
                    tc::tc_cp_sf(sfc + 4 + 4 * j, tc::desc_sf_atom(tc::smem_u32(ssf + 512 * (1 + j))));
#pragma unroll
                for (int kb = 0; kb < 4; kb++) {
                    const uint64_t da = tc::desc_kmajor_sw128(tc::smem_u32(sa) + 32 * kb);
                    const uint32_t id = idesc0 | ((uint32_t)kb << 4) | ((uint32_t)kb << 29);
#pragma unroll
                    for (int j = 0; j < PF_J; j++) {
                        const uint64_t db = tc::desc_kmajor_sw128(tc::smem_u32(sb + j * PT_BJ) + 32 * kb);
                        tc::tc_mma_mx(d, da, db, id, sfc | ((uint32_t)kb << 30),
                                      (sfc + 4 + 4 * j) | ((uint32_t)kb << 30), (kt | kb | j) != 0);
                    }
                }
                tc::tc_commit(&empty[st]);
            }
            if (ok) tc::tc_commit(&tfull[a]);
        }
    } else if (warp >= 2) {
        // ------------------------------------------------------------ epilogue
        // Every epilogue warp runs every item and every named barrier even after a failed
        // wait (it then skips the TMEM reads and the stores), so no barrier strands a warp.
        const int q = warp & 3;                 // TMEM lane quadrant
        const int row = 32 * q + lane;          // weight row within the tile
        const uint32_t lane_base = (uint32_t)(32 * q) << 16;
        uint32_t li = 0;
        for (int it = blockIdx.x; it < n_items; it += gridDim.x, li++) {
            const int s = p.list[it / RT], rt = it % RT;
            const uint32_t a = li & 1u;
            const SlotPf sl = p.slots[s];
            const int n = sl.ntok;
            const bool ok = *(volatile int *)p.err == 0 && tc::mbar_wait(&tfull[a], (li >> 1) & 1u, p.err, 53);
            __syncwarp();
            tc::tc_fence_after();
            if constexpr (GU) {
                const int col = 64 * rt + (row & 63);       // intermediate index of this row
                const int KTd = p.I / 128;
#pragma unroll 1
                for (int c0 = 0; c0 < n; c0 += 32) {
                    uint32_t v[32];
                    if (ok) {
                        tc::tmem_ld32(tmem + lane_base + a * PT_NMAX + c0, v);
                        tc::tmem_ld_wait();
                    }
                    if (ok && q >= 2) {
#pragma unroll
                        for (int i = 0; i < 32; i++) tile[(row - 64) * (PT_NMAX + 1) + c0 + i] = __uint_as_float(v[i]);
                    }
                    tc::named_bar_sync(1, 128);
                    if (ok && q < 2) {
                        const int cn = min(32, n - c0);
#pragma unroll
                        for (int i = 0; i < 32; i++) {
                            if (i >= cn) break;
                            const int pl = c0 + i;
                            const float av = act_fast(__uint_as_float(v[i]), tile[row * (PT_NMAX + 1) + pl], p.act);
                            quantize_block<PF_J>(
                                av,
                                [&](int j, uint32_t qv) {
                                    p.act_q[((size_t)j * p.rows_cap + sl.row0 + pl) * p.I + col] = (uint8_t)qv;
                                },
                                [&](int j, uint32_t sf) {
                                    p.act_sf[(((size_t)s * PF_J + j) * KTd + col / 128) * 512 +
                                             atom_byte(pl, (col % 128) / 32)] = (uint8_t)sf;
                                });
                        }
                    }
                    tc::named_bar_sync(1, 128);           // the tile is rewritten by the next chunk
                }
            } else if (ok) {
                const int h = 128 * rt + row;
#pragma unroll 1
                for (int c0 = 0; c0 < n; c0 += 32) {
                    uint32_t v[32];
                    tc::tmem_ld32(tmem + lane_base + a * PT_NMAX + c0, v);
                    tc::tmem_ld_wait();
                    const int cn = min(32, n - c0);
#pragma unroll
                    for (int i = 0; i < 32; i++) {
                        if (i >= cn) break;
                        const size_t pr = (size_t)s * PF_M + c0 + i;
                        const int g = p.pair_tok[pr];
                        const float f = __uint_as_float(v[i]);
                        p.contrib[g / p.tmax][((size_t)(g % p.tmax) * p.kstride + p.pair_k[pr]) * p.H + h] =
                            (uint16_t)(f32x2_to_bf16x2(f, 0.0f) & 0xFFFFu);
                    }
                }
            }
            tc::tc_fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&tempty[a]);
        }
    }
    if constexpr (!GU) __threadfence_system();
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    if (warp == 1) tc::tmem_dealloc(tmem, PT_TMEM);
}

// ------------------------------------------------------------------ host side
struct PfBufs {
    int *idx, *pe, *rank, *cnt, *chunk_base, *slot_base, *eoff, *n_slots, *n_rows, *err, *pair_tok, *pair_k,
        *row_tok, *full_ids, *tail_ids, *n_full, *n_tail, *pair_row, *sh_row0;
    float *wt;
    uint16_t *contrib;
    double *rpart;
    uint8_t *dropped, *xq, *xsf, *sfa_x, *actq, *actsf;
    SlotPf *slots;
    int max_slots, nchunk, rows_cap;
};

static bool carve_pf(Carve &cv, PfBufs &b, const k3c_moe_pool_layer *L, int T, bool own_contrib = true) {
    const int H = L->hidden, I = L->inter, E = L->n_experts, K = L->topk;
    const size_t P = (size_t)T * K;
    b.nchunk = (int)((P + PF_CHUNK - 1) / PF_CHUNK);
    b.max_slots = (int)((P + PF_M - 1) / PF_M) + E + (T + PF_M - 1) / PF_M + 1;
    b.rows_cap = (int)P + T;
    b.idx = cv.take<int>(P);
    b.wt = cv.take<float>(P);
    b.rpart = cv.take<double>(router_scratch_bytes(H, E, T) / sizeof(double));
    b.pe = cv.take<int>(P);
    b.rank = cv.take<int>(P);
    b.dropped = cv.take<uint8_t>(P + T);   // + per-token need flags (expert parallelism)
    b.cnt = cv.take<int>((size_t)b.nchunk * E);
    b.chunk_base = cv.take<int>((size_t)b.nchunk * E);
    b.slot_base = cv.take<int>(E);
    b.eoff = cv.take<int>(E);
    b.n_slots = cv.take<int>(1);
    b.n_rows = cv.take<int>(1);
    b.err = cv.take<int>(1);
    b.slots = cv.take<SlotPf>(b.max_slots);
    b.full_ids = cv.take<int>(b.max_slots);
    b.tail_ids = cv.take<int>(b.max_slots);
    b.n_full = cv.take<int>(1);
    b.n_tail = cv.take<int>(1);
    b.pair_tok = cv.take<int>((size_t)b.max_slots * PF_M);
    b.pair_k = cv.take<int>((size_t)b.max_slots * PF_M);
    b.row_tok = cv.take<int>(b.rows_cap);
    b.xq = cv.take<uint8_t>((size_t)PF_J * b.rows_cap * H, 1024);
    b.pair_row = cv.take<int>(P);
    b.sh_row0 = cv.take<int>(1);
    b.xsf = cv.take<uint8_t>((size_t)PF_J * T * (H / 32));
    b.sfa_x = cv.take<uint8_t>((size_t)b.max_slots * PF_J * (H / 128) * 512);
    b.actq = cv.take<uint8_t>((size_t)PF_J * b.rows_cap * I, 1024);
    b.actsf = cv.take<uint8_t>((size_t)b.max_slots * PF_J * (I / 128) * 512);
    b.contrib = own_contrib ? cv.take<uint16_t>((size_t)T * (K + 1) * H) : reinterpret_cast<uint16_t *>(16);
    return b.idx && b.wt && b.rpart && b.pe && b.rank && b.dropped && b.cnt && b.chunk_base && b.slot_base &&
           b.eoff && b.n_slots && b.n_rows && b.err && b.slots && b.full_ids && b.tail_ids && b.n_full && b.n_tail &&
           b.pair_tok && b.pair_k && b.row_tok && b.xq &&
           b.pair_row && b.sh_row0 && b.xsf && b.sfa_x && b.actq && b.actsf && b.contrib;
}

static char *const kPfSizing = reinterpret_cast<char *>(4096);

// The combine over bf16 pair rows [ntok][topk+1][H]: out[t] = sum over k in top-k order of
// wt[t][k] * row[t][k] (fp32 product and sum, each rounded, as k3_ops.c:641-642 with
// -ffp-contract=off), then + row[t][topk] (the shared expert, unweighted). A pair is skipped
// when dropped[t*topk+k] is set (single GPU: the expert has no run here) or, under expert
// parallelism, when its expert id is outside [0, n_experts) or no rank holds it
// (expert_rank[e] < 0). Eight columns per thread (one 16-byte load per row).
__global__ void __launch_bounds__(128) k_pair_combine(float *__restrict__ out, const uint16_t *__restrict__ rows,
                                                      const float *__restrict__ wt, const uint8_t *__restrict__ dropped,
                                                      const int *__restrict__ ids, const int *__restrict__ expert_rank,
                                                      int n_experts, int topk, int h8, int has_shared) {
    const int t = blockIdx.y, ks = topk + 1;
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= h8) return;
    const uint4 *r4 = reinterpret_cast<const uint4 *>(rows) + (size_t)t * ks * h8 + c;
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; i++) acc[i] = 0.0f;
    auto add = [&](uint4 u, float w, bool weighted) {
        const uint32_t v[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const float lo = __uint_as_float(v[i] << 16), hi = __uint_as_float(v[i] & 0xFFFF0000u);
            acc[2 * i] = __fadd_rn(acc[2 * i], weighted ? __fmul_rn(w, lo) : lo);
            acc[2 * i + 1] = __fadd_rn(acc[2 * i + 1], weighted ? __fmul_rn(w, hi) : hi);
        }
    };
    constexpr int JM = 8;   // rows loaded ahead of their use
    for (int j0 = 0; j0 < topk; j0 += JM) {
        uint4 cj[JM];
        bool use[JM];
#pragma unroll
        for (int i = 0; i < JM; i++) {
            const int j = j0 + i, pi = t * topk + j;
            bool u = j < topk;
            if (u && dropped) u = !dropped[pi];
            if (u && ids) {
                const int e = ids[pi];
                u = (unsigned)e < (unsigned)n_experts && expert_rank[e] >= 0;
            }
            use[i] = u;
            if (u) cj[i] = r4[(size_t)j * h8];
        }
#pragma unroll
        for (int i = 0; i < JM; i++)
            if (use[i]) add(cj[i], wt[t * topk + j0 + i], true);
    }
    if (has_shared) add(r4[(size_t)topk * h8], 1.0f, false);
    float4 *o = reinterpret_cast<float4 *>(out + (size_t)t * 8 * h8) + 2 * c;
    o[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
    o[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
}

static int launch_pair_combine(float *out, const uint16_t *rows, const float *wt, const uint8_t *dropped,
                               const int *ids, const int *expert_rank, int n_experts, int ntok, int topk, int hidden,
                               int has_shared, cudaStream_t s) {
    if (ntok <= 0) return K3C_OK;
    if (hidden % 8 || ((uintptr_t)out & 15) || ((uintptr_t)rows & 15))
        return set_error(K3C_EINVAL, "pair_combine: hidden=%d (a multiple of 8) and 16-byte aligned rows", hidden);
    const int h8 = hidden / 8;
    k_pair_combine<<<dim3((h8 + 127) / 128, ntok), 128, 0, s>>>(out, rows, wt, dropped, ids, expert_rank, n_experts,
                                                                 topk, h8, has_shared);
    K3C_CHECK_LAUNCH();
    return K3C_OK;
}

size_t moe_prefill_tc_scratch(const k3c_moe_pool_layer *L, int T, bool own_contrib = true) {
    if (!L || T <= 0) return 0;
    Carve cv{kPfSizing, (size_t)-1 / 2, 0};
    PfBufs b;
    carve_pf(cv, b, L, T, own_contrib);
    return cv.used + 1024;
}

// Every rank's top-k ids, ranks after one another ([world*t_max][topk]); rows at or past a
// rank's token count get -1 (no pair), and so do the pairs of other ranks' tokens with an
// expert every rank holds (ep.local_only: its owner runs them). need[g] = 1 when token g has a
// pair on this rank (its expert resident here) or is this rank's own token with a shared
// expert: only those tokens are quantised.
__global__ void k_ep_gather_idx(int *__restrict__ all, uint8_t *__restrict__ need, k3c_ep_peers ep, int topk,
                                const int *__restrict__ run_of, int n_experts, int has_shared) {
    const int n = ep.world * ep.t_max;
    for (int g = blockIdx.x * blockDim.x + threadIdx.x; g < n; g += gridDim.x * blockDim.x) {
        const int q = g / ep.t_max, t = g % ep.t_max;
        const bool live = t < ep.ntok[q];
        bool here = live && has_shared && q == ep.rank;
        for (int k = 0; k < topk; k++) {
            int e = live ? ep.idx[q][(size_t)t * topk + k] : -1;
            if (ep.local_only && q != ep.rank && e >= 0 && e < n_experts && ep.local_only[e]) e = -1;
            all[(size_t)g * topk + k] = e;
            here |= e >= 0 && e < n_experts && run_of[e] >= 0;
        }
        need[g] = here;
    }
}

// routed: idx_out/wt_out hold the routing on entry (ids < 0 or not resident are skipped and
// counted in drops when it is given) and the router is not run.
// ep: expert-parallel step 2 (k3c_moe_prefill_ep_experts): T is world * t_max virtual tokens,
// x/idx come from the ranks' buffers, pair outputs go to the owning rank's contrib, no router,
// no drop counting and no combine.
int launch_moe_prefill_tc(float *out, const void *x, int x_dtype, int T, const k3c_moe_pool_layer *L,
                          int *idx_out, float *wt_out, int *drops, void *scratch, size_t scratch_bytes,
                          cudaStream_t s, bool routed = false, const k3c_ep_peers *ep = nullptr) {
    if (!L) return set_error(K3C_EINVAL, "moe_prefill_tc: null layer");
    const int H = L->hidden, I = L->inter, E = L->n_experts, K = L->topk;
    if (H <= 0 || I <= 0 || H % PF_N || I % 128)
        return set_error(K3C_EINVAL, "moe_prefill_tc: hidden=%d must be a multiple of 256, inter=%d of 128", H, I);
    if (T <= 0) return K3C_OK;
    if (K <= 0 || K > K3_MAX_TOPK || K > E) return set_error(K3C_EINVAL, "moe_prefill_tc: topk=%d", K);
    if (T > 65535 || ((long long)T * K + T) * H > (1LL << 40) || (long long)T * K + T > (1LL << 30))
        return set_error(K3C_EINVAL, "moe_prefill_tc: ntok=%d too large", T);
    if (x_dtype != K3C_BF16 && x_dtype != K3C_F32) return set_error(K3C_EINVAL, "moe_prefill_tc: x_dtype=%d", x_dtype);
    if (!ep && ((uintptr_t)x & 15) != 0) return set_error(K3C_EINVAL, "moe_prefill_tc: x must be 16-byte aligned");
    if (!L->arena || !L->run_of || L->n_runs <= 0 || L->run_stride % 256 ||
        L->run_stride < pool_geom(H, I).run || ((uintptr_t)L->arena & 255) || L->shared_run >= L->n_runs)
        return set_error(K3C_EINVAL, "moe_prefill_tc: bad arena");
    Carve cv{(char *)scratch, scratch_bytes, 0};
    PfBufs b;
    if (!carve_pf(cv, b, L, T, !ep))
        return set_error(K3C_EINVAL, "moe_prefill_tc: scratch too small (%zu)", scratch_bytes);
    int *idx = idx_out ? idx_out : b.idx;
    float *wt = wt_out ? wt_out : b.wt;
    const int P = T * K;
    if (routed && !ep && (!idx_out || !wt_out)) return set_error(K3C_EINVAL, "moe_prefill_tc_routed: null routing");
    if (ep) {
        routed = true;
        drops = nullptr;
        idx = b.idx;
        k_ep_gather_idx<<<sm_count() * 4, 256, 0, s>>>(idx, b.dropped + P, *ep, K, L->run_of, E,
                                                       L->shared_run >= 0 ? 1 : 0);
        K3C_CHECK_LAUNCH();
    }
    K3C_TRY_CUDA(cudaMemsetAsync(b.err, 0, sizeof(int), s));
    // scale atoms of rows past a slot's pairs stay 2^0 (never NaN)
    K3C_TRY_CUDA(cudaMemsetAsync(b.actsf, 127, (size_t)b.max_slots * PF_J * (I / 128) * 512, s));
    if (!routed) {
        stage_begin(STAGE_ROUTER, s);
        K3C_TRY(launch_router(idx, wt, nullptr, x, x_dtype, L->router_w, L->router_dtype, L->router_bias, H, E,
                              K, L->renorm, L->routed_scale, T, b.rpart, s));
        stage_end(STAGE_ROUTER, s);
    }
    // plan: counting sort of the pairs by expert
    const size_t csmem = ((size_t)E + PF_CHUNK) * sizeof(int);
    if (csmem > 48 * 1024) K3C_TRY_CUDA(cudaFuncSetAttribute(k_pf_count, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)csmem));
    k_pf_count<<<b.nchunk, PF_CHUNK, csmem, s>>>(b.pe, b.rank, b.cnt, b.dropped, drops, idx, P, L->run_of, E, L->n_runs);
    K3C_CHECK_LAUNCH();
    const int sh_base = ep ? ep->rank * ep->t_max : 0, sh_n = ep ? ep->ntok[ep->rank] : T;
    k_pf_slots<<<1, 1024, 0, s>>>(b.n_slots, b.slots, b.pair_tok, b.pair_k, b.row_tok, b.n_rows, b.chunk_base,
                                  b.slot_base, b.eoff, b.cnt, b.nchunk, L->run_of, E, sh_base, sh_n, K,
                                  L->shared_run, b.sh_row0);
    K3C_CHECK_LAUNCH();
    K3C_TRY_CUDA(cudaMemsetAsync(b.pair_row, 0xFF, (size_t)P * sizeof(int), s));   // -1: runs nowhere here
    k_pf_scatter<<<b.nchunk, PF_CHUNK, 0, s>>>(b.pair_tok, b.pair_k, b.row_tok, b.pair_row, b.pe, b.rank,
                                               b.chunk_base, b.slot_base, b.eoff, P, E, K);
    K3C_CHECK_LAUNCH();
    // every token read and quantised once, its terms stored in its pairs' compact rows; each slot's
    // scale atoms from the per-token scales
    const size_t nthr = (size_t)T * (H / 32);
    const unsigned qblocks = (unsigned)((nthr + 255) / 256);
    XSrc xs{};
    if (ep) {
        for (int q = 0; q < ep->world; q++) {
            xs.x[q] = ep->x[q];
            xs.ntok[q] = ep->ntok[q];
        }
        xs.tmax = ep->t_max;
        xs.need = b.dropped + P;
    } else {
        xs.x[0] = x;
        xs.ntok[0] = T;
        xs.tmax = T;
    }
    // expert parallelism: the other ranks' token rows may still be arriving on another stream
    if (ep && ep->x_ready) K3C_TRY_CUDA(cudaStreamWaitEvent(s, (cudaEvent_t)ep->x_ready, 0));
    stage_begin(STAGE_DISPATCH, s);
    if (x_dtype == K3C_BF16)
        k_pf_quant_pairs<uint16_t><<<qblocks, 256, 0, s>>>(b.xq, b.xsf, xs, b.pair_row, b.sh_row0, sh_base, sh_n, T, H,
                                                            K, b.rows_cap);
    else
        k_pf_quant_pairs<float><<<qblocks, 256, 0, s>>>(b.xq, b.xsf, xs, b.pair_row, b.sh_row0, sh_base, sh_n, T, H,
                                                         K, b.rows_cap);
    K3C_CHECK_LAUNCH();
    stage_end(STAGE_DISPATCH, s);
    k_pf_slot_sf<<<dim3(b.max_slots, PF_J), 256, 0, s>>>(b.sfa_x, b.xsf, b.row_tok, b.n_slots, b.slots, b.n_rows, T, H);
    K3C_CHECK_LAUNCH();
    // K3C_PF_TAIL=1: slots of at most PT_NMAX pairs on the weight-major kernel, the rest on the
    // token-major one. Off by default: with N of 16..64 a block-scaled MMA costs the tensor
    // pipe nearly as much as one with N = 256 (its pipe was 61% busy at 13% math), and the
    // split measured 5.58 ms for the config[2] expert stage against 4.90 ms with every slot
    // on the token-major kernel.
    const int use_tail = getenv("K3C_PF_TAIL") ? atoi(getenv("K3C_PF_TAIL")) : 0;
    k_pf_split<<<1, 1024, 0, s>>>(b.full_ids, b.n_full, b.tail_ids, b.n_tail, b.n_slots, b.slots, use_tail ? 0 : 1);
    K3C_CHECK_LAUNCH();
    // experts
    const PoolGeom g = pool_geom(H, I);
    CUtensorMap tmX, tmGU, tmAct, tmD;
    K3C_TRY(make_map3(&tmX, CU_TENSOR_MAP_DATA_TYPE_UINT8, b.xq, H, b.rows_cap, PF_J, H, (uint64_t)b.rows_cap * H, 128,
                      PF_M));
    K3C_TRY(make_map3(&tmGU, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, L->arena + g.gu_p, H, 2 * I, L->n_runs, H / 2,
                      L->run_stride, 128, PF_N));
    K3C_TRY(make_map3(&tmAct, CU_TENSOR_MAP_DATA_TYPE_UINT8, b.actq, I, b.rows_cap, PF_J, I, (uint64_t)b.rows_cap * I,
                      128, PF_M));
    K3C_TRY(make_map3(&tmD, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, L->arena + g.d_p, I, H, L->n_runs, I / 2,
                      L->run_stride, 128, PF_N));
    CUtensorMap tmX16, tmGU128, tmAct16, tmD128;   // the tail kernel's boxes
    K3C_TRY(make_map3(&tmX16, CU_TENSOR_MAP_DATA_TYPE_UINT8, b.xq, H, b.rows_cap, PF_J, H, (uint64_t)b.rows_cap * H,
                      128, 16));
    K3C_TRY(make_map3(&tmGU128, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, L->arena + g.gu_p, H, 2 * I, L->n_runs, H / 2,
                      L->run_stride, 128, 128));
    K3C_TRY(make_map3(&tmAct16, CU_TENSOR_MAP_DATA_TYPE_UINT8, b.actq, I, b.rows_cap, PF_J, I,
                      (uint64_t)b.rows_cap * I, 128, 16));
    K3C_TRY(make_map3(&tmD128, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, L->arena + g.d_p, I, H, L->n_runs, I / 2,
                      L->run_stride, 128, 128));
    PfArgs a;
    a.slots = b.slots;
    a.pair_tok = b.pair_tok;
    a.pair_k = b.pair_k;
    a.arena = L->arena;
    a.run_stride = L->run_stride;
    a.act_q = b.actq;
    a.act_sf = b.actsf;
    a.contrib[0] = b.contrib;   // one rank: the pair rows stay here ([T][topk+1][H])
    if (ep)                     // expert parallelism: each pair's row goes to its token's owner
        for (int q = 0; q < ep->world; q++) a.contrib[q] = ep->recv[q];
    // pair token g (of T = world * t_max under expert parallelism) is row g % tmax of rank
    // g / tmax's receive buffer, which holds t_max rows
    a.tmax = ep ? ep->t_max : T;
    a.kstride = K + 1;
    a.T = T;
    a.H = H;
    a.I = I;
    a.act = L->act;
    a.rows_cap = b.rows_cap;
    a.err = b.err;
    K3C_TRY_CUDA(cudaFuncSetAttribute(k_pf_moe<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, PF_BYTES));
    K3C_TRY_CUDA(cudaFuncSetAttribute(k_pf_moe<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, PF_BYTES));
    K3C_TRY_CUDA(cudaFuncSetAttribute(k_pf_tail<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, PT_BYTES));
    K3C_TRY_CUDA(cudaFuncSetAttribute(k_pf_tail<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, PT_BYTES));
    const int grid = sm_count();
    stage_begin(STAGE_EXPERTS, s);
    a.sfa = b.sfa_x;
    a.sfb = b.sfa_x;
    a.n_list = b.n_full;
    a.list = b.full_ids;
    k_pf_moe<true><<<grid, PF_THREADS, PF_BYTES, s>>>(tmX, tmGU, a);
    K3C_CHECK_LAUNCH();
    if (use_tail) {
        a.n_list = b.n_tail;
        a.list = b.tail_ids;
        k_pf_tail<true><<<grid, PT_THREADS, PT_BYTES, s>>>(tmGU128, tmX16, a);
        K3C_CHECK_LAUNCH();
    }
    a.sfa = b.actsf;
    a.sfb = b.actsf;
    a.n_list = b.n_full;
    a.list = b.full_ids;
    k_pf_moe<false><<<grid, PF_THREADS, PF_BYTES, s>>>(tmAct, tmD, a);
    K3C_CHECK_LAUNCH();
    if (use_tail) {
        a.n_list = b.n_tail;
        a.list = b.tail_ids;
        k_pf_tail<false><<<grid, PT_THREADS, PT_BYTES, s>>>(tmD128, tmAct16, a);
        K3C_CHECK_LAUNCH();
    }
    stage_end(STAGE_EXPERTS, s);
    if (!ep) {
        stage_begin(STAGE_COMBINE, s);
        K3C_TRY(launch_pair_combine(out, b.contrib, wt, b.dropped, nullptr, nullptr, 0, T, K, H,
                                    L->shared_run >= 0 ? 1 : 0, s));
        stage_end(STAGE_COMBINE, s);
    }
    // K3C_SYNC_CHECK=1: synchronise and report the kernels' own error code (a bounded wait
    // that gave up, or a failed alignment self-check). Off by default: it costs a host sync.
    static const int sync_check = getenv("K3C_SYNC_CHECK") ? 1 : 0;
    if (sync_check) {
        int code = 0;
        K3C_TRY_CUDA(cudaMemcpyAsync(&code, b.err, sizeof(int), cudaMemcpyDeviceToHost, s));
        K3C_TRY_CUDA(cudaStreamSynchronize(s));
        if (code) return set_error(K3C_ETIMEOUT, "moe_prefill_tc: device check code %d", code);
    }
    return K3C_OK;
}

}  // namespace k3c

extern "C" size_t k3c_moe_prefill_tc_scratch(const k3c_moe_pool_layer *L, int ntok) {
    return k3c::moe_prefill_tc_scratch(L, ntok);
}

extern "C" int k3c_moe_prefill_tc_routed(float *out, const void *x, int x_dtype, int ntok,
                                         const k3c_moe_pool_layer *L, const int *idx, const float *wt, int *drops,
                                         void *scratch, size_t scratch_bytes, k3c_stream_t stream) {
    k3c::clear_error();
    return k3c::launch_moe_prefill_tc(out, x, x_dtype, ntok, L, const_cast<int *>(idx), const_cast<float *>(wt),
                                      drops, scratch, scratch_bytes, (cudaStream_t)stream, true);
}

extern "C" int k3c_moe_prefill_tc(float *out, const void *x, int x_dtype, int ntok, const k3c_moe_pool_layer *L,
                                  int *idx, float *wt, int *drops, void *scratch, size_t scratch_bytes,
                                  k3c_stream_t stream) {
    k3c::clear_error();
    return k3c::launch_moe_prefill_tc(out, x, x_dtype, ntok, L, idx, wt, drops, scratch, scratch_bytes,
                                      (cudaStream_t)stream);
}

static int check_ep(const k3c_moe_pool_layer *L, const k3c_ep_peers *ep) {
    if (!L || !ep || ep->world < 1 || ep->world > K3C_EP_MAX || ep->rank < 0 || ep->rank >= ep->world ||
        ep->t_max <= 0 || (long long)ep->world * ep->t_max > 65535)
        return k3c::set_error(K3C_EINVAL, "moe_prefill_ep: bad peers (world, rank or t_max)");
    if (ep->x_dtype != K3C_BF16 && ep->x_dtype != K3C_F32)
        return k3c::set_error(K3C_EINVAL, "moe_prefill_ep: x_dtype=%d", ep->x_dtype);
    for (int q = 0; q < ep->world; q++)
        if (ep->ntok[q] < 0 || ep->ntok[q] > ep->t_max || !ep->x[q] || !ep->idx[q] || !ep->wt[q] ||
            !ep->recv[q] || ((uintptr_t)ep->x[q] & 15) || ((uintptr_t)ep->recv[q] & 15))
            return k3c::set_error(K3C_EINVAL, "moe_prefill_ep: rank %d's buffers (ntok %d)", q, ep->ntok[q]);
    if (L->hidden % 8) return k3c::set_error(K3C_EINVAL, "moe_prefill_ep: hidden=%d", L->hidden);
    return K3C_OK;
}

extern "C" size_t k3c_moe_prefill_ep_scratch(const k3c_moe_pool_layer *L, const k3c_ep_peers *peers) {
    if (check_ep(L, peers)) return 0;
    return k3c::moe_prefill_tc_scratch(L, peers->world * peers->t_max, false);   // pair rows go to peers
}

extern "C" int k3c_moe_ep_combine(float *out, const k3c_ep_peers *peers, int hidden, int topk,
                                  const int *expert_rank, int n_experts, int has_shared, k3c_stream_t stream) {
    k3c::clear_error();
    if (!peers || peers->world < 1 || peers->world > K3C_EP_MAX || peers->rank < 0 || peers->rank >= peers->world ||
        hidden <= 0 || topk <= 0 || topk > K3_MAX_TOPK || !expert_rank || n_experts <= 0 ||
        !peers->recv[peers->rank] || !peers->idx[peers->rank] || !peers->wt[peers->rank])
        return k3c::set_error(K3C_EINVAL, "moe_ep_combine: bad arguments");
    const int r = peers->rank;
    k3c::stage_begin(k3c::STAGE_COMBINE, (cudaStream_t)stream);
    const int rc = k3c::launch_pair_combine(out, peers->recv[r], peers->wt[r], nullptr, peers->idx[r], expert_rank,
                                            n_experts, peers->ntok[r], topk, hidden, has_shared, (cudaStream_t)stream);
    k3c::stage_end(k3c::STAGE_COMBINE, (cudaStream_t)stream);
    return rc;
}

extern "C" int k3c_moe_prefill_ep_experts(const k3c_moe_pool_layer *L, const k3c_ep_peers *peers, void *scratch,
                                          size_t scratch_bytes, k3c_stream_t stream) {
    k3c::clear_error();
    K3C_TRY(check_ep(L, peers));
    return k3c::launch_moe_prefill_tc(nullptr, nullptr, peers->x_dtype, peers->world * peers->t_max, L, nullptr,
                                      nullptr, nullptr, scratch, scratch_bytes, (cudaStream_t)stream, true, peers);
}

extern "C" int k3c_moe_combine(float *out, const float *contrib, const float *wt, const int *idx, int n_experts,
                               int ntok, int topk, int hidden, int has_shared, k3c_stream_t stream) {
    k3c::clear_error();
    if (ntok < 0 || topk <= 0 || topk > K3_MAX_TOPK || hidden <= 0 || (ntok > 0 && (!out || !contrib || !wt)))
        return k3c::set_error(K3C_EINVAL, "moe_combine: ntok=%d topk=%d hidden=%d", ntok, topk, hidden);
    return k3c::launch_moe_combine_ids(out, contrib, wt, nullptr, idx, n_experts, ntok, topk, hidden, has_shared,
                                       (cudaStream_t)stream);
}
