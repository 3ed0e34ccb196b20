// q8.cu -- INT8 per-row-scaled trunk projection (reference k3_matmul_q8,
// src/core/k3_ops.c:1204-1272; layout include/k3/k3.h:265-303) on the tcgen05 tensor cores.
//
// The reference keeps each row inline as [f32 scale][int8 * in] with stride 4+in bytes,
// which is not 16-byte aligned at in = 7168. k3c_q8_pack rewrites it once into a pool
// layout: int8 rows of ldw bytes (ldw a multiple of 32, zero-padded) plus a separate fp32
// scale array, which TMA streams as 128x128-byte tiles.
//
// y[t][o] = wscale[o] * sum_i w[o][i] * x[t][i] is computed as an integer product:
//   * a small pre-kernel (k_q8_terms) splits each token's activations over each K slice of
//     the split-K into J = 4 signed 8-bit terms under one power-of-two scale 2^e per
//     (token, slice), e chosen so |x| / 2^e < 64:
//     x ~= 2^e * (q0 + q1/2^7 + q2/2^14 + q3/2^21), |qj| <= 64. Every bf16 value at least
//     2^-20 times the slice maximum is represented exactly; smaller ones carry an absolute
//     error below 2^(e-22). The GEMV is launched as its programmatic dependent, so its
//     first weight tiles stream while the terms are being written.
//   * tcgen05.mma kind::i8 multiplies the weight tile (M=128 rows, straight from TMA, no
//     conversion) by the J*16 term rows (N=64) into an int32 TMEM accumulator; int32 sums
//     of int8 products are exact (|acc| <= 127*64*in < 2^31 for in <= 262144).
//   * the epilogue forms 2^e * sum_j acc_j / 2^(7j) in double -- exact, the terms span 47
//     bits -- so a CTA's partial is the exact dot product of the represented activations.
//   * split-K: S CTAs take consecutive K slices of the same 128 output rows and store their
//     partials (L2-resident workspace); the last of them to finish (an atomic counter per
//     tile elects it) adds the S partials in slice order -- the result does not depend on
//     which CTA finishes last -- multiplies by the row scale and rounds once to fp32.
//     With S = 1 the CTA writes y directly. (Thread-block clusters with a shared-memory
//     reduction were tried first: at 7168x7168 the launch reported at most 33 active
//     clusters of 4 CTAs, so the 224-CTA grid ran in two waves.)
// The reference accumulates in fp32, so this result is the more accurate of the two; a
// token with a non-finite activation gets NaN outputs.
#include <cuda.h>
#include <cuda_runtime.h>
#include <float.h>
#include <stdlib.h>

#include "common.cuh"
#include "tc_common.cuh"
#include "tc_host.cuh"

namespace k3c {

__global__ void k_q8_pack(int8_t *__restrict__ wq, float *__restrict__ wscale, int ldw,
                          const uint8_t *__restrict__ rows, int in, int out) {
    const size_t rowb = (size_t)4 + in;
    for (int o = blockIdx.x; o < out; o += gridDim.x) {
        const uint8_t *r = rows + (size_t)o * rowb;
        if (threadIdx.x == 0) {
            uint32_t b = (uint32_t)r[0] | ((uint32_t)r[1] << 8) | ((uint32_t)r[2] << 16) |
                         ((uint32_t)r[3] << 24);
            wscale[o] = __int_as_float((int)b);
        }
        for (int i = threadIdx.x; i < ldw; i += blockDim.x)
            wq[(size_t)o * ldw + i] = i < in ? (int8_t)r[4 + i] : (int8_t)0;
    }
}

namespace {
constexpr int Q8_NT = 16;                // tokens per CTA
constexpr int Q8_J = 4;                  // int8 terms per activation
constexpr int Q8_N = Q8_J * Q8_NT;       // MMA N (term-major rows j*16 + t)
constexpr int Q8_A = 128 * 128;          // weight tile: 128 rows x 128 int8
constexpr int Q8_B = Q8_N * 128;         // term tile: 64 rows x 128 int8
constexpr int Q8_STAGE = Q8_A + Q8_B;
constexpr int q8_bytes(int stages) { return 1024 + stages * Q8_STAGE + 256; }
constexpr int Q8_THREADS = 192;          // warp 0 TMA, warp 1 MMA, warps 2-5 epilogue
constexpr int Q8_TMEM_COLS = 64;
constexpr int Q8_BAD = -0x7FFFFFFF;      // exponent slot of a token with a non-finite input
}  // namespace

struct Q8Args {
    float *y;
    int ldy, ntok, nslots;
    const int *texp;                     // [S][nslots] term exponent per (K slice, token slot)
    const float *wscale;
    int out, KT, S;
    double *part;                        // [TB][MT][S][16][128] partial sums
    int *count;                          // [TB][MT] finished slices, zeroed by the term kernel
    int *err;
};

static __device__ int g_q8_err;

// 2^e as a double, |e| <= 1022.
__device__ __forceinline__ double pow2d(int e) { return __longlong_as_double((long long)(e + 1023) << 52); }

__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename XT>
__device__ __forceinline__ float xval(const XT *p);
template <>
__device__ __forceinline__ float xval<float>(const float *p) { return *p; }
template <>
__device__ __forceinline__ float xval<uint16_t>(const uint16_t *p) { return bf16_bits_to_f32(*p); }

// V consecutive activations from k (zero at and beyond lim); whole 16-byte vectors when vec
// (row 16-byte aligned, k a multiple of 16 / sizeof(XT), V * sizeof(XT) a multiple of 16).
template <typename XT, int V>
__device__ __forceinline__ void load_x(const XT *row, int k, int lim, bool vec, float (&v)[V]) {
    static_assert((V * sizeof(XT)) % 16 == 0, "whole vectors");
    constexpr int E = 16 / sizeof(XT);   // elements per vector
    if (vec && k + V <= lim) {
#pragma unroll
        for (int u = 0; u < V / E; u++) {
            const uint4 w = *reinterpret_cast<const uint4 *>(row + k + u * E);
            const XT *e = reinterpret_cast<const XT *>(&w);
#pragma unroll
            for (int q = 0; q < E; q++) v[u * E + q] = xval<XT>(e + q);
        }
    } else {
#pragma unroll
        for (int q = 0; q < V; q++) v[q] = k + q < lim ? xval<XT>(row + k + q) : 0.0f;
    }
}

// grid (token slots, S): block (slot, s) covers K tiles [s*KT/S, (s+1)*KT/S) of one token
// slot (16 slots per token block, slots past ntok are zero). The slice maximum m fixes the
// exponent e (|x| / 2^e < 64), then the terms
//   terms[tb*64 + j*16 + t][k], j = 0..3, k in the slice (zero past `in`)
// are written for the TMA loads of the GEMV. texp[s][slot] = e, or Q8_BAD.
// Eight activations -> the J terms of each (8 bytes per term row) under 2^-e = inv.
__device__ __forceinline__ void split_terms8(const float (&v)[8], double inv, uint32_t (&w)[Q8_J][2]) {
#pragma unroll
    for (int j = 0; j < Q8_J; j++) w[j][0] = w[j][1] = 0u;
#pragma unroll
    for (int q = 0; q < 8; q++) {
        float r = (float)((double)v[q] * inv);   // exact, |r| < 64
#pragma unroll
        for (int j = 0; j < Q8_J; j++) {
            const float qv = rintf(r);
            r = (r - qv) * 128.0f;                // exact remainder, |r| <= 64
            w[j][q >> 2] |= ((uint32_t)(int)qv & 0xFFu) << (8 * (q & 3));
        }
    }
}

template <typename XT>
__global__ void __launch_bounds__(256) k_q8_terms(int8_t *__restrict__ terms, int *__restrict__ texp,
                                                  int *__restrict__ count, int ncount,
                                                  const XT *__restrict__ x, int ldx, int ntok, int in,
                                                  int kpad, int KT, int vec) {
    constexpr int R = 2;   // chunks of 8 held in registers per thread: slices up to 4096 load once
    grid_dep_launch();     // the GEMV may start streaming weights now
    if (blockIdx.x == 0 && blockIdx.y == 0)
        for (int i = threadIdx.x; i < ncount; i += 256) count[i] = 0;
    __shared__ float wm[8];
    __shared__ int wb[8];
    const int slot = blockIdx.x, tb = slot / Q8_NT, t = slot % Q8_NT;
    const int S = gridDim.y, sl = blockIdx.y;
    const int k_lo = (int)((long long)sl * KT / S) * 128, k_end = (int)((long long)(sl + 1) * KT / S) * 128;
    const int k_hi = min(k_end, in);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const bool real = slot < ntok;
    const XT *xr = x + (size_t)(real ? slot : 0) * ldx;
    float keep[R][8];
    float m = 0.0f;
    int bad = 0;
#pragma unroll
    for (int r = 0; r < R; r++) {
        const int k = k_lo + (threadIdx.x + 256 * r) * 8;
        if (real && k < k_hi) load_x<XT, 8>(xr, k, k_hi, vec != 0, keep[r]);
        else
#pragma unroll
            for (int q = 0; q < 8; q++) keep[r][q] = 0.0f;
    }
    for (int k = k_lo + (threadIdx.x + 256 * R) * 8; real && k < k_hi; k += 256 * 8) {
        float v[8];
        load_x<XT, 8>(xr, k, k_hi, vec != 0, v);
#pragma unroll
        for (int q = 0; q < 8; q++) {
            bad |= !(fabsf(v[q]) <= FLT_MAX);
            m = fmaxf(m, fabsf(v[q]));
        }
    }
#pragma unroll
    for (int r = 0; r < R; r++)
#pragma unroll
        for (int q = 0; q < 8; q++) {
            bad |= !(fabsf(keep[r][q]) <= FLT_MAX);
            m = fmaxf(m, fabsf(keep[r][q]));
        }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    bad = __any_sync(0xffffffffu, bad);
    if (lane == 0) {
        wm[warp] = m;
        wb[warp] = bad;
    }
    __syncthreads();
    m = wm[0];
    bad = wb[0];
    for (int w = 1; w < 8; w++) {
        m = fmaxf(m, wm[w]);
        bad |= wb[w];
    }
    int ex = 0;
    frexpf(m, &ex);                                   // m < 2^ex
    const int e = (m > 0.0f && !bad) ? ex - 6 : 0;
    if (threadIdx.x == 0) texp[(size_t)sl * gridDim.x + slot] = bad ? Q8_BAD : e;
    const double inv = pow2d(-e);
    const bool live = real && !bad;
    int8_t *trow = terms + (size_t)(tb * Q8_N + t) * kpad;
#pragma unroll
    for (int r = 0; r < R; r++) {
        const int k = k_lo + (threadIdx.x + 256 * r) * 8;
        if (k < k_end) {
            uint32_t w[Q8_J][2];
            if (!live)
#pragma unroll
                for (int q = 0; q < 8; q++) keep[r][q] = 0.0f;
            split_terms8(keep[r], inv, w);
#pragma unroll
            for (int j = 0; j < Q8_J; j++)
                *reinterpret_cast<uint2 *>(trow + (size_t)j * Q8_NT * kpad + k) = make_uint2(w[j][0], w[j][1]);
        }
    }
    for (int k = k_lo + (threadIdx.x + 256 * R) * 8; k < k_end; k += 256 * 8) {
        float v[8];
        if (live) load_x<XT, 8>(xr, k, in, vec != 0, v);
        else
#pragma unroll
            for (int q = 0; q < 8; q++) v[q] = 0.0f;
        uint32_t w[Q8_J][2];
        split_terms8(v, inv, w);
#pragma unroll
        for (int j = 0; j < Q8_J; j++)
            *reinterpret_cast<uint2 *>(trow + (size_t)j * Q8_NT * kpad + k) = make_uint2(w[j][0], w[j][1]);
    }
}

// grid (S * MT, TB): CTA (mt, rank) multiplies rows [128*mt, 128*mt+128) by K tiles
// [rank*KT/S, (rank+1)*KT/S) for token block blockIdx.y.
template <int Q8_STAGES>
__global__ void __launch_bounds__(Q8_THREADS) k_q8_tc(const __grid_constant__ CUtensorMap tmW,
                                                      const __grid_constant__ CUtensorMap tmT, Q8Args p) {
    extern __shared__ uint8_t q8_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(((uintptr_t)q8_raw + 1023) & ~(uintptr_t)1023);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + Q8_STAGES * Q8_STAGE);
    uint64_t *empty = full + Q8_STAGES;
    uint64_t *tfull = empty + Q8_STAGES;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(tfull + 1);
    int *last = reinterpret_cast<int *>(tmem_slot + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int S = p.S;
    const int rank = blockIdx.x % S;                       // K slice
    const int mt = blockIdx.x / S;                         // 128-row output tile
    const int MT = gridDim.x / S;
    const int tb = blockIdx.y;
    const int t0 = tb * Q8_NT;
    const int nt = min(Q8_NT, p.ntok - t0);
    const int kt0 = (int)((long long)rank * p.KT / S), kt1 = (int)((long long)(rank + 1) * p.KT / S);
    const int nk = kt1 - kt0;

    if (threadIdx.x == 0) {
        for (int i = 0; i < Q8_STAGES; i++) {
            tc::mbar_init(&full[i], 1);
            tc::mbar_init(&empty[i], 1);
        }
        tc::mbar_init(tfull, 1);
        tc::fence_mbar_init();
    }
    if (warp == 1) tc::tmem_alloc(tmem_slot, Q8_TMEM_COLS);
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---------------------------------------------------------------- producer
        if (lane == 0) {
            bool ok = tc::tc_check((tc::smem_u32(smem) & 1023) == 0, p.err, 30);
            tc::prefetch_tmap(&tmW);
            tc::prefetch_tmap(&tmT);
            const uint64_t pol = tc::l2_evict_first_policy();
            // weights of the first stages need nothing from the term kernel: start them first
            const int pre = ok ? min(nk, Q8_STAGES) : 0;
            for (int i = 0; i < pre; i++) {
                tc::mbar_expect_tx(&full[i], Q8_A + Q8_B);
                tc::tma_load_3d_hint(smem + i * Q8_STAGE, &tmW, &full[i], (kt0 + i) * 128, mt * 128, 0, pol);
            }
            grid_dep_wait();
            for (int i = 0; i < pre; i++)
                tc::tma_load_3d(smem + i * Q8_STAGE + Q8_A, &tmT, &full[i], (kt0 + i) * 128, tb * Q8_N, 0);
            int issued = pre;
            for (int i = pre; ok && i < nk; i++) {
                const int st = i % Q8_STAGES;
                const uint32_t ph = (i / Q8_STAGES) & 1u;
                if (!tc::mbar_wait(&empty[st], ph ^ 1u, p.err, 31)) { ok = false; break; }
                uint8_t *sa = smem + st * Q8_STAGE;
                tc::mbar_expect_tx(&full[st], Q8_A + Q8_B);
                tc::tma_load_3d_hint(sa, &tmW, &full[st], (kt0 + i) * 128, mt * 128, 0, pol);
                tc::tma_load_3d(sa + Q8_A, &tmT, &full[st], (kt0 + i) * 128, tb * Q8_N, 0);
                issued = i + 1;
            }
            // every issued copy has landed before the CTA can leave (immediate when consumed)
            for (int i = issued - Q8_STAGES < 0 ? 0 : issued - Q8_STAGES; i < issued; i++)
                tc::mbar_wait(&full[i % Q8_STAGES], (i / Q8_STAGES) & 1u, p.err, 32);
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------------- MMA issuer
        if (lane == 0) {
            const uint32_t idesc = tc::idesc_i8(Q8_N);
            for (int i = 0; i < nk; i++) {
                const int st = i % Q8_STAGES;
                const uint32_t ph = (i / Q8_STAGES) & 1u;
                if (!tc::mbar_wait(&full[st], ph, p.err, 33)) break;
                tc::tc_fence_after();
                const uint32_t sa = tc::smem_u32(smem + st * Q8_STAGE), sb = sa + Q8_A;
#pragma unroll
                for (int kb = 0; kb < 4; kb++)
                    tc::tc_mma_i8(tmem, tc::desc_kmajor_sw128(sa + 32 * kb), tc::desc_kmajor_sw128(sb + 32 * kb),
                                  idesc, (i | kb) != 0);
                tc::tc_commit(&empty[st]);
            }
            tc::tc_commit(tfull);   // also after a failed wait: lets the CTA drain its MMAs
        }
    } else {
        // ---------------------------------------------------------------- epilogue
        grid_dep_wait();                        // texp is written by the term kernel
        const int q = warp & 3;                 // TMEM lane quadrant
        const int row = 32 * q + lane;
        const bool okt = tc::mbar_wait(tfull, 0, p.err, 36);
        __syncwarp();
        tc::tc_fence_after();
        uint32_t v[64];
        tc::tmem_ld32(tmem + ((uint32_t)(32 * q) << 16), *reinterpret_cast<uint32_t(*)[32]>(v));
        tc::tmem_ld32(tmem + ((uint32_t)(32 * q) << 16) + 32, *reinterpret_cast<uint32_t(*)[32]>(v + 32));
        tc::tmem_ld_wait();
        const int o = mt * 128 + row;
        double *mine = S > 1 ? p.part + (((size_t)tb * MT + mt) * S + rank) * (Q8_NT * 128) : nullptr;
        // the 16 exponents in one round trip (lane t holds token t's), not one load per token
        const int my_e = p.texp[(size_t)rank * p.nslots + t0 + (lane & (Q8_NT - 1))];
        double own[Q8_NT];
#pragma unroll
        for (int tk = 0; tk < Q8_NT; tk++) {
            const int e = __shfl_sync(0xffffffffu, my_e, tk);
            double part = (double)(int)v[tk] + (double)(int)v[16 + tk] * 0x1p-7 +
                          (double)(int)v[32 + tk] * 0x1p-14 + (double)(int)v[48 + tk] * 0x1p-21;
            own[tk] = (e == Q8_BAD || !okt) ? __longlong_as_double(0x7FF8000000000000ll) : part * pow2d(e);
            if (S > 1) __stcg(mine + tk * 128 + row, own[tk]);
        }
        bool finish = S == 1;
        if (S > 1) {
            // publish the partial; the last slice of the tile to finish adds all S of them
            __threadfence();
            tc::named_bar_sync(1, 128);
            if (threadIdx.x == 64) *last = atomicAdd(p.count + (size_t)tb * MT + mt, 1) == S - 1;
            tc::named_bar_sync(1, 128);
            finish = *last != 0;
            if (finish) {
                __threadfence();
                const double *all = p.part + ((size_t)tb * MT + mt) * S * (Q8_NT * 128);
                double acc[Q8_NT];
#pragma unroll
                for (int tk = 0; tk < Q8_NT; tk++) acc[tk] = 0.0;
                for (int r = 0; r < S; r++) {   // slice order, whichever CTA finishes last
                    double v2[Q8_NT];
                    if (r == rank) {
#pragma unroll
                        for (int tk = 0; tk < Q8_NT; tk++) v2[tk] = own[tk];
                    } else {
#pragma unroll
                        for (int tk = 0; tk < Q8_NT; tk++) v2[tk] = __ldcg(all + (size_t)r * (Q8_NT * 128) + tk * 128 + row);
                    }
#pragma unroll
                    for (int tk = 0; tk < Q8_NT; tk++) acc[tk] += v2[tk];
                }
#pragma unroll
                for (int tk = 0; tk < Q8_NT; tk++) own[tk] = acc[tk];
            }
        }
        if (finish && o < p.out) {
            const double sc = (double)p.wscale[o];
#pragma unroll
            for (int tk = 0; tk < Q8_NT; tk++)
                if (tk < nt) p.y[(size_t)(t0 + tk) * p.ldy + o] = (float)(own[tk] * sc);
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    if (warp == 1) {
        tc::mbar_wait(tfull, 0, p.err, 37);
        tc::tmem_dealloc(tmem, Q8_TMEM_COLS);
    }
}

int launch_q8_pack(int8_t *wq, float *wscale, int ldw, const void *rows, int in, int out,
                   cudaStream_t s) {
    if (in <= 0 || out <= 0 || ldw < in || (ldw % 16))
        return set_error(K3C_EINVAL, "q8_pack: in=%d out=%d ldw=%d", in, out, ldw);
    k_q8_pack<<<out < 4096 ? out : 4096, 256, 0, s>>>(wq, wscale, ldw, (const uint8_t *)rows, in, out);
    K3C_CHECK_LAUNCH();
    return K3C_OK;
}

// Pipeline depth and split-K factor. Deep: 8 stages (192 KB, one CTA per SM); shallow: 4
// stages (96 KB, two CTAs per SM). The split S keeps the grid within one wave of resident
// CTAs, at most 16 and at most the K tile count. K3C_Q8_STAGES=4|8 and K3C_Q8_SPLIT=<1..16>
// override the defaults (tuning sweeps).
static int q8_stages() {
    static const int forced = getenv("K3C_Q8_STAGES") ? atoi(getenv("K3C_Q8_STAGES")) : 0;
    return forced == 4 ? 4 : 8;
}
static int q8_split(int tiles, int KT, int per_sm) {
    static const int forced = getenv("K3C_Q8_SPLIT") ? atoi(getenv("K3C_Q8_SPLIT")) : 0;
    int S = forced >= 1 && forced <= 16 ? forced : (sm_count() * per_sm) / (tiles > 0 ? tiles : 1);
    if (S > 16) S = 16;
    if (S > KT) S = KT;
    return S < 1 ? 1 : S;
}

// The launch geometry and the device scratch of one projection: split-K partials (double),
// the activation terms, their exponents and the per-tile arrival counters.
struct Q8Plan {
    int KT, kpad, MT, TB, stages, S;
    size_t term_bytes, part_bytes, texp_bytes, total;
};
static Q8Plan q8_plan(int ntok, int in, int out) {
    Q8Plan p;
    p.KT = (in + 127) / 128;
    p.kpad = p.KT * 128;
    p.MT = (out + 127) / 128;
    p.TB = (ntok + Q8_NT - 1) / Q8_NT;
    p.stages = q8_stages();
    p.S = q8_split(p.MT * p.TB, p.KT, p.stages == 8 ? 1 : 2);
    p.term_bytes = (size_t)p.TB * Q8_N * p.kpad;
    p.part_bytes = p.S > 1 ? (size_t)p.TB * p.MT * p.S * Q8_NT * 128 * sizeof(double) : 0;
    p.texp_bytes = align_up((size_t)p.S * p.TB * Q8_NT * sizeof(int), 256);
    p.total = p.part_bytes + p.term_bytes + p.texp_bytes + (size_t)p.TB * p.MT * sizeof(int);
    return p;
}

// scratch: caller-owned device memory of at least q8_plan().total bytes, 256-byte aligned, or
// nullptr to take it from the stream-ordered pool for this call.
template <typename XT>
static int launch_q8_tc(float *y, int ldy, const void *x, int ldx, int ntok, const int8_t *wq,
                        const float *wscale, int ldw, int in, int out, void *scratch, cudaStream_t s) {
    static int *err_of[64] = {};
    int *&err = err_of[cur_dev()];
    if (!err) K3C_TRY_CUDA(cudaGetSymbolAddress((void **)&err, g_q8_err));
    const Q8Plan p = q8_plan(ntok, in, out);
    const int KT = p.KT, kpad = p.kpad, MT = p.MT, TB = p.TB, stages = p.stages, S = p.S;
    const size_t term_bytes = p.term_bytes, part_bytes = p.part_bytes, texp_bytes = p.texp_bytes;
    char *buf = reinterpret_cast<char *>(scratch);
    if (!buf) {
        k3c::keep_async_pool();
        K3C_TRY_CUDA(cudaMallocAsync((void **)&buf, p.total, s));
    }
    double *part = reinterpret_cast<double *>(buf);
    int8_t *terms = reinterpret_cast<int8_t *>(buf + part_bytes);
    int *texp = reinterpret_cast<int *>(buf + part_bytes + term_bytes);
    int *count = reinterpret_cast<int *>(buf + part_bytes + term_bytes + texp_bytes);
    int rc = K3C_OK;
    do {
        CUtensorMap tmW, tmT;
        rc = make_map3(&tmW, CU_TENSOR_MAP_DATA_TYPE_UINT8, wq, ldw, out, 1, ldw, (uint64_t)ldw * out, 128, 128);
        if (rc) break;
        rc = make_map3(&tmT, CU_TENSOR_MAP_DATA_TYPE_UINT8, terms, kpad, (uint64_t)TB * Q8_N, 1, kpad,
                       term_bytes, 128, Q8_N);
        if (rc) break;
        const int vec = ((uintptr_t)x % 16 == 0) && (ldx % (int)(16 / sizeof(XT)) == 0);
        k_q8_terms<XT><<<dim3(TB * Q8_NT, S), 256, 0, s>>>(terms, texp, count, TB * MT, (const XT *)x, ldx, ntok,
                                                           in, kpad, KT, vec);
        count_launch();
        if (cudaGetLastError() != cudaSuccess) { rc = set_error(K3C_ECUDA, "q8_gemv: term kernel launch failed"); break; }
        Q8Args a;
        a.y = y;
        a.ldy = ldy;
        a.ntok = ntok;
        a.nslots = TB * Q8_NT;
        a.texp = texp;
        a.wscale = wscale;
        a.out = out;
        a.KT = KT;
        a.S = S;
        a.part = part;
        a.count = count;
        a.err = err;
        auto kern = stages == 8 ? k_q8_tc<8> : k_q8_tc<4>;
        const int smem = q8_bytes(stages);
        cudaError_t ce = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (ce == cudaSuccess) ce = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
        cudaLaunchConfig_t cfg = {};
        cudaLaunchAttribute at[1];
        at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        at[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.gridDim = dim3(a.S * MT, TB, 1);
        cfg.blockDim = dim3(Q8_THREADS, 1, 1);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = s;
        cfg.attrs = at;
        cfg.numAttrs = 1;
        if (ce == cudaSuccess) ce = cudaLaunchKernelEx(&cfg, kern, tmW, tmT, a);
        count_launch();
        if (ce != cudaSuccess) rc = set_error(K3C_ECUDA, "q8_gemv: %s", cudaGetErrorString(ce));
    } while (0);
    if (!scratch) cudaFreeAsync(buf, s);
    if (rc) return rc;
    // K3C_SYNC_CHECK=1: synchronise and report the kernel's own error code (a bounded wait
    // that gave up, or a failed alignment self-check).
    static const int sync_check = getenv("K3C_SYNC_CHECK") ? 1 : 0;
    if (sync_check) {
        int code = 0;
        K3C_TRY_CUDA(cudaStreamSynchronize(s));
        K3C_TRY_CUDA(cudaMemcpy(&code, err, sizeof(int), cudaMemcpyDeviceToHost));
        if (code) {
            const int zero = 0;
            cudaMemcpy(err, &zero, sizeof(int), cudaMemcpyHostToDevice);
            return set_error(K3C_ETIMEOUT, "q8_gemv: device check code %d", code);
        }
    }
    return K3C_OK;
}

static int launch_q8_gemv_impl(float *y, int ldy, const void *x, int x_dtype, int ldx, int ntok,
                               const int8_t *wq, const float *wscale, int ldw, int in, int out, void *scratch,
                               cudaStream_t s) {
    if (in <= 0 || out <= 0 || ldw < in || (ldw % 32) || ((uintptr_t)wq & 15) || in > 262144)
        return set_error(K3C_EINVAL, "q8_gemv: in=%d out=%d ldw=%d (ldw must be a multiple of 32, in <= 262144)",
                         in, out, ldw);
    if (ntok < 0 || (ntok > 0 && (ldy < out || ldx < in)))
        return set_error(K3C_EINVAL, "q8_gemv: ntok=%d ldy=%d ldx=%d", ntok, ldy, ldx);
    if (ntok == 0) return K3C_OK;
    if (x_dtype == K3C_BF16) return launch_q8_tc<uint16_t>(y, ldy, x, ldx, ntok, wq, wscale, ldw, in, out, scratch, s);
    if (x_dtype == K3C_F32) return launch_q8_tc<float>(y, ldy, x, ldx, ntok, wq, wscale, ldw, in, out, scratch, s);
    return set_error(K3C_EINVAL, "q8_gemv: x_dtype=%d", x_dtype);
}

int launch_q8_gemv(float *y, int ldy, const void *x, int x_dtype, int ldx, int ntok,
                   const int8_t *wq, const float *wscale, int ldw, int in, int out,
                   cudaStream_t s) {
    return launch_q8_gemv_impl(y, ldy, x, x_dtype, ldx, ntok, wq, wscale, ldw, in, out, nullptr, s);
}

size_t q8_scratch_bytes(int ntok, int in, int out) {
    if (ntok <= 0 || in <= 0 || out <= 0) return 0;
    return q8_plan(ntok, in, out).total + 256;
}

int launch_q8_gemv_ws(float *y, int ldy, const void *x, int x_dtype, int ldx, int ntok, const int8_t *wq,
                      const float *wscale, int ldw, int in, int out, void *scratch, size_t scratch_bytes,
                      cudaStream_t s) {
    if (ntok <= 0 || in <= 0 || out <= 0)
        return launch_q8_gemv_impl(y, ldy, x, x_dtype, ldx, ntok, wq, wscale, ldw, in, out, nullptr, s);
    const size_t need = q8_plan(ntok, in, out).total;
    char *base = reinterpret_cast<char *>(((uintptr_t)scratch + 255) & ~(uintptr_t)255);
    if (!scratch || (size_t)(base - (char *)scratch) + need > scratch_bytes)
        return set_error(K3C_EINVAL, "q8_gemv: scratch of %zu bytes, %zu needed", scratch_bytes, need + 256);
    return launch_q8_gemv_impl(y, ldy, x, x_dtype, ldx, ntok, wq, wscale, ldw, in, out, base, s);
}

}  // namespace k3c

extern "C" int k3c_q8_pack(int8_t *wq, float *wscale, int ldw, const void *w_rows, int in,
                           int out, k3c_stream_t stream) {
    k3c::clear_error();
    return k3c::launch_q8_pack(wq, wscale, ldw, w_rows, in, out, (cudaStream_t)stream);
}

extern "C" int k3c_q8_gemv(float *y, int ldy, const void *x, int x_dtype, int ldx, int ntok,
                           const int8_t *wq, const float *wscale, int ldw, int in, int out,
                           k3c_stream_t stream) {
    k3c::clear_error();
    k3c::stage_begin(k3c::STAGE_Q8, (cudaStream_t)stream);
    int rc = k3c::launch_q8_gemv(y, ldy, x, x_dtype, ldx, ntok, wq, wscale, ldw, in, out,
                                 (cudaStream_t)stream);
    k3c::stage_end(k3c::STAGE_Q8, (cudaStream_t)stream);
    return rc;
}

extern "C" size_t k3c_q8_gemv_scratch(int ntok, int in, int out) { return k3c::q8_scratch_bytes(ntok, in, out); }

extern "C" int k3c_q8_gemv_ws(float *y, int ldy, const void *x, int x_dtype, int ldx, int ntok, const int8_t *wq,
                              const float *wscale, int ldw, int in, int out, void *scratch, size_t scratch_bytes,
                              k3c_stream_t stream) {
    k3c::clear_error();
    k3c::stage_begin(k3c::STAGE_Q8, (cudaStream_t)stream);
    int rc = k3c::launch_q8_gemv_ws(y, ldy, x, x_dtype, ldx, ntok, wq, wscale, ldw, in, out, scratch, scratch_bytes,
                                    (cudaStream_t)stream);
    k3c::stage_end(k3c::STAGE_Q8, (cudaStream_t)stream);
    return rc;
}
