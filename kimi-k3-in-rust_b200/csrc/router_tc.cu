// router_tc.cu -- router logits on the tensor cores, exactly, for bf16 activations and bf16
// router weights at prefill sizes (the logit loop of src/core/k3_ops.c:445-452).
//
// Every bf16 value is an 8-bit integer times a power of two, so a dot product of two bf16
// rows is a sum of exact products. Each row (token or expert) is written on its own power of
// two 2^(E-6) with max|v| < 2^E as three balanced base-128 digits,
//     v = 2^(E-6) * (q0 + q1/128 + q2/128^2) + r,     |qj| <= 64,
// where the residual r is zero unless v is more than 13 binades below the row maximum (a few
// elements per 7168-wide Gaussian row). The digit part of the logit,
//     sum_k Rx[k] Rw[k] = 2^(Ex+Ew-12) * sum_{i,j} 128^-(i+j) * sum_k qx_i[k] qw_j[k],
// runs as kind::i8 MMAs with int32 accumulation (|sum| < 3 * 64 * 64 * 7168 < 2^31: exact),
// one TMEM accumulator per diagonal s = i+j. The residuals are kept as per-row lists of
// (k, r) and their terms, rx*w + Rx*rw (exact products), are added in double by the select
// kernel, which also computes a row's logits as a plain double dot product when a list
// overflowed or the row holds a NaN or an infinity. The double combination rounds like the
// reference's own double accumulator; the float rounding of the logit absorbs it.
#include <cuda.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>
#include <stdlib.h>

#include "common.cuh"
#include "rt_tc.cuh"
#include "tc_common.cuh"
#include "tc_host.cuh"

namespace k3c {

namespace {

// grid (ceil(rows/8)), 256 threads, one warp per row: digits, exponent and residual list of a
// bf16 row (H a multiple of 8). Digit j of row r goes to dig[j*rows*H + r*H + k]; list entry i
// of row r to ek/er[r*rs + i*is], in k order. Rows with a NaN or an infinity get zero digits
// and count cap+1. Warp-level reductions and scans only: a row is 28 loads of 16 bytes per lane
// at H = 7168, too little work to amortise block-wide barriers.
__global__ void __launch_bounds__(256) k_rt_digits(const uint16_t *__restrict__ src, int ld, int rows, int H,
                                                   int8_t *__restrict__ dig, int *__restrict__ exps,
                                                   int *__restrict__ cnt, int *__restrict__ ek,
                                                   float *__restrict__ er, int rs, int is, int cap) {
    const int lane = threadIdx.x & 31;
    const int r = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (r >= rows) return;
    const uint16_t *row = src + (size_t)r * ld;
    float m = 0.0f;
    int bad = 0;
    for (int k = lane * 8; k < H; k += 32 * 8) {
        const uint4 u = *reinterpret_cast<const uint4 *>(row + k);
        const uint32_t w4[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const float a = __uint_as_float(w4[i] << 16), b = __uint_as_float(w4[i] & 0xFFFF0000u);
            bad |= !(fabsf(a) <= 3.4e38f) | !(fabsf(b) <= 3.4e38f);
            m = fmaxf(m, fmaxf(fabsf(a), fabsf(b)));
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    bad = __any_sync(0xffffffffu, bad);
    int E = 0;
    if (!bad && m > 0.0f) frexpf(m, &E);                  // m < 2^E
    if (lane == 0) exps[r] = E;
    const size_t dstride = (size_t)rows * H;
    int8_t *d0 = dig + (size_t)r * H;
    int base = 0;
    for (int k0 = 0; k0 < H; k0 += 32 * 8) {
        const int k = k0 + lane * 8;
        uint32_t q[3][2] = {{0, 0}, {0, 0}, {0, 0}};
        float res[8];
        int nres = 0;
        if (k < H) {
            const uint4 u = *reinterpret_cast<const uint4 *>(row + k);
            const uint32_t w4[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const uint32_t b = (i & 1) ? (w4[i >> 1] & 0xFFFF0000u) : (w4[i >> 1] << 16);
                int a0 = 0, a1 = 0, a2 = 0;
                res[i] = bad ? 0.0f : rt_split(__uint_as_float(b), E, a0, a1, a2);
                q[0][i >> 2] |= (uint32_t)(a0 & 0xFF) << (8 * (i & 3));
                q[1][i >> 2] |= (uint32_t)(a1 & 0xFF) << (8 * (i & 3));
                q[2][i >> 2] |= (uint32_t)(a2 & 0xFF) << (8 * (i & 3));
                nres += res[i] != 0.0f;
            }
#pragma unroll
            for (int j = 0; j < 3; j++)
                *reinterpret_cast<uint2 *>(d0 + j * dstride + k) = make_uint2(q[j][0], q[j][1]);
        } else {
#pragma unroll
            for (int i = 0; i < 8; i++) res[i] = 0.0f;
        }
        // list entries in k order: warp-wide exclusive scan of the per-lane counts (most chunks
        // of an ordinary row have none)
        if (!__any_sync(0xffffffffu, nres != 0)) continue;
        int incl = nres;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += v;
        }
        int pos = base + incl - nres;
        if (nres) {
#pragma unroll
            for (int i = 0; i < 8; i++)
                if (res[i] != 0.0f) {
                    if (pos < cap) {
                        ek[(size_t)r * rs + (size_t)pos * is] = k + i;
                        er[(size_t)r * rs + (size_t)pos * is] = res[i];
                    }
                    pos++;
                }
        }
        base += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) cnt[r] = bad ? cap + 1 : base;
}

// ------------------------------------------------------------------ the MMA kernel
constexpr int RT_STAGE_A = 3 * 128 * 128;               // three token digits, 128 rows x 128 B
template <int N>
struct RtCfg {
    static constexpr int STAGE_B = 3 * N * 128;
    static constexpr int STAGE = RT_STAGE_A + STAGE_B;
    static constexpr int STAGES = (220 * 1024) / STAGE;
    static constexpr int COLS = 5 * N;                  // five diagonal accumulators
    static constexpr int TMEM = COLS <= 256 ? 256 : 512;
    static constexpr int SMEM = 1024 + STAGES * STAGE + 256;
};
constexpr int RT_THREADS = 192;   // warp 0 TMA, warp 1 MMA, warps 2-5 epilogue

struct RtArgs {
    double *part;         // [S][T][E]
    const int *xexp, *wexp;
    int T, E, KB, S;      // tokens, experts, 128-wide K blocks, K slices
    int *err;
};

// grid (ceil(E/N) * S, ceil(T/128)): CTA (et, slice) multiplies 128 tokens by N experts over
// K blocks [slice*KB/S, (slice+1)*KB/S).
template <int N>
__global__ void __launch_bounds__(RT_THREADS, 1) k_rt_tc(const __grid_constant__ CUtensorMap tmX,
                                                         const __grid_constant__ CUtensorMap tmW, RtArgs p) {
    using C = RtCfg<N>;
    extern __shared__ uint8_t rt_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(((uintptr_t)rt_raw + 1023) & ~(uintptr_t)1023);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + C::STAGES * C::STAGE);
    uint64_t *empty = full + C::STAGES;
    uint64_t *tfull = empty + C::STAGES;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(tfull + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int slice = blockIdx.x % p.S, et = blockIdx.x / p.S, tt = blockIdx.y;
    const int kb0 = (int)((long long)slice * p.KB / p.S), kb1 = (int)((long long)(slice + 1) * p.KB / p.S);
    const int nk = kb1 - kb0;
    if (threadIdx.x == 0) {
        for (int i = 0; i < C::STAGES; i++) {
            tc::mbar_init(&full[i], 1);
            tc::mbar_init(&empty[i], 1);
        }
        tc::mbar_init(tfull, 1);
        tc::fence_mbar_init();
    }
    if (warp == 1) tc::tmem_alloc(tmem_slot, C::TMEM);
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    if (warp == 0) {
        if (lane == 0) {
            bool ok = tc::tc_check((tc::smem_u32(smem) & 1023) == 0, p.err, 60);
            tc::prefetch_tmap(&tmX);
            tc::prefetch_tmap(&tmW);
            int issued = 0;
            for (int i = 0; ok && i < nk; i++) {
                const int st = i % C::STAGES;
                const uint32_t ph = (i / C::STAGES) & 1u;
                if (i >= C::STAGES && !tc::mbar_wait(&empty[st], ph ^ 1u, p.err, 61)) { ok = false; break; }
                uint8_t *sa = smem + st * C::STAGE;
                tc::mbar_expect_tx(&full[st], C::STAGE);
                tc::tma_load_3d(sa, &tmX, &full[st], (kb0 + i) * 128, tt * 128, 0);
                tc::tma_load_3d(sa + RT_STAGE_A, &tmW, &full[st], (kb0 + i) * 128, et * N, 0);
                issued = i + 1;
            }
            for (int i = issued - C::STAGES < 0 ? 0 : issued - C::STAGES; i < issued; i++)
                tc::mbar_wait(&full[i % C::STAGES], (i / C::STAGES) & 1u, p.err, 62);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t idesc = tc::idesc_i8(N);
            for (int i = 0; i < nk; i++) {
                const int st = i % C::STAGES;
                const uint32_t ph = (i / C::STAGES) & 1u;
                if (!tc::mbar_wait(&full[st], ph, p.err, 63)) break;
                tc::tc_fence_after();
                const uint32_t sa = tc::smem_u32(smem + st * C::STAGE), sb = sa + RT_STAGE_A;
#pragma unroll
                for (int kb = 0; kb < 4; kb++) {
                    uint32_t seen = 0;
#pragma unroll
                    for (int a = 0; a < 3; a++)
#pragma unroll
                        for (int b = 0; b < 3; b++) {
                            const int s = a + b;
                            const uint32_t acc = (i | kb) != 0 || ((seen >> s) & 1u);
                            seen |= 1u << s;
                            tc::tc_mma_i8(tmem + (uint32_t)(s * N),
                                          tc::desc_kmajor_sw128(sa + a * (128 * 128) + 32 * kb),
                                          tc::desc_kmajor_sw128(sb + b * (N * 128) + 32 * kb), idesc, acc);
                        }
                }
                tc::tc_commit(&empty[st]);
            }
            tc::tc_commit(tfull);
        }
    } else {
        const int q = warp & 3;
        const int row = 32 * q + lane, t = tt * 128 + row;
        const bool okt = tc::mbar_wait(tfull, 0, p.err, 64);
        __syncwarp();
        tc::tc_fence_after();
        const int ex = t < p.T ? p.xexp[t] : 0;
        double *out = p.part + ((size_t)slice * p.T + (t < p.T ? t : 0)) * p.E;
        const uint32_t lane_addr = tmem + ((uint32_t)(32 * q) << 16);
#pragma unroll 1
        for (int c0 = 0; c0 < N; c0 += 16) {
            uint32_t v[5][16];
#pragma unroll
            for (int s = 0; s < 5; s++) tc::tmem_ld16(lane_addr + s * N + c0, v[s]);
            tc::tmem_ld_wait();
#pragma unroll
            for (int c = 0; c < 16; c++) {
                const int e = et * N + c0 + c;
                const double sum = (double)(int)v[0][c] + (double)(int)v[1][c] * 0x1p-7 +
                                   (double)(int)v[2][c] * 0x1p-14 + (double)(int)v[3][c] * 0x1p-21 +
                                   (double)(int)v[4][c] * 0x1p-28;
                if (t < p.T && e < p.E)
                    out[e] = okt ? sum * rt_p2(ex + __ldg(p.wexp + e) - 12) : __longlong_as_double(0x7FF8000000000000ll);
            }
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    if (warp == 1) {
        tc::mbar_wait(tfull, 0, p.err, 65);
        tc::tmem_dealloc(tmem, C::TMEM);
    }
}

inline size_t up128(size_t v) { return (v + 127) & ~(size_t)127; }

struct RtBufs {
    int8_t *xd, *wd;
    double *part;
    int *xexp, *wexp, *xcnt, *wcnt, *xk, *wk;
    float *xr, *wr;
    size_t bytes;
};

RtBufs carve_rt(void *base, int H, int E, int T, int S) {
    RtBufs b{};
    uintptr_t o = base ? (((uintptr_t)base + 127) & ~(uintptr_t)127) : 0;
    const uintptr_t o0 = (uintptr_t)base;
    auto take = [&](size_t n) { uintptr_t r = o; o += up128(n); return r; };
    b.xd = (int8_t *)take((size_t)3 * T * H);
    b.wd = (int8_t *)take((size_t)3 * E * H);
    b.part = (double *)take((size_t)S * T * E * sizeof(double));
    b.xexp = (int *)take((size_t)T * 4);
    b.wexp = (int *)take((size_t)E * 4);
    b.xcnt = (int *)take((size_t)T * 4);
    b.wcnt = (int *)take((size_t)E * 4);
    b.xk = (int *)take((size_t)T * RT_CAP * 4);
    b.xr = (float *)take((size_t)T * RT_CAP * 4);
    b.wk = (int *)take((size_t)E * RT_CAP * 4);
    b.wr = (float *)take((size_t)E * RT_CAP * 4);
    b.bytes = (size_t)(o - o0) + 128;
    return b;
}

int make_digit_map(CUtensorMap *m, const int8_t *base, int H, int rows, int box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return set_error(K3C_ECUDA, "router_tc: cuTensorMapEncodeTiled unavailable");
    cuuint64_t dims[3] = {(cuuint64_t)H, (cuuint64_t)rows, 3};
    cuuint64_t strides[2] = {(cuuint64_t)H, (cuuint64_t)H * rows};
    cuuint32_t box[3] = {128, (cuuint32_t)box_rows, 3}, es[3] = {1, 1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<int8_t *>(base), dims, strides, box, es,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(K3C_ECUDA, "router_tc: tensor map encode failed (%d)", (int)r);
    return K3C_OK;
}

constexpr int RT_N = 96;

int rt_slices(int H, int E, int T) {
    const int KB = (H + 127) / 128;
    const int tiles = ((E + RT_N - 1) / RT_N) * ((T + 127) / 128);
    int S = sm_count() / tiles;
    if (const char *v = getenv("K3C_RT_SPLIT")) S = atoi(v);
    return S < 1 ? 1 : (S > KB ? KB : S);
}

}  // namespace

bool router_tc_applies(int x_dtype, int w_dtype, int hidden, int ntok) {
    int min_tok = RT_TC_MIN_TOKENS;
    if (const char *v = getenv("K3C_ROUTER_TC")) {
        if (v[0] == '0') return false;
        if (atoi(v) > 1) min_tok = atoi(v);   // K3C_ROUTER_TC=<n>: tensor cores from n tokens
    }
    return x_dtype == K3C_BF16 && w_dtype == K3C_BF16 && hidden % 16 == 0 && ntok >= min_tok;
}

size_t router_tc_scratch_bytes(int hidden, int n_experts, int ntok) {
    return carve_rt(nullptr, hidden, n_experts, ntok, rt_slices(hidden, n_experts, ntok)).bytes;
}

static __device__ int g_rt_err;

int router_tc_check(cudaStream_t s) {
    int *err = nullptr;
    K3C_TRY_CUDA(cudaGetSymbolAddress((void **)&err, g_rt_err));
    int code = 0;
    K3C_TRY_CUDA(cudaStreamSynchronize(s));
    K3C_TRY_CUDA(cudaMemcpy(&code, err, sizeof(int), cudaMemcpyDeviceToHost));
    if (code) {
        const int zero = 0;
        cudaMemcpy(err, &zero, sizeof(int), cudaMemcpyHostToDevice);
        return set_error(K3C_ETIMEOUT, "router_tc: device check code %d", code);
    }
    return K3C_OK;
}

// Digits of both operands and the MMA kernel; the select kernel then adds the S slices of
// *part in order and the residual terms described by *fix.
int launch_router_tc(RtFix *fix, double **part, int *nslices, const void *x, const void *W, int hidden,
                     int n_experts, int ntok, void *scratch, cudaStream_t s) {
    const int H = hidden, E = n_experts, T = ntok, S = rt_slices(H, E, T);
    if ((uintptr_t)x % 16 || (uintptr_t)W % 16 || H % 16)
        return set_error(K3C_EINVAL, "router_tc: x and W must be 16-byte aligned, hidden a multiple of 16");
    static int *err_of[64] = {};
    int *&err = err_of[cur_dev()];
    if (!err) K3C_TRY_CUDA(cudaGetSymbolAddress((void **)&err, g_rt_err));
    RtBufs b = carve_rt(scratch, H, E, T, S);
    k_rt_digits<<<(T + 7) / 8, 256, 0, s>>>((const uint16_t *)x, H, T, H, b.xd, b.xexp, b.xcnt, b.xk, b.xr, RT_CAP, 1, RT_CAP);
    K3C_CHECK_LAUNCH();
    k_rt_digits<<<(E + 7) / 8, 256, 0, s>>>((const uint16_t *)W, H, E, H, b.wd, b.wexp, b.wcnt, b.wk, b.wr, 1, E, RT_CAP);
    K3C_CHECK_LAUNCH();
    CUtensorMap mx, mw;
    K3C_TRY(make_digit_map(&mx, b.xd, H, T, 128));
    K3C_TRY(make_digit_map(&mw, b.wd, H, E, RT_N));
    using C = RtCfg<RT_N>;
    static bool attr_of[64] = {};
    bool &attr = attr_of[cur_dev()];
    if (!attr) {
        K3C_TRY_CUDA(cudaFuncSetAttribute(k_rt_tc<RT_N>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
        attr = true;
    }
    RtArgs a{b.part, b.xexp, b.wexp, T, E, (H + 127) / 128, S, err};
    const dim3 grid(((E + RT_N - 1) / RT_N) * S, (T + 127) / 128);
    k_rt_tc<RT_N><<<grid, RT_THREADS, C::SMEM, s>>>(mx, mw, a);
    K3C_CHECK_LAUNCH();
    *fix = RtFix{(const uint16_t *)x, (const uint16_t *)W, H, b.xexp, b.xcnt, b.xk, b.xr, b.wcnt, b.wk, b.wr, RT_CAP};
    *part = b.part;
    *nslices = S;
    return K3C_OK;
}

}  // namespace k3c
