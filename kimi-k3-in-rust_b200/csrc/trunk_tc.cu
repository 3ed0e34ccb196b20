// trunk_tc.cu -- bf16 trunk matrices on the tensor cores, for many tokens:
//     y[t][o] (+)= sum_i W[o][i] x[t][i],   W bf16 [out][in] (the row layout of the reference's
//     k3_mmw, include/k3/k3.h:289-296), x fp32 [T][in], y fp32.
// The activations enter as two bf16 terms, x = hi + lo with hi = bf16(x) and lo = bf16(x - hi)
// (x - hi is exact in fp32; |x - hi - lo| <= 2^-17 |x|), and both terms are multiplied into one
// fp32 TMEM accumulator by tcgen05.mma kind::f16 (bf16 x bf16 products are exact in fp32). The
// result is not bit-exact with the reference's double accumulator (k3_matmul_bf16,
// src/core/k3_ops.c:1091-1196) -- the drop-ins and the few-token layer keep the exact k_mmw --
// but lies within ~1e-6 of the sum's magnitude, far inside the MoE layer's 2e-2 bar.
//
// k_tg_split writes the two terms of every activation row, K padded with zeros to a multiple of
// 64; k_tg_gemm is one 128-token x 256-row tile per CTA: warp 0 streams 64-wide K blocks of
// both activation terms and of W through a 3-stage TMA ring (128-byte swizzle; W rows past
// `out` and K past `in` read as zeros), warp 1 issues 2 x 4 MMAs (M128 N256 K16) per K block,
// warps 2-5 drain the accumulator (one token row per thread) into y.
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdlib.h>

#include "common.cuh"
#include "tc_common.cuh"
#include "tc_host.cuh"

namespace k3c {

namespace {

constexpr int TG_M = 128;                       // tokens per tile
constexpr int TG_N = 256;                       // W rows per tile
constexpr int TG_KB = 64;                       // bf16 per K block (128 bytes)
constexpr int TG_A = 2 * TG_M * 128;            // both activation terms of a K block
constexpr int TG_B = TG_N * 128;
constexpr int TG_STAGE = TG_A + TG_B;           // 64 KB
constexpr int TG_STAGES = 3;
constexpr int TG_SMEM = 1024 + TG_STAGES * TG_STAGE + 256;
constexpr int TG_THREADS = 192;                 // warp 0 TMA, warp 1 MMA, warps 2-5 epilogue

// kind::f16 instruction descriptor: bf16 A and B, both K-major, fp32 accumulator, M = 128.
__host__ __device__ constexpr uint32_t idesc_bf16(uint32_t n) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((n >> 3) << 17) | ((128u >> 4) << 24);
}

__device__ __forceinline__ void tc_mma_f16(uint32_t tmem_d, uint64_t desc_a, uint64_t desc_b, uint32_t idesc,
                                           uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(desc_a), "l"(desc_b), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Two bf16 terms of x: a[t][k] = hi, a[T*Kp + t*Kp + k] = lo, zeros for k in [in, Kp).
// One thread per 8 consecutive k of one row.
__global__ void __launch_bounds__(256) k_tg_split(uint16_t *__restrict__ a, const float *__restrict__ x, int ldx,
                                                  int T, int in, int Kp) {
    const int groups = Kp / 8;
    const size_t n = (size_t)T * groups;
    const size_t plane = (size_t)T * Kp;
    for (size_t g = (size_t)blockIdx.x * blockDim.x + threadIdx.x; g < n; g += (size_t)gridDim.x * blockDim.x) {
        const int t = (int)(g / groups), k = (int)(g % groups) * 8;
        const float *xr = x + (size_t)t * ldx + k;
        uint32_t hi[4], lo[4];
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const float v0 = k + 2 * j < in ? xr[2 * j] : 0.0f;
            const float v1 = k + 2 * j + 1 < in ? xr[2 * j + 1] : 0.0f;
            hi[j] = f32x2_to_bf16x2(v0, v1);
            const float h0 = __uint_as_float(hi[j] << 16), h1 = __uint_as_float(hi[j] & 0xFFFF0000u);
            lo[j] = f32x2_to_bf16x2(v0 - h0, v1 - h1);
        }
        *reinterpret_cast<uint4 *>(a + (size_t)t * Kp + k) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
        *reinterpret_cast<uint4 *>(a + plane + (size_t)t * Kp + k) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    }
}

struct TgArgs {
    float *y;
    int ldy, T, out, KB, accumulate, vec;
    int *err;
};

// grid (ceil(T/128), ceil(out/256)): CTA (tt, nt) computes tokens [128 tt, +128) x rows
// [256 nt, +256) over all K blocks.
__global__ void __launch_bounds__(TG_THREADS, 1) k_tg_gemm(const __grid_constant__ CUtensorMap tmA,
                                                           const __grid_constant__ CUtensorMap tmW, TgArgs p) {
    extern __shared__ uint8_t tg_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(((uintptr_t)tg_raw + 1023) & ~(uintptr_t)1023);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + TG_STAGES * TG_STAGE);
    uint64_t *empty = full + TG_STAGES;
    uint64_t *tfull = empty + TG_STAGES;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(tfull + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tt = blockIdx.x, nt = blockIdx.y;
    if (threadIdx.x == 0) {
        for (int i = 0; i < TG_STAGES; i++) {
            tc::mbar_init(&full[i], 1);
            tc::mbar_init(&empty[i], 1);
        }
        tc::mbar_init(tfull, 1);
        tc::fence_mbar_init();
    }
    if (warp == 1) tc::tmem_alloc(tmem_slot, TG_N);
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    if (warp == 0) {
        if (lane == 0) {
            bool ok = tc::tc_check((tc::smem_u32(smem) & 1023) == 0, p.err, 70);
            tc::prefetch_tmap(&tmA);
            tc::prefetch_tmap(&tmW);
            int issued = 0;
            for (int i = 0; ok && i < p.KB; i++) {
                const int st = i % TG_STAGES;
                const uint32_t ph = (i / TG_STAGES) & 1u;
                if (i >= TG_STAGES && !tc::mbar_wait(&empty[st], ph ^ 1u, p.err, 71)) { ok = false; break; }
                uint8_t *sa = smem + st * TG_STAGE;
                tc::mbar_expect_tx(&full[st], TG_STAGE);
                tc::tma_load_3d(sa, &tmA, &full[st], i * 128, tt * TG_M, 0);
                tc::tma_load_3d(sa + TG_A, &tmW, &full[st], i * 128, nt * TG_N, 0);
                issued = i + 1;
            }
            // no copy may still be landing when the CTA exits
            for (int i = issued - TG_STAGES < 0 ? 0 : issued - TG_STAGES; i < issued; i++)
                tc::mbar_wait(&full[i % TG_STAGES], (i / TG_STAGES) & 1u, p.err, 72);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_bf16(TG_N);
            for (int i = 0; i < p.KB; i++) {
                const int st = i % TG_STAGES;
                const uint32_t ph = (i / TG_STAGES) & 1u;
                if (!tc::mbar_wait(&full[st], ph, p.err, 73)) break;
                tc::tc_fence_after();
                const uint32_t sa = tc::smem_u32(smem + st * TG_STAGE), sb = sa + TG_A;
#pragma unroll
                for (int term = 0; term < 2; term++)
#pragma unroll
                    for (int k = 0; k < 4; k++)
                        tc_mma_f16(tmem, tc::desc_kmajor_sw128(sa + term * (TG_M * 128) + 32 * k),
                                   tc::desc_kmajor_sw128(sb + 32 * k), idesc, (i | term | k) != 0);
                tc::tc_commit(&empty[st]);
            }
            tc::tc_commit(tfull);
        }
    } else {
        const int q = warp & 3;
        const int t = tt * TG_M + 32 * q + lane;
        const bool okt = tc::mbar_wait(tfull, 0, p.err, 74);
        __syncwarp();
        tc::tc_fence_after();
        const uint32_t lane_addr = tmem + ((uint32_t)(32 * q) << 16);
        float *yr = p.y + (size_t)(t < p.T ? t : 0) * p.ldy;
#pragma unroll 1
        for (int c0 = 0; c0 < TG_N; c0 += 32) {
            uint32_t v[32];
            tc::tmem_ld32(lane_addr + c0, v);
            tc::tmem_ld_wait();
            const int n0 = nt * TG_N + c0;
            if (t >= p.T || n0 >= p.out) continue;
            float f[32];
#pragma unroll
            for (int j = 0; j < 32; j++) f[j] = okt ? __uint_as_float(v[j]) : __int_as_float(0x7FC00000);
            if (p.vec && n0 + 32 <= p.out) {
                float4 *dst = reinterpret_cast<float4 *>(yr + n0);
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    float4 o = make_float4(f[4 * j], f[4 * j + 1], f[4 * j + 2], f[4 * j + 3]);
                    if (p.accumulate) {
                        const float4 a = dst[j];
                        o = make_float4(__fadd_rn(a.x, o.x), __fadd_rn(a.y, o.y), __fadd_rn(a.z, o.z),
                                        __fadd_rn(a.w, o.w));
                    }
                    dst[j] = o;
                }
            } else {
#pragma unroll
                for (int j = 0; j < 32; j++)
                    if (n0 + j < p.out) yr[n0 + j] = p.accumulate ? __fadd_rn(yr[n0 + j], f[j]) : f[j];
            }
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    if (warp == 1) {
        tc::mbar_wait(tfull, 0, p.err, 75);
        tc::tmem_dealloc(tmem, TG_N);
    }
}

int make_map_terms(CUtensorMap *m, const uint16_t *a, int T, int Kp) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return set_error(K3C_ECUDA, "mmw_tc: cuTensorMapEncodeTiled unavailable");
    cuuint64_t dims[3] = {(cuuint64_t)Kp * 2, (cuuint64_t)T, 2};
    cuuint64_t strides[2] = {(cuuint64_t)Kp * 2, (cuuint64_t)Kp * 2 * T};
    cuuint32_t box[3] = {128, (cuuint32_t)TG_M, 2}, es[3] = {1, 1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<uint16_t *>(a), dims, strides, box, es,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(K3C_ECUDA, "mmw_tc: tensor map encode failed (%d)", (int)r);
    return K3C_OK;
}

static __device__ int g_tg_err;

}  // namespace

static int kpad64(int in) { return (in + TG_KB - 1) / TG_KB * TG_KB; }

// Bytes of the two-term activation buffer of ntok rows of width in (256-byte aligned start).
size_t mmw_tc_terms_bytes(int ntok, int in) {
    if (ntok <= 0 || in <= 0) return 0;
    return (size_t)2 * ntok * kpad64(in) * sizeof(uint16_t) + 256;
}

// Whether a matrix can take the tensor-core path: bf16 rows 16-byte aligned (in a multiple of
// 8, W 16-byte aligned). K3C_TRUNK_EXACT=1 keeps every trunk matrix on the exact k_mmw.
bool mmw_tc_applies(const void *W, int in) {
    static const int exact = getenv("K3C_TRUNK_EXACT") ? atoi(getenv("K3C_TRUNK_EXACT")) : 0;
    return !exact && W && in > 0 && in % 8 == 0 && ((uintptr_t)W % 16) == 0;
}

// The two bf16 terms of x [ntok][ldx] (width in) into terms (mmw_tc_terms_bytes).
int launch_mmw_tc_split(void *terms, const float *x, int ldx, int ntok, int in, cudaStream_t s) {
    if (ntok <= 0) return K3C_OK;
    if (!terms || !x || in <= 0 || ldx < in) return set_error(K3C_EINVAL, "mmw_tc: split in=%d ldx=%d", in, ldx);
    uint16_t *a = reinterpret_cast<uint16_t *>(((uintptr_t)terms + 255) & ~(uintptr_t)255);
    const int Kp = kpad64(in);
    const size_t groups = (size_t)ntok * (Kp / 8);
    const unsigned grid = (unsigned)((groups + 255) / 256 < 4096 ? (groups + 255) / 256 : 4096);
    k_tg_split<<<grid, 256, 0, s>>>(a, x, ldx, ntok, in, Kp);
    K3C_CHECK_LAUNCH();
    count_launch();
    return K3C_OK;
}

// y (+)= W x for the split activations in terms (launch_mmw_tc_split of the same ntok and in).
int launch_mmw_tc_gemm(float *y, int ldy, const void *terms, int ntok, const void *W, int in, int out,
                       int accumulate, cudaStream_t s) {
    if (ntok <= 0 || out <= 0) return K3C_OK;
    if (!mmw_tc_applies(W, in) || !y || ldy < out)
        return set_error(K3C_EINVAL, "mmw_tc: in=%d (a multiple of 8), W 16-byte aligned, ldy=%d >= out=%d", in, ldy,
                         out);
    static int *err_of[64] = {};
    int *&err = err_of[cur_dev()];
    if (!err) K3C_TRY_CUDA(cudaGetSymbolAddress((void **)&err, g_tg_err));
    const uint16_t *a = reinterpret_cast<const uint16_t *>(((uintptr_t)terms + 255) & ~(uintptr_t)255);
    const int Kp = kpad64(in);
    CUtensorMap ma, mw;
    K3C_TRY(make_map_terms(&ma, a, ntok, Kp));
    K3C_TRY(make_map3(&mw, CU_TENSOR_MAP_DATA_TYPE_UINT8, W, (uint64_t)in * 2, (uint64_t)out, 1, (uint64_t)in * 2,
                      (uint64_t)in * 2 * out, 128, TG_N));
    static bool attr_of[64] = {};
    bool &attr = attr_of[cur_dev()];
    if (!attr) {
        K3C_TRY_CUDA(cudaFuncSetAttribute(k_tg_gemm, cudaFuncAttributeMaxDynamicSharedMemorySize, TG_SMEM));
        attr = true;
    }
    TgArgs p;
    p.y = y;
    p.ldy = ldy;
    p.T = ntok;
    p.out = out;
    p.KB = Kp / TG_KB;
    p.accumulate = accumulate ? 1 : 0;
    p.vec = ((uintptr_t)y % 16 == 0) && (ldy % 4 == 0);
    p.err = err;
    const dim3 grid((ntok + TG_M - 1) / TG_M, (out + TG_N - 1) / TG_N);
    k_tg_gemm<<<grid, TG_THREADS, TG_SMEM, s>>>(ma, mw, p);
    K3C_CHECK_LAUNCH();
    count_launch();
    static const int sync_check = getenv("K3C_SYNC_CHECK") ? 1 : 0;
    if (sync_check) {
        int code = 0;
        K3C_TRY_CUDA(cudaStreamSynchronize(s));
        K3C_TRY_CUDA(cudaMemcpy(&code, err, sizeof(int), cudaMemcpyDeviceToHost));
        if (code) {
            const int zero = 0;
            cudaMemcpy(err, &zero, sizeof(int), cudaMemcpyHostToDevice);
            return set_error(K3C_ETIMEOUT, "mmw_tc: device check code %d", code);
        }
    }
    return K3C_OK;
}

}  // namespace k3c

extern "C" size_t k3c_mmw_tc_scratch(int ntok, int in) { return k3c::mmw_tc_terms_bytes(ntok, in); }

extern "C" int k3c_mmw_tc(float *y, int ldy, const float *x, int ldx, int ntok, const void *W, int in, int out,
                          int accumulate, void *scratch, size_t scratch_bytes, k3c_stream_t stream) {
    k3c::clear_error();
    if (ntok <= 0 || out <= 0) return K3C_OK;
    if (scratch_bytes < k3c::mmw_tc_terms_bytes(ntok, in))
        return k3c::set_error(K3C_EINVAL, "mmw_tc: scratch of %zu bytes, %zu needed", scratch_bytes,
                              k3c::mmw_tc_terms_bytes(ntok, in));
    if (!k3c::mmw_tc_applies(W, in))
        return k3c::set_error(K3C_EINVAL, "mmw_tc: in=%d must be a multiple of 8 and W 16-byte aligned", in);
    cudaStream_t s = (cudaStream_t)stream;
    K3C_TRY(k3c::launch_mmw_tc_split(scratch, x, ldx, ntok, in, s));
    return k3c::launch_mmw_tc_gemm(y, ldy, scratch, ntok, W, in, out, accumulate, s);
}
