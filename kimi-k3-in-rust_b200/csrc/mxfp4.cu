// mxfp4.cu -- MXFP4 dequant and batched GEMV (CUDA-core path).
//
// Layout is the reference's: packed [rows][in/2] bytes (low nibble = even element),
// scales [rows][ceil(in/group)] E8M0 bytes (src/core/k3_ops.c:1363-1800, k3.h:523-566).
//
// The GEMV has two paths:
//   fast     group == 32, in % 32 == 0, 16-byte aligned rows: one 16-byte load is exactly
//            one scale group; each group's 32 unscaled products are summed in fp32 and the
//            sum is multiplied by the exact power-of-two scale. Groups whose scale byte is
//            >= 250 (where E2M1*2^(s-127) can overflow fp32) fold the scale into each
//            weight instead, so inf/NaN propagate exactly as in the reference's flat path
//            (src/core/k3_ops.c:1420-1427). A 255 scale skips its group (:1519).
//   generic  any group <= 64 and even `in`: weights formed as fp32 E2M1*scale, products and
//            sum in double -- the reference's arithmetic, for odd shapes and the drop-in.
#include <cuda_runtime.h>

#include "common.cuh"
#include "gemv_core.cuh"

namespace k3c {

// ------------------------------------------------------------------------ dequant
__global__ void k_mx_dequant(float *__restrict__ out, const uint8_t *__restrict__ packed,
                             const uint8_t *__restrict__ scales, int rows, int pcols,
                             int group, int ngrp) {
    const size_t total = (size_t)rows * pcols;
    for (size_t b = blockIdx.x * (size_t)blockDim.x + threadIdx.x; b < total;
         b += (size_t)gridDim.x * blockDim.x) {
        const int r = (int)(b / pcols), j = (int)(b % pcols);
        const uint32_t byte = packed[b];
        const int i0 = 2 * j, i1 = 2 * j + 1;
        const float s0 = e8m0_to_f32(scales[(size_t)r * ngrp + i0 / group]);
        const float s1 = e8m0_to_f32(scales[(size_t)r * ngrp + i1 / group]);
        float2 v;
        v.x = e2m1_to_f32(byte & 15u) * s0;   // low nibble = EVEN element
        v.y = e2m1_to_f32(byte >> 4) * s1;
        reinterpret_cast<float2 *>(out + (size_t)r * 2 * pcols)[j] = v;
    }
}

// y[t*ldy + r] for rows [row0, row0 + 2*warps) and tokens [t0, t0+NT): one warp, 2 rows.
template <int NT>
__global__ void __launch_bounds__(256) k_mx_gemv_fast(float *__restrict__ y, int ldy,
                                                      const float *__restrict__ x, int ldx,
                                                      int ntok, const uint8_t *__restrict__ packed,
                                                      const uint8_t *__restrict__ scales, int in,
                                                      int rows) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r0 = (blockIdx.x * 8 + warp) * 2;
    if (r0 >= rows) return;
    const int r1 = r0 + 1 < rows ? r0 + 1 : r0;
    const size_t pitch = (size_t)in / 2, spitch = (size_t)in / 32;
    const uint8_t *prow[2] = {packed + r0 * pitch, packed + r1 * pitch};
    const uint8_t *srow[2] = {scales + r0 * spitch, scales + r1 * spitch};
    for (int t0 = blockIdx.y * NT; t0 < ntok; t0 += gridDim.y * NT) {
        const int nt = ntok - t0 < NT ? ntok - t0 : NT;
        const float *xrow[NT];
#pragma unroll
        for (int t = 0; t < NT; t++) xrow[t] = x + (size_t)(t0 + (t < nt ? t : 0)) * ldx;
        float acc[2][NT];
        mx_dot_rows<2, NT>(prow, srow, xrow, nt, in / 32, acc);
#pragma unroll
        for (int r = 0; r < 2; r++)
#pragma unroll
            for (int t = 0; t < NT; t++) {
                const float v = warp_sum(acc[r][t]);
                if (lane == 0 && t < nt && (r == 0 || r1 != r0))
                    y[(size_t)(t0 + t) * ldy + (r == 0 ? r0 : r1)] = v;
            }
    }
}

// Generic path: one warp per (row, token); weights folded to fp32 E2M1*scale, products and
// sums in double, one rounding to float (the reference's arithmetic, any group <= 64).
__global__ void __launch_bounds__(256) k_mx_gemv_generic(float *__restrict__ y, int ldy,
                                                         const float *__restrict__ x, int ldx,
                                                         int ntok, const uint8_t *__restrict__ packed,
                                                         const uint8_t *__restrict__ scales, int in,
                                                         int rows, int group) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long long item = (long long)blockIdx.x * 8 + warp;
    if (item >= (long long)rows * ntok) return;
    const int r = (int)(item % rows), t = (int)(item / rows);
    const int pcols = in / 2, ngrp = (in + group - 1) / group;
    const uint8_t *pr = packed + (size_t)r * pcols;
    const uint8_t *sr = scales + (size_t)r * ngrp;
    const float *xt = x + (size_t)t * ldx;
    double acc = 0.0;
    for (int b = lane; b < pcols; b += 32) {
        const uint32_t byte = pr[b];
        const int i0 = 2 * b;
        const uint32_t s0 = sr[i0 / group], s1 = sr[(i0 + 1) / group];
        if (s0 != 255u) acc += (double)(e2m1_to_f32(byte & 15u) * e8m0_to_f32(s0)) * (double)xt[i0];
        if (s1 != 255u) acc += (double)(e2m1_to_f32(byte >> 4) * e8m0_to_f32(s1)) * (double)xt[i0 + 1];
    }
    acc = warp_sum_d(acc);
    if (lane == 0) y[(size_t)t * ldy + r] = (float)acc;
}

// The reference's AVX2 flat row path reproduced bit for bit (src/core/k3_ops.c:1418-1508; taken
// there when group is a multiple of 16): lane l of a 16-thread group accumulates the elements
// i = l (mod 16) of whole 16-element chunks as fma((double)w, (double)x[i], a_l) in element
// order, w = E2M1(nibble) * 2^(s-127) formed in fp32 (exact, or +-inf where it overflows);
// a chunk whose scale byte is 255 contributes no operation at all. The lanes are combined as
// q_l = (a_l + a_{l+8}) + (a_{l+4} + a_{l+12}) and then (q_0 + q_2) + (q_1 + q_3), the
// in % 16 tail is fused in element order with w = E2M1 * E8M0 (255 -> 0), and the sum is
// rounded to float once.
template <int NT>
__global__ void __launch_bounds__(256) k_mx_exact(float *__restrict__ y, int ldy, const float *__restrict__ x,
                                                  int ldx, int ntok, const uint8_t *__restrict__ packed,
                                                  const uint8_t *__restrict__ scales, int in, int rows, int group) {
    const int l = threadIdx.x & 15;
    const int row = blockIdx.x * 16 + (threadIdx.x >> 4);
    const int r = row < rows ? row : rows - 1;   // rows past the end compute row rows-1, unstored
    const int pcols = in / 2, ngrp = (in + group - 1) / group, in16 = in & ~15;
    const uint8_t *pr = packed + (size_t)r * pcols;
    const uint8_t *sr = scales + (size_t)r * ngrp;
    for (int t0 = blockIdx.y * NT; t0 < ntok; t0 += gridDim.y * NT) {
        double a[NT];
#pragma unroll
        for (int t = 0; t < NT; t++) a[t] = 0.0;
        for (int i = l; i < in16; i += 16) {
            const uint32_t sb = sr[i / group];
            if (sb == 255u) continue;
            const uint32_t byte = pr[i >> 1];
            const double w = (double)(e2m1_to_f32((i & 1) ? byte >> 4 : byte & 15u) * e8m0_to_f32(sb));
#pragma unroll
            for (int t = 0; t < NT; t++)
                if (t0 + t < ntok) a[t] = fma(w, (double)x[(size_t)(t0 + t) * ldx + i], a[t]);
        }
#pragma unroll
        for (int t = 0; t < NT; t++) {
            double v = a[t];
            v += __shfl_down_sync(0xffffffffu, v, 8, 16);
            v += __shfl_down_sync(0xffffffffu, v, 4, 16);
            v += __shfl_down_sync(0xffffffffu, v, 2, 16);
            v += __shfl_down_sync(0xffffffffu, v, 1, 16);
            if (l == 0 && row < rows && t0 + t < ntok) {
                const float *xt = x + (size_t)(t0 + t) * ldx;
                for (int i = in16; i < in; i++) {
                    const uint32_t byte = pr[i >> 1];
                    const float w = e2m1_to_f32((i & 1) ? byte >> 4 : byte & 15u) * e8m0_to_f32(sr[i / group]);
                    v = fma((double)w, (double)xt[i], v);
                }
                y[(size_t)(t0 + t) * ldy + row] = __double2float_rn(v);
            }
        }
    }
}

int mx_check(int in, int rows, int group) {
    if (in <= 0 || rows <= 0) return set_error(K3C_EINVAL, "mxfp4: in=%d rows=%d", in, rows);
    if (in & 1) return set_error(K3C_EINVAL, "mxfp4: odd in=%d", in);
    if (group <= 0 || group > 64) return set_error(K3C_EINVAL, "mxfp4: group=%d outside 1..64", group);
    return K3C_OK;
}

int launch_mx_gemv(float *y, int ldy, const float *x, int ldx, int ntok,
                   const uint8_t *packed, const uint8_t *scales, int in, int rows, int group,
                   cudaStream_t s) {
    K3C_TRY(mx_check(in, rows, group));
    if (ntok <= 0) return K3C_OK;
    const bool fast = group == 32 && (in % 32) == 0 && ((uintptr_t)packed & 15) == 0 &&
                      ((uintptr_t)x & 15) == 0 && (ldx % 4) == 0;
    if (fast) {
        dim3 grid((rows + 15) / 16, 1);
        if (ntok <= 1) {
            k_mx_gemv_fast<1><<<grid, 256, 0, s>>>(y, ldy, x, ldx, ntok, packed, scales, in, rows);
        } else if (ntok <= 2) {
            k_mx_gemv_fast<2><<<grid, 256, 0, s>>>(y, ldy, x, ldx, ntok, packed, scales, in, rows);
        } else {
            grid.y = (ntok + 3) / 4;
            if (grid.y > 16) grid.y = 16;
            k_mx_gemv_fast<4><<<grid, 256, 0, s>>>(y, ldy, x, ldx, ntok, packed, scales, in, rows);
        }
    } else {
        const long long items = (long long)rows * ntok;
        k_mx_gemv_generic<<<(unsigned)((items + 7) / 8), 256, 0, s>>>(y, ldy, x, ldx, ntok,
                                                                    packed, scales, in, rows, group);
    }
    K3C_CHECK_LAUNCH();
    return K3C_OK;
}

// k3_matmul_mxfp4's result bit for bit when group is a multiple of 16 (k_mx_exact); other
// groups take the generic kernel (double sums in another order, within a few ulps of double).
int launch_mx_exact(float *y, int ldy, const float *x, int ldx, int ntok, const uint8_t *packed,
                    const uint8_t *scales, int in, int rows, int group, cudaStream_t s) {
    K3C_TRY(mx_check(in, rows, group));
    if (ntok <= 0) return K3C_OK;
    if (group % 16) return launch_mx_gemv(y, ldy, x, ldx, ntok, packed, scales, in, rows, group, s);
    dim3 grid((rows + 15) / 16, 1);
    if (ntok == 1) {
        k_mx_exact<1><<<grid, 256, 0, s>>>(y, ldy, x, ldx, ntok, packed, scales, in, rows, group);
    } else {
        grid.y = (ntok + 3) / 4 < 16 ? (ntok + 3) / 4 : 16;
        k_mx_exact<4><<<grid, 256, 0, s>>>(y, ldy, x, ldx, ntok, packed, scales, in, rows, group);
    }
    K3C_CHECK_LAUNCH();
    return K3C_OK;
}

int launch_mx_dequant(float *out, const uint8_t *packed, const uint8_t *scales, int rows,
                      int pcols, int group, cudaStream_t s) {
    if (rows <= 0 || pcols <= 0) return set_error(K3C_EINVAL, "dequant: rows=%d pcols=%d", rows, pcols);
    if (group <= 0) return set_error(K3C_EINVAL, "dequant: group=%d", group);
    const int ngrp = (2 * pcols + group - 1) / group;
    const size_t total = (size_t)rows * pcols;
    unsigned blocks = (unsigned)((total + 255) / 256);
    if (blocks > 148u * 32u) blocks = 148u * 32u;
    k_mx_dequant<<<blocks, 256, 0, s>>>(out, packed, scales, rows, pcols, group, ngrp);
    K3C_CHECK_LAUNCH();
    return K3C_OK;
}

}  // namespace k3c

extern "C" int k3c_mxfp4_dequant(float *out, const uint8_t *packed, const uint8_t *scales,
                                 int rows, int pcols, int group, k3c_stream_t stream) {
    k3c::clear_error();
    return k3c::launch_mx_dequant(out, packed, scales, rows, pcols, group, (cudaStream_t)stream);
}

extern "C" int k3c_mxfp4_gemv(float *y, int ldy, const float *x, int ldx, int ntok,
                              const uint8_t *packed, const uint8_t *scales, int in, int rows,
                              int group, k3c_stream_t stream) {
    k3c::clear_error();
    return k3c::launch_mx_gemv(y, ldy, x, ldx, ntok, packed, scales, in, rows, group,
                               (cudaStream_t)stream);
}
