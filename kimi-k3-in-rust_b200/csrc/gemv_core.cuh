// gemv_core.cuh -- warp-cooperative MXFP4 dot products shared by the GEMV and MoE kernels.
#pragma once

#include "common.cuh"

namespace k3c {

// ---------------------------------------------------------------- fast GEMV core
// Warp-cooperative partial dot products of RW MXFP4 rows against NT fp32 activation rows.
// Lane l visits 16-byte chunks c = l, l+32, ... (chunk c = elements 32c..32c+31 = scale
// group c). acc[r][t] receives this lane's partial sum; the caller reduces over the warp.
// The chunks are fetched CPL per lane at a time, all requested before any is used, so a warp
// keeps RW*CPL*512 bytes of weights in flight; the per-lane summation order is c ascending.
// Eight E2M1 codes (element k in bits 4k..4k+3) -> fp32 through the hardware FP4 -> f16x2
// conversion (one instruction per byte; every E2M1 value is exact in f16 and in fp32).
__device__ __forceinline__ void e2m1x8_cvt(uint32_t w, float (&f)[8]) {
    asm("{\n\t"
        ".reg .b8 b0, b1, b2, b3;\n\t"
        ".reg .b32 h0, h1, h2, h3;\n\t"
        ".reg .f16 e0, e1, e2, e3, e4, e5, e6, e7;\n\t"
        "mov.b32 {b0, b1, b2, b3}, %8;\n\t"
        "cvt.rn.f16x2.e2m1x2 h0, b0;\n\t"
        "cvt.rn.f16x2.e2m1x2 h1, b1;\n\t"
        "cvt.rn.f16x2.e2m1x2 h2, b2;\n\t"
        "cvt.rn.f16x2.e2m1x2 h3, b3;\n\t"
        "mov.b32 {e0, e1}, h0;\n\t"
        "mov.b32 {e2, e3}, h1;\n\t"
        "mov.b32 {e4, e5}, h2;\n\t"
        "mov.b32 {e6, e7}, h3;\n\t"
        "cvt.f32.f16 %0, e0;\n\t"
        "cvt.f32.f16 %1, e1;\n\t"
        "cvt.f32.f16 %2, e2;\n\t"
        "cvt.f32.f16 %3, e3;\n\t"
        "cvt.f32.f16 %4, e4;\n\t"
        "cvt.f32.f16 %5, e5;\n\t"
        "cvt.f32.f16 %6, e6;\n\t"
        "cvt.f32.f16 %7, e7;\n\t"
        "}"
        : "=f"(f[0]), "=f"(f[1]), "=f"(f[2]), "=f"(f[3]), "=f"(f[4]), "=f"(f[5]), "=f"(f[6]), "=f"(f[7])
        : "r"(w));
}

// P += (f[2m] x[2m], f[2m+1] x[2m+1]) for m < 4: four packed fp32 FMAs (even and odd
// elements in the two lanes of P).
__device__ __forceinline__ void dot8_f32x2(const float (&f)[8], const float (&x)[8], float &p0, float &p1) {
    asm("{\n\t"
        ".reg .b64 A, F0, F1, F2, F3, X0, X1, X2, X3;\n\t"
        "mov.b64 A, {%0, %1};\n\t"
        "mov.b64 F0, {%2, %3};\n\t"
        "mov.b64 F1, {%4, %5};\n\t"
        "mov.b64 F2, {%6, %7};\n\t"
        "mov.b64 F3, {%8, %9};\n\t"
        "mov.b64 X0, {%10, %11};\n\t"
        "mov.b64 X1, {%12, %13};\n\t"
        "mov.b64 X2, {%14, %15};\n\t"
        "mov.b64 X3, {%16, %17};\n\t"
        "fma.rn.f32x2 A, F0, X0, A;\n\t"
        "fma.rn.f32x2 A, F1, X1, A;\n\t"
        "fma.rn.f32x2 A, F2, X2, A;\n\t"
        "fma.rn.f32x2 A, F3, X3, A;\n\t"
        "mov.b64 {%0, %1}, A;\n\t"
        "}"
        : "+f"(p0), "+f"(p1)
        : "f"(f[0]), "f"(f[1]), "f"(f[2]), "f"(f[3]), "f"(f[4]), "f"(f[5]), "f"(f[6]), "f"(f[7]),
          "f"(x[0]), "f"(x[1]), "f"(x[2]), "f"(x[3]), "f"(x[4]), "f"(x[5]), "f"(x[6]), "f"(x[7]));
}

template <int RW, int CPL>
struct MxChunks {
    uint4 wv[CPL][RW];
    uint32_t sb[CPL][RW];

    // chunks c0 + lane + 32 i, i < CPL
    __device__ __forceinline__ void load(const uint8_t *const (&prow)[RW], const uint8_t *const (&srow)[RW],
                                         int c0, int nchunk) {
        const int lane = threadIdx.x & 31;
#pragma unroll
        for (int i = 0; i < CPL; i++) {
            const int c = c0 + lane + 32 * i;
#pragma unroll
            for (int r = 0; r < RW; r++) {
                if (c < nchunk) {
                    wv[i][r] = ldg_nc_v4(prow[r] + (size_t)c * 16);
                    sb[i][r] = srow[r][c];
                } else {
                    wv[i][r] = make_uint4(0, 0, 0, 0);
                    sb[i][r] = 255u;
                }
            }
        }
    }

    // fma with the activation rows in shared memory (row t at sx + t * ld, x_swz order).
    // Per chunk and row: the 32 products accumulate pairwise (even/odd elements) in packed
    // fp32 FMAs, then one multiply-add by the chunk's scale; a scale of 250 or more is folded
    // into the weights first (as mac does), scale byte 255 contributes nothing.
    template <int NT>
    __device__ __forceinline__ void fma_smem(const float *sx, int ld, int ntok, int c0, int nchunk,
                                             float (&acc)[RW][NT]) const {
        const int lane = threadIdx.x & 31;
#pragma unroll
        for (int i = 0; i < CPL; i++) {
            const int c = c0 + lane + 32 * i;
            if (c >= nchunk) break;
            float pe[RW][NT], po[RW][NT];
#pragma unroll
            for (int r = 0; r < RW; r++)
#pragma unroll
                for (int t = 0; t < NT; t++) pe[r][t] = po[r][t] = 0.f;
#pragma unroll
            for (int q = 0; q < 4; q++) {
                float xv[NT][8];
#pragma unroll
                for (int t = 0; t < NT; t++) {
                    if (t < ntok) {
                        const float *xr = sx + t * ld + (c << 5);
                        const float4 a = *reinterpret_cast<const float4 *>(xr + (((2 * q) ^ (c & 7)) << 2));
                        const float4 b = *reinterpret_cast<const float4 *>(xr + (((2 * q + 1) ^ (c & 7)) << 2));
                        xv[t][0] = a.x; xv[t][1] = a.y; xv[t][2] = a.z; xv[t][3] = a.w;
                        xv[t][4] = b.x; xv[t][5] = b.y; xv[t][6] = b.z; xv[t][7] = b.w;
                    } else {
#pragma unroll
                        for (int k = 0; k < 8; k++) xv[t][k] = 0.f;
                    }
                }
#pragma unroll
                for (int r = 0; r < RW; r++) {
                    const uint32_t w = q == 0 ? wv[i][r].x : q == 1 ? wv[i][r].y : q == 2 ? wv[i][r].z : wv[i][r].w;
                    float f[8];
                    e2m1x8_cvt(w, f);
                    if (sb[i][r] >= 250u) {
                        const float sc = e8m0_to_f32(sb[i][r]);
#pragma unroll
                        for (int k = 0; k < 8; k++) f[k] *= sc;
                    }
#pragma unroll
                    for (int t = 0; t < NT; t++) dot8_f32x2(f, xv[t], pe[r][t], po[r][t]);
                }
            }
#pragma unroll
            for (int r = 0; r < RW; r++) {
                if (sb[i][r] == 255u) continue;
                const float sc = e8m0_to_f32(sb[i][r]);
                const bool fold = sb[i][r] >= 250u;
#pragma unroll
                for (int t = 0; t < NT; t++) {
                    const float p = pe[r][t] + po[r][t];
                    acc[r][t] = fold ? acc[r][t] + p : fmaf(p, sc, acc[r][t]);
                }
            }
        }
    }

    // the weight side of one 8-element group: decode, scale, multiply-add into acc
    template <int NT>
    __device__ __forceinline__ void mac(int i, int q, const float (&xv)[NT][8], float (&acc)[RW][NT]) const {
#pragma unroll
        for (int r = 0; r < RW; r++) {
            if (sb[i][r] == 255u) continue;
            const uint32_t w = q == 0 ? wv[i][r].x : q == 1 ? wv[i][r].y : q == 2 ? wv[i][r].z : wv[i][r].w;
            float f[8];
            e2m1x8_to_f32(w, f);
            const float sc = e8m0_to_f32(sb[i][r]);
            const bool fold = sb[i][r] >= 250u;
            if (fold) {
#pragma unroll
                for (int k = 0; k < 8; k++) f[k] *= sc;
            }
#pragma unroll
            for (int t = 0; t < NT; t++) {
                float p = 0.f;
#pragma unroll
                for (int k = 0; k < 8; k++) p = fmaf(f[k], xv[t][k], p);
                acc[r][t] = fold ? acc[r][t] + p : fmaf(p, sc, acc[r][t]);
            }
        }
    }

    template <int NT>
    __device__ __forceinline__ void fma(const float *const (&xrow)[NT], int ntok, int c0, int nchunk,
                                        float (&acc)[RW][NT]) const {
        const int lane = threadIdx.x & 31;
#pragma unroll
        for (int i = 0; i < CPL; i++) {
            const int c = c0 + lane + 32 * i;
            if (c >= nchunk) break;
#pragma unroll
            for (int q = 0; q < 4; q++) {  // 8 elements per 32-bit word
                float xv[NT][8];
#pragma unroll
                for (int t = 0; t < NT; t++) {
                    if (t < ntok) {
                        const float4 *xp = reinterpret_cast<const float4 *>(xrow[t] + 32 * c + 8 * q);
                        float4 a = __ldg(xp), b = __ldg(xp + 1);
                        xv[t][0] = a.x; xv[t][1] = a.y; xv[t][2] = a.z; xv[t][3] = a.w;
                        xv[t][4] = b.x; xv[t][5] = b.y; xv[t][6] = b.z; xv[t][7] = b.w;
                    } else {
#pragma unroll
                        for (int k = 0; k < 8; k++) xv[t][k] = 0.f;
                    }
                }
                mac(i, q, xv, acc);
            }
        }
    }
};

// Activations staged in shared memory for MxChunks::fma_smem: element e = 32c + 4u + w of a
// row is stored at 32c + 4(u ^ (c & 7)) + w, so the eight lanes reading chunks c..c+7 touch
// eight different 16-byte units and a warp's float4 reads cost the minimum four wavefronts
// (unswizzled, the 128-byte chunk stride puts every lane on the same four banks).
__device__ __forceinline__ int x_swz(int e) {
    const int c = e >> 5;
    return (c << 5) | ((((e >> 2) & 7) ^ (c & 7)) << 2) | (e & 3);
}
// Copies n floats (n a multiple of 4, src 16-byte aligned) into dst in the swizzled order;
// every thread of the block takes part.
__device__ __forceinline__ void stage_x_swz(float *dst, const float *__restrict__ src, int n) {
    for (int v = threadIdx.x; v < n / 4; v += blockDim.x)
        *reinterpret_cast<float4 *>(dst + x_swz(4 * v)) = __ldg(reinterpret_cast<const float4 *>(src) + v);
}

template <int RW, int NT, int CPL = 4>
__device__ __forceinline__ void mx_dot_rows(const uint8_t *const (&prow)[RW],
                                            const uint8_t *const (&srow)[RW],
                                            const float *const (&xrow)[NT], int ntok,
                                            int nchunk, float (&acc)[RW][NT]) {
#pragma unroll
    for (int r = 0; r < RW; r++)
#pragma unroll
        for (int t = 0; t < NT; t++) acc[r][t] = 0.f;
    MxChunks<RW, CPL> ch;
    for (int c0 = 0; c0 < nchunk; c0 += 32 * CPL) {
        ch.load(prow, srow, c0, nchunk);
        ch.template fma<NT>(xrow, ntok, c0, nchunk, acc);
    }
}

}  // namespace k3c
