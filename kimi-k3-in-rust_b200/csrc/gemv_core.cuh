// gemv_core.cuh -- warp-cooperative MXFP4 dot products shared by the GEMV and MoE kernels.
#pragma once

#include "common.cuh"

namespace k3c {

// ---------------------------------------------------------------- fast GEMV core
// Warp-cooperative partial dot products of RW MXFP4 rows against NT fp32 activation rows.
// Lane l visits 16-byte chunks c = l, l+32, ... (chunk c = elements 32c..32c+31 = scale
// group c). acc[r][t] receives this lane's partial sum; the caller reduces over the warp.
template <int RW, int NT>
__device__ __forceinline__ void mx_dot_rows(const uint8_t *const (&prow)[RW],
                                            const uint8_t *const (&srow)[RW],
                                            const float *const (&xrow)[NT], int ntok,
                                            int nchunk, float (&acc)[RW][NT]) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int r = 0; r < RW; r++)
#pragma unroll
        for (int t = 0; t < NT; t++) acc[r][t] = 0.f;
    for (int c = lane; c < nchunk; c += 32) {
        uint4 wv[RW];
        uint32_t sb[RW];
#pragma unroll
        for (int r = 0; r < RW; r++) {
            wv[r] = ldg_nc_v4(prow[r] + (size_t)c * 16);
            sb[r] = srow[r][c];
        }
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
#pragma unroll
            for (int r = 0; r < RW; r++) {
                if (sb[r] == 255u) continue;
                const uint32_t w = q == 0 ? wv[r].x : q == 1 ? wv[r].y : q == 2 ? wv[r].z : wv[r].w;
                float f[8];
                e2m1x8_to_f32(w, f);
                const float sc = e8m0_to_f32(sb[r]);
                const bool fold = sb[r] >= 250u;
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
    }
}

}  // namespace k3c
