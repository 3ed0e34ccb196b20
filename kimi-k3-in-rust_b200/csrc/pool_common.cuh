// pool_common.cuh -- pool-format geometry and the activation-term quantiser shared by the
// tcgen05 MoE kernels (decode: moe_pool.cu, prefill: moe_prefill.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "tc_common.cuh"

namespace k3c {

struct PoolGeom {
    size_t gu_p, gu_s, d_p, d_s, run;
};
__host__ __device__ inline PoolGeom pool_geom(int H, int I) {
    PoolGeom g;
    g.gu_p = 0;
    g.gu_s = (size_t)I * H;                                // 2I rows x H/2 bytes
    g.d_p = g.gu_s + (size_t)(2 * I / 128) * (H / 128) * 512;
    g.d_s = g.d_p + (size_t)H * I / 2;
    g.run = g.d_s + (size_t)(H / 128) * (I / 128) * 512;
    return g;
}

// GU row R -> (source matrix: 0 gate / 1 up, source row).
__host__ __device__ inline void gu_source(int R, int &which, int &row) {
    const int b = R / 128, m = R % 128;
    which = m >= 64;
    row = 64 * b + (m & 63);
}

__device__ __forceinline__ size_t atom_byte(int m, int g) {  // m: row in tile, g: group 0..3
    return (size_t)(16 * (m & 31) + 4 * (m >> 5) + g);
}

// ------------------------------------------------------------------ activation terms
// Block exponent e for a block maximum amax so that amax / 2^e <= 448 (the E4M3 maximum):
// e = ceil(log2(amax / 448)), clamped to the UE8M0 range used here [-127, 120].
__device__ __forceinline__ int block_exp(float amax) {
    const uint32_t u = __float_as_uint(amax);
    const int E = (int)((u >> 23) & 0xFF) - 127;
    if (amax == 0.0f || E < -119) return -127;
    int e = ((u & 0x7FFFFF) > 0x600000) ? E - 7 : E - 8;  // mantissa > 1.75 -> one more
    return e < -127 ? -127 : (e > 120 ? 120 : e);
}
__device__ __forceinline__ float exp2i(int e) {  // 2^e, e in [-126, 127]
    return __uint_as_float((uint32_t)(e + 127) << 23);
}

// One warp quantises one 32-element block held one element per lane into J terms.
// Writes each term's byte through qdst(j) and its scale byte through sfdst(j) (lane 0).
template <int J, class QF, class SF>
__device__ __forceinline__ void quantize_block(float a, QF qdst, SF sfdst) {
#pragma unroll
    for (int j = 0; j < J; j++) {
        float amax = fabsf(a);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        const int e = block_exp(amax);                 // e in [-127, 120]
        const uint32_t q = tc::f32_to_e4m3(a * exp2i(-e)); // 2^-e in [2^-120, 2^127]: exact
        qdst(j, q);
        if ((threadIdx.x & 31) == 0) sfdst(j, (uint32_t)(e + 127));
        const float back = tc::e4m3_to_f32(q);
        // back * 2^e exactly; 2^-127 is formed as 2^-126 / 2
        a = a - (e >= -126 ? back * exp2i(e) : (back * exp2i(-126)) * 0.5f);
    }
}

__device__ __forceinline__ float sigmoid_f(float v) { return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-v))); }
__device__ __forceinline__ float act_apply(float g, float u, int act) {
    if (act == K3C_ACT_SITU) {
        const float a = __fmul_rn(__fmul_rn(4.0f, tanhf(__fdiv_rn(g, 4.0f))), sigmoid_f(g));
        return __fmul_rn(a, __fmul_rn(25.0f, tanhf(__fdiv_rn(u, 25.0f))));
    }
    return __fmul_rn(__fmul_rn(g, sigmoid_f(g)), u);
}

}  // namespace k3c
