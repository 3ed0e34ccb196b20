// q8.cu -- INT8 per-row-scaled trunk projection (reference k3_matmul_q8,
// src/core/k3_ops.c:1204-1272; layout include/k3/k3.h:265-303).
//
// The reference keeps each row inline as [f32 scale][int8 * in] with stride 4+in bytes,
// which is not 16-byte aligned at in = 7168. k3c_q8_pack rewrites it once into a pool
// layout: int8 rows of ldw bytes (ldw a multiple of 16) plus a separate fp32 scale array,
// so the GEMV streams 16-byte vectors. y = scale * sum(int8 * x) with an fp32 accumulator,
// like the reference (which states no determinism contract for this kernel).
#include <cuda_runtime.h>

#include "common.cuh"

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

// Four int8 in a word -> four exact floats: place each byte (offset to unsigned) under the
// exponent of 2^23 and subtract 2^23 + 128.
__device__ __forceinline__ void s8x4_to_f32(uint32_t w, float (&f)[4]) {
    const uint32_t u = w ^ 0x80808080u;
    f[0] = __int_as_float((int)__byte_perm(u, 0x4B000000u, 0x7540u)) - 8388736.0f;
    f[1] = __int_as_float((int)__byte_perm(u, 0x4B000000u, 0x7541u)) - 8388736.0f;
    f[2] = __int_as_float((int)__byte_perm(u, 0x4B000000u, 0x7542u)) - 8388736.0f;
    f[3] = __int_as_float((int)__byte_perm(u, 0x4B000000u, 0x7543u)) - 8388736.0f;
}

template <typename XT>
__device__ __forceinline__ float xload(const XT *x, size_t i);
template <>
__device__ __forceinline__ float xload<float>(const float *x, size_t i) { return x[i]; }
template <>
__device__ __forceinline__ float xload<uint16_t>(const uint16_t *x, size_t i) {
    return bf16_bits_to_f32(x[i]);
}

// Block = 4 warps = 32 output rows; lane l of every warp owns row 32*bx + l, warp w owns the
// K-quarter [w*KQ, (w+1)*KQ). Each warp stages its own activations for 16 tokens in chunks
// of 256 K (fp32, exact widening) so every activation is one shared-memory broadcast feeding
// 32 FMAs (one per row); a lane streams its row 32 int8 weights (two full 16-byte vectors of
// one 32-byte sector) per step. The four quarter sums are added in a fixed order.
template <typename XT>
__global__ void __launch_bounds__(128, 3) k_q8_gemv(float *__restrict__ y, int ldy,
                                                 const XT *__restrict__ x, int ldx, int ntok,
                                                 const int8_t *__restrict__ wq,
                                                 const float *__restrict__ wscale, int ldw,
                                                 int in, int out) {
    constexpr int TCH = 16, KC = 256;
    extern __shared__ __align__(16) float q8_smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float *xs = q8_smem + (size_t)warp * TCH * KC;    // this warp's [16][256] chunk
    float *red = q8_smem + (size_t)4 * TCH * KC;       // [4][32][16] quarter sums
    const int row = blockIdx.x * 32 + lane;
    const int rowc = row < out ? row : out - 1;
    const int8_t *wrow = wq + (size_t)rowc * ldw;
    const int kq = ((ldw / 32 + 3) / 4) * 32;          // K-quarter, a multiple of 32
    const int kbeg = warp * kq, kend = min(ldw, kbeg + kq);
    for (int t0 = 0; t0 < ntok; t0 += TCH) {
        const int nt = ntok - t0 < TCH ? ntok - t0 : TCH;
        float acc[TCH];
#pragma unroll
        for (int t = 0; t < TCH; t++) acc[t] = 0.f;
        for (int k0 = kbeg; k0 < kend; k0 += KC) {
            __syncwarp();
            for (int i = lane; i < TCH * KC; i += 32) {  // coalesced: consecutive k per lane
                const int t = i / KC, k = k0 + i % KC;
                xs[i] = (t < nt && k < in && k < kend) ? xload<XT>(x, (size_t)(t0 + t) * ldx + k) : 0.0f;
            }
            __syncwarp();
            const int kk_end = min(KC, kend - k0);
            for (int kk = 0; kk < kk_end; kk += 32) {
                const uint4 v0 = ldg_nc_v4(wrow + k0 + kk);
                const uint4 v1 = ldg_nc_v4(wrow + k0 + kk + 16);
                float f[32];
                s8x4_to_f32(v0.x, *reinterpret_cast<float(*)[4]>(f + 0));
                s8x4_to_f32(v0.y, *reinterpret_cast<float(*)[4]>(f + 4));
                s8x4_to_f32(v0.z, *reinterpret_cast<float(*)[4]>(f + 8));
                s8x4_to_f32(v0.w, *reinterpret_cast<float(*)[4]>(f + 12));
                s8x4_to_f32(v1.x, *reinterpret_cast<float(*)[4]>(f + 16));
                s8x4_to_f32(v1.y, *reinterpret_cast<float(*)[4]>(f + 20));
                s8x4_to_f32(v1.z, *reinterpret_cast<float(*)[4]>(f + 24));
                s8x4_to_f32(v1.w, *reinterpret_cast<float(*)[4]>(f + 28));
#pragma unroll
                for (int t = 0; t < TCH; t++) {
                    const float4 *xp = reinterpret_cast<const float4 *>(xs + t * KC + kk);
#pragma unroll
                    for (int q = 0; q < 8; q++) {
                        const float4 xv = xp[q];  // same address in every lane: a broadcast
                        acc[t] = fmaf(f[4 * q + 0], xv.x, acc[t]);
                        acc[t] = fmaf(f[4 * q + 1], xv.y, acc[t]);
                        acc[t] = fmaf(f[4 * q + 2], xv.z, acc[t]);
                        acc[t] = fmaf(f[4 * q + 3], xv.w, acc[t]);
                    }
                }
            }
        }
#pragma unroll
        for (int t = 0; t < TCH; t++) red[(warp * 32 + lane) * TCH + t] = acc[t];
        __syncthreads();
        if (warp == 0 && row < out) {
            for (int t = 0; t < nt; t++) {
                float a = red[(0 * 32 + lane) * TCH + t];
                a += red[(1 * 32 + lane) * TCH + t];
                a += red[(2 * 32 + lane) * TCH + t];
                a += red[(3 * 32 + lane) * TCH + t];
                y[(size_t)(t0 + t) * ldy + row] = a * wscale[row];
            }
        }
        __syncthreads();
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

int launch_q8_gemv(float *y, int ldy, const void *x, int x_dtype, int ldx, int ntok,
                   const int8_t *wq, const float *wscale, int ldw, int in, int out,
                   cudaStream_t s) {
    if (in <= 0 || out <= 0 || ldw < in || (ldw % 32) || ((uintptr_t)wq & 15))
        return set_error(K3C_EINVAL, "q8_gemv: in=%d out=%d ldw=%d (ldw must be a multiple of 32)", in, out, ldw);
    if (ntok <= 0) return K3C_OK;
    const size_t smem = (size_t)(4 * 16 * 256 + 4 * 32 * 16) * sizeof(float);  // 72 KB
    const unsigned blocks = (unsigned)((out + 31) / 32);
    if (x_dtype == K3C_BF16) {
        K3C_TRY_CUDA(cudaFuncSetAttribute(k_q8_gemv<uint16_t>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        k_q8_gemv<uint16_t><<<blocks, 128, smem, s>>>(y, ldy, (const uint16_t *)x, ldx, ntok, wq, wscale, ldw, in, out);
    } else if (x_dtype == K3C_F32) {
        K3C_TRY_CUDA(cudaFuncSetAttribute(k_q8_gemv<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        k_q8_gemv<float><<<blocks, 128, smem, s>>>(y, ldy, (const float *)x, ldx, ntok, wq, wscale, ldw, in, out);
    } else {
        return set_error(K3C_EINVAL, "q8_gemv: x_dtype=%d", x_dtype);
    }
    K3C_CHECK_LAUNCH();
    return K3C_OK;
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
