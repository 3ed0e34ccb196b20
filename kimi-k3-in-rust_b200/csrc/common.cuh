// common.cuh -- shared helpers for libk3cuda.so: status plumbing and MXFP4 decode.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

#include "../../include/k3c.h"

namespace k3c {

// ------------------------------------------------------------------ status plumbing
// Records a message for k3c_last_error() and returns `code`.
int set_error(int code, const char *fmt, ...);
void clear_error();
// Counts kernel launches made by this library (read by k3c_launch_count()).
void count_launch();
// Stage timing: when enabled, stage_begin/stage_end record CUDA events around a named
// stage on the launching stream; k3c_timing_read() sums the elapsed times per stage.
enum Stage { STAGE_EXPERTS = 0, STAGE_ROUTER = 1, STAGE_COMBINE = 2, STAGE_Q8 = 3, STAGE_DISPATCH = 4, STAGE_N = 5 };
void stage_begin(int stage, cudaStream_t s);
void stage_end(int stage, cudaStream_t s);

#define K3C_TRY_CUDA(expr)                                                             \
    do {                                                                               \
        cudaError_t e_ = (expr);                                                       \
        if (e_ != cudaSuccess)                                                         \
            return ::k3c::set_error(K3C_ECUDA, "%s:%d %s: %s", __FILE__, __LINE__, #expr, \
                                    cudaGetErrorString(e_));                           \
    } while (0)

#define K3C_TRY(expr)                                                                  \
    do {                                                                               \
        int rc_ = (expr);                                                              \
        if (rc_ != K3C_OK) return rc_;                                                 \
    } while (0)

#define K3C_CHECK_LAUNCH()             \
    do {                               \
        ::k3c::count_launch();         \
        K3C_TRY_CUDA(cudaGetLastError()); \
    } while (0)

static inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// The current device (0..63) for per-device caches of symbol addresses and function
// attributes: a process may drive several GPUs, and a __device__ symbol's address and a
// kernel's shared-memory opt-in are per device.
inline int cur_dev() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = 0;
    return dev;
}

// Entry points that allocate their scratch per call (k3c_router, k3c_q8_gemv) use the
// device's default stream-ordered pool. Its default release threshold of 0 hands freed memory
// back to the driver at every synchronisation, so the next call maps it again (hundreds of
// ms for a few hundred MB); keeping it in the pool for the life of the process makes a
// repeated call an O(1) suballocation. This is a per-process attribute of the pool.
inline void keep_async_pool() {
    static bool done[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64 || done[dev]) return;
    cudaMemPool_t pool;
    if (cudaDeviceGetDefaultMemPool(&pool, dev) == cudaSuccess) {
        uint64_t keep = ~0ull;
        cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep);
    }
    done[dev] = true;
}

// Launch as a programmatic dependent of the previous work in the stream: the kernel may be
// scheduled before its predecessor ends, and must execute griddepcontrol.wait before it
// reads anything the predecessor writes.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                              Args... args) {
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// Bump allocator over caller-provided device scratch.
struct Carve {
    char *base;
    size_t cap, used;
    template <class T>
    T *take(size_t n, size_t align = 256) {
        size_t off = align_up(used, align);
        if (off + n * sizeof(T) > cap) return nullptr;
        used = off + n * sizeof(T);
        return reinterpret_cast<T *>(base + off);
    }
};

// ------------------------------------------------------------------ MXFP4 decode
// E8M0 byte -> 2^(b-127) as fp32 (b=0 gives the subnormal 2^-127); 255 -> 0.
__device__ __forceinline__ float e8m0_to_f32(uint32_t b) {
    if (b == 255u) return 0.0f;
    if (b == 0u) return __int_as_float(0x00400000);
    return __int_as_float((int)(b << 23));
}

// E2M1 code (0..15) -> fp32. Bit 3 is the sign; code 8 is -0.0.
__device__ __forceinline__ float e2m1_to_f32(uint32_t c) {
    // bf16 patterns of {0,.5,1,1.5,2,3,4,6}: hi bytes 00 3F 3F 3F 40 40 40 40,
    // lo bytes 00 00 80 C0 00 40 80 C0.
    uint32_t m = c & 7u;
    uint32_t hi = __byte_perm(0x3F3F3F00u, 0x40404040u, m);
    uint32_t lo = __byte_perm(0xC0800000u, 0xC0804000u, m);
    uint32_t bits = ((hi & 0xFFu) << 24) | ((lo & 0xFFu) << 16) | ((c & 8u) << 28);
    return __int_as_float((int)bits);
}

// Eight E2M1 codes packed in w (element k in bits 4k..4k+3, i.e. the low nibble of each
// byte is the even element) -> eight fp32 values, unscaled. Table lookups run through
// byte permutes: the bf16 high/low bytes of the eight magnitudes, indexed by the 3-bit
// magnitude, then interleaved into bf16 pairs and the sign bit merged.
__device__ __forceinline__ void e2m1x8_to_f32(uint32_t w, float (&f)[8]) {
    const uint32_t m = w & 0x77777777u;
    const uint32_t mh = m >> 16;
    const uint32_t lo_a = __byte_perm(0xC0800000u, 0xC0804000u, m);
    const uint32_t hi_a = __byte_perm(0x3F3F3F00u, 0x40404040u, m);
    const uint32_t lo_b = __byte_perm(0xC0800000u, 0xC0804000u, mh);
    const uint32_t hi_b = __byte_perm(0x3F3F3F00u, 0x40404040u, mh);
    const uint32_t w4 = w << 4;
    uint32_t p01 = __byte_perm(lo_a, hi_a, 0x5140u) ^ (__byte_perm(w4, w, 0x4000u) & 0x80008000u);
    uint32_t p23 = __byte_perm(lo_a, hi_a, 0x7362u) ^ (__byte_perm(w4, w, 0x5010u) & 0x80008000u);
    uint32_t p45 = __byte_perm(lo_b, hi_b, 0x5140u) ^ (__byte_perm(w4, w, 0x6020u) & 0x80008000u);
    uint32_t p67 = __byte_perm(lo_b, hi_b, 0x7362u) ^ (__byte_perm(w4, w, 0x7030u) & 0x80008000u);
    f[0] = __int_as_float((int)(p01 << 16)); f[1] = __int_as_float((int)(p01 & 0xFFFF0000u));
    f[2] = __int_as_float((int)(p23 << 16)); f[3] = __int_as_float((int)(p23 & 0xFFFF0000u));
    f[4] = __int_as_float((int)(p45 << 16)); f[5] = __int_as_float((int)(p45 & 0xFFFF0000u));
    f[6] = __int_as_float((int)(p67 << 16)); f[7] = __int_as_float((int)(p67 & 0xFFFF0000u));
}

__device__ __forceinline__ float bf16_bits_to_f32(uint16_t h) {
    return __int_as_float((int)((uint32_t)h << 16));
}

// Two floats rounded to bf16 (nearest even), lo in bits 0..15, hi in bits 16..31.
__device__ __forceinline__ uint32_t f32x2_to_bf16x2(float lo, float hi) {
    uint32_t d;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
    return d;
}

__device__ __forceinline__ uint4 ldg_nc_v4(const void *p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

}  // namespace k3c
