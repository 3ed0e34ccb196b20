// tc_host.cuh -- host-side helpers of the tcgen05 kernels: TMA tensor-map encoding through
// the driver entry point (no libcuda link dependency) and the SM count.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include "common.cuh"

namespace k3c {

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                  const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                  const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

// 3-D tiled map (d0 innermost, strides in bytes), box b0 x b1 x 1, 128-byte swizzle.
inline int make_map3(CUtensorMap *m, CUtensorMapDataType dt, const void *base, uint64_t d0, uint64_t d1,
                     uint64_t d2, uint64_t s1, uint64_t s2, uint32_t b0, uint32_t b1) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return set_error(K3C_ECUDA, "tc: cuTensorMapEncodeTiled unavailable");
    cuuint64_t dims[3] = {d0, d1, d2}, strides[2] = {s1, s2};
    cuuint32_t box[3] = {b0, b1, 1}, es[3] = {1, 1, 1};
    CUresult r = fn(m, dt, 3, const_cast<void *>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(K3C_ECUDA, "tc: tensor map encode failed (%d)", (int)r);
    return K3C_OK;
}

// 2-D tiled map (d0 innermost, row stride s1 bytes), box b0 x b1, 128-byte swizzle.
inline int make_map2(CUtensorMap *m, CUtensorMapDataType dt, const void *base, uint64_t d0, uint64_t d1,
                     uint64_t s1, uint32_t b0, uint32_t b1) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return set_error(K3C_ECUDA, "tc: cuTensorMapEncodeTiled unavailable");
    cuuint64_t dims[2] = {d0, d1}, strides[1] = {s1};
    cuuint32_t box[2] = {b0, b1}, es[2] = {1, 1};
    CUresult r = fn(m, dt, 2, const_cast<void *>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(K3C_ECUDA, "tc: tensor map encode failed (%d)", (int)r);
    return K3C_OK;
}

inline int sm_count() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
    }
    return n;
}

}  // namespace k3c
