// moe_noalloc.cu -- k3c_moe_decode_noalloc: the MoE decode entry point that allocates
// nothing.
//
// k3c_moe_decode needs caller-provided device scratch. Some callers cannot provide it: an
// engine that owns every byte of device memory and hands this library no allocator, or a
// latency-bound decode loop whose host code must never call cudaMalloc (it can block and
// synchronise the device). This entry point runs the same kernels with its scratch taken
// from a fixed array in this file instead.
//
// The array is a file-scope __device__ variable of K3C_NOALLOC_SCRATCH_BYTES bytes: every
// GPU that loads this library holds it until the process exits. In host code its name is
// only a host-side stand-in, so the device address is looked up once per device with
// cudaGetSymbolAddress, with that device current, by the first call made on that device.
// Every call on a device shares the one array and leaves its contents behind; nothing in it
// is read before the same call writes it, but two calls whose kernels overlap on the GPU
// (for example on two streams) race on it.
#include <cuda_runtime.h>

#include <mutex>

#include "common.cuh"

namespace k3c {

int launch_moe_decode(float *out, const void *x, int x_dtype, int ntok, const k3c_moe_layer *L,
                      int *idx_out, float *wt_out, int *drops, void *scratch,
                      size_t scratch_bytes, cudaStream_t s);
size_t moe_decode_scratch(const k3c_moe_layer *L, int ntok);

static __device__ __align__(256) unsigned char g_noalloc_scratch[K3C_NOALLOC_SCRATCH_BYTES];

namespace {
struct DeviceScratch {
    std::once_flag once;
    void *ptr = nullptr;
    cudaError_t err = cudaSuccess;
};
constexpr int kMaxDevices = 64;
DeviceScratch g_scratch_addr[kMaxDevices];
}  // namespace

// Device address of g_noalloc_scratch on the current device (looked up on first use).
static int noalloc_scratch(void **out) {
    int dev = -1;
    K3C_TRY_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) return set_error(K3C_EINVAL, "noalloc: device %d out of range", dev);
    DeviceScratch &d = g_scratch_addr[dev];
    std::call_once(d.once, [&d] { d.err = cudaGetSymbolAddress(&d.ptr, g_noalloc_scratch); });
    if (d.err != cudaSuccess || d.ptr == nullptr)
        return set_error(K3C_ECUDA, "noalloc: cudaGetSymbolAddress on device %d: %s", dev,
                         cudaGetErrorString(d.err));
    *out = d.ptr;
    return K3C_OK;
}

}  // namespace k3c

extern "C" int k3c_moe_decode_noalloc(float *out, const void *x, int x_dtype, int ntok,
                                      const k3c_moe_layer *L, int *idx, float *wt, int *drops,
                                      k3c_stream_t stream) {
    k3c::clear_error();
    if (!L) return k3c::set_error(K3C_EINVAL, "moe_decode_noalloc: null layer");
    const size_t need = k3c::moe_decode_scratch(L, ntok);
    if (need > (size_t)K3C_NOALLOC_SCRATCH_BYTES)
        return k3c::set_error(K3C_EINVAL,
                              "moe_decode_noalloc: %d tokens need %zu bytes of scratch; the static "
                              "maximum is %zu bytes (K3C_NOALLOC_SCRATCH_BYTES): use fewer tokens "
                              "per call or k3c_moe_decode with caller scratch",
                              ntok, need, (size_t)K3C_NOALLOC_SCRATCH_BYTES);
    void *scratch = nullptr;
    K3C_TRY(k3c::noalloc_scratch(&scratch));
    return k3c::launch_moe_decode(out, x, x_dtype, ntok, L, idx, wt, drops, scratch,
                                  (size_t)K3C_NOALLOC_SCRATCH_BYTES, (cudaStream_t)stream);
}
