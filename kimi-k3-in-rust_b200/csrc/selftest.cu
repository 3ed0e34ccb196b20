// selftest.cu -- a check of the bounded device waits every pipelined kernel of this library
// relies on (tc_common.cuh: mbar_wait_ns for mbarrier phases, wait_count_ns for the
// release/acquire counters between the decode kernels). The production kernels wait at most
// ~2 s, record a code in their error word and return; this entry point runs the same helpers
// on a wait that nothing will ever satisfy, with a short limit, and reports the outcome the
// way the kernels' callers do (K3C_ETIMEOUT), leaving the CUDA context usable. No copy is in
// flight when the waits give up and no tensor memory is held.
#include <cuda_runtime.h>

#include "common.cuh"
#include "tc_common.cuh"

namespace k3c {

// kind 0: an mbarrier that nobody arrives at; kind 1: a counter that nobody increments;
// kind 2: a counter that is already at its target (the wait must succeed at once).
__global__ void k_selftest_wait(int kind, uint64_t limit_ns, int *err, const int *ctr) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x == 0) {
        tc::mbar_init(&bar, 1);
        tc::fence_mbar_init();
    }
    __syncthreads();
    if (threadIdx.x != 0) return;
    bool ok;
    if (kind == 0)
        ok = tc::mbar_wait_ns(&bar, 0, err, 77, limit_ns);
    else
        ok = tc::wait_count_ns(ctr, 1, err, 78, limit_ns);
    if (ok && kind != 2) atomicExch(err, 99);   // a wait that should not have ended did
}

}  // namespace k3c

extern "C" int k3c_selftest_wait(int kind, double limit_ms, k3c_stream_t stream) {
    k3c::clear_error();
    if (kind < 0 || kind > 2 || !(limit_ms > 0.0) || limit_ms > 2000.0)
        return k3c::set_error(K3C_EINVAL, "selftest_wait: kind=%d limit_ms=%g", kind, limit_ms);
    cudaStream_t s = (cudaStream_t)stream;
    int *buf = nullptr;   // [0] error word, [1] counter
    K3C_TRY_CUDA(cudaMallocAsync((void **)&buf, 2 * sizeof(int), s));
    const int init[2] = {0, kind == 2 ? 1 : 0};
    cudaError_t e = cudaMemcpyAsync(buf, init, sizeof init, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) {
        k3c::k_selftest_wait<<<1, 32, 0, s>>>(kind, (uint64_t)(limit_ms * 1e6), buf, buf + 1);
        k3c::count_launch();
        e = cudaGetLastError();
    }
    int code = 0;
    if (e == cudaSuccess) e = cudaMemcpyAsync(&code, buf, sizeof(int), cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    cudaFreeAsync(buf, s);
    if (e != cudaSuccess) return k3c::set_error(K3C_ECUDA, "selftest_wait: %s", cudaGetErrorString(e));
    if (code == 99) return k3c::set_error(K3C_EINVAL, "selftest_wait: an unsatisfiable wait returned success");
    if (code) return k3c::set_error(K3C_ETIMEOUT, "selftest_wait: bounded wait gave up (device code %d)", code);
    return K3C_OK;
}
