// ep.cu -- device buffers shared between the processes of one node for the expert-parallel
// prefill (k3c_moe_prefill_ep_experts): plain cudaMalloc allocations exported and mapped with
// CUDA IPC handles, so peer kernels read and write them with ordinary loads and stores over
// NVLink.
#include <cuda_runtime.h>
#include <string.h>

#include "common.cuh"

static_assert(sizeof(cudaIpcMemHandle_t) <= sizeof(k3c_ipc_handle), "IPC handle fits the ABI type");

extern "C" int k3c_ep_alloc(void **ptr, size_t bytes, k3c_ipc_handle *handle) {
    k3c::clear_error();
    if (!ptr || !handle || bytes == 0) return k3c::set_error(K3C_EINVAL, "ep_alloc: bad arguments");
    *ptr = nullptr;
    K3C_TRY_CUDA(cudaMalloc(ptr, bytes));
    cudaIpcMemHandle_t h;
    const cudaError_t e = cudaIpcGetMemHandle(&h, *ptr);
    if (e != cudaSuccess) {
        cudaFree(*ptr);
        *ptr = nullptr;
        return k3c::set_error(K3C_ECUDA, "ep_alloc: %s", cudaGetErrorString(e));
    }
    memset(handle, 0, sizeof(*handle));
    memcpy(handle->bytes, &h, sizeof(h));
    return K3C_OK;
}

extern "C" int k3c_ep_free(void *ptr) {
    k3c::clear_error();
    if (ptr) K3C_TRY_CUDA(cudaFree(ptr));
    return K3C_OK;
}

extern "C" int k3c_ep_open(void **ptr, const k3c_ipc_handle *handle) {
    k3c::clear_error();
    if (!ptr || !handle) return k3c::set_error(K3C_EINVAL, "ep_open: bad arguments");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle->bytes, sizeof(h));
    K3C_TRY_CUDA(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
    return K3C_OK;
}

extern "C" int k3c_ep_close(void *peer_ptr) {
    k3c::clear_error();
    if (peer_ptr) K3C_TRY_CUDA(cudaIpcCloseMemHandle(peer_ptr));
    return K3C_OK;
}
