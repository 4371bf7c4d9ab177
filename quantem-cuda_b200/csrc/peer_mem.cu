// peer_mem.cu — device memory that the other processes of a multi-GPU job can
// map (CUDA IPC), for the D-slab halo exchange and the cross-rank loss
// reduction that store straight into a peer's memory over NVLink.
#include <string.h>

#include "qc_common.cuh"

static_assert(sizeof(cudaIpcMemHandle_t) == QC_IPC_HANDLE_BYTES, "IPC handle size");

extern "C" {

int quantem_cuda_peer_alloc(size_t bytes, void **d_ptr) {
    QC_RETURN_IF(d_ptr == nullptr, QC_ERR_INVALID_ARGUMENT, "quantem_cuda_peer_alloc: null d_ptr");
    QC_RETURN_IF(bytes == 0, QC_ERR_INVALID_ARGUMENT, "quantem_cuda_peer_alloc: zero bytes");
    *d_ptr = nullptr;
    void *p = nullptr;
    QC_CUDA_TRY(cudaMalloc(&p, bytes), "cudaMalloc(peer memory)");
    cudaError_t e = cudaMemset(p, 0, bytes);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        cudaFree(p);
        return qc::check_cuda(e, "cudaMemset(peer memory)");
    }
    *d_ptr = p;
    return 0;
}

int quantem_cuda_peer_free(void *d_ptr) {
    if (d_ptr == nullptr) return 0;
    QC_CUDA_TRY(cudaFree(d_ptr), "cudaFree(peer memory)");
    return 0;
}

int quantem_cuda_ipc_handle(void *d_ptr, void *handle_out) {
    QC_RETURN_IF(d_ptr == nullptr || handle_out == nullptr, QC_ERR_INVALID_ARGUMENT,
                 "quantem_cuda_ipc_handle: null pointer");
    cudaIpcMemHandle_t h;
    QC_CUDA_TRY(cudaIpcGetMemHandle(&h, d_ptr), "cudaIpcGetMemHandle");
    memcpy(handle_out, &h, sizeof(h));
    return 0;
}

int quantem_cuda_ipc_open(const void *handle, void **d_ptr) {
    QC_RETURN_IF(handle == nullptr || d_ptr == nullptr, QC_ERR_INVALID_ARGUMENT,
                 "quantem_cuda_ipc_open: null pointer");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    *d_ptr = nullptr;
    QC_CUDA_TRY(cudaIpcOpenMemHandle(d_ptr, h, cudaIpcMemLazyEnablePeerAccess),
                "cudaIpcOpenMemHandle");
    return 0;
}

int quantem_cuda_ipc_close(void *d_ptr) {
    if (d_ptr == nullptr) return 0;
    QC_CUDA_TRY(cudaIpcCloseMemHandle(d_ptr), "cudaIpcCloseMemHandle");
    return 0;
}

}  // extern "C"
