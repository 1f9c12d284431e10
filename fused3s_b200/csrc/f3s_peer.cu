// f3s_peer.cu -- buffers that other processes on the box can map (CUDA IPC),
// and stream-ordered copies into them.  Used to exchange rows of O between
// the ranks of a sharded forward over NVLink with the copy engines, which
// need no SMs and so run beside the fused kernel (a collective kernel would
// wait for the SMs the persistent kernel holds).
#include <cstring>
#include "f3s_internal.cuh"

static_assert(sizeof(cudaIpcMemHandle_t) == F3S_IPC_HANDLE_BYTES, "IPC handle size");

extern "C" {

int f3s_peer_alloc(size_t bytes, void** d_ptr, void* ipc_handle) {
    if (!d_ptr || !ipc_handle || bytes == 0) return F3S_ERR_INVALID_VALUE;
    *d_ptr = nullptr;
    void* p = nullptr;
    F3S_CUDA_TRY(cudaMalloc(&p, bytes));  // a base address: exportable as is
    cudaIpcMemHandle_t h;
    const cudaError_t e = cudaIpcGetMemHandle(&h, p);
    if (e != cudaSuccess) {
        f3s::note_cuda_error(e);
        cudaFree(p);
        return F3S_ERR_CUDA;
    }
    memcpy(ipc_handle, &h, sizeof(h));
    *d_ptr = p;
    return F3S_SUCCESS;
}

int f3s_peer_open(const void* ipc_handle, void** d_ptr) {
    if (!ipc_handle || !d_ptr) return F3S_ERR_INVALID_VALUE;
    *d_ptr = nullptr;
    cudaIpcMemHandle_t h;
    memcpy(&h, ipc_handle, sizeof(h));
    F3S_CUDA_TRY(cudaIpcOpenMemHandle(d_ptr, h, cudaIpcMemLazyEnablePeerAccess));
    return F3S_SUCCESS;
}

int f3s_peer_close(void* d_ptr) {
    if (!d_ptr) return F3S_ERR_INVALID_VALUE;
    F3S_CUDA_TRY(cudaIpcCloseMemHandle(d_ptr));
    return F3S_SUCCESS;
}

int f3s_peer_free(void* d_ptr) {
    if (!d_ptr) return F3S_ERR_INVALID_VALUE;
    F3S_CUDA_TRY(cudaFree(d_ptr));
    return F3S_SUCCESS;
}

int f3s_peer_copy(void* d_dst, const void* d_src, size_t bytes, f3s_stream_t stream) {
    if (bytes == 0) return F3S_SUCCESS;
    if (!d_dst || !d_src) return F3S_ERR_INVALID_VALUE;
    F3S_CUDA_TRY(cudaMemcpyAsync(d_dst, d_src, bytes, cudaMemcpyDefault, (cudaStream_t)stream));
    return F3S_SUCCESS;
}

}  // extern "C"
