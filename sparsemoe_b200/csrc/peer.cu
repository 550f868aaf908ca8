// Peer device memory for expert parallelism over NVLink: buffers that other
// processes on the node map through CUDA IPC, so that the dispatch copies
// rows straight into the owner's receive buffer (copy engines, no SMs) and
// the owner's down-GEMM epilogue stores each result row straight into its
// sender's buffer (the transfer overlaps the GEMM tile by tile).
#include "moe_internal.h"

#include <cstring>

extern "C" int moe_peer_alloc(size_t bytes, void** ptr, void* handle64) {
    if (!ptr || !handle64 || bytes == 0) return MOE_ERR_INVALID_ARG;
    void* p = nullptr;
    if (cudaMalloc(&p, bytes) != cudaSuccess) return MOE_ERR_CUDA;
    cudaIpcMemHandle_t h;
    if (cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
        cudaFree(p);
        return MOE_ERR_CUDA;
    }
    std::memcpy(handle64, &h, sizeof(h));
    *ptr = p;
    return MOE_OK;
}

extern "C" int moe_peer_open(const void* handle64, void** ptr) {
    if (!ptr || !handle64) return MOE_ERR_INVALID_ARG;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle64, sizeof(h));
    return cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}

extern "C" int moe_peer_close(void* ptr) {
    return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}

extern "C" int moe_peer_free(void* ptr) { return cudaFree(ptr) == cudaSuccess ? MOE_OK : MOE_ERR_CUDA; }

extern "C" int moe_memcpy_async(void* dst, const void* src, size_t bytes, cudaStream_t stream) {
    if (bytes == 0) return MOE_OK;
    return cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, stream) == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}
