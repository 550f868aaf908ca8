// Peer device memory for expert parallelism over NVLink: buffers that other
// processes on the node map through CUDA IPC, so that the dispatch's gather
// kernels store rows straight into the owner's receive buffer and the
// owner's down-GEMM epilogue stores each result row straight into its
// sender's buffer (the transfer overlaps the GEMM tile by tile).  Failures
// return MOE_ERR_CUDA with the CUDA error text in moe_last_error().
#include "moe_internal.h"

#include <cstring>

namespace {

int fail(const char* what, cudaError_t err) {
    moe::set_error("%s: %s", what, cudaGetErrorString(err));
    return MOE_ERR_CUDA;
}

}  // namespace

extern "C" int moe_peer_alloc(size_t bytes, void** ptr, void* handle64) {
    if (!ptr || !handle64 || bytes == 0) return MOE_ERR_INVALID_ARG;
    void* p = nullptr;
    cudaError_t err = cudaMalloc(&p, bytes);
    if (err != cudaSuccess) return fail("moe_peer_alloc: cudaMalloc", err);
    cudaIpcMemHandle_t h;
    err = cudaIpcGetMemHandle(&h, p);
    if (err != cudaSuccess) {
        cudaFree(p);
        return fail("moe_peer_alloc: cudaIpcGetMemHandle", err);
    }
    std::memcpy(handle64, &h, sizeof(h));
    *ptr = p;
    return MOE_OK;
}

extern "C" int moe_peer_open(const void* handle64, void** ptr) {
    if (!ptr || !handle64) return MOE_ERR_INVALID_ARG;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle64, sizeof(h));
    const cudaError_t err = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
    return err == cudaSuccess ? MOE_OK : fail("moe_peer_open: cudaIpcOpenMemHandle", err);
}

extern "C" int moe_peer_close(void* ptr) {
    const cudaError_t err = cudaIpcCloseMemHandle(ptr);
    return err == cudaSuccess ? MOE_OK : fail("moe_peer_close: cudaIpcCloseMemHandle", err);
}

extern "C" int moe_peer_free(void* ptr) {
    const cudaError_t err = cudaFree(ptr);
    return err == cudaSuccess ? MOE_OK : fail("moe_peer_free: cudaFree", err);
}

extern "C" int moe_memcpy_async(void* dst, const void* src, size_t bytes, cudaStream_t stream) {
    if (bytes == 0) return MOE_OK;
    const cudaError_t err = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, stream);
    return err == cudaSuccess ? MOE_OK : fail("moe_memcpy_async: cudaMemcpyAsync", err);
}
