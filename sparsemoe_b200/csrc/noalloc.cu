// moe_solve_v2_noalloc: the whole layer with its scratch in a fixed,
// statically sized device array instead of memory the library allocates.
//
// Who needs it: callers that cannot let this library call cudaMalloc --
// engines that hand out every byte of device memory from their own
// pre-planned pool (a side allocation breaks their accounting and can fail
// once the pool has taken the GPU), and latency-critical serving loops where
// the implicit device synchronisation of cudaMalloc / cudaFree is not
// acceptable.  They still pass every input and output buffer in MoEArgs;
// only the library's own routing tables move into the array below.
//
// Limits and sharing:
//  * The array is kNoAllocScratchBytes (4 MiB) per GPU that loads the library
//    and stays allocated until the process exits.  A call whose scratch
//    (moe_workspace_bytes(dims)) exceeds it is rejected with
//    MOE_ERR_UNSUPPORTED and a message naming both sizes.  4 MiB covers, for
//    example, the Mixtral-shape call of 16384 tokens at top-2 over 8 experts
//    (about 0.14 MiB) or a decode call of 512 tokens at top-8 over 256
//    experts with d_model = 1024 (about 1 MiB); routers over 64 or more
//    experts add 4 * tokens * experts * ceil(d_model / 512) bytes of partial
//    logits, so large many-expert calls need moe_solve_v2.
//  * Every call on a device shares the one array and leaves its contents
//    behind.  The kernels rewrite every table entry they read in each call;
//    the status word is cleared at the start of each call.  Two calls whose
//    kernels overlap on the GPU (different streams, no ordering between them)
//    race on the array; order them on one stream or with events.
//  * The first call on each device looks up the array's device address with
//    cudaGetSymbolAddress (with that device current) and caches it; make that
//    first call before any stream capture.  The cache lives as long as the
//    process's CUDA context: after cudaDeviceReset the cached address is
//    stale, so a process that resets a device must not call this entry point
//    on that device again.
//  * MoeDims.act_scale is honoured as in moe_solve_v2 (the dynamic formats'
//    per-row activation scales go to the caller's buffer instead of the
//    array; the size check still counts them).  MoeDims.scratch must be
//    null: a caller that has scratch of its own calls moe_solve_v2 with it.
#include "moe_internal.h"

#include <mutex>

namespace moe {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(4) << 20;
constexpr int kMaxDevicesNoAlloc = 64;

__device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kMaxDevicesNoAlloc] = {};

// Device address of g_noalloc_scratch on `dev` (the current device).  In host
// code the symbol itself is only a host-side stand-in, never a device address.
int scratch_address(int dev, void** out) {
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) {
            set_error("cudaGetSymbolAddress(no-alloc scratch): %s", cudaGetErrorString(e));
            return MOE_ERR_CUDA;
        }
        g_noalloc_ptr[dev] = p;
    }
    *out = g_noalloc_ptr[dev];
    return MOE_OK;
}

}  // namespace
}  // namespace moe

using namespace moe;

extern "C" size_t moe_noalloc_scratch_bytes(void) { return kNoAllocScratchBytes; }

extern "C" int moe_solve_v2_noalloc(const MoEArgs* a, const MoeDims* dims, cudaStream_t stream) {
    Shape s;
    int rc = make_shape_checked(dims, &s);
    if (rc != MOE_OK) return rc;
    rc = check_args(a, s.dtype);
    if (rc != MOE_OK) return rc;
    rc = check_norm(dims);
    if (rc != MOE_OK) return rc;
    if (dims->scratch) {
        set_error("moe_solve_v2_noalloc: MoeDims.scratch must be null (pass caller scratch to moe_solve_v2)");
        return MOE_ERR_INVALID_ARG;
    }
    const size_t need = workspace_bytes(s);
    if (need > kNoAllocScratchBytes) {
        set_error("moe_solve_v2_noalloc: this call needs %zu bytes of scratch, the static array holds %zu "
                  "(use moe_solve_v2 for larger calls)",
                  need, kNoAllocScratchBytes);
        return MOE_ERR_UNSUPPORTED;
    }
    int dev = 0, num_sms = 0;
    rc = current_device(&dev, &num_sms);
    if (rc != MOE_OK) return rc;
    if (dev >= kMaxDevicesNoAlloc) {
        set_error("device ordinal %d too large", dev);
        return MOE_ERR_INVALID_ARG;
    }
    void* base = nullptr;
    rc = scratch_address(dev, &base);
    if (rc != MOE_OK) return rc;
    Workspace ws;
    carve_workspace(base, s, &ws);
    if (dims->act_scale) ws.a_scale = dims->act_scale;
    note_status_word(dev, ws.status);
    return enqueue_layer(a, dims, s, ws, num_sms, stream);
}
