// Relay merge without caller-provided scratch: the no-allocation entry point.
//
// dbl_relay_merge_decode needs a workspace for the split-softmax partials, which the caller
// allocates.  Some callers cannot allocate device memory at the call site: a host whose device
// memory is owned by its own pooling allocator (the reference runs on Burn/CubeCL, whose runtime
// owns every device buffer it hands out), or a serving loop that must not call cudaMalloc /
// cudaFree on its critical path, since those calls can block on the device and can fail once
// memory is fragmented.  For them this variant keeps the scratch in a fixed array in device
// memory that is part of the library image: it is reserved when the library's module loads on a
// device and stays reserved on every device that loaded it until the process exits.
#include <cuda.h>

#include <mutex>

#include "common.cuh"

namespace dbl {

int relay_validate(const dbl_relay_merge_args* a);
size_t relay_call_workspace_bytes(const dbl_relay_merge_args* a);
int relay_launch(const dbl_relay_merge_args* a, void* ws, cudaStream_t st);

namespace {

constexpr size_t kScratchBytes = DBL_RELAY_NOALLOC_SCRATCH_BYTES;
static_assert(kScratchBytes % 256 == 0, "scratch size must keep the 256-byte section alignment");

// One copy per device.  In host code this name is only a host-side stand-in for the symbol, not
// a device address: the device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_relay_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mutex;
// Per device: the address resolved for the context whose id is g_scratch_ctx[dev].  Context ids
// (cuCtxGetId) are never reused within a process, so an address resolved in a context that was
// since destroyed (cudaDeviceReset) or in another context of the same device is never handed out.
void* g_scratch_ptr[kMaxDevices] = {};
unsigned long long g_scratch_ctx[kMaxDevices] = {};

typedef CUresult (*CtxGetCurrentFn)(CUcontext*);
typedef CUresult (*CtxGetIdFn)(CUcontext, unsigned long long*);

// Id of the calling thread's current context, or 0 when it cannot be read.
unsigned long long current_context_id() {
    static CtxGetCurrentFn get_current = nullptr;
    static CtxGetIdFn get_id = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult qr;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &qr) == cudaSuccess &&
            qr == cudaDriverEntryPointSuccess)
            get_current = reinterpret_cast<CtxGetCurrentFn>(p);
        p = nullptr;
        if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &qr) == cudaSuccess &&
            qr == cudaDriverEntryPointSuccess)
            get_id = reinterpret_cast<CtxGetIdFn>(p);
    });
    CUcontext ctx = nullptr;
    unsigned long long id = 0;
    if (!get_current || !get_id || get_current(&ctx) != CUDA_SUCCESS || !ctx || get_id(ctx, &id) != CUDA_SUCCESS)
        return 0;
    return id;
}

// The device address of the scratch array in the current context, resolved with
// cudaGetSymbolAddress the first time a context of this device calls (and again whenever the
// current context changes).
int scratch_for_current_device(void** out) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_status(e, "relay_noalloc: cudaGetDevice");
    if (dev < 0 || dev >= kMaxDevices) return fail(DBL_ERR_UNSUPPORTED, "relay_noalloc: device ordinal %d out of range", dev);
    const unsigned long long ctx = current_context_id();  // 0 until the runtime's context exists
    std::lock_guard<std::mutex> lock(g_mutex);
    if (!g_scratch_ptr[dev] || ctx == 0 || g_scratch_ctx[dev] != ctx) {
        void* ptr = nullptr;
        e = cudaGetSymbolAddress(&ptr, g_relay_scratch);  // also makes the device's context current
        if (e != cudaSuccess) return cuda_status(e, "relay_noalloc: cudaGetSymbolAddress");
        g_scratch_ptr[dev] = ptr;
        g_scratch_ctx[dev] = current_context_id();
    }
    *out = g_scratch_ptr[dev];
    return DBL_OK;
}

}  // namespace
}  // namespace dbl

// Same contract and results as dbl_relay_merge_decode, with the partials in the library's own
// fixed scratch array instead of a caller workspace.  No allocation of any kind is made.
extern "C" int dbl_relay_merge_decode_noalloc(const dbl_relay_merge_args* a, dbl_stream_t stream) {
    using namespace dbl;
    int rc = relay_validate(a);
    if (rc != DBL_OK) return rc;
    const size_t need = relay_call_workspace_bytes(a);
    if (need > kScratchBytes)
        return fail(DBL_ERR_WORKSPACE,
                    "relay_noalloc: this call needs %zu bytes of scratch, more than the fixed %zu-byte array; "
                    "use dbl_relay_merge_decode with a workspace",
                    need, kScratchBytes);
    void* ws = nullptr;
    rc = scratch_for_current_device(&ws);
    if (rc != DBL_OK) return rc;
    return relay_launch(a, ws, reinterpret_cast<cudaStream_t>(stream));
}
