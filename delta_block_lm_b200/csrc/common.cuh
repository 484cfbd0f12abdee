// Shared helpers for the GDN-2 sm_100a kernels and their C-ABI wrappers.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <cstdarg>
#include <cstdio>

#include "../../include/dbl_gdn2.h"

namespace dbl {

// Records the reason for a failure in thread-local storage and returns `status`.
int fail(int status, const char* fmt, ...);
// Device address of the library's kernel error word (read and cleared by dbl_device_error).
int device_error_record(int** out);

// Converts a CUDA error into DBL_ERR_CUDA with a message naming the call site.
inline int cuda_status(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return DBL_OK;
    return fail(DBL_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

// Checks the last launch on this thread.
inline int launch_status(const char* what) { return cuda_status(cudaGetLastError(), what); }

// Runs `set` (returning a DBL status) once per device for one call site, e.g. a kernel attribute,
// which the runtime keeps per device; `done` is the site's static set of devices already handled.
template <typename F>
inline int once_per_device(std::atomic<uint64_t>& done, F&& set) {
    int dev = 0;
    const cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_status(e, "cudaGetDevice");
    const uint64_t bit = dev >= 0 && dev < 64 ? uint64_t(1) << dev : 0;
    if (bit && (done.load(std::memory_order_acquire) & bit)) return DBL_OK;
    const int rc = set();
    if (rc == DBL_OK && bit) done.fetch_or(bit, std::memory_order_acq_rel);
    return rc;
}

template <typename T>
__device__ __forceinline__ float to_f32(T x);
template <>
__device__ __forceinline__ float to_f32<float>(float x) { return x; }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 x) {
    return __bfloat162float(x);
}

template <typename T>
__device__ __forceinline__ T from_f32(float x);
template <>
__device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) {
    return __float2bfloat16_rn(x);
}

// Fills `out` with the contiguous strides of a row-major tensor when `in` is all zeros,
// otherwise copies `in`.
inline void resolve_strides(const int64_t* in, const int64_t* dims, int rank, int64_t* out) {
    bool zero = true;
    for (int d = 0; d < rank; ++d) zero = zero && in[d] == 0;
    if (!zero) {
        for (int d = 0; d < rank; ++d) out[d] = in[d];
        return;
    }
    int64_t s = 1;
    for (int d = rank - 1; d >= 0; --d) {
        out[d] = s;
        s *= dims[d];
    }
}

inline bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

inline size_t dtype_size(int dtype) { return dtype == DBL_BF16 ? 2 : 4; }

}  // namespace dbl
