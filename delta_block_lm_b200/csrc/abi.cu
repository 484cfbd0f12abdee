// Status strings, thread-local error messages and the ABI version of libdbl_gdn2.
#include "common.cuh"

namespace dbl {

static thread_local char g_last_error[512] = "no error";

int fail(int status, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
    va_end(ap);
    return status;
}

}  // namespace dbl

extern "C" const char* dbl_status_string(int status) {
    switch (status) {
        case DBL_OK: return "ok";
        case DBL_ERR_INVALID_ARGUMENT: return "invalid argument";
        case DBL_ERR_UNSUPPORTED: return "unsupported configuration";
        case DBL_ERR_CUDA: return "CUDA error";
        case DBL_ERR_WORKSPACE: return "workspace missing or too small";
        case DBL_ERR_TIMEOUT: return "timed out";
        default: return "unknown status";
    }
}

extern "C" const char* dbl_last_error(void) { return dbl::g_last_error; }

extern "C" int dbl_abi_version(void) { return 10100; }  // 1.1.0: span fold, segmented and time-sharded prefill, per-call relay workspace size
