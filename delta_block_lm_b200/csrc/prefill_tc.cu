// Chunked GDN-2 prefill on tcgen05 tensor cores (bf16, K = V = 128, chunk 64).
// Selection hook used by prefill.cu; the kernel itself is added in this file.
#include "common.cuh"

namespace dbl {

int tc_prefill_supported(const dbl_prefill_args*, const int64_t*, const int64_t*, const int64_t*, const int64_t*) {
    return 0;
}

int tc_prefill_launch(const dbl_prefill_args*, const int64_t*, const int64_t*, const int64_t*, const int64_t*,
                      const int64_t*, const int64_t*, int, float*, cudaStream_t) {
    return fail(DBL_ERR_UNSUPPORTED, "tensor-core prefill is not available");
}

}  // namespace dbl
