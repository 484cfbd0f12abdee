// dbl_gdn2_prefill / dbl_gdn2_span_transition: validation and kernel selection.
//
// bf16 q/k/v with K = V = 128 and unit inner strides run on the chunked tcgen05 kernel
// (prefill_tc.cu).  Every other accepted shape (f32 inputs, K or V of 64, strided inner axes)
// runs on the token-sequential kernel (scan_seq.cu) in f32.  Both are CUDA kernels; there is
// no host fallback.
#include "scan_seq_params.cuh"

namespace dbl {

// prefill_tc.cu
int tc_prefill_supported(const dbl_prefill_args* a, const int64_t* qs, const int64_t* ks, const int64_t* vs,
                         const int64_t* os);
int tc_prefill_launch(const dbl_prefill_args* a, const int64_t* qs, const int64_t* ks, const int64_t* vs,
                      const int64_t* as, const int64_t* bs, const int64_t* os, int mode, float* transition,
                      cudaStream_t st);

namespace {

int validate_prefill(const dbl_prefill_args* a, bool need_values) {
    if (!a) return fail(DBL_ERR_INVALID_ARGUMENT, "prefill: null args");
    if (a->batch <= 0 || a->time <= 0 || a->heads <= 0)
        return fail(DBL_ERR_INVALID_ARGUMENT, "GDN-2 requires nonempty axes");
    if (a->key_dim <= 0 || a->value_dim <= 0)
        return fail(DBL_ERR_INVALID_ARGUMENT, "GDN-2 requires nonempty key and value widths");
    if (a->batch > 0x7fffffff || a->time > 0x7fffffff || a->heads > 0x7fffffff)
        return fail(DBL_ERR_UNSUPPORTED, "GDN-2 axis exceeds 32-bit limits");
    if (a->dtype != DBL_F32 && a->dtype != DBL_BF16)
        return fail(DBL_ERR_INVALID_ARGUMENT, "prefill: dtype must be f32 or bf16");
    if (a->chunk_size != 0 && a->chunk_size != 64)
        return fail(DBL_ERR_UNSUPPORTED, "prefill: chunk_size must be 64 (or 0 for the default)");
    if (!a->q || !a->k || !a->alpha || !a->beta)
        return fail(DBL_ERR_INVALID_ARGUMENT, "prefill: q, k, alpha and beta are required");
    if (need_values && !a->v) return fail(DBL_ERR_INVALID_ARGUMENT, "prefill: v is required");
    if ((a->valid == nullptr) != (a->reset == nullptr))
        return fail(DBL_ERR_INVALID_ARGUMENT, "prefill: valid and reset must be given together");
    return DBL_OK;
}

}  // namespace

// mode 0: prefill; mode 1: span transition (identity initial state, zero values).
int prefill_dispatch(const dbl_prefill_args* a, int mode, float* transition, cudaStream_t st) {
    const int64_t dk[4] = {a->batch, a->time, a->heads, a->key_dim};
    const int64_t dv[4] = {a->batch, a->time, a->heads, a->value_dim};
    const int64_t dg[3] = {a->batch, a->time, a->heads};
    int64_t qs[4], ks[4], vs[4], os[4], as[3], bs[3];
    resolve_strides(a->q_stride, dk, 4, qs);
    resolve_strides(a->k_stride, dk, 4, ks);
    resolve_strides(a->v_stride, dv, 4, vs);
    resolve_strides(a->out_stride, dv, 4, os);
    resolve_strides(a->alpha_stride, dg, 3, as);
    resolve_strides(a->beta_stride, dg, 3, bs);
    if (tc_prefill_supported(a, qs, ks, vs, os)) return tc_prefill_launch(a, qs, ks, vs, as, bs, os, mode, transition, st);

    SeqParams p{};
    p.B = (int)a->batch;
    p.T = (int)a->time;
    p.H = (int)a->heads;
    p.K = (int)a->key_dim;
    p.V = mode == 1 ? (int)a->key_dim : (int)a->value_dim;
    p.q = a->q;
    p.k = a->k;
    p.v = mode == 1 ? a->k : a->v;  // unused in transition mode (v_zero)
    for (int d = 0; d < 4; ++d) {
        p.qs[d] = qs[d];
        p.ks[d] = ks[d];
        p.vs[d] = mode == 1 ? ks[d] : vs[d];
        p.os[d] = os[d];
    }
    p.gate_mode = 1;
    p.alpha = a->alpha;
    p.erase = a->beta;
    for (int d = 0; d < 3; ++d) {
        p.as[d] = as[d];
        p.es[d] = bs[d];
    }
    p.scale = a->scale;
    p.mask_mode = a->valid ? 1 : 0;
    p.valid = a->valid;
    p.reset = a->reset;
    if (mode == 1) {
        p.init_mode = 2;
        p.v_zero = 1;
        p.out = nullptr;
        p.final_state = transition;
    } else {
        p.init_mode = a->initial_state ? 1 : 0;
        p.initial = a->initial_state;
        p.out = a->out;
        p.out_dtype = a->dtype;
        p.final_state = a->final_state;
    }
    return launch_seq_scan(p, a->dtype, st);
}

}  // namespace dbl

extern "C" int dbl_gdn2_prefill(const dbl_prefill_args* a, dbl_stream_t stream) {
    using namespace dbl;
    int rc = validate_prefill(a, true);
    if (rc != DBL_OK) return rc;
    if (a->initial_state && !aligned(a->initial_state, 16))
        return fail(DBL_ERR_INVALID_ARGUMENT, "prefill: initial_state must be 16-byte aligned");
    if (a->final_state && !aligned(a->final_state, 16))
        return fail(DBL_ERR_INVALID_ARGUMENT, "prefill: final_state must be 16-byte aligned");
    return prefill_dispatch(a, 0, nullptr, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int dbl_gdn2_span_transition(const dbl_prefill_args* a, float* transition, dbl_stream_t stream) {
    using namespace dbl;
    int rc = validate_prefill(a, false);
    if (rc != DBL_OK) return rc;
    if (!transition) return fail(DBL_ERR_INVALID_ARGUMENT, "span_transition: transition output is required");
    if (!aligned(transition, 16)) return fail(DBL_ERR_INVALID_ARGUMENT, "span_transition: transition must be 16-byte aligned");
    return prefill_dispatch(a, 1, transition, reinterpret_cast<cudaStream_t>(stream));
}
