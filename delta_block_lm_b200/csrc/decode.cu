// Single-token GDN-2 decode step, state updated in place.
//
// One CTA per (sequence, head).  The K x V f32 state is streamed once from HBM into registers
// with 16-byte loads (warp w owns rows [w*K/8, (w+1)*K/8), lane l owns columns
// [l*V/32, (l+1)*V/32)), reduced against k and q, and written back once.  With
// S' = alpha S the reference step (crates/mixers/src/gdn2_reference.rs:52-83, scalar gates) is
//     edit_j = beta v_j - alpha beta (k^T S)_j
//     o_j    = alpha (q^T S)_j + (q . k) edit_j
//     S_ij  <- alpha S_ij + k_i edit_j
// so the old state is read once and the new one written once: 2*K*V*4 bytes per head-step,
// the algorithmic minimum.  Roofline: HBM.
#include "common.cuh"

namespace dbl {
namespace {

struct DecodeParams {
    int N, H;
    float scale;
    const void *q, *k, *v;
    int64_t qs[3], ks[3], vs[3], os[3];
    const float *alpha, *beta;
    float* state;
    void* out;
};

template <int V>
struct Vec;
template <>
struct Vec<128> {
    using type = float4;
    static constexpr int n = 4;
};
template <>
struct Vec<64> {
    using type = float2;
    static constexpr int n = 2;
};

template <int K, int V, typename T>
__global__ void __launch_bounds__(256, 2) decode_step_kernel(const DecodeParams p) {
    constexpr int NW = 8;
    constexpr int VEC = Vec<V>::n;
    constexpr int ROWS = K / NW;
    using VT = typename Vec<V>::type;
    static_assert(V == 32 * VEC, "lane covers V/32 columns");

    __shared__ float sq[K], sk[K], sv[V];
    __shared__ __align__(16) float red[2][NW][V];
    __shared__ float s_qk;

    const int nh = blockIdx.x;
    const int n = nh / p.H, h = nh - n * p.H;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    // Issue the state loads first: ROWS x 16 B per thread in flight.
    float* S = p.state + (size_t)nh * K * V;
    VT s[ROWS];
#pragma unroll
    for (int r = 0; r < ROWS; ++r)
        s[r] = __ldcs(reinterpret_cast<const VT*>(S + (size_t)(warp * ROWS + r) * V) + lane);

    const T* q = static_cast<const T*>(p.q) + n * p.qs[0] + h * p.qs[1];
    const T* k = static_cast<const T*>(p.k) + n * p.ks[0] + h * p.ks[1];
    const T* v = static_cast<const T*>(p.v) + n * p.vs[0] + h * p.vs[1];
    for (int i = tid; i < K; i += 256) {
        sq[i] = to_f32(q[i * p.qs[2]]) * p.scale;
        sk[i] = to_f32(k[i * p.ks[2]]);
    }
    for (int j = tid; j < V; j += 256) sv[j] = to_f32(v[j * p.vs[2]]);
    const float alpha = p.alpha[nh];
    const float beta = p.beta[nh];
    __syncthreads();

    float ak[VEC], aq[VEC];
#pragma unroll
    for (int c = 0; c < VEC; ++c) ak[c] = aq[c] = 0.f;
#pragma unroll
    for (int r = 0; r < ROWS; ++r) {
        const float ki = sk[warp * ROWS + r], qi = sq[warp * ROWS + r];
        const float* sr = reinterpret_cast<const float*>(&s[r]);
#pragma unroll
        for (int c = 0; c < VEC; ++c) {
            ak[c] = fmaf(ki, sr[c], ak[c]);
            aq[c] = fmaf(qi, sr[c], aq[c]);
        }
    }
#pragma unroll
    for (int c = 0; c < VEC; ++c) {
        red[0][warp][lane * VEC + c] = ak[c];
        red[1][warp][lane * VEC + c] = aq[c];
    }
    if (warp == 0) {
        float d = 0.f;
        for (int i = lane; i < K; i += 32) d = fmaf(sq[i], sk[i], d);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
        if (lane == 0) s_qk = d;
    }
    __syncthreads();

    float edit[VEC], outv[VEC];
#pragma unroll
    for (int c = 0; c < VEC; ++c) {
        float a = 0.f, b = 0.f;
#pragma unroll
        for (int w = 0; w < NW; ++w) {
            a += red[0][w][lane * VEC + c];
            b += red[1][w][lane * VEC + c];
        }
        const int j = lane * VEC + c;
        edit[c] = beta * sv[j] - alpha * beta * a;
        outv[c] = alpha * b + s_qk * edit[c];
    }
    if (warp == 0) {
        T* o = static_cast<T*>(p.out) + n * p.os[0] + h * p.os[1];
#pragma unroll
        for (int c = 0; c < VEC; ++c) o[(lane * VEC + c) * p.os[2]] = from_f32<T>(outv[c]);
    }
#pragma unroll
    for (int r = 0; r < ROWS; ++r) {
        const float ki = sk[warp * ROWS + r];
        float* sr = reinterpret_cast<float*>(&s[r]);
#pragma unroll
        for (int c = 0; c < VEC; ++c) sr[c] = fmaf(alpha, sr[c], ki * edit[c]);
        __stcs(reinterpret_cast<VT*>(S + (size_t)(warp * ROWS + r) * V) + lane, s[r]);
    }
}

template <int K, int V>
int launch_decode(const DecodeParams& p, int dtype, cudaStream_t st) {
    const unsigned grid = (unsigned)(p.N * p.H);
    if (dtype == DBL_BF16)
        decode_step_kernel<K, V, __nv_bfloat16><<<grid, 256, 0, st>>>(p);
    else
        decode_step_kernel<K, V, float><<<grid, 256, 0, st>>>(p);
    return launch_status("decode_step_kernel");
}

}  // namespace
}  // namespace dbl

extern "C" int dbl_gdn2_decode_step(const dbl_decode_args* a, dbl_stream_t stream) {
    using namespace dbl;
    if (!a) return fail(DBL_ERR_INVALID_ARGUMENT, "decode: null args");
    if (a->batch <= 0 || a->heads <= 0)
        return fail(DBL_ERR_INVALID_ARGUMENT, "decode: batch and heads must be positive");
    if (a->batch * a->heads > 0x7fffffffLL)
        return fail(DBL_ERR_UNSUPPORTED, "decode: batch*heads exceeds the grid limit");
    const int64_t K = a->key_dim, V = a->value_dim;
    if (!((K == 64 || K == 128) && (V == 64 || V == 128)))
        return fail(DBL_ERR_UNSUPPORTED, "decode: key_dim and value_dim must be 64 or 128 (got %lld, %lld)",
                    (long long)K, (long long)V);
    if (a->dtype != DBL_F32 && a->dtype != DBL_BF16)
        return fail(DBL_ERR_INVALID_ARGUMENT, "decode: dtype must be f32 or bf16");
    if (!a->q || !a->k || !a->v || !a->alpha || !a->beta || !a->state || !a->out)
        return fail(DBL_ERR_INVALID_ARGUMENT, "decode: q, k, v, alpha, beta, state and out are required");
    if (!aligned(a->state, 16))
        return fail(DBL_ERR_INVALID_ARGUMENT, "decode: state must be 16-byte aligned");
    DecodeParams p{};
    p.N = (int)a->batch;
    p.H = (int)a->heads;
    p.scale = a->scale;
    p.q = a->q;
    p.k = a->k;
    p.v = a->v;
    const int64_t dk[3] = {a->batch, a->heads, K}, dv[3] = {a->batch, a->heads, V};
    resolve_strides(a->q_stride, dk, 3, p.qs);
    resolve_strides(a->k_stride, dk, 3, p.ks);
    resolve_strides(a->v_stride, dv, 3, p.vs);
    resolve_strides(a->out_stride, dv, 3, p.os);
    p.alpha = a->alpha;
    p.beta = a->beta;
    p.state = a->state;
    p.out = a->out;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (K == 128 && V == 128) return launch_decode<128, 128>(p, a->dtype, st);
    if (K == 128 && V == 64) return launch_decode<128, 64>(p, a->dtype, st);
    if (K == 64 && V == 128) return launch_decode<64, 128>(p, a->dtype, st);
    return launch_decode<64, 64>(p, a->dtype, st);
}
