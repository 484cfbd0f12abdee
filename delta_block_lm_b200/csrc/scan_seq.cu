// Token-sequential GDN-2 scan: the reference's stateful fused recurrence, generalised.
//
// Serves the reference contracts that carry channel-wise gates and masks:
//   dbl_gdn_training_scan  <- delta_kernels::gdn_training_scan (gdn_training.rs:12-115)
//   dbl_gdn2_scan          <- delta_kernels::gdn2_scan (ops.rs:251-276; doc-limit masks)
// and the scalar-gate prefill at shapes the tensor-core kernel does not take (f32 inputs,
// K or V other than 128), e.g. BASELINE config 0.
//
// One CTA per (b, h); four lanes (two when V > 128) share state column j, each holding every
// fourth row (the reference kernel gives a lane a whole value column, gdn_training.rs:28-49), so
// that a step's row sums are short chains plus two shuffles.  Tokens are staged TOK at a time in
// shared memory (k, q, gates and each column's write v) so a CTA synchronises twice per TOK tokens,
// not per token.  Step order is the
// reference's (reference.rs:62-108): padding -> o = 0, state kept; reset -> S = 0; decay;
// edit = write v - sum_i erase_i k_i S_i; score = |k||edit|; S += k edit; o = q^T S.
#include "scan_seq_params.cuh"

namespace dbl {



namespace {

constexpr int TOKB = 8;  // tokens staged per group (doubled for small key widths)

// TPC lanes share value column j (lane / TPC within the warp's group of 32 / TPC columns); lane g =
// lane % TPC owns state rows i = g, g + TPC, g + 2 TPC, ... (strided, so that the TPC lanes read
// adjacent shared-memory words), KMAX / TPC of them.  The two row sums of a step (k^T bar erase and
// q^T S) are reduced over the TPC lanes with shuffles.
template <int TPC>
__device__ __forceinline__ float row_sum(float x) {
#pragma unroll
    for (int o = 1; o < TPC; o <<= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
    return x;
}

template <int KMAX, typename T, bool SCALAR, int TPC>
__global__ void __launch_bounds__(512) seq_scan_kernel(const SeqParams p) {
    constexpr int R = KMAX / TPC;
    // tokens staged per group: 16 where the group's arrays still fit the static shared memory
    constexpr int TOK = KMAX <= 32 ? 2 * TOKB : TOKB;
    __shared__ float sk[TOK][KMAX], sq[TOK][KMAX];
    __shared__ float sa[SCALAR ? 1 : TOK][KMAX], se[SCALAR ? 1 : TOK][KMAX];  // se: erase_i k_i
    __shared__ float sga[TOK], sgb[TOK];  // scalar gates
    __shared__ int sact[TOK], srst[TOK];
    __shared__ float sdl[TOK][256];       // each column's edit, for the scores after the group
    __shared__ float svw[TOK][256];       // write_j v_j (beta: v_j) of the staged tokens

    const int bh = blockIdx.x;
    // routed launches: this (b, h) is served by the tensor-core kernel of the call
    if (p.route && ((p.route[bh] != 0) != (p.route_want != 0))) return;
    const int b = bh / p.H, h = bh - b * p.H;
    const int tid = threadIdx.x, nthr = blockDim.x;
    const int warp = tid >> 5, lane = tid & 31, nwarps = nthr >> 5;
    const int g = lane % TPC;
    const int j = warp * (32 / TPC) + lane / TPC;  // value column
    const bool col = j < p.V;

    float S[R];
    const size_t sbase = ((size_t)b * p.H + h) * p.K * p.V;
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const int i = g + TPC * r;
        float x = 0.f;
        if (col && i < p.K) {
            if (p.init_mode == 1) x = p.initial[sbase + (size_t)i * p.V + j];
            else if (p.init_mode == 2) x = (i == j) ? 1.f : 0.f;
        }
        S[r] = x;
    }

    const T* qb = static_cast<const T*>(p.q) + b * p.qs[0] + h * p.qs[2];
    const T* kb = static_cast<const T*>(p.k) + b * p.ks[0] + h * p.ks[2];
    const T* vb = static_cast<const T*>(p.v) + b * p.vs[0] + h * p.vs[2];

    for (int t0 = 0; t0 < p.T; t0 += TOK) {
        const int nt = min(TOK, p.T - t0);
        __syncthreads();  // previous group's shared reads are complete
        for (int x = tid; x < TOK * KMAX; x += nthr) {
            const int u = x / KMAX, i = x - u * KMAX;
            float kv = 0.f, qv = 0.f, av = 1.f, ev = 0.f;
            if (u < nt && i < p.K) {
                const int t = t0 + u;
                kv = to_f32(kb[t * p.ks[1] + i * p.ks[3]]);
                qv = to_f32(qb[t * p.qs[1] + i * p.qs[3]]) * p.scale;
                if (!SCALAR) {
                    const size_t ga = (size_t)b * p.as[0] + (size_t)t * p.as[1] + (size_t)h * p.as[2] + (size_t)i * p.as[3];
                    const size_t ge = (size_t)b * p.es[0] + (size_t)t * p.es[1] + (size_t)h * p.es[2] + (size_t)i * p.es[3];
                    av = p.alpha[ga];
                    ev = p.erase[ge];
                }
            }
            sk[u][i] = kv;
            sq[u][i] = qv;
            if (!SCALAR) {
                sa[u][i] = av;
                se[u][i] = ev * kv;
            }
        }
        if (g == 0 && col) {
            // this column's write * v for the group: every load in flight before the stores
            float vv[TOK], ww[TOK];
#pragma unroll
            for (int u = 0; u < TOK; ++u) {
                const int t = t0 + u;
                vv[u] = (u < nt && !p.v_zero) ? to_f32(vb[t * p.vs[1] + j * p.vs[3]]) : 0.f;
                ww[u] = (u < nt && !SCALAR)
                            ? p.write[(size_t)b * p.ws[0] + (size_t)t * p.ws[1] + (size_t)h * p.ws[2] + (size_t)j * p.ws[3]]
                            : 0.f;
            }
#pragma unroll
            for (int u = 0; u < TOK; ++u) svw[u][j] = SCALAR ? vv[u] : ww[u] * vv[u];
        }
        if (tid < TOK) {
            const int u = tid, t = t0 + u;
            int act = 0, rst = 0;
            float ga = 1.f, gb = 0.f;
            if (u < nt) {
                if (p.mask_mode == 1) {
                    act = p.valid[(size_t)b * p.T + t] != 0.f;
                    rst = p.reset[(size_t)b * p.T + t] != 0.f;
                } else if (p.mask_mode == 2) {
                    const int32_t st = p.doc_start[(size_t)b * p.T + t], en = p.doc_end[(size_t)b * p.T + t];
                    act = en >= st;
                    rst = st == t;
                } else {
                    act = 1;
                }
                if (SCALAR) {
                    ga = p.alpha[(size_t)b * p.as[0] + (size_t)t * p.as[1] + (size_t)h * p.as[2]];
                    gb = p.erase[(size_t)b * p.es[0] + (size_t)t * p.es[1] + (size_t)h * p.es[2]];
                }
            }
            sact[u] = act;
            srst[u] = rst;
            sga[u] = ga;
            sgb[u] = gb;
        }
        __syncthreads();

        for (int u = 0; u < nt; ++u) {
            const int t = t0 + u;
            const bool act = sact[u] != 0;
            float delta = 0.f, o = 0.f;
            if (act) {
                const bool rst = srst[u] != 0;
                const float wv = col ? svw[u][j] : 0.f;
                float part = 0.f;
                if (SCALAR) {
                    const float a = rst ? 0.f : sga[u];
#pragma unroll
                    for (int r = 0; r < R; ++r) {
                        const int i = g + TPC * r;
                        S[r] *= a;
                        part = fmaf(sk[u][i], S[r], part);
                    }
                    // beta v - beta k^T S
                    delta = sgb[u] * (wv - row_sum<TPC>(part));
                } else {
#pragma unroll
                    for (int r = 0; r < R; ++r) {
                        const int i = g + TPC * r;
                        S[r] = rst ? 0.f : S[r] * sa[u][i];
                        part = fmaf(se[u][i], S[r], part);
                    }
                    delta = wv - row_sum<TPC>(part);
                }
                float op = 0.f;
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    const int i = g + TPC * r;
                    S[r] = fmaf(sk[u][i], delta, S[r]);
                    op = fmaf(sq[u][i], S[r], op);
                }
                o = row_sum<TPC>(op);
            }
            if (p.out && col && g == 0) {
                const size_t oi = (size_t)b * p.os[0] + (size_t)t * p.os[1] + (size_t)h * p.os[2] + (size_t)j * p.os[3];
                if (p.out_dtype == DBL_BF16) static_cast<__nv_bfloat16*>(p.out)[oi] = __float2bfloat16_rn(o);
                else static_cast<float*>(p.out)[oi] = o;
            }
            if (p.scores && g == 0 && col) sdl[u][j] = delta;
        }
        if (p.scores) {
            // score = |k| |edit| per token of the group: one warp per token
            __syncthreads();
            for (int u = warp; u < nt; u += nwarps) {
                const int t = t0 + u;
                float kk = 0.f, d2 = 0.f;
                for (int i = lane; i < p.K; i += 32) kk = fmaf(sk[u][i], sk[u][i], kk);
                for (int c = lane; c < p.V; c += 32) d2 = fmaf(sdl[u][c], sdl[u][c], d2);
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) {
                    kk += __shfl_xor_sync(0xffffffffu, kk, off);
                    d2 += __shfl_xor_sync(0xffffffffu, d2, off);
                }
                if (lane == 0) p.scores[((size_t)b * p.T + t) * p.H + h] = sact[u] ? sqrtf(kk) * sqrtf(d2) : 0.f;
            }
        }
    }
    if (p.final_state && col) {
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const int i = g + TPC * r;
            if (i < p.K) p.final_state[sbase + (size_t)i * p.V + j] = S[r];
        }
    }
}

template <int KMAX, typename T>
int launch_seq_t(const SeqParams& p, cudaStream_t st) {
    const unsigned grid = (unsigned)(p.B * p.H);
    // four lanes per value column up to 128 columns, two beyond (at most 512 threads)
    if (p.V <= 128) {
        const int threads = ((p.V * 4 + 31) / 32) * 32;
        if (p.gate_mode == 1) seq_scan_kernel<KMAX, T, true, 4><<<grid, threads, 0, st>>>(p);
        else seq_scan_kernel<KMAX, T, false, 4><<<grid, threads, 0, st>>>(p);
    } else {
        const int threads = ((p.V * 2 + 31) / 32) * 32;
        if (p.gate_mode == 1) seq_scan_kernel<KMAX, T, true, 2><<<grid, threads, 0, st>>>(p);
        else seq_scan_kernel<KMAX, T, false, 2><<<grid, threads, 0, st>>>(p);
    }
    return launch_status("seq_scan_kernel");
}

}  // namespace

// Validates shape limits shared by every caller, then launches.
int launch_seq_scan(const SeqParams& p, int in_dtype, cudaStream_t st) {
    if (p.B <= 0 || p.T <= 0 || p.H <= 0 || p.K <= 0 || p.V <= 0)
        return fail(DBL_ERR_INVALID_ARGUMENT, "GDN-2 requires nonempty axes");
    if (p.K > 128) return fail(DBL_ERR_UNSUPPORTED, "sequential scan supports key_dim <= 128 (got %d)", p.K);
    if (p.V > 256) return fail(DBL_ERR_UNSUPPORTED, "sequential scan supports value_dim <= 256 (got %d)", p.V);
    if ((int64_t)p.B * p.H > 0x7fffffffLL) return fail(DBL_ERR_UNSUPPORTED, "batch*heads exceeds the grid limit");
    if (chunk_scan_supported(p)) return launch_chunk_scan(p, in_dtype, st);
    const bool bf = in_dtype == DBL_BF16;
    if (p.K <= 32) return bf ? launch_seq_t<32, __nv_bfloat16>(p, st) : launch_seq_t<32, float>(p, st);
    if (p.K <= 64) return bf ? launch_seq_t<64, __nv_bfloat16>(p, st) : launch_seq_t<64, float>(p, st);
    return bf ? launch_seq_t<128, __nv_bfloat16>(p, st) : launch_seq_t<128, float>(p, st);
}

}  // namespace dbl

// --------------------------------------------------------------------------------------------
namespace dbl {

// Checks the arguments of the training-scan forward and fills the scan parameters.
int training_scan_params(const dbl_training_scan_args* a, SeqParams* out) {
    if (!a) return fail(DBL_ERR_INVALID_ARGUMENT, "gdn_training_scan: null args");
    if (a->batch <= 0 || a->time <= 0 || a->heads <= 0)
        return fail(DBL_ERR_INVALID_ARGUMENT, "GDN-2 requires nonempty axes");
    if (a->key_dim <= 0 || a->value_dim <= 0)
        return fail(DBL_ERR_INVALID_ARGUMENT, "GDN-2 requires nonempty key and value widths");
    if (a->chunk_size < 1 || a->chunk_size > 16)
        return fail(DBL_ERR_INVALID_ARGUMENT, "GDN-2 checkpoint chunk must be 1..=16");
    if (a->dtype != DBL_F32 && a->dtype != DBL_BF16)
        return fail(DBL_ERR_INVALID_ARGUMENT, "fused GDN-2 supports f32 or bf16 q/k/v");
    if (!a->q || !a->k || !a->v || !a->alpha || !a->erase || !a->write || !a->valid || !a->reset || !a->output)
        return fail(DBL_ERR_INVALID_ARGUMENT,
                    "gdn_training_scan: q, k, v, alpha, erase, write, valid, reset and output are required");
    if (a->batch > 0x7fffffff || a->time > 0x7fffffff || a->heads > 0x7fffffff || a->key_dim > 0x7fffffff ||
        a->value_dim > 0x7fffffff)
        return fail(DBL_ERR_UNSUPPORTED, "GDN-2 axis exceeds 32-bit limits");
    SeqParams p{};
    p.B = (int)a->batch;
    p.T = (int)a->time;
    p.H = (int)a->heads;
    p.K = (int)a->key_dim;
    p.V = (int)a->value_dim;
    const int64_t dk[4] = {a->batch, a->time, a->heads, a->key_dim};
    const int64_t dv[4] = {a->batch, a->time, a->heads, a->value_dim};
    const int64_t z[4] = {0, 0, 0, 0};
    p.q = a->q;
    p.k = a->k;
    p.v = a->v;
    resolve_strides(z, dk, 4, p.qs);
    resolve_strides(z, dk, 4, p.ks);
    resolve_strides(z, dv, 4, p.vs);
    p.gate_mode = 0;
    p.alpha = a->alpha;
    p.erase = a->erase;
    p.write = a->write;
    resolve_strides(z, dk, 4, p.as);
    resolve_strides(z, dk, 4, p.es);
    resolve_strides(z, dv, 4, p.ws);
    p.scale = 1.f;
    p.mask_mode = 1;
    p.valid = a->valid;
    p.reset = a->reset;
    p.init_mode = a->initial_state ? 1 : 0;
    p.initial = a->initial_state;
    p.out = a->output;
    p.out_dtype = DBL_F32;
    resolve_strides(z, dv, 4, p.os);
    p.final_state = a->final_state;
    p.scores = a->scores;
    *out = p;
    return DBL_OK;
}

}  // namespace dbl

// delta_kernels::gdn_training_scan (crates/kernels/src/gdn_training_ops.rs:288-333) forward.
namespace dbl {

bool tc_training_scan_supported(const dbl_training_scan_args* a);
int tc_training_scan_launch(const dbl_training_scan_args* a, const int* route, int route_want, cudaStream_t st);

namespace {

// flags[b * H + h] |= 1 when some token row of (b, h) has alpha, erase or write that differ across
// channels.  One warp per (b, t, h) row; K = V = 128 (four channels per lane).
__global__ void __launch_bounds__(256) gate_uniform_kernel(const float* __restrict__ alpha,
                                                           const float* __restrict__ erase,
                                                           const float* __restrict__ write, int64_t rows, int TH,
                                                           int H, int* flags) {
    const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    bool diff = false;
    const int ng = write == erase ? 2 : 3;  // the same tensor as erase and write is read once
    const float* gates[3] = {alpha, erase, write};
    for (int i = 0; i < ng; ++i) {
        const float4 x = reinterpret_cast<const float4*>(gates[i] + row * 128)[lane];
        const float x0 = __shfl_sync(0xffffffffu, x.x, 0);
        diff |= (x.x != x0) | (x.y != x0) | (x.z != x0) | (x.w != x0);
    }
    if (__any_sync(0xffffffffu, diff) && lane == 0) {
        const int64_t b = row / TH;
        atomicOr(flags + b * H + (int)(row % H), 1);
    }
}

}  // namespace

// The training scan at K = V = 128 with bf16 inputs: a check kernel marks every (b, h) whose gates
// vary across channels; the tensor-core kernel scans the others (gates read at channel 0) and the
// token-sequential kernel the marked ones.  Both are launched; a CTA whose (b, h) belongs to the
// other kernel returns at once, so the choice needs no host synchronisation.
int training_scan_routed(const dbl_training_scan_args* a, SeqParams& p, cudaStream_t st) {
    const int64_t nbh = a->batch * a->heads, rows = a->batch * a->time * a->heads;
    for (const void* ptr : {static_cast<const void*>(a->alpha), static_cast<const void*>(a->erase),
                            static_cast<const void*>(a->write)})
        if (!aligned(ptr, 16)) return launch_seq_scan(p, a->dtype, st);
    int* flags = nullptr;
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    cudaError_t e = cudaStreamIsCapturing(st, &cap);
    if (e != cudaSuccess) return cuda_status(e, "training scan: cudaStreamIsCapturing");
    if (cap == cudaStreamCaptureStatusActive) {
        e = cudaMallocAsync(reinterpret_cast<void**>(&flags), nbh * sizeof(int), st);
    } else {
        cudaMemPool_t pool = nullptr;
        const int rc = scratch_pool(&pool);
        if (rc != DBL_OK) return rc;
        e = cudaMallocFromPoolAsync(reinterpret_cast<void**>(&flags), nbh * sizeof(int), pool, st);
    }
    if (e != cudaSuccess) return cuda_status(e, "training scan: route flags");
    int rc = cuda_status(cudaMemsetAsync(flags, 0, nbh * sizeof(int), st), "training scan: clear route flags");
    if (rc == DBL_OK) {
        const int64_t blocks = (rows + 7) / 8;
        if (blocks > 0x7fffffffLL) rc = fail(DBL_ERR_UNSUPPORTED, "training scan: too many rows");
        else {
            gate_uniform_kernel<<<(unsigned)blocks, 256, 0, st>>>(a->alpha, a->erase, a->write, rows,
                                                                (int)(a->time * a->heads), (int)a->heads, flags);
            rc = launch_status("gate_uniform_kernel");
        }
    }
    if (rc == DBL_OK) rc = tc_training_scan_launch(a, flags, 0, st);
    if (rc == DBL_OK) {
        p.route = flags;
        p.route_want = 1;
        rc = launch_seq_scan(p, a->dtype, st);
    }
    const cudaError_t ef = cudaFreeAsync(flags, st);
    if (rc == DBL_OK) rc = cuda_status(ef, "training scan: route flags release");
    return rc;
}

}  // namespace dbl

extern "C" int dbl_gdn_training_scan(const dbl_training_scan_args* a, dbl_stream_t stream) {
    using namespace dbl;
    SeqParams p{};
    const int rc = training_scan_params(a, &p);
    if (rc != DBL_OK) return rc;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (tc_training_scan_supported(a)) return training_scan_routed(a, p, st);
    return launch_seq_scan(p, a->dtype, st);
}

// delta_kernels::gdn2_scan (crates/kernels/src/ops.rs:251-276): doc-limit masks, zero initial.
extern "C" int dbl_gdn2_scan(const dbl_gdn2_scan_args* a, dbl_stream_t stream) {
    using namespace dbl;
    if (!a) return fail(DBL_ERR_INVALID_ARGUMENT, "gdn2_scan: null args");
    if (a->batch <= 0 || a->time <= 0 || a->heads <= 0 || a->key_dim <= 0 || a->value_dim <= 0)
        return fail(DBL_ERR_INVALID_ARGUMENT, "GDN-2 requires nonempty axes");
    if (a->dtype != DBL_F32 && a->dtype != DBL_BF16)
        return fail(DBL_ERR_INVALID_ARGUMENT, "gdn2_scan: dtype must be f32 or bf16");
    if (!a->q || !a->k || !a->v || !a->alpha || !a->erase || !a->write || !a->doc_start || !a->doc_end || !a->output)
        return fail(DBL_ERR_INVALID_ARGUMENT, "gdn2_scan: every pointer is required");
    if (a->batch > 0x7fffffff || a->time > 0x7fffffff || a->heads > 0x7fffffff || a->key_dim > 0x7fffffff ||
        a->value_dim > 0x7fffffff)
        return fail(DBL_ERR_UNSUPPORTED, "GDN-2 axis exceeds 32-bit limits");
    SeqParams p{};
    p.B = (int)a->batch;
    p.T = (int)a->time;
    p.H = (int)a->heads;
    p.K = (int)a->key_dim;
    p.V = (int)a->value_dim;
    const int64_t dk[4] = {a->batch, a->time, a->heads, a->key_dim};
    const int64_t dv[4] = {a->batch, a->time, a->heads, a->value_dim};
    const int64_t z[4] = {0, 0, 0, 0};
    p.q = a->q;
    p.k = a->k;
    p.v = a->v;
    resolve_strides(z, dk, 4, p.qs);
    resolve_strides(z, dk, 4, p.ks);
    resolve_strides(z, dv, 4, p.vs);
    p.gate_mode = 0;
    p.alpha = a->alpha;
    p.erase = a->erase;
    p.write = a->write;
    resolve_strides(z, dk, 4, p.as);
    resolve_strides(z, dk, 4, p.es);
    resolve_strides(z, dv, 4, p.ws);
    p.scale = 1.f;
    p.mask_mode = 2;
    p.doc_start = a->doc_start;
    p.doc_end = a->doc_end;
    p.init_mode = 0;
    p.out = a->output;
    p.out_dtype = a->dtype;
    resolve_strides(z, dv, 4, p.os);
    return launch_seq_scan(p, a->dtype, reinterpret_cast<cudaStream_t>(stream));
}
